// Shared description of one attention-core call (see attention.cu for the
// semantics) and the tcgen05 kernel's entry, used by attention.cu's dispatcher.
#pragma once

#include "common.cuh"

namespace widek {

struct AttnArgs {
    const void* q;
    const void* k;
    const void* v;
    void* o;
    const void* mask;            // nullable
    int64_t sq, sk, sv, so;      // row strides (elements) of q, k, v, o
    int64_t ms_b, ms_h, ms_q, ms_k;  // mask strides (elements) over [nb, h, tq, tk]
    int nb, heads, tq, tk, dh;
    int causal, mask_kind;       // mask_kind: 0 none, 1 bool (uint8), 2 additive (same dtype as q), 3 additive fp32
    float scale;
};

// Launches the tcgen05/TMEM flash kernel (attention_sm100.cu) when the call
// fits it (bf16/f16, head_dim 64, any mask kind, positive scale, 16-byte
// aligned rows). Returns WIDEK_ERR_UNSUPPORTED without launching anything
// when it does not, so that the caller can take another kernel.
template <typename T>
int launch_attn_tc(const AttnArgs& a, cudaStream_t st);

// 0: tcgen05 kernel where it applies (default); 1: warp-level MMA kernel.
int attn_variant();
// Column pairs out of every 4 whose exponentials the tcgen05 kernel computes
// with the FMA-pipe polynomial instead of ex2.approx (0..2).
int attn_poly_pairs();

}  // namespace widek
