/*
 * widek.h — C-ABI of libwidek, the sm_100a kernels behind wide_compiler's
 * N-first wide primitives.
 *
 * Conventions (all entry points):
 *   - Every pointer is a device pointer on the CUDA device that is current
 *     for the calling thread; `stream` is a cudaStream_t (NULL = legacy
 *     default stream). Work is enqueued asynchronously on that stream.
 *   - The library never allocates device memory on these paths; the caller
 *     owns every buffer.
 *   - Tensors are dense and row-major ("contiguous") unless a stride
 *     argument says otherwise. `n` is always the number of fused models and
 *     every N-first tensor is laid out [n, ...].
 *   - dtype is one of WIDEK_F32 / WIDEK_BF16 / WIDEK_F16; arithmetic is
 *     carried out in fp32 whatever the storage type.
 *   - Return value: WIDEK_OK (0) or a negative WIDEK_ERR_* code. The message
 *     of the last failure on the calling thread is available through
 *     widek_last_error(). Nothing traps on the device: kernels that give up
 *     on a bounded wait record a code that widek_device_error() returns.
 *   - Entry points are re-entrant and may be called from several host
 *     threads on different streams.
 *
 * Each function cites the reference (WideCompiler v0.6.0, Python) call site
 * whose torch arithmetic it replaces, as path:line inside that project.
 */
#ifndef WIDEK_H_
#define WIDEK_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WIDEK_API __attribute__((visibility("default")))
#else
#define WIDEK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define WIDEK_OK 0
#define WIDEK_ERR_INVALID -1      /* bad shape, dtype, pointer or alignment */
#define WIDEK_ERR_UNSUPPORTED -2  /* valid request this build does not serve */
#define WIDEK_ERR_CUDA -3         /* a CUDA runtime call or launch failed */
#define WIDEK_ERR_TIMEOUT -4      /* a bounded device-side wait ran out */

#define WIDEK_F32 0
#define WIDEK_BF16 1
#define WIDEK_F16 2

#define WIDEK_ACT_NONE 0
#define WIDEK_ACT_RELU 1
#define WIDEK_ACT_GELU 2 /* exact erf form, torch.nn.functional.gelu default */

/* ---- library state ---------------------------------------------------- */

/* ABI version (major*100 + minor). */
WIDEK_API int widek_version(void);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len). Returns the code of that error (0 if none). */
WIDEK_API int widek_last_error(char* buf, size_t len);

/* Synchronizes the current device, returns the device-side error word in
 * *code (0 = none) and clears it. Returns WIDEK_OK or WIDEK_ERR_CUDA. */
WIDEK_API int widek_device_error(int* code);

/* Device error word codes (widek_device_error). */
#define WIDEK_DEV_ERR_GEMM_TIMEOUT 101  /* tcgen05 GEMM pipeline wait ran out */
#define WIDEK_DEV_ERR_RNN_TIMEOUT 102   /* recurrent kernel cluster wait ran out */
#define WIDEK_DEV_ERR_ATTN_TIMEOUT 103  /* attention pipeline wait ran out */
#define WIDEK_DEV_ERR_CONV_TIMEOUT 104  /* conv pipeline wait ran out */
#define WIDEK_DEV_ERR_NORM_TIMEOUT 105  /* BatchNorm ring wait ran out */
#define WIDEK_DEV_ERR_WAIT_PROBE 106    /* widek_test_bounded_wait ran out, as it must */
#define WIDEK_DEV_ERR_INDEX 110         /* an index input was out of range (skipped) */

/* Test hook for the failure path: launches one kernel that waits, for at
 * most limit_ns nanoseconds (0 < limit_ns <= 1 s), on an mbarrier that
 * nothing arrives at; the wait runs out, the kernel records
 * WIDEK_DEV_ERR_WAIT_PROBE in the device error word and returns, exactly as
 * the library's other bounded waits do. No fault, no trap; the context stays
 * usable. No counterpart in the reference. */
WIDEK_API int widek_test_bounded_wait(uint64_t limit_ns, void* stream);

/* ---- WideLinear -------------------------------------------------------- */

/* y[i] = act(x[i] @ w[i]^T + bias[i]) for every model i in [0, n).
 *   x: [n, m, k], w: [n, o, k], bias: [n, o] or NULL, y: [n, m, o].
 * bf16/f16 with k % 8 == 0 and 16-byte aligned pointers run on the tcgen05
 * tensor-core kernel. fp32 without an activation, with k % 4 == 0 and
 * 16-byte aligned rows, runs on the tensor cores with each operand split
 * into three bf16 pieces (the six piece products of order >= 2^-18
 * accumulated in fp32: each product as accurate as an fp32 multiply, so
 * the sums match an fp32 GEMM up to accumulation order with TF32 off);
 * every other case runs the CUDA-core kernel (fp32 FFMA).
 * Replaces: wide_compiler/core/primitives/wide_linear.py:165
 *           (einsum 'noi,nbi->nbo') and :168 (bias add). */
WIDEK_API int widek_linear_fwd(const void* x, const void* w, const void* bias, void* y,
                     int64_t n, int64_t m, int64_t k, int64_t o,
                     int dtype, int act, void* stream);

/* Same contraction forced onto the CUDA-core kernel (any dtype/alignment).
 * Replaces the same call site; exposed for testing and small problems. */
WIDEK_API int widek_linear_fwd_simt(const void* x, const void* w, const void* bias, void* y,
                          int64_t n, int64_t m, int64_t k, int64_t o,
                          int dtype, int act, void* stream);

/* widek_linear_fwd with the rows of x (in_layout) and y (out_layout) in
 * WIDEK_LAYOUT_NFIRST ([n, m, *]) or WIDEK_LAYOUT_PACKED, the
 * TracedWideModel boundary layout [B, n*T, *] with m = B*T and
 * rows_per_block = T (model i's row b*T + t at (b*n + i)*T + t). The tensor
 * maps read and write the packed rows in place, so a graph whose first or
 * last stage is a Linear on [B, T, features] inputs needs no unpack / pack
 * copy. The tensor-core kernel takes packed rows when T is a multiple or a
 * divisor of 128; other T run on the CUDA-core kernel.
 * Replaces: wide_compiler/core/traced_wide.py:463-469 / :527-532 around
 * wide_linear.py:165-168. */
WIDEK_API int widek_linear_fwd_ex(const void* x, const void* w, const void* bias, void* y,
                                  int64_t n, int64_t m, int64_t k, int64_t o, int64_t rows_per_block,
                                  int in_layout, int out_layout, int dtype, int act, void* stream);

/* y = LayerNorm(x @ w^T + bias) * ln_w + ln_b per model and row, in one
 * launch: the attention output projection and the WideLayerNorm after it.
 * Rows and layouts as widek_linear_fwd_ex (N-first or packed on either side,
 * rows_per_block for the packed form); ln_w, ln_b: [n, o] (the flat [n*o]
 * parameters of WideLayerNorm); bias [n, o] or NULL; biased variance with
 * eps; statistics in fp32 from the unrounded projection. bf16/f16 with
 * o a multiple of 16 up to 512, k a multiple of 8 and 16-byte aligned x, w
 * and y; otherwise returns WIDEK_ERR_UNSUPPORTED, launching nothing (run
 * widek_linear_fwd_ex and widek_layernorm_fwd_ex instead). Replaces the
 * output projection of wide_compiler/core/primitives/wide_attention.py:233-236
 * followed by wide_layernorm.py:62-65. */
WIDEK_API int widek_linear_ln_fwd_ex(const void* x, const void* w, const void* bias, const void* ln_w,
                                     const void* ln_b, void* y, int64_t n, int64_t m, int64_t k, int64_t o,
                                     int64_t rows_per_block, int in_layout, int out_layout, double eps,
                                     int dtype, void* stream);

/* Selects the tensor-core tiling of widek_linear_fwd for this process:
 * 0 = automatic (single-CTA 128xBN tiles), 1 = single-CTA tiles,
 * 2 = CTA-pair (cta_group::2) 256x256 tiles when m > 128 and o > 128,
 * 3 = single-CTA 128x128 tiles (6-stage ring), 4 = as 1 without L2 hints,
 * 5 = direct global stores instead of the TMA store, 6 = fp32 always on the
 * CUDA-core kernel (instead of the split-operand tensor-core kernel).
 * A measurement knob (process-wide, not synchronized with running calls).
 * No counterpart in the reference. */
WIDEK_API int widek_linear_set_variant(int variant);

/* A chain of wide Linear layers with activations, one launch:
 *   h_0 = x;  h_{l+1}[i] = act_l(h_l[i] @ weights[l][i]^T + biases[l][i])
 * for every model i in [0, n), l in [0, layers); y = h_layers.
 *   weights[l]: [n, dims[l+1], dims[l]]; biases[l]: [n, dims[l+1]] or NULL;
 *   dims: layers + 1 widths; acts: layers WIDEK_ACT_* codes;
 *   x: [n, batch, dims[0]] (in_layout NFIRST) or [batch, n*dims[0]] (PACKED);
 *   y: [n, batch, dims[layers]] (out_layout NFIRST) or [batch, n*dims[layers]].
 * One CTA per model keeps the activations and one layer's weights in shared
 * memory; fp32 arithmetic, each layer's output rounded to the storage dtype
 * as a layer-by-layer run stores it. fp32 chains whose layers are at most
 * 128 wide and 256 deep (widths multiples of 4, 16-byte aligned tensors)
 * can run on tcgen05 instead (widek_mlp_chain_set_variant(1)): per layer
 * D^T = W . h^T with the weights as the 128-row A operand and the batch
 * rows as N, every fp32 operand split into bf16 hi + lo and accumulated as
 * hi*hi + hi*lo + lo*hi in fp32 (each product within ~2^-17 of the fp32
 * one). Returns WIDEK_ERR_UNSUPPORTED (launching
 * nothing) when the chain does not fit (widek_mlp_chain_supported says in
 * advance). Replaces, for a TracedWideModel whose graph is such a chain, the
 * boundary unpack, the per-node WideLinear (wide_compiler/core/primitives/
 * wide_linear.py:165-168) and activation calls, and the boundary pack
 * (wide_compiler/core/traced_wide.py:450-532). */
WIDEK_API int widek_mlp_chain_fwd(const void* x, void* y, const void* const* weights,
                                  const void* const* biases, const int64_t* dims, const int* acts,
                                  int layers, int64_t n, int64_t batch, int in_layout, int out_layout,
                                  int dtype, void* stream);

/* 1 if widek_mlp_chain_fwd would run this chain (1..8 layers, widths
 * 1..4096, batch <= 4096, activations and one layer's weights within one
 * SM's shared memory), else 0. Launches nothing. */
WIDEK_API int widek_mlp_chain_supported(const int64_t* dims, const int* acts, int layers, int64_t n,
                                        int64_t batch, int dtype);

/* Kernel choice for fp32 chains: 0 = the CUDA-core kernel (default), 1 =
 * the tcgen05 split-operand kernel wherever it fits (measured no faster at
 * the sizes it fits). Process-wide; for tests and measurements. No
 * reference counterpart. */
WIDEK_API int widek_mlp_chain_set_variant(int variant);

/* ---- WideLayerNorm ----------------------------------------------------- */

/* Per-row LayerNorm over the last dim d with per-model affine:
 *   x, y: [n, rows_per_model, d]; w, b: [n, d] (flat [n*d] in the module).
 * Biased variance, statistics in fp32.
 * Replaces: wide_compiler/core/primitives/wide_layernorm.py:62-65. */
WIDEK_API int widek_layernorm_fwd(const void* x, const void* w, const void* b, void* y,
                        int64_t n, int64_t rows_per_model, int64_t d,
                        double eps, int dtype, void* stream);

/* widek_layernorm_fwd on rows laid out [outer][n][inner][d]: row r uses the
 * affine of model (r / inner) % n. outer = 1, inner = rows_per_model is the
 * N-first layout; the packed TracedWideModel boundary layout [B, n*T, d]
 * (and [B, n*d], T = 1) is outer = B, inner = T, so a graph whose first or
 * last stage is a LayerNorm needs no unpack / pack copy.
 * Replaces: wide_compiler/core/traced_wide.py:463-469 / :527-532 (the
 * unpack / pack around wide_layernorm.py:62-65). */
WIDEK_API int widek_layernorm_fwd_ex(const void* x, const void* w, const void* b, void* y, int64_t n,
                                     int64_t outer, int64_t inner, int64_t d, double eps, int dtype,
                                     void* stream);

/* ---- layout boundary (pack / unpack) ----------------------------------- */

/* dst[j, i, :] = src[i, j, :] for src [a, b, inner_bytes] (bytes).
 * N-first [N, B, R] <-> channel-packed [B, N, R] in both directions.
 * Replaces: wide_compiler/core/traced_wide.py:463-469 (unpack view +
 * first-stage copy) and :531-532 (pack movedim+reshape). */
WIDEK_API int widek_swap01(const void* src, void* dst, int64_t a, int64_t b,
                 int64_t inner_bytes, void* stream);

/* Stacks n separate [b, inner_bytes] buffers into dst [b, n, inner_bytes].
 * srcs is a HOST array of n device pointers.
 * Replaces: wide_compiler/core/ensemble_util.py:45 (torch.stack(dim=1)). */
WIDEK_API int widek_pack(const void* const* srcs, int64_t n, void* dst, int64_t b,
               int64_t inner_bytes, void* stream);

/* Strided 2-D copy: rows of row_bytes bytes from src (row pitch src_pitch
 * bytes) to dst (row pitch dst_pitch bytes); pitches >= row_bytes.
 * Used where N is sharded over GPUs: a rank's channel slice
 * x[:, lo*C:hi*C] of the packed [B, N*C, ...] input, and the placement of
 * gathered rank outputs into the full packed output. No reference
 * counterpart: the reference runs on one device
 * (wide_compiler/core/traced_wide.py:463-469 and :527-532 are the
 * single-device unpack / pack this slices). */
WIDEK_API int widek_copy2d(const void* src, int64_t src_pitch, void* dst, int64_t dst_pitch,
                           int64_t rows, int64_t row_bytes, void* stream);

/* ---- elementwise glue --------------------------------------------------- */

#define WIDEK_UNARY_RELU 0
#define WIDEK_UNARY_GELU 1
#define WIDEK_UNARY_SIGMOID 2
#define WIDEK_UNARY_TANH 3
#define WIDEK_UNARY_SILU 4

#define WIDEK_BINARY_ADD 0
#define WIDEK_BINARY_MUL 1
#define WIDEK_BINARY_SUB 2
#define WIDEK_BINARY_DIV 3

/* y = op(x) over numel elements.
 * Replaces: wide_compiler/core/traced_wide.py:174-186 (FunctionalOp on
 * F.relu / F.gelu / torch.sigmoid / torch.tanh / F.silu). */
WIDEK_API int widek_unary(const void* x, void* y, int64_t numel, int op, int dtype,
                void* stream);

/* y = a op b over numel elements (same shape, dense).
 * Replaces: wide_compiler/core/traced_wide.py:189-211 (BinaryOp add / mul /
 * sub / div). */
WIDEK_API int widek_binary(const void* a, const void* b, void* y, int64_t numel, int op,
                 int dtype, void* stream);

/* ---- WideBatchNorm1d / WideBatchNorm2d ---------------------------------- */

/* Normalization with given statistics (eval mode, running stats):
 *   x, y: [n, batch, c, l] (l = spatial size, 1 for [n, batch, c]);
 *   weight, bias (nullable), mean, var: flat [n*c].
 * y = (x - mean) / sqrt(var + eps) * weight + bias per (model, channel).
 * Replaces: wide_compiler/core/primitives/wide_batchnorm_2d.py:53-72 and
 *           wide_batchnorm_1d.py:53-73 (permute copies + nn.BatchNorm(N*C)). */
WIDEK_API int widek_batchnorm_fwd(const void* x, void* y, const void* weight, const void* bias,
                                  const void* mean, const void* var, int64_t n, int64_t batch,
                                  int64_t c, int64_t l, double eps, int dtype, void* stream);

/* Bytes of workspace widek_batchnorm_train_fwd needs for this shape on the
 * current device (fp64 partial sums). */
WIDEK_API size_t widek_batchnorm_train_workspace(int64_t n, int64_t batch, int64_t c, int64_t l);

/* Training-mode normalization with batch statistics per (model, channel)
 * over batch*l elements; updates running_mean / running_var in place
 * (momentum; unbiased variance) when given, writes save_mean / save_invstd
 * (fp32 [n*c], nullable). `workspace` is caller-provided device memory of at
 * least widek_batchnorm_train_workspace() bytes.
 * Replaces: the same call sites in training mode (nn.BatchNorm batch
 * statistics and running-stat update). */
WIDEK_API int widek_batchnorm_train_fwd(const void* x, void* y, const void* weight, const void* bias,
                                        void* running_mean, void* running_var, float* save_mean,
                                        float* save_invstd, void* workspace, size_t workspace_bytes,
                                        int64_t n, int64_t batch, int64_t c, int64_t l,
                                        double momentum, double eps, int dtype, void* stream);

/* Allocation-free variant of widek_batchnorm_train_fwd for callers that
 * cannot allocate device memory (a runtime that owns all device memory in
 * its own fixed pool, a latency-critical path that must not risk cudaMalloc's
 * implicit synchronization, an FFI caller with no allocator). This entry
 * point has no counterpart in the reference.
 * Same arguments and results as widek_batchnorm_train_fwd minus the
 * workspace: the fp64 partial sums live in a fixed 1 MiB device array inside
 * the library (held on every GPU that loads it until exit), so at most
 * 65536 channels (n*c) are accepted; larger requests return
 * WIDEK_ERR_INVALID. The first call on a device resolves that array's device
 * address (cudaGetSymbolAddress), so make that first call before any stream
 * capture. All calls share the array: calls that overlap on the GPU race and
 * must be serialized by the caller. Nothing in the array has to start at zero
 * (every slot is written before it is read). Allocates nothing.
 * The resolved address is kept for the life of the process: do not use this
 * entry point across a cudaDeviceReset of a device it has run on (the array's
 * address on that device may change). */
WIDEK_API int widek_batchnorm_train_fwd_noalloc(const void* x, void* y, const void* weight,
                                                const void* bias, void* running_mean,
                                                void* running_var, float* save_mean,
                                                float* save_invstd, int64_t n, int64_t batch,
                                                int64_t c, int64_t l, double momentum, double eps,
                                                int dtype, void* stream);

/* ---- WideGroupNorm / WideInstanceNorm1d/2d -------------------------------- */

/* Statistics per (model, sample, group) over the group's (c/groups)*l
 * elements, per-channel affine (weight/bias flat [n*c], nullable).
 *   x, y: [n, batch, c, l]. row_mean / row_var (fp32 [n*batch*groups],
 * nullable together) receive each group's mean and biased variance.
 * InstanceNorm is groups == c.
 * Replaces: wide_compiler/core/primitives/wide_groupnorm.py:90-117 and
 *           wide_instancenorm.py:89-108, :222-240. */
WIDEK_API int widek_groupnorm_fwd(const void* x, void* y, const void* weight, const void* bias,
                                  float* row_mean, float* row_var, int64_t n, int64_t batch,
                                  int64_t c, int64_t l, int64_t groups, double eps, int dtype,
                                  void* stream);

/* ---- WideEmbedding ------------------------------------------------------ */

/* out[i, j, :] = weight[i, idx[j], :] for every model i; idx: int64 [num_idx]
 * shared by all models; weight: [n, v, d]; out: [n, num_idx, d]. Negative
 * indices wrap once; indices outside [-v, v) give a zero row and set the
 * device error word.
 * Replaces: wide_compiler/core/primitives/wide_embedding.py:85-99
 *           (weight[:, idx]). */
WIDEK_API int widek_embedding_fwd(const int64_t* idx, const void* weight, void* out, int64_t n,
                                  int64_t num_idx, int64_t v, int64_t d, int dtype, void* stream);

/* ---- WideGRU / WideLSTM --------------------------------------------------- */

/* GRU recurrence over `steps` time steps in one launch (gate order r, z, n):
 *   gates_x: [n, batch, steps, 3*hidden] = x @ W_ih^T + b_ih for every step
 *            (computed beforehand with widek_linear_fwd);
 *   w_hh: [n, 3*hidden, hidden]; b_hh: [n, 3*hidden] or NULL;
 *   h0: [n, batch, hidden] or NULL (zeros);
 *   out: [n, batch, steps, hidden]; h_n: [n, batch, hidden].
 * One thread-block cluster per model keeps W_hh on chip across all steps.
 * Replaces: wide_compiler/core/primitives/wide_gru.py:181-213 (per-step
 * einsum, bias, chunk, sigmoid/tanh, blend, stack). */
WIDEK_API int widek_gru_recurrence(const void* gates_x, const void* w_hh, const void* b_hh,
                                   const void* h0, void* out, void* h_n, int64_t n,
                                   int64_t batch, int64_t steps, int64_t hidden, int dtype,
                                   void* stream);

/* LSTM recurrence (gate order i, f, g, o) with the same conventions:
 *   gates_x: [n, batch, steps, 4*hidden]; w_hh: [n, 4*hidden, hidden] (the
 *   diagonal blocks of the block-diagonal module parameter); b_hh:
 *   [n, 4*hidden] or NULL; h0, c0: [n, batch, hidden] or NULL;
 *   out: [n, batch, steps, hidden]; h_n, c_n: [n, batch, hidden].
 * Replaces: wide_compiler/core/primitives/wide_lstm.py:184-234. */
WIDEK_API int widek_lstm_recurrence(const void* gates_x, const void* w_hh, const void* b_hh,
                                    const void* h0, const void* c0, void* out, void* h_n,
                                    void* c_n, int64_t n, int64_t batch, int64_t steps,
                                    int64_t hidden, int dtype, void* stream);

/* Whole GRU / LSTM forward in one call: the input projection
 * x @ W_ih^T + b_ih into the caller's workspace (CUDA-core grouped GEMM,
 * fp32 arithmetic), then the recurrence, with both weights addressed by
 * stride so that no re-laid-out copy is needed:
 *   x: [n, batch, steps, input]; out: [n, batch, steps, hidden];
 *   h0 (and c0 for LSTM): [n, batch, hidden] or NULL; h_n, c_n likewise;
 *   b_ih, b_hh: [n, G*hidden] or NULL (G = 3 for GRU r,z,n; 4 for LSTM i,f,g,o);
 *   model i's W_ih [G*hidden, input] block starts at w_ih + i*w_strides[0]
 *   with rows w_strides[1] elements apart, its W_hh [G*hidden, hidden] block
 *   at w_hh + i*w_strides[2], rows w_strides[3] apart (w_strides NULL =
 *   dense [n, G*hidden, ...]). The strides let WideLSTM pass its
 *   block-diagonal [n*4H, n*I] / [n*4H, n*H] parameters as they are.
 *   workspace: widek_rnn_workspace(...) bytes (the projected gates).
 * Replaces: wide_compiler/core/primitives/wide_gru.py:148-213 and
 * wide_lstm.py:158-234 (block extraction :184-199, input projection
 * :168 / :190, the per-step loop). */
WIDEK_API int widek_gru_fwd(const void* x, const void* w_ih, const void* w_hh, const void* b_ih,
                            const void* b_hh, const void* h0, void* out, void* h_n,
                            const int64_t* w_strides, void* workspace, size_t workspace_bytes,
                            int64_t n, int64_t batch, int64_t steps, int64_t input, int64_t hidden,
                            int dtype, void* stream);
WIDEK_API int widek_lstm_fwd(const void* x, const void* w_ih, const void* w_hh, const void* b_ih,
                             const void* b_hh, const void* h0, const void* c0, void* out, void* h_n,
                             void* c_n, const int64_t* w_strides, void* workspace,
                             size_t workspace_bytes, int64_t n, int64_t batch, int64_t steps,
                             int64_t input, int64_t hidden, int dtype, void* stream);

/* widek_gru_fwd / widek_lstm_fwd with explicit layouts of x (in_layout) and
 * out (out_layout), each WIDEK_LAYOUT_NFIRST ([n, batch, steps, *]) or
 * WIDEK_LAYOUT_PACKED (the TracedWideModel boundary layout [batch,
 * n*steps, *]): the projection reads a packed input in place and the
 * recurrence writes a packed output directly (h_n / c_n stay N-first), so a
 * graph that starts or ends with the recurrent layer needs no unpack / pack
 * copy. Replaces: wide_compiler/core/traced_wide.py:463-469 / :527-532
 * around wide_gru.py:148-213, wide_lstm.py:158-234. */
WIDEK_API int widek_gru_fwd_ex(const void* x, const void* w_ih, const void* w_hh, const void* b_ih,
                               const void* b_hh, const void* h0, void* out, void* h_n,
                               const int64_t* w_strides, void* workspace, size_t workspace_bytes,
                               int64_t n, int64_t batch, int64_t steps, int64_t input, int64_t hidden,
                               int in_layout, int out_layout, int dtype, void* stream);
WIDEK_API int widek_lstm_fwd_ex(const void* x, const void* w_ih, const void* w_hh, const void* b_ih,
                                const void* b_hh, const void* h0, const void* c0, void* out, void* h_n,
                                void* c_n, const int64_t* w_strides, void* workspace,
                                size_t workspace_bytes, int64_t n, int64_t batch, int64_t steps,
                                int64_t input, int64_t hidden, int in_layout, int out_layout, int dtype,
                                void* stream);

/* Workspace bytes of widek_gru_fwd (lstm = 0) / widek_lstm_fwd (lstm = 1). */
WIDEK_API size_t widek_rnn_workspace(int lstm, int64_t n, int64_t batch, int64_t steps, int64_t hidden,
                                     int dtype);

/* Kernel choice for the recurrences: 0 = the register-resident kernel where
 * it applies (hidden size 128, at most 128 gate rows per cluster CTA; W_hh
 * held in registers, hidden state passed by DSMEM stores and mbarrier
 * signals), else the shared-memory cluster kernel (default); 1 = the
 * shared-memory cluster kernel only. Process-wide; for tests and
 * measurements. No reference counterpart. */
WIDEK_API int widek_rnn_set_variant(int variant);

/* ---- WideConv1d / WideConv2d / WideConv3d -------------------------------- */

/* Repacks conv weights [rows][cin][taps] -> [rows][taps][cin_p] (rows =
 * n*cout, taps = kd*kh*kw, cin_p = cin rounded up to a multiple of 64, the
 * extra channels of every tap zero) for the tensor-core path; elem_bytes 2
 * or 4. w_packed holds widek_conv_packed_weight_elems(rows, cin, taps)
 * elements. */
WIDEK_API int widek_conv_pack_weight(const void* w, void* w_packed, int64_t rows, int64_t cin,
                                     int64_t taps, int64_t elem_bytes, void* stream);

/* Elements of widek_conv_pack_weight's output: rows * taps * cin_p (-1 for a
 * negative size). */
WIDEK_API int64_t widek_conv_packed_weight_elems(int64_t rows, int64_t cin, int64_t taps);

/* Bytes of the channels-last staging workspace widek_conv_fwd uses on the
 * tensor-core path (n*batch*cin_s*d*h*w elements, cin_s = cin rounded up to
 * a multiple of 8). */
WIDEK_API size_t widek_conv_workspace(int64_t n, int64_t batch, int64_t cin, int64_t d, int64_t h,
                                      int64_t w, int dtype);

/* One independent convolution per model on the N-first layout:
 *   x: [n, batch, cin, d, h, w] (d = 1 for 2-D; d = h = 1 for 1-D);
 *   w: [n*cout, cin, kd, kh, kw]; y: [n, batch, cout, od, oh, ow].
 * geom = 22 int64: n, batch, cin, cout, d, h, w, kd, kh, kw, sd, sh, sw,
 *        pd, ph, pw, dd, dh, dw, od, oh, ow (stride s, padding p, dilation d).
 * Epilogue per output element of channel c of model i (ch = i*cout + c):
 *   v = acc + bias[ch]; v *= scale[ch]; v += shift[ch];
 *   residual_first ? v = act(v + residual) : v = act(v) + residual
 * (each term skipped when its pointer is NULL).
 * bf16/f16 convs of any rank, channel counts and dilation, with H and W
 * strides up to 8 (and an output tile whose input box fits 256 elements per
 * dimension: tile width x stride along W, 128 / tile width x stride along
 * H), run on the tcgen05 implicit-GEMM kernels when w_packed (from
 * widek_conv_pack_weight) and a workspace of widek_conv_workspace() bytes
 * are given; fp32 and everything else runs a CUDA-core direct convolution
 * (widek_conv_path tells which).
 * Replaces: wide_compiler/core/primitives/wide_conv2d.py:169-194 (permute
 * copies + grouped F.conv2d), wide_conv1d.py:118-135, wide_conv3d.py:102-125. */
WIDEK_API int widek_conv_fwd(const void* x, const void* w, const void* w_packed, const void* bias,
                             const void* scale, const void* shift, const void* residual, void* y,
                             void* workspace, size_t workspace_bytes, const int64_t* geom, int act,
                             int residual_first, int dtype, void* stream);

/* Number of kernels the library has launched in this process (all entry
 * points; a launch captured into a CUDA graph counts once, at capture). For
 * measurements. No reference counterpart. */
WIDEK_API long long widek_launch_count(void);

/* Tensor layouts for widek_conv_fwd_ex (N models, batch B, C channels,
 * spatial S):
 *   WIDEK_LAYOUT_NFIRST  [N][B][C][S]   the N-first layout of the wide primitives
 *   WIDEK_LAYOUT_PACKED  [B][N*C][S]    the packed layout at a TracedWideModel
 *                                       boundary (ensemble_util pack_inputs)
 *   WIDEK_LAYOUT_CLAST   [N][B][S][C]   channels-last (tensor-core path only) */
#define WIDEK_LAYOUT_NFIRST 0
#define WIDEK_LAYOUT_PACKED 1
#define WIDEK_LAYOUT_CLAST 2

/* widek_conv_fwd with explicit layouts of x (in_layout), y (out_layout) and
 * the residual (res_layout: NFIRST or PACKED). Reading a packed input fuses
 * the boundary unpack into the channels-last staging; a channels-last input
 * skips the staging; packed and channels-last outputs (and a packed
 * residual) are written / read by the halo-reuse kernel's TMA maps, so a
 * chain of convolutions needs no separate pack, unpack or transpose.
 * Returns WIDEK_ERR_UNSUPPORTED, launching nothing, when the combination
 * cannot be served for this geometry (the caller then uses the N-first
 * layouts). No reference counterpart: the reference materialises the
 * N-first tensors between ops (wide_compiler/core/traced_wide.py:463-469,
 * :531-532). */
WIDEK_API int widek_conv_fwd_ex(const void* x, const void* w, const void* w_packed, const void* bias,
                                const void* scale, const void* shift, const void* residual, void* y,
                                void* workspace, size_t workspace_bytes, const int64_t* geom, int act,
                                int residual_first, int in_layout, int out_layout, int res_layout,
                                int dtype, void* stream);

/* Which kernel widek_conv_fwd_ex would run for this geometry, dtype and
 * layouts (pointers assumed 16-byte aligned, workspace large enough):
 * WIDEK_CONV_PATH_DIRECT (CUDA cores), _TAPS (tcgen05 per-tap implicit GEMM
 * on channels-last input), _HALO (tcgen05 halo-reuse on channels-last
 * input), or -1 when the combination is not served. Launches nothing.
 * No counterpart in the reference (a query for tests and planners). */
#define WIDEK_CONV_PATH_DIRECT 0
#define WIDEK_CONV_PATH_TAPS 1
#define WIDEK_CONV_PATH_HALO 2
WIDEK_API int widek_conv_path(const int64_t* geom, int dtype, int in_layout, int out_layout,
                              int res_layout, int has_residual);

/* 1 if widek_conv_fwd_ex would run this geometry/dtype/layout combination
 * (assuming 16-byte aligned device pointers and a large enough workspace),
 * else 0. Launches nothing. */
WIDEK_API int widek_conv_layouts_supported(const int64_t* geom, int dtype, int in_layout, int out_layout,
                                           int res_layout, int has_residual);

/* Kernel choice for widek_conv_fwd's tensor-core path: 0 = halo-reuse kernel
 * where it applies (64-channel output tiles, output width a multiple of 8;
 * 8 x 16 pixel tiles with one shared halo buffer for channels-last outputs,
 * 16 x 8 tiles with column-shifted subtiles otherwise), else the per-tap
 * kernel (default); 1 = per-tap kernel only; 2 = as 0 with the shared halo
 * buffer for every output layout. Process-wide; for tests and
 * measurements. No reference counterpart. */
WIDEK_API int widek_conv_set_variant(int variant);

/* ---- WideAttention -------------------------------------------------------- */

#define WIDEK_MASK_NONE 0
#define WIDEK_MASK_BOOL 1       /* uint8, nonzero = attend */
#define WIDEK_MASK_ADD 2        /* additive, same dtype as q */
#define WIDEK_MASK_ADD_F32 3    /* additive, fp32 */

/* Scaled dot-product attention core for nb*heads independent heads:
 *   q: rows [nb, tq] with row stride q_row_stride elements, head h at
 *      columns [h*head_dim, (h+1)*head_dim); k, v likewise with tk rows;
 *   o: [nb, tq] rows of o_row_stride elements, head h at h*head_dim.
 * softmax(q k^T * scale [+ mask]) v per head; causal = key index <= query
 * index (top-left aligned). mask (nullable) is addressed as
 * mask[b*s0 + h*s1 + i*s2 + j*s3] with mask_strides = {s0, s1, s2, s3}
 * (0 for broadcast dims). Rows with no attended key produce zeros.
 * Replaces: wide_compiler/core/primitives/wide_attention.py:217-231
 * (head split copies, F.scaled_dot_product_attention, head merge). */
WIDEK_API int widek_attention_fwd(const void* q, const void* k, const void* v, void* o,
                                  int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride,
                                  int64_t o_row_stride, int64_t nb, int64_t heads, int64_t tq,
                                  int64_t tk, int64_t head_dim, int causal, const void* mask,
                                  int mask_kind, const int64_t* mask_strides, double scale,
                                  int dtype, void* stream);

/* Kernel choice for widek_attention_fwd: 0 = tcgen05/TMEM flash kernel
 * where it applies (bf16/f16, head_dim 64; causal or not, with or without
 * an explicit bool / additive mask of any strides), else the
 * warp-level MMA or CUDA-core kernels (default); 1 = never the tcgen05
 * kernel; 10 + k (k = 0, 1, 2) = as 0, with k of every 4 column pairs of
 * exponentials computed by an FMA-pipe polynomial instead of the
 * special-function unit (0 and 1 reset k to its default, 1).
 * Process-wide; for tests and measurements. No reference counterpart (the
 * reference has a single torch SDPA call). */
WIDEK_API int widek_attention_set_variant(int variant);

/* ---- Backward (training) ------------------------------------------------
 * The reference differentiates its primitives' torch forward with autograd
 * (gradient flow tested at wide_compiler/core/primitives/wide_lstm.py:744-762);
 * these entries compute the same gradients on the GPU. */

/* y[b] = x[b]^T for x [batch, rows, cols] -> y [batch, cols, rows], any
 * dtype (bytes are moved, not converted). */
WIDEK_API int widek_transpose(const void* x, void* y, int64_t batch, int64_t rows, int64_t cols,
                              int dtype, void* stream);

/* Workspace bytes widek_linear_bwd needs (-1 for bad arguments). */
WIDEK_API int64_t widek_linear_bwd_workspace(int64_t n, int64_t m, int64_t k, int64_t o, int dtype);

/* Gradients of widek_linear_fwd without activation (y = x W^T + b per
 * model; x [n, m, k], W [n, o, k], dy [n, m, o], all dense):
 *   dx [n, m, k] = dy W,  dw [n, o, k] = dy^T x,  db [n, o] = sum_m dy.
 * Any of dx / dw / db may be null (not computed). The two products run on
 * widek_linear_fwd (tcgen05 for bf16/f16, split-operand tcgen05 or CUDA
 * cores for fp32) over transposed copies of W, dy and x in the workspace;
 * db is a column sum in fp32 (fixed summation order). Replaces the
 * autograd of wide_compiler/core/primitives/wide_linear.py:162-171
 * (einsum 'noi,nbi->nbo' + bias). */
WIDEK_API int widek_linear_bwd(const void* x, const void* w, const void* dy, void* dx, void* dw,
                               void* db, int64_t n, int64_t m, int64_t k, int64_t o, int dtype,
                               void* workspace, int64_t workspace_bytes, void* stream);

/* dpre = dy * act'(saved) elementwise over count elements: act RELU with
 * saved = the activation's output (gradient 1 where it is > 0), act GELU
 * (exact erf form) with saved = its input: Phi(s) + s * phi(s). Replaces the
 * autograd of torch.relu / F.gelu after a WideLinear
 * (wide_compiler/core/traced_wide.py:174-211). */
WIDEK_API int widek_act_bwd(const void* dy, const void* saved, void* dpre, int64_t count, int act,
                            int dtype, void* stream);

/* Workspace bytes widek_layernorm_bwd needs (-1 for bad arguments). */
WIDEK_API int64_t widek_layernorm_bwd_workspace(int64_t n, int64_t outer, int64_t d);

/* Gradients of widek_layernorm_fwd (x, dy, dx [n, outer, d] dense; gamma
 * flat [n*d]): dx = rstd * (g - mean(g) - x_hat * mean(g * x_hat)) with
 * g = dy * gamma, dgamma = sum_rows dy * x_hat, dbeta = sum_rows dy (mean
 * and rstd recomputed from x with the forward's eps; biased variance).
 * dw / db may be null. d <= 1024. Replaces the autograd of
 * wide_compiler/core/primitives/wide_layernorm.py:62-65. */
WIDEK_API int widek_layernorm_bwd(const void* x, const void* w, const void* dy, void* dx,
                                  void* dw, void* db, int64_t n, int64_t outer, int64_t d,
                                  double eps, int dtype, void* workspace, int64_t workspace_bytes,
                                  void* stream);

/* Gradients of widek_batchnorm_fwd / widek_batchnorm_train_fwd on
 * x, dy, dx: [n, batch, c, l] dense; weight (nullable: no affine),
 * running_mean / running_var flat [n*c]. batch_stats = 1: the statistics
 * of the batch (recomputed from x; biased variance), dx = rstd * (g -
 * mean(g) - x_hat * mean(g * x_hat)) with g = dy * gamma; batch_stats = 0
 * (eval mode): the running statistics, dx = rstd * g. dw / db ([n*c],
 * nullable) = sum of dy * x_hat / of dy per (model, channel). Replaces the
 * autograd of wide_compiler/core/primitives/wide_batchnorm_2d.py:53-72 and
 * wide_batchnorm_1d.py:53-73. */
WIDEK_API int widek_batchnorm_bwd(const void* x, const void* dy, const void* weight,
                                  const void* running_mean, const void* running_var, void* dx,
                                  void* dw, void* db, int64_t n, int64_t batch, int64_t c,
                                  int64_t l, int batch_stats, double eps, int dtype, void* stream);

/* Workspace bytes widek_groupnorm_bwd needs (-1 for bad arguments). */
WIDEK_API int64_t widek_groupnorm_bwd_workspace(int64_t n, int64_t batch, int64_t c);

/* Gradients of widek_groupnorm_fwd (statistics per (model, sample, group),
 * recomputed from x; per-channel affine weight [n*c], nullable): dx as for
 * batch statistics above over each group's elements; dw / db ([n*c],
 * nullable) summed over the batch in a fixed order. InstanceNorm is the
 * case groups = c. Replaces the autograd of
 * wide_compiler/core/primitives/wide_groupnorm.py:90-117 and
 * wide_instancenorm.py:89-108. */
WIDEK_API int widek_groupnorm_bwd(const void* x, const void* dy, const void* weight, void* dx,
                                  void* dw, void* db, int64_t n, int64_t batch, int64_t c,
                                  int64_t l, int64_t groups, double eps, int dtype,
                                  void* workspace, int64_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WIDEK_H_ */
