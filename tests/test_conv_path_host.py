"""Which conv kernel the library picks (widek_conv_path, a host-only
decision: no device needed) for the geometries of the reference's conv
primitives (wide_conv1d.py:118-135, wide_conv2d.py:169-194,
wide_conv3d.py:102-125): strided, dilated, 3-D and odd channel counts run on
the tcgen05 per-tap kernel, stride-1 2-D convs with 64-channel multiples on
the halo kernel, fp32 and strides beyond the TMA traversal limit on CUDA
cores. Also the packed-weight and staging sizes."""
import pytest
import torch

from wide_compiler import _native as N
from wide_compiler import ops

BF16 = torch.bfloat16


@pytest.mark.parametrize("cin,cout,sp,k,s,p,d,dtype,want", [
    (64, 64, (32, 32), 3, 1, 1, 1, BF16, ops.CONV_PATH_HALO),        # cfg3
    (64, 64, (32, 32), 3, 2, 1, 1, BF16, ops.CONV_PATH_TAPS),        # stride 2
    (64, 128, (16, 16), 1, 2, 0, 1, BF16, ops.CONV_PATH_TAPS),       # 1x1 downsample
    (3, 64, (64, 64), 7, 2, 3, 1, BF16, ops.CONV_PATH_TAPS),         # RGB stem, cin 3
    (96, 64, (16, 16), 3, 1, 1, 1, BF16, ops.CONV_PATH_TAPS),        # cin % 64 != 0
    (64, 10, (12, 12), 3, 1, 1, 1, torch.float16, ops.CONV_PATH_TAPS),   # cout % 16 != 0
    (32, 32, (6, 10, 10), 3, 1, 1, 1, BF16, ops.CONV_PATH_TAPS),     # Conv3d
    (64, 64, (8, 16, 16), 3, 2, 1, 1, BF16, ops.CONV_PATH_TAPS),     # strided Conv3d
    (32, 48, (100,), 5, 2, 2, 1, BF16, ops.CONV_PATH_TAPS),          # strided Conv1d
    (64, 64, (17, 19), 3, 2, 2, 2, BF16, ops.CONV_PATH_TAPS),        # dilated + strided
    (64, 64, (32, 32), 3, 9, 1, 1, BF16, ops.CONV_PATH_DIRECT),      # stride > 8
    (64, 64, (32, 32), 3, 1, 1, 1, torch.float32, ops.CONV_PATH_DIRECT),
])
def test_conv_path_choice(cin, cout, sp, k, s, p, d, dtype, want):
    nd = len(sp)
    got = ops.conv_path(2, 2, cin, cout, sp, (k,) * nd, (s,) * nd, (p,) * nd, (d,) * nd, dtype)
    assert got == want


def test_conv_path_box_limit():
    # a 1-pixel-wide output row makes the tile 1 x 128: at H stride 4 its
    # input box would span 512 rows (> 256), so the conv stays on CUDA cores
    assert ops.conv_path(1, 1, 64, 64, (600, 1), (3, 1), (4, 1), (1, 0), (1, 1), BF16) == ops.CONV_PATH_DIRECT
    assert ops.conv_path(1, 1, 64, 64, (600, 1), (3, 1), (2, 1), (1, 0), (1, 1), BF16) == ops.CONV_PATH_TAPS


def test_packed_weight_and_staging_sizes():
    lib = N.load()
    assert lib.widek_conv_packed_weight_elems(128, 64, 9) == 128 * 9 * 64
    assert lib.widek_conv_packed_weight_elems(64, 3, 49) == 64 * 49 * 64       # padded to one 64-block
    assert lib.widek_conv_packed_weight_elems(64, 96, 9) == 64 * 9 * 128
    assert lib.widek_conv_packed_weight_elems(-1, 3, 1) == -1
    assert lib.widek_conv_workspace(2, 3, 3, 1, 10, 10, N.dtype_code(torch.zeros(1, dtype=BF16))) == 2 * 3 * 8 * 100 * 2
    assert lib.widek_conv_workspace(2, 3, 64, 4, 10, 10, N.dtype_code(torch.zeros(1, dtype=BF16))) == \
        2 * 3 * 64 * 400 * 2
