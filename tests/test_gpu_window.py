"""Sliding-window kernels (depthwise conv, max / average pooling) on every
staging plan band_window_kernel has, against the oracle:
  * whole planes per batch (small planes, several per CTA batch) and row
    bands of one plane (large planes), with plane and row sizes that are not
    multiples of 4 floats and input / output pointers off a 16-byte boundary
    (the unaligned head and tail of each contiguous copy);
  * the 3x3 stride-1 and stride-2 register paths and the generic window path;
  * rows too wide to stage, which go to the one-thread-per-output kernels.
Max pooling must match bit for bit; depthwise and average pooling within
1e-6 normwise (the reference's summation order, fp32)."""
import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu

# (n, c, h, w), (kh, kw), (sh, sw), (ph, pw)
WINDOW_CASES = {
    "whole_3x3_s1_odd_plane": ((3, 7, 13, 11), (3, 3), (1, 1), (1, 1)),
    "whole_3x3_s2_p0": ((2, 9, 14, 14), (3, 3), (2, 2), (0, 0)),
    "whole_3x3_s1_14x14_many_planes": ((4, 100, 14, 14), (3, 3), (1, 1), (1, 1)),
    "band_3x3_s1_odd_row": ((2, 3, 150, 121), (3, 3), (1, 1), (1, 1)),
    "band_3x3_s2_odd_row": ((2, 3, 151, 121), (3, 3), (2, 2), (1, 1)),
    "band_3x3_s2_one_row_bands": ((1, 2, 40, 2000), (3, 3), (2, 2), (1, 1)),
    "generic_5x3_s2x1": ((3, 5, 19, 9), (5, 3), (2, 1), (2, 0)),
    "generic_2x2_s2": ((3, 4, 17, 19), (2, 2), (2, 2), (0, 0)),
    "generic_band_4x4_s3": ((1, 2, 130, 130), (4, 4), (3, 3), (1, 1)),
    "wide_rows_fallback": ((1, 2, 5, 9001), (3, 3), (2, 2), (1, 1)),
}


def _out_hw(shape, k, s, p):
    _, _, h, w = shape
    return (h + 2 * p[0] - k[0]) // s[0] + 1, (w + 2 * p[1] - k[1]) // s[1] + 1


def _offset_tensor(torch, shape, gen, offset):
    """Random tensor whose data starts `offset` floats past an allocation."""
    n = int(np.prod(shape))
    base = torch.randn(n + offset, device="cuda", generator=gen)
    return base[offset:].view(*shape)


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("name", list(WINDOW_CASES))
def test_depthwise_plans(name, offset):
    import torch
    lib = S.gpu_lib()
    shape, k, s, p = WINDOW_CASES[name]
    n, c, h, w = shape
    ho, wo = _out_hw(shape, k, s, p)
    gen = torch.Generator(device="cuda").manual_seed(len(name) + offset)
    x = _offset_tensor(torch, shape, gen, offset)
    wt = torch.randn(c, 1, k[0], k[1], device="cuda", generator=gen) * 0.3
    bias = torch.randn(c, device="cuda", generator=gen) if offset else None
    y = _offset_tensor(torch, (n, c, ho, wo), gen, 3 * offset).fill_(float("nan"))
    g = nb.NplkConvGeom(n, c, h, w, c, k[0], k[1], s[0], s[1], p[0], p[1], 1, 1, ho, wo)
    rc = lib.nplk_depthwise_conv2d(S.cuda_stream(), C.byref(g), S.dptr(x), S.dptr(wt),
                                   S.dptr(bias) if bias is not None else None, S.dptr(y))
    assert rc == 0, rc
    torch.cuda.synchronize()
    ref = S.o_depthwise(x.cpu().numpy(), wt.cpu().numpy(), s, p,
                        bias.cpu().numpy() if bias is not None else None)
    got = y.cpu().numpy()
    assert not np.isnan(got).any()
    assert S.normwise_err(got, ref) < 1e-6


@pytest.mark.parametrize("kind,cip", [(0, 0), (1, 0), (1, 1)])
@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("name", list(WINDOW_CASES))
def test_pooling_plans(name, offset, kind, cip):
    import torch
    lib = S.gpu_lib()
    shape, k, s, p = WINDOW_CASES[name]
    n, c, h, w = shape
    ho, wo = _out_hw(shape, k, s, p)
    gen = torch.Generator(device="cuda").manual_seed(len(name) + 7 * offset + kind)
    x = _offset_tensor(torch, shape, gen, offset)
    y = _offset_tensor(torch, (n, c, ho, wo), gen, 2 * offset).fill_(float("nan"))
    rc = lib.nplk_pool2d(S.cuda_stream(), n, c, h, w, k[0], k[1], s[0], s[1], p[0], p[1], ho,
                         wo, kind, cip, S.dptr(x), S.dptr(y))
    assert rc == 0, rc
    torch.cuda.synchronize()
    ref = S.o_pool(x.cpu().numpy(), k, s, p, kind, cip)
    got = y.cpu().numpy()
    if kind == 0:
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    else:
        assert not np.isnan(got).any()
        assert S.normwise_err(got, ref) < 1e-6


def test_max_pool_signed_zero_and_infinity_order():
    # The reference's running max keeps the first of equal values (-0 before
    # +0) and starts at -inf; a window of -inf stays -inf.
    import torch
    lib = S.gpu_lib()
    x = np.zeros((1, 2, 6, 6), np.float32)
    x[0, 0, ::2, :] = -0.0
    x[0, 1] = -np.inf
    xt = torch.from_numpy(x).cuda()
    y = torch.full((1, 2, 3, 3), float("nan"), device="cuda")
    assert lib.nplk_pool2d(S.cuda_stream(), 1, 2, 6, 6, 3, 3, 2, 2, 1, 1, 3, 3, 0, 0,
                           S.dptr(xt), S.dptr(y)) == 0
    torch.cuda.synchronize()
    ref = S.o_pool(x, (3, 3), (2, 2), (1, 1), 0, 0)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("stride", [1, 2])
def test_depthwise_non_finite_weights_skip_padding(stride):
    # With a non-finite weight, 0 * w on a padded cell would turn the border
    # outputs into NaN; the reference skips padded cells, and so must we.
    import torch
    lib = S.gpu_lib()
    rng = S.rng(11)
    n, c, h, w = 2, 4, 14, 14
    x = rng.normal(0, 1, (n, c, h, w)).astype(np.float32)
    wt = rng.normal(0, 0.3, (c, 1, 3, 3)).astype(np.float32)
    wt[0, 0, 0, 0] = np.inf
    wt[1, 0, 2, 2] = np.nan
    wt[2, 0, 1, 0] = -np.inf
    ho = (h + 2 - 3) // stride + 1
    wo = (w + 2 - 3) // stride + 1
    xt, wtt = torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda()
    y = torch.zeros((n, c, ho, wo), device="cuda")
    g = nb.NplkConvGeom(n, c, h, w, c, 3, 3, stride, stride, 1, 1, 1, 1, ho, wo)
    assert lib.nplk_depthwise_conv2d(S.cuda_stream(), C.byref(g), S.dptr(xt), S.dptr(wtt), None,
                                     S.dptr(y)) == 0
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    ref = S.o_depthwise(x, wt, (stride, stride), (1, 1))
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    assert np.array_equal(got[np.isinf(got)], ref[np.isinf(ref)])
    fin = np.isfinite(ref)
    assert fin[:, 0].any() and fin[:, 3].all()  # finite where inf only meets padding
    assert S.normwise_err(got[fin], ref[fin]) < 1e-6


def test_pool_bands_inside_padding():
    # Padding larger than the window: the last output rows' windows lie wholly
    # in the padding (their bands stage no input rows).
    import torch
    lib = S.gpu_lib()
    rng = S.rng(12)
    n, c, h, w, k, s, p = 1, 3, 4, 600, 1, 1, 2  # 2400-float planes: row bands
    x = rng.normal(0, 1, (n, c, h, w)).astype(np.float32)
    ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    for kind in (0, 1):
        y = torch.full((n, c, ho, wo), float("nan"), device="cuda")
        xt = torch.from_numpy(x).cuda()
        assert lib.nplk_pool2d(S.cuda_stream(), n, c, h, w, k, k, s, s, p, p, ho, wo, kind, 1,
                               S.dptr(xt), S.dptr(y)) == 0
        torch.cuda.synchronize()
        ref = S.o_pool(x, (k, k), (s, s), (p, p), kind, 1)
        got = y.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)) or \
            S.normwise_err(got, ref) < 1e-6


@pytest.mark.parametrize("offset", [0, 3])
@pytest.mark.parametrize("planes,hw", [(131072 // 64, 196), (1000, 49), (777, 63), (50, 1776),
                                       (40, 3136), (5, 1)])
def test_global_avg_pool_plane_sizes(planes, hw, offset):
    # Plane sizes a multiple of 4 (16-byte loads, several planes per warp)
    # and not, an unaligned start when offset != 0, and large planes.
    import torch
    lib = S.gpu_lib()
    gen = torch.Generator(device="cuda").manual_seed(planes + hw + offset)
    x = _offset_tensor(torch, (planes, hw), gen, offset)
    y = torch.full((planes,), float("nan"), device="cuda")
    assert lib.nplk_global_avg_pool(S.cuda_stream(), planes, hw, S.dptr(x), S.dptr(y)) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    got = y.cpu().numpy()
    ref = S.o_gap(x.cpu().numpy().reshape(planes, 1, hw))[:, 0]
    assert not np.isnan(got).any()
    assert S.normwise_err(got, ref) < 1e-6


@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("rows,cols", [(1, 2048), (7, 4100), (300, 8192), (33, 12000),
                                       (150, 16384), (5, 16388)])
def test_layer_norm_long_rows(rows, cols, offset):
    # Rows of 2 K..16 K elements (a multiple of 4, aligned) go through the
    # staged ring kernel; an unaligned start or longer rows take the
    # register-row or three-pass kernels.
    import torch
    lib = S.gpu_lib()
    gen = torch.Generator(device="cuda").manual_seed(rows + cols + offset)
    x = _offset_tensor(torch, (rows, cols), gen, offset) * 3 + 1
    y = torch.full((rows, cols), float("nan"), device="cuda")
    gamma = torch.rand(cols, device="cuda", generator=gen) + 0.5
    beta = torch.rand(cols, device="cuda", generator=gen) - 0.5
    assert lib.nplk_layer_norm(S.cuda_stream(), rows, cols, S.dptr(x), S.dptr(y), S.dptr(gamma),
                               S.dptr(beta), 1e-5) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    got = y.cpu().numpy()
    ref = S.o_layer_norm(x.cpu().numpy(), cols, gamma.cpu().numpy(), beta.cpu().numpy())
    assert not np.isnan(got).any()
    assert S.normwise_err(got, ref) < 1e-5
