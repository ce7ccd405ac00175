"""Every conv kernel (nplk_conv2d_run_algo) against the direct-gather kernel
and the oracle:
  * IM2COL: NHWC tf32 hi/lo planes of x, one im2col TMA load per k-block;
  * WINDOW: one raw NHWC plane, one im2col TMA window per (tile, channel
    block, kh) shared by the KW taps (tf32 lo part formed in shared memory);
  * WINDOW_GATHER: the same windows gathered from NCHW x by the kernel;
  * WINDOW_PAIR: the gather windows on CTA pairs, each MMA spanning two SMs
    (C_out <= 64).

All kernels share the k order, the split, the MMA sequence and the
epilogue, so their outputs must agree bit for bit; the launch counter shows
how many kernels each ran (2 for the plane-based ones: NHWC rewrite + conv).
Against the oracle (the reference's direct conv loop) the tolerance is the
3xTF32 one: normwise max rel err <= 1e-4."""
import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu
TOL = 1e-4


def geom(n, c, h, w, cout, kh, kw, sh, sw, pt, pl, dh, dw, ho=None, wo=None):
    """Geometry with independent top/left padding; ho/wo default to the
    symmetric-padding output size."""
    if ho is None:
        ho = (h + 2 * pt - (dh * (kh - 1) + 1)) // sh + 1
    if wo is None:
        wo = (w + 2 * pl - (dw * (kw - 1) + 1)) // sw + 1
    return nb.NplkConvGeom(n, c, h, w, cout, kh, kw, sh, sw, pt, pl, dh, dw, ho, wo)


def oracle_conv_bn(x, w, g, bias, bn, act):
    """Oracle conv with explicit top/left padding and bottom/right padding
    implied by the output size, then inference BN and the activation."""
    gamma, beta, mean, var = bn
    pb = (g.h_out - 1) * g.stride_h + (g.kh - 1) * g.dil_h + 1 - g.h - g.pad_top
    pr = (g.w_out - 1) * g.stride_w + (g.kw - 1) * g.dil_w + 1 - g.w - g.pad_left
    xp = np.pad(x, ((0, 0), (0, 0), (g.pad_top, max(pb, 0)), (g.pad_left, max(pr, 0))))
    xp = xp[:, :, :g.pad_top + g.h + pb, :g.pad_left + g.w + pr]
    y = S.o_conv2d(np.ascontiguousarray(xp), w, (g.stride_h, g.stride_w), (0, 0),
                   (g.dil_h, g.dil_w), bias)
    assert y.shape[2:] == (g.h_out, g.w_out)
    return S.o_activation(S.o_batch_norm(y, mean, var, gamma, beta, 1e-5), act, 0.01)


CASES = {
    "3x3_s1_p1": geom(4, 64, 28, 28, 64, 3, 3, 1, 1, 1, 1, 1, 1),
    "3x3_s2_p1_cout96": geom(2, 32, 33, 29, 96, 3, 3, 2, 2, 1, 1, 1, 1),
    "1x1_cout200_two_blocks": geom(3, 64, 20, 20, 200, 1, 1, 1, 1, 0, 0, 1, 1),
    "1x1_s2_downsample": geom(2, 128, 28, 28, 64, 1, 1, 2, 2, 0, 0, 1, 1),
    "5x5_dil2_p4": geom(2, 32, 30, 30, 48, 5, 5, 1, 1, 4, 4, 2, 2),
    "3x3_asym_pad_t0_l2": geom(1, 32, 64, 50, 64, 3, 3, 1, 1, 0, 2, 1, 1, ho=63, wo=51),
    "3x3_hw_odd_scalar_split": geom(2, 32, 31, 31, 64, 3, 3, 1, 1, 1, 1, 1, 1),
    "3x3_wide_224": geom(1, 32, 224, 224, 32, 3, 3, 1, 1, 1, 1, 1, 1),
    "8x8_s8_patchify": geom(1, 32, 64, 64, 32, 8, 8, 8, 8, 0, 0, 1, 1),
    "3x3_s1_p0_valid_rect": geom(3, 96, 17, 40, 130, 3, 3, 1, 1, 0, 0, 1, 1),
    "7x7_s1_p3": geom(2, 32, 40, 36, 64, 7, 7, 1, 1, 3, 3, 1, 1),
    "3x3_sh2_sw1": geom(2, 64, 30, 44, 64, 3, 3, 2, 1, 1, 1, 1, 1),
    "3x3_dil3_p3": geom(2, 32, 33, 35, 40, 3, 3, 1, 1, 3, 3, 3, 3),
    "3x3_dil5_unshared": geom(1, 32, 60, 60, 64, 3, 3, 1, 1, 5, 5, 5, 5),
    "3x3_s1_cout256": geom(2, 64, 24, 24, 256, 3, 3, 1, 1, 1, 1, 1, 1),
}


ALGOS = {nb.NPLK_CONV_ALGO_DIRECT: 1, nb.NPLK_CONV_ALGO_IM2COL: 2, nb.NPLK_CONV_ALGO_WINDOW: 2,
         nb.NPLK_CONV_ALGO_WINDOW_GATHER: 1,
         nb.NPLK_CONV_ALGO_WINDOW_PAIR: 1}  # algo -> kernel launches per run


def _run(lib, g, x, w, bias, bn, act, algo, ws_bytes, work):
    import torch
    gamma, beta, mean, var = bn
    y = torch.full((g.n, g.c_out, g.h_out, g.w_out), float("nan"), device="cuda")
    s = S.cuda_stream()
    assert lib.nplk_conv2d_prepare(s, C.byref(g), S.dptr(w), S.dptr(bias), S.dptr(mean),
                                   S.dptr(var), S.dptr(gamma), S.dptr(beta), 1e-5,
                                   S.dptr(work), ws_bytes) == 0
    torch.cuda.synchronize()
    lib.nplk_take_launch_count()
    rc = lib.nplk_conv2d_run_algo(s, C.byref(g), S.dptr(x), act, 0.01, S.dptr(y), S.dptr(work),
                                  ws_bytes, None, algo)
    launches = lib.nplk_take_launch_count()
    assert rc == 0, rc
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0
    return y, launches


@pytest.mark.parametrize("name", list(CASES))
def test_all_conv_kernels_match_direct_bitwise_and_oracle(name):
    import torch
    lib = S.gpu_lib()
    g = CASES[name]
    small = lib.nplk_conv_workspace_min_size(C.byref(g))
    sizes = {a: lib.nplk_conv_workspace_size_algo(C.byref(g), a) for a in ALGOS}
    assert sizes[nb.NPLK_CONV_ALGO_DIRECT] == small
    plane = g.n * g.h * g.w * g.c_in * 4
    if sizes[nb.NPLK_CONV_ALGO_IM2COL]:
        assert sizes[nb.NPLK_CONV_ALGO_IM2COL] >= small + 2 * plane
    if sizes[nb.NPLK_CONV_ALGO_WINDOW]:
        assert sizes[nb.NPLK_CONV_ALGO_WINDOW] >= small + plane
        assert sizes[nb.NPLK_CONV_ALGO_WINDOW_GATHER] == small
    # every geometry here suits at least one TMA kernel
    assert sizes[nb.NPLK_CONV_ALGO_IM2COL] or sizes[nb.NPLK_CONV_ALGO_WINDOW]
    gen = torch.Generator(device="cuda").manual_seed(len(name))
    x = torch.rand(g.n, g.c_in, g.h, g.w, device="cuda", generator=gen) * 2 - 1
    w = torch.randn(g.c_out, g.c_in, g.kh, g.kw, device="cuda", generator=gen) * 0.05
    bias = torch.randn(g.c_out, device="cuda", generator=gen) * 0.1
    bn = [torch.rand(g.c_out, device="cuda", generator=gen) + 0.5,
          torch.rand(g.c_out, device="cuda", generator=gen) * 0.2 - 0.1,
          torch.randn(g.c_out, device="cuda", generator=gen) * 0.1,
          torch.rand(g.c_out, device="cuda", generator=gen) + 0.5]
    work = torch.empty(max(sizes.values()) // 4 + 64, device="cuda")
    act = nb.NPL_ACT_LEAKY_RELU
    outs = {}
    for algo, n_launch in ALGOS.items():
        if not sizes[algo]:
            continue
        y, launches = _run(lib, g, x, w, bias, bn, act, algo, sizes[algo], work)
        assert launches == n_launch, (algo, launches)
        outs[algo] = y.cpu().numpy()
    ref_dir = outs[nb.NPLK_CONV_ALGO_DIRECT]
    assert not np.isnan(ref_dir).any()
    for algo, a in outs.items():
        assert np.array_equal(a, ref_dir), f"algo {algo}: max diff {np.abs(a - ref_dir).max()}"
    ref = oracle_conv_bn(x.cpu().numpy(), w.cpu().numpy(), g, bias.cpu().numpy(),
                         [t.cpu().numpy() for t in bn], act)
    assert S.normwise_err(ref_dir, ref) < TOL


def test_algo_selection_rules():
    lib = S.gpu_lib()
    A = nb
    g = geom(2, 64, 28, 28, 64, 3, 3, 1, 1, 1, 1, 1, 1)     # stride 1, 3x3: windows apply
    assert lib.nplk_conv_workspace_size(C.byref(g)) == lib.nplk_conv_workspace_min_size(C.byref(g))
    assert lib.nplk_conv_workspace_size_algo(C.byref(g), A.NPLK_CONV_ALGO_WINDOW_GATHER) > 0
    g2 = geom(2, 64, 28, 28, 64, 3, 3, 2, 2, 1, 1, 1, 1)    # stride 2: im2col planes
    assert lib.nplk_conv_workspace_size(C.byref(g2)) == \
        lib.nplk_conv_workspace_size_algo(C.byref(g2), A.NPLK_CONV_ALGO_IM2COL)
    assert lib.nplk_conv_workspace_size_algo(C.byref(g2), 99) == 0


def test_small_or_unaligned_geometries_keep_the_direct_path():
    lib = S.gpu_lib()
    for g in (geom(1, 3, 224, 224, 64, 7, 7, 2, 2, 3, 3, 1, 1),    # C_in % 32 != 0
              geom(1, 32, 8, 8, 32, 3, 3, 1, 1, 1, 1, 1, 1),        # input plane < 128 KiB
              geom(1, 32, 64, 64, 32, 9, 9, 9, 9, 0, 0, 1, 1)):     # stride above 8
        assert lib.nplk_conv_workspace_size(C.byref(g)) == \
            lib.nplk_conv_workspace_min_size(C.byref(g))
        for algo in (nb.NPLK_CONV_ALGO_IM2COL, nb.NPLK_CONV_ALGO_WINDOW,
                     nb.NPLK_CONV_ALGO_WINDOW_GATHER):
            assert lib.nplk_conv_workspace_size_algo(C.byref(g), algo) == 0
