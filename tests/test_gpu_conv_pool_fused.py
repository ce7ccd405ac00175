"""The fused stem block nplk_conv2d_maxpool_fused (conv + BN + activation,
then 3x3/s2/p1 max pool) against the two separate calls it replaces --
nplk_conv2d_fused then nplk_pool2d, i.e. the reference's
npl_conv2d_bn_activation (npl_convolution.cpp:92-137) then npl_pooling max
(npl_pooling.cpp:129-219) -- bit for bit, and against the oracle within the
3xTF32 tolerance. Geometries cover GEMM tiles that start mid-row and straddle
images (the left neighbour from the previous tile), negative outputs
(no activation), an odd number of output rows and both row-order widths."""
import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu

CASES = {
    # name: (n, c, h, w, cout, k, stride, pad, act)
    "stem_224_relu": (4, 3, 224, 224, 64, 7, 2, 3, nb.NPL_ACT_RELU),
    "7x7_100_no_act": (3, 3, 100, 100, 64, 7, 2, 3, 0),
    "7x7_odd_rows_leaky": (2, 3, 101, 100, 48, 7, 2, 3, nb.NPL_ACT_LEAKY_RELU),
    "3x3_s1_row_order_4": (2, 3, 64, 64, 32, 3, 1, 1, nb.NPL_ACT_RELU),
    "5x5_s2_c5": (2, 5, 92, 92, 64, 5, 2, 2, 0),
}


def _inputs(g, seed):
    import torch
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.rand(g.n, g.c_in, g.h, g.w, device="cuda", generator=gen) * 2 - 1
    w = torch.randn(g.c_out, g.c_in, g.kh, g.kw, device="cuda", generator=gen) * 0.2
    bias = torch.randn(g.c_out, device="cuda", generator=gen) * 0.1
    bn = [torch.rand(g.c_out, device="cuda", generator=gen) + 0.5,      # gamma
          torch.rand(g.c_out, device="cuda", generator=gen) * 0.2 - 0.1,  # beta
          torch.randn(g.c_out, device="cuda", generator=gen) * 0.1,      # mean
          torch.rand(g.c_out, device="cuda", generator=gen) + 0.5]       # var
    return x, w, bias, bn


@pytest.mark.parametrize("name", list(CASES))
def test_fused_conv_maxpool_matches_conv_then_pool_bitwise(name):
    import torch
    lib = S.gpu_lib()
    n, c, h, w_, cout, k, stride, pad, act = CASES[name]
    g = nb.conv_geom(n, c, h, w_, cout, k, k, stride, pad)
    x, w, bias, bn = _inputs(g, len(name))
    gamma, beta, mean, var = bn
    s = S.cuda_stream()
    po, wp = (g.h_out - 1) // 2 + 1, g.w_out // 2
    # the two separate calls
    ws = lib.nplk_conv_workspace_size(C.byref(g))
    work = torch.empty(ws // 4 + 64, device="cuda")
    y = torch.empty(g.n, g.c_out, g.h_out, g.w_out, device="cuda")
    assert lib.nplk_conv2d_fused(s, C.byref(g), S.dptr(x), S.dptr(w), S.dptr(bias), S.dptr(mean),
                                 S.dptr(var), S.dptr(gamma), S.dptr(beta), 1e-5, act, 0.01,
                                 S.dptr(y), S.dptr(work), ws, None) == 0
    ref = torch.empty(g.n, g.c_out, po, wp, device="cuda")
    assert lib.nplk_pool2d(s, g.n, g.c_out, g.h_out, g.w_out, 3, 3, 2, 2, 1, 1, po, wp, 0, 0,
                           S.dptr(y), S.dptr(ref)) == 0
    # the fused call
    fws = lib.nplk_conv2d_maxpool_workspace_size(C.byref(g))
    assert fws > 0
    fwork = torch.empty(fws // 4 + 64, device="cuda")
    out = torch.full((g.n, g.c_out, po, wp), float("nan"), device="cuda")
    lib.nplk_take_launch_count()
    assert lib.nplk_conv2d_maxpool_fused(s, C.byref(g), S.dptr(x), S.dptr(w), S.dptr(bias),
                                         S.dptr(mean), S.dptr(var), S.dptr(gamma), S.dptr(beta),
                                         1e-5, act, 0.01, S.dptr(out), S.dptr(fwork), fws,
                                         None) == 0
    assert lib.nplk_take_launch_count() == 3  # weight preparation, conv, vertical pass
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0
    got, want = out.cpu().numpy(), ref.cpu().numpy()
    assert not np.isnan(got).any()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"max diff {np.abs(got - want).max()}"
    # and the oracle: conv (3xTF32 tolerance) -> BN -> activation -> pool
    xo = x.cpu().numpy()
    yo = S.o_conv2d(xo, w.cpu().numpy(), (stride, stride), (pad, pad), bias=bias.cpu().numpy())
    yo = S.o_activation(S.o_batch_norm(yo, mean.cpu().numpy(), var.cpu().numpy(),
                                       gamma.cpu().numpy(), beta.cpu().numpy()), act, 0.01)
    assert S.normwise_err(got, S.o_pool(yo, (3, 3), (2, 2), (1, 1), 0)) < 1e-4


def test_fused_conv_maxpool_rejects_other_geometries():
    import torch
    lib = S.gpu_lib()
    for g in (nb.conv_geom(2, 64, 56, 56, 64, 3, 3, 1, 1),   # C_in % 32 == 0: not the row order
              nb.conv_geom(2, 3, 224, 224, 96, 7, 7, 2, 3),  # C_out > 64
              nb.conv_geom(2, 3, 225, 225, 64, 7, 7, 2, 3)):  # odd output width (113)
        assert lib.nplk_conv2d_maxpool_workspace_size(C.byref(g)) == 0
        dummy = torch.empty(64, device="cuda")
        assert lib.nplk_conv2d_maxpool_fused(S.cuda_stream(), C.byref(g), S.dptr(dummy),
                                             S.dptr(dummy), None, None, None, None, None, 1e-5,
                                             1, 0.0, S.dptr(dummy), S.dptr(dummy), 256,
                                             None) == nb.NPL_ERR_UNSUPPORTED
