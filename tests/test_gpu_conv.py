"""Parity of the tcgen05 implicit-GEMM convolution (npl_conv2d,
npl_conv2d_bn_activation, nplk_conv2d_fused) with the oracle: the reference's
direct conv loop, followed for the fused op by the reference's inference batch
norm and activation. Tolerance: normwise max relative error <= 1e-4 (3xTF32)."""
import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu
TOL = 1e-4


def bn_params(c, rng):
    gamma = rng.uniform(0.5, 1.5, c).astype(np.float32)
    beta = rng.uniform(-0.1, 0.1, c).astype(np.float32)
    mean = rng.normal(0, 0.1, c).astype(np.float32)
    var = rng.uniform(0.5, 1.5, c).astype(np.float32)
    return gamma, beta, mean, var


def conv_host(lib, x, w, bias=None, stride=(1, 1), pad=(0, 0), dil=(1, 1),
              padding=nb.NPL_PAD_EXPLICIT, out_shape=None, layout=nb.NPL_LAYOUT_NCHW):
    h = S.HostTensors(lib)
    if out_shape is None:
        ho, wo = S.conv_out_hw(x.shape[2], x.shape[3], w.shape[2], w.shape[3], stride[0],
                               stride[1], pad[0], pad[0], pad[1], pad[1], dil[0], dil[1])
        out_shape = (x.shape[0], w.shape[0], ho, wo)
    y = np.zeros(out_shape, np.float32)
    p = nb.conv_params(w.shape[2], w.shape[3], stride, pad, dil, padding=padding)
    rc = S.npl_call(lib, "npl_conv2d", h.t(x, layout), h.t(w),
                    h.t(bias) if bias is not None else None, p, h.t(y), None)
    return rc, y


def fused_host(lib, x, w, bn, act, stride=(1, 1), pad=(0, 0), bias=None):
    gamma, beta, mean, var = bn
    h = S.HostTensors(lib)
    ho, wo = S.conv_out_hw(x.shape[2], x.shape[3], w.shape[2], w.shape[3], stride[0],
                           stride[1], pad[0], pad[0], pad[1], pad[1])
    y = np.zeros((x.shape[0], w.shape[0], ho, wo), np.float32)
    p = nb.conv_params(w.shape[2], w.shape[3], stride, pad, padding=nb.NPL_PAD_EXPLICIT)
    bnp = nb.NplBatchnormParams(mean.ctypes.data, var.ctypes.data, gamma.ctypes.data,
                                beta.ctypes.data, 1e-5, 0, 0.1)
    st = nb.NplPerfStats()
    rc = S.npl_call(lib, "npl_conv2d_bn_activation", h.t(x), h.t(w),
                    h.t(bias) if bias is not None else None, p, bnp, act, h.t(y), st)
    assert rc == 0, lib.npl_strerror(rc)
    return y, st


def oracle_fused(x, w, bn, act, stride=(1, 1), pad=(0, 0), bias=None):
    gamma, beta, mean, var = bn
    conv = S.o_conv2d(x, w, stride, pad, bias=bias)
    return S.o_activation(S.o_batch_norm(conv, mean, var, gamma, beta, 1e-5), act, 0.01)


def test_conv2d_known_answer():
    # npl_test.cpp:206-274: expected 27.5 everywhere
    rc, y = conv_host(S.gpu_lib(), np.ones((1, 3, 8, 8), np.float32),
                      np.ones((2, 3, 3, 3), np.float32), np.full(2, 0.5, np.float32),
                      padding=nb.NPL_PAD_VALID)
    assert rc == 0 and y.shape == (1, 2, 6, 6)
    assert np.all(np.abs(y - 27.5) < 0.01)


@pytest.mark.parametrize("name", ["conv2d_winograd", "conv2d_direct"])
def test_conv2d_golden(name):
    g = dict(np.load(S.GOLDEN / f"{name}.npz"))
    rc, y = conv_host(S.gpu_lib(), g["x"], g["w"], g["bias"], tuple(g["stride"]),
                      tuple(g["pad"]), tuple(g["dil"]))
    assert rc == 0
    assert S.normwise_err(y, g["y"]) < TOL


def test_conv_bn_relu_golden():
    g = dict(np.load(S.GOLDEN / "conv_bn_relu.npz"))
    y, st = fused_host(S.gpu_lib(), g["x"], g["w"], (g["gamma"], g["beta"], g["mean"], g["var"]),
                       nb.NPL_ACT_RELU, pad=(1, 1))
    assert S.normwise_err(y, g["y"]) < TOL
    assert st.was_fused == 1


def test_conv_bn_relu_3x3_n32_c64_56x56_full():
    # ResNet 3x3 layer: N=32, Cin=64, 56x56, Cout=64, stride 1, pad 1, no bias.
    lib = S.gpu_lib()
    rng = S.rng(0)
    x = rng.uniform(0, 1, (32, 64, 56, 56)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / (9 * 64)), (64, 64, 3, 3)).astype(np.float32)
    bn = bn_params(64, rng)
    y, st = fused_host(lib, x, w, bn, nb.NPL_ACT_RELU, pad=(1, 1))
    err = S.normwise_err(y, oracle_fused(x, w, bn, 1, pad=(1, 1)))
    print(f"3x3 N=32 64->64 56x56 normwise err {err:.3e}")
    assert err < TOL


def test_stem_conv_bn_relu_then_maxpool():
    # Stem block family (N reduced from 128 to 4; per-image work identical):
    # 7x7/s2/p3, Cin=3, Cout=64 -> 112x112, BN, ReLU; then max pool 3x3/s2/p1.
    lib = S.gpu_lib()
    rng = S.rng(1)
    x = rng.uniform(-1, 1, (4, 3, 224, 224)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / 147), (64, 3, 7, 7)).astype(np.float32)
    bn = bn_params(64, rng)
    y, _ = fused_host(lib, x, w, bn, nb.NPL_ACT_RELU, stride=(2, 2), pad=(3, 3))
    ref = oracle_fused(x, w, bn, 1, stride=(2, 2), pad=(3, 3))
    assert S.normwise_err(y, ref) < TOL
    h = S.HostTensors(lib)
    pooled = np.zeros((4, 64, 56, 56), np.float32)
    pp = nb.NplPoolingParams(3, 3, 2, 2, 1, 1, nb.NPL_POOL_MAX, 0)
    assert S.npl_call(lib, "npl_pooling", h.t(y), pp, h.t(pooled), None) == 0
    assert np.array_equal(pooled, S.o_pool(y, (3, 3), (2, 2), (1, 1), 0))


@pytest.mark.parametrize("n,cin,h,w,cout,k,stride,pad,dil", [
    (1, 1, 5, 5, 1, (1, 1), (1, 1), (0, 0), (1, 1)),
    (2, 3, 17, 13, 5, (3, 3), (2, 2), (1, 1), (1, 1)),
    (1, 16, 20, 20, 130, (3, 3), (1, 1), (1, 1), (1, 1)),   # two Cout blocks of 128
    (3, 32, 9, 11, 64, (1, 1), (1, 1), (0, 0), (1, 1)),
    (1, 5, 30, 30, 7, (5, 5), (3, 2), (2, 1), (1, 1)),
    (2, 8, 16, 16, 12, (3, 3), (1, 1), (2, 2), (2, 2)),     # dilation 2
    (1, 100, 7, 7, 96, (3, 3), (1, 1), (1, 1), (1, 1)),     # K = 900, not a multiple of 32
    (5, 3, 31, 33, 64, (7, 7), (2, 2), (3, 3), (1, 1)),     # tiles straddle images
    (1, 12, 15, 16, 33, (4, 4), (2, 2), (1, 1), (1, 1)),    # row order, 4 slots all used
    (2, 7, 19, 23, 40, (2, 6), (1, 2), (0, 2), (1, 1)),     # row order, 8 slots, KH != KW
    (2, 6, 20, 18, 16, (3, 5), (1, 1), (2, 2), (2, 1)),     # row order with vertical dilation
    (2, 16, 32, 32, 130, (3, 3), (1, 1), (1, 1), (1, 1)),   # row order, 16 x 8 tiles, two Cout blocks
    (3, 3, 64, 64, 64, (7, 7), (2, 2), (3, 3), (1, 1)),     # stem-like, 16 x 8 tiles over 3 images
])
def test_conv2d_shapes(n, cin, h, w, cout, k, stride, pad, dil):
    lib = S.gpu_lib()
    rng = S.rng(n * 100 + cin + cout)
    x = rng.uniform(-1, 1, (n, cin, h, w)).astype(np.float32)
    wt = rng.normal(0, 0.2, (cout, cin, *k)).astype(np.float32)
    bias = rng.normal(0, 0.1, cout).astype(np.float32)
    rc, y = conv_host(lib, x, wt, bias, stride, pad, dil)
    assert rc == 0
    assert S.normwise_err(y, S.o_conv2d(x, wt, stride, pad, dil, bias)) < TOL


@pytest.mark.parametrize("act", [nb.NPL_ACT_NONE, nb.NPL_ACT_RELU6, nb.NPL_ACT_LEAKY_RELU,
                                 nb.NPL_ACT_SIGMOID, nb.NPL_ACT_TANH, nb.NPL_ACT_GELU,
                                 nb.NPL_ACT_SWISH, nb.NPL_ACT_ELU])
def test_fused_activations(act):
    lib = S.gpu_lib()
    rng = S.rng(act)
    x = rng.uniform(-1, 1, (2, 16, 12, 12)).astype(np.float32)
    w = rng.normal(0, 0.3, (24, 16, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, 24).astype(np.float32)
    bn = bn_params(24, rng)
    y, _ = fused_host(lib, x, w, bn, act, pad=(1, 1), bias=bias)
    assert S.normwise_err(y, oracle_fused(x, w, bn, act, pad=(1, 1), bias=bias)) < TOL


def test_conv_same_padding_and_nhwc_layout_quirk():
    lib = S.gpu_lib()
    rng = S.rng(11)
    x = rng.uniform(-1, 1, (1, 4, 10, 10)).astype(np.float32)
    w = rng.normal(0, 0.3, (3, 4, 3, 3)).astype(np.float32)
    # SAME, stride 1: total pad k-1 = 2 split 1/1 (npl_convolution.cpp:204-214)
    rc, y = conv_host(lib, x, w, padding=nb.NPL_PAD_SAME, out_shape=(1, 3, 10, 10))
    assert rc == 0 and S.normwise_err(y, S.o_conv2d(x, w, pad=(1, 1))) < TOL
    # VALID still takes pad_h/pad_w (npl_convolution.cpp:219-222)
    rc, y = conv_host(lib, x, w, pad=(1, 1), padding=nb.NPL_PAD_VALID)
    assert rc == 0 and S.normwise_err(y, S.o_conv2d(x, w, pad=(1, 1))) < TOL
    # An NHWC tag changes how the dimensions are read, not the indexing
    # (PrepareConvContext reads [N,H,W,C]; ExecuteConvDirect indexes NCHW).
    xn = rng.uniform(-1, 1, (1, 6, 5, 4)).astype(np.float32)   # N=1, H=6, W=5, C=4
    rc, y = conv_host(lib, xn, w, pad=(1, 1), layout=nb.NPL_LAYOUT_NHWC,
                      out_shape=(1, 3, 6, 5))
    assert rc == 0
    as_nchw = xn.reshape(1, 4, 6, 5)
    assert S.normwise_err(y, S.o_conv2d(as_nchw, w, pad=(1, 1))) < TOL


def test_conv_errors():
    lib = S.gpu_lib()
    x = np.ones((1, 3, 8, 8), np.float32)
    w = np.ones((2, 3, 3, 3), np.float32)
    h = S.HostTensors(lib)
    y = np.zeros((1, 2, 6, 6), np.float32)
    p = nb.conv_params(3, 3, 0, 0)
    assert S.npl_call(lib, "npl_conv2d", h.t(x), h.t(w), None, p, h.t(y), None) == \
        nb.NPL_ERR_INVALID_ARG
    p = nb.conv_params(3, 3, 1, 0, groups=0)
    assert S.npl_call(lib, "npl_conv2d", h.t(x), h.t(w), None, p, h.t(y), None) == \
        nb.NPL_ERR_INVALID_ARG
    small = np.zeros((1, 2, 5, 5), np.float32)
    p = nb.conv_params(3, 3, 1, 0)
    assert S.npl_call(lib, "npl_conv2d", h.t(x), h.t(w), None, p, h.t(small), None) == \
        nb.NPL_ERR_SHAPE_MISMATCH
    assert S.npl_call(lib, "npl_conv2d", None, h.t(w), None, p, h.t(y), None) == \
        nb.NPL_ERR_INVALID_ARG


def test_conv_device_pointers_and_stats():
    import torch
    lib = S.gpu_lib()
    g = nb.conv_geom(8, 64, 28, 28, 64, 3, 3, 1, 1)
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = torch.rand(8, 64, 28, 28, device="cuda", generator=gen)
    w = torch.randn(64, 64, 3, 3, device="cuda", generator=gen) * 0.05
    y = torch.empty(8, 64, 28, 28, device="cuda")
    ws = lib.nplk_conv_workspace_size(C.byref(g))
    work = torch.empty(ws // 4 + 64, device="cuda")
    rc = lib.nplk_conv2d_fused(S.cuda_stream(), C.byref(g), S.dptr(x), S.dptr(w), None, None,
                               None, None, None, 0.0, 1, 0.0, S.dptr(y), S.dptr(work), ws, None)
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    xn, wn = x.cpu().numpy(), w.cpu().numpy()
    ref = S.o_activation(S.o_conv2d(xn, wn, pad=(1, 1)), 1)
    assert S.normwise_err(y.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("n", [16, 13])
def test_conv_bn_act_pinned_host_buffers_pipelined(n):
    # Page-locked host input/output take the chunked copy/compute pipeline
    # (n = 13: the last chunk is ragged); per-image results are those of the
    # same call on device tensors, bit for bit.
    import torch
    lib = S.gpu_lib()
    gen = torch.Generator().manual_seed(n)
    x = torch.rand(n, 64, 56, 56, generator=gen).pin_memory()
    w = (torch.randn(64, 64, 3, 3, generator=gen) * 0.05).pin_memory()
    bn = [(torch.rand(64, generator=gen) + 0.5) for _ in range(4)]
    y = torch.zeros(n, 64, 56, 56).pin_memory()
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    bnp = nb.NplBatchnormParams(bn[0].data_ptr(), bn[1].data_ptr(), bn[2].data_ptr(),
                                bn[3].data_ptr(), 1e-5, 0, 0.1)
    t = lambda a: nb.tensor(lib, a.data_ptr(), a.shape)  # noqa: E731
    st = nb.NplPerfStats()
    rc = lib.npl_conv2d_bn_activation(C.byref(t(x)), C.byref(t(w)), None, C.byref(p),
                                      C.byref(bnp), nb.NPL_ACT_RELU, C.byref(t(y)), C.byref(st))
    assert rc == 0
    assert st.was_fused == 1 and st.elapsed_ms > 0
    xd, wd, yd = x.cuda(), w.cuda(), torch.zeros(n, 64, 56, 56, device="cuda")
    bnd = [v.cuda() for v in bn]
    bnpd = nb.NplBatchnormParams(*(v.data_ptr() for v in bnd), 1e-5, 0, 0.1)
    rc = lib.npl_conv2d_bn_activation(C.byref(t(xd)), C.byref(t(wd)), None, C.byref(p),
                                      C.byref(bnpd), nb.NPL_ACT_RELU, C.byref(t(yd)), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(y, yd.cpu())
    mean, var, gamma, beta = (b.numpy() for b in bn)
    ref = oracle_fused(x[:2].numpy(), w.numpy(), (gamma, beta, mean, var), 1, pad=(1, 1))
    assert S.normwise_err(y[:2].numpy(), ref) < TOL
