"""Cross-checks the C oracle against the reference's own NPL code
(oracle/_ref/libnpl_ref.so, built from the reference sources) on seeded
random inputs with the benchmark workloads' shape families at reduced sizes, plus edge
cases. Skipped where the reference build is absent."""
import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.skipif(not S.REF_LIB.exists(), reason="reference build absent")


def ref():
    return S.reference()


def test_matmul_vs_reference_openblas():
    lib = ref()
    rng = S.rng(1)
    for (m, k, n, alpha, beta) in [(64, 48, 80, 1.0, 0.0), (129, 257, 31, 0.5, 1.0),
                                   (600, 520, 530, 1.0, 0.0)]:
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        c0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
        h = S.HostTensors(lib)
        c = c0.copy()
        assert S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(alpha),
                          C.c_float(beta), None) == 0
        o = S.o_sgemm(a, b, alpha, beta, c0)
        assert S.normwise_err(c, o) < 1e-6


@pytest.mark.parametrize("shape,k,stride,pad", [
    ((2, 8, 14, 14), (3, 3), (1, 1), (1, 1)),    # ResNet 3x3 family (Winograd in the reference)
    ((2, 3, 23, 23), (2, 2), (2, 2), (1, 1)),    # direct path, stride 2
    ((1, 4, 9, 11), (3, 1), (1, 2), (0, 1)),     # asymmetric
])
def test_conv_vs_reference(shape, k, stride, pad):
    lib = ref()
    rng = S.rng(2)
    x = rng.uniform(-1, 1, shape).astype(np.float32)
    w = rng.normal(0, 0.2, (6, shape[1], *k)).astype(np.float32)
    bias = rng.normal(0, 0.1, 6).astype(np.float32)
    o = S.o_conv2d(x, w, stride, pad, bias=bias)
    y = np.zeros_like(o)
    h = S.HostTensors(lib)
    p = nb.conv_params(k[0], k[1], stride, pad, padding=nb.NPL_PAD_EXPLICIT)
    assert S.npl_call(lib, "npl_conv2d", h.t(x), h.t(w), h.t(bias), p, h.t(y), None) == 0
    assert S.normwise_err(y, o) < 2e-6


def test_conv7x7_reference_fails_as_documented():
    # The reference's im2col path (kernel area > 9) always fails
    # (npl_convolution.cpp:240-241, 380-526); the oracle computes the conv.
    lib = ref()
    x = np.ones((1, 3, 16, 16), np.float32)
    w = np.ones((4, 3, 7, 7), np.float32)
    y = np.zeros((1, 4, 8, 8), np.float32)
    h = S.HostTensors(lib)
    p = nb.conv_params(7, 7, 2, 3, padding=nb.NPL_PAD_EXPLICIT)
    rc = S.npl_call(lib, "npl_conv2d", h.t(x), h.t(w), None, p, h.t(y), None)
    assert rc in (nb.NPL_ERR_INTERNAL, nb.NPL_ERR_NOT_INITIALIZED)
    assert S.o_conv2d(x, w, (2, 2), (3, 3))[0, 0, 4, 4] == 147.0


def test_fused_reference_is_conv_only():
    # npl_conv2d_bn_activation in the reference skips BN and the activation
    # (npl_convolution.cpp:116-126): its output equals the plain conv.
    lib = ref()
    rng = S.rng(3)
    x = rng.uniform(-1, 1, (1, 3, 8, 8)).astype(np.float32)
    w = rng.normal(0, 0.3, (4, 3, 3, 3)).astype(np.float32)
    mean = np.full(4, 5.0, np.float32)
    var = np.full(4, 4.0, np.float32)
    bn = nb.NplBatchnormParams(mean.ctypes.data, var.ctypes.data, None, None, 1e-5, 0, 0.1)
    y = np.zeros((1, 4, 8, 8), np.float32)
    h = S.HostTensors(lib)
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    assert S.npl_call(lib, "npl_conv2d_bn_activation", h.t(x), h.t(w), None, p, bn,
                      nb.NPL_ACT_RELU, h.t(y), None) == 0
    assert S.normwise_err(y, S.o_conv2d(x, w, pad=(1, 1))) < 1e-6
    assert (y < 0).any()  # no ReLU applied


def test_bandwidth_ops_vs_reference():
    lib = ref()
    rng = S.rng(4)
    x = rng.normal(0, 1, (4, 16, 14, 14)).astype(np.float32)
    h = S.HostTensors(lib)
    # depthwise
    w = rng.normal(0, 0.3, (16, 1, 3, 3)).astype(np.float32)
    y = np.zeros_like(x)
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    assert S.npl_call(lib, "npl_depthwise_conv2d", h.t(x), h.t(w), None, p, h.t(y), None) == 0
    assert np.array_equal(y, S.o_depthwise(x, w, pad=(1, 1)))
    # batch norm
    mean = rng.normal(0, 0.1, 16).astype(np.float32)
    var = rng.uniform(0.5, 1.5, 16).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 16).astype(np.float32)
    beta = rng.uniform(-0.1, 0.1, 16).astype(np.float32)
    bn = nb.NplBatchnormParams(mean.ctypes.data, var.ctypes.data, gamma.ctypes.data,
                               beta.ctypes.data, 1e-5, 0, 0.1)
    y = np.zeros_like(x)
    assert S.npl_call(lib, "npl_batch_norm", h.t(x), bn, h.t(y), None) == 0
    assert S.normwise_err(y, S.o_batch_norm(x, mean, var, gamma, beta)) < 1e-6
    # gap, softmax
    g = np.zeros((4, 16), np.float32)
    assert S.npl_call(lib, "npl_global_avg_pool", h.t(x), h.t(g), None) == 0
    assert np.array_equal(g, S.o_gap(x))
    s = np.zeros_like(g)
    assert S.npl_call(lib, "npl_softmax", h.t(g), 1, h.t(s), None) == 0
    assert S.normwise_err(s, S.o_softmax(g, 1)) < 1e-6
    # max pool
    y = np.zeros((4, 16, 7, 7), np.float32)
    pp = nb.NplPoolingParams(3, 3, 2, 2, 1, 1, nb.NPL_POOL_MAX, 0)
    assert S.npl_call(lib, "npl_pooling", h.t(x), pp, h.t(y), None) == 0
    assert np.array_equal(y, S.o_pool(x, (3, 3), (2, 2), (1, 1), 0))
    # layer norm over a long row
    xl = rng.normal(0, 1, (3, 4096)).astype(np.float32)
    yl = np.zeros_like(xl)
    lp = nb.NplLayernormParams(None, None, 1e-5, 4096)
    assert S.npl_call(lib, "npl_layer_norm", h.t(xl), lp, h.t(yl), None) == 0
    assert S.normwise_err(yl, S.o_layer_norm(xl, 4096)) < 1e-6
