"""Generates the golden fixtures in this directory from the reference's own
NPL code. The reference sources are compiled for the CPU by
``make -C oracle ref`` into oracle/_ref/libnpl_ref.so (test infrastructure).

Every fixture is a small seeded case (inputs, parameters and the reference's
outputs) saved as ``<name>.npz``. The tests use them to pin the C oracle
(tests/test_oracle_golden.py) and the B200 library (the golden cases of
tests/test_gpu_gemm.py, test_gpu_conv.py and test_gpu_bandwidth.py) to the
reference on machines where the reference tree is absent.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

import support as S  # noqa: E402
from support import nb  # noqa: E402


def _ref():
    lib = S.reference()
    if lib is None:
        raise SystemExit(f"{S.REF_LIB} missing: build it with `make -C oracle ref`")
    return lib


def _t(h, a, layout=nb.NPL_LAYOUT_NCHW):
    return h.t(np.ascontiguousarray(a, dtype=np.float32), layout)


def matmul(lib, rng):
    out = {}
    a = rng.uniform(-1, 1, (17, 33)).astype(np.float32)
    b = rng.uniform(-1, 1, (33, 9)).astype(np.float32)
    c0 = rng.uniform(-1, 1, (17, 9)).astype(np.float32)
    h = S.HostTensors(lib)
    c = c0.copy()
    ta, tb, tc = _t(h, a), _t(h, b), h.t(c)
    assert S.npl_call(lib, "npl_matmul", ta, tb, tc, C.c_float(1.5), C.c_float(0.5), None) == 0
    out.update(a=a, b=b, c0=c0, alpha=np.float32(1.5), beta=np.float32(0.5), c=c)
    # the reference's own known-answer case: 32^3 of ones -> every element 32
    ones = np.ones((32, 32), np.float32)
    c1 = np.zeros((32, 32), np.float32)
    assert S.npl_call(lib, "npl_matmul", _t(h, ones), _t(h, ones), h.t(c1), C.c_float(1.0),
                      C.c_float(0.0), None) == 0
    out.update(ones_c=c1)
    return out


def conv2d_winograd(lib, rng):
    # 3x3, stride 1, dilation 1: the reference runs Winograd F(2x2,3x3).
    x = rng.uniform(-1, 1, (2, 3, 10, 9)).astype(np.float32)
    w = rng.normal(0, 0.3, (4, 3, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, (4,)).astype(np.float32)
    y = np.zeros((2, 4, 10, 9), np.float32)
    h = S.HostTensors(lib)
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    assert S.npl_call(lib, "npl_conv2d", _t(h, x), _t(h, w), _t(h, bias), p, h.t(y), None) == 0
    return dict(x=x, w=w, bias=bias, y=y, stride=[1, 1], pad=[1, 1], dil=[1, 1])


def conv2d_direct(lib, rng):
    # kernel area <= 9 and not 3x3/s1: the reference's direct loop.
    x = rng.uniform(-1, 1, (1, 2, 9, 8)).astype(np.float32)
    w = rng.normal(0, 0.3, (3, 2, 2, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, (3,)).astype(np.float32)
    stride, pad, dil = [2, 1], [1, 0], [1, 2]
    ho, wo = S.conv_out_hw(9, 8, 2, 3, 2, 1, 1, 1, 0, 0, 1, 2)
    y = np.zeros((1, 3, ho, wo), np.float32)
    h = S.HostTensors(lib)
    p = nb.conv_params(2, 3, stride, pad, dil, padding=nb.NPL_PAD_EXPLICIT)
    assert S.npl_call(lib, "npl_conv2d", _t(h, x), _t(h, w), _t(h, bias), p, h.t(y), None) == 0
    return dict(x=x, w=w, bias=bias, y=y, stride=stride, pad=pad, dil=dil)


def conv_bn_relu(lib, rng):
    # The reference's fused call runs the conv only; the fixture composes it
    # with the reference's npl_batch_norm and npl_relu, the specified result.
    x = rng.uniform(0, 1, (2, 4, 7, 7)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / 36), (5, 4, 3, 3)).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 5).astype(np.float32)
    beta = rng.uniform(-0.1, 0.1, 5).astype(np.float32)
    mean = rng.normal(0, 0.1, 5).astype(np.float32)
    var = rng.uniform(0.5, 1.5, 5).astype(np.float32)
    h = S.HostTensors(lib)
    conv = np.zeros((2, 5, 7, 7), np.float32)
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    bn = nb.NplBatchnormParams(mean.ctypes.data, var.ctypes.data, gamma.ctypes.data,
                               beta.ctypes.data, 1e-5, 0, 0.1)
    assert S.npl_call(lib, "npl_conv2d_bn_activation", _t(h, x), _t(h, w), None, p, bn,
                      nb.NPL_ACT_RELU, h.t(conv), None) == 0
    bnout = np.zeros_like(conv)
    assert S.npl_call(lib, "npl_batch_norm", h.t(conv), bn, h.t(bnout), None) == 0
    y = np.zeros_like(conv)
    assert S.npl_call(lib, "npl_relu", h.t(bnout), h.t(y), None) == 0
    return dict(x=x, w=w, gamma=gamma, beta=beta, mean=mean, var=var, conv_only=conv, y=y)


def depthwise(lib, rng):
    x = rng.normal(0, 1, (2, 3, 7, 6)).astype(np.float32)
    w = rng.normal(0, 0.3, (3, 1, 3, 3)).astype(np.float32)
    bias = rng.normal(0, 0.1, 3).astype(np.float32)
    y = np.zeros((2, 3, 7, 6), np.float32)
    h = S.HostTensors(lib)
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    assert S.npl_call(lib, "npl_depthwise_conv2d", _t(h, x), _t(h, w), _t(h, bias), p, h.t(y),
                      None) == 0
    return dict(x=x, w=w, bias=bias, y=y)


def batch_norm(lib, rng):
    x = rng.normal(0, 1, (2, 3, 5, 4)).astype(np.float32)
    mean = rng.normal(0, 0.1, 3).astype(np.float32)
    var = rng.uniform(0.5, 1.5, 3).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 3).astype(np.float32)
    beta = rng.uniform(-0.1, 0.1, 3).astype(np.float32)
    h = S.HostTensors(lib)
    y = np.zeros_like(x)
    bn = nb.NplBatchnormParams(mean.ctypes.data, var.ctypes.data, gamma.ctypes.data,
                               beta.ctypes.data, 1e-5, 0, 0.1)
    assert S.npl_call(lib, "npl_batch_norm", _t(h, x), bn, h.t(y), None) == 0
    rm, rv = mean.copy(), var.copy()
    yt = np.zeros_like(x)
    bnt = nb.NplBatchnormParams(rm.ctypes.data, rv.ctypes.data, gamma.ctypes.data,
                                beta.ctypes.data, 1e-5, 1, 0.1)
    assert S.npl_call(lib, "npl_batch_norm", _t(h, x), bnt, h.t(yt), None) == 0
    return dict(x=x, mean=mean, var=var, gamma=gamma, beta=beta, y=y, y_train=yt,
                run_mean=rm, run_var=rv)


def activations(lib, rng):
    x = np.concatenate([rng.normal(0, 2, 997).astype(np.float32),
                        np.array([0.0, -0.0, 7.5], np.float32)])
    h = S.HostTensors(lib)
    out = {"x": x}
    for name, act in [("relu", nb.NPL_ACT_RELU), ("relu6", nb.NPL_ACT_RELU6),
                      ("tanh", nb.NPL_ACT_TANH), ("sigmoid", nb.NPL_ACT_SIGMOID),
                      ("gelu", nb.NPL_ACT_GELU), ("swish", nb.NPL_ACT_SWISH),
                      ("leaky", nb.NPL_ACT_LEAKY_RELU), ("elu", nb.NPL_ACT_ELU),
                      ("selu", nb.NPL_ACT_SELU), ("softplus", nb.NPL_ACT_SOFTPLUS)]:
        y = np.zeros_like(x)
        assert S.npl_call(lib, "npl_activation", _t(h, x), act, h.t(y), None) == 0
        out[name] = y
    y = np.zeros_like(x)
    assert S.npl_call(lib, "npl_leaky_relu", _t(h, x), C.c_float(0.2), h.t(y), None) == 0
    out["leaky_0p2"] = y
    return out


def softmax(lib, rng):
    h = S.HostTensors(lib)
    x2 = np.tile(np.arange(10, dtype=np.float32), (2, 1))  # the reference test's input
    y2 = np.zeros_like(x2)
    assert S.npl_call(lib, "npl_softmax", _t(h, x2), 1, h.t(y2), None) == 0
    x3 = rng.normal(0, 3, (4, 5, 6)).astype(np.float32)
    y3 = np.zeros_like(x3)
    assert S.npl_call(lib, "npl_softmax", _t(h, x3), -2, h.t(y3), None) == 0
    return dict(x2=x2, y2=y2, x3=x3, y3=y3)


def layer_norm(lib, rng):
    h = S.HostTensors(lib)
    x = (np.arange(4 * 128) % 20 - 10).astype(np.float32).reshape(4, 128)
    y = np.zeros_like(x)
    p = nb.NplLayernormParams(None, None, 1e-5, 128)
    assert S.npl_call(lib, "npl_layer_norm", _t(h, x), p, h.t(y), None) == 0
    x2 = rng.normal(1, 2, (3, 7)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, 7).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, 7).astype(np.float32)
    y2 = np.zeros_like(x2)
    p2 = nb.NplLayernormParams(g.ctypes.data, b.ctypes.data, 1e-5, 7)
    assert S.npl_call(lib, "npl_layer_norm", _t(h, x2), p2, h.t(y2), None) == 0
    return dict(x=x, y=y, x2=x2, gamma2=g, beta2=b, y2=y2)


def pooling(lib, rng):
    h = S.HostTensors(lib)
    x = rng.normal(0, 1, (2, 2, 9, 9)).astype(np.float32)
    ymax = np.zeros((2, 2, 5, 5), np.float32)
    p = nb.NplPoolingParams(3, 3, 2, 2, 1, 1, nb.NPL_POOL_MAX, 0)
    assert S.npl_call(lib, "npl_pooling", _t(h, x), p, h.t(ymax), None) == 0
    yavg = np.zeros((2, 2, 5, 5), np.float32)
    p = nb.NplPoolingParams(3, 3, 2, 2, 1, 1, nb.NPL_POOL_AVG, 0)
    assert S.npl_call(lib, "npl_pooling", _t(h, x), p, h.t(yavg), None) == 0
    yavg_pad = np.zeros((2, 2, 5, 5), np.float32)
    p = nb.NplPoolingParams(3, 3, 2, 2, 1, 1, nb.NPL_POOL_AVG, 1)
    assert S.npl_call(lib, "npl_pooling", _t(h, x), p, h.t(yavg_pad), None) == 0
    xg = rng.normal(0, 1, (2, 3, 7, 7)).astype(np.float32)
    yg = np.zeros((2, 3), np.float32)
    assert S.npl_call(lib, "npl_global_avg_pool", _t(h, xg), h.t(yg), None) == 0
    return dict(x=x, ymax=ymax, yavg=yavg, yavg_pad=yavg_pad, xg=xg, yg=yg)


def elementwise(lib, rng):
    h = S.HostTensors(lib)
    a = np.arange(1024, dtype=np.float32)
    b = np.full(1024, 2.0, np.float32)
    add = np.zeros_like(a)
    mul = np.zeros_like(a)
    assert S.npl_call(lib, "npl_add", _t(h, a), _t(h, b), h.t(add), None) == 0
    assert S.npl_call(lib, "npl_mul", _t(h, a), _t(h, b), h.t(mul), None) == 0
    x4 = rng.normal(0, 1, (2, 3, 4, 5)).astype(np.float32)
    s4 = rng.normal(0, 1, (1, 3, 1, 1)).astype(np.float32)
    mulc = np.zeros_like(x4)
    assert S.npl_call(lib, "npl_mul", _t(h, x4), _t(h, s4), h.t(mulc), None) == 0
    return dict(a=a, b=b, add=add, mul=mul, x4=x4, s4=s4, mulc=mulc)


CASES = [matmul, conv2d_winograd, conv2d_direct, conv_bn_relu, depthwise, batch_norm,
         activations, softmax, layer_norm, pooling, elementwise]


def main():
    lib = _ref()
    for i, fn in enumerate(CASES):
        data = fn(lib, np.random.default_rng(1000 + i))
        np.savez_compressed(HERE / f"{fn.__name__}.npz", **data)
        print("wrote", fn.__name__)


if __name__ == "__main__":
    main()
