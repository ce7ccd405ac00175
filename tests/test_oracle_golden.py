"""Pins the C oracle (oracle/npl_oracle.c) to the reference: every golden
fixture in tests/golden/ was produced by the reference's own NPL code
(tests/golden/make_golden.py) and must be reproduced by the oracle, including
the reference test-suite's known answers (npl_test.cpp:104-555)."""
import numpy as np
import pytest

import support as S


def load(name):
    return dict(np.load(S.GOLDEN / f"{name}.npz"))


def test_matmul_golden():
    g = load("matmul")
    c = S.o_sgemm(g["a"], g["b"], float(g["alpha"]), float(g["beta"]), g["c0"])
    assert S.normwise_err(c, g["c"]) < 1e-6
    ones = np.ones((32, 32), np.float32)
    assert np.all(S.o_sgemm(ones, ones) == 32.0)
    assert np.all(g["ones_c"] == 32.0)  # npl_test.cpp:104-149


@pytest.mark.parametrize("name", ["conv2d_winograd", "conv2d_direct"])
def test_conv2d_golden(name):
    g = load(name)
    y = S.o_conv2d(g["x"], g["w"], tuple(g["stride"]), tuple(g["pad"]), tuple(g["dil"]),
                   g["bias"])
    # The reference runs Winograd for 3x3/s1, whose transforms round
    # differently from the direct sum: relative agreement ~1e-7.
    assert y.shape == g["y"].shape
    assert S.normwise_err(y, g["y"]) < 2e-6


def test_conv2d_known_answer():
    # npl_test.cpp:206-274: ones input/weights, bias 0.5, VALID -> 27.5
    x = np.ones((1, 3, 8, 8), np.float32)
    w = np.ones((2, 3, 3, 3), np.float32)
    b = np.full(2, 0.5, np.float32)
    y = S.o_conv2d(x, w, bias=b)
    assert y.shape == (1, 2, 6, 6) and np.all(y == 27.5)


def test_conv_bn_relu_golden():
    g = load("conv_bn_relu")
    conv = S.o_conv2d(g["x"], g["w"], pad=(1, 1))
    assert S.normwise_err(conv, g["conv_only"]) < 1e-6
    bn = S.o_batch_norm(conv, g["mean"], g["var"], g["gamma"], g["beta"], 1e-5)
    y = S.o_activation(bn, 1)
    assert S.normwise_err(y, g["y"]) < 1e-6


def test_depthwise_golden():
    g = load("depthwise")
    y = S.o_depthwise(g["x"], g["w"], pad=(1, 1), bias=g["bias"])
    assert np.array_equal(y, g["y"])


def test_batch_norm_golden():
    g = load("batch_norm")
    y = S.o_batch_norm(g["x"], g["mean"], g["var"], g["gamma"], g["beta"], 1e-5)
    assert S.normwise_err(y, g["y"]) < 1e-6
    rm, rv = g["mean"].copy(), g["var"].copy()
    yt = S.o_batch_norm_train(g["x"], rm, rv, g["gamma"], g["beta"], 1e-5, 0.1)
    assert S.normwise_err(yt, g["y_train"]) < 1e-6
    assert S.normwise_err(rm, g["run_mean"]) < 1e-6
    assert S.normwise_err(rv, g["run_var"]) < 1e-6


ACTS = {"relu": 1, "relu6": 2, "tanh": 3, "sigmoid": 4, "gelu": 5, "swish": 6, "leaky": 7,
        "elu": 8, "selu": 9, "softplus": 10}


@pytest.mark.parametrize("name", sorted(ACTS))
def test_activation_golden(name):
    g = load("activations")
    y = S.o_activation(g["x"], ACTS[name], 0.01)
    if name in ("relu", "relu6", "leaky"):
        assert np.array_equal(y.view(np.uint32), g[name].view(np.uint32))  # incl. -0.0
    else:
        assert S.normwise_err(y, g[name]) < 1e-6


def test_leaky_relu_alpha_golden():
    g = load("activations")
    assert np.array_equal(S.o_activation(g["x"], 7, 0.2), g["leaky_0p2"])


def test_softmax_golden():
    g = load("softmax")
    assert S.normwise_err(S.o_softmax(g["x2"], 1), g["y2"]) < 1e-6
    assert np.allclose(g["y2"].sum(axis=1), 1.0, atol=1e-3)  # npl_test.cpp:339-377
    assert S.normwise_err(S.o_softmax(g["x3"], -2), g["y3"]) < 1e-6


def test_layer_norm_golden():
    g = load("layer_norm")
    assert S.normwise_err(S.o_layer_norm(g["x"], 128), g["y"]) < 1e-6
    assert S.normwise_err(S.o_layer_norm(g["x2"], 7, g["gamma2"], g["beta2"]), g["y2"]) < 1e-6


def test_pooling_golden():
    g = load("pooling")
    assert np.array_equal(S.o_pool(g["x"], (3, 3), (2, 2), (1, 1), 0), g["ymax"])
    assert S.normwise_err(S.o_pool(g["x"], (3, 3), (2, 2), (1, 1), 1, 0), g["yavg"]) < 1e-6
    assert S.normwise_err(S.o_pool(g["x"], (3, 3), (2, 2), (1, 1), 1, 1), g["yavg_pad"]) < 1e-6
    assert np.array_equal(S.o_gap(g["xg"]), g["yg"])


def test_gap_known_answer():
    x = np.ones((2, 64, 7, 7), np.float32)  # npl_test.cpp:520-555
    assert np.all(S.o_gap(x) == 1.0)


def test_elementwise_golden():
    g = load("elementwise")
    assert np.array_equal(g["a"] + g["b"], g["add"])
    assert np.array_equal(g["a"] * g["b"], g["mul"])
    assert np.array_equal(g["x4"] * g["s4"], g["mulc"])
