"""nplk_depthwise_bn_act_gap: the bandwidth chain's depthwise conv, inference
batch norm, activation and global average pool in one pass, checked bit for
bit against the four separate kernels (nplk_depthwise_conv2d ->
nplk_batch_norm_infer -> nplk_activation -> nplk_global_avg_pool), which the
rest of the suite pins to the reference (npl_convolution.cpp:60-90,
npl_activation_norm.cpp:118-153 and :51-54, npl_pooling.cpp:63-87), and the
composed chain with its softmax against the reference's own chain."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb
from npl_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _separate(lib, g, x, w, bias, mean, var, gamma, beta, eps, act, alpha):
    import torch
    n, c = x.shape[0], x.shape[1]
    ho, wo = g.h_out, g.w_out
    dw = torch.empty(n, c, ho, wo, device="cuda")
    bn = torch.empty_like(dw)
    gap = torch.empty(n * c, device="cuda")
    st = S.cuda_stream()
    p = lambda t: S.dptr(t) if t is not None else None  # noqa: E731
    assert lib.nplk_depthwise_conv2d(st, C.byref(g), p(x), p(w), p(bias), p(dw)) == 0
    assert lib.nplk_batch_norm_infer(st, n, c, ho * wo, p(dw), p(bn), p(mean), p(var), p(gamma),
                                     p(beta), eps) == 0
    assert lib.nplk_activation(st, bn.numel(), p(bn), p(bn), act, alpha, 0) == 0
    assert lib.nplk_global_avg_pool(st, n * c, ho * wo, p(bn), p(gap)) == 0
    return bn, gap


def _fused(lib, g, x, w, bias, mean, var, gamma, beta, eps, act, alpha, with_map=True):
    import torch
    n, c = x.shape[0], x.shape[1]
    y = torch.full((n, c, g.h_out, g.w_out), float("nan"), device="cuda") if with_map else None
    gap = torch.full((n * c,), float("nan"), device="cuda")
    p = lambda t: S.dptr(t) if t is not None else None  # noqa: E731
    rc = lib.nplk_depthwise_bn_act_gap(S.cuda_stream(), C.byref(g), p(x), p(w), p(bias), p(mean),
                                       p(var), p(gamma), p(beta), eps, act, alpha, p(y), p(gap))
    return rc, y, gap


def _inputs(n, c, h, wd, k, bias, affine, seed):
    import torch
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(n, c, h, wd, device="cuda", generator=gen)
    w = torch.randn(c, 1, k, k, device="cuda", generator=gen) * 0.3
    b = torch.randn(c, device="cuda", generator=gen) * 0.1 if bias else None
    mean = torch.randn(c, device="cuda", generator=gen) * 0.1
    var = torch.rand(c, device="cuda", generator=gen) + 0.5
    gamma = torch.rand(c, device="cuda", generator=gen) + 0.5 if affine else None
    beta = (torch.rand(c, device="cuda", generator=gen) - 0.5) * 0.2 if affine else None
    return x, w, b, mean, var, gamma, beta


# (n, c, h, w, k, stride, pad, bias, affine, act, alpha): the benchmark's
# 14x14 3x3 layer, stride 2, no padding, a 5x5 filter, a bias, no affine
# parameters, other activations, and plane sizes that take each kernel form.
CASES = [
    (8, 64, 14, 14, 3, 1, 1, False, True, 1, 0.0),
    (4, 32, 16, 16, 3, 2, 1, True, True, 1, 0.0),
    (4, 32, 14, 14, 3, 1, 0, False, False, 0, 0.0),
    (3, 16, 8, 8, 5, 1, 2, True, True, 7, 0.1),
    (2, 24, 20, 20, 3, 1, 1, False, True, 5, 0.0),
    (2, 8, 32, 32, 3, 2, 1, False, True, 4, 0.0),
    (2, 8, 12, 12, 3, 1, 1, True, False, 6, 0.0),
    (2, 16, 14, 14, 3, 1, 1, True, True, 7, 0.1),
    (2, 16, 16, 16, 3, 1, 1, False, True, 1, 0.0),
]


@pytest.mark.parametrize("n,c,h,wd,k,stride,pad,bias,affine,act,alpha", CASES)
def test_fused_chain_equals_separate_kernels(n, c, h, wd, k, stride, pad, bias, affine, act,
                                             alpha):
    import torch
    lib = S.gpu_lib()
    x, w, b, mean, var, gamma, beta = _inputs(n, c, h, wd, k, bias, affine, n * c + h + k)
    g = nb.conv_geom(n, c, h, wd, c, k, k, stride, pad)
    bn, gap = _separate(lib, g, x, w, b, mean, var, gamma, beta, 1e-5, act, alpha)
    rc, y, fgap = _fused(lib, g, x, w, b, mean, var, gamma, beta, 1e-5, act, alpha)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(y, bn)
    assert torch.equal(fgap, gap)
    # without the map
    rc, _, fgap2 = _fused(lib, g, x, w, b, mean, var, gamma, beta, 1e-5, act, alpha,
                          with_map=False)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(fgap2, gap)


@pytest.mark.parametrize("hw", [14, 16])
def test_fused_chain_non_finite_weight(hw):
    # A channel whose filter holds inf: its outputs take the per-output path
    # (padding skipped, not multiplied by zero), as in the depthwise kernel.
    import torch
    lib = S.gpu_lib()
    x, w, b, mean, var, gamma, beta = _inputs(2, 8, hw, hw, 3, False, True, 7)
    w[3, 0, 0, 0] = float("inf")
    w[5, 0, 2, 1] = float("-inf")
    g = nb.conv_geom(2, 8, hw, hw, 8, 3, 3, 1, 1)
    bn, gap = _separate(lib, g, x, w, b, mean, var, gamma, beta, 1e-5, 1, 0.0)
    rc, y, fgap = _fused(lib, g, x, w, b, mean, var, gamma, beta, 1e-5, 1, 0.0)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.allclose(y, bn, rtol=0, atol=0, equal_nan=True)
    assert torch.allclose(fgap, gap, rtol=0, atol=0, equal_nan=True)


def test_fused_chain_refuses_unsupported_planes():
    import torch
    lib = S.gpu_lib()
    x, w, b, mean, var, gamma, beta = _inputs(2, 4, 28, 28, 3, False, True, 1)
    # 28x28 output planes (784 > 512 elements per plane)
    g = nb.conv_geom(2, 4, 28, 28, 4, 3, 3, 1, 1)
    rc, _, _ = _fused(lib, g, x, w, b, mean, var, gamma, beta, 1e-5, 1, 0.0)
    assert rc == nb.NPL_ERR_UNSUPPORTED
    # input not 16-byte aligned
    xs = torch.empty(x.numel() + 1, device="cuda")[1:].view_as(x)
    xs.copy_(x)
    g = nb.conv_geom(2, 4, 28, 28, 4, 3, 3, 2, 1)
    rc, _, _ = _fused(lib, g, xs, w, b, mean, var, gamma, beta, 1e-5, 1, 0.0)
    assert rc == nb.NPL_ERR_UNSUPPORTED


def test_fused_bandwidth_chain_matches_separate_chain_and_reference():
    """The benchmark's chain on [256,512,14,14] with its value distributions:
    the fused form's average pool and softmax equal the separate calls' bit
    for bit, and the reference's chain (depthwise, BN, ReLU, GAP, softmax)
    on a block of images within the chain's tolerances."""
    import torch
    lib = S.gpu_lib()
    rng = S.rng(0)
    n, c, hw = 256, 512, 14
    x = rng.normal(0, 1, (n, c, hw, hw)).astype(np.float32)
    w = rng.normal(0, 0.3, (c, 1, 3, 3)).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, c).astype(np.float32)
    beta = rng.uniform(-0.1, 0.1, c).astype(np.float32)
    mean = rng.normal(0, 0.1, c).astype(np.float32)
    var = rng.uniform(0.5, 1.5, c).astype(np.float32)
    d = {k: torch.from_numpy(v).cuda() for k, v in dict(x=x, w=w, gamma=gamma, beta=beta,
                                                        mean=mean, var=var).items()}
    dw = torch.empty(n, c, hw, hw, device="cuda")
    act = torch.empty_like(dw)
    gap, probs = torch.empty(n, c, device="cuda"), torch.empty(n, c, device="cuda")
    assert W.bandwidth_chain(lib, S.cuda_stream(), d["x"], d["w"], d["mean"], d["var"],
                             d["gamma"], d["beta"], dw, act, gap, probs) == 0
    fgap, fprobs = torch.empty_like(gap), torch.empty_like(probs)
    assert W.bandwidth_chain_fused(lib, S.cuda_stream(), d["x"], d["w"], d["mean"], d["var"],
                                   d["gamma"], d["beta"], fgap, fprobs) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    assert torch.equal(fgap, gap)
    assert torch.equal(fprobs, probs)
    # the reference chain on 8 images (the reference build's calls, or the C
    # restatement of the same loops where that build is absent)
    from test_gpu_workloads import _reference_bandwidth_chain
    k = 8
    _, _, r_gap, r_sm = _reference_bandwidth_chain(np.ascontiguousarray(x[:k]), w, mean, var,
                                                   gamma, beta)
    got_gap = fgap[:k].cpu().numpy()
    got_sm = fprobs[:k].cpu().numpy()
    assert S.normwise_err(got_gap, r_gap.reshape(got_gap.shape)) <= 1e-6
    assert S.normwise_err(got_sm, r_sm.reshape(got_sm.shape)) <= 1e-5
