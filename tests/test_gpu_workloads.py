"""Parity of the composed workloads exactly as the benchmark runs them on the
device (npl_b200.workloads), against the reference's own CPU code run as the
same chain on the same inputs (oracle/_ref, built from the reference sources;
the C restatement in oracle/ stands in where that build is absent), and the
reference's own test program run against this library.

* Bandwidth chain on [256,512,14,14]: depthwise 3x3 -> BN -> ReLU -> global
  average pool -> softmax, each GPU kernel fed the previous GPU kernel's
  output. Tolerances: 1e-6 normwise on the intermediates, 1e-5 on softmax.
* Large GEMM + norm: ReLU(A @ B + bias) with the bias through beta = 1 on a
  pre-filled C and ReLU in the GEMM epilogue, then layer norm over rows of
  16384, for the whole [8192x4096] @ [4096x16384] product on the device; a
  block of 512 rows is compared with the reference's npl_matmul (beta = 1) ->
  npl_relu -> npl_layer_norm on the same rows, at 1e-4.
"""
import ctypes as C
import subprocess

import numpy as np
import pytest

import support as S
from support import nb
from npl_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _ref_call(lib, name, *args):
    rc = S.npl_call(lib, name, *args)
    assert rc == 0, (name, rc)


def _reference_bandwidth_chain(x, w, mean, var, gamma, beta):
    ref = S.reference()
    if ref is None:  # the C restatement of the same loops
        dw = S.o_depthwise(x, w, pad=(1, 1))
        act = S.o_activation(S.o_batch_norm(dw, mean, var, gamma, beta), 1)
        gap = S.o_gap(act)
        return dw, act, gap, S.o_softmax(gap, 1)
    h = S.HostTensors(ref)
    dw, bn, act = np.zeros_like(x), np.zeros_like(x), np.zeros_like(x)
    n, c = x.shape[:2]
    gap, sm = np.zeros((n, c), np.float32), np.zeros((n, c), np.float32)
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    bnp = nb.NplBatchnormParams(mean.ctypes.data, var.ctypes.data, gamma.ctypes.data,
                                beta.ctypes.data, 1e-5, 0, 0.1)
    _ref_call(ref, "npl_depthwise_conv2d", h.t(x), h.t(w), None, p, h.t(dw), None)
    _ref_call(ref, "npl_batch_norm", h.t(dw), bnp, h.t(bn), None)
    _ref_call(ref, "npl_relu", h.t(bn), h.t(act), None)
    _ref_call(ref, "npl_global_avg_pool", h.t(act), h.t(gap), None)
    _ref_call(ref, "npl_softmax", h.t(gap), 1, h.t(sm), None)
    return dw, act, gap, sm


def test_bandwidth_chain_on_device_matches_reference_chain():
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
    d = {k: torch.from_numpy(v).cuda() for k, v in
         dict(x=x, w=w, gamma=gamma, beta=beta, mean=mean, var=var).items()}
    dw = torch.empty_like(d["x"])
    act = torch.empty_like(d["x"])
    gap = torch.empty(n, c, device="cuda")
    probs = torch.empty(n, c, device="cuda")
    rc = W.bandwidth_chain(lib, S.cuda_stream(), d["x"], d["w"], d["mean"], d["var"],
                           d["gamma"], d["beta"], dw, act, gap, probs)
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    r_dw, r_act, r_gap, r_sm = _reference_bandwidth_chain(x, w, mean, var, gamma, beta)
    assert S.normwise_err(dw.cpu().numpy(), r_dw) < 1e-6
    assert S.normwise_err(act.cpu().numpy(), r_act) < 1e-6
    assert S.normwise_err(gap.cpu().numpy(), r_gap) < 1e-6
    assert S.normwise_err(probs.cpu().numpy(), r_sm) < 1e-5


def _reference_gemm_relu_ln(a, b, bias):
    ref = S.reference()
    m, n = a.shape[0], b.shape[1]
    c = np.ascontiguousarray(np.broadcast_to(bias, (m, n)))
    y = np.zeros((m, n), np.float32)
    if ref is None:
        c = np.maximum(S.o_sgemm(a, b, 1.0, 1.0, c), 0).astype(np.float32)
        return c, S.o_layer_norm(c, n)
    h = S.HostTensors(ref)
    tc = h.t(c)
    _ref_call(ref, "npl_matmul", h.t(a), h.t(b), tc, C.c_float(1.0), C.c_float(1.0), None)
    _ref_call(ref, "npl_relu", tc, tc, None)
    _ref_call(ref, "npl_layer_norm", tc, nb.NplLayernormParams(None, None, 1e-5, n), h.t(y),
              None)
    return c, y


def test_gemm_bias_relu_layer_norm_on_device_matches_reference_rows():
    import torch
    lib = S.gpu_lib()
    M, K, N = 8192, 4096, 16384
    gen = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(M, K, device="cuda", generator=gen)
    B = torch.randn(K, N, device="cuda", generator=gen) / 64.0
    bias = torch.randn(N, device="cuda", generator=gen) * 0.02
    Cm = torch.empty(M, N, device="cuda")
    Y = torch.empty(M, N, device="cuda")
    ws = lib.nplk_gemm_workspace_size(M, N, K)
    work = torch.empty(ws // 4 + 64, device="cuda")
    W.fill_bias_rows(Cm, bias)
    assert W.gemm_bias_relu_layer_norm(lib, S.cuda_stream(), A, B, Cm, Y, work, ws) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    r0 = 2560  # a block of 512 rows
    a_blk = A[r0:r0 + 512].cpu().numpy()
    got_c = Cm[r0:r0 + 512].cpu().numpy()
    got_y = Y[r0:r0 + 512].cpu().numpy()
    del Cm, Y, work
    ref_c, ref_y = _reference_gemm_relu_ln(a_blk, B.cpu().numpy(), bias.cpu().numpy())
    assert S.normwise_err(got_c, ref_c) < 1e-4
    assert S.normwise_err(got_y, ref_y) < 1e-4


def test_reference_test_program_passes_on_this_library():
    # advanced/neural_layer/src/npl_test.cpp:56-803, compiled unchanged against
    # include/neural_primitives.h and linked to libnpl_b200.so (make -C oracle
    # reftest): its 11 API tests, quiet mode, exit 0 = all passed.
    exe = S.REPO / "oracle" / "_ref" / "npl_test_b200"
    if not exe.exists():
        pytest.skip("oracle/_ref/npl_test_b200 was not built (needs the reference tree)")
    res = subprocess.run([str(exe), "-q"], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-2000:]
    assert "[FAIL]" not in res.stdout
