"""Failure paths on the device, exercised without faulting the GPU.

Bounded waits: every mbarrier wait in the tcgen05 kernels gives up after a
limit, records a code in a status word, raises the CTA's abort flag, lets its
copies in flight land, frees TMEM and returns. nplk_debug_arm_wait_timeout
arms one launch whose MMA issuer waits on a barrier nothing arrives on, with a
short limit, so the timeout path runs for real. The tests check that the kernel
returns, that the status word holds the MMA-wait code (102), that the npl_*
layer turns it into NPL_ERR_INTERNAL, and that the next ordinary call on the
same context succeeds with correct results (TMEM was released, nothing is
left armed).

Allocation failures: nplk_debug_fail_next_allocations makes the next device
allocations of npl_* calls fail as out of memory: npl_matmul then falls back
to the raw-operand GEMM, which needs no workspace (npl_tensor_ops.cpp:145-147
is the reference's matmul entry), and a call that cannot stage its host
tensors returns NPL_ERR_OOM (neural_primitives.h:52-59)."""
import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu
STALL_US = 50_000  # 50 ms instead of the kernels' 4 s


def _gemm_dev(lib, m=256, n=192, k=96, status=None):
    import torch
    gen = torch.Generator(device="cuda").manual_seed(m + n + k)
    A = torch.rand(m, k, device="cuda", generator=gen) * 2 - 1
    B = torch.rand(k, n, device="cuda", generator=gen) * 2 - 1
    Cm = torch.zeros(m, n, device="cuda")
    ws = lib.nplk_gemm_workspace_size(m, n, k)
    work = torch.empty(ws // 4 + 64, device="cuda")
    rc = lib.nplk_gemm(S.cuda_stream(), m, n, k, 1.0, S.dptr(A), k, S.dptr(B), n, 0.0,
                       S.dptr(Cm), n, None, 0, 0.0, 0, S.dptr(work), ws,
                       S.dptr(status) if status is not None else None)
    assert rc == 0
    torch.cuda.synchronize()
    ref = A.double().cpu().numpy() @ B.double().cpu().numpy()
    return Cm.cpu().numpy(), ref


def test_gemm_wait_timeout_reports_status_and_recovers():
    lib = S.gpu_lib()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    assert lib.nplk_debug_arm_wait_timeout(nb.NPLK_DEBUG_GEMM, STALL_US) == 0
    _gemm_dev(lib)  # the armed launch: returns, output undefined
    assert lib.nplk_read_status(S.cuda_stream()) == nb.NPLK_STATUS_TIMEOUT_MMA
    # the next launch is not armed; TMEM was freed, so it runs normally
    got, ref = _gemm_dev(lib)
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    assert S.normwise_err(got, ref) < 1e-4


def test_gemm_wait_timeout_into_a_caller_status_word():
    import torch
    lib = S.gpu_lib()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.nplk_debug_arm_wait_timeout(nb.NPLK_DEBUG_GEMM, STALL_US) == 0
    _gemm_dev(lib, 384, 320, 64, status=st)
    assert int(st.item()) == nb.NPLK_STATUS_TIMEOUT_MMA
    assert lib.nplk_read_status(S.cuda_stream()) == 0  # the library's own word is untouched
    st.zero_()
    got, ref = _gemm_dev(lib, 384, 320, 64, status=st)
    assert int(st.item()) == 0
    assert S.normwise_err(got, ref) < 1e-4


def test_npl_matmul_timeout_returns_internal_error():
    lib = S.gpu_lib()
    rng = S.rng(11)
    a = rng.uniform(-1, 1, (200, 130)).astype(np.float32)
    b = rng.uniform(-1, 1, (130, 170)).astype(np.float32)
    h = S.HostTensors(lib)
    c = np.zeros((200, 170), np.float32)
    assert lib.nplk_debug_arm_wait_timeout(nb.NPLK_DEBUG_GEMM, STALL_US) == 0
    rc = S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(1.0), C.c_float(0.0),
                    None)
    assert rc == nb.NPL_ERR_INTERNAL
    rc = S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(1.0), C.c_float(0.0),
                    None)
    assert rc == nb.NPL_OK
    assert S.normwise_err(c, S.o_sgemm(a, b)) < 1e-4


def _conv_case(seed):
    rng = S.rng(seed)
    x = rng.uniform(0, 1, (4, 64, 28, 28)).astype(np.float32)
    w = rng.normal(0, np.sqrt(2 / 576), (64, 64, 3, 3)).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 64).astype(np.float32)
    beta = rng.uniform(-0.1, 0.1, 64).astype(np.float32)
    mean = rng.normal(0, 0.1, 64).astype(np.float32)
    var = rng.uniform(0.5, 1.5, 64).astype(np.float32)
    return x, w, gamma, beta, mean, var


def test_conv_window_timeout_through_npl_call_and_recovery():
    # 3x3 stride-1 layer with C_in = 64: the window-gather kernel (two MMA
    # pipelines per CTA, both stalled by the armed launch).
    lib = S.gpu_lib()
    x, w, gamma, beta, mean, var = _conv_case(12)
    h = S.HostTensors(lib)
    y = np.zeros((4, 64, 28, 28), np.float32)
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    bn = nb.NplBatchnormParams(mean.ctypes.data, var.ctypes.data, gamma.ctypes.data,
                               beta.ctypes.data, 1e-5, 0, 0.1)
    args = (h.t(x), h.t(w), None, p, bn, nb.NPL_ACT_RELU, h.t(y), None)
    assert lib.nplk_debug_arm_wait_timeout(nb.NPLK_DEBUG_CONV_WINDOW, STALL_US) == 0
    assert S.npl_call(lib, "npl_conv2d_bn_activation", *args) == nb.NPL_ERR_INTERNAL
    assert S.npl_call(lib, "npl_conv2d_bn_activation", *args) == nb.NPL_OK
    ref = S.o_activation(S.o_batch_norm(S.o_conv2d(x, w, pad=(1, 1)), mean, var, gamma, beta),
                         1)
    assert S.normwise_err(y, ref) < 1e-4


def test_allocation_failure_falls_back_or_reports_oom():
    lib = S.gpu_lib()
    rng = S.rng(13)
    m, k, n = 256, 128, 192
    # Library-allocated (managed) tensors need no staging: the only device
    # allocation is the GEMM's operand workspace, whose failure makes
    # npl_matmul read A and B in place (raw-operand form), same results.
    ts = [nb.tensor(lib, None, shape) for shape in ([m, k], [k, n], [m, n])]
    for t in ts:
        assert lib.npl_allocate_tensor(C.byref(t)) == 0
    try:
        arrs = [np.ctypeslib.as_array(C.cast(t.data, C.POINTER(C.c_float)), shape=shp)
                for t, shp in zip(ts, ([m, k], [k, n], [m, n]))]
        arrs[0][:] = rng.uniform(-1, 1, (m, k))
        arrs[1][:] = rng.uniform(-1, 1, (k, n))
        assert lib.nplk_debug_fail_next_allocations(1) == 0
        rc = lib.npl_matmul(C.byref(ts[0]), C.byref(ts[1]), C.byref(ts[2]), 1.0, 0.0, None)
        assert rc == nb.NPL_OK
        assert lib.nplk_debug_fail_next_allocations(0) == 0  # the one failure was used
        assert S.normwise_err(arrs[2], S.o_sgemm(arrs[0].copy(), arrs[1].copy())) < 1e-4
    finally:
        for t in ts:
            lib.npl_free_tensor(C.byref(t))
    # Plain host tensors are staged: a failed staging allocation is NPL_ERR_OOM,
    # and the call after it succeeds.
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = np.zeros((m, n), np.float32)
    h = S.HostTensors(lib)
    assert lib.nplk_debug_fail_next_allocations(1) == 0
    rc = S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(1.0), C.c_float(0.0),
                    None)
    assert rc == nb.NPL_ERR_OOM
    assert lib.nplk_debug_fail_next_allocations(0) == 0
    rc = S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(1.0), C.c_float(0.0),
                    None)
    assert rc == nb.NPL_OK
    assert S.normwise_err(c, S.o_sgemm(a, b)) < 1e-4
