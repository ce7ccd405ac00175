"""Parity of the tcgen05 3xTF32 GEMM behind npl_matmul / nplk_gemm with the
oracle (fp64-accumulated sgemm) and with the reference's own npl_matmul
(OpenBLAS) where its CPU build is present. Tolerance: normwise max relative
error <= 1e-4 (3xTF32); the plain-TF32 fast mode is reported separately."""
import ctypes as C
import os

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu
TOL = 1e-4


def matmul_host(lib, a, b, alpha=1.0, beta=0.0, c0=None):
    h = S.HostTensors(lib)
    c = np.zeros((a.shape[0], b.shape[1]), np.float32) if c0 is None else c0.copy()
    st = nb.NplPerfStats()
    rc = S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(alpha),
                    C.c_float(beta), st)
    assert rc == nb.NPL_OK, lib.npl_strerror(rc)
    return c, st


def test_matmul_known_answer_managed():
    # npl_test.cpp:104-149 through library-allocated (managed) tensors.
    lib = S.gpu_lib()
    ts = [nb.tensor(lib, None, [32, 32]) for _ in range(3)]
    for t in ts:
        assert lib.npl_allocate_tensor(C.byref(t)) == 0
    for t in ts[:2]:
        arr = np.ctypeslib.as_array(C.cast(t.data, C.POINTER(C.c_float)), shape=(32, 32))
        arr[:] = 1.0
    assert lib.npl_matmul(C.byref(ts[0]), C.byref(ts[1]), C.byref(ts[2]), 1.0, 0.0, None) == 0
    out = np.ctypeslib.as_array(C.cast(ts[2].data, C.POINTER(C.c_float)), shape=(32, 32))
    assert np.all(np.abs(out - 32.0) < 1e-3)
    for t in ts:
        lib.npl_free_tensor(C.byref(t))
        assert not t.data


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 5, 3), (128, 128, 32), (129, 65, 33),
                                   (256, 512, 1024), (300, 17, 513), (33, 1000, 77),
                                   (1, 4096, 300), (2048, 8, 64)])
def test_matmul_shapes(m, n, k):
    lib = S.gpu_lib()
    rng = S.rng(m * 7 + n * 3 + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c, _ = matmul_host(lib, a, b)
    err = S.normwise_err(c, S.o_sgemm(a, b))
    assert err < TOL, err


def test_matmul_alpha_beta():
    lib = S.gpu_lib()
    rng = S.rng(5)
    a = rng.uniform(-1, 1, (200, 300)).astype(np.float32)
    b = rng.uniform(-1, 1, (300, 260)).astype(np.float32)
    c0 = rng.uniform(-1, 1, (200, 260)).astype(np.float32)
    c, _ = matmul_host(lib, a, b, 0.5, 2.0, c0)
    assert S.normwise_err(c, S.o_sgemm(a, b, 0.5, 2.0, c0)) < TOL
    # beta == 0 must not read C (NaN in C stays out of the result)
    c0[:] = np.nan
    c, _ = matmul_host(lib, a, b, 1.0, 0.0, c0)
    assert np.isfinite(c).all()


def test_matmul_golden():
    g = dict(np.load(S.GOLDEN / "matmul.npz"))
    c, _ = matmul_host(S.gpu_lib(), g["a"], g["b"], float(g["alpha"]), float(g["beta"]),
                       g["c0"])
    assert S.normwise_err(c, g["c"]) < TOL


def test_matmul_1024_vs_oracle_and_reference():
    # npl_matmul fp32 1024^3, A and B uniform[-1,1] from seed 0.
    lib = S.gpu_lib()
    rng = S.rng(0)
    a = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
    b = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
    c, st = matmul_host(lib, a, b)
    o = S.o_sgemm(a, b)
    err = S.normwise_err(c, o)
    assert err < TOL, err
    assert st.gflops > 0 and b"3xTF32" in st.backend_used
    ref = S.reference()
    if ref is not None:
        r = np.zeros_like(c)
        h = S.HostTensors(ref)
        assert S.npl_call(ref, "npl_matmul", h.t(a), h.t(b), h.t(r), C.c_float(1.0),
                          C.c_float(0.0), None) == 0
        assert S.normwise_err(c, r) < TOL


def test_matmul_tf32_fast_mode_reported_separately():
    lib = S.gpu_lib()
    rng = S.rng(0)
    a = rng.uniform(-1, 1, (512, 512)).astype(np.float32)
    b = rng.uniform(-1, 1, (512, 512)).astype(np.float32)
    o = S.o_sgemm(a, b)
    os.environ["NPL_TF32_FAST"] = "1"
    try:
        c, st = matmul_host(lib, a, b)
    finally:
        del os.environ["NPL_TF32_FAST"]
    fast_err = S.normwise_err(c, o)
    c3, _ = matmul_host(lib, a, b)
    err3 = S.normwise_err(c3, o)
    print(f"TF32 fast mode normwise err {fast_err:.3e}; 3xTF32 {err3:.3e}")
    assert b"TF32" in st.backend_used
    assert err3 < TOL and fast_err < 5e-3 and err3 < fast_err


def test_matmul_batched():
    lib = S.gpu_lib()
    rng = S.rng(9)
    a = rng.uniform(-1, 1, (3, 40, 50)).astype(np.float32)
    b = rng.uniform(-1, 1, (3, 50, 60)).astype(np.float32)
    h = S.HostTensors(lib)
    c = np.zeros((3, 40, 60), np.float32)
    assert S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(1.0),
                      C.c_float(0.0), None) == 0
    for i in range(3):
        assert S.normwise_err(c[i], S.o_sgemm(a[i], b[i])) < TOL


def test_gemm_8192x4096x16384_device_sampled_rows():
    # npl_matmul fp32 [8192x4096] @ [4096x16384] with the per-column bias fed
    # through beta=1 on a pre-filled C (the large-GEMM benchmark case); parity on a
    # seeded sample of rows against an fp64 product.
    import torch
    lib = S.gpu_lib()
    M, K, N = 8192, 4096, 16384
    gen = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(M, K, device="cuda", generator=gen)
    B = torch.randn(K, N, device="cuda", generator=gen) * (1.0 / 64.0)
    bias = torch.randn(N, device="cuda", generator=gen) * 0.02
    Cm = bias.expand(M, N).contiguous()
    ws = lib.nplk_gemm_workspace_size(M, N, K)
    work = torch.empty(ws // 4 + 64, device="cuda", dtype=torch.float32)
    rc = lib.nplk_gemm(S.cuda_stream(), M, N, K, 1.0, S.dptr(A), K, S.dptr(B), N, 1.0,
                       S.dptr(Cm), N, None, 0, 0.0, 0, S.dptr(work), ws, None)
    assert rc == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    rows = torch.randint(0, M, (24,), generator=torch.Generator().manual_seed(1))
    a64 = A[rows].double().cpu().numpy()
    ref = a64 @ B.double().cpu().numpy() + bias.double().cpu().numpy()[None, :]
    got = Cm[rows].cpu().numpy()
    assert S.normwise_err(got, ref) < TOL


FORM_SHAPES = [(128, 128, 32), (256, 192, 96), (300, 260, 100), (64, 40, 8), (129, 100, 36),
               (1024, 1024, 1024), (640, 4096, 256)]


@pytest.mark.parametrize("form", ["raw", "split"])
@pytest.mark.parametrize("m,n,k", FORM_SHAPES)
def test_gemm_operand_forms(m, n, k, form):
    # Both operand forms (raw: A and B read in place, lo parts formed in shared
    # memory; split: hi/lo copies in the workspace) with alpha, beta, bias and
    # ReLU in the epilogue and padded leading dimensions, against fp64.
    import torch
    lib = S.gpu_lib()
    gen = torch.Generator(device="cuda").manual_seed(m + n + k)
    lda, ldb, ldc = k + 4, n + 8, n + 4
    A = (torch.rand(m, lda, device="cuda", generator=gen) * 2 - 1)
    B = (torch.rand(k, ldb, device="cuda", generator=gen) * 2 - 1)
    C0 = torch.rand(m, ldc, device="cuda", generator=gen) - 0.5
    bias = torch.rand(n, device="cuda", generator=gen) - 0.5
    Cm = C0.clone()
    flags = nb.NPLK_GEMM_RAW_OPERANDS if form == "raw" else nb.NPLK_GEMM_SPLIT_OPERANDS
    ws = lib.nplk_gemm_workspace_size(m, n, k) if form == "split" else 0
    work = torch.empty(ws // 4 + 64, device="cuda") if ws else None
    rc = lib.nplk_gemm(S.cuda_stream(), m, n, k, 0.75, S.dptr(A), lda, S.dptr(B), ldb, 0.5,
                       S.dptr(Cm), ldc, S.dptr(bias), nb.NPL_ACT_RELU, 0.0, flags,
                       S.dptr(work) if work is not None else None, ws, None)
    assert rc == 0, rc
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    a64 = A[:, :k].double().cpu().numpy()
    b64 = B[:, :n].double().cpu().numpy()
    ref = 0.75 * (a64 @ b64) + 0.5 * C0[:, :n].double().cpu().numpy() + \
        bias.double().cpu().numpy()[None, :]
    ref = np.maximum(ref, 0.0)
    got = Cm.cpu().numpy()
    assert S.normwise_err(got[:, :n], ref) < TOL
    assert np.array_equal(got[:, n:], C0[:, n:].cpu().numpy())  # padding untouched


@pytest.mark.parametrize("form", ["raw", "split"])
def test_gemm_infinity_and_raw_eligibility(form):
    # An infinite entry of A stays confined to its row in both operand forms
    # (its own lo part is 0, not inf - inf; the row itself holds +inf or NaN:
    # 3xTF32 forms inf * lo(B), which is NaN where lo(B) is 0). Forcing the raw
    # form on operands TMA cannot read in place (lda not a multiple of 4) is
    # refused.
    import torch
    lib = S.gpu_lib()
    m, n, k = 256, 128, 64
    gen = torch.Generator(device="cuda").manual_seed(5)
    A = torch.rand(m, k, device="cuda", generator=gen) + 0.5
    B = torch.rand(k, n, device="cuda", generator=gen) + 0.5
    A[3, 7] = float("inf")
    Cm = torch.zeros(m, n, device="cuda")
    ws = lib.nplk_gemm_workspace_size(m, n, k) if form == "split" else 0
    work = torch.empty(ws // 4 + 64, device="cuda") if ws else None
    flags = nb.NPLK_GEMM_RAW_OPERANDS if form == "raw" else nb.NPLK_GEMM_SPLIT_OPERANDS
    rc = lib.nplk_gemm(S.cuda_stream(), m, n, k, 1.0, S.dptr(A), k, S.dptr(B), n, 0.0,
                       S.dptr(Cm), n, None, 0, 0.0, flags,
                       S.dptr(work) if work is not None else None, ws, None)
    assert rc == 0
    torch.cuda.synchronize()
    got = Cm.cpu().numpy()
    assert not np.isfinite(got[3]).any() and not np.isneginf(got[3]).any()
    assert np.all(np.isfinite(np.delete(got, 3, axis=0)))
    if form == "split":
        return
    A2 = torch.rand(m, k + 1, device="cuda", generator=gen)
    rc = lib.nplk_gemm(S.cuda_stream(), m, n, k, 1.0, S.dptr(A2), k + 1, S.dptr(B), n, 0.0,
                       S.dptr(Cm), n, None, 0, 0.0, nb.NPLK_GEMM_RAW_OPERANDS, None, 0, None)
    assert rc == nb.NPL_ERR_UNSUPPORTED


@pytest.mark.parametrize("m,n,k", [(1024, 1024, 1024), (300, 260, 520), (128, 1000, 4096),
                                   (1000, 96, 2048)])
def test_gemm_split_k_plain_products(m, n, k):
    # Small products whose 128-wide tiles fill at most half the SMs run with K
    # cut in two slices added into a zeroed C (beta 0, no bias, no activation):
    # checked against fp64, deterministic from call to call, and with a
    # pre-filled C (beta 0 must not read it).
    import torch
    lib = S.gpu_lib()
    gen = torch.Generator(device="cuda").manual_seed(m + 7 * n + k)
    A = torch.rand(m, k, device="cuda", generator=gen) * 2 - 1
    B = torch.rand(k, n, device="cuda", generator=gen) * 2 - 1
    ws = lib.nplk_gemm_workspace_size(m, n, k)
    work = torch.empty(ws // 4 + 64, device="cuda")
    outs = []
    for fill in (float("nan"), 3.0):
        Cm = torch.full((m, n), fill, device="cuda")
        rc = lib.nplk_gemm(S.cuda_stream(), m, n, k, 0.5, S.dptr(A), k, S.dptr(B), n, 0.0,
                           S.dptr(Cm), n, None, 0, 0.0, 0, S.dptr(work), ws, None)
        assert rc == 0
        torch.cuda.synchronize()
        outs.append(Cm.clone())
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    assert torch.equal(outs[0], outs[1])
    ref = 0.5 * (A.double() @ B.double())
    assert ((outs[0].double() - ref).abs().max() / ref.abs().max()).item() < TOL
