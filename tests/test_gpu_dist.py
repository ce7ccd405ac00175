"""Multi-GPU building blocks on one device: the column-shard relayout kernel
and the column-sharded GEMM, whose per-rank blocks are computed here one after
another and joined exactly as the all-gather delivers them."""
import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("g,rows,cps", [(2, 5, 8), (3, 17, 7), (8, 64, 256), (4, 1, 1)])
def test_colshard_relayout(g, rows, cps):
    import torch
    from npl_b200 import dist as nd
    S.gpu_lib()
    src = torch.arange(g * rows * cps, dtype=torch.float32, device="cuda")
    out = nd.cuda_relayout(src, g, rows, cps).cpu().numpy()
    ref = src.cpu().numpy().reshape(g, rows, cps).transpose(1, 0, 2).reshape(rows, g * cps)
    assert np.array_equal(out, ref)


def test_column_sharded_gemm_simulated_4_ranks():
    import torch
    from npl_b200 import dist as nd
    S.gpu_lib()
    gen = torch.Generator(device="cuda").manual_seed(0)
    M, K, N, g = 512, 384, 1024, 4
    A = torch.randn(M, K, device="cuda", generator=gen)
    B = torch.randn(K, N, device="cuda", generator=gen) / 20.0
    bias = torch.randn(N, device="cuda", generator=gen) * 0.02
    blocks = [nd.column_sharded_gemm(A, B, bias, world=g, rank=r, gather=False)
              for r in range(g)]
    gathered = torch.cat([b.reshape(-1) for b in blocks])  # all-gather order
    full = nd.cuda_relayout(gathered, g, M, N // g)
    torch.cuda.synchronize()
    ref = A.double().cpu().numpy() @ B.double().cpu().numpy() + bias.double().cpu().numpy()
    assert S.normwise_err(full.cpu().numpy(), ref) < 1e-4
    one = nd.column_sharded_gemm(A, B, bias, world=1, rank=0)
    assert S.normwise_err(one.cpu().numpy(), full.cpu().numpy()) < 1e-6


def _allgather_simulated(lib, g, M, K, w, act, form):
    import torch
    gen = torch.Generator(device="cuda").manual_seed(g * M + w)
    N = g * w
    A = torch.randn(M, K, device="cuda", generator=gen)
    B = torch.randn(K, N, device="cuda", generator=gen) / 10.0
    bias = torch.randn(N, device="cuda", generator=gen) * 0.1
    Cs = [torch.full((M, N), float("nan"), device="cuda") for _ in range(g)]
    dst = (C.c_void_p * g)(*[c.data_ptr() for c in Cs])
    raw = form == "raw"
    flags = {"raw": nb.NPLK_GEMM_RAW_OPERANDS, "sm": 0, "tma": nb.NPLK_GEMM_PEER_TMA_STORES}[form]
    ws = 0 if raw else lib.nplk_gemm_workspace_size(M, w, K)
    work = torch.empty(ws // 4 + 64, device="cuda") if ws else None
    for r in range(g):
        rc = lib.nplk_gemm_allgather(
            S.cuda_stream(), M, w, K, 1.0, S.dptr(A), K, C.c_void_p(B.data_ptr() + 4 * r * w), N,
            C.c_void_p(bias.data_ptr() + 4 * r * w), act, 0.0, dst, g, r * w, N, flags,
            S.dptr(work) if work is not None else None, ws, None)
        assert rc == 0, rc
    torch.cuda.synchronize()
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    return A, B, bias, [c.cpu().numpy() for c in Cs]


# "sm": the default exchange, 16-byte stores from the epilogue threads; "tma":
# NPLK_GEMM_PEER_TMA_STORES, through the TMA unit (w a multiple of 4; w = 50
# takes the thread stores either way).
@pytest.mark.parametrize("g,M,K,w,act,form", [(4, 300, 200, 96, 0, "raw"), (3, 129, 64, 50, 1, "tma"),
                                              (2, 64, 4096, 256, 0, "tma"),
                                              (2, 64, 4096, 256, 0, "sm"),
                                              (3, 300, 160, 100, 1, "tma"),
                                              (3, 300, 160, 100, 1, "sm"),
                                              (2, 70, 96, 36, 0, "tma"),
                                              (8, 257, 128, 64, 0, "tma"),
                                              (8, 257, 128, 64, 0, "sm")])
def test_gemm_allgather_fused_epilogue_simulated(g, M, K, w, act, form):
    # The fused GEMM + all-gather on one device: g buffers stand for the g
    # ranks' C; each "rank" computes its column block and its epilogue stores
    # the block into all g buffers, which must all end up holding the whole
    # C = act(A @ B + bias), bit for bit alike (ragged rows and column blocks
    # included: the TMA unit clips its boxes at the block's edges).
    lib = S.gpu_lib()
    A, B, bias, Cs = _allgather_simulated(lib, g, M, K, w, act, form)
    ref = A.double().cpu().numpy() @ B.double().cpu().numpy() + bias.double().cpu().numpy()
    if act:
        ref = np.maximum(ref, 0.0)
    first = Cs[0]
    assert not np.isnan(first).any()
    assert S.normwise_err(first, ref) < 1e-4
    for c in Cs[1:]:
        assert np.array_equal(c, first)


def test_gemm_allgather_tma_and_thread_stores_agree():
    lib = S.gpu_lib()
    _, _, _, tma = _allgather_simulated(lib, 4, 300, 256, 128, 1, "tma")
    _, _, _, sm = _allgather_simulated(lib, 4, 300, 256, 128, 1, "sm")
    assert np.array_equal(tma[0], sm[0]) and np.array_equal(tma[3], sm[3])


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ipc_rank(rank, world, port, results):
    import os
    import torch
    import torch.distributed as dist
    from npl_b200 import dist as nd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank % torch.cuda.device_count())
        gen = torch.Generator(device="cuda").manual_seed(0)  # the same A, B on every rank
        M, K, N = 256, 192, world * 128
        A = torch.randn(M, K, device="cuda", generator=gen)
        B = torch.randn(K, N, device="cuda", generator=gen) / 10.0
        bias = torch.randn(N, device="cuda", generator=gen) * 0.1
        full = torch.full((M, N), float("nan"), device="cuda")
        peers = nd.PeerBuffers(full, world, rank)
        nd.column_sharded_gemm_fused(A, B, peers, bias)
        torch.cuda.synchronize()
        dist.barrier()  # every rank's blocks have landed in every C
        ref = A.double().cpu().numpy() @ B.double().cpu().numpy() + bias.double().cpu().numpy()
        got = full.cpu().numpy()
        results[rank] = (float(np.isnan(got).sum()), S.normwise_err(got, ref))
        peers.close()
    finally:
        dist.destroy_process_group()


def test_gemm_allgather_ipc_two_processes():
    # Two ranks (their own GPUs when there are two, else both on one): CUDA IPC
    # handles exchanged over gloo, each rank's GEMM epilogue writing into both
    # ranks' C.
    import torch.multiprocessing as mp
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_ipc_rank, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn", join=True)
    assert sorted(results.keys()) == [0, 1]
    for nan_count, err in results.values():
        assert nan_count == 0 and err < 1e-4


def _multicast_rank(rank, world, port, results):
    import os
    import torch
    import torch.distributed as dist
    from npl_b200 import dist as nd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        gen = torch.Generator(device="cuda").manual_seed(0)  # the same A, B on every rank
        M, K, N = 384, 200, world * 136
        A = torch.randn(M, K, device="cuda", generator=gen)
        B = torch.randn(K, N, device="cuda", generator=gen) / 10.0
        bias = torch.randn(N, device="cuda", generator=gen) * 0.1
        full = torch.full((M, N), float("nan"), device="cuda")
        peers = nd.PeerBuffers(full, world, rank)
        nd.column_sharded_gemm_fused(A, B, peers, bias, act=1)
        torch.cuda.synchronize()
        dist.barrier()
        peers.close()
        mc = nd.MulticastBuffers((M, N), world, rank)
        got = []
        try:  # every rank releases the mapping together, also on an error
            mc.tensor.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            for _ in range(2):  # two calls in a row, same result
                nd.column_sharded_gemm_fused(A, B, mc, bias, act=1, barrier_before=True)
                torch.cuda.synchronize()
                dist.barrier()  # every rank's multicast stores have landed in every C
                got.append(mc.tensor.cpu().numpy())
        finally:
            mc.close()
        ref = np.maximum(A.double().cpu().numpy() @ B.double().cpu().numpy()
                         + bias.double().cpu().numpy(), 0.0)
        ipc = full.cpu().numpy()
        results[rank] = (float(np.isnan(got[1]).sum()), S.normwise_err(got[1], ref),
                         bool(np.array_equal(got[0], ipc) and np.array_equal(got[1], ipc)))
    finally:
        dist.destroy_process_group()


def test_gemm_allgather_multicast_two_gpus():
    # Two ranks on two GPUs: every rank's C bound to one NVLink multicast
    # object; each rank's GEMM epilogue stores its block once (multimem.st)
    # and both ranks end with the whole C, bit-identical to the peer-store
    # form. Needs two GPUs with NVLink multicast.
    import torch
    import torch.multiprocessing as mp
    from torch._C._autograd import DeviceType
    from torch._C._distributed_c10d import _SymmetricMemory
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if not all(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, d) for d in (0, 1)):
        pytest.skip("no NVLink multicast on these GPUs")
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_multicast_rank, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn", join=True)
    assert sorted(results.keys()) == [0, 1]
    for nan_count, err, same_as_ipc in results.values():
        assert nan_count == 0 and err < 1e-4 and same_as_ipc

