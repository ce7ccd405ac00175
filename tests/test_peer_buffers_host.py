"""Host logic of PeerBuffers (npl_b200.dist) on CPU ranks (gloo, world size
3): the handle exchange, the order of the mapped pointers, close() unmapping
every peer it mapped, and a failed nplk_ipc_open_handle unmapping the peers
already opened before it raises; and the arguments column_sharded_gemm_fused
passes to nplk_gemm_allgather on each rank. The library's entry points are
replaced by fakes (IPC handles that name the exporting rank, a GEMM that
records its call), so no GPU is involved."""
import ctypes as C
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HANDLE_BYTES = 64


def fake_addr(exporter: int, off: int) -> int:
    return 0x100000 * (exporter + 1) + off


def fake_offset(rank: int) -> int:
    return 16 * (rank + 1)


class FakeIpcLib:
    """The four nplk_ipc_* entry points: rank r's handle is HANDLE_BYTES bytes
    of r + 1 and its offset fake_offset(r); opening a handle maps it at
    fake_addr(exporter, offset), or fails with -7 for the exporter `fail_on`."""

    def __init__(self, rank: int, fail_on=None):
        self.rank, self.fail_on = rank, fail_on
        self.opened, self.closed = [], []

    def nplk_ipc_handle_size(self):
        return HANDLE_BYTES

    def nplk_ipc_get_handle(self, ptr, handle, offset_ref):
        for i in range(HANDLE_BYTES):
            handle[i] = self.rank + 1
        offset_ref._obj.value = fake_offset(self.rank)
        return 0

    def nplk_ipc_open_handle(self, handle, off, ptr_ref):
        exporter = handle[0] - 1
        assert all(handle[i] == exporter + 1 for i in range(HANDLE_BYTES))
        if exporter == self.fail_on:
            return -7
        ptr_ref._obj.value = fake_addr(exporter, off)
        self.opened.append((exporter, off))
        return 0

    def nplk_ipc_close_handle(self, ptr, off):
        self.closed.append((ptr.value, off))
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, fail_rank, fail_exporter, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import npl_b200
        from npl_b200 import dist as nd

        fake = FakeIpcLib(rank, fail_exporter if rank == fail_rank else None)
        npl_b200.load = lambda *a, **k: fake
        torch.cuda.synchronize = lambda *a, **k: None  # CPU tensors stand in for device ones
        t = torch.zeros(8)
        try:
            pb = nd.PeerBuffers(t, world, rank)
        except RuntimeError as e:
            results[rank] = ("raised", str(e), fake.opened, fake.closed)
            return
        ptrs = list(pb.ptrs)
        if fail_rank is None:
            pb.close()
        results[rank] = ("ok", ptrs, t.data_ptr(), fake.opened, fake.closed)
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank=None, fail_exporter=None):
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), fail_rank, fail_exporter, results),
                       nprocs=world, start_method="spawn", join=True)
    return dict(results)


def test_peer_buffers_exchange_and_close_gloo_world3():
    world = 3
    res = _run(world)
    assert sorted(res) == list(range(world))
    for r in range(world):
        status, ptrs, own, opened, closed = res[r]
        assert status == "ok"
        others = [q for q in range(world) if q != r]
        assert ptrs == [own if q == r else fake_addr(q, fake_offset(q)) for q in range(world)]
        assert opened == [(q, fake_offset(q)) for q in others]
        assert closed == [(fake_addr(q, fake_offset(q)), fake_offset(q)) for q in others]


def test_peer_buffers_unmaps_opened_peers_when_an_open_fails():
    # Rank 0 maps rank 1's buffer, then fails on rank 2's: it must unmap rank
    # 1's before raising; the other ranks map both peers.
    world = 3
    res = _run(world, fail_rank=0, fail_exporter=2)
    status, msg, opened, closed = res[0]
    assert status == "raised" and "rank 2" in msg and "-7" in msg
    assert opened == [(1, fake_offset(1))]
    assert closed == [(fake_addr(1, fake_offset(1)), fake_offset(1))]
    for r in (1, 2):
        status, ptrs, own, opened, closed = res[r]
        assert status == "ok" and ptrs[r] == own
        assert [q for q, _ in opened] == [q for q in range(world) if q != r]
        assert closed == []  # close() is collective; not called once a rank failed


class RecordingGemmLib:
    """nplk_gemm_workspace_size and nplk_gemm_allgather, recording the call."""

    def __init__(self):
        self.calls = []

    def nplk_gemm_workspace_size(self, m, n, k):
        return 4 * (m * k + n * k) * 2

    def nplk_gemm_allgather(self, *args):
        self.calls.append(args)
        return 0


class _Peers:
    def __init__(self, lib, tensor, world, rank, ptrs):
        self.lib, self.tensor, self.world, self.rank, self.ptrs = lib, tensor, world, rank, ptrs


def test_column_sharded_gemm_fused_arguments(monkeypatch):
    # Each rank passes its column block of B and bias, every rank's C as the
    # destinations, its column offset and the full row pitch.
    from npl_b200 import dist as nd

    class _Stream:
        cuda_stream = 0

    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: _Stream())
    M, K, N, world = 64, 48, 96, 3
    A = torch.zeros(M, K)
    B = torch.zeros(K, N)
    bias = torch.zeros(N)
    ptrs = [0x100000, 0x200000, 0x300000]
    for rank in range(world):
        lib = RecordingGemmLib()
        C_full = torch.zeros(M, N)
        out = nd.column_sharded_gemm_fused(A, B, _Peers(lib, C_full, world, rank, ptrs), bias,
                                           act=1)
        assert out is C_full and len(lib.calls) == 1
        (stream, m, w, k, alpha, a, lda, b, ldb, bias_p, act, act_alpha, dst, n_dst, col0, ldc,
         flags, work, ws, status) = lib.calls[0]
        c0, c1 = nd.column_block(N, world, rank)
        assert (m, w, k, lda, ldb, ldc, n_dst, col0) == (M, c1 - c0, K, K, N, N, world, c0)
        assert alpha == 1.0 and act == 1 and flags == 0 and status is None
        assert a.value == A.data_ptr()
        assert b.value == B.data_ptr() + 4 * c0
        assert bias_p.value == bias.data_ptr() + 4 * c0
        assert [dst[i] for i in range(world)] == ptrs
        assert ws == lib.nplk_gemm_workspace_size(M, c1 - c0, K) and work.value is not None
