"""Host logic of PeerBuffers (npl_b200.dist) on CPU ranks (gloo, world size
3): the handle exchange, the order of the mapped pointers, close() unmapping
every peer it mapped, and a failed nplk_ipc_open_handle unmapping the peers
already opened before it raises. The library's IPC entry points are replaced
by a fake whose handles name the exporting rank, so no GPU is involved."""
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
