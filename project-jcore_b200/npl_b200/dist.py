"""Multi-GPU plumbing for the NPL backend (one process per GPU, torch.distributed).

Two partitionings, following the reference's workloads:
  * convolutions shard by batch: every rank runs npl_conv2d_bn_activation on its
    own images; there is no data exchange (``batch_shard``);
  * the large GEMM shards B and C by column blocks: rank r computes
    C[:, r*N/g:(r+1)*N/g] = A @ B[:, r*N/g:(r+1)*N/g] (+ bias) with A replicated.
    Fused form (``PeerBuffers`` + ``column_sharded_gemm_fused``): every rank
    holds a full row-major C whose address the others map (CUDA IPC), and the
    GEMM's epilogue stores each output tile into all ranks' C over NVLink
    (nplk_gemm_allgather) -- no separate collective, no relayout; with
    ``MulticastBuffers`` instead, every C is bound to one NVLink multicast
    object and the epilogue stores each tile once for all ranks. Unfused form
    (``column_sharded_gemm``): the blocks are all-gathered ([g][M][N/g], one
    NCCL collective) and rewritten to row-major [M][N] by the relayout kernel.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's block when n items are split into `world`
    contiguous blocks (the first n % world blocks get one extra item)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def batch_shard(n_images: int, world: int, rank: int) -> tuple[int, int]:
    """Images of this rank for the batch-sharded convolution."""
    return shard_range(n_images, world, rank)


def column_block(n_cols: int, world: int, rank: int) -> tuple[int, int]:
    """Columns of C (and B) owned by this rank. The all-gather needs equal
    blocks, so n_cols must be divisible by the number of ranks."""
    if n_cols % world:
        raise ValueError(f"{n_cols} columns do not split evenly over {world} ranks")
    w = n_cols // world
    return rank * w, (rank + 1) * w


def gather_column_blocks(local, world: int, group=None,
                         relayout: Callable | None = None):
    """All-gathers every rank's [M][N/g] block and returns row-major [M][N].

    `relayout(src_flat, g, M, cols_per_shard)` turns the gathered
    [g][M][N/g] buffer into [M][N]; on CUDA tensors the default is the library's
    nplk_colshard_relayout kernel."""
    import torch
    import torch.distributed as dist

    m, w = local.shape
    local = local.contiguous()
    gathered = torch.empty(world * m * w, dtype=local.dtype, device=local.device)
    if world == 1:
        gathered.copy_(local.reshape(-1))
    elif local.is_cuda:
        dist.all_gather_into_tensor(gathered, local.reshape(-1), group=group)
    else:
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local, group=group)
        gathered = torch.cat([p.reshape(-1) for p in parts])
    if relayout is None:
        relayout = cuda_relayout
    return relayout(gathered, world, m, w)


def cuda_relayout(src_flat, g: int, rows: int, cols_per_shard: int):
    """[g][rows][cols] -> [rows][g*cols] with nplk_colshard_relayout."""
    import torch
    from . import load

    if not src_flat.is_cuda:
        raise RuntimeError("the relayout kernel needs CUDA tensors")
    lib = load()
    out = torch.empty(rows, g * cols_per_shard, dtype=src_flat.dtype, device=src_flat.device)
    stream = C.c_void_p(torch.cuda.current_stream(src_flat.device).cuda_stream)
    rc = lib.nplk_colshard_relayout(stream, g, rows, cols_per_shard,
                                    C.c_void_p(src_flat.data_ptr()), C.c_void_p(out.data_ptr()))
    if rc != 0:
        raise RuntimeError(f"nplk_colshard_relayout failed: {rc}")
    return out


def column_sharded_gemm(A, B, bias=None, world: int = 1, rank: int = 0, group=None,
                        workspace=None, gather: bool = True):
    """C = A @ B + bias with B/C column-sharded over the ranks (CUDA tensors).

    Returns the full row-major C when `gather` is set, else this rank's block.
    The local block is computed by the tcgen05 3xTF32 GEMM (nplk_gemm) reading
    B's column block in place (ldb = N)."""
    import torch
    from . import load

    lib = load()
    M, K = A.shape
    N = B.shape[1]
    c0, c1 = column_block(N, world, rank)
    w = c1 - c0
    local = torch.empty(M, w, dtype=torch.float32, device=A.device)
    ws = lib.nplk_gemm_workspace_size(M, w, K)
    if workspace is None or workspace.numel() * 4 < ws:
        workspace = torch.empty(ws // 4 + 64, dtype=torch.float32, device=A.device)
    stream = C.c_void_p(torch.cuda.current_stream(A.device).cuda_stream)
    b_ptr = B.data_ptr() + c0 * B.element_size()
    bias_ptr = C.c_void_p(bias.data_ptr() + c0 * bias.element_size()) if bias is not None else None
    rc = lib.nplk_gemm(stream, M, w, K, 1.0, C.c_void_p(A.data_ptr()), K, C.c_void_p(b_ptr), N,
                       0.0, C.c_void_p(local.data_ptr()), w, bias_ptr, 0, 0.0, 0,
                       C.c_void_p(workspace.data_ptr()), ws, None)
    if rc != 0:
        raise RuntimeError(f"nplk_gemm failed: {rc}")
    if not gather:
        return local
    return gather_column_blocks(local, world, group)


class PeerBuffers:
    """Every rank's copy of one device tensor, mapped into every rank.

    Collective: all ranks construct it together with same-shaped tensors. Each
    rank exports a CUDA IPC handle of its tensor (nplk_ipc_get_handle), the
    handles are all-gathered over the process group, and each rank opens the
    others' (nplk_ipc_open_handle). ``ptrs[r]`` is rank r's tensor as seen
    from this rank (this rank's own entry is the tensor itself). close() --
    also collective -- unmaps them; the tensors must outlive it."""

    def __init__(self, tensor, world: int, rank: int, group=None):
        import torch
        import torch.distributed as dist
        from . import load

        self.lib = load()
        self.tensor = tensor
        self.world, self.rank, self.group = world, rank, group
        size = int(self.lib.nplk_ipc_handle_size())
        handle = (C.c_uint8 * size)()
        offset = C.c_uint64(0)
        rc = self.lib.nplk_ipc_get_handle(C.c_void_p(tensor.data_ptr()), handle, C.byref(offset))
        if rc != 0:
            raise RuntimeError(f"nplk_ipc_get_handle failed: {rc}")
        mine = (bytes(handle), int(offset.value))
        allh = [None] * world
        dist.all_gather_object(allh, mine, group=group)
        self.ptrs, self._opened = [], []
        for r, (h, off) in enumerate(allh):
            if r == rank:
                self.ptrs.append(tensor.data_ptr())
                continue
            hb = (C.c_uint8 * size).from_buffer_copy(h)
            p = C.c_void_p()
            rc = self.lib.nplk_ipc_open_handle(hb, off, C.byref(p))
            if rc != 0:
                for q, qoff in self._opened:  # do not leak the mappings made so far
                    self.lib.nplk_ipc_close_handle(C.c_void_p(q), qoff)
                self._opened = []
                raise RuntimeError(f"nplk_ipc_open_handle(rank {r}) failed: {rc}")
            self.ptrs.append(p.value)
            self._opened.append((p.value, off))
        torch.cuda.synchronize(tensor.device)

    def close(self):
        import torch.distributed as dist

        dist.barrier(group=self.group)  # no rank still writes into a peer
        for p, off in self._opened:
            self.lib.nplk_ipc_close_handle(C.c_void_p(p), off)
        self._opened = []
        dist.barrier(group=self.group)


class MulticastBuffers:
    """Every rank's C bound to one NVLink multicast object.

    Collective: all ranks construct it together with the same shape. Each
    rank's C is allocated in symmetric memory (torch.distributed's
    symmetric-memory allocator, outside its pool, so that every C starts its
    own allocation) and the allocations are bound to one multicast object at
    the rendezvous. ``ptrs == [mc_ptr]``: this rank's C as seen through the
    multicast mapping, where one store reaches the same element of every
    rank's C (NVSwitch fan-out); ``tensor`` is this rank's C for reading.
    Raises RuntimeError, on every rank, when a GPU or the fabric offers no
    multicast. close() -- also collective -- releases the mapping after every
    rank is done with it; no rank may exit or fail while another rank's
    kernel still stores through it."""

    store_flags = 16  # NPLK_GEMM_MULTIMEM_STORES

    def __init__(self, shape, world: int, rank: int, group=None, device=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from torch._C._autograd import DeviceType
        from torch._C._distributed_c10d import _SymmetricMemory
        from . import load

        self.lib = load()
        self.world, self.rank, self.group = world, rank, group
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        ok = bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, dev.index))
        self._all_or_raise(ok, "NVLink multicast is not supported on this GPU or fabric")
        size = tuple(int(d) for d in shape)
        stride = torch._prims_common.make_contiguous_strides_for(size)
        self.tensor = _SymmetricMemory.empty_strided_p2p(size, stride, torch.float32, dev)
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm_mem.rendezvous(self.tensor, grp)
        mc = int(self.handle.multicast_ptr or 0)
        # The multicast address is that of the allocation; C starts it.
        good = mc != 0 and int(self.handle.offset) == 0 and mc % 16 == 0
        try:
            self._all_or_raise(good, "no multicast mapping of C after the rendezvous")
        except RuntimeError:
            self.handle = None
            self.tensor = None
            raise
        self.mc_ptr = mc
        self.ptrs = [mc]
        torch.cuda.synchronize(dev)

    def _all_or_raise(self, ok: bool, why: str):
        import torch.distributed as dist

        flags = [None] * self.world
        dist.all_gather_object(flags, bool(ok), group=self.group)
        if not all(flags):
            raise RuntimeError(f"MulticastBuffers: {why} (ranks: {flags})")

    def close(self):
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank still stores through the mapping
        self.handle = None
        self.tensor = None
        torch.cuda.synchronize()
        dist.barrier(group=self.group)


def column_sharded_gemm_fused(A, B, peers, bias=None, workspace=None,
                              act: int = 0, barrier_before: bool = False, flags: int = 0):
    """C = act(A @ B + bias) with B column-sharded, written by every rank
    straight into every rank's C (``peers.tensor``, row-major [M][N]) by the
    GEMM epilogue (nplk_gemm_allgather). ``peers`` is a PeerBuffers (the
    epilogue stores each tile into every rank's C over NVLink) or a
    MulticastBuffers (it stores each tile once through the multicast mapping
    and NVSwitch delivers it to every rank). Asynchronous on the current
    stream.

    Two orderings are the caller's to keep, because peers store straight into
    this rank's C:
      * after: C is complete on all ranks once every rank's stream has passed
        this call (synchronise, then barrier);
      * before: every rank must be done reading or writing its C from the
        previous call before ANY rank issues the next one, or a fast rank's
        stores overwrite a result a slower peer is still reading. Either
        barrier before each call (``barrier_before=True`` synchronises this
        rank's device and then barriers the process group), or order the
        calls by a barrier the caller already has (one per iteration after
        the completion barrier above suffices).
    ``flags`` go to nplk_gemm_allgather (NPLK_GEMM_PEER_TMA_STORES: the TMA
    unit stores into the peers instead of the epilogue threads)."""
    import torch
    import torch.distributed as dist

    if barrier_before:
        torch.cuda.synchronize(A.device)
        dist.barrier(group=peers.group)

    lib = peers.lib
    M, K = A.shape
    N = B.shape[1]
    c0, c1 = column_block(N, peers.world, peers.rank)
    w = c1 - c0
    ws = lib.nplk_gemm_workspace_size(M, w, K)
    if workspace is None or workspace.numel() * 4 < ws:
        workspace = torch.empty(ws // 4 + 64, dtype=torch.float32, device=A.device)
    stream = C.c_void_p(torch.cuda.current_stream(A.device).cuda_stream)
    dst = (C.c_void_p * len(peers.ptrs))(*peers.ptrs)
    flags |= getattr(peers, "store_flags", 0)
    b_ptr = B.data_ptr() + c0 * B.element_size()
    bias_ptr = C.c_void_p(bias.data_ptr() + c0 * bias.element_size()) if bias is not None else None
    rc = lib.nplk_gemm_allgather(stream, M, w, K, 1.0, C.c_void_p(A.data_ptr()), K,
                                 C.c_void_p(b_ptr), N, bias_ptr, act, 0.0, dst, len(peers.ptrs), c0,
                                 N, flags, C.c_void_p(workspace.data_ptr()), ws, None)
    if rc != 0:
        raise RuntimeError(f"nplk_gemm_allgather failed: {rc}")
    return peers.tensor
