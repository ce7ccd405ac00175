"""Multi-GPU plumbing for the NPL backend (one process per GPU, torch.distributed).

Two partitionings, following the reference's workloads:
  * convolutions shard by batch: every rank runs npl_conv2d_bn_activation on its
    own images; there is no data exchange (``batch_shard``);
  * the large GEMM shards B and C by column blocks: rank r computes
    C[:, r*N/g:(r+1)*N/g] = A @ B[:, r*N/g:(r+1)*N/g] (+ bias) with A replicated,
    then the blocks are all-gathered ([g][M][N/g], one NCCL collective) and
    rewritten to row-major [M][N] by the relayout kernel
    (``column_sharded_gemm``).
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
