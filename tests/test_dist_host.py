"""Host logic of the multi-GPU paths on CPU ranks (gloo, world sizes 2 and 4): the
batch and column shard plans and the gather order of the column-sharded GEMM.
Each rank computes its column block with the oracle GEMM (the stand-in for
nplk_gemm on CPU), the blocks are all-gathered over gloo and laid out with a
CPU restatement of nplk_colshard_relayout; the result must equal the full
product."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import support as S
from npl_b200 import dist as nd


def test_shard_plans():
    assert [nd.shard_range(10, 4, r) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert [nd.batch_shard(32, 8, r) for r in range(8)] == [(4 * r, 4 * r + 4) for r in range(8)]
    assert nd.column_block(16384, 8, 3) == (6144, 8192)
    with pytest.raises(ValueError):
        nd.column_block(10, 4, 0)
    with pytest.raises(ValueError):
        nd.shard_range(10, 2, 2)


def cpu_relayout(src_flat, g, rows, cps):
    """[g][rows][cps] -> [rows][g*cps] (what nplk_colshard_relayout computes)."""
    out = torch.empty(rows, g * cps, dtype=src_flat.dtype)
    src = src_flat.view(g, rows, cps)
    for s in range(g):
        out[:, s * cps:(s + 1) * cps] = src[s]
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        M, K, N = 24, 40, 32
        A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
        bias = rng.normal(0, 0.02, N).astype(np.float32)
        c0, c1 = nd.column_block(N, world, rank)
        local = S.o_sgemm(A, np.ascontiguousarray(B[:, c0:c1])) + bias[c0:c1]
        full = nd.gather_column_blocks(torch.from_numpy(local), world, relayout=cpu_relayout)
        ref = S.o_sgemm(A, B) + bias
        results[rank] = float(np.abs(full.numpy() - ref).max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_column_sharded_gemm_gather_gloo(world):
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn", join=True)
    assert sorted(results.keys()) == list(range(world))
    assert max(results.values()) < 1e-6
