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
