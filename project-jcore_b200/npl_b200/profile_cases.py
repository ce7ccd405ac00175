"""Small, fixed workloads for profiling the NPL kernels (for example under
``ncu``). Each case allocates its inputs on cuda:0, runs the kernel a few times
and checks the kernel status word.

    python -m npl_b200.profile_cases conv      # 3x3 conv+BN+ReLU, N=32 64->64 56x56 (default kernel)
    python -m npl_b200.profile_cases conv_direct  # the same on the direct-gather kernel
    python -m npl_b200.profile_cases conv_window_tma  # ... on TMA windows over an NHWC plane
    python -m npl_b200.profile_cases conv_s2   # 3x3 stride 2, N=32 64->128 56x56 (im2col kernel)
    python -m npl_b200.profile_cases stem      # 7x7/s2 conv+BN+ReLU, N=16 3->64 224x224
    python -m npl_b200.profile_cases gemm      # 4096x4096x8192 3xTF32 GEMM
    python -m npl_b200.profile_cases chain     # depthwise, BN, ReLU, GAP, softmax 256x512x14x14
    python -m npl_b200.profile_cases chain_fused # the same chain, its first four calls in one pass
    python -m npl_b200.profile_cases layernorm # 8192 x 16384 rows
    python -m npl_b200.profile_cases pool      # max pool 3x3/s2 [32,64,112,112] -> 56x56
    python -m npl_b200.profile_cases gemm_raw  # the 4096x4096x8192 GEMM, raw operand form
    python -m npl_b200.profile_cases gemm_1024 # 1024^3 (split kernels + GEMM)
    python -m npl_b200.profile_cases bandwidth # BN, ReLU, GAP on 256x512x14x14; softmax 102400x1000
    python -m npl_b200.profile_cases allgather # fused GEMM all-gather epilogue, 2 simulated ranks
    python -m npl_b200.profile_cases conv_pair # the 3x3 conv on CTA pairs
    python -m npl_b200.profile_cases conv_n256 # the 3x3 conv at N=256 (output beyond L2)
    python -m npl_b200.profile_cases stem_fused # stem conv + pool, and the fused form (N=16)

Run from the package directory (``project-jcore_b200``) or with it on sys.path.
"""
from __future__ import annotations

import ctypes as C
import sys


def _setup():
    import torch
    from . import load
    torch.cuda.set_device(0)
    lib = load()
    return torch, lib, C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return C.c_void_p(t.data_ptr())


def case_conv(reps: int = 3, n: int = 32, c: int = 64, hw: int = 56, cout: int = 64,
              k: int = 3, stride: int = 1, pad: int = 1, algo: int = 0):
    from . import conv_geom
    torch, lib, s = _setup()
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = torch.rand(n, c, hw, hw, device="cuda", generator=gen)
    w = torch.randn(cout, c, k, k, device="cuda", generator=gen) * 0.05
    bn = [torch.rand(cout, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    g = conv_geom(n, c, hw, hw, cout, k, k, stride, pad)
    y = torch.empty(n, cout, g.h_out, g.w_out, device="cuda")
    ws = lib.nplk_conv_workspace_size_algo(C.byref(g), algo)
    assert ws > 0
    work = torch.empty(ws // 4 + 64, device="cuda")
    for _ in range(reps):
        rc = lib.nplk_conv2d_prepare(s, C.byref(g), _p(w), None, _p(bn[0]), _p(bn[1]), _p(bn[2]),
                                     _p(bn[3]), 1e-5, _p(work), ws)
        assert rc == 0, rc
        rc = lib.nplk_conv2d_run_algo(s, C.byref(g), _p(x), 1, 0.0, _p(y), _p(work), ws, None,
                                      algo)
        assert rc == 0, rc
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0


def case_stem(reps: int = 3):
    case_conv(reps, n=16, c=3, hw=224, cout=64, k=7, stride=2, pad=3)


def case_gemm(reps: int = 3, m: int = 4096, n: int = 4096, k: int = 8192, raw: bool = False):
    torch, lib, s = _setup()
    gen = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(m, k, device="cuda", generator=gen)
    b = torch.randn(k, n, device="cuda", generator=gen) / 64.0
    c = torch.empty(m, n, device="cuda")
    ws = 0 if raw else lib.nplk_gemm_workspace_size(m, n, k)
    work = None if raw else torch.empty(ws // 4 + 64, device="cuda")
    for _ in range(reps):
        rc = lib.nplk_gemm(s, m, n, k, 1.0, _p(a), k, _p(b), n, 0.0, _p(c), n, None, 0, 0.0, 0,
                           _p(work) if work is not None else None, ws, None)
        assert rc == 0, rc
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0


def case_chain(reps: int = 3):
    from . import conv_geom
    torch, lib, s = _setup()
    gen = torch.Generator(device="cuda").manual_seed(0)
    n, c, hw = 256, 512, 14
    x = torch.randn(n, c, hw, hw, device="cuda", generator=gen)
    w = torch.randn(c, 1, 3, 3, device="cuda", generator=gen) * 0.3
    bn = [torch.rand(c, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    t1, t2 = torch.empty_like(x), torch.empty_like(x)
    gap = torch.empty(n, c, device="cuda")
    sm = torch.empty_like(gap)
    g = conv_geom(n, c, hw, hw, c, 3, 3, 1, 1)
    for _ in range(reps):
        assert lib.nplk_depthwise_conv2d(s, C.byref(g), _p(x), _p(w), None, _p(t1)) == 0
        assert lib.nplk_batch_norm_infer(s, n, c, hw * hw, _p(t1), _p(t2), _p(bn[0]), _p(bn[1]),
                                         _p(bn[2]), _p(bn[3]), 1e-5) == 0
        assert lib.nplk_activation(s, t2.numel(), _p(t2), _p(t2), 1, 0.0, 0) == 0
        assert lib.nplk_global_avg_pool(s, n * c, hw * hw, _p(t2), _p(gap)) == 0
        assert lib.nplk_softmax(s, n, c, 1, _p(gap), _p(sm)) == 0
    torch.cuda.synchronize()


def case_chain_fused(reps: int = 3):
    """The bandwidth chain's fused pass (nplk_depthwise_bn_act_gap, no map
    written) and its softmax on [256,512,14,14]."""
    from . import workloads
    torch, lib, s = _setup()
    gen = torch.Generator(device="cuda").manual_seed(0)
    n, c, hw = 256, 512, 14
    x = torch.randn(n, c, hw, hw, device="cuda", generator=gen)
    w = torch.randn(c, 1, 3, 3, device="cuda", generator=gen) * 0.3
    bn = [torch.rand(c, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    gap, sm = torch.empty(n, c, device="cuda"), torch.empty(n, c, device="cuda")
    for _ in range(reps):
        assert workloads.bandwidth_chain_fused(lib, s, x, w, bn[0], bn[1], bn[2], bn[3], gap,
                                               sm) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0


def case_pool(reps: int = 3):
    torch, lib, s = _setup()
    x = torch.randn(32, 64, 112, 112, device="cuda")
    y = torch.empty(32, 64, 56, 56, device="cuda")
    for _ in range(reps):
        assert lib.nplk_pool2d(s, 32, 64, 112, 112, 3, 3, 2, 2, 1, 1, 56, 56, 0, 0, _p(x),
                               _p(y)) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0


def case_layernorm(reps: int = 3):
    torch, lib, s = _setup()
    x = torch.randn(8192, 16384, device="cuda")
    y = torch.empty_like(x)
    for _ in range(reps):
        assert lib.nplk_layer_norm(s, 8192, 16384, _p(x), _p(y), None, None, 1e-5) == 0
    torch.cuda.synchronize()


def case_bandwidth(reps: int = 2):
    """Batch norm (inference), ReLU and global average pool on [256,512,14,14]
    (103 MB) and softmax over 102400 rows of 1000 (410 MB), `reps` rounds in
    that order."""
    torch, lib, s = _setup()
    gen = torch.Generator(device="cuda").manual_seed(0)
    n, c, hw = 256, 512, 14
    x = torch.randn(n, c, hw, hw, device="cuda", generator=gen)
    y = torch.empty_like(x)
    bn = [torch.rand(c, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    gap = torch.empty(n * c, device="cuda")
    logits = torch.randn(102400, 1000, device="cuda", generator=gen)
    probs = torch.empty_like(logits)
    for _ in range(reps):
        assert lib.nplk_batch_norm_infer(s, n, c, hw * hw, _p(x), _p(y), _p(bn[0]), _p(bn[1]),
                                         _p(bn[2]), _p(bn[3]), 1e-5) == 0
        assert lib.nplk_activation(s, x.numel(), _p(x), _p(y), 1, 0.0, 0) == 0
        assert lib.nplk_global_avg_pool(s, n * c, hw * hw, _p(x), _p(gap)) == 0
        assert lib.nplk_softmax(s, 102400, 1000, 1, _p(logits), _p(probs)) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0


def case_allgather(reps: int = 2, m: int = 4096, n_local: int = 2048, k: int = 4096,
                   ranks: int = 2):
    """The fused GEMM + all-gather epilogue (nplk_gemm_allgather) with `ranks`
    simulated ranks on one GPU: every output tile is stored into `ranks` full
    row-major C buffers (on this device), as the multi-GPU form stores into
    every rank's C; then the NCCL form's relayout kernel on [ranks][m][n_local]."""
    torch, lib, s = _setup()
    gen = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(m, k, device="cuda", generator=gen)
    b = torch.randn(k, n_local, device="cuda", generator=gen) / 64.0
    cs = [torch.empty(m, ranks * n_local, device="cuda") for _ in range(ranks)]
    dst = (C.c_void_p * ranks)(*[t.data_ptr() for t in cs])
    ws = lib.nplk_gemm_workspace_size(m, n_local, k)
    work = torch.empty(ws // 4 + 64, device="cuda")
    blocks = torch.randn(ranks * m * n_local, device="cuda", generator=gen)
    out = torch.empty(m, ranks * n_local, device="cuda")
    for _ in range(reps):
        rc = lib.nplk_gemm_allgather(s, m, n_local, k, 1.0, _p(a), k, _p(b), n_local, None, 0,
                                     0.0, dst, ranks, 0, ranks * n_local, 0, _p(work), ws, None)
        assert rc == 0, rc
        assert lib.nplk_colshard_relayout(s, ranks, m, n_local, _p(blocks), _p(out)) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0


def case_stem_fused(reps: int = 2, n: int = 16):
    """The stem block both ways: conv (+BN+ReLU) then 3x3/s2 max pool, and the
    fused nplk_conv2d_maxpool_fused, `reps` rounds."""
    from . import conv_geom
    torch, lib, s = _setup()
    gen = torch.Generator(device="cuda").manual_seed(0)
    g = conv_geom(n, 3, 224, 224, 64, 7, 7, 2, 3)
    x = torch.rand(n, 3, 224, 224, device="cuda", generator=gen) * 2 - 1
    w = torch.randn(64, 3, 7, 7, device="cuda", generator=gen) * (2.0 / 147) ** 0.5
    bn = [torch.rand(64, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    y = torch.empty(n, 64, 112, 112, device="cuda")
    pooled = torch.empty(n, 64, 56, 56, device="cuda")
    fused = torch.empty_like(pooled)
    ws = lib.nplk_conv_workspace_size(C.byref(g))
    work = torch.empty(ws // 4 + 64, device="cuda")
    fws = lib.nplk_conv2d_maxpool_workspace_size(C.byref(g))
    fwork = torch.empty(fws // 4 + 64, device="cuda")
    for _ in range(reps):
        assert lib.nplk_conv2d_fused(s, C.byref(g), _p(x), _p(w), None, _p(bn[0]), _p(bn[1]),
                                     _p(bn[2]), _p(bn[3]), 1e-5, 1, 0.0, _p(y), _p(work), ws,
                                     None) == 0
        assert lib.nplk_pool2d(s, n, 64, 112, 112, 3, 3, 2, 2, 1, 1, 56, 56, 0, 0, _p(y),
                               _p(pooled)) == 0
        assert lib.nplk_conv2d_maxpool_fused(s, C.byref(g), _p(x), _p(w), None, _p(bn[0]),
                                             _p(bn[1]), _p(bn[2]), _p(bn[3]), 1e-5, 1, 0.0,
                                             _p(fused), _p(fwork), fws, None) == 0
    torch.cuda.synchronize()
    assert lib.nplk_read_status(s) == 0
    assert torch.equal(fused, pooled)


CASES = {"conv": case_conv, "chain_fused": case_chain_fused,
         "conv_direct": lambda: case_conv(algo=1),
         "conv_window_tma": lambda: case_conv(algo=3),
         "conv_s2": lambda: case_conv(cout=128, stride=2),
         "stem": case_stem, "gemm": case_gemm, "chain": case_chain,
         "layernorm": case_layernorm, "pool": case_pool,
         "gemm_raw": lambda: case_gemm(raw=True),
         "gemm_1024": lambda: case_gemm(m=1024, n=1024, k=1024),
         "gemm_raw_1024": lambda: case_gemm(m=1024, n=1024, k=1024, raw=True),
         "bandwidth": case_bandwidth, "allgather": case_allgather,
         "conv_pair": lambda: case_conv(algo=5),
         "conv_n256": lambda: case_conv(n=256),
         "stem_fused": case_stem_fused}

if __name__ == "__main__":
    name = sys.argv[1] if len(sys.argv) > 1 else "conv"
    CASES[name]()
    print("ok", name)
