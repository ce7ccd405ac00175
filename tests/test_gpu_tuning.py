"""The tile-configuration cache on the device: nplk_conv2d_tune and
nplk_gemm_tune measure the candidates and cache the fastest; the AUTO paths
follow the cache (a cached choice the workspace cannot hold falls back to the
uncached choice); every cached choice gives the same bits as the direct
kernel; and npl_init / npl_shutdown load and save the file NPL_TUNING_CACHE
names, with NPL_AUTOTUNE=1 tuning a shape on its first call."""
import ctypes as C
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu


@pytest.fixture()
def lib():
    lib = S.gpu_lib()
    lib.nplk_tuning_cache_clear()
    yield lib
    lib.nplk_tuning_cache_clear()


def _conv_inputs(g, seed=0):
    import torch
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.rand(g.n, g.c_in, g.h, g.w, device="cuda", generator=gen)
    w = torch.randn(g.c_out, g.c_in, g.kh, g.kw, device="cuda", generator=gen) * 0.05
    bn = [torch.rand(g.c_out, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    return x, w, bn


def _key(lib, g):
    buf = C.create_string_buffer(256)
    lib.nplk_tuning_key_conv(C.byref(g), buf, 256)
    return buf.value


def test_conv_tune_caches_a_kernel_with_identical_output(lib):
    import torch
    g = nb.conv_geom(4, 64, 28, 28, 64, 3, 3, 1, 1)
    x, w, bn = _conv_inputs(g)
    ws = max(lib.nplk_conv_workspace_size_algo(C.byref(g), a) for a in range(1, 6))
    work = torch.empty(ws // 4 + 64, device="cuda")
    y = torch.empty(g.n, g.c_out, g.h_out, g.w_out, device="cuda")
    best, us = C.c_int(), C.c_float()
    rc = lib.nplk_conv2d_tune(S.cuda_stream(), C.byref(g), S.dptr(x), S.dptr(w), None,
                              S.dptr(bn[0]), S.dptr(bn[1]), S.dptr(bn[2]), S.dptr(bn[3]), 1e-5,
                              nb.NPL_ACT_RELU, 0.0, S.dptr(y), S.dptr(work), ws, 3,
                              C.byref(best), C.byref(us))
    assert rc == 0
    assert best.value in range(1, 6) and us.value > 0
    choice = C.c_int()
    assert lib.nplk_tuning_cache_get(_key(lib, g), C.byref(choice), None) == 1
    assert choice.value == best.value
    ref = torch.empty_like(y)
    assert lib.nplk_conv2d_run_algo(S.cuda_stream(), C.byref(g), S.dptr(x), nb.NPL_ACT_RELU,
                                    0.0, S.dptr(ref), S.dptr(work), ws, None,
                                    nb.NPLK_CONV_ALGO_DIRECT) == 0
    torch.cuda.synchronize()
    assert torch.equal(y, ref)  # the tuning call leaves the conv's output


def test_auto_follows_the_cache_and_falls_back_when_the_workspace_is_small(lib):
    import torch
    g = nb.conv_geom(4, 64, 28, 28, 64, 3, 3, 1, 1)  # AUTO alone: window gather, no planes
    x, w, bn = _conv_inputs(g, 1)
    small = lib.nplk_conv_workspace_min_size(C.byref(g))
    assert lib.nplk_conv_workspace_size(C.byref(g)) == small
    full_im2col = lib.nplk_conv_workspace_size_algo(C.byref(g), nb.NPLK_CONV_ALGO_IM2COL)
    assert lib.nplk_tuning_cache_put(_key(lib, g), nb.NPLK_CONV_ALGO_IM2COL, 1.0) == 0
    assert lib.nplk_conv_workspace_size(C.byref(g)) == full_im2col  # AUTO now means IM2COL
    work = torch.empty(full_im2col // 4 + 64, device="cuda")
    outs = []
    for ws, launches in ((full_im2col, 3), (small, 2)):  # prep + (NHWC rewrite +) conv
        y = torch.empty(g.n, g.c_out, g.h_out, g.w_out, device="cuda")
        lib.nplk_take_launch_count()
        assert lib.nplk_conv2d_fused(S.cuda_stream(), C.byref(g), S.dptr(x), S.dptr(w), None,
                                     S.dptr(bn[0]), S.dptr(bn[1]), S.dptr(bn[2]), S.dptr(bn[3]),
                                     1e-5, nb.NPL_ACT_RELU, 0.0, S.dptr(y), S.dptr(work), ws,
                                     None) == 0
        assert lib.nplk_take_launch_count() == launches
        torch.cuda.synchronize()
        outs.append(y)
    assert torch.equal(outs[0], outs[1])
    st = nb.NplkTuningStats()
    lib.nplk_tuning_cache_stats(C.byref(st))
    assert st.hits >= 2


@pytest.mark.parametrize("bn_forced", [64, 128, 1128])
def test_gemm_follows_a_cached_tile_width(lib, bn_forced):
    import torch
    m = n = k = 512
    gen = torch.Generator(device="cuda").manual_seed(bn_forced)
    A = torch.rand(m, k, device="cuda", generator=gen) * 2 - 1
    B = torch.rand(k, n, device="cuda", generator=gen) * 2 - 1
    buf = C.create_string_buffer(256)
    lib.nplk_tuning_key_gemm(m, n, k, buf, 256)
    assert lib.nplk_tuning_cache_put(buf.value, bn_forced, 1.0) == 0
    ws = lib.nplk_gemm_workspace_size(m, n, k)
    work = torch.empty(ws // 4 + 64, device="cuda")
    Cm = torch.empty(m, n, device="cuda")
    assert lib.nplk_gemm(S.cuda_stream(), m, n, k, 1.0, S.dptr(A), k, S.dptr(B), n, 0.0,
                         S.dptr(Cm), n, None, 0, 0.0, 0, S.dptr(work), ws, None) == 0
    torch.cuda.synchronize()
    ref = A.double() @ B.double()
    assert ((Cm.double() - ref).abs().max() / ref.abs().max()).item() < 1e-4


def test_gemm_tune_caches_the_faster_tile_width(lib):
    import torch
    m, n, k = 1024, 1024, 1024
    gen = torch.Generator(device="cuda").manual_seed(3)
    A = torch.rand(m, k, device="cuda", generator=gen) * 2 - 1
    B = torch.rand(k, n, device="cuda", generator=gen) * 2 - 1
    Cm = torch.empty(m, n, device="cuda")
    ws = lib.nplk_gemm_workspace_size(m, n, k)
    work = torch.empty(ws // 4 + 64, device="cuda")
    best, us = C.c_int(), C.c_float()
    assert lib.nplk_gemm_tune(S.cuda_stream(), m, n, k, S.dptr(A), k, S.dptr(B), n, S.dptr(Cm), n,
                              S.dptr(work), ws, 5, C.byref(best), C.byref(us)) == 0
    assert best.value in (64, 128, 1128) and us.value > 0
    torch.cuda.synchronize()
    ref = A.double() @ B.double()
    assert ((Cm.double() - ref).abs().max() / ref.abs().max()).item() < 1e-4


def test_cache_file_persists_across_processes_with_autotune(tmp_path):
    # Process 1 tunes on first use (NPL_AUTOTUNE=1) and npl_shutdown writes the
    # file; process 2 loads it at npl_init and its call hits the cache.
    path = tmp_path / "tiles.cache"
    script = textwrap.dedent(f"""
        import ctypes as C, sys
        sys.path.insert(0, {str(S.REPO / 'tests')!r})
        import numpy as np, support as S
        from support import nb
        lib = S.gpu_lib()
        rng = np.random.default_rng(0)
        a = rng.uniform(-1, 1, (384, 256)).astype(np.float32)
        b = rng.uniform(-1, 1, (256, 320)).astype(np.float32)
        c = np.zeros((384, 320), np.float32)
        h = S.HostTensors(lib)
        assert S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(1.0),
                          C.c_float(0.0), None) == 0
        assert S.normwise_err(c, a.astype(np.float64) @ b) < 1e-4
        st = nb.NplkTuningStats()
        lib.nplk_tuning_cache_stats(C.byref(st))
        print("entries", st.entries, "hits", st.hits, "tunes", st.tunes)
        lib.npl_shutdown()
    """)
    env = dict(os.environ, NPL_TUNING_CACHE=str(path), NPL_AUTOTUNE="1")
    r1 = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True,
                        timeout=300)
    assert r1.returncode == 0, r1.stderr[-3000:]
    assert "entries 1 " in r1.stdout and "tunes 1" in r1.stdout
    assert path.exists() and "gemm m=384 n=320 k=256" in path.read_text()
    r2 = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True,
                        timeout=300)
    assert r2.returncode == 0, r2.stderr[-3000:]
    assert "entries 1 " in r2.stdout and "tunes 0" in r2.stdout
    hits = int(r2.stdout.split("hits")[1].split()[0])
    assert hits >= 1
