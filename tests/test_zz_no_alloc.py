"""The no-allocation conv entry point (nplk_conv2d_fused_noalloc).

Some callers cannot allocate device memory: serving hosts that reserve their
whole device budget at start-up, code running inside an allocator callback,
and foreign-language callers that must not trigger the device-wide
synchronisation cudaMalloc/cudaFree can cause. For them the library keeps the
conv workspace in a fixed array of its own. These tests call that entry point
through the C ABI, twice in a row with different weights and BN parameters,
and compare each result with the regular workspace-taking entry point
(nplk_conv2d_fused) within the conv parity tolerance. This file is collected
last so that a run stopping at its first failure has already run every other
test.
"""
import ctypes as C

import numpy as np
import pytest

import support as S
from support import nb

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _inputs(seed, n=4, c=64, hw=28, cout=64):
    import torch
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.rand(n, c, hw, hw, device="cuda", generator=gen)
    w = torch.randn(cout, c, 3, 3, device="cuda", generator=gen) * 0.05
    bn = [torch.rand(cout, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    return x, w, bn


def _inputs_geom(seed, g):
    import torch
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.rand(g.n, g.c_in, g.h, g.w, device="cuda", generator=gen)
    w = torch.randn(g.c_out, g.c_in, g.kh, g.kw, device="cuda", generator=gen) * 0.05
    bn = [torch.rand(g.c_out, device="cuda", generator=gen) + 0.5 for _ in range(4)]
    return x, w, bn


def _regular(lib, g, x, w, bn, act):
    import torch
    y = torch.empty(g.n, g.c_out, g.h_out, g.w_out, device="cuda")
    ws = lib.nplk_conv_workspace_size(C.byref(g))
    work = torch.empty(ws // 4 + 64, device="cuda")
    gamma, beta, mean, var = bn
    rc = lib.nplk_conv2d_fused(S.cuda_stream(), C.byref(g), S.dptr(x), S.dptr(w), None,
                               S.dptr(mean), S.dptr(var), S.dptr(gamma), S.dptr(beta), 1e-5,
                               act, 0.01, S.dptr(y), S.dptr(work), ws, None)
    assert rc == 0
    torch.cuda.synchronize()
    return y


def _noalloc(lib, g, x, w, bn, act):
    import torch
    y = torch.empty(g.n, g.c_out, g.h_out, g.w_out, device="cuda")
    gamma, beta, mean, var = bn
    rc = lib.nplk_conv2d_fused_noalloc(S.cuda_stream(), C.byref(g), S.dptr(x), S.dptr(w), None,
                                       S.dptr(mean), S.dptr(var), S.dptr(gamma), S.dptr(beta),
                                       1e-5, act, 0.01, S.dptr(y), None)
    assert rc == 0
    torch.cuda.synchronize()
    return y


def test_noalloc_matches_regular_entry_point_twice():
    lib = S.gpu_lib()
    g = nb.conv_geom(4, 64, 28, 28, 64, 3, 3, 1, 1)
    x1, w1, bn1 = _inputs(1)
    x2, w2, bn2 = _inputs(2)
    # two calls in a row with different weights: the shared scratch must be
    # rewritten by the second call
    y1 = _noalloc(lib, g, x1, w1, bn1, nb.NPL_ACT_RELU)
    y2 = _noalloc(lib, g, x2, w2, bn2, nb.NPL_ACT_RELU)
    r1 = _regular(lib, g, x1, w1, bn1, nb.NPL_ACT_RELU)
    r2 = _regular(lib, g, x2, w2, bn2, nb.NPL_ACT_RELU)
    assert S.normwise_err(y1.cpu().numpy(), r1.cpu().numpy()) < TOL
    assert S.normwise_err(y2.cpu().numpy(), r2.cpu().numpy()) < TOL
    assert S.normwise_err(y1.cpu().numpy(), r2.cpu().numpy()) > 1e-2  # really different


def test_noalloc_rejects_geometry_beyond_its_scratch():
    lib = S.gpu_lib()
    # 1024 output channels x (512*3*3) reduction needs ~38 MB of split weights
    g = nb.conv_geom(1, 512, 8, 8, 1024, 3, 3, 1, 1)
    assert lib.nplk_conv_workspace_size(C.byref(g)) > (8 << 20)
    import torch
    x = torch.zeros(1, 512, 8, 8, device="cuda")
    w = torch.zeros(1024, 512, 3, 3, device="cuda")
    y = torch.empty(1, 1024, 8, 8, device="cuda")
    rc = lib.nplk_conv2d_fused_noalloc(S.cuda_stream(), C.byref(g), S.dptr(x), S.dptr(w), None,
                                       None, None, None, None, 1e-5, 0, 0.0, S.dptr(y), None)
    assert rc == nb.NPL_ERR_UNSUPPORTED


def test_noalloc_direct_kernel_when_the_planes_do_not_fit():
    # A 3x3 stride-2 layer runs on the TMA im2col kernel, whose NHWC tf32
    # planes (51 MB here) do not fit the fixed array while the split weights
    # and constants do: the entry point then runs the direct-gather kernel.
    lib = S.gpu_lib()
    g = nb.conv_geom(32, 64, 56, 56, 64, 3, 3, 2, 1)
    full = lib.nplk_conv_workspace_size(C.byref(g))
    need = lib.nplk_conv_workspace_min_size(C.byref(g))
    assert full > (8 << 20) >= need > 0
    x1, w1, bn1 = _inputs_geom(3, g)
    x2, w2, bn2 = _inputs_geom(4, g)
    y1 = _noalloc(lib, g, x1, w1, bn1, nb.NPL_ACT_RELU)
    y2 = _noalloc(lib, g, x2, w2, bn2, nb.NPL_ACT_RELU)
    r1 = _regular(lib, g, x1, w1, bn1, nb.NPL_ACT_RELU)
    r2 = _regular(lib, g, x2, w2, bn2, nb.NPL_ACT_RELU)
    assert S.normwise_err(y1.cpu().numpy(), r1.cpu().numpy()) < TOL
    assert S.normwise_err(y2.cpu().numpy(), r2.cpu().numpy()) < TOL
    assert lib.nplk_read_status(S.cuda_stream()) == 0


def test_noalloc_timeout_is_readable_without_allocating():
    # With status == NULL a bounded-wait timeout lands in the entry point's own
    # word; nplk_read_status() reads and clears it. The armed launch stalls the
    # window kernel's MMA issuers for 50 ms (nplk_debug_arm_wait_timeout).
    lib = S.gpu_lib()
    g = nb.conv_geom(4, 64, 28, 28, 64, 3, 3, 1, 1)
    x, w, bn = _inputs(5)
    _noalloc(lib, g, x, w, bn, nb.NPL_ACT_RELU)  # set-up on this device
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    assert lib.nplk_debug_arm_wait_timeout(nb.NPLK_DEBUG_CONV_WINDOW, 50_000) == 0
    _noalloc(lib, g, x, w, bn, nb.NPL_ACT_RELU)
    assert lib.nplk_read_status(S.cuda_stream()) == nb.NPLK_STATUS_TIMEOUT_MMA
    assert lib.nplk_read_status(S.cuda_stream()) == 0  # read clears it
    y = _noalloc(lib, g, x, w, bn, nb.NPL_ACT_RELU)
    assert lib.nplk_read_status(S.cuda_stream()) == 0
    r = _regular(lib, g, x, w, bn, nb.NPL_ACT_RELU)
    assert S.normwise_err(y.cpu().numpy(), r.cpu().numpy()) < TOL

