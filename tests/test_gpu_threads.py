"""Concurrent npl_* calls from several host threads on distinct tensors (the
boundary's contract: ops are unlocked, calls from different threads may
overlap). Each thread runs GEMMs, fused conv + BN + ReLU and ReLU on its own
host tensors and checks every result against the oracle. ctypes releases the
GIL for the duration of each foreign call, so the calls do overlap."""
import ctypes as C
import threading

import numpy as np
import pytest

import support as S
from support import nb
from test_gpu_conv import bn_params, fused_host, oracle_fused

pytestmark = pytest.mark.gpu


def _worker(lib, i, errors):
    try:
        rng = S.rng(1000 + i)
        h = S.HostTensors(lib)
        for it in range(4):
            m, k, n = 96 + 32 * i, 64 + 16 * it, 80 + 8 * i
            a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
            b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
            c = np.zeros((m, n), np.float32)
            rc = S.npl_call(lib, "npl_matmul", h.t(a), h.t(b), h.t(c), C.c_float(1.0),
                            C.c_float(0.0), None)
            assert rc == 0, ("matmul", i, it, rc)
            assert S.normwise_err(c, S.o_sgemm(a, b)) < 1e-4, ("matmul", i, it)

            x = rng.uniform(-1, 1, (2, 16, 20 + i, 18)).astype(np.float32)
            w = rng.normal(0, 0.2, (24, 16, 3, 3)).astype(np.float32)
            bn = bn_params(24, rng)
            y, _ = fused_host(lib, x, w, bn, nb.NPL_ACT_RELU, pad=(1, 1))
            ref = oracle_fused(x, w, bn, nb.NPL_ACT_RELU, pad=(1, 1))
            assert S.normwise_err(y, ref) < 1e-4, ("conv", i, it)

            r = rng.normal(0, 1, 5000 + 17 * i).astype(np.float32)
            out = np.zeros_like(r)
            assert S.npl_call(lib, "npl_relu", h.t(r), h.t(out), None) == 0
            assert np.array_equal(out, np.maximum(r, 0.0)), ("relu", i, it)
    except Exception as e:  # reported by the main thread
        errors.append(f"thread {i}: {e!r}")


def test_concurrent_calls_from_host_threads():
    lib = S.gpu_lib()
    errors = []
    threads = [threading.Thread(target=_worker, args=(lib, i, errors)) for i in range(6)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not any(t.is_alive() for t in threads), "a thread did not finish"
    assert not errors, errors
    assert lib.nplk_read_status(None) == 0
