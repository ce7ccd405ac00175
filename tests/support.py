"""Shared helpers for the NPL test-suite: library loading, the oracle, inputs
and error metrics. The oracle libraries under oracle/ are test infrastructure:
they are loaded here only as the checker."""
from __future__ import annotations

import ctypes as C
import os
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "project-jcore_b200"
if str(PKG) not in sys.path:
    sys.path.insert(0, str(PKG))

import npl_b200 as nb  # noqa: E402

ORACLE_LIB = REPO / "oracle" / "lib" / "libnpl_oracle.so"
REF_LIB = REPO / "oracle" / "_ref" / "libnpl_ref.so"
GOLDEN = REPO / "tests" / "golden"

_f = C.c_float
_i64 = C.c_int64
_p = C.c_void_p


def fptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.c_void_p)


_oracle = None


def oracle() -> C.CDLL:
    """The plain-C restatement of the reference (oracle/npl_oracle.c)."""
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists():
            raise RuntimeError(f"{ORACLE_LIB} missing: run `make -C oracle oracle`")
        lib = C.CDLL(str(ORACLE_LIB))
        lib.oracle_set_threads.argtypes = [C.c_int]
        lib.oracle_sgemm.argtypes = [_i64, _i64, _i64, _f, _p, _i64, _p, _i64, _f, _p, _i64]
        lib.oracle_conv2d.argtypes = [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p]
        lib.oracle_depthwise_conv2d.argtypes = [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64,
                                                _i64, _i64, _i64, _i64, _i64, _i64, _p, _p]
        lib.oracle_batch_norm.argtypes = [_p, _i64, _i64, _i64, _p, _p, _p, _p, _f, _p]
        lib.oracle_batch_norm_train.argtypes = [_p, _i64, _i64, _i64, _p, _p, _p, _p, _f, _f, _p]
        lib.oracle_activation.argtypes = [_p, _i64, C.c_int, _f, C.c_int, _p]
        lib.oracle_softmax.argtypes = [_p, _i64, _i64, _i64, _p]
        lib.oracle_layer_norm.argtypes = [_p, _i64, _i64, _p, _p, _f, _p]
        lib.oracle_pool2d.argtypes = [_p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _i64, C.c_int, C.c_int, _p]
        lib.oracle_global_avg_pool.argtypes = [_p, _i64, _i64, _p]
        lib.oracle_set_threads(os.cpu_count() or 1)
        _oracle = lib
    return _oracle


_ref = None


def reference() -> C.CDLL | None:
    """The reference's own NPL sources built for the CPU (oracle/_ref), or None."""
    global _ref
    if _ref is None and REF_LIB.exists():
        lib = C.CDLL(str(REF_LIB))
        nb.bind(lib, nb.NPL_SIGNATURES)
        cfg = nb.NplConfig()
        lib.npl_get_default_config(C.byref(cfg))
        cfg.num_threads = os.cpu_count() or 1
        assert lib.npl_init(C.byref(cfg)) == 0
        _ref = lib
    return _ref


def rng(seed: int = 0) -> np.random.Generator:
    return np.random.default_rng(seed)


def normwise_err(y: np.ndarray, r: np.ndarray) -> float:
    """max|y - r| / max|r| (the parity metric; 0 for an all-zero reference)."""
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    scale = np.max(np.abs(r)) if r.size else 0.0
    d = np.max(np.abs(y - r)) if r.size else 0.0
    return float(d / scale) if scale > 0 else float(d)


# ---- oracle wrappers (numpy in, numpy out) -------------------------------------

def o_sgemm(a, b, alpha=1.0, beta=0.0, c=None):
    m, k = a.shape
    n = b.shape[1]
    out = np.zeros((m, n), np.float32) if c is None else c.copy()
    oracle().oracle_sgemm(m, n, k, alpha, fptr(a), k, fptr(b), n, beta, fptr(out), n)
    return out


def conv_out_hw(h, w, kh, kw, sh, sw, pt, pb, pl, pr, dh=1, dw=1):
    return ((h + pt + pb - (dh * (kh - 1) + 1)) // sh + 1,
            (w + pl + pr - (dw * (kw - 1) + 1)) // sw + 1)


def o_conv2d(x, w, stride=(1, 1), pad=(0, 0), dil=(1, 1), bias=None):
    n, c, h, wd = x.shape
    co, _, kh, kw = w.shape
    ho, wo = conv_out_hw(h, wd, kh, kw, stride[0], stride[1], pad[0], pad[0], pad[1], pad[1],
                         dil[0], dil[1])
    out = np.empty((n, co, ho, wo), np.float32)
    oracle().oracle_conv2d(fptr(x), n, c, h, wd, fptr(w), co, kh, kw, stride[0], stride[1],
                           pad[0], pad[1], dil[0], dil[1], ho, wo, fptr(bias), fptr(out))
    return out


def o_depthwise(x, w, stride=(1, 1), pad=(0, 0), bias=None):
    n, c, h, wd = x.shape
    kh, kw = w.shape[-2:]
    ho, wo = conv_out_hw(h, wd, kh, kw, stride[0], stride[1], pad[0], pad[0], pad[1], pad[1])
    out = np.empty((n, c, ho, wo), np.float32)
    oracle().oracle_depthwise_conv2d(fptr(x), n, c, h, wd, fptr(w), kh, kw, stride[0],
                                     stride[1], pad[0], pad[1], ho, wo, fptr(bias), fptr(out))
    return out


def o_batch_norm(x, mean, var, gamma=None, beta=None, eps=1e-5):
    n, c = x.shape[:2]
    hw = int(np.prod(x.shape[2:]))
    out = np.empty_like(x)
    oracle().oracle_batch_norm(fptr(x), n, c, hw, fptr(mean), fptr(var), fptr(gamma),
                               fptr(beta), eps, fptr(out))
    return out


def o_batch_norm_train(x, run_mean, run_var, gamma=None, beta=None, eps=1e-5, momentum=0.1):
    n, c = x.shape[:2]
    hw = int(np.prod(x.shape[2:]))
    out = np.empty_like(x)
    oracle().oracle_batch_norm_train(fptr(x), n, c, hw, fptr(run_mean), fptr(run_var),
                                     fptr(gamma), fptr(beta), eps, momentum, fptr(out))
    return out


def o_activation(x, act, alpha=0.01, scalar=0):
    out = np.empty_like(x)
    oracle().oracle_activation(fptr(x), x.size, act, alpha, scalar, fptr(out))
    return out


def o_softmax(x, axis):
    axis = axis % x.ndim
    outer = int(np.prod(x.shape[:axis]))
    inner = int(np.prod(x.shape[axis + 1:]))
    out = np.empty_like(x)
    oracle().oracle_softmax(fptr(x), outer, x.shape[axis], inner, fptr(out))
    return out


def o_layer_norm(x, cols, gamma=None, beta=None, eps=1e-5):
    rows = x.size // cols
    out = np.zeros_like(x)
    oracle().oracle_layer_norm(fptr(x), rows, cols, fptr(gamma), fptr(beta), eps, fptr(out))
    return out


def o_pool(x, k, s, p, kind=0, count_include_pad=0):
    n, c, h, w = x.shape
    ho = (h + 2 * p[0] - k[0]) // s[0] + 1
    wo = (w + 2 * p[1] - k[1]) // s[1] + 1
    out = np.empty((n, c, ho, wo), np.float32)
    oracle().oracle_pool2d(fptr(x), n, c, h, w, k[0], k[1], s[0], s[1], p[0], p[1], ho, wo,
                           kind, count_include_pad, fptr(out))
    return out


def o_gap(x):
    n, c = x.shape[:2]
    hw = int(np.prod(x.shape[2:]))
    out = np.empty((n, c), np.float32)
    oracle().oracle_global_avg_pool(fptr(x), n * c, hw, fptr(out))
    return out


# ---- calling an npl_* library on host numpy buffers -----------------------------

class HostTensors:
    """Keeps numpy buffers alive while npl_tensor_t descriptors point at them."""

    def __init__(self, lib):
        self.lib = lib
        self.keep = []

    def t(self, arr: np.ndarray, layout=nb.NPL_LAYOUT_NCHW):
        assert arr.dtype == np.float32 and arr.flags.c_contiguous
        self.keep.append(arr)
        return nb.tensor(self.lib, arr.ctypes.data, arr.shape, nb.NPL_DTYPE_FP32, layout)


def npl_call(lib, name, *args):
    return getattr(lib, name)(*[C.byref(a) if isinstance(a, C.Structure) else a for a in args])


_gpu_lib = None


def gpu_lib() -> C.CDLL:
    """libnpl_b200.so initialised on cuda:0 (torch's current device)."""
    global _gpu_lib
    if _gpu_lib is None:
        import torch
        torch.cuda.init()
        torch.cuda.set_device(0)
        lib = nb.load()
        assert lib.npl_init(None) == nb.NPL_OK
        _gpu_lib = lib
    return _gpu_lib


def dptr(t):
    """Device address of a contiguous torch tensor as a c_void_p."""
    assert t.is_contiguous()
    return C.c_void_p(t.data_ptr())


def cuda_stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)
