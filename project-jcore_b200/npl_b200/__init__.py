"""ctypes bindings for the NPL C ABI (``include/neural_primitives.h``) and the
device-level ABI of the B200 backend (``include/npl_kernels.h``).

The same struct definitions bind any library that exports the reference's
``npl_*`` ABI (advanced/neural_layer/include/neural_primitives.h:44-579), so
callers can drive the B200 library and a CPU build of the reference through one
interface. ``load()`` opens the in-tree ``lib/libnpl_b200.so`` and fails loudly
when it has not been built: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_DIR / "lib" / "libnpl_b200.so"

# ---- return codes (neural_primitives.h:52-59) ---------------------------------
NPL_OK = 0
NPL_ERR_NOT_INITIALIZED = -1
NPL_ERR_INVALID_ARG = -2
NPL_ERR_NO_MEMORY = -3
NPL_ERR_INTERNAL = -4
NPL_ERR_UNSUPPORTED = -5
NPL_ERR_SHAPE_MISMATCH = -6
NPL_ERR_OOM = -7

NPL_LAYOUT_NCHW, NPL_LAYOUT_NHWC, NPL_LAYOUT_NCHW_VECT_C = 0, 1, 2
NPL_DTYPE_FP32, NPL_DTYPE_FP16, NPL_DTYPE_BF16, NPL_DTYPE_INT8, NPL_DTYPE_INT32 = range(5)
(NPL_ACT_NONE, NPL_ACT_RELU, NPL_ACT_RELU6, NPL_ACT_TANH, NPL_ACT_SIGMOID, NPL_ACT_GELU,
 NPL_ACT_SWISH, NPL_ACT_LEAKY_RELU, NPL_ACT_ELU, NPL_ACT_SELU, NPL_ACT_SOFTPLUS) = range(11)
NPL_PAD_VALID, NPL_PAD_SAME, NPL_PAD_EXPLICIT = 0, 1, 2
NPL_POOL_MAX, NPL_POOL_AVG, NPL_POOL_GLOBAL_AVG, NPL_POOL_GLOBAL_MAX = 0, 1, 2, 3
NPL_MAX_DIMS = 8
NPLK_CONV_ALGO_AUTO, NPLK_CONV_ALGO_DIRECT, NPLK_CONV_ALGO_IM2COL = 0, 1, 2
NPLK_CONV_ALGO_WINDOW, NPLK_CONV_ALGO_WINDOW_GATHER, NPLK_CONV_ALGO_WINDOW_PAIR = 3, 4, 5
NPLK_GEMM_TF32_FAST = 1
NPLK_GEMM_SPLIT_OPERANDS = 2
NPLK_GEMM_RAW_OPERANDS = 4
NPLK_GEMM_PEER_TMA_STORES = 8
NPLK_GEMM_MULTIMEM_STORES = 16
NPLK_DEBUG_GEMM, NPLK_DEBUG_CONV_WINDOW = 1, 2
NPLK_STATUS_TIMEOUT_MMA = 102


class NplConfig(C.Structure):
    _fields_ = [
        ("num_threads", C.c_size_t),
        ("enable_fusion", C.c_int),
        ("enable_graph_optimization", C.c_int),
        ("enable_jit", C.c_int),
        ("enable_poly", C.c_int),
        ("enable_vectorization", C.c_int),
        ("enable_numa", C.c_int),
        ("enable_memory_pooling", C.c_int),
        ("workspace_size_mb", C.c_size_t),
        ("verbose", C.c_int),
    ]


class NplTensor(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("ndim", C.c_size_t),
        ("shape", C.c_size_t * NPL_MAX_DIMS),
        ("strides", C.c_size_t * NPL_MAX_DIMS),
        ("dtype", C.c_int),
        ("layout", C.c_int),
        ("size_bytes", C.c_size_t),
        ("is_contiguous", C.c_int),
    ]


class NplPerfStats(C.Structure):
    _fields_ = [
        ("elapsed_ms", C.c_double),
        ("gflops", C.c_double),
        ("bandwidth_gbps", C.c_double),
        ("operations_fused", C.c_size_t),
        ("memory_saved_bytes", C.c_size_t),
        ("backend_used", C.c_char_p),
        ("was_fused", C.c_int),
    ]


class NplConvParams(C.Structure):
    _fields_ = [
        ("kernel_h", C.c_size_t), ("kernel_w", C.c_size_t),
        ("stride_h", C.c_size_t), ("stride_w", C.c_size_t),
        ("pad_h", C.c_size_t), ("pad_w", C.c_size_t),
        ("dilation_h", C.c_size_t), ("dilation_w", C.c_size_t),
        ("groups", C.c_size_t),
        ("padding", C.c_int), ("activation", C.c_int), ("use_bias", C.c_int),
    ]


class NplBatchnormParams(C.Structure):
    _fields_ = [
        ("mean", C.c_void_p), ("variance", C.c_void_p),
        ("gamma", C.c_void_p), ("beta", C.c_void_p),
        ("epsilon", C.c_float), ("training", C.c_int), ("momentum", C.c_float),
    ]


class NplLayernormParams(C.Structure):
    _fields_ = [
        ("gamma", C.c_void_p), ("beta", C.c_void_p),
        ("epsilon", C.c_float), ("normalized_shape", C.c_size_t),
    ]


class NplPoolingParams(C.Structure):
    _fields_ = [
        ("kernel_h", C.c_size_t), ("kernel_w", C.c_size_t),
        ("stride_h", C.c_size_t), ("stride_w", C.c_size_t),
        ("pad_h", C.c_size_t), ("pad_w", C.c_size_t),
        ("type", C.c_int), ("count_include_pad", C.c_int),
    ]


class NplkConvGeom(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "n", "c_in", "h", "w", "c_out", "kh", "kw", "stride_h", "stride_w",
        "pad_top", "pad_left", "dil_h", "dil_w", "h_out", "w_out")]


class NplkTuningStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("entries", "hits", "misses", "tunes", "evictions")]


_P = C.POINTER
_T = _P(NplTensor)
_S = _P(NplPerfStats)

# name -> (restype, argtypes) for the public npl_* ABI
NPL_SIGNATURES = {
    "npl_init": (C.c_int, [_P(NplConfig)]),
    "npl_shutdown": (None, []),
    "npl_is_initialized": (C.c_int, []),
    "npl_get_default_config": (C.c_int, [_P(NplConfig)]),
    "npl_create_tensor": (C.c_int, [C.c_void_p, C.c_size_t, _P(C.c_size_t), C.c_int, C.c_int, _T]),
    "npl_allocate_tensor": (C.c_int, [_T]),
    "npl_free_tensor": (None, [_T]),
    "npl_reshape_tensor": (C.c_int, [_T, C.c_size_t, _P(C.c_size_t), _T]),
    "npl_conv2d": (C.c_int, [_T, _T, _T, _P(NplConvParams), _T, _S]),
    "npl_depthwise_conv2d": (C.c_int, [_T, _T, _T, _P(NplConvParams), _T, _S]),
    "npl_conv2d_bn_activation": (C.c_int, [_T, _T, _T, _P(NplConvParams),
                                           _P(NplBatchnormParams), C.c_int, _T, _S]),
    "npl_activation": (C.c_int, [_T, C.c_int, _T, _S]),
    "npl_relu": (C.c_int, [_T, _T, _S]),
    "npl_leaky_relu": (C.c_int, [_T, C.c_float, _T, _S]),
    "npl_softmax": (C.c_int, [_T, C.c_int, _T, _S]),
    "npl_batch_norm": (C.c_int, [_T, _P(NplBatchnormParams), _T, _S]),
    "npl_layer_norm": (C.c_int, [_T, _P(NplLayernormParams), _T, _S]),
    "npl_pooling": (C.c_int, [_T, _P(NplPoolingParams), _T, _S]),
    "npl_global_avg_pool": (C.c_int, [_T, _T, _S]),
    "npl_matmul": (C.c_int, [_T, _T, _T, C.c_float, C.c_float, _S]),
    "npl_add": (C.c_int, [_T, _T, _T, _S]),
    "npl_mul": (C.c_int, [_T, _T, _T, _S]),
    "npl_conv2d_output_shape": (C.c_int, [_P(C.c_size_t), _P(NplConvParams), _P(C.c_size_t)]),
    "npl_strerror": (C.c_char_p, [C.c_int]),
    "npl_get_system_info": (C.c_char_p, []),
    "npl_self_test": (C.c_int, [C.c_int]),
}

_VP, _F, _I64 = C.c_void_p, C.c_float, C.c_int64
_G = _P(NplkConvGeom)
# device-level nplk_* ABI (include/npl_kernels.h)
NPLK_SIGNATURES = {
    "nplk_gemm_workspace_size": (C.c_size_t, [_I64, _I64, _I64]),
    "nplk_gemm": (C.c_int, [_VP, _I64, _I64, _I64, _F, _VP, _I64, _VP, _I64, _F, _VP, _I64,
                            _VP, C.c_int, _F, C.c_uint, _VP, C.c_size_t, _VP]),
    "nplk_conv_workspace_size": (C.c_size_t, [_G]),
    "nplk_conv_workspace_min_size": (C.c_size_t, [_G]),
    "nplk_conv_workspace_size_algo": (C.c_size_t, [_G, C.c_int]),
    "nplk_conv2d_fused": (C.c_int, [_VP, _G, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _F, C.c_int,
                                    _F, _VP, _VP, C.c_size_t, _VP]),
    "nplk_conv2d_prepare": (C.c_int, [_VP, _G, _VP, _VP, _VP, _VP, _VP, _VP, _F, _VP,
                                      C.c_size_t]),
    "nplk_conv2d_run": (C.c_int, [_VP, _G, _VP, C.c_int, _F, _VP, _VP, C.c_size_t, _VP]),
    "nplk_conv2d_run_algo": (C.c_int, [_VP, _G, _VP, C.c_int, _F, _VP, _VP, C.c_size_t, _VP,
                                        C.c_int]),
    "nplk_conv2d_stage_input": (C.c_int, [_VP, _G, _VP, _VP, C.c_size_t]),
    "nplk_conv2d_run_staged": (C.c_int, [_VP, _G, C.c_int, _F, _VP, _VP, C.c_size_t, _VP]),
    "nplk_conv2d_fused_noalloc": (C.c_int, [_VP, _G, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _F,
                                            C.c_int, _F, _VP, _VP]),
    "nplk_conv2d_maxpool_workspace_size": (C.c_size_t, [_G]),
    "nplk_conv2d_maxpool_fused": (C.c_int, [_VP, _G, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _F,
                                            C.c_int, _F, _VP, _VP, C.c_size_t, _VP]),
    "nplk_depthwise_conv2d": (C.c_int, [_VP, _G, _VP, _VP, _VP, _VP]),
    "nplk_depthwise_bn_act_gap": (C.c_int, [_VP, _G, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _F,
                                            C.c_int, _F, _VP, _VP]),
    "nplk_batch_norm_infer": (C.c_int, [_VP, _I64, _I64, _I64, _VP, _VP, _VP, _VP, _VP, _VP, _F]),
    "nplk_batch_norm_stats": (C.c_int, [_VP, _I64, _I64, _I64, _VP, _VP, _VP]),
    "nplk_bn_update_running": (C.c_int, [_VP, _I64, _VP, _VP, _VP, _VP, _F]),
    "nplk_activation": (C.c_int, [_VP, _I64, _VP, _VP, C.c_int, _F, C.c_int]),
    "nplk_softmax": (C.c_int, [_VP, _I64, _I64, _I64, _VP, _VP]),
    "nplk_layer_norm": (C.c_int, [_VP, _I64, _I64, _VP, _VP, _VP, _VP, _F]),
    "nplk_pool2d": (C.c_int, [_VP] + [_I64] * 12 + [C.c_int, C.c_int, _VP, _VP]),
    "nplk_global_avg_pool": (C.c_int, [_VP, _I64, _I64, _VP, _VP]),
    "nplk_binary": (C.c_int, [_VP, C.c_int, _I64, _VP, _VP, _VP, C.c_int, _I64, _I64]),
    "nplk_colshard_relayout": (C.c_int, [_VP, _I64, _I64, _I64, _VP, _VP]),
    "nplk_ipc_handle_size": (C.c_size_t, []),
    "nplk_ipc_get_handle": (C.c_int, [_VP, _VP, _P(C.c_uint64)]),
    "nplk_ipc_open_handle": (C.c_int, [_VP, C.c_uint64, _P(C.c_void_p)]),
    "nplk_ipc_close_handle": (C.c_int, [_VP, C.c_uint64]),
    "nplk_gemm_allgather": (C.c_int, [_VP, _I64, _I64, _I64, _F, _VP, _I64, _VP, _I64, _VP,
                                      C.c_int, _F, _P(C.c_void_p), C.c_int, _I64, _I64,
                                      C.c_uint, _VP, C.c_size_t, _VP]),
    "nplk_read_status": (C.c_int, [_VP]),
    "nplk_take_launch_count": (C.c_uint64, []),
    "nplk_tuning_cache_load": (C.c_int, [C.c_char_p]),
    "nplk_tuning_cache_save": (C.c_int, [C.c_char_p]),
    "nplk_tuning_cache_clear": (None, []),
    "nplk_tuning_cache_stats": (C.c_int, [_P(NplkTuningStats)]),
    "nplk_tuning_cache_set_max_entries": (C.c_int, [C.c_size_t]),
    "nplk_tuning_key_conv": (C.c_size_t, [_G, C.c_char_p, C.c_size_t]),
    "nplk_tuning_key_gemm": (C.c_size_t, [_I64, _I64, _I64, C.c_char_p, C.c_size_t]),
    "nplk_tuning_cache_put": (C.c_int, [C.c_char_p, C.c_int, _F]),
    "nplk_tuning_cache_get": (C.c_int, [C.c_char_p, _P(C.c_int), _P(C.c_float)]),
    "nplk_conv2d_tune": (C.c_int, [_VP, _G, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _F, C.c_int, _F,
                                   _VP, _VP, C.c_size_t, C.c_int, _P(C.c_int), _P(C.c_float)]),
    "nplk_gemm_tune": (C.c_int, [_VP, _I64, _I64, _I64, _VP, _I64, _VP, _I64, _VP, _I64, _VP,
                                 C.c_size_t, C.c_int, _P(C.c_int), _P(C.c_float)]),
    "nplk_debug_arm_wait_timeout": (C.c_int, [C.c_int, C.c_uint32]),
    "nplk_debug_fail_next_allocations": (C.c_int, [C.c_int]),
}


def bind(lib: C.CDLL, signatures: dict) -> C.CDLL:
    """Sets restype/argtypes on every function of `signatures` the library exports."""
    for name, (res, args) in signatures.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    return lib


_lib: C.CDLL | None = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Opens libnpl_b200.so (built in-tree); raises if it is missing."""
    global _lib
    if path is None and _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python -m npl_b200.build` (needs nvcc); "
            "this package has no CPU fallback")
    lib = C.CDLL(str(p))
    bind(lib, NPL_SIGNATURES)
    bind(lib, NPLK_SIGNATURES)
    if path is None:
        _lib = lib
    return lib


def tensor(lib: C.CDLL, data_ptr: int | None, shape, dtype: int = NPL_DTYPE_FP32,
           layout: int = NPL_LAYOUT_NCHW) -> NplTensor:
    """Creates an npl_tensor_t over `data_ptr` (host or device address) via npl_create_tensor."""
    t = NplTensor()
    arr = (C.c_size_t * len(shape))(*[int(s) for s in shape])
    rc = lib.npl_create_tensor(C.c_void_p(data_ptr) if data_ptr else None, len(shape), arr,
                               dtype, layout, C.byref(t))
    if rc != NPL_OK:
        raise ValueError(f"npl_create_tensor failed: {rc}")
    return t


def conv_params(kh, kw, stride=1, pad=0, dilation=1, groups=1, padding=NPL_PAD_EXPLICIT,
                activation=NPL_ACT_NONE, use_bias=0) -> NplConvParams:
    sh, sw = (stride, stride) if isinstance(stride, int) else stride
    ph, pw = (pad, pad) if isinstance(pad, int) else pad
    dh, dw = (dilation, dilation) if isinstance(dilation, int) else dilation
    return NplConvParams(kh, kw, sh, sw, ph, pw, dh, dw, groups, padding, activation, use_bias)


def conv_geom(n, c, h, w, cout, kh, kw, stride=1, pad=0, dilation=1) -> NplkConvGeom:
    sh, sw = (stride, stride) if isinstance(stride, int) else stride
    ph, pw = (pad, pad) if isinstance(pad, int) else pad
    dh, dw = (dilation, dilation) if isinstance(dilation, int) else dilation
    ho = (h + 2 * ph - (dh * (kh - 1) + 1)) // sh + 1
    wo = (w + 2 * pw - (dw * (kw - 1) + 1)) // sw + 1
    return NplkConvGeom(n, c, h, w, cout, kh, kw, sh, sw, ph, pw, dh, dw, ho, wo)
