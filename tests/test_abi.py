"""ABI and host-side behaviour of libnpl_b200.so that needs no GPU: every symbol
declared in include/*.h is exported, struct layouts match the reference's Java
FFM bindings (ffm_api/jcorex/.../Tensors.java:24-45, Config.java:19-31), and
the pure host functions behave like the reference's. No compute calls."""
import ctypes as C
import re
import subprocess

import pytest

import support as S
from support import nb


def declared(header):
    text = (S.REPO / "include" / header).read_text()
    return sorted(set(re.findall(r"NPL_API\s+[\w\s\*]*?\b(npl\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return nb.load()


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(nb.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    names = declared("neural_primitives.h") + declared("npl_kernels.h")
    assert len(declared("neural_primitives.h")) == 26
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert getattr(lib, n) is not None


def test_reference_abi_covered():
    # Every npl_* entry point of the reference header is exported (the
    # reference itself defines NPL_strerror instead of the declared name).
    ref_hdr = declared("neural_primitives.h")
    for name in ["npl_init", "npl_shutdown", "npl_is_initialized", "npl_get_default_config",
                 "npl_create_tensor", "npl_allocate_tensor", "npl_free_tensor",
                 "npl_reshape_tensor", "npl_conv2d", "npl_depthwise_conv2d",
                 "npl_conv2d_bn_activation", "npl_activation", "npl_relu", "npl_leaky_relu",
                 "npl_softmax", "npl_batch_norm", "npl_layer_norm", "npl_pooling",
                 "npl_global_avg_pool", "npl_matmul", "npl_add", "npl_mul",
                 "npl_conv2d_output_shape", "npl_strerror", "npl_get_system_info",
                 "npl_self_test"]:
        assert name in ref_hdr


def test_struct_layouts_match_java_ffm():
    assert C.sizeof(nb.NplTensor) == 168
    offs = {f: getattr(nb.NplTensor, f).offset for f, _ in nb.NplTensor._fields_}
    assert offs == {"data": 0, "ndim": 8, "shape": 16, "strides": 80, "dtype": 144,
                    "layout": 148, "size_bytes": 152, "is_contiguous": 160}
    assert C.sizeof(nb.NplConfig) == 56
    assert nb.NplConfig.workspace_size_mb.offset == 40 and nb.NplConfig.verbose.offset == 48
    assert C.sizeof(nb.NplPerfStats) == 56
    assert nb.NplPerfStats.backend_used.offset == 40 and nb.NplPerfStats.was_fused.offset == 48


def test_create_and_reshape_tensor(lib):
    t = nb.tensor(lib, None, [2, 3, 4, 4])
    assert t.ndim == 4 and list(t.shape[:4]) == [2, 3, 4, 4]
    assert list(t.strides[:4]) == [48, 16, 4, 1]
    assert t.size_bytes == 2 * 3 * 4 * 4 * 4 and t.is_contiguous == 1
    out = nb.NplTensor()
    shape = (C.c_size_t * 2)(6, 16)
    assert lib.npl_reshape_tensor(C.byref(t), 2, shape, C.byref(out)) == nb.NPL_OK
    assert list(out.strides[:2]) == [16, 1]
    bad = (C.c_size_t * 2)(5, 16)
    assert lib.npl_reshape_tensor(C.byref(t), 2, bad, C.byref(out)) == nb.NPL_ERR_SHAPE_MISMATCH
    shp = (C.c_size_t * 9)(*([1] * 9))
    assert lib.npl_create_tensor(None, 0, shp, 0, 0, C.byref(out)) == nb.NPL_ERR_INVALID_ARG
    assert lib.npl_create_tensor(None, 9, shp, 0, 0, C.byref(out)) == nb.NPL_ERR_INVALID_ARG
    assert lib.npl_create_tensor(None, 2, shp, 0, 0, None) == nb.NPL_ERR_INVALID_ARG
    half = nb.tensor(lib, None, [3, 5], nb.NPL_DTYPE_BF16)
    assert half.size_bytes == 30


def test_default_config_and_strerror(lib):
    cfg = nb.NplConfig()
    assert lib.npl_get_default_config(C.byref(cfg)) == nb.NPL_OK
    assert (cfg.num_threads, cfg.enable_fusion, cfg.enable_vectorization,
            cfg.workspace_size_mb, cfg.verbose) == (0, 1, 1, 256, 0)
    assert lib.npl_get_default_config(None) == nb.NPL_ERR_INVALID_ARG
    assert lib.npl_strerror(0) == b"Success"
    assert lib.npl_strerror(-6) == b"Tensor shape mismatch"
    assert lib.npl_strerror(-7) == b"Out of memory during execution"
    assert lib.npl_strerror(42) == b"Unknown error"


def test_conv_output_shape(lib):
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_EXPLICIT)
    inp = (C.c_size_t * 4)(32, 64, 56, 56)
    out = (C.c_size_t * 4)()
    assert lib.npl_conv2d_output_shape(inp, C.byref(p), out) == 0
    assert list(out) == [32, 64, 56, 56]  # channel slot copied from the input
    p = nb.conv_params(7, 7, 2, 3, padding=nb.NPL_PAD_EXPLICIT)
    inp = (C.c_size_t * 4)(128, 3, 224, 224)
    assert lib.npl_conv2d_output_shape(inp, C.byref(p), out) == 0
    assert list(out)[2:] == [112, 112]
    p = nb.conv_params(3, 3, 2, 5, padding=nb.NPL_PAD_SAME)
    assert lib.npl_conv2d_output_shape(inp, C.byref(p), out) == 0
    assert list(out)[2:] == [112, 112]
    p = nb.conv_params(3, 3, 1, 1, padding=nb.NPL_PAD_VALID)  # pads ignored here
    assert lib.npl_conv2d_output_shape(inp, C.byref(p), out) == 0
    assert list(out)[2:] == [222, 222]


def test_ops_before_init_report_not_initialized(lib):
    if lib.npl_is_initialized():
        pytest.skip("library already initialised in this process")
    t = nb.tensor(lib, None, [4])
    assert lib.npl_relu(C.byref(t), C.byref(t), None) == nb.NPL_ERR_NOT_INITIALIZED
    assert lib.npl_matmul(C.byref(t), C.byref(t), C.byref(t), 1.0, 0.0, None) == \
        nb.NPL_ERR_NOT_INITIALIZED
    assert lib.npl_get_system_info() == b"JCore Neural Primitives Layer: Not initialized"
    assert lib.npl_self_test(0) == nb.NPL_ERR_NOT_INITIALIZED


def test_kernel_abi_argument_checks(lib):
    # Argument validation happens before any device work.
    assert lib.nplk_gemm_workspace_size(0, 4, 4) == 0
    assert lib.nplk_gemm(None, 0, 4, 4, 1.0, None, 4, None, 4, 0.0, None, 4, None, 0, 0.0, 0,
                         None, 0, None) == nb.NPL_ERR_INVALID_ARG
    g = nb.conv_geom(1, 3, 8, 8, 2, 3, 3)
    g.stride_h = 0
    assert lib.nplk_conv_workspace_size(C.byref(g)) == 0
    assert lib.nplk_softmax(None, 0, 4, 1, None, None) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_pool2d(None, 1, 1, 4, 4, 2, 2, 2, 2, 0, 0, 2, 2, 5, 0, None, None) == \
        nb.NPL_ERR_INVALID_ARG
    # fused depthwise -> BN -> activation -> average pool: missing tensors, a
    # c_out that differs from c_in, an unknown activation
    gd = nb.conv_geom(2, 4, 8, 8, 4, 3, 3, 1, 1)
    fake = C.c_void_p(256)  # never dereferenced: the checks come first
    assert lib.nplk_depthwise_bn_act_gap(None, C.byref(gd), None, fake, None, fake, fake, None,
                                         None, 1e-5, 1, 0.0, None, fake) == nb.NPL_ERR_INVALID_ARG
    gbad = nb.conv_geom(2, 4, 8, 8, 5, 3, 3, 1, 1)
    assert lib.nplk_depthwise_bn_act_gap(None, C.byref(gbad), fake, fake, None, fake, fake,
                                         None, None, 1e-5, 1, 0.0, None, fake) == \
        nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_depthwise_bn_act_gap(None, C.byref(gd), fake, fake, None, fake, fake, None,
                                         None, 1e-5, 11, 0.0, None, fake) == nb.NPL_ERR_INVALID_ARG
    # planes the one-pass form does not take (output plane of 7x7 = 49, not a
    # multiple of 4) are refused before any device work
    g7 = nb.conv_geom(2, 4, 7, 7, 4, 3, 3, 1, 1)
    assert lib.nplk_depthwise_bn_act_gap(None, C.byref(g7), fake, fake, None, fake, fake, None,
                                         None, 1e-5, 1, 0.0, None, fake) == nb.NPL_ERR_UNSUPPORTED


def test_multi_gpu_entry_points_argument_checks(lib):
    # The fused GEMM all-gather and the IPC calls reject bad arguments before
    # any device work.
    assert lib.nplk_ipc_handle_size() == 64  # cudaIpcMemHandle_t
    h = (C.c_uint8 * 64)()
    off = C.c_uint64(0)
    p = C.c_void_p()
    assert lib.nplk_ipc_get_handle(None, h, C.byref(off)) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_ipc_get_handle(C.c_void_p(0x1000), None, C.byref(off)) == \
        nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_ipc_get_handle(C.c_void_p(0x1000), h, None) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_ipc_open_handle(None, 0, C.byref(p)) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_ipc_open_handle(h, 0, None) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_ipc_close_handle(None, 0) == nb.NPL_ERR_INVALID_ARG

    fake = C.c_void_p(0x1000)  # never dereferenced: every call below fails its checks

    def allgather(dst, n_dst, col_offset, ldc, n_local=64, flags=0):
        return lib.nplk_gemm_allgather(None, 128, n_local, 64, 1.0, fake, 64, fake, 128, None, 0,
                                       0.0, dst, n_dst, col_offset, ldc, flags, None, 0, None)

    two = (C.c_void_p * 2)(0x1000, 0x2000)
    nine = (C.c_void_p * 9)(*([0x1000] * 9))
    with_null = (C.c_void_p * 2)(0x1000, None)
    assert allgather(None, 2, 0, 128) == nb.NPL_ERR_INVALID_ARG          # no destinations
    assert allgather(two, 0, 0, 128) == nb.NPL_ERR_INVALID_ARG           # n_dst < 1
    assert allgather(nine, 9, 0, 128) == nb.NPL_ERR_INVALID_ARG          # n_dst > 8
    assert allgather(two, 2, -4, 128) == nb.NPL_ERR_INVALID_ARG          # negative column
    assert allgather(two, 2, 96, 128) == nb.NPL_ERR_INVALID_ARG          # block past ldc
    assert allgather(with_null, 2, 0, 128) == nb.NPL_ERR_INVALID_ARG     # a null destination
    # The multicast form: exactly one 16-byte aligned destination, whole
    # 16-byte pieces (ldc, N_local, col_offset multiples of 4), no TMA stores.
    mm = nb.NPLK_GEMM_MULTIMEM_STORES
    one = (C.c_void_p * 1)(0x1000)
    odd = (C.c_void_p * 1)(0x1004)
    assert allgather(two, 2, 0, 128, flags=mm) == nb.NPL_ERR_INVALID_ARG
    assert allgather(odd, 1, 0, 128, flags=mm) == nb.NPL_ERR_INVALID_ARG
    assert allgather(one, 1, 2, 128, flags=mm) == nb.NPL_ERR_INVALID_ARG
    assert allgather(one, 1, 0, 130, flags=mm) == nb.NPL_ERR_INVALID_ARG
    assert allgather(one, 1, 0, 128, n_local=62, flags=mm) == nb.NPL_ERR_INVALID_ARG
    assert allgather(one, 1, 0, 128, flags=mm | nb.NPLK_GEMM_PEER_TMA_STORES) == \
        nb.NPL_ERR_INVALID_ARG


def test_fault_injection_hooks_arm_and_disarm(lib):
    # Arming touches no device: unknown kernel families and limits above a
    # minute are rejected; 0 disarms. The allocation hook returns the count
    # that was still armed.
    assert lib.nplk_debug_arm_wait_timeout(0, 1000) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_debug_arm_wait_timeout(3, 1000) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_debug_arm_wait_timeout(nb.NPLK_DEBUG_GEMM, 60_000_001) == \
        nb.NPL_ERR_INVALID_ARG
    for which in (nb.NPLK_DEBUG_GEMM, nb.NPLK_DEBUG_CONV_WINDOW):
        assert lib.nplk_debug_arm_wait_timeout(which, 1000) == 0
        assert lib.nplk_debug_arm_wait_timeout(which, 0) == 0
    assert lib.nplk_debug_fail_next_allocations(2) == 0
    assert lib.nplk_debug_fail_next_allocations(-5) == 2
    assert lib.nplk_debug_fail_next_allocations(0) == 0
