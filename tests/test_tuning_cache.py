"""The tile-configuration cache (replacing the reference's tuning result
cache, composite/tuning_rCache/src/tuning_cache.cpp:186-506) on the host: keys,
put/get, hit and miss counting, the entry limit with oldest-first eviction,
save/load round trips, and rejection of files from another format version or
another device (the reference's ERR_VERSION_MISMATCH / ERR_HARDWARE_MISMATCH).
No compute calls."""
import ctypes as C

import pytest

import support as S
from support import nb


@pytest.fixture()
def lib():
    lib = nb.load()
    lib.nplk_tuning_cache_clear()
    lib.nplk_tuning_cache_set_max_entries(0)
    yield lib
    lib.nplk_tuning_cache_clear()
    lib.nplk_tuning_cache_set_max_entries(0)


def key_conv(lib, g):
    buf = C.create_string_buffer(256)
    n = lib.nplk_tuning_key_conv(C.byref(g), buf, 256)
    assert n == len(buf.value)
    return buf.value


def key_gemm(lib, m, n, k):
    buf = C.create_string_buffer(256)
    lib.nplk_tuning_key_gemm(m, n, k, buf, 256)
    return buf.value


def stats(lib):
    st = nb.NplkTuningStats()
    assert lib.nplk_tuning_cache_stats(C.byref(st)) == 0
    return st


def test_keys_name_the_shape_and_the_sm_count(lib):
    g = nb.conv_geom(32, 64, 56, 56, 64, 3, 3, 1, 1)
    k = key_conv(lib, g)
    assert k.startswith(b"conv n=32 c=64 h=56 w=56 co=64 k=3x3 s=1x1 p=1x1 d=1x1 o=56x56 sm=")
    assert key_gemm(lib, 1024, 2048, 512).startswith(b"gemm m=1024 n=2048 k=512 sm=")
    g2 = nb.conv_geom(32, 64, 56, 56, 64, 3, 3, 2, 1)
    assert key_conv(lib, g2) != k
    short = C.create_string_buffer(8)
    assert lib.nplk_tuning_key_gemm(1, 2, 3, short, 8) > 7 and len(short.value) == 7


def test_put_get_and_entry_limit(lib):
    choice, us = C.c_int(), C.c_float()
    assert lib.nplk_tuning_cache_get(b"gemm m=1 n=1 k=1 sm=148", C.byref(choice), None) == 0
    for i in range(5):
        assert lib.nplk_tuning_cache_put(b"gemm m=%d n=1 k=1 sm=148" % i, 64, 10.0 + i) == 0
    assert stats(lib).entries == 5
    assert lib.nplk_tuning_cache_get(b"gemm m=3 n=1 k=1 sm=148", C.byref(choice),
                                     C.byref(us)) == 1
    assert choice.value == 64 and abs(us.value - 13.0) < 1e-6
    assert lib.nplk_tuning_cache_put(b"gemm m=3 n=1 k=1 sm=148", 128, 9.0) == 0  # replace
    assert lib.nplk_tuning_cache_get(b"gemm m=3 n=1 k=1 sm=148", C.byref(choice), None) == 1
    assert choice.value == 128
    lib.nplk_tuning_cache_set_max_entries(3)  # evicts the two oldest inserted: m=0, m=1
    st = stats(lib)
    assert st.entries == 3 and st.evictions == 2
    assert lib.nplk_tuning_cache_get(b"gemm m=0 n=1 k=1 sm=148", None, None) == 0
    assert lib.nplk_tuning_cache_get(b"gemm m=1 n=1 k=1 sm=148", None, None) == 0
    assert lib.nplk_tuning_cache_get(b"gemm m=3 n=1 k=1 sm=148", None, None) == 1
    assert lib.nplk_tuning_cache_put(b"bad\tkey", 1, 1.0) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_tuning_cache_put(b"", 1, 1.0) == nb.NPL_ERR_INVALID_ARG


def test_save_load_round_trip_and_mismatches(lib, tmp_path):
    path = tmp_path / "tiles.cache"
    g = nb.conv_geom(8, 64, 28, 28, 64, 3, 3, 1, 1)
    kc, kg = key_conv(lib, g), key_gemm(lib, 1024, 1024, 1024)
    assert lib.nplk_tuning_cache_put(kc, nb.NPLK_CONV_ALGO_WINDOW_GATHER, 12.5) == 0
    assert lib.nplk_tuning_cache_put(kg, 64, 30.0) == 0
    assert lib.nplk_tuning_cache_save(str(path).encode()) == 2
    lines = path.read_text().splitlines()
    assert lines[0] == "npl_b200-tuning-cache 1" and lines[1].startswith("hardware ")
    assert len(lines) == 4 and all("\t" in ln for ln in lines[2:])
    lib.nplk_tuning_cache_clear()
    assert stats(lib).entries == 0
    assert lib.nplk_tuning_cache_load(str(path).encode()) == 2
    choice = C.c_int()
    assert lib.nplk_tuning_cache_get(kc, C.byref(choice), None) == 1
    assert choice.value == nb.NPLK_CONV_ALGO_WINDOW_GATHER
    # another format version: rejected, nothing loaded
    lib.nplk_tuning_cache_clear()
    other = tmp_path / "v2.cache"
    other.write_text("\n".join(["npl_b200-tuning-cache 2"] + lines[1:]) + "\n")
    assert lib.nplk_tuning_cache_load(str(other).encode()) == nb.NPL_ERR_UNSUPPORTED
    # another device: rejected, nothing loaded
    dev = tmp_path / "dev.cache"
    dev.write_text("\n".join([lines[0], "hardware Some Other GPU|cc=9.0|sm=132|l2=1"] +
                             lines[2:]) + "\n")
    assert lib.nplk_tuning_cache_load(str(dev).encode()) == nb.NPL_ERR_UNSUPPORTED
    assert stats(lib).entries == 0
    # malformed files and missing paths
    bad = tmp_path / "bad.cache"
    bad.write_text("not a cache\n")
    assert lib.nplk_tuning_cache_load(str(bad).encode()) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_tuning_cache_load(str(tmp_path / "absent").encode()) == \
        nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_tuning_cache_load(None) == nb.NPL_ERR_INVALID_ARG


def test_tune_entry_points_check_arguments(lib):
    best, us = C.c_int(), C.c_float()
    fake = C.c_void_p(0x1000)  # never dereferenced: every call fails its checks
    g = nb.conv_geom(1, 32, 8, 8, 32, 3, 3, 1, 1)
    assert lib.nplk_conv2d_tune(None, C.byref(g), None, fake, None, None, None, None, None, 1e-5,
                                0, 0.0, fake, fake, 1 << 20, 3, C.byref(best), None) == \
        nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_conv2d_tune(None, C.byref(g), fake, fake, None, None, None, None, None, 1e-5,
                                0, 0.0, fake, fake, 1 << 20, 0, C.byref(best), None) == \
        nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_gemm_tune(None, 0, 4, 4, fake, 4, fake, 4, fake, 4, fake, 1 << 20, 3,
                              C.byref(best), C.byref(us)) == nb.NPL_ERR_INVALID_ARG
    assert lib.nplk_gemm_tune(None, 4, 4, 4, fake, 4, fake, 4, None, 4, fake, 1 << 20, 3,
                              C.byref(best), C.byref(us)) == nb.NPL_ERR_INVALID_ARG
