"""The C ABI library loads without a GPU, exports every entry point that
include/ecc_kv_b200.h declares, and rejects bad arguments with the documented
codes before touching the device.  No compute calls."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ecc_kv_b200.h")
LIB = os.path.join(ROOT, "ecc-kv-cache_b200", "custom_ecc_cuda", "libeccb200.so")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ecc_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    assert os.path.exists(LIB), "build libeccb200.so first (__graft_entry__.build())"
    return ctypes.CDLL(LIB)


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("ecc_compress", "ecc_compress_strided", "ecc_decode", "ecc_decode_partials", "ecc_lse_merge",
                 "ecc_hadamard_f16", "ecc_hadamard_f32", "ecc_get_block_metadata", "ecc_strerror"):
        assert must in names


def test_every_declared_symbol_is_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_strerror_and_version(lib):
    lib.ecc_strerror.restype = ctypes.c_char_p
    lib.ecc_strerror.argtypes = [ctypes.c_int]
    assert lib.ecc_strerror(0) == b"ok"
    for code in range(-10, 0):
        assert lib.ecc_strerror(code) not in (b"ok", b"unknown error")
    assert lib.ecc_version() == 100


def test_argument_validation_before_any_device_call(lib):
    p = ctypes.c_void_p
    lib.ecc_compress.argtypes = [p, p, ctypes.c_int64, ctypes.c_int, p]
    assert lib.ecc_compress(None, None, 0, 1, None) == 0          # nothing to do
    assert lib.ecc_compress(None, None, 4, 1, None) == -1         # NULL
    assert lib.ecc_compress(p(16), p(128), -1, 1, None) == -2      # bad n
    assert lib.ecc_compress(p(17), p(128), 4, 1, None) == -3       # misaligned input
    assert lib.ecc_compress(p(16), p(64), 4, 1, None) == -3        # blocks not 128-aligned
    lib.ecc_hadamard_f16.argtypes = [p, ctypes.c_int64, ctypes.c_int, p]
    assert lib.ecc_hadamard_f16(p(16), 4, 100, None) == -2         # not a power of two
    assert lib.ecc_hadamard_f16(p(16), 4, 2048, None) == -2        # > 1024
    i32, i64, f32, sz = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    lib.ecc_decode.argtypes = [p, p, p, i64, i64, p, p, sz, i32, i32, i32, i64, f32, i32, i32, p]
    assert lib.ecc_decode(None, p(128), p(128), 0, 0, p(16), p(256), 1 << 20, 1, 4, 2, 8, 0.0, 0, 0, None) == -1
    assert lib.ecc_decode(p(16), p(128), p(128), 0, 0, p(16), p(256), 1 << 20, 1, 6, 4, 8, 0.0, 0, 0, None) == -4
    assert lib.ecc_decode(p(16), p(128), p(128), 0, 0, p(16), None, 0, 1, 4, 2, 8, 0.0, 0, 0, None) == -5
    lib.ecc_lse_merge.argtypes = [p, p, p, i64, i32, p, i32, p]
    assert lib.ecc_lse_merge(p(16), p(16), p(16), 4, 0, p(16), 0, None) == -2
    lib.ecc_lse_merge_to_record.argtypes = [p, p, p, i64, i32, p, p]
    assert lib.ecc_lse_merge_to_record(p(16), p(16), p(16), 4, 0, p(16), None) == -2
    assert lib.ecc_lse_merge_to_record(p(16), p(16), p(16), 4, 3, None, None) == -1
    lib.ecc_lse_merge_records.argtypes = [p, i64, i32, i64, p, i32, p]
    assert lib.ecc_lse_merge_records(p(16), 4, 0, 520, p(16), 0, None) == -2
    assert lib.ecc_lse_merge_records(None, 4, 2, 520, p(16), 0, None) == -1
    assert lib.ecc_lse_merge_records(p(16), 4, 2, 100, p(16), 0, None) == -2  # overlapping record sets


@pytest.mark.skipif(torch.cuda.is_available(), reason="only meaningful on a host without a GPU")
def test_no_cpu_fallback(lib):
    """With valid arguments but no device, compute entry points report
    ECC_ERR_DEVICE instead of computing anything on the CPU."""
    p = ctypes.c_void_p
    lib.ecc_compress.argtypes = [p, p, ctypes.c_int64, ctypes.c_int, p]
    buf_in = (ctypes.c_uint8 * (4 * 256 + 16))()
    buf_out = (ctypes.c_uint8 * (4 * 128 + 128))()
    a = (ctypes.addressof(buf_in) + 15) // 16 * 16
    b = (ctypes.addressof(buf_out) + 127) // 128 * 128
    assert lib.ecc_compress(p(a), p(b), 4, 1, None) == -8
    assert bytes(buf_out) == bytes(len(buf_out))


def test_workspace_size_is_host_only(lib):
    lib.ecc_decode_workspace_size.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int]
    lib.ecc_decode_workspace_size.restype = ctypes.c_size_t
    # explicit split count: (2 + 128) floats per (b, q head, split) + alignment slack
    assert lib.ecc_decode_workspace_size(2, 8, 2, 4096, 4) == 2 * 8 * 4 * 130 * 4 + 256
    assert lib.ecc_decode_workspace_size(0, 8, 2, 4096, 4) == 0


def test_calibrated_compress_rejects_bad_parameters(lib):
    p, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    fn = lib.ecc_compress_strided_calibrated
    fn.argtypes = [p, i64, i64, i64, p, i64, i64, i32, i32, i64, i32, f32, f32, f32, p]
    fn.restype = i32
    args = (p(16), 0, 0, 128, p(128), 0, 0, 1, 1, 4, 1)
    assert fn(*args, 0.0, 0.0, 0.1, None) == -10            # scale <= 0
    assert fn(*args, -1.0, 0.0, 0.1, None) == -10
    assert fn(*args, float("nan"), 0.0, 0.1, None) == -10
    assert fn(*args, 1.0, float("inf"), 0.1, None) == -10   # zero not finite
    assert fn(*args, 1.0, 0.0, float("nan"), None) == -10   # alpha not finite
    assert fn(None, 0, 0, 128, None, 0, 0, 1, 1, 4, 1, 1.0, 0.0, 0.1, None) == -1  # NULL, checked before the device
