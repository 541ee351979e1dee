"""CPU tests of the C ABI surface: the library loads, exports every declared entry point,
and rejects bad arguments with status codes (no GPU work is issued)."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "qwen38-mlx-swift_b200", "libq38.so")
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared_symbols():
    names = []
    for h in HEADERS:
        text = open(h).read()
        names += re.findall(r"Q38_API\s+[\w\s\*]+?\b(q38_\w+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        pytest.fail("libq38.so is not built (run __graft_entry__.build())")
    return C.CDLL(LIB)


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("q38_quantized_matmul", "q38_gather_quantized_matmul", "q38_dequantize",
                 "q38_quantize", "q38_unpack_codes", "q38_hadamard_rotate", "q38_moe_route",
                 "q38_moe_route_logits", "q38_moe_sort", "q38_switch_glu"):
        assert must in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_version_and_status_strings(lib):
    lib.q38_version.restype = C.c_int
    assert lib.q38_version() >= 100
    lib.q38_status_string.restype = C.c_char_p
    lib.q38_status_string.argtypes = [C.c_int]
    assert lib.q38_status_string(0) == b"ok"
    assert lib.q38_status_string(1) == b"invalid argument"
    assert lib.q38_status_string(99) == b"unknown status"


def test_null_context_is_rejected(lib):
    f = lib.q38_quantized_matmul
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_void_p,
                  C.c_void_p, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
    assert f(None, None, 1, 64, 0, None, None, None, 0, 8, 1, 64, 4, 0, None) == 1
    lib.q38_ctx_destroy.argtypes = [C.c_void_p]
    lib.q38_ctx_destroy.restype = C.c_int
    assert lib.q38_ctx_destroy(None) == 0


def test_context_creation_without_device_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    lib.q38_ctx_create.argtypes = [C.c_int, C.POINTER(C.c_void_p)]
    lib.q38_ctx_create.restype = C.c_int
    p = C.c_void_p()
    assert lib.q38_ctx_create(0, C.byref(p)) != 0
    assert not p.value


def test_library_has_no_oracle_dependency():
    """The product library must not link or embed the CPU oracle."""
    data = open(LIB, "rb").read()
    assert b"q38o_" not in data
    assert b"libq38_oracle" not in data


def test_comm_unique_id_needs_no_device(lib):
    """Rank 0's rendezvous id comes from NCCL's bootstrap alone (no GPU work)."""
    class Id(C.Structure):
        _fields_ = [("bytes", C.c_ubyte * 128)]
    lib.q38_comm_get_unique_id.argtypes = [C.POINTER(Id)]
    lib.q38_comm_get_unique_id.restype = C.c_int
    a, b = Id(), Id()
    assert lib.q38_comm_get_unique_id(C.byref(a)) == 0
    assert lib.q38_comm_get_unique_id(C.byref(b)) == 0
    assert bytes(a.bytes) != bytes(b.bytes)


def test_comm_init_rejects_bad_arguments(lib):
    class Id(C.Structure):
        _fields_ = [("bytes", C.c_ubyte * 128)]
    f = lib.q38_comm_init_rank
    f.argtypes = [C.POINTER(Id), C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]
    f.restype = C.c_int
    p = C.c_void_p()
    i = Id()
    assert f(C.byref(i), 2, 2, 0, 1000, C.byref(p)) == 1   # rank >= world
    assert f(C.byref(i), 0, 0, 0, 1000, C.byref(p)) == 1   # world < 1
    assert f(C.byref(i), 2, 0, 0, 0, C.byref(p)) == 1      # no timeout
    assert not p.value
