"""GPU test of q38_quantized_matmul_noalloc, the entry point for callers that cannot
allocate device memory where they run a projection (a host that owns all device memory
and passes only input and output buffers, or a decode loop that must not stall on an
allocation).

Each case calls it twice in a row (the second call reuses the fixed scratch array that
the first left behind) and checks both results against the CPU oracle and against the
ordinary q38_quantized_matmul, within the product bar of the other tests.  This file is
collected last so that a run stopping at the first failure has run every other test.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "qwen38-mlx-swift_b200", "libq38.so")
TOL = 2e-2  # max |y - y_ref| <= TOL * RMS(y_ref), as in the other product tests


def _lib():
    lib = C.CDLL(LIB)
    f = lib.q38_quantized_matmul_noalloc
    f.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                  C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    lib.q38_noalloc_check_device.argtypes = [C.c_void_p]
    lib.q38_noalloc_check_device.restype = C.c_int
    return lib


def _dev(a, view):
    return torch.from_numpy(np.ascontiguousarray(a).view(view)).cuda()


def _check(y, ref):
    yf = y.float()
    assert torch.isfinite(yf).all()
    rms = ref.pow(2).mean().sqrt().item()
    err = (yf - ref).abs().max().item()
    assert err <= TOL * rms, f"max err {err} > {TOL} * rms {rms}"


# (16, 32768, 512) fills the whole 2 MiB partial-sum region
@pytest.mark.parametrize("bits,M,N,K,biased,default_stream",
                         [(4, 1, 4096, 4096, True, False), (3, 8, 1000, 2048, True, False),
                          (2, 16, 2048, 5120, True, False), (8, 5, 640, 1536, True, False),
                          (4, 16, 32768, 512, True, False), (3, 4, 768, 1024, False, True)])
def test_noalloc_matches_oracle_and_allocating_entry_point(bits, M, N, K, biased, default_stream):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import q38

    lib = _lib()
    c, s, b = O.quantize(O.normal_f32(9000 + bits + N, (N, K), 0.02), 64, bits)
    if not biased:
        b = None
    x = O.normal_bf16(9100 + M, (M, K))
    ref_cpu = torch.from_numpy(O.qmm(x, c, s, b, 64, bits, f32=True).astype(np.float32)).cuda()
    tx = _dev(x, np.int16).view(torch.bfloat16)
    tc, ts = _dev(c, np.int32), _dev(s, np.int16).view(torch.bfloat16)
    tb = None if b is None else _dev(b, np.int16).view(torch.bfloat16)
    ref_dev = q38.quantized_matmul(tx, tc, ts, tb, True, 64, bits).float()
    torch.cuda.synchronize()
    stream = None if default_stream else torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = lib.q38_quantized_matmul_noalloc(tx.data_ptr(), M, K, tc.data_ptr(), ts.data_ptr(),
                                              None if tb is None else tb.data_ptr(), N, 64, bits, y.data_ptr(),
                                              stream)
        assert st == 0
        assert lib.q38_noalloc_check_device(stream) == 0
        torch.cuda.synchronize()
        _check(y, ref_cpu)
        _check(y, ref_dev)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib()
    z = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = z.data_ptr()
    assert lib.q38_quantized_matmul_noalloc(p, 17, 512, p, p, p, 64, 64, 4, p, None) == 1   # M > 16
    assert lib.q38_quantized_matmul_noalloc(p, 1, 512, p, p, p, 40000, 64, 4, p, None) == 1  # N > 32768
    assert lib.q38_quantized_matmul_noalloc(p, 1, 40960, p, p, p, 64, 64, 4, p, None) == 1  # K > 32768
    assert lib.q38_quantized_matmul_noalloc(p, 1, 500, p, p, p, 64, 64, 4, p, None) == 1    # K % 512
    assert lib.q38_noalloc_check_device(None) == 0
