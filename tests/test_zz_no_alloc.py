"""GPU test of q38_quantized_matmul_noalloc, the entry point for callers that cannot
allocate device memory (a host that owns all device memory and passes only input and
output buffers, or a decode loop that must not stall on an allocation).

It is compared with the ordinary q38_quantized_matmul on the same inputs, twice in a
row (the second call reuses the fixed scratch array left by the first).  This file is
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
    return lib


def _dev(a, view):
    return torch.from_numpy(np.ascontiguousarray(a).view(view)).cuda()


@pytest.mark.parametrize("bits,M,N,K", [(4, 1, 4096, 4096), (3, 8, 1000, 2048), (2, 16, 2048, 5120),
                                        (8, 5, 640, 1536)])
def test_noalloc_matches_allocating_entry_point(bits, M, N, K):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import q38

    lib = _lib()
    c, s, b = O.quantize(O.normal_f32(9000 + bits, (N, K), 0.02), 64, bits)
    x = O.normal_bf16(9100 + M, (M, K))
    tx = _dev(x, np.int16).view(torch.bfloat16)
    tc, ts, tb = _dev(c, np.int32), _dev(s, np.int16).view(torch.bfloat16), _dev(b, np.int16).view(torch.bfloat16)
    ref = q38.quantized_matmul(tx, tc, ts, tb, True, 64, bits).float()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = lib.q38_quantized_matmul_noalloc(tx.data_ptr(), M, K, tc.data_ptr(), ts.data_ptr(), tb.data_ptr(),
                                              N, 64, bits, y.data_ptr(), stream)
        assert st == 0
        torch.cuda.synchronize()
        yf = y.float()
        assert torch.isfinite(yf).all()
        rms = ref.pow(2).mean().sqrt().item()
        err = (yf - ref).abs().max().item()
        assert err <= TOL * rms, f"max err {err} > {TOL} * rms {rms}"


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
