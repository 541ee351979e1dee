"""GPU parity of the decode product over the Bonsai 2 pack layout: 2-bit codes with f16 scales
and biases in groups of 128 (the layout of the published pack; the reference runs it
through MLX.quantizedMM, Bonsai2/Qwen38HadamardModules.swift:37-39), bf16 activations.

Reference: the affine rule w = scale * q + bias with the f16 scale and bias of each 128-group,
evaluated in float64 and multiplied by the bf16 activations.  Bar: max |y - ref| <= 2e-2 *
RMS(ref) plus one bf16 step of |ref|, as for the other products.  A width that is not a
multiple of 1024 takes the CUDA-core product and must meet the same bar.
"""
import numpy as np
import pytest
import torch

import oracle as O
from test_qmm_gpu import dev_bf16, dev_u32, host_bf16

pytestmark = pytest.mark.gpu


def pack_case(seed, N, K, ternary=False, biased=True, bits=2):
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 3 if ternary else 2 ** bits, size=(N, K)).astype(np.uint8)
    codes = O.pack(q, bits)
    s = (np.abs(rng.normal(0, 0.02, size=(N, K // 128))) + 1e-3).astype(np.float16)
    if ternary:
        b = (-s).astype(np.float16)
    else:
        b = rng.normal(0, 0.02, size=(N, K // 128)).astype(np.float16) if biased else None
    return q, codes, s, b


def reference(x_bits, q, s, b):
    x = O.bf16_to_f32(x_bits).astype(np.float64)
    g = np.arange(q.shape[1]) // 128
    w = s.astype(np.float64)[:, g] * q.astype(np.float64)
    if b is not None:
        w += b.astype(np.float64)[:, g]
    return x @ w.T


def check(y_bits, ref):
    y = O.bf16_to_f32(y_bits).astype(np.float64)
    rms = np.sqrt((ref ** 2).mean())
    step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -126))) - 7)
    assert np.isfinite(y).all()
    excess = (np.abs(y - ref) - step).max()
    assert excess <= 2e-2 * rms, f"max excess {excess:.4g} > 2e-2 * rms {rms:.4g}"


def run(q38, seed, M, N, K, bits=2, **kw):
    q, codes, s, b = pack_case(seed, N, K, bits=bits, **kw)
    x = O.normal_bf16(seed + 1, (M, K))
    ds = torch.from_numpy(s).cuda()
    db = None if b is None else torch.from_numpy(b).cuda()
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(codes), ds, db, True, 128, bits)
    torch.cuda.synchronize()
    q38.check_device()
    return host_bf16(y), reference(x, q, s, b)


@pytest.mark.parametrize("M", [1, 3, 8, 16])
@pytest.mark.parametrize("NK", [(200, 1024), (1000, 2048), (17408, 5120)])
def test_pack_layout_decode(q38, M, NK):
    y, ref = run(q38, 60 + M, M, *NK)
    check(y, ref)


def test_pack_layout_ternary_and_unbiased(q38):
    y, ref = run(q38, 71, 1, 5120, 17408, ternary=True)
    check(y, ref)
    y, ref = run(q38, 72, 4, 512, 3072, biased=False)
    check(y, ref)


def test_pack_layout_width_outside_the_decode_kernel(q38):
    # K = 1536 is not a multiple of 1024: the CUDA-core product
    y, ref = run(q38, 73, 2, 300, 1536)
    check(y, ref)


def test_bonsai_pack_projection_with_rotation(q38):
    # the full Bonsai 2 projection: rotate (block 1024, signs before), then the product
    M, N, K = 2, 640, 2048
    q, codes, s, b = pack_case(74, N, K, ternary=True)
    x = O.normal_bf16(75, (M, K))
    signs = np.where(np.random.default_rng(76).random(K) < 0.5, -1.0, 1.0).astype(np.float32)
    lin = q38.HadamardQuantizedLinear(
        q38.QuantizedLinear(dev_u32(codes), torch.from_numpy(s).cuda(), torch.from_numpy(b).cuda(), None, 128, 2),
        torch.from_numpy(signs).cuda(), 1024)
    y = lin(dev_bf16(x))
    torch.cuda.synchronize()
    q38.check_device()
    xr = O.hadamard_rotate(x, 1024, signs)
    check(host_bf16(y), reference(xr, q, s, b))


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("M", [64, 300])
@pytest.mark.parametrize("NK", [(1000, 2048), (512, 5120)])
def test_pack_layout_prefill(q38, bits, M, NK):
    # prompt-sized inputs: the tensor-core prefill product with f16 scales loaded per row
    y, ref = run(q38, 80 + M + bits, M, *NK, bits=bits)
    check(y, ref)
