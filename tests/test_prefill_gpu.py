"""GPU parity of the prompt-sized product (M > 16 tokens, tensor-core path) against the
CPU oracle, through libq38.so's C ABI.

Bar: max|y - y_oracle| <= 2e-2 * RMS(y_oracle), fp32 accumulation on both sides.  The
weights are dequantized to bf16 with one rounding before the tensor-core product, the
oracle keeps them in fp32; the difference (<= 2^-9 relative per weight) is far inside
the bar.  At the full prompt sizes the oracle checks a sample of tokens: a product's
token rows are independent, so the sample's rows of the full product must equal the
oracle's product of the sampled tokens alone.
"""
import numpy as np
import pytest
import torch

import oracle as O
from test_qmm_gpu import check_close, dev_bf16, dev_u32, host_bf16, make_weight

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("M,N,K", [(17, 128, 512), (64, 200, 1024), (128, 256, 512), (200, 1000, 2048),
                                   (333, 384, 1536), (300, 512, 2176), (96, 640, 1152), (257, 264, 128)])
def test_prefill_parity(q38, bits, M, N, K):
    c, s, b = make_weight(5000 + bits + N, N, K, bits)
    x = O.normal_bf16(5100 + M, (M, K))
    ref = O.qmm(x, c, s, b, 64, bits, f32=True)
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 64, bits)
    torch.cuda.synchronize()
    check_close(host_bf16(y), ref)
    q38.check_device()


@pytest.mark.parametrize("bits", [4, 2])
def test_prefill_without_biases(q38, bits):
    N, K, M = 300, 1024, 96
    c, s, _ = make_weight(5200, N, K, bits)
    x = O.normal_bf16(5201, (M, K))
    ref = O.qmm(x, c, s, None, 64, bits, f32=True)
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), None, True, 64, bits)
    check_close(host_bf16(y), ref)


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("M,N,K", [(4096, 17408, 5120), (2048, 5120, 17408)])
def test_prefill_full_size_sampled_tokens(q38, bits, M, N, K):
    """The prompt sweep's full shapes; 6 sampled tokens (first, last and four inside,
    including both sides of a 128-token tile boundary) checked against the oracle."""
    c, s, b = make_weight(5300 + bits + N, N, K, bits)
    x = O.normal_bf16(5301 + M, (M, K))
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    rows = np.array([0, 127, 128, M // 2 + 5, M - 129, M - 1])
    ref = O.qmm(np.ascontiguousarray(x[rows]), c, s, b, 64, bits, f32=True)
    check_close(host_bf16(y[torch.from_numpy(rows).cuda()]), ref)


def test_prefill_repeat_is_deterministic(q38):
    """Each output element is accumulated by one CTA in a fixed order: repeats are bitwise equal."""
    c, s, b = make_weight(5400, 512, 2048, 4)
    x = dev_bf16(O.normal_bf16(5401, (300, 2048)))
    W = [dev_u32(c), dev_bf16(s), dev_bf16(b)]
    y1 = q38.quantized_matmul(x, *W, True, 64, 4)
    y2 = q38.quantized_matmul(x, *W, True, 64, 4)
    assert torch.equal(y1, y2)


def test_prefill_then_decode_share_the_context(q38):
    """Alternating prompt and decode products on one context (shared scratch workspace)."""
    c, s, b = make_weight(5500, 640, 1024, 4)
    W = [dev_u32(c), dev_bf16(s), dev_bf16(b)]
    xp = O.normal_bf16(5501, (100, 1024))
    xd = O.normal_bf16(5502, (4, 1024))
    yp = q38.quantized_matmul(dev_bf16(xp), *W, True, 64, 4)
    yd = q38.quantized_matmul(dev_bf16(xd), *W, True, 64, 4)
    yp2 = q38.quantized_matmul(dev_bf16(xp), *W, True, 64, 4)
    check_close(host_bf16(yp), O.qmm(xp, c, s, b, 64, 4, f32=True))
    check_close(host_bf16(yd), O.qmm(xd, c, s, b, 64, 4, f32=True))
    assert torch.equal(yp, yp2)
