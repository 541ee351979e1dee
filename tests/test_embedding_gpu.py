"""GPU parity of the quantized embedding (Qwen4ExpPrequantizedEmbedding) and of its tied
output projection at vocabulary size.

Bars: each looked-up row equals the oracle's dequantization of that table row bit for bit
(same fp32 multiply-add, one rounding to the output dtype); an out-of-range id yields a
zero row and is reported by check_device; the output projection over 248,320 rows is
within 2e-2 * RMS of the oracle on sampled rows (fp32 accumulation on both sides).
"""
import numpy as np
import pytest
import torch

import oracle as O
from test_qmm_gpu import dev_bf16, dev_u32, host_bf16, make_weight

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_embedding_rows_bit_exact(q38, bits):
    rows, K = 300, 1024
    c, s, b = make_weight(800 + bits, rows, K, bits)
    ids = np.random.default_rng(bits).integers(0, rows, size=(3, 17)).astype(np.int32)
    emb = q38.QuantizedEmbedding(dev_u32(c), dev_bf16(s), dev_bf16(b), 64, bits)
    out = emb(torch.from_numpy(ids).cuda())
    torch.cuda.synchronize()
    assert out.shape == (3, 17, K) and out.dtype == torch.bfloat16
    table = O.dequantize(c, s, b, 64, bits)  # fp32 [rows, K]
    np.testing.assert_array_equal(host_bf16(out).reshape(-1, K), O.f32_to_bf16(table[ids.reshape(-1)]))


def test_embedding_f32_output_and_no_biases(q38):
    rows, K, bits = 64, 512, 4
    c, s, _ = make_weight(901, rows, K, bits)
    ids = np.array([5, 0, 63, 5], np.int32)
    out = q38.quantized_embedding(torch.from_numpy(ids).cuda(), dev_u32(c), dev_bf16(s), None, 64, bits,
                                  out_dtype=torch.float32)
    torch.cuda.synchronize()
    table = O.dequantize(c, s, None, 64, bits)  # fp32 [rows, K]
    np.testing.assert_array_equal(out.cpu().numpy(), table[ids])


def test_embedding_out_of_range_id(q38):
    rows, K, bits = 32, 256, 4
    c, s, b = make_weight(902, rows, K, bits)
    ids = torch.tensor([1, rows, 2], dtype=torch.int32, device="cuda")
    out = q38.quantized_embedding(ids, dev_u32(c), dev_bf16(s), dev_bf16(b), 64, bits)
    with pytest.raises(q38.Q38Error):
        q38.check_device()
    assert torch.count_nonzero(out[1]).item() == 0
    table = O.dequantize(c, s, b, 64, bits)
    np.testing.assert_array_equal(host_bf16(out)[[0, 2]], O.f32_to_bf16(table[[1, 2]]))


def test_tied_output_projection_vocabulary_size(q38):
    # lm_head of a 248,320-token vocabulary through the decode product; rows sampled
    rows, K, bits = 248320, 5120, 4
    g = torch.Generator(device="cuda").manual_seed(903)
    c = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows, K * bits // 32), dtype=torch.int32, device="cuda", generator=g)
    s = (torch.rand((rows, K // 64), device="cuda", generator=g) * 0.01).to(torch.bfloat16)
    b = ((torch.rand((rows, K // 64), device="cuda", generator=g) - 0.5) * 0.02).to(torch.bfloat16)
    emb = q38.QuantizedEmbedding(c, s, b, 64, bits)
    x = O.normal_bf16(904, (1, K))
    y = emb.as_linear(dev_bf16(x))
    torch.cuda.synchronize()
    q38.check_device()
    pick = np.sort(np.random.default_rng(905).choice(rows, 96, replace=False))
    idx = torch.from_numpy(pick).cuda()
    cs = c[idx].cpu().numpy().view(np.uint32)
    ss = s[idx].view(torch.int16).cpu().numpy().view(np.uint16)
    bs = b[idx].view(torch.int16).cpu().numpy().view(np.uint16)
    ref = O.qmm(x, cs, ss, bs, 64, bits, f32=True)
    got = O.bf16_to_f32(host_bf16(y)[:, pick]).astype(np.float64)
    full_rms = float(y.float().pow(2).mean().sqrt())
    assert np.abs(got - ref).max() <= 2e-2 * full_rms
