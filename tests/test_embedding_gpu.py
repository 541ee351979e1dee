"""GPU parity of the quantized embedding (Qwen4ExpPrequantizedEmbedding), of its tied
output projection at vocabulary size, and of the rotated Bonsai 2 embedding
(Qwen38HadamardQuantizedEmbedding).

Bars: each looked-up row equals the oracle's dequantization of that table row bit for bit
(same fp32 multiply-add, one rounding to the output dtype); an out-of-range id yields a
zero row and is reported by check_device; the output projection over 248,320 rows is
within 2e-2 * RMS of the oracle on sampled rows (fp32 accumulation on both sides).  A
rotated row equals the oracle's inverse rotation of the bf16 dequantized row bit for bit
(the butterflies are the same IEEE adds in the same order), and in f16 with the real
pack's layout (group 128, block 1024) it equals the lookup followed by the library's own
inverse rotation bit for bit.
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


@pytest.mark.parametrize("block", [256, 1024, 4096])
def test_hadamard_embedding_bit_exact(q38, block):
    rows, K, bits = 200, 4096, 2
    c, s, b = make_weight(910, rows, K, bits)
    signs = np.where(np.random.default_rng(block).random(K) < 0.5, -1.0, 1.0).astype(np.float32)
    ids = np.random.default_rng(911).integers(0, rows, size=(2, 9)).astype(np.int32)
    emb = q38.QuantizedEmbedding(dev_u32(c), dev_bf16(s), dev_bf16(b), 64, bits)
    rot = q38.HadamardQuantizedEmbedding(emb, torch.from_numpy(signs).cuda(), block)
    out = rot(torch.from_numpy(ids).cuda())
    torch.cuda.synchronize()
    q38.check_device()
    assert out.shape == (2, 9, K) and out.dtype == torch.bfloat16
    rows_bf16 = O.f32_to_bf16(O.dequantize(c, s, b, 64, bits)[ids.reshape(-1)])
    ref = O.hadamard_rotate(rows_bf16, block, signs, inverse=True)
    np.testing.assert_array_equal(host_bf16(out).reshape(-1, K), ref)


def test_hadamard_embedding_bonsai_layout_f16(q38):
    # the real pack: group 128, f16 scales, biases = -scales (ternary), block 1024
    rows, K, bits, group, block = 96, 2048, 2, 128, 1024
    g = torch.Generator(device="cuda").manual_seed(912)
    codes = torch.randint(0, 3, (rows, K), device="cuda", generator=g, dtype=torch.int32)
    packed = torch.zeros((rows, K * bits // 32), dtype=torch.int64, device="cuda")
    for j in range(16):
        packed |= codes[:, j::16].to(torch.int64) << (2 * j)
    packed = torch.where(packed >= 2 ** 31, packed - 2 ** 32, packed).to(torch.int32)  # u32 bit patterns
    scales = (torch.rand((rows, K // group), device="cuda", generator=g) * 0.02 + 0.001).half()
    biases = -scales
    signs = torch.where(torch.rand(K, device="cuda", generator=g) < 0.5, -1.0, 1.0)
    ids = torch.tensor([[3, 95, 0, 3], [50, 1, 2, 94]], dtype=torch.int32, device="cuda")
    got = q38.hadamard_quantized_embedding(ids, packed, scales, biases, signs, block, group, bits)
    looked_up = q38.quantized_embedding(ids, packed, scales, biases, group, bits)
    ref = q38.hadamard_rotate(looked_up, signs, block, inverse=True)
    torch.cuda.synchronize()
    q38.check_device()
    assert got.dtype == torch.float16 and got.shape == (2, 4, K)
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_hadamard_embedding_out_of_range_and_arguments(q38):
    rows, K, bits = 16, 512, 2
    c, s, b = make_weight(913, rows, K, bits)
    ids = torch.tensor([rows + 4, 1], dtype=torch.int32, device="cuda")
    out = q38.hadamard_quantized_embedding(ids, dev_u32(c), dev_bf16(s), dev_bf16(b), None, 256, 64, bits)
    with pytest.raises(q38.Q38Error):
        q38.check_device()
    assert torch.count_nonzero(out[0]).item() == 0
    ref = O.hadamard_rotate(O.f32_to_bf16(O.dequantize(c, s, b, 64, bits)[[1]]), 256, None, inverse=True)
    np.testing.assert_array_equal(host_bf16(out)[[1]], ref)
    with pytest.raises(q38.Q38Error):  # block does not divide K
        q38.hadamard_quantized_embedding(ids, dev_u32(c), dev_bf16(s), dev_bf16(b), None, 1024, 64, bits)
    with pytest.raises(q38.Q38Error):  # block not a power of two
        q38.hadamard_quantized_embedding(ids, dev_u32(c), dev_bf16(s), dev_bf16(b), None, 384, 64, bits)


@pytest.mark.parametrize("bits,block,K", [(3, 512, 2048), (4, 8192, 8192), (8, 64, 1024)])
def test_hadamard_embedding_other_widths(q38, bits, block, K):
    # 3-bit codes (decoded one by one), the shared-memory kernel for blocks above 4096, and
    # blocks small enough that one CTA holds several
    rows = 40
    c, s, b = make_weight(920 + bits, rows, K, bits)
    signs = np.where(np.random.default_rng(block).random(K) < 0.5, -1.0, 1.0).astype(np.float32)
    ids = np.random.default_rng(921).integers(0, rows, size=(5,)).astype(np.int32)
    out = q38.hadamard_quantized_embedding(torch.from_numpy(ids).cuda(), dev_u32(c), dev_bf16(s), dev_bf16(b),
                                           torch.from_numpy(signs).cuda(), block, 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    ref = O.hadamard_rotate(O.f32_to_bf16(O.dequantize(c, s, b, 64, bits)[ids]), block, signs, inverse=True)
    np.testing.assert_array_equal(host_bf16(out), ref)


def test_embedding_many_ids(q38):
    # more ids than one grid dimension holds (65,535): the lookup loops over the rest
    rows, K, bits = 300, 256, 4
    c, s, b = make_weight(930, rows, K, bits)
    ids = np.random.default_rng(931).integers(0, rows, size=(70000,)).astype(np.int32)
    out = q38.quantized_embedding(torch.from_numpy(ids).cuda(), dev_u32(c), dev_bf16(s), dev_bf16(b), 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    table = O.f32_to_bf16(O.dequantize(c, s, b, 64, bits))
    np.testing.assert_array_equal(host_bf16(out), table[ids])
