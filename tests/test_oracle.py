"""CPU tests of the oracle: pinned against the golden fixtures of the packed format and
against the properties the reference's own tests check."""
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "affine_format.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_dequant_matches_independent_format_implementation(golden, bits):
    """The oracle's unpack+dequantize equals a third-party MLX-format implementation
    bit for bit on codes that implementation packed."""
    codes = golden[f"b{bits}_codes"]
    deq = O.dequantize(codes, golden[f"b{bits}_scales"], golden[f"b{bits}_biases"], 64, bits)
    np.testing.assert_array_equal(deq, golden[f"b{bits}_dequant"])


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_oracle_quantizer_output_reads_back_identically(golden, bits):
    """Codes packed by the oracle's quantizer are read identically by the third-party
    dequantizer (same bit order on the producer side too)."""
    codes = golden[f"b{bits}_oracle_codes"]
    deq = O.dequantize(codes, golden[f"b{bits}_oracle_scales"], golden[f"b{bits}_oracle_biases"], 64, bits)
    np.testing.assert_array_equal(deq, golden[f"b{bits}_oracle_dequant_3p"])
    # and the oracle's quantizer is deterministic
    w = O.normal_f32(1000 + bits, (32, 256), 0.02)
    c2, s2, b2 = O.quantize(w, 64, bits)
    np.testing.assert_array_equal(c2, codes)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_qmm_matches_golden_product(golden, bits):
    x = golden[f"b{bits}_x"]
    y = O.qmm(x, golden[f"b{bits}_codes"], golden[f"b{bits}_scales"], golden[f"b{bits}_biases"], 64,
              bits, f32=True)
    ref = golden[f"b{bits}_y"]
    rms = np.sqrt((ref.astype(np.float64) ** 2).mean())
    assert np.abs(y - ref).max() <= 1e-5 * max(rms, 1.0)


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_pack_unpack_roundtrip(bits):
    rng = np.random.default_rng(bits)
    q = rng.integers(0, 1 << bits, size=(7, 192), dtype=np.uint8)
    codes = O.pack(q, bits)
    assert codes.shape == (7, 192 * bits // 32)
    np.testing.assert_array_equal(O.unpack(codes, 192, bits), q)


def test_three_bit_bitstream_layout():
    """3-bit codes straddle words: code k occupies bits [3k, 3k+3) of the row stream."""
    q = np.zeros((1, 32), dtype=np.uint8)
    q[0, 10] = 7  # bits 30..32 -> straddles word 0 / word 1
    codes = O.pack(q, 3)
    assert codes[0, 0] == (3 << 30)
    assert codes[0, 1] == 1
    assert codes[0, 2] == 0


def test_packed_shapes_match_reference_containers():
    """Packed shapes of Tests/Qwen38Tests/Qwen38Tests.swift:2786-2856."""
    w = O.normal_f32(7, (128, 256), 0.02)
    c, s, b = O.quantize(w, 32, 4)
    assert c.shape == (128, 32) and s.shape == (128, 8) and b.shape == (128, 8)
    w3 = O.normal_f32(8, (8, 128, 256), 0.02)
    c3, s3, _ = O.quantize(w3, 64, 3)
    assert c3.shape == (8, 128, 24) and s3.shape == (8, 128, 4)
    wd = O.normal_f32(9, (8, 256, 128), 0.02)
    cd, sd, _ = O.quantize(wd, 64, 3)
    assert cd.shape == (8, 256, 12) and sd.shape == (8, 256, 2)
    for bits in (2, 3, 4, 5, 6, 8):
        c, s, _ = O.quantize(O.normal_f32(10, (4, 256), 0.02), 64, bits)
        assert c.shape == (4, 256 * bits // 32)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_quantizer_properties(bits):
    """The larger-magnitude extreme of each group is reproduced (up to bf16 storage of
    scale/bias) and every code is in range.  Rounding error is at most half a step; the
    opposite extreme can additionally be clamped (scale = edge / rint(edge / scale0) may
    shrink the grid), so the bound is one step."""
    w = O.normal_f32(20 + bits, (64, 512), 0.02)
    c, s, b = O.quantize(w, 64, bits)
    q = O.unpack(c, 512, bits)
    assert q.max() <= (1 << bits) - 1
    deq = O.dequantize(c, s, b, 64, bits)
    sf = np.abs(O.bf16_to_f32(s)).repeat(64, axis=1)
    err = np.abs(deq - w)
    # bf16 storage of scale and bias adds up to 2^-9 relative error on each
    gmax = np.abs(w.reshape(64, 8, 64)).max(axis=2).repeat(64, axis=1)
    assert (err <= 1.5 * sf + 4e-3 * gmax + 1e-6).all()
    assert np.median(err / sf) < 0.3
    g = w.reshape(64, 8, 64)
    idx = np.abs(g).argmax(axis=2)
    edge = np.take_along_axis(g, idx[..., None], 2)[..., 0]
    dg = deq.reshape(64, 8, 64)
    dedge = np.take_along_axis(dg, idx[..., None], 2)[..., 0]
    np.testing.assert_allclose(dedge, edge, rtol=8e-3, atol=1e-6)


def test_router_survives_bf16_probabilities():
    """Re-creation of qwen4ExpSparseMoERoutingSurvivesImpreciseSoftmax
    (Tests/Qwen38Tests/Qwen38Tests.swift:3040-3066): 200 logit vectors U(-8, 8) of width
    512, top-10; the selected set equals the exact top-10 of the logits except where the
    10th and 11th bf16 probabilities tie (the canonical id order then decides)."""
    rng = np.random.default_rng(20260909)
    logits = O.f32_to_bf16(rng.uniform(-8, 8, size=(200, 512)).astype(np.float32))
    idx, sc, probs = O.route_from_logits(logits, 10, normalize=True)
    lf = O.bf16_to_f32(logits)
    flips = 0
    for t in range(200):
        exact = set(np.argsort(-lf[t], kind="stable")[:10].tolist())
        if exact != set(idx[t].tolist()):
            pf = O.bf16_to_f32(probs[t])
            srt = np.sort(pf)[::-1]
            assert srt[9] == srt[10], "membership changed without a bf16 tie at the boundary"
            flips += 1
    assert flips <= 5
    # canonical order: probabilities non-increasing, ties by ascending id
    pf = O.bf16_to_f32(probs)
    sel = np.take_along_axis(pf, idx, 1)
    assert (np.diff(sel, axis=1) <= 0).all()
    s = O.bf16_to_f32(sc).sum(axis=1)
    assert np.abs(s - 1).max() < 2e-2


def test_router_from_x_matches_logits_path():
    x = O.normal_bf16(31, (5, 256))
    wr = O.normal_bf16(32, (64, 256), 0.02)
    idx, sc, probs = O.moe_route(x, wr, 4, True, want_probs=True)
    logits = O.f32_to_bf16(O.bf16_to_f32(x) @ O.bf16_to_f32(wr).T)
    idx2, sc2, p2 = O.route_from_logits(logits, 4, True)
    # logits identical up to fp32 summation order; indices equal unless a near-tie
    assert (idx == idx2).mean() > 0.9


def test_sort_by_expert_is_stable():
    rng = np.random.default_rng(3)
    ind = rng.integers(0, 16, size=(40, 4)).astype(np.int32)
    perm, off = O.sort_by_expert(ind, 16)
    flat = ind.reshape(-1)
    assert off[0] == 0 and off[-1] == flat.size
    for e in range(16):
        run = perm[off[e]:off[e + 1]]
        assert (flat[run] == e).all()
        assert (np.diff(run) > 0).all()


@pytest.mark.parametrize("block", [4, 256, 1024])
def test_hadamard_is_orthonormal_and_inverse(block):
    x = O.normal_bf16(41, (3, 2048))
    signs = np.where(np.arange(2048) % 3 == 0, -1.0, 1.0).astype(np.float32)
    y = O.hadamard_rotate(x, block, signs)
    xf, yf = O.bf16_to_f32(x), O.bf16_to_f32(y)
    np.testing.assert_allclose(np.linalg.norm(yf, axis=1), np.linalg.norm(xf, axis=1), rtol=1e-2)
    back = O.bf16_to_f32(O.hadamard_rotate(y, block, signs, inverse=True))
    assert np.abs(back - xf).max() < 0.05 * np.abs(xf).max()
    # block transform equals the explicit Sylvester matrix
    H = np.array([[1.0]])
    while H.shape[0] < block:
        H = np.block([[H, H], [H, -H]])
    ref = (xf * signs).reshape(3, -1, block) @ H.T / np.sqrt(block)
    assert np.abs(yf - ref.reshape(3, 2048)).max() < 1e-2 * np.abs(ref).max()


def test_switch_glu_matches_dense_restatement():
    T, H, I, E, k = 3, 128, 64, 6, 2
    x = O.normal_bf16(51, (T, H))
    mk = lambda seed, shape: O.quantize(O.normal_f32(seed, shape, 0.02), 64, 4)
    gate, up, down = mk(52, (E, I, H)), mk(53, (E, I, H)), mk(54, (E, H, I))
    ind = np.array([[0, 5], [2, 2], [4, 1]], dtype=np.int32)
    sc = O.f32_to_bf16(np.array([[0.6, 0.4], [0.5, 0.5], [0.9, 0.1]], dtype=np.float32))
    out = O.bf16_to_f32(O.switch_glu(x, ind, sc, gate, up, down, 64, 4))
    xf = O.bf16_to_f32(x)
    dq = lambda t: O.dequantize(*t, 64, 4)
    G, U, D = dq(gate), dq(up), dq(down)
    ref = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in range(k):
            e = ind[t, j]
            g = xf[t] @ G[e].T
            u = xf[t] @ U[e].T
            h = g / (1 + np.exp(-g)) * u
            ref[t] += O.bf16_to_f32(sc[t:t + 1, j])[0] * (h @ D[e].T)
    rms = np.sqrt((ref ** 2).mean())
    assert np.abs(out - ref).max() <= 2e-2 * rms


def test_gather_qmm_matches_per_expert_qmm():
    E, N, K = 4, 32, 128
    c, s, b = O.quantize(O.normal_f32(61, (E, N, K), 0.02), 64, 4)
    x = O.normal_bf16(62, (3, 2, K))
    lhs = np.array([0, 2, 1, 2], np.int32)
    rhs = np.array([3, 0, 3, 1], np.int32)
    out = O.gather_qmm(x, c, s, b, lhs, rhs, 64, 4)
    for p in range(4):
        ref = O.qmm(x[lhs[p]], c[rhs[p]], s[rhs[p]], b[rhs[p]], 64, 4)
        np.testing.assert_array_equal(out[p], ref)


def test_switch_glu_bf16_weight_mode_matches_restatement():
    """weights_bf16 rounds each dequantized weight once to bf16: equal to a dense
    restatement that rounds the (exact) s*q + b to bf16 before the products."""
    T, H, I, E, k = 4, 128, 64, 5, 2
    x = O.normal_bf16(71, (T, H))
    mk = lambda seed, shape: O.quantize(O.normal_f32(seed, shape, 0.02), 64, 3)
    gate, up, down = mk(72, (E, I, H)), mk(73, (E, I, H)), mk(74, (E, H, I))
    ind = np.array([[0, 4], [2, 1], [3, 3], [1, 0]], dtype=np.int32)
    sc = O.f32_to_bf16(np.array([[0.7, 0.3], [0.5, 0.5], [0.6, 0.4], [0.2, 0.8]], dtype=np.float32))
    out = O.bf16_to_f32(O.switch_glu(x, ind, sc, gate, up, down, 64, 3, weights_bf16=True))
    rb = lambda a: O.bf16_to_f32(O.f32_to_bf16(np.asarray(a, np.float32)))

    def wq(t, n, kk):
        q = O.unpack(t[0].reshape(E * n, -1), kk, 3).astype(np.float64)
        s = np.repeat(O.bf16_to_f32(t[1].reshape(E * n, -1)).astype(np.float64), 64, axis=1)
        b = np.repeat(O.bf16_to_f32(t[2].reshape(E * n, -1)).astype(np.float64), 64, axis=1)
        return rb(s * q + b).reshape(E, n, kk)  # s*q + b exact in float64, one rounding
    G, U, D = wq(gate, I, H), wq(up, I, H), wq(down, H, I)
    xf, s = O.bf16_to_f32(x), O.bf16_to_f32(sc)
    ref = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in range(k):
            e = ind[t, j]
            g, u = rb(G[e] @ xf[t]), rb(U[e] @ xf[t])
            ref[t] += s[t, j] * rb(D[e] @ rb(g / (1 + np.exp(-g)) * u))
    ref = rb(ref)
    rms = np.sqrt((ref.astype(np.float64) ** 2).mean())
    assert np.abs(out - ref).max() <= 2e-2 * rms
