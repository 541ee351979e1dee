"""GPU parity of the sparse-MoE layer (router, expert sort, SwitchGLU) against the oracle,
through libq38.so's C ABI.

Bars: router indices, scores and probabilities bit-exact given identical logits; the sort
permutation and offsets bit-exact.  Router decisions from x (logits computed on each side
with its own fp32 summation order) must agree except at a probability tie at the top-k
boundary.

SwitchGLU outputs: |y - y_oracle| <= 2e-2 * RMS(y_oracle) + one bf16 step of |y_oracle|
per element, fp32 accumulation on both sides.  The output is bf16 and its largest values
are 5-10x its RMS, where one representable step (2^-8 relative) already exceeds 2e-2 * RMS:
a different fp32 summation order may round the same value to the neighbouring bf16.
The comparison is against the oracle with weights_bf16: the tensor-core path multiplies bf16
operands, so each dequantized weight s*q + b is rounded once to bf16 before the product,
and the oracle applies the same single rounding.  (Against fp32-evaluated weights the
layer's own bf16 roundings of g, u, h and y_ts amplify that operand rounding to a few
bf16 steps at the largest outputs; test_switch_glu_fp32_weight_oracle bounds that case
statistically.)
"""
import numpy as np
import pytest
import torch

import oracle as O
from test_qmm_gpu import dev_bf16, dev_u32, host_bf16

pytestmark = pytest.mark.gpu


def check_close(y_gpu_bf16, y_ref, tol=2e-2):
    y = O.bf16_to_f32(y_gpu_bf16).astype(np.float64)
    ref = np.asarray(y_ref, dtype=np.float64)
    assert np.isfinite(y).all()
    rms = np.sqrt((ref ** 2).mean())
    step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -126))) - 7)  # bf16 spacing at |ref|
    excess = (np.abs(y - ref) - step).max()
    assert excess <= tol * rms, f"max err beyond one bf16 step {excess:.4g} > {tol} * rms {rms:.4g}"


def check_stat(y_gpu_bf16, y_ref):
    """Against fp32-evaluated weights: error RMS <= 1e-2 * RMS, max <= 1e-1 * RMS."""
    y = O.bf16_to_f32(y_gpu_bf16).astype(np.float64)
    ref = np.asarray(y_ref, dtype=np.float64)
    assert np.isfinite(y).all()
    rms = np.sqrt((ref ** 2).mean())
    err = np.abs(y - ref)
    assert np.sqrt((err ** 2).mean()) <= 1e-2 * rms
    assert err.max() <= 1e-1 * rms


def dev_i32(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).cuda()


@pytest.mark.parametrize("normalize", [True, False])
@pytest.mark.parametrize("T,E,k,dist", [(200, 512, 10, "uniform8"), (64, 512, 10, "normal"),
                                        (33, 64, 4, "normal"), (5, 1000, 32, "uniform8"), (7, 8, 8, "normal")])
def test_router_selection_bit_exact(q38, T, E, k, dist, normalize):
    rng = np.random.default_rng(T * 1000 + E + k)
    raw = rng.uniform(-8, 8, (T, E)) if dist == "uniform8" else rng.normal(0, 1.5, (T, E))
    logits = O.f32_to_bf16(raw.astype(np.float32))
    idx, sc, pr = O.route_from_logits(logits, k, normalize)
    gi, gs, gp = q38.moe_route_logits(dev_bf16(logits), k, normalize, want_probs=True)
    np.testing.assert_array_equal(host_bf16(gp), pr)
    np.testing.assert_array_equal(gi.cpu().numpy(), idx)
    np.testing.assert_array_equal(host_bf16(gs), sc)


def test_router_ties_take_the_lower_expert_id(q38):
    logits = O.f32_to_bf16(np.zeros((3, 64), np.float32))  # all probabilities equal
    logits[1, 40] = O.f32_to_bf16(np.array([2.0], np.float32))[0]
    gi, _ = q38.moe_route_logits(dev_bf16(logits), 6)
    idx, _, _ = O.route_from_logits(logits, 6)
    np.testing.assert_array_equal(gi.cpu().numpy(), idx)
    assert list(idx[0]) == [0, 1, 2, 3, 4, 5] and idx[1][0] == 40


@pytest.mark.parametrize("T", [1, 8, 64, 300, 4096])
def test_router_from_activations(q38, T):
    """Flash-Next router: H 2048, 512 experts, top-10; x N(0,1), Wr N(0, 0.02^2).  T <= 64
    takes the CUDA-core logits, larger T the tcgen05 GEMM."""
    H, E, k = 2048, 512, 10
    x = O.normal_bf16(7000 + T, (T, H))
    wr = O.normal_bf16(7001, (E, H), 0.02)
    idx, sc, pr = O.moe_route(x, wr, k, True, want_probs=True)
    gi, gs, gp = q38.moe_route(dev_bf16(x), dev_bf16(wr), k, True, want_probs=True)
    gi, gp = gi.cpu().numpy(), O.bf16_to_f32(host_bf16(gp))
    pf = O.bf16_to_f32(pr)
    # probabilities: the same up to one bf16 rounding of a logit
    assert np.abs(gp - pf).max() <= 2e-2 * pf.max()
    flips = 0
    for t in range(T):
        if set(gi[t]) != set(idx[t]):
            srt = np.sort(pf[t])[::-1]
            assert srt[k - 1] - srt[k] <= 2 * 2.0 ** -8 * srt[k - 1], "selection differs away from a near-tie"
            flips += 1
    assert flips <= max(2, T // 100)
    # where the selection agrees, the canonical order and scores agree too
    same = [t for t in range(T) if (gi[t] == idx[t]).all()]
    assert len(same) >= T - flips - max(2, T // 100)


@pytest.mark.parametrize("P,E", [(1, 8), (10, 512), (80, 512), (640, 512), (40960, 512), (5000, 1000)])
def test_sort_by_expert_bit_exact(q38, P, E):
    rng = np.random.default_rng(P + E)
    ind = rng.integers(0, E, size=P).astype(np.int32)
    perm, off = O.sort_by_expert(ind, E)
    gperm, goff = q38.moe_sort(dev_i32(ind), E)
    np.testing.assert_array_equal(goff.cpu().numpy(), off)
    np.testing.assert_array_equal(gperm.cpu().numpy(), perm)


def test_sort_reports_bad_index(q38):
    ind = np.array([1, 2, 9, 0], np.int32)
    perm, off = q38.moe_sort(dev_i32(ind), 4)
    with pytest.raises(q38.Q38ArgumentError):
        q38.check_device()
    assert list(off.cpu().numpy()) == [0, 1, 2, 3, 3]
    assert list(perm.cpu().numpy()[:3]) == [3, 0, 1]
    q38.check_device()


def make_experts(q38, seed, E, I, H, bits):
    """Expert stacks quantized on the GPU (bit-exact with the oracle's quantizer), copied back
    for the oracle."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    trip = []
    for (n, k) in ((I, H), (I, H), (H, I)):
        w = torch.randn((E * n, k), generator=g, device="cuda") * 0.02
        c, s, b = q38.quantize(w, 64, bits, scales_dtype=torch.bfloat16)
        trip.append(((c.view(torch.int32).view(E, n, -1), s.view(E, n, -1), b.view(E, n, -1)),
                     (c.view(torch.int32).cpu().numpy().view(np.uint32).reshape(E, n, -1),
                      host_bf16(s).reshape(E, n, -1), host_bf16(b).reshape(E, n, -1))))
        del w
    return [t[0] for t in trip], [t[1] for t in trip]


def route_inputs(T, E, k, seed):
    rng = np.random.default_rng(seed)
    logits = O.f32_to_bf16(rng.normal(0, 1.0, (T, E)).astype(np.float32))
    idx, sc, _ = O.route_from_logits(logits, k, True)
    return idx, sc


@pytest.mark.parametrize("bits", [3, 2, 4])
@pytest.mark.parametrize("T,E,k,H,I", [(5, 16, 4, 512, 512), (64, 32, 10, 2048, 512), (1, 32, 10, 2048, 512),
                                       (300, 8, 2, 1024, 1024)])
def test_switch_glu_parity(q38, bits, T, E, k, H, I):
    dev, host = make_experts(q38, 8000 + bits + T, E, I, H, bits)
    x = O.normal_bf16(8100 + T, (T, H))
    idx, sc = route_inputs(T, E, k, 8200 + T)
    ref = O.switch_glu(x, idx, sc, *host, 64, bits, weights_bf16=True)
    out = q38.switch_glu(dev_bf16(x), dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))


def test_switch_glu_fp32_weight_oracle(q38):
    T, E, k, H, I, bits = 64, 32, 10, 2048, 512, 3
    dev, host = make_experts(q38, 8050, E, I, H, bits)
    x = O.normal_bf16(8051, (T, H))
    idx, sc = route_inputs(T, E, k, 8052)
    ref = O.switch_glu(x, idx, sc, *host, 64, bits)
    out = q38.switch_glu(dev_bf16(x), dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    check_stat(host_bf16(out), O.bf16_to_f32(ref))


def test_switch_glu_without_biases(q38):
    T, E, k, H, I, bits = 20, 8, 3, 512, 512, 3
    dev, host = make_experts(q38, 8300, E, I, H, bits)
    dev = [(c, s, None) for (c, s, b) in dev]
    host = [(c, s, None) for (c, s, b) in host]
    x = O.normal_bf16(8301, (T, H))
    idx, sc = route_inputs(T, E, k, 8302)
    ref = O.switch_glu(x, idx, sc, *host, 64, bits, weights_bf16=True)
    out = q38.switch_glu(dev_bf16(x), dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))


def test_switch_glu_prompt_sampled_tokens(q38):
    """4096 tokens over 64 experts (about 640 pairs per expert: runs of 128 pairs, several
    per expert); 8 sampled tokens checked against the oracle (a token's output depends only
    on its own row, experts and scores)."""
    T, E, k, H, I, bits = 4096, 64, 10, 2048, 512, 3
    dev, host = make_experts(q38, 8400, E, I, H, bits)
    x = O.normal_bf16(8401, (T, H))
    idx, sc = route_inputs(T, E, k, 8402)
    out = q38.switch_glu(dev_bf16(x), dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    rows = np.array([0, 1, 127, 128, 2000, 3001, 4094, 4095])
    ref = O.switch_glu(np.ascontiguousarray(x[rows]), idx[rows], sc[rows], *host, 64, bits, weights_bf16=True)
    check_close(host_bf16(out[torch.from_numpy(rows).cuda()]), O.bf16_to_f32(ref).astype(np.float64))


def test_sparse_moe_block_end_to_end(q38):
    """Router + SwitchGLU through the module classes (Flash-Next shapes, 32 experts)."""
    T, E, k, H, I, bits = 16, 32, 10, 2048, 512, 3
    dev, host = make_experts(q38, 8500, E, I, H, bits)
    x = O.normal_bf16(8501, (T, H))
    wr = O.normal_bf16(8502, (E, H), 0.02)
    sw = q38.SwitchGLU(*[q38.QuantizedSwitchLinear(c, s, b, 64, bits) for (c, s, b) in dev])
    block = q38.SparseMoeBlock(dev_bf16(wr), sw, k)
    out = block(dev_bf16(x))
    gi, gs = q38.moe_route(dev_bf16(x), dev_bf16(wr), k)
    ref = O.switch_glu(x, gi.cpu().numpy(), host_bf16(gs), *host, 64, bits, weights_bf16=True)
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))


# ------------------------------------------------------------------ Flash-Next at full size
# The benchmark configuration of the MoE layer: hidden 2048, 512 experts, intermediate 512,
# top-10, 3-bit group 64, router Wr N(0, 0.02^2).  The expert stacks (704 MB of codes) are
# quantized once per module.

FN_E, FN_I, FN_H, FN_K, FN_BITS = 512, 512, 2048, 10, 3


@pytest.fixture(scope="module")
def flash_next(q38):
    dev, host = make_experts(q38, 8600, FN_E, FN_I, FN_H, FN_BITS)
    wr = O.normal_bf16(8601, (FN_E, FN_H), 0.02)
    return dev, host, wr


def error_summary(y_gpu_bf16, y_ref):
    """max |err| / RMS, max excess over one bf16 step / RMS, RMS(err) / RMS."""
    y = O.bf16_to_f32(y_gpu_bf16).astype(np.float64)
    ref = np.asarray(y_ref, dtype=np.float64)
    rms = np.sqrt((ref ** 2).mean())
    err = np.abs(y - ref)
    step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -126))) - 7)
    return err.max() / rms, max((err - step).max(), 0.0) / rms, np.sqrt((err ** 2).mean()) / rms


@pytest.mark.parametrize("T", [1, 8, 64])
def test_switch_glu_flash_next_512_experts(q38, flash_next, T):
    """SwitchGLU at the MoE benchmark's full expert count, routed by the router from x."""
    dev, host, wr = flash_next
    x = O.normal_bf16(8610 + T, (T, FN_H))
    gi, gs = q38.moe_route(dev_bf16(x), dev_bf16(wr), FN_K)
    idx, sc = gi.cpu().numpy(), host_bf16(gs)
    out = q38.switch_glu(dev_bf16(x), gi, gs, *dev, 64, FN_BITS)
    torch.cuda.synchronize()
    q38.check_device()
    ref = O.switch_glu(x, idx, sc, *host, 64, FN_BITS, weights_bf16=True)
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))
    # against fp32-evaluated weights (the literal MLX arithmetic): reported, bounded
    ref32 = O.bf16_to_f32(O.switch_glu(x, idx, sc, *host, 64, FN_BITS))
    mx, ex, er = error_summary(host_bf16(out), ref32)
    print(f"\nflash-next E=512 T={T} vs fp32 weights: max/rms {mx:.4f}, "
          f"max beyond one bf16 step/rms {ex:.4f}, rms(err)/rms {er:.5f}")
    check_stat(host_bf16(out), ref32)


def test_switch_glu_flash_next_4096_tokens_sampled(q38, flash_next):
    """4096 tokens over the 512 experts (all experts touched, ~80 pairs each); 8 sampled
    tokens checked against the oracle."""
    dev, host, wr = flash_next
    T = 4096
    x = O.normal_bf16(8620, (T, FN_H))
    gi, gs = q38.moe_route(dev_bf16(x), dev_bf16(wr), FN_K)
    out = q38.switch_glu(dev_bf16(x), gi, gs, *dev, 64, FN_BITS)
    torch.cuda.synchronize()
    q38.check_device()
    rows = np.array([0, 1, 127, 128, 2000, 3001, 4094, 4095])
    idx, sc = gi.cpu().numpy()[rows], host_bf16(gs)[rows]
    ref = O.switch_glu(np.ascontiguousarray(x[rows]), idx, sc, *host, 64, FN_BITS, weights_bf16=True)
    check_close(host_bf16(out[torch.from_numpy(rows).cuda()]), O.bf16_to_f32(ref).astype(np.float64))


@pytest.mark.parametrize("T", [1, 8])
def test_sparse_moe_block_flash_next_512_experts(q38, flash_next, T):
    """Router + SwitchGLU through the module classes at 512 experts."""
    dev, host, wr = flash_next
    x = O.normal_bf16(8630 + T, (T, FN_H))
    sw = q38.SwitchGLU(*[q38.QuantizedSwitchLinear(c, s, b, 64, FN_BITS) for (c, s, b) in dev])
    block = q38.SparseMoeBlock(dev_bf16(wr), sw, FN_K)
    out = block(dev_bf16(x))
    idx, sc, _ = O.moe_route(x, wr, FN_K, True, want_probs=True)
    gi, gs = q38.moe_route(dev_bf16(x), dev_bf16(wr), FN_K)
    # the oracle's routing decides which experts are used; it agrees with the device's
    # except at near-ties, where the device's choice is used for the product check
    ref = O.switch_glu(x, gi.cpu().numpy(), host_bf16(gs), *host, 64, FN_BITS, weights_bf16=True)
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))
    assert (gi.cpu().numpy() == idx).mean() >= 0.9


# ------------------------------------------------------------- decode-shaped SwitchGLU
# T <= 16 tokens with T * top_k <= 256 run on the decode kernel: the selected experts'
# gate/up rows for all tokens (only selecting pairs stored), then the down rows with h
# formed from the gate/up sums.  The weights enter the products exactly (scales applied in
# fp32 to exact code sums), so the bar is the fp32-weight oracle's.

@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("T,E,k,H,I", [(1, 64, 10, 2048, 512), (2, 16, 8, 512, 1024), (16, 64, 10, 1024, 512),
                                       (16, 32, 16, 512, 512), (7, 300, 4, 1536, 512)])
def test_switch_glu_decode_parity(q38, bits, T, E, k, H, I):
    dev, host = make_experts(q38, 8700 + bits + T + E, E, I, H, bits)
    x = O.normal_bf16(8710 + T, (T, H))
    idx, sc = route_inputs(T, E, k, 8720 + T + E)
    out = q38.switch_glu(dev_bf16(x), dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    ref = O.switch_glu(x, idx, sc, *host, 64, bits)
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))


def test_switch_glu_decode_empty_slots_and_no_biases(q38):
    T, E, k, H, I, bits = 5, 24, 6, 1024, 512, 3
    dev, host = make_experts(q38, 8730, E, I, H, bits)
    dev = [(c, s, None) for (c, s, b) in dev]
    host = [(c, s, None) for (c, s, b) in host]
    x = O.normal_bf16(8731, (T, H))
    idx, sc = route_inputs(T, E, k, 8732)
    idx = idx.copy()
    idx[1, 2] = -1
    idx[3, :] = -1  # a token without experts gives zeros
    out = q38.switch_glu(dev_bf16(x), dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    ref = O.switch_glu(x, idx, sc, *host, 64, bits)
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))
    assert (host_bf16(out)[3] == 0).all()


def test_switch_glu_decode_is_deterministic(q38):
    T, E, k, H, I, bits = 8, 64, 10, 2048, 512, 3
    dev, _ = make_experts(q38, 8740, E, I, H, bits)
    x = dev_bf16(O.normal_bf16(8741, (T, H)))
    idx, sc = route_inputs(T, E, k, 8742)
    a = q38.switch_glu(x, dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    b = q38.switch_glu(x, dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("T", [3, 16, 40, 300])
def test_switch_glu_8bit_experts(q38, T):
    """8-bit experts: the decode path up to 16 tokens (fp32-weight oracle), the grouped
    tensor-core path beyond (bf16-rounded weights, as for the narrower widths)."""
    E, k, H, I, bits = 32, 8, 1024, 512, 8
    dev, host = make_experts(q38, 8800 + T, E, I, H, bits)
    x = O.normal_bf16(8810 + T, (T, H))
    idx, sc = route_inputs(T, E, k, 8820 + T)
    out = q38.switch_glu(dev_bf16(x), dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    ref = O.switch_glu(x, idx, sc, *host, 64, bits, weights_bf16=T > 16)
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))


@pytest.mark.parametrize("E,k", [(512, 10), (1000, 32), (100, 4), (256, 8)])
def test_router_single_token_matches_multi_token_path(q38, E, k):
    """One token's selection (spread over a block's four warps) equals, bit for bit, the
    selection of the same token routed together with another (one warp per token)."""
    H = 2048
    x = O.normal_bf16(8900 + E, (1, H))
    wr = O.normal_bf16(8901 + E, (E, H), 0.02)
    i1, s1, p1 = q38.moe_route(dev_bf16(x), dev_bf16(wr), k, True, want_probs=True)
    x2 = np.concatenate([x, O.normal_bf16(8902, (1, H))])
    i2, s2, p2 = q38.moe_route(dev_bf16(x2), dev_bf16(wr), k, True, want_probs=True)
    assert torch.equal(i1[0], i2[0]) and torch.equal(s1[0], s2[0]) and torch.equal(p1[0], p2[0])


@pytest.mark.parametrize("T", [1, 3, 8])
def test_sparse_moe_equals_route_then_switch_glu(q38, flash_next, T):
    """q38_sparse_moe (router, then SwitchGLU, in one call) equals the two calls made
    separately, bit for bit."""
    dev, host, wr = flash_next
    x = dev_bf16(O.normal_bf16(8640 + T, (T, FN_H)))
    sw = q38.SwitchGLU(*[q38.QuantizedSwitchLinear(c, s, b, 64, FN_BITS) for (c, s, b) in dev])
    out, idx, sc = q38.sparse_moe(x, dev_bf16(wr), sw, FN_K)
    gi, gs = q38.moe_route(x, dev_bf16(wr), FN_K)
    ref = q38.switch_glu(x, gi, gs, *dev, 64, FN_BITS)
    torch.cuda.synchronize()
    q38.check_device()
    assert torch.equal(idx, gi) and torch.equal(sc, gs) and torch.equal(out, ref)


@pytest.mark.parametrize("T", [1, 8, 64])
@pytest.mark.parametrize("group,bits", [(32, 4), (64, 3), (64, 4)])
def test_shared_expert(q38, T, group, bits):
    """The shared-expert term of the sparse-MoE block at Flash-Next sizes (hidden 2048,
    shared intermediate 512; the published checkpoint quantizes it 4-bit group 32), added to
    a routed output, against the oracle's composition of bf16-rounded products."""
    H, I = 2048, 512
    mats = []
    for i, (n, k) in enumerate(((I, H), (I, H), (H, I), (1, H))):
        w = O.normal_f32(9100 + 10 * i + bits + group, (n, k), 0.02)
        mats.append(O.quantize(w, group, bits))
    x = O.normal_bf16(9150 + T, (T, H))
    routed = O.normal_bf16(9160 + T, (T, H), 0.05)
    # more than 16 tokens on the tensor-core path: bf16-rounded weight operands
    ref = O.shared_expert(x, routed, *mats, group, bits, weights_bf16=T > 16)
    lin = [q38.QuantizedLinear(dev_u32(c), dev_bf16(s), dev_bf16(b), None, group, bits) for c, s, b in mats]
    out = q38.shared_expert(dev_bf16(x), dev_bf16(routed), *lin)
    torch.cuda.synchronize()
    q38.check_device()
    check_close(host_bf16(out), O.bf16_to_f32(ref).astype(np.float64))
    # in place on the routed buffer, through the block's own path
    r = dev_bf16(routed)
    q38.shared_expert(dev_bf16(x), r, *lin, out=r)
    torch.cuda.synchronize()
    assert torch.equal(r, out)


def test_shared_expert_rejects_mixed_quantization(q38):
    H, I = 512, 512
    c, s, b = O.quantize(O.normal_f32(9190, (I, H), 0.02), 64, 4)
    lin = q38.QuantizedLinear(dev_u32(c), dev_bf16(s), dev_bf16(b), None, 64, 4)
    c3, s3, b3 = O.quantize(O.normal_f32(9191, (1, H), 0.02), 64, 3)
    gate3 = q38.QuantizedLinear(dev_u32(c3), dev_bf16(s3), dev_bf16(b3), None, 64, 3)
    x = dev_bf16(O.normal_bf16(9192, (2, H)))
    with pytest.raises(q38.Q38Error):
        q38.shared_expert(x, x, lin, lin, lin, gate3)
