"""GPU parity of q38_quantized_gate_up: h = bf16(silu(bf16(x.Wg^T)) * bf16(x.Wu^T)).

Checked against (1) the same computation composed from the existing operators
(quantized_matmul twice, then silu_mul): the fused decode pass sums the fp32 partials in
a different order than two separate products, so a bf16 output may differ by one
representable step; bar max|h - h_ref| <= 2e-2 * RMS(h_ref) + one bf16 step of |h_ref|,
the bar of the SwitchGLU tests.  (2) The CPU oracle's two products passed through the
same roundings: g and u may each differ from the oracle by the product bar (2e-2 * RMS
plus one bf16 step), and h = silu(g) * u carries both, so each element of h must lie
within those input errors propagated to first order,
  |silu'(g) * u| * (2e-2 RMS(g) + step(g)) + |silu(g)| * (2e-2 RMS(u) + step(u)) + step(h),
and the RMS of the error must stay below 1e-2 * RMS(h).  Repeated calls must give the same
result (the partial-sum workspace is returned to zero by every call).
"""
import numpy as np
import pytest
import torch

import oracle as O
from test_qmm_gpu import dev_bf16, dev_u32, host_bf16, make_weight

pytestmark = pytest.mark.gpu


def bf16_round(a):
    return O.bf16_to_f32(O.f32_to_bf16(np.asarray(a, np.float32))).astype(np.float64)


def check_h(h, ref):
    h = O.bf16_to_f32(h).astype(np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt((ref ** 2).mean())
    step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -126))) - 7)
    assert np.isfinite(h).all()
    excess = (np.abs(h - ref) - step).max()
    assert excess <= 2e-2 * rms, f"max excess {excess:.4g} > 2e-2 * rms {rms:.4g}"


def step_of(v):
    return 2.0 ** (np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -126))) - 7)


def check_oracle(h, gu):
    g, u = gu
    sig = 1.0 / (1.0 + np.exp(-g))
    ref = g * sig * u
    dsilu = sig * (1.0 + g * (1.0 - sig))
    rms_g, rms_u = np.sqrt((g ** 2).mean()), np.sqrt((u ** 2).mean())
    bound = (np.abs(dsilu * u) * (2e-2 * rms_g + step_of(g)) + np.abs(g * sig) * (2e-2 * rms_u + step_of(u))
             + step_of(ref))
    h = O.bf16_to_f32(h).astype(np.float64)
    assert np.isfinite(h).all()
    worst = (np.abs(h - ref) / bound).max()
    assert worst <= 1.0, f"an element exceeds its propagated bound by {worst:.3g}x"
    rms = np.sqrt((ref ** 2).mean())
    erms = np.sqrt(((h - ref) ** 2).mean())
    assert erms <= 1e-2 * rms, f"error rms {erms:.4g} > 1e-2 * rms {rms:.4g}"


def oracle_gate_up(x, gate, up, bits):
    g = bf16_round(O.qmm(x, *gate, 64, bits, f32=True))
    u = bf16_round(O.qmm(x, *up, 64, bits, f32=True))
    return g, u


def run(q38, bits, M, N, K, biased=True, seed=0):
    gate = make_weight(300 + seed + bits, N, K, bits)
    up = make_weight(400 + seed + bits, N, K, bits)
    if not biased:
        gate, up = (gate[0], gate[1], None), (up[0], up[1], None)
    x = O.normal_bf16(500 + seed + M, (M, K))
    dg = (dev_u32(gate[0]), dev_bf16(gate[1]), None if gate[2] is None else dev_bf16(gate[2]))
    du = (dev_u32(up[0]), dev_bf16(up[1]), None if up[2] is None else dev_bf16(up[2]))
    dx = dev_bf16(x)
    h = q38.quantized_gate_up(dx, dg, du, 64, bits)
    h2 = q38.quantized_gate_up(dx, dg, du, 64, bits)
    comp = q38.silu_mul(q38.quantized_matmul(dx, *dg, True, 64, bits), q38.quantized_matmul(dx, *du, True, 64, bits))
    torch.cuda.synchronize()
    q38.check_device()
    return x, gate, up, host_bf16(h), host_bf16(h2), host_bf16(comp)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("M", [1, 3, 8, 16])
@pytest.mark.parametrize("NK", [(200, 512), (1000, 2048)])
def test_gate_up_decode(q38, bits, M, NK):
    N, K = NK
    x, gate, up, h, h2, comp = run(q38, bits, M, N, K)
    check_h(h, O.bf16_to_f32(comp))
    check_h(h2, O.bf16_to_f32(comp))
    check_oracle(h, oracle_gate_up(x, gate, up, bits))


@pytest.mark.parametrize("bits", [4, 3])
def test_gate_up_without_biases(q38, bits):
    x, gate, up, h, h2, comp = run(q38, bits, 2, 384, 1024, biased=False, seed=7)
    check_h(h, O.bf16_to_f32(comp))
    check_oracle(h, oracle_gate_up(x, gate, up, bits))


@pytest.mark.parametrize("bits", [2, 4])
def test_gate_up_prompt_sized(q38, bits):
    # 64 tokens: the two products and the SiLU product run in sequence
    x, gate, up, h, h2, comp = run(q38, bits, 64, 512, 1024, seed=11)
    assert np.array_equal(h, comp)
    check_oracle(h, oracle_gate_up(x, gate, up, bits))


def test_gate_up_rejects_mixed_biases(q38):
    gate = make_weight(1, 128, 512, 4)
    up = make_weight(2, 128, 512, 4)
    dg = (dev_u32(gate[0]), dev_bf16(gate[1]), dev_bf16(gate[2]))
    du = (dev_u32(up[0]), dev_bf16(up[1]), None)
    with pytest.raises(ValueError):
        q38.quantized_gate_up(dev_bf16(O.normal_bf16(3, (1, 512))), dg, du, 64, 4)


def pack_weight(seed, N, K):
    """Bonsai 2 pack layout on the device: ternary 2-bit codes, f16 scales, biases = -scales,
    groups of 128."""
    rng = np.random.default_rng(seed)
    codes = O.pack(rng.integers(0, 3, size=(N, K)).astype(np.uint8), 2)
    s = (np.abs(rng.normal(0, 0.02, size=(N, K // 128))) + 1e-3).astype(np.float16)
    return dev_u32(codes), torch.from_numpy(s).cuda(), torch.from_numpy(-s).cuda()


def composition(q38, x, gate, up, group, bits, signs=None, block=None):
    xr = x if block is None else q38.hadamard_rotate(x, signs, block)
    return q38.silu_mul(q38.quantized_matmul(xr, *gate, True, group, bits),
                        q38.quantized_matmul(xr, *up, True, group, bits))


@pytest.mark.parametrize("M", [1, 8, 16])
def test_gate_up_pack_layout(q38, M):
    # one pass over two weights in the pack's layout (f16 scales, group 128)
    N, K = 1000, 2048
    gate, up = pack_weight(31, N, K), pack_weight(32, N, K)
    x = dev_bf16(O.normal_bf16(33 + M, (M, K)))
    h = q38.quantized_gate_up(x, gate, up, 128, 2)
    comp = composition(q38, x, gate, up, 128, 2)
    torch.cuda.synchronize()
    q38.check_device()
    check_h(host_bf16(h), O.bf16_to_f32(host_bf16(comp)))


@pytest.mark.parametrize("layout", ["group64", "pack"])
@pytest.mark.parametrize("M", [1, 8, 32])
def test_hadamard_gate_up(q38, layout, M):
    # one rotation shared by gate and up; M = 32 takes the two products and the SiLU product,
    # whose up product follows the rotated x in the activation buffer
    N, K = 768, 2048
    if layout == "pack":
        gate, up, group, block = pack_weight(41, N, K), pack_weight(42, N, K), 128, 1024
    else:
        g, u = O.ternary(43, N, K), O.ternary(44, N, K)
        gate = (dev_u32(g[0]), dev_bf16(g[1]), dev_bf16(g[2]))
        up = (dev_u32(u[0]), dev_bf16(u[1]), dev_bf16(u[2]))
        group, block = 64, 256
    signs = torch.from_numpy(np.where(np.random.default_rng(45).random(K) < 0.5, -1.0, 1.0).astype(np.float32)).cuda()
    x = dev_bf16(O.normal_bf16(46 + M, (M, K)))
    h = q38.hadamard_quantized_gate_up(x, signs, block, gate, up, group, 2)
    h2 = q38.hadamard_quantized_gate_up(x, signs, block, gate, up, group, 2)
    comp = composition(q38, x, gate, up, group, 2, signs, block)
    torch.cuda.synchronize()
    q38.check_device()
    if M > 16:
        assert torch.equal(h, comp) and torch.equal(h2, comp)
    else:
        check_h(host_bf16(h), O.bf16_to_f32(host_bf16(comp)))
        check_h(host_bf16(h2), O.bf16_to_f32(host_bf16(comp)))


@pytest.mark.parametrize("kind", ["plain", "rotated", "rotated_distinct_signs"])
def test_quantized_mlp_module(q38, kind):
    # the module's fused paths against the composition of its projections
    D, F, M = 1024, 2048, 3
    if kind == "plain":
        w = [make_weight(50 + i, n, k, 4) for i, (n, k) in enumerate(((F, D), (F, D), (D, F)))]
        lins = [q38.QuantizedLinear(dev_u32(c), dev_bf16(s), dev_bf16(b), None, 64, 4) for (c, s, b) in w]
    else:
        rng = np.random.default_rng(55)
        signs = lambda n: torch.from_numpy(np.where(rng.random(n) < 0.5, -1.0, 1.0).astype(np.float32)).cuda()
        sd = signs(D)
        lins = []
        for i, (n, k) in enumerate(((F, D), (F, D), (D, F))):
            c, s, b = pack_weight(56 + i, n, k)
            sg = sd if (k == D and not (kind == "rotated_distinct_signs" and i == 1)) else signs(k)
            lins.append(q38.HadamardQuantizedLinear(q38.QuantizedLinear(c, s, b, None, 128, 2), sg, 1024))
    mlp = q38.QuantizedMLP(*lins)
    assert mlp._fused == (kind != "rotated_distinct_signs")
    x = dev_bf16(O.normal_bf16(57, (M, D)))
    y = mlp(x)
    ref = lins[2](q38.silu_mul(lins[0](x), lins[1](x)))
    torch.cuda.synchronize()
    q38.check_device()
    if kind == "rotated_distinct_signs":
        assert torch.equal(y, ref)
    else:
        check_h(host_bf16(y), O.bf16_to_f32(host_bf16(ref)))
