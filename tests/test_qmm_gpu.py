"""GPU parity of the quantized product and the format kernels against the CPU oracle.

Every call goes through libq38.so's C ABI (q38.py is a ctypes layer).  Bar: unpacked
codes, quantize/dequantize and the Hadamard rotation bit-exact; products within
max|y - y_oracle| <= 2e-2 * RMS(y_oracle) (fp32 accumulation on both sides).
"""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


def dev_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def dev_u32(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()


def host_bf16(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def make_weight(seed, N, K, bits, group=64):
    w = O.normal_f32(seed, (N, K), 0.02)
    return O.quantize(w, group, bits)


def check_close(y_gpu_bf16: np.ndarray, y_ref: np.ndarray, tol=TOL):
    y = O.bf16_to_f32(y_gpu_bf16).astype(np.float64)
    ref = y_ref.astype(np.float64)
    rms = np.sqrt((ref ** 2).mean())
    err = np.abs(y - ref).max()
    assert np.isfinite(y).all()
    assert err <= tol * rms, f"max err {err:.4g} > {tol} * rms {rms:.4g}"
    return err / rms


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("NK", [(200, 512), (1000, 2048), (64, 1536)])
def test_qmm_decode_parity(q38, bits, M, NK):
    N, K = NK
    c, s, b = make_weight(100 + bits, N, K, bits)
    x = O.normal_bf16(7 + M, (M, K))
    ref = O.qmm(x, c, s, b, 64, bits, f32=True)
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 64, bits)
    torch.cuda.synchronize()
    check_close(host_bf16(y), ref)


@pytest.mark.parametrize("bits", [4, 3])
def test_qmm_without_biases(q38, bits):
    N, K, M = 128, 1024, 4
    c, s, _ = make_weight(300, N, K, bits)
    x = O.normal_bf16(301, (M, K))
    ref = O.qmm(x, c, s, None, 64, bits, f32=True)
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), None, True, 64, bits)
    check_close(host_bf16(y), ref)


def test_qmm_config0_single_4bit(q38):
    """x bf16 [16, 4096], W [11008, 4096] N(0, 0.02^2) quantized 4-bit g64."""
    c, s, b = make_weight(2026, 11008, 4096, 4)
    x = O.normal_bf16(2027, (16, 4096))
    ref = O.qmm(x, c, s, b, 64, 4, f32=True)
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 64, 4)
    check_close(host_bf16(y), ref)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("NK", [(17408, 5120), (5120, 17408), (6144, 5120)])
def test_qmm_decode_sweep_shapes(q38, bits, NK):
    """The decode sweep's full shapes at M=1 and M=8."""
    N, K = NK
    c, s, b = make_weight(4000 + bits + N, N, K, bits)
    for M in (1, 8):
        x = O.normal_bf16(4100 + M, (M, K))
        ref = O.qmm(x, c, s, b, 64, bits, f32=True)
        y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 64, bits)
        check_close(host_bf16(y), ref)


@pytest.mark.parametrize("deterministic", [True, False])
def test_decode_products_repeat_across_calls(q38, deterministic):
    """Default mode: the partial sums of the k-chunks are added into a zero-at-rest region
    in arrival order, so repeats may differ by rounding (at most one bf16 ulp); leftover
    region contents would show up as errors of the size of y itself.  Deterministic mode
    (q38_ctx_set_deterministic): every chunk's sums have a slot of their own and are added
    in a fixed order, so interleaved shapes and repeats give bitwise equal results."""
    q38.set_deterministic(deterministic)
    try:
        _repeat_case(q38, deterministic)
    finally:
        q38.set_deterministic(False)


def _repeat_case(q38, exact):
    ca = make_weight(501, 5120, 17408, 4)
    cb = make_weight(502, 1000, 2048, 2)
    xa = O.normal_bf16(503, (8, 17408))
    xb = O.normal_bf16(504, (3, 2048))
    Wa = [dev_u32(ca[0]), dev_bf16(ca[1]), dev_bf16(ca[2])]
    Wb = [dev_u32(cb[0]), dev_bf16(cb[1]), dev_bf16(cb[2])]
    ya1 = q38.quantized_matmul(dev_bf16(xa), *Wa, True, 64, 4)
    yb1 = q38.quantized_matmul(dev_bf16(xb), *Wb, True, 64, 2)
    ya2 = q38.quantized_matmul(dev_bf16(xa), *Wa, True, 64, 4)
    yb2 = q38.quantized_matmul(dev_bf16(xb), *Wb, True, 64, 2)
    torch.cuda.synchronize()
    for y1, y2 in ((ya1, ya2), (yb1, yb2)):
        if exact:
            assert torch.equal(y1, y2)
        else:
            a, b = y1.float(), y2.float()
            assert ((a - b).abs() <= a.abs() * 2.0 ** -7 + 1e-6).all()
    check_close(host_bf16(ya2), O.qmm(xa, *ca, 64, 4, f32=True))
    check_close(host_bf16(yb2), O.qmm(xb, *cb, 64, 2, f32=True))
    q38.check_device()


@pytest.mark.parametrize("group,bits,K,xdt", [(32, 4, 256, torch.bfloat16), (128, 2, 512, torch.bfloat16),
                                              (64, 5, 320, torch.bfloat16), (64, 6, 192, torch.bfloat16),
                                              (64, 4, 576, torch.float16), (64, 3, 128, torch.bfloat16)])
def test_qmm_general_shapes(q38, group, bits, K, xdt):
    N, M = 96, 37
    c, s, b = make_weight(600 + bits, N, K, bits, group)
    x = O.normal_bf16(601, (M, K))
    ref = O.qmm(x, c, s, b, group, bits, f32=True)
    xt = dev_bf16(x).to(xdt)
    st, bt = dev_bf16(s).to(xdt), dev_bf16(b).to(xdt)
    y = q38.quantized_matmul(xt, dev_u32(c), st, bt, True, group, bits)
    check_close(host_bf16(y.to(torch.bfloat16)), ref)


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_unpack_codes_bit_exact(q38, bits):
    c, _, _ = make_weight(700 + bits, 37, 512, bits)
    q = q38.unpack_codes(dev_u32(c), bits).cpu().numpy()
    np.testing.assert_array_equal(q, O.unpack(c, 512, bits))


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_quantize_bit_exact(q38, bits, group):
    w = O.normal_f32(800 + bits, (45, 1024), 0.02)
    c, s, b = O.quantize(w, group, bits)
    gc, gs, gb = q38.quantize(torch.from_numpy(w).cuda(), group, bits, scales_dtype=torch.bfloat16)
    np.testing.assert_array_equal(gc.view(torch.int32).cpu().numpy().view(np.uint32), c)
    np.testing.assert_array_equal(host_bf16(gs), s)
    np.testing.assert_array_equal(host_bf16(gb), b)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_dequantize_bit_exact(q38, bits):
    c, s, b = make_weight(900 + bits, 33, 512, bits)
    d = q38.dequantize(dev_u32(c), dev_bf16(s), dev_bf16(b), 64, bits, out_dtype=torch.float32)
    np.testing.assert_array_equal(d.cpu().numpy(), O.dequantize(c, s, b, 64, bits))


@pytest.mark.parametrize("block", [4, 16, 64, 128, 256, 512, 1024, 2048, 4096, 8192])
@pytest.mark.parametrize("inverse", [False, True])
def test_hadamard_bit_exact(q38, block, inverse):
    # D = 4096 + block: the blocks do not fill the last CTA of the small-block kernel
    D = 4096 + block if block <= 4096 else block
    x = O.normal_bf16(1000 + block, (5, D))
    signs = np.where((np.arange(D) * 7) % 5 < 2, -1.0, 1.0).astype(np.float32)
    ref = O.hadamard_rotate(x, block, signs, inverse)
    y = q38.hadamard_rotate(dev_bf16(x), torch.from_numpy(signs).cuda(), block, inverse)
    np.testing.assert_array_equal(host_bf16(y), ref)
    ref0 = O.hadamard_rotate(x, block, None, inverse)
    y0 = q38.hadamard_rotate(dev_bf16(x), None, block, inverse)
    np.testing.assert_array_equal(host_bf16(y0), ref0)


def test_hadamard_unaligned_buffers(q38):
    # x and y two bytes past an 8-byte boundary: element-wise accesses instead of 8-byte ones
    block, D, rows = 256, 1024, 3
    x = O.normal_bf16(1050, (rows, D))
    xb = torch.zeros(rows * D + 1, dtype=torch.bfloat16, device="cuda")
    xb[1:] = dev_bf16(x).reshape(-1)
    xv = xb[1:].view(rows, D)
    assert xv.data_ptr() % 8 == 2
    y = q38.hadamard_rotate(xv, None, block)
    np.testing.assert_array_equal(host_bf16(y.contiguous()), O.hadamard_rotate(x, block, None))


@pytest.mark.parametrize("M", [1, 8])
def test_bonsai_hadamard_ternary_projection(q38, M):
    """Bonsai-style: ternary 2-bit codes, bias = -scale, x rotated by block-256 FWHT."""
    N, K = 1024, 5120
    c, s, b = O.ternary(1100, N, K)
    x = O.normal_bf16(1101, (M, K))
    xr = O.hadamard_rotate(x, 256, None)
    ref = O.qmm(xr, c, s, b, 64, 2, f32=True)
    lin = q38.HadamardQuantizedLinear(q38.QuantizedLinear(dev_u32(c), dev_bf16(s), dev_bf16(b), None, 64, 2),
                                      None, 256)
    y = lin(dev_bf16(x))
    check_close(host_bf16(y), ref)


def test_gather_qmm_parity(q38):
    E, N, K = 8, 96, 512
    c, s, b = make_weight(1200, E * N, K, 3)
    c, s, b = c.reshape(E, N, -1), s.reshape(E, N, -1), b.reshape(E, N, -1)
    x = O.normal_bf16(1201, (4, 2, K))
    lhs = np.array([0, 3, 1, 1, 2], np.int32)
    rhs = np.array([7, 0, 7, 2, 5], np.int32)
    ref = O.gather_qmm(x, c, s, b, lhs, rhs, 64, 3)
    out = q38.gather_qmm(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b),
                         torch.from_numpy(lhs).cuda(), torch.from_numpy(rhs).cuda(), True, 64, 3)
    for p in range(5):
        check_close(host_bf16(out[p]), O.bf16_to_f32(ref[p]).astype(np.float64), tol=2e-2)


def test_gather_qmm_bad_index_is_reported(q38):
    E, N, K = 2, 32, 128
    c, s, b = make_weight(1300, E * N, K, 4)
    x = O.normal_bf16(1301, (1, 1, K))
    rhs = torch.tensor([5], dtype=torch.int32, device="cuda")
    q38.gather_qmm(dev_bf16(x), dev_u32(c.reshape(E, N, -1)), dev_bf16(s.reshape(E, N, -1)),
                   dev_bf16(b.reshape(E, N, -1)), None, rhs, True, 64, 4)
    with pytest.raises(q38.Q38ArgumentError):
        q38.check_device()
    q38.check_device()  # cleared


def test_argument_errors(q38):
    x = torch.zeros(2, 100, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(8, 100 * 4 // 32, dtype=torch.int32, device="cuda")
    s = torch.zeros(8, 2, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(q38.Q38ArgumentError):
        q38.quantized_matmul(x, w, s, s, True, 64, 4)  # K not a multiple of the group
    with pytest.raises(q38.Q38Error):
        q38.quantized_matmul(x, w, s, s, False, 50, 4)


@pytest.mark.parametrize("NK", [(17408, 5120), (5120, 17408)])
def test_bonsai_ternary_projection_full_size(q38, NK):
    """The Bonsai ternary benchmark configuration at its full shapes: codes uniform in
    {0, 1, 2} (w in {-s, 0, +s}), bias = -scale, x rotated by the block-256 Walsh-Hadamard
    transform; M = 1 and 8 in full, M = 2048 on 6 sampled tokens (a token's output
    depends only on its own row of x)."""
    N, K = NK
    c, s, b = O.ternary(1400 + N, N, K)
    lin = q38.HadamardQuantizedLinear(q38.QuantizedLinear(dev_u32(c), dev_bf16(s), dev_bf16(b), None, 64, 2),
                                      None, 256)
    for M in (1, 8):
        x = O.normal_bf16(1401 + M, (M, K))
        ref = O.qmm(O.hadamard_rotate(x, 256, None), c, s, b, 64, 2, f32=True)
        y = lin(dev_bf16(x))
        torch.cuda.synchronize()
        check_close(host_bf16(y), ref)
    M = 2048
    x = O.normal_bf16(1410, (M, K))
    y = lin(dev_bf16(x))
    torch.cuda.synchronize()
    q38.check_device()
    rows = np.array([0, 127, 128, 1000, 2046, 2047])
    ref = O.qmm(O.hadamard_rotate(np.ascontiguousarray(x[rows]), 256, None), c, s, b, 64, 2, f32=True)
    check_close(host_bf16(y[torch.from_numpy(rows).cuda()]), ref)


@pytest.mark.parametrize("M,N,K", [(17, 256, 1024), (64, 1000, 2048), (300, 512, 5120), (600, 1280, 384)])
def test_qmm_8bit_prompt_sizes(q38, M, N, K):
    """8-bit codes with more than 16 tokens (the tensor-core prompt product; K = 384 reads
    the scales without the TMA boxes, as every 8-bit prompt product does)."""
    c, s, b = make_weight(1500 + M, N, K, 8)
    x = O.normal_bf16(1501 + M, (M, K))
    ref = O.qmm(x, c, s, b, 64, 8, f32=True)
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 64, 8)
    torch.cuda.synchronize()
    check_close(host_bf16(y), ref)
    q38.check_device()


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("M,N,K", [(300, 1024, 2048), (40, 640, 384)])
def test_qmm_group32_prompt_sizes(q38, bits, M, N, K):
    """Group 32 (the outer quantization of the published Flash-Next checkpoint) with more than
    16 tokens: the tensor-core prompt product with two scales per 64-code group."""
    c, s, b = make_weight(1700 + bits + M, N, K, bits, 32)
    x = O.normal_bf16(1701 + M, (M, K))
    ref = O.qmm(x, c, s, b, 32, bits, f32=True)
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 32, bits)
    torch.cuda.synchronize()
    check_close(host_bf16(y), ref)
    q38.check_device()


@pytest.mark.parametrize("M", [1, 8, 64])
@pytest.mark.parametrize("group,bits,xdt", [(32, 4, torch.bfloat16), (32, 3, torch.bfloat16),
                                            (64, 4, torch.float16), (128, 4, torch.bfloat16)])
def test_qmm_other_groups_and_dtypes(q38, M, group, bits, xdt):
    """Group 32 (the outer quantization of the published Flash-Next checkpoint), group 128,
    and f16 activations/scales, at decode and prompt token counts."""
    N, K = 1536, 2048
    c, s, b = make_weight(1600 + group + bits, N, K, bits, group)
    x = O.normal_bf16(1601 + M, (M, K))
    if xdt == torch.float16:
        # the oracle sees the same f16-representable values the device gets
        x = O.f32_to_bf16(torch.from_numpy(O.bf16_to_f32(x)).half().float().numpy())
        s = O.f32_to_bf16(torch.from_numpy(O.bf16_to_f32(s)).half().float().numpy())
        b = O.f32_to_bf16(torch.from_numpy(O.bf16_to_f32(b)).half().float().numpy())
    ref = O.qmm(x, c, s, b, group, bits, f32=True)
    y = q38.quantized_matmul(dev_bf16(x).to(xdt), dev_u32(c), dev_bf16(s).to(xdt), dev_bf16(b).to(xdt), True,
                             group, bits)
    torch.cuda.synchronize()
    check_close(host_bf16(y.to(torch.bfloat16)), ref)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_deterministic_mode_matches_oracle(q38, bits):
    """The ordered-sum mode at the decode sweep's shapes, M = 1 and 8, against the oracle."""
    N, K = 6144, 5120
    c, s, b = make_weight(1800 + bits, N, K, bits)
    q38.set_deterministic(True)
    try:
        for M in (1, 8):
            x = O.normal_bf16(1850 + M, (M, K))  # a seed no weight uses (equal seeds correlate x and W)
            y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 64, bits)
            torch.cuda.synchronize()
            check_close(host_bf16(y), O.qmm(x, c, s, b, 64, bits, f32=True))
    finally:
        q38.set_deterministic(False)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("P,with_lhs", [(10, True), (80, True), (7, False), (160, True)])
def test_gather_qmm_decode_path(q38, bits, P, with_lhs):
    """gatherQuantizedMM at QuantizedSwitchLinear's decode shapes (one activation row per
    token, up to 256 (token, slot) pairs): the decode kernel over the pairs' distinct
    experts, checked pair by pair against the oracle."""
    E, N, K = 64, 512, 2048
    c, s, b = make_weight(1900 + bits, E * N, K, bits)
    c, s, b = c.reshape(E, N, -1), s.reshape(E, N, -1), b.reshape(E, N, -1)
    rng = np.random.default_rng(1901 + P)
    T = max(1, P // 10) if with_lhs else P
    x = O.normal_bf16(1950 + P, (T, 1, K))
    lhs = (np.arange(P) // 10 % T).astype(np.int32) if with_lhs else None
    rhs = rng.integers(0, E, size=P).astype(np.int32)
    out = q38.gather_qmm(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b),
                         None if lhs is None else torch.from_numpy(lhs).cuda(), torch.from_numpy(rhs).cuda(),
                         True, 64, bits)
    torch.cuda.synchronize()
    q38.check_device()
    ref = O.gather_qmm(x, c, s, b, lhs if lhs is not None else np.arange(P, dtype=np.int32), rhs, 64, bits)
    # both sides round their fp32 sums to bf16: allow one bf16 step of the reference on top
    # of the bar
    y = O.bf16_to_f32(host_bf16(out)).astype(np.float64)
    r = O.bf16_to_f32(ref).astype(np.float64)
    for p in range(P):
        rms = np.sqrt((r[p] ** 2).mean())
        step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(r[p]), 2.0 ** -126))) - 7)
        assert (np.abs(y[p] - r[p]) - step).max() <= TOL * rms, p


def test_gather_qmm_decode_path_bad_index(q38):
    E, N, K = 4, 64, 512
    c, s, b = make_weight(1960, E * N, K, 4)
    x = O.normal_bf16(1961, (2, 1, K))
    rhs = torch.tensor([1, 9], dtype=torch.int32, device="cuda")
    out = q38.gather_qmm(dev_bf16(x), dev_u32(c.reshape(E, N, -1)), dev_bf16(s.reshape(E, N, -1)),
                         dev_bf16(b.reshape(E, N, -1)), None, rhs, True, 64, 4)
    with pytest.raises(q38.Q38ArgumentError):
        q38.check_device()
    assert (out[1].float() == 0).all()
    q38.check_device()


@pytest.mark.parametrize("block", [16, 256, 512, 1024])
@pytest.mark.parametrize("with_signs", [True, False])
def test_rotation_inside_decode_kernel_is_bit_identical(q38, block, with_signs):
    """Decode-shaped rotated products rotate x in the product kernel: the result equals the
    rotation kernel followed by the product, bit for bit (deterministic mode, so the two
    products add their chunk sums in the same order)."""
    N, K = 1024, 4096
    c, s, b = make_weight(2100 + block, N, K, 4)
    signs = torch.from_numpy(np.where((np.arange(K) * 5) % 7 < 3, -1.0, 1.0).astype(np.float32)).cuda() \
        if with_signs else None
    W = [dev_u32(c), dev_bf16(s), dev_bf16(b)]
    q38.set_deterministic(True)
    try:
        for M in (1, 3, 8, 16):
            x = dev_bf16(O.normal_bf16(2150 + M, (M, K)))
            lin = q38.HadamardQuantizedLinear(q38.QuantizedLinear(*W, None, 64, 4), signs, block)
            fused = lin(x)
            sep = q38.quantized_matmul(q38.hadamard_rotate(x, signs, block), *W, True, 64, 4)
            torch.cuda.synchronize()
            assert torch.equal(fused, sep), (M, block)
            xr = q38.hadamard_rotate(x, signs, block)
            check_close(host_bf16(fused), O.qmm(host_bf16(xr), c, s, b, 64, 4, f32=True))
    finally:
        q38.set_deterministic(False)


def test_quantized_matmul_into_caller_buffer(q38):
    """`out=` writes the product into a slice of a caller's buffer: the same bits as a
    freshly allocated result, and a wrongly shaped buffer is refused."""
    N, K = 1024, 2048
    c, s, b = make_weight(2300, N, K, 4)
    W = [dev_u32(c), dev_bf16(s), dev_bf16(b)]
    for M in (1, 40):
        x = dev_bf16(O.normal_bf16(2301 + M, (M, K)))
        ref = q38.quantized_matmul(x, *W, True, 64, 4)
        buf = torch.zeros(3 * M * N, dtype=torch.bfloat16, device="cuda")
        view = buf[M * N:2 * M * N].view(M, N)
        got = q38.quantized_matmul(x, *W, True, 64, 4, out=view)
        torch.cuda.synchronize()
        assert got.data_ptr() == view.data_ptr()
        assert torch.equal(view, ref)
        assert (buf[:M * N] == 0).all() and (buf[2 * M * N:] == 0).all()
    with pytest.raises(ValueError):
        q38.quantized_matmul(x, *W, True, 64, 4, out=torch.empty((M, N + 1), dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("block", [16, 256, 1024])
@pytest.mark.parametrize("with_signs", [True, False])
def test_rotation_inside_prompt_product_is_bit_identical(q38, block, with_signs):
    """Prompt-shaped rotated products rotate x in the tensor-core product's prologue: the
    result equals the rotation kernel followed by the product, bit for bit (the prompt
    product is deterministic), for groups 64, 32 and the Bonsai 2 pack's f16 group 128."""
    N, K = 1024, 4096
    signs = torch.from_numpy(np.where((np.arange(K) * 3) % 5 < 2, -1.0, 1.0).astype(np.float32)).cuda() \
        if with_signs else None
    for (group, bits, f16) in ((64, 4, False), (64, 2, False), (64, 3, False), (64, 8, False), (32, 4, False),
                               (128, 2, True)):
        c, s, b = make_weight(2400 + bits + group, N, K, bits, group)
        ts, tb = dev_bf16(s), dev_bf16(b)
        if f16:
            ts, tb = ts.half(), tb.half()
        W = [dev_u32(c), ts, tb]
        for M in (17, 300):
            x = dev_bf16(O.normal_bf16(2450 + M + block, (M, K)))
            lin = q38.HadamardQuantizedLinear(q38.QuantizedLinear(*W, None, group, bits), signs, block)
            fused = lin(x)
            sep = q38.quantized_matmul(q38.hadamard_rotate(x, signs, block), *W, True, group, bits)
            torch.cuda.synchronize()
            assert torch.equal(fused, sep), (group, bits, M, block)
    q38.check_device()
