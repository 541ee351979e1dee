// SwitchGLU expert products for few tokens (decode-sized MoE layers): every expert sees
// one or a handful of (token, slot) pairs, so the weights are streamed once and each
// weight meets only a few activations.  CUDA cores, no tensor-core handshakes:
//
//  * A CTA owns one tile = (expert e, run of <= NP pairs, block of weight rows); 8 warps.
//    One thread per weight row; the reduction dimension is split across the CTA's warps
//    (gate/up: 32 rows per CTA, 8 k-slices; down: 128 rows, 2 k-slices), partial sums are
//    added through shared memory.
//  * The run's activations (already expert-ordered, permuted and 2^-p-scaled like the
//    tensor-core path) are staged in shared memory; all lanes of a warp read the same
//    activation words (broadcast).
//  * Codes become exact bf16 weights exactly as in the tensor-core path (magic-number
//    extraction, bf16x2 subtract and fused multiply-add, one rounding of s*q + b), and
//    mixed-precision FMAs (bf16 operands, fp32 accumulation, every product exact) add
//    weight x activation: the same products as the tensor cores form, in another order.
//  * gate/up tiles hold the gate row and the up row of the same index in one thread, which
//    forms h = bf16(silu(bf16 g) * bf16 u) and writes it permuted for the down projection;
//    down tiles write y = bf16(h . Wd^T) per pair.
#include "moe_internal.h"
#include "tc_pipeline.cuh"

namespace q38 {
namespace {

constexpr int MG_NP = 8;        // pairs per run
constexpr int MG_WIN = 16;      // 16-code windows per thread slice (256 k)
constexpr int MG_THREADS = 256;

__device__ __forceinline__ float fma_bf16(uint32_t a_half_lo_hi, uint32_t b_half_lo_hi, float c, bool hi) {
    float d;
    if (hi) {
        asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
            "fma.rn.f32.bf16 %0, ah, bh, %3;\n\t}"
            : "=f"(d) : "r"(a_half_lo_hi), "r"(b_half_lo_hi), "f"(c));
    } else {
        asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
            "fma.rn.f32.bf16 %0, al, bl, %3;\n\t}"
            : "=f"(d) : "r"(a_half_lo_hi), "r"(b_half_lo_hi), "f"(c));
    }
    return d;
}

// Window wl (16 codes) of a slice held in registers -> 8 bf16x2 operands.
template <int BITS>
__device__ __forceinline__ void slice_window(const uint32_t* c, int wl, uint32_t* v) {
    uint32_t win[2];
    if constexpr (BITS == 2) {
        win[0] = c[wl];
    } else if constexpr (BITS == 4) {
        win[0] = c[2 * wl];
        win[1] = c[2 * wl + 1];
    } else {
        const int k0 = (3 * wl) >> 1;
        if (wl & 1) {
            win[0] = __funnelshift_r(c[k0], c[k0 + 1], 16);
            win[1] = c[k0 + 1] >> 16;
        } else {
            win[0] = c[k0];
            win[1] = c[k0 + 1];
        }
    }
    extract<BITS>(win, v);
}

template <int BITS, bool GATE_UP>
__global__ void __launch_bounds__(MG_THREADS) moe_gemv_kernel(
    const __nv_bfloat16* __restrict__ xs, int K, const MoeTile* __restrict__ tiles, const int* __restrict__ ntiles,
    const uint32_t* __restrict__ w0, const uint32_t* __restrict__ w1, const uint16_t* __restrict__ s0,
    const uint16_t* __restrict__ s1, const uint16_t* __restrict__ b0, const uint16_t* __restrict__ b1,
    int rows_per_expert, __nv_bfloat16* __restrict__ out, int out_ld) {
    // Slices of 256 k per row: KS = K / 256; the 8 warps split as KW k-warps x RW row-warps.
    const int KS = K / (16 * MG_WIN);
    const int KW = KS < 8 ? KS : 8, RW = 8 / KW;
    extern __shared__ __align__(16) uint8_t sm[];
    griddep_wait();
    griddep_launch_dependents();
    if (static_cast<int>(blockIdx.x) >= *ntiles) return;
    const MoeTile t = tiles[blockIdx.x];
    const int nw = K / 16;  // code windows per row
    uint32_t* xsm = reinterpret_cast<uint32_t*>(sm);                   // [NP][K/2] bf16x2
    float* red = reinterpret_cast<float*>(sm + MG_NP * K * 2);         // [8 warps][32][2][NP]

    // stage the run's activations
    const int np = t.np;
    for (int i = threadIdx.x; i < np * (K / 8); i += MG_THREADS) {
        const int p = i / (K / 8), c = i % (K / 8);
        reinterpret_cast<uint4*>(xsm)[p * (K / 8) + c] =
            __ldg(reinterpret_cast<const uint4*>(xs + static_cast<size_t>(t.p0 + p) * K) + c);
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rw = warp % RW, kw = warp / RW;
    const int r = t.rb * (32 * RW) + rw * 32 + lane;  // row within the expert
    const int G = K / 64;
    const size_t grow = static_cast<size_t>(t.e) * rows_per_expert + r;
    const int kwords = K * BITS / 32;
    const uint32_t* c0 = w0 + grow * kwords;
    const uint32_t* c1 = GATE_UP ? w1 + grow * kwords : nullptr;
    float acc0[MG_NP], acc1[MG_NP];
#pragma unroll
    for (int p = 0; p < MG_NP; ++p) acc0[p] = acc1[p] = 0.f;
    // This thread's slice: MG_WIN windows of 16 codes (MG_WIN/4 groups), loaded up front as
    // 16-byte vectors so that one memory latency covers the whole slice.
    constexpr int SW_WORDS = MG_WIN * BITS / 2;  // code words of the slice
    for (int slice = kw; slice < KS; slice += KW) {
    const int wb = slice * MG_WIN;
    uint32_t ca[SW_WORDS], cb[GATE_UP ? SW_WORDS : 1];
    {
        const uint4* pa = reinterpret_cast<const uint4*>(c0 + wb * BITS / 2);
#pragma unroll
        for (int i = 0; i < SW_WORDS / 4; ++i) {
            const uint4 u = __ldg(pa + i);
            ca[4 * i] = u.x; ca[4 * i + 1] = u.y; ca[4 * i + 2] = u.z; ca[4 * i + 3] = u.w;
        }
        if constexpr (GATE_UP) {
            const uint4* pb = reinterpret_cast<const uint4*>(c1 + wb * BITS / 2);
#pragma unroll
            for (int i = 0; i < SW_WORDS / 4; ++i) {
                const uint4 u = __ldg(pb + i);
                cb[4 * i] = u.x; cb[4 * i + 1] = u.y; cb[4 * i + 2] = u.z; cb[4 * i + 3] = u.w;
            }
        }
    }
    constexpr int NG = MG_WIN / 4;
    uint32_t sga[NG], bga[NG], sgb[NG], bgb[NG];
#pragma unroll
    for (int i = 0; i < NG; ++i) {
        const size_t gi = grow * G + wb / 4 + i;
        sga[i] = __ldg(s0 + gi);
        bga[i] = b0 ? __ldg(b0 + gi) : 0u;
        if constexpr (GATE_UP) {
            sgb[i] = __ldg(s1 + gi);
            bgb[i] = b1 ? __ldg(b1 + gi) : 0u;
        }
    }
#pragma unroll
    for (int i = 0; i < NG; ++i) {
        const uint32_t s2a = sga[i] * 0x10001u, s2b = GATE_UP ? sgb[i] * 0x10001u : 0u;
        uint32_t b2a[8], b2b[8];
        const float bfa = bf16_bits_to_f32(bga[i]), bfb = GATE_UP ? bf16_bits_to_f32(bgb[i]) : 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            b2a[q] = (__float_as_uint(bfa * (1.0f / pair_mult<BITS>(q, 0))) >> 16) |
                     (__float_as_uint(bfa * (1.0f / pair_mult<BITS>(q, 1))) & 0xFFFF0000u);
            b2b[q] = (__float_as_uint(bfb * (1.0f / pair_mult<BITS>(q, 0))) >> 16) |
                     (__float_as_uint(bfb * (1.0f / pair_mult<BITS>(q, 1))) & 0xFFFF0000u);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int wl = 4 * i + j, w = wb + wl;
            uint32_t va[8], vb[8];
            slice_window<BITS>(ca, wl, va);
#pragma unroll
            for (int q = 0; q < 8; ++q) va[q] = bf2_fma(bf2_sub(va[q], MAGIC), s2a, b2a[q]);
            if constexpr (GATE_UP) {
                slice_window<BITS>(cb, wl, vb);
#pragma unroll
                for (int q = 0; q < 8; ++q) vb[q] = bf2_fma(bf2_sub(vb[q], MAGIC), s2b, b2b[q]);
            }
#pragma unroll
            for (int p = 0; p < MG_NP; ++p) {
                if (p < np) {
                    const uint4* xq = reinterpret_cast<const uint4*>(xsm + p * (K / 2) + w * 8);
                    const uint4 xa = xq[0], xb = xq[1];
                    const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        acc0[p] = fma_bf16(va[q], xw[q], acc0[p], false);
                        acc0[p] = fma_bf16(va[q], xw[q], acc0[p], true);
                        if constexpr (GATE_UP) {
                            acc1[p] = fma_bf16(vb[q], xw[q], acc1[p], false);
                            acc1[p] = fma_bf16(vb[q], xw[q], acc1[p], true);
                        }
                    }
                }
            }
        }
    }
    }  // slices
    // reduce the k-slices through shared memory
    const int slot = (warp * 32 + lane) * 2 * MG_NP;
#pragma unroll
    for (int p = 0; p < MG_NP; ++p) {
        red[slot + p] = acc0[p];
        red[slot + MG_NP + p] = acc1[p];
    }
    __syncthreads();
    if (kw != 0) return;
    float f0[MG_NP], f1[MG_NP];
#pragma unroll
    for (int p = 0; p < MG_NP; ++p) f0[p] = f1[p] = 0.f;
    for (int k2 = 0; k2 < KW; ++k2) {
        const int sl = ((k2 * RW + rw) * 32 + lane) * 2 * MG_NP;
#pragma unroll
        for (int p = 0; p < MG_NP; ++p) {
            f0[p] += red[sl + p];
            f1[p] += red[sl + MG_NP + p];
        }
    }
    if constexpr (GATE_UP) {
        const int g64 = r & ~63, c = r & 15, tq = (r & 63) >> 4;
        const int pos = g64 + 16 * tq + window_slot<BITS>(c);
        const float mult = window_mult<BITS>(c);
#pragma unroll
        for (int p = 0; p < MG_NP; ++p) {
            if (p < np) {
                const float gv = bf16_bits_to_f32(f32_to_bf16_bits(f0[p]));
                const float uv = bf16_bits_to_f32(f32_to_bf16_bits(f1[p]));
                const float h = bf16_bits_to_f32(f32_to_bf16_bits(gv / (1.0f + expf(-gv)) * uv));
                out[static_cast<size_t>(t.p0 + p) * out_ld + pos] = __float2bfloat16_rn(h * mult);
            }
        }
    } else {
#pragma unroll
        for (int p = 0; p < MG_NP; ++p)
            if (p < np) out[static_cast<size_t>(t.p0 + p) * out_ld + r] = __float2bfloat16_rn(f0[p]);
    }
}

template <int BITS, bool GATE_UP>
q38_status launch_mg(q38_ctx* ctx, const GroupedProblem& p) {
    const size_t smem = static_cast<size_t>(MG_NP) * p.K * 2 + static_cast<size_t>(8) * 32 * 2 * MG_NP * 4;
    auto kern = moe_gemv_kernel<BITS, GATE_UP>;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
        return check_launch(ctx, "cudaFuncSetAttribute");
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.max_tiles));
    cfg.blockDim = dim3(MG_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, static_cast<const __nv_bfloat16*>(p.x), p.K, p.tiles, p.ntiles, p.w0, p.w1,
                           static_cast<const uint16_t*>(p.s0), static_cast<const uint16_t*>(p.s1),
                           static_cast<const uint16_t*>(p.b0), static_cast<const uint16_t*>(p.b1), p.rows_per_expert,
                           static_cast<__nv_bfloat16*>(p.out), p.out_ld) != cudaSuccess)
        return check_launch(ctx, "moe_gemv");
    return check_launch(ctx, "moe_gemv");
}

}  // namespace

int moe_gemv_run_pairs() { return MG_NP; }

int moe_gemv_rows_per_tile(int64_t K) {
    const int64_t ks = K / (16 * MG_WIN);
    return 32 * static_cast<int>(8 / (ks < 8 ? ks : 8));
}

q38_status moe_gemv_gate_up(q38_ctx* ctx, const GroupedProblem& p, int bits) {
    switch (bits) {
        case 2: return launch_mg<2, true>(ctx, p);
        case 3: return launch_mg<3, true>(ctx, p);
        default: return launch_mg<4, true>(ctx, p);
    }
}

q38_status moe_gemv_down(q38_ctx* ctx, const GroupedProblem& p, int bits) {
    switch (bits) {
        case 2: return launch_mg<2, false>(ctx, p);
        case 3: return launch_mg<3, false>(ctx, p);
        default: return launch_mg<4, false>(ctx, p);
    }
}

}  // namespace q38
