// MLX affine format kernels: quantize, dequantize, unpack, and the general-shape
// quantized product used where the decode fast path does not apply.
//
// Format (Sources/Qwen38Core/FlashNext/Qwen4ExpPrequantized.swift:60-72, :86-96): codes
// uint32 [rows, K*bits/32], code k of a row at bit k*bits of the row's little-endian
// bitstream; scales/biases [rows, K/group]; w = scale*q + bias.
#include "affine_scalar.cuh"
#include "ptx.cuh"

namespace q38 {
namespace {

using namespace dev;

// ------------------------------------------------------------------------ unpack
__global__ void unpack_kernel(const uint32_t* __restrict__ w, int64_t rows, int64_t K, int bits,
                              uint8_t* __restrict__ q) {
    const int64_t n = rows * K;
    const int64_t kw = K * bits / 32;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / K, k = i % K;
        q[i] = static_cast<uint8_t>(get_code(w + r * kw, k, bits));
    }
}

// -------------------------------------------------------------------- dequantize
// scale*q + bias with separately rounded multiply and add (no contraction), the same
// operation sequence as the CPU restatement, so fp32 results agree bit for bit.
template <typename ST, typename OT>
__global__ void dequant_kernel(const uint32_t* __restrict__ w, const ST* __restrict__ s,
                               const ST* __restrict__ b, int64_t rows, int64_t K, int group,
                               int bits, OT* __restrict__ out) {
    const int64_t n = rows * K;
    const int64_t kw = K * bits / 32, G = K / group;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / K, k = i % K;
        const float sc = to_f32(s[r * G + k / group]);
        const float bi = b ? to_f32(b[r * G + k / group]) : 0.0f;
        const float q = static_cast<float>(get_code(w + r * kw, k, bits));
        out[i] = from_f32<OT>(__fadd_rn(__fmul_rn(sc, q), bi));
    }
}

// ------------------------------------------------------------------- embedding
// out[t, :] = dequant(row ids[t]) with the arithmetic of dequant_kernel (so a gathered row
// equals the dequantized table's row bit for bit).  An id outside [0, rows) yields a zero
// row and sets the device status bit for an out-of-range index.
template <typename ST, typename OT>
__global__ void embed_kernel(const int32_t* __restrict__ ids, int64_t n, const uint32_t* __restrict__ w,
                             const ST* __restrict__ s, const ST* __restrict__ b, int64_t rows, int64_t K,
                             int group, int bits, OT* __restrict__ out, uint32_t* status) {
    const int64_t total = n * K;
    const int64_t kw = K * bits / 32, G = K / group;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / K, k = i % K;
        const int64_t r = ids[t];
        if (r < 0 || r >= rows) {
            out[i] = from_f32<OT>(0.0f);
            if (k == 0) atomicOr(status, Q38_DEV_BAD_INDEX);
            continue;
        }
        const float sc = to_f32(s[r * G + k / group]);
        const float bi = b ? to_f32(b[r * G + k / group]) : 0.0f;
        const float q = static_cast<float>(get_code(w + r * kw, k, bits));
        out[i] = from_f32<OT>(__fadd_rn(__fmul_rn(sc, q), bi));
    }
}

// 2-, 4- and 8-bit codes: one thread per 32-bit code word (its 32/BITS codes share a group),
// the same arithmetic as embed_kernel, outputs written as 16- or 8-byte stores when `vec`
// (16-byte aligned output, rows a multiple of 16 bytes).  Grid: x over the words of a row,
// y over the ids.
template <typename ST, typename OT, int BITS>
__global__ void __launch_bounds__(128) embed_word_kernel(const int32_t* __restrict__ ids, int64_t n,
                                                         const uint32_t* __restrict__ w, const ST* __restrict__ s,
                                                         const ST* __restrict__ b, int64_t rows, int64_t K, int group,
                                                         bool vec, OT* __restrict__ out, uint32_t* status) {
    constexpr int CPW = 32 / BITS;
    constexpr int BYTES = CPW * static_cast<int>(sizeof(OT));
    const int64_t kw = K / CPW;
    const int64_t wi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (wi >= kw) return;
    const int64_t k0 = wi * CPW, G = K / group, gi = k0 / group;
    for (int64_t t = blockIdx.y; t < n; t += gridDim.y) {
        const int64_t r = ids[t];
        __align__(16) OT o[CPW];
        if (r < 0 || r >= rows) {
#pragma unroll
            for (int c = 0; c < CPW; ++c) o[c] = from_f32<OT>(0.0f);
            if (wi == 0) atomicOr(status, Q38_DEV_BAD_INDEX);
        } else {
            const uint32_t word = w[r * kw + wi];
            const float sc = to_f32(s[r * G + gi]);
            const float bi = b ? to_f32(b[r * G + gi]) : 0.0f;
#pragma unroll
            for (int c = 0; c < CPW; ++c) {
                const float q = static_cast<float>((word >> (c * BITS)) & ((1u << BITS) - 1u));
                o[c] = from_f32<OT>(__fadd_rn(__fmul_rn(sc, q), bi));
            }
        }
        OT* dst = out + t * K + k0;
        if (BYTES % 16 == 0 && vec) {
#pragma unroll
            for (int v = 0; v < BYTES / 16; ++v)
                reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(o)[v];
        } else if (BYTES % 8 == 0 && vec) {
#pragma unroll
            for (int v = 0; v < BYTES / 8; ++v)
                reinterpret_cast<uint2*>(dst)[v] = reinterpret_cast<const uint2*>(o)[v];
        } else {
#pragma unroll
            for (int c = 0; c < CPW; ++c) dst[c] = o[c];
        }
    }
}

// ---------------------------------------------------------------------- quantize
// One thread per group.  MLX affine rule (MLX C++ 0.31 affine quantize, called through
// mx.quantize at Scripts/qwen4-exp-requantize-experts.py:246-251): the extreme of larger
// magnitude ("edge") is exactly representable: scale = edge / rint(edge / scale0),
// bias = edge; q = clamp(rint((w - bias) / scale), 0, 2^bits - 1) with the fp32
// scale/bias, which are then stored in the scales dtype.  IEEE division and rint make
// the result identical to the CPU restatement.
template <typename WT, typename ST>
__global__ void quant_kernel(const WT* __restrict__ w, int64_t rows, int64_t K, int group, int bits,
                             uint32_t* __restrict__ codes, ST* __restrict__ s, ST* __restrict__ b) {
    const int64_t G = K / group;
    const int64_t ngroups = rows * G;
    const float n_bins = static_cast<float>((1 << bits) - 1);
    const float eps = 1e-7f;
    for (int64_t gid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gid < ngroups;
         gid += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = gid / G, g = gid % G;
        const WT* wg = w + r * K + g * group;
        float wmin = INFINITY, wmax = -INFINITY;
        for (int j = 0; j < group; ++j) {
            const float v = to_f32(wg[j]);
            wmax = fmaxf(wmax, v);
            wmin = fminf(wmin, v);
        }
        const bool mask = fabsf(wmin) > fabsf(wmax);
        float scale = fmaxf(__fdiv_rn(wmax - wmin, n_bins), eps);
        scale = mask ? scale : -scale;
        const float edge = mask ? wmin : wmax;
        const float q0 = rintf(__fdiv_rn(edge, scale));
        float bias = 0.0f;
        if (q0 != 0.0f) {
            scale = __fdiv_rn(edge, q0);
            bias = edge;
        }
        s[gid] = from_f32<ST>(scale);
        b[gid] = from_f32<ST>(bias);
        // codes of this group occupy bits [g*group*bits, (g+1)*group*bits) of the row;
        // group*bits is a multiple of 32 for every supported (group, bits) pair.
        uint32_t* row = codes + r * (K * bits / 32) + (g * group * bits) / 32;
        uint64_t accw = 0;
        int nacc = 0, wo = 0;
        for (int j = 0; j < group; ++j) {
            float v = rintf(__fdiv_rn(to_f32(wg[j]) - bias, scale));
            v = fminf(fmaxf(v, 0.0f), n_bins);
            accw |= static_cast<uint64_t>(static_cast<uint32_t>(v)) << nacc;
            nacc += bits;
            if (nacc >= 32) {
                row[wo++] = static_cast<uint32_t>(accw);
                accw >>= 32;
                nacc -= 32;
            }
        }
    }
}

// ------------------------------------------------------------- generic product
// One warp per output row n and 8 tokens; lanes stride over K.  Used for shapes and
// dtypes outside the fast paths (odd K, group 32/128, bits 5/6, f16).
template <typename XT, typename ST>
__global__ void __launch_bounds__(256) qmm_generic_kernel(const XT* __restrict__ x, int64_t M,
                                                          int64_t K, const uint32_t* __restrict__ w,
                                                          const ST* __restrict__ s,
                                                          const ST* __restrict__ b, int64_t N,
                                                          int group, int bits, XT* __restrict__ y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n = blockIdx.x * 8LL + warp;
    const int64_t m0 = blockIdx.y * 8LL;
    if (n >= N) return;
    const int64_t kw = K * bits / 32, G = K / group;
    const uint32_t* wr = w + n * kw;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t k = lane; k < K; k += 32) {
        const int64_t gi = k / group;
        const float wv = to_f32(s[n * G + gi]) * static_cast<float>(get_code(wr, k, bits)) +
                         (b ? to_f32(b[n * G + gi]) : 0.0f);
#pragma unroll
        for (int mi = 0; mi < 8; ++mi)
            if (m0 + mi < M) acc[mi] = fmaf(to_f32(x[(m0 + mi) * K + k]), wv, acc[mi]);
    }
#pragma unroll
    for (int mi = 0; mi < 8; ++mi) {
        float v = acc[mi];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && m0 + mi < M) y[(m0 + mi) * N + n] = from_f32<XT>(v);
    }
}

// Gathered variant: blockIdx.y enumerates (output p, 8-token chunk).  An index outside
// [0, Bx) or [0, E) writes zeros for that output and raises Q38_DEV_BAD_INDEX.
template <typename XT, typename ST>
__global__ void __launch_bounds__(256) gather_generic_kernel(
    const XT* __restrict__ x, int64_t Bx, int64_t M, int64_t K, const uint32_t* __restrict__ w,
    const ST* __restrict__ s, const ST* __restrict__ b, int64_t E, int64_t N,
    const int32_t* __restrict__ lhs, const int32_t* __restrict__ rhs, int group, int bits,
    XT* __restrict__ out, uint32_t* status) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n = blockIdx.x * 8LL + warp;
    const int64_t mchunks = (M + 7) / 8;
    const int64_t p = blockIdx.y / mchunks;
    const int64_t m0 = (blockIdx.y % mchunks) * 8;
    if (n >= N) return;
    const int64_t li = lhs ? lhs[p] : p;
    const int64_t e = rhs[p];
    XT* y = out + p * M * N;
    if (li < 0 || li >= Bx || e < 0 || e >= E) {
        if (lane == 0) {
            for (int mi = 0; mi < 8; ++mi)
                if (m0 + mi < M) y[(m0 + mi) * N + n] = from_f32<XT>(0.0f);
            if (n == 0 && m0 == 0) atomicOr(status, Q38_DEV_BAD_INDEX);
        }
        return;
    }
    const int64_t kw = K * bits / 32, G = K / group;
    const uint32_t* wr = w + (e * N + n) * kw;
    const ST* sr = s + (e * N + n) * G;
    const ST* br = b ? b + (e * N + n) * G : nullptr;
    const XT* xb = x + li * M * K;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t k = lane; k < K; k += 32) {
        const int64_t gi = k / group;
        const float wv = to_f32(sr[gi]) * static_cast<float>(get_code(wr, k, bits)) + (br ? to_f32(br[gi]) : 0.0f);
#pragma unroll
        for (int mi = 0; mi < 8; ++mi)
            if (m0 + mi < M) acc[mi] = fmaf(to_f32(xb[(m0 + mi) * K + k]), wv, acc[mi]);
    }
#pragma unroll
    for (int mi = 0; mi < 8; ++mi) {
        float v = acc[mi];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && m0 + mi < M) y[(m0 + mi) * N + n] = from_f32<XT>(v);
    }
}

int grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    if (g > 148 * 64) g = 148 * 64;
    return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

q38_status unpack_launch(q38_ctx* ctx, const uint32_t* w, int64_t rows, int64_t K, int bits,
                         uint8_t* q) {
    unpack_kernel<<<grid_for(rows * K, 256), 256, 0, ctx->stream>>>(w, rows, K, bits, q);
    return check_launch(ctx, "unpack");
}

q38_status dequantize_launch(q38_ctx* ctx, const uint32_t* w, const void* s, const void* b,
                             q38_dtype sd, int64_t rows, int64_t K, int group, int bits,
                             void* out, q38_dtype od) {
    const int grid = grid_for(rows * K, 256);
#define Q38_DQ(ST, OT)                                                                    \
    dequant_kernel<ST, OT><<<grid, 256, 0, ctx->stream>>>(                                \
        w, static_cast<const ST*>(s), static_cast<const ST*>(b), rows, K, group, bits, \
        static_cast<OT*>(out))
    if (sd == Q38_BF16) {
        if (od == Q38_BF16) Q38_DQ(__nv_bfloat16, __nv_bfloat16);
        else if (od == Q38_F16) Q38_DQ(__nv_bfloat16, __half);
        else Q38_DQ(__nv_bfloat16, float);
    } else if (sd == Q38_F16) {
        if (od == Q38_BF16) Q38_DQ(__half, __nv_bfloat16);
        else if (od == Q38_F16) Q38_DQ(__half, __half);
        else Q38_DQ(__half, float);
    } else {
        if (od == Q38_BF16) Q38_DQ(float, __nv_bfloat16);
        else if (od == Q38_F16) Q38_DQ(float, __half);
        else Q38_DQ(float, float);
    }
#undef Q38_DQ
    return check_launch(ctx, "dequantize");
}

q38_status embedding_launch(q38_ctx* ctx, const int32_t* ids, int64_t n, const uint32_t* w, const void* s,
                            const void* b, q38_dtype sd, int64_t rows, int64_t K, int group, int bits, void* out,
                            q38_dtype od) {
    if (bits == 2 || bits == 4 || bits == 8) {
        const int64_t kw = K * bits / 32;
        const int osize = od == Q38_F32 ? 4 : 2;
        const bool vec = (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && (K * osize) % 16 == 0;
        const dim3 grid(static_cast<unsigned>((kw + 127) / 128), static_cast<unsigned>(n < 65535 ? n : 65535));
        auto go = [&](auto st, auto ot) {
            using ST = decltype(st);
            using OT = decltype(ot);
            const ST* sp = static_cast<const ST*>(s);
            const ST* bp = static_cast<const ST*>(b);
            OT* op = static_cast<OT*>(out);
            if (bits == 2)
                embed_word_kernel<ST, OT, 2><<<grid, 128, 0, ctx->stream>>>(ids, n, w, sp, bp, rows, K, group, vec, op, ctx->d_status);
            else if (bits == 4)
                embed_word_kernel<ST, OT, 4><<<grid, 128, 0, ctx->stream>>>(ids, n, w, sp, bp, rows, K, group, vec, op, ctx->d_status);
            else
                embed_word_kernel<ST, OT, 8><<<grid, 128, 0, ctx->stream>>>(ids, n, w, sp, bp, rows, K, group, vec, op, ctx->d_status);
        };
        auto pick_out = [&](auto st) {
            if (od == Q38_BF16) go(st, __nv_bfloat16());
            else if (od == Q38_F16) go(st, __half());
            else go(st, 0.0f);
        };
        if (sd == Q38_BF16) pick_out(__nv_bfloat16());
        else if (sd == Q38_F16) pick_out(__half());
        else pick_out(0.0f);
        return check_launch(ctx, "quantized_embedding");
    }
    const int grid = grid_for(n * K, 256);
#define Q38_EM(ST, OT)                                                                            \
    embed_kernel<ST, OT><<<grid, 256, 0, ctx->stream>>>(ids, n, w, static_cast<const ST*>(s),         \
                                                        static_cast<const ST*>(b), rows, K, group, bits, \
                                                        static_cast<OT*>(out), ctx->d_status)
    if (sd == Q38_BF16) {
        if (od == Q38_BF16) Q38_EM(__nv_bfloat16, __nv_bfloat16);
        else if (od == Q38_F16) Q38_EM(__nv_bfloat16, __half);
        else Q38_EM(__nv_bfloat16, float);
    } else if (sd == Q38_F16) {
        if (od == Q38_BF16) Q38_EM(__half, __nv_bfloat16);
        else if (od == Q38_F16) Q38_EM(__half, __half);
        else Q38_EM(__half, float);
    } else {
        if (od == Q38_BF16) Q38_EM(float, __nv_bfloat16);
        else if (od == Q38_F16) Q38_EM(float, __half);
        else Q38_EM(float, float);
    }
#undef Q38_EM
    return check_launch(ctx, "quantized_embedding");
}

q38_status quantize_launch(q38_ctx* ctx, const void* w, q38_dtype wd, int64_t rows, int64_t K,
                           int group, int bits, uint32_t* codes, void* s, void* b,
                           q38_dtype sd) {
    const int grid = grid_for(rows * (K / group), 128);
#define Q38_Q(WT, ST)                                                                         \
    quant_kernel<WT, ST><<<grid, 128, 0, ctx->stream>>>(static_cast<const WT*>(w), rows, K, \
                                                        group, bits, codes, static_cast<ST*>(s), \
                                                        static_cast<ST*>(b))
    if (wd == Q38_F32) {
        if (sd == Q38_BF16) Q38_Q(float, __nv_bfloat16);
        else if (sd == Q38_F16) Q38_Q(float, __half);
        else Q38_Q(float, float);
    } else if (wd == Q38_BF16) {
        if (sd == Q38_BF16) Q38_Q(__nv_bfloat16, __nv_bfloat16);
        else if (sd == Q38_F16) Q38_Q(__nv_bfloat16, __half);
        else Q38_Q(__nv_bfloat16, float);
    } else {
        if (sd == Q38_BF16) Q38_Q(__half, __nv_bfloat16);
        else if (sd == Q38_F16) Q38_Q(__half, __half);
        else Q38_Q(__half, float);
    }
#undef Q38_Q
    return check_launch(ctx, "quantize");
}

q38_status qmm_generic(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype xd,
                       const uint32_t* w, const void* s, const void* b, q38_dtype sd,
                       int64_t N, int group, int bits, void* y) {
    dim3 grid(static_cast<unsigned>((N + 7) / 8), static_cast<unsigned>((M + 7) / 8));
    if (grid.y > 65535) return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: M too large for the generic path");
#define Q38_G(XT, ST)                                                                       \
    qmm_generic_kernel<XT, ST><<<grid, 256, 0, ctx->stream>>>(                              \
        static_cast<const XT*>(x), M, K, w, static_cast<const ST*>(s), static_cast<const ST*>(b), \
        N, group, bits, static_cast<XT*>(y))
    if (xd == Q38_BF16) {
        if (sd == Q38_BF16) Q38_G(__nv_bfloat16, __nv_bfloat16);
        else if (sd == Q38_F16) Q38_G(__nv_bfloat16, __half);
        else Q38_G(__nv_bfloat16, float);
    } else {
        if (sd == Q38_BF16) Q38_G(__half, __nv_bfloat16);
        else if (sd == Q38_F16) Q38_G(__half, __half);
        else Q38_G(__half, float);
    }
#undef Q38_G
    return check_launch(ctx, "qmm_generic");
}

q38_status gather_generic(q38_ctx* ctx, const void* x, int64_t Bx, int64_t M, int64_t K, q38_dtype xd,
                          const uint32_t* w, const void* s, const void* b, q38_dtype sd, int64_t E,
                          int64_t N, const int32_t* lhs, const int32_t* rhs, int64_t P, int group,
                          int bits, void* out) {
    const int64_t gy = P * ((M + 7) / 8);
    if (gy > 65535) return fail(ctx, Q38_ERR_UNSUPPORTED, "gather_quantized_matmul: too many outputs for the generic path");
    dim3 grid(static_cast<unsigned>((N + 7) / 8), static_cast<unsigned>(gy));
#define Q38_GG(XT, ST)                                                                          \
    gather_generic_kernel<XT, ST><<<grid, 256, 0, ctx->stream>>>(                               \
        static_cast<const XT*>(x), Bx, M, K, w, static_cast<const ST*>(s), static_cast<const ST*>(b), \
        E, N, lhs, rhs, group, bits, static_cast<XT*>(out), ctx->d_status)
    if (xd == Q38_BF16) {
        if (sd == Q38_BF16) Q38_GG(__nv_bfloat16, __nv_bfloat16);
        else if (sd == Q38_F16) Q38_GG(__nv_bfloat16, __half);
        else Q38_GG(__nv_bfloat16, float);
    } else {
        if (sd == Q38_BF16) Q38_GG(__half, __nv_bfloat16);
        else if (sd == Q38_F16) Q38_GG(__half, __half);
        else Q38_GG(__half, float);
    }
#undef Q38_GG
    return check_launch(ctx, "gather_generic");
}

}  // namespace q38
