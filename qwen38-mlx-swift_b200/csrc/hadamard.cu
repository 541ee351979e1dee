// Block-diagonal normalised Walsh-Hadamard rotation of activations (Bonsai 2 packs).
//
// Replaces hadamardRotate (Sources/Qwen38Core/Bonsai2/Qwen38HadamardModules.swift:10-19):
// fp32 copy of x, signs multiplied before the transform (forward) or after it (inverse),
// Sylvester-order transform over blocks of `block` along the last axis, scaled by
// 1/sqrt(block), cast back to the input dtype.  Butterfly stage h combines elements j and
// j+h as (a+b, a-b) for h = 1, 2, 4, ...; each butterfly is one IEEE add/subtract of the
// same two operands as the CPU restatement, so results agree bit for bit.
#include "affine_scalar.cuh"
#include "ptx.cuh"

namespace q38 {
namespace {

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p);
template <>
__device__ __forceinline__ float ld_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
}
template <>
__device__ __forceinline__ float ld_f32<__half>(const __half* p) {
    return __half2float(*p);
}
template <typename T>
__device__ __forceinline__ void st_f32(T* p, float v);
template <>
__device__ __forceinline__ void st_f32<__nv_bfloat16>(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void st_f32<__half>(__half* p, float v) {
    *p = __float2half_rn(v);
}

// One CTA per (row, block) through shared memory, any power-of-two block <= 8192.
template <typename T>
__global__ void __launch_bounds__(512) fwht_smem_kernel(const T* __restrict__ x, int64_t D,
                                                        int block, const float* __restrict__ signs,
                                                        int inverse, float scale,
                                                        T* __restrict__ y) {
    extern __shared__ float sv[];
    const int64_t per_row = D / block;
    const int64_t row = blockIdx.x / per_row, col0 = (blockIdx.x % per_row) * block;
    for (int i = threadIdx.x; i < block; i += blockDim.x) {
        float f = ld_f32(x + row * D + col0 + i);
        if (!inverse && signs) f = f * signs[col0 + i];
        sv[i] = f;
    }
    __syncthreads();
    for (int h = 1; h < block; h <<= 1) {
        for (int p = threadIdx.x; p < block / 2; p += blockDim.x) {
            const int j = (p / h) * 2 * h + (p % h);
            const float a = sv[j], b = sv[j + h];
            sv[j] = a + b;
            sv[j + h] = a - b;
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < block; i += blockDim.x) {
        float f = sv[i] * scale;
        if (inverse && signs) f = f * signs[col0 + i];
        st_f32(y + row * D + col0 + i, f);
    }
}

// The butterfly stages of one block of tpb * 4 elements, 4 consecutive elements per thread
// (`lt` = thread within the block, blocks aligned to tpb threads): h = 1, 2 in registers,
// h = 4 .. 64 by warp shuffles, larger h through the block's shared-memory area `mine`.
// Every thread of the CTA calls it (it synchronises the CTA when tpb > 32).
__device__ __forceinline__ void fwht4_stages(float (&v)[4], int lt, int tpb, float* mine) {
    constexpr int E = 4;
#pragma unroll
    for (int h = 1; h < E; h <<= 1)
#pragma unroll
        for (int i = 0; i < E; ++i)
            if ((i & h) == 0) {
                const float a = v[i], b = v[i + h];
                v[i] = a + b;
                v[i + h] = a - b;
            }
    const int lane = threadIdx.x & 31;
    for (int lh = 1; lh < 32 && lh < tpb; lh <<= 1) {
        const bool upper = (lane & lh) != 0;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            const float p = __shfl_xor_sync(0xffffffffu, v[i], lh);
            v[i] = upper ? (p - v[i]) : (v[i] + p);
        }
    }
    for (int th = 32; th < tpb; th <<= 1) {  // partner thread lt ^ th, element distance th * E
#pragma unroll
        for (int i = 0; i < E; ++i) mine[lt * E + i] = v[i];
        __syncthreads();
        const bool upper = (lt & th) != 0;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            const float p = mine[(lt ^ th) * E + i];
            v[i] = upper ? (p - v[i]) : (v[i] + p);
        }
        __syncthreads();
    }
}

// Blocks of up to 4096: each thread holds 4 consecutive elements of one block (B / 4
// threads per block, 256 / (B / 4) blocks per CTA of at least 256 threads).  Butterfly
// stages h = 1, 2 run in registers, h = 4 .. 64 by warp shuffles, larger h through shared
// memory, all in increasing h with the operands of the other kernels (lower element a + b,
// upper a - b), so the results are the same bit for bit.
template <typename T, bool VEC>
__global__ void __launch_bounds__(1024) fwht_block_kernel(const T* __restrict__ x, int64_t nblocks, int64_t D,
                                                          int block, const float* __restrict__ signs,
                                                          int inverse, float scale, T* __restrict__ y) {
    constexpr int E = 4;
    extern __shared__ float sv[];
    const int tpb = block / E;                            // threads per block
    const int local = threadIdx.x / tpb;                  // block within the CTA
    const int lt = threadIdx.x % tpb;                     // thread within the block
    const int64_t bid = static_cast<int64_t>(blockIdx.x) * (blockDim.x / tpb) + local;
    const bool live = bid < nblocks;
    const int64_t per_row = D / block;
    const int64_t row = live ? bid / per_row : 0, col0 = live ? (bid % per_row) * block + lt * E : 0;
    float v[E];
    if (VEC && live) {  // the 4 elements in one 8-byte load
        const uint2 u = *reinterpret_cast<const uint2*>(x + row * D + col0);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int i = 0; i < E; ++i) v[i] = ld_f32(e + i);
    } else {
#pragma unroll
        for (int i = 0; i < E; ++i) v[i] = live ? ld_f32(x + row * D + col0 + i) : 0.0f;
    }
    if (!inverse && signs && live)
#pragma unroll
        for (int i = 0; i < E; ++i) v[i] = v[i] * signs[col0 + i];
    fwht4_stages(v, lt, tpb, sv + local * block);
    if (!live) return;
    T* dst = y + row * D + col0;
    __align__(8) T o[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
        float f = v[i] * scale;
        if (inverse && signs) f = f * signs[col0 + i];
        st_f32(o + i, f);
    }
    if (VEC) {
        *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o);
    } else {
#pragma unroll
        for (int i = 0; i < E; ++i) dst[i] = o[i];
    }
}

template <typename T>
q38_status launch(q38_ctx* ctx, const void* x, int64_t rows, int64_t D, const float* signs,
                  int block, int inverse, void* y) {
    const float scale = 1.0f / sqrtf(static_cast<float>(block));
    const int64_t nblocks = rows * (D / block);
    const T* xs = static_cast<const T*>(x);
    T* ys = static_cast<T*>(y);
    if (block >= 4 && block <= 4096) {
        // 4 elements per thread, at least 256 threads per CTA
        const int tpb = block / 4;
        const int per_cta = tpb >= 256 ? 1 : 256 / tpb;
        const int64_t ctas = (nblocks + per_cta - 1) / per_cta;
        if (ctas > 0x7fffffffLL) return fail(ctx, Q38_ERR_UNSUPPORTED, "hadamard_rotate: too many blocks");
        const unsigned threads = static_cast<unsigned>(tpb * per_cta);
        const size_t smem = static_cast<size_t>(per_cta) * block * sizeof(float);
        // 8-byte accesses when both buffers allow them (rows of D elements keep the alignment)
        const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 7u) == 0;
        if (vec)
            fwht_block_kernel<T, true><<<static_cast<unsigned>(ctas), threads, smem, ctx->stream>>>(
                xs, nblocks, D, block, signs, inverse, scale, ys);
        else
            fwht_block_kernel<T, false><<<static_cast<unsigned>(ctas), threads, smem, ctx->stream>>>(
                xs, nblocks, D, block, signs, inverse, scale, ys);
        return check_launch(ctx, "hadamard_rotate");
    }
    // larger blocks: one CTA per block through shared memory
    if (nblocks > 0x7fffffffLL) return fail(ctx, Q38_ERR_UNSUPPORTED, "hadamard_rotate: too many blocks");
    const int threads = block / 2 < 512 ? (block / 2 < 32 ? 32 : block / 2) : 512;
    fwht_smem_kernel<T><<<static_cast<unsigned>(nblocks), threads, block * sizeof(float), ctx->stream>>>(
        xs, D, block, signs, inverse, scale, ys);
    return check_launch(ctx, "hadamard_rotate");
}

// Rotated embedding rows, blocks of up to 4096: 4 consecutive codes per thread (one code word
// for 2-, 4- and 8-bit codes), dequantized into T with the lookup kernel's arithmetic, then
// fwht4_stages, scale, signs and one rounding to T: the same values as the kernel below and
// as the lookup followed by the inverse rotation.
template <typename T>
__global__ void __launch_bounds__(1024) embed_rotate_block_kernel(
    const int32_t* __restrict__ ids, int64_t nblocks, const uint32_t* __restrict__ w, const T* __restrict__ s,
    const T* __restrict__ b, int64_t rows, int64_t K, int group, int bits, const float* __restrict__ signs, int block,
    float scale, T* __restrict__ out, uint32_t* status) {
    using namespace dev;
    constexpr int E = 4;
    extern __shared__ float sv[];
    const int tpb = block / E;
    const int local = threadIdx.x / tpb, lt = threadIdx.x % tpb;
    const int64_t bid = static_cast<int64_t>(blockIdx.x) * (blockDim.x / tpb) + local;
    const bool live = bid < nblocks;
    const int64_t per_row = K / block;
    const int64_t t = live ? bid / per_row : 0, k0 = live ? (bid % per_row) * block + lt * E : 0;
    const int64_t r = live ? ids[t] : 0;
    const bool valid = live && r >= 0 && r < rows;
    if (live && !valid && lt == 0 && k0 == 0) atomicOr(status, Q38_DEV_BAD_INDEX);
    float v[E] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
        const int64_t G = K / group;
        const uint32_t* wr = w + r * (K * bits / 32);
        const float sc = to_f32(s[r * G + k0 / group]);  // the 4 codes share a group
        const float bi = b ? to_f32(b[r * G + k0 / group]) : 0.0f;
        uint32_t q[E];
        if (bits == 2 || bits == 4 || bits == 8) {
            const int64_t bit = k0 * bits;
            const uint32_t word = wr[bit >> 5] >> (bit & 31);
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = (word >> (i * bits)) & ((1u << bits) - 1u);
        } else {
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = get_code(wr, k0 + i, bits);
        }
#pragma unroll
        for (int i = 0; i < E; ++i)
            v[i] = to_f32(from_f32<T>(__fadd_rn(__fmul_rn(sc, static_cast<float>(q[i])), bi)));
    }
    fwht4_stages(v, lt, tpb, sv + local * block);
    if (!live) return;
    T* dst = out + t * K + k0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
        float f = v[i] * scale;
        if (signs) f = f * signs[k0 + i];
        dst[i] = from_f32<T>(f);
    }
}

// Rotated embedding rows (Qwen38HadamardQuantizedEmbedding.callAsFunction,
// Sources/Qwen38Core/Bonsai2/Qwen38HadamardModules.swift:71-79): the row of ids[t] is
// dequantized into the scales' dtype T (scale*q + bias in fp32, one rounding, as the
// lookup kernel does), then inverse-rotated: fp32 transform, 1/sqrt(block), signs after,
// one rounding to T.  One CTA per (id, block) in shared memory, with the butterfly order
// of the rotation kernels, so the result equals the lookup followed by the inverse
// rotation bit for bit.  An id outside [0, rows) transforms a zero row and sets the
// out-of-range status bit.
template <typename T>
__global__ void __launch_bounds__(512) embed_rotate_kernel(const int32_t* __restrict__ ids,
                                                           const uint32_t* __restrict__ w,
                                                           const T* __restrict__ s, const T* __restrict__ b,
                                                           int64_t rows, int64_t K, int group, int bits,
                                                           const float* __restrict__ signs, int block,
                                                           float scale, T* __restrict__ out, uint32_t* status) {
    using namespace dev;
    extern __shared__ float sv[];
    const int64_t per_row = K / block;
    const int64_t t = blockIdx.x / per_row, col0 = (blockIdx.x % per_row) * block;
    const int64_t r = ids[t];
    const bool valid = r >= 0 && r < rows;
    if (!valid && threadIdx.x == 0 && col0 == 0) atomicOr(status, Q38_DEV_BAD_INDEX);
    const int64_t G = K / group;
    const uint32_t* wr = w + (valid ? r : 0) * (K * bits / 32);
    for (int i = threadIdx.x; i < block; i += blockDim.x) {
        float f = 0.0f;
        if (valid) {
            const int64_t k = col0 + i;
            const float sc = to_f32(s[r * G + k / group]);
            const float bi = b ? to_f32(b[r * G + k / group]) : 0.0f;
            f = to_f32(from_f32<T>(__fadd_rn(__fmul_rn(sc, static_cast<float>(get_code(wr, k, bits))), bi)));
        }
        sv[i] = f;
    }
    __syncthreads();
    for (int h = 1; h < block; h <<= 1) {
        for (int p = threadIdx.x; p < block / 2; p += blockDim.x) {
            const int j = (p / h) * 2 * h + (p % h);
            const float a = sv[j], c = sv[j + h];
            sv[j] = a + c;
            sv[j + h] = a - c;
        }
        __syncthreads();
    }
    T* dst = out + t * K + col0;
    for (int i = threadIdx.x; i < block; i += blockDim.x) {
        float f = sv[i] * scale;
        if (signs) f = f * signs[col0 + i];
        dst[i] = from_f32<T>(f);
    }
}

}  // namespace

q38_status hadamard_embedding_launch(q38_ctx* ctx, const int32_t* ids, int64_t n, const uint32_t* w,
                                     const void* s, const void* b, q38_dtype sd, int64_t rows, int64_t K,
                                     int group, int bits, const float* signs, int block, void* out) {
    const int64_t nblocks = n * (K / block);
    if (nblocks > 0x7fffffffLL) return fail(ctx, Q38_ERR_UNSUPPORTED, "hadamard_quantized_embedding: too many blocks");
    const float scale = 1.0f / sqrtf(static_cast<float>(block));
    if (block >= 4 && block <= 4096) {
        const int tpb = block / 4;
        const int per_cta = tpb >= 256 ? 1 : 256 / tpb;
        const unsigned ctas = static_cast<unsigned>((nblocks + per_cta - 1) / per_cta);
        const unsigned threads = static_cast<unsigned>(tpb * per_cta);
        const size_t smem = static_cast<size_t>(per_cta) * block * sizeof(float);
        if (sd == Q38_BF16)
            embed_rotate_block_kernel<__nv_bfloat16><<<ctas, threads, smem, ctx->stream>>>(
                ids, nblocks, w, static_cast<const __nv_bfloat16*>(s), static_cast<const __nv_bfloat16*>(b), rows, K,
                group, bits, signs, block, scale, static_cast<__nv_bfloat16*>(out), ctx->d_status);
        else
            embed_rotate_block_kernel<__half><<<ctas, threads, smem, ctx->stream>>>(
                ids, nblocks, w, static_cast<const __half*>(s), static_cast<const __half*>(b), rows, K, group, bits,
                signs, block, scale, static_cast<__half*>(out), ctx->d_status);
        return check_launch(ctx, "hadamard_quantized_embedding");
    }
    const int threads = block / 2 < 512 ? (block / 2 < 32 ? 32 : block / 2) : 512;
    const size_t smem = static_cast<size_t>(block) * sizeof(float);
    const unsigned grid = static_cast<unsigned>(nblocks);
    if (sd == Q38_BF16)
        embed_rotate_kernel<__nv_bfloat16><<<grid, threads, smem, ctx->stream>>>(
            ids, w, static_cast<const __nv_bfloat16*>(s), static_cast<const __nv_bfloat16*>(b), rows, K, group, bits,
            signs, block, scale, static_cast<__nv_bfloat16*>(out), ctx->d_status);
    else
        embed_rotate_kernel<__half><<<grid, threads, smem, ctx->stream>>>(
            ids, w, static_cast<const __half*>(s), static_cast<const __half*>(b), rows, K, group, bits, signs, block,
            scale, static_cast<__half*>(out), ctx->d_status);
    return check_launch(ctx, "hadamard_quantized_embedding");
}

q38_status hadamard_launch(q38_ctx* ctx, const void* x, int64_t rows, int64_t D, q38_dtype xd,
                           const float* signs, int block, int inverse, void* y) {
    if (xd == Q38_BF16) return launch<__nv_bfloat16>(ctx, x, rows, D, signs, block, inverse, y);
    return launch<__half>(ctx, x, rows, D, signs, block, inverse, y);
}

}  // namespace q38
