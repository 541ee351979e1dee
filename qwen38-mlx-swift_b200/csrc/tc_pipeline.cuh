// Building blocks shared by the tcgen05 quantized products (dense prefill and grouped
// expert kernels): bounded mbarrier waits with a cooperative abort, the packed-code stage
// layout, the exact bf16 dequantization of one 64-code group into TMEM operand order, and
// the matching activation permutation.
#pragma once

#include "affine_codes.cuh"

namespace q38 {
namespace {

// Codes of one 128-k stage for a block of weight rows, as a TMA box of CODE_W words per
// row: 2-bit rows (32 B) use the 32-byte swizzle, 4-bit rows (64 B) the 64-byte swizzle,
// 8-bit rows (128 B) the 128-byte swizzle, 3-bit rows (48 B) none.
template <int BITS>
struct CodeLayout {
    static constexpr int CODE_W = 4 * BITS;
    static constexpr int SW = BITS == 2 ? 32 : BITS == 4 ? 64 : BITS == 8 ? 128 : 0;
};

template <int BITS>
constexpr CUtensorMapSwizzle code_swizzle() {
    return CodeLayout<BITS>::SW == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
           : CodeLayout<BITS>::SW == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
           : CodeLayout<BITS>::SW == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                        : CU_TENSOR_MAP_SWIZZLE_NONE;
}

// Operand order of the tensor-core paths.  8-bit codes stay whole: operand q of a
// 16-code window pairs codes 2q and 2q + 1 with weight 1, so the activations keep their
// natural order.  The narrower widths use the magic-number pair tables.
template <int BITS>
__host__ __device__ constexpr int tc_pair_code(int q, int hi) {
    return BITS == 8 ? 2 * q + hi : pair_code<BITS>(q, hi);
}
template <int BITS>
__host__ __device__ constexpr float tc_pair_mult(int q, int hi) {
    return BITS == 8 ? 1.0f : pair_mult<BITS>(q, hi);
}

// Bounded mbarrier wait.  On expiry records the timeout and raises the abort flag of the
// CTA (and of the other CTA of a pair), so every role leaves its loop at its next wait.
struct Abort {
    volatile int* local;
    uint32_t peer;  // the other CTA's flag (cluster address); unused when !has_peer
    uint32_t* status;
    bool has_peer;
};

template <bool CLUSTER>
__device__ __forceinline__ bool p_wait(uint64_t* bar, uint32_t parity, const Abort& ab) {
    auto poll = [&]() { return CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity); };
    if (poll()) return true;
    const long long t0 = clock64();
    while (!poll()) {
        if (*ab.local) return false;
        if (clock64() - t0 > kWaitLimitCycles) {
            if (ab.status) atomicOr(ab.status, Q38_DEV_TIMEOUT);
            *ab.local = 1;
            if (ab.has_peer) st_shared_cluster_u32(ab.peer, 1u);
            return false;
        }
    }
    return true;
}

// Every lane waits (each observes the phase, so TMA-written data is visible to it); the
// warp then agrees on the outcome so that the .sync.aligned TMEM accesses stay convergent.
template <bool CLUSTER>
__device__ __forceinline__ bool p_wait_warp(uint64_t* bar, uint32_t parity, const Abort& ab) {
    const bool ok = p_wait<CLUSTER>(bar, parity, ab);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
    __nv_bfloat162 r = __hfma2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b),
                               *reinterpret_cast<__nv_bfloat162*>(&c));
    return *reinterpret_cast<uint32_t*>(&r);
}

// Words of group gg (0/1) of the stage for this row -> exact bf16 weights (x 2^p) in
// A-column order, 32 bf16x2 values.  sbits/bbits: the group's bf16 scale and bias; with G32
// (quantization groups of 32) the two groups' values, the first 32 codes' in the low half.
template <int BITS, bool G32 = false>
__device__ __forceinline__ void dequant_group(const uint8_t* codes, int row, int gg, uint32_t sbits, uint32_t bbits,
                                              uint32_t* a) {
    using F = CodeLayout<BITS>;
    // the scale and bias of the codes from 32 * half on
    auto half_bits = [&](uint32_t v, int half) { return G32 ? (half ? v >> 16 : v & 0xFFFFu) : v; };
    if constexpr (BITS == 8) {
        // A byte permute places code q in the low mantissa bits of fp32 2^23, so that
        // subtracting 2^23 leaves q exactly; q pairs convert exactly to bf16x2, and
        // a = s * q + b is rounded once, as for the narrower widths.
        const int swz = row & 7;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t s2 = half_bits(sbits, i >> 1) * 0x10001u, b2 = half_bits(bbits, i >> 1) * 0x10001u;
            const int c = gg * 4 + i;  // 16-byte chunk of the 128-byte row
            const uint4 v = *reinterpret_cast<const uint4*>(codes + row * 128 + ((c ^ swz) << 4));
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float q[4];
#pragma unroll
                for (int t = 0; t < 4; ++t)
                    q[t] = __uint_as_float(__byte_perm(wv[j], 0x4B000000u, 0x7440u + t)) - 8388608.0f;
                const __nv_bfloat162 p01 = __floats2bfloat162_rn(q[0], q[1]);
                const __nv_bfloat162 p23 = __floats2bfloat162_rn(q[2], q[3]);
                a[8 * i + 2 * j] = bf2_fma(*reinterpret_cast<const uint32_t*>(&p01), s2, b2);
                a[8 * i + 2 * j + 1] = bf2_fma(*reinterpret_cast<const uint32_t*>(&p23), s2, b2);
            }
        }
    } else {
    constexpr int GW = 2 * BITS;  // words per row per group
    uint32_t w[8];
    if constexpr (BITS == 3) {
        const uint2* p = reinterpret_cast<const uint2*>(codes + row * F::CODE_W * 4 + gg * GW * 4);
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            const uint2 v = p[i];
            w[2 * i] = v.x;
            w[2 * i + 1] = v.y;
        }
    } else {
        constexpr int CPR = F::SW / 16;         // 16-byte chunks per code row
        constexpr int GC = GW / 4;              // chunks per group: 1 (2-bit), 2 (4-bit)
        const int swz = F::SW == 64 ? ((row >> 1) & 3) : ((row >> 2) & 1);
#pragma unroll
        for (int i = 0; i < GC; ++i) {
            const int c = gg * GC + i;
            const uint4 v = *reinterpret_cast<const uint4*>(codes + row * F::SW + (((c ^ swz) & (CPR - 1)) << 4));
            w[4 * i] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
    }
    // s and 2^p b as bf16x2 with integer operations only: the scale broadcast, and the
    // bias times a power of two, exact in fp32 and so exactly the bf16 in its high half.
    uint32_t s2 = 0u, b2[8];
    auto set_group = [&](int half) {
        s2 = half_bits(sbits, half) * 0x10001u;
        const float bf = bf16_bits_to_f32(half_bits(bbits, half));
#pragma unroll
        for (int q = 0; q < 8; ++q)
            b2[q] = (__float_as_uint(bf * (1.0f / tc_pair_mult<BITS>(q, 0))) >> 16) |
                    (__float_as_uint(bf * (1.0f / tc_pair_mult<BITS>(q, 1))) & 0xFFFF0000u);
    };
    set_group(0);
#pragma unroll
    for (int tq = 0; tq < 4; ++tq) {
        if (G32 && tq == 2) set_group(1);  // windows 2 and 3 hold codes 32-63
        uint32_t win[2];
        if constexpr (BITS == 2) {
            win[0] = w[tq];
        } else if constexpr (BITS == 4) {
            win[0] = w[2 * tq];
            win[1] = w[2 * tq + 1];
        } else {
            const int k0 = (3 * tq) >> 1;
            if (tq & 1) {
                win[0] = __funnelshift_r(w[k0], w[k0 + 1], 16);
                win[1] = w[k0 + 1] >> 16;
            } else {
                win[0] = w[k0];
                win[1] = w[k0 + 1];
            }
        }
        uint32_t v[8];
        extract<BITS>(win, v);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            // v - 128 = 2^p q exactly; a = s * (2^p q) + 2^p b, rounded once
            a[tq * 8 + q] = bf2_fma(bf2_sub(v[q], MAGIC), s2, b2[q]);
        }
    }
    }
}

// Position and multiplier of code c (0..15 within a 16-code window) in the extraction
// order: the operand slot 2*q + hi whose pair_code is c.
template <int BITS>
__host__ __device__ constexpr int window_slot(int c) {
    for (int q = 0; q < 8; ++q)
        for (int hi = 0; hi < 2; ++hi)
            if (tc_pair_code<BITS>(q, hi) == c) return 2 * q + hi;
    return -1;
}
template <int BITS>
__host__ __device__ constexpr float window_mult(int c) {
    const int s = window_slot<BITS>(c);
    return tc_pair_mult<BITS>(s >> 1, s & 1);
}

// One 64-element group of bf16 activations -> extraction order, scaled by 2^-p.
template <int BITS>
__device__ __forceinline__ void permute_group(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    float xv[64];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 u = s4[i];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            xv[8 * i + 2 * j] = bf16_bits_to_f32(w[j] & 0xFFFFu);
            xv[8 * i + 2 * j + 1] = bf16_bits_to_f32(w[j] >> 16);
        }
    }
    uint32_t out[32];
#pragma unroll
    for (int col = 0; col < 32; ++col) {
        const int tq = col / 8, q = col % 8;
        out[col] = pack_bf16x2(xv[16 * tq + tc_pair_code<BITS>(q, 0)] * tc_pair_mult<BITS>(q, 0),
                               xv[16 * tq + tc_pair_code<BITS>(q, 1)] * tc_pair_mult<BITS>(q, 1));
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 8; ++i) d4[i] = make_uint4(out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
}

}  // namespace
}  // namespace q38
