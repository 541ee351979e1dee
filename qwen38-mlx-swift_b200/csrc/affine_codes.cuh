// MLX packed codes -> bf16 operands without integer-to-float conversion.
//
// A code masked into the mantissa of bf16 128.0 (0x4300) reads as 128 + 2^p * q, where p is
// the bit position of the code inside the 16-bit half.  Extraction produces bf16x2 pairs
// (two codes per 32-bit register); which codes land in which pair, and the weight 2^p each
// code carries, are fixed per bit width by the tables below.  Kernels pair the extracted
// operands with activations permuted and scaled (x * 2^-p) by the same tables.
#pragma once

#include "ptx.cuh"

namespace q38 {
namespace {

using namespace dev;

constexpr uint32_t MAGIC = 0x43004300u;  // bf16 128.0 in both halves

// The same constant read from constant memory.  The compiler cannot turn it into an
// immediate, so it stays in a register and `(code & mask) | magic` compiles to one
// three-input logic instruction; with two immediates it compiles to two.
__constant__ uint32_t c_magic = MAGIC;

// ---------------------------------------------------------------------------------
// Pair tables: for bf16x2 operand q of a thread's 16 codes (per row and group), the
// code index feeding its low and high half and the power-of-two weight the code has
// inside that half (the activation is pre-multiplied by the inverse).
// ---------------------------------------------------------------------------------
template <int BITS>
__host__ __device__ constexpr int pair_code(int q, int hi) {
    if (BITS == 2) return q + (hi ? 8 : 0);
    if (BITS == 3) return q < 4 ? q + (hi ? 4 : 0) : q + 4 + (hi ? 4 : 0);
    if (BITS == 4) return (q / 4) * 8 + (q % 4) + (hi ? 4 : 0);
    /* 8 */ return (q / 4) * 4 + ((q % 4) >> 1) + (hi ? 2 : 0);
}

// Multiplier applied to the activation for the slot (1 / weight of the code's bits).
template <int BITS>
__host__ __device__ constexpr float pair_mult(int q, int hi) {
    if (BITS == 2) {
        const int pos = (q % 3 == 0) ? 0 : (q % 3 == 1) ? 2 : 4;  // q: 0,1,2,3,4,5,6,7
        return pos == 0 ? 1.0f : pos == 2 ? 0.25f : 0.0625f;
    }
    if (BITS == 3) return hi ? 1.0f : 0.0625f;
    if (BITS == 4) return 1.0f;
    /* 8: odd q = high nibble, weight 16 */ return (q & 1) ? 16.0f : 1.0f;
}

// Extract the NP bf16x2 operands of one thread-row-group from its code window.
// w[] holds the window: bits 2 -> 1 word, 3 -> 2 words (48 valid bits), 4 -> 2, 8 -> 4.
template <int BITS>
__device__ __forceinline__ void extract(const uint32_t* w, uint32_t* a) {
    const uint32_t MAGIC = c_magic;
    if constexpr (BITS == 2) {
        const uint32_t v = w[0], v6 = v >> 6, v12 = v >> 12;
        a[0] = (v & 0x00030003u) | MAGIC;
        a[1] = (v & 0x000C000Cu) | MAGIC;
        a[2] = (v & 0x00300030u) | MAGIC;
        a[3] = (v6 & 0x00030003u) | MAGIC;
        a[4] = (v6 & 0x000C000Cu) | MAGIC;
        a[5] = (v6 & 0x00300030u) | MAGIC;
        a[6] = (v12 & 0x00030003u) | MAGIC;
        a[7] = (v12 & 0x000C000Cu) | MAGIC;
    } else if constexpr (BITS == 3) {
        const uint32_t A = w[0], B = w[1];
        constexpr uint32_t m = 0x00070070u;
        a[0] = ((A << 4) & m) | MAGIC;
        a[1] = ((A << 1) & m) | MAGIC;
        a[2] = ((A >> 2) & m) | MAGIC;
        a[3] = ((A >> 5) & m) | MAGIC;
        a[4] = (__funnelshift_r(A, B, 20) & m) | MAGIC;
        a[5] = (__funnelshift_r(A, B, 23) & m) | MAGIC;
        a[6] = (__funnelshift_r(A, B, 26) & m) | MAGIC;
        a[7] = (__funnelshift_r(A, B, 29) & m) | MAGIC;
    } else {
        constexpr int NW = BITS == 4 ? 2 : 4;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            const uint32_t v = w[i];
            a[4 * i + 0] = (v & 0x000F000Fu) | MAGIC;
            a[4 * i + 1] = ((v >> 4) & 0x000F000Fu) | MAGIC;
            a[4 * i + 2] = ((v >> 8) & 0x000F000Fu) | MAGIC;
            a[4 * i + 3] = ((v >> 12) & 0x000F000Fu) | MAGIC;
        }
    }
}

// ---------------------------------------------------------------------------------
// f16 variant for 4- and 8-bit codes.  f16 1024.0 (0x6400) has a 10-bit mantissa, so a
// code masked into it at bit p < 10 - bits reads as 1024 + 2^p * q: nibbles at bit 0 and
// bit 4 of a half, and whole bytes at bit 0, need no shift.
//   4 bits: word v -> (n0,n4), 16*(n1,n5), (n2,n6), 16*(n3,n7)   [v, v >> 8]
//   8 bits: word v -> (b0,b2), (b1,b3)                           [v, v >> 8]
// ---------------------------------------------------------------------------------
constexpr uint32_t MAGIC16 = 0x64006400u;  // f16 1024.0 in both halves
__constant__ uint32_t c_magic16 = MAGIC16;

template <int BITS>
__host__ __device__ constexpr int pair_code16(int q, int hi) {
    if (BITS == 4) return (q / 4) * 8 + (q % 4) + (hi ? 4 : 0);
    /* 8 */ return (q / 2) * 4 + (q % 2) + (hi ? 2 : 0);
}

template <int BITS>
__host__ __device__ constexpr float pair_mult16(int q, int) {
    return (BITS == 4 && (q & 1)) ? 0.0625f : 1.0f;
}

// The 8 f16x2 operands of one thread-row-group (16 codes: 2 words of 4-bit, 4 of 8-bit).
template <int BITS>
__device__ __forceinline__ void extract16(const uint32_t* w, uint32_t* a) {
    const uint32_t M16 = c_magic16;
    if constexpr (BITS == 4) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t v = w[i], v8 = v >> 8;
            a[4 * i + 0] = (v & 0x000F000Fu) | M16;
            a[4 * i + 1] = (v & 0x00F000F0u) | M16;
            a[4 * i + 2] = (v8 & 0x000F000Fu) | M16;
            a[4 * i + 3] = (v8 & 0x00F000F0u) | M16;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t v = w[i];
            a[2 * i + 0] = (v & 0x00FF00FFu) | M16;
            a[2 * i + 1] = ((v >> 8) & 0x00FF00FFu) | M16;
        }
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return static_cast<uint32_t>(f32_to_bf16_bits(lo)) |
           (static_cast<uint32_t>(f32_to_bf16_bits(hi)) << 16);
}

}  // namespace
}  // namespace q38
