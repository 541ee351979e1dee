// Decode-shaped MLX-affine quantized product: y[M,N] = x[M,K] . dequant(W)[N,K]^T for
// M <= 16, group 64, K % 512 == 0, bits 2/3/4/8, bf16 activations and scales.
//
// Replaces the Metal `qmv` kernel behind MLX.quantizedMM (QuantizedLinear.callAsFunction,
// Sources/Qwen38Core/FlashNext/Qwen4ExpPrequantized.swift:156-159).
//
// Design (HBM-bound: the packed codes are the stream):
//  * Work unit = 16 weight rows x 512 k ("subunit").  A CTA owns a contiguous range of
//    subunits in (64-row tile, k-chunk, 16-row subtile) order, so every CTA streams the
//    same number of bytes (+-1 subunit) whatever N and K are.
//  * One producer warp streams each (tile, chunk) stage with TMA: the codes of the
//    active 16-row subtiles (swizzled boxes) and the 64x8 bf16 scales and biases.  One
//    activation warp writes the chunk's activation fragments into the same stage, built
//    from x in global memory.  Four consumer warps each own one 16-row subtile.  Stages
//    cycle through an mbarrier ring.
//  * Codes are turned into bf16 operands without integer->float conversion: a code
//    masked into the mantissa of 0x4300 (bf16 128.0) reads as 128 + 2^p*q.  The
//    activation fragments hold x permuted and scaled (x * 2^-p) into the order that
//    matches the extraction, plus per-group sums.  One m16n8k16 bf16 MMA dots 16 codes
//    of 16 rows with 8 columns; per group D = sum(q*x) + 128*sum(x'), and y += scale*D.
//  * The 8 columns are (group slot, token) pairs, so a product serves 8/MP groups of
//    MP tokens at once and each accumulator set spans several groups: the scales are
//    applied once per chunk, not after every group's MMA chain.  The -128*scale*sum(x')
//    and bias*sum(x) terms of all 8 groups of a chunk are folded into two extra MMA
//    steps whose operands are the scales/biases and hi/lo bf16 splits of the sums.
//  * Consumers do no address arithmetic in the inner loop: swizzled code offsets are
//    precomputed per thread and the fragment offsets are constants.
//  * Every warp adds its subtile partial sums into an fp32 zero-at-rest region with
//    fire-and-forget reductions (no fences or counters in the main kernel); a small
//    epilogue kernel converts the sums to y and zeroes them again, so no per-call clearing
//    is needed.  The fp32 additions land in arrival order, so repeats may differ in the
//    last bit; a context set to deterministic mode instead stores each k-chunk's sums in a
//    slot of its own and the epilogue adds the slots in a fixed order (bitwise
//    reproducible, about 1 us more per product).
//  * The main kernel is launched with programmatic dependent launch: its producer
//    streams the first stages of weights while the previous kernel is still running.
#include <algorithm>
#include <mutex>
#include <numeric>
#include <type_traits>

#include "affine_codes.cuh"

namespace q38 {
namespace {

using namespace dev;

constexpr int KC = 512;        // k per chunk
constexpr int GROUPS = 8;      // groups of 64 per chunk
constexpr int NCW = 4;         // 16-row subtiles per stage (one consumer warp each)
constexpr int WG = 2;          // consumer warp groups; group j takes the stages i with i % WG == j
constexpr int THREADS = (NCW * WG + 2) * 32;  // + weight producer + activation warp
static_assert(8 * WG + 8 + 4 <= 1024 / 8, "landing, empty and x barriers fit the first 1 KiB");

template <int BITS>
struct Fmt {
    static constexpr bool F16 = BITS == 4 || BITS == 8;  // f16 operands (else bf16)
    static constexpr int SPG = 4;                      // k16 MMA steps per group
    static constexpr int NP = 2 * SPG;                 // operand pairs per thread-row-group
    static constexpr float OFFSET = F16 ? 1024.0f : 128.0f;  // value of the magic number
    static constexpr int SW = BITS == 3 ? 64 : 128;    // swizzle span of a code box (bytes)
    static constexpr int ROW_BYTES = KC * BITS / 8;    // code bytes per row per chunk
    static constexpr int ROW_WORDS = ROW_BYTES / 4;
    static constexpr int BOXES = ROW_BYTES / SW;       // code boxes per subtile
    static constexpr int SUB_BYTES = 16 * ROW_BYTES;   // code bytes per subtile
    static constexpr int XF_FRAG = 256 * SPG;          // fragment bytes per token per chunk
    static constexpr int XF_PER_M = XF_FRAG + 64;      // + bias-step fragments
};

// Byte offset of word `wi` of row `r` (of the subtile's 16) inside a subtile's codes.  A
// stage holds BOXES column boxes of 64 rows x SW bytes (TMA swizzle of 16-byte chunks
// within SW-byte rows); a subtile's rows start 16*SW bytes into each box.  Rows r and r+8
// share the swizzle, so row r+8 sits exactly 8*SW bytes after row r.
template <int SW>
__device__ __forceinline__ uint32_t code_off(int r, int wi) {
    constexpr int WPB = SW / 4;  // words per box row
    const int box = wi / WPB, iw = wi % WPB;
    const int swz = SW == 128 ? (r & 7) : ((r >> 1) & 3);
    return box * (64 * SW) + r * SW + ((((iw >> 2) ^ swz)) << 4) + (iw & 3) * 4;
}

// First (and for 3 bits, second) word of the window of (row r, group gi, quarter t).
template <int BITS>
__device__ __forceinline__ void window_words(int gi, int t, int& w0, int& w1) {
    if constexpr (BITS == 3) {
        w0 = 6 * gi + ((t * 3) >> 1);  // t: 0,1,2,3 -> word 0,1,3,4 (bit 48t of the group)
        w1 = w0 + 1;
    } else {
        w0 = gi * 2 * BITS + t * (BITS / 2);
        w1 = w0;
    }
}

// Load the code window at precomputed offsets (3 bits: two words, realigned for odd t).
template <int BITS>
__device__ __forceinline__ void load_window(const uint8_t* p, uint32_t offA, uint32_t offB, bool odd,
                                            uint32_t* w) {
    if constexpr (BITS == 2) {
        w[0] = *reinterpret_cast<const uint32_t*>(p + offA);
    } else if constexpr (BITS == 4) {
        const uint2 v = *reinterpret_cast<const uint2*>(p + offA);
        w[0] = v.x;
        w[1] = v.y;
    } else if constexpr (BITS == 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(p + offA);
        w[0] = v.x;
        w[1] = v.y;
        w[2] = v.z;
        w[3] = v.w;
    } else {
        const uint32_t a = *reinterpret_cast<const uint32_t*>(p + offA);
        const uint32_t b = *reinterpret_cast<const uint32_t*>(p + offB);
        w[0] = odd ? __funnelshift_r(a, b, 16) : a;
        w[1] = odd ? (b >> 16) : b;
    }
}


// ---------------------------------------------------------------------------------
// Activation fragments of one 512-k chunk, written by one warp.
// Layout per token m (stride XF_PER_M bytes):
//   [group 8][k-step pair SPG/2][t 4][16 B]  then  [t 4][16 B]
// The first part holds x' (x permuted into extraction order and scaled by 2^-p) as
// MMA B operands: f16x2 for 4- and 8-bit codes (after a power-of-two range factor of
// the chunk, kept after the token blocks), bf16x2 otherwise.  The second holds, for lane quarter t, the B operands of the
// offset-and-bias steps: groups 2t and 2t+1 of -128 * sum(x') and of sum(x), each split
// into a bf16 high part (words 0, 1) and the bf16 of the remainder (words 2, 3).
// ---------------------------------------------------------------------------------
template <int BITS>
__device__ __forceinline__ void build_fragments(const uint8_t* xc, int M, uint8_t* base, uint8_t* hdr,
                                                float (*s_xs)[16], float (*s_xp)[16], int lane) {
    using F = Fmt<BITS>;
    constexpr uint32_t ONE2 = 0x3F803F80u;  // bf16x2 (1, 1)
    // f16 operands: scale the chunk by 2^-e so that its largest |x| stays below 2^15; the
    // consumers multiply the group scales by 2^e (stored after the token blocks).
    float down = 1.0f;
    if constexpr (F::F16) {
        uint32_t mx = 0;
        const uint32_t* xw = reinterpret_cast<const uint32_t*>(xc);
        for (int p = lane; p < M * (KC / 2); p += 32) {
            const uint32_t wv = xw[p];
            mx = max(mx, max(wv & 0x7FFFu, (wv >> 16) & 0x7FFFu));
        }
        mx = __reduce_max_sync(0xffffffffu, mx);
        const int E = static_cast<int>(mx >> 7);  // bf16 exponent field of the largest |x|
        const int esh = E > 141 ? E - 141 : 0;
        down = __uint_as_float(static_cast<uint32_t>(127 - esh) << 23);
        if (lane == 0) *reinterpret_cast<float*>(hdr) = __uint_as_float(static_cast<uint32_t>(127 + esh) << 23);
    }
    // 32 * M items: every iteration has all 32 lanes, and lanes 4i..4i+3 share (group, token)
    const int items = GROUPS * M * 4;
    for (int i = lane; i < items; i += 32) {
        const int t = i & 3, gm = i >> 2, m = gm % M, gi = gm / M;
        const uint4* src = reinterpret_cast<const uint4*>(xc + m * (KC * 2) + (gi * 64 + t * 16) * 2);
        const uint4 u0 = src[0], u1 = src[1];
        const uint32_t raw[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        float xs = 0.f, xp = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) xs = fma2_bf16_f32(raw[j], ONE2, xs);
        uint32_t* dst = reinterpret_cast<uint32_t*>(base + m * F::XF_PER_M + gi * (F::SPG / 2) * 64 + t * 16);
#pragma unroll
        for (int q = 0; q < F::NP; ++q) {
            // pair (code a, code b) = (element a, element b) of the 16
            const int ea = F::F16 ? pair_code16<BITS>(q, 0) : pair_code<BITS>(q, 0);
            const int eb = F::F16 ? pair_code16<BITS>(q, 1) : pair_code<BITS>(q, 1);
            const uint32_t lo = (ea & 1) ? (raw[ea >> 1] >> 16) : (raw[ea >> 1] & 0xFFFFu);
            const uint32_t hi = (eb & 1) ? (raw[eb >> 1] & 0xFFFF0000u) : (raw[eb >> 1] << 16);
            const uint32_t pr = lo | hi;  // bf16x2 (x_a, x_b)
            const float ma = F::F16 ? pair_mult16<BITS>(q, 0) : pair_mult<BITS>(q, 0);
            const float mb = F::F16 ? pair_mult16<BITS>(q, 1) : pair_mult<BITS>(q, 1);
            const uint32_t mult2 = static_cast<uint32_t>(f32_to_bf16_bits(ma)) |
                                   (static_cast<uint32_t>(f32_to_bf16_bits(mb)) << 16);
            if constexpr (F::F16) {
                // f16x2 of (x_a * ma, x_b * mb) * 2^-e, rounded once (exact unless tiny)
                const float fa = __uint_as_float(lo << 16) * (ma * down);
                const float fb = __uint_as_float(hi & 0xFFFF0000u) * (mb * down);
                uint32_t h2;
                asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h2) : "f"(fb), "f"(fa));
                dst[(q / 4) * 16 + (q % 4)] = h2;
                if (BITS != 8) xp = fma2_bf16_f32(pr, mult2, xp);
            } else {
                const uint32_t scaled = (ma != 1.0f || mb != 1.0f) ? mul_bf16x2(pr, mult2) : pr;
                if (BITS != 4) xp = fma2_bf16_f32(scaled, ONE2, xp);
                dst[(q / 4) * 16 + (q % 4)] = scaled;
            }
        }
        if (BITS == 8) xp = xs;  // every factor is 1
        xs += __shfl_xor_sync(0xffffffffu, xs, 1);
        xs += __shfl_xor_sync(0xffffffffu, xs, 2);
        xp += __shfl_xor_sync(0xffffffffu, xp, 1);
        xp += __shfl_xor_sync(0xffffffffu, xp, 2);
        if (t == 0) {
            s_xs[gi][m] = xs;
            s_xp[gi][m] = xp;
        }
    }
    __syncwarp();
    // offset-and-bias operands of quarter t: groups 2t, 2t+1
    for (int i = lane; i < 4 * M; i += 32) {
        const int t = i & 3, m = i >> 2;
        float v[4] = {-F::OFFSET * s_xp[2 * t][m], -F::OFFSET * s_xp[2 * t + 1][m], s_xs[2 * t][m],
                      s_xs[2 * t + 1][m]};
        uint32_t hb[4], lb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            hb[j] = f32_to_bf16_bits(v[j]);
            lb[j] = f32_to_bf16_bits(v[j] - bf16_bits_to_f32(hb[j]));
        }
        *reinterpret_cast<uint4*>(base + m * F::XF_PER_M + F::XF_FRAG + t * 16) =
            make_uint4(hb[0] | (hb[1] << 16), hb[2] | (hb[3] << 16), lb[0] | (lb[1] << 16), lb[2] | (lb[3] << 16));
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------------
// Main kernel.
// ---------------------------------------------------------------------------------
// Tensor maps of one weight: codes in 16-row and 64-row boxes, scales, biases.
struct WeightMaps {
    CUtensorMap codes16, codes64, scales, biases;
};

// How the partial sums of a subunit leave the kernel, and which rows and activations a
// tile has.
enum : int {
    // Plain product.  Partial sums are added into a zero-at-rest fp32 region with
    // fire-and-forget reductions; the epilogue converts and re-zeroes (arrival order
    // decides the fp32 rounding, so repeats may differ in the last bit).
    MODE_ATOMIC = 0,
    // Plain product.  Each subunit stores its partial sums into the slot of its k-chunk
    // (every (chunk, token, row) is written by exactly one warp); the epilogue adds the
    // chunks in order, so results are bitwise reproducible.
    MODE_SLOTS = 1,
    // MoE gate and up projections of a few tokens: the tiles are the gate rows, then the
    // up rows, of the experts the tokens selected (expert-stacked weights, distinct experts
    // in ascending order); every token's activations are used for every expert, and only
    // the (token, slot) pairs that selected the expert are stored, per k-chunk, at
    // [chunk][pair][2 * rows_per_expert] (gate columns, then up columns).
    MODE_MOE_GU = 2,
    // MoE down projection: the tiles are the output rows of the selected experts; the
    // activations of an expert are the rows of h (x = h [pairs, K]) of the pairs that selected
    // it; sums are stored at [chunk][pair][rows_per_expert].
    MODE_MOE_DOWN = 3
};

constexpr int MOE_MAX_T = 16;      // tokens of a decode-shaped MoE call
constexpr int MOE_MAX_PAIRS = 256; // (token, slot) pairs, hence distinct experts
constexpr int MOE_MAX_E = 1024;    // experts (one bit each in a 32-word bitmap)
// Per-CTA plan of a MoE call in dynamic shared memory: number of distinct experts, the
// selection bitmap and its word prefix counts, the distinct experts ascending, and for
// each distinct expert the slot through which each token selected it (-1: not selected).
constexpr int PLAN_BITS = 16, PLAN_PRE = PLAN_BITS + 128, PLAN_EX = PLAN_PRE + 128,
              PLAN_SLOT = PLAN_EX + 2 * MOE_MAX_PAIRS, PLAN_BYTES = PLAN_SLOT + MOE_MAX_PAIRS * MOE_MAX_T;

// Header of an activation-fragment slot, after the token blocks: the f16 range factor,
// the number of tokens of the segment, and (MODE_MOE_DOWN) the pair of each token.
constexpr int HDR_XUP = 0, HDR_MSEG = 4, HDR_PAIRS = 16, HDR_BYTES = 16 + 4 * MOE_MAX_T;

// The tiles cover one weight of N rows, or two (gate and up of an MLP): tiles [0, tiles_a)
// are rows of the first, the rest rows of the second, whose partial sums go to workspace
// columns [N, 2N) (row length ld = N or 2N).  MoE modes take their tiles from the plan.
struct MainArgs {
    const __nv_bfloat16* x;
    __nv_bfloat16* y;
    float* ws;
    uint32_t* status;
    int M, N, K, C, tiles, tiles_a, ld, stages, lands, stage_bytes, has_bias;
    // MoE modes
    const int32_t* idx;  // [T = M, topk] expert of each (token, slot); -1 marks an empty slot
    int topk, E, rpe, tpe, P, plan_off;
    // MODE_MOE_DOWN used for a gathered product: the activation row of pair p is
    // lhs[p] (checked against Bx; out of range gives a zero row), else p
    const int32_t* lhs;
    int Bx;
    // Plain modes: x rotated in the activation warp before its fragments are built
    // (Qwen38HadamardQuantizedLinear): signs (fp32 [K] or null), block (0: none), 1/sqrt(block)
    const float* signs;
    int rot;
    float rot_scale;
    // MODE_MOE_DOWN of the decode SwitchGLU: the indices come from the router two kernels
    // back, which has completed before this grid can start (the gate/up kernel triggers its
    // dependents only after waiting for the router), so the plan is built and the weights
    // stream before the wait for h.
    int early_plan;
};

// The rotation of an activation product: hadamardRotate's arguments.
struct Rot {
    const float* signs;
    int block;  // power of two <= 512 that divides K (one token only); 0 for none
};

// Rotation of one staged window of W = max(512, block) activations of a token (EPL = W / 32
// elements per lane, lane l holding [l * EPL, l * EPL + EPL)): signs first, then the
// butterfly stages h = 1, 2, 4, ... < block (lower element a + b, upper a - b: the pairs and
// order of the rotation kernel, so the results are the same bit for bit), the 1/sqrt(block)
// scale, and the rounding to bf16; the 512 activations of chunk `part` of the window are
// written to `dst`.
template <int EPL>
__device__ __forceinline__ void rotate_window(const uint8_t* src, uint8_t* dst, const float* signs, int block,
                                              float scale, int part, int lane) {
    float v[EPL];
    const uint32_t* w = reinterpret_cast<const uint32_t*>(src) + lane * (EPL / 2);
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
        const uint32_t u = w[i];
        v[2 * i] = bf16_bits_to_f32(u & 0xFFFFu);
        v[2 * i + 1] = bf16_bits_to_f32(u >> 16);
    }
    if (signs) {
#pragma unroll
        for (int i = 0; i < EPL; ++i) v[i] = v[i] * signs[lane * EPL + i];
    }
#pragma unroll
    for (int h = 1; h < EPL; h <<= 1) {
        if (h >= block) break;
#pragma unroll
        for (int i = 0; i < EPL; ++i)
            if ((i & h) == 0) {
                const float a = v[i], b = v[i + h];
                v[i] = a + b;
                v[i + h] = a - b;
            }
    }
    for (int lh = 1; lh < 32 && lh * EPL < block; lh <<= 1) {
        const bool upper = (lane & lh) != 0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const float q = __shfl_xor_sync(0xffffffffu, v[i], lh);
            v[i] = upper ? (q - v[i]) : (v[i] + q);
        }
    }
    __syncwarp();
    // lanes whose elements fall into the chunk write them (EPL * 32 = W, the chunk 512)
    const int first = lane * EPL - part * 512;
    if (first >= 0 && first < 512) {
        uint32_t* o = reinterpret_cast<uint32_t*>(dst) + first / 2;
#pragma unroll
        for (int i = 0; i < EPL / 2; ++i) o[i] = pack_bf16x2(v[2 * i] * scale, v[2 * i + 1] * scale);
    }
    __syncwarp();
}

// Accumulator columns.  An m16n8k16 product has 8 columns; with MP (1, 2, 4 or 8) token
// columns per group, one product serves 8/MP groups at once: column n = slot * MP + token,
// and the B operand of group g is non-zero only in the columns of its slot (g mod 8/MP).
// The MMAs of a chunk therefore accumulate 8/MP groups into one register set, and the
// per-group scales are applied once per chunk instead of once per group.

// Where the sums of one subunit go.
struct FlushDst {
    float* base;            // workspace at the subunit's chunk slot (MODE_ATOMIC: the region)
    int col0;               // workspace column of the tile's first row
    int nrows;              // rows of the tile that exist (64 except at the end of a plain weight)
    int ld;                 // workspace row length
    const int8_t* slot_of;  // MODE_MOE_GU: slot of each token for this expert (-1: not selected)
    const int* pairs;       // MODE_MOE_DOWN: pair of each segment token
    int mseg, topk;         // tokens with activations; slots per token
};

// Workspace row of token m, or -1 when nothing is stored for it.
template <int MODE>
__device__ __forceinline__ int out_row(const FlushDst& d, int m) {
    if (m >= d.mseg) return -1;
    if constexpr (MODE == MODE_MOE_GU) {
        const int s = d.slot_of[m];
        return s < 0 ? -1 : m * d.topk + s;
    } else if constexpr (MODE == MODE_MOE_DOWN) {
        return d.pairs[m];
    } else {
        return m;
    }
}

template <int MODE>
__device__ __forceinline__ void put(const FlushDst& d, int m, int r, float v) {
    const int row = out_row<MODE>(d, m);
    if (row < 0 || r >= d.nrows) return;
    float* p = d.base + static_cast<size_t>(row) * d.ld + d.col0 + r;
    if constexpr (MODE == MODE_ATOMIC)
        atomicAdd(p, v);
    else
        *p = v;
}

// Writes a warp's partial sums of one 16-row subtile after summing the columns that belong
// to the same token.  Stores and reductions are fire-and-forget: the epilogue kernel, which
// runs after this grid has completed, reads them.
template <int MODE, int MP, int TB>
__device__ __forceinline__ void flush_subtile(float (&acc)[TB][4], int warp, const FlushDst& d, int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int r0 = warp * 16 + g;  // row within the tile
#pragma unroll
    for (int tb = 0; tb < TB; ++tb) {
        if (MP == 1) {  // every column is token 0
            float v0 = acc[tb][0] + acc[tb][1], v2 = acc[tb][2] + acc[tb][3];
            v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
            v2 += __shfl_xor_sync(0xffffffffu, v2, 1);
            v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
            v2 += __shfl_xor_sync(0xffffffffu, v2, 2);
            if (t == 0) {
                put<MODE>(d, 0, r0, v0);
                put<MODE>(d, 0, r0 + 8, v2);
            }
            continue;
        }
        float v[4] = {acc[tb][0], acc[tb][1], acc[tb][2], acc[tb][3]};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (MP <= 2) v[e] += __shfl_xor_sync(0xffffffffu, v[e], 1);
            if (MP <= 4) v[e] += __shfl_xor_sync(0xffffffffu, v[e], 2);
        }
        const int writers = MP <= 2 ? 1 : MP / 2;
        if (t < writers) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = r0 + ((e >> 1) << 3);
                const int m = tb * 8 + (2 * t + (e & 1)) % MP;
                put<MODE>(d, m, r, v[e]);
            }
        }
    }
}

// y = bf16(partial sums); the sums are returned to zero for the next product (MODE_ATOMIC).
__global__ void __launch_bounds__(256) qgemv_epilogue(float* __restrict__ ws, __nv_bfloat16* __restrict__ y,
                                                      int total) {
    griddep_launch_dependents();
    griddep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        y[i] = __float2bfloat16_rn(__ldcg(ws + i));
        __stcg(ws + i, 0.0f);
    }
}

__device__ __forceinline__ float silu_mul_bf16(float g, float u) {
    g = bf16_bits_to_f32(f32_to_bf16_bits(g));
    u = bf16_bits_to_f32(f32_to_bf16_bits(u));
    return g / (1.0f + expf(-g)) * u;
}

// Ordered sums of the C chunk slots (MODE_SLOTS).  A block of 8 warps covers 8/S groups of
// 32 consecutive outputs; in a group, warp j adds the slots c = j, j + S, j + 2S, ... in that
// order (its loads in flight together), then the S warp sums are added in warp order.  S
// (1, 2, 4 or 8) depends only on the shape, so the result is bitwise reproducible; the host
// picks it so that small outputs still spread their loads over many threads.
constexpr int EPI_WARPS = 8;

__device__ __forceinline__ float slot_sum(const float* __restrict__ ws, size_t stride, int C, int j, int S) {
    float acc = 0.0f;
    int c = j;
    for (; c + 3 * S < C; c += 4 * S) {
        const float v0 = __ldcg(ws + static_cast<size_t>(c) * stride);
        const float v1 = __ldcg(ws + static_cast<size_t>(c + S) * stride);
        const float v2 = __ldcg(ws + static_cast<size_t>(c + 2 * S) * stride);
        const float v3 = __ldcg(ws + static_cast<size_t>(c + 3 * S) * stride);
        acc += v0;
        acc += v1;
        acc += v2;
        acc += v3;
    }
    for (; c < C; c += S) acc += __ldcg(ws + static_cast<size_t>(c) * stride);
    return acc;
}

int epilogue_split(long long total, int C) {
    // enough threads to hide the load latency (about 64K), at most C warps per group
    int S = 8;
    while (S > 1 && (total * S > 65536 || S > C)) S >>= 1;
    return S;
}

// y = bf16(ordered sum of the chunk slots [C][total]).
__global__ void __launch_bounds__(32 * EPI_WARPS) qgemv_epilogue_slots(const float* __restrict__ ws,
                                                                       __nv_bfloat16* __restrict__ y, int total, int C,
                                                                       int S) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float part[EPI_WARPS][32];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = EPI_WARPS / S, grp = w / S, j = w - grp * S;
    const int i = (blockIdx.x * G + grp) * 32 + lane;
    part[w][lane] = i < total ? slot_sum(ws + i, static_cast<size_t>(total), C, j, S) : 0.0f;
    __syncthreads();
    if (j == 0 && i < total) {
        float acc = part[w][lane];
        for (int q = 1; q < S; ++q) acc += part[w + q][lane];
        y[i] = __float2bfloat16_rn(acc);
    }
}

// The same from chunk slots [C][M][2N]: h = bf16(silu(bf16 g) * bf16 u).
__global__ void __launch_bounds__(32 * EPI_WARPS) qgemv_epilogue_glu_slots(const float* __restrict__ ws,
                                                                           __nv_bfloat16* __restrict__ h, int N,
                                                                           int total, int C, int S) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float pg[EPI_WARPS][32], pu[EPI_WARPS][32];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = EPI_WARPS / S, grp = w / S, j = w - grp * S;
    const int i = (blockIdx.x * G + grp) * 32 + lane;
    const int m = i / N, n = i - m * N;
    const float* base = ws + static_cast<size_t>(m) * 2 * N + n;
    const size_t stride = static_cast<size_t>(2) * total;
    pg[w][lane] = i < total ? slot_sum(base, stride, C, j, S) : 0.0f;
    pu[w][lane] = i < total ? slot_sum(base + N, stride, C, j, S) : 0.0f;
    __syncthreads();
    if (j == 0 && i < total) {
        float g = pg[w][lane], u = pu[w][lane];
        for (int q = 1; q < S; ++q) {
            g += pg[w + q][lane];
            u += pu[w + q][lane];
        }
        h[i] = __float2bfloat16_rn(silu_mul_bf16(g, u));
    }
}

// Shared memory: [0, 1 KiB) barriers, [1, 3 KiB) zeros (B operand of columns that do not
// belong to a group), [3 KiB, ...) the stage ring, then two activation-fragment slots and
// one staging copy of a chunk of x (and the MoE plan).
constexpr int ZERO_OFF = 1024, ZERO_BYTES = 2048, RING_OFF = 3072;
constexpr int MAX_DYN_SMEM = 226 * 1024;  // 227 KiB per CTA less the static per-group sums

// Gate/up epilogue: h = bf16(silu(g) * u) with g = bf16(gate sums), u = bf16(up sums),
// the rounding of an MLP whose gate and up projections return bf16; the sums [M][2N]
// are returned to zero (MODE_ATOMIC).
__global__ void __launch_bounds__(256) qgemv_epilogue_glu(float* __restrict__ ws, __nv_bfloat16* __restrict__ h,
                                                          int N, int total) {
    griddep_launch_dependents();
    griddep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int m = i / N, n = i - m * N;
        float* wg = ws + static_cast<size_t>(m) * 2 * N + n;
        h[i] = __float2bfloat16_rn(silu_mul_bf16(__ldcg(wg), __ldcg(wg + N)));
        __stcg(wg, 0.0f);
        __stcg(wg + N, 0.0f);
    }
}

// MoE: h[p, k] = bf16(silu(bf16 g) * bf16 u) of every selecting pair p from the gate/up
// chunk slots [C][P][2I] (chunks added in order); h is the down projection's activation.
__global__ void __launch_bounds__(256) moe_decode_glu(const float* __restrict__ ws, const int32_t* __restrict__ idx,
                                                      int P, int E, int I, int C, __nv_bfloat16* __restrict__ h) {
    griddep_launch_dependents();
    griddep_wait();
    const size_t ld = static_cast<size_t>(2) * I, cstride = static_cast<size_t>(P) * ld;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P * I; i += gridDim.x * blockDim.x) {
        const int p = i / I, k = i - p * I;
        const int e = idx[p];
        if (e < 0 || e >= E) continue;
        const float* src = ws + static_cast<size_t>(p) * ld + k;
        float g = 0.0f, u = 0.0f;
#pragma unroll 4
        for (int c = 0; c < C; ++c) {
            g += __ldcg(src + c * cstride);
            u += __ldcg(src + c * cstride + I);
        }
        h[i] = __float2bfloat16_rn(silu_mul_bf16(g, u));
    }
}

// MoE combine: out[t, r] = bf16(sum over slots s, in order, of score[t, s] * y_ts[r]) with
// y_ts = bf16(sum of the down chunk slots [C][P][H] of pair t*topk + s); empty or invalid
// slots contribute nothing (the weightedExpertSum of SwitchGLU, in its rounding).  One
// block row per token: the token's experts and scores are read once into shared memory,
// then every thread's loads of its output's expert rows are in flight together.
constexpr int COMBINE_MAXK = 32;

__global__ void __launch_bounds__(256) moe_decode_combine(const float* __restrict__ ws, const int32_t* __restrict__ idx,
                                                          const __nv_bfloat16* __restrict__ scores, int T, int topk,
                                                          int E, int H, int C, __nv_bfloat16* __restrict__ out) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float s_sc[COMBINE_MAXK];
    __shared__ int s_ok[COMBINE_MAXK];
    const int t = blockIdx.y;
    const int P = T * topk;
    if (threadIdx.x < topk) {
        const int p = t * topk + threadIdx.x;
        const int e = idx[p];
        s_ok[threadIdx.x] = e >= 0 && e < E;
        s_sc[threadIdx.x] = __bfloat162float(scores[p]);
    }
    __syncthreads();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= H) return;
    // every slot's first chunk in flight at once, then the further chunks (I > 512)
    const float* base = ws + static_cast<size_t>(t) * topk * H + r;
    const size_t cstride = static_cast<size_t>(P) * H;
    float y[COMBINE_MAXK];
#pragma unroll
    for (int s = 0; s < COMBINE_MAXK; ++s) y[s] = (s < topk && s_ok[s]) ? __ldcg(base + static_cast<size_t>(s) * H) : 0.0f;
    for (int c = 1; c < C; ++c) {
#pragma unroll
        for (int s = 0; s < COMBINE_MAXK; ++s)
            if (s < topk && s_ok[s]) y[s] += __ldcg(base + c * cstride + static_cast<size_t>(s) * H);
    }
    float acc = 0.0f;
#pragma unroll
    for (int s = 0; s < COMBINE_MAXK; ++s)
        if (s < topk && s_ok[s]) acc = __fadd_rn(acc, __fmul_rn(s_sc[s], bf16_bits_to_f32(f32_to_bf16_bits(y[s]))));
    out[static_cast<size_t>(t) * H + r] = __float2bfloat16_rn(acc);
}

// Gathered product: out[p, n] = bf16(sum of the chunk slots [C][P][N] of pair p, in chunk
// order), zeros for a pair whose expert index is outside [0, E).
__global__ void __launch_bounds__(256) gather_decode_out(const float* __restrict__ ws, const int32_t* __restrict__ rhs,
                                                         int P, int E, int N, int C, __nv_bfloat16* __restrict__ out) {
    griddep_launch_dependents();
    griddep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P * N; i += gridDim.x * blockDim.x) {
        const int p = i / N;
        const int e = rhs[p];
        float v = 0.0f;
        if (e >= 0 && e < E) {
            const float* src = ws + i;
#pragma unroll 4
            for (int c = 0; c < C; ++c) v += __ldcg(src + static_cast<size_t>(c) * P * N);
        }
        out[i] = __float2bfloat16_rn(v);
    }
}

// An f16 value (11 significant bits) as fp32 and as an exact sum of two bf16 values (8 and
// at most 3 significant bits), each duplicated into both halves of a word.
__device__ __forceinline__ void split_f16(uint16_t h, float& f, uint32_t& hi2, uint32_t& lo2) {
    f = __half2float(__ushort_as_half(h));
    const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(f));
    const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(f - __uint_as_float(hi << 16)));
    hi2 = hi | (hi << 16);
    lo2 = lo | (lo << 16);
}

// Position of stage i of a CTA: its k-chunk and tile, in (chunk, tile) order.
struct StageCursor {
    int chunk, tile, tiles;
    __device__ __forceinline__ void next() {
        if (++tile == tiles) {
            tile = 0;
            ++chunk;
        }
    }
};

// Where tile `tile` of a kernel lives: which weight (0 or 1), the TMA row of its first row,
// the rows that exist, the workspace column of its first row, and (MoE) the index of its
// expert among the distinct experts.
template <int MODE>
struct TileInfo {
    int wsel, row0, nrows, col0, dslot;
    __device__ __forceinline__ TileInfo(const MainArgs& a, int tile, int nd, const int16_t* ex) {
        if constexpr (MODE == MODE_MOE_GU) {
            const int per = nd * a.tpe;
            wsel = tile >= per;
            const int jj = wsel ? tile - per : tile;
            dslot = jj / a.tpe;
            const int rt = jj - dslot * a.tpe;
            row0 = ex[dslot] * a.rpe + rt * 64;
            nrows = 64;
            col0 = wsel * a.rpe + rt * 64;
        } else if constexpr (MODE == MODE_MOE_DOWN) {
            wsel = 0;
            dslot = tile / a.tpe;
            const int rt = tile - dslot * a.tpe;
            row0 = ex[dslot] * a.rpe + rt * 64;
            nrows = 64;
            col0 = rt * 64;
        } else {
            wsel = tile >= a.tiles_a;
            const int lt = wsel ? tile - a.tiles_a : tile;
            row0 = lt * 64;
            nrows = min(64, a.N - lt * 64);
            col0 = (wsel ? a.N : 0) + lt * 64;
            dslot = 0;
        }
    }
};

// Activation segment of a stage: stages with equal keys share their activation fragments.
template <int MODE>
__device__ __forceinline__ int seg_key(const MainArgs& a, int chunk, int tile) {
    if constexpr (MODE == MODE_MOE_DOWN)
        return chunk * MOE_MAX_PAIRS + tile / a.tpe;
    else
        return chunk;
}

// PACK: f16 scales and biases with group 128 (the layout of the Bonsai 2 packs); each 64-k
// subgroup uses the scale of its 128-group, read from a stage box that holds the 8 groups of
// an aligned pair of chunks.
template <int BITS, int MP, int TB, bool PACK, int MODE, bool ROT = false>
__global__ void __launch_bounds__(THREADS, WG == 1 && TB == 1 ? 3 : 2) qgemv_main(const __grid_constant__ WeightMaps maps,
                                                                      const __grid_constant__ WeightMaps maps_b,
                                                                      const MainArgs a) {
    using F = Fmt<BITS>;
    constexpr bool MOE = MODE == MODE_MOE_GU || MODE == MODE_MOE_DOWN;
    constexpr int GPER = 8 / MP;                 // groups sharing one accumulator set
    constexpr int UG = 2;                        // groups extracted together
    constexpr int FLUSH = TB == 1 ? GROUPS : UG; // groups between scale applications
    constexpr int LIVE = TB == 1 ? MP : UG;      // accumulator sets alive between applications
    constexpr int SPLIT = (TB == 1 && MP <= 2 && UG == 2) ? 2 : 1;  // shorter MMA chains
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    // Landing barriers: stage i signals full[i % lands], lands = lcm(stages, WG).  A parity
    // wait only tells the awaited phase from its neighbours, so each waiter must be within
    // one phase of the barrier.  When WG does not divide the ring, a data slot passes from
    // group to group, and one group could reach a slot's next stage before another group's
    // stage in that slot had landed.  With a period that WG divides, every phase of a
    // landing barrier belongs to one group, which has waited for the previous phase itself;
    // with a period that the ring divides, the next phase cannot land before this one is
    // consumed (each stage lands only after the previous stage of its data slot is consumed).
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + a.lands;
    uint64_t* xfull = empty + a.stages;
    uint64_t* xempty = xfull + 2;
    const uint8_t* zeros = smem + ZERO_OFF;
    uint8_t* stage0 = smem + RING_OFF;
    uint8_t* xslots = stage0 + static_cast<size_t>(a.stages) * a.stage_bytes;
    const int xslot_bytes = a.M * F::XF_PER_M + HDR_BYTES;
    uint8_t* xstage = xslots + 2 * xslot_bytes;
    __shared__ float s_xs[GROUPS][16], s_xp[GROUPS][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // MoE: the plan, computed by every CTA from the routing indices (written by an earlier
    // kernel on the stream, so everything waits for it first).
    int nd = 0;
    const int16_t* ex = nullptr;
    const int8_t* slot_tab = nullptr;
    int tiles = a.tiles;
    if constexpr (MOE) {
        if (!(MODE == MODE_MOE_DOWN && a.early_plan)) griddep_wait();
        uint8_t* plan = smem + a.plan_off;
        uint32_t* bits = reinterpret_cast<uint32_t*>(plan + PLAN_BITS);
        int* pre = reinterpret_cast<int*>(plan + PLAN_PRE);
        int16_t* exw = reinterpret_cast<int16_t*>(plan + PLAN_EX);
        int8_t* slw = reinterpret_cast<int8_t*>(plan + PLAN_SLOT);
        for (int i = threadIdx.x; i < 32; i += blockDim.x) bits[i] = 0u;
        for (int i = threadIdx.x; i < MOE_MAX_PAIRS * MOE_MAX_T / 4; i += blockDim.x)
            reinterpret_cast<uint32_t*>(slw)[i] = 0xFFFFFFFFu;
        __syncthreads();
        bool bad = false;
        for (int i = threadIdx.x; i < a.P; i += blockDim.x) {
            const int e = __ldcg(a.idx + i);  // past L1: written by another grid
            if (e >= 0 && e < a.E)
                atomicOr(&bits[e >> 5], 1u << (e & 31));
            else if (e != -1)
                bad = true;
        }
        if (bad && blockIdx.x == 0) atomicOr(a.status, Q38_DEV_BAD_INDEX);
        __syncthreads();
        if (warp == 0) {
            uint32_t w = bits[lane];
            const int c = __popc(w);
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            int base = incl - c;
            pre[lane] = base;
            while (w) {
                exw[base++] = static_cast<int16_t>(lane * 32 + __ffs(w) - 1);
                w &= w - 1;
            }
            if (lane == 31) *reinterpret_cast<int*>(plan) = incl;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < a.P; i += blockDim.x) {
            const int e = __ldcg(a.idx + i);
            if (e < 0 || e >= a.E) continue;
            const int j = pre[e >> 5] + __popc(bits[e >> 5] & ((1u << (e & 31)) - 1u));
            slw[j * MOE_MAX_T + i / a.topk] = static_cast<int8_t>(i % a.topk);
        }
        __syncthreads();
        nd = *reinterpret_cast<const int*>(plan);
        ex = exw;
        slot_tab = slw;
        tiles = (MODE == MODE_MOE_GU ? 2 : 1) * nd * a.tpe;
    }

    // Subunit range of this CTA in (chunk, tile, subtile) order: a CTA covers one or two
    // chunks of k, so its activation fragments are built once per chunk (MODE_MOE_DOWN: once
    // per chunk and expert).
    const int total_sub = tiles * a.C * 4;  // host guarantees < 2^31
    const int s0 = static_cast<int>(static_cast<long long>(total_sub) * blockIdx.x / gridDim.x);
    const int s1 = static_cast<int>(static_cast<long long>(total_sub) * (blockIdx.x + 1) / gridDim.x);
    if (s1 <= s0) return;
    const int st_first = s0 >> 2, st_last = (s1 - 1) >> 2;
    const int nst = st_last - st_first + 1;
    const int lo_first = s0 - 4 * st_first, hi_last = s1 - 4 * st_last;

    for (int i = threadIdx.x; i < ZERO_BYTES / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem + ZERO_OFF)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (!a.has_bias)  // the bias operands of the offset-and-bias steps are then zeros
        for (int i = threadIdx.x; i < a.stages * 64; i += blockDim.x)
            reinterpret_cast<uint4*>(stage0 + static_cast<size_t>(i >> 6) * a.stage_bytes + NCW * F::SUB_BYTES +
                                     1024)[i & 63] = make_uint4(0u, 0u, 0u, 0u);
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.lands; ++i) mbar_init(&full[i], 1);
        for (int i = 0; i < a.stages; ++i) mbar_init(&empty[i], NCW);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], NCW * WG);
        }
        fence_mbar_init();
    }
    __syncthreads();
    // The next kernel on the stream may start now: it waits for this grid before reading
    // or writing anything this grid touches.
    griddep_launch_dependents();

    if (warp == NCW * WG) {
        // ------------------------------------------------------------ weight producer
        // Streams codes, scales and biases; they are read-only inputs, so the ring fills
        // while the previous kernel on the stream is still finishing (plain modes).
        if (lane == 0) {
            prefetch_tensormap(&maps.codes16);
            prefetch_tensormap(&maps.codes64);
            prefetch_tensormap(&maps.scales);
            if (a.has_bias) prefetch_tensormap(&maps.biases);
            if (MODE == MODE_MOE_GU || a.tiles_a < a.tiles) {
                prefetch_tensormap(&maps_b.codes16);
                prefetch_tensormap(&maps_b.codes64);
                prefetch_tensormap(&maps_b.scales);
                if (a.has_bias) prefetch_tensormap(&maps_b.biases);
            }
            StageCursor cur{st_first / tiles, st_first % tiles, tiles};
            int slot = 0, fslot = 0;
            uint32_t ph = 0;
            for (int i = 0; i < nst; ++i) {
                if (i >= a.stages && !mbar_wait(&empty[slot], ph ^ 1, a.status)) {
                    // the consumers have given up: let the copies already issued land
                    // before the CTA can exit (each wait is bounded)
                    for (int j = i - a.stages; j < i; ++j)
                        if (!mbar_wait(&full[j % a.lands], (j / a.lands) & 1, a.status)) break;
                    return;
                }
                const int sub_lo = i == 0 ? lo_first : 0;
                const int sub_hi = i == nst - 1 ? hi_last : 4;
                uint8_t* sbase = stage0 + static_cast<size_t>(slot) * a.stage_bytes;
                uint64_t* fb = &full[fslot];
                const TileInfo<MODE> ti(a, cur.tile, nd, ex);
                const WeightMaps& wm = ti.wsel ? maps_b : maps;
                // whole 64-row tiles inside the matrix in one box per column range,
                // otherwise one 16-row box per active subtile
                const bool whole = sub_lo == 0 && sub_hi == 4 && ti.nrows == 64;
                int nact = 0;
                for (int s = sub_lo; s < sub_hi; ++s) nact += (16 * s < ti.nrows);
                if (whole) nact = 4;
                const uint32_t bytes = nact * F::SUB_BYTES + 1024 + (a.has_bias ? 1024 : 0);
                mbar_arrive_expect_tx(fb, bytes);
                if (whole) {
#pragma unroll
                    for (int bx = 0; bx < F::BOXES; ++bx)
                        tma_load_2d(sbase + bx * 64 * F::SW, &wm.codes64, fb,
                                    cur.chunk * F::ROW_WORDS + bx * (F::SW / 4), ti.row0);
                } else {
                    for (int s = sub_lo; s < sub_hi; ++s) {
                        if (16 * s >= ti.nrows) continue;
#pragma unroll
                        for (int bx = 0; bx < F::BOXES; ++bx)
                            tma_load_2d(sbase + bx * 64 * F::SW + s * 16 * F::SW, &wm.codes16, fb,
                                        cur.chunk * F::ROW_WORDS + bx * (F::SW / 4), ti.row0 + 16 * s);
                    }
                }
                uint8_t* sc = sbase + NCW * F::SUB_BYTES;
                const int gx = PACK ? (cur.chunk >> 1) * GROUPS : cur.chunk * GROUPS;  // 16-byte aligned
                tma_load_2d(sc, &wm.scales, fb, gx, ti.row0);
                if (a.has_bias) tma_load_2d(sc + 1024, &wm.biases, fb, gx, ti.row0);
                if (++slot == a.stages) {
                    slot = 0;
                    ph ^= 1;
                }
                if (++fslot == a.lands) fslot = 0;
                cur.next();
            }
        }
        return;
    }

    if (warp == NCW * WG + 1) {
        // ------------------------------------------------------------ activation warp
        // x is written by the previous kernel on the stream: wait for it to complete.
        if constexpr (!MOE) griddep_wait();
        if constexpr (MODE == MODE_MOE_DOWN) {
            if (a.early_plan) griddep_wait();  // h comes from the previous kernel
        }
        StageCursor cur{st_first / tiles, st_first % tiles, tiles};
        int ci = -1, key = -1;
        for (int i = 0; i < nst; ++i, cur.next()) {
            const int k2 = seg_key<MODE>(a, cur.chunk, cur.tile);
            if (k2 == key) continue;
            key = k2;
            ++ci;
            const int c = cur.chunk;
            uint8_t* slotp = xslots + (ci & 1) * xslot_bytes;
            uint8_t* hdr = slotp + a.M * F::XF_PER_M;
            int mseg = a.M;
            if constexpr (MODE == MODE_MOE_DOWN) {
                // tokens that selected this expert, in token order, and their pairs; their
                // activations are the rows of h (bf16 [P, K]) of those pairs
                const int js = cur.tile / a.tpe;
                const int8_t* so = slot_tab + js * MOE_MAX_T;
                const int s_l = lane < a.M ? so[lane] : -1;
                const uint32_t sel = __ballot_sync(0xffffffffu, s_l >= 0);
                mseg = __popc(sel);
                const bool ok = ci < 2 || mbar_wait(&xempty[ci & 1], ((ci >> 1) & 1) ^ 1, a.status);
                if (!ok) return;
                int* prs = reinterpret_cast<int*>(hdr + HDR_PAIRS);
                if (s_l >= 0) prs[__popc(sel & ((1u << lane) - 1u))] = lane * a.topk + s_l;
                if (lane == 0) *reinterpret_cast<int*>(hdr + HDR_MSEG) = mseg;
                __syncwarp();
                for (int q = lane; q < mseg * (KC / 8); q += 32) {
                    const int m = q / (KC / 8), o = q % (KC / 8);
                    int row = prs[m];
                    if (a.lhs) {
                        row = a.lhs[row];
                        if (row < 0 || row >= a.Bx) {  // a zero row; reported once per CTA and chunk
                            *reinterpret_cast<uint4*>(xstage + m * (KC * 2) + o * 16) = make_uint4(0u, 0u, 0u, 0u);
                            if (o == 0 && blockIdx.x == 0) atomicOr(a.status, Q38_DEV_BAD_INDEX);
                            continue;
                        }
                    }
                    cp_async16(xstage + m * (KC * 2) + o * 16, a.x + static_cast<size_t>(row) * a.K + c * KC + o * 8);
                }
                cp_async_commit();
                cp_async_wait<0>();
                __syncwarp();
            } else {
                // all of the chunk's copies in flight at once
                for (int p = lane; p < a.M * (KC / 8); p += 32) {
                    const int m = p / (KC / 8), q = p % (KC / 8);
                    cp_async16(xstage + m * (KC * 2) + q * 16, a.x + static_cast<size_t>(m) * a.K + c * KC + q * 8);
                }
                cp_async_commit();
                const bool ok = ci < 2 || mbar_wait(&xempty[ci & 1], ((ci >> 1) & 1) ^ 1, a.status);
                cp_async_wait<0>();
                __syncwarp();
                if (!ok) return;
                if (lane == 0) *reinterpret_cast<int*>(hdr + HDR_MSEG) = mseg;
                if constexpr (ROT) {  // one token, blocks of at most a chunk
                    rotate_window<16>(xstage, xstage, a.signs ? a.signs + c * KC : nullptr, a.rot, a.rot_scale, 0, lane);
                }
            }
            build_fragments<BITS>(xstage, mseg, slotp, hdr, s_xs, s_xp, lane);
            if (lane == 0) mbar_arrive(&xfull[ci & 1]);
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    // The partial sums may still be in use by the previous product's epilogue until it
    // has completed.
    if constexpr (!MOE) griddep_wait();
    const int wgrp = warp / NCW;  // this warp's group: it computes the stages i with i % WG == wgrp
    const int sw_i = warp % NCW;  // and, in each, subtile sw_i
    const int g = lane >> 2, t = lane & 3;
    const bool odd = (t & 1) != 0;
    // swizzled code offsets of (row g, group gi); row g+8 is 8*SW bytes further
    uint32_t offA[GROUPS], offB[GROUPS];
#pragma unroll
    for (int gi = 0; gi < GROUPS; ++gi) {
        int w0, w1;
        window_words<BITS>(gi, t, w0, w1);
        offA[gi] = code_off<F::SW>(g, w0);
        offB[gi] = code_off<F::SW>(g, w1);
    }
    constexpr uint32_t ROW8 = 8 * F::SW;
    // B operand of column g (this lane's column): token and group slot
    const int ml = g % MP, gsl = g / MP;
    int tok[TB];
#pragma unroll
    for (int tb = 0; tb < TB; ++tb) tok[tb] = TB == 1 ? ml : tb * 8 + g;
    const int srow0 = sw_i * 16 + g;  // scale row of row g (row g+8 is 64 halfwords further)

    int cur_key = -1, ci = -1;
    int mseg = a.M;
    const uint8_t* xf = xslots;
    float xup = 1.0f;  // range factor of the chunk's f16 activations
    // per group: where this lane's B operand comes from (its fragments, or zeros)
    const uint8_t* pg[TB == 1 ? GROUPS : TB];
    StageCursor cur{st_first / tiles, st_first % tiles, tiles};
    int slot = 0, fslot = 0;  // data slot i % stages, landing barrier i % lands
    uint32_t fph = 0;         // phase parity of the landing barrier
    int own = 0;  // i % WG
    for (int i = 0; i < nst; ++i) {
        const int sub_lo = i == 0 ? lo_first : 0;
        const int sub_hi = i == nst - 1 ? hi_last : 4;
        const int chunk = cur.chunk;
        const int key = seg_key<MODE>(a, chunk, cur.tile);
        if (key != cur_key) {
            // the previous segment's fragments are no longer needed; wait for this one's
            if (ci >= 0) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&xempty[ci & 1]);
            }
            ++ci;
            if (!mbar_wait(&xfull[ci & 1], (ci >> 1) & 1, a.status)) return;
            cur_key = key;
            xf = xslots + (ci & 1) * xslot_bytes;
            const uint8_t* hdr = xf + a.M * F::XF_PER_M;
            if (F::F16) xup = *reinterpret_cast<const float*>(hdr + HDR_XUP);
            mseg = *reinterpret_cast<const int*>(hdr + HDR_MSEG);
            if (TB == 1) {
#pragma unroll
                for (int gi = 0; gi < (TB == 1 ? GROUPS : TB); ++gi)
                    pg[gi] = (tok[0] < mseg && gi % GPER == gsl) ? xf + tok[0] * F::XF_PER_M + t * 16 : zeros;
            } else {
#pragma unroll
                for (int tb = 0; tb < TB; ++tb) pg[tb] = tok[tb] < mseg ? xf + tok[tb] * F::XF_PER_M + t * 16 : zeros;
            }
        }
        const bool mine = own == wgrp;
        const TileInfo<MODE> ti(a, cur.tile, nd, ex);
        const bool active = mine && sw_i >= sub_lo && sw_i < sub_hi && 16 * sw_i < ti.nrows;
        if (mine && !mbar_wait(&full[fslot], fph, a.status)) return;
        float acc[TB][4];
        if (active) {
            const uint8_t* sbase = stage0 + static_cast<size_t>(slot) * a.stage_bytes;
            const uint8_t* sub = sbase + sw_i * 16 * F::SW;
            const uint16_t* scl = reinterpret_cast<const uint16_t*>(sbase + NCW * F::SUB_BYTES) + srow0 * GROUPS;
            // scales of rows g and g+8 for groups 2t, 2t+1 (one bf16 word each), biases likewise;
            // PACK: both groups lie in 128-group t, whose f16 scale is split into bf16 high and
            // low words for the offset-and-bias steps and used in fp32 for the group sums
            uint32_t s_g, s_g8, b_g, b_g8, s_gl = 0, s_g8l = 0, b_gl = 0, b_g8l = 0;
            float f_g = 0.f, f_g8 = 0.f;
            if constexpr (!PACK) {
                const uint32_t* sw = reinterpret_cast<const uint32_t*>(scl) + t;
                s_g = sw[0];
                s_g8 = sw[32];
                b_g = sw[256];
                b_g8 = sw[256 + 32];
            } else {
                const uint16_t* sp = scl + (chunk & 1) * 4 + t;
                float fb;
                split_f16(sp[0], f_g, s_g, s_gl);
                split_f16(sp[64], f_g8, s_g8, s_g8l);
                split_f16(sp[512], fb, b_g, b_gl);
                split_f16(sp[512 + 64], fb, b_g8, b_g8l);
            }
#pragma unroll
            for (int tb = 0; tb < TB; ++tb)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[tb][e] = 0.f;
            float d[LIVE * SPLIT][TB][4];
            // code windows and B operands of a pair of groups; loaded one pair ahead
            auto load_pair = [&](int gb, uint32_t (&w)[UG][2][4], uint2 (&xb)[UG][TB][F::SPG]) {
#pragma unroll
                for (int u = 0; u < UG; ++u) {
                    load_window<BITS>(sub, offA[gb + u], offB[gb + u], odd, w[u][0]);
                    load_window<BITS>(sub + ROW8, offA[gb + u], offB[gb + u], odd, w[u][1]);
                }
#pragma unroll
                for (int u = 0; u < UG; ++u) {
                    const int gi = gb + u;
#pragma unroll
                    for (int tb = 0; tb < TB; ++tb) {
                        const uint8_t* p = TB == 1 ? pg[gi % (TB == 1 ? GROUPS : TB)] : pg[tb % (TB == 1 ? GROUPS : TB)];
#pragma unroll
                        for (int j = 0; j < F::SPG; ++j)
                            xb[u][tb][j] = *reinterpret_cast<const uint2*>(p + (gi * (F::SPG / 2) + j / 2) * 64 + (j & 1) * 8);
                    }
                }
            };
            uint32_t wn[UG][2][4];
            uint2 xn[UG][TB][F::SPG];
            load_pair(0, wn, xn);
#pragma unroll
            for (int gb = 0; gb < GROUPS; gb += UG) {
                if (gb % FLUSH == 0) {
#pragma unroll
                    for (int s = 0; s < LIVE * SPLIT; ++s)
#pragma unroll
                        for (int tb = 0; tb < TB; ++tb)
#pragma unroll
                            for (int e = 0; e < 4; ++e) d[s][tb][e] = 0.f;
                }
                uint32_t w[UG][2][4], ar[UG][2][F::NP];
                uint2 xb[UG][TB][F::SPG];
#pragma unroll
                for (int u = 0; u < UG; ++u)
#pragma unroll
                    for (int r = 0; r < 2; ++r)
#pragma unroll
                        for (int k = 0; k < 4; ++k) w[u][r][k] = wn[u][r][k];
#pragma unroll
                for (int u = 0; u < UG; ++u)
#pragma unroll
                    for (int tb = 0; tb < TB; ++tb)
#pragma unroll
                        for (int j = 0; j < F::SPG; ++j) xb[u][tb][j] = xn[u][tb][j];
                if (gb + UG < GROUPS) load_pair(gb + UG, wn, xn);
#pragma unroll
                for (int u = 0; u < UG; ++u) {
                    if constexpr (F::F16) {
                        extract16<BITS>(w[u][0], ar[u][0]);
                        extract16<BITS>(w[u][1], ar[u][1]);
                    } else {
                        extract<BITS>(w[u][0], ar[u][0]);
                        extract<BITS>(w[u][1], ar[u][1]);
                    }
                }
#pragma unroll
                for (int j = 0; j < F::SPG; ++j)
#pragma unroll
                    for (int u = 0; u < UG; ++u) {
                        const int gi = gb + u;
                        const int s = ((gi / GPER) % LIVE) + (SPLIT > 1 ? LIVE * u : 0);
#pragma unroll
                        for (int tb = 0; tb < TB; ++tb) {
                            if constexpr (F::F16)
                                mma_f16_16816(d[s][tb], ar[u][0][2 * j], ar[u][1][2 * j], ar[u][0][2 * j + 1],
                                              ar[u][1][2 * j + 1], xb[u][tb][j].x, xb[u][tb][j].y, d[s][tb]);
                            else
                                mma_bf16_16816(d[s][tb], ar[u][0][2 * j], ar[u][1][2 * j], ar[u][0][2 * j + 1],
                                               ar[u][1][2 * j + 1], xb[u][tb][j].x, xb[u][tb][j].y, d[s][tb]);
                        }
                    }
                if ((gb + UG) % FLUSH == 0) {
                    // scale the finished sets: column 2t + c of set s belongs to group
                    // (set index) * GPER + (2t + c) / MP
                    const int gset0 = (gb + UG - FLUSH) / GPER;  // absolute index of live set 0
#pragma unroll
                    for (int s = 0; s < LIVE; ++s) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            float sc;
                            if (MP == 1) {  // groups 2t, 2t+1: the words loaded above
                                if constexpr (PACK) {
                                    sc = (e >> 1) ? f_g8 : f_g;
                                } else {
                                    const uint32_t wv = (e >> 1) ? s_g8 : s_g;
                                    sc = __uint_as_float((e & 1) ? (wv & 0xFFFF0000u) : (wv << 16));
                                }
                            } else {
                                const int gi = (gset0 + s) * GPER + (2 * t) / MP;
                                if constexpr (PACK)
                                    sc = __half2float(__ushort_as_half(scl[((e >> 1) << 6) + (chunk & 1) * 4 + gi / 2]));
                                else
                                    sc = bf16_bits_to_f32(scl[((e >> 1) << 6) + gi]);
                            }
                            if (F::F16) sc *= xup;
#pragma unroll
                            for (int tb = 0; tb < TB; ++tb) {
                                float v = d[s][tb][e];
                                if (SPLIT > 1) v += d[s + LIVE][tb][e];
                                acc[tb][e] = fmaf(sc, v, acc[tb][e]);
                            }
                        }
                    }
                }
            }
            // offset and bias terms of the chunk's 8 groups: two MMA steps (high and low
            // parts of the sums) into column (slot 0, token), which the flush adds to the
            // token's other columns.  A = (scales of groups 0-7, biases of groups 0-7).
#pragma unroll
            for (int tb = 0; tb < TB; ++tb) {
                uint4 bb = make_uint4(0u, 0u, 0u, 0u);
                const int mt = tb * 8 + g;  // token of column g in slot 0
                if (mt < mseg && (TB > 1 || g < MP))
                    bb = *reinterpret_cast<const uint4*>(xf + mt * F::XF_PER_M + F::XF_FRAG + t * 16);
                mma_bf16_16816(acc[tb], s_g, s_g8, b_g, b_g8, bb.x, bb.y, acc[tb]);
                mma_bf16_16816(acc[tb], s_g, s_g8, b_g, b_g8, bb.z, bb.w, acc[tb]);
                if constexpr (PACK) {  // the low bf16 parts of the f16 scales and biases
                    mma_bf16_16816(acc[tb], s_gl, s_g8l, b_gl, b_g8l, bb.x, bb.y, acc[tb]);
                    mma_bf16_16816(acc[tb], s_gl, s_g8l, b_gl, b_g8l, bb.z, bb.w, acc[tb]);
                }
            }
        }
        // Release the stage before writing the sums: the arrive orders this warp's earlier
        // memory operations, and the stores have not completed yet.
        if (mine) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (active) {
            FlushDst dst;
            dst.col0 = ti.col0;
            dst.nrows = ti.nrows;
            dst.ld = a.ld;
            dst.mseg = mseg;
            dst.topk = a.topk;
            dst.slot_of = nullptr;
            dst.pairs = nullptr;
            if constexpr (MODE == MODE_ATOMIC) {
                dst.base = a.ws;
            } else if constexpr (MODE == MODE_SLOTS) {
                dst.base = a.ws + static_cast<size_t>(chunk) * a.M * a.ld;
            } else {
                dst.base = a.ws + static_cast<size_t>(chunk) * a.P * a.ld;
                if constexpr (MODE == MODE_MOE_GU) dst.slot_of = slot_tab + ti.dslot * MOE_MAX_T;
                if constexpr (MODE == MODE_MOE_DOWN)
                    dst.pairs = reinterpret_cast<const int*>(xf + a.M * F::XF_PER_M + HDR_PAIRS);
            }
            flush_subtile<MODE, MP, TB>(acc, sw_i, dst, lane);
        }
        if (++own == WG) own = 0;
        if (++slot == a.stages) slot = 0;
        if (++fslot == a.lands) {
            fslot = 0;
            fph ^= 1;
        }
        cur.next();
    }
}

// Launch geometry shared by the context path and the allocation-free path.
struct Plan {
    int C, tiles, stage_bytes, stages, smem, plan_off;
};

template <int BITS>
bool make_plan(int M, int K, int N, Plan& p, bool two_weights = false, bool moe = false) {
    using F = Fmt<BITS>;
    p.C = K / KC;
    p.tiles = (N + 63) / 64 * (two_weights ? 2 : 1);
    if (static_cast<long long>(p.tiles) * p.C * 4 >= (1LL << 31)) return false;
    p.stage_bytes = NCW * F::SUB_BYTES + 2048;  // a multiple of 1 KiB
    // fragment slots (with their headers) + staging copy of x (+ the MoE plan)
    const int xbytes = 2 * (M * F::XF_PER_M + HDR_BYTES) + M * KC * 2 + (moe ? PLAN_BYTES + 16 : 0);
    // 76 KiB per CTA in all (ring, header, zeros, fragments, alignment slack, 1 KiB of
    // static sums) lets three CTAs (12 consumer warps) share an SM; 113 KiB two (also for
    // 9-16 tokens, where two CTAs per SM with registers capped at 102 beat one CTA with
    // more: 16 x 4096 -> 11008 4-bit 21.5 -> 18.5 us)
    const int budget = (WG == 1 ? (M > 8 ? 113 : 76) : 113) * 1024 - 1024 - RING_OFF - 1024 - xbytes;
    int stages = budget / p.stage_bytes;
    if (stages > 8) stages = 8;  // (the lcm(stages, WG) + stages + 4 barriers then fit the first 1 KiB)
    if (stages < 2) stages = 2;
    int smem = 1024 + RING_OFF + stages * p.stage_bytes + xbytes;  // + alignment slack
    while (smem > MAX_DYN_SMEM && stages > 2) {
        --stages;
        smem = 1024 + RING_OFF + stages * p.stage_bytes + xbytes;
    }
    p.stages = stages;
    p.smem = smem;
    // the plan sits after the staging copy of x, 16-byte aligned (offsets from the
    // 1024-aligned base)
    p.plan_off = static_cast<int>(align_up(static_cast<size_t>(RING_OFF) + static_cast<size_t>(stages) * p.stage_bytes +
                                               2 * (M * F::XF_PER_M + HDR_BYTES) + M * KC * 2,
                                           16));
    return smem <= MAX_DYN_SMEM;
}

// Encodes the tensor maps of a weight (codes in two box heights, scales, biases).
template <int BITS>
bool make_maps(const uint32_t* w, const void* s, const void* b, int K, int N, WeightMaps* m, bool pack = false) {
    using F = Fmt<BITS>;
    const uint64_t kw = static_cast<uint64_t>(K) * BITS / 32;
    const CUtensorMapSwizzle swz = F::SW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const CUtensorMapDataType sdt = pack ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const int group = pack ? 128 : 64;
    return make_map_2d(&m->codes16, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w, kw, N, F::SW / 4, 16, swz) &&
           make_map_2d(&m->codes64, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w, kw, N, F::SW / 4, 64, swz) &&
           make_map_2d(&m->scales, sdt, 2, s, K / group, N, GROUPS, 64, CU_TENSOR_MAP_SWIZZLE_NONE) &&
           make_map_2d(&m->biases, sdt, 2, b ? b : s, K / group, N, GROUPS, 64, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Encoded maps of recently used weights.  A decode loop calls the same projections again
// and again, and the encoding depends only on the pointers and the shape, so a hit is
// always valid (a new weight at an old address with the same shape encodes identically).
template <int BITS, bool PACK = false>
bool cached_maps(const uint32_t* w, const void* s, const void* b, int K, int N, WeightMaps* maps) {
    struct Entry {
        const void* w;
        const void* s;
        const void* b;
        int K, N;
        bool used;
        WeightMaps maps;
    };
    static std::mutex mu;
    static Entry cache[64];
    const uintptr_t h = (reinterpret_cast<uintptr_t>(w) >> 8) ^ (reinterpret_cast<uintptr_t>(s) >> 6) ^
                        static_cast<uintptr_t>(K) * 31u ^ static_cast<uintptr_t>(N) * 17u;
    Entry& e = cache[(h ^ (h >> 12)) & 63u];
    std::lock_guard<std::mutex> lk(mu);
    if (e.used && e.w == w && e.s == s && e.b == b && e.K == K && e.N == N) {
        *maps = e.maps;
        return true;
    }
    if (!make_maps<BITS>(w, s, b, K, N, maps, PACK)) return false;
    e.w = w;
    e.s = s;
    e.b = b;
    e.K = K;
    e.N = N;
    e.maps = *maps;
    e.used = true;
    return true;
}

// Per template instance and device (and context): the shared-memory opt-in of the main
// kernel and its occupancy at a given ring size.  (Templated on the instance's parameters,
// not on the kernel's type, which all instances share: each instance keeps its own state.)
template <int BITS, int MP, int TB, bool PACK, int MODE, bool ROT = false>
cudaError_t configure_main(int device, int smem, int* occ_out) {
    auto kmain = qgemv_main<BITS, MP, TB, PACK, MODE, ROT>;
    static std::mutex mu;
    static const void* configured[64] = {};
    static int occ_smem[64][16] = {}, occ_val[64][16] = {};
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(mu);
    const void* key = current_context_key();
    if (!key || configured[device] != key) {
        cudaError_t e = cudaFuncSetAttribute(kmain, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_DYN_SMEM);
        if (e != cudaSuccess) return e;
        configured[device] = key;
        for (int i = 0; i < 16; ++i) occ_smem[device][i] = 0;
    }
    int occ = 0, slot = -1;
    for (int i = 0; i < 16; ++i) {
        if (occ_smem[device][i] == smem) {
            occ = occ_val[device][i];
            break;
        }
        if (occ_smem[device][i] == 0 && slot < 0) slot = i;
    }
    if (occ == 0) {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kmain, THREADS, smem);
        if (occ < 1) occ = 1;
        if (slot >= 0) {
            occ_smem[device][slot] = smem;
            occ_val[device][slot] = occ;
        }
    }
    *occ_out = occ;
    return cudaSuccess;
}

MainArgs base_args(const Plan& p, const void* x, int M, int K, int N, float* part, uint32_t* status, bool has_bias) {
    MainArgs args = {};
    args.x = static_cast<const __nv_bfloat16*>(x);
    args.ws = part;
    args.status = status;
    args.M = M;
    args.N = N;
    args.K = K;
    args.C = p.C;
    args.tiles = p.tiles;
    args.tiles_a = p.tiles;
    args.ld = N;
    args.stages = p.stages;
    args.lands = std::lcm(p.stages, WG);
    args.stage_bytes = p.stage_bytes;
    args.has_bias = has_bias;
    args.plan_off = p.plan_off;
    return args;
}

cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, cudaLaunchAttribute* attr) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// Launches the main kernel on `args` over `total_sub` subunits (an upper bound for MoE).
template <int BITS, int MP, int TB, bool PACK, int MODE, bool ROT = false>
cudaError_t launch_main(const Plan& p, int device, int num_sms, const WeightMaps& maps, const WeightMaps& maps_b,
                        const MainArgs& args, long long total_sub, cudaStream_t stream) {
    auto kmain = qgemv_main<BITS, MP, TB, PACK, MODE, ROT>;
    int occ = 0;
    cudaError_t e = configure_main<BITS, MP, TB, PACK, MODE, ROT>(device, p.smem, &occ);
    if (e != cudaSuccess) return e;
    long long grid = static_cast<long long>(num_sms) * occ;
    if (grid > total_sub) grid = total_sub;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>(grid)), dim3(THREADS), p.smem, stream, attr);
    return cudaLaunchKernelEx(&cfg, kmain, maps, maps_b, args);
}

int epilogue_blocks(long long total, int num_sms) {
    long long b = (total + 255) / 256;
    if (b > num_sms * 4) b = num_sms * 4;
    return static_cast<int>(b < 1 ? 1 : b);
}

// Launches the main kernel and the epilogue with the given scratch.  Returns a CUDA error code.
// With `maps_b` the tiles cover two weights of N rows each (gate, then up) and the epilogue
// writes y = bf16(silu(gate) * up) [M, N].  SLOTS: partial sums per k-chunk in `part`
// (C x M x N floats, 2N with maps_b), added in order by the epilogue; otherwise `part` is
// the zero-at-rest region of M x N (2N) floats.
template <int BITS, int MP, int TB, bool PACK = false, bool SLOTS = true, bool ROT = false>
cudaError_t launch_kernels(const Plan& p, int device, int num_sms, const void* x, int M, int K,
                           const WeightMaps& maps, bool has_bias, int N, void* y, float* part, uint32_t* status,
                           cudaStream_t stream, const WeightMaps* maps_b = nullptr, Rot rot = Rot{nullptr, 0}) {
    constexpr int MODE = SLOTS ? MODE_SLOTS : MODE_ATOMIC;
    MainArgs args = base_args(p, x, M, K, N, part, status, has_bias);
    args.signs = rot.signs;
    args.rot = rot.block;
    args.rot_scale = rot.block ? 1.0f / sqrtf(static_cast<float>(rot.block)) : 1.0f;
    args.y = static_cast<__nv_bfloat16*>(y);
    args.tiles_a = maps_b ? p.tiles / 2 : p.tiles;
    args.ld = maps_b ? 2 * N : N;
    const long long total_sub = static_cast<long long>(p.tiles) * p.C * 4;
    cudaError_t e = launch_main<BITS, MP, TB, PACK, MODE, ROT>(p, device, num_sms, maps, maps_b ? *maps_b : maps,
                                                               args, total_sub, stream);
    if (e != cudaSuccess) return e;

    const int total = M * N;
    cudaLaunchAttribute attr[1];
    const int S = epilogue_split(total, p.C), G = EPI_WARPS / S;
    cudaLaunchConfig_t ecfg =
        SLOTS ? pdl_config(dim3((total + 32 * G - 1) / (32 * G)), dim3(32 * EPI_WARPS), 0, stream, attr)
              : pdl_config(dim3(epilogue_blocks(total, num_sms)), dim3(256), 0, stream, attr);
    __nv_bfloat16* yb = static_cast<__nv_bfloat16*>(y);
    if (SLOTS)
        e = maps_b ? cudaLaunchKernelEx(&ecfg, qgemv_epilogue_glu_slots, static_cast<const float*>(part), yb, N, total,
                                        p.C, S)
                   : cudaLaunchKernelEx(&ecfg, qgemv_epilogue_slots, static_cast<const float*>(part), yb, total, p.C,
                                        S);
    else
        e = maps_b ? cudaLaunchKernelEx(&ecfg, qgemv_epilogue_glu, part, yb, N, total)
                   : cudaLaunchKernelEx(&ecfg, qgemv_epilogue, part, yb, total);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// Chunk slots of a plain product in the context's workspace.
q38_status slot_workspace(q38_ctx* ctx, const Plan& p, int M, int N, bool two, float** out) {
    const size_t bytes = static_cast<size_t>(p.C) * M * N * (two ? 2 : 1) * sizeof(float);
    q38_status st = ensure_workspace(ctx, bytes);
    if (st != Q38_OK) return st;
    *out = static_cast<float*>(ctx->workspace);
    return Q38_OK;
}

// The partial sums of a context's product: chunk slots in the workspace when the context
// asks for reproducible results, else the zero-at-rest region of M x N (x2) floats.
q38_status partial_sums(q38_ctx* ctx, const Plan& p, int M, int N, bool two, float** out) {
    if (ctx->deterministic) return slot_workspace(ctx, p, M, N, two, out);
    uint32_t* unused = nullptr;
    return ensure_zero_region(ctx, 0, static_cast<size_t>(M) * N * (two ? 2 : 1), &unused, out);
}

template <int BITS, int MP, int TB, bool PACK = false>
cudaError_t launch_ctx(q38_ctx* ctx, const Plan& p, const void* x, int M, int K, const WeightMaps& maps,
                       bool has_bias, int N, void* y, float* part, const WeightMaps* maps_b = nullptr,
                       Rot rot = Rot{nullptr, 0}) {
    if constexpr (MP == 1 && TB == 1) {  // rotation inside the kernel: one token, blocks <= 512
        if (rot.block) {
            if (ctx->deterministic)
                return launch_kernels<BITS, 1, 1, PACK, true, true>(p, ctx->device, ctx->num_sms, x, M, K, maps,
                                                                    has_bias, N, y, part, ctx->d_status, ctx->stream,
                                                                    maps_b, rot);
            return launch_kernels<BITS, 1, 1, PACK, false, true>(p, ctx->device, ctx->num_sms, x, M, K, maps, has_bias,
                                                                 N, y, part, ctx->d_status, ctx->stream, maps_b, rot);
        }
    }
    if (ctx->deterministic)
        return launch_kernels<BITS, MP, TB, PACK, true>(p, ctx->device, ctx->num_sms, x, M, K, maps, has_bias, N, y,
                                                        part, ctx->d_status, ctx->stream, maps_b);
    return launch_kernels<BITS, MP, TB, PACK, false>(p, ctx->device, ctx->num_sms, x, M, K, maps, has_bias, N, y,
                                                     part, ctx->d_status, ctx->stream, maps_b);
}

template <int BITS, int MP, int TB>
q38_status launch(q38_ctx* ctx, const void* x, int M, int K, const uint32_t* w, const void* s,
                  const void* b, int N, void* y, Rot rot) {
    Plan p;
    if (!make_plan<BITS>(M, K, N, p)) return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: shape too large");
    float* part = nullptr;
    q38_status st = partial_sums(ctx, p, M, N, false, &part);
    if (st != Q38_OK) return st;
    WeightMaps maps;
    if (!cached_maps<BITS>(w, s, b, K, N, &maps))
        return fail(ctx, Q38_ERR_CUDA, "quantized_matmul: tensor map encoding failed");
    const cudaError_t e = launch_ctx<BITS, MP, TB>(ctx, p, x, M, K, maps, b != nullptr, N, y, part, nullptr, rot);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_CUDA, "quantized_matmul: launch failed: %s", cudaGetErrorString(e));
    }
    return Q38_OK;
}

// The same product over f16 scales with group 128 (PACK).
template <int BITS, int MP, int TB>
q38_status launch_pack(q38_ctx* ctx, const void* x, int M, int K, const uint32_t* w, const void* s,
                       const void* b, int N, void* y, Rot rot) {
    Plan p;
    if (!make_plan<BITS>(M, K, N, p)) return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: shape too large");
    float* part = nullptr;
    q38_status st = partial_sums(ctx, p, M, N, false, &part);
    if (st != Q38_OK) return st;
    WeightMaps maps;
    if (!cached_maps<BITS, true>(w, s, b, K, N, &maps))
        return fail(ctx, Q38_ERR_CUDA, "quantized_matmul: tensor map encoding failed");
    const cudaError_t e = launch_ctx<BITS, MP, TB, true>(ctx, p, x, M, K, maps, b != nullptr, N, y, part, nullptr, rot);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_CUDA, "quantized_matmul: launch failed: %s", cudaGetErrorString(e));
    }
    return Q38_OK;
}

// Gate and up projections of an MLP in one pass: h = bf16(silu(x.Wg^T) * (x.Wu^T)).
template <int BITS, int MP, int TB, bool PACK = false>
q38_status launch_gate_up(q38_ctx* ctx, const void* x, int M, int K, const uint32_t* wg, const void* sg,
                          const void* bg, const uint32_t* wu, const void* su, const void* bu, int N, void* h,
                          Rot rot) {
    Plan p;
    if (!make_plan<BITS>(M, K, N, p, true)) return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_gate_up: shape too large");
    float* part = nullptr;
    q38_status st = partial_sums(ctx, p, M, N, true, &part);
    if (st != Q38_OK) return st;
    WeightMaps mg, mu;
    if (!cached_maps<BITS, PACK>(wg, sg, bg, K, N, &mg) || !cached_maps<BITS, PACK>(wu, su, bu, K, N, &mu))
        return fail(ctx, Q38_ERR_CUDA, "quantized_gate_up: tensor map encoding failed");
    const cudaError_t e = launch_ctx<BITS, MP, TB, PACK>(ctx, p, x, M, K, mg, bg != nullptr, N, h, part, &mu, rot);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_CUDA, "quantized_gate_up: launch failed: %s", cudaGetErrorString(e));
    }
    return Q38_OK;
}

// Decode-shaped SwitchGLU: gate/up over the selected experts (all T tokens' activations,
// only selecting pairs stored), down over the same experts with h formed from the gate/up
// slots, then the score-weighted combine.  Three launches, chained with programmatic
// dependent launch; scratch: the chunk slots of both products in the workspace.
template <int BITS, int MP, int TB>
q38_status launch_moe_decode(q38_ctx* ctx, const void* x, int T, int H, int I, int E, int topk, const int32_t* idx,
                             const void* scores, const uint32_t* gw, const void* gs, const void* gb,
                             const uint32_t* uw, const void* us, const void* ub, const uint32_t* dw, const void* ds,
                             const void* db, void* out) {
    const int P = T * topk;
    const int nd_max = std::min(E, P);
    Plan pg, pd;
    // gate/up: K = H, rows per expert I; down: K = I, rows per expert H
    if (!make_plan<BITS>(T, H, nd_max * I, pg, true, true) || !make_plan<BITS>(T, I, nd_max * H, pd, false, true))
        return fail(ctx, Q38_ERR_UNSUPPORTED, "switch_glu: decode plan does not fit");
    const size_t gu_floats = static_cast<size_t>(pg.C) * P * 2 * I;
    const size_t dn_floats = static_cast<size_t>(pd.C) * P * H;
    const size_t h_bytes = align_up(static_cast<size_t>(P) * I * 2, 256);
    q38_status st = ensure_workspace(ctx, (gu_floats + dn_floats) * sizeof(float) + h_bytes);
    if (st != Q38_OK) return st;
    float* gu_slots = static_cast<float*>(ctx->workspace);
    float* dn_slots = gu_slots + gu_floats;
    __nv_bfloat16* hbuf = reinterpret_cast<__nv_bfloat16*>(dn_slots + dn_floats);
    WeightMaps mg, mu, md;
    if (!cached_maps<BITS>(gw, gs, gb, H, E * I, &mg) || !cached_maps<BITS>(uw, us, ub, H, E * I, &mu) ||
        !cached_maps<BITS>(dw, ds, db, I, E * H, &md))
        return fail(ctx, Q38_ERR_CUDA, "switch_glu: tensor map encoding failed");
    const bool has_bias = gb != nullptr;

    MainArgs a = base_args(pg, x, T, H, 0, gu_slots, ctx->d_status, has_bias);
    a.idx = idx;
    a.topk = topk;
    a.E = E;
    a.P = P;
    a.rpe = I;
    a.tpe = I / 64;
    a.ld = 2 * I;
    cudaError_t e = launch_main<BITS, MP, TB, false, MODE_MOE_GU>(pg, ctx->device, ctx->num_sms, mg, mu, a,
                                                                  static_cast<long long>(pg.tiles) * pg.C * 4,
                                                                  ctx->stream);
    cudaLaunchAttribute attr[1];
    if (e == cudaSuccess) {
        cudaLaunchConfig_t cfg = pdl_config(dim3(epilogue_blocks(static_cast<long long>(P) * I, ctx->num_sms)),
                                            dim3(256), 0, ctx->stream, attr);
        e = cudaLaunchKernelEx(&cfg, moe_decode_glu, static_cast<const float*>(gu_slots), idx, P, E, I, pg.C, hbuf);
    }
    if (e == cudaSuccess) {
        MainArgs d = base_args(pd, hbuf, T, I, 0, dn_slots, ctx->d_status, has_bias);
        d.idx = idx;
        d.topk = topk;
        d.E = E;
        d.P = P;
        d.rpe = H;
        d.tpe = H / 64;
        d.ld = H;
        d.early_plan = 1;
        e = launch_main<BITS, MP, TB, false, MODE_MOE_DOWN>(pd, ctx->device, ctx->num_sms, md, md, d,
                                                            static_cast<long long>(pd.tiles) * pd.C * 4, ctx->stream);
    }
    if (e == cudaSuccess) {
        cudaLaunchConfig_t cfg = pdl_config(dim3((H + 255) / 256, T), dim3(256), 0, ctx->stream, attr);
        e = cudaLaunchKernelEx(&cfg, moe_decode_combine, static_cast<const float*>(dn_slots), idx,
                               static_cast<const __nv_bfloat16*>(scores), T, topk, E, H, pd.C,
                               static_cast<__nv_bfloat16*>(out));
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_CUDA, "switch_glu: decode launch failed: %s", cudaGetErrorString(e));
    }
    return Q38_OK;
}

// Gathered product of up to 16 pairs (one activation row each): the down-projection mode
// of the decode kernel over the pairs' distinct experts, then the chunk sums.
template <int BITS, int MP, int TB>
q38_status launch_gather(q38_ctx* ctx, const void* x, int Bx, int K, const uint32_t* w, const void* s, const void* b,
                         int E, int N, const int32_t* lhs, const int32_t* rhs, int P, void* out) {
    Plan pd;
    if (!make_plan<BITS>(P, K, std::min(E, P) * N, pd, false, true))
        return fail(ctx, Q38_ERR_UNSUPPORTED, "gather_quantized_matmul: decode plan does not fit");
    q38_status st = ensure_workspace(ctx, static_cast<size_t>(pd.C) * P * N * sizeof(float));
    if (st != Q38_OK) return st;
    float* slots = static_cast<float*>(ctx->workspace);
    WeightMaps md;
    if (!cached_maps<BITS>(w, s, b, K, E * N, &md))
        return fail(ctx, Q38_ERR_CUDA, "gather_quantized_matmul: tensor map encoding failed");
    MainArgs d = base_args(pd, x, P, K, 0, slots, ctx->d_status, b != nullptr);
    d.idx = rhs;
    d.topk = 1;
    d.E = E;
    d.P = P;
    d.rpe = N;
    d.tpe = N / 64;
    d.ld = N;
    d.lhs = lhs;
    d.Bx = Bx;
    cudaError_t e = launch_main<BITS, MP, TB, false, MODE_MOE_DOWN>(pd, ctx->device, ctx->num_sms, md, md, d,
                                                                    static_cast<long long>(pd.tiles) * pd.C * 4,
                                                                    ctx->stream);
    if (e == cudaSuccess) {
        cudaLaunchAttribute attr[1];
        cudaLaunchConfig_t cfg = pdl_config(dim3(epilogue_blocks(static_cast<long long>(P) * N, ctx->num_sms)),
                                            dim3(256), 0, ctx->stream, attr);
        e = cudaLaunchKernelEx(&cfg, gather_decode_out, static_cast<const float*>(slots), rhs, P, E, N, pd.C,
                               static_cast<__nv_bfloat16*>(out));
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_CUDA, "gather_quantized_matmul: decode launch failed: %s", cudaGetErrorString(e));
    }
    return Q38_OK;
}

// Token layout by M: MP token columns per group slot, TB blocks of 8 tokens.
template <int BITS, typename L>
q38_status dispatch_m(int M, L&& run) {
    if (M == 1) return run(std::integral_constant<int, 1>(), std::integral_constant<int, 1>());
    if (M == 2) return run(std::integral_constant<int, 2>(), std::integral_constant<int, 1>());
    if (M <= 4) return run(std::integral_constant<int, 4>(), std::integral_constant<int, 1>());
    if (M <= 8) return run(std::integral_constant<int, 8>(), std::integral_constant<int, 1>());
    return run(std::integral_constant<int, 8>(), std::integral_constant<int, 2>());
}

}  // namespace

bool qgemv_fast_supported(int64_t M, int64_t K, int group, int bits, q38_dtype xd, q38_dtype sd,
                          const void* x, const void* w, const void* s, const void* b,
                          const void* y) {
    if (M < 1 || M > 16 || group != 64 || K % KC != 0 || K <= 0) return false;
    if (bits != 2 && bits != 3 && bits != 4 && bits != 8) return false;
    if (xd != Q38_BF16 || sd != Q38_BF16) return false;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!al(x) || !al(w) || !al(s) || (b && !al(b))) return false;
    (void)y;
    return true;
}

bool qgemv_pack_supported(int64_t M, int64_t K, int group, int bits, q38_dtype xd, q38_dtype sd,
                          const void* x, const void* w, const void* s, const void* b) {
    if (M < 1 || M > 16 || group != 128 || bits != 2 || K <= 0 || K % 1024 != 0) return false;
    if (xd != Q38_BF16 || sd != Q38_F16) return false;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return al(x) && al(w) && al(s) && (!b || al(b));
}

q38_status qgemv_pack(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w, const void* s,
                      const void* b, int64_t N, void* y, const float* signs, int rot_block) {
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    return dispatch_m<2>(m, [&](auto mp, auto tb) {
        return launch_pack<2, decltype(mp)::value, decltype(tb)::value>(ctx, x, m, k, w, s, b, n, y,
                                                                        Rot{signs, rot_block});
    });
}

q38_status qgemv_fast(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w,
                      const void* s, const void* b, int64_t N, int bits, void* y, const float* signs, int rot_block) {
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    auto go = [&](auto bits_c) {
        constexpr int B = decltype(bits_c)::value;
        return dispatch_m<B>(m, [&](auto mp, auto tb) {
            return launch<B, decltype(mp)::value, decltype(tb)::value>(ctx, x, m, k, w, s, b, n, y,
                                                                       Rot{signs, rot_block});
        });
    };
    switch (bits) {
        case 2: return go(std::integral_constant<int, 2>());
        case 3: return go(std::integral_constant<int, 3>());
        case 4: return go(std::integral_constant<int, 4>());
        case 8: return go(std::integral_constant<int, 8>());
    }
    return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: bits %d not on the fast path", bits);
}

q38_status qgemv_gate_up_pack(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* wg,
                              const void* sg, const void* bg, const uint32_t* wu, const void* su, const void* bu,
                              int64_t N, void* h, const float* signs, int rot_block) {
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    return dispatch_m<2>(m, [&](auto mp, auto tb) {
        return launch_gate_up<2, decltype(mp)::value, decltype(tb)::value, true>(ctx, x, m, k, wg, sg, bg, wu, su, bu,
                                                                               n, h, Rot{signs, rot_block});
    });
}

q38_status qgemv_gate_up_fast(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* wg,
                              const void* sg, const void* bg, const uint32_t* wu, const void* su, const void* bu,
                              int64_t N, int bits, void* h, const float* signs, int rot_block) {
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    auto go = [&](auto bits_c) {
        constexpr int B = decltype(bits_c)::value;
        return dispatch_m<B>(m, [&](auto mp, auto tb) {
            return launch_gate_up<B, decltype(mp)::value, decltype(tb)::value>(ctx, x, m, k, wg, sg, bg, wu, su, bu, n, h,
                                                                               Rot{signs, rot_block});
        });
    };
    switch (bits) {
        case 2: return go(std::integral_constant<int, 2>());
        case 3: return go(std::integral_constant<int, 3>());
        case 4: return go(std::integral_constant<int, 4>());
        case 8: return go(std::integral_constant<int, 8>());
    }
    return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_gate_up: bits %d not on the fast path", bits);
}

bool qgemv_moe_supported(int64_t T, int64_t H, int64_t I, int64_t E, int topk, int group, int bits, const void* x,
                         const void* gw, const void* gs, const void* gb, const void* uw, const void* us,
                         const void* ub, const void* dw, const void* ds, const void* db) {
    if (T < 1 || T > MOE_MAX_T || T * topk > MOE_MAX_PAIRS || topk > COMBINE_MAXK || E < 1 || E > MOE_MAX_E ||
        group != 64)
        return false;
    if (bits != 2 && bits != 3 && bits != 4 && bits != 8) return false;
    if (H % KC || I % KC || H <= 0 || I <= 0) return false;
    if (E * std::max(H, I) >= (1LL << 31)) return false;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    for (const void* p : {x, gw, gs, uw, us, dw, ds})
        if (!al(p)) return false;
    for (const void* p : {gb, ub, db})
        if (p && !al(p)) return false;
    return true;
}

q38_status qgemv_moe_decode(q38_ctx* ctx, const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int topk,
                            const int32_t* idx, const void* scores, const uint32_t* gw, const void* gs,
                            const void* gb, const uint32_t* uw, const void* us, const void* ub, const uint32_t* dw,
                            const void* ds, const void* db, int bits, void* out) {
    const int t = static_cast<int>(T), h = static_cast<int>(H), i = static_cast<int>(I), e = static_cast<int>(E);
    auto go = [&](auto bits_c) {
        constexpr int B = decltype(bits_c)::value;
        return dispatch_m<B>(t, [&](auto mp, auto tb) {
            return launch_moe_decode<B, decltype(mp)::value, decltype(tb)::value>(ctx, x, t, h, i, e, topk, idx, scores,
                                                                                  gw, gs, gb, uw, us, ub, dw, ds, db,
                                                                                  out);
        });
    };
    switch (bits) {
        case 2: return go(std::integral_constant<int, 2>());
        case 3: return go(std::integral_constant<int, 3>());
        case 4: return go(std::integral_constant<int, 4>());
        case 8: return go(std::integral_constant<int, 8>());
    }
    return fail(ctx, Q38_ERR_UNSUPPORTED, "switch_glu: bits %d not on the decode path", bits);
}

bool qgemv_gather_supported(int64_t M, int64_t K, int64_t E, int64_t N, int64_t P, int group, int bits, q38_dtype xd,
                            q38_dtype sd, const void* x, const void* w, const void* s, const void* b) {
    if (M != 1 || P < 1 || P > 256 || E < 1 || E > MOE_MAX_E || group != 64 || K % KC || K <= 0 || N % 64 || N <= 0)
        return false;
    if (bits != 2 && bits != 3 && bits != 4 && bits != 8) return false;
    if (xd != Q38_BF16 || sd != Q38_BF16 || E * N >= (1LL << 31)) return false;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return al(x) && al(w) && al(s) && (!b || al(b));
}

// Pairs in pieces of 16 (each piece reads the weights of its own distinct experts).
q38_status qgemv_gather(q38_ctx* ctx, const void* x, int64_t Bx, int64_t K, const uint32_t* w, const void* s,
                        const void* b, int64_t E, int64_t N, const int32_t* lhs, const int32_t* rhs, int64_t P,
                        int bits, void* out) {
    for (int64_t p0 = 0; p0 < P; p0 += MOE_MAX_T) {
        const int pc = static_cast<int>(std::min<int64_t>(MOE_MAX_T, P - p0));
        const int32_t* lh = lhs ? lhs + p0 : nullptr;
        const void* xp = lhs ? x : static_cast<const uint8_t*>(x) + static_cast<size_t>(p0) * K * 2;
        const int bx = lhs ? static_cast<int>(Bx) : pc;
        void* op = static_cast<uint8_t*>(out) + static_cast<size_t>(p0) * N * 2;
        auto go = [&](auto bits_c) {
            constexpr int B = decltype(bits_c)::value;
            return dispatch_m<B>(pc, [&](auto mp, auto tb) {
                return launch_gather<B, decltype(mp)::value, decltype(tb)::value>(
                    ctx, xp, bx, static_cast<int>(K), w, s, b, static_cast<int>(E), static_cast<int>(N), lh, rhs + p0,
                    pc, op);
            });
        };
        q38_status st;
        switch (bits) {
            case 2: st = go(std::integral_constant<int, 2>()); break;
            case 3: st = go(std::integral_constant<int, 3>()); break;
            case 4: st = go(std::integral_constant<int, 4>()); break;
            default: st = go(std::integral_constant<int, 8>()); break;
        }
        if (st != Q38_OK) return st;
    }
    return Q38_OK;
}

// ---------------------------------------------------------------------------------
// Allocation-free variant of the decode product (q38_quantized_matmul_noalloc).
//
// Some hosts cannot call cudaMalloc on the path where they run a projection: code
// that runs inside an allocator-free region (a custom memory manager that owns all
// device memory, a real-time decode loop that forbids allocation, or a plugin whose
// host framework hands it only input and output buffers).  This entry point takes its
// scratch from one fixed array in device memory, reserved when the library is loaded
// on a GPU and held until the process exits.
// ---------------------------------------------------------------------------------
namespace {

constexpr int64_t NA_MAX_M = 16, NA_MAX_N = 32768, NA_MAX_K = 32768;
constexpr size_t NA_ACC_BYTES = static_cast<size_t>(NA_MAX_M) * NA_MAX_N * 4;  // 2 MiB
constexpr size_t NA_STATUS_OFF = 0;
constexpr size_t NA_ACC_OFF = 256;
constexpr size_t NA_TOTAL = NA_ACC_OFF + NA_ACC_BYTES;

// The scratch of every no-alloc call on a device (status word, fp32 partial sums).  In
// host code this name is only a stand-in for the device array; its device address comes
// from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[NA_TOTAL];

std::mutex g_noalloc_mu;
struct NoallocDevice {
    const void* ctx_key;  // the context the address below belongs to
    uint8_t* ptr;
};
NoallocDevice g_noalloc[64] = {};

// Set-up, once per device and context, with that device current: resolve the array's
// device address and clear it (status word and partial sums start at zero; every
// product's epilogue returns the sums to zero, so no call clears them again).  The clear
// synchronises the device, which is why the first call must come before any capture.
q38_status noalloc_scratch(int device, uint8_t** out) {
    if (device < 0 || device >= 64) return Q38_ERR_INVALID_ARGUMENT;
    const void* key = current_context_key();
    if (!key) return Q38_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoallocDevice& d = g_noalloc[device];
    if (d.ctx_key != key || !d.ptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return Q38_ERR_CUDA;
        }
        if (cudaMemset(p, 0, NA_TOTAL) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            cudaGetLastError();
            return Q38_ERR_CUDA;
        }
        d.ptr = static_cast<uint8_t*>(p);
        d.ctx_key = key;
    }
    *out = d.ptr;
    return Q38_OK;
}

template <int BITS, int MP, int TB>
q38_status launch_noalloc(uint8_t* scratch, int device, int num_sms, const void* x, int M, int K,
                          const uint32_t* w, const void* s, const void* b, int N, void* y,
                          cudaStream_t stream) {
    Plan p;
    if (!make_plan<BITS>(M, K, N, p)) return Q38_ERR_UNSUPPORTED;
    uint32_t* status = reinterpret_cast<uint32_t*>(scratch + NA_STATUS_OFF);
    float* part = reinterpret_cast<float*>(scratch + NA_ACC_OFF);
    WeightMaps maps;
    if (!cached_maps<BITS>(w, s, b, K, N, &maps)) return Q38_ERR_CUDA;
    const cudaError_t e = launch_kernels<BITS, MP, TB, false, false>(p, device, num_sms, x, M, K, maps, b != nullptr,
                                                                     N, y, part, status, stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        // the main kernel may have run without its epilogue: put the sums back to zero
        cudaMemsetAsync(part, 0, static_cast<size_t>(M) * N * 4, stream);
        cudaGetLastError();
        return Q38_ERR_CUDA;
    }
    return Q38_OK;
}

}  // namespace
}  // namespace q38

extern "C" Q38_API q38_status q38_quantized_matmul_noalloc(const void* x, int64_t M, int64_t K,
                                                          const uint32_t* w, const void* scales,
                                                          const void* biases, int64_t N, int group_size,
                                                          int bits, void* y, void* stream) {
    using namespace q38;
    if (!x || !w || !scales || !y) return Q38_ERR_INVALID_ARGUMENT;
    if (group_size != 64 || (bits != 2 && bits != 3 && bits != 4 && bits != 8)) return Q38_ERR_UNSUPPORTED;
    if (M < 1 || N < 1 || K < KC || K % KC != 0) return Q38_ERR_INVALID_ARGUMENT;
    if (M > NA_MAX_M || N > NA_MAX_N || K > NA_MAX_K) return Q38_ERR_INVALID_ARGUMENT;  // beyond the fixed scratch
    if (!qgemv_fast_supported(M, K, group_size, bits, Q38_BF16, Q38_BF16, x, w, scales, biases, y))
        return Q38_ERR_INVALID_ARGUMENT;
    int device = 0, sms = 0;
    if (cudaGetDevice(&device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
        cudaGetLastError();
        return Q38_ERR_CUDA;
    }
    uint8_t* scratch = nullptr;
    q38_status st = noalloc_scratch(device, &scratch);
    if (st != Q38_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    auto go = [&](auto bits_c) {
        constexpr int B = decltype(bits_c)::value;
        return dispatch_m<B>(m, [&](auto mp, auto tb) {
            return launch_noalloc<B, decltype(mp)::value, decltype(tb)::value>(scratch, device, sms, x, m, k, w,
                                                                              scales, biases, n, y, s);
        });
    };
    switch (bits) {
        case 2: return go(std::integral_constant<int, 2>());
        case 3: return go(std::integral_constant<int, 3>());
        case 4: return go(std::integral_constant<int, 4>());
        default: return go(std::integral_constant<int, 8>());
    }
}

extern "C" Q38_API q38_status q38_noalloc_check_device(void* stream) {
    using namespace q38;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return Q38_ERR_CUDA;
    }
    uint8_t* scratch = nullptr;
    q38_status st = noalloc_scratch(device, &scratch);
    if (st != Q38_OK) return st;
    uint32_t v = 0;
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess ||
        cudaMemcpy(&v, scratch + NA_STATUS_OFF, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return Q38_ERR_CUDA;
    }
    if (v == 0) return Q38_OK;
    if (cudaMemsetAsync(scratch + NA_STATUS_OFF, 0, sizeof(v), static_cast<cudaStream_t>(stream)) != cudaSuccess ||
        cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess)
        cudaGetLastError();
    return (v & Q38_DEV_TIMEOUT) ? Q38_ERR_DEVICE_TIMEOUT : Q38_ERR_INVALID_ARGUMENT;
}
