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
//    active 16-row subtiles (swizzled boxes), the 64x8 bf16 scales and biases, and the
//    chunk's pre-arranged activation fragments.  Four consumer warps each own one
//    16-row subtile.  Stages cycle through an mbarrier ring.
//  * Codes are turned into bf16 operands without integer->float conversion: a code
//    masked into the mantissa of 0x4300 (bf16 128.0) reads as 128 + 2^p*q.  A tiny
//    prologue kernel permutes and scales the activations (x * 2^-p) into the MMA
//    fragment order that matches the extraction, and precomputes per-group sums.
//    One m16n8k16 bf16 MMA then dots 16 codes x 8 tokens; per group
//    D = sum(q*x) + 128*sum(x'), and y += scale*D.  The -128*scale*sum(x') and
//    bias*sum(x) terms of all 8 groups of a chunk are folded into two extra MMA
//    steps whose operands are the scales/biases and hi/lo bf16 splits of the sums.
//  * Consumers do no address arithmetic in the inner loop: swizzled code offsets are
//    precomputed per thread, fragments are token-major so their offsets are constants,
//    and the 8 groups of a stage are unrolled so their MMA chains overlap.
//  * Every warp adds its subtile partial sums into an fp32 workspace with fire-and-forget
//    reductions (no fences or counters in the main kernel); a small epilogue kernel
//    converts the sums to y and zeroes them again, so no per-call clearing is needed.
//  * The main kernel is launched with programmatic dependent launch: its producer
//    streams the first stages of weights while the prologue kernel is still running.
#include <mutex>

#include "affine_codes.cuh"

namespace q38 {
namespace {

using namespace dev;

constexpr int KC = 512;        // k per chunk
constexpr int GROUPS = 8;      // groups of 64 per chunk
constexpr int NCW = 4;         // consumer warps (one 16-row subtile each)
constexpr int THREADS = (NCW + 1) * 32;

template <int BITS>
struct Fmt {
    static constexpr int SPG = BITS == 8 ? 8 : 4;     // k16 MMA steps per group
    static constexpr int NP = 2 * SPG;                 // bf16x2 pairs per thread-row-group
    static constexpr int SW = BITS == 3 ? 64 : 128;    // swizzle span of a code box (bytes)
    static constexpr int ROW_BYTES = KC * BITS / 8;    // code bytes per row per chunk
    static constexpr int ROW_WORDS = ROW_BYTES / 4;
    static constexpr int BOXES = ROW_BYTES / SW;       // code boxes per subtile
    static constexpr int SUB_BYTES = 16 * ROW_BYTES;   // code bytes per subtile
    static constexpr int XF_FRAG = 256 * SPG;          // fragment bytes per token per chunk
    static constexpr int XF_PER_M = XF_FRAG + 64;      // + bias-step fragments
};

// Byte offset of word `wi` of subtile row `r` inside a subtile's swizzled code block
// (boxes of 16 rows x SW bytes, TMA swizzle of 16-byte chunks within SW-byte rows).
// Rows r and r+8 share the swizzle, so row r+8 sits exactly 8*SW bytes after row r.
template <int SW>
__device__ __forceinline__ uint32_t code_off(int r, int wi) {
    constexpr int WPB = SW / 4;  // words per box row
    const int box = wi / WPB, iw = wi % WPB;
    const int swz = SW == 128 ? (r & 7) : ((r >> 1) & 3);
    return box * (16 * SW) + r * SW + ((((iw >> 2) ^ swz)) << 4) + (iw & 3) * 4;
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
// Prologue: activation fragments + per-group sums, one CTA per 512-k chunk.
// Layout per chunk, token-major with a per-token stride of XF_PER_M bytes:
//   [m][group 8][half SPG/2][t 4][16 B]  then  [sigma 2][t 4][8 B] (bias-step operands).
// A 64-byte tail per token shifts consecutive tokens by 16 banks.
// ---------------------------------------------------------------------------------
template <int BITS>
__global__ void __launch_bounds__(256) qgemv_prep(const __nv_bfloat16* __restrict__ x, int M,
                                                  int K, uint8_t* __restrict__ xfrag) {
    using F = Fmt<BITS>;
    // Let the main kernel start streaming weights now; x is produced by the previous
    // kernel on the stream, and the fragment buffer is read by the previous product:
    // both are touched only after that kernel has completed.
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float s_xs[GROUPS][16], s_xp[GROUPS][16];
    const int c = blockIdx.x;
    uint8_t* base = xfrag + static_cast<size_t>(c) * M * F::XF_PER_M;
    const int items = GROUPS * M * 4;
    for (int i = threadIdx.x; i < items; i += blockDim.x) {
        const int t = i & 3, gm = i >> 2, m = gm % M, gi = gm / M;
        const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * K +
                                                          c * KC + gi * 64 + t * 16);
        const uint4 u0 = src[0], u1 = src[1];
        const uint32_t raw[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        float xv[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            xv[2 * j] = bf16_bits_to_f32(raw[j] & 0xFFFFu);
            xv[2 * j + 1] = bf16_bits_to_f32(raw[j] >> 16);
        }
        float xs = 0.f, xp = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) xs += xv[j];
        uint32_t* dst = reinterpret_cast<uint32_t*>(base + m * F::XF_PER_M + gi * (F::SPG / 2) * 64 + t * 16);
#pragma unroll
        for (int q = 0; q < F::NP; ++q) {
            const float lo = xv[pair_code<BITS>(q, 0)] * pair_mult<BITS>(q, 0);
            const float hi = xv[pair_code<BITS>(q, 1)] * pair_mult<BITS>(q, 1);
            xp += lo + hi;
            dst[(q / 4) * 16 + (q % 4)] = pack_bf16x2(lo, hi);
        }
        xs += __shfl_xor_sync(0xffffffffu, xs, 1);
        xs += __shfl_xor_sync(0xffffffffu, xs, 2);
        xp += __shfl_xor_sync(0xffffffffu, xp, 1);
        xp += __shfl_xor_sync(0xffffffffu, xp, 2);
        if (t == 0) {
            s_xs[gi][m] = xs;
            s_xp[gi][m] = xp;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 8 * M; i += blockDim.x) {
        const int t = i & 3, mm = i >> 2, m = mm % M, sigma = mm / M;
        uint32_t out[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int gi = 4 * sigma + 2 * h + (t >> 1);
            const float v = (t & 1) ? s_xs[gi][m] : s_xp[gi][m];
            const float vhi = bf16_bits_to_f32(f32_to_bf16_bits(v));
            const float vlo = v - vhi;
            const float f = (t & 1) ? 1.0f : -128.0f;
            out[h] = pack_bf16x2(vhi * f, vlo * f);
        }
        uint32_t* d = reinterpret_cast<uint32_t*>(base + m * F::XF_PER_M + F::XF_FRAG + sigma * 32 + t * 8);
        d[0] = out[0];
        d[1] = out[1];
    }
}

// ---------------------------------------------------------------------------------
// Main kernel.
// ---------------------------------------------------------------------------------
struct MainArgs {
    const uint8_t* xfrag;
    __nv_bfloat16* y;
    float* ws;
    uint32_t* status;
    int M, N, C, tiles, stages, stage_bytes, has_bias;
};

// Adds a warp's partial sums of one 16-row subtile into the fp32 workspace.  The
// reductions are fire-and-forget (no fence, no counter): the epilogue kernel, which
// runs after this grid has completed, converts the sums to y and zeroes them again.
template <int NT>
__device__ __forceinline__ void flush_subtile(const float (&acc)[NT][4], int tile, int warp,
                                              const MainArgs& a, int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int r0 = tile * 64 + warp * 16 + g;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = r0 + ((e >> 1) << 3), m = nt * 8 + 2 * t + (e & 1);
            if (r < a.N && m < a.M) atomicAdd(a.ws + static_cast<size_t>(m) * a.N + r, acc[nt][e]);
        }
}

// y = bf16(partial sums); the sums are returned to zero for the next product.
__global__ void __launch_bounds__(256) qgemv_epilogue(float* __restrict__ ws, __nv_bfloat16* __restrict__ y,
                                                      int total) {
    griddep_launch_dependents();
    griddep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        y[i] = __float2bfloat16_rn(__ldcg(ws + i));
        __stcg(ws + i, 0.0f);
    }
}

template <int BITS, int NT>
__global__ void __launch_bounds__(THREADS, NT == 1 ? 3 : 2) qgemv_main(const __grid_constant__ CUtensorMap map_codes,
                                                      const __grid_constant__ CUtensorMap map_scales,
                                                      const __grid_constant__ CUtensorMap map_biases,
                                                      const MainArgs a) {
    using F = Fmt<BITS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + a.stages;
    uint8_t* stage0 = smem + 1024;

    // subunit range of this CTA (host guarantees tiles * C * 4 < 2^31)
    const int total_sub = a.tiles * a.C * 4;
    const int s0 = static_cast<int>(static_cast<long long>(total_sub) * blockIdx.x / gridDim.x);
    const int s1 = static_cast<int>(static_cast<long long>(total_sub) * (blockIdx.x + 1) / gridDim.x);
    if (s1 <= s0) return;
    const int st_first = s0 >> 2, st_last = (s1 - 1) >> 2;
    const int nst = st_last - st_first + 1;
    const int lo_first = s0 - 4 * st_first, hi_last = s1 - 4 * st_last;
    const int xf_bytes = a.M * F::XF_PER_M;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NCW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    // The next product's prologue may start now: it waits for this grid before writing
    // anything this grid reads.
    griddep_launch_dependents();

    if (warp == NCW) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tensormap(&map_codes);
            prefetch_tensormap(&map_scales);
            if (a.has_bias) prefetch_tensormap(&map_biases);
            bool waited = false;
            int issued_xf = 0, xf_chunk = st_first % a.C;  // fragments issued so far, their next chunk
            int tile = st_first / a.C, chunk = st_first % a.C;
            for (int i = 0; i < nst; ++i) {
                const int slot = i % a.stages;
                const uint32_t ph = (i / a.stages) & 1;
                if (i >= a.stages && !mbar_wait(&empty[slot], ph ^ 1, a.status)) return;
                const int sub_lo = i == 0 ? lo_first : 0;
                const int sub_hi = i == nst - 1 ? hi_last : 4;
                uint8_t* sbase = stage0 + static_cast<size_t>(slot) * a.stage_bytes;
                int nact = 0;
                for (int s = sub_lo; s < sub_hi; ++s) nact += (tile * 64 + 16 * s < a.N);
                const uint32_t bytes = nact * F::SUB_BYTES + 1024 + (a.has_bias ? 1024 : 0) + xf_bytes;
                mbar_arrive_expect_tx(&full[slot], bytes);
                for (int s = sub_lo; s < sub_hi; ++s) {
                    if (tile * 64 + 16 * s >= a.N) continue;
#pragma unroll
                    for (int bx = 0; bx < F::BOXES; ++bx)
                        tma_load_2d(sbase + s * F::SUB_BYTES + bx * 16 * F::SW, &map_codes, &full[slot],
                                    chunk * F::ROW_WORDS + bx * (F::SW / 4), tile * 64 + 16 * s);
                }
                uint8_t* sc = sbase + NCW * F::SUB_BYTES;
                tma_load_2d(sc, &map_scales, &full[slot], chunk * GROUPS, tile * 64);
                if (a.has_bias) tma_load_2d(sc + 1024, &map_biases, &full[slot], chunk * GROUPS, tile * 64);
                // Activation fragments come from the prologue kernel: wait for it only
                // once the ring is full of weight loads.
                if (!waited && (i == a.stages - 1 || i == nst - 1)) {
                    griddep_wait();
                    waited = true;
                }
                if (waited) {
                    for (; issued_xf <= i; ++issued_xf) {
                        const int sl = issued_xf % a.stages;
                        uint8_t* dst = stage0 + static_cast<size_t>(sl) * a.stage_bytes + NCW * F::SUB_BYTES + 2048;
                        bulk_load(dst, a.xfrag + static_cast<size_t>(xf_chunk) * xf_bytes, xf_bytes, &full[sl]);
                        if (++xf_chunk == a.C) xf_chunk = 0;
                    }
                }
                if (++chunk == a.C) {
                    chunk = 0;
                    ++tile;
                }
            }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    // Partial sums, counters and y may still be in use by the previous product on the
    // stream until the prologue kernel (which waits for it) has completed.
    griddep_wait();
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
    // activation fragments: token m = nt*8 + g, quarter t
    uint32_t xoff[NT];
    bool xval[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int m = nt * 8 + g;
        xval[nt] = m < a.M;
        xoff[nt] = (xval[nt] ? m : 0) * F::XF_PER_M + t * 16;
    }
    const int srow0 = warp * 16 + g;  // scale row of row g (row g+8 is 64 halfwords further)
    const bool use_bias_operand = !odd || a.has_bias;
    const int ga0 = t >> 1;           // bias step: group offset of operand pair 0

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    int cur_tile = -1, nchunks = 0;
    int tile = st_first / a.C, chunk = st_first % a.C;
    for (int i = 0; i < nst; ++i) {
        const int slot = i % a.stages;
        const uint32_t ph = (i / a.stages) & 1;
        const int sub_lo = i == 0 ? lo_first : 0;
        const int sub_hi = i == nst - 1 ? hi_last : 4;
        if (tile != cur_tile) {
            if (nchunks > 0) flush_subtile<NT>(acc, cur_tile, warp, a, lane);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
            cur_tile = tile;
            nchunks = 0;
        }
        const bool active = warp >= sub_lo && warp < sub_hi && tile * 64 + 16 * warp < a.N;
        if (!mbar_wait(&full[slot], ph, a.status)) return;
        if (active) {
            const uint8_t* sbase = stage0 + static_cast<size_t>(slot) * a.stage_bytes;
            const uint8_t* sub = sbase + warp * F::SUB_BYTES;
            const uint16_t* scl = reinterpret_cast<const uint16_t*>(sbase + NCW * F::SUB_BYTES) + srow0 * GROUPS;
            const uint16_t* bia = scl + 512;
            const uint8_t* xf = sbase + NCW * F::SUB_BYTES + 2048;
            // two groups per iteration: independent MMA chains interleaved step by step
#pragma unroll
            for (int gp = 0; gp < GROUPS; gp += 2) {
                uint32_t w[2][2][4], ar[2][2][F::NP], xb[2][NT][F::NP];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int gi = gp + u;
                    load_window<BITS>(sub, offA[gi], offB[gi], odd, w[u][0]);
                    load_window<BITS>(sub + ROW8, offA[gi], offB[gi], odd, w[u][1]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int h = 0; h < F::SPG / 2; ++h) {
                            uint4 v = make_uint4(0u, 0u, 0u, 0u);
                            if (xval[nt])
                                v = *reinterpret_cast<const uint4*>(xf + xoff[nt] + (gi * (F::SPG / 2) + h) * 64);
                            xb[u][nt][4 * h + 0] = v.x;
                            xb[u][nt][4 * h + 1] = v.y;
                            xb[u][nt][4 * h + 2] = v.z;
                            xb[u][nt][4 * h + 3] = v.w;
                        }
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    extract<BITS>(w[u][0], ar[u][0]);
                    extract<BITS>(w[u][1], ar[u][1]);
                }
                float d[2][NT][4];
#pragma unroll
                for (int u = 0; u < 2; ++u)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) d[u][nt][e] = 0.f;
#pragma unroll
                for (int j = 0; j < F::SPG; ++j)
#pragma unroll
                    for (int u = 0; u < 2; ++u)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
                            mma_bf16_16816(d[u][nt], ar[u][0][2 * j], ar[u][1][2 * j], ar[u][0][2 * j + 1],
                                           ar[u][1][2 * j + 1], xb[u][nt][2 * j], xb[u][nt][2 * j + 1], d[u][nt]);
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const float sc0 = bf16_bits_to_f32(scl[gp + u]);
                    const float sc1 = bf16_bits_to_f32(scl[64 + gp + u]);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        acc[nt][0] = fmaf(sc0, d[u][nt][0], acc[nt][0]);
                        acc[nt][1] = fmaf(sc0, d[u][nt][1], acc[nt][1]);
                        acc[nt][2] = fmaf(sc1, d[u][nt][2], acc[nt][2]);
                        acc[nt][3] = fmaf(sc1, d[u][nt][3], acc[nt][3]);
                    }
                }
            }
            // bias and offset terms of the chunk's 8 groups: two MMA steps
            const uint16_t* src = odd ? bia : scl;
#pragma unroll
            for (int sigma = 0; sigma < 2; ++sigma) {
                const int ga = 4 * sigma + ga0, gb = ga + 2;
                const uint32_t v0a = use_bias_operand ? src[ga] * 0x00010001u : 0u;
                const uint32_t v1a = use_bias_operand ? src[64 + ga] * 0x00010001u : 0u;
                const uint32_t v0b = use_bias_operand ? src[gb] * 0x00010001u : 0u;
                const uint32_t v1b = use_bias_operand ? src[64 + gb] * 0x00010001u : 0u;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    uint2 bb = make_uint2(0u, 0u);
                    if (xval[nt])
                        bb = *reinterpret_cast<const uint2*>(xf + xoff[nt] - t * 16 + F::XF_FRAG + sigma * 32 + t * 8);
                    mma_bf16_16816(acc[nt], v0a, v1a, v0b, v1b, bb.x, bb.y, acc[nt]);
                }
            }
            ++nchunks;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++chunk == a.C) {
            chunk = 0;
            ++tile;
        }
    }
    if (nchunks > 0) flush_subtile<NT>(acc, cur_tile, warp, a, lane);
}

// Launch geometry shared by the context path and the allocation-free path.
struct Plan {
    int C, tiles, stage_bytes, stages, smem;
    size_t xf_bytes;
};

template <int BITS>
bool make_plan(int M, int K, int N, Plan& p) {
    using F = Fmt<BITS>;
    p.C = K / KC;
    p.tiles = (N + 63) / 64;
    if (static_cast<long long>(p.tiles) * p.C * 4 >= (1LL << 31)) return false;
    p.xf_bytes = static_cast<size_t>(M) * F::XF_PER_M;
    p.stage_bytes = static_cast<int>(align_up(NCW * F::SUB_BYTES + 2048 + p.xf_bytes, 1024));
    // about 72 KiB of ring per CTA lets three CTAs (12 consumer warps) share an SM
    int stages = (72 * 1024) / p.stage_bytes;
    if (stages > 6) stages = 6;
    if (stages < 2) stages = 2;
    int smem = 2048 + stages * p.stage_bytes;
    while (smem > 227 * 1024 && stages > 2) {
        --stages;
        smem = 2048 + stages * p.stage_bytes;
    }
    p.stages = stages;
    p.smem = smem;
    return smem <= 227 * 1024;
}

// Encodes the three tensor maps of a weight (codes, scales, biases).
template <int BITS>
bool make_maps(const uint32_t* w, const void* s, const void* b, int K, int N, CUtensorMap* mc,
               CUtensorMap* ms, CUtensorMap* mb) {
    using F = Fmt<BITS>;
    const uint64_t kw = static_cast<uint64_t>(K) * BITS / 32;
    return make_map_2d(mc, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w, kw, N, F::SW / 4, 16,
                       F::SW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B) &&
           make_map_2d(ms, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s, K / 64, N, GROUPS, 64,
                       CU_TENSOR_MAP_SWIZZLE_NONE) &&
           make_map_2d(mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b ? b : s, K / 64, N, GROUPS, 64,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Launches prologue + main kernel with the given scratch.  Returns a CUDA error code.
template <int BITS, int NT>
cudaError_t launch_kernels(const Plan& p, int device, int num_sms, const void* x, int M, int K,
                           const CUtensorMap& mc, const CUtensorMap& ms, const CUtensorMap& mb,
                           bool has_bias, int N, void* y, uint8_t* xfrag, float* part,
                           uint32_t* status, cudaStream_t stream) {
    auto kmain = qgemv_main<BITS, NT>;
    // per template instance and device: smem opt-in and occupancy at the largest ring
    static std::mutex mu;
    static bool configured[64] = {};
    static int occ_smem[64][16] = {}, occ_val[64][16] = {};
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    int occ = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!configured[device]) {
            cudaError_t e = cudaFuncSetAttribute(kmain, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            if (e != cudaSuccess) return e;
            configured[device] = true;
        }
        int slot = -1;
        for (int i = 0; i < 16; ++i) {
            if (occ_smem[device][i] == p.smem) {
                occ = occ_val[device][i];
                break;
            }
            if (occ_smem[device][i] == 0 && slot < 0) slot = i;
        }
        if (occ == 0) {
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kmain, THREADS, p.smem);
            if (occ < 1) occ = 1;
            if (slot >= 0) {
                occ_smem[device][slot] = p.smem;
                occ_val[device][slot] = occ;
            }
        }
    }
    const long long total_sub = static_cast<long long>(p.tiles) * p.C * 4;
    long long grid = static_cast<long long>(num_sms) * occ;
    if (grid > total_sub) grid = total_sub;

    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t pcfg = {};
    pcfg.gridDim = dim3(static_cast<unsigned>(p.C));
    pcfg.blockDim = dim3(256);
    pcfg.stream = stream;
    pcfg.attrs = attr;
    pcfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&pcfg, qgemv_prep<BITS>, static_cast<const __nv_bfloat16*>(x), M, K, xfrag);
    if (e != cudaSuccess) return e;

    MainArgs args;
    args.xfrag = xfrag;
    args.y = static_cast<__nv_bfloat16*>(y);
    args.ws = part;
    args.status = status;
    args.M = M;
    args.N = N;
    args.C = p.C;
    args.tiles = p.tiles;
    args.stages = p.stages;
    args.stage_bytes = p.stage_bytes;
    args.has_bias = has_bias;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kmain, mc, ms, mb, args);
    if (e != cudaSuccess) return e;

    const int total = M * N;
    int eblocks = (total + 255) / 256;
    if (eblocks > num_sms * 4) eblocks = num_sms * 4;
    cudaLaunchConfig_t ecfg = {};
    ecfg.gridDim = dim3(static_cast<unsigned>(eblocks));
    ecfg.blockDim = dim3(256);
    ecfg.stream = stream;
    ecfg.attrs = attr;
    ecfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&ecfg, qgemv_epilogue, part, static_cast<__nv_bfloat16*>(y), total);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <int BITS, int NT>
q38_status launch(q38_ctx* ctx, const void* x, int M, int K, const uint32_t* w, const void* s,
                  const void* b, int N, void* y) {
    Plan p;
    if (!make_plan<BITS>(M, K, N, p)) return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: shape too large");
    q38_status st = ensure_workspace(ctx, p.C * p.xf_bytes);
    if (st != Q38_OK) return st;
    uint32_t* cnt = nullptr;  // (no counters are used)
    float* part = nullptr;
    st = ensure_zero_region(ctx, 0, static_cast<size_t>(M) * N, &cnt, &part);
    if (st != Q38_OK) return st;
    CUtensorMap mc, ms, mb;
    if (!make_maps<BITS>(w, s, b, K, N, &mc, &ms, &mb))
        return fail(ctx, Q38_ERR_CUDA, "quantized_matmul: tensor map encoding failed");
    const cudaError_t e = launch_kernels<BITS, NT>(p, ctx->device, ctx->num_sms, x, M, K, mc, ms, mb, b != nullptr, N,
                                                   y, static_cast<uint8_t*>(ctx->workspace), part,
                                                   ctx->d_status, ctx->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_CUDA, "quantized_matmul: launch failed: %s", cudaGetErrorString(e));
    }
    return Q38_OK;
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

q38_status qgemv_fast(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w,
                      const void* s, const void* b, int64_t N, int bits, void* y) {
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    const bool two = M > 8;
    switch (bits) {
        case 2: return two ? launch<2, 2>(ctx, x, m, k, w, s, b, n, y) : launch<2, 1>(ctx, x, m, k, w, s, b, n, y);
        case 3: return two ? launch<3, 2>(ctx, x, m, k, w, s, b, n, y) : launch<3, 1>(ctx, x, m, k, w, s, b, n, y);
        case 4: return two ? launch<4, 2>(ctx, x, m, k, w, s, b, n, y) : launch<4, 1>(ctx, x, m, k, w, s, b, n, y);
        case 8: return two ? launch<8, 2>(ctx, x, m, k, w, s, b, n, y) : launch<8, 1>(ctx, x, m, k, w, s, b, n, y);
    }
    return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: bits %d not on the fast path", bits);
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
constexpr size_t NA_ACC_BYTES = static_cast<size_t>(NA_MAX_M) * NA_MAX_N * 4;          // 2 MiB
constexpr size_t NA_XF_BYTES = static_cast<size_t>(NA_MAX_K / KC) * NA_MAX_M * (256 * 8 + 64);  // 2.06 MiB
constexpr size_t NA_STATUS_OFF = 0;
constexpr size_t NA_ACC_OFF = 256;
constexpr size_t NA_XF_OFF = NA_ACC_OFF + NA_ACC_BYTES;
constexpr size_t NA_TOTAL = NA_XF_OFF + NA_XF_BYTES;

// The scratch of every no-alloc call on a device (status word, fp32 partial sums,
// activation fragments).  In host code this name is only a stand-in for
// the device array; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[NA_TOTAL];

std::mutex g_noalloc_mu;
uint8_t* g_noalloc_ptr[64] = {};

// Once per device, with that device current: resolve the array's device address.
q38_status noalloc_scratch(int device, uint8_t** out) {
    if (device < 0 || device >= 64) return Q38_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return Q38_ERR_CUDA;
        }
        g_noalloc_ptr[device] = static_cast<uint8_t*>(p);
    }
    *out = g_noalloc_ptr[device];
    return Q38_OK;
}

template <int BITS, int NT>
q38_status launch_noalloc(uint8_t* scratch, int device, int num_sms, const void* x, int M, int K,
                          const uint32_t* w, const void* s, const void* b, int N, void* y,
                          cudaStream_t stream) {
    Plan p;
    if (!make_plan<BITS>(M, K, N, p)) return Q38_ERR_UNSUPPORTED;
    uint32_t* status = reinterpret_cast<uint32_t*>(scratch + NA_STATUS_OFF);
    float* part = reinterpret_cast<float*>(scratch + NA_ACC_OFF);
    uint8_t* xfrag = scratch + NA_XF_OFF;
    // the partial sums must start at zero; a previous call leaves them zero, but clear
    // them anyway so an interrupted call cannot poison the next one
    if (cudaMemsetAsync(part, 0, static_cast<size_t>(M) * N * 4, stream) != cudaSuccess) {
        cudaGetLastError();
        return Q38_ERR_CUDA;
    }
    CUtensorMap mc, ms, mb;
    if (!make_maps<BITS>(w, s, b, K, N, &mc, &ms, &mb)) return Q38_ERR_CUDA;
    const cudaError_t e = launch_kernels<BITS, NT>(p, device, num_sms, x, M, K, mc, ms, mb, b != nullptr, N, y,
                                                   xfrag, part, status, stream);
    if (e != cudaSuccess) {
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
    const bool two = M > 8;
    switch (bits) {
        case 2: return two ? launch_noalloc<2, 2>(scratch, device, sms, x, m, k, w, scales, biases, n, y, s)
                           : launch_noalloc<2, 1>(scratch, device, sms, x, m, k, w, scales, biases, n, y, s);
        case 3: return two ? launch_noalloc<3, 2>(scratch, device, sms, x, m, k, w, scales, biases, n, y, s)
                           : launch_noalloc<3, 1>(scratch, device, sms, x, m, k, w, scales, biases, n, y, s);
        case 4: return two ? launch_noalloc<4, 2>(scratch, device, sms, x, m, k, w, scales, biases, n, y, s)
                           : launch_noalloc<4, 1>(scratch, device, sms, x, m, k, w, scales, biases, n, y, s);
        default: return two ? launch_noalloc<8, 2>(scratch, device, sms, x, m, k, w, scales, biases, n, y, s)
                            : launch_noalloc<8, 1>(scratch, device, sms, x, m, k, w, scales, biases, n, y, s);
    }
}
