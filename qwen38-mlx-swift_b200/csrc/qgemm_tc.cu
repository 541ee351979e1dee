// Prefill-shaped MLX-affine quantized product on the 5th-generation tensor cores:
// y[M,N] = x[M,K] . dequant(W)[N,K]^T for M > 16 tokens, group 64 or 32, K % 128 == 0,
// bits 2/3/4/8, bf16 activations and scales.  Replaces the Metal `qmm` kernel behind
// MLX.quantizedMM (QuantizedLinear.callAsFunction,
// Sources/Qwen38Core/FlashNext/Qwen4ExpPrequantized.swift:156-159) for prompt-sized inputs.
//
// CTA pairs (clusters of 2 on one SM pair), persistent over 256-row x 256-token output
// tiles.  The pair's MMA is tcgen05.mma.cta_group::2 with M = 256 weight rows (128 in
// each CTA's TMEM) and N = 256 tokens (128 staged in each CTA's shared memory), so every
// byte a CTA stages feeds twice the math of a single-CTA 128x128 tile.  Roles per CTA:
//   warp 0      activation producer: per 128-k stage, the CTA's 128 tokens of permuted
//               activations (two 128-byte-swizzled 64-element TMA boxes) into a 5-deep
//               ring, completion counted on the pair leader's barrier.
//   warp 1      allocates the pair's TMEM; in the leader, issues the pair MMAs (A = the
//               dequantized weights in TMEM, B = activations in shared memory, D in TMEM).
//   warp 2      weight producer: the CTA's 128 weight rows' packed codes (swizzled box)
//               into a separate ring, so the small weight stages run ahead of the large
//               activation stages.  Scales and biases (4 bytes per row and stage) are read
//               by the dequantizing threads themselves, one stage ahead, which keeps the
//               scale array's row stride free of TMA's 16-byte rule (K % 128 suffices).
//   warps 3-10  dequantize, two sets of four alternating stages: one thread per weight row
//               turns its 128 codes per stage into exact bf16 weights w = scale*q + bias
//               (magic-number extraction, bf16x2 subtract and fused multiply-add, one
//               rounding) and stores them into a TMEM operand slot with tcgen05.st -- the
//               weights never pass through shared memory.
//   warps 11-18 epilogue: two warps per TMEM lane quarter drain the finished accumulator
//               (128 rows x 256 tokens per CTA), convert to bf16 and store.
// The extraction yields codes in a fixed permuted order, some pre-multiplied by 2^p; the
// prologue kernel writes the activations permuted and scaled by 2^-p to match, so the
// products pair up exactly: sum_k' (2^p w_k)(2^-p x_k) = sum_k w_k x_k.
#include <algorithm>
#include <mutex>

#include "tc_pipeline.cuh"

namespace q38 {
namespace {

constexpr int P_ROWS = 128;    // weight rows per CTA (TMEM lanes); a pair covers 2 x 128 (MMA M)
constexpr int P_TOK = 256;     // tokens per pair tile (MMA N)
constexpr int P_HTOK = 128;    // tokens staged per CTA (its half of N)
constexpr int P_KS = 128;      // k per stage (2 groups)
constexpr int P_ASLOTS = 4;    // TMEM weight-operand slots, 64 columns each (columns 0-255)
constexpr uint32_t P_DCOL = 256;  // accumulator: columns 256-511, one per token of the tile
constexpr int P_DEQ_WARPS = 8;  // two sets of four (one warp per TMEM lane quarter), alternate stages
constexpr int P_EPI_WARPS = 8;  // two per TMEM lane quarter, one per half of the tile's tokens
constexpr int P_WARP_DEQ0 = 3, P_WARP_EPI0 = P_WARP_DEQ0 + P_DEQ_WARPS;
constexpr int P_THREADS = (P_WARP_EPI0 + P_EPI_WARPS) * 32;
constexpr uint32_t P_IDESC = idesc_bf16_f32(2 * P_ROWS, P_TOK);

// SB_TMA: scales/biases ride in the weight stage as {8 groups, 128 rows} TMA boxes (needs
// K % 512 == 0 for the 16-byte row stride of the scale arrays); otherwise the dequantizing
// threads read them from global memory one stage ahead.
template <int BITS, bool SB_TMA>
struct PF {
    static constexpr int CODE_W = CodeLayout<BITS>::CODE_W;  // code words per row per stage
    static constexpr int CODE_B = P_ROWS * CODE_W * 4;       // 4 / 6 / 8 KiB
    static constexpr int X_B = 2 * P_HTOK * 128;          // two 64-element 128-byte-swizzled boxes
    static constexpr int W_STAGE = (CODE_B + (SB_TMA ? 4096 : 0) + 1023) / 1024 * 1024;
    static constexpr int X_STAGES = BITS == 8 ? 4 : 5;  // 8-bit: room for four or more 16 KiB weight stages
    static constexpr int W_STAGES_MAX = (227 * 1024 - 2048 - X_STAGES * X_B) / W_STAGE;
    static constexpr int W_STAGES = W_STAGES_MAX > 8 ? 8 : W_STAGES_MAX;
    static constexpr int SMEM = 2048 + X_STAGES * X_B + W_STAGES * W_STAGE;
};

// Prologue: x' = activations permuted within each 64-group into extraction order and
// scaled by 2^-p, so that the dequantized weights pair with them in the MMA.
template <int BITS>
__global__ void __launch_bounds__(256) qgemm_prep(const __nv_bfloat16* __restrict__ x, int64_t M, int K,
                                                  __nv_bfloat16* __restrict__ xp) {
    griddep_wait();
    griddep_launch_dependents();
    const int G = K / 64;
    const int64_t item = blockIdx.x * 256LL + threadIdx.x;  // (token, group)
    if (item >= M * G) return;
    const int64_t m = item / G;
    const int g = static_cast<int>(item % G);
    permute_group<BITS>(x + m * K + g * 64, xp + m * K + g * 64);
}

// Prologue with the Hadamard rotation of Qwen38HadamardQuantizedLinear
// (Sources/Qwen38Core/Bonsai2/Qwen38HadamardModules.swift:10-19, 37-39): one warp per
// (token, window of W = 32 * EPL activations, W = max(256, block)); lane l holds elements
// [l * EPL, l * EPL + EPL).  Signs first, the butterfly stages h = 1, 2, 4, ... < block
// (lower a + b, upper a - b, in the order of the rotation kernel, so the values are the same
// bit for bit), 1/sqrt(block), rounding to bf16; then each 64-group of the window is
// permuted and 2^-p-scaled into x' as qgemm_prep does.
template <int BITS, int EPL>
__global__ void __launch_bounds__(128) qgemm_prep_rot(const __nv_bfloat16* __restrict__ x, int64_t M, int K,
                                                      const float* __restrict__ signs, int block, float scale,
                                                      __nv_bfloat16* __restrict__ xp) {
    griddep_wait();
    griddep_launch_dependents();
    constexpr int W = 32 * EPL;
    __shared__ __align__(16) __nv_bfloat16 s_rot[4][W];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwin = K / W;
    const int64_t item = blockIdx.x * 4LL + warp;  // (token, window)
    if (item >= M * nwin) return;
    const int64_t m = item / nwin;
    const int j = static_cast<int>(item % nwin);
    const __nv_bfloat16* src = x + m * K + static_cast<int64_t>(j) * W + lane * EPL;
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL / 8; ++i) {
        const uint4 u = reinterpret_cast<const uint4*>(src)[i];
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            v[8 * i + 2 * t] = bf16_bits_to_f32(q[t] & 0xFFFFu);
            v[8 * i + 2 * t + 1] = bf16_bits_to_f32(q[t] >> 16);
        }
    }
    if (signs) {
        const float* sg = signs + static_cast<int64_t>(j) * W + lane * EPL;
#pragma unroll
        for (int i = 0; i < EPL; ++i) v[i] = v[i] * sg[i];
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
    uint32_t* o = reinterpret_cast<uint32_t*>(&s_rot[warp][lane * EPL]);
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) o[i] = pack_bf16x2(v[2 * i] * scale, v[2 * i + 1] * scale);
    __syncwarp();
    for (int g = lane; g < W / 64; g += 32)
        permute_group<BITS>(&s_rot[warp][g * 64], xp + m * K + static_cast<int64_t>(j) * W + g * 64);
}

struct PArgs {
    const uint16_t* scales;  // [N, K/64] bf16 bits, or with `pack` [N, K/128] f16 bits
    const uint16_t* biases;  // same, or null
    __nv_bfloat16* y;
    uint32_t* status;
    int M, N, K, nR, ntiles, has_bias;
    int pack;  // f16 scales and biases in groups of 128 (direct scale loads only)
};

template <int BITS, bool SB_TMA, bool G32 = false>
__global__ void __launch_bounds__(P_THREADS, 1) qgemm_tc(const __grid_constant__ CUtensorMap map_x,
                                                        const __grid_constant__ CUtensorMap map_codes,
                                                        const __grid_constant__ CUtensorMap map_scales,
                                                        const __grid_constant__ CUtensorMap map_biases,
                                                        const PArgs a) {
    using F = PF<BITS, SB_TMA>;
    constexpr int SX = F::X_STAGES, SW = F::W_STAGES;
    static_assert(SW <= 8, "2 * SW landing barriers are laid out");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint64_t* x_full = reinterpret_cast<uint64_t*>(smem);  // both CTAs' activation halves landed (leader)
    uint64_t* x_empty = x_full + 8;                        // pair MMAs reading the slot done (local)
    uint64_t* w_full = x_empty + 8;                        // codes + scales landed (local), 2 * SW
    uint64_t* w_empty = w_full + 16;                        // dequant warps done reading (local)
    uint64_t* a_full = w_empty + 8;                        // both CTAs' weight slots written (leader)
    uint64_t* a_free = a_full + P_ASLOTS;                  // pair MMAs reading the slot done (local)
    uint64_t* d_full = a_free + P_ASLOTS;                  // tile accumulated (local)
    uint64_t* d_free = d_full + 1;                         // both CTAs' accumulators drained (leader)
    uint64_t* final_bar = d_free + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* xring = smem + 1024;
    uint8_t* wring = xring + SX * F::X_B;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int ksteps = a.K / P_KS;
    const int my_tiles = pair < a.ntiles ? (a.ntiles - 1 - pair) / npairs + 1 : 0;
    const int total = my_tiles * ksteps;  // stages this pair runs
    if (threadIdx.x == 0) {
        for (int i = 0; i < SX; ++i) {
            mbar_init(&x_full[i], 1);
            mbar_init(&x_empty[i], 1);
        }
        for (int i = 0; i < SW; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_full[SW + i], 1);
            mbar_init(&w_empty[i], 4);
        }
        for (int i = 0; i < P_ASLOTS; ++i) {
            mbar_init(&a_full[i], 8);  // 4 dequant warps in each CTA
            mbar_init(&a_free[i], 1);
        }
        mbar_init(d_full, 1);
        mbar_init(d_free, 2 * P_EPI_WARPS);
        mbar_init(final_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    griddep_launch_dependents();
    const uint32_t tmem = *tmem_slot;
    const Abort ab{abort_flag, mapa_shared(const_cast<int*>(abort_flag), rank ^ 1u), a.status, true};

    if (warp == 0) {
        // ------------------------------------------------------- activation producer
        if (lane == 0) {
            prefetch_tensormap(&map_x);
            griddep_wait();  // the permuted activations come from the prologue kernel
            int gs = 0;
            for (; gs < total && !*abort_flag; ++gs) {
                const int slot = gs % SX, tile = pair + (gs / ksteps) * npairs, ks = gs % ksteps;
                if (gs >= SX && !p_wait<false>(&x_empty[slot], ((gs / SX) - 1) & 1, ab)) break;
                const int m0 = (tile / a.nR) * P_TOK + rank * P_HTOK, k0 = ks * P_KS;
                uint8_t* st = xring + slot * F::X_B;
                if (leader) mbar_arrive_expect_tx(&x_full[slot], 2 * F::X_B);
                const uint32_t xbar = mapa_shared(&x_full[slot], 0);
                tma_load_2d_pair(st, &map_x, xbar, k0, m0);
                tma_load_2d_pair(st + P_HTOK * 128, &map_x, xbar, k0 + 64, m0);
            }
            // No copy may still be landing when the CTA exits (matters only after an abort:
            // otherwise the MMAs have consumed every fill).
            if (leader)
                for (int i = 1; i <= (gs < SX ? gs : SX); ++i)
                    mbar_wait(&x_full[(gs - i) % SX], ((gs - i) / SX) & 1, a.status);
        }
    } else if (warp == 2) {
        // ----------------------------------------------------------- weight producer
        if (lane == 0) {
            prefetch_tensormap(&map_codes);
            if (SB_TMA) {
                prefetch_tensormap(&map_scales);
                if (a.has_bias) prefetch_tensormap(&map_biases);
            }
            const uint32_t wbytes = F::CODE_B + (SB_TMA ? 2048u * (a.has_bias ? 2u : 1u) : 0u);
            int gs = 0;
            for (; gs < total && !*abort_flag; ++gs) {
                const int slot = gs % SW, tile = pair + (gs / ksteps) * npairs, ks = gs % ksteps;
                if (gs >= SW && !p_wait<false>(&w_empty[slot], ((gs / SW) - 1) & 1, ab)) break;
                const int n0 = (tile % a.nR) * (2 * P_ROWS) + rank * P_ROWS, k0 = ks * P_KS;
                uint8_t* st = wring + slot * F::W_STAGE;
                uint64_t* wl = &w_full[gs % (2 * SW)];
                mbar_arrive_expect_tx(wl, wbytes);
                tma_load_2d(st, &map_codes, wl, k0 * BITS / 32, n0);
                if (SB_TMA) {
                    tma_load_2d(st + F::CODE_B, &map_scales, wl, (k0 / 512) * 8, n0);
                    if (a.has_bias)
                        tma_load_2d(st + F::CODE_B + 2048, &map_biases, wl, (k0 / 512) * 8, n0);
                }
            }
            for (int i = 1; i <= (gs < SW ? gs : SW); ++i)
                mbar_wait(&w_full[(gs - i) % (2 * SW)], ((gs - i) / (2 * SW)) & 1, a.status);
        }
    } else if (warp == 1) {
        // -------------------------------------------------- pair MMA issuer (leader)
        if (leader && lane == 0) {
            int gs = 0;
            bool ok = true;
            for (int tc = 0; tc < my_tiles && ok && !*abort_flag; ++tc) {
                if (tc >= 1 && !p_wait<true>(d_free, (tc - 1) & 1, ab)) break;
                tc_fence_after();
                for (int ks = 0; ks < ksteps; ++ks, ++gs) {
                    const int xs = gs % SX, as = gs % P_ASLOTS;
                    if (!p_wait<false>(&x_full[xs], (gs / SX) & 1, ab) ||
                        !p_wait<true>(&a_full[as], (gs / P_ASLOTS) & 1, ab)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xa = smem_u32(xring + xs * F::X_B);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t bd = smem_desc(xa + (kk >> 2) * (P_HTOK * 128) + (kk & 3) * 32, 16, 1024, 2);
                        tc_mma_ts_pair(tmem + P_DCOL, tmem + as * 64 + kk * 8, bd, P_IDESC,
                                       (ks > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit_pair(&x_empty[xs], 3);
                    tc_commit_pair(&a_free[as], 3);
                }
                if (ok) tc_commit_pair(d_full, 3);
            }
            // every MMA (and its TMEM reads) has finished before the teardown frees TMEM
            tc_commit_pair(final_bar, 1);
            mbar_wait(final_bar, 0, a.status);
        }
    } else if (warp < P_WARP_EPI0) {
        // ----------------------------------------------------------------- dequant
        // Stage gs lands on w_full[gs % (2 * SW)].  A parity wait only tells neighbouring
        // phases apart; with one landing barrier per slot and an odd ring a slot alternates
        // between the two sets, and a set could pass the wait of a slot's next stage while
        // the other set's stage in that slot was still landing.  With the even period each
        // landing barrier serves one set, which has waited for its previous phase itself.
        // Set 0 dequantizes the even stages, set 1 the odd ones; within a set, one warp
        // per TMEM lane quarter, one thread per weight row.
        const int set = (warp - P_WARP_DEQ0) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t a_full_leader = mapa_shared(a_full, 0);
        // Scales and biases of the two groups of a stage come straight from global memory
        // (4 bytes each per row), loaded one stage of this set ahead.
        const int G = a.K / (G32 ? 32 : 64);
        // sv/bv: the stage's two 64-code groups' scale and bias words (G32: each word the
        // two 32-groups' values)
        auto sb_load = [&](int g, uint2& sv, uint2& bv) {
            sv = make_uint2(0u, 0u);
            bv = make_uint2(0u, 0u);
            if (SB_TMA || g >= total) return;
            const int tile = pair + (g / ksteps) * npairs;
            const int n = (tile % a.nR) * (2 * P_ROWS) + rank * P_ROWS + row;
            if (n >= a.N) return;
            if (a.pack) {
                // one 128-group per 128-k stage: its f16 scale and bias as bf16 for both
                // 64-halves (the dequantized weight is rounded to bf16 in any case)
                const size_t off = static_cast<size_t>(n) * (a.K / 128) + (g % ksteps);
                auto cvt = [](uint16_t h) {
                    const uint32_t v = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(__ushort_as_half(h))));
                    return v | (v << 16);
                };
                const uint32_t sw = cvt(__ldg(a.scales + off)), bw = a.biases ? cvt(__ldg(a.biases + off)) : 0u;
                sv = make_uint2(sw & 0xFFFFu, sw >> 16);
                bv = make_uint2(bw & 0xFFFFu, bw >> 16);
                return;
            }
            if constexpr (G32) {
                const size_t off = static_cast<size_t>(n) * G + 4 * (g % ksteps);
                sv = __ldg(reinterpret_cast<const uint2*>(a.scales + off));
                if (a.biases) bv = __ldg(reinterpret_cast<const uint2*>(a.biases + off));
            } else {
                const size_t off = static_cast<size_t>(n) * G + 2 * (g % ksteps);
                const uint32_t sw = __ldg(reinterpret_cast<const unsigned int*>(a.scales + off));
                const uint32_t bw = a.biases ? __ldg(reinterpret_cast<const unsigned int*>(a.biases + off)) : 0u;
                sv = make_uint2(sw & 0xFFFFu, sw >> 16);
                bv = make_uint2(bw & 0xFFFFu, bw >> 16);
            }
        };
        uint2 s_next, b_next;
        sb_load(set, s_next, b_next);
        for (int gs = set; gs < total; gs += 2) {
            const int slot = gs % SW, as = gs % P_ASLOTS;
            uint2 s01 = s_next, b01 = b_next;
            sb_load(gs + 2, s_next, b_next);
            if (!p_wait_warp<false>(&w_full[gs % (2 * SW)], (gs / (2 * SW)) & 1, ab)) break;
            // Dequantize into registers first: the TMEM slot is waited for only afterwards,
            // so the arithmetic overlaps the MMAs that still read the slot.
            const uint8_t* st = wring + slot * F::W_STAGE;
            if (SB_TMA) {
                const uint32_t* sb = reinterpret_cast<const uint32_t*>(st + F::CODE_B);
                const int ks = gs % ksteps;
                const uint32_t sw = sb[row * 4 + (ks & 3)];
                const uint32_t bw = a.has_bias ? sb[512 + row * 4 + (ks & 3)] : 0u;
                s01 = make_uint2(sw & 0xFFFFu, sw >> 16);
                b01 = make_uint2(bw & 0xFFFFu, bw >> 16);
            }
            uint32_t av0[32], av1[32];
            dequant_group<BITS, G32>(st, row, 0, s01.x, b01.x, av0);
            dequant_group<BITS, G32>(st, row, 1, s01.y, b01.y, av1);
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_empty[slot]);  // codes read; the slot may refill
            if (gs >= P_ASLOTS && !p_wait_warp<false>(&a_free[as], ((gs / P_ASLOTS) - 1) & 1, ab)) break;
            tc_fence_after();
            tmem_st32(tmem + lane_off + as * 64, av0);
            tmem_st32(tmem + lane_off + as * 64 + 32, av1);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(a_full_leader + as * 8);
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int quarter = warp & 3, half = (warp - P_WARP_EPI0) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t d_free_leader = mapa_shared(d_free, 0);
        for (int tc = 0; tc < my_tiles; ++tc) {
            if (!p_wait_warp<false>(d_full, tc & 1, ab)) break;
            tc_fence_after();
            const int tile = pair + tc * npairs;
            const int n = (tile % a.nR) * (2 * P_ROWS) + rank * P_ROWS + row;
            const int m0 = (tile / a.nR) * P_TOK + half * (P_TOK / 2);
#pragma unroll 1
            for (int ch = 0; ch < P_TOK / 64; ++ch) {
                float v[32];
                tmem_ld32(tmem + lane_off + P_DCOL + half * (P_TOK / 2) + ch * 32, v);
                const int mc = m0 + ch * 32;
                const int mlim = n < a.N ? min(32, a.M - mc) : 0;
                __nv_bfloat16* out = a.y + static_cast<size_t>(mc) * a.N + n;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if (i < mlim) *out = __float2bfloat16_rn(v[i]);
                    out += a.N;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(d_free_leader);
        }
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, 512);
}

struct PairLaunch {
    int smem = 0;
    int max_pairs = 0;
};

template <int BITS, bool SB_TMA, bool G32>
q38_status pair_config(q38_ctx* ctx, int smem, PairLaunch* out) {
    static std::mutex mu;
    static PairLaunch cached[64];
    std::lock_guard<std::mutex> lk(mu);
    const int dev = ctx->device;
    if (dev < 64 && cached[dev].max_pairs > 0) {
        *out = cached[dev];
        return Q38_OK;
    }
    auto kmain = qgemm_tc<BITS, SB_TMA, G32>;
    if (cudaFuncSetAttribute(kmain, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return check_launch(ctx, "cudaFuncSetAttribute");
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (ctx->num_sms / 2));
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kmain, &cfg) != cudaSuccess)
        return check_launch(ctx, "cudaOccupancyMaxActiveClusters");
    if (clusters < 1) return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: no CTA pair fits on this device");
    PairLaunch pl;
    pl.smem = smem;
    pl.max_pairs = clusters;
    if (dev < 64) cached[dev] = pl;
    *out = pl;
    return Q38_OK;
}

template <int BITS, bool SB_TMA, bool G32 = false>
q38_status launch(q38_ctx* ctx, const void* x, int M, int K, const uint32_t* w, const void* s, const void* b,
                  int N, void* y, bool pack = false, const float* signs = nullptr, int rot_block = 0) {
    using F = PF<BITS, SB_TMA>;
    q38_status st = ensure_workspace(ctx, static_cast<size_t>(M) * K * 2);
    if (st != Q38_OK) return st;
    __nv_bfloat16* xp = static_cast<__nv_bfloat16*>(ctx->workspace);

    CUtensorMap mx, mc, ms = {}, mb = {};
    const CUtensorMapSwizzle cswz = code_swizzle<BITS>();
    if (!make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xp, K, M, 64, P_HTOK, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&mc, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w, static_cast<uint64_t>(K) * BITS / 32, N,
                     F::CODE_W, P_ROWS, cswz) ||
        (SB_TMA && (!make_map_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s, K / 64, N, 8, P_ROWS,
                                 CU_TENSOR_MAP_SWIZZLE_NONE) ||
                    !make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b ? b : s, K / 64, N, 8, P_ROWS,
                                 CU_TENSOR_MAP_SWIZZLE_NONE))))
        return fail(ctx, Q38_ERR_CUDA, "quantized_matmul: tensor map encoding failed");

    static_assert(F::W_STAGES >= 4 && F::SMEM <= 227 * 1024, "prefill stages do not fit");
    PairLaunch pl;
    if ((st = pair_config<BITS, SB_TMA, G32>(ctx, F::SMEM, &pl)) != Q38_OK) return st;

    const int nR = (N + 2 * P_ROWS - 1) / (2 * P_ROWS), nT = (M + P_TOK - 1) / P_TOK;
    const int ntiles = nR * nT;
    const int pairs = ntiles < pl.max_pairs ? ntiles : pl.max_pairs;

    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t pcfg = {};
    pcfg.stream = ctx->stream;
    pcfg.attrs = attr;
    pcfg.numAttrs = 1;
    if (rot_block > 0) {
        // x rotated in the prologue; windows of max(256, block) activations, one warp each
        const int win = rot_block > 256 ? rot_block : 256;
        const long long warps = static_cast<long long>(M) * (K / win);
        pcfg.gridDim = dim3(static_cast<unsigned>((warps + 3) / 4));
        pcfg.blockDim = dim3(128);
        const float sc = 1.0f / sqrtf(static_cast<float>(rot_block));
        const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
        cudaError_t e;
        if (win == 256)
            e = cudaLaunchKernelEx(&pcfg, qgemm_prep_rot<BITS, 8>, xb, static_cast<int64_t>(M), K, signs, rot_block, sc,
                                   xp);
        else if (win == 512)
            e = cudaLaunchKernelEx(&pcfg, qgemm_prep_rot<BITS, 16>, xb, static_cast<int64_t>(M), K, signs, rot_block,
                                   sc, xp);
        else
            e = cudaLaunchKernelEx(&pcfg, qgemm_prep_rot<BITS, 32>, xb, static_cast<int64_t>(M), K, signs, rot_block,
                                   sc, xp);
        if (e != cudaSuccess) return check_launch(ctx, "qgemm_prep_rot");
    } else {
        const long long items = static_cast<long long>(M) * (K / 64);
        pcfg.gridDim = dim3(static_cast<unsigned>((items + 255) / 256));
        pcfg.blockDim = dim3(256);
        if (cudaLaunchKernelEx(&pcfg, qgemm_prep<BITS>, static_cast<const __nv_bfloat16*>(x), static_cast<int64_t>(M),
                               K, xp) != cudaSuccess)
            return check_launch(ctx, "qgemm_prep");
    }

    PArgs args;
    args.scales = static_cast<const uint16_t*>(s);
    args.biases = static_cast<const uint16_t*>(b);
    args.y = static_cast<__nv_bfloat16*>(y);
    args.status = ctx->d_status;
    args.M = M;
    args.N = N;
    args.K = K;
    args.nR = nR;
    args.ntiles = ntiles;
    args.has_bias = b != nullptr;
    args.pack = pack ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, qgemm_tc<BITS, SB_TMA, G32>, mx, mc, ms, mb, args) != cudaSuccess)
        return check_launch(ctx, "qgemm_tc");
    return check_launch(ctx, "qgemm_tc");
}

}  // namespace

bool qgemm_tc_supported(int64_t M, int64_t K, int group, int bits, q38_dtype xd, q38_dtype sd, const void* x,
                        const void* w, const void* s, const void* b, const void* y) {
    if (M < 17 || M > (1 << 24) || K % 128 != 0 || K <= 0 || K > (1 << 20)) return false;
    if (bits != 2 && bits != 3 && bits != 4 && bits != 8) return false;
    if (xd != Q38_BF16) return false;
    // groups of 64 or 32 with bf16 scales, or the Bonsai 2 pack's group 128 with f16 scales
    // (2 and 4 bits)
    const bool std_layout = (group == 64 || group == 32) && sd == Q38_BF16;
    const bool pack_layout = group == 128 && sd == Q38_F16 && (bits == 2 || bits == 4);
    if (!std_layout && !pack_layout) return false;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return al(x) && al(w) && al(s) && (!b || al(b)) && al(y);
}

q38_status qgemm_tc_run(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w, const void* s,
                        const void* b, int64_t N, int bits, void* y, int group, const float* signs, int rot_block) {
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    const float* sg = signs;
    const int rb = rot_block;
    if (group == 128) {  // the pack layout: scales loaded directly by the dequantizing warps
        if (bits == 2) return launch<2, false>(ctx, x, m, k, w, s, b, n, y, true, sg, rb);
        return launch<4, false>(ctx, x, m, k, w, s, b, n, y, true, sg, rb);
    }
    if (group == 32) {  // scales and biases read by the dequantizing warps, 4 groups per stage
        switch (bits) {
            case 2: return launch<2, false, true>(ctx, x, m, k, w, s, b, n, y, false, sg, rb);
            case 3: return launch<3, false, true>(ctx, x, m, k, w, s, b, n, y, false, sg, rb);
            case 8: return launch<8, false, true>(ctx, x, m, k, w, s, b, n, y, false, sg, rb);
            default: return launch<4, false, true>(ctx, x, m, k, w, s, b, n, y, false, sg, rb);
        }
    }
    const bool tma_scales = k % 512 == 0;
    switch (bits) {
        case 2: return tma_scales ? launch<2, true>(ctx, x, m, k, w, s, b, n, y, false, sg, rb) : launch<2, false>(ctx, x, m, k, w, s, b, n, y, false, sg, rb);
        case 3: return tma_scales ? launch<3, true>(ctx, x, m, k, w, s, b, n, y, false, sg, rb) : launch<3, false>(ctx, x, m, k, w, s, b, n, y, false, sg, rb);
        case 8: return tma_scales ? launch<8, true>(ctx, x, m, k, w, s, b, n, y, false, sg, rb) : launch<8, false>(ctx, x, m, k, w, s, b, n, y, false, sg, rb);
        default: return tma_scales ? launch<4, true>(ctx, x, m, k, w, s, b, n, y, false, sg, rb) : launch<4, false>(ctx, x, m, k, w, s, b, n, y, false, sg, rb);
    }
}

}  // namespace q38
