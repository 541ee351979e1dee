// Grouped MLX-affine quantized products of the SwitchGLU expert stack on tcgen05:
// the work of MLX.gatherQuantizedMM behind QuantizedSwitchLinear
// (Vendor/mlx-swift-lm-local.patch:184-218) for the gate, up and down projections of
// SwitchGLU (used at Sources/Qwen38Core/FlashNext/Qwen4ExpSparseMoE.swift:294), with the
// (token, slot) pairs sorted by expert so that each expert's weights are read once per
// run of up to 128 pairs.
//
// A tile is (expert e, block of weight rows, run of <= 128 consecutive sorted pairs of e).
// One CTA per SM, persistent over a device-built tile list.  The MMA is
// tcgen05.mma.cta_group::1 with M = 128 weight rows (A: dequantized weights in TMEM),
// N = the run's pairs rounded up to 16 (B: permuted activations in shared memory), and
// a double-buffered fp32 accumulator in TMEM.  Two modes:
//   GATE_UP  rows 0-63 of a tile are gate rows i0..i0+63 of expert e, rows 64-127 the
//            same up rows; the epilogue forms h = bf16(silu(bf16 g) * bf16 u) and writes
//            it, permuted and 2^-p-scaled for the down projection's extraction order, to
//            h'[pair, I] -- the gate, up and SiLU-gate of a pair never leave the chip
//            separately.
//   DOWN     rows are 128 rows of expert e's down projection; y[pair, H] = bf16(h . Wd^T).
// Warp roles as in the dense prefill kernel: activation producer, MMA issuer, weight
// producer, eight dequantizing warps (two alternating sets), four epilogue warps.
#include <algorithm>
#include <mutex>

#include "moe_internal.h"
#include "tc_pipeline.cuh"

namespace q38 {
namespace {

constexpr int G_ROWS = 128;
constexpr int G_TOK = 128;
constexpr int G_KS = 128;
constexpr int G_ASLOTS = 4;
constexpr uint32_t G_DCOL = 256;
constexpr int G_WARP_DEQ0 = 3, G_WARP_EPI0 = 11, G_EPI_WARPS = 4;
constexpr int G_THREADS = (G_WARP_EPI0 + G_EPI_WARPS) * 32;
constexpr int G_XBOX = 32;  // activation rows per TMA box

// XR: activation rows (pairs) staged per k-step, the longest run a tile may have.  Short
// runs (few tokens per expert) get proportionally deeper activation rings for the same
// 128 KiB, so the ring covers the TMA round trip.
template <int BITS, int XR>
struct GF {
    static constexpr int CODE_W = CodeLayout<BITS>::CODE_W;
    static constexpr int CODE_B = G_ROWS * CODE_W * 4;
    static constexpr int X_B = 2 * XR * 128;
    static constexpr int W_STAGE = (CODE_B + 4096 + 1023) / 1024 * 1024;
    static constexpr int X_STAGES = (128 * 1024 / X_B) > 16 ? 16 : (128 * 1024 / X_B);
    static constexpr int EX_B = 32 * 64 * 2;  // up values of one 32-pair chunk (gate/up mode)
    static constexpr int W_MAX = (227 * 1024 - 2048 - X_STAGES * X_B - EX_B) / W_STAGE;
    static constexpr int W_STAGES = W_MAX > 8 ? 8 : W_MAX;
    static constexpr int SMEM = 2048 + X_STAGES * X_B + EX_B + W_STAGES * W_STAGE;
};

struct GArgs {
    const MoeTile* tiles;
    const int* ntiles;
    __nv_bfloat16* out;
    uint32_t* status;
    int K;               // reduction length (H for gate/up, I for down)
    int rows_per_expert; // I (gate/up) or H (down)
    int out_ld;          // I (gate/up) or H (down)
    int has_bias;
};

__device__ __forceinline__ void named_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int BITS, bool GATE_UP, int XR>
__global__ void __launch_bounds__(G_THREADS, 1) qgemm_grouped(
    const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_c0,
    const __grid_constant__ CUtensorMap map_c1, const __grid_constant__ CUtensorMap map_s0,
    const __grid_constant__ CUtensorMap map_s1, const __grid_constant__ CUtensorMap map_b0,
    const __grid_constant__ CUtensorMap map_b1, const GArgs a) {
    using F = GF<BITS, XR>;
    constexpr int SX = F::X_STAGES, SW = F::W_STAGES;
    static_assert(SW <= 8, "2 * SW landing barriers are laid out");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint64_t* x_full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* x_empty = x_full + 16;
    uint64_t* w_full = x_empty + 16;  // landing barriers, 2 * SW
    uint64_t* w_empty = w_full + 16;
    uint64_t* a_full = w_empty + 8;
    uint64_t* a_free = a_full + G_ASLOTS;
    uint64_t* d_full = a_free + G_ASLOTS;  // 2 accumulators
    uint64_t* d_free = d_full + 2;
    uint64_t* final_bar = d_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* xring = smem + 1024;
    uint16_t* ex = reinterpret_cast<uint16_t*>(xring + SX * F::X_B);
    uint8_t* wring = xring + SX * F::X_B + F::EX_B;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ksteps = a.K / G_KS;
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
        for (int i = 0; i < G_ASLOTS; ++i) {
            mbar_init(&a_full[i], 4);
            mbar_init(&a_free[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&d_full[i], 1);
            mbar_init(&d_free[i], G_EPI_WARPS);
        }
        mbar_init(final_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_wait();  // tile list, activations and indices come from earlier kernels
    griddep_launch_dependents();
    const uint32_t tmem = *tmem_slot;
    const Abort ab{abort_flag, 0u, a.status, false};
    const int ntiles = *a.ntiles;
    const int my_tiles = static_cast<int>(blockIdx.x) < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int total = my_tiles * ksteps;
    auto tile_of = [&](int tc) { return a.tiles[blockIdx.x + tc * gridDim.x]; };

    if (warp == 0) {
        // ------------------------------------------------------- activation producer
        if (lane == 0) {
            prefetch_tensormap(&map_x);
            int gs = 0;
            for (int tc = 0; tc < my_tiles && !*abort_flag; ++tc) {
                const MoeTile t = tile_of(tc);
                const int nb = (t.np + G_XBOX - 1) / G_XBOX;
                bool ok = true;
                for (int ks = 0; ks < ksteps; ++ks, ++gs) {
                    const int slot = gs % SX;
                    if (gs >= SX && !p_wait<false>(&x_empty[slot], ((gs / SX) - 1) & 1, ab)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = xring + slot * F::X_B;
                    mbar_arrive_expect_tx(&x_full[slot], static_cast<uint32_t>(nb) * 2 * G_XBOX * 128);
                    for (int b = 0; b < nb; ++b)
                        for (int kh = 0; kh < 2; ++kh)
                            tma_load_2d(st + kh * (XR * 128) + b * (G_XBOX * 128), &map_x, &x_full[slot],
                                        ks * G_KS + kh * 64, t.p0 + b * G_XBOX);
                }
                if (!ok) break;
            }
            for (int i = 1; i <= (gs < SX ? gs : SX); ++i)
                mbar_wait(&x_full[(gs - i) % SX], ((gs - i) / SX) & 1, a.status);
        }
    } else if (warp == 2) {
        // ----------------------------------------------------------- weight producer
        if (lane == 0) {
            prefetch_tensormap(&map_c0);
            prefetch_tensormap(&map_c1);
            prefetch_tensormap(&map_s0);
            prefetch_tensormap(&map_s1);
            if (a.has_bias) {
                prefetch_tensormap(&map_b0);
                prefetch_tensormap(&map_b1);
            }
            const uint32_t wbytes = F::CODE_B + (a.has_bias ? 4096u : 2048u);
            int gs = 0;
            for (; gs < total && !*abort_flag; ++gs) {
                const int slot = gs % SW, ks = gs % ksteps;
                if (gs >= SW && !p_wait<false>(&w_empty[slot], ((gs / SW) - 1) & 1, ab)) break;
                const MoeTile t = tile_of(gs / ksteps);
                // gate/up: 64 gate rows then the same 64 up rows; down: 128 consecutive rows
                const int r0 = t.e * a.rows_per_expert + t.rb * (GATE_UP ? 64 : 128);
                const int r1 = GATE_UP ? r0 : r0 + 64;
                uint8_t* st = wring + slot * F::W_STAGE;
                const int k0 = ks * G_KS;
                uint64_t* wl = &w_full[gs % (2 * SW)];
                mbar_arrive_expect_tx(wl, wbytes);
                tma_load_2d(st, &map_c0, wl, k0 * BITS / 32, r0);
                tma_load_2d(st + F::CODE_B / 2, &map_c1, wl, k0 * BITS / 32, r1);
                tma_load_2d(st + F::CODE_B, &map_s0, wl, (k0 / 512) * 8, r0);
                tma_load_2d(st + F::CODE_B + 1024, &map_s1, wl, (k0 / 512) * 8, r1);
                if (a.has_bias) {
                    tma_load_2d(st + F::CODE_B + 2048, &map_b0, wl, (k0 / 512) * 8, r0);
                    tma_load_2d(st + F::CODE_B + 3072, &map_b1, wl, (k0 / 512) * 8, r1);
                }
            }
            for (int i = 1; i <= (gs < SW ? gs : SW); ++i)
                mbar_wait(&w_full[(gs - i) % (2 * SW)], ((gs - i) / (2 * SW)) & 1, a.status);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int gs = 0;
            bool ok = true;
            for (int tc = 0; tc < my_tiles && ok && !*abort_flag; ++tc) {
                const MoeTile t = tile_of(tc);
                const int n_mma = (t.np + 15) & ~15;
                const uint32_t idesc = idesc_bf16_f32(G_ROWS, n_mma);
                const int db = tc & 1;
                if (tc >= 2 && !p_wait<false>(&d_free[db], ((tc >> 1) - 1) & 1, ab)) break;
                tc_fence_after();
                for (int ks = 0; ks < ksteps; ++ks, ++gs) {
                    const int xs = gs % SX, as = gs % G_ASLOTS;
                    if (!p_wait<false>(&x_full[xs], (gs / SX) & 1, ab) ||
                        !p_wait<false>(&a_full[as], (gs / G_ASLOTS) & 1, ab)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xa = smem_u32(xring + xs * F::X_B);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t bd = smem_desc(xa + (kk >> 2) * (XR * 128) + (kk & 3) * 32, 16, 1024, 2);
                        tc_mma_ts(tmem + G_DCOL + db * G_TOK, tmem + as * 64 + kk * 8, bd, idesc,
                                  (ks > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(&x_empty[xs]);
                    tc_commit(&a_free[as]);
                }
                if (ok) tc_commit(&d_full[db]);
            }
            tc_commit(final_bar);
            mbar_wait(final_bar, 0, a.status);
        }
    } else if (warp < G_WARP_EPI0) {
        // ------------------------------------------------------------------- dequant
        // Set 0 dequantizes the even stages, set 1 the odd ones.
        // Stage gs lands on w_full[gs % (2 * SW)].  A parity wait only tells neighbouring
        // phases apart; with one landing barrier per slot and an odd ring a slot alternates
        // between the two sets, and a set could pass the wait of a slot's next stage while
        // the other set's stage in that slot was still landing.  With the even period each
        // landing barrier serves one set, which has waited for its previous phase itself.
        const int set = (warp - G_WARP_DEQ0) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        for (int gs = set; gs < total; gs += 2) {
            const int slot = gs % SW, as = gs % G_ASLOTS, ks = gs % ksteps;
            if (!p_wait_warp<false>(&w_full[gs % (2 * SW)], (gs / (2 * SW)) & 1, ab)) break;
            const uint8_t* st = wring + slot * F::W_STAGE;
            const uint32_t* sb = reinterpret_cast<const uint32_t*>(st + F::CODE_B);
            const uint32_t s01 = sb[row * 4 + (ks & 3)];
            const uint32_t b01 = a.has_bias ? sb[512 + row * 4 + (ks & 3)] : 0u;
            uint32_t av0[32], av1[32];
            dequant_group<BITS>(st, row, 0, s01 & 0xFFFFu, b01 & 0xFFFFu, av0);
            dequant_group<BITS>(st, row, 1, s01 >> 16, b01 >> 16, av1);
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_empty[slot]);
            if (gs >= G_ASLOTS && !p_wait_warp<false>(&a_free[as], ((gs / G_ASLOTS) - 1) & 1, ab)) break;
            tc_fence_after();
            tmem_st32(tmem + lane_off + as * 64, av0);
            tmem_st32(tmem + lane_off + as * 64 + 32, av1);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[as]);
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int quarter = warp & 3;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        for (int tc = 0; tc < my_tiles; ++tc) {
            const int db = tc & 1;
            if (!p_wait_warp<false>(&d_full[db], (tc >> 1) & 1, ab)) break;
            tc_fence_after();
            const MoeTile t = tile_of(tc);
            const uint32_t dcol = tmem + lane_off + G_DCOL + db * G_TOK;
            const int nch = (t.np + 31) >> 5;
            if constexpr (GATE_UP) {
                // quarters 2,3 hold up rows: hand them to the gate quarters through shared memory
                const int i = t.rb * 64 + (quarter & 1) * 32 + lane;  // gate/up row within the expert
                const int g64 = i & ~63, c = i & 15, tq = (i & 63) >> 4;
                const int pos = g64 + 16 * tq + window_slot<BITS>(c);
                const float mult = window_mult<BITS>(c);
                for (int ch = 0; ch < nch; ++ch) {
                    float v[32];
                    tmem_ld32(dcol + ch * 32, v);
                    if (quarter >= 2) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) ex[j * 64 + (quarter - 2) * 32 + lane] = f32_to_bf16_bits(v[j]);
                    }
                    named_bar(1, G_EPI_WARPS * 32);
                    if (quarter < 2) {
                        const int jlim = min(32, t.np - ch * 32);
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (j < jlim) {
                                const float g = bf16_bits_to_f32(f32_to_bf16_bits(v[j]));
                                const float u = bf16_bits_to_f32(ex[j * 64 + quarter * 32 + lane]);
                                const float h = bf16_bits_to_f32(f32_to_bf16_bits(g / (1.0f + expf(-g)) * u));
                                a.out[static_cast<size_t>(t.p0 + ch * 32 + j) * a.out_ld + pos] =
                                    __float2bfloat16_rn(h * mult);
                            }
                        }
                    }
                    named_bar(1, G_EPI_WARPS * 32);
                }
            } else {
                const int n = t.rb * 128 + quarter * 32 + lane;
                for (int ch = 0; ch < nch; ++ch) {
                    float v[32];
                    tmem_ld32(dcol + ch * 32, v);
                    const int jlim = min(32, t.np - ch * 32);
                    __nv_bfloat16* o = a.out + static_cast<size_t>(t.p0 + ch * 32) * a.out_ld + n;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (j < jlim) *o = __float2bfloat16_rn(v[j]);
                        o += a.out_ld;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_free[db]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

template <int BITS, bool GATE_UP, int XR>
q38_status launch_grouped_xr(q38_ctx* ctx, const GroupedProblem& p) {
    using F = GF<BITS, XR>;
    static_assert(F::W_STAGES >= 4 && F::SMEM <= 227 * 1024, "grouped stages do not fit");
    auto kern = qgemm_grouped<BITS, GATE_UP, XR>;
    static std::mutex mu;
    static bool configured[64] = {};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device < 64 && !configured[ctx->device]) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, F::SMEM) != cudaSuccess)
                return check_launch(ctx, "cudaFuncSetAttribute");
            configured[ctx->device] = true;
        }
    }
    constexpr int rows_box = 64;  // every weight box is 64 rows, two per tile
    const uint64_t kw = static_cast<uint64_t>(p.K) * BITS / 32;
    const uint64_t rows = static_cast<uint64_t>(p.E) * p.rows_per_expert;
    CUtensorMap mx, mc0, mc1, ms0, ms1, mb0, mb1;
    const CUtensorMapSwizzle cswz = code_swizzle<BITS>();
    const void* b0 = p.b0 ? p.b0 : p.s0;
    const void* b1 = p.b1 ? p.b1 : p.s1;
    if (!make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.x, p.K, p.pairs, 64, G_XBOX,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&mc0, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.w0, kw, rows, F::CODE_W, rows_box, cswz) ||
        !make_map_2d(&mc1, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.w1, kw, rows, F::CODE_W, rows_box, cswz) ||
        !make_map_2d(&ms0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.s0, p.K / 64, rows, 8, rows_box,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&ms1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.s1, p.K / 64, rows, 8, rows_box,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&mb0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b0, p.K / 64, rows, 8, rows_box,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&mb1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b1, p.K / 64, rows, 8, rows_box,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(ctx, Q38_ERR_CUDA, "switch_glu: tensor map encoding failed");
    GArgs args;
    args.tiles = p.tiles;
    args.ntiles = p.ntiles;
    args.out = static_cast<__nv_bfloat16*>(p.out);
    args.status = ctx->d_status;
    args.K = p.K;
    args.rows_per_expert = p.rows_per_expert;
    args.out_ld = p.out_ld;
    args.has_bias = p.b0 != nullptr;
    int grid = ctx->num_sms;
    if (grid > p.max_tiles) grid = p.max_tiles;
    if (grid < 1) grid = 1;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(G_THREADS);
    cfg.dynamicSmemBytes = F::SMEM;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, mx, mc0, mc1, ms0, ms1, mb0, mb1, args) != cudaSuccess)
        return check_launch(ctx, "qgemm_grouped");
    return check_launch(ctx, "qgemm_grouped");
}

template <int BITS, bool GATE_UP>
q38_status launch_grouped(q38_ctx* ctx, const GroupedProblem& p) {
    switch (p.xr) {
        case 32: return launch_grouped_xr<BITS, GATE_UP, 32>(ctx, p);
        case 64: return launch_grouped_xr<BITS, GATE_UP, 64>(ctx, p);
        default: return launch_grouped_xr<BITS, GATE_UP, 128>(ctx, p);
    }
}

}  // namespace

q38_status grouped_gate_up(q38_ctx* ctx, const GroupedProblem& p, int bits) {
    switch (bits) {
        case 2: return launch_grouped<2, true>(ctx, p);
        case 3: return launch_grouped<3, true>(ctx, p);
        case 8: return launch_grouped<8, true>(ctx, p);
        default: return launch_grouped<4, true>(ctx, p);
    }
}

q38_status grouped_down(q38_ctx* ctx, const GroupedProblem& p, int bits) {
    switch (bits) {
        case 2: return launch_grouped<2, false>(ctx, p);
        case 3: return launch_grouped<3, false>(ctx, p);
        case 8: return launch_grouped<8, false>(ctx, p);
        default: return launch_grouped<4, false>(ctx, p);
    }
}

// Activations of the gate/up products, gathered into expert-sorted pair order, permuted
// and 2^-p-scaled per 64-group: xs[j] = permute(x[perm[j] / top_k]).
template <int BITS>
__global__ void __launch_bounds__(256) moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int H,
                                                         const int32_t* __restrict__ perm, int pairs, int top_k,
                                                         const int32_t* __restrict__ valid,
                                                         __nv_bfloat16* __restrict__ xs) {
    griddep_wait();
    griddep_launch_dependents();
    // 16-byte chunks (8 activations each), consecutive lanes on consecutive chunks of a row;
    // a 64-group spans 8 lanes, and each of its 16-element quarters two neighbouring lanes,
    // which swap their chunks to form the quarter's permuted words.  Grid-stride over the
    // valid pairs only (the grid is sized for the GPU, not for every pair: most pairs of an
    // expert-parallel exchange are empty slots); runs start at multiples of the warp, so a
    // lane pair always steps together.
    const int CH = H / 8;
    const int64_t n = static_cast<int64_t>(min(pairs, *valid)) * CH;  // pairs past *valid feed no tile
    const int lane = threadIdx.x & 31;
    // each warp takes U runs of 32 consecutive chunks per step, their loads issued together;
    // a run lies in one row (CH is a multiple of 64), found by one division per step
    constexpr int U = 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * U;
    for (int64_t base = (static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31)) * U; base < n;
         base += stride) {
        const int j0 = static_cast<int>(base / CH), c0 = static_cast<int>(base - static_cast<int64_t>(j0) * CH);
        int jr[U], chr[U];
        uint4 u[U];
#pragma unroll
        for (int r = 0; r < U; ++r) {
            const int cc = c0 + r * 32;
            const int dj = cc / CH;
            jr[r] = j0 + dj;
            chr[r] = cc - dj * CH + lane;
            u[r] = make_uint4(0u, 0u, 0u, 0u);
            if (base + r * 32 < n)
                u[r] = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(perm[jr[r]] / top_k) * H + chr[r] * 8);
        }
#pragma unroll
        for (int r = 0; r < U; ++r) {
            uint4 v;
            v.x = __shfl_xor_sync(0xffffffffu, u[r].x, 1);
            v.y = __shfl_xor_sync(0xffffffffu, u[r].y, 1);
            v.z = __shfl_xor_sync(0xffffffffu, u[r].z, 1);
            v.w = __shfl_xor_sync(0xffffffffu, u[r].w, 1);
            if (base + r * 32 >= n) continue;  // whole runs: n is a multiple of CH
            const int j = jr[r], ch = chr[r];
            const bool odd = ch & 1;
            const uint4 lo = odd ? v : u[r], hi = odd ? u[r] : v;  // elements 0-7 and 8-15 of the quarter
            const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            float e[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                e[2 * i] = bf16_bits_to_f32(w[i] & 0xFFFFu);
                e[2 * i + 1] = bf16_bits_to_f32(w[i] >> 16);
            }
            uint32_t o[4];
            if (odd) {
#pragma unroll
                for (int t = 0; t < 4; ++t)
                    o[t] = pack_bf16x2(e[tc_pair_code<BITS>(4 + t, 0)] * tc_pair_mult<BITS>(4 + t, 0),
                                       e[tc_pair_code<BITS>(4 + t, 1)] * tc_pair_mult<BITS>(4 + t, 1));
            } else {
#pragma unroll
                for (int t = 0; t < 4; ++t)
                    o[t] = pack_bf16x2(e[tc_pair_code<BITS>(t, 0)] * tc_pair_mult<BITS>(t, 0),
                                       e[tc_pair_code<BITS>(t, 1)] * tc_pair_mult<BITS>(t, 1));
            }
            *reinterpret_cast<uint4*>(xs + static_cast<size_t>(j) * H + ch * 8) =
                make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

q38_status moe_gather_launch(q38_ctx* ctx, const void* x, int H, const int32_t* perm, int pairs, int top_k,
                             const int32_t* valid, void* xs, int bits) {
    const long long items = static_cast<long long>(pairs) * (H / 8);
    const long long cap = static_cast<long long>(ctx->num_sms) * 32;  // 4 waves of 8 resident blocks per SM
    const long long need = (items + 4 * 256 - 1) / (4 * 256);     // 4 chunks per thread and step
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(std::max(1LL, std::min(cap, need))));
    cfg.blockDim = dim3(256);
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(xs);
    cudaError_t e;
    switch (bits) {
        case 2: e = cudaLaunchKernelEx(&cfg, moe_gather_kernel<2>, xb, H, perm, pairs, top_k, valid, o); break;
        case 3: e = cudaLaunchKernelEx(&cfg, moe_gather_kernel<3>, xb, H, perm, pairs, top_k, valid, o); break;
        case 8: e = cudaLaunchKernelEx(&cfg, moe_gather_kernel<8>, xb, H, perm, pairs, top_k, valid, o); break;
        default: e = cudaLaunchKernelEx(&cfg, moe_gather_kernel<4>, xb, H, perm, pairs, top_k, valid, o); break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_CUDA, "moe_gather: launch failed: %s", cudaGetErrorString(e));
    }
    return check_launch(ctx, "moe_gather");
}

}  // namespace q38
