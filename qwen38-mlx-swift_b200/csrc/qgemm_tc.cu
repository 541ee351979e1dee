// Prefill-shaped MLX-affine quantized product on the 5th-generation tensor cores:
// y[M,N] = x[M,K] . dequant(W)[N,K]^T for M > 16 tokens, group 64, K % 128 == 0,
// bits 2/3/4, bf16 activations and scales.  Replaces the Metal `qmm` kernel behind
// MLX.quantizedMM (QuantizedLinear.callAsFunction,
// Sources/Qwen38Core/FlashNext/Qwen4ExpPrequantized.swift:156-159) for prompt-sized inputs.
//
// Roles per CTA (one CTA per SM, persistent over 128-row x 128-token output tiles):
//   warp 0     TMA producer: per 128-k stage, the activation tile (two 128-byte-swizzled
//              64-element boxes), the weight rows' packed codes (swizzled box) and the
//              8-group scale/bias boxes, into a ring of stages.
//   warp 1     allocates TMEM; issues tcgen05.mma (M = 128 weight rows, N = 128 tokens,
//              K = 16) with the weights as the TMEM operand and the activations as the
//              shared-memory operand, accumulating the tile in TMEM (double-buffered).
//   warps 2-5  dequantize: one thread per weight row turns its 128 codes per stage into
//              exact bf16 weights w = scale*q + bias (magic-number extraction, bf16x2
//              subtract and fused multiply-add, one rounding) and stores them to a TMEM
//              operand slot with tcgen05.st -- the weights never pass through shared memory.
//   warps 6-9  epilogue: read a finished accumulator tile from TMEM, convert to bf16, store.
// The extraction yields codes in a fixed permuted order, some pre-multiplied by 2^p; the
// prologue kernel writes the activations permuted and scaled by 2^-p to match, so the
// products pair up exactly: sum_k' (2^p w_k)(2^-p x_k) = sum_k w_k x_k.
#include <mutex>

#include "affine_codes.cuh"

namespace q38 {
namespace {

constexpr int P_ROWS = 128;   // weight rows per tile (MMA M, TMEM lanes)
constexpr int P_TOK = 128;    // tokens per tile (MMA N)
constexpr int P_KS = 128;     // k per stage (2 groups)
constexpr int P_ASLOTS = 4;   // TMEM weight-operand slots, 64 columns each
constexpr int P_THREADS = 10 * 32;
constexpr uint32_t P_IDESC = idesc_bf16_f32(P_ROWS, P_TOK);

template <int BITS>
struct PF {
    static constexpr int CODE_W = 4 * BITS;               // code words per row per stage
    static constexpr int CODE_B = P_ROWS * CODE_W * 4;    // 4 / 6 / 8 KiB
    static constexpr int SW = BITS == 2 ? 32 : BITS == 4 ? 64 : 0;  // code box swizzle span
    static constexpr int X_B = 2 * P_TOK * 128;           // two 64-element 128-byte-swizzled boxes
    static constexpr int SB_B = 2 * 2048;                 // scales + biases, {8 groups, 128 rows}
    static constexpr int STAGE = (X_B + CODE_B + SB_B + 1023) / 1024 * 1024;
};

// ---------------------------------------------------------------------------------
// Prologue: x' = activations permuted within each 64-group into extraction order and
// scaled by 2^-p (slot k' = 2*col + half, col = quarter*8 + pair).
// ---------------------------------------------------------------------------------
template <int BITS>
__global__ void __launch_bounds__(256) qgemm_prep(const __nv_bfloat16* __restrict__ x, int64_t M, int K,
                                                  __nv_bfloat16* __restrict__ xp) {
    griddep_launch_dependents();
    griddep_wait();
    const int G = K / 64;
    const int64_t item = blockIdx.x * 256LL + threadIdx.x;  // (token, group)
    if (item >= M * G) return;
    const int64_t m = item / G;
    const int g = static_cast<int>(item % G);
    const uint4* src = reinterpret_cast<const uint4*>(x + m * K + g * 64);
    float xv[64];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 u = src[i];
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
        out[col] = pack_bf16x2(xv[16 * tq + pair_code<BITS>(q, 0)] * pair_mult<BITS>(q, 0),
                               xv[16 * tq + pair_code<BITS>(q, 1)] * pair_mult<BITS>(q, 1));
    }
    uint4* dst = reinterpret_cast<uint4*>(xp + m * K + g * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_uint4(out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
}

struct PArgs {
    __nv_bfloat16* y;
    uint32_t* status;
    int M, N, K, nN, ntiles, stages, has_bias;
};

__device__ __forceinline__ bool p_wait(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (clock64() - t0 > kWaitLimitCycles) {
            if (status) atomicOr(status, Q38_DEV_TIMEOUT);
            *abort = 1;
            return false;
        }
    }
    return true;
}

// Every lane waits (each observes the phase, so TMA-written data is visible to it); the
// warp then agrees on the outcome so that the .sync.aligned TMEM accesses stay convergent.
__device__ __forceinline__ bool p_wait_warp(uint64_t* bar, uint32_t parity, uint32_t* status, volatile int* abort) {
    const bool ok = p_wait(bar, parity, status, abort);
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
// A-column order, 32 bf16x2 values.
template <int BITS>
__device__ __forceinline__ void dequant_group(const uint8_t* codes, int row, int gg, float s, float b, uint32_t* a) {
    using F = PF<BITS>;
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
    const uint32_t s2 = pack_bf16x2(s, s);
#pragma unroll
    for (int tq = 0; tq < 4; ++tq) {
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
            const uint32_t b2 = pack_bf16x2(b / pair_mult<BITS>(q, 0), b / pair_mult<BITS>(q, 1));
            a[tq * 8 + q] = bf2_fma(bf2_sub(v[q], MAGIC), s2, b2);
        }
    }
}

template <int BITS>
__global__ void __launch_bounds__(P_THREADS, 1) qgemm_tc(const __grid_constant__ CUtensorMap map_x,
                                                        const __grid_constant__ CUtensorMap map_codes,
                                                        const __grid_constant__ CUtensorMap map_scales,
                                                        const __grid_constant__ CUtensorMap map_biases,
                                                        const PArgs a) {
    using F = PF<BITS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* stage_full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* stage_empty = stage_full + 8;
    uint64_t* a_full = stage_empty + 8;
    uint64_t* a_free = a_full + P_ASLOTS;
    uint64_t* d_full = a_free + P_ASLOTS;
    uint64_t* d_free = d_full + 2;
    uint64_t* final_bar = d_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* stages = smem + 1024;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ksteps = a.K / P_KS;
    if (threadIdx.x == 0) {
        for (int i = 0; i < a.stages; ++i) {
            mbar_init(&stage_full[i], 1);
            mbar_init(&stage_empty[i], 5);  // 4 dequant warps + the MMA commit
        }
        for (int i = 0; i < P_ASLOTS; ++i) {
            mbar_init(&a_full[i], 4);
            mbar_init(&a_free[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&d_full[i], 1);
            mbar_init(&d_free[i], 4);
        }
        mbar_init(final_bar, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_launch_dependents();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tensormap(&map_x);
            prefetch_tensormap(&map_codes);
            prefetch_tensormap(&map_scales);
            if (a.has_bias) prefetch_tensormap(&map_biases);
            const uint32_t bytes = F::X_B + F::CODE_B + 2048u * (a.has_bias ? 2u : 1u);
            bool waited = false;
            int gs = 0;
            for (int tile = blockIdx.x; tile < a.ntiles && !*abort; tile += gridDim.x) {
                const int n0 = (tile % a.nN) * P_ROWS, m0 = (tile / a.nN) * P_TOK;
                for (int ks = 0; ks < ksteps; ++ks, ++gs) {
                    const int slot = gs % a.stages;
                    if (gs >= a.stages && !p_wait(&stage_empty[slot], ((gs / a.stages) - 1) & 1, a.status, abort))
                        break;
                    uint8_t* st = stages + static_cast<size_t>(slot) * F::STAGE;
                    const int k0 = ks * P_KS;
                    mbar_arrive_expect_tx(&stage_full[slot], bytes);
                    tma_load_2d(st + F::X_B, &map_codes, &stage_full[slot], k0 * BITS / 32, n0);
                    tma_load_2d(st + F::X_B + F::CODE_B, &map_scales, &stage_full[slot], (k0 / 512) * 8, n0);
                    if (a.has_bias)
                        tma_load_2d(st + F::X_B + F::CODE_B + 2048, &map_biases, &stage_full[slot], (k0 / 512) * 8, n0);
                    if (!waited) {
                        griddep_wait();  // the permuted activations come from the prologue kernel
                        waited = true;
                    }
                    tma_load_2d(st, &map_x, &stage_full[slot], k0, m0);
                    tma_load_2d(st + P_TOK * 128, &map_x, &stage_full[slot], k0 + 64, m0);
                }
            }
            // No copy may still be landing when the CTA exits (matters only after an abort:
            // otherwise the consumers have already waited for every fill).
            const int last = gs < a.stages ? gs : a.stages;
            for (int i = 1; i <= last; ++i) {
                const int g = gs - i;
                mbar_wait(&stage_full[g % a.stages], (g / a.stages) & 1, a.status);
            }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int gs = 0, tc = 0;
            for (int tile = blockIdx.x; tile < a.ntiles && !*abort; tile += gridDim.x, ++tc) {
                const int db = tc & 1;
                if (tc >= 2 && !p_wait(&d_free[db], ((tc >> 1) - 1) & 1, a.status, abort)) break;
                tc_fence_after();
                const uint32_t dcol = tmem + 256 + db * P_TOK;
                bool ok = true;
                for (int ks = 0; ks < ksteps; ++ks, ++gs) {
                    const int slot = gs % a.stages, as = gs % P_ASLOTS;
                    if (!p_wait(&stage_full[slot], (gs / a.stages) & 1, a.status, abort) ||
                        !p_wait(&a_full[as], (gs / P_ASLOTS) & 1, a.status, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xs = smem_u32(stages + static_cast<size_t>(slot) * F::STAGE);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t bd = smem_desc(xs + (kk >> 2) * (P_TOK * 128) + (kk & 3) * 32, 16, 1024, 2);
                        tc_mma_ts(dcol, tmem + as * 64 + kk * 8, bd, P_IDESC, (ks > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(&stage_empty[slot]);
                    tc_commit(&a_free[as]);
                }
                if (!ok) break;
                tc_commit(&d_full[db]);
            }
            // every MMA (and its TMEM reads) has finished before the teardown frees TMEM
            tc_commit(final_bar);
            mbar_wait(final_bar, 0, a.status);
        }
    } else if (warp < 6) {
        // ----------------------------------------------------------------- dequant
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        int gs = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x) {
            for (int ks = 0; ks < ksteps; ++ks, ++gs) {
                const int slot = gs % a.stages, as = gs % P_ASLOTS;
                if (!p_wait_warp(&stage_full[slot], (gs / a.stages) & 1, a.status, abort)) {
                    ok = false;
                    break;
                }
                if (gs >= P_ASLOTS && !p_wait_warp(&a_free[as], ((gs / P_ASLOTS) - 1) & 1, a.status, abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint8_t* st = stages + static_cast<size_t>(slot) * F::STAGE;
                const uint16_t* sc = reinterpret_cast<const uint16_t*>(st + F::X_B + F::CODE_B) + row * 8 +
                                     ((ks * P_KS / 64) & 7);
                const float s0 = bf16_bits_to_f32(sc[0]), s1 = bf16_bits_to_f32(sc[1]);
                const float b0 = a.has_bias ? bf16_bits_to_f32(sc[1024]) : 0.f;
                const float b1 = a.has_bias ? bf16_bits_to_f32(sc[1025]) : 0.f;
                uint32_t av[32];
                dequant_group<BITS>(st + F::X_B, row, 0, s0, b0, av);
                tmem_st32(tmem + lane_off + as * 64, av);
                dequant_group<BITS>(st + F::X_B, row, 1, s1, b1, av);
                tmem_st32(tmem + lane_off + as * 64 + 32, av);
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[as]);
                    mbar_arrive(&stage_empty[slot]);
                }
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        int tc = 0;
        for (int tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x, ++tc) {
            const int db = tc & 1;
            if (!p_wait_warp(&d_full[db], (tc >> 1) & 1, a.status, abort)) break;
            tc_fence_after();
            const int n = (tile % a.nN) * P_ROWS + row, m0 = (tile / a.nN) * P_TOK;
#pragma unroll 1
            for (int ch = 0; ch < P_TOK / 32; ++ch) {
                float v[32];
                tmem_ld32(tmem + lane_off + 256 + db * P_TOK + ch * 32, v);
                if (n < a.N) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int m = m0 + ch * 32 + i;
                        if (m < a.M) a.y[static_cast<size_t>(m) * a.N + n] = __float2bfloat16_rn(v[i]);
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

template <int BITS>
q38_status launch(q38_ctx* ctx, const void* x, int M, int K, const uint32_t* w, const void* s, const void* b,
                  int N, void* y) {
    using F = PF<BITS>;
    q38_status st = ensure_workspace(ctx, static_cast<size_t>(M) * K * 2);
    if (st != Q38_OK) return st;
    __nv_bfloat16* xp = static_cast<__nv_bfloat16*>(ctx->workspace);

    CUtensorMap mx, mc, ms, mb;
    const CUtensorMapSwizzle cswz = F::SW == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                    : F::SW == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                  : CU_TENSOR_MAP_SWIZZLE_NONE;
    if (!make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xp, K, M, 64, P_TOK, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&mc, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w, static_cast<uint64_t>(K) * BITS / 32, N,
                     F::CODE_W, P_ROWS, cswz) ||
        !make_map_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s, K / 64, N, 8, P_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b ? b : s, K / 64, N, 8, P_ROWS,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return fail(ctx, Q38_ERR_CUDA, "quantized_matmul: tensor map encoding failed");

    int stages = (227 * 1024 - 2048) / F::STAGE;
    if (stages > 8) stages = 8;
    if (stages < 2) return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: prefill stage too large");
    const int smem = 2048 + stages * F::STAGE;

    auto kmain = qgemm_tc<BITS>;
    static std::mutex mu;
    static bool configured[64] = {};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device < 64 && !configured[ctx->device]) {
            if (cudaFuncSetAttribute(kmain, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
                return check_launch(ctx, "cudaFuncSetAttribute");
            configured[ctx->device] = true;
        }
    }
    const int nN = (N + P_ROWS - 1) / P_ROWS, nM = (M + P_TOK - 1) / P_TOK;
    const int ntiles = nN * nM;
    const int grid = ntiles < ctx->num_sms ? ntiles : ctx->num_sms;

    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    const long long items = static_cast<long long>(M) * (K / 64);
    cudaLaunchConfig_t pcfg = {};
    pcfg.gridDim = dim3(static_cast<unsigned>((items + 255) / 256));
    pcfg.blockDim = dim3(256);
    pcfg.stream = ctx->stream;
    pcfg.attrs = attr;
    pcfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&pcfg, qgemm_prep<BITS>, static_cast<const __nv_bfloat16*>(x), static_cast<int64_t>(M), K,
                           xp) != cudaSuccess)
        return check_launch(ctx, "qgemm_prep");

    PArgs args;
    args.y = static_cast<__nv_bfloat16*>(y);
    args.status = ctx->d_status;
    args.M = M;
    args.N = N;
    args.K = K;
    args.nN = nN;
    args.ntiles = ntiles;
    args.stages = stages;
    args.has_bias = b != nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kmain, mx, mc, ms, mb, args) != cudaSuccess) return check_launch(ctx, "qgemm_tc");
    return check_launch(ctx, "qgemm_tc");
}

}  // namespace

bool qgemm_tc_supported(int64_t M, int64_t K, int group, int bits, q38_dtype xd, q38_dtype sd, const void* x,
                        const void* w, const void* s, const void* b, const void* y) {
    if (M < 17 || M > (1 << 24) || group != 64 || K % 512 != 0 || K <= 0 || K > (1 << 20)) return false;
    if (bits != 2 && bits != 3 && bits != 4) return false;
    if (xd != Q38_BF16 || sd != Q38_BF16) return false;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return al(x) && al(w) && al(s) && (!b || al(b)) && al(y);
}

q38_status qgemm_tc_run(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w, const void* s,
                        const void* b, int64_t N, int bits, void* y) {
    const int m = static_cast<int>(M), k = static_cast<int>(K), n = static_cast<int>(N);
    switch (bits) {
        case 2: return launch<2>(ctx, x, m, k, w, s, b, n, y);
        case 3: return launch<3>(ctx, x, m, k, w, s, b, n, y);
        default: return launch<4>(ctx, x, m, k, w, s, b, n, y);
    }
}

}  // namespace q38
