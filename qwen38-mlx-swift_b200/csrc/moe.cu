// The sparse-MoE layer of Flash-Next (Qwen4ExpSparseMoE.callAsFunction,
// Sources/Qwen38Core/FlashNext/Qwen4ExpSparseMoE.swift:275-294): router, expert sort and
// SwitchGLU with the score-weighted combine.
//
//   router   logits = bf16(x . Wr^T) (fp32 accumulation; CUDA cores for a few tokens, a
//            tcgen05 GEMM for prompts), probs = bf16(softmax_fp32(logits)), top-k in the
//            canonical order (probability descending, expert id ascending on ties),
//            scores = probs[idx] renormalised by bf16(sum) when asked (:208-214, :275-281).
//            The softmax fixes its arithmetic: exp by Cody-Waite reduction and a degree-7
//            Taylor polynomial (fused multiply-adds), the sum as 32 per-lane strided sums
//            folded by a butterfly, IEEE division -- so equal logits give bit-equal
//            probabilities, indices and scores on any implementation that follows it.
//   sort     stable counting sort of the T*k (token, slot) pairs by expert: perm, per-expert
//            offsets and the inverse permutation (SwitchGLU's sort by expert).
//   SwitchGLU per pair down(silu(gate(x)) * up(x)) on the selected expert, as grouped
//            tcgen05 products over expert-sorted pairs (qgemm_grouped.cu), then
//            out_t = bf16(sum_k score_tk * y_tk) in slot order.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "affine_scalar.cuh"
#include "moe_internal.h"
#include "tc_pipeline.cuh"

namespace q38 {
namespace {

// ------------------------------------------------------------------------- router
// exp(x) for x <= 0: n = rint(x log2 e), r = x - n ln2 (ln2 split in a high part with
// trailing zero bits and a low part), e^r by its Taylor polynomial to degree 7 in Horner
// form with fused multiply-adds, times 2^n; 0 below -87.
__device__ __forceinline__ float router_exp(float x) {
    if (x < -87.0f) return 0.0f;
    const float n = rintf(x * 1.44269504088896341f);
    float r = __fmaf_rn(-n, 0.693145751953125f, x);
    r = __fmaf_rn(-n, 1.42860682030941723e-6f, r);
    float p = 1.0f / 5040.0f;
    p = __fmaf_rn(p, r, 1.0f / 720.0f);
    p = __fmaf_rn(p, r, 1.0f / 120.0f);
    p = __fmaf_rn(p, r, 1.0f / 24.0f);
    p = __fmaf_rn(p, r, 1.0f / 6.0f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = static_cast<int>(n);
    return __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(ni + 127) << 23));
}

// logits for a few tokens on CUDA cores: one warp per expert (4 per block), NT (1-8)
// tokens staged in shared memory; each lane accumulates 8-element slices of the row, the
// warp reduces.
template <int NT>
__global__ void __launch_bounds__(128) router_logits_small(const __nv_bfloat16* __restrict__ x, int T, int H,
                                                           const __nv_bfloat16* __restrict__ wr, int E,
                                                           __nv_bfloat16* __restrict__ logits) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    extern __shared__ uint4 xs4[];
    const int t0 = blockIdx.y * NT;
    const int nt = min(NT, T - t0);
    const int vec = H / 8;
    for (int i = threadIdx.x; i < NT * vec; i += 128) {
        const int t = i / vec;
        xs4[i] = t < nt ? reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0 + t) * H)[i % vec]
                        : make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * 4 + warp;
    if (e >= E) return;
    const uint4* wrow = reinterpret_cast<const uint4*>(wr + static_cast<size_t>(e) * H);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    for (int v0 = lane; v0 < vec; v0 += 32 * 8) {
        uint4 wu[8];  // eight 16-byte loads in flight per lane
#pragma unroll
        for (int i = 0; i < 8; ++i) wu[i] = v0 + 32 * i < vec ? __ldg(wrow + v0 + 32 * i) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + 32 * i;
            if (v >= vec) break;
            const uint32_t q[4] = {wu[i].x, wu[i].y, wu[i].z, wu[i].w};
            float wv[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                wv[2 * j] = bf16_bits_to_f32(q[j] & 0xFFFFu);
                wv[2 * j + 1] = bf16_bits_to_f32(q[j] >> 16);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const uint4 xu = xs4[t * vec + v];
                const uint32_t xq[4] = {xu.x, xu.y, xu.z, xu.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[t] = fmaf(wv[2 * j], bf16_bits_to_f32(xq[j] & 0xFFFFu), acc[t]);
                    acc[t] = fmaf(wv[2 * j + 1], bf16_bits_to_f32(xq[j] >> 16), acc[t]);
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && t < nt) logits[static_cast<size_t>(t0 + t) * E + e] = __float2bfloat16_rn(v);
    }
}

// logits for prompts on the tensor cores: one CTA per 128 tokens x 128 experts, both
// operands TMA-loaded with the 128-byte swizzle (64-element k boxes, 6-stage ring), the
// fp32 accumulator in TMEM, four warps drain it with 16-byte stores.
constexpr int R_STAGES = 6;
constexpr int R_N = 128;
constexpr int R_A = 128 * 128, R_B = R_N * 128;

__global__ void __launch_bounds__(128, 1) router_logits_tc(const __grid_constant__ CUtensorMap map_x,
                                                           const __grid_constant__ CUtensorMap map_w, int T, int H,
                                                           int E, __nv_bfloat16* __restrict__ logits,
                                                           uint32_t* status) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + R_STAGES;
    uint64_t* done = empty + R_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    uint8_t* ring = smem + 1024;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * 128, e0 = blockIdx.y * R_N;
    const int ksteps = H / 64;
    if (threadIdx.x == 0) {
        for (int i = 0; i < R_STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, R_N);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    if (warp == 0 && lane == 0) {
        for (int ks = 0; ks < ksteps; ++ks) {
            const int s = ks % R_STAGES;
            if (ks >= R_STAGES && !mbar_wait(&empty[s], ((ks / R_STAGES) - 1) & 1, status)) break;
            uint8_t* st = ring + s * (R_A + R_B);
            mbar_arrive_expect_tx(&full[s], R_A + R_B);
            tma_load_2d(st, &map_x, &full[s], ks * 64, t0);
            tma_load_2d(st + R_A, &map_w, &full[s], ks * 64, e0);
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = idesc_bf16_f32(128, R_N);
        for (int ks = 0; ks < ksteps && ok; ++ks) {
            const int s = ks % R_STAGES;
            if (!mbar_wait(&full[s], (ks / R_STAGES) & 1, status)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a = smem_u32(ring + s * (R_A + R_B));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc_mma_ss(tmem, smem_desc(a + kk * 32, 16, 1024, 2), smem_desc(a + R_A + kk * 32, 16, 1024, 2), idesc,
                          (ks > 0 || kk > 0) ? 1u : 0u);
            tc_commit(&empty[s]);
        }
        tc_commit(done);
    }
    __syncwarp();
    // all four warps: wait for the accumulator, drain 128 tokens x 256 experts
    const bool got = mbar_wait(done, 0, status);
    tc_fence_after();
    const int t = t0 + warp * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const bool vec = (E % 8) == 0;
#pragma unroll 1
    for (int ch = 0; ch < R_N / 32; ++ch) {
        float v[32];
        tmem_ld32(tmem + lane_off + ch * 32, v);
        const int ec = e0 + ch * 32;
        if (got && t < T && vec && ec + 32 <= E) {
            uint4* dst = reinterpret_cast<uint4*>(logits + static_cast<size_t>(t) * E + ec);
#pragma unroll
            for (int q = 0; q < 4; ++q)
                dst[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                                    pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
        } else if (got && t < T) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int e = ec + i;
                if (e < E) logits[static_cast<size_t>(t) * E + e] = __float2bfloat16_rn(v[i]);
            }
        }
    }
    // drain outstanding loads before the CTA exits (only matters after a timeout)
    if (warp == 0 && lane == 0)
        for (int ks = max(0, ksteps - R_STAGES); ks < ksteps; ++ks)
            mbar_wait(&full[ks % R_STAGES], (ks / R_STAGES) & 1, status);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, R_N);
}

// softmax + top-k of one token by one warp; lane l holds experts l, l+32, ... (NJ per lane).
// The r-th winner is kept by lane r; the renormalisation sum accumulates in selection
// order on every lane.  CG: read the logits past L1 (they were written by other blocks of
// the same grid).
template <int NJ, bool CG>
__device__ __forceinline__ void topk_token(const __nv_bfloat16* __restrict__ logits, int t, int E, int top_k,
                                           int normalize, int32_t* __restrict__ indices,
                                           __nv_bfloat16* __restrict__ scores, __nv_bfloat16* __restrict__ probs,
                                           int lane) {
    const uint16_t* l = reinterpret_cast<const uint16_t*>(logits) + static_cast<size_t>(t) * E;
    float v[NJ];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        v[j] = e < E ? bf16_bits_to_f32(CG ? __ldcg(l + e) : l[e]) : -INFINITY;
        mx = fmaxf(mx, v[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float part = 0.0f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        if (lane + 32 * j < E) {
            v[j] = router_exp(__fsub_rn(v[j], mx));
            part = __fadd_rn(part, v[j]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        if (e < E) {
            const uint16_t pb = f32_to_bf16_bits(__fdiv_rn(v[j], part));
            v[j] = bf16_bits_to_f32(pb);
            if (probs) reinterpret_cast<uint16_t*>(probs)[static_cast<size_t>(t) * E + e] = pb;
        } else {
            v[j] = -1.0f;  // never selected: probabilities are >= 0
        }
    }
    // Selection on 32-bit keys: the probability's bf16 bits (order-preserving for values
    // >= 0) above 0xFFFF - expert id, so one warp max picks the largest probability and,
    // among equal ones, the lowest id.  Taken and padding entries have key 0.
    uint32_t key[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        key[j] = e < E ? (static_cast<uint32_t>(f32_to_bf16_bits(v[j])) << 16) | (0xFFFFu - static_cast<uint32_t>(e))
                       : 0u;
    }
    float ssum = 0.0f, my_v = 0.0f;
    int my_i = 0;
    for (int r = 0; r < top_k; ++r) {
        uint32_t m = 0;
#pragma unroll
        for (int j = 0; j < NJ; ++j) m = max(m, key[j]);
        m = __reduce_max_sync(0xffffffffu, m);
        const int bi = static_cast<int>(0xFFFFu - (m & 0xFFFFu));
        const float bv = bf16_bits_to_f32(m >> 16);
        if ((bi & 31) == lane) {
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                if (j == (bi >> 5)) key[j] = 0u;  // taken
        }
        if (lane == r) {
            my_v = bv;
            my_i = bi;
        }
        ssum = __fadd_rn(ssum, bv);
    }
    if (lane < top_k) {
        const float denom = bf16_bits_to_f32(f32_to_bf16_bits(ssum));
        indices[static_cast<size_t>(t) * top_k + lane] = my_i;
        scores[static_cast<size_t>(t) * top_k + lane] = __float2bfloat16_rn(normalize ? __fdiv_rn(my_v, denom) : my_v);
    }
}

// The same selection for one token by the four warps of a block (the one-launch router's
// last block with a single token): the exponentials, divisions and keys are spread over the
// warps (warp w takes the experts lane + 32 j with j = w mod 4), the per-lane sums keep
// topk_token's order (lane l adds its experts l, l + 32, ... in turn), so the results are
// bit-identical to topk_token's.
template <int NJ>
__device__ __forceinline__ void topk_token_block4(const __nv_bfloat16* __restrict__ logits, int E, int top_k,
                                                  int normalize, int32_t* __restrict__ indices,
                                                  __nv_bfloat16* __restrict__ scores,
                                                  __nv_bfloat16* __restrict__ probs, int warp, int lane) {
    __shared__ float s_ev[32 * NJ];
    __shared__ uint32_t s_key[32 * NJ];
    __shared__ float s_red[4];
    const uint16_t* l = reinterpret_cast<const uint16_t*>(logits);
    float v[NJ / 4];
    float mx = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < NJ / 4; ++jj) {
        const int e = lane + 32 * (4 * jj + warp);
        v[jj] = e < E ? bf16_bits_to_f32(__ldcg(l + e)) : -INFINITY;
        mx = fmaxf(mx, v[jj]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
#pragma unroll
    for (int jj = 0; jj < NJ / 4; ++jj) {
        const int e = lane + 32 * (4 * jj + warp);
        if (e < E) s_ev[e] = router_exp(__fsub_rn(v[jj], mx));
    }
    __syncthreads();
    if (warp == 0) {
        float part = 0.0f;
#pragma unroll
        for (int j = 0; j < NJ; ++j)
            if (lane + 32 * j < E) part = __fadd_rn(part, s_ev[lane + 32 * j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
        if (lane == 0) s_red[0] = part;
    }
    __syncthreads();
    const float part = s_red[0];
#pragma unroll
    for (int jj = 0; jj < NJ / 4; ++jj) {
        const int e = lane + 32 * (4 * jj + warp);
        uint32_t key = 0u;
        if (e < E) {
            const uint16_t pb = f32_to_bf16_bits(__fdiv_rn(s_ev[e], part));
            if (probs) reinterpret_cast<uint16_t*>(probs)[e] = pb;
            key = (static_cast<uint32_t>(pb) << 16) | (0xFFFFu - static_cast<uint32_t>(e));
        }
        s_key[lane + 32 * (4 * jj + warp)] = key;
    }
    __syncthreads();
    if (warp != 0) return;
    uint32_t key[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) key[j] = s_key[lane + 32 * j];
    float ssum = 0.0f, my_v = 0.0f;
    int my_i = 0;
    for (int r = 0; r < top_k; ++r) {
        uint32_t m = 0;
#pragma unroll
        for (int j = 0; j < NJ; ++j) m = max(m, key[j]);
        m = __reduce_max_sync(0xffffffffu, m);
        const int bi = static_cast<int>(0xFFFFu - (m & 0xFFFFu));
        const float bv = bf16_bits_to_f32(m >> 16);
        if ((bi & 31) == lane) {
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                if (j == (bi >> 5)) key[j] = 0u;
        }
        if (lane == r) {
            my_v = bv;
            my_i = bi;
        }
        ssum = __fadd_rn(ssum, bv);
    }
    if (lane < top_k) {
        const float denom = bf16_bits_to_f32(f32_to_bf16_bits(ssum));
        indices[lane] = my_i;
        scores[lane] = __float2bfloat16_rn(normalize ? __fdiv_rn(my_v, denom) : my_v);
    }
}

// softmax + top-k, one warp per token.
template <int NJ>
__global__ void __launch_bounds__(256) router_topk(const __nv_bfloat16* __restrict__ logits, int T, int E,
                                                   int top_k, int normalize, int32_t* __restrict__ indices,
                                                   __nv_bfloat16* __restrict__ scores,
                                                   __nv_bfloat16* __restrict__ probs) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    topk_token<NJ, false>(logits, t, E, top_k, normalize, indices, scores, probs, lane);
}

// Router for a few tokens (decode) in one launch: block (b, t) computes the logits of
// experts 4b..4b+3 for token t (one warp each, x_t staged in shared memory, eight 16-byte
// loads in flight per lane), stores them as bf16, and counts itself done on token t's
// counter; the last block of a token (device-scope fence, then the atomic count, which it
// returns to zero) runs that token's softmax and top-k with its four warps.  The tokens'
// selections thus run in parallel on different SMs.
template <int NJ>
__global__ void __launch_bounds__(128) router_decode(const __nv_bfloat16* __restrict__ x, int H,
                                                     const __nv_bfloat16* __restrict__ wr, int E, int top_k,
                                                     int normalize, __nv_bfloat16* __restrict__ logits,
                                                     int32_t* __restrict__ indices, __nv_bfloat16* __restrict__ scores,
                                                     __nv_bfloat16* __restrict__ probs, unsigned int* counters) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    extern __shared__ uint4 xs4[];
    __shared__ bool s_last;
    const int t = blockIdx.y;
    const int vec = H / 8;
    for (int i = threadIdx.x; i < vec; i += 128) xs4[i] = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H)[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * 4 + warp;
    __nv_bfloat16* lt = logits + static_cast<size_t>(t) * E;
    if (e < E) {
        const uint4* wrow = reinterpret_cast<const uint4*>(wr + static_cast<size_t>(e) * H);
        float acc = 0.0f;
        for (int v0 = lane; v0 < vec; v0 += 32 * 8) {
            uint4 wu[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) wu[i] = v0 + 32 * i < vec ? __ldg(wrow + v0 + 32 * i) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int v = v0 + 32 * i;
                if (v >= vec) break;
                const uint32_t q[4] = {wu[i].x, wu[i].y, wu[i].z, wu[i].w};
                const uint4 xu = xs4[v];
                const uint32_t xq[4] = {xu.x, xu.y, xu.z, xu.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc = fmaf(bf16_bits_to_f32(q[j] & 0xFFFFu), bf16_bits_to_f32(xq[j] & 0xFFFFu), acc);
                    acc = fmaf(bf16_bits_to_f32(q[j] >> 16), bf16_bits_to_f32(xq[j] >> 16), acc);
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) lt[e] = __float2bfloat16_rn(acc);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&counters[t], 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    topk_token_block4<NJ>(lt, E, top_k, normalize, indices + static_cast<size_t>(t) * top_k,
                          scores + static_cast<size_t>(t) * top_k, probs ? probs + static_cast<size_t>(t) * E : nullptr,
                          warp, lane);
    if (threadIdx.x == 0) atomicExch(&counters[t], 0u);
}

// --------------------------------------------------------------------------- sort
// Stable counting sort of pairs by expert (key), indices outside [0, E) in an extra
// bucket E after all experts (flagged unless -1, the empty-slot marker).  Pairs are cut into segments of up to 32 per
// warp; per-warp, per-key counts give every (warp, key) run its start, and each warp then
// places its pairs in order (ranks within a warp by __match_any_sync).
//   * up to 1024 pairs: one block, one kernel;
//   * more: blocks of 1024 pairs -- per-block counts, a scan over blocks and keys, and a
//     placement pass that recomputes the per-warp counts.

// -1 marks an empty slot (expert-parallel partial sums): sorted after all experts like an
// invalid index, but not reported.
__device__ __forceinline__ int sort_key(const int32_t* idx, int p, int E, uint32_t* status, bool flag) {
    int e = idx[p];
    if (e < 0 || e >= E) {
        if (flag && e != -1) atomicOr(status, Q38_DEV_BAD_INDEX);
        e = E;
    }
    return e;
}

// Per-warp counts of this block's segment into cnt[warp][B]; each warp walks pairs
// [s0, s1) in chunks of 32.
__device__ __forceinline__ void warp_counts(const int32_t* idx, int s0, int s1, int E, int B, int* cnt,
                                            uint32_t* status, bool flag) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int base = s0; base < s1; base += 32) {
        const int p = base + lane;
        const bool act = p < s1;
        const int e = act ? sort_key(idx, p, E, status, flag) : -1;
        const unsigned am = __ballot_sync(0xffffffffu, act);
        if (act) {
            const unsigned m = __match_any_sync(am, e);
            if ((__ffs(m) - 1) == lane) cnt[warp * B + e] += __popc(m);
        }
        __syncwarp();
    }
}

// Places the segment's pairs given cnt[warp][key] = global start of that warp's run.
__device__ __forceinline__ void warp_place(const int32_t* idx, int s0, int s1, int E, int B, int* cnt,
                                           int32_t* perm, int32_t* inv) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int base = s0; base < s1; base += 32) {
        const int p = base + lane;
        const bool act = p < s1;
        const int e = act ? sort_key(idx, p, E, nullptr, false) : -1;
        const unsigned am = __ballot_sync(0xffffffffu, act);
        if (act) {
            const unsigned m = __match_any_sync(am, e);
            const int pos = cnt[warp * B + e] + __popc(m & ((1u << lane) - 1u));
            perm[pos] = p;
            inv[p] = pos;
            __syncwarp(am);
            if ((__ffs(m) - 1) == lane) cnt[warp * B + e] += __popc(m);
        }
        __syncwarp();
    }
}

// exclusive prefix over the block's warps for every key, in place; block totals to tot[]
__device__ __forceinline__ void warp_prefix(int* cnt, int nw, int B, int* tot) {
    for (int e = threadIdx.x; e < B; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < nw; ++w) {
            const int c = cnt[w * B + e];
            cnt[w * B + e] = run;
            run += c;
        }
        tot[e] = run;
    }
}

// exclusive scan of tot[0..B) (B <= 2048) by the whole block into out[0..B), out[B] = total;
// every thread of the block calls it; blockDim.x == 1024
__device__ __forceinline__ void key_scan_block(const int* tot, int B, int32_t* out, int* wsum) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int a = 2 * t < B ? tot[2 * t] : 0, b = 2 * t + 1 < B ? tot[2 * t + 1] : 0;
    const int v = a + b;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int w = wsum[lane];
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += n;
        }
        wsum[lane] = wi - w;
        if (lane == 31) wsum[32] = wi;
    }
    __syncthreads();
    const int ex = wsum[warp] + incl - v;
    if (2 * t < B) out[2 * t] = ex;
    if (2 * t + 1 < B) out[2 * t + 1] = ex + a;
    if (t == 0) out[B] = wsum[32];
}

// one block of 1024 threads for up to 1024 pairs; nw = ceil(P / 32) warps hold pairs
__global__ void __launch_bounds__(1024, 1) moe_sort_small(const int32_t* __restrict__ idx, int P, int E, int nw,
                                                          int32_t* __restrict__ perm, int32_t* __restrict__ offsets,
                                                          int32_t* __restrict__ inv, uint32_t* status) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    extern __shared__ int cnt[];  // [nw][B] then tot[B] then 33 warp sums
    const int B = E + 1;
    int* tot = cnt + nw * B;
    int* wsum = tot + B;
    for (int i = threadIdx.x; i < nw * B; i += 1024) cnt[i] = 0;
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    if (warp < nw) warp_counts(idx, warp * 32, min(P, warp * 32 + 32), E, B, cnt, status, true);
    __syncthreads();
    warp_prefix(cnt, nw, B, tot);
    __syncthreads();
    key_scan_block(tot, B, offsets, wsum);
    __syncthreads();
    for (int i = threadIdx.x; i < nw * B; i += 1024) cnt[i] += offsets[i % B];
    __syncthreads();
    if (warp < nw) warp_place(idx, warp * 32, min(P, warp * 32 + 32), E, B, cnt, perm, inv);
}

// blocks of 1024 pairs: per-block key totals -> gcnt[block][B]
__global__ void __launch_bounds__(1024, 1) moe_sort_count(const int32_t* __restrict__ idx, int P, int E,
                                                          int* __restrict__ gcnt, uint32_t* status) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    extern __shared__ int cnt[];  // [32][B]
    const int B = E + 1;
    for (int i = threadIdx.x; i < 32 * B; i += 1024) cnt[i] = 0;
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    const int s0 = blockIdx.x * 1024 + warp * 32, s1 = min(P, s0 + 32);
    warp_counts(idx, s0, s1, E, B, cnt, status, true);
    __syncthreads();
    warp_prefix(cnt, 32, B, gcnt + static_cast<size_t>(blockIdx.x) * B);
}

// gcnt[block][key] -> global start of each block's run of each key; offsets
__global__ void __launch_bounds__(1024, 1) moe_sort_scan(int* __restrict__ gcnt, int nblk, int E,
                                                         int32_t* __restrict__ offsets) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    __shared__ int tot[1025];
    const int B = E + 1;
    // per bucket, the exclusive prefix over the blocks' counts; the counts are read eight
    // at a time (all loads in flight before the dependent sums and stores)
    for (int e = threadIdx.x; e < B; e += 1024) {
        int run = 0;
        for (int b0 = 0; b0 < nblk; b0 += 8) {
            int c[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = b0 + i < nblk ? gcnt[static_cast<size_t>(b0 + i) * B + e] : 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (b0 + i < nblk) gcnt[static_cast<size_t>(b0 + i) * B + e] = run;
                run += c[i];
            }
        }
        tot[e] = run;
    }
    __shared__ int wsum[33];
    __syncthreads();
    key_scan_block(tot, B, offsets, wsum);
    __syncthreads();
    for (int e = threadIdx.x; e < B; e += 1024) {
        const int o = offsets[e];
        for (int b0 = 0; b0 < nblk; b0 += 8) {
            int c[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = b0 + i < nblk ? gcnt[static_cast<size_t>(b0 + i) * B + e] : 0;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (b0 + i < nblk) gcnt[static_cast<size_t>(b0 + i) * B + e] = c[i] + o;
        }
    }
}

__global__ void __launch_bounds__(1024, 1) moe_sort_place(const int32_t* __restrict__ idx, int P, int E,
                                                          const int* __restrict__ gbase, int32_t* __restrict__ perm,
                                                          int32_t* __restrict__ inv) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    extern __shared__ int cnt[];  // [32][B] then tot[B]
    const int B = E + 1;
    int* tot = cnt + 32 * B;
    for (int i = threadIdx.x; i < 32 * B; i += 1024) cnt[i] = 0;
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    const int s0 = blockIdx.x * 1024 + warp * 32, s1 = min(P, s0 + 32);
    warp_counts(idx, s0, s1, E, B, cnt, nullptr, false);
    __syncthreads();
    warp_prefix(cnt, 32, B, tot);
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * B; i += 1024) cnt[i] += gbase[static_cast<size_t>(blockIdx.x) * B + i % B];
    __syncthreads();
    warp_place(idx, s0, s1, E, B, cnt, perm, inv);
}

// ---------------------------------------------------------------------- tile lists
// Per expert: ceil(n_e / run) runs of pairs, each crossed with the row blocks of the
// gate/up (I / 64) and down (H / 128) products.
__global__ void __launch_bounds__(1024, 1) moe_tiles_kernel(const int32_t* __restrict__ offsets, int E, int run,
                                                            int rb_gu, int rb_d, MoeTile* __restrict__ gu,
                                                            MoeTile* __restrict__ dn, int* __restrict__ counts) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    __shared__ int warp_tot[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = threadIdx.x;  // E <= 1024: one expert per thread
    const int n = e < E ? offsets[e + 1] - offsets[e] : 0;
    const int runs = (n + run - 1) / run;
    int incl = runs;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int w = warp_tot[lane];
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += v;
        }
        warp_tot[lane] = wi - w;  // exclusive warp offsets
        if (lane == 31) {
            counts[0] = wi * rb_gu;
            counts[1] = wi * rb_d;
        }
    }
    __syncthreads();
    // each expert's first run and run count, then the tiles written by whole warps (one
    // expert at a time per warp, its entries spread over the lanes)
    __shared__ int s_base[1024], s_runs[1024];
    s_base[e] = warp_tot[warp] + incl - runs;
    s_runs[e] = runs;
    __syncthreads();
    const int per = rb_gu + rb_d;
    for (int ee = warp; ee < E; ee += 32) {
        const int nr = s_runs[ee], b0 = s_base[ee], o0 = offsets[ee], ne = offsets[ee + 1] - o0;
        for (int q = lane; q < nr * per; q += 32) {
            const int r = q / per, b = q - r * per;
            const int p0 = o0 + r * run, np = min(run, ne - r * run);
            if (b < rb_gu)
                gu[(b0 + r) * rb_gu + b] = MoeTile{ee, b, p0, np};
            else
                dn[(b0 + r) * rb_d + (b - rb_gu)] = MoeTile{ee, b - rb_gu, p0, np};
        }
    }
}

// ------------------------------------------------------------------------ combine
// out[t] = bf16(sum_k score[t,k] * y[inv[t*k + k']]) in slot order (fp32).
__global__ void __launch_bounds__(256) moe_combine_kernel(const __nv_bfloat16* __restrict__ y, int H,
                                                          const int32_t* __restrict__ inv,
                                                          const int32_t* __restrict__ idx,
                                                          const __nv_bfloat16* __restrict__ scores, int top_k, int E,
                                                          __nv_bfloat16* __restrict__ out) {
    griddep_wait();
    griddep_launch_dependents();
    const int t = blockIdx.x;
    for (int c = threadIdx.x * 8; c < H; c += 256 * 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int s = 0; s < top_k; ++s) {
            const int p = t * top_k + s;
            const int e = idx[p];
            if (e < 0 || e >= E) continue;
            const float sc = __bfloat162float(scores[p]);
            const uint4 u = *reinterpret_cast<const uint4*>(y + static_cast<size_t>(inv[p]) * H + c);
            const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[2 * j] = __fadd_rn(acc[2 * j], __fmul_rn(sc, bf16_bits_to_f32(q[j] & 0xFFFFu)));
                acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], __fmul_rn(sc, bf16_bits_to_f32(q[j] >> 16)));
            }
        }
        uint4 o;
        o.x = pack_bf16x2(acc[0], acc[1]);
        o.y = pack_bf16x2(acc[2], acc[3]);
        o.z = pack_bf16x2(acc[4], acc[5]);
        o.w = pack_bf16x2(acc[6], acc[7]);
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + c) = o;
    }
}

// h = bf16(silu(g) * u), silu(g) = g / (1 + exp(-g)) in fp32; 8 elements per thread.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ g,
                                                       const __nv_bfloat16* __restrict__ u, int64_t n,
                                                       __nv_bfloat16* __restrict__ h) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    const int64_t i = (blockIdx.x * 256LL + threadIdx.x) * 8;
    if (i >= n) return;
    if (i + 8 <= n) {
        const uint4 gv = *reinterpret_cast<const uint4*>(g + i), uv = *reinterpret_cast<const uint4*>(u + i);
        const uint32_t gq[4] = {gv.x, gv.y, gv.z, gv.w}, uq[4] = {uv.x, uv.y, uv.z, uv.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float g0 = bf16_bits_to_f32(gq[j] & 0xFFFFu), g1 = bf16_bits_to_f32(gq[j] >> 16);
            const float u0 = bf16_bits_to_f32(uq[j] & 0xFFFFu), u1 = bf16_bits_to_f32(uq[j] >> 16);
            o[j] = pack_bf16x2(g0 / (1.0f + expf(-g0)) * u0, g1 / (1.0f + expf(-g1)) * u1);
        }
        *reinterpret_cast<uint4*>(h + i) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
        for (int64_t j = i; j < n; ++j) {
            const float gv = __bfloat162float(g[j]);
            h[j] = __float2bfloat16_rn(gv / (1.0f + expf(-gv)) * __bfloat162float(u[j]));
        }
    }
}

// Expert-parallel dispatch: pair j of the destination order (perm) -> its token's row of
// x and its expert's index within the destination rank's contiguous block of experts.
__global__ void __launch_bounds__(256) moe_pack_kernel(const __nv_bfloat16* __restrict__ x, int H,
                                                       const int32_t* __restrict__ idx,
                                                       const int32_t* __restrict__ perm, int64_t P, int top_k,
                                                       int epr, __nv_bfloat16* __restrict__ rows,
                                                       int32_t* __restrict__ local_e) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    const int64_t j = blockIdx.x;
    if (j >= P) return;
    const int p = perm[j];
    const int t = p / top_k;
    if (threadIdx.x == 0) local_e[j] = idx[p] % epr;
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
    uint4* dst = reinterpret_cast<uint4*>(rows + static_cast<size_t>(j) * H);
    for (int c = threadIdx.x; c < H / 8; c += 256) dst[c] = src[c];
}

__global__ void __launch_bounds__(256) invert_perm_kernel(const int32_t* __restrict__ perm, int64_t P,
                                                          int32_t* __restrict__ inv) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    const int64_t j = blockIdx.x * 256LL + threadIdx.x;
    if (j < P) inv[perm[j]] = static_cast<int32_t>(j);
}

// Launch with programmatic dependent launch: the kernel may be scheduled while the
// previous kernel on the stream finishes; every kernel here waits for it (griddepcontrol)
// before touching memory.
template <typename... KArgs, typename... Args>
q38_status launch_pdl(q38_ctx* ctx, const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    return check_launch(ctx, what);
}

// Expert-parallel dispatch plan, one block: token t sends one row to every rank owning one
// of its experts; rows are laid out rank-major, tokens ascending within a rank.
// rowpos[t * world + r] = row index or -1; counts[r] = rows for rank r.
__global__ void __launch_bounds__(1024, 1) ep_plan_kernel(const int32_t* __restrict__ idx, int T, int top_k, int epr,
                                                          int world, int32_t* __restrict__ rowpos,
                                                          int32_t* __restrict__ counts) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    __shared__ int wsum[33];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int base = 0;
    for (int r = 0; r < world; ++r) {
        const int start = base;
        for (int t0 = 0; t0 < T; t0 += 1024) {
            const int t = t0 + threadIdx.x;
            int f = 0;
            if (t < T)
                for (int s2 = 0; s2 < top_k; ++s2) {
                    const int e = idx[static_cast<size_t>(t) * top_k + s2];
                    f |= (e >= 0 && e / epr == r);
                }
            int incl = f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            if (lane == 31) wsum[warp] = incl;
            __syncthreads();
            if (warp == 0) {
                const int w = wsum[lane];
                int wi = w;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int n = __shfl_up_sync(0xffffffffu, wi, o);
                    if (lane >= o) wi += n;
                }
                wsum[lane] = wi - w;
                if (lane == 31) wsum[32] = wi;
            }
            __syncthreads();
            if (t < T) rowpos[static_cast<size_t>(t) * world + r] = f ? base + wsum[warp] + incl - f : -1;
            base += wsum[32];
            __syncthreads();
        }
        if (threadIdx.x == 0) counts[r] = base - start;
    }
}

// rows[rowpos[t, r]] = x[t]; meta row = local expert per slot (or -1 when the slot's expert
// lives elsewhere) followed by the slot scores' bf16 bits.
__global__ void __launch_bounds__(256) ep_pack_kernel(const __nv_bfloat16* __restrict__ x, int H,
                                                      const int32_t* __restrict__ idx,
                                                      const __nv_bfloat16* __restrict__ scores, int top_k, int epr,
                                                      int world, const int32_t* __restrict__ rowpos,
                                                      __nv_bfloat16* __restrict__ rows, int64_t rows_ld,
                                                      int32_t* __restrict__ meta, int64_t meta_ld) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    const int t = blockIdx.x;
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
    for (int r = 0; r < world; ++r) {
        const int row = rowpos[static_cast<size_t>(t) * world + r];
        if (row < 0) continue;
        uint4* dst = reinterpret_cast<uint4*>(rows + static_cast<size_t>(row) * rows_ld);
        for (int c = threadIdx.x; c < H / 8; c += 256) dst[c] = src[c];
        if (threadIdx.x < top_k) {
            const int e = idx[static_cast<size_t>(t) * top_k + threadIdx.x];
            int32_t* m = meta + static_cast<size_t>(row) * meta_ld;
            m[threadIdx.x] = (e >= 0 && e / epr == r) ? e % epr : -1;
            m[top_k + threadIdx.x] =
                reinterpret_cast<const uint16_t*>(scores)[static_cast<size_t>(t) * top_k + threadIdx.x];
        }
    }
}

// out[t] = bf16(sum over ranks r, in rank order, of partial[rowpos[t, r]]) in fp32
__global__ void __launch_bounds__(256) ep_reduce_kernel(const __nv_bfloat16* __restrict__ partial, int H,
                                                        const int32_t* __restrict__ rowpos, int world,
                                                        __nv_bfloat16* __restrict__ out) {
    griddep_wait();  // inputs come from the previous kernel on the stream
    griddep_launch_dependents();
    const int t = blockIdx.x;
    for (int c = threadIdx.x * 8; c < H; c += 256 * 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int r = 0; r < world; ++r) {
            const int row = rowpos[static_cast<size_t>(t) * world + r];
            if (row < 0) continue;
            const uint4 u = *reinterpret_cast<const uint4*>(partial + static_cast<size_t>(row) * H + c);
            const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[2 * j] = __fadd_rn(acc[2 * j], bf16_bits_to_f32(q[j] & 0xFFFFu));
                acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], bf16_bits_to_f32(q[j] >> 16));
            }
        }
        uint4 o;
        o.x = pack_bf16x2(acc[0], acc[1]);
        o.y = pack_bf16x2(acc[2], acc[3]);
        o.z = pack_bf16x2(acc[4], acc[5]);
        o.w = pack_bf16x2(acc[6], acc[7]);
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + c) = o;
    }
}

q38_status set_dev(q38_ctx* ctx) {
    if (cudaSetDevice(ctx->device) != cudaSuccess) return check_launch(ctx, "cudaSetDevice");
    return Q38_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

q38_status topk_launch(q38_ctx* ctx, const void* logits, int64_t T, int64_t E, int top_k, int normalize,
                       int32_t* indices, void* scores, void* probs) {
    const dim3 grid(static_cast<unsigned>((T + 7) / 8));
    auto go = [&](auto kern) {
        return launch_pdl(ctx, "router_topk", kern, grid, dim3(256), 0, static_cast<const __nv_bfloat16*>(logits),
                          static_cast<int>(T), static_cast<int>(E), top_k, normalize, indices,
                          static_cast<__nv_bfloat16*>(scores), static_cast<__nv_bfloat16*>(probs));
    };
    if (E <= 128) return go(router_topk<4>);
    if (E <= 256) return go(router_topk<8>);
    if (E <= 512) return go(router_topk<16>);
    return go(router_topk<32>);
}

q38_status logits_launch(q38_ctx* ctx, const void* x, int64_t T, int64_t H, const void* wr, int64_t E, void* logits) {
    if (T <= 64) {
        const int nt = T >= 8 ? 8 : T >= 4 ? 4 : T >= 2 ? 2 : 1;
        const size_t sm = static_cast<size_t>(2) * nt * H;
        static std::mutex mu;
        static bool big[64] = {};
        if (sm > 48 * 1024) {
            std::lock_guard<std::mutex> lk(mu);
            if (ctx->device < 64 && !big[ctx->device]) {
                if (cudaFuncSetAttribute(router_logits_small<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024) != cudaSuccess ||
                    cudaFuncSetAttribute(router_logits_small<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024) != cudaSuccess ||
                    cudaFuncSetAttribute(router_logits_small<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024) != cudaSuccess ||
                    cudaFuncSetAttribute(router_logits_small<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024) != cudaSuccess)
                    return check_launch(ctx, "cudaFuncSetAttribute");
                big[ctx->device] = true;
            }
        }
        const dim3 grid(static_cast<unsigned>((E + 3) / 4), static_cast<unsigned>((T + nt - 1) / nt));
        auto go = [&](auto kern) {
            return launch_pdl(ctx, "router_logits_small", kern, grid, dim3(128), sm, static_cast<const __nv_bfloat16*>(x),
                              static_cast<int>(T), static_cast<int>(H), static_cast<const __nv_bfloat16*>(wr),
                              static_cast<int>(E), static_cast<__nv_bfloat16*>(logits));
        };
        switch (nt) {
            case 1: return go(router_logits_small<1>);
            case 2: return go(router_logits_small<2>);
            case 4: return go(router_logits_small<4>);
            default: return go(router_logits_small<8>);
        }
    }
    CUtensorMap mx, mw;
    if (!make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, H, T, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wr, H, E, 64, R_N, CU_TENSOR_MAP_SWIZZLE_128B))
        return fail(ctx, Q38_ERR_CUDA, "moe_route: tensor map encoding failed");
    const int smem = 2048 + R_STAGES * (R_A + R_B);
    static std::mutex mu2;
    static bool cfg[64] = {};
    {
        std::lock_guard<std::mutex> lk(mu2);
        if (ctx->device < 64 && !cfg[ctx->device]) {
            if (cudaFuncSetAttribute(router_logits_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
                return check_launch(ctx, "cudaFuncSetAttribute");
            cfg[ctx->device] = true;
        }
    }
    dim3 grid(static_cast<unsigned>((T + 127) / 128), static_cast<unsigned>((E + R_N - 1) / R_N));
    return launch_pdl(ctx, "router_logits_tc", router_logits_tc, grid, dim3(128), smem, mx, mw, static_cast<int>(T),
                      static_cast<int>(H), static_cast<int>(E), static_cast<__nv_bfloat16*>(logits), ctx->d_status);
}

// The one-launch router for up to 16 tokens (each block stages one token's x in shared
// memory; one counter per token in the zero-at-rest region).
q38_status route_decode_launch(q38_ctx* ctx, const void* x, int64_t T, int64_t H, const void* wr, int64_t E,
                               int top_k, int normalize, void* logits, int32_t* indices, void* scores, void* probs) {
    uint32_t* cnt = nullptr;
    float* unused = nullptr;
    q38_status st = ensure_zero_region(ctx, 16, 0, &cnt, &unused);
    if (st != Q38_OK) return st;
    const size_t sm = static_cast<size_t>(2) * H;
    const dim3 grid(static_cast<unsigned>((E + 3) / 4), static_cast<unsigned>(T));
    auto go = [&](auto kern) -> q38_status {
        static std::mutex mu;
        static const void* done[64] = {};
        if (sm > 48 * 1024) {
            std::lock_guard<std::mutex> lk(mu);
            const void* key = current_context_key();
            if (ctx->device < 64 && (!key || done[ctx->device] != key)) {
                if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024) != cudaSuccess)
                    return check_launch(ctx, "cudaFuncSetAttribute");
                done[ctx->device] = key;
            }
        }
        return launch_pdl(ctx, "router_decode", kern, grid, dim3(128), sm, static_cast<const __nv_bfloat16*>(x),
                          static_cast<int>(H), static_cast<const __nv_bfloat16*>(wr), static_cast<int>(E), top_k,
                          normalize, static_cast<__nv_bfloat16*>(logits), indices,
                          static_cast<__nv_bfloat16*>(scores), static_cast<__nv_bfloat16*>(probs),
                          reinterpret_cast<unsigned int*>(cnt));
    };
    if (E <= 128) return go(router_decode<4>);
    if (E <= 256) return go(router_decode<8>);
    if (E <= 512) return go(router_decode<16>);
    return go(router_decode<32>);
}

// Scratch ints the sort needs beyond its outputs (per-block counts for large P).
size_t sort_scratch_ints(int64_t P, int64_t E) {
    return P > 1024 ? static_cast<size_t>((P + 1023) / 1024) * (E + 1) : 1;
}

q38_status sort_launch(q38_ctx* ctx, const int32_t* idx, int64_t P, int64_t E, int32_t* perm, int32_t* offsets,
                       int32_t* inv, int* scratch) {
    static std::mutex mu;
    static bool cfg[64] = {};
    {
        std::lock_guard<std::mutex> lk(mu);
        if (ctx->device < 64 && !cfg[ctx->device]) {
            if (cudaFuncSetAttribute(moe_sort_small, cudaFuncAttributeMaxDynamicSharedMemorySize, 140 * 1024) !=
                    cudaSuccess ||
                cudaFuncSetAttribute(moe_sort_count, cudaFuncAttributeMaxDynamicSharedMemorySize, 140 * 1024) !=
                    cudaSuccess ||
                cudaFuncSetAttribute(moe_sort_place, cudaFuncAttributeMaxDynamicSharedMemorySize, 140 * 1024) !=
                    cudaSuccess)
                return check_launch(ctx, "cudaFuncSetAttribute");
            cfg[ctx->device] = true;
        }
    }
    const int B = static_cast<int>(E + 1);
    if (P <= 1024) {
        const int nw = P > 0 ? static_cast<int>((P + 31) / 32) : 1;
        return launch_pdl(ctx, "moe_sort", moe_sort_small, dim3(1), dim3(1024),
                          static_cast<size_t>(nw + 1) * B * 4 + 33 * 4, idx, static_cast<int>(P), static_cast<int>(E),
                          nw, perm, offsets, inv, ctx->d_status);
    }
    const int nblk = static_cast<int>((P + 1023) / 1024);
    q38_status st = launch_pdl(ctx, "moe_sort_count", moe_sort_count, dim3(nblk), dim3(1024),
                               static_cast<size_t>(32) * B * 4, idx, static_cast<int>(P), static_cast<int>(E), scratch,
                               ctx->d_status);
    if (st != Q38_OK) return st;
    if ((st = launch_pdl(ctx, "moe_sort_scan", moe_sort_scan, dim3(1), dim3(1024), 0, scratch, nblk,
                         static_cast<int>(E), offsets)) != Q38_OK)
        return st;
    return launch_pdl(ctx, "moe_sort_place", moe_sort_place, dim3(nblk), dim3(1024), static_cast<size_t>(33) * B * 4,
                      idx, static_cast<int>(P), static_cast<int>(E), scratch, perm, inv);
}

// The shared expert's contribution added to the routed output (the `shared` term of
// Qwen4ExpSparseMoE.callAsFunction, Sources/Qwen38Core/FlashNext/Qwen4ExpSparseMoE.swift:295-298):
//   out[t] = bf16(routed[t] + bf16(s_t * ys[t])),  s_t = bf16(sigmoid(bf16(x_t . dequant(wsg)))),
// the gate logit a quantized [1, H] product accumulated in fp32 (w = scale * q + bias).  One
// block per token; `routed` and `out` may be the same buffer.
template <typename S>
__global__ void __launch_bounds__(256) shared_expert_combine(const __nv_bfloat16* __restrict__ x, int H,
                                                             const uint32_t* __restrict__ gw, const S* __restrict__ gs,
                                                             const S* __restrict__ gb, int group, int bits,
                                                             const __nv_bfloat16* __restrict__ ys,
                                                             const __nv_bfloat16* routed, __nv_bfloat16* out) {
    griddep_wait();
    griddep_launch_dependents();
    const size_t t0 = static_cast<size_t>(blockIdx.x) * H;
    float acc = 0.f;
    for (int k = threadIdx.x; k < H; k += blockDim.x) {
        const int g = k / group;
        const float w = __fadd_rn(__fmul_rn(to_f32(gs[g]), static_cast<float>(get_code(gw, k, bits))),
                                  gb ? to_f32(gb[g]) : 0.f);
        acc = fmaf(__bfloat162float(x[t0 + k]), w, acc);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    __shared__ float part[8];
    __shared__ float s_gate;
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = 0.f;
        for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) v += part[i];
        const float l = bf16_bits_to_f32(f32_to_bf16_bits(v));
        s_gate = bf16_bits_to_f32(f32_to_bf16_bits(1.0f / (1.0f + expf(-l))));
    }
    __syncthreads();
    const float sg = s_gate;
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
        const float sh = bf16_bits_to_f32(f32_to_bf16_bits(sg * __bfloat162float(ys[t0 + j])));
        out[t0 + j] = __float2bfloat16_rn(__bfloat162float(routed[t0 + j]) + sh);
    }
}

}  // namespace

q38_status shared_combine_launch(q38_ctx* ctx, const void* x, int64_t T, int64_t H, const uint32_t* gw,
                                 const void* gs, const void* gb, q38_dtype sd, int group, int bits, const void* ys,
                                 const void* routed, void* out) {
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
    const __nv_bfloat16* yb = static_cast<const __nv_bfloat16*>(ys);
    const __nv_bfloat16* rb = static_cast<const __nv_bfloat16*>(routed);
    __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(out);
    const dim3 grid(static_cast<unsigned>(T)), block(256);
    const int h = static_cast<int>(H);
    switch (sd) {
        case Q38_F16:
            return launch_pdl(ctx, "shared_expert_combine", shared_expert_combine<__half>, grid, block, 0, xb, h, gw,
                              static_cast<const __half*>(gs), static_cast<const __half*>(gb), group, bits, yb, rb, ob);
        case Q38_F32:
            return launch_pdl(ctx, "shared_expert_combine", shared_expert_combine<float>, grid, block, 0, xb, h, gw,
                              static_cast<const float*>(gs), static_cast<const float*>(gb), group, bits, yb, rb, ob);
        default:
            return launch_pdl(ctx, "shared_expert_combine", shared_expert_combine<__nv_bfloat16>, grid, block, 0, xb,
                              h, gw, static_cast<const __nv_bfloat16*>(gs), static_cast<const __nv_bfloat16*>(gb),
                              group, bits, yb, rb, ob);
    }
}

}  // namespace q38

using namespace q38;

extern "C" {

q38_status q38_moe_route(q38_ctx* ctx, const void* x, int64_t T, int64_t H, q38_dtype x_dtype, const void* wr,
                         int64_t E, int top_k, int normalize, int32_t* indices, void* scores, void* probs) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (x_dtype != Q38_BF16) return fail(ctx, Q38_ERR_UNSUPPORTED, "moe_route: x and the router weight must be bf16");
    if (T < 0 || H <= 0 || H % 64 || E < 1 || E > 1024 || top_k < 1 || top_k > 32 || top_k > E)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT,
                    "moe_route: need H %% 64 == 0, 1 <= E <= 1024, 1 <= top_k <= min(32, E) (H=%lld E=%lld k=%d)",
                    (long long)H, (long long)E, top_k);
    if (T == 0) return Q38_OK;
    if (!x || !wr || !indices || !scores) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_route: null pointer");
    if (!aligned16(x) || !aligned16(wr)) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_route: x and wr must be 16-byte aligned");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    if ((st = ensure_workspace(ctx, static_cast<size_t>(T) * E * 2)) != Q38_OK) return st;
    void* logits = ctx->workspace;
    if (T <= 16 && static_cast<size_t>(H) * 2 <= 96 * 1024) return route_decode_launch(ctx, x, T, H, wr, E, top_k,
                                                                                            normalize, logits, indices,
                                                                                            scores, probs);
    if ((st = logits_launch(ctx, x, T, H, wr, E, logits)) != Q38_OK) return st;
    return topk_launch(ctx, logits, T, E, top_k, normalize, indices, scores, probs);
}

q38_status q38_moe_route_logits(q38_ctx* ctx, const void* logits, int64_t T, int64_t E, int top_k, int normalize,
                                int32_t* indices, void* scores, void* probs) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (T < 0 || E < 1 || E > 1024 || top_k < 1 || top_k > 32 || top_k > E)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_route_logits: need 1 <= E <= 1024, 1 <= top_k <= min(32, E)");
    if (T == 0) return Q38_OK;
    if (!logits || !indices || !scores) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_route_logits: null pointer");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    return topk_launch(ctx, logits, T, E, top_k, normalize, indices, scores, probs);
}

q38_status q38_moe_sort(q38_ctx* ctx, const int32_t* indices, int64_t pairs, int64_t E, int32_t* perm,
                        int32_t* offsets) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (pairs < 0 || pairs > (1 << 30) || E < 1 || E > 1024)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_sort: need 1 <= E <= 1024");
    if (!indices || !perm || !offsets) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_sort: null pointer");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    // offsets has E + 1 entries for the caller; the kernel also writes a bad-index bucket
    void* scratch;
    const size_t inv_bytes = align_up(static_cast<size_t>(std::max<int64_t>(pairs, 1)) * 4, 256);
    const size_t off_bytes = align_up(static_cast<size_t>(E + 2) * 4, 256);
    if ((st = ensure_aux(ctx, inv_bytes + off_bytes + sort_scratch_ints(pairs, E) * 4, &scratch)) != Q38_OK)
        return st;
    int32_t* inv = static_cast<int32_t*>(scratch);
    int32_t* off2 = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(scratch) + inv_bytes);
    int* sscr = reinterpret_cast<int*>(static_cast<uint8_t*>(scratch) + inv_bytes + off_bytes);
    if ((st = sort_launch(ctx, indices, pairs, E, perm, off2, inv, sscr)) != Q38_OK) return st;
    if (cudaMemcpyAsync(offsets, off2, static_cast<size_t>(E + 1) * 4, cudaMemcpyDeviceToDevice, ctx->stream) !=
        cudaSuccess)
        return check_launch(ctx, "moe_sort offsets");
    return Q38_OK;
}

q38_status q38_switch_glu(q38_ctx* ctx, const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int top_k,
                          const int32_t* indices, const void* scores, const uint32_t* gate_w, const void* gate_s,
                          const void* gate_b, const uint32_t* up_w, const void* up_s, const void* up_b,
                          const uint32_t* down_w, const void* down_s, const void* down_b, q38_dtype dtype,
                          int group_size, int bits, void* out) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (dtype != Q38_BF16) return fail(ctx, Q38_ERR_UNSUPPORTED, "switch_glu: x, scales, biases and out must be bf16");
    if (group_size != 64 || (bits != 2 && bits != 3 && bits != 4 && bits != 8))
        return fail(ctx, Q38_ERR_UNSUPPORTED, "switch_glu: implemented for group 64, bits 2/3/4/8 (got %d, %d)",
                    group_size, bits);
    if (T < 0 || H <= 0 || I <= 0 || H % 512 || I % 512 || E < 1 || E > 1024 || top_k < 1 || top_k > E)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT,
                    "switch_glu: need H %% 512 == 0, I %% 512 == 0, 1 <= E <= 1024, 1 <= top_k <= E");
    if ((gate_b == nullptr) != (up_b == nullptr) || (gate_b == nullptr) != (down_b == nullptr))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "switch_glu: biases must be given for all three projections or none");
    if (T == 0) return Q38_OK;
    if (!x || !indices || !scores || !gate_w || !gate_s || !up_w || !up_s || !down_w || !down_s || !out)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "switch_glu: null pointer");
    const int64_t P = T * top_k;
    if (P > (1 << 24)) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "switch_glu: more than 2^24 (token, slot) pairs");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    // a few tokens (decode): the selected experts' weights streamed by the decode kernel
    if (qgemv_moe_supported(T, H, I, E, top_k, group_size, bits, x, gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w,
                            down_s, down_b))
        return qgemv_moe_decode(ctx, x, T, H, I, E, top_k, indices, scores, gate_w, gate_s, gate_b, up_w, up_s, up_b,
                                down_w, down_s, down_b, bits, out);
    const int rb_gu = static_cast<int>(I / 64), rb_d = static_cast<int>(H / 128);
    // An expert receives at most one pair per token, so runs never exceed T pairs.
    // (Runs of at most 96 pairs, for a deeper activation ring at a mean run of 80, measured
    // slower at 4096 tokens: 701 -> 728 us per layer.)
    const int xr = T <= 32 ? 32 : T <= 64 ? 64 : 128;
    const int64_t max_runs = std::min<int64_t>(E, P) + P / xr + 1;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += align_up(bytes, 256);
        return o;
    };
    const size_t o_perm = take(P * 4), o_inv = take(P * 4), o_off = take((E + 2) * 4),
                 o_sscr = take(sort_scratch_ints(P, E) * 4);
    const size_t o_cnt = take(16), o_gu = take(max_runs * rb_gu * sizeof(MoeTile)),
                 o_dn = take(max_runs * rb_d * sizeof(MoeTile));
    const size_t o_xs = take(static_cast<size_t>(P) * H * 2), o_h = take(static_cast<size_t>(P) * I * 2),
                 o_y = take(static_cast<size_t>(P) * H * 2);
    void* base;
    if ((st = ensure_aux(ctx, off, &base)) != Q38_OK) return st;
    uint8_t* b8 = static_cast<uint8_t*>(base);
    int32_t* perm = reinterpret_cast<int32_t*>(b8 + o_perm);
    int32_t* inv = reinterpret_cast<int32_t*>(b8 + o_inv);
    int32_t* offs = reinterpret_cast<int32_t*>(b8 + o_off);
    int* counts = reinterpret_cast<int*>(b8 + o_cnt);
    MoeTile* gu = reinterpret_cast<MoeTile*>(b8 + o_gu);
    MoeTile* dn = reinterpret_cast<MoeTile*>(b8 + o_dn);
    void* xs = b8 + o_xs;
    void* hp = b8 + o_h;
    void* y = b8 + o_y;

    if ((st = sort_launch(ctx, indices, P, E, perm, offs, inv, reinterpret_cast<int*>(b8 + o_sscr))) != Q38_OK)
        return st;
    if ((st = launch_pdl(ctx, "moe_tiles", moe_tiles_kernel, dim3(1), dim3(1024), 0, offs, static_cast<int>(E), xr,
                         rb_gu, rb_d, gu, dn, counts)) != Q38_OK)
        return st;
    if ((st = moe_gather_launch(ctx, x, static_cast<int>(H), perm, static_cast<int>(P), top_k, offs + E, xs, bits)) !=
        Q38_OK)
        return st;
    GroupedProblem g;
    g.x = xs;
    g.pairs = static_cast<int>(P);
    g.K = static_cast<int>(H);
    g.w0 = gate_w;
    g.w1 = up_w;
    g.s0 = gate_s;
    g.s1 = up_s;
    g.b0 = gate_b;
    g.b1 = up_b;
    g.E = static_cast<int>(E);
    g.rows_per_expert = static_cast<int>(I);
    g.tiles = gu;
    g.ntiles = counts;
    g.max_tiles = static_cast<int>(max_runs * rb_gu);
    g.out = hp;
    g.out_ld = static_cast<int>(I);
    g.xr = xr;
    if ((st = grouped_gate_up(ctx, g, bits)) != Q38_OK) return st;
    GroupedProblem d;
    d.x = hp;
    d.pairs = static_cast<int>(P);
    d.K = static_cast<int>(I);
    d.w0 = down_w;
    d.w1 = down_w;
    d.s0 = down_s;
    d.s1 = down_s;
    d.b0 = down_b;
    d.b1 = down_b;
    d.E = static_cast<int>(E);
    d.rows_per_expert = static_cast<int>(H);
    d.tiles = dn;
    d.ntiles = counts + 1;
    d.max_tiles = static_cast<int>(max_runs * rb_d);
    d.out = y;
    d.out_ld = static_cast<int>(H);
    d.xr = xr;
    if ((st = grouped_down(ctx, d, bits)) != Q38_OK) return st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(T));
    cfg.blockDim = dim3(256);
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, moe_combine_kernel, static_cast<const __nv_bfloat16*>(y), static_cast<int>(H),
                           static_cast<const int32_t*>(inv), indices, static_cast<const __nv_bfloat16*>(scores), top_k,
                           static_cast<int>(E), static_cast<__nv_bfloat16*>(out)) != cudaSuccess)
        return check_launch(ctx, "moe_combine");
    return check_launch(ctx, "moe_combine");
}

q38_status q38_sparse_moe(q38_ctx* ctx, const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int top_k,
                          int normalize, const void* wr, const uint32_t* gate_w, const void* gate_s,
                          const void* gate_b, const uint32_t* up_w, const void* up_s, const void* up_b,
                          const uint32_t* down_w, const void* down_s, const void* down_b, q38_dtype dtype,
                          int group_size, int bits, int32_t* indices, void* scores, void* out) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (T == 0) return Q38_OK;
    if (!indices || !scores) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "sparse_moe: indices and scores are required");
    const bool decode = T <= 16 && H > 0 && static_cast<size_t>(H) * 2 <= 96 * 1024 && E >= 1 && E <= 1024 &&
                        top_k >= 1 && top_k <= 32 && top_k <= E && dtype == Q38_BF16 && x && wr && aligned16(x) &&
                        aligned16(wr) &&
                        qgemv_moe_supported(T, H, I, E, top_k, group_size, bits, x, gate_w, gate_s, gate_b, up_w,
                                            up_s, up_b, down_w, down_s, down_b);
    if (!decode) {
        q38_status st = q38_moe_route(ctx, x, T, H, dtype, wr, E, top_k, normalize, indices, scores, nullptr);
        if (st != Q38_OK) return st;
        return q38_switch_glu(ctx, x, T, H, I, E, top_k, indices, scores, gate_w, gate_s, gate_b, up_w, up_s, up_b,
                              down_w, down_s, down_b, dtype, group_size, bits, out);
    }
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    if ((st = ensure_workspace(ctx, static_cast<size_t>(T) * E * 2)) != Q38_OK) return st;
    if ((st = route_decode_launch(ctx, x, T, H, wr, E, top_k, normalize, ctx->workspace, indices, scores, nullptr)) !=
        Q38_OK)
        return st;
    return qgemv_moe_decode(ctx, x, T, H, I, E, top_k, indices, scores, gate_w, gate_s, gate_b, up_w, up_s, up_b,
                            down_w, down_s, down_b, bits, out);
}

q38_status q38_silu_mul(q38_ctx* ctx, const void* g, const void* u, int64_t n, void* h) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (n < 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "silu_mul: negative size");
    if (n == 0) return Q38_OK;
    if (!g || !u || !h) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "silu_mul: null pointer");
    if (!aligned16(g) || !aligned16(u) || !aligned16(h))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "silu_mul: pointers must be 16-byte aligned");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    const int64_t blocks = (n + 8 * 256 - 1) / (8 * 256);
    return launch_pdl(ctx, "silu_mul", silu_mul_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                      static_cast<const __nv_bfloat16*>(g), static_cast<const __nv_bfloat16*>(u), n,
                      static_cast<__nv_bfloat16*>(h));
}

q38_status q38_moe_dispatch_pack(q38_ctx* ctx, const void* x, int64_t H, const int32_t* indices, const int32_t* perm,
                                 int64_t pairs, int top_k, int64_t experts_per_rank, void* rows,
                                 int32_t* local_experts) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (H <= 0 || H % 8 || top_k < 1 || experts_per_rank < 1 || pairs < 0 || pairs > (1 << 30))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_dispatch_pack: bad sizes");
    if (pairs == 0) return Q38_OK;
    if (!x || !indices || !perm || !rows || !local_experts)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_dispatch_pack: null pointer");
    if (!aligned16(x) || !aligned16(rows)) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_dispatch_pack: rows must be 16-byte aligned");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    return launch_pdl(ctx, "moe_dispatch_pack", moe_pack_kernel, dim3(static_cast<unsigned>(pairs)), dim3(256), 0,
                      static_cast<const __nv_bfloat16*>(x), static_cast<int>(H), indices, perm, pairs, top_k,
                      static_cast<int>(experts_per_rank), static_cast<__nv_bfloat16*>(rows), local_experts);
}

q38_status q38_moe_combine(q38_ctx* ctx, const void* y, int64_t H, const int32_t* perm, const int32_t* indices,
                           const void* scores, int64_t T, int top_k, int64_t E, void* out) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (H <= 0 || H % 8 || T < 0 || top_k < 1 || E < 1)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_combine: bad sizes");
    if (T == 0) return Q38_OK;
    if (!y || !perm || !indices || !scores || !out) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_combine: null pointer");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    const int64_t P = T * top_k;
    void* scratch;
    if ((st = ensure_aux(ctx, static_cast<size_t>(P) * 4, &scratch)) != Q38_OK) return st;
    int32_t* inv = static_cast<int32_t*>(scratch);
    if ((st = launch_pdl(ctx, "moe_combine", invert_perm_kernel, dim3(static_cast<unsigned>((P + 255) / 256)),
                         dim3(256), 0, perm, P, inv)) != Q38_OK)
        return st;
    return launch_pdl(ctx, "moe_combine", moe_combine_kernel, dim3(static_cast<unsigned>(T)), dim3(256), 0,
                      static_cast<const __nv_bfloat16*>(y), static_cast<int>(H), static_cast<const int32_t*>(inv),
                      indices, static_cast<const __nv_bfloat16*>(scores), top_k, static_cast<int>(E),
                      static_cast<__nv_bfloat16*>(out));
}

q38_status q38_moe_ep_plan(q38_ctx* ctx, const int32_t* indices, int64_t T, int top_k, int64_t experts_per_rank,
                           int world, int32_t* rowpos, int32_t* counts) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (T < 0 || top_k < 1 || experts_per_rank < 1 || world < 1 || world > 1024)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_ep_plan: bad sizes");
    if (!indices || !rowpos || !counts) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_ep_plan: null pointer");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    return launch_pdl(ctx, "moe_ep_plan", ep_plan_kernel, dim3(1), dim3(1024), 0, indices, static_cast<int>(T), top_k,
                      static_cast<int>(experts_per_rank), world, rowpos, counts);
}

q38_status q38_moe_ep_pack(q38_ctx* ctx, const void* x, int64_t H, const int32_t* indices, const void* scores,
                           int64_t T, int top_k, int64_t experts_per_rank, int world, const int32_t* rowpos,
                           void* rows, int64_t rows_ld, int32_t* meta, int64_t meta_ld) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (T < 0 || H <= 0 || H % 8 || top_k < 1 || top_k > 256 || experts_per_rank < 1 || world < 1 || rows_ld < H ||
        rows_ld % 8 || meta_ld < 2 * top_k)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_ep_pack: bad sizes or strides");
    if (T == 0) return Q38_OK;
    if (!x || !indices || !scores || !rowpos || !rows || !meta)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_ep_pack: null pointer");
    if (!aligned16(x) || !aligned16(rows)) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_ep_pack: rows must be 16-byte aligned");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    return launch_pdl(ctx, "moe_ep_pack", ep_pack_kernel, dim3(static_cast<unsigned>(T)), dim3(256), 0,
                      static_cast<const __nv_bfloat16*>(x), static_cast<int>(H), indices,
                      static_cast<const __nv_bfloat16*>(scores), top_k, static_cast<int>(experts_per_rank), world,
                      rowpos, static_cast<__nv_bfloat16*>(rows), rows_ld, meta, meta_ld);
}

q38_status q38_moe_ep_reduce(q38_ctx* ctx, const void* partial, int64_t H, const int32_t* rowpos, int64_t T,
                             int world, void* out) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (T < 0 || H <= 0 || H % 8 || world < 1) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_ep_reduce: bad sizes");
    if (T == 0) return Q38_OK;
    if (!partial || !rowpos || !out) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "moe_ep_reduce: null pointer");
    q38_status st = set_dev(ctx);
    if (st != Q38_OK) return st;
    return launch_pdl(ctx, "moe_ep_reduce", ep_reduce_kernel, dim3(static_cast<unsigned>(T)), dim3(256), 0,
                      static_cast<const __nv_bfloat16*>(partial), static_cast<int>(H), rowpos, world,
                      static_cast<__nv_bfloat16*>(out));
}

}  // extern "C"
