/*
 * q38.h -- C ABI of the B200 (sm_100a) MLX-affine quantized matrix-product library.
 *
 * The library replaces the MLX operators that the Qwen3.8 MLX Swift models call for
 * every quantized projection: quantizedMM / gatherQuantizedMM / dequantized /
 * quantize / hadamardTransform, and the QuantizedLinear, QuantizedSwitchLinear and
 * SwitchGLU modules built on them.  Argument meaning follows those operators; the
 * packed layout is MLX's on-disk layout, so checkpoint tensors are passed unchanged:
 *
 *   weight  uint32 [.., N, K*bits/32]   code k of a row at bit k*bits of the row's
 *                                       little-endian bitstream (LSB first)
 *   scales  bf16   [.., N, K/group]     w = scale * q + bias, per group along K
 *   biases  bf16   [.., N, K/group]     (nullable: treated as zero)
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer (cudaMalloc'd, or any memory the
 *     device can address) unless stated otherwise; the caller owns all buffers.
 *   - Every call is enqueued on the context's stream (q38_ctx_set_stream) and returns
 *     without synchronising.  Calls never abort the process: they return a status and
 *     q38_last_error(ctx) describes the most recent failure.
 *   - A context belongs to one device and one host thread at a time; calls on one
 *     context are not re-entrant.  The context owns a device workspace that grows on
 *     demand (the growth itself synchronises the device); q38_ctx_reserve pre-sizes it
 *     so that steady-state calls allocate nothing (and can be captured in a CUDA graph).
 *   - Device kernels never spin without bound: a wait that exceeds about one second
 *     records Q38_ERR_DEVICE_TIMEOUT in the context's device status word, which
 *     q38_ctx_check_device reads.
 */
#ifndef Q38_H
#define Q38_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define Q38_API __declspec(dllexport)
#else
#define Q38_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum q38_status {
    Q38_OK = 0,
    Q38_ERR_INVALID_ARGUMENT = 1, /* shape, pointer or parameter rejected */
    Q38_ERR_UNSUPPORTED = 2,      /* valid MLX arguments this build does not implement */
    Q38_ERR_CUDA = 3,             /* a CUDA runtime call failed */
    Q38_ERR_OUT_OF_MEMORY = 4,    /* workspace growth failed */
    Q38_ERR_DEVICE_TIMEOUT = 5,   /* a bounded device-side wait expired */
    Q38_ERR_COMM = 6              /* a collective failed or timed out */
} q38_status;

typedef enum q38_dtype {
    Q38_BF16 = 0,
    Q38_F16 = 1,
    Q38_F32 = 2
} q38_dtype;

/* MLX QuantizationMode; only .affine is implemented. */
typedef enum q38_mode {
    Q38_MODE_AFFINE = 0
} q38_mode;

typedef struct q38_ctx q38_ctx;

/* ------------------------------------------------------------------ context */

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
Q38_API int q38_version(void);
Q38_API const char* q38_status_string(q38_status status);

/* Create a context on `device` (cudaSetDevice index).  The context starts on the
 * legacy default stream. */
Q38_API q38_status q38_ctx_create(int device, q38_ctx** out);
Q38_API q38_status q38_ctx_destroy(q38_ctx* ctx);
/* `stream` is a cudaStream_t (NULL = legacy default stream). */
Q38_API q38_status q38_ctx_set_stream(q38_ctx* ctx, void* stream);
Q38_API void* q38_ctx_get_stream(const q38_ctx* ctx);
/* Grow the device workspace to at least `bytes` now (synchronises the device). */
Q38_API q38_status q38_ctx_reserve(q38_ctx* ctx, size_t bytes);
Q38_API size_t q38_ctx_workspace_bytes(const q38_ctx* ctx);
/* Reproducible decode products.  A decode-shaped product (M <= 16) splits its reduction
 * dimension over many CTAs; by default their fp32 partial sums are added in arrival order,
 * so two runs of the same product may differ in the last bit of a few outputs.  With
 * `on` != 0 each k-chunk's sums go to a slot of their own and are added in a fixed order:
 * bitwise reproducible results (MLX's decode is reproducible too) for about one
 * microsecond more per product.  Off by default. */
Q38_API q38_status q38_ctx_set_deterministic(q38_ctx* ctx, int on);
/* Pieces of q38_ep_switch_glu's exchange (1, 2 or 4; 0 = chosen by the library): the
 * capacity rows go in that many chunks whose exchanges overlap the experts' work of the
 * previous chunk.  Every rank of a communicator must use the same setting.  Results do not
 * depend on it. */
Q38_API q38_status q38_ctx_set_ep_chunks(q38_ctx* ctx, int chunks);
/* Synchronise the stream and return Q38_ERR_DEVICE_TIMEOUT if any kernel recorded a
 * bounded-wait expiry since the last check (the word is then cleared). */
Q38_API q38_status q38_ctx_check_device(q38_ctx* ctx);
/* Message of the last failed call on this context ("" if none). */
Q38_API const char* q38_last_error(const q38_ctx* ctx);
/* Exercises the timeout path: enqueues a one-thread kernel whose bounded wait (the one
 * every kernel here uses) waits for an mbarrier phase that nothing completes, with a
 * limit of `limit_cycles` SM clock cycles instead of the usual one second.  The wait
 * runs out, the kernel records the expiry in the context's status word and returns, so
 * the next q38_ctx_check_device returns Q38_ERR_DEVICE_TIMEOUT and the context stays
 * usable.  No counterpart in the reference (its MLX kernels have no bounded waits). */
Q38_API q38_status q38_ctx_test_wait_timeout(q38_ctx* ctx, int64_t limit_cycles);

/* ------------------------------------------------------------- operators */

/* quantizedMM -- replaces MLX.quantizedMM(x, w, scales:, biases:, transpose:,
 * groupSize:, bits:, mode:) as called by QuantizedLinear.callAsFunction
 * (Sources/Qwen38Core/FlashNext/Qwen4ExpPrequantized.swift:156-159; packed shapes built
 * at :77-106).  transpose != 0: y[M,N] = x[M,K] . dequant(w)[N,K]^T with w uint32
 * [N, K*bits/32] and scales/biases [N, K/group_size].  x and y share `x_dtype`
 * (bf16 or f16); scales/biases use `scales_dtype`.  Accumulation is fp32.
 * bits in {2,3,4,5,6,8}; group_size in {32,64,128}; transpose == 0 is rejected with
 * Q38_ERR_UNSUPPORTED (no call site in the reference uses it). */
Q38_API q38_status q38_quantized_matmul(q38_ctx* ctx, const void* x, int64_t M, int64_t K,
                                q38_dtype x_dtype, const uint32_t* w, const void* scales,
                                const void* biases, q38_dtype scales_dtype, int64_t N,
                                int transpose, int group_size, int bits, q38_mode mode,
                                void* y);

/* gatherQuantizedMM -- replaces MLX.gatherQuantizedMM(x, w, scales:, biases:,
 * lhsIndices:, rhsIndices:, transpose:, groupSize:, bits:, sortedIndices:) behind
 * QuantizedSwitchLinear.callAsFunction (Vendor/mlx-swift-lm-local.patch:184-218):
 * out[p] (M x N) = x[lhs[p]] (M x K) . dequant(w[rhs[p]])^T for p < P, with
 * x [Bx, M, K], w [E, N, K*bits/32], scales/biases [E, N, K/group_size], out [P, M, N].
 * lhs_indices may be NULL (lhs[p] = p, requires Bx >= P).  sorted_indices is MLX's hint
 * that rhs is non-decreasing; results do not depend on it.  Indices are int32. */
Q38_API q38_status q38_gather_quantized_matmul(q38_ctx* ctx, const void* x, int64_t Bx, int64_t M,
                                       int64_t K, q38_dtype x_dtype, const uint32_t* w,
                                       const void* scales, const void* biases,
                                       q38_dtype scales_dtype, int64_t E, int64_t N,
                                       const int32_t* lhs_indices, const int32_t* rhs_indices,
                                       int64_t P, int transpose, int group_size, int bits,
                                       q38_mode mode, int sorted_indices, void* out);

/* dequantized -- replaces MLX.dequantized(w, scales:, biases:, groupSize:, bits:, mode:)
 * (Sources/Qwen38Core/FlashNext/Qwen4ExpCheckpointLayerLoader.swift:299-305,
 * Qwen4ExpPrequantized.swift:146-151): out[rows, K] = scale*q + bias, computed in fp32
 * and stored as `out_dtype` (round to nearest even for bf16/f16). */
Q38_API q38_status q38_dequantize(q38_ctx* ctx, const uint32_t* w, const void* scales,
                          const void* biases, q38_dtype scales_dtype, int64_t rows, int64_t K,
                          int group_size, int bits, q38_mode mode, void* out,
                          q38_dtype out_dtype);

/* quantize -- replaces mx.quantize(w, group_size:, bits:, mode: "affine")
 * (Scripts/qwen4-exp-requantize-experts.py:246-251): w [rows, K] of `w_dtype` ->
 * codes uint32 [rows, K*bits/32], scales/biases [rows, K/group_size] of `scales_dtype`.
 * Per group the larger-magnitude extreme is represented exactly (MLX affine rule). */
Q38_API q38_status q38_quantize(q38_ctx* ctx, const void* w, q38_dtype w_dtype, int64_t rows,
                        int64_t K, int group_size, int bits, q38_mode mode, uint32_t* codes,
                        void* scales, void* biases, q38_dtype scales_dtype);

/* Unpacked integer codes q[rows, K] (one byte each) of a packed weight; the
 * bit-exactness probe of the packed format. */
Q38_API q38_status q38_unpack_codes(q38_ctx* ctx, const uint32_t* w, int64_t rows, int64_t K, int bits,
                            uint8_t* q);

/* hadamardRotate -- replaces the rotation of Qwen38HadamardQuantizedLinear /
 * Qwen38HadamardQuantizedEmbedding (Sources/Qwen38Core/Bonsai2/
 * Qwen38HadamardModules.swift:10-19): fp32(x) * signs (forward) or signs applied after
 * the transform (inverse), normalised Walsh-Hadamard transform (Sylvester order) over
 * blocks of `block` along the last axis, scaled by 1/sqrt(block), cast back to x_dtype.
 * x, y [rows, D]; signs fp32 [D] or NULL (all +1); block a power of two <= 8192. */
Q38_API q38_status q38_hadamard_rotate(q38_ctx* ctx, const void* x, int64_t rows, int64_t D,
                               q38_dtype x_dtype, const float* signs, int block, int inverse,
                               void* y);

/* Qwen38HadamardQuantizedLinear.callAsFunction (Bonsai2/Qwen38HadamardModules.swift:37-39):
 * y = quantizedMM(hadamardRotate(x, signs, block), w, ...).  The rotated activations
 * are rounded to x_dtype before the product, as in the reference. */
Q38_API q38_status q38_hadamard_quantized_matmul(q38_ctx* ctx, const void* x, int64_t M, int64_t K,
                                         q38_dtype x_dtype, const float* signs, int block,
                                         const uint32_t* w, const void* scales,
                                         const void* biases, q38_dtype scales_dtype, int64_t N,
                                         int group_size, int bits, void* y);

/* ------------------------------------------------------------------ sparse MoE layer
 * Replaces the pieces of Qwen4ExpSparseMoE.callAsFunction
 * (Sources/Qwen38Core/FlashNext/Qwen4ExpSparseMoE.swift:275-294): the router (gate Linear,
 * softmax(precise:), argPartition, takeAlong, renormalisation, :208-214 and :275-281), the
 * SwitchGLU's sort of (token, slot) pairs by expert, and SwitchGLU + weightedExpertSum
 * (:294, built at :225-232) over QuantizedSwitchLinear gate/up/down projections
 * (Vendor/mlx-swift-lm-local.patch:184-218). */

/* Router: logits = bf16(x . wr^T) (fp32 accumulation), probs = bf16(softmax_fp32(logits)),
 * the top_k experts per token in canonical order (probability descending, expert id
 * ascending on ties), scores = probs[indices], divided by bf16(sum of the k scores) when
 * normalize != 0.  x bf16 [T, H], wr bf16 [E, H] (H % 64 == 0, E <= 1024, top_k <= 32);
 * indices int32 [T, top_k]; scores bf16 [T, top_k]; probs bf16 [T, E] or NULL. */
Q38_API q38_status q38_moe_route(q38_ctx* ctx, const void* x, int64_t T, int64_t H, q38_dtype x_dtype,
                                 const void* wr, int64_t E, int top_k, int normalize, int32_t* indices,
                                 void* scores, void* probs);

/* The same selection from given bf16 logits [T, E]. */
Q38_API q38_status q38_moe_route_logits(q38_ctx* ctx, const void* logits, int64_t T, int64_t E, int top_k,
                                        int normalize, int32_t* indices, void* scores, void* probs);

/* Stable sort of the `pairs` flat (token, slot) entries of `indices` by expert:
 * perm[j] = flat index of the j-th pair in expert order (pairs of one expert in flat
 * order), offsets[E + 1] = start of each expert's run (offsets[E] = number of valid pairs).
 * Indices outside [0, E) are placed after all experts and reported by
 * q38_ctx_check_device as an invalid argument. */
Q38_API q38_status q38_moe_sort(q38_ctx* ctx, const int32_t* indices, int64_t pairs, int64_t E, int32_t* perm,
                                int32_t* offsets);

/* SwitchGLU + weightedExpertSum: for every token t and slot s with expert e = indices[t, s]
 *   g = bf16(x_t . Wg[e]^T), u = bf16(x_t . Wu[e]^T), h = bf16(silu(g) * u),
 *   y_ts = bf16(h . Wd[e]^T), out_t = bf16(sum_s scores[t, s] * y_ts).
 * x bf16 [T, H]; indices int32 / scores bf16 [T, top_k]; gate/up codes [E, I, H*bits/32],
 * scales/biases bf16 [E, I, H/64]; down codes [E, H, I*bits/32], scales/biases
 * [E, H, I/64]; out bf16 [T, H].  Biases are given for all three projections or none.
 * An index of -1 marks an empty slot: it contributes nothing and is not an error.
 * Implemented for group 64, bits 2/3/4/8, H % 512 == 0, I % 512 == 0, E <= 1024.  Up to 16
 * tokens (with T*top_k <= 256) stream the selected experts' weights on the decode kernel;
 * more tokens run the grouped tensor-core products over expert-sorted pairs.  Uses the
 * context's activation buffer (about
 * T*top_k*(2H + I)*2 bytes) and workspace. */
Q38_API q38_status q38_switch_glu(q38_ctx* ctx, const void* x, int64_t T, int64_t H, int64_t I, int64_t E,
                                  int top_k, const int32_t* indices, const void* scores,
                                  const uint32_t* gate_w, const void* gate_scales, const void* gate_biases,
                                  const uint32_t* up_w, const void* up_scales, const void* up_biases,
                                  const uint32_t* down_w, const void* down_scales, const void* down_biases,
                                  q38_dtype dtype, int group_size, int bits, void* out);

/* The routed-expert layer in one call: q38_moe_route (x, router weight wr [E, H]) then
 * q38_switch_glu, the pair Qwen4ExpSparseMoE.callAsFunction runs
 * (Sources/Qwen38Core/FlashNext/Qwen4ExpSparseMoE.swift:275-294).  indices [T, top_k]
 * (int32) and scores [T, top_k] (bf16) receive the routing.  Results equal the two calls
 * made separately, bit for bit. */
Q38_API q38_status q38_sparse_moe(q38_ctx* ctx, const void* x, int64_t T, int64_t H, int64_t I, int64_t E,
                                  int top_k, int normalize, const void* wr, const uint32_t* gate_w,
                                  const void* gate_scales, const void* gate_biases, const uint32_t* up_w,
                                  const void* up_scales, const void* up_biases, const uint32_t* down_w,
                                  const void* down_scales, const void* down_biases, q38_dtype dtype, int group_size,
                                  int bits, int32_t* indices, void* scores, void* out);

/* The shared-expert half of the sparse-MoE block, added to the routed output: the `shared`
 * term of Qwen4ExpSparseMoE.callAsFunction (Sources/Qwen38Core/FlashNext/Qwen4ExpSparseMoE.swift:295-298)
 * with Qwen4ExpSharedExpert (:47-82):
 *   h = bf16(silu(bf16(x . Wg^T)) * bf16(x . Wu^T)), ys = bf16(h . Wd^T),
 *   s = bf16(sigmoid(bf16(x . Wsg^T))), out = bf16(routed + bf16(s * ys)).
 * x, routed, out bf16 [T, H] (routed and out may be the same buffer); gate/up codes
 * [I, H*bits/32], down [H, I*bits/32], the shared-expert gate Wsg [1, H*bits/32]; scales and
 * biases [rows, K/group_size] of scales_dtype, all four projections with the same group
 * size and bits (the published checkpoint quantizes them 4-bit, group 32).  Gate and up
 * carry biases both or neither.  Uses the context's activation buffer (T*(2I + H)*2
 * bytes) and workspace. */
Q38_API q38_status q38_shared_expert(q38_ctx* ctx, const void* x, int64_t T, int64_t H, int64_t I,
                                     const uint32_t* gate_w, const void* gate_scales, const void* gate_biases,
                                     const uint32_t* up_w, const void* up_scales, const void* up_biases,
                                     const uint32_t* down_w, const void* down_scales, const void* down_biases,
                                     const uint32_t* sgate_w, const void* sgate_scales, const void* sgate_biases,
                                     q38_dtype scales_dtype, int group_size, int bits, const void* routed,
                                     void* out);

/* h = bf16(silu(g) * u) elementwise with silu(g) = g / (1 + exp(-g)) in fp32: the
 * SiLU-gate between the gate/up and down projections of the dense MLP (MLX's compiled
 * silu product).  g, u, h bf16 [n], 16-byte aligned. */
Q38_API q38_status q38_silu_mul(q38_ctx* ctx, const void* g, const void* u, int64_t n, void* h);

/* Expert-parallel dispatch (experts split contiguously, experts_per_rank per rank): for
 * j < pairs, rows[j] = x[perm[j] / top_k] (bf16 [*, H]) and local_experts[j] =
 * indices[perm[j]] % experts_per_rank, where perm orders the flat (token, slot) pairs by
 * destination rank (q38_moe_sort of indices / experts_per_rank). */
Q38_API q38_status q38_moe_dispatch_pack(q38_ctx* ctx, const void* x, int64_t H, const int32_t* indices,
                                         const int32_t* perm, int64_t pairs, int top_k, int64_t experts_per_rank,
                                         void* rows, int32_t* local_experts);

/* weightedExpertSum over expert outputs held in dispatch order: out_t = bf16(sum_s
 * scores[t, s] * y[j(t, s)]) in slot order, j(t, s) the position of pair t*top_k + s in
 * perm.  Pairs whose index is outside [0, E) contribute nothing. */
Q38_API q38_status q38_moe_combine(q38_ctx* ctx, const void* y, int64_t H, const int32_t* perm,
                                   const int32_t* indices, const void* scores, int64_t T, int top_k, int64_t E,
                                   void* out);

/* Expert-parallel exchange with one row per (token, destination rank).  Experts are split
 * contiguously, experts_per_rank per rank.
 *   q38_moe_ep_plan: rowpos[t * world + r] = the row token t sends to rank r (rank-major,
 *     tokens ascending within a rank), or -1 when none of its experts lives on r;
 *     counts[r] = rows for rank r.  One block; indices int32 [T, top_k].
 *   q38_moe_ep_pack: rows[rowpos] = x[t] (bf16, row stride rows_ld >= H, a multiple of 8);
 *     meta (int32, row stride meta_ld >= 2 * top_k) = the rank-local expert of each slot
 *     or -1 (expert elsewhere), then the slot scores' bf16 bits.  meta may point into the
 *     rows buffer (at column H) so that one exchange moves both.  The receiving rank runs q38_switch_glu on the rows with those indices
 *     and scores (slots of -1 contribute nothing), which yields each row's partial sum.
 *   q38_moe_ep_reduce: out[t] = bf16(sum over r, in rank order, of partial[rowpos[t, r]])
 *     with fp32 accumulation. */
Q38_API q38_status q38_moe_ep_plan(q38_ctx* ctx, const int32_t* indices, int64_t T, int top_k,
                                   int64_t experts_per_rank, int world, int32_t* rowpos, int32_t* counts);
Q38_API q38_status q38_moe_ep_pack(q38_ctx* ctx, const void* x, int64_t H, const int32_t* indices, const void* scores,
                                   int64_t T, int top_k, int64_t experts_per_rank, int world, const int32_t* rowpos,
                                   void* rows, int64_t rows_ld, int32_t* meta, int64_t meta_ld);
Q38_API q38_status q38_moe_ep_reduce(q38_ctx* ctx, const void* partial, int64_t H, const int32_t* rowpos, int64_t T,
                                     int world, void* out);

/* Quantized embedding lookup: out[t, :] = dequant(w, scales, biases)[ids[t], :] for
 * t < n, the Qwen4ExpPrequantizedEmbedding.callAsFunction of
 * Sources/Qwen38Core/FlashNext/Qwen4ExpPrequantized.swift:141-151 (rows gathered, then
 * MLX.dequantized).  w [rows, K*bits/32] packed, scales/biases [rows, K/group_size];
 * each output row equals that row of q38_dequantize bit for bit.  An id outside
 * [0, rows) gives a zero row and is reported by q38_ctx_check_device.  The tied output
 * projection (asLinear, :154-158) is q38_quantized_matmul with the same tensors. */
Q38_API q38_status q38_quantized_embedding(q38_ctx* ctx, const int32_t* ids, int64_t n, const uint32_t* w,
                                           const void* scales, const void* biases, q38_dtype scales_dtype,
                                           int64_t rows, int64_t K, int group_size, int bits, q38_mode mode,
                                           void* out, q38_dtype out_dtype);

/* Rotated quantized embedding lookup (Bonsai 2 packs): the
 * Qwen38HadamardQuantizedEmbedding.callAsFunction of
 * Sources/Qwen38Core/Bonsai2/Qwen38HadamardModules.swift:71-79.  Each row of ids is
 * dequantized into the scales' dtype (bf16 or f16), then rotated back:
 * out = cast(signs * H_block(row) / sqrt(block)) in fp32 with the block-diagonal
 * Walsh-Hadamard transform H over blocks of `block` (a power of two in [2, 8192] that
 * divides K), signs (fp32 [K], may be NULL) applied after the transform (hadamardRotate
 * with inverse = true, :10-19).  out [n, K] has the scales' dtype and equals
 * q38_quantized_embedding followed by q38_hadamard_rotate(inverse = 1) bit for bit.  An
 * id outside [0, rows) gives the rotation of a zero row (zeros) and is reported by
 * q38_ctx_check_device. */
Q38_API q38_status q38_hadamard_quantized_embedding(q38_ctx* ctx, const int32_t* ids, int64_t n, const uint32_t* w,
    const void* scales, const void* biases, q38_dtype scales_dtype, int64_t rows, int64_t K, int group_size,
    int bits, q38_mode mode, const float* signs, int block, void* out);

/* Gate and up projections of a gated MLP in one call:
 *   h[M, N] = bf16( silu(bf16(x . dequant(Wg)^T)) * bf16(x . dequant(Wu)^T) ),
 * the `silu(gate(x)) * up(x)` of the reference's MLPs (the fused gate/up pattern of
 * Sources/Qwen38Core/FlashNext/Qwen4ExpFusion.swift:158-186; the shared expert and the
 * dense Qwen3.5 MLP), with the rounding of two bf16 QuantizedLinear outputs followed by the
 * SiLU product.  Wg and Wu are two packed weights of the same shape [N, K*bits/32] with
 * their own scales/biases (both biased or neither).  For M <= 16 tokens (decode) one
 * streaming pass reads both weights and applies the SiLU-gate in its epilogue; larger M
 * runs the two products and the SiLU product in sequence. */
Q38_API q38_status q38_quantized_gate_up(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype x_dtype,
                                         const uint32_t* w_gate, const void* s_gate, const void* b_gate,
                                         const uint32_t* w_up, const void* s_up, const void* b_up,
                                         q38_dtype scales_dtype, int64_t N, int group_size, int bits,
                                         q38_mode mode, void* h);

/* Gate and up projections of a Bonsai 2 MLP from one rotation of x: h = bf16(silu(bf16(
 * xr.Wg^T)) * bf16(xr.Wu^T)) with xr = hadamardRotate(x, signs, block) rounded to bf16.  The
 * reference applies Qwen38HadamardQuantizedLinear to gate and up separately
 * (Sources/Qwen38Core/Bonsai2/Qwen38HadamardModules.swift:37-39, signs before the transform);
 * the pack stores the same signs for every module of one input width, so the two rotations
 * are one, and the products take one pass over both weights where the decode kernel takes
 * the layout (M <= 16: bf16 scales in groups of 64, or the pack's f16 scales in groups of
 * 128 with K % 1024 == 0).  Callers whose gate and up signs differ call
 * q38_hadamard_quantized_matmul twice instead.  Arguments as q38_quantized_gate_up and
 * q38_hadamard_rotate. */
Q38_API q38_status q38_hadamard_quantized_gate_up(q38_ctx* ctx, const void* x, int64_t M, int64_t K,
    q38_dtype x_dtype, const float* signs, int block, const uint32_t* w_gate, const void* s_gate, const void* b_gate,
    const uint32_t* w_up, const void* s_up, const void* b_up, q38_dtype scales_dtype, int64_t N, int group_size,
    int bits, void* h);

/* Allocation-free decode product.  No counterpart in the reference: it exists for
 * callers that must not allocate device memory on the calling path (a host framework
 * that owns all device memory and hands a plugin only its input and output buffers, or
 * a latency-critical decode loop where an allocation would stall or fail).  Same
 * product as q38_quantized_matmul (transpose = true, affine, group 64, bits 2/3/4/8,
 * bf16 x/y/scales/biases, 16-byte-aligned pointers; biases may be NULL) with no
 * context: it runs on the calling thread's current device and on `stream` (a
 * cudaStream_t, NULL = legacy default stream).  Its scratch is one fixed 2 MiB array in
 * device memory that the library holds on every GPU it is loaded on until the process
 * exits, so the limits are M <= 16, N <= 32768, K <= 32768 (K % 512 == 0); larger
 * shapes return Q38_ERR_INVALID_ARGUMENT.  The first call on a device (and the first
 * after the device's context was re-created, e.g. after cudaDeviceReset) resolves the
 * array's address and clears it, which synchronises the device: make that first call
 * before any stream capture.  Later calls clear nothing (each product returns its
 * partial sums to zero).  All calls on a device share the one array: calls that may
 * overlap on the GPU (different streams without ordering between them) race and
 * produce wrong results.  Returns a status only; there is no context to hold an error
 * message.  A device-side wait that runs out is not visible in the returned status
 * (the call returns before the kernels run): q38_noalloc_check_device reports it. */
Q38_API q38_status q38_quantized_matmul_noalloc(const void* x, int64_t M, int64_t K,
                                                const uint32_t* w, const void* scales,
                                                const void* biases, int64_t N, int group_size,
                                                int bits, void* y, void* stream);

/* Companion of q38_quantized_matmul_noalloc, also without allocation or context:
 * synchronises `stream`, then reads and clears the status word in the fixed array of the
 * current device.  Returns Q38_ERR_DEVICE_TIMEOUT if a bounded device-side wait of an
 * allocation-free product ran out since the last check (that product's y is then not
 * valid), else Q38_OK.  No counterpart in the reference. */
Q38_API q38_status q38_noalloc_check_device(void* stream);

/* ------------------------------------------------------------- multi-GPU
 * One communicator rank per GPU over NCCL (NVLink / NVSwitch), loaded at run time
 * (libnccl.so.2; Q38_NCCL_LIBRARY names another copy).  These replace the single-device
 * calls of the reference's model code (FlashNext/Qwen4ExpSparseMoE.swift:275-294 for the
 * experts, FlashNext/Qwen4ExpPrequantized.swift:156-159 for the dense MLP's projections)
 * when the weights are sharded over several GPUs; the reference itself runs on one
 * device.  Every collective is enqueued on the context's stream (or on the communicator's
 * own stream, joined back to it) and never synchronises the host. */
typedef struct q38_comm q38_comm;
typedef struct q38_comm_id {
    unsigned char bytes[128];
} q38_comm_id;

/* Message of the last failed communicator call on this thread. */
Q38_API const char* q38_comm_error(void);
/* A fresh rendezvous id; rank 0 creates it and hands it to the other ranks (any host
 * channel).  Needs no GPU. */
Q38_API q38_status q38_comm_get_unique_id(q38_comm_id* id);
/* Joins rank `rank` of `world` on `device`.  Non-blocking under the hood: if the other
 * ranks have not all joined within `timeout_ms`, the communicator is aborted and
 * Q38_ERR_COMM is returned (q38_comm_error says why); later collectives on a
 * communicator also give up with Q38_ERR_COMM after `timeout_ms` without progress. */
Q38_API q38_status q38_comm_init_rank(const q38_comm_id* id, int world, int rank, int device, int timeout_ms,
                                      q38_comm** out);
/* All ranks of one process, one per device in `devices` (a host that drives every GPU
 * from one thread). */
Q38_API q38_status q38_comm_init_all(int ndev, const int* devices, int timeout_ms, q38_comm** comms);
Q38_API q38_status q38_comm_destroy(q38_comm* comm);
/* Aborts the communicator's collectives (after a peer failed); destroy it afterwards. */
Q38_API q38_status q38_comm_abort(q38_comm* comm);
Q38_API int q38_comm_rank(const q38_comm* comm);
Q38_API int q38_comm_size(const q38_comm* comm);
/* Sum of `count` elements over all ranks (recv may equal send), on the context's stream. */
Q38_API q38_status q38_comm_all_reduce(q38_ctx* ctx, q38_comm* comm, const void* send, void* recv, int64_t count,
                                       q38_dtype dtype);

/* Tensor-parallel gated MLP, y[M, D] = down(silu(gate(x)) * up(x)) summed over the ranks:
 * each rank holds gate and up split by output rows (F_local rows of [F, D*bits/32]) and
 * down split by its reduction dimension ([D, F_local*bits/32], whole groups and words),
 * computes its partial y and all-reduces it (bf16 sum).  h = silu(gate) * up is formed for
 * all tokens in one pass; the down projection then runs in `chunks` pieces of whole
 * 128-token tiles, the all-reduce of one piece on the communicator's stream while the next
 * piece computes; chunks <= 0 picks the count (1 to 4) that keeps two waves of tensor-core
 * tiles in each piece.  x, y bf16 [M, D] on every rank. */
Q38_API q38_status q38_tp_mlp(q38_ctx* ctx, q38_comm* comm, const void* x, int64_t M, int64_t D,
                              const uint32_t* gate_w, const void* gate_s, const void* gate_b,
                              const uint32_t* up_w, const void* up_s, const void* up_b,
                              const uint32_t* down_w, const void* down_s, const void* down_b, int64_t F_local,
                              q38_dtype dtype, int group_size, int bits, int chunks, void* y);

/* Expert-parallel SwitchGLU + weightedExpertSum (q38_switch_glu's arithmetic) with the E
 * experts split contiguously over the ranks (this rank holds experts [rank*E/world,
 * (rank+1)*E/world): gate/up [E/world, I, H*bits/32], down [E/world, H, I*bits/32]).  x
 * [T, H], indices/scores [T, top_k] (global expert ids, from this rank's router) and out
 * [T, H] are this rank's tokens.  Fixed capacity: every rank contributes `capacity` rows
 * (T <= capacity, the same capacity on every rank; rows past T carry empty slots), so the
 * exchange sizes are known in advance and nothing is read back to the host (the call can
 * be captured in a CUDA graph).  The rows, slot experts and scores of all ranks are
 * all-gathered; each rank runs its own experts over every row (the slots of other ranks'
 * experts are empty), and a bf16 reduce-scatter sums the ranks' partial outputs into each
 * token's home rank: out_t = the sum over ranks of bf16(sum of that rank's slots), added
 * in NCCL's order. */
Q38_API q38_status q38_ep_switch_glu(q38_ctx* ctx, q38_comm* comm, const void* x, int64_t T, int64_t H, int64_t I,
                                     int64_t E, int top_k, const int32_t* indices, const void* scores,
                                     const uint32_t* gate_w, const void* gate_s, const void* gate_b,
                                     const uint32_t* up_w, const void* up_s, const void* up_b,
                                     const uint32_t* down_w, const void* down_s, const void* down_b,
                                     q38_dtype dtype, int group_size, int bits, int64_t capacity, void* out);

/* ------------------------------------------------------------- safetensors */

/* Checkpoint reader.  MLX checkpoints are safetensors files whose packed tensors
 * (`<module>.weight` U32, `.scales` and `.biases` BF16/F16, Bonsai 2 `.signs` F32) are
 * already the layout these operators take, so loading is a copy: the reference attaches
 * them with loadArrays (Sources/Qwen38Core/FlashNext/Qwen4ExpCheckpointLayerLoader.swift:74,
 * Sources/Qwen38Core/Bonsai2/Qwen38Bonsai2Container.swift:30) and this reader replaces that
 * step.  The file is mapped read-only; its header is parsed and checked (known dtypes,
 * sizes that match the shapes, byte ranges that tile the data buffer exactly).  Host
 * functions need no context or device; the pointers they return are host pointers into
 * the mapping and stay valid until q38_st_close.  A handle may be shared by threads. */
typedef struct q38_st_file q38_st_file;

/* Opens and validates `path`.  On failure returns Q38_ERR_INVALID_ARGUMENT and
 * q38_st_open_error() (per thread) says why. */
Q38_API q38_status q38_st_open(const char* path, q38_st_file** out);
Q38_API const char* q38_st_open_error(void);
Q38_API void q38_st_close(q38_st_file* f);
/* Tensors in header order; q38_st_find returns the index of `name` or -1. */
Q38_API int64_t q38_st_count(const q38_st_file* f);
Q38_API int64_t q38_st_find(const q38_st_file* f, const char* name);
/* name and dtype ("U32", "BF16", "F16", "F32", ... as written in the file) are owned by
 * the handle; shape needs room for 8 entries.  Any output may be NULL. */
Q38_API q38_status q38_st_info(const q38_st_file* f, int64_t i, const char** name, const char** dtype, int* ndim,
                               int64_t* shape, uint64_t* nbytes);
/* Host address of tensor i's bytes inside the mapping. */
Q38_API const void* q38_st_data(const q38_st_file* f, int64_t i);
/* The header's "__metadata__" string map, in file order. */
Q38_API int64_t q38_st_metadata_count(const q38_st_file* f);
Q38_API q38_status q38_st_metadata_entry(const q38_st_file* f, int64_t i, const char** key, const char** value);
/* Copies tensor i (all nbytes of it; dst_bytes >= nbytes) to the device buffer dst,
 * enqueued on the context's stream through pinned staging owned by the context.  The
 * call returns once the host has handed every byte to a copy; the copies complete in
 * stream order. */
Q38_API q38_status q38_st_copy_to_device(q38_ctx* ctx, const q38_st_file* f, int64_t i, void* dst,
                                         uint64_t dst_bytes);
/* Copies a 2-D block of tensor i seen as rows of row_bytes bytes: rows [row0, row0+rows)
 * and bytes [col_byte0, col_byte0+col_bytes) of each row, to dst with row pitch dst_pitch.
 * A tensor-parallel shard loads this way without the rest of the tensor: output rows of
 * a packed weight are whole rows; a shard of its reduction dimension is a byte range of
 * each row (whole 32-bit words of codes, whole groups of scales and biases). */
Q38_API q38_status q38_st_copy_block_to_device(q38_ctx* ctx, const q38_st_file* f, int64_t i, uint64_t row_bytes,
                                               uint64_t row0, uint64_t rows, uint64_t col_byte0, uint64_t col_bytes,
                                               void* dst, uint64_t dst_pitch);

#ifdef __cplusplus
}
#endif
#endif /* Q38_H */
