/*
 * q38_oracle.h -- CPU restatement of the MLX affine-quantized matrix-product path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA library
 * (libq38.so) and the timed CPU baseline; it is never linked into, loaded by or
 * called from the product path.
 *
 * Parity status: the packed bit order and dequantization for bits 2/4/8 are
 * pinned against an independent implementation of the same MLX packed format
 * (tests/golden/make_golden.py); the 3-bit bitstream order, the quantizer's
 * scale/bias selection and the qmm numerics against MLX itself are UNPINNED
 * (no MLX build can run in this environment).  Every function cites the
 * reference call site whose semantics it restates.
 *
 * Conventions: bf16 values travel as uint16_t bit patterns; rounding to bf16
 * is round-to-nearest-even.  Packed codes are row-major [rows, K*bits/32]
 * uint32 words; scales/biases are row-major [rows, K/group] bf16.
 */
#ifndef Q38_ORACLE_H
#define Q38_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float q38o_bf16_to_f32(uint16_t h);
uint16_t q38o_f32_to_bf16(float f);

/* Number of worker threads used by the parallel entry points (0 = all cores). */
void q38o_set_threads(int n);
int q38o_get_threads(void);

/* Unpack codes [rows, K*bits/32] -> q [rows, K] (one byte per code). */
int q38o_unpack(const uint32_t* codes, int64_t rows, int64_t K, int bits, uint8_t* q);
/* Pack q [rows, K] -> codes [rows, K*bits/32]. */
int q38o_pack(const uint8_t* q, int64_t rows, int64_t K, int bits, uint32_t* codes);

/* MLX affine quantize of w [rows, K] (fp32 values) -> codes, bf16 scales and biases. */
int q38o_quantize(const float* w, int64_t rows, int64_t K, int group, int bits,
                  uint32_t* codes, uint16_t* scales, uint16_t* biases);

/* Dequantize -> fp32 [rows, K]: w = scale*q + bias (scale/bias widened from bf16). */
int q38o_dequantize(const uint32_t* codes, const uint16_t* scales, const uint16_t* biases,
                    int64_t rows, int64_t K, int group, int bits, float* w);

/* y[M,N] (bf16) = x[M,K] (bf16) . dequant(w)[N,K]^T, fp32 accumulation. */
int q38o_qmm(const uint16_t* x, int64_t M, int64_t K, const uint32_t* codes,
             const uint16_t* scales, const uint16_t* biases, int64_t N, int group,
             int bits, uint16_t* y);

/* Same product with fp32 output (no final bf16 rounding); used for error budgets. */
int q38o_qmm_f32(const uint16_t* x, int64_t M, int64_t K, const uint32_t* codes,
                 const uint16_t* scales, const uint16_t* biases, int64_t N, int group,
                 int bits, float* y);

/* gatherQuantizedMM: out[p] (M x N, bf16) = x[lhs[p]] (M x K) . dequant(w[rhs[p]])^T.
 * x: [Bx, M, K]; w codes: [E, N, K*bits/32]; scales/biases: [E, N, K/group];
 * lhs may be NULL (then lhs[p] = p). */
int q38o_gather_qmm(const uint16_t* x, int64_t Bx, int64_t M, int64_t K,
                    const uint32_t* codes, const uint16_t* scales, const uint16_t* biases,
                    int64_t E, int64_t N, int group, int bits,
                    const int32_t* lhs, const int32_t* rhs, int64_t P, uint16_t* out);

/* Router: logits = bf16(x . Wr^T) with Wr [E, H] bf16, probs = bf16(softmax_fp32(logits)),
 * top-k in canonical order (probability descending, expert id ascending on ties),
 * scores = probs[idx], renormalised when normalize != 0.  probs_out may be NULL. */
int q38o_moe_route(const uint16_t* x, int64_t T, int64_t H, const uint16_t* wr, int64_t E,
                   int top_k, int normalize, int32_t* indices, uint16_t* scores,
                   uint16_t* probs_out);
/* Same selection from given bf16 logits [T, E] (isolates top-k from the logits product). */
int q38o_route_from_logits(const uint16_t* logits, int64_t T, int64_t E, int top_k,
                           int normalize, int32_t* indices, uint16_t* scores,
                           uint16_t* probs_out);

/* Stable sort of the T*k (token, slot) pairs by expert: perm[j] = flat pair index,
 * offsets[E+1] = start of each expert's run. */
int q38o_sort_by_expert(const int32_t* indices, int64_t pairs, int64_t E, int32_t* perm,
                        int32_t* offsets);

/* SwitchGLU + weightedExpertSum:
 *   g = bf16(x_t . Wg[e]^T), u = bf16(x_t . Wu[e]^T), h = bf16(silu(g) * u),
 *   y_tk = bf16(h . Wd[e]^T), out_t = bf16(sum_k score_tk * y_tk).
 * x [T,H]; indices/scores [T,k]; gate/up codes [E, I, H*bits/32], scales [E, I, H/group];
 * down codes [E, H, I*bits/32], scales [E, H, I/group].
 * weights_bf16 != 0 rounds every dequantized weight s*q + b once to bf16 (the operand of
 * a bf16 tensor-core product) instead of evaluating it in fp32.  An index of -1 marks an
 * empty slot that contributes nothing. */
int q38o_switch_glu(const uint16_t* x, int64_t T, int64_t H, int64_t I, int64_t E, int top_k,
                    const int32_t* indices, const uint16_t* scores,
                    const uint32_t* gw, const uint16_t* gs, const uint16_t* gb,
                    const uint32_t* uw, const uint16_t* us, const uint16_t* ub,
                    const uint32_t* dw, const uint16_t* ds, const uint16_t* db,
                    int group, int bits, int weights_bf16, uint16_t* out);

/* hadamardRotate: y = bf16( FWHT_block( fp32(x) * signs ) / sqrt(block) ) (forward), or
 * signs applied after the transform (inverse).  signs may be NULL (all +1). */
int q38o_hadamard_rotate(const uint16_t* x, int64_t rows, int64_t D, const float* signs,
                         int block, int inverse, uint16_t* y);

/* Sample generators shared by the tests and the benchmark (SplitMix64 + Box-Muller). */
void q38o_fill_normal_bf16(uint64_t seed, float stddev, uint16_t* out, int64_t n);
void q38o_fill_normal_f32(uint64_t seed, float stddev, float* out, int64_t n);
/* Bonsai-style ternary weights: q uniform in {0,1,2}, scale = |N(0, sd^2)|, bias = -scale. */
void q38o_fill_ternary(uint64_t seed, float stddev, int64_t rows, int64_t K, int group,
                       uint32_t* codes, uint16_t* scales, uint16_t* biases);

#ifdef __cplusplus
}
#endif
#endif
