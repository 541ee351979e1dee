/*
 * q38_oracle.c -- CPU restatement of the MLX affine-quantized matrix-product path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library and the timed CPU
 * baseline.  Nothing in the product links, loads or calls this file.
 *
 * The arithmetic of the path lives in the third-party packages the reference
 * pins, which are not vendored in the reference tree:
 *   - ml-explore/mlx-swift 0.31.6 (rev 0bb916c67f4b9e5c682cbe02a42c701c93ab5021,
 *     Package.swift:17, Package.resolved), bundling MLX C++ 0.31.1:
 *     quantize / dequantized / quantizedMM / gatherQuantizedMM / hadamardTransform;
 *   - ml-explore/mlx-swift-lm @ ee673d6a71d76e67b532dc7eaf91d92edc3bb8bb
 *     (Package.swift:20): SwitchGLU, QuantizedSwitchLinear, weightedExpertSum.
 * The functions below restate MLX's published affine-quantization algorithm and
 * anchor on the reference's call sites, cited per function.
 *
 * Parity status: packing/dequantization for bits 2/4/8 is pinned against an
 * independent implementation of the MLX packed format (tests/golden); the 3-bit
 * bitstream order, quantizer scale selection and the product numerics against
 * MLX itself are unpinned.
 */
#include "q38_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------ bf16 */

float q38o_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t q38o_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb; /* round to nearest even */
    return (uint16_t)(u >> 16);
}

static inline float bf(uint16_t h) { return q38o_bf16_to_f32(h); }
static inline float round_bf(float f) { return bf(q38o_f32_to_bf16(f)); }

/* ------------------------------------------------------------ threading */

static int g_threads = 0;

void q38o_set_threads(int n) { g_threads = n; }

int q38o_get_threads(void) {
    if (g_threads > 0) return g_threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef void (*range_fn)(void* ctx, int64_t begin, int64_t end);

typedef struct {
    range_fn fn;
    void* ctx;
    int64_t begin, end;
} range_job;

static void* range_thread(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

/* Split [0, n) into contiguous chunks, one per worker thread. */
static void parallel_for(int64_t n, range_fn fn, void* ctx) {
    int nt = q38o_get_threads();
    if (nt > n) nt = (int)(n > 0 ? n : 1);
    if (nt <= 1) {
        fn(ctx, 0, n);
        return;
    }
    pthread_t th[256];
    range_job jobs[256];
    if (nt > 256) nt = 256;
    for (int i = 0; i < nt; ++i) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].begin = n * i / nt;
        jobs[i].end = n * (i + 1) / nt;
    }
    for (int i = 1; i < nt; ++i) pthread_create(&th[i], NULL, range_thread, &jobs[i]);
    range_thread(&jobs[0]);
    for (int i = 1; i < nt; ++i) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------- packing */

static int valid_bits(int bits) {
    return bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8;
}

/* Code k of a row sits at bit k*bits of the row's little-endian bitstream: for
 * bits 2/4/8 that is word k/(32/bits), shift (k mod 32/bits)*bits; for 3/5/6 the
 * codes straddle words.  Packed row width is K*bits/32 words
 * (FlashNext/Qwen4ExpPrequantized.swift:60-64). */
static inline uint32_t get_code(const uint32_t* row, int64_t k, int bits) {
    int64_t bit = k * bits;
    int64_t w = bit >> 5;
    int off = (int)(bit & 31);
    uint64_t v = row[w];
    if (off + bits > 32) v |= (uint64_t)row[w + 1] << 32;
    return (uint32_t)(v >> off) & ((1u << bits) - 1u);
}

int q38o_unpack(const uint32_t* codes, int64_t rows, int64_t K, int bits, uint8_t* q) {
    if (!valid_bits(bits) || (K * bits) % 32) return -1;
    int64_t kw = K * bits / 32;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < K; ++k) q[r * K + k] = (uint8_t)get_code(codes + r * kw, k, bits);
    return 0;
}

int q38o_pack(const uint8_t* q, int64_t rows, int64_t K, int bits, uint32_t* codes) {
    if (!valid_bits(bits) || (K * bits) % 32) return -1;
    int64_t kw = K * bits / 32;
    memset(codes, 0, (size_t)(rows * kw) * 4);
    uint32_t mask = (1u << bits) - 1u;
    for (int64_t r = 0; r < rows; ++r) {
        uint32_t* row = codes + r * kw;
        for (int64_t k = 0; k < K; ++k) {
            uint64_t v = (uint64_t)(q[r * K + k] & mask);
            int64_t bit = k * bits;
            int64_t w = bit >> 5;
            int off = (int)(bit & 31);
            row[w] |= (uint32_t)(v << off);
            if (off + bits > 32) row[w + 1] |= (uint32_t)(v >> (32 - off));
        }
    }
    return 0;
}

/* ------------------------------------------------------------ quantize */

typedef struct {
    const float* w;
    int64_t K;
    int group, bits;
    uint32_t* codes;
    uint16_t* scales;
    uint16_t* biases;
} quant_ctx;

/* MLX affine quantization of one row (MLX C++ 0.31 affine quantize, as called by
 * Scripts/qwen4-exp-requantize-experts.py:246-251 via mx.quantize(mode="affine")).
 * Per group: the extreme with the larger magnitude ("edge") is made exactly
 * representable; scale = edge/q0 with q0 = rint(edge/scale0), bias = edge; codes
 * q = clamp(rint((w - bias)/scale), 0, 2^bits-1) computed with the fp32
 * scale/bias, which are then stored as bf16. */
static void quant_rows(void* p, int64_t r0, int64_t r1) {
    quant_ctx* c = (quant_ctx*)p;
    const float n_bins = (float)((1 << c->bits) - 1);
    const float eps = 1e-7f;
    int64_t K = c->K, G = K / c->group, kw = K * c->bits / 32;
    uint8_t* q = (uint8_t*)malloc((size_t)K);
    for (int64_t r = r0; r < r1; ++r) {
        const float* wr = c->w + r * K;
        for (int64_t g = 0; g < G; ++g) {
            const float* wg = wr + g * c->group;
            float wmin = INFINITY, wmax = -INFINITY;
            for (int j = 0; j < c->group; ++j) {
                wmax = fmaxf(wmax, wg[j]);
                wmin = fminf(wmin, wg[j]);
            }
            int mask = fabsf(wmin) > fabsf(wmax);
            float scale = fmaxf((wmax - wmin) / n_bins, eps);
            scale = mask ? scale : -scale;
            float edge = mask ? wmin : wmax;
            float q0 = rintf(edge / scale);
            float bias = 0.0f;
            if (q0 != 0.0f) {
                scale = edge / q0;
                bias = edge;
            }
            for (int j = 0; j < c->group; ++j) {
                float v = rintf((wg[j] - bias) / scale);
                v = fminf(fmaxf(v, 0.0f), n_bins);
                q[g * c->group + j] = (uint8_t)v;
            }
            c->scales[r * G + g] = q38o_f32_to_bf16(scale);
            c->biases[r * G + g] = q38o_f32_to_bf16(bias);
        }
        q38o_pack(q, 1, K, c->bits, c->codes + r * kw);
    }
    free(q);
}

int q38o_quantize(const float* w, int64_t rows, int64_t K, int group, int bits,
                  uint32_t* codes, uint16_t* scales, uint16_t* biases) {
    if (!valid_bits(bits) || group <= 0 || K % group || (K * bits) % 32) return -1;
    quant_ctx c = {w, K, group, bits, codes, scales, biases};
    parallel_for(rows, quant_rows, &c);
    return 0;
}

/* ---------------------------------------------------------- dequantize */

/* MLX.dequantized(w, scales:, biases:, groupSize:, bits:) as used by
 * FlashNext/Qwen4ExpCheckpointLayerLoader.swift:299-305: w = scale*q + bias. */
int q38o_dequantize(const uint32_t* codes, const uint16_t* scales, const uint16_t* biases,
                    int64_t rows, int64_t K, int group, int bits, float* w) {
    if (!valid_bits(bits) || group <= 0 || K % group || (K * bits) % 32) return -1;
    int64_t kw = K * bits / 32, G = K / group;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < K; ++k) {
            float s = bf(scales[r * G + k / group]);
            float b = biases ? bf(biases[r * G + k / group]) : 0.0f;
            w[r * K + k] = s * (float)get_code(codes + r * kw, k, bits) + b;
        }
    return 0;
}

/* ------------------------------------------------------------------ qmm */

typedef struct {
    const float* xf; /* [M, K] fp32 copy of x */
    int64_t M, K, N;
    const uint32_t* codes;
    const uint16_t* scales;
    const uint16_t* biases;
    int group, bits;
    float* y; /* [M, N] */
} qmm_ctx;

/* 8-way partial sums so the inner dot vectorises. */
static inline float dot_f32(const float* a, const float* b, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int j = 0;
    for (; j + 8 <= n; j += 8)
        for (int l = 0; l < 8; ++l) acc[l] += a[j + l] * b[j + l];
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    for (; j < n; ++j) s += a[j] * b[j];
    return s;
}

/* Product of QuantizedLinear.callAsFunction -> MLX.quantizedMM(x, w, scales:, biases:,
 * transpose: true, groupSize:, bits:) (FlashNext/Qwen4ExpPrequantized.swift:156-159):
 * y[m,n] = sum_k x[m,k] * (scale[n,k/g]*q[n,k] + bias[n,k/g]), fp32 accumulation. */
static void qmm_rows(void* p, int64_t n0, int64_t n1) {
    qmm_ctx* c = (qmm_ctx*)p;
    int64_t K = c->K, G = K / c->group, kw = K * c->bits / 32;
    float* wrow = (float*)malloc((size_t)K * sizeof(float));
    for (int64_t n = n0; n < n1; ++n) {
        const uint32_t* cr = c->codes + n * kw;
        for (int64_t g = 0; g < G; ++g) {
            float s = bf(c->scales[n * G + g]);
            float b = c->biases ? bf(c->biases[n * G + g]) : 0.0f;
            for (int j = 0; j < c->group; ++j) {
                int64_t k = g * c->group + j;
                wrow[k] = s * (float)get_code(cr, k, c->bits) + b;
            }
        }
        for (int64_t m = 0; m < c->M; ++m) c->y[m * c->N + n] = dot_f32(c->xf + m * K, wrow, (int)K);
    }
    free(wrow);
}

int q38o_qmm_f32(const uint16_t* x, int64_t M, int64_t K, const uint32_t* codes,
                 const uint16_t* scales, const uint16_t* biases, int64_t N, int group,
                 int bits, float* y) {
    if (!valid_bits(bits) || group <= 0 || K % group || (K * bits) % 32) return -1;
    float* xf = (float*)malloc((size_t)(M * K) * sizeof(float));
    for (int64_t i = 0; i < M * K; ++i) xf[i] = bf(x[i]);
    qmm_ctx c = {xf, M, K, N, codes, scales, biases, group, bits, y};
    parallel_for(N, qmm_rows, &c);
    free(xf);
    return 0;
}

int q38o_qmm(const uint16_t* x, int64_t M, int64_t K, const uint32_t* codes,
             const uint16_t* scales, const uint16_t* biases, int64_t N, int group,
             int bits, uint16_t* y) {
    float* yf = (float*)malloc((size_t)(M * N) * sizeof(float));
    int rc = q38o_qmm_f32(x, M, K, codes, scales, biases, N, group, bits, yf);
    if (rc == 0)
        for (int64_t i = 0; i < M * N; ++i) y[i] = q38o_f32_to_bf16(yf[i]);
    free(yf);
    return rc;
}

/* ------------------------------------------------------------ gather qmm */

/* gatherQuantizedMM(x, w, scales:, biases:, lhsIndices:, rhsIndices:, transpose: true)
 * behind QuantizedSwitchLinear.callAsFunction (Vendor/mlx-swift-lm-local.patch:184-218;
 * SwitchLayers.swift:528-540 upstream as cited in
 * docs/knowledge/investigations/p3-expert-offload.md:51-62): every output p multiplies
 * x[lhs[p]] by expert rhs[p]'s dequantized weight. */
int q38o_gather_qmm(const uint16_t* x, int64_t Bx, int64_t M, int64_t K,
                    const uint32_t* codes, const uint16_t* scales, const uint16_t* biases,
                    int64_t E, int64_t N, int group, int bits,
                    const int32_t* lhs, const int32_t* rhs, int64_t P, uint16_t* out) {
    if (!valid_bits(bits) || group <= 0 || K % group || (K * bits) % 32) return -1;
    int64_t kw = K * bits / 32, G = K / group;
    for (int64_t p = 0; p < P; ++p) {
        int64_t li = lhs ? lhs[p] : p;
        int64_t e = rhs[p];
        if (li < 0 || li >= Bx || e < 0 || e >= E) return -2;
        int rc = q38o_qmm(x + li * M * K, M, K, codes + e * N * kw, scales + e * N * G,
                          biases ? biases + e * N * G : NULL, N, group, bits, out + p * M * N);
        if (rc) return rc;
    }
    return 0;
}

/* -------------------------------------------------------------- router */

/* exp for x <= 0 by Cody-Waite range reduction x = n*ln2 + r, |r| <= ln2/2, and a
 * degree-7 Taylor polynomial of e^r in Horner form (fma); 2^n applied on the
 * exponent bits.  The CUDA router uses the identical operation sequence, so the
 * two agree bit for bit on identical inputs. */
static float q38_exp_nonpos(float x) {
    if (x < -87.0f) return 0.0f;
    const float log2e = 1.44269504088896341f;
    const float ln2_hi = 0.693145751953125f;      /* 0x3F317200: low mantissa bits zero */
    const float ln2_lo = 1.42860682030941723e-6f; /* ln2 - ln2_hi */
    float n = rintf(x * log2e);
    float r = fmaf(-n, ln2_hi, x);
    r = fmaf(-n, ln2_lo, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    uint32_t bits = (uint32_t)(ni + 127) << 23;
    float two_n;
    memcpy(&two_n, &bits, 4);
    return p * two_n;
}

/* Sum of 512-or-fewer values in the fixed tree the CUDA router uses: 32 strided
 * partial sums (lane l adds v[l], v[l+32], ... in order), then an xor-butterfly
 * over the 32 partials (offsets 16, 8, 4, 2, 1). */
static float tree_sum32(const float* v, int64_t n) {
    float part[32];
    for (int l = 0; l < 32; ++l) {
        float s = 0.0f;
        for (int64_t i = l; i < n; i += 32) s += v[i];
        part[l] = s;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; ++l) nxt[l] = part[l] + part[l ^ off];
        memcpy(part, nxt, sizeof(part));
    }
    return part[0];
}

/* Router of Qwen4ExpSparseMoE.callAsFunction (FlashNext/Qwen4ExpSparseMoE.swift:275-281):
 * softmax(precise) in fp32 rounded to bf16, argPartition top-k, takeAlong, and the
 * optional renormalisation scores / sum(scores).  argPartition's within-k order is
 * implementation-defined, so this restatement returns the canonical order:
 * probability descending, expert id ascending on ties. */
int q38o_route_from_logits(const uint16_t* logits, int64_t T, int64_t E, int top_k,
                           int normalize, int32_t* indices, uint16_t* scores,
                           uint16_t* probs_out) {
    if (top_k < 1 || top_k > E) return -1;
    float* e = (float*)malloc((size_t)E * sizeof(float));
    uint16_t* p = (uint16_t*)malloc((size_t)E * sizeof(uint16_t));
    uint8_t* taken = (uint8_t*)malloc((size_t)E);
    for (int64_t t = 0; t < T; ++t) {
        const uint16_t* l = logits + t * E;
        float mx = -INFINITY;
        for (int64_t i = 0; i < E; ++i) mx = fmaxf(mx, bf(l[i]));
        for (int64_t i = 0; i < E; ++i) e[i] = q38_exp_nonpos(bf(l[i]) - mx);
        float sum = tree_sum32(e, E);
        for (int64_t i = 0; i < E; ++i) p[i] = q38o_f32_to_bf16(e[i] / sum);
        if (probs_out) memcpy(probs_out + t * E, p, (size_t)E * 2);
        memset(taken, 0, (size_t)E);
        float ssum = 0.0f;
        for (int j = 0; j < top_k; ++j) {
            int64_t best = -1;
            float bv = -INFINITY;
            for (int64_t i = 0; i < E; ++i) {
                if (taken[i]) continue;
                float v = bf(p[i]);
                if (best < 0 || v > bv) {
                    best = i;
                    bv = v;
                }
            }
            taken[best] = 1;
            indices[t * top_k + j] = (int32_t)best;
            scores[t * top_k + j] = p[best];
            ssum += bv;
        }
        if (normalize) {
            float denom = round_bf(ssum);
            for (int j = 0; j < top_k; ++j)
                scores[t * top_k + j] = q38o_f32_to_bf16(bf(scores[t * top_k + j]) / denom);
        }
    }
    free(e);
    free(p);
    free(taken);
    return 0;
}

/* gate(x) is an unquantized Linear (FlashNext/Qwen4ExpSparseMoE.swift:208-214):
 * logits = bf16(x . Wr^T), fp32 accumulation. */
int q38o_moe_route(const uint16_t* x, int64_t T, int64_t H, const uint16_t* wr, int64_t E,
                   int top_k, int normalize, int32_t* indices, uint16_t* scores,
                   uint16_t* probs_out) {
    float* xf = (float*)malloc((size_t)H * sizeof(float));
    float* wf = (float*)malloc((size_t)(E * H) * sizeof(float));
    uint16_t* logits = (uint16_t*)malloc((size_t)(T * E) * 2);
    for (int64_t i = 0; i < E * H; ++i) wf[i] = bf(wr[i]);
    for (int64_t t = 0; t < T; ++t) {
        for (int64_t k = 0; k < H; ++k) xf[k] = bf(x[t * H + k]);
        for (int64_t i = 0; i < E; ++i) logits[t * E + i] = q38o_f32_to_bf16(dot_f32(xf, wf + i * H, (int)H));
    }
    int rc = q38o_route_from_logits(logits, T, E, top_k, normalize, indices, scores, probs_out);
    free(xf);
    free(wf);
    free(logits);
    return rc;
}

/* SwitchGLU's sort of (token, slot) pairs by expert when indices.size >= 64
 * (upstream SwitchLayers.swift:210/375, cited in p3-expert-offload.md:51-62), made
 * canonical: a stable counting sort, pairs of one expert in flat-index order. */
int q38o_sort_by_expert(const int32_t* indices, int64_t pairs, int64_t E, int32_t* perm,
                        int32_t* offsets) {
    memset(offsets, 0, (size_t)(E + 1) * sizeof(int32_t));
    for (int64_t i = 0; i < pairs; ++i) {
        if (indices[i] < 0 || indices[i] >= E) return -2;
        offsets[indices[i] + 1]++;
    }
    for (int64_t e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
    int32_t* fill = (int32_t*)malloc((size_t)E * sizeof(int32_t));
    memcpy(fill, offsets, (size_t)E * sizeof(int32_t));
    for (int64_t i = 0; i < pairs; ++i) perm[fill[indices[i]]++] = (int32_t)i;
    free(fill);
    return 0;
}

/* ------------------------------------------------------------ SwitchGLU */

typedef struct {
    const float* xf;
    int64_t H, I, top_k, kwh, kwi, Gh, Gi;
    const int32_t* indices;
    const uint16_t* scores;
    const uint32_t *gw, *uw, *dw;
    const uint16_t *gs, *gb, *us, *ub, *ds, *db;
    int group, bits, weights_bf16;
    uint16_t* out;
} glu_ctx;

static float silu_f32(float v) { return v / (1.0f + expf(-v)); }

/* Round an exactly known value (a double holding s*q + b without error: bf16 s and b
 * have 8 significant bits, q < 2^8) to the nearest bf16, ties to even, in one step. */
static float bf16_of_exact(double v) {
    if (v == 0.0) return 0.0f;
    int ex;
    double m = frexp(v, &ex); /* v = m * 2^ex, 0.5 <= |m| < 1 */
    return (float)ldexp(nearbyint(m * 256.0), ex - 8);
}

/* Dequantized row in fp32 (w = s*q + b evaluated in fp32), or -- weights_bf16 -- the
 * weight operand of a bf16 tensor-core product: s*q + b rounded once to bf16. */
static void dequant_row(const uint32_t* cr, const uint16_t* s, const uint16_t* b, int64_t K,
                        int group, int bits, int weights_bf16, float* w) {
    for (int64_t k = 0; k < K; ++k) {
        const float sv = bf(s[k / group]), bv = b ? bf(b[k / group]) : 0.0f;
        const uint32_t q = get_code(cr, k, bits);
        w[k] = weights_bf16 ? bf16_of_exact((double)sv * (double)q + (double)bv) : sv * (float)q + bv;
    }
}

/* SwitchGLU.callAsFunction + weightedExpertSum as used at
 * FlashNext/Qwen4ExpSparseMoE.swift:294: per (token, slot) the selected expert's
 * down(silu(gate(x)) * up(x)); the k slot outputs are combined with the router scores. */
static void glu_tokens(void* p, int64_t t0, int64_t t1) {
    glu_ctx* c = (glu_ctx*)p;
    int64_t H = c->H, I = c->I;
    float* w = (float*)malloc((size_t)(H > I ? H : I) * sizeof(float));
    float* h = (float*)malloc((size_t)I * sizeof(float));
    float* acc = (float*)malloc((size_t)H * sizeof(float));
    for (int64_t t = t0; t < t1; ++t) {
        const float* xt = c->xf + t * H;
        for (int64_t j = 0; j < H; ++j) acc[j] = 0.0f;
        for (int64_t s = 0; s < c->top_k; ++s) {
            int64_t e = c->indices[t * c->top_k + s];
            if (e < 0) continue; /* -1: an empty slot (expert-parallel partial sums) */
            float score = bf(c->scores[t * c->top_k + s]);
            for (int64_t i = 0; i < I; ++i) {
                int64_t row = e * I + i;
                dequant_row(c->gw + row * c->kwh, c->gs + row * c->Gh,
                            c->gb ? c->gb + row * c->Gh : NULL, H, c->group, c->bits, c->weights_bf16, w);
                float g = round_bf(dot_f32(xt, w, (int)H));
                dequant_row(c->uw + row * c->kwh, c->us + row * c->Gh,
                            c->ub ? c->ub + row * c->Gh : NULL, H, c->group, c->bits, c->weights_bf16, w);
                float u = round_bf(dot_f32(xt, w, (int)H));
                h[i] = round_bf(silu_f32(g) * u);
            }
            for (int64_t j = 0; j < H; ++j) {
                int64_t row = e * H + j;
                dequant_row(c->dw + row * c->kwi, c->ds + row * c->Gi,
                            c->db ? c->db + row * c->Gi : NULL, I, c->group, c->bits, c->weights_bf16, w);
                float y = round_bf(dot_f32(h, w, (int)I));
                acc[j] += score * y;
            }
        }
        for (int64_t j = 0; j < H; ++j) c->out[t * H + j] = q38o_f32_to_bf16(acc[j]);
    }
    free(w);
    free(h);
    free(acc);
}

int q38o_switch_glu(const uint16_t* x, int64_t T, int64_t H, int64_t I, int64_t E, int top_k,
                    const int32_t* indices, const uint16_t* scores,
                    const uint32_t* gw, const uint16_t* gs, const uint16_t* gb,
                    const uint32_t* uw, const uint16_t* us, const uint16_t* ub,
                    const uint32_t* dw, const uint16_t* ds, const uint16_t* db,
                    int group, int bits, int weights_bf16, uint16_t* out) {
    if (!valid_bits(bits) || group <= 0 || H % group || I % group) return -1;
    if ((H * bits) % 32 || (I * bits) % 32) return -1;
    for (int64_t i = 0; i < T * top_k; ++i)
        if (indices[i] < -1 || indices[i] >= E) return -2;
    float* xf = (float*)malloc((size_t)(T * H) * sizeof(float));
    for (int64_t i = 0; i < T * H; ++i) xf[i] = bf(x[i]);
    glu_ctx c = {xf, H, I, top_k, H * bits / 32, I * bits / 32, H / group, I / group,
                 indices, scores, gw, uw, dw, gs, gb, us, ub, ds, db, group, bits, weights_bf16, out};
    parallel_for(T, glu_tokens, &c);
    free(xf);
    return 0;
}

/* ------------------------------------------------------------- Hadamard */

/* hadamardRotate (Bonsai2/Qwen38HadamardModules.swift:10-19): fp32 copy, signs before
 * the transform (forward) or after it (inverse), normalised Sylvester-order
 * Walsh-Hadamard transform per block (butterfly stages h = 1, 2, 4, ...; a+b, a-b),
 * scaled by 1/sqrt(block), cast back to bf16. */
int q38o_hadamard_rotate(const uint16_t* x, int64_t rows, int64_t D, const float* signs,
                         int block, int inverse, uint16_t* y) {
    if (block <= 0 || (block & (block - 1)) || D % block) return -1;
    float scale = 1.0f / sqrtf((float)block);
    float* v = (float*)malloc((size_t)block * sizeof(float));
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b0 = 0; b0 < D; b0 += block) {
            for (int i = 0; i < block; ++i) {
                float f = bf(x[r * D + b0 + i]);
                if (!inverse && signs) f *= signs[b0 + i];
                v[i] = f;
            }
            for (int h = 1; h < block; h <<= 1)
                for (int i = 0; i < block; i += 2 * h)
                    for (int j = i; j < i + h; ++j) {
                        float a = v[j], b = v[j + h];
                        v[j] = a + b;
                        v[j + h] = a - b;
                    }
            for (int i = 0; i < block; ++i) {
                float f = v[i] * scale;
                if (inverse && signs) f *= signs[b0 + i];
                y[r * D + b0 + i] = q38o_f32_to_bf16(f);
            }
        }
    free(v);
    return 0;
}

/* ----------------------------------------------------------- generators */

static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* Counter-based normal sample i of stream `seed` (Box-Muller on two SplitMix64 draws). */
static inline double normal_at(uint64_t seed, int64_t i) {
    uint64_t a = splitmix64(seed * 0x100000001b3ull + 2 * (uint64_t)i);
    uint64_t b = splitmix64(seed * 0x100000001b3ull + 2 * (uint64_t)i + 1);
    double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740993.0);
    double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

typedef struct {
    uint64_t seed;
    float sd;
    void* out;
    int bf16;
} fill_ctx;

static void fill_range(void* p, int64_t i0, int64_t i1) {
    fill_ctx* c = (fill_ctx*)p;
    for (int64_t i = i0; i < i1; ++i) {
        float v = (float)(normal_at(c->seed, i) * c->sd);
        if (c->bf16)
            ((uint16_t*)c->out)[i] = q38o_f32_to_bf16(v);
        else
            ((float*)c->out)[i] = v;
    }
}

void q38o_fill_normal_bf16(uint64_t seed, float stddev, uint16_t* out, int64_t n) {
    fill_ctx c = {seed, stddev, out, 1};
    parallel_for(n, fill_range, &c);
}

void q38o_fill_normal_f32(uint64_t seed, float stddev, float* out, int64_t n) {
    fill_ctx c = {seed, stddev, out, 0};
    parallel_for(n, fill_range, &c);
}

void q38o_fill_ternary(uint64_t seed, float stddev, int64_t rows, int64_t K, int group,
                       uint32_t* codes, uint16_t* scales, uint16_t* biases) {
    int64_t G = K / group;
    uint8_t* q = (uint8_t*)malloc((size_t)K);
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t k = 0; k < K; ++k) {
            uint64_t z = splitmix64((seed ^ 0x5bd1e995ull) * 0x100000001b3ull + (uint64_t)(r * K + k));
            q[k] = (uint8_t)((z >> 11) % 3u);
        }
        q38o_pack(q, 1, K, 2, codes + r * (K / 16));
        for (int64_t g = 0; g < G; ++g) {
            uint16_t s = q38o_f32_to_bf16(fabsf((float)(normal_at(seed, r * G + g) * stddev)));
            scales[r * G + g] = s;
            biases[r * G + g] = s ^ 0x8000u;
        }
    }
    free(q);
}
