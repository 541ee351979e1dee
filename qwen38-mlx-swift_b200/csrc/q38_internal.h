// Internal declarations shared by the translation units of libq38.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/q38.h"

// Device-side status bits (ctx->d_status).
#define Q38_DEV_TIMEOUT 1u
#define Q38_DEV_BAD_INDEX 2u

struct q38_ctx {
    int device = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    void* workspace = nullptr;  // scratch; grows on demand, no content invariant
    size_t workspace_bytes = 0;
    // Zero-at-rest accumulators: every kernel that uses them returns them to zero.
    // Layout: [counters: zcnt_cap uint32][pad to 256][fp32 partial sums: zacc_cap floats]
    void* zws = nullptr;
    size_t zcnt_cap = 0, zacc_cap = 0;
    void* aux = nullptr;  // activation-sized intermediates (rotated x, MoE buffers)
    size_t aux_bytes = 0;
    uint32_t* d_status = nullptr;  // device status word (timeouts)
    int deterministic = 0;  // decode products: ordered chunk sums (bitwise reproducible)
    int ep_chunks = 0;      // pieces of the expert-parallel exchange (0: the library's choice)
    // Pinned host staging of the safetensors reader: two halves used alternately, each
    // guarded by an event of its last host->device copy.
    void* host_stage = nullptr;
    size_t host_stage_bytes = 0;  // per half
    cudaEvent_t stage_done[2] = {nullptr, nullptr};
    std::string last_error;
};

namespace q38 {

// Records the message on the context and returns the status.
q38_status fail(q38_ctx* ctx, q38_status st, const char* fmt, ...);

// Checks the most recent launch; converts a CUDA error into Q38_ERR_CUDA.
q38_status check_launch(q38_ctx* ctx, const char* what);

// Makes sure the scratch workspace holds at least `bytes`.
q38_status ensure_workspace(q38_ctx* ctx, size_t bytes);
// Makes sure the activation buffer holds `bytes`; returns its address.
q38_status ensure_aux(q38_ctx* ctx, size_t bytes, void** out);
// Makes sure the zero-at-rest region holds `counters` uint32 and `accs` floats; returns
// their device addresses.  Growth reallocates and zero-fills (synchronising the device).
q38_status ensure_zero_region(q38_ctx* ctx, size_t counters, size_t accs, uint32_t** cnt,
                              float** acc);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// h = bf16(silu(x.Wg^T) * x.Wu^T) [M, N]: one pass over both weights where the decode kernel
// takes the layout, otherwise two products and the SiLU product, the up product held at byte
// `up_offset` of the activation buffer.
q38_status gate_up_run(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype x_dtype,
                       const uint32_t* w_gate, const void* s_gate, const void* b_gate, const uint32_t* w_up,
                       const void* s_up, const void* b_up, q38_dtype scales_dtype, int64_t N, int group_size, int bits,
                       q38_mode mode, void* h, size_t up_offset);

// out[t] = bf16(routed[t] + bf16(s_t * ys[t])) with s_t = bf16(sigmoid(bf16(x_t . dequant(wsg))))
// for wsg a quantized [1, H] row: the shared-expert term of the sparse-MoE block.
q38_status shared_combine_launch(q38_ctx* ctx, const void* x, int64_t T, int64_t H, const uint32_t* gw,
                                 const void* gs, const void* gb, q38_dtype sd, int group, int bits, const void* ys,
                                 const void* routed, void* out);

// Driver entry point for cuTensorMapEncodeTiled (resolved once, no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();

// The calling thread's current CUDA context as an opaque key (nullptr if it cannot be
// read).  Per-device caches of module state (a symbol's address, a kernel attribute) are
// keyed on it, so that a context created anew after a reset sets them up again.
const void* current_context_key();

// 2-D tiled tensor map over a row-major [rows, cols] array.
bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, size_t elem_bytes, const void* base,
                 uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swz);

// ---- kernel launchers (each returns Q38_OK or an error recorded on ctx) ----

// Decode-shaped product (M <= 16, group 64, K % 512 == 0, bits 2/3/4/8, bf16).
bool qgemv_fast_supported(int64_t M, int64_t K, int group, int bits, q38_dtype xd,
                          q38_dtype sd, const void* x, const void* w, const void* s,
                          const void* b, const void* y);
// Rows ids[0..n) of a packed table, dequantized (quant.cu).
q38_status embedding_launch(q38_ctx* ctx, const int32_t* ids, int64_t n, const uint32_t* w, const void* s,
                            const void* b, q38_dtype sd, int64_t rows, int64_t K, int group, int bits, void* out,
                            q38_dtype od);
// Decode product over the Bonsai 2 pack layout: 2-bit codes, f16 scales and biases, group 128,
// bf16 x, K % 1024 == 0, M <= 16.
bool qgemv_pack_supported(int64_t M, int64_t K, int group, int bits, q38_dtype xd, q38_dtype sd,
                          const void* x, const void* w, const void* s, const void* b);
// With rot_block > 0 (M == 1, a power of two <= 512 dividing K) the kernel first rotates x
// as hadamardRotate does (signs fp32 [K] or null), in the activation warp: bit-identical to
// q38_hadamard_rotate followed by the product.
q38_status qgemv_pack(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w, const void* s,
                      const void* b, int64_t N, void* y, const float* signs = nullptr, int rot_block = 0);
q38_status qgemv_fast(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w,
                      const void* s, const void* b, int64_t N, int bits, void* y, const float* signs = nullptr,
                      int rot_block = 0);
// h = bf16(silu(x.Wg^T) * (x.Wu^T)) in one decode pass (same conditions as qgemv_fast for
// both weights, which must both have biases or neither).
// Gate/up in one pass over the Bonsai 2 pack layout (both weights qgemv_pack_supported).
q38_status qgemv_gate_up_pack(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* wg,
                              const void* sg, const void* bg, const uint32_t* wu, const void* su, const void* bu,
                              int64_t N, void* h, const float* signs = nullptr, int rot_block = 0);
q38_status qgemv_gate_up_fast(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* wg,
                              const void* sg, const void* bg, const uint32_t* wu, const void* su, const void* bu,
                              int64_t N, int bits, void* h, const float* signs = nullptr, int rot_block = 0);

// Decode-shaped SwitchGLU (T <= 16 tokens, T * top_k <= 256, group 64, bits 2/3/4/8, bf16,
// H and I multiples of 512): the selected experts' gate/up and down products on the decode
// kernel, h formed between them, then the score-weighted combine.
bool qgemv_moe_supported(int64_t T, int64_t H, int64_t I, int64_t E, int topk, int group, int bits, const void* x,
                         const void* gw, const void* gs, const void* gb, const void* uw, const void* us,
                         const void* ub, const void* dw, const void* ds, const void* db);
q38_status qgemv_moe_decode(q38_ctx* ctx, const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int topk,
                            const int32_t* idx, const void* scores, const uint32_t* gw, const void* gs,
                            const void* gb, const uint32_t* uw, const void* us, const void* ub, const uint32_t* dw,
                            const void* ds, const void* db, int bits, void* out);

// Gathered product out[p] = x[lhs[p]] . dequant(w[rhs[p]])^T on the decode kernel: one
// activation row per batch entry (M == 1), up to 256 pairs (in pieces of 16), group 64,
// bits 2/3/4/8, bf16, K % 512 == 0, N % 64 == 0.
bool qgemv_gather_supported(int64_t M, int64_t K, int64_t E, int64_t N, int64_t P, int group, int bits, q38_dtype xd,
                            q38_dtype sd, const void* x, const void* w, const void* s, const void* b);
q38_status qgemv_gather(q38_ctx* ctx, const void* x, int64_t Bx, int64_t K, const uint32_t* w, const void* s,
                        const void* b, int64_t E, int64_t N, const int32_t* lhs, const int32_t* rhs, int64_t P,
                        int bits, void* out);

// Prompt-shaped product on the tensor cores (M >= 17, groups 64 and 32 with bf16 scales or
// the pack's group 128 with f16 scales, K % 128 == 0, bits 2/3/4/8, bf16 x).  Uses the
// scratch workspace for the permuted activations (M*K bf16).  With rot_block > 0 (a power
// of two <= 1024; K a multiple of max(256, rot_block)) the prologue first rotates x as
// hadamardRotate does (signs fp32 [K] or null): bit-identical to q38_hadamard_rotate
// followed by the product.
bool qgemm_tc_supported(int64_t M, int64_t K, int group, int bits, q38_dtype xd, q38_dtype sd,
                        const void* x, const void* w, const void* s, const void* b, const void* y);
q38_status qgemm_tc_run(q38_ctx* ctx, const void* x, int64_t M, int64_t K, const uint32_t* w,
                        const void* s, const void* b, int64_t N, int bits, void* y, int group = 64,
                        const float* signs = nullptr, int rot_block = 0);

// General product, any supported shape (CUDA cores; correctness path for odd shapes).
q38_status qmm_generic(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype xd,
                       const uint32_t* w, const void* s, const void* b, q38_dtype sd,
                       int64_t N, int group, int bits, void* y);

// Gathered product of the general path (any supported shape).
q38_status gather_generic(q38_ctx* ctx, const void* x, int64_t Bx, int64_t M, int64_t K, q38_dtype xd,
                          const uint32_t* w, const void* s, const void* b, q38_dtype sd, int64_t E,
                          int64_t N, const int32_t* lhs, const int32_t* rhs, int64_t P, int group,
                          int bits, void* out);

q38_status dequantize_launch(q38_ctx* ctx, const uint32_t* w, const void* s, const void* b,
                             q38_dtype sd, int64_t rows, int64_t K, int group, int bits,
                             void* out, q38_dtype od);
q38_status quantize_launch(q38_ctx* ctx, const void* w, q38_dtype wd, int64_t rows, int64_t K,
                           int group, int bits, uint32_t* codes, void* s, void* b,
                           q38_dtype sd);
q38_status unpack_launch(q38_ctx* ctx, const uint32_t* w, int64_t rows, int64_t K, int bits,
                         uint8_t* q);
q38_status hadamard_embedding_launch(q38_ctx* ctx, const int32_t* ids, int64_t n, const uint32_t* w,
                                     const void* s, const void* b, q38_dtype sd, int64_t rows, int64_t K,
                                     int group, int bits, const float* signs, int block, void* out);
q38_status hadamard_launch(q38_ctx* ctx, const void* x, int64_t rows, int64_t D, q38_dtype xd,
                           const float* signs, int block, int inverse, void* y);

}  // namespace q38
