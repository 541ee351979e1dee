// C ABI entry points of libq38: context management, argument validation (the checks
// MLX's operators perform, reported as status codes instead of process aborts) and
// dispatch to the kernels.
#include <cudaTypedefs.h>

#include <mutex>

#include "ptx.cuh"
#include "q38_internal.h"

namespace q38 {

q38_status fail(q38_ctx* ctx, q38_status st, const char* fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return st;
}

q38_status check_launch(q38_ctx* ctx, const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return Q38_OK;
    return fail(ctx, Q38_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

q38_status ensure_workspace(q38_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->workspace_bytes) return Q38_OK;
    size_t want = align_up(bytes + bytes / 4, 1 << 20);
    if (ctx->workspace) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->workspace);
        ctx->workspace = nullptr;
        ctx->workspace_bytes = 0;
    }
    if (cudaMalloc(&ctx->workspace, want) != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_OUT_OF_MEMORY, "workspace of %zu bytes could not be allocated", want);
    }
    ctx->workspace_bytes = want;
    return Q38_OK;
}

q38_status ensure_aux(q38_ctx* ctx, size_t bytes, void** out) {
    if (bytes > ctx->aux_bytes) {
        const size_t want = align_up(bytes + bytes / 4, 1 << 20);
        if (ctx->aux) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(ctx->aux);
            ctx->aux = nullptr;
            ctx->aux_bytes = 0;
        }
        if (cudaMalloc(&ctx->aux, want) != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, Q38_ERR_OUT_OF_MEMORY, "activation buffer of %zu bytes could not be allocated", want);
        }
        ctx->aux_bytes = want;
    }
    *out = ctx->aux;
    return Q38_OK;
}

q38_status ensure_zero_region(q38_ctx* ctx, size_t counters, size_t accs, uint32_t** cnt,
                              float** acc) {
    if (counters > ctx->zcnt_cap || accs > ctx->zacc_cap || !ctx->zws) {
        size_t nc = counters > ctx->zcnt_cap ? align_up(counters + counters / 4, 1024) : ctx->zcnt_cap;
        size_t na = accs > ctx->zacc_cap ? align_up(accs + accs / 4, 1 << 16) : ctx->zacc_cap;
        if (nc == 0) nc = 1024;
        if (na == 0) na = 1 << 16;
        if (ctx->zws) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(ctx->zws);
            ctx->zws = nullptr;
        }
        const size_t bytes = align_up(nc * 4, 256) + na * 4;
        if (cudaMalloc(&ctx->zws, bytes) != cudaSuccess) {
            cudaGetLastError();
            ctx->zcnt_cap = ctx->zacc_cap = 0;
            return fail(ctx, Q38_ERR_OUT_OF_MEMORY, "accumulator region of %zu bytes could not be allocated", bytes);
        }
        if (cudaMemset(ctx->zws, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            return fail(ctx, Q38_ERR_CUDA, "accumulator region could not be cleared");
        }
        ctx->zcnt_cap = nc;
        ctx->zacc_cap = na;
    }
    *cnt = static_cast<uint32_t*>(ctx->zws);
    *acc = reinterpret_cast<float*>(static_cast<uint8_t*>(ctx->zws) + align_up(ctx->zcnt_cap * 4, 256));
    return Q38_OK;
}

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

const void* current_context_key() {
    typedef CUresult (*GetCurrentFn)(CUcontext*);
    static GetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetCurrentFn>(p);
    });
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, size_t elem_bytes, const void* base,
                 uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * elem_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace q38

using namespace q38;

namespace {

// One thread waits, with the library's bounded wait and the given limit, on an mbarrier
// phase that nothing completes: the wait runs out, records Q38_DEV_TIMEOUT in the status
// word and returns.  This is how the timeout path is exercised without a fault.
__global__ void wait_timeout_selftest(uint32_t* status, long long limit) {
    __shared__ __align__(8) uint64_t bar;
    dev::mbar_init(&bar, 1);
    dev::fence_mbar_init();
    dev::mbar_wait(&bar, 0, status, limit);
}

bool valid_bits(int bits) {
    return bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8;
}

bool valid_dtype(q38_dtype d) { return d == Q38_BF16 || d == Q38_F16 || d == Q38_F32; }

// The packing precondition of the reference (FlashNext/Qwen4ExpPrequantized.swift:60-72):
// K*bits % 32 == 0 and K % group == 0.
q38_status check_format(q38_ctx* ctx, const char* op, int64_t K, int group, int bits, q38_mode mode) {
    if (mode != Q38_MODE_AFFINE) return fail(ctx, Q38_ERR_UNSUPPORTED, "%s: only affine mode is implemented", op);
    if (!valid_bits(bits)) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: bits must be one of 2,3,4,5,6,8 (got %d)", op, bits);
    if (group != 32 && group != 64 && group != 128)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: group_size must be 32, 64 or 128 (got %d)", op, group);
    if (K <= 0 || K % group) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: K=%lld is not a multiple of group_size %d", op, (long long)K, group);
    if ((K * bits) % 32) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: K*bits=%lld is not a multiple of 32", op, (long long)(K * bits));
    return Q38_OK;
}

q38_status set_device(q38_ctx* ctx) {
    if (cudaSetDevice(ctx->device) != cudaSuccess) return check_launch(ctx, "cudaSetDevice");
    return Q38_OK;
}

}  // namespace

extern "C" {

int q38_version(void) { return 100; }

const char* q38_status_string(q38_status s) {
    switch (s) {
        case Q38_OK: return "ok";
        case Q38_ERR_INVALID_ARGUMENT: return "invalid argument";
        case Q38_ERR_UNSUPPORTED: return "unsupported";
        case Q38_ERR_CUDA: return "cuda error";
        case Q38_ERR_OUT_OF_MEMORY: return "out of memory";
        case Q38_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case Q38_ERR_COMM: return "communication error";
    }
    return "unknown status";
}

q38_status q38_ctx_create(int device, q38_ctx** out) {
    if (!out) return Q38_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return Q38_ERR_INVALID_ARGUMENT;
    }
    q38_ctx* c = new q38_ctx();
    c->device = device;
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaMalloc(&c->d_status, sizeof(uint32_t)) != cudaSuccess ||
        cudaMemset(c->d_status, 0, sizeof(uint32_t)) != cudaSuccess) {
        cudaGetLastError();
        delete c;
        return Q38_ERR_CUDA;
    }
    *out = c;
    return Q38_OK;
}

q38_status q38_ctx_destroy(q38_ctx* ctx) {
    if (!ctx) return Q38_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->workspace) cudaFree(ctx->workspace);
    if (ctx->zws) cudaFree(ctx->zws);
    if (ctx->aux) cudaFree(ctx->aux);
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->host_stage) cudaFreeHost(ctx->host_stage);
    for (cudaEvent_t e : ctx->stage_done)
        if (e) cudaEventDestroy(e);
    delete ctx;
    return Q38_OK;
}

q38_status q38_ctx_set_stream(q38_ctx* ctx, void* stream) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    ctx->stream = static_cast<cudaStream_t>(stream);
    return Q38_OK;
}

void* q38_ctx_get_stream(const q38_ctx* ctx) { return ctx ? ctx->stream : nullptr; }

q38_status q38_ctx_reserve(q38_ctx* ctx, size_t bytes) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = set_device(ctx);
    if (st != Q38_OK) return st;
    return ensure_workspace(ctx, bytes);
}

size_t q38_ctx_workspace_bytes(const q38_ctx* ctx) { return ctx ? ctx->workspace_bytes : 0; }

q38_status q38_ctx_set_deterministic(q38_ctx* ctx, int on) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    ctx->deterministic = on ? 1 : 0;
    return Q38_OK;
}

q38_status q38_ctx_set_ep_chunks(q38_ctx* ctx, int chunks) {
    if (!ctx || (chunks != 0 && chunks != 1 && chunks != 2 && chunks != 4)) return Q38_ERR_INVALID_ARGUMENT;
    ctx->ep_chunks = chunks;
    return Q38_OK;
}

q38_status q38_ctx_check_device(q38_ctx* ctx) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = set_device(ctx);
    if (st != Q38_OK) return st;
    uint32_t v = 0;
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess ||
        cudaMemcpy(&v, ctx->d_status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
        return check_launch(ctx, "check_device");
    if (v) {
        cudaMemset(ctx->d_status, 0, sizeof(uint32_t));
        if (v & Q38_DEV_TIMEOUT)
            return fail(ctx, Q38_ERR_DEVICE_TIMEOUT, "a device-side wait exceeded its limit (status 0x%x)", v);
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "an index argument was out of range (status 0x%x)", v);
    }
    return Q38_OK;
}

const char* q38_last_error(const q38_ctx* ctx) { return ctx ? ctx->last_error.c_str() : ""; }

q38_status q38_ctx_test_wait_timeout(q38_ctx* ctx, int64_t limit_cycles) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (limit_cycles < 0 || limit_cycles > 4000000000LL)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "test_wait_timeout: limit must be in [0, 4e9] cycles");
    q38_status st = set_device(ctx);
    if (st != Q38_OK) return st;
    wait_timeout_selftest<<<1, 1, 0, ctx->stream>>>(ctx->d_status, static_cast<long long>(limit_cycles));
    return check_launch(ctx, "test_wait_timeout");
}

q38_status q38_quantized_matmul(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype x_dtype,
                                const uint32_t* w, const void* scales, const void* biases,
                                q38_dtype scales_dtype, int64_t N, int transpose, int group_size,
                                int bits, q38_mode mode, void* y) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = check_format(ctx, "quantized_matmul", K, group_size, bits, mode);
    if (st != Q38_OK) return st;
    if (!transpose) return fail(ctx, Q38_ERR_UNSUPPORTED, "quantized_matmul: transpose=false is not implemented");
    if (x_dtype != Q38_BF16 && x_dtype != Q38_F16)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantized_matmul: x must be bf16 or f16");
    if (!valid_dtype(scales_dtype)) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantized_matmul: bad scales dtype");
    if (M < 0 || N <= 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantized_matmul: bad shape M=%lld N=%lld", (long long)M, (long long)N);
    if (M == 0) return Q38_OK;
    if (!x || !w || !scales || !y) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantized_matmul: null pointer");
    if ((st = set_device(ctx)) != Q38_OK) return st;
    if (qgemv_fast_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w, scales, biases, y))
        return qgemv_fast(ctx, x, M, K, w, scales, biases, N, bits, y);
    if (qgemv_pack_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w, scales, biases))
        return qgemv_pack(ctx, x, M, K, w, scales, biases, N, y);
    if (qgemm_tc_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w, scales, biases, y))
        return qgemm_tc_run(ctx, x, M, K, w, scales, biases, N, bits, y, group_size);
    return qmm_generic(ctx, x, M, K, x_dtype, w, scales, biases, scales_dtype, N, group_size, bits, y);
}



}  // extern "C"

namespace {

// Checks shared by the gate/up entries.
q38_status gate_up_check(q38_ctx* ctx, const char* op, const void* x, int64_t M, int64_t K, q38_dtype x_dtype,
                         const uint32_t* w_gate, const void* s_gate, const void* b_gate, const uint32_t* w_up,
                         const void* s_up, const void* b_up, q38_dtype scales_dtype, int64_t N, int group_size,
                         int bits, q38_mode mode, void* h) {
    q38_status st = check_format(ctx, op, K, group_size, bits, mode);
    if (st != Q38_OK) return st;
    if (x_dtype != Q38_BF16) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: x must be bf16", op);
    if (!valid_dtype(scales_dtype)) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: bad scales dtype", op);
    if (M < 0 || N <= 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: bad shape M=%lld N=%lld", op, (long long)M, (long long)N);
    if (M > 0 && (!x || !w_gate || !s_gate || !w_up || !s_up || !h))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: null pointer", op);
    if ((b_gate == nullptr) != (b_up == nullptr))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: gate and up must both have biases or neither", op);
    return Q38_OK;
}

}  // namespace

namespace q38 {

// h = bf16(silu(x.Wg^T) * x.Wu^T): one pass over both weights where the decode kernel takes
// the layout, otherwise the two products and the SiLU product, with the up product at byte
// `up_offset` of the activation buffer (the bytes before it may hold x).
q38_status gate_up_run(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype x_dtype,
                       const uint32_t* w_gate, const void* s_gate, const void* b_gate, const uint32_t* w_up,
                       const void* s_up, const void* b_up, q38_dtype scales_dtype, int64_t N, int group_size, int bits,
                       q38_mode mode, void* h, size_t up_offset) {
    if (qgemv_fast_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w_gate, s_gate, b_gate, h) &&
        qgemv_fast_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w_up, s_up, b_up, h))
        return qgemv_gate_up_fast(ctx, x, M, K, w_gate, s_gate, b_gate, w_up, s_up, b_up, N, bits, h);
    if (qgemv_pack_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w_gate, s_gate, b_gate) &&
        qgemv_pack_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w_up, s_up, b_up) &&
        (reinterpret_cast<uintptr_t>(h) & 15u) == 0)
        return qgemv_gate_up_pack(ctx, x, M, K, w_gate, s_gate, b_gate, w_up, s_up, b_up, N, h);
    void* base = nullptr;
    q38_status st;
    if ((st = ensure_aux(ctx, up_offset + static_cast<size_t>(M) * N * 2, &base)) != Q38_OK) return st;
    void* up = static_cast<uint8_t*>(base) + up_offset;
    if ((st = q38_quantized_matmul(ctx, x, M, K, x_dtype, w_gate, s_gate, b_gate, scales_dtype, N, 1, group_size,
                                   bits, mode, h)) != Q38_OK ||
        (st = q38_quantized_matmul(ctx, x, M, K, x_dtype, w_up, s_up, b_up, scales_dtype, N, 1, group_size, bits,
                                   mode, up)) != Q38_OK)
        return st;
    return q38_silu_mul(ctx, h, up, M * N, h);
}

}  // namespace q38

extern "C" {

q38_status q38_quantized_gate_up(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype x_dtype,
                                 const uint32_t* w_gate, const void* s_gate, const void* b_gate,
                                 const uint32_t* w_up, const void* s_up, const void* b_up, q38_dtype scales_dtype,
                                 int64_t N, int group_size, int bits, q38_mode mode, void* h) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = gate_up_check(ctx, "quantized_gate_up", x, M, K, x_dtype, w_gate, s_gate, b_gate, w_up, s_up,
                                  b_up, scales_dtype, N, group_size, bits, mode, h);
    if (st != Q38_OK || M == 0) return st;
    if ((st = set_device(ctx)) != Q38_OK) return st;
    return gate_up_run(ctx, x, M, K, x_dtype, w_gate, s_gate, b_gate, w_up, s_up, b_up, scales_dtype, N, group_size,
                       bits, mode, h, 0);
}

q38_status q38_hadamard_quantized_gate_up(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype x_dtype,
                                          const float* signs, int block, const uint32_t* w_gate, const void* s_gate,
                                          const void* b_gate, const uint32_t* w_up, const void* s_up,
                                          const void* b_up, q38_dtype scales_dtype, int64_t N, int group_size,
                                          int bits, void* h) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = gate_up_check(ctx, "hadamard_quantized_gate_up", x, M, K, x_dtype, w_gate, s_gate, b_gate, w_up,
                                  s_up, b_up, scales_dtype, N, group_size, bits, Q38_MODE_AFFINE, h);
    if (st != Q38_OK || M == 0) return st;
    if ((st = set_device(ctx)) != Q38_OK) return st;
    // decode-shaped: one pass over both weights with x rotated inside the kernel
    if (M == 1 && block >= 2 && block <= 512 && (block & (block - 1)) == 0 && K % block == 0) {
        if (qgemv_fast_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w_gate, s_gate, b_gate, h) &&
            qgemv_fast_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w_up, s_up, b_up, h))
            return qgemv_gate_up_fast(ctx, x, M, K, w_gate, s_gate, b_gate, w_up, s_up, b_up, N, bits, h, signs, block);
        if (qgemv_pack_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w_gate, s_gate, b_gate) &&
            qgemv_pack_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w_up, s_up, b_up) &&
            (reinterpret_cast<uintptr_t>(h) & 15u) == 0)
            return qgemv_gate_up_pack(ctx, x, M, K, w_gate, s_gate, b_gate, w_up, s_up, b_up, N, h, signs, block);
    }
    // the activation buffer holds the rotated x (rounded to bf16, as the reference rounds it
    // before each product), followed by room for the up product of the general path
    const size_t xbytes = align_up(static_cast<size_t>(M) * K * 2, 256);
    void* xr = nullptr;
    if ((st = ensure_aux(ctx, xbytes + static_cast<size_t>(M) * N * 2, &xr)) != Q38_OK) return st;
    if ((st = q38_hadamard_rotate(ctx, x, M, K, x_dtype, signs, block, 0, xr)) != Q38_OK) return st;
    return gate_up_run(ctx, xr, M, K, x_dtype, w_gate, s_gate, b_gate, w_up, s_up, b_up, scales_dtype, N, group_size,
                       bits, Q38_MODE_AFFINE, h, xbytes);
}

q38_status q38_shared_expert(q38_ctx* ctx, const void* x, int64_t T, int64_t H, int64_t I, const uint32_t* gate_w,
                             const void* gate_s, const void* gate_b, const uint32_t* up_w, const void* up_s,
                             const void* up_b, const uint32_t* down_w, const void* down_s, const void* down_b,
                             const uint32_t* sg_w, const void* sg_s, const void* sg_b, q38_dtype scales_dtype,
                             int group_size, int bits, const void* routed, void* out) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = gate_up_check(ctx, "shared_expert", x, T, H, Q38_BF16, gate_w, gate_s, gate_b, up_w, up_s, up_b,
                                  scales_dtype, I, group_size, bits, Q38_MODE_AFFINE, out);
    if (st != Q38_OK) return st;
    if ((st = check_format(ctx, "shared_expert", I, group_size, bits, Q38_MODE_AFFINE)) != Q38_OK) return st;
    if (T == 0) return Q38_OK;
    if (!down_w || !down_s || !sg_w || !sg_s || !routed)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "shared_expert: null pointer");
    if (T > (1 << 30) || H > (1 << 30))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "shared_expert: shape too large");
    if ((st = set_device(ctx)) != Q38_OK) return st;
    // activation buffer: h [T, I], the shared output ys [T, H], then the up product of the
    // general gate/up path; sized once so that the buffer does not move in between
    const size_t o_ys = align_up(static_cast<size_t>(T) * I * 2, 256);
    const size_t o_up = o_ys + align_up(static_cast<size_t>(T) * H * 2, 256);
    void* base = nullptr;
    if ((st = ensure_aux(ctx, o_up + static_cast<size_t>(T) * I * 2, &base)) != Q38_OK) return st;
    uint8_t* b8 = static_cast<uint8_t*>(base);
    if ((st = gate_up_run(ctx, x, T, H, Q38_BF16, gate_w, gate_s, gate_b, up_w, up_s, up_b, scales_dtype, I,
                          group_size, bits, Q38_MODE_AFFINE, b8, o_up)) != Q38_OK)
        return st;
    if ((st = q38_quantized_matmul(ctx, b8, T, I, Q38_BF16, down_w, down_s, down_b, scales_dtype, H, 1, group_size,
                                   bits, Q38_MODE_AFFINE, b8 + o_ys)) != Q38_OK)
        return st;
    return shared_combine_launch(ctx, x, T, H, sg_w, sg_s, sg_b, scales_dtype, group_size, bits, b8 + o_ys, routed,
                                 out);
}

q38_status q38_dequantize(q38_ctx* ctx, const uint32_t* w, const void* scales, const void* biases,
                          q38_dtype scales_dtype, int64_t rows, int64_t K, int group_size, int bits,
                          q38_mode mode, void* out, q38_dtype out_dtype) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = check_format(ctx, "dequantize", K, group_size, bits, mode);
    if (st != Q38_OK) return st;
    if (!valid_dtype(scales_dtype) || !valid_dtype(out_dtype))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "dequantize: bad dtype");
    if (rows < 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "dequantize: rows < 0");
    if (rows == 0) return Q38_OK;
    if (!w || !scales || !out) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "dequantize: null pointer");
    if ((st = set_device(ctx)) != Q38_OK) return st;
    return dequantize_launch(ctx, w, scales, biases, scales_dtype, rows, K, group_size, bits, out, out_dtype);
}

q38_status q38_quantized_embedding(q38_ctx* ctx, const int32_t* ids, int64_t n, const uint32_t* w,
                                   const void* scales, const void* biases, q38_dtype scales_dtype, int64_t rows,
                                   int64_t K, int group_size, int bits, q38_mode mode, void* out,
                                   q38_dtype out_dtype) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = check_format(ctx, "quantized_embedding", K, group_size, bits, mode);
    if (st != Q38_OK) return st;
    if (!valid_dtype(scales_dtype) || !valid_dtype(out_dtype))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantized_embedding: bad dtype");
    if (n < 0 || rows <= 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantized_embedding: bad sizes");
    if (n == 0) return Q38_OK;
    if (!ids || !w || !scales || !out) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantized_embedding: null pointer");
    if ((st = set_device(ctx)) != Q38_OK) return st;
    return embedding_launch(ctx, ids, n, w, scales, biases, scales_dtype, rows, K, group_size, bits, out, out_dtype);
}

q38_status q38_hadamard_quantized_embedding(q38_ctx* ctx, const int32_t* ids, int64_t n, const uint32_t* w,
                                            const void* scales, const void* biases, q38_dtype scales_dtype,
                                            int64_t rows, int64_t K, int group_size, int bits, q38_mode mode,
                                            const float* signs, int block, void* out) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = check_format(ctx, "hadamard_quantized_embedding", K, group_size, bits, mode);
    if (st != Q38_OK) return st;
    if (scales_dtype != Q38_BF16 && scales_dtype != Q38_F16)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_quantized_embedding: scales must be bf16 or f16");
    if (block < 2 || block > 8192 || (block & (block - 1)))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT,
                    "hadamard_quantized_embedding: block must be a power of two in [2, 8192]");
    if (K % block)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT,
                    "hadamard_quantized_embedding: Hadamard block does not divide the embedding width");
    if (n < 0 || rows <= 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_quantized_embedding: bad sizes");
    if (n == 0) return Q38_OK;
    if (!ids || !w || !scales || !out)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_quantized_embedding: null pointer");
    if ((st = set_device(ctx)) != Q38_OK) return st;
    return hadamard_embedding_launch(ctx, ids, n, w, scales, biases, scales_dtype, rows, K, group_size, bits, signs,
                                     block, out);
}

q38_status q38_quantize(q38_ctx* ctx, const void* w, q38_dtype w_dtype, int64_t rows, int64_t K,
                        int group_size, int bits, q38_mode mode, uint32_t* codes, void* scales,
                        void* biases, q38_dtype scales_dtype) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = check_format(ctx, "quantize", K, group_size, bits, mode);
    if (st != Q38_OK) return st;
    if (!valid_dtype(w_dtype) || !valid_dtype(scales_dtype))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantize: bad dtype");
    if (rows < 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantize: rows < 0");
    if (rows == 0) return Q38_OK;
    if (!w || !codes || !scales || !biases) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "quantize: null pointer");
    if ((st = set_device(ctx)) != Q38_OK) return st;
    return quantize_launch(ctx, w, w_dtype, rows, K, group_size, bits, codes, scales, biases, scales_dtype);
}

q38_status q38_unpack_codes(q38_ctx* ctx, const uint32_t* w, int64_t rows, int64_t K, int bits, uint8_t* q) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (!valid_bits(bits) || K <= 0 || (K * bits) % 32 || rows < 0)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "unpack_codes: bad shape or bits");
    if (rows == 0) return Q38_OK;
    if (!w || !q) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "unpack_codes: null pointer");
    q38_status st = set_device(ctx);
    if (st != Q38_OK) return st;
    return unpack_launch(ctx, w, rows, K, bits, q);
}

q38_status q38_hadamard_rotate(q38_ctx* ctx, const void* x, int64_t rows, int64_t D, q38_dtype x_dtype,
                               const float* signs, int block, int inverse, void* y) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (block < 2 || block > 8192 || (block & (block - 1)))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_rotate: block must be a power of two in [2, 8192]");
    if (D <= 0 || D % block) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_rotate: Hadamard block does not divide activation width");
    if (x_dtype != Q38_BF16 && x_dtype != Q38_F16) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_rotate: x must be bf16 or f16");
    if (rows < 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_rotate: rows < 0");
    if (rows == 0) return Q38_OK;
    if (!x || !y) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_rotate: null pointer");
    q38_status st = set_device(ctx);
    if (st != Q38_OK) return st;
    return hadamard_launch(ctx, x, rows, D, x_dtype, signs, block, inverse, y);
}

q38_status q38_hadamard_quantized_matmul(q38_ctx* ctx, const void* x, int64_t M, int64_t K, q38_dtype x_dtype,
                                         const float* signs, int block, const uint32_t* w, const void* scales,
                                         const void* biases, q38_dtype scales_dtype, int64_t N, int group_size,
                                         int bits, void* y) {
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (M < 0 || K <= 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_quantized_matmul: bad shape");
    if (M == 0) return Q38_OK;
    if (!x || !w || !scales || !y) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_quantized_matmul: null pointer");
    q38_status st = set_device(ctx);
    if (st != Q38_OK) return st;
    // Decode-shaped products rotate x inside the product kernel (its activation warp stages
    // x anyway); bit-identical to the rotation kernel followed by the product.
    // (one token, blocks of at most 512: wider blocks or more tokens make the activation warp
    // the bottleneck, and those run the rotation kernel first)
    if (M == 1 && block >= 2 && block <= 512 && (block & (block - 1)) == 0 && K % block == 0) {
        if (qgemv_fast_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w, scales, biases, y))
            return qgemv_fast(ctx, x, M, K, w, scales, biases, N, bits, y, signs, block);
        if (qgemv_pack_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w, scales, biases))
            return qgemv_pack(ctx, x, M, K, w, scales, biases, N, y, signs, block);
    }
    // Prompt-shaped products rotate x in the tensor-core product's prologue (which permutes
    // x anyway); bit-identical to the rotation kernel followed by the product.  Blocks of at
    // most 512 (a 1024 block in one warp made the prologue slower than the two kernels: 2048
    // tokens, pack layout 5120 -> 17408, 377.8 -> 382.1 us; block 256, 17408 -> 5120,
    // 463.5 -> 452.5 us).
    if (block >= 2 && block <= 512 && (block & (block - 1)) == 0 && K % 256 == 0 &&
        qgemm_tc_supported(M, K, group_size, bits, x_dtype, scales_dtype, x, w, scales, biases, y)) {
        if ((st = check_format(ctx, "hadamard_quantized_matmul", K, group_size, bits, Q38_MODE_AFFINE)) != Q38_OK)
            return st;
        if (N <= 0) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "hadamard_quantized_matmul: bad shape N=%lld", (long long)N);
        return qgemm_tc_run(ctx, x, M, K, w, scales, biases, N, bits, y, group_size, signs, block);
    }
    // The rotated activations (rounded to x_dtype, as the reference does before the
    // product) live in the context's activation buffer.
    void* xr = nullptr;
    if ((st = ensure_aux(ctx, static_cast<size_t>(M) * K * 2, &xr)) != Q38_OK) return st;
    st = q38_hadamard_rotate(ctx, x, M, K, x_dtype, signs, block, 0, xr);
    if (st != Q38_OK) return st;
    return q38_quantized_matmul(ctx, xr, M, K, x_dtype, w, scales, biases, scales_dtype, N, 1, group_size, bits,
                                Q38_MODE_AFFINE, y);
}

q38_status q38_gather_quantized_matmul(q38_ctx* ctx, const void* x, int64_t Bx, int64_t M, int64_t K,
                                       q38_dtype x_dtype, const uint32_t* w, const void* scales,
                                       const void* biases, q38_dtype scales_dtype, int64_t E, int64_t N,
                                       const int32_t* lhs_indices, const int32_t* rhs_indices, int64_t P,
                                       int transpose, int group_size, int bits, q38_mode mode,
                                       int sorted_indices, void* out) {
    (void)sorted_indices;
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    q38_status st = check_format(ctx, "gather_quantized_matmul", K, group_size, bits, mode);
    if (st != Q38_OK) return st;
    if (!transpose) return fail(ctx, Q38_ERR_UNSUPPORTED, "gather_quantized_matmul: transpose=false is not implemented");
    if (x_dtype != Q38_BF16 && x_dtype != Q38_F16)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "gather_quantized_matmul: x must be bf16 or f16");
    if (!valid_dtype(scales_dtype)) return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "gather_quantized_matmul: bad scales dtype");
    if (Bx <= 0 || M < 0 || E <= 0 || N <= 0 || P < 0)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "gather_quantized_matmul: bad shape");
    if (!lhs_indices && Bx < P)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "gather_quantized_matmul: lhs_indices NULL requires Bx >= P");
    if (P == 0 || M == 0) return Q38_OK;
    if (!x || !w || !scales || !rhs_indices || !out)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "gather_quantized_matmul: null pointer");
    if ((st = set_device(ctx)) != Q38_OK) return st;
    if (qgemv_gather_supported(M, K, E, N, P, group_size, bits, x_dtype, scales_dtype, x, w, scales, biases))
        return qgemv_gather(ctx, x, Bx, K, w, scales, biases, E, N, lhs_indices, rhs_indices, P, bits, out);
    return gather_generic(ctx, x, Bx, M, K, x_dtype, w, scales, biases, scales_dtype, E, N, lhs_indices,
                          rhs_indices, P, group_size, bits, out);
}

}  // extern "C"
