// Multi-GPU layouts of the quantized products behind the C ABI, over NCCL (NVLink /
// NVSwitch on B200), one communicator rank per GPU:
//
//   q38_tp_mlp         the dense 27B MLP block split tensor-parallel: gate/up by output rows,
//                      down by its reduction dimension, partial outputs summed by an
//                      all-reduce; the tokens are cut into chunks so that the all-reduce of
//                      chunk i (on the communicator's stream) runs while chunk i+1 computes.
//   q38_ep_switch_glu  the routed experts of the Flash-Next MoE layer
//                      (Sources/Qwen38Core/FlashNext/Qwen4ExpSparseMoE.swift:275-294) split
//                      expert-parallel: every rank's tokens (a fixed capacity of rows, so all
//                      exchange sizes are known in advance and nothing is read back to the
//                      host) are all-gathered with their slot experts and scores; each rank
//                      runs SwitchGLU over its own experts on every row (q38_switch_glu, the
//                      other ranks' slots empty) and a bf16 reduce-scatter sums the partial
//                      outputs into each token's home rank.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2; the copy already in the process is
// reused), so the library has no link-time dependency on it.  Communicators are created
// non-blocking with a host deadline: a rank that never joins makes init return
// Q38_ERR_COMM after the timeout (the communicator is aborted) instead of hanging.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "affine_codes.cuh"
#include "q38_internal.h"

namespace q38 {
namespace {

using namespace dev;

// ------------------------------------------------------------------ NCCL at run time
struct Nccl {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
    ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*ReduceScatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char* (*GetErrorString)(ncclResult_t);
    bool ok = false;
    std::string why;
};

const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* env = getenv("Q38_NCCL_LIBRARY");
        void* h = nullptr;
        if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy already loaded
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            n.why = std::string("libnccl.so.2 could not be loaded: ") + (dlerror() ? dlerror() : "not found");
            return;
        }
        bool all = true;
        auto sym = [&](auto& fp, const char* name) {
            fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(dlsym(h, name));
            if (!fp) all = false;
        };
        sym(n.GetUniqueId, "ncclGetUniqueId");
        sym(n.CommInitRankConfig, "ncclCommInitRankConfig");
        sym(n.CommInitAll, "ncclCommInitAll");
        sym(n.CommDestroy, "ncclCommDestroy");
        sym(n.CommAbort, "ncclCommAbort");
        sym(n.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(n.AllReduce, "ncclAllReduce");
        sym(n.Send, "ncclSend");
        sym(n.Recv, "ncclRecv");
        sym(n.AllGather, "ncclAllGather");
        sym(n.ReduceScatter, "ncclReduceScatter");
        sym(n.GroupStart, "ncclGroupStart");
        sym(n.GroupEnd, "ncclGroupEnd");
        sym(n.GetErrorString, "ncclGetErrorString");
        n.ok = all;
        if (!all) n.why = "libnccl.so.2 lacks an entry point this library needs";
    });
    return n;
}

thread_local std::string t_comm_error;

q38_status comm_fail(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_comm_error = buf;
    return Q38_ERR_COMM;
}

}  // namespace
}  // namespace q38

struct q38_comm {
    ncclComm_t nc = nullptr;
    int rank = 0, world = 1, device = 0;
    int timeout_ms = 0;
    bool aborted = false;
    cudaStream_t stream = nullptr;  // the collectives' stream (overlap with the context's)
    std::vector<cudaEvent_t> events;
    cudaEvent_t joined = nullptr;
    // exchange buffers, grown on demand
    void* buf = nullptr;
    size_t buf_bytes = 0;
};

namespace q38 {
namespace {

// Waits (bounded) until the communicator's last operation has been accepted.
q38_status settle(q38_comm* c, const char* what) {
    const Nccl& n = nccl();
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(c->timeout_ms);
    for (;;) {
        ncclResult_t st = ncclSuccess;
        if (n.CommGetAsyncError(c->nc, &st) != ncclSuccess) st = ncclSystemError;
        if (st == ncclSuccess) return Q38_OK;
        if (st != ncclInProgress) {
            return comm_fail("%s: %s", what, n.GetErrorString(st));
        }
        if (std::chrono::steady_clock::now() > deadline) {
            n.CommAbort(c->nc);
            c->aborted = true;
            return comm_fail("%s: no progress within %d ms (communicator aborted)", what, c->timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

q38_status nccl_call(q38_ctx* ctx, q38_comm* c, ncclResult_t r, const char* what) {
    if (r != ncclSuccess && r != ncclInProgress)
        return fail(ctx, Q38_ERR_COMM, "%s: %s", what, nccl().GetErrorString(r));
    if (settle(c, what) != Q38_OK) return fail(ctx, Q38_ERR_COMM, "%s", t_comm_error.c_str());
    return Q38_OK;
}

q38_status comm_buffer(q38_ctx* ctx, q38_comm* c, size_t bytes, uint8_t** out) {
    if (bytes > c->buf_bytes) {
        const size_t want = align_up(bytes + bytes / 4, 1 << 20);
        if (c->buf) {
            cudaDeviceSynchronize();
            cudaFree(c->buf);
            c->buf = nullptr;
            c->buf_bytes = 0;
        }
        if (cudaMalloc(&c->buf, want) != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, Q38_ERR_OUT_OF_MEMORY, "communicator buffer of %zu bytes could not be allocated", want);
        }
        c->buf_bytes = want;
    }
    *out = static_cast<uint8_t*>(c->buf);
    return Q38_OK;
}

q38_status check_pair(q38_ctx* ctx, q38_comm* c, const char* op) {
    if (!ctx || !c) return Q38_ERR_INVALID_ARGUMENT;
    if (c->aborted) return fail(ctx, Q38_ERR_COMM, "%s: the communicator was aborted", op);
    if (ctx->device != c->device)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "%s: context device %d, communicator device %d", op, ctx->device,
                    c->device);
    if (cudaSetDevice(ctx->device) != cudaSuccess) return check_launch(ctx, op);
    return Q38_OK;
}

cudaEvent_t comm_event(q38_comm* c, size_t i) {
    while (c->events.size() <= i) {
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
        c->events.push_back(e);
    }
    return c->events[i];
}

// ------------------------------------------------------------------ EP kernels
// This rank's slot metadata for the gather: rows t < T carry the token's experts and scores,
// rows T..C-1 (capacity padding) empty slots.
__global__ void __launch_bounds__(256) ep_own_meta(const int32_t* __restrict__ idx,
                                                   const __nv_bfloat16* __restrict__ scores, int T, int C, int k,
                                                   int32_t* __restrict__ ids, __nv_bfloat16* __restrict__ sc) {
    griddep_wait();
    griddep_launch_dependents();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < C * k; i += gridDim.x * blockDim.x) {
        const bool live = i < T * k;
        ids[i] = live ? idx[i] : -1;
        sc[i] = live ? scores[i] : __float2bfloat16_rn(0.0f);
    }
}

// Gathered expert ids -> this rank's local ids, -1 for experts of other ranks (and for
// padding or out-of-range ids).
__global__ void __launch_bounds__(256) ep_localize(int32_t* __restrict__ ids, int n, int E, int epr, int rank) {
    griddep_wait();
    griddep_launch_dependents();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int e = ids[i];
        ids[i] = (e >= 0 && e < E && e / epr == rank) ? e - rank * epr : -1;
    }
}

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, cudaStream_t stream, cudaLaunchAttribute* attr) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

}  // namespace
}  // namespace q38

using namespace q38;

extern "C" {

const char* q38_comm_error(void) { return t_comm_error.c_str(); }

q38_status q38_comm_get_unique_id(q38_comm_id* id) {
    if (!id) return Q38_ERR_INVALID_ARGUMENT;
    const Nccl& n = nccl();
    if (!n.ok) return comm_fail("%s", n.why.c_str());
    static_assert(sizeof(ncclUniqueId) <= sizeof(id->bytes), "NCCL unique id fits");
    ncclUniqueId u;
    const ncclResult_t r = n.GetUniqueId(&u);
    if (r != ncclSuccess) return comm_fail("ncclGetUniqueId: %s", n.GetErrorString(r));
    memset(id->bytes, 0, sizeof(id->bytes));
    memcpy(id->bytes, &u, sizeof(u));
    return Q38_OK;
}

q38_status q38_comm_init_rank(const q38_comm_id* id, int world, int rank, int device, int timeout_ms,
                              q38_comm** out) {
    if (!id || !out || world < 1 || world > 32 || rank < 0 || rank >= world || timeout_ms < 1)
        return Q38_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    const Nccl& n = nccl();
    if (!n.ok) return comm_fail("%s", n.why.c_str());
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return comm_fail("cudaSetDevice(%d) failed", device);
    }
    q38_comm* c = new q38_comm();
    c->rank = rank;
    c->world = world;
    c->device = device;
    c->timeout_ms = timeout_ms;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->joined, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        delete c;
        return comm_fail("stream or event creation failed");
    }
    ncclUniqueId u;
    memcpy(&u, id->bytes, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // returns at once; progress is polled against the deadline
    const ncclResult_t r = n.CommInitRankConfig(&c->nc, world, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        cudaStreamDestroy(c->stream);
        cudaEventDestroy(c->joined);
        delete c;
        return comm_fail("ncclCommInitRankConfig: %s", n.GetErrorString(r));
    }
    if (settle(c, "communicator init") != Q38_OK) {
        // aborted by settle (a rank did not join in time)
        cudaStreamDestroy(c->stream);
        cudaEventDestroy(c->joined);
        delete c;
        return Q38_ERR_COMM;
    }
    *out = c;
    return Q38_OK;
}

q38_status q38_comm_init_all(int ndev, const int* devices, int timeout_ms, q38_comm** comms) {
    if (ndev < 1 || ndev > 32 || !devices || !comms || timeout_ms < 1) return Q38_ERR_INVALID_ARGUMENT;
    q38_comm_id id;
    q38_status st = q38_comm_get_unique_id(&id);
    if (st != Q38_OK) return st;
    for (int i = 0; i < ndev; ++i) comms[i] = nullptr;
    // every rank's non-blocking init is issued first, then all are settled
    const Nccl& n = nccl();
    ncclUniqueId u;
    memcpy(&u, id.bytes, sizeof(u));
    std::vector<q38_comm*> cs(ndev, nullptr);
    bool bad = false;
    n.GroupStart();
    for (int i = 0; i < ndev && !bad; ++i) {
        if (cudaSetDevice(devices[i]) != cudaSuccess) {
            cudaGetLastError();
            bad = true;
            break;
        }
        q38_comm* c = new q38_comm();
        c->rank = i;
        c->world = ndev;
        c->device = devices[i];
        c->timeout_ms = timeout_ms;
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        cudaEventCreateWithFlags(&c->joined, cudaEventDisableTiming);
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        const ncclResult_t r = n.CommInitRankConfig(&c->nc, ndev, u, i, &cfg);
        cs[i] = c;
        if (r != ncclSuccess && r != ncclInProgress) bad = true;
    }
    n.GroupEnd();
    for (int i = 0; i < ndev && !bad; ++i)
        if (cs[i] && settle(cs[i], "communicator init") != Q38_OK) bad = true;
    if (bad) {
        for (q38_comm* c : cs) {
            if (!c) continue;
            if (c->nc && !c->aborted) n.CommAbort(c->nc);
            if (c->stream) cudaStreamDestroy(c->stream);
            if (c->joined) cudaEventDestroy(c->joined);
            delete c;
        }
        if (t_comm_error.empty()) t_comm_error = "communicator init failed";
        return Q38_ERR_COMM;
    }
    for (int i = 0; i < ndev; ++i) comms[i] = cs[i];
    return Q38_OK;
}

q38_status q38_comm_destroy(q38_comm* c) {
    if (!c) return Q38_OK;
    const Nccl& n = nccl();
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->nc && !c->aborted) n.CommDestroy(c->nc);
    if (c->buf) cudaFree(c->buf);
    for (cudaEvent_t e : c->events) cudaEventDestroy(e);
    if (c->joined) cudaEventDestroy(c->joined);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return Q38_OK;
}

q38_status q38_comm_abort(q38_comm* c) {
    if (!c) return Q38_ERR_INVALID_ARGUMENT;
    if (c->nc && !c->aborted) nccl().CommAbort(c->nc);
    c->aborted = true;
    return Q38_OK;
}

int q38_comm_rank(const q38_comm* c) { return c ? c->rank : -1; }
int q38_comm_size(const q38_comm* c) { return c ? c->world : 0; }

q38_status q38_comm_all_reduce(q38_ctx* ctx, q38_comm* c, const void* send, void* recv, int64_t count,
                               q38_dtype dtype) {
    q38_status st = check_pair(ctx, c, "all_reduce");
    if (st != Q38_OK) return st;
    if (count < 0 || (count > 0 && (!send || !recv)))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "all_reduce: bad buffer");
    if (count == 0) return Q38_OK;
    const ncclDataType_t t = dtype == Q38_BF16 ? ncclBfloat16 : dtype == Q38_F16 ? ncclFloat16 : ncclFloat32;
    return nccl_call(ctx, c, nccl().AllReduce(send, recv, static_cast<size_t>(count), t, ncclSum, c->nc, ctx->stream),
                     "all_reduce");
}

q38_status q38_tp_mlp(q38_ctx* ctx, q38_comm* c, const void* x, int64_t M, int64_t D, const uint32_t* gate_w,
                      const void* gate_s, const void* gate_b, const uint32_t* up_w, const void* up_s,
                      const void* up_b, const uint32_t* down_w, const void* down_s, const void* down_b,
                      int64_t F_local, q38_dtype dtype, int group_size, int bits, int chunks, void* y) {
    q38_status st = check_pair(ctx, c, "tp_mlp");
    if (st != Q38_OK) return st;
    if (dtype != Q38_BF16) return fail(ctx, Q38_ERR_UNSUPPORTED, "tp_mlp: bf16 activations and scales only");
    if (M < 0 || D <= 0 || F_local <= 0)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "tp_mlp: bad shape");
    if (M == 0) return Q38_OK;
    if (!x || !gate_w || !gate_s || !up_w || !up_s || !down_w || !down_s || !y)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "tp_mlp: null pointer");
    if (chunks <= 0) {
        // as many pieces as keep four waves of 256 x 256 down-projection tiles in each (a
        // smaller piece leaves tensor cores idle, and its all-reduce's blocks slow the next
        // piece, for longer than the overlap gains), at most 4
        const int64_t tiles = ((D + 255) / 256) * ((M + 255) / 256) / 2;
        chunks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(4, tiles / std::max(1, ctx->num_sms))));
    }
    // chunks of whole 128-token tiles
    int64_t step = (M + chunks - 1) / chunks;
    step = std::max<int64_t>(128, (step + 127) / 128 * 128);
    uint8_t* hbuf = nullptr;
    if ((st = comm_buffer(ctx, c, static_cast<size_t>(M) * F_local * 2, &hbuf)) != Q38_OK) return st;
    const Nccl& n = nccl();
    // h for all tokens in one pass (the gate/up products have the most tiles that way), then
    // the down projection piece by piece, each piece's all-reduce beside the next piece
    if ((st = q38_quantized_gate_up(ctx, x, M, D, Q38_BF16, gate_w, gate_s, gate_b, up_w, up_s, up_b, Q38_BF16,
                                    F_local, group_size, bits, Q38_MODE_AFFINE, hbuf)) != Q38_OK)
        return st;
    size_t ev = 0;
    for (int64_t m0 = 0; m0 < M; m0 += step) {
        const int64_t mi = std::min(step, M - m0);
        const uint8_t* hi = hbuf + static_cast<size_t>(m0) * F_local * 2;
        uint8_t* yi = static_cast<uint8_t*>(y) + static_cast<size_t>(m0) * D * 2;
        if ((st = q38_quantized_matmul(ctx, hi, mi, F_local, Q38_BF16, down_w, down_s, down_b, Q38_BF16, D, 1,
                                       group_size, bits, Q38_MODE_AFFINE, yi)) != Q38_OK)
            return st;
        if (c->world == 1) continue;
        // the all-reduce of this piece on the communicator's stream, after its product
        cudaEvent_t e = comm_event(c, ev++);
        if (!e || cudaEventRecord(e, ctx->stream) != cudaSuccess || cudaStreamWaitEvent(c->stream, e, 0) != cudaSuccess)
            return check_launch(ctx, "tp_mlp: stream ordering");
        if ((st = nccl_call(ctx, c, n.AllReduce(yi, yi, static_cast<size_t>(mi) * D, ncclBfloat16, ncclSum, c->nc,
                                                c->stream),
                            "tp_mlp all_reduce")) != Q38_OK)
            return st;
    }
    if (c->world > 1) {
        // the context's stream continues after the last all-reduce
        if (cudaEventRecord(c->joined, c->stream) != cudaSuccess || cudaStreamWaitEvent(ctx->stream, c->joined, 0) != cudaSuccess)
            return check_launch(ctx, "tp_mlp: stream join");
    }
    return Q38_OK;
}

q38_status q38_ep_switch_glu(q38_ctx* ctx, q38_comm* c, const void* x, int64_t T, int64_t H, int64_t I, int64_t E,
                             int top_k, const int32_t* indices, const void* scores, const uint32_t* gate_w,
                             const void* gate_s, const void* gate_b, const uint32_t* up_w, const void* up_s,
                             const void* up_b, const uint32_t* down_w, const void* down_s, const void* down_b,
                             q38_dtype dtype, int group_size, int bits, int64_t capacity, void* out) {
    q38_status st = check_pair(ctx, c, "ep_switch_glu");
    if (st != Q38_OK) return st;
    const int W = c->world;
    if (dtype != Q38_BF16) return fail(ctx, Q38_ERR_UNSUPPORTED, "ep_switch_glu: bf16 only");
    if (T < 0 || H <= 0 || H % 8 || I <= 0 || E < W || E % W || top_k < 1 || top_k > E || capacity < 1 || T > capacity)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT,
                    "ep_switch_glu: need E %% world == 0, 1 <= top_k <= E, T <= capacity, H %% 8 == 0");
    if (W > 32) return fail(ctx, Q38_ERR_UNSUPPORTED, "ep_switch_glu: at most 32 ranks");
    if (!x || !indices || !scores || !gate_w || !gate_s || !up_w || !up_s || !down_w || !down_s || !out)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "ep_switch_glu: null pointer");
    const int64_t C = capacity, epr = E / W, R = W * C;
    // The exchange is two collectives per chunk: an all-gather of every rank's capacity rows
    // (x, slot experts, scores), and after the local experts' work a reduce-scatter (bf16 sum)
    // of the partial outputs, whose block r is rank r's tokens.
    const size_t xrow = static_cast<size_t>(H) * 2;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += align_up(b, 256);
        return o;
    };
    const size_t o_xs = take(T < C ? C * xrow : 0), o_out = take(T < C ? C * xrow : 0), o_ids = take(C * top_k * 4),
                 o_sc = take(C * top_k * 2), o_xg = take(R * xrow), o_idg = take(R * top_k * 4),
                 o_scg = take(R * top_k * 2), o_part = take(R * xrow);
    uint8_t* b = nullptr;
    if ((st = comm_buffer(ctx, c, off, &b)) != Q38_OK) return st;
    const uint8_t* xsend = static_cast<const uint8_t*>(x);
    uint8_t* obuf = T < C ? b + o_out : static_cast<uint8_t*>(out);
    if (T < C) {
        if (T > 0 && cudaMemcpyAsync(b + o_xs, x, T * xrow, cudaMemcpyDeviceToDevice, ctx->stream) != cudaSuccess)
            return check_launch(ctx, "ep_switch_glu: staging");
        xsend = b + o_xs;
    }
    int32_t* ids = reinterpret_cast<int32_t*>(b + o_ids);
    __nv_bfloat16* sc = reinterpret_cast<__nv_bfloat16*>(b + o_sc);
    cudaLaunchAttribute attr[1];
    {
        cudaLaunchConfig_t cfg = pdl_cfg(dim3(static_cast<unsigned>(std::min<int64_t>((C * top_k + 255) / 256, 1184))),
                                         dim3(256), ctx->stream, attr);
        if (cudaLaunchKernelEx(&cfg, ep_own_meta, indices, static_cast<const __nv_bfloat16*>(scores),
                               static_cast<int>(T), static_cast<int>(C), top_k, ids, sc) != cudaSuccess)
            return check_launch(ctx, "ep_own_meta");
    }
    const Nccl& n = nccl();
    uint8_t* xg = b + o_xg;
    int32_t* idg = reinterpret_cast<int32_t*>(b + o_idg);
    __nv_bfloat16* scg = reinterpret_cast<__nv_bfloat16*>(b + o_scg);
    uint8_t* part = b + o_part;
    int NCH = 1;
    {
        const bool big = static_cast<double>(W - 1) * C * xrow >= 64.0 * (1 << 20);
        const double pairs_per_expert = static_cast<double>(C) * W * top_k / E;
        if (big && C % 2 == 0 && pairs_per_expert >= 256.0) NCH = 2;
    }
    if (ctx->ep_chunks > 0) NCH = C % ctx->ep_chunks == 0 ? ctx->ep_chunks : 1;
    const int64_t Cc = C / NCH, Rc = W * Cc;
    size_t ev = 0;
    auto order = [&](cudaStream_t from, cudaStream_t to) -> q38_status {
        cudaEvent_t e = comm_event(c, ev++);
        if (!e || cudaEventRecord(e, from) != cudaSuccess || cudaStreamWaitEvent(to, e, 0) != cudaSuccess)
            return check_launch(ctx, "ep_switch_glu: stream ordering");
        return Q38_OK;
    };
    // chunk q's rows [q*Cc, (q+1)*Cc) of every rank, gathered rank-major into chunk q's region
    auto gather = [&](int q) -> q38_status {
        const int64_t r0 = q * Cc;
        n.GroupStart();
        n.AllGather(xsend + r0 * xrow, xg + q * Rc * xrow, Cc * H, ncclBfloat16, c->nc, c->stream);
        n.AllGather(ids + r0 * top_k, idg + q * Rc * top_k, Cc * top_k, ncclInt32, c->nc, c->stream);
        n.AllGather(sc + r0 * top_k, scg + q * Rc * top_k, Cc * top_k, ncclBfloat16, c->nc, c->stream);
        return nccl_call(ctx, c, n.GroupEnd(), "ep_switch_glu gather");
    };
    // every rank's partial sums of chunk q summed into each token's home rank
    auto scatter = [&](int q) -> q38_status {
        return nccl_call(ctx, c,
                         n.ReduceScatter(part + q * Rc * xrow, obuf + q * Cc * xrow, Cc * H, ncclBfloat16, ncclSum,
                                         c->nc, c->stream),
                         "ep_switch_glu reduce-scatter");
    };
    std::vector<cudaEvent_t> landed(NCH, nullptr);
    auto mark = [&](int q) -> q38_status {
        landed[q] = comm_event(c, ev++);
        if (!landed[q] || cudaEventRecord(landed[q], c->stream) != cudaSuccess)
            return check_launch(ctx, "ep_switch_glu: stream ordering");
        return Q38_OK;
    };
    if ((st = order(ctx->stream, c->stream)) != Q38_OK) return st;  // staging and metadata
    if ((st = gather(0)) != Q38_OK || (st = mark(0)) != Q38_OK) return st;
    for (int q = 0; q < NCH; ++q) {
        if (cudaStreamWaitEvent(ctx->stream, landed[q], 0) != cudaSuccess)
            return check_launch(ctx, "ep_switch_glu: stream ordering");
        {
            cudaLaunchConfig_t cfg = pdl_cfg(dim3(static_cast<unsigned>(std::min<int64_t>((Rc * top_k + 255) / 256, 1184))),
                                             dim3(256), ctx->stream, attr);
            if (cudaLaunchKernelEx(&cfg, ep_localize, idg + q * Rc * top_k, static_cast<int>(Rc * top_k),
                                   static_cast<int>(E), static_cast<int>(epr), c->rank) != cudaSuccess)
                return check_launch(ctx, "ep_localize");
        }
        // this rank's experts over chunk q's rows (slots of other ranks' experts are -1)
        if ((st = q38_switch_glu(ctx, xg + q * Rc * xrow, Rc, H, I, epr, top_k, idg + q * Rc * top_k,
                                 scg + q * Rc * top_k, gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s,
                                 down_b, dtype, group_size, bits, part + q * Rc * xrow)) != Q38_OK)
            return st;
        if (q + 1 < NCH && ((st = gather(q + 1)) != Q38_OK || (st = mark(q + 1)) != Q38_OK)) return st;
        if ((st = order(ctx->stream, c->stream)) != Q38_OK) return st;  // chunk q computed
        if ((st = scatter(q)) != Q38_OK) return st;
    }
    if (cudaEventRecord(c->joined, c->stream) != cudaSuccess || cudaStreamWaitEvent(ctx->stream, c->joined, 0) != cudaSuccess)
        return check_launch(ctx, "ep_switch_glu: stream join");
    if (T < C && T > 0 &&
        cudaMemcpyAsync(out, obuf, T * xrow, cudaMemcpyDeviceToDevice, ctx->stream) != cudaSuccess)
        return check_launch(ctx, "ep_switch_glu: output copy");
    return Q38_OK;
}

}  // extern "C"
