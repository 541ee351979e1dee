"""Python binding of libq38 (the sm_100a MLX-affine quantized-matmul library).

This is a thin ctypes layer over the C ABI declared in include/q38.h.  Tensors are
torch CUDA tensors (torch provides device memory and streams only); every call goes
to libq38.so on the tensor's device and current torch stream.  There is no fallback:
if libq38.so is missing, importing this module raises.

Operator functions mirror the MLX operators the reference calls (argument names and
meaning as at the reference call sites); the module classes mirror MLXNN/MLXLMCommon's
QuantizedLinear, QuantizedSwitchLinear and SwitchGLU and the reference's
Qwen38HadamardQuantizedLinear.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libq38.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"libq38.so not found at {LIB_PATH}; build it with "
                      f"python {os.path.join(_HERE, 'build.py')}")

_lib = C.CDLL(LIB_PATH)

Q38_OK = 0
_STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "cuda error", 4: "out of memory",
           5: "device wait timed out", 6: "communication error"}
BF16, F16, F32 = 0, 1, 2
_DTYPE = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32}

_P, _I, _i, _S = C.c_void_p, C.c_int64, C.c_int, C.c_size_t


def _sig(name, args, res=C.c_int):
    fn = getattr(_lib, name)
    fn.argtypes = args
    fn.restype = res
    return fn


_sig("q38_version", [])
_sig("q38_status_string", [_i], C.c_char_p)
_sig("q38_ctx_create", [_i, C.POINTER(_P)])
_sig("q38_ctx_destroy", [_P])
_sig("q38_ctx_set_stream", [_P, _P])
_sig("q38_ctx_get_stream", [_P], _P)
_sig("q38_ctx_reserve", [_P, _S])
_sig("q38_ctx_workspace_bytes", [_P], _S)
_sig("q38_ctx_check_device", [_P])
_sig("q38_last_error", [_P], C.c_char_p)
_sig("q38_ctx_test_wait_timeout", [_P, _I])
_sig("q38_ctx_set_deterministic", [_P, _i])
_sig("q38_ctx_set_ep_chunks", [_P, _i])
_sig("q38_quantized_matmul", [_P, _P, _I, _I, _i, _P, _P, _P, _i, _I, _i, _i, _i, _i, _P])
_sig("q38_quantized_embedding", [_P, _P, _I, _P, _P, _P, _i, _I, _I, _i, _i, _i, _P, _i])
_sig("q38_hadamard_quantized_embedding", [_P, _P, _I, _P, _P, _P, _i, _I, _I, _i, _i, _i, _P, _i, _P])
_sig("q38_hadamard_quantized_gate_up", [_P, _P, _I, _I, _i, _P, _i, _P, _P, _P, _P, _P, _P, _i, _I, _i, _i, _P])
_sig("q38_quantized_gate_up", [_P, _P, _I, _I, _i, _P, _P, _P, _P, _P, _P, _i, _I, _i, _i, _i, _P])
_sig("q38_gather_quantized_matmul",
     [_P, _P, _I, _I, _I, _i, _P, _P, _P, _i, _I, _I, _P, _P, _I, _i, _i, _i, _i, _i, _P])
_sig("q38_dequantize", [_P, _P, _P, _P, _i, _I, _I, _i, _i, _i, _P, _i])
_sig("q38_quantize", [_P, _P, _i, _I, _I, _i, _i, _i, _P, _P, _P, _i])
_sig("q38_unpack_codes", [_P, _P, _I, _I, _i, _P])
_sig("q38_hadamard_rotate", [_P, _P, _I, _I, _i, _P, _i, _i, _P])
_sig("q38_hadamard_quantized_matmul", [_P, _P, _I, _I, _i, _P, _i, _P, _P, _P, _i, _I, _i, _i, _P])
_sig("q38_moe_route", [_P, _P, _I, _I, _i, _P, _I, _i, _i, _P, _P, _P])
_sig("q38_moe_route_logits", [_P, _P, _I, _I, _i, _i, _P, _P, _P])
_sig("q38_moe_sort", [_P, _P, _I, _I, _P, _P])
_sig("q38_silu_mul", [_P, _P, _P, _I, _P])
_sig("q38_moe_dispatch_pack", [_P, _P, _I, _P, _P, _I, _i, _I, _P, _P])
_sig("q38_moe_combine", [_P, _P, _I, _P, _P, _P, _I, _i, _I, _P])
_sig("q38_moe_ep_plan", [_P, _P, _I, _i, _I, _i, _P, _P])
_sig("q38_moe_ep_pack", [_P, _P, _I, _P, _P, _I, _i, _I, _i, _P, _P, _I, _P, _I])
_sig("q38_moe_ep_reduce", [_P, _P, _I, _P, _I, _i, _P])
_U64 = C.c_uint64
_sig("q38_st_open", [C.c_char_p, C.POINTER(_P)])
_sig("q38_st_open_error", [], C.c_char_p)
_sig("q38_st_close", [_P], None)
_sig("q38_st_count", [_P], _I)
_sig("q38_st_find", [_P, C.c_char_p], _I)
_sig("q38_st_info", [_P, _I, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p), C.POINTER(_i), C.POINTER(_I),
                     C.POINTER(_U64)])
_sig("q38_st_data", [_P, _I], _P)
_sig("q38_st_metadata_count", [_P], _I)
_sig("q38_st_metadata_entry", [_P, _I, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p)])
_sig("q38_st_copy_to_device", [_P, _P, _I, _P, _U64])
_sig("q38_st_copy_block_to_device", [_P, _P, _I, _U64, _U64, _U64, _U64, _U64, _P, _U64])
_sig("q38_switch_glu", [_P, _P, _I, _I, _I, _I, _i, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _i, _i, _i, _P])
_sig("q38_sparse_moe", [_P, _P, _I, _I, _I, _I, _i, _i, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _i, _i, _i, _P, _P,
                        _P])
_sig("q38_shared_expert", [_P, _P, _I, _I, _I] + [_P] * 12 + [_i, _i, _i, _P, _P])


class _CommId(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 128)]


_sig("q38_comm_error", [], C.c_char_p)
_sig("q38_comm_get_unique_id", [C.POINTER(_CommId)])
_sig("q38_comm_init_rank", [C.POINTER(_CommId), _i, _i, _i, _i, C.POINTER(_P)])
_sig("q38_comm_destroy", [_P])
_sig("q38_comm_abort", [_P])
_sig("q38_comm_rank", [_P])
_sig("q38_comm_size", [_P])
_sig("q38_comm_all_reduce", [_P, _P, _P, _P, _I, _i])
_sig("q38_tp_mlp", [_P, _P, _P, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _i, _i, _i, _i, _P])
_sig("q38_ep_switch_glu", [_P, _P, _P, _I, _I, _I, _I, _i, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _i, _i, _i,
                           _I, _P])


class Q38Error(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS.get(status, status)}: {message}")
        self.status = status


class Q38ArgumentError(Q38Error, ValueError):
    pass


_ctx_lock = threading.Lock()
_ctxs: dict[tuple[int, int], int] = {}


def context(device: int | torch.device | None = None) -> int:
    """Context handle for `device` on this host thread (created on first use)."""
    if device is None:
        device = torch.cuda.current_device()
    if isinstance(device, torch.device):
        device = device.index if device.index is not None else torch.cuda.current_device()
    key = (threading.get_ident(), int(device))
    with _ctx_lock:
        h = _ctxs.get(key)
        if h is None:
            p = _P()
            st = _lib.q38_ctx_create(int(device), C.byref(p))
            if st != Q38_OK:
                raise Q38Error(st, f"context creation on device {device} failed")
            h = p.value
            _ctxs[key] = h
    return h


_tls = threading.local()
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _bind(t: torch.Tensor) -> int:
    """This thread's context for t's device, bound to the current torch stream."""
    dev = t.get_device()
    slots = getattr(_tls, "slots", None)
    if slots is None:
        slots = _tls.slots = {}
    ent = slots.get(dev)
    if ent is None:
        ent = slots[dev] = [context(dev), None]
    stream = _raw_stream(dev) if _raw_stream is not None else torch.cuda.current_stream(t.device).cuda_stream
    if stream != ent[1]:
        _lib.q38_ctx_set_stream(ent[0], stream)
        ent[1] = stream
    return ent[0]


def _check(ctx: int, st: int) -> None:
    if st != Q38_OK:
        msg = (_lib.q38_last_error(ctx) or b"").decode()
        if st in (1,):
            raise Q38ArgumentError(st, msg)
        raise Q38Error(st, msg)


def check_device(device=None) -> None:
    """Synchronise and raise if a kernel reported a timeout or an out-of-range index."""
    ctx = context(device)
    _lib.q38_ctx_set_stream(ctx, torch.cuda.current_stream(device).cuda_stream)
    slots = getattr(_tls, "slots", None)
    if slots:  # the context's stream was set here, not by _bind: bind again next time
        for ent in slots.values():
            if ent[0] == ctx:
                ent[1] = None
    _check(ctx, _lib.q38_ctx_check_device(ctx))


def set_deterministic(on: bool = True, device=None) -> None:
    """Bitwise reproducible decode products (ordered chunk sums) on this thread's context
    for `device`; off by default (arrival-order fp32 sums, about 1 us faster)."""
    ctx = context(device)
    _check(ctx, _lib.q38_ctx_set_deterministic(ctx, int(bool(on))))


def set_ep_chunks(chunks: int = 0, device=None) -> None:
    """Pieces of the expert-parallel exchange on this thread's context for `device` (1, 2
    or 4; 0 lets the library choose).  Every rank must use the same setting."""
    ctx = context(device)
    _check(ctx, _lib.q38_ctx_set_ep_chunks(ctx, int(chunks)))


def test_wait_timeout(limit_cycles: int, device=None) -> None:
    """Enqueue the bounded-wait self-test: a kernel waits for an mbarrier phase that never
    completes, with a limit of `limit_cycles` SM cycles, and records the expiry.  The next
    check_device() raises Q38Error with status 5 (device wait timed out)."""
    ctx = context(device)
    _lib.q38_ctx_set_stream(ctx, torch.cuda.current_stream(device).cuda_stream)
    slots = getattr(_tls, "slots", None)
    if slots:
        for ent in slots.values():
            if ent[0] == ctx:
                ent[1] = None
    _check(ctx, _lib.q38_ctx_test_wait_timeout(ctx, int(limit_cycles)))


def reserve(nbytes: int, device=None) -> None:
    ctx = context(device)
    _check(ctx, _lib.q38_ctx_reserve(ctx, int(nbytes)))


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _as_u32(w: torch.Tensor) -> torch.Tensor:
    if w.dtype == torch.int32:
        return w
    if w.dtype == torch.uint32:
        return w.view(torch.int32)
    raise ValueError("packed weight must be uint32 (or int32 bit-identical storage)")


# ----------------------------------------------------------------------- operators

def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                     biases: torch.Tensor | None = None, transpose: bool = True,
                     group_size: int = 64, bits: int = 4, mode: str = "affine",
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """MLX.quantizedMM: x[..., K] . dequant(w)^T -> [..., N] (transpose=true).  `out`
    (contiguous, x's dtype and device, [..., N]) receives the result instead of a new tensor."""
    if mode != "affine":
        raise Q38Error(2, f"mode {mode!r} is not implemented")
    _need(x, "x"), _need(w, "w"), _need(scales, "scales")
    if biases is not None:
        _need(biases, "biases")
    w = _as_u32(w)
    K = x.shape[-1]
    N = w.shape[0]
    M = x.numel() // K if K else 0
    if out is None:
        y = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
    else:
        _need(out, "out")
        if out.dtype != x.dtype or out.device != x.device or out.numel() != M * N or out.shape[-1] != N:
            raise ValueError(f"out must be {x.dtype} on {x.device} with {M} x {N} elements")
        y = out
    ctx = _bind(x)
    _check(ctx, _lib.q38_quantized_matmul(ctx, _ptr(x), M, K, _DTYPE[x.dtype], _ptr(w), _ptr(scales),
                                          _ptr(biases), _DTYPE[scales.dtype], N, int(transpose),
                                          group_size, bits, 0, _ptr(y)))
    return y


def quantized_embedding(ids: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                        biases: torch.Tensor | None = None, group_size: int = 64, bits: int = 4,
                        mode: str = "affine", out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Prequantized embedding lookup: ids [...] (int32) -> [..., K] = dequant(w)[ids]."""
    if mode != "affine":
        raise Q38Error(2, f"mode {mode!r} is not implemented")
    _need(ids, "ids"), _need(w, "w"), _need(scales, "scales")
    if biases is not None:
        _need(biases, "biases")
    if ids.dtype != torch.int32:
        raise ValueError("ids must be int32")
    w = _as_u32(w)
    rows = w.shape[0]
    K = w.shape[-1] * 32 // bits
    od = out_dtype or scales.dtype
    out = torch.empty(tuple(ids.shape) + (K,), dtype=od, device=w.device)
    ctx = _bind(w)
    _check(ctx, _lib.q38_quantized_embedding(ctx, _ptr(ids), ids.numel(), _ptr(w), _ptr(scales), _ptr(biases),
                                             _DTYPE[scales.dtype], rows, K, group_size, bits, 0, _ptr(out),
                                             _DTYPE[od]))
    return out


def hadamard_quantized_embedding(ids: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                                 biases: torch.Tensor | None, signs: torch.Tensor | None, block: int,
                                 group_size: int = 64, bits: int = 2, mode: str = "affine") -> torch.Tensor:
    """Rotated embedding lookup of Qwen38HadamardQuantizedEmbedding.callAsFunction
    (Bonsai2/Qwen38HadamardModules.swift:71-79): dequantized rows in the scales' dtype,
    then hadamardRotate(inverse=True)."""
    if mode != "affine":
        raise Q38Error(2, f"mode {mode!r} is not implemented")
    _need(ids, "ids"), _need(w, "w"), _need(scales, "scales")
    if biases is not None:
        _need(biases, "biases")
    if signs is not None:
        _need(signs, "signs")
        if signs.dtype != torch.float32:
            signs = signs.float().contiguous()
    if ids.dtype != torch.int32:
        raise ValueError("ids must be int32")
    w = _as_u32(w)
    rows = w.shape[0]
    K = w.shape[-1] * 32 // bits
    out = torch.empty(tuple(ids.shape) + (K,), dtype=scales.dtype, device=w.device)
    ctx = _bind(w)
    _check(ctx, _lib.q38_hadamard_quantized_embedding(ctx, _ptr(ids), ids.numel(), _ptr(w), _ptr(scales),
                                                      _ptr(biases), _DTYPE[scales.dtype], rows, K, group_size,
                                                      bits, 0, _ptr(signs), block, _ptr(out)))
    return out


def quantized_gate_up(x: torch.Tensor, gate, up, group_size: int = 64, bits: int = 4,
                      mode: str = "affine") -> torch.Tensor:
    """silu(gate(x)) * up(x) of a gated MLP, each projection a bf16 QuantizedLinear
    (transpose=true): gate and up are (w, scales, biases) triples of one shape.  Decode-sized
    x (<= 16 tokens) reads both weights in one pass with the SiLU-gate in its epilogue."""
    if mode != "affine":
        raise Q38Error(2, f"mode {mode!r} is not implemented")
    wg, sg, bg = gate
    wu, su, bu = up
    for t, n in ((x, "x"), (wg, "gate w"), (sg, "gate scales"), (wu, "up w"), (su, "up scales")):
        _need(t, n)
    for t, n in ((bg, "gate biases"), (bu, "up biases")):
        if t is not None:
            _need(t, n)
    wg, wu = _as_u32(wg), _as_u32(wu)
    if wg.shape != wu.shape or sg.shape != su.shape:
        raise ValueError("quantized_gate_up: gate and up weights must have one shape")
    K = x.shape[-1]
    N = wg.shape[0]
    M = x.numel() // K if K else 0
    h = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
    ctx = _bind(x)
    _check(ctx, _lib.q38_quantized_gate_up(ctx, _ptr(x), M, K, _DTYPE[x.dtype], _ptr(wg), _ptr(sg), _ptr(bg),
                                           _ptr(wu), _ptr(su), _ptr(bu), _DTYPE[sg.dtype], N, group_size, bits,
                                           0, _ptr(h)))
    return h


def hadamard_quantized_gate_up(x: torch.Tensor, signs: torch.Tensor | None, block: int, gate, up,
                               group_size: int = 64, bits: int = 2) -> torch.Tensor:
    """silu(gate(xr)) * up(xr) with xr = hadamardRotate(x, signs, block): the gate and up
    Qwen38HadamardQuantizedLinear projections of a Bonsai 2 MLP
    (Bonsai2/Qwen38HadamardModules.swift:37-39) when both carry the same signs (the pack
    stores one sign vector per input width).  gate and up are (w, scales, biases) triples."""
    wg, sg, bg = gate
    wu, su, bu = up
    for t, n in ((x, "x"), (wg, "gate w"), (sg, "gate scales"), (wu, "up w"), (su, "up scales")):
        _need(t, n)
    for t, n in ((bg, "gate biases"), (bu, "up biases")):
        if t is not None:
            _need(t, n)
    if signs is not None:
        _need(signs, "signs")
        if signs.dtype != torch.float32:
            signs = signs.float().contiguous()
    wg, wu = _as_u32(wg), _as_u32(wu)
    if wg.shape != wu.shape or sg.shape != su.shape:
        raise ValueError("hadamard_quantized_gate_up: gate and up weights must have one shape")
    K = x.shape[-1]
    N = wg.shape[0]
    M = x.numel() // K if K else 0
    h = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
    ctx = _bind(x)
    _check(ctx, _lib.q38_hadamard_quantized_gate_up(ctx, _ptr(x), M, K, _DTYPE[x.dtype], _ptr(signs), block,
                                                    _ptr(wg), _ptr(sg), _ptr(bg), _ptr(wu), _ptr(su), _ptr(bu),
                                                    _DTYPE[sg.dtype], N, group_size, bits, _ptr(h)))
    return h


def gather_qmm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
               biases: torch.Tensor | None = None, lhs_indices: torch.Tensor | None = None,
               rhs_indices: torch.Tensor | None = None, transpose: bool = True,
               group_size: int = 64, bits: int = 4, mode: str = "affine",
               sorted_indices: bool = False) -> torch.Tensor:
    """MLX.gatherQuantizedMM with flattened batch: x [Bx, M, K], w [E, N, K*bits/32],
    rhs_indices [P] (int32), lhs_indices [P] or None -> out [P, M, N]."""
    if mode != "affine":
        raise Q38Error(2, f"mode {mode!r} is not implemented")
    if rhs_indices is None:
        raise ValueError("rhs_indices is required")
    _need(x, "x"), _need(w, "w"), _need(scales, "scales"), _need(rhs_indices, "rhs_indices")
    w = _as_u32(w)
    Bx, M, K = x.shape
    E, N = w.shape[0], w.shape[1]
    P = rhs_indices.numel()
    out = torch.empty((P, M, N), dtype=x.dtype, device=x.device)
    ctx = _bind(x)
    _check(ctx, _lib.q38_gather_quantized_matmul(
        ctx, _ptr(x), Bx, M, K, _DTYPE[x.dtype], _ptr(w), _ptr(scales), _ptr(biases),
        _DTYPE[scales.dtype], E, N, _ptr(lhs_indices), _ptr(rhs_indices), P, int(transpose),
        group_size, bits, 0, int(sorted_indices), _ptr(out)))
    return out


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor | None = None,
               group_size: int = 64, bits: int = 4, mode: str = "affine",
               out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """MLX.dequantized: w [..., K*bits/32] -> [..., K] = scale*q + bias."""
    if mode != "affine":
        raise Q38Error(2, f"mode {mode!r} is not implemented")
    _need(w, "w"), _need(scales, "scales")
    w = _as_u32(w)
    K = w.shape[-1] * 32 // bits
    rows = w.numel() // w.shape[-1]
    od = out_dtype or scales.dtype
    out = torch.empty(w.shape[:-1] + (K,), dtype=od, device=w.device)
    ctx = _bind(w)
    _check(ctx, _lib.q38_dequantize(ctx, _ptr(w), _ptr(scales), _ptr(biases), _DTYPE[scales.dtype],
                                    rows, K, group_size, bits, 0, _ptr(out), _DTYPE[od]))
    return out


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4, mode: str = "affine",
             scales_dtype: torch.dtype | None = None):
    """mx.quantize(mode="affine"): w [..., K] -> (codes uint32 [..., K*bits/32], scales, biases)."""
    if mode != "affine":
        raise Q38Error(2, f"mode {mode!r} is not implemented")
    _need(w, "w")
    K = w.shape[-1]
    rows = w.numel() // K
    sd = scales_dtype or (w.dtype if w.dtype != torch.float32 else torch.bfloat16)
    codes = torch.empty(w.shape[:-1] + (K * bits // 32,), dtype=torch.int32, device=w.device)
    s = torch.empty(w.shape[:-1] + (K // group_size,), dtype=sd, device=w.device)
    b = torch.empty_like(s)
    ctx = _bind(w)
    _check(ctx, _lib.q38_quantize(ctx, _ptr(w), _DTYPE[w.dtype], rows, K, group_size, bits, 0,
                                  _ptr(codes), _ptr(s), _ptr(b), _DTYPE[sd]))
    return codes.view(torch.uint32), s, b


def unpack_codes(w: torch.Tensor, bits: int) -> torch.Tensor:
    _need(w, "w")
    w = _as_u32(w)
    K = w.shape[-1] * 32 // bits
    rows = w.numel() // w.shape[-1]
    q = torch.empty(w.shape[:-1] + (K,), dtype=torch.uint8, device=w.device)
    ctx = _bind(w)
    _check(ctx, _lib.q38_unpack_codes(ctx, _ptr(w), rows, K, bits, _ptr(q)))
    return q


def hadamard_rotate(x: torch.Tensor, signs: torch.Tensor | None, block: int,
                    inverse: bool = False) -> torch.Tensor:
    """hadamardRotate of Bonsai2/Qwen38HadamardModules.swift:10-19."""
    _need(x, "x")
    if signs is not None:
        _need(signs, "signs")
        if signs.dtype != torch.float32:
            signs = signs.float().contiguous()
    D = x.shape[-1]
    rows = x.numel() // D
    y = torch.empty_like(x)
    ctx = _bind(x)
    _check(ctx, _lib.q38_hadamard_rotate(ctx, _ptr(x), rows, D, _DTYPE[x.dtype], _ptr(signs), block,
                                         int(inverse), _ptr(y)))
    return y


def moe_route(x: torch.Tensor, wr: torch.Tensor, top_k: int, normalize: bool = True,
              want_probs: bool = False):
    """Router of Qwen4ExpSparseMoE (FlashNext/Qwen4ExpSparseMoE.swift:208-214, :275-281):
    x bf16 [T, H], wr bf16 [E, H] -> (indices int32 [T, k], scores bf16 [T, k][, probs [T, E]])
    in canonical order (probability descending, expert id ascending on ties)."""
    _need(x, "x"), _need(wr, "wr")
    H = x.shape[-1]
    T = x.numel() // H
    E = wr.shape[0]
    idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    sc = torch.empty((T, top_k), dtype=torch.bfloat16, device=x.device)
    pr = torch.empty((T, E), dtype=torch.bfloat16, device=x.device) if want_probs else None
    ctx = _bind(x)
    _check(ctx, _lib.q38_moe_route(ctx, _ptr(x), T, H, _DTYPE[x.dtype], _ptr(wr), E, top_k, int(normalize),
                                   _ptr(idx), _ptr(sc), _ptr(pr)))
    return (idx, sc, pr) if want_probs else (idx, sc)


def moe_route_logits(logits: torch.Tensor, top_k: int, normalize: bool = True, want_probs: bool = False):
    """The router's selection from given bf16 logits [T, E]."""
    _need(logits, "logits")
    T, E = logits.shape
    idx = torch.empty((T, top_k), dtype=torch.int32, device=logits.device)
    sc = torch.empty((T, top_k), dtype=torch.bfloat16, device=logits.device)
    pr = torch.empty((T, E), dtype=torch.bfloat16, device=logits.device) if want_probs else None
    ctx = _bind(logits)
    _check(ctx, _lib.q38_moe_route_logits(ctx, _ptr(logits), T, E, top_k, int(normalize), _ptr(idx), _ptr(sc),
                                          _ptr(pr)))
    return (idx, sc, pr) if want_probs else (idx, sc)


def moe_sort(indices: torch.Tensor, num_experts: int):
    """Stable sort of the flat (token, slot) pairs by expert -> (perm [P], offsets [E + 1])."""
    _need(indices, "indices")
    P = indices.numel()
    perm = torch.empty(P, dtype=torch.int32, device=indices.device)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=indices.device)
    ctx = _bind(indices)
    _check(ctx, _lib.q38_moe_sort(ctx, _ptr(indices), P, num_experts, _ptr(perm), _ptr(offsets)))
    return perm, offsets


def switch_glu(x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor, gate, up, down,
               group_size: int = 64, bits: int = 3) -> torch.Tensor:
    """SwitchGLU + weightedExpertSum (FlashNext/Qwen4ExpSparseMoE.swift:294): gate/up/down are
    (codes, scales, biases) triples of expert-stacked weights; x bf16 [T, H] -> bf16 [T, H]."""
    _need(x, "x"), _need(indices, "indices"), _need(scores, "scores")
    T, H = x.shape
    k = indices.shape[-1]
    gw, gs, gb = gate
    uw, us, ub = up
    dw, ds, db = down
    E, I = gw.shape[0], gw.shape[1]
    out = torch.empty_like(x)
    ctx = _bind(x)
    _check(ctx, _lib.q38_switch_glu(ctx, _ptr(x), T, H, I, E, k, _ptr(indices), _ptr(scores),
                                    _ptr(_as_u32(gw)), _ptr(gs), _ptr(gb), _ptr(_as_u32(uw)), _ptr(us), _ptr(ub),
                                    _ptr(_as_u32(dw)), _ptr(ds), _ptr(db), _DTYPE[x.dtype], group_size, bits,
                                    _ptr(out)))
    return out


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """h = bf16(silu(g) * u), fp32 inside (the MLP's SiLU-gate)."""
    _need(g, "g"), _need(u, "u")
    if g.shape != u.shape or g.dtype != torch.bfloat16 or u.dtype != torch.bfloat16:
        raise ValueError("silu_mul: g and u must be bf16 tensors of one shape")
    h = torch.empty_like(g)
    ctx = _bind(g)
    _check(ctx, _lib.q38_silu_mul(ctx, _ptr(g), _ptr(u), g.numel(), _ptr(h)))
    return h


def moe_dispatch_pack(x: torch.Tensor, indices: torch.Tensor, perm: torch.Tensor, experts_per_rank: int):
    """Rows of x and rank-local expert ids of the (token, slot) pairs in perm's order."""
    _need(x, "x"), _need(indices, "indices"), _need(perm, "perm")
    T, H = x.shape
    k = indices.shape[-1]
    P = perm.numel()
    rows = torch.empty((P, H), dtype=x.dtype, device=x.device)
    local = torch.empty((P,), dtype=torch.int32, device=x.device)
    ctx = _bind(x)
    _check(ctx, _lib.q38_moe_dispatch_pack(ctx, _ptr(x), H, _ptr(indices), _ptr(perm), P, k, experts_per_rank,
                                           _ptr(rows), _ptr(local)))
    return rows, local


def moe_combine(y: torch.Tensor, perm: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor,
                num_experts: int) -> torch.Tensor:
    """weightedExpertSum of expert outputs held in perm's order: [P, H] -> [T, H]."""
    _need(y, "y"), _need(perm, "perm"), _need(indices, "indices"), _need(scores, "scores")
    T, k = indices.shape
    H = y.shape[-1]
    out = torch.empty((T, H), dtype=torch.bfloat16, device=indices.device)
    ctx = _bind(indices)
    _check(ctx, _lib.q38_moe_combine(ctx, _ptr(y), H, _ptr(perm), _ptr(indices), _ptr(scores), T, k,
                                     num_experts, _ptr(out)))
    return out


def moe_ep_plan(indices: torch.Tensor, experts_per_rank: int, world: int):
    """-> (rowpos int32 [T, world], counts int32 [world]) of the one-row-per-(token, rank)
    expert-parallel dispatch."""
    _need(indices, "indices")
    T, k = indices.shape
    rowpos = torch.empty((T, world), dtype=torch.int32, device=indices.device)
    counts = torch.empty((world,), dtype=torch.int32, device=indices.device)
    ctx = _bind(indices)
    _check(ctx, _lib.q38_moe_ep_plan(ctx, _ptr(indices), T, k, experts_per_rank, world, _ptr(rowpos), _ptr(counts)))
    return rowpos, counts


def moe_ep_pack(x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor, rowpos: torch.Tensor,
                experts_per_rank: int, rows_total: int) -> torch.Tensor:
    """-> packed bf16 [rows_total, H + 4k rounded up to 8]: each row = the token's activations,
    then its slot metadata (k rank-local expert ids or -1, then k score bit patterns, as
    int32)."""
    _need(x, "x"), _need(indices, "indices"), _need(scores, "scores"), _need(rowpos, "rowpos")
    T, H = x.shape
    k = indices.shape[1]
    world = rowpos.shape[1]
    ld = H + (4 * k + 7) // 8 * 8  # rows stay 16-byte aligned
    packed = torch.empty((rows_total, ld), dtype=x.dtype, device=x.device)
    meta = packed[:, H:]
    ctx = _bind(x)
    _check(ctx, _lib.q38_moe_ep_pack(ctx, _ptr(x), H, _ptr(indices), _ptr(scores), T, k, experts_per_rank, world,
                                     _ptr(rowpos), _ptr(packed), ld, meta.data_ptr() if rows_total else None, ld // 2))
    return packed


def split_ep_packed(packed: torch.Tensor, H: int, k: int):
    """packed [R, H + 4k (+ padding)] -> (rows [R, H], rank-local expert ids int32 [R, k],
    scores bf16 [R, k])."""
    rows = packed[:, :H].contiguous()
    meta = packed[:, H:H + 4 * k].contiguous().view(torch.int32)
    return rows, meta[:, :k].contiguous(), meta[:, k:].to(torch.int16).view(torch.bfloat16).contiguous()


def moe_ep_reduce(partial: torch.Tensor, rowpos: torch.Tensor) -> torch.Tensor:
    _need(partial, "partial"), _need(rowpos, "rowpos")
    T, world = rowpos.shape
    H = partial.shape[1]
    out = torch.empty((T, H), dtype=torch.bfloat16, device=rowpos.device)
    ctx = _bind(rowpos)
    _check(ctx, _lib.q38_moe_ep_reduce(ctx, _ptr(partial), H, _ptr(rowpos), T, world, _ptr(out)))
    return out


# ------------------------------------------------------------------------- modules

class QuantizedLinear:
    """MLXNN.QuantizedLinear: parameters `weight` (packed uint32), `scales`, `biases`,
    optional `bias`; callAsFunction = quantizedMM(x, weight, ..., transpose: true) + bias."""

    def __init__(self, weight, scales, biases=None, bias=None, group_size: int = 64, bits: int = 4,
                 mode: str = "affine"):
        self.weight, self.scales, self.biases, self.bias = weight, scales, biases, bias
        self.group_size, self.bits, self.mode = group_size, bits, mode

    @property
    def shape(self):
        return (self.weight.shape[0], self.weight.shape[-1] * 32 // self.bits)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        y = quantized_matmul(x, self.weight, self.scales, self.biases, True, self.group_size,
                             self.bits, self.mode)
        return y if self.bias is None else y + self.bias


class QuantizedEmbedding:
    """Qwen4ExpPrequantizedEmbedding (FlashNext/Qwen4ExpPrequantized.swift:108-160):
    parameters `weight` (packed uint32 [count, dims*bits/32]), `scales`, `biases`;
    callAsFunction gathers and dequantizes rows, asLinear is the tied output projection."""

    def __init__(self, weight, scales, biases=None, group_size: int = 64, bits: int = 4, mode: str = "affine"):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits, self.mode = group_size, bits, mode

    @property
    def shape(self):
        return (self.weight.shape[0], self.weight.shape[-1] * 32 // self.bits)

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        return quantized_embedding(ids.to(torch.int32).contiguous(), self.weight, self.scales, self.biases,
                                   self.group_size, self.bits, self.mode)

    def as_linear(self, x: torch.Tensor) -> torch.Tensor:
        return quantized_matmul(x, self.weight, self.scales, self.biases, True, self.group_size, self.bits,
                                self.mode)


class HadamardQuantizedEmbedding(QuantizedEmbedding):
    """Qwen38HadamardQuantizedEmbedding (Bonsai2/Qwen38HadamardModules.swift:49-80): the
    source embedding's tables, looked up, dequantized and rotated back (signs after the
    transform).  The reference class defines no output projection of its own."""

    def __init__(self, source: QuantizedEmbedding, signs: torch.Tensor | None, block: int):
        super().__init__(source.weight, source.scales, source.biases, source.group_size, source.bits, source.mode)
        self.signs = None if signs is None else signs.float().contiguous()
        self.block = block

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        return hadamard_quantized_embedding(ids.to(torch.int32).contiguous(), self.weight, self.scales,
                                            self.biases, self.signs, self.block, self.group_size, self.bits,
                                            self.mode)

    def as_linear(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError("the rotated embedding has no tied output projection")


class HadamardQuantizedLinear(QuantizedLinear):
    """Qwen38HadamardQuantizedLinear (Bonsai2/Qwen38HadamardModules.swift:24-40): rotate the
    input (signs before the transform), round to x's dtype, then the quantized product."""

    def __init__(self, source: QuantizedLinear, signs: torch.Tensor | None, block: int):
        super().__init__(source.weight, source.scales, source.biases, source.bias,
                         source.group_size, source.bits, source.mode)
        self.signs = None if signs is None else signs.float().contiguous()
        self.block = block

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        _need(x, "x")
        K = x.shape[-1]
        M = x.numel() // K
        N = self.weight.shape[0]
        y = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
        ctx = _bind(x)
        _check(ctx, _lib.q38_hadamard_quantized_matmul(
            ctx, _ptr(x), M, K, _DTYPE[x.dtype], _ptr(self.signs), self.block, _ptr(_as_u32(self.weight)),
            _ptr(self.scales), _ptr(self.biases), _DTYPE[self.scales.dtype], N, self.group_size,
            self.bits, _ptr(y)))
        return y if self.bias is None else y + self.bias


class QuantizedSwitchLinear:
    """MLXLMCommon.QuantizedSwitchLinear: expert-stacked packed weight [E, N, K*bits/32];
    callAsFunction(x, indices) = gatherQuantizedMM(x, weight, ..., rhsIndices: indices)."""

    def __init__(self, weight, scales, biases=None, group_size: int = 64, bits: int = 4,
                 mode: str = "affine"):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits, self.mode = group_size, bits, mode

    def __call__(self, x: torch.Tensor, indices: torch.Tensor, sorted_indices: bool = False):
        """x [T, K] (one row per token), indices [T, k] -> [T, k, N]."""
        T, K = x.shape
        k = indices.shape[-1]
        idx = indices.reshape(-1).to(torch.int32).contiguous()
        lhs = torch.arange(T, device=x.device, dtype=torch.int32).repeat_interleave(k)
        out = gather_qmm(x.reshape(T, 1, K).contiguous(), self.weight, self.scales, self.biases,
                         lhs, idx, True, self.group_size, self.bits, self.mode, sorted_indices)
        return out.reshape(T, k, -1)


class QuantizedMLP:
    """The gated MLP of the dense and Bonsai 2 models, down(silu(gate(x)) * up(x)), over
    QuantizedLinear projections (Qwen3.5's MLP; Bonsai 2 packs make each projection a
    HadamardQuantizedLinear, Bonsai2/Qwen38HadamardModules.swift:24-40).  Gate and up run as
    one pass over both weights (quantized_gate_up); rotated gate and up with equal signs and
    block share one rotation (hadamard_quantized_gate_up).  Other pairs are composed from
    the two projections and silu_mul.  Without biases on the Linear layers (`bias`), as in
    those models; a Linear bias falls back to the composition."""

    def __init__(self, gate: QuantizedLinear, up: QuantizedLinear, down: QuantizedLinear):
        self.gate, self.up, self.down = gate, up, down
        g, u = gate, up
        same = (type(g) is type(u) and g.weight.shape == u.weight.shape and g.scales.dtype == u.scales.dtype and
                (g.group_size, g.bits, g.mode) == (u.group_size, u.bits, u.mode) and g.mode == "affine" and
                g.bias is None and u.bias is None and (g.biases is None) == (u.biases is None))
        if same and isinstance(g, HadamardQuantizedLinear):
            same = g.block == u.block and ((g.signs is None and u.signs is None) or
                                           (g.signs is not None and u.signs is not None and torch.equal(g.signs, u.signs)))
        self._fused = same

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        g, u = self.gate, self.up
        if self._fused and x.dtype == torch.bfloat16:
            gw, uw = (g.weight, g.scales, g.biases), (u.weight, u.scales, u.biases)
            if isinstance(g, HadamardQuantizedLinear):
                h = hadamard_quantized_gate_up(x, g.signs, g.block, gw, uw, g.group_size, g.bits)
            else:
                h = quantized_gate_up(x, gw, uw, g.group_size, g.bits)
        else:
            h = silu_mul(g(x), u(x))
        return self.down(h)


class SwitchGLU:
    """MLXLMCommon.SwitchGLU over QuantizedSwitchLinear gate/up/down projections with the
    weighted expert sum of Qwen4ExpSparseMoE: __call__(x, indices, scores) -> [T, H]."""

    def __init__(self, gate: QuantizedSwitchLinear, up: QuantizedSwitchLinear, down: QuantizedSwitchLinear):
        self.gate, self.up, self.down = gate, up, down

    def __call__(self, x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        g, u, d = self.gate, self.up, self.down
        return switch_glu(x, indices, scores, (g.weight, g.scales, g.biases), (u.weight, u.scales, u.biases),
                          (d.weight, d.scales, d.biases), g.group_size, g.bits)


class SparseMoeBlock:
    """Qwen4ExpSparseMoE.callAsFunction (FlashNext/Qwen4ExpSparseMoE.swift:275-298): router
    (unquantized gate Linear, softmax, top-k, renormalisation) then SwitchGLU; with
    `shared_expert` (a QuantizedMLP) and `shared_expert_gate` (a QuantizedLinear [1, H]) the
    output adds sigmoid(shared_expert_gate(x)) * shared_expert(x)."""

    def __init__(self, router_weight: torch.Tensor, switch: SwitchGLU, top_k: int, normalize: bool = True,
                 shared_expert: "QuantizedMLP | None" = None, shared_expert_gate: "QuantizedLinear | None" = None):
        if (shared_expert is None) != (shared_expert_gate is None):
            raise Q38Error(1, "shared_expert and shared_expert_gate are given together")
        self.router_weight, self.switch, self.top_k, self.normalize = router_weight, switch, top_k, normalize
        self.shared_expert, self.shared_expert_gate = shared_expert, shared_expert_gate

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        routed = sparse_moe(x, self.router_weight, self.switch, self.top_k, self.normalize)[0]
        if self.shared_expert is None:
            return routed
        m = self.shared_expert
        return shared_expert(x, routed, m.gate, m.up, m.down, self.shared_expert_gate, out=routed)


def shared_expert(x: torch.Tensor, routed: torch.Tensor, gate: "QuantizedLinear", up: "QuantizedLinear",
                  down: "QuantizedLinear", shared_gate: "QuantizedLinear", out: torch.Tensor | None = None):
    """routed + sigmoid(shared_gate(x)) * down(silu(gate(x)) * up(x)) (q38_shared_expert), the
    four projections quantized alike (group size, bits, scales dtype)."""
    _need(x, "x"), _need(routed, "routed")
    T, H = x.shape
    I = gate.weight.shape[0]
    layers = (gate, up, down, shared_gate)
    if any((l.group_size, l.bits, l.scales.dtype) != (gate.group_size, gate.bits, gate.scales.dtype) for l in layers):
        raise Q38Error(1, "shared_expert: the four projections must share group size, bits and scales dtype")
    if out is None:
        out = torch.empty_like(routed)
    args = []
    for l in layers:
        args += [_ptr(_as_u32(l.weight)), _ptr(l.scales), _ptr(l.biases)]
    ctx = _bind(x)
    _check(ctx, _lib.q38_shared_expert(ctx, _ptr(x), T, H, I, *args, _DTYPE[gate.scales.dtype], gate.group_size,
                                       gate.bits, _ptr(routed), _ptr(out)))
    return out


def sparse_moe(x: torch.Tensor, router_weight: torch.Tensor, switch: "SwitchGLU", top_k: int,
               normalize: bool = True):
    """Router + SwitchGLU in one call (q38_sparse_moe): -> (out, indices, scores)."""
    _need(x, "x"), _need(router_weight, "router_weight")
    T, H = x.shape
    E = router_weight.shape[0]
    g, u, d = switch.gate, switch.up, switch.down
    I = g.weight.shape[1]
    idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    sc = torch.empty((T, top_k), dtype=torch.bfloat16, device=x.device)
    out = torch.empty_like(x)
    ctx = _bind(x)
    _check(ctx, _lib.q38_sparse_moe(ctx, _ptr(x), T, H, I, E, top_k, int(normalize), _ptr(router_weight),
                                    _ptr(_as_u32(g.weight)), _ptr(g.scales), _ptr(g.biases),
                                    _ptr(_as_u32(u.weight)), _ptr(u.scales), _ptr(u.biases),
                                    _ptr(_as_u32(d.weight)), _ptr(d.scales), _ptr(d.biases), _DTYPE[x.dtype],
                                    g.group_size, g.bits, _ptr(idx), _ptr(sc), _ptr(out)))
    return out, idx, sc


# ------------------------------------------------------------------------ multi-GPU

def comm_unique_id() -> bytes:
    """A rendezvous id for a new communicator (rank 0 makes it, every rank passes it in)."""
    uid = _CommId()
    st = _lib.q38_comm_get_unique_id(C.byref(uid))
    if st != Q38_OK:
        raise Q38Error(st, (_lib.q38_comm_error() or b"").decode())
    return bytes(uid.bytes)


class Communicator:
    """One NCCL rank of libq38 (q38_comm_init_rank): `world` ranks, this one `rank` on
    `device`.  Init gives up with Q38Error (status 6) after `timeout_ms` if a rank does not
    join."""

    def __init__(self, uid: bytes, world: int, rank: int, device: int | None = None, timeout_ms: int = 60000):
        if device is None:
            device = torch.cuda.current_device()
        cid = _CommId()
        C.memmove(cid.bytes, uid, 128)
        p = _P()
        st = _lib.q38_comm_init_rank(C.byref(cid), int(world), int(rank), int(device), int(timeout_ms), C.byref(p))
        if st != Q38_OK:
            raise Q38Error(st, (_lib.q38_comm_error() or b"").decode())
        self.handle, self.world, self.rank, self.device = p.value, world, rank, device

    def destroy(self):
        if self.handle:
            _lib.q38_comm_destroy(self.handle)
            self.handle = None

    def abort(self):
        if self.handle:
            _lib.q38_comm_abort(self.handle)

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over the ranks."""
        _need(t, "t")
        ctx = _bind(t)
        _check(ctx, _lib.q38_comm_all_reduce(ctx, self.handle, _ptr(t), _ptr(t), t.numel(), _DTYPE[t.dtype]))
        return t


def tp_mlp(comm: Communicator, x: torch.Tensor, gate, up, down, group_size: int = 64, bits: int = 4,
           chunks: int = 0) -> torch.Tensor:
    """Tensor-parallel gated MLP (q38_tp_mlp): gate/up this rank's output-row shards, down its
    reduction-dimension shard; y [M, D] = the all-reduced sum on every rank.  chunks = 0 lets
    the library choose the number of overlapped token pieces."""
    _need(x, "x")
    M, D = x.shape
    gw, gs, gb = gate
    uw, us, ub = up
    dw, ds, db = down
    F_local = gw.shape[0]
    y = torch.empty_like(x)
    ctx = _bind(x)
    _check(ctx, _lib.q38_tp_mlp(ctx, comm.handle, _ptr(x), M, D, _ptr(_as_u32(gw)), _ptr(gs), _ptr(gb),
                                _ptr(_as_u32(uw)), _ptr(us), _ptr(ub), _ptr(_as_u32(dw)), _ptr(ds), _ptr(db),
                                F_local, _DTYPE[x.dtype], group_size, bits, chunks, _ptr(y)))
    return y


def ep_switch_glu(comm: Communicator, x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor, gate, up, down,
                  num_experts: int, capacity: int, group_size: int = 64, bits: int = 3) -> torch.Tensor:
    """Expert-parallel SwitchGLU (q38_ep_switch_glu): gate/up/down are this rank's expert
    stacks (num_experts / world experts), indices/scores the global routing of this rank's
    tokens; every rank uses the same `capacity` >= its token count."""
    _need(x, "x"), _need(indices, "indices"), _need(scores, "scores")
    T, H = x.shape
    k = indices.shape[-1]
    gw, gs, gb = gate
    uw, us, ub = up
    dw, ds, db = down
    I = gw.shape[1]
    out = torch.empty_like(x)
    ctx = _bind(x)
    _check(ctx, _lib.q38_ep_switch_glu(ctx, comm.handle, _ptr(x), T, H, I, num_experts, k, _ptr(indices),
                                       _ptr(scores), _ptr(_as_u32(gw)), _ptr(gs), _ptr(gb), _ptr(_as_u32(uw)),
                                       _ptr(us), _ptr(ub), _ptr(_as_u32(dw)), _ptr(ds), _ptr(db), _DTYPE[x.dtype],
                                       group_size, bits, capacity, _ptr(out)))
    return out
