"""ctypes view of the CPU oracle (liboracle: oracle/q38_oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker; the product (libq38.so and its
Python binding) never imports it.  bf16 arrays travel as numpy uint16 bit
patterns.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libq38_oracle.so")
_lib = None

_P = C.c_void_p
_I = C.c_int64
_i = C.c_int


def build() -> str:
    """Compile the oracle library in place (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        sig = {
            "q38o_unpack": [_P, _I, _I, _i, _P],
            "q38o_pack": [_P, _I, _I, _i, _P],
            "q38o_quantize": [_P, _I, _I, _i, _i, _P, _P, _P],
            "q38o_dequantize": [_P, _P, _P, _I, _I, _i, _i, _P],
            "q38o_qmm": [_P, _I, _I, _P, _P, _P, _I, _i, _i, _P],
            "q38o_qmm_f32": [_P, _I, _I, _P, _P, _P, _I, _i, _i, _P],
            "q38o_gather_qmm": [_P, _I, _I, _I, _P, _P, _P, _I, _I, _i, _i, _P, _P, _I, _P],
            "q38o_moe_route": [_P, _I, _I, _P, _I, _i, _i, _P, _P, _P],
            "q38o_route_from_logits": [_P, _I, _I, _i, _i, _P, _P, _P],
            "q38o_sort_by_expert": [_P, _I, _I, _P, _P],
            "q38o_switch_glu": [_P, _I, _I, _I, _I, _i, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                _i, _i, _i, _P],
            "q38o_hadamard_rotate": [_P, _I, _I, _P, _i, _i, _P],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _i
        L.q38o_fill_normal_bf16.argtypes = [C.c_uint64, C.c_float, _P, _I]
        L.q38o_fill_normal_bf16.restype = None
        L.q38o_fill_normal_f32.argtypes = [C.c_uint64, C.c_float, _P, _I]
        L.q38o_fill_normal_f32.restype = None
        L.q38o_fill_ternary.argtypes = [C.c_uint64, C.c_float, _I, _I, _i, _P, _P, _P]
        L.q38o_fill_ternary.restype = None
        L.q38o_set_threads.argtypes = [_i]
        L.q38o_set_threads.restype = None
        L.q38o_get_threads.argtypes = []
        L.q38o_get_threads.restype = _i
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _check(rc, what):
    if rc != 0:
        raise ValueError(f"oracle {what} failed with status {rc}")


# ----------------------------------------------------------------- bf16 helpers

def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def set_threads(n: int) -> None:
    lib().q38o_set_threads(int(n))


def threads() -> int:
    return int(lib().q38o_get_threads())


# -------------------------------------------------------------------- generators

def normal_bf16(seed: int, shape, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.uint16)
    lib().q38o_fill_normal_bf16(seed, std, _p(out), out.size)
    return out


def normal_f32(seed: int, shape, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    lib().q38o_fill_normal_f32(seed, std, _p(out), out.size)
    return out


def ternary(seed: int, rows: int, K: int, group: int = 64, std: float = 0.02):
    codes = np.empty((rows, K // 16), dtype=np.uint32)
    s = np.empty((rows, K // group), dtype=np.uint16)
    b = np.empty((rows, K // group), dtype=np.uint16)
    lib().q38o_fill_ternary(seed, std, rows, K, group, _p(codes), _p(s), _p(b))
    return codes, s, b


# ------------------------------------------------------------------- operators

def quantize(w: np.ndarray, group: int = 64, bits: int = 4):
    w = np.ascontiguousarray(w, dtype=np.float32)
    lead, K = w.shape[:-1], w.shape[-1]
    rows = int(np.prod(lead)) if lead else 1
    codes = np.empty(lead + (K * bits // 32,), dtype=np.uint32)
    s = np.empty(lead + (K // group,), dtype=np.uint16)
    b = np.empty(lead + (K // group,), dtype=np.uint16)
    _check(lib().q38o_quantize(_p(w), rows, K, group, bits, _p(codes), _p(s), _p(b)), "quantize")
    return codes, s, b


def unpack(codes: np.ndarray, K: int, bits: int) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    rows = codes.size // (K * bits // 32)
    q = np.empty(codes.shape[:-1] + (K,), dtype=np.uint8)
    _check(lib().q38o_unpack(_p(codes), rows, K, bits, _p(q)), "unpack")
    return q


def pack(q: np.ndarray, bits: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    K = q.shape[-1]
    rows = q.size // K
    codes = np.empty(q.shape[:-1] + (K * bits // 32,), dtype=np.uint32)
    _check(lib().q38o_pack(_p(q), rows, K, bits, _p(codes)), "pack")
    return codes


def dequantize(codes, scales, biases, group: int, bits: int) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    K = codes.shape[-1] * 32 // bits
    rows = codes.size // codes.shape[-1]
    out = np.empty(codes.shape[:-1] + (K,), dtype=np.float32)
    _check(lib().q38o_dequantize(_p(codes), _p(np.ascontiguousarray(scales)),
                                 _p(None if biases is None else np.ascontiguousarray(biases)),
                                 rows, K, group, bits, _p(out)), "dequantize")
    return out


def qmm(x, codes, scales, biases, group: int, bits: int, f32: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    M, K = x.shape
    N = codes.shape[0]
    if f32:
        y = np.empty((M, N), dtype=np.float32)
        fn = lib().q38o_qmm_f32
    else:
        y = np.empty((M, N), dtype=np.uint16)
        fn = lib().q38o_qmm
    _check(fn(_p(x), M, K, _p(codes), _p(np.ascontiguousarray(scales)),
              _p(None if biases is None else np.ascontiguousarray(biases)), N, group, bits,
              _p(y)), "qmm")
    return y


def gather_qmm(x, codes, scales, biases, lhs, rhs, group: int, bits: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    Bx, M, K = x.shape
    E, N = codes.shape[0], codes.shape[1]
    rhs = np.ascontiguousarray(rhs, dtype=np.int32)
    P = rhs.size
    out = np.empty((P, M, N), dtype=np.uint16)
    lhs_a = None if lhs is None else np.ascontiguousarray(lhs, dtype=np.int32)
    _check(lib().q38o_gather_qmm(_p(x), Bx, M, K, _p(np.ascontiguousarray(codes)),
                                 _p(np.ascontiguousarray(scales)),
                                 _p(None if biases is None else np.ascontiguousarray(biases)),
                                 E, N, group, bits, _p(lhs_a), _p(rhs), P, _p(out)), "gather_qmm")
    return out


def moe_route(x, wr, top_k: int, normalize: bool = True, want_probs: bool = False):
    x = np.ascontiguousarray(x, dtype=np.uint16)
    wr = np.ascontiguousarray(wr, dtype=np.uint16)
    T, H = x.shape
    E = wr.shape[0]
    idx = np.empty((T, top_k), dtype=np.int32)
    sc = np.empty((T, top_k), dtype=np.uint16)
    probs = np.empty((T, E), dtype=np.uint16) if want_probs else None
    _check(lib().q38o_moe_route(_p(x), T, H, _p(wr), E, top_k, int(normalize), _p(idx), _p(sc),
                                _p(probs)), "moe_route")
    return (idx, sc, probs) if want_probs else (idx, sc)


def route_from_logits(logits, top_k: int, normalize: bool = True):
    logits = np.ascontiguousarray(logits, dtype=np.uint16)
    T, E = logits.shape
    idx = np.empty((T, top_k), dtype=np.int32)
    sc = np.empty((T, top_k), dtype=np.uint16)
    probs = np.empty((T, E), dtype=np.uint16)
    _check(lib().q38o_route_from_logits(_p(logits), T, E, top_k, int(normalize), _p(idx), _p(sc),
                                        _p(probs)), "route_from_logits")
    return idx, sc, probs


def sort_by_expert(indices, E: int):
    indices = np.ascontiguousarray(indices, dtype=np.int32).reshape(-1)
    perm = np.empty(indices.size, dtype=np.int32)
    offsets = np.empty(E + 1, dtype=np.int32)
    _check(lib().q38o_sort_by_expert(_p(indices), indices.size, E, _p(perm), _p(offsets)), "sort")
    return perm, offsets


def switch_glu(x, indices, scores, gate, up, down, group: int, bits: int,
               weights_bf16: bool = False) -> np.ndarray:
    """gate/up/down are (codes, scales, biases) triples of expert-stacked weights.
    weights_bf16 rounds each dequantized weight once to bf16, as a bf16 tensor-core product
    consumes it; otherwise weights are evaluated in fp32."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    T, H = x.shape
    E, I = gate[0].shape[0], gate[0].shape[1]
    top_k = indices.shape[1]
    out = np.empty((T, H), dtype=np.uint16)
    c = [np.ascontiguousarray(a) if a is not None else None for t in (gate, up, down) for a in t]
    _check(lib().q38o_switch_glu(_p(x), T, H, I, E, top_k,
                                 _p(np.ascontiguousarray(indices, dtype=np.int32)),
                                 _p(np.ascontiguousarray(scores, dtype=np.uint16)),
                                 *[_p(a) for a in c], group, bits, int(weights_bf16), _p(out)), "switch_glu")
    return out


def shared_expert(x, routed, gate, up, down, shared_gate, group: int, bits: int,
                  weights_bf16: bool = False) -> np.ndarray:
    """The shared-expert term of Qwen4ExpSparseMoE.callAsFunction (FlashNext/Qwen4ExpSparseMoE.swift:297,
    Qwen4ExpSharedExpert :77-82) added to the routed output; every projection is a quantized
    product rounded to bf16 (an MLX bf16 array), the SiLU product rounded once (the compiled
    silu product), sigmoid in fp32 rounded to bf16:
      out = bf16(routed + bf16(bf16(sigmoid(sg(x))) * down(bf16(silu(gate(x)) * up(x))))).
    weights_bf16 rounds the dequantized gate, up and down weights to bf16 before their
    products (the operands of a bf16 tensor-core product), fp32 accumulation."""
    f = lambda a: bf16_to_f32(a).astype(np.float32)

    def proj(a, w):
        if not weights_bf16:
            return f(qmm(a, *w, group, bits))
        wb = f(f32_to_bf16(dequantize(w[0], w[1], w[2], group, bits)))
        return f(f32_to_bf16(f(a) @ wb.T))
    g = proj(x, gate)
    u = proj(x, up)
    h = f32_to_bf16((g / (np.float32(1) + np.exp(-g))) * u)
    ys = proj(h, down)
    logit = f(qmm(x, *shared_gate, group, bits))
    s = f(f32_to_bf16(np.float32(1) / (np.float32(1) + np.exp(-logit))))
    sh = f(f32_to_bf16(s * ys))
    return f32_to_bf16(f(routed) + sh)


def hadamard_rotate(x, block: int, signs=None, inverse: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    D = x.shape[-1]
    rows = x.size // D
    y = np.empty_like(x)
    s = None if signs is None else np.ascontiguousarray(signs, dtype=np.float32)
    _check(lib().q38o_hadamard_rotate(_p(x), rows, D, _p(s), block, int(inverse), _p(y)),
           "hadamard_rotate")
    return y
