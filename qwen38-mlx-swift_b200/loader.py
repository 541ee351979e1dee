"""Checkpoint loading: MLX safetensors checkpoints into device tensors and the quantized
modules of the q38 binding, including the Bonsai 2 Hadamard pack.

The reference loads checkpoints with MLX's `loadArrays` and attaches the arrays to modules
built in packed form (Sources/Qwen38Core/FlashNext/Qwen4ExpCheckpointLayerLoader.swift:74,
Qwen4ExpPrequantized.swift:77-106, :165-187): nothing is repacked, the on-disk layout is
the operator layout.  Here the file is read by libq38's safetensors reader (mapped
read-only, header validated) and each tensor is copied to the device unchanged.

* SafetensorsFile -- one file: names, dtypes, shapes, metadata, host copies, device
  copies of whole tensors or of row / column blocks (tensor-parallel shards).
* load_mlx_modules -- every `<path>.scales` in a checkpoint becomes a QuantizedLinear,
  QuantizedEmbedding or (expert-stacked weight) QuantizedSwitchLinear with the group size
  and bits of config.json's `quantization` (per-module overrides included); the other
  tensors are returned as device tensors.
* load_quantized_shard -- one rank's shard of a packed weight, read from the file without
  the rest of it (output rows, or a range of the reduction dimension).
* Bonsai2Loader / load_bonsai2 -- Qwen38Bonsai2Loader (Bonsai2/Qwen38Bonsai2Loader.swift:40-153)
  and the weight steps of Qwen38Bonsai2.loadContainer (Bonsai2/Qwen38Bonsai2Container.swift:21-64):
  config.json's `modules[]` validated (Hadamard block in {512, 1024, 2048, 4096}, dtype
  float16), every `.signs` vector checked to be +-1, the packed modules replaced by their
  Hadamard-rotated forms, the replacement count checked.
"""
from __future__ import annotations

import ctypes as C
import glob
import json
import os

import numpy as np
import torch

import q38

_TORCH = {
    "BOOL": torch.bool, "U8": torch.uint8, "I8": torch.int8, "I16": torch.int16, "U16": torch.int16,
    "F16": torch.float16, "BF16": torch.bfloat16, "I32": torch.int32, "U32": torch.int32, "F32": torch.float32,
    "F64": torch.float64, "I64": torch.int64, "U64": torch.int64, "F8_E4M3": torch.float8_e4m3fn,
    "F8_E5M2": torch.float8_e5m2,
}
# host views: unsigned types keep their own numpy type; bf16 and fp8 are raw bit patterns
_NUMPY = {
    "BOOL": np.bool_, "U8": np.uint8, "I8": np.int8, "I16": np.int16, "U16": np.uint16, "F16": np.float16,
    "BF16": np.uint16, "I32": np.int32, "U32": np.uint32, "F32": np.float32, "F64": np.float64,
    "I64": np.int64, "U64": np.uint64, "F8_E4M3": np.uint8, "F8_E5M2": np.uint8,
}


class SafetensorsError(ValueError):
    pass


class SafetensorsFile:
    """A safetensors file opened through libq38 (`q38_st_open`)."""

    def __init__(self, path: str):
        self.path = path
        h = C.c_void_p()
        st = q38._lib.q38_st_open(os.fsencode(path), C.byref(h))
        if st != q38.Q38_OK:
            raise SafetensorsError(f"{path}: {(q38._lib.q38_st_open_error() or b'').decode()}")
        self._h = h
        self._close = q38._lib.q38_st_close  # usable during interpreter shutdown
        n = q38._lib.q38_st_count(h)
        self._names = []
        self._info = {}
        name, dt = C.c_char_p(), C.c_char_p()
        nd = C.c_int()
        shape = (C.c_int64 * 8)()
        nb = C.c_uint64()
        for i in range(n):
            q38._lib.q38_st_info(h, i, C.byref(name), C.byref(dt), C.byref(nd), shape, C.byref(nb))
            key = name.value.decode("utf-8")
            self._names.append(key)
            self._info[key] = (i, dt.value.decode(), tuple(shape[d] for d in range(nd.value)), nb.value)
        k, v = C.c_char_p(), C.c_char_p()
        self.metadata = {}
        for i in range(q38._lib.q38_st_metadata_count(h)):
            q38._lib.q38_st_metadata_entry(h, i, C.byref(k), C.byref(v))
            self.metadata[k.value.decode("utf-8")] = v.value.decode("utf-8")

    def close(self):
        if getattr(self, "_h", None):
            self._close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        self.close()

    def keys(self) -> list[str]:
        return list(self._names)

    def __contains__(self, name: str) -> bool:
        return name in self._info

    def info(self, name: str):
        """(dtype as written in the file, shape, nbytes)."""
        _, dt, shape, nb = self._info[name]
        return dt, shape, nb

    def numpy(self, name: str) -> np.ndarray:
        """A host copy (bf16 and fp8 as their uint bit patterns)."""
        i, dt, shape, nb = self._info[name]
        if nb == 0:
            return np.zeros(shape, dtype=_NUMPY[dt])
        buf = (C.c_uint8 * nb).from_address(q38._lib.q38_st_data(self._h, i))
        return np.frombuffer(buf, dtype=_NUMPY[dt]).reshape(shape).copy()

    def _device(self, device):
        if device is None:
            return torch.device("cuda", torch.cuda.current_device())
        return torch.device(device)

    def to_device(self, name: str, device=None) -> torch.Tensor:
        """The whole tensor on the device (U32 as int32 bit patterns, the packed-code dtype
        the operators take)."""
        i, dt, shape, nb = self._info[name]
        t = torch.empty(shape, dtype=_TORCH[dt], device=self._device(device))
        if nb:
            ctx = q38._bind(t)
            q38._check(ctx, q38._lib.q38_st_copy_to_device(ctx, self._h, i, t.data_ptr(), nb))
        return t

    def _block(self, name, row_bytes, row0, rows, byte0, nbytes, out_shape, device):
        i, dt, _, _ = self._info[name]
        t = torch.empty(out_shape, dtype=_TORCH[dt], device=self._device(device))
        if t.numel():
            ctx = q38._bind(t)
            q38._check(ctx, q38._lib.q38_st_copy_block_to_device(ctx, self._h, i, row_bytes, row0, rows, byte0,
                                                                 nbytes, t.data_ptr(), nbytes))
        return t

    def to_device_rows(self, name: str, row0: int, rows: int, device=None) -> torch.Tensor:
        """Rows [row0, row0+rows) of the first dimension."""
        _, dt, shape, nb = self._info[name]
        if not shape or row0 < 0 or rows < 0 or row0 + rows > shape[0]:
            raise SafetensorsError(f"{name}: rows [{row0}, {row0 + rows}) outside shape {shape}")
        rb = nb // shape[0] if shape[0] else 0
        return self._block(name, rb, row0, rows, 0, rb, (rows,) + shape[1:], device)

    def to_device_cols(self, name: str, col0: int, cols: int, device=None) -> torch.Tensor:
        """Columns [col0, col0+cols) of the last dimension, for every leading index."""
        _, dt, shape, nb = self._info[name]
        if not shape or col0 < 0 or cols < 0 or col0 + cols > shape[-1]:
            raise SafetensorsError(f"{name}: columns [{col0}, {col0 + cols}) outside shape {shape}")
        es = nb // max(1, int(np.prod(shape)))
        lead = int(np.prod(shape[:-1]))
        return self._block(name, shape[-1] * es, 0, lead, col0 * es, cols * es, shape[:-1] + (cols,), device)


# ----------------------------------------------------------------- checkpoints

def read_config(directory: str) -> dict:
    with open(os.path.join(directory, "config.json")) as fh:
        return json.load(fh)


def quantization_for(config: dict, path: str):
    """(group_size, bits, mode) of module `path`, or None when it is not quantized: the
    checkpoint-wide `quantization` (or `quantization_config`) entry, overridden by an entry
    keyed by the module path (a dict of parameters, or false)."""
    q = config.get("quantization", config.get("quantization_config"))
    if not isinstance(q, dict):
        return None
    o = q.get(path)
    if o is False:
        return None
    base = {k: q[k] for k in ("group_size", "bits", "mode") if k in q}
    if isinstance(o, dict):
        base.update(o)
    if "bits" not in base or "group_size" not in base:
        return None
    return int(base["group_size"]), int(base["bits"]), str(base.get("mode", "affine"))


def checkpoint_files(directory: str) -> list[str]:
    """The safetensors files of a checkpoint: the shards of model.safetensors.index.json,
    else every *.safetensors in the directory."""
    idx = os.path.join(directory, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as fh:
            wm = json.load(fh)["weight_map"]
        return [os.path.join(directory, f) for f in sorted(set(wm.values()))]
    return sorted(glob.glob(os.path.join(directory, "*.safetensors")))


def _module_of(weight, scales, biases, bias, gs, bits, mode, embedding):
    if weight.dim() == 3:
        return q38.QuantizedSwitchLinear(weight, scales, biases, gs, bits, mode)
    if embedding:
        return q38.QuantizedEmbedding(weight, scales, biases, gs, bits, mode)
    return q38.QuantizedLinear(weight, scales, biases, bias, gs, bits, mode)


def _check_packed(path, wshape, sshape, gs, bits):
    K = wshape[-1] * 32 // bits
    if wshape[-1] * 32 % bits or K % gs or sshape[-1] != K // gs or tuple(wshape[:-1]) != tuple(sshape[:-1]):
        raise SafetensorsError(f"{path}: weight {wshape} and scales {sshape} do not match group {gs}, bits {bits}")


def load_mlx_modules(directory: str, device=None, skip=None, embeddings=None, config=None):
    """Loads a checkpoint directory.  Returns (modules, tensors): `modules` maps each module
    path that has `.scales` to its quantized module (`.weight`, `.scales`, `.biases` and a
    Linear's `.bias` consumed), `tensors` maps every other name to its device tensor.
    `skip(name)` excludes tensors; a module is an embedding when its path ends in
    "embed_tokens" or is listed in `embeddings`."""
    config = read_config(directory) if config is None else config
    files = [SafetensorsFile(p) for p in checkpoint_files(directory)]
    try:
        where = {}
        for f in files:
            for k in f.keys():
                if skip is not None and skip(k):
                    continue
                where[k] = f
        modules, used = {}, set()
        for key in sorted(where):
            if not key.endswith(".scales"):
                continue
            path = key[: -len(".scales")]
            wkey = path + ".weight"
            if wkey not in where:
                raise SafetensorsError(f"{path}: scales without a packed weight")
            q = quantization_for(config, path)
            if q is None:
                raise SafetensorsError(f"{path}: packed weight but no quantization parameters in config.json")
            gs, bits, mode = q
            _check_packed(path, where[wkey].info(wkey)[1], where[key].info(key)[1], gs, bits)
            w = where[wkey].to_device(wkey, device)
            s = where[key].to_device(key, device)
            bkey, biaskey = path + ".biases", path + ".bias"
            b = where[bkey].to_device(bkey, device) if bkey in where else None
            is_emb = path.endswith("embed_tokens") or (embeddings is not None and path in embeddings)
            bias = where[biaskey].to_device(biaskey, device) if (biaskey in where and not is_emb) else None
            modules[path] = _module_of(w, s, b, bias, gs, bits, mode, is_emb)
            used.update({wkey, key, bkey, biaskey} if bias is not None else {wkey, key, bkey})
        tensors = {k: f.to_device(k, device) for k, f in where.items() if k not in used}
        return modules, tensors
    finally:
        for f in files:
            f.close()


def load_quantized_shard(f: SafetensorsFile, path: str, rank: int, world: int, axis: str, group_size: int,
                         bits: int, device=None):
    """(codes, scales, biases) of rank's shard of the packed weight `path`, read from the
    file alone: axis "rows" keeps output rows [rank*N/world, ...) (column-parallel), axis
    "k" keeps K/world of the reduction dimension, which must be whole groups and whole
    32-bit words (row-parallel)."""
    wk, sk, bk = path + ".weight", path + ".scales", path + ".biases"
    wshape, sshape = f.info(wk)[1], f.info(sk)[1]
    _check_packed(path, wshape, sshape, group_size, bits)
    has_b = bk in f
    if axis == "rows":
        N = wshape[0]
        if N % world:
            raise ValueError(f"{N} rows do not split over {world} ranks")
        n = N // world
        return (f.to_device_rows(wk, rank * n, n, device), f.to_device_rows(sk, rank * n, n, device),
                f.to_device_rows(bk, rank * n, n, device) if has_b else None)
    if axis == "k":
        K = sshape[-1] * group_size
        if K % world or (K // world) % group_size or ((K // world) * bits) % 32:
            raise ValueError(f"K={K} does not split into whole groups and words over {world} ranks")
        kp = K // world
        wpr, gpr = kp * bits // 32, kp // group_size
        return (f.to_device_cols(wk, rank * wpr, wpr, device), f.to_device_cols(sk, rank * gpr, gpr, device),
                f.to_device_cols(bk, rank * gpr, gpr, device) if has_b else None)
    raise ValueError(f"axis must be 'rows' or 'k', not {axis!r}")


# -------------------------------------------------------------------- Bonsai 2

_BONSAI_BLOCKS = (512, 1024, 2048, 4096)
# raw values of MLX's QuantizationMode
_MODES = ("affine", "mxfp4", "mxfp8", "nvfp4")


class Bonsai2LoaderError(ValueError):
    """Qwen38Bonsai2LoaderError (Bonsai2/Qwen38Bonsai2Loader.swift:6-30): `kind` is one of
    unsupportedBlock, unsupportedDtype, missingSigns, invalidSigns,
    unexpectedReplacementCount, missingWeights."""

    def __init__(self, kind: str, detail):
        self.kind, self.detail = kind, detail
        super().__init__(f"Bonsai 2 pack: {kind} ({detail})")


def _signs_are_unit(v: np.ndarray) -> bool:
    # allClose(abs(signs), 1.0) with MLX's default tolerances (rtol 1e-5, atol 1e-8)
    a = np.abs(v.astype(np.float64))
    return bool(np.all(np.abs(a - 1.0) <= 1e-8 + 1e-5 * 1.0))


class Bonsai2Loader:
    """Reads config.json's `modules[]` and the `.signs` vectors of model.safetensors and
    replaces the packed modules with their Hadamard-rotated forms."""

    def __init__(self, directory: str):
        config = read_config(directory)
        mode = config["quantization"]["mode"]
        if mode not in _MODES:
            raise Bonsai2LoaderError("unsupportedDtype", mode)
        for e in config["modules"]:
            if e["block"] not in _BONSAI_BLOCKS:
                raise Bonsai2LoaderError("unsupportedBlock", e["block"])
            if e["dtype"] != "float16":
                raise Bonsai2LoaderError("unsupportedDtype", e["dtype"])
        signs = {}
        with SafetensorsFile(os.path.join(directory, "model.safetensors")) as f:
            for key in f.keys():
                if not key.endswith(".signs"):
                    continue
                path = key[: -len(".signs")]
                v = f.numpy(key)
                if not _signs_are_unit(v):
                    raise Bonsai2LoaderError("invalidSigns", path)
                signs[path] = v.astype(np.float32)
        for e in config["modules"]:
            path = "language_model." + e["path"]
            if path not in signs:
                raise Bonsai2LoaderError("missingSigns", path)
        self.entries = config["modules"]
        self.signs = signs
        self.expected_replacement_count = len(self.entries)

    def install(self, modules: dict, device=None) -> int:
        """Replaces modules[path] in place; returns the number replaced.  A module that is
        absent or of the wrong kind means the checkpoint does not match its config.json."""
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        updates = {}
        for e in self.entries:
            path = "language_model." + e["path"]
            if path not in modules:
                raise RuntimeError(f"Bonsai 2 pack: module {path} not found")
            cur = modules[path]
            signs = torch.from_numpy(self.signs[path]).to(dev)
            if e["embedding"]:
                if not isinstance(cur, q38.QuantizedEmbedding):
                    raise RuntimeError(f"Bonsai 2 pack: {path} is not a QuantizedEmbedding")
                updates[path] = q38.HadamardQuantizedEmbedding(cur, signs, e["block"])
            else:
                if not isinstance(cur, q38.QuantizedLinear):
                    raise RuntimeError(f"Bonsai 2 pack: {path} is not a QuantizedLinear")
                updates[path] = q38.HadamardQuantizedLinear(cur, signs, e["block"])
        modules.update(updates)
        return len(updates)


def load_bonsai2(directory: str, device=None, text_only: bool = False):
    """The weight steps of Qwen38Bonsai2.loadContainer: every tensor except the `.signs`
    vectors (and, text_only, the vision tower's) loaded, the packed modules built with the
    pack's quantization, each module named in config.json's `modules[]` present, then the
    Hadamard modules installed and their count checked.  Returns (modules, tensors)."""
    config = read_config(directory)

    def skip(name):
        return name.endswith(".signs") or (text_only and name.startswith("vision_tower."))

    emb = {"language_model." + e["path"] for e in config.get("modules", []) if e.get("embedding")}
    modules, tensors = load_mlx_modules(directory, device, skip=skip, embeddings=emb, config=config)
    missing = []
    for e in config.get("modules", []):
        path = "language_model." + e["path"]
        if path not in modules:
            missing += [path + ".weight", path + ".scales", path + ".biases"]
    if missing:
        raise Bonsai2LoaderError("missingWeights", missing[:3])
    installer = Bonsai2Loader(directory)
    replaced = installer.install(modules, device)
    if replaced != installer.expected_replacement_count:
        raise Bonsai2LoaderError("unexpectedReplacementCount",
                                 {"expected": installer.expected_replacement_count, "actual": replaced})
    return modules, tensors
