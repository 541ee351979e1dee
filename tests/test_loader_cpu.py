"""Checkpoint reader and loader host logic (no GPU): libq38's safetensors reader against
files written by the official safetensors package, its rejection of malformed files, the
per-module quantization lookup, and the Bonsai 2 loader's validations
(Bonsai2/Qwen38Bonsai2Loader.swift:65-107: Hadamard block in {512, 1024, 2048, 4096},
module dtype float16, a known quantization mode, +-1 signs present for every module).
"""
import json
import struct

import numpy as np
import pytest
import torch
import safetensors.torch as st

import loader


def _tensors():
    g = torch.Generator().manual_seed(5)
    return {
        "model.layers.0.mlp.gate_proj.weight": torch.randint(0, 2 ** 31 - 1, (6, 16), generator=g,
                                                            dtype=torch.int64).to(torch.uint32),
        "model.layers.0.mlp.gate_proj.scales": torch.randn(6, 2, generator=g).bfloat16(),
        "half": torch.randn(7, generator=g).half(),
        "scalar": torch.tensor(3.5),
        "empty": torch.zeros(0, 4),
        "flags": torch.tensor([True, False, True]),
        "f8": torch.randn(4, generator=g).to(torch.float8_e4m3fn),
        "i64": torch.arange(6, dtype=torch.int64).reshape(2, 3),
        "u8": torch.arange(10, dtype=torch.uint8),
        "éè 😀": torch.ones(2, dtype=torch.float64),
    }


def _raw(v: torch.Tensor) -> bytes:
    return v.reshape(-1).contiguous().view(torch.uint8).numpy().tobytes() if v.numel() else b""


def test_reader_matches_official_writer(tmp_path):
    t = _tensors()
    path = str(tmp_path / "m.safetensors")
    st.save_file(t, path, metadata={"format": "mlx", "note": "x"})
    with loader.SafetensorsFile(path) as f:
        assert sorted(f.keys()) == sorted(t)
        assert f.metadata == {"format": "mlx", "note": "x"}
        for k, v in t.items():
            dt, shape, nb = f.info(k)
            assert shape == tuple(v.shape) and nb == v.numel() * v.element_size()
            assert f.numpy(k).tobytes() == _raw(v)
        assert f.info("model.layers.0.mlp.gate_proj.weight")[0] == "U32"
        assert f.info("model.layers.0.mlp.gate_proj.scales")[0] == "BF16"


def _write(path, header, data: bytes, raw_header: bytes | None = None):
    h = raw_header if raw_header is not None else json.dumps(header).encode()
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)) + h + data)


def _one(name="a", dtype="F32", shape=(2,), off=(0, 8)):
    return {name: {"dtype": dtype, "shape": list(shape), "data_offsets": list(off)}}


@pytest.mark.parametrize("case, header, data, message", [
    ("gap", {**_one("a", off=(0, 8)), **_one("b", off=(12, 20))}, bytes(20), "gap or overlap"),
    ("overlap", {**_one("a", off=(0, 8)), **_one("b", off=(4, 12))}, bytes(12), "gap or overlap"),
    ("uncovered", _one(), bytes(12), "cover"),
    ("size", _one(shape=(3,)), bytes(8), "disagree"),
    ("dtype", _one(dtype="Q4"), bytes(8), "unknown dtype"),
    ("fields", {"a": {"dtype": "F32", "shape": [2]}}, bytes(8), "lacks"),
    ("offsets", {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0]}}, bytes(8), "two entries"),
    ("negative", {"a": {"dtype": "F32", "shape": [-2], "data_offsets": [0, 8]}}, bytes(8), "integer"),
    ("reversed", _one(off=(8, 0)), bytes(8), "disagree"),
])
def test_reader_rejects_malformed_headers(tmp_path, case, header, data, message):
    path = str(tmp_path / f"{case}.safetensors")
    _write(path, header, data)
    with pytest.raises(loader.SafetensorsError, match=message):
        loader.SafetensorsFile(path)


@pytest.mark.parametrize("case, raw, message", [
    ("truncated_json", b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}', "expected"),
    ("duplicate", b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},'
                  b' "a": {"dtype": "F32", "shape": [0], "data_offsets": [8, 8]}}', "duplicate"),
    ("trailing", b'{} x', "trailing"),
    ("bad_escape", b'{"\\q": {}}', "bad escape"),
    ("lone_surrogate", b'{"\\ud83d": {}}', "surrogate"),
    ("float_shape", b'{"a": {"dtype": "F32", "shape": [2.0], "data_offsets": [0, 8]}}', "integer"),
])
def test_reader_rejects_malformed_json(tmp_path, case, raw, message):
    path = str(tmp_path / f"{case}.safetensors")
    _write(path, None, bytes(8), raw_header=raw)
    with pytest.raises(loader.SafetensorsError, match=message):
        loader.SafetensorsFile(path)


def test_reader_rejects_short_and_oversized_headers(tmp_path):
    p = tmp_path / "short.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(loader.SafetensorsError, match="shorter"):
        loader.SafetensorsFile(str(p))
    p.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(loader.SafetensorsError, match="beyond the end"):
        loader.SafetensorsFile(str(p))
    p.write_bytes(struct.pack("<Q", 200_000_000) + b"{}")
    with pytest.raises(loader.SafetensorsError, match="limit"):
        loader.SafetensorsFile(str(p))
    with pytest.raises(loader.SafetensorsError, match="cannot open"):
        loader.SafetensorsFile(str(tmp_path / "absent.safetensors"))


def test_reader_escapes_padding_and_unknown_fields(tmp_path):
    raw = (b'{"__metadata__": {"k\\n": "v\\u00e9"}, '
           b'"\\u00e9\\ud83d\\ude00\\t\\"\\\\/": {"dtype": "U8", "shape": [3], "data_offsets": [0, 3], '
           b'"extra": {"nested": [1, 2.5e3, true, null]}}}      ')
    path = str(tmp_path / "esc.safetensors")
    _write(path, None, b"\x07\x08\x09", raw_header=raw)
    with loader.SafetensorsFile(path) as f:
        name = "é\U0001F600\t\"\\/"
        assert f.keys() == [name]
        assert f.metadata == {"k\n": "vé"}
        assert f.numpy(name).tolist() == [7, 8, 9]


def test_empty_file_header(tmp_path):
    path = str(tmp_path / "empty.safetensors")
    _write(path, {}, b"")
    with loader.SafetensorsFile(path) as f:
        assert f.keys() == [] and f.metadata == {}


def test_quantization_for_per_module_overrides():
    cfg = {"quantization": {"group_size": 64, "bits": 4, "mode": "affine",
                            "model.layers.0.mlp.experts": {"bits": 3},
                            "model.layers.0.router": False}}
    assert loader.quantization_for(cfg, "model.layers.0.mlp.gate_proj") == (64, 4, "affine")
    assert loader.quantization_for(cfg, "model.layers.0.mlp.experts") == (64, 3, "affine")
    assert loader.quantization_for(cfg, "model.layers.0.router") is None
    assert loader.quantization_for({"quantization_config": {"group_size": 32, "bits": 8}}, "x") == (32, 8, "affine")
    assert loader.quantization_for({}, "x") is None


# ----------------------------------------------------------------- Bonsai 2 pack

def bonsai_pack(directory, K=2048, N=64, vocab=48, block=1024, signs_ok=True, drop_signs=None,
                mode="affine", dtype="float16", seed=0):
    """A miniature Bonsai 2 pack: one rotated linear and the rotated embedding, 2-bit
    group-128 ternary codes with f16 scales and biases = -scales, f32 signs."""
    g = torch.Generator().manual_seed(seed)
    t = {}
    mods = [("model.layers.0.mlp.gate_proj", N, False), ("model.embed_tokens", vocab, True)]
    for path, rows, _emb in mods:
        codes = torch.randint(0, 3, (rows, K), generator=g)
        words = torch.zeros((rows, K // 16), dtype=torch.int64)
        for j in range(16):
            words |= codes[:, j::16] << (2 * j)
        scales = (torch.rand((rows, K // 128), generator=g) * 0.02 + 0.001).half()
        full = "language_model." + path
        t[full + ".weight"] = words.to(torch.uint32)
        t[full + ".scales"] = scales
        t[full + ".biases"] = -scales
        if drop_signs != full:
            s = torch.where(torch.rand(K, generator=g) < 0.5, -1.0, 1.0)
            if not signs_ok and path.endswith("gate_proj"):
                s[3] = 0.5
            t[full + ".signs"] = s
    t["language_model.model.norm.weight"] = torch.ones(K).bfloat16()
    t["vision_tower.blocks.0.weight"] = torch.ones(4, 4).half()
    st.save_file(t, str(directory / "model.safetensors"), metadata={"format": "mlx"})
    cfg = {"model_type": "prism_hadamard_qwen35",
           "quantization": {"group_size": 128, "bits": 2, "mode": mode},
           "modules": [{"path": p, "block": block, "embedding": e, "dtype": dtype} for p, _, e in mods]}
    (directory / "config.json").write_text(json.dumps(cfg))
    return t, cfg


def test_bonsai2_loader_accepts_a_valid_pack(tmp_path):
    t, cfg = bonsai_pack(tmp_path)
    ld = loader.Bonsai2Loader(str(tmp_path))
    assert ld.expected_replacement_count == 2
    assert set(ld.signs) == {"language_model.model.layers.0.mlp.gate_proj", "language_model.model.embed_tokens"}
    np.testing.assert_array_equal(ld.signs["language_model.model.embed_tokens"],
                                  t["language_model.model.embed_tokens.signs"].numpy())


@pytest.mark.parametrize("kwargs, kind", [
    ({"block": 256}, "unsupportedBlock"),
    ({"block": 8192}, "unsupportedBlock"),
    ({"dtype": "bfloat16"}, "unsupportedDtype"),
    ({"mode": "int4"}, "unsupportedDtype"),
    ({"signs_ok": False}, "invalidSigns"),
    ({"drop_signs": "language_model.model.embed_tokens"}, "missingSigns"),
])
def test_bonsai2_loader_rejections(tmp_path, kwargs, kind):
    bonsai_pack(tmp_path, **kwargs)
    with pytest.raises(loader.Bonsai2LoaderError) as e:
        loader.Bonsai2Loader(str(tmp_path))
    assert e.value.kind == kind
