"""Checkpoint loading onto the GPU: device copies through libq38's reader (whole tensors,
row blocks and column blocks, through the pinned staging in several pieces), MLX
checkpoints into quantized modules (results equal the operators on the original tensors
and the oracle), tensor-parallel shards read from the file (equal to sharding the full
tensors), and a miniature Bonsai 2 pack end to end (replacement count, rotated modules
equal to the rotation operators on the same tensors).
"""
import json

import numpy as np
import pytest
import torch
import safetensors.torch as st

import oracle as O
import loader
import parallel
from test_loader_cpu import bonsai_pack, _tensors
from test_qmm_gpu import dev_bf16, host_bf16

pytestmark = pytest.mark.gpu


def _bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.shape != b.shape:
        return False
    if a.numel() == 0:
        return True
    return torch.equal(a.reshape(-1).contiguous().view(torch.uint8).cpu(), b.reshape(-1).contiguous().view(torch.uint8).cpu())


def test_to_device_every_dtype(q38, tmp_path):
    t = _tensors()
    path = str(tmp_path / "m.safetensors")
    st.save_file(t, path)
    with loader.SafetensorsFile(path) as f:
        for k, v in t.items():
            d = f.to_device(k)
            assert d.is_cuda
            assert _bits_equal(d, v), k


def test_copies_larger_than_the_staging(q38, tmp_path):
    g = torch.Generator().manual_seed(7)
    big = torch.randint(-2 ** 31, 2 ** 31 - 1, (3, 5_000_000), generator=g, dtype=torch.int32)  # 60 MB
    wide = torch.randint(-2 ** 31, 2 ** 31 - 1, (2, 9_000_000), generator=g, dtype=torch.int32)  # rows of 36 MB
    path = str(tmp_path / "big.safetensors")
    st.save_file({"big": big, "wide": wide}, path)
    with loader.SafetensorsFile(path) as f:
        assert torch.equal(f.to_device("big").cpu(), big)
        assert torch.equal(f.to_device_rows("big", 1, 2).cpu(), big[1:3])
        assert torch.equal(f.to_device_cols("big", 1_000_003, 2_500_000).cpu(), big[:, 1_000_003:3_500_003])
        assert torch.equal(f.to_device_cols("wide", 17, 8_500_000).cpu(), wide[:, 17:8_500_017])
        with pytest.raises(loader.SafetensorsError):
            f.to_device_rows("big", 2, 2)


def _mini_checkpoint(directory):
    """Gate projection 4-bit g64, embedding 4-bit, expert stack 3-bit (per-module override),
    a norm weight; the packed tensors made by the oracle's quantizer."""
    gate = O.quantize(O.normal_f32(21, (256, 512), 0.02), 64, 4)
    emb = O.quantize(O.normal_f32(22, (100, 512), 0.02), 64, 4)
    sw = O.quantize(O.normal_f32(23, (4 * 128, 512), 0.02), 64, 3)
    u32 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).view(torch.uint32)
    b16 = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    t = {
        "model.layers.0.mlp.gate_proj.weight": u32(gate[0]), "model.layers.0.mlp.gate_proj.scales": b16(gate[1]),
        "model.layers.0.mlp.gate_proj.biases": b16(gate[2]),
        "model.embed_tokens.weight": u32(emb[0]), "model.embed_tokens.scales": b16(emb[1]),
        "model.embed_tokens.biases": b16(emb[2]),
        "model.layers.0.mlp.switch_mlp.gate_proj.weight": u32(sw[0]).reshape(4, 128, -1),
        "model.layers.0.mlp.switch_mlp.gate_proj.scales": b16(sw[1]).reshape(4, 128, -1),
        "model.layers.0.mlp.switch_mlp.gate_proj.biases": b16(sw[2]).reshape(4, 128, -1),
        "model.norm.weight": torch.ones(512).bfloat16(),
    }
    st.save_file(t, str(directory / "model.safetensors"), metadata={"format": "mlx"})
    cfg = {"quantization": {"group_size": 64, "bits": 4, "model.layers.0.mlp.switch_mlp.gate_proj": {"bits": 3}}}
    (directory / "config.json").write_text(json.dumps(cfg))
    return gate, emb, sw, t


def test_mlx_checkpoint_into_modules(q38, tmp_path):
    gate, emb, sw, t = _mini_checkpoint(tmp_path)
    modules, tensors = loader.load_mlx_modules(str(tmp_path))
    assert set(modules) == {"model.layers.0.mlp.gate_proj", "model.embed_tokens",
                            "model.layers.0.mlp.switch_mlp.gate_proj"}
    assert set(tensors) == {"model.norm.weight"}
    lin = modules["model.layers.0.mlp.gate_proj"]
    em = modules["model.embed_tokens"]
    sx = modules["model.layers.0.mlp.switch_mlp.gate_proj"]
    assert isinstance(lin, q38.QuantizedLinear) and (lin.group_size, lin.bits) == (64, 4)
    assert isinstance(em, q38.QuantizedEmbedding)
    assert isinstance(sx, q38.QuantizedSwitchLinear) and sx.bits == 3 and tuple(sx.weight.shape) == (4, 128, 48)
    x = O.normal_bf16(24, (3, 512))
    y = lin(dev_bf16(x))
    ids = np.array([0, 99, 7], np.int32)
    rows = em(torch.from_numpy(ids).cuda())
    torch.cuda.synchronize()
    ref = O.qmm(x, *gate, 64, 4, f32=True)
    got = O.bf16_to_f32(host_bf16(y)).astype(np.float64)
    assert np.abs(got - ref).max() <= 2e-2 * np.sqrt((ref ** 2).mean())
    np.testing.assert_array_equal(host_bf16(rows), O.f32_to_bf16(O.dequantize(*emb, 64, 4)[ids]))
    assert _bits_equal(sx.weight, t["model.layers.0.mlp.switch_mlp.gate_proj.weight"])


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_shards_read_from_the_file(q38, tmp_path, world):
    _mini_checkpoint(tmp_path)
    modules, _ = loader.load_mlx_modules(str(tmp_path))
    lin = modules["model.layers.0.mlp.gate_proj"]
    full = (lin.weight, lin.scales, lin.biases)
    with loader.SafetensorsFile(str(tmp_path / "model.safetensors")) as f:
        for rank in range(world):
            got_r = loader.load_quantized_shard(f, "model.layers.0.mlp.gate_proj", rank, world, "rows", 64, 4)
            ref_r = parallel.shard_rows(*full, rank, world)
            got_k = loader.load_quantized_shard(f, "model.layers.0.mlp.gate_proj", rank, world, "k", 64, 4)
            ref_k = parallel.shard_k(*full, rank, world, 4, 64)
            for a, b in zip(got_r + got_k, ref_r + ref_k):
                assert _bits_equal(a, b)


def test_bonsai2_pack_end_to_end(q38, tmp_path):
    t, cfg = bonsai_pack(tmp_path)
    modules, tensors = loader.load_bonsai2(str(tmp_path))
    lin = modules["language_model.model.layers.0.mlp.gate_proj"]
    em = modules["language_model.model.embed_tokens"]
    assert isinstance(lin, q38.HadamardQuantizedLinear) and isinstance(em, q38.HadamardQuantizedEmbedding)
    assert (lin.group_size, lin.bits, lin.block) == (128, 2, 1024) and lin.scales.dtype == torch.float16
    assert not any(k.endswith(".signs") for k in tensors)
    assert "vision_tower.blocks.0.weight" in tensors
    x = torch.randn((2, 2048), device="cuda").half()
    y = lin(x)
    w, s, b, sg = (t["language_model.model.layers.0.mlp.gate_proj." + k].cuda() for k in ("weight", "scales", "biases", "signs"))
    ref = q38.quantized_matmul(q38.hadamard_rotate(x, sg, 1024), w.view(torch.int32), s, b, True, 128, 2)
    ids = torch.tensor([0, 47, 3], dtype=torch.int32, device="cuda")
    e = em(ids)
    ew, es, eb, esg = (t["language_model.model.embed_tokens." + k].cuda() for k in ("weight", "scales", "biases", "signs"))
    eref = q38.hadamard_rotate(q38.quantized_embedding(ids, ew.view(torch.int32), es, eb, 128, 2), esg, 1024,
                               inverse=True)
    torch.cuda.synchronize()
    q38.check_device()
    assert _bits_equal(y, ref) and _bits_equal(e, eref)
    _, text_only = loader.load_bonsai2(str(tmp_path), text_only=True)
    assert "vision_tower.blocks.0.weight" not in text_only


def test_bonsai2_missing_weights(q38, tmp_path):
    bonsai_pack(tmp_path)
    cfg = json.loads((tmp_path / "config.json").read_text())
    cfg["modules"].append({"path": "model.layers.1.mlp.up_proj", "block": 1024, "embedding": False,
                           "dtype": "float16"})
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(loader.Bonsai2LoaderError) as e:
        loader.load_bonsai2(str(tmp_path))
    assert e.value.kind == "missingWeights"
