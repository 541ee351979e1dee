"""Generate the golden fixtures that pin the oracle's packed-format handling.

MLX itself cannot run in this environment, so the packed layout is pinned against
an independent implementation of the same MLX affine format: the
``_affine_quantize_tensor`` / ``_affine_dequantize_tensor`` pair in
transformers 5.5 (``transformers/integrations/metal_quantization.py``), which
packs element ``i`` of each uint32 word at bit ``bits*i`` (LSB first) and
dequantizes ``w = scale*q + bias`` per group.  It covers bits 2, 4 and 8 (powers
of two only); the 3-bit bitstream layout stays unpinned.

Run from the repository root:  python tests/golden/make_golden.py
Writes tests/golden/affine_format.npz (a few hundred KB).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402

from transformers.integrations.metal_quantization import (  # noqa: E402
    _affine_dequantize_tensor,
    _affine_quantize_tensor,
)


def main() -> None:
    out = {}
    N, K, M, group = 32, 256, 4, 64
    for bits in (2, 4, 8):
        seed = 1000 + bits
        w = O.normal_f32(seed, (N, K), 0.02)
        x = O.normal_bf16(seed + 1, (M, K), 1.0)
        # third-party quantizer + packer; scales/biases narrowed to bf16 (the MLX storage type)
        packed, s32, b32 = _affine_quantize_tensor(torch.from_numpy(w), group, bits)
        codes = packed.numpy().view(np.uint32).copy()
        s16 = O.f32_to_bf16(s32.numpy())
        b16 = O.f32_to_bf16(b32.numpy())
        deq = _affine_dequantize_tensor(
            torch.from_numpy(codes.view(np.int32)).to(torch.uint32),
            torch.from_numpy(O.bf16_to_f32(s16)), torch.from_numpy(O.bf16_to_f32(b16)), group, bits,
        ).numpy()
        # reference product in float64 from the third-party dequantization
        y64 = O.bf16_to_f32(x).astype(np.float64) @ deq.astype(np.float64).T
        out[f"b{bits}_codes"] = codes
        out[f"b{bits}_scales"] = s16
        out[f"b{bits}_biases"] = b16
        out[f"b{bits}_dequant"] = deq.astype(np.float32)
        out[f"b{bits}_x"] = x
        out[f"b{bits}_y"] = y64.astype(np.float32)
        # the oracle's own quantizer output dequantized by the third-party routine
        oc, os_, ob = O.quantize(w, group, bits)
        odeq = _affine_dequantize_tensor(
            torch.from_numpy(oc.view(np.int32)).to(torch.uint32),
            torch.from_numpy(O.bf16_to_f32(os_)), torch.from_numpy(O.bf16_to_f32(ob)), group, bits,
        ).numpy()
        out[f"b{bits}_oracle_codes"] = oc
        out[f"b{bits}_oracle_scales"] = os_
        out[f"b{bits}_oracle_biases"] = ob
        out[f"b{bits}_oracle_dequant_3p"] = odeq.astype(np.float32)
    path = os.path.join(HERE, "affine_format.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
