"""Benchmark of the MLX-affine quantized products on B200: the decode GEMV sweep (the
headline line), plus the MoE expert-stack layer ("moe") and the prompt-shaped GEMM
("prefill") as secondary objects of the same JSON line.

Workload (one "step"): the decode GEMV sweep -- x bf16 N(0,1), W N(0, 0.02^2) quantized
affine group 64 at bits {2,3,4,8}, shapes N x K in {17408x5120, 5120x17408, 6144x5120},
M in {1, 8}: 24 products.  All M=1 products run before the M=8 ones, so the ~550 MB of
packed weights a step streams evict each other from the 126 MB L2 between reuses.

Reported metric: achieved algorithmic HBM GB/s over the whole step
(bytes = codes + bf16 scales/biases + x + y per product), device-timed with CUDA events,
max over ranks.  With --gpus N each rank runs an independent replica (the decode product
does not shard; weak scaling).

--impl reference times the CPU restatement of the same operator (the reference's own
implementation is MLX on Apple silicon and cannot run here) on a bounded sample of the
same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen38-mlx-swift_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

SHAPES = [(17408, 5120), (5120, 17408), (6144, 5120)]
BITS = [2, 3, 4, 8]
MS = [1, 8]
GROUP = 64
METRIC = "qmm decode HBM GB/s (% of 8 TB/s); MoE expert-stack tokens/s at 1/2/4/8 B200"


def algo_bytes(M, N, K, bits, group=GROUP):
    return N * K * bits // 8 + N * (K // group) * 2 * 2 + 2 * M * K + 2 * M * N


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Polls nvidia-smi for SM clocks and throttle reasons while the timed work runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, period: float = 0.05):
        self.index = index
        self.period = period
        self.lines: list[str] = []
        self.stop_evt = threading.Event()
        self.t = None
        self.ok = True

    def _poll(self):
        while not self.stop_evt.is_set():
            try:
                r = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                    "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10)
                if r.returncode == 0:
                    self.lines += [ln.strip() for ln in r.stdout.splitlines() if ln.strip()]
            except (OSError, subprocess.SubprocessError):
                self.ok = False
                return
            self.stop_evt.wait(self.period)

    def start(self):
        self.t = threading.Thread(target=self._poll, daemon=True)
        self.t.start()

    def stop(self):
        self.stop_evt.set()
        if self.t:
            self.t.join(timeout=15)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


def physical_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p for p in vis.split(",") if p.strip()]
        if local_rank < len(parts) and parts[local_rank].strip().isdigit():
            return int(parts[local_rank])
    return local_rank


def build_case_weights(torch, O, dev, bits, N, K, seed, copies=1):
    """Quantized weights for one (bits, shape): generated once on the CPU oracle for the
    first copy; extra copies are device clones (distinct memory, same values)."""
    w = O.normal_f32(seed, (N, K), 0.02)
    c, s, b = O.quantize(w, GROUP, bits)
    del w
    tc = torch.from_numpy(c.view(np.int32)).to(dev)
    ts = torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).to(dev)
    tb = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(dev)
    out = [(tc, ts, tb)]
    for _ in range(copies - 1):
        out.append((tc.clone(), ts.clone(), tb.clone()))
    return out


# ------------------------------------------------------------------------ gate/up
def run_gate_up(torch, q38, O, dev, stream, quick=False):
    """Gate and up projections of the dense MLP at decode (4-bit, 17408x5120 each, M 1 and 8):
    q38_quantized_gate_up (one pass over both weights, SiLU-gate in the epilogue) against
    the same work as two products and the SiLU product.  CUDA-graph replays over 4 weight
    pairs (357 MB, more than L2), CUDA events."""
    N, K, bits, copies = 17408, 5120, 4, 4
    gw = build_case_weights(torch, O, dev, bits, N, K, 6101, copies)
    uw = build_case_weights(torch, O, dev, bits, N, K, 6102, copies)
    nbytes = 2 * (N * K * bits // 8 + N * (K // GROUP) * 4)
    out = {}
    reps = 40 if quick else 200
    for M in (1, 8):
        x = torch.randn((M, K), device=dev).to(torch.bfloat16)

        def fused():
            for i in range(reps):
                q38.quantized_gate_up(x, gw[i % copies], uw[i % copies], GROUP, bits)

        def separate():
            for i in range(reps):
                q38.silu_mul(q38.quantized_matmul(x, *gw[i % copies], True, GROUP, bits),
                             q38.quantized_matmul(x, *uw[i % copies], True, GROUP, bits))

        res = {}
        for name, fn in (("fused", fused), ("separate", separate)):
            fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            res[name] = e0.elapsed_time(e1) * 1e3 / reps
            del g
        out[str(M)] = {"fused_us": round(res["fused"], 2), "separate_us": round(res["separate"], 2),
                       "fused_GBps": round(nbytes / (res["fused"] * 1e-6) / 1e9, 1)}
    return {"workload": "MLP gate+up at decode: 4-bit g64, gate and up 17408x5120, h = silu(gate) * up",
            "bytes_per_call": nbytes, "per_M": out}


def run_loader(torch, q38, dev, quick=False):
    """Checkpoint loading: a safetensors file shaped like 16 packed 4-bit 17408x5120
    projections (codes U32, scales and biases BF16; 800 MB) read into device tensors
    through libq38's reader (mapped file -> pinned staging -> device), host clock around
    the whole load plus a device synchronise, page cache warm.  Beside it, for context, the
    safetensors package loading the same file straight to the device."""
    import json as _json
    import shutil
    import struct
    import tempfile
    import time
    import loader
    n_proj = 4 if quick else 16
    N, K, bits = 17408, 5120, 4
    d = tempfile.mkdtemp(prefix="q38_load_")
    path = os.path.join(d, "model.safetensors")
    try:
        header, off, parts = {}, 0, []
        rng = np.random.default_rng(77)
        codes = rng.integers(0, 2 ** 32, size=(N, K * bits // 32), dtype=np.uint32)
        sc = rng.integers(0, 2 ** 16, size=(N, K // GROUP), dtype=np.uint16)
        for i in range(n_proj):
            for name, arr, dt in (("weight", codes, "U32"), ("scales", sc, "BF16"), ("biases", sc, "BF16")):
                key = f"model.layers.{i}.mlp.proj.{name}"
                header[key] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + arr.nbytes]}
                off += arr.nbytes
                parts.append(arr)
        h = _json.dumps(header).encode()
        h += b" " * (-len(h) % 8)
        with open(path, "wb") as fh:
            fh.write(struct.pack("<Q", len(h)) + h)
            for a in parts:
                fh.write(a.tobytes())
        total = off
        with open(path, "rb") as fh:  # page cache warm
            while fh.read(1 << 26):
                pass

        def ours():
            with loader.SafetensorsFile(path) as f:
                out = [f.to_device(k, dev) for k in f.keys()]
            torch.cuda.synchronize()
            return out

        def package():
            import safetensors.torch as st
            out = st.load_file(path, device=str(dev))
            torch.cuda.synchronize()
            return out

        res = {}
        for name, fn in (("q38_reader", ours), ("safetensors_package", package)):
            best = None
            for _ in range(3):
                t0 = time.perf_counter()
                out = fn()
                dt = time.perf_counter() - t0
                best = dt if best is None else min(best, dt)
                del out
            res[name] = {"seconds": round(best, 4), "GBps": round(total / best / 1e9, 2)}
        return {"workload": f"{n_proj} packed 4-bit 17408x5120 projections (U32 codes, BF16 scales/biases)",
                "bytes": total, "timing": "host clock, best of 3, page cache warm", **res}
    finally:
        shutil.rmtree(d, ignore_errors=True)


def _ternary_weight(torch, dev, g, N, K, group, sdtype):
    """Bonsai-style weight: codes uniform in {0, 1, 2} (w in {-s, 0, +s}), 2-bit packed,
    scale |N(0, 0.02^2)| per group, bias = -scale."""
    codes = torch.randint(0, 3, (N, K), generator=g, device=dev, dtype=torch.int64)
    words = torch.zeros((N, K // 16), dtype=torch.int64, device=dev)
    for j in range(16):
        words |= codes[:, j::16] << (2 * j)
    del codes
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    s = (torch.randn((N, K // group), generator=g, device=dev) * 0.02).abs().to(sdtype)
    return words, s, -s


def _graph_us(torch, fn, reps):
    fn()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        fn()
    gr.replay()
    torch.cuda.synchronize()
    best = None
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gr.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e3 / reps
        best = t if best is None else min(best, t)
    del gr
    return best


def run_bonsai(torch, q38, dev, quick=False):
    """Bonsai ternary 2-bit projections with Hadamard-rotated activations (rotation, then the
    product: q38_hadamard_quantized_matmul through HadamardQuantizedLinear), block 256,
    group 64, bf16 scales, N x K in {17408 x 5120, 5120 x 17408}, M in {1, 8, 2048};
    CUDA-graph replays over 8 weight copies (more than L2).  Also the published pack's layout
    (group 128, f16 scales and biases, block 1024) at decode, bf16 activations."""
    out = {}
    g = torch.Generator(device=dev).manual_seed(4040)
    copies = 8
    for (N, K) in ((17408, 5120), (5120, 17408)):
        mods = []
        for _ in range(copies):
            w, s, b = _ternary_weight(torch, dev, g, N, K, GROUP, torch.bfloat16)
            signs = torch.where(torch.rand(K, generator=g, device=dev) < 0.5, -1.0, 1.0)
            mods.append(q38.HadamardQuantizedLinear(q38.QuantizedLinear(w, s, b, None, GROUP, 2), signs, 256))
        wbytes = N * K // 4 + N * (K // GROUP) * 4
        for M in ((1, 8) if quick else (1, 8, 2048)):
            x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
            reps = 8 if M == 2048 else 200

            def fn():
                for i in range(reps):
                    mods[i % copies](x)

            us = _graph_us(torch, fn, reps)
            row = {"us": round(us, 2), "GBps": round((wbytes + 2 * M * K + 2 * M * N) / (us * 1e-6) / 1e9, 1)}
            if M == 2048:
                row["TFLOPs"] = round(2 * M * N * K / (us * 1e-6) / 1e12, 1)
            out[f"{N}x{K} M={M}"] = row
        del mods
    # the published pack's layout at decode: group 128, f16 scales, block 1024
    N, K = 17408, 5120
    mods = []
    for _ in range(copies):
        w, s, b = _ternary_weight(torch, dev, g, N, K, 128, torch.float16)
        signs = torch.where(torch.rand(K, generator=g, device=dev) < 0.5, -1.0, 1.0)
        mods.append(q38.HadamardQuantizedLinear(q38.QuantizedLinear(w, s, b, None, 128, 2), signs, 1024))
    for M in ((1, 8) if quick else (1, 8, 2048)):
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        reps = 8 if M == 2048 else 100

        def fn2():
            for i in range(reps):
                mods[i % copies](x)

        us = _graph_us(torch, fn2, reps)
        wbytes = N * K // 4 + N * (K // 128) * 4
        row = {"us": round(us, 2), "GBps": round(wbytes / (us * 1e-6) / 1e9, 1)}
        if M == 2048:
            row["TFLOPs"] = round(2 * M * N * K / (us * 1e-6) / 1e12, 1)
        out[f"pack layout g128 f16 {N}x{K} M={M}"] = row
    # MLP gate + up over the pack layout: one rotation and one pass over both weights
    # (q38_hadamard_quantized_gate_up) against two rotated projections and the SiLU product
    sg = mods[0].signs
    pairs = [((mods[2 * i].weight, mods[2 * i].scales, mods[2 * i].biases),
              (mods[2 * i + 1].weight, mods[2 * i + 1].scales, mods[2 * i + 1].biases)) for i in range(copies // 2)]
    for M in (1, 8):
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)

        def fused():
            for i in range(100):
                q38.hadamard_quantized_gate_up(x, sg, 1024, *pairs[i % len(pairs)], 128, 2)

        def separate():
            for i in range(100):
                gp, up = pairs[i % len(pairs)]
                q38.silu_mul(q38.quantized_matmul(q38.hadamard_rotate(x, sg, 1024), *gp, True, 128, 2),
                             q38.quantized_matmul(q38.hadamard_rotate(x, sg, 1024), *up, True, 128, 2))

        fus, sep = _graph_us(torch, fused, 100), _graph_us(torch, separate, 100)
        out[f"pack layout MLP gate+up {N}x{K} M={M}"] = {
            "fused_us": round(fus, 2), "separate_us": round(sep, 2),
            "fused_GBps": round(2 * (N * K // 4 + N * (K // 128) * 4) / (fus * 1e-6) / 1e9, 1)}
    del mods
    return {"workload": "Bonsai ternary 2-bit: rotation (block 256) + product, group 64 bf16; ternary codes, "
                        "bias = -scale", "per_case": out,
            "timing": "CUDA-graph replays over 8 weight copies, CUDA events, best of 3"}


def run_lm_head(torch, q38, dev, quick=False):
    """Tied output projection of a 248,320-token vocabulary (4-bit g64, K = 5120, 636 MB of
    codes, larger than L2) at M = 1 and 8, and the embedding lookup of 1 and 8 ids."""
    rows, K, bits = 248320, 5120, 4
    g = torch.Generator(device=dev).manual_seed(5050)
    c = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows, K * bits // 32), dtype=torch.int32, device=dev, generator=g)
    s = (torch.rand((rows, K // GROUP), device=dev, generator=g) * 0.01).to(torch.bfloat16)
    b = ((torch.rand((rows, K // GROUP), device=dev, generator=g) - 0.5) * 0.02).to(torch.bfloat16)
    emb = q38.QuantizedEmbedding(c, s, b, GROUP, bits)
    wbytes = rows * K * bits // 8 + rows * (K // GROUP) * 4
    out = {}
    for M in (1, 8):
        x = torch.randn((M, K), device=dev, generator=g).to(torch.bfloat16)
        reps = 10 if quick else 40

        def fn():
            for _ in range(reps):
                emb.as_linear(x)

        us = _graph_us(torch, fn, reps)
        out[f"as_linear M={M}"] = {"us": round(us, 2), "GBps": round(wbytes / (us * 1e-6) / 1e9, 1)}
    for n in (1, 8):
        ids = torch.randint(0, rows, (n,), device=dev, generator=g, dtype=torch.int32)

        def fl():
            for _ in range(100):
                emb(ids)

        out[f"lookup ids={n}"] = {"us": round(_graph_us(torch, fl, 100), 2)}
    del emb, c, s, b
    return {"workload": "248,320 x 5120 4-bit g64 embedding: tied output projection and lookup",
            "weight_bytes": wbytes, "per_case": out, "timing": "CUDA-graph replays, CUDA events, best of 3"}


# ----------------------------------------------------------------------------- MoE
MOE = {"H": 2048, "I": 512, "E": 512, "k": 10, "bits": 3}
MOE_T = [1, 8, 64, 4096]


def moe_expert_bytes():
    H, I, bits = MOE["H"], MOE["I"], MOE["bits"]
    per = 0
    for (n, k) in ((I, H), (I, H), (H, I)):
        per += n * k * bits // 8 + n * (k // GROUP) * 2 * 2
    return per


def build_moe(torch, q38, dev, seed=3030):
    """Flash-Next-shaped expert stack: gate/up [512, 512, 2048], down [512, 2048, 512], each
    N(0, 0.02^2) quantized 3-bit group 64 on the device (the quantizer is bit-exact with the
    oracle's); router weight [512, 2048] bf16 N(0, 0.02^2)."""
    H, I, E, bits = MOE["H"], MOE["I"], MOE["E"], MOE["bits"]
    g = torch.Generator(device=dev).manual_seed(seed)
    W = []
    for (n, k) in ((I, H), (I, H), (H, I)):
        w = torch.randn((E * n, k), generator=g, device=dev) * 0.02
        c, s, b = q38.quantize(w, GROUP, bits, scales_dtype=torch.bfloat16)
        W.append((c.view(torch.int32).view(E, n, -1), s.view(E, n, -1), b.view(E, n, -1)))
        del w
    wr = (torch.randn((E, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    sw = q38.SwitchGLU(*[q38.QuantizedSwitchLinear(c, s, b, GROUP, bits) for (c, s, b) in W])
    return q38.SparseMoeBlock(wr, sw, MOE["k"]), g


def make_comm(q38, dist, rank, world, dev):
    """libq38 communicator (q38_comm_init_rank): rank 0's id reaches the others through the
    torch process group (host plumbing only)."""
    box = [q38.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return q38.Communicator(box[0], world, rank, dev.index, timeout_ms=120000)


def run_moe_ep(torch, q38, dev, stream, world, rank, dist, comm, quick=False):
    """Expert-parallel MoE layer through the C ABI (q38_moe_route on each rank's tokens, then
    q38_ep_switch_glu: experts split contiguously over the ranks, fixed-capacity NCCL
    exchange of every rank's T tokens to every rank, partial sums returned and added at
    home).  T tokens per rank (weak scaling); the R layer calls of a step are captured in a
    CUDA graph with their NCCL exchanges and replayed; CUDA events, max over ranks."""
    H, I, E, k, bits = MOE["H"], MOE["I"], MOE["E"], MOE["k"], MOE["bits"]
    epr = E // world
    g = torch.Generator(device=dev).manual_seed(3030 + rank)
    mine = []
    for (n, kk) in ((I, H), (I, H), (H, I)):
        w = torch.randn((epr * n, kk), generator=g, device=dev) * 0.02
        c, s, b = q38.quantize(w, GROUP, bits, scales_dtype=torch.bfloat16)
        mine.append((c.view(torch.int32).view(epr, n, -1), s.view(epr, n, -1), b.view(epr, n, -1)))
        del w
    gw = torch.Generator(device=dev).manual_seed(3131)  # router weight identical on all ranks
    wr = (torch.randn((E, H), generator=gw, device=dev) * 0.02).to(torch.bfloat16)

    def layer(x):
        idx, sc = q38.moe_route(x, wr, k)
        return q38.ep_switch_glu(comm, x, idx, sc, *mine, E, x.shape[0], GROUP, bits)
    out = {}
    for T in MOE_T:
        R = 4 if T <= 64 else 2
        reps = (3 if quick else 10) if T <= 64 else (2 if quick else 5)
        xs = [torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16) for _ in range(R)]
        for x in xs:
            layer(x)
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for x in xs:
                layer(x)
        graph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * R)
        t = torch.tensor([us], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
        del graph  # released before the communicators and the process group
        out[str(T)] = {"tokens_per_s": round(world * T / (us * 1e-6), 1), "us_per_layer": round(us, 2),
                       "tokens_per_rank": T}
        del xs
    del mine
    torch.cuda.synchronize()
    return {"metric": "MoE expert-stack tokens/s (router + SwitchGLU + combine, one layer)", "unit": "tokens/s",
            "per_T": out,
            "config": {"workload": "Flash-Next MoE layer: hidden 2048, 512 experts, intermediate 512, top-10, "
                                   "3-bit group 64, router [512, 2048] bf16",
                       "parallelism": f"expert parallel x{world} ({epr} experts per GPU), T tokens per GPU",
                       "scaling": "weak",
                       "timing": "q38_moe_route + q38_ep_switch_glu (fixed capacity = T per rank, NCCL inside "
                                 "libq38) captured in a CUDA graph, CUDA events, max over ranks"}}


def run_moe(torch, q38, dev, stream, world, dist, quick=False):
    """One MoE layer (router + SwitchGLU + combine) per step at each token count, timed as
    CUDA-graph replays; each replay cycles through R different token batches so that the
    experts a batch selects are not L2-resident from the previous one."""
    blk, g = build_moe(torch, q38, dev)
    H, k = MOE["H"], MOE["k"]
    ebytes = moe_expert_bytes()
    out = {}
    for T in MOE_T:
        R = 16 if T <= 64 else 2
        reps = (5 if quick else 30) if T <= 64 else (2 if quick else 10)
        xs = [torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16) for _ in range(R)]
        for x in xs:
            blk(x)
        torch.cuda.synchronize()
        touched = sum(int(torch.unique(q38.moe_route(x, blk.router_weight, k)[0]).numel()) for x in xs) / R
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for x in xs:
                blk(x)
        gr.replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            gr.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * R)
        if dist:
            t = torch.tensor([us], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item())
        del gr
        # e2e through the public API: host batch -> device, layer, result -> host
        hx = xs[0].cpu().pin_memory()
        hy = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
        dx = torch.empty_like(xs[0])
        n_e2e = 3 if T == 4096 else 20

        def e2e_once():
            dx.copy_(hx, non_blocking=True)
            hy.copy_(blk(dx), non_blocking=True)
        e2e_once()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(n_e2e):
            e2e_once()
        a1.record(stream)
        torch.cuda.synchronize()
        e2e_us = a0.elapsed_time(a1) * 1e3 / n_e2e
        if dist:
            t = torch.tensor([e2e_us], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_us = float(t.item())
        wbytes = touched * ebytes + MOE["E"] * H * 2 + 2 * T * H * 2
        flops = T * k * 2 * (3 * MOE["I"] * H) + T * 2 * H * MOE["E"]
        out[str(T)] = {"tokens_per_s": round(world * T / (us * 1e-6), 1), "us_per_layer": round(us, 2),
                       "experts_touched": round(touched, 1), "weight_GBps": round(wbytes / (us * 1e-6) / 1e9, 1),
                       "TFLOPs": round(flops / (us * 1e-6) / 1e12, 2),
                       "e2e_tokens_per_s": round(world * T / (e2e_us * 1e-6), 1),
                       "e2e_h2d_bytes": T * H * 2, "e2e_d2h_bytes": T * H * 2}
        del xs, hx, hy, dx
    del blk
    torch.cuda.synchronize()
    return {"metric": "MoE expert-stack tokens/s (router + SwitchGLU + combine, one layer)",
            "unit": "tokens/s", "per_T": out,
            "config": {"workload": "Flash-Next MoE layer: hidden 2048, 512 experts, intermediate 512, top-10, "
                                   "3-bit group 64, router [512, 2048] bf16",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "timing": "CUDA-graph replays cycling 16 (T<=64) or 2 (T=4096) token batches, CUDA events"},
            "bytes_per_expert": ebytes}


# ------------------------------------------------------------------------- prefill
def run_prefill_tp(torch, q38, dev, stream, world, rank, dist, comm, quick=False):
    """Tensor-parallel dense MLP stack at 4096 tokens, 4-bit, through the C ABI
    (q38_tp_mlp): per layer gate/up split by output rows, down by its reduction dimension,
    partial outputs summed by a bf16 all-reduce inside libq38 that overlaps the next token
    chunk's products; 64 layers of random-init weights, every layer reading the same x
    (strong scaling: the whole stack on every step)."""
    M, D, F = 4096, 5120, 17408
    L = 8 if quick else 64
    Fl = F // world
    g = torch.Generator(device=dev).manual_seed(4040 + rank)
    layers = []
    for _ in range(L):
        mats = []
        for (n, k) in ((Fl, D), (Fl, D), (D, Fl)):  # this rank's shards (random: every rank its own)
            w = torch.randn((n, k), generator=g, device=dev) * 0.02
            c, s, b = q38.quantize(w, GROUP, 4, scales_dtype=torch.bfloat16)
            mats.append((c.view(torch.int32), s, b))
            del w
        layers.append(mats)
    gx = torch.Generator(device=dev).manual_seed(4141)
    x = torch.randn((M, D), generator=gx, device=dev).to(torch.bfloat16)
    outs = [torch.empty_like(x) for _ in range(2)]

    def stack():
        for i, (ga, up, dn) in enumerate(layers):
            outs[i & 1].copy_(q38.tp_mlp(comm, x, ga, up, dn, GROUP, 4, chunks=0))
    stack()
    torch.cuda.synchronize()
    dist.barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        stack()
    graph.replay()
    torch.cuda.synchronize()
    reps = 1 if quick else 3
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    t = torch.tensor([us], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item())
    del graph
    flops = L * 3 * 2 * M * F * D
    peak = None
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peak = float(json.load(open(p))["bf16_tflops_sustained"])
    tf = flops / (us * 1e-6) / 1e12
    del layers, x, outs
    torch.cuda.synchronize()
    return {"metric": "prefill quantized MLP stack TFLOP/s (tensor pipe)", "unit": "TFLOP/s", "value": round(tf, 1),
            "us_per_stack": round(us, 1), "us_per_layer": round(us / L, 1), "layers": L,
            "frac_of_measured_bf16_peak_sustained_per_gpu": round(tf / world / peak, 4) if peak else None,
            "tokens_per_s": round(M / (us * 1e-6), 1),
            "config": {"workload": f"{L} layers x 4096 tokens x 4-bit g64 MLP: gate, up 17408x5120 -> SiLU-gate -> "
                                   "down 5120x17408, bf16 all-reduce; every layer reads the same x",
                       "parallelism": f"tensor parallel x{world}", "scaling": "strong",
                       "timing": "q38_tp_mlp (token chunks chosen by the library, all-reduce overlapped, NCCL inside libq38) "
                                 "stack captured in a CUDA graph, CUDA events, max over ranks"}}


def run_prefill(torch, q38, dev, stream, world, dist, quick=False):
    """Dense-27B MLP stack at 4096 tokens, 4-bit group 64: 64 layers of random-init weights,
    each down(silu(gate(x)) * up(x)) through q38.QuantizedMLP (gate, up 17408 x 5120; the
    SiLU product; down 5120 x 17408).  Every layer reads the same x [4096, 5120]: random
    layers stacked on each other's output grow without bound (no normalisation or
    residual here), so the stack feeds each layer the same activations."""
    M, D, F = 4096, 5120, 17408
    L = 8 if quick else 64
    g = torch.Generator(device=dev).manual_seed(4040)
    layers = []
    for _ in range(L):
        mats = []
        for (n, k) in ((F, D), (F, D), (D, F)):
            w = torch.randn((n, k), generator=g, device=dev) * 0.02
            c, s, b = q38.quantize(w, GROUP, 4, scales_dtype=torch.bfloat16)
            mats.append(q38.QuantizedLinear(c.view(torch.int32), s, b, None, GROUP, 4))
            del w
        layers.append(q38.QuantizedMLP(*mats))
    x = torch.randn((M, D), generator=g, device=dev).to(torch.bfloat16)
    outs = [torch.empty((M, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]

    def stack():
        for i, mlp in enumerate(layers):
            outs[i & 1].copy_(mlp(x))
    stack()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        stack()
    gr.replay()
    torch.cuda.synchronize()
    reps = 1 if quick else 3
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        gr.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    if dist:
        t = torch.tensor([us], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
    flops = L * 3 * 2 * M * F * D
    peak = None
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peak = float(json.load(open(p))["bf16_tflops_sustained"])
    tf = flops / (us * 1e-6) / 1e12
    del gr, layers, x, outs
    torch.cuda.synchronize()
    return {"metric": "prefill quantized MLP stack TFLOP/s (tensor pipe)", "unit": "TFLOP/s",
            "value": round(world * tf, 1), "us_per_stack": round(us, 1), "us_per_layer": round(us / L, 1),
            "layers": L, "frac_of_measured_bf16_peak_sustained": round(tf / peak, 4) if peak else None,
            "tokens_per_s": round(world * M / (us * 1e-6), 1),
            "config": {"workload": f"{L} layers x 4096 tokens x 4-bit g64 MLP (QuantizedMLP: gate, up 17408x5120, "
                                   "SiLU product, down 5120x17408); every layer reads the same x",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "timing": "CUDA-graph replay of the whole stack, CUDA events; peak = sustained bf16 "
                                 "(a seconds-long step)"}}


def run_prefill_bits(torch, q38, dev, stream, quick=False):
    """One prompt-sized product per code width on the tensor-core prefill kernel: x bf16
    [4096, 5120] . W [17408, 5120]^T, group 64, bits 2/3/4/8 (random-init weights quantized
    on the device).  CUDA-graph replays cycling 4 weight copies, CUDA events, best of 3;
    peak = burst bf16 (the replay lasts milliseconds)."""
    M, N, K = 4096, 17408, 5120
    g = torch.Generator(device=dev).manual_seed(4141)
    x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
    peak = None
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peak = float(json.load(open(p))["bf16_tflops"])
    nrep = 8 if quick else 20
    out = {}
    for bits in (2, 3, 4, 8):
        w = torch.randn((N, K), generator=g, device=dev) * 0.02
        c, s, b = q38.quantize(w, GROUP, bits, scales_dtype=torch.bfloat16)
        del w
        mats = [(c.view(torch.int32), s, b)]
        mats += [(m[0].clone(), m[1].clone(), m[2].clone()) for m in mats * 3]

        def body():
            for i in range(nrep):
                q38.quantized_matmul(x, *mats[i % 4], True, GROUP, bits)
        body()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            body()
        gr.replay()
        torch.cuda.synchronize()
        best = None
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            gr.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / nrep
            best = us if best is None else min(best, us)
        tf = 2.0 * M * N * K / (best * 1e-6) / 1e12
        out[str(bits)] = {"us": round(best, 1), "TFLOPs": round(tf, 1),
                          "frac_of_measured_bf16_peak": round(tf / peak, 4) if peak else None}
        del gr, mats, c, s, b
        torch.cuda.synchronize()
    q38.check_device()
    return {"workload": "x bf16 [4096, 5120] . W[17408, 5120]^T, group 64, per code width",
            "timing": "CUDA-graph replays over 4 weight copies, CUDA events, best of 3; peak = burst bf16",
            "per_bits": out}


def run_config1(torch, q38, O, dev, stream):
    """The single-product configuration: x bf16 [16, 4096] . W [11008, 4096]^T, 4-bit g64;
    200 launches in one graph over 8 weight copies (200 MB, more than L2)."""
    rot = build_case_weights(torch, O, dev, 4, 11008, 4096, 2026, copies=8)
    x = torch.from_numpy(O.normal_bf16(2027, (16, 4096)).view(np.int16)).view(torch.bfloat16).to(dev)
    y = torch.empty((16, 11008), dtype=torch.bfloat16, device=dev)
    nrep = 200

    def body():
        for i in range(nrep):
            q38.quantized_matmul(x, *rot[i % 8], True, GROUP, 4)
    body()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        body()
    g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / nrep
    nb = algo_bytes(16, 11008, 4096, 4)
    del g, rot
    return {"workload": "x bf16 [16, 4096] . W[11008, 4096]^T, 4-bit g64", "us": round(us, 2),
            "GBps": round(nb / (us * 1e-6) / 1e9, 1), "bytes": nb}


def run_ours(args, rank, world, local_rank):
    import torch
    import oracle as O
    import q38

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))

    # the sweep's weights and activations, built once on the host (the CPU baseline below
    # runs the oracle over the same arrays)
    host_cases = sweep_sample(O)
    cases = []  # (M, N, K, bits)
    weights, xs = {}, {}
    for (M, N, K, bits, c, s, b, x) in host_cases:
        cases.append((M, N, K, bits))
        if (bits, N, K) not in weights:
            weights[(bits, N, K)] = (torch.from_numpy(c.view(np.int32)).to(dev),
                                     torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).to(dev),
                                     torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(dev))
        if (M, K) not in xs:
            xs[(M, K)] = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
    ys = {(M, N): torch.empty((M, N), dtype=torch.bfloat16, device=dev) for M in MS for (N, _) in SHAPES}
    step_bytes = sum(algo_bytes(M, N, K, b) for (M, N, K, b) in cases)

    ctx = q38.context(dev)
    stream = torch.cuda.current_stream(dev)
    lib = q38._lib

    def call(M, N, K, bits, x, y, w=None):
        c, s, b = w if w is not None else weights[(bits, N, K)]
        lib.q38_ctx_set_stream(ctx, torch.cuda.current_stream(dev).cuda_stream)
        st = lib.q38_quantized_matmul(ctx, x.data_ptr(), M, K, 0, c.data_ptr(), s.data_ptr(), b.data_ptr(),
                                      0, N, 1, GROUP, bits, 0, y.data_ptr())
        if st != 0:
            raise RuntimeError(lib.q38_last_error(ctx).decode())

    def step():
        for (M, N, K, bits) in cases:
            call(M, N, K, bits, xs[(M, K)], ys[(M, N)])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
        return g

    # One step = one replay of a CUDA graph holding the 24 products (72 kernel launches);
    # replays are timed with CUDA events on the replaying stream.
    step_graph = capture(step)
    sampler = ClockSampler(physical_index(local_rank))
    sampler.start()
    for _ in range(max(args.warmup, 200)):
        step_graph.replay()
    torch.cuda.synchronize()
    q38.check_device(dev)

    # ---------------------------------------------------------------- timed region
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * step_bytes / (ms * 1e-3) / 1e9

    # eager (no graph) step time, for reference: includes host launch overhead
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(3):
        step()
    f1.record(stream)
    torch.cuda.synchronize()
    eager_ms = f0.elapsed_time(f1) / 3

    # per-case breakdown: a graph of 8 back-to-back launches of each product
    per_case = []
    for (M, N, K, bits) in cases:
        g = capture(lambda: [call(M, N, K, bits, xs[(M, K)], ys[(M, N)]) for _ in range(8)])
        g.replay()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(3):
            g.replay()
        c1.record(stream)
        torch.cuda.synchronize()
        us = c0.elapsed_time(c1) / 24 * 1e3
        per_case.append({"bits": bits, "M": M, "N": N, "K": K, "us": round(us, 2),
                         "GBps": round(algo_bytes(M, N, K, bits) / (us * 1e-6) / 1e9, 1)})
        del g

    # roofline of the dominant kernel: 4-bit 17408x5120 M=1, rotating 4 weight copies
    # (4 x 50 MB > L2) so every launch streams from HBM; 200 launches in one graph
    peak, peak_kind = measured_peaks()
    rot = build_case_weights(torch, O, dev, 4, 17408, 5120, 4242, copies=4)
    xr = xs[(1, 5120)]
    yr = ys[(1, 17408)]
    nrep = 200
    rg = capture(lambda: [call(1, 17408, 5120, 4, xr, yr, rot[i % 4]) for i in range(nrep)])
    rg.replay()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record(stream)
    rg.replay()
    r1.record(stream)
    torch.cuda.synchronize()
    launch_us = r0.elapsed_time(r1) / nrep * 1e3
    rbytes = algo_bytes(1, 17408, 5120, 4)
    achieved = rbytes / (launch_us * 1e-6) / 1e9
    roofline = {"bound": "hbm", "kernel": "qgemv_main<4,1,1> (+ qgemv_epilogue) 17408x5120 4-bit M=1",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "frac_of_8TBps": round(achieved / 8000.0, 4),
                "algorithmic_bytes_per_launch": rbytes, "launch_us": round(launch_us, 2),
                "timing": "CUDA events around one graph replay of 200 products (main kernel + epilogue each)",
                "traffic": None}
    tr = os.path.join(ROOT, "profiles", "qgemv_traffic.json")
    if os.path.exists(tr):
        roofline["traffic"] = json.load(open(tr)).get("bytes_per_launch")
    del rg, rot, step_graph
    torch.cuda.synchronize()

    # e2e through the public API with host buffers, inside the timed region every step: one
    # H2D copy of the step's inputs (each product's x, packed in one pinned buffer), the
    # products through q38.quantized_matmul writing into slices of one device buffer, and one
    # D2H copy of all the results
    x_off, y_off, xo, yo = [], [], 0, 0
    for (M, N, K, b) in cases:
        x_off.append(xo)
        y_off.append(yo)
        xo += M * K
        yo += M * N
    hx_all = torch.empty(xo, dtype=torch.bfloat16).pin_memory()
    for i, (M, N, K, b) in enumerate(cases):
        hx_all[x_off[i]:x_off[i] + M * K].copy_(xs[(M, K)].reshape(-1).cpu())
    hy_all = torch.empty(yo, dtype=torch.bfloat16).pin_memory()
    dx_all = torch.empty(xo, dtype=torch.bfloat16, device=dev)
    dy_all = torch.empty(yo, dtype=torch.bfloat16, device=dev)
    dxv = [dx_all[x_off[i]:x_off[i] + M * K].view(M, K) for i, (M, N, K, b) in enumerate(cases)]
    dyv = [dy_all[y_off[i]:y_off[i] + M * N].view(M, N) for i, (M, N, K, b) in enumerate(cases)]
    h2d = 2 * xo
    d2h = 2 * yo

    def e2e_step():
        dx_all.copy_(hx_all, non_blocking=True)
        for i, (M, N, K, bits) in enumerate(cases):
            q38.quantized_matmul(dxv[i], *weights[(bits, N, K)], True, GROUP, bits, out=dyv[i])
        hy_all.copy_(dy_all, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    a1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = a0.elapsed_time(a1) / args.steps
    if dist:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)}

    if world > 1:
        comm = make_comm(q38, dist, rank, world, dev) if not (args.skip_moe and args.skip_prefill) else None
        moe = None if args.skip_moe else run_moe_ep(torch, q38, dev, stream, world, rank, dist, comm, args.quick)
        prefill = None if args.skip_prefill else run_prefill_tp(torch, q38, dev, stream, world, rank, dist, comm,
                                                                args.quick)
        if comm is not None:
            torch.cuda.synchronize()
            dist.barrier()
            comm.destroy()
    else:
        moe = None if args.skip_moe else run_moe(torch, q38, dev, stream, world, dist, args.quick)
        prefill = None if args.skip_prefill else run_prefill(torch, q38, dev, stream, world, dist, args.quick)
    gate_up = None if (args.skip_prefill or world > 1) else run_gate_up(torch, q38, O, dev, stream, args.quick)
    load = None if (args.skip_prefill or world > 1) else run_loader(torch, q38, dev, args.quick)
    bonsai = None if (args.skip_prefill or world > 1) else run_bonsai(torch, q38, dev, args.quick)
    lm_head = None if (args.skip_prefill or world > 1) else run_lm_head(torch, q38, dev, args.quick)
    config1 = run_config1(torch, q38, O, dev, stream) if world == 1 else None
    prefill_bits = None if (args.skip_prefill or world > 1) else run_prefill_bits(torch, q38, dev, stream, args.quick)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(O, seconds=args.cpu_seconds, cases=host_cases)

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02^2) weights quantized by the oracle)",
        "config": {"workload": SWEEP_CONFIG["workload"],
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2: 550 MB of packed weights per step, M=1 pass before M=8 pass",
                   "step_bytes": step_bytes,
                   "timing": "one CUDA-graph replay per step (48 launches), CUDA events, max over ranks"},
        "frac_of_8TBps": round(value / world / 8000.0, 4),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": clocks,
        "gpu_launches": 2 * len(cases) * args.steps,
        "eager_ms_per_step": round(eager_ms, 4),
        "cases": per_case,
        "moe": moe,
        "prefill": prefill,
        "gate_up": gate_up,
        "loader": load,
        "bonsai": bonsai,
        "lm_head": lm_head,
        "config1": config1,
        "prefill_bits": prefill_bits,
    }
    return line


def sweep_sample(O):
    """The decode sweep's 24 products on the host: the same seeded weights (quantized by the
    oracle) and activations as the GPU arm builds."""
    cases = []
    w = {}
    for bi, bits in enumerate(BITS):
        for si, (N, K) in enumerate(SHAPES):
            wf = O.normal_f32(1000 + 10 * bi + si, (N, K), 0.02)
            w[(bits, N, K)] = O.quantize(wf, GROUP, bits)
            del wf
    xs = {(M, K): O.normal_bf16(77 + M + K, (M, K)) for M in MS for (_, K) in SHAPES}
    for M in MS:
        for bits in BITS:
            for (N, K) in SHAPES:
                cases.append((M, N, K, bits, *w[(bits, N, K)], xs[(M, K)]))
    return cases


def time_sweep(O, cases):
    """One pass over the sweep on the host cores; returns (bytes, seconds)."""
    nbytes = 0
    t0 = time.perf_counter()
    for (M, N, K, bits, c, s, b, x) in cases:
        O.qmm(x, c, s, b, GROUP, bits)
        nbytes += algo_bytes(M, N, K, bits)
    return nbytes, time.perf_counter() - t0


def cpu_baseline(O, seconds: float = 12.0, threads: int = 0, cases=None):
    """Oracle restatement of the whole decode sweep (24 products, the GPU arm's workload) on
    the host cores, repeated until `seconds` have passed (at least once)."""
    if threads:
        O.set_threads(threads)
    cores = O.threads()
    if cases is None:
        cases = sweep_sample(O)
    total_bytes, total_t, n = 0, 0.0, 0
    while True:
        b, t = time_sweep(O, cases)
        total_bytes += b
        total_t += t
        n += 1
        if total_t >= seconds:
            break
    return {"value": round(total_bytes / total_t / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{n} full decode sweeps (24 products, {total_bytes // n} bytes each) in {total_t:.1f} s"}


SWEEP_CONFIG = {"workload": "decode GEMV sweep: bits {2,3,4,8} x NxK {17408x5120, 5120x17408, 6144x5120} "
                            "x M {1,8}, affine group 64, 24 products per step"}


def run_reference(args, rank, world):
    """CPU reference arm: the oracle restatement of the decode sweep on the host cores, rank
    0 only; a step is one pass over all 24 products of the sweep."""
    if rank != 0:
        return None
    import oracle as O
    cores = O.threads()
    cases = sweep_sample(O)
    for _ in range(max(args.warmup, 1)):
        _, t_sweep = time_sweep(O, cases)
    # as many timed steps as fit about two minutes (the throughput does not depend on it)
    steps = max(1, min(args.steps, int(120.0 / max(t_sweep, 1e-3))))
    nbytes, secs = 0, 0.0
    for _ in range(steps):
        b, t = time_sweep(O, cases)
        nbytes += b
        secs += t
    v = round(nbytes / secs / 1e9, 3)
    return {
        "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(secs / steps * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": dict(SWEEP_CONFIG, parallelism="host CPU"),
        "impl": "reference",
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{steps} full decode sweeps (24 products each) in {secs:.1f} s"
                                   + ("" if steps == args.steps else f" (of {args.steps} requested: "
                                                                     "capped at about two minutes)")},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "MLX (the reference's implementation of this path) runs only on Apple silicon; "
                "this arm times the C restatement of its CPU semantics",
    }


def run_profile_case(args):
    """Small fixed workload for ncu captures: `--profile-bits` product of 17408x5120 at
    M=`--profile-m`, 4 rotated weight copies (> L2), 12 launches."""
    import torch
    import oracle as O
    import q38

    dev = torch.device("cuda", 0)
    bits, M, N, K = args.profile_bits, args.profile_m, 17408, 5120
    rot = build_case_weights(torch, O, dev, bits, N, K, 4242, copies=4)
    x = torch.from_numpy(O.normal_bf16(9, (M, K)).view(np.int16)).view(torch.bfloat16).to(dev)
    ys = []
    for i in range(12):
        ys.append(q38.quantized_matmul(x, *rot[i % 4], True, GROUP, bits))
    torch.cuda.synchronize()
    q38.check_device()
    print(json.dumps({"profile_case": {"bits": bits, "M": M, "N": N, "K": K, "launches": 12,
                                       "algorithmic_bytes_per_launch": algo_bytes(M, N, K, bits)}}))


def run_profile_prefill(args):
    """Small prompt-shaped case for ncu: `--profile-bits` codes, M=1024 tokens, N=9472 (37 row
    pairs x 4 token tiles = 148 pair tiles), K=5120; 3 products."""
    import torch
    import q38
    dev = torch.device("cuda", 0)
    M, N, K, bits = 1024, 9472, 5120, args.profile_bits
    g = torch.Generator(device=dev).manual_seed(5050)
    c, s, b = q38.quantize(torch.randn((N, K), generator=g, device=dev) * 0.02, GROUP, bits,
                           scales_dtype=torch.bfloat16)
    x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
    for _ in range(3):
        y = q38.quantized_matmul(x, c.view(torch.int32), s, b, True, GROUP, bits)
    torch.cuda.synchronize()
    q38.check_device()
    print(json.dumps({"profile_prefill": {"M": M, "N": N, "K": K, "bits": bits, "launches": 3,
                                          "flops_per_launch": 2 * M * N * K, "mean_abs_y": float(y.float().abs().mean())}}))


def run_profile_bonsai(args):
    """Small fixed workload for ncu captures of the Bonsai 2 pack path: 12 rotated projections
    (block 1024, then the group-128 f16-scale decode product) of 17408x5120 at M=1 over 8
    weight copies (200 MB, more than L2), then 3 rotations of a 2048 x 5120 prompt at block
    256."""
    import torch
    import q38
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(6060)
    N, K = 17408, 5120
    mods = []
    for _ in range(8):
        w, s, b = _ternary_weight(torch, dev, g, N, K, 128, torch.float16)
        signs = torch.where(torch.rand(K, generator=g, device=dev) < 0.5, -1.0, 1.0)
        mods.append(q38.HadamardQuantizedLinear(q38.QuantizedLinear(w, s, b, None, 128, 2), signs, 1024))
    x = torch.randn((1, K), generator=g, device=dev).to(torch.bfloat16)
    for i in range(12):
        y = mods[i % 8](x)
    xp = torch.randn((2048, K), generator=g, device=dev).to(torch.bfloat16)
    for _ in range(3):
        r = q38.hadamard_rotate(xp, None, 256)
    torch.cuda.synchronize()
    q38.check_device()
    print(json.dumps({"profile_bonsai": {"N": N, "K": K, "projections": 12, "rotations_2048": 3,
                                         "weight_bytes": N * K // 4 + N * (K // 128) * 4,
                                         "mean_abs_y": float(y.float().abs().mean()),
                                         "mean_abs_r": float(r.float().abs().mean())}}))


def run_profile_embedding(args):
    """Small fixed workload for ncu captures of the embedding lookups: 4096 ids from a 248,320 x
    5120 4-bit g64 table (bf16 rows out, 42 MB), then the same ids from a 2-bit g128 f16 table
    rotated back at block 1024 (the Bonsai 2 embedding); 3 calls each."""
    import torch
    import q38
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7070)
    rows, K = 248320, 5120
    c4 = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows, K // 8), dtype=torch.int32, device=dev, generator=g)
    s4 = (torch.rand((rows, K // GROUP), device=dev, generator=g) * 0.01).to(torch.bfloat16)
    ids = torch.randint(0, rows, (4096,), device=dev, generator=g, dtype=torch.int32)
    for _ in range(3):
        e4 = q38.quantized_embedding(ids, c4, s4, -s4, GROUP, 4)
    del c4, s4
    w2, s2, b2 = _ternary_weight(torch, dev, g, rows, K, 128, torch.float16)
    signs = torch.where(torch.rand(K, generator=g, device=dev) < 0.5, -1.0, 1.0)
    for _ in range(3):
        e2 = q38.hadamard_quantized_embedding(ids, w2, s2, b2, signs, 1024, 128, 2)
    torch.cuda.synchronize()
    q38.check_device()
    print(json.dumps({"profile_embedding": {"ids": 4096, "K": K, "out_bytes": 4096 * K * 2,
                                            "row_bytes_4bit": K // 2 + (K // GROUP) * 4,
                                            "row_bytes_2bit_pack": K // 4 + (K // 128) * 4,
                                            "mean_abs": [float(e4.float().abs().mean()), float(e2.float().abs().mean())]}}))


def run_profile_moe(args):
    """One MoE layer (Flash-Next shapes) at T = --profile-t tokens, 2 calls, for ncu."""
    import torch
    import q38
    dev = torch.device("cuda", 0)
    blk, g = build_moe(torch, q38, dev)
    x = torch.randn((args.profile_t, MOE["H"]), generator=g, device=dev).to(torch.bfloat16)
    for _ in range(2):
        y = blk(x)
    torch.cuda.synchronize()
    q38.check_device()
    print(json.dumps({"profile_moe": {"T": args.profile_t, "calls": 2, "mean_abs_y": float(y.float().abs().mean())}}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile-case", action="store_true")
    ap.add_argument("--profile-bits", type=int, default=4)
    ap.add_argument("--profile-m", type=int, default=1)
    ap.add_argument("--profile-prefill", action="store_true")
    ap.add_argument("--profile-moe", action="store_true")
    ap.add_argument("--profile-bonsai", action="store_true")
    ap.add_argument("--profile-embedding", action="store_true")
    ap.add_argument("--profile-t", type=int, default=4096)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip-moe", action="store_true")
    ap.add_argument("--skip-prefill", action="store_true")
    ap.add_argument("--quick", action="store_true", help="fewer replays in the MoE and prefill sections")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.profile_case:
        run_profile_case(args)
        return
    if args.profile_prefill:
        run_profile_prefill(args)
        return
    if args.profile_moe:
        run_profile_moe(args)
        return
    if args.profile_bonsai:
        run_profile_bonsai(args)
        return
    if args.profile_embedding:
        run_profile_embedding(args)
        return
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        line = run_ours(args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
