"""GPU checks of the pieces the multi-GPU layouts use (silu_mul, dispatch pack, combine),
and -- with two or more GPUs -- the expert-parallel MoE and tensor-parallel MLP over NCCL
against the single-GPU layer.

Bars: pack and combine bit-exact with a restatement of the same arithmetic; silu_mul
within one bf16 step (exp differs in its last bits between libraries).  Expert parallel
(one row per token and destination rank, partial sums returned): bit-exact with the sum in
rank order of single-GPU SwitchGLU partials over each rank's experts (each pair's products
do not depend on which other pairs share its tile), and within 2e-2 * RMS plus one bf16
step of the single-GPU layer.  Tensor parallel on 2 GPUs: within 2e-2 * RMS plus one bf16 step of the
unsharded layer, error RMS <= 1e-2 * RMS.
"""
import os
import socket

import numpy as np
import pytest
import torch

import oracle as O
from test_moe_gpu import dev_i32, make_experts
from test_qmm_gpu import dev_bf16, host_bf16

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_silu_mul(q38):
    g = O.normal_bf16(9000, (3, 1000), 3.0)
    u = O.normal_bf16(9001, (3, 1000))
    h = host_bf16(q38.silu_mul(dev_bf16(g), dev_bf16(u)))
    gf, uf = O.bf16_to_f32(g).astype(np.float64), O.bf16_to_f32(u).astype(np.float64)
    ref = gf / (1 + np.exp(-gf)) * uf
    step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -126))) - 7)
    assert (np.abs(O.bf16_to_f32(h) - ref) <= step).all()


def test_dispatch_pack_and_combine(q38):
    T, k, H, E, epr = 37, 4, 256, 16, 4
    rng = np.random.default_rng(9100)
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    sc = O.f32_to_bf16(rng.uniform(0, 1, (T, k)).astype(np.float32))
    x = O.normal_bf16(9101, (T, H))
    dest = (idx // epr).reshape(-1)
    perm, off = O.sort_by_expert(dest, E // epr)
    rows, loc = q38.moe_dispatch_pack(dev_bf16(x), dev_i32(idx), dev_i32(perm), epr)
    np.testing.assert_array_equal(host_bf16(rows), x[perm // k])
    np.testing.assert_array_equal(loc.cpu().numpy(), idx.reshape(-1)[perm] % epr)
    y = O.normal_bf16(9102, (T * k, H))
    out = host_bf16(q38.moe_combine(dev_bf16(y), dev_i32(perm), dev_i32(idx), dev_bf16(sc), E))
    inv = np.empty(T * k, np.int64)
    inv[perm] = np.arange(T * k)
    yf, s = O.bf16_to_f32(y), O.bf16_to_f32(sc)
    ref = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in range(k):
            ref[t] += np.float32(s[t, j]) * yf[inv[t * k + j]]
    np.testing.assert_array_equal(out, O.f32_to_bf16(ref))


def rank_partials_sum(q38, x, idx, sc, dev, epr, world, bits=3):
    """bf16(sum over ranks, in order, of SwitchGLU over that rank's experts), fp32 sum."""
    acc = torch.zeros((x.shape[0], x.shape[1]), dtype=torch.float32, device=x.device)
    for r in range(world):
        lidx = torch.where(torch.div(idx, epr, rounding_mode="floor") == r, idx % epr,
                           torch.full_like(idx, -1)).to(torch.int32).contiguous()
        ws = [(c[r * epr:(r + 1) * epr].contiguous(), s[r * epr:(r + 1) * epr].contiguous(),
               b[r * epr:(r + 1) * epr].contiguous()) for (c, s, b) in dev]
        acc += q38.switch_glu(x, lidx, sc, *ws, 64, bits).float()
    return acc.to(torch.bfloat16)


def test_ep_exchange_kernels_single_gpu(q38):
    """plan -> pack -> per-rank partial SwitchGLU -> reduce, with the exchange done by
    slicing the packed buffer (world 4 simulated on one GPU)."""
    E, I, H, k, bits, world = 32, 512, 1024, 6, 3, 4
    epr = E // world
    dev, _ = make_experts(q38, 9600, E, I, H, bits)
    wr = dev_bf16(O.normal_bf16(9601, (E, H), 0.02))
    x = dev_bf16(O.normal_bf16(9602, (90, H)))
    idx, sc = q38.moe_route(x, wr, k)
    rowpos, counts = q38.moe_ep_plan(idx, epr, world)
    cnt = counts.tolist()
    rp = rowpos.cpu().numpy()
    # every token appears once per rank holding one of its experts, in token order
    ii = idx.cpu().numpy()
    base = 0
    for r in range(world):
        m = ((ii // epr) == r).any(axis=1)
        assert cnt[r] == int(m.sum())
        np.testing.assert_array_equal(rp[m, r], base + np.arange(cnt[r]))
        assert (rp[~m, r] == -1).all()
        base += cnt[r]
    packed = q38.moe_ep_pack(x, idx, sc, rowpos, epr, sum(cnt))
    parts = []
    off = 0
    for r in range(world):
        rr, lidx, lsc = q38.split_ep_packed(packed[off:off + cnt[r]], H, k)
        ws = [(c[r * epr:(r + 1) * epr].contiguous(), s[r * epr:(r + 1) * epr].contiguous(),
               b[r * epr:(r + 1) * epr].contiguous()) for (c, s, b) in dev]
        parts.append(q38.switch_glu(rr, lidx, lsc, *ws, 64, bits))
        off += cnt[r]
    out = q38.moe_ep_reduce(torch.cat(parts), rowpos)
    assert torch.equal(out, rank_partials_sum(q38, x, idx, sc, dev, epr, world))
    q38.check_device()


def free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "qwen38-mlx-swift_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch.distributed as dist
    import q38
    from parallel import ExpertParallelMoE, TensorParallelMLP
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from test_moe_gpu import make_experts as mk
        E, I, H, k, bits = 32, 512, 2048, 10, 3
        dev, _ = mk(q38, 9200, E, I, H, bits)  # same seed on every rank: identical full stacks
        wr = dev_bf16(O.normal_bf16(9201, (E, H), 0.02))
        epr = E // world
        mine = [(c[rank * epr:(rank + 1) * epr].contiguous(), s[rank * epr:(rank + 1) * epr].contiguous(),
                 b[rank * epr:(rank + 1) * epr].contiguous()) for (c, s, b) in dev]
        x = dev_bf16(O.normal_bf16(9300 + rank, (100 + 16 * rank, H)))
        ep = ExpertParallelMoE(wr, mine, E, k, 64, bits)
        out = ep(x)
        idx, sc = q38.moe_route(x, wr, k)
        ep_ok = bool(torch.equal(out, rank_partials_sum(q38, x, idx, sc, dev, epr, world)))
        # fixed-capacity exchange: 128 rows per destination (this rank has 100 + 16 * rank)
        fixed = ExpertParallelMoE(wr, mine, E, k, 64, bits, capacity=128)
        ep_ok = ep_ok and bool(torch.equal(fixed(x), out))
        full = q38.switch_glu(x, idx, sc, *dev, 64, bits).float()
        rms0 = float((full ** 2).mean().sqrt())
        step0 = torch.exp2(torch.floor(torch.log2(full.abs().clamp_min(2.0 ** -126))) - 7)
        ep_ok = ep_ok and float(((out.float() - full).abs() - step0).max()) <= 2e-2 * rms0
        # tensor-parallel MLP, 4-bit
        D, F = 1024, 2048
        g = torch.Generator(device="cuda").manual_seed(9400)
        ws = []
        for (n, kk) in ((F, D), (F, D), (D, F)):
            c, s, b = q38.quantize(torch.randn((n, kk), generator=g, device="cuda") * 0.02, 64, 4,
                                   scales_dtype=torch.bfloat16)
            ws.append((c.view(torch.int32), s, b))
        xt = torch.randn((300, D), generator=g, device="cuda").to(torch.bfloat16)
        tp = TensorParallelMLP(*ws, 64, 4, reduce_dtype=torch.float32)
        y = tp(xt).float()
        full = q38.quantized_matmul(q38.silu_mul(q38.quantized_matmul(xt, *ws[0], True, 64, 4),
                                                 q38.quantized_matmul(xt, *ws[1], True, 64, 4)),
                                    *ws[2], True, 64, 4).float()
        rms = float((full ** 2).mean().sqrt())
        step = torch.exp2(torch.floor(torch.log2(full.abs().clamp_min(2.0 ** -126))) - 7)
        excess = float(((y - full).abs() - step).max()) / rms
        erms = float(((y - full) ** 2).mean().sqrt()) / rms
        q.put((rank, ep_ok, excess, erms))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_expert_and_tensor_parallel(q38):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for (rank, ep_ok, excess, erms) in res:
        assert ep_ok, f"rank {rank}: expert-parallel output differs from the single-GPU layer"
        assert excess <= 2e-2 and erms <= 1e-2, (rank, excess, erms)


def test_expert_parallel_single_rank_equals_switch_glu(q38):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "qwen38-mlx-swift_b200"))
    from parallel import ExpertParallelMoE
    E, I, H, k, bits = 16, 512, 1024, 4, 3
    dev, _ = make_experts(q38, 9500, E, I, H, bits)
    wr = dev_bf16(O.normal_bf16(9501, (E, H), 0.02))
    x = dev_bf16(O.normal_bf16(9502, (70, H)))
    out = ExpertParallelMoE(wr, dev, E, k, 64, bits)(x)
    idx, sc = q38.moe_route(x, wr, k)
    assert torch.equal(out, q38.switch_glu(x, idx, sc, *dev, 64, bits))
