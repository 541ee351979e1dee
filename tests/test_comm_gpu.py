"""GPU tests of the multi-GPU entry points of the C ABI (q38_comm_*, q38_tp_mlp,
q38_ep_switch_glu), NCCL inside libq38.

* One rank (world 1, any GPU count): the tensor-parallel MLP equals the single-device MLP
  within 2e-2 * RMS plus one bf16 step, and the expert-parallel SwitchGLU equals
  q38_switch_glu bit for bit (the exchange to itself moves bytes unchanged; rows past the
  tokens carry only empty slots), the large capacities through the pipelined chunks.
* A rank whose peer never joins: init gives up with Q38_ERR_COMM after its timeout, the
  communicator aborted, no GPU work involved.
* Two GPUs (skipped with one): the id goes from rank 0 to rank 1 through a host queue;
  tensor parallel within 2e-2 * RMS plus one bf16 step of the unsharded MLP (the bf16
  all-reduce adds one rounding), expert parallel within the same bar of the single-GPU
  layer.  Both run with NCCL_NVLS_ENABLE=0.
"""
import os
import time

import numpy as np
import pytest
import torch

import oracle as O
from test_moe_gpu import dev_i32, make_experts, route_inputs
from test_qmm_gpu import dev_bf16, host_bf16

pytestmark = pytest.mark.gpu


def excess_over_step(y, ref):
    y, ref = y.float(), ref.float()
    rms = float((ref ** 2).mean().sqrt())
    step = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(2.0 ** -126))) - 7)
    return float(((y - ref).abs() - step).max()) / rms


def mlp_weights(q38, seed, D, F, bits=4):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ws = []
    for (n, k) in ((F, D), (F, D), (D, F)):
        c, s, b = q38.quantize(torch.randn((n, k), generator=g, device="cuda") * 0.02, 64, bits,
                               scales_dtype=torch.bfloat16)
        ws.append((c.view(torch.int32), s, b))
    return ws


def test_single_rank_tp_mlp_and_ep_switch_glu(q38):
    comm = q38.Communicator(q38.comm_unique_id(), 1, 0, timeout_ms=30000)
    try:
        D, F = 1024, 2048
        ws = mlp_weights(q38, 9600, D, F)
        x = dev_bf16(O.normal_bf16(9601, (300, D)))
        y = q38.tp_mlp(comm, x, *ws, 64, 4, chunks=3)
        full = q38.quantized_matmul(q38.quantized_gate_up(x, ws[0], ws[1], 64, 4), *ws[2], True, 64, 4)
        assert excess_over_step(y, full) <= 2e-2
        E, I, H, k, bits = 16, 512, 1024, 4, 3
        dev, _ = make_experts(q38, 9602, E, I, H, bits)
        # the large capacities also through 2 and 4 pipelined chunks of the exchange
        for T, cap, pieces in ((5, 5, 0), (5, 9, 0), (40, 64, 0), (600, 1024, 2), (2048, 2048, 4)):
            xe = dev_bf16(O.normal_bf16(9603 + T, (T, H)))
            idx, sc = route_inputs(T, E, k, 9604 + T)
            q38.set_ep_chunks(pieces)
            try:
                out = q38.ep_switch_glu(comm, xe, dev_i32(idx), dev_bf16(sc), *dev, E, cap, 64, bits)
            finally:
                q38.set_ep_chunks(0)
            ref = q38.switch_glu(xe, dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
            torch.cuda.synchronize()
            assert torch.equal(out, ref), (T, cap, pieces)
        q38.check_device()
    finally:
        comm.destroy()


def test_comm_init_gives_up_when_a_rank_never_joins(q38):
    uid = q38.comm_unique_id()
    t0 = time.time()
    with pytest.raises(q38.Q38Error) as e:
        q38.Communicator(uid, 2, 0, timeout_ms=3000)  # rank 1 never comes
    assert e.value.status == 6
    assert time.time() - t0 < 60
    # the device is still usable
    x = torch.ones(8, device="cuda")
    assert float(x.sum()) == 8.0


def _worker(rank, world, q_id, q_out):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(root, "qwen38-mlx-swift_b200"), os.path.join(root, "oracle"), os.path.join(root, "tests")):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    import q38
    if rank == 0:
        uid = q38.comm_unique_id()
        for _ in range(world - 1):
            q_id.put(uid)
    else:
        uid = q_id.get(timeout=120)
    comm = q38.Communicator(uid, world, rank, rank, timeout_ms=60000)
    try:
        from test_moe_gpu import make_experts as mk, route_inputs as ri
        # tensor parallel at the dense-27B MLP's width (D 5120, F 17408): this rank's shards
        # of the same full weights on every rank
        D, F = 5120, 17408
        ws = mlp_weights(q38, 9700, D, F)
        Fl = F // world
        gate = tuple(t[rank * Fl:(rank + 1) * Fl].contiguous() for t in ws[0])
        up = tuple(t[rank * Fl:(rank + 1) * Fl].contiguous() for t in ws[1])
        kw = Fl * 4 // 32
        down = (ws[2][0][:, rank * kw:(rank + 1) * kw].contiguous(), ws[2][1][:, rank * Fl // 64:(rank + 1) * Fl // 64].contiguous(),
                ws[2][2][:, rank * Fl // 64:(rank + 1) * Fl // 64].contiguous())
        x = dev_bf16(O.normal_bf16(9701, (384, D)))
        y = q38.tp_mlp(comm, x, gate, up, down, 64, 4, chunks=3)
        y0 = q38.tp_mlp(comm, x, gate, up, down, 64, 4)  # the library's piece count
        assert torch.equal(y, y0)
        full = q38.quantized_matmul(q38.quantized_gate_up(x, ws[0], ws[1], 64, 4), *ws[2], True, 64, 4)
        tp_err = excess_over_step(y, full)
        # expert parallel
        E, I, H, k, bits = 32, 512, 2048, 10, 3
        dev, _ = mk(q38, 9702, E, I, H, bits)
        epr = E // world
        mine = [tuple(t[rank * epr:(rank + 1) * epr].contiguous() for t in trip) for trip in dev]
        errs = []
        for T, cap, pieces in ((1, 1, 0), (8, 8, 0), (100 + 16 * rank, 160, 0), (1500 + 16 * rank, 2048, 4),
                               (1500 + 16 * rank, 2048, 0)):
            xe = dev_bf16(O.normal_bf16(9703 + T + rank, (T, H)))
            idx, sc = ri(T, E, k, 9704 + T + rank)
            q38.set_ep_chunks(pieces)
            out = q38.ep_switch_glu(comm, xe, dev_i32(idx), dev_bf16(sc), *mine, E, cap, 64, bits)
            q38.set_ep_chunks(0)
            ref = q38.switch_glu(xe, dev_i32(idx), dev_bf16(sc), *dev, 64, bits)
            errs.append(excess_over_step(out, ref))
        torch.cuda.synchronize()
        q_out.put((rank, tp_err, max(errs)))
    finally:
        comm.destroy()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_tp_mlp_and_ep_switch_glu_through_the_c_abi(q38):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, q_id, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q_out.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for (rank, tp_err, ep_err) in res:
        assert tp_err <= 2e-2, (rank, tp_err)
        assert ep_err <= 2e-2, (rank, ep_err)
