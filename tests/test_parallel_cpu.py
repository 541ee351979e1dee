"""Host logic of the multi-GPU layouts on CPU: two gloo ranks run ExpertParallelMoE and
TensorParallelMLP with the oracle standing in for the kernels.

* Expert parallel: the routed output of every rank's tokens must equal, bit for bit, the
  sum in rank order of the oracle SwitchGLU partial sums over each rank's experts (slots
  of other ranks marked -1) -- the plan, the packing of rows and slot metadata, the
  exchanges and the reduction reproduce that arithmetic exactly -- and match the
  single-process SwitchGLU within 2e-2 * RMS plus one bf16 step.
* Tensor parallel: the all-reduced output must match the unsharded oracle MLP within
  2e-2 * RMS plus one bf16 step of the output, with error RMS <= 1e-2 * RMS: every rank's
  partial product is rounded to bf16 before the sum, and partials can exceed the total.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O


def bf(t):  # torch bf16 (CPU) -> numpy uint16 bits
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def tb(a):  # numpy uint16 bits -> torch bf16 (CPU)
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


class OracleOps:
    """The oracle behind the kernel interface of parallel.DeviceOps (CPU tensors)."""

    def qmm(self, x, c, s, b, group, bits):
        return tb(O.qmm(bf(x), c.numpy().view(np.uint32), bf(s), None if b is None else bf(b), group, bits))

    def silu_mul(self, g, u):
        gf, uf = O.bf16_to_f32(bf(g)), O.bf16_to_f32(bf(u))
        return tb(O.f32_to_bf16((gf / (np.float32(1) + np.exp(-gf)) * uf).astype(np.float32)))

    def route(self, x, wr, k, normalize=True):
        idx, sc = O.moe_route(bf(x), bf(wr), k, normalize)
        return torch.from_numpy(idx), tb(sc)

    def ep_plan(self, idx, epr, world):
        i = idx.numpy()
        T = i.shape[0]
        rowpos = np.full((T, world), -1, np.int32)
        counts = np.zeros(world, np.int32)
        base = 0
        for r in range(world):
            m = ((i // epr) == r).any(axis=1)
            pos = np.cumsum(m) - 1
            rowpos[m, r] = base + pos[m]
            counts[r] = int(m.sum())
            base += counts[r]
        return torch.from_numpy(rowpos), torch.from_numpy(counts)

    def ep_pack(self, x, idx, sc, rowpos, epr, rows_total):
        i, rp = idx.numpy(), rowpos.numpy()
        T, k = i.shape
        rows = torch.zeros((rows_total, x.shape[1]), dtype=torch.bfloat16)
        meta = np.zeros((rows_total, 2 * k), np.int32)
        sbits = bf(sc).astype(np.int32)
        for t in range(T):
            for r in range(rp.shape[1]):
                row = rp[t, r]
                if row < 0:
                    continue
                rows[row] = x[t]
                meta[row, :k] = np.where(i[t] // epr == r, i[t] % epr, -1)
                meta[row, k:] = sbits[t]
        return torch.cat([rows, torch.from_numpy(meta).view(torch.bfloat16)], dim=1)

    def ep_unpack(self, packed, H, k):
        meta = packed[:, H:].contiguous().view(torch.int32)
        return packed[:, :H].contiguous(), meta[:, :k].contiguous(), meta[:, k:].to(torch.int16).view(torch.bfloat16)

    def partial_experts(self, rows, lidx, lsc, weights, group, bits):
        n = rows.shape[0]
        if n == 0:
            return rows.clone()
        w = [(c.numpy().view(np.uint32), bf(s), None if b is None else bf(b)) for (c, s, b) in weights]
        return tb(O.switch_glu(bf(rows), lidx.numpy(), bf(lsc), *w, group, bits))

    def ep_reduce(self, partial, rowpos):
        rp = rowpos.numpy()
        pf = O.bf16_to_f32(bf(partial))
        out = np.zeros((rp.shape[0], partial.shape[1]), np.float32)
        for t in range(rp.shape[0]):
            for r in range(rp.shape[1]):
                if rp[t, r] >= 0:
                    out[t] += pf[rp[t, r]]
        return tb(O.f32_to_bf16(out))


def free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


H, I, E, K_TOP, BITS = 256, 128, 8, 3, 3


def moe_weights():
    mk = lambda seed, shape: O.quantize(O.normal_f32(seed, shape, 0.05), 64, BITS)
    return mk(11, (E, I, H)), mk(12, (E, I, H)), mk(13, (E, H, I))


def ep_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "qwen38-mlx-swift_b200"))
    from parallel import ExpertParallelMoE
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gate, up, down = moe_weights()
        epr = E // world
        sl = slice(rank * epr, (rank + 1) * epr)
        mine = [(torch.from_numpy(c[sl].view(np.int32)), tb(s[sl]), tb(b[sl])) for (c, s, b) in (gate, up, down)]
        wr = O.normal_bf16(14, (E, H), 0.05)
        x = O.normal_bf16(100 + rank, (5 + rank, H))
        moe = ExpertParallelMoE(tb(wr), mine, E, K_TOP, 64, BITS, ops=OracleOps())
        out = bf(moe(tb(x)))
        idx, sc = O.moe_route(x, wr, K_TOP, True)
        acc = np.zeros((x.shape[0], H), np.float32)
        for r in range(world):
            lidx = np.where(idx // epr == r, idx % epr, -1).astype(np.int32)
            ws = [(c[r * epr:(r + 1) * epr], s[r * epr:(r + 1) * epr], b[r * epr:(r + 1) * epr]) for (c, s, b) in (gate, up, down)]
            acc += O.bf16_to_f32(O.switch_glu(x, lidx, sc, *ws, 64, BITS))
        exact = bool(np.array_equal(out, O.f32_to_bf16(acc)))
        # fixed-capacity exchange (8 rows per destination; this rank has 5 + rank tokens)
        fixed = ExpertParallelMoE(tb(wr), mine, E, K_TOP, 64, BITS, ops=OracleOps(), capacity=8)
        exact = exact and bool(np.array_equal(bf(fixed(tb(x))), out))
        try:
            ExpertParallelMoE(tb(wr), mine, E, K_TOP, 64, BITS, ops=OracleOps(), capacity=4)(tb(x))
            exact = False
        except ValueError:
            pass
        full = O.bf16_to_f32(O.switch_glu(x, idx, sc, gate, up, down, 64, BITS)).astype(np.float64)
        y = O.bf16_to_f32(out).astype(np.float64)
        rms = np.sqrt((full ** 2).mean())
        step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(full), 2.0 ** -126))) - 7)
        q.put((rank, exact, float((np.abs(y - full) - step).max() / rms)))
    finally:
        dist.destroy_process_group()


def tp_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "qwen38-mlx-swift_b200"))
    from parallel import TensorParallelMLP
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        D, F = 256, 512
        mk = lambda seed, shape: O.quantize(O.normal_f32(seed, shape, 0.05), 64, 4)
        gate, up, down = mk(21, (F, D)), mk(22, (F, D)), mk(23, (D, F))
        to_t = lambda w: (torch.from_numpy(w[0].view(np.int32)), tb(w[1]), tb(w[2]))
        x = O.normal_bf16(24, (7, D))
        mlp = TensorParallelMLP(to_t(gate), to_t(up), to_t(down), 64, 4, ops=OracleOps(), reduce_dtype=torch.float32)
        y = O.bf16_to_f32(bf(mlp(tb(x)))).astype(np.float64)
        ops = OracleOps()
        g, u = ops.qmm(tb(x), *to_t(gate), 64, 4), ops.qmm(tb(x), *to_t(up), 64, 4)
        ref = O.bf16_to_f32(bf(ops.qmm(ops.silu_mul(g, u), *to_t(down), 64, 4))).astype(np.float64)
        rms = np.sqrt((ref ** 2).mean())
        step = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -126))) - 7)
        q.put((rank, float((np.abs(y - ref) - step).max() / rms), float(np.sqrt(((y - ref) ** 2).mean()) / rms)))
    finally:
        dist.destroy_process_group()


def run2(fn):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=fn, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(res)


def test_expert_parallel_exchange_matches_single_process():
    res = run2(ep_worker)
    assert all(exact and err <= 2e-2 for (_, exact, err) in res), res


def test_tensor_parallel_mlp_matches_unsharded():
    res = run2(tp_worker)
    assert all(err <= 2e-2 and erms <= 1e-2 for (_, err, erms) in res), res


def test_shard_helpers_split_whole_groups_and_words():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "qwen38-mlx-swift_b200"))
    from parallel import shard_k, shard_rows
    c, s, b = O.quantize(O.normal_f32(31, (64, 17408), 0.02), 64, 4)
    ct, st, bt = torch.from_numpy(c.view(np.int32)), tb(s), tb(b)
    parts = [shard_k(ct, st, bt, r, 8, 4) for r in range(8)]
    assert all(p[0].shape == (64, 2176 * 4 // 32) and p[1].shape == (64, 34) for p in parts)
    assert np.array_equal(np.concatenate([p[0].numpy() for p in parts], axis=1), c.view(np.int32))
    rows = [shard_rows(ct, st, bt, r, 4) for r in range(4)]
    assert np.array_equal(np.concatenate([p[0].numpy() for p in rows], axis=0), c.view(np.int32))
    with pytest.raises(ValueError):
        shard_k(ct, st, bt, 0, 3, 4)


def absent_peer_worker(rank, world, port, q):
    """Rank 1 leaves without joining (scenario 'init') or right after joining, before the
    first collective (scenario 'collective'); rank 0 must get an error within its timeout."""
    import datetime
    import time
    scenario = os.environ["Q38_TEST_SCENARIO"]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == 1 and scenario == "init":
        q.put((rank, "left", 0.0))
        return
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        dist.barrier()  # one completed step: the ranks' connections exist
        if rank == 1:
            q.put((rank, "left", 0.0))
            q.close()
            q.join_thread()  # the message is out before the process ends
            os._exit(0)  # leaves between steps: nothing of it is in flight
        dist.all_reduce(torch.ones(4))
        q.put((rank, "completed", time.time() - t0))
    except Exception as e:  # the failure is reported, not hung on
        q.put((rank, type(e).__name__, time.time() - t0))


@pytest.mark.parametrize("scenario", ["init", "collective"])
def test_absent_peer_is_reported_within_the_timeout(scenario):
    os.environ["Q38_TEST_SCENARIO"] = scenario
    try:
        res = run2(absent_peer_worker)
    finally:
        del os.environ["Q38_TEST_SCENARIO"]
    (r0, what0, secs0), (r1, what1, _) = res
    assert r0 == 0 and what1 == "left"
    assert what0 not in ("completed",), res
    assert secs0 < 60, res
