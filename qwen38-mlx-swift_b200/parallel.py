"""Multi-GPU layouts of the quantized products: one process per GPU, torch.distributed
(NCCL over NVLink on B200; gloo on CPU for the host-logic tests) for the exchanges, the
compute on libq38.

* TensorParallelMLP -- the dense MLP block of the 27B model (gate/up column-sharded, down
  row-sharded, one all-reduce of the partial outputs), the layout of the tensor-parallel
  prefill configuration.
* ExpertParallelMoE -- the routed experts of the Flash-Next sparse MoE layer
  (FlashNext/Qwen4ExpSparseMoE.swift:275-294) split contiguously over the ranks: each rank
  routes its own tokens and sends each token's activation row once to every rank that owns
  one of its experts (all-to-all), with the rank-local expert ids and router scores of its
  slots; the receiving rank runs SwitchGLU over its experts only (other slots marked -1),
  which gives the token's partial score-weighted sum; the partial rows return (all-to-all)
  and the home rank adds them in rank order.  With a fixed `capacity` (tokens per rank per
  call, the same on every rank) each rank sends `capacity` rows to every rank (token t at
  row t of each destination's block, unused rows marked empty), so the exchange sizes are
  known in advance: no count exchange, no host synchronisation, and the layer can be
  captured in a CUDA graph.  The result is bit-identical to the exact-size exchange.

The compute goes through an `ops` object (DeviceOps = libq38 on the GPU); tests substitute
CPU restatements to check the exchange bookkeeping without a GPU.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class DeviceOps:
    """libq38 kernels."""

    def __init__(self):
        import q38
        self.q = q38

    def qmm(self, x, c, s, b, group, bits):
        return self.q.quantized_matmul(x, c, s, b, True, group, bits)

    def silu_mul(self, g, u):
        return self.q.silu_mul(g, u)

    def route(self, x, wr, k, normalize=True):
        return self.q.moe_route(x, wr, k, normalize)

    def ep_plan(self, idx, epr, world):
        return self.q.moe_ep_plan(idx, epr, world)

    def ep_pack(self, x, idx, sc, rowpos, epr, rows_total):
        return self.q.moe_ep_pack(x, idx, sc, rowpos, epr, rows_total)

    def ep_unpack(self, packed, H, k):
        return self.q.split_ep_packed(packed, H, k)

    def partial_experts(self, rows, local_idx, scores, weights, group, bits):
        return self.q.switch_glu(rows, local_idx, scores, *weights, group, bits)

    def ep_reduce(self, partial, rowpos):
        return self.q.moe_ep_reduce(partial, rowpos)


def _rank_world(group=None):
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def shard_rows(c, s, b, rank, world):
    """Output-row (column-parallel) shard of a packed weight [N, ...]."""
    N = c.shape[0]
    if N % world:
        raise ValueError(f"{N} rows do not split over {world} ranks")
    n = N // world
    sl = slice(rank * n, (rank + 1) * n)
    return c[sl].contiguous(), s[sl].contiguous(), None if b is None else b[sl].contiguous()


def shard_k(c, s, b, rank, world, bits, group=64):
    """Reduction-dimension (row-parallel) shard of a packed weight [N, K*bits/32]: each rank
    keeps K/world columns, which must be whole groups and whole 32-bit words."""
    G = s.shape[-1]
    K = G * group
    if K % world or (K // world) % group or ((K // world) * bits) % 32:
        raise ValueError(f"K={K} does not split into whole groups and words over {world} ranks")
    kp = K // world
    wsl = slice(rank * kp * bits // 32, (rank + 1) * kp * bits // 32)
    gsl = slice(rank * kp // group, (rank + 1) * kp // group)
    return c[:, wsl].contiguous(), s[:, gsl].contiguous(), None if b is None else b[:, gsl].contiguous()


class TensorParallelMLP:
    """y = down(silu(gate(x)) * up(x)) with gate/up split by output rows and down by its
    reduction dimension; the partial outputs are summed by an all-reduce."""

    def __init__(self, gate, up, down, group_size=64, bits=4, ops=None, process_group=None,
                 reduce_dtype=None):
        self.ops = ops or DeviceOps()
        self.pg = process_group
        self.rank, self.world = _rank_world(process_group)
        self.group, self.bits = group_size, bits
        self.gate = shard_rows(*gate, self.rank, self.world)
        self.up = shard_rows(*up, self.rank, self.world)
        self.down = shard_k(*down, self.rank, self.world, bits, group_size)
        self.reduce_dtype = reduce_dtype

    def __call__(self, x):
        o = self.ops
        g = o.qmm(x, *self.gate, self.group, self.bits)
        u = o.qmm(x, *self.up, self.group, self.bits)
        h = o.silu_mul(g, u)
        y = o.qmm(h, *self.down, self.group, self.bits)
        if self.world > 1:
            if self.reduce_dtype is not None and y.dtype != self.reduce_dtype:
                yr = y.to(self.reduce_dtype)
                dist.all_reduce(yr, group=self.pg)
                y = yr.to(y.dtype)
            else:
                dist.all_reduce(y, group=self.pg)
        return y


def _exchange(t, send, recv, pg):
    """All-to-all of the rows of t: send[r] rows go to rank r, recv[r] rows arrive from it.
    Rows travel as 32-bit words (bit-identical for any element type)."""
    flat = t.reshape(t.shape[0], -1)
    if flat.element_size() != 4:
        flat = flat.contiguous().view(torch.int32)
    out = flat.new_empty((sum(recv),) + tuple(flat.shape[1:]))
    dist.all_to_all_single(out, flat.contiguous(), output_split_sizes=recv, input_split_sizes=send, group=pg)
    if t.element_size() != 4:
        out = out.view(t.dtype)
    return out.reshape((sum(recv),) + tuple(t.shape[1:]))


class ExpertParallelMoE:
    """Routed experts of the sparse-MoE layer over expert-parallel ranks.

    `experts` are this rank's (codes, scales, biases) triples for gate, up and down of the
    experts [rank*E/world, (rank+1)*E/world); `router_weight` [E, H] is replicated."""

    def __init__(self, router_weight, experts, num_experts, top_k, group_size=64, bits=3, normalize=True,
                 ops=None, process_group=None, capacity=None):
        self.ops = ops or DeviceOps()
        self.pg = process_group
        self.rank, self.world = _rank_world(process_group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.wr, self.experts = router_weight, experts
        self.E, self.k, self.epr = num_experts, top_k, num_experts // self.world
        self.group, self.bits, self.normalize = group_size, bits, normalize
        if capacity is not None and capacity < 1:
            raise ValueError("capacity must be at least one token")
        self.capacity = capacity

    def __call__(self, x):
        o = self.ops
        k = self.k
        if self.capacity is not None and x.shape[0] > self.capacity:
            raise ValueError(f"{x.shape[0]} tokens exceed the exchange capacity {self.capacity}")
        idx, sc = o.route(x, self.wr, k, self.normalize)
        if self.world == 1:
            return o.partial_experts(x, idx, sc, self.experts, self.group, self.bits)
        if self.capacity is not None:
            return self._fixed_exchange(x, idx, sc)
        rowpos, counts = o.ep_plan(idx, self.epr, self.world)
        send_t = counts.to(torch.int64)
        recv_t = torch.empty_like(send_t)
        dist.all_to_all_single(recv_t, send_t, group=self.pg)
        send, recv = send_t.tolist(), recv_t.tolist()
        # one exchange moves each row with its slot metadata: [rows, H + 4k] bf16
        packed = o.ep_pack(x, idx, sc, rowpos, self.epr, sum(send))
        rrows, lidx, lsc = o.ep_unpack(_exchange(packed, send, recv, self.pg), x.shape[1], k)
        part = o.partial_experts(rrows, lidx, lsc, self.experts, self.group, self.bits)
        back = _exchange(part, recv, send, self.pg)
        return o.ep_reduce(back, rowpos)

    def _fixed_exchange(self, x, idx, sc):
        """The exchange of q38_ep_switch_glu: every rank's `capacity` rows (padding rows with
        empty slots) gathered with their global slot experts and scores, this rank's experts
        over all of them (other ranks' slots -1), and the partial outputs summed into each
        token's home rank (here an fp32 all-reduce of which this rank keeps its block, the
        reduce-scatter's result)."""
        o, k, W, C = self.ops, self.k, self.world, self.capacity
        T, H = x.shape
        xs = torch.zeros((C, H), dtype=x.dtype, device=x.device)
        xs[:T] = x
        ids = torch.full((C, k), -1, dtype=torch.int32, device=x.device)
        ids[:T] = idx.to(torch.int32)
        scs = torch.zeros((C, k), dtype=sc.dtype, device=x.device)
        scs[:T] = sc

        def gather(t):
            parts = [torch.empty_like(t) for _ in range(W)]
            dist.all_gather(parts, t, group=self.pg)
            return torch.cat(parts)
        rows, gidx, gsc = gather(xs), gather(ids), gather(scs)
        mine = (gidx >= 0) & (gidx // self.epr == self.rank)
        local = torch.where(mine, gidx - self.rank * self.epr, torch.full_like(gidx, -1)).contiguous()
        part = o.partial_experts(rows, local, gsc, self.experts, self.group, self.bits).float()
        dist.all_reduce(part, group=self.pg)
        return part[self.rank * C:self.rank * C + T].to(x.dtype)
