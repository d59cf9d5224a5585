"""Expert parallelism (EP) for the SwiGLU MoE layer: the NCCL transport, and the layer
class that can also run the NVLink peer-memory transport of ep_peer.py.

The reference has no distributed code (tests/test_moe.py:1-9: "no distributed comms");
this is the B200 extension its benchmark configs 4-5 ask for.  Rank r of W owns experts
[r*E/W, (r+1)*E/W).  One layer step on each rank, with its own tokens:

  1. router + fused top-k softmax (router weight replicated);
  2. permute by *global* expert: the permuted rows are grouped by destination rank, so the
     permuted buffer is the all-to-all send buffer (no extra copy);
  3. exchange per-(rank, local expert) row counts (one all_to_all of W*E/W int32) and read
     the W send / W receive sizes on the host (NCCL needs split sizes);
  4. all_to_all of rows (differentiable; backward is the reverse exchange);
  5. regroup the received rows (source-rank-major) to local-expert-major with the same
     counting-sort permute (K=1), giving the local grouped-GEMM offsets;
  6. the SwiGLU expert MLP on the local experts (gate/up + SwiGLU in one launch, then the
     down GEMM);
  7. undo the regroup (permute_backward, an exact gather), all_to_all back;
  8. unpermute weighted by the routing probabilities.

Autograd runs through every step; wgrad stays local.  No collective other than the two
all-to-alls (and the count exchange) is used; no tensor-core load reads another GPU's
memory.

The arithmetic on the token path goes through an `ops` object.  The default is this
library's CUDA ops; the CPU tests plug in a restatement (gloo ranks cannot run CUDA
kernels) to check the index bookkeeping and the exchange.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist
import torch.nn.functional as F


@dataclass
class EPOps:
    """The per-rank operators the EP layer composes (all autograd-capable)."""
    topk: Callable          # (logits, K) -> (weights, indices int32)
    permute: Callable       # (x, indices [T,K], E) -> (permuted, row_id_map, offsets[E+1])
    unpermute: Callable     # (rows, row_id_map, prob | None (K=1 gather), T, K) -> out [T, d]
    grouped_gemm: Callable  # (A, B [E,N,K], offsets) -> C
    swiglu: Callable = None  # (gate, up) -> silu(gate) * up; None = PyTorch elementwise
    # (A, W_gate, W_up, W_down, offsets) -> the SwiGLU expert MLP in fused launches; None =
    # grouped_gemm / swiglu above
    expert_mlp: Callable = None


def cuda_ops() -> EPOps:
    from . import fused_topk_softmax, grouped_gemm, permute, unpermute
    from .permute_ops import gather_rows
    from .gate_up_ops import grouped_swiglu_mlp
    from .swiglu_ops import swiglu

    def _unpermute(rows, rid, prob, T, K):
        if prob is None:
            assert K == 1
            return gather_rows(rows, rid)
        return unpermute(rows, rid, prob, T, K)

    return EPOps(topk=lambda lg, K: fused_topk_softmax(lg, K),
                 permute=lambda x, idx, E: permute(x, idx, E=E),
                 unpermute=_unpermute,
                 grouped_gemm=lambda a, b, off: grouped_gemm(a, b, off, True),
                 swiglu=swiglu,
                 expert_mlp=lambda a, wg, wu, wd, off: grouped_swiglu_mlp(a, wg, wu, wd, off, True))


# ------------------------------------------------------------------ index bookkeeping


def send_counts(offsets: torch.Tensor, world: int) -> torch.Tensor:
    """Rows of the globally permuted buffer per (destination rank, local expert):
    int32 [W * E_local] from offsets [E+1]."""
    counts = (offsets[1:] - offsets[:-1]).to(torch.int32)
    assert counts.numel() % world == 0
    return counts


def local_expert_ids(recv_counts: torch.Tensor, world: int, n_recv: int) -> torch.Tensor:
    """Local expert id of every received row.  Received rows arrive source-rank-major and,
    within a source, grouped by local expert: recv_counts is [W, E_local]."""
    el = recv_counts.numel() // world
    ids = torch.arange(el, device=recv_counts.device, dtype=torch.int32).repeat(world)
    return torch.repeat_interleave(ids, recv_counts.reshape(-1).to(torch.int64),
                                   output_size=n_recv)


def exchange_counts(counts: torch.Tensor, world: int, group=None):
    """all_to_all of the [W*E_local] counts; returns (recv_counts [W*E_local] on the
    device, send_sizes [W], recv_sizes [W] as host lists)."""
    el = counts.numel() // world
    recv = torch.empty_like(counts)
    dist.all_to_all_single(recv, counts, group=group)
    both = torch.stack([counts.reshape(world, el).sum(1), recv.reshape(world, el).sum(1)]).cpu()
    return recv, both[0].tolist(), both[1].tolist()


class _AllToAll(torch.autograd.Function):
    """Row all_to_all with split sizes; backward is the reverse exchange."""

    @staticmethod
    def forward(ctx, x, send_sizes, recv_sizes, group):
        ctx.send_sizes, ctx.recv_sizes, ctx.group = send_sizes, recv_sizes, group
        out = x.new_empty(sum(recv_sizes), x.shape[1])
        dist.all_to_all_single(out, x.contiguous(), recv_sizes, send_sizes, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty(sum(ctx.send_sizes), g.shape[1])
        dist.all_to_all_single(out, g.contiguous(), ctx.send_sizes, ctx.recv_sizes, group=ctx.group)
        return out, None, None, None


def all_to_all_rows(x, send_sizes, recv_sizes, group=None):
    return _AllToAll.apply(x, send_sizes, recv_sizes, group)


# ------------------------------------------------------------------ the layer


def ep_moe_forward(x: torch.Tensor, w_router: torch.Tensor, w_gate_local: torch.Tensor,
                   w_up_local: torch.Tensor, w_down_local: torch.Tensor, top_k: int,
                   num_experts: int, ops: EPOps | None = None, group=None,
                   fp32_routing: bool = False,
                   router_bias: torch.Tensor | None = None,
                   stats: dict | None = None) -> torch.Tensor:
    """One expert-parallel SwiGLU MoE layer on this rank's tokens x [T, d].

    w_router [E, d] is replicated; w_*_local hold this rank's E/W experts
    ([E/W, H, d], [E/W, H, d], [E/W, d, H])."""
    ops = ops or cuda_ops()
    world = dist.get_world_size(group)
    el = w_gate_local.shape[0]
    assert el * world == num_experts, "num_experts must equal world_size * local experts"
    T = x.shape[0]
    logits = x @ w_router.t()
    if router_bias is not None:
        logits = logits + router_bias
    if fp32_routing:
        logits = logits.float()
    weights, indices = ops.topk(logits, top_k)
    permuted, rid, offsets = ops.permute(x, indices, num_experts)
    counts = send_counts(offsets, world)
    recv_counts, send_sizes, recv_sizes = exchange_counts(counts, world, group)
    n_recv = sum(recv_sizes)
    if stats is not None:
        stats["local_rows"] = n_recv
    recv = all_to_all_rows(permuted[: T * top_k], send_sizes, recv_sizes, group)
    ids = local_expert_ids(recv_counts, world, n_recv)
    grouped, rid2, off2 = ops.permute(recv, ids.unsqueeze(1), el)
    if ops.expert_mlp is not None:
        down = ops.expert_mlp(grouped, w_gate_local, w_up_local, w_down_local, off2)
    else:
        gate = ops.grouped_gemm(grouped, w_gate_local, off2)
        up = ops.grouped_gemm(grouped, w_up_local, off2)
        h = ops.swiglu(gate, up) if ops.swiglu is not None else F.silu(gate) * up
        down = ops.grouped_gemm(h, w_down_local, off2)
    back = ops.unpermute(down, rid2, None, n_recv, 1)
    home = all_to_all_rows(back, recv_sizes, send_sizes, group)
    return ops.unpermute(home, rid, weights, T, top_k)


class EPMoELayer(torch.nn.Module):
    """Expert-parallel SwiGLU MoE layer: this rank's share of the experts plus the
    replicated router (parameter shapes as in moe_layer.MoELayer, experts E / world)."""

    def __init__(self, d_model: int, num_experts: int, top_k: int, hidden: int, group=None,
                 fp32_routing: bool = False, device=None, dtype=None):
        super().__init__()
        world = dist.get_world_size(group)
        assert num_experts % world == 0, "num_experts must be a multiple of the world size"
        el = num_experts // world
        kw = dict(device=device, dtype=dtype)
        self.num_experts, self.top_k, self.group, self.fp32_routing = num_experts, top_k, group, fp32_routing
        self.w_router = torch.nn.Parameter(torch.empty(num_experts, d_model, **kw))
        self.w_gate = torch.nn.Parameter(torch.empty(el, hidden, d_model, **kw))
        self.w_up = torch.nn.Parameter(torch.empty(el, hidden, d_model, **kw))
        self.w_down = torch.nn.Parameter(torch.empty(el, d_model, hidden, **kw))
        self.router_bias = None  # optional fixed per-expert logit bias [E]
        # > 0: pipeline the expert segment over this many chunks of local experts so the
        # all-to-alls overlap the GEMMs; 0: the plain sequence (ep_moe_forward).  Measured on
        # cfg4: 2 chunks win at 2 ranks (16.26 vs 16.49 ms) but lose at 8 (15.45 vs 14.2 ms,
        # the per-chunk GEMMs get too small), so the default is the plain sequence.
        self.chunks = 0
        # "nccl": dispatch / combine as NCCL all-to-alls (the tested default at every world
        # size); "nvlink": straight over peer memory (ep_peer.py), no host sync in the step.
        # The peer path needs the same token count on every rank.
        self.transport = "nccl"
        self._peer = None
        self._peer_tokens = 0
        # Largest token count any rank passes (sizes the peer buffers); None: the largest T
        # of the first call, agreed on by all ranks.
        self.max_tokens = None
        self._last_local_rows = 0

    def _forward_peer(self, x):
        from .ep_peer import NVLinkTransport, capacity_rows, peer_experts
        from .fused_topk_softmax_ops import fused_topk_softmax

        world = dist.get_world_size(self.group)
        T = x.shape[0]
        if self._peer is None:
            # Collective on every rank: the buffers are sized for the largest token count of
            # any rank (max_tokens if set, else the largest T of this first call), so a slot
            # can never land past the end of a peer's receive buffer, whatever the ranks'
            # token counts are later (each at most that size).
            if self.max_tokens is not None:
                t_max = int(self.max_tokens)
            else:
                t = torch.tensor([T], dtype=torch.int64, device=x.device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
                t_max = int(t.item())
            self._peer = NVLinkTransport(self.group, capacity_rows(t_max, self.top_k, world),
                                         x.shape[1], x.dtype, x.device)
            self._peer_tokens = t_max
        elif not torch.cuda.is_current_stream_capturing():
            self._peer.check_health()
        if T > self._peer_tokens or x.shape[1] != self._peer.cols or x.dtype != self._peer.dtype:
            # Rebuilding here would be a collective that only this rank enters.
            raise RuntimeError(
                f"EP peer transport was built for at most {self._peer_tokens} tokens of "
                f"{self._peer.cols} {self._peer.dtype} columns per rank; got {tuple(x.shape)} "
                f"{x.dtype}. Call close() on every rank (or set max_tokens) to rebuild it.")
        logits = x @ self.w_router.t()
        if self.router_bias is not None:
            logits = logits + self.router_bias
        if self.fp32_routing:
            logits = logits.float()
        weights, indices = fused_topk_softmax(logits, self.top_k)
        return peer_experts(x, weights, indices, self.w_gate, self.w_up, self.w_down, self._peer,
                            self.num_experts)

    def local_rows(self) -> int:
        """Rows this rank's experts computed on in the last forward (synchronises): the
        count the grouped GEMMs' FLOPs follow, whatever the buffers' capacity."""
        if self.transport == "nvlink" and self._peer is not None:
            return int(self._peer.last_local_rows.item())
        return int(self._last_local_rows)

    def health_ok(self) -> bool:
        """True unless a peer-memory barrier gave up (synchronises; NCCL path: True)."""
        return self._peer is None or self._peer.barrier_ok()

    def close(self):
        """Releases the peer-memory buffers (collective when they exist: every rank calls
        it).  Tensors viewing them must not be used afterwards."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def forward(self, x):
        if self.transport == "nvlink":
            return self._forward_peer(x)
        if self.chunks > 0:
            stats = {}
            out = ep_moe_forward_overlapped(x, self.w_router, self.w_gate, self.w_up, self.w_down,
                                            self.top_k, self.num_experts, group=self.group,
                                            fp32_routing=self.fp32_routing,
                                            router_bias=self.router_bias, chunks=self.chunks,
                                            stats=stats)
            self._last_local_rows = stats["local_rows"]
            return out
        stats = {}
        out = ep_moe_forward(x, self.w_router, self.w_gate, self.w_up, self.w_down, self.top_k,
                             self.num_experts, group=self.group, fp32_routing=self.fp32_routing,
                             router_bias=self.router_bias, stats=stats)
        self._last_local_rows = stats["local_rows"]
        return out


# ------------------------------------------------------------------ overlapped expert segment


def _chunk_bounds(el: int, chunks: int) -> list[tuple[int, int]]:
    """Local-expert ranges of the pipeline chunks (contiguous, as equal as possible)."""
    chunks = max(1, min(chunks, el))
    return [(c * el // chunks, (c + 1) * el // chunks) for c in range(chunks)]


def _segment_plan(send_cnt: list[list[int]], recv_cnt: list[list[int]], bounds):
    """Row slices of every chunk.  send_cnt[r][e]: rows this rank sends to rank r for
    rank r's local expert e (the permuted buffer holds, per destination rank, its experts'
    rows in expert order); recv_cnt[s][e]: rows rank s sends here for local expert e.
    Returns per chunk: (send slices [(start, len)] per destination, recv lengths per source,
    per-(source, expert) counts of the chunk)."""
    world = len(send_cnt)
    seg_start, acc = [], 0
    for r in range(world):
        seg_start.append(acc)
        acc += sum(send_cnt[r])
    plan = []
    for e0, e1 in bounds:
        sends = []
        for r in range(world):
            off = seg_start[r] + sum(send_cnt[r][:e0])
            sends.append((off, sum(send_cnt[r][e0:e1])))
        recvs = [sum(recv_cnt[s][e0:e1]) for s in range(world)]
        counts = [recv_cnt[s][e] for s in range(world) for e in range(e0, e1)]
        plan.append((sends, recvs, counts))
    return plan


def _a2a_slices(dst: torch.Tensor, dst_parts, src: torch.Tensor, src_parts, group):
    """Asynchronous all_to_all between row slices: src_parts[r] = (start, len) rows of src
    go to rank r, dst_parts[s] = (start, len) rows of dst come from rank s."""
    outs = [dst[a:a + n] for a, n in dst_parts]
    ins = [src[a:a + n] for a, n in src_parts]
    return dist.all_to_all(outs, ins, group=group, async_op=True)


class _OverlappedExperts(torch.autograd.Function):
    """dispatch -> regroup -> gate/up GEMMs -> SwiGLU -> down GEMM -> un-regroup -> combine,
    pipelined over chunks of local experts in forward and backward: while one chunk
    computes, the next chunk's dispatch (or the previous chunk's combine) is in flight on
    the process group's NCCL stream."""

    @staticmethod
    def forward(ctx, permuted, w_gate, w_up, w_down, plan, group):
        from .gate_up_ops import gmm_gate_up_fwd_raw
        from .grouped_gemm_ops import gmm_fwd_raw
        from .permute_ops import permute_backward, permute_countsort

        world = dist.get_world_size(group)
        bounds = plan["bounds"]
        recv_bufs, works = [], []
        for c, (sends, recvs, _) in enumerate(plan["chunks"]):
            buf = permuted.new_empty(sum(recvs), permuted.shape[1])
            dparts, a = [], 0
            for n in recvs:
                dparts.append((a, n))
                a += n
            works.append(_a2a_slices(buf, dparts, permuted, sends, group))
            recv_bufs.append((buf, dparts))
        home = torch.empty_like(permuted)
        saved, combines = [], []
        for c, (sends, recvs, counts) in enumerate(plan["chunks"]):
            e0, e1 = bounds[c]
            works[c].wait()
            buf, dparts = recv_bufs[c]
            n = buf.shape[0]
            cnt = torch.tensor(counts, dtype=torch.int32, device=buf.device)
            ids = local_expert_ids(cnt, world, n)
            grouped, rid2, off2 = permute_countsort(buf, ids.unsqueeze(1), 0, e1 - e0)
            gate, up, h = gmm_gate_up_fwd_raw(grouped, w_gate[e0:e1], w_up[e0:e1], off2, True)
            down = gmm_fwd_raw(h, w_down[e0:e1], off2, True)
            back = permute_backward(down, rid2, n, 1)
            combines.append(_a2a_slices(home, sends, back, dparts, group))
            saved.append((grouped, gate, up, h, rid2, off2, back))
        for w in combines:
            w.wait()
        ctx.plan, ctx.group, ctx.saved_chunks = plan, group, saved
        ctx.save_for_backward(w_gate, w_up, w_down)
        ctx.n_rows = permuted.shape[0]
        return home

    @staticmethod
    def backward(ctx, grad_home):
        from .gate_up_ops import gmm_dgrad_dual_raw, gmm_dgrad_swiglu_bwd_raw
        from .grouped_gemm_ops import _gmm_call
        from .permute_ops import permute_backward

        w_gate, w_up, w_down = ctx.saved_tensors
        plan, group = ctx.plan, ctx.group
        grad_home = grad_home.contiguous()
        g_gate, g_up, g_down = (torch.empty_like(w) for w in (w_gate, w_up, w_down))
        grad_perm = torch.empty(ctx.n_rows, grad_home.shape[1], device=grad_home.device,
                                dtype=grad_home.dtype)
        recvs, works = [], []
        for c, (sends, rc, _) in enumerate(plan["chunks"]):
            n = sum(rc)
            buf = grad_home.new_empty(n, grad_home.shape[1])
            dparts, a = [], 0
            for m in rc:
                dparts.append((a, m))
                a += m
            works.append(_a2a_slices(buf, dparts, grad_home, sends, group))
            recvs.append((buf, dparts))
        returns = []
        for c, (sends, rc, _) in enumerate(plan["chunks"]):
            e0, e1 = plan["bounds"][c]
            grouped, gate, up, h, rid2, off2, back = ctx.saved_chunks[c]
            works[c].wait()
            buf, dparts = recvs[c]
            n = buf.shape[0]
            el = e1 - e0
            g_down_rows = torch.ops.moeb200.scatter_rows(buf, rid2, n, 1)  # recv -> grouped order
            dgate, dup = gmm_dgrad_swiglu_bwd_raw(g_down_rows, w_down[e0:e1], gate, up, off2, True)
            _gmm_call("moe_gmm_wgrad", h, g_down_rows, g_down[e0:e1], off2, n, w_down.shape[1],
                      w_down.shape[2], el, True)
            dgrouped = gmm_dgrad_dual_raw(dgate, w_gate[e0:e1], dup, w_up[e0:e1], off2, True)
            _gmm_call("moe_gmm_wgrad", grouped, dgate, g_gate[e0:e1], off2, n, w_gate.shape[1],
                      w_gate.shape[2], el, True)
            _gmm_call("moe_gmm_wgrad", grouped, dup, g_up[e0:e1], off2, n, w_up.shape[1],
                      w_up.shape[2], el, True)
            drecv = permute_backward(dgrouped, rid2, n, 1)  # grouped -> recv order
            returns.append(_a2a_slices(grad_perm, sends, drecv, dparts, group))
            ctx.saved_chunks[c] = None
        for w in returns:
            w.wait()
        return grad_perm, g_gate, g_up, g_down, None, None


def ep_moe_forward_overlapped(x, w_router, w_gate_local, w_up_local, w_down_local, top_k,
                              num_experts, group=None, fp32_routing=False, router_bias=None,
                              chunks: int = 2, stats: dict | None = None):
    """ep_moe_forward with the dispatch / combine all-to-alls overlapped with the expert
    GEMMs (CUDA ops only)."""
    from . import fused_topk_softmax, permute, unpermute

    world = dist.get_world_size(group)
    el = w_gate_local.shape[0]
    assert el * world == num_experts, "num_experts must equal world_size * local experts"
    T = x.shape[0]
    logits = x @ w_router.t()
    if router_bias is not None:
        logits = logits + router_bias
    weights, indices = fused_topk_softmax(logits, top_k, fp32_routing=fp32_routing)
    permuted, rid, offsets = permute(x, indices, E=num_experts)
    counts = send_counts(offsets, world)
    recv = torch.empty_like(counts)
    dist.all_to_all_single(recv, counts, group=group)
    both = torch.stack([counts, recv]).cpu()
    send_cnt = both[0].reshape(world, el).tolist()
    recv_cnt = both[1].reshape(world, el).tolist()
    if stats is not None:
        stats["local_rows"] = sum(map(sum, recv_cnt))
    bounds = _chunk_bounds(el, chunks)
    plan = {"bounds": bounds, "chunks": _segment_plan(send_cnt, recv_cnt, bounds)}
    home = _OverlappedExperts.apply(permuted[: T * top_k], w_gate_local, w_up_local,
                                    w_down_local, plan, group)
    return unpermute(home, rid, weights, T, top_k)
