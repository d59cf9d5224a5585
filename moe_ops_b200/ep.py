"""Expert parallelism (EP) for the SwiGLU MoE layer over NCCL.

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
  6. gate / up grouped GEMMs, SwiGLU, down grouped GEMM on the local experts;
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


def cuda_ops() -> EPOps:
    from . import fused_topk_softmax, grouped_gemm, permute, unpermute
    from .permute_ops import gather_rows
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
                 swiglu=swiglu)


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
                   router_bias: torch.Tensor | None = None) -> torch.Tensor:
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
    recv = all_to_all_rows(permuted[: T * top_k], send_sizes, recv_sizes, group)
    ids = local_expert_ids(recv_counts, world, n_recv)
    grouped, rid2, off2 = ops.permute(recv, ids.unsqueeze(1), el)
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

    def forward(self, x):
        return ep_moe_forward(x, self.w_router, self.w_gate, self.w_up, self.w_down, self.top_k,
                              self.num_experts, group=self.group, fp32_routing=self.fp32_routing,
                              router_bias=self.router_bias)
