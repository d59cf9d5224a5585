"""SwiGLU MoE layer assembled from the library's ops (single GPU).

Same structure as the reference's example layer SingleGpuMoE (tests/test_moe.py:49-87):

    logits  = x @ w_router^T                          (torch GEMM, [T, E])
    w, idx  = fused_topk_softmax(logits, K)
    perm, row_id_map, offsets = permute(x, idx, E=E)
    h       = silu(grouped_gemm(perm, w_gate, offsets)) * grouped_gemm(perm, w_up, offsets)
    down    = grouped_gemm(h, w_down, offsets)        [T*K, d]
              (grouped_swiglu_mlp: gate/up + SwiGLU in one launch; in the backward the down
              projection's dgrad carries the SwiGLU backward in its epilogue)
    out     = unpermute(down, row_id_map, w, T, K)

Weights: w_router [E, d], w_gate / w_up [E, H, d], w_down [E, d, H] (trans_b=True layout).
"""
from __future__ import annotations

import torch

from .fused_topk_softmax_ops import fused_topk_softmax
from .gate_up_ops import grouped_swiglu_mlp
from .fused_permute_ops import gathered_path_ok, grouped_swiglu_mlp_gathered, permute_index
from .permute_ops import permute, permute_with_capacity
from .unpermute_ops import unpermute


def moe_layer_forward(x: torch.Tensor, w_router: torch.Tensor, w_gate: torch.Tensor,
                      w_up: torch.Tensor, w_down: torch.Tensor, top_k: int,
                      fp32_routing: bool = False,
                      router_bias: torch.Tensor | None = None,
                      capacity: int = 0, fused_permute: bool = False) -> torch.Tensor:
    """capacity > 0: each expert takes at most that many slots (its first in token order);
    a dropped slot adds nothing to its token's output (permute_with_capacity).
    fused_permute: the expert GEMMs read their rows from x through the permutation (TMA
    gather4) instead of from a permuted copy (fused_permute_ops); same results bit for bit."""
    E = w_gate.shape[0]
    num_tokens = x.shape[0]
    logits = x @ w_router.t()
    if router_bias is not None:
        logits = logits + router_bias
    weights, indices = fused_topk_softmax(logits, top_k, fp32_routing=fp32_routing)
    if fused_permute and capacity <= 0 and gathered_path_ok(x, w_gate.shape[1]):
        row_id_map, offsets, row_src = permute_index(indices, E)
        down = grouped_swiglu_mlp_gathered(x.contiguous(), row_src, row_id_map, w_gate, w_up,
                                           w_down, offsets, num_tokens, top_k)
        return unpermute(down, row_id_map, weights, num_tokens, top_k)
    if capacity > 0:
        permuted, row_id_map, offsets = permute_with_capacity(x, indices, E, capacity)
    else:
        permuted, row_id_map, offsets = permute(x, indices, E=E)
    down = grouped_swiglu_mlp(permuted, w_gate, w_up, w_down, offsets, trans_b=True)
    return unpermute(down, row_id_map, weights, num_tokens, top_k)


class MoELayer(torch.nn.Module):
    """Single-GPU SwiGLU MoE layer (parameters as in the reference's SingleGpuMoE)."""

    def __init__(self, d_model: int, num_experts: int, top_k: int, hidden: int,
                 fp32_routing: bool = False, device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.num_experts = num_experts
        self.top_k = top_k
        self.fp32_routing = fp32_routing
        self.w_router = torch.nn.Parameter(torch.empty(num_experts, d_model, **kw))
        self.w_gate = torch.nn.Parameter(torch.empty(num_experts, hidden, d_model, **kw))
        self.w_up = torch.nn.Parameter(torch.empty(num_experts, hidden, d_model, **kw))
        self.w_down = torch.nn.Parameter(torch.empty(num_experts, d_model, hidden, **kw))
        self.router_bias = None  # optional fixed per-expert logit bias [E]
        # > 0: expert capacity = ceil(capacity_factor * T * K / E) slots (token dropping)
        self.capacity_factor = 0.0
        # True: the expert GEMMs gather their rows from x (no permuted copy is written)
        self.fused_permute = False

    @torch.no_grad()
    def init_normal(self, std: float = 0.02, generator=None) -> "MoELayer":
        for p in self.parameters():
            p.normal_(0.0, std, generator=generator)
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        cap = 0
        if self.capacity_factor > 0:
            cap = -(-int(self.capacity_factor * x.shape[0] * self.top_k) // self.num_experts)
        return moe_layer_forward(x, self.w_router, self.w_gate, self.w_up, self.w_down,
                                 self.top_k, self.fp32_routing, self.router_bias, cap,
                                 self.fused_permute)


def layer_gemm_flops(num_tokens: int, top_k: int, d_model: int, hidden: int,
                     backward: bool = True) -> float:
    """Grouped-GEMM FLOPs of one layer step: 3 GEMMs forward (+ 6 backward)."""
    per_gemm = 2.0 * num_tokens * top_k * d_model * hidden
    return per_gemm * (9 if backward else 3)
