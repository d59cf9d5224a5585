"""Fused top-k softmax router (forward + backward), one warp per token.

Drop-in for the reference's fused_topk_softmax
(triton_gmm_ops/fused_topk_softmax_ops.py:121-207).
"""
from __future__ import annotations

import torch

from . import _lib

_NS = "moeb200"


@torch.library.custom_op(f"{_NS}::fused_topk_softmax_fwd", mutates_args=())
def fused_topk_softmax_fwd(logits: torch.Tensor, K: int) -> tuple[torch.Tensor, torch.Tensor]:
    """weights [T, K] (logits dtype), indices [T, K] int32.

    Top-K by value (ties go to the lower expert index), softmax over the K values in fp32.
    """
    _lib.require_cuda(logits)
    logits = logits.contiguous()
    num_tokens, E = logits.shape
    weights = torch.empty((num_tokens, K), device=logits.device, dtype=logits.dtype)
    indices = torch.empty((num_tokens, K), device=logits.device, dtype=torch.int32)
    with torch.cuda.device(logits.device):
        st = _lib.load().moe_topk_softmax_fwd(
            _lib.ptr(logits), _lib.dtype_code(logits.dtype), num_tokens, E, K,
            _lib.ptr(weights), _lib.ptr(indices), _lib.stream_of(logits))
    _lib.check(st, "moe_topk_softmax_fwd")
    _lib.count_launches(1)
    return weights, indices


@fused_topk_softmax_fwd.register_fake
def _(logits, K):
    T = logits.shape[0]
    return (torch.empty((T, K), device=logits.device, dtype=logits.dtype),
            torch.empty((T, K), device=logits.device, dtype=torch.int32))


@torch.library.custom_op(f"{_NS}::fused_topk_softmax_bwd", mutates_args=())
def fused_topk_softmax_bwd(grad_weights: torch.Tensor, weights: torch.Tensor,
                           indices: torch.Tensor, num_tokens: int, E: int, K: int) -> torch.Tensor:
    """grad_logits [T, E] (weights dtype): w*(g - sum_k g*w) at the picked experts, else 0."""
    _lib.require_cuda(grad_weights, weights, indices)
    grad_weights = grad_weights.to(weights.dtype).contiguous()
    weights = weights.contiguous()
    indices = indices.to(torch.int32).contiguous()
    grad_logits = torch.empty((num_tokens, E), device=weights.device, dtype=weights.dtype)
    with torch.cuda.device(weights.device):
        st = _lib.load().moe_topk_softmax_bwd(
            _lib.ptr(grad_weights), _lib.ptr(weights), _lib.ptr(indices),
            _lib.dtype_code(weights.dtype), num_tokens, E, K, _lib.ptr(grad_logits),
            _lib.stream_of(weights))
    _lib.check(st, "moe_topk_softmax_bwd")
    _lib.count_launches(1)
    return grad_logits


@fused_topk_softmax_bwd.register_fake
def _(grad_weights, weights, indices, num_tokens, E, K):
    return torch.empty((num_tokens, E), device=weights.device, dtype=weights.dtype)


class FusedTopkSoftmaxFunction(torch.autograd.Function):
    """Same contract as the reference's FusedTopkSoftmaxFunction
    (fused_topk_softmax_ops.py:174-190)."""

    @staticmethod
    def forward(ctx, logits, K):
        weights, indices = torch.ops.moeb200.fused_topk_softmax_fwd(logits, K)
        ctx.save_for_backward(weights, indices)
        ctx.E = logits.shape[1]
        ctx.mark_non_differentiable(indices)
        return weights, indices

    @staticmethod
    def backward(ctx, grad_weights, grad_indices):
        weights, indices = ctx.saved_tensors
        num_tokens, K = weights.shape
        grad_logits = torch.ops.moeb200.fused_topk_softmax_bwd(
            grad_weights, weights, indices, num_tokens, ctx.E, K)
        return grad_logits, None


def fused_topk_softmax(logits: torch.Tensor, K: int,
                       fp32_routing: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused top-K softmax.

    Args:
        logits: [num_tokens, num_experts].
        K: number of experts per token.
        fp32_routing: compute (and return) the routing weights in float32.

    Returns:
        weights [num_tokens, K] and indices [num_tokens, K] (int32).
    """
    if fp32_routing and logits.dtype != torch.float32:
        logits = logits.float()
    return FusedTopkSoftmaxFunction.apply(logits, K)
