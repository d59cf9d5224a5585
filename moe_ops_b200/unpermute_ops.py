"""Unpermute (weighted gather-reduce back to token order) and its backward.

Drop-in for the reference's unpermute API (triton_gmm_ops/unpermute_ops.py:58-208):

    unpermute(input, row_id_map, prob, num_tokens, num_topK, max_tokens=-1)
    unpermute_forward(...) / unpermute_backward(grad_out, input_fwd, row_id_map, prob,
                                                num_tokens, num_topK) -> (act_grad, prob_grad)

out[t] = sum_k prob[t,k] * input[row_id_map[k*T+t]] with fp32 accumulation in k order.
``max_tokens`` larger than ``num_tokens`` yields zero rows past ``num_tokens``; the
reference kernel indexes row_id_map with max_tokens in that case
(unpermute_ops.py:65-67), which only agrees with this when max_tokens == num_tokens.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_NS = "moeb200"


def _unpermute_call(input: torch.Tensor, row_id_map: torch.Tensor, prob: Optional[torch.Tensor],
                    num_tokens: int, topK: int, max_tokens: int = -1) -> torch.Tensor:
    _lib.require_cuda(input, row_id_map, prob)
    input = input.contiguous()
    row_id_map = row_id_map.to(torch.int32).contiguous()
    if prob is not None:
        prob = prob.contiguous()
    if max_tokens == -1:
        max_tokens = num_tokens
    if max_tokens < num_tokens:
        raise ValueError("unpermute: max_tokens must be -1 or >= num_tokens")
    num_cols = input.shape[1]
    alloc = torch.zeros if max_tokens > num_tokens else torch.empty
    out = alloc(max_tokens, num_cols, device=input.device, dtype=input.dtype)
    with torch.cuda.device(input.device):
        st = _lib.load().moe_unpermute_fwd(
            _lib.ptr(input), _lib.dtype_code(input.dtype), _lib.ptr(row_id_map), _lib.ptr(prob),
            _lib.dtype_code(prob.dtype) if prob is not None else 0, num_tokens, topK, num_cols,
            _lib.ptr(out), _lib.stream_of(input))
    _lib.check(st, "moe_unpermute_fwd")
    _lib.count_launches(1)
    return out


@torch.library.custom_op(f"{_NS}::unpermute_forward", mutates_args=())
def unpermute_forward(input: torch.Tensor, row_id_map: torch.Tensor, prob: torch.Tensor,
                      num_tokens: int, num_topK: int, max_tokens: int = -1) -> torch.Tensor:
    return _unpermute_call(input, row_id_map, prob, num_tokens, num_topK, max_tokens)


@unpermute_forward.register_fake
def _(input, row_id_map, prob, num_tokens, num_topK, max_tokens=-1):
    if max_tokens == -1:
        max_tokens = num_tokens
    return torch.empty(max_tokens, input.shape[1], device=input.device, dtype=input.dtype)


@torch.library.custom_op(f"{_NS}::unpermute_backward", mutates_args=())
def unpermute_backward(grad_out: torch.Tensor, input_fwd: torch.Tensor, row_id_map: torch.Tensor,
                       prob: torch.Tensor, num_tokens: int,
                       num_topK: int) -> tuple[torch.Tensor, torch.Tensor]:
    """act_grad[i] = prob[t,k]*grad_out[t]; prob_grad[t,k] = <grad_out[t], input_fwd[i]>.

    One kernel for both outputs; rows of act_grad not named by row_id_map are left
    uninitialised, as in the reference (unpermute_ops.py:159).
    """
    _lib.require_cuda(grad_out, input_fwd, row_id_map, prob)
    grad_out = grad_out.to(input_fwd.dtype).contiguous()
    input_fwd = input_fwd.contiguous()
    row_id_map = row_id_map.to(torch.int32).contiguous()
    prob = prob.contiguous()
    num_cols = input_fwd.shape[1]
    act_grad = torch.empty_like(input_fwd)
    prob_grad = torch.empty(num_tokens, num_topK, device=prob.device, dtype=prob.dtype)
    with torch.cuda.device(input_fwd.device):
        st = _lib.load().moe_unpermute_bwd(
            _lib.ptr(grad_out), _lib.ptr(input_fwd), _lib.dtype_code(input_fwd.dtype),
            _lib.ptr(row_id_map), _lib.ptr(prob), _lib.dtype_code(prob.dtype), num_tokens,
            num_topK, num_cols, _lib.ptr(act_grad), _lib.ptr(prob_grad), _lib.stream_of(input_fwd))
    _lib.check(st, "moe_unpermute_bwd")
    _lib.count_launches(1)
    return act_grad, prob_grad


@unpermute_backward.register_fake
def _(grad_out, input_fwd, row_id_map, prob, num_tokens, num_topK):
    return (torch.empty_like(input_fwd),
            torch.empty(num_tokens, num_topK, device=prob.device, dtype=prob.dtype))


class UnpermuteAutograd(torch.autograd.Function):
    """Same contract as the reference's UnpermuteAutograd (unpermute_ops.py:182-198)."""

    @staticmethod
    def forward(ctx, input, row_id_map, prob, num_tokens, num_topK, max_tokens=-1):
        if max_tokens == -1:
            max_tokens = num_tokens
        ctx.save_for_backward(input, row_id_map, prob)
        ctx.num_tokens = num_tokens
        ctx.num_topK = num_topK
        return torch.ops.moeb200.unpermute_forward(input, row_id_map, prob, num_tokens, num_topK,
                                                  max_tokens)

    @staticmethod
    def backward(ctx, grad_out):
        input, row_id_map, prob = ctx.saved_tensors
        g = grad_out[: ctx.num_tokens]
        act_grad, prob_grad = torch.ops.moeb200.unpermute_backward(
            g, input, row_id_map, prob, ctx.num_tokens, ctx.num_topK)
        return act_grad, None, prob_grad, None, None, None


def unpermute(input, row_id_map, prob, num_tokens, num_topK, max_tokens: int = -1):
    """Differentiable unpermute: weighted sum of each token's K expert rows."""
    return UnpermuteAutograd.apply(input, row_id_map, prob, num_tokens, num_topK, max_tokens)
