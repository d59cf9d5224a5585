"""Gate and up projections of a SwiGLU expert layer, fused with the SwiGLU.

The reference's example layer runs two grouped GEMMs and a PyTorch SwiGLU
(tests/test_moe.py:80-82):

    gate = grouped_gemm(permuted, w_gate, offsets)
    up   = grouped_gemm(permuted, w_up, offsets)
    h    = F.silu(gate) * up

``grouped_gemm_swiglu(permuted, w_gate, w_up, offsets)`` returns the same ``h`` from one
tensor-core launch: each tile accumulates 128 gate and 128 up columns of the same rows, and
its epilogue writes gate, up (kept for the backward) and h.  The three outputs equal the
unfused sequence bit for bit (same accumulation order, same rounding steps).  The backward
is the unfused one: SwiGLU backward, two dgrad GEMMs summed, two wgrad GEMMs.
"""
from __future__ import annotations

import torch

from . import _lib
from . import swiglu_ops  # noqa: F401  (registers moeb200::swiglu_bwd)
from .grouped_gemm_ops import _norm_offsets, gmm_bwd_B_raw, gmm_dgrad_raw

_NS = "moeb200"


@torch.library.custom_op(f"{_NS}::gmm_gate_up_fwd_raw", mutates_args=())
def gmm_gate_up_fwd_raw(A: torch.Tensor, B_gate: torch.Tensor, B_up: torch.Tensor,
                        offsets: torch.Tensor,
                        trans_b: bool = True) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(gate, up, h): gate = A . B_gate[e]^T, up = A . B_up[e]^T (trans_b; else A . B[e]),
    h = silu(gate) * up, per expert row range."""
    assert A.dtype == B_gate.dtype == B_up.dtype, "A and the weights must share one dtype"
    assert B_gate.shape == B_up.shape, "gate and up weights must have the same shape"
    _lib.require_cuda(A, B_gate, B_up, offsets)
    A, B_gate, B_up = A.contiguous(), B_gate.contiguous(), B_up.contiguous()
    total, K = A.shape
    E = B_gate.shape[0]
    N = B_gate.shape[1] if trans_b else B_gate.shape[2]
    assert (B_gate.shape[2] if trans_b else B_gate.shape[1]) == K, "weights' contraction dim must match A"
    offsets = _norm_offsets(offsets, E)
    gate = torch.empty((total, N), device=A.device, dtype=A.dtype)
    up = torch.empty_like(gate)
    h = torch.empty_like(gate)
    lib = _lib.load()
    timing = _lib.gemm_timing
    with torch.cuda.device(A.device):
        if timing is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        st = lib.moe_gmm_gate_up_fwd(
            _lib.ptr(A), _lib.ptr(B_gate), _lib.ptr(B_up), _lib.ptr(gate), _lib.ptr(up),
            _lib.ptr(h), _lib.ptr(offsets), offsets.numel(), total, N, K, E, int(bool(trans_b)),
            _lib.dtype_code(A.dtype), _lib.stream_of(A))
        if timing is not None:
            ev1.record()
            es = A.element_size()
            timing.append(("moe_gmm_gate_up_fwd", ev0, ev1, 4.0 * total * N * K,
                           2 * E * N * K * es + total * K * es, 3 * total * N * es))
    _lib.check(st, "moe_gmm_gate_up_fwd")
    _lib.count_launches(1)
    return gate, up, h


@gmm_gate_up_fwd_raw.register_fake
def _(A, B_gate, B_up, offsets, trans_b=True):
    N = B_gate.shape[1] if trans_b else B_gate.shape[2]
    shape = (A.shape[0], N)
    return (A.new_empty(shape), A.new_empty(shape), A.new_empty(shape))


class GroupedGateUpSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, B_gate, B_up, offsets, trans_b):
        gate, up, h = torch.ops.moeb200.gmm_gate_up_fwd_raw(A, B_gate, B_up, offsets, trans_b)
        ctx.save_for_backward(A, B_gate, B_up, offsets, gate, up)
        ctx.trans_b = trans_b
        return h

    @staticmethod
    def backward(ctx, grad_h):
        A, B_gate, B_up, offsets, gate, up = ctx.saved_tensors
        trans_b = ctx.trans_b
        dgate, dup = torch.ops.moeb200.swiglu_bwd(grad_h, gate, up)
        grad_A = grad_g = grad_u = None
        if ctx.needs_input_grad[0]:
            grad_A = gmm_dgrad_raw(dgate, B_gate, offsets, trans_b)
            grad_A += gmm_dgrad_raw(dup, B_up, offsets, trans_b)
        if ctx.needs_input_grad[1]:
            grad_g = gmm_bwd_B_raw(A, B_gate, offsets, dgate, trans_b)
        if ctx.needs_input_grad[2]:
            grad_u = gmm_bwd_B_raw(A, B_up, offsets, dup, trans_b)
        return grad_A, grad_g, grad_u, None, None


def grouped_gemm_swiglu(A: torch.Tensor, B_gate: torch.Tensor, B_up: torch.Tensor,
                        offsets: torch.Tensor, trans_b: bool = True) -> torch.Tensor:
    """silu(grouped_gemm(A, B_gate)) * grouped_gemm(A, B_up), differentiable, one forward
    launch.  Shapes as in ``grouped_gemm``; B_gate and B_up have the same shape."""
    return GroupedGateUpSwiGLU.apply(A, B_gate, B_up, offsets, trans_b)


__all__ = ["grouped_gemm_swiglu", "gmm_gate_up_fwd_raw"]
