"""Fused SwiGLU, h = silu(gate) * up, between the gate/up and down grouped GEMMs.

Replaces the reference layer's `F.silu(gate) * up` (tests/test_moe.py:82): one kernel
forward (2 reads, 1 write) and one backward (3 reads, 2 writes) instead of five PyTorch
elementwise passes, with the same rounding sequence.
"""
from __future__ import annotations

import torch

from . import _lib

_NS = "moeb200"


@torch.library.custom_op(f"{_NS}::swiglu_fwd", mutates_args=())
def swiglu_fwd(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    _lib.require_cuda(gate, up)
    assert gate.shape == up.shape and gate.dtype == up.dtype
    gate, up = gate.contiguous(), up.contiguous()
    out = torch.empty_like(gate)
    with torch.cuda.device(gate.device):
        st = _lib.load().moe_swiglu_fwd(_lib.ptr(gate), _lib.ptr(up), _lib.ptr(out), gate.numel(),
                                        _lib.dtype_code(gate.dtype), _lib.stream_of(gate))
    _lib.check(st, "moe_swiglu_fwd")
    _lib.count_launches(1)
    return out


@swiglu_fwd.register_fake
def _(gate, up):
    return torch.empty_like(gate)


@torch.library.custom_op(f"{_NS}::swiglu_bwd", mutates_args=())
def swiglu_bwd(grad_out: torch.Tensor, gate: torch.Tensor,
               up: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _lib.require_cuda(grad_out, gate, up)
    grad_out = grad_out.to(gate.dtype).contiguous()
    gate, up = gate.contiguous(), up.contiguous()
    dg, du = torch.empty_like(gate), torch.empty_like(up)
    with torch.cuda.device(gate.device):
        st = _lib.load().moe_swiglu_bwd(_lib.ptr(grad_out), _lib.ptr(gate), _lib.ptr(up),
                                        _lib.ptr(dg), _lib.ptr(du), gate.numel(),
                                        _lib.dtype_code(gate.dtype), _lib.stream_of(gate))
    _lib.check(st, "moe_swiglu_bwd")
    _lib.count_launches(1)
    return dg, du


@swiglu_bwd.register_fake
def _(grad_out, gate, up):
    return torch.empty_like(gate), torch.empty_like(up)


class SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate, up):
        ctx.save_for_backward(gate, up)
        return torch.ops.moeb200.swiglu_fwd(gate, up)

    @staticmethod
    def backward(ctx, grad_out):
        gate, up = ctx.saved_tensors
        return torch.ops.moeb200.swiglu_bwd(grad_out, gate, up)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up (differentiable)."""
    return SwiGLU.apply(gate, up)
