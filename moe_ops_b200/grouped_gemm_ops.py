"""Grouped GEMM (forward, dgrad, wgrad) on the sm_100a tensor cores.

Drop-in for the reference's grouped GEMM API
(triton_gmm_ops/grouped_gemm_ops_sm90.py:199-241 and triton_gmm_ops/grouped_gemm_ops.py:75-226):

    grouped_gemm(A, B, offsets, trans_b=True) -> C        (differentiable)
    A:       [total_tokens, K]           (all experts stacked along rows)
    B:       [E, N, K] if trans_b else [E, K, N]
    offsets: int32 [E+1] (offsets[0] = 0, offsets[e+1] = end row of expert e) or [E] ends
    C:       [total_tokens, N]

Raw custom ops live in the ``moeb200`` namespace (``torch.ops.moeb200.gmm_fwd_raw`` ...);
the namespace differs from the reference's ``tg`` so both libraries can be loaded in one
process.  Every op calls libmoe_b200.so; there is no CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_NS = "moeb200"


def supports_tma(dtype: Optional[torch.dtype] = None) -> bool:
    """True when grouped_gemm runs on the TMA + tcgen05 tensor-core kernel.

    Mirrors the reference's gate (grouped_gemm_ops_sm90.py:19-25): half-precision dtypes on
    a GPU that has TMA.  This library targets sm_100a only.
    """
    if dtype is not None and dtype not in (torch.float16, torch.bfloat16):
        return False
    return torch.cuda.is_available() and torch.cuda.get_device_capability()[0] >= 10


def _norm_offsets(offsets: torch.Tensor, E: int) -> torch.Tensor:
    if offsets.numel() not in (E, E + 1):
        raise ValueError(f"offsets must have E ({E}) or E+1 entries, got {offsets.numel()}")
    if offsets.dtype != torch.int32:
        offsets = offsets.to(torch.int32)
    return offsets.contiguous()


def _gmm_call(fn_name: str, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor,
              offsets: torch.Tensor, m_total: int, n: int, k: int, E: int, trans_b: bool) -> None:
    _lib.require_cuda(x, w, out, offsets)
    lib = _lib.load()
    timing = _lib.gemm_timing
    with torch.cuda.device(x.device):
        if timing is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        st = getattr(lib, fn_name)(
            _lib.ptr(x), _lib.ptr(w), _lib.ptr(out), _lib.ptr(offsets), offsets.numel(),
            m_total, n, k, E, int(bool(trans_b)), _lib.dtype_code(x.dtype), _lib.stream_of(x))
        if timing is not None:
            ev1.record()
            es = x.element_size()
            w_bytes, mk, mn = E * n * k * es, m_total * k * es, m_total * n * es
            rd, wr = {"moe_gmm_fwd": (w_bytes + mk, mn), "moe_gmm_dgrad": (w_bytes + mn, mk),
                      "moe_gmm_wgrad": (mk + mn, w_bytes)}[fn_name]
            timing.append((fn_name, ev0, ev1, 2.0 * m_total * n * k, rd, wr))
    _lib.check(st, fn_name)
    _lib.count_launches(1)


@torch.library.custom_op(f"{_NS}::gmm_fwd_raw", mutates_args=())
def gmm_fwd_raw(A: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor,
                trans_b: bool = True) -> torch.Tensor:
    """C = A . B[e]^T (trans_b) or A . B[e] per expert row range."""
    assert A.dtype == B.dtype, "A and B must share the same dtype"
    A = A.contiguous()
    B = B.contiguous()
    total, K = A.shape
    E = B.shape[0]
    N = B.shape[1] if trans_b else B.shape[2]
    assert (B.shape[2] if trans_b else B.shape[1]) == K, "B's contraction dim must match A"
    offsets = _norm_offsets(offsets, E)
    C = torch.empty((total, N), device=A.device, dtype=A.dtype)
    _gmm_call("moe_gmm_fwd", A, B, C, offsets, total, N, K, E, trans_b)
    return C


@gmm_fwd_raw.register_fake
def _(A, B, offsets, trans_b=True):
    N = B.shape[1] if trans_b else B.shape[2]
    return torch.empty((A.shape[0], N), device=A.device, dtype=A.dtype)


@torch.library.custom_op(f"{_NS}::gmm_dgrad_raw", mutates_args=())
def gmm_dgrad_raw(grad_output: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor,
                  trans_b: bool = True) -> torch.Tensor:
    """grad_A = grad_C . B[e] (trans_b) or grad_C . B[e]^T, reading B in place.

    The reference builds a transposed contiguous copy of B for this
    (grouped_gemm_ops_sm90.py:229); the tcgen05 kernel reads B through an MN-major
    shared-memory descriptor instead.
    """
    assert grad_output.dtype == B.dtype, "grad_output and B must share the same dtype"
    grad_output = grad_output.contiguous()
    B = B.contiguous()
    total, N = grad_output.shape
    E = B.shape[0]
    K = B.shape[2] if trans_b else B.shape[1]
    offsets = _norm_offsets(offsets, E)
    grad_A = torch.empty((total, K), device=grad_output.device, dtype=grad_output.dtype)
    _gmm_call("moe_gmm_dgrad", grad_output, B, grad_A, offsets, total, N, K, E, trans_b)
    return grad_A


@gmm_dgrad_raw.register_fake
def _(grad_output, B, offsets, trans_b=True):
    K = B.shape[2] if trans_b else B.shape[1]
    return torch.empty((grad_output.shape[0], K), device=grad_output.device, dtype=grad_output.dtype)


@torch.library.custom_op(f"{_NS}::gmm_bwd_B_raw", mutates_args=())
def gmm_bwd_B_raw(A: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor,
                  grad_output: torch.Tensor, trans_b: bool = True) -> torch.Tensor:
    """grad_B[e] = grad_C_e^T . A_e ([E, N, K], trans_b) or A_e^T . grad_C_e ([E, K, N]).

    Same signature as the reference's tg::gmm_bwd_B_raw (grouped_gemm_ops.py:174-192),
    which supports trans_b=True only; both layouts are supported here.  Experts without
    rows get zeros.
    """
    A = A.contiguous()
    grad_output = grad_output.contiguous()
    E = B.shape[0]
    total, K = A.shape
    N = B.shape[1] if trans_b else B.shape[2]
    offsets = _norm_offsets(offsets, E)
    shape = (E, N, K) if trans_b else (E, K, N)
    grad_B = torch.empty(shape, device=A.device, dtype=A.dtype)
    _gmm_call("moe_gmm_wgrad", A, grad_output, grad_B, offsets, total, N, K, E, trans_b)
    return grad_B


@gmm_bwd_B_raw.register_fake
def _(A, B, offsets, grad_output, trans_b=True):
    E = B.shape[0]
    K = A.shape[1]
    N = B.shape[1] if trans_b else B.shape[2]
    shape = (E, N, K) if trans_b else (E, K, N)
    return torch.empty(shape, device=A.device, dtype=A.dtype)


class GroupedGEMMAutograd(torch.autograd.Function):
    """Autograd wrapper; same contract as GroupedGEMMAutogradSM90
    (grouped_gemm_ops_sm90.py:213-236)."""

    @staticmethod
    def forward(ctx, A, B, offsets, trans_b=True):
        ctx.save_for_backward(A, B, offsets)
        ctx.trans_b = trans_b
        return torch.ops.moeb200.gmm_fwd_raw(A, B, offsets, trans_b=trans_b)

    @staticmethod
    def backward(ctx, grad_output):
        A, B, offsets = ctx.saved_tensors
        grad_A = grad_B = None
        if ctx.needs_input_grad[0]:
            grad_A = torch.ops.moeb200.gmm_dgrad_raw(grad_output, B, offsets, trans_b=ctx.trans_b)
        if ctx.needs_input_grad[1]:
            grad_B = torch.ops.moeb200.gmm_bwd_B_raw(A, B, offsets, grad_output, ctx.trans_b)
        return grad_A, grad_B, None, None


def grouped_gemm(A, B, offsets, trans_b: bool = True):
    """Differentiable grouped GEMM on the sm_100a tensor cores."""
    return GroupedGEMMAutograd.apply(A, B, offsets, trans_b)
