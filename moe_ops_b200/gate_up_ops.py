"""The SwiGLU expert MLP's fused launches: gate/up projections with the SwiGLU, and the
down projection's dgrad with the SwiGLU backward.

The reference's example layer runs two grouped GEMMs and a PyTorch SwiGLU
(tests/test_moe.py:80-82):

    gate = grouped_gemm(permuted, w_gate, offsets)
    up   = grouped_gemm(permuted, w_up, offsets)
    h    = F.silu(gate) * up

``grouped_gemm_swiglu(permuted, w_gate, w_up, offsets)`` returns the same ``h`` from one
tensor-core launch: each tile accumulates 128 gate and 128 up columns of the same rows, and
its epilogue writes gate, up (kept for the backward) and h.  The three outputs equal the
unfused sequence bit for bit (same accumulation order, same rounding steps).  Its backward:
SwiGLU backward, the two dgrad GEMMs as one two-segment launch into one accumulator
(``gmm_dgrad_dual_raw``: rounded once, so it differs from the unfused dgrad + dgrad + add by
at most the add's rounding), two wgrad GEMMs.

``grouped_swiglu_mlp(permuted, w_gate, w_up, w_down, offsets)`` is the whole expert MLP,
``grouped_gemm(h, w_down)`` on top of the above.  Its backward runs the down projection's
dgrad with the SwiGLU backward in the epilogue (``gmm_dgrad_swiglu_bwd_raw``): the gradient
of h is never written, and grad_gate / grad_up equal dgrad GEMM + SwiGLU backward bit for
bit.
"""
from __future__ import annotations

import torch

from . import _lib
from . import swiglu_ops  # noqa: F401  (registers moeb200::swiglu_bwd)
from .grouped_gemm_ops import _norm_offsets, gmm_bwd_B_raw, gmm_dgrad_raw, gmm_fwd_raw

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


@torch.library.custom_op(f"{_NS}::gmm_dgrad_swiglu_bwd_raw", mutates_args=())
def gmm_dgrad_swiglu_bwd_raw(grad_output: torch.Tensor, B: torch.Tensor, gate: torch.Tensor,
                             up: torch.Tensor, offsets: torch.Tensor,
                             trans_b: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """(grad_gate, grad_up) = swiglu_bwd(gmm_dgrad_raw(grad_output, B), gate, up) in one
    launch; gate / up are the forward's projections (the shape of the dgrad result)."""
    assert grad_output.dtype == B.dtype == gate.dtype == up.dtype, "operands must share one dtype"
    _lib.require_cuda(grad_output, B, gate, up, offsets)
    grad_output, B = grad_output.contiguous(), B.contiguous()
    gate, up = gate.contiguous(), up.contiguous()
    total, N = grad_output.shape
    E = B.shape[0]
    K = B.shape[2] if trans_b else B.shape[1]
    assert gate.shape == up.shape == (total, K), "gate / up must match the dgrad result"
    offsets = _norm_offsets(offsets, E)
    grad_gate = torch.empty_like(gate)
    grad_up = torch.empty_like(up)
    lib = _lib.load()
    timing = _lib.gemm_timing
    with torch.cuda.device(grad_output.device):
        if timing is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        st = lib.moe_gmm_dgrad_swiglu_bwd(
            _lib.ptr(grad_output), _lib.ptr(B), _lib.ptr(gate), _lib.ptr(up), _lib.ptr(grad_gate),
            _lib.ptr(grad_up), _lib.ptr(offsets), offsets.numel(), total, N, K, E,
            int(bool(trans_b)), _lib.dtype_code(grad_output.dtype), _lib.stream_of(grad_output))
        if timing is not None:
            ev1.record()
            es = grad_output.element_size()
            timing.append(("moe_gmm_dgrad_swiglu_bwd", ev0, ev1, 2.0 * total * N * K,
                           E * N * K * es + total * N * es + 2 * total * K * es,
                           2 * total * K * es))
    _lib.check(st, "moe_gmm_dgrad_swiglu_bwd")
    _lib.count_launches(1)
    return grad_gate, grad_up


@gmm_dgrad_swiglu_bwd_raw.register_fake
def _(grad_output, B, gate, up, offsets, trans_b=True):
    return torch.empty_like(gate), torch.empty_like(up)


def dgrad_dual_ok(g1: torch.Tensor, B1: torch.Tensor, g2: torch.Tensor, B2: torch.Tensor) -> bool:
    """True when moe_gmm_dgrad_dual takes these operands (its tensor-core conditions)."""
    ts = (g1, B1, g2, B2)
    return (g1.dtype in (torch.float16, torch.bfloat16)
            and all(t.dtype == g1.dtype and t.is_contiguous() and t.data_ptr() % 16 == 0 for t in ts)
            and g1.shape[1] % 8 == 0 and g2.shape[1] % 8 == 0 and B1.shape[0] <= 1024
            and B1.shape[1] % 8 == 0 and B1.shape[2] % 8 == 0)


def dgrad_dual_into(g1, B1, g2, B2, out, offsets, m_total: int, trans_b: bool) -> None:
    """out[:m_total] = g1 . op(B1[e]) + g2 . op(B2[e]) per expert row range, in one
    tensor-core launch (moe_gmm_dgrad_dual); the operands must pass dgrad_dual_ok."""
    _lib.require_cuda(g1, B1, g2, B2, out, offsets)
    E = B1.shape[0]
    k = B1.shape[2] if trans_b else B1.shape[1]
    n1, n2 = g1.shape[1], g2.shape[1]
    lib = _lib.load()
    timing = _lib.gemm_timing
    with torch.cuda.device(g1.device):
        if timing is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        st = lib.moe_gmm_dgrad_dual(
            _lib.ptr(g1), _lib.ptr(B1), _lib.ptr(g2), _lib.ptr(B2), _lib.ptr(out),
            _lib.ptr(offsets), offsets.numel(), m_total, n1, n2, k, E, int(bool(trans_b)),
            _lib.dtype_code(g1.dtype), _lib.stream_of(g1))
        if timing is not None:
            ev1.record()
            es = g1.element_size()
            timing.append(("moe_gmm_dgrad_dual", ev0, ev1, 2.0 * m_total * (n1 + n2) * k,
                           E * (n1 + n2) * k * es + m_total * (n1 + n2) * es, m_total * k * es))
    _lib.check(st, "moe_gmm_dgrad_dual")
    _lib.count_launches(1)


@torch.library.custom_op(f"{_NS}::gmm_dgrad_dual_raw", mutates_args=())
def gmm_dgrad_dual_raw(grad_1: torch.Tensor, B_1: torch.Tensor, grad_2: torch.Tensor,
                       B_2: torch.Tensor, offsets: torch.Tensor,
                       trans_b: bool = True) -> torch.Tensor:
    """grad_A = dgrad(grad_1, B_1) + dgrad(grad_2, B_2) with one rounding, one launch when
    the tensor-core path takes the operands, else two dgrad launches and an add."""
    grad_1, grad_2 = grad_1.contiguous(), grad_2.contiguous()
    B_1, B_2 = B_1.contiguous(), B_2.contiguous()
    E = B_1.shape[0]
    offsets = _norm_offsets(offsets, E)
    if not dgrad_dual_ok(grad_1, B_1, grad_2, B_2):
        out = gmm_dgrad_raw(grad_1, B_1, offsets, trans_b)
        out += gmm_dgrad_raw(grad_2, B_2, offsets, trans_b)
        return out
    k = B_1.shape[2] if trans_b else B_1.shape[1]
    out = torch.empty((grad_1.shape[0], k), device=grad_1.device, dtype=grad_1.dtype)
    dgrad_dual_into(grad_1, B_1, grad_2, B_2, out, offsets, grad_1.shape[0], trans_b)
    return out


@gmm_dgrad_dual_raw.register_fake
def _(grad_1, B_1, grad_2, B_2, offsets, trans_b=True):
    k = B_1.shape[2] if trans_b else B_1.shape[1]
    return torch.empty((grad_1.shape[0], k), device=grad_1.device, dtype=grad_1.dtype)


_SIDE = {}


def side_stream(device: torch.device):
    """A second stream per device for a backward GEMM that needs none of the others' outputs
    (the down projection's wgrad), so its tiles can fill the SMs the input-gradient GEMM's
    last wave of tiles leaves idle.  Opt-in (MOE_B200_BWD_STREAMS=1): on one GPU it measured
    no gain (cfg4: 16.29 vs 16.26 ms per step); it targets steps with only a few waves of
    tiles per GEMM (expert parallelism over many GPUs)."""
    import os

    if os.environ.get("MOE_B200_BWD_STREAMS", "0") != "1":
        return None
    key = torch.device(device).index
    if key not in _SIDE:
        _SIDE[key] = torch.cuda.Stream(device=device)
    return _SIDE[key]


def run_on_side(fn, device):
    """fn() on the side stream after the current stream's work so far; returns (result,
    join) where join() makes the current stream wait for it.  Without a side stream, fn()
    runs here."""
    side = side_stream(device)
    if side is None:
        out = fn()
        return out, (lambda: None)
    cur = torch.cuda.current_stream(device)
    side.wait_stream(cur)
    with torch.cuda.stream(side):
        out = fn()

    def join():
        cur.wait_stream(side)
        if out is not None:
            out.record_stream(cur)

    return out, join


def _gate_up_backward(A, B_gate, B_up, offsets, dgate, dup, trans_b, needs):
    grad_A = grad_g = grad_u = None
    if needs[0]:
        # dgrad of both projections into one accumulator: one launch, one rounding
        grad_A = gmm_dgrad_dual_raw(dgate, B_gate, dup, B_up, offsets, trans_b)
    if needs[1]:
        grad_g = gmm_bwd_B_raw(A, B_gate, offsets, dgate, trans_b)
    if needs[2]:
        grad_u = gmm_bwd_B_raw(A, B_up, offsets, dup, trans_b)
    return grad_A, grad_g, grad_u


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
        grads = _gate_up_backward(A, B_gate, B_up, offsets, dgate, dup, trans_b,
                                  ctx.needs_input_grad[:3])
        return (*grads, None, None)


def grouped_gemm_swiglu(A: torch.Tensor, B_gate: torch.Tensor, B_up: torch.Tensor,
                        offsets: torch.Tensor, trans_b: bool = True) -> torch.Tensor:
    """silu(grouped_gemm(A, B_gate)) * grouped_gemm(A, B_up), differentiable, one forward
    launch.  Shapes as in ``grouped_gemm``; B_gate and B_up have the same shape."""
    return GroupedGateUpSwiGLU.apply(A, B_gate, B_up, offsets, trans_b)


class GroupedSwiGLUMLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, B_gate, B_up, B_down, offsets, trans_b):
        gate, up, h = torch.ops.moeb200.gmm_gate_up_fwd_raw(A, B_gate, B_up, offsets, trans_b)
        out = gmm_fwd_raw(h, B_down, offsets, trans_b)
        ctx.save_for_backward(A, B_gate, B_up, B_down, offsets, gate, up, h)
        ctx.trans_b = trans_b
        return out

    @staticmethod
    def backward(ctx, grad_out):
        A, B_gate, B_up, B_down, offsets, gate, up, h = ctx.saved_tensors
        trans_b = ctx.trans_b
        grad_out = grad_out.contiguous()
        dgate, dup = gmm_dgrad_swiglu_bwd_raw(grad_out, B_down, gate, up, offsets, trans_b)
        grad_d, join = (run_on_side(lambda: gmm_bwd_B_raw(h, B_down, offsets, grad_out, trans_b),
                                    grad_out.device)
                        if ctx.needs_input_grad[3] else (None, lambda: None))
        grads = _gate_up_backward(A, B_gate, B_up, offsets, dgate, dup, trans_b,
                                  ctx.needs_input_grad[:3])
        join()
        return (*grads, grad_d, None, None)


def grouped_swiglu_mlp(A: torch.Tensor, B_gate: torch.Tensor, B_up: torch.Tensor,
                       B_down: torch.Tensor, offsets: torch.Tensor,
                       trans_b: bool = True) -> torch.Tensor:
    """grouped_gemm(silu(grouped_gemm(A, B_gate)) * grouped_gemm(A, B_up), B_down),
    differentiable: the SwiGLU expert MLP over grouped rows with both fused launches."""
    return GroupedSwiGLUMLP.apply(A, B_gate, B_up, B_down, offsets, trans_b)


__all__ = ["grouped_gemm_swiglu", "grouped_swiglu_mlp", "gmm_gate_up_fwd_raw",
           "gmm_dgrad_swiglu_bwd_raw", "gmm_dgrad_dual_raw"]
