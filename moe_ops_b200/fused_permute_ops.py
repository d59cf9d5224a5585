"""Permute fused into the expert GEMMs: the permuted copy of the tokens is never written.

The reference's experiment ``develop/experiment/fused_ops.py:31-107`` (and its weight
gradient kernel after it) reads the GEMM's A rows from the token-order input through a
row -> token map (``sorted_id_map``) instead of from a permuted buffer.  Here:

    row_id_map, offsets, row_src = permute_index(indices, E)      index pass only
    down = grouped_swiglu_mlp_gathered(x, row_src, row_id_map, w_gate, w_up, w_down,
                                       offsets, T, K)             [T*K, d], permuted order
    out  = unpermute(down, row_id_map, weights, T, K)

The gate/up GEMM fetches its A rows x[row_src[r]] with TMA gather4 (one-row boxes), and in
the backward the gate / up weight gradients fetch the same rows the same way; the input
gradient goes back to token order with permute_backward.  Every output and gradient equals
the layer over permute() + grouped_swiglu_mlp() bit for bit: the GEMMs see the same row
values in the same order and accumulate identically.
"""
from __future__ import annotations

import torch

from . import _lib
from .gate_up_ops import gmm_dgrad_dual_raw, gmm_dgrad_swiglu_bwd_raw
from .grouped_gemm_ops import _norm_offsets, gmm_bwd_B_raw, gmm_fwd_raw
from .permute_ops import permute_backward

_NS = "moeb200"


@torch.library.custom_op(f"{_NS}::permute_index", mutates_args=())
def permute_index(indices: torch.Tensor, E: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(row_id_map [T*K], offsets [E+1], row_src [T*K]) of the stable counting-sort permute,
    without copying rows; row_src[row] is the token whose slot lands in that row."""
    _lib.require_cuda(indices)
    if indices.dim() == 1:
        indices = indices.unsqueeze(1)
    T, K = indices.shape
    flat = indices.reshape(-1).to(torch.int32).contiguous()
    lib = _lib.load()
    dev = indices.device
    rid = torch.empty(T * K, dtype=torch.int32, device=dev)
    off = torch.empty(E + 1, dtype=torch.int32, device=dev)
    src = torch.empty(T * K, dtype=torch.int32, device=dev)
    ws_bytes = lib.moe_permute_workspace_bytes(T, K, E)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.moe_permute_index(_lib.ptr(flat), T, K, E, _lib.ptr(rid), _lib.ptr(off),
                                   _lib.ptr(src), _lib.ptr(ws), ws_bytes, _lib.stream_of(flat))
    _lib.check(st, "moe_permute_index")
    _lib.count_launches(2)
    return rid, off, src


@permute_index.register_fake
def _(indices, E):
    n = indices.numel()
    dev = indices.device
    return (torch.empty(n, dtype=torch.int32, device=dev),
            torch.empty(E + 1, dtype=torch.int32, device=dev),
            torch.empty(n, dtype=torch.int32, device=dev))


def _gather_call(fn_name, x, row_src, outs, w, offsets, m_total, n, k, E, flops, rd, wr,
                 extra=()):
    _lib.require_cuda(x, row_src, w, offsets)
    lib = _lib.load()
    timing = _lib.gemm_timing
    with torch.cuda.device(x.device):
        if timing is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        st = getattr(lib, fn_name)(
            _lib.ptr(x), _lib.ptr(row_src), x.shape[0], *extra, *[_lib.ptr(o) for o in outs],
            _lib.ptr(offsets), offsets.numel(), m_total, n, k, E, 1, _lib.dtype_code(x.dtype),
            _lib.stream_of(x))
        if timing is not None:
            ev1.record()
            timing.append((fn_name, ev0, ev1, flops, rd, wr))
    _lib.check(st, fn_name)
    _lib.count_launches(1)


@torch.library.custom_op(f"{_NS}::gmm_gate_up_fwd_gather_raw", mutates_args=())
def gmm_gate_up_fwd_gather_raw(x: torch.Tensor, row_src: torch.Tensor, B_gate: torch.Tensor,
                               B_up: torch.Tensor, offsets: torch.Tensor
                               ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(gate, up, h) of the gate/up + SwiGLU launch over the rows x[row_src[r]] (trans_b)."""
    x, B_gate, B_up = x.contiguous(), B_gate.contiguous(), B_up.contiguous()
    row_src = row_src.to(torch.int32).contiguous()
    E, N, K = B_gate.shape
    offsets = _norm_offsets(offsets, E)
    m = row_src.numel()
    gate = torch.empty((m, N), device=x.device, dtype=x.dtype)
    up, h = torch.empty_like(gate), torch.empty_like(gate)
    es = x.element_size()
    _gather_call("moe_gmm_gate_up_fwd_gather", x, row_src, (B_gate, B_up, gate, up, h), B_gate,
                 offsets, m, N, K, E, 2 * 2.0 * m * N * K, 2 * E * N * K * es + m * K * es,
                 3 * m * N * es)
    return gate, up, h


@gmm_gate_up_fwd_gather_raw.register_fake
def _(x, row_src, B_gate, B_up, offsets):
    g = torch.empty((row_src.numel(), B_gate.shape[1]), device=x.device, dtype=x.dtype)
    return g, torch.empty_like(g), torch.empty_like(g)


@torch.library.custom_op(f"{_NS}::gmm_wgrad_gather_raw", mutates_args=())
def gmm_wgrad_gather_raw(x: torch.Tensor, row_src: torch.Tensor, grad_C: torch.Tensor,
                         offsets: torch.Tensor, E: int) -> torch.Tensor:
    """grad_B[e] [N, K] = grad_C_e^T . x[row_src]_e over each expert's rows (trans_b)."""
    x, grad_C = x.contiguous(), grad_C.contiguous()
    row_src = row_src.to(torch.int32).contiguous()
    offsets = _norm_offsets(offsets, E)
    m, N = grad_C.shape
    K = x.shape[1]
    grad_B = torch.empty((E, N, K), device=x.device, dtype=x.dtype)
    es = x.element_size()
    _gather_call("moe_gmm_wgrad_gather", x, row_src, (grad_C, grad_B), grad_C, offsets, m, N, K, E,
                 2.0 * m * N * K, m * (N + K) * es, E * N * K * es)
    return grad_B


@gmm_wgrad_gather_raw.register_fake
def _(x, row_src, grad_C, offsets, E):
    return torch.empty((E, grad_C.shape[1], x.shape[1]), device=x.device, dtype=x.dtype)


class GroupedSwiGLUMLPGathered(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, row_src, row_id_map, B_gate, B_up, B_down, offsets, T, K):
        gate, up, h = torch.ops.moeb200.gmm_gate_up_fwd_gather_raw(x, row_src, B_gate, B_up, offsets)
        out = gmm_fwd_raw(h, B_down, offsets, True)
        ctx.save_for_backward(x, row_src, row_id_map, B_gate, B_up, B_down, offsets, gate, up, h)
        ctx.T, ctx.K = T, K
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, row_src, row_id_map, B_gate, B_up, B_down, offsets, gate, up, h = ctx.saved_tensors
        E = B_gate.shape[0]
        grad_out = grad_out.contiguous()
        dgate, dup = gmm_dgrad_swiglu_bwd_raw(grad_out, B_down, gate, up, offsets, True)
        g_down = gmm_bwd_B_raw(h, B_down, offsets, grad_out, True)
        grad_x = None
        if ctx.needs_input_grad[0]:
            d_rows = gmm_dgrad_dual_raw(dgate, B_gate, dup, B_up, offsets, True)
            grad_x = permute_backward(d_rows, row_id_map, ctx.T, ctx.K)
        g_gate = torch.ops.moeb200.gmm_wgrad_gather_raw(x, row_src, dgate, offsets, E)
        g_up = torch.ops.moeb200.gmm_wgrad_gather_raw(x, row_src, dup, offsets, E)
        return grad_x, None, None, g_gate, g_up, g_down, None, None, None


def grouped_swiglu_mlp_gathered(x, row_src, row_id_map, B_gate, B_up, B_down, offsets, T, K):
    """The SwiGLU expert MLP over the permuted rows x[row_src[r]] without materialising them
    (weights in the trans_b layout [E, N, K]); differentiable in x and the three weights.
    Returns the down projection's rows in permuted order [T*K, d]."""
    return GroupedSwiGLUMLPGathered.apply(x, row_src, row_id_map, B_gate, B_up, B_down, offsets,
                                          T, K)


def gathered_path_ok(x: torch.Tensor, d_hidden: int) -> bool:
    """True when the gathered launches take these shapes (the tensor-core path)."""
    return (x.dtype in (torch.float16, torch.bfloat16) and x.shape[1] % 8 == 0
            and d_hidden % 8 == 0 and x.is_contiguous() and x.data_ptr() % 16 == 0)


__all__ = ["permute_index", "grouped_swiglu_mlp_gathered", "gmm_gate_up_fwd_gather_raw",
           "gmm_wgrad_gather_raw"]
