"""Counting-sort permute and its backward.

Drop-in for the reference's permute API (triton_gmm_ops/permute_ops.py:82-159):

    permute(input, indices, num_out_tokens=0, E=None) -> (permuted, row_id_map, offsets)
    permute_backward(grad_permuted, row_id_map, num_tokens, topK) -> grad_input

``offsets`` is int32 [E+1] with offsets[0] = 0 and offsets[e+1] the end row of expert e,
exactly what grouped_gemm consumes.  ``row_id_map[k*T + t]`` is the row of ``permuted``
holding token t's k-th slot.  Unlike the reference's atomic scatter, rows inside an
expert group come out in slot order (stable), so results are deterministic.
"""
from __future__ import annotations

import torch

from . import _lib
from .unpermute_ops import _unpermute_call

_NS = "moeb200"


@torch.library.custom_op(f"{_NS}::permute_countsort", mutates_args=())
def permute_countsort(input: torch.Tensor, indices: torch.Tensor, num_out_tokens: int = 0,
                      E: int = 0) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    _lib.require_cuda(input, indices)
    input = input.contiguous()
    if indices.dim() == 1:
        indices = indices.unsqueeze(1)
    num_tokens, num_cols = input.shape
    topK = indices.shape[1]
    flat = indices.reshape(-1)
    if flat.dtype != torch.int32:
        flat = flat.to(torch.int32)
    flat = flat.contiguous()
    num_total = num_tokens * topK
    num_out = num_out_tokens if num_out_tokens > 0 else num_total
    # offsets always sum to num_total, so permuted holds at least that many rows
    # (capacity dropping is not part of the reference contract either).
    num_out = max(num_out, num_total)
    if E <= 0:
        E = int(flat.max()) + 1 if num_total > 0 else 1
    lib = _lib.load()
    permuted = torch.empty(num_out, num_cols, device=input.device, dtype=input.dtype)
    row_id_map = torch.empty(num_total, dtype=torch.int32, device=input.device)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=input.device)
    ws_bytes = lib.moe_permute_workspace_bytes(num_tokens, topK, E)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=input.device)
    with torch.cuda.device(input.device):
        st = lib.moe_permute(
            _lib.ptr(input), _lib.dtype_code(input.dtype), _lib.ptr(flat), num_tokens, topK,
            num_cols, E, num_out, _lib.ptr(permuted), _lib.ptr(row_id_map), _lib.ptr(offsets),
            _lib.ptr(ws), ws_bytes, _lib.stream_of(input))
    _lib.check(st, "moe_permute")
    _lib.count_launches(4)
    return permuted, row_id_map, offsets


@permute_countsort.register_fake
def _(input, indices, num_out_tokens=0, E=0):
    num_tokens, num_cols = input.shape
    topK = indices.shape[1] if indices.dim() > 1 else 1
    num_total = num_tokens * topK
    num_out = max(num_out_tokens, num_total)
    off_len = E + 1 if E > 0 else num_total + 1
    return (torch.empty(num_out, num_cols, device=input.device, dtype=input.dtype),
            torch.empty(num_total, device=input.device, dtype=torch.int32),
            torch.empty(off_len, device=input.device, dtype=torch.int32))


def permute_backward(grad_permuted: torch.Tensor, row_id_map: torch.Tensor,
                     num_tokens: int, topK: int) -> torch.Tensor:
    """grad_input[t] = sum_k grad_permuted[row_id_map[k*T+t]] (fp32 accumulation).

    Same as unpermute with prob = 1 (permute_ops.py:130-133); no ones tensor is built.
    """
    return _unpermute_call(grad_permuted, row_id_map, None, num_tokens, topK)


class PermuteAutograd(torch.autograd.Function):
    """Same contract as the reference's PermuteAutograd (permute_ops.py:136-154)."""

    @staticmethod
    def forward(ctx, input, indices, num_out_tokens=0, E=None):
        ctx.num_tokens = input.shape[0]
        ctx.topK = indices.shape[1] if indices.ndim > 1 else 1
        e = E if E is not None else 0
        permuted, row_id_map, offsets = torch.ops.moeb200.permute_countsort(
            input, indices, num_out_tokens, e)
        ctx.save_for_backward(row_id_map)
        ctx.mark_non_differentiable(row_id_map, offsets)
        return permuted, row_id_map, offsets

    @staticmethod
    def backward(ctx, grad_permuted, grad_row_id_map, grad_offsets):
        (row_id_map,) = ctx.saved_tensors
        grad_input = permute_backward(grad_permuted, row_id_map, ctx.num_tokens, ctx.topK)
        return grad_input, None, None, None


def permute(input, indices, num_out_tokens=0, E=None):
    """Differentiable counting-sort permute."""
    return PermuteAutograd.apply(input, indices, num_out_tokens, E)


# ---------------------------------------------------------------- permute with dropping


def capacity_rows(num_slots: int, num_experts: int, capacity: int, num_out_tokens: int) -> int:
    """Rows of the permuted buffer of permute_with_capacity (known on the host, no sync):
    num_out_tokens if given, else the most rows the capacity can keep."""
    if num_out_tokens > 0:
        return num_out_tokens
    if capacity > 0:
        return min(num_slots, num_experts * capacity)
    return num_slots


@torch.library.custom_op(f"{_NS}::permute_capacity", mutates_args=())
def permute_capacity(input: torch.Tensor, indices: torch.Tensor, E: int, capacity: int = 0,
                     num_out_tokens: int = 0) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Counting-sort permute that drops slots past an expert's capacity (the first
    `capacity` slots of each expert in token order are kept) or past num_out_tokens rows."""
    _lib.require_cuda(input, indices)
    input = input.contiguous()
    if indices.dim() == 1:
        indices = indices.unsqueeze(1)
    num_tokens, num_cols = input.shape
    topK = indices.shape[1]
    flat = indices.reshape(-1).to(torch.int32).contiguous()
    num_out = capacity_rows(num_tokens * topK, E, capacity, num_out_tokens)
    lib = _lib.load()
    permuted = torch.empty(num_out, num_cols, device=input.device, dtype=input.dtype)
    row_id_map = torch.empty(num_tokens * topK, dtype=torch.int32, device=input.device)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=input.device)
    ws_bytes = lib.moe_permute_workspace_bytes(num_tokens, topK, E)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=input.device)
    with torch.cuda.device(input.device):
        st = lib.moe_permute_capacity(
            _lib.ptr(input), _lib.dtype_code(input.dtype), _lib.ptr(flat), num_tokens, topK,
            num_cols, E, capacity, num_out, _lib.ptr(permuted), _lib.ptr(row_id_map),
            _lib.ptr(offsets), _lib.ptr(ws), ws_bytes, _lib.stream_of(input))
    _lib.check(st, "moe_permute_capacity")
    _lib.count_launches(3)
    return permuted, row_id_map, offsets


@permute_capacity.register_fake
def _(input, indices, E, capacity=0, num_out_tokens=0):
    num_tokens, num_cols = input.shape
    topK = indices.shape[1] if indices.dim() > 1 else 1
    num_out = capacity_rows(num_tokens * topK, E, capacity, num_out_tokens)
    return (torch.empty(num_out, num_cols, device=input.device, dtype=input.dtype),
            torch.empty(num_tokens * topK, device=input.device, dtype=torch.int32),
            torch.empty(E + 1, device=input.device, dtype=torch.int32))


class PermuteCapacityAutograd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input, indices, E, capacity, num_out_tokens):
        ctx.num_tokens = input.shape[0]
        ctx.topK = indices.shape[1] if indices.ndim > 1 else 1
        permuted, row_id_map, offsets = torch.ops.moeb200.permute_capacity(
            input, indices, E, capacity, num_out_tokens)
        ctx.save_for_backward(row_id_map)
        ctx.mark_non_differentiable(row_id_map, offsets)
        return permuted, row_id_map, offsets

    @staticmethod
    def backward(ctx, grad_permuted, grad_row_id_map, grad_offsets):
        (row_id_map,) = ctx.saved_tensors
        # dropped slots (row -1) contribute nothing
        grad_input = permute_backward(grad_permuted, row_id_map, ctx.num_tokens, ctx.topK)
        return grad_input, None, None, None, None


def permute_with_capacity(input, indices, E: int, capacity: int = 0, num_out_tokens: int = 0):
    """Differentiable permute with token dropping; returns (permuted, row_id_map, offsets)
    as permute() does.  Each expert keeps its first `capacity` slots in token order
    (capacity <= 0: all); with num_out_tokens > 0 the permuted buffer has that many rows and
    slots whose row would fall past it are dropped too (the highest experts' last slots
    first).  Dropped slots have row_id_map = -1: unpermute gives them zero weight in the
    output and a zero routing-weight gradient.  The reference's permute has no dropping
    (permute_ops.py:89-93 raises num_out_tokens to T*K); permute() here keeps that contract."""
    return PermuteCapacityAutograd.apply(input, indices, E, capacity, num_out_tokens)


# ---------------------------------------------------------------- rows through a given map


@torch.library.custom_op(f"{_NS}::scatter_rows", mutates_args=())
def scatter_rows(input: torch.Tensor, row_id_map: torch.Tensor, num_out: int,
                 topK: int) -> torch.Tensor:
    """out[row_id_map[k*T+t]] = input[t] for every k: the copy step of permute with a given
    map (rows the map does not name are left unwritten)."""
    _lib.require_cuda(input, row_id_map)
    input = input.contiguous()
    row_id_map = row_id_map.to(torch.int32).contiguous()
    T, C = input.shape
    out = torch.empty(num_out, C, device=input.device, dtype=input.dtype)
    with torch.cuda.device(input.device):
        st = _lib.load().moe_scatter_rows(_lib.ptr(input), _lib.dtype_code(input.dtype),
                                          _lib.ptr(row_id_map), T, topK, C, _lib.ptr(out),
                                          _lib.stream_of(input))
    _lib.check(st, "moe_scatter_rows")
    _lib.count_launches(1)
    return out


@scatter_rows.register_fake
def _(input, row_id_map, num_out, topK):
    return torch.empty(num_out, input.shape[1], device=input.device, dtype=input.dtype)


class GatherRows(torch.autograd.Function):
    """rows -> token order through a one-to-one map (K = 1): out[t] = rows[row_id_map[t]].
    Forward is permute_backward (exact for K = 1), backward the matching scatter."""

    @staticmethod
    def forward(ctx, rows, row_id_map):
        ctx.save_for_backward(row_id_map)
        ctx.n = rows.shape[0]
        return permute_backward(rows, row_id_map, row_id_map.numel(), 1)

    @staticmethod
    def backward(ctx, g):
        (row_id_map,) = ctx.saved_tensors
        return torch.ops.moeb200.scatter_rows(g, row_id_map, ctx.n, 1), None


def gather_rows(rows, row_id_map):
    return GatherRows.apply(rows, row_id_map)
