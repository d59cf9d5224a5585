"""CPU oracle for the MoE hot path — TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU, the algorithms of the reference (echogujy/moe_ops,
package triton_gmm_ops) for every op on the hot path.  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg use it, and only as the checker or the timed CPU
reference; the product (moe_ops_b200) never imports it.

Parity is pinned: tests/test_oracle_golden.py checks every function here against golden
vectors produced by the reference's own Triton kernels (run on the CPU through the Triton
interpreter by tests/golden/make_golden.py) and by the reference's PyTorch oracles.

Integer/index work uses numpy; floating-point work uses torch on the CPU so that bf16/fp16
rounding is the real one.  Each function cites the reference lines it follows.
"""
from __future__ import annotations

import numpy as np
import torch

# ----------------------------------------------------------------------------- rounding


def round_rne(x32: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp32 -> dtype with round-to-nearest-even (torch's cast; the GPU's cvt.rn)."""
    return x32.to(dtype)


def round_trunc(x32: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp32 -> bf16 by dropping the low 16 bits: how the Triton *interpreter* casts, which
    is how the golden fixtures made on the CPU round their bf16 outputs.  Non-bf16 targets
    fall back to round_rne."""
    if dtype != torch.bfloat16:
        return x32.to(dtype)
    bits = x32.contiguous().view(torch.int32) & ~0xFFFF
    return bits.view(torch.float32).to(torch.bfloat16)


# ----------------------------------------------------------------------------- top-k softmax


def topk_softmax_fwd(logits: torch.Tensor, K: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Reference kernel triton_gmm_ops/fused_topk_softmax_ops.py:17-70.

    K rounds of (max, argmax with lowest index on ties, overwrite with -inf) over the
    logits in fp32, then softmax over the K picked values in fp32; weights are cast to
    the logits dtype, indices are int32.
    """
    x = logits.detach().to(torch.float32).numpy().copy()
    T, E = x.shape
    vals = np.empty((T, K), dtype=np.float32)
    idx = np.empty((T, K), dtype=np.int32)
    rows = np.arange(T)
    for k in range(K):
        i = np.argmax(x, axis=1)          # first (lowest) index among equal maxima
        vals[:, k] = x[rows, i]
        idx[:, k] = i
        x[rows, i] = -np.inf
    v = torch.from_numpy(vals)
    m = v.max(dim=1, keepdim=True).values
    e = torch.exp(v - m)
    s = e.sum(dim=1, keepdim=True)
    w = (e / s).to(logits.dtype)
    return w, torch.from_numpy(idx)


def topk_softmax_bwd(grad_w: torch.Tensor, w: torch.Tensor, idx: torch.Tensor,
                     E: int, cast=round_rne) -> torch.Tensor:
    """Reference kernel triton_gmm_ops/fused_topk_softmax_ops.py:83-114 (+ :150-165).

    dlogit[t, idx[t,k]] = w*(g - sum_k g*w) in fp32, cast to the weights dtype; zeros
    elsewhere.
    """
    g = grad_w.detach().to(torch.float32)
    wf = w.detach().to(torch.float32)
    s = (g * wf).sum(dim=1, keepdim=True)
    dy = cast(wf * (g - s), w.dtype)
    out = torch.zeros(w.shape[0], E, dtype=w.dtype)
    out.scatter_(1, idx.to(torch.int64), dy)
    return out


# ----------------------------------------------------------------------------- permute


def group_offsets(flat: np.ndarray, E: int) -> np.ndarray:
    """Reference triton_gmm_ops/permute_ops.py:17-43: histogram + inclusive prefix into
    offsets[E+1] with offsets[0] = 0."""
    counts = np.bincount(flat.astype(np.int64), minlength=E)[:E]
    off = np.zeros(E + 1, dtype=np.int32)
    off[1:] = np.cumsum(counts)
    return off


def permute(input: torch.Tensor, indices: torch.Tensor, E: int | None = None,
            num_out_tokens: int = 0) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Reference triton_gmm_ops/permute_ops.py:82-110 with the slot order of the
    reference's PyTorch oracle tests/test_permute.py:16-37 (stable argsort of the
    flattened expert ids; the Triton scatter is unordered within an expert, and its
    interpreter run produces exactly this order).

    Returns (permuted [max(num_out, T*K), C], row_id_map [K*T] int32, offsets [E+1] int32).
    Rows past T*K are zero here (the device op leaves them unwritten).
    """
    T, C = input.shape
    ind = indices.reshape(T, -1)
    K = ind.shape[1]
    flat = ind.reshape(-1).numpy().astype(np.int64)
    if E is None:
        E = int(flat.max()) + 1 if flat.size else 1
    order = np.argsort(flat, kind="stable")
    num_out = max(num_out_tokens if num_out_tokens > 0 else T * K, T * K)
    permuted = torch.zeros(num_out, C, dtype=input.dtype)
    permuted[: T * K] = input[torch.from_numpy(order // K)]
    row_id_map = np.full(T * K, -1, dtype=np.int32)
    t_idx, k_idx = order // K, order % K
    row_id_map[k_idx * T + t_idx] = np.arange(T * K, dtype=np.int32)
    return permuted, torch.from_numpy(row_id_map), torch.from_numpy(group_offsets(flat, E))


def permute_capacity(input: torch.Tensor, indices: torch.Tensor, E: int, capacity: int = 0,
                     num_out_tokens: int = 0) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Capacity dropping, which the reference leaves out (permute_ops.py:89-93 raises
    num_out_tokens to T*K): this library's definition, restated plainly.  Slots in stable
    argsort order of the flattened expert ids (as permute above); inside each expert the
    first `capacity` slots (lowest t*K + k) are kept (capacity <= 0: all), the kept slots are
    laid out expert by expert, and slots whose row would be >= num_out (> 0) are dropped
    too.  Dropped slots get row -1.  Returns (permuted [num_out or kept rows, C],
    row_id_map [K*T], offsets [E+1] of the kept rows)."""
    T, C = input.shape
    ind = indices.reshape(T, -1)
    K = ind.shape[1]
    flat = ind.reshape(-1).numpy().astype(np.int64)
    order = np.argsort(flat, kind="stable")
    cap = capacity if capacity > 0 else T * K
    row_id_map = np.full(T * K, -1, dtype=np.int32)
    counts = np.zeros(E, dtype=np.int64)
    kept = []
    for j in order:  # expert by expert, stable inside each
        e = flat[j]
        if counts[e] < cap:
            counts[e] += 1
            kept.append(j)
    if num_out_tokens > 0:
        kept = kept[:num_out_tokens]
        rows = num_out_tokens
    else:
        rows = min(T * K, E * capacity) if capacity > 0 else T * K
    permuted = torch.zeros(rows, C, dtype=input.dtype)
    kept = np.asarray(kept, dtype=np.int64)
    if kept.size:
        permuted[: kept.size] = input[torch.from_numpy(kept // K)]
        row_id_map[(kept % K) * T + kept // K] = np.arange(kept.size, dtype=np.int32)
    kept_counts = np.bincount(flat[kept], minlength=E) if kept.size else np.zeros(E, np.int64)
    offsets = np.zeros(E + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(kept_counts)
    return permuted, torch.from_numpy(row_id_map), torch.from_numpy(offsets)


# ----------------------------------------------------------------------------- unpermute


def unpermute_fwd(input: torch.Tensor, row_id_map: torch.Tensor, prob: torch.Tensor | None,
                  num_tokens: int, K: int, cast=round_rne) -> torch.Tensor:
    """Reference triton_gmm_ops/unpermute_ops.py:20-72 with the rounding sequence of the
    reference's PyTorch oracle tests/test_unpermute.py:25-35:
    acc = 0 (fp32); for k: acc = acc + fp32(prob[t,k]) * fp32(input[row]); cast once.
    prob None means ones (permute_backward, triton_gmm_ops/permute_ops.py:130-133).
    """
    C = input.shape[1]
    rmap = row_id_map.reshape(K, num_tokens).to(torch.int64)
    acc = torch.zeros(num_tokens, C, dtype=torch.float32)
    for k in range(K):
        src = rmap[k]
        valid = src >= 0
        g = input[src.clamp(min=0)].to(torch.float32) * valid[:, None].to(torch.float32)
        if prob is None:
            acc = acc + g
        else:
            acc = acc + prob[:, k:k + 1].to(torch.float32) * g
    return cast(acc, input.dtype)


def permute_backward(grad_permuted: torch.Tensor, row_id_map: torch.Tensor, num_tokens: int,
                     K: int, cast=round_rne) -> torch.Tensor:
    """Reference triton_gmm_ops/permute_ops.py:130-133 (unpermute with prob = 1)."""
    return unpermute_fwd(grad_permuted, row_id_map, None, num_tokens, K, cast)


def unpermute_bwd(grad_out: torch.Tensor, input_fwd: torch.Tensor, row_id_map: torch.Tensor,
                  prob: torch.Tensor, num_tokens: int, K: int,
                  cast=round_rne) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Reference kernel triton_gmm_ops/unpermute_ops.py:93-150.

    act_grad[i] = cast(fp32(g[t]) * fp32(p[t,k])), prob_grad[t,k] = sum_c g[t,c]*in[i,c]
    (fp32 here, summed in float64 then rounded: the device sum order differs, so callers
    compare prob_grad with a tolerance).  Returns (act_grad, prob_grad, written_mask) where
    written_mask marks the act_grad rows the op defines.
    """
    rmap = row_id_map.reshape(K, num_tokens).to(torch.int64)
    act = torch.zeros_like(input_fwd)
    written = torch.zeros(input_fwd.shape[0], dtype=torch.bool)
    pg = torch.zeros(num_tokens, K, dtype=torch.float64)
    g32 = grad_out.to(torch.float32)
    for k in range(K):
        src = rmap[k]
        valid = src >= 0
        s = src[valid]
        p = prob[:, k].to(torch.float32)[valid]
        act[s] = cast(g32[valid] * p[:, None], input_fwd.dtype)
        written[s] = True
        pg[valid, k] = (g32[valid].double() * input_fwd[s].double()).sum(dim=1)
    return act, pg.to(torch.float32).to(prob.dtype), written


# ----------------------------------------------------------------------------- grouped GEMM


def _ranges(offsets: torch.Tensor, E: int) -> list[tuple[int, int]]:
    off = [int(v) for v in offsets.tolist()]
    if len(off) == E:           # end offsets (grouped_gemm_ops_sm90.py:172-175)
        off = [0] + off
    return [(off[g], off[g + 1]) for g in range(E)]


def gmm_fwd(A: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor,
            trans_b: bool = True, acc: torch.dtype = torch.float64) -> torch.Tensor:
    """Reference triton_gmm_ops/grouped_gemm_ops.py:20-69 and the fp32 per-expert loop
    of tests/test_grouped_gemm.py:70-83: C[rows_g] = A[rows_g] @ (B[g]^T or B[g]) in
    fp32 (float64 by default; callers compare with a tolerance).  Works on whatever
    device the inputs live on (the tests use the GPU's fp64 units for the large configs)."""
    E = B.shape[0]
    N = B.shape[1] if trans_b else B.shape[2]
    C = torch.zeros(A.shape[0], N, dtype=acc, device=A.device)
    Ad = A.to(acc)
    for g, (s, e) in enumerate(_ranges(offsets, E)):
        if e > s:
            W = B[g].to(acc)
            C[s:e] = Ad[s:e] @ (W.t() if trans_b else W)
    return C


def gmm_dgrad(grad_C: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor,
              trans_b: bool = True, acc: torch.dtype = torch.float64) -> torch.Tensor:
    """grad_A of the reference's backward (grouped_gemm_ops_sm90.py:224-233)."""
    E = B.shape[0]
    K = B.shape[2] if trans_b else B.shape[1]
    gA = torch.zeros(grad_C.shape[0], K, dtype=acc, device=grad_C.device)
    G = grad_C.to(acc)
    for g, (s, e) in enumerate(_ranges(offsets, E)):
        if e > s:
            W = B[g].to(acc)
            gA[s:e] = G[s:e] @ (W if trans_b else W.t())
    return gA


def gmm_wgrad(A: torch.Tensor, grad_C: torch.Tensor, offsets: torch.Tensor, E: int,
              trans_b: bool = True, acc: torch.dtype = torch.float64) -> torch.Tensor:
    """Reference triton_gmm_ops/grouped_gemm_ops.py:126-192: grad_B[g] = G_g^T @ A_g
    ([E, N, K]); with trans_b False, A_g^T @ G_g ([E, K, N]).  Zeros for empty experts."""
    K = A.shape[1]
    N = grad_C.shape[1]
    gB = torch.zeros((E, N, K) if trans_b else (E, K, N), dtype=acc, device=A.device)
    Ad, G = A.to(acc), grad_C.to(acc)
    for g, (s, e) in enumerate(_ranges(offsets, E)):
        if e > s:
            gB[g] = G[s:e].t() @ Ad[s:e] if trans_b else Ad[s:e].t() @ G[s:e]
    return gB


def rel_frobenius(x: torch.Tensor, ref: torch.Tensor) -> float:
    """||x - ref||_F / ||ref||_F in float64 (0 when both are zero)."""
    x, ref = x.double(), ref.double()
    den = ref.norm().item()
    num = (x - ref).norm().item()
    return num / den if den > 0 else num


# ----------------------------------------------------------------------------- MoE layer


def grouped_mm_loop(A: torch.Tensor, W: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    """The reference's per-expert loop (tests/test_moe.py:28-36) for B [E, N, K], trans_b:
    differentiable through torch autograd."""
    E = W.shape[0]
    outs = []
    for g, (s, e) in enumerate(_ranges(offsets, E)):
        outs.append(A[s:e] @ W[g].t())
    return torch.cat(outs, dim=0) if outs else A.new_zeros(0, W.shape[1])


def moe_layer_forward(x: torch.Tensor, w_router: torch.Tensor, w_gate: torch.Tensor,
                      w_up: torch.Tensor, w_down: torch.Tensor, K: int, E: int,
                      fp32_routing: bool = False, num_out_tokens: int = 0,
                      routing: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """The reference's SwiGLU MoE layer (tests/test_moe.py:68-87) on the CPU with
    PyTorch-native pieces: router x @ Wr^T, top-k softmax, stable permute, per-expert
    gate/up GEMMs, silu(gate)*up, down GEMM, unpermute weighted by the routing probs.
    Differentiable with torch autograd (x, router and expert weights).  `routing`
    = (probs [T, K], indices [T, K]) replaces the router (used to compare layers whose
    router logits were rounded differently)."""
    T = x.shape[0]
    if routing is None:
        logits = x @ w_router.t()
        if fp32_routing:
            logits = logits.float()
        vals, idx = torch.topk(logits, K, dim=-1)
        probs = torch.softmax(vals.float(), dim=-1).to(logits.dtype)
    else:
        probs, idx = routing
        idx = idx.to(torch.int64)
    flat = idx.reshape(-1)
    order = torch.argsort(flat, stable=True)
    permuted = x[order // K]
    counts = torch.bincount(flat, minlength=E)
    offsets = torch.zeros(E + 1, dtype=torch.int64)
    offsets[1:] = counts.cumsum(0)
    gate = grouped_mm_loop(permuted, w_gate, offsets)
    up = grouped_mm_loop(permuted, w_up, offsets)
    h = torch.nn.functional.silu(gate) * up
    down = grouped_mm_loop(h, w_down, offsets)
    # unpermute: slot j = t*K + k sits at permuted row inv[j]
    inv = torch.empty_like(order)
    inv[order] = torch.arange(order.numel())
    rows = down[inv].reshape(T, K, -1).float()
    out = (rows * probs.float().unsqueeze(-1)).sum(dim=1)
    return out.to(x.dtype)
