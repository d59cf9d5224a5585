"""Generates the golden fixtures in tests/golden/*.npz from the REFERENCE implementation.

Runs the reference package (echogujy/moe_ops, ``triton_gmm_ops``) on the CPU through the
Triton interpreter (TRITON_INTERPRET=1) on small seeded inputs and stores inputs and
outputs.  The interpreter runs one program at a time, so the reference's atomic permute
scatter comes out in slot order (the order of its PyTorch oracle, a stable argsort).

Usage (needs the reference source tree; it is not needed to run the tests):

    python tests/golden/make_golden.py /path/to/reference

Autotuning has no GPU to benchmark on; the harness makes the autotuner pick the first
config (the same shim noted in the survey of the reference).
"""
from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _pack(t: torch.Tensor) -> np.ndarray:
    """Stores bf16/fp16 as their 16-bit patterns (numpy has no bf16)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().copy()
    return t.numpy().copy()


def save(name: str, **arrays) -> None:
    out = {}
    for k, v in arrays.items():
        if isinstance(v, torch.Tensor):
            out[k] = _pack(v)
            out[k + "__dtype"] = np.array(str(v.dtype).replace("torch.", ""))
        else:
            out[k] = np.asarray(v)
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


def main(ref_root: str) -> None:
    import triton.runtime.autotuner as at

    at.Autotuner.do_bench = property(lambda s: (lambda fn, quantiles=None, **k: [1.0] * 3))
    sys.path.insert(0, ref_root)
    import triton_gmm_ops as tg  # the reference

    # ---------------------------------------------------------------- top-k softmax
    topk_cases = [
        ("topk_f32_E8_K2", 33, 8, 2, torch.float32, "randn"),
        ("topk_f32_E64_K4", 40, 64, 4, torch.float32, "randn"),
        ("topk_f32_E256_K8", 24, 256, 8, torch.float32, "randn"),
        ("topk_bf16_E64_K2", 48, 64, 2, torch.bfloat16, "randn"),
        ("topk_bf16_E20_K3", 17, 20, 3, torch.bfloat16, "randn"),
        ("topk_f32_ties_E16_K4", 32, 16, 4, torch.float32, "ties"),
    ]
    for i, (name, T, E, K, dt, kind) in enumerate(topk_cases):
        g = torch.Generator().manual_seed(100 + i)
        if kind == "ties":
            logits = torch.randint(0, 4, (T, E), generator=g).float() * 0.5
        else:
            logits = torch.randn(T, E, generator=g)
        logits = logits.to(dt)
        grad_w = torch.randn(T, K, generator=g).to(dt)
        if dt == torch.float32:
            lg = logits.clone().requires_grad_(True)
            w, idx = tg.fused_topk_softmax(lg, K)
            w.backward(grad_w)
            grad_logits = lg.grad
        else:
            # The interpreter cannot build bf16 constants, so the forward kernel runs on the
            # exact fp32 image of the bf16 logits (the kernel compares and exponentiates in
            # fp32 either way) and the result is rounded to bf16 as the kernel's store does;
            # the backward kernel runs on the bf16 tensors themselves.
            w32, idx = tg.fused_topk_softmax(logits.float(), K)
            w = w32.to(dt)
            grad_logits = torch.ops.tg.fused_topk_softmax_bwd(grad_w, w, idx, T, E, K)
        save(name, logits=logits, K=K, weights=w, indices=idx, grad_weights=grad_w,
             grad_logits=grad_logits)

    # ---------------------------------------------------------------- permute / unpermute
    perm_cases = [
        ("perm_f32_T50_C24_K2_E8", 50, 24, 2, 8, torch.float32, ()),
        ("perm_f32_T37_C16_K4_E16_empty", 37, 16, 4, 16, torch.float32, (3, 7, 15)),
        ("perm_f32_T20_C8_K1_E4", 20, 8, 1, 4, torch.float32, ()),
        ("perm_bf16_T64_C32_K2_E8", 64, 32, 2, 8, torch.bfloat16, ()),
    ]
    for i, (name, T, C, K, E, dt, empty) in enumerate(perm_cases):
        g = torch.Generator().manual_seed(200 + i)
        x = torch.randn(T, C, generator=g).to(dt)
        allowed = torch.tensor([e for e in range(E) if e not in empty])
        idx = allowed[torch.randint(0, len(allowed), (T, K), generator=g)].to(torch.int32)
        permuted, rid, off = tg.permute(x, idx, E=E)
        grad_perm = torch.randn(T * K, C, generator=g).to(dt)
        grad_in = tg.permute_backward(grad_perm, rid, T, K)
        prob = torch.softmax(torch.randn(T, K, generator=g), dim=-1)
        prob_bf16 = prob.to(torch.bfloat16)
        unp_in = torch.randn(T * K, C, generator=g).to(dt)
        out_f32p = tg.unpermute_forward(unp_in, rid, prob, T, K)
        out_bf16p = tg.unpermute_forward(unp_in, rid, prob_bf16, T, K)
        grad_out = torch.randn(T, C, generator=g).to(dt)
        act_grad, prob_grad = tg.unpermute_backward(grad_out, unp_in, rid, prob, T, K)
        save(name, x=x, indices=idx, E=E, K=K, permuted=permuted, row_id_map=rid, offsets=off,
             grad_permuted=grad_perm, grad_input=grad_in, prob=prob, prob_bf16=prob_bf16,
             unp_input=unp_in, unp_out_f32prob=out_f32p, unp_out_bf16prob=out_bf16p,
             grad_out=grad_out, act_grad=act_grad, prob_grad=prob_grad)

    # ---------------------------------------------------------------- grouped GEMM (fp32)
    gmm_cases = [
        ("gmm_f32_transb_E4", [5, 0, 17, 9], 40, 24, True),
        ("gmm_f32_transb_E3_partial", [100, 130, 70], 72, 40, True),
        ("gmm_f32_notransb_E4", [7, 12, 0, 20], 32, 48, False),
    ]
    for i, (name, sizes, K, N, trans_b) in enumerate(gmm_cases):
        g = torch.Generator().manual_seed(300 + i)
        E = len(sizes)
        M = sum(sizes)
        A = torch.randn(M, K, generator=g).requires_grad_(True)
        Bshape = (E, N, K) if trans_b else (E, K, N)
        B = (torch.randn(*Bshape, generator=g) * 0.1).requires_grad_(trans_b)
        off = torch.zeros(E + 1, dtype=torch.int32)
        off[1:] = torch.tensor(sizes).cumsum(0).to(torch.int32)
        C = tg.grouped_gemm(A, B, off, trans_b=trans_b)
        gC = torch.randn(M, N, generator=g)
        C.backward(gC)
        extra = {"grad_B": B.grad} if trans_b else {}
        save(name, A=A, B=B, offsets=off, trans_b=trans_b, C=C, grad_C=gC, grad_A=A.grad, **extra)

    # ---------------------------------------------------------------- config 1: small layer
    # T=256, d=512, E=8, K=2, H=1024, fp32, seed 0 (the first BASELINE config); the inputs
    # are regenerated from the seed by the tests (tests/moe_cfg1.py).
    sys.path.insert(0, os.path.dirname(HERE))
    from moe_cfg1 import make_cfg1

    x, w_router, w_gate, w_up, w_down, E, K = make_cfg1()
    x.requires_grad_(True)
    for p in (w_router, w_gate, w_up, w_down):
        p.requires_grad_(True)
    logits = x @ w_router
    weights, ind = tg.fused_topk_softmax(logits, K)
    permuted, rid, off = tg.permute(x, ind.to(torch.int32), num_out_tokens=512, E=E)
    gate = tg.grouped_gemm(permuted, w_gate, off, trans_b=True)
    up = tg.grouped_gemm(permuted, w_up, off, trans_b=True)
    h = torch.nn.functional.silu(gate) * up
    down = tg.grouped_gemm(h, w_down, off, trans_b=True)
    out = tg.unpermute(down, rid, weights, x.shape[0], K)
    loss = (out * out).sum()
    loss.backward()
    save("cfg1_layer_f32", out=out, loss=loss.detach(), grad_x=x.grad, grad_router=w_router.grad,
         indices=ind, weights=weights, offsets=off,
         grad_w_down_e0_rows32=w_down.grad[0, :32], grad_w_gate_e0_rows32=w_gate.grad[0, :32])


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the reference checkout>")
    main(sys.argv[1])
