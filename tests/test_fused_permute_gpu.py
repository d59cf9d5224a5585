"""The permute fused into the expert GEMMs (moe_ops_b200.fused_permute_ops): the GEMMs read
their A rows from the token-order input through the row -> token map (TMA gather4), as the
reference's experiment develop/experiment/fused_ops.py:31-107 does with `sorted_id_map`.
The bar is bit equality with the same GEMMs on the materialised permuted rows, and with the
whole layer over permute(): outputs and every gradient."""
import os

import pytest
import torch

import moe_ops_b200 as M
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _routing(T, K, E, seed, dev, skew=True):
    g = torch.Generator().manual_seed(seed)
    w = torch.rand(E, generator=g) ** (3 if skew else 0)
    idx = torch.stack([torch.multinomial(w, K, replacement=False, generator=g) for _ in range(T)])
    return idx.to(torch.int32).to(dev), g


@pytest.mark.parametrize("T,K,E", [(300, 2, 8), (1000, 4, 16), (64, 1, 3)])
def test_permute_index_matches_permute(cuda_dev, T, K, E):
    idx, _ = _routing(T, K, E, T, cuda_dev)
    x = torch.randn(T, 32, device=cuda_dev).bfloat16()
    perm, rid, off = M.permute(x, idx, E=E)
    rid2, off2, src = M.permute_index(idx, E)
    assert torch.equal(rid, rid2) and torch.equal(off, off2)
    assert torch.equal(x[src.long()], perm)  # row r of the permuted rows is x[row_src[r]]
    _, rr, _ = O.permute(x.cpu(), idx.cpu(), E=E)
    assert torch.equal(rid.cpu(), rr)


@pytest.mark.parametrize("cg", ["1", "2"])
def test_gathered_gemms_bit_equal(cuda_dev, cg, monkeypatch):
    from moe_ops_b200.fused_permute_ops import gmm_gate_up_fwd_gather_raw, gmm_wgrad_gather_raw
    from moe_ops_b200.gate_up_ops import gmm_gate_up_fwd_raw
    from moe_ops_b200.grouped_gemm_ops import gmm_bwd_B_raw

    monkeypatch.setenv("MOE_B200_GMM_CG", cg)  # wgrad on 1-SM tiles or SM pairs
    T, K, E, d, H = 700, 2, 6, 256, 392
    idx, g = _routing(T, K, E, 7, cuda_dev)
    x = torch.randn(T, d, generator=g).bfloat16().to(cuda_dev)
    Wg = (torch.randn(E, H, d, generator=g) * 0.05).bfloat16().to(cuda_dev)
    Wu = (torch.randn(E, H, d, generator=g) * 0.05).bfloat16().to(cuda_dev)
    perm, rid, off = M.permute(x, idx, E=E)
    _, _, src = M.permute_index(idx, E)
    ref = gmm_gate_up_fwd_raw(perm, Wg, Wu, off, True)
    got = gmm_gate_up_fwd_gather_raw(x, src, Wg, Wu, off)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    dC = torch.randn(T * K, H, generator=g).bfloat16().to(cuda_dev)
    for _ in range(2):  # two calls in a row
        assert torch.equal(gmm_wgrad_gather_raw(x, src, dC, off, E),
                           gmm_bwd_B_raw(perm, Wg, off, dC, True))


def test_layer_fused_permute_bit_equal(cuda_dev):
    from moe_ops_b200.moe_layer import MoELayer

    T, d, E, K, H = 512, 256, 8, 2, 384
    gen = torch.Generator(device=cuda_dev).manual_seed(9)
    layer = MoELayer(d, E, K, H, device=cuda_dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.05, generator=gen)
    x = torch.randn(T, d, device=cuda_dev, generator=gen).bfloat16()
    go = torch.randn(T, d, device=cuda_dev, generator=gen).bfloat16()
    res = []
    for fused in (False, True):
        layer.fused_permute = fused
        for p in layer.parameters():
            p.grad = None
        xi = x.clone().requires_grad_(True)
        out = layer(xi)
        out.backward(go)
        res.append([out.detach(), xi.grad] + [p.grad.clone() for p in layer.parameters()])
    for a, b in zip(*res):
        assert torch.equal(a, b)
