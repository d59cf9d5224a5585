"""GPU parity of fused_topk_softmax against the oracle and the reference's golden vectors."""
import pytest
import torch

import moe_ops_b200 as M
from conftest import golden_names, load_golden
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_names("topk_"))
def test_golden(cuda_dev, name):
    g = load_golden(name)
    K = int(g["K"])
    logits = g["logits"].to(cuda_dev).requires_grad_(True)
    w, idx = M.fused_topk_softmax(logits, K)
    assert torch.equal(idx.cpu(), g["indices"].to(torch.int32))
    ref_w, _ = O.topk_softmax_fwd(g["logits"], K)  # RNE rounding, as on the GPU
    if w.dtype == torch.float32:
        assert (w.detach().cpu() - g["weights"]).abs().max().item() <= 1e-6
    else:
        assert (w.detach().cpu().float() - ref_w.float()).abs().max().item() <= 2 ** -8
    w.backward(g["grad_weights"].to(cuda_dev))
    ref_gl = O.topk_softmax_bwd(g["grad_weights"], w.detach().cpu(), idx.cpu(), logits.shape[1])
    tol = 1e-6 if w.dtype == torch.float32 else 0.0
    assert (logits.grad.cpu().float() - ref_gl.float()).abs().max().item() <= tol


def _tie_free_logits(T, E, dtype, seed):
    # tests/test_topk_softmax.py:37-41 of the reference: separated columns, no ties.
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(T, E, generator=g) * 0.05
    return (raw + torch.arange(E).float() * 0.5).to(dtype)


@pytest.mark.parametrize("E,K", [(16, 2), (64, 4), (256, 16), (64, 2), (256, 8), (20, 3), (1024, 32)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_reference_configs(cuda_dev, E, K, dtype):
    T = 8192 if E <= 256 else 1024
    logits = _tie_free_logits(T, E, dtype, seed=E * 100 + K)
    lg = logits.to(cuda_dev).requires_grad_(True)
    w, idx = M.fused_topk_softmax(lg, K)
    ref_w, ref_idx = O.topk_softmax_fwd(logits, K)
    assert torch.equal(idx.cpu(), ref_idx)
    diff = (w.detach().cpu().float() - ref_w.float()).abs().max().item()
    assert diff <= (1e-6 if dtype == torch.float32 else 1e-2)
    gw = torch.randn(T, K, generator=torch.Generator().manual_seed(7)).to(dtype)
    w.backward(gw.to(cuda_dev))
    ref_gl = O.topk_softmax_bwd(gw, w.detach().cpu(), idx.cpu(), E)
    assert (lg.grad.cpu().float() - ref_gl.float()).abs().max().item() <= (1e-6 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("fp32_routing", [False, True])
def test_cfg3_and_random_ties(cuda_dev, fp32_routing):
    # Config 3: logits [8192, 64] fp32 ~ N(0,1), K=2; plus bf16 logits with real ties.
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(8192, 64, generator=g)
    w, idx = M.fused_topk_softmax(logits.to(cuda_dev), 2, fp32_routing=fp32_routing)
    ref_w, ref_idx = O.topk_softmax_fwd(logits, 2)
    assert torch.equal(idx.cpu(), ref_idx)
    assert (w.cpu() - ref_w).abs().max().item() <= 1e-6
    lb = torch.randint(0, 5, (4096, 64), generator=g).to(torch.bfloat16)  # many ties
    w, idx = M.fused_topk_softmax(lb.to(cuda_dev), 4, fp32_routing=fp32_routing)
    ref_w, ref_idx = O.topk_softmax_fwd(lb, 4)
    assert torch.equal(idx.cpu(), ref_idx)
    assert w.dtype == (torch.float32 if fp32_routing else torch.bfloat16)


def test_cfg5_skewed(cuda_dev):
    # Config 5 router: [32768, 256] ~ N(0,1) + 1.5*log(1/rank^1.2) bias, K=8, fp32 routing.
    g = torch.Generator().manual_seed(5)
    E = 256
    perm = torch.randperm(E, generator=g)
    rank = torch.empty(E)
    rank[perm] = torch.arange(1, E + 1).float()
    logits = torch.randn(32768, E, generator=g) + 1.5 * torch.log(1.0 / rank ** 1.2)
    w, idx = M.fused_topk_softmax(logits.to(cuda_dev).bfloat16(), 8, fp32_routing=True)
    ref_w, ref_idx = O.topk_softmax_fwd(logits.bfloat16().float(), 8)
    assert torch.equal(idx.cpu(), ref_idx)
    assert (w.cpu() - ref_w).abs().max().item() <= 1e-6
