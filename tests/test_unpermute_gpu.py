"""GPU parity of unpermute forward/backward against the oracle and golden vectors."""
import pytest
import torch

import moe_ops_b200 as M
from conftest import golden_names, load_golden
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_names("perm_"))
def test_golden(cuda_dev, name):
    g = load_golden(name)
    T, K = g["x"].shape[0], int(g["K"])
    rid = g["row_id_map"].to(torch.int32)
    inp = g["unp_input"]
    for pkey, okey in (("prob", "unp_out_f32prob"), ("prob_bf16", "unp_out_bf16prob")):
        out = M.unpermute_forward(inp.to(cuda_dev), rid.to(cuda_dev), g[pkey].to(cuda_dev), T, K)
        assert torch.equal(out.cpu(), O.unpermute_fwd(inp, rid, g[pkey], T, K))
        if out.dtype == torch.float32:
            assert torch.equal(out.cpu(), g[okey])
    act, pg = M.unpermute_backward(g["grad_out"].to(cuda_dev), inp.to(cuda_dev), rid.to(cuda_dev),
                                   g["prob"].to(cuda_dev), T, K)
    ract, rpg, written = O.unpermute_bwd(g["grad_out"], inp, rid, g["prob"], T, K)
    assert torch.equal(act.cpu()[written], ract[written])
    assert (pg.cpu() - g["prob_grad"]).abs().max().item() <= 1e-4 * max(1.0, g["prob_grad"].abs().max().item())


def _routing(T, K, E, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
    _, rid, _ = O.permute(torch.zeros(T, 1), idx, E=E)
    prob = torch.softmax(torch.randn(T, K, generator=g), dim=-1)
    return rid, prob, g


@pytest.mark.parametrize("prob_dtype", [torch.float32, torch.bfloat16])
def test_cfg3_bitexact(cuda_dev, prob_dtype):
    # Config 3: permuted rows [16384, 4096] bf16 with top-2 probs over 64 experts.
    T, K, E, C = 8192, 2, 64, 4096
    rid, prob, g = _routing(T, K, E, 1)
    prob = prob.to(prob_dtype)
    inp = torch.randn(T * K, C, generator=g).to(torch.bfloat16)
    out = M.unpermute(inp.to(cuda_dev), rid.to(cuda_dev), prob.to(cuda_dev), T, K)
    assert torch.equal(out.cpu(), O.unpermute_fwd(inp, rid, prob, T, K))
    go = torch.randn(T, C, generator=g).to(torch.bfloat16)
    act, pg = M.unpermute_backward(go.to(cuda_dev), inp.to(cuda_dev), rid.to(cuda_dev),
                                   prob.to(cuda_dev), T, K)
    ract, rpg, written = O.unpermute_bwd(go, inp, rid, prob, T, K)
    assert written.all()
    assert torch.equal(act.cpu(), ract)
    rel = ((pg.cpu().float() - rpg.float()).abs() / rpg.float().abs().clamp(min=1.0)).max().item()
    assert rel <= (1e-4 if prob_dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("T,C,K,E,dtype", [
    (77, 13, 3, 5, torch.float32),
    (513, 7168, 8, 256, torch.bfloat16),
    (1000, 520, 2, 16, torch.float16),
    (64, 4096, 1, 16, torch.bfloat16),
])
def test_shapes(cuda_dev, T, C, K, E, dtype):
    rid, prob, g = _routing(T, K, E, T + C)
    inp = torch.randn(T * K, C, generator=g).to(dtype)
    out = M.unpermute_forward(inp.to(cuda_dev), rid.to(cuda_dev), prob.to(cuda_dev), T, K)
    assert torch.equal(out.cpu(), O.unpermute_fwd(inp, rid, prob, T, K))
    go = torch.randn(T, C, generator=g).to(dtype)
    act, pg = M.unpermute_backward(go.to(cuda_dev), inp.to(cuda_dev), rid.to(cuda_dev),
                                   prob.to(cuda_dev), T, K)
    ract, rpg, written = O.unpermute_bwd(go, inp, rid, prob, T, K)
    assert torch.equal(act.cpu()[written], ract[written])
    assert (pg.cpu() - rpg).abs().max().item() <= 1e-3 * max(1.0, rpg.abs().max().item())


def test_missing_slots_and_max_tokens(cuda_dev):
    # A row id of -1 contributes nothing; max_tokens > T gives zero rows past T.
    T, K, C = 16, 2, 64
    rid, prob, g = _routing(T, K, 4, 9)
    rid[3] = -1
    inp = torch.randn(T * K, C, generator=g)
    out = M.unpermute_forward(inp.to(cuda_dev), rid.to(cuda_dev), prob.to(cuda_dev), T, K,
                              max_tokens=T + 5)
    assert out.shape == (T + 5, C)
    assert torch.equal(out[:T].cpu(), O.unpermute_fwd(inp, rid, prob, T, K))
    assert (out[T:] == 0).all()


def test_finite_difference(cuda_dev):
    # The reference's FD check (tests/test_unpermute.py:71-110), fp32, 32x64 and 64x128.
    for T, C, E in ((32, 64, 8), (64, 128, 16)):
        K = 2
        rid, prob, g = _routing(T, K, E, C)
        a = torch.randn(T * K, C, generator=g).to(cuda_dev).requires_grad_(True)
        b = prob.to(cuda_dev).requires_grad_(True)
        M.unpermute(a, rid.to(cuda_dev), b, T, K).sum().backward()
        eps = 1e-3
        pg_num = torch.zeros(T, K)
        for t in range(0, T, 7):
            for k in range(K):
                bp = b.detach().clone(); bp[t, k] += eps
                bn = b.detach().clone(); bn[t, k] -= eps
                fp = M.unpermute_forward(a.detach(), rid.to(cuda_dev), bp, T, K).sum().item()
                fn = M.unpermute_forward(a.detach(), rid.to(cuda_dev), bn, T, K).sum().item()
                pg_num[t, k] = (fp - fn) / (2 * eps)
                assert abs(b.grad[t, k].item() - pg_num[t, k].item()) < 5e-2
        # act_grad of sum() is prob broadcast over the row
        rmap = rid.reshape(K, T).long()
        for k in range(K):
            assert torch.allclose(a.grad[rmap[k].to(cuda_dev)].sum(1).cpu(), b.detach()[:, k].cpu() * C,
                                  rtol=1e-5, atol=1e-4)
