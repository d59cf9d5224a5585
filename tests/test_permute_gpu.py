"""GPU parity of permute / permute_backward: bit-exact against the oracle (stable slot
order) and the reference's golden vectors."""
import pytest
import torch

import moe_ops_b200 as M
from conftest import golden_names, load_golden
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _check_permute(x, idx, E, num_out=0):
    T = x.shape[0]
    K = idx.shape[1] if idx.dim() > 1 else 1
    dev = torch.device("cuda:0")
    p, r, o = M.permute(x.to(dev), idx.to(dev), num_out_tokens=num_out, E=E)
    rp, rr, ro = O.permute(x, idx, E=E, num_out_tokens=num_out)
    assert torch.equal(o.cpu(), ro)
    assert torch.equal(r.cpu(), rr)
    assert p.shape == rp.shape
    assert torch.equal(p[: T * K].cpu(), rp[: T * K])
    return p, r, o


@pytest.mark.parametrize("name", golden_names("perm_"))
def test_golden(cuda_dev, name):
    g = load_golden(name)
    T, K, E = g["x"].shape[0], int(g["K"]), int(g["E"])
    p, r, o = M.permute(g["x"].to(cuda_dev), g["indices"].to(cuda_dev), E=E)
    assert torch.equal(o.cpu(), g["offsets"].to(torch.int32))
    assert torch.equal(r.cpu(), g["row_id_map"].to(torch.int32))
    assert torch.equal(p[: T * K].cpu(), g["permuted"][: T * K])
    gi = M.permute_backward(g["grad_permuted"].to(cuda_dev), r, T, K)
    assert torch.equal(gi.cpu(), O.permute_backward(g["grad_permuted"], r.cpu(), T, K))
    if gi.dtype == torch.float32:  # fp32 outputs need no rounding: equal to the reference's
        assert torch.equal(gi.cpu(), g["grad_input"])


def test_cfg3_bitexact(cuda_dev):
    # Config 3: x [8192, 4096] bf16, indices from top-2 of [8192, 64] logits, num_out 16384.
    g = torch.Generator().manual_seed(1)
    x = torch.randn(8192, 4096, generator=g).to(torch.bfloat16)
    logits = torch.randn(8192, 64, generator=g)
    _, idx = O.topk_softmax_fwd(logits, 2)
    p, r, o = _check_permute(x, idx, 64, num_out=16384)
    grad = torch.randn(16384, 4096, generator=g).to(torch.bfloat16)
    gi = M.permute_backward(grad.to(cuda_dev), r, 8192, 2)
    assert torch.equal(gi.cpu(), O.permute_backward(grad, r.cpu(), 8192, 2))
    # round trip: permute_backward(permuted) / K == x
    rt = M.permute_backward(p, r, 8192, 2).float() / 2
    assert torch.equal(rt.cpu().to(torch.bfloat16), x)


@pytest.mark.parametrize("T,C,K,E,dtype", [
    (1, 8, 1, 1, torch.float32),          # single token, single expert
    (300, 13, 3, 7, torch.bfloat16),      # odd widths: element path
    (1000, 24, 2, 1024, torch.float16),   # more experts than slots (most empty)
    (4097, 256, 8, 256, torch.bfloat16),  # cfg5-like fan-out, ragged tile tail
    (2048, 4096, 1, 64, torch.float32),   # K=1, fp32 rows
])
def test_edge_shapes(cuda_dev, T, C, K, E, dtype):
    g = torch.Generator().manual_seed(T + C + K + E)
    x = torch.randn(T, C, generator=g).to(dtype)
    idx = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
    _check_permute(x, idx, E)


def test_skewed_and_empty_experts(cuda_dev):
    g = torch.Generator().manual_seed(3)
    T, K, E = 5000, 4, 64
    probs = torch.zeros(E)
    probs[:5] = torch.tensor([50.0, 20.0, 5.0, 1.0, 1.0])  # 59 empty experts
    idx = torch.multinomial(probs.expand(T, E), K, replacement=True, generator=g).to(torch.int32)
    x = torch.randn(T, 128, generator=g).to(torch.bfloat16)
    _, _, o = _check_permute(x, idx, E, num_out=T * K + 100)
    assert (o[6:] == T * K).all()


def test_infers_E_and_int64_indices(cuda_dev):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(64, 32, generator=g)
    idx = torch.randint(0, 9, (64, 2), generator=g)
    p, r, o = M.permute(x.to(cuda_dev), idx.to(cuda_dev))
    rp, rr, ro = O.permute(x, idx)
    assert torch.equal(o.cpu(), ro) and torch.equal(r.cpu(), rr)


def test_deterministic_repeat(cuda_dev):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(8192, 1024, generator=g).to(torch.bfloat16).to(cuda_dev)
    idx = torch.randint(0, 64, (8192, 2), generator=g, dtype=torch.int32).to(cuda_dev)
    a = M.permute(x, idx, E=64)
    for _ in range(3):
        b = M.permute(x, idx, E=64)
        assert all(torch.equal(u, v) for u, v in zip(a, b))


def test_autograd(cuda_dev):
    g = torch.Generator().manual_seed(6)
    x = torch.randn(256, 64, generator=g).to(cuda_dev).requires_grad_(True)
    idx = torch.randint(0, 8, (256, 2), generator=g, dtype=torch.int32).to(cuda_dev)
    p, r, o = M.permute(x, idx, E=8)
    gp = torch.randn_like(p)
    p.backward(gp)
    ref = O.permute_backward(gp.cpu(), r.cpu(), 256, 2)
    assert torch.equal(x.grad.cpu(), ref)
