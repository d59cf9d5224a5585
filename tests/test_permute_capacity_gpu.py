"""Token dropping (moe_ops_b200.permute_with_capacity, C ABI moe_permute_capacity) against
the oracle's definition (oracle.moe_oracle.permute_capacity), bit for bit: kept rows, the
row_id_map with -1 for dropped slots, and the offsets of the kept rows; then unpermute and
the backward through dropped slots.  The reference has no dropping (its permute raises
num_out_tokens to T*K, triton_gmm_ops/permute_ops.py:89-93)."""
import pytest
import torch

import moe_ops_b200 as M
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,C,K,E,cap,num_out", [
    (512, 256, 2, 8, 100, 0),      # per-expert capacity below the mean load (128)
    (512, 256, 2, 8, 0, 700),      # a global row budget only
    (512, 256, 2, 8, 150, 900),    # both
    (333, 72, 4, 16, 1, 0),        # capacity 1, rows not a 16-byte multiple of 64
    (1000, 128, 1, 64, 20, 0),     # K = 1, many experts (some empty)
    (256, 64, 2, 4, 10_000, 0),    # capacity above every load: nothing dropped
])
def test_capacity_matches_oracle(cuda_dev, T, C, K, E, cap, num_out):
    g = torch.Generator().manual_seed(T + E + cap)
    x = torch.randn(T, C, generator=g).bfloat16()
    # skewed routing so that some experts overflow and some stay empty
    w = torch.rand(E, generator=g) ** 3
    idx = torch.stack([torch.multinomial(w, K, replacement=False, generator=g) for _ in range(T)])
    idx = idx.to(torch.int32)
    p, r, o = M.permute_with_capacity(x.to(cuda_dev), idx.to(cuda_dev), E, cap, num_out)
    rp, rr, ro = O.permute_capacity(x, idx, E, cap, num_out)
    assert torch.equal(o.cpu(), ro)
    assert torch.equal(r.cpu(), rr)
    n = int(ro[-1])
    assert p.shape == rp.shape
    assert torch.equal(p[:n].cpu(), rp[:n])
    if cap >= T * K:
        assert int((rr < 0).sum()) == 0


def test_dropped_slots_in_unpermute_and_backward(cuda_dev):
    T, C, K, E, cap = 256, 128, 2, 8, 40
    g = torch.Generator().manual_seed(3)
    x = torch.randn(T, C, generator=g).bfloat16()
    idx = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
    prob = torch.rand(T, K, generator=g)
    xd = x.to(cuda_dev).requires_grad_(True)
    pd = prob.to(cuda_dev).requires_grad_(True)
    perm, rid, off = M.permute_with_capacity(xd, idx.to(cuda_dev), E, cap)
    out = M.unpermute(perm, rid, pd, T, K)
    go = torch.randn(T, C, generator=g).bfloat16()
    out.backward(go.to(cuda_dev))
    rp, rr, ro = O.permute_capacity(x, idx, E, cap)
    assert int((rr < 0).sum()) > 0, "the case must drop slots"
    ref = O.unpermute_fwd(rp, rr, prob, T, K)
    assert torch.equal(out.detach().cpu(), ref)
    # a dropped slot's routing weight gets no gradient; its token gets none through it
    dropped = (rr.view(K, T).t() < 0)
    assert (pd.grad.cpu()[dropped] == 0).all()
    all_dropped = dropped.all(1)
    assert (xd.grad.cpu()[all_dropped] == 0).all()


def test_layer_with_capacity_factor(cuda_dev):
    """MoELayer.capacity_factor: the layer equals the plain composition over
    permute_with_capacity, and with a factor large enough to keep every slot it equals the
    layer without dropping, bit for bit."""
    from moe_ops_b200.moe_layer import MoELayer

    T, d, E, K, H = 256, 128, 8, 2, 192
    gen = torch.Generator(device=cuda_dev).manual_seed(5)
    layer = MoELayer(d, E, K, H, device=cuda_dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.05, generator=gen)
    x = torch.randn(T, d, device=cuda_dev, generator=gen).bfloat16()
    base = layer(x)
    layer.capacity_factor = float(E)  # capacity = T*K: nothing can be dropped
    assert torch.equal(layer(x), base)
    layer.capacity_factor = 0.5       # capacity 32 of a mean load of 64
    out = layer(x)
    w, idx = M.fused_topk_softmax(x @ layer.w_router.t(), K)
    perm, rid, off = M.permute_with_capacity(x, idx, E, 32)
    down = M.grouped_swiglu_mlp(perm, layer.w_gate, layer.w_up, layer.w_down, off)
    assert torch.equal(out, M.unpermute(down, rid, w, T, K))
    assert int((rid < 0).sum()) > 0
