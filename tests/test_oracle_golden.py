"""Pins the CPU oracle against golden vectors made by the reference itself
(tests/golden/make_golden.py runs triton_gmm_ops through the Triton interpreter)."""
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import moe_oracle as O


@pytest.mark.parametrize("name", golden_names("topk_"))
def test_topk_oracle_matches_reference(name):
    g = load_golden(name)
    w, idx = O.topk_softmax_fwd(g["logits"], int(g["K"]))
    assert torch.equal(idx, g["indices"].to(torch.int32))
    if w.dtype == torch.float32:
        assert (w - g["weights"]).abs().max().item() <= 1e-6
    else:  # bf16: the only difference can be fp32 exp/sum rounding crossing a bf16 tie
        assert (w.float() - g["weights"].float()).abs().max().item() <= 2 ** -8
    E = g["logits"].shape[1]
    gl = O.topk_softmax_bwd(g["grad_weights"], g["weights"], g["indices"], E, cast=O.round_trunc)
    if gl.dtype == torch.float32:
        assert (gl - g["grad_logits"]).abs().max().item() <= 1e-6
    else:
        assert torch.equal(gl, g["grad_logits"])


@pytest.mark.parametrize("name", golden_names("perm_"))
def test_permute_oracle_matches_reference(name):
    # The fixtures come from the Triton interpreter, which casts fp32 -> bf16 by
    # truncation; the oracle's fp32 accumulators are rounded the same way here (the GPU
    # and the reference's PyTorch oracles round to nearest even: O.round_rne).
    tr = O.round_trunc
    g = load_golden(name)
    T, K, E = g["x"].shape[0], int(g["K"]), int(g["E"])
    perm, rid, off = O.permute(g["x"], g["indices"], E=E)
    assert torch.equal(off, g["offsets"].to(torch.int32))
    assert torch.equal(rid, g["row_id_map"].to(torch.int32))
    assert torch.equal(perm[: T * K], g["permuted"][: T * K])
    gi = O.permute_backward(g["grad_permuted"], rid, T, K, tr)
    assert torch.equal(gi, g["grad_input"])
    out = O.unpermute_fwd(g["unp_input"], rid, g["prob"], T, K, tr)
    assert torch.equal(out, g["unp_out_f32prob"])
    out_b = O.unpermute_fwd(g["unp_input"], rid, g["prob_bf16"], T, K, tr)
    assert torch.equal(out_b, g["unp_out_bf16prob"])
    act, pg, written = O.unpermute_bwd(g["grad_out"], g["unp_input"], rid, g["prob"], T, K, tr)
    assert torch.equal(act[written], g["act_grad"][written])
    assert (pg - g["prob_grad"]).abs().max().item() <= 1e-5 * max(1.0, g["prob_grad"].abs().max().item())


@pytest.mark.parametrize("name", golden_names("gmm_"))
def test_gmm_oracle_matches_reference(name):
    g = load_golden(name)
    trans_b = bool(g["trans_b"])
    E = g["B"].shape[0]
    C = O.gmm_fwd(g["A"], g["B"], g["offsets"], trans_b)
    assert O.rel_frobenius(g["C"], C) < 1e-5
    gA = O.gmm_dgrad(g["grad_C"], g["B"], g["offsets"], trans_b)
    assert O.rel_frobenius(g["grad_A"], gA) < 1e-5
    if "grad_B" in g:
        gB = O.gmm_wgrad(g["A"], g["grad_C"], g["offsets"], E, trans_b)
        assert O.rel_frobenius(g["grad_B"], gB) < 1e-5
    # E-length (end offsets) form gives the same result.
    C2 = O.gmm_fwd(g["A"], g["B"], g["offsets"][1:], trans_b)
    assert torch.equal(C, C2)


def test_cfg1_layer_oracle_matches_reference():
    from moe_cfg1 import make_cfg1

    g = load_golden("cfg1_layer_f32")
    x, wr, wg, wu, wd, E, K = make_cfg1()
    x.requires_grad_(True)
    wr.requires_grad_(True)
    out = O.moe_layer_forward(x, wr.t(), wg, wu, wd, K, E)
    loss = (out * out).sum()
    loss.backward()
    assert O.rel_frobenius(out.detach(), g["out"]) < 1e-5
    assert abs(loss.item() - float(g["loss"])) <= 1e-4 * abs(float(g["loss"]))
    assert O.rel_frobenius(x.grad, g["grad_x"]) < 1e-4
    assert O.rel_frobenius(wr.grad, g["grad_router"]) < 1e-4


def test_capacity_oracle_hand_case():
    """The dropping definition on a case worked by hand: T=4, K=2, E=3, capacity 2.
    Slots j = t*K+k route to experts [0,1 | 0,2 | 0,1 | 1,2].  Expert 0 has slots 0,2,4 and
    keeps 0,2; expert 1 has 1,5,6 and keeps 1,5; expert 2 has 3,7 and keeps both."""
    x = torch.arange(4 * 2, dtype=torch.float32).view(4, 2)
    idx = torch.tensor([[0, 1], [0, 2], [0, 1], [1, 2]], dtype=torch.int32)
    p, r, o = O.permute_capacity(x, idx, 3, capacity=2)
    assert o.tolist() == [0, 2, 4, 6]
    assert r.tolist() == [0, 1, -1, -1, 2, 4, 3, 5]  # row_id_map[k*T + t]
    assert [int(v) for v in p[:, 0] // 2] == [0, 1, 0, 2, 1, 3]  # tokens of the kept rows
    # a global budget of 5 rows also drops the last kept slot (expert 2, token 3)
    p5, r5, o5 = O.permute_capacity(x, idx, 3, capacity=2, num_out_tokens=5)
    assert o5.tolist() == [0, 2, 4, 5]
    assert r5.tolist() == [0, 1, -1, -1, 2, 4, 3, -1]
    assert p5.shape[0] == 5
