"""GPU parity of grouped_gemm_swiglu, the fused gate/up GEMM with the SwiGLU epilogue.

The bar is bit equality with the unfused sequence the reference's layer runs
(tests/test_moe.py:80-82): two grouped GEMMs and the SwiGLU, i.e. this library's
grouped_gemm and swiglu kernels, whose own parity against the oracle is tested in
test_grouped_gemm_gpu.py and test_swiglu_gpu.py.  Gradients go through the same kernels,
so they must match bit for bit too.  One case also checks h against the fp64 oracle.
"""
import pytest
import torch

import moe_ops_b200 as M
from moe_ops_b200.gate_up_ops import gmm_gate_up_fwd_raw
from moe_ops_b200.grouped_gemm_ops import gmm_fwd_raw
from moe_ops_b200.swiglu_ops import swiglu, swiglu_fwd
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _case(sizes, K, N, dtype, trans_b, seed, dev):
    g = torch.Generator().manual_seed(seed)
    E, Mt = len(sizes), sum(sizes)
    A = torch.randn(Mt, K, generator=g).to(dtype).to(dev)
    shape = (E, N, K) if trans_b else (E, K, N)
    Wg = (torch.randn(*shape, generator=g) * 0.05).to(dtype).to(dev)
    Wu = (torch.randn(*shape, generator=g) * 0.05).to(dtype).to(dev)
    off = torch.zeros(E + 1, dtype=torch.int32)
    off[1:] = torch.tensor(sizes, dtype=torch.int64).cumsum(0).to(torch.int32)
    dh = torch.randn(Mt, N, generator=g).to(dtype).to(dev)
    return A, Wg, Wu, off.to(dev), dh


def _check_forward(A, Wg, Wu, off, trans_b):
    gate, up, h = gmm_gate_up_fwd_raw(A, Wg, Wu, off, trans_b)
    gate_ref = gmm_fwd_raw(A, Wg, off, trans_b)
    up_ref = gmm_fwd_raw(A, Wu, off, trans_b)
    h_ref = swiglu_fwd(gate_ref, up_ref)
    torch.cuda.synchronize()
    assert torch.equal(gate, gate_ref), "gate differs from grouped_gemm"
    assert torch.equal(up, up_ref), "up differs from grouped_gemm"
    assert torch.equal(h, h_ref), "h differs from grouped_gemm + swiglu"
    return h


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("trans_b", [True, False])
def test_forward_bit_equal_ragged(cuda_dev, dtype, trans_b):
    # Empty experts, tails of 1..127 rows, a column block cut at N=200 (not a multiple of
    # the 128-column tile), rows spanning several tiles.
    A, Wg, Wu, off, _ = _case([5, 0, 17, 300, 129, 128, 1, 0, 64, 96], K=192, N=200,
                              dtype=dtype, trans_b=trans_b, seed=21, dev=cuda_dev)
    _check_forward(A, Wg, Wu, off, trans_b)


def test_forward_bit_equal_cfg4_slice(cuda_dev):
    # cfg4 shapes (d=4096, H=11008) on 8 experts with 256 +- 16 rows each.
    g = torch.Generator().manual_seed(22)
    sizes = (256 + torch.randint(-16, 17, (8,), generator=g)).tolist()
    A, Wg, Wu, off, _ = _case(sizes, K=4096, N=11008, dtype=torch.bfloat16, trans_b=True,
                              seed=23, dev=cuda_dev)
    _check_forward(A, Wg, Wu, off, True)


def test_against_fp64_oracle(cuda_dev):
    A, Wg, Wu, off, _ = _case([40, 0, 170, 90], K=128, N=136, dtype=torch.bfloat16,
                              trans_b=True, seed=24, dev=cuda_dev)
    h = M.grouped_gemm_swiglu(A, Wg, Wu, off)
    Ac, Wgc, Wuc, offc = (t.cpu() for t in (A, Wg, Wu, off))
    gate = O.gmm_fwd(Ac, Wgc, offc, True)
    up = O.gmm_fwd(Ac, Wuc, offc, True)
    h_ref = torch.nn.functional.silu(gate) * up
    assert O.rel_frobenius(h.cpu(), h_ref) <= 1e-2


def test_unaligned_and_fp32_take_the_unfused_kernels(cuda_dev):
    # K=130 rows are not 16-byte multiples, fp32 has no tensor-core path: both run the
    # CUDA-core GEMMs and the SwiGLU kernel inside the same entry point.
    for dtype, K in ((torch.bfloat16, 130), (torch.float32, 96)):
        A, Wg, Wu, off, _ = _case([10, 0, 70, 33], K=K, N=80, dtype=dtype, trans_b=True,
                                  seed=25, dev=cuda_dev)
        _check_forward(A, Wg, Wu, off, True)


@pytest.mark.parametrize("trans_b", [True, False])
def test_backward_bit_equal(cuda_dev, trans_b):
    A, Wg, Wu, off, dh = _case([33, 0, 250, 128, 7], K=256, N=264, dtype=torch.bfloat16,
                               trans_b=trans_b, seed=26, dev=cuda_dev)
    leaves = [t.clone().requires_grad_(True) for t in (A, Wg, Wu)]
    h = M.grouped_gemm_swiglu(leaves[0], leaves[1], leaves[2], off, trans_b)
    h.backward(dh)
    ref = [t.clone().requires_grad_(True) for t in (A, Wg, Wu)]
    gate = M.grouped_gemm(ref[0], ref[1], off, trans_b)
    up = M.grouped_gemm(ref[0], ref[2], off, trans_b)
    h_ref = swiglu(gate, up)
    h_ref.backward(dh)
    torch.cuda.synchronize()
    assert torch.equal(h, h_ref)
    for name, a, b in zip(("W_gate", "W_up"), leaves[1:], ref[1:]):
        assert torch.equal(a.grad, b.grad), f"grad of {name} differs"
    _check_dual_sum(leaves[0].grad, ref[0].grad)


# ------------------------------------------------------------------ down dgrad + SwiGLU backward


def _bwd_case(sizes, H, d, dtype, trans_b, seed, dev):
    g = torch.Generator().manual_seed(seed)
    E, Mt = len(sizes), sum(sizes)
    gy = torch.randn(Mt, d, generator=g).to(dtype).to(dev)  # gradient of the down output
    Wd = (torch.randn(*((E, d, H) if trans_b else (E, H, d)), generator=g) * 0.05).to(dtype).to(dev)
    gate = torch.randn(Mt, H, generator=g).to(dtype).to(dev)
    up = torch.randn(Mt, H, generator=g).to(dtype).to(dev)
    off = torch.zeros(E + 1, dtype=torch.int32)
    off[1:] = torch.tensor(sizes, dtype=torch.int64).cumsum(0).to(torch.int32)
    return gy, Wd, gate, up, off.to(dev)


def _check_dgrad_swiglu(gy, Wd, gate, up, off, trans_b):
    from moe_ops_b200.gate_up_ops import gmm_dgrad_swiglu_bwd_raw
    from moe_ops_b200.grouped_gemm_ops import gmm_dgrad_raw
    from moe_ops_b200.swiglu_ops import swiglu_bwd
    dg, du = gmm_dgrad_swiglu_bwd_raw(gy, Wd, gate, up, off, trans_b)
    dh = gmm_dgrad_raw(gy, Wd, off, trans_b)
    dg_ref, du_ref = swiglu_bwd(dh, gate, up)
    torch.cuda.synchronize()
    assert torch.equal(dg, dg_ref), "grad_gate differs from dgrad + swiglu_bwd"
    assert torch.equal(du, du_ref), "grad_up differs from dgrad + swiglu_bwd"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("trans_b", [True, False])
def test_dgrad_swiglu_bwd_bit_equal_ragged(cuda_dev, dtype, trans_b):
    # H=264 cuts the last 256-column tile; tails of 1..127 rows; empty experts.
    case = _bwd_case([5, 0, 17, 300, 129, 128, 1, 0, 64, 96], H=264, d=192, dtype=dtype,
                     trans_b=trans_b, seed=31, dev=cuda_dev)
    _check_dgrad_swiglu(*case, trans_b)


def test_dgrad_swiglu_bwd_bit_equal_cfg4_slice(cuda_dev):
    g = torch.Generator().manual_seed(32)
    sizes = (256 + torch.randint(-16, 17, (8,), generator=g)).tolist()
    case = _bwd_case(sizes, H=11008, d=4096, dtype=torch.bfloat16, trans_b=True, seed=33,
                     dev=cuda_dev)
    _check_dgrad_swiglu(*case, True)


def test_dgrad_swiglu_bwd_unfused_paths(cuda_dev):
    # H=130 (rows not 16-byte multiples) and fp32 run the CUDA-core GEMM and the SwiGLU
    # backward kernel in place inside the same entry point.
    for dtype, H in ((torch.bfloat16, 130), (torch.float32, 96)):
        case = _bwd_case([10, 0, 70, 33], H=H, d=64, dtype=dtype, trans_b=True, seed=34,
                         dev=cuda_dev)
        _check_dgrad_swiglu(*case, True)


@pytest.mark.parametrize("trans_b", [True, False])
def test_mlp_backward_bit_equal(cuda_dev, trans_b):
    # The whole expert MLP against the unfused autograd chain the reference's layer uses.
    g = torch.Generator().manual_seed(35)
    sizes, d, H = [33, 0, 250, 128, 7], 192, 264
    E, Mt = len(sizes), sum(sizes)
    A = torch.randn(Mt, d, generator=g).to(torch.bfloat16).to(cuda_dev)
    shape_gu = (E, H, d) if trans_b else (E, d, H)
    shape_d = (E, d, H) if trans_b else (E, H, d)
    Wg = (torch.randn(*shape_gu, generator=g) * 0.05).to(torch.bfloat16).to(cuda_dev)
    Wu = (torch.randn(*shape_gu, generator=g) * 0.05).to(torch.bfloat16).to(cuda_dev)
    Wd = (torch.randn(*shape_d, generator=g) * 0.05).to(torch.bfloat16).to(cuda_dev)
    gy = torch.randn(Mt, d, generator=g).to(torch.bfloat16).to(cuda_dev)
    off = torch.zeros(E + 1, dtype=torch.int32)
    off[1:] = torch.tensor(sizes, dtype=torch.int64).cumsum(0).to(torch.int32)
    off = off.to(cuda_dev)
    fused = [t.clone().requires_grad_(True) for t in (A, Wg, Wu, Wd)]
    out = M.grouped_swiglu_mlp(*fused, off, trans_b)
    out.backward(gy)
    ref = [t.clone().requires_grad_(True) for t in (A, Wg, Wu, Wd)]
    h_ref = swiglu(M.grouped_gemm(ref[0], ref[1], off, trans_b), M.grouped_gemm(ref[0], ref[2], off, trans_b))
    out_ref = M.grouped_gemm(h_ref, ref[3], off, trans_b)
    out_ref.backward(gy)
    torch.cuda.synchronize()
    assert torch.equal(out, out_ref)
    for name, a, b in zip(("W_gate", "W_up", "W_down"), fused[1:], ref[1:]):
        assert torch.equal(a.grad, b.grad), f"grad of {name} differs"
    _check_dual_sum(fused[0].grad, ref[0].grad)


def _check_dual_sum(dual, unfused):
    """The input gradient of the fused MLP sums the gate and up dgrads in one fp32
    accumulator and rounds once; the unfused chain rounds each dgrad, then their sum.  They
    differ by those extra roundings only (a few bf16 units in the last place)."""
    from oracle.moe_oracle import rel_frobenius

    assert rel_frobenius(dual.float().cpu(), unfused.float().cpu()) < 4e-3


@pytest.mark.parametrize("trans_b", [True, False])
def test_dgrad_dual_against_fp64_oracle(cuda_dev, trans_b):
    """moe_gmm_dgrad_dual: dgrad(g1, B1) + dgrad(g2, B2) in one launch, against the fp64
    oracle, on ragged experts with an empty one, unequal segment lengths (n1 != n2, one not a
    multiple of the 64-deep k-block) and a partial output tile."""
    from moe_ops_b200.gate_up_ops import gmm_dgrad_dual_raw
    from oracle import moe_oracle as O

    g = torch.Generator().manual_seed(36)
    sizes, k, n1, n2 = [40, 0, 300, 129, 5], 200, 264, 96
    E, Mt = len(sizes), sum(sizes)
    bf = torch.bfloat16
    g1 = torch.randn(Mt, n1, generator=g).to(bf)
    g2 = torch.randn(Mt, n2, generator=g).to(bf)
    B1 = (torch.randn(*((E, n1, k) if trans_b else (E, k, n1)), generator=g) * 0.05).to(bf)
    B2 = (torch.randn(*((E, n2, k) if trans_b else (E, k, n2)), generator=g) * 0.05).to(bf)
    off = torch.zeros(E + 1, dtype=torch.int32)
    off[1:] = torch.tensor(sizes).cumsum(0).to(torch.int32)
    out = gmm_dgrad_dual_raw(g1.to(cuda_dev), B1.to(cuda_dev), g2.to(cuda_dev), B2.to(cuda_dev),
                             off.to(cuda_dev), trans_b)
    ref = (O.gmm_dgrad(g1.double(), B1.double(), off, trans_b)
           + O.gmm_dgrad(g2.double(), B2.double(), off, trans_b))
    assert O.rel_frobenius(out.cpu().double(), ref) < 1e-2 / 4
    # two calls in a row give the same bits
    out2 = gmm_dgrad_dual_raw(g1.to(cuda_dev), B1.to(cuda_dev), g2.to(cuda_dev), B2.to(cuda_dev),
                              off.to(cuda_dev), trans_b)
    assert torch.equal(out, out2)
