"""GPU parity of grouped_gemm (forward, dgrad, wgrad).

Tolerance (the hot path's stated bar): relative Frobenius error against an fp32/fp64
computation <= 1e-2 for bf16 and <= 2e-3 for fp16; fp32 inputs (CUDA-core path) <= 1e-5.
"""
import pytest
import torch

import moe_ops_b200 as M
from conftest import golden_names, load_golden
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 1e-2, torch.float16: 2e-3, torch.float32: 1e-5}


@pytest.fixture(params=["auto", "1", "2"])
def cta_group(request, monkeypatch):
    """Runs a test with the automatic CTA-group choice, single-CTA tiles and SM-pair tiles."""
    if request.param != "auto":
        monkeypatch.setenv("MOE_B200_GMM_CG", request.param)
    else:
        monkeypatch.delenv("MOE_B200_GMM_CG", raising=False)
    return request.param


def _offsets(sizes):
    off = torch.zeros(len(sizes) + 1, dtype=torch.int32)
    off[1:] = torch.tensor(sizes, dtype=torch.int64).cumsum(0).to(torch.int32)
    return off


def _run(sizes, K, N, dtype, trans_b=True, seed=0, end_offsets=False, bscale=0.02):
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(seed)
    E, Mt = len(sizes), sum(sizes)
    A = torch.randn(Mt, K, generator=g).to(dtype)
    B = (torch.randn(*((E, N, K) if trans_b else (E, K, N)), generator=g) * bscale).to(dtype)
    gC = torch.randn(Mt, N, generator=g).to(dtype)
    off = _offsets(sizes)
    off_dev = (off[1:] if end_offsets else off).to(dev)
    Ad = A.to(dev).requires_grad_(True)
    Bd = B.to(dev).requires_grad_(True)
    C = M.grouped_gemm(Ad, Bd, off_dev, trans_b=trans_b)
    C.backward(gC.to(dev))
    torch.cuda.synchronize()
    tol = TOL[dtype]
    # fp64 reference; on the GPU's fp64 units for the large configs, on the CPU otherwise.
    rd = dev if Mt * N * K > 2 ** 31 else torch.device("cpu")
    A_, B_, gC_, off_ = A.to(rd), B.to(rd), gC.to(rd), off.to(rd)
    e_fwd = O.rel_frobenius(C.detach().to(rd), O.gmm_fwd(A_, B_, off_, trans_b))
    e_dg = O.rel_frobenius(Ad.grad.to(rd), O.gmm_dgrad(gC_, B_, off_, trans_b))
    e_wg = O.rel_frobenius(Bd.grad.to(rd), O.gmm_wgrad(A_, gC_, off_, E, trans_b))
    assert e_fwd <= tol, f"forward rel err {e_fwd}"
    assert e_dg <= tol, f"dgrad rel err {e_dg}"
    assert e_wg <= tol, f"wgrad rel err {e_wg}"
    # experts without rows get exactly zero weight gradients
    for e, s in enumerate(sizes):
        if s == 0:
            assert (Bd.grad[e] == 0).all()
    return C


@pytest.mark.parametrize("name", golden_names("gmm_"))
def test_golden_fp32(cuda_dev, name):
    g = load_golden(name)
    trans_b = bool(g["trans_b"])
    A = g["A"].to(cuda_dev).requires_grad_(True)
    B = g["B"].to(cuda_dev).requires_grad_(trans_b)
    C = M.grouped_gemm(A, B, g["offsets"].to(cuda_dev), trans_b=trans_b)
    assert O.rel_frobenius(C.detach().cpu(), g["C"]) <= 1e-5
    C.backward(g["grad_C"].to(cuda_dev))
    assert O.rel_frobenius(A.grad.cpu(), g["grad_A"]) <= 1e-5
    if trans_b:
        assert O.rel_frobenius(B.grad.cpu(), g["grad_B"]) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("trans_b", [True, False])
def test_small_ragged(cuda_dev, cta_group, dtype, trans_b):
    _run([5, 0, 17, 300, 129, 128, 1, 0], K=192, N=264, dtype=dtype, trans_b=trans_b, seed=1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_partial_tiles(cuda_dev, cta_group, dtype):
    # The deprecated partial-tile test's row counts (develop/deprecated/test_grouped_gemm.py
    # :227-253), with N=200 and K=136 (multiples of 8 keep the TMA path).
    _run([100, 250, 130, 300], K=136, N=200, dtype=dtype, seed=2)
    _run([100, 250, 130, 300], K=136, N=200, dtype=dtype, trans_b=False, seed=3)


@pytest.mark.parametrize("trans_b", [True, False])
def test_tail_tile_boundaries(cuda_dev, cta_group, trans_b):
    # Last row tiles of 32, 64, 65, 96, 128 and 127 rows (half pair tiles with 0, 1 or 2
    # full 32-row groups per CTA), 192 and 255 (full pair tiles with a short peer).
    _run([32, 64, 65, 96, 192, 255, 320, 383, 128 + 256], K=128, N=320, dtype=torch.bfloat16,
         trans_b=trans_b, seed=10)


def test_unaligned_falls_back_to_cuda_cores(cuda_dev):
    # K=130 rows are not 16-byte multiples: served by the CUDA-core kernel, same contract.
    _run([100, 250, 130, 300], K=130, N=202, dtype=torch.bfloat16, seed=4)


def test_end_offsets_form(cuda_dev, cta_group):
    _run([64, 0, 200, 33], K=256, N=256, dtype=torch.bfloat16, seed=5, end_offsets=True)


def test_fp32(cuda_dev):
    _run([10, 0, 70, 33], K=96, N=80, dtype=torch.float32, seed=6)


def test_all_empty(cuda_dev, cta_group):
    dev = cuda_dev
    A = torch.randn(0, 64, device=dev, dtype=torch.bfloat16, requires_grad=True)
    B = torch.randn(4, 128, 64, device=dev, dtype=torch.bfloat16, requires_grad=True)
    off = torch.zeros(5, dtype=torch.int32, device=dev)
    C = M.grouped_gemm(A, B, off)
    assert C.shape == (0, 128)
    C.sum().backward()
    assert (B.grad == 0).all()


def test_cfg2_uniform(cuda_dev, cta_group):
    # Config 2: A [16384, 4096], B [16, 4096, 4096], 1024 rows per expert.
    _run([1024] * 16, K=4096, N=4096, dtype=torch.bfloat16, seed=7)


def test_cfg2_zipf(cuda_dev, cta_group):
    # Config 2 variant: Zipf(s=1.1) sizes summing to 16384 with 2 empty experts.
    w = 1.0 / torch.arange(1, 15).double() ** 1.1
    sizes = (w / w.sum() * 16384).floor().long().tolist()
    sizes[0] += 16384 - sum(sizes)
    sizes = sizes[:7] + [0] + sizes[7:12] + [0] + sizes[12:]
    assert len(sizes) == 16 and sum(sizes) == 16384
    _run(sizes, K=4096, N=4096, dtype=torch.bfloat16, seed=8)


def test_deep_contraction_wgrad(cuda_dev, cta_group):
    # One expert with many rows: long ragged contraction in wgrad.
    _run([7000, 3, 1000], K=512, N=768, dtype=torch.bfloat16, seed=9)
