"""GPU parity of the fused SwiGLU against the reference layer's PyTorch passes
(F.silu(gate) * up, tests/test_moe.py:82, and its autograd backward)."""
import pytest
import torch
import torch.nn.functional as F

from moe_ops_b200.swiglu_ops import swiglu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(4096, 11008), (7, 13)])
def test_swiglu_matches_torch(cuda_dev, dtype, shape):
    g = torch.Generator(device=cuda_dev).manual_seed(1)
    gate = (torch.randn(*shape, device=cuda_dev, generator=g) * 3).to(dtype)
    up = torch.randn(*shape, device=cuda_dev, generator=g).to(dtype)
    dh = torch.randn(*shape, device=cuda_dev, generator=g).to(dtype)
    a, b = gate.clone().requires_grad_(True), up.clone().requires_grad_(True)
    h = swiglu(a, b)
    h.backward(dh)
    ra, rb = gate.clone().requires_grad_(True), up.clone().requires_grad_(True)
    rh = F.silu(ra) * rb
    rh.backward(dh)
    # One unit in the last place of the dtype (exp implementations may differ by an ulp).
    ulp = {torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10, torch.float32: 2 ** -22}[dtype]
    for x, r in ((h, rh), (a.grad, ra.grad), (b.grad, rb.grad)):
        err = ((x.float() - r.float()).abs() / r.float().abs().clamp(min=1e-2)).max().item()
        assert err <= 2 * ulp, err
