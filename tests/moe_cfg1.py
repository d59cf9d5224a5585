"""Seeded inputs of the first BASELINE configuration (small SwiGLU MoE layer, fp32).

T=256 tokens, d=512, router weight [512, 8] ~ N(0, 0.02), E=8, topK=2,
W_gate / W_up [8, 1024, 512] and W_down [8, 512, 1024] ~ N(0, 0.02), x ~ N(0, 1), seed 0.
Generated on the CPU so that every machine with the same torch build sees the same values.
"""
import torch


def make_cfg1(dtype=torch.float32):
    g = torch.Generator().manual_seed(0)
    T, d, E, K, H = 256, 512, 8, 2, 1024
    x = torch.randn(T, d, generator=g)
    w_router = torch.randn(d, E, generator=g) * 0.02
    w_gate = torch.randn(E, H, d, generator=g) * 0.02
    w_up = torch.randn(E, H, d, generator=g) * 0.02
    w_down = torch.randn(E, d, H, generator=g) * 0.02
    cast = lambda t: t.to(dtype)  # noqa: E731
    return cast(x), cast(w_router), cast(w_gate), cast(w_up), cast(w_down), E, K
