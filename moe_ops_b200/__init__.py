"""moe_ops_b200 — B200 (sm_100a) MoE operator library.

Drop-in replacement for the public API of ``triton_gmm_ops`` (echogujy/moe_ops,
triton_gmm_ops/__init__.py:34-48).  Every op runs a hand-written sm_100a CUDA kernel from
libmoe_b200.so through its C ABI (include/moe_b200.h):

    grouped_gemm(A, B, offsets, trans_b=True) -> C            tcgen05 + TMEM + TMA
    supports_tma(dtype=None) -> bool
    permute(input, indices, num_out_tokens=0, E=None) -> (permuted, row_id_map, offsets)
    permute_backward(grad_permuted, row_id_map, num_tokens, topK)
    unpermute(input, row_id_map, prob, num_tokens, num_topK, max_tokens=-1)
    unpermute_forward(...), unpermute_backward(...)
    fused_topk_softmax(logits, K, fp32_routing=False) -> (weights, indices)

Beyond the reference: grouped_gemm_swiglu / grouped_swiglu_mlp (the SwiGLU expert MLP in
fused launches), permute_with_capacity (token dropping at a per-expert capacity), and
permute_index + grouped_swiglu_mlp_gathered (the permute fused into the expert GEMMs).

Layout conventions (same as the reference):
    A:        [total_tokens, K]   (all experts stacked along rows)
    B:        [E, N, K] if trans_b else [E, K, N]
    offsets:  int32 [E+1], offsets[0] = 0 and offsets[e+1] = end row of expert e
              ([E] end offsets are accepted too)
    C:        [total_tokens, N]
"""
from .grouped_gemm_ops import grouped_gemm, supports_tma
from .permute_ops import permute, permute_backward, permute_with_capacity
from .unpermute_ops import unpermute, unpermute_forward, unpermute_backward
from .fused_topk_softmax_ops import fused_topk_softmax
from .gate_up_ops import grouped_gemm_swiglu, grouped_swiglu_mlp
from .fused_permute_ops import grouped_swiglu_mlp_gathered, permute_index

__all__ = [
    "grouped_gemm",
    "supports_tma",
    "permute",
    "permute_backward",
    "unpermute",
    "unpermute_forward",
    "unpermute_backward",
    "fused_topk_softmax",
    # beyond the reference's API: the SwiGLU expert MLP's fused launches, token dropping
    "grouped_gemm_swiglu",
    "permute_with_capacity",
    # the permute fused into the expert GEMMs (rows gathered from x, no permuted copy)
    "permute_index",
    "grouped_swiglu_mlp_gathered",
    "grouped_swiglu_mlp",
]
