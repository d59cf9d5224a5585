"""CPU checks of the C-ABI library: it loads, exports every symbol include/moe_b200.h
declares, and its host-side argument validation works without a GPU."""
import ctypes
import os
import re

import pytest
import torch

from conftest import REPO


def _declared_functions():
    src = open(os.path.join(REPO, "include", "moe_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from moe_ops_b200 import build, _lib

    build.build()
    return _lib.load()


def test_header_declares_the_reference_surface():
    names = _declared_functions()
    for required in ["moe_topk_softmax_fwd", "moe_topk_softmax_bwd", "moe_permute",
                     "moe_permute_workspace_bytes", "moe_unpermute_fwd", "moe_unpermute_bwd",
                     "moe_gmm_fwd", "moe_gmm_dgrad", "moe_gmm_wgrad", "moe_last_error_string"]:
        assert required in names


def test_every_declared_symbol_is_exported_and_bound(lib):
    from moe_ops_b200 import _lib

    for name in _declared_functions():
        assert hasattr(lib, name), f"{name} not exported by libmoe_b200.so"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_workspace(lib):
    assert lib.moe_version().startswith(b"moe_b200")
    # one int32 count per (expert, 512-slot tile) + 16 bytes
    assert lib.moe_permute_workspace_bytes(8192, 2, 64) == 64 * 32 * 4 + 16
    assert lib.moe_permute_workspace_bytes(0, 2, 64) == 16


def test_argument_validation_is_host_side(lib):
    # Bad offsets length, bad dtype and bad K are rejected before any CUDA call.
    st = lib.moe_gmm_fwd(None, None, None, None, 3, 16, 8, 8, 8, 1, 2, None)
    assert st == 1 and b"num_offsets" in lib.moe_last_error_string()
    st = lib.moe_gmm_fwd(None, None, None, None, 9, 16, 8, 8, 8, 1, 7, None)
    assert st == 1 and b"dtype" in lib.moe_last_error_string()
    st = lib.moe_topk_softmax_fwd(None, 0, 16, 8, 9, None, None, None)
    assert st == 1
    st = lib.moe_permute(None, 2, None, 16, 2, 64, 8, 8, None, None, None, None, 0, None)
    assert st == 1 and b"num_out" in lib.moe_last_error_string()
    st = lib.moe_permute(None, 2, None, 16, 2, 64, 4096, 32, None, None, None, None, 0, None)
    assert st == 1


def test_ops_refuse_cpu_tensors():
    import moe_ops_b200 as M

    x = torch.randn(8, 16)
    idx = torch.zeros(8, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        M.permute(x, idx, E=4)
    with pytest.raises(RuntimeError, match="CUDA"):
        M.fused_topk_softmax(torch.randn(8, 4), 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        M.grouped_gemm(x, torch.randn(2, 4, 16), torch.tensor([0, 4, 8], dtype=torch.int32))


def test_fake_impls_give_reference_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    import moe_ops_b200  # noqa: F401  (registers the ops)

    with FakeTensorMode():
        A = torch.empty(100, 64, dtype=torch.bfloat16)
        B = torch.empty(4, 32, 64, dtype=torch.bfloat16)
        off = torch.empty(5, dtype=torch.int32)
        assert torch.ops.moeb200.gmm_fwd_raw(A, B, off, True).shape == (100, 32)
        assert torch.ops.moeb200.gmm_bwd_B_raw(A, B, off, torch.empty(100, 32, dtype=torch.bfloat16),
                                               True).shape == (4, 32, 64)
        x = torch.empty(50, 64, dtype=torch.bfloat16)
        idx = torch.empty(50, 2, dtype=torch.int32)
        p, r, o = torch.ops.moeb200.permute_countsort(x, idx, 0, 8)
        assert p.shape == (100, 64) and r.shape == (100,) and o.shape == (9,)
        w, i = torch.ops.moeb200.fused_topk_softmax_fwd(torch.empty(50, 8), 2)
        assert w.shape == (50, 2) and i.dtype == torch.int32


def test_every_custom_op_has_a_fake_impl():
    """Each torch.ops.moeb200 op runs under FakeTensorMode (what torch.compile traces with)
    and returns the shapes and dtypes the real op returns.  The list below must name every
    op the package registers."""
    import glob
    import re

    from torch._subclasses.fake_tensor import FakeTensorMode
    import moe_ops_b200  # noqa: F401  (registers the ops)
    from moe_ops_b200 import fused_permute_ops, gate_up_ops, swiglu_ops  # noqa: F401

    bf = torch.bfloat16
    ops = torch.ops.moeb200
    T, K, E, d, H = 50, 2, 8, 64, 96
    with FakeTensorMode():
        x = torch.empty(T, d, dtype=bf)
        A = torch.empty(T * K, d, dtype=bf)
        off = torch.empty(E + 1, dtype=torch.int32)
        Wgu = torch.empty(E, H, d, dtype=bf)
        Wd = torch.empty(E, d, H, dtype=bf)
        idx = torch.empty(T, K, dtype=torch.int32)
        rid = torch.empty(T * K, dtype=torch.int32)
        prob = torch.empty(T, K)
        gate = torch.empty(T * K, H, dtype=bf)
        checks = {
            "gmm_fwd_raw": (ops.gmm_fwd_raw(A, Wgu, off, True), [((T * K, H), bf)]),
            "gmm_dgrad_raw": (ops.gmm_dgrad_raw(gate, Wgu, off, True), [((T * K, d), bf)]),
            "gmm_bwd_B_raw": (ops.gmm_bwd_B_raw(A, Wgu, off, gate, True), [((E, H, d), bf)]),
            "gmm_gate_up_fwd_raw": (ops.gmm_gate_up_fwd_raw(A, Wgu, Wgu, off, True),
                                    [((T * K, H), bf)] * 3),
            "gmm_dgrad_dual_raw": (ops.gmm_dgrad_dual_raw(gate, Wgu, gate, Wgu, off, True),
                                   [((T * K, d), bf)]),
            "gmm_dgrad_swiglu_bwd_raw": (
                ops.gmm_dgrad_swiglu_bwd_raw(A, Wd, gate, gate, off, True), [((T * K, H), bf)] * 2),
            "permute_countsort": (ops.permute_countsort(x, idx, 0, E),
                                  [((T * K, d), bf), ((T * K,), torch.int32), ((E + 1,), torch.int32)]),
            "scatter_rows": (ops.scatter_rows(x, rid, T * K, K), [((T * K, d), bf)]),
            "permute_index": (ops.permute_index(idx, E),
                              [((T * K,), torch.int32), ((E + 1,), torch.int32), ((T * K,), torch.int32)]),
            "gmm_gate_up_fwd_gather_raw": (ops.gmm_gate_up_fwd_gather_raw(x, rid, Wgu, Wgu, off),
                                           [((T * K, H), bf)] * 3),
            "gmm_wgrad_gather_raw": (ops.gmm_wgrad_gather_raw(x, rid, gate, off, E),
                                     [((E, H, d), bf)]),
            "permute_capacity": (ops.permute_capacity(x, idx, E, 5, 0),
                                 [((E * 5, d), bf), ((T * K,), torch.int32), ((E + 1,), torch.int32)]),
            "unpermute_forward": (ops.unpermute_forward(A, rid, prob, T, K), [((T, d), bf)]),
            "unpermute_backward": (ops.unpermute_backward(x, A, rid, prob, T, K),
                                   [((T * K, d), bf), ((T, K), torch.float32)]),
            "fused_topk_softmax_fwd": (ops.fused_topk_softmax_fwd(torch.empty(T, E), K),
                                       [((T, K), torch.float32), ((T, K), torch.int32)]),
            "fused_topk_softmax_bwd": (
                ops.fused_topk_softmax_bwd(prob, prob, idx, T, E, K), [((T, E), torch.float32)]),
            "swiglu_fwd": (ops.swiglu_fwd(gate, gate), [((T * K, H), bf)]),
            "swiglu_bwd": (ops.swiglu_bwd(gate, gate, gate), [((T * K, H), bf)] * 2),
        }
    for name, (out, want) in checks.items():
        outs = out if isinstance(out, (tuple, list)) else (out,)
        got = [(tuple(o.shape), o.dtype) for o in outs]
        assert got == want, f"{name}: fake gives {got}, expected {want}"
    registered = set()
    for path in glob.glob(os.path.join(REPO, "moe_ops_b200", "*.py")):
        registered |= set(re.findall(r'custom_op\(f"\{_NS\}::([A-Za-z0-9_]+)"', open(path).read()))
    assert registered == set(checks), (f"untested: {sorted(registered - set(checks))}, "
                                       f"not registered: {sorted(set(checks) - registered)}")

