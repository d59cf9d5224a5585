"""The allocation-free permute entry point, called through the C ABI.

moe_permute_noalloc serves callers that cannot allocate device memory when they call the
library (work recorded into a captured stream, code running inside an allocator, runtimes
that plan every buffer ahead): its scratch counts live in a fixed array inside the
library.  Its outputs must equal moe_permute's, call after call, because every call
reuses the same array.  This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from moe_ops_b200 import _lib

pytestmark = pytest.mark.gpu


def _permute_both(lib, x, idx, E):
    dev = x.device
    T, C = x.shape
    K = idx.shape[1]
    n = T * K
    code = _lib.dtype_code(x.dtype)
    stream = torch.cuda.current_stream(dev).cuda_stream
    outs = []
    for noalloc in (False, True):
        perm = torch.empty(n, C, device=dev, dtype=x.dtype)
        rid = torch.empty(n, device=dev, dtype=torch.int32)
        off = torch.empty(E + 1, device=dev, dtype=torch.int32)
        if noalloc:
            st = lib.moe_permute_noalloc(x.data_ptr(), code, idx.data_ptr(), T, K, C, E, n,
                                         perm.data_ptr(), rid.data_ptr(), off.data_ptr(), stream)
        else:
            ws_bytes = lib.moe_permute_workspace_bytes(T, K, E)
            ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
            st = lib.moe_permute(x.data_ptr(), code, idx.data_ptr(), T, K, C, E, n,
                                 perm.data_ptr(), rid.data_ptr(), off.data_ptr(), ws.data_ptr(),
                                 ws_bytes, stream)
        _lib.check(st, "permute")
        outs.append((perm, rid, off))
    torch.cuda.synchronize()
    return outs


def test_noalloc_matches_permute_on_consecutive_calls(cuda_dev):
    lib = _lib.load()
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    # Two calls in a row with different routing (and more experts the second time), so a
    # stale count left in the shared array by the first call would show up.
    for T, C, K, E in ((4096, 1024, 2, 64), (3000, 512, 4, 128)):
        x = torch.randn(T, C, device=cuda_dev, generator=g).to(torch.bfloat16)
        idx = torch.randint(0, E, (T, K), device=cuda_dev, generator=g, dtype=torch.int32)
        (p0, r0, o0), (p1, r1, o1) = _permute_both(lib, x, idx, E)
        assert torch.equal(o0, o1)
        assert torch.equal(r0, r1)
        assert torch.equal(p0, p1)


def test_noalloc_rejects_oversized_requests(cuda_dev):
    lib = _lib.load()
    E = 256
    max_slots = lib.moe_permute_noalloc_max_slots(E)
    assert max_slots > 0
    K = 8
    T = max_slots // K + 512  # one tile too many
    st = lib.moe_permute_noalloc(None, 2, None, T, K, 64, E, T * K, None, None, None, None)
    assert st == 1
    assert b"scratch" in ctypes.c_char_p(lib.moe_last_error_string()).value


@pytest.mark.parametrize("E,K,C", [(256, 8, 64), (1024, 2, 64)])
def test_noalloc_accepts_its_documented_maximum(cuda_dev, E, K, C):
    """T*K == moe_permute_noalloc_max_slots(E) is the largest size the header promises."""
    lib = _lib.load()
    max_slots = lib.moe_permute_noalloc_max_slots(E)
    assert max_slots % K == 0
    T = max_slots // K
    g = torch.Generator(device=cuda_dev).manual_seed(E)
    x = torch.randn(T, C, device=cuda_dev, generator=g).to(torch.bfloat16)
    idx = torch.randint(0, E, (T, K), device=cuda_dev, generator=g, dtype=torch.int32)
    for _ in range(2):
        (p0, r0, o0), (p1, r1, o1) = _permute_both(lib, x, idx, E)
        assert torch.equal(o0, o1)
        assert torch.equal(r0, r1)
        assert torch.equal(p0, p1)
