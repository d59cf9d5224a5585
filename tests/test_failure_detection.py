"""Failure detection without faulting a GPU.

GPU: a bounded mbarrier wait that nothing satisfies gives up after a short limit, reports
through the library's device error word and leaves the context usable.
CPU (gloo): a rank that fails before the token exchange makes its peer's collective end
with an error after the process-group timeout instead of hanging."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_context_survives(cuda_dev):
    import moe_ops_b200 as M
    from moe_ops_b200 import _lib

    lib = _lib.load()
    assert _lib.read_device_error() == 0
    res = torch.full((1,), -1, dtype=torch.int32, device=cuda_dev)
    st = lib.moe_selftest_bounded_wait(50_000_000, res.data_ptr(),  # 50 ms
                                       torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert res.item() == 0  # the wait gave up
    assert _lib.read_device_error() == 1
    assert _lib.read_device_error() == 0  # reading clears it
    # the context still works
    x = torch.randn(64, 32, device=cuda_dev)
    idx = torch.randint(0, 4, (64, 2), device=cuda_dev, dtype=torch.int32)
    p, r, o = M.permute(x, idx, E=4)
    assert int(o[-1]) == 128


def _rank_main(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("injected failure before the exchange")
        from moe_ops_b200.ep import exchange_counts

        try:
            exchange_counts(torch.ones(4, dtype=torch.int32), 2)
            q.put((rank, "no error"))
        except Exception as e:  # noqa: BLE001 - the timeout surfaces as a runtime error
            q.put((rank, f"error: {type(e).__name__}"))
    except RuntimeError:
        q.put((rank, "failed"))


def test_peer_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "failed"
    assert got[0].startswith("error"), got[0]
