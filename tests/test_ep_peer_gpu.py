"""Expert parallelism over peer memory (moe_ops_b200/ep_peer.py).

- W ranks emulated in one process on one GPU (threads; host barriers in place of the
  device barrier, since waits between kernels on one GPU are not allowed): output and every
  gradient must equal the single-GPU composition over all ranks' tokens bit for bit, with
  the same routing.
- Out-of-range destinations are refused (rank -1, device error 3) instead of stored.
- The barrier's bounded wait: a flag nothing sets makes it give up with status 0.
- The real transport on 2 GPUs (CUDA IPC + device barrier), skipped with fewer GPUs.
"""
import os
import socket
import threading

import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(world, T=192, d=256, E=8, K=2, H=384, seed=3):
    g = torch.Generator().manual_seed(seed)
    xs = [torch.randn(T, d, generator=g).bfloat16() for _ in range(world)]
    gos = [torch.randn(T, d, generator=g).bfloat16() for _ in range(world)]
    logits = [torch.randn(T, E, generator=g) for _ in range(world)]
    wg, wu = ((torch.randn(E, H, d, generator=g) * 0.05).bfloat16() for _ in range(2))
    wd = (torch.randn(E, d, H, generator=g) * 0.05).bfloat16()
    return xs, gos, logits, wg, wu, wd, E, K


def _reference(xs, gos, logits, wg, wu, wd, E, K, dev):
    """Single GPU, all tokens: permute -> fused SwiGLU MLP -> unpermute."""
    import moe_ops_b200 as M

    x = torch.cat(xs).to(dev).requires_grad_(True)
    w_, idx = M.fused_topk_softmax(torch.cat(logits).to(dev), K)
    w_ = w_.detach().requires_grad_(True)
    ws = [t.to(dev).requires_grad_(True) for t in (wg, wu, wd)]
    perm, rid, off = M.permute(x, idx, E=E)
    down = M.grouped_swiglu_mlp(perm, *ws, off)
    out = M.unpermute(down, rid, w_, x.shape[0], K)
    out.backward(torch.cat(gos).to(dev))
    return out.detach(), x.grad, w_.grad, [t.grad for t in ws], idx


class _Ctx:
    """Stands in for autograd's context: the emulated ranks call the Function's forward and
    backward themselves, because autograd runs all of one device's backward work on one
    worker thread, where a rank waiting at a host barrier would block the others."""

    needs_input_grad = (True,) * 8

    def save_for_backward(self, *tensors):
        self.saved_tensors = tensors


class _EmulatedTransport:
    """W ranks as threads on one GPU: every rank's buffers are visible to every other; the
    all-gather and the barriers go through the host (after a device synchronisation)."""

    def __init__(self, rank, shared):
        from moe_ops_b200.ep_peer import _KINDS

        self.rank, self.world, self.capacity = rank, shared["world"], shared["capacity"]
        self._sh = shared
        self.buffers = shared["buffers"][rank]
        dev = self.buffers["recv"].device
        self.bases = {k: torch.tensor([shared["buffers"][r][k].data_ptr() for r in range(self.world)],
                                      dtype=torch.int64, device=dev) for k in _KINDS}

    def all_gather_counts(self, counts):
        torch.cuda.synchronize()
        self._sh["counts"][self.rank] = counts.clone()
        self._sh["bar"].wait()
        out = torch.stack(self._sh["counts"])
        self._sh["bar"].wait()
        return out

    def barrier(self):
        torch.cuda.synchronize()
        self._sh["bar"].wait()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_emulated_ranks_match_single_gpu(cuda_dev, world):
    import moe_ops_b200 as M
    from moe_ops_b200 import _lib
    from moe_ops_b200.ep_peer import _KINDS, _PeerExperts, capacity_rows

    xs, gos, logits, wg, wu, wd, E, K = _problem(world)
    ref_out, ref_gx, ref_gw, ref_gwe, _ = _reference(xs, gos, logits, wg, wu, wd, E, K, cuda_dev)
    T, d = xs[0].shape
    cap = capacity_rows(T, K, world)
    shared = {"world": world, "capacity": cap, "counts": [None] * world,
              "bar": threading.Barrier(world, timeout=120),
              "buffers": [{k: torch.zeros(cap, d, dtype=torch.bfloat16, device=cuda_dev) for k in _KINDS}
                          for _ in range(world)]}
    el = E // world
    results, errors = [None] * world, []

    def run(rank):
        try:
            tr = _EmulatedTransport(rank, shared)
            sl = slice(rank * el, (rank + 1) * el)
            x = xs[rank].to(cuda_dev)
            w_, idx = M.fused_topk_softmax(logits[rank].to(cuda_dev), K)
            ws = [t[sl].to(cuda_dev) for t in (wg, wu, wd)]
            ctx = _Ctx()
            with torch.no_grad():
                out = _PeerExperts.forward(ctx, x, w_, idx, *ws, tr, E)
                gx, gw, _, gg, gu, gd, _, _ = _PeerExperts.backward(ctx, gos[rank].to(cuda_dev))
            torch.cuda.synchronize()
            results[rank] = (out, gx, gw, [gg, gu, gd])
        except BaseException as exc:  # noqa: BLE001
            errors.append((rank, exc))
            shared["bar"].abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    assert _lib.read_device_error() == 0
    for r in range(world):
        out, gx, gw, gwe = results[r]
        rows = slice(r * T, (r + 1) * T)
        sl = slice(r * el, (r + 1) * el)
        assert torch.equal(out, ref_out[rows]), f"rank {r}: output"
        assert torch.equal(gx, ref_gx[rows]), f"rank {r}: grad x"
        assert torch.equal(gw, ref_gw[rows]), f"rank {r}: grad of the routing weights"
        for name, a, b in zip(("gate", "up", "down"), gwe, ref_gwe):
            assert torch.equal(a, b[sl]), f"rank {r}: grad W_{name}"


def test_out_of_range_destination_is_refused(cuda_dev):
    from moe_ops_b200 import _lib

    lib = _lib.load()
    T, K, E, W = 64, 2, 4, 2
    idx = torch.randint(0, E, (T, K), dtype=torch.int32, device=cuda_dev)
    rid = torch.arange(T * K, dtype=torch.int32, device=cuda_dev)
    delta = torch.tensor([0, 0, 10_000, 0], dtype=torch.int32, device=cuda_dev)  # expert 2 off the end
    ranks = torch.empty(T * K, dtype=torch.int32, device=cuda_dev)
    rows = torch.empty_like(ranks)
    st = lib.moe_ep_slot_map(_lib.ptr(idx), _lib.ptr(rid), _lib.ptr(delta), T, K, E, E // W, W,
                             T * K * W, _lib.ptr(ranks), _lib.ptr(rows), _lib.stream_of(idx))
    assert st == 0
    flat = idx.t().reshape(-1)  # slot j = k*T + t
    assert (ranks[flat == 2] == -1).all() and (ranks[flat != 2] == flat[flat != 2] // 2).all()
    # A dispatch over these slots stores nothing for the refused ones.
    bufs = [torch.zeros(T * K * W, 16, dtype=torch.bfloat16, device=cuda_dev) for _ in range(W)]
    bases = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=cuda_dev)
    x = torch.ones(T, 16, dtype=torch.bfloat16, device=cuda_dev)
    assert lib.moe_ep_dispatch(_lib.ptr(x), 2, _lib.ptr(bases), _lib.ptr(ranks), _lib.ptr(rows),
                               T, K, 16, None, _lib.stream_of(x)) == 0
    written = sum(int((b != 0).any(1).sum()) for b in bufs)
    assert written == int((flat != 2).sum())
    assert _lib.read_device_error() == 3  # read and cleared
    # After a barrier gave up (status 0) the row kernels touch no peer buffer at all.
    for b in bufs:
        b.zero_()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    assert lib.moe_ep_dispatch(_lib.ptr(x), 2, _lib.ptr(bases), _lib.ptr(ranks), _lib.ptr(rows),
                               T, K, 16, _lib.ptr(status), _lib.stream_of(x)) == 0
    out = torch.full((T, 16), 7.0, dtype=torch.bfloat16, device=cuda_dev)
    assert lib.moe_ep_combine(_lib.ptr(bases), 2, _lib.ptr(ranks), _lib.ptr(rows), None, 0, T, K,
                              16, _lib.ptr(out), _lib.ptr(status), _lib.stream_of(x)) == 0
    torch.cuda.synchronize()
    assert sum(int((b != 0).any(1).sum()) for b in bufs) == 0
    assert (out == 0).all()  # every slot read as absent


def test_barrier_gives_up_on_a_silent_peer(cuda_dev):
    from moe_ops_b200 import _lib

    lib = _lib.load()
    flags = [torch.zeros(2, dtype=torch.int64, device=cuda_dev) for _ in range(2)]
    table = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=cuda_dev)
    status = torch.ones(1, dtype=torch.int32, device=cuda_dev)
    epoch_a = torch.zeros(1, dtype=torch.int64, device=cuda_dev)
    epoch_b = torch.zeros(1, dtype=torch.int64, device=cuda_dev)
    # One rank alone: its own signal satisfies it, the status stays 1 and its epoch counter
    # advances on the device.
    one = torch.tensor([flags[0].data_ptr()], dtype=torch.int64, device=cuda_dev)
    assert lib.moe_ep_barrier(_lib.ptr(one), 0, 1, _lib.ptr(epoch_a), 50_000_000, _lib.ptr(status),
                              None) == 0
    assert status.item() == 1 and epoch_a.item() == 1
    # Rank 0 of 2: rank 1 never signals, so the wait runs out after 50 ms.
    assert lib.moe_ep_barrier(_lib.ptr(table), 0, 2, _lib.ptr(epoch_b), 50_000_000, _lib.ptr(status),
                              None) == 0
    assert status.item() == 0
    assert flags[1][0].item() == 1  # its own signal reached the silent peer's array
    assert _lib.read_device_error() == 4
    # A later barrier that completes leaves the failure recorded.
    assert lib.moe_ep_barrier(_lib.ptr(one), 0, 1, _lib.ptr(epoch_a), 50_000_000, _lib.ptr(status),
                              None) == 0
    assert status.item() == 0 and epoch_a.item() == 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nvlink_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    tr = None
    try:
        import moe_ops_b200 as M
        from moe_ops_b200 import _lib
        from moe_ops_b200.ep_peer import NVLinkTransport, capacity_rows, peer_experts

        dev = torch.device("cuda", rank)
        xs, gos, logits, wg, wu, wd, E, K = _problem(world)
        T, d = xs[0].shape
        el = E // world
        sl = slice(rank * el, (rank + 1) * el)
        tr = NVLinkTransport(None, capacity_rows(T, K, world), d, torch.bfloat16, dev, timeout_s=5.0)
        for step in range(2):  # twice: buffer reuse across steps goes through the barriers
            x = xs[rank].to(dev).requires_grad_(True)
            w_, idx = M.fused_topk_softmax(logits[rank].to(dev), K)
            w_ = w_.detach().requires_grad_(True)
            ws = [t[sl].to(dev).requires_grad_(True) for t in (wg, wu, wd)]
            out = peer_experts(x, w_, idx, *ws, tr, E)
            out.backward(gos[rank].to(dev))
        torch.cuda.synchronize()
        ok = tr.barrier_ok() and _lib.read_device_error() == 0
        ref_out, ref_gx, ref_gw, ref_gwe, _ = _reference(xs, gos, logits, wg, wu, wd, E, K, dev)
        rows = slice(rank * T, (rank + 1) * T)
        same = {"out": torch.equal(out.detach(), ref_out[rows]),
                "grad_x": torch.equal(x.grad, ref_gx[rows]),
                "grad_w": torch.equal(w_.grad, ref_gw[rows]),
                "grad_experts": all(torch.equal(a.grad, b[sl]) for a, b in zip(ws, ref_gwe))}
        # The same step captured in a CUDA graph (no host sync, barrier epochs on the device)
        # and replayed twice: still bit-exact.
        x = xs[rank].to(dev).requires_grad_(True)
        w_, idx = M.fused_topk_softmax(logits[rank].to(dev), K)
        w_ = w_.detach().requires_grad_(True)
        ws = [t[sl].to(dev).requires_grad_(True) for t in (wg, wu, wd)]
        g_out = gos[rank].to(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            peer_experts(x, w_, idx, *ws, tr, E).backward(g_out)
        torch.cuda.current_stream(dev).wait_stream(side)
        for t in (x, w_, *ws):
            t.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            gout = peer_experts(x, w_, idx, *ws, tr, E)
            gout.backward(g_out)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        ok = ok and tr.barrier_ok() and _lib.read_device_error() == 0
        same["graph_out"] = torch.equal(gout.detach(), ref_out[rows])
        same["graph_grads"] = (torch.equal(x.grad, ref_gx[rows]) and torch.equal(w_.grad, ref_gw[rows])
                               and all(torch.equal(a.grad, b[sl]) for a, b in zip(ws, ref_gwe)))
        q.put((rank, ok, same))
    finally:
        if tr is not None:
            tr.close()
        dist.destroy_process_group()


def test_nvlink_transport_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nvlink_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    for _ in range(2):
        rank, ok, same = q.get(timeout=10)
        assert ok, f"rank {rank}: a barrier timed out or a device error was raised"
        assert all(same.values()), f"rank {rank}: {same}"
