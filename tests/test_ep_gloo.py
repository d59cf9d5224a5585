"""Expert parallelism on CPU: two gloo ranks run moe_ops_b200.ep.ep_moe_forward with a
PyTorch restatement of the per-rank ops (gloo ranks cannot launch the CUDA kernels) and
must reproduce a single-process layer over all ranks' tokens: outputs, input gradients and
each rank's expert-weight gradients."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _cpu_ops():
    from moe_ops_b200.ep import EPOps
    from oracle.moe_oracle import grouped_mm_loop

    def topk(lg, K):
        v, i = torch.topk(lg, K, dim=-1)
        return torch.softmax(v.float(), dim=-1).to(lg.dtype), i.to(torch.int32)

    def permute(x, idx, E):
        T, K = idx.shape
        flat = idx.reshape(-1).long()
        order = torch.argsort(flat, stable=True)
        permuted = x[order // K]
        rid = torch.empty(T * K, dtype=torch.int32)
        rid[(order % K) * T + order // K] = torch.arange(T * K, dtype=torch.int32)
        off = torch.zeros(E + 1, dtype=torch.int32)
        off[1:] = torch.bincount(flat, minlength=E).cumsum(0).to(torch.int32)
        return permuted, rid, off

    def unpermute(rows, rid, prob, T, K):
        r = rid.reshape(K, T).long()
        if prob is None:
            return rows[r[0]]
        return sum(prob[:, k:k + 1].float() * rows[r[k]].float() for k in range(K)).to(rows.dtype)

    return EPOps(topk=topk, permute=permute, unpermute=unpermute,
                 grouped_gemm=lambda a, w, off: grouped_mm_loop(a, w, off.long()))


def _inputs(world, T, d, E, H):
    g = torch.Generator().manual_seed(3)
    xs = [torch.randn(T, d, generator=g) for _ in range(world)]
    gos = [torch.randn(T, d, generator=g) for _ in range(world)]
    wr = torch.randn(E, d, generator=g) * 0.3
    wg = torch.randn(E, H, d, generator=g) * 0.1
    wu = torch.randn(E, H, d, generator=g) * 0.1
    wd = torch.randn(E, d, H, generator=g) * 0.1
    return xs, gos, wr, wg, wu, wd


def _worker(rank, world, port, T, d, E, H, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from moe_ops_b200.ep import ep_moe_forward
        from oracle.moe_oracle import moe_layer_forward

        xs, gos, wr, wg, wu, wd = _inputs(world, T, d, E, H)
        el = E // world
        sl = slice(rank * el, (rank + 1) * el)
        x = xs[rank].clone().requires_grad_(True)
        lg, lu, ld = (w[sl].clone().requires_grad_(True) for w in (wg, wu, wd))
        out = ep_moe_forward(x, wr, lg, lu, ld, K, E, ops=_cpu_ops())
        out.backward(gos[rank])

        # single-process reference over every rank's tokens
        xr = [t.clone().requires_grad_(True) for t in xs]
        fg, fu, fd = (w.clone().requires_grad_(True) for w in (wg, wu, wd))
        loss = 0
        refs = []
        for r in range(world):
            o = moe_layer_forward(xr[r], wr, fg, fu, fd, K, E)
            refs.append(o)
            loss = loss + (o * gos[r]).sum()
        loss.backward()
        errs = {
            "out": (out - refs[rank]).abs().max().item(),
            "grad_x": (x.grad - xr[rank].grad).abs().max().item(),
            "grad_gate": (lg.grad - fg.grad[sl]).abs().max().item(),
            "grad_up": (lu.grad - fu.grad[sl]).abs().max().item(),
            "grad_down": (ld.grad - fd.grad[sl]).abs().max().item(),
        }
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,E,K", [(2, 8, 2), (2, 4, 3)])
def test_ep_matches_single_process(world, E, K):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 24, 16, E, 32, K, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in results.items():
        for k, v in errs.items():
            assert v < 1e-4, f"rank {rank} {k} differs by {v}"


def test_counts_and_expert_ids():
    from moe_ops_b200.ep import local_expert_ids, send_counts

    off = torch.tensor([0, 2, 2, 5, 9], dtype=torch.int32)  # 4 experts, 2 ranks
    assert send_counts(off, 2).tolist() == [2, 0, 3, 4]
    recv = torch.tensor([2, 1, 0, 3], dtype=torch.int32)  # [src, local expert]
    assert local_expert_ids(recv, 2, 6).tolist() == [0, 0, 1, 1, 1, 1]
