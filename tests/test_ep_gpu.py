"""Expert parallelism on 2 GPUs over NCCL with the CUDA kernels: each rank's output and
gradients must match the single-GPU layer over all ranks' tokens (same tolerance as the
layer tests: relative Frobenius error in bf16).  Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q, overlapped):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        from moe_ops_b200.ep import ep_moe_forward, ep_moe_forward_overlapped
        from moe_ops_b200.moe_layer import moe_layer_forward
        from oracle.moe_oracle import rel_frobenius

        dev = torch.device("cuda", rank)
        T, d, E, K, H = 512, 256, 8, 2, 512
        g = torch.Generator().manual_seed(5)
        xs = [torch.randn(T, d, generator=g).bfloat16() for _ in range(world)]
        gos = [torch.randn(T, d, generator=g).bfloat16() for _ in range(world)]
        wr = (torch.randn(E, d, generator=g) * 0.5).bfloat16()
        wg, wu = ((torch.randn(E, H, d, generator=g) * 0.05).bfloat16() for _ in range(2))
        wd = (torch.randn(E, d, H, generator=g) * 0.05).bfloat16()
        el = E // world
        sl = slice(rank * el, (rank + 1) * el)
        x = xs[rank].to(dev).requires_grad_(True)
        lg, lu, ld = (w[sl].to(dev).requires_grad_(True) for w in (wg, wu, wd))
        fwd = ep_moe_forward_overlapped if overlapped else ep_moe_forward
        out = fwd(x, wr.to(dev), lg, lu, ld, K, E)
        out.backward(gos[rank].to(dev))
        # single-GPU layer (same kernels, all experts) over every rank's tokens
        fg, fu, fd = (w.to(dev).requires_grad_(True) for w in (wg, wu, wd))
        ref_out = None
        ref_gx = None
        for r in range(world):
            xr = xs[r].to(dev).requires_grad_(True)
            o = moe_layer_forward(xr, wr.to(dev), fg, fu, fd, K)
            o.backward(gos[r].to(dev))
            if r == rank:
                ref_out, ref_gx = o.detach(), xr.grad
        errs = {"out": rel_frobenius(out.detach().cpu(), ref_out.cpu()),
                "grad_x": rel_frobenius(x.grad.cpu(), ref_gx.cpu()),
                "grad_gate": rel_frobenius(lg.grad.cpu(), fg.grad[sl].cpu()),
                "grad_down": rel_frobenius(ld.grad.cpu(), fd.grad[sl].cpu())}
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("overlapped", [False, True])
def test_ep_two_gpus_matches_single_gpu(overlapped):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, overlapped)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in results.items():
        for k, v in errs.items():
            assert v < 1e-2, f"rank {rank} {k} rel err {v}"
