"""Benchmark: SwiGLU MoE layer forward + backward on B200 (the reference's headline path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the largest single-GPU config of the headline metric):
T=8192 tokens, d=4096, E=64 experts, top-2, H=11008, bf16 SwiGLU; router weight
[4096, 64] ~ N(0, 0.02) on x ~ N(0, 1); expert weights ~ N(0, 0.02); grad_out ~ N(0, 1).
A step = router GEMM + fused top-k softmax + permute + 3 grouped GEMMs + SwiGLU +
unpermute, then the full backward (6 grouped GEMMs, unpermute/permute/top-k backward).

`value` is grouped-GEMM TFLOP/s of the whole job (9 GEMMs per step, 2*T*K*d*H FLOPs each).
Inputs (17.3 GB of weights) are far larger than L2, so no flush is needed between steps.
Under torchrun (N > 1) the layer is expert-parallel (moe_ops_b200.ep): each rank holds
E/N experts and 8192/N of the tokens (strong scaling, as config 4 is written), and rows go
to their experts' ranks and back over NVLink peer memory (--ep-transport nccl: NCCL
all-to-alls).  Before timing, an N > 1 run checks the EP layer over the same transport on
a small problem against the single-GPU layer and the CPU oracle ("ep_parity"), and exits
non-zero if that fails; after timing it reads the device error word and the peer barriers'
status ("device_error", "peer_barriers_ok") and exits non-zero if either is set.
At N = 1 the line also carries per-op figures ("ops": config 2 grouped GEMMs beside torch
grouped_mm and the reference's own Triton grouped GEMM, config 3 routing primitives).

`--impl reference` times the reference's PyTorch-native CPU path (restated in oracle/)
on the host cores, on a bounded sample of the same workload (8 of the 64 experts with
the same 256 rows per expert), and reports the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

CONFIGS = {
    # BASELINE config 4 (the headline): 8192 tokens in total, split evenly over the ranks
    # (strong scaling, as the config is written).
    "cfg4": dict(tokens=8192, d_model=4096, experts=64, top_k=2, hidden=11008, fp32_routing=False,
                 zipf=False, global_tokens=True, router_std=0.02,
                 workload="cfg4 SwiGLU MoE layer fwd+bwd, T=8192 (in total) d=4096 E=64 topK=2 "
                          "H=11008 bf16"),
    # Not a BASELINE config: cfg4's layer with 8192 tokens on every rank (weak scaling).
    "cfg4-weak": dict(tokens=8192, d_model=4096, experts=64, top_k=2, hidden=11008,
                      fp32_routing=False, zipf=False, global_tokens=False, router_std=0.02,
                      workload="cfg4 layer with 8192 tokens PER RANK (weak scaling; not the "
                               "BASELINE config), d=4096 E=64 topK=2 H=11008 bf16"),
    # 32768 tokens in total split over the ranks (strong scaling), router
    # logits ~ N(0, 1) plus a Zipf bias 1.5*log(1/rank^1.2) over a random expert order.
    "cfg5": dict(tokens=32768, d_model=7168, experts=256, top_k=8, hidden=2048, fp32_routing=True,
                 zipf=True, global_tokens=True, router_std=None,
                 workload="cfg5 skewed SwiGLU MoE fwd+bwd, T=32768 d=7168 E=256 topK=8 H=2048 bf16, "
                          "fp32 routing, Zipf(1.2) router bias"),
}
CFG = CONFIGS["cfg4"]
METRIC = "moe_layer_fwd_bwd_grouped_gemm_tflops"


def _write_bandwidth(dev, nbytes=4 << 30, reps=5):
    """DRAM write bandwidth (GB/s) of this GPU now: the library's 16-byte-store fill
    (moe_write_probe) over a buffer far larger than L2, timed with CUDA events."""
    from moe_ops_b200 import _lib

    lib = _lib.load()
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def fill():
        _lib.check(lib.moe_write_probe(buf.data_ptr(), nbytes, stream.cuda_stream), "moe_write_probe")

    fill()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(reps):
        fill()
    ev1.record(stream)
    ev1.synchronize()
    del buf
    return nbytes * reps / (ev0.elapsed_time(ev1) * 1e-3) / 1e9


def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _traffic_per_launch():
    """DRAM bytes per grouped-GEMM launch from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "gmm_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return None


class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons through NVML in a
    background thread while the timed region runs (reads only; changes no setting)."""

    REASONS = {  # NVML clocks-event reason bits
        0x0000000000000001: "gpu_idle",
        0x0000000000000002: "applications_clocks_setting",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000010: "sync_boost",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
        0x0000000000000100: "display_clock_setting",
    }

    def __init__(self, gpu_index: int, period_s: float = 0.005):
        self.gpu = gpu_index
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.bits = 0
        self.smax = None
        self._stop = None
        self._thread = None
        self.error = None

    def start(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.gpu]) if vis and vis.split(",")[0].isdigit() else self.gpu
            h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception as e:  # noqa: BLE001
            self.error = f"nvml unavailable: {e}"[:80]
            return
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                    bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.bits |= bits
                    for b, n in self.REASONS.items():
                        if bits & b:
                            self.reasons.add(n)
                except Exception:  # noqa: BLE001
                    pass
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()

    def stop(self):
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error or "not sampled"]}
        self._stop.set()
        self._thread.join()
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.smax, "reasons": sorted(self.reasons),
                "reason_bits": hex(self.bits), "samples": len(self.samples)}


def _progress(msg: str) -> None:
    """One line on stderr per phase of a run (rank-tagged), so a run cut short shows where."""
    if os.environ.get("MOE_BENCH_QUIET"):
        return
    sys.stderr.write(f"[bench rank {os.environ.get('RANK', '0')} {time.strftime('%H:%M:%S')}] {msg}\n")
    sys.stderr.flush()


def _make_inputs(dev, T, d, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16)
    go = torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16)
    return x, go


def ep_parity_check(world, rank, dev, transport, T=512, d=256, K=2, H=512, tol=1e-2):
    """Before the timed region of an N > 1 run: the expert-parallel layer, over the transport
    the run times, on a small seeded problem (T tokens per rank, E = 4*N experts), against
    the single-GPU layer over all ranks' tokens on this GPU (output, x, router and expert
    weight gradients), and on rank 0 the layer output against the CPU oracle
    (oracle.moe_oracle, fp32; the checker, never the timed path).  Returns
    {"max_rel_err", "ok", "checks"}; the errors are maxima over ranks."""
    import torch.distributed as dist

    from moe_ops_b200 import _lib
    from moe_ops_b200.ep import EPMoELayer
    from moe_ops_b200.moe_layer import MoELayer

    E = 4 * world
    el = E // world
    g = torch.Generator().manual_seed(2024)
    xs = [torch.randn(T, d, generator=g).bfloat16() for _ in range(world)]
    gos = [torch.randn(T, d, generator=g).bfloat16() for _ in range(world)]
    wr = (torch.randn(E, d, generator=g) * 0.5).bfloat16()
    wg, wu = ((torch.randn(E, H, d, generator=g) * 0.05).bfloat16() for _ in range(2))
    wd = (torch.randn(E, d, H, generator=g) * 0.05).bfloat16()
    sl = slice(rank * el, (rank + 1) * el)

    ep = EPMoELayer(d, E, K, H, device=dev, dtype=torch.bfloat16)
    ep.transport = transport
    with torch.no_grad():
        ep.w_router.copy_(wr)
        for p, w in ((ep.w_gate, wg), (ep.w_up, wu), (ep.w_down, wd)):
            p.copy_(w[sl])
    x = xs[rank].to(dev).requires_grad_(True)
    out = ep(x)
    out.backward(gos[rank].to(dev))
    torch.cuda.synchronize()
    healthy = ep.health_ok()
    ep.close()
    g_router = ep.w_router.grad.float().clone()
    dist.all_reduce(g_router)  # the router is replicated: its gradient sums over ranks

    full = MoELayer(d, E, K, H, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for p, w in ((full.w_router, wr), (full.w_gate, wg), (full.w_up, wu), (full.w_down, wd)):
            p.copy_(w)
    xa = torch.cat(xs).to(dev).requires_grad_(True)
    ref = full(xa)
    ref.backward(torch.cat(gos).to(dev))
    rows = slice(rank * T, (rank + 1) * T)

    def rel(a, b):
        a, b = a.detach().double().cpu(), b.detach().double().cpu()
        return float((a - b).norm() / b.norm().clamp_min(1e-30))

    errs = {"out": rel(out, ref[rows]), "grad_x": rel(x.grad, xa.grad[rows]),
            "grad_router": rel(g_router, full.w_router.grad.float()),
            "grad_w_gate": rel(ep.w_gate.grad, full.w_gate.grad[sl]),
            "grad_w_up": rel(ep.w_up.grad, full.w_up.grad[sl]),
            "grad_w_down": rel(ep.w_down.grad, full.w_down.grad[sl])}
    if rank == 0:
        from oracle.moe_oracle import moe_layer_forward
        import moe_ops_b200 as M

        w_, idx = M.fused_topk_softmax(xa.detach() @ full.w_router.detach().t(), K)
        o = moe_layer_forward(xa.detach().cpu().float(), wr.float(), wg.float(), wu.float(),
                              wd.float(), K, E, routing=(w_.cpu().float(), idx.cpu()))
        errs["out_vs_oracle"] = rel(ref, o)
    # Every rank contributes the same entries (a collective over tensors of different sizes
    # would never complete): the oracle entry is rank 0's and reads 0 elsewhere.
    errs.setdefault("out_vs_oracle", 0.0)
    names = sorted(errs)
    t = torch.tensor([errs[n] for n in names] + [0.0 if healthy else 1.0,
                                                 float(_lib.read_device_error())],
                     device=dev, dtype=torch.float64)
    allt = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(allt, t)
    mx = torch.stack(allt).max(0).values.tolist()
    checks = {n: float(f"{v:.3e}") for n, v in zip(names, mx[:len(names)])}
    bad = mx[len(names)] > 0 or mx[len(names) + 1] > 0
    worst = max(checks.values())
    del full, ep
    torch.cuda.empty_cache()
    return {"max_rel_err": float(f"{worst:.3e}"), "ok": bool(worst < tol and not bad),
            "tolerance": tol, "checks": checks, "transport": transport,
            "problem": f"{T} tokens/rank, d={d}, E={E}, K={K}, H={H}, bf16",
            "barrier_or_device_error": bool(bad)}


def run_ours(args):
    import torch.distributed as dist

    from moe_ops_b200 import _lib
    from moe_ops_b200.moe_layer import MoELayer, layer_gemm_flops

    world, rank, local = _dist_env()
    if world > 1:
        dist.init_process_group("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = CONFIGS[args.config]
    d, E, K, H = cfg["d_model"], cfg["experts"], cfg["top_k"], cfg["hidden"]
    T = cfg["tokens"] // world if cfg["global_tokens"] else cfg["tokens"]
    if args.experts and args.experts != E:
        # A slice of the config for profiling: fewer experts, tokens scaled to keep the
        # rows per expert.  Not the headline workload; the JSON line says so.
        T = T * args.experts // E
        E = args.experts
        cfg = dict(cfg, workload=cfg["workload"] + f" [slice: E={E}, T={T}]")
    router_std = cfg["router_std"] or d ** -0.5  # None: logits ~ N(0, 1)

    parity = None
    if world == 1:
        layer = MoELayer(d, E, K, H, fp32_routing=cfg["fp32_routing"], device=dev,
                         dtype=torch.bfloat16)
        gen = torch.Generator(device=dev).manual_seed(1234)
        with torch.no_grad():
            for w in (layer.w_gate, layer.w_up, layer.w_down):
                w.normal_(0.0, 0.02, generator=gen)
        layer.fused_permute = args.fused_permute
    else:
        # Expert parallelism: this rank holds E/world experts, the router is replicated.
        from moe_ops_b200.ep import EPMoELayer

        transport = args.ep_transport if args.ep_transport != "auto" else "nvlink"
        args.ep_transport = transport
        # Correctness of the multi-GPU layer, over the same transport, before timing it.
        _progress(f"ep parity check ({transport})")
        parity = ep_parity_check(world, rank, dev, transport)
        _progress(f"ep parity: ok={parity['ok']} max_rel_err={parity['max_rel_err']}")
        if not parity["ok"]:
            if rank == 0:
                print(json.dumps({"metric": METRIC, "error": "ep parity check failed",
                                  "ep_parity": parity}), flush=True)
            dist.destroy_process_group()
            sys.exit(3)
        layer = EPMoELayer(d, E, K, H, fp32_routing=cfg["fp32_routing"], device=dev,
                           dtype=torch.bfloat16)
        layer.transport = transport
        with torch.no_grad():
            gen = torch.Generator(device=dev).manual_seed(1234 + rank)
            for w in (layer.w_gate, layer.w_up, layer.w_down):
                w.normal_(0.0, 0.02, generator=gen)
    with torch.no_grad():
        layer.w_router.normal_(0.0, router_std, generator=torch.Generator(device=dev).manual_seed(4321))
    if cfg["zipf"]:
        cg = torch.Generator().manual_seed(5)
        order = torch.randperm(E, generator=cg)
        expert_rank = torch.empty(E)
        expert_rank[order] = torch.arange(1, E + 1, dtype=torch.float32)
        layer.router_bias = (1.5 * torch.log(1.0 / expert_rank ** 1.2)).to(dev)
    x, grad_out = _make_inputs(dev, T, d, 99 + rank)
    flops_step = layer_gemm_flops(T, K, d, H)

    def step(xin, gin):
        for p in layer.parameters():
            p.grad = None
        xin = xin.detach().requires_grad_(True)
        out = layer(xin)
        out.backward(gin)
        return out, xin

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    _progress("warm-up")
    for _ in range(max(args.warmup, 3)):
        step(x, grad_out)
    barrier()
    torch.cuda.reset_peak_memory_stats(dev)
    _progress("timed region")

    # ------------------------------------------------------------ device-timed region
    sampler = ClockSampler(local)
    sampler.start()
    _lib.gemm_timing = []
    launches0 = _lib.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record()
    for _ in range(args.steps):
        step(x, grad_out)
    ev1.record()
    barrier()
    clocks = sampler.stop()
    ms_total = ev0.elapsed_time(ev1)
    launches = _lib.launch_count - launches0
    timing, _lib.gemm_timing = _lib.gemm_timing, None
    # GEMM time = the union of the launches' [start, end] intervals (launches on two streams
    # may overlap; a plain sum would count the overlap twice).
    if timing:
        ref_ev = timing[0][1]
        spans = sorted((ref_ev.elapsed_time(t[1]), ref_ev.elapsed_time(t[2])) for t in timing)
        gemm_ms, cur_a, cur_b = 0.0, spans[0][0], spans[0][1]
        for a_, b_ in spans[1:]:
            if a_ > cur_b:
                gemm_ms += cur_b - cur_a
                cur_a, cur_b = a_, b_
            else:
                cur_b = max(cur_b, b_)
        gemm_ms += cur_b - cur_a
    else:
        gemm_ms = 0.0
    # The grouped GEMMs' FLOPs from the rows the experts actually computed on: T*K on one
    # GPU; under EP the rows this rank received (the peer transport's GEMM calls are sized
    # for its worst-case buffers, so their nominal row counts would overstate the work).
    live_rows = T * K if world == 1 else layer.local_rows()
    gemm_flops = 9 * 2.0 * live_rows * d * H * args.steps
    # Per-launch roofline time: max(FLOPs / tensor peak, DRAM bytes / copy bandwidth,
    # written bytes / write bandwidth measured now on this GPU), rows scaled to the live ones.
    peaks_, _ = _peaks()
    write_gbs = _write_bandwidth(dev)
    t_roof = 0.0
    nominal = sum(t[3] for t in timing)
    scale = gemm_flops / nominal if nominal else 1.0
    for t in timing:
        flop_s = t[3] * scale / (peaks_.get("bf16_tflops_sustained", 1400.0) * 1e12)
        mem_s = max((t[4] + t[5]) / (peaks_["hbm_gbs"] * 1e9), t[5] / (write_gbs * 1e9))
        t_roof += max(flop_s, mem_s)
    peak_mem_gb = torch.cuda.max_memory_allocated(dev) / 1e9
    eager_ms_total, eager_clocks = ms_total, clocks
    # Per kind of grouped-GEMM launch: ms per step and TFLOP/s over the live rows.
    by_kind = {}
    for t in timing:
        k = by_kind.setdefault(t[0], [0.0, 0.0, 0])
        k[0] += t[1].elapsed_time(t[2])
        k[1] += t[3] * scale
        k[2] += 1
    gemm_kinds = {name: {"launches_per_step": n // args.steps,
                         "ms_per_step": round(ms / args.steps, 4),
                         "tflops": round(fl / (ms * 1e-3) / 1e12, 1)}
                  for name, (ms, fl, n) in sorted(by_kind.items())}
    launches_per_step = launches / args.steps

    # ------------------------------------------------------------ the same step as a CUDA graph
    # One training step (forward and backward) captured once and replayed: the same kernels
    # on the same buffers without the host's per-launch work.  The step has no host sync on
    # one GPU and on the peer-memory transport (whose barriers keep their epochs on the
    # device); the NCCL transport syncs with the host every step, so it runs eager.  Used by
    # default for N > 1 on the peer-memory transport, where a rank's share of the step is
    # short enough for launch overhead to matter.
    use_graph = args.graph == "on" or (args.graph == "auto" and world > 1 and args.ep_transport == "nvlink")
    if use_graph:
        _progress("graph capture")
        static_x = x.detach().clone().requires_grad_(True)
        static_g = grad_out.clone()
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                for p in layer.parameters():
                    p.grad = None
                static_x.grad = None
                layer(static_x).backward(static_g)
        torch.cuda.current_stream(dev).wait_stream(side)
        for p in layer.parameters():
            p.grad = None
        static_x.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_out = layer(static_x)
            static_out.backward(static_g)
        for _ in range(3):
            graph.replay()
        barrier()
        _progress("graph timed region")
        sampler = ClockSampler(local)
        sampler.start()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        g0.record()
        for _ in range(args.steps):
            graph.replay()
        g1.record()
        barrier()
        clocks = sampler.stop()
        ms_total = g0.elapsed_time(g1)

    # ------------------------------------------------------------ end to end (host buffers)
    # Every step: the activations and the output gradient come from pinned host memory, and
    # the layer output and the input gradient go back to pinned host memory.
    x_host = x.cpu().pin_memory()
    g_host = grad_out.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    gx_host = torch.empty_like(x_host).pin_memory()
    # Device-side staging buffers: the copies from and to the host run on two copy streams
    # and overlap the compute of this step and its neighbours; the compute's own inputs and
    # outputs move to and from the staging buffers with device copies.
    x_stage, g_stage = torch.empty_like(x), torch.empty_like(grad_out)
    out_stage, gx_stage = torch.empty_like(x), torch.empty_like(x)
    if use_graph:
        x_dev, g_dev = static_x, static_g
    else:
        x_dev, g_dev = torch.empty_like(x), torch.empty_like(grad_out)

    h2d = torch.cuda.Stream(device=dev)
    d2h = torch.cuda.Stream(device=dev)

    def h2d_inputs():
        with torch.cuda.stream(h2d):
            x_stage.copy_(x_host, non_blocking=True)
            g_stage.copy_(g_host, non_blocking=True)

    def e2e_step(last):
        main = torch.cuda.current_stream(dev)
        main.wait_stream(h2d)  # this step's inputs have landed in the staging buffers
        with torch.no_grad():
            x_dev.copy_(x_stage)
            g_dev.copy_(g_stage)
        if not last:
            h2d.wait_stream(main)  # the staging buffers are free: next step's inputs
            h2d_inputs()
        if use_graph:
            graph.replay()
            out, gx = static_out, static_x.grad
        else:
            for p in layer.parameters():
                p.grad = None
            xin = x_dev.detach().requires_grad_(True)
            out = layer(xin)
            out.backward(g_dev)
            gx = xin.grad
        main.wait_stream(d2h)  # the previous step's results have left the staging buffers
        with torch.no_grad():
            out_stage.copy_(out.detach())
            gx_stage.copy_(gx)
        d2h.wait_stream(main)
        with torch.cuda.stream(d2h):
            out_host.copy_(out_stage, non_blocking=True)
            gx_host.copy_(gx_stage, non_blocking=True)

    _progress("end-to-end region")
    h2d.wait_stream(torch.cuda.current_stream(dev))
    h2d_inputs()
    e2e_step(last=True)
    torch.cuda.current_stream(dev).wait_stream(d2h)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    # Every step's H2D copy (the first one issued here, each later one during the step
    # before) and D2H copy lie inside the timed region.
    h2d.wait_stream(torch.cuda.current_stream(dev))
    h2d_inputs()
    for i in range(args.steps):
        e2e_step(last=(i == args.steps - 1))
    torch.cuda.current_stream(dev).wait_stream(d2h)  # the last copies back are inside
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # Device-side health after both timed regions: the library's error word (a bounded
    # wait that gave up, a refused slot) and, under EP, the peer barriers' status.
    _progress("health and reduction")
    dev_err = _lib.read_device_error()
    healthy = layer.health_ok() if world > 1 else True

    # max over ranks (times, errors); every rank's live rows
    t = torch.tensor([ms_total, e2e_ms, float(dev_err), 0.0 if healthy else 1.0, peak_mem_gb,
                      eager_ms_total], device=dev, dtype=torch.float64)
    rows_all = [live_rows]
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gath = [None] * world
        dist.all_gather_object(gath, live_rows)
        rows_all = gath
    ms_total, e2e_ms, dev_err, unhealthy, peak_mem_gb, eager_ms_total = t.tolist()
    ms_step = ms_total / args.steps
    value = flops_step * world / (ms_step * 1e-3) / 1e12
    e2e_value = flops_step * world / (e2e_ms / args.steps * 1e-3) / 1e12

    peaks, peak_kind = _peaks()
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
    peak = peaks.get("bf16_tflops_sustained", 1400.0)
    traffic = _traffic_per_launch()
    ep_label = f"ep{world}" if world > 1 else "single"
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if cfg["global_tokens"] else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) random-init weights)",
        "config": {
            "workload": cfg["workload"],
            "model": "moe_layer_swiglu", "global_batch": T * world, "seq_len": 1,
            "parallelism": ep_label,
            "ep_transport": args.ep_transport if world > 1 else None,
            "tokens_per_rank": T,
            "fused_permute": bool(args.fused_permute) if world == 1 else None,
            "l2": "inputs larger than L2 (expert weights 17.3 GB cfg4 / 22.5 GB cfg5 in total), "
                  "no flush",
            "gemm_flops_per_step": flops_step * world,
        },
        "roofline": {
            "bound": "tensor",
            "kernel": "gmm_sm100_kernel (grouped GEMM fwd/dgrad/wgrad, tcgen05)",
            "achieved": round(achieved, 2) if achieved else None,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4) if achieved else None,
            "peak_kind": f"{peak_kind} bf16_tflops_sustained (kernel timed inside a long step)",
            "live_rows_per_rank": rows_all,
            "by_launch_kind": gemm_kinds,
            "gemm_share_of_step": round(gemm_ms / eager_ms_total, 4) if eager_ms_total else None,
            "measured_on": "the eager timed region (per-launch CUDA events cannot be recorded "
                           "inside a CUDA graph); same kernels and buffers as the graph replays"
                           if use_graph else "the timed region",
            "eager_clocks": eager_clocks if use_graph else None,
            "gemm_time_vs_roofline": round(t_roof * 1e3 / gemm_ms, 4) if gemm_ms else None,
            "roofline_note": "achieved = 9 GEMMs x 2*rows*d*H over the rows the experts computed "
                             "on (rank 0's, live_rows_per_rank[0]) / rank 0's GEMM time (the union "
                             "of the launches' CUDA-event intervals); gemm_time_vs_roofline = sum over launches of "
                             "max(FLOP/tensor peak, DRAM bytes/copy BW, written bytes/"
                             f"{write_gbs:.0f} GB/s write BW measured in this run) / GEMM time",
            "traffic": traffic.get("bytes_per_launch") if traffic else None,
            "write_gbs": round(write_gbs, 1),
        },
        "e2e": {
            "value": round(e2e_value, 2), "unit": "TFLOP/s",
            "ms_per_step": round(e2e_ms / args.steps, 4),
            "h2d_bytes_per_step": x.numel() * 2 + grad_out.numel() * 2,
            "d2h_bytes_per_step": out_host.numel() * 2 + gx_host.numel() * 2,
            "note": "per rank and step: activations and output gradient copied in from pinned "
                    "host memory, layer output and input gradient copied back to pinned host "
                    "memory, on two copy streams through device staging buffers so that the "
                    "copies overlap the neighbouring steps' compute; the step runs as `value` "
                    "does (graph replay or eager); the first H2D and the last D2H lie inside "
                    "the timed region",
            "execution": ("CUDA graph replay" if use_graph else "eager"),
        },
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "execution": ("CUDA graph of one fwd+bwd step, replayed" if use_graph else "eager"),
        "eager_ms_per_step": round(eager_ms_total / args.steps, 4),
        "device_error": int(dev_err),
        "peer_barriers_ok": not unhealthy,
        "peak_mem_gb_per_rank": round(peak_mem_gb, 2),
        "clocks": clocks,
    }
    if parity is not None:
        line["ep_parity"] = parity
    if rank == 0 and world == 1 and not args.no_ops and args.config == "cfg4" and not args.experts:
        line["ops"] = ops_block(dev, steps=20, warmup=3)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config == "cfg4":
        line["cpu_baseline"] = cpu_baseline(steps=1, warmup=1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    failed = int(dev_err) != 0 or unhealthy
    if world > 1:
        dist.destroy_process_group()
    if failed:
        sys.exit(4)


def _cfg2_sizes(zipf: bool):
    """BASELINE config 2 group sizes: 16 x 1024, or Zipf(s=1.1) sizes summing to 16384 with
    2 empty experts."""
    if not zipf:
        return [1024] * 16
    w = 1.0 / torch.arange(1, 15).double() ** 1.1
    sizes = (w / w.sum() * 16384).floor().long().tolist()
    sizes[0] += 16384 - sum(sizes)
    return sizes[:7] + [0] + sizes[7:12] + [0] + sizes[12:]


def _reference_triton():
    """The reference package (triton_gmm_ops, installed unchanged into baseline/_ref) for
    timing its own Triton grouped GEMM on this GPU, or None with the reason."""
    path = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "triton_gmm_ops")):
        return None, "baseline/_ref not installed"
    if path not in sys.path:
        sys.path.append(path)
    try:
        import triton_gmm_ops as tg  # noqa: F401
        return tg, None
    except Exception as e:  # noqa: BLE001
        return None, f"import failed: {e}"[:120]


def ops_block(dev, steps=20, warmup=3):
    """Per-op figures on this GPU, beside the library bars BASELINE names
    grouped GEMMs (uniform and Zipf; forward, dgrad, wgrad) with torch's grouped_mm and the
    reference's own Triton grouped GEMM on the same inputs, and the config 3 routing
    primitives.  GEMM inputs are 0.67 GB (> L2); routing ops are captured in CUDA graphs."""
    import moe_ops_b200 as M
    from moe_ops_b200.grouped_gemm_ops import gmm_bwd_B_raw, gmm_dgrad_raw, gmm_fwd_raw

    peaks, kind = _peaks()
    burst = peaks.get("bf16_tflops", 1590.0)
    res = {"peak_kind": f"{kind} bf16_tflops (burst: ops timed alone) / hbm_gbs",
           "bf16_tflops_peak": burst, "hbm_gbs_peak": peaks["hbm_gbs"]}
    tg, why = _reference_triton()
    g = torch.Generator(device=dev).manual_seed(7)
    E, Kd, N = 16, 4096, 4096
    A = torch.randn(16384, Kd, device=dev, generator=g).to(torch.bfloat16)
    B = (torch.randn(E, N, Kd, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    gC = torch.randn(16384, N, device=dev, generator=g).to(torch.bfloat16)
    fl = 2.0 * 16384 * N * Kd
    for name, zipf in (("cfg2_uniform", False), ("cfg2_zipf", True)):
        sizes = _cfg2_sizes(zipf)
        off = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        off[1:] = torch.tensor(sizes, device=dev).cumsum(0).to(torch.int32)
        ends = off[1:].contiguous()
        Bt = B.transpose(1, 2)
        r = {}
        fns = {"fwd": lambda: gmm_fwd_raw(A, B, off, True),
               "dgrad": lambda: gmm_dgrad_raw(gC, B, off, True),
               "wgrad": lambda: gmm_bwd_B_raw(A, B, off, gC, True),
               "torch_grouped_mm_fwd": lambda: torch.nn.functional.grouped_mm(A, Bt, offs=ends),
               "torch_grouped_mm_dgrad": lambda: torch.nn.functional.grouped_mm(gC, B, offs=ends)}
        if tg is not None:
            fns["reference_triton_fwd"] = lambda: tg.grouped_gemm(A, B, off, trans_b=True)
            # its grad_A GEMM (the TMA forward on a transposed weight copy, as its autograd
            # backward runs it, grouped_gemm_ops_sm90.py:228-231) and its weight gradient
            fns["reference_triton_dgrad"] = lambda: torch.ops.tg.gmm_tma_fwd_raw(
                gC, B.transpose(1, 2).contiguous(), off, trans_b=False)
            fns["reference_triton_wgrad"] = lambda: torch.ops.tg.gmm_bwd_B_raw(A, B, off, gC, True)
        for k, fn in fns.items():
            try:
                ms = _time_events(fn, steps, warmup)
            except Exception as e:  # noqa: BLE001
                r[k] = {"error": f"{type(e).__name__}: {e}"[:120]}
                continue
            tf = fl / (ms * 1e-3) / 1e12
            r[k] = {"ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / burst, 4)}
        res[name] = r
    if tg is None:
        res["reference_triton"] = f"not timed: {why}"
    else:
        res["reference_triton"] = "triton_gmm_ops from baseline/_ref, unchanged: grouped_gemm " \
                                  "forward (its sm90+ TMA path, autotuned on first call), its " \
                                  "dgrad as its backward runs it (weight transpose copy + TMA " \
                                  "forward) and its wgrad kernel (tg::gmm_bwd_B_raw)"
    del A, B, gC
    res["cfg3_routing"] = _routing_ops(dev, steps=max(steps, 50), warmup=warmup)
    if tg is not None:
        res["cfg3_routing_reference_triton"] = _routing_ops(dev, steps=max(steps, 50),
                                                            warmup=warmup, impl=tg)
    return res


def _routing_ops(dev, steps, warmup, impl=None):
    """BASELINE config 3 routing primitives (T=8192, d=4096 bf16, E=64, K=2), each captured
    in a CUDA graph and replayed (GPU time only); GB/s of unique bytes and the fraction of
    the measured HBM copy bandwidth.  impl: a module with the reference's API (its own
    Triton kernels, from baseline/_ref) in place of this library."""
    import moe_ops_b200

    M = impl or moe_ops_b200

    peaks, _ = _peaks()
    g = torch.Generator(device=dev).manual_seed(1)
    T, d, E, K = 8192, 4096, 64, 2
    x = torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, device=dev, generator=g)
    w, idx = M.fused_topk_softmax(logits, K)
    perm, rid, off = M.permute(x, idx, E=E)
    prob = w.float()
    gout = torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16)
    row = T * d * 2
    cases = {
        "topk_fwd": (lambda: M.fused_topk_softmax(logits, K), T * E * 4 + T * K * 8),
        "permute": (lambda: M.permute(x, idx, E=E), row * (1 + K) + T * K * 12),
        "unpermute_fwd": (lambda: M.unpermute_forward(perm, rid, prob, T, K), row * (1 + K)),
        "permute_backward": (lambda: M.permute_backward(perm, rid, T, K), row * (1 + K)),
        "unpermute_bwd": (lambda: M.unpermute_backward(gout, perm, rid, prob, T, K), row * (1 + 2 * K)),
    }
    res = {}
    for name, (fn, nbytes) in cases.items():
        try:
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            ms = _time_events(graph.replay, steps, warmup)
        except Exception as e:  # noqa: BLE001  (a reference op that cannot run or be captured)
            torch.cuda.synchronize()
            res[name] = {"error": f"{type(e).__name__}: {e}"[:120]}
            continue
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[name] = {"us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                     "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4), "bytes": nbytes}
    return res


def cpu_baseline(steps: int = 1, warmup: int = 1, sample_experts: int = 8):
    """The reference's PyTorch-native layer (oracle/moe_oracle.moe_layer_forward, the
    per-expert loop of tests/test_moe.py:28-36) on the host cores, bf16, fwd + bwd, on a
    sample: `sample_experts` experts with 256 rows each (T = 128 * sample_experts)."""
    from oracle.moe_oracle import moe_layer_forward

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    d, K, H = CFG["d_model"], CFG["top_k"], CFG["hidden"]
    E = sample_experts
    T = 128 * E
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16)
    go = torch.randn(T, d, generator=g).to(torch.bfloat16)
    wr = (torch.randn(E, d, generator=g) * 0.02).to(torch.bfloat16).requires_grad_(True)
    wg = (torch.randn(E, H, d, generator=g) * 0.02).to(torch.bfloat16).requires_grad_(True)
    wu = (torch.randn(E, H, d, generator=g) * 0.02).to(torch.bfloat16).requires_grad_(True)
    wd = (torch.randn(E, d, H, generator=g) * 0.02).to(torch.bfloat16).requires_grad_(True)

    def step():
        for p in (wr, wg, wu, wd):
            p.grad = None
        xi = x.detach().requires_grad_(True)
        out = moe_layer_forward(xi, wr, wg, wu, wd, K, E)
        out.backward(go)

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    sec = (time.perf_counter() - t0) / steps
    flops = 9 * 2.0 * T * K * d * H
    return {"value": round(flops / sec / 1e12, 4), "unit": "TFLOP/s", "cores": threads,
            "kind": "port", "seconds_per_step": round(sec, 3),
            "sample": f"{E} of 64 experts, T={T} tokens (256 rows/expert as in cfg4), "
                      "d=4096 H=11008 top-2 bf16 fwd+bwd, torch CPU per-expert loop"}


def run_reference(args):
    world, rank, _ = _dist_env()
    if rank != 0:
        return
    # Every step is the bounded sample (8 of 64 experts, ~5 s of CPU work on 8 cores), so
    # the driver's --steps / --warmup are honoured as given.
    steps, warmup = max(1, args.steps), max(3, args.warmup)
    base = cpu_baseline(steps=steps, warmup=warmup, sample_experts=args.cpu_sample_experts)
    ms_step = base["seconds_per_step"] * 1e3
    line = {
        "metric": METRIC, "value": base["value"], "unit": "TFLOP/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(ms_step, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded)", "impl": "reference",
        "config": {"workload": CFG["workload"],
                   "model": "moe_layer_swiglu", "sample": base["sample"]},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _time_events(fn, steps, warmup):
    for _ in range(max(warmup, 3)):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def run_case(args):
    """Single-op cases (one GPU): per-op throughput and roofline fraction, and small
    targets for ncu.  `gmm-*`: one grouped GEMM at cfg4 shapes (256 +- 16 rows per expert,
    d=4096, H=11008) over --experts experts, or cfg2 (--cfg2).  `routing`: the cfg3
    primitives (top-k, permute, unpermute fwd/bwd, permute_backward) on T=8192, d=4096."""
    from moe_ops_b200 import _lib  # noqa: F401
    import moe_ops_b200 as M
    from moe_ops_b200.grouped_gemm_ops import gmm_bwd_B_raw, gmm_dgrad_raw, gmm_fwd_raw

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, kind = _peaks()
    g = torch.Generator(device=dev).manual_seed(7)
    res = {"case": args.case}
    if args.case.startswith("gmm-"):
        op = args.case[4:]
        if args.cfg2:
            E, K, N = 16, 4096, 4096
            sizes = [1024] * 16
        else:
            E, K, N = args.experts or 64, 4096, 11008
            cpu_g = torch.Generator().manual_seed(0)
            sizes = torch.bincount(torch.randint(0, E, (args.rows_per_expert * E,), generator=cpu_g),
                                   minlength=E).tolist()
        Mt = sum(sizes)
        A = torch.randn(Mt, K, device=dev, generator=g).to(torch.bfloat16)
        B = (torch.randn(E, N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        gC = torch.randn(Mt, N, device=dev, generator=g).to(torch.bfloat16)
        off = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        off[1:] = torch.tensor(sizes, device=dev).cumsum(0).to(torch.int32)
        fn = {"fwd": lambda: gmm_fwd_raw(A, B, off, True),
              "dgrad": lambda: gmm_dgrad_raw(gC, B, off, True),
              "wgrad": lambda: gmm_bwd_B_raw(A, B, off, gC, True)}[op]
        ms = _time_events(fn, args.steps, args.warmup)
        tf = 2.0 * Mt * N * K / (ms * 1e-3) / 1e12
        res.update({"config": {"E": E, "rows": Mt, "K": K, "N": N, "cfg2": bool(args.cfg2)},
                    "ms": round(ms, 4), "tflops": round(tf, 1),
                    "frac_of_burst_peak": round(tf / peaks["bf16_tflops"], 4),
                    "peak_kind": kind})
    elif args.case == "hbm-write":
        # DRAM write bandwidth: 16-byte stores over 5.77 GB (one cfg4 weight gradient).
        gbs = _write_bandwidth(dev, nbytes=5768732672, reps=max(args.steps, 1))
        res.update({"GB/s": round(gbs, 1), "bytes": 5768732672,
                    "frac_of_copy_peak": round(gbs / peaks["hbm_gbs"], 4), "peak_kind": kind})
    elif args.case == "routing":
        res.update(_routing_ops(dev, steps=args.steps, warmup=args.warmup))
        res["peak_kind"] = kind
    elif args.case == "ops":
        res.update(ops_block(dev, steps=args.steps, warmup=args.warmup))
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg4",
                    help="layer workload: cfg4 (headline, default; 8192 tokens split over the "
                         "ranks), cfg4-weak (8192 tokens per rank) or cfg5")
    ap.add_argument("--case", default="layer",
                    help="layer (default) | gmm-fwd | gmm-dgrad | gmm-wgrad | routing | ops | hbm-write")
    ap.add_argument("--experts", type=int, default=None,
                    help="gmm-* cases: experts (cfg4 shapes, default 64); layer case: run a "
                         "slice of the config with this many experts (profiling)")
    ap.add_argument("--cfg2", action="store_true", help="gmm-* cases: BASELINE config 2 shapes")
    ap.add_argument("--rows-per-expert", type=int, default=256, help="gmm-* cases: mean rows")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--ep-transport", choices=["auto", "nccl", "nvlink"], default="auto",
                    help="N > 1: dispatch / combine over NVLink peer memory (auto) or as NCCL "
                         "all-to-alls")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ops", action="store_true", help="N = 1: leave out the per-op block")
    ap.add_argument("--fused-permute", action="store_true",
                    help="N = 1: the expert GEMMs gather their rows from x (no permuted copy)")
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="time the step as a replayed CUDA graph (auto: N > 1 on the peer-memory "
                         "transport, where the host's per-launch work would otherwise pace the "
                         "short per-rank steps; one GPU measured no gain; the NCCL transport "
                         "syncs with the host every step)")
    ap.add_argument("--cpu-sample-experts", type=int, default=8,
                    help="experts in the CPU baseline's sample (256 rows each)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.case != "layer":
        run_case(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
