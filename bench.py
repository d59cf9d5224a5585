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
E/N experts and its own 8192 tokens, tokens go to their experts' ranks and back through
NCCL all-to-alls (weak scaling: per-rank work is fixed as N grows).

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
    # BASELINE config 4 (the headline): every rank holds 8192 tokens (weak scaling).
    "cfg4": dict(tokens=8192, d_model=4096, experts=64, top_k=2, hidden=11008, fp32_routing=False,
                 zipf=False, global_tokens=False, router_std=0.02,
                 workload="cfg4 SwiGLU MoE layer fwd+bwd, T=8192 d=4096 E=64 topK=2 H=11008 bf16"),
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


def _make_inputs(dev, T, d, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16)
    go = torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16)
    return x, go


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

    if world == 1:
        layer = MoELayer(d, E, K, H, fp32_routing=cfg["fp32_routing"], device=dev,
                         dtype=torch.bfloat16)
        gen = torch.Generator(device=dev).manual_seed(1234)
        with torch.no_grad():
            for w in (layer.w_gate, layer.w_up, layer.w_down):
                w.normal_(0.0, 0.02, generator=gen)
    else:
        # Expert parallelism: this rank holds E/world experts, the router is replicated.
        from moe_ops_b200.ep import EPMoELayer

        layer = EPMoELayer(d, E, K, H, fp32_routing=cfg["fp32_routing"], device=dev,
                           dtype=torch.bfloat16)
        # auto: peer memory up to 4 ranks, where it has run bit-exact against the single-GPU
        # layer on real GPUs (and measured 6.5 % faster than NCCL on cfg4 at 2 ranks); NCCL
        # at 8 ranks until the peer path has run there.
        layer.transport = (("nvlink" if world <= 4 else "nccl") if args.ep_transport == "auto"
                           else args.ep_transport)
        args.ep_transport = layer.transport
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
        return out

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        step(x, grad_out)
    barrier()

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
    gemm_ms = sum(t[1].elapsed_time(t[2]) for t in timing)
    gemm_flops = sum(t[3] for t in timing)
    # Per-launch roofline time: max(FLOPs / tensor peak, DRAM bytes / copy bandwidth,
    # written bytes / write bandwidth measured now on this GPU).
    peaks_, _ = _peaks()
    write_gbs = _write_bandwidth(dev)
    t_roof = 0.0
    for t in timing:
        flop_s = t[3] / (peaks_.get("bf16_tflops_sustained", 1400.0) * 1e12)
        mem_s = max((t[4] + t[5]) / (peaks_["hbm_gbs"] * 1e9), t[5] / (write_gbs * 1e9))
        t_roof += max(flop_s, mem_s)

    # ------------------------------------------------------------ end to end (host buffers)
    x_host = x.cpu().pin_memory()
    g_host = grad_out.cpu().pin_memory()
    res_host = torch.empty(1, dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)
    g_dev = torch.empty_like(grad_out)

    copy_stream = torch.cuda.Stream(device=dev)

    def e2e_step():
        # The activations are copied on the compute stream (the forward needs them first);
        # the output gradient is copied on a copy stream while the forward runs, and the
        # backward waits for it.  Both copies happen every step.
        main = torch.cuda.current_stream(dev)
        x_dev.copy_(x_host, non_blocking=True)
        copy_stream.wait_stream(main)  # the previous step's backward has read g_dev
        with torch.cuda.stream(copy_stream):
            g_dev.copy_(g_host, non_blocking=True)
        for p in layer.parameters():
            p.grad = None
        xin = x_dev.detach().requires_grad_(True)
        out = layer(xin)
        main.wait_stream(copy_stream)
        out.backward(g_dev)
        res_host.copy_(out.detach().float().sum().reshape(1), non_blocking=True)

    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # max over ranks
    t = torch.tensor([ms_total, e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms = t.tolist()
    ms_step = ms_total / args.steps
    value = flops_step * world / (ms_step * 1e-3) / 1e12
    e2e_value = flops_step * world / (e2e_ms / args.steps * 1e-3) / 1e12

    peaks, peak_kind = _peaks()
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
    peak = peaks.get("bf16_tflops_sustained", 1400.0)
    traffic = _traffic_per_launch()
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
            "parallelism": f"ep{world}" if world > 1 else "single",
            "ep_transport": args.ep_transport if world > 1 else None,
            "tokens_per_rank": T,
            "l2": "inputs larger than L2 (expert weights 17.3 GB cfg4 / 22.5 GB cfg5), no flush",
            "gemm_flops_per_step": flops_step,
        },
        "roofline": {
            "bound": "tensor",
            "kernel": "gmm_sm100_kernel (grouped GEMM fwd/dgrad/wgrad, tcgen05)",
            "achieved": round(achieved, 2) if achieved else None,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4) if achieved else None,
            "peak_kind": f"{peak_kind} bf16_tflops_sustained (kernel timed inside a long step)",
            "gemm_share_of_step": round(gemm_ms / ms_total, 4) if ms_total else None,
            "gemm_time_vs_roofline": round(t_roof * 1e3 / gemm_ms, 4) if gemm_ms else None,
            "roofline_note": "frac = achieved / tensor peak; gemm_time_vs_roofline = sum over "
                             "launches of max(FLOP/tensor peak, DRAM bytes/copy BW, written "
                             f"bytes/{write_gbs:.0f} GB/s write BW measured in this run) / measured GEMM time",
            "traffic": traffic.get("bytes_per_launch") if traffic else None,
            "write_gbs": round(write_gbs, 1),
        },
        "e2e": {
            "value": round(e2e_value, 2), "unit": "TFLOP/s",
            "ms_per_step": round(e2e_ms / args.steps, 4),
            "h2d_bytes_per_step": x.numel() * 2 + grad_out.numel() * 2,
            "d2h_bytes_per_step": 4,
            "note": "pinned host inputs copied every step: activations before the forward, "
                    "the output gradient on a copy stream during the forward",
        },
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config == "cfg4":
        line["cpu_baseline"] = cpu_baseline(steps=1, warmup=1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


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
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded)", "impl": "reference",
        "config": {"workload": "cfg4 SwiGLU MoE layer fwd+bwd, T=8192 d=4096 E=64 topK=2 H=11008 bf16",
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
        for name, (fn, nbytes) in cases.items():
            # Captured in a CUDA graph and replayed: GPU time only (eager timing of these
            # short ops would measure the Python/launch path instead).
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            ms = _time_events(graph.replay, args.steps, args.warmup)
            gbs = nbytes / (ms * 1e-3) / 1e9
            res[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1),
                         "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4), "bytes": nbytes}
        res["peak_kind"] = kind
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg4",
                    help="layer workload: cfg4 (headline, default) or cfg5")
    ap.add_argument("--case", default="layer",
                    help="layer (default) | gmm-fwd | gmm-dgrad | gmm-wgrad | routing | hbm-write")
    ap.add_argument("--experts", type=int, default=None,
                    help="gmm-* cases: experts (cfg4 shapes, default 64); layer case: run a "
                         "slice of the config with this many experts (profiling)")
    ap.add_argument("--cfg2", action="store_true", help="gmm-* cases: BASELINE config 2 shapes")
    ap.add_argument("--rows-per-expert", type=int, default=256, help="gmm-* cases: mean rows")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--ep-transport", choices=["auto", "nccl", "nvlink"], default="auto",
                    help="N > 1: dispatch / combine as NCCL all-to-alls, or over NVLink peer "
                         "memory; auto = nvlink up to 4 ranks, nccl above")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
