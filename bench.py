"""Benchmark of the FP8 MoE-layer forward (headline workload: T=32768, H=4096, I=1024, E=128, K=8).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one inference forward of the layer on one batch of synthetic input: router logits
(cuBLAS bf16 GEMM, kept for bit-exact routing as in the reference), then the engine's six
kernels (router top-k + tile histogram, metadata scan, metadata scatter, quantise + pack, up-proj
GEMM + SwiGLU + requant, down-proj GEMM + weighted combine).  Inputs are resident in HBM before
the timed region and larger than L2 (x 268 MB, e4m3 weights 1.6 GB), so no explicit L2 flush.
The timed steps replay a CUDA graph of the forward, as the reference benchmark does
(benchmarks/moe-cute.py:308-331).

Synthetic data (the headline workload's shapes and distributions): x ~ N(0,1) bf16, router/expert weights ~ N(0, 0.02) bf16,
expert weights quantised to e4m3 with 128x128 UE8M0 scales before timing (weight preparation is
not part of the forward).  FLOPs per forward: 6*T*K*H*I (benchmarks/moe-cute.py:281-284).

N > 1 (torchrun): expert parallel.  Each rank keeps T=32768 tokens (weak scaling) and E/N of the
128 experts; one step = router GEMM, dispatch (top-k + e4m3 records per destination rank), NCCL
all-to-all of counts and records, the local expert GEMMs, NCCL all-to-all of the bf16 partial rows
back, and the fp32 combine (sonicmoe.ep).  The step time is the max over ranks.  The expert-parallel
step reads the record counts on the host, so it is timed as eager launches, not a CUDA graph.

--impl reference: the reference's eager CPU path (oracle.layer.reference_port, a line-by-line
restatement of sonicmoe/moe.py:278-360 that reproduces it bit for bit) on the host cores, on a
bounded token sample of the same configuration, reported as tokens/s.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "sonic-moe_b200"))
sys.path.insert(0, ROOT)

METRIC = "FP8 MoE fwd TFLOPS/GPU & tokens/s (T32k,H4096,I1024,E128,K8) at 1/2/4/8 B200"
CFG = dict(T=32768, H=4096, I=1024, E=128, K=8)
HEADLINE_T = CFG["T"]  # --tokens overrides CFG["T"] for smaller profiling cases
CPU_SAMPLE_TOKENS = 2048


def flops_fwd(T, H, I, K):
    return 6.0 * T * K * H * I


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "MEASURED_PEAKS.json"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def committed_traffic():
    """Per-launch DRAM bytes of the GEMM kernels from the committed ncu summary (or None)."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons sampled every 5 ms through NVML on a
    background thread during the timed region."""

    REASONS = {  # NVML clocks-event reason bits
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4,
    }

    def __init__(self, gpu_index, interval=0.005):
        self.gpu = gpu_index
        self.interval = interval
        self.samples = []
        self.max_mhz = None
        self._stop = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.gpu]) if vis else self.gpu
            h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def sample():
                return (pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                        pynvml.nvmlDeviceGetCurrentClocksEventReasons(h),
                        pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0)

            # the first queries after nvmlInit can take a few hundred ms and hold up the CUDA
            # launches of the timed loop if they run during it: take them here, untimed
            sample()
        except Exception:
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(sample())
                except Exception:
                    pass
                time.sleep(self.interval)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *a):
        if self._stop is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        sm = [s[0] for s in self.samples]
        reasons = sorted(n for n, bit in self.REASONS.items() if any(s[1] & bit for s in self.samples))
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "power_w_max": max((s[2] for s in self.samples), default=None)}


def build_ep_workload(dev, rank, world, T, H, I, E, K):
    """This rank's tokens and expert shard.  Router weights and each expert's weights are drawn from
    per-tensor seeds, so every world size builds the same global model."""
    import torch

    from sonicmoe import ops

    g = torch.Generator(device=dev).manual_seed(1111 + rank)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    g.manual_seed(7)
    rw = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    El = E // world
    w1 = torch.empty(El, 2 * I, H, dtype=torch.bfloat16, device=dev)
    w2 = torch.empty(El, H, I, dtype=torch.bfloat16, device=dev)
    for j in range(El):
        g.manual_seed(100003 * (rank * El + j) + 11)
        w1[j] = (torch.randn(2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w2[j] = (torch.randn(H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    return x, rw, ops.weight_prep(w1), ops.weight_prep(w2)


def run_ep(args, rank, world, local_rank, cfg):
    import torch
    import torch.distributed as dist

    from sonicmoe.ep import ExpertParallelMoE

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T, H, I, E, K = cfg["T"], cfg["H"], cfg["I"], cfg["E"], cfg["K"]
    x, rw, w1p, w2p = build_ep_workload(dev, rank, world, T, H, I, E, K)
    moe = ExpertParallelMoE(rw, w1p, w2p, E, K, max_tokens=T, hidden_size=H, chunks=args.ep_chunks,
                            reserve_sms=args.ep_reserve_sms, transport=args.ep_transport)
    for _ in range(args.warmup):
        moe.forward(x)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        ev0.record()
        for _ in range(args.steps):
            moe.forward(x)
        ev1.record()
        torch.cuda.synchronize()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = t.item() / args.steps
    # end to end through the public API with pinned host buffers (copies overlapped with the
    # forward on their own streams, as in the 1-GPU e2e leg)
    from sonicmoe.pipeline import OverlappedHostRunner

    x_host = x.cpu().pin_memory()
    o_host = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    runner = OverlappedHostRunner(lambda xd: moe.forward(xd)[0], (T, H), x.dtype, dev, depth=2)
    steps_e2e = max(3, min(args.steps, 10))
    for _ in range(2):
        runner.submit(x_host, o_host)
    runner.drain()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps_e2e):
        runner.submit(x_host, o_host)
    runner.drain()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps_e2e], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    # NVLink bytes into the busiest rank per forward (records from peers + partial rows back)
    bx = torch.tensor([float(moe.last_exchange["bytes_in"]) if moe.last_exchange else 0.0], device=dev)
    dist.all_reduce(bx, op=dist.ReduceOp.MAX)
    transport, chunks = moe.transport, moe.chunks
    moe.close()
    return {
        "ms_step": ms_step,
        "tokens_per_s": world * T / (ms_step / 1e3),
        "tflops_per_gpu": flops_fwd(T, H, I, K) / (ms_step / 1e3) / 1e12,
        "e2e": {"ms_step": t.item(), "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2},
        "clocks": clk.summary(),
        "nvlink_bytes_in": bx.item(),
        "transport": transport,
        "chunks": chunks,
    }


def build_workload(dev, T, H, I, E, K, seed=1111):
    import torch

    from sonicmoe import ops

    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w1p = ops.weight_prep(w1)
    w2p = ops.weight_prep(w2)
    return x, rw, w1, w2, w1p, w2p


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.nn.functional as F

    from sonicmoe import ops
    from sonicmoe.functional import moe_TC_softmax_topk_layer

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T, H, I, E, K = CFG["T"], CFG["H"], CFG["I"], CFG["E"], CFG["K"]
    x, rw, w1, w2, w1p, w2p = build_workload(dev, T, H, I, E, K, seed=1111 + rank)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    freq = torch.empty(E, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def forward():
        logits = F.linear(x, rw)
        ops.moe_forward(x, logits, w1p, w2p, K, out=out, expert_frequency=freq, err=err)

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            forward()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            forward()
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    if err.item() != 0:
        raise RuntimeError(f"kernel error word {err.item()} during warm-up")

    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        time.sleep(0.02)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
    ms_total = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = t.item()
        dist.barrier()
    assert err.item() == 0, f"kernel error word {err.item()}"
    ms_step = ms_total / args.steps

    # per-stage device times from events captured inside a graph of the staged pipeline
    stage = time_stages(x, rw, w1p, w2p, K, reps=10)

    # end to end through the public API: pinned host input -> device, forward, result -> host
    e2e = time_e2e(x, rw, w1, w2, K, dev, steps=max(3, min(args.steps, 10)))
    if dist is not None:
        t = torch.tensor([e2e["ms_step"]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["ms_step"] = t.item()

    res = {
        "ms_step": ms_step,
        "tokens_per_s": world * T / (ms_step / 1e3),
        "tflops_per_gpu": flops_fwd(T, H, I, K) / (ms_step / 1e3) / 1e12,
        "stage": stage,
        "e2e": e2e,
        "clocks": clk.summary(),
        "weights": (rw, w1, w2),
    }
    del graph
    return res


def run_train(args):
    """One training step of the layer through the public API on one GPU: the training forward of
    ``moe_TC_softmax_topk_layer`` (is_inference_mode_enabled=False, weights requiring grad; the up GEMM
    also stores h) and ``backward`` of a fixed output gradient through the FP8 backward.  The
    expert weights are bumped in place before every step, as an optimiser step would, so their
    e4m3 preparation is part of every step.  Eager steps (autograd), CUDA events around the loop.
    FLOPs per step: 18*T*K*H*I (forward 6, backward 12: dA', dX, dW1, dW2)."""
    import torch

    from sonicmoe.functional import moe_TC_softmax_topk_layer

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, H, I, E, K = args.tokens, CFG["H"], CFG["I"], CFG["E"], CFG["K"]  # --tokens: smaller profiling cases
    g = torch.Generator(device=dev).manual_seed(1111)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16).requires_grad_()
    rw = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16).requires_grad_()
    w1 = (torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16).requires_grad_()
    w2 = (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16).requires_grad_()
    dout = (torch.randn(T, H, generator=g, device=dev) * 0.1).to(torch.bfloat16)

    def step():
        # a new weight version, as after an optimiser step (no data pass: only the version counter)
        torch.autograd.graph.increment_version(w1)
        torch.autograd.graph.increment_version(w2)
        o, _, _ = moe_TC_softmax_topk_layer(x, rw, w1.permute(1, 2, 0), None, w2.permute(1, 2, 0), None, K, None,
                                            is_inference_mode_enabled=False)
        o.backward(dout)
        x.grad = rw.grad = w1.grad = w2.grad = None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if args.profile:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
        return
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    name = "config 2" if T == HEADLINE_T else f"config 2 shapes at T={T}"
    print(json.dumps({"workload": f"{name} training step (forward + FP8 backward), one GPU", "T": T, "H": H, "I": I,
                      "E": E, "K": K, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
                      "tflops": 18.0 * T * K * H * I / (ms / 1e3) / 1e12, "steps": args.steps,
                      "clocks": clk.summary()}))


def run_profile(args, local_rank):
    """Eager forwards only, with the bf16 expert weights freed after preparation (smaller footprint)."""
    import torch
    import torch.nn.functional as F

    from sonicmoe import ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T, H, I, E, K = CFG["T"], CFG["H"], CFG["I"], CFG["E"], CFG["K"]
    x, rw, w1, w2, w1p, w2p = build_workload(dev, T, H, I, E, K)
    del w1, w2
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    freq = torch.empty(E, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(args.warmup + args.steps):
        logits = F.linear(x, rw)
        ops.moe_forward(x, logits, w1p, w2p, K, out=out, expert_frequency=freq, err=err)
    torch.cuda.synchronize()
    assert err.item() == 0, f"kernel error word {err.item()}"


def time_stages(x, rw, w1p, w2p, K, reps):
    """Per-stage device times of the forward: `reps` copies of the staged pipeline (router logits
    + top-k, routing plan, quantise + pack, output memset, up GEMM, down GEMM + combine) captured
    back to back in one CUDA graph, with timing events between the stages.  One replay runs the
    copies as consecutive forwards (the regime of the timed loop); the tensor maps are encoded at
    capture, so no host work sits between the events.  Returns per-stage medians over the copies
    (ms); they add up to the staged step."""
    import torch
    import torch.nn.functional as F

    from sonicmoe import ops

    T, H = x.shape
    E = rw.shape[0]
    err = torch.zeros(1, dtype=torch.int32, device=x.device)
    names = ["route", "plan", "pack", "memset", "up", "down"]
    evs = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(names) + 1)] for _ in range(reps)]
    last = {}

    def staged(ev):
        ev[0].record()
        logits = F.linear(x, rw)
        scores, idx = ops.router_topk(logits, K)
        ev[1].record()
        plan = ops.route_plan(idx, E, err)
        ev[2].record()
        xq, xsf = ops.quant_pack(x, idx, plan)
        ev[3].record()
        out = torch.zeros(T, H, dtype=torch.bfloat16, device=x.device)
        ev[4].record()
        aq, asf = ops.moe_up(xq, xsf, w1p, plan, err)
        ev[5].record()
        ops.moe_down_combine(aq, asf, w2p, plan, scores, T, err, out=out)
        ev[6].record()
        last["n_blocks"] = plan.n_blocks

    stream = torch.cuda.Stream(device=x.device)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        staged(evs[0])
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for ev in evs:  # each copy's buffers are freed before the next: the graph pool reuses them
                staged(ev)
        graph.replay()  # warm
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
    assert err.item() == 0, f"kernel error word {err.item()}"
    res = {f"{n}_ms": statistics.median(ev[i].elapsed_time(ev[i + 1]) for ev in evs) for i, n in enumerate(names)}
    res["staged_step_ms"] = statistics.median(ev[0].elapsed_time(ev[-1]) for ev in evs)
    res["n_blocks"] = int(last["n_blocks"].item())
    del graph
    return res


def time_e2e(x, rw, w1, w2, K, dev, steps):
    """Public-API forward on batches that live in pinned host memory: every step copies its input
    host->device and its output device->host inside the timed region.  The copies run on their own
    streams (sonicmoe.pipeline.OverlappedHostRunner), so step i+1's input copy and step i-1's
    output copy overlap step i's forward."""
    import torch

    from sonicmoe.functional import moe_TC_softmax_topk_layer
    from sonicmoe.pipeline import OverlappedHostRunner

    T, H = x.shape
    x_host = x.cpu().pin_memory()
    o_host = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    w1v, w2v = w1.permute(1, 2, 0), w2.permute(1, 2, 0)

    def fwd(xd):
        o, _, _ = moe_TC_softmax_topk_layer(xd, rw, w1v, None, w2v, None, K, None, is_inference_mode_enabled=True)
        return o

    runner = OverlappedHostRunner(fwd, (T, H), x.dtype, dev, depth=2)
    for _ in range(3):
        runner.submit(x_host, o_host)
    runner.drain()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        runner.submit(x_host, o_host)
    runner.drain()
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    nbytes = x.numel() * x.element_size()
    return {"ms_step": ms, "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": T * H * 2,
            "overlap": "H2D / forward / D2H on three streams, 2 batches in flight"}


def cpu_reference(T_sample, reps, threads=None, weights=None):
    """Reference eager CPU forward (fp32) on T_sample tokens of config 2; returns (tokens/s, cores, sample, sec).

    weights: optional (router_w, w1, w2) device tensors of the GPU run, widened to fp32 on the host,
    so both arms see the same layer; otherwise drawn here from the same distributions.
    """
    import torch

    from oracle.layer import reference_port

    cores = threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    T, H, I, E, K = T_sample, CFG["H"], CFG["I"], CFG["E"], CFG["K"]
    g = torch.Generator().manual_seed(1111)
    if weights is not None:
        rw, w1, w2 = (w.float().cpu() for w in weights)
    else:
        rw = torch.randn(E, H, generator=g).mul_(0.02).bfloat16().float()
        w1 = torch.randn(E, 2 * I, H, generator=g).mul_(0.02).bfloat16().float()
        w2 = torch.randn(E, H, I, generator=g).mul_(0.02).bfloat16().float()
    x = torch.randn(T, H, generator=g).bfloat16().float()
    with torch.no_grad():
        reference_port(x, rw, w1, w2, K)  # warm-up
        times = []
        for _ in range(reps):
            t0 = time.perf_counter()
            reference_port(x, rw, w1, w2, K)
            times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    sample = f"T={T} tokens of config 2 (H={H}, I={I}, E={E}, K={K}), fp32 eager reference path, median of {reps}"
    return T / sec, cores, sample, sec


SIDE_WORKLOADS = {
    # name: (T, H, I, E, K, description)
    "c3": (16384, 2048, 768, 128, 8, "config 3 (Qwen3-style): top-k over softmax + renorm, concatenated w1"),
    "c5_64": (64, 4096, 1536, 128, 8, "config 5 (decode, T=64): Zipf(1.2) routing via moe_general_routing_inputs"),
    "c5_512": (512, 4096, 1536, 128, 8, "config 5 (decode, T=512): Zipf(1.2) routing via moe_general_routing_inputs"),
    "c4": (8192, 7168, 2048, 256, 8, "config 4 (DeepSeek-V3-style layer, one GPU's share of tokens): all 256 experts "
                                     "on one GPU, softmax over top-k"),
}

# configurations the expert-parallel (N > 1) bench runs: tokens per GPU, all E experts sharded over the ranks
EP_WORKLOADS = {
    "c2": dict(CFG, desc="config 2: FP8 MoE forward T=32768 H=4096 I=1024 E=128 K=8 per GPU, SwiGLU, interleaved w1"),
    "c4": dict(T=8192, H=7168, I=2048, E=256, K=8,
               desc="config 4 (DeepSeek-V3-style): T=8192 per GPU, H=7168, I=2048, E=256 sharded over the ranks, K=8"),
}


def run_side_workload(args):
    """One of the benchmark's other configurations on one GPU (not the headline line): the public
    functional call replayed from a CUDA graph.  Config 3 is tensor-bound (TFLOP/s against the
    measured FP8 peak); decode is bound by the expert weight bytes it streams (GB/s against the
    measured HBM copy bandwidth)."""
    import numpy as np
    import torch

    from sonicmoe import ops
    from sonicmoe.functional import moe_general_routing_inputs, moe_TC_softmax_topk_layer

    T, H, I, E, K, desc = SIDE_WORKLOADS[args.workload]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1111)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w1 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=dev)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16, device=dev)
    for e in range(E):  # expert by expert: no fp32 copy of all the weights at once
        w1[e] = (torch.randn(2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w2[e] = (torch.randn(H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w1v, w2v = w1.permute(1, 2, 0), w2.permute(1, 2, 0)
    if args.workload in ("c3", "c4"):
        c3 = args.workload == "c3"

        def forward():
            moe_TC_softmax_topk_layer(x, rw, w1v, None, w2v, None, K, None, is_inference_mode_enabled=True,
                                      is_softmax_over_topk=not c3, norm_topk_probs=c3, concat_layout=c3)
        active = E
    else:
        rs = np.random.RandomState(1111)
        rank = np.empty(E)
        rank[rs.permutation(E)] = np.arange(1, E + 1)
        p = rank ** -1.2
        logits = torch.from_numpy((rs.randn(T, E) + np.log(p / p.sum())).astype(np.float32)).to(dev)
        scores, idx = ops.router_topk(logits, K)  # routed once, outside the timed region
        active = int((torch.bincount(idx.reshape(-1).long(), minlength=E) > 0).sum().item())
        sc = scores.reshape(-1).contiguous()
        tok = torch.arange(T, dtype=torch.int32, device=dev).repeat_interleave(K)
        ex = idx.reshape(-1).to(torch.int32).contiguous()

        def forward():
            moe_general_routing_inputs(x, sc, tok, ex, w1v, None, w2v, None, E, None, is_inference_mode_enabled=True)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            forward()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            forward()
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    peaks, src = measured_peaks()
    line = {"workload": desc, "T": T, "H": H, "I": I, "E": E, "K": K, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
            "steps": args.steps, "clocks": clk.summary()}
    if args.workload in ("c3", "c4"):
        tf = flops_fwd(T, H, I, K) / (ms / 1e3) / 1e12
        line["roofline"] = {"bound": "tensor", "achieved": tf, "peak": 2 * peaks["bf16_tflops"], "unit": "TFLOP/s",
                            "frac": tf / (2 * peaks["bf16_tflops"]), "peak_source": src}
    else:
        # e4m3 weights of the experts the batch touches, plus their 128x128 scale bytes
        wbytes = active * (3 * H * I + 3 * H * I // (128 * 128))
        gbs = wbytes / (ms / 1e3) / 1e9
        line["active_experts"] = active
        line["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                            "frac": gbs / peaks["hbm_gbs"], "traffic_basis": "expert weight bytes per forward",
                            "peak_source": src}
    del graph
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tokens", type=int, default=CFG["T"], help="tokens per GPU (profiling of smaller cases)")
    ap.add_argument("--ep-transport", choices=["p2p", "copy", "nccl", "home"], default=None,
                    help="N>1: expert-parallel transport (default: the layer's)")
    ap.add_argument("--ep-chunks", type=int, default=None,
                    help="N>1: token chunks of the pipelined expert-parallel forward (default: the layer's)")
    ap.add_argument("--ep-reserve-sms", type=int, default=None,
                    help="N>1: SMs the GEMMs leave to the overlapped dispatch/combine (default: the layer's)")
    ap.add_argument("--workload", choices=["c2"] + sorted(SIDE_WORKLOADS), default="c2",
                    help="c2 = the headline configuration (default, the contract line); the others time the "
                         "benchmark's remaining configurations (c4 also expert parallel with --gpus N > 1)")
    ap.add_argument("--train", action="store_true",
                    help="time one GPU's training step (forward + FP8 backward) of config 2 instead of the forward")
    ap.add_argument("--profile", action="store_true",
                    help="only run warmup + steps eager forwards (no graph, baselines or extra timing), "
                         "for ncu captures; prints nothing")
    args = ap.parse_args()
    CFG["T"] = args.tokens
    EP_WORKLOADS["c2"]["T"] = args.tokens
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload != "c2" and (world == 1 or args.workload not in EP_WORKLOADS):
        if rank == 0:
            run_side_workload(args)
        return
    ep_cfg = EP_WORKLOADS[args.workload]
    T, H, I, E, K = ep_cfg["T"], ep_cfg["H"], ep_cfg["I"], ep_cfg["E"], ep_cfg["K"]
    config = {"workload": ep_cfg["desc"],
              "T_per_gpu": T, "H": H, "I": I, "E": E, "K": K, "routing": "softmax_over_topk",
              "l2": "expert weights (e4m3) and activations larger than L2 per step; no flush",
              "timing": "CUDA graph replay of the forward, CUDA events, max over ranks"}

    if args.impl == "reference":
        if rank != 0:
            return
        cores = len(os.sched_getaffinity(0))
        tps, cores, sample, sec = cpu_reference(CPU_SAMPLE_TOKENS, reps=max(1, min(args.steps, 3)), threads=cores)
        line = {"metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                "config": dict(config, parallelism="cpu", sample_tokens=CPU_SAMPLE_TOKENS),
                "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
                "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import datetime

    import torch

    if args.train:
        if rank == 0:
            run_train(args)
        return
    if args.profile:
        run_profile(args, local_rank)
        return

    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if world > 1:
        import torch.distributed as dist

        res = run_ep(args, rank, world, local_rank, ep_cfg)
        dist.barrier()
        dist.destroy_process_group()
        if rank != 0:
            return
        e2e = res["e2e"]
        metric = METRIC if args.workload == "c2" else \
            f"FP8 MoE fwd TFLOPS/GPU & tokens/s (T{T // 1024}k/GPU,H{H},I{I},E{E},K{K}) expert parallel, B200"
        line = {
            "metric": metric, "value": res["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3", "data": "synthetic",
            "config": dict(config, parallelism=f"ep{world}", experts_per_rank=E // world,
                           timing=("eager steps (no host wait: device-side record counts)"
                                   if res["transport"] == "home" and res["chunks"] == 1 else
                                   "eager steps (host reads record counts)") + ", CUDA events, max over ranks"),
            # per chunk: dispatch 6 kernels, expert stage 7, combine 1 (router logits are cuBLAS); home
            # transport per forward: top-k 1, routing plan 3, then per chunk records 5 and up stage 6
            # (one chunk: 7, with the device-side count resolve), down 1
            "tflops_per_gpu": res["tflops_per_gpu"],
            "gpu_launches": (17 if res["transport"] == "home" and res["chunks"] == 1 else
                             5 + 11 * res["chunks"] if res["transport"] == "home" else
                             14 * res["chunks"]) * args.steps,
            "e2e": {"value": world * T / (e2e["ms_step"] / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": e2e["h2d_bytes_per_step"], "d2h_bytes_per_step": e2e["d2h_bytes_per_step"]},
            "clocks": res["clocks"],
        }
        # roofline of a compute + exchange step: the slower of the tensor work at the sustained FP8
        # peak (the step runs back to back for the whole timed region) and the NVLink bytes into the
        # busiest rank at the measured 770 GB/s per direction; frac = that target / measured step
        peaks, peak_src = measured_peaks()
        fp8_sust = 2.0 * float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1590.0)))
        t_tensor = flops_fwd(T, H, I, K) / (fp8_sust * 1e12) * 1e3
        t_link = res["nvlink_bytes_in"] / 770e9 * 1e3
        target = max(t_tensor, t_link)
        line["roofline"] = {
            "bound": "tensor" if t_tensor >= t_link else "nvlink", "achieved": res["tflops_per_gpu"],
            "peak": fp8_sust, "unit": "TFLOP/s", "frac": target / res["ms_step"], "traffic": None,
            "target_ms": target, "tensor_ms": t_tensor, "nvlink_ms": t_link,
            "nvlink_bytes_in_per_rank": res["nvlink_bytes_in"],
            "basis": "fused compute+exchange: target = max(FLOPs / (2 x sustained bf16 of " + peak_src +
                     "), NVLink bytes into the busiest rank / 770 GB/s); frac = target / measured step",
        }
        line["config"]["transport"] = f"{res['transport']}, {res['chunks']} chunk(s)"
        print(json.dumps(line))
        return
    res = run_ours(args, rank, world, local_rank)

    peaks, peak_src = measured_peaks()
    fp8_peak = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    st = res["stage"]
    up_flops = 4.0 * T * K * H * I
    down_flops = 2.0 * T * K * H * I
    up_tflops = up_flops / (st["up_ms"] / 1e3) / 1e12
    down_tflops = down_flops / (st["down_ms"] / 1e3) / 1e12
    traffic = committed_traffic().get("moe_gemm_up_per_launch_bytes")
    cpu = None
    if not args.no_cpu_baseline:
        tps, cores, sample, _ = cpu_reference(CPU_SAMPLE_TOKENS, reps=2, weights=res["weights"])
        cpu = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    e2e = res["e2e"]
    line = {
        "metric": METRIC,
        "value": res["tokens_per_s"],
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": res["ms_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3",
        "data": "synthetic",
        "config": dict(config, parallelism="replicas" if world > 1 else "single"),
        "tflops_per_gpu": res["tflops_per_gpu"],
        "gpu_launches": 6 * args.steps,
        "e2e": {"value": world * T / (e2e["ms_step"] / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": e2e["h2d_bytes_per_step"], "d2h_bytes_per_step": e2e["d2h_bytes_per_step"]},
        "roofline": {"bound": "tensor", "kernel": "moe_gemm_kernel<up> (up-proj GEMM + SwiGLU + requant)",
                     "achieved": up_tflops, "peak": fp8_peak, "unit": "TFLOP/s", "frac": up_tflops / fp8_peak,
                     "traffic": traffic,
                     "peak_source": f"2 x bf16_tflops of {peak_src} (tcgen05 e4m3 rate = 2 x bf16)",
                     "down_kernel_tflops": down_tflops,
                     "stages_ms": {k[:-3]: round(v, 4) for k, v in st.items() if k.endswith("_ms")},
                     "stage_timing": "events between the stages of 10 back-to-back staged forwards captured "
                                     "in one CUDA graph; medians over the copies"},
        "clocks": res["clocks"],
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line))


if __name__ == "__main__":
    main()
