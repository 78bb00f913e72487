"""Benchmark of the B200 video self-attention block (LTX-2.3, as served by plugyawn/opengenie).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

One step = one forward of the video self-attention block (AdaZero -> FP8 QKV ->
Q/K RMSNorm + RoPE -> attention -> FP8 out-projection + gated residual) over the
configuration's synthetic inputs (seeded, random-init weights; see
opengenie_b200/synthetic.py).  The metric is the block's attention throughput,
TFLOP/s = 4*L^2*128*32 / t_block, as BASELINE.json defines it; µs per block is
`ms_per_step`.  N > 1 runs one process per GPU (torchrun) with Ulysses head
sharding; `value` is then the whole job's throughput on one block (strong scaling).

Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "video self-attn block µs & TFLOP/s (% BF16 peak) at L=9216, 1/2/4/8 B200"
UNIT = "TFLOP/s"
L2_BYTES = 126 * 1024 * 1024


def attn_flops(L: int, heads: int = 32, d: int = 128) -> float:
    return 4.0 * L * L * d * heads


def fp8_peak() -> tuple[float, str]:
    """Dense FP8 (e4m3) tensor peak: torch._scaled_mm at 8192^3 measured on a B200 of this pool (burst), from
    profiles/fp8_peak.json; without the file, twice the bf16 figure (tcgen05 kind::f8f6f4 runs at twice the
    kind::f16 rate), said so in the peak_kind."""
    path = os.path.join(REPO, "profiles", "fp8_peak.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["fp8_e4m3_tflops"]["burst"]), "measured torch._scaled_mm e4m3 8192^3 (burst)"
    peaks, kind = measured_peaks()
    return 2.0 * peaks["bf16_tflops"], f"2 x {kind} bf16 dense (burst), no FP8 measurement"


def measured_peaks() -> tuple[dict, str]:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks
            self._nvml = None
        self.period = period_s

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM))
                mask = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist.group.WORLD
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local, pg


def barrier(pg):
    if pg is not None:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, pg) -> float:
    if pg is None:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- CPU reference arm
REF_BUDGET_S = 150.0  # wall-clock cap of the reference arm's warm-up + timed blocks


def time_cpu_steps(run, steps: int, warmup: int, budget_s: float) -> tuple[list[float], int]:
    """Runs ``run()`` ``warmup`` untimed times then up to ``steps`` timed times, stopping early once the
    elapsed wall time would pass ``budget_s`` (estimated from the runs so far).  Returns the timed
    durations (s) and the number of warm-up runs done."""
    t_start = time.perf_counter()
    done_warm, times = 0, []
    est = None
    with torch.no_grad():
        for _ in range(max(0, warmup)):
            t0 = time.perf_counter()
            run()
            est = time.perf_counter() - t0
            done_warm += 1
            if time.perf_counter() - t_start + est > budget_s:
                break
        for _ in range(max(1, steps)):
            if times and time.perf_counter() - t_start + (est or 0.0) > budget_s:
                break
            t0 = time.perf_counter()
            run()
            times.append(time.perf_counter() - t0)
            est = times[-1]
    return times, done_warm


def cpu_reference(cfg_name: str, steps: int, warmup: int, budget_s: float = REF_BUDGET_S) -> dict:
    """The reference's algorithm for the block on the host cores (the oracle port), timed on full blocks.

    Input scales are calibrated on the same input the way the GPU arm calibrates them (amax/448 of the
    AdaZero output and of the attention output; one untimed block), then ``warmup`` untimed and up to
    ``steps`` timed blocks run within ``budget_s`` of wall time.  ``steps`` in the result is the number of
    blocks actually timed and ``ms_per_block`` their mean."""
    from oracle import ltx_block_oracle as O
    from opengenie_b200 import synthetic

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    cfg = synthetic.CONFIGS[cfg_name]
    inp = synthetic.make_inputs(cfg, seed=1)
    w = synthetic.make_weights(seed=0)
    ts_view = inp.timestep.reshape(1, cfg.tokens, 6, 4096)
    with torch.no_grad():
        O.video_block_cpu_fp32(inp.x, ts_view, inp.cos, inp.sin, w, calibrate=True)

    def run():
        O.video_block_cpu_fp32(inp.x, ts_view, inp.cos, inp.sin, w)

    times, done_warm = time_cpu_steps(run, steps, warmup, budget_s)
    per_block = statistics.mean(times)
    return {
        "value": attn_flops(cfg.tokens) / per_block / 1e12,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{len(times)} full {cfg_name} block(s) (L={cfg.tokens}) in torch fp32 on the host after "
                  f"{done_warm} untimed, input scales calibrated as on the GPU; mean {per_block * 1e3:.0f} ms/block",
        "ms_per_block": per_block * 1e3,
        "steps": len(times),
        "warmup": done_warm,
    }


def cpu_reference_branch(args, budget_s: float = REF_BUDGET_S) -> dict:
    """The oracle port of the FFN branch, the text cross-attention branch or one layer's video branches on the
    host cores (torch fp32, all threads), timed on full-size inputs (input scales calibrated as the GPU arm
    calibrates them, one untimed run; then ``--warmup`` untimed and up to ``--steps`` timed runs within
    ``budget_s``).  Returns the same metric, unit and FLOP accounting as the GPU arm of that branch, the
    number of runs timed and their mean."""
    from oracle import ltx_block_oracle as O
    from opengenie_b200 import synthetic

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    cfg = synthetic.CONFIGS[args.config]
    L = cfg.tokens
    if args.branch == "ffn":
        inp = synthetic.make_inputs(cfg, seed=1)
        fw = synthetic.make_ffn_weights(seed=0)
        ts_view = inp.timestep.reshape(1, L, 6, 4096)
        with torch.no_grad():
            O.video_ffn_cpu_fp32(inp.x, ts_view, fw, calibrate=True)

        def run():
            O.video_ffn_cpu_fp32(inp.x, ts_view, fw)
        flops, metric, what = ffn_flops(L), FFN_METRIC, "FFN branch"
        workload = f"LTX-2.3 video FFN branch, {args.config}"
    elif args.branch == "text":
        L_ctx = args.context_tokens
        inp = synthetic.make_text_inputs(L, L_ctx, seed=1)
        tw = synthetic.make_text_attention_weights(seed=0)
        ts_view = inp.timestep.reshape(1, L, 9, 4096)
        pts_view = inp.prompt_timestep.reshape(1, L_ctx, 2, 4096)
        with torch.no_grad():
            O.video_text_cross_attention_cpu_fp32(inp.x, ts_view, inp.context, pts_view, tw, calibrate=True)

        def run():
            O.video_text_cross_attention_cpu_fp32(inp.x, ts_view, inp.context, pts_view, tw)
        flops, metric, what = text_flops(L, L_ctx), TEXT_METRIC, f"text cross-attention branch ({L_ctx} context tokens)"
        workload = f"LTX-2.3 video text cross-attention branch, {args.config}"
    else:  # layers: one layer's video branches, scaled by the layer count
        L_ctx = args.context_tokens
        inp = synthetic.make_layer_inputs(cfg, L_ctx, seed=1)
        w, fw = synthetic.make_weights(seed=100), synthetic.make_ffn_weights(seed=200)
        tw = synthetic.make_text_attention_weights(seed=300)
        table = torch.cat([w.scale_shift_table[0:3], fw.scale_shift_table[3:6], tw.scale_shift_table[6:9]]).float()
        w.scale_shift_table = fw.scale_shift_table = tw.scale_shift_table = table  # the layer's one 9-slot table
        ts_view = inp.timestep.reshape(1, L, 9, 4096)
        pts_view = inp.prompt_timestep.reshape(1, L_ctx, 2, 4096)
        with torch.no_grad():
            y0 = O.video_block_cpu_fp32(inp.x, ts_view, inp.cos, inp.sin, w, calibrate=True).to(torch.bfloat16)
            y0 = O.video_text_cross_attention_cpu_fp32(y0, ts_view, inp.context, pts_view, tw,
                                                       calibrate=True).to(torch.bfloat16)
            O.video_ffn_cpu_fp32(y0, ts_view, fw, calibrate=True)

        def run():
            y = O.video_block_cpu_fp32(inp.x, ts_view, inp.cos, inp.sin, w).to(torch.bfloat16)
            y = O.video_text_cross_attention_cpu_fp32(y, ts_view, inp.context, pts_view, tw).to(torch.bfloat16)
            O.video_ffn_cpu_fp32(y, ts_view, fw)
        flops, metric = args.layers * layer_flops(L, L_ctx), layers_metric(args.layers, L, L_ctx)
        what = "layer (self-attention + text cross-attention + FFN)"
        workload = f"LTX-2.3 video DiT layers (self-attention + text cross-attention + FFN), {args.config}"
    times, done_warm = time_cpu_steps(run, args.steps, args.warmup, budget_s)
    per = statistics.mean(times)
    ms = per * 1e3 * (args.layers if args.branch == "layers" else 1)
    sample = (f"{len(times)} full {what} run(s) (L={L}) in torch fp32 on the host after {done_warm} untimed, input "
              f"scales calibrated as on the GPU; mean {per * 1e3:.0f} ms")
    if args.branch == "layers":
        sample += f" per layer, x {args.layers} layers"
    return {"metric": metric, "value": flops / (ms * 1e-3) / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": sample, "ms": ms, "workload": workload, "steps": len(times), "warmup": done_warm}


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.branch != "attention":
        cb = cpu_reference_branch(args)
        line = {
            "metric": cb["metric"], "impl": "reference", "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": cb["steps"], "warmup": cb["warmup"], "ms_per_step": cb["ms"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16/e4m3 (fp32 on CPU)", "data": "synthetic",
            "config": {"workload": cb["workload"], "branch": args.branch},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return
    cb = cpu_reference(args.config, args.steps, args.warmup)
    line = {
        "metric": METRIC, "impl": "reference", "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": cb["steps"], "warmup": cb["warmup"], "ms_per_step": cb["ms_per_block"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16/e4m3 (fp32 on CPU)", "data": "synthetic",
        "config": config_dict(args.config, args.gpus, args.exchange),
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def rope_input(args, cfg, inp, dev):
    """The block's RoPE input: cos/sin generated in the RoPE kernel from the tokens' (t, h, w) positions (the
    default: no cos/sin tables are read), or the [1, 32, L, 64] tables of the reference's interface
    (--rope-tables).  Both hold the same angles (synthetic.rope_tables / synthetic.rope_positions)."""
    from opengenie_b200 import synthetic

    if args.rope_tables:
        return (inp.cos, inp.sin)
    return synthetic.rope_positions(cfg.frames, cfg.grid_h, cfg.grid_w, device=dev)


def config_dict(name: str, n: int, exchange: str = "nvlink") -> dict:
    from opengenie_b200 import synthetic

    cfg = synthetic.CONFIGS[name]
    return {
        "workload": f"LTX-2.3 video self-attention block, {name}",
        "tokens": cfg.tokens, "latent_grid": [cfg.frames, cfg.grid_h, cfg.grid_w], "hidden": 4096, "heads": 32,
        "head_dim": 128, "batch": 1, "qkv_out_proj": "e4m3 per-tensor scales, fp32 accumulate",
        "attention": "bf16, fp32 softmax/accumulate", "per_token_timestep": cfg.per_token_timestep,
        "parallelism": "single GPU" if n == 1 else f"ulysses heads {32 // n}/GPU, {exchange} exchange",
        "l2": "inputs larger than L2 (x 75 MB + weights 67 MB read per block, qkv 226 MB written and re-read)",
    }


# --------------------------------------------------------------------------- the video FFN branch
FFN_METRIC = "video FFN branch µs & TFLOP/s (FP8 projections 4096->16384->4096) at L=9216, 1/2/4/8 B200"


def ffn_flops(L: int, dim: int = 4096, hidden: int = 16384) -> float:
    return 4.0 * L * dim * hidden


def run_ffn(args) -> None:
    """``--branch ffn``: the same layer's video feed-forward branch (sequence-local: at N GPUs each rank
    runs its L/N tokens, no exchange).  Same timing rules as the attention block."""
    from opengenie_b200 import _lib, synthetic
    from opengenie_b200.graphs import StepGraph
    from opengenie_b200.streaming import HostPipeline
    from opengenie_b200.video_ffn import VideoFeedForward
    from oracle import ltx_block_oracle as O

    rank, world, local, pg = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    cfg = synthetic.CONFIGS[args.config]
    L = cfg.tokens
    if L % world:
        raise SystemExit(f"{L} tokens do not split over {world} ranks")
    Ll = L // world
    inp_cpu = synthetic.make_inputs(cfg, seed=1)
    ts_full = inp_cpu.timestep
    x_loc_cpu = inp_cpu.x[:, rank * Ll:(rank + 1) * Ll].contiguous()
    ts_loc_cpu = ts_full[:, rank * Ll:(rank + 1) * Ll]
    x_loc = x_loc_cpu.to(dev)
    ts_loc = (ts_loc_cpu[:, :1].to(dev).expand(ts_loc_cpu.shape) if ts_loc_cpu.stride(1) == 0
              else ts_loc_cpu.contiguous().to(dev))
    ffn = VideoFeedForward(synthetic.make_ffn_weights(seed=0), dev)
    inp_dev = inp_cpu.to(dev)
    ffn.calibrate_input_scales(inp_dev.x, inp_dev.timestep)  # static scales from all L tokens
    del inp_dev
    out_dev = torch.empty_like(x_loc)

    def step():
        ffn(x_loc, ts_loc, out=out_dev)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    run_step = step
    if not args.no_graph:
        graph = StepGraph(step, dev)
        run_step = graph.replay
        for _ in range(2):
            run_step()
        torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    barrier(pg)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            run_step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(pg)
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, pg)

    # e2e: pinned host x in, output back, through the host pipeline
    x_host = x_loc_cpu.pin_memory()
    out_hosts = [torch.empty_like(x_host).pin_memory() for _ in range(2)]
    pipe = HostPipeline(lambda xd, yd: ffn(xd, ts_loc, out=yd), tuple(x_host.shape), x_host.dtype, dev,
                        graphs=not args.no_graph)
    pipe.run([x_host] * 2, out_hosts)
    torch.cuda.synchronize(dev)
    barrier(pg)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pipe.start_after(e0)
    pipe.run([x_host] * args.steps, [out_hosts[i % 2] for i in range(args.steps)])
    pipe.wait_streams(stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(pg)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, pg)

    # dominant kernel: the GELU-epilogue GEMM (4096 -> 16384) timed alone
    from opengenie_b200 import ltx_ops

    w = ffn.w
    xq = ltx_ops.fused_adazero_from_ada_fp8(x_loc, w.norm_eps, w.scale_shift_table, ts_loc, w.proj.input_scale,
                                            shift_index=3, scale_index=4)
    hq = torch.empty((Ll, ffn.hidden), device=dev, dtype=torch.float8_e4m3fn)

    def gemm1():
        ltx_ops.fp8_scaled_mm_gelu_e4m3(xq, w.proj.weight, w.proj.input_scale, w.proj.weight_scale,
                                        w.out.input_scale, bias=w.proj.bias, out=hq)

    for _ in range(args.warmup):
        gemm1()
    torch.cuda.synchronize(dev)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    for _ in range(args.steps):
        gemm1()
    k1.record(stream)
    torch.cuda.synchronize(dev)
    gemm_ms = max_over_ranks(k0.elapsed_time(k1) / args.steps, pg)
    status = _lib.device_status(clear=True)

    if rank == 0:
        peaks, peak_kind = measured_peaks()
        fp8_pk, fp8_kind = fp8_peak()
        g_flops = 2.0 * Ll * 4096 * 16384
        achieved = g_flops / (gemm_ms * 1e-3) / 1e12
        line = {
            "metric": FFN_METRIC, "value": ffn_flops(L) / (ms * 1e-3) / 1e12, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "us_per_block": ms * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 projections, fp32 accumulate",
            "data": "synthetic (seeded inputs, random-init weights)",
            "config": {"workload": f"LTX-2.3 video FFN branch, {args.config}", "tokens": L, "hidden": 4096,
                       "ffn_hidden": 16384, "batch": 1, "per_token_timestep": cfg.per_token_timestep,
                       "parallelism": "single GPU" if world == 1 else f"tokens split over {world} GPUs",
                       "l2": "inputs larger than L2 (x 75 MB + weights 134 MB per branch)",
                       "launch": "eager launches" if args.no_graph else "one CUDA graph replay per step"},
            "roofline": {"bound": "tensor", "kernel": "fp8_gemm_kernel<EPI_GELU_QUANT> (4096 -> 16384, dominant)",
                         "achieved": achieved, "peak": fp8_pk, "unit": "TFLOP/s", "frac": achieved / fp8_pk,
                         "peak_kind": fp8_kind, "algorithmic_flops_per_launch": g_flops,
                         "kernel_ms": gemm_ms, "traffic": None},
            "e2e": {"value": ffn_flops(L) / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": x_host.numel() * 2 * world, "d2h_bytes_per_step": x_host.numel() * 2 * world},
            "gpu_launches": VideoFeedForward.kernel_launches_per_step * args.steps,
            "clocks": clk.summary(), "device_status": status,
        }
        if world == 1 and not args.no_cpu_baseline:
            ts_view = inp_cpu.timestep.reshape(1, L, 6, 4096)
            threads = len(os.sched_getaffinity(0))
            torch.set_num_threads(threads)
            fw_cpu = ffn.w.to("cpu")
            t0 = time.perf_counter()
            with torch.no_grad():
                O.video_ffn_cpu_fp32(inp_cpu.x, ts_view, fw_cpu)
            per = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": ffn_flops(L) / per / 1e12, "unit": UNIT, "cores": threads,
                                    "kind": "port", "sample": f"1 full FFN branch (L={L}) in torch fp32 on the host; "
                                                              f"{per * 1e3:.0f} ms"}
        print(json.dumps(line), flush=True)
    if pg is not None:
        import torch.distributed as dist

        dist.destroy_process_group()


# --------------------------------------------------------------------------- the text cross-attention branch
TEXT_METRIC = ("video text cross-attention branch µs & TFLOP/s (attn2 with cross-attention AdaLN: FP8 projections, "
               "bf16 attention over the prompt context) at L=9216, 1/2/4/8 B200")


def text_flops(L: int, L_ctx: int, dim: int = 4096) -> float:
    """to_q and to_out (2·L·D² each), the context's K/V projections (2·L_ctx·D·2D) and the attention
    (4·L·L_ctx·D)."""
    return 4.0 * L * dim * dim + 4.0 * L_ctx * dim * dim + 4.0 * L * L_ctx * dim


def run_text(args) -> None:
    """``--branch text``: the same layer's video text cross-attention (sequence-local for the video tokens: at
    N GPUs each rank runs its L/N tokens against the whole context, no exchange).  Same timing rules as the
    attention block; the prompt context and its timestep embedding stay resident (they are fixed for all
    steps of a request), the video tokens come from the host in the e2e leg."""
    from opengenie_b200 import _lib, ltx_ops, synthetic
    from opengenie_b200.graphs import StepGraph
    from opengenie_b200.streaming import HostPipeline
    from opengenie_b200.video_text_attention import VideoTextCrossAttention
    from oracle import ltx_block_oracle as O

    rank, world, local, pg = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    cfg = synthetic.CONFIGS[args.config]
    L, L_ctx = cfg.tokens, args.context_tokens
    if L % world:
        raise SystemExit(f"{L} tokens do not split over {world} ranks")
    Ll = L // world
    inp_cpu = synthetic.make_text_inputs(L, L_ctx, seed=1)
    x_loc_cpu = inp_cpu.x[:, rank * Ll:(rank + 1) * Ll].contiguous()
    x_loc = x_loc_cpu.to(dev)
    ts_loc = inp_cpu.timestep[:, :1].to(dev).expand(1, Ll, inp_cpu.timestep.shape[-1])
    context = inp_cpu.context.to(dev)
    pts = inp_cpu.prompt_timestep[:, :1].to(dev).expand(inp_cpu.prompt_timestep.shape)
    br = VideoTextCrossAttention(synthetic.make_text_attention_weights(seed=0), dev)
    inp_dev = inp_cpu.to(dev)
    br.calibrate_input_scales(inp_dev.x, inp_dev.timestep, inp_dev.context, inp_dev.prompt_timestep)  # all L tokens
    del inp_dev
    out_dev = torch.empty_like(x_loc)

    def step():
        br(x_loc, ts_loc, context, pts, out=out_dev)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    run_step = step
    if not args.no_graph:
        graph = StepGraph(step, dev)
        run_step = graph.replay
        for _ in range(2):
            run_step()
        torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    barrier(pg)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            run_step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(pg)
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, pg)

    # e2e: pinned host x in, output back, through the host pipeline
    x_host = x_loc_cpu.pin_memory()
    out_hosts = [torch.empty_like(x_host).pin_memory() for _ in range(2)]
    pipe = HostPipeline(lambda xd, yd: br(xd, ts_loc, context, pts, out=yd), tuple(x_host.shape), x_host.dtype, dev,
                        graphs=not args.no_graph)
    pipe.run([x_host] * 2, out_hosts)
    torch.cuda.synchronize(dev)
    barrier(pg)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pipe.start_after(e0)
    pipe.run([x_host] * args.steps, [out_hosts[i % 2] for i in range(args.steps)])
    pipe.wait_streams(stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(pg)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, pg)

    # the two largest kernels timed alone on the workspace the last step left: the attention over the context
    # and the to_out GEMM with its gated-residual epilogue; the longer one is the roofline kernel
    w = br.w
    D = br.dim
    ws = br.workspace(Ll, L_ctx)
    q, k, v = ws["q"].unsqueeze(0), ws["kv"][:, :D].unsqueeze(0), ws["kv"][:, D:].unsqueeze(0)
    oq = torch.empty_like(ws["oq"])
    y = torch.empty_like(x_loc)

    def attn():
        ltx_ops.attention(q, k, v, br.heads, out=oq, out_e4m3_scale=w.to_out.input_scale)

    def out_gemm():
        ltx_ops.fp8_scaled_mm_residual_gate(ws["oq"], w.to_out.weight, w.to_out.input_scale, w.to_out.weight_scale,
                                            w.to_out.bias, x_loc, w.scale_shift_table, ts_loc, gate_index=8, out=y)

    def time_alone(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for _ in range(args.steps):
            fn()
        k1.record(stream)
        torch.cuda.synchronize(dev)
        return max_over_ranks(k0.elapsed_time(k1) / args.steps, pg)

    attn_ms, gemm_ms = time_alone(attn), time_alone(out_gemm)
    status = _lib.device_status(clear=True)

    if rank == 0:
        peaks, peak_kind = measured_peaks()
        a_flops = 4.0 * Ll * L_ctx * D
        g_flops = 2.0 * Ll * D * D
        if attn_ms >= gemm_ms:
            achieved, peak = a_flops / (attn_ms * 1e-3) / 1e12, peaks["bf16_tflops"]
            roof = {"kernel": f"attn_fwd_kernel<e4m3 out> ({Ll} queries over {L_ctx} keys, dominant)",
                    "peak_kind": f"{peak_kind} bf16 dense (burst)", "algorithmic_flops_per_launch": a_flops,
                    "kernel_ms": attn_ms}
        else:
            fp8_pk, fp8_kind = fp8_peak()
            achieved, peak = g_flops / (gemm_ms * 1e-3) / 1e12, fp8_pk
            roof = {"kernel": "fp8_gemm_kernel<EPI_RESIDUAL> (to_out, dominant)",
                    "peak_kind": fp8_kind, "algorithmic_flops_per_launch": g_flops, "kernel_ms": gemm_ms}
        line = {
            "metric": TEXT_METRIC, "value": text_flops(L, L_ctx) / (ms * 1e-3) / 1e12, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "us_per_block": ms * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "e4m3 projections, bf16 attention, fp32 accumulate",
            "data": "synthetic (seeded inputs, random-init weights)",
            "config": {"workload": f"LTX-2.3 video text cross-attention branch, {args.config}", "tokens": L,
                       "context_tokens": L_ctx, "hidden": D, "heads": br.heads, "batch": 1,
                       "parallelism": ("single GPU" if world == 1 else
                                       f"video tokens split over {world} GPUs, whole context on each"),
                       "l2": "inputs larger than L2 (x 75 MB + weights 67 MB + context 8 MB per branch)",
                       "launch": "eager launches" if args.no_graph else "one CUDA graph replay per step"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None, **roof,
                         "other_kernel_ms": gemm_ms if attn_ms >= gemm_ms else attn_ms},
            "e2e": {"value": text_flops(L, L_ctx) / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": x_host.numel() * 2 * world, "d2h_bytes_per_step": x_host.numel() * 2 * world},
            "gpu_launches": VideoTextCrossAttention.kernel_launches_per_step * args.steps,
            "clocks": clk.summary(), "device_status": status,
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = len(os.sched_getaffinity(0))
            torch.set_num_threads(threads)
            tw_cpu = br.w.to("cpu")
            t0 = time.perf_counter()
            with torch.no_grad():
                O.video_text_cross_attention_cpu_fp32(inp_cpu.x, inp_cpu.timestep.reshape(1, L, 9, D), inp_cpu.context,
                                                      inp_cpu.prompt_timestep.reshape(1, L_ctx, 2, D), tw_cpu)
            per = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": text_flops(L, L_ctx) / per / 1e12, "unit": UNIT, "cores": threads,
                                    "kind": "port", "sample": f"1 full branch (L={L}, {L_ctx} context tokens) in torch "
                                                              f"fp32 on the host; {per * 1e3:.0f} ms"}
        print(json.dumps(line), flush=True)
    if pg is not None:
        import torch.distributed as dist

        dist.destroy_process_group()


# --------------------------------------------------------------------------- a stack of layers
def layers_metric(layers: int, L: int, L_ctx: int) -> str:
    return (f"video branches of {layers} DiT layers (self-attention + text cross-attention over {L_ctx} context "
            f"tokens + FFN) ms per denoising step at L={L}, 1 B200")


def layer_flops(L: int, L_ctx: int) -> float:
    """One layer's video branches: the self-attention (bf16 attention + FP8 Q/K/V and out-projection), the text
    cross-attention and the FFN."""
    return attn_flops(L) + 2.0 * L * 4096 * (3 * 4096 + 4096) + text_flops(L, L_ctx) + ffn_flops(L)


def run_layers(args) -> None:
    """``--branch layers``: the video branches (self-attention, text cross-attention over ``--context-tokens``
    prompt tokens, FFN) of ``--layers`` DiT layers, one denoising step through the stack per timed step,
    captured as one CUDA graph (1 GPU).  Layers cycle through ``--distinct-weights`` random weight sets (every
    layer still holds its own device copy)."""
    from opengenie_b200 import _lib, synthetic
    from opengenie_b200.graphs import StepGraph
    from opengenie_b200.video_layer import VideoLayer, VideoLayerStack

    rank, world, local, pg = dist_setup(args.gpus)
    if world != 1:
        raise SystemExit("--branch layers runs on one GPU")
    dev = torch.device("cuda", local)
    cfg = synthetic.CONFIGS[args.config]
    L = cfg.tokens
    L_ctx = args.context_tokens
    inp = synthetic.make_layer_inputs(cfg, L_ctx, seed=1).to(dev)
    sets = [(synthetic.make_weights(seed=100 + i), synthetic.make_ffn_weights(seed=200 + i),
             synthetic.make_text_attention_weights(seed=300 + i)) for i in range(max(1, args.distinct_weights))]
    stack = VideoLayerStack([VideoLayer(*sets[i % len(sets)][:2], dev, text_weights=sets[i % len(sets)][2])
                             for i in range(args.layers)])
    pe = rope_input(args, cfg, inp, dev)
    ctx = dict(context=inp.context, prompt_timestep=inp.prompt_timestep)
    stack.calibrate_input_scales(inp.x, inp.timestep, pe, **ctx)
    out = torch.empty_like(inp.x)

    def step():
        stack(inp.x, inp.timestep, pe, out=out, **ctx)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    graph = StepGraph(step, dev)
    graph.replay()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    status = _lib.device_status(clear=True)
    finite = bool(torch.isfinite(out.float()).all())
    per_layer = layer_flops(L, L_ctx)
    line = {
        "metric": layers_metric(args.layers, L, L_ctx),
        "value": args.layers * per_layer / (ms * 1e-3) / 1e12, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "us_per_layer": ms * 1e3 / args.layers, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 attention / e4m3 projections",
        "data": "synthetic (seeded inputs, random-init weights)",
        "config": {"workload": f"LTX-2.3 video DiT layers (self-attention + text cross-attention + FFN), "
                               f"{args.config}", "tokens": L, "context_tokens": L_ctx,
                   "layers": args.layers, "distinct_weight_sets": len(sets),
                   "flops_per_layer": per_layer, "launch": "one CUDA graph replay per step",
                   "scope": "the audio-video cross-attention branch of the layer is not part of this library"},
        "gpu_launches": stack.kernel_launches_per_step * args.steps, "clocks": clk.summary(),
        "device_status": status, "output_finite": finite,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c1_l9216")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="issue each step's launches eagerly")
    ap.add_argument("--exchange", choices=["nvlink", "nccl"], default="nvlink",
                    help="N>1: peer stores over NVLink from the producing kernels, or NCCL all-to-alls")
    ap.add_argument("--phases", action="store_true", help="add a per-stage time breakdown (separate, untimed run)")
    ap.add_argument("--branch", choices=["attention", "ffn", "text", "layers"], default="attention",
                    help="the video self-attention block (the headline), the same layer's video FFN branch or "
                         "text cross-attention branch, or a stack of layers' video branches")
    ap.add_argument("--rope-tables", action="store_true",
                    help="feed the RoPE kernel cos/sin tables (the reference's interface) instead of positions")
    ap.add_argument("--context-tokens", type=int, default=1024, help="--branch text: prompt context tokens")
    ap.add_argument("--layers", type=int, default=48, help="--branch layers: layers in the stack")
    ap.add_argument("--distinct-weights", type=int, default=2, help="--branch layers: random weight sets")
    ap.add_argument("--distinct-input-scales", action="store_true",
                    help="Q, K and V linears with different input scales (a checkpoint calibrated per linear): "
                         "K's and V's are set to 1.25x and 0.8x the calibrated Q scale")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.branch == "ffn" and args.impl == "ours":
        run_ffn(args)
        return
    if args.branch == "text" and args.impl == "ours":
        run_text(args)
        return
    if args.branch == "layers" and args.impl == "ours":
        run_layers(args)
        return

    if args.impl == "reference":
        run_reference_arm(args)
        return

    from opengenie_b200 import _lib, synthetic
    from opengenie_b200.video_block import VideoSelfAttentionBlock

    rank, world, local, pg = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    cfg = synthetic.CONFIGS[args.config]
    L = cfg.tokens
    inp_cpu = synthetic.make_inputs(cfg, seed=1)
    w = synthetic.make_weights(seed=0)
    inp = inp_cpu.to(dev)
    pe = rope_input(args, cfg, inp, dev)

    def distinct_scales(block) -> None:
        bw = block.w
        bw.to_k.input_scale = (bw.to_q.input_scale * 1.25).contiguous()
        bw.to_v.input_scale = (bw.to_q.input_scale * 0.8).contiguous()
        block.input_scales_changed()

    if world == 1:
        blk = VideoSelfAttentionBlock(w, dev)
        blk.calibrate_input_scales(inp.x, inp.timestep, pe)
        if args.distinct_input_scales:
            distinct_scales(blk)
        launches_per_step = 5
        out_dev = torch.empty_like(inp.x)

        def step():
            blk(inp.x, inp.timestep, pe, out=out_dev)
    else:
        from opengenie_b200.ulysses import UlyssesVideoSelfAttention

        blk = UlyssesVideoSelfAttention(w, dev, pg, exchange=args.exchange)
        blk.calibrate_input_scales(inp.x, inp.timestep, pe)
        if args.distinct_input_scales:
            distinct_scales(blk.blk)
        launches_per_step = blk.kernel_launches_per_step
        x_loc = blk.local_slice(inp.x)
        out_dev = torch.empty_like(x_loc)

        def step():
            blk.forward_local(x_loc, inp.timestep, pe, out=out_dev)

    # the step as one CUDA graph replay (NCCL's all-to-alls stay eager)
    use_graph = not args.no_graph and (world == 1 or args.exchange == "nvlink")
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    run_step = step
    if use_graph:
        from opengenie_b200.graphs import StepGraph

        graph = StepGraph(step, dev)
        run_step = graph.replay
        for _ in range(2):
            run_step()
        torch.cuda.synchronize(dev)
    if _lib.device_status(clear=True):
        raise SystemExit("device status reported a timed-out wait during warm-up")

    # ---- device-timed region: K block forwards, inputs resident in HBM
    barrier(pg)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        if world > 1:
            # the ranks leave the host barrier up to milliseconds apart; one untimed step, whose in-graph peer
            # barriers hold every GPU until the last rank arrives, lines the devices up before the start event
            run_step()
        ev0.record(stream)
        for _ in range(args.steps):
            run_step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(pg)
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, pg)
    value = attn_flops(L) / (ms * 1e-3) / 1e12

    # ---- e2e: host x (pinned) -> device, block, device -> host output, every step, through the public
    # API's host pipeline (copy in, compute and copy out of consecutive steps overlap on three streams)
    from opengenie_b200.streaming import HostPipeline

    x_host = (inp_cpu.x if world == 1 else blk.local_slice(inp_cpu.x)).contiguous().pin_memory()
    out_hosts = [torch.empty_like(x_host).pin_memory() for _ in range(2)]
    if world == 1:
        def host_step(xd, yd):
            blk(xd, inp.timestep, pe, out=yd)
    else:
        def host_step(xd, yd):
            blk.forward_local(xd, inp.timestep, pe, out=yd)
    pipe = HostPipeline(host_step, tuple(x_host.shape), x_host.dtype, dev, graphs=use_graph)
    pipe.run([x_host] * 2, out_hosts)  # warm-up
    torch.cuda.synchronize(dev)
    barrier(pg)
    if world > 1:
        # as before the device-timed region: one untimed step, held by its in-graph peer barriers until the
        # last rank arrives, lines the GPUs up before the start event
        pipe.run([x_host], [out_hosts[0]])
        pipe.wait_streams(stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pipe.start_after(e0)
    pipe.run([x_host] * args.steps, [out_hosts[i % 2] for i in range(args.steps)])
    pipe.wait_streams(stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(pg)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, pg)
    h2d = x_host.numel() * x_host.element_size()
    d2h = out_hosts[0].numel() * out_hosts[0].element_size()

    # ---- dominant kernel (attention) timed alone on the launching stream
    attn_ms = blk.time_attention(args.steps, args.warmup) if hasattr(blk, "time_attention") else None
    attn_ms = max_over_ranks(attn_ms, pg) if attn_ms is not None else None
    phases = None
    if args.phases and hasattr(blk, "time_stages"):
        # each stage replayed alone from a CUDA graph (device time, max over ranks); NVLink exchange only
        stage_ms = blk.time_stages(x_loc, inp.timestep, pe, args.steps, args.warmup)
        phases = {name: max_over_ranks(ms_, pg) for name, ms_ in stage_ms.items()} or None
    status = _lib.device_status(clear=True)

    if rank == 0:
        peaks, peak_kind = measured_peaks()
        heads_local = 32 // world
        attn_unit_flops = attn_flops(L, heads=heads_local)
        achieved = attn_unit_flops / (attn_ms * 1e-3) / 1e12 if attn_ms else None
        traffic = None
        tpath = os.path.join(REPO, "profiles", "fmha_traffic.json")
        if os.path.exists(tpath):
            with open(tpath) as f:
                t = json.load(f)
            # bytes per (head, 256-query block) CTA scale with L: K/V re-reads per query block
            traffic = t.get("bytes_per_launch", {}).get(f"{args.config}_h{heads_local}")
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "us_per_block": ms * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16 attention / e4m3 projections",
            "data": "synthetic (seeded inputs, random-init weights)", "config": config_dict(args.config, world, args.exchange),
            "launch": "one CUDA graph replay per step" if use_graph else "eager launches",
            "qkv_input_scales": ("distinct per linear (three e4m3 copies from one AdaZero, one GEMM over the planes)"
                                 if args.distinct_input_scales else "one shared scale"),
            "rope": ("cos/sin tables [1, 32, L, 64] read by the RoPE kernel" if args.rope_tables else
                     "cos/sin generated in the RoPE kernel from the tokens' (t, h, w) positions"),
            "roofline": {
                "bound": "tensor", "kernel": "attn_fwd_kernel (attention, dominant)",
                "achieved": achieved, "peak": peaks.get("bf16_tflops"), "unit": "TFLOP/s",
                "frac": (achieved / peaks["bf16_tflops"]) if achieved else None,
                "peak_kind": f"{peak_kind} bf16 dense (burst)",
                "algorithmic_flops_per_launch": attn_unit_flops, "kernel_ms": attn_ms, "traffic": traffic,
                "block_frac_of_bf16_peak": value / peaks["bf16_tflops"],
            },
            "e2e": {"value": attn_flops(L) / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
            "device_status": status,
        }
        if phases is not None:
            line["phases_ms"] = phases
            line["phases_method"] = ("each stage of the step replayed alone from a CUDA graph on the buffers of a "
                                     "full step, CUDA events, max over ranks; exchange stages include their barrier")
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_reference(args.config, 3, 1, budget_s=30.0)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    if pg is not None:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
