"""Times one kernel of the block alone, at any size: a CLI for sweeps and for profiler captures of a
single launch on a small case.

    python -m opengenie_b200.kernel_bench attention --tokens 9216 --heads 4 [--e4m3] [--kv-tokens 1024]
    python -m opengenie_b200.kernel_bench gemm --m 9216 --n 12288 --k 4096 [--residual]
    python -m opengenie_b200.kernel_bench adazero --tokens 9216
    python -m opengenie_b200.kernel_bench rope --tokens 9216 [--positions]
    python -m opengenie_b200.kernel_bench qk_rmsnorm --tokens 9216 --kv-tokens 1024
    python -m opengenie_b200.kernel_bench compare --tokens 9216
    python -m opengenie_b200.kernel_bench fp8_peak

``compare`` times the library kernels a user of the reference would otherwise run on this GPU next to
this library's: torch SDPA on the cuDNN backend (the reference's production ``sdpa-cudnn`` attention) and
torch's flash backend against the attention kernel, and ``torch._scaled_mm`` (the reference's FP8Linear
path) against the FP8 GEMM, at the block's shapes; one JSON line per kernel and a ratio line.
``fp8_peak`` measures the dense FP8 (e4m3) tensor peak as ``torch._scaled_mm`` at 8192^3, as a burst
(best of 10) and sustained (back to back for 4 s), next to the bf16 matmul at the same size.

Prints one JSON line: the average device time of a launch (CUDA events on the launching stream,
after warm-up) and the algorithmic rate (TFLOP/s for the contractions, GB/s of unique bytes for the
memory-bound kernels).  Inputs are seeded random tensors laid out as the block lays them out.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import ltx_ops, synthetic


def _time(fn, steps: int, warmup: int) -> float:
    """Device time per launch: the `steps` launches are captured in one CUDA graph and replayed, so host
    overhead (a few tens of microseconds per eager call) does not hide short kernels.  Consecutive launches
    overlap their set-up as in the block (programmatic dependent launch)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        for _ in range(steps):
            fn()
    graph.replay()  # warm
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def bench_attention(a) -> dict:
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    L, H = a.tokens, a.heads
    L_kv = a.kv_tokens or L
    if a.kv_tokens:
        # text cross-attention: q [L][H*128] from to_q, k/v the halves of the packed [L_kv][2][H*128] rows
        q = torch.randn((1, L, H * 128), device="cuda", generator=g).to(torch.bfloat16)
        kv = torch.randn((L_kv, 2 * H * 128), device="cuda", generator=g).to(torch.bfloat16)
        k, v = kv[:, :H * 128].unsqueeze(0), kv[:, H * 128:].unsqueeze(0)
    else:
        # packed [L][3][H*128] rows, as the QKV projection leaves them
        qkv = torch.randn((L, 3 * H * 128), device="cuda", generator=g).to(torch.bfloat16)
        q, k, v = (qkv[:, i * H * 128:(i + 1) * H * 128].unsqueeze(0) for i in range(3))
    if a.e4m3:
        out = torch.empty((1, L, H * 128), device="cuda", dtype=torch.float8_e4m3fn)
        scale = torch.tensor(0.01, device="cuda")
        fn = lambda: ltx_ops.attention(q, k, v, H, out=out, out_e4m3_scale=scale)  # noqa: E731
    else:
        out = torch.empty((1, L, H * 128), device="cuda", dtype=torch.bfloat16)
        fn = lambda: ltx_ops.attention(q, k, v, H, out=out)  # noqa: E731
    ms = _time(fn, a.steps, a.warmup)
    flops = 4.0 * L * L_kv * 128 * H
    return {"kernel": "attn_fwd_kernel", "tokens": L, "kv_tokens": L_kv, "heads": H, "e4m3_out": a.e4m3, "ms": ms,
            "tflops": flops / (ms * 1e-3) / 1e12}


def bench_gemm(a) -> dict:
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    M, N, K = a.m, a.n, a.k
    xq = (torch.randn((M, K), device="cuda", generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    w = (torch.randn((N, K), device="cuda", generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    s_in = torch.tensor(1e-3, device="cuda")
    s_w = torch.full((1,), 1e-3, device="cuda")
    bias = (torch.randn((N,), device="cuda", generator=g) * 0.01).to(torch.bfloat16)
    if a.residual:
        x = torch.randn((1, M, N), device="cuda", generator=g).to(torch.bfloat16)
        table = torch.randn((6, N), device="cuda", generator=g) * 0.02
        ts = torch.randn((1, 1, 6 * N), device="cuda", generator=g).to(torch.bfloat16).expand(1, M, 6 * N)
        fn = lambda: ltx_ops.fp8_scaled_mm_residual_gate(xq.view(1, M, K), w, s_in, s_w, bias, x, table, ts,  # noqa: E731
                                                         gate_index=2)
    else:
        out = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
        fn = lambda: ltx_ops.fp8_scaled_mm(xq, w, s_in, s_w, bias=bias, out=out)  # noqa: E731
    ms = _time(fn, a.steps, a.warmup)
    return {"kernel": "fp8_gemm_kernel", "m": M, "n": N, "k": K, "residual_epilogue": a.residual, "ms": ms,
            "tflops": 2.0 * M * N * K / (ms * 1e-3) / 1e12}


def bench_adazero(a) -> dict:
    cfg = synthetic.small_config(1, 1, a.tokens)
    inp = synthetic.make_inputs(cfg, seed=a.seed).to("cuda")
    w = synthetic.make_weights(seed=a.seed + 1).to("cuda")
    s = torch.tensor(0.01, device="cuda")
    fn = lambda: ltx_ops.fused_adazero_from_ada_fp8(inp.x, 1e-6, w.scale_shift_table, inp.timestep, s,  # noqa: E731
                                                    shift_index=0, scale_index=1)
    ms = _time(fn, a.steps, a.warmup)
    nbytes = a.tokens * 4096 * 3  # bf16 x read + e4m3 write (the uniform timestep rows stay in cache)
    return {"kernel": "adazero_ring_kernel", "tokens": a.tokens, "ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9}


def bench_rope(a) -> dict:
    cfg = synthetic.small_config(1, 1, a.tokens)
    inp = synthetic.make_inputs(cfg, seed=a.seed).to("cuda")
    w = synthetic.make_weights(seed=a.seed + 1).to("cuda")
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    qkv = torch.randn((a.tokens, 3 * 4096), device="cuda", generator=g).to(torch.bfloat16)
    q, k = qkv[:, :4096].unsqueeze(0), qkv[:, 4096:8192].unsqueeze(0)
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    nbytes = a.tokens * 4096 * 2 * 4  # q, k read + written
    if a.positions:
        # cos/sin generated from positions of an LTX-like raster (18 x 32 latent grid per frame)
        pos = synthetic.rope_positions((a.tokens + 575) // 576, 18, 32, device="cuda")
        fn = lambda: ltx_ops.fused_video_qk_rmsnorm_rope_positions(  # noqa: E731
            q, k, w.q_norm_weight, w.k_norm_weight, 1e-6, pos, out=(qo, ko))
    else:
        fn = lambda: ltx_ops.fused_video_qk_rmsnorm_rope(q, k, w.q_norm_weight, w.k_norm_weight, 1e-6,  # noqa: E731
                                                         inp.cos, inp.sin, out=(qo, ko))
        nbytes += 2 * a.tokens * 32 * 64 * inp.cos.element_size()  # cos, sin read
    ms = _time(fn, a.steps, a.warmup)
    return {"kernel": "qk_rmsnorm_rope_ring_kernel", "tokens": a.tokens, "cos_sin": "generated" if a.positions else
            "tables", "ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9}


def bench_qk_rmsnorm(a) -> dict:
    """Q/K RMSNorm without RoPE (the text cross-attention), in place on q [L, 4096] and the K half of a packed
    [L_kv, 2*4096] K/V buffer, as the branch runs it."""
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    L_kv = a.kv_tokens or a.tokens
    q = torch.randn((1, a.tokens, 4096), device="cuda", generator=g).to(torch.bfloat16)
    kv = torch.randn((L_kv, 8192), device="cuda", generator=g).to(torch.bfloat16)
    k = kv[:, :4096].unsqueeze(0)
    qw = (1 + 0.1 * torch.randn((4096,), device="cuda", generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn((4096,), device="cuda", generator=g)).to(torch.bfloat16)
    fn = lambda: ltx_ops.fused_qk_rmsnorm(q, k, qw, kw, 1e-6, out=(q, k))  # noqa: E731
    ms = _time(fn, a.steps, a.warmup)
    nbytes = (a.tokens + L_kv) * 4096 * 2 * 2  # rows read + written
    return {"kernel": "qk_rmsnorm_ring_kernel", "tokens": a.tokens, "kv_tokens": L_kv, "ms": ms,
            "gbs": nbytes / (ms * 1e-3) / 1e9}


def _time_eager(fn, steps: int, warmup: int) -> float:
    """Device time per call of a library function, CUDA events around ``steps`` eager calls (the call's
    own host work included, as a user of the reference pays it)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _sdpa_backend_call(backend):
    """The reference's SDPA attention backend: q/k/v [B, L, H*d] viewed [B, L, H, d], transposed to
    [B, H, L, d] for torch SDPA on one backend, and the output brought back to [B, L, H*d]."""
    from torch.nn.attention import sdpa_kernel

    def call(q, k, v, heads):
        b, L, hd = q.shape
        d = hd // heads
        qh, kh, vh = (t.view(b, -1, heads, d).transpose(1, 2) for t in (q, k, v))
        with sdpa_kernel([backend]):
            o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)
        return o.transpose(1, 2).reshape(b, L, hd)
    return call


def bench_compare(a) -> list[dict]:
    """This library's attention and FP8 GEMM next to the library kernels the reference would run here."""
    from torch.nn.attention import SDPBackend

    g = torch.Generator(device="cuda").manual_seed(a.seed)
    L, H = a.tokens, a.heads
    qkv = torch.randn((L, 3 * H * 128), device="cuda", generator=g).to(torch.bfloat16)
    q, k, v = (qkv[:, i * H * 128:(i + 1) * H * 128].unsqueeze(0) for i in range(3))
    flops = 4.0 * L * L * 128 * H
    rows = []
    out = torch.empty((1, L, H * 128), device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: ltx_ops.attention(q, k, v, H, out=out), a.steps, a.warmup)
    ours_attn = ms
    rows.append({"op": "attention", "impl": "ogx attn_fwd_kernel (bf16 out)", "tokens": L, "heads": H, "ms": ms,
                 "tflops": flops / (ms * 1e-3) / 1e12})
    for name, be in (("torch sdpa, cuDNN backend (the reference's sdpa-cudnn)", SDPBackend.CUDNN_ATTENTION),
                     ("torch sdpa, flash backend", SDPBackend.FLASH_ATTENTION)):
        call = _sdpa_backend_call(be)
        try:
            ms = _time_eager(lambda: call(q, k, v, H), a.steps, a.warmup)
            ref = call(q, k, v, H)
            d = (ref.float() - out.float()).abs()
            rows.append({"op": "attention", "impl": name, "tokens": L, "heads": H, "ms": ms,
                         "tflops": flops / (ms * 1e-3) / 1e12, "ours_speedup": ms / ours_attn,
                         "max_abs_vs_ours": float(d.max())})
        except Exception as e:  # backend not available for this GPU / build
            rows.append({"op": "attention", "impl": name, "unavailable": f"{type(e).__name__}: {e}"[:200]})

    for (M, N, K) in ((L, 3 * 4096, 4096), (L, 4096, 4096), (L, 16384, 4096)):
        xq = (torch.randn((M, K), device="cuda", generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
        w = (torch.randn((N, K), device="cuda", generator=g) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
        s_in = torch.tensor(1e-3, device="cuda")
        s_w = torch.full((1,), 1e-3, device="cuda")
        bias = (torch.randn((N,), device="cuda", generator=g) * 0.01).to(torch.bfloat16)
        o = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
        ms_ours = _time(lambda: ltx_ops.fp8_scaled_mm(xq, w, s_in, s_w, bias=bias, out=o), a.steps, a.warmup)
        f = 2.0 * M * N * K
        rows.append({"op": "fp8 linear + bias", "impl": "ogx fp8_gemm_kernel", "m": M, "n": N, "k": K, "ms": ms_ours,
                     "tflops": f / (ms_ours * 1e-3) / 1e12})
        sw0 = s_w.reshape(())
        wt = w.t()
        try:
            ms = _time_eager(lambda: torch._scaled_mm(xq, wt, scale_a=s_in, scale_b=sw0, bias=bias,
                                                     out_dtype=torch.bfloat16, use_fast_accum=True), a.steps, a.warmup)
            rows.append({"op": "fp8 linear + bias", "impl": "torch._scaled_mm (the reference's FP8Linear path)",
                         "m": M, "n": N, "k": K, "ms": ms, "tflops": f / (ms * 1e-3) / 1e12,
                         "ours_speedup": ms / ms_ours})
        except Exception as e:
            rows.append({"op": "fp8 linear + bias", "impl": "torch._scaled_mm", "unavailable": str(e)[:200]})
    return rows


def bench_fp8_peak(a) -> dict:
    """Dense FP8 (e4m3 x e4m3 -> bf16) and bf16 tensor throughput of torch's library GEMMs at 8192^3."""
    import time

    n = 8192
    g = torch.Generator(device="cuda").manual_seed(a.seed)
    x8 = (torch.randn((n, n), device="cuda", generator=g) * 50).clamp(-448, 448).to(torch.float8_e4m3fn)
    w8 = (torch.randn((n, n), device="cuda", generator=g) * 50).clamp(-448, 448).to(torch.float8_e4m3fn).t()
    one = torch.tensor(1.0, device="cuda")
    xb = torch.randn((n, n), device="cuda", generator=g).to(torch.bfloat16)
    wb = torch.randn((n, n), device="cuda", generator=g).to(torch.bfloat16)
    flops = 2.0 * n ** 3
    res = {"size": n}
    for name, fn in (("fp8_e4m3", lambda: torch._scaled_mm(x8, w8, scale_a=one, scale_b=one, out_dtype=torch.bfloat16,
                                                           use_fast_accum=True)),
                     ("bf16", lambda: torch.matmul(xb, wb))):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        # sustained: back to back for about 4 s
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(1, int(4000.0 / best))
        t0 = time.perf_counter()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        res[name] = {"burst_tflops": flops / (best * 1e-3) / 1e12,
                     "sustained_tflops": flops * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12,
                     "sustained_s": wall, "reps": reps}
    return res


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("kernel", choices=["attention", "gemm", "adazero", "rope", "qk_rmsnorm", "compare", "fp8_peak"])
    ap.add_argument("--tokens", type=int, default=9216)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--e4m3", action="store_true")
    ap.add_argument("--kv-tokens", type=int, default=0,
                    help="attention / qk_rmsnorm: keys from a sequence of this length")
    ap.add_argument("--m", type=int, default=9216)
    ap.add_argument("--n", type=int, default=12288)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--residual", action="store_true")
    ap.add_argument("--positions", action="store_true", help="rope: generate cos/sin from positions")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    fn = {"attention": bench_attention, "gemm": bench_gemm, "adazero": bench_adazero, "rope": bench_rope,
          "qk_rmsnorm": bench_qk_rmsnorm, "compare": bench_compare, "fp8_peak": bench_fp8_peak}[a.kernel]
    res = fn(a)
    for row in (res if isinstance(res, list) else [res]):
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
