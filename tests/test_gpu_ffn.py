"""GPU parity of the video FFN branch (AdaZero idx 3/4 + quantiser, FP8 GEMM with GELU + quantiser in its
epilogue, FP8 GEMM with bias + gate idx 5 + residual) and of the GELU + quantiser op, through the C ABI."""

import os

import numpy as np
import pytest
import torch

from gpu_util import (O, accum_atol, bf16_ulp, block_tolerance, codes, from_bits, status_clean, to_np, within_ulps)

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("tag", ["bf16", "f16"])
def test_gelu_quant_every_bit_pattern(ogx_lib, tag):
    """Every bf16 / fp16 bit pattern: GELU within one ulp of the reference's CPU GELU (tanhf on the GPU
    against the CPU's tanh) plus |x| * 2^-22 (for x << 0, 1 + tanh(...) cancels and a one-ulp difference
    of tanh near -1 is a large relative change of a tiny result), the codes bit-exact to the torch-path
    quantiser of the kernel's own GELU, and equal to the reference's codes wherever the two GELUs agree."""
    from opengenie_b200 import ltx_ops

    d = np.load(os.path.join(GOLD, "gelu_quant.npz"))
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    dt = torch.bfloat16 if tag == "bf16" else torch.float16
    x = torch.from_numpy(allbits.view(np.int16)).view(dt).reshape(256, 256).cuda()
    ref_gelu_bits = d[f"{tag}_gelu"]
    for s, ref_codes in zip(d[f"{tag}_scales"], d[f"{tag}_codes"]):
        q, gelu = ltx_ops.fused_gelu_tanh_fp8_quantize_e4m3(x, torch.tensor(float(s), device="cuda"), return_gelu=True)
        gbits = gelu.cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1)
        if tag == "bf16":
            g, gref = O.bf16_from_bits(gbits), O.bf16_from_bits(ref_gelu_bits)
        else:
            g, gref = gbits.view(np.float16).astype(np.float32), ref_gelu_bits.view(np.float16).astype(np.float32)
        both_nan = np.isnan(g) & np.isnan(gref)
        finite = ~(np.isnan(g) | np.isnan(gref))
        assert (both_nan | finite).all()
        xf = O.bf16_from_bits(allbits) if tag == "bf16" else allbits.view(np.float16).astype(np.float32)
        with np.errstate(invalid="ignore", over="ignore"):
            ulp = bf16_ulp(gref) if tag == "bf16" else np.maximum(
                np.exp2(np.floor(np.log2(np.maximum(np.abs(gref), 2.0 ** -24))) - 10), 2.0 ** -24)
            ulp = ulp + np.abs(xf) * 2.0 ** -22
            diff = np.where(finite, np.abs(g - gref), 0)
        same_inf = np.isinf(g) & np.isinf(gref) & (np.sign(g) == np.sign(gref))
        assert ((diff <= ulp) | same_inf | both_nan).all()
        got = codes(q).reshape(-1)
        assert np.array_equal(got, O.quantize_e4m3(g, float(s), in_dtype=tag))
        agree = gbits == ref_gelu_bits
        assert np.array_equal(got[agree], ref_codes[agree])
        print(tag, s, "GELU bits equal to the reference on", agree.mean())
    assert status_clean()


def test_gelu_quant_ragged_size_matches_vector_path(ogx_lib):
    from opengenie_b200 import ltx_ops

    x = (torch.randn(1_000_003, device="cuda") * 3).to(torch.bfloat16)
    s = torch.tensor(0.01, device="cuda")
    q = ltx_ops.fused_gelu_tanh_fp8_quantize_e4m3(x, s)
    q8 = ltx_ops.fused_gelu_tanh_fp8_quantize_e4m3(x[:1_000_000].contiguous(), s)
    assert torch.equal(q[:1_000_000].view(torch.uint8), q8.view(torch.uint8))
    _, gelu = ltx_ops.fused_gelu_tanh_fp8_quantize_e4m3(x, s, return_gelu=True)
    assert np.array_equal(codes(q), O.quantize_e4m3(to_np(gelu), 0.01))


@pytest.mark.parametrize("M,N,K", [(300, 1024, 4096), (128, 16384, 4096), (77, 512, 1024)])
def test_gemm_gelu_epilogue_equals_gemm_then_gelu_quant(ogx_lib, M, N, K):
    """The fused epilogue is exactly the bf16 GEMM (+ bias) followed by the GELU + quantiser op."""
    from opengenie_b200 import ltx_ops

    g = torch.Generator(device="cuda").manual_seed(M + N)
    a = (torch.randn((M, K), device="cuda", generator=g) * 64).clamp(-448, 448).to(torch.float8_e4m3fn)
    w = (torch.randn((N, K), device="cuda", generator=g) * 64).clamp(-448, 448).to(torch.float8_e4m3fn)
    sa, sw = torch.tensor(2e-3, device="cuda"), torch.tensor([1e-3], device="cuda")
    bias = (torch.randn((N,), device="cuda", generator=g) * 0.3).to(torch.bfloat16)
    qs = torch.tensor(0.02, device="cuda")
    fused = ltx_ops.fp8_scaled_mm_gelu_e4m3(a, w, sa, sw, qs, bias=bias)
    hidden = ltx_ops.fp8_scaled_mm(a, w, sa, sw, bias=bias)
    two_step = ltx_ops.fused_gelu_tanh_fp8_quantize_e4m3(hidden, qs)
    assert torch.equal(fused.view(torch.uint8), two_step.view(torch.uint8))
    assert status_clean()


def _ffn(seed_w, grid=None, cfg=None, seed_in=0):
    from opengenie_b200 import synthetic
    from opengenie_b200.video_ffn import VideoFeedForward

    cfg = cfg or synthetic.small_config(*grid)
    inp = synthetic.make_inputs(cfg, seed=seed_in)
    ffn = VideoFeedForward(synthetic.make_ffn_weights(seed=seed_w), "cuda")
    return cfg, inp, ffn


@pytest.mark.parametrize("grid", [(1, 2, 8), (2, 6, 25)])
def test_ffn_stage_by_stage_vs_oracle(ogx_lib, grid):
    """Every stage of the fused FFN against the oracle fed the kernel's own input to that stage, and the
    branch's output equal to the composition of those stages."""
    from opengenie_b200 import ltx_ops

    cfg, inp, ffn = _ffn(61, grid=grid, seed_in=62)
    L = cfg.tokens
    dev = inp.to("cuda")
    ffn.calibrate_input_scales(dev.x, dev.timestep)
    w = ffn.w
    out = ffn(dev.x, dev.timestep)
    ts_view = inp.timestep.reshape(1, L, 6, 4096)
    s1, s2 = float(w.proj.input_scale), float(w.out.input_scale)
    # 1. AdaZero idx 3/4 (+ fused quantiser)
    xq, norm = ltx_ops.fused_adazero_from_ada_fp8(dev.x, 1e-6, w.scale_shift_table, dev.timestep, w.proj.input_scale,
                                                  shift_index=3, scale_index=4, return_bf16=True)
    ok, worst = within_ulps(to_np(norm), O.adazero_from_ada(inp.x, 1e-6, w.scale_shift_table.cpu(), ts_view,
                                                            shift_index=3, scale_index=4), ulps=1.0, atol=1e-5)
    assert ok, worst
    assert np.array_equal(codes(xq), O.quantize_e4m3(to_np(norm), s1))
    # 2. proj + bias (bf16 hidden, for the check) and the fused GELU + quantiser epilogue
    hidden = ltx_ops.fp8_scaled_mm(xq, w.proj.weight, w.proj.input_scale, w.proj.weight_scale, bias=w.proj.bias)
    wc = codes(w.proj.weight)
    ref = O.fp8_linear(codes(xq), s1, wc, float(w.proj.weight_scale), w.proj.bias.float().cpu().numpy())
    pre = O.fp8_linear(codes(xq), s1, wc, float(w.proj.weight_scale))
    atol = accum_atol(codes(xq), s1, wc, float(w.proj.weight_scale)) + bf16_ulp(pre).reshape(L, -1)
    ok, worst = within_ulps(to_np(hidden).reshape(L, -1), ref.reshape(L, -1), ulps=1.0, atol=atol)
    assert ok, worst
    hq_fused = ltx_ops.fp8_scaled_mm_gelu_e4m3(xq, w.proj.weight, w.proj.input_scale, w.proj.weight_scale,
                                               w.out.input_scale, bias=w.proj.bias)
    hq, gelu = ltx_ops.fused_gelu_tanh_fp8_quantize_e4m3(hidden, w.out.input_scale, return_gelu=True)
    assert torch.equal(hq_fused.view(torch.uint8), hq.view(torch.uint8))
    ok, worst = within_ulps(to_np(gelu), O.gelu_tanh(to_np(hidden)), ulps=1.0,
                            atol=np.abs(to_np(hidden)) * 2.0 ** -22 + 1e-30)
    assert ok, worst
    assert np.array_equal(codes(hq), O.quantize_e4m3(to_np(gelu), s2))
    # 3. second projection + bias + gate (idx 5) + residual
    y = ltx_ops.fp8_scaled_mm_residual_gate(hq.view(1, L, -1), w.out.weight, w.out.input_scale, w.out.weight_scale,
                                            w.out.bias, dev.x, w.scale_shift_table, dev.timestep, gate_index=5)
    yc = codes(w.out.weight)
    y_ref = O.fp8_linear(codes(hq), s2, yc, float(w.out.weight_scale))
    ref_out = O.residual_gate_bias_from_ada(inp.x, y_ref.reshape(1, L, -1), w.out.bias.float().cpu().numpy(),
                                            w.scale_shift_table.cpu(), ts_view, gate_index=5)
    gate = np.abs(O.ada_value(w.scale_shift_table.cpu(), ts_view, 5, table_is_bf16=False, ts_is_bf16=True))
    yb = O.bias_add_bf16(y_ref, w.out.bias.float().cpu().numpy())
    acc = accum_atol(codes(hq), s2, yc, float(w.out.weight_scale))
    atol = gate * (bf16_ulp(y_ref) + bf16_ulp(yb) + acc.reshape(y_ref.shape)) + bf16_ulp(yb * gate)
    ok, worst = within_ulps(to_np(y), ref_out, ulps=1.0, atol=atol)
    assert ok, worst
    assert torch.equal(out, y)
    assert status_clean()


def test_ffn_stages_vs_reference_golden(ogx_lib):
    """Each GPU stage fed the reference's own input to that stage (golden from its CPU functions)."""
    from opengenie_b200 import ltx_ops, synthetic
    from opengenie_b200.video_ffn import VideoFeedForward

    d = np.load(os.path.join(GOLD, "ffn.npz"))
    inp = synthetic.make_inputs(synthetic.small_config(1, 2, 8), seed=int(d["seed_inputs"]))
    fw = synthetic.make_ffn_weights(seed=int(d["seed_weights"]))
    fw.proj.input_scale = torch.tensor(float(d["s1"]), dtype=torch.float32)
    fw.out.input_scale = torch.tensor(float(d["s2"]), dtype=torch.float32)
    ffn = VideoFeedForward(fw, "cuda")
    w = ffn.w
    xq = torch.from_numpy(d["xq"]).view(torch.float8_e4m3fn).cuda().reshape(16, 4096)
    hidden = ltx_ops.fp8_scaled_mm(xq, w.proj.weight, w.proj.input_scale, w.proj.weight_scale, bias=w.proj.bias)
    tol = block_tolerance(to_np(hidden), O.bf16_from_bits(d["hidden"]).reshape(16, -1))
    assert tol["ok"], tol
    hq_ref = torch.from_numpy(d["hq"]).cuda().view(torch.float8_e4m3fn).reshape(16, -1)
    hq = ltx_ops.fused_gelu_tanh_fp8_quantize_e4m3(from_bits(d["hidden"]).reshape(16, -1), w.out.input_scale)
    assert (codes(hq) == codes(hq_ref)).mean() >= 0.999  # tanhf vs the CPU's tanh: rare one-ulp GELU flips
    ts = inp.timestep[:, :1].cuda().expand(inp.timestep.shape)
    out = ltx_ops.fp8_scaled_mm_residual_gate(hq_ref.view(1, 16, -1), w.out.weight, w.out.input_scale,
                                              w.out.weight_scale, w.out.bias, inp.x.cuda(), w.scale_shift_table, ts,
                                              gate_index=5)
    # K = 16384: CPU _scaled_mm and the tensor cores sum in different orders, so bf16(acc * s) may sit one
    # ulp apart, which the gate and the residual add can carry to two ulps of the output
    tol = block_tolerance(to_np(out), O.bf16_from_bits(d["out"]).reshape(out.shape), ulps=2.0)
    assert tol["ok"], tol
    assert status_clean()


@pytest.mark.parametrize("name", ["c1_l9216", "c2_df_l9216"])
def test_ffn_full_size_vs_fp32_reference_on_gpu(ogx_lib, name):
    """L=9216: the fused FFN branch against the same stages with fp32 matmuls on the dequantised e4m3
    operands (torch on the GPU).  sum|d|/sum|ref| <= 1e-2 and max|d| within 2e-2 plus two bf16 ulps of
    |ref| at 99.99 % of the elements (an e4m3 code flip in the 16384-wide hidden moves an output by
    up to a few ulps)."""
    from opengenie_b200 import synthetic

    cfg = synthetic.CONFIGS[name]
    _, inp, ffn = _ffn(71, cfg=cfg, seed_in=72)
    inp = inp.to("cuda")
    ffn.calibrate_input_scales(inp.x, inp.timestep)
    out = ffn(inp.x, inp.timestep)
    ts_view = inp.timestep.reshape(1, cfg.tokens, 6, 4096)
    with torch.no_grad():
        ref = to_np(O.video_ffn_cpu_fp32(inp.x, ts_view, ffn.w))
    tol = block_tolerance(to_np(out), ref, ulps=2.0)
    d = np.abs(to_np(out).astype(np.float64) - ref)
    within = (d <= 2e-2 + 2.0 * np.abs(ref) * 2.0 ** -7).mean()
    print(name, tol, "within 2e-2 + 2 ulps:", within)
    assert tol["mean_rel"] <= 1e-2, tol
    assert within >= 0.9999, within
    assert status_clean()


def test_ffn_graph_replay_matches_eager(ogx_lib):
    from opengenie_b200.graphs import StepGraph

    cfg, inp, ffn = _ffn(81, grid=(2, 6, 25), seed_in=82)
    dev = inp.to("cuda")
    ffn.calibrate_input_scales(dev.x, dev.timestep)
    out = torch.empty_like(dev.x)
    ffn(dev.x, dev.timestep, out=out)
    g = StepGraph(lambda: ffn(dev.x, dev.timestep, out=out), "cuda")
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ffn(dev.x, dev.timestep))
