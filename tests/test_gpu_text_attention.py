"""GPU parity of the text cross-attention: attention over keys of another length, Q/K RMSNorm without RoPE,
and the fused branch (attn2 with cross-attention AdaLN, eight launches through the C ABI) against the
oracle, stage by stage and at full size."""

import os

import numpy as np
import pytest
import torch

from gpu_util import O, accum_atol, bf16_ulp, block_tolerance, codes, from_bits, status_clean, to_np, within_ulps

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ops(ogx_lib):
    from opengenie_b200 import ltx_ops

    return ltx_ops


def _qkv(B, L, L_kv, H, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, L, H * 128), generator=g).to(torch.bfloat16)
    k = torch.randn((B, L_kv, H * 128), generator=g).to(torch.bfloat16)
    v = torch.randn((B, L_kv, H * 128), generator=g).to(torch.bfloat16)
    return q, k, v


@pytest.mark.parametrize("B,L,L_kv,H", [(1, 300, 77, 2), (1, 128, 1, 1), (2, 200, 64, 2), (1, 1, 130, 1),
                                        (1, 256, 1024, 2), (1, 17, 500, 3)])
def test_attention_keys_of_another_length_vs_oracle(ops, B, L, L_kv, H):
    q, k, v = _qkv(B, L, L_kv, H, seed=L + 7 * L_kv + H)
    out = ops.attention(q.cuda(), k.cuda(), v.cuda(), H)
    assert out.shape == (B, L, H * 128)
    tol = block_tolerance(to_np(out), O.attention(q, k, v, H))
    assert tol["ok"], tol
    assert status_clean()


def test_attention_key_length_entry_equals_self_attention_entry(ops):
    """Equal lengths with k/v strided unlike q take the key-length entry point; bit-equal to the
    self-attention entry point on copies sharing q's strides, and its e4m3 epilogue equals the quantiser
    on its bf16 output."""
    q, k, v = _qkv(1, 300, 300, 2, seed=5)
    q = q.cuda()
    kv = torch.cat([k, v], dim=-1).cuda()
    k2, v2 = kv[..., :256], kv[..., 256:]
    a = ops.attention(q, k2, v2, 2)
    b = ops.attention(q, k.cuda(), v.cuda(), 2)
    assert torch.equal(a, b)
    s = torch.tensor(0.005, device="cuda")
    oq = ops.attention(q, k2, v2, 2, out_e4m3_scale=s)
    assert np.array_equal(codes(oq), codes(ops.fused_fp8_quantize_e4m3(a, s)))
    assert status_clean()


def test_qk_rmsnorm_vs_oracle_and_rope_with_unit_rotation(ops):
    g = torch.Generator().manual_seed(12)
    q = torch.randn((1, 37, 4096), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 11, 4096), generator=g).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn((4096,), generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn((4096,), generator=g)).to(torch.bfloat16)
    qd, kd, qwd, kwd = q.cuda(), k.cuda(), qw.cuda(), kw.cuda()
    qn, kn = ops.fused_qk_rmsnorm(qd, kd, qwd, kwd, 1e-6)
    for got, x, w in ((qn, q, qw), (kn, k, kw)):
        ok, worst = within_ulps(to_np(got), O.qk_rmsnorm(x, w, 1e-6), ulps=1.0, atol=1e-6)
        assert ok, worst
    # equal lengths: bit-equal to the RoPE kernel with cos = 1, sin = 0
    k37 = torch.randn((1, 37, 4096), generator=g).to(torch.bfloat16).cuda()
    cos = torch.ones((1, 32, 37, 64), device="cuda", dtype=torch.bfloat16)
    sin = torch.zeros((1, 32, 37, 64), device="cuda", dtype=torch.bfloat16)
    rq, rk = ops.fused_video_qk_rmsnorm_rope(qd, k37, qwd, kwd, 1e-6, cos, sin)
    qn2, kn2 = ops.fused_qk_rmsnorm(qd, k37, qwd, kwd, 1e-6)
    assert torch.equal(rq, qn2) and torch.equal(rk, kn2)
    # in place on strided rows (the K half of a packed K/V buffer) with fp32 weights
    kv = torch.randn((11, 8192), generator=g).to(torch.bfloat16).cuda()
    k_view = kv[:, :4096].unsqueeze(0)
    ref_k = O.qk_rmsnorm(to_np(k_view), kw.float(), 1e-6)
    v_before = kv[:, 4096:].clone()
    ops.fused_qk_rmsnorm(qd, k_view, qwd.float(), kwd.float(), 1e-6, out=(torch.empty_like(qd), k_view))
    ok, worst = within_ulps(to_np(k_view), ref_k, ulps=1.0, atol=1e-6)
    assert ok, worst
    assert torch.equal(kv[:, 4096:], v_before)
    with pytest.raises(ValueError, match="qk_shape"):
        ops.fused_qk_rmsnorm(qd[..., :2048], kd, qwd, kwd, 1e-6)
    assert status_clean()


def _branch(L, L_ctx, seed):
    from opengenie_b200 import synthetic
    from opengenie_b200.video_text_attention import VideoTextCrossAttention

    inp = synthetic.make_text_inputs(L, L_ctx, seed=seed)
    br = VideoTextCrossAttention(synthetic.make_text_attention_weights(seed=seed + 1), "cuda")
    dev = inp.to("cuda")
    br.calibrate_input_scales(dev.x, dev.timestep, dev.context, dev.prompt_timestep)
    return inp, dev, br


def _gemm_atol(a_codes, s_a, w_codes, s_w, pre_bias, rows):
    """fp32-accumulation allowance plus one ulp of the pre-bias value (its bf16 rounding precedes the bias
    add, and a bias that nearly cancels it turns that ulp into many ulps of the sum)."""
    return accum_atol(a_codes, s_a, w_codes, s_w) + bf16_ulp(pre_bias).reshape(rows, -1)


@pytest.mark.parametrize("L,L_ctx", [(16, 24), (300, 77), (1000, 256)])
def test_text_xattn_stage_by_stage_vs_oracle(ogx_lib, L, L_ctx):
    """Every stage of the fused branch against the oracle fed the kernel's own input to that stage, and the
    branch's output equal to the composition of those stages."""
    from opengenie_b200 import ltx_ops

    inp, dev, br = _branch(L, L_ctx, seed=51 + L)
    bw = br.w
    wc = bw.to("cpu")
    out = br(dev.x, dev.timestep, dev.context, dev.prompt_timestep)
    ts_view = inp.timestep.reshape(1, L, 9, 4096)
    pts_view = inp.prompt_timestep.reshape(1, L_ctx, 2, 4096)
    s_q, s_kv, s_out = float(bw.to_q.input_scale), float(bw.to_k.input_scale), float(bw.to_out.input_scale)
    # 1-2. the context's Ada affine and the K/V quantiser: bit-exact
    ctx = ltx_ops.fused_adaln_affine_from_ada(dev.context, bw.prompt_scale_shift_table, dev.prompt_timestep,
                                              shift_index=0, scale_index=1)
    assert np.array_equal(to_np(ctx), O.adaln_affine_from_ada(inp.context, wc.prompt_scale_shift_table, pts_view,
                                                              shift_index=0, scale_index=1))
    cq = ltx_ops.fused_fp8_quantize_e4m3(ctx, bw.to_k.input_scale)
    assert np.array_equal(codes(cq), O.quantize_e4m3(to_np(ctx), s_kv))
    # 3. packed K/V GEMM
    kv = ltx_ops.fp8_scaled_mm(cq, br.w_kv, bw.to_k.input_scale, br.s_kv, bias=br.b_kv, n_per_scale=4096)
    kv = kv.reshape(L_ctx, -1)
    s_kv_w = br.s_kv.cpu().numpy()
    ref = O.fp8_linear(codes(cq), s_kv, codes(br.w_kv), s_kv_w, br.b_kv.cpu())
    pre = O.fp8_linear(codes(cq), s_kv, codes(br.w_kv), s_kv_w)
    ok, worst = within_ulps(to_np(kv), ref.reshape(L_ctx, -1), ulps=1.0,
                            atol=_gemm_atol(codes(cq), s_kv, codes(br.w_kv), s_kv_w, pre, L_ctx))
    assert ok, worst
    # 4. AdaZero (slots 6/7) + the to_q quantiser
    xq, norm = ltx_ops.fused_adazero_from_ada_fp8(dev.x, 1e-6, bw.scale_shift_table, dev.timestep, bw.to_q.input_scale,
                                                  shift_index=6, scale_index=7, return_bf16=True)
    ok, worst = within_ulps(to_np(norm), O.adazero_from_ada(inp.x, 1e-6, wc.scale_shift_table, ts_view, shift_index=6,
                                                            scale_index=7), ulps=1.0, atol=1e-5)
    assert ok, worst
    assert np.array_equal(codes(xq), O.quantize_e4m3(to_np(norm), s_q))
    # 5. to_q
    q = ltx_ops.fp8_scaled_mm(xq, bw.to_q.weight, bw.to_q.input_scale, bw.to_q.weight_scale, bias=bw.to_q.bias)
    wq = codes(bw.to_q.weight)
    s_wq = float(bw.to_q.weight_scale)
    ref = O.fp8_linear(codes(xq), s_q, wq, s_wq, wc.to_q.bias)
    pre = O.fp8_linear(codes(xq), s_q, wq, s_wq)
    ok, worst = within_ulps(to_np(q).reshape(L, -1), ref.reshape(L, -1), ulps=1.0,
                            atol=_gemm_atol(codes(xq), s_q, wq, s_wq, pre, L))
    assert ok, worst
    # 6. Q/K RMSNorm without RoPE
    k = kv[:, :4096].unsqueeze(0)
    v = kv[:, 4096:].unsqueeze(0).contiguous()  # k and v of one attention call share strides
    qn, kn = ltx_ops.fused_qk_rmsnorm(q, k, bw.q_norm_weight, bw.k_norm_weight, 1e-6)
    for got, x, wt in ((qn, q, wc.q_norm_weight), (kn, k, wc.k_norm_weight)):
        ok, worst = within_ulps(to_np(got), O.qk_rmsnorm(to_np(x), wt, 1e-6), ulps=1.0, atol=1e-6)
        assert ok, worst
    # 7. attention of the L queries over the L_ctx keys
    attn = ltx_ops.attention(qn, kn, v, 32)
    tol = block_tolerance(to_np(attn), O.attention(to_np(qn), to_np(kn), to_np(v), 32))
    assert tol["ok"], tol
    # 8. e4m3 epilogue + to_out + bias + gate (slot 8) + residual
    oq = ltx_ops.attention(qn, kn, v, 32, out_e4m3_scale=bw.to_out.input_scale)
    assert np.array_equal(codes(oq), O.quantize_e4m3(to_np(attn), s_out))
    y = ltx_ops.fp8_scaled_mm_residual_gate(oq, bw.to_out.weight, bw.to_out.input_scale, bw.to_out.weight_scale,
                                            bw.to_out.bias, dev.x, bw.scale_shift_table, dev.timestep, gate_index=8)
    wo = codes(bw.to_out.weight)
    s_wo = float(bw.to_out.weight_scale)
    y_ref = O.fp8_linear(codes(oq), s_out, wo, s_wo)
    yb = O.bias_add_bf16(y_ref, wc.to_out.bias)
    gate = O.ada_value(wc.scale_shift_table, ts_view, 8, table_is_bf16=False, ts_is_bf16=True)
    ref_out = O.residual_gate_bf16(inp.x, yb, gate)
    acc = accum_atol(codes(oq), s_out, wo, s_wo)
    atol = np.abs(gate) * (bf16_ulp(y_ref) + bf16_ulp(yb) + acc.reshape(y_ref.shape)) + bf16_ulp(yb * gate)
    ok, worst = within_ulps(to_np(y), ref_out, ulps=1.0, atol=atol)
    assert ok, worst
    # the branch is exactly this composition
    assert torch.equal(out, y)
    assert status_clean()


def test_text_xattn_stages_vs_reference_golden(ogx_lib):
    """The GPU stages fed the reference's own input to each stage (golden from its CPU functions)."""
    from opengenie_b200 import ltx_ops, synthetic
    from opengenie_b200.video_text_attention import VideoTextCrossAttention

    d = np.load(os.path.join(GOLD, "text_xattn.npz"))
    L, L_ctx = int(d["tokens"]), int(d["context_tokens"])
    inp = synthetic.make_text_inputs(L, L_ctx, seed=int(d["seed_inputs"]))
    tw = synthetic.make_text_attention_weights(seed=int(d["seed_weights"]))
    tw.to_q.input_scale = torch.tensor(float(d["s_q"]), dtype=torch.float32)
    for lin in (tw.to_k, tw.to_v):
        lin.input_scale = torch.tensor(float(d["s_kv"]), dtype=torch.float32)
    tw.to_out.input_scale = torch.tensor(float(d["s_out"]), dtype=torch.float32)
    br = VideoTextCrossAttention(tw, "cuda")
    dev = inp.to("cuda")
    bw = br.w
    ctx = ltx_ops.fused_adaln_affine_from_ada(dev.context, bw.prompt_scale_shift_table, dev.prompt_timestep,
                                              shift_index=0, scale_index=1)
    assert np.array_equal(to_np(ctx), O.bf16_from_bits(d["ctx"]))
    cq = torch.from_numpy(d["cq"]).view(torch.float8_e4m3fn).cuda().reshape(L_ctx, 4096)
    kv = ltx_ops.fp8_scaled_mm(cq, br.w_kv, bw.to_k.input_scale, br.s_kv, bias=br.b_kv, n_per_scale=4096)
    assert block_tolerance(to_np(kv[:, 4096:]).reshape(1, L_ctx, 4096), O.bf16_from_bits(d["v"]))["ok"]
    qn, kn = ltx_ops.fused_qk_rmsnorm(from_bits(d["q_proj"]), from_bits(d["k_proj"]), bw.q_norm_weight,
                                      bw.k_norm_weight, 1e-6)
    for got, key in ((qn, "q"), (kn, "k")):
        ref = O.bf16_from_bits(d[key])
        # one rounding here, two in torch's rms_norm with weight (normalised value, then the product)
        assert (np.abs(to_np(got) - ref) <= np.abs(ref) * 2.0 ** -6).all()
    attn = ltx_ops.attention(from_bits(d["q"]), from_bits(d["k"]), from_bits(d["v"]), 32)
    assert block_tolerance(to_np(attn), O.bf16_from_bits(d["attn"]))["ok"]
    oq = torch.from_numpy(d["oq"]).view(torch.float8_e4m3fn).cuda().reshape(1, L, 4096)
    out = ltx_ops.fp8_scaled_mm_residual_gate(oq, bw.to_out.weight, bw.to_out.input_scale, bw.to_out.weight_scale,
                                              bw.to_out.bias, dev.x, bw.scale_shift_table, dev.timestep, gate_index=8)
    tol = block_tolerance(to_np(out), O.bf16_from_bits(d["out"]))
    assert tol["ok"], tol
    assert status_clean()


def test_text_xattn_full_size_vs_fp32_reference_on_gpu(ogx_lib):
    """9216 video tokens over a 1024-token context: the fused branch against the same stages in torch fp32 on
    the GPU (fp32 matmuls on the dequantised e4m3 operands, fp32 SDPA); sum|d|/sum|ref| <= 1e-2."""
    from opengenie_b200 import synthetic

    inp, dev, br = _branch(9216, synthetic.TEXT_CONTEXT_TOKENS, seed=61)
    out = br(dev.x, dev.timestep, dev.context, dev.prompt_timestep)
    with torch.no_grad():
        ref = to_np(O.video_text_cross_attention_cpu_fp32(
            dev.x, dev.timestep.reshape(1, 9216, 9, 4096), dev.context,
            dev.prompt_timestep.reshape(1, synthetic.TEXT_CONTEXT_TOKENS, 2, 4096), br.w))
    tol = block_tolerance(to_np(out), ref, ulps=2.0)
    print("text cross-attention vs fp32:", tol)
    assert tol["mean_rel"] <= 1e-2, tol
    assert status_clean()


def test_text_xattn_graph_replay_matches_eager(ogx_lib):
    from opengenie_b200.graphs import StepGraph

    inp, dev, br = _branch(300, 77, seed=71)
    eager = br(dev.x, dev.timestep, dev.context, dev.prompt_timestep).clone()
    buf = torch.empty_like(dev.x)
    graph = StepGraph(lambda: br(dev.x, dev.timestep, dev.context, dev.prompt_timestep, out=buf), "cuda")
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(buf, eager)
    assert status_clean()
