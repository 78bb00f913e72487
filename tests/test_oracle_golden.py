"""The CPU oracle pinned against the reference's own outputs (tests/golden, made by make_golden.py)."""

import os

import numpy as np
import pytest
import torch

from oracle import ltx_block_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def g(name):
    return np.load(os.path.join(GOLD, name))


def bf(bits):
    return O.bf16_from_bits(bits)


def test_quantiser_bf16_every_bit_pattern_matches_reference_torch_path():
    d = g("quant_bf16.npz")
    x = bf(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    for s, codes in zip(d["scales"], d["codes"]):
        got = O.quantize_e4m3(x, float(s), in_dtype="bf16", mode="torch")
        assert np.array_equal(got, codes), f"scale {s}: {(got != codes).sum()} codes differ"


def test_quantiser_f16_every_bit_pattern_matches_reference_torch_path():
    d = g("quant_f16.npz")
    x = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    for s, codes in zip(d["scales"], d["codes"]):
        got = O.quantize_e4m3(x, float(s), in_dtype="f16", mode="torch")
        assert np.array_equal(got, codes), f"scale {s}: {(got != codes).sum()} codes differ"


def test_single_rounding_semantics_differ_from_torch_path_on_some_codes():
    # The reference's Triton kernel rounds once; its torch path rounds twice.  The
    # oracle reproduces both and they must disagree somewhere (triton_ltx_ops.py:146-148 vs :3443).
    x = bf(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    a = O.quantize_e4m3(x, 0.0371, mode="torch")
    b = O.quantize_e4m3(x, 0.0371, mode="single")
    assert (a != b).sum() > 0


def test_e4m3_codes_round_trip():
    codes = np.arange(256, dtype=np.uint8)
    vals = O.e4m3_to_f32(codes)
    back = O.f32_to_e4m3(vals)
    finite = ~np.isnan(vals)
    assert np.array_equal(back[finite], codes[finite])
    assert set(back[~finite].tolist()) == {0x7F, 0xFF}


def test_bf16_round_matches_torch():
    x = torch.randn(100000) * 100
    x[::7] *= 1e-30
    ours = O.bf16_round(x.numpy())
    ref = x.to(torch.bfloat16).float().numpy()
    assert np.array_equal(ours, ref)


@pytest.mark.parametrize("tag", ["a", "b"])
def test_adazero_oracle_vs_reference_torch_path(tag):
    d = g("ops.npz")
    x = bf(d[f"ada_{tag}_x"])
    table = d[f"ada_{tag}_table"]
    tb = bool(d[f"ada_{tag}_table_bf16"])
    cols = x.shape[-1]
    ts = bf(d[f"ada_{tag}_ts"]).reshape(x.shape[0], x.shape[1], 6, cols)
    sh, sc = (int(v) for v in d[f"ada_{tag}_idx"])
    y = O.adazero_from_ada(x, 1e-6, table, ts, shift_index=sh, scale_index=sc, table_is_bf16=tb, ts_is_bf16=True)
    ref = bf(d[f"ada_{tag}_y"])
    # the reference's own tolerance between its kernel and its torch path (tests/test_triton_ltx_ops.py:92)
    assert np.abs(y - ref).max() <= 0.0625


def test_bias_add_oracle_bitwise():
    d = g("ops.npz")
    got = O.bias_add_bf16(bf(d["bias_x"]), d["bias_b"])
    assert np.array_equal(got, bf(d["bias_y"]))


def test_residual_gate_bias_oracle_bitwise():
    d = g("ops.npz")
    x, y = bf(d["res_x"]), bf(d["res_y"])
    ts = bf(d["res_ts"]).reshape(1, 9, 9, 2048)
    got = O.residual_gate_bias_from_ada(x, y, d["res_bias"], d["res_table"], ts, gate_index=8, table_is_bf16=False,
                                        ts_is_bf16=True)
    assert np.array_equal(got, bf(d["res_out"]))


def test_rope_oracle_vs_reference_restatement():
    d = g("ops.npz")
    x = bf(d["rope_x"])
    w = bf(d["rope_w"])
    cos, sin = bf(d["rope_cos"]), bf(d["rope_sin"])
    got = O.qk_rmsnorm_rope(x, w, 1e-6, cos, sin)
    ref = bf(d["rope_out"])
    # the reference test's tolerance (tests/test_triton_ltx_ops.py:228)
    assert np.abs(got - ref).max() <= 0.125
    assert np.abs(got - ref).mean() < 4e-3


def _block_case():
    from opengenie_b200 import synthetic

    d = g("block.npz")
    inp = synthetic.make_inputs(synthetic.small_config(1, 2, 8), seed=int(d["seed_inputs"]))
    w = synthetic.make_weights(seed=int(d["seed_weights"]))
    for lin in (w.to_q, w.to_k, w.to_v):
        lin.input_scale = torch.tensor(float(d["s_in"]), dtype=torch.float32)
    w.to_out.input_scale = torch.tensor(float(d["s_out"]), dtype=torch.float32)
    return d, inp, w


def test_synthetic_inputs_regenerate_identically():
    d, inp, _ = _block_case()
    assert np.array_equal(inp.x.contiguous().view(torch.int16).numpy().view(np.uint16), d["x"])


def _close(got, ref, atol=2e-2, rel_ulps=1.0):
    """|d| <= atol + rel_ulps bf16 ulps of |ref| everywhere, and sum|d| / sum|ref| <= 1e-2."""
    d = np.abs(got - ref)
    bound = atol + rel_ulps * np.abs(ref) * 2.0 ** -7
    assert (d <= bound).all(), f"max excess {(d - bound).max()}"
    assert d.sum() / max(np.abs(ref).sum(), 1e-30) <= 1e-2


def test_block_oracle_stages_vs_reference_composition():
    """Each stage of the oracle block, fed the reference's own input to that stage."""
    d, inp, w = _block_case()
    ts_view = inp.timestep.reshape(1, inp.x.shape[1], 6, 4096)
    table = w.scale_shift_table
    # Q/K/V from the reference's quantised activation: the oracle quantises internally, so feed it
    # the dequantised codes times the scale (exactly the bf16 values that quantise back to them).
    s_in = float(d["s_in"])
    xq_vals = O.e4m3_to_f32(d["xq"]).reshape(1, -1, 4096) * np.float32(s_in)
    assert np.array_equal(O.quantize_e4m3(xq_vals, s_in), d["xq"].reshape(1, -1, 4096))
    q, k, v = O.block_qkv(xq_vals, w, cos=inp.cos, sin=inp.sin)
    _close(v, bf(d["v"]), atol=2e-2, rel_ulps=1.0)  # CPU _scaled_mm vs float64 accumulation
    # the reference's RoPE restatement rounds after every op: its own test tolerance is atol 0.125
    _close(q, bf(d["q"]), atol=0.125, rel_ulps=0.0)
    _close(k, bf(d["k"]), atol=0.125, rel_ulps=0.0)
    # attention from the reference's q/k/v (fp32 SDPA there, float64 here)
    attn = O.attention(bf(d["q"]), bf(d["k"]), bf(d["v"]), 32)
    _close(O.bf16_round(attn), bf(d["attn"]), atol=2e-2, rel_ulps=1.0)
    # out-projection + bias + gate + residual from the reference's attention output
    out, _ = O.block_epilogue(inp.x, bf(d["attn"]), w, table, ts_view)
    _close(out, bf(d["out"]), atol=2e-2, rel_ulps=1.0)


def test_block_cpu_fp32_baseline_agrees_with_oracle():
    d, inp, w = _block_case()
    ts_view = inp.timestep.reshape(1, inp.x.shape[1], 6, 4096)
    a = O.video_block(inp.x, ts_view, inp.cos, inp.sin, w)
    b = O.video_block_cpu_fp32(inp.x, ts_view, inp.cos, inp.sin, w).numpy()
    # same stages and rounding points; fp32 vs float64 sums flip a few e4m3 codes, which a
    # 16-token block (little averaging in attention) carries to a few-ulp output difference
    d = np.abs(a - b)
    assert d.sum() / np.abs(a).sum() <= 1e-3
    assert d.max() <= 0.125


@pytest.mark.parametrize("tag,in_dtype", [("bf16", "bf16"), ("f16", "f16")])
def test_gelu_quantiser_every_bit_pattern_matches_reference_torch_path(tag, in_dtype):
    """GELU (tanh) + quantiser (triton_ltx_ops.py:164-169) on every bf16 / fp16 bit pattern."""
    d = g("gelu_quant.npz")
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    if in_dtype == "bf16":
        x = bf(allbits)
        gelu_ref = bf(d[f"{tag}_gelu"])
    else:
        x = allbits.view(np.float16).astype(np.float32)
        gelu_ref = d[f"{tag}_gelu"].view(np.float16).astype(np.float32)
    gelu = O.gelu_tanh(x, in_dtype=in_dtype)
    same = (gelu == gelu_ref) | (np.isnan(gelu) & np.isnan(gelu_ref))
    assert same.all(), f"{(~same).sum()} GELU values differ"
    for s, codes in zip(d[f"{tag}_scales"], d[f"{tag}_codes"]):
        got = O.gelu_tanh_quantize_e4m3(x, float(s), in_dtype=in_dtype)
        assert np.array_equal(got, codes), f"scale {s}: {(got != codes).sum()} codes differ"


def _ffn_case():
    from opengenie_b200 import synthetic

    d = g("ffn.npz")
    inp = synthetic.make_inputs(synthetic.small_config(1, 2, 8), seed=int(d["seed_inputs"]))
    fw = synthetic.make_ffn_weights(seed=int(d["seed_weights"]))
    fw.proj.input_scale = torch.tensor(float(d["s1"]), dtype=torch.float32)
    fw.out.input_scale = torch.tensor(float(d["s2"]), dtype=torch.float32)
    return d, inp, fw


def test_ffn_oracle_stages_vs_reference_composition():
    """Each stage of the oracle FFN branch, fed the reference's own input to that stage."""
    d, inp, fw = _ffn_case()
    ts_view = inp.timestep.reshape(1, inp.x.shape[1], 6, 4096)
    s1, s2 = float(d["s1"]), float(d["s2"])
    # AdaZero idx 3/4 + quantiser: the reference's CPU AdaZero rounds after every op, so compare the
    # codes where the oracle's bf16 AdaZero output quantises identically (the reference test's 0.0625
    # AdaZero tolerance moves some codes by one step)
    _, mid = O.video_ffn(inp.x, ts_view, fw, return_intermediates=True)
    xq_ref = d["xq"].reshape(mid["xq"].shape)
    step = np.abs(O.e4m3_to_f32(mid["xq"]) - O.e4m3_to_f32(xq_ref))
    assert (mid["xq"] == xq_ref).mean() >= 0.95 and (step <= 0.0625 / s1 + 64).all()
    # proj + bias from the reference's quantised activation (CPU _scaled_mm vs float64 accumulation)
    hidden = O.fp8_linear(xq_ref.reshape(16, 4096), s1, fw.proj.weight.view(torch.uint8).numpy(),
                          float(fw.proj.weight_scale), fw.proj.bias.float().numpy())
    _close(hidden, bf(d["hidden"]).reshape(hidden.shape), atol=2e-2, rel_ulps=1.0)
    # GELU + quantiser from the reference's hidden: bit-exact
    assert np.array_equal(O.gelu_tanh_quantize_e4m3(bf(d["hidden"]), s2).reshape(-1), d["hq"].reshape(-1))
    # second projection from the reference's codes
    y = O.fp8_linear(d["hq"].reshape(16, -1), s2, fw.out.weight.view(torch.uint8).numpy(), float(fw.out.weight_scale))
    _close(y, bf(d["y"]).reshape(y.shape), atol=2e-2, rel_ulps=1.0)
    # bias + gate (idx 5) + residual from the reference's y: bit-exact
    out = O.residual_gate_bias_from_ada(inp.x, bf(d["y"]).reshape(1, 16, 4096), fw.out.bias.float().numpy(),
                                        fw.scale_shift_table, ts_view, gate_index=5)
    assert np.array_equal(out, bf(d["out"]).reshape(out.shape))


def test_ffn_cpu_fp32_baseline_agrees_with_oracle():
    d, inp, fw = _ffn_case()
    ts_view = inp.timestep.reshape(1, inp.x.shape[1], 6, 4096)
    a = O.video_ffn(inp.x, ts_view, fw)
    b = O.video_ffn_cpu_fp32(inp.x, ts_view, fw).float().numpy()
    diff = np.abs(a - b)
    assert diff.sum() / np.abs(a).sum() <= 1e-3
    assert diff.max() <= 0.125


def test_residual_gate_without_bias_oracle_bitwise():
    """``fused_residual_gate_from_ada`` (:640-694) is the bias residual with a zero bias, bit for bit."""
    d = g("residual_nobias.npz")
    x, y = bf(d["x"]).reshape(1, 9, 2048), bf(d["y"]).reshape(1, 9, 2048)
    ts = bf(d["ts"]).reshape(1, 9, 9, 2048)
    out = O.residual_gate_bias_from_ada(x, y, np.zeros(2048, np.float32), d["table"], ts, gate_index=8)
    assert np.array_equal(out.reshape(-1), bf(d["out"]).reshape(-1))


@pytest.mark.parametrize("tag", ["a", "b"])
def test_adaln_affine_oracle_bitwise(tag):
    """``fused_adaln_affine_from_ada`` (:94-141): the oracle equals the reference's torch path bit for bit."""
    d = g("adaln_affine.npz")
    x = bf(d[f"{tag}_x"])
    rows, cols = x.shape[1], x.shape[2]
    ts = bf(d[f"{tag}_ts"]).reshape(1, rows, 9, cols)
    sh, sc = (int(i) for i in d[f"{tag}_idx"])
    out = O.adaln_affine_from_ada(x, d[f"{tag}_table"], ts, shift_index=sh, scale_index=sc,
                                  table_is_bf16=bool(d[f"{tag}_table_bf16"]))
    assert np.array_equal(out, bf(d[f"{tag}_y"]))


def test_head_gate_oracle_bitwise():
    d = g("head_gate.npz")
    out = O.head_gate_mul_bf16(bf(d["out"]), bf(d["gates"]), 32, 128)
    assert np.array_equal(out, bf(d["y"]))


def test_mul_from_ada_and_residual_gate_bf16_oracle_bitwise():
    d = g("ada_misc.npz")
    out = O.mul_from_ada(bf(d["mul_x"]), d["mul_table"], bf(d["mul_ts"]).reshape(1, 6, 9, 4096), gate_index=4)
    assert np.array_equal(out, bf(d["mul_y"]))
    x, y = bf(d["res_x"]), bf(d["res_y"])
    assert np.array_equal(O.residual_gate_bf16(x, y, bf(d["res_gate_tok"])), bf(d["res_out_tok"]))
    assert np.array_equal(O.residual_gate_bf16(x, y, bf(d["res_gate_sample"])), bf(d["res_out_sample"]))


def test_adazero_explicit_oracle_vs_reference_torch_path():
    """``fused_adazero`` (:8-37): the oracle follows its GPU kernel (one rounding); the torch path rounds
    after each op and agrees within the reference test's AdaZero tolerance (0.0625)."""
    d = g("ada_misc.npz")
    out = O.adazero_explicit(bf(d["ada_x"]), 1e-6, bf(d["ada_scale"]), bf(d["ada_shift"]))
    assert np.abs(out - bf(d["ada_y"])).max() <= 0.0625


def _text_case():
    from opengenie_b200 import synthetic

    d = g("text_xattn.npz")
    L, Lc = int(d["tokens"]), int(d["context_tokens"])
    inp = synthetic.make_text_inputs(L, Lc, seed=int(d["seed_inputs"]))
    tw = synthetic.make_text_attention_weights(seed=int(d["seed_weights"]))
    tw.to_q.input_scale = torch.tensor(float(d["s_q"]), dtype=torch.float32)
    for lin in (tw.to_k, tw.to_v):
        lin.input_scale = torch.tensor(float(d["s_kv"]), dtype=torch.float32)
    tw.to_out.input_scale = torch.tensor(float(d["s_out"]), dtype=torch.float32)
    ts_view = inp.timestep.reshape(1, L, 9, 4096)
    pts_view = inp.prompt_timestep.reshape(1, Lc, 2, 4096)
    return d, inp, tw, ts_view, pts_view


def test_text_xattn_inputs_regenerate_identically():
    d, inp, _, _, _ = _text_case()
    assert inp.x.shape == (1, int(d["tokens"]), 4096) and inp.context.shape == (1, int(d["context_tokens"]), 4096)
    assert inp.timestep.stride(1) == 0 and inp.prompt_timestep.stride(1) == 0


def test_text_xattn_oracle_stages_vs_reference_composition():
    """Each stage of the oracle's text cross-attention branch, fed the reference's own input to that stage."""
    d, inp, tw, ts_view, pts_view = _text_case()
    L, Lc = int(d["tokens"]), int(d["context_tokens"])
    s_q, s_kv, s_out = float(d["s_q"]), float(d["s_kv"]), float(d["s_out"])
    _, mid = O.video_text_cross_attention(inp.x, ts_view, inp.context, pts_view, tw, return_intermediates=True)
    # the context's Ada affine with the prompt table, and its K/V codes: bit-exact
    assert np.array_equal(mid["ctx"], bf(d["ctx"]))
    assert np.array_equal(O.quantize_e4m3(bf(d["ctx"]), s_kv), d["cq"])
    # the query side: the oracle's AdaZero rounds once, the reference's rms_norm + affine after each op;
    # within the reference's AdaZero test tolerance (tests/test_triton_ltx_ops.py:92), codes mostly equal
    assert np.abs(mid["norm"] - bf(d["attn_input"])).max() <= 0.0625
    assert (O.quantize_e4m3(mid["norm"], s_q) == d["xq"]).mean() >= 0.95

    def lin(codes, s, layer, rows):
        return O.fp8_linear(codes.reshape(rows, 4096), s, layer.weight.view(torch.uint8).numpy(),
                            float(layer.weight_scale), layer.bias.float().numpy())

    # projections from the reference's codes (CPU _scaled_mm vs float64 accumulation)
    _close(lin(d["xq"], s_q, tw.to_q, L), bf(d["q_proj"]).reshape(L, 4096), atol=2e-2, rel_ulps=1.0)
    _close(lin(d["cq"], s_kv, tw.to_k, Lc), bf(d["k_proj"]).reshape(Lc, 4096), atol=2e-2, rel_ulps=1.0)
    _close(lin(d["cq"], s_kv, tw.to_v, Lc), bf(d["v"]).reshape(Lc, 4096), atol=2e-2, rel_ulps=1.0)
    # Q/K RMSNorm without RoPE from the reference's projections: one rounding against torch's rms_norm
    _close(O.qk_rmsnorm(bf(d["q_proj"]), tw.q_norm_weight, 1e-6), bf(d["q"]), atol=0.0, rel_ulps=1.0)
    _close(O.qk_rmsnorm(bf(d["k_proj"]), tw.k_norm_weight, 1e-6), bf(d["k"]), atol=0.0, rel_ulps=1.0)
    # attention of 16 queries over the 24 context keys (fp32 SDPA there, float64 here)
    attn = O.attention(bf(d["q"]), bf(d["k"]), bf(d["v"]), 32)
    _close(O.bf16_round(attn), bf(d["attn"]), atol=2e-2, rel_ulps=1.0)
    # to_out's quantiser: bit-exact; to_out from its codes
    assert np.array_equal(O.quantize_e4m3(bf(d["attn"]), s_out), d["oq"])
    _close(lin(d["oq"], s_out, tw.to_out, L), bf(d["y"]).reshape(L, 4096), atol=2e-2, rel_ulps=1.0)
    # the gated residual (slot 8) from the reference's y: bit-exact
    gate = O.ada_value(tw.scale_shift_table, ts_view, 8, table_is_bf16=False, ts_is_bf16=True)
    assert np.array_equal(O.residual_gate_bf16(inp.x, bf(d["y"]), gate), bf(d["out"]))


def test_text_xattn_cpu_fp32_baseline_agrees_with_oracle():
    d, inp, tw, ts_view, pts_view = _text_case()
    a = O.video_text_cross_attention(inp.x, ts_view, inp.context, pts_view, tw)
    b = O.video_text_cross_attention_cpu_fp32(inp.x, ts_view, inp.context, pts_view, tw).numpy()
    diff = np.abs(a - b)
    assert diff.sum() / np.abs(a).sum() <= 1e-3
    assert diff.max() <= 0.125


def test_qk_rmsnorm_is_rope_with_unit_rotation():
    """The RMSNorm-only restatement equals the RMSNorm + RoPE one with cos = 1, sin = 0, bit for bit."""
    gen = torch.Generator().manual_seed(3)
    x = torch.randn((1, 5, 4096), generator=gen).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn((4096,), generator=gen)).to(torch.bfloat16)
    cos, sin = torch.ones((1, 32, 5, 64)), torch.zeros((1, 32, 5, 64))
    assert np.array_equal(O.qk_rmsnorm(x, w, 1e-6), O.qk_rmsnorm_rope(x, w, 1e-6, cos, sin))


def test_attention_oracle_keys_of_another_length():
    """softmax(q k^T / sqrt(d)) v per head with 7 queries over 3 keys, against a direct evaluation."""
    gen = torch.Generator().manual_seed(4)
    q = torch.randn((2, 7, 2 * 128), generator=gen, dtype=torch.float64)
    k = torch.randn((2, 3, 2 * 128), generator=gen, dtype=torch.float64)
    v = torch.randn((2, 3, 2 * 128), generator=gen, dtype=torch.float64)
    got = O.attention(q.numpy(), k.numpy(), v.numpy(), 2)
    for b in range(2):
        for h in range(2):
            sl = slice(h * 128, (h + 1) * 128)
            s = q[b, :, sl] @ k[b, :, sl].T / np.sqrt(128.0)
            ref = torch.softmax(s, dim=-1) @ v[b, :, sl]
            assert np.allclose(got[b, :, sl], ref.numpy(), rtol=1e-6, atol=1e-6)
