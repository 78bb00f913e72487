"""Generates the golden fixtures in this directory from the reference itself.

Run in a container where the reference (plugyawn/opengenie) is importable:

    python tests/golden/make_golden.py --reference /path/to/opengenie

It imports ``ltx_serve.triton_ltx_ops`` on the CPU, where every CUDA/Triton guard
fails and the reference's own torch paths run, and records their outputs on
seeded inputs:

- quant_bf16.npz / quant_f16.npz: ``fused_fp8_quantize_e4m3`` (torch path,
  triton_ltx_ops.py:146-148) on every bf16 / fp16 bit pattern for several scales;
- ops.npz: ``fused_adazero_from_ada`` (:40-91), ``fused_bias_add_bf16`` (:185-201),
  ``fused_residual_gate_bias_from_ada`` (:204-262, residual mode
  "triton_simple_bf16_round" as production sets it) and the reference test's
  split-RoPE restatement (tests/test_triton_ltx_ops.py:232-249);
- block.npz: the video self-attention block composed from those functions with
  CPU ``torch._scaled_mm`` (the FP8 linears) and fp32 SDPA, for a 16-token input
  with the synthetic weights of ``opengenie_b200.synthetic.make_weights(seed=7)``;
- gelu_quant.npz: ``fused_gelu_tanh_fp8_quantize_e4m3`` (:164-169) on every bf16 /
  fp16 bit pattern, and the GELU it quantises;
- ffn.npz: the video FFN branch (:3224-3258) composed the same way, 16 tokens,
  ``opengenie_b200.synthetic.make_ffn_weights(seed=9)``;
- residual_nobias.npz: ``fused_residual_gate_from_ada`` (:640-694);
- adaln_affine.npz: ``fused_adaln_affine_from_ada`` (:94-141);
- head_gate.npz: ``fused_head_gate_mul_bf16`` (:614-637);
- ada_misc.npz: ``fused_mul_from_ada`` (:695-741), ``fused_residual_gate_bf16`` (:590-611) and
  ``fused_adazero`` (:8-37);
- text_xattn.npz: the video text cross-attention branch with cross-attention AdaLN (:2810-2888)
  composed the same way, 16 video tokens over a 24-token context,
  ``opengenie_b200.synthetic.make_text_attention_weights(seed=17)``.  Its ``rms_norm`` and the
  attention module's ``q_norm`` / ``k_norm`` live in the un-vendored ltx_core; they are taken as
  ``torch.nn.functional.rms_norm`` (without / with the norm weight), the function the reference's
  own ``fused_adazero`` fallback calls (:9-10).

``--only NAME`` (NAME without .npz) regenerates one fixture.

Inputs that are cheap to regenerate (seeded ``torch.Generator``) are stored too so
the tests do not depend on regeneration.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

QUANT_SCALES_BF16 = [1.0, 0.0371, 0.00123, 3.7, 0.0107421875, 1.0 / 448.0]
QUANT_SCALES_F16 = [1.0, 0.0371, 0.5]


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def load_reference(root: str):
    sys.path.insert(0, root)
    import ltx_serve.triton_ltx_ops as ops  # noqa: E402

    ops._BLOCK_RESIDUAL_MODE = "triton_simple_bf16_round"
    spec = importlib.util.spec_from_file_location("ref_kernel_tests", os.path.join(root, "tests", "test_triton_ltx_ops.py"))
    tests = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tests)
    return ops, tests._torch_video_rmsnorm_split_rope


def make_quant(ops) -> None:
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    xb = torch.from_numpy(allbits.view(np.int16)).view(torch.bfloat16)
    codes = []
    for s in QUANT_SCALES_BF16:
        q = ops.fused_fp8_quantize_e4m3(xb.reshape(256, 256), torch.tensor(s, dtype=torch.float32))
        codes.append(q.view(torch.uint8).reshape(-1).numpy().copy())
    np.savez_compressed(os.path.join(HERE, "quant_bf16.npz"), scales=np.array(QUANT_SCALES_BF16, np.float32),
                        codes=np.stack(codes))
    xh = torch.from_numpy(allbits.view(np.int16)).view(torch.float16)
    codes = []
    for s in QUANT_SCALES_F16:
        q = ops.fused_fp8_quantize_e4m3(xh.reshape(256, 256), torch.tensor(s, dtype=torch.float32))
        codes.append(q.view(torch.uint8).reshape(-1).numpy().copy())
    np.savez_compressed(os.path.join(HERE, "quant_f16.npz"), scales=np.array(QUANT_SCALES_F16, np.float32),
                        codes=np.stack(codes))


def make_ops(ops, rope_ref) -> None:
    out = {}
    g = torch.Generator().manual_seed(2024)
    # AdaZero from table: [1, 5, 4096] with uniform (stride-0) timestep, idx 0/1, fp32 table
    for tag, cols, rows, tdt, sh, sc in (("a", 4096, 5, torch.float32, 0, 1), ("b", 2048, 7, torch.bfloat16, 3, 4)):
        x = torch.randn((1, rows, cols), generator=g).to(torch.bfloat16)
        table = (torch.randn((6, cols), generator=g) * 0.5).to(tdt)
        ts = torch.randn((1, rows, 6 * cols), generator=g).to(torch.bfloat16)
        y = ops.fused_adazero_from_ada(x, 1e-6, table, ts, shift_index=sh, scale_index=sc)
        out[f"ada_{tag}_x"] = bits(x)
        out[f"ada_{tag}_table"] = table.float().numpy()
        out[f"ada_{tag}_table_bf16"] = np.array(tdt == torch.bfloat16)
        out[f"ada_{tag}_ts"] = bits(ts)
        out[f"ada_{tag}_idx"] = np.array([sh, sc])
        out[f"ada_{tag}_y"] = bits(y)
    # bias add [11, 2048] with fp32 bias
    x = torch.randn((11, 2048), generator=g).to(torch.bfloat16)
    bias = torch.randn((2048,), generator=g)
    out["bias_x"], out["bias_b"] = bits(x), bias.numpy()
    out["bias_y"] = bits(ops.fused_bias_add_bf16(x, bias))
    # bias + gate + residual [1, 9, 2048], fp32 table with 9 slots, gate idx 8 (the reference test's shape)
    x = torch.randn((1, 9, 2048), generator=g).to(torch.bfloat16)
    y = torch.randn((1, 9, 2048), generator=g).to(torch.bfloat16)
    bias = torch.randn((2048,), generator=g)
    table = torch.randn((9, 2048), generator=g)
    ts = torch.randn((1, 9, 9 * 2048), generator=g).to(torch.bfloat16)
    r = ops.fused_residual_gate_bias_from_ada(x, y, bias, table, ts, gate_index=8)
    out.update(res_x=bits(x), res_y=bits(y), res_bias=bias.numpy(), res_table=table.numpy(), res_ts=bits(ts),
               res_out=bits(r))
    # Q/K RMSNorm + split RoPE restatement (tests/test_triton_ltx_ops.py:232-249), 17 tokens
    q = torch.randn((1, 17, 4096), generator=g).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn((4096,), generator=g)).to(torch.bfloat16)
    freqs = torch.randn((1, 32, 17, 64), generator=g)
    cos, sin = freqs.cos().to(torch.bfloat16), freqs.sin().to(torch.bfloat16)
    o = rope_ref(q, w, 1e-6, cos, sin)
    out.update(rope_x=bits(q), rope_w=bits(w), rope_cos=bits(cos), rope_sin=bits(sin), rope_out=bits(o))
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **out)


def make_block(ops, rope_ref) -> None:
    from opengenie_b200 import synthetic

    cfg = synthetic.small_config(1, 2, 8)  # 16 tokens
    inp = synthetic.make_inputs(cfg, seed=11)
    w = synthetic.make_weights(seed=7)
    x, ts, cos, sin = inp.x, inp.timestep, inp.cos, inp.sin
    table = w.scale_shift_table
    # static input scales (amax/448 of each FP8 linear's input), fixed here and stored
    norm = ops.fused_adazero_from_ada(x, 1e-6, table, ts, shift_index=0, scale_index=1)
    s_in = (norm.float().abs().amax() / 448.0).to(torch.float32)

    def linear(inp_q, s_a, lin, bias=True):
        o = torch._scaled_mm(inp_q.reshape(-1, inp_q.shape[-1]), lin.weight.t(), scale_a=s_a, scale_b=lin.weight_scale,
                             out_dtype=torch.bfloat16, use_fast_accum=True)
        if bias:
            o = ops.fused_bias_add_bf16(o, lin.bias)
        return o.reshape(1, -1, o.shape[-1])

    xq = ops.fused_fp8_quantize_e4m3(norm, s_in)
    q, k, v = (linear(xq, s_in, lin) for lin in (w.to_q, w.to_k, w.to_v))
    qr = rope_ref(q, w.q_norm_weight, 1e-6, cos, sin)
    kr = rope_ref(k, w.k_norm_weight, 1e-6, cos, sin)
    qh, kh, vh = (t.float().view(1, -1, 32, 128).transpose(1, 2) for t in (qr, kr, v))
    attn = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2).reshape(1, -1, 4096)
    attn = attn.to(torch.bfloat16)
    s_out = (attn.float().abs().amax() / 448.0).to(torch.float32)
    oq = ops.fused_fp8_quantize_e4m3(attn, s_out)
    y = linear(oq, s_out, w.to_out, bias=False)
    out = ops.fused_residual_gate_bias_from_ada(x, y, w.to_out.bias, table, ts, gate_index=2)
    np.savez_compressed(
        os.path.join(HERE, "block.npz"),
        s_in=s_in.numpy(), s_out=s_out.numpy(), x=bits(x), out=bits(out), attn=bits(attn), q=bits(qr), k=bits(kr),
        v=bits(v), xq=xq.view(torch.uint8).numpy(), seed_inputs=np.array(11), seed_weights=np.array(7),
    )


def make_residual_nobias(ops) -> None:
    """``fused_residual_gate_from_ada`` (:640-694, residual mode "triton_simple_bf16_round") on a
    [1, 9, 2048] case with an fp32 table of 9 slots, gate idx 8."""
    g = torch.Generator().manual_seed(2025)
    x = torch.randn((1, 9, 2048), generator=g).to(torch.bfloat16)
    y = torch.randn((1, 9, 2048), generator=g).to(torch.bfloat16)
    table = torch.randn((9, 2048), generator=g)
    ts = torch.randn((1, 9, 9 * 2048), generator=g).to(torch.bfloat16)
    r = ops.fused_residual_gate_from_ada(x, y, table, ts, gate_index=8)
    np.savez_compressed(os.path.join(HERE, "residual_nobias.npz"), x=bits(x), y=bits(y), table=table.numpy(),
                        ts=bits(ts), out=bits(r))


def make_adaln_affine(ops) -> None:
    """``fused_adaln_affine_from_ada`` (:94-141) on [1, 7, 4096] (fp32 table, bf16 timestep, idx 6/7) and
    [1, 5, 2048] (bf16 table, idx 0/1): the reference's torch path there rounds after each op, like its
    kernel (:3469-3534)."""
    g = torch.Generator().manual_seed(2026)
    out = {}
    for tag, cols, rows, tdt, sh, sc in (("a", 4096, 7, torch.float32, 6, 7), ("b", 2048, 5, torch.bfloat16, 0, 1)):
        x = torch.randn((1, rows, cols), generator=g).to(torch.bfloat16)
        table = (torch.randn((9, cols), generator=g) * 0.5).to(tdt)
        ts = torch.randn((1, rows, 9 * cols), generator=g).to(torch.bfloat16)
        y = ops.fused_adaln_affine_from_ada(x, table, ts, shift_index=sh, scale_index=sc)
        out.update({f"{tag}_x": bits(x), f"{tag}_table": table.float().numpy(), f"{tag}_table_bf16": np.array(tdt == torch.bfloat16),
                    f"{tag}_ts": bits(ts), f"{tag}_idx": np.array([sh, sc]), f"{tag}_y": bits(y)})
    np.savez_compressed(os.path.join(HERE, "adaln_affine.npz"), **out)


def make_head_gate(ops) -> None:
    """``fused_head_gate_mul_bf16`` (:614-637, torch path there) on [1, 11, 32 x 128] with gates 2*sigmoid."""
    g = torch.Generator().manual_seed(2027)
    out = torch.randn((1, 11, 4096), generator=g).to(torch.bfloat16)
    gates = (2.0 * torch.sigmoid(torch.randn((1, 11, 32), generator=g))).to(torch.bfloat16)
    y = ops.fused_head_gate_mul_bf16(out, gates, 32, 128)
    np.savez_compressed(os.path.join(HERE, "head_gate.npz"), out=bits(out), gates=bits(gates), y=bits(y))


def make_ada_misc(ops) -> None:
    """``fused_mul_from_ada`` (:695-741), ``fused_residual_gate_bf16`` (:590-611, per-token and per-sample gate)
    and ``fused_adazero`` (:8-37, explicit per-sample scale/shift; its torch path rounds after each op)."""
    g = torch.Generator().manual_seed(2028)
    out = {}
    x = torch.randn((1, 6, 4096), generator=g).to(torch.bfloat16)
    table = torch.randn((9, 4096), generator=g) * 0.5
    ts = torch.randn((1, 6, 9 * 4096), generator=g).to(torch.bfloat16)
    out.update(mul_x=bits(x), mul_table=table.numpy(), mul_ts=bits(ts),
               mul_y=bits(ops.fused_mul_from_ada(x, table, ts, gate_index=4)))
    x = torch.randn((2, 5, 2048), generator=g).to(torch.bfloat16)
    y = torch.randn((2, 5, 2048), generator=g).to(torch.bfloat16)
    gate_tok = torch.randn((2, 5, 2048), generator=g).to(torch.bfloat16)
    gate_sample = torch.randn((2, 1, 2048), generator=g).to(torch.bfloat16)
    out.update(res_x=bits(x), res_y=bits(y), res_gate_tok=bits(gate_tok), res_gate_sample=bits(gate_sample),
               res_out_tok=bits(ops.fused_residual_gate_bf16(x, y, gate_tok)),
               res_out_sample=bits(ops.fused_residual_gate_bf16(x, y, gate_sample)))
    x = torch.randn((2, 7, 4096), generator=g).to(torch.bfloat16)
    scale = (torch.randn((2, 1, 4096), generator=g) * 0.3).to(torch.bfloat16)
    shift = (torch.randn((2, 1, 4096), generator=g) * 0.3).to(torch.bfloat16)
    out.update(ada_x=bits(x), ada_scale=bits(scale), ada_shift=bits(shift),
               ada_y=bits(ops.fused_adazero(x, 1e-6, scale, shift)))
    np.savez_compressed(os.path.join(HERE, "ada_misc.npz"), **out)


GELU_SCALES_BF16 = [1.0, 0.0371, 1.0 / 448.0]
GELU_SCALES_F16 = [1.0, 0.0371]


def make_gelu(ops) -> None:
    """``fused_gelu_tanh_fp8_quantize_e4m3`` (torch path, triton_ltx_ops.py:164-169) on every bf16 and
    fp16 bit pattern, and the GELU it quantises (the reference's own expression, :166)."""
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out = {}
    for tag, dt, scales in (("bf16", torch.bfloat16, GELU_SCALES_BF16), ("f16", torch.float16, GELU_SCALES_F16)):
        x = torch.from_numpy(allbits.view(np.int16)).view(dt).reshape(256, 256)
        out[f"{tag}_gelu"] = bits(torch.nn.functional.gelu(x, approximate="tanh")).reshape(-1)
        codes = [ops.fused_gelu_tanh_fp8_quantize_e4m3(x, torch.tensor(s, dtype=torch.float32))
                 .view(torch.uint8).reshape(-1).numpy().copy() for s in scales]
        out[f"{tag}_scales"] = np.array(scales, np.float32)
        out[f"{tag}_codes"] = np.stack(codes)
    np.savez_compressed(os.path.join(HERE, "gelu_quant.npz"), **out)


def make_ffn(ops) -> None:
    """The video FFN branch (triton_ltx_ops.py:3224-3258, production flags) composed from the reference's
    CPU functions with CPU ``torch._scaled_mm``, for 16 tokens with the synthetic FFN weights of
    ``opengenie_b200.synthetic.make_ffn_weights(seed=9)``."""
    from opengenie_b200 import synthetic

    cfg = synthetic.small_config(1, 2, 8)
    inp = synthetic.make_inputs(cfg, seed=13)
    fw = synthetic.make_ffn_weights(seed=9)
    x, ts, table = inp.x, inp.timestep, fw.scale_shift_table
    norm = ops.fused_adazero_from_ada(x, 1e-6, table, ts, shift_index=3, scale_index=4)
    s1 = (norm.float().abs().amax() / 448.0).to(torch.float32)

    def mm(q, s_a, lin):
        return torch._scaled_mm(q.reshape(-1, q.shape[-1]), lin.weight.t(), scale_a=s_a, scale_b=lin.weight_scale,
                                out_dtype=torch.bfloat16, use_fast_accum=True)

    xq = ops.fused_fp8_quantize_e4m3(norm, s1)
    hidden = ops.fused_bias_add_bf16(mm(xq, s1, fw.proj), fw.proj.bias)
    gelu = torch.nn.functional.gelu(hidden, approximate="tanh")
    s2 = (gelu.float().abs().amax() / 448.0).to(torch.float32)
    hq = ops.fused_gelu_tanh_fp8_quantize_e4m3(hidden, s2)
    y = mm(hq, s2, fw.out).reshape(1, -1, x.shape[-1])
    out = ops.fused_residual_gate_bias_from_ada(x, y, fw.out.bias, table, ts, gate_index=5)
    np.savez_compressed(
        os.path.join(HERE, "ffn.npz"),
        s1=s1.numpy(), s2=s2.numpy(), x=bits(x), out=bits(out), hidden=bits(hidden), xq=xq.view(torch.uint8).numpy(),
        hq=hq.view(torch.uint8).numpy(), y=bits(y), seed_inputs=np.array(13), seed_weights=np.array(9),
    )


def make_text_xattn(ops) -> None:
    """The video text cross-attention branch (triton_ltx_ops.py:2810-2888, production flags) composed from
    the reference's CPU functions with CPU ``torch._scaled_mm`` and fp32 SDPA, 16 video tokens over a
    24-token prompt context, ``opengenie_b200.synthetic.make_text_attention_weights(seed=17)``."""
    from opengenie_b200 import synthetic

    inp = synthetic.make_text_inputs(16, 24, seed=15)
    tw = synthetic.make_text_attention_weights(seed=17)
    x, ts, context, pts = inp.x, inp.timestep, inp.context, inp.prompt_timestep
    table = tw.scale_shift_table
    D = x.shape[-1]
    # context: Ada affine with the prompt table (:2842-2851)
    ctx = ops.fused_adaln_affine_from_ada(context, tw.prompt_scale_shift_table, pts, shift_index=0, scale_index=1)
    # x: rms_norm, then the Ada affine of slots 6/7 (:2856-2862)
    x_norm = torch.nn.functional.rms_norm(x, (D,), eps=tw.norm_eps)
    attn_input = ops.fused_adaln_affine_from_ada(x_norm, table, ts, shift_index=6, scale_index=7)
    s_q = (attn_input.float().abs().amax() / 448.0).to(torch.float32)
    s_kv = (ctx.float().abs().amax() / 448.0).to(torch.float32)

    def linear(inp_q, s_a, lin):
        o = torch._scaled_mm(inp_q.reshape(-1, inp_q.shape[-1]), lin.weight.t(), scale_a=s_a, scale_b=lin.weight_scale,
                             out_dtype=torch.bfloat16, use_fast_accum=True)
        return ops.fused_bias_add_bf16(o, lin.bias).reshape(1, -1, o.shape[-1])

    # attn(attn_input, context=ctx): FP8Linear.forward per projection (:1676-1716), q_norm / k_norm without
    # RoPE (:1864-1865), attention over the context, to_out with its bias
    xq = ops.fused_fp8_quantize_e4m3(attn_input, s_q)
    cq = ops.fused_fp8_quantize_e4m3(ctx, s_kv)
    q_proj = linear(xq, s_q, tw.to_q)
    k_proj = linear(cq, s_kv, tw.to_k)
    v = linear(cq, s_kv, tw.to_v)
    q = torch.nn.functional.rms_norm(q_proj, (D,), weight=tw.q_norm_weight, eps=tw.qk_eps)
    k = torch.nn.functional.rms_norm(k_proj, (D,), weight=tw.k_norm_weight, eps=tw.qk_eps)
    qh, kh, vh = (t.float().view(1, -1, 32, 128).transpose(1, 2) for t in (q, k, v))
    attn = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2).reshape(1, -1, D)
    attn = attn.to(torch.bfloat16)
    s_out = (attn.float().abs().amax() / 448.0).to(torch.float32)
    oq = ops.fused_fp8_quantize_e4m3(attn, s_out)
    y = linear(oq, s_out, tw.to_out)
    # gated residual with slot 8 (:2882-2888)
    out = ops.fused_residual_gate_from_ada(x, y, table, ts, gate_index=8, count_video_ada=False)
    np.savez_compressed(
        os.path.join(HERE, "text_xattn.npz"),
        s_q=s_q.numpy(), s_kv=s_kv.numpy(), s_out=s_out.numpy(), ctx=bits(ctx), attn_input=bits(attn_input),
        xq=xq.view(torch.uint8).numpy(), cq=cq.view(torch.uint8).numpy(), q_proj=bits(q_proj), k_proj=bits(k_proj),
        q=bits(q), k=bits(k), v=bits(v), attn=bits(attn), oq=oq.view(torch.uint8).numpy(), y=bits(y), out=bits(out),
        seed_inputs=np.array(15), seed_weights=np.array(17), tokens=np.array(16), context_tokens=np.array(24),
    )


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the plugyawn/opengenie checkout")
    ap.add_argument("--only", default=None, help="regenerate one fixture (its name without .npz)")
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ops, rope_ref = load_reference(args.reference)
    makers = {
        "quant": lambda: make_quant(ops),
        "ops": lambda: make_ops(ops, rope_ref),
        "block": lambda: make_block(ops, rope_ref),
        "gelu_quant": lambda: make_gelu(ops),
        "ffn": lambda: make_ffn(ops),
        "residual_nobias": lambda: make_residual_nobias(ops),
        "adaln_affine": lambda: make_adaln_affine(ops),
        "head_gate": lambda: make_head_gate(ops),
        "ada_misc": lambda: make_ada_misc(ops),
        "text_xattn": lambda: make_text_xattn(ops),
    }
    if args.only is not None:
        makers[args.only]()
    else:
        for make in makers.values():
            make()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
