"""CPU oracle for the LTX-2.3 video self-attention block (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker or the timed CPU baseline; the
product path (``opengenie_b200``) never calls it.

It restates the reference's arithmetic for the hot path (plugyawn/opengenie,
ltx_serve/triton_ltx_ops.py; cited per function) with numpy for every bit-level
step (bf16 rounding, E4M3 encoding, the quantiser) and float32/float64 torch on
the CPU for the contractions (FP8 linears as dequantise -> matmul, attention as
softmax(QK^T/sqrt(d))V).

Parity pins (tests/test_oracle_golden.py):
- the quantiser against the reference's own torch path run in this container on
  every bf16 and fp16 bit pattern (tests/golden/quant_*.npz),
- AdaZero, bias add, bias+gate+residual and RoPE against the reference's torch
  fallbacks / its test restatement on seeded inputs (tests/golden/ops.npz),
- the whole block against a composition of the reference's CPU functions with
  CPU ``torch._scaled_mm`` (tests/golden/block.npz).
The generating script is tests/golden/make_golden.py.
"""

from __future__ import annotations

import numpy as np
import torch

FP8_MAX = 448.0

# ----------------------------------------------------------------------------- bit-level helpers


def bf16_round(a) -> np.ndarray:
    """fp32 -> bf16 round-to-nearest-even, returned as float32 values (NaN stays NaN, sign kept).

    The rounding of `_round_f32_to_bf16_f32` (ltx_serve/triton_ltx_ops.py:3315-3320)
    and of torch's bf16 casts.
    """
    a = np.asarray(a, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> np.uint64(16)) & np.uint64(1)
    rounded = ((bits + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.copysign(np.float32("nan"), a[nan])
    return out


def f16_round(a) -> np.ndarray:
    """fp32 -> fp16 round-to-nearest-even, returned as float32 values."""
    with np.errstate(over="ignore"):
        return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def bf16_from_bits(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_e4m3(t) -> np.ndarray:
    """float32 -> float8_e4m3fn codes, round-to-nearest-even, finite saturation at 448,
    NaN -> 0x7F with the NaN's sign bit (as torch's float8_e4m3fn cast does).

    E4M3 (bias 7): normals 2^-6 .. 448 with 3 mantissa bits, subnormals k * 2^-9.
    """
    t = np.asarray(t, dtype=np.float32).astype(np.float64)
    nan = np.isnan(t)
    sign = np.signbit(t).astype(np.uint8)
    a = np.abs(np.where(nan, 0.0, t))
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)
    quantum = np.exp2(e - 3.0)
    v = np.rint(a / quantum) * quantum  # np.rint rounds half to even
    v = np.minimum(v, FP8_MAX)
    normal = v >= 2.0 ** -6
    ev = np.floor(np.log2(np.where(normal, v, 1.0)))
    mant = np.where(normal, (v / np.exp2(ev) - 1.0) * 8.0, 0.0)
    code_n = ((ev + 7.0).astype(np.int64) << 3) | np.rint(mant).astype(np.int64)
    code_s = np.rint(v / 2.0 ** -9).astype(np.int64)
    code = np.where(normal, code_n, code_s).astype(np.uint8) | (sign << 7)
    code[nan] = 0x7F | (sign[nan] << 7)
    return code.astype(np.uint8)


def e4m3_to_f32(codes) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
    return np.copysign(val, sign).astype(np.float32)


def quantize_e4m3(x, input_scale: float, *, in_dtype: str = "bf16", mode: str = "torch") -> np.ndarray:
    """Per-tensor E4M3 quantiser.

    mode="torch":  the reference's torch path, ltx_serve/triton_ltx_ops.py:146-148,
                   ``clamp(x * input_scale.reciprocal(), -448, 448).to(e4m3)`` on a bf16
                   (or fp16) tensor: r = 1/s in fp32, the product rounded once to the
                   input dtype, clamp (NaN passes), RNE cast.  torch's vectorised
                   fp32->bf16 cast turns every NaN into 0xFFFF, so on bf16 input every
                   NaN quantises to 0xFF; fp16 keeps the NaN's sign (0x7F / 0xFF).
    mode="single": the reference's Triton kernel, :3429-3444: e4m3(clamp(x_f32 / s)).
    ``x`` holds float32 values exactly representable in ``in_dtype``.
    """
    x = np.asarray(x, dtype=np.float32)
    s = np.float32(input_scale)
    np_err = np.seterr(invalid="ignore", over="ignore")
    if mode == "torch":
        r = np.float32(1.0) / s
        t = x * r
        if in_dtype == "bf16":
            t = bf16_round(t)
            t = np.where(np.isnan(t), np.float32(-np.nan), t)
        else:
            t = f16_round(t)
    elif mode == "single":
        t = x / s
    else:
        raise ValueError(mode)
    t = np.where(np.isnan(t), t, np.clip(t, -FP8_MAX, FP8_MAX))
    np.seterr(**np_err)
    return f32_to_e4m3(t)


def gelu_tanh(x, *, in_dtype: str = "bf16") -> np.ndarray:
    """``torch.nn.functional.gelu(x, approximate="tanh")`` on a bf16 (or fp16) tensor on the CPU, as the
    reference's torch path evaluates it (ltx_serve/triton_ltx_ops.py:166): fp32 math, one rounding to the
    input dtype.  Returned as float32 values exactly representable in ``in_dtype``."""
    dt = torch.bfloat16 if in_dtype == "bf16" else torch.float16
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dt)
    return torch.nn.functional.gelu(t, approximate="tanh").float().numpy()


def gelu_tanh_quantize_e4m3(x, input_scale: float, *, in_dtype: str = "bf16") -> np.ndarray:
    """``fused_gelu_tanh_fp8_quantize_e4m3`` torch path (ltx_serve/triton_ltx_ops.py:164-169): GELU (tanh)
    rounded to the input dtype, then the torch-path quantiser on that tensor."""
    return quantize_e4m3(gelu_tanh(x, in_dtype=in_dtype), input_scale, in_dtype=in_dtype)


# ----------------------------------------------------------------------------- Ada / elementwise


def _np(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        return t.detach().to("cpu", torch.float32).numpy()
    return np.asarray(t, dtype=np.float32)


def ada_value(table, ts_view, index: int, *, table_is_bf16: bool, ts_is_bf16: bool) -> np.ndarray:
    """``table.to(ts.dtype)[idx] + ts[:, :, idx, :]``; reference `_torch_ada_values_from_table`,
    ltx_serve/triton_ltx_ops.py:983-998 (rounding flags as in the kernel :3359-3427)."""
    tab = _np(table)[index]
    if table_is_bf16 != ts_is_bf16:
        tab = bf16_round(tab)
    v = tab[None, None, :] + _np(ts_view)[:, :, index, :]
    return bf16_round(v) if ts_is_bf16 else v.astype(np.float32)


def adazero_from_ada(x, eps, table, ts_view, *, shift_index: int, scale_index: int, table_is_bf16=False, ts_is_bf16=True):
    """rmsnorm(x) * (1 + scale) + shift, exact math, one bf16 rounding.

    The semantics of the reference's GPU kernel `_adazero_from_ada_kernel`
    (ltx_serve/triton_ltx_ops.py:3359-3427); the torch fallback (:51-60 -> :9-10)
    rounds after every op and agrees within the reference's test tolerance (0.0625).
    """
    xf = _np(x).astype(np.float64)
    shift = ada_value(table, ts_view, shift_index, table_is_bf16=table_is_bf16, ts_is_bf16=ts_is_bf16)
    scale = ada_value(table, ts_view, scale_index, table_is_bf16=table_is_bf16, ts_is_bf16=ts_is_bf16)
    inv = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + eps)
    y = xf * inv * (1.0 + scale.astype(np.float64)) + shift.astype(np.float64)
    return bf16_round(y.astype(np.float32))


def adazero_explicit(x, eps, scale, shift) -> np.ndarray:
    """``fused_adazero`` (ltx_serve/triton_ltx_ops.py:8-37, GPU kernel :3319-3357): rmsnorm(x) * (1 + scale)
    + shift with explicit scale/shift rows (broadcast over the rows of x), exact math, one bf16 rounding."""
    xf = _np(x).astype(np.float64)
    inv = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + eps)
    y = xf * inv * (1.0 + _np(scale).astype(np.float64)) + _np(shift).astype(np.float64)
    return bf16_round(y.astype(np.float32))


def mul_from_ada(x, table, ts_view, *, gate_index: int, table_is_bf16=False, ts_is_bf16=True) -> np.ndarray:
    """``fused_mul_from_ada`` (ltx_serve/triton_ltx_ops.py:695-741, kernel :3723-3771): bf16(x * gate)."""
    gate = ada_value(table, ts_view, gate_index, table_is_bf16=table_is_bf16, ts_is_bf16=ts_is_bf16)
    return bf16_round(_np(x).astype(np.float32) * gate)


def residual_gate_bf16(x, y, gate) -> np.ndarray:
    """``fused_residual_gate_bf16`` (ltx_serve/triton_ltx_ops.py:590-611, kernel :3552-3582):
    bf16(x + bf16(y * gate))."""
    return bf16_round(_np(x).astype(np.float32) + bf16_round(_np(y).astype(np.float32) * _np(gate).astype(np.float32)))


def head_gate_mul_bf16(out, gates, heads: int, dim_head: int) -> np.ndarray:
    """``fused_head_gate_mul_bf16``, ltx_serve/triton_ltx_ops.py:614-637: bf16(out * gate[head])."""
    o = _np(out).astype(np.float32)
    B, L, _ = o.shape
    g = _np(gates).astype(np.float32).reshape(B, L, heads, 1)
    return bf16_round(o.reshape(B, L, heads, dim_head) * g).reshape(B, L, heads * dim_head)


def adaln_affine_from_ada(x, table, ts_view, *, shift_index: int, scale_index: int, table_is_bf16=False,
                          ts_is_bf16=True) -> np.ndarray:
    """``fused_adaln_affine_from_ada``, ltx_serve/triton_ltx_ops.py:94-141 (kernel :3469-3534):
    bf16(bf16(x * bf16(1 + scale)) + shift), Ada values rounded as in ``ada_value``."""
    shift = ada_value(table, ts_view, shift_index, table_is_bf16=table_is_bf16, ts_is_bf16=ts_is_bf16)
    scale = ada_value(table, ts_view, scale_index, table_is_bf16=table_is_bf16, ts_is_bf16=ts_is_bf16)
    factor = bf16_round(np.float32(1.0) + scale)
    return bf16_round(bf16_round(_np(x).astype(np.float32) * factor) + shift)


def bias_add_bf16(x, bias) -> np.ndarray:
    """bf16(x + bf16(bias)); ltx_serve/triton_ltx_ops.py:3446-3464."""
    return bf16_round(_np(x) + bf16_round(_np(bias)))


def residual_gate_bias(x, y, bias, gate) -> np.ndarray:
    """bf16(x + bf16(bf16(y + bf16(bias)) * gate)); ltx_serve/triton_ltx_ops.py:3663-3721."""
    yb = bf16_round(_np(y) + bf16_round(_np(bias)))
    prod = bf16_round(yb * _np(gate))
    return bf16_round(_np(x) + prod)


def residual_gate_bias_from_ada(x, y, bias, table, ts_view, *, gate_index: int, table_is_bf16=False, ts_is_bf16=True):
    gate = ada_value(table, ts_view, gate_index, table_is_bf16=table_is_bf16, ts_is_bf16=ts_is_bf16)
    return residual_gate_bias(x, y, bias, gate)


def qk_rmsnorm_rope(x, weight, eps, cos, sin) -> np.ndarray:
    """RMSNorm over the full row with weight, then split RoPE per head, exact math, one bf16 rounding.

    ltx_serve/triton_ltx_ops.py:3901-3978; the reference's test restatement is
    tests/test_triton_ltx_ops.py:232-249.  x [1, L, H*d], cos/sin [1, H, L, d/2].
    """
    xf = _np(x).astype(np.float64)
    w = _np(weight).astype(np.float64)
    inv = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + eps)
    n = xf * inv * w
    B, L, D = n.shape
    H = _np(cos).shape[1]
    hd = D // H
    half = hd // 2
    nh = n.reshape(B, L, H, hd)
    c = _np(cos).astype(np.float64).transpose(0, 2, 1, 3)  # [1, L, H, half]
    s = _np(sin).astype(np.float64).transpose(0, 2, 1, 3)
    first, second = nh[..., :half], nh[..., half:]
    out = np.concatenate([first * c - second * s, second * c + first * s], axis=-1)
    return bf16_round(out.reshape(B, L, D).astype(np.float32))


def qk_rmsnorm(x, weight, eps) -> np.ndarray:
    """RMSNorm over the full row with weight and no rotation, exact math, one bf16 rounding.

    The pre-attention when no positional embedding is given, ``attn.q_norm(q)`` / ``attn.k_norm(k)``
    (ltx_serve/triton_ltx_ops.py:1864-1865: the text cross-attention), restated with the arithmetic of
    ``qk_rmsnorm_rope`` (the reference's fused Q/K kernel, :3901-3978) without the rotation.
    """
    xf = _np(x).astype(np.float64)
    w = _np(weight).astype(np.float64)
    inv = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + eps)
    return bf16_round((xf * inv * w).astype(np.float32))


# ----------------------------------------------------------------------------- contractions


def fp8_linear(qcodes, input_scale: float, wcodes, weight_scale, bias=None) -> np.ndarray:
    """bf16(acc * s_in * s_w) (+ bf16(bias) with another bf16 rounding).

    `torch._scaled_mm(q, W.t(), scale_a, scale_b, out_dtype=bf16)` (+ `fused_bias_add_bf16`),
    ltx_serve/triton_ltx_ops.py:1695-1707; e4m3 products are exact, the sum is
    accumulated in float64 here.  ``weight_scale`` may be an array with one entry per
    equal column segment.
    """
    a = torch.from_numpy(e4m3_to_f32(qcodes).astype(np.float64))
    w = torch.from_numpy(e4m3_to_f32(wcodes).astype(np.float64))
    acc = (a.reshape(-1, a.shape[-1]) @ w.T).numpy()
    ws = np.asarray(weight_scale, dtype=np.float32).reshape(-1)
    seg = acc.shape[1] // ws.size
    scale = np.repeat(np.float32(input_scale) * ws, seg).astype(np.float32)
    y = bf16_round((acc * scale.astype(np.float64)).astype(np.float32))
    if bias is not None:
        y = bias_add_bf16(y, bias)
    return y.reshape(*np.shape(qcodes)[:-1], -1)


def attention(q, k, v, heads: int, scale: float | None = None) -> np.ndarray:
    """softmax(q k^T * scale) v per head in float64 (returned as float32, not rounded).

    The attention backend contract, benchmarks/official_ltx23_benchmark.py:3289-3373.
    q [B, L, H*d]; k/v [B, L_kv, H*d] (L_kv != L for the text cross-attention, whose keys come
    from the prompt context; the backend views k and v as [b, -1, heads, d], :3305).
    """
    qt = torch.from_numpy(_np(q).astype(np.float64))
    kt = torch.from_numpy(_np(k).astype(np.float64))
    vt = torch.from_numpy(_np(v).astype(np.float64))
    B, L, D = qt.shape
    d = D // heads
    sc = d ** -0.5 if scale is None else scale
    qh = qt.view(B, L, heads, d).transpose(1, 2)
    kh = kt.view(B, -1, heads, d).transpose(1, 2)
    vh = vt.view(B, -1, heads, d).transpose(1, 2)
    out = torch.empty_like(qh)
    for h in range(heads):  # one head at a time keeps the L x L_kv scores small
        s = (qh[:, h] @ kh[:, h].transpose(-1, -2)) * sc
        p = torch.softmax(s, dim=-1)
        out[:, h] = p @ vh[:, h]
    return out.transpose(1, 2).reshape(B, L, D).numpy().astype(np.float32)


def attention_fp32_torch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int) -> torch.Tensor:
    """Fast fp32 CPU attention (torch SDPA math) for the timed CPU baseline; k/v may be shorter than q."""
    B, L, D = q.shape
    d = D // heads
    qh = q.float().view(B, L, heads, d).transpose(1, 2)
    kh, vh = (t.float().view(B, -1, heads, d).transpose(1, 2) for t in (k, v))
    o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)
    return o.transpose(1, 2).reshape(B, L, D)


# ----------------------------------------------------------------------------- the block


def block_qkv(norm, w, *, qk_eps: float = 1e-6, cos=None, sin=None):
    """Stage 2-3 of the block: per-linear E4M3 quant -> FP8 Q/K/V + bias -> Q/K RMSNorm + RoPE.

    FP8Linear.forward per projection (ltx_serve/triton_ltx_ops.py:1676-1716) then
    fused_video_qk_rmsnorm_rope (:320-378).  Returns bf16-valued q, k (roped) and v.
    """
    proj = []
    for lin in (w.to_q, w.to_k, w.to_v):
        s_in = float(lin.input_scale)
        xq = quantize_e4m3(norm, s_in)
        proj.append(fp8_linear(xq, s_in, lin.weight.view(torch.uint8).numpy(), float(lin.weight_scale), _np(lin.bias)))
    q, k, v = proj
    return qk_rmsnorm_rope(q, w.q_norm_weight, qk_eps, cos, sin), qk_rmsnorm_rope(k, w.k_norm_weight, qk_eps, cos, sin), v


def block_epilogue(x, attn_bf16, w, table, timestep_view):
    """Stage 5-6: E4M3 quant of the attention output -> FP8 out-proj (no bias) ->
    bias + gate (idx 2) + residual (:762-781, :204-262)."""
    tab_bf16 = table.dtype == torch.bfloat16
    ts_bf16 = timestep_view.dtype == torch.bfloat16
    s_out = float(w.to_out.input_scale)
    oq = quantize_e4m3(attn_bf16, s_out)
    y = fp8_linear(oq, s_out, w.to_out.weight.view(torch.uint8).numpy(), float(w.to_out.weight_scale))
    out = residual_gate_bias_from_ada(x, y, _np(w.to_out.bias), table, timestep_view, gate_index=2,
                                      table_is_bf16=tab_bf16, ts_is_bf16=ts_bf16)
    return out, y


def video_block(x, timestep_view, cos, sin, w, *, eps: float = 1e-6, qk_eps: float = 1e-6, heads: int = 32,
                return_intermediates: bool = False):
    """The video self-attention block in the reference's order and rounding points.

    `_video_msa_branch_from_ada` (ltx_serve/triton_ltx_ops.py:2891-2981) with the
    production flags: AdaZero idx 0/1 -> per-linear E4M3 quant -> FP8 Q/K/V + bias ->
    Q/K RMSNorm + split RoPE -> attention -> quant -> FP8 out-proj (no bias) ->
    bias + gate (idx 2) + residual.  ``w`` carries the synthetic BlockWeights
    (e4m3 weights with per-tensor scales, biases, norm weights, table).
    """
    table = w.scale_shift_table
    tab_bf16 = table.dtype == torch.bfloat16
    ts_bf16 = timestep_view.dtype == torch.bfloat16
    norm = adazero_from_ada(x, eps, table, timestep_view, shift_index=0, scale_index=1, table_is_bf16=tab_bf16,
                            ts_is_bf16=ts_bf16)
    qr, kr, v = block_qkv(norm, w, qk_eps=qk_eps, cos=cos, sin=sin)
    attn = attention(qr, kr, v, heads)
    attn_bf16 = bf16_round(attn)
    out, y = block_epilogue(x, attn_bf16, w, table, timestep_view)
    if return_intermediates:
        return out, {"norm": norm, "q": qr, "k": kr, "v": v, "attn": attn, "attn_bf16": attn_bf16, "y": y}
    return out


def video_block_cpu_fp32(x: torch.Tensor, timestep_view: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, w, *,
                         eps: float = 1e-6, qk_eps: float = 1e-6, heads: int = 32,
                         calibrate: bool = False) -> torch.Tensor:
    """The same block on CPU torch in float32 (multi-threaded), used as the timed CPU baseline.

    Same stages and rounding points as ``video_block`` (torch ops instead of float64
    numpy), so it runs at full-size configurations in seconds, not hours.  With
    ``calibrate`` the static input scales are first set from this input the way the
    GPU block calibrates them: amax/448 of the AdaZero output for to_q/to_k/to_v and
    of the bf16 attention output for to_out (written into ``w``).
    """
    def r16(t):
        return t.to(torch.bfloat16).float()

    table = w.scale_shift_table.float()
    if (w.scale_shift_table.dtype == torch.bfloat16) != (timestep_view.dtype == torch.bfloat16):
        table = r16(table)
    ts = timestep_view.float()

    def ada(idx):
        v = table[idx].view(1, 1, -1) + ts[:, :, idx, :]
        return r16(v) if timestep_view.dtype == torch.bfloat16 else v

    xf = x.float()
    norm = r16(xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1 + ada(1)) + ada(0))
    if calibrate:
        s_in = (norm.abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
        for lin_ in (w.to_q, w.to_k, w.to_v):
            lin_.input_scale = s_in.clone()

    def quant(t, s):
        r = torch.tensor(1.0, dtype=torch.float32) / s.float()
        return torch.clamp(r16(t * r), -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)

    def lin(tq, s_in, l, bias=True):
        acc = tq.reshape(-1, tq.shape[-1]).float() @ l.weight.float().T
        y = r16(acc * (s_in.float() * l.weight_scale.float()))
        if bias:
            y = r16(y + r16(l.bias.float()))
        return y.view(*tq.shape[:-1], -1)

    xq = quant(norm, w.to_q.input_scale)
    q = lin(xq, w.to_q.input_scale, w.to_q)
    k = lin(xq if torch.equal(w.to_k.input_scale, w.to_q.input_scale) else quant(norm, w.to_k.input_scale),
            w.to_k.input_scale, w.to_k)
    v = lin(xq if torch.equal(w.to_v.input_scale, w.to_q.input_scale) else quant(norm, w.to_v.input_scale),
            w.to_v.input_scale, w.to_v)

    def rope(t, weight):
        n = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + qk_eps) * weight.float()
        B, L, D = n.shape
        H = cos.shape[1]
        nh = n.view(B, L, H, D // H).transpose(1, 2)
        half = D // H // 2
        c, s = cos.float(), sin.float()
        f, sd = nh[..., :half], nh[..., half:]
        o = torch.cat([f * c - sd * s, sd * c + f * s], dim=-1)
        return r16(o.transpose(1, 2).reshape(B, L, D))

    qr, kr = rope(q, w.q_norm_weight), rope(k, w.k_norm_weight)
    attn = r16(attention_fp32_torch(qr, kr, v, heads))
    if calibrate:
        w.to_out.input_scale = (attn.abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
    oq = quant(attn, w.to_out.input_scale)
    y = lin(oq, w.to_out.input_scale, w.to_out, bias=False)
    gate = ada(2)
    yb = r16(y + r16(w.to_out.bias.float()))
    return r16(xf + r16(yb * gate))


# ----------------------------------------------------------------------------- the video FFN branch


def video_ffn(x, timestep_view, fw, *, eps: float = 1e-6, return_intermediates: bool = False):
    """The video feed-forward branch in the reference's order and rounding points.

    ltx_serve/triton_ltx_ops.py:3224-3258 with the production flags: AdaZero idx 3/4
    (``fused_adazero_from_ada``) -> ``ff.net[0]``: E4M3 quant + FP8 proj + bias (FP8Linear.forward
    :1676-1716) and GELU tanh -> ``ff.net[2]`` without bias (``_feedforward_without_out_bias``
    :2796-2807: ``fp8_linear_without_bias`` :762-781) -> bias + gate (idx 5) + residual
    (``fused_residual_gate_bias_from_ada`` :204-262).  ``fw`` carries the synthetic FfnWeights.
    """
    table = fw.scale_shift_table
    tab_bf16 = table.dtype == torch.bfloat16
    ts_bf16 = timestep_view.dtype == torch.bfloat16
    norm = adazero_from_ada(x, eps, table, timestep_view, shift_index=3, scale_index=4, table_is_bf16=tab_bf16,
                            ts_is_bf16=ts_bf16)
    s1 = float(fw.proj.input_scale)
    xq = quantize_e4m3(norm, s1)
    hidden = fp8_linear(xq, s1, fw.proj.weight.view(torch.uint8).numpy(), float(fw.proj.weight_scale),
                        _np(fw.proj.bias))
    g = gelu_tanh(hidden)
    s2 = float(fw.out.input_scale)
    hq = quantize_e4m3(g, s2)
    y = fp8_linear(hq, s2, fw.out.weight.view(torch.uint8).numpy(), float(fw.out.weight_scale))
    out = residual_gate_bias_from_ada(x, y, _np(fw.out.bias), table, timestep_view, gate_index=5,
                                      table_is_bf16=tab_bf16, ts_is_bf16=ts_bf16)
    if return_intermediates:
        return out, {"norm": norm, "xq": xq, "hidden": hidden, "gelu": g, "hq": hq, "y": y}
    return out


def video_ffn_cpu_fp32(x: torch.Tensor, timestep_view: torch.Tensor, fw, *, eps: float = 1e-6,
                      calibrate: bool = False) -> torch.Tensor:
    """The same branch with every contraction in fp32 torch (on the tensors' device): the timed CPU
    baseline and the fp32 reference of the full-size GPU tolerance test.  Same stages and rounding
    points as ``video_ffn``; the quantisers keep the reference's torch-path semantics (activations are
    FP8 in the model), with 1/s kept in fp32 as the reference's CPU path computes it.  With
    ``calibrate`` the two input scales are first set to amax/448 of the AdaZero output and of the GELU
    output, as the GPU branch calibrates them (written into ``fw``)."""
    dev = x.device

    def r16(t):
        return t.to(torch.bfloat16).float()

    table = fw.scale_shift_table.to(dev).float()
    if (fw.scale_shift_table.dtype == torch.bfloat16) != (timestep_view.dtype == torch.bfloat16):
        table = r16(table)
    ts = timestep_view.to(dev).float()

    def ada(idx):
        v = table[idx].view(1, 1, -1) + ts[:, :, idx, :]
        return r16(v) if timestep_view.dtype == torch.bfloat16 else v

    xf = x.float()
    norm = r16(xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1 + ada(4)) + ada(3))

    def quant(t, s):
        r = torch.tensor(1.0, dtype=torch.float32, device=dev) / s.to(dev).float()
        return torch.clamp(r16(t * r), -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)

    def lin(tq, s_in, l, bias=True):
        acc = tq.reshape(-1, tq.shape[-1]).float() @ l.weight.to(dev).float().T
        y = r16(acc * (s_in.to(dev).float() * l.weight_scale.to(dev).float()))
        if bias:
            y = r16(y + r16(l.bias.to(dev).float()))
        return y.view(*tq.shape[:-1], -1)

    if calibrate:
        fw.proj.input_scale = (norm.abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
    hidden = lin(quant(norm, fw.proj.input_scale), fw.proj.input_scale, fw.proj)
    g = torch.nn.functional.gelu(hidden.to(torch.bfloat16), approximate="tanh").float()
    if calibrate:
        fw.out.input_scale = (g.abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
    y = lin(quant(g, fw.out.input_scale), fw.out.input_scale, fw.out, bias=False)
    yb = r16(y + r16(fw.out.bias.to(dev).float()))
    return r16(xf + r16(yb * ada(5))).to(torch.bfloat16)


# ----------------------------------------------------------------------------- the video text cross-attention


def video_text_cross_attention(x, timestep_view, context, prompt_timestep_view, tw, *, heads: int = 32,
                               return_intermediates: bool = False):
    """The video branch's text cross-attention (attn2) with cross-attention AdaLN, in the reference's order and
    rounding points.

    `_apply_video_text_cross_attention_adaln_from_ada` (ltx_serve/triton_ltx_ops.py:2810-2888) with the
    production flags: the context through ``fused_adaln_affine_from_ada`` with the prompt table (slots 0/1,
    :2842-2851); x through RMSNorm and the Ada affine of slots 6/7 (:2856-2862), here as the fused
    ``adazero_from_ada`` of the reference's other cross-attention path (``fused_adazero``, :1780); then
    ``attn(attn_input, context=...)`` (:2880; ``_attention_without_out_bias`` declines without a positional
    embedding, :2574): FP8Linear.forward for to_q on x and to_k/to_v on the context (:1676-1716), Q/K RMSNorm
    without RoPE (:1864-1865), attention over the context, to_out with its bias; and
    ``fused_residual_gate_from_ada`` with slot 8 (:2882-2888): bf16(x + bf16(out * gate)).
    ``timestep_view`` is [1, L, 9, D], ``prompt_timestep_view`` [1, L_ctx, 2, D]; ``tw`` carries the
    synthetic TextAttentionWeights.
    """
    table = tw.scale_shift_table
    tab_bf16 = table.dtype == torch.bfloat16
    ts_bf16 = timestep_view.dtype == torch.bfloat16
    ptab = tw.prompt_scale_shift_table
    ctx = adaln_affine_from_ada(context, ptab, prompt_timestep_view, shift_index=0, scale_index=1,
                                table_is_bf16=ptab.dtype == torch.bfloat16,
                                ts_is_bf16=prompt_timestep_view.dtype == torch.bfloat16)
    norm = adazero_from_ada(x, tw.norm_eps, table, timestep_view, shift_index=6, scale_index=7,
                            table_is_bf16=tab_bf16, ts_is_bf16=ts_bf16)

    def linear(inp, lin, bias=True):
        s_in = float(lin.input_scale)
        return fp8_linear(quantize_e4m3(inp, s_in), s_in, lin.weight.view(torch.uint8).numpy(), float(lin.weight_scale),
                          _np(lin.bias) if bias else None)

    q = qk_rmsnorm(linear(norm, tw.to_q), tw.q_norm_weight, tw.qk_eps)
    k = qk_rmsnorm(linear(ctx, tw.to_k), tw.k_norm_weight, tw.qk_eps)
    v = linear(ctx, tw.to_v)
    attn = attention(q, k, v, heads)
    attn_bf16 = bf16_round(attn)
    y = linear(attn_bf16, tw.to_out)  # to_out with its bias: bf16(bf16(acc) + bf16(bias))
    gate = ada_value(table, timestep_view, 8, table_is_bf16=tab_bf16, ts_is_bf16=ts_bf16)
    out = residual_gate_bf16(x, y, gate)
    if return_intermediates:
        return out, {"ctx": ctx, "norm": norm, "q": q, "k": k, "v": v, "attn": attn, "attn_bf16": attn_bf16, "y": y}
    return out


def video_text_cross_attention_cpu_fp32(x: torch.Tensor, timestep_view: torch.Tensor, context: torch.Tensor,
                                        prompt_timestep_view: torch.Tensor, tw, *, heads: int = 32,
                                        calibrate: bool = False) -> torch.Tensor:
    """The same branch on CPU torch in float32 (multi-threaded): same stages and rounding points as
    ``video_text_cross_attention``, fp32 contractions, so full-size configurations finish in seconds.
    With ``calibrate`` the input scales are first set to amax/448 of each linear's input (the AdaZero
    output for to_q, the context after its affine for to_k/to_v, the attention output for to_out), as
    the GPU branch calibrates them (written into ``tw``)."""
    def r16(t):
        return t.to(torch.bfloat16).float()

    def ada_fn(table, ts_view):
        tab = table.float()
        if (table.dtype == torch.bfloat16) != (ts_view.dtype == torch.bfloat16):
            tab = r16(tab)
        ts = ts_view.float()

        def ada(idx):
            v = tab[idx].view(1, 1, -1) + ts[:, :, idx, :]
            return r16(v) if ts_view.dtype == torch.bfloat16 else v
        return ada

    ada = ada_fn(tw.scale_shift_table, timestep_view)
    pada = ada_fn(tw.prompt_scale_shift_table, prompt_timestep_view)
    xf = x.float()
    ctx = r16(r16(context.float() * r16(1 + pada(1))) + pada(0))
    norm = r16(xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + tw.norm_eps) * (1 + ada(7)) + ada(6))

    def quant(t, s):
        r = torch.tensor(1.0, dtype=torch.float32) / s.float()
        return torch.clamp(r16(t * r), -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)

    def lin(t, l):
        tq = quant(t, l.input_scale)
        acc = tq.reshape(-1, tq.shape[-1]).float() @ l.weight.float().T
        y = r16(acc * (l.input_scale.float() * l.weight_scale.float()))
        y = r16(y + r16(l.bias.float()))
        return y.view(*t.shape[:-1], -1)

    def rms(t, weight):
        return r16(t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + tw.qk_eps) * weight.float())

    def amax_scale(t):
        return (t.abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)

    if calibrate:
        tw.to_q.input_scale = amax_scale(norm)
        tw.to_k.input_scale = amax_scale(ctx)
        tw.to_v.input_scale = tw.to_k.input_scale.clone()
    q = rms(lin(norm, tw.to_q), tw.q_norm_weight)
    k = rms(lin(ctx, tw.to_k), tw.k_norm_weight)
    v = lin(ctx, tw.to_v)
    attn = r16(attention_fp32_torch(q, k, v, heads))
    if calibrate:
        tw.to_out.input_scale = amax_scale(attn)
    y = lin(attn, tw.to_out)
    return r16(xf + r16(y * ada(8)))
