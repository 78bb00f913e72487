"""Helpers shared by the GPU parity tests."""

import numpy as np
import torch

from oracle import ltx_block_oracle as O


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def codes(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy()


def from_bits(bits: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def within_ulps(got: np.ndarray, ref: np.ndarray, ulps: float = 1.0, atol: float = 0.0) -> tuple[bool, float]:
    """|got - ref| <= atol + ulps * bf16-ulp(ref) elementwise; returns (ok, worst ratio)."""
    ref = np.asarray(ref, np.float32)
    mag = np.maximum(np.abs(ref), np.float32(2.0 ** -126))
    ulp = np.exp2(np.floor(np.log2(mag)) - 7.0)
    bound = atol + ulps * ulp
    d = np.abs(np.asarray(got, np.float32) - ref)
    return bool((d <= bound).all()), float((d / bound).max())


def block_tolerance(got: np.ndarray, ref: np.ndarray, *, atol: float = 2e-2, mean_rel: float = 1e-2,
                    ulps: float = 1.0) -> dict:
    """The north-star tolerance: max-abs <= 2e-2 plus ``ulps`` bf16 ulps of |ref| (a bf16 output's own
    rounding is half an ulp, which exceeds 2e-2 once |out| >= 8) and sum|d| / sum|ref| <= 1e-2.
    Returns the measured figures."""
    d = np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64))
    excess = d - (atol + ulps * np.abs(ref) * 2.0 ** -7)
    ref_formula = float((d / np.maximum(np.abs(ref), 1e-6)).mean())  # the reference's own mean_rel
    return {
        "max_abs": float(d.max()),
        "max_excess": float(excess.max()),
        "mean_rel": float(d.sum() / max(np.abs(ref).sum(), 1e-30)),
        "ref_mean_rel": ref_formula,
        "ok": bool(excess.max() <= 0 and d.sum() / max(np.abs(ref).sum(), 1e-30) <= mean_rel),
    }


def reference_gpu_path_block(x, ts_view, cos, sin, w, *, eps=1e-6, heads=32):
    """The reference's production GPU path for the block, rebuilt from torch's own GPU kernels:
    single-rounding AdaZero / quantiser / RoPE (its Triton kernels, ltx_serve/triton_ltx_ops.py:3359-3444,
    :3901-3978), torch._scaled_mm with use_fast_accum (:1695-1703) + bias add, SDPA on bf16 with the
    cuDNN backend ('sdpa-cudnn', modal_apps/ltx23_live_h100_worker.py:49), the residual rounding of :3663-3721.
    Used to put the fused block's deviation from the fp32 reference next to the reference's own."""
    import torch.nn.functional as F

    def r16(t):
        return t.to(torch.bfloat16)

    table = w.scale_shift_table.float()
    if (w.scale_shift_table.dtype == torch.bfloat16) != (ts_view.dtype == torch.bfloat16):
        table = r16(table).float()
    ts = ts_view.float()

    def ada(i):
        v = table[i].view(1, 1, -1) + ts[:, :, i, :]
        return r16(v).float() if ts_view.dtype == torch.bfloat16 else v

    def quant(t, s):
        return torch.clamp(t.float() / s.float(), -448.0, 448.0).to(torch.float8_e4m3fn)

    xf = x.float()
    norm = r16(xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1 + ada(1)) + ada(0))

    def lin(q2, s_in, l, bias=True):
        y = torch._scaled_mm(q2.reshape(-1, q2.shape[-1]), l.weight.t(), scale_a=s_in, scale_b=l.weight_scale,
                             out_dtype=torch.bfloat16, use_fast_accum=True)
        if bias:
            y = r16(y.float() + r16(l.bias).float())
        return y.view(1, -1, y.shape[-1])

    q = lin(quant(norm, w.to_q.input_scale), w.to_q.input_scale, w.to_q)
    k = lin(quant(norm, w.to_k.input_scale), w.to_k.input_scale, w.to_k)
    v = lin(quant(norm, w.to_v.input_scale), w.to_v.input_scale, w.to_v)

    def rope(t, weight):
        tf = t.float()
        n = tf * torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
        B, L, D = n.shape
        nh = n.view(B, L, heads, D // heads).transpose(1, 2)
        half = D // heads // 2
        c, s_ = cos.float(), sin.float()
        f, sd = nh[..., :half], nh[..., half:]
        return r16(torch.cat([f * c - sd * s_, sd * c + f * s_], dim=-1).transpose(1, 2).reshape(B, L, D))

    qr, kr = rope(q, w.q_norm_weight), rope(k, w.k_norm_weight)
    B, L, D = qr.shape
    from torch.nn.attention import SDPBackend, sdpa_kernel

    qh, kh, vh = (t.view(B, L, heads, D // heads).transpose(1, 2) for t in (qr, kr, v))
    try:
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            o = F.scaled_dot_product_attention(qh, kh, vh)
    except RuntimeError:
        o = F.scaled_dot_product_attention(qh, kh, vh)
    attn = o.transpose(1, 2).reshape(B, L, D)
    y = lin(quant(attn, w.to_out.input_scale), w.to_out.input_scale, w.to_out, bias=False)
    yb = r16(y.float() + r16(w.to_out.bias).float())
    gate = ada(2)
    return r16(xf + r16(yb.float() * gate).float())


def accum_atol(a_codes, s_a, w_codes, s_w):
    """fp32-accumulation allowance of an FP8 GEMM against the float64 oracle:
    max(K/32, 128) * 2^-24 * sum_k |a_k w_k| * scale (the K/32 chained fp32 adds of tensor-core partial
    sums are within K/32 * 2^-24 of that sum)."""
    absdot = np.abs(O.e4m3_to_f32(a_codes).reshape(-1, a_codes.shape[-1])).astype(np.float64) @ \
        np.abs(O.e4m3_to_f32(w_codes)).astype(np.float64).T
    s_w = np.asarray(s_w, np.float64).reshape(-1)
    k = a_codes.shape[-1]
    return max(k / 32, 128) * 2.0 ** -24 * absdot * np.repeat(np.float64(s_a) * s_w, absdot.shape[1] // s_w.size)


def bf16_ulp(x) -> np.ndarray:
    mag = np.maximum(np.abs(np.asarray(x, np.float32)), np.float32(2.0 ** -126))
    return np.exp2(np.floor(np.log2(mag)) - 7.0)


def status_clean():
    from opengenie_b200 import _lib

    torch.cuda.synchronize()
    return _lib.device_status(clear=True) == 0


__all__ = ["O", "to_np", "bf16_bits", "codes", "from_bits", "within_ulps", "block_tolerance", "status_clean"]
