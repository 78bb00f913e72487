"""B200-native operator surface of the LTX-2.3 video self-attention block.

Drop-in counterparts of the hot-path functions of ``ltx_serve/triton_ltx_ops.py``
(same names, argument meaning and reason strings).  Every op runs a hand-written
sm_100a kernel through the C ABI in ``libogx.so``.  Where the reference's guard
would fall back to eager torch, these ops raise ``ValueError(reason)``: there is
no CPU or torch fallback.

Ownership follows the reference wrappers: outputs are allocated here with
``torch.empty_like`` / ``torch.empty`` on the input's device and the kernels
only read inputs and write outputs, on the current CUDA stream.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import DTYPE_BF16, DTYPE_F16, DTYPE_F32, QUANT_SINGLE, QUANT_TORCH

# Call counters, as the reference keeps them (triton_ltx_ops.py:1902-1946).
_VIDEO_ADA_VALUES_CALLS = 0
_VIDEO_TEXT_ADALN_CALLS = 0

_DTYPE_CODES = {torch.bfloat16: DTYPE_BF16, torch.float32: DTYPE_F32, torch.float16: DTYPE_F16}


def _code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {t.dtype}") from exc


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("device: the B200 ops need CUDA tensors (there is no CPU path)")


# ---------------------------------------------------------------- guards (reference reason strings)
def ada_from_table_guard_reason(x: torch.Tensor, scale_shift_table: torch.Tensor, timestep: torch.Tensor) -> str | None:
    """Mirrors `_can_use_ada_from_table` (ltx_serve/triton_ltx_ops.py:1001-1018) as a reason string."""
    if not x.is_cuda or not x.is_contiguous() or x.dtype != torch.bfloat16:
        return "x_device_or_dtype"
    if x.ndim != 3 or x.shape[-1] not in (2048, 4096):
        return "x_shape"
    if not scale_shift_table.is_cuda or scale_shift_table.dtype not in (torch.bfloat16, torch.float32):
        return "table_device_or_dtype"
    if scale_shift_table.ndim != 2 or scale_shift_table.shape[-1] != x.shape[-1]:
        return "table_shape"
    if scale_shift_table.stride(-1) != 1:
        return "table_stride"
    if not timestep.is_cuda or timestep.dtype not in (torch.bfloat16, torch.float32) or timestep.ndim < 2:
        return "timestep_device_or_dtype"
    if timestep.shape[0] != x.shape[0] or timestep.shape[1] != x.shape[1]:
        return "timestep_shape"
    if timestep.numel() != x.shape[0] * x.shape[1] * scale_shift_table.shape[0] * x.shape[-1]:
        return "timestep_numel"
    return None


def _ts_view(x: torch.Tensor, table: torch.Tensor, timestep: torch.Tensor) -> torch.Tensor:
    ts_view = timestep.reshape(x.shape[0], timestep.shape[1], table.shape[0], x.shape[-1])
    if ts_view.stride(-1) != 1:
        ts_view = ts_view.contiguous()
    return ts_view


def _check_index(table: torch.Tensor, *indices: int) -> None:
    for idx in indices:
        if not 0 <= idx < table.shape[0]:
            raise ValueError("ada_index")


# ---------------------------------------------------------------- AdaZero
def fused_adazero_from_ada(
    x: torch.Tensor,
    eps: float,
    scale_shift_table: torch.Tensor,
    timestep: torch.Tensor,
    *,
    shift_index: int,
    scale_index: int,
    counter: str = "video",
) -> torch.Tensor:
    """`rmsnorm(x)*(1+scale)+shift` with shift/scale from the table + timestep.

    Reference: fused_adazero_from_ada, ltx_serve/triton_ltx_ops.py:40-91 (GPU kernel
    :3359-3427: fp32 math, one bf16 rounding).
    """
    global _VIDEO_ADA_VALUES_CALLS
    reason = ada_from_table_guard_reason(x, scale_shift_table, timestep)
    if reason is not None:
        raise ValueError(reason)
    _check_index(scale_shift_table, shift_index, scale_index)
    if counter == "video":
        _VIDEO_ADA_VALUES_CALLS += 1
    ts_view = _ts_view(x, scale_shift_table, timestep)
    y = torch.empty_like(x)
    _lib.call(
        "ogx_adazero_from_ada",
        x.data_ptr(), x.shape[0], x.shape[1], x.shape[2],
        scale_shift_table.data_ptr(), _code(scale_shift_table), scale_shift_table.stride(0),
        ts_view.data_ptr(), _code(ts_view), ts_view.stride(0), ts_view.stride(1), ts_view.stride(2),
        shift_index, scale_index, float(eps), y.data_ptr(), _stream(x),
    )
    return y


def fused_adaln_affine_from_ada(
    x: torch.Tensor,
    scale_shift_table: torch.Tensor,
    timestep: torch.Tensor,
    *,
    shift_index: int,
    scale_index: int,
) -> torch.Tensor:
    """`x*(1+scale)+shift` (no norm) with shift/scale from the table + timestep, bf16 rounding after each op.

    Reference: fused_adaln_affine_from_ada, ltx_serve/triton_ltx_ops.py:94-141 (GPU kernel :3469-3534).
    """
    global _VIDEO_TEXT_ADALN_CALLS
    reason = ada_from_table_guard_reason(x, scale_shift_table, timestep)
    if reason is not None:
        raise ValueError(reason)
    _check_index(scale_shift_table, shift_index, scale_index)
    _VIDEO_TEXT_ADALN_CALLS += 1
    ts_view = _ts_view(x, scale_shift_table, timestep)
    y = torch.empty_like(x)
    _lib.call(
        "ogx_adaln_affine_from_ada",
        x.data_ptr(), x.shape[0], x.shape[1], x.shape[2],
        scale_shift_table.data_ptr(), _code(scale_shift_table), scale_shift_table.stride(0),
        ts_view.data_ptr(), _code(ts_view), ts_view.stride(0), ts_view.stride(1), ts_view.stride(2),
        shift_index, scale_index, y.data_ptr(), _stream(x),
    )
    return y


def fused_mul_from_ada(
    x: torch.Tensor,
    scale_shift_table: torch.Tensor,
    timestep: torch.Tensor,
    *,
    gate_index: int,
) -> torch.Tensor:
    """``x * gate`` (bf16) with the gate from the table + timestep.

    Reference: fused_mul_from_ada, ltx_serve/triton_ltx_ops.py:695-741 (GPU kernel :3723-3771).
    """
    global _VIDEO_TEXT_ADALN_CALLS
    reason = ada_from_table_guard_reason(x, scale_shift_table, timestep)
    if reason is not None:
        raise ValueError(reason)
    _check_index(scale_shift_table, gate_index)
    _VIDEO_TEXT_ADALN_CALLS += 1
    ts_view = _ts_view(x, scale_shift_table, timestep)
    y = torch.empty_like(x)
    _lib.call(
        "ogx_mul_from_ada",
        x.data_ptr(), x.shape[0], x.shape[1], x.shape[2],
        scale_shift_table.data_ptr(), _code(scale_shift_table), scale_shift_table.stride(0),
        ts_view.data_ptr(), _code(ts_view), ts_view.stride(0), ts_view.stride(1), ts_view.stride(2),
        gate_index, y.data_ptr(), _stream(x),
    )
    return y


def _row_broadcast(v: torch.Tensor, batch: int, tokens: int, reason: str) -> torch.Tensor:
    """[S, D] per-row values (S = 1, batch or batch*tokens, the row mapping of the reference's explicit-value
    kernels) as a [batch, tokens, ..., D]-indexable view without copying."""
    D = v.shape[-1]
    flat = v.reshape(-1, *v.shape[-2:]) if v.ndim >= 3 and v.shape[-2] != D else v.reshape(-1, D)
    S = flat.shape[0]
    if S == 1:
        return flat.reshape(1, 1, *flat.shape[1:]).expand(batch, tokens, *flat.shape[1:])
    if S == batch:
        return flat.reshape(batch, 1, *flat.shape[1:]).expand(batch, tokens, *flat.shape[1:])
    if S == batch * tokens:
        return flat.reshape(batch, tokens, *flat.shape[1:])
    raise ValueError(reason)


def fused_adazero(x: torch.Tensor, eps: float, scale: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    """``rmsnorm(x)*(1+scale)+shift`` with explicit scale/shift (fp32 math, one bf16 rounding).

    Reference: fused_adazero, ltx_serve/triton_ltx_ops.py:8-37 (kernel :3319-3357): scale/shift hold 1,
    batch or batch*tokens rows of D values.  Runs the table kernel with a zero table and scale/shift as the
    two timestep slots (``0 + v = v`` exactly).
    """
    _require_cuda(x, scale, shift)
    if x.dtype != torch.bfloat16 or x.ndim < 2 or x.shape[-1] not in (2048, 4096) or not x.is_contiguous():
        raise ValueError("x_shape")
    D = x.shape[-1]
    if scale.shape[-1] != D or shift.shape[-1] != D or scale.numel() != shift.numel() or scale.numel() % D:
        raise ValueError("scale_shape")
    x3 = x.reshape(-1, x.shape[-2], D) if x.ndim >= 3 else x.reshape(1, -1, D)
    B, L = x3.shape[0], x3.shape[1]
    dt = torch.float32 if torch.float32 in (scale.dtype, shift.dtype) else torch.bfloat16
    slots = torch.stack([shift.reshape(-1, D).to(dt), scale.reshape(-1, D).to(dt)], dim=1)  # [S, 2, D]
    ts = _row_broadcast(slots, B, L, "scale_shape")  # [B, L, 2, D]
    table = torch.zeros((2, D), device=x.device, dtype=dt)
    y = torch.empty_like(x3)
    _lib.call(
        "ogx_adazero_from_ada",
        x3.data_ptr(), B, L, D, table.data_ptr(), _code(table), table.stride(0),
        ts.data_ptr(), _code(ts), ts.stride(0), ts.stride(1), ts.stride(2), 0, 1, float(eps), y.data_ptr(),
        _stream(x),
    )
    return y.reshape(x.shape)


def fused_adazero_from_ada_fp8(
    x: torch.Tensor,
    eps: float,
    scale_shift_table: torch.Tensor,
    timestep: torch.Tensor,
    input_scale: torch.Tensor,
    *,
    shift_index: int,
    scale_index: int,
    return_bf16: bool = False,
    quant_mode: int = QUANT_TORCH,
    out: torch.Tensor | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """AdaZero fused with the E4M3 quantiser of the following FP8 linear.

    Equals ``fused_fp8_quantize_e4m3(fused_adazero_from_ada(...), input_scale)``
    bit for bit (reference :40-91 then :144-161), without writing the bf16
    activation unless ``return_bf16``.  ``out``: a caller-provided e4m3 output of x's shape.
    """
    global _VIDEO_ADA_VALUES_CALLS
    reason = ada_from_table_guard_reason(x, scale_shift_table, timestep)
    if reason is not None:
        raise ValueError(reason)
    _check_index(scale_shift_table, shift_index, scale_index)
    if input_scale.numel() != 1 or not input_scale.is_cuda or input_scale.dtype != torch.float32:
        raise ValueError("input_scale")
    _VIDEO_ADA_VALUES_CALLS += 1
    ts_view = _ts_view(x, scale_shift_table, timestep)
    if out is not None and (out.dtype != torch.float8_e4m3fn or out.shape != x.shape or not out.is_contiguous()):
        raise ValueError("out_shape")
    q = out if out is not None else torch.empty(x.shape, device=x.device, dtype=torch.float8_e4m3fn)
    y = torch.empty_like(x) if return_bf16 else None
    _lib.call(
        "ogx_adazero_from_ada_e4m3",
        x.data_ptr(), x.shape[0], x.shape[1], x.shape[2],
        scale_shift_table.data_ptr(), _code(scale_shift_table), scale_shift_table.stride(0),
        ts_view.data_ptr(), _code(ts_view), ts_view.stride(0), ts_view.stride(1), ts_view.stride(2),
        shift_index, scale_index, float(eps), input_scale.data_ptr(), int(quant_mode), _ptr(y), q.data_ptr(),
        _stream(x),
    )
    return (q, y) if return_bf16 else q


def fused_adazero_from_ada_fp8_planes(
    x: torch.Tensor,
    eps: float,
    scale_shift_table: torch.Tensor,
    timestep: torch.Tensor,
    input_scales: torch.Tensor,
    *,
    shift_index: int,
    scale_index: int,
    out: torch.Tensor | None = None,
    quant_mode: int = QUANT_TORCH,
) -> torch.Tensor:
    """AdaZero fused with up to three E4M3 quantisers of the same bf16 output: plane i of the result
    [n, *x.shape] equals ``fused_adazero_from_ada_fp8(..., input_scales[i])`` bit for bit, with x read once.

    For a checkpoint whose Q, K and V linears carry different input scales, where the reference quantises
    the bf16 AdaZero output once per linear inside FP8Linear.forward (ltx_serve/triton_ltx_ops.py:1692,
    :1676-1716).  ``input_scales``: float32 [n] on the device, n in 1..3; ``out``: e4m3 [n, *x.shape]."""
    global _VIDEO_ADA_VALUES_CALLS
    reason = ada_from_table_guard_reason(x, scale_shift_table, timestep)
    if reason is not None:
        raise ValueError(reason)
    _check_index(scale_shift_table, shift_index, scale_index)
    n = input_scales.numel()
    if (n < 1 or n > 3 or not input_scales.is_cuda or input_scales.dtype != torch.float32
            or not input_scales.is_contiguous()):
        raise ValueError("input_scale")
    if out is None:
        out = torch.empty((n, *x.shape), device=x.device, dtype=torch.float8_e4m3fn)
    if out.dtype != torch.float8_e4m3fn or tuple(out.shape) != (n, *x.shape) or not out.is_contiguous():
        raise ValueError("out_shape")
    _VIDEO_ADA_VALUES_CALLS += 1
    ts_view = _ts_view(x, scale_shift_table, timestep)
    _lib.call(
        "ogx_adazero_from_ada_e4m3_planes",
        x.data_ptr(), x.shape[0], x.shape[1], x.shape[2],
        scale_shift_table.data_ptr(), _code(scale_shift_table), scale_shift_table.stride(0),
        ts_view.data_ptr(), _code(ts_view), ts_view.stride(0), ts_view.stride(1), ts_view.stride(2),
        shift_index, scale_index, float(eps), input_scales.data_ptr(), n, int(quant_mode), None, out.data_ptr(),
        out.stride(0), _stream(x),
    )
    return out


def fused_head_gate_mul_bf16(out: torch.Tensor, gates: torch.Tensor, heads: int, dim_head: int) -> torch.Tensor:
    """``out.view(B, L, H, d) * gates[..., None]`` (bf16): the optional per-head gate of the attention output.

    Reference: fused_head_gate_mul_bf16, ltx_serve/triton_ltx_ops.py:614-637 (kernel :3584-3609; guard
    ``_can_use_fused_head_gate_mul`` :1612-1623).
    """
    _require_cuda(out, gates)
    if out.dtype != torch.bfloat16 or not out.is_contiguous() or out.ndim != 3 or out.shape[-1] != heads * dim_head:
        raise ValueError("out_shape")
    if gates.dtype != torch.bfloat16 or gates.shape != (out.shape[0], out.shape[1], heads):
        raise ValueError("gates_shape")
    g2 = gates.reshape(-1, heads)
    y = torch.empty_like(out)
    _lib.call(
        "ogx_head_gate_mul_bf16", out.data_ptr(), out.numel() // out.shape[-1], heads, dim_head, g2.data_ptr(),
        g2.stride(0), g2.stride(1), y.data_ptr(), _stream(out),
    )
    return y


# ---------------------------------------------------------------- quantiser
def fused_fp8_quantize_e4m3(x: torch.Tensor, input_scale: torch.Tensor, *, quant_mode: int = QUANT_TORCH) -> torch.Tensor:
    """Per-tensor E4M3 quantisation, bit-exact to the reference's torch path.

    Reference: fused_fp8_quantize_e4m3, ltx_serve/triton_ltx_ops.py:144-161; the
    torch path :146-148 is ``clamp(x * input_scale.reciprocal(), -448, 448).to(e4m3)``.
    ``quant_mode=QUANT_SINGLE`` gives the single-rounding semantics of the
    reference's Triton kernel (:3429-3444) instead.
    """
    _require_cuda(x, input_scale)
    if not x.is_contiguous() or input_scale.numel() != 1 or x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("fp8_quantize_input")
    if input_scale.dtype != torch.float32:
        raise ValueError("input_scale")
    q = torch.empty_strided(x.shape, x.stride(), device=x.device, dtype=torch.float8_e4m3fn)
    _lib.call(
        "ogx_fp8_quantize_e4m3",
        x.data_ptr(), _code(x), x.numel(), input_scale.data_ptr(), int(quant_mode), q.data_ptr(), _stream(x),
    )
    return q


def fused_gelu_tanh_fp8_quantize_e4m3(x: torch.Tensor, input_scale: torch.Tensor, *,
                                      return_gelu: bool = False):
    """GELU (tanh approximation) fused with the per-tensor E4M3 quantiser.

    Reference: fused_gelu_tanh_fp8_quantize_e4m3, ltx_serve/triton_ltx_ops.py:164-182; its torch path
    (:166-169) is ``clamp(gelu(x, approximate="tanh") * input_scale.reciprocal(), -448, 448).to(e4m3)``.
    With ``return_gelu`` the rounded GELU values are returned too, ``(q, gelu)``.
    """
    _require_cuda(x, input_scale)
    if not x.is_contiguous() or input_scale.numel() != 1 or x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("fp8_quantize_input")
    if input_scale.dtype != torch.float32:
        raise ValueError("input_scale")
    q = torch.empty_strided(x.shape, x.stride(), device=x.device, dtype=torch.float8_e4m3fn)
    gelu = torch.empty_like(x) if return_gelu else None
    _lib.call(
        "ogx_gelu_tanh_fp8_quantize_e4m3",
        x.data_ptr(), _code(x), x.numel(), input_scale.data_ptr(), q.data_ptr(), _ptr(gelu), _stream(x),
    )
    return (q, gelu) if return_gelu else q


# ---------------------------------------------------------------- bias add / residual
def fused_bias_add_bf16(x: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """``x + bias.to(bf16)``; reference ltx_serve/triton_ltx_ops.py:185-201."""
    _require_cuda(x, bias)
    if not x.is_contiguous() or x.dtype != torch.bfloat16 or x.ndim < 2:
        raise ValueError("bias_add_input")
    if bias.ndim != 1 or bias.shape[0] != x.shape[-1] or bias.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("bias_shape")
    out = torch.empty_like(x)
    cols = x.shape[-1]
    _lib.call(
        "ogx_bias_add_bf16", x.data_ptr(), x.numel() // cols, cols, bias.contiguous().data_ptr(), _code(bias),
        out.data_ptr(), _stream(x),
    )
    return out


def fused_residual_gate_bias_from_ada(
    x: torch.Tensor,
    y_no_bias: torch.Tensor,
    bias: torch.Tensor,
    scale_shift_table: torch.Tensor,
    timestep: torch.Tensor,
    *,
    gate_index: int,
    count_video_ada: bool = True,
) -> torch.Tensor:
    """``x + (y + bias.to(bf16)) * gate`` with bf16 rounding after each op.

    Reference: fused_residual_gate_bias_from_ada, ltx_serve/triton_ltx_ops.py:204-262
    (kernel :3663-3721), pinned bitwise by tests/test_triton_ltx_ops.py:182-204.
    """
    global _VIDEO_ADA_VALUES_CALLS, _VIDEO_TEXT_ADALN_CALLS
    reason = ada_from_table_guard_reason(x, scale_shift_table, timestep)
    if reason is not None:
        raise ValueError(reason)
    if not y_no_bias.is_contiguous() or y_no_bias.shape != x.shape or y_no_bias.dtype != torch.bfloat16:
        raise ValueError("y_shape")
    if bias.ndim != 1 or bias.shape[0] != x.shape[-1] or bias.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("bias_shape")
    _check_index(scale_shift_table, gate_index)
    if count_video_ada:
        _VIDEO_ADA_VALUES_CALLS += 1
    else:
        _VIDEO_TEXT_ADALN_CALLS += 1
    ts_view = _ts_view(x, scale_shift_table, timestep)
    out = torch.empty_like(x)
    _lib.call(
        "ogx_residual_gate_bias_from_ada",
        x.data_ptr(), y_no_bias.data_ptr(), x.shape[0], x.shape[1], x.shape[2],
        bias.contiguous().data_ptr(), _code(bias),
        scale_shift_table.data_ptr(), _code(scale_shift_table), scale_shift_table.stride(0),
        ts_view.data_ptr(), _code(ts_view), ts_view.stride(0), ts_view.stride(1), ts_view.stride(2),
        gate_index, out.data_ptr(), _stream(x),
    )
    return out


_ZERO_BIAS: dict[tuple[torch.device, int], torch.Tensor] = {}


def fused_residual_gate_from_ada(
    x: torch.Tensor,
    y: torch.Tensor,
    scale_shift_table: torch.Tensor,
    timestep: torch.Tensor,
    *,
    gate_index: int,
    count_video_ada: bool = True,
) -> torch.Tensor:
    """``x + y * gate`` with the gate from the table + timestep and bf16 rounding after the product.

    Reference: fused_residual_gate_from_ada, ltx_serve/triton_ltx_ops.py:640-694 (kernel :3612-3661):
    ``bf16(x + bf16(y * gate))``.  That is the bias kernel with a zero bias (``bf16(y + 0) = y`` for bf16 y).
    """
    key = (x.device, x.shape[-1])
    zero = _ZERO_BIAS.get(key)
    if zero is None:
        zero = _ZERO_BIAS[key] = torch.zeros(x.shape[-1], device=x.device, dtype=torch.bfloat16)
    return fused_residual_gate_bias_from_ada(x, y, zero, scale_shift_table, timestep, gate_index=gate_index,
                                             count_video_ada=count_video_ada)


def fused_residual_gate_bf16(x: torch.Tensor, y: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """``bf16(x + bf16(y * gate))`` with an explicit bf16 gate of 1, batch or batch*tokens rows.

    Reference: fused_residual_gate_bf16, ltx_serve/triton_ltx_ops.py:590-611 (kernel :3552-3582; guard
    ``_can_use_fused_residual_gate`` :1596-1609).  Runs the table residual kernel with a zero table and bias
    and the gate as the timestep slot.
    """
    _require_cuda(x, y, gate)
    if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16 or x.shape != y.shape or x.ndim < 2:
        raise ValueError("x_shape")
    if x.shape[-1] not in (2048, 4096) or not x.is_contiguous() or not y.is_contiguous():
        raise ValueError("x_shape")
    D = x.shape[-1]
    if gate.dtype != torch.bfloat16 or gate.shape[-1] != D or gate.numel() % D:
        raise ValueError("gate_shape")
    x3 = x.reshape(-1, x.shape[-2], D) if x.ndim >= 3 else x.reshape(1, -1, D)
    B, L = x3.shape[0], x3.shape[1]
    ts = _row_broadcast(gate.reshape(-1, D), B, L, "gate_shape")  # [B, L, D]
    key = (x.device, D)
    zero = _ZERO_BIAS.get(key)
    if zero is None:
        zero = _ZERO_BIAS[key] = torch.zeros(D, device=x.device, dtype=torch.bfloat16)
    out = fused_residual_gate_bias_from_ada(x3, y.reshape(x3.shape), zero, zero.view(1, D), ts, gate_index=0,
                                            count_video_ada=False)
    return out.reshape(x.shape)


# ---------------------------------------------------------------- Q/K RMSNorm + split RoPE
def _qk_guard_reason(q: torch.Tensor, k: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor) -> str | None:
    if not q.is_cuda or not k.is_cuda or q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        return "qk_device_or_dtype"
    if q.shape != k.shape or q.ndim != 3 or q.shape[0] != 1 or q.shape[-1] != 4096:
        return "qk_shape"
    if q.shape[1] < 1:
        return "empty_tokens"
    if q.stride(-1) != 1 or k.stride(-1) != 1 or q.stride(1) != k.stride(1) or q.stride(1) % 8:
        return "qk_noncontiguous"
    if q_weight.shape != (4096,) or k_weight.shape != (4096,) or q_weight.dtype != k_weight.dtype:
        return "qk_weight_shape"
    return None


def fused_video_qk_rmsnorm_rope_guard_reason(
    q: torch.Tensor, k: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
) -> str | None:
    """Mirrors `_fused_video_qk_rmsnorm_rope_guard_reason` (ltx_serve/triton_ltx_ops.py:1513-1537)."""
    reason = _qk_guard_reason(q, k, q_weight, k_weight)
    if reason is not None:
        return reason
    if cos.ndim != 4 or sin.ndim != 4 or cos.shape != sin.shape or cos.stride() != sin.stride() or cos.dtype != sin.dtype:
        return "rope_shape"
    if cos.shape[0] not in (1, q.shape[0]) or cos.shape[1] != 32 or cos.shape[2] != q.shape[1] or cos.shape[3] != 64:
        return "rope_shape"
    if cos.stride(-1) != 1:
        return "rope_shape"
    return None


def fused_video_qk_rmsnorm_rope(
    q: torch.Tensor,
    k: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    eps: float,
    cos: torch.Tensor,
    sin: torch.Tensor,
    *,
    out: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Q/K RMSNorm over 4096 columns + split RoPE per head; q/k [1, L, 4096] bf16, cos/sin [1|B, 32, L, 64].

    Reference: fused_video_qk_rmsnorm_rope, ltx_serve/triton_ltx_ops.py:320-378
    (kernel :3901-3978).  ``out`` may alias (q, k) for an in-place update.
    """
    reason = fused_video_qk_rmsnorm_rope_guard_reason(q, k, q_weight, k_weight, cos, sin)
    if reason is not None:
        raise ValueError(reason)
    if out is None:
        q_out, k_out = torch.empty_like(q), torch.empty_like(k)
    else:
        q_out, k_out = out
        if q_out.stride(1) != k_out.stride(1) or q_out.shape != q.shape or k_out.shape != k.shape:
            raise ValueError("qk_out_shape")
    _lib.call(
        "ogx_video_qk_rmsnorm_rope",
        q.data_ptr(), k.data_ptr(), q.shape[1], q.stride(1),
        q_weight.contiguous().data_ptr(), k_weight.contiguous().data_ptr(), _code(q_weight), float(eps),
        cos.data_ptr(), sin.data_ptr(), _code(cos), cos.stride(1), cos.stride(2),
        q_out.data_ptr(), k_out.data_ptr(), q_out.stride(1), _stream(q),
    )
    return q_out, k_out


@dataclass(frozen=True)
class RopePositions:
    """Split-RoPE angles generated from latent positions instead of cos/sin tables.

    Token i of a sequence (global index ``token0 + i``) sits at (t, h, w) of a [frames, grid_h, grid_w]
    raster (t slowest, the order of the video tokens); rotary slot g = 64 * head + j (32 heads x 64) turns by
    ``position[slot_axis[g]] * inv_freq[g]`` radians (axis 0 = t, 1 = h, 2 = w).  The tables are the
    caller's: the construction of the un-vendored ltx_core preprocessor that the reference's cos/sin come from
    is not available, so this library's synthetic configurations define one (``synthetic.rope_positions``).
    ``inv_freq`` is float64 [2048] and ``slot_axis`` uint8 [2048], both on the GPU."""

    inv_freq: torch.Tensor
    slot_axis: torch.Tensor
    frames: int
    grid_h: int
    grid_w: int

    @property
    def tokens(self) -> int:
        return self.frames * self.grid_h * self.grid_w

    def to(self, device) -> "RopePositions":
        return RopePositions(self.inv_freq.to(device), self.slot_axis.to(device), self.frames, self.grid_h, self.grid_w)


def rope_positions_guard_reason(pos: "RopePositions", device: torch.device) -> str | None:
    if pos.inv_freq.dtype != torch.float64 or pos.inv_freq.shape != (2048,) or not pos.inv_freq.is_contiguous():
        return "rope_shape"
    if pos.slot_axis.dtype != torch.uint8 or pos.slot_axis.shape != (2048,) or not pos.slot_axis.is_contiguous():
        return "rope_shape"
    if pos.inv_freq.device != device or pos.slot_axis.device != device:
        return "qk_device_or_dtype"
    if pos.grid_h < 1 or pos.grid_w < 1 or pos.frames < 1:
        return "rope_shape"
    return None


def fused_video_qk_rmsnorm_rope_positions(
    q: torch.Tensor,
    k: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    eps: float,
    positions: RopePositions,
    *,
    token0: int = 0,
    out: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``fused_video_qk_rmsnorm_rope`` with cos/sin generated in the kernel from the tokens' (t, h, w)
    positions (rounded to bf16 like the reference's tables) instead of read from [1, 32, L, 64] tables: the
    same arithmetic, 2 x 2 B x 2048 fewer HBM bytes per token.  q/k hold tokens [token0, token0 + L) of the
    raster.  ``rope_tables_from_positions`` returns the tables these angles make, for the table interface."""
    reason = _qk_guard_reason(q, k, q_weight, k_weight)
    if reason is None:
        reason = rope_positions_guard_reason(positions, q.device)
    if reason is None and (token0 < 0 or token0 + q.shape[1] > positions.tokens):
        reason = "rope_shape"
    if reason is not None:
        raise ValueError(reason)
    if out is None:
        q_out, k_out = torch.empty_like(q), torch.empty_like(k)
    else:
        q_out, k_out = out
        if q_out.stride(1) != k_out.stride(1) or q_out.shape != q.shape or k_out.shape != k.shape:
            raise ValueError("qk_out_shape")
    _lib.call(
        "ogx_video_qk_rmsnorm_rope_positions",
        q.data_ptr(), k.data_ptr(), q.shape[1], q.stride(1),
        q_weight.contiguous().data_ptr(), k_weight.contiguous().data_ptr(), _code(q_weight), float(eps),
        positions.inv_freq.data_ptr(), positions.slot_axis.data_ptr(), positions.grid_h, positions.grid_w, int(token0),
        q_out.data_ptr(), k_out.data_ptr(), q_out.stride(1), _stream(q),
    )
    return q_out, k_out


def rope_tables_from_positions(positions: RopePositions, *, token0: int = 0, tokens: int | None = None,
                               dtype: torch.dtype = torch.bfloat16) -> tuple[torch.Tensor, torch.Tensor]:
    """The cos/sin the generating RoPE kernel uses, as [1, 32, tokens, 64] tables (the reference's layout)."""
    dev = positions.inv_freq.device
    reason = rope_positions_guard_reason(positions, dev)
    if tokens is None:
        tokens = positions.tokens - token0
    if reason is None and (tokens < 1 or token0 < 0 or token0 + tokens > positions.tokens):
        reason = "rope_shape"
    if reason is None and dtype not in (torch.bfloat16, torch.float32):
        reason = "qk_device_or_dtype"
    if reason is not None:
        raise ValueError(reason)
    cos = torch.empty((1, 32, tokens, 64), device=dev, dtype=dtype)
    sin = torch.empty_like(cos)
    _lib.call(
        "ogx_rope_tables_from_positions",
        positions.inv_freq.data_ptr(), positions.slot_axis.data_ptr(), positions.grid_h, positions.grid_w,
        int(token0), tokens, _code(cos), cos.data_ptr(), sin.data_ptr(), torch.cuda.current_stream(dev).cuda_stream,
    )
    return cos, sin


def fused_video_qkv_rmsnorm_rope_pack(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    eps: float,
    cos: torch.Tensor,
    sin: torch.Tensor,
) -> torch.Tensor:
    """Q/K RMSNorm + split RoPE as ``fused_video_qk_rmsnorm_rope``, packed with V into qkv [1, L, 3, 32, 128]
    (the FlashAttention qkvpacked layout).

    Reference: fused_video_qkv_rmsnorm_rope_pack, ltx_serve/triton_ltx_ops.py:381-429 (kernel :3980-4061).
    q, k and v share their token stride.
    """
    reason = fused_video_qk_rmsnorm_rope_guard_reason(q, k, q_weight, k_weight, cos, sin)
    if reason is not None:
        raise ValueError(reason)
    if v.shape != q.shape or v.dtype != torch.bfloat16 or not v.is_cuda or v.stride(-1) != 1 or v.stride(1) != q.stride(1):
        raise ValueError("qkv_shape")
    L = q.shape[1]
    qkv = torch.empty((1, L, 3, 32, 128), device=q.device, dtype=torch.bfloat16)
    _lib.call(
        "ogx_video_qkv_rmsnorm_rope_scatter",
        q.data_ptr(), k.data_ptr(), v.data_ptr(), L, q.stride(1),
        q_weight.contiguous().data_ptr(), k_weight.contiguous().data_ptr(), _code(q_weight), float(eps),
        cos.data_ptr(), sin.data_ptr(), _code(cos), cos.stride(1), cos.stride(2),
        qkv[:, :, 0].data_ptr(), qkv[:, :, 1].data_ptr(), qkv[:, :, 2].data_ptr(), qkv.stride(1), 0, 32,
        _stream(q),
    )
    return qkv


def _norm_rows(t: torch.Tensor) -> tuple[int, int]:
    """(rows, row stride) of a [B, L, 4096] bf16 tensor whose rows are evenly strided."""
    if t.ndim != 3 or t.shape[-1] != 4096 or t.dtype != torch.bfloat16 or not t.is_cuda:
        raise ValueError("qk_shape")
    B, L, _ = t.shape
    if t.stride(-1) != 1 or t.stride(1) % 8 or (B > 1 and t.stride(0) != L * t.stride(1)):
        raise ValueError("qk_noncontiguous")
    return B * L, t.stride(1)


def fused_qk_rmsnorm(
    q: torch.Tensor,
    k: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    eps: float,
    *,
    out: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Q/K RMSNorm over 4096 columns with weight and no rotary embedding: q [B, L, 4096] and k [B, L_kv, 4096]
    bf16 (the lengths may differ), one launch for both.

    Reference: the pre-attention without positional embedding, ``q = attn.q_norm(q); k = attn.k_norm(k)``
    (ltx_serve/triton_ltx_ops.py:1864-1865), which the text cross-attention takes (:2880).  The arithmetic is
    that of ``fused_video_qk_rmsnorm_rope`` (fp32, one bf16 rounding) with the rotation left out.  ``out``
    may alias (q, k) for an in-place update.
    """
    q_rows, q_stride = _norm_rows(q)
    k_rows, k_stride = _norm_rows(k)
    if q_weight.shape != (4096,) or k_weight.shape != (4096,) or q_weight.dtype != k_weight.dtype:
        raise ValueError("qk_weight_shape")
    if out is None:
        q_out, k_out = torch.empty_like(q), torch.empty_like(k)
    else:
        q_out, k_out = out
        if q_out.shape != q.shape or k_out.shape != k.shape:
            raise ValueError("qk_out_shape")
    _, q_out_stride = _norm_rows(q_out)
    _, k_out_stride = _norm_rows(k_out)
    _lib.call(
        "ogx_qk_rmsnorm",
        q.data_ptr(), q_rows, q_stride, k.data_ptr(), k_rows, k_stride,
        q_weight.contiguous().data_ptr(), k_weight.contiguous().data_ptr(), _code(q_weight), float(eps),
        q_out.data_ptr(), q_out_stride, k_out.data_ptr(), k_out_stride, _stream(q),
    )
    return q_out, k_out


# ---------------------------------------------------------------- FP8 linears
def _scale_ptr(t: torch.Tensor) -> int:
    if t.numel() != 1 or t.dtype != torch.float32 or not t.is_cuda:
        raise ValueError("scale")
    return t.data_ptr()


def fp8_scaled_mm(
    qinput: torch.Tensor,
    weight: torch.Tensor,
    scale_a: torch.Tensor,
    scale_b: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    n_per_scale: int | None = None,
) -> torch.Tensor:
    """``bf16(qinput @ weight.t() * scale_a * scale_b) (+ bf16(bias))`` on tcgen05.

    Counterpart of ``torch._scaled_mm(qinput, weight.t(), scale_a, scale_b,
    out_dtype=bf16, use_fast_accum=True)`` followed by the bias add of
    FP8Linear.forward (ltx_serve/triton_ltx_ops.py:1695-1707).  ``scale_b`` may
    hold one scale per ``n_per_scale`` output columns (packed Q/K/V weights).
    A caller-provided ``out`` ([M, N], any row stride) is returned as given; otherwise the
    result has qinput's leading shape.
    """
    _require_cuda(qinput, weight, scale_a, scale_b)
    if qinput.dtype != torch.float8_e4m3fn or weight.dtype != torch.float8_e4m3fn:
        raise ValueError("fp8_dtype")
    a2 = qinput.reshape(-1, qinput.shape[-1])
    if a2.stride(-1) != 1 or weight.stride(-1) != 1 or weight.ndim != 2 or weight.shape[1] != a2.shape[1]:
        raise ValueError("fp8_shape")
    M, K = a2.shape
    N = weight.shape[0]
    if scale_a.numel() != 1 or scale_a.dtype != torch.float32 or scale_b.dtype != torch.float32:
        raise ValueError("scale")
    nps = n_per_scale if n_per_scale is not None else N // scale_b.numel()
    if nps * scale_b.numel() != N:
        raise ValueError("scale")
    given = out is not None
    if out is None:
        out = torch.empty((M, N), device=qinput.device, dtype=torch.bfloat16)
    if out.dtype != torch.bfloat16 or out.ndim != 2 or out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out_shape: out must be a [M, N] bf16 matrix with unit column stride")
    if bias is not None and (bias.ndim != 1 or bias.shape[0] != N):
        raise ValueError("bias_shape")
    _lib.call(
        "ogx_fp8_scaled_mm",
        a2.data_ptr(), M, K, a2.stride(0), weight.data_ptr(), N, weight.stride(0),
        scale_a.data_ptr(), scale_b.contiguous().data_ptr(), nps,
        _ptr(bias.contiguous()) if bias is not None else None, _code(bias) if bias is not None else DTYPE_BF16,
        out.data_ptr(), out.stride(0), _stream(qinput),
    )
    return out if given else out.reshape(*qinput.shape[:-1], N)


def fp8_scaled_mm_planes(
    qplanes: torch.Tensor,
    weight: torch.Tensor,
    scales_a: torch.Tensor,
    scales_b: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``fp8_scaled_mm`` over n activation planes: output columns [i*N/n, (i+1)*N/n) are
    ``bf16(qplanes[i] @ weight[i*N/n:(i+1)*N/n].t() * scales_a[i] * scales_b[i]) (+ bf16(bias))``, one launch.

    The packed Q/K/V projection of a checkpoint whose three linears quantise their input with different
    scales (the reference runs FP8Linear.forward once per linear, ltx_serve/triton_ltx_ops.py:1695-1707).
    ``qplanes``: e4m3 [n, ..., K] (each plane contiguous rows); ``scales_a``, ``scales_b``: float32 [n];
    N / n a multiple of 256.  Returns bf16 [M, N] (or the caller's ``out``)."""
    _require_cuda(qplanes, weight, scales_a, scales_b)
    if qplanes.dtype != torch.float8_e4m3fn or weight.dtype != torch.float8_e4m3fn:
        raise ValueError("fp8_dtype")
    n = qplanes.shape[0]
    K = qplanes.shape[-1]
    a3 = qplanes.reshape(n, -1, K)
    if not a3.is_contiguous() or weight.stride(-1) != 1 or weight.ndim != 2 or weight.shape[1] != K:
        raise ValueError("fp8_shape")
    M = a3.shape[1]
    N = weight.shape[0]
    if (scales_a.numel() != n or scales_b.numel() != n or scales_a.dtype != torch.float32
            or scales_b.dtype != torch.float32 or N % n):
        raise ValueError("scale")
    given = out is not None
    if out is None:
        out = torch.empty((M, N), device=qplanes.device, dtype=torch.bfloat16)
    if out.dtype != torch.bfloat16 or out.ndim != 2 or out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out_shape: out must be a [M, N] bf16 matrix with unit column stride")
    if bias is not None and (bias.ndim != 1 or bias.shape[0] != N):
        raise ValueError("bias_shape")
    _lib.call(
        "ogx_fp8_scaled_mm_planes",
        a3.data_ptr(), n, M, K, a3.stride(1), weight.data_ptr(), N, weight.stride(0),
        scales_a.contiguous().data_ptr(), scales_b.contiguous().data_ptr(),
        _ptr(bias.contiguous()) if bias is not None else None, _code(bias) if bias is not None else DTYPE_BF16,
        out.data_ptr(), out.stride(0), _stream(qplanes),
    )
    return out


def fp8_scaled_mm_gelu_e4m3(
    qinput: torch.Tensor,
    weight: torch.Tensor,
    scale_a: torch.Tensor,
    scale_b: torch.Tensor,
    q_scale: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """The FFN's first projection with GELU and the next projection's quantiser in its epilogue:
    ``fused_gelu_tanh_fp8_quantize_e4m3(fp8_scaled_mm(qinput, weight, scale_a, scale_b, bias=bias), q_scale)``
    without the bf16 hidden activation in memory (ltx_serve/triton_ltx_ops.py:1695-1707, :164-169, as
    ``_feedforward_without_out_bias`` :2796-2807 and ``fp8_linear_without_bias`` :770-771 chain them).
    Returns e4m3 [..., N] (or the caller's [M, N] ``out``)."""
    _require_cuda(qinput, weight, scale_a, scale_b, q_scale)
    if qinput.dtype != torch.float8_e4m3fn or weight.dtype != torch.float8_e4m3fn:
        raise ValueError("fp8_dtype")
    a2 = qinput.reshape(-1, qinput.shape[-1])
    if a2.stride(-1) != 1 or weight.stride(-1) != 1 or weight.ndim != 2 or weight.shape[1] != a2.shape[1]:
        raise ValueError("fp8_shape")
    M, K = a2.shape
    N = weight.shape[0]
    if scale_a.numel() != 1 or scale_a.dtype != torch.float32 or scale_b.dtype != torch.float32:
        raise ValueError("scale")
    if scale_b.numel() != 1:
        raise ValueError("scale")
    given = out is not None
    if out is None:
        out = torch.empty((M, N), device=qinput.device, dtype=torch.float8_e4m3fn)
    if out.dtype != torch.float8_e4m3fn or out.ndim != 2 or out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out_shape: out must be a [M, N] e4m3 matrix with unit column stride")
    if bias is not None and (bias.ndim != 1 or bias.shape[0] != N):
        raise ValueError("bias_shape")
    _lib.call(
        "ogx_fp8_scaled_mm_gelu_e4m3",
        a2.data_ptr(), M, K, a2.stride(0), weight.data_ptr(), N, weight.stride(0),
        scale_a.data_ptr(), scale_b.contiguous().data_ptr(), N,
        _ptr(bias.contiguous()) if bias is not None else None, _code(bias) if bias is not None else DTYPE_BF16,
        _scale_ptr(q_scale), out.data_ptr(), out.stride(0), _stream(qinput),
    )
    return out if given else out.reshape(*qinput.shape[:-1], N)


def fp8_linear_from_quantized_e4m3(linear, qinput: torch.Tensor, *, out_dtype: torch.dtype) -> torch.Tensor:
    """Reference: fp8_linear_from_quantized_e4m3, ltx_serve/triton_ltx_ops.py:742-759."""
    if out_dtype != torch.bfloat16:
        raise ValueError("out_dtype")
    return fp8_scaled_mm(qinput, linear.weight, linear.input_scale, linear.weight_scale, bias=linear.bias)


def fp8_linear_without_bias(linear, x: torch.Tensor, *, out_dtype: torch.dtype) -> torch.Tensor:
    """Quantise x with the linear's input scale and run the FP8 matmul without bias.

    Reference: fp8_linear_without_bias, ltx_serve/triton_ltx_ops.py:762-781.
    """
    if out_dtype != torch.bfloat16:
        raise ValueError("out_dtype")
    if x.shape[-1] != linear.in_features:
        raise ValueError("in_features")
    qinput = fused_fp8_quantize_e4m3(x.contiguous(), linear.input_scale)
    return fp8_scaled_mm(qinput, linear.weight, linear.input_scale, linear.weight_scale)


def fp8_linear_forward(linear, x: torch.Tensor) -> torch.Tensor:
    """The patched FP8Linear.forward (ltx_serve/triton_ltx_ops.py:1676-1716): quant -> scaled-mm -> bias."""
    qinput = fused_fp8_quantize_e4m3(x.contiguous(), linear.input_scale)
    return fp8_scaled_mm(qinput, linear.weight, linear.input_scale, linear.weight_scale, bias=linear.bias)


def fp8_qkv_from_shared_quantized_input(attn, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None:
    """Q/K/V from one quantised input; reference ltx_serve/triton_ltx_ops.py:805-819.

    Returns None when the three input scales differ (as the reference's guard does).
    """
    scales = [attn.to_q.input_scale, attn.to_k.input_scale, attn.to_v.input_scale]
    if not all(torch.equal(scales[0], s) for s in scales[1:]):
        return None
    qinput = fused_fp8_quantize_e4m3(x.contiguous(), attn.to_q.input_scale)
    return (
        fp8_linear_from_quantized_e4m3(attn.to_q, qinput, out_dtype=x.dtype),
        fp8_linear_from_quantized_e4m3(attn.to_k, qinput, out_dtype=x.dtype),
        fp8_linear_from_quantized_e4m3(attn.to_v, qinput, out_dtype=x.dtype),
    )


def fp8_scaled_mm_residual_gate(
    qinput: torch.Tensor,
    weight: torch.Tensor,
    scale_a: torch.Tensor,
    scale_b: torch.Tensor,
    bias: torch.Tensor,
    x: torch.Tensor,
    scale_shift_table: torch.Tensor,
    timestep: torch.Tensor,
    *,
    gate_index: int,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Out-projection fused with bias + Ada-gated residual (batch 1).

    Equals ``fused_residual_gate_bias_from_ada(x, fp8_linear_without_bias(...), bias,
    table, timestep, gate_index=...)`` (reference :762-781 then :204-262) given the
    same fp32 accumulation.
    """
    global _VIDEO_ADA_VALUES_CALLS
    reason = ada_from_table_guard_reason(x, scale_shift_table, timestep)
    if reason is not None:
        raise ValueError(reason)
    if x.shape[0] != 1:
        raise ValueError("x_shape")
    _check_index(scale_shift_table, gate_index)
    _require_cuda(qinput, weight, scale_a, scale_b, bias)
    if qinput.dtype != torch.float8_e4m3fn or weight.dtype != torch.float8_e4m3fn:
        raise ValueError("fp8_dtype")
    a2 = qinput.reshape(-1, qinput.shape[-1])
    M, K = a2.shape
    if weight.ndim != 2 or weight.shape[1] != K or weight.stride(-1) != 1 or a2.stride(-1) != 1:
        raise ValueError("fp8_shape")
    N = weight.shape[0]
    if x.shape[1] != M or x.shape[2] != N:
        raise ValueError("x_shape")
    if bias.ndim != 1 or bias.shape[0] != N:
        raise ValueError("bias_shape")
    _VIDEO_ADA_VALUES_CALLS += 1
    ts_view = _ts_view(x, scale_shift_table, timestep)
    if out is None:
        out = torch.empty_like(x)
    elif out.shape != x.shape or out.dtype != torch.bfloat16 or out.device != x.device or out.stride(-1) != 1:
        raise ValueError("out_shape: out must be a bf16 tensor shaped like x with unit column stride")
    _lib.call(
        "ogx_fp8_scaled_mm_residual_gate",
        a2.data_ptr(), M, K, a2.stride(0), weight.data_ptr(), N, weight.stride(0),
        _scale_ptr(scale_a), _scale_ptr(scale_b), N,
        bias.contiguous().data_ptr(), _code(bias), x.data_ptr(), x.stride(1),
        scale_shift_table.data_ptr(), _code(scale_shift_table), scale_shift_table.stride(0),
        ts_view.data_ptr(), _code(ts_view), ts_view.stride(1), ts_view.stride(2), gate_index,
        out.data_ptr(), out.stride(1), _stream(x),
    )
    return out


# ---------------------------------------------------------------- attention
def attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    heads: int,
    *,
    softmax_scale: float | None = None,
    out: torch.Tensor | None = None,
    out_e4m3_scale: torch.Tensor | None = None,
) -> torch.Tensor:
    """Dense bidirectional attention, q [B, L, H*128] and k/v [B, L_kv, H*128] bf16 (token rows may be
    strided; k and v share their strides).

    The attention-backend contract of the reference (benchmarks/official_ltx23_benchmark.py:3289-3373;
    call sites ltx_serve/triton_ltx_ops.py:2636 for the self-attention and :2880 for the text
    cross-attention, whose keys/values come from the prompt context: the backend views k and v as
    [b, -1, heads, d], :3305).  With ``out_e4m3_scale`` the bf16 result is quantised to e4m3 in the
    epilogue (torch-path semantics).
    """
    _require_cuda(q, k, v)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("qkv_dtype")
    if q.ndim != 3 or k.ndim != 3 or k.shape != v.shape or k.shape[0] != q.shape[0] or k.shape[2] != q.shape[2]:
        raise ValueError("qkv_shape")
    B, L, HD = q.shape
    L_kv = k.shape[1]
    if L < 1 or L_kv < 1:
        raise ValueError("qkv_shape")
    if HD % heads or HD // heads != 128:
        raise ValueError("head_dim")
    if k.stride() != v.stride() or q.stride(-1) != 1 or k.stride(-1) != 1:
        raise ValueError("qkv_stride")
    scale = float(softmax_scale) if softmax_scale is not None else 128 ** -0.5
    self_attention = L_kv == L and q.stride() == k.stride()
    if out is not None:
        want = torch.bfloat16 if out_e4m3_scale is None else torch.float8_e4m3fn
        if (out.shape != (B, L, HD) or out.dtype != want or out.device != q.device or out.stride(-1) != 1
                or (L > 1 and out.stride(1) < HD)):
            raise ValueError("out_shape: out must be [B, L, H*128] of the output dtype with unit column stride")
    if out_e4m3_scale is None:
        if out is None:
            out = torch.empty((B, L, HD), device=q.device, dtype=torch.bfloat16)
        if self_attention:
            _lib.call(
                "ogx_attention_fwd",
                q.data_ptr(), k.data_ptr(), v.data_ptr(), B, L, heads, 128, q.stride(0), q.stride(1), scale,
                out.data_ptr(), out.stride(0), out.stride(1), _stream(q),
            )
        else:
            _lib.call(
                "ogx_attention_fwd_kv",
                q.data_ptr(), k.data_ptr(), v.data_ptr(), B, L, L_kv, heads, 128, q.stride(0), q.stride(1),
                k.stride(0), k.stride(1), scale, out.data_ptr(), out.stride(0), out.stride(1), _stream(q),
            )
    else:
        if out is None:
            out = torch.empty((B, L, HD), device=q.device, dtype=torch.float8_e4m3fn)
        if self_attention:
            _lib.call(
                "ogx_attention_fwd_e4m3",
                q.data_ptr(), k.data_ptr(), v.data_ptr(), B, L, heads, 128, q.stride(0), q.stride(1), scale,
                _scale_ptr(out_e4m3_scale), out.data_ptr(), out.stride(0), out.stride(1), _stream(q),
            )
        else:
            _lib.call(
                "ogx_attention_fwd_kv_e4m3",
                q.data_ptr(), k.data_ptr(), v.data_ptr(), B, L, L_kv, heads, 128, q.stride(0), q.stride(1),
                k.stride(0), k.stride(1), scale, _scale_ptr(out_e4m3_scale), out.data_ptr(), out.stride(0),
                out.stride(1), _stream(q),
            )
    return out


def collect_video_ada_values_calls() -> int:
    return _VIDEO_ADA_VALUES_CALLS


__all__ = [
    "QUANT_SINGLE",
    "QUANT_TORCH",
    "RopePositions",
    "ada_from_table_guard_reason",
    "attention",
    "collect_video_ada_values_calls",
    "fp8_linear_forward",
    "fp8_linear_from_quantized_e4m3",
    "fp8_linear_without_bias",
    "fp8_qkv_from_shared_quantized_input",
    "fp8_scaled_mm",
    "fp8_scaled_mm_gelu_e4m3",
    "fp8_scaled_mm_planes",
    "fp8_scaled_mm_residual_gate",
    "fused_adaln_affine_from_ada",
    "fused_adazero",
    "fused_adazero_from_ada",
    "fused_adazero_from_ada_fp8",
    "fused_adazero_from_ada_fp8_planes",
    "fused_bias_add_bf16",
    "fused_fp8_quantize_e4m3",
    "fused_gelu_tanh_fp8_quantize_e4m3",
    "fused_head_gate_mul_bf16",
    "fused_mul_from_ada",
    "fused_qk_rmsnorm",
    "fused_residual_gate_bf16",
    "fused_residual_gate_bias_from_ada",
    "fused_residual_gate_from_ada",
    "fused_video_qk_rmsnorm_rope",
    "fused_video_qk_rmsnorm_rope_guard_reason",
    "fused_video_qk_rmsnorm_rope_positions",
    "fused_video_qkv_rmsnorm_rope_pack",
    "rope_positions_guard_reason",
    "rope_tables_from_positions",
]
