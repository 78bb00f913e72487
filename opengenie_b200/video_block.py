"""The fused LTX-2.3 video self-attention block on one B200.

The reference runs this block as ~12 launches from Python
(`_video_msa_branch_from_ada`, ltx_serve/triton_ltx_ops.py:2891-2981, with the
production flags of remote_official_worker.py:938-972):

    adazero_from_table -> 3 x (quant -> scaled_mm -> bias add) -> Q/K RMSNorm + RoPE
    -> attention -> quant -> scaled_mm (out, no bias) -> bias + gate + residual

Here it is five kernels with the same arithmetic and rounding points:

 1. AdaZero (idx 0/1) fused with the E4M3 quantiser     -> e4m3 [L, 4096]
 2. packed Q/K/V FP8 GEMM (one scale per Q/K/V weight) + bias -> bf16 [L, 3*4096]
 3. Q/K RMSNorm + split RoPE, in place on the packed rows
 4. attention (tcgen05) with the output quantised for the out-projection -> e4m3 [L, 4096]
 5. out-projection FP8 GEMM fused with bias + Ada gate (idx 2) + residual -> bf16 [L, 4096]

When the three Q/K/V input scales differ (the reference then quantises once per
linear, :1692) the activation is quantised once per distinct scale and each
projection writes its column slice of the packed buffer.
"""

from __future__ import annotations

import torch

from . import ltx_ops
from .synthetic import FP8_MAX, BlockWeights


class VideoSelfAttentionBlock:
    """One DiT layer's video self-attention branch with weights resident in HBM."""

    kernel_launches_per_step = 5  # without the optional per-head gate

    def __init__(self, weights: BlockWeights, device: torch.device | str = "cuda", *, to_gate_logits=None):
        """``to_gate_logits``: for checkpoints with gated attention, the module (or callable) mapping the
        AdaZero output [1, L, D] bf16 to per-head gate logits [1, L, H]; the attention output is then
        multiplied per head by 2*sigmoid(logits) before the out-projection (the reference's
        `_video_msa_gated_attention`, ltx_serve/triton_ltx_ops.py:2282-2302)."""
        self.device = torch.device(device)
        self.to_gate_logits = to_gate_logits
        w = weights.to(self.device)
        self.w = w
        self.dim = w.to_q.in_features
        self.heads = self.dim // 128
        self.w_qkv = torch.cat([w.to_q.weight, w.to_k.weight, w.to_v.weight], dim=0).contiguous()
        self.s_qkv = torch.stack([w.to_q.weight_scale, w.to_k.weight_scale, w.to_v.weight_scale]).reshape(3).contiguous()
        self.b_qkv = torch.cat([w.to_q.bias, w.to_k.bias, w.to_v.bias]).contiguous()
        # the per-linear weights, scales and biases become views of the packed copies: one copy in HBM
        D = w.to_q.weight.shape[0]
        for i, lin in enumerate((w.to_q, w.to_k, w.to_v)):
            lin.weight = self.w_qkv[i * D:(i + 1) * D]
            lin.weight_scale = self.s_qkv[i]
            lin.bias = self.b_qkv[i * D:(i + 1) * D]
        self.input_scales_changed()
        self._ws: dict[int, dict[str, torch.Tensor]] = {}

    def input_scales_changed(self) -> None:
        """Re-reads the Q/K/V input scales: whether one quantiser serves all three linears, and the packed
        [3] scales of the per-linear path.  Called at construction and by calibrate_input_scales; a caller
        that replaces the input scales by hand calls it too (it compares device scalars, which synchronises,
        so not inside a graph capture)."""
        w = self.w
        self.shared_quant = bool(
            torch.equal(w.to_q.input_scale, w.to_k.input_scale) and torch.equal(w.to_q.input_scale, w.to_v.input_scale)
        )
        self.s_in3 = torch.stack([w.to_q.input_scale, w.to_k.input_scale, w.to_v.input_scale]).reshape(3).contiguous()

    # ------------------------------------------------------------------ workspace
    def workspace(self, tokens: int) -> dict[str, torch.Tensor]:
        ws = self._ws.get(tokens)
        if ws is None:
            D = self.dim
            ws = {
                "xq": torch.empty((1, tokens, D), device=self.device, dtype=torch.float8_e4m3fn),
                "qkv": torch.empty((tokens, 3 * D), device=self.device, dtype=torch.bfloat16),
                "oq": torch.empty((1, tokens, D), device=self.device, dtype=torch.float8_e4m3fn),
            }
            self._ws[tokens] = ws
        return ws

    # ------------------------------------------------------------------ stages
    def qkv_projection(self, vx: torch.Tensor, timestep: torch.Tensor, ws: dict[str, torch.Tensor]) -> torch.Tensor:
        w = self.w
        D = self.dim
        if self.shared_quant:
            if self.to_gate_logits is not None:  # the gate logits read the bf16 AdaZero output
                ltx_ops_xq, ws["norm"] = ltx_ops.fused_adazero_from_ada_fp8(
                    vx, w.norm_eps, w.scale_shift_table, timestep, w.to_q.input_scale, shift_index=0, scale_index=1,
                    return_bf16=True)
            else:
                ltx_ops_xq = ltx_ops.fused_adazero_from_ada_fp8(
                    vx, w.norm_eps, w.scale_shift_table, timestep, w.to_q.input_scale, shift_index=0, scale_index=1
                )
            ws["xq"] = ltx_ops_xq
            ltx_ops.fp8_scaled_mm(
                ltx_ops_xq, self.w_qkv, w.to_q.input_scale, self.s_qkv, bias=self.b_qkv, out=ws["qkv"], n_per_scale=D
            )
        else:
            # a checkpoint whose Q, K and V linears quantise their input with different scales: one AdaZero
            # launch writes the three e4m3 copies, one GEMM launch reads copy i for output columns of linear i
            if self.to_gate_logits is not None:
                ws["norm"] = ltx_ops.fused_adazero_from_ada(vx, w.norm_eps, w.scale_shift_table, timestep,
                                                            shift_index=0, scale_index=1)
            xq3 = ltx_ops.fused_adazero_from_ada_fp8_planes(vx, w.norm_eps, w.scale_shift_table, timestep, self.s_in3,
                                                           shift_index=0, scale_index=1, out=ws.get("xq3"))
            ws["xq3"] = xq3
            ltx_ops.fp8_scaled_mm_planes(xq3, self.w_qkv, self.s_in3, self.s_qkv, bias=self.b_qkv, out=ws["qkv"])
        return ws["qkv"]

    def forward(
        self,
        vx: torch.Tensor,
        timestep: torch.Tensor,
        pe: tuple[torch.Tensor, torch.Tensor],
        *,
        out: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """vx [1, L, 4096] bf16 -> vx + gate * (out_proj(attn(...)) + bias), bf16.  ``pe``: (cos, sin) tables or
        ``ltx_ops.RopePositions``."""
        if vx.ndim != 3 or vx.shape[0] != 1 or vx.shape[-1] != self.dim:
            raise ValueError("shape")
        w = self.w
        L = vx.shape[1]
        D = self.dim
        ws = self.workspace(L)
        qkv = self.qkv_projection(vx, timestep, ws)
        q = qkv[:, :D].unsqueeze(0)
        k = qkv[:, D:2 * D].unsqueeze(0)
        v = qkv[:, 2 * D:].unsqueeze(0)
        self.rope(q, k, pe)
        if self.to_gate_logits is not None:
            ws["oq"] = ltx_ops.fused_fp8_quantize_e4m3(self._gated_attention(q, k, v, ws["norm"]),
                                                       w.to_out.input_scale)
        else:
            ltx_ops.attention(q, k, v, self.heads, out=ws["oq"], out_e4m3_scale=w.to_out.input_scale)
        return ltx_ops.fp8_scaled_mm_residual_gate(
            ws["oq"], w.to_out.weight, w.to_out.input_scale, w.to_out.weight_scale, w.to_out.bias,
            vx, w.scale_shift_table, timestep, gate_index=2, out=out,
        )

    __call__ = forward

    def rope(self, q: torch.Tensor, k: torch.Tensor, pe) -> None:
        """Q/K RMSNorm + split RoPE in place; ``pe`` is (cos, sin) tables [1, 32, L, 64] (the reference's
        interface) or ``ltx_ops.RopePositions`` (cos/sin generated in the kernel from the tokens' positions)."""
        w = self.w
        if isinstance(pe, ltx_ops.RopePositions):
            ltx_ops.fused_video_qk_rmsnorm_rope_positions(q, k, w.q_norm_weight, w.k_norm_weight, w.qk_eps, pe,
                                                          out=(q, k))
        else:
            cos, sin = pe
            ltx_ops.fused_video_qk_rmsnorm_rope(q, k, w.q_norm_weight, w.k_norm_weight, w.qk_eps, cos, sin, out=(q, k))

    def _gated_attention(self, q, k, v, norm: torch.Tensor) -> torch.Tensor:
        """bf16 attention output times 2*sigmoid(gate logits) per head (the gated checkpoints)."""
        gates = (2.0 * torch.sigmoid(self.to_gate_logits(norm))).to(torch.bfloat16).contiguous()
        return ltx_ops.fused_head_gate_mul_bf16(ltx_ops.attention(q, k, v, self.heads), gates, self.heads, 128)

    def time_attention(self, steps: int, warmup: int = 3, tokens: int | None = None) -> float:
        """Average device time (ms) of the attention kernel alone (launches replayed from one CUDA graph on the
        current stream) over the Q/K/V the last forward left in the workspace."""
        from .graphs import time_launches

        if tokens is None:
            tokens = max(self._ws)
        ws = self.workspace(tokens)
        D = self.dim
        qkv = ws["qkv"]
        q, k, v = (qkv[:, i * D:(i + 1) * D].unsqueeze(0) for i in range(3))
        out = torch.empty((1, tokens, D), device=self.device, dtype=torch.float8_e4m3fn)
        return time_launches(
            lambda: ltx_ops.attention(q, k, v, self.heads, out=out, out_e4m3_scale=self.w.to_out.input_scale),
            steps, warmup, self.device)

    # ------------------------------------------------------------------ calibration
    @torch.no_grad()
    def calibrate_input_scales(self, vx: torch.Tensor, timestep: torch.Tensor, pe: tuple[torch.Tensor, torch.Tensor]) -> None:
        """Sets static per-tensor input scales = amax/448 of the activations feeding each FP8 linear.

        Stands in for the calibrated input_scale of the FP8 checkpoint (used as a static
        scalar by the reference, ltx_serve/triton_ltx_ops.py:1692-1698).
        """
        w = self.w
        D = self.dim
        norm = ltx_ops.fused_adazero_from_ada(vx, w.norm_eps, w.scale_shift_table, timestep, shift_index=0, scale_index=1)
        s_in = (norm.float().abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
        for lin in (w.to_q, w.to_k, w.to_v):
            lin.input_scale = s_in.clone()
        self.input_scales_changed()
        ws = self.workspace(vx.shape[1])
        qkv = self.qkv_projection(vx, timestep, ws)
        q = qkv[:, :D].unsqueeze(0)
        k = qkv[:, D:2 * D].unsqueeze(0)
        v = qkv[:, 2 * D:].unsqueeze(0)
        self.rope(q, k, pe)
        if self.to_gate_logits is not None:
            attn = self._gated_attention(q, k, v, ws["norm"])
        else:
            attn = ltx_ops.attention(q, k, v, self.heads)
        w.to_out.input_scale = (attn.float().abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
