"""The video feed-forward branch of the same LTX-2.3 DiT layer on one B200.

The reference runs it (ltx_serve/triton_ltx_ops.py:3224-3258 with the production flags) as

    adazero_from_table (idx 3/4) -> quant -> scaled_mm -> bias add -> gelu(tanh) -> quant
    -> scaled_mm (no bias) -> bias + gate (idx 5) + residual

(``ff.net[0]`` is FP8Linear.forward :1676-1716 followed by GELU; ``_feedforward_without_out_bias``
:2796-2807 runs ``ff.net[2]`` through ``fp8_linear_without_bias`` :762-781).  Here it is three kernels
with the same arithmetic and rounding points:

 1. AdaZero (idx 3/4) fused with the E4M3 quantiser             -> e4m3 [L, 4096]
 2. FP8 GEMM 4096 -> 16384 with bias, GELU and the next quantiser in the epilogue -> e4m3 [L, 16384]
 3. FP8 GEMM 16384 -> 4096 fused with bias + Ada gate (idx 5) + residual        -> bf16 [L, 4096]

The bf16 hidden activation of the reference (302 MB at L=9216, written and read twice) never reaches
HBM.  The branch is sequence-local: on several GPUs each rank runs it on its own tokens.
"""

from __future__ import annotations

import torch

from . import ltx_ops
from .synthetic import FP8_MAX, FfnWeights


class VideoFeedForward:
    """One DiT layer's video FFN branch with weights resident in HBM."""

    kernel_launches_per_step = 3

    def __init__(self, weights: FfnWeights, device: torch.device | str = "cuda"):
        self.device = torch.device(device)
        self.w = weights.to(self.device)
        self.dim = self.w.proj.in_features
        self.hidden = self.w.proj.out_features
        self._ws: dict[int, torch.Tensor] = {}

    def _hq(self, tokens: int) -> torch.Tensor:
        hq = self._ws.get(tokens)
        if hq is None:
            hq = self._ws[tokens] = torch.empty((tokens, self.hidden), device=self.device, dtype=torch.float8_e4m3fn)
        return hq

    def forward(self, vx: torch.Tensor, timestep: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
        """vx [1, L, 4096] bf16 -> vx + gate * (ff(adazero(vx)) + bias), bf16."""
        if vx.ndim != 3 or vx.shape[0] != 1 or vx.shape[-1] != self.dim:
            raise ValueError("shape")
        w = self.w
        L = vx.shape[1]
        xq = ltx_ops.fused_adazero_from_ada_fp8(vx, w.norm_eps, w.scale_shift_table, timestep, w.proj.input_scale,
                                                shift_index=3, scale_index=4)
        hq = ltx_ops.fp8_scaled_mm_gelu_e4m3(xq, w.proj.weight, w.proj.input_scale, w.proj.weight_scale,
                                             w.out.input_scale, bias=w.proj.bias, out=self._hq(L))
        return ltx_ops.fp8_scaled_mm_residual_gate(
            hq.view(1, L, self.hidden), w.out.weight, w.out.input_scale, w.out.weight_scale, w.out.bias, vx,
            w.scale_shift_table, timestep, gate_index=5, out=out,
        )

    __call__ = forward

    @torch.no_grad()
    def calibrate_input_scales(self, vx: torch.Tensor, timestep: torch.Tensor) -> None:
        """Static per-tensor input scales = amax/448 of the activations feeding each FP8 linear (the
        AdaZero output and the GELU output); stand-ins for a checkpoint's calibrated input_scale."""
        w = self.w
        norm = ltx_ops.fused_adazero_from_ada(vx, w.norm_eps, w.scale_shift_table, timestep, shift_index=3,
                                              scale_index=4)
        w.proj.input_scale = (norm.float().abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
        xq = ltx_ops.fused_fp8_quantize_e4m3(norm, w.proj.input_scale)
        hidden = ltx_ops.fp8_scaled_mm(xq, w.proj.weight, w.proj.input_scale, w.proj.weight_scale, bias=w.proj.bias)
        gelu = torch.nn.functional.gelu(hidden, approximate="tanh")
        w.out.input_scale = (gelu.float().abs().amax().clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
