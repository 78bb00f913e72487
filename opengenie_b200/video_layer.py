"""The video branches of LTX-2.3 DiT layers, chained in the reference's order: self-attention, text
cross-attention, feed-forward per layer; a stack of layers per denoising step, captured once as a CUDA graph.

In the reference's layer (``BasicAVTransformerBlock._forward`` patched by
``_patch_ltx_block_residuals``, ltx_serve/triton_ltx_ops.py:2984-3300) the video stream runs the
self-attention branch (Ada slots 0-2, :3006-3083), then the text cross-attention with its AdaLN (slots 6-8,
``_apply_video_text_cross_attention_adaln_from_ada``, :2810-2888), then the audio-video cross-attention, then
the feed-forward branch (slots 3-5, :3224-3258).  A ``VideoLayer`` here is the self-attention block, the text
cross-attention branch when the layer is given its weights, and the FFN branch; all three read one 9-slot Ada
table and one 9-slot timestep embedding, as the reference's layer does.  Without text weights the layer is
self-attention + FFN over a 6-slot table.  The audio-video cross-attention is not part of this library.

A layer is 8 kernel launches (5 self-attention + 3 FFN), 16 with the text branch; a stack of 48 layers is
384 or 768, which one graph replay issues at once.
"""

from __future__ import annotations

import torch

from .synthetic import BlockWeights, FfnWeights, TextAttentionWeights
from .video_block import VideoSelfAttentionBlock
from .video_ffn import VideoFeedForward
from .video_text_attention import VideoTextCrossAttention


class VideoLayer:
    def __init__(self, block_weights: BlockWeights, ffn_weights: FfnWeights, device,
                 text_weights: TextAttentionWeights | None = None):
        """``text_weights``: the layer's text cross-attention (attn2) weights.  When given, the layer's Ada table
        is the 9-slot table of the reference's layer: rows 0-2 from the self-attention weights' table, 3-5
        from the FFN weights' table, 6-8 from the text weights' table, shared by the three branches."""
        self.device = torch.device(device)
        self.attn = VideoSelfAttentionBlock(block_weights, self.device)
        self.ffn = VideoFeedForward(ffn_weights, self.device)
        self.text: VideoTextCrossAttention | None = None
        if text_weights is not None:
            self.text = VideoTextCrossAttention(text_weights, self.device)
            table = torch.cat([self.attn.w.scale_shift_table[0:3], self.ffn.w.scale_shift_table[3:6],
                               self.text.w.scale_shift_table[6:9]]).to(torch.float32).contiguous()
            self.attn.w.scale_shift_table = table
            self.ffn.w.scale_shift_table = table
            self.text.w.scale_shift_table = table
        self.kernel_launches_per_step = self.attn.kernel_launches_per_step + self.ffn.kernel_launches_per_step + (
            self.text.kernel_launches_per_step if self.text is not None else 0)
        self._mid: dict[tuple[int, int], torch.Tensor] = {}

    @property
    def ada_slots(self) -> int:
        return 9 if self.text is not None else 6

    def _buf(self, vx: torch.Tensor, i: int) -> torch.Tensor:
        b = self._mid.get((vx.shape[1], i))
        if b is None:
            b = self._mid[(vx.shape[1], i)] = torch.empty_like(vx)
        return b

    def _check_context(self, context, prompt_timestep) -> None:
        if (self.text is None) != (context is None) or (context is None) != (prompt_timestep is None):
            raise ValueError("context" if self.text is not None else "no_text_branch")

    @torch.no_grad()
    def calibrate_input_scales(self, vx, timestep, pe, *, context=None, prompt_timestep=None) -> torch.Tensor:
        """Calibrates every branch on this input, in the layer's order; returns the layer's output (the next
        layer's input)."""
        self._check_context(context, prompt_timestep)
        self.attn.calibrate_input_scales(vx, timestep, pe)
        x = self.attn(vx, timestep, pe)
        if self.text is not None:
            self.text.calibrate_input_scales(x, timestep, context, prompt_timestep)
            x = self.text(x, timestep, context, prompt_timestep)
        self.ffn.calibrate_input_scales(x, timestep)
        return self.ffn(x, timestep)

    def forward(self, vx, timestep, pe, *, context=None, prompt_timestep=None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """vx [1, L, 4096] bf16, timestep [1, L, slots*4096] (9 slots with the text branch, else 6), pe the
        RoPE tables or positions; context [1, L_ctx, 4096] bf16 and prompt_timestep [1, L_ctx, 2*4096] with
        the text branch."""
        self._check_context(context, prompt_timestep)
        x = self.attn(vx, timestep, pe, out=self._buf(vx, 0))
        if self.text is not None:
            x = self.text(x, timestep, context, prompt_timestep, out=self._buf(vx, 1))
        return self.ffn(x, timestep, out=out)

    __call__ = forward


class VideoLayerStack:
    """Layers applied in order; two ping-pong buffers carry the residual stream between them."""

    def __init__(self, layers: list[VideoLayer]):
        if not layers:
            raise ValueError("layers")
        if len({layer.text is None for layer in layers}) != 1:
            raise ValueError("mixed_text_branch")
        self.layers = layers
        self.kernel_launches_per_step = sum(layer.kernel_launches_per_step for layer in layers)
        self._pp: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        # the layers run one after another on one stream, so they share their intermediate buffers
        for layer in layers[1:]:
            layer.attn._ws = layers[0].attn._ws
            layer.ffn._ws = layers[0].ffn._ws
            if layer.text is not None:
                layer.text._ws = layers[0].text._ws
            layer._mid = layers[0]._mid

    @torch.no_grad()
    def calibrate_input_scales(self, vx, timestep, pe, *, context=None, prompt_timestep=None) -> None:
        for layer in self.layers:
            vx = layer.calibrate_input_scales(vx, timestep, pe, context=context, prompt_timestep=prompt_timestep)

    def forward(self, vx, timestep, pe, *, context=None, prompt_timestep=None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        pp = self._pp.get(vx.shape[1])
        if pp is None:
            pp = self._pp[vx.shape[1]] = (torch.empty_like(vx), torch.empty_like(vx))
        x = vx
        for i, layer in enumerate(self.layers):
            last = i == len(self.layers) - 1
            x = layer(x, timestep, pe, context=context, prompt_timestep=prompt_timestep,
                      out=out if (last and out is not None) else pp[i & 1])
        return x

    __call__ = forward
