"""The video branches of LTX-2.3 DiT layers, chained: self-attention then feed-forward per layer, a
stack of layers per denoising step, captured once as a CUDA graph.

In the reference's layer (``BasicAVTransformerBlock._forward`` patched by
``_patch_ltx_block_residuals``, ltx_serve/triton_ltx_ops.py:2984-3300) the video stream runs the
self-attention branch (Ada slots 0-2, :3006-3083), then the text cross-attention (slots 6-8) and the
audio-video cross-attention, then the feed-forward branch (slots 3-5, :3224-3258).  A ``VideoLayer`` here is
the self-attention block followed directly by the FFN branch: the text cross-attention branch exists on its
own (``video_text_attention.VideoTextCrossAttention``) and is not chained in yet, and the audio-video
cross-attention is not part of this library.  Each layer is 8 kernel launches; a stack of 48 is 384, which
one graph replay issues at once.
"""

from __future__ import annotations

import torch

from .synthetic import BlockWeights, FfnWeights
from .video_block import VideoSelfAttentionBlock
from .video_ffn import VideoFeedForward


class VideoLayer:
    kernel_launches_per_step = 8

    def __init__(self, block_weights: BlockWeights, ffn_weights: FfnWeights, device):
        self.device = torch.device(device)
        self.attn = VideoSelfAttentionBlock(block_weights, self.device)
        self.ffn = VideoFeedForward(ffn_weights, self.device)
        self._mid: dict[int, torch.Tensor] = {}

    def _buf(self, vx: torch.Tensor) -> torch.Tensor:
        b = self._mid.get(vx.shape[1])
        if b is None:
            b = self._mid[vx.shape[1]] = torch.empty_like(vx)
        return b

    @torch.no_grad()
    def calibrate_input_scales(self, vx, timestep, pe) -> torch.Tensor:
        """Calibrates both branches on this input; returns the layer's output (the next layer's input)."""
        self.attn.calibrate_input_scales(vx, timestep, pe)
        mid = self.attn(vx, timestep, pe)
        self.ffn.calibrate_input_scales(mid, timestep)
        return self.ffn(mid, timestep)

    def forward(self, vx, timestep, pe, *, out: torch.Tensor | None = None) -> torch.Tensor:
        mid = self.attn(vx, timestep, pe, out=self._buf(vx))
        return self.ffn(mid, timestep, out=out)

    __call__ = forward


class VideoLayerStack:
    """Layers applied in order; two ping-pong buffers carry the residual stream between them."""

    def __init__(self, layers: list[VideoLayer]):
        if not layers:
            raise ValueError("layers")
        self.layers = layers
        self.kernel_launches_per_step = sum(layer.kernel_launches_per_step for layer in layers)
        self._pp: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        # the layers run one after another on one stream, so they share their intermediate buffers
        for layer in layers[1:]:
            layer.attn._ws = layers[0].attn._ws
            layer.ffn._ws = layers[0].ffn._ws
            layer._mid = layers[0]._mid

    @torch.no_grad()
    def calibrate_input_scales(self, vx, timestep, pe) -> None:
        for layer in self.layers:
            vx = layer.calibrate_input_scales(vx, timestep, pe)

    def forward(self, vx, timestep, pe, *, out: torch.Tensor | None = None) -> torch.Tensor:
        pp = self._pp.get(vx.shape[1])
        if pp is None:
            pp = self._pp[vx.shape[1]] = (torch.empty_like(vx), torch.empty_like(vx))
        x = vx
        for i, layer in enumerate(self.layers):
            last = i == len(self.layers) - 1
            x = layer(x, timestep, pe, out=out if (last and out is not None) else pp[i & 1])
        return x

    __call__ = forward
