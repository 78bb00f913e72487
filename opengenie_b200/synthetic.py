"""Seeded synthetic inputs for the video self-attention block configurations.

The reference measures on a real LTX-2.3 checkpoint and real latents, neither of
which exists here, so seeded tensors with the shapes and value distributions of
the benchmark configurations stand in for them:

- x ~ N(0, 1) bf16 [1, L, 4096]; in the diffusion-forcing configuration the first
  ``clean_frames`` latent frames are clean context with x ~ N(0, 0.5);
- scale_shift_table ~ N(0, 0.02) fp32 [6, 4096];
- timestep embedding: one N(0, 1) vector per Ada slot ([6*4096] bf16) broadcast over
  tokens as a stride-0 view (the uniform-timestep layout, ltx_serve/triton_ltx_ops.py:2355-2358),
  or, for diffusion forcing, two such vectors (clean / noisy tokens) materialised per
  token [1, L, 6*4096] (the clean-prefix `denoise_mask` of ltx_serve/latent_continuity.py:50-53);
- Q/K/V/out weights ~ N(0, 0.02) quantised to e4m3 with weight_scale = amax/448,
  biases ~ N(0, 0.01) bf16, Q/K RMSNorm weights ~ N(1, 0.1) bf16, eps 1e-6;
- split-RoPE cos/sin [1, 32, L, 64] bf16 from integer (t, h, w) latent positions with
  theta 10000 (construction in ``rope_tables``; the exact LTX frequency mapping lives in
  the un-vendored ltx_core preprocessor, so kernel and oracle both consume these tensors).

For the text cross-attention branch (attn2): the layer's Ada table has 9 slots (6/7 the query-side
AdaLN shift/scale, 8 the gate; ~N(0, 0.02) fp32 [9, 4096]) with a 9-slot uniform timestep embedding;
the prompt context is ``TEXT_CONTEXT_TOKENS`` = 1024 tokens of x ~ N(0, 1) bf16 [1, 1024, 4096] (the
caption length after the un-vendored ltx_core text connector is not fixed by the reference; 1024 is
this library's stand-in) with a 2-slot prompt table ~N(0, 0.02) and a uniform N(0, 1) prompt timestep
embedding.

Everything is drawn on the CPU from ``torch.Generator().manual_seed(seed)`` so the
same seed gives the same tensors on any machine with this torch version.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

DIM = 4096
HEADS = 32
HEAD_DIM = 128
ADA_SLOTS = 6
TEXT_ADA_SLOTS = 9  # + query-side shift/scale (6/7) and gate (8) of the text cross-attention
PROMPT_ADA_SLOTS = 2
TEXT_CONTEXT_TOKENS = 1024
FP8_MAX = 448.0


@dataclass(frozen=True)
class BlockConfig:
    name: str
    frames: int
    grid_h: int
    grid_w: int
    clean_frames: int = 0
    per_token_timestep: bool = False

    @property
    def tokens(self) -> int:
        return self.frames * self.grid_h * self.grid_w


# The benchmark configurations (token counts: 4x18x32, 16x18x32, 16x45x40).
CONFIGS = {
    "c0_l2304": BlockConfig("c0_l2304", 4, 18, 32),
    "c1_l9216": BlockConfig("c1_l9216", 16, 18, 32),
    "c2_df_l9216": BlockConfig("c2_df_l9216", 16, 18, 32, clean_frames=3, per_token_timestep=True),
    "c4_l28800": BlockConfig("c4_l28800", 16, 45, 40),
}


def rope_tables(frames: int, grid_h: int, grid_w: int, *, theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Split-RoPE cos/sin [1, 32, L, 64] (bf16) for tokens ordered (t, h, w).

    The 2048 rotary frequencies (32 heads x 64) are dealt round-robin to the three
    position axes: global slot g = 64*head + j uses axis g % 3 with inverse frequency
    theta ** -((g // 3) / ceil(2048 / 3)); angle = position[axis] * inv_freq.
    """
    L = frames * grid_h * grid_w
    t = torch.arange(frames, dtype=torch.float64).repeat_interleave(grid_h * grid_w)
    h = torch.arange(grid_h, dtype=torch.float64).repeat_interleave(grid_w).repeat(frames)
    w = torch.arange(grid_w, dtype=torch.float64).repeat(frames * grid_h)
    pos = torch.stack([t, h, w], dim=0)  # [3, L]
    inv_freq, axis = rope_slot_frequencies(theta=theta)
    angle = pos[axis.long()] * inv_freq[:, None]  # [2048, L]
    angle = angle.reshape(HEADS, HEAD_DIM // 2, L).permute(0, 2, 1).unsqueeze(0)  # [1, 32, L, 64]
    return angle.cos().to(torch.bfloat16).contiguous(), angle.sin().to(torch.bfloat16).contiguous()


def rope_slot_frequencies(*, theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """The per-slot construction behind ``rope_tables``: (inverse frequency float64 [2048], position axis
    uint8 [2048]) for slot g = 64 * head + j: axis g % 3, inverse frequency theta ** -((g // 3) / ceil(2048 / 3))."""
    g = torch.arange(HEADS * HEAD_DIM // 2, dtype=torch.int64)
    axis = (g % 3).to(torch.uint8)
    rank = (g // 3).to(torch.float64)
    inv_freq = theta ** (-rank / math.ceil(g.numel() / 3))
    return inv_freq.contiguous(), axis.contiguous()


def rope_positions(frames: int, grid_h: int, grid_w: int, *, theta: float = 10000.0, device="cpu"):
    """The same angles as ``rope_tables`` for the kernels that generate cos/sin from the tokens' (t, h, w)
    positions (``ltx_ops.RopePositions``)."""
    from .ltx_ops import RopePositions

    inv_freq, axis = rope_slot_frequencies(theta=theta)
    return RopePositions(inv_freq.to(device), axis.to(device), frames, grid_h, grid_w)


def quantize_weight_e4m3(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor e4m3 weight quantisation with weight_scale = amax / 448."""
    scale = (w.abs().amax().clamp_min(1e-12) / FP8_MAX).to(torch.float32)
    q = torch.clamp(w / scale, -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q, scale


@dataclass
class Fp8Linear:
    """The attributes of ltx_core's FP8Linear the reference's fast paths read."""

    weight: torch.Tensor  # e4m3 [out, in]
    weight_scale: torch.Tensor  # fp32 scalar
    input_scale: torch.Tensor  # fp32 scalar
    bias: torch.Tensor | None  # bf16 [out]

    @property
    def in_features(self) -> int:
        return self.weight.shape[1]

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    def to(self, device) -> "Fp8Linear":
        return Fp8Linear(
            self.weight.to(device),
            self.weight_scale.to(device),
            self.input_scale.to(device),
            None if self.bias is None else self.bias.to(device),
        )


@dataclass
class BlockWeights:
    to_q: Fp8Linear
    to_k: Fp8Linear
    to_v: Fp8Linear
    to_out: Fp8Linear
    q_norm_weight: torch.Tensor
    k_norm_weight: torch.Tensor
    scale_shift_table: torch.Tensor
    norm_eps: float = 1e-6
    qk_eps: float = 1e-6

    def to(self, device) -> "BlockWeights":
        return BlockWeights(
            self.to_q.to(device), self.to_k.to(device), self.to_v.to(device), self.to_out.to(device),
            self.q_norm_weight.to(device), self.k_norm_weight.to(device), self.scale_shift_table.to(device),
            self.norm_eps, self.qk_eps,
        )


def make_weights(seed: int = 0, *, dim: int = DIM, qkv_input_scale: float = 1.0, out_input_scale: float = 1.0) -> BlockWeights:
    """Random-init block weights (CPU).  Input scales are placeholders until calibrated."""
    g = torch.Generator().manual_seed(seed)

    def linear() -> Fp8Linear:
        w = torch.randn((dim, dim), generator=g) * 0.02
        q, s = quantize_weight_e4m3(w)
        b = (torch.randn((dim,), generator=g) * 0.01).to(torch.bfloat16)
        return Fp8Linear(q, s, torch.tensor(qkv_input_scale, dtype=torch.float32), b)

    to_q, to_k, to_v, to_out = linear(), linear(), linear(), linear()
    to_out.input_scale = torch.tensor(out_input_scale, dtype=torch.float32)
    q_norm = (1.0 + 0.1 * torch.randn((dim,), generator=g)).to(torch.bfloat16)
    k_norm = (1.0 + 0.1 * torch.randn((dim,), generator=g)).to(torch.bfloat16)
    table = torch.randn((ADA_SLOTS, dim), generator=g) * 0.02
    return BlockWeights(to_q, to_k, to_v, to_out, q_norm, k_norm, table.to(torch.float32))


FFN_HIDDEN = 4 * DIM


@dataclass
class FfnWeights:
    """The video feed-forward branch of the same layer: ``ff.net[0].proj`` (D -> 4D, with bias), GELU
    (tanh), ``ff.net[2]`` (4D -> D, bias applied with the gated residual), and the layer's Ada table
    (slots 3/4 for the AdaZero shift/scale, 5 for the gate)."""

    proj: Fp8Linear
    out: Fp8Linear
    scale_shift_table: torch.Tensor
    norm_eps: float = 1e-6

    def to(self, device) -> "FfnWeights":
        return FfnWeights(self.proj.to(device), self.out.to(device), self.scale_shift_table.to(device), self.norm_eps)


def make_ffn_weights(seed: int = 0, *, dim: int = DIM, hidden: int = FFN_HIDDEN) -> FfnWeights:
    """Random-init FFN weights (CPU): W ~ N(0, 0.02) pre-quantised to e4m3 with amax/448 scales, biases
    ~ N(0, 0.01), table ~ N(0, 0.02).  Input scales are placeholders until calibrated."""
    g = torch.Generator().manual_seed(seed)

    def linear(n_out: int, n_in: int) -> Fp8Linear:
        w = torch.randn((n_out, n_in), generator=g) * 0.02
        q, s = quantize_weight_e4m3(w)
        b = (torch.randn((n_out,), generator=g) * 0.01).to(torch.bfloat16)
        return Fp8Linear(q, s, torch.tensor(1.0, dtype=torch.float32), b)

    proj = linear(hidden, dim)
    out = linear(dim, hidden)
    table = torch.randn((ADA_SLOTS, dim), generator=g) * 0.02
    return FfnWeights(proj, out, table.to(torch.float32))


@dataclass
class TextAttentionWeights:
    """The video text cross-attention (attn2) of the same layer with cross-attention AdaLN: to_q on the video
    tokens, to_k/to_v on the prompt context, to_out with its bias, Q/K RMSNorm weights, the layer's 9-slot
    Ada table (6/7 query-side shift/scale, 8 gate) and the 2-slot prompt table (context shift/scale)."""

    to_q: Fp8Linear
    to_k: Fp8Linear
    to_v: Fp8Linear
    to_out: Fp8Linear
    q_norm_weight: torch.Tensor
    k_norm_weight: torch.Tensor
    scale_shift_table: torch.Tensor
    prompt_scale_shift_table: torch.Tensor
    norm_eps: float = 1e-6
    qk_eps: float = 1e-6

    def to(self, device) -> "TextAttentionWeights":
        return TextAttentionWeights(
            self.to_q.to(device), self.to_k.to(device), self.to_v.to(device), self.to_out.to(device),
            self.q_norm_weight.to(device), self.k_norm_weight.to(device), self.scale_shift_table.to(device),
            self.prompt_scale_shift_table.to(device), self.norm_eps, self.qk_eps,
        )


def make_text_attention_weights(seed: int = 0, *, dim: int = DIM) -> TextAttentionWeights:
    """Random-init text cross-attention weights (CPU), distributed as ``make_weights``'s; input scales are
    placeholders until calibrated."""
    g = torch.Generator().manual_seed(seed)

    def linear() -> Fp8Linear:
        w = torch.randn((dim, dim), generator=g) * 0.02
        q, s = quantize_weight_e4m3(w)
        b = (torch.randn((dim,), generator=g) * 0.01).to(torch.bfloat16)
        return Fp8Linear(q, s, torch.tensor(1.0, dtype=torch.float32), b)

    to_q, to_k, to_v, to_out = linear(), linear(), linear(), linear()
    q_norm = (1.0 + 0.1 * torch.randn((dim,), generator=g)).to(torch.bfloat16)
    k_norm = (1.0 + 0.1 * torch.randn((dim,), generator=g)).to(torch.bfloat16)
    table = (torch.randn((TEXT_ADA_SLOTS, dim), generator=g) * 0.02).to(torch.float32)
    prompt_table = (torch.randn((PROMPT_ADA_SLOTS, dim), generator=g) * 0.02).to(torch.float32)
    return TextAttentionWeights(to_q, to_k, to_v, to_out, q_norm, k_norm, table, prompt_table)


@dataclass
class TextInputs:
    x: torch.Tensor  # bf16 [1, L, D]
    timestep: torch.Tensor  # bf16 [1, L, 9*D], stride-0 over tokens
    context: torch.Tensor  # bf16 [1, L_ctx, D]
    prompt_timestep: torch.Tensor  # bf16 [1, L_ctx, 2*D], stride-0 over tokens

    def to(self, device) -> "TextInputs":
        return TextInputs(
            self.x.to(device), self.timestep[:, :1].to(device).expand(self.timestep.shape), self.context.to(device),
            self.prompt_timestep[:, :1].to(device).expand(self.prompt_timestep.shape),
        )


def make_text_inputs(tokens: int, context_tokens: int = TEXT_CONTEXT_TOKENS, seed: int = 1, *,
                     dim: int = DIM) -> TextInputs:
    """Seeded inputs (CPU) of the text cross-attention branch: video tokens, their 9-slot uniform timestep
    embedding, the prompt context and its 2-slot uniform prompt timestep embedding."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((1, tokens, dim), generator=g).to(torch.bfloat16)
    ts = torch.randn((TEXT_ADA_SLOTS * dim,), generator=g).to(torch.bfloat16).view(1, 1, -1)
    context = torch.randn((1, context_tokens, dim), generator=g).to(torch.bfloat16)
    pts = torch.randn((PROMPT_ADA_SLOTS * dim,), generator=g).to(torch.bfloat16).view(1, 1, -1)
    return TextInputs(x, ts.expand(1, tokens, -1), context, pts.expand(1, context_tokens, -1))


@dataclass
class BlockInputs:
    x: torch.Tensor  # bf16 [1, L, D]
    timestep: torch.Tensor  # bf16 [1, L, 6*D] (stride-0 over tokens when uniform)
    cos: torch.Tensor
    sin: torch.Tensor

    def to(self, device) -> "BlockInputs":
        ts = self.timestep
        if ts.stride(1) == 0:
            ts = ts[:, :1].to(device).expand(ts.shape)
        else:
            ts = ts.to(device)
        return BlockInputs(self.x.to(device), ts, self.cos.to(device), self.sin.to(device))


def make_inputs(cfg: BlockConfig, seed: int = 1, *, dim: int = DIM, slots: int = ADA_SLOTS) -> BlockInputs:
    """Seeded block inputs (CPU) for one configuration; ``slots`` Ada slots in the timestep embedding (6 for
    the self-attention and FFN branches, 9 with the text cross-attention)."""
    g = torch.Generator().manual_seed(seed)
    L = cfg.tokens
    x = torch.randn((1, L, dim), generator=g)
    clean_tokens = cfg.clean_frames * cfg.grid_h * cfg.grid_w
    if clean_tokens:
        x[:, :clean_tokens] *= 0.5
    x = x.to(torch.bfloat16)
    if cfg.per_token_timestep:
        ts_clean = torch.randn((slots * dim,), generator=g)
        ts_noisy = torch.randn((slots * dim,), generator=g)
        is_clean = (torch.arange(L) < clean_tokens)[:, None]
        ts = torch.where(is_clean, ts_clean[None], ts_noisy[None]).unsqueeze(0).to(torch.bfloat16).contiguous()
    else:
        ts_vec = torch.randn((slots * dim,), generator=g).to(torch.bfloat16)
        ts = ts_vec.view(1, 1, -1).expand(1, L, slots * dim)
    cos, sin = rope_tables(cfg.frames, cfg.grid_h, cfg.grid_w)
    return BlockInputs(x, ts, cos, sin)


@dataclass
class LayerInputs:
    """Inputs of one DiT layer's video branches with the text cross-attention: the video tokens, their 9-slot
    timestep embedding (slots 0-2 self-attention, 3-5 FFN, 6-8 text cross-attention), the RoPE tables and the
    prompt context with its 2-slot timestep embedding."""

    x: torch.Tensor  # bf16 [1, L, D]
    timestep: torch.Tensor  # bf16 [1, L, 9*D] (stride-0 over tokens when uniform)
    cos: torch.Tensor
    sin: torch.Tensor
    context: torch.Tensor  # bf16 [1, L_ctx, D]
    prompt_timestep: torch.Tensor  # bf16 [1, L_ctx, 2*D], stride-0 over tokens

    def to(self, device) -> "LayerInputs":
        b = BlockInputs(self.x, self.timestep, self.cos, self.sin).to(device)
        pts = self.prompt_timestep[:, :1].to(device).expand(self.prompt_timestep.shape)
        return LayerInputs(b.x, b.timestep, b.cos, b.sin, self.context.to(device), pts)


def make_layer_inputs(cfg: BlockConfig, context_tokens: int = TEXT_CONTEXT_TOKENS, seed: int = 1, *,
                      dim: int = DIM) -> LayerInputs:
    """Seeded inputs (CPU) of a layer with the text cross-attention: ``make_inputs`` with 9 Ada slots, then the
    prompt context ~ N(0, 1) and its uniform 2-slot timestep embedding from a second generator."""
    b = make_inputs(cfg, seed, dim=dim, slots=TEXT_ADA_SLOTS)
    g = torch.Generator().manual_seed(seed + 7919)
    context = torch.randn((1, context_tokens, dim), generator=g).to(torch.bfloat16)
    pts = torch.randn((PROMPT_ADA_SLOTS * dim,), generator=g).to(torch.bfloat16).view(1, 1, -1)
    return LayerInputs(b.x, b.timestep, b.cos, b.sin, context, pts.expand(1, context_tokens, -1))


def small_config(tokens_frames: int = 1, grid_h: int = 2, grid_w: int = 8, **kw) -> BlockConfig:
    """A few-token configuration for parity tests."""
    return BlockConfig(f"small_{tokens_frames}x{grid_h}x{grid_w}", tokens_frames, grid_h, grid_w, **kw)
