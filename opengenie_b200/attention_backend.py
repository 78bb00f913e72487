"""Attention-backend switch and block-branch installers with the B200-native path registered.

Mirrors the reference's switch (benchmarks/official_ltx23_benchmark.py:49-63 choices, `_resolve_attention`
:3746-3759, `_pin_attention` :3667-3703) and adds ``"b200-native"`` next to ``"sdpa-cudnn"``.  The
reference installs backends by monkey-patching ltx_core classes (`FlashAttention3.__call__`, :3374) or with
`set_attention_module_op` on the transformer builder; ltx_core is an external package, so the installers
here patch a class or a module tree handed to them, following the same pattern.

Also provides `video_msa_branch`, the counterpart of `_video_msa_branch_from_ada`
(ltx_serve/triton_ltx_ops.py:2891-2981): the whole video self-attention branch of a DiT block as one
fail-closed call that either returns the new residual stream or declines with a recorded reason; and
`video_text_cross_attention_branch`, the same for the text cross-attention with cross-attention AdaLN
(`_apply_video_text_cross_attention_adaln_from_ada`, :2810-2888).
"""

from __future__ import annotations

import importlib
import weakref
from collections import Counter

import torch

from . import ltx_ops

# The reference's choices plus the B200-native backend.
ATTENTION_CHOICES = (
    "h100-fa3", "h100-fa4", "automatic", "flash-attn-3", "flash-attn-4",
    "sdpa-flash", "sdpa-cudnn", "sdpa-efficient", "sdpa-math", "b200-native",
)


def _importable(module: str, attr: str | None = None) -> bool:
    try:
        mod = importlib.import_module(module)
        return attr is None or hasattr(mod, attr)
    except Exception:
        return False


def resolve_attention(attention: str) -> str:
    """`_resolve_attention` (official_ltx23_benchmark.py:3746-3759) with ``b200-native`` passed through."""
    if attention not in ATTENTION_CHOICES:
        raise ValueError(f"unknown attention backend: {attention}")
    if attention == "h100-fa3":
        return "flash-attn-3" if _importable("flash_attn_interface") else resolve_attention("h100-fa4")
    if attention != "h100-fa4":
        return attention
    return "flash-attn-4" if _importable("flash_attn.cute", "flash_attn_func") else "sdpa-cudnn"


class B200NativeAttention:
    """Attention backend callable with the reference's contract: ``(q, k, v, heads) -> out``, q [B, L, H*d]
    and k/v [B, L_kv, H*d] bf16, d = 128, no mask, scale d^-0.5 (official_ltx23_benchmark.py:3289-3373).
    L_kv may differ from L: the same backend serves the self-attention (attn1) and the text cross-attention
    (attn2, keys/values from the prompt context; the reference views k and v as [b, -1, heads, d], :3305)."""

    name = "b200-native"

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, mask=None) -> torch.Tensor:
        if mask is not None:
            raise ValueError("mask: the b200-native backend is dense bidirectional attention")
        return ltx_ops.attention(q, k, v, heads)


class TorchSdpaAttention:
    """torch SDPA with a fixed backend (the reference's ``sdpa-*`` names), for side-by-side runs."""

    _BACKENDS = {"sdpa-flash": "FLASH_ATTENTION", "sdpa-cudnn": "CUDNN_ATTENTION",
                 "sdpa-efficient": "EFFICIENT_ATTENTION", "sdpa-math": "MATH"}

    def __init__(self, name: str):
        from torch.nn.attention import SDPBackend

        self.name = name
        self.backend = getattr(SDPBackend, self._BACKENDS[name])

    def __call__(self, q, k, v, heads, mask=None):
        from torch.nn.attention import sdpa_kernel

        b, L, hd = q.shape
        qh, kh, vh = (t.reshape(b, -1, heads, hd // heads).transpose(1, 2) for t in (q, k, v))
        with sdpa_kernel(self.backend):
            o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask)
        return o.transpose(1, 2).reshape(b, -1, hd)


def attention_function(attention: str):
    """The backend callable for a (resolved) backend name."""
    name = resolve_attention(attention)
    if name == "b200-native":
        return B200NativeAttention()
    if name.startswith("sdpa-"):
        return TorchSdpaAttention(name)
    raise ImportError(f"backend {name} needs an external package (flash_attn / ltx_core) that is not installed")


def pin_attention(model: torch.nn.Module, attention: str) -> int:
    """Sets ``attention_function`` on every module of ``model`` that has one (the attention modules),
    as `_pin_attention`'s module op does for ltx_core's Attention; returns how many were pinned."""
    fn = attention_function(attention)
    n = 0
    for mod in model.modules():
        if hasattr(mod, "attention_function"):
            mod.attention_function = fn
            n += 1
    return n


def install_attention_class(cls, attention: str = "b200-native"):
    """Replaces ``cls.__call__`` with the backend (the reference's FlashAttention3.__call__ patch,
    official_ltx23_benchmark.py:3374); returns the previous ``__call__``."""
    fn = attention_function(attention)
    previous = cls.__call__

    def _call(self, q, k, v, heads, *args, **kwargs):
        return fn(q, k, v, heads)

    cls.__call__ = _call
    return previous


# ---------------------------------------------------------------- the whole branch
class _BranchCache:
    """Fused branches per reference block.  Entries are keyed weakly by the block object, so a freed block's
    entry goes with it and a new block at the same address never meets it; a block that cannot be weakly
    referenced is kept alive by its entry instead.  Each entry remembers the address and in-place version
    counter of every source tensor it was built from, and is rebuilt when one of them changed (weights
    reloaded in place, or a parameter replaced)."""

    def __init__(self):
        self._weak: weakref.WeakKeyDictionary = weakref.WeakKeyDictionary()
        self._strong: dict[int, tuple[object, tuple]] = {}

    @staticmethod
    def _source_key(tensors) -> tuple:
        return tuple((t.data_ptr(), t._version) for t in tensors if isinstance(t, torch.Tensor))

    def _lookup(self, block):
        try:
            return self._weak.get(block)
        except TypeError:  # not weakly referenceable
            entry = self._strong.get(id(block))
            return entry[1] if entry is not None and entry[0] is block else None

    def _store(self, block, value) -> None:
        try:
            self._weak[block] = value
        except TypeError:
            self._strong[id(block)] = (block, value)

    def get(self, block, tensors, build):
        """The cached branch of ``block`` if its source ``tensors`` are unchanged, else ``build()`` cached."""
        key = self._source_key(tensors)
        hit = self._lookup(block)
        if hit is None or hit[0] != key:
            hit = (key, build())
            self._store(block, hit)
        return hit[1]

    def __len__(self) -> int:
        return len(self._weak) + len(self._strong)


def _linear_tensors(m) -> list:
    return [getattr(m, name, None) for name in ("weight", "weight_scale", "input_scale", "bias")]


_MSA_BRANCH_CALLS = 0
_MSA_BRANCH_FALLBACK_REASONS: Counter = Counter()
_MSA_BLOCKS = _BranchCache()


def _decline(reason: str):
    _MSA_BRANCH_FALLBACK_REASONS[reason] += 1
    return None


def video_msa_branch(block, video, vx: torch.Tensor, *, token_counts: set[int] | None = None):
    """Video self-attention branch of a DiT block on the B200 kernels, or None with a recorded reason.

    Counterpart of `_video_msa_branch_from_ada` (ltx_serve/triton_ltx_ops.py:2891-2981): same
    fail-closed checks and reason names (`shape`, `token_count`, `mask`, `all_perturbed`,
    `missing_rope`), then AdaZero(0/1) -> FP8 Q/K/V -> Q/K RMSNorm + RoPE -> attention ->
    out-projection -> bias + gate(2) + residual as five sm_100a kernels.  ``block`` provides
    ``scale_shift_table``, ``norm_eps`` and ``attn1`` (FP8 linears ``to_q/to_k/to_v/to_out[0]`` with
    ``weight``/``weight_scale``/``input_scale``/``bias``, and ``q_norm``/``k_norm`` with ``weight``/``eps``);
    ``video`` provides ``timesteps`` and ``positional_embeddings`` (cos, sin).
    """
    global _MSA_BRANCH_CALLS
    from .synthetic import BlockWeights, Fp8Linear
    from .video_block import VideoSelfAttentionBlock

    if vx.ndim != 3 or vx.shape[0] != 1 or vx.shape[-1] != 4096:
        return _decline("shape")
    if token_counts is not None and vx.shape[1] not in token_counts:
        return _decline("token_count")
    if getattr(video, "self_attention_mask", None) is not None:
        return _decline("mask")
    if getattr(video, "self_attn_all_perturbed", False):
        return _decline("all_perturbed")
    if getattr(video, "self_attn_perturbation_mask", None) is not None:
        return _decline("perturbation_mask")
    pe = getattr(video, "positional_embeddings", None)
    if pe is None:
        return _decline("missing_rope")
    attn = block.attn1

    def build():
        def lin(m):
            return Fp8Linear(m.weight, m.weight_scale, m.input_scale, m.bias)

        w = BlockWeights(lin(attn.to_q), lin(attn.to_k), lin(attn.to_v), lin(attn.to_out[0]), attn.q_norm.weight,
                         attn.k_norm.weight, block.scale_shift_table, float(block.norm_eps),
                         float(getattr(attn.q_norm, "eps", 1e-6)))
        # gated checkpoints: the per-head gate 2*sigmoid(to_gate_logits(norm)) scales the attention output
        return VideoSelfAttentionBlock(w, vx.device, to_gate_logits=getattr(attn, "to_gate_logits", None))

    sources = [t for m in (attn.to_q, attn.to_k, attn.to_v, attn.to_out[0]) for t in _linear_tensors(m)]
    sources += [attn.q_norm.weight, attn.k_norm.weight, block.scale_shift_table]
    fused = _MSA_BLOCKS.get(block, sources, build)
    _MSA_BRANCH_CALLS += 1
    return fused(vx, video.timesteps, (pe[0], pe[1]))


def collect_video_msa_branch_stats() -> dict:
    """Call / decline counters, as `collect_video_msa_branch_stats` (triton_ltx_ops.py:2235-2266)."""
    return {"calls": _MSA_BRANCH_CALLS, "fallbacks": sum(_MSA_BRANCH_FALLBACK_REASONS.values()),
            "fallback_reasons": dict(_MSA_BRANCH_FALLBACK_REASONS)}


_TEXT_BRANCH_CALLS = 0
_TEXT_BRANCH_FALLBACK_REASONS: Counter = Counter()
_TEXT_BRANCHES = _BranchCache()


def _decline_text(reason: str):
    _TEXT_BRANCH_FALLBACK_REASONS[reason] += 1
    return None


def text_attention_weights_from_modules(block, attn):
    """The text cross-attention's weights read from the reference's module objects: ``attn`` (attn2) with FP8
    linears ``to_q/to_k/to_v/to_out[0]`` (``weight``, ``weight_scale``, ``input_scale``, ``bias``) and
    ``q_norm``/``k_norm`` (``weight``, ``eps``); ``block`` with the layer's ``scale_shift_table`` (9 slots),
    ``prompt_scale_shift_table`` and ``norm_eps``.  Tensors are taken as they are, not copied."""
    from .synthetic import Fp8Linear, TextAttentionWeights

    def lin(m):
        return Fp8Linear(m.weight, m.weight_scale, m.input_scale, m.bias)

    return TextAttentionWeights(lin(attn.to_q), lin(attn.to_k), lin(attn.to_v), lin(attn.to_out[0]),
                                attn.q_norm.weight, attn.k_norm.weight, block.scale_shift_table,
                                block.prompt_scale_shift_table, float(block.norm_eps),
                                float(getattr(attn.q_norm, "eps", 1e-6)))


def video_text_cross_attention_branch(block, x: torch.Tensor, context: torch.Tensor, attn, timestep: torch.Tensor,
                                      prompt_timestep: torch.Tensor, context_mask=None):
    """Video text cross-attention with cross-attention AdaLN on the B200 kernels, returning the new residual
    stream, or None with a recorded reason.

    Counterpart of `_apply_video_text_cross_attention_adaln_from_ada` (ltx_serve/triton_ltx_ops.py:2810-2888),
    same arguments.  Declines (the caller keeps the reference's path) when the block has no cross-attention
    AdaLN or no prompt table (`no_cross_attention_adaln`, `no_prompt_table`; the reference's own branches
    :2821-2835), on shapes other than batch 1 x 4096 (`shape`, `context_shape`), a table of fewer than 9
    slots (`table_shape`), a context mask (`mask`: pass the prompt's valid tokens as the context instead) and
    gated attention (`gated_attention`).  Otherwise the eight launches of ``VideoTextCrossAttention``, built
    once per block from its modules (and again when one of their tensors is replaced or changed in place).
    """
    global _TEXT_BRANCH_CALLS
    from .video_text_attention import VideoTextCrossAttention

    if not getattr(block, "cross_attention_adaln", False):
        return _decline_text("no_cross_attention_adaln")
    if getattr(block, "prompt_scale_shift_table", None) is None:
        return _decline_text("no_prompt_table")
    if x.ndim != 3 or x.shape[0] != 1 or x.shape[-1] != 4096:
        return _decline_text("shape")
    if context.ndim != 3 or context.shape[0] != 1 or context.shape[-1] != 4096 or context.shape[1] < 1:
        return _decline_text("context_shape")
    if block.scale_shift_table.ndim != 2 or block.scale_shift_table.shape[0] < 9:
        return _decline_text("table_shape")
    if context_mask is not None:
        return _decline_text("mask")
    if getattr(attn, "to_gate_logits", None) is not None:
        return _decline_text("gated_attention")
    sources = [t for m in (attn.to_q, attn.to_k, attn.to_v, attn.to_out[0]) for t in _linear_tensors(m)]
    sources += [attn.q_norm.weight, attn.k_norm.weight, block.scale_shift_table,
                getattr(block, "prompt_scale_shift_table", None)]
    branch = _TEXT_BRANCHES.get(
        block, sources, lambda: VideoTextCrossAttention(text_attention_weights_from_modules(block, attn), x.device))
    _TEXT_BRANCH_CALLS += 1
    return branch(x, timestep, context, prompt_timestep)


def collect_video_text_branch_stats() -> dict:
    """Call / decline counters of ``video_text_cross_attention_branch``."""
    return {"calls": _TEXT_BRANCH_CALLS, "fallbacks": sum(_TEXT_BRANCH_FALLBACK_REASONS.values()),
            "fallback_reasons": dict(_TEXT_BRANCH_FALLBACK_REASONS)}
