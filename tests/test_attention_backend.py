"""Host logic of the attention-backend switch, the fail-closed video MSA branch (CPU, plus its GPU run) and the
fail-closed text cross-attention branch (CPU: declines and the weights it reads from the reference's modules)."""

import types

import pytest
import torch

from opengenie_b200 import attention_backend as ab


def test_choices_extend_the_reference_switch():
    assert "sdpa-cudnn" in ab.ATTENTION_CHOICES and "b200-native" in ab.ATTENTION_CHOICES
    assert ab.resolve_attention("b200-native") == "b200-native"
    assert ab.resolve_attention("sdpa-math") == "sdpa-math"
    # h100-fa3 falls through to h100-fa4 and then to sdpa-cudnn when neither FA3 nor FA4 imports
    assert ab.resolve_attention("h100-fa3") in ("flash-attn-3", "flash-attn-4", "sdpa-cudnn")
    with pytest.raises(ValueError):
        ab.resolve_attention("nope")


def test_pin_attention_sets_every_attention_module():
    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.attention_function = None

    model = torch.nn.Sequential(Attn(), torch.nn.Linear(2, 2), torch.nn.Sequential(Attn()))
    assert ab.pin_attention(model, "b200-native") == 2
    assert isinstance(model[0].attention_function, ab.B200NativeAttention)


def test_install_attention_class_patches_call():
    class FakeFlash:
        def __call__(self, q, k, v, heads):
            return "old"

    prev = ab.install_attention_class(FakeFlash, "b200-native")
    assert prev is not FakeFlash.__call__
    with pytest.raises(ValueError):  # CPU tensors: the b200 op refuses, no fallback
        FakeFlash()(torch.zeros(1, 4, 128, dtype=torch.bfloat16), torch.zeros(1, 4, 128, dtype=torch.bfloat16),
                    torch.zeros(1, 4, 128, dtype=torch.bfloat16), 1)


def test_video_msa_branch_declines_with_reference_reasons():
    block = types.SimpleNamespace(attn1=types.SimpleNamespace(to_gate_logits=None))
    vx = torch.zeros(1, 8, 4096)
    base = dict(self_attention_mask=None, self_attn_all_perturbed=False, self_attn_perturbation_mask=None,
                positional_embeddings=(None, None), timesteps=None)
    assert ab.video_msa_branch(block, types.SimpleNamespace(**base), torch.zeros(2, 8, 4096)) is None
    assert ab.video_msa_branch(block, types.SimpleNamespace(**{**base, "self_attention_mask": 1}), vx) is None
    assert ab.video_msa_branch(block, types.SimpleNamespace(**{**base, "self_attn_all_perturbed": True}), vx) is None
    assert ab.video_msa_branch(block, types.SimpleNamespace(**{**base, "positional_embeddings": None}), vx) is None
    assert ab.video_msa_branch(block, types.SimpleNamespace(**base), vx, token_counts={9216}) is None
    reasons = ab.collect_video_msa_branch_stats()["fallback_reasons"]
    for r in ("shape", "mask", "all_perturbed", "missing_rope", "token_count"):
        assert reasons.get(r, 0) >= 1


@pytest.mark.gpu
def test_video_msa_branch_equals_fused_block(ogx_lib):
    from opengenie_b200 import synthetic
    from opengenie_b200.video_block import VideoSelfAttentionBlock

    cfg = synthetic.small_config(1, 8, 16)
    inp = synthetic.make_inputs(cfg, seed=61).to("cuda")
    w = synthetic.make_weights(seed=62).to("cuda")
    ref_blk = VideoSelfAttentionBlock(w, "cuda")
    ref_blk.calibrate_input_scales(inp.x, inp.timestep, (inp.cos, inp.sin))
    w = ref_blk.w

    def lin(l):
        return types.SimpleNamespace(weight=l.weight, weight_scale=l.weight_scale, input_scale=l.input_scale, bias=l.bias)

    attn1 = types.SimpleNamespace(to_q=lin(w.to_q), to_k=lin(w.to_k), to_v=lin(w.to_v), to_out=[lin(w.to_out)],
                                  q_norm=types.SimpleNamespace(weight=w.q_norm_weight, eps=1e-6),
                                  k_norm=types.SimpleNamespace(weight=w.k_norm_weight, eps=1e-6), to_gate_logits=None)
    block = types.SimpleNamespace(attn1=attn1, scale_shift_table=w.scale_shift_table, norm_eps=1e-6)
    video = types.SimpleNamespace(timesteps=inp.timestep, positional_embeddings=(inp.cos, inp.sin),
                                  self_attention_mask=None, self_attn_all_perturbed=False,
                                  self_attn_perturbation_mask=None)
    out = ab.video_msa_branch(block, video, inp.x)
    assert out is not None
    assert torch.equal(out, ref_blk(inp.x, inp.timestep, (inp.cos, inp.sin)))


def _text_modules():
    def lin(i):
        return types.SimpleNamespace(weight=torch.full((2, 2), float(i)), weight_scale=torch.tensor(0.1 * i),
                                     input_scale=torch.tensor(0.01 * i), bias=torch.full((2,), float(i)))

    attn2 = types.SimpleNamespace(to_q=lin(1), to_k=lin(2), to_v=lin(3), to_out=[lin(4)],
                                  q_norm=types.SimpleNamespace(weight=torch.ones(4), eps=1e-5),
                                  k_norm=types.SimpleNamespace(weight=torch.ones(4) * 2, eps=1e-5), to_gate_logits=None)
    block = types.SimpleNamespace(cross_attention_adaln=True, scale_shift_table=torch.zeros(9, 4096),
                                  prompt_scale_shift_table=torch.zeros(2, 4096), norm_eps=1e-6)
    return block, attn2


def test_text_cross_attention_branch_declines_with_reasons():
    block, attn2 = _text_modules()
    x, ctx = torch.zeros(1, 8, 4096), torch.zeros(1, 5, 4096)
    call = ab.video_text_cross_attention_branch
    assert call(types.SimpleNamespace(**{**vars(block), "cross_attention_adaln": False}), x, ctx, attn2, None,
                None) is None
    assert call(types.SimpleNamespace(**{**vars(block), "prompt_scale_shift_table": None}), x, ctx, attn2, None,
                None) is None
    assert call(block, torch.zeros(2, 8, 4096), ctx, attn2, None, None) is None
    assert call(block, x, torch.zeros(1, 0, 4096), attn2, None, None) is None
    assert call(types.SimpleNamespace(**{**vars(block), "scale_shift_table": torch.zeros(6, 4096)}), x, ctx, attn2,
                None, None) is None
    assert call(block, x, ctx, attn2, None, None, context_mask=torch.ones(1, 5)) is None
    assert call(block, x, ctx, types.SimpleNamespace(**{**vars(attn2), "to_gate_logits": object()}), None,
                None) is None
    reasons = ab.collect_video_text_branch_stats()["fallback_reasons"]
    for r in ("no_cross_attention_adaln", "no_prompt_table", "shape", "context_shape", "table_shape", "mask",
              "gated_attention"):
        assert reasons.get(r, 0) >= 1, r


def test_text_attention_weights_read_from_the_reference_modules():
    block, attn2 = _text_modules()
    w = ab.text_attention_weights_from_modules(block, attn2)
    for got, mod in ((w.to_q, attn2.to_q), (w.to_k, attn2.to_k), (w.to_v, attn2.to_v), (w.to_out, attn2.to_out[0])):
        assert got.weight is mod.weight and got.weight_scale is mod.weight_scale
        assert got.input_scale is mod.input_scale and got.bias is mod.bias
    assert w.q_norm_weight is attn2.q_norm.weight and w.k_norm_weight is attn2.k_norm.weight
    assert w.scale_shift_table is block.scale_shift_table
    assert w.prompt_scale_shift_table is block.prompt_scale_shift_table
    assert w.norm_eps == 1e-6 and w.qk_eps == 1e-5


def test_branch_cache_rebuilds_on_changed_weights_and_forgets_freed_blocks():
    """The fused-branch caches key blocks weakly and check their source tensors: the same block with unchanged
    tensors gets the cached branch; an in-place change or a replaced tensor rebuilds it; a freed block's entry
    goes away (so a new block at a reused address is built afresh); blocks that cannot be weakly referenced
    are held by their entry."""
    import gc

    cache = ab._BranchCache()
    built = []

    def build():
        built.append(object())
        return built[-1]

    mod = torch.nn.Linear(4, 4)
    srcs = lambda: [mod.weight, mod.bias]  # noqa: E731
    first = cache.get(mod, srcs(), build)
    assert cache.get(mod, srcs(), build) is first and len(built) == 1
    with torch.no_grad():
        mod.weight.add_(1.0)  # in place: same address, new version
    second = cache.get(mod, srcs(), build)
    assert second is not first and len(built) == 2
    mod.bias = torch.nn.Parameter(torch.zeros(4))  # replaced tensor
    third = cache.get(mod, srcs(), build)
    assert third is not second and len(built) == 3
    assert len(cache) == 1
    del mod
    gc.collect()
    assert len(cache) == 0

    ns = types.SimpleNamespace(w=torch.ones(2))
    a = cache.get(ns, [ns.w], build)
    assert cache.get(ns, [ns.w], build) is a
    other = types.SimpleNamespace(w=torch.ones(2))
    assert cache.get(other, [other.w], build) is not a
    assert len(cache) == 2
