"""Host logic of the attention-backend switch and the fail-closed video MSA branch (CPU), plus its GPU run."""

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
