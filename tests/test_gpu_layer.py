"""The video branches of DiT layers chained (self-attention block then FFN branch per layer): the stack equals
the composition of its parts, and one CUDA graph replay of the stack equals the eager stack."""

import pytest
import torch

from gpu_util import status_clean

pytestmark = pytest.mark.gpu


def test_layer_stack_equals_composition_and_graph_replay(ogx_lib):
    from opengenie_b200 import synthetic
    from opengenie_b200.graphs import StepGraph
    from opengenie_b200.video_layer import VideoLayer, VideoLayerStack

    cfg = synthetic.small_config(2, 6, 25)
    inp = synthetic.make_inputs(cfg, seed=91).to("cuda")
    pe = (inp.cos, inp.sin)
    layers = [VideoLayer(synthetic.make_weights(seed=92 + i), synthetic.make_ffn_weights(seed=95 + i), "cuda")
              for i in range(3)]
    stack = VideoLayerStack(layers)
    stack.calibrate_input_scales(inp.x, inp.timestep, pe)
    out = stack(inp.x, inp.timestep, pe).clone()
    x = inp.x
    for layer in layers:
        x = layer.ffn(layer.attn(x, inp.timestep, pe), inp.timestep)
    assert torch.equal(out, x)
    buf = torch.empty_like(inp.x)
    g = StepGraph(lambda: stack(inp.x, inp.timestep, pe, out=buf), "cuda")
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(buf, out)
    assert torch.isfinite(out.float()).all()
    assert status_clean()
