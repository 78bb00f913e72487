"""Multi-GPU parity: the Ulysses-sharded block (NCCL all-to-alls, one process per GPU) returns, for every
rank's tokens, exactly the single-GPU block's output.  Runs on 2+ GPUs; skipped on one."""

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg_name, exchange, result):
    import torch.distributed as dist

    from opengenie_b200 import _lib, synthetic
    from opengenie_b200.ulysses import UlyssesVideoSelfAttention
    from opengenie_b200.video_block import VideoSelfAttentionBlock

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg = synthetic.CONFIGS[cfg_name]
        inp = synthetic.make_inputs(cfg, seed=51).to(f"cuda:{rank}")
        w = synthetic.make_weights(seed=52)
        ul = UlyssesVideoSelfAttention(w, f"cuda:{rank}", dist.group.WORLD, exchange=exchange)
        ul.calibrate_input_scales(inp.x, inp.timestep, (inp.cos, inp.sin))
        out = ul(inp.x, inp.timestep, (inp.cos, inp.sin))
        single = VideoSelfAttentionBlock(w, f"cuda:{rank}")
        single.calibrate_input_scales(inp.x, inp.timestep, (inp.cos, inp.sin))
        ref = single(inp.x, inp.timestep, (inp.cos, inp.sin))
        t0, t1 = ul.plan.token_range(cfg.tokens)
        same_scales = bool(torch.equal(ul.w.to_out.input_scale, single.w.to_out.input_scale)
                           and torch.equal(ul.w.to_q.input_scale, single.w.to_q.input_scale))
        torch.cuda.synchronize()
        dist.barrier()  # the ranks enter the second step together (the peer barrier's wait is bounded)
        # a second step through the same buffers (the exchange's barriers order reuse)
        out2 = ul(inp.x, inp.timestep, (inp.cos, inp.sin))
        torch.cuda.synchronize()
        ok = bool(torch.equal(out, ref[:, t0:t1])) and bool(torch.equal(out2, ref[:, t0:t1]))
        if ul.peer is not None:
            # the step (launches and peer barriers) captured once as a CUDA graph, replayed twice
            from opengenie_b200.graphs import StepGraph

            x_loc = ul.local_slice(inp.x)
            out_g = torch.empty_like(x_loc)
            dist.barrier()
            g = StepGraph(lambda: ul.forward_local(x_loc, inp.timestep, (inp.cos, inp.sin), out=out_g),
                          f"cuda:{rank}")
            for _ in range(2):
                out_g.zero_()
                dist.barrier()
                g.replay()
                torch.cuda.synchronize()
                ok = ok and bool(torch.equal(out_g, ref[:, t0:t1]))
            del g
        result[rank] = (ok, same_scales, _lib.device_status(clear=True))
        if ul.peer is not None:
            dist.barrier()
            ul.peer.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
@pytest.mark.parametrize("cfg_name", ["c0_l2304", "c2_df_l9216", "c4_l28800"])
@pytest.mark.parametrize("exchange", ["nvlink", "nccl"])
def test_ulysses_block_equals_single_gpu(ogx_lib, cfg_name, exchange):
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    world = 8 if world >= 8 else (4 if world >= 4 else 2)
    result = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), cfg_name, exchange, result), nprocs=world,
                       start_method="spawn",
                       join=True)
    assert dict(result) == {r: (True, True, 0) for r in range(world)}
