"""The multi-GPU (Ulysses) host logic on CPU: two gloo ranks run the real partition and both exchanges of
UlyssesPlan; the send buffers are filled with the layout the RoPE-scatter kernel writes (that kernel's
layout is checked on the GPU in test_gpu_ops.py::test_qkv_rope_scatter_layout)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from opengenie_b200.ulysses import UlyssesPlan


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def scatter_like_kernel(q, k, v, plan: UlyssesPlan):
    """[L/P, 4096] x3 -> send [P][L/P][3][H/P][128]: head h -> group h // (H/P), slot h % (H/P)."""
    Ll = q.shape[0]
    send = torch.empty(plan.qkv_send_shape(Ll), dtype=q.dtype)
    for j, t in enumerate((q, k, v)):
        th = t.view(Ll, plan.world, plan.heads_local, 128).permute(1, 0, 2, 3)
        send[:, :, j] = th
    return send


def _worker(rank, world, port, L, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = UlyssesPlan(world, rank)
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn((L, 4096), generator=g).to(torch.bfloat16) for _ in range(3))
        t0, t1 = plan.token_range(L)
        send = scatter_like_kernel(q[t0:t1], k[t0:t1], v[t0:t1], plan)
        recv = torch.empty_like(send)
        plan.exchange_qkv(send, recv)
        qv, kv, vv = plan.attention_views(recv, L)
        h0 = rank * plan.heads_local * 128
        h1 = h0 + plan.heads_local * 128
        ok1 = all(torch.equal(view[0], full[:, h0:h1]) for view, full in ((qv, q), (kv, k), (vv, v)))
        # exchange 2: per-rank attention output for its heads over all tokens, [L, H/P*128]
        o_full = torch.arange(L * 4096, dtype=torch.int32).view(L, 4096).to(torch.uint8)
        send2 = o_full[:, h0:h1].contiguous()
        recv2 = torch.empty(plan.out_send_shape(t1 - t0), dtype=torch.uint8)
        plan.exchange_out(send2, recv2)
        # the k-blocked A operand: A[t, s*H/P*128 + j] = recv2[s, t, j]
        a = recv2.permute(1, 0, 2).reshape(t1 - t0, 4096)
        ok2 = torch.equal(a, o_full[t0:t1])
        result[rank] = int(ok1) + 2 * int(ok2)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_exchanges_gloo(world):
    L = 8 * world
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, L, result), nprocs=world, start_method="spawn", join=True)
    assert dict(result) == {r: 3 for r in range(world)}


def test_plan_partition_and_guards():
    plan = UlyssesPlan(8, 3)
    assert plan.heads_local == 4
    assert plan.token_range(9216) == (3 * 1152, 4 * 1152)
    assert plan.qkv_send_shape(1152) == (8, 1152, 3, 4, 128)
    assert plan.out_send_shape(3600) == (8, 3600, 512)
    with pytest.raises(ValueError):
        plan.tokens_local(9217)
    with pytest.raises(ValueError):
        UlyssesPlan(3, 0)
    # the configurations' token counts split over 2/4/8 ranks
    for L in (2304, 9216, 28800):
        for P in (2, 4, 8):
            assert UlyssesPlan(P, 0).tokens_local(L) * P == L
