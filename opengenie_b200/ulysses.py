"""Ulysses sequence parallelism for the video self-attention block on one 8xB200 box.

One process per GPU.  Rank r owns tokens [r*L/P, (r+1)*L/P) for every
sequence-local stage (AdaZero + quantiser, Q/K/V GEMM, Q/K RMSNorm + RoPE,
out-projection + gated residual: RMSNorm spans all 32 heads, so it must run
before the exchange).  Around attention two all-to-alls over NVLink (NCCL) swap
the sharding:

  exchange 1 (sequence -> heads): the RoPE kernel writes Q/K/V straight into the
      send buffer [P dst][L/P][3][H/P][128]; the receive buffer
      [P src][L/P][3][H/P][128] is [L][3][H/P][128] in token order and feeds the
      attention kernel as strided q/k/v rows.
  exchange 2 (heads -> sequence): attention writes its e4m3-quantised output
      [L][H/P*128] (= [P dst][L/P][H/P*128]); the receive buffer
      [P src][L/P][H/P*128] is read by the out-projection GEMM through a 3-D
      tensor map (k-blocked A operand), so no permute runs.

The per-tensor activation scales are static, so quantising before exchange 2 is
exact and halves its bytes.  The reference is single-GPU (no collective anywhere);
this module is the multi-GPU extension the block needs at 2/4/8 GPUs.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ltx_ops
from ._lib import DTYPE_BF16
from .synthetic import FP8_MAX, BlockWeights
from .video_block import VideoSelfAttentionBlock


class UlyssesPlan:
    """Token partition, buffer shapes and the two exchanges (host logic; no kernels)."""

    def __init__(self, world: int, rank: int, *, heads: int = 32, head_dim: int = 128, group=None):
        if heads % world:
            raise ValueError(f"{heads} heads do not split over {world} ranks")
        self.world, self.rank, self.heads, self.head_dim, self.group = world, rank, heads, head_dim, group
        self.heads_local = heads // world

    def tokens_local(self, tokens: int) -> int:
        if tokens % self.world:
            raise ValueError(f"{tokens} tokens do not split over {self.world} ranks")
        return tokens // self.world

    def token_range(self, tokens: int) -> tuple[int, int]:
        n = self.tokens_local(tokens)
        return self.rank * n, (self.rank + 1) * n

    def qkv_send_shape(self, tokens_local: int) -> tuple[int, ...]:
        return (self.world, tokens_local, 3, self.heads_local, self.head_dim)

    def out_send_shape(self, tokens_local: int) -> tuple[int, ...]:
        return (self.world, tokens_local, self.heads_local * self.head_dim)

    def _all_to_all(self, recv: torch.Tensor, send: torch.Tensor) -> None:
        dist.all_to_all_single(recv.view(torch.uint8), send.view(torch.uint8), group=self.group)

    def exchange_qkv(self, send: torch.Tensor, recv: torch.Tensor) -> None:
        """Sequence -> heads: send [P dst][L/P][3][H/P][d] -> recv [P src][L/P][3][H/P][d]."""
        self._all_to_all(recv, send)

    def exchange_out(self, send: torch.Tensor, recv: torch.Tensor) -> None:
        """Heads -> sequence: send [P dst][L/P][H/P*d] -> recv [P src][L/P][H/P*d]."""
        self._all_to_all(recv, send)

    def attention_views(self, recv: torch.Tensor, tokens: int):
        """q/k/v [1, L, H/P*d] views of the receive buffer (token rows strided by 3*H/P*d)."""
        flat = recv.reshape(1, tokens, 3 * self.heads_local * self.head_dim)
        w = self.heads_local * self.head_dim
        return flat[..., :w], flat[..., w:2 * w], flat[..., 2 * w:]


class PeerExchange:
    """Receive buffers shared between the ranks' processes with CUDA IPC, and the cross-GPU barrier.

    `share(t)` returns, for every rank, a device pointer to that rank's copy of ``t`` (the local
    pointer for this rank, IPC mappings for the others), so kernels can store straight into a peer's
    buffer over NVLink.  `barrier()` orders those stores before the peers read them (a bounded-wait
    signal exchange, one 32-thread kernel on the current stream).
    """

    def __init__(self, group, device):
        self._ct = ctypes
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self._opened: dict[bytes, int] = {}
        # [0, 8) arrival slots written by the peers, [8] barriers passed (advanced by the kernel)
        self.signals = torch.zeros(16, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)  # zeroed before any peer can store into it
        self.signal_ptrs = self.share(self.signals)
        self._signal_arr = (ctypes.c_void_p * self.world)(*self.signal_ptrs)

    def share(self, t: torch.Tensor) -> list[int]:
        ct = self._ct
        handle = (ct.c_char * 64)()
        off = ct.c_int64(0)
        _lib.call("ogx_ipc_get_handle", t.data_ptr(), handle, ct.byref(off))
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, (bytes(handle), int(off.value)), group=self.group)
        ptrs = []
        for r, (h, o) in enumerate(gathered):
            if r == self.rank:
                ptrs.append(t.data_ptr())
                continue
            base = self._opened.get(h)
            if base is None:
                b = ct.c_void_p()
                _lib.call("ogx_ipc_open_handle", h, ct.byref(b))
                base = self._opened[h] = int(b.value)
            ptrs.append(base + o)
        return ptrs

    def barrier(self) -> None:
        """Enqueues the barrier on the current stream (capturable: the epoch lives in device memory)."""
        _lib.call("ogx_peer_barrier", self.signals.data_ptr(), self._signal_arr, self.rank, self.world,
                  torch.cuda.current_stream(self.device).cuda_stream)

    def close(self) -> None:
        for base in self._opened.values():
            _lib.call("ogx_ipc_close_handle", base)
        self._opened.clear()


class UlyssesVideoSelfAttention:
    """The video self-attention block sharded over the ranks of ``group`` (one GPU each)."""


    def __init__(self, weights: BlockWeights, device, group=None, *, exchange: str = "nvlink"):
        """``exchange``: "nvlink" (producer kernels store into the peers' receive buffers, shared with
        CUDA IPC) or "nccl" (two all_to_all_single collectives)."""
        if exchange not in ("nvlink", "nccl"):
            raise ValueError(exchange)
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.plan = UlyssesPlan(world, rank, group=group)
        self.exchange = exchange
        self.peer = PeerExchange(group, device) if exchange == "nvlink" else None
        # adazero+quant, QKV GEMM, RoPE, attention, out-proj GEMM (+ two peer barriers over NVLink)
        self.kernel_launches_per_step = 7 if self.peer is not None else 5
        self.blk = VideoSelfAttentionBlock(weights, device)
        self.w = self.blk.w
        self.device = self.blk.device
        self._ws: dict[int, dict[str, torch.Tensor]] = {}
        # (name, start, end) CUDA events per stage when profiling (as the reference's
        # `_profile_video_msa_phase`, ltx_serve/triton_ltx_ops.py:2270-2279)
        self.profile = False
        self.phase_events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def _phase(self, name: str):
        """Context manager recording CUDA events around a stage on the current stream."""
        blk = self

        class _P:
            def __enter__(self):
                if blk.profile:
                    self.e0 = torch.cuda.Event(enable_timing=True)
                    self.e0.record()

            def __exit__(self, *exc):
                if blk.profile:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record()
                    blk.phase_events.append((name, self.e0, e1))

        return _P()

    def phase_summary(self) -> dict[str, float]:
        """Average ms per stage over the profiled calls (synchronises)."""
        torch.cuda.synchronize(self.device)
        acc: dict[str, list[float]] = {}
        for name, e0, e1 in self.phase_events:
            acc.setdefault(name, []).append(e0.elapsed_time(e1))
        return {k: sum(v) / len(v) for k, v in acc.items()}

    # ------------------------------------------------------------------ buffers
    def workspace(self, tokens_local: int) -> dict[str, torch.Tensor]:
        ws = self._ws.get(tokens_local)
        if ws is None:
            p = self.plan
            L = tokens_local * p.world
            ws = {
                "xq": torch.empty((1, tokens_local, 4096), device=self.device, dtype=torch.float8_e4m3fn),
                "xq3": torch.empty((3, 1, tokens_local, 4096), device=self.device, dtype=torch.float8_e4m3fn),
                "qkv": torch.empty((tokens_local, 3 * 4096), device=self.device, dtype=torch.bfloat16),
                "send1": torch.empty(p.qkv_send_shape(tokens_local), device=self.device, dtype=torch.bfloat16),
                "recv1": torch.empty(p.qkv_send_shape(tokens_local), device=self.device, dtype=torch.bfloat16),
                "send2": torch.empty((L, p.heads_local * p.head_dim), device=self.device, dtype=torch.float8_e4m3fn),
                "recv2": torch.empty(p.out_send_shape(tokens_local), device=self.device, dtype=torch.float8_e4m3fn),
            }
            if self.peer is not None:
                # where this rank's slot starts in every rank's receive buffers
                slot1 = p.rank * tokens_local * 3 * p.heads_local * p.head_dim * 2
                slot2 = p.rank * tokens_local * p.heads_local * p.head_dim
                dst1 = [ptr + slot1 for ptr in self.peer.share(ws["recv1"])]
                dst2 = [ptr + slot2 for ptr in self.peer.share(ws["recv2"])]
                ws["recv1_dst"] = (ctypes.c_void_p * p.world)(*dst1)
                ws["recv2_dst"] = (ctypes.c_void_p * p.world)(*dst2)
            self._ws[tokens_local] = ws
        return ws

    def local_slice(self, t: torch.Tensor) -> torch.Tensor:
        t0, t1 = self.plan.token_range(t.shape[1])
        return t[:, t0:t1]

    # ------------------------------------------------------------------ stages
    def _rope_source(self, rope, Ll: int) -> tuple:
        """The rope arguments of the entry points: (cos, sin) tables of this rank's tokens, or
        (RopePositions, first token of the slice) -> frequency tables, grid, first token."""
        if isinstance(rope[0], ltx_ops.RopePositions):
            pos, token0 = rope
            reason = ltx_ops.rope_positions_guard_reason(pos, self.device)
            if reason is None and (token0 < 0 or token0 + Ll > pos.tokens):
                reason = "rope_shape"
            if reason is not None:
                raise ValueError(reason)
            return True, (pos.inv_freq.data_ptr(), pos.slot_axis.data_ptr(), pos.grid_h, pos.grid_w, int(token0))
        cos_loc, sin_loc = rope
        if cos_loc.shape[2] != Ll or sin_loc.shape != cos_loc.shape:
            raise ValueError("rope_shape")
        return False, (cos_loc.data_ptr(), sin_loc.data_ptr(), ltx_ops._code(cos_loc), cos_loc.stride(1),
                       cos_loc.stride(2))

    def _stage_adazero(self, x_loc, ts_loc, ws) -> None:
        w = self.w
        if self.blk.shared_quant:
            ltx_ops.fused_adazero_from_ada_fp8(x_loc, w.norm_eps, w.scale_shift_table, ts_loc, w.to_q.input_scale,
                                               shift_index=0, scale_index=1, out=ws["xq"])
        else:  # Q, K and V linears with different input scales: one e4m3 copy of the activations per linear
            ltx_ops.fused_adazero_from_ada_fp8_planes(x_loc, w.norm_eps, w.scale_shift_table, ts_loc, self.blk.s_in3,
                                                      shift_index=0, scale_index=1, out=ws["xq3"])

    def _stage_qkv_gemm(self, ws) -> None:
        w = self.w
        if self.blk.shared_quant:
            ltx_ops.fp8_scaled_mm(ws["xq"], self.blk.w_qkv, w.to_q.input_scale, self.blk.s_qkv, bias=self.blk.b_qkv,
                                  out=ws["qkv"], n_per_scale=4096)
        else:
            ltx_ops.fp8_scaled_mm_planes(ws["xq3"], self.blk.w_qkv, self.blk.s_in3, self.blk.s_qkv,
                                         bias=self.blk.b_qkv, out=ws["qkv"])

    def _stage_rope_to_peers(self, Ll: int, rope, ws) -> None:
        """Q/K RMSNorm + RoPE storing each head group into its rank's receive buffer, then the barrier."""
        w, p = self.w, self.plan
        qkv = ws["qkv"]
        D = 4096
        positions, src = self._rope_source(rope, Ll)
        _lib.call(
            "ogx_video_qkv_rmsnorm_rope_positions_to_peers" if positions else "ogx_video_qkv_rmsnorm_rope_to_peers",
            qkv.data_ptr(), qkv[:, D:].data_ptr(), qkv[:, 2 * D:].data_ptr(), Ll, qkv.stride(0),
            w.q_norm_weight.data_ptr(), w.k_norm_weight.data_ptr(), ltx_ops._code(w.q_norm_weight),
            float(w.qk_eps), *src, ws["recv1_dst"], p.world, 3 * p.heads_local * p.head_dim,
            ltx_ops._stream(qkv),
        )

    def _stage_attention_to_peers(self, L: int, Ll: int, ws) -> None:
        """Attention on this rank's heads, each output row stored into the owning rank's receive buffer."""
        w, p = self.w, self.plan
        q, k, v = p.attention_views(ws["recv1"], L)
        _lib.call(
            "ogx_attention_fwd_e4m3_to_peers",
            q.data_ptr(), k.data_ptr(), v.data_ptr(), L, p.heads_local, q.stride(1), 128 ** -0.5,
            w.to_out.input_scale.data_ptr(), ws["recv2_dst"], p.world, Ll, p.heads_local * p.head_dim,
            ltx_ops._stream(q),
        )

    def _stage_out_proj(self, x_loc, ts_loc, ws, out) -> None:
        w, p = self.w, self.plan
        Ll = x_loc.shape[1]
        ts_view = ltx_ops._ts_view(x_loc, w.scale_shift_table, ts_loc)
        recv2 = ws["recv2"]
        if (recv2.shape != p.out_send_shape(Ll) or ts_view.shape[1] != Ll or x_loc.shape != out.shape
                or not out.is_contiguous()):
            raise ValueError("out_projection_shape")
        _lib.call(
            "ogx_fp8_scaled_mm_residual_gate_kblocked",
            recv2.data_ptr(), Ll, 4096, p.heads_local * p.head_dim, w.to_out.weight.data_ptr(), 4096,
            w.to_out.weight.stride(0), w.to_out.input_scale.data_ptr(), w.to_out.weight_scale.data_ptr(), 4096,
            w.to_out.bias.data_ptr(), ltx_ops._code(w.to_out.bias), x_loc.data_ptr(), x_loc.stride(1),
            w.scale_shift_table.data_ptr(), ltx_ops._code(w.scale_shift_table), w.scale_shift_table.stride(0),
            ts_view.data_ptr(), ltx_ops._code(ts_view), ts_view.stride(1), ts_view.stride(2), 2,
            out.data_ptr(), out.stride(1), ltx_ops._stream(x_loc),
        )

    def _qkv_and_exchange(self, x_loc, ts_loc, rope, ws):
        """``rope``: (cos, sin) tables of this rank's tokens, or (RopePositions, first token of the slice)."""
        w = self.w
        p = self.plan
        Ll = x_loc.shape[1]
        qkv = ws["qkv"]
        if qkv.shape != (Ll, 3 * 4096) or not qkv.is_contiguous():
            raise ValueError("qkv workspace shape")
        with self._phase("adazero_quant"):
            self._stage_adazero(x_loc, ts_loc, ws)
        with self._phase("qkv_gemm"):
            self._stage_qkv_gemm(ws)
        send = ws["send1"]
        D = 4096
        if send.shape != p.qkv_send_shape(Ll):
            raise ValueError("rope_shape")
        if self.peer is not None:
            with self._phase("rope_to_peers"):
                self._stage_rope_to_peers(Ll, rope, ws)
            with self._phase("barrier_seq_to_heads"):
                self.peer.barrier()
            return p.attention_views(ws["recv1"], Ll * p.world)
        positions, src = self._rope_source(rope, Ll)
        self._phase_ctx = self._phase("rope_scatter")
        self._phase_ctx.__enter__()
        _lib.call(
            "ogx_video_qkv_rmsnorm_rope_positions_scatter" if positions else "ogx_video_qkv_rmsnorm_rope_scatter",
            qkv.data_ptr(), qkv[:, D:].data_ptr(), qkv[:, 2 * D:].data_ptr(), Ll, qkv.stride(0),
            w.q_norm_weight.data_ptr(), w.k_norm_weight.data_ptr(), ltx_ops._code(w.q_norm_weight), float(w.qk_eps),
            *src, send[:, :, 0].data_ptr(), send[:, :, 1].data_ptr(), send[:, :, 2].data_ptr(), send.stride(1),
            send.stride(0), p.heads_local, ltx_ops._stream(qkv),
        )
        self._phase_ctx.__exit__(None, None, None)
        with self._phase("exchange_seq_to_heads"):
            p.exchange_qkv(send, ws["recv1"])
        return p.attention_views(ws["recv1"], Ll * p.world)

    def forward_local(self, x_loc: torch.Tensor, timestep: torch.Tensor, pe: tuple[torch.Tensor, torch.Tensor], *,
                      out: torch.Tensor | None = None):
        """x_loc: this rank's tokens [1, L/P, 4096]; timestep and pe span all L tokens."""
        p = self.plan
        w = self.w
        Ll = x_loc.shape[1]
        L = Ll * p.world
        t0 = p.rank * Ll
        ts_loc = timestep[:, t0:t0 + Ll]
        if isinstance(pe, ltx_ops.RopePositions):
            rope = (pe, t0)
        else:
            rope = (pe[0][:, :, t0:t0 + Ll], pe[1][:, :, t0:t0 + Ll])
        ws = self.workspace(Ll)
        q, k, v = self._qkv_and_exchange(x_loc, ts_loc, rope, ws)
        send2 = ws["send2"]
        if self.peer is not None:
            with self._phase("attention_to_peers"):
                self._stage_attention_to_peers(L, Ll, ws)
            with self._phase("barrier_heads_to_seq"):
                self.peer.barrier()
        else:
            with self._phase("attention"):
                ltx_ops.attention(q, k, v, p.heads_local, out=send2.view(1, L, -1),
                                  out_e4m3_scale=w.to_out.input_scale)
            with self._phase("exchange_heads_to_seq"):
                p.exchange_out(send2, ws["recv2"])
        if out is None:
            out = torch.empty_like(x_loc)
        with self._phase("out_gemm_residual"):
            self._stage_out_proj(x_loc, ts_loc, ws, out)
        return out

    def forward(self, x: torch.Tensor, timestep: torch.Tensor, pe: tuple[torch.Tensor, torch.Tensor]):
        """x: all tokens [1, L, 4096] (each rank reads its own slice); returns this rank's output slice."""
        return self.forward_local(self.local_slice(x), timestep, pe)

    __call__ = forward

    # ------------------------------------------------------------------ calibration / timing
    @torch.no_grad()
    def calibrate_input_scales(self, x: torch.Tensor, timestep: torch.Tensor, pe) -> None:
        """Static input scales = global amax / 448 (max over ranks) of each FP8 linear's input."""
        p = self.plan
        w = self.w
        x_loc = self.local_slice(x)
        Ll = x_loc.shape[1]
        t0 = p.rank * Ll
        ts_loc = timestep[:, t0:t0 + Ll]
        norm = ltx_ops.fused_adazero_from_ada(x_loc, w.norm_eps, w.scale_shift_table, ts_loc, shift_index=0,
                                              scale_index=1)
        amax = norm.float().abs().amax().reshape(1)
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
        s_in = (amax.clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)
        for lin in (w.to_q, w.to_k, w.to_v):
            lin.input_scale = s_in.clone()
        self.blk.input_scales_changed()
        ws = self.workspace(Ll)
        rope = (pe, t0) if isinstance(pe, ltx_ops.RopePositions) else (pe[0][:, :, t0:t0 + Ll], pe[1][:, :, t0:t0 + Ll])
        q, k, v = self._qkv_and_exchange(x_loc, ts_loc, rope, ws)
        attn = ltx_ops.attention(q, k, v, p.heads_local)
        amax = attn.float().abs().amax().reshape(1)
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
        w.to_out.input_scale = (amax.clamp_min(1e-12) / FP8_MAX).reshape(()).to(torch.float32)

    def time_stages(self, x_loc: torch.Tensor, timestep: torch.Tensor, pe, steps: int = 20,
                    warmup: int = 3) -> dict[str, float]:
        """Device time (ms) of each stage of a step on this rank, every stage replayed alone from a CUDA graph
        on the buffers a full step left (``time_launches``), so host overhead adds nothing.  The exchange
        stages include their barrier, and every rank replays the same stages in the same order, so a barrier
        stage also holds the wait for the slowest rank.  NVLink exchange only (NCCL's collectives stay
        eager); returns {} otherwise."""
        from .graphs import time_launches

        if self.peer is None:
            return {}
        p = self.plan
        Ll = x_loc.shape[1]
        L = Ll * p.world
        t0 = p.rank * Ll
        ts_loc = timestep[:, t0:t0 + Ll]
        rope = (pe, t0) if isinstance(pe, ltx_ops.RopePositions) else (pe[0][:, :, t0:t0 + Ll], pe[1][:, :, t0:t0 + Ll])
        out = torch.empty_like(x_loc)
        self.forward_local(x_loc, timestep, pe, out=out)
        ws = self.workspace(Ll)

        def rope_exchange():
            self._stage_rope_to_peers(Ll, rope, ws)
            self.peer.barrier()

        def attention_exchange():
            self._stage_attention_to_peers(L, Ll, ws)
            self.peer.barrier()

        stages = {
            "adazero_quant": lambda: self._stage_adazero(x_loc, ts_loc, ws),
            "qkv_gemm": lambda: self._stage_qkv_gemm(ws),
            "rope_to_peers+barrier": rope_exchange,
            "attention_to_peers+barrier": attention_exchange,
            "out_gemm_residual": lambda: self._stage_out_proj(x_loc, ts_loc, ws, out),
            "barrier_alone": self.peer.barrier,
        }
        return {name: time_launches(fn, steps, warmup, self.device) for name, fn in stages.items()}

    def time_attention(self, steps: int, warmup: int = 3) -> float:
        """Average device time (ms) of this rank's attention kernel (H/P heads over all L tokens), launches
        replayed from one CUDA graph."""
        from .graphs import time_launches

        Ll = max(self._ws)
        ws = self._ws[Ll]
        L = Ll * self.plan.world
        q, k, v = self.plan.attention_views(ws["recv1"], L)
        out = ws["send2"].view(1, L, -1)
        return time_launches(
            lambda: ltx_ops.attention(q, k, v, self.plan.heads_local, out=out, out_e4m3_scale=self.w.to_out.input_scale),
            steps, warmup, self.device)


__all__ = ["UlyssesPlan", "UlyssesVideoSelfAttention", "DTYPE_BF16"]
