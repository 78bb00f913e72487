"""GPU parity of the HBM-bound stages (C ABI through opengenie_b200.ltx_ops) against the oracle and the
reference's golden outputs.  Bit-exact where the reference is bitwise; <= 1 bf16 ulp where the kernel and
the oracle share single-rounding semantics; the reference's own tolerances against its torch fallbacks."""

import os

import numpy as np
import pytest
import torch

from gpu_util import O, bf16_bits, codes, from_bits, status_clean, to_np, within_ulps

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ops(ogx_lib):
    from opengenie_b200 import ltx_ops

    return ltx_ops


def test_quantiser_bf16_all_bit_patterns_bit_exact(ops):
    d = np.load(os.path.join(GOLD, "quant_bf16.npz"))
    x = from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16)).reshape(256, 256)
    for s, ref in zip(d["scales"], d["codes"]):
        q = ops.fused_fp8_quantize_e4m3(x, torch.tensor(float(s), device="cuda"))
        got = codes(q).reshape(-1)
        assert np.array_equal(got, ref), f"scale {s}: {(got != ref).sum()} codes differ"
    assert status_clean()


def test_quantiser_f16_all_bit_patterns_bit_exact(ops):
    d = np.load(os.path.join(GOLD, "quant_f16.npz"))
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = torch.from_numpy(bits.view(np.int16)).view(torch.float16).cuda().reshape(256, 256)
    for s, ref in zip(d["scales"], d["codes"]):
        got = codes(ops.fused_fp8_quantize_e4m3(x, torch.tensor(float(s), device="cuda"))).reshape(-1)
        assert np.array_equal(got, ref), f"scale {s}: {(got != ref).sum()} codes differ"


def test_quantiser_single_rounding_mode_matches_oracle(ops):
    x = from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16)).reshape(256, 256)
    xf = O.bf16_from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    for s in (1.0, 0.0371, 0.00123):
        got = codes(ops.fused_fp8_quantize_e4m3(x, torch.tensor(s, device="cuda"), quant_mode=ops.QUANT_SINGLE)).reshape(-1)
        ref = O.quantize_e4m3(xf, s, mode="single")
        finite = ~np.isnan(xf)
        assert np.array_equal(got[finite], ref[finite])


@pytest.mark.parametrize("n", [0, 1, 7, 4096 * 3 + 5, 9216 * 4096])
def test_quantiser_sizes_with_outliers_bit_exact(ops, n):
    """C3's activation distribution: N(0,1) with 0.1% outliers x50, s = amax/448; ragged tails."""
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, generator=g)
    if n:
        idx = torch.randperm(n, generator=g)[: max(1, n // 1000)]
        x[idx] *= 50
    xb = x.to(torch.bfloat16)
    s = float(xb.float().abs().amax() / 448.0) if n else 1.0
    got = codes(ops.fused_fp8_quantize_e4m3(xb.cuda(), torch.tensor(s, device="cuda")))
    ref = O.quantize_e4m3(xb.float().numpy(), s)
    assert np.array_equal(got, ref)


def test_quantiser_vs_torch_cuda_path_is_reported(ops, capsys):
    """Informational: the reference's torch expression evaluated by torch on the GPU (where the 0-dim
    fp32 reciprocal meets the bf16 tensor through torch's CUDA type promotion)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(9216 * 512, generator=g).to(torch.bfloat16).cuda()
    s = torch.tensor(0.0371, device="cuda")
    torch_cuda = torch.clamp(x * s.reciprocal(), -448.0, 448.0).to(torch.float8_e4m3fn)
    ours = ops.fused_fp8_quantize_e4m3(x, s)
    differ = int((codes(torch_cuda) != codes(ours)).sum())
    print(f"torch-on-CUDA path vs kernel (CPU torch-path semantics): {differ} of {x.numel()} codes differ")


def _ada_case(rows, cols, table_dtype, ts_dtype, uniform, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((1, rows, cols), generator=g).to(torch.bfloat16)
    table = (torch.randn((6, cols), generator=g) * 0.5).to(table_dtype)
    if uniform:
        ts = torch.randn((6 * cols,), generator=g).to(ts_dtype).view(1, 1, -1).expand(1, rows, 6 * cols)
    else:
        ts = torch.randn((1, rows, 6 * cols), generator=g).to(ts_dtype)
    return x, table, ts


@pytest.mark.parametrize("cols", [2048, 4096])
@pytest.mark.parametrize("table_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ts_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("uniform", [True, False])
def test_adazero_from_ada_vs_oracle(ops, cols, table_dtype, ts_dtype, uniform):
    x, table, ts = _ada_case(13, cols, table_dtype, ts_dtype, uniform, seed=cols)
    ts_d = ts[:, :1].cuda().expand(ts.shape) if uniform else ts.cuda()
    y = ops.fused_adazero_from_ada(x.cuda(), 1e-6, table.cuda(), ts_d, shift_index=0, scale_index=1)
    ref = O.adazero_from_ada(x, 1e-6, table, ts.reshape(1, 13, 6, cols), shift_index=0, scale_index=1,
                             table_is_bf16=table_dtype == torch.bfloat16, ts_is_bf16=ts_dtype == torch.bfloat16)
    # fp32 arithmetic (as the reference's kernel) vs exact: 1 ulp, plus 1e-5 absolute where
    # shift nearly cancels x*inv_rms*(1+scale)
    ok, worst = within_ulps(to_np(y), ref, ulps=1.0, atol=1e-5)
    assert ok, worst


@pytest.mark.parametrize("tag", ["a", "b"])
def test_adazero_vs_reference_golden(ops, tag):
    d = np.load(os.path.join(GOLD, "ops.npz"))
    x = from_bits(d[f"ada_{tag}_x"])
    tdt = torch.bfloat16 if bool(d[f"ada_{tag}_table_bf16"]) else torch.float32
    table = torch.from_numpy(d[f"ada_{tag}_table"]).to(tdt).cuda()
    ts = from_bits(d[f"ada_{tag}_ts"])
    sh, sc = (int(v) for v in d[f"ada_{tag}_idx"])
    y = ops.fused_adazero_from_ada(x, 1e-6, table, ts, shift_index=sh, scale_index=sc)
    ref = O.bf16_from_bits(d[f"ada_{tag}_y"])
    assert np.abs(to_np(y) - ref).max() <= 0.0625  # tests/test_triton_ltx_ops.py:92


def test_adazero_fused_quant_equals_separate_quant(ops):
    x, table, ts = _ada_case(37, 4096, torch.float32, torch.bfloat16, True, seed=5)
    x, table = x.cuda(), table.cuda()
    ts = ts[:, :1].cuda().expand(ts.shape)
    s = torch.tensor(0.0123, device="cuda")
    q, y = ops.fused_adazero_from_ada_fp8(x, 1e-6, table, ts, s, shift_index=0, scale_index=1, return_bf16=True)
    y2 = ops.fused_adazero_from_ada(x, 1e-6, table, ts, shift_index=0, scale_index=1)
    assert torch.equal(y, y2)
    assert np.array_equal(codes(q), codes(ops.fused_fp8_quantize_e4m3(y, s)))
    assert np.array_equal(codes(q), O.quantize_e4m3(to_np(y), 0.0123))
    q_only = ops.fused_adazero_from_ada_fp8(x, 1e-6, table, ts, s, shift_index=0, scale_index=1)
    assert np.array_equal(codes(q_only), codes(q))


@pytest.mark.parametrize("planes", [1, 2, 3])
@pytest.mark.parametrize("uniform", [True, False])
def test_adazero_fp8_planes_equal_one_call_per_scale(ops, planes, uniform):
    """The multi-scale AdaZero (one e4m3 copy per input scale, x read once) equals one fused AdaZero+quant
    call per scale, code for code, for token-uniform and per-token timesteps."""
    x, table, ts = _ada_case(300, 4096, torch.float32, torch.bfloat16, uniform, seed=17 + planes)
    x, table = x.cuda(), table.cuda()
    ts = ts[:, :1].cuda().expand(ts.shape) if uniform else ts.cuda()
    scales = torch.tensor([0.0123, 0.0071, 0.0302][:planes], device="cuda")
    q3 = ops.fused_adazero_from_ada_fp8_planes(x, 1e-6, table, ts, scales, shift_index=0, scale_index=1)
    assert q3.shape == (planes, *x.shape)
    for i in range(planes):
        qi = ops.fused_adazero_from_ada_fp8(x, 1e-6, table, ts, scales[i].clone(), shift_index=0, scale_index=1)
        assert np.array_equal(codes(q3[i]), codes(qi)), i
    assert status_clean()


@pytest.mark.parametrize("rows", [1157, 2307, 4609])
def test_adazero_rows_per_cta_widths_vs_oracle(ops, rows):
    """Row counts whose grids give each CTA 2, 4 and 8 rows (the host spreads short inputs over at least
    4 CTAs per SM), each with a ragged last CTA, with the fused quantiser on."""
    x, table, ts = _ada_case(rows, 4096, torch.float32, torch.bfloat16, True, seed=rows)
    s = torch.tensor(0.0123, device="cuda")
    q, y = ops.fused_adazero_from_ada_fp8(x.cuda(), 1e-6, table.cuda(), ts[:, :1].cuda().expand(ts.shape), s,
                                          shift_index=0, scale_index=1, return_bf16=True)
    ref = O.adazero_from_ada(x, 1e-6, table, ts.reshape(1, rows, 6, 4096), shift_index=0, scale_index=1,
                             table_is_bf16=False, ts_is_bf16=True)
    ok, worst = within_ulps(to_np(y), ref, ulps=1.0, atol=1e-5)
    assert ok, worst
    assert np.array_equal(codes(q), O.quantize_e4m3(to_np(y), 0.0123))


def test_bias_add_bitwise(ops):
    d = np.load(os.path.join(GOLD, "ops.npz"))
    out = ops.fused_bias_add_bf16(from_bits(d["bias_x"]), torch.from_numpy(d["bias_b"]).cuda())
    assert np.array_equal(bf16_bits(out), d["bias_y"])
    g = torch.Generator().manual_seed(1)
    x = torch.randn((33, 4096), generator=g).to(torch.bfloat16)
    b = torch.randn((4096,), generator=g).to(torch.bfloat16)
    out = ops.fused_bias_add_bf16(x.cuda(), b.cuda())
    assert np.array_equal(to_np(out), O.bias_add_bf16(x, b))


def test_residual_gate_bias_bitwise_vs_golden(ops):
    d = np.load(os.path.join(GOLD, "ops.npz"))
    out = ops.fused_residual_gate_bias_from_ada(
        from_bits(d["res_x"]), from_bits(d["res_y"]), torch.from_numpy(d["res_bias"]).cuda(),
        torch.from_numpy(d["res_table"]).cuda(), from_bits(d["res_ts"]), gate_index=8)
    assert np.array_equal(bf16_bits(out), d["res_out"])


@pytest.mark.parametrize("table_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ts_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("bias_dtype", [torch.float32, torch.bfloat16])
def test_residual_gate_bias_bitwise_vs_oracle(ops, table_dtype, ts_dtype, bias_dtype):
    x, table, ts = _ada_case(11, 4096, table_dtype, ts_dtype, False, seed=9)
    g = torch.Generator().manual_seed(10)
    y = torch.randn((1, 11, 4096), generator=g).to(torch.bfloat16)
    bias = torch.randn((4096,), generator=g).to(bias_dtype)
    out = ops.fused_residual_gate_bias_from_ada(x.cuda(), y.cuda(), bias.cuda(), table.cuda(), ts.cuda(), gate_index=2)
    ref = O.residual_gate_bias_from_ada(x, y, bias, table, ts.reshape(1, 11, 6, 4096), gate_index=2,
                                        table_is_bf16=table_dtype == torch.bfloat16, ts_is_bf16=ts_dtype == torch.bfloat16)
    assert np.array_equal(to_np(out), ref)


def _rope_case(tokens, seed, cs_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((1, tokens, 4096), generator=g).to(torch.bfloat16)
    k = torch.randn((1, tokens, 4096), generator=g).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn((4096,), generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn((4096,), generator=g)).to(torch.bfloat16)
    f = torch.randn((1, 32, tokens, 64), generator=g)
    return q, k, qw, kw, f.cos().to(cs_dtype), f.sin().to(cs_dtype)


@pytest.mark.parametrize("tokens", [1, 17, 300])
@pytest.mark.parametrize("cs_dtype", [torch.bfloat16, torch.float32])
def test_qk_rmsnorm_rope_vs_oracle(ops, tokens, cs_dtype):
    q, k, qw, kw, cos, sin = _rope_case(tokens, tokens, cs_dtype)
    oq, ok_ = ops.fused_video_qk_rmsnorm_rope(q.cuda(), k.cuda(), qw.cuda(), kw.cuda(), 1e-6, cos.cuda(), sin.cuda())
    for got, x, w in ((oq, q, qw), (ok_, k, kw)):
        ref = O.qk_rmsnorm_rope(x, w, 1e-6, cos, sin)
        ok, worst = within_ulps(to_np(got), ref, ulps=1.0, atol=1e-6)
        assert ok, worst


def test_qk_rmsnorm_rope_vs_reference_golden(ops):
    d = np.load(os.path.join(GOLD, "ops.npz"))
    x = from_bits(d["rope_x"])
    w = from_bits(d["rope_w"])
    out, _ = ops.fused_video_qk_rmsnorm_rope(x, x, w, w, 1e-6, from_bits(d["rope_cos"]), from_bits(d["rope_sin"]))
    assert np.abs(to_np(out) - O.bf16_from_bits(d["rope_out"])).max() <= 0.125  # tests/test_triton_ltx_ops.py:228


def test_qk_rmsnorm_rope_in_place_on_packed_rows(ops):
    q, k, qw, kw, cos, sin = _rope_case(40, 4)
    packed = torch.cat([q, k, torch.zeros_like(q)], dim=-1).cuda()  # [1, L, 3*4096]
    pq, pk = packed[..., :4096], packed[..., 4096:8192]
    ops.fused_video_qk_rmsnorm_rope(pq, pk, qw.cuda(), kw.cuda(), 1e-6, cos.cuda(), sin.cuda(), out=(pq, pk))
    assert np.array_equal(to_np(pq), to_np(ops.fused_video_qk_rmsnorm_rope(q.cuda(), k.cuda(), qw.cuda(), kw.cuda(),
                                                                          1e-6, cos.cuda(), sin.cuda())[0]))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_qkv_rope_scatter_layout(ops, world):
    """Sequence-to-head send layout [dst][L][3][H/P][128] written directly by the RoPE kernel."""
    from opengenie_b200 import _lib
    from opengenie_b200.ltx_ops import _stream

    q, k, qw, kw, cos, sin = _rope_case(24, 7)
    v = torch.randn((1, 24, 4096), generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    q, k, v, qw, kw, cos, sin = (t.cuda() for t in (q, k, v, qw, kw, cos, sin))
    hpg = 32 // world
    send = torch.empty((world, 24, 3, hpg, 128), device="cuda", dtype=torch.bfloat16)
    _lib.call("ogx_video_qkv_rmsnorm_rope_scatter", q.data_ptr(), k.data_ptr(), v.data_ptr(), 24, 4096,
              qw.data_ptr(), kw.data_ptr(), 0, 1e-6, cos.data_ptr(), sin.data_ptr(), 0, cos.stride(1), cos.stride(2),
              send[:, :, 0].data_ptr(), send[:, :, 1].data_ptr(), send[:, :, 2].data_ptr(),
              send.stride(1), send.stride(0), hpg, _stream(q))
    rq, rk = ops.fused_video_qk_rmsnorm_rope(q, k, qw, kw, 1e-6, cos, sin)
    for j, ref in enumerate((rq, rk, v)):
        got = send[:, :, j].permute(1, 0, 2, 3).reshape(1, 24, 4096)
        assert torch.equal(got, ref)
    assert status_clean()


@pytest.mark.parametrize("grid", [(2, 3, 5), (16, 18, 32), (3, 45, 40)])
def test_rope_tables_from_positions_vs_construction(ops, grid):
    """The cos/sin the kernels generate from (t, h, w) positions against the construction evaluated in float64
    on the CPU and rounded to bf16 (synthetic.rope_tables): within one bf16 ulp everywhere, equal almost
    everywhere (the hardware sin/cos after an exact reduction in turns are within ~4e-7 of the exact values, so
    only values that fall that close to a bf16 rounding boundary round the other way)."""
    from opengenie_b200 import synthetic

    pos = synthetic.rope_positions(*grid, device="cuda")
    cos, sin = ops.rope_tables_from_positions(pos)
    ref_c, ref_s = synthetic.rope_tables(*grid)
    for got, ref in ((cos, ref_c), (sin, ref_s)):
        g, r = to_np(got), to_np(ref)
        ok, worst = within_ulps(g, r, ulps=1.0, atol=2.0 ** -24)
        assert ok, worst
        assert (g != r).mean() < 2e-3, (g != r).mean()
    # a slice of tokens starting at token0 is the same slice of the whole table
    t0, n = pos.tokens // 3, pos.tokens // 2
    c2, s2 = ops.rope_tables_from_positions(pos, token0=t0, tokens=n)
    assert torch.equal(c2, cos[:, :, t0:t0 + n]) and torch.equal(s2, sin[:, :, t0:t0 + n])
    assert status_clean()


@pytest.mark.parametrize("tokens,token0", [(1, 0), (300, 0), (1152, 5000)])
@pytest.mark.parametrize("wdtype", [torch.bfloat16, torch.float32])
def test_qk_rmsnorm_rope_positions_equals_table_kernel(ops, tokens, token0, wdtype):
    """Generated cos/sin: bit for bit the table kernel given the tables of the same values, for any slice of
    the raster and both weight dtypes; and within one ulp of the float64 oracle on those tables."""
    from opengenie_b200 import synthetic

    pos = synthetic.rope_positions(16, 18, 32, device="cuda")
    q, k, qw, kw, _, _ = _rope_case(tokens, tokens + 3)
    q, k = q.cuda(), k.cuda()
    qw, kw = qw.to(wdtype).cuda(), kw.to(wdtype).cuda()
    cos, sin = ops.rope_tables_from_positions(pos, token0=token0, tokens=tokens)
    tq, tk = ops.fused_video_qk_rmsnorm_rope(q, k, qw, kw, 1e-6, cos, sin)
    gq, gk = ops.fused_video_qk_rmsnorm_rope_positions(q, k, qw, kw, 1e-6, pos, token0=token0)
    assert torch.equal(gq, tq) and torch.equal(gk, tk)
    if tokens <= 300:
        for got, x, w in ((gq, q, qw), (gk, k, kw)):
            ref = O.qk_rmsnorm_rope(x.cpu(), w.float().cpu(), 1e-6, cos.cpu(), sin.cpu())
            ok, worst = within_ulps(to_np(got), ref, ulps=1.0, atol=1e-6)
            assert ok, worst
    with pytest.raises(ValueError, match="rope_shape"):
        ops.fused_video_qk_rmsnorm_rope_positions(q, k, qw, kw, 1e-6, pos, token0=pos.tokens - tokens + 1)
    assert status_clean()


@pytest.mark.parametrize("world", [2, 8])
def test_qkv_rope_positions_scatter_layout(ops, world):
    """The send layout of the sequence-to-head exchange written with generated cos/sin equals the one written
    from the tables of the same values."""
    from opengenie_b200 import _lib, synthetic
    from opengenie_b200.ltx_ops import _stream

    L, t0 = 24, 40
    pos = synthetic.rope_positions(2, 8, 16, device="cuda")
    q, k, qw, kw, _, _ = _rope_case(L, 11)
    v = torch.randn((1, L, 4096), generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    q, k, v, qw, kw = (t.cuda() for t in (q, k, v, qw, kw))
    cos, sin = ops.rope_tables_from_positions(pos, token0=t0, tokens=L)
    hpg = 32 // world
    sends = []
    for gen in (False, True):
        send = torch.empty((world, L, 3, hpg, 128), device="cuda", dtype=torch.bfloat16)
        rope = ((pos.inv_freq.data_ptr(), pos.slot_axis.data_ptr(), pos.grid_h, pos.grid_w, t0) if gen else
                (cos.data_ptr(), sin.data_ptr(), 0, cos.stride(1), cos.stride(2)))
        _lib.call("ogx_video_qkv_rmsnorm_rope_positions_scatter" if gen else "ogx_video_qkv_rmsnorm_rope_scatter",
                  q.data_ptr(), k.data_ptr(), v.data_ptr(), L, 4096, qw.data_ptr(), kw.data_ptr(), 0, 1e-6, *rope,
                  send[:, :, 0].data_ptr(), send[:, :, 1].data_ptr(), send[:, :, 2].data_ptr(),
                  send.stride(1), send.stride(0), hpg, _stream(q))
        sends.append(send)
    assert torch.equal(sends[0], sends[1])
    assert status_clean()


def test_qkv_rmsnorm_rope_pack_layout(ops):
    """fused_video_qkv_rmsnorm_rope_pack: [1, L, 3, 32, 128] holding the roped q and k and the untouched v,
    bit for bit the separate op's q/k."""
    q, k, qw, kw, cos, sin = _rope_case(37, 9)
    v = torch.randn((1, 37, 4096), generator=torch.Generator().manual_seed(10)).to(torch.bfloat16)
    q, k, v, qw, kw, cos, sin = (t.cuda() for t in (q, k, v, qw, kw, cos, sin))
    qkv = ops.fused_video_qkv_rmsnorm_rope_pack(q, k, v, qw, kw, 1e-6, cos, sin)
    assert qkv.shape == (1, 37, 3, 32, 128)
    rq, rk = ops.fused_video_qk_rmsnorm_rope(q, k, qw, kw, 1e-6, cos, sin)
    for j, ref in enumerate((rq, rk, v)):
        assert torch.equal(qkv[:, :, j].reshape(1, 37, 4096), ref)
    with pytest.raises(ValueError, match="qkv_shape"):
        ops.fused_video_qkv_rmsnorm_rope_pack(q, k, v[:, :36], qw, kw, 1e-6, cos, sin)
    assert status_clean()


def test_residual_gate_without_bias_bitwise_vs_golden(ops):
    d = np.load(os.path.join(GOLD, "residual_nobias.npz"))
    out = ops.fused_residual_gate_from_ada(from_bits(d["x"]), from_bits(d["y"]), torch.from_numpy(d["table"]).cuda(),
                                           from_bits(d["ts"]), gate_index=8)
    assert np.array_equal(bf16_bits(out).reshape(-1), d["out"].reshape(-1))
    assert status_clean()


@pytest.mark.parametrize("tag", ["a", "b"])
def test_adaln_affine_bitwise_vs_golden(ops, tag):
    d = np.load(os.path.join(GOLD, "adaln_affine.npz"))
    table = torch.from_numpy(d[f"{tag}_table"])
    if bool(d[f"{tag}_table_bf16"]):
        table = table.to(torch.bfloat16)
    sh, sc = (int(i) for i in d[f"{tag}_idx"])
    out = ops.fused_adaln_affine_from_ada(from_bits(d[f"{tag}_x"]), table.cuda(), from_bits(d[f"{tag}_ts"]),
                                          shift_index=sh, scale_index=sc)
    assert np.array_equal(bf16_bits(out), d[f"{tag}_y"])
    assert status_clean()


@pytest.mark.parametrize("table_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ts_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("uniform", [False, True])
def test_adaln_affine_bitwise_vs_oracle(ops, table_dtype, ts_dtype, uniform):
    x, table, ts = _ada_case(13, 4096, table_dtype, ts_dtype, uniform, seed=21)
    out = ops.fused_adaln_affine_from_ada(x.cuda(), table.cuda(), ts.cuda() if not uniform else
                                          ts[:, :1].cuda().expand(ts.shape), shift_index=6 % table.shape[0],
                                          scale_index=1)
    ref = O.adaln_affine_from_ada(x, table, ts.reshape(1, 13, table.shape[0], 4096), shift_index=6 % table.shape[0],
                                  scale_index=1, table_is_bf16=table_dtype == torch.bfloat16,
                                  ts_is_bf16=ts_dtype == torch.bfloat16)
    assert np.array_equal(to_np(out), ref)


def test_head_gate_mul_bitwise_vs_golden(ops):
    d = np.load(os.path.join(GOLD, "head_gate.npz"))
    y = ops.fused_head_gate_mul_bf16(from_bits(d["out"]), from_bits(d["gates"]), 32, 128)
    assert np.array_equal(bf16_bits(y), d["y"])
    g = torch.Generator().manual_seed(3)
    out = torch.randn((1, 300, 16 * 64), generator=g).to(torch.bfloat16)
    gates = torch.rand((1, 300, 16), generator=g).to(torch.bfloat16)
    y2 = ops.fused_head_gate_mul_bf16(out.cuda(), gates.cuda(), 16, 64)
    assert np.array_equal(to_np(y2), O.head_gate_mul_bf16(out, gates, 16, 64))
    assert status_clean()


def test_mul_from_ada_and_residual_gate_bf16_bitwise_vs_golden(ops):
    d = np.load(os.path.join(GOLD, "ada_misc.npz"))
    y = ops.fused_mul_from_ada(from_bits(d["mul_x"]), torch.from_numpy(d["mul_table"]).cuda(), from_bits(d["mul_ts"]),
                               gate_index=4)
    assert np.array_equal(bf16_bits(y), d["mul_y"])
    x, yy = from_bits(d["res_x"]), from_bits(d["res_y"])
    for tag in ("tok", "sample"):
        out = ops.fused_residual_gate_bf16(x, yy, from_bits(d[f"res_gate_{tag}"]))
        assert np.array_equal(bf16_bits(out), d[f"res_out_{tag}"])
    assert status_clean()


def test_explicit_value_ops_take_noncontiguous_rows(ops):
    """The reference's strided-input cases (tests/test_triton_ltx_ops.py:8-47): scale/shift and gate as slices
    of a [1, rows, 3, cols] tensor (token stride 3*cols).  AdaZero within one ulp of the one-rounding oracle;
    the gated residual bit-equal to torch's ``x + y * gate``, as the reference asserts."""
    g = torch.Generator().manual_seed(0)
    rows, cols = 7, 2048
    x = torch.randn((1, rows, cols), generator=g).to(torch.bfloat16)
    scale_shift = torch.randn((1, rows, 3, cols), generator=g).to(torch.bfloat16).cuda()
    scale, shift = scale_shift[:, :, 1, :], scale_shift[:, :, 2, :]
    assert not scale.is_contiguous() and scale.stride(1) == 3 * cols
    out = ops.fused_adazero(x.cuda(), 1e-6, scale, shift)
    ok, worst = within_ulps(to_np(out), O.adazero_explicit(x, 1e-6, scale.float().cpu(), shift.float().cpu()),
                            ulps=1.0, atol=1e-5)
    assert ok, worst
    xr = torch.randn((1, rows, cols), generator=g).to(torch.bfloat16).cuda()
    y = torch.randn((1, rows, cols), generator=g).to(torch.bfloat16).cuda()
    gate = scale_shift[:, :, 1, :]
    out = ops.fused_residual_gate_bf16(xr, y, gate)
    assert torch.equal(out, xr + y * gate)
    assert status_clean()


@pytest.mark.parametrize("rows", ["one", "sample", "token"])
def test_adazero_explicit_vs_oracle(ops, rows):
    """``fused_adazero`` with explicit scale/shift of 1, batch or batch*tokens rows: within one bf16 ulp of the
    one-rounding oracle, and within 0.0625 of the reference's torch path on its golden."""
    g = torch.Generator().manual_seed(17)
    x = torch.randn((2, 9, 4096), generator=g).to(torch.bfloat16)
    shape = {"one": (1, 1, 4096), "sample": (2, 1, 4096), "token": (2, 9, 4096)}[rows]
    scale = (torch.randn(shape, generator=g) * 0.3).to(torch.bfloat16)
    shift = torch.randn(shape, generator=g) * 0.3  # fp32 shift with a bf16 scale
    out = ops.fused_adazero(x.cuda(), 1e-6, scale.cuda(), shift.cuda())
    ref = O.adazero_explicit(x, 1e-6, scale.float(), shift)
    ok, worst = within_ulps(to_np(out), ref, ulps=1.0, atol=1e-5)
    assert ok, worst
    d = np.load(os.path.join(GOLD, "ada_misc.npz"))
    got = ops.fused_adazero(from_bits(d["ada_x"]), 1e-6, from_bits(d["ada_scale"]), from_bits(d["ada_shift"]))
    assert np.abs(to_np(got) - O.bf16_from_bits(d["ada_y"])).max() <= 0.0625
    assert status_clean()
