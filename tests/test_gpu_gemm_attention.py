"""GPU parity of the tensor-core stages: the tcgen05 FP8 GEMM (bias and residual epilogues) and the
tcgen05 attention, against the float64 oracle on small/ragged shapes and against torch's own GPU
kernels (cuBLAS scaled-mm, SDPA) at the full configuration sizes."""

import numpy as np
import pytest
import torch

from gpu_util import O, accum_atol, bf16_ulp, block_tolerance, codes, status_clean, to_np, within_ulps

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(ogx_lib):
    from opengenie_b200 import ltx_ops

    return ltx_ops


def _fp8_case(M, N, K, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn((M, K), generator=g)
    if outliers and M * K:
        idx = torch.randperm(M * K, generator=g)[: max(1, M * K // 1000)]
        a.view(-1)[idx] *= 50
    ab = a.to(torch.bfloat16)
    s_a = float(ab.float().abs().amax() / 448.0)
    aq = torch.from_numpy(O.quantize_e4m3(ab.float().numpy(), s_a)).view(torch.float8_e4m3fn)
    w = torch.randn((N, K), generator=g) * 0.02
    s_w = float(w.abs().amax() / 448.0)
    wq = torch.clamp(w / s_w, -448, 448).to(torch.float8_e4m3fn)
    bias = (torch.randn((N,), generator=g) * 0.01).to(torch.bfloat16)
    return aq, s_a, wq, s_w, bias


def _accum_atol(aq, s_a, wq, s_w):
    return accum_atol(codes(aq), s_a, codes(wq), s_w)


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (17, 256, 4096), (300, 512, 4096), (256, 4096, 1024), (1, 32, 16),
                                   (3600, 512, 4096)])
def test_fp8_gemm_bias_vs_oracle(ops, M, N, K):
    """(3600, ...): the per-GPU row count of the 720p-class window (L = 28800) over 8 GPUs, whose last row
    tile is ragged (3600 = 14 * 256 + 16)."""
    aq, s_a, wq, s_w, bias = _fp8_case(M, N, K, seed=M * 7 + N)
    out = ops.fp8_scaled_mm(aq.cuda(), wq.cuda(), torch.tensor(s_a, device="cuda"), torch.tensor([s_w], device="cuda"),
                            bias=bias.cuda())
    ref = O.fp8_linear(codes(aq), s_a, codes(wq), s_w, bias)
    pre_bias = O.fp8_linear(codes(aq), s_a, codes(wq), s_w)
    ok, worst = within_ulps(to_np(out), ref, ulps=1.0, atol=_accum_atol(aq, s_a, wq, s_w) + bf16_ulp(pre_bias))
    assert ok, worst
    assert status_clean()


def test_fp8_gemm_packed_qkv_segment_scales(ops):
    aq, s_a, wq, _, bias = _fp8_case(130, 3 * 512, 512, seed=3)
    seg_scales = [0.01, 0.002, 0.05]
    out = ops.fp8_scaled_mm(aq.cuda(), wq.cuda(), torch.tensor(s_a, device="cuda"),
                            torch.tensor(seg_scales, device="cuda"), bias=bias.cuda())
    ref = O.fp8_linear(codes(aq), s_a, codes(wq), np.array(seg_scales, np.float32), bias)
    pre_bias = O.fp8_linear(codes(aq), s_a, codes(wq), np.array(seg_scales, np.float32))
    ok, worst = within_ulps(to_np(out), ref, ulps=1.0,
                            atol=_accum_atol(aq, s_a, wq, np.array(seg_scales)) + bf16_ulp(pre_bias))
    assert ok, worst


def test_fp8_gemm_strided_output_columns(ops):
    aq, s_a, wq, s_w, bias = _fp8_case(64, 256, 256, seed=4)
    big = torch.zeros((64, 3 * 256), device="cuda", dtype=torch.bfloat16)
    ops.fp8_scaled_mm(aq.cuda(), wq.cuda(), torch.tensor(s_a, device="cuda"), torch.tensor([s_w], device="cuda"),
                      bias=bias.cuda(), out=big[:, 256:512])
    ref = ops.fp8_scaled_mm(aq.cuda(), wq.cuda(), torch.tensor(s_a, device="cuda"), torch.tensor([s_w], device="cuda"),
                            bias=bias.cuda())
    assert torch.equal(big[:, 256:512], ref)
    assert (big[:, :256] == 0).all() and (big[:, 512:] == 0).all()


@pytest.mark.parametrize("M,K", [(300, 4096), (1152, 1024), (9216, 4096)])
def test_fp8_gemm_planes_equal_one_gemm_per_plane(ops, M, K):
    """The packed Q/K/V GEMM over three activation planes (one e4m3 copy per linear, each with its own
    input scale) equals three GEMMs, one per plane and weight segment, bit for bit."""
    g = torch.Generator(device="cuda").manual_seed(M + K)
    N = 3 * 4096
    a3 = (torch.randn((3, M, K), device="cuda", generator=g) * 40).to(torch.float8_e4m3fn)
    w = (torch.randn((N, K), device="cuda", generator=g) * 40).to(torch.float8_e4m3fn)
    s_a = torch.tensor([0.011, 0.017, 0.0053], device="cuda")
    s_b = torch.tensor([0.0021, 0.0013, 0.0034], device="cuda")
    bias = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    out = ops.fp8_scaled_mm_planes(a3, w, s_a, s_b, bias=bias)
    for i in range(3):
        seg = slice(i * 4096, (i + 1) * 4096)
        ref = ops.fp8_scaled_mm(a3[i], w[seg], s_a[i].clone(), s_b[i].clone().reshape(1), bias=bias[seg])
        assert torch.equal(out[:, seg], ref), i
    assert status_clean()


@pytest.mark.parametrize("N", [12288, 16384])
def test_fp8_gemm_full_size_vs_cublas(ops, N):
    """C3: M=9216, K=4096, N in {12288, 16384} against torch._scaled_mm (cuBLASLt) on the same GPU."""
    M, K = 9216, 4096
    g = torch.Generator(device="cuda").manual_seed(N)
    a = torch.randn((M, K), device="cuda", generator=g)
    a.view(-1)[torch.randint(0, M * K, (M * K // 1000,), device="cuda", generator=g)] *= 50
    ab = a.to(torch.bfloat16)
    s_a = (ab.float().abs().amax() / 448.0).reshape(())
    aq = ops.fused_fp8_quantize_e4m3(ab, s_a)
    w = torch.randn((N, K), device="cuda", generator=g) * 0.02
    s_w = (w.abs().amax() / 448.0).reshape(())
    wq = torch.clamp(w / s_w, -448, 448).to(torch.float8_e4m3fn)
    bias = (torch.randn((N,), device="cuda", generator=g) * 0.01).to(torch.bfloat16)
    ours = ops.fp8_scaled_mm(aq, wq, s_a, s_w.reshape(1), bias=bias)
    ref = torch._scaled_mm(aq, wq.t(), scale_a=s_a, scale_b=s_w, out_dtype=torch.bfloat16, use_fast_accum=True)
    ref = (ref.float() + bias.float()).to(torch.bfloat16)
    d = (ours.float() - ref.float()).abs()
    ulp = torch.exp2(torch.floor(torch.log2(ref.float().abs().clamp_min(2.0 ** -126))) - 7)
    assert (d <= 2 * ulp + 1e-4).float().mean().item() >= 0.9999
    assert (d.sum() / ref.float().abs().sum()).item() < 1e-3
    assert status_clean()


def test_fp8_gemm_residual_epilogue_vs_oracle(ops):
    M, N, K = 40, 4096, 512
    aq, s_a, wq, s_w, bias = _fp8_case(M, N, K, seed=11)
    g = torch.Generator().manual_seed(12)
    x = torch.randn((1, M, N), generator=g).to(torch.bfloat16)
    table = torch.randn((6, N), generator=g) * 0.02
    ts = torch.randn((6 * N,), generator=g).to(torch.bfloat16).view(1, 1, -1).expand(1, M, 6 * N)
    out = ops.fp8_scaled_mm_residual_gate(aq.cuda().view(1, M, K), wq.cuda(), torch.tensor(s_a, device="cuda"),
                                          torch.tensor(s_w, device="cuda"), bias.cuda(), x.cuda(), table.cuda(),
                                          ts[:, :1].cuda().expand(ts.shape), gate_index=2)
    y = O.fp8_linear(codes(aq), s_a, codes(wq), s_w)
    ref = O.residual_gate_bias_from_ada(x, y, bias, table, ts.reshape(1, M, 6, N), gate_index=2)
    # y may differ by one bf16 ulp (accumulation order), which the gate/residual roundings keep within 2 ulps
    gate = np.abs(O.ada_value(table, ts.reshape(1, M, 6, N), 2, table_is_bf16=False, ts_is_bf16=True))
    ok, worst = within_ulps(to_np(out), ref, ulps=2.0, atol=(_accum_atol(aq, s_a, wq, s_w) * gate[0] + 1e-6))
    assert ok, worst


@pytest.mark.parametrize("M,blocks", [(4608, 2), (1152, 8), (300, 4), (3600, 8)])
def test_fp8_gemm_residual_kblocked_equals_plain(ops, M, blocks):
    """The out-projection reading A as `blocks` column blocks [blocks][M][K/blocks] (the Ulysses receive
    buffer, through a 3-D tensor map) equals the same GEMM on the assembled [M, K] operand, bit for bit,
    for shapes that run as CTA pairs (M = 4608) and as single CTAs."""
    from opengenie_b200 import _lib, ltx_ops

    K, N = 4096, 4096
    kb = K // blocks
    g = torch.Generator(device="cuda").manual_seed(M + blocks)
    a = (torch.randn((M, K), device="cuda", generator=g) * 64).clamp(-448, 448).to(torch.float8_e4m3fn)
    w = (torch.randn((N, K), device="cuda", generator=g) * 64).clamp(-448, 448).to(torch.float8_e4m3fn)
    sa, sw = torch.tensor(2e-4, device="cuda"), torch.tensor(1e-3, device="cuda")
    bias = (torch.randn((N,), device="cuda", generator=g) * 0.01).to(torch.bfloat16)
    x = torch.randn((1, M, N), device="cuda", generator=g).to(torch.bfloat16)
    table = torch.randn((6, N), device="cuda", generator=g) * 0.02
    ts = torch.randn((1, 1, 6 * N), device="cuda", generator=g).to(torch.bfloat16).expand(1, M, 6 * N)
    plain = ops.fp8_scaled_mm_residual_gate(a.view(1, M, K), w, sa, sw, bias, x, table, ts, gate_index=2)
    a_blocked = a.view(M, blocks, kb).transpose(0, 1).contiguous()  # [blocks][M][kb]
    ts_view = ltx_ops._ts_view(x, table, ts)
    out = torch.empty_like(x)
    _lib.call(
        "ogx_fp8_scaled_mm_residual_gate_kblocked",
        a_blocked.data_ptr(), M, K, kb, w.data_ptr(), N, w.stride(0), sa.data_ptr(), sw.data_ptr(), N,
        bias.data_ptr(), ltx_ops._code(bias), x.data_ptr(), x.stride(1), table.data_ptr(), ltx_ops._code(table),
        table.stride(0), ts_view.data_ptr(), ltx_ops._code(ts_view), ts_view.stride(1), ts_view.stride(2), 2,
        out.data_ptr(), out.stride(1), ltx_ops._stream(x),
    )
    assert torch.equal(out, plain)
    assert status_clean()


def _qkv(B, L, H, seed, packed=False):
    g = torch.Generator().manual_seed(seed)
    if packed:
        qkv = torch.randn((B, L, 3 * H * 128), generator=g).to(torch.bfloat16)
        return qkv, None, None
    q = torch.randn((B, L, H * 128), generator=g).to(torch.bfloat16)
    k = torch.randn((B, L, H * 128), generator=g).to(torch.bfloat16)
    v = torch.randn((B, L, H * 128), generator=g).to(torch.bfloat16)
    return q, k, v


@pytest.mark.parametrize("B,L,H", [(1, 128, 1), (1, 256, 2), (1, 17, 2), (1, 300, 3), (2, 384, 2), (1, 1000, 1)])
def test_attention_vs_oracle(ops, B, L, H):
    q, k, v = _qkv(B, L, H, seed=L + H)
    out = ops.attention(q.cuda(), k.cuda(), v.cuda(), H)
    ref = O.attention(q, k, v, H)
    tol = block_tolerance(to_np(out), ref)
    assert tol["ok"], tol
    assert status_clean()


def test_attention_peaked_scores_rescale_path(ops):
    """Scores spread over > 2^8 in log2 units so the running-max rescale of O is exercised."""
    q, k, v = _qkv(1, 512, 1, seed=99)
    q = (q.float() * 6).to(torch.bfloat16)
    k[:, 300:] = (k[:, 300:].float() * 3).to(torch.bfloat16)
    out = ops.attention(q.cuda(), k.cuda(), v.cuda(), 1)
    tol = block_tolerance(to_np(out), O.attention(q, k, v, 1))
    assert tol["ok"], tol


def test_attention_packed_rows_and_e4m3_epilogue(ops):
    qkv, _, _ = _qkv(1, 256, 2, seed=5, packed=True)
    qkv = qkv.cuda()
    D = 256
    q, k, v = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
    out = ops.attention(q, k, v, 2)
    ref = O.attention(q.cpu(), k.cpu(), v.cpu(), 2)
    assert block_tolerance(to_np(out), ref)["ok"]
    s = torch.tensor(0.005, device="cuda")
    oq = ops.attention(q, k, v, 2, out_e4m3_scale=s)
    assert np.array_equal(codes(oq), codes(ops.fused_fp8_quantize_e4m3(out, s)))


@pytest.mark.parametrize("L", [2304, 9216, 28800])
def test_attention_full_size_vs_torch_sdpa(ops, L):
    """Full configuration sizes against torch SDPA on the same GPU (fp32 math per head), within the north-star
    bound as stated: max|d| <= 2e-2 and sum|d|/sum|ref| <= 1e-2.  L = 28800 (the 720p-class window) ends in
    a ragged query block: 28800 = 112 * 256 + 128, so the last CTA's second 128-query tile is all padding."""
    H = 32
    g = torch.Generator(device="cuda").manual_seed(L)
    q, k, v = (torch.randn((1, L, H * 128), device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    out = ops.attention(q, k, v, H)
    qh, kh, vh = (t.view(1, L, H, 128).transpose(1, 2) for t in (q, k, v))
    worst_max, num, den = 0.0, 0.0, 0.0
    for h in range(0, H, 4):
        ref = torch.nn.functional.scaled_dot_product_attention(qh[:, h:h + 4].float(), kh[:, h:h + 4].float(),
                                                               vh[:, h:h + 4].float())
        got = out.view(1, L, H, 128).transpose(1, 2)[:, h:h + 4].float()
        d = (got - ref).abs()
        worst_max = max(worst_max, d.max().item())
        num += d.sum().item()
        den += ref.abs().sum().item()
    assert worst_max <= 2e-2
    assert num / den <= 1e-2
    assert status_clean()


@pytest.mark.parametrize("mode", ["1", "2"])
def test_attention_cta_pair_kernel_same_cases(mode):
    """The CTA-pair attention kernel (selected with OGX_ATTN_PAIRS=1, or 2 for its split score MMAs; read
    once per process) passes the same attention cases as the default kernel: oracle shapes, the rescale
    path, the e4m3 epilogue and the full sizes.  Runs them in a child pytest with the variable set."""
    import os
    import subprocess
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, OGX_ATTN_PAIRS=mode)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(here, "test_gpu_gemm_attention.py"), "-k", "attention and not cta_pair"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "failed" not in r.stdout
