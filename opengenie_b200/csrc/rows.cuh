// Row-pipeline kernels for the HBM-bound stages that normalise whole 4096-column rows: AdaZero (+ the
// E4M3 quantiser) and the Q/K RMSNorm + split RoPE (+ the sequence-to-head scatter).
//
// A row's RMS needs every column before any output can be written, so a kernel that holds the row in
// registers keeps few rows in flight per SM and leaves HBM idle between a row's load and its reduction.
// Here one persistent CTA per SM streams its rows through a ring of shared-memory stages instead:
//   the last warp (one thread)   issues cp.async.bulk copies of whole rows (8 KB per 4096-column bf16
//                                row) into the ring, a row as soon as its stage is free;
//   warps 0..W-1                 each take every W-th row of the CTA (W = the kernel's consumer warps,
//                                or the stage count where fewer stages fit): wait for its stage, reduce
//                                the sum of squares from shared memory (warp shuffles, no block
//                                barrier), write the outputs with 16-byte stores, free the stage.
// The stage count is a multiple of W, so a stage is always consumed by the same warp (see ring_warps).
// With 7-24 stages (up to ~190 KB) a SM keeps enough row loads in flight for the HBM latency; no
// register holds a row.  Every wait is bounded (a wait that runs out records OGX_ERR_TIMEOUT, the
// CTA stops and lets its copies in flight land before it exits).
//
// The split-RoPE cos/sin are either read from [heads, tokens, 64] tables (the reference's interface,
// fused_video_qk_rmsnorm_rope, ltx_serve/triton_ltx_ops.py:320-378) or generated here from each token's
// (t, h, w) latent position and a per-slot inverse frequency: angle = position[axis(slot)] * inv_freq(slot),
// reduced exactly in turns (double-single frequency, exact product for positions below 256), sin/cos by
// quadrant and Taylor series, and one rounding to bf16, the precision of the reference's tables.  That removes the
// tables' 2 x 2 B x 2048 per token of HBM reads; a kernel writing the same values as tables
// (rope_tables_kernel) lets tests compare both paths bit for bit.
#pragma once

#include "ogx_sm100.cuh"
#include "elementwise.cuh"

namespace ogx {
namespace rows {

// Consumer warps per CTA (at most; never more than the ring has stages): 10 for the RoPE kernel, whose
// ring holds 10 Q+K stages, and 16 for AdaZero and the RMSNorm-only kernel.  A row's work is a long chain
// of dependent shared-memory loads and packed arithmetic, so the more warps per SM sub-partition, the more
// of the issue slots are used.
constexpr int kConsumerWarps = 8;
constexpr int kRopeWarps = 10;
constexpr int kWideWarps = 16;
__host__ __device__ constexpr int ring_threads(int consumer_warps) { return (consumer_warps + 1) * 32; }
constexpr int kRopeThreads = ring_threads(kRopeWarps);
constexpr int kWideThreads = ring_threads(kWideWarps);
// Shared memory per CTA on sm_100 is at most 232448 bytes; 1 KB stays for the static ring state and the
// 128-byte alignment of the dynamic part.
constexpr int kDynLimit = 232448 - 1024;

// cp.async.bulk global -> shared: both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

constexpr int kMaxStages = 24;

struct Ring {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  int abort;
};

// Consumer warps and ring stages a kernel uses out of `stages` that fit: as many warps as stages (at most
// the kernel's consumer warps, cw) and the stages rounded down to a multiple of that, so row k goes to
// stage k % S and to warp k % W with W dividing S: each stage is always consumed by the same warp.  A
// parity wait cannot tell the phase it waits for from the one before it, so a warp reaching a stage one
// use ahead of the stage's other consumer would take the previous fill for its own; with one consumer per
// stage that cannot happen.
__host__ __device__ constexpr int ring_warps(int stages, int cw = kConsumerWarps) { return stages < cw ? stages : cw; }
__host__ __device__ constexpr int ring_stages(int stages, int cw = kConsumerWarps) {
  return stages / ring_warps(stages, cw) * ring_warps(stages, cw);
}

__device__ __forceinline__ void ring_init(Ring& r, int stages) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&r.full[s], 1);
      mbar_init(&r.empty[s], 1);
    }
    r.abort = 0;
    fence_mbar_init();
  }
}

// The producer thread: for row k of the CTA (k in [0, n)), waits for stage k % S to be free, announces
// `bytes` on the stage's full barrier and calls `issue(k, stage_ptr, bar)`, which must copy exactly that
// many bytes into the stage with completion counted on `bar`.
template <typename Issue>
__device__ __forceinline__ void ring_produce(Ring& r, uint8_t* ring, int stages, uint32_t stage_bytes, int n,
                                             uint32_t bytes, Issue issue) {
  volatile int* abort = &r.abort;
  int k = 0;
  for (; k < n; ++k) {
    const int s = k % stages;
    const uint32_t ph = (k / stages) & 1;
    if (!mbar_wait(&r.empty[s], ph ^ 1u, abort)) break;
    mbar_arrive_expect_tx(&r.full[s], bytes);
    issue(k, ring + static_cast<size_t>(s) * stage_bytes, &r.full[s]);
  }
  if (k < n) {
    // stopped early: let the copies already issued land before the CTA exits
    for (int j = k - 1; j >= 0 && j > k - 1 - stages; --j) mbar_wait(&r.full[j % stages], (j / stages) & 1, nullptr);
  }
}

// The two bf16 values of a packed word as fp32 (low half first).
__device__ __forceinline__ f2 bf16x2_to_f2(uint32_t w) { return f2{__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u)}; }

// Sum of squares of the 8 bf16 values of a 16-byte vector into two packed accumulators.
__device__ __forceinline__ void sumsq8(const uint4& v, f2& a, f2& b) {
  const f2 p0 = bf16x2_to_f2(v.x), p1 = bf16x2_to_f2(v.y), p2 = bf16x2_to_f2(v.z), p3 = bf16x2_to_f2(v.w);
  a = fma2(p0, p0, a);
  b = fma2(p1, p1, b);
  a = fma2(p2, p2, a);
  b = fma2(p3, p3, b);
}

// The reference's torch-path quantiser (triton_ltx_ops.py:146-148) of two bf16-valued floats: t = bf16(y * r)
// by a packed RNE conversion, then the saturating e4m3 conversion, which also performs the clamp to +-448
// (finite values past 448 and infinities saturate, as clamp then cast does).  NaN comes out as an e4m3 NaN
// code (low 7 bits 0x7F) and is patched to 0xFF per byte by the caller (torch's bf16 path, bf16 NaN -> 0xFF).
__device__ __forceinline__ uint32_t quant2_torch(f2 yb, f2 r2) {
  const f2 t = mul2(yb, r2);
  const f2 tb = bf16x2_to_f2(pack_bf16x2(t.x, t.y));
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(tb.x, tb.y), __NV_SATFINITE, __NV_E4M3)) & 0xFFFFu;
}

// Every byte of w whose low 7 bits are all ones (an e4m3 NaN code) becomes 0xFF.
__device__ __forceinline__ uint32_t nan_bytes_to_ff(uint32_t w) {
  const uint32_t hit = ((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u;
  return w | (hit - (hit >> 7)) | hit;
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Rows [r0, r1) of `rows` for this CTA (contiguous, balanced to within one row).
__device__ __forceinline__ void cta_rows(int64_t rows, int64_t& r0, int64_t& r1) {
  r0 = rows * blockIdx.x / gridDim.x;
  r1 = rows * (blockIdx.x + 1) / gridDim.x;
}

// ----------------------------------------------------------------------------------------------- AdaZero
// y = rmsnorm(x) * (1 + scale) + shift with shift/scale = table + timestep slot (ada_values8's rounding),
// fp32 math and one bf16 rounding (the reference's GPU kernel, triton_ltx_ops.py:3359-3427), optionally
// quantised to e4m3 from the bf16 value.  Shared memory: the Ada values of this CTA's columns (token-uniform
// timestep: computed once; per-token timestep: the table part, plus the token's two timestep slot rows
// copied into each stage with its x row), then the ring.
template <int COLS, typename TsT>
struct AdaLayout {
  static constexpr int kAda = 2 * COLS * 4;  // fp32 per column: shift and 1 + scale (uniform) or the table parts
  static constexpr int kStageUniform = COLS * 2;
  static constexpr int kStagePerToken = COLS * 2 + 2 * COLS * static_cast<int>(sizeof(TsT));
  __host__ __device__ static constexpr int stage_bytes(bool uniform) { return uniform ? kStageUniform : kStagePerToken; }
  __host__ __device__ static constexpr int stages(bool uniform) {
    return ring_stages(((kDynLimit - kAda) / stage_bytes(uniform)) > kMaxStages ? kMaxStages
                                                                                 : ((kDynLimit - kAda) / stage_bytes(uniform)),
                       kWideWarps);
  }
  __host__ __device__ static constexpr int smem_bytes(bool uniform) { return kAda + stages(uniform) * stage_bytes(uniform); }
};

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]);
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(p) = pack8(f);
}
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&f)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

template <int COLS, typename TableT, typename TsT, bool QUANT, int QMODE, bool UNIFORM>
__global__ void __launch_bounds__(kWideThreads, 1) adazero_ring_kernel(AdaArgs a) {
  pdl_trigger();
  using Lay = AdaLayout<COLS, TsT>;
  constexpr int S = Lay::stages(UNIFORM);  // a multiple of W
  constexpr int W = ring_warps(S, kWideWarps);
  constexpr uint32_t SB = Lay::stage_bytes(UNIFORM);
  constexpr int VPL = COLS / 8 / 32;  // 16-byte vectors per lane
  extern __shared__ uint8_t smem_raw[];
  __shared__ Ring ring;
  uint8_t* smem = smem_raw + (((smem_u32(smem_raw) + 127u) & ~127u) - smem_u32(smem_raw));
  // uniform timestep: ada0 = shift, ada1 = 1 + scale; per-token timestep: ada0 / ada1 = the table parts of
  // shift / scale (rounded to the timestep's dtype when the dtypes differ)
  float* ada0 = reinterpret_cast<float*>(smem);
  float* ada1 = ada0 + COLS;
  uint8_t* stages = smem + Lay::kAda;
  ring_init(ring, S);
  int64_t r0, r1;
  cta_rows(a.rows, r0, r1);
  const int n = static_cast<int>(r1 - r0);
  pdl_wait();  // the table, timestep and x may be written by the previous kernel

  {
    constexpr bool round_table = !std::is_same<TableT, TsT>::value;
    const TableT* table = static_cast<const TableT*>(a.table);
    const TsT* ts = static_cast<const TsT*>(a.ts);
    for (int c8 = threadIdx.x; c8 < COLS / 8; c8 += blockDim.x) {
      const int col = c8 * 8;
      float sh[8], sc[8];
      if (UNIFORM) {
        ada_values8<TableT, TsT>(table + a.shift_index * a.table_stride_row + col, ts + a.shift_index * a.ts_stride_p + col, sh);
        ada_values8<TableT, TsT>(table + a.scale_index * a.table_stride_row + col, ts + a.scale_index * a.ts_stride_p + col, sc);
#pragma unroll
        for (int i = 0; i < 8; ++i) sc[i] = 1.0f + sc[i];
      } else {
        load8<TableT>(table + a.shift_index * a.table_stride_row + col, sh);
        load8<TableT>(table + a.scale_index * a.table_stride_row + col, sc);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          sh[i] = round_table ? bf16_round(sh[i]) : sh[i];
          sc[i] = round_table ? bf16_round(sc[i]) : sc[i];
        }
      }
      store8<float>(ada0 + col, sh);
      store8<float>(ada1 + col, sc);
    }
  }
  __syncthreads();
  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;

  if (warp == kWideWarps) {
    if (elect_one()) {
      const TsT* ts = static_cast<const TsT*>(a.ts);
      ring_produce(ring, stages, S, SB, n, SB, [&](int k, uint8_t* st, uint64_t* bar) {
        const int64_t row = r0 + k;
        bulk_load(st, a.x + row * COLS, COLS * 2, bar);
        if (!UNIFORM) {
          const int64_t b = row / a.tokens;
          const int64_t t = row - b * a.tokens;
          const TsT* tr = ts + b * a.ts_stride_b + t * a.ts_stride_t;
          bulk_load(st + COLS * 2, tr + a.shift_index * a.ts_stride_p, COLS * sizeof(TsT), bar);
          bulk_load(st + COLS * 2 + COLS * sizeof(TsT), tr + a.scale_index * a.ts_stride_p, COLS * sizeof(TsT), bar);
        }
      });
    }
  } else {
    constexpr bool round_ada = std::is_same<TsT, __nv_bfloat16>::value;
    constexpr bool fast_quant = QUANT && QMODE == kQuantTorch;
    // up to three e4m3 outputs of the same bf16 value, each with its own input scale (the per-linear scales
    // of a checkpoint whose Q, K and V projections were calibrated apart)
    const int nq = a.nq > 1 ? (a.nq < 3 ? a.nq : 3) : 1;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
    if (QUANT) {
      s0 = __ldg(a.input_scale);
      s1 = nq > 1 ? __ldg(a.input_scale + 1) : s0;
      s2 = nq > 2 ? __ldg(a.input_scale + 2) : s0;
    }
    const float rcp0 = __frcp_rn(s0), rcp1 = __frcp_rn(s1), rcp2 = __frcp_rn(s2);
    volatile int* abort = &ring.abort;
    for (int k = static_cast<int>(warp); warp < W && k < n; k += W) {
      const int st = k % S;
      if (!mbar_wait(&ring.full[st], (k / S) & 1, abort)) break;
      const uint8_t* stage = stages + static_cast<size_t>(st) * SB;
      const uint4* xs = reinterpret_cast<const uint4*>(stage);
      f2 acc0{0.f, 0.f}, acc1{0.f, 0.f};
#pragma unroll
      for (int j = 0; j < VPL; ++j) sumsq8(xs[j * 32 + lane], acc0, acc1);
      const float ss = warp_allsum((acc0.x + acc0.y) + (acc1.x + acc1.y));
      const float inv_rms = rsqrtf(ss / static_cast<float>(COLS) + a.eps);
      const f2 inv2{inv_rms, inv_rms};
      const int64_t row = r0 + k;
#pragma unroll 4
      for (int j = 0; j < VPL; ++j) {
        const int vec = j * 32 + static_cast<int>(lane);
        const int col = vec * 8;
        const uint4 xv = xs[vec];
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
        float sh[8], sc1[8];
        load8<float>(ada0 + col, sh);
        load8<float>(ada1 + col, sc1);
        if (!UNIFORM) {
          const TsT* tsh = reinterpret_cast<const TsT*>(stage + COLS * 2);
          const TsT* tsc = tsh + COLS;
          float a0[8], a1[8];
          load8<TsT>(tsh + col, a0);
          load8<TsT>(tsc + col, a1);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            sh[i] = round_ada ? bf16_round(sh[i] + a0[i]) : sh[i] + a0[i];
            const float scv = round_ada ? bf16_round(sc1[i] + a1[i]) : sc1[i] + a1[i];
            sc1[i] = 1.0f + scv;
          }
        }
        uint32_t yw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // y = (x * inv_rms) * (1 + scale) + shift, one rounding to bf16
          const f2 y = fma2(mul2(bf16x2_to_f2(xw[i]), inv2), f2{sc1[2 * i], sc1[2 * i + 1]}, f2{sh[2 * i], sh[2 * i + 1]});
          yw[i] = pack_bf16x2(y.x, y.y);
        }
        if (a.y != nullptr) reinterpret_cast<uint4*>(a.y + row * COLS)[vec] = make_uint4(yw[0], yw[1], yw[2], yw[3]);
        if (QUANT) {
#pragma unroll 1
          for (int qi = 0; qi < nq; ++qi) {
            const float sq = qi == 0 ? s0 : (qi == 1 ? s1 : s2);
            const float rq = qi == 0 ? rcp0 : (qi == 1 ? rcp1 : rcp2);
            uint8_t* qrow = a.q + qi * a.q_plane + row * COLS;
            if (fast_quant) {
              const f2 r2{rq, rq};
              const uint32_t lo = quant2_torch(bf16x2_to_f2(yw[0]), r2) | (quant2_torch(bf16x2_to_f2(yw[1]), r2) << 16);
              const uint32_t hi = quant2_torch(bf16x2_to_f2(yw[2]), r2) | (quant2_torch(bf16x2_to_f2(yw[3]), r2) << 16);
              reinterpret_cast<uint2*>(qrow)[vec] = make_uint2(nan_bytes_to_ff(lo), nan_bytes_to_ff(hi));
            } else {
              float yb[8];
              unpack8(make_uint4(yw[0], yw[1], yw[2], yw[3]), yb);
              reinterpret_cast<uint2*>(qrow)[vec] = quant8<__nv_bfloat16, QMODE>(yb, sq, rq);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ring.empty[st]);
    }
  }
}

// ----------------------------------------------------------------------------------------------- RoPE
// Per token, for Q and for K: n = x * rsqrt(mean(x^2) + eps) * w over all 4096 columns, then per head h and
// half index j < 64:  o[j] = n[j] cos - n[j+64] sin,  o[j+64] = n[j+64] cos + n[j] sin  (fp32, one bf16
// rounding: the reference's GPU kernel, triton_ltx_ops.py:3901-3978).  A lane handles 8 of the 256
// (head, 8-column half-block) pairs of a row: the 8 columns j..j+7 and their partners j+64..j+71 read
// straight from the staged row, with the 8 angles of those columns computed (or loaded) once for Q and K.
// Outputs go through the head-group table of RopeArgs (plain [L, 4096] rows, or each head group's GPU).
struct RopeSource {
  // generated cos/sin (inv_freq != null): slot g = 64 * head + j uses position axis slot_axis[g]
  // (0: latent frame t, 1: row h, 2: column w of the token's (t, h, w) in a [frames, grid_h, grid_w]
  // raster of global token index token0 + local index) and inverse frequency inv_freq[g] (radians per
  // position unit)
  const double* inv_freq;
  const uint8_t* slot_axis;
  int grid_h, grid_w;
  int64_t token0;
};

constexpr int kRopeSlots = 2048;  // 32 heads x 64 rotary frequencies
constexpr int kRopePairs = 256;   // 32 heads x 8 eight-column half-blocks
// shared memory ahead of the ring: Q and K weights as fp32 and the frequency table (per pair p and angle
// pair k = e / 2 of its 8 angles: (hi, hi, lo, lo) of angles 2k and 2k + 1, laid out [4][256] so a warp's
// lanes read consecutive 16-byte words; then the 8 position axes of each pair packed 2 bits each)
struct RopeLayout {
  static constexpr int kWeights = 2 * 4096 * 4;
  static constexpr int kFreq = 4 * kRopePairs * 16 + kRopePairs * 4;
  static constexpr int kFixed = kWeights + kFreq;
  __host__ __device__ static constexpr int stage_bytes(bool copy_v) { return (copy_v ? 3 : 2) * 4096 * 2; }
  __host__ __device__ static constexpr int stages(bool copy_v) {
    return ring_stages(((kDynLimit - kFixed) / stage_bytes(copy_v)) > kMaxStages
                           ? kMaxStages
                           : ((kDynLimit - kFixed) / stage_bytes(copy_v)),
                       kRopeWarps);
  }
  __host__ __device__ static constexpr int smem_bytes(bool copy_v) { return kFixed + stages(copy_v) * stage_bytes(copy_v); }
};

// Two angles at once: cos and sin (bf16-rounded, as fp32) of pos * inverse frequency, the frequency given in
// turns as hi + lo with hi holding at most 16 significant bits: pos * hi is exact for integer positions below
// 2^8, its fractional part is exact, and lo adds the rest, so the reduced angle rt is within a few 2^-24
// turns.  The quadrant q = rint(4 rt) leaves x = 2 pi (rt - q / 4) in [-pi/4, pi/4], where the Taylor series
// of sin to x^9 and of cos to x^10 are within 2e-10 (the next terms' size at pi/4), so cos and sin come out
// within a few fp32 ulps, relative to the value for small angles too; cos(x + q pi/2) and sin(x + q pi/2) by
// swapping and negating.
__device__ __forceinline__ void rope_cos_sin2(f2 pos, f2 hi, f2 lo, f2& c, f2& s) {
  const f2 a = mul2(pos, hi);
  const f2 rt = fma2(pos, lo, sub2(a, f2{rintf(a.x), rintf(a.y)}));  // turns, in [-1/2, 1/2] up to rounding
  const f2 r4 = mul2(rt, f2{4.0f, 4.0f});
  const f2 qf{rintf(r4.x), rintf(r4.y)};  // quadrants, -2..2
  const f2 x = mul2(fma2(qf, f2{-0.25f, -0.25f}, rt), f2{6.28318530717958647692f, 6.28318530717958647692f});
  const f2 x2 = mul2(x, x);
  // Taylor coefficients: 1/9!, -1/7!, 1/5!, -1/3!  and  -1/10!, 1/8!, -1/6!, 1/4!, -1/2
  f2 ps = fma2(x2, f2{2.75573192e-6f, 2.75573192e-6f}, f2{-1.98412698e-4f, -1.98412698e-4f});
  ps = fma2(x2, ps, f2{8.33333333e-3f, 8.33333333e-3f});
  ps = fma2(x2, ps, f2{-1.66666667e-1f, -1.66666667e-1f});
  const f2 sn = fma2(mul2(x, x2), ps, x);
  f2 pc = fma2(x2, f2{-2.75573192e-7f, -2.75573192e-7f}, f2{2.48015873e-5f, 2.48015873e-5f});
  pc = fma2(x2, pc, f2{-1.38888889e-3f, -1.38888889e-3f});
  pc = fma2(x2, pc, f2{4.16666667e-2f, 4.16666667e-2f});
  pc = fma2(x2, pc, f2{-0.5f, -0.5f});
  const f2 cs = fma2(x2, pc, f2{1.0f, 1.0f});
  const int q0 = static_cast<int>(qf.x), q1 = static_cast<int>(qf.y);
  // odd quadrants swap cos and sin; cos is negated in quadrants 1 and 2, sin in 2 and 3 (= -1 and -2)
  float c0 = (q0 & 1) ? sn.x : cs.x, s0 = (q0 & 1) ? cs.x : sn.x;
  float c1 = (q1 & 1) ? sn.y : cs.y, s1 = (q1 & 1) ? cs.y : sn.y;
  c0 = __uint_as_float(__float_as_uint(c0) ^ ((static_cast<uint32_t>(q0 + 1) & 2u) << 30));
  c1 = __uint_as_float(__float_as_uint(c1) ^ ((static_cast<uint32_t>(q1 + 1) & 2u) << 30));
  s0 = __uint_as_float(__float_as_uint(s0) ^ ((static_cast<uint32_t>(q0) & 2u) << 30));
  s1 = __uint_as_float(__float_as_uint(s1) ^ ((static_cast<uint32_t>(q1) & 2u) << 30));
  c = bf16x2_to_f2(pack_bf16x2(c0, c1));
  s = bf16x2_to_f2(pack_bf16x2(s0, s1));
}

// Splits inv_freq / 2pi (turns per position unit) into the (hi, lo) pair rope_cos_sin2 expects.
__device__ __forceinline__ float2 turns_split(double inv_freq) {
  const double t = inv_freq * 0.15915494309189533577;  // 1 / (2 pi)
  const float hi = __uint_as_float(__float_as_uint(static_cast<float>(t)) & 0xFFFFFF00u);
  return make_float2(hi, static_cast<float>(t - static_cast<double>(hi)));
}

// Fills the frequency table of this CTA: fr[k][p] = (hi, hi, lo, lo) of slots 8 p + 2 k and 8 p + 2 k + 1
// (slot 64 * head + j with j = 8 * (p % 8) + e, so slot = 8 p + e), ax[p] the packed axes of slots 8 p ..
// 8 p + 7.
__device__ __forceinline__ void rope_freq_table(const RopeSource& src, float4* fr, uint32_t* ax) {
  for (int i = threadIdx.x; i < kRopeSlots / 2; i += blockDim.x) {
    const int p = i >> 2, k = i & 3;
    const float2 f0 = turns_split(src.inv_freq[p * 8 + 2 * k]);
    const float2 f1 = turns_split(src.inv_freq[p * 8 + 2 * k + 1]);
    fr[k * kRopePairs + p] = make_float4(f0.x, f1.x, f0.y, f1.y);
  }
  for (int p = threadIdx.x; p < kRopePairs; p += blockDim.x) {
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) packed |= (static_cast<uint32_t>(src.slot_axis[p * 8 + e]) & 3u) << (2 * e);
    ax[p] = packed;
  }
}

__device__ __forceinline__ void token_position(const RopeSource& src, int64_t local_t, float (&pos)[3]) {
  const int64_t gt = src.token0 + local_t;
  const int64_t hw = static_cast<int64_t>(src.grid_h) * src.grid_w;
  const int64_t f = gt / hw;
  const int64_t rem = gt - f * hw;
  const int64_t h = rem / src.grid_w;
  pos[0] = static_cast<float>(f);
  pos[1] = static_cast<float>(h);
  pos[2] = static_cast<float>(rem - h * src.grid_w);
}

__device__ __forceinline__ float axis_pos(const float (&pos)[3], uint32_t axe) {
  return axe == 0 ? pos[0] : (axe == 1 ? pos[1] : pos[2]);
}

// The 8 cos/sin of pair p for a token at `pos` (generated), as 4 packed pairs each.
__device__ __forceinline__ void pair_cos_sin_gen(const float4* fr, const uint32_t* ax, int p, const float (&pos)[3],
                                                 f2 (&c)[4], f2 (&s)[4]) {
  const uint32_t axes = ax[p];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float4 f = fr[k * kRopePairs + p];
    const f2 ps{axis_pos(pos, (axes >> (4 * k)) & 3u), axis_pos(pos, (axes >> (4 * k + 2)) & 3u)};
    rope_cos_sin2(ps, f2{f.x, f.y}, f2{f.z, f.w}, c[k], s[k]);
  }
}

// Normalises, weights and rotates the 16 columns of pair p of one tensor's staged row and stores them.
__device__ __forceinline__ void rope_pair(const uint4* row, const float* w, int c0, f2 inv2, const f2 (&c)[4],
                                          const f2 (&s)[4], __nv_bfloat16* dst) {
  const uint4 x0 = row[c0 / 8], x1 = row[c0 / 8 + 8];
  const uint32_t w0[4] = {x0.x, x0.y, x0.z, x0.w}, w1[4] = {x1.x, x1.y, x1.z, x1.w};
  const float4* wv = reinterpret_cast<const float4*>(w + c0);
  const float4 wa0 = wv[0], wa1 = wv[1], wb0 = wv[16], wb1 = wv[17];  // columns c0..c0+7 and c0+64..c0+71
  const f2 ww0[4] = {f2{wa0.x, wa0.y}, f2{wa0.z, wa0.w}, f2{wa1.x, wa1.y}, f2{wa1.z, wa1.w}};
  const f2 ww1[4] = {f2{wb0.x, wb0.y}, f2{wb0.z, wb0.w}, f2{wb1.x, wb1.y}, f2{wb1.z, wb1.w}};
  uint32_t o0[4], o1[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const f2 n0 = mul2(mul2(bf16x2_to_f2(w0[k]), inv2), ww0[k]);  // (x * inv_rms) * w
    const f2 n1 = mul2(mul2(bf16x2_to_f2(w1[k]), inv2), ww1[k]);
    // o[j] = n[j] cos - n[j+64] sin,  o[j+64] = n[j+64] cos + n[j] sin
    const f2 a = fma2(n0, c[k], mul2(n1, f2{-s[k].x, -s[k].y}));
    const f2 b = fma2(n1, c[k], mul2(n0, s[k]));
    o0[k] = pack_bf16x2(a.x, a.y);
    o1[k] = pack_bf16x2(b.x, b.y);
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(o0[0], o0[1], o0[2], o0[3]);
  *reinterpret_cast<uint4*>(dst + 64) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
}

template <typename WT, typename CsT, bool GEN, bool COPY_V>
__global__ void __launch_bounds__(kRopeThreads, 1) qk_rmsnorm_rope_ring_kernel(RopeArgs a, RopeSource src) {
  pdl_trigger();
  constexpr int S = RopeLayout::stages(COPY_V);  // a multiple of W
  constexpr int W = ring_warps(S, kRopeWarps);
  constexpr uint32_t SB = RopeLayout::stage_bytes(COPY_V);
  extern __shared__ uint8_t smem_raw[];
  __shared__ Ring ring;
  uint8_t* smem = smem_raw + (((smem_u32(smem_raw) + 127u) & ~127u) - smem_u32(smem_raw));
  float* wq = reinterpret_cast<float*>(smem);
  float* wk = wq + 4096;
  float4* fr = reinterpret_cast<float4*>(smem + RopeLayout::kWeights);
  uint32_t* ax = reinterpret_cast<uint32_t*>(fr + 4 * kRopePairs);
  uint8_t* stages = smem + RopeLayout::kFixed;
  ring_init(ring, S);
  int64_t r0, r1;
  cta_rows(a.tokens, r0, r1);
  const int n = static_cast<int>(r1 - r0);
  pdl_wait();
  for (int i = threadIdx.x; i < 4096 / 8; i += blockDim.x) {
    float f[8];
    load8<WT>(static_cast<const WT*>(a.q_weight) + i * 8, f);
    store8<float>(wq + i * 8, f);
    load8<WT>(static_cast<const WT*>(a.k_weight) + i * 8, f);
    store8<float>(wk + i * 8, f);
  }
  if (GEN) rope_freq_table(src, fr, ax);
  __syncthreads();
  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;

  if (warp == kRopeWarps) {
    if (elect_one()) {
      ring_produce(ring, stages, S, SB, n, SB, [&](int k, uint8_t* st, uint64_t* bar) {
        const int64_t t = r0 + k;
        bulk_load(st, a.q + t * a.in_stride_t, 8192, bar);
        bulk_load(st + 8192, a.k + t * a.in_stride_t, 8192, bar);
        if (COPY_V) bulk_load(st + 16384, a.v + t * a.in_stride_t, 8192, bar);
      });
    }
  } else {
    volatile int* abort = &ring.abort;
    const CsT* cosb = static_cast<const CsT*>(a.cos);
    const CsT* sinb = static_cast<const CsT*>(a.sin);
    for (int k = static_cast<int>(warp); warp < W && k < n; k += W) {
      const int st = k % S;
      if (!mbar_wait(&ring.full[st], (k / S) & 1, abort)) break;
      const uint8_t* stage = stages + static_cast<size_t>(st) * SB;
      const uint4* rq = reinterpret_cast<const uint4*>(stage);
      const uint4* rk = rq + 512;
      f2 aq0{0.f, 0.f}, aq1{0.f, 0.f}, ak0{0.f, 0.f}, ak1{0.f, 0.f};
#pragma unroll 8
      for (int j = 0; j < 16; ++j) {
        sumsq8(rq[j * 32 + lane], aq0, aq1);
        sumsq8(rk[j * 32 + lane], ak0, ak1);
      }
      const float sq = warp_allsum((aq0.x + aq0.y) + (aq1.x + aq1.y));
      const float sk = warp_allsum((ak0.x + ak0.y) + (ak1.x + ak1.y));
      const float inv_q = rsqrtf(sq / 4096.f + a.eps);
      const float inv_k = rsqrtf(sk / 4096.f + a.eps);
      const int64_t t = r0 + k;
      float pos[3] = {0.f, 0.f, 0.f};
      if (GEN) token_position(src, t, pos);
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        const int p = i * 32 + static_cast<int>(lane);  // pair: head p / 8, columns 8 * (p % 8) + [0, 8) (+ 64)
        const int head = p >> 3;
        const int c0 = head * 128 + (p & 7) * 8;
        f2 c[4], s[4];
        if (GEN) {
          pair_cos_sin_gen(fr, ax, p, pos, c, s);
        } else {
          const int64_t off = head * a.cs_stride_h + t * a.cs_stride_t + (p & 7) * 8;
          float cf[8], sf[8];
          load8<CsT>(cosb + off, cf);
          load8<CsT>(sinb + off, sf);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            c[e] = f2{cf[2 * e], cf[2 * e + 1]};
            s[e] = f2{sf[2 * e], sf[2 * e + 1]};
          }
        }
        const int g = head / a.heads_per_group;
        const int hl = head - g * a.heads_per_group;
        const int64_t o = t * a.out_stride_t + hl * 128 + (p & 7) * 8;
        rope_pair(rq, wq, c0, f2{inv_q, inv_q}, c, s, group_base(a.dst[0], g) + o);
        rope_pair(rk, wk, c0, f2{inv_k, inv_k}, c, s, group_base(a.dst[1], g) + o);
      }
      if (COPY_V) {
        const uint4* rv = rq + 1024;
#pragma unroll 4
        for (int j = 0; j < 16; ++j) {
          const int vec = j * 32 + static_cast<int>(lane);
          const int head = vec >> 4;
          const int g = head / a.heads_per_group;
          const int hl = head - g * a.heads_per_group;
          *reinterpret_cast<uint4*>(group_base(a.dst[2], g) + t * a.out_stride_t + hl * 128 + (vec & 15) * 8) = rv[vec];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ring.empty[st]);
    }
  }
  if (a.system_fence) {
    // one system-scope fence per CTA after the barrier: fences are cumulative, so it orders every thread's
    // peer stores before the signal the next kernel releases
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
  }
}

// ------------------------------------------------------------------------------------- Q/K RMSNorm only
// RmsRowsArgs rows through the ring: a warp per row, the RoPE kernel's sum of squares and normalisation
// ((x * inv_rms) * w, one bf16 rounding); the row is staged whole before its first store, so the output
// may alias the input.
constexpr int kRmsFixed = 2 * 4096 * 4;  // Q and K weights as fp32
constexpr int kRmsStages = ring_stages(
    ((kDynLimit - kRmsFixed) / 8192) > kMaxStages ? kMaxStages : ((kDynLimit - kRmsFixed) / 8192), kWideWarps);
constexpr int kRmsSmem = kRmsFixed + kRmsStages * 8192;

template <typename WT>
__global__ void __launch_bounds__(kWideThreads, 1) qk_rmsnorm_ring_kernel(RmsRowsArgs a) {
  pdl_trigger();
  constexpr int S = kRmsStages;  // a multiple of W
  constexpr int W = ring_warps(S, kWideWarps);
  extern __shared__ uint8_t smem_raw[];
  __shared__ Ring ring;
  uint8_t* smem = smem_raw + (((smem_u32(smem_raw) + 127u) & ~127u) - smem_u32(smem_raw));
  float* wq = reinterpret_cast<float*>(smem);
  float* wk = wq + 4096;
  uint8_t* stages = smem + kRmsFixed;
  ring_init(ring, S);
  int64_t r0, r1;
  cta_rows(a.rows, r0, r1);
  const int n = static_cast<int>(r1 - r0);
  pdl_wait();
  for (int i = threadIdx.x; i < 4096 / 8; i += blockDim.x) {
    float f[8];
    load8<WT>(static_cast<const WT*>(a.weight[0]) + i * 8, f);
    store8<float>(wq + i * 8, f);
    load8<WT>(static_cast<const WT*>(a.weight[1]) + i * 8, f);
    store8<float>(wk + i * 8, f);
  }
  __syncthreads();
  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;
  if (warp == kWideWarps) {
    if (elect_one()) {
      ring_produce(ring, stages, S, 8192u, n, 8192u, [&](int k, uint8_t* st, uint64_t* bar) {
        const int64_t r = r0 + k;
        // selects, not a.in[j]: a runtime index into the parameter arrays would copy them to local memory
        const bool is_k = r >= a.rows_q;
        const int64_t t = is_k ? r - a.rows_q : r;
        bulk_load(st, (is_k ? a.in[1] : a.in[0]) + t * (is_k ? a.in_stride[1] : a.in_stride[0]), 8192, bar);
      });
    }
  } else {
    volatile int* abort = &ring.abort;
    for (int k = static_cast<int>(warp); warp < W && k < n; k += W) {
      const int st = k % S;
      if (!mbar_wait(&ring.full[st], (k / S) & 1, abort)) break;
      const uint4* row = reinterpret_cast<const uint4*>(stages + static_cast<size_t>(st) * 8192);
      f2 a0{0.f, 0.f}, a1{0.f, 0.f};
#pragma unroll 8
      for (int j = 0; j < 16; ++j) sumsq8(row[j * 32 + lane], a0, a1);
      const float ss = warp_allsum((a0.x + a0.y) + (a1.x + a1.y));
      const f2 inv2{rsqrtf(ss / 4096.f + a.eps), rsqrtf(ss / 4096.f + a.eps)};
      const int64_t r = r0 + k;
      const bool is_k = r >= a.rows_q;
      const int64_t t = is_k ? r - a.rows_q : r;
      __nv_bfloat16* out = (is_k ? a.out[1] : a.out[0]) + t * (is_k ? a.out_stride[1] : a.out_stride[0]);
      const float* w = is_k ? wk : wq;
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        const int vec = j * 32 + static_cast<int>(lane);
        const uint4 xv = row[vec];
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
        const float4 wa = reinterpret_cast<const float4*>(w + vec * 8)[0];
        const float4 wb = reinterpret_cast<const float4*>(w + vec * 8)[1];
        const f2 ww[4] = {f2{wa.x, wa.y}, f2{wa.z, wa.w}, f2{wb.x, wb.y}, f2{wb.z, wb.w}};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const f2 nv = mul2(mul2(bf16x2_to_f2(xw[i]), inv2), ww[i]);
          o[i] = pack_bf16x2(nv.x, nv.y);
        }
        reinterpret_cast<uint4*>(out)[vec] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ring.empty[st]);
    }
  }
}

// The cos/sin the generating RoPE kernel uses, written as [32, tokens, 64] tables (same element order as the
// reference's tables): one thread per (head, token, 8 columns), the same arithmetic as the kernel.
template <typename CsT>
__global__ void __launch_bounds__(256) rope_tables_kernel(RopeSource src, int64_t tokens, CsT* cos_out, CsT* sin_out) {
  const int64_t total = 32 * tokens * 8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int pv = static_cast<int>(i & 7);
    const int64_t ht = i >> 3;
    const int head = static_cast<int>(ht / tokens);
    const int64_t t = ht - static_cast<int64_t>(head) * tokens;
    float pos[3];
    token_position(src, t, pos);
    float c[8], s[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int slot = head * 64 + pv * 8 + 2 * k;
      const float2 f0 = turns_split(src.inv_freq[slot]), f1 = turns_split(src.inv_freq[slot + 1]);
      const f2 ps{axis_pos(pos, src.slot_axis[slot] & 3u), axis_pos(pos, src.slot_axis[slot + 1] & 3u)};
      f2 cc, ss;
      rope_cos_sin2(ps, f2{f0.x, f1.x}, f2{f0.y, f1.y}, cc, ss);
      c[2 * k] = cc.x;
      c[2 * k + 1] = cc.y;
      s[2 * k] = ss.x;
      s[2 * k + 1] = ss.y;
    }
    store8<CsT>(cos_out + ht * 64 + pv * 8, c);
    store8<CsT>(sin_out + ht * 64 + pv * 8, s);
  }
}

}  // namespace rows
}  // namespace ogx
