// Row-pipeline kernels for the HBM-bound stages that normalise whole 4096-column rows: AdaZero (+ the
// E4M3 quantiser) and the Q/K RMSNorm + split RoPE (+ the sequence-to-head scatter).
//
// A row's RMS needs every column before any output can be written, so a kernel that holds the row in
// registers keeps few rows in flight per SM and leaves HBM idle between a row's load and its reduction.
// Here one persistent CTA per SM streams its rows through a ring of shared-memory stages instead:
//   warp 8 (one elected thread)  issues cp.async.bulk copies of whole rows (8 KB per 4096-column bf16
//                                row) into the ring, a row as soon as its stage is free;
//   warps 0..7                   each take every eighth row of the CTA: wait for its stage, reduce the
//                                sum of squares from shared memory (warp shuffles, no block barrier),
//                                write the outputs with 16-byte stores, free the stage.
// With 11-16 stages a SM keeps 128-176 KB of row loads in flight, which is what the HBM latency needs;
// no register holds a row.  Every wait is bounded (a wait that runs out records OGX_ERR_TIMEOUT, the
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

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
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

struct Ring {
  uint64_t full[16];
  uint64_t empty[16];
  int abort;
};

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
  static constexpr int kAda = 2 * COLS * static_cast<int>(sizeof(TsT));  // shift, scale (bf16-exact for bf16 ts)
  static constexpr int kStageUniform = COLS * 2;
  static constexpr int kStagePerToken = COLS * 2 + 2 * COLS * static_cast<int>(sizeof(TsT));
  __host__ __device__ static constexpr int stage_bytes(bool uniform) { return uniform ? kStageUniform : kStagePerToken; }
  __host__ __device__ static constexpr int stages(bool uniform) {
    return ((kDynLimit - kAda) / stage_bytes(uniform)) > 16 ? 16 : ((kDynLimit - kAda) / stage_bytes(uniform));
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
__global__ void __launch_bounds__(kThreads, 1) adazero_ring_kernel(AdaArgs a) {
  pdl_trigger();
  using Lay = AdaLayout<COLS, TsT>;
  constexpr int S = Lay::stages(UNIFORM);
  constexpr uint32_t SB = Lay::stage_bytes(UNIFORM);
  constexpr int VPL = COLS / 8 / 32;  // 16-byte vectors per lane
  extern __shared__ uint8_t smem_raw[];
  __shared__ Ring ring;
  uint8_t* smem = smem_raw + (((smem_u32(smem_raw) + 127u) & ~127u) - smem_u32(smem_raw));
  TsT* ada_shift = reinterpret_cast<TsT*>(smem);
  TsT* ada_scale = ada_shift + COLS;
  uint8_t* stages = smem + Lay::kAda;
  ring_init(ring, S);
  int64_t r0, r1;
  cta_rows(a.rows, r0, r1);
  const int n = static_cast<int>(r1 - r0);
  pdl_wait();  // the table, timestep and x may be written by the previous kernel

  // Ada values per column: uniform -> round(table + ts); per token -> the (rounded) table part only
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
      } else {
        load8<TableT>(table + a.shift_index * a.table_stride_row + col, sh);
        load8<TableT>(table + a.scale_index * a.table_stride_row + col, sc);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          sh[i] = round_table ? bf16_round(sh[i]) : sh[i];
          sc[i] = round_table ? bf16_round(sc[i]) : sc[i];
        }
      }
      store8<TsT>(ada_shift + col, sh);
      store8<TsT>(ada_scale + col, sc);
    }
  }
  __syncthreads();
  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;

  if (warp == kConsumerWarps) {
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
    float s = 0.f, r = 0.f;
    if (QUANT) {
      s = __ldg(a.input_scale);
      r = __frcp_rn(s);
    }
    volatile int* abort = &ring.abort;
    for (int k = static_cast<int>(warp); k < n; k += kConsumerWarps) {
      const int st = k % S;
      if (!mbar_wait(&ring.full[st], (k / S) & 1, abort)) break;
      const uint8_t* stage = stages + static_cast<size_t>(st) * SB;
      const uint4* xs = reinterpret_cast<const uint4*>(stage);
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        float f[8];
        unpack8(xs[j * 32 + lane], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
      }
      ss = warp_allsum(ss);
      const float inv_rms = rsqrtf(ss / static_cast<float>(COLS) + a.eps);
      const int64_t row = r0 + k;
#pragma unroll 4
      for (int j = 0; j < VPL; ++j) {
        const int vec = j * 32 + static_cast<int>(lane);
        const int col = vec * 8;
        float f[8], sh[8], sc[8], y[8];
        unpack8(xs[vec], f);
        load8<TsT>(ada_shift + col, sh);
        load8<TsT>(ada_scale + col, sc);
        if (!UNIFORM) {
          const TsT* tsh = reinterpret_cast<const TsT*>(stage + COLS * 2);
          const TsT* tsc = tsh + COLS;
          float a0[8], a1[8];
          load8<TsT>(tsh + col, a0);
          load8<TsT>(tsc + col, a1);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            sh[i] = round_ada ? bf16_round(sh[i] + a0[i]) : sh[i] + a0[i];
            sc[i] = round_ada ? bf16_round(sc[i] + a1[i]) : sc[i] + a1[i];
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = fmaf(f[i] * inv_rms, 1.0f + sc[i], sh[i]);
        const uint4 yv = pack8(y);
        if (a.y != nullptr) reinterpret_cast<uint4*>(a.y + row * COLS)[vec] = yv;
        if (QUANT) {
          float yb[8];
          unpack8(yv, yb);
          reinterpret_cast<uint2*>(a.q + row * COLS)[vec] = quant8<__nv_bfloat16, QMODE>(yb, s, r);
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
// shared memory ahead of the ring: Q and K weights (bf16 or fp32) and the frequency table
// (per pair: 8 (hi, lo) turn frequencies laid out [8][256] so a warp's lanes read consecutive words,
// and the 8 axes packed 2 bits each)
template <typename WT>
struct RopeLayout {
  static constexpr int kWeights = 2 * 4096 * static_cast<int>(sizeof(WT));
  static constexpr int kFreq = 8 * kRopePairs * 8 + kRopePairs * 4;
  static constexpr int kFixed = kWeights + kFreq;
  __host__ __device__ static constexpr int stage_bytes(bool copy_v) { return (copy_v ? 3 : 2) * 4096 * 2; }
  __host__ __device__ static constexpr int stages(bool copy_v) {
    return ((kDynLimit - kFixed) / stage_bytes(copy_v)) > 16 ? 16 : ((kDynLimit - kFixed) / stage_bytes(copy_v));
  }
  __host__ __device__ static constexpr int smem_bytes(bool copy_v) { return kFixed + stages(copy_v) * stage_bytes(copy_v); }
};

// cos and sin (bf16-rounded, as fp32) of position * inverse frequency, the frequency given in turns as
// hi + lo with hi holding at most 16 significant bits: pos * hi is exact for integer positions below 2^8,
// its fractional part is exact, and lo adds the rest, so the reduced angle rt is within a few 2^-24 turns.
// Then the quadrant q = rint(4 rt) leaves x = 2 pi (rt - q / 4) in [-pi/4, pi/4], where the Taylor series
// of sin to x^9 and of cos to x^10 are within 2e-10 (the next terms' size at pi/4), so cos and sin come out
// within a few fp32 ulps, relative to the value for small angles too; cos(x + q pi/2), sin(x + q pi/2) by
// swapping and negating.
__device__ __forceinline__ void rope_cos_sin(float pos, float hi, float lo, float& c, float& s) {
  const float a = pos * hi;
  const float rt = fmaf(pos, lo, a - rintf(a));  // turns, in [-1/2, 1/2] up to rounding
  const float qf = rintf(rt * 4.0f);             // quadrant, -2..2
  const float x = fmaf(qf, -0.25f, rt) * 6.28318530717958647692f;
  const float x2 = x * x;
  // Taylor coefficients: 1/9!, -1/7!, 1/5!, -1/3!  and  -1/10!, 1/8!, -1/6!, 1/4!, -1/2
  float ps = fmaf(x2, 2.75573192e-6f, -1.98412698e-4f);
  ps = fmaf(x2, ps, 8.33333333e-3f);
  ps = fmaf(x2, ps, -1.66666667e-1f);
  const float sn = fmaf(x * x2, ps, x);
  float pc = fmaf(x2, -2.75573192e-7f, 2.48015873e-5f);
  pc = fmaf(x2, pc, -1.38888889e-3f);
  pc = fmaf(x2, pc, 4.16666667e-2f);
  pc = fmaf(x2, pc, -0.5f);
  const float cs = fmaf(x2, pc, 1.0f);
  const int q = static_cast<int>(qf);
  const float c0 = (q & 1) ? sn : cs;
  const float s0 = (q & 1) ? cs : sn;
  float cv = ((q + 1) & 2) ? -c0 : c0;
  float sv = (q & 2) ? -s0 : s0;
  bf16_round2(cv, sv);
  c = cv;
  s = sv;
}

// Splits inv_freq / 2pi (turns per position unit) into the (hi, lo) pair rope_cos_sin expects.
__device__ __forceinline__ float2 turns_split(double inv_freq) {
  const double t = inv_freq * 0.15915494309189533577;  // 1 / (2 pi)
  const float hi = __uint_as_float(__float_as_uint(static_cast<float>(t)) & 0xFFFFFF00u);
  return make_float2(hi, static_cast<float>(t - static_cast<double>(hi)));
}

// Fills the frequency table of this CTA: fr[e][p] = turns of slot 64 * (p / 8) + 8 * (p % 8) + e, ax[p] the
// packed axes.
__device__ __forceinline__ void rope_freq_table(const RopeSource& src, float2* fr, uint32_t* ax) {
  for (int i = threadIdx.x; i < kRopeSlots; i += blockDim.x) {
    const int p = i >> 3, e = i & 7;  // slot i = 64 * head + j, j = 8 * (p % 8) + e  ->  p = i / 8
    fr[e * kRopePairs + p] = turns_split(src.inv_freq[i]);
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

template <typename WT, typename CsT, bool GEN, bool COPY_V>
__global__ void __launch_bounds__(kThreads, 1) qk_rmsnorm_rope_ring_kernel(RopeArgs a, RopeSource src) {
  pdl_trigger();
  using Lay = RopeLayout<WT>;
  constexpr int S = Lay::stages(COPY_V);
  constexpr uint32_t SB = Lay::stage_bytes(COPY_V);
  extern __shared__ uint8_t smem_raw[];
  __shared__ Ring ring;
  uint8_t* smem = smem_raw + (((smem_u32(smem_raw) + 127u) & ~127u) - smem_u32(smem_raw));
  WT* wq = reinterpret_cast<WT*>(smem);
  WT* wk = wq + 4096;
  float2* fr = reinterpret_cast<float2*>(smem + Lay::kWeights);
  uint32_t* ax = reinterpret_cast<uint32_t*>(fr + 8 * kRopePairs);
  uint8_t* stages = smem + Lay::kFixed;
  ring_init(ring, S);
  int64_t r0, r1;
  cta_rows(a.tokens, r0, r1);
  const int n = static_cast<int>(r1 - r0);
  pdl_wait();
  for (int i = threadIdx.x; i < 4096 / 8; i += blockDim.x) {
    float f[8];
    load8<WT>(static_cast<const WT*>(a.q_weight) + i * 8, f);
    store8<WT>(wq + i * 8, f);
    load8<WT>(static_cast<const WT*>(a.k_weight) + i * 8, f);
    store8<WT>(wk + i * 8, f);
  }
  if (GEN) rope_freq_table(src, fr, ax);
  __syncthreads();
  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;

  if (warp == kConsumerWarps) {
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
    for (int k = static_cast<int>(warp); k < n; k += kConsumerWarps) {
      const int st = k % S;
      if (!mbar_wait(&ring.full[st], (k / S) & 1, abort)) break;
      const uint8_t* stage = stages + static_cast<size_t>(st) * SB;
      const uint4* rq = reinterpret_cast<const uint4*>(stage);
      const uint4* rk = rq + 512;
      float sq = 0.f, sk = 0.f;
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        float f[8], g[8];
        unpack8(rq[j * 32 + lane], f);
        unpack8(rk[j * 32 + lane], g);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          sq = fmaf(f[i], f[i], sq);
          sk = fmaf(g[i], g[i], sk);
        }
      }
      sq = warp_allsum(sq);
      sk = warp_allsum(sk);
      const float inv_q = rsqrtf(sq / 4096.f + a.eps);
      const float inv_k = rsqrtf(sk / 4096.f + a.eps);
      const int64_t t = r0 + k;
      float pos[3] = {0.f, 0.f, 0.f};
      if (GEN) token_position(src, t, pos);
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        const int p = i * 32 + static_cast<int>(lane);  // pair: head p / 8, columns 8 * (p % 8) + [0, 8) (+ 64)
        const int head = p >> 3;
        const int c0 = head * 128 + (p & 7) * 8;
        float c[8], s[8];
        if (GEN) {
          const uint32_t axes = ax[p];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t axe = (axes >> (2 * e)) & 3u;
            const float ps = axe == 0 ? pos[0] : (axe == 1 ? pos[1] : pos[2]);
            const float2 f = fr[e * kRopePairs + p];
            rope_cos_sin(ps, f.x, f.y, c[e], s[e]);
          }
        } else {
          const int64_t off = head * a.cs_stride_h + t * a.cs_stride_t + (p & 7) * 8;
          load8<CsT>(cosb + off, c);
          load8<CsT>(sinb + off, s);
        }
        const int g = head / a.heads_per_group;
        const int hl = head - g * a.heads_per_group;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const uint4* rr = which ? rk : rq;
          const WT* w = which ? wk : wq;
          const float inv = which ? inv_k : inv_q;
          float x0[8], x1[8], w0[8], w1[8], n0[8], n1[8], o0[8], o1[8];
          unpack8(rr[c0 / 8], x0);
          unpack8(rr[c0 / 8 + 8], x1);
          load8<WT>(w + c0, w0);
          load8<WT>(w + c0 + 64, w1);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            n0[e] = x0[e] * inv * w0[e];
            n1[e] = x1[e] * inv * w1[e];
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            o0[e] = fmaf(n0[e], c[e], -(n1[e] * s[e]));
            o1[e] = fmaf(n1[e], c[e], n0[e] * s[e]);
          }
          __nv_bfloat16* dst = group_base(a.dst[which], g) + t * a.out_stride_t + hl * 128 + (p & 7) * 8;
          *reinterpret_cast<uint4*>(dst) = pack8(o0);
          *reinterpret_cast<uint4*>(dst + 64) = pack8(o1);
        }
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

// The cos/sin the generating RoPE kernel uses, written as [32, tokens, 64] tables (same element order as the
// reference's tables): one thread per (head, token, 8 columns).
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
    for (int e = 0; e < 8; ++e) {
      const int slot = head * 64 + pv * 8 + e;
      const float2 f = turns_split(src.inv_freq[slot]);
      const uint32_t axe = src.slot_axis[slot] & 3u;
      rope_cos_sin(axe == 0 ? pos[0] : (axe == 1 ? pos[1] : pos[2]), f.x, f.y, c[e], s[e]);
    }
    store8<CsT>(cos_out + ht * 64 + pv * 8, c);
    store8<CsT>(sin_out + ht * 64 + pv * 8, s);
  }
}

}  // namespace rows
}  // namespace ogx
