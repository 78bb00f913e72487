// Dense bidirectional attention, head_dim 128, bf16 in / fp32 softmax and
// accumulation / bf16 (or e4m3) out, on the 5th-generation tensor cores:
//   O[b, t, h, :] = softmax(Q[b, t, h, :] . K[b, :, h, :]^T * scale) V[b, :, h, :]
// This is the contract of the reference's attention backends
// (benchmarks/official_ltx23_benchmark.py:3289-3373: q/k/v [B, L, H*d] viewed
// [B, L, H, d], scale d^-0.5, no mask).
//
// One CTA per (256-query block, head, batch), 12 warps:
//   warp 0        TMA producer: Q (2 tiles x 128 rows, once), then K/V tiles
//                 of 128 keys through a 2-deep ring (128-byte swizzle)
//   warp 1        MMA issuer:   S_q = Q_q K^T (tcgen05 kind::f16, both operands
//                 in shared memory) and O_q += P_q V (P read straight from
//                 TMEM, V as an MN-major shared-memory operand)
//   warps 4..7    softmax for Q tile 0; warps 8..11 for Q tile 1.  Each thread
//                 owns one query row: it reads its 128 scores from TMEM, keeps
//                 a running max/sum, writes P (bf16) back into TMEM over the
//                 consumed scores, rescales its O row in TMEM when the max grew
//                 by more than 2^8, and finally normalises O and stores it.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512);
// P_q occupies the first 64 columns of S_q (two bf16 per 32-bit column).
// The MMA order S0(j+1) after PV0(j) keeps the tensor pipe busy while the
// other tile's softmax runs; tcgen05.mma operations issued by one thread
// execute in issue order, which makes writing S0(j+1) over P0(j) safe.
#pragma once

#include "ogx_sm100.cuh"
#include "elementwise.cuh"

namespace ogx {
namespace fmha {

constexpr int HD = 128;
constexpr int BQ = 128;
constexpr int NQ = 2;
constexpr int BKV = 128;
constexpr int STAGES = 2;
constexpr int HALF_BYTES = 128 * 64 * 2;  // one 64-column half of a 128-row tile
constexpr int TILE_BYTES = 2 * HALF_BYTES;
constexpr int SMEM_BYTES = (NQ + 2 * STAGES) * TILE_BYTES + 1024;
constexpr int kThreads = 384;
// Register split (setmaxnreg): the kernel is launched with kLaunchRegs per thread (the host checks the
// built count before launching); warpgroup 0 (TMA / MMA) drops to kRegsProducer and the two softmax
// warpgroups rise to kRegsSoftmax.  The split must fit in what the launch reserved, or the increase
// would wait forever: 128 * 96 + 256 * 200 = 63488 <= 384 * 168 = 64512.
constexpr int kLaunchRegs = 168;
constexpr uint32_t kRegsProducer = 96;
constexpr uint32_t kRegsSoftmax = 200;
static_assert(128 * kRegsProducer + 256 * kRegsSoftmax <= kThreads * kLaunchRegs, "register split exceeds the launch");
constexpr uint32_t TMEM_COLS = 512;
// A row's running max only moves when a new score exceeds it by more than
// this many log2 units, so P <= 2^8 and most tiles need no O rescale.
constexpr float kRescaleThreshold = 8.0f;

struct Params {
  int L;             // tokens (keys == queries)
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* out;  // bf16 output (when out_q is null)
  uint8_t* out_q;      // e4m3 output (quantised with *out_scale, torch-path semantics)
  const float* out_scale;
  int64_t out_stride_b, out_stride_t;  // elements; the head stride is 128
};

struct SharedState {
  uint64_t q_full;
  uint64_t k_full[STAGES], k_empty[STAGES];
  uint64_t v_full[STAGES], v_empty[STAGES];
  uint64_t s_full[NQ];
  uint64_t p_full[NQ];
  uint64_t o_done[NQ];
  uint64_t drained;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for the share of the exponentials the MUFU unit cannot
// absorb at tensor-core rate.  x = j + f with j = round(x) taken from the bits of
// x + 1.5*2^23 and f in [-1/2, 1/2]; 2^f by a degree-3 polynomial fitted here to
// 2^f on [-1/2, 1/2] (least squares on Chebyshev nodes with Lawson reweighting
// towards minimax; max relative error 7.5e-5, far below bf16's 2^-9); 2^j is
// added to the exponent field.  x is clamped at -126 (P rounds to 0 there).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = x + 12582912.0f;  // 1.5 * 2^23: the low mantissa bits hold round(x)
  const float f = x - (t - 12582912.0f);
  float p = fmaf(0.0551716648f, f, 0.2426111251f);
  p = fmaf(p, f, 0.6932609677f);
  p = fmaf(p, f, 0.9999280572f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Which 32-column chunks of a score row use the polynomial instead of the MUFU ex2.
constexpr uint32_t kPolyChunkMask = 0x8u;

// Packed two-lane fp32 arithmetic (sm_100 f32x2 instructions): one issue slot for two values.
struct f2 {
  float x, y;
};
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("{.reg .b64 A, B, C, D;\n\t"
      "mov.b64 A, {%2, %3};\n\tmov.b64 B, {%4, %5};\n\tmov.b64 C, {%6, %7};\n\t"
      "fma.rn.f32x2 D, A, B, C;\n\tmov.b64 {%0, %1}, D;}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 d;
  asm("{.reg .b64 A, B, D;\n\tmov.b64 A, {%2, %3};\n\tmov.b64 B, {%4, %5};\n\t"
      "add.f32x2 D, A, B;\n\tmov.b64 {%0, %1}, D;}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 d;
  asm("{.reg .b64 A, B, D;\n\tmov.b64 A, {%2, %3};\n\tmov.b64 B, {%4, %5};\n\t"
      "sub.f32x2 D, A, B;\n\tmov.b64 {%0, %1}, D;}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// ex2_poly on two lanes with packed arithmetic (same polynomial and reduction).
__device__ __forceinline__ f2 ex2_poly2(f2 x) {
  const f2 magic{12582912.0f, 12582912.0f};
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const f2 t = add2(x, magic);
  const f2 f = sub2(x, sub2(t, magic));
  f2 p = fma2(f2{0.0551716648f, 0.0551716648f}, f, f2{0.2426111251f, 0.2426111251f});
  p = fma2(p, f, f2{0.6932609677f, 0.6932609677f});
  p = fma2(p, f, f2{0.9999280572f, 0.9999280572f});
  return f2{__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
            __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23))};
}

// Q/K/V tensor maps are 4-D {d (128), head, token, batch} with a box of
// {64, 1, 128, 1}: one 64-column half of a 128-row tile, 128-byte swizzled.
__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int head, int row0,
                                          int batch) {
  tma_load_4d(dst, map, bar, 0, head, row0, batch);
  tma_load_4d(dst + HALF_BYTES, map, bar, 64, head, row0, batch);
}

template <bool OUT_E4M3>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedState st;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (smem_base - smem_u32(smem_raw));
  // [Q0][Q1][K stage 0][K stage 1][V stage 0][V stage 1], TILE_BYTES each
  uint8_t* q_tiles = smem;
  uint8_t* k_tiles = smem + NQ * TILE_BYTES;
  uint8_t* v_tiles = smem + (NQ + STAGES) * TILE_BYTES;

  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  const int q_block0 = blockIdx.x * (NQ * BQ);
  const int nkv = (p.L + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(&st.q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&st.k_full[s], 1);
      mbar_init(&st.k_empty[s], 1);
      mbar_init(&st.v_full[s], 1);
      mbar_init(&st.v_empty[s], 1);
    }
    for (int q = 0; q < NQ; ++q) {
      mbar_init(&st.s_full[q], 1);
      mbar_init(&st.p_full[q], 128);
      mbar_init(&st.o_done[q], 1);
    }
    mbar_init(&st.drained, 1);
    st.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&st.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = st.tmem_base;
  volatile int* abort = &st.abort;

  if (warp < 4) {
    reg_dealloc<kRegsProducer>();
    if (warp == 0 && elect_one()) {
      // ---------------------------------------------------------- TMA producer
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_arrive_expect_tx(&st.q_full, NQ * TILE_BYTES);
      for (int q = 0; q < NQ; ++q) load_tile(q_tiles + q * TILE_BYTES, &tq, &st.q_full, head, q_block0 + q * BQ, batch);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&st.k_empty[s], ph ^ 1u, abort)) { ok = false; break; }
        mbar_arrive_expect_tx(&st.k_full[s], TILE_BYTES);
        load_tile(k_tiles + s * TILE_BYTES, &tk, &st.k_full[s], head, j * BKV, batch);
        if (!mbar_wait(&st.v_empty[s], ph ^ 1u, abort)) { ok = false; issued = 2 * j + 1; break; }
        mbar_arrive_expect_tx(&st.v_full[s], TILE_BYTES);
        load_tile(v_tiles + s * TILE_BYTES, &tv, &st.v_full[s], head, j * BKV, batch);
        issued = 2 * j + 2;
      }
      if (!ok) {
        // let the copies already in flight land before the CTA exits
        mbar_wait(&st.q_full, 0, nullptr);
        const int last_j = (issued - 1) / 2;
        for (int j = last_j; j >= 0 && j > last_j - STAGES; --j) {
          const int s = j % STAGES;
          const uint32_t ph = (j / STAGES) & 1;
          mbar_wait(&st.k_full[s], ph, nullptr);
          if (2 * j + 1 < issued) mbar_wait(&st.v_full[s], ph, nullptr);
        }
      }
    } else if (warp == 1 && elect_one()) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_qk = make_idesc(1, 1, 0, 0, BQ, BKV);  // bf16, K-major A and B
      constexpr uint32_t idesc_pv = make_idesc(1, 1, 0, 1, BQ, HD);   // bf16, V is MN-major
      const uint32_t q_addr = smem_u32(q_tiles);
      const uint32_t k_addr = smem_u32(k_tiles);
      const uint32_t v_addr = smem_u32(v_tiles);
      bool ok = mbar_wait(&st.q_full, 0, abort);
      auto issue_s = [&](int q, int s) {
        const uint32_t qa = q_addr + q * TILE_BYTES;
        const uint32_t ka = k_addr + s * TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
          mma_f16_ss(tmem + q * 128, make_sdesc_sw128(qa + off, 16, 1024), make_sdesc_sw128(ka + off, 16, 1024),
                     idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(&st.s_full[q]);
      };
      auto issue_pv = [&](int q, int s, bool accumulate, bool last) {
        const uint32_t va = v_addr + s * TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          mma_f16_ts(tmem + 256 + q * 128, tmem + q * 128 + kk * 8, make_sdesc_sw128(va + kk * 2048, HALF_BYTES, 1024),
                     idesc_pv, (accumulate || kk > 0) ? 1u : 0u);
        }
        if (last) mma_commit(&st.o_done[q]);  // O_q is final once this fires
      };
      if (ok && mbar_wait(&st.k_full[0], 0, abort)) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        mma_commit(&st.k_empty[0]);
      } else {
        ok = false;
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        const int sn = (j + 1) % STAGES;
        const uint32_t phn = ((j + 1) / STAGES) & 1;
        const bool has_next = j + 1 < nkv;
        if (!mbar_wait(&st.v_full[s], ph, abort) || !mbar_wait(&st.p_full[0], j & 1, abort)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, s, j > 0, !has_next);
        if (has_next) {
          if (!mbar_wait(&st.k_full[sn], phn, abort)) { ok = false; break; }
          tc_fence_after();
          issue_s(0, sn);
        }
        if (!mbar_wait(&st.p_full[1], j & 1, abort)) { ok = false; break; }
        tc_fence_after();
        issue_pv(1, s, j > 0, !has_next);
        mma_commit(&st.v_empty[s]);
        if (has_next) {
          issue_s(1, sn);
          mma_commit(&st.k_empty[sn]);
        }
      }
      mma_commit(&st.drained);
      mbar_wait(&st.drained, 0, nullptr);
    }
  } else {
    reg_alloc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax + epilogue
    const int q = (warp - 4) >> 2;            // Q tile of this warpgroup
    const uint32_t quarter = warp & 3;        // TMEM lane quarter of this warp
    const int row = quarter * 32 + lane;      // row within the Q tile
    const uint32_t lane_off = (quarter * 32u) << 16;
    const uint32_t s_tmem = tmem + lane_off + q * 128;
    const uint32_t o_tmem = tmem + lane_off + 256 + q * 128;
    const float c = p.scale_log2;
    float m_run = -INFINITY;  // running max, already multiplied by c
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait(&st.s_full[q], j & 1, abort)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[128];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld32(s_tmem + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[cc * 32]));
      tmem_ld_wait();
      float* sf = reinterpret_cast<float*>(sr);
      const int kv_valid = p.L - j * BKV;
      if (kv_valid < BKV) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= kv_valid) sf[i] = -INFINITY;
      }
      float mx = fmaxf(sf[0], sf[127]);
#pragma unroll
      for (int i = 1; i < 127; i += 2) mx = max3(mx, sf[i], sf[i + 1]);
      const float m_tile = mx * c;
      float m_use = m_run;
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_use = m_tile;
      } else if (m_tile > m_run + kRescaleThreshold) {
        m_use = m_tile;
        alpha = ex2(m_run - m_tile);
        rescale = true;
      }
      f2 rowsum2{0.f, 0.f};
      const f2 c2{c, c};
      const f2 negm{-m_use, -m_use};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t pk[16];
        const bool poly = (kPolyChunkMask >> cc) & 1u;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const f2 a = fma2(f2{sf[cc * 32 + 2 * i], sf[cc * 32 + 2 * i + 1]}, c2, negm);
          const f2 pr = poly ? ex2_poly2(a) : f2{ex2(a.x), ex2(a.y)};
          rowsum2 = add2(rowsum2, pr);
          __nv_bfloat162 b2 = __floats2bfloat162_rn(pr.x, pr.y);
          pk[i] = *reinterpret_cast<uint32_t*>(&b2);
        }
        // P chunk cc -> TMEM columns [16cc, 16cc+16) of S_q (all of S is already in registers)
        tmem_st16(s_tmem + cc * 16, pk);
      }
      const float rowsum = rowsum2.x + rowsum2.y;
      l_run = l_run * alpha + rowsum;
      m_run = m_use;
      if (__any_sync(0xffffffffu, rescale)) {
        // O already holds PV(j-1): S_q(j) was issued after PV_q(j-1), and the commit that
        // fired s_full tracks every tcgen05 operation issued before it.
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t orr[32];
          tmem_ld32(o_tmem + cc * 32, orr);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
          tmem_st32(o_tmem + cc * 32, orr);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&st.p_full[q]);
    }
    if (ok && mbar_wait(&st.o_done[q], 0, abort)) {
      tc_fence_after();
      const int token = q_block0 + q * BQ + row;
      const float inv_l = 1.f / l_run;
      float qs = 0.f, qr = 0.f;
      if (OUT_E4M3) {
        qs = __ldg(p.out_scale);
        qr = __frcp_rn(qs);
      }
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t orr[32];
        tmem_ld32(o_tmem + cc * 32, orr);
        tmem_ld_wait();
        if (token < p.L) {
          const int64_t base = static_cast<int64_t>(batch) * p.out_stride_b +
                               static_cast<int64_t>(token) * p.out_stride_t + static_cast<int64_t>(head) * HD +
                               cc * 32;
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(orr[v8 * 8 + i]) * inv_l;
            const uint4 packed = pack8(f);
            if (OUT_E4M3) {
              float fb[8];
              unpack8(packed, fb);
              *reinterpret_cast<uint2*>(p.out_q + base + v8 * 8) = quant8<__nv_bfloat16, kQuantTorch>(fb, qs, qr);
            } else {
              *reinterpret_cast<uint4*>(p.out + base + v8 * 8) = packed;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace fmha
}  // namespace ogx
