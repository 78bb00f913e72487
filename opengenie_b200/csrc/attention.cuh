// Dense bidirectional attention, head_dim 128, bf16 in / fp32 softmax and
// accumulation / bf16 (or e4m3) out, on the 5th-generation tensor cores:
//   O[b, t, h, :] = softmax(Q[b, t, h, :] . K[b, :, h, :]^T * scale) V[b, :, h, :]
// This is the contract of the reference's attention backends
// (benchmarks/official_ltx23_benchmark.py:3289-3373: q/k/v [B, L, H*d] viewed
// [B, L, H, d], scale d^-0.5, no mask).  Keys and values may come from a
// sequence of another length (the text cross-attention: queries from the video
// tokens, keys/values from the prompt context; the backend views k and v as
// [b, -1, heads, d], :3305).
//
// One CTA per (256-query block, head, batch), 12 warps:
//   warp 0        TMA producer: Q (2 tiles x 128 rows, once), then K and V
//                 tiles of 64 keys through 4-deep rings (128-byte swizzle)
//   warp 1        MMA issuer:   S_q = Q_q K^T (tcgen05 kind::f16, M=128 N=64,
//                 both operands in shared memory) and O_q += P_q V (M=128
//                 N=128, P read straight from TMEM, V an MN-major operand)
//   warps 4..7    softmax for Q tile 0; warps 8..11 for Q tile 1.  Each thread
//                 owns one query row: it reads 64 scores from TMEM, keeps a
//                 running max/sum, writes P (bf16) back over the consumed
//                 scores, rescales its O row when the max grew by more than 2^8,
//                 and finally normalises O and stores it.
// TMEM (512 columns): O0 [0,128) O1 [128,256), then two 64-column score
// buffers per Q tile: S0 [256,320) [320,384), S1 [384,448) [448,512); P of a
// key tile occupies the first 32 columns of its score buffer.  With two score
// buffers per tile the MMA issues S_q(j+2) right after PV_q(j), so the scores
// of the next key tile are ready while the softmax of the current one runs and
// the softmax, not the MMA chain, sets each tile's pace.  tcgen05.mma
// operations issued by one thread execute in order, which makes writing
// S_q(j+2) over P_q(j) safe.
#pragma once

#include "ogx_sm100.cuh"
#include "elementwise.cuh"

namespace ogx {
namespace attn {

constexpr int HD = 128;
constexpr int BQ = 128;
constexpr int NQ = 2;
constexpr int BKV = 64;
constexpr int KV_STAGES = 4;
constexpr int Q_HALF_BYTES = BQ * 64 * 2;      // 64-column half of a 128-row Q tile
constexpr int Q_TILE_BYTES = 2 * Q_HALF_BYTES;
constexpr int KV_HALF_BYTES = BKV * 64 * 2;    // 64-column half of a 64-row K/V tile
constexpr int KV_TILE_BYTES = 2 * KV_HALF_BYTES;
constexpr int SMEM_BYTES = NQ * Q_TILE_BYTES + 2 * KV_STAGES * KV_TILE_BYTES + 1024;
constexpr int kThreads = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TMEM_O = 0;      // + 128 * q
constexpr uint32_t TMEM_S = 256;    // + 128 * q + 64 * buffer
// A row's running max only moves when a new score exceeds it by more than
// this many log2 units, so P <= 2^8 and most key tiles need no O rescale.
constexpr float kRescaleThreshold = 8.0f;
// Register split (setmaxnreg): the kernel is launched with kLaunchRegs per thread (the host checks the
// built count before launching); warpgroup 0 (TMA / MMA) drops to kRegsProducer and the two softmax
// warpgroups rise to kRegsSoftmax.  The split must fit in what the launch reserved, or the increase
// would wait forever: 128 * 96 + 256 * 200 = 63488 <= 384 * 168 = 64512.
constexpr int kLaunchRegs = 168;
constexpr uint32_t kRegsProducer = 96;
constexpr uint32_t kRegsSoftmax = 200;
static_assert(128 * kRegsProducer + 256 * kRegsSoftmax <= kThreads * kLaunchRegs, "register split exceeds the launch");

struct Params {
  int L;             // query tokens
  int L_kv;          // key/value tokens (== L for self-attention)
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* out;  // bf16 output (when out_q is null)
  uint8_t* out_q;      // e4m3 output (quantised with *out_scale, torch-path semantics)
  const float* out_scale;
  int64_t out_stride_b, out_stride_t;  // elements; the head stride is 128
  // e4m3 output to other GPUs (sequence-parallel exchange): when peer_tokens > 0,
  // token t's row goes to out_peer[t / peer_tokens] + (t % peer_tokens) * out_stride_t
  // over NVLink instead of out_q.
  uint8_t* out_peer[8];
  int peer_tokens;
};

struct SharedState {
  uint64_t q_full;
  uint64_t k_full[KV_STAGES], k_empty[KV_STAGES];
  uint64_t v_full[KV_STAGES], v_empty[KV_STAGES];
  uint64_t s_full[NQ][2];  // scores of tile q in buffer b are in TMEM
  uint64_t p_full[NQ][2];  // P of tile q in buffer b is in TMEM (128 softmax threads arrive)
  uint64_t o_ready[NQ];    // completes once per PV_q(j)
  uint64_t o_done[NQ];     // the last PV_q completed
  uint64_t drained;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x on the FMA pipe (two lanes), for the share of the exponentials the MUFU
// unit cannot absorb at tensor-core rate.  x = j + f with j = round(x) taken
// from the bits of x + 1.5*2^23 and f in [-1/2, 1/2]; 2^f by a degree-3
// polynomial fitted here to 2^f on [-1/2, 1/2] (least squares on Chebyshev
// nodes with Lawson reweighting towards minimax; max relative error 7.5e-5, far
// below bf16's 2^-9); 2^j is added to the exponent field.  x is clamped at -126
// (P rounds to 0 there).
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

// The same 2^x for one lane, in scalar instructions whose constants are immediates: no registers held for
// them across a loop that keeps a whole row of scores live.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = x + 12582912.0f;
  const float f = x - (t - 12582912.0f);
  float p = fmaf(0.0551716648f, f, 0.2426111251f);
  p = fmaf(p, f, 0.6932609677f);
  p = fmaf(p, f, 0.9999280572f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Which 16-column chunks of a 64-score row use the polynomial instead of the MUFU ex2.
constexpr uint32_t kPolyChunkMask = 0x8u;

// Q/K/V tensor maps are 4-D {d (128), head, token, batch}; a box is one
// 64-column half of a row tile (128 rows for Q, 64 for K/V), 128-byte swizzled.
__device__ __forceinline__ void load_rows(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int half_bytes, int head,
                                          int row0, int batch) {
  tma_load_4d(dst, map, bar, 0, head, row0, batch);
  tma_load_4d(dst + half_bytes, map, bar, 64, head, row0, batch);
}

template <bool OUT_E4M3>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, Params p) {
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedState st;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (smem_base - smem_u32(smem_raw));
  // [Q0][Q1][K stages][V stages]
  uint8_t* q_tiles = smem;
  uint8_t* k_tiles = smem + NQ * Q_TILE_BYTES;
  uint8_t* v_tiles = k_tiles + KV_STAGES * KV_TILE_BYTES;

  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  const int q_block0 = blockIdx.x * (NQ * BQ);
  const int nkv = (p.L_kv + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(&st.q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&st.k_full[s], 1);
      mbar_init(&st.k_empty[s], 1);
      mbar_init(&st.v_full[s], 1);
      mbar_init(&st.v_empty[s], 1);
    }
    for (int q = 0; q < NQ; ++q) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&st.s_full[q][b], 1);
        mbar_init(&st.p_full[q][b], 128);
      }
      mbar_init(&st.o_ready[q], 1);
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
  pdl_wait();  // everything above touches only this CTA's shared memory and TMEM
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
      mbar_arrive_expect_tx(&st.q_full, NQ * Q_TILE_BYTES);
      for (int q = 0; q < NQ; ++q)
        load_rows(q_tiles + q * Q_TILE_BYTES, &tq, &st.q_full, Q_HALF_BYTES, head, q_block0 + q * BQ, batch);
      int issued = 0;  // K/V tile loads issued (K of tile j is 2j, V is 2j+1)
      for (int j = 0; j < nkv; ++j) {
        const int s = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        if (!mbar_wait(&st.k_empty[s], ph ^ 1u, abort)) break;
        mbar_arrive_expect_tx(&st.k_full[s], KV_TILE_BYTES);
        load_rows(k_tiles + s * KV_TILE_BYTES, &tk, &st.k_full[s], KV_HALF_BYTES, head, j * BKV, batch);
        ++issued;
        if (!mbar_wait(&st.v_empty[s], ph ^ 1u, abort)) break;
        mbar_arrive_expect_tx(&st.v_full[s], KV_TILE_BYTES);
        load_rows(v_tiles + s * KV_TILE_BYTES, &tv, &st.v_full[s], KV_HALF_BYTES, head, j * BKV, batch);
        ++issued;
      }
      if (*abort) {
        // let the copies already in flight land before the CTA exits
        mbar_wait(&st.q_full, 0, nullptr);
        const int last_j = (issued - 1) / 2;
        for (int j = last_j; j >= 0 && j > last_j - KV_STAGES; --j) {
          const int s = j % KV_STAGES;
          const uint32_t ph = (j / KV_STAGES) & 1;
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
      auto issue_s = [&](int q, int j) {  // S_q(j) into score buffer j % 2
        const uint32_t qa = q_addr + q * Q_TILE_BYTES;
        const uint32_t ka = k_addr + (j % KV_STAGES) * KV_TILE_BYTES;
        const uint32_t d = tmem + TMEM_S + q * 128 + (j & 1) * 64;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t qoff = (kk >> 2) * Q_HALF_BYTES + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * KV_HALF_BYTES + (kk & 3) * 32;
          mma_f16_ss(d, make_sdesc_sw128(qa + qoff, 16, 1024), make_sdesc_sw128(ka + koff, 16, 1024), idesc_qk,
                     kk > 0 ? 1u : 0u);
        }
        mma_commit(&st.s_full[q][j & 1]);
      };
      auto issue_pv = [&](int q, int j) {  // O_q += P_q(j) V(j)
        const uint32_t va = v_addr + (j % KV_STAGES) * KV_TILE_BYTES;
        const uint32_t pa = tmem + TMEM_S + q * 128 + (j & 1) * 64;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          mma_f16_ts(tmem + TMEM_O + q * 128, pa + kk * 8, make_sdesc_sw128(va + kk * 2048, KV_HALF_BYTES, 1024),
                     idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&st.o_ready[q]);
        if (j + 1 == nkv) mma_commit(&st.o_done[q]);
      };
      bool ok = mbar_wait(&st.q_full, 0, abort);
      // prologue: the scores of key tiles 0 and 1
      for (int j = 0; j < 2 && j < nkv && ok; ++j) {
        const int s = j % KV_STAGES;
        if (!mbar_wait(&st.k_full[s], (j / KV_STAGES) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        issue_s(0, j);
        issue_s(1, j);
        mma_commit(&st.k_empty[s]);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        const uint32_t pph = (j >> 1) & 1;
        const int j2 = j + 2;
        const int s2 = j2 % KV_STAGES;
        if (!mbar_wait(&st.v_full[s], ph, abort) || !mbar_wait(&st.p_full[0][j & 1], pph, abort)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, j);
        if (j2 < nkv) {
          if (!mbar_wait(&st.k_full[s2], (j2 / KV_STAGES) & 1, abort)) { ok = false; break; }
          tc_fence_after();
          issue_s(0, j2);
        }
        if (!mbar_wait(&st.p_full[1][j & 1], pph, abort)) { ok = false; break; }
        tc_fence_after();
        issue_pv(1, j);
        mma_commit(&st.v_empty[s]);
        if (j2 < nkv) {
          issue_s(1, j2);
          mma_commit(&st.k_empty[s2]);
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
    const uint32_t o_tmem = tmem + lane_off + TMEM_O + q * 128;
    const float c = p.scale_log2;
    float m_run = -INFINITY;  // running max, already multiplied by c
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int b = j & 1;
      const uint32_t s_tmem = tmem + lane_off + TMEM_S + q * 128 + b * 64;
      if (!mbar_wait(&st.s_full[q][b], (j >> 1) & 1, abort)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32(s_tmem, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_ld32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tmem_ld_wait();
      float* sf = reinterpret_cast<float*>(sr);
      const int kv_valid = p.L_kv - j * BKV;
      if (kv_valid < BKV) {
#pragma unroll
        for (int i = 0; i < BKV; ++i)
          if (i >= kv_valid) sf[i] = -INFINITY;
      }
      // row max: four independent chains of 3-input max (a single chain would put 31 dependent max
      // operations on the path from the scores to P)
      float mq[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float m = fmaxf(sf[h * 16], sf[h * 16 + 15]);
#pragma unroll
        for (int i = 1; i < 15; i += 2) m = max3(m, sf[h * 16 + i], sf[h * 16 + i + 1]);
        mq[h] = m;
      }
      float mx = max3(fmaxf(mq[0], mq[1]), mq[2], mq[3]);
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
        uint32_t pk[8];
        const bool poly = (kPolyChunkMask >> cc) & 1u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const f2 a = fma2(f2{sf[cc * 16 + 2 * i], sf[cc * 16 + 2 * i + 1]}, c2, negm);
          const f2 pr = poly ? ex2_poly2(a) : f2{ex2(a.x), ex2(a.y)};
          rowsum2 = add2(rowsum2, pr);
          pk[i] = pack_bf16x2(pr.x, pr.y);
        }
        // P chunk cc -> TMEM columns [8cc, 8cc+8) of this score buffer (all scores are in registers)
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(s_tmem + cc * 8),
            "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3]), "r"(pk[4]), "r"(pk[5]), "r"(pk[6]), "r"(pk[7])
            : "memory");
      }
      l_run = l_run * alpha + (rowsum2.x + rowsum2.y);
      m_run = m_use;
      if (__any_sync(0xffffffffu, rescale)) {
        // O must hold PV_q(j-1) before it is rescaled.  o_ready completes once per PV_q; S_q(j) was
        // issued after PV_q(j-2), so it is at most one phase behind phase j-1 here.
        if (!mbar_wait(&st.o_ready[q], (j - 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int oc = 0; oc < 4; ++oc) {
          uint32_t orr[32];
          tmem_ld32(o_tmem + oc * 32, orr);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
          tmem_st32(o_tmem + oc * 32, orr);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&st.p_full[q][b]);
    }
    if (ok && mbar_wait(&st.o_done[q], 0, abort)) {
      tc_fence_after();
      const int token = q_block0 + q * BQ + row;
      const float inv_l = 1.f / l_run;
      if constexpr (OUT_E4M3) {
        // e4m3 rows are 128 bytes.  Each thread owns one row, so storing straight from registers
        // would scatter 32 rows per instruction; instead the warp stages its 32 quantised rows in
        // its quarter of this Q tile's shared memory (idle now: every S_q MMA completed before
        // o_done) with 16-byte granules XOR-swizzled by row (conflict-free both ways), then stores
        // whole rows, 8 lanes per row and 4 rows per instruction.  Full-line stores are what makes
        // the peer path (NVLink) efficient.
        const float qs = __ldg(p.out_scale);
        const float qr = __frcp_rn(qs);
        uint8_t* stage = q_tiles + q * Q_TILE_BYTES + quarter * 4096u;
#pragma unroll 1
        for (int oc = 0; oc < 4; ++oc) {
          uint32_t orr[32];
          tmem_ld32(o_tmem + oc * 32, orr);
          tmem_ld_wait();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint2 half[2];
#pragma unroll
            for (int v8 = 0; v8 < 2; ++v8) {
              float f[8], fb[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(orr[h * 16 + v8 * 8 + i]) * inv_l;
              unpack8(pack8(f), fb);  // the attention output is bf16 before it is quantised
              half[v8] = quant8<__nv_bfloat16, kQuantTorch>(fb, qs, qr);
            }
            const uint32_t gi = static_cast<uint32_t>(oc * 2 + h);
            *reinterpret_cast<uint4*>(stage + lane * 128u + ((gi ^ (lane & 7u)) << 4)) =
                make_uint4(half[0].x, half[0].y, half[1].x, half[1].y);
          }
        }
        __syncwarp();
        const uint32_t g = lane & 7u;
#pragma unroll
        for (int s8 = 0; s8 < 8; ++s8) {
          const uint32_t r = static_cast<uint32_t>(s8 * 4) + (lane >> 3);
          const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128u + ((g ^ (r & 7u)) << 4));
          const int tok = q_block0 + q * BQ + static_cast<int>(quarter * 32u + r);
          if (tok < p.L) {
            uint8_t* dst;
            if (p.peer_tokens > 0) {
              const int d = tok / p.peer_tokens;
              // constant-index selects: a runtime index into the parameter array would copy it to local memory
              uint8_t* peer = p.out_peer[0];
#pragma unroll
              for (int i = 1; i < 8; ++i) peer = (d == i) ? p.out_peer[i] : peer;
              dst = peer + static_cast<int64_t>(tok - d * p.peer_tokens) * p.out_stride_t;
            } else {
              dst = p.out_q + static_cast<int64_t>(batch) * p.out_stride_b + static_cast<int64_t>(tok) * p.out_stride_t;
            }
            *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(head) * HD + g * 16u) = v;
          }
        }
      } else {
#pragma unroll 1
        for (int oc = 0; oc < 4; ++oc) {
          uint32_t orr[32];
          tmem_ld32(o_tmem + oc * 32, orr);
          tmem_ld_wait();
          if (token < p.L) {
            const int64_t base = static_cast<int64_t>(batch) * p.out_stride_b +
                                 static_cast<int64_t>(token) * p.out_stride_t + static_cast<int64_t>(head) * HD +
                                 oc * 32;
#pragma unroll
            for (int v8 = 0; v8 < 4; ++v8) {
              float f[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(orr[v8 * 8 + i]) * inv_l;
              *reinterpret_cast<uint4*>(p.out + base + v8 * 8) = pack8(f);
            }
          }
        }
      }
    }
  }

  if (OUT_E4M3 && p.peer_tokens > 0) __threadfence_system();  // peer stores visible before any signal
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------------
// CTA-pair attention.  The single-CTA kernel above runs 64-key score MMAs (M=128, N=64, K=128) that read
// the whole 32 KB Q tile and a 16 KB K tile from shared memory per 256 tensor-core cycles: 192 B per cycle
// against the SM's 128, so the tensor pipe waits on shared memory.  Here two CTAs of a cluster run each
// MMA together (tcgen05 cta_group::2, M=256): each CTA holds its own 128 query rows of the pair's 256-row
// Q tile and half of each 128-key tile's operand (K: 64 keys x 128 d; V: 128 keys x 64 d), the pair's
// first CTA issues M=256, N=128 MMAs that read both CTAs' shared memory, and each CTA receives its rows of
// S and O in its own TMEM.  Per SM that is 96 B per tensor-core cycle for the score MMAs and 32 B for P.V.
//
// The softmax is the other bound: 2^x runs on the MUFU at 4 lanes per cycle per SM sub-partition, so the
// 128 x 128 exponentials of a key tile (three quarters on the MUFU, one quarter as a polynomial on the FMA
// pipe) take ~770 cycles per sub-partition against ~1024 tensor cycles, and the score loads, row max and
// handoffs around them add a few hundred more.  Two softmax warp groups therefore split the key tiles:
// group 0 takes the even tiles, group 1 the odd ones, each with its own score buffer, running max, row sum
// and O accumulator in TMEM; the two partial results are merged once, in the epilogue.  Nothing ties the
// groups together inside the key loop, so on each sub-partition one group's loads and row max overlap the
// other group's exponentials, and the tensor pipe alternates between the groups' tiles.
//
// Per CTA, 10 warps:
//   warps 0..7  softmax + epilogue: warps 0..3 are group 0, warps 4..7 group 1.  A thread owns one query
//               row and holds its 128 scores of a key tile in registers (a warp may only touch its TMEM
//               lane quarter, warp % 4).
//   warp 8      TMA: its Q rows once, then its K and V halves of every key tile (plain cta_group::2 loads
//               into its own shared memory, completion counted on the first CTA's barrier)
//   warp 9      TMEM allocation; (first CTA) MMA issuer for the pair: S(j) = Q K^T and O_g += P(j) V
// TMEM per CTA: O of group g at [128g, 128g+128), S of group g at [256+128g, 384+128g).  P(j) (bf16) goes to
// the first 64 columns of its group's S buffer, over scores its threads hold in registers.  S(j+2) goes to
// the buffer PV(j) has just read; it is issued right behind PV(j) and, in the tensor pipe's order,
// completes after it, so a thread that sees S(j) complete may rescale its group's O at once.
constexpr int PBKV = 128;                       // keys per tile
constexpr int P_STAGES = 5;
constexpr int PQ_TILE_BYTES = 2 * Q_HALF_BYTES;  // this CTA's 128 rows x 128 d
constexpr int PK_HALF_BYTES = 64 * 64 * 2;       // 64 keys x 64 d (one 128-byte column half)
constexpr int PK_BYTES = 2 * PK_HALF_BYTES;      // this CTA's 64 keys x 128 d
constexpr int PV_BYTES = PBKV * 64 * 2;          // 128 keys x this CTA's 64 d
constexpr int PAIR_SMEM_BYTES = PQ_TILE_BYTES + P_STAGES * (PK_BYTES + PV_BYTES) + 1024;
constexpr int kPairThreads = 320;
constexpr uint32_t kPairTmaWarp = 8;
constexpr uint32_t kPairMmaWarp = 9;
constexpr uint32_t PTMEM_O = 0;    // + 128 * group
constexpr uint32_t PTMEM_S = 256;  // + 128 * group

struct PairShared {
  uint64_t q_full;                             // first CTA: both CTAs' Q bytes
  uint64_t k_full[P_STAGES], v_full[P_STAGES];  // first CTA: both CTAs' halves
  uint64_t k_empty[P_STAGES], v_empty[P_STAGES];
  uint64_t s_full[2];  // S(j) in group j % 2's buffer complete (both CTAs, committed by the first)
  uint64_t p_full[2];  // first CTA: P(j) written, one arrival per warp of group j % 2 in both CTAs (8)
  uint64_t s_read[2];  // first CTA (split scores): S(j) loaded into registers by group j % 2 (8 arrivals)
  uint64_t o_done;     // the last PV complete (both CTAs)
  uint64_t drained;
  float red[2][2][128];  // [group][running max, row sum][row]: the partial results the epilogue merges
  uint32_t tmem_base;
  int abort;
};
static_assert(PAIR_SMEM_BYTES + sizeof(PairShared) <= 232448, "pair attention shared memory");

// Which 16-column chunks of a 128-score row use the polynomial exp2 instead of the MUFU ex2 (1 of 8): the
// last, when most of the scores are spent and the polynomial has registers to work in.
constexpr uint32_t kPairPolyChunkMask = 0x80u;

// Split scores (SPLIT_S): each S(j) is two N=64 MMAs.  With cta_group::2 each CTA supplies half of the
// N keys, so the first MMA (S_lo, TMEM columns [0, 64)) covers keys [0, 32) and [64, 96) of the tile (the
// first 32 of each CTA's 64) and the second (S_hi, columns [64, 128)) keys [32, 64) and [96, 128): column c
// holds key c with bits 5 and 6 swapped.  P(j) goes to columns [64, 128) of the group's buffer, so S_lo(j+2)
// is issued as soon as the group has loaded S(j) into registers, while its exponentials run; only
// PV(j) and S_hi(j+2) then stand between P(j) and the group's next scores.
__host__ __device__ constexpr int split_key_of_col(int c) { return (c & ~0x60) | ((c & 0x20) << 1) | ((c & 0x40) >> 1); }

template <bool OUT_E4M3, bool SPLIT_S>
__global__ void __launch_bounds__(kPairThreads, 1)
    attn_fwd_pair_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, Params p) {
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  __shared__ PairShared st;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (smem_base - smem_u32(smem_raw));
  // [Q][K stages][V stages]
  uint8_t* q_tile = smem;
  uint8_t* k_tiles = smem + PQ_TILE_BYTES;
  uint8_t* v_tiles = k_tiles + P_STAGES * PK_BYTES;

  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();  // 0: the pair's first CTA (issues the MMAs)
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  const int q_block0 = static_cast<int>(blockIdx.x >> 1) * (2 * BQ);  // 256 queries per pair
  const int row0 = q_block0 + static_cast<int>(crank) * BQ;           // this CTA's first query row
  const int nkv = (p.L_kv + PBKV - 1) / PBKV;

  if (threadIdx.x == 0) {
    mbar_init(&st.q_full, 1);
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&st.k_full[s], 1);
      mbar_init(&st.v_full[s], 1);
      mbar_init(&st.k_empty[s], 1);
      mbar_init(&st.v_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&st.s_full[g], 1);
      mbar_init(&st.p_full[g], 8);
      mbar_init(&st.s_read[g], 8);
    }
    mbar_init(&st.o_done, 1);
    mbar_init(&st.drained, 1);
    st.abort = 0;
    fence_mbar_init();
  }
  if (warp == kPairMmaWarp) {
    tmem_alloc_pair(&st.tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  pdl_wait();  // everything above touches only this CTA's shared memory and TMEM
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
  tc_fence_after();
  const uint32_t tmem = st.tmem_base;
  volatile int* abort = &st.abort;
  const uint32_t peer_abort = cluster_addr(&st.abort, crank ^ 1u);
  auto abort_pair = [&]() {  // this CTA stops; tell the peer CTA too
    *abort = 1;
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1u) : "memory");
  };

  if (warp == kPairTmaWarp) {
    if (elect_one()) {
      // ---------------------------------------------------------- TMA producer (both CTAs)
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      const uint32_t qf = cluster_addr(&st.q_full, 0);
      if (crank == 0) mbar_arrive_expect_tx(&st.q_full, 2 * PQ_TILE_BYTES);
      tma_load_4d_pair(q_tile, &tq, qf, 0, head, row0, batch);
      tma_load_4d_pair(q_tile + Q_HALF_BYTES, &tq, qf, 64, head, row0, batch);
      int issued = 0;  // K/V tile loads issued (K of tile j is 2j, V is 2j+1)
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % P_STAGES;
        const uint32_t ph = (j / P_STAGES) & 1;
        if (!mbar_wait(&st.k_empty[s], ph ^ 1u, abort)) { ok = false; break; }
        if (crank == 0) mbar_arrive_expect_tx(&st.k_full[s], 2 * PK_BYTES);
        const uint32_t kf = cluster_addr(&st.k_full[s], 0);
        const int key0 = j * PBKV + static_cast<int>(crank) * 64;
        tma_load_4d_pair(k_tiles + s * PK_BYTES, &tk, kf, 0, head, key0, batch);
        tma_load_4d_pair(k_tiles + s * PK_BYTES + PK_HALF_BYTES, &tk, kf, 64, head, key0, batch);
        ++issued;
        if (!mbar_wait(&st.v_empty[s], ph ^ 1u, abort)) { ok = false; break; }
        if (crank == 0) mbar_arrive_expect_tx(&st.v_full[s], 2 * PV_BYTES);
        tma_load_4d_pair(v_tiles + s * PV_BYTES, &tv, cluster_addr(&st.v_full[s], 0), static_cast<int>(crank) * 64,
                         head, j * PBKV, batch);
        ++issued;
      }
      if (!ok) abort_pair();
      if (*abort && crank == 0) {
        // let the copies already in flight land before the pair exits (the first CTA counts both CTAs')
        mbar_wait(&st.q_full, 0, nullptr);
        const int last_j = (issued - 1) / 2;
        for (int j = last_j; j >= 0 && j > last_j - P_STAGES; --j) {
          const int s = j % P_STAGES;
          const uint32_t ph = (j / P_STAGES) & 1;
          mbar_wait(&st.k_full[s], ph, nullptr);
          if (2 * j + 1 < issued) mbar_wait(&st.v_full[s], ph, nullptr);
        }
      }
    }
  } else if (warp == kPairMmaWarp) {
    if (crank == 0 && elect_one()) {
      // ---------------------------------------------------------- MMA issuer (first CTA, for the pair)
      constexpr uint32_t idesc_qk = make_idesc(1, 1, 0, 0, 2 * BQ, PBKV);  // bf16, K-major A and B
      constexpr uint32_t idesc_qk_half = make_idesc(1, 1, 0, 0, 2 * BQ, PBKV / 2);
      constexpr uint32_t idesc_pv = make_idesc(1, 1, 0, 1, 2 * BQ, HD);    // bf16, A in TMEM, V MN-major
      // descriptors of the stage-0 operands; a stage's are these plus its byte offset / 16 (addresses stay
      // below 2^18, so the 14-bit address field never carries)
      const uint64_t q_desc = make_sdesc_sw128(smem_u32(q_tile), 16, 1024);
      const uint64_t k_desc0 = make_sdesc_sw128(smem_u32(k_tiles), 16, 1024);
      // each CTA holds one 64-column block of V (its half of N), so the block stride is unused; it is kept
      // inside the stage
      const uint64_t v_desc0 = make_sdesc_sw128(smem_u32(v_tiles), PV_BYTES / 2, 1024);
      auto both = [&](uint64_t* bar) {  // commit to the barrier in both CTAs
        mma_commit_pair(cluster_addr(bar, 0));
        mma_commit_pair(cluster_addr(bar, 1));
      };
      auto issue_s = [&](int j) {  // S(j) into group j % 2's buffer
        const uint64_t kd = k_desc0 + (((j % P_STAGES) * PK_BYTES) >> 4);
        const uint32_t d = tmem + PTMEM_S + (j & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t qoff = ((kk >> 2) * Q_HALF_BYTES + (kk & 3) * 32) >> 4;
          const uint32_t koff = ((kk >> 2) * PK_HALF_BYTES + (kk & 3) * 32) >> 4;
          mma_f16_ss_pair(d, q_desc + qoff, kd + koff, idesc_qk, kk > 0 ? 1u : 0u);
        }
        both(&st.s_full[j & 1]);
        both(&st.k_empty[j % P_STAGES]);
      };
      // split scores: half h of S(j) (keys [32h, 32h + 32) of each CTA's 64) into columns [64h, 64h + 64)
      auto issue_s_half = [&](int j, int h) {
        const uint64_t kd = k_desc0 + (((j % P_STAGES) * PK_BYTES + h * 4096) >> 4);
        const uint32_t d = tmem + PTMEM_S + (j & 1) * 128 + h * 64;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t qoff = ((kk >> 2) * Q_HALF_BYTES + (kk & 3) * 32) >> 4;
          const uint32_t koff = ((kk >> 2) * PK_HALF_BYTES + (kk & 3) * 32) >> 4;
          mma_f16_ss_pair(d, q_desc + qoff, kd + koff, idesc_qk_half, kk > 0 ? 1u : 0u);
        }
        if (h == 1) {
          both(&st.s_full[j & 1]);
          both(&st.k_empty[j % P_STAGES]);
        }
      };
      auto issue_pv = [&](int j) {  // O_g += P(j) V(j), g = j % 2; each group's first PV overwrites
        const uint64_t vd = v_desc0 + (((j % P_STAGES) * PV_BYTES) >> 4);
        const uint32_t pa = tmem + PTMEM_S + (j & 1) * 128 + (SPLIT_S ? 64 : 0);
        const uint32_t o = tmem + PTMEM_O + (j & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < PBKV / 16; ++kk) {
          // P columns [8kk, 8kk + 8) hold the scores' columns [16kk, 16kk + 16): keys of V block kk, or with
          // split scores of V block split_key_of_col(16kk) / 16
          const int vb = SPLIT_S ? split_key_of_col(16 * kk) / 16 : kk;
          mma_f16_ts_pair(o, pa + kk * 8, vd + ((vb * 2048) >> 4), idesc_pv, (j > 1 || kk > 0) ? 1u : 0u);
        }
        both(&st.v_empty[j % P_STAGES]);
        if (j + 1 == nkv) both(&st.o_done);
      };
      bool ok = mbar_wait(&st.q_full, 0, abort);
      for (int j = 0; j < 2 && j < nkv && ok; ++j) {
        if (!mbar_wait(&st.k_full[j], 0, abort)) { ok = false; break; }
        tc_fence_after();
        if constexpr (SPLIT_S) {
          issue_s_half(j, 0);
          issue_s_half(j, 1);
        } else {
          issue_s(j);
        }
      }
      for (int j = 0; j < nkv && ok && SPLIT_S; ++j) {
        // S_lo(j+2) as soon as group j % 2 holds S(j) in registers; then PV(j) and S_hi(j+2) behind it
        const int s = j % P_STAGES;
        const int j2 = j + 2;
        if (j2 < nkv) {
          if (!mbar_wait(&st.s_read[j & 1], (j >> 1) & 1, abort) ||
              !mbar_wait(&st.k_full[j2 % P_STAGES], (j2 / P_STAGES) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s_half(j2, 0);
        }
        if (!mbar_wait(&st.v_full[s], (j / P_STAGES) & 1, abort) || !mbar_wait(&st.p_full[j & 1], (j >> 1) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(j);
        if (j2 < nkv) issue_s_half(j2, 1);
      }
      for (int j = 0; j < nkv && ok && !SPLIT_S; ++j) {
        const int s = j % P_STAGES;
        if (!mbar_wait(&st.v_full[s], (j / P_STAGES) & 1, abort) || !mbar_wait(&st.p_full[j & 1], (j >> 1) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(j);
        const int j2 = j + 2;  // its scores go to the buffer PV(j) has just read
        if (j2 < nkv) {
          if (!mbar_wait(&st.k_full[j2 % P_STAGES], (j2 / P_STAGES) & 1, abort)) { ok = false; break; }
          tc_fence_after();
          issue_s(j2);
        }
      }
      if (!ok) abort_pair();
      mma_commit_pair(cluster_addr(&st.drained, 0));
      mbar_wait(&st.drained, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue (both CTAs)
    const uint32_t quarter = warp & 3;             // TMEM lane quarter of this warp
    const int g = static_cast<int>(warp >> 2);     // group: key tiles j with j % 2 == g
    const int row = static_cast<int>(quarter * 32 + lane);
    const uint32_t lane_off = (quarter * 32u) << 16;
    const uint32_t o_tmem = tmem + lane_off + PTMEM_O + g * 128;  // this group's O row
    const uint32_t s_tmem = tmem + lane_off + PTMEM_S + g * 128;  // its scores, then its P
    const float c = p.scale_log2;
    float m_run = -INFINITY;  // running max over this group's tiles, already multiplied by c
    float l_run = 0.f;        // row sum over this group's tiles
    bool ok = true;
    for (int j = g; j < nkv; j += 2) {
      if (!mbar_wait(&st.s_full[g], (j >> 1) & 1, abort)) {
        ok = false;
        abort_pair();
        break;
      }
      tc_fence_after();
      uint32_t sr[PBKV];
#pragma unroll
      for (int h = 0; h < 4; ++h) tmem_ld32(s_tmem + h * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[h * 32]));
      tmem_ld_wait();
      if constexpr (SPLIT_S) {  // the scores are in registers: S_lo(j+2) may overwrite columns [0, 64)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (crank == 0)
            mbar_arrive(&st.s_read[g]);
          else
            mbar_arrive_peer(cluster_addr(&st.s_read[g], 0));
        }
      }
      float* sf = reinterpret_cast<float*>(sr);
      const int kv_valid = p.L_kv - j * PBKV;
      if (kv_valid < PBKV) {
#pragma unroll
        for (int i = 0; i < PBKV; ++i)
          if ((SPLIT_S ? split_key_of_col(i) : i) >= kv_valid) sf[i] = -INFINITY;
      }
      // row max: eight independent chains of 3-input max, then a tree
      float mq[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        float m = fmaxf(sf[h * 16], sf[h * 16 + 15]);
#pragma unroll
        for (int i = 1; i < 15; i += 2) m = max3(m, sf[h * 16 + i], sf[h * 16 + i + 1]);
        mq[h] = m;
      }
      const float m_tile = fmaxf(max3(mq[0], mq[1], mq[2]), max3(mq[3], mq[4], max3(mq[5], mq[6], mq[7]))) * c;
      float m_use = m_run;
      float alpha = 1.f;
      bool rescale = false;
      if (j == g) {
        m_use = m_tile;
      } else if (m_tile > m_run + kRescaleThreshold) {
        m_use = m_tile;
        alpha = ex2(m_run - m_tile);
        rescale = true;
      }
      f2 rs[4] = {f2{0.f, 0.f}, f2{0.f, 0.f}, f2{0.f, 0.f}, f2{0.f, 0.f}};
      const f2 c2{c, c};
      const f2 negm{-m_use, -m_use};
#pragma unroll
      for (int cc = 0; cc < PBKV / 16; ++cc) {
        uint32_t pk[8];
        const bool poly = (kPairPolyChunkMask >> cc) & 1u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const f2 a = fma2(f2{sf[cc * 16 + 2 * i], sf[cc * 16 + 2 * i + 1]}, c2, negm);
          const f2 pr = poly ? f2{ex2_poly(a.x), ex2_poly(a.y)} : f2{ex2(a.x), ex2(a.y)};
          rs[i & 3] = add2(rs[i & 3], pr);
          pk[i] = pack_bf16x2(pr.x, pr.y);
        }
        // P chunk cc -> TMEM columns [8cc, 8cc+8) (+64 with split scores): scores this thread has already read
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(s_tmem + (SPLIT_S ? 64 : 0) + cc * 8),
            "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3]), "r"(pk[4]), "r"(pk[5]), "r"(pk[6]), "r"(pk[7])
            : "memory");
      }
      const f2 r01 = add2(rs[0], rs[1]), r23 = add2(rs[2], rs[3]);
      l_run = l_run * alpha + ((r01.x + r23.x) + (r01.y + r23.y));
      m_run = m_use;
      // O_g is rescaled after the scores are spent (fewer live registers) and before P(j) is published, so
      // before PV(j) adds to it.  S(j) was issued behind PV(j-2), this group's previous PV, and completed
      // after it: O_g is settled.
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int oc = 0; oc < 4; ++oc) {
          uint32_t orr[32];
          tmem_ld32(o_tmem + oc * 32, orr);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
          tmem_st32(o_tmem + oc * 32, orr);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (crank == 0)
          mbar_arrive(&st.p_full[g]);
        else
          mbar_arrive_peer(cluster_addr(&st.p_full[g], 0));
      }
    }
    // merge the groups: O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m)),
    // m = max(m_0, m_1); the thread of group g writes output columns [64g, 64g + 64) of its row
    st.red[g][0][row] = m_run;
    st.red[g][1][row] = l_run;
    named_bar_sync(1, 256);
    const bool two = nkv > 1;  // group 1 has key tiles (else its O was never written)
    const float m0 = st.red[0][0][row], m1 = st.red[1][0][row];
    const float m = two ? fmaxf(m0, m1) : m0;
    const float a0 = ex2(m0 - m);
    const float a1 = two ? ex2(m1 - m) : 0.f;
    const float inv_l = 1.f / (st.red[0][1][row] * a0 + st.red[1][1][row] * a1);
    const bool have_o = ok && mbar_wait(&st.o_done, 0, abort);
    if (have_o) tc_fence_after();
    const uint32_t o0 = tmem + lane_off + PTMEM_O + g * 64;  // O_0, columns [64g, 64g + 64)
    const uint32_t o1 = o0 + 128;                             // O_1, the same columns
    const float w0 = a0 * inv_l, w1 = a1 * inv_l;
    // 32 output columns [64g + 32oc, +32) as fp32
    auto merged = [&](int oc, float (&f)[32]) {
      uint32_t ra[32];
      tmem_ld32(o0 + oc * 32, ra);
      if (two) {
        uint32_t rb[32];
        tmem_ld32(o1 + oc * 32, rb);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(ra[i]) * w0 + __uint_as_float(rb[i]) * w1;
      } else {
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(ra[i]) * w0;
      }
    };
    if constexpr (OUT_E4M3) {
      // The warp quantises its 32 rows x 64 columns and stages them in the (idle) Q tile's shared memory:
      // 128-byte rows, 16-byte granules XOR-swizzled by row, both groups' columns of a row side by side;
      // after the barrier each warp stores 16 whole rows, 8 lanes per row and 4 rows per instruction.
      // Full-line stores are what makes the peer path (NVLink) efficient.
      uint8_t* stage = q_tile + quarter * 4096u;
      if (have_o) {
        const float qs = __ldg(p.out_scale);
        const float qr = __frcp_rn(qs);
#pragma unroll 1
        for (int oc = 0; oc < 2; ++oc) {
          float f[32];
          merged(oc, f);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint2 half[2];
#pragma unroll
            for (int v8 = 0; v8 < 2; ++v8) {
              float fb[8];
              unpack8(pack8(*reinterpret_cast<const float(*)[8]>(&f[h * 16 + v8 * 8])), fb);  // the attention output is bf16 before it is quantised
              half[v8] = quant8<__nv_bfloat16, kQuantTorch>(fb, qs, qr);
            }
            const uint32_t gi = static_cast<uint32_t>(g * 4 + oc * 2 + h);
            *reinterpret_cast<uint4*>(stage + lane * 128u + ((gi ^ (lane & 7u)) << 4)) =
                make_uint4(half[0].x, half[0].y, half[1].x, half[1].y);
          }
        }
      }
      named_bar_sync(1, 256);
      if (have_o) {
        const uint32_t gl = lane & 7u;
#pragma unroll
        for (int s8 = 0; s8 < 4; ++s8) {
          const uint32_t r = static_cast<uint32_t>(g * 16 + s8 * 4) + (lane >> 3);
          const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128u + ((gl ^ (r & 7u)) << 4));
          const int tok = row0 + static_cast<int>(quarter * 32u + r);
          if (tok < p.L) {
            uint8_t* dst;
            if (p.peer_tokens > 0) {
              const int d = tok / p.peer_tokens;
              // constant-index selects: a runtime index into the parameter array would copy it to local memory
              uint8_t* peer = p.out_peer[0];
#pragma unroll
              for (int i = 1; i < 8; ++i) peer = (d == i) ? p.out_peer[i] : peer;
              dst = peer + static_cast<int64_t>(tok - d * p.peer_tokens) * p.out_stride_t;
            } else {
              dst = p.out_q + static_cast<int64_t>(batch) * p.out_stride_b + static_cast<int64_t>(tok) * p.out_stride_t;
            }
            *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(head) * HD + gl * 16u) = v;
          }
        }
      }
    } else if (have_o) {
      const int token = row0 + row;
#pragma unroll 1
      for (int oc = 0; oc < 2; ++oc) {
        float f[32];
        merged(oc, f);
        if (token < p.L) {
          const int64_t base = static_cast<int64_t>(batch) * p.out_stride_b + static_cast<int64_t>(token) * p.out_stride_t +
                               static_cast<int64_t>(head) * HD + g * 64 + oc * 32;
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) *reinterpret_cast<uint4*>(p.out + base + v8 * 8) = pack8(*reinterpret_cast<const float(*)[8]>(&f[v8 * 8]));
        }
      }
    }
  }

  if (OUT_E4M3 && p.peer_tokens > 0) __threadfence_system();  // peer stores visible before any signal
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves (or frees TMEM) while the pair's MMAs may still use it
  if (warp == kPairMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

}  // namespace attn
}  // namespace ogx
