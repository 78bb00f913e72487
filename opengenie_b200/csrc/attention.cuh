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
      float mx = fmaxf(sf[0], sf[63]);
#pragma unroll
      for (int i = 1; i < 63; i += 2) mx = max3(mx, sf[i], sf[i + 1]);
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

}  // namespace attn
}  // namespace ogx
