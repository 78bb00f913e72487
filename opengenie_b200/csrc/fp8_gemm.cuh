// FP8 (e4m3 x e4m3 -> fp32) GEMM on the 5th-generation tensor cores:
//   out[m, n] = epilogue( scale_a * scale_b[n / n_per_scale] * sum_k A[m, k] * W[n, k] )
// A is the quantised activation [M, K] and W the quantised weight [N, K]
// (nn.Linear layout), both K-major, which is exactly torch._scaled_mm(A, W.t()).
//
// Persistent kernel, one CTA per SM, 128x256 output tiles (PAIR = false), or
// CTA pairs (clusters of two) computing 256x256 tiles with tcgen05 cta_group::2
// (PAIR = true): each CTA of the pair loads its 128 rows of A and half (128
// rows) of the B tile, the pair's first CTA issues M=256 N=256 MMAs that read
// both CTAs' shared memory, and each CTA receives its 128 rows of the result
// in its own TMEM.  Per SM that halves the B bytes moved per FLOP, which is
// what the single-CTA tiles are short of (L2 -> shared-memory traffic and
// bytes in flight), and leaves room for a 6-deep ring.  Layout per CTA:
//   warp 0      TMA producer: A/W tiles (128-byte swizzle) into a 4-stage ring
//   warp 1      MMA issuer:   tcgen05.mma kind::f8f6f4, M=128 N=256 K=32,
//                             fp32 accumulators in TMEM (2 x 256 columns, so
//                             the epilogue of one tile overlaps the next tile)
//   warps 2..9  epilogue:     tcgen05.ld -> scale -> bf16 -> bias (-> gate +
//                             residual) -> global; two warps per TMEM lane
//                             quarter split the tile's columns, 16-byte vector
//                             loads of bias / gate / timestep / residual
// Epilogues reproduce the reference's rounding sequence:
//   EPI_BIAS:     bf16(bf16(acc*s) + bf16(bias))            (scaled_mm, then
//                 fused_bias_add_bf16, triton_ltx_ops.py:1695-1707)
//   EPI_RESIDUAL: bf16(x + bf16(bf16(bf16(acc*s) + bf16(bias)) * gate))
//                 (fp8_linear_without_bias :762-781 then
//                 fused_residual_gate_bias_from_ada :204-262)
//   EPI_GELU_QUANT: e4m3 quant(bf16(gelu(bf16(bf16(acc*s) + bf16(bias)))))
//                 (the FFN's first projection, GELU and the second
//                 projection's input quantiser: FP8Linear.forward :1695-1707,
//                 gelu(approximate="tanh"), fused_fp8_quantize_e4m3 :144-161
//                 as fp8_linear_without_bias :770-771 applies it)
#pragma once

#include "ogx_sm100.cuh"
#include "elementwise.cuh"

namespace ogx {
namespace gemm {

constexpr int BM = 128;  // A rows per CTA
constexpr int BN = 256;  // output columns per tile
constexpr int BK = 128;  // fp8 elements = bytes per row of a stage
constexpr int A_STAGE_BYTES = BM * BK;
// B rows a CTA loads per stage, ring depth and stage size: single CTAs load all 256 B rows (4 stages of
// 48 KB), pairs 128 each (6 stages of 32 KB); both rings take 192 KB.
__host__ __device__ constexpr int b_rows(bool pair) { return pair ? BN / 2 : BN; }
__host__ __device__ constexpr int stages(bool pair) { return pair ? 6 : 4; }
__host__ __device__ constexpr int stage_bytes(bool pair) { return A_STAGE_BYTES + b_rows(pair) * BK; }
constexpr int MAX_STAGES = 6;
constexpr int STAGE_BYTES = stage_bytes(false);
constexpr int STAGES = stages(false);
static_assert(stages(true) * stage_bytes(true) == STAGES * STAGE_BYTES, "both rings take the same shared memory");
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = 512;
constexpr int kThreads = 320;  // TMA warp, MMA warp, 8 epilogue warps
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
// EPI_RESIDUAL keeps per-column constants (rounded bias, gate or its table part) for up to
// RES_MAX_N columns in shared memory after the pipeline stages.
constexpr int RES_MAX_N = 4096;
constexpr int SMEM_BYTES_RESIDUAL = SMEM_BYTES + 2 * RES_MAX_N * 4;

enum Epilogue : int { EPI_BIAS = 0, EPI_RESIDUAL = 1, EPI_GELU_QUANT = 2 };

struct Params {
  int M, N, K;
  // 0: A is a plain [M, K] map.  > 0: A is stored as K / a_k_block blocks of
  // [M, a_k_block] (the receive buffer of the head-to-sequence exchange:
  // block s holds the columns of source rank s), read through a 3-D map
  // {a_k_block, M, K / a_k_block}; a_k_block is a multiple of BK.
  int a_k_block;
  // 0: as above.  > 0: A is a_planes planes [M, K] (plane stride M * lda bytes) read through a 3-D map
  // {K, M, a_planes}; output column n uses plane n / n_per_scale and its scale scale_a[n / n_per_scale]
  // (one quantised copy of the activations per linear, each with its own input scale).  n_per_scale is a
  // multiple of BN, so every tile reads one plane.
  int a_planes;
  const float* scale_a;  // device scalar; with a_planes > 0 one per plane
  const float* scale_b;  // device array, one entry per n_per_scale columns
  int n_per_scale;
  const void* bias;  // [N] or null
  int bias_fp32;
  __nv_bfloat16* out;
  int64_t ldo;
  // EPI_RESIDUAL only
  const __nv_bfloat16* resid_x;
  int64_t ldx;
  const void* table;
  int table_fp32;
  int64_t table_stride_row;
  const void* ts;
  int ts_fp32;
  int64_t ts_stride_t, ts_stride_p;
  int gate_index;
  // EPI_GELU_QUANT only: e4m3 output [M, N] (row stride ldq) and its device scalar scale
  uint8_t* out_q;
  int64_t ldq;
  const float* q_scale;
};

// Per-column constants of the residual epilogue, computed once per CTA:
// bias rounded to bf16, and the Ada gate (token-uniform timestep) or its table
// part rounded as the reference rounds it (per-token timestep).
template <typename T>
__device__ __forceinline__ float ld1(const void* p, int64_t i) {
  return std::is_same<T, float>::value ? __ldg(static_cast<const float*>(p) + i)
                                       : __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

struct SharedState {
  uint64_t full[MAX_STAGES];   // (pairs: the first CTA's counts both CTAs' bytes)
  uint64_t empty[MAX_STAGES];
  uint64_t tmem_full[NUM_ACC];
  uint64_t tmem_empty[NUM_ACC];
  uint64_t drained;
  uint32_t tmem_base;
  int abort;
};

template <int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    Params p) {
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedState st;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* smem_aligned = smem_raw + (smem_base - smem_u32(smem_raw));

  constexpr int NST = stages(PAIR);
  constexpr int SBYTES = stage_bytes(PAIR);
  constexpr int TM = PAIR ? 2 * BM : BM;  // output rows per tile
  const uint32_t warp = warp_idx();
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;  // 0: the pair's first CTA (issues the MMAs)
  const int num_m = (p.M + TM - 1) / TM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (p.K + BK - 1) / BK;
  const int tile0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tile_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&st.full[s], 1);
      mbar_init(&st.empty[s], 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(&st.tmem_full[a], 1);
      // single CTA: every epilogue thread arrives; pairs: one arrival per epilogue warp of both CTAs
      mbar_init(&st.tmem_empty[a], PAIR ? 16 : 256);
    }
    mbar_init(&st.drained, 1);
    st.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(&st.tmem_base, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&st.tmem_base, TMEM_COLS);
      tmem_relinquish();
    }
  }
  pdl_wait();  // everything above touches only this CTA's shared memory and TMEM
  float* col_bias = reinterpret_cast<float*>(smem_aligned + NST * SBYTES);
  float* col_gate = col_bias + RES_MAX_N;
  const bool gate_uniform = p.ts_stride_t == 0;
  if (EPI == EPI_RESIDUAL) {
    for (int n = threadIdx.x; n < p.N; n += blockDim.x) {
      col_bias[n] = p.bias == nullptr ? 0.f
                                      : bf16_round(p.bias_fp32 ? ld1<float>(p.bias, n) : ld1<__nv_bfloat16>(p.bias, n));
      const int64_t tb = p.gate_index * p.table_stride_row + n;
      float t = p.table_fp32 ? ld1<float>(p.table, tb) : ld1<__nv_bfloat16>(p.table, tb);
      if (p.table_fp32 != p.ts_fp32) t = bf16_round(t);
      if (gate_uniform) {
        const int64_t so = p.gate_index * p.ts_stride_p + n;
        float g = t + (p.ts_fp32 ? ld1<float>(p.ts, so) : ld1<__nv_bfloat16>(p.ts, so));
        t = p.ts_fp32 ? g : bf16_round(g);
      }
      col_gate[n] = t;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
  tc_fence_after();
  const uint32_t tmem_base = st.tmem_base;
  volatile int* abort = &st.abort;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = tile0; tile < num_tiles && ok; tile += tile_step) {
        const int m0 = (tile % num_m) * TM + static_cast<int>(crank) * BM;  // this CTA's A rows
        const int n0 = (tile / num_m) * BN + static_cast<int>(crank) * b_rows(PAIR);  // this CTA's B rows
        const int plane = p.a_planes > 0 ? (tile / num_m) * BN / p.n_per_scale : 0;  // A plane of the tile
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&st.empty[stage], phase ^ 1u, abort)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem_aligned + stage * SBYTES;
          uint8_t* sb = sa + A_STAGE_BYTES;
          if (PAIR) {
            // both CTAs' copies complete on the first CTA's barrier, which expects both
            const uint32_t fb = cluster_addr(&st.full[stage], 0);
            if (crank == 0) mbar_arrive_expect_tx(&st.full[stage], 2 * SBYTES);
            if (p.a_k_block > 0)
              tma_load_3d_pair(sa, &tmap_a, fb, (kb * BK) % p.a_k_block, m0, (kb * BK) / p.a_k_block);
            else if (p.a_planes > 0)
              tma_load_3d_pair(sa, &tmap_a, fb, kb * BK, m0, plane);
            else
              tma_load_2d_pair(sa, &tmap_a, fb, kb * BK, m0);
            tma_load_2d_pair(sb, &tmap_b, fb, kb * BK, n0);
          } else {
            mbar_arrive_expect_tx(&st.full[stage], SBYTES);
            if (p.a_k_block > 0)
              tma_load_3d(sa, &tmap_a, &st.full[stage], (kb * BK) % p.a_k_block, m0, (kb * BK) / p.a_k_block);
            else if (p.a_planes > 0)
              tma_load_3d(sa, &tmap_a, &st.full[stage], kb * BK, m0, plane);
            else
              tma_load_2d(sa, &tmap_a, &st.full[stage], kb * BK, m0);
            tma_load_2d(sb, &tmap_b, &st.full[stage], kb * BK, n0);
          }
          ++issued;
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && (!PAIR || crank == 0)) {
        // Let the copies already in flight land before the CTA exits (a pair's first CTA counts the
        // second's copies too, and the pair leaves together through the closing cluster barrier).
        for (int i = 0; i < NST && i < issued; ++i) {
          int s = stage - 1 - i;
          uint32_t ph = phase;
          if (s < 0) {
            s += NST;
            ph ^= 1u;
          }
          mbar_wait(&st.full[s], ph, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if ((!PAIR || crank == 0) && elect_one()) {
      constexpr uint32_t idesc = make_idesc(0, 0, 0, 0, TM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = tile0; tile < num_tiles && ok; tile += tile_step, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&st.tmem_empty[acc], acc_phase ^ 1u, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&st.full[stage], phase, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * SBYTES;
          const uint32_t sb = sa + A_STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t adesc = make_sdesc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bdesc = make_sdesc_sw128(sb + kk * 32, 16, 1024);
            if (PAIR)
              mma_f8_ss_pair(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
            else
              mma_f8_ss(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          if (PAIR) {  // both CTAs' producers refill this stage
            mma_commit_pair(cluster_addr(&st.empty[stage], 0));
            mma_commit_pair(cluster_addr(&st.empty[stage], 1));
          } else {
            mma_commit(&st.empty[stage]);
          }
          if (++stage == NST) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          if (PAIR) {
            mma_commit_pair(cluster_addr(&st.tmem_full[acc], 0));
            mma_commit_pair(cluster_addr(&st.tmem_full[acc], 1));
          } else {
            mma_commit(&st.tmem_full[acc]);
          }
        }
      }
      // every MMA issued above has completed once `drained` fires
      if (PAIR)
        mma_commit_pair(cluster_addr(&st.drained, 0));
      else
        mma_commit(&st.drained);
      mbar_wait(&st.drained, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // 8 warps: warp w reads TMEM lane quarter (w % 4) and column half (w - 2) / 4 of the tile.
    const uint32_t quarter = warp & 3;
    const int half = (static_cast<int>(warp) - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const float sa = __ldg(p.scale_a);
    const float qs = EPI == EPI_GELU_QUANT ? __ldg(p.q_scale) : 1.f;
    const float qr = __frcp_rn(qs);
    int local = 0;
    for (int tile = tile0; tile < num_tiles; tile += tile_step, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&st.tmem_full[acc], acc_phase, abort)) break;
      tc_fence_after();
      const int m0 = (tile % num_m) * TM + static_cast<int>(crank) * BM;
      const int n0 = (tile / num_m) * BN + half * (BN / 2);
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + acc * BN + half * (BN / 2);
      uint32_t ra[32], rb[32];
      tmem_ld32(taddr, ra);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < BN / 2 / 32; ++c) {
        uint32_t(&cur)[32] = (c & 1) ? rb : ra;
        uint32_t(&nxt)[32] = (c & 1) ? ra : rb;
        if (c + 1 < BN / 2 / 32) tmem_ld32(taddr + (c + 1) * 32, nxt);  // in flight while `cur` is processed
        const int col0 = n0 + c * 32;
        if (row_ok && col0 < p.N) {
          const float scale = (p.a_planes > 0 ? __ldg(p.scale_a + col0 / p.n_per_scale) : sa) *
                              __ldg(p.scale_b + col0 / p.n_per_scale);
          __nv_bfloat16* orow = p.out + static_cast<int64_t>(row) * p.ldo + col0;
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            const int cb = col0 + v8 * 8;
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = __uint_as_float(cur[v8 * 8 + i]) * scale;
            if (EPI == EPI_RESIDUAL) {
              // y = bf16(acc*s); yb = bf16(y + bf16(bias)); prod = bf16(yb * gate); out = bf16(x + prod)
              float xf[8], bb[8], g[8];
              unpack8(__ldg(reinterpret_cast<const uint4*>(p.resid_x + static_cast<int64_t>(row) * p.ldx + cb)), xf);
              *reinterpret_cast<float4*>(&bb[0]) = *reinterpret_cast<const float4*>(col_bias + cb);
              *reinterpret_cast<float4*>(&bb[4]) = *reinterpret_cast<const float4*>(col_bias + cb + 4);
              *reinterpret_cast<float4*>(&g[0]) = *reinterpret_cast<const float4*>(col_gate + cb);
              *reinterpret_cast<float4*>(&g[4]) = *reinterpret_cast<const float4*>(col_gate + cb + 4);
              if (!gate_uniform) {
                float sg[8];
                const int64_t tso = static_cast<int64_t>(row) * p.ts_stride_t + p.gate_index * p.ts_stride_p + cb;
                if (p.ts_fp32)
                  load8<float>(static_cast<const float*>(p.ts) + tso, sg);
                else
                  load8<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(p.ts) + tso, sg);
#pragma unroll
                for (int i = 0; i < 8; ++i) g[i] += sg[i];
                if (!p.ts_fp32) {
#pragma unroll
                  for (int i = 0; i < 8; i += 2) bf16_round2(g[i], g[i + 1]);
                }
              }
#pragma unroll
              for (int i = 0; i < 8; i += 2) bf16_round2(o[i], o[i + 1]);
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] += bb[i];
#pragma unroll
              for (int i = 0; i < 8; i += 2) bf16_round2(o[i], o[i + 1]);
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] *= g[i];
#pragma unroll
              for (int i = 0; i < 8; i += 2) bf16_round2(o[i], o[i + 1]);
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] += xf[i];
            } else if (p.bias != nullptr) {
              // out = bf16(bf16(acc*s) + bf16(bias)); the final rounding is the bf16 pack below
              float bb[8];
              if (p.bias_fp32) {
                load8<float>(static_cast<const float*>(p.bias) + cb, bb);
#pragma unroll
                for (int i = 0; i < 8; i += 2) bf16_round2(bb[i], bb[i + 1]);
              } else {
                load8<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(p.bias) + cb, bb);
              }
#pragma unroll
              for (int i = 0; i < 8; i += 2) bf16_round2(o[i], o[i + 1]);
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] += bb[i];
            }
            if (EPI == EPI_GELU_QUANT) {
              float h[8];
              unpack8(pack8(o), h);  // the bf16 hidden activation
#pragma unroll
              for (int i = 0; i < 8; ++i) h[i] = gelu_tanh(h[i]);
#pragma unroll
              for (int i = 0; i < 8; i += 2) bf16_round2(h[i], h[i + 1]);
              *reinterpret_cast<uint2*>(p.out_q + static_cast<int64_t>(row) * p.ldq + cb) =
                  quant8<__nv_bfloat16, kQuantTorch>(h, qs, qr);
            } else {
              reinterpret_cast<uint4*>(orow)[v8] = pack8(o);
            }
          }
        }
        tmem_ld_wait();
      }
      tc_fence_before();
      if (PAIR) {
        // one arrival per warp on the first CTA's barrier, once all of the warp's TMEM reads are done
        __syncwarp();
        if (lane == 0) {
          if (crank == 0)
            mbar_arrive(&st.tmem_empty[acc]);
          else
            mbar_arrive_remote(cluster_addr(&st.tmem_empty[acc], 0));
        }
      } else {
        mbar_arrive(&st.tmem_empty[acc]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // neither CTA leaves (or frees TMEM) while the other may still signal it
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace ogx
