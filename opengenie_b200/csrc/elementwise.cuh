// HBM-bound stages of the video self-attention block and the numerics they share:
// the E4M3 quantiser, the standalone quantiser and GELU + quantiser kernels, the
// bf16 bias add, the bias + Ada-gated residual, the Ada affine / multiply, the
// per-head gate and the Q/K RMSNorm without RoPE; the argument blocks of the
// row-pipeline AdaZero and Q/K RMSNorm + RoPE kernels (rows.cuh).
//
// All of them move 16-byte vectors (8 x bf16) per lane so every warp access is
// a fully used 512-byte span, keep fp32 arithmetic and round to bf16 exactly
// where the reference rounds.
#pragma once

#include "ogx_sm100.cuh"

namespace ogx {

// ----------------------------------------------------------------- dtype helpers
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 p = __bfloat1622float2(h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  return v;
}

// Loads 8 consecutive values of type T (bf16, fp16 or fp32) as fp32.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]);

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[8]) {
  unpack8(*reinterpret_cast<const uint4*>(p), f);
}

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&f)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&f)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __half22float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Ada value for one slot: table row (rounded to bf16 when the table's dtype
// differs from the timestep's) plus the timestep slot, rounded to bf16 when
// the timestep is bf16.  Mirrors `_torch_ada_values_from_table`
// (ltx_serve/triton_ltx_ops.py:983-998): `table.to(ts.dtype)[idx] + ts[..., idx, :]`.
template <typename TableT, typename TsT>
__device__ __forceinline__ void ada_values8(const TableT* table_row, const TsT* ts_row, float (&out)[8]) {
  constexpr bool round_table = !std::is_same<TableT, TsT>::value;
  constexpr bool round_ada = std::is_same<TsT, __nv_bfloat16>::value;
  float t[8], s[8];
  load8<TableT>(table_row, t);
  load8<TsT>(ts_row, s);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float a = round_table ? bf16_round(t[i]) : t[i];
    float v = a + s[i];
    out[i] = round_ada ? bf16_round(v) : v;
  }
}

// ----------------------------------------------------------------- E4M3
// Round-to-nearest-even fp32 -> e4m3fn with saturation to +-448 (finite
// inputs; NaN is handled by the caller).
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// Quantiser semantics.
//  kQuantTorch : the reference's torch path, triton_ltx_ops.py:146-148:
//                t = round_to_input_dtype(float(x) * (1/s)); clamp(t, +-448); e4m3 RNE.
//                (x * s.reciprocal() on a bf16/fp16 tensor and an fp32 0-dim
//                tensor keeps the fp32 reciprocal and rounds the product once
//                to the input dtype; clamp is exact; the cast is RNE.)
//  kQuantSingle: the reference's Triton kernel, triton_ltx_ops.py:3429-3444:
//                e4m3(clamp(float(x) / s, +-448)), one rounding.
enum QuantMode : int { kQuantTorch = 0, kQuantSingle = 1 };

template <typename InT>
__device__ __forceinline__ float round_to(float v);
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float v) {
  return bf16_round(v);
}
template <>
__device__ __forceinline__ float round_to<__half>(float v) {
  return __half2float(__float2half_rn(v));
}

// NaN inputs: torch's vectorised fp32->bf16 cast returns 0xFFFF for every
// NaN, so the bf16 torch path quantises any NaN to 0xFF; fp16 (and the
// single-rounding path) keep the NaN's sign: 0x7F | sign.
template <typename InT, int MODE>
__device__ __forceinline__ uint8_t quant_one(float x, float s, float r) {
  if (x != x) {
    if (MODE == kQuantTorch && std::is_same<InT, __nv_bfloat16>::value) return 0xFF;
    return static_cast<uint8_t>(0x7F | ((__float_as_uint(x) >> 24) & 0x80));
  }
  float t;
  if (MODE == kQuantTorch) {
    t = round_to<InT>(__fmul_rn(x, r));
  } else {
    t = __fdiv_rn(x, s);
  }
  // t is not NaN here (NaN inputs returned above); inf saturates like torch.clamp
  t = (t < -448.0f) ? -448.0f : ((t > 448.0f) ? 448.0f : t);
  return f32_to_e4m3(t);
}

template <typename InT, int MODE>
__device__ __forceinline__ uint2 quant8(const float (&f)[8], float s, float r) {
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) lo |= static_cast<uint32_t>(quant_one<InT, MODE>(f[i], s, r)) << (8 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) hi |= static_cast<uint32_t>(quant_one<InT, MODE>(f[4 + i], s, r)) << (8 * i);
  return make_uint2(lo, hi);
}

// The torch-path quantiser on bf16 input (the hot case), two values per
// conversion instruction: t = bf16(x * r) by a packed RNE, clamp, packed
// saturating e4m3 conversion; NaN lanes patched to 0xFF afterwards.
template <>
__device__ __forceinline__ uint2 quant8<__nv_bfloat16, kQuantTorch>(const float (&f)[8], float s, float r) {
  uint32_t w[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float t0 = __fmul_rn(f[2 * i], r), t1 = __fmul_rn(f[2 * i + 1], r);
    bf16_round2(t0, t1);
    t0 = fminf(fmaxf(t0, -448.0f), 448.0f);
    t1 = fminf(fmaxf(t1, -448.0f), 448.0f);
    const uint32_t c2 = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(t0, t1), __NV_SATFINITE, __NV_E4M3));
    w[i >> 1] |= (c2 & 0xFFFFu) << (16 * (i & 1));
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (f[i] != f[i]) w[i >> 2] |= 0xFFu << (8 * (i & 3));
  return make_uint2(w[0], w[1]);
}

// ----------------------------------------------------------------- AdaZero arguments
// y = rmsnorm(x) * (1 + scale) + shift with shift/scale read from scale_shift_table + timestep (the
// row-pipeline kernel in rows.cuh; the Ada elementwise kernels below take the same arguments).
struct AdaArgs {
  const __nv_bfloat16* x;
  const void* table;
  const void* ts;
  int64_t ts_stride_b, ts_stride_t, ts_stride_p;  // elements; innermost stride is 1
  int64_t table_stride_row;                       // elements; innermost stride is 1
  int64_t rows, tokens;
  int shift_index, scale_index;
  float eps;
  const float* input_scale;  // device scalar (QUANT only); with nq > 1 an array of nq scales
  __nv_bfloat16* y;          // may be null when only q is wanted
  uint8_t* q;                // e4m3 output (QUANT only)
  int nq;                    // e4m3 outputs (QUANT only; 0 means 1): output i, quantised with input_scale[i],
  int64_t q_plane;           // at q + i * q_plane (bytes)
};

// ----------------------------------------------------------------- per-head gate
// y = bf16(x * gate[row, col / dim_head]) for bf16 x [rows, cols] and bf16 gates: the optional gated
// attention of the video self-attention branch (fused_head_gate_mul_bf16, triton_ltx_ops.py:614-637,
// kernel :3584-3609).  dim_head is a multiple of 8, so the 8 columns of a vector share one gate.
__global__ void __launch_bounds__(256) head_gate_mul_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                             int64_t cols, const __nv_bfloat16* __restrict__ gates,
                                                             int64_t gate_stride_row, int64_t gate_stride_head,
                                                             int dim_head, __nv_bfloat16* __restrict__ y) {
  const int64_t nvec = rows * cols / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const int64_t row = v * 8 / cols;
    const int64_t col = v * 8 - row * cols;
    const float g = __bfloat162float(gates[row * gate_stride_row + (col / dim_head) * gate_stride_head]);
    float f[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(x) + v), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] *= g;
    reinterpret_cast<uint4*>(y)[v] = pack8(f);
  }
}

// ----------------------------------------------------------------- AdaLN affine / Ada multiply
// MUL = false: y = bf16(bf16(x * bf16(1 + scale)) + shift), shift/scale from table + timestep (rounded as
// in ada_values8): the reference's GPU kernel for fused_adaln_affine_from_ada (triton_ltx_ops.py:3469-3534),
// which rounds after each op.  MUL = true: y = bf16(x * gate), gate = the Ada value of slot shift_index
// (fused_mul_from_ada, :695-741, kernel :3723-3771).  Eight columns per thread and iteration.
template <typename TableT, typename TsT, bool MUL>
__global__ void __launch_bounds__(256) adaln_affine_from_ada_kernel(AdaArgs a, int64_t cols) {
  const TableT* table = static_cast<const TableT*>(a.table);
  const TsT* ts = static_cast<const TsT*>(a.ts);
  const int64_t nvec = a.rows * cols / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const int64_t row = v * 8 / cols;
    const int64_t col = v * 8 - row * cols;
    const int64_t b = row / a.tokens;
    const TsT* tsr = ts + b * a.ts_stride_b + (row - b * a.tokens) * a.ts_stride_t + col;
    float sh[8], sc[8], xf[8], o[8];
    ada_values8<TableT, TsT>(table + a.shift_index * a.table_stride_row + col, tsr + a.shift_index * a.ts_stride_p, sh);
    unpack8(__ldg(reinterpret_cast<const uint4*>(a.x) + v), xf);
    if (MUL) {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = xf[i] * sh[i];
    } else {
      ada_values8<TableT, TsT>(table + a.scale_index * a.table_stride_row + col, tsr + a.scale_index * a.ts_stride_p,
                               sc);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = bf16_round(xf[i] * bf16_round(1.0f + sc[i])) + sh[i];
    }
    reinterpret_cast<uint4*>(a.y)[v] = pack8(o);
  }
}

// ----------------------------------------------------------------- quantiser
template <typename InT, int MODE>
__global__ void __launch_bounds__(256) fp8_quantize_kernel(const InT* __restrict__ x, int64_t n,
                                                           const float* __restrict__ input_scale,
                                                           uint8_t* __restrict__ q) {
  const float s = __ldg(input_scale);
  const float r = __frcp_rn(s);
  const int64_t nvec = n >> 3;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x) + v);
    float f[8];
    if (std::is_same<InT, __nv_bfloat16>::value) {
      unpack8(raw, f);
      reinterpret_cast<uint2*>(q)[v] = quant8<InT, MODE>(f, s, r);
    } else {
      const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 p = __half22float2(h[i]);
        f[2 * i] = p.x;
        f[2 * i + 1] = p.y;
      }
      uint2 codes = quant8<InT, MODE>(f, s, r);
      // half -> float conversion canonicalises NaN; restore each NaN's sign from the raw bits
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      uint32_t* c = reinterpret_cast<uint32_t*>(&codes);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t hb = (w[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;
        if ((hb & 0x7C00u) == 0x7C00u && (hb & 0x03FFu) != 0u) {
          const uint32_t code = 0x7Fu | ((hb >> 8) & 0x80u);
          const int word = i >> 2, sh = 8 * (i & 3);
          c[word] = (c[word] & ~(0xFFu << sh)) | (code << sh);
        }
      }
      reinterpret_cast<uint2*>(q)[v] = codes;
    }
  }
  // ragged tail (n % 8), handled by the first threads of block 0
  if (blockIdx.x == 0) {
    const int64_t tail0 = nvec << 3;
    for (int64_t i = tail0 + threadIdx.x; i < n; i += blockDim.x) {
      float f;
      if (std::is_same<InT, __nv_bfloat16>::value) {
        f = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
        q[i] = quant_one<InT, MODE>(f, s, r);
      } else {
        const uint32_t hb = reinterpret_cast<const uint16_t*>(x)[i];
        f = __half2float(reinterpret_cast<const __half*>(x)[i]);
        q[i] = ((hb & 0x7C00u) == 0x7C00u && (hb & 0x03FFu) != 0u) ? static_cast<uint8_t>(0x7Fu | ((hb >> 8) & 0x80u))
                                                                  : quant_one<InT, MODE>(f, s, r);
      }
    }
  }
}

// ----------------------------------------------------------------- GELU (tanh) + quantiser
// gelu(x) = 0.5 x (1 + tanh(u)), u = sqrt(2/pi) (x + 0.044715 x^3): the GELU the reference's FFN uses
// (torch.nn.functional.gelu(approximate="tanh"), triton_ltx_ops.py:166, and its Triton kernel
// :3546-3548).  Evaluated through the identity 0.5 (1 + tanh(u)) = 1 / (1 + e^(-2u)) with the hardware
// ex2 and reciprocal approximations: a few instructions instead of a tanh, and no cancellation for
// x << 0 where 1 + tanh(u) loses the digits of a tiny result.  Infinities and NaN propagate as in the
// tanh form (gelu(+inf) = +inf, gelu(-inf) = NaN).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * (x * x * x));
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-2.8853900817779268f * u));  // e^(-2u) = 2^(-2u log2 e)
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return x * r;
}

// q = quant(round_to_input_dtype(gelu(x))) with the torch-path quantiser (the reference's torch path
// rounds the GELU output to the input dtype, then multiplies by 1/s in that dtype:
// triton_ltx_ops.py:164-169).  gelu_out (may be null) receives the rounded GELU values.
template <typename InT>
__global__ void __launch_bounds__(256) gelu_tanh_quantize_kernel(const InT* __restrict__ x, int64_t n,
                                                                 const float* __restrict__ input_scale,
                                                                 uint8_t* __restrict__ q, InT* __restrict__ gelu_out) {
  const float s = __ldg(input_scale);
  const float r = __frcp_rn(s);
  const int64_t nvec = n >> 3;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    float f[8];
    load8<InT>(x + v * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = round_to<InT>(gelu_tanh(f[i]));
    reinterpret_cast<uint2*>(q)[v] = quant8<InT, kQuantTorch>(f, s, r);
    if (gelu_out != nullptr) {
      if (std::is_same<InT, __nv_bfloat16>::value) {
        reinterpret_cast<uint4*>(gelu_out)[v] = pack8(f);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) reinterpret_cast<__half*>(gelu_out)[v * 8 + i] = __float2half_rn(f[i]);
      }
    }
  }
  if (blockIdx.x == 0) {
    for (int64_t i = (nvec << 3) + threadIdx.x; i < n; i += blockDim.x) {
      float f;
      if (std::is_same<InT, __nv_bfloat16>::value)
        f = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
      else
        f = __half2float(reinterpret_cast<const __half*>(x)[i]);
      f = round_to<InT>(gelu_tanh(f));
      q[i] = quant_one<InT, kQuantTorch>(f, s, r);
      if (gelu_out != nullptr) {
        if (std::is_same<InT, __nv_bfloat16>::value)
          reinterpret_cast<__nv_bfloat16*>(gelu_out)[i] = __float2bfloat16_rn(f);
        else
          reinterpret_cast<__half*>(gelu_out)[i] = __float2half_rn(f);
      }
    }
  }
}

// ----------------------------------------------------------------- bias add
// out = bf16(x + bf16(bias)) (triton_ltx_ops.py:3446-3464; the bias is rounded
// to bf16 first when it is fp32, like `bias.to(x.dtype)`).
template <typename BiasT>
__global__ void __launch_bounds__(256) bias_add_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const BiasT* __restrict__ bias, int64_t rows, int64_t cols,
                                                       __nv_bfloat16* __restrict__ out) {
  const int64_t cvec = cols >> 3;
  const int64_t nvec = rows * cvec;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const int64_t c = (v % cvec) << 3;
    float f[8], bb[8], o[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(x) + v), f);
    load8<BiasT>(bias + c, bb);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = f[i] + bf16_round(bb[i]);
    reinterpret_cast<uint4*>(out)[v] = pack8(o);
  }
}

// ----------------------------------------------------------------- bias + gate + residual
// out = bf16(x + bf16(bf16(y + bf16(bias)) * gate)), gate from the table and
// timestep slot `gate_index` (triton_ltx_ops.py:3663-3721).
struct ResidualArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* y;
  const void* bias;
  const void* table;
  const void* ts;
  int64_t ts_stride_b, ts_stride_t, ts_stride_p;
  int64_t table_stride_row;
  int64_t rows, tokens, cols;
  int gate_index;
  __nv_bfloat16* out;
};

template <typename BiasT, typename TableT, typename TsT>
__global__ void __launch_bounds__(256) residual_gate_bias_kernel(ResidualArgs a) {
  const int64_t cvec = a.cols >> 3;
  const int64_t nvec = a.rows * cvec;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const BiasT* bias = static_cast<const BiasT*>(a.bias);
  const TableT* tgate = static_cast<const TableT*>(a.table) + a.gate_index * a.table_stride_row;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const int64_t row = v / cvec;
    const int64_t c = (v - row * cvec) << 3;
    const int64_t b = row / a.tokens;
    const int64_t t = row - b * a.tokens;
    const TsT* sgate = static_cast<const TsT*>(a.ts) + b * a.ts_stride_b + t * a.ts_stride_t +
                       a.gate_index * a.ts_stride_p;
    float xf[8], yf[8], bf[8], g[8], o[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(a.x) + v), xf);
    unpack8(__ldg(reinterpret_cast<const uint4*>(a.y) + v), yf);
    load8<BiasT>(bias + c, bf);
    ada_values8<TableT, TsT>(tgate + c, sgate + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float yb = bf16_round(yf[i] + bf16_round(bf[i]));
      const float prod = bf16_round(yb * g[i]);
      o[i] = xf[i] + prod;
    }
    reinterpret_cast<uint4*>(a.out)[v] = pack8(o);
  }
}

// ----------------------------------------------------------------- Q/K RMSNorm + split RoPE arguments
// Per token: q_hat = q * rsqrt(mean(q^2) + eps) * w_q over all 4096 columns,
// then per head h and half index j < 64:
//   o[j]    = q_hat[j] * cos[h,t,j] - q_hat[j+64] * sin[h,t,j]
//   o[j+64] = q_hat[j+64] * cos[h,t,j] + q_hat[j] * sin[h,t,j]
// in fp32 with one bf16 rounding (triton_ltx_ops.py:3901-3978).  Same for k.  The kernel is the
// row-pipeline qk_rmsnorm_rope_ring_kernel (rows.cuh).
//
// Outputs are addressed per (token, head) through a table of group bases:
// dst[j][h / heads_per_group] + t*out_stride_t + (h % heads_per_group)*128 + d,
// which is the plain [L, 4096] layout for heads_per_group = 32 and, with one
// base per GPU, the receive buffers of the sequence-to-head exchange written
// directly over NVLink.  V (optional) is copied through the same addressing.
struct RopeArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;  // optional
  int64_t in_stride_t;      // elements between tokens of q/k/v
  const void* q_weight;
  const void* k_weight;
  const void* cos;
  const void* sin;
  int64_t cs_stride_h, cs_stride_t;  // elements; innermost stride 1
  int64_t tokens;
  float eps;
  // Destination of head h of tensor j (0 q, 1 k, 2 v) for token t:
  // dst[j][h / heads_per_group] + t * out_stride_t + (h % heads_per_group) * 128.
  // The group bases may point into other GPUs' memory (peer stores over NVLink).
  __nv_bfloat16* dst[3][8];
  int64_t out_stride_t;
  int heads_per_group;
  int copy_v;        // also copy v (dst[2] valid)
  int system_fence;  // fence the stores system-wide at exit (peer destinations)
};

// Base pointer of head group g (< 8) by constant-index selects: a runtime index into the kernel's parameter
// array would copy the array to local memory.
__device__ __forceinline__ __nv_bfloat16* group_base(__nv_bfloat16* const (&bases)[8], int g) {
  __nv_bfloat16* b = bases[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) b = (g == i) ? bases[i] : b;
  return b;
}

// Q/K RMSNorm without rotary embedding (attention whose keys come from another sequence): rows
// [0, rows_q) are Q rows, [rows_q, rows_q + rows_k) K rows, each normalised over its 4096 columns and
// multiplied by its tensor's weight with the arithmetic of the RoPE kernel (fp32, one bf16 rounding, the
// same order of the sum of squares), so with cos = 1 and sin = 0 the two agree bit for bit.  The kernel is
// the row-pipeline qk_rmsnorm_ring_kernel (rows.cuh).
struct RmsRowsArgs {
  const __nv_bfloat16* in[2];
  int64_t in_stride[2];  // elements between rows
  __nv_bfloat16* out[2];
  int64_t out_stride[2];
  const void* weight[2];
  int64_t rows_q, rows;  // Q rows, all rows
  float eps;
};

}  // namespace ogx
