// C ABI of the B200 video self-attention block (declarations and reference
// citations in include/ogx.h).  Host-side guards mirror the reference's
// `_can_use_*` / `*_guard_reason` checks; a failed guard is an error (no
// fallback).  Tensor maps for TMA are built per call on the host with the
// driver's cuTensorMapEncodeTiled, fetched through the runtime so the library
// does not link libcuda directly.

#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <atomic>
#include <unordered_map>
#include <utility>
#include <cstdlib>

#include "../../include/ogx.h"
#include "elementwise.cuh"
#include "attention.cuh"
#include "rows.cuh"
#include "fp8_gemm.cuh"
#include "peer.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(OGX_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return OGX_OK;
}

int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

// The block's kernels are launched with programmatic stream serialization (each calls pdl_wait() before
// touching global memory), so a kernel's set-up overlaps the tail of the one before it in the stream.
// OGX_PDL=0 in the environment turns it off.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("OGX_PDL");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

// cluster_x > 1 launches clusters of that many CTAs along x (the GEMM's CTA pairs).
template <typename... KArgs, typename... Args>
void launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, unsigned cluster_x,
                    Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  launch_cluster(kernel, grid, block, smem, s, 1u, std::forward<Args>(args)...);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// ------------------------------------------------------------- tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

int make_map(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(OGX_ECUDA, "cuTensorMapEncodeTiled unavailable");
  uint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), dims, strides_bytes, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OGX_EINVAL, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return OGX_OK;
}

// Raise the dynamic shared-memory limit of a kernel once per (kernel, device).
template <typename K>
int ensure_smem(K kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, uint64_t> done;  // kernel -> one bit per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(OGX_ECUDA, "cudaGetDevice failed");
  const void* key = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  uint64_t& mask = done[key];
  if (dev < 64 && (mask >> dev) & 1u) return OGX_OK;
  int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                      "cudaFuncSetAttribute");
  if (rc == OGX_OK && dev < 64) mask |= (uint64_t{1} << dev);
  return rc;
}

bool dtype_ok(int dt) { return dt == OGX_DTYPE_BF16 || dt == OGX_DTYPE_F32; }

// ------------------------------------------------------------- AdaZero
// One persistent row-pipeline CTA per SM (csrc/rows.cuh), at most one per row.
template <int COLS, typename TableT, typename TsT, bool QUANT, int QMODE, bool UNIFORM>
int launch_ada_ring(const ogx::AdaArgs& a, cudaStream_t s) {
  auto kern = ogx::rows::adazero_ring_kernel<COLS, TableT, TsT, QUANT, QMODE, UNIFORM>;
  const int smem = ogx::rows::AdaLayout<COLS, TsT>::smem_bytes(UNIFORM) + 128;
  int rc = ensure_smem(kern, smem);
  if (rc) return rc;
  const int64_t sms = sm_count();
  const dim3 grid(static_cast<unsigned>(a.rows < sms ? a.rows : sms));
  launch(kern, grid, ogx::rows::kWideThreads, static_cast<size_t>(smem), s, a);
  return OGX_OK;
}

template <int COLS, typename TableT, typename TsT, bool UNIFORM>
int launch_ada_u(const ogx::AdaArgs& a, bool quant, int qmode, cudaStream_t s) {
  if (!quant) return launch_ada_ring<COLS, TableT, TsT, false, 0, UNIFORM>(a, s);
  if (qmode == OGX_QUANT_TORCH) return launch_ada_ring<COLS, TableT, TsT, true, ogx::kQuantTorch, UNIFORM>(a, s);
  return launch_ada_ring<COLS, TableT, TsT, true, ogx::kQuantSingle, UNIFORM>(a, s);
}

template <int COLS, typename TableT, typename TsT>
int launch_ada_cols(const ogx::AdaArgs& a, bool quant, int qmode, cudaStream_t s) {
  // token-uniform timestep: every row of every batch reads the same Ada slots
  const bool uniform = a.ts_stride_t == 0 && (a.ts_stride_b == 0 || a.rows <= a.tokens);
  if (uniform) return launch_ada_u<COLS, TableT, TsT, true>(a, quant, qmode, s);
  return launch_ada_u<COLS, TableT, TsT, false>(a, quant, qmode, s);
}

template <typename TableT, typename TsT>
int launch_ada_t(const ogx::AdaArgs& a, int64_t cols, bool quant, int qmode, cudaStream_t s) {
  if (cols == 4096) return launch_ada_cols<4096, TableT, TsT>(a, quant, qmode, s);
  return launch_ada_cols<2048, TableT, TsT>(a, quant, qmode, s);
}

int ada_guard(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table, int table_dtype,
              const void* ts, int ts_dtype, int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p,
              int idx0, int idx1) {
  if (x == nullptr || table == nullptr || ts == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (batch < 1 || tokens < 0) return fail(OGX_EINVAL, "x_shape");
  if (cols != 2048 && cols != 4096) return fail(OGX_EINVAL, "cols");
  if (!dtype_ok(table_dtype)) return fail(OGX_EINVAL, "table_dtype");
  if (!dtype_ok(ts_dtype)) return fail(OGX_EINVAL, "timestep_dtype");
  if (idx0 < 0 || idx1 < 0) return fail(OGX_EINVAL, "ada_index");
  const int esz = ts_dtype == OGX_DTYPE_F32 ? 4 : 2;
  if (!aligned16(x) || !aligned16(table) || !aligned16(ts)) return fail(OGX_EINVAL, "alignment");
  if ((ts_stride_b * esz) % 16 || (ts_stride_t * esz) % 16 || (ts_stride_p * esz) % 16)
    return fail(OGX_EINVAL, "timestep_stride");
  return OGX_OK;
}

int ada_dispatch(const ogx::AdaArgs& a, int64_t cols, int table_dtype, int ts_dtype, bool quant, int qmode,
                 cudaStream_t s) {
  if (a.rows == 0) return OGX_OK;
  int rc;
  if (table_dtype == OGX_DTYPE_F32 && ts_dtype == OGX_DTYPE_BF16)
    rc = launch_ada_t<float, __nv_bfloat16>(a, cols, quant, qmode, s);
  else if (table_dtype == OGX_DTYPE_BF16 && ts_dtype == OGX_DTYPE_BF16)
    rc = launch_ada_t<__nv_bfloat16, __nv_bfloat16>(a, cols, quant, qmode, s);
  else if (table_dtype == OGX_DTYPE_F32 && ts_dtype == OGX_DTYPE_F32)
    rc = launch_ada_t<float, float>(a, cols, quant, qmode, s);
  else
    rc = launch_ada_t<__nv_bfloat16, float>(a, cols, quant, qmode, s);
  if (rc) return rc;
  return check_launch("adazero_ring_kernel");
}

// ------------------------------------------------------------- Q/K RMSNorm + RoPE
// One persistent row-pipeline CTA per SM (csrc/rows.cuh), at most one per token; cos/sin from tables
// (src == nullptr) or generated from the tokens' positions.
template <typename WT, typename CsT, bool GEN, bool COPY_V>
int launch_rope_ring(const ogx::RopeArgs& a, const ogx::rows::RopeSource& src, cudaStream_t s) {
  auto kern = ogx::rows::qk_rmsnorm_rope_ring_kernel<WT, CsT, GEN, COPY_V>;
  const int smem = ogx::rows::RopeLayout::smem_bytes(COPY_V) + 128;
  int rc = ensure_smem(kern, smem);
  if (rc) return rc;
  const int64_t sms = sm_count();
  const dim3 grid(static_cast<unsigned>(a.tokens < sms ? a.tokens : sms));
  launch(kern, grid, ogx::rows::kRopeThreads, static_cast<size_t>(smem), s, a, src);
  return OGX_OK;
}

template <typename WT>
int rope_dispatch_w(const ogx::RopeArgs& a, const ogx::rows::RopeSource* src, int cs_dtype, cudaStream_t s) {
  const ogx::rows::RopeSource none{};
  if (src != nullptr)
    return a.copy_v ? launch_rope_ring<WT, __nv_bfloat16, true, true>(a, *src, s)
                    : launch_rope_ring<WT, __nv_bfloat16, true, false>(a, *src, s);
  if (cs_dtype == OGX_DTYPE_F32)
    return a.copy_v ? launch_rope_ring<WT, float, false, true>(a, none, s)
                    : launch_rope_ring<WT, float, false, false>(a, none, s);
  return a.copy_v ? launch_rope_ring<WT, __nv_bfloat16, false, true>(a, none, s)
                  : launch_rope_ring<WT, __nv_bfloat16, false, false>(a, none, s);
}

int rope_dispatch(const ogx::RopeArgs& a, const ogx::rows::RopeSource* src, int weight_dtype, int cs_dtype,
                  cudaStream_t s) {
  const int rc = weight_dtype == OGX_DTYPE_F32 ? rope_dispatch_w<float>(a, src, cs_dtype, s)
                                               : rope_dispatch_w<__nv_bfloat16>(a, src, cs_dtype, s);
  if (rc) return rc;
  return check_launch("qk_rmsnorm_rope_ring_kernel");
}

// Checks of the generated-cos/sin arguments: the 2048-slot frequency and axis tables (device memory) and
// the latent grid that maps a token index to its (t, h, w) position.
int rope_source(const void* inv_freq, const void* slot_axis, int64_t grid_h, int64_t grid_w, int64_t token0,
                ogx::rows::RopeSource* src) {
  if (inv_freq == nullptr || slot_axis == nullptr) return fail(OGX_EINVAL, "rope_shape: null frequency table");
  if (reinterpret_cast<uintptr_t>(inv_freq) & 7u) return fail(OGX_EINVAL, "alignment");
  if (grid_h < 1 || grid_w < 1 || grid_h > INT32_MAX || grid_w > INT32_MAX || token0 < 0)
    return fail(OGX_EINVAL, "rope_shape: grid");
  src->inv_freq = static_cast<const double*>(inv_freq);
  src->slot_axis = static_cast<const uint8_t*>(slot_axis);
  src->grid_h = static_cast<int>(grid_h);
  src->grid_w = static_cast<int>(grid_w);
  src->token0 = token0;
  return OGX_OK;
}

int grid_for(int64_t nvec) {
  const int64_t want = (nvec + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

}  // namespace

extern "C" {

int ogx_version(void) { return 1; }

const char* ogx_last_error(void) { return g_last_error.c_str(); }

int ogx_device_status(unsigned int* status, int clear) {
  unsigned int v = 0;
  int rc = check_cuda(cudaMemcpyFromSymbol(&v, g_ogx_status, sizeof(v)), "read status");
  if (rc != OGX_OK) return rc;
  if (status) *status = v;
  if (clear) {
    const unsigned int z = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_ogx_status, &z, sizeof(z)), "clear status");
  }
  return rc;
}

int ogx_adazero_from_ada(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                         int table_dtype, int64_t table_stride_row, const void* timestep, int timestep_dtype,
                         int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int shift_index,
                         int scale_index, float eps, void* y, void* stream) {
  int rc = ada_guard(x, batch, tokens, cols, table, table_dtype, timestep, timestep_dtype, ts_stride_b, ts_stride_t,
                     ts_stride_p, shift_index, scale_index);
  if (rc) return rc;
  if (y == nullptr || !aligned16(y)) return fail(OGX_EINVAL, "output");
  ogx::AdaArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.table = table;
  a.ts = timestep;
  a.ts_stride_b = ts_stride_b;
  a.ts_stride_t = ts_stride_t;
  a.ts_stride_p = ts_stride_p;
  a.table_stride_row = table_stride_row;
  a.rows = batch * tokens;
  a.tokens = tokens > 0 ? tokens : 1;
  a.shift_index = shift_index;
  a.scale_index = scale_index;
  a.eps = eps;
  a.y = static_cast<__nv_bfloat16*>(y);
  return ada_dispatch(a, cols, table_dtype, timestep_dtype, false, 0, static_cast<cudaStream_t>(stream));
}

static int ada_elementwise(bool mul, const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                    int table_dtype, int64_t table_stride_row, const void* timestep, int timestep_dtype,
                    int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int idx0, int idx1, void* y,
                    void* stream) {
  int rc = ada_guard(x, batch, tokens, cols, table, table_dtype, timestep, timestep_dtype, ts_stride_b, ts_stride_t,
                     ts_stride_p, idx0, idx1);
  if (rc) return rc;
  if (y == nullptr || !aligned16(y)) return fail(OGX_EINVAL, "output");
  ogx::AdaArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.table = table;
  a.ts = timestep;
  a.ts_stride_b = ts_stride_b;
  a.ts_stride_t = ts_stride_t;
  a.ts_stride_p = ts_stride_p;
  a.table_stride_row = table_stride_row;
  a.rows = batch * tokens;
  a.tokens = tokens > 0 ? tokens : 1;
  a.shift_index = idx0;
  a.scale_index = idx1;
  a.y = static_cast<__nv_bfloat16*>(y);
  if (a.rows == 0) return OGX_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(a.rows * cols / 8);
  const bool tf = table_dtype == OGX_DTYPE_F32, sf = timestep_dtype == OGX_DTYPE_F32;
#define OGX_ADA_EW(T, S)                                                                   \
  (mul ? ogx::adaln_affine_from_ada_kernel<T, S, true><<<grid, 256, 0, s>>>(a, cols)       \
       : ogx::adaln_affine_from_ada_kernel<T, S, false><<<grid, 256, 0, s>>>(a, cols))
  if (tf && sf)
    OGX_ADA_EW(float, float);
  else if (tf)
    OGX_ADA_EW(float, __nv_bfloat16);
  else if (sf)
    OGX_ADA_EW(__nv_bfloat16, float);
  else
    OGX_ADA_EW(__nv_bfloat16, __nv_bfloat16);
#undef OGX_ADA_EW
  return check_launch(mul ? "mul_from_ada" : "adaln_affine_from_ada_kernel");
}

int ogx_adaln_affine_from_ada(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                              int table_dtype, int64_t table_stride_row, const void* timestep, int timestep_dtype,
                              int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int shift_index,
                              int scale_index, void* y, void* stream) {
  return ada_elementwise(false, x, batch, tokens, cols, table, table_dtype, table_stride_row, timestep,
                         timestep_dtype, ts_stride_b, ts_stride_t, ts_stride_p, shift_index, scale_index, y, stream);
}

int ogx_head_gate_mul_bf16(const void* x, int64_t rows, int64_t heads, int64_t dim_head, const void* gates,
                           int64_t gate_stride_row, int64_t gate_stride_head, void* y, void* stream) {
  if (x == nullptr || gates == nullptr || y == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (rows < 0 || heads < 1 || dim_head < 8 || dim_head % 8) return fail(OGX_EINVAL, "shape");
  if (!aligned16(x) || !aligned16(y) || (reinterpret_cast<uintptr_t>(gates) & 1u)) return fail(OGX_EINVAL, "alignment");
  if (rows == 0) return OGX_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t cols = heads * dim_head;
  ogx::head_gate_mul_kernel<<<grid_for(rows * cols / 8), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x), rows, cols, static_cast<const __nv_bfloat16*>(gates), gate_stride_row,
      gate_stride_head, static_cast<int>(dim_head), static_cast<__nv_bfloat16*>(y));
  return check_launch("head_gate_mul_kernel");
}

int ogx_mul_from_ada(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table, int table_dtype,
                     int64_t table_stride_row, const void* timestep, int timestep_dtype, int64_t ts_stride_b,
                     int64_t ts_stride_t, int64_t ts_stride_p, int gate_index, void* y, void* stream) {
  return ada_elementwise(true, x, batch, tokens, cols, table, table_dtype, table_stride_row, timestep,
                         timestep_dtype, ts_stride_b, ts_stride_t, ts_stride_p, gate_index, gate_index, y, stream);
}

int ogx_adazero_from_ada_e4m3(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                              int table_dtype, int64_t table_stride_row, const void* timestep, int timestep_dtype,
                              int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int shift_index,
                              int scale_index, float eps, const float* input_scale, int quant_mode, void* y,
                              void* q, void* stream) {
  int rc = ada_guard(x, batch, tokens, cols, table, table_dtype, timestep, timestep_dtype, ts_stride_b, ts_stride_t,
                     ts_stride_p, shift_index, scale_index);
  if (rc) return rc;
  if (q == nullptr || (y != nullptr && !aligned16(y)) || (reinterpret_cast<uintptr_t>(q) & 7u))
    return fail(OGX_EINVAL, "output");
  if (input_scale == nullptr) return fail(OGX_EINVAL, "input_scale");
  if (quant_mode != OGX_QUANT_TORCH && quant_mode != OGX_QUANT_SINGLE) return fail(OGX_EINVAL, "quant_mode");
  ogx::AdaArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.table = table;
  a.ts = timestep;
  a.ts_stride_b = ts_stride_b;
  a.ts_stride_t = ts_stride_t;
  a.ts_stride_p = ts_stride_p;
  a.table_stride_row = table_stride_row;
  a.rows = batch * tokens;
  a.tokens = tokens > 0 ? tokens : 1;
  a.shift_index = shift_index;
  a.scale_index = scale_index;
  a.eps = eps;
  a.input_scale = input_scale;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.q = static_cast<uint8_t*>(q);
  return ada_dispatch(a, cols, table_dtype, timestep_dtype, true, quant_mode, static_cast<cudaStream_t>(stream));
}

int ogx_adazero_from_ada_e4m3_planes(const void* x, int64_t batch, int64_t tokens, int64_t cols, const void* table,
                                     int table_dtype, int64_t table_stride_row, const void* timestep,
                                     int timestep_dtype, int64_t ts_stride_b, int64_t ts_stride_t,
                                     int64_t ts_stride_p, int shift_index, int scale_index, float eps,
                                     const float* input_scales, int planes, int quant_mode, void* y, void* q,
                                     int64_t q_plane_stride, void* stream) {
  int rc = ada_guard(x, batch, tokens, cols, table, table_dtype, timestep, timestep_dtype, ts_stride_b, ts_stride_t,
                     ts_stride_p, shift_index, scale_index);
  if (rc) return rc;
  if (planes < 1 || planes > 3) return fail(OGX_EINVAL, "planes: 1 to 3 e4m3 outputs");
  if (q == nullptr || (y != nullptr && !aligned16(y)) || !aligned16(q)) return fail(OGX_EINVAL, "output");
  if (planes > 1 && (q_plane_stride % 16 || q_plane_stride < batch * tokens * cols))
    return fail(OGX_EINVAL, "output: plane stride");
  if (input_scales == nullptr) return fail(OGX_EINVAL, "input_scale");
  if (quant_mode != OGX_QUANT_TORCH && quant_mode != OGX_QUANT_SINGLE) return fail(OGX_EINVAL, "quant_mode");
  ogx::AdaArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.table = table;
  a.ts = timestep;
  a.ts_stride_b = ts_stride_b;
  a.ts_stride_t = ts_stride_t;
  a.ts_stride_p = ts_stride_p;
  a.table_stride_row = table_stride_row;
  a.rows = batch * tokens;
  a.tokens = tokens > 0 ? tokens : 1;
  a.shift_index = shift_index;
  a.scale_index = scale_index;
  a.eps = eps;
  a.input_scale = input_scales;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.q = static_cast<uint8_t*>(q);
  a.nq = planes;
  a.q_plane = q_plane_stride;
  return ada_dispatch(a, cols, table_dtype, timestep_dtype, true, quant_mode, static_cast<cudaStream_t>(stream));
}

int ogx_fp8_quantize_e4m3(const void* x, int x_dtype, int64_t n, const float* input_scale, int quant_mode, void* q,
                          void* stream) {
  if (x_dtype != OGX_DTYPE_BF16 && x_dtype != OGX_DTYPE_F16) return fail(OGX_EINVAL, "x_dtype");
  if (quant_mode != OGX_QUANT_TORCH && quant_mode != OGX_QUANT_SINGLE) return fail(OGX_EINVAL, "quant_mode");
  if (n < 0) return fail(OGX_EINVAL, "numel");
  if (n == 0) return OGX_OK;
  if (x == nullptr || q == nullptr || input_scale == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u)) return fail(OGX_EINVAL, "alignment");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for((n >> 3) > 0 ? (n >> 3) : 1);
  if (x_dtype == OGX_DTYPE_BF16) {
    if (quant_mode == OGX_QUANT_TORCH)
      ogx::fp8_quantize_kernel<__nv_bfloat16, ogx::kQuantTorch><<<grid, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), n, input_scale, static_cast<uint8_t*>(q));
    else
      ogx::fp8_quantize_kernel<__nv_bfloat16, ogx::kQuantSingle><<<grid, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), n, input_scale, static_cast<uint8_t*>(q));
  } else {
    if (quant_mode == OGX_QUANT_TORCH)
      ogx::fp8_quantize_kernel<__half, ogx::kQuantTorch><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), n,
                                                                              input_scale, static_cast<uint8_t*>(q));
    else
      ogx::fp8_quantize_kernel<__half, ogx::kQuantSingle><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), n,
                                                                               input_scale, static_cast<uint8_t*>(q));
  }
  return check_launch("fp8_quantize_kernel");
}

int ogx_gelu_tanh_fp8_quantize_e4m3(const void* x, int x_dtype, int64_t n, const float* input_scale, void* q,
                                    void* gelu_out, void* stream) {
  if (x_dtype != OGX_DTYPE_BF16 && x_dtype != OGX_DTYPE_F16) return fail(OGX_EINVAL, "x_dtype");
  if (n < 0) return fail(OGX_EINVAL, "numel");
  if (n == 0) return OGX_OK;
  if (x == nullptr || q == nullptr || input_scale == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u) || (gelu_out != nullptr && !aligned16(gelu_out)))
    return fail(OGX_EINVAL, "alignment");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for((n >> 3) > 0 ? (n >> 3) : 1);
  if (x_dtype == OGX_DTYPE_BF16)
    ogx::gelu_tanh_quantize_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), n, input_scale, static_cast<uint8_t*>(q),
        static_cast<__nv_bfloat16*>(gelu_out));
  else
    ogx::gelu_tanh_quantize_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), n, input_scale,
                                                                static_cast<uint8_t*>(q),
                                                                static_cast<__half*>(gelu_out));
  return check_launch("gelu_tanh_quantize_kernel");
}

int ogx_bias_add_bf16(const void* x, int64_t rows, int64_t cols, const void* bias, int bias_dtype, void* out,
                      void* stream) {
  if (x == nullptr || bias == nullptr || out == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (!dtype_ok(bias_dtype)) return fail(OGX_EINVAL, "bias_dtype");
  if (rows < 0 || cols <= 0 || cols % 8) return fail(OGX_EINVAL, "shape");
  if (!aligned16(x) || !aligned16(out) || !aligned16(bias)) return fail(OGX_EINVAL, "alignment");
  if (rows == 0) return OGX_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(rows * cols / 8);
  if (bias_dtype == OGX_DTYPE_F32)
    ogx::bias_add_kernel<float><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                     static_cast<const float*>(bias), rows, cols,
                                                     static_cast<__nv_bfloat16*>(out));
  else
    ogx::bias_add_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                             static_cast<const __nv_bfloat16*>(bias), rows, cols,
                                                             static_cast<__nv_bfloat16*>(out));
  return check_launch("bias_add_kernel");
}

int ogx_residual_gate_bias_from_ada(const void* x, const void* y, int64_t batch, int64_t tokens, int64_t cols,
                                    const void* bias, int bias_dtype, const void* table, int table_dtype,
                                    int64_t table_stride_row, const void* timestep, int timestep_dtype,
                                    int64_t ts_stride_b, int64_t ts_stride_t, int64_t ts_stride_p, int gate_index,
                                    void* out, void* stream) {
  int rc = ada_guard(x, batch, tokens, cols, table, table_dtype, timestep, timestep_dtype, ts_stride_b, ts_stride_t,
                     ts_stride_p, gate_index, gate_index);
  if (rc) return rc;
  if (y == nullptr || bias == nullptr || out == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (!dtype_ok(bias_dtype)) return fail(OGX_EINVAL, "bias_dtype");
  if (!aligned16(y) || !aligned16(out) || !aligned16(bias)) return fail(OGX_EINVAL, "alignment");
  const int64_t rows = batch * tokens;
  if (rows == 0) return OGX_OK;
  ogx::ResidualArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.y = static_cast<const __nv_bfloat16*>(y);
  a.bias = bias;
  a.table = table;
  a.ts = timestep;
  a.ts_stride_b = ts_stride_b;
  a.ts_stride_t = ts_stride_t;
  a.ts_stride_p = ts_stride_p;
  a.table_stride_row = table_stride_row;
  a.rows = rows;
  a.tokens = tokens;
  a.cols = cols;
  a.gate_index = gate_index;
  a.out = static_cast<__nv_bfloat16*>(out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(rows * cols / 8);
  const bool bf = bias_dtype == OGX_DTYPE_F32;
  const bool tf = table_dtype == OGX_DTYPE_F32;
  const bool sf = timestep_dtype == OGX_DTYPE_F32;
#define OGX_RES(B, T, S) ogx::residual_gate_bias_kernel<B, T, S><<<grid, 256, 0, s>>>(a)
  if (bf) {
    if (tf) { if (sf) OGX_RES(float, float, float); else OGX_RES(float, float, __nv_bfloat16); }
    else { if (sf) OGX_RES(float, __nv_bfloat16, float); else OGX_RES(float, __nv_bfloat16, __nv_bfloat16); }
  } else {
    if (tf) { if (sf) OGX_RES(__nv_bfloat16, float, float); else OGX_RES(__nv_bfloat16, float, __nv_bfloat16); }
    else {
      if (sf) OGX_RES(__nv_bfloat16, __nv_bfloat16, float);
      else OGX_RES(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16);
    }
  }
#undef OGX_RES
  return check_launch("residual_gate_bias_kernel");
}

}  // extern "C"

namespace {

// Q/K RMSNorm + RoPE into [tokens][..] rows per head group; cos/sin from the tables, or generated (src).
int rope_scatter_impl(const void* q, const void* k, const void* v, int64_t tokens, int64_t in_stride_t,
                      const void* q_weight, const void* k_weight, int weight_dtype, float eps, const void* cos,
                      const void* sin, int cs_dtype, int64_t cs_stride_h, int64_t cs_stride_t,
                      const ogx::rows::RopeSource* src, void* q_out, void* k_out, void* v_out, int64_t out_stride_t,
                      int64_t out_stride_g, int heads_per_group, void* stream) {
  if (q == nullptr || k == nullptr || q_out == nullptr || k_out == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (q_weight == nullptr || k_weight == nullptr) return fail(OGX_EINVAL, "qk_weight_shape");
  if (src == nullptr && (cos == nullptr || sin == nullptr)) return fail(OGX_EINVAL, "rope_shape");
  if (tokens < 1) return fail(OGX_EINVAL, "empty_tokens");
  if (!dtype_ok(weight_dtype) || (src == nullptr && !dtype_ok(cs_dtype))) return fail(OGX_EINVAL, "qk_device_or_dtype");
  if (heads_per_group < 4 || 32 % heads_per_group) return fail(OGX_EINVAL, "heads_per_group");
  if (in_stride_t % 8 || out_stride_t % 8 || out_stride_g % 8) return fail(OGX_EINVAL, "qk_noncontiguous");
  if (src == nullptr) {
    const int cesz = cs_dtype == OGX_DTYPE_F32 ? 4 : 2;
    if ((cs_stride_h * cesz) % 16 || (cs_stride_t * cesz) % 16) return fail(OGX_EINVAL, "rope_shape");
    if (!aligned16(cos) || !aligned16(sin)) return fail(OGX_EINVAL, "alignment");
  }
  if (!aligned16(q) || !aligned16(k) || !aligned16(q_out) || !aligned16(k_out) || !aligned16(q_weight) ||
      !aligned16(k_weight) || (v && !aligned16(v)) || (v_out && !aligned16(v_out)))
    return fail(OGX_EINVAL, "alignment");
  ogx::RopeArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.in_stride_t = in_stride_t;
  a.q_weight = q_weight;
  a.k_weight = k_weight;
  a.cos = cos;
  a.sin = sin;
  a.cs_stride_h = cs_stride_h;
  a.cs_stride_t = cs_stride_t;
  a.tokens = tokens;
  a.eps = eps;
  for (int g = 0; g < 32 / heads_per_group && g < 8; ++g) {
    a.dst[0][g] = static_cast<__nv_bfloat16*>(q_out) + g * out_stride_g;
    a.dst[1][g] = static_cast<__nv_bfloat16*>(k_out) + g * out_stride_g;
    a.dst[2][g] = v_out ? static_cast<__nv_bfloat16*>(v_out) + g * out_stride_g : nullptr;
  }
  a.out_stride_t = out_stride_t;
  a.heads_per_group = heads_per_group;
  a.copy_v = (v != nullptr && v_out != nullptr) ? 1 : 0;
  a.system_fence = 0;
  return rope_dispatch(a, src, weight_dtype, cs_dtype, static_cast<cudaStream_t>(stream));
}

}  // namespace

extern "C" {

int ogx_video_qkv_rmsnorm_rope_scatter(const void* q, const void* k, const void* v, int64_t tokens,
                                       int64_t in_stride_t, const void* q_weight, const void* k_weight,
                                       int weight_dtype, float eps, const void* cos, const void* sin, int cs_dtype,
                                       int64_t cs_stride_h, int64_t cs_stride_t, void* q_out, void* k_out,
                                       void* v_out, int64_t out_stride_t, int64_t out_stride_g,
                                       int heads_per_group, void* stream) {
  return rope_scatter_impl(q, k, v, tokens, in_stride_t, q_weight, k_weight, weight_dtype, eps, cos, sin, cs_dtype,
                           cs_stride_h, cs_stride_t, nullptr, q_out, k_out, v_out, out_stride_t, out_stride_g,
                           heads_per_group, stream);
}

int ogx_video_qk_rmsnorm_rope_positions(const void* q, const void* k, int64_t tokens, int64_t in_stride_t,
                                        const void* q_weight, const void* k_weight, int weight_dtype, float eps,
                                        const double* inv_freq, const unsigned char* slot_axis, int64_t grid_h,
                                        int64_t grid_w, int64_t token0, void* q_out, void* k_out,
                                        int64_t out_stride_t, void* stream) {
  ogx::rows::RopeSource src{};
  const int rc = rope_source(inv_freq, slot_axis, grid_h, grid_w, token0, &src);
  if (rc) return rc;
  return rope_scatter_impl(q, k, nullptr, tokens, in_stride_t, q_weight, k_weight, weight_dtype, eps, nullptr,
                           nullptr, OGX_DTYPE_BF16, 0, 0, &src, q_out, k_out, nullptr, out_stride_t, 0, 32, stream);
}

int ogx_video_qkv_rmsnorm_rope_positions_scatter(const void* q, const void* k, const void* v, int64_t tokens,
                                                 int64_t in_stride_t, const void* q_weight, const void* k_weight,
                                                 int weight_dtype, float eps, const double* inv_freq,
                                                 const unsigned char* slot_axis, int64_t grid_h, int64_t grid_w,
                                                 int64_t token0, void* q_out, void* k_out, void* v_out,
                                                 int64_t out_stride_t, int64_t out_stride_g, int heads_per_group,
                                                 void* stream) {
  ogx::rows::RopeSource src{};
  const int rc = rope_source(inv_freq, slot_axis, grid_h, grid_w, token0, &src);
  if (rc) return rc;
  return rope_scatter_impl(q, k, v, tokens, in_stride_t, q_weight, k_weight, weight_dtype, eps, nullptr, nullptr,
                           OGX_DTYPE_BF16, 0, 0, &src, q_out, k_out, v_out, out_stride_t, out_stride_g,
                           heads_per_group, stream);
}

int ogx_rope_tables_from_positions(const double* inv_freq, const unsigned char* slot_axis, int64_t grid_h,
                                   int64_t grid_w, int64_t token0, int64_t tokens, int cs_dtype, void* cos_out,
                                   void* sin_out, void* stream) {
  ogx::rows::RopeSource src{};
  int rc = rope_source(inv_freq, slot_axis, grid_h, grid_w, token0, &src);
  if (rc) return rc;
  if (tokens < 1) return fail(OGX_EINVAL, "empty_tokens");
  if (!dtype_ok(cs_dtype)) return fail(OGX_EINVAL, "qk_device_or_dtype");
  if (cos_out == nullptr || sin_out == nullptr || !aligned16(cos_out) || !aligned16(sin_out))
    return fail(OGX_EINVAL, "output");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(32 * tokens * 8);
  if (cs_dtype == OGX_DTYPE_F32)
    ogx::rows::rope_tables_kernel<float><<<grid, 256, 0, s>>>(src, tokens, static_cast<float*>(cos_out),
                                                              static_cast<float*>(sin_out));
  else
    ogx::rows::rope_tables_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        src, tokens, static_cast<__nv_bfloat16*>(cos_out), static_cast<__nv_bfloat16*>(sin_out));
  return check_launch("rope_tables_kernel");
}

int ogx_video_qk_rmsnorm_rope(const void* q, const void* k, int64_t tokens, int64_t in_stride_t,
                              const void* q_weight, const void* k_weight, int weight_dtype, float eps,
                              const void* cos, const void* sin, int cs_dtype, int64_t cs_stride_h,
                              int64_t cs_stride_t, void* q_out, void* k_out, int64_t out_stride_t, void* stream) {
  return ogx_video_qkv_rmsnorm_rope_scatter(q, k, nullptr, tokens, in_stride_t, q_weight, k_weight, weight_dtype, eps,
                                            cos, sin, cs_dtype, cs_stride_h, cs_stride_t, q_out, k_out, nullptr,
                                            out_stride_t, 0, 32, stream);
}

int ogx_qk_rmsnorm(const void* q, int64_t q_rows, int64_t q_stride, const void* k, int64_t k_rows, int64_t k_stride,
                   const void* q_weight, const void* k_weight, int weight_dtype, float eps, void* q_out,
                   int64_t q_out_stride, void* k_out, int64_t k_out_stride, void* stream) {
  if (q == nullptr || k == nullptr || q_out == nullptr || k_out == nullptr || q_weight == nullptr ||
      k_weight == nullptr)
    return fail(OGX_EINVAL, "null_pointer");
  if (q_rows < 0 || k_rows < 0 || q_rows + k_rows > INT32_MAX) return fail(OGX_EINVAL, "qk_shape");
  if (!dtype_ok(weight_dtype)) return fail(OGX_EINVAL, "weight_dtype");
  if (q_stride < 4096 || k_stride < 4096 || q_out_stride < 4096 || k_out_stride < 4096 || q_stride % 8 ||
      k_stride % 8 || q_out_stride % 8 || k_out_stride % 8)
    return fail(OGX_EINVAL, "qk_stride");
  if (!aligned16(q) || !aligned16(k) || !aligned16(q_out) || !aligned16(k_out) || !aligned16(q_weight) ||
      !aligned16(k_weight))
    return fail(OGX_EINVAL, "alignment");
  if (q_rows + k_rows == 0) return OGX_OK;
  ogx::RmsRowsArgs a{};
  a.in[0] = static_cast<const __nv_bfloat16*>(q);
  a.in[1] = static_cast<const __nv_bfloat16*>(k);
  a.in_stride[0] = q_stride;
  a.in_stride[1] = k_stride;
  a.out[0] = static_cast<__nv_bfloat16*>(q_out);
  a.out[1] = static_cast<__nv_bfloat16*>(k_out);
  a.out_stride[0] = q_out_stride;
  a.out_stride[1] = k_out_stride;
  a.weight[0] = q_weight;
  a.weight[1] = k_weight;
  a.rows_q = q_rows;
  a.rows = q_rows + k_rows;
  a.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t sms = sm_count();
  const dim3 grid(static_cast<unsigned>(a.rows < sms ? a.rows : sms));
  const size_t smem = ogx::rows::kRmsSmem + 128;
  int rc;
  if (weight_dtype == OGX_DTYPE_F32) {
    rc = ensure_smem(ogx::rows::qk_rmsnorm_ring_kernel<float>, static_cast<int>(smem));
    if (rc) return rc;
    launch(ogx::rows::qk_rmsnorm_ring_kernel<float>, grid, ogx::rows::kWideThreads, smem, s, a);
  } else {
    rc = ensure_smem(ogx::rows::qk_rmsnorm_ring_kernel<__nv_bfloat16>, static_cast<int>(smem));
    if (rc) return rc;
    launch(ogx::rows::qk_rmsnorm_ring_kernel<__nv_bfloat16>, grid, ogx::rows::kWideThreads, smem, s, a);
  }
  return check_launch("qk_rmsnorm_ring_kernel");
}

}  // extern "C"

namespace {

// CTA pairs (256x256 tiles, tcgen05 cta_group::2) or single CTAs (128x256 tiles), whichever the
// persistent schedule finishes sooner: the number of tiles the busiest pair or CTA computes, a pair
// tile taking 0.89 of a single-CTA tile's time per SM (measured: 334 vs 375 us at 9216x12288x4096).
// Pairs lose where their coarser tiles leave a short last round (the 1152-row slices of 8 GPUs).
// OGX_GEMM_PAIRS=0 keeps single CTAs.
bool gemm_use_pairs(int64_t M, int64_t N) {
  static const bool on = [] {
    const char* e = getenv("OGX_GEMM_PAIRS");
    return e == nullptr || e[0] != '0';
  }();
  if (!on || M <= ogx::gemm::BM) return false;
  const int64_t nn = (N + ogx::gemm::BN - 1) / ogx::gemm::BN;
  const int64_t single = (M + ogx::gemm::BM - 1) / ogx::gemm::BM * nn;
  const int64_t pair = (M + 2 * ogx::gemm::BM - 1) / (2 * ogx::gemm::BM) * nn;
  const int64_t ctas = sm_count(), pairs = sm_count() / 2;
  const double t_single = static_cast<double>((single + ctas - 1) / ctas);
  const double t_pair = 0.89 * static_cast<double>((pair + pairs - 1) / pairs);
  return t_pair < t_single;
}

int gemm_common(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                const float* scale_a, const float* scale_b, int64_t n_per_scale, CUtensorMap* ma, CUtensorMap* mb,
                int64_t a_k_block = 0, int64_t a_planes = 0) {
  if (a == nullptr || w == nullptr || scale_a == nullptr || scale_b == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (M < 0 || N <= 0 || K <= 0) return fail(OGX_EINVAL, "shape");
  if (K % 16 || N % 32) return fail(OGX_EINVAL, "shape: K % 16 and N % 32 must be 0");
  if ((a_k_block == 0 && lda < K) || ldw < K || lda % 16 || ldw % 16) return fail(OGX_EINVAL, "leading_dimension");
  if (n_per_scale <= 0 || n_per_scale % 32) return fail(OGX_EINVAL, "n_per_scale");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(OGX_EINVAL, "shape");
  if (!aligned16(a) || !aligned16(w)) return fail(OGX_EINVAL, "alignment");
  if (M == 0) return OGX_OK;
  int rc;
  if (a_planes > 0) {
    // one [M, K] plane (row stride lda) per N segment of n_per_scale columns
    if (a_k_block > 0 || N % a_planes || n_per_scale != N / a_planes || n_per_scale % ogx::gemm::BN)
      return fail(OGX_EINVAL, "a_planes: N must split into planes of a multiple of %d columns", ogx::gemm::BN);
    const uint64_t da[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint64_t>(a_planes)};
    const uint64_t sa[2] = {static_cast<uint64_t>(lda), static_cast<uint64_t>(lda * M)};
    const uint32_t ba[3] = {static_cast<uint32_t>(ogx::gemm::BK), static_cast<uint32_t>(ogx::gemm::BM), 1};
    rc = make_map(ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a, da, sa, ba);
  } else if (a_k_block > 0) {
    if (a_k_block % ogx::gemm::BK || K % a_k_block) return fail(OGX_EINVAL, "a_k_block");
    const uint64_t da[3] = {static_cast<uint64_t>(a_k_block), static_cast<uint64_t>(M),
                            static_cast<uint64_t>(K / a_k_block)};
    const uint64_t sa[2] = {static_cast<uint64_t>(a_k_block), static_cast<uint64_t>(a_k_block * M)};
    const uint32_t ba[3] = {static_cast<uint32_t>(ogx::gemm::BK), static_cast<uint32_t>(ogx::gemm::BM), 1};
    rc = make_map(ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a, da, sa, ba);
  } else {
    const uint64_t da[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t sa[1] = {static_cast<uint64_t>(lda)};
    const uint32_t ba[2] = {static_cast<uint32_t>(ogx::gemm::BK), static_cast<uint32_t>(ogx::gemm::BM)};
    rc = make_map(ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, da, sa, ba);
  }
  if (rc) return rc;
  const uint64_t db[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
  const uint64_t sb[1] = {static_cast<uint64_t>(ldw)};
  const uint32_t bb[2] = {static_cast<uint32_t>(ogx::gemm::BK),
                         static_cast<uint32_t>(ogx::gemm::b_rows(gemm_use_pairs(M, N)))};
  return make_map(mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, db, sb, bb);
}

template <int EPI>
int gemm_launch(const CUtensorMap& ma, const CUtensorMap& mb, const ogx::gemm::Params& p, cudaStream_t s) {
  const int smem = EPI == ogx::gemm::EPI_RESIDUAL ? ogx::gemm::SMEM_BYTES_RESIDUAL : ogx::gemm::SMEM_BYTES;
  if (EPI == ogx::gemm::EPI_RESIDUAL && p.N > ogx::gemm::RES_MAX_N)
    return fail(OGX_EINVAL, "shape: the residual epilogue supports N <= %d", ogx::gemm::RES_MAX_N);
  const int num_n = (p.N + ogx::gemm::BN - 1) / ogx::gemm::BN;
  if (gemm_use_pairs(p.M, p.N)) {  // the same choice gemm_common made for the B tensor map
    auto kern = ogx::gemm::fp8_gemm_kernel<EPI, true>;
    int rc = ensure_smem(kern, smem);
    if (rc) return rc;
    const int tiles = ((p.M + 2 * ogx::gemm::BM - 1) / (2 * ogx::gemm::BM)) * num_n;
    // a persistent grid of pairs no larger than what can be resident at once (an SM left without a
    // partner in its GPC cannot host a pair)
    // looked up once per (epilogue, device); concurrent first calls compute the same value
    static std::atomic<int> resident[3][64];
    int dev = 0;
    rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return fail(OGX_EINVAL, "device ordinal %d out of range", dev);
    int pairs = resident[EPI][dev].load(std::memory_order_relaxed);
    if (pairs == 0) {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(2 * (sm_count() / 2));
      cfg.blockDim = dim3(ogx::gemm::kThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      rc = check_cuda(cudaOccupancyMaxActiveClusters(&n, kern, &cfg), "cudaOccupancyMaxActiveClusters");
      if (rc) return rc;
      if (n < 1) return fail(OGX_ECUDA, "no CTA pair of the GEMM fits on this GPU");
      pairs = n < sm_count() / 2 ? n : sm_count() / 2;
      resident[EPI][dev].store(pairs, std::memory_order_relaxed);
    }
    const int grid = 2 * (tiles < pairs ? tiles : pairs);
    launch_cluster(kern, grid, ogx::gemm::kThreads, smem, s, 2u, ma, mb, p);
    return check_launch("fp8_gemm_kernel (CTA pairs)");
  }
  auto kern = ogx::gemm::fp8_gemm_kernel<EPI, false>;
  int rc = ensure_smem(kern, smem);
  if (rc) return rc;
  const int tiles = ((p.M + ogx::gemm::BM - 1) / ogx::gemm::BM) * num_n;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  launch(kern, grid, ogx::gemm::kThreads, smem, s, ma, mb, p);
  return check_launch("fp8_gemm_kernel");
}

// The attention kernel: the single-CTA kernel with 64-key tiles (the default), or CTA pairs
// (attn_fwd_pair_kernel, 128-key tiles, M=256 MMAs over two SMs) when OGX_ATTN_PAIRS=1 is set in the
// environment, with split score MMAs when it is 2.
int attn_pairs_mode() {
  static const int mode = [] {
    const char* e = std::getenv("OGX_ATTN_PAIRS");
    return (e != nullptr && (e[0] == '1' || e[0] == '2')) ? e[0] - '0' : 0;
  }();
  return mode;
}
bool attn_use_pairs() { return attn_pairs_mode() != 0; }

int attention_common(const void* q, const void* k, const void* v, int64_t batch, int64_t tokens, int64_t kv_tokens,
                     int64_t heads, int64_t head_dim, int64_t stride_b, int64_t stride_t, int64_t kv_stride_b,
                     int64_t kv_stride_t, CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv) {
  if (q == nullptr || k == nullptr || v == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (head_dim != 128) return fail(OGX_EINVAL, "head_dim: only 128 is supported");
  if (batch < 1 || tokens < 1 || kv_tokens < 1 || heads < 1) return fail(OGX_EINVAL, "shape");
  if (tokens > INT32_MAX || kv_tokens > INT32_MAX || heads > 65535 || batch > 65535) return fail(OGX_EINVAL, "shape");
  if (stride_t % 8 || stride_b % 8 || stride_t < heads * 128) return fail(OGX_EINVAL, "stride");
  if (kv_stride_t % 8 || kv_stride_b % 8 || kv_stride_t < heads * 128) return fail(OGX_EINVAL, "stride");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v)) return fail(OGX_EINVAL, "alignment");
  const uint64_t qdims[4] = {128, static_cast<uint64_t>(heads), static_cast<uint64_t>(tokens),
                             static_cast<uint64_t>(batch)};
  const uint64_t qstrides[3] = {256, static_cast<uint64_t>(stride_t) * 2, static_cast<uint64_t>(stride_b) * 2};
  const uint64_t kvdims[4] = {128, static_cast<uint64_t>(heads), static_cast<uint64_t>(kv_tokens),
                              static_cast<uint64_t>(batch)};
  const uint64_t kvstrides[3] = {256, static_cast<uint64_t>(kv_stride_t) * 2, static_cast<uint64_t>(kv_stride_b) * 2};
  const uint32_t qbox[4] = {64, 1, static_cast<uint32_t>(ogx::attn::BQ), 1};
  // single CTA: K and V tiles of 64 keys; pairs: each CTA loads 64 keys of K and 128 keys of its V columns
  const uint32_t kbox[4] = {64, 1, 64u, 1};
  const uint32_t vbox[4] = {64, 1, attn_use_pairs() ? static_cast<uint32_t>(ogx::attn::PBKV) : 64u, 1};
  int rc = make_map(mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, q, qdims, qstrides, qbox);
  if (rc) return rc;
  rc = make_map(mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, k, kvdims, kvstrides, kbox);
  if (rc) return rc;
  return make_map(mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, v, kvdims, kvstrides, vbox);
}

template <bool E4M3>
int attention_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, int64_t batch,
                     int64_t tokens, int64_t heads, const ogx::attn::Params& p, cudaStream_t s) {
  if (attn_use_pairs()) {
    auto kern = attn_pairs_mode() == 2 ? ogx::attn::attn_fwd_pair_kernel<E4M3, true>
                                       : ogx::attn::attn_fwd_pair_kernel<E4M3, false>;
    int rc = ensure_smem(kern, ogx::attn::PAIR_SMEM_BYTES);
    if (rc) return rc;
    // one pair of CTAs (a cluster of two) per 256 queries and head
    const dim3 grid(static_cast<unsigned>(2 * ((tokens + 255) / 256)), static_cast<unsigned>(heads),
                    static_cast<unsigned>(batch));
    launch_cluster(kern, grid, dim3(ogx::attn::kPairThreads), ogx::attn::PAIR_SMEM_BYTES, s, 2u, mq, mk, mv, p);
    return check_launch("attn_fwd_pair_kernel");
  }
  auto kern = ogx::attn::attn_fwd_kernel<E4M3>;
  int rc = ensure_smem(kern, ogx::attn::SMEM_BYTES);
  if (rc) return rc;
  // The softmax warpgroups raise their register limit with setmaxnreg, drawing on the registers the
  // launch reserved; only launch a build whose per-thread count is the one the split was sized for.
  cudaFuncAttributes attr;
  rc = check_cuda(cudaFuncGetAttributes(&attr, kern), "cudaFuncGetAttributes");
  if (rc) return rc;
  if (attr.numRegs != ogx::attn::kLaunchRegs)
    return fail(OGX_ECUDA, "attention kernel built with %d registers per thread, the register split needs %d", attr.numRegs,
                ogx::attn::kLaunchRegs);
  const dim3 grid(static_cast<unsigned>((tokens + 255) / 256), static_cast<unsigned>(heads),
                  static_cast<unsigned>(batch));
  launch(kern, grid, ogx::attn::kThreads, ogx::attn::SMEM_BYTES, s, mq, mk, mv, p);
  return check_launch("attn_fwd_kernel");
}

}  // namespace

extern "C" {

int ogx_fp8_scaled_mm(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N, int64_t ldw,
                      const float* scale_a, const float* scale_b, int64_t n_per_scale, const void* bias,
                      int bias_dtype, void* out, int64_t ldo, void* stream) {
  CUtensorMap ma, mb;
  int rc = gemm_common(a, M, K, lda, w, N, ldw, scale_a, scale_b, n_per_scale, &ma, &mb);
  if (rc || M == 0) return rc;
  if (out == nullptr || !aligned16(out) || ldo % 8 || ldo < N) return fail(OGX_EINVAL, "output");
  if (bias != nullptr && (!dtype_ok(bias_dtype) || !aligned16(bias))) return fail(OGX_EINVAL, "bias");
  ogx::gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.scale_a = scale_a;
  p.scale_b = scale_b;
  p.n_per_scale = static_cast<int>(n_per_scale);
  p.bias = bias;
  p.bias_fp32 = bias_dtype == OGX_DTYPE_F32;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  return gemm_launch<ogx::gemm::EPI_BIAS>(ma, mb, p, static_cast<cudaStream_t>(stream));
}

int ogx_fp8_scaled_mm_planes(const void* a, int64_t planes, int64_t M, int64_t K, int64_t lda, const void* w,
                             int64_t N, int64_t ldw, const float* scale_a, const float* scale_b, const void* bias,
                             int bias_dtype, void* out, int64_t ldo, void* stream) {
  if (planes < 1 || planes > 8) return fail(OGX_EINVAL, "a_planes: 1 to 8 planes");
  if (N % planes) return fail(OGX_EINVAL, "a_planes: N must split into planes of a multiple of %d columns",
                              ogx::gemm::BN);
  CUtensorMap ma, mb;
  int rc = gemm_common(a, M, K, lda, w, N, ldw, scale_a, scale_b, N / planes, &ma, &mb, 0, planes);
  if (rc || M == 0) return rc;
  if (out == nullptr || !aligned16(out) || ldo % 8 || ldo < N) return fail(OGX_EINVAL, "output");
  if (bias != nullptr && (!dtype_ok(bias_dtype) || !aligned16(bias))) return fail(OGX_EINVAL, "bias");
  ogx::gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.a_planes = static_cast<int>(planes);
  p.scale_a = scale_a;
  p.scale_b = scale_b;
  p.n_per_scale = static_cast<int>(N / planes);
  p.bias = bias;
  p.bias_fp32 = bias_dtype == OGX_DTYPE_F32;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  return gemm_launch<ogx::gemm::EPI_BIAS>(ma, mb, p, static_cast<cudaStream_t>(stream));
}

int ogx_fp8_scaled_mm_gelu_e4m3(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N,
                                int64_t ldw, const float* scale_a, const float* scale_b, int64_t n_per_scale,
                                const void* bias, int bias_dtype, const float* q_scale, void* out_q, int64_t ldq,
                                void* stream) {
  CUtensorMap ma, mb;
  int rc = gemm_common(a, M, K, lda, w, N, ldw, scale_a, scale_b, n_per_scale, &ma, &mb);
  if (rc || M == 0) return rc;
  if (out_q == nullptr || q_scale == nullptr || !aligned16(out_q) || ldq % 16 || ldq < N)
    return fail(OGX_EINVAL, "output");
  if (bias != nullptr && (!dtype_ok(bias_dtype) || !aligned16(bias))) return fail(OGX_EINVAL, "bias");
  ogx::gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.scale_a = scale_a;
  p.scale_b = scale_b;
  p.n_per_scale = static_cast<int>(n_per_scale);
  p.bias = bias;
  p.bias_fp32 = bias_dtype == OGX_DTYPE_F32;
  p.out_q = static_cast<uint8_t*>(out_q);
  p.ldq = ldq;
  p.q_scale = q_scale;
  return gemm_launch<ogx::gemm::EPI_GELU_QUANT>(ma, mb, p, static_cast<cudaStream_t>(stream));
}

static int residual_gate_impl(int64_t a_k_block, const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N,
                                    int64_t ldw, const float* scale_a, const float* scale_b, int64_t n_per_scale,
                                    const void* bias, int bias_dtype, const void* x, int64_t ldx,
                                    const void* table, int table_dtype, int64_t table_stride_row,
                                    const void* timestep, int timestep_dtype, int64_t ts_stride_t,
                                    int64_t ts_stride_p, int gate_index, void* out, int64_t ldo, void* stream) {
  CUtensorMap ma, mb;
  int rc = gemm_common(a, M, K, lda, w, N, ldw, scale_a, scale_b, n_per_scale, &ma, &mb, a_k_block);
  if (rc || M == 0) return rc;
  if (out == nullptr || !aligned16(out) || ldo % 8 || ldo < N) return fail(OGX_EINVAL, "output");
  if (bias != nullptr && (!dtype_ok(bias_dtype) || !aligned16(bias))) return fail(OGX_EINVAL, "bias");
  if (x == nullptr || !aligned16(x) || ldx % 8 || ldx < N) return fail(OGX_EINVAL, "residual");
  if (table == nullptr || timestep == nullptr || !dtype_ok(table_dtype) || !dtype_ok(timestep_dtype) ||
      gate_index < 0)
    return fail(OGX_EINVAL, "ada");
  const int tesz = timestep_dtype == OGX_DTYPE_F32 ? 4 : 2;
  const int tbsz = table_dtype == OGX_DTYPE_F32 ? 4 : 2;
  if (!aligned16(table) || !aligned16(timestep) || (ts_stride_t * tesz) % 16 || (ts_stride_p * tesz) % 16 ||
      (table_stride_row * tbsz) % 16)
    return fail(OGX_EINVAL, "timestep_stride");
  ogx::gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.scale_a = scale_a;
  p.scale_b = scale_b;
  p.n_per_scale = static_cast<int>(n_per_scale);
  p.bias = bias;
  p.bias_fp32 = bias_dtype == OGX_DTYPE_F32;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.resid_x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.table = table;
  p.table_fp32 = table_dtype == OGX_DTYPE_F32;
  p.table_stride_row = table_stride_row;
  p.ts = timestep;
  p.ts_fp32 = timestep_dtype == OGX_DTYPE_F32;
  p.ts_stride_t = ts_stride_t;
  p.ts_stride_p = ts_stride_p;
  p.gate_index = gate_index;
  p.a_k_block = static_cast<int>(a_k_block);
  return gemm_launch<ogx::gemm::EPI_RESIDUAL>(ma, mb, p, static_cast<cudaStream_t>(stream));
}

int ogx_fp8_scaled_mm_residual_gate(const void* a, int64_t M, int64_t K, int64_t lda, const void* w, int64_t N,
                                    int64_t ldw, const float* scale_a, const float* scale_b, int64_t n_per_scale,
                                    const void* bias, int bias_dtype, const void* x, int64_t ldx,
                                    const void* table, int table_dtype, int64_t table_stride_row,
                                    const void* timestep, int timestep_dtype, int64_t ts_stride_t,
                                    int64_t ts_stride_p, int gate_index, void* out, int64_t ldo, void* stream) {
  return residual_gate_impl(0, a, M, K, lda, w, N, ldw, scale_a, scale_b, n_per_scale, bias, bias_dtype, x, ldx, table,
                            table_dtype, table_stride_row, timestep, timestep_dtype, ts_stride_t, ts_stride_p,
                            gate_index, out, ldo, stream);
}

int ogx_fp8_scaled_mm_residual_gate_kblocked(const void* a, int64_t M, int64_t K, int64_t k_block, const void* w,
                                             int64_t N, int64_t ldw, const float* scale_a, const float* scale_b,
                                             int64_t n_per_scale, const void* bias, int bias_dtype, const void* x,
                                             int64_t ldx, const void* table, int table_dtype,
                                             int64_t table_stride_row, const void* timestep, int timestep_dtype,
                                             int64_t ts_stride_t, int64_t ts_stride_p, int gate_index, void* out,
                                             int64_t ldo, void* stream) {
  if (k_block <= 0) return fail(OGX_EINVAL, "a_k_block");
  return residual_gate_impl(k_block, a, M, K, k_block, w, N, ldw, scale_a, scale_b, n_per_scale, bias, bias_dtype, x,
                            ldx, table, table_dtype, table_stride_row, timestep, timestep_dtype, ts_stride_t,
                            ts_stride_p, gate_index, out, ldo, stream);
}

int ogx_attention_fwd(const void* q, const void* k, const void* v, int64_t batch, int64_t tokens, int64_t heads,
                      int64_t head_dim, int64_t stride_b, int64_t stride_t, float softmax_scale, void* out,
                      int64_t out_stride_b, int64_t out_stride_t, void* stream) {
  CUtensorMap mq, mk, mv;
  int rc = attention_common(q, k, v, batch, tokens, tokens, heads, head_dim, stride_b, stride_t, stride_b, stride_t,
                            &mq, &mk, &mv);
  if (rc) return rc;
  if (out == nullptr || !aligned16(out) || out_stride_t % 8 || out_stride_b % 8) return fail(OGX_EINVAL, "output");
  ogx::attn::Params p{};
  p.L = static_cast<int>(tokens);
  p.L_kv = p.L;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_b = out_stride_b;
  p.out_stride_t = out_stride_t;
  return attention_launch<false>(mq, mk, mv, batch, tokens, heads, p, static_cast<cudaStream_t>(stream));
}

int ogx_attention_fwd_e4m3(const void* q, const void* k, const void* v, int64_t batch, int64_t tokens,
                           int64_t heads, int64_t head_dim, int64_t stride_b, int64_t stride_t, float softmax_scale,
                           const float* out_scale, void* out_q, int64_t out_stride_b, int64_t out_stride_t,
                           void* stream) {
  CUtensorMap mq, mk, mv;
  int rc = attention_common(q, k, v, batch, tokens, tokens, heads, head_dim, stride_b, stride_t, stride_b, stride_t,
                            &mq, &mk, &mv);
  if (rc) return rc;
  if (out_q == nullptr || out_scale == nullptr || !aligned16(out_q) || out_stride_t % 16 || out_stride_b % 16)
    return fail(OGX_EINVAL, "output");
  ogx::attn::Params p{};
  p.L = static_cast<int>(tokens);
  p.L_kv = p.L;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.out_q = static_cast<uint8_t*>(out_q);
  p.out_scale = out_scale;
  p.out_stride_b = out_stride_b;
  p.out_stride_t = out_stride_t;
  return attention_launch<true>(mq, mk, mv, batch, tokens, heads, p, static_cast<cudaStream_t>(stream));
}

int ogx_attention_fwd_kv(const void* q, const void* k, const void* v, int64_t batch, int64_t q_tokens,
                         int64_t kv_tokens, int64_t heads, int64_t head_dim, int64_t q_stride_b, int64_t q_stride_t,
                         int64_t kv_stride_b, int64_t kv_stride_t, float softmax_scale, void* out,
                         int64_t out_stride_b, int64_t out_stride_t, void* stream) {
  CUtensorMap mq, mk, mv;
  int rc = attention_common(q, k, v, batch, q_tokens, kv_tokens, heads, head_dim, q_stride_b, q_stride_t, kv_stride_b,
                            kv_stride_t, &mq, &mk, &mv);
  if (rc) return rc;
  if (out == nullptr || !aligned16(out) || out_stride_t % 8 || out_stride_b % 8) return fail(OGX_EINVAL, "output");
  ogx::attn::Params p{};
  p.L = static_cast<int>(q_tokens);
  p.L_kv = static_cast<int>(kv_tokens);
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_b = out_stride_b;
  p.out_stride_t = out_stride_t;
  return attention_launch<false>(mq, mk, mv, batch, q_tokens, heads, p, static_cast<cudaStream_t>(stream));
}

int ogx_attention_fwd_kv_e4m3(const void* q, const void* k, const void* v, int64_t batch, int64_t q_tokens,
                              int64_t kv_tokens, int64_t heads, int64_t head_dim, int64_t q_stride_b,
                              int64_t q_stride_t, int64_t kv_stride_b, int64_t kv_stride_t, float softmax_scale,
                              const float* out_scale, void* out_q, int64_t out_stride_b, int64_t out_stride_t,
                              void* stream) {
  CUtensorMap mq, mk, mv;
  int rc = attention_common(q, k, v, batch, q_tokens, kv_tokens, heads, head_dim, q_stride_b, q_stride_t, kv_stride_b,
                            kv_stride_t, &mq, &mk, &mv);
  if (rc) return rc;
  if (out_q == nullptr || out_scale == nullptr || !aligned16(out_q) || out_stride_t % 16 || out_stride_b % 16)
    return fail(OGX_EINVAL, "output");
  ogx::attn::Params p{};
  p.L = static_cast<int>(q_tokens);
  p.L_kv = static_cast<int>(kv_tokens);
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.out_q = static_cast<uint8_t*>(out_q);
  p.out_scale = out_scale;
  p.out_stride_b = out_stride_b;
  p.out_stride_t = out_stride_t;
  return attention_launch<true>(mq, mk, mv, batch, q_tokens, heads, p, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ------------------------------------------------------------- peer exchange over NVLink
extern "C" {

int ogx_ipc_get_handle(const void* ptr, void* handle, int64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return fail(OGX_EINVAL, "null_pointer");
  auto fn = address_range_fn();
  if (fn == nullptr) return fail(OGX_ECUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(OGX_EINVAL, "pointer is not device memory");
  cudaIpcMemHandle_t h;
  int rc = check_cuda(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  if (rc) return rc;
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return OGX_OK;
}

int ogx_ipc_open_handle(const void* handle, void** base) {
  if (handle == nullptr || base == nullptr) return fail(OGX_EINVAL, "null_pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int ogx_ipc_close_handle(void* base) {
  if (base == nullptr) return fail(OGX_EINVAL, "null_pointer");
  return check_cuda(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

int ogx_peer_barrier(unsigned int* local_signals, void* const* peer_signals, int rank, int world, void* stream) {
  if (local_signals == nullptr || peer_signals == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (world < 1 || world > 8 || rank < 0 || rank >= world) return fail(OGX_EINVAL, "world");
  ogx::PeerSignals ps{};
  for (int i = 0; i < world; ++i) {
    if (peer_signals[i] == nullptr) return fail(OGX_EINVAL, "null_pointer");
    ps.slot[i] = static_cast<unsigned int*>(peer_signals[i]);
  }
  launch(ogx::peer_barrier_kernel, 1, 32, 0, static_cast<cudaStream_t>(stream), local_signals, ps, rank, world);
  return check_launch("peer_barrier_kernel");
}

}  // extern "C"

namespace {

int rope_to_peers_impl(const void* q, const void* k, const void* v, int64_t tokens, int64_t in_stride_t,
                       const void* q_weight, const void* k_weight, int weight_dtype, float eps, const void* cos,
                       const void* sin, int cs_dtype, int64_t cs_stride_h, int64_t cs_stride_t,
                       const ogx::rows::RopeSource* src, void* const* group_bases, int groups, int64_t out_stride_t,
                       void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || group_bases == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (groups < 1 || groups > 8 || 32 % groups) return fail(OGX_EINVAL, "groups");
  const int hpg = 32 / groups;
  if (q_weight == nullptr || k_weight == nullptr) return fail(OGX_EINVAL, "qk_weight_shape");
  if (src == nullptr && (cos == nullptr || sin == nullptr)) return fail(OGX_EINVAL, "rope_shape");
  if (tokens < 1) return fail(OGX_EINVAL, "empty_tokens");
  if (!dtype_ok(weight_dtype) || (src == nullptr && !dtype_ok(cs_dtype))) return fail(OGX_EINVAL, "qk_device_or_dtype");
  if (in_stride_t % 8 || out_stride_t % 8 || out_stride_t < 3 * hpg * 128) return fail(OGX_EINVAL, "qk_noncontiguous");
  if (src == nullptr) {
    const int cesz = cs_dtype == OGX_DTYPE_F32 ? 4 : 2;
    if ((cs_stride_h * cesz) % 16 || (cs_stride_t * cesz) % 16) return fail(OGX_EINVAL, "rope_shape");
    if (!aligned16(cos) || !aligned16(sin)) return fail(OGX_EINVAL, "alignment");
  }
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(q_weight) || !aligned16(k_weight))
    return fail(OGX_EINVAL, "alignment");
  ogx::RopeArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.in_stride_t = in_stride_t;
  a.q_weight = q_weight;
  a.k_weight = k_weight;
  a.cos = cos;
  a.sin = sin;
  a.cs_stride_h = cs_stride_h;
  a.cs_stride_t = cs_stride_t;
  a.tokens = tokens;
  a.eps = eps;
  for (int g = 0; g < groups; ++g) {
    if (group_bases[g] == nullptr || !aligned16(group_bases[g])) return fail(OGX_EINVAL, "alignment");
    auto* base = static_cast<__nv_bfloat16*>(group_bases[g]);
    a.dst[0][g] = base;
    a.dst[1][g] = base + hpg * 128;
    a.dst[2][g] = base + 2 * hpg * 128;
  }
  a.out_stride_t = out_stride_t;
  a.heads_per_group = hpg;
  a.copy_v = 1;
  a.system_fence = 1;
  return rope_dispatch(a, src, weight_dtype, cs_dtype, static_cast<cudaStream_t>(stream));
}

}  // namespace

extern "C" {

int ogx_video_qkv_rmsnorm_rope_to_peers(const void* q, const void* k, const void* v, int64_t tokens,
                                        int64_t in_stride_t, const void* q_weight, const void* k_weight,
                                        int weight_dtype, float eps, const void* cos, const void* sin, int cs_dtype,
                                        int64_t cs_stride_h, int64_t cs_stride_t, void* const* group_bases,
                                        int groups, int64_t out_stride_t, void* stream) {
  return rope_to_peers_impl(q, k, v, tokens, in_stride_t, q_weight, k_weight, weight_dtype, eps, cos, sin, cs_dtype,
                            cs_stride_h, cs_stride_t, nullptr, group_bases, groups, out_stride_t, stream);
}

int ogx_video_qkv_rmsnorm_rope_positions_to_peers(const void* q, const void* k, const void* v, int64_t tokens,
                                                  int64_t in_stride_t, const void* q_weight, const void* k_weight,
                                                  int weight_dtype, float eps, const double* inv_freq,
                                                  const unsigned char* slot_axis, int64_t grid_h, int64_t grid_w,
                                                  int64_t token0, void* const* group_bases, int groups,
                                                  int64_t out_stride_t, void* stream) {
  ogx::rows::RopeSource src{};
  const int rc = rope_source(inv_freq, slot_axis, grid_h, grid_w, token0, &src);
  if (rc) return rc;
  return rope_to_peers_impl(q, k, v, tokens, in_stride_t, q_weight, k_weight, weight_dtype, eps, nullptr, nullptr,
                            OGX_DTYPE_BF16, 0, 0, &src, group_bases, groups, out_stride_t, stream);
}

int ogx_attention_fwd_e4m3_to_peers(const void* q, const void* k, const void* v, int64_t tokens, int64_t heads,
                                    int64_t stride_t, float softmax_scale, const float* out_scale,
                                    void* const* peer_bases, int peers, int64_t tokens_per_peer,
                                    int64_t out_stride_t, void* stream) {
  CUtensorMap mq, mk, mv;
  int rc = attention_common(q, k, v, 1, tokens, tokens, heads, 128, tokens * stride_t, stride_t, tokens * stride_t,
                            stride_t, &mq, &mk, &mv);
  if (rc) return rc;
  if (peer_bases == nullptr || out_scale == nullptr || peers < 1 || peers > 8) return fail(OGX_EINVAL, "peers");
  if (tokens_per_peer < 1 || tokens_per_peer * peers != tokens) return fail(OGX_EINVAL, "tokens_per_peer");
  if (out_stride_t % 16 || out_stride_t < heads * 128) return fail(OGX_EINVAL, "output");
  ogx::attn::Params p{};
  p.L = static_cast<int>(tokens);
  p.L_kv = p.L;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.out_scale = out_scale;
  p.out_stride_t = out_stride_t;
  p.peer_tokens = static_cast<int>(tokens_per_peer);
  for (int i = 0; i < peers; ++i) {
    if (peer_bases[i] == nullptr || !aligned16(peer_bases[i])) return fail(OGX_EINVAL, "output");
    p.out_peer[i] = static_cast<uint8_t*>(peer_bases[i]);
  }
  p.out_q = p.out_peer[0];
  return attention_launch<true>(mq, mk, mv, 1, tokens, heads, p, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------
// Cross-GPU barrier without caller-allocated memory.
//
// ogx_peer_barrier needs a 16-word signal block per rank, allocated by the caller.  Some callers
// cannot allocate device memory: a runtime that drives all of its GPUs from one process and reserves
// their memory up front for its own pool, so that no cudaMalloc may run once serving has started.
// For them the barrier count lives in a file-scope device array (one per GPU that loads the library,
// 64 bytes, held until the process exits) and the arrival slots in one page of host memory inside the
// library, page-locked and mapped into every GPU of the process at the first call.  No GPU touches another
// GPU's memory, so the ranks need no peer access between them; ogx_peer_barrier_static takes the ranks'
// device ordinals instead of block pointers.
namespace {

// [8] barriers passed on this device; zero when the library loads and never cleared after: the barrier
// numbers only grow, so no call needs it zeroed again.
static __device__ __align__(256) unsigned int g_static_peer_block[ogx::kPeerSignalWords];

constexpr int kMaxDevices = 64;

// The arrival slots: row d (kPeerSignalWords words) of device d, word r the latest barrier number rank r
// announced to it.  One 4 KB page.
alignas(4096) unsigned int g_static_host_slots[kMaxDevices * ogx::kPeerSignalWords];
static_assert(sizeof(g_static_host_slots) == 4096, "one page of arrival slots");

// Device address of g_static_peer_block on `dev`, looked up once per device with that device current.
int static_peer_block(int dev, unsigned int** out) {
  static std::mutex mu;
  static unsigned int* addr[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return fail(OGX_EINVAL, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    int prev = 0;
    int rc = check_cuda(cudaGetDevice(&prev), "cudaGetDevice");
    if (rc) return rc;
    rc = check_cuda(cudaSetDevice(dev), "cudaSetDevice");
    if (rc) return rc;
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_peer_block);
    cudaSetDevice(prev);
    rc = check_cuda(e, "cudaGetSymbolAddress");
    if (rc) return rc;
    addr[dev] = static_cast<unsigned int*>(p);
  }
  *out = addr[dev];
  return OGX_OK;
}

// The device address of the arrival slots (the same in every GPU of the process: portable, mapped
// page-locked memory under unified addressing), page-locked once per process.
int static_host_slots(unsigned int** out) {
  static std::mutex mu;
  static unsigned int* dev_ptr = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (dev_ptr == nullptr) {
    cudaError_t e = cudaHostRegister(g_static_host_slots, sizeof(g_static_host_slots),
                                     cudaHostRegisterPortable | cudaHostRegisterMapped);
    if (e == cudaErrorHostMemoryAlreadyRegistered) {
      cudaGetLastError();
    } else if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(OGX_ECUDA, "cudaHostRegister of the barrier's arrival slots: %s", cudaGetErrorString(e));
    }
    void* p = nullptr;
    const int rc = check_cuda(cudaHostGetDevicePointer(&p, g_static_host_slots, 0), "cudaHostGetDevicePointer");
    if (rc) return rc;
    dev_ptr = static_cast<unsigned int*>(p);
  }
  *out = dev_ptr;
  return OGX_OK;
}

}  // namespace

extern "C" {

int ogx_peer_barrier_static(int rank, int world, const int* devices, unsigned int* count_out, void* stream) {
  if (devices == nullptr) return fail(OGX_EINVAL, "null_pointer");
  if (world < 1 || world > 8)
    return fail(OGX_EINVAL, "world: the static barrier holds at most 8 ranks (got %d)", world);
  if (rank < 0 || rank >= world) return fail(OGX_EINVAL, "world: rank %d outside [0, %d)", rank, world);
  int cur = 0;
  int rc = check_cuda(cudaGetDevice(&cur), "cudaGetDevice");
  if (rc) return rc;
  if (devices[rank] != cur)
    return fail(OGX_EINVAL, "devices[rank] is %d but the current device is %d", devices[rank], cur);
  ogx::DeviceList devs{};
  for (int i = 0; i < world; ++i) {
    if (devices[i] < 0 || devices[i] >= kMaxDevices)
      return fail(OGX_EINVAL, "device ordinal %d out of range", devices[i]);
    devs.d[i] = devices[i];
  }
  // Two ranks on one ordinal would share one arrival row and one count: their barrier numbers would drift
  // apart and every later wait would run out.
  for (int i = 0; i < world; ++i)
    for (int j = i + 1; j < world; ++j)
      if (devices[i] == devices[j])
        return fail(OGX_EINVAL, "devices: ranks %d and %d both name device %d", i, j, devices[i]);
  unsigned int* local = nullptr;
  rc = static_peer_block(cur, &local);
  if (rc) return rc;
  unsigned int* slots = nullptr;
  rc = static_host_slots(&slots);
  if (rc) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  ogx::host_slot_barrier_kernel<<<1, 32, 0, s>>>(local, slots, devs, rank, world);
  rc = check_launch("host_slot_barrier_kernel");
  if (rc || count_out == nullptr) return rc;
  return check_cuda(cudaMemcpyAsync(count_out, local + ogx::kPeerCountWord, sizeof(unsigned int),
                                    cudaMemcpyDeviceToDevice, s),
                    "cudaMemcpyAsync");
}

}  // extern "C"
