// Kernel (1b): Veda predictor tile logits (core/predictor.py:63-80):
//   x_hat = F @ P[h] + F[:, :128]      (F = [mean | max | min], 384 wide)
//   logits[h, i, j] = q_hat_i . k_hat_j / sqrt(128)
// fp32 on CUDA cores: about 1.2 GFLOP for 24 heads x 256 tiles, far below
// anything worth a tensor-core pipeline, and fp32 keeps the logits (and so
// the selection) within rounding of the reference's fp32 bmm.

#include <cuda_fp8.h>

#include "common.cuh"

namespace veda {
namespace {

constexpr int kFeat = 3 * kDim;   // 384
constexpr int kProjRows = 16;     // rows of F per CTA in the projection
constexpr int kLogitTile = 32;    // 32 x 32 logits per CTA

template <typename PT>
__device__ __forceinline__ float to_f(PT v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f<__nv_fp8_e4m3>(__nv_fp8_e4m3 v) {
  return static_cast<float>(v);
}

// A projection weight as the scoring arithmetic sees it. fp8 weights carry a
// per-head scale and become bf16(w * scale) in fp32, which is what the
// reference's bundle loader stores for them (core/bundle.py:176-180: the
// fp32 product rounded to bf16) before its fp32 bmm.
template <typename PT>
__device__ __forceinline__ float weight(PT v, float scale) {
  return to_f(v);
}
template <>
__device__ __forceinline__ float weight<__nv_fp8_e4m3>(__nv_fp8_e4m3 v,
                                                      float scale) {
  return __bfloat162float(__float2bfloat16_rn(to_f(v) * scale));
}

// grid (ceil(n / 16), heads, 2): z = 0 projects q features, z = 1 k.
// sq / sk: per-head scales of fp8 projections (unused otherwise).
template <typename PT>
__global__ void __launch_bounds__(256)
    project_kernel(const float* fq, const float* fk, const PT* pq,
                   const PT* pk, const float* sq, const float* sk, int n_q,
                   int n_k, float* hat_q, float* hat_k) {
  __shared__ float f_sh[kProjRows][kFeat];
  const bool is_k = blockIdx.z == 1;
  const int n = is_k ? n_k : n_q;
  const int head = blockIdx.y;
  const int row0 = blockIdx.x * kProjRows;
  if (row0 >= n) return;
  const float* f = (is_k ? fk : fq) + (static_cast<int64_t>(head) * n + row0) * kFeat;
  const PT* proj = (is_k ? pk : pq) + static_cast<int64_t>(head) * kFeat * kDim;
  const float* scales = is_k ? sk : sq;
  const float scale = scales != nullptr ? scales[head] : 1.0f;
  float* out = (is_k ? hat_k : hat_q) + (static_cast<int64_t>(head) * n + row0) * kDim;
  const int rows = min(kProjRows, n - row0);
  for (int i = threadIdx.x; i < kProjRows * kFeat; i += blockDim.x) {
    const int r = i / kFeat;
    f_sh[r][i % kFeat] = r < rows ? f[i] : 0.0f;
  }
  __syncthreads();
  const int d = threadIdx.x & (kDim - 1);
  const int r0 = (threadIdx.x >> 7) * (kProjRows / 2);
  float acc[kProjRows / 2];
#pragma unroll
  for (int r = 0; r < kProjRows / 2; ++r) acc[r] = 0.0f;
  for (int k = 0; k < kFeat; ++k) {
    const float w = weight(proj[static_cast<int64_t>(k) * kDim + d], scale);
#pragma unroll
    for (int r = 0; r < kProjRows / 2; ++r)
      acc[r] = fmaf(f_sh[r0 + r][k], w, acc[r]);
  }
#pragma unroll
  for (int r = 0; r < kProjRows / 2; ++r)
    if (r0 + r < rows) out[(r0 + r) * kDim + d] = acc[r] + f_sh[r0 + r][d];
}

// grid (ceil(n_k / 32), ceil(n_q / 32), heads), 256 threads, 4 logits each.
__global__ void __launch_bounds__(256)
    logits_kernel(const float* hat_q, const float* hat_k, int n_q, int n_k,
                  float* logits) {
  __shared__ float q_sh[kLogitTile][kDim + 1];
  __shared__ float k_sh[kLogitTile][kDim + 1];
  const int head = blockIdx.z;
  const int i0 = blockIdx.y * kLogitTile, j0 = blockIdx.x * kLogitTile;
  const float* qh = hat_q + static_cast<int64_t>(head) * n_q * kDim;
  const float* kh = hat_k + static_cast<int64_t>(head) * n_k * kDim;
  for (int e = threadIdx.x; e < kLogitTile * kDim; e += blockDim.x) {
    const int r = e / kDim, c = e % kDim;
    q_sh[r][c] = i0 + r < n_q ? qh[static_cast<int64_t>(i0 + r) * kDim + c] : 0.0f;
    k_sh[r][c] = j0 + r < n_k ? kh[static_cast<int64_t>(j0 + r) * kDim + c] : 0.0f;
  }
  __syncthreads();
  const int tj = threadIdx.x & 31;
  const int ti = (threadIdx.x >> 5) * 4;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int c = 0; c < kDim; ++c) {
    const float kv = k_sh[tj][c];
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r] = fmaf(q_sh[ti + r][c], kv, acc[r]);
  }
  const float root = 11.313708498984761f;  // sqrt(128)
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = i0 + ti + r, j = j0 + tj;
    if (i < n_q && j < n_k)
      logits[(static_cast<int64_t>(head) * n_q + i) * n_k + j] =
          __fdiv_rn(acc[r], root);
  }
}

// Scratch of veda_tile_logits_static: the projected features (q_hat, k_hat)
// of at most VEDA_STATIC_LOGITS_ROWS rows, 8 MiB in every device context
// that loads this library. Nothing in it needs to start at zero: each call's
// projection writes every element its logits then read.
static __device__ __align__(256) float g_static_logits_scratch[
    static_cast<int64_t>(VEDA_STATIC_LOGITS_ROWS) * kDim];

// Address of the scratch in the current device's context. It is looked up on
// every call rather than cached: after a device reset the module is loaded
// again and the array may sit at another address.
int static_scratch(float** out) {
  void* address = nullptr;
  const cudaError_t err =
      cudaGetSymbolAddress(&address, g_static_logits_scratch);
  if (err != cudaSuccess)
    return cuda_fail(err, "cudaGetSymbolAddress(static logits scratch)");
  *out = static_cast<float*>(address);
  return VEDA_OK;
}

int check_logits_args(const float* feats_q, const float* feats_k,
                      const void* proj_q, const void* proj_k, int heads,
                      int n_q, int n_k, const float* logits) {
  if (heads <= 0 || heads > 65535 || n_q <= 0 || n_k <= 0)
    return fail(VEDA_ERR_INVALID, "bad sizes: heads %d, n_q %d, n_k %d", heads,
                n_q, n_k);
  if (feats_q == nullptr || feats_k == nullptr || proj_q == nullptr ||
      proj_k == nullptr || logits == nullptr)
    return fail(VEDA_ERR_INVALID, "null pointer argument");
  return VEDA_OK;
}

int launch_tile_logits(const float* feats_q, const float* feats_k,
                       const void* proj_q, const void* proj_k, int proj_dtype,
                       const float* scale_q, const float* scale_k, int heads,
                       int n_q, int n_k, float* workspace, float* logits,
                       cudaStream_t s) {
  float* hat_q = workspace;
  float* hat_k = workspace + static_cast<int64_t>(heads) * n_q * kDim;
  const int n_max = n_q > n_k ? n_q : n_k;
  dim3 pgrid((n_max + kProjRows - 1) / kProjRows, heads, 2);
  switch (proj_dtype) {
    case VEDA_BF16:
      project_kernel<__nv_bfloat16><<<pgrid, 256, 0, s>>>(
          feats_q, feats_k, static_cast<const __nv_bfloat16*>(proj_q),
          static_cast<const __nv_bfloat16*>(proj_k), nullptr, nullptr, n_q,
          n_k, hat_q, hat_k);
      break;
    case VEDA_F16:
      project_kernel<__half><<<pgrid, 256, 0, s>>>(
          feats_q, feats_k, static_cast<const __half*>(proj_q),
          static_cast<const __half*>(proj_k), nullptr, nullptr, n_q, n_k,
          hat_q, hat_k);
      break;
    case VEDA_F32:
      project_kernel<float><<<pgrid, 256, 0, s>>>(
          feats_q, feats_k, static_cast<const float*>(proj_q),
          static_cast<const float*>(proj_k), nullptr, nullptr, n_q, n_k,
          hat_q, hat_k);
      break;
    case VEDA_FP8_E4M3:
      if (scale_q == nullptr || scale_k == nullptr)
        return fail(VEDA_ERR_INVALID, "fp8 projections need per-head scales");
      project_kernel<__nv_fp8_e4m3><<<pgrid, 256, 0, s>>>(
          feats_q, feats_k, static_cast<const __nv_fp8_e4m3*>(proj_q),
          static_cast<const __nv_fp8_e4m3*>(proj_k), scale_q, scale_k, n_q,
          n_k, hat_q, hat_k);
      break;
    default:
      return fail(VEDA_ERR_INVALID,
                  "proj dtype must be bf16, fp16, fp32 or fp8 e4m3");
  }
  VEDA_CHECK_CUDA(cudaGetLastError());
  dim3 lgrid((n_k + kLogitTile - 1) / kLogitTile,
             (n_q + kLogitTile - 1) / kLogitTile, heads);
  logits_kernel<<<lgrid, 256, 0, s>>>(hat_q, hat_k, n_q, n_k, logits);
  VEDA_CHECK_CUDA(cudaGetLastError());
  return VEDA_OK;
}

}  // namespace
}  // namespace veda

using namespace veda;

extern "C" int veda_tile_logits(const float* feats_q, const float* feats_k,
                                const void* proj_q, const void* proj_k,
                                int proj_dtype, int heads, int n_q, int n_k,
                                float* workspace, float* logits,
                                void* stream) {
  if (int rc = check_device()) return rc;
  if (int rc = check_logits_args(feats_q, feats_k, proj_q, proj_k, heads, n_q,
                                 n_k, logits))
    return rc;
  if (workspace == nullptr) return fail(VEDA_ERR_INVALID, "null workspace");
  if (proj_dtype == VEDA_FP8_E4M3)
    return fail(VEDA_ERR_INVALID,
                "fp8 projections go through veda_tile_logits_scaled");
  return launch_tile_logits(feats_q, feats_k, proj_q, proj_k, proj_dtype,
                            nullptr, nullptr, heads, n_q, n_k, workspace,
                            logits, static_cast<cudaStream_t>(stream));
}

extern "C" int veda_tile_logits_scaled(const float* feats_q,
                                       const float* feats_k,
                                       const void* proj_q, const void* proj_k,
                                       int proj_dtype, const float* scale_q,
                                       const float* scale_k, int heads,
                                       int n_q, int n_k, float* workspace,
                                       float* logits, void* stream) {
  if (int rc = check_device()) return rc;
  if (int rc = check_logits_args(feats_q, feats_k, proj_q, proj_k, heads, n_q,
                                 n_k, logits))
    return rc;
  if (workspace == nullptr) return fail(VEDA_ERR_INVALID, "null workspace");
  return launch_tile_logits(feats_q, feats_k, proj_q, proj_k, proj_dtype,
                            scale_q, scale_k, heads, n_q, n_k, workspace,
                            logits, static_cast<cudaStream_t>(stream));
}

extern "C" int veda_tile_logits_static(const float* feats_q,
                                       const float* feats_k,
                                       const void* proj_q, const void* proj_k,
                                       int proj_dtype, int heads, int n_q,
                                       int n_k, float* logits, void* stream) {
  // Sizes first, before anything touches a device: a call past the limit
  // is the caller's error whatever the device.
  if (int rc = check_logits_args(feats_q, feats_k, proj_q, proj_k, heads, n_q,
                                 n_k, logits))
    return rc;
  const int64_t rows = (static_cast<int64_t>(n_q) + n_k) * heads;
  if (n_q > VEDA_STATIC_LOGITS_ROWS || n_k > VEDA_STATIC_LOGITS_ROWS ||
      rows > VEDA_STATIC_LOGITS_ROWS)
    return fail(VEDA_ERR_INVALID,
                "(n_q + n_k) * heads = %lld rows exceeds the static scratch "
                "limit of %d rows; use veda_tile_logits with a workspace",
                static_cast<long long>(rows), VEDA_STATIC_LOGITS_ROWS);
  if (int rc = check_device()) return rc;
  float* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  if (proj_dtype == VEDA_FP8_E4M3)
    return fail(VEDA_ERR_INVALID,
                "fp8 projections go through veda_tile_logits_scaled");
  return launch_tile_logits(feats_q, feats_k, proj_q, proj_k, proj_dtype,
                            nullptr, nullptr, heads, n_q, n_k, scratch,
                            logits, static_cast<cudaStream_t>(stream));
}
