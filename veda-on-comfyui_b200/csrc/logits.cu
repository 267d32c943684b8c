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
constexpr int kProjRows = 32;     // rows of F per CTA in the projection
constexpr int kProjChunk = 32;    // features of P per shared-memory pass
constexpr int kLogitTile = 64;    // 64 x 64 logits per CTA
constexpr int kLogitChunk = 32;   // dims of q_hat / k_hat per shared-memory pass

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

// grid (ceil(n / 32), heads, 2): z = 0 projects q features, z = 1 k.
// sq / sk: per-head scales of fp8 projections (unused otherwise).
// A CTA takes 32 rows of F and all 128 outputs; thread (warp w, lane l)
// accumulates rows 4 w .. 4 w + 3 x columns 4 l .. 4 l + 3, one FMA per
// feature in ascending order (one rounding per step, as a sequential fp32
// sum). F (transposed, feature-major) and the weights (widened to fp32)
// pass through shared memory 32 features at a time.
template <typename PT>
__global__ void __launch_bounds__(256)
    project_kernel(const float* fq, const float* fk, const PT* pq,
                   const PT* pk, const float* sq, const float* sk, int n_q,
                   int n_k, float* hat_q, float* hat_k) {
  __shared__ __align__(16) float f_t[kProjChunk][kProjRows];  // [feature][row]
  __shared__ __align__(16) float w_sh[kProjChunk][kDim];
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
  // Each thread stages 4 features of one row of F and 16 consecutive
  // weights per chunk; the next chunk's loads are issued before this
  // chunk's FMAs.
  constexpr int kWords = 16 * sizeof(PT) / 16;  // 16-byte loads of weights
  const int wi = 16 * threadIdx.x;              // first weight of the thread
  auto load_f = [&](int k0) {
    return lane < rows ? *reinterpret_cast<const float4*>(f + lane * kFeat +
                                                          k0 + 4 * warp)
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  };
  auto load_w = [&](int k0, uint4* raw) {
    const uint4* src = reinterpret_cast<const uint4*>(
        proj + static_cast<int64_t>(k0) * kDim + wi);
#pragma unroll
    for (int q = 0; q < kWords; ++q) raw[q] = src[q];
  };
  float4 fnext = load_f(0);
  uint4 wnext[kWords];
  load_w(0, wnext);
  for (int k0 = 0; k0 < kFeat; k0 += kProjChunk) {
    __syncthreads();  // the last chunk is read
    // F transposed: lane = row, so a warp's shared stores are consecutive
    // words
    f_t[4 * warp][lane] = fnext.x;
    f_t[4 * warp + 1][lane] = fnext.y;
    f_t[4 * warp + 2][lane] = fnext.z;
    f_t[4 * warp + 3][lane] = fnext.w;
    {
      const PT* wv = reinterpret_cast<const PT*>(wnext);
      float* dst = &w_sh[0][0] + wi;
#pragma unroll
      for (int e = 0; e < 16; e += 4)
        *reinterpret_cast<float4*>(dst + e) =
            make_float4(weight(wv[e], scale), weight(wv[e + 1], scale),
                        weight(wv[e + 2], scale), weight(wv[e + 3], scale));
    }
    if (k0 + kProjChunk < kFeat) {
      fnext = load_f(k0 + kProjChunk);
      load_w(k0 + kProjChunk, wnext);
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kProjChunk; ++k) {
      const float4 fv = *reinterpret_cast<const float4*>(&f_t[k][4 * warp]);
      const float4 wv = *reinterpret_cast<const float4*>(&w_sh[k][4 * lane]);
      const float fr[4] = {fv.x, fv.y, fv.z, fv.w};
      const float wc[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(fr[r], wc[c], acc[r][c]);
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int row = 4 * warp + r;
    if (row < rows) {
      // + F[:, :128]
      const float4 x =
          *reinterpret_cast<const float4*>(f + row * kFeat + 4 * lane);
      float4 o;
      o.x = acc[r][0] + x.x;
      o.y = acc[r][1] + x.y;
      o.z = acc[r][2] + x.z;
      o.w = acc[r][3] + x.w;
      *reinterpret_cast<float4*>(out + row * kDim + 4 * lane) = o;
    }
  }
}

// grid (ceil(n_k / 64), ceil(n_q / 64), heads), 256 threads. A CTA takes
// 64 x 64 logits of one head; thread (ti = t / 16, tj = t % 16) sums
// rows 4 ti .. 4 ti + 3 x columns 4 tj .. 4 tj + 3 over the 128 dims in
// ascending order (one fused rounding per step), with q_hat and k_hat
// staged transposed (dim-major) 32 dims at a time.
__global__ void __launch_bounds__(256)
    logits_kernel(const float* hat_q, const float* hat_k, int n_q, int n_k,
                  float* logits) {
  __shared__ __align__(16) float q_t[kLogitChunk][kLogitTile];
  __shared__ __align__(16) float k_t[kLogitChunk][kLogitTile];
  const int head = blockIdx.z;
  const int i0 = blockIdx.y * kLogitTile, j0 = blockIdx.x * kLogitTile;
  const float* qh = hat_q + static_cast<int64_t>(head) * n_q * kDim;
  const float* kh = hat_k + static_cast<int64_t>(head) * n_k * kDim;
  const int t = threadIdx.x;
  const int ti = t >> 4, tj = t & 15;
  // staging: thread t moves dims 4 (t / 64) .. + 3 of row t % 64 (q and k),
  // twice per chunk (dims +16)
  const int sr = t & 63, sd = 4 * (t >> 6);
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
  for (int c0 = 0; c0 < kDim; c0 += kLogitChunk) {
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int d = c0 + sd + 16 * h;
      const float4 qv =
          i0 + sr < n_q ? *reinterpret_cast<const float4*>(
                              qh + static_cast<int64_t>(i0 + sr) * kDim + d)
                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      const float4 kv =
          j0 + sr < n_k ? *reinterpret_cast<const float4*>(
                              kh + static_cast<int64_t>(j0 + sr) * kDim + d)
                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      const int dd = sd + 16 * h;
      q_t[dd][sr] = qv.x;
      q_t[dd + 1][sr] = qv.y;
      q_t[dd + 2][sr] = qv.z;
      q_t[dd + 3][sr] = qv.w;
      k_t[dd][sr] = kv.x;
      k_t[dd + 1][sr] = kv.y;
      k_t[dd + 2][sr] = kv.z;
      k_t[dd + 3][sr] = kv.w;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < kLogitChunk; ++c) {
      const float4 qv = *reinterpret_cast<const float4*>(&q_t[c][4 * ti]);
      const float4 kv = *reinterpret_cast<const float4*>(&k_t[c][4 * tj]);
      const float qr[4] = {qv.x, qv.y, qv.z, qv.w};
      const float kc[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          acc[r][cc] = fmaf(qr[r], kc[cc], acc[r][cc]);
    }
  }
  const float root = 11.313708498984761f;  // sqrt(128)
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = i0 + 4 * ti + r;
    if (i >= n_q) continue;
    float* dst = logits + (static_cast<int64_t>(head) * n_q + i) * n_k;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int j = j0 + 4 * tj + cc;
      if (j < n_k) dst[j] = __fdiv_rn(acc[r][cc], root);
    }
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
  // the kernels read features and weights as 16-byte vectors
  if (!aligned16(feats_q) || !aligned16(feats_k) || !aligned16(proj_q) ||
      !aligned16(proj_k))
    return fail(VEDA_ERR_INVALID,
                "features and projections must be 16-byte aligned");
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
  if (!aligned16(workspace))
    return fail(VEDA_ERR_INVALID, "workspace must be 16-byte aligned");
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
  if (!aligned16(workspace))
    return fail(VEDA_ERR_INVALID, "workspace must be 16-byte aligned");
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
