// Tile-order permutation of packed rows and its inverse
// (core/tiling.py:227-252, gather_tiles / scatter_tiles_): one 16-byte
// vector (8 elements of a 128-wide row) per thread, grid-stride.
// Row ids outside [0, seq_len) and head ids outside [0, total_heads) are
// skipped (gather writes zeros for them), so no access leaves the buffers.
#include "common.cuh"

namespace veda {
namespace {

__global__ void gather_kernel(const uint16_t* x, int64_t stride_s,
                              int64_t stride_h, int seq_len, int total_heads,
                              const int64_t* perm, int64_t n_slots,
                              const int64_t* heads, int n_heads,
                              uint16_t* out) {
  const int64_t total = n_slots * n_heads * (kDim / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
       i < total; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int chunk = static_cast<int>(i % (kDim / 8));
    const int64_t sj = i / (kDim / 8);
    const int j = static_cast<int>(sj % n_heads);
    const int64_t slot = sj / n_heads;
    const int64_t row = perm[slot];
    const int64_t h = heads[j];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row >= 0 && row < seq_len && h >= 0 && h < total_heads)
      v = __ldg(reinterpret_cast<const uint4*>(x + row * stride_s +
                                               h * stride_h + 8 * chunk));
    reinterpret_cast<uint4*>(out)[i] = v;
  }
}

__global__ void scatter_kernel(const uint16_t* tiled, const int64_t* perm,
                               int64_t n_slots, const int64_t* heads,
                               int n_heads, int total_heads, int seq_len,
                               uint16_t* out, int64_t stride_s,
                               int64_t stride_h) {
  const int64_t total = n_slots * n_heads * (kDim / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
       i < total; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int chunk = static_cast<int>(i % (kDim / 8));
    const int64_t sj = i / (kDim / 8);
    const int j = static_cast<int>(sj % n_heads);
    const int64_t slot = sj / n_heads;
    const int64_t row = perm[slot];
    const int64_t h = heads[j];
    if (row < 0 || row >= seq_len || h < 0 || h >= total_heads) continue;
    *reinterpret_cast<uint4*>(out + row * stride_s + h * stride_h + 8 * chunk) =
        reinterpret_cast<const uint4*>(tiled)[i];
  }
}

int grid_for(int64_t total) {
  int64_t blocks = (total + 255) / 256;
  return static_cast<int>(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1)
                                            : 148 * 16);
}

}  // namespace
}  // namespace veda

using namespace veda;

extern "C" int veda_gather_tiles(const void* x, int dtype, int64_t stride_s,
                                 int64_t stride_h, int seq_len,
                                 int total_heads, const int64_t* perm,
                                 int n_slots, const int64_t* heads,
                                 int n_heads, void* out, void* stream) {
  if (int rc = check_device()) return rc;
  if (dtype != VEDA_BF16 && dtype != VEDA_F16)
    return fail(VEDA_ERR_INVALID, "dtype must be bf16 or fp16");
  if (x == nullptr || perm == nullptr || heads == nullptr || out == nullptr)
    return fail(VEDA_ERR_INVALID, "null pointer argument");
  if (n_slots <= 0 || n_heads <= 0 || seq_len <= 0 || total_heads <= 0)
    return fail(VEDA_ERR_INVALID, "sizes must be positive");
  if (!aligned16(x) || !aligned16(out) || (stride_s * 2) % 16 != 0 ||
      (stride_h * 2) % 16 != 0)
    return fail(VEDA_ERR_INVALID, "rows must be 16-byte aligned");
  const int64_t total = static_cast<int64_t>(n_slots) * n_heads * (kDim / 8);
  gather_kernel<<<grid_for(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), stride_s, stride_h, seq_len,
      total_heads, perm, n_slots, heads, n_heads, static_cast<uint16_t*>(out));
  VEDA_CHECK_CUDA(cudaGetLastError());
  return VEDA_OK;
}

extern "C" int veda_scatter_tiles(const void* tiled, int dtype,
                                  const int64_t* perm, int n_slots,
                                  const int64_t* heads, int n_heads,
                                  int total_heads, void* out, int64_t stride_s,
                                  int64_t stride_h, int seq_len,
                                  void* stream) {
  if (int rc = check_device()) return rc;
  if (dtype != VEDA_BF16 && dtype != VEDA_F16)
    return fail(VEDA_ERR_INVALID, "dtype must be bf16 or fp16");
  if (tiled == nullptr || perm == nullptr || heads == nullptr ||
      out == nullptr)
    return fail(VEDA_ERR_INVALID, "null pointer argument");
  if (n_slots <= 0 || n_heads <= 0 || seq_len <= 0 || total_heads <= 0)
    return fail(VEDA_ERR_INVALID, "sizes must be positive");
  if (!aligned16(tiled) || !aligned16(out) || (stride_s * 2) % 16 != 0 ||
      (stride_h * 2) % 16 != 0)
    return fail(VEDA_ERR_INVALID, "rows must be 16-byte aligned");
  const int64_t total = static_cast<int64_t>(n_slots) * n_heads * (kDim / 8);
  scatter_kernel<<<grid_for(total), 256, 0,
                   static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(tiled), perm, n_slots, heads, n_heads,
      total_heads, seq_len, static_cast<uint16_t*>(out), stride_s, stride_h);
  VEDA_CHECK_CUDA(cudaGetLastError());
  return VEDA_OK;
}
