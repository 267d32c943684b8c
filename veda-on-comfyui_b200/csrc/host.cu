// Host-side helpers of the C ABI: error reporting, device checks and TMA
// tensor-map encoding (through the driver entry point, so the library needs
// no link-time dependency on libcuda).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace veda {
namespace {
thread_local char g_last_error[512] = "no error";
}

int fail(int code, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(VEDA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(err),
              cudaGetErrorString(err));
}

int current_device() {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return -1;
  return device;
}

bool is_sm100(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor,
                             device) != cudaSuccess)
    return false;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor,
                             device) != cudaSuccess)
    return false;
  return major == 10 && minor == 0;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank,
                 const void* base, const uint64_t* dims,
                 const uint64_t* strides, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult query;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                cudaEnableDefault, &query) == cudaSuccess &&
        query == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr)
    return fail(VEDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(VEDA_ERR_INVALID, "TMA base address is not 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    if ((strides[i] & 15) != 0)
      return fail(VEDA_ERR_INVALID, "TMA stride %llu is not a multiple of 16",
                  static_cast<unsigned long long>(strides[i]));
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult res = g_encode(map, dtype, rank, const_cast<void*>(base), dims,
                          strides, box, elem_strides,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS)
    return fail(VEDA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)",
                static_cast<int>(res));
  return VEDA_OK;
}

}  // namespace veda

extern "C" int veda_abi_version(void) { return VEDA_ABI_VERSION; }

extern "C" const char* veda_last_error(void) { return veda::g_last_error; }

extern "C" int veda_device_supported(int device) {
  return veda::is_sm100(device) ? 1 : 0;
}
