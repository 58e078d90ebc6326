// Library-level entry points: error strings, the device error word, device properties, PDL switch.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace dk {

// One copy per device that loads the library; kernels receive its address (DeviceInfo::err_word).
__device__ int g_device_error = 0;

namespace {
thread_local char t_last_error[1024] = "";
bool g_pdl = true;
}  // namespace

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(DK_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return DK_OK;
}

bool pdl_enabled() { return g_pdl; }

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}
}  // namespace

bool make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner,
                        uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) {
    set_error(DK_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(DK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for a %llux%llu map, box %ux%u", (int)r,
              (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
    return false;
  }
  return true;
}

const DeviceInfo& device_info() {
  static std::mutex mu;
  static std::vector<DeviceInfo> cache;
  static std::vector<bool> have;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= static_cast<int>(cache.size())) {
    cache.resize(dev + 1);
    have.resize(dev + 1, false);
  }
  if (!have[dev]) {
    DeviceInfo d = {};
    cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) p = nullptr;
    d.err_word = static_cast<int*>(p);
    cache[dev] = d;
    have[dev] = true;
  }
  return cache[dev];
}

}  // namespace dk

extern "C" {

int dk_abi_version(void) { return DK_ABI_VERSION; }
int dk_matmul_config_size(void) { return static_cast<int>(sizeof(dk_matmul_config)); }

const char* dk_last_error(void) { return dk::t_last_error; }

int dk_device_error(int32_t* code) {
  if (code == nullptr) return dk::set_error(DK_ERR_INVALID, "dk_device_error: code is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return dk::set_error(DK_ERR_CUDA, "dk_device_error: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, dk::g_device_error, sizeof(int));
  if (e != cudaSuccess) return dk::set_error(DK_ERR_CUDA, "dk_device_error: %s", cudaGetErrorString(e));
  *code = v;
  return DK_OK;
}

int dk_clear_device_error(void) {
  int zero = 0;
  cudaError_t e = cudaMemcpyToSymbol(dk::g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) return dk::set_error(DK_ERR_CUDA, "dk_clear_device_error: %s", cudaGetErrorString(e));
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return dk::set_error(DK_ERR_CUDA, "dk_clear_device_error: %s", cudaGetErrorString(e));
  return DK_OK;
}

int dk_set_pdl(int32_t enabled) {
  dk::g_pdl = enabled != 0;
  return DK_OK;
}

}  // extern "C"
