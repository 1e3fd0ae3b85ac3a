// Library-level C ABI: version, error text, device error words, device checks and the TMA
// tensor-map encoder shared by the kernels.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <mutex>

#include "host_common.h"

namespace vb200 {

namespace {
thread_local char g_last_error[1024] = "";
std::atomic<unsigned long long> g_launches{0};
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(VB200_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int check_sm100(void) {
  int dev = 0;
  VB200_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  int major = 0, minor = 0;
  VB200_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev),
                   "cudaDeviceGetAttribute");
  VB200_CHECK_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev),
                   "cudaDeviceGetAttribute");
  if (major != 10 || minor != 0)
    return set_error(VB200_EUNSUPPORTED,
                     "device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev,
                     major, minor);
  return VB200_OK;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_status = cudaSuccess;

void load_encode() {
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  g_encode_status =
      cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
  if (g_encode_status == cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}
}  // namespace

int encode_tiled_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                     CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr)
    return set_error(VB200_ECUDA, "cuTensorMapEncodeTiled is unavailable (%s)",
                     cudaGetErrorString(g_encode_status));
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return set_error(VB200_EINVAL, "TMA base address %p is not 16-byte aligned", base);
  for (int i = 0; i + 1 < rank; ++i) {
    if (strides_bytes[i] % 16 != 0 || strides_bytes[i] >= (1ull << 40))
      return set_error(VB200_EINVAL, "TMA stride %d (%llu bytes) must be a multiple of 16", i + 1,
                       (unsigned long long)strides_bytes[i]);
  }
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), dims, strides_bytes, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(VB200_EINVAL, "cuTensorMapEncodeTiled failed with CUresult %d", (int)r);
  return VB200_OK;
}

}  // namespace vb200

extern "C" {

int vb200_version(void) { return 1; }

unsigned long long vb200_launch_count(void) {
  return vb200::g_launches.load(std::memory_order_relaxed);
}

const char* vb200_last_error(void) { return vb200::g_last_error; }

int vb200_device_error_flags(unsigned* flags, int clear) {
  if (flags == nullptr) return vb200::set_error(VB200_EINVAL, "flags must not be NULL");
  VB200_CHECK_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  *flags = vb200::attention_error_word(clear) | vb200::projection_error_word(clear) |
           vb200::merge_error_word(clear) | vb200::plan_error_word(clear) |
           vb200::peer_error_word(clear);
  VB200_CHECK_CUDA(cudaGetLastError(), "reading device error words");
  return VB200_OK;
}

}  // extern "C"
