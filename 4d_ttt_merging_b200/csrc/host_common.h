// Host-side helpers shared by the translation units behind the C ABI: thread-local error
// text, CUDA error mapping and TMA tensor-map encoding through the driver entry point.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstddef>
#include <cstdint>

#include "../../include/vggt_b200.h"

namespace vb200 {

int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
int check_sm100(void);  // VB200_OK when the current device is compute capability 10.x

// Encode a tiled TMA map.  dims / strides follow cuTensorMapEncodeTiled: dims[0] is the
// innermost (contiguous) dimension; strides_bytes has rank-1 entries for dims 1..rank-1.
int encode_tiled_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                     CUtensorMapSwizzle swizzle);

// Per-TU device error words: each returns the word's value and optionally clears it.
unsigned attention_error_word(int clear);
unsigned projection_error_word(int clear);
unsigned merge_error_word(int clear);
unsigned plan_error_word(int clear);
unsigned peer_error_word(int clear);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace vb200

#define VB200_CHECK_CUDA(expr, what)                        \
  do {                                                      \
    cudaError_t e_ = (expr);                                \
    if (e_ != cudaSuccess) return vb200::cuda_error(e_, what); \
  } while (0)

namespace vb200 {
void count_launch();  // one of this library's kernels was launched
}

#define VB200_CHECK_LAUNCH(what)                     \
  do {                                               \
    vb200::count_launch();                           \
    VB200_CHECK_CUDA(cudaGetLastError(), what);      \
  } while (0)

#define VB200_REQUIRE(cond, ...)                                     \
  do {                                                               \
    if (!(cond)) return vb200::set_error(VB200_EINVAL, __VA_ARGS__); \
  } while (0)
