// Merge step: cosine-similarity GEMM with a fused running top-k epilogue (sm_100a).
#include "common.cuh"
#include "host_common.h"

namespace vb200 {
namespace {
static __device__ unsigned g_merge_err;
}  // namespace

unsigned merge_error_word(int clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_merge_err, sizeof(v));
  if (clear) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_merge_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace vb200

extern "C" int vb200_sim_topk(const void*, int64_t, const void*, int64_t, int64_t, int64_t, int64_t,
                              int, const int64_t*, const int64_t*, int64_t, float*, int64_t*,
                              void*) {
  return vb200::set_error(VB200_EUNSUPPORTED, "vb200_sim_topk is not built yet");
}
