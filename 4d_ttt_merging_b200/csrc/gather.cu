// Rank-ordered exchange of equally sized row blocks through other GPUs' memory.
//
// The sharded global block (query rows split over the GPUs of one node; the reference itself
// runs inference on one GPU) needs every merged key / value row and the log-mass vector of
// every rank.  The buffers are
// mapped into this process (peer-accessible allocations such as PyTorch symmetric memory), so
// the exchange is plain NVLink peer loads (peer_gather: row i of rank r lands at row
// r * rows + i of a local buffer) or posted peer stores (peer_push: this rank's rows land at
// its offset in every rank's buffer).  One warp per (rank, row) moves 16-byte vectors.  The
// caller orders the kernels between cross-GPU barriers.  Measured on two B200s for the
// config-2 K|V block (16.9 MB per rank): gather 52 us, push 54 us, the copy engines
// (cudaMemcpy2DAsync per peer) 53 us, NCCL all_gather_into_tensor 58 us for one call.
//
// peer_barrier is the cross-GPU barrier that orders those kernels: each rank release-stores an
// epoch into its slot of every rank's signal pad and acquire-waits until every slot of its own
// pad holds that epoch.  The wait is bounded by the global timer; when it runs out the kernel
// records kErrWaitTimeout in this file's error word and returns (no trap), so a rank that
// never arrives leaves the others with a readable error instead of a faulted context.
#include <cstdint>

#include "common.cuh"
#include "host_common.h"

namespace vb200 {
namespace {

constexpr int kMaxPeers = 16;
constexpr int kGatherWarps = 8;

__device__ unsigned g_peer_err = 0;

struct PeerTable {
  uint64_t src[kMaxPeers];
};

template <bool kVec16>
__global__ void __launch_bounds__(kGatherWarps * 32)
    peer_gather_kernel(const __grid_constant__ PeerTable peers, int world, long long rows, long long src_stride,
                       long long row_bytes, uint8_t* __restrict__ dst, long long dst_stride) {
  const long long w = static_cast<long long>(blockIdx.x) * kGatherWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= world * rows) return;
  const int r = static_cast<int>(w / rows);
  const long long i = w - static_cast<long long>(r) * rows;
  const uint8_t* s = reinterpret_cast<const uint8_t*>(peers.src[r]) + i * src_stride;
  uint8_t* d = dst + w * dst_stride;
  if constexpr (kVec16) {
    // up to kBatch 16-byte loads per lane are in flight before the first store (a peer load
    // is a full NVLink round trip)
    constexpr int kBatch = 8;
    const long long n = row_bytes / 16;
    const uint4* __restrict__ sv = reinterpret_cast<const uint4*>(s);
    uint4* __restrict__ dv = reinterpret_cast<uint4*>(d);
    for (long long k0 = lane; k0 < n; k0 += 32 * kBatch) {
      uint4 v[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b)
        if (k0 + 32 * b < n) v[b] = __ldg(sv + k0 + 32 * b);
#pragma unroll
      for (int b = 0; b < kBatch; ++b)
        if (k0 + 32 * b < n) dv[k0 + 32 * b] = v[b];
    }
  } else {
    const long long n = row_bytes / 4;
    for (long long k = lane; k < n; k += 32)
      reinterpret_cast<uint32_t*>(d)[k] = reinterpret_cast<const uint32_t*>(s)[k];
  }
}

// Push form: this rank's rows (local src) are written into every rank's destination at row
// offset dst_row0 (posted NVLink stores), then a system-scope fence orders them before
// whatever the stream signals next.
__global__ void __launch_bounds__(kGatherWarps * 32)
    peer_push_kernel(const uint8_t* __restrict__ src, long long rows, long long src_stride, long long row_bytes,
                     const __grid_constant__ PeerTable peers, int world, long long dst_row0, long long dst_stride) {
  const long long w = static_cast<long long>(blockIdx.x) * kGatherWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w < world * rows) {
    const int r = static_cast<int>(w / rows);
    const long long i = w - static_cast<long long>(r) * rows;
    const uint4* __restrict__ sv = reinterpret_cast<const uint4*>(src + i * src_stride);
    uint4* dv = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(peers.src[r]) + (dst_row0 + i) * dst_stride);
    const long long n = row_bytes / 16;
    for (long long k = lane; k < n; k += 32) dv[k] = __ldg(sv + k);
  }
  __threadfence_system();
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One block, thread p < world talks to rank p.  pads.src[r] is rank r's signal pad (world
// uint32 slots, slot q written by rank q); *epoch counts this rank's barriers on the pad and
// lives in device memory, so a recorded graph replays with a fresh epoch every time.
__global__ void peer_barrier_kernel(const __grid_constant__ PeerTable pads, int world, int rank,
                                    unsigned* __restrict__ epoch, unsigned long long timeout_ns) {
  __shared__ unsigned e_s;
  if (threadIdx.x == 0) e_s = *epoch + 1u;
  __syncthreads();
  const unsigned e = e_s;
  const int p = threadIdx.x;
  if (p < world) {
    __threadfence_system();  // this rank's earlier writes (earlier kernels) before the signal
    st_release_sys(reinterpret_cast<unsigned*>(pads.src[p]) + rank, e);
    const unsigned* mine = reinterpret_cast<const unsigned*>(pads.src[rank]) + p;
    const uint64_t t0 = global_timer_ns();
    while (static_cast<int>(ld_acquire_sys(mine) - e) < 0) {
      if (global_timer_ns() - t0 > timeout_ns) {
        atomicOr(&g_peer_err, kErrWaitTimeout);
        break;
      }
      __nanosleep(100);
    }
    __threadfence_system();
  }
  __syncthreads();
  if (threadIdx.x == 0) *epoch = e;
}

}  // namespace

unsigned peer_error_word(int clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_peer_err, sizeof(v));
  if (clear) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_peer_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace vb200

using namespace vb200;

extern "C" int vb200_peer_barrier(const uint64_t* pad_ptrs, int world, int rank, uint32_t* epoch,
                                  int64_t timeout_ns, void* stream) {
  VB200_REQUIRE(world >= 1 && world <= kMaxPeers, "peer_barrier: world must be in [1, %d] (got %d)", kMaxPeers,
                world);
  VB200_REQUIRE(rank >= 0 && rank < world, "peer_barrier: rank %d outside [0, %d)", rank, world);
  VB200_REQUIRE(pad_ptrs != nullptr && epoch != nullptr, "peer_barrier: null pointer");
  VB200_REQUIRE((reinterpret_cast<uintptr_t>(epoch) & 3u) == 0, "peer_barrier: epoch must be 4-byte aligned");
  VB200_REQUIRE(timeout_ns > 0, "peer_barrier: the timeout must be positive");
  PeerTable tab{};
  for (int r = 0; r < world; ++r) {
    VB200_REQUIRE(pad_ptrs[r] != 0 && (pad_ptrs[r] & 3u) == 0,
                  "peer_barrier: signal pad of rank %d is null or not 4-byte aligned", r);
    tab.src[r] = pad_ptrs[r];
  }
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      tab, world, rank, reinterpret_cast<unsigned*>(epoch), static_cast<unsigned long long>(timeout_ns));
  VB200_CHECK_LAUNCH("peer_barrier_kernel");
  return VB200_OK;
}

extern "C" int vb200_peer_push(const void* src, int64_t rows, int64_t src_stride_bytes, int64_t row_bytes,
                               const uint64_t* dst_ptrs, int world, int64_t dst_row0, int64_t dst_stride_bytes,
                               void* stream) {
  VB200_REQUIRE(world >= 1 && world <= kMaxPeers, "peer_push: world must be in [1, %d] (got %d)", kMaxPeers, world);
  VB200_REQUIRE(rows >= 0 && row_bytes >= 0 && dst_row0 >= 0, "peer_push: negative size");
  if (rows == 0 || row_bytes == 0) return VB200_OK;
  VB200_REQUIRE(src != nullptr && dst_ptrs != nullptr, "peer_push: null pointer");
  VB200_REQUIRE(row_bytes % 16 == 0 && src_stride_bytes % 16 == 0 && dst_stride_bytes % 16 == 0 &&
                    (reinterpret_cast<uintptr_t>(src) & 15u) == 0,
                "peer_push: rows, strides and addresses must be 16-byte aligned");
  VB200_REQUIRE(src_stride_bytes >= row_bytes && dst_stride_bytes >= row_bytes, "peer_push: strides must cover a row");
  PeerTable tab{};
  for (int r = 0; r < world; ++r) {
    VB200_REQUIRE(dst_ptrs[r] != 0 && (dst_ptrs[r] & 15u) == 0,
                  "peer_push: destination of rank %d is null or not 16-byte aligned", r);
    tab.src[r] = dst_ptrs[r];
  }
  const long long warps = static_cast<long long>(world) * rows;
  const unsigned blocks = static_cast<unsigned>((warps + kGatherWarps - 1) / kGatherWarps);
  peer_push_kernel<<<blocks, kGatherWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), rows, src_stride_bytes, row_bytes, tab, world, dst_row0, dst_stride_bytes);
  VB200_CHECK_LAUNCH("peer_push_kernel");
  return VB200_OK;
}

extern "C" int vb200_peer_gather(const uint64_t* src_ptrs, int world, int64_t rows, int64_t src_stride_bytes,
                                 int64_t row_bytes, void* dst, int64_t dst_stride_bytes, void* stream) {
  VB200_REQUIRE(world >= 1 && world <= kMaxPeers, "peer_gather: world must be in [1, %d] (got %d)", kMaxPeers, world);
  VB200_REQUIRE(rows >= 0 && row_bytes >= 0, "peer_gather: negative size");
  if (rows == 0 || row_bytes == 0) return VB200_OK;
  VB200_REQUIRE(src_ptrs != nullptr && dst != nullptr, "peer_gather: null pointer");
  VB200_REQUIRE(row_bytes % 4 == 0 && src_stride_bytes % 4 == 0 && dst_stride_bytes % 4 == 0,
                "peer_gather: row sizes and strides must be multiples of 4 bytes");
  VB200_REQUIRE(src_stride_bytes >= row_bytes && dst_stride_bytes >= row_bytes,
                "peer_gather: strides must cover a row");
  PeerTable tab{};
  bool vec16 = row_bytes % 16 == 0 && src_stride_bytes % 16 == 0 && dst_stride_bytes % 16 == 0 &&
               (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  for (int r = 0; r < world; ++r) {
    VB200_REQUIRE(src_ptrs[r] != 0, "peer_gather: null source pointer for rank %d", r);
    VB200_REQUIRE((src_ptrs[r] & 3u) == 0, "peer_gather: source of rank %d is not 4-byte aligned", r);
    tab.src[r] = src_ptrs[r];
    vec16 = vec16 && (src_ptrs[r] & 15u) == 0;
  }
  const long long warps = static_cast<long long>(world) * rows;
  const unsigned blocks = static_cast<unsigned>((warps + kGatherWarps - 1) / kGatherWarps);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (vec16) {
    peer_gather_kernel<true><<<blocks, kGatherWarps * 32, 0, st>>>(tab, world, rows, src_stride_bytes, row_bytes,
                                                                   static_cast<uint8_t*>(dst), dst_stride_bytes);
  } else {
    peer_gather_kernel<false><<<blocks, kGatherWarps * 32, 0, st>>>(tab, world, rows, src_stride_bytes, row_bytes,
                                                                    static_cast<uint8_t*>(dst), dst_stride_bytes);
  }
  VB200_CHECK_LAUNCH("peer_gather_kernel");
  return VB200_OK;
}
