// Bandwidth-bound kernels of the top-4 sparse-convex projection and the merge step:
//   proj_gather   merged -> tokens (WeightedBilinearTokenPlan.restore, token_merging.py:387-414)
//   proj_scatter  tokens -> merged (WeightedBilinearTokenPlan.compact, token_merging.py:343-370;
//                 TokenPlan.compact, token_merging.py:176-191)
//   plan_csr      per-plan grouping by parent + mass / log-mass
//                 (WeightedBilinearTokenPlan.__post_init__ :323-333,
//                  deterministic_weighted_normalizer :40-59)
//   row_gather    compact_key (:372-376), TokenPlan.restore (:193-196)
//   row_normalize F.normalize(x.float()).to(bf16) of build_fastvggt_plan (:1102-1103)
//
// All row kernels assign one warp per output row and move 16-byte vectors, so a 1024-channel
// bf16 row is 4 coalesced 512-byte sweeps of the warp.  No kernel uses atomics on data: the
// scatter direction reads a CSR built once per plan, so every output row is reduced by one
// warp in a fixed order (keep row, then corner 0..3 partial sums, each in source order).
#include <cub/cub.cuh>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "host_common.h"

namespace vb200 {
namespace {

static __device__ unsigned g_proj_err;

constexpr int kWarpsPerBlock = 8;

template <typename T>
struct Vec {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[Vec<T>::N]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  if constexpr (sizeof(T) == 4) {
    v[0] = __uint_as_float(raw.x);
    v[1] = __uint_as_float(raw.y);
    v[2] = __uint_as_float(raw.z);
    v[3] = __uint_as_float(raw.w);
  } else {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < Vec<T>::N; ++i) v[i] = to_f32<T>(e[i]);
  }
}

template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[Vec<T>::N]) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<uint4*>(p) = raw;
}

// Round through T (identity for fp32).
template <typename T>
__device__ __forceinline__ float round_t(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// ------------------------------------------------------------------------------------------
// row gather: out[i] = x[index[i]]
// ------------------------------------------------------------------------------------------
__global__ void row_gather_kernel(const uint8_t* __restrict__ x, long long x_rows, long long xs_bytes,
                                  const int64_t* __restrict__ index, long long R,
                                  uint8_t* __restrict__ out, long long os_bytes, int row_vecs) {
  const long long r = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const int64_t src = index[r];
  if (src < 0 || src >= x_rows) {
    if (lane == 0) atomicOr(&g_proj_err, kErrBadArgument);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(x + src * xs_bytes);
  uint4* d = reinterpret_cast<uint4*>(out + r * os_bytes);
  for (int i = lane; i < row_vecs; i += 32) d[i] = __ldg(s + i);
}

// ------------------------------------------------------------------------------------------
// gather (restore): keep rows copied, source rows = sum_c w_c * y[parent_c]
// ------------------------------------------------------------------------------------------
// Keep rows of the gather: out[keep[r]] = y[r], one warp per row, 16-byte vectors.
template <typename T>
__device__ __forceinline__ void gather_keep_row(const T* __restrict__ y, long long ys, const int64_t* __restrict__ keep,
                                                long long r, T* __restrict__ out, long long os, long long N_out,
                                                int nvec, int lane) {
  const int64_t dst = keep[r];
  if (dst < 0 || dst >= N_out) {
    if (lane == 0) atomicOr(&g_proj_err, kErrBadArgument);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(y + r * ys);
  uint4* d = reinterpret_cast<uint4*>(out + dst * os);
  for (int i = lane; i < nvec; i += 32) d[i] = __ldg(s + i);
}

// Source rows [base, base + per_warp) of the gather (per_warp <= 32), one warp.  Lane l first
// loads the indices of source base + l (destination, parents, weights, staging slots: coalesced,
// one round trip for the batch), then the warp walks the batch with the indices broadcast by
// shuffles, so
// each source costs one round trip for its parent rows alone.  All four parents' vectors of a
// 32 x kGatherQ column block are loaded before any is used: kGatherQ = 4 (a whole 1024-channel
// bf16 row, 8 KB per warp, ~125 registers) for large plans, kGatherQ = 1 (one vector per lane,
// ~60 registers, twice the resident warps) with one source per warp for small ones.  (Half rows
// at 64 registers with 32-source batches measured slower on config 5: 1.11 vs 0.89 ms.)  With
// `hot` the parents that have a staging slot are read from that shared-memory copy.
template <typename T, bool kHot, int kGatherQ>
__device__ __forceinline__ void gather_sources(const T* __restrict__ y, long long ys, long long K,
                                               const int64_t* __restrict__ src, const int64_t* __restrict__ parent,
                                               const float* __restrict__ w, long long S, int corners,
                                               T* __restrict__ out, long long os, long long N_out, int C,
                                               long long base, int per_warp, int lane,
                                               const int32_t* __restrict__ hot_slot, const T* hot) {
  constexpr int V = Vec<T>::N;
  const int nvec = C / V;
  // ---- per-lane indices of source base + lane (lanes < per_warp) ----
  const long long sl = lane < per_warp ? base + lane : S;
  long long dst = -1;
  int prow[4] = {0, 0, 0, 0};  // parent row of y, or ~slot when the row is staged
  float wl[4] = {0.f, 0.f, 0.f, 0.f};
  if (sl < S) {
    dst = src[sl];
    if (dst < 0 || dst >= N_out) {
      atomicOr(&g_proj_err, kErrBadArgument);
      dst = -1;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (c < corners) {
        int64_t pc = parent[sl * corners + c];
        if (pc < 0 || pc >= K) {
          atomicOr(&g_proj_err, kErrBadArgument);
          pc = 0;
        }
        int slot = -1;
        if constexpr (kHot) slot = hot_slot[pc];
        prow[c] = slot >= 0 ? ~slot : static_cast<int>(pc);
        wl[c] = round_t<T>(w[sl * corners + c]);  // weights.to(value.dtype)
      }
    }
  }
  const int n = static_cast<int>(min(static_cast<long long>(per_warp), S - base));
  for (int t = 0; t < n; ++t) {
    const long long d = __shfl_sync(0xffffffffu, dst, t);
    int pr[4];
    float wc[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      pr[c] = __shfl_sync(0xffffffffu, prow[c], t);
      wc[c] = __shfl_sync(0xffffffffu, wl[c], t);
    }
    if (d < 0) continue;  // warp-uniform
    T* drow = out + d * os;
    for (int i0 = 0; i0 < nvec; i0 += 32 * kGatherQ) {
      uint4 raw[4][kGatherQ];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c < corners) {
          const bool staged = kHot && pr[c] < 0;
          const T* row = staged ? hot + static_cast<long long>(~pr[c]) * C : y + static_cast<long long>(pr[c]) * ys;
#pragma unroll
          for (int q = 0; q < kGatherQ; ++q) {
            const int i = i0 + lane + 32 * q;
            if (i < nvec) {
              if (staged) raw[c][q] = *reinterpret_cast<const uint4*>(row + i * V);
              else raw[c][q] = __ldg(reinterpret_cast<const uint4*>(row + i * V));
            }
          }
        }
      }
#pragma unroll
      for (int q = 0; q < kGatherQ; ++q) {
        const int i = i0 + lane + 32 * q;
        if (i >= nvec) continue;
        float acc[V];
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          // bf16: the rounded products w_c * y come from packed bf16 multiplies (the exact
          // product of two bf16 values fits in fp32, so one correctly rounded bf16 multiply
          // equals rounding the fp32 product), then each pair is widened and summed in fp32 in
          // corner order.
          uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c < corners) {
              const __nv_bfloat162 w2 = __float2bfloat162_rn(wc[c]);
              const uint32_t* xw = reinterpret_cast<const uint32_t*>(&raw[c][q]);
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const __nv_bfloat162 prod = __hmul2(w2, *reinterpret_cast<const __nv_bfloat162*>(&xw[h]));
                const uint32_t pw = *reinterpret_cast<const uint32_t*>(&prod);
                acc2[h] = fadd2(acc2[h], pk2(__uint_as_float(pw << 16), __uint_as_float(pw & 0xffff0000u)));
              }
            }
          }
#pragma unroll
          for (int h = 0; h < 4; ++h) upk2(acc2[h], acc[2 * h], acc[2 * h + 1]);
        } else {
#pragma unroll
          for (int e = 0; e < V; ++e) acc[e] = 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c < corners) {
              const T* e8 = reinterpret_cast<const T*>(&raw[c][q]);
#pragma unroll
              for (int e = 0; e < V; ++e) acc[e] += round_t<T>(__fmul_rn(wc[c], to_f32<T>(e8[e])));
            }
          }
        }
        store_vec<T>(drow + i * V, acc);
      }
    }
  }
}

// Plain form: warps [0, K) copy one keep row each; every further warp gathers per_warp sources
// (fewer on small plans, so the batches still fill the GPU), every parent read from global memory (the merged table fits in L2, or the plan is
// too small for the staging below to pay).
template <typename T, int kMaxCorners, int kGatherQ>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    proj_gather_kernel(const T* __restrict__ y, long long ys, const int64_t* __restrict__ keep,
                       long long K, const int64_t* __restrict__ src,
                       const int64_t* __restrict__ parent, const float* __restrict__ w,
                       long long S, int corners, T* __restrict__ out, long long os,
                       long long N_out, int C, int per_warp) {
  static_assert(kMaxCorners == 4, "four corners at most");
  const long long wid = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long K_copy = keep != nullptr ? K : 0;  // no keep table: sources only (K bounds the parents)
  if (wid < K_copy) {
    gather_keep_row<T>(y, ys, keep, wid, out, os, N_out, C / Vec<T>::N, lane);
    return;
  }
  const long long base = (wid - K_copy) * per_warp;
  if (base >= S) return;
  gather_sources<T, false, kGatherQ>(y, ys, K, src, parent, w, S, corners, out, os, N_out, C, base, per_warp, lane,
                                     nullptr, nullptr);
}

// Skewed plans: the most-referenced merged rows (hot_rows, chosen once per plan by
// vb200_plan_hot_rows) are staged once per CTA in shared memory and every reference to them is
// served from there, which takes their share of the 4 x 2 KB parent reads per token off the L2
// (the bound of the plain kernel on config 5: ~8 GB of L2 reads per restore).  One CTA of
// kHotWarps warps per SM walks the keep rows, then the 32-source batches, in grid stride.
constexpr int kHotWarps = 16;
constexpr long long kGatherBatchMin = 1 << 17;  // sources from which the plain gather batches
constexpr int kMaxHotRows = 128;
constexpr long long kHotSmemBytes = 200 * 1024;  // shared memory for staged rows per CTA

template <typename T, int kMaxCorners>
__global__ void __launch_bounds__(kHotWarps * 32, 1)
    proj_gather_hot_kernel(const T* __restrict__ y, long long ys, const int64_t* __restrict__ keep, long long K,
                           const int64_t* __restrict__ src, const int64_t* __restrict__ parent,
                           const float* __restrict__ w, long long S, int corners, T* __restrict__ out, long long os,
                           long long N_out, int C, const int32_t* __restrict__ hot_rows,
                           const int32_t* __restrict__ hot_slot, const int32_t* __restrict__ n_hot_p,
                           int max_hot) {
  static_assert(kMaxCorners == 4, "four corners at most");
  extern __shared__ __align__(16) uint8_t hot_smem[];
  T* hot = reinterpret_cast<T*>(hot_smem);
  const int n_hot = min(*n_hot_p, max_hot);
  const int vecs = C * static_cast<int>(sizeof(T)) / 16;
  for (int i = threadIdx.x; i < n_hot * vecs; i += blockDim.x) {
    const int r = i / vecs, v = i - r * vecs;
    const int row = hot_rows[r];
    uint4 val = make_uint4(0, 0, 0, 0);
    if (row >= 0 && row < K) val = __ldg(reinterpret_cast<const uint4*>(y + row * ys) + v);
    reinterpret_cast<uint4*>(hot + static_cast<long long>(r) * C)[v] = val;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long warp0 = static_cast<long long>(blockIdx.x) * kHotWarps + (threadIdx.x >> 5);
  const long long nwarps = static_cast<long long>(gridDim.x) * kHotWarps;
  if (keep != nullptr)
    for (long long r = warp0; r < K; r += nwarps) gather_keep_row<T>(y, ys, keep, r, out, os, N_out, C / Vec<T>::N, lane);
  for (long long base = warp0 * 32; base < S; base += nwarps * 32)
    gather_sources<T, true, 4>(y, ys, K, src, parent, w, S, corners, out, os, N_out, C, base, 32, lane, hot_slot,
                               hot);
}

// Hot-row selection (one block): row j's reference count is its CSR length; counts are bucketed
// by (log2, 3 mantissa bits), whole buckets are taken from the top while the total stays within
// max_hot, and every row of a taken bucket gets a slot.  Which row lands in which slot does not
// change any result (staged rows are exact copies).
constexpr int kHotBuckets = 256;

__device__ __forceinline__ int hot_bucket(int len) {
  if (len <= 1) return 0;  // a row referenced once gains nothing from staging
  const int lg = 31 - __clz(len);
  const int mant = lg >= 3 ? (len >> (lg - 3)) & 7 : (len << (3 - lg)) & 7;
  return min(kHotBuckets - 1, 1 + lg * 8 + mant);
}

__global__ void __launch_bounds__(1024)
    plan_hot_rows_kernel(const int32_t* __restrict__ seg_offsets, long long M, int corners, int max_hot,
                         int32_t* __restrict__ hot_rows, int32_t* __restrict__ hot_slot, int32_t* __restrict__ n_hot) {
  __shared__ int hist[kHotBuckets];
  __shared__ int cut, count;
  for (int b = threadIdx.x; b < kHotBuckets; b += blockDim.x) hist[b] = 0;
  if (threadIdx.x == 0) count = 0;
  __syncthreads();
  for (long long j = threadIdx.x; j < M; j += blockDim.x)
    atomicAdd(&hist[hot_bucket(seg_offsets[(j + 1) * corners] - seg_offsets[j * corners])], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    int total = 0, b = kHotBuckets - 1;
    for (; b > 0; --b) {
      if (total + hist[b] > max_hot) break;
      total += hist[b];
    }
    cut = b + 1;  // buckets >= cut are staged (bucket 0 never is)
  }
  __syncthreads();
  for (long long j = threadIdx.x; j < M; j += blockDim.x) {
    int slot = -1;
    if (hot_bucket(seg_offsets[(j + 1) * corners] - seg_offsets[j * corners]) >= cut) {
      slot = atomicAdd(&count, 1);
      hot_rows[slot] = static_cast<int32_t>(j);
    }
    hot_slot[j] = slot;
  }
  __syncthreads();
  if (threadIdx.x == 0) *n_hot = count;
}

template <typename T>
__global__ void zero_rows_kernel(T* out, long long os, long long N, int C) {
  constexpr int V = Vec<T>::N;
  const long long r = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= N) return;
  uint4* d = reinterpret_cast<uint4*>(out + r * os);
  for (int i = lane; i < C / V; i += 32) d[i] = make_uint4(0, 0, 0, 0);
}

// ------------------------------------------------------------------------------------------
// scatter (compact): out[j] = (keep_j + sum_c part_c) / normalizer_j, part_c = the fp32 sum of
// w * x over the sources whose corner-c parent is j, in source order (the CSR order).
//
// The kernels read whole source rows: lane l of a warp owns 16-byte vectors l, l + 32, l + 64,
// l + 96 of a 32 x 4-vector column block (one 1024-channel bf16 row), so each CSR entry is one
// 2 KB row read, and kScatterInFlight entries are loaded before any is summed (8 KB in flight
// per warp).  Memory-level parallelism, not bandwidth, bounded the earlier one-vector-per-pass
// form (ncu: long-scoreboard stalls, 20-30% of warps active).
//
// Skewed plans: a merged row with more than kScatterChunk CSR entries (a Zipf-popular parent can
// own a tenth of all entries) is reduced as a fixed two-level tree.  Level 0: one warp per chunk
// of kScatterChunk consecutive entries writes the chunk's fp32 sum (sequential within the
// chunk).  Level 1: a row with more than kScatterGroup chunks gets one warp per group of
// kScatterGroup consecutive chunk sums.  scatter_finish_kernel then adds the keep row and the
// row's level-1 sums (or level-0 sums) in order.  Level 0 and the short rows run in ONE launch
// (scatter_work_kernel), so the GPU stays full while the long rows' chunks are summed.  The
// result is deterministic (fixed order) and no warp walks more than kScatterChunk rows or
// kScatterGroup partial sums (up to rows of kScatterChunk * kScatterGroup^2 entries).
// ------------------------------------------------------------------------------------------
constexpr int kScatterChunk = 128;   // entries per level-0 chunk (and the long-row threshold)
constexpr int kScatterGroup = 64;    // level-0 partials per level-1 sum
constexpr int kScatterInFlight = 4;  // entries loaded before any is summed
constexpr int kScatterQ = 4;         // 16-byte vectors per lane per column block

__global__ void scatter_count_kernel(const int32_t* __restrict__ seg_offsets, long long M, int corners,
                                     int32_t* __restrict__ nchunk, int32_t* __restrict__ ngroup) {
  const long long j = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (j > M) return;
  if (j == M) {
    nchunk[j] = 0;
    ngroup[j] = 0;
    return;
  }
  const int len = seg_offsets[(j + 1) * corners] - seg_offsets[j * corners];
  const int n0 = len > kScatterChunk ? (len + kScatterChunk - 1) / kScatterChunk : 0;
  nchunk[j] = n0;
  ngroup[j] = n0 > kScatterGroup ? (n0 + kScatterGroup - 1) / kScatterGroup : 0;
}

// Sum of partial rows [k0, k1) of `src` (C floats each) over the channels of this lane, kept in
// flight kSumInFlight rows at a time, added in row order.
template <int kSumInFlight>
__device__ __forceinline__ void sum_partials(const float* __restrict__ src, int k0, int k1, int C, int col,
                                             float (&acc)[8], int V) {
  for (int kb = k0; kb < k1; kb += kSumInFlight) {
    float4 a[kSumInFlight], b[kSumInFlight];
#pragma unroll
    for (int u = 0; u < kSumInFlight; ++u) {
      if (kb + u < k1) {
        const float* pr = src + static_cast<long long>(kb + u) * C + col;
        a[u] = *reinterpret_cast<const float4*>(pr);
        if (V == 8) b[u] = *reinterpret_cast<const float4*>(pr + 4);
      }
    }
#pragma unroll
    for (int u = 0; u < kSumInFlight; ++u) {
      if (kb + u < k1) {
        acc[0] = __fadd_rn(acc[0], a[u].x); acc[1] = __fadd_rn(acc[1], a[u].y);
        acc[2] = __fadd_rn(acc[2], a[u].z); acc[3] = __fadd_rn(acc[3], a[u].w);
        if (V == 8) {
          acc[4] = __fadd_rn(acc[4], b[u].x); acc[5] = __fadd_rn(acc[5], b[u].y);
          acc[6] = __fadd_rn(acc[6], b[u].z); acc[7] = __fadd_rn(acc[7], b[u].w);
        }
      }
    }
  }
}

// Level 1: warp g sums group g's kScatterGroup (or fewer) consecutive level-0 partial rows.
template <int V>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    scatter_group_kernel(long long M, const int32_t* __restrict__ chunk_base, const int32_t* __restrict__ group_base,
                         const float* __restrict__ partials, float* __restrict__ partials1, int C) {
  const long long g = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (g >= group_base[M]) return;
  long long lo = 0, hi = M;  // row j with group_base[j] <= g < group_base[j + 1]
  while (hi - lo > 1) {
    const long long mid = (lo + hi) / 2;
    if (group_base[mid] <= g) lo = mid;
    else hi = mid;
  }
  const long long j = lo;
  const int k0 = chunk_base[j] + static_cast<int>(g - group_base[j]) * kScatterGroup;
  const int k1 = k0 + kScatterGroup < chunk_base[j + 1] ? k0 + kScatterGroup : chunk_base[j + 1];
  for (int col = lane * V; col < C; col += 32 * V) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    sum_partials<8>(partials, k0, k1, C, col, acc, V);
    float* dst = partials1 + g * C + col;
#pragma unroll
    for (int q = 0; q < V; ++q) dst[q] = acc[q];
  }
}

// One 16-byte vector of T as fp32 pairs (V / 2 pairs).
template <typename T>
__device__ __forceinline__ void widen_pairs(const uint4& raw, uint64_t (&p)[Vec<T>::N / 2]) {
  const uint32_t* wv = reinterpret_cast<const uint32_t*>(&raw);
  if constexpr (sizeof(T) == 4) {
    p[0] = pk2(__uint_as_float(wv[0]), __uint_as_float(wv[1]));
    p[1] = pk2(__uint_as_float(wv[2]), __uint_as_float(wv[3]));
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
    for (int h = 0; h < 4; ++h) p[h] = pk2(__uint_as_float(wv[h] << 16), __uint_as_float(wv[h] & 0xffff0000u));
  } else {
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[h]));
      p[h] = pk2(f.x, f.y);
    }
  }
}

// part[q] (V/2 fp32 pairs per owned vector q) += w_e * x[src_e] for CSR entries [e0, e1), in
// entry order; each product rounded to fp32 before the add (the reference multiplies, then
// sums).  The lane's vectors of the column block starting at col0: (lane + 32 q) * V.
template <typename T>
__device__ __forceinline__ void scatter_entries(const T* __restrict__ x, long long x_rows, long long xs,
                                                const int32_t* __restrict__ entry_src,
                                                const float* __restrict__ entry_w, int e0, int e1, int col0,
                                                int C, int lane, uint64_t (&part)[kScatterQ][Vec<T>::N / 2]) {
  constexpr int V = Vec<T>::N;
  for (int eb = e0; eb < e1; eb += kScatterInFlight) {
    uint4 raw[kScatterInFlight][kScatterQ];
    float w[kScatterInFlight];
#pragma unroll
    for (int u = 0; u < kScatterInFlight; ++u) {
      int su = 0;
      w[u] = 0.f;
      if (eb + u < e1) {
        su = __ldg(entry_src + eb + u);
        w[u] = __ldg(entry_w + eb + u);
        if (su < 0 || su >= x_rows) {
          su = 0;
          w[u] = 0.f;
          if (lane == 0) atomicOr(&g_proj_err, kErrBadArgument);
        }
      }
      const T* row = x + static_cast<long long>(su) * xs;
#pragma unroll
      for (int q = 0; q < kScatterQ; ++q) {
        const int col = col0 + (lane + 32 * q) * V;
        if (eb + u < e1 && col < C) raw[u][q] = __ldg(reinterpret_cast<const uint4*>(row + col));
      }
    }
#pragma unroll
    for (int u = 0; u < kScatterInFlight; ++u) {
      if (eb + u < e1) {
        const uint64_t w2 = pk2(w[u], w[u]);
#pragma unroll
        for (int q = 0; q < kScatterQ; ++q) {
          if (col0 + (lane + 32 * q) * V < C) {
            uint64_t xv[V / 2];
            widen_pairs<T>(raw[u][q], xv);
#pragma unroll
            for (int h = 0; h < V / 2; ++h) part[q][h] = fadd2(part[q][h], fmul2(w2, xv[h]));
          }
        }
      }
    }
  }
}

// Level 0 and short rows in one launch: warps [0, chunk_warps) sum the level-0 chunks of long
// rows (warps past the real chunk count exit); warp chunk_warps + j reduces short row j
// completely (keep row + corner partial sums in corner order, divided by the normaliser).
template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, 2)
    scatter_work_kernel(const T* __restrict__ x, long long x_rows, long long xs, const int64_t* __restrict__ keep,
                        long long M, int corners, const int32_t* __restrict__ seg_offsets,
                        const int32_t* __restrict__ entry_src, const float* __restrict__ entry_w,
                        const float* __restrict__ normalizer, T* __restrict__ out, long long os, int C,
                        const int32_t* __restrict__ chunk_base, float* __restrict__ partials,
                        long long chunk_warps, float* __restrict__ numerators) {
  constexpr int V = Vec<T>::N;
  const long long w = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w < chunk_warps) {
    const long long c = w;
    if (c >= chunk_base[M]) return;
    long long lo = 0, hi = M;  // the row j with chunk_base[j] <= c < chunk_base[j + 1]
    while (hi - lo > 1) {
      const long long mid = (lo + hi) / 2;
      if (chunk_base[mid] <= c) lo = mid;
      else hi = mid;
    }
    const long long j = lo;
    const int r0 = seg_offsets[j * corners], r1 = seg_offsets[(j + 1) * corners];
    const int e0 = r0 + static_cast<int>(c - chunk_base[j]) * kScatterChunk;
    const int e1 = e0 + kScatterChunk < r1 ? e0 + kScatterChunk : r1;
    float* pr = partials + c * C;
    for (int col0 = 0; col0 < C; col0 += 32 * kScatterQ * V) {
      uint64_t part[kScatterQ][V / 2];
#pragma unroll
      for (int q = 0; q < kScatterQ; ++q)
#pragma unroll
        for (int h = 0; h < V / 2; ++h) part[q][h] = 0ull;
      scatter_entries<T>(x, x_rows, xs, entry_src, entry_w, e0, e1, col0, C, lane, part);
#pragma unroll
      for (int q = 0; q < kScatterQ; ++q) {
        const int col = col0 + (lane + 32 * q) * V;
        if (col < C) {
#pragma unroll
          for (int h = 0; h < V / 2; ++h) {
            float a, b;
            upk2(part[q][h], a, b);
            *reinterpret_cast<float2*>(pr + col + 2 * h) = make_float2(a, b);
          }
        }
      }
    }
    return;
  }
  const long long j = w - chunk_warps;
  if (j >= M) return;
  if (chunk_base != nullptr && chunk_base[j + 1] > chunk_base[j]) return;  // long row: finished later
  const float norm = numerators != nullptr ? 1.f : normalizer[j];
  const T* krow = nullptr;
  if (keep != nullptr) {
    const int64_t kr = keep[j];
    if (kr >= 0 && kr < x_rows) {
      krow = x + kr * xs;
    } else if (lane == 0) {
      atomicOr(&g_proj_err, kErrBadArgument);
    }
  }
  const int32_t* seg = seg_offsets + j * corners;
  T* drow = numerators != nullptr ? nullptr : out + j * os;
  // the row's accumulator lives in shared memory (each lane its own words), so the registers
  // hold only the in-flight source rows and the current corner's partial sums
  __shared__ uint64_t acc_s[kWarpsPerBlock][kScatterQ][V / 2][32];
  uint64_t (&acc)[kScatterQ][V / 2][32] = acc_s[threadIdx.x >> 5];
  for (int col0 = 0; col0 < C; col0 += 32 * kScatterQ * V) {
#pragma unroll
    for (int q = 0; q < kScatterQ; ++q) {
      const int col = col0 + (lane + 32 * q) * V;
      uint64_t k2[V / 2];
      if (krow != nullptr && col < C) {
        widen_pairs<T>(__ldg(reinterpret_cast<const uint4*>(krow + col)), k2);
      } else {
#pragma unroll
        for (int h = 0; h < V / 2; ++h) k2[h] = 0ull;
      }
#pragma unroll
      for (int h = 0; h < V / 2; ++h) acc[q][h][lane] = k2[h];
    }
    for (int c = 0; c < corners; ++c) {
      const int e0 = seg[c], e1 = seg[c + 1];
      if (e0 == e1) continue;
      uint64_t part[kScatterQ][V / 2];
#pragma unroll
      for (int q = 0; q < kScatterQ; ++q)
#pragma unroll
        for (int h = 0; h < V / 2; ++h) part[q][h] = 0ull;
      scatter_entries<T>(x, x_rows, xs, entry_src, entry_w, e0, e1, col0, C, lane, part);
#pragma unroll
      for (int q = 0; q < kScatterQ; ++q)
#pragma unroll
        for (int h = 0; h < V / 2; ++h) acc[q][h][lane] = fadd2(acc[q][h][lane], part[q][h]);
    }
#pragma unroll
    for (int q = 0; q < kScatterQ; ++q) {
      const int col = col0 + (lane + 32 * q) * V;
      if (col < C) {
        if (numerators != nullptr) {  // partial numerator: the fp32 sum as it stands
          float* nrow = numerators + j * C + col;
#pragma unroll
          for (int h = 0; h < V / 2; ++h) {
            float a, b;
            upk2(acc[q][h][lane], a, b);
            *reinterpret_cast<float2*>(nrow + 2 * h) = make_float2(a, b);
          }
          continue;
        }
        float o[V];
#pragma unroll
        for (int h = 0; h < V / 2; ++h) {
          float a, b;
          upk2(acc[q][h][lane], a, b);
          o[2 * h] = __fdiv_rn(a, norm);
          o[2 * h + 1] = __fdiv_rn(b, norm);
        }
        store_vec<T>(drow + col, o);
      }
    }
  }
}

// Long rows: keep row + the row's level-1 sums (or its level-0 chunk sums), in order, divided by
// the normaliser.  One warp per merged row; short rows exit.
template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    scatter_finish_kernel(const T* __restrict__ x, long long x_rows, long long xs, const int64_t* __restrict__ keep,
                          long long M, const float* __restrict__ normalizer, T* __restrict__ out, long long os,
                          int C, const int32_t* __restrict__ chunk_base, const float* __restrict__ partials,
                          const int32_t* __restrict__ group_base, const float* __restrict__ partials1,
                          float* __restrict__ numerators) {
  constexpr int V = Vec<T>::N;
  const long long j = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (j >= M || chunk_base[j + 1] == chunk_base[j]) return;
  const float norm = numerators != nullptr ? 1.f : normalizer[j];
  const T* krow = nullptr;
  if (keep != nullptr) {
    const int64_t kr = keep[j];
    if (kr >= 0 && kr < x_rows) {
      krow = x + kr * xs;
    } else if (lane == 0) {
      atomicOr(&g_proj_err, kErrBadArgument);
    }
  }
  const bool grouped = group_base[j + 1] > group_base[j];
  const float* src = grouped ? partials1 : partials;
  const int k0 = grouped ? group_base[j] : chunk_base[j];
  const int k1 = grouped ? group_base[j + 1] : chunk_base[j + 1];
  T* drow = out + j * os;
  for (int col = lane * V; col < C; col += 32 * V) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (krow != nullptr) {
      float kv[V];
      load_vec<T>(krow + col, kv);
#pragma unroll
      for (int e = 0; e < V; ++e) acc[e] = kv[e];
    }
    sum_partials<4>(src, k0, k1, C, col, acc, V);
    if (numerators != nullptr) {
#pragma unroll
      for (int e = 0; e < V; ++e) numerators[j * C + col + e] = acc[e];
      continue;
    }
    float o[V];
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = __fdiv_rn(acc[e], norm);
    store_vec<T>(drow + col, o);
  }
}

// Rank-ordered reduction of partial numerators (the sharded scatter): out[j] = (x[keep[j]] +
// sum over r = 0..R-1, in rank order, of partials[r][j]) / normalizer[j], fp32 sums rounded to T
// once.  partials [R, rows, C] fp32 (what an all-to-all delivered, rank r's slice at r);
// keep[j] < 0: no keep row.  One warp per row, 16-byte vectors.
template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    rank_reduce_rows_kernel(const float* __restrict__ partials, int R, long long rows, int C,
                            const T* __restrict__ x, long long x_rows, long long xs, const int64_t* __restrict__ keep,
                            const float* __restrict__ normalizer, T* __restrict__ out, long long os) {
  constexpr int V = Vec<T>::N;
  const long long j = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (j >= rows) return;
  const T* krow = nullptr;
  if (keep != nullptr && keep[j] >= 0) {
    if (keep[j] < x_rows) krow = x + keep[j] * xs;
    else if (lane == 0) atomicOr(&g_proj_err, kErrBadArgument);
  }
  const float norm = normalizer[j];
  for (int col = lane * V; col < C; col += 32 * V) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (krow != nullptr) {
      float kv[V];
      load_vec<T>(krow + col, kv);
#pragma unroll
      for (int e = 0; e < V; ++e) acc[e] = kv[e];
    }
    for (int r = 0; r < R; ++r) {
      const float* pr = partials + (static_cast<long long>(r) * rows + j) * C + col;
      const float4 a = *reinterpret_cast<const float4*>(pr);
      acc[0] = __fadd_rn(acc[0], a.x); acc[1] = __fadd_rn(acc[1], a.y);
      acc[2] = __fadd_rn(acc[2], a.z); acc[3] = __fadd_rn(acc[3], a.w);
      if (V == 8) {
        const float4 b = *reinterpret_cast<const float4*>(pr + 4);
        acc[4] = __fadd_rn(acc[4], b.x); acc[5] = __fadd_rn(acc[5], b.y);
        acc[6] = __fadd_rn(acc[6], b.z); acc[7] = __fadd_rn(acc[7], b.w);
      }
    }
    float o[V];
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = __fdiv_rn(acc[e], norm);
    store_vec<T>(out + j * os + col, o);
  }
}

// ------------------------------------------------------------------------------------------
// fused q/k LayerNorm + Q||K||V compaction
//
// The qkv row of a token is [q | k | v], each C = heads * 64 channels.  One warp per compact
// row j; lane l holds 16-byte vector l of every 256-channel chunk, i.e. channels [8l, 8l+8),
// so one head's 64 channels sit on 8 consecutive lanes and the LayerNorm statistics of a head
// are two 3-step shuffle reductions inside that lane octet.  For q and k every loaded row is
// normalised (fp32, biased variance, as nn.LayerNorm) before it is weighted, which is the
// reference order: q_norm / k_norm on every token, then compaction
// (vggt_omega/models/layers/attention.py:337-339, 354-374).  Tensor t is pooled (keep row +
// corner partial sums, divided by the normaliser) when bit t of pool_mask is set, otherwise
// it is the (normalised) keep row alone, as compact_key (token_merging.py:372-376).
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void layer_norm_octet(float (&x)[8], const float (&w)[8], const float (&b)[8],
                                                 float eps) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += x[i];
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  const float mean = s * (1.f / 64.f);
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float d = x[i] - mean;
    var = fmaf(d, d, var);
  }
  var += __shfl_xor_sync(0xffffffffu, var, 1);
  var += __shfl_xor_sync(0xffffffffu, var, 2);
  var += __shfl_xor_sync(0xffffffffu, var, 4);
  const float rstd = rsqrtf(var * (1.f / 64.f) + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = fmaf((x[i] - mean) * rstd, w[i], b[i]);
}

// LayerNorm statistics (mean, 1/sqrt(var + eps)) of every 64-channel head of the q and k
// blocks of each qkv row: stats[row][h] for q heads h < H, stats[row][H + h] for k heads.
template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    head_stats_kernel(const T* __restrict__ qkv, long long rows, long long xs, int C, float eps,
                      float2* __restrict__ stats) {
  constexpr int V = 8;
  const long long r = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int heads2 = 2 * C / 64;
  constexpr int kBatch = 8;  // 16-byte loads issued before any is reduced (2C <= 8 * 256 per pass)
  for (int base = 0; base < 2 * C; base += kBatch * 32 * V) {
  uint4 raw[kBatch];
#pragma unroll
  for (int b = 0; b < kBatch; ++b) {
    const int col = base + (b * 32 + lane) * V;
    if (col < 2 * C) raw[b] = __ldg(reinterpret_cast<const uint4*>(qkv + r * xs + col));
  }
#pragma unroll
  for (int b = 0; b < kBatch; ++b) {
    const int col = base + (b * 32 + lane) * V;
    if (col >= 2 * C) break;  // uniform across the warp
    float x[V];
    const T* xe = reinterpret_cast<const T*>(&raw[b]);
#pragma unroll
    for (int i = 0; i < V; ++i) x[i] = to_f32<T>(xe[i]);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) s += x[i];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    const float mean = s * (1.f / 64.f);
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float d = x[i] - mean;
      var = fmaf(d, d, var);
    }
    var += __shfl_xor_sync(0xffffffffu, var, 1);
    var += __shfl_xor_sync(0xffffffffu, var, 2);
    var += __shfl_xor_sync(0xffffffffu, var, 4);
    if ((lane & 7) == 0) stats[r * heads2 + col / 64] = make_float2(mean, rsqrtf(var * (1.f / 64.f) + eps));
  }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, 2)
    compact_qkv_kernel(const T* __restrict__ qkv, long long rows, long long xs, int C,
                       const float* __restrict__ ln_w, const float* __restrict__ ln_b,
                       const float2* __restrict__ stats, const int64_t* __restrict__ keep, long long M,
                       int corners, const int32_t* __restrict__ seg_offsets, const int32_t* __restrict__ entry_src,
                       const float* __restrict__ entry_w, const float* __restrict__ normalizer,
                       int pool_mask, T* __restrict__ out, long long os) {
  // One warp per (compact row j, tensor t, 256-channel chunk); lane = one 16-byte vector.
  // Warps of one row are adjacent, so its CSR entries are shared through L1, and four
  // entries are loaded before any is reduced to keep four row fetches in flight per lane.
  // For q and k the LayerNorm is folded into the weighted sum: with (mu_e, r_e) the
  // statistics of the entry's head,
  //   sum_e w_e LN(x_e)_i = g_i (sum_e w_e r_e x_e,i - sum_e w_e r_e mu_e) + b_i sum_e w_e,
  // so each gathered element costs one FMA and the statistics come from head_stats_kernel.
  constexpr int V = 8;
  constexpr int kUnroll = 8;
  const int nch = C / (32 * V);
  const long long w_id = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long per_row = 3ll * nch;
  const long long j = w_id / per_row;
  if (j >= M) return;
  const int rem = static_cast<int>(w_id - j * per_row);
  const int t = rem / nch;
  const int col = (rem - t * nch) * 32 * V + lane * V;  // channel within the tensor
  const bool ln = ln_w != nullptr && t < 2;
  const bool pooled = (pool_mask >> t) & 1;
  const int heads2 = 2 * C / 64;
  const int head = t * (C / 64) + col / 64;  // index into a row of stats (q heads, then k heads)
  int64_t kr = keep[j];
  if (kr < 0 || kr >= rows) {
    if (lane == 0) atomicOr(&g_proj_err, kErrBadArgument);
    kr = 0;
  }
  const T* xcol = qkv + t * C + col;
  float acc[V];
  float csum = 0.f, wsum = 1.f;  // the keep row enters with weight 1
  load_vec<T>(xcol + kr * xs, acc);
  if (ln) {
    const float2 st = stats[kr * heads2 + head];
#pragma unroll
    for (int q = 0; q < V; ++q) acc[q] *= st.y;
    csum = st.x * st.y;
  }
  if (pooled) {
    // The row's entries of all corners are one contiguous CSR range (corner-major, source
    // order inside a corner); walking it as one list keeps kUnroll fetches in flight.
    const int e0 = seg_offsets[j * corners], e1 = seg_offsets[(j + 1) * corners];
    {
      float part[V];
      float pc = 0.f, pw = 0.f;
#pragma unroll
      for (int q = 0; q < V; ++q) part[q] = 0.f;
      for (int e = e0; e < e1; e += kUnroll) {
        uint4 x[kUnroll];  // raw 16-bit rows, converted when reduced (keeps registers low)
        float w[kUnroll];
        float2 st[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          int s = 0;
          w[u] = 0.f;
          if (e + u < e1) {
            s = __ldg(entry_src + e + u);
            w[u] = __ldg(entry_w + e + u);
            if (s < 0 || s >= rows) {
              if (lane == 0) atomicOr(&g_proj_err, kErrBadArgument);
              s = 0;
              w[u] = 0.f;
            }
          }
          x[u] = __ldg(reinterpret_cast<const uint4*>(xcol + static_cast<long long>(s) * xs));
          st[u] = ln ? stats[static_cast<long long>(s) * heads2 + head] : make_float2(0.f, 1.f);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const float a = w[u] * st[u].y;  // w_e r_e (w_e for v)
          const T* xe = reinterpret_cast<const T*>(&x[u]);
#pragma unroll
          for (int q = 0; q < V; ++q) part[q] = fmaf(a, to_f32<T>(xe[q]), part[q]);
          pc = fmaf(a, st[u].x, pc);
          pw += w[u];
        }
      }
#pragma unroll
      for (int q = 0; q < V; ++q) acc[q] += part[q];
      csum += pc;
      wsum += pw;
    }
  }
  if (ln) {
    const int oct = lane & 7;
#pragma unroll
    for (int q = 0; q < V; ++q)
      acc[q] = fmaf(ln_w[t * 64 + oct * 8 + q], acc[q] - csum, ln_b[t * 64 + oct * 8 + q] * wsum);
  }
  if (pooled) {
    const float norm = normalizer[j];
#pragma unroll
    for (int q = 0; q < V; ++q) acc[q] = __fdiv_rn(acc[q], norm);
  }
  store_vec<T>(out + j * os + t * C + col, acc);
}

// Staged compaction for C <= 1024: the same result as compact_qkv_kernel, with the source rows
// fetched by the bulk-copy engine instead of per-thread loads.
//   warps 0 .. 3C/256-1   consumers: thread i owns channels [8i, 8i + 8) of the q|k|v row
//   last warp             producer: for every item (the keep row, then the CSR entries of the
//                         merged row) one cp.async.bulk of the whole 3C-channel source row and
//                         one of its 2H LayerNorm statistics into a ring of shared-memory slots.
// CTAs take merged rows j = blockIdx.x, blockIdx.x + gridDim.x, ..., so at any time the GPU works
// on neighbouring merged rows, whose sources overlap and stay in L2.  Per item a consumer thread
// reads 16 bytes and one float2 of statistics from shared memory and does 4 packed FMAs; the
// copy engine keeps up to kStageSlots rows in flight per CTA without holding registers.
// Ring slots per CTA.  Measured on config 2 (compact_qkv incl. statistics, 16 channels per
// thread): 16 slots x 2 CTAs/SM 171 us, 10 x 3 159 us, 8 x 3 146 us, 8 x 4 138 us (8-channel
// threads, 16 x 2: 165 us).  Many small CTAs beat deep rings.
constexpr int kStageSlots = 8;
constexpr int kIssueLanes = 4;  // producer lanes that issue copies together
constexpr int kStageHeaderBytes = 512;

// Two 16-bit values of one 32-bit word as an fp32 pair (low half first).  bf16 -> fp32 is a
// shift of the bit pattern.
template <typename T>
__device__ __forceinline__ uint64_t unpack2(uint32_t w);
template <>
__device__ __forceinline__ uint64_t unpack2<__nv_bfloat16>(uint32_t w) {
  return pk2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ uint64_t unpack2<__half>(uint32_t w) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
  return pk2(f.x, f.y);
}
struct StageSlotMeta {
  int src;
  float w;
};
// Destinations of the compacted k|v rows in other GPUs' memory (peer-mapped buffers): row j
// of this call lands at row row0 + j of every listed buffer, k then v ([rows, 2C]).
constexpr int kMaxKvPeers = 16;
struct KvPeers {
  uint64_t dst[kMaxKvPeers];
  long long row0, stride;  // stride in elements
  int world;               // 0: no peer writes
  int multicast;           // 1: dst[0] is a multicast (NVLS) address covering every rank's buffer
};

// One 16-byte store through a multicast address: the NVLink switch writes it into the memory of
// every GPU bound to the multicast object.
__device__ __forceinline__ void multimem_st16(void* p, const uint4& v) {
  asm volatile("multimem.st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
static_assert(2 * kStageSlots * 8 + kStageSlots * sizeof(StageSlotMeta) <= kStageHeaderBytes, "stage header");

// kCh channels per consumer thread: 16 when 3C/16 threads make whole warps (C = 512, 1024),
// else 8 (C = 256); 16 halves the per-item bookkeeping (slot wait, vote, release) per channel.
template <typename T, int kCh>
__global__ void __launch_bounds__(kCh == 8 ? 416 : 224, kCh == 8 ? 2 : 4)
    compact_qkv_staged_kernel(const T* __restrict__ qkv, long long rows, long long xs, int C,
                              const float* __restrict__ ln_w, const float* __restrict__ ln_b,
                              const float2* __restrict__ stats, const int64_t* __restrict__ keep, long long M,
                              int corners, const int32_t* __restrict__ seg_offsets,
                              const int32_t* __restrict__ entry_src, const float* __restrict__ entry_w,
                              const float* __restrict__ normalizer, int pool_mask, T* __restrict__ out,
                              long long os, const __grid_constant__ KvPeers peers) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int n_cons = 3 * C / kCh;  // consumer threads, a whole number of warps
  const int heads2 = 2 * C / 64;
  const uint32_t row_bytes = static_cast<uint32_t>(3 * C * sizeof(T));
  const uint32_t stat_bytes = ln_w != nullptr ? static_cast<uint32_t>(heads2 * sizeof(float2)) : 0u;
  const uint32_t slot_bytes = row_bytes + stat_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStageSlots;
  StageSlotMeta* meta = reinterpret_cast<StageSlotMeta*>(empty + kStageSlots);
  uint8_t* data = smem + kStageHeaderBytes;  // after the barriers (256 B) and slot metadata (128 B)
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cons_warps = n_cons / 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStageSlots; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), cons_warps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const bool pooled_any = pool_mask != 0;

  if (warp == cons_warps) {
    // ------------------------------- producer -------------------------------
    // The whole warp walks the item stream; lane u holds entry u of the current merged row
    // (loaded together, one row ahead of use), and lane 0 issues each item's copies as soon as
    // its slot is free, taking (source, weight) from the owning lane by shuffle.
    long long item = 0;
    bool ok = true;
    auto load_row = [&](long long jr, int& e0, int& e1, long long& kr, int& src, float& w) {
      e0 = pooled_any ? seg_offsets[jr * corners] : 0;
      e1 = pooled_any ? seg_offsets[(jr + 1) * corners] : 0;
      kr = keep[jr];
      src = 0;
      w = 0.f;
      if (e0 + lane < e1) {
        src = entry_src[e0 + lane];
        w = entry_w[e0 + lane];
      }
    };
    int e0 = 0, e1 = 0, src = 0;
    long long kr = 0;
    float w = 0.f;
    if (blockIdx.x < M) load_row(blockIdx.x, e0, e1, kr, src, w);
    for (long long j = blockIdx.x; j < M && ok; j += gridDim.x) {
      int ne0 = 0, ne1 = 0, nsrc = 0;
      long long nkr = 0;
      float nw = 0.f;
      if (j + gridDim.x < M) load_row(j + gridDim.x, ne0, ne1, nkr, nsrc, nw);  // next row, ahead of use
      const int n_items = e1 - e0 + 1;  // the keep row, then the entries
      for (int u0 = 0; u0 < n_items && ok; u0 += kIssueLanes) {
        // lanes 0..kIssueLanes-1 take items u0 + lane: a batch waits only for the oldest
        // kIssueLanes slots, so the ring stays at least kStageSlots - kIssueLanes deep
        const int u = u0 + lane;
        long long s = __shfl_sync(0xffffffffu, src, (u - 1) & 31);
        float wi = __shfl_sync(0xffffffffu, w, (u - 1) & 31);
        const bool mine = lane < kIssueLanes && u < n_items;
        bool wok = true;
        if (mine) {
          if (u == 0) {
            s = kr;
            wi = 1.f;
          } else if (u > 32) {  // rows with more than 32 entries: read the rest directly
            s = entry_src[e0 + u - 1];
            wi = entry_w[e0 + u - 1];
          }
          if (s < 0 || s >= rows) {
            atomicOr(&g_proj_err, kErrBadArgument);
            s = 0;
            wi = 0.f;
          }
          const long long it = item + u;
          if (it >= kStageSlots)
            wok = mbar_wait(smem_u32(&empty[it % kStageSlots]), static_cast<uint32_t>((it / kStageSlots) - 1) & 1u,
                            &g_proj_err);
        }
        ok = __all_sync(0xffffffffu, wok);
        if (ok && mine) {
          const int slot = static_cast<int>((item + u) % kStageSlots);
          meta[slot].src = static_cast<int>(s);
          meta[slot].w = wi;
          const uint32_t dst = smem_u32(data + static_cast<size_t>(slot) * slot_bytes);
          const uint32_t bar = smem_u32(&full[slot]);
          mbar_arrive_expect_tx(bar, slot_bytes);
          bulk_load(dst, qkv + s * xs, row_bytes, bar);
          if (stat_bytes) bulk_load(dst + row_bytes, stats + s * heads2, stat_bytes, bar);
        }
      }
      item += n_items;
      e0 = ne0;
      e1 = ne1;
      kr = nkr;
      src = nsrc;
      w = nw;
    }
    return;  // no block-wide barrier follows
  }

  // ------------------------------- consumers -------------------------------
  // Thread i owns channels [kCh i, kCh i + kCh) of the q|k|v row (one tensor, one LayerNorm
  // head).  Each item is released as soon as the warp has read it; each 16-bit pair becomes an
  // fp32 pair for one packed FMA.
  constexpr int kVecs = kCh / 8;  // 16-byte vectors per thread
  const int i = threadIdx.x;
  const int t = i / (C / kCh);               // tensor: 0 q, 1 k, 2 v
  const int col = (i - t * (C / kCh)) * kCh;  // channel within the tensor
  const bool ln = ln_w != nullptr && t < 2;
  const bool pooled_t = (pool_mask >> t) & 1;
  const int stat_idx = t * (C / 64) + col / 64;
  long long item = 0;
  bool ok = true;
  for (long long j = blockIdx.x; j < M && ok; j += gridDim.x) {
    const int e0 = pooled_any ? seg_offsets[j * corners] : 0;
    const int e1 = pooled_any ? seg_offsets[(j + 1) * corners] : 0;
    const int n_items = e1 - e0 + 1;
    uint64_t acc2[kCh / 2];
#pragma unroll
    for (int q = 0; q < kCh / 2; ++q) acc2[q] = 0ull;  // (+0.0f, +0.0f)
    float csum = 0.f, wsum = 0.f;
    for (int u = 0; u < n_items; ++u) {
      const long long it = item + u;
      const int slot = static_cast<int>(it % kStageSlots);
      ok = __all_sync(0xffffffffu,
                      mbar_wait(smem_u32(&full[slot]), static_cast<uint32_t>(it / kStageSlots) & 1u, &g_proj_err));
      if (!ok) break;
      if (u == 0 || pooled_t) {  // item 0 is the keep row
        const uint8_t* base = data + static_cast<size_t>(slot) * slot_bytes;
        float a = meta[slot].w;
        wsum += a;
        if (ln) {
          const float2 st = reinterpret_cast<const float2*>(base + row_bytes)[stat_idx];
          a *= st.y;  // w r
          csum = fmaf(a, st.x, csum);
        }
        uint4 r0[kVecs];
#pragma unroll
        for (int v = 0; v < kVecs; ++v) r0[v] = reinterpret_cast<const uint4*>(base)[i * kVecs + v];
        const uint64_t a2 = pk2(a, a);
#pragma unroll
        for (int v = 0; v < kVecs; ++v) {
          acc2[4 * v + 0] = ffma2(a2, unpack2<T>(r0[v].x), acc2[4 * v + 0]);
          acc2[4 * v + 1] = ffma2(a2, unpack2<T>(r0[v].y), acc2[4 * v + 1]);
          acc2[4 * v + 2] = ffma2(a2, unpack2<T>(r0[v].z), acc2[4 * v + 2]);
          acc2[4 * v + 3] = ffma2(a2, unpack2<T>(r0[v].w), acc2[4 * v + 3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty[slot]));
    }
    item += n_items;
    if (!ok) break;
    float acc[kCh];
#pragma unroll
    for (int q = 0; q < kCh / 2; ++q) upk2(acc2[q], acc[2 * q], acc[2 * q + 1]);
    if (ln) {
#pragma unroll
      for (int q = 0; q < kCh; ++q)
        acc[q] = fmaf(__ldg(ln_w + t * 64 + col % 64 + q), acc[q] - csum, __ldg(ln_b + t * 64 + col % 64 + q) * wsum);
    }
    if (pooled_t) {
      const float norm = normalizer[j];
#pragma unroll
      for (int q = 0; q < kCh; ++q) acc[q] = __fdiv_rn(acc[q], norm);
    }
    uint4 raw[kVecs];
    T* e = reinterpret_cast<T*>(raw);
#pragma unroll
    for (int q = 0; q < kCh; ++q) e[q] = from_f32<T>(acc[q]);
#pragma unroll
    for (int v = 0; v < kVecs; ++v) reinterpret_cast<uint4*>(out + j * os + t * C + col)[v] = raw[v];
    if (t > 0 && peers.world > 0) {
      // the k|v all-gather, fused: posted stores straight into every rank's key/value buffer
      // (one multicast store, or one store per rank)
      const long long off = (peers.row0 + j) * peers.stride + (t - 1) * C + col;
#pragma unroll
      for (int v = 0; v < kVecs; ++v) {
        if (peers.multicast) {
          multimem_st16(reinterpret_cast<T*>(peers.dst[0]) + off + 8 * v, raw[v]);
        } else {
          for (int r = 0; r < peers.world; ++r)
            reinterpret_cast<uint4*>(reinterpret_cast<T*>(peers.dst[r]) + off)[v] = raw[v];
        }
      }
    }
  }
  if (peers.world > 0) {
    // peer / multicast stores ordered before whatever the stream signals next
    if (peers.multicast) asm volatile("fence.proxy.alias;" ::: "memory");
    __threadfence_system();
  }
}

// Per-head LayerNorm of the q block of qkv rows (query-preserving plans keep every query).
template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    head_layernorm_kernel(const T* __restrict__ x, long long rows, long long xs, int C,
                          const float* __restrict__ w, const float* __restrict__ b, float eps,
                          T* __restrict__ out, long long os) {
  constexpr int V = 8;
  const long long r = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int oct = lane & 7;
  float lw[8], lb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    lw[i] = w[oct * 8 + i];
    lb[i] = b[oct * 8 + i];
  }
  for (int col = lane * V; col < C; col += 32 * V) {
    float v[V];
    load_vec<T>(x + r * xs + col, v);
    layer_norm_octet(v, lw, lb, eps);
    store_vec<T>(out + r * os + col, v);
  }
}

// ------------------------------------------------------------------------------------------
// plan CSR
// ------------------------------------------------------------------------------------------
__global__ void csr_keys_kernel(const int64_t* __restrict__ parent, long long n, int corners,
                                long long M, int32_t* __restrict__ keys, int32_t* __restrict__ vals,
                                int32_t* __restrict__ counts, int32_t dropped_key) {
  const long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const long long s = e / corners;
  const int c = static_cast<int>(e - s * corners);
  const int64_t p = parent[e];
  int32_t key = dropped_key;  // sorts after every valid key; never counted
  if (p >= 0 && p < M) {
    key = static_cast<int32_t>(p * corners + c);
    atomicAdd(counts + key, 1);  // integer counts: order-independent
  } else {
    atomicOr(&g_proj_err, kErrBadArgument);
  }
  keys[e] = key;
  vals[e] = static_cast<int32_t>(s);
}

__global__ void csr_entries_kernel(const int32_t* __restrict__ sorted_keys,
                                   const int32_t* __restrict__ sorted_src, long long n, int corners,
                                   const float* __restrict__ weights, const int64_t* __restrict__ src_rows,
                                   int32_t* __restrict__ entry_src, float* __restrict__ entry_w,
                                   int32_t dropped_key) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t key = sorted_keys[i];
  const int32_t s = sorted_src[i];
  if (key == dropped_key) {
    entry_src[i] = 0;
    entry_w[i] = 0.f;
    return;
  }
  const int c = key % corners;
  entry_src[i] = src_rows ? static_cast<int32_t>(src_rows[s]) : s;
  entry_w[i] = weights[static_cast<long long>(s) * corners + c];
}

// mass_j = 1 + sum_c (sum of segment (j, c)); one warp per row, fixed-order warp reduction.
__global__ void csr_mass_kernel(const int32_t* __restrict__ seg_offsets, const float* __restrict__ entry_w,
                                long long M, int corners, float* __restrict__ mass,
                                float* __restrict__ log_mass) {
  const long long j = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (j >= M) return;
  float total = 1.f;
  for (int c = 0; c < corners; ++c) {
    const int e0 = seg_offsets[j * corners + c], e1 = seg_offsets[j * corners + c + 1];
    float part = 0.f;
    for (int e = e0 + lane; e < e1; e += 32) part += entry_w[e];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    total += part;
  }
  if (lane == 0) {
    if (mass) mass[j] = total;
    if (log_mass) log_mass[j] = logf(total);
  }
}

// Grouped plans (every source's parents inside its own group of merged rows, as the
// frame-group planners build them): one CTA per group builds the group's part of the CSR in
// shared memory instead of the radix sort + scans of the general path.  Counts per segment
// (shared-memory atomics, order-independent), a block-wide exclusive scan, placement of
// (source, weight) pairs by per-segment cursors, then every segment's few entries are put in
// ascending source order (insertion sort, one thread per segment) and the group's entries are
// written out in order, so the result equals the general path's bit for bit.  Group g: sources
// [q_begin[g], q_begin[g+1]), merged rows [b_begin[g], b_begin[g+1]); its entries fill
// [q_begin[g], q_begin[g+1]) x corners of the entry arrays.  Masses follow in csr_mass_kernel.
constexpr int kCsrGroupThreads = 1024;
constexpr int kCsrMaxParts = 8;  // CTAs per frame group in the grouped CSR build
constexpr int kCsrGroupMaxSegments = 8 * 1024;    // shared-memory counters per group
constexpr int kCsrGroupMaxEntries = 16 * 1024;    // shared-memory entries per group (10 bytes each)

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int t = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += n;
    }
    if (lane < nw) warp_tot[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  const int base = warp > 0 ? warp_tot[warp - 1] : 0;
  return base + inc - v;
}

__global__ void __launch_bounds__(kCsrGroupThreads)
    csr_grouped_kernel(const int64_t* __restrict__ parent, const float* __restrict__ weights,
                       const int64_t* __restrict__ src_rows, int corners, long long M,
                       const int64_t* __restrict__ q_begin, const int64_t* __restrict__ b_begin, int groups,
                       int parts, int max_segments, int max_entries, int32_t* __restrict__ seg_offsets,
                       int32_t* __restrict__ entry_src, float* __restrict__ entry_w) {
  extern __shared__ __align__(16) int csr_smem[];
  __shared__ int warp_tot[32];
  __shared__ int n_staged, n_below;
  // shared memory: counters [max_segments] | placed weights [max_entries] | staged segment of each
  // pair (int16) | staged source (int16) | placed source (int16); a staged pair's weight is read
  // again from global memory (an L2 hit) when it is placed
  int* cnt = csr_smem;
  float* e_w = reinterpret_cast<float*>(cnt + max_segments);
  uint16_t* st_seg = reinterpret_cast<uint16_t*>(e_w + max_entries);
  uint16_t* st_src = st_seg + max_entries;
  uint16_t* e_src = st_src + max_entries;
  const int g = blockIdx.x / parts, part = blockIdx.x - (blockIdx.x / parts) * parts;
  const long long q0 = q_begin[g], q1 = q_begin[g + 1], b0 = b_begin[g], b1 = b_begin[g + 1];
  const int rows = static_cast<int>(b1 - b0);
  const int per = (rows + parts - 1) / parts;
  const int lo = min(rows, part * per), hi = min(rows, lo + per);  // this CTA's merged rows [lo, hi)
  const int nseg = (hi - lo) * corners;
  const int n = static_cast<int>((q1 - q0) * corners);
  const long long e_base = q0 * corners;
  if (nseg > max_segments || n > max_entries || (rows == 0 && n > 0)) {
    if (threadIdx.x == 0) atomicOr(&g_proj_err, kErrBadArgument);  // the host checks make this unreachable
    return;
  }
  if (threadIdx.x == 0) {
    n_staged = 0;
    n_below = 0;
  }
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  // Every part scans all of the group's pairs: it stages the pairs whose parent lies in its rows
  // and counts the valid pairs below them (its entries' offset in the group).  Four coalesced
  // loads per thread in flight at a time, one error report per thread.
  bool bad = false;
  int below = 0;
  const int stride = blockDim.x;
  for (int e0 = threadIdx.x; e0 < n; e0 += 4 * stride) {
    int64_t pv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = e0 + u * stride;
      if (e < n) pv[u] = parent[e_base + e];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = e0 + u * stride;
      if (e < n) {
        const long long p = pv[u] - b0;
        const bool ok = p >= 0 && p < rows;
        bad |= !ok;
        if (ok && p < lo) {
          ++below;
        } else if (ok && p < hi) {
          const int slot = atomicAdd(&n_staged, 1);
          st_seg[slot] = static_cast<uint16_t>((p - lo) * corners + e % corners);
          st_src[slot] = static_cast<uint16_t>(e / corners);
        }
      }
    }
  }
  if (bad && part == 0) atomicOr(&g_proj_err, kErrBadArgument);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) below += __shfl_xor_sync(0xffffffffu, below, o);
  if ((threadIdx.x & 31) == 0 && below) atomicAdd(&n_below, below);
  __syncthreads();
  const int staged = n_staged;
  for (int i = threadIdx.x; i < staged; i += blockDim.x) atomicAdd(&cnt[st_seg[i]], 1);
  __syncthreads();
  // exclusive scan: thread t scans a contiguous chunk of the counts
  const long long off0 = e_base + n_below;  // this part's first entry
  const int chunk = (nseg + blockDim.x - 1) / blockDim.x;
  const int i0 = min(nseg, static_cast<int>(threadIdx.x) * chunk), i1 = min(nseg, i0 + chunk);
  int local = 0;
  for (int i = i0; i < i1; ++i) local += cnt[i];
  int run = block_exclusive_scan(local, warp_tot);
  for (int i = i0; i < i1; ++i) {
    const int c = cnt[i];
    cnt[i] = run;  // the segment's first entry (part-relative), the cursor below
    seg_offsets[(b0 + lo) * corners + i] = static_cast<int32_t>(off0 + run);
    run += c;
  }
  __syncthreads();
  // placement (arbitrary order inside a segment for now)
  for (int i = threadIdx.x; i < staged; i += blockDim.x) {
    const int sg = st_seg[i];
    const int pos = atomicAdd(&cnt[sg], 1);
    e_src[pos] = st_src[i];
    e_w[pos] = weights[e_base + static_cast<long long>(st_src[i]) * corners + sg % corners];
  }
  __syncthreads();
  if (g == groups - 1 && part == parts - 1 && threadIdx.x == 0)
    for (long long j = b1 * corners; j <= M * corners; ++j) seg_offsets[j] = static_cast<int32_t>(off0 + staged);
  // ascending source order inside each segment (segments hold a few entries each)
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) {
    const int a = i > 0 ? cnt[i - 1] : 0, b = cnt[i];
    for (int x = a + 1; x < b; ++x) {
      const uint16_t ks = e_src[x];
      const float kw = e_w[x];
      int y = x - 1;
      while (y >= a && e_src[y] > ks) {
        e_src[y + 1] = e_src[y];
        e_w[y + 1] = e_w[y];
        --y;
      }
      e_src[y + 1] = ks;
      e_w[y + 1] = kw;
    }
  }
  __syncthreads();
  for (int e0 = threadIdx.x; e0 < staged; e0 += 4 * stride) {
    long long sv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = e0 + u * stride;
      if (e < staged) {
        const long long src = q0 + e_src[e];
        sv[u] = src_rows ? src_rows[src] : src;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = e0 + u * stride;
      if (e < staged) {
        entry_src[off0 + e] = static_cast<int32_t>(sv[u]);
        entry_w[off0 + e] = e_w[e];
      }
    }
  }
}

// ------------------------------------------------------------------------------------------
// row normalisation to bf16
// ------------------------------------------------------------------------------------------
// One warp per row.  Rows of up to kNormVecs 16-byte vectors per lane (2048 bf16 channels) are
// read once into registers, reduced, and scaled from registers; wider rows take a second read.
constexpr int kNormVecs = 8;
template <typename T>
__global__ void row_normalize_kernel(const T* __restrict__ x, long long x_rows, long long xs,
                                     const int64_t* __restrict__ rows, long long R, int C, float eps,
                                     __nv_bfloat16* __restrict__ out, long long os) {
  constexpr int V = Vec<T>::N;
  const long long r = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const long long src = rows ? rows[r] : r;
  if (src < 0 || src >= x_rows) {
    if (lane == 0) atomicOr(&g_proj_err, kErrBadArgument);
    return;
  }
  const T* xr = x + src * xs;
  __nv_bfloat16* orow = out + r * os;
  const int nvec = C / V;
  // V input values -> V bf16 outputs (16 bytes for 16-bit input; two 16-byte halves for fp32)
  auto emit = [&](int i, const float (&v)[V], float denom) {
    uint32_t w[V / 2];
#pragma unroll
    for (int e = 0; e < V; e += 2) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(__fdiv_rn(v[e], denom), __fdiv_rn(v[e + 1], denom));
      w[e / 2] = *reinterpret_cast<const uint32_t*>(&b);
    }
    if constexpr (V == 8) {
      *reinterpret_cast<uint4*>(orow + i * V) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      *reinterpret_cast<uint2*>(orow + i * V) = make_uint2(w[0], w[1]);
    }
  };
  if (nvec <= 32 * kNormVecs) {
    uint4 raw[kNormVecs];
#pragma unroll
    for (int k = 0; k < kNormVecs; ++k)
      if (lane + 32 * k < nvec) raw[k] = __ldg(reinterpret_cast<const uint4*>(xr) + lane + 32 * k);
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kNormVecs; ++k) {
      if (lane + 32 * k < nvec) {
        const T* e = reinterpret_cast<const T*>(&raw[k]);
#pragma unroll
        for (int q = 0; q < V; ++q) {
          const float f = to_f32<T>(e[q]);
          ss = fmaf(f, f, ss);
        }
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float denom = fmaxf(sqrtf(ss), eps);
#pragma unroll
    for (int k = 0; k < kNormVecs; ++k) {
      if (lane + 32 * k < nvec) {
        float v[V];
        const T* e = reinterpret_cast<const T*>(&raw[k]);
#pragma unroll
        for (int q = 0; q < V; ++q) v[q] = to_f32<T>(e[q]);
        emit(lane + 32 * k, v, denom);
      }
    }
    return;
  }
  float ss = 0.f;
  for (int i = lane; i < nvec; i += 32) {
    float v[V];
    load_vec<T>(xr + i * V, v);
#pragma unroll
    for (int e = 0; e < V; ++e) ss = fmaf(v[e], v[e], ss);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float denom = fmaxf(sqrtf(ss), eps);
  for (int i = lane; i < nvec; i += 32) {
    float v[V];
    load_vec<T>(xr + i * V, v);
    emit(i, v, denom);
  }
}

inline int elem_size(int dtype) { return dtype == VB200_F32 ? 4 : 2; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline unsigned row_blocks(long long rows) {
  return static_cast<unsigned>((rows + kWarpsPerBlock - 1) / kWarpsPerBlock);
}

int check_rows(int dtype, const void* p, int64_t row_stride, int64_t C, const char* name) {
  const int es = elem_size(dtype);
  VB200_REQUIRE((C * es) % 16 == 0, "%s: channels (%lld) must be a multiple of %d", name,
                (long long)C, 16 / es);
  VB200_REQUIRE(aligned16(p) && (row_stride * es) % 16 == 0,
                "%s: rows must be 16-byte aligned (row stride %lld elements)", name,
                (long long)row_stride);
  return VB200_OK;
}

struct CsrWorkspace {
  size_t keys_in, keys_out, vals_in, vals_out, counts, sort_tmp, scan_tmp, total;
  size_t sort_bytes, scan_bytes;
};

CsrWorkspace csr_layout(int64_t S, int64_t corners, int64_t M) {
  const int n = static_cast<int>(S * corners);
  const int nseg = static_cast<int>(M * corners + 1);
  CsrWorkspace w{};
  size_t sort_bytes = 0, scan_bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, static_cast<int32_t*>(nullptr),
                                  static_cast<int32_t*>(nullptr), static_cast<int32_t*>(nullptr),
                                  static_cast<int32_t*>(nullptr), n > 0 ? n : 1);
  cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<int32_t*>(nullptr),
                                static_cast<int32_t*>(nullptr), nseg);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t nb = static_cast<size_t>(n > 0 ? n : 1) * 4;
  w.keys_in = take(nb);
  w.keys_out = take(nb);
  w.vals_in = take(nb);
  w.vals_out = take(nb);
  w.counts = take(static_cast<size_t>(nseg) * 4);
  w.sort_tmp = take(sort_bytes);
  w.scan_tmp = take(scan_bytes);
  w.total = off;
  w.sort_bytes = sort_bytes;
  w.scan_bytes = scan_bytes;
  return w;
}

}  // namespace

unsigned projection_error_word(int clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_proj_err, sizeof(v));
  if (clear) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_proj_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace vb200

using namespace vb200;

extern "C" int vb200_row_gather(int dtype, const void* x, int64_t x_rows, int64_t xs, const int64_t* index,
                                int64_t R, void* out, int64_t os, int64_t C, void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "row_gather: bad dtype %d", dtype);
  VB200_REQUIRE(R >= 0 && C >= 0, "row_gather: negative size");
  if (R == 0 || C == 0) return VB200_OK;
  VB200_REQUIRE(x && out && index, "row_gather: null pointer");
  int rc;
  if ((rc = check_rows(dtype, x, xs, C, "row_gather input")) != VB200_OK) return rc;
  if ((rc = check_rows(dtype, out, os, C, "row_gather output")) != VB200_OK) return rc;
  const int es = elem_size(dtype);
  row_gather_kernel<<<row_blocks(R), kWarpsPerBlock * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(x), x_rows, xs * es, index, R, static_cast<uint8_t*>(out), os * es,
      static_cast<int>(C * es / 16));
  VB200_CHECK_LAUNCH("row_gather_kernel");
  return VB200_OK;
}

extern "C" int vb200_proj_gather(int dtype, const void* y, int64_t ys, const int64_t* keep,
                                 int64_t K, const int64_t* src, const int64_t* parent,
                                 const float* w, int64_t S, int64_t corners, void* out, int64_t os,
                                 int64_t N_out, int64_t C, int zero_fill, void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "proj_gather: bad dtype %d", dtype);
  VB200_REQUIRE(K >= 0 && S >= 0 && N_out >= 0 && C >= 0, "proj_gather: negative size");
  VB200_REQUIRE(corners >= 1 && corners <= 4, "proj_gather: corners must be in [1, 4] (got %lld)",
                (long long)corners);
  if (C == 0 || N_out == 0) return VB200_OK;
  VB200_REQUIRE(out != nullptr && (K == 0 || y) && (S == 0 || (src && parent && w)), "proj_gather: null pointer");
  VB200_REQUIRE(S == 0 || K > 0, "proj_gather: sources need at least one compact row to read");
  int rc;
  if (K > 0 && (rc = check_rows(dtype, y, ys, C, "proj_gather input")) != VB200_OK) return rc;
  if ((rc = check_rows(dtype, out, os, C, "proj_gather output")) != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (zero_fill) {
#define VB200_ZERO(T) zero_rows_kernel<T><<<row_blocks(N_out), kWarpsPerBlock * 32, 0, st>>>( \
      static_cast<T*>(out), os, N_out, static_cast<int>(C))
    if (dtype == VB200_F32) VB200_ZERO(float);
    else if (dtype == VB200_BF16) VB200_ZERO(__nv_bfloat16);
    else VB200_ZERO(__half);
#undef VB200_ZERO
    VB200_CHECK_LAUNCH("zero_rows_kernel");
  }
  if (K + S == 0) return VB200_OK;
  // Large plans: batches of up to 32 sources per warp with whole rows in flight (one coalesced
  // index load per batch; at least ~16 resident warps' worth of batches per SM).  Small plans:
  // one source per warp, one vector per lane, twice the resident warps.
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool batched = S >= kGatherBatchMin;
  const int per_warp =
      batched ? static_cast<int>(std::max<long long>(1, std::min<long long>(32, S / (static_cast<long long>(sms) * 16))))
              : 1;
  const unsigned grid = row_blocks((keep != nullptr ? K : 0) + (S + per_warp - 1) / per_warp);
#define VB200_GATHER(T)                                                                                    \
  do {                                                                                                     \
    if (batched)                                                                                           \
      proj_gather_kernel<T, 4, 4><<<grid, kWarpsPerBlock * 32, 0, st>>>(                                   \
          static_cast<const T*>(y), ys, keep, K, src, parent, w, S, static_cast<int>(corners),             \
          static_cast<T*>(out), os, N_out, static_cast<int>(C), per_warp);                                 \
    else                                                                                                   \
      proj_gather_kernel<T, 4, 1><<<grid, kWarpsPerBlock * 32, 0, st>>>(                                   \
          static_cast<const T*>(y), ys, keep, K, src, parent, w, S, static_cast<int>(corners),             \
          static_cast<T*>(out), os, N_out, static_cast<int>(C), per_warp);                                 \
  } while (0)
  if (dtype == VB200_F32) VB200_GATHER(float);
  else if (dtype == VB200_BF16) VB200_GATHER(__nv_bfloat16);
  else VB200_GATHER(__half);
#undef VB200_GATHER
  VB200_CHECK_LAUNCH("proj_gather_kernel");
  return VB200_OK;
}

extern "C" int vb200_plan_hot_rows(const int32_t* seg_offsets, int64_t M, int64_t corners, int max_hot,
                                   int32_t* hot_rows, int32_t* hot_slot, int32_t* n_hot, void* stream) {
  VB200_REQUIRE(M >= 0 && corners >= 1 && max_hot >= 0, "plan_hot_rows: bad sizes");
  VB200_REQUIRE(seg_offsets && hot_slot && n_hot && (max_hot == 0 || hot_rows), "plan_hot_rows: null pointer");
  plan_hot_rows_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(seg_offsets, M, static_cast<int>(corners),
                                                                          max_hot, hot_rows, hot_slot, n_hot);
  VB200_CHECK_LAUNCH("plan_hot_rows_kernel");
  return VB200_OK;
}

extern "C" int vb200_proj_gather_hot_capacity(int dtype, int64_t C) {
  const int es = elem_size(dtype);
  if (C <= 0) return 0;
  const long long row = C * es;
  return static_cast<int>(std::min<long long>(kMaxHotRows, kHotSmemBytes / row));
}

extern "C" int vb200_proj_gather_hot(int dtype, const void* y, int64_t ys, const int64_t* keep, int64_t K,
                                     const int64_t* src, const int64_t* parent, const float* w, int64_t S,
                                     int64_t corners, void* out, int64_t os, int64_t N_out, int64_t C,
                                     const int32_t* hot_rows, const int32_t* hot_slot, const int32_t* n_hot,
                                     int max_hot, void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "proj_gather_hot: bad dtype %d",
                dtype);
  VB200_REQUIRE(K >= 0 && S >= 0 && N_out >= 0 && C >= 0, "proj_gather_hot: negative size");
  VB200_REQUIRE(corners >= 1 && corners <= 4, "proj_gather_hot: corners must be in [1, 4] (got %lld)",
                (long long)corners);
  if (C == 0 || N_out == 0 || K + S == 0) return VB200_OK;
  VB200_REQUIRE(out != nullptr && (K == 0 || y) && (S == 0 || (src && parent && w)), "proj_gather_hot: null pointer");
  VB200_REQUIRE(hot_slot && n_hot && hot_rows, "proj_gather_hot: null hot-row table");
  VB200_REQUIRE(S == 0 || K > 0, "proj_gather_hot: sources need at least one compact row to read");
  const int cap = vb200_proj_gather_hot_capacity(dtype, C);
  VB200_REQUIRE(max_hot >= 0 && max_hot <= cap, "proj_gather_hot: max_hot %d exceeds the shared-memory capacity %d",
                max_hot, cap);
  int rc;
  if (K > 0 && (rc = check_rows(dtype, y, ys, C, "proj_gather_hot input")) != VB200_OK) return rc;
  if ((rc = check_rows(dtype, out, os, C, "proj_gather_hot output")) != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = static_cast<size_t>(max_hot) * static_cast<size_t>(C) * elem_size(dtype);
  int dev = 0, sms = 0;
  VB200_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  VB200_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
  const long long rows = K + S;
  const unsigned grid = static_cast<unsigned>(std::max<long long>(1, std::min<long long>(sms, (rows + kHotWarps - 1) / kHotWarps)));
#define VB200_GATHER_HOT(T)                                                                                \
  do {                                                                                                     \
    VB200_CHECK_CUDA(cudaFuncSetAttribute(proj_gather_hot_kernel<T, 4>,                                    \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)), \
                     "cudaFuncSetAttribute");                                                              \
    proj_gather_hot_kernel<T, 4><<<grid, kHotWarps * 32, smem, st>>>(                                      \
        static_cast<const T*>(y), ys, keep, K, src, parent, w, S, static_cast<int>(corners),               \
        static_cast<T*>(out), os, N_out, static_cast<int>(C), hot_rows, hot_slot, n_hot, max_hot);         \
  } while (0)
  if (dtype == VB200_F32) VB200_GATHER_HOT(float);
  else if (dtype == VB200_BF16) VB200_GATHER_HOT(__nv_bfloat16);
  else VB200_GATHER_HOT(__half);
#undef VB200_GATHER_HOT
  VB200_CHECK_LAUNCH("proj_gather_hot_kernel");
  return VB200_OK;
}

struct ScatterWorkspace {
  size_t nchunk, chunk_base, ngroup, group_base, scan_tmp, partials, partials1, total, scan_bytes;
  long long bound, bound1;  // upper bounds on the numbers of level-0 chunks and level-1 groups
};

ScatterWorkspace scatter_layout(int64_t M, int64_t n_entries, int64_t C) {
  ScatterWorkspace w{};
  size_t scan_bytes = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<int32_t*>(nullptr), static_cast<int32_t*>(nullptr),
                                static_cast<int>(M + 1));
  // a long row (> L entries) has ceil(len / L) <= 2 len / L chunks, so all chunks <= 2 n / L
  w.bound = 2 * ((n_entries + kScatterChunk - 1) / kScatterChunk) + 1;
  w.bound1 = 2 * ((w.bound + kScatterGroup - 1) / kScatterGroup) + 1;  // same argument, one level up
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  w.nchunk = take(static_cast<size_t>(M + 1) * 4);
  w.chunk_base = take(static_cast<size_t>(M + 1) * 4);
  w.ngroup = take(static_cast<size_t>(M + 1) * 4);
  w.group_base = take(static_cast<size_t>(M + 1) * 4);
  w.scan_tmp = take(scan_bytes);
  w.partials = take(static_cast<size_t>(w.bound) * static_cast<size_t>(C) * 4);
  w.partials1 = take(static_cast<size_t>(w.bound1) * static_cast<size_t>(C) * 4);
  w.total = off;
  w.scan_bytes = scan_bytes;
  return w;
}

extern "C" size_t vb200_proj_scatter_workspace_size(int64_t M, int64_t n_entries, int64_t C) {
  if (M < 0 || n_entries < 0 || C < 0) return 0;
  return scatter_layout(M, n_entries, C).total;
}

namespace vb200 {
namespace {
// Both scatter forms: out = (keep + sums) / normalizer, or (numerators != NULL, keep and
// normalizer unused) the fp32 sums alone in numerators [M, C].
int scatter_launch(int dtype, const void* x, int64_t x_rows, int64_t xs, const int64_t* keep, int64_t M,
                   int64_t corners, const int32_t* seg_offsets, const int32_t* entry_src, const float* entry_w,
                   const float* normalizer, void* out, int64_t os, int64_t C, int64_t n_entries, void* workspace,
                   size_t workspace_bytes, float* numerators, void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "proj_scatter: bad dtype %d", dtype);
  VB200_REQUIRE(M >= 0 && C >= 0 && corners >= 1 && n_entries >= 0, "proj_scatter: bad sizes");
  if (M == 0 || C == 0) return VB200_OK;
  VB200_REQUIRE(x && seg_offsets && x_rows > 0 && (numerators != nullptr || (out && normalizer)),
                "proj_scatter: null pointer or empty input");
  const ScatterWorkspace lay = scatter_layout(M, n_entries, C);
  VB200_REQUIRE(workspace != nullptr && workspace_bytes >= lay.total,
                "proj_scatter: workspace of %zu bytes required (got %zu)", lay.total, workspace_bytes);
  int rc;
  if ((rc = check_rows(dtype, x, xs, C, "proj_scatter input")) != VB200_OK) return rc;
  if (numerators == nullptr && (rc = check_rows(dtype, out, os, C, "proj_scatter output")) != VB200_OK) return rc;
  VB200_REQUIRE(numerators == nullptr || (reinterpret_cast<uintptr_t>(numerators) & 15u) == 0,
                "proj_scatter: numerators must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* nchunk = reinterpret_cast<int32_t*>(ws + lay.nchunk);
  int32_t* chunk_base = reinterpret_cast<int32_t*>(ws + lay.chunk_base);
  float* partials = reinterpret_cast<float*>(ws + lay.partials);
  int32_t* ngroup = reinterpret_cast<int32_t*>(ws + lay.ngroup);
  int32_t* group_base = reinterpret_cast<int32_t*>(ws + lay.group_base);
  float* partials1 = reinterpret_cast<float*>(ws + lay.partials1);
  scatter_count_kernel<<<static_cast<unsigned>((M + 1 + 255) / 256), 256, 0, st>>>(
      seg_offsets, M, static_cast<int>(corners), nchunk, ngroup);
  VB200_CHECK_LAUNCH("scatter_count_kernel");
  size_t scan_bytes = lay.scan_bytes;
  VB200_CHECK_CUDA(cub::DeviceScan::ExclusiveSum(ws + lay.scan_tmp, scan_bytes, nchunk, chunk_base,
                                                 static_cast<int>(M + 1), st),
                   "cub::DeviceScan::ExclusiveSum");
  scan_bytes = lay.scan_bytes;
  VB200_CHECK_CUDA(cub::DeviceScan::ExclusiveSum(ws + lay.scan_tmp, scan_bytes, ngroup, group_base,
                                                 static_cast<int>(M + 1), st),
                   "cub::DeviceScan::ExclusiveSum");
  const bool tree = n_entries > kScatterChunk;  // some row may be long
  const long long chunk_warps = tree ? lay.bound : 0;
#define VB200_WORK(T)                                                                                    \
  scatter_work_kernel<T><<<row_blocks(chunk_warps + M), kWarpsPerBlock * 32, 0, st>>>(                    \
      static_cast<const T*>(x), x_rows, xs, keep, M, static_cast<int>(corners), seg_offsets, entry_src, entry_w, \
      normalizer, static_cast<T*>(out), os, static_cast<int>(C), chunk_base, partials, chunk_warps, numerators)
  if (dtype == VB200_F32) VB200_WORK(float);
  else if (dtype == VB200_BF16) VB200_WORK(__nv_bfloat16);
  else VB200_WORK(__half);
#undef VB200_WORK
  VB200_CHECK_LAUNCH("scatter_work_kernel");
  if (!tree) return VB200_OK;
  const int V = dtype == VB200_F32 ? 4 : 8;
  if (V == 8) {
    scatter_group_kernel<8><<<row_blocks(lay.bound1), kWarpsPerBlock * 32, 0, st>>>(
        M, chunk_base, group_base, partials, partials1, static_cast<int>(C));
  } else {
    scatter_group_kernel<4><<<row_blocks(lay.bound1), kWarpsPerBlock * 32, 0, st>>>(
        M, chunk_base, group_base, partials, partials1, static_cast<int>(C));
  }
  VB200_CHECK_LAUNCH("scatter_group_kernel");
#define VB200_FINISH(T)                                                                            \
  scatter_finish_kernel<T><<<row_blocks(M), kWarpsPerBlock * 32, 0, st>>>(                          \
      static_cast<const T*>(x), x_rows, xs, keep, M, normalizer, static_cast<T*>(out), os, static_cast<int>(C), \
      chunk_base, partials, group_base, partials1, numerators)
  if (dtype == VB200_F32) VB200_FINISH(float);
  else if (dtype == VB200_BF16) VB200_FINISH(__nv_bfloat16);
  else VB200_FINISH(__half);
#undef VB200_FINISH
  VB200_CHECK_LAUNCH("scatter_finish_kernel");
  return VB200_OK;
}

}  // namespace
}  // namespace vb200

extern "C" int vb200_proj_scatter(int dtype, const void* x, int64_t x_rows, int64_t xs, const int64_t* keep,
                                  int64_t M, int64_t corners, const int32_t* seg_offsets,
                                  const int32_t* entry_src, const float* entry_w,
                                  const float* normalizer, void* out, int64_t os, int64_t C,
                                  int64_t n_entries, void* workspace, size_t workspace_bytes, void* stream) {
  VB200_REQUIRE(out && normalizer, "proj_scatter: null pointer");
  return scatter_launch(dtype, x, x_rows, xs, keep, M, corners, seg_offsets, entry_src, entry_w, normalizer, out, os,
                        C, n_entries, workspace, workspace_bytes, nullptr, stream);
}

extern "C" int vb200_proj_scatter_numerators(int dtype, const void* x, int64_t x_rows, int64_t xs, int64_t M,
                                             int64_t corners, const int32_t* seg_offsets, const int32_t* entry_src,
                                             const float* entry_w, float* numerators, int64_t C, int64_t n_entries,
                                             void* workspace, size_t workspace_bytes, void* stream) {
  VB200_REQUIRE(numerators != nullptr, "proj_scatter_numerators: null pointer");
  return scatter_launch(dtype, x, x_rows, xs, nullptr, M, corners, seg_offsets, entry_src, entry_w, nullptr, nullptr,
                        0, C, n_entries, workspace, workspace_bytes, numerators, stream);
}

extern "C" int vb200_rank_reduce_rows(int dtype, const float* partials, int R, int64_t rows, int64_t C, const void* x,
                                      int64_t x_rows, int64_t xs, const int64_t* keep, const float* normalizer,
                                      void* out, int64_t os, void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "rank_reduce_rows: bad dtype %d",
                dtype);
  VB200_REQUIRE(R >= 1 && rows >= 0 && C >= 0, "rank_reduce_rows: bad sizes");
  if (rows == 0 || C == 0) return VB200_OK;
  VB200_REQUIRE(partials && normalizer && out && (keep == nullptr || (x && x_rows > 0)),
                "rank_reduce_rows: null pointer");
  VB200_REQUIRE(C % 8 == 0 && (reinterpret_cast<uintptr_t>(partials) & 15u) == 0,
                "rank_reduce_rows: C must be a multiple of 8 and partials 16-byte aligned");
  int rc;
  if (keep != nullptr && (rc = check_rows(dtype, x, xs, C, "rank_reduce_rows input")) != VB200_OK) return rc;
  if ((rc = check_rows(dtype, out, os, C, "rank_reduce_rows output")) != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define VB200_RR(T)                                                                                         \
  rank_reduce_rows_kernel<T><<<row_blocks(rows), kWarpsPerBlock * 32, 0, st>>>(                              \
      partials, R, rows, static_cast<int>(C), static_cast<const T*>(x), x_rows, xs, keep, normalizer,        \
      static_cast<T*>(out), os)
  if (dtype == VB200_F32) VB200_RR(float);
  else if (dtype == VB200_BF16) VB200_RR(__nv_bfloat16);
  else VB200_RR(__half);
#undef VB200_RR
  VB200_CHECK_LAUNCH("rank_reduce_rows_kernel");
  return VB200_OK;
}

extern "C" size_t vb200_plan_csr_workspace_size(int64_t S, int64_t corners, int64_t M) {
  if (S < 0 || corners < 1 || M < 0) return 0;
  return csr_layout(S, corners, M).total;
}

extern "C" int vb200_plan_csr_build(const int64_t* parent, const float* weights,
                                    const int64_t* src_rows, int64_t S, int64_t corners, int64_t M,
                                    int32_t* seg_offsets, int32_t* entry_src, float* entry_w,
                                    float* mass, float* log_mass, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  VB200_REQUIRE(S >= 0 && M >= 0 && corners >= 1 && corners <= 16, "plan_csr_build: bad sizes");
  VB200_REQUIRE(S * corners < (1ll << 30) && M * corners < (1ll << 30),
                "plan_csr_build: sizes exceed the int32 index range");
  VB200_REQUIRE(seg_offsets != nullptr, "plan_csr_build: seg_offsets must not be NULL");
  VB200_REQUIRE(S == 0 || (parent && weights && entry_src && entry_w), "plan_csr_build: null pointer");
  const CsrWorkspace lay = csr_layout(S, corners, M);
  VB200_REQUIRE(workspace != nullptr && workspace_bytes >= lay.total,
                "plan_csr_build: workspace of %zu bytes required (got %zu)", lay.total, workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* keys_in = reinterpret_cast<int32_t*>(ws + lay.keys_in);
  int32_t* keys_out = reinterpret_cast<int32_t*>(ws + lay.keys_out);
  int32_t* vals_in = reinterpret_cast<int32_t*>(ws + lay.vals_in);
  int32_t* vals_out = reinterpret_cast<int32_t*>(ws + lay.vals_out);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + lay.counts);
  const long long n = S * corners;
  const int nseg = static_cast<int>(M * corners + 1);
  const int32_t dropped = static_cast<int32_t>(M * corners);
  VB200_CHECK_CUDA(cudaMemsetAsync(counts, 0, static_cast<size_t>(nseg) * 4, st), "cudaMemsetAsync");
  if (n > 0) {
    csr_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(
        parent, n, static_cast<int>(corners), M, keys_in, vals_in, counts, dropped);
    VB200_CHECK_LAUNCH("csr_keys_kernel");
    int end_bit = 1;
    while ((1ll << end_bit) <= dropped) ++end_bit;
    size_t sort_bytes = lay.sort_bytes;
    VB200_CHECK_CUDA(cub::DeviceRadixSort::SortPairs(ws + lay.sort_tmp, sort_bytes, keys_in, keys_out,
                                                     vals_in, vals_out, static_cast<int>(n), 0,
                                                     end_bit, st),
                     "cub::DeviceRadixSort::SortPairs");
  }
  size_t scan_bytes = lay.scan_bytes;
  VB200_CHECK_CUDA(cub::DeviceScan::ExclusiveSum(ws + lay.scan_tmp, scan_bytes, counts, seg_offsets,
                                                 nseg, st),
                   "cub::DeviceScan::ExclusiveSum");
  if (n > 0) {
    csr_entries_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(
        keys_out, vals_out, n, static_cast<int>(corners), weights, src_rows, entry_src, entry_w, dropped);
    VB200_CHECK_LAUNCH("csr_entries_kernel");
  }
  if (M > 0 && (mass || log_mass)) {
    csr_mass_kernel<<<row_blocks(M), kWarpsPerBlock * 32, 0, st>>>(
        seg_offsets, entry_w, M, static_cast<int>(corners), mass, log_mass);
    VB200_CHECK_LAUNCH("csr_mass_kernel");
  }
  return VB200_OK;
}

extern "C" int vb200_plan_csr_build_grouped(const int64_t* parent, const float* weights, const int64_t* src_rows,
                                            int64_t S, int64_t corners, int64_t M, const int64_t* q_begin,
                                            const int64_t* b_begin, int groups, int max_group_rows,
                                            int max_group_sources, int32_t* seg_offsets, int32_t* entry_src,
                                            float* entry_w, float* mass, float* log_mass, void* stream) {
  VB200_REQUIRE(S >= 0 && M >= 0 && corners >= 1 && corners <= 16 && groups >= 1, "plan_csr_build_grouped: bad sizes");
  VB200_REQUIRE(S * corners < (1ll << 30) && M * corners < (1ll << 30),
                "plan_csr_build_grouped: sizes exceed the int32 index range");
  VB200_REQUIRE(max_group_rows >= 0 && static_cast<long long>(max_group_rows) * corners <= kCsrGroupMaxSegments &&
                    max_group_sources >= 0 && static_cast<long long>(max_group_sources) * corners <= kCsrGroupMaxEntries,
                "plan_csr_build_grouped: a group of %d rows / %d sources x %lld corners exceeds %d segments or %d "
                "entries; use vb200_plan_csr_build",
                max_group_rows, max_group_sources, (long long)corners, kCsrGroupMaxSegments, kCsrGroupMaxEntries);
  VB200_REQUIRE(seg_offsets && q_begin && b_begin && (S == 0 || (parent && weights && entry_src && entry_w)),
                "plan_csr_build_grouped: null pointer");
  // parts per group: enough CTAs to spread the build over the GPU (each part owns a range of the
  // group's merged rows and scans all of its pairs)
  int sms = 0, dev = 0;
  VB200_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  VB200_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
  const int parts = std::max(1, std::min({kCsrMaxParts, sms / groups, std::max(1, max_group_rows)}));
  const int per = (max_group_rows + parts - 1) / parts;
  const int max_segments = static_cast<int>(std::max<long long>(1, static_cast<long long>(per) * corners));
  const int max_entries = static_cast<int>(std::max<long long>(2, (static_cast<long long>(max_group_sources) * corners + 1) & ~1ll));
  const size_t smem = static_cast<size_t>(max_segments) * 4 + static_cast<size_t>(max_entries) * 10;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  VB200_CHECK_CUDA(cudaFuncSetAttribute(csr_grouped_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)),
                   "cudaFuncSetAttribute");
  csr_grouped_kernel<<<groups * parts, kCsrGroupThreads, smem, st>>>(
      parent, weights, src_rows, static_cast<int>(corners), M, q_begin, b_begin, groups, parts, max_segments,
      max_entries, seg_offsets, entry_src, entry_w);
  VB200_CHECK_LAUNCH("csr_grouped_kernel");
  if (M > 0 && (mass || log_mass)) {
    csr_mass_kernel<<<row_blocks(M), kWarpsPerBlock * 32, 0, st>>>(seg_offsets, entry_w, M, static_cast<int>(corners),
                                                                   mass, log_mass);
    VB200_CHECK_LAUNCH("csr_mass_kernel");
  }
  return VB200_OK;
}

extern "C" int vb200_row_normalize_bf16(int dtype, const void* x, int64_t x_rows, int64_t xs, const int64_t* rows,
                                        int64_t R, int64_t C, float eps, void* out, int64_t os,
                                        void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "row_normalize: bad dtype %d", dtype);
  VB200_REQUIRE(R >= 0 && C >= 0, "row_normalize: negative size");
  if (R == 0 || C == 0) return VB200_OK;
  VB200_REQUIRE(x && out, "row_normalize: null pointer");
  int rc;
  if ((rc = check_rows(dtype, x, xs, C, "row_normalize input")) != VB200_OK) return rc;
  if ((rc = check_rows(VB200_BF16, out, os, C, "row_normalize output")) != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define VB200_NORM(T)                                                                  \
  row_normalize_kernel<T><<<row_blocks(R), kWarpsPerBlock * 32, 0, st>>>(              \
      static_cast<const T*>(x), x_rows, xs, rows, R, static_cast<int>(C), eps,         \
      static_cast<__nv_bfloat16*>(out), os)
  if (dtype == VB200_F32) VB200_NORM(float);
  else if (dtype == VB200_BF16) VB200_NORM(__nv_bfloat16);
  else VB200_NORM(__half);
#undef VB200_NORM
  VB200_CHECK_LAUNCH("row_normalize_kernel");
  return VB200_OK;
}

extern "C" size_t vb200_compact_qkv_workspace_size(int64_t rows, int64_t C) {
  if (rows < 0 || C < 0) return 0;
  return align_up(static_cast<size_t>(rows > 0 ? rows : 1) * static_cast<size_t>(2 * C / 64) * sizeof(float2), 256);
}

namespace {
int compact_qkv_impl(int dtype, const void* qkv, int64_t rows, int64_t xs, int64_t C, const float* ln_weight,
                     const float* ln_bias, float eps, const int64_t* keep, int64_t M, int64_t corners,
                     const int32_t* seg_offsets, const int32_t* entry_src, const float* entry_w,
                     const float* normalizer, int pool_mask, void* out, int64_t os, void* workspace,
                     size_t workspace_bytes, const KvPeers& peers, void* stream) {
  VB200_REQUIRE(dtype == VB200_BF16 || dtype == VB200_F16, "compact_qkv: dtype must be bf16 or fp16 (got %d)", dtype);
  VB200_REQUIRE(C > 0 && C % 256 == 0, "compact_qkv: channels per tensor must be a multiple of 256 (got %lld)",
                (long long)C);
  VB200_REQUIRE(M >= 0 && rows > 0 && corners >= 1, "compact_qkv: bad sizes");
  VB200_REQUIRE((ln_weight == nullptr) == (ln_bias == nullptr), "compact_qkv: pass both LayerNorm tensors or neither");
  if (M == 0) return VB200_OK;
  VB200_REQUIRE(qkv && keep && out && normalizer && (pool_mask == 0 || seg_offsets),
                "compact_qkv: null pointer");
  int rc;
  if ((rc = check_rows(dtype, qkv, xs, 3 * C, "compact_qkv input")) != VB200_OK) return rc;
  if ((rc = check_rows(dtype, out, os, 3 * C, "compact_qkv output")) != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  VB200_REQUIRE((pool_mask & ~(7 | VB200_STATS_READY)) == 0, "compact_qkv: bad pool_mask %d", pool_mask);
  const bool stats_ready = (pool_mask & VB200_STATS_READY) != 0;
  pool_mask &= 7;
  float2* stats = nullptr;
  if (ln_weight != nullptr) {
    const size_t need = vb200_compact_qkv_workspace_size(rows, C);
    VB200_REQUIRE(workspace != nullptr && workspace_bytes >= need,
                  "compact_qkv: workspace of %zu bytes required (got %zu)", need, workspace_bytes);
    stats = static_cast<float2*>(workspace);
  }
  if (ln_weight != nullptr && !stats_ready) {
#define VB200_STATS(T)                                                                            \
  head_stats_kernel<T><<<row_blocks(rows), kWarpsPerBlock * 32, 0, st>>>(static_cast<const T*>(qkv), rows, \
                                                                       xs, static_cast<int>(C), eps, stats)
    if (dtype == VB200_BF16) VB200_STATS(__nv_bfloat16);
    else VB200_STATS(__half);
#undef VB200_STATS
    VB200_CHECK_LAUNCH("head_stats_kernel");
  }
  if (C <= 1024) {
    // staged path: one producer warp + 3C/kCh consumer threads per CTA; four CTAs per SM with
    // 16-channel threads, two with 8
    const int ch = (3 * C / 16) % 32 == 0 ? 16 : 8;
    const int threads = static_cast<int>(3 * C / ch) + 32;
    const size_t smem = kStageHeaderBytes +
                        static_cast<size_t>(kStageSlots) * (3 * C * 2 + (ln_weight ? 2 * C / 64 * sizeof(float2) : 0));
    int dev = 0, sms = 0;
    VB200_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    VB200_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
    const long long per_sm = ch == 16 ? 4 : 2;
    const unsigned grid = static_cast<unsigned>(M < per_sm * sms ? M : per_sm * sms);
#define VB200_CQKV_STAGED(T, CH)                                                                               \
  VB200_CHECK_CUDA(cudaFuncSetAttribute(compact_qkv_staged_kernel<T, CH>,                                      \
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),  \
                   "cudaFuncSetAttribute");                                                                    \
  compact_qkv_staged_kernel<T, CH><<<grid, threads, smem, st>>>(                                               \
      static_cast<const T*>(qkv), rows, xs, static_cast<int>(C), ln_weight, ln_bias, stats, keep, M,           \
      static_cast<int>(corners), seg_offsets, entry_src, entry_w, normalizer, pool_mask, static_cast<T*>(out), \
      os, peers)
    if (dtype == VB200_BF16) {
      if (ch == 16) {
        VB200_CQKV_STAGED(__nv_bfloat16, 16);
      } else {
        VB200_CQKV_STAGED(__nv_bfloat16, 8);
      }
    } else {
      if (ch == 16) {
        VB200_CQKV_STAGED(__half, 16);
      } else {
        VB200_CQKV_STAGED(__half, 8);
      }
    }
#undef VB200_CQKV_STAGED
    VB200_CHECK_LAUNCH("compact_qkv_staged_kernel");
    return VB200_OK;
  }
  VB200_REQUIRE(peers.world == 0, "compact_qkv_peer: peer destinations need C <= 1024");
#define VB200_CQKV(T)                                                                                     \
  compact_qkv_kernel<T><<<row_blocks(M * 3 * (C / 256)), kWarpsPerBlock * 32, 0, st>>>(                   \
      static_cast<const T*>(qkv), rows, xs, static_cast<int>(C), ln_weight, ln_bias, stats, keep, M,      \
      static_cast<int>(corners), seg_offsets, entry_src, entry_w, normalizer, pool_mask, static_cast<T*>(out), os)
  if (dtype == VB200_BF16) VB200_CQKV(__nv_bfloat16);
  else VB200_CQKV(__half);
#undef VB200_CQKV
  VB200_CHECK_LAUNCH("compact_qkv_kernel");
  return VB200_OK;
}
}  // namespace

extern "C" int vb200_qkv_head_stats(int dtype, const void* qkv, int64_t rows, int64_t xs, int64_t C, float eps,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  VB200_REQUIRE(dtype == VB200_BF16 || dtype == VB200_F16, "qkv_head_stats: dtype must be bf16 or fp16 (got %d)",
                dtype);
  VB200_REQUIRE(rows >= 0 && C > 0 && C % 256 == 0, "qkv_head_stats: bad sizes");
  if (rows == 0) return VB200_OK;
  VB200_REQUIRE(qkv != nullptr, "qkv_head_stats: null pointer");
  const size_t need = vb200_compact_qkv_workspace_size(rows, C);
  VB200_REQUIRE(workspace != nullptr && workspace_bytes >= need,
                "qkv_head_stats: workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  int rc;
  if ((rc = check_rows(dtype, qkv, xs, 3 * C, "qkv_head_stats input")) != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float2* stats = static_cast<float2*>(workspace);
  if (dtype == VB200_BF16)
    head_stats_kernel<__nv_bfloat16><<<row_blocks(rows), kWarpsPerBlock * 32, 0, st>>>(
        static_cast<const __nv_bfloat16*>(qkv), rows, xs, static_cast<int>(C), eps, stats);
  else
    head_stats_kernel<__half><<<row_blocks(rows), kWarpsPerBlock * 32, 0, st>>>(static_cast<const __half*>(qkv), rows,
                                                                                  xs, static_cast<int>(C), eps, stats);
  VB200_CHECK_LAUNCH("head_stats_kernel");
  return VB200_OK;
}

extern "C" int vb200_compact_qkv(int dtype, const void* qkv, int64_t rows, int64_t xs, int64_t C,
                                 const float* ln_weight, const float* ln_bias, float eps, const int64_t* keep,
                                 int64_t M, int64_t corners, const int32_t* seg_offsets,
                                 const int32_t* entry_src, const float* entry_w, const float* normalizer,
                                 int pool_mask, void* out, int64_t os, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  KvPeers none{};
  return compact_qkv_impl(dtype, qkv, rows, xs, C, ln_weight, ln_bias, eps, keep, M, corners, seg_offsets, entry_src,
                          entry_w, normalizer, pool_mask, out, os, workspace, workspace_bytes, none, stream);
}

extern "C" int vb200_compact_qkv_peer(int dtype, const void* qkv, int64_t rows, int64_t xs, int64_t C,
                                      const float* ln_weight, const float* ln_bias, float eps, const int64_t* keep,
                                      int64_t M, int64_t corners, const int32_t* seg_offsets,
                                      const int32_t* entry_src, const float* entry_w, const float* normalizer,
                                      int pool_mask, void* out, int64_t os, const uint64_t* kv_dst_ptrs, int world,
                                      int multicast, int64_t kv_row0, int64_t kv_row_stride, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  VB200_REQUIRE(world >= 1 && world <= kMaxKvPeers, "compact_qkv_peer: world must be in [1, %d] (got %d)",
                kMaxKvPeers, world);
  VB200_REQUIRE(kv_dst_ptrs != nullptr && kv_row0 >= 0 && kv_row_stride >= 2 * C && kv_row_stride % 8 == 0,
                "compact_qkv_peer: bad destination layout (row stride %lld elements for C=%lld)",
                (long long)kv_row_stride, (long long)C);
  KvPeers peers{};
  const int n_dst = multicast ? 1 : world;
  for (int r = 0; r < n_dst; ++r) {
    VB200_REQUIRE(kv_dst_ptrs[r] != 0 && (kv_dst_ptrs[r] & 15u) == 0,
                  "compact_qkv_peer: destination of rank %d is null or not 16-byte aligned", r);
    peers.dst[r] = kv_dst_ptrs[r];
  }
  peers.world = world;
  peers.multicast = multicast ? 1 : 0;
  peers.row0 = kv_row0;
  peers.stride = kv_row_stride;
  return compact_qkv_impl(dtype, qkv, rows, xs, C, ln_weight, ln_bias, eps, keep, M, corners, seg_offsets, entry_src,
                          entry_w, normalizer, pool_mask, out, os, workspace, workspace_bytes, peers, stream);
}

extern "C" int vb200_head_layernorm(int dtype, const void* x, int64_t rows, int64_t xs, int64_t C,
                                    const float* weight, const float* bias, float eps, void* out, int64_t os,
                                    void* stream) {
  VB200_REQUIRE(dtype == VB200_BF16 || dtype == VB200_F16, "head_layernorm: dtype must be bf16 or fp16");
  VB200_REQUIRE(C > 0 && C % 64 == 0 && rows >= 0, "head_layernorm: channels must be a multiple of 64");
  if (rows == 0) return VB200_OK;
  VB200_REQUIRE(x && out && weight && bias, "head_layernorm: null pointer");
  VB200_REQUIRE(C % 256 == 0, "head_layernorm: channels must be a multiple of 256");
  int rc;
  if ((rc = check_rows(dtype, x, xs, C, "head_layernorm input")) != VB200_OK) return rc;
  if ((rc = check_rows(dtype, out, os, C, "head_layernorm output")) != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == VB200_BF16)
    head_layernorm_kernel<__nv_bfloat16><<<row_blocks(rows), kWarpsPerBlock * 32, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), rows, xs, static_cast<int>(C), weight, bias, eps,
        static_cast<__nv_bfloat16*>(out), os);
  else
    head_layernorm_kernel<__half><<<row_blocks(rows), kWarpsPerBlock * 32, 0, st>>>(
        static_cast<const __half*>(x), rows, xs, static_cast<int>(C), weight, bias, eps, static_cast<__half*>(out), os);
  VB200_CHECK_LAUNCH("head_layernorm_kernel");
  return VB200_OK;
}
