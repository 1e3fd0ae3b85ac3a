// Device-side plan construction for the merge step (no host synchronisation):
//
//   merge_assign  ranking + keep / inverse maps of build_fastvggt_plan
//                 (vggt_omega/models/token_merging.py:1112-1121): sources are ordered by their
//                 best score (stable, descending), the first `removed` are merged into their
//                 argmax destination, the survivors are renumbered in token order.
//   support_fit   Gram / right-hand side of each source's four supports
//                 (vggt_omega/models/sparse_convex.py:2314-2316: gram = S S^T, rhs = S x) and,
//                 optionally, the four-support projected-gradient solve
//                 (sparse_convex_kernels.py:214-280) fused in the same kernel.
#include <cub/cub.cuh>

#include "common.cuh"
#include "host_common.h"

namespace vb200 {
namespace {

static __device__ unsigned g_plan_err;

__global__ void iota_kernel(int32_t* v, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) v[i] = static_cast<int32_t>(i);
}

// flags[n] = 1 for kept tokens; remap[n] = original id of the destination a removed token
// merges into.
__global__ void mark_removed_kernel(const int32_t* __restrict__ order, const int64_t* __restrict__ target,
                                    const int64_t* __restrict__ source_idx, const int64_t* __restrict__ dest_idx,
                                    long long removed, long long Dn, long long total,
                                    int32_t* __restrict__ kept_flag, int64_t* __restrict__ remap) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= removed) return;
  const int32_t s = order[i];
  const int64_t n = source_idx[s];
  const int64_t t = target[s];
  if (n < 0 || n >= total || t < 0 || t >= Dn || dest_idx[t] < 0 || dest_idx[t] >= total) {
    atomicOr(&g_plan_err, kErrBadArgument);
    return;
  }
  kept_flag[n] = 0;
  remap[n] = dest_idx[t];
}

__global__ void fill_ones_kernel(int32_t* v, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) v[i] = 1;
}

__global__ void keep_inverse_kernel(const int32_t* __restrict__ kept_flag, const int32_t* __restrict__ compact,
                                    const int64_t* __restrict__ remap, long long total, long long keep_len,
                                    int64_t* __restrict__ keep, int64_t* __restrict__ inverse) {
  const long long n = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (n >= total) return;
  if (kept_flag[n]) {
    if (compact[n] >= keep_len) {  // duplicate source ids removed fewer tokens than declared
      atomicOr(&g_plan_err, kErrBadArgument);
      inverse[n] = -1;
      return;
    }
    keep[compact[n]] = n;
    inverse[n] = compact[n];
  } else {
    const int64_t t = remap[n];
    inverse[n] = kept_flag[t] ? compact[t] : -1;  // a destination is never removed
  }
}

struct AssignWorkspace {
  size_t keys_out, vals_in, vals_out, flags, compact, remap, sort_tmp, scan_tmp, total;
  size_t sort_bytes, scan_bytes;
};

AssignWorkspace assign_layout(int64_t S, int64_t total) {
  const int s = static_cast<int>(S > 0 ? S : 1);
  const int t = static_cast<int>(total > 0 ? total : 1);
  size_t sort_bytes = 0, scan_bytes = 0;
  cub::DeviceRadixSort::SortPairsDescending(nullptr, sort_bytes, static_cast<float*>(nullptr),
                                            static_cast<float*>(nullptr), static_cast<int32_t*>(nullptr),
                                            static_cast<int32_t*>(nullptr), s);
  cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<int32_t*>(nullptr),
                                static_cast<int32_t*>(nullptr), t);
  AssignWorkspace w{};
  size_t off = 0;
  auto take = [&](size_t b) { const size_t o = off; off = align_up(off + b, 256); return o; };
  w.keys_out = take(static_cast<size_t>(s) * 4);
  w.vals_in = take(static_cast<size_t>(s) * 4);
  w.vals_out = take(static_cast<size_t>(s) * 4);
  w.flags = take(static_cast<size_t>(t) * 4);
  w.compact = take(static_cast<size_t>(t) * 4);
  w.remap = take(static_cast<size_t>(t) * 8);
  w.sort_tmp = take(sort_bytes);
  w.scan_tmp = take(scan_bytes);
  w.total = off;
  w.sort_bytes = sort_bytes;
  w.scan_bytes = scan_bytes;
  return w;
}

// One warp per source: the 4x4 Gram of its supports and the 4 support-source products,
// accumulated in fp32 over the channels (lane-strided, then a fixed butterfly).  With steps > 0
// the block's kFitWarps systems go through shared memory to warp 0, whose lanes run the
// projected-gradient solves side by side (one source per lane) instead of one lane per warp.
constexpr int kFitWarps = 8;
__constant__ int kFitPairI[10] = {0, 0, 0, 0, 1, 1, 1, 2, 2, 3};  // Gram entry (i, j), i <= j, row-major
__constant__ int kFitPairJ[10] = {0, 1, 2, 3, 1, 2, 3, 2, 3, 3};

// A 32-bit word of two 16-bit values as an fp32 pair (low half first).
template <typename T>
__device__ __forceinline__ uint64_t widen2(uint32_t w);
template <>
__device__ __forceinline__ uint64_t widen2<__nv_bfloat16>(uint32_t w) {
  return pk2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ uint64_t widen2<__half>(uint32_t w) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
  return pk2(f.x, f.y);
}
template <>
__device__ __forceinline__ uint64_t widen2<float>(uint32_t w) {
  return pk2(__uint_as_float(w), 0.f);  // unused: fp32 features take the scalar path
}
template <typename T>
__global__ void __launch_bounds__(kFitWarps * 32)
    support_fit_kernel(const T* __restrict__ feat, long long rows, long long fs,
                                   const int64_t* __restrict__ src_rows,
                                   const int64_t* __restrict__ parent_rows, long long S, int D,
                                   float* __restrict__ gram, float* __restrict__ rhs,
                                   float* __restrict__ alpha, int steps) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float sys[kFitWarps][20];  // G (16) and rhs (4) of each warp's source
  const int warp = threadIdx.x >> 5;
  const long long s = static_cast<long long>(blockIdx.x) * kFitWarps + warp;
  const int lane = threadIdx.x & 31;
  if (s < S) {
    long long r[5];
    r[0] = src_rows ? src_rows[s] : s;
#pragma unroll
    for (int c = 0; c < 4; ++c) r[c + 1] = parent_rows[s * 4 + c];
    bool bad = false;
#pragma unroll
    for (int c = 0; c < 5; ++c) {
      if (r[c] < 0 || r[c] >= rows) { bad = true; r[c] = 0; }
    }
    if (bad && lane == 0) atomicOr(&g_plan_err, kErrBadArgument);
    // products: g[i][j] for i <= j (10) + rhs[i] (4), accumulated per lane in fp32
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
    if constexpr (sizeof(T) == 2) {
      // 16-bit features: each 32-bit word is widened to an fp32 pair and the 14 products are
      // packed FMAs on (even, odd) channel pairs; the two halves are added at the end
      uint64_t acc2[14];
#pragma unroll
      for (int i = 0; i < 14; ++i) acc2[i] = 0ull;
      for (int v0 = lane * V; v0 < D; v0 += 32 * V) {
        uint4 raw[5];
#pragma unroll
        for (int c = 0; c < 5; ++c) raw[c] = __ldg(reinterpret_cast<const uint4*>(feat + r[c] * fs + v0));
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          uint64_t x[5];
#pragma unroll
          for (int c = 0; c < 5; ++c) x[c] = widen2<T>(reinterpret_cast<const uint32_t*>(&raw[c])[h]);
          int idx = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = i; j < 4; ++j) {
              acc2[idx] = ffma2(x[i + 1], x[j + 1], acc2[idx]);
              ++idx;
            }
#pragma unroll
          for (int i = 0; i < 4; ++i) acc2[10 + i] = ffma2(x[i + 1], x[0], acc2[10 + i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 14; ++i) {
        float lo, hi;
        upk2(acc2[i], lo, hi);
        acc[i] = lo + hi;
      }
    } else {
      for (int v0 = lane * V; v0 < D; v0 += 32 * V) {
        float x[5][V];
#pragma unroll
        for (int c = 0; c < 5; ++c) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(feat + r[c] * fs + v0));
          const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int q = 0; q < V; ++q) x[c][q] = to_f32<T>(e[q]);
        }
#pragma unroll
        for (int q = 0; q < V; ++q) {
          int idx = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = i; j < 4; ++j) {
              acc[idx] = fmaf(x[i + 1][q], x[j + 1][q], acc[idx]);
              ++idx;
            }
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[10 + i] = fmaf(x[i + 1][q], x[0][q], acc[10 + i]);
        }
      }
    }
    // Transposing warp reduction of the 16 (14 used) values: each xor step halves the values a
    // lane holds while summing over the partner lane, so lane L ends with the full sum of
    // value (L >> 1) in 16 shuffles instead of 14 x 5.
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = acc[i];
#pragma unroll
    for (int n = 8; n >= 1; n >>= 1) {
      const bool upper = (lane & (2 * n)) != 0;
#pragma unroll
      for (int i = 0; i < n; ++i) {
        const float send = upper ? v[i] : v[i + n];
        const float keep = upper ? v[i + n] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2 * n);
      }
    }
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    const int vidx = lane >> 1;  // the value this lane now holds
    if ((lane & 1) == 0 && vidx < 14) {
      if (vidx < 10) {
        sys[warp][kFitPairI[vidx] * 4 + kFitPairJ[vidx]] = v[0];
        sys[warp][kFitPairJ[vidx] * 4 + kFitPairI[vidx]] = v[0];
      } else {
        sys[warp][16 + vidx - 10] = v[0];
      }
    }
    __syncwarp();
    if (lane == 0) {
      if (gram) {
#pragma unroll
        for (int i = 0; i < 16; ++i) gram[s * 16 + i] = sys[warp][i];
      }
      if (rhs) {
#pragma unroll
        for (int i = 0; i < 4; ++i) rhs[s * 4 + i] = sys[warp][16 + i];
      }
    }
  }  // s < S
  if (alpha == nullptr) return;
  __syncthreads();
  const long long sl = static_cast<long long>(blockIdx.x) * kFitWarps + lane;  // warp 0, lane = source
  if (warp != 0 || lane >= kFitWarps || sl >= S) return;
  float G[16], R4[4];
#pragma unroll
  for (int i = 0; i < 16; ++i) G[i] = sys[lane][i];
#pragma unroll
  for (int i = 0; i < 4; ++i) R4[i] = sys[lane][16 + i];
  // projected gradient on the simplex (same iteration as the standalone solver)
  const float n0 = fabsf(G[0]) + fabsf(G[1]) + fabsf(G[2]) + fabsf(G[3]);
  const float n1 = fabsf(G[4]) + fabsf(G[5]) + fabsf(G[6]) + fabsf(G[7]);
  const float n2 = fabsf(G[8]) + fabsf(G[9]) + fabsf(G[10]) + fabsf(G[11]);
  const float n3 = fabsf(G[12]) + fabsf(G[13]) + fabsf(G[14]) + fabsf(G[15]);
  const float step = 0.95f / fmaxf(fmaxf(fmaxf(n0, n1), fmaxf(n2, n3)), 1.0e-4f);
  float a0 = 1.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  for (int it = 0; it < steps; ++it) {
    const float p0 = a0 - step * (G[0] * a0 + G[1] * a1 + G[2] * a2 + G[3] * a3 - R4[0]);
    const float p1 = a1 - step * (G[4] * a0 + G[5] * a1 + G[6] * a2 + G[7] * a3 - R4[1]);
    const float p2 = a2 - step * (G[8] * a0 + G[9] * a1 + G[10] * a2 + G[11] * a3 - R4[2]);
    const float p3 = a3 - step * (G[12] * a0 + G[13] * a1 + G[14] * a2 + G[15] * a3 - R4[3]);
    float s0 = fmaxf(p0, p1), s1 = fminf(p0, p1), s2 = fmaxf(p2, p3), s3 = fminf(p2, p3), t;
    t = fmaxf(s0, s2); s2 = fminf(s0, s2); s0 = t;
    t = fmaxf(s1, s3); s3 = fminf(s1, s3); s1 = t;
    t = fmaxf(s1, s2); s2 = fminf(s1, s2); s1 = t;
    float theta = s0 - 1.f;
    const float th2 = (s0 + s1 - 1.f) * 0.5f;
    theta = s1 > th2 ? th2 : theta;
    const float th3 = (s0 + s1 + s2 - 1.f) / 3.f;
    theta = s2 > th3 ? th3 : theta;
    const float th4 = (s0 + s1 + s2 + s3 - 1.f) * 0.25f;
    theta = s3 > th4 ? th4 : theta;
    a0 = fmaxf(p0 - theta, 0.f);
    a1 = fmaxf(p1 - theta, 0.f);
    a2 = fmaxf(p2 - theta, 0.f);
    a3 = fmaxf(p3 - theta, 0.f);
  }
  alpha[sl * 4 + 0] = a0;
  alpha[sl * 4 + 1] = a1;
  alpha[sl * 4 + 2] = a2;
  alpha[sl * 4 + 3] = a3;
}

// 16 channels of a feature row as fp32 (two 16-byte loads for 16-bit types, four for fp32).
template <typename T>
__device__ __forceinline__ void load16(const T* __restrict__ p, float (&v)[16]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(p) + h);
      v[4 * h] = f.x; v[4 * h + 1] = f.y; v[4 * h + 2] = f.z; v[4 * h + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p) + h);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) v[8 * h + q] = to_f32<T>(e[q]);
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Certificate of a four-support convex fit (the reference's solve epilogue,
// sparse_convex.py:575-583 and :316-319): reconstruction r = sum_c alpha_c * support_c (fp32
// products added in support order), cosine = <x, r> / (max(|x|, 1e-8) max(|r|, 1e-8)),
// residual = |x - r|, reconstruction norm = |r|.  One warp per source, 16 channels per lane
// per pass, fp32 sums reduced across the warp.
template <typename T>
__global__ void __launch_bounds__(kFitWarps * 32)
    support_certificate_kernel(const T* __restrict__ feat, long long rows, long long fs,
                               const int64_t* __restrict__ src_rows, const int64_t* __restrict__ parent_rows,
                               const float* __restrict__ alpha, long long S, int D, float* __restrict__ cosine,
                               float* __restrict__ residual, float* __restrict__ recon_norm) {
  const long long s = static_cast<long long>(blockIdx.x) * kFitWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (s >= S) return;
  long long r[5];
  r[0] = src_rows ? src_rows[s] : s;
#pragma unroll
  for (int c = 0; c < 4; ++c) r[c + 1] = parent_rows[s * 4 + c];
  bool bad = false;
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    if (r[c] < 0 || r[c] >= rows) { bad = true; r[c] = 0; }
  }
  if (bad && lane == 0) atomicOr(&g_plan_err, kErrBadArgument);
  float a[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) a[c] = alpha[s * 4 + c];
  float xr = 0.f, xx = 0.f, rr = 0.f, dd = 0.f;
  for (int d0 = lane * 16; d0 < D; d0 += 32 * 16) {
    float x[16], rc[16], t[16];
    load16<T>(feat + r[0] * fs + d0, x);
#pragma unroll
    for (int q = 0; q < 16; ++q) rc[q] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      load16<T>(feat + r[c + 1] * fs + d0, t);
#pragma unroll
      for (int q = 0; q < 16; ++q) rc[q] = __fadd_rn(rc[q], __fmul_rn(a[c], t[q]));
    }
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      xr = fmaf(x[q], rc[q], xr);
      xx = fmaf(x[q], x[q], xx);
      rr = fmaf(rc[q], rc[q], rr);
      const float e = x[q] - rc[q];
      dd = fmaf(e, e, dd);
    }
  }
  xr = warp_sum(xr);
  xx = warp_sum(xx);
  rr = warp_sum(rr);
  dd = warp_sum(dd);
  if (lane == 0) {
    const float nx = sqrtf(xx), nr = sqrtf(rr);
    cosine[s] = xr / (fmaxf(nx, 1e-8f) * fmaxf(nr, 1e-8f));
    residual[s] = sqrtf(dd);
    recon_norm[s] = nr;
  }
}

// For each query row, the largest fp32 dot product with its targets (targets [Q, T], -1 =
// none; a query with no target gets -inf): the top-1 cosine that prunes redundant uniform
// anchors in the protected skeleton (sparse_convex.py:1404-1418).  One warp per query.
template <typename T>
__global__ void __launch_bounds__(kFitWarps * 32)
    row_max_dot_kernel(const T* __restrict__ feat, long long rows, long long fs, const int64_t* __restrict__ query,
                       const int64_t* __restrict__ targets, int n_targets, long long Q, int D,
                       float* __restrict__ out) {
  const long long q = static_cast<long long>(blockIdx.x) * kFitWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= Q) return;
  long long qr = query[q];
  if (qr < 0 || qr >= rows) {
    if (lane == 0) atomicOr(&g_plan_err, kErrBadArgument);
    qr = 0;
  }
  float best = -INFINITY;
  for (int t = 0; t < n_targets; ++t) {
    const long long tr = targets[q * n_targets + t];
    if (tr < 0) continue;  // uniform across the warp
    if (tr >= rows) {
      if (lane == 0) atomicOr(&g_plan_err, kErrBadArgument);
      continue;
    }
    float acc = 0.f;
    for (int d0 = lane * 16; d0 < D; d0 += 32 * 16) {
      float x[16], y[16];
      load16<T>(feat + qr * fs + d0, x);
      load16<T>(feat + tr * fs + d0, y);
#pragma unroll
      for (int i = 0; i < 16; ++i) acc = fmaf(x[i], y[i], acc);
    }
    best = fmaxf(best, warp_sum(acc));
  }
  if (lane == 0) out[q] = best;
}

// The Pareto-guarded geometry route's selection (sparse_convex.py:502-531, :263-306), one
// thread per source: from the row's top-k feature shortlist (bf16 scores, best first, -1 for
// empty slots) the joint value score - w * sum_d (g_s - g_c)^2 (fp32, squares added in order
// d = 0..3, no contraction), its top-4 positions (ties to the lower position), reordered by
// feature score (insertion sort, equal scores keep the joint order).  feature_ids = the first
// four shortlist ids; changed = the two id lists differ anywhere.
__global__ void geometry_shortlist_kernel(const float* __restrict__ values, const int64_t* __restrict__ indices,
                                          long long S, int k, const float* __restrict__ query_geo,
                                          const float* __restrict__ basis_geo, long long Nb, float weight,
                                          int64_t* __restrict__ feature_ids, int64_t* __restrict__ joint_ids,
                                          int32_t* __restrict__ changed) {
  const long long s = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (s >= S) return;
  float v[16], joint[16];
  int64_t id[16];
  const float4 gs = *reinterpret_cast<const float4*>(query_geo + s * 4);
  for (int c = 0; c < k; ++c) {
    v[c] = values[s * k + c];
    id[c] = indices[s * k + c];
    joint[c] = -INFINITY;
    if (id[c] < 0) continue;
    if (id[c] >= Nb) {
      atomicOr(&g_plan_err, kErrBadArgument);
      id[c] = -1;
      continue;
    }
    const float4 gc = *reinterpret_cast<const float4*>(basis_geo + id[c] * 4);
    const float d0 = __fsub_rn(gs.x, gc.x), d1 = __fsub_rn(gs.y, gc.y);
    const float d2 = __fsub_rn(gs.z, gc.z), d3 = __fsub_rn(gs.w, gc.w);
    float dist = __fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1));
    dist = __fadd_rn(dist, __fmul_rn(d2, d2));
    dist = __fadd_rn(dist, __fmul_rn(d3, d3));
    joint[c] = __fsub_rn(v[c], __fmul_rn(weight, dist));
  }
  int pos[4];
  unsigned taken = 0u;
  for (int j = 0; j < 4; ++j) {
    int best = -1;
    for (int c = 0; c < k; ++c) {
      if (taken & (1u << c)) continue;
      if (best < 0 || joint[c] > joint[best]) best = c;
    }
    pos[j] = best;
    taken |= 1u << best;
  }
  for (int j = 1; j < 4; ++j) {  // stable descending by feature score
    const int p = pos[j];
    int i = j - 1;
    while (i >= 0 && v[pos[i]] < v[p]) {
      pos[i + 1] = pos[i];
      --i;
    }
    pos[i + 1] = p;
  }
  int diff = 0;
  for (int j = 0; j < 4; ++j) {
    feature_ids[s * 4 + j] = id[j];
    joint_ids[s * 4 + j] = id[pos[j]];
    diff |= id[pos[j]] != id[j];
  }
  changed[s] = diff;
}

__device__ __forceinline__ float geometry_residual(const float* __restrict__ geo, long long rows, float4 gs,
                                                   const int64_t* ids, const float* w) {
  float r[4] = {0.f, 0.f, 0.f, 0.f};
  for (int c = 0; c < 4; ++c) {
    long long id = ids[c];
    if (id < 0 || id >= rows) {
      atomicOr(&g_plan_err, kErrBadArgument);
      id = 0;
    }
    const float4 g = *reinterpret_cast<const float4*>(geo + id * 4);
    r[0] = __fadd_rn(r[0], __fmul_rn(w[c], g.x));
    r[1] = __fadd_rn(r[1], __fmul_rn(w[c], g.y));
    r[2] = __fadd_rn(r[2], __fmul_rn(w[c], g.z));
    r[3] = __fadd_rn(r[3], __fmul_rn(w[c], g.w));
  }
  const float e0 = gs.x - r[0], e1 = gs.y - r[1], e2 = gs.z - r[2], e3 = gs.w - r[3];
  return sqrtf(e0 * e0 + e1 * e1 + e2 * e2 + e3 * e3);
}

// The Pareto guard (sparse_convex.py:586-639, :335-367), one thread per source: the joint set
// wins only where it differs from the feature top-4, its cosine and residual are no worse up
// to the tolerance, and its 4-D residual || g_s - sum_c w_c g_c || is strictly smaller.
__global__ void geometry_guard_kernel(long long S, const float* __restrict__ geo, long long rows,
                                      const int64_t* __restrict__ source_ids, const int64_t* __restrict__ fid,
                                      const float* __restrict__ fw, const float* __restrict__ fcos,
                                      const float* __restrict__ fres, const float* __restrict__ fnrm,
                                      const int64_t* __restrict__ jid, const float* __restrict__ jw,
                                      const float* __restrict__ jcos, const float* __restrict__ jres,
                                      const float* __restrict__ jnrm, const int32_t* __restrict__ changed, float tol,
                                      int64_t* __restrict__ out_id, float* __restrict__ out_w,
                                      float* __restrict__ out_cos, float* __restrict__ out_res,
                                      float* __restrict__ out_nrm, int32_t* __restrict__ chosen) {
  const long long s = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (s >= S) return;
  long long src = source_ids[s];
  if (src < 0 || src >= rows) {
    atomicOr(&g_plan_err, kErrBadArgument);
    src = 0;
  }
  const float4 gs = *reinterpret_cast<const float4*>(geo + src * 4);
  const float gf = geometry_residual(geo, rows, gs, fid + s * 4, fw + s * 4);
  const float gj = geometry_residual(geo, rows, gs, jid + s * 4, jw + s * 4);
  const bool pick = changed[s] != 0 && __fadd_rn(jcos[s], tol) >= fcos[s] && jres[s] <= __fadd_rn(fres[s], tol) &&
                    gj < gf;
  for (int c = 0; c < 4; ++c) {
    out_id[s * 4 + c] = pick ? jid[s * 4 + c] : fid[s * 4 + c];
    out_w[s * 4 + c] = pick ? jw[s * 4 + c] : fw[s * 4 + c];
  }
  out_cos[s] = pick ? jcos[s] : fcos[s];
  out_res[s] = pick ? jres[s] : fres[s];
  out_nrm[s] = pick ? jnrm[s] : fnrm[s];
  chosen[s] = pick;
}

inline unsigned blocks(long long n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

}  // namespace

unsigned plan_error_word(int clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_plan_err, sizeof(v));
  if (clear) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_plan_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace vb200

using namespace vb200;

extern "C" size_t vb200_merge_assign_workspace_size(int64_t S, int64_t total) {
  if (S < 0 || total < 0) return 0;
  return assign_layout(S, total).total;
}

extern "C" int vb200_merge_assign(const float* best, const int64_t* target, const int64_t* source_idx,
                                  const int64_t* dest_idx, int64_t S, int64_t Dn, int64_t total,
                                  int64_t removed, int64_t* keep, int64_t* inverse, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  VB200_REQUIRE(S >= 0 && Dn >= 0 && total >= 0 && removed >= 0 && removed <= S && S <= total,
                "merge_assign: bad sizes S=%lld Dn=%lld total=%lld removed=%lld", (long long)S,
                (long long)Dn, (long long)total, (long long)removed);
  VB200_REQUIRE(total < (1ll << 31), "merge_assign: total exceeds the int32 index range");
  if (total == 0) return VB200_OK;
  VB200_REQUIRE(keep && inverse, "merge_assign: null output");
  VB200_REQUIRE(removed == 0 || (best && target && source_idx && dest_idx && Dn > 0),
                "merge_assign: null input");
  const AssignWorkspace lay = assign_layout(S, total);
  VB200_REQUIRE(workspace != nullptr && workspace_bytes >= lay.total,
                "merge_assign: workspace of %zu bytes required (got %zu)", lay.total, workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* keys_out = reinterpret_cast<float*>(ws + lay.keys_out);
  int32_t* vals_in = reinterpret_cast<int32_t*>(ws + lay.vals_in);
  int32_t* vals_out = reinterpret_cast<int32_t*>(ws + lay.vals_out);
  int32_t* flags = reinterpret_cast<int32_t*>(ws + lay.flags);
  int32_t* compact = reinterpret_cast<int32_t*>(ws + lay.compact);
  int64_t* remap = reinterpret_cast<int64_t*>(ws + lay.remap);
  fill_ones_kernel<<<blocks(total, 256), 256, 0, st>>>(flags, total);
  VB200_CHECK_LAUNCH("fill_ones_kernel");
  if (removed > 0) {
    iota_kernel<<<blocks(S, 256), 256, 0, st>>>(vals_in, S);
    VB200_CHECK_LAUNCH("iota_kernel");
    size_t sort_bytes = lay.sort_bytes;
    // radix sort is stable: equal scores keep ascending source order (argsort(stable=True))
    VB200_CHECK_CUDA(cub::DeviceRadixSort::SortPairsDescending(ws + lay.sort_tmp, sort_bytes, best, keys_out,
                                                               vals_in, vals_out, static_cast<int>(S), 0, 32, st),
                     "cub::DeviceRadixSort::SortPairsDescending");
    mark_removed_kernel<<<blocks(removed, 256), 256, 0, st>>>(vals_out, target, source_idx, dest_idx, removed,
                                                              Dn, total, flags, remap);
    VB200_CHECK_LAUNCH("mark_removed_kernel");
  }
  size_t scan_bytes = lay.scan_bytes;
  VB200_CHECK_CUDA(cub::DeviceScan::ExclusiveSum(ws + lay.scan_tmp, scan_bytes, flags, compact,
                                                 static_cast<int>(total), st),
                   "cub::DeviceScan::ExclusiveSum");
  keep_inverse_kernel<<<blocks(total, 256), 256, 0, st>>>(flags, compact, remap, total, total - removed, keep,
                                                          inverse);
  VB200_CHECK_LAUNCH("keep_inverse_kernel");
  return VB200_OK;
}

extern "C" int vb200_support_fit(int dtype, const void* feat, int64_t rows, int64_t row_stride,
                                 const int64_t* src_rows, const int64_t* parent_rows, int64_t S,
                                 int64_t D, float* gram, float* rhs, float* alpha, int steps,
                                 void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16,
                "support_fit: bad dtype %d", dtype);
  VB200_REQUIRE(S >= 0 && D > 0 && rows > 0 && steps >= 0, "support_fit: bad sizes");
  if (S == 0) return VB200_OK;
  VB200_REQUIRE(feat && parent_rows, "support_fit: null pointer");
  const int es = dtype == VB200_F32 ? 4 : 2;
  VB200_REQUIRE((D * es) % 16 == 0 && (row_stride * es) % 16 == 0 &&
                    (reinterpret_cast<uintptr_t>(feat) & 15u) == 0,
                "support_fit: rows must be 16-byte aligned and D a multiple of %d", 16 / es);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define VB200_FIT(T)                                                                                \
  support_fit_kernel<T><<<blocks(S, kFitWarps), kFitWarps * 32, 0, st>>>(static_cast<const T*>(feat), rows, row_stride, \
                                                       src_rows, parent_rows, S, static_cast<int>(D),  \
                                                       gram, rhs, alpha, steps)
  if (dtype == VB200_F32) VB200_FIT(float);
  else if (dtype == VB200_BF16) VB200_FIT(__nv_bfloat16);
  else VB200_FIT(__half);
#undef VB200_FIT
  VB200_CHECK_LAUNCH("support_fit_kernel");
  return VB200_OK;
}

extern "C" int vb200_support_certificate(int dtype, const void* feat, int64_t rows, int64_t row_stride,
                                         const int64_t* src_rows, const int64_t* parent_rows, const float* alpha,
                                         int64_t S, int64_t D, float* cosine, float* residual, float* recon_norm,
                                         void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16,
                "support_certificate: bad dtype %d", dtype);
  VB200_REQUIRE(S >= 0 && D > 0 && rows > 0, "support_certificate: bad sizes");
  if (S == 0) return VB200_OK;
  VB200_REQUIRE(feat && parent_rows && alpha && cosine && residual && recon_norm, "support_certificate: null pointer");
  const int es = dtype == VB200_F32 ? 4 : 2;
  VB200_REQUIRE(D % 16 == 0 && (row_stride * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(feat) & 15u) == 0,
                "support_certificate: rows must be 16-byte aligned and D a multiple of 16");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define VB200_CERT(T)                                                                                   \
  support_certificate_kernel<T><<<blocks(S, kFitWarps), kFitWarps * 32, 0, st>>>(                        \
      static_cast<const T*>(feat), rows, row_stride, src_rows, parent_rows, alpha, S, static_cast<int>(D), \
      cosine, residual, recon_norm)
  if (dtype == VB200_F32) VB200_CERT(float);
  else if (dtype == VB200_BF16) VB200_CERT(__nv_bfloat16);
  else VB200_CERT(__half);
#undef VB200_CERT
  VB200_CHECK_LAUNCH("support_certificate_kernel");
  return VB200_OK;
}

extern "C" int vb200_row_max_dot(int dtype, const void* feat, int64_t rows, int64_t row_stride, const int64_t* query,
                                 const int64_t* targets, int n_targets, int64_t Q, int64_t D, float* out,
                                 void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "row_max_dot: bad dtype %d", dtype);
  VB200_REQUIRE(Q >= 0 && D > 0 && rows > 0 && n_targets >= 0, "row_max_dot: bad sizes");
  if (Q == 0) return VB200_OK;
  VB200_REQUIRE(feat && query && out && (n_targets == 0 || targets), "row_max_dot: null pointer");
  const int es = dtype == VB200_F32 ? 4 : 2;
  VB200_REQUIRE(D % 16 == 0 && (row_stride * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(feat) & 15u) == 0,
                "row_max_dot: rows must be 16-byte aligned and D a multiple of 16");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define VB200_RMD(T)                                                                                      \
  row_max_dot_kernel<T><<<blocks(Q, kFitWarps), kFitWarps * 32, 0, st>>>(                                  \
      static_cast<const T*>(feat), rows, row_stride, query, targets, n_targets, Q, static_cast<int>(D), out)
  if (dtype == VB200_F32) VB200_RMD(float);
  else if (dtype == VB200_BF16) VB200_RMD(__nv_bfloat16);
  else VB200_RMD(__half);
#undef VB200_RMD
  VB200_CHECK_LAUNCH("row_max_dot_kernel");
  return VB200_OK;
}

extern "C" int vb200_geometry_shortlist(const float* values, const int64_t* indices, int64_t S, int k,
                                        const float* query_geo, const float* basis_geo, int64_t Nb, float weight,
                                        int64_t* feature_ids, int64_t* joint_ids, int32_t* changed, void* stream) {
  VB200_REQUIRE(S >= 0 && k >= 4 && k <= 16 && Nb >= 0, "geometry_shortlist: need 4 <= k <= 16");
  if (S == 0) return VB200_OK;
  VB200_REQUIRE(values && indices && query_geo && basis_geo && feature_ids && joint_ids && changed,
                "geometry_shortlist: null pointer");
  VB200_REQUIRE((reinterpret_cast<uintptr_t>(query_geo) & 15u) == 0 && (reinterpret_cast<uintptr_t>(basis_geo) & 15u) == 0,
                "geometry_shortlist: geometry rows must be 16-byte aligned [rows, 4] fp32");
  geometry_shortlist_kernel<<<blocks(S, 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      values, indices, S, k, query_geo, basis_geo, Nb, weight, feature_ids, joint_ids, changed);
  VB200_CHECK_LAUNCH("geometry_shortlist_kernel");
  return VB200_OK;
}

extern "C" int vb200_geometry_guard(int64_t S, const float* geometry, int64_t rows, const int64_t* source_ids,
                                    const int64_t* feature_ids, const float* feature_w, const float* feature_cos,
                                    const float* feature_res, const float* feature_nrm, const int64_t* joint_ids,
                                    const float* joint_w, const float* joint_cos, const float* joint_res,
                                    const float* joint_nrm, const int32_t* changed, float tolerance, int64_t* out_ids,
                                    float* out_w, float* out_cos, float* out_res, float* out_nrm, int32_t* chosen,
                                    void* stream) {
  VB200_REQUIRE(S >= 0 && rows > 0 && tolerance >= 0.f, "geometry_guard: bad sizes or negative tolerance");
  if (S == 0) return VB200_OK;
  VB200_REQUIRE(geometry && source_ids && feature_ids && feature_w && feature_cos && feature_res && feature_nrm &&
                    joint_ids && joint_w && joint_cos && joint_res && joint_nrm && changed && out_ids && out_w &&
                    out_cos && out_res && out_nrm && chosen,
                "geometry_guard: null pointer");
  VB200_REQUIRE((reinterpret_cast<uintptr_t>(geometry) & 15u) == 0,
                "geometry_guard: geometry must be 16-byte aligned [rows, 4] fp32");
  geometry_guard_kernel<<<blocks(S, 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      S, geometry, rows, source_ids, feature_ids, feature_w, feature_cos, feature_res, feature_nrm, joint_ids, joint_w,
      joint_cos, joint_res, joint_nrm, changed, tolerance, out_ids, out_w, out_cos, out_res, out_nrm, chosen);
  VB200_CHECK_LAUNCH("geometry_guard_kernel");
  return VB200_OK;
}
