// The flow-free TTT pre-pass (vggt_omega/utils/ttt_kernels.py): the per-clip work that turns
// patch descriptors into the labels, sensitivity and geometry the released planner consumes.
//
//   row_l2_normalize   descriptor rows / max(||row||, eps), fp32 out (normalize_rows,
//                      ttt_kernels.py:233-249; the reference's default is F.normalize(eps=1e-6)).
//   local_top2_match   exact-window cosine top-2 between the patch grids of two frames
//                      (_local_top2_match_kernel, ttt_kernels.py:45-101, wrapper :252-277): for
//                      every source patch the best and second-best dot over the targets within
//                      (2 ry + 1) x (2 rx + 1), in the reference's candidate order (row-major
//                      offsets, or reversed for the backward direction); a candidate replaces
//                      the best only when strictly greater, so the first of equal maxima wins.
//   integer_warp       border-clamped integer gather of a [B,H,W,C] field by a truncated
//                      integer flow (ttt_kernels.py:104-127, :280-297).
//   motion_cues        per patch: mean |flow - predicted| over the available directions, the
//                      smaller confidence, and |flow - 3x3 zero-padded box mean| (:130-196, :300-318).
//   sensitivity_labels 0.45 novelty + 0.35 residual + 0.20 boundary (clamped units) and the
//                      low-confidence / raw-event predicates (:199-230, :321-341).
//
// All arithmetic is fp32 with IEEE division and square root.  The descriptors are small
// (a few hundred thousand patches of 32-256 channels); the match gives each candidate of a patch
// its own lane and reads the candidate rows through L1, where neighbouring patches' windows
// overlap.
#include "common.cuh"
#include "host_common.h"

namespace vb200 {
namespace {

constexpr int kTttWarps = 8;

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline unsigned blocks_of(long long n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

// G lanes per row (G a power of two, G x 16-byte vectors cover the row in as few passes as
// possible: 32 / G rows per warp), the sum of squares reduced over the G lanes, fp32 out.
template <typename T>
__global__ void __launch_bounds__(kTttWarps * 32)
    row_l2_normalize_kernel(const T* __restrict__ x, long long rows, int C, int G, float eps, float* __restrict__ out) {
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  const int lane = threadIdx.x & 31;
  const long long r = (static_cast<long long>(blockIdx.x) * kTttWarps + (threadIdx.x >> 5)) * (32 / G) + lane / G;
  const int sub = lane % G;
  const int nv = C / V;
  constexpr int kKeep = 4;  // vectors per lane kept in registers between the two passes
  const uint4* xr = reinterpret_cast<const uint4*>(x + r * C);
  uint4 keep[kKeep];
  float ss = 0.f;
  auto sumsq = [&](const uint4& raw) {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float f = to_f32<T>(e[i]);
      ss = fmaf(f, f, ss);
    }
  };
  if (r < rows) {
#pragma unroll
    for (int j = 0; j < kKeep; ++j) {
      if (sub + j * G < nv) {
        keep[j] = __ldg(xr + sub + j * G);
        sumsq(keep[j]);
      }
    }
    for (int v = sub + kKeep * G; v < nv; v += G) sumsq(__ldg(xr + v));
  }
  for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (r >= rows) return;
  const float norm = fmaxf(sqrtf(ss), eps);
  auto scale = [&](const uint4& raw, int v) {
    const T* e = reinterpret_cast<const T*>(&raw);
    float o[V];
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = __fdiv_rn(to_f32<T>(e[i]), norm);
#pragma unroll
    for (int i = 0; i < V; i += 4)
      *reinterpret_cast<float4*>(out + r * C + v * V + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
  };
#pragma unroll
  for (int j = 0; j < kKeep; ++j)
    if (sub + j * G < nv) scale(keep[j], sub + j * G);
  for (int v = sub + kKeep * G; v < nv; v += G) scale(__ldg(xr + v), v);
}

// Rows that are not 16-byte vectors (C not a multiple of the vector, or unaligned): one warp per
// row, scalar loads.
template <typename T>
__global__ void __launch_bounds__(kTttWarps * 32)
    row_l2_normalize_scalar_kernel(const T* __restrict__ x, long long rows, int C, float eps, float* __restrict__ out) {
  const long long r = static_cast<long long>(blockIdx.x) * kTttWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const T* xr = x + r * C;
  float ss = 0.f;
  for (int c = lane; c < C; c += 32) {
    const float v = to_f32<T>(xr[c]);
    ss = fmaf(v, v, ss);
  }
  const float norm = fmaxf(sqrtf(warp_allsum(ss)), eps);
  for (int c = lane; c < C; c += 32) out[r * C + c] = __fdiv_rn(to_f32<T>(xr[c]), norm);
}

// One warp per source patch, one lane per candidate (lane l takes candidates l, l + 32, ...):
// the source row sits in shared memory (read as broadcasts), each lane walks its candidate's
// target row in 16-byte vectors (L1 hits: neighbouring patches share most of their windows) and
// keeps its own best (strict '>' in candidate order, so the first of equal maxima) and second.
// The warp then combines them: best = the largest value at the lowest candidate index, second
// = the largest of everything else (the owning lane's second, every other lane's best), which is
// what the reference's sequential scan produces.  C <= 256.
template <typename T>
__device__ __forceinline__ float dot_row(const float* __restrict__ s, const T* __restrict__ t, int C) {
  float acc = 0.f;
  if constexpr (sizeof(T) == 4) {
    for (int c = 0; c < C; c += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(t + c));
      acc = fmaf(s[c], v.x, acc);
      acc = fmaf(s[c + 1], v.y, acc);
      acc = fmaf(s[c + 2], v.z, acc);
      acc = fmaf(s[c + 3], v.w, acc);
    }
  } else {
    for (int c = 0; c < C; c += 8) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(t + c));
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = fmaf(s[c + i], to_f32<T>(e[i]), acc);
    }
  }
  return acc;
}

template <typename T>
__global__ void __launch_bounds__(kTttWarps * 32)
    local_top2_match_kernel(const T* __restrict__ source, const T* __restrict__ target, long long rows, int H, int W,
                            int C, int ry, int rx, int reverse, float* __restrict__ best_out,
                            float* __restrict__ second_out, int32_t* __restrict__ dy_out,
                            int32_t* __restrict__ dx_out) {
  __shared__ float src_s[kTttWarps][256];
  const int warp = threadIdx.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * kTttWarps + warp;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long long pc = static_cast<long long>(H) * W;
  const long long pair = row / pc;
  const int patch = static_cast<int>(row - pair * pc);
  const int y = patch / W, x = patch - (patch / W) * W;
  float* s = src_s[warp];
  for (int c = lane; c < C; c += 32) s[c] = to_f32<T>(source[row * C + c]);
  __syncwarp();
  const int span_x = 2 * rx + 1;
  const int candidates = (2 * ry + 1) * span_x;
  float best = -INFINITY, second = -INFINITY;
  int bk = 0x7fffffff;
  for (int k = lane; k < candidates; k += 32) {
    const int cy = k / span_x, cx = k - (k / span_x) * span_x;
    const int ty = y + (reverse ? ry - cy : cy - ry), tx = x + (reverse ? rx - cx : cx - rx);
    float sim = -INFINITY;
    if (ty >= 0 && ty < H && tx >= 0 && tx < W)
      sim = dot_row<T>(s, target + (pair * pc + static_cast<long long>(ty) * W + tx) * C, C);
    const bool better = sim > best;
    second = better ? best : fmaxf(second, sim);
    if (better) {
      best = sim;
      bk = k;
    }
  }
  // warp combine: the largest best, at the lowest candidate index among equal values
  float m = best;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  int kmin = best == m ? bk : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
  float sec = bk == kmin ? second : best;  // the owner offers its second, every other lane its best
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sec = fmaxf(sec, __shfl_xor_sync(0xffffffffu, sec, o));
  if (lane == 0) {
    const int cy = kmin / span_x, cx = kmin - (kmin / span_x) * span_x;
    best_out[row] = m;
    second_out[row] = sec;
    dy_out[row] = reverse ? ry - cy : cy - ry;
    dx_out[row] = reverse ? rx - cx : cx - rx;
  }
}

// Tiled form (the default when the window fits): one CTA per (pair, tile x tile source patches).
// The tile's target window with its halo ((tile + 2 ry) x (tile + 2 rx) rows of C channels, fp32)
// and the tile's source rows are staged in shared memory once, so every target row is read from
// L2 once per tile instead of once per neighbouring patch.  Each warp then takes the tile's
// patches in turn, one lane per candidate as in local_top2_match_kernel (same order and
// tie-breaking); the target rows are padded by 4 floats so that the lanes' 16-byte reads of
// different rows spread over all banks.
constexpr int kTiledWarps = 16;

__global__ void __launch_bounds__(kTiledWarps * 32)
    local_top2_tiled_kernel(const float* __restrict__ source, const float* __restrict__ target, int H, int W, int C,
                            int ry, int rx, int reverse, int tile, float* __restrict__ best_out,
                            float* __restrict__ second_out, int32_t* __restrict__ dy_out,
                            int32_t* __restrict__ dx_out) {
  extern __shared__ __align__(16) float tsm[];
  const int tiles_x = (W + tile - 1) / tile;
  const int ty0 = (blockIdx.x / tiles_x) * tile, tx0 = (blockIdx.x % tiles_x) * tile;
  const long long pair = blockIdx.y;
  const long long pc = static_cast<long long>(H) * W;
  const int HY = tile + 2 * ry, HX = tile + 2 * rx;
  const int stride = C + 4;  // floats per staged target row
  float* tgt_s = tsm;
  float* src_s = tsm + static_cast<size_t>(HY) * HX * stride;
  const int q4 = C / 4;
  // stage the target window (rows outside the grid are never read) and the tile's source rows
#pragma unroll 4
  for (int i = threadIdx.x; i < HY * HX * q4; i += blockDim.x) {
    const int r = i / q4, q = i - r * q4;
    const int gy = ty0 - ry + r / HX, gx = tx0 - rx + r % HX;
    if (gy >= 0 && gy < H && gx >= 0 && gx < W)
      *reinterpret_cast<float4*>(tgt_s + static_cast<size_t>(r) * stride + 4 * q) =
          __ldg(reinterpret_cast<const float4*>(target + ((pair * pc + static_cast<long long>(gy) * W + gx) * C) + 4 * q));
  }
  for (int i = threadIdx.x; i < tile * tile * q4; i += blockDim.x) {
    const int r = i / q4, q = i - r * q4;
    const int gy = ty0 + r / tile, gx = tx0 + r % tile;
    if (gy < H && gx < W)
      *reinterpret_cast<float4*>(src_s + static_cast<size_t>(r) * C + 4 * q) =
          __ldg(reinterpret_cast<const float4*>(source + ((pair * pc + static_cast<long long>(gy) * W + gx) * C) + 4 * q));
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int span_x = 2 * rx + 1;
  const int candidates = (2 * ry + 1) * span_x;
  for (int p = warp; p < tile * tile; p += kTiledWarps) {
    const int y = ty0 + p / tile, x = tx0 + p % tile;
    if (y >= H || x >= W) continue;  // uniform across the warp
    const float* sv = src_s + static_cast<size_t>(p) * C;
    float best = -INFINITY, second = -INFINITY;
    int bk = 0x7fffffff;
    for (int k = lane; k < candidates; k += 32) {
      const int cy = k / span_x, cx = k - (k / span_x) * span_x;
      const int oy = reverse ? ry - cy : cy - ry, ox = reverse ? rx - cx : cx - rx;
      float sim = -INFINITY;
      if (y + oy >= 0 && y + oy < H && x + ox >= 0 && x + ox < W) {
        const float* tv = tgt_s + static_cast<size_t>((p / tile + ry + oy) * HX + (p % tile + rx + ox)) * stride;
        // four independent partial sums (channel c mod 4), added at the end
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
        for (int c = 0; c < C; c += 4) {
          const float4 a = *reinterpret_cast<const float4*>(sv + c);
          const float4 b = *reinterpret_cast<const float4*>(tv + c);
          a0 = fmaf(a.x, b.x, a0);
          a1 = fmaf(a.y, b.y, a1);
          a2 = fmaf(a.z, b.z, a2);
          a3 = fmaf(a.w, b.w, a3);
        }
        sim = (a0 + a1) + (a2 + a3);
      }
      const bool better = sim > best;
      second = better ? best : fmaxf(second, sim);
      if (better) {
        best = sim;
        bk = k;
      }
    }
    float m = best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int kmin = best == m ? bk : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    float sec = bk == kmin ? second : best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sec = fmaxf(sec, __shfl_xor_sync(0xffffffffu, sec, o));
    if (lane == 0) {
      const long long row = pair * pc + static_cast<long long>(y) * W + x;
      const int cy = kmin / span_x, cx = kmin - (kmin / span_x) * span_x;
      best_out[row] = m;
      second_out[row] = sec;
      dy_out[row] = reverse ? ry - cy : cy - ry;
      dx_out[row] = reverse ? rx - cx : cx - rx;
    }
  }
}

constexpr size_t kTileSmemMax = 200 * 1024;

inline size_t tiled_smem(int tile, int ry, int rx, int C) {
  return (static_cast<size_t>(tile + 2 * ry) * (tile + 2 * rx) * (C + 4) + static_cast<size_t>(tile) * tile * C) *
         sizeof(float);
}

// One thread per element; flow (x, y) is truncated toward zero like a float -> int cast.
template <typename T>
__global__ void integer_warp_kernel(const T* __restrict__ field, const float* __restrict__ flow, long long elements,
                                    int H, int W, int C, T* __restrict__ out) {
  const long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= elements) return;
  const long long row = e / C;
  const int ch = static_cast<int>(e - row * C);
  const long long pc = static_cast<long long>(H) * W;
  const long long b = row / pc;
  const int patch = static_cast<int>(row - b * pc);
  const int y = patch / W, x = patch - (patch / W) * W;
  const int fx = static_cast<int>(flow[row * 2]);
  const int fy = static_cast<int>(flow[row * 2 + 1]);
  const int sx = min(max(x + fx, 0), W - 1);
  const int sy = min(max(y + fy, 0), H - 1);
  out[e] = field[(b * pc + static_cast<long long>(sy) * W + sx) * C + ch];
}

__device__ __forceinline__ float hyp(float a, float b) { return sqrtf(a * a + b * b); }

// One thread per patch of frame f: forward flow of pair f (f + 1 < F), backward flow of pair
// f - 1 (f > 0); absent directions contribute nothing and count nothing.
__global__ void motion_cues_kernel(const float* __restrict__ fwd, const float* __restrict__ bwd,
                                   const float* __restrict__ pred, const float* __restrict__ fconf,
                                   const float* __restrict__ bconf, int F, int H, int W, float* __restrict__ residual,
                                   float* __restrict__ confidence, float* __restrict__ boundary) {
  const long long pc = static_cast<long long>(H) * W;
  const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= F * pc) return;
  const int f = static_cast<int>(row / pc);
  const int patch = static_cast<int>(row - f * pc);
  const int y = patch / W, x = patch - (patch / W) * W;
  const bool has_f = f + 1 < F, has_b = f > 0;
  const long long frow = f * pc + patch, brow = (f - 1) * pc + patch;
  const float fdx = has_f ? fwd[frow * 2] : 0.f, fdy = has_f ? fwd[frow * 2 + 1] : 0.f;
  const float bdx = has_b ? bwd[brow * 2] : 0.f, bdy = has_b ? bwd[brow * 2 + 1] : 0.f;
  const float pfx = has_f ? pred[row * 4] : 0.f, pfy = has_f ? pred[row * 4 + 1] : 0.f;
  const float pbx = has_b ? pred[row * 4 + 2] : 0.f, pby = has_b ? pred[row * 4 + 3] : 0.f;
  const float f_res = hyp(fdx - pfx, fdy - pfy);
  const float b_res = hyp(bdx - pbx, bdy - pby);
  const float count = static_cast<float>(has_f) + static_cast<float>(has_b);
  float fmx = 0.f, fmy = 0.f, bmx = 0.f, bmy = 0.f;
  for (int oy = -1; oy <= 1; ++oy) {
    for (int ox = -1; ox <= 1; ++ox) {
      const int ny = y + oy, nx = x + ox;
      const bool inside = ny >= 0 && ny < H && nx >= 0 && nx < W;
      const long long np = static_cast<long long>(ny) * W + nx;
      const bool fi = has_f && inside, bi = has_b && inside;
      fmx += __fdiv_rn(fi ? fwd[(f * pc + np) * 2] : 0.f, 9.f);
      fmy += __fdiv_rn(fi ? fwd[(f * pc + np) * 2 + 1] : 0.f, 9.f);
      bmx += __fdiv_rn(bi ? bwd[((f - 1) * pc + np) * 2] : 0.f, 9.f);
      bmy += __fdiv_rn(bi ? bwd[((f - 1) * pc + np) * 2 + 1] : 0.f, 9.f);
    }
  }
  const float f_bnd = hyp(fdx - fmx, fdy - fmy);
  const float b_bnd = hyp(bdx - bmx, bdy - bmy);
  const float fc = has_f ? fconf[frow] : 1.f, bc = has_b ? bconf[brow] : 1.f;
  const float denom = fmaxf(count, 1.f);
  residual[row] = __fdiv_rn(f_res + b_res, denom);
  confidence[row] = fminf(fc, bc);
  boundary[row] = __fdiv_rn(f_bnd + b_bnd, denom);
}

__device__ __forceinline__ float clamp01(float v) { return fminf(fmaxf(v, 0.f), 1.f); }

__global__ void sensitivity_kernel(const float* __restrict__ residual, const float* __restrict__ confidence,
                                   const float* __restrict__ boundary, long long rows, long long pc, float uc,
                                   const float* __restrict__ rs, const float* __restrict__ bs,
                                   const float* __restrict__ rt, const float* __restrict__ bt,
                                   float* __restrict__ sens, int8_t* __restrict__ low, int8_t* __restrict__ event) {
  const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const bool later = row / pc > 0;
  const float res = residual[row], conf = confidence[row], bnd = boundary[row];
  const float novelty = 1.f - conf;
  const float ru = clamp01(__fdiv_rn(res, fmaxf(*rs, 1e-6f)));
  const float bu = clamp01(__fdiv_rn(bnd, fmaxf(*bs, 1e-6f)));
  sens[row] = clamp01(0.45f * novelty + 0.35f * ru + 0.20f * bu);
  low[row] = later && conf < uc;
  event[row] = later && ((res >= *rt && conf >= uc) || bnd >= *bt || novelty >= 0.55f);
}

}  // namespace
}  // namespace vb200

using namespace vb200;

extern "C" int vb200_row_l2_normalize(int dtype, const void* x, int64_t rows, int64_t C, float eps, float* out,
                                      void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "row_l2_normalize: bad dtype %d",
                dtype);
  VB200_REQUIRE(rows >= 0 && C > 0 && eps >= 0.f, "row_l2_normalize: bad sizes");
  if (rows == 0) return VB200_OK;
  VB200_REQUIRE(x && out, "row_l2_normalize: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define VB200_NRM(T)                                                                                   \
  do {                                                                                                  \
    constexpr int V = 16 / static_cast<int>(sizeof(T));                                                 \
    if (C % V == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) { \
      int G = 1;                                                                                        \
      while (G < 32 && G * 2 * V <= C) G *= 2;                                                          \
      const long long warps = (rows + (32 / G) - 1) / (32 / G);                                        \
      row_l2_normalize_kernel<T><<<blocks_of(warps, kTttWarps), kTttWarps * 32, 0, st>>>(               \
          static_cast<const T*>(x), rows, static_cast<int>(C), G, eps, out);                            \
    } else {                                                                                            \
      row_l2_normalize_scalar_kernel<T><<<blocks_of(rows, kTttWarps), kTttWarps * 32, 0, st>>>(         \
          static_cast<const T*>(x), rows, static_cast<int>(C), eps, out);                               \
    }                                                                                                   \
  } while (0)
  if (dtype == VB200_F32) VB200_NRM(float);
  else if (dtype == VB200_BF16) VB200_NRM(__nv_bfloat16);
  else VB200_NRM(__half);
#undef VB200_NRM
  VB200_CHECK_LAUNCH("row_l2_normalize_kernel");
  return VB200_OK;
}

extern "C" int vb200_local_top2_match(int dtype, const void* source, const void* target, int64_t pairs, int64_t H,
                                      int64_t W, int64_t C, int radius_y, int radius_x, int reverse, float* best,
                                      float* second, int32_t* dy, int32_t* dx, void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "local_top2_match: bad dtype %d",
                dtype);
  VB200_REQUIRE(pairs >= 0 && H > 0 && W > 0 && C >= 1 && C <= 256, "local_top2_match: need 1 <= C <= 256");
  VB200_REQUIRE(C % (dtype == VB200_F32 ? 4 : 8) == 0 && (reinterpret_cast<uintptr_t>(target) & 15u) == 0,
                "local_top2_match: rows must be 16-byte aligned (C a multiple of 4 for f32, 8 for 16-bit)");
  VB200_REQUIRE(radius_y >= 0 && radius_x >= 0 && radius_y < H && radius_x < W,
                "local_top2_match: radii must lie in [0, H) x [0, W)");
  const long long rows = pairs * H * W;
  if (rows == 0) return VB200_OK;
  VB200_REQUIRE(source && target && best && second && dy && dx, "local_top2_match: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == VB200_F32 && (reinterpret_cast<uintptr_t>(source) & 15u) == 0 && pairs <= 65535) {
    // the tiled kernel when an 8 x 8 (or 4 x 4) tile's window fits in shared memory
    for (int tile : {8, 4}) {
      const size_t smem = tiled_smem(tile, radius_y, radius_x, static_cast<int>(C));
      if (smem > kTileSmemMax) continue;
      VB200_CHECK_CUDA(cudaFuncSetAttribute(local_top2_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(smem)),
                       "cudaFuncSetAttribute");
      const dim3 grid(static_cast<unsigned>(((H + tile - 1) / tile) * ((W + tile - 1) / tile)),
                      static_cast<unsigned>(pairs));
      local_top2_tiled_kernel<<<grid, kTiledWarps * 32, smem, st>>>(
          static_cast<const float*>(source), static_cast<const float*>(target), static_cast<int>(H),
          static_cast<int>(W), static_cast<int>(C), radius_y, radius_x, reverse ? 1 : 0, tile, best, second, dy, dx);
      VB200_CHECK_LAUNCH("local_top2_tiled_kernel");
      return VB200_OK;
    }
  }
#define VB200_LTM(T)                                                                                     \
  local_top2_match_kernel<T><<<blocks_of(rows, kTttWarps), kTttWarps * 32, 0, st>>>(                     \
      static_cast<const T*>(source), static_cast<const T*>(target), rows, static_cast<int>(H),            \
      static_cast<int>(W), static_cast<int>(C), radius_y, radius_x, reverse ? 1 : 0, best, second, dy, dx)
  if (dtype == VB200_F32) VB200_LTM(float);
  else if (dtype == VB200_BF16) VB200_LTM(__nv_bfloat16);
  else VB200_LTM(__half);
#undef VB200_LTM
  VB200_CHECK_LAUNCH("local_top2_match_kernel");
  return VB200_OK;
}

extern "C" int vb200_integer_warp(int dtype, const void* field, const float* flow, int64_t B, int64_t H, int64_t W,
                                  int64_t C, void* out, void* stream) {
  VB200_REQUIRE(dtype == VB200_F32 || dtype == VB200_BF16 || dtype == VB200_F16, "integer_warp: bad dtype %d", dtype);
  VB200_REQUIRE(B >= 0 && H > 0 && W > 0 && C > 0, "integer_warp: bad sizes");
  const long long elements = B * H * W * C;
  if (elements == 0) return VB200_OK;
  VB200_REQUIRE(field && flow && out, "integer_warp: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define VB200_IW(T)                                                                                           \
  integer_warp_kernel<T><<<blocks_of(elements, 256), 256, 0, st>>>(static_cast<const T*>(field), flow, elements, \
                                                                   static_cast<int>(H), static_cast<int>(W),      \
                                                                   static_cast<int>(C), static_cast<T*>(out))
  if (dtype == VB200_F32) VB200_IW(float);
  else if (dtype == VB200_BF16) VB200_IW(__nv_bfloat16);
  else VB200_IW(__half);
#undef VB200_IW
  VB200_CHECK_LAUNCH("integer_warp_kernel");
  return VB200_OK;
}

extern "C" int vb200_motion_cues(const float* forward_flow, const float* backward_flow, const float* predicted,
                                 const float* forward_conf, const float* backward_conf, int64_t F, int64_t H,
                                 int64_t W, float* residual, float* confidence, float* boundary, void* stream) {
  VB200_REQUIRE(F >= 1 && H > 0 && W > 0, "motion_cues: bad sizes");
  VB200_REQUIRE(predicted && residual && confidence && boundary &&
                    (F == 1 || (forward_flow && backward_flow && forward_conf && backward_conf)),
                "motion_cues: null pointer");
  const long long rows = F * H * W;
  motion_cues_kernel<<<blocks_of(rows, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      forward_flow, backward_flow, predicted, forward_conf, backward_conf, static_cast<int>(F), static_cast<int>(H),
      static_cast<int>(W), residual, confidence, boundary);
  VB200_CHECK_LAUNCH("motion_cues_kernel");
  return VB200_OK;
}

extern "C" int vb200_sensitivity_labels(const float* residual, const float* confidence, const float* boundary,
                                        int64_t rows, int64_t patch_count, float uncertain_confidence,
                                        const float* residual_scale, const float* boundary_scale,
                                        const float* residual_threshold, const float* boundary_threshold,
                                        float* sensitivity, int8_t* low_confidence, int8_t* raw_event,
                                        void* stream) {
  VB200_REQUIRE(rows >= 0 && patch_count > 0, "sensitivity_labels: bad sizes");
  if (rows == 0) return VB200_OK;
  VB200_REQUIRE(residual && confidence && boundary && residual_scale && boundary_scale && residual_threshold &&
                    boundary_threshold && sensitivity && low_confidence && raw_event,
                "sensitivity_labels: null pointer");
  sensitivity_kernel<<<blocks_of(rows, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      residual, confidence, boundary, rows, patch_count, uncertain_confidence, residual_scale, boundary_scale,
      residual_threshold, boundary_threshold, sensitivity, low_confidence, raw_event);
  VB200_CHECK_LAUNCH("sensitivity_kernel");
  return VB200_OK;
}
