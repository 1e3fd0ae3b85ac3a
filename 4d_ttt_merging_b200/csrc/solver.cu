// Four-support simplex least-squares solvers used by the sparse-convex planner:
//   min_a ||S a - x||^2  s.t. a >= 0, sum a = 1, given gram = S S^T [4x4] and rhs = S x [4].
//
// projected_gradient follows _four_support_projected_gradient_kernel
// (vggt_omega/models/sparse_convex_kernels.py:214-280): a = e0, step = 0.95 / max(max row
// abs-sum of gram, 1e-4), `steps` iterations of a gradient step followed by the Euclidean
// projection onto the simplex computed from a 4-value sorting network.
// active_set follows _four_support_active_candidates_kernel + _select_active_candidate_kernel
// (sparse_convex_kernels.py:96-212): the 15 non-empty active sets are solved in closed form
// (Cramer's rule on the reduced system with the last active variable eliminated), infeasible
// or singular candidates are discarded, the lowest objective wins and the one-hot first support
// replaces it when its cosine is higher.
// One thread per row; both are tiny next to the GEMMs that produce gram / rhs.
#include "common.cuh"
#include "host_common.h"

namespace vb200 {
namespace {

__global__ void projected_gradient_kernel(const float* __restrict__ gram, const float* __restrict__ rhs,
                                          float* __restrict__ out, long long rows, int steps) {
  const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float* g = gram + row * 16;
  const float* r = rhs + row * 4;
  float G[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) G[i] = g[i];
  const float r0 = r[0], r1 = r[1], r2 = r[2], r3 = r[3];
  const float n0 = fabsf(G[0]) + fabsf(G[1]) + fabsf(G[2]) + fabsf(G[3]);
  const float n1 = fabsf(G[4]) + fabsf(G[5]) + fabsf(G[6]) + fabsf(G[7]);
  const float n2 = fabsf(G[8]) + fabsf(G[9]) + fabsf(G[10]) + fabsf(G[11]);
  const float n3 = fabsf(G[12]) + fabsf(G[13]) + fabsf(G[14]) + fabsf(G[15]);
  const float lip = fmaxf(fmaxf(n0, n1), fmaxf(n2, n3));
  const float step = 0.95f / fmaxf(lip, 1.0e-4f);
  float a0 = 1.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  for (int it = 0; it < steps; ++it) {
    const float p0 = a0 - step * (G[0] * a0 + G[1] * a1 + G[2] * a2 + G[3] * a3 - r0);
    const float p1 = a1 - step * (G[4] * a0 + G[5] * a1 + G[6] * a2 + G[7] * a3 - r1);
    const float p2 = a2 - step * (G[8] * a0 + G[9] * a1 + G[10] * a2 + G[11] * a3 - r2);
    const float p3 = a3 - step * (G[12] * a0 + G[13] * a1 + G[14] * a2 + G[15] * a3 - r3);
    // descending sorting network; only the threshold uses the sorted order
    float s0 = fmaxf(p0, p1), s1 = fminf(p0, p1);
    float s2 = fmaxf(p2, p3), s3 = fminf(p2, p3);
    float t;
    t = fmaxf(s0, s2); s2 = fminf(s0, s2); s0 = t;
    t = fmaxf(s1, s3); s3 = fminf(s1, s3); s1 = t;
    t = fmaxf(s1, s2); s2 = fminf(s1, s2); s1 = t;
    float theta = s0 - 1.f;
    const float theta2 = (s0 + s1 - 1.f) * 0.5f;
    theta = s1 > theta2 ? theta2 : theta;
    const float theta3 = (s0 + s1 + s2 - 1.f) / 3.f;
    theta = s2 > theta3 ? theta3 : theta;
    const float theta4 = (s0 + s1 + s2 + s3 - 1.f) * 0.25f;
    theta = s3 > theta4 ? theta4 : theta;
    a0 = fmaxf(p0 - theta, 0.f);
    a1 = fmaxf(p1 - theta, 0.f);
    a2 = fmaxf(p2 - theta, 0.f);
    a3 = fmaxf(p3 - theta, 0.f);
  }
  float* o = out + row * 4;
  o[0] = a0;
  o[1] = a1;
  o[2] = a2;
  o[3] = a3;
}

// Active sets in the order of the reference table: ids padded with the last active id.
__constant__ int kActiveIds[15][4] = {
    {0, 0, 0, 0}, {1, 1, 1, 1}, {2, 2, 2, 2}, {3, 3, 3, 3}, {0, 1, 1, 1},
    {0, 2, 2, 2}, {0, 3, 3, 3}, {1, 2, 2, 2}, {1, 3, 3, 3}, {2, 3, 3, 3},
    {0, 1, 2, 2}, {0, 1, 3, 3}, {0, 2, 3, 3}, {1, 2, 3, 3}, {0, 1, 2, 3}};
__constant__ int kActiveCount[15] = {1, 1, 1, 1, 2, 2, 2, 2, 2, 2, 3, 3, 3, 3, 4};

__global__ void active_set_kernel(const float* __restrict__ gram, const float* __restrict__ rhs,
                                  float* __restrict__ out, long long rows, float ridge) {
  const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float G[16], R[4];
#pragma unroll
  for (int i = 0; i < 16; ++i) G[i] = gram[row * 16 + i];
#pragma unroll
  for (int i = 0; i < 4; ++i) R[i] = rhs[row * 4 + i];
  auto ge = [&](int a, int b) { return G[a * 4 + b] + (a == b ? ridge : 0.f); };
  float best_obj = INFINITY;
  float best[4] = {0.f, 0.f, 0.f, 0.f};
  bool have_best = false;
  for (int set = 0; set < 15; ++set) {
    const int count = kActiveCount[set];
    const int i0 = kActiveIds[set][0], i1 = kActiveIds[set][1], i2 = kActiveIds[set][2];
    const int p = kActiveIds[set][count - 1];
    const float hp = ge(p, p);
    const float rp = R[p];
    const float h00 = ge(i0, i0) - 2.f * ge(i0, p) + hp;
    const float h01 = ge(i0, i1) - ge(i0, p) - ge(p, i1) + hp;
    const float h02 = ge(i0, i2) - ge(i0, p) - ge(p, i2) + hp;
    const float h10 = ge(i1, i0) - ge(i1, p) - ge(p, i0) + hp;
    const float h11 = ge(i1, i1) - 2.f * ge(i1, p) + hp;
    const float h12 = ge(i1, i2) - ge(i1, p) - ge(p, i2) + hp;
    const float h20 = ge(i2, i0) - ge(i2, p) - ge(p, i0) + hp;
    const float h21 = ge(i2, i1) - ge(i2, p) - ge(p, i1) + hp;
    const float h22 = ge(i2, i2) - 2.f * ge(i2, p) + hp;
    const float c0 = R[i0] - rp - ge(i0, p) + hp;
    const float c1 = R[i1] - rp - ge(i1, p) + hp;
    const float c2 = R[i2] - rp - ge(i2, p) + hp;
    const float safe_h00 = fabsf(h00) > 1.0e-12f ? h00 : 1.f;
    const float one_x = c0 / safe_h00;
    const float det2 = h00 * h11 - h01 * h10;
    const float safe_det2 = fabsf(det2) > 1.0e-12f ? det2 : 1.f;
    const float two_x = (c0 * h11 - h01 * c1) / safe_det2;
    const float two_y = (h00 * c1 - h10 * c0) / safe_det2;
    const float det3 = h00 * (h11 * h22 - h12 * h21) - h01 * (h10 * h22 - h12 * h20) +
                       h02 * (h10 * h21 - h11 * h20);
    const float safe_det3 = fabsf(det3) > 1.0e-12f ? det3 : 1.f;
    const float three_x =
        (c0 * (h11 * h22 - h12 * h21) - h01 * (c1 * h22 - h12 * c2) + h02 * (c1 * h21 - h11 * c2)) /
        safe_det3;
    const float three_y =
        (h00 * (c1 * h22 - h12 * c2) - c0 * (h10 * h22 - h12 * h20) + h02 * (h10 * c2 - c1 * h20)) /
        safe_det3;
    const float three_z =
        (h00 * (h11 * c2 - c1 * h21) - h01 * (h10 * c2 - c1 * h20) + c0 * (h10 * h21 - h11 * h20)) /
        safe_det3;
    const int dim = count - 1;
    const float b0 = dim == 1 ? one_x : (dim == 2 ? two_x : (dim == 3 ? three_x : 0.f));
    const float b1 = dim == 2 ? two_y : (dim == 3 ? three_y : 0.f);
    const float b2 = dim == 3 ? three_z : 0.f;
    const float ap = 1.f - b0 - b1 - b2;
    float a[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      a[q] = (i0 == q ? b0 : 0.f) + (i1 == q ? b1 : 0.f) + (i2 == q ? b2 : 0.f) + (p == q ? ap : 0.f);
    const bool stable = count == 1 || (dim == 1 && fabsf(h00) > 1.0e-12f) ||
                        (dim == 2 && fabsf(det2) > 1.0e-12f) || (dim == 3 && fabsf(det3) > 1.0e-12f);
    const bool feasible = stable && a[0] >= -1.0e-5f && a[1] >= -1.0e-5f && a[2] >= -1.0e-5f &&
                          a[3] >= -1.0e-5f;
#pragma unroll
    for (int q = 0; q < 4; ++q) a[q] = fmaxf(a[q], 0.f);
    const float asum = fmaxf(a[0] + a[1] + a[2] + a[3], 1.0e-12f);
#pragma unroll
    for (int q = 0; q < 4; ++q) a[q] = a[q] / asum;
    float obj = 0.f;
    {
      float qv[4];
#pragma unroll
      for (int rr = 0; rr < 4; ++rr)
        qv[rr] = G[rr * 4 + 0] * a[0] + G[rr * 4 + 1] * a[1] + G[rr * 4 + 2] * a[2] + G[rr * 4 + 3] * a[3];
      obj = a[0] * qv[0] + a[1] * qv[1] + a[2] * qv[2] + a[3] * qv[3] -
            2.f * (a[0] * R[0] + a[1] * R[1] + a[2] * R[2] + a[3] * R[3]);
    }
    if (!feasible) obj = INFINITY;
    // argmin keeps the first minimum, as tl.argmin does
    if (!have_best || obj < best_obj) {
      best_obj = obj;
#pragma unroll
      for (int q = 0; q < 4; ++q) best[q] = a[q];
      have_best = true;
    }
  }
  const float bsum = fmaxf(best[0] + best[1] + best[2] + best[3], 1.0e-12f);
#pragma unroll
  for (int q = 0; q < 4; ++q) best[q] = best[q] / bsum;
  float quad[4];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr)
    quad[rr] = G[rr * 4 + 0] * best[0] + G[rr * 4 + 1] * best[1] + G[rr * 4 + 2] * best[2] + G[rr * 4 + 3] * best[3];
  const float num = best[0] * R[0] + best[1] * R[1] + best[2] * R[2] + best[3] * R[3];
  const float sq = best[0] * quad[0] + best[1] * quad[1] + best[2] * quad[2] + best[3] * quad[3];
  const float cosine = num * rsqrtf(fmaxf(sq, 1.0e-12f));
  const bool use_single = R[0] > cosine;
  float* o = out + row * 4;
#pragma unroll
  for (int q = 0; q < 4; ++q) o[q] = use_single ? (q == 0 ? 1.f : 0.f) : best[q];
}

}  // namespace
}  // namespace vb200

using namespace vb200;

extern "C" int vb200_four_support_projected_gradient(const float* gram, const float* rhs, float* out,
                                                     int64_t rows, int steps, void* stream) {
  VB200_REQUIRE(rows >= 0 && steps >= 0, "four_support_projected_gradient: bad sizes");
  if (rows == 0) return VB200_OK;
  VB200_REQUIRE(gram && rhs && out, "four_support_projected_gradient: null pointer");
  projected_gradient_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0,
                              static_cast<cudaStream_t>(stream)>>>(gram, rhs, out, rows, steps);
  VB200_CHECK_LAUNCH("projected_gradient_kernel");
  return VB200_OK;
}

extern "C" int vb200_four_support_active_set(const float* gram, const float* rhs, float* out,
                                             int64_t rows, float ridge, void* stream) {
  VB200_REQUIRE(rows >= 0, "four_support_active_set: bad sizes");
  if (rows == 0) return VB200_OK;
  VB200_REQUIRE(gram && rhs && out, "four_support_active_set: null pointer");
  active_set_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0,
                      static_cast<cudaStream_t>(stream)>>>(gram, rhs, out, rows, ridge);
  VB200_CHECK_LAUNCH("active_set_kernel");
  return VB200_OK;
}
