// Merge step for B200 (sm_100a): cosine-similarity GEMM with a fused running top-k epilogue.
//
//   score[r, n] = bf16_round( sum_d query[r, d] * basis[n, d] )     (fp32 accumulation)
//   out[r]      = the k highest scores of row r (k = 1 or 4), best first, ties -> lower n
//
// This is the bf16 GEMM + max(-1) of build_fastvggt_plan (vggt_omega/models/token_merging.py:
// 1100-1111) and the bf16 GEMM + topk(4) support retrieval (vggt_omega/models/sparse_convex.py:
// 264, 294, 546-547) / streaming_top4 (vggt_omega/models/sparse_convex_kernels.py:20-93, which
// rounds the accumulator to bf16 before ranking, :51-54), without writing the score matrix.
//
// Kernel (one CTA per 128 query rows of one group, 6 warps):
//   warp 0      TMA producer: for every basis tile of 256 rows and every 64-channel k-block,
//               the query k-block [128 x 64] and the basis k-block [256 x 64] (128-byte
//               swizzle), 4-stage ring.
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32 accumulators) and issues
//               tcgen05.mma M=128 N=256 K=16, committing each finished tile to the epilogue.
//   warps 2..5  epilogue: thread t owns query row t, reads its 256 scores per tile from TMEM,
//               rounds each to bf16 and keeps a running top-k in registers; the accumulator
//               buffer is handed back as soon as it has been read, so tile t+1's MMAs overlap
//               tile t's ranking.
// Groups restrict query rows [q_begin[g], q_begin[g+1]) to basis rows [b_begin[g],
// b_begin[g+1]) (frame-group-local matching); columns outside the group are masked.
#include <cudaTypedefs.h>

#include <vector>

#include "common.cuh"
#include "host_common.h"

namespace vb200 {
namespace {

static __device__ unsigned g_merge_err;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;  // channels per k-block (128 bytes of bf16: one swizzle row)
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr int kMaxGroups = 64;  // groups per launch (kernel-parameter table)

constexpr int kOffStage = 0;
constexpr int kOffBar = kStages * kStageBytes;
constexpr int kBarFull = 0;
constexpr int kBarEmpty = kStages;
constexpr int kBarAccFull = 2 * kStages;
constexpr int kBarAccEmpty = kBarAccFull + 2;
constexpr int kNumBars = kBarAccEmpty + 2;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;
constexpr uint32_t kTmemCols = 512;

struct GroupTable {
  long long q_begin[kMaxGroups + 1];
  long long b_begin[kMaxGroups + 1];
};

struct TopkParams {
  float* values;        // [R, k]
  int64_t* indices;     // [R, k]
  int k;
  int k_blocks;         // D / 64
};

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

template <int K>
__device__ __forceinline__ void topk_insert(float (&tv)[4], int (&ti)[4], float v, int n) {
  if constexpr (K == 1) {
    if (v > tv[0]) { tv[0] = v; ti[0] = n; }
  } else {
    if (v > tv[3]) {
      // strict comparisons: an equal score never displaces an earlier (lower) index
      if (v > tv[0]) {
        tv[3] = tv[2]; ti[3] = ti[2]; tv[2] = tv[1]; ti[2] = ti[1]; tv[1] = tv[0]; ti[1] = ti[0];
        tv[0] = v; ti[0] = n;
      } else if (v > tv[1]) {
        tv[3] = tv[2]; ti[3] = ti[2]; tv[2] = tv[1]; ti[2] = ti[1];
        tv[1] = v; ti[1] = n;
      } else if (v > tv[2]) {
        tv[3] = tv[2]; ti[3] = ti[2];
        tv[2] = v; ti[2] = n;
      } else {
        tv[3] = v; ti[3] = n;
      }
    }
  }
}

template <int K>
__global__ void __launch_bounds__(kThreads, 1)
    sim_topk_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ GroupTable groups, TopkParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.y;
  const long long q0 = groups.q_begin[g], q1 = groups.q_begin[g + 1];
  const long long b0 = groups.b_begin[g], b1 = groups.b_begin[g + 1];
  const long long row0 = q0 + static_cast<long long>(blockIdx.x) * kBM;
  if (row0 >= q1) return;  // uniform across the CTA, before any barrier or TMEM use
  const int n_tiles = static_cast<int>((b1 - b0 + kBN - 1) / kBN);
  const int kb = p.k_blocks;
  auto bar = [&](int i) -> uint32_t { return sbase + kOffBar + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffTmemSlot + 8);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarFull + s), 1);
      mbar_init(bar(kBarEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kBarAccFull + b), 1);
      mbar_init(bar(kBarAccEmpty + b), 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(sbase + kOffTmemSlot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kOffTmemSlot);

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      int it = 0;
      for (int t = 0; t < n_tiles && !*abort_flag; ++t) {
        for (int k = 0; k < kb; ++k, ++it) {
          const int s = it % kStages;
          if (it >= kStages &&
              !mbar_wait(bar(kBarEmpty + s), ((it / kStages) - 1) & 1, &g_merge_err)) {
            *abort_flag = 1;
            break;
          }
          const uint32_t st = sbase + kOffStage + s * kStageBytes;
          mbar_arrive_expect_tx(bar(kBarFull + s), kStageBytes);
          tma_load_2d(st, &tmap_q, bar(kBarFull + s), k * kBK, static_cast<int32_t>(row0));
          tma_load_2d(st + kABytes, &tmap_b, bar(kBarFull + s), k * kBK,
                      static_cast<int32_t>(b0 + static_cast<long long>(t) * kBN));
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc = idesc_f16(kBM, kBN, 1, 0, 0);
      int it = 0;
      bool ok = true;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int ab = t & 1;
        if (t >= 2 && !mbar_wait(bar(kBarAccEmpty + ab), ((t - 2) >> 1) & 1, &g_merge_err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + ab * kBN;
        for (int k = 0; k < kb; ++k, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(bar(kBarFull + s), (it / kStages) & 1, &g_merge_err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t st = sbase + kOffStage + s * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = smem_desc_sw128(st + kk * 32, 16, 1024);
            const uint64_t bdesc = smem_desc_sw128(st + kABytes + kk * 32, 16, 1024);
            umma_ss(d_tmem, adesc, bdesc, idesc, (k > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar(kBarEmpty + s));
        }
        if (!ok) break;
        umma_commit(bar(kBarAccFull + ab));
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    float tv[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    int ti[4] = {-1, -1, -1, -1};
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
      const int ab = t & 1;
      if (!mbar_wait(bar(kBarAccFull + ab), (t >> 1) & 1, &g_merge_err)) { ok = false; break; }
      tc_fence_after();
      const long long col0 = b0 + static_cast<long long>(t) * kBN;
      const long long remaining = b1 - col0;
      const int valid = remaining < kBN ? static_cast<int>(remaining) : kBN;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32x32b_x32(tmem + lane_off + ab * kBN + c * 32, r);
        if (c * 32 < valid) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int local = c * 32 + i;
            if (local < valid)
              topk_insert<K>(tv, ti, bf16_round(__uint_as_float(r[i])), static_cast<int>(col0 + local));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar(kBarAccEmpty + ab));
    }
    if (!ok) *abort_flag = 1;
    const long long grow = row0 + row;
    if (grow < q1) {
#pragma unroll
      for (int i = 0; i < K; ++i) {
        p.values[grow * K + i] = tv[i];
        p.indices[grow * K + i] = ti[i];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int make_rows_map(CUtensorMap* map, const void* base, long long rows, long long D, long long stride,
                  int box_rows) {
  uint64_t dims[2] = {static_cast<uint64_t>(D), static_cast<uint64_t>(rows)};
  uint64_t strides[1] = {static_cast<uint64_t>(stride) * 2};
  uint32_t box[2] = {static_cast<uint32_t>(kBK), static_cast<uint32_t>(box_rows)};
  return encode_tiled_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
}

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

using namespace vb200;

extern "C" int vb200_sim_topk(const void* query, int64_t q_row_stride, const void* basis,
                              int64_t b_row_stride, int64_t R, int64_t Nb, int64_t D, int k,
                              const int64_t* q_begin, const int64_t* b_begin, int64_t groups,
                              float* values, int64_t* indices, void* stream) {
  VB200_REQUIRE(k == 1 || k == 4, "sim_topk: k must be 1 or 4 (got %d)", k);
  VB200_REQUIRE(R >= 0 && Nb >= 0 && D > 0 && D % kBK == 0,
                "sim_topk: D must be a positive multiple of 64 (got %lld)", (long long)D);
  VB200_REQUIRE(groups >= 1, "sim_topk: groups must be >= 1");
  VB200_REQUIRE((q_begin == nullptr) == (b_begin == nullptr), "sim_topk: pass both group tables or neither");
  VB200_REQUIRE(q_begin != nullptr || groups == 1, "sim_topk: group tables required for groups > 1");
  if (R == 0) return VB200_OK;
  VB200_REQUIRE(query && basis && values && indices, "sim_topk: null pointer");
  VB200_REQUIRE(q_row_stride % 8 == 0 && b_row_stride % 8 == 0,
                "sim_topk: row strides must be multiples of 8 elements");
  std::vector<long long> qb(groups + 1), bb(groups + 1);
  if (q_begin == nullptr) {
    qb[0] = 0; qb[1] = R; bb[0] = 0; bb[1] = Nb;
  } else {
    for (int64_t g = 0; g <= groups; ++g) { qb[g] = q_begin[g]; bb[g] = b_begin[g]; }
  }
  for (int64_t g = 0; g < groups; ++g) {
    VB200_REQUIRE(qb[g] >= 0 && qb[g] <= qb[g + 1] && qb[g + 1] <= R,
                  "sim_topk: query group %lld [%lld, %lld) outside [0, %lld)", (long long)g, qb[g], qb[g + 1], (long long)R);
    VB200_REQUIRE(bb[g] >= 0 && bb[g] <= bb[g + 1] && bb[g + 1] <= Nb,
                  "sim_topk: basis group %lld [%lld, %lld) outside [0, %lld)", (long long)g, bb[g], bb[g + 1], (long long)Nb);
  }
  int rc = check_sm100();
  if (rc != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tq, tb;
  if ((rc = make_rows_map(&tq, query, R, D, q_row_stride, kBM)) != VB200_OK) return rc;
  if (Nb > 0 && (rc = make_rows_map(&tb, basis, Nb, D, b_row_stride, kBN)) != VB200_OK) return rc;
  if (Nb == 0) tb = tq;  // never read: every group then has zero basis tiles
  TopkParams prm{values, indices, k, static_cast<int>(D / kBK)};
  auto kernel = k == 1 ? sim_topk_kernel<1> : sim_topk_kernel<4>;
  VB200_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                   "cudaFuncSetAttribute");
  for (int64_t g0 = 0; g0 < groups; g0 += kMaxGroups) {
    const int64_t ng = std::min<int64_t>(kMaxGroups, groups - g0);
    GroupTable tab{};
    long long max_rows = 0;
    for (int64_t i = 0; i <= ng; ++i) {
      tab.q_begin[i] = qb[g0 + i];
      tab.b_begin[i] = bb[g0 + i];
    }
    for (int64_t i = 0; i < ng; ++i) max_rows = std::max(max_rows, tab.q_begin[i + 1] - tab.q_begin[i]);
    if (max_rows == 0) continue;
    const dim3 grid(static_cast<unsigned>((max_rows + kBM - 1) / kBM), static_cast<unsigned>(ng));
    kernel<<<grid, kThreads, kSmemBytes, st>>>(tq, tb, tab, prm);
    VB200_CHECK_LAUNCH("sim_topk_kernel");
  }
  return VB200_OK;
}
