// Merge step for B200 (sm_100a): cosine-similarity GEMM with a fused running top-k epilogue.
//
//   score[r, n] = bf16_round( sum_d query[r, d] * basis[n, d] )     (fp32 accumulation)
//   out[r]      = the k highest scores of row r (k = 1, 4 or 16), best first, ties -> lower n
//
// This is the bf16 GEMM + max(-1) of build_fastvggt_plan (vggt_omega/models/token_merging.py:
// 1100-1111) and the bf16 GEMM + topk(4) support retrieval (vggt_omega/models/sparse_convex.py:
// 264, 294, 546-547) / streaming_top4 (vggt_omega/models/sparse_convex_kernels.py:20-93, which
// rounds the accumulator to bf16 before ranking, :51-54), without writing the score matrix.
// k = 16 is the semantic shortlist of the geometry-guarded support route (sparse_convex.py:
// 263-266, 506-508: score.topk(16)).
//
// Kernel (one CTA per 128 query rows of one group, 6 warps):
//   warp 0      TMA producer: for every basis tile of tile_n rows and every 64-channel
//               k-block, the query k-block [128 x 64] and the basis k-block [tile_n x 64]
//               (128-byte swizzle), 4-stage ring.  tile_n (<= 256, a multiple of 16) is chosen
//               per launch so the tiles cover the largest basis group with little padding
//               (1029 rows: 5 x 208 instead of 5 x 256).
//   warp 1      allocates 512 TMEM columns (two 128 x tile_n fp32 accumulators, 256 apart) and
//               issues tcgen05.mma M=128 N=tile_n K=16 as a converged warp (one asm block per
//               k-block), committing each finished tile to the epilogue.
//   warps 2..5  epilogue: thread t owns query row t, reads its tile_n scores per tile from TMEM,
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
constexpr int kBN = 256;  // largest basis tile (rows); the launch picks tile_n <= kBN
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
  int tile_n;           // basis rows per tile (multiple of 16, <= kBN)
  int split;            // CTAs per query block, each over a contiguous range of basis tiles
};

// One k-block (K = 64) of the score tile: four K=16 steps, both descriptors advancing 32 bytes
// (2 units) per step, issued by one elected lane of the converged warp, then a commit.
__device__ __forceinline__ void issue_kblock(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                             uint32_t acc_first, uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, %4, 0;\n\t"
      "setp.eq.b32 pt, 0, 0;\n\t"
      "add.s64 a1, %1, 2;\n\tadd.s64 b1, %2, 2;\n\t"
      "add.s64 a2, %1, 4;\n\tadd.s64 b2, %2, 4;\n\t"
      "add.s64 a3, %1, 6;\n\tadd.s64 b3, %2, 6;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pf;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, pt;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc_first), "r"(bar)
      : "memory");
}

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

// Branch-free top-4: an order-preserving 32-bit key per (score, column).  High half: the score's
// bf16 bit pattern mapped so that unsigned order is numeric order (sign bit set for positive
// values, all bits flipped for negative ones; -0 is folded to +0 first so equal scores compare
// equal).  Low half: 65535 - column (group-local).  A larger key is a higher score or, on equal
// scores, the lower column, which is the order of the strict-> running top-k; inserting is
// then a 4-level max/min cascade with no divergent branches.  Key 0 marks an empty slot.
// (A NaN score ranks above +inf here.)
__device__ __forceinline__ uint32_t score_key(float s, int col) {
  const float z = s + 0.0f;  // -0 -> +0
  const uint32_t b = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(z))) << 16;
  const uint32_t o = b ^ (static_cast<uint32_t>(static_cast<int32_t>(b) >> 31) | 0x80000000u);
  return (o & 0xFFFF0000u) | static_cast<uint32_t>(0xFFFF - col);
}
__device__ __forceinline__ float key_score(uint32_t k) {
  const uint32_t o = k & 0xFFFF0000u;
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : (~o & 0xFFFF0000u));
}
__device__ __forceinline__ void key_insert(uint32_t (&kk)[4], uint32_t key) {
  uint32_t m;
  m = max(kk[0], key); key = min(kk[0], key); kk[0] = m;
  m = max(kk[1], key); key = min(kk[1], key); kk[1] = m;
  m = max(kk[2], key); key = min(kk[2], key); kk[2] = m;
  kk[3] = max(kk[3], key);
}
// Sixteen slots: the cascade runs only for a key above the current 16th (after the first few
// tiles almost no score is), so the common case is one compare.
__device__ __forceinline__ void key_insert(uint32_t (&kk)[16], uint32_t key) {
  if (key <= kk[15]) return;
#pragma unroll
  for (int i = 0; i < 15; ++i) {
    const uint32_t m = max(kk[i], key);
    key = min(kk[i], key);
    kk[i] = m;
  }
  kk[15] = max(kk[15], key);
}

// kKeys: top-K (K = 4 or 16) through score_key (every basis group has at most 65536 rows).
template <int K, bool kKeys>
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
  const int tile_n = p.tile_n;
  // this CTA's basis tiles [t_begin, t_begin + n_tiles) (all of them unless the search is split)
  const int n_tiles_all = static_cast<int>((b1 - b0 + tile_n - 1) / tile_n);
  const int t_begin = static_cast<int>(static_cast<long long>(n_tiles_all) * blockIdx.z / p.split);
  const int n_tiles = static_cast<int>(static_cast<long long>(n_tiles_all) * (blockIdx.z + 1) / p.split) - t_begin;
  const int kb = p.k_blocks;
  const uint32_t b_bytes = static_cast<uint32_t>(tile_n) * kBK * 2;
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
          mbar_arrive_expect_tx(bar(kBarFull + s), kABytes + b_bytes);
          tma_load_2d(st, &tmap_q, bar(kBarFull + s), k * kBK, static_cast<int32_t>(row0));
          tma_load_2d(st + kABytes, &tmap_b, bar(kBarFull + s), k * kBK,
                      static_cast<int32_t>(b0 + static_cast<long long>(t_begin + t) * tile_n));
        }
      }
    }
  } else if (warp == 1) {
    if (n_tiles > 0) {
      const uint32_t idesc = idesc_f16(kBM, tile_n, 1, 0, 0);
      const uint64_t a_desc = smem_desc_sw128(sbase + kOffStage, 16, 1024);
      const uint64_t b_desc = smem_desc_sw128(sbase + kOffStage + kABytes, 16, 1024);
      int it = 0;
      bool ok = true;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int ab = t & 1;
        if (t >= 2) ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarAccEmpty + ab), ((t - 2) >> 1) & 1, &g_merge_err));
        if (!ok) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + ab * kBN;
        for (int k = 0; k < kb; ++k, ++it) {
          const int s = it % kStages;
          ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarFull + s), (it / kStages) & 1, &g_merge_err));
          if (!ok) break;
          tc_fence_after();
          const uint64_t so = static_cast<uint64_t>(s * (kStageBytes >> 4));
          issue_kblock(d_tmem, a_desc + so, b_desc + so, idesc, k > 0 ? 1u : 0u, bar(kBarEmpty + s));
        }
        if (!ok) break;
        umma_commit_warp(bar(kBarAccFull + ab));
      }
      if (!ok && lane == 0) *abort_flag = 1;
    }
  } else {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    constexpr int KS = K < 4 ? 4 : K;  // slots (K = 1 uses the first of four)
    float tv[KS];
    int ti[KS];
    uint32_t kk[KS];
#pragma unroll
    for (int i = 0; i < KS; ++i) {
      tv[i] = -INFINITY;
      ti[i] = -1;
      kk[i] = 0u;
    }
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
      const int ab = t & 1;
      if (!mbar_wait(bar(kBarAccFull + ab), (t >> 1) & 1, &g_merge_err)) { ok = false; break; }
      tc_fence_after();
      const long long col0 = b0 + static_cast<long long>(t_begin + t) * tile_n;
      const long long remaining = b1 - col0;
      const int valid = remaining < tile_n ? static_cast<int>(remaining) : tile_n;
#pragma unroll 1
      for (int c = 0; c < tile_n / 16; ++c) {
        uint32_t r[16];
        tmem_ld32x32b_x16(tmem + lane_off + ab * kBN + c * 16, r);
        if constexpr (kKeys) {
          const int gcol = (t_begin + t) * tile_n + c * 16;  // group-local column of r[0]
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint32_t key = score_key(__uint_as_float(r[i]), gcol + i);
            key_insert(kk, c * 16 + i < valid ? key : 0u);
          }
        } else if (c * 16 < valid) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int local = c * 16 + i;
            if (local < valid)
              topk_insert<K>(tv, ti, bf16_round(__uint_as_float(r[i])), static_cast<int>(col0 + local));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar(kBarAccEmpty + ab));
    }
    if (!ok) *abort_flag = 1;
    bool piece_written = false;
    if constexpr (kKeys) {
      if (K == 4 && p.split > 1) {
        // split search: this piece's four keys go to slot z of the row's 48 output bytes
        // (slot 0: the row of `values`, slots 1-2: the halves of the row of `indices`);
        // topk_merge_kernel combines the slots and writes the final row
        const long long grow = row0 + row;
        if (grow < q1) {
          uint4* slot = blockIdx.z == 0 ? reinterpret_cast<uint4*>(p.values) + grow
                                        : reinterpret_cast<uint4*>(p.indices) + 2 * grow + (blockIdx.z - 1);
          *slot = make_uint4(kk[0], kk[1], kk[2], kk[KS - 1]);
        }
        piece_written = true;
      }
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        tv[i] = kk[i] ? key_score(kk[i]) : -INFINITY;
        ti[i] = kk[i] ? static_cast<int>(b0 + (0xFFFF - static_cast<int>(kk[i] & 0xFFFFu))) : -1;
      }
    }
    const long long grow = row0 + row;
    if (grow < q1 && !piece_written) {
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

// Combines the per-piece top-4 keys of a split search (see sim_topk_kernel): one thread per
// query row inserts every piece's keys into one running top-4 (the keys' order is the
// search's order, so the result equals the unsplit search) and writes values and indices.
__global__ void topk_merge_kernel(const __grid_constant__ GroupTable groups, float* values, int64_t* indices,
                                  int split) {
  const int g = blockIdx.y;
  const long long q0 = groups.q_begin[g], q1 = groups.q_begin[g + 1];
  const long long b0 = groups.b_begin[g];
  const long long r = q0 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= q1) return;
  uint4 sl[3];
  sl[0] = reinterpret_cast<const uint4*>(values)[r];
  if (split > 1) sl[1] = reinterpret_cast<const uint4*>(indices)[2 * r];
  if (split > 2) sl[2] = reinterpret_cast<const uint4*>(indices)[2 * r + 1];
  uint32_t kk[4] = {0u, 0u, 0u, 0u};
  for (int z = 0; z < split; ++z) {
    key_insert(kk, sl[z].x);
    key_insert(kk, sl[z].y);
    key_insert(kk, sl[z].z);
    key_insert(kk, sl[z].w);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    values[r * 4 + i] = kk[i] ? key_score(kk[i]) : -INFINITY;
    indices[r * 4 + i] = kk[i] ? static_cast<int64_t>(b0 + (0xFFFF - static_cast<int>(kk[i] & 0xFFFFu))) : -1;
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

int sm_count_cached() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev < 64) cached[dev] = n;
  return n;
}

// Pieces per query block for a launch of `ctas` CTAs over n_tiles basis tiles, one CTA per SM:
// time ~ waves x (tiles per piece + ramp), plus about one tile for the merge launch when split;
// at most 3 pieces (their keys fill the 48 output bytes of a row).
int choose_split(long long ctas, int n_tiles, int sms) {
  if (sms <= 0 || ctas <= 0) return 1;
  int best = 1;
  double best_t = 0.0;
  for (int s = 1; s <= 3 && s <= n_tiles; ++s) {
    const long long waves = (ctas * s + sms - 1) / sms;
    const double t = static_cast<double>(waves) * ((n_tiles + s - 1) / s + 0.5) + (s > 1 ? 1.0 : 0.0);
    if (s == 1 || t < best_t - 1e-9) {
      best_t = t;
      best = s;
    }
  }
  return best;
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

extern "C" int vb200_sim_topk_split(int64_t ctas, int n_tiles, int sms) {
  return choose_split(ctas, n_tiles, sms);
}

extern "C" int vb200_sim_topk(const void* query, int64_t q_row_stride, const void* basis,
                              int64_t b_row_stride, int64_t R, int64_t Nb, int64_t D, int k,
                              const int64_t* q_begin, const int64_t* b_begin, int64_t groups,
                              float* values, int64_t* indices, void* stream) {
  VB200_REQUIRE(k == 1 || k == 4 || k == 16, "sim_topk: k must be 1, 4 or 16 (got %d)", k);
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
  // basis tile: the fewest tiles of <= kBN rows that cover the largest group, each as narrow as
  // possible (multiple of 16)
  long long max_nb = 0;
  for (int64_t g = 0; g < groups; ++g) max_nb = std::max(max_nb, bb[g + 1] - bb[g]);
  const long long n_tiles_max = std::max(1ll, (max_nb + kBN - 1) / kBN);
  const int tile_n = static_cast<int>(std::max(16ll, (((max_nb + n_tiles_max - 1) / n_tiles_max) + 15) / 16 * 16));
  CUtensorMap tq, tb;
  if ((rc = make_rows_map(&tq, query, R, D, q_row_stride, kBM)) != VB200_OK) return rc;
  if (Nb > 0 && (rc = make_rows_map(&tb, basis, Nb, D, b_row_stride, tile_n)) != VB200_OK) return rc;
  if (Nb == 0) tb = tq;  // never read: every group then has zero basis tiles
  VB200_REQUIRE(k != 16 || max_nb <= 65536, "sim_topk: k = 16 needs basis groups of at most 65536 rows");
  const bool keys4 = k == 4 && max_nb <= 65536;
  TopkParams prm{values, indices, k, static_cast<int>(D / kBK), tile_n, 1};
  auto kernel = k == 1 ? sim_topk_kernel<1, false>
                       : k == 16 ? sim_topk_kernel<16, true>
                                 : (keys4 ? sim_topk_kernel<4, true> : sim_topk_kernel<4, false>);
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
    const long long ctas = ((max_rows + kBM - 1) / kBM) * ng;
    // the split search keeps its per-piece keys in the 16-byte aligned output rows
    const bool aligned = (reinterpret_cast<uintptr_t>(values) & 15u) == 0 && (reinterpret_cast<uintptr_t>(indices) & 15u) == 0;
    prm.split = keys4 && aligned ? choose_split(ctas, static_cast<int>(n_tiles_max), sm_count_cached()) : 1;
    const dim3 grid(static_cast<unsigned>((max_rows + kBM - 1) / kBM), static_cast<unsigned>(ng),
                    static_cast<unsigned>(prm.split));
    kernel<<<grid, kThreads, kSmemBytes, st>>>(tq, tb, tab, prm);
    VB200_CHECK_LAUNCH("sim_topk_kernel");
    if (prm.split > 1) {
      const dim3 mgrid(static_cast<unsigned>((max_rows + 127) / 128), static_cast<unsigned>(ng));
      topk_merge_kernel<<<mgrid, 128, 0, st>>>(tab, values, indices, prm.split);
      VB200_CHECK_LAUNCH("topk_merge_kernel");
    }
  }
  return VB200_OK;
}
