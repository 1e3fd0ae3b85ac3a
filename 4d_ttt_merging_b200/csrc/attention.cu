// Mass-bias attention forward for B200 (sm_100a):
//   O = softmax(Q K^T / sqrt(64) + log m) V      per (batch, head), head_dim 64.
//
// Reference behaviour (vggt_omega/models/mass_bias_attention.py:17-82, :85-129): the per-key
// bias is log(mass) rounded to the input dtype, added in the log2 domain
// (logit * log2e/sqrt(d) + bias * log2e), online softmax with fp32 running max / sum / output,
// probabilities rounded to the value dtype before the PV product, output divided by the
// running sum and written in the input dtype.
//
// Kernel design: one CTA per 256 query rows (two 128-row tiles) and (batch, head), 20 warps,
// one CTA per SM; see mass_bias_attention_tc_kernel.  Shared-memory tiles use the 128-byte
// swizzle written by TMA; the UMMA descriptors describe the same layout (K-major for Q and K,
// MN-major for V).  No TMA multicast is used.
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "host_common.h"

namespace vb200 {
namespace {

static __device__ unsigned g_attn_err;

constexpr int kBM = 128;  // query rows per tile (one TMEM lane per row)
constexpr int kQT = 2;    // query tiles per CTA, two softmax warpgroups each
constexpr int kBN = 128;  // keys per tile
constexpr int kHD = 64;   // head dim
constexpr int kStages = 4;
constexpr int kTileBytes = kBM * kHD * 2;  // 16 KB: one Q, K or V tile
// The per-key bias rides in the QK product: an extra K=16 chunk holds 1 in column 0 of every
// query row (kOffQx, written once per CTA) and 8 * bias_j in column 0 of key row j (kx tiles
// prepared in global memory), so S' = q.k + 8 bias_j and the log2-domain logit is
// S' * log2(e)/8 (8 = sqrt(64); multiplying a 16-bit value by 8 is exact).  The chunk uses the
// no-swizzle K-major layout: [16 row groups][2 K halves][8 rows][16 bytes].
constexpr int kKxBytes = 4096;
constexpr int kStageStride = 36864;        // K, V (16 KB each) + extra K chunk (4 KB)
constexpr int kHalfKeys = kBN / 2;        // key columns per softmax warpgroup
constexpr int kSoftmaxWarps = 16;         // four softmax warpgroups: 2 query tiles x 2 column halves
constexpr int kWarpProducer = kSoftmaxWarps;
constexpr int kWarpMma = kSoftmaxWarps + 1;
constexpr int kThreads = (kSoftmaxWarps + 4) * 32;  // + one warpgroup for the producer and MMA warps
// Register split (setmaxnreg): the block launches with kLaunchRegs per thread; the producer
// warpgroup drops to kRegsLow and the softmax warpgroups rise to kRegsHigh.  The shares add up
// exactly to the launch total, which the host checks before every launch.
constexpr int kLaunchRegs = 96;
constexpr int kRegsHigh = 104;
constexpr int kRegsLow = 64;
static_assert(kSoftmaxWarps * 32 * kRegsHigh + 128 * kRegsLow == kThreads * kLaunchRegs, "register split");
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // lazy rescale: P stays <= 2^8
// Of every 8 exponent pairs, how many are computed on the FMA pipe (exp2_poly2) instead of
// MUFU (16 exponentials per clock per SM).  Measured on the config-2 attention (split launch):
// 1: 399 us, 2: 413 us, 3: 430 us; with the earlier per-tile max exchange 2 of 8 had been
// fastest (0: 459, 1: 414, 2: 407, 3: 457 us).  Beyond that the extra instructions take issue
// slots from the MMA warp.
constexpr int kPolyPairs = 1;
constexpr int kNamedBarPair = 1;  // named barriers 1, 2: the two warpgroups of query tile 0, 1
constexpr int kNamedBarSoftmax = 3;  // all softmax warps (the split epilogue)
// Key-range split of the last partial wave: at most this many pieces per (query block, head).
constexpr int kMaxSplit = 4;

// Shared-memory layout (offsets from a 1024-byte aligned base).
constexpr int kOffQ = 0;                                  // kQT tiles
constexpr int kOffQx = kOffQ + kQT * kTileBytes;          // constant extra Q chunk
constexpr int kOffStage = kOffQx + kKxBytes;              // kStages x {K, V, extra K chunk}
constexpr int kOffBar = kOffStage + kStages * kStageStride;
constexpr int kBarQFull = 0;
constexpr int kBarKVFull = 1;
constexpr int kBarKVEmpty = kBarKVFull + kStages;
constexpr int kBarSFull = kBarKVEmpty + kStages;
constexpr int kBarPFull = kBarSFull + kQT;
constexpr int kBarODone = kBarPFull + kQT;
constexpr int kBarSFree = kBarODone + kQT;
constexpr int kNumBars = kBarSFree + kQT;
constexpr int kOffRed = kOffBar + kNumBars * 8;  // [tile][half][parity][row] fp32 slots (final sums)
constexpr int kOffTmemSlot = kOffRed + kQT * 2 * 2 * kBM * 4;
constexpr int kSmemUsed = kOffTmemSlot + 16;
constexpr int kSmemBytes = kSmemUsed + 1024;  // slack for aligning the dynamic base
constexpr uint32_t kTmemCols = 512;           // S_t at 128t, P_t at 256 + 64t, O_t at 384 + 64t
constexpr uint32_t kTmemP = 256;
constexpr uint32_t kTmemO = 384;
static_assert(kStageStride >= 2 * kTileBytes + kKxBytes && kStageStride % 1024 == 0, "stage layout");

// Work items are (query block, batch*head) pairs, numbered query block fastest.  CTA c < n_full
// runs item c over all key tiles.  When the items do not fill whole waves of the GPU, the
// remaining items (n_full, n_full + 1, ...) are each split into `split` key ranges run by
// `split` CTAs; every piece writes its unnormalised O, running max and sum to o_part / ml_part,
// and the piece that finishes last (counted in counters[item - n_full]) merges all pieces in
// piece order and writes the output.
struct AttnParams {
  const uint8_t* kx;  // [n_tiles][kKxBytes] extra K chunks (8 * bias, masked past Nk)
  void* out;
  long long o_sb, o_sh, o_sn;  // element strides
  int H, Nq, Nk, n_tiles;
  int qblocks, n_full, split;
  float* o_part;          // [tail items][split][kQT][kBM][kHD]
  float2* ml_part;        // [tail items][split][kQT][kBM]: (running max, running sum)
  unsigned* counters;     // [tail items], zeroed by prepare_kx_kernel before every launch
  float scale_log2;  // log2(e) / sqrt(64)
};

// MMA groups, each one asm block executed by the whole MMA warp: elect.sync once, then the
// elected lane issues every MMA of the group and the commit(s).  The MMA warp shares its SM
// sub-partition with four busy softmax warps and only gets a small share of the issue slots,
// so the instruction count per MMA (not the tensor pipe) sets the pace: one descriptor add
// and one tcgen05.mma per step keeps the stream close to the pipe rate (measured: 1.8x
// faster than one helper call per MMA under full contention).
//
// S_t = Q_t K^T over head_dim 64 (four K=16 steps; both descriptors' start addresses advance by
// 32 bytes = 2 units per step) + the bias chunk (xa, xb); the first step overwrites.
__device__ __forceinline__ void issue_qk_group(uint32_t d, uint64_t a, uint64_t b, uint64_t xa, uint64_t xb,
                                               uint32_t idesc, uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, 0, 0;\n\t"
      "setp.eq.b32 pt, 0, 0;\n\t"
      "add.s64 a1, %1, 2;\n\tadd.s64 b1, %2, 2;\n\t"
      "add.s64 a2, %1, 4;\n\tadd.s64 b2, %2, 4;\n\t"
      "add.s64 a3, %1, 6;\n\tadd.s64 b3, %2, 6;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %5, pf;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %5, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %5, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %5, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %4, %5, pt;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t}" ::"r"(d),
      "l"(a), "l"(b), "l"(xa), "l"(xb), "r"(idesc), "r"(bar)
      : "memory");
}
// O_t (+)= P_t V over 128 keys: eight K=16 steps; P_t in TMEM (A advances 8 columns = 16
// packed keys per step), V MN-major (B advances 2048 bytes = 128 units per step).  Commits to
// `bar`, and also to `bar2` when use_bar2 is nonzero.
__device__ __forceinline__ void issue_pv_group(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                               uint32_t acc_first, uint32_t bar, uint32_t bar2,
                                               uint32_t use_bar2) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt, p2;\n\t.reg .b64 b1, b2, b3, b4, b5, b6, b7;\n\t"
      ".reg .b32 a1, a2, a3, a4, a5, a6, a7;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, %4, 0;\n\t"
      "setp.eq.b32 pt, 0, 0;\n\t"
      "setp.ne.and.b32 p2, %7, 0, e;\n\t"
      "add.s32 a1, %1, 8;\n\tadd.s64 b1, %2, 128;\n\t"
      "add.s32 a2, %1, 16;\n\tadd.s64 b2, %2, 256;\n\t"
      "add.s32 a3, %1, 24;\n\tadd.s64 b3, %2, 384;\n\t"
      "add.s32 a4, %1, 32;\n\tadd.s64 b4, %2, 512;\n\t"
      "add.s32 a5, %1, 40;\n\tadd.s64 b5, %2, 640;\n\t"
      "add.s32 a6, %1, 48;\n\tadd.s64 b6, %2, 768;\n\t"
      "add.s32 a7, %1, 56;\n\tadd.s64 b7, %2, 896;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, pf;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], b4, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a5], b5, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a6], b6, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a7], b7, %3, pt;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t"
      "@p2 tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc_first), "r"(bar), "r"(bar2), "r"(use_bar2)
      : "memory");
}

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }

// Mass-bias attention, two query tiles per CTA:
//   warps 0-15   four softmax warpgroups; warpgroup 2t+h owns query tile t (thread = query row =
//                TMEM lane) and key columns [64h, 64h+64) of every S tile.  Each half also
//                reads the other half's 64 columns for the row max, so both compute the same
//                tile max and take the same rescale decisions without any exchange: they share
//                one running max and one O accumulator (measured 2% faster than exchanging the
//                half maxima through shared memory behind a named barrier per tile).  Four
//                softmax warps per SM sub-partition keep the exponential unit busy while other
//                warps load S, reduce maxima or store P.
//   warp 16      TMA producer: both Q tiles once; K_j, V_j and the bias chunk of key tile j
//                into a 4-stage ring.
//   warp 17      TMEM allocation and the MMA stream (converged warp, one elected lane issues).
//                Per key tile j and query tile t it issues QK_t(j+1) as soon as both halves have
//                read S_t(j), then PV_t(j) once P_t(j) is written (QK_0 PV_0 QK_1 PV_1), so
//                the next scores are computed underneath the current softmax.
//   warps 18-19  idle (they complete the warpgroup that setmaxnreg.dec applies to).
// TMEM (512 columns): S_t in [128t, 128t+128), P_t as packed 16-bit values in
// [256+64t, 256+64t+64) (the A operand of the TS-MMA), O_t accumulating in [384+64t, ...).
// The running max is lazy: O_t is rescaled (in TMEM, each half rescaling its 32 columns) only
// when a row's max grows by more than 2^8; otherwise P is formed against the stale max, which
// the final division by the matching running sum cancels exactly.
template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    mass_bias_attention_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                                  const __grid_constant__ CUtensorMap tmap_k,
                                  const __grid_constant__ CUtensorMap tmap_v, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // this CTA's work item and key-tile range [kt0, kt0 + n_tiles)
  const int cta = static_cast<int>(blockIdx.x);
  const bool piece_cta = cta >= p.n_full;
  int item = cta, piece = 0, kt0 = 0, kt1 = p.n_tiles;
  if (piece_cta) {
    const int k = (cta - p.n_full) / p.split;
    piece = cta - p.n_full - k * p.split;
    item = p.n_full + k;
    kt0 = static_cast<int>(static_cast<long long>(piece) * p.n_tiles / p.split);
    kt1 = static_cast<int>(static_cast<long long>(piece + 1) * p.n_tiles / p.split);
  }
  const int q_block = item % p.qblocks;  // kQT * kBM query rows
  const int bh = item / p.qblocks;
  const int batch = bh / p.H;
  const int head = bh - batch * p.H;
  const int n_tiles = kt1 - kt0;
  auto bar = [=](int i) -> uint32_t { return sbase + kOffBar + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffTmemSlot + 8);

  if (threadIdx.x == 0) {
    mbar_init(bar(kBarQFull), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarKVFull + s), 1);
      mbar_init(bar(kBarKVEmpty + s), 1);
    }
    for (int t = 0; t < kQT; ++t) {
      mbar_init(bar(kBarSFull + t), 1);
      mbar_init(bar(kBarPFull + t), 2 * 128);
      mbar_init(bar(kBarODone + t), 1);
      mbar_init(bar(kBarSFree + t), 2 * 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < kKxBytes / 16) {
    // extra Q chunk: 1 in column 0 of every row (half 0 of each 8-row group), 0 elsewhere
    const int half = (threadIdx.x >> 3) & 1;
    const uint32_t one = kBF16 ? 0x3F80u : 0x3C00u;  // 1.0 in bf16 / fp16
    *reinterpret_cast<uint4*>(smem + kOffQx + 16 * threadIdx.x) = make_uint4(half == 0 ? one : 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();  // generic-proxy writes become visible to the tensor core
  }
  if (warp == kWarpProducer && lane == 0) {
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
  }
  if (warp == kWarpMma) {
    tmem_alloc(sbase + kOffTmemSlot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kOffTmemSlot);

  // Each role's code is dominated by its own setmaxnreg (no merge point in between), so the
  // register allocator gives every branch the budget its warpgroup actually holds.
  if (warp >= kSoftmaxWarps) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
  if (warp == kWarpProducer) {
    // ------------------------------- producer -------------------------------
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(bar(kBarQFull), kQT * kTileBytes);
      for (int t = 0; t < kQT; ++t)  // an empty query tile loads zeros (rows past Nq)
        tma_load_4d(sbase + kOffQ + t * kTileBytes, &tmap_q, bar(kBarQFull), 0, (q_block * kQT + t) * kBM,
                    head, batch);
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j % kStages;
        if (*abort_flag) { ok = false; break; }
        if (j >= kStages && !mbar_wait(bar(kBarKVEmpty + s), ((j / kStages) - 1) & 1, &g_attn_err)) {
          ok = false;
          break;
        }
        const uint32_t st = sbase + kOffStage + s * kStageStride;
        mbar_arrive_expect_tx(bar(kBarKVFull + s), 2 * kTileBytes + kKxBytes);
        tma_load_4d(st, &tmap_k, bar(kBarKVFull + s), 0, (kt0 + j) * kBN, head, batch);
        tma_load_4d(st + kTileBytes, &tmap_v, bar(kBarKVFull + s), 0, (kt0 + j) * kBN, head, batch);
        bulk_load(st + 2 * kTileBytes, p.kx + static_cast<size_t>(kt0 + j) * kKxBytes, kKxBytes,
                  bar(kBarKVFull + s));
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == kWarpMma) {
    // ------------------------------- MMA issuer -------------------------------
    // The whole warp runs this loop (every lane waits on the barriers) and one elected lane
    // issues each tcgen05 operation.  Descriptors are built once for Q tile 0 / stage 0; the
    // start-address field counts 16-byte units, so a byte offset b is added as b >> 4 (shared
    // addresses stay below 256 KB, so the 14-bit field never carries).
    constexpr uint32_t idesc_qk = idesc_f16(kBM, kBN, kBF16 ? 1 : 0, 0, 0);
    constexpr uint32_t idesc_pv = idesc_f16(kBM, kHD, kBF16 ? 1 : 0, 0, 1);
    const uint64_t q_desc = smem_desc_sw128(sbase + kOffQ, 16, 1024);
    const uint64_t k_desc = smem_desc_sw128(sbase + kOffStage, 16, 1024);
    // V is MN-major: key rows of 128 bytes, so a K-step of 16 keys spans two 1024-byte atoms
    const uint64_t v_desc = smem_desc_sw128(sbase + kOffStage + kTileBytes, 16384, 1024);
    // the bias chunk (no swizzle: LBO 128 B along K, SBO 256 B between 8-row groups)
    const uint64_t qx_desc = smem_desc_noswz(sbase + kOffQx, 128, 256);
    const uint64_t kx_desc = smem_desc_noswz(sbase + kOffStage + 2 * kTileBytes, 128, 256);
    // S_t = Q_t K_j^T + 1 * (8 bias_j)
    auto issue_qk = [=](int t, int j) {
      const uint64_t so = static_cast<uint64_t>((j % kStages) * (kStageStride >> 4));
      issue_qk_group(tmem + t * 128, q_desc + t * (kTileBytes >> 4), k_desc + so, qx_desc, kx_desc + so, idesc_qk,
                     bar(kBarSFull + t));
    };
    // O_t += P_t V_j (P_t from TMEM); the CTA's last query tile's group also frees the K/V stage
    // the last block of a ragged Nq may leave query tile 1 empty: its MMAs are skipped
    const bool single_qt = (q_block * kQT + 1) * kBM >= p.Nq;
    auto issue_pv = [=](int t, int j) {
      const uint64_t so = static_cast<uint64_t>((j % kStages) * (kStageStride >> 4));
      issue_pv_group(tmem + kTmemO + t * kHD, tmem + kTmemP + t * kHD, v_desc + so, idesc_pv, j > 0 ? 1u : 0u,
                     bar(kBarODone + t), bar(kBarKVEmpty + j % kStages), (t == kQT - 1 || single_qt) ? 1u : 0u);
    };
    auto wait_all = [&](int b, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, &g_attn_err));
    };
    bool ok = wait_all(kBarQFull, 0) && wait_all(kBarKVFull + 0, 0);
    if (ok) {
      tc_fence_after();
      for (int t = 0; t < kQT; ++t)
        if (t == 0 || !single_qt) issue_qk(t, 0);
    }
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
      if (j + 1 < n_tiles) ok = wait_all(kBarKVFull + (j + 1) % kStages, ((j + 1) / kStages) & 1);
      // Per query tile: the next scores as soon as S_t(j) is in registers, then O_t += P_t V_j.
      // Tile by tile (QK_0, PV_0, QK_1, PV_1) measured 2-7% faster than both QKs first.
      for (int t = 0; t < kQT && ok; ++t) {
        if (t > 0 && single_qt) break;
        if (j + 1 < n_tiles) {
          ok = wait_all(kBarSFree + t, j & 1);
          if (!ok) break;
          tc_fence_after();
          issue_qk(t, j + 1);
        }
        ok = wait_all(kBarPFull + t, j & 1);
        if (!ok) break;
        tc_fence_after();
        issue_pv(t, j);
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ------------------------------- softmax warpgroups -------------------------------
    // Warpgroup g = 2t + h owns query tile t and key columns [64h, 64h + 64) of every S tile;
    // its partner (same t, other h) owns the other 64 columns of the same rows.
    const int g = warp >> 2;
    const int t = g >> 1;
    const int h = g & 1;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + t * 128 + h * kHalfKeys;
    const uint32_t s_other = tmem + lane_off + t * 128 + (1 - h) * kHalfKeys;
    const uint32_t p_addr = tmem + lane_off + kTmemP + t * kHD + h * (kHalfKeys / 2);
    const uint32_t o_addr = tmem + lane_off + kTmemO + t * kHD + h * (kHD / 2);
    float* red_mine = reinterpret_cast<float*>(smem + kOffRed) + ((t * 2 + h) * 2) * kBM + row;
    const float* red_other = reinterpret_cast<const float*>(smem + kOffRed) + ((t * 2 + (1 - h)) * 2) * kBM + row;
    const int pair_bar = kNamedBarPair + t;
    const float scale = p.scale_log2;
    const uint64_t scale2 = pk2(scale, scale);
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    // an empty query tile (rows past Nq only) skips everything but the barriers
    const bool active = t == 0 || (q_block * kQT + 1) * kBM < p.Nq;

    for (int j = 0; j < (active ? n_tiles : 0); ++j) {
      ok = ok && !*abort_flag;
      if (ok) ok = mbar_wait(bar(kBarSFull + t), j & 1, &g_attn_err);
      ok = __all_sync(0xffffffffu, ok);  // warp-uniform before warp-collective TMEM access
      uint32_t r[kHalfKeys];
      float mx = -INFINITY;
      if (ok) {
        tc_fence_after();
        tmem_ld32x32b_x32_nowait(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32x32b_x32_nowait(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_wait_ld();
        reg_fence32(*reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        reg_fence32(*reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        float mxa = -INFINITY, mxb = -INFINITY, mxc = -INFINITY, mxd = -INFINITY;
        // the partner half's 64 columns, for the max only (16 at a time)
#pragma unroll
        for (int c = 0; c < kHalfKeys; c += 16) {
          uint32_t pr[16];
          tmem_ld32x32b_x16(s_other + c, pr);
#pragma unroll
          for (int i = 0; i < 16; i += 8) {
            mxa = fmax3(mxa, u2f(pr[i + 0]), u2f(pr[i + 1]));
            mxb = fmax3(mxb, u2f(pr[i + 2]), u2f(pr[i + 3]));
            mxc = fmax3(mxc, u2f(pr[i + 4]), u2f(pr[i + 5]));
            mxd = fmax3(mxd, u2f(pr[i + 6]), u2f(pr[i + 7]));
          }
        }
        tc_fence_before();
        mbar_arrive(bar(kBarSFree + t));  // S_t(j) is no longer needed by this warp
#pragma unroll
        for (int i = 0; i < kHalfKeys; i += 8) {
          mxa = fmax3(mxa, u2f(r[i + 0]), u2f(r[i + 1]));
          mxb = fmax3(mxb, u2f(r[i + 2]), u2f(r[i + 3]));
          mxc = fmax3(mxc, u2f(r[i + 4]), u2f(r[i + 5]));
          mxd = fmax3(mxd, u2f(r[i + 6]), u2f(r[i + 7]));
        }
        mx = fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd));
      }
      if (ok) {
        // Lazy running max: move it (and rescale O_t, l) only when the row max grows by more
        // than kRescaleThreshold, so P = 2^(S' * scale - m) stays <= 2^kRescaleThreshold.
        const float m_new = fmaxf(m_run, mx * scale);
        const bool need = __any_sync(0xffffffffu, m_new > m_run + kRescaleThreshold);  // true on the first tile
        const float m_tgt = (m_new > m_run + kRescaleThreshold) ? m_new : m_run;
        const float alpha = ex2_approx(m_run - m_tgt);  // 0 on the first tile, 1 if unchanged
        const float m_use = (m_tgt == -INFINITY) ? 0.f : m_tgt;
        // P packed in place: r[i] <- (p[2i], p[2i+1]).  kPolyPairs of every 8 pairs use the
        // FMA-pipe exponential instead of MUFU.
        const uint64_t neg_m2 = pk2(-m_use, -m_use);
        uint64_t ls0 = pk2(0.f, 0.f), ls1 = pk2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < kHalfKeys / 2; ++i) {
          float e0, e1, p0, p1;
          upk2(ffma2(pk2(u2f(r[2 * i]), u2f(r[2 * i + 1])), scale2, neg_m2), e0, e1);
          if ((i & 7) < kPolyPairs) {
            exp2_poly2(e0, e1, p0, p1);
          } else {
            p0 = ex2_approx(e0);
            p1 = ex2_approx(e1);
          }
          if (i & 1) ls1 = fadd2(ls1, pk2(p0, p1));
          else ls0 = fadd2(ls0, pk2(p0, p1));
          r[i] = kBF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
        }
        float a0, a1, b0, b1;
        upk2(ls0, a0, a1);
        upk2(ls1, b0, b1);
        l_run = l_run * alpha + ((a0 + a1) + (b0 + b1));
        m_run = m_tgt;
        if (j > 0) {
          // PV_t(j-1) must be complete before P_t is overwritten or O_t is rescaled
          ok = mbar_wait(bar(kBarODone + t), (j - 1) & 1, &g_attn_err);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) tc_fence_after();
          if (ok && need) {
#pragma unroll
            for (int c = 0; c < kHD / 2; c += 16) {  // this warpgroup's 32 columns of O_t
              uint32_t o[16];
              tmem_ld32x32b_x16(o_addr + c, o);
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = f2u(u2f(o[i]) * alpha);
              tmem_st32x32b_x16(o_addr + c, o);
            }
          }
        }
        if (ok) {
          tmem_st32x32b_x32(p_addr, *reinterpret_cast<const uint32_t(*)[32]>(&r[0]));
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(bar(kBarPFull + t));
        }
      }
    }

    // Both halves' running sums share one scale: O_t / (l_half0 + l_half1).
    red_mine[(n_tiles & 1) * kBM] = l_run;
    named_bar_sync(pair_bar, 256);
    const float l_tot = l_run + red_other[(n_tiles & 1) * kBM];
    if (ok && active) {
      ok = mbar_wait(bar(kBarODone + t), (n_tiles - 1) & 1, &g_attn_err);
      ok = __all_sync(0xffffffffu, ok);
    }
    uint32_t o[kHD / 2];
    if (ok && active) {
      tc_fence_after();
      tmem_ld32x32b_x32_nowait(o_addr, o);
      tmem_wait_ld();
      reg_fence32(o);
    }
    const int grow = (q_block * kQT + t) * kBM + row;
    const long long orow_off = batch * p.o_sb + head * p.o_sh + static_cast<long long>(grow) * p.o_sn + h * (kHD / 2);
    if (!piece_cta) {
      if (ok && grow < p.Nq) {
        const float inv = 1.f / l_tot;
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + 2 * orow_off;
#pragma unroll
        for (int c = 0; c < kHD / 16; ++c) {
          uint4 w;
          uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float a = u2f(o[c * 8 + 2 * i]) * inv, b2 = u2f(o[c * 8 + 2 * i + 1]) * inv;
            wp[i] = kBF16 ? pack_bf16x2(a, b2) : pack_f16x2(a, b2);
          }
          *reinterpret_cast<uint4*>(orow + c * 16) = w;
        }
      }
    } else {
      // One key range of a split item: publish (O, m, l) of this piece, then the piece that
      // arrives last merges all pieces in piece order (deterministic for any arrival order).
      const long long slot0 = static_cast<long long>(item - p.n_full) * p.split;
      const long long rowi = (slot0 + piece) * kQT * kBM + t * kBM + row;  // this piece's row record
      if (ok && active) {
        float4* dst = reinterpret_cast<float4*>(p.o_part + rowi * kHD + h * (kHD / 2));
#pragma unroll
        for (int i = 0; i < kHD / 8; ++i)
          dst[i] = make_float4(u2f(o[4 * i]), u2f(o[4 * i + 1]), u2f(o[4 * i + 2]), u2f(o[4 * i + 3]));
        if (h == 0) p.ml_part[rowi] = make_float2(m_run, l_tot);
      }
      __threadfence();
      named_bar_sync(kNamedBarSoftmax, kSoftmaxWarps * 32);
      volatile int* last_flag = abort_flag + 1;
      if (threadIdx.x == 0) *last_flag = atomicAdd(p.counters + (item - p.n_full), 1u) == static_cast<unsigned>(p.split - 1);
      named_bar_sync(kNamedBarSoftmax, kSoftmaxWarps * 32);
      if (*last_flag && ok && grow < p.Nq) {
        __threadfence();
        const long long stride = static_cast<long long>(kQT) * kBM;  // row records between pieces
        const long long row0 = slot0 * stride + t * kBM + row;       // piece 0's record of this row
        // Loads are unrolled over the pieces so that each group goes out together (one L2
        // round trip per group instead of one per piece).
        float w[kMaxSplit];
        float m_star = -INFINITY;
#pragma unroll
        for (int q = 0; q < kMaxSplit; ++q) {
          w[q] = 0.f;
          if (q < p.split) {
            const float2 ml = __ldcg(&p.ml_part[row0 + q * stride]);
            w[q] = ml.x;  // running max for now
            m_star = fmaxf(m_star, ml.x);
          }
        }
        float l_sum = 0.f;
#pragma unroll
        for (int q = 0; q < kMaxSplit; ++q) {
          if (q < p.split) {
            w[q] = exp2f(w[q] - m_star);
            l_sum = fmaf(w[q], __ldcg(&p.ml_part[row0 + q * stride]).y, l_sum);
          }
        }
        const float inv = 1.f / l_sum;
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + 2 * orow_off;
#pragma unroll 1
        for (int c = 0; c < kHD / 2; c += 8) {  // 8 output columns at a time
          float4 x[kMaxSplit][2];
#pragma unroll
          for (int q = 0; q < kMaxSplit; ++q) {
            if (q < p.split) {
              const float4* src = reinterpret_cast<const float4*>(p.o_part + (row0 + q * stride) * kHD + h * (kHD / 2) + c);
              x[q][0] = __ldcg(src);
              x[q][1] = __ldcg(src + 1);
            }
          }
          float acc[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
          for (int q = 0; q < kMaxSplit; ++q) {
            if (q < p.split) {
              acc[0] = fmaf(w[q], x[q][0].x, acc[0]);
              acc[1] = fmaf(w[q], x[q][0].y, acc[1]);
              acc[2] = fmaf(w[q], x[q][0].z, acc[2]);
              acc[3] = fmaf(w[q], x[q][0].w, acc[3]);
              acc[4] = fmaf(w[q], x[q][1].x, acc[4]);
              acc[5] = fmaf(w[q], x[q][1].y, acc[5]);
              acc[6] = fmaf(w[q], x[q][1].z, acc[6]);
              acc[7] = fmaf(w[q], x[q][1].w, acc[7]);
            }
          }
          uint4 wv;
          uint32_t* wp = reinterpret_cast<uint32_t*>(&wv);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float a = acc[2 * i] * inv, b2 = acc[2 * i + 1] * inv;
            wp[i] = kBF16 ? pack_bf16x2(a, b2) : pack_f16x2(a, b2);
          }
          *reinterpret_cast<uint4*>(orow + 2 * c) = wv;
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Padded log2-domain bias: bias[j] = float(round_to_dtype(log_mass[j])) * log2(e) for j < Nk,
// 0 when no bias is given, -inf for the padding up to a whole key tile.
template <typename TB, typename TQ>
__global__ void prepare_bias_kernel(const TB* log_mass, float* bias, int Nk, int padded) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= padded) return;
  float v = -INFINITY;
  if (j < Nk) {
    if (log_mass == nullptr) {
      v = 0.f;
    } else {
      const float lm = to_f32<TB>(log_mass[j]);
      v = to_f32<TQ>(from_f32<TQ>(lm)) * kLog2e;
    }
  }
  bias[j] = v;
}

// Extra K chunks of the tensor-core path, one 4 KB tile per 128 keys in the no-swizzle K-major
// layout [16 row groups][2 K halves][8 rows][8 elements]: column 0 of key row j holds
// 8 * round_to_dtype(log_mass[j]) (0 without a bias), keys past Nk hold a large negative value
// (their exponential underflows to 0), every other element is 0.  Also zeroes the arrival
// counters of the split items (n_counters <= total).
template <typename TB, typename TQ>
__global__ void prepare_kx_kernel(const TB* log_mass, TQ* kx, int Nk, long long total, unsigned* counters,
                                  int n_counters) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx < n_counters) counters[idx] = 0u;
  if (idx >= total) return;
  const long long tile = idx >> 11;
  const int rem = static_cast<int>(idx & 2047);
  const int g = rem >> 7, half = (rem >> 6) & 1, r8 = (rem >> 3) & 7, e = rem & 7;
  float val = 0.f;
  if (half == 0 && e == 0) {
    const long long key = tile * kBN + g * 8 + r8;
    if (key < Nk) {
      val = log_mass == nullptr ? 0.f : 8.f * to_f32<TQ>(from_f32<TQ>(to_f32<TB>(log_mass[key])));
    } else {
      val = sizeof(TQ) == 2 && std::is_same<TQ, __half>::value ? -65504.f : -1.0e30f;
    }
  }
  kx[idx] = from_f32<TQ>(val);
}

// fp32 path: one warp per (query row, batch*head); lanes stride over keys with their own
// online-softmax state, merged across the warp at the end.  FMA arithmetic throughout.
__global__ void __launch_bounds__(256)
    mass_bias_attention_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                   const float* __restrict__ v, const float* __restrict__ bias,
                                   float* __restrict__ out, long long q_sb, long long q_sh,
                                   long long q_sn, long long k_sb, long long k_sh, long long k_sn,
                                   long long v_sb, long long v_sh, long long v_sn,
                                   long long o_sb, long long o_sh, long long o_sn, int H, int Nq,
                                   int Nk, float scale_log2) {
  __shared__ float qs[8][kHD];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long gw = static_cast<long long>(blockIdx.x) * 8 + warp;
  const int bh = blockIdx.y;
  if (gw >= Nq) return;
  const int batch = bh / H, head = bh - (bh / H) * H;
  const float* qrow = q + batch * q_sb + head * q_sh + gw * q_sn;
  qs[warp][lane] = qrow[lane];
  qs[warp][lane + 32] = qrow[lane + 32];
  __syncwarp();
  float m = -INFINITY, l = 0.f, acc[kHD];
#pragma unroll
  for (int i = 0; i < kHD; ++i) acc[i] = 0.f;
  const float* kb = k + batch * k_sb + head * k_sh;
  const float* vb = v + batch * v_sb + head * v_sh;
  for (int key = lane; key < Nk; key += 32) {
    const float4* kr = reinterpret_cast<const float4*>(kb + key * k_sn);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kHD / 4; ++i) {
      const float4 kv = kr[i];
      dot = fmaf(qs[warp][4 * i + 0], kv.x, dot);
      dot = fmaf(qs[warp][4 * i + 1], kv.y, dot);
      dot = fmaf(qs[warp][4 * i + 2], kv.z, dot);
      dot = fmaf(qs[warp][4 * i + 3], kv.w, dot);
    }
    const float x = dot * scale_log2 + bias[key];
    const float m_new = fmaxf(m, x);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float corr = exp2f(m - m_use);
    const float pr = exp2f(x - m_use);
    l = l * corr + pr;
    const float4* vr = reinterpret_cast<const float4*>(vb + key * v_sn);
#pragma unroll
    for (int i = 0; i < kHD / 4; ++i) {
      const float4 vv = vr[i];
      acc[4 * i + 0] = fmaf(pr, vv.x, acc[4 * i + 0] * corr);
      acc[4 * i + 1] = fmaf(pr, vv.y, acc[4 * i + 1] * corr);
      acc[4 * i + 2] = fmaf(pr, vv.z, acc[4 * i + 2] * corr);
      acc[4 * i + 3] = fmaf(pr, vv.w, acc[4 * i + 3] * corr);
    }
    m = m_new;
  }
  // merge lane states (butterfly)
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, off);
    const float lo = __shfl_xor_sync(0xffffffffu, l, off);
    const float mn = fmaxf(m, mo);
    const float mu = (mn == -INFINITY) ? 0.f : mn;
    const float ca = exp2f(m - mu), cb = exp2f(mo - mu);
#pragma unroll
    for (int i = 0; i < kHD; ++i) {
      const float ao = __shfl_xor_sync(0xffffffffu, acc[i], off);
      acc[i] = acc[i] * ca + ao * cb;
    }
    l = l * ca + lo * cb;
    m = mn;
  }
  float* orow = out + batch * o_sb + head * o_sh + gw * o_sn;
  const float inv = 1.f / l;
  // every lane holds the merged row; lane i writes elements i and i + 32
#pragma unroll
  for (int i = 0; i < kHD; ++i) {
    if ((i & 31) == lane) orow[i] = acc[i] * inv;
  }
}

}  // namespace

unsigned attention_error_word(int clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_attn_err, sizeof(v));
  if (clear) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_attn_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace vb200

using namespace vb200;

extern "C" size_t vb200_mass_bias_attention_workspace_size(int64_t Nk) {
  // the larger of the fp32 path's padded bias (512 B per key tile) and the tensor-core
  // path's extra K chunks (4 KB per key tile)
  const int64_t tiles = (Nk + kBN - 1) / kBN;
  return align_up(static_cast<size_t>(tiles > 0 ? tiles : 1) * kKxBytes, 256);
}

namespace {

// How the tensor-core launch divides its work items over the GPU (see AttnParams).
struct SplitPlan {
  long long items = 0, n_full = 0, n_tail = 0;
  int split = 1;
  size_t o_bytes = 0, ml_bytes = 0, cnt_bytes = 0;  // partial-result regions of the workspace
};

int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev < 64) cached[dev] = n;
  return n;
}

// The kernel runs one CTA per SM, so `items` CTAs take ceil(items / SMs) waves and the last
// wave leaves SMs idle.  Splitting each of the last wave's items into s key ranges turns that
// wave into ceil(tail * s / SMs) rounds of 1/s of an item (plus a per-CTA ramp of about three
// key tiles); s is the cheapest choice up to kMaxSplit.
SplitPlan plan_split(long long B, long long H, long long Nq, int n_tiles, int n_sm) {
  SplitPlan sp;
  const long long qblocks = (Nq + kQT * kBM - 1) / (kQT * kBM);
  sp.items = qblocks * B * H;
  sp.n_full = sp.items;
  if (n_sm <= 0 || n_tiles < 2 || sp.items <= 0) return sp;
  const long long tail = sp.items % n_sm;
  if (tail == 0) return sp;
  const double ramp = 3.0 / n_tiles;
  double best = 1.0 + ramp;
  int best_s = 1;
  for (int s = 2; s <= kMaxSplit && s <= n_tiles; ++s) {
    const long long rounds = (tail * s + n_sm - 1) / n_sm;
    const double cost = static_cast<double>(rounds) * (1.0 / s + ramp);
    if (cost < best - 1e-9) {
      best = cost;
      best_s = s;
    }
  }
  if (best_s == 1) return sp;
  sp.split = best_s;
  sp.n_tail = tail;
  sp.n_full = sp.items - tail;
  const size_t rows = static_cast<size_t>(tail) * best_s * kQT * kBM;
  sp.o_bytes = align_up(rows * kHD * sizeof(float), 256);
  sp.ml_bytes = align_up(rows * sizeof(float2), 256);
  sp.cnt_bytes = align_up(static_cast<size_t>(tail) * sizeof(unsigned), 256);
  return sp;
}

}  // namespace

extern "C" int vb200_mass_bias_attention_plan(int64_t B, int64_t H, int64_t Nq, int64_t Nk, int sms, int64_t* out) {
  VB200_REQUIRE(out != nullptr && B >= 1 && H >= 1 && Nq >= 0 && Nk >= 1 && sms >= 0,
                "mass_bias_attention_plan: bad arguments");
  const SplitPlan sp = plan_split(B, H, Nq, static_cast<int>((Nk + kBN - 1) / kBN), sms);
  out[0] = sp.items;
  out[1] = sp.n_full;
  out[2] = sp.n_tail;
  out[3] = sp.split;
  out[4] = static_cast<int64_t>(sp.o_bytes + sp.ml_bytes + sp.cnt_bytes);
  return VB200_OK;
}

extern "C" size_t vb200_mass_bias_attention_split_workspace_size(int64_t B, int64_t H, int64_t Nq, int64_t Nk) {
  const size_t base = vb200_mass_bias_attention_workspace_size(Nk);
  if (B < 1 || H < 1 || Nq < 1 || Nk < 1) return base;
  const SplitPlan sp = plan_split(B, H, Nq, static_cast<int>((Nk + kBN - 1) / kBN), sm_count());
  return base + sp.o_bytes + sp.ml_bytes + sp.cnt_bytes;
}

namespace {

int launch_bias(int dtype, const void* log_mass, int bias_dtype, float* bias, int Nk, int padded,
                cudaStream_t st) {
  const dim3 grid((padded + 255) / 256), block(256);
  // TQ is the attention dtype the bias is rounded to; TB the stored bias type.
#define VB200_BIAS_CASE(TB, TQ) \
  prepare_bias_kernel<TB, TQ><<<grid, block, 0, st>>>(static_cast<const TB*>(log_mass), bias, Nk, padded)
  if (bias_dtype == VB200_F32) {
    if (dtype == VB200_BF16) VB200_BIAS_CASE(float, __nv_bfloat16);
    else if (dtype == VB200_F16) VB200_BIAS_CASE(float, __half);
    else VB200_BIAS_CASE(float, float);
  } else if (bias_dtype == VB200_BF16) {
    if (dtype == VB200_BF16) VB200_BIAS_CASE(__nv_bfloat16, __nv_bfloat16);
    else if (dtype == VB200_F16) VB200_BIAS_CASE(__nv_bfloat16, __half);
    else VB200_BIAS_CASE(__nv_bfloat16, float);
  } else {
    if (dtype == VB200_BF16) VB200_BIAS_CASE(__half, __nv_bfloat16);
    else if (dtype == VB200_F16) VB200_BIAS_CASE(__half, __half);
    else VB200_BIAS_CASE(__half, float);
  }
#undef VB200_BIAS_CASE
  VB200_CHECK_LAUNCH("prepare_bias_kernel");
  return VB200_OK;
}

int launch_kx(int dtype, const void* log_mass, int bias_dtype, void* kx, int Nk, int n_tiles, unsigned* counters,
              int n_counters, cudaStream_t st) {
  const long long total = static_cast<long long>(n_tiles) * (kKxBytes / 2);
  const dim3 grid(static_cast<unsigned>((total + 255) / 256)), block(256);
#define VB200_KX_CASE(TB, TQ)                                                                                     \
  prepare_kx_kernel<TB, TQ><<<grid, block, 0, st>>>(static_cast<const TB*>(log_mass), static_cast<TQ*>(kx), Nk, total, \
                                                    counters, n_counters)
  if (bias_dtype == VB200_F32) {
    if (dtype == VB200_BF16) VB200_KX_CASE(float, __nv_bfloat16);
    else VB200_KX_CASE(float, __half);
  } else if (bias_dtype == VB200_BF16) {
    if (dtype == VB200_BF16) VB200_KX_CASE(__nv_bfloat16, __nv_bfloat16);
    else VB200_KX_CASE(__nv_bfloat16, __half);
  } else {
    if (dtype == VB200_BF16) VB200_KX_CASE(__half, __nv_bfloat16);
    else VB200_KX_CASE(__half, __half);
  }
#undef VB200_KX_CASE
  VB200_CHECK_LAUNCH("prepare_kx_kernel");
  return VB200_OK;
}

int make_qkv_map(CUtensorMap* map, const void* base, int dtype, int64_t N, int64_t H, int64_t B,
                 const int64_t* strides) {
  // dims: (d, token, head, batch); size-1 dims get a harmless stride.
  const uint64_t esz = 2;
  uint64_t dims[4] = {static_cast<uint64_t>(kHD), static_cast<uint64_t>(N),
                      static_cast<uint64_t>(H), static_cast<uint64_t>(B)};
  uint64_t sn = static_cast<uint64_t>(strides[2]) * esz;
  uint64_t sh = static_cast<uint64_t>(strides[1]) * esz;
  uint64_t sb = static_cast<uint64_t>(strides[0]) * esz;
  if (N == 1) sn = kHD * esz;
  if (H == 1) sh = sn * static_cast<uint64_t>(N);
  if (B == 1) sb = sh * static_cast<uint64_t>(H);
  uint64_t str[3] = {sn, sh, sb};
  uint32_t box[4] = {static_cast<uint32_t>(kHD), static_cast<uint32_t>(kBM), 1, 1};
  const CUtensorMapDataType dt =
      dtype == VB200_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode_tiled_map(map, dt, 4, base, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

extern "C" int vb200_mass_bias_attention(int dtype, const void* q, const void* k, const void* v,
                                         const void* log_key_mass, int bias_dtype, void* out,
                                         int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t D,
                                         const int64_t* qs, const int64_t* ks, const int64_t* vs,
                                         const int64_t* os, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  VB200_REQUIRE(dtype == VB200_BF16 || dtype == VB200_F16 || dtype == VB200_F32,
                "mass_bias_attention: unsupported dtype code %d", dtype);
  VB200_REQUIRE(bias_dtype == VB200_BF16 || bias_dtype == VB200_F16 || bias_dtype == VB200_F32,
                "mass_bias_attention: unsupported bias dtype code %d", bias_dtype);
  VB200_REQUIRE(D == kHD, "the fused kernel supports head_dim=64 only (got %lld)", (long long)D);
  VB200_REQUIRE(B >= 1 && H >= 1 && Nq >= 0 && Nk >= 1, "invalid sizes B=%lld H=%lld Nq=%lld Nk=%lld",
                (long long)B, (long long)H, (long long)Nq, (long long)Nk);
  VB200_REQUIRE(Nq < (1ll << 31) && Nk < (1ll << 31) && B * H < 65536, "sizes exceed the kernel's index range");
  VB200_REQUIRE(q && k && v && out && qs && ks && vs && os, "null pointer argument");
  if (Nq == 0) return VB200_OK;
  const size_t need = vb200_mass_bias_attention_workspace_size(Nk);
  VB200_REQUIRE(workspace != nullptr && workspace_bytes >= need,
                "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  VB200_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, "workspace must be 256-byte aligned");
  int rc = check_sm100();
  if (rc != VB200_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n_tiles = static_cast<int>((Nk + kBN - 1) / kBN);
  const float scale_log2 = kLog2e / std::sqrt(static_cast<float>(kHD));

  if (dtype == VB200_F32) {
    float* bias = static_cast<float*>(workspace);
    rc = launch_bias(dtype, log_key_mass, bias_dtype, bias, static_cast<int>(Nk), n_tiles * kBN, st);
    if (rc != VB200_OK) return rc;
    const dim3 grid(static_cast<unsigned>((Nq + 7) / 8), static_cast<unsigned>(B * H));
    mass_bias_attention_f32_kernel<<<grid, 256, 0, st>>>(
        static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v),
        bias, static_cast<float*>(out), qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1],
        vs[2], os[0], os[1], os[2], static_cast<int>(H), static_cast<int>(Nq),
        static_cast<int>(Nk), scale_log2);
    VB200_CHECK_LAUNCH("mass_bias_attention_f32_kernel");
    return VB200_OK;
  }

  VB200_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15u) == 0 && os[0] % 8 == 0 && os[1] % 8 == 0 &&
                    os[2] % 8 == 0,
                "output rows must be 16-byte aligned");
  // Split the last partial wave when the workspace holds the partial results (see AttnParams).
  SplitPlan sp = plan_split(B, H, Nq, n_tiles, sm_count());
  if (sp.split > 1 && workspace_bytes < need + sp.o_bytes + sp.ml_bytes + sp.cnt_bytes) {
    sp.split = 1;
    sp.n_full = sp.items;
    sp.n_tail = 0;
  }
  uint8_t* part = static_cast<uint8_t*>(workspace) + need;
  unsigned* counters = sp.split > 1 ? reinterpret_cast<unsigned*>(part + sp.o_bytes + sp.ml_bytes) : nullptr;
  rc = launch_kx(dtype, log_key_mass, bias_dtype, workspace, static_cast<int>(Nk), n_tiles, counters,
                 static_cast<int>(sp.n_tail), st);
  if (rc != VB200_OK) return rc;
  CUtensorMap tq, tk, tv;
  if ((rc = make_qkv_map(&tq, q, dtype, Nq, H, B, qs)) != VB200_OK) return rc;
  if ((rc = make_qkv_map(&tk, k, dtype, Nk, H, B, ks)) != VB200_OK) return rc;
  if ((rc = make_qkv_map(&tv, v, dtype, Nk, H, B, vs)) != VB200_OK) return rc;

  AttnParams prm;
  prm.kx = static_cast<const uint8_t*>(workspace);
  prm.out = out;
  prm.o_sb = os[0];
  prm.o_sh = os[1];
  prm.o_sn = os[2];
  prm.H = static_cast<int>(H);
  prm.Nq = static_cast<int>(Nq);
  prm.Nk = static_cast<int>(Nk);
  prm.n_tiles = n_tiles;
  prm.qblocks = static_cast<int>((Nq + kQT * kBM - 1) / (kQT * kBM));
  prm.n_full = static_cast<int>(sp.n_full);
  prm.split = sp.split;
  prm.o_part = sp.split > 1 ? reinterpret_cast<float*>(part) : nullptr;
  prm.ml_part = sp.split > 1 ? reinterpret_cast<float2*>(part + sp.o_bytes) : nullptr;
  prm.counters = counters;
  prm.scale_log2 = scale_log2;
  VB200_REQUIRE(sp.n_full + sp.n_tail * sp.split < (1ll << 31), "too many work items");
  const dim3 grid(static_cast<unsigned>(sp.n_full + sp.n_tail * sp.split));
  // The register split inside the kernel is only valid with exactly kLaunchRegs registers per
  // thread at launch: refuse to launch anything else.
  {
    cudaFuncAttributes fa{};
    VB200_CHECK_CUDA(cudaFuncGetAttributes(&fa, dtype == VB200_BF16 ? mass_bias_attention_tc_kernel<true>
                                                                     : mass_bias_attention_tc_kernel<false>),
                     "cudaFuncGetAttributes");
    if (fa.numRegs != kLaunchRegs)
      return set_error(VB200_EUNSUPPORTED,
                       "mass_bias_attention_tc_kernel was built with %d registers per thread; its register "
                       "split needs exactly %d",
                       fa.numRegs, kLaunchRegs);
  }
  // The shared-memory opt-in is per device: set it on every call (cheap, host-side only).
  if (dtype == VB200_BF16) {
    VB200_CHECK_CUDA(cudaFuncSetAttribute(mass_bias_attention_tc_kernel<true>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                     "cudaFuncSetAttribute");
    mass_bias_attention_tc_kernel<true><<<grid, kThreads, kSmemBytes, st>>>(tq, tk, tv, prm);
  } else {
    VB200_CHECK_CUDA(cudaFuncSetAttribute(mass_bias_attention_tc_kernel<false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
                     "cudaFuncSetAttribute");
    mass_bias_attention_tc_kernel<false><<<grid, kThreads, kSmemBytes, st>>>(tq, tk, tv, prm);
  }
  VB200_CHECK_LAUNCH("mass_bias_attention_tc_kernel");
  return VB200_OK;
}

// ------------------------------------------------------------------------------------------
// No-allocation variant.
//
// Some callers of this library cannot call cudaMalloc or any allocator: code that only
// receives raw device pointers from another runtime's memory arena (with no allocator handle
// to obtain scratch from), and latency-critical serving loops that must not call cudaMalloc /
// cudaFree because those calls synchronise the device.  For them the attention's only scratch
// buffer — the padded log2-domain bias — lives in a fixed file-scope device array instead of a
// caller workspace.  Every GPU that loads this library holds the array (4 MiB) until exit.
// ------------------------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocMaxKeys = 131072;  // keys per call; a multiple of the 128-key tile
constexpr size_t kNoAllocBytes = static_cast<size_t>(kNoAllocMaxKeys / kBN) * kKxBytes;  // 4 MiB
static __device__ __align__(256) uint8_t g_noalloc_bias[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_bias on the current device.  In host code the symbol is a
// host-side stand-in, so its address is resolved once per device (with that device current)
// through cudaGetSymbolAddress and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  VB200_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(VB200_EUNSUPPORTED, "device ordinal %d exceeds %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    VB200_CHECK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_bias), "cudaGetSymbolAddress(g_noalloc_bias)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return VB200_OK;
}

}  // namespace

extern "C" int vb200_mass_bias_attention_noalloc(int dtype, const void* q, const void* k, const void* v,
                                                 const void* log_key_mass, int bias_dtype, void* out,
                                                 int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t D,
                                                 const int64_t* qs, const int64_t* ks, const int64_t* vs,
                                                 const int64_t* os, void* stream) {
  if (Nk > kNoAllocMaxKeys)
    return set_error(VB200_EINVAL,
                     "mass_bias_attention_noalloc: %lld keys exceed the fixed scratch of %lld keys; "
                     "use vb200_mass_bias_attention with a caller workspace",
                     (long long)Nk, (long long)kNoAllocMaxKeys);
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != VB200_OK) return rc;
  // The bias kernel rewrites every scratch entry the attention kernel reads (real keys and the
  // -inf padding of the last tile), so nothing carries over from a previous call.  Only the
  // bias operand's share of the array is offered as workspace: with no room for split partial
  // results the launch is always the unsplit one, so the fixed array holds nothing but the bias
  // and the result equals vb200_mass_bias_attention given workspace_size(Nk) bytes.
  return vb200_mass_bias_attention(dtype, q, k, v, log_key_mass, bias_dtype, out, B, H, Nq, Nk, D, qs, ks,
                                   vs, os, scratch, vb200_mass_bias_attention_workspace_size(Nk), stream);
}

// ------------------------------------------------------------------------------------------
// The FMA-pipe exponential used by the softmax, exposed for testing against exact 2^x.
// ------------------------------------------------------------------------------------------
namespace vb200 {
namespace {
__global__ void exp2_poly_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  const long long i = 2 * (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  float p0, p1;
  exp2_poly2(x[i], i + 1 < n ? x[i + 1] : 0.f, p0, p1);
  y[i] = p0;
  if (i + 1 < n) y[i + 1] = p1;
}
}  // namespace
}  // namespace vb200

extern "C" int vb200_exp2_poly(const float* x, float* y, int64_t n, void* stream) {
  VB200_REQUIRE(n >= 0, "exp2_poly: negative size");
  if (n == 0) return VB200_OK;
  VB200_REQUIRE(x && y, "exp2_poly: null pointer");
  const long long pairs = (n + 1) / 2;
  exp2_poly_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
  VB200_CHECK_LAUNCH("exp2_poly_kernel");
  return VB200_OK;
}
