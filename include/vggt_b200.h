/*
 * vggt_b200.h — C ABI of the B200 (sm_100a) kernels for VGGT-Omega's token-merged global
 * attention: the merge step, mass-bias attention and the top-4 sparse-convex projection.
 *
 * Conventions
 *   - Every entry point returns 0 on success and a negative VB200_E* code on failure; the
 *     text of the last failure on the calling thread is returned by vb200_last_error().
 *     Argument errors are detected on the host before anything is launched.
 *   - Pointers are device pointers unless stated; sizes and strides are in ELEMENTS.
 *   - Work is enqueued on `stream` (a cudaStream_t, passed as void*); nothing synchronises
 *     the stream and nothing allocates device memory unless the entry point says so.
 *   - Index tensors are int64 (torch.long), as in the reference plans.
 *
 * Each declaration names the reference interface it replaces (paths inside
 * shuang-yang18/4D_TTT_merging).
 */
#ifndef VGGT_B200_H_
#define VGGT_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VB200_API __attribute__((visibility("default")))
#else
#define VB200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define VB200_F32 0
#define VB200_BF16 1
#define VB200_F16 2

/* status codes */
#define VB200_OK 0
#define VB200_EINVAL -1      /* shape / dtype / stride / alignment error   (Python: ValueError) */
#define VB200_ECUDA -2       /* CUDA runtime or driver error               (Python: RuntimeError) */
#define VB200_EUNSUPPORTED -3 /* device is not sm_100 / feature not built  (Python: RuntimeError) */

/* ---- library ---------------------------------------------------------------------------- */
VB200_API int vb200_version(void);
VB200_API const char* vb200_last_error(void);
/* Number of kernels this library has launched in the process (all devices, all threads). */
VB200_API unsigned long long vb200_launch_count(void);
/* OR of the error words that kernels write when a bounded wait runs out (bit 0) or an index
 * is out of range (bit 1).  Synchronises the current device; clears the words when clear!=0. */
VB200_API int vb200_device_error_flags(unsigned* flags, int clear);

/* ---- a1/a2/a3: mass-bias attention --------------------------------------------------------
 * out = softmax(q k^T / sqrt(D) + log_key_mass) v for every (batch, head); D must be 64.
 * Replaces mass_bias_attention() / _mass_bias_attention_fwd
 *   (vggt_omega/models/mass_bias_attention.py:85-129, :17-82) and the SDPA-with-mask call
 *   (vggt_omega/models/layers/attention.py:400); with log_key_mass == NULL it is the dense
 *   special-query SDPA (attention.py:406-423).
 * dtype: VB200_BF16 / VB200_F16 run on tcgen05 tensor cores (fp32 softmax state); VB200_F32
 *   runs an fp32 FMA path.  log_key_mass has `bias_dtype` and Nk entries; as in the
 *   reference it is rounded to `dtype` before use.
 * strides: {batch, head, token} for each of q, k, v, out; the channel stride is 1.
 * workspace: device scratch of vb200_mass_bias_attention_workspace_size(Nk) bytes (4 KB per
 *   128-key tile: the bias operand of the QK product, or the padded fp32 bias of the fp32
 *   path), 256-byte aligned; or vb200_mass_bias_attention_split_workspace_size bytes (below)
 *   for the split launch.  The call rewrites everything it reads from the workspace, so
 *   nothing carries over between calls, but calls that may run concurrently (other streams)
 *   need separate workspaces. */
VB200_API size_t vb200_mass_bias_attention_workspace_size(int64_t Nk);
/* Workspace that also lets the tensor-core launch split its last, partially filled wave of
 * (256-query block, head) items into key ranges on the current device: the bytes above plus
 * fp32 partial results (O, running max and sum) of the split items and their arrival
 * counters.  The split pieces are merged in a fixed order, so results do not depend on
 * timing; they can differ from the unsplit launch in the last fp32 bits before rounding.
 * With a workspace of vb200_mass_bias_attention_workspace_size(Nk) bytes the launch runs
 * unsplit. */
VB200_API size_t vb200_mass_bias_attention_split_workspace_size(int64_t B, int64_t H, int64_t Nq, int64_t Nk);
/* The launch plan of the tensor-core attention for `sms` SMs (host arithmetic only, no device
 * call): out[0] work items ((256-query block, head) pairs), out[1] items run whole, out[2]
 * items of the last partial wave split into key ranges, out[3] key ranges per split item,
 * out[4] extra workspace bytes for the split (beyond workspace_size(Nk)). */
VB200_API int vb200_mass_bias_attention_plan(int64_t B, int64_t H, int64_t Nq, int64_t Nk, int sms, int64_t* out);
VB200_API int vb200_mass_bias_attention(int dtype, const void* q, const void* k, const void* v,
                              const void* log_key_mass, int bias_dtype, void* out, int64_t B,
                              int64_t H, int64_t Nq, int64_t Nk, int64_t D,
                              const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, const int64_t* o_strides,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Same computation as vb200_mass_bias_attention given the minimal workspace
 * (vb200_mass_bias_attention_workspace_size(Nk) bytes): it always takes the unsplit launch,
 * and its output is bit-identical to that call's.  It is for callers that cannot allocate device
 * memory: code that only holds raw device pointers handed over by another runtime (no
 * allocator to get a workspace from) and latency-critical loops that must not call
 * cudaMalloc / cudaFree, which synchronise the device.  It allocates nothing: its scratch (the
 * per-key-tile bias operand) is a fixed 4 MiB array inside the library, present on every GPU that
 * loads it until the process exits, so Nk is limited to 131,072 keys (larger Nk returns
 * VB200_EINVAL).
 * The first call on a device resolves that array's device address (cudaGetSymbolAddress) with
 * the device current; make that first call before any stream capture.  All calls share the
 * array: calls that may overlap on the GPU (different streams, or different host threads on one
 * device) race on it.  Nothing carries over between calls: each call rewrites every entry it
 * reads.  This entry point has no counterpart in the reference. */
VB200_API int vb200_mass_bias_attention_noalloc(int dtype, const void* q, const void* k, const void* v,
                                                const void* log_key_mass, int bias_dtype, void* out,
                                                int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t D,
                                                const int64_t* q_strides, const int64_t* k_strides,
                                                const int64_t* v_strides, const int64_t* o_strides,
                                                void* stream);

/* The FMA-pipe exponential the attention softmax uses for part of each tile: y = 2^x by
 * range reduction and a degree-3 minimax polynomial (max relative error 7.5e-5 for x in
 * [-125, 64]; below -125 the result is about 2^-125).  Device arrays of n floats.  Test and
 * inspection entry point; no counterpart in the reference. */
VB200_API int vb200_exp2_poly(const float* x, float* y, int64_t n, void* stream);

/* ---- a7/a8: plan preprocessing --------------------------------------------------------------
 * Groups the S*corners (source, corner) pairs of a weighted plan by compact parent so that
 * every reduction below runs in a fixed order with no atomics.  Segment (j, c) lists, in
 * ascending source order, the sources whose corner-c parent is j; segments are laid out
 * j-major, c-minor.  Also emits mass_j = 1 + sum of the weights in j's segments (summed
 * corner by corner, source order inside a corner) and log(mass_j).
 * Replaces WeightedBilinearTokenPlan.__post_init__ (models/token_merging.py:323-333) and
 * deterministic_weighted_normalizer (token_merging.py:40-59).
 * parent: [S, corners] int64 compact ids in [0, M); weights: [S, corners] fp32;
 * src_rows: [S] int64 token row of each source (the plan's source_original), or NULL for
 *   identity.  Outputs: seg_offsets [M*corners + 1] int32, entry_src [S*corners] int32 (the
 *   token row of the entry's source), entry_w [S*corners] fp32, mass [M] fp32, log_mass [M]
 *   fp32 (either may be NULL).  A parent outside [0, M) sets device error bit 1 and the pair
 *   is dropped.
 * workspace: vb200_plan_csr_workspace_size(S, corners, M) bytes, 256-byte aligned. */
VB200_API size_t vb200_plan_csr_workspace_size(int64_t S, int64_t corners, int64_t M);
VB200_API int vb200_plan_csr_build(const int64_t* parent, const float* weights, const int64_t* src_rows,
                         int64_t S, int64_t corners, int64_t M, int32_t* seg_offsets,
                         int32_t* entry_src, float* entry_w, float* mass, float* log_mass,
                         void* workspace, size_t workspace_bytes, void* stream);
/* The same CSR, masses and log-masses for grouped plans, in one launch: group g's sources
 * [q_begin[g], q_begin[g+1]) all have their parents among merged rows [b_begin[g], b_begin[g+1])
 * (the frame-group planners; DEVICE int64 arrays of groups+1 entries, non-decreasing, ending at S
 * and M).  One CTA per group builds its part in shared memory; max_group_rows / max_group_sources
 * bound every group (rows x corners <= 8,192, sources x corners <= 16,384; larger groups:
 * vb200_plan_csr_build).  A parent outside its group sets device error bit 1 and its entry is
 * dropped.  Output identical to vb200_plan_csr_build.  Needs no workspace. */
VB200_API int vb200_plan_csr_build_grouped(const int64_t* parent, const float* weights, const int64_t* src_rows,
                                           int64_t S, int64_t corners, int64_t M, const int64_t* q_begin,
                                           const int64_t* b_begin, int groups, int max_group_rows,
                                           int max_group_sources, int32_t* seg_offsets, int32_t* entry_src,
                                           float* entry_w, float* mass, float* log_mass, void* stream);

/* ---- a4: top-4 scatter-accumulate (tokens -> merged) ----------------------------------------
 * out[j] = (x[keep[j]] + sum_c sum_{e in seg(j,c)} w_e * x[entry_src[e]]) / normalizer[j]
 * accumulated in fp32 (each product rounded to fp32, corner partial sums added in corner
 * order; the entries of a merged row with more than 256 of them are summed as a fixed two-level
 * tree: 256-entry chunk sums, then sums of 64 consecutive chunk sums, added in order), written
 * in `dtype`.  keep may be NULL (hard-merge mean pooling: the accumulator
 * starts at zero).  Row strides in elements; C % 8 == 0 for 16-bit types, C % 4 for fp32;
 * rows 16-byte aligned.  Rows of x outside [0, x_rows) referenced by keep or entry_src set
 * device error bit 1 and are skipped (keep: the accumulator starts at zero).
 * Replaces WeightedBilinearTokenPlan.compact / compact_query (token_merging.py:343-370,
 * :382-385) and TokenPlan.compact (token_merging.py:176-191, deterministic here). */
VB200_API int vb200_proj_scatter(int dtype, const void* x, int64_t x_rows, int64_t x_row_stride,
                       const int64_t* keep, int64_t M, int64_t corners,
                       const int32_t* seg_offsets, const int32_t* entry_src,
                       const float* entry_w, const float* normalizer, void* out,
                       int64_t out_row_stride, int64_t C, int64_t n_entries, void* workspace,
                       size_t workspace_bytes, void* stream);
/* The scatter's partial numerators for the query-sharded projection: numerators[j] = the fp32
 * sums of the plan's corner segments of row j (same order and tree as vb200_proj_scatter),
 * without the keep row and without dividing by the normaliser; numerators [M, C] fp32,
 * 16-byte aligned.  Each rank passes the CSR of its own sources; the owners then combine the
 * ranks' numerators with vb200_rank_reduce_rows.  No reference counterpart (the reference's
 * compact runs on one GPU, token_merging.py:343-370). */
VB200_API int vb200_proj_scatter_numerators(int dtype, const void* x, int64_t x_rows, int64_t x_row_stride, int64_t M,
                                            int64_t corners, const int32_t* seg_offsets, const int32_t* entry_src,
                                            const float* entry_w, float* numerators, int64_t C, int64_t n_entries,
                                            void* workspace, size_t workspace_bytes, void* stream);
/* out[j] = (x[keep[j]] + partials[0][j] + partials[1][j] + ... + partials[R-1][j]) / normalizer[j],
 * summed in fp32 in rank order and rounded to dtype once: the deterministic cross-rank reduction
 * of the query-sharded compact.  partials [R, rows, C] fp32 (rank r's numerators of these rows
 * at r, as an all-to-all delivers them); keep[j] < 0 or keep NULL: no keep row.  C % 8 == 0. */
VB200_API int vb200_rank_reduce_rows(int dtype, const float* partials, int R, int64_t rows, int64_t C, const void* x,
                                     int64_t x_rows, int64_t x_row_stride, const int64_t* keep, const float* normalizer,
                                     void* out, int64_t out_row_stride, void* stream);
/* Scratch of vb200_proj_scatter for M merged rows, n_entries CSR entries (the length of
 * entry_src) and C channels.  Merged rows with more than 256 entries (skewed plans) are split
 * into 256-entry chunks and groups of 64 chunks; the scratch holds the fp32 chunk and group
 * sums (at most 2 * ceil(n_entries / 256) + 1 chunks and 2 * ceil(chunks / 64) + 1 groups of
 * C floats) plus the scan arrays that place them. */
VB200_API size_t vb200_proj_scatter_workspace_size(int64_t M, int64_t n_entries, int64_t C);

/* ---- a4 + q/k norm fused: Q||K||V compaction of the qkv projection ---------------------------
 * qkv: [rows, 3C] rows of [q | k | v] (C = heads * 64, C % 256 == 0), bf16 or fp16.  q and k
 * are LayerNorm-ed per 64-channel head (weights ln_weight[0:64] / ln_bias[0:64] for q,
 * [64:128] for k, fp32, biased variance, `eps`) on every row they are read from, then for
 * tensor t in {q, k, v}: out[j, t] = (keep row + sum_c corner partial sums) / normalizer[j]
 * when bit t of pool_mask is set, else the keep row alone (compact_key).  fp32 accumulation,
 * one rounding to `dtype`.  out: [M, 3C].  ln_weight / ln_bias NULL: no normalisation.
 * Replaces the q_norm / k_norm + compact / compact_key sequence of
 * vggt_omega/models/layers/attention.py:337-374 (token_merging.py:343-376).
 * workspace: vb200_compact_qkv_workspace_size(rows, C) bytes (per-head LayerNorm statistics of
 * every row), 256-byte aligned; unused when ln_weight is NULL.  pool_mask | VB200_STATS_READY:
 * the workspace already holds those statistics, written by vb200_qkv_head_stats for the same
 * qkv and eps (e.g. on the stream of the qkv GEMM, concurrently with the plan); the call then
 * launches the compaction alone. */
#define VB200_STATS_READY 8
VB200_API size_t vb200_compact_qkv_workspace_size(int64_t rows, int64_t C);
/* The per-head LayerNorm statistics (mean, 1 / sqrt(var + eps)) of the q and k blocks of every
 * qkv row, into a workspace of vb200_compact_qkv_workspace_size(rows, C) bytes: the first step of
 * vb200_compact_qkv on its own, so that it can run as soon as the qkv GEMM has finished. */
VB200_API int vb200_qkv_head_stats(int dtype, const void* qkv, int64_t rows, int64_t row_stride, int64_t C, float eps,
                                   void* workspace, size_t workspace_bytes, void* stream);
VB200_API int vb200_compact_qkv(int dtype, const void* qkv, int64_t rows, int64_t row_stride, int64_t C,
                                const float* ln_weight, const float* ln_bias, float eps, const int64_t* keep,
                                int64_t M, int64_t corners, const int32_t* seg_offsets,
                                const int32_t* entry_src, const float* entry_w, const float* normalizer,
                                int pool_mask, void* out, int64_t out_row_stride, void* workspace,
                                size_t workspace_bytes, void* stream);
/* vb200_compact_qkv with the k|v all-gather of the query-sharded layer fused in: besides out,
 * the k and v parts of merged row j ([2C] elements, k then v) are stored into each of the
 * `world` buffers kv_dst_ptrs[r] (peer-mapped memory of the other GPUs, this GPU's own buffer
 * included) at row kv_row0 + j, row stride kv_row_stride elements; the stores are posted
 * NVLink writes from the consumer threads, overlapping the compaction, followed by a
 * system-scope fence.  multicast != 0: kv_dst_ptrs[0] is instead the address of the buffers
 * in a multicast object (NVLS) that binds every rank's buffer, and each row part is written
 * once with multimem.st (the switch replicates it to all GPUs).  The caller orders them between cross-GPU barriers (every rank has
 * finished reading the buffers before; every rank's writes have landed after).  Needs
 * C <= 1024.  Replaces the compaction + NCCL all-gather of merged K/V of the sharded layer
 * (the reference's aggregator runs the layer on one GPU: aggregator.py:901-1215). */
VB200_API int vb200_compact_qkv_peer(int dtype, const void* qkv, int64_t rows, int64_t row_stride, int64_t C,
                                     const float* ln_weight, const float* ln_bias, float eps, const int64_t* keep,
                                     int64_t M, int64_t corners, const int32_t* seg_offsets,
                                     const int32_t* entry_src, const float* entry_w, const float* normalizer,
                                     int pool_mask, void* out, int64_t out_row_stride,
                                     const uint64_t* kv_dst_ptrs, int world, int multicast, int64_t kv_row0,
                                     int64_t kv_row_stride, void* workspace, size_t workspace_bytes,
                                     void* stream);
/* Per-64-channel-head LayerNorm of rows (the dense queries of query-preserving plans and the
 * special queries): out[r] = LN(x[r]).  C % 256 == 0. */
VB200_API int vb200_head_layernorm(int dtype, const void* x, int64_t rows, int64_t row_stride, int64_t C,
                                   const float* weight, const float* bias, float eps, void* out,
                                   int64_t out_row_stride, void* stream);

/* ---- a6: top-4 gather (merged -> tokens) ----------------------------------------------------
 * out[keep[k]] = y[k];  out[src[s]] = sum_c w[s,c] * y[parent[s,c]]
 * For 16-bit dtypes the weights are rounded to `dtype` and each product is rounded to
 * `dtype` before the (fp32) 4-term sum, which is rounded once — the reference's
 * value-dtype arithmetic.  Rows of `out` covered by neither keep nor src are left as they
 * are unless zero_fill != 0 (then they are zeroed), as new_zeros does in the reference.
 * keep may be NULL: only the source rows are written (K still bounds the parent ids).
 * Replaces WeightedBilinearTokenPlan.restore / restore_query (token_merging.py:387-426). */
VB200_API int vb200_proj_gather(int dtype, const void* y, int64_t y_row_stride, const int64_t* keep,
                      int64_t K, const int64_t* src, const int64_t* parent, const float* w,
                      int64_t S, int64_t corners, void* out, int64_t out_row_stride,
                      int64_t N_out, int64_t C, int zero_fill, void* stream);
/* Same result as vb200_proj_gather (bit for bit, zero_fill excluded: the caller zeroes rows that
 * neither keep nor src covers), for skewed plans: the merged rows listed in hot_rows (n_hot[0]
 * of them, at most max_hot, a DEVICE int32) are copied once per CTA into shared memory and
 * every reference to them is read from there; hot_slot [K] maps a merged row to its slot or -1.
 * The table comes from vb200_plan_hot_rows.  max_hot must not exceed
 * vb200_proj_gather_hot_capacity(dtype, C) (staged rows take max_hot * C elements of shared
 * memory per CTA).  Replaces the same reference function as vb200_proj_gather. */
VB200_API int vb200_proj_gather_hot(int dtype, const void* y, int64_t y_row_stride, const int64_t* keep,
                                    int64_t K, const int64_t* src, const int64_t* parent, const float* w,
                                    int64_t S, int64_t corners, void* out, int64_t out_row_stride,
                                    int64_t N_out, int64_t C, const int32_t* hot_rows, const int32_t* hot_slot,
                                    const int32_t* n_hot, int max_hot, void* stream);
VB200_API int vb200_proj_gather_hot_capacity(int dtype, int64_t C);
/* The staging table of vb200_proj_gather_hot from a plan CSR (vb200_plan_csr_build): the merged
 * rows with the most (source, corner) references, at most max_hot of them, chosen on the device
 * (one block; whole reference-count buckets from the top).  hot_rows [max_hot], hot_slot [M],
 * n_hot [1], all device int32. */
VB200_API int vb200_plan_hot_rows(const int32_t* seg_offsets, int64_t M, int64_t corners, int max_hot,
                                  int32_t* hot_rows, int32_t* hot_slot, int32_t* n_hot, void* stream);

/* ---- a5/a10: plain row gather -----------------------------------------------------------------
 * out[i] = x[index[i]] for i < R; an index outside [0, x_rows) sets device error bit 1 and
 * leaves out[i] untouched.  Replaces compact_key (token_merging.py:372-376),
 * TokenPlan.restore (token_merging.py:193-196) and the keep gathers of TokenPlan.compact. */
VB200_API int vb200_row_gather(int dtype, const void* x, int64_t x_rows, int64_t x_row_stride, const int64_t* index,
                     int64_t R, void* out, int64_t out_row_stride, int64_t C, void* stream);

/* ---- e: rank-ordered gather from other GPUs (sharded global block) ----------------------------
 * dst row (r * rows + i) = row i of rank r's block at src_ptrs[r] (row stride src_stride_bytes),
 * for r < world (<= 16) and i < rows; row_bytes per row.  src_ptrs is a HOST array of device
 * addresses that are valid in this process (peer memory mapped by the caller, e.g. PyTorch
 * symmetric memory; the local block may be one of them).  Sizes and strides must be multiples of
 * 4 bytes (16-byte aligned blocks use 16-byte peer loads).  The caller orders the launch after
 * the peers have written their blocks and before they overwrite them.  Replaces the merged-K/V
 * and log-mass all-gather of the sharded path (NCCL all_gather_into_tensor). */
VB200_API int vb200_peer_gather(const uint64_t* src_ptrs, int world, int64_t rows, int64_t src_stride_bytes,
                                int64_t row_bytes, void* dst, int64_t dst_stride_bytes, void* stream);
/* Push form of the same exchange: this rank's rows (local src) are stored into every rank's
 * destination dst_ptrs[r] at rows [dst_row0, dst_row0 + rows) (dst_ptrs: HOST array of
 * peer-mapped device addresses, 16-byte aligned; all sizes and strides multiples of 16 bytes),
 * followed by a system-scope fence. */
VB200_API int vb200_peer_push(const void* src, int64_t rows, int64_t src_stride_bytes, int64_t row_bytes,
                              const uint64_t* dst_ptrs, int world, int64_t dst_row0, int64_t dst_stride_bytes,
                              void* stream);
/* Cross-GPU barrier that orders the exchange kernels above (no reference counterpart: the
 * reference has no multi-GPU inference path).  pad_ptrs: HOST array of every rank's signal pad
 * (world uint32 slots each, peer-mapped, zeroed on every rank before the first barrier);
 * epoch: a uint32 in this rank's device memory, zero-initialised, advanced by every barrier
 * (so a recorded CUDA graph replays correctly).  Each rank stores the new epoch into its slot
 * of every pad (release, system scope) and waits until every slot of its own pad holds it
 * (acquire).  The wait gives up after timeout_ns of global time: it then sets device error
 * bit 0 (vb200_device_error_flags) and returns; the context stays usable. */
VB200_API int vb200_peer_barrier(const uint64_t* pad_ptrs, int world, int rank, uint32_t* epoch,
                                 int64_t timeout_ns, void* stream);

/* ---- a9/a11: merge step ----------------------------------------------------------------------
 * Row L2 normalisation to bf16 (F.normalize(x.float(), dim=-1, eps).to(bfloat16)),
 * as in build_fastvggt_plan (token_merging.py:1102-1103).  `rows` may be NULL (identity)
 * or gather rows of x. */
VB200_API int vb200_row_normalize_bf16(int dtype, const void* x, int64_t x_rows, int64_t x_row_stride, const int64_t* rows,
                             int64_t R, int64_t C, float eps, void* out, int64_t out_row_stride,
                             void* stream);

/* Basis-range pieces per query block that vb200_sim_topk uses for a launch of `ctas` CTAs over
 * n_tiles basis tiles on `sms` SMs (host arithmetic only; 1 = unsplit, at most 3; a split search
 * stores per-piece keys in the output rows and merges them in a second small kernel). */
VB200_API int vb200_sim_topk_split(int64_t ctas, int n_tiles, int sms);

/* Cosine-similarity GEMM with a fused running top-k epilogue (k = 1, 4 or 16; 16 is the
 * semantic shortlist of the geometry-guarded route, sparse_convex.py:263-266, 506-508, and needs
 * basis groups of at most 65,536 rows).
 * score[r, n] = bf16_round( <query[r], basis[n]> ) over D channels (fp32 accumulation on
 * tcgen05), ranked per row; ties keep the lower basis index.  With groups: query rows
 * [q_begin[g], q_begin[g+1]) are matched only against basis rows [b_begin[g], b_begin[g+1]);
 * groups == 1 with NULL tables means all rows against all basis rows.  q_begin / b_begin are
 * HOST arrays of groups+1 int64 entries (read before the launch).  Rows whose group has no
 * basis row get values -inf and indices -1.
 * query: [R, D] bf16, row stride q_row_stride; basis: [Nb, D] bf16 (K-major, i.e. the rows
 * of the dictionary, row stride b_row_stride).  D % 64 == 0.  values [R, k] fp32,
 * indices [R, k] int64 (basis index, global), ordered best first.
 * Replaces streaming_top4 (models/sparse_convex_kernels.py:309-329), the
 * `(q.bf16 @ basis.bf16).topk(4)` retrievals (models/sparse_convex.py:264, 294, 546-547,
 * 2402-2404) and the bmm + max(-1) of build_fastvggt_plan (token_merging.py:1106-1111). */
VB200_API int vb200_sim_topk(const void* query, int64_t q_row_stride, const void* basis,
                   int64_t b_row_stride, int64_t R, int64_t Nb, int64_t D, int k,
                   const int64_t* q_begin, const int64_t* b_begin, int64_t groups,
                   float* values, int64_t* indices, void* stream);

/* Ranking and keep / inverse maps of the FastVGGT merge (token_merging.py:1112-1121):
 * the S sources are ordered by best score (stable, descending); the first `removed` are
 * merged into destination dest_idx[target[s]]; keep [total-removed] lists the surviving
 * token ids in order and inverse [total] maps every token to its compact index.
 * best [S] fp32, target [S] int64 (index into dest_idx), source_idx [S], dest_idx [Dn] int64
 * token ids.  workspace: vb200_merge_assign_workspace_size(S, total) bytes. */
VB200_API size_t vb200_merge_assign_workspace_size(int64_t S, int64_t total);
VB200_API int vb200_merge_assign(const float* best, const int64_t* target, const int64_t* source_idx,
                                 const int64_t* dest_idx, int64_t S, int64_t Dn, int64_t total,
                                 int64_t removed, int64_t* keep, int64_t* inverse, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Support Gram and right-hand side of each source (sparse_convex.py:2314-2316):
 * gram[s] = F[p] F[p]^T over its four support rows p = parent_rows[s, :], rhs[s] = F[p] x_s
 * with x_s = F[src_rows[s]] (src_rows NULL: row s), fp32 accumulation.  With alpha != NULL
 * the four-support projected-gradient solve (`steps` iterations, as
 * vb200_four_support_projected_gradient) runs in the same kernel.  gram / rhs may be NULL.
 * F: [rows, D] of `dtype` with row stride row_stride.  Rows outside [0, rows) set device
 * error bit 1 and read row 0 instead. */
VB200_API int vb200_support_fit(int dtype, const void* feat, int64_t rows, int64_t row_stride,
                                const int64_t* src_rows, const int64_t* parent_rows, int64_t S,
                                int64_t D, float* gram, float* rhs, float* alpha, int steps,
                                void* stream);
/* Certificate of the fits above (the reference's solve epilogue, models/sparse_convex.py:575-583,
 * :316-319 and the acceptance test :648-653 that reads it): per source the reconstruction
 * r = sum_c alpha[s,c] * feat[parent_rows[s,c]], cosine = <x, r> / (max(|x|,1e-8) max(|r|,1e-8)),
 * residual = |x - r|, recon_norm = |r|, with x = feat[src_rows[s]] (src_rows NULL: row s).
 * alpha [S,4] fp32; outputs [S] fp32.  D % 16 == 0. */
VB200_API int vb200_support_certificate(int dtype, const void* feat, int64_t rows, int64_t row_stride,
                                        const int64_t* src_rows, const int64_t* parent_rows, const float* alpha,
                                        int64_t S, int64_t D, float* cosine, float* residual, float* recon_norm,
                                        void* stream);
/* The geometry-guarded support route of the released planner (support_geometry_weight > 0 with
 * a guard tolerance; sparse_convex.py:502-531, 586-639 (temporal-local) and 263-367 (global)).
 *
 * vb200_geometry_shortlist: per source row, from its top-k feature shortlist (values / indices
 * of vb200_sim_topk with k = 16: bf16 scores best first, indices into the basis rows, -1 for
 * empty slots) the joint value score - weight * |g_s - g_c|^2 (fp32), its top-4 shortlist
 * positions (ties to the lower position) reordered by feature score (stable), written as basis
 * indices to joint_ids [S, 4]; feature_ids [S, 4] = the first four shortlist indices; changed[s]
 * = 1 where the two differ.  query_geo [S, 4] and basis_geo [Nb, 4] fp32, 16-byte aligned. */
VB200_API int vb200_geometry_shortlist(const float* values, const int64_t* indices, int64_t S, int k,
                                       const float* query_geo, const float* basis_geo, int64_t Nb, float weight,
                                       int64_t* feature_ids, int64_t* joint_ids, int32_t* changed, void* stream);
/* vb200_geometry_guard: given both fits (ids [S, 4] into the rows of geometry [rows, 4], weights
 * [S, 4], cosine / residual / reconstruction norm [S] from vb200_support_fit and
 * vb200_support_certificate), keep the joint fit where changed[s] and joint cosine + tolerance >=
 * feature cosine and joint residual <= feature residual + tolerance and the joint 4-D residual
 * |g_s - sum_c w_c g_c| is strictly smaller; else the feature fit.  Writes the chosen ids,
 * weights and certificate, and chosen[s] (0 / 1). */
VB200_API int vb200_geometry_guard(int64_t S, const float* geometry, int64_t rows, const int64_t* source_ids,
                                   const int64_t* feature_ids, const float* feature_w, const float* feature_cos,
                                   const float* feature_res, const float* feature_nrm, const int64_t* joint_ids,
                                   const float* joint_w, const float* joint_cos, const float* joint_res,
                                   const float* joint_nrm, const int32_t* changed, float tolerance, int64_t* out_ids,
                                   float* out_w, float* out_cos, float* out_res, float* out_nrm, int32_t* chosen,
                                   void* stream);
/* out[q] = max over t of the fp32 dot product <feat[query[q]], feat[targets[q, t]]> (targets
 * [Q, n_targets] int64, -1 = no target; -inf when a query has none): the top-1 cosine that
 * prunes redundant uniform anchors in the released planner's protected skeleton
 * (models/sparse_convex.py:1404-1418).  D % 16 == 0. */
VB200_API int vb200_row_max_dot(int dtype, const void* feat, int64_t rows, int64_t row_stride, const int64_t* query,
                                const int64_t* targets, int n_targets, int64_t Q, int64_t D, float* out,
                                void* stream);

/* ---- next tier: 4-support simplex solvers ------------------------------------------------
 * Replaces four_support_projected_gradient (models/sparse_convex_kernels.py:283-296) and
 * four_support_active_set (sparse_convex_kernels.py:332-353).  gram [rows,4,4], rhs
 * [rows,4], out [rows,4], all fp32 contiguous. */
VB200_API int vb200_four_support_projected_gradient(const float* gram, const float* rhs, float* out,
                                          int64_t rows, int steps, void* stream);
VB200_API int vb200_four_support_active_set(const float* gram, const float* rhs, float* out,
                                  int64_t rows, float ridge, void* stream);

/* ---- (f) next, 4: TTT pre-pass kernels ------------------------------------------------------
 * The flow-free token-matching TTT's per-clip kernels (vggt_omega/utils/ttt_kernels.py).  All
 * arithmetic is fp32; descriptor / field inputs may be f32, bf16 or f16 (dtype), contiguous. */

/* out[r] = x[r] / max(||x[r]||_2, eps), fp32 [rows, C].  Replaces normalize_rows
 * (ttt_kernels.py:233-249), whose default is F.normalize(value.float(), eps=1e-6). */
VB200_API int vb200_row_l2_normalize(int dtype, const void* x, int64_t rows, int64_t C, float eps, float* out,
                                     void* stream);
/* Exact-window cosine top-2 of [pairs, H, W, C] descriptors (1 <= C <= 256, C a multiple of 4
 * for f32 and of 8 for 16-bit types, rows 16-byte aligned): for every source
 * patch (p, y, x) the best and second-best dot product with target[p, y + oy, x + ox] over
 * |oy| <= radius_y, |ox| <= radius_x inside the grid, and the (dy, dx) of the best.  Candidates
 * run in row-major offset order (reverse != 0: the reversed order the backward match uses); a
 * later candidate replaces the best only when strictly greater.  best/second fp32, dy/dx int32,
 * each [pairs * H * W].  Replaces local_top2_match / _local_top2_match_kernel
 * (ttt_kernels.py:252-277, :45-101). */
VB200_API int vb200_local_top2_match(int dtype, const void* source, const void* target, int64_t pairs, int64_t H,
                                     int64_t W, int64_t C, int radius_y, int radius_x, int reverse, float* best,
                                     float* second, int32_t* dy, int32_t* dx, void* stream);
/* out[b, y, x] = field[b, clamp(y + int(flow_y)), clamp(x + int(flow_x))] with the flow
 * [B, H, W, 2] (x, y) truncated toward zero; field / out [B, H, W, C] of dtype.  Replaces
 * integer_gather_warp (ttt_kernels.py:280-297, :104-127). */
VB200_API int vb200_integer_warp(int dtype, const void* field, const float* flow, int64_t B, int64_t H, int64_t W,
                                 int64_t C, void* out, void* stream);
/* Per patch of F frames: residual = mean over the available directions (forward flow of pair f
 * when f + 1 < F, backward flow of pair f - 1 when f > 0) of |flow - predicted|; confidence =
 * the smaller of those directions' confidences (1 where absent); boundary = mean of |flow - its
 * 3 x 3 zero-padded box mean|.  forward/backward flow [F-1, H, W, 2], predicted [F, H, W, 4]
 * (forward dx, dy, backward dx, dy), confidences [F-1, H, W]; outputs fp32 [F, H, W].  Replaces
 * fused_motion_cues (ttt_kernels.py:300-318, :130-196). */
VB200_API int vb200_motion_cues(const float* forward_flow, const float* backward_flow, const float* predicted,
                                const float* forward_conf, const float* backward_conf, int64_t F, int64_t H,
                                int64_t W, float* residual, float* confidence, float* boundary, void* stream);
/* sensitivity = clamp(0.45 (1 - conf) + 0.35 clamp(residual / max(rs, 1e-6)) + 0.20
 * clamp(boundary / max(bs, 1e-6)), 0, 1); for patches after the first frame (row >= patch_count)
 * low = conf < uncertain_confidence and event = (residual >= rt and conf >= uncertain) or
 * boundary >= bt or 1 - conf >= 0.55 (int8 0/1).  rs, bs, rt, bt are device fp32 scalars.
 * Replaces fused_sensitivity_labels (ttt_kernels.py:321-341, :199-230). */
VB200_API int vb200_sensitivity_labels(const float* residual, const float* confidence, const float* boundary,
                                       int64_t rows, int64_t patch_count, float uncertain_confidence,
                                       const float* residual_scale, const float* boundary_scale,
                                       const float* residual_threshold, const float* boundary_threshold,
                                       float* sensitivity, int8_t* low_confidence, int8_t* raw_event, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VGGT_B200_H_ */
