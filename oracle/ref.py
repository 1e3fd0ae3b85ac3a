"""numpy restatement of the reference's token-merged global-attention path (TEST ORACLE).

Every function restates one reference function of shuang-yang18/4D_TTT_merging; the file and
lines are given in each docstring.  Floating-point work that the reference does in fp32 is
done here in float64 (then rounded where the reference rounds), so the oracle is at least as
accurate as the reference; bf16 / fp16 rounding is emulated bit-exactly (round to nearest
even) wherever the reference rounds to a 16-bit type.
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "round_bf16", "round_f16", "round_to", "bf16_to_f32_bits",
    "mass_bias_attention", "normalizer", "compact", "compact_key", "restore",
    "token_plan_compact", "token_plan_restore", "topk_scores", "similarity_topk",
    "torch_cpu_rand", "fastvggt_plan", "fastvggt_assign", "fastvggt_removed", "normalize_bf16", "projected_gradient", "active_set",
    "simplex_project", "layer_norm", "global_attention_forward",
]


# ------------------------------------------------------------------------------------------
# 16-bit rounding
# ------------------------------------------------------------------------------------------
def round_bf16(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    out[nan] = np.nan
    return out


def round_f16(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    return np.asarray(x, dtype=np.float32)


def bf16_to_f32_bits(bits: np.ndarray) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32 values."""
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------------------------------
# a1/a2/a3: mass-bias attention
# ------------------------------------------------------------------------------------------
def mass_bias_attention(q, k, v, log_key_mass=None, dtype: str = "f32", round_p: bool = False):
    """softmax(q k^T / sqrt(d) + bias) v per (batch, head).

    Restates vggt_omega/models/mass_bias_attention.py:85-129 (and the SDPA-with-mask call of
    vggt_omega/models/layers/attention.py:400): the bias is ``log_key_mass`` rounded to the
    attention dtype (:109); with ``round_p`` the probabilities are rounded to the value dtype
    before the PV product as the fused kernel does (:74).  q [B,H,Nq,d], k/v [B,H,Nk,d]
    (values already representable in ``dtype``).  Returns float64."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    d = q.shape[-1]
    logits = np.matmul(q, np.swapaxes(k, -1, -2)) / math.sqrt(d)
    if log_key_mass is not None:
        bias = round_to(np.asarray(log_key_mass, dtype=np.float32).reshape(-1), dtype).astype(np.float64)
        logits = logits + bias[None, None, None, :]
    m = logits.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(logits - m)
    denom = p.sum(axis=-1, keepdims=True)
    if round_p:
        p = round_to(p.astype(np.float32), dtype).astype(np.float64)
    return np.matmul(p, v) / denom


# ------------------------------------------------------------------------------------------
# a7: mass / normalizer
# ------------------------------------------------------------------------------------------
def normalizer(parent, weights, kept: int) -> np.ndarray:
    """mass_j = 1 + sum over corners of the weights of sources whose corner-c parent is j,
    each corner summed in ascending source order (stable argsort + segment_reduce).
    Restates deterministic_weighted_normalizer, vggt_omega/models/token_merging.py:40-59.
    parent/weights [S, corners]; returns float32 [kept]."""
    parent = np.asarray(parent, dtype=np.int64)
    weights = np.asarray(weights, dtype=np.float32)
    mass = np.ones(kept, dtype=np.float32)
    for c in range(parent.shape[1]):
        seg = np.zeros(kept, dtype=np.float32)
        order = np.argsort(parent[:, c], kind="stable")
        np.add.at(seg, parent[order, c], weights[order, c])  # fp32, in source order
        mass = (mass + seg).astype(np.float32)
    return mass


def _segment_sums(x32, parent_c, weight_c, kept):
    """Per-parent fp32 sums of weight * x in ascending source order (vectorised over C)."""
    C = x32.shape[1]
    out = np.zeros((kept, C), dtype=np.float32)
    order = np.argsort(parent_c, kind="stable")
    prod = (x32[order] * weight_c[order, None]).astype(np.float32)  # fp32 products
    # sequential fp32 accumulation per segment, in order (np.add.at is unbuffered and
    # applies the updates in array order)
    np.add.at(out, parent_c[order], prod)
    return out


# ------------------------------------------------------------------------------------------
# a4/a5: compact (tokens -> merged)
# ------------------------------------------------------------------------------------------
def compact(value, keep, source_original, parent, pool_weights, norm, dtype: str = "f32",
            pool_source_content: bool = True) -> np.ndarray:
    """Restates WeightedBilinearTokenPlan.compact, vggt_omega/models/token_merging.py:343-370:
    gather the kept rows, add each corner's segment sum of weight * source (fp32, stable
    source order), divide by the normalizer and round to the value dtype.
    value [N, C]; keep [K]; source_original [S]; parent/pool_weights [S, corners]; norm [K]."""
    value = np.asarray(value, dtype=np.float32)
    keep = np.asarray(keep, dtype=np.int64)
    acc = value[keep].astype(np.float32)
    src = np.asarray(source_original, dtype=np.int64)
    if len(src) == 0 or not pool_source_content:
        return round_to(acc, dtype)
    parent = np.asarray(parent, dtype=np.int64)
    pool_weights = np.asarray(pool_weights, dtype=np.float32)
    x_src = value[src]
    for c in range(parent.shape[1]):
        acc = (acc + _segment_sums(x_src, parent[:, c], pool_weights[:, c], len(keep))).astype(np.float32)
    out = (acc / np.asarray(norm, dtype=np.float32).reshape(-1, 1)).astype(np.float32)
    return round_to(out, dtype)


def compact_key(value, keep, dtype: str = "f32") -> np.ndarray:
    """Restates compact_key's physical-key gather, token_merging.py:372-376."""
    return round_to(np.asarray(value, dtype=np.float32)[np.asarray(keep, dtype=np.int64)], dtype)


# ------------------------------------------------------------------------------------------
# a6: restore (merged -> tokens)
# ------------------------------------------------------------------------------------------
def restore(value, keep, source_original, parent, restore_weights, original_tokens: int,
            dtype: str = "f32") -> np.ndarray:
    """Restates WeightedBilinearTokenPlan.restore, token_merging.py:387-414: zeros, kept rows
    copied, source rows = sum_c w_c * value[parent_c] computed in the value dtype (weights
    rounded to it, each product rounded to it, fp32 sum rounded once).  value [K, C]."""
    value = np.asarray(value, dtype=np.float32)
    out = np.zeros((original_tokens, value.shape[1]), dtype=np.float32)
    keep = np.asarray(keep, dtype=np.int64)
    out[keep] = value
    src = np.asarray(source_original, dtype=np.int64)
    if len(src):
        parent = np.asarray(parent, dtype=np.int64)
        w = round_to(np.asarray(restore_weights, dtype=np.float32), dtype)
        acc = np.zeros((len(src), value.shape[1]), dtype=np.float32)
        for c in range(parent.shape[1]):
            prod = round_to((value[parent[:, c]] * w[:, c, None]).astype(np.float32), dtype)
            acc = (acc + prod).astype(np.float32)
        out[src] = round_to(acc, dtype)
    return out


# ------------------------------------------------------------------------------------------
# a12: the global-attention call site
# ------------------------------------------------------------------------------------------
def layer_norm(x, weight, bias, eps: float = 1e-5) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    mu = x.mean(axis=-1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * np.asarray(weight, np.float64) + np.asarray(bias, np.float64)


def global_attention_forward(x, params: dict, plan: dict, heads: int, preserve_queries: bool,
                             dense_special: bool = True) -> np.ndarray:
    """Restates SelfAttention.forward with a WeightedBilinearTokenPlan in fp32
    (vggt_omega/models/layers/attention.py:264-314, :328-439): qkv projection (k bias masked,
    :195-207), q/k LayerNorm over the head dim, compaction (compact-query plans compact Q, K
    and V; query-preserving plans keep physical keys and pool V), attention with the
    key_log_mass bias, exact dense attention for the special queries, output projection and
    restore.  x [N, dim]; params: the module's parameters by name; plan: keep, source, parent,
    weights, normalizer, special, special_compact.  Returns [N, dim] float32."""
    x = np.asarray(x, dtype=np.float64)
    N, dim = x.shape
    hd = dim // heads
    w_qkv = np.asarray(params["qkv.weight"], np.float64)
    b_qkv = np.asarray(params["qkv.bias"], np.float64) * np.asarray(params["qkv.bias_mask"], np.float64)
    qkv = (x @ w_qkv.T + b_qkv).reshape(N, 3, heads, hd)
    q = layer_norm(qkv[:, 0], params["q_norm.weight"], params["q_norm.bias"])  # [N,H,hd]
    k = layer_norm(qkv[:, 1], params["k_norm.weight"], params["k_norm.bias"])
    v = qkv[:, 2]
    flat = lambda t: t.reshape(N, dim).astype(np.float32)
    keep, src, parent, w = plan["keep"], plan["source"], plan["parent"], plan["weights"]
    norm = plan["normalizer"]
    K = len(keep)
    vc = compact(flat(v), keep, src, parent, w, norm)
    if preserve_queries:
        qc = flat(q)
        kc = compact_key(flat(k), keep)
    else:
        qc = compact(flat(q), keep, src, parent, w, norm)
        kc = compact(flat(k), keep, src, parent, w, norm)
    to_bh = lambda t: np.asarray(t, np.float64).reshape(1, -1, heads, hd).transpose(0, 2, 1, 3)
    log_mass = np.log(np.asarray(norm, np.float32)).astype(np.float32)
    o = mass_bias_attention(to_bh(qc), to_bh(kc), to_bh(vc), log_mass)  # [1,H,Nq,hd]
    if dense_special:
        special = np.asarray(plan["special"], np.int64)
        exact = mass_bias_attention(to_bh(flat(q)[special]), to_bh(flat(k)), to_bh(flat(v)), None)
        out_index = special if preserve_queries else np.asarray(plan["special_compact"], np.int64)
        o[:, :, out_index] = exact
    o = o.transpose(0, 2, 1, 3).reshape(-1, dim)
    y = o @ np.asarray(params["proj.weight"], np.float64).T + np.asarray(params["proj.bias"], np.float64)
    y = y.astype(np.float32)
    if preserve_queries:
        return y
    return restore(y, keep, src, parent, w, N)


# ------------------------------------------------------------------------------------------
# a10: hard-merge TokenPlan
# ------------------------------------------------------------------------------------------
def token_plan_compact(value, inverse, kept: int, pool_mask=None, dtype: str = "f32") -> np.ndarray:
    """Restates TokenPlan.compact (merge=True), token_merging.py:176-191: fp32 sums of the
    contributing tokens per compact index (index order) divided by their counts.
    value [N, C], inverse [N]."""
    value = np.asarray(value, dtype=np.float32)
    inverse = np.asarray(inverse, dtype=np.int64)
    contribution = np.ones(len(inverse), np.float32) if pool_mask is None else np.asarray(pool_mask, np.float32)
    sums = np.zeros((kept, value.shape[1]), dtype=np.float32)
    counts = np.zeros(kept, dtype=np.float32)
    for n in range(len(inverse)):
        sums[inverse[n]] = (sums[inverse[n]] + value[n] * contribution[n]).astype(np.float32)
        counts[inverse[n]] += contribution[n]
    with np.errstate(divide="ignore", invalid="ignore"):
        out = (sums / counts[:, None]).astype(np.float32)
    return round_to(out, dtype)


def token_plan_restore(value, inverse) -> np.ndarray:
    """Restates TokenPlan.restore, token_merging.py:193-196 (gather by inverse)."""
    return np.asarray(value)[np.asarray(inverse, dtype=np.int64)]


# ------------------------------------------------------------------------------------------
# a9/a11: similarity ranking
# ------------------------------------------------------------------------------------------
def topk_scores(query_bf16, basis_bf16) -> np.ndarray:
    """bf16 GEMM with fp32 accumulation, result rounded to bf16: the score matrix of
    ``source.bf16 @ basis.bf16.T`` (vggt_omega/models/sparse_convex.py:264, 294, 546) and the
    bmm of build_fastvggt_plan (token_merging.py:1106).  Accumulated in float64 here, so a
    value that lands on a bf16 rounding boundary may differ by one bf16 ulp."""
    q = np.asarray(query_bf16, dtype=np.float64)
    b = np.asarray(basis_bf16, dtype=np.float64)
    return round_bf16((q @ b.T).astype(np.float32))


def similarity_topk(query_bf16, basis_bf16, k: int):
    """(values, indices) of the k highest bf16 scores per row, best first, ties to the lower
    index (the order of a stable descending sort).  Restates the ``.topk(4)`` retrieval of
    sparse_convex.py:264/294 and ``streaming_top4`` (sparse_convex_kernels.py:20-93, which
    rounds the accumulator to bf16 before ranking, :51-54)."""
    scores = topk_scores(query_bf16, basis_bf16)
    order = np.argsort(-scores, axis=1, kind="stable")[:, :k]
    return np.take_along_axis(scores, order, axis=1), order


# ------------------------------------------------------------------------------------------
# a9: FastVGGT plan
# ------------------------------------------------------------------------------------------
def torch_cpu_rand(seed: int, count: int) -> np.ndarray:
    """The float32 stream of ``torch.rand(count, generator=torch.Generator('cpu').manual_seed(seed))``:
    MT19937 seeded with ``seed``, each float built from the low 24 bits of one 32-bit draw."""
    rs = np.random.RandomState(seed)
    key, pos = rs.get_state()[1], rs.get_state()[2]
    mt = np.random.MT19937()
    mt.state = {"bit_generator": "MT19937", "state": {"key": key, "pos": pos}}
    raw = mt.random_raw(count).astype(np.uint64)
    return ((raw & ((1 << 24) - 1)).astype(np.float64) * 2.0 ** -24).astype(np.float32)


def normalize_bf16(x, eps: float = 1e-12) -> np.ndarray:
    """``F.normalize(x.float(), dim=-1, eps=eps).to(bfloat16)`` (token_merging.py:1102-1103;
    eps 1e-8 in sparse_convex.py:1791-1793): the row norm in float64 rounded to fp32, clamped at
    eps, the fp32 quotient rounded to bf16."""
    x = np.asarray(x, dtype=np.float32)
    x64 = x.astype(np.float64)
    n = np.sqrt((x64 * x64).sum(axis=1, keepdims=True)).astype(np.float32)
    return round_bf16((x / np.maximum(n, np.float32(eps))).astype(np.float32))


def _patch_ids(frames, tokens_per_frame, patch_token_start):
    patches = tokens_per_frame - patch_token_start
    return (np.arange(frames)[:, None] * tokens_per_frame + patch_token_start + np.arange(patches)[None, :])


def fastvggt_plan(tokens, *, frames, tokens_per_frame, patch_token_start, patch_hw,
                  merge_ratio=0.9, protect_ratio=0.10, seed=0):
    """Restates build_fastvggt_plan, vggt_omega/models/token_merging.py:1045-1122, for batch 1:
    frame 0's patches and one seeded random patch per 2x2 cell of every later frame are
    destinations; special tokens, frame 0 and every (total // count)-th token are protected;
    every other patch is a source.  Sources are ranked by their best bf16 cosine score against
    all destinations (stable, descending) and the top ``removed`` are merged into their
    argmax destination.  tokens [N, D].  Returns (keep [K], inverse [N], best [S],
    target [S], source_indices [S], destination_indices [Dn])."""
    tokens = np.asarray(tokens, dtype=np.float32)
    total = tokens.shape[0]
    height, width = patch_hw
    patches = height * width
    if total != frames * tokens_per_frame or patch_token_start + patches != tokens_per_frame:
        raise ValueError("Invalid Omega FastVGGT frame/patch/special-token layout")
    identity = np.arange(total)
    if frames == 1 or merge_ratio == 0:
        return identity, identity, None, None, None, None
    patch_ids = _patch_ids(frames, tokens_per_frame, patch_token_start)
    destination = np.zeros(total, dtype=bool)
    destination[patch_ids[0]] = True
    rows = np.arange(0, height, 2)
    cols = np.arange(0, width, 2)
    choices = torch_cpu_rand(seed, (frames - 1) * len(rows) * len(cols) * 2).reshape(
        frames - 1, len(rows), len(cols), 2)
    row = rows[None, :, None] + (choices[..., 0] * np.minimum(height - rows, 2)[None, :, None].astype(np.float32)).astype(np.int64)
    col = cols[None, None, :] + (choices[..., 1] * np.minimum(width - cols, 2)[None, None, :].astype(np.float32)).astype(np.int64)
    selected = (row * width + col).reshape(frames - 1, -1)
    destination[np.take_along_axis(patch_ids[1:], selected, axis=1).reshape(-1)] = True
    protected = np.ones(total, dtype=bool)
    protected[patch_ids.reshape(-1)] = False
    protected[patch_ids[0]] = True
    count = int(total * protect_ratio)
    if count:
        protected[np.arange(0, total, max(1, total // count))[:count]] = True
    source_indices = np.nonzero(~(destination | protected))[0]
    destination_indices = np.nonzero(destination)[0]
    removed = fastvggt_removed(total, merge_ratio, source_indices.size)
    if removed == 0:
        return identity, identity, None, None, None, None

    src = normalize_bf16(tokens[source_indices])
    dst = normalize_bf16(tokens[destination_indices])
    values, idx = similarity_topk(src, dst, 1)
    best, targets = values[:, 0], idx[:, 0]
    keep, inverse = fastvggt_assign(best, targets, source_indices, destination_indices, total, removed)
    return keep, inverse, best, targets, source_indices, destination_indices


def fastvggt_removed(total: int, merge_ratio: float, sources: int) -> int:
    """Number of merged sources, token_merging.py:1096."""
    return min(int(total * merge_ratio), sources)


def fastvggt_assign(best, targets, source_indices, destination_indices, total: int, removed: int):
    """The ranking half of build_fastvggt_plan (token_merging.py:1112-1121): sources sorted by
    their best score, descending and stable; the first ``removed`` are merged into their
    argmax destination.  Returns (keep [total - removed], inverse [total])."""
    best = np.asarray(best, dtype=np.float32)
    targets = np.asarray(targets, dtype=np.int64)
    source_indices = np.asarray(source_indices, dtype=np.int64)
    destination_indices = np.asarray(destination_indices, dtype=np.int64)
    identity = np.arange(total)
    ranked = np.argsort(-best, kind="stable")
    removed_source = source_indices[ranked[:removed]]
    target_original = destination_indices[targets[ranked[:removed]]]
    kept_mask = np.ones(total, dtype=bool)
    kept_mask[removed_source] = False
    keep = identity[kept_mask]
    original_to_compact = np.full(total, -1, dtype=np.int64)
    original_to_compact[keep] = np.arange(keep.size)
    inverse = original_to_compact.copy()
    inverse[removed_source] = original_to_compact[target_original]
    return keep, inverse


# ------------------------------------------------------------------------------------------
# next tier: four-support simplex solvers
# ------------------------------------------------------------------------------------------
def simplex_project(values) -> np.ndarray:
    """Euclidean projection of rows of 4 onto the probability simplex (the threshold form of
    token_merging.py:429-437 and sparse_convex_kernels.py:258-275)."""
    v = np.asarray(values, dtype=np.float32)
    s = -np.sort(-v, axis=-1)
    cssv = np.cumsum(s, axis=-1, dtype=np.float32) - np.float32(1.0)
    ranks = np.arange(1, v.shape[-1] + 1, dtype=np.float32)
    active = s > cssv / ranks
    rho = np.maximum(active.sum(axis=-1), 1) - 1
    theta = np.take_along_axis(cssv, rho[..., None], axis=-1)[..., 0] / (rho.astype(np.float32) + 1)
    return np.maximum(v - theta[..., None], 0).astype(np.float32)


def projected_gradient(gram, rhs, steps: int = 32) -> np.ndarray:
    """Restates four_support_projected_gradient (sparse_convex_kernels.py:214-296) and the
    "adaptive_convex" loop of sparse_convex.py:146-156: a = e0, step = 0.95 / max(max row
    abs-sum, 1e-4), ``steps`` projected-gradient iterations.  gram [R,4,4], rhs [R,4]."""
    gram = np.asarray(gram, dtype=np.float32)
    rhs = np.asarray(rhs, dtype=np.float32)
    step = (np.float32(0.95) / np.maximum(np.abs(gram).sum(axis=-1).max(axis=-1), np.float32(1e-4))).astype(np.float32)
    alpha = np.zeros_like(rhs)
    alpha[:, 0] = 1
    for _ in range(steps):
        grad = (np.einsum("rij,rj->ri", gram, alpha) - rhs).astype(np.float32)
        alpha = simplex_project((alpha - step[:, None] * grad).astype(np.float32))
    return alpha


_ACTIVE_IDS = np.array([
    [0, 0, 0, 0], [1, 1, 1, 1], [2, 2, 2, 2], [3, 3, 3, 3],
    [0, 1, 1, 1], [0, 2, 2, 2], [0, 3, 3, 3], [1, 2, 2, 2], [1, 3, 3, 3], [2, 3, 3, 3],
    [0, 1, 2, 2], [0, 1, 3, 3], [0, 2, 3, 3], [1, 2, 3, 3], [0, 1, 2, 3]])
_ACTIVE_COUNT = np.array([1, 1, 1, 1, 2, 2, 2, 2, 2, 2, 3, 3, 3, 3, 4])


def active_set(gram, rhs, ridge: float = 1e-4) -> np.ndarray:
    """Restates four_support_active_set (sparse_convex_kernels.py:96-212, :332-353): for each of
    the 15 active sets eliminate the last active variable, solve the reduced system (Cramer,
    ridge on the Gram diagonal), drop infeasible / singular candidates, keep the first lowest
    objective, normalise, and fall back to the one-hot first support when its cosine is
    higher.  Float64 arithmetic."""
    G = np.asarray(gram, dtype=np.float64)
    R = np.asarray(rhs, dtype=np.float64)
    rows = len(G)
    best = np.zeros((rows, 4))
    best_obj = np.full(rows, np.inf)
    chosen = np.zeros(rows, dtype=bool)
    ge = lambda a, b: G[:, a, b] + (ridge if a == b else 0.0)
    for s in range(15):
        cnt = _ACTIVE_COUNT[s]
        i0, i1, i2 = _ACTIVE_IDS[s, :3]
        p = _ACTIVE_IDS[s, cnt - 1]
        hp = ge(p, p)
        rp = R[:, p]
        h = lambda a, b: ge(a, b) - ge(a, p) - ge(p, b) + hp
        h00, h01, h02 = h(i0, i0), h(i0, i1), h(i0, i2)
        h10, h11, h12 = h(i1, i0), h(i1, i1), h(i1, i2)
        h20, h21, h22 = h(i2, i0), h(i2, i1), h(i2, i2)
        c0 = R[:, i0] - rp - ge(i0, p) + hp
        c1 = R[:, i1] - rp - ge(i1, p) + hp
        c2 = R[:, i2] - rp - ge(i2, p) + hp
        safe = lambda d: np.where(np.abs(d) > 1e-12, d, 1.0)
        one_x = c0 / safe(h00)
        det2 = h00 * h11 - h01 * h10
        two_x = (c0 * h11 - h01 * c1) / safe(det2)
        two_y = (h00 * c1 - h10 * c0) / safe(det2)
        det3 = h00 * (h11 * h22 - h12 * h21) - h01 * (h10 * h22 - h12 * h20) + h02 * (h10 * h21 - h11 * h20)
        three_x = (c0 * (h11 * h22 - h12 * h21) - h01 * (c1 * h22 - h12 * c2) + h02 * (c1 * h21 - h11 * c2)) / safe(det3)
        three_y = (h00 * (c1 * h22 - h12 * c2) - c0 * (h10 * h22 - h12 * h20) + h02 * (h10 * c2 - c1 * h20)) / safe(det3)
        three_z = (h00 * (h11 * c2 - c1 * h21) - h01 * (h10 * c2 - c1 * h20) + c0 * (h10 * h21 - h11 * h20)) / safe(det3)
        dim = cnt - 1
        zero = np.zeros(rows)
        b0 = {0: zero, 1: one_x, 2: two_x, 3: three_x}[dim]
        b1 = {0: zero, 1: zero, 2: two_y, 3: three_y}[dim]
        b2 = three_z if dim == 3 else zero
        ap = 1.0 - b0 - b1 - b2
        a = np.zeros((rows, 4))
        for q in range(4):
            a[:, q] = (b0 if i0 == q else 0) + (b1 if i1 == q else 0) + (b2 if i2 == q else 0) + (ap if p == q else 0)
        stable = {0: np.ones(rows, bool), 1: np.abs(h00) > 1e-12, 2: np.abs(det2) > 1e-12, 3: np.abs(det3) > 1e-12}[dim]
        feasible = stable & (a >= -1e-5).all(axis=1)
        a = np.maximum(a, 0)
        a = a / np.maximum(a.sum(axis=1, keepdims=True), 1e-12)
        obj = np.einsum("ri,rij,rj->r", a, G, a) - 2 * (a * R).sum(axis=1)
        obj = np.where(feasible, obj, np.inf)
        take = (~chosen) | (obj < best_obj)
        best[take] = a[take]
        best_obj[take] = obj[take]
        chosen |= take
    best = best / np.maximum(best.sum(axis=1, keepdims=True), 1e-12)
    num = (best * R).sum(axis=1)
    sq = np.einsum("ri,rij,rj->r", best, G, best)
    cosine = num / np.sqrt(np.maximum(sq, 1e-12))
    single = R[:, 0] > cosine
    best[single] = np.array([1.0, 0.0, 0.0, 0.0])
    return best.astype(np.float32)
