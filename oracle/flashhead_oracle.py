"""CPU oracle for FlashHead's decode-step LM-head path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU legs of ``bench.py`` may import this module, and only as the checker or
as the timed CPU baseline. The product path (the ``flash_head`` package and
its CUDA library) never imports it and has no CPU fallback.

A numpy restatement of the reference algorithm (embedl/flash-head,
``src/flash_head/flash_head.py`` and ``src/flash_head/fused.py``) with float64
accumulation, so it serves as the numerical truth that the tolerance rule is
applied against:

  * greedy token ids must be identical unless the two competing logits are
    within ``rtol`` (1e-2 relative) of each other;
  * probe sets must be identical unless the differing clusters' centroid
    scores are within ``rtol`` of the p-th score;
  * sampling must be distribution-equivalent (chi-squared, see tests).

Parity pin: ``tests/test_oracle.py`` checks this module against golden
vectors produced by running the reference's own ``FlashHead`` on CPU
(``tests/golden/make_golden.py``).

Conventions shared with the CUDA kernels (so results can be compared exactly
where the arithmetic allows):

  * probe selection = the p clusters with the largest score, ties broken
    towards the smaller cluster id; probe lists are returned sorted by id;
  * greedy winner = largest fp32 logit, ties broken towards the smaller
    vocab id (fused.py:148-163 packs ``~vocab_id`` under the logit key);
  * sampling = Gumbel-top-p over ``score / T`` for clusters and Gumbel-max
    over ``logit / T`` for candidate tokens, with Philox-4x32-10 uniforms
    keyed by (seed, offset, stage, row, element id).
"""

from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------
# Number formats
# ----------------------------------------------------------------------------


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen raw bf16 bit patterns (uint16) to float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 with round-to-nearest-even, returning uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = 0x7FFF + ((u >> 16) & 1)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, np.uint16(0x7FC0), out)
    return out


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def _fp8_e4m3_table() -> np.ndarray:
    """Value of every e4m3 (OCP 'fn' variant) byte: bias 7, no infinities,
    S.1111.111 is NaN, subnormals 2^-6 * m/8."""
    vals = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            vals[b] = np.nan
        elif e == 0:
            vals[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            vals[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


FP8_E4M3_VALUES = _fp8_e4m3_table()


def fp8_e4m3_decode(raw: np.ndarray) -> np.ndarray:
    """Decode raw e4m3 bytes (uint8) to float32."""
    return FP8_E4M3_VALUES[raw.astype(np.uint8)]


# ----------------------------------------------------------------------------
# Load-time layout (flash_head.py:81-118, :136-188)
# ----------------------------------------------------------------------------


def vocab_maps_from_assignments(assign: np.ndarray, n_clusters: int) -> np.ndarray:
    """[K, cap] vocab ids per cluster, ascending inside each cluster.

    Follows get_flash_head_parameters (flash_head.py:100-113): cluster i lists
    ``where(assign == i)`` (ascending ids) and every cluster must have the same
    size, else ValueError.
    """
    assign = np.asarray(assign, dtype=np.int64)
    counts = np.bincount(assign, minlength=n_clusters)
    sizes = set(counts.tolist())
    if len(sizes) != 1 or len(counts) != n_clusters:
        raise ValueError(
            f"FlashHead requires balanced clusters; got cluster sizes {sorted(sizes)}")
    order = np.argsort(assign, kind="stable")
    return order.reshape(n_clusters, int(counts[0]))


def normalized_cluster_weight(centroids_dk: np.ndarray) -> np.ndarray:
    """Stage-1 matrix: centroid columns L2-normalised, transposed to [K, D]
    (flash_head.py:158). Computed in float32 as the loader does."""
    c = np.asarray(centroids_dk, dtype=np.float32)
    norm = np.sqrt((c.astype(np.float64) ** 2).sum(axis=0, keepdims=True)).astype(np.float32)
    return np.ascontiguousarray((c / norm).T)


def permute_weight(weight_vd: np.ndarray, vocab_maps: np.ndarray) -> np.ndarray:
    """w_perm[K, cap, D] = weight rows in cluster order (flash_head.py:162-168)."""
    K, cap = vocab_maps.shape
    return weight_vd[vocab_maps.reshape(-1)].reshape(K, cap, -1)


# ----------------------------------------------------------------------------
# Stage 1: centroid scores and probe selection (flash_head.py:190-221)
# ----------------------------------------------------------------------------


def cluster_scores(h: np.ndarray, cluster_w: np.ndarray,
                   row_scale: np.ndarray | None = None) -> np.ndarray:
    """scores[B, K] = h @ cluster_w^T (float64), times an optional per-row scale."""
    s = np.asarray(h, dtype=np.float64) @ np.asarray(cluster_w, dtype=np.float64).T
    if row_scale is not None:
        s = s * np.asarray(row_scale, dtype=np.float64)[None, :]
    return s


def top_probes(scores: np.ndarray, p: int) -> np.ndarray:
    """The p largest scores of one row, ties -> smaller cluster id; sorted by id.

    The reference uses ``torch.topk(sorted=False)`` (flash_head.py:214) whose
    choice among tied scores is unspecified; this fixes the tie rule.
    """
    scores = np.asarray(scores)
    K = scores.shape[0]
    if not 0 < p <= K:
        raise ValueError(f"n_probes={p} outside 1..{K}")
    order = np.lexsort((np.arange(K), -scores))
    return np.sort(order[:p])


def probe_set_within_tolerance(mine: np.ndarray, ref: np.ndarray,
                               scores: np.ndarray, rtol: float = 1e-2) -> bool:
    """True if two probe sets differ only in clusters whose scores are within
    ``rtol`` (relative to the boundary score) of the p-th score."""
    mine, ref = set(int(x) for x in mine), set(int(x) for x in ref)
    if len(mine) != len(ref):
        return False
    diff = mine.symmetric_difference(ref)
    if not diff:
        return True
    p = len(ref)
    kth = np.sort(scores)[::-1][p - 1]
    band = rtol * max(abs(kth), 1e-30)
    return all(abs(scores[c] - kth) <= band for c in diff)


def probe_rule_vs_reference_list(mine: np.ndarray, ref_probes: np.ndarray, top_vals: np.ndarray,
                                 top_ids: np.ndarray, rtol: float = 1e-2):
    """The probe-set rule judged on the reference's own scores.

    top_vals / top_ids: the reference's largest bf16 scores of the row
    (descending) with their cluster ids, at least p + 1 of them; every cluster
    not listed scores at most top_vals[-1]. Returns (ok, recall, n_outside):
    ok when every cluster in exactly one of the two sets scores within rtol of
    the p-th score (a cluster of `mine` missing from the list counts as
    outside the band unless the list's last score is still inside it);
    recall = |mine & ref| / p.
    """
    mine = set(int(x) for x in mine)
    ref = set(int(x) for x in ref_probes)
    p = len(ref)
    kth = float(top_vals[p - 1])
    band = rtol * max(abs(kth), 1e-30)
    score = {int(c): float(v) for c, v in zip(top_ids, top_vals)}
    last = float(top_vals[-1])
    outside = 0
    for c in mine.symmetric_difference(ref):
        v = score.get(c)
        if v is None:
            outside += not (abs(last - kth) <= band)
        else:
            outside += not (abs(v - kth) <= band)
    recall = len(mine & ref) / p
    return len(mine) == p and outside == 0, recall, outside


# ----------------------------------------------------------------------------
# Stage 2: block-sparse logits + argmax (fused.py:119-188, flash_head.py:223-261)
# ----------------------------------------------------------------------------


def candidate_logits(h: np.ndarray, w_perm: np.ndarray, vocab_maps: np.ndarray,
                     probes: np.ndarray, special_ids=()) -> tuple[np.ndarray, np.ndarray]:
    """Vocab ids and float64 logits of every candidate of one row: the tokens of
    the probed clusters plus the special tokens (deduplicated, ascending id)."""
    K, cap, D = w_perm.shape
    probes = np.asarray(probes, dtype=np.int64)
    slots = (probes[:, None] * cap + np.arange(cap)[None, :]).reshape(-1)
    vids = vocab_maps.reshape(-1)[slots]
    if len(special_ids):
        flat = vocab_maps.reshape(-1)
        inv = np.empty_like(flat)
        inv[flat] = np.arange(flat.size)
        sp = np.asarray(special_ids, dtype=np.int64)
        slots = np.concatenate([slots, inv[sp]])
        vids = np.concatenate([vids, sp])
    vids, first = np.unique(vids, return_index=True)
    slots = slots[first]
    rows = w_perm.reshape(K * cap, D)[slots].astype(np.float64)
    return vids, rows @ np.asarray(h, dtype=np.float64)


def argmax_smallest_id(vids: np.ndarray, logits: np.ndarray) -> tuple[int, float]:
    """Largest logit, ties -> smallest vocab id."""
    best = logits.max()
    cand = vids[logits == best]
    return int(cand.min()), float(best)


def greedy_token(h, w_perm, vocab_maps, cluster_w, p, row_scale=None, special_ids=()):
    """Full greedy step for one row: (token, probes, scores)."""
    scores = cluster_scores(h[None, :], cluster_w, row_scale)[0]
    probes = top_probes(scores, p)
    vids, logits = candidate_logits(h, w_perm, vocab_maps, probes, special_ids)
    tok, _ = argmax_smallest_id(vids, logits)
    return tok, probes, scores


def dense_argmax(h: np.ndarray, weight_vd: np.ndarray) -> int:
    """Full-vocabulary greedy token (flash_head.py:263-275, :292-301)."""
    logits = np.asarray(weight_vd, dtype=np.float64) @ np.asarray(h, dtype=np.float64)
    return int(np.argmax(logits))


def token_within_tolerance(mine: int, ref: int, logit_of, rtol: float = 1e-2) -> bool:
    """Greedy rule: identical ids, or the two ids' logits within rtol."""
    if int(mine) == int(ref):
        return True
    a, b = float(logit_of(int(mine))), float(logit_of(int(ref)))
    return abs(a - b) <= rtol * max(abs(a), abs(b), 1e-30)


# ----------------------------------------------------------------------------
# Packed (key, id) words (fused.py:148-163)
# ----------------------------------------------------------------------------


def mono_key_u32(x: np.ndarray) -> np.ndarray:
    """Order-preserving map of float32 onto uint32 (unsigned compare)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    return np.where(u & 0x80000000, ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def pack_u64(x: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """(mono(x) << 32) | (0xFFFFFFFF - id): unsigned max = largest x, then smallest id."""
    return (mono_key_u32(x).astype(np.uint64) << np.uint64(32)) | (
        np.uint64(0xFFFFFFFF) - np.asarray(ids, dtype=np.uint64))


def unpack_id(packed: np.ndarray) -> np.ndarray:
    return (np.uint64(0xFFFFFFFF) - (np.asarray(packed, dtype=np.uint64) & np.uint64(0xFFFFFFFF))).astype(np.int64)


def reference_signed_pack(x: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """The reference's signed int64 word (fused.py:158-163), for cross-checks."""
    bits = np.asarray(x, dtype=np.float32).view(np.int32).astype(np.int64)
    key = np.where(bits >= 0, bits, (~bits) ^ np.int64(-2147483648))
    key = key.astype(np.int32).astype(np.int64)
    return (key << 32) | ((~np.asarray(ids, dtype=np.int64)) & 0xFFFFFFFF)


# ----------------------------------------------------------------------------
# Philox-4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy
# as 1, 2, 3", SC'11) and Gumbel noise
# ----------------------------------------------------------------------------

_PHILOX_M0 = np.uint64(0xD2511F53)
_PHILOX_M1 = np.uint64(0xCD9E8D57)
_PHILOX_W0 = np.uint32(0x9E3779B9)
_PHILOX_W1 = np.uint32(0xBB67AE85)
_MASK32 = np.uint64(0xFFFFFFFF)

STAGE_CLUSTERS = 1
STAGE_TOKENS = 2


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Ten Philox rounds on arrays of 32-bit counters; returns four uint32 arrays."""
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint32).copy() for c in (c0, c1, c2, c3))
    k0 = np.uint32(k0)
    k1 = np.uint32(k1)
    for _ in range(10):
        p0 = _PHILOX_M0 * c0.astype(np.uint64)
        p1 = _PHILOX_M1 * c2.astype(np.uint64)
        hi0 = (p0 >> np.uint64(32)).astype(np.uint32)
        lo0 = (p0 & _MASK32).astype(np.uint32)
        hi1 = (p1 >> np.uint64(32)).astype(np.uint32)
        lo1 = (p1 & _MASK32).astype(np.uint32)
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        k0 = np.uint32((int(k0) + int(_PHILOX_W0)) & 0xFFFFFFFF)
        k1 = np.uint32((int(k1) + int(_PHILOX_W1)) & 0xFFFFFFFF)
    return c0, c1, c2, c3


def philox_uniform(seed: int, offset: int, stage: int, row, ids) -> np.ndarray:
    """float32 uniforms in (0,1) for (seed, offset, stage, row, id)."""
    ids = np.asarray(ids, dtype=np.uint64)
    row = np.broadcast_to(np.asarray(row, dtype=np.uint64), ids.shape)
    c0 = (ids & _MASK32).astype(np.uint32)
    c1 = (row & _MASK32).astype(np.uint32)
    c2 = np.full(ids.shape, offset & 0xFFFFFFFF, dtype=np.uint32)
    c3 = np.full(ids.shape, (((offset >> 32) & 0x3FFFFFFF) | (stage << 30)) & 0xFFFFFFFF,
                 dtype=np.uint32)
    x, _, _, _ = philox4x32_10(c0, c1, c2, c3, seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
    return ((x >> np.uint32(8)).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -24)


def gumbel(seed: int, offset: int, stage: int, row, ids) -> np.ndarray:
    """Standard Gumbel noise -log(-log(u)) in float32."""
    u = philox_uniform(seed, offset, stage, row, ids)
    return -np.log(-np.log(u))


def sample_token(h, w_perm, vocab_maps, centroids_kd, p, temperature, seed, offset, row,
                 special_ids=()):
    """One sampled token for one row (flash_head.py:202-211, :326-328).

    Stage 1 draws p clusters without replacement with probabilities
    softmax(h . C / T) over the RAW centroids (Gumbel-top-p); stage 2 draws one
    candidate with probabilities softmax(logit / T) (Gumbel-max).
    Returns (token, probes).
    """
    T = np.float32(temperature)
    s = cluster_scores(h[None, :], centroids_kd)[0].astype(np.float32)
    K = s.shape[0]
    keys = s / T + gumbel(seed, offset, STAGE_CLUSTERS, row, np.arange(K))
    probes = top_probes(keys, p)
    vids, logits = candidate_logits(h, w_perm, vocab_maps, probes, special_ids)
    k2 = logits.astype(np.float32) / T + gumbel(seed, offset, STAGE_TOKENS, row, vids)
    tok, _ = argmax_smallest_id(vids, k2)
    return tok, probes


def softmax_probe_marginals(scores: np.ndarray, temperature: float) -> np.ndarray:
    """softmax(scores / T), the first-draw distribution over clusters."""
    z = np.asarray(scores, dtype=np.float64) / temperature
    z = np.exp(z - z.max())
    return z / z.sum()


def chi2_homogeneity(counts_a: np.ndarray, counts_b: np.ndarray, min_expected: float = 5.0):
    """Two-sample chi-squared test of homogeneity.

    Bins are visited in decreasing pooled count and merged greedily until
    each merged bin expects at least ``min_expected`` draws in both samples
    (a leftover partial bin joins the last one). The binning depends only on
    the pooled counts, which are exchangeable under the null hypothesis.
    Returns (statistic, dof, p_value).
    """
    from scipy.stats import chi2

    a = np.asarray(counts_a, dtype=np.float64).ravel()
    b = np.asarray(counts_b, dtype=np.float64).ravel()
    na, nb = a.sum(), b.sum()
    fa, fb = na / (na + nb), nb / (na + nb)
    tot = a + b
    order = np.argsort(-tot, kind="stable")
    order = order[tot[order] > 0]
    A, B = [], []
    ca = cb = 0.0
    for i in order:
        ca += a[i]
        cb += b[i]
        if (ca + cb) * fa >= min_expected and (ca + cb) * fb >= min_expected:
            A.append(ca)
            B.append(cb)
            ca = cb = 0.0
    if ca + cb > 0:
        if A:
            A[-1] += ca
            B[-1] += cb
        else:
            A.append(ca)
            B.append(cb)
    A, B = np.array(A), np.array(B)
    T = A + B
    EA, EB = T * fa, T * fb
    stat = float((((A - EA) ** 2) / EA).sum() + (((B - EB) ** 2) / EB).sum())
    dof = len(A) - 1
    return stat, dof, float(chi2.sf(stat, dof)) if dof > 0 else 1.0


# ----------------------------------------------------------------------------
# Speculative decoding: acceptance of draft tokens against FlashHead ids
# (patches/rejection_sampler.py:55-76)
# ----------------------------------------------------------------------------


def spec_accept(draft_ids, target_ids, bonus_ids, num_draft, max_spec_len,
                placeholder: int = -1, bonus_without_drafts: bool = True) -> np.ndarray:
    """[batch, max_spec_len + 1] int32 output token ids. Per request, drafts
    are accepted while they equal the target id at the same flat position;
    the first mismatch takes the target id and ends the row; a fully
    accepted row gets its bonus id after its drafts. The reference's loop
    adds the bonus only when the request had drafts
    (``bonus_without_drafts=False``); vLLM's own rejection sampler, which
    the library follows, adds it for rows without drafts too."""
    draft = np.asarray(draft_ids).ravel()
    target = np.asarray(target_ids).ravel()
    bonus = np.asarray(bonus_ids).ravel()
    out = np.full((len(num_draft), max_spec_len + 1), placeholder, dtype=np.int32)
    offset = 0
    for i, n in enumerate(num_draft):
        all_ok = True
        for j in range(n):
            if draft[offset + j] == target[offset + j]:
                out[i, j] = draft[offset + j]
            else:
                out[i, j] = target[offset + j]
                all_ok = False
                break
        if all_ok and (n > 0 or bonus_without_drafts):
            out[i, n] = bonus[i]
        offset += n
    return out
