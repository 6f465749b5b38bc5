"""Offline balanced clustering of an LM head and the clustering cache writer.

The reference reads ``<model>/<cache_dir>/clustering_cache.safetensors``
(``centroids`` [D, K], ``cluster_assignments`` [V] int64; flash_head.py:41-78)
and requires every cluster to hold the same number of tokens
(flash_head.py:108-113), but ships no tool that makes such a file
(README.md:65). This module makes one from the LM-head weight alone:

``balanced_clusters(weight, cap)``
    Spherical balanced k-means on the unit-normalised rows of the [V, D]
    weight: K = V / cap clusters of exactly ``cap`` tokens each.

    * Initial partition by recursive balanced bisection: a set of k * cap
      tokens is split into k1 * cap and (k - k1) * cap tokens (k1 = k // 2)
      by their projection on the set's leading principal direction (a few
      power iterations); K leaves of cap tokens each.
    * Refinement: centroids = normalised member means; every token lists its
      ``n_candidates`` most similar centroids; capacity-constrained
      assignment in rounds (each unassigned token proposes to its best
      cluster that still has room, each cluster accepts its best proposers
      up to its remaining capacity, rejected tokens move down their list);
      tokens whose lists run out are placed by the same rounds over all
      clusters with room. Stops when no assignment changes or after
      ``iters`` rounds.

    Returns the assignments and the centroids in the cache layout: the
    per-cluster means of the raw weight rows, [D, K] float32 (FlashHead
    normalises them for stage 1 and uses them raw for sampling).

``save_clustering_cache(cache_dir, centroids, assignments)``
    Writes the two tensors in the reference's file layout.

``build_clustering_cache(model, cache_dir, cap)``
    Reads the LM-head weight of a checkpoint (``loading.LM_HEAD_KEYS``),
    clusters it and writes the cache.

Everything runs in PyTorch on ``device`` (CPU by default; a CUDA device
speeds up the similarity products of large heads). This is offline tooling:
nothing here is on the decode path.
"""

from __future__ import annotations

import os
from typing import Optional, Tuple

import numpy as np
import torch

CACHE_FILE = "clustering_cache.safetensors"


def _unit_rows(w: torch.Tensor) -> torch.Tensor:
    x = w.to(torch.float32)
    n = x.norm(dim=1, keepdim=True)
    return x / n.clamp_min(1e-30)


def _leading_direction(x: torch.Tensor, gen: torch.Generator, n_power: int) -> torch.Tensor:
    """Leading principal direction of the rows of x (centred), by power
    iteration from a seeded random start."""
    xc = x - x.mean(dim=0, keepdim=True)
    v = torch.randn(x.shape[1], generator=gen, device="cpu").to(x.device)
    v = v / v.norm().clamp_min(1e-30)
    for _ in range(n_power):
        v = xc.t() @ (xc @ v)
        nv = v.norm()
        if float(nv) == 0.0:
            break
        v = v / nv
    return xc @ v


def _bisect(x: torch.Tensor, cap: int, gen: torch.Generator, n_power: int) -> np.ndarray:
    """Initial partition of the V rows of x into V / cap groups of cap rows by
    recursive balanced bisection along principal directions."""
    V = x.shape[0]
    K = V // cap
    labels = np.empty(V, dtype=np.int64)
    stack = [(np.arange(V), K, 0)]  # (token ids, clusters to make, first cluster id)
    while stack:
        ids, k, c0 = stack.pop()
        if k == 1:
            labels[ids] = c0
            continue
        k1 = k // 2
        proj = _leading_direction(x[torch.from_numpy(ids).to(x.device)], gen, n_power)
        order = np.argsort(proj.cpu().numpy(), kind="stable")
        cut = k1 * cap
        stack.append((ids[order[:cut]], k1, c0))
        stack.append((ids[order[cut:]], k - k1, c0 + k1))
    return labels


def _propose_accept(cand: np.ndarray, score: np.ndarray, room: np.ndarray,
                    assign: np.ndarray, tokens: np.ndarray) -> np.ndarray:
    """Capacity-constrained assignment of `tokens` in rounds over their
    candidate lists (cand/score rows in the same order as `tokens`, best
    first). Updates `room` and `assign`; returns the tokens left unassigned."""
    n, m = cand.shape
    ptr = np.zeros(n, dtype=np.int64)
    live = np.arange(n)
    while live.size:
        # move each live token past clusters that are full
        while True:
            c = cand[live, ptr[live]]
            full = room[c] <= 0
            if not full.any():
                break
            ptr[live[full]] += 1
            keep = ptr[live] < m
            live = live[keep]
            if not live.size:
                break
        if not live.size:
            break
        c = cand[live, ptr[live]]
        s = score[live, ptr[live]]
        # per cluster, accept the best proposers up to its room (ties: token id)
        order = np.lexsort((tokens[live], -s, c))
        c_sorted = c[order]
        first = np.searchsorted(c_sorted, c_sorted, side="left")
        rank = np.arange(order.size) - first
        ok = rank < room[c_sorted]
        acc = live[order[ok]]
        assign[tokens[acc]] = cand[acc, ptr[acc]]
        np.subtract.at(room, cand[acc, ptr[acc]], 1)
        rej = live[order[~ok]]
        ptr[rej] += 1
        live = rej[ptr[rej] < m]
    return tokens[assign[tokens] < 0]


def _topk_chunked(x: torch.Tensor, c: torch.Tensor, k: int, chunk: int):
    vals, idx = [], []
    for i in range(0, x.shape[0], chunk):
        s = x[i:i + chunk] @ c.t()
        v, j = torch.topk(s, k, dim=1)
        vals.append(v.cpu())
        idx.append(j.cpu())
    return torch.cat(vals).numpy(), torch.cat(idx).numpy()


def _balanced_assign(x: torch.Tensor, cent: torch.Tensor, cap: int, n_candidates: int,
                     chunk: int) -> np.ndarray:
    V, K = x.shape[0], cent.shape[0]
    m = min(n_candidates, K)
    score, cand = _topk_chunked(x, cent, m, chunk)
    assign = np.full(V, -1, dtype=np.int64)
    room = np.full(K, cap, dtype=np.int64)
    left = _propose_accept(cand, score, room, assign, np.arange(V))
    if left.size:  # lists ran out: rank every cluster that still has room
        open_ids = np.nonzero(room > 0)[0]
        s = (x[torch.from_numpy(left).to(x.device)] @
             cent[torch.from_numpy(open_ids).to(x.device)].t()).cpu().numpy()
        order = np.argsort(-s, axis=1, kind="stable")
        left = _propose_accept(open_ids[order], np.take_along_axis(s, order, axis=1), room,
                               assign, left)
    if left.size or (room != 0).any():
        raise RuntimeError("balanced assignment left tokens or room unassigned")
    return assign


def _centroids(x: torch.Tensor, assign: np.ndarray, K: int) -> torch.Tensor:
    a = torch.from_numpy(assign).to(x.device)
    s = torch.zeros(K, x.shape[1], dtype=torch.float32, device=x.device)
    s.index_add_(0, a, x.to(torch.float32))
    return s / float(x.shape[0] // K)


def balanced_clusters(weight: torch.Tensor, cap: int = 16, iters: int = 10,
                      n_candidates: int = 16, seed: int = 0, n_power: int = 8,
                      device: Optional[torch.device] = None,
                      chunk: int = 8192) -> Tuple[torch.Tensor, torch.Tensor]:
    """K = V / cap clusters of exactly `cap` tokens of the [V, D] LM-head
    weight. Returns (assignments [V] int64, centroids [D, K] float32), both
    on the CPU, in the ``clustering_cache.safetensors`` layout."""
    if weight.ndim != 2:
        raise ValueError(f"weight must be [V, D], got {tuple(weight.shape)}")
    V, D = weight.shape
    if cap < 1 or V % cap != 0:
        raise ValueError(f"vocabulary {V} is not a multiple of the cluster size {cap}")
    K = V // cap
    dev = torch.device(device) if device is not None else weight.device
    w = weight.to(dev)
    x = _unit_rows(w)
    gen = torch.Generator(device="cpu").manual_seed(seed)
    assign = _bisect(x, cap, gen, n_power)
    for _ in range(iters):
        cent = _unit_rows(_centroids(x, assign, K))
        new = _balanced_assign(x, cent, cap, n_candidates, chunk)
        changed = int((new != assign).sum())
        assign = new
        if changed == 0:
            break
    centroids = _centroids(w.to(torch.float32), assign, K).t().contiguous().cpu()
    return torch.from_numpy(assign), centroids


def save_clustering_cache(cache_dir: str, centroids: torch.Tensor,
                          assignments: torch.Tensor) -> str:
    """Write ``<cache_dir>/clustering_cache.safetensors`` (``centroids`` [D, K]
    float32, ``cluster_assignments`` [V] int64), the file FlashHead reads."""
    from safetensors.torch import save_file
    if centroids.ndim != 2 or assignments.ndim != 1:
        raise ValueError("centroids must be [D, K] and assignments [V]")
    K = centroids.shape[1]
    a = assignments.to(torch.int64).cpu()
    if int(a.min()) < 0 or int(a.max()) >= K:
        raise ValueError(f"assignments outside 0..{K - 1}")
    counts = torch.bincount(a, minlength=K)
    if int(counts.min()) != int(counts.max()):
        raise ValueError(f"clusters are not balanced: sizes {sorted(set(counts.tolist()))}")
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, CACHE_FILE)
    save_file({"centroids": centroids.to(torch.float32).contiguous().cpu(),
               "cluster_assignments": a.contiguous()}, path)
    return path


def build_clustering_cache(model: str, cache_dir: str, cap: int = 16, iters: int = 10,
                           seed: int = 0, device: Optional[str] = None) -> str:
    """Cluster the LM head of checkpoint `model` (a local directory or a hub
    id) and write the cache into `cache_dir`; returns the file path. The
    model's config.json names the directory in ``flash_head_cache_dir``."""
    from .assets import ModelFiles, lm_head_weight
    w, _ = lm_head_weight(ModelFiles(model))
    if w.shape[0] < w.shape[1]:
        w = w.t()
    assign, cent = balanced_clusters(w, cap=cap, iters=iters, seed=seed, device=device)
    return save_clustering_cache(cache_dir, cent, assign)
