"""Torch-CPU restatement of the reference FlashHead path, op for op.

TEST INFRASTRUCTURE ONLY (see ``flashhead_oracle.py``): imported by tests as
a checker and by ``bench.py`` as the timed CPU baseline / reference arm, never
by the product.

The reference (embedl/flash-head ``src/flash_head/flash_head.py``) runs on
CPU through these branches of ``FlashHead.get_next_token`` (:277-334):

  * greedy with ``use_identical_tiebreak=True`` or with special tokens:
    ``_get_top_clusters`` (:190-221) -> ``_gather_cluster_logits`` (:223-261)
    -> argmax (:329-332);
  * sampling (:202-211 then :326-328);
  * the dense branch for ``hidden_states.shape[0] > 10`` (:292-301).

The default greedy branch calls a Triton kernel (fused.py:119-188) and cannot
run on a CPU; ``block_sparse_argmax`` below restates its arithmetic (fp32
dots, per-probe max, smallest-vocab-id tie break) with torch ops.

The load-time re-layout follows ``loading.get_flash_head`` (loading.py:144-164):
parameters are derived from an fp32 copy of the weight and the whole module is
then cast to the model dtype.
"""

from __future__ import annotations

from typing import Iterable, Optional, Union

import torch


class ReferenceHeadCPU:
    """CPU FlashHead with the reference's parameters and per-step op sequence."""

    def __init__(self, weight: torch.Tensor, centroids: torch.Tensor,
                 assignments: torch.Tensor, n_probes: Optional[int] = None,
                 special_token_ids: Optional[Union[int, Iterable[int]]] = None,
                 dtype: torch.dtype = torch.bfloat16):
        V, D = weight.shape
        w32 = weight.detach().to(torch.float32)
        cent32 = centroids.detach().to(torch.float32)
        if cent32.dim() > 2:
            cent32 = cent32.squeeze(0).squeeze(0)
        K = cent32.shape[1]
        assign = assignments.to(torch.int64)
        counts = torch.bincount(assign, minlength=K)
        if counts.numel() != K or int(counts.min()) != int(counts.max()):
            raise ValueError("FlashHead requires balanced clusters; got cluster sizes "
                             f"{sorted(set(counts.tolist()))}")
        cap = int(counts[0])
        # flash_head.py:100-102 lists where(assign == i) per cluster: ascending ids.
        self.vocab_maps = torch.argsort(assign, stable=True).view(K, cap)
        self.K, self.cap, self.D, self.V = K, cap, D, V
        self.n_probes = int(n_probes if n_probes is not None else K / 16)
        self.dtype = dtype
        # flash_head.py:157-160: raw centroids [D, K] and the column-normalised
        # stage-1 matrix [K, D]; then the module cast (loading.py:164).
        self.centroids = cent32.to(dtype)
        self.cluster_w = (cent32 / cent32.norm(dim=0, keepdim=True)).t().contiguous().to(dtype)
        # flash_head.py:162-168
        self.w_perm = w32.index_select(0, self.vocab_maps.reshape(-1)).to(dtype).view(K, cap, D)
        st = [int(t) for t in ([special_token_ids] if isinstance(special_token_ids, int)
                               else list(special_token_ids or [])) if 0 <= int(t) < V]
        self.special = torch.tensor(st, dtype=torch.int64)

    # -- stage 1 ---------------------------------------------------------------
    def top_clusters(self, h: torch.Tensor, do_sample: bool = False,
                     temperature: float = 1.0) -> torch.Tensor:
        """[1, 1, D] -> [1, 1, p] probed cluster ids (flash_head.py:190-221)."""
        if do_sample:
            sims = torch.nn.functional.linear(h, self.centroids.t())
            probs = torch.softmax(sims / temperature, dim=-1)
            return torch.multinomial(probs.view(-1, probs.shape[-1]), self.n_probes,
                                     replacement=False).view(1, 1, self.n_probes)
        sims = torch.nn.functional.linear(h, self.cluster_w)
        return torch.topk(sims, k=self.n_probes, dim=-1, sorted=False).indices

    def scores(self, h: torch.Tensor) -> torch.Tensor:
        """Stage-1 similarities as the reference computes them (bf16 output)."""
        return torch.nn.functional.linear(h, self.cluster_w)

    # -- stage 2 ---------------------------------------------------------------
    def gather_logits(self, h: torch.Tensor, clusters: torch.Tensor, tiebreak: bool):
        """Candidate logits over the probed clusters (+ special tokens),
        flash_head.py:223-261."""
        ci = clusters if clusters.dim() == 1 else clusters[0, 0]
        rows = (ci.unsqueeze(1) * self.cap + torch.arange(self.cap)).reshape(-1)
        ids = self.vocab_maps.index_select(0, ci).reshape(-1)
        if self.special.numel():
            flat = self.vocab_maps.reshape(-1)
            sp_rows = (flat.unsqueeze(0) == self.special.unsqueeze(1)).int().argmax(dim=1)
            rows = torch.cat([rows, sp_rows])
            ids = torch.cat([ids, self.special])
            ids, inverse = torch.unique(ids, return_inverse=True)
            rows = torch.zeros_like(ids).scatter_(0, inverse, rows)
        mapping = None
        if tiebreak:
            srt = ids.sort()
            ids, mapping = srt.values, srt.indices
            rows = rows.index_select(0, mapping)
        w_rows = self.w_perm.view(-1, self.D).index_select(0, rows)
        return torch.nn.functional.linear(h, w_rows), mapping, ids

    def block_sparse_argmax(self, h2d: torch.Tensor, clusters: torch.Tensor) -> torch.Tensor:
        """CPU statement of the Triton greedy kernel (fused.py:119-188):
        per row, fp32 dots over the probed clusters, winner = largest fp32
        logit with ties to the smallest vocab id. [T, D] x [T, p] -> [T, 1]."""
        out = []
        for t in range(h2d.shape[0]):
            ci = clusters[t].to(torch.int64)
            w = self.w_perm.index_select(0, ci).to(torch.float32).reshape(-1, self.D)
            logits = w @ h2d[t].to(torch.float32)
            ids = self.vocab_maps.index_select(0, ci).reshape(-1)
            best = logits.max()
            out.append(int(ids[logits == best].min()))
        return torch.tensor(out, dtype=torch.int64).view(-1, 1)

    # -- dispatch ----------------------------------------------------------------
    def get_next_token(self, hidden_states: torch.Tensor, do_sample: bool = False,
                       temperature: float = 1.0, use_identical_tiebreak: bool = False):
        """Mirror of FlashHead.get_next_token (flash_head.py:277-334) on CPU."""
        if hidden_states.shape[0] > 10:
            logits = torch.nn.functional.linear(hidden_states, self.w_perm.view(-1, self.D))
            if do_sample:
                probs = (logits[:, -1, :] / temperature).softmax(dim=-1)
                slot = torch.multinomial(probs, num_samples=1)
            else:
                slot = logits[:, -1:].argmax(dim=-1)
            return self.vocab_maps.view(-1)[slot]
        top = self.top_clusters(hidden_states, do_sample, temperature)
        if not do_sample and not use_identical_tiebreak and self.special.numel() == 0:
            B, T, D = hidden_states.shape
            return self.block_sparse_argmax(hidden_states.view(T, D), top.view(T, -1))
        logits, mapping, ids = self.gather_logits(hidden_states, top, use_identical_tiebreak)
        if do_sample:
            probs = (logits[:, -1, :] / temperature).softmax(dim=-1)
            idx = torch.multinomial(probs, num_samples=1)
        else:
            idx = logits.argmax(dim=-1, keepdim=True)
            if use_identical_tiebreak:
                idx = mapping[idx]
        return ids[idx][0]
