"""Tensor-parallel FlashHead: clusters partitioned across the ranks of a group.

The reference replicates the whole head on every tensor-parallel rank
(loading.py:144-164) and bypasses vLLM's logits gather. Here rank r of R owns
the contiguous cluster range ``cluster_range(K, R, r)`` with its w_perm rows,
stage-1 rows and vocab ids; hidden states are replicated (as after vLLM's TP
all-reduce). One step:

  1. local stage 1 + local top-p -> [rows, p] candidate words
     (mono(score) << 32 | ~global cluster id, exchanged as signed int64);
  2. all-gather -> [R, rows, p] on every rank;
  3. every rank selects the same global top-p (exact: the global top-p is a
     subset of the union of local top-p lists), scores the probes it owns
     and packs (mono(logit) << 32 | ~vocab id) per row;
  4. max all-reduce over ranks -> the winner;
  5. unpack to token ids.

Sampling uses the same exchange with Gumbel-perturbed keys; noise is keyed by
global cluster and vocab ids, so draws do not depend on R.

Collectives go through ``torch.distributed`` (NCCL on GPUs, gloo in the CPU
tests) on the current stream, so a step can be captured in a CUDA graph.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .native import NativeHead, derive_buffers, shard_buffers


def cluster_range(n_clusters: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous cluster range [lo, hi) owned by ``rank`` of ``world``."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return rank * n_clusters // world, (rank + 1) * n_clusters // world


def exchange_step(hidden: torch.Tensor, group,
                  local_candidates: Callable[[torch.Tensor], torch.Tensor],
                  select_and_score: Callable[[torch.Tensor, torch.Tensor, int], torch.Tensor],
                  finalize: Callable[[torch.Tensor], torch.Tensor]) -> torch.Tensor:
    """Run steps 1-5 with the given per-rank kernels; returns [rows] token ids.

    ``local_candidates(h) -> [rows, p] int64``,
    ``select_and_score(h, all_cand [R, rows, p], R) -> [rows] int64``,
    ``finalize(best [rows]) -> [rows] int64``. Every rank issues the same two
    collectives in the same order.
    """
    world = dist.get_world_size(group)
    cand = local_candidates(hidden)
    rows, p = cand.shape
    gathered = torch.empty(world * rows * p, dtype=torch.int64, device=cand.device)
    dist.all_gather_into_tensor(gathered, cand.contiguous().view(-1), group=group)
    best = select_and_score(hidden, gathered.view(world, rows, p), world)
    dist.all_reduce(best, op=dist.ReduceOp.MAX, group=group)
    return finalize(best)


class ShardedFlashHead:
    """This rank's shard of a FlashHead, stepping with its peers over ``group``.

    :param w_perm: [K, cap, D] cluster-ordered LM-head rows of the WHOLE head
        (any device; only this rank's slice is kept on ``device``)
    :param vocab_maps: [K, cap] vocab ids
    :param cluster_w: [K, D] normalised centroids (stage 1, greedy)
    :param centroids: [D, K] raw centroids (stage 1, sampling)
    :param special_ids: [S] special token ids (each rank scores its own)
    """

    def __init__(self, w_perm: torch.Tensor, vocab_maps: torch.Tensor, cluster_w: torch.Tensor,
                 centroids: torch.Tensor, n_probes: int, special_ids: Optional[torch.Tensor] = None,
                 stage1_dtype: str = "model", group=None, device: Optional[torch.device] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        K, cap, D = w_perm.shape
        self.K, self.cap, self.D, self.p = K, cap, D, n_probes
        self.lo, self.hi = cluster_range(K, self.world, self.rank)
        if self.hi - self.lo < n_probes:
            raise ValueError(f"rank {self.rank} owns {self.hi - self.lo} clusters < n_probes "
                             f"{n_probes}; use fewer ranks or fewer probes")
        device = torch.device(device or w_perm.device)
        sp = special_ids if special_ids is not None else torch.zeros(0, dtype=torch.int64)
        # Slice before deriving so a rank never holds more than its share on
        # the device (fp8 row scales are per row, so slicing commutes).
        sl = slice(self.lo, self.hi)
        part = derive_buffers(w_perm[sl].to(device), vocab_maps[sl].to(device),
                              cluster_w[sl].to(device), centroids[:, sl].to(device),
                              torch.zeros(0, dtype=torch.int64), stage1_dtype)
        flat_vm = vocab_maps.reshape(-1).to(torch.int64).cpu()
        inv = torch.empty_like(flat_vm)
        inv[flat_vm] = torch.arange(flat_vm.numel())
        slots = inv[sp.to(torch.int64).cpu()]
        mine = slots[(slots >= self.lo * cap) & (slots < self.hi * cap)] - self.lo * cap
        part["special_slots"] = (mine.to(device=device, dtype=torch.int32).contiguous()
                                 if mine.numel() else None)
        self.native = NativeHead(part, D, cap, n_probes, cluster_base=self.lo)

    @classmethod
    def from_flash_head(cls, head, group=None, device=None) -> "ShardedFlashHead":
        """Shard an unsharded ``FlashHead`` (its buffers on any device)."""
        return cls(head.w_perm, head.vocab_maps, head.cluster_linear.weight.detach(),
                   head.centroids, head.n_probes, head.special_token_ids_tensor,
                   head.stage1_dtype, group=group, device=device)

    def get_next_token_batched(self, hidden: torch.Tensor, do_sample: bool = False,
                               temperature: float = 1.0, seed: int = 0,
                               offset: int = 0) -> torch.Tensor:
        """[N, D] replicated hidden states -> [N] int64 token ids (same on every rank)."""
        nh = self.native

        def local(h):
            return nh.tp_local_candidates(h, do_sample, temperature, seed, offset)

        def select(h, all_cand, world):
            return nh.tp_select_and_score(h, all_cand, world, do_sample, temperature, seed,
                                          offset)

        return exchange_step(hidden.reshape(-1, self.D), self.group, local, select,
                             NativeHead.tp_finalize)
