"""Seeded synthetic FlashHead heads and hidden states.

No checkpoint or dataset is involved: every head used by the tests and the
benchmark is generated here from a seed, with the shapes of real LM heads
(Llama-3.2-1B: D=2048, V=128256; Llama-3.1-8B: D=4096; Qwen2.5-1.5B: D=1536,
V=151936; Llama-3.1-70B: D=8192).

Generator (balanced by construction, cluster size ``cap``):
  * K cluster centres, each dimension ~ N(0, center_std^2)      (0.02)
  * token -> cluster assignment: a seeded permutation of arange(V) % K,
    so every cluster owns exactly V / K tokens
  * token row = its centre + N(0, noise_std^2)                   (0.005)
  * centroids = per-cluster mean of the member rows, stored [D, K] exactly
    like the ``centroids`` tensor of ``clustering_cache.safetensors``
    (flash_head.py:48-59, :98 in the reference)
  * hidden states ~ N(0, 1) * hidden_std (0.5), cast to the head dtype.

Everything is drawn from a ``torch.Generator`` so a CPU-generated head is
bit-identical on any machine running the same torch build.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass(frozen=True)
class HeadShape:
    """Shape of one synthetic head: hidden D, vocab V, clusters K of size cap."""

    hidden: int
    vocab: int
    n_clusters: int
    cluster_size: int = 16
    n_probes: int = 256

    def __post_init__(self):
        if self.n_clusters * self.cluster_size != self.vocab:
            raise ValueError(
                f"unbalanced shape: {self.n_clusters} clusters x {self.cluster_size} "
                f"!= vocab {self.vocab}")


# Head shapes of the workloads the benchmark and the tests name.
LLAMA32_1B = HeadShape(hidden=2048, vocab=128256, n_clusters=8016)
LLAMA31_8B = HeadShape(hidden=4096, vocab=128256, n_clusters=8016)
QWEN25_15B = HeadShape(hidden=1536, vocab=151936, n_clusters=9496)
LLAMA31_70B = HeadShape(hidden=8192, vocab=128256, n_clusters=8016)


@dataclass
class SyntheticHead:
    """A generated head in the reference's asset layout.

    weight       [V, D]  LM-head weight (head dtype)
    centroids    [D, K]  fp32 per-cluster means (``clustering_cache`` layout)
    assignments  [V]     int64 token -> cluster id
    """

    weight: torch.Tensor
    centroids: torch.Tensor
    assignments: torch.Tensor
    shape: HeadShape
    seed: int


def make_head(shape: HeadShape, seed: int = 0, dtype: torch.dtype = torch.bfloat16,
              device: str | torch.device = "cpu", center_std: float = 0.02,
              noise_std: float = 0.005) -> SyntheticHead:
    """Generate a balanced centre+noise head (see module docstring)."""
    D, V, K = shape.hidden, shape.vocab, shape.n_clusters
    g = torch.Generator(device=device).manual_seed(seed)
    centers = torch.randn(K, D, generator=g, device=device) * center_std
    perm = torch.randperm(V, generator=g, device=device)
    assign = torch.empty(V, dtype=torch.int64, device=device)
    assign[perm] = torch.arange(V, device=device) % K
    weight = torch.randn(V, D, generator=g, device=device).mul_(noise_std)
    weight += centers.index_select(0, assign)
    del centers
    weight = weight.to(dtype)
    # Centroids are the means of the rows as stored (in the head dtype).
    sums = torch.zeros(K, D, device=device, dtype=torch.float32)
    sums.index_add_(0, assign, weight.float())
    centroids = (sums / shape.cluster_size).t().contiguous()
    return SyntheticHead(weight=weight, centroids=centroids, assignments=assign,
                         shape=shape, seed=seed)


def make_hidden(rows: int, hidden: int, seed: int = 1, dtype: torch.dtype = torch.bfloat16,
                device: str | torch.device = "cpu", std: float = 0.5) -> torch.Tensor:
    """Decode-step hidden states [rows, hidden] ~ N(0,1)*std in the head dtype."""
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(rows, hidden, generator=g, device=device) * std).to(dtype)


def head_checksum(head: SyntheticHead) -> list[float]:
    """Cheap fingerprint used by fixtures to confirm a regenerated head is identical."""
    w = head.weight.float()
    return [float(w[:64].sum()), float(w[-64:].sum()),
            float(head.centroids[:, :8].sum()), float(head.assignments[:4096].sum())]


def save_assets(head: SyntheticHead, model_dir: str, n_probes: Optional[int] = None,
                special_token_ids: Optional[list[int]] = None,
                cache_dir: str = "flash_head_assets",
                lm_head_key: str = "lm_head.weight") -> str:
    """Write the head in the reference's on-disk layout.

    ``<model_dir>/config.json`` carries ``flash_head_cache_dir`` (+ optional
    ``n_probes`` / ``flash_head_special_token_ids``), the weight goes to
    ``model.safetensors`` under ``lm_head_key`` and the clustering to
    ``<cache_dir>/clustering_cache.safetensors`` with keys ``centroids`` and
    ``cluster_assignments`` (loading.py:179-205, flash_head.py:41-78).
    """
    import json
    import os

    from safetensors.torch import save_file

    os.makedirs(os.path.join(model_dir, cache_dir), exist_ok=True)
    cfg = {"architectures": ["FlashHeadLlamaForCausalLM"],
           "hidden_size": head.shape.hidden, "vocab_size": head.shape.vocab,
           "flash_head_cache_dir": cache_dir}
    if n_probes is not None:
        cfg["n_probes"] = int(n_probes)
    if special_token_ids is not None:
        cfg["flash_head_special_token_ids"] = list(special_token_ids)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(cfg, f)
    save_file({lm_head_key: head.weight.contiguous().cpu()},
              os.path.join(model_dir, "model.safetensors"))
    save_file({"centroids": head.centroids.contiguous().cpu(),
               "cluster_assignments": head.assignments.contiguous().cpu()},
              os.path.join(model_dir, cache_dir, "clustering_cache.safetensors"))
    return model_dir
