"""Reading a FlashHead model's assets from disk or the Hugging Face hub.

The layout is the reference's asset contract (embedl/flash-head,
src/flash_head/loading.py and flash_head.py:41-78), which a drop-in must read
unchanged:

  <model>/config.json                       ``flash_head_cache_dir`` (+ optional
                                            ``flash_head_special_token_ids``,
                                            ``n_probes``)
  <model>/model.safetensors                 the LM-head weight under one of
  or model.safetensors.index.json + shards  LM_HEAD_KEYS
  <model>/<cache_dir>/clustering_cache.safetensors
                                            ``centroids`` [D, K] and
                                            ``cluster_assignments`` [V]

A model is a local directory or a hub id; hub files are taken from the local
hub cache when present and downloaded otherwise. Error types and messages
follow the reference's, since callers may match on them.
"""

from __future__ import annotations

import json
import os
from typing import Iterable, Optional, Tuple

import torch

CONFIG_JSON = "config.json"
SINGLE_FILE = "model.safetensors"
SHARD_INDEX = "model.safetensors.index.json"
CLUSTERING_CACHE = "clustering_cache.safetensors"

# Keys of the LM-head weight, in order of preference; the input embedding
# stands in for tied heads.
LM_HEAD_KEYS = [
    "lm_head.weight",
    "model.lm_head.weight",
    "transformer.lm_head.weight",
    "model.embed_tokens.weight",
]
_HEAD_SUFFIXES = ("lm_head.weight", "embed_tokens.weight")


class ModelFiles:
    """The files of one model, local or on the hub."""

    def __init__(self, model: str):
        self.model = model
        self.is_local = os.path.isdir(model)

    def locate(self, name: str) -> Optional[str]:
        """Local path of `name`, or None if the model has no such file."""
        if self.is_local:
            path = os.path.join(self.model, name)
            return path if os.path.exists(path) else None
        try:
            return self._from_hub(name)
        except Exception:
            return None

    def require(self, name: str) -> str:
        """Local path of `name`; a missing local file raises FileNotFoundError,
        a hub failure raises the hub's own error."""
        if self.is_local:
            path = os.path.join(self.model, name)
            if not os.path.exists(path):
                raise FileNotFoundError(f"Missing local asset: {path}")
            return path
        return self._from_hub(name)

    def _from_hub(self, name: str) -> str:
        from huggingface_hub import hf_hub_download, try_to_load_from_cache
        hit = try_to_load_from_cache(self.model, name)
        return hit if isinstance(hit, str) else hf_hub_download(repo_id=self.model, filename=name)

    def read_json(self, name: str) -> Optional[dict]:
        path = self.locate(name)
        if path is None:
            return None
        with open(path, encoding="utf-8") as f:
            return json.load(f)

    def resolve_dir(self, rel: str) -> str:
        """A directory named in config.json: relative to a local model, as is
        for hub ids (resolved file by file)."""
        return os.path.join(self.model, rel) if self.is_local and not os.path.isabs(rel) else rel


def pick_lm_head_key(keys: Iterable[str], by_suffix: bool) -> Optional[str]:
    """The LM-head key among `keys`: the first of LM_HEAD_KEYS present, else
    (by_suffix) any key ending in lm_head.weight / embed_tokens.weight."""
    keys = list(keys)
    present = set(keys)
    for k in LM_HEAD_KEYS:
        if k in present:
            return k
    if by_suffix:
        return next((k for k in keys if k.endswith(_HEAD_SUFFIXES)), None)
    return None


def lm_head_weight(files: ModelFiles) -> Tuple[torch.Tensor, str]:
    """(weight, key) of the model's LM head, from a sharded checkpoint (its
    index names the shard) or from a single safetensors file."""
    from safetensors import safe_open

    index = files.read_json(SHARD_INDEX)
    if index is not None:
        weight_map = index.get("weight_map", {})
        key = pick_lm_head_key(weight_map, by_suffix=True)
        if key is None:
            raise KeyError(f"No lm_head/tied embedding key found in index. Looked for: {LM_HEAD_KEYS}")
        shard = weight_map[key]
        shard_path = files.locate(shard)
        if shard_path is None:
            raise FileNotFoundError(f"Could not resolve shard: {shard}")
        with safe_open(shard_path, framework="pt", device="cpu") as f:
            if key not in f.keys():
                raise KeyError(f"Expected {key} in {shard}, but not found.")
            return f.get_tensor(key), key
    single = files.locate(SINGLE_FILE)
    if single is None:
        raise FileNotFoundError(f"No supported weight files found for {files.model}. "
                                "Expected model.safetensors(.index.json).")
    with safe_open(single, framework="pt", device="cpu") as f:
        key = pick_lm_head_key(f.keys(), by_suffix=False)
        if key is None:
            raise KeyError("Could not find lm_head/tied embedding weight in model.safetensors. "
                           f"Looked for: {LM_HEAD_KEYS}")
        return f.get_tensor(key), key


def clustering(files: ModelFiles, cache_dir: str,
               vocab_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(centroids, cluster_assignments) from ``<cache_dir>/clustering_cache.safetensors``,
    checked against the vocabulary size; any failure is reported as
    ValueError("Error loading cache: ...")."""
    from safetensors.torch import load_file

    path = files.require(os.path.join(cache_dir, CLUSTERING_CACHE))
    try:
        tensors = load_file(path)
        missing = {"centroids", "cluster_assignments"} - tensors.keys()
        if missing:
            raise KeyError(f"Cache missing required tensors. Found keys: {list(tensors.keys())}")
        assign = tensors["cluster_assignments"]
        if tuple(assign.shape) != (vocab_size,):
            raise ValueError(f"cluster_assignments shape {tuple(assign.shape)}; "
                             f"expected ({vocab_size},)")
        return tensors["centroids"], assign
    except Exception as e:
        raise ValueError(f"Error loading cache: {e}") from e
