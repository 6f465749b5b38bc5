"""Loading FlashHead assets for vLLM workers (reference: src/flash_head/loading.py).

The on-disk layout is the reference's, unchanged:
  <model>/config.json                      ``flash_head_cache_dir`` (+ optional
                                           ``flash_head_special_token_ids``,
                                           ``n_probes``)
  <model>/model.safetensors(.index.json)   LM-head weight under one of
                                           LM_HEAD_KEYS
  <model>/<cache_dir>/clustering_cache.safetensors
                                           ``centroids`` [D, K],
                                           ``cluster_assignments`` [V]

The engine process writes a small metadata file
(``load_flash_head_from_checkpoint`` + ``set_flash_head``); each worker builds
its head on the GPU from it (``get_flash_head``). Unlike the reference, the
worker derives the cluster layout on the GPU and the vLLM hook builds the head
at warm-up rather than inside the first decode step.
"""

from __future__ import annotations

import json
import logging
import os
import tempfile
from typing import Optional, Tuple

import torch
from torch import nn

from .flash_head import FlashHead, get_flash_head_parameters

logger = logging.getLogger(__name__)

METADATA_PATH = os.path.join(tempfile.gettempdir(), "flashhead_metadata.pt")

LM_HEAD_KEYS = [
    "lm_head.weight",
    "model.lm_head.weight",
    "transformer.lm_head.weight",
    "model.embed_tokens.weight",  # tied embedding fallback
]


def _is_local_dir(path: str) -> bool:
    return os.path.isdir(path)


def _resolve_file(model: str, filename: str) -> Optional[str]:
    """Local file, else the HF cache, else a hub download; None if absent
    (loading.py:37-52)."""
    if _is_local_dir(model):
        p = os.path.join(model, filename)
        return p if os.path.exists(p) else None
    try:
        from huggingface_hub import hf_hub_download, try_to_load_from_cache
        cached = try_to_load_from_cache(model, filename)
        if isinstance(cached, str):
            return cached
        return hf_hub_download(repo_id=model, filename=filename)
    except Exception:
        return None


def _find_weight_key_in_index(index_json: dict) -> Optional[str]:
    """LM_HEAD_KEYS in order, then any ``*lm_head.weight`` / ``*embed_tokens.weight``
    (loading.py:55-63)."""
    weight_map = index_json.get("weight_map", {})
    for k in LM_HEAD_KEYS:
        if k in weight_map:
            return k
    for k in weight_map:
        if k.endswith("lm_head.weight") or k.endswith("embed_tokens.weight"):
            return k
    return None


def _load_lm_head_weight(model: str) -> Tuple[torch.Tensor, str]:
    """(weight, key) from a sharded or single-file safetensors checkpoint
    (loading.py:66-106; same errors)."""
    from safetensors import safe_open

    index_path = _resolve_file(model, "model.safetensors.index.json")
    if index_path is not None:
        with open(index_path, encoding="utf-8") as f:
            index = json.load(f)
        chosen = _find_weight_key_in_index(index)
        if chosen is None:
            raise KeyError(f"No lm_head/tied embedding key found in index. Looked for: {LM_HEAD_KEYS}")
        shard_name = index["weight_map"][chosen]
        shard_path = _resolve_file(model, shard_name)
        if shard_path is None:
            raise FileNotFoundError(f"Could not resolve shard: {shard_name}")
        with safe_open(shard_path, framework="pt", device="cpu") as f:
            if chosen not in f.keys():
                raise KeyError(f"Expected {chosen} in {shard_name}, but not found.")
            return f.get_tensor(chosen), chosen
    st_path = _resolve_file(model, "model.safetensors")
    if st_path is not None:
        with safe_open(st_path, framework="pt", device="cpu") as f:
            keys = f.keys()
            for k in LM_HEAD_KEYS:
                if k in keys:
                    return f.get_tensor(k), k
        raise KeyError("Could not find lm_head/tied embedding weight in model.safetensors. "
                       f"Looked for: {LM_HEAD_KEYS}")
    raise FileNotFoundError(f"No supported weight files found for {model}. "
                            "Expected model.safetensors(.index.json).")


def _read_config_json(model: str) -> Optional[dict]:
    path = _resolve_file(model, "config.json")
    if path is None:
        return None
    with open(path) as f:
        return json.load(f)


def build_flash_head(model_path: str, cache_dir: str, special_token_ids=None, n_probes=None,
                     dtype: torch.dtype = torch.bfloat16, device="cuda",
                     stage1_dtype: Optional[str] = None) -> FlashHead:
    """Build a FlashHead on ``device`` from on-disk assets.

    The weight is moved to the device first and the clustering layout is
    derived there; the stage-1 matrix is normalised in fp32 and then cast, as
    the reference's loader does with its fp32 stand-in head
    (loading.py:152-164)."""
    w, chosen_key = _load_lm_head_weight(model_path)
    if w.shape[0] >= w.shape[1]:
        vocab_size, hidden_size = w.shape
    else:
        hidden_size, vocab_size = w.shape
        w = w.t().contiguous()
    with torch.device("meta"):
        lm = nn.Linear(hidden_size, vocab_size, bias=False)
    lm.weight = nn.Parameter(w.to(device=device, dtype=torch.float32), requires_grad=False)
    params = get_flash_head_parameters(lm, cache_dir=cache_dir, model_or_dir=model_path)
    head = FlashHead(lm, **params, n_probes=n_probes, special_token_ids=special_token_ids,
                     stage1_dtype=stage1_dtype).to(device=device, dtype=dtype)
    del lm
    logger.info("[FlashHead] Built on %s using '%s'", device, chosen_key)
    return head


def get_flash_head() -> Optional[nn.Module]:
    """Build the FlashHead described by METADATA_PATH on the current CUDA
    device, or return None if there is no metadata (loading.py:126-167)."""
    if not os.path.exists(METADATA_PATH):
        return None
    metadata = torch.load(METADATA_PATH, map_location="cpu", weights_only=True)
    dtype_str = metadata.get("dtype", "torch.bfloat16")
    dtype = torch.bfloat16 if dtype_str == "torch.bfloat16" else torch.float16
    return build_flash_head(metadata["model_path"], metadata["cache_dir"],
                            special_token_ids=metadata["special_token_ids"],
                            n_probes=metadata.get("n_probes"), dtype=dtype, device="cuda")


def set_flash_head(flash_head_or_metadata):
    """Save FlashHead metadata for the worker processes (None removes it)."""
    if flash_head_or_metadata is not None:
        torch.save(flash_head_or_metadata, METADATA_PATH)
    elif os.path.exists(METADATA_PATH):
        os.remove(METADATA_PATH)


def load_flash_head_from_checkpoint(model: str, dtype=torch.bfloat16):
    """Metadata dict for a model whose config.json has ``flash_head_cache_dir``,
    else None (loading.py:179-205)."""
    config_dict = _read_config_json(model)
    if config_dict is None or "flash_head_cache_dir" not in config_dict:
        return None
    cache_dir = config_dict["flash_head_cache_dir"]
    if _is_local_dir(model) and not os.path.isabs(cache_dir):
        cache_dir = os.path.join(model, cache_dir)
    metadata = {
        "model_path": model,
        "cache_dir": cache_dir,
        "special_token_ids": config_dict.get("flash_head_special_token_ids"),
        "n_probes": config_dict.get("n_probes"),
        "dtype": str(dtype),
    }
    logger.info("[FlashHead] Metadata prepared for lazy loading from %s", cache_dir)
    return metadata
