"""FlashHead assets for vLLM's engine and worker processes.

The engine process reads the model's config.json and, when it asks for
FlashHead (``flash_head_cache_dir``), publishes a small metadata file
(``load_flash_head_from_checkpoint`` + ``set_flash_head``; reference
src/flash_head/loading.py:170-205). vLLM then starts its workers; each
worker builds its head on its GPU from that file (``get_flash_head``,
reference :126-167). The metadata file's path and keys (model_path,
cache_dir, special_token_ids, n_probes, dtype) are the reference's, so either
side can read what the other wrote.

Unlike the reference, the worker moves the weight to the GPU before deriving
the cluster layout (fast even for 150K-token heads), and the vLLM warm-up
hook builds the head before any decode step or graph capture.
"""

from __future__ import annotations

import dataclasses
import logging
import os
import tempfile
from typing import Optional

import torch
from torch import nn

from .assets import LM_HEAD_KEYS, ModelFiles, lm_head_weight  # noqa: F401
from .flash_head import FlashHead, get_flash_head_parameters

logger = logging.getLogger(__name__)

METADATA_PATH = os.path.join(tempfile.gettempdir(), "flashhead_metadata.pt")

_DTYPES = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16}


@dataclasses.dataclass
class HeadMetadata:
    """What a worker needs to build the head (stored as a plain dict)."""

    model_path: str
    cache_dir: str
    special_token_ids: Optional[list] = None
    n_probes: Optional[int] = None
    dtype: str = "torch.bfloat16"

    @classmethod
    def from_config(cls, model: str, dtype=torch.bfloat16) -> Optional["HeadMetadata"]:
        files = ModelFiles(model)
        cfg = files.read_json("config.json")
        if not cfg or "flash_head_cache_dir" not in cfg:
            return None
        return cls(model_path=model, cache_dir=files.resolve_dir(cfg["flash_head_cache_dir"]),
                   special_token_ids=cfg.get("flash_head_special_token_ids"),
                   n_probes=cfg.get("n_probes"), dtype=str(dtype))

    @property
    def torch_dtype(self) -> torch.dtype:
        return _DTYPES.get(self.dtype, torch.float16)


def build_flash_head(model_path: str, cache_dir: str, special_token_ids=None, n_probes=None,
                     dtype: torch.dtype = torch.bfloat16, device="cuda",
                     stage1_dtype: Optional[str] = None) -> FlashHead:
    """FlashHead on `device` from on-disk assets.

    The stored weight may be [V, D] or [D, V] (the vocabulary is the larger
    dimension). It goes to the device in fp32 and the cluster layout and
    normalised centroids are derived there, then everything is cast to
    `dtype`, as the reference derives them from its fp32 stand-in head
    (loading.py:152-164)."""
    w, key = lm_head_weight(ModelFiles(model_path))
    if w.shape[0] < w.shape[1]:
        w = w.t()
    vocab, hidden = w.shape
    with torch.device("meta"):
        lm = nn.Linear(hidden, vocab, bias=False)
    lm.weight = nn.Parameter(w.to(device=device, dtype=torch.float32).contiguous(),
                             requires_grad=False)
    params = get_flash_head_parameters(lm, cache_dir=cache_dir, model_or_dir=model_path)
    head = FlashHead(lm, **params, n_probes=n_probes, special_token_ids=special_token_ids,
                     stage1_dtype=stage1_dtype).to(device=device, dtype=dtype)
    logger.info("[FlashHead] Built on %s from '%s'", device, key)
    return head


def get_flash_head() -> Optional[nn.Module]:
    """The head described by the published metadata, built on the current
    CUDA device; None when no metadata was published."""
    if not os.path.exists(METADATA_PATH):
        return None
    meta = HeadMetadata(**torch.load(METADATA_PATH, map_location="cpu", weights_only=True))
    return build_flash_head(meta.model_path, meta.cache_dir,
                            special_token_ids=meta.special_token_ids, n_probes=meta.n_probes,
                            dtype=meta.torch_dtype, device="cuda")


def set_flash_head(flash_head_or_metadata):
    """Publish metadata for the workers (a dict); None withdraws it."""
    if flash_head_or_metadata is None:
        try:
            os.remove(METADATA_PATH)
        except FileNotFoundError:
            pass
        return
    torch.save(dict(flash_head_or_metadata), METADATA_PATH)


def load_flash_head_from_checkpoint(model: str, dtype=torch.bfloat16):
    """The metadata dict for `model` when its config.json names a
    ``flash_head_cache_dir`` (relative paths are taken inside a local model
    directory), else None. Reads config.json only."""
    meta = HeadMetadata.from_config(model, dtype)
    if meta is None:
        return None
    logger.info("[FlashHead] Metadata prepared for lazy loading from %s", meta.cache_dir)
    return dataclasses.asdict(meta)
