"""Hook vLLM's LogitsProcessor so decode steps return FlashHead token ids.

Contract (reference patches/logits_processor.py:32-45): when a FlashHead is
loaded and the step has ``1 <= num_tokens <= FLASHHEAD_MAX_DECODE_ROWS`` rows
(default 1, the reference's gate), ``_get_logits`` returns int32 token ids
[num_tokens, 1] instead of logits; otherwise vLLM's own path runs. The
patched ``forward`` also leaves such ids untouched by the logit soft-cap and
scale that vLLM applies to real logits.
"""

import contextlib
import logging
import os

import torch

logger = logging.getLogger(__name__)

_FLASH_HEAD_NOT_LOADED = object()
_flash_head = _FLASH_HEAD_NOT_LOADED


def max_decode_rows() -> int:
    return max(1, int(os.environ.get("FLASHHEAD_MAX_DECODE_ROWS", "1")))


def _get_flash_head():
    """The worker's FlashHead (built on first use), or None for other models."""
    global _flash_head
    if _flash_head is _FLASH_HEAD_NOT_LOADED:
        from flash_head.loading import get_flash_head
        _flash_head = get_flash_head()
        if _flash_head is not None:
            _flash_head.prepare(max_decode_rows())
    return _flash_head


# hidden states of the last step that returned FlashHead ids; the sampler
# hook reads them when the step's requests ask for logprobs
_last_hidden = None
# > 0 while vLLM must see real logits (its sampler warm-up)
_full_logits_depth = 0


@contextlib.contextmanager
def full_logits():
    """Within the block, _get_logits returns vLLM's logits for every step."""
    global _full_logits_depth
    _full_logits_depth += 1
    try:
        yield
    finally:
        _full_logits_depth -= 1


def flash_head_token_ids(hidden_states: torch.Tensor):
    """Token ids [n, 1] int32 for a decode step, or None if FlashHead does not apply."""
    global _last_hidden
    if _full_logits_depth > 0:
        _last_hidden = None
        return None
    fh = _get_flash_head()
    n = hidden_states.shape[0]
    if fh is None or not (1 <= n <= max_decode_rows()):
        _last_hidden = None
        return None
    h = hidden_states.reshape(n, -1)
    _last_hidden = h
    return fh.get_next_token_batched(h).view(n, 1).to(torch.int32)


def step_candidate_logprobs(token_ids: torch.Tensor, num_logprobs: int):
    """(ids, logprobs, ranks) of the last FlashHead step over its candidate
    set (FlashHead.candidate_logprobs), or None when there is no such step."""
    fh = _flash_head
    if fh is _FLASH_HEAD_NOT_LOADED or fh is None or _last_hidden is None:
        return None
    if _last_hidden.shape[0] != token_ids.numel():
        return None
    return fh.candidate_logprobs(_last_hidden, token_ids, num_logprobs)


def patch_logits_processor():
    from vllm.model_executor.layers.logits_processor import LogitsProcessor

    _original_get_logits = LogitsProcessor._get_logits
    _original_forward = LogitsProcessor.forward

    def _patched_get_logits(self, hidden_states, lm_head, embedding_bias):
        ids = flash_head_token_ids(hidden_states)
        if ids is not None:
            return ids
        return _original_get_logits(self, hidden_states, lm_head, embedding_bias)

    def _patched_forward(self, lm_head, hidden_states, embedding_bias=None):
        if self.logits_as_input:
            return _original_forward(self, lm_head, hidden_states, embedding_bias)
        logits = self._get_logits(hidden_states, lm_head, embedding_bias)
        if logits is None or not torch.is_floating_point(logits):
            return logits  # FlashHead token ids: no soft-cap / scale
        if self.soft_cap is not None:
            logits = torch.tanh(logits / self.soft_cap) * self.soft_cap
        if self.scale != 1.0:
            logits = logits * self.scale
        return logits

    LogitsProcessor._get_logits = _patched_get_logits
    LogitsProcessor.forward = _patched_forward
    logger.info("[FlashHead] Patched LogitsProcessor._get_logits and forward")
