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


# below this temperature a request is greedy (vLLM's sampler uses the same bound)
_SAMPLING_EPS = 1e-5
_warned = set()


def _warn_once(key, msg):
    if key not in _warned:
        _warned.add(key)
        logger.warning(msg)


def _row_seed(rows, generators):
    """A Philox seed for a group of rows: drawn from the first seeded row's
    generator (so seeded requests repeat), else from torch's default one."""
    for r in rows:
        g = generators.get(int(r)) if generators else None
        if g is not None:
            return int(torch.randint(0, 2**62, (1,), generator=g, device=g.device).item())
    return int(torch.randint(0, 2**62, (1,)).item())


def step_sampled_ids(greedy_ids: torch.Tensor, sampling_metadata):
    """The last FlashHead step's ids with each non-greedy request sampled at its
    own temperature (FlashHead.get_next_token_batched(do_sample=True), one call
    per distinct temperature); greedy rows keep greedy_ids. Where the reference
    hook decodes every request greedily (patches/logits_processor.py:38), this
    routes vLLM's per-request temperature to the sampling kernels. top-k / top-p
    / min-p are not applied on this path (a warning says so once)."""
    md = sampling_metadata
    if md is None or getattr(md, "all_greedy", True) or getattr(md, "temperature", None) is None:
        return greedy_ids
    fh = _flash_head
    h = _last_hidden
    n = greedy_ids.numel()
    if fh is _FLASH_HEAD_NOT_LOADED or fh is None or h is None or h.shape[0] != n:
        return greedy_ids
    if getattr(md, "top_k", None) is not None or getattr(md, "top_p", None) is not None:
        _warn_once("topkp", "[FlashHead] top-k / top-p are not applied on the FlashHead "
                            "path: requests sample from the candidate set at their temperature")
    temps = md.temperature.detach().float().view(-1)[:n].cpu()
    out = greedy_ids.clone()
    random_rows = torch.nonzero(temps >= _SAMPLING_EPS).view(-1)
    for t in torch.unique(temps[random_rows]).tolist():
        rows = random_rows[temps[random_rows] == t]
        idx = rows.to(h.device)
        ids = fh.get_next_token_batched(h.index_select(0, idx), do_sample=True, temperature=float(t),
                                        seed=_row_seed(rows.tolist(), getattr(md, "generators", None)),
                                        offset=0)
        out.view(-1).index_copy_(0, idx.to(out.device), ids.to(out.dtype).view(-1))
    return out


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
