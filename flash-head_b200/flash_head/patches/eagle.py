"""Hook vLLM's EAGLE-style draft proposers for FlashHead ids (reference
patches/eagle.py, which looked for the method under several names; vLLM
0.22 has ``_greedy_sample`` and ``_sample_from_logits`` on the proposer base
class).

A draft model that shares the target's LM head gets FlashHead token ids
([N, 1]) from ``compute_logits``; taking ``argmax`` of those would return 0
for every row. The hooks pass such ids through as the draft tokens (no draft
probabilities)."""

import logging

logger = logging.getLogger(__name__)


def _is_ids(t):
    return t is not None and t.ndim == 2 and t.shape[1] == 1


def patch_eagle():
    try:
        from vllm.v1.spec_decode.eagle import EagleProposer
    except ImportError:
        logger.debug("[FlashHead] EagleProposer not available, skipping patch")
        return
    import torch

    if hasattr(EagleProposer, "_greedy_sample"):
        _original_greedy = EagleProposer._greedy_sample

        def _patched_greedy_sample(self, hidden_states):
            if getattr(self, "use_local_argmax_reduction", False):
                return _original_greedy(self, hidden_states)
            logits = self.model.compute_logits(hidden_states)
            if _is_ids(logits):
                return logits.view(-1).to(torch.int64)
            return logits.argmax(dim=-1)

        EagleProposer._greedy_sample = _patched_greedy_sample
    if hasattr(EagleProposer, "_sample_from_logits"):
        _original_sample = EagleProposer._sample_from_logits

        def _patched_sample_from_logits(self, logits, sampling_metadata):
            if _is_ids(logits):
                return logits.view(-1).to(torch.int64), None
            return _original_sample(self, logits, sampling_metadata)

        EagleProposer._sample_from_logits = _patched_sample_from_logits
    logger.info("[FlashHead] Patched EagleProposer draft sampling")
