"""Hook vLLM's Sampler to pass FlashHead token ids through (reference
patches/sampler.py:16-29): 1-D or [N, 1] input is treated as sampled ids and
returned as ``SamplerOutput(sampled_token_ids=[N, 1] int32, ...)``. Requests
with a temperature are sampled by FlashHead's sampling kernels at that
temperature (``logits_processor.step_sampled_ids``) instead of decoded
greedily.

Where the reference always returns ``logprobs_tensors=None``, requests that
ask for k logprobs get them over the step's candidate set
(``FlashHead.candidate_logprobs``: the probed clusters' tokens, the special
tokens and the sampled token, softmax renormalised over that set) in the
layout of vLLM's own ``gather_logprobs``. Full-vocabulary logprobs (k = -1)
and logprobs of named tokens are not available on this path (None).
"""

import logging

logger = logging.getLogger(__name__)
_warned = set()


def _warn_once(key, msg):
    if key not in _warned:
        _warned.add(key)
        logger.warning(msg)


def flash_head_logprobs(sampled, sampling_metadata):
    """LogprobsTensors for the FlashHead step's sampled ids [N] int64, or None."""
    k = getattr(sampling_metadata, "max_num_logprobs", None) if sampling_metadata else None
    if k is None:
        return None
    if k < 0 or getattr(sampling_metadata, "logprob_token_ids", None):
        _warn_once("full", "[FlashHead] full-vocabulary or named-token logprobs are not "
                           "available on the FlashHead path; returning none")
        return None
    from vllm.v1.outputs import LogprobsTensors

    from flash_head.patches.logits_processor import step_candidate_logprobs
    res = step_candidate_logprobs(sampled, int(k))
    if res is None:
        return None
    ids, lps, ranks = res
    return LogprobsTensors(ids, lps, ranks)


def patch_sampler():
    import torch
    from vllm.v1.sample.sampler import Sampler, SamplerOutput

    _original_forward = Sampler.forward

    def _patched_forward(self, logits, sampling_metadata, predict_bonus_token=False,
                         logprobs_mode_override=None):
        if logits.ndim == 1 or (logits.ndim == 2 and logits.shape[-1] == 1):
            from flash_head.patches.logits_processor import step_sampled_ids
            sampled = step_sampled_ids(logits.view(-1).to(torch.int32), sampling_metadata)
            lp = flash_head_logprobs(sampled.to(torch.int64), sampling_metadata)
            return SamplerOutput(sampled_token_ids=sampled.unsqueeze(-1), logprobs_tensors=lp)
        return _original_forward(self, logits, sampling_metadata,
                                 predict_bonus_token=predict_bonus_token,
                                 logprobs_mode_override=logprobs_mode_override)

    Sampler.forward = _patched_forward
    logger.info("[FlashHead] Patched Sampler.forward")
