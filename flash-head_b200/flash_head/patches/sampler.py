"""Hook vLLM's Sampler to pass FlashHead token ids through (reference
patches/sampler.py:16-29): 1-D or [N, 1] input is treated as sampled ids and
returned as ``SamplerOutput(sampled_token_ids=[N, 1] int32,
logprobs_tensors=None)``."""

import logging

logger = logging.getLogger(__name__)


def patch_sampler():
    import torch
    from vllm.v1.sample.sampler import Sampler, SamplerOutput

    _original_forward = Sampler.forward

    def _patched_forward(self, logits, sampling_metadata, predict_bonus_token=False,
                         logprobs_mode_override=None):
        if logits.ndim == 1 or (logits.ndim == 2 and logits.shape[-1] == 1):
            sampled = logits.view(-1).to(torch.int32)
            return SamplerOutput(sampled_token_ids=sampled.unsqueeze(-1), logprobs_tensors=None)
        return _original_forward(self, logits, sampling_metadata,
                                 predict_bonus_token=predict_bonus_token,
                                 logprobs_mode_override=logprobs_mode_override)

    Sampler.forward = _patched_forward
    logger.info("[FlashHead] Patched Sampler.forward")
