"""Hook vLLM's RejectionSampler for speculative decoding with FlashHead ids
(reference patches/rejection_sampler.py, written against an older vLLM
signature; this one has vLLM 0.22's ``forward(metadata, draft_probs, logits,
sampling_metadata)``).

When the verification step's "logits" are FlashHead token ids ([N, 1]), the
target ids at the draft positions and the bonus ids are taken from them and
``flash_head.spec.accept_draft_tokens`` compares drafts on the device. Any
other input goes to vLLM's own rejection sampler. Logprobs are not returned
on this path.
"""

import logging

logger = logging.getLogger(__name__)


def flash_head_verify(metadata, logits):
    """SamplerOutput of a verification step whose logits are token ids [N, 1]."""
    import torch
    from vllm.v1.sample.rejection_sampler import PLACEHOLDER_TOKEN_ID, SamplerOutput

    from flash_head.spec import accept_draft_tokens
    ids = logits.view(-1)
    target = ids.index_select(0, metadata.target_logits_indices.to(ids.device, torch.int64))
    bonus = ids.index_select(0, metadata.bonus_logits_indices.to(ids.device, torch.int64))
    out = accept_draft_tokens(metadata.draft_token_ids, target, bonus,
                              metadata.cu_num_draft_tokens, metadata.max_spec_len,
                              placeholder=PLACEHOLDER_TOKEN_ID)
    return SamplerOutput(sampled_token_ids=out, logprobs_tensors=None)


def patch_rejection_sampler():
    try:
        from vllm.v1.sample.rejection_sampler import RejectionSampler
    except ImportError:
        logger.debug("[FlashHead] RejectionSampler not available, skipping patch")
        return

    _original_forward = RejectionSampler.forward

    def _patched_forward(self, metadata, draft_probs, logits, sampling_metadata):
        if logits is not None and logits.ndim == 2 and logits.shape[1] == 1:
            return flash_head_verify(metadata, logits)
        return _original_forward(self, metadata, draft_probs, logits, sampling_metadata)

    RejectionSampler.forward = _patched_forward
    logger.info("[FlashHead] Patched RejectionSampler.forward")
