"""Runtime hooks into vLLM, applied by ``flash_head.register()``.

1. LogitsProcessor._get_logits / forward - return FlashHead token ids for
   decode steps (reference patches/logits_processor.py)
2. Sampler.forward - pass token ids through (reference patches/sampler.py)
3. GPUModelRunner._dummy_sampler_run - build the head and warm its kernels at
   worker warm-up, then let vLLM warm its sampler on real logits (the role
   of reference patches/gpu_model_runner.py)
4. LLMEngine.from_engine_args - publish the head metadata (offline ``LLM``)
   (reference patches/llm.py)
5. AsyncLLM.__init__ - publish the head metadata (``vllm serve``)
   (reference patches/async_llm.py)
6. RejectionSampler.forward - verify speculative drafts against FlashHead
   ids on the device (reference patches/rejection_sampler.py)
7. EagleProposer._greedy_sample / _sample_from_logits - pass FlashHead ids
   through as draft tokens (reference patches/eagle.py)
"""

import logging

logger = logging.getLogger(__name__)


def apply_all():
    """Apply every FlashHead hook; a hook whose vLLM class is missing is skipped."""
    from flash_head.patches.eagle import patch_eagle
    from flash_head.patches.engine import patch_async_llm, patch_llm_engine
    from flash_head.patches.logits_processor import patch_logits_processor
    from flash_head.patches.rejection_sampler import patch_rejection_sampler
    from flash_head.patches.sampler import patch_sampler
    from flash_head.patches.warmup import patch_sampler_warmup

    patch_logits_processor()
    patch_sampler()
    patch_rejection_sampler()
    patch_eagle()
    patch_sampler_warmup()
    patch_llm_engine()
    patch_async_llm()
    logger.info("[FlashHead] All patches applied")
