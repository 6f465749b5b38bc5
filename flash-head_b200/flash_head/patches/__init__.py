"""Runtime hooks into vLLM, applied by ``flash_head.register()``.

1. LogitsProcessor._get_logits / forward - return FlashHead token ids for
   decode steps (reference patches/logits_processor.py)
2. Sampler.forward - pass token ids through (reference patches/sampler.py)
3. GPUModelRunner._dummy_sampler_run - build the head at warm-up and accept
   token ids there (reference patches/gpu_model_runner.py)
4. LLMEngine.from_engine_args - write the head metadata (offline ``LLM``)
   (reference patches/llm.py)
5. AsyncLLM.__init__ - write the head metadata (``vllm serve``)
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
    from flash_head.patches.async_llm import patch_async_llm
    from flash_head.patches.gpu_model_runner import patch_gpu_model_runner
    from flash_head.patches.llm import patch_llm
    from flash_head.patches.logits_processor import patch_logits_processor
    from flash_head.patches.eagle import patch_eagle
    from flash_head.patches.rejection_sampler import patch_rejection_sampler
    from flash_head.patches.sampler import patch_sampler

    patch_logits_processor()
    patch_sampler()
    patch_rejection_sampler()
    patch_eagle()
    patch_gpu_model_runner()
    patch_llm()
    patch_async_llm()
    logger.info("[FlashHead] All patches applied")
