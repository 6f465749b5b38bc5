"""Hook GPUModelRunner's sampler warm-up (reference patches/gpu_model_runner.py).

The warm-up builds the FlashHead (so no decode step, and no CUDA-graph
capture, ever pays for loading it) and, like the reference, accepts the
[N, 1] token ids FlashHead returns where vLLM's dummy sampler run expects
logits.
"""

import logging

logger = logging.getLogger(__name__)


def patch_gpu_model_runner():
    try:
        from vllm.v1.worker.gpu_model_runner import GPUModelRunner
    except ImportError:
        logger.debug("[FlashHead] GPUModelRunner not available, skipping patch")
        return
    if not hasattr(GPUModelRunner, "_dummy_sampler_run"):
        logger.debug("[FlashHead] GPUModelRunner._dummy_sampler_run not found, skipping patch")
        return

    _original = GPUModelRunner._dummy_sampler_run

    def _patched_dummy_sampler_run(self, *args, **kwargs):
        from flash_head.patches.logits_processor import _get_flash_head
        _get_flash_head()  # build eagerly, before any graph capture
        try:
            return _original(self, *args, **kwargs)
        except Exception:
            hidden_states = args[0] if args else kwargs.get("hidden_states")
            if hidden_states is not None:
                logits = self.model.compute_logits(hidden_states)
                if logits is not None and (logits.dim() < 2 or logits.size(1) == 1):
                    return logits
            raise

    GPUModelRunner._dummy_sampler_run = _patched_dummy_sampler_run
    logger.info("[FlashHead] Patched GPUModelRunner._dummy_sampler_run")
