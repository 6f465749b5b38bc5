"""Worker warm-up hook (the role of the reference's
patches/gpu_model_runner.py).

vLLM's ``GPUModelRunner._dummy_sampler_run`` warms its sampler (and sizes the
memory it needs) on the logits of ``compute_logits`` for a batch of dummy rows.
The hook:
  1. builds this worker's FlashHead, so no decode step and no CUDA-graph
     capture ever pays for loading it, and runs one FlashHead step on random
     rows (the dummy hidden states may hold inf / nan), which loads the
     kernels and sizes the head's workspace;
  2. runs vLLM's own warm-up with the FlashHead decode shortcut switched off,
     so the sampler is warmed on real [rows, vocab] logits, which steps with
     more rows than FlashHead serves still produce.
"""

import logging

logger = logging.getLogger(__name__)


def patch_sampler_warmup():
    try:
        from vllm.v1.worker.gpu_model_runner import GPUModelRunner
    except ImportError:
        logger.debug("[FlashHead] GPUModelRunner not available, skipping patch")
        return
    original = getattr(GPUModelRunner, "_dummy_sampler_run", None)
    if original is None:
        logger.debug("[FlashHead] GPUModelRunner._dummy_sampler_run not found, skipping patch")
        return

    def _dummy_sampler_run(self, hidden_states, *args, **kwargs):
        import torch

        from flash_head.patches import logits_processor as lp
        fh = lp._get_flash_head()
        if fh is not None and hidden_states is not None and hidden_states.numel():
            rows = min(hidden_states.shape[0], lp.max_decode_rows())
            fh.get_next_token_batched(torch.rand_like(hidden_states[:rows]))
        with lp.full_logits():
            return original(self, hidden_states, *args, **kwargs)

    GPUModelRunner._dummy_sampler_run = _dummy_sampler_run
    logger.info("[FlashHead] Patched GPUModelRunner._dummy_sampler_run")
