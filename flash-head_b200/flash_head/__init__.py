"""FlashHead for B200: a clustering-based LM head as a vLLM plugin.

Drop-in for the reference plugin (embedl/flash-head, src/flash_head/__init__.py):
the same ``vllm.general_plugins`` entry point ``flash_head = flash_head:register``,
the same ``FLASHHEAD_ENABLED`` switch and the same ``FlashHead*`` architecture
aliases. The per-step head runs in sm_100a CUDA kernels (libflashhead_b200.so).
"""

import logging
import os

from flash_head._version import __version__

logger = logging.getLogger(__name__)

_patches_applied = False

# FlashHead checkpoint architecture names -> the base vLLM model classes
# (lazy "module:Class" strings, so registering does not initialise CUDA).
_FLASHHEAD_ARCHITECTURES = {
    "FlashHeadLlamaForCausalLM": "vllm.model_executor.models.llama:LlamaForCausalLM",
    "FlashHeadQwen3ForCausalLM": "vllm.model_executor.models.qwen3:Qwen3ForCausalLM",
    "FlashHeadQwen3VLForConditionalGeneration":
        "vllm.model_executor.models.qwen3_vl:Qwen3VLForConditionalGeneration",
    "FlashHeadQwen3_5ForCausalLM": "vllm.model_executor.models.qwen3_5:Qwen3_5ForCausalLM",
    "FlashHeadQwen3_5MoeForCausalLM": "vllm.model_executor.models.qwen3_5:Qwen3_5MoeForCausalLM",
    "FlashHeadQwen3_5ForConditionalGeneration":
        "vllm.model_executor.models.qwen3_5:Qwen3_5ForConditionalGeneration",
    "FlashHeadQwen3_5MoeForConditionalGeneration":
        "vllm.model_executor.models.qwen3_5:Qwen3_5MoeForConditionalGeneration",
    "FlashHeadGemma3ForCausalLM": "vllm.model_executor.models.gemma3:Gemma3ForCausalLM",
}


def register():
    """vLLM plugin entry point, called in every process before model init.

    Idempotent. Registers the architecture aliases, then (unless
    FLASHHEAD_ENABLED=0) applies the vLLM hooks (reference __init__.py:22-38).
    """
    global _patches_applied
    if _patches_applied:
        return
    _patches_applied = True
    _register_architectures()
    if os.environ.get("FLASHHEAD_ENABLED", "1") == "0":
        logger.info("[FlashHead] Disabled via FLASHHEAD_ENABLED=0")
        return
    from flash_head.patches import apply_all
    apply_all()
    logger.info("[FlashHead] Plugin registered")


def _register_architectures():
    """Let vLLM accept FlashHead architecture names (reference __init__.py:41-73)."""
    try:
        from vllm import ModelRegistry
        supported = ModelRegistry.get_supported_archs()
        for fh_arch, model_cls_path in _FLASHHEAD_ARCHITECTURES.items():
            if fh_arch not in supported:
                ModelRegistry.register_model(fh_arch, model_cls_path)
                logger.info("[FlashHead] Registered architecture %s", fh_arch)
    except Exception as e:  # vLLM missing or incompatible: plugin stays inert
        logger.debug("[FlashHead] Architecture registration skipped: %s", e)


def __getattr__(name):
    # Lazy public API: importing the plugin must not import torch-heavy modules.
    if name in ("FlashHead", "get_flash_head_parameters"):
        from flash_head import flash_head as _fh
        return getattr(_fh, name)
    raise AttributeError(name)
