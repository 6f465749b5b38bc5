"""Hook LLMEngine.from_engine_args to write FlashHead metadata (offline ``LLM``).

``register()`` runs inside ``LLM.__init__`` (from EngineArgs), so the hook
sits on ``LLMEngine.from_engine_args``, which runs after it (reference
patches/llm.py:17-42).
"""

import json
import logging
import os

logger = logging.getLogger(__name__)


def patch_llm():
    from vllm.v1.engine.llm_engine import LLMEngine

    _original_from_engine_args = LLMEngine.from_engine_args

    @classmethod
    def _patched_from_engine_args(cls, engine_args, *args, **kwargs):
        model = engine_args.model
        try:
            from flash_head.loading import load_flash_head_from_checkpoint, set_flash_head
            meta = load_flash_head_from_checkpoint(model)
            set_flash_head(meta)
            if meta:
                logger.info("[FlashHead] Metadata saved for model: %s", model)
            else:
                _warn_if_flashhead_model(model)
        except Exception as e:
            logger.warning("[FlashHead] Metadata loading skipped: %s", e)
        return _original_from_engine_args.__func__(cls, engine_args, *args, **kwargs)

    LLMEngine.from_engine_args = _patched_from_engine_args
    logger.info("[FlashHead] Patched LLMEngine.from_engine_args")


def _warn_if_flashhead_model(model: str):
    """Warn when a local model asks for FlashHead but it did not activate."""
    config_path = os.path.join(model, "config.json")
    if not os.path.isdir(model) or not os.path.exists(config_path):
        return
    try:
        with open(config_path) as f:
            config = json.load(f)
        if config.get("flash_head_cache_dir"):
            logger.warning(
                "[FlashHead] Model has flash_head_cache_dir in config but FlashHead did NOT "
                "activate; inference will be slower. Check that FLASHHEAD_ENABLED is not 0.")
    except Exception:
        pass
