"""Engine-side hooks: publish the FlashHead metadata before vLLM starts workers.

The engine is reached two ways: the offline ``LLM`` class goes through
``LLMEngine.from_engine_args`` (``register()`` runs inside ``LLM.__init__``,
before it), and ``vllm serve`` constructs ``AsyncLLM`` directly. Both are
wrapped to read the model's config.json and publish the worker metadata, or
withdraw a stale file left by an earlier model, before the original runs
(reference patches/llm.py and patches/async_llm.py). Publishing never stops
the engine: on any failure the model keeps its own LM head.
"""

import functools
import logging

logger = logging.getLogger(__name__)


def publish_metadata(model) -> bool:
    """Publish (or withdraw) the FlashHead metadata of `model`; True when the
    model asks for FlashHead."""
    if not model:
        return False
    try:
        from flash_head.loading import load_flash_head_from_checkpoint, set_flash_head
        meta = load_flash_head_from_checkpoint(model)
        set_flash_head(meta)
    except Exception as e:  # noqa: BLE001 - the engine must start regardless
        logger.warning("[FlashHead] Metadata loading skipped: %s", e)
        return False
    if meta:
        logger.info("[FlashHead] Metadata saved for model: %s", model)
    return meta is not None


def _model_of_engine_args(engine_args):
    return getattr(engine_args, "model", None)


def _model_of_vllm_config(vllm_config):
    return getattr(getattr(vllm_config, "model_config", None), "model", None)


def patch_llm_engine():
    """LLMEngine.from_engine_args(engine_args, ...) publishes first."""
    from vllm.v1.engine.llm_engine import LLMEngine
    original = LLMEngine.from_engine_args.__func__  # the classmethod's function

    @functools.wraps(original)
    def from_engine_args(cls, engine_args, *args, **kwargs):
        publish_metadata(_model_of_engine_args(engine_args))
        return original(cls, engine_args, *args, **kwargs)

    LLMEngine.from_engine_args = classmethod(from_engine_args)
    logger.info("[FlashHead] Patched LLMEngine.from_engine_args")


def patch_async_llm():
    """AsyncLLM.__init__(vllm_config, ...) publishes first."""
    try:
        from vllm.v1.engine.async_llm import AsyncLLM
    except Exception as e:  # noqa: BLE001 - older or trimmed vLLM builds
        logger.debug("[FlashHead] AsyncLLM not available, skipping patch: %s", e)
        return
    original = AsyncLLM.__init__

    @functools.wraps(original)
    def __init__(self, vllm_config, *args, **kwargs):
        publish_metadata(_model_of_vllm_config(vllm_config))
        return original(self, vllm_config, *args, **kwargs)

    AsyncLLM.__init__ = __init__
    logger.info("[FlashHead] Patched AsyncLLM.__init__")
