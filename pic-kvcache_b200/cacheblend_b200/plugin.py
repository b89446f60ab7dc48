"""vLLM general-plugin hook that lets the connector find the serving model.

Same contract as cacheblend_vllm/plugin.py:13-30 and models.py:17-37: the
Qwen3 / Qwen3-MoE architectures are re-registered as transparent subclasses
whose constructor publishes the model object under the engine id when the
engine uses ``CacheBlendConnectorV1``; forward and weight loading are vLLM's.
"""

from __future__ import annotations

import threading

from .registry import register_model

_lock = threading.Lock()
_registered = False


def publish_model(vllm_config, model) -> None:
    transfer = getattr(vllm_config, "kv_transfer_config", None)
    if transfer is None or transfer.kv_connector != "CacheBlendConnectorV1":
        return
    if not transfer.engine_id:
        raise ValueError("CacheBlendConnectorV1 requires kv_transfer_config.engine_id")
    register_model(str(transfer.engine_id), model)


def _adapters():
    from vllm.model_executor.models.qwen3 import Qwen3ForCausalLM
    from vllm.model_executor.models.qwen3_moe import Qwen3MoeForCausalLM

    class CacheBlendQwen3ForCausalLM(Qwen3ForCausalLM):
        def __init__(self, *, vllm_config, prefix: str = ""):
            super().__init__(vllm_config=vllm_config, prefix=prefix)
            publish_model(vllm_config, self)

    class CacheBlendQwen3MoeForCausalLM(Qwen3MoeForCausalLM):
        def __init__(self, *, vllm_config, prefix: str = ""):
            super().__init__(vllm_config=vllm_config, prefix=prefix)
            publish_model(vllm_config, self)

    return CacheBlendQwen3ForCausalLM, CacheBlendQwen3MoeForCausalLM


def register() -> None:
    """Register the adapters once per process (``vllm.general_plugins`` entry point)."""
    global _registered
    with _lock:
        if _registered:
            return
        from vllm import ModelRegistry

        dense, moe = _adapters()
        ModelRegistry.register_model("Qwen3ForCausalLM", dense)
        ModelRegistry.register_model("Qwen3MoeForCausalLM", moe)
        _registered = True
