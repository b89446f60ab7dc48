"""Process-local registry of the serving model and of the worker stores.

The model registry has the contract of cacheblend_vllm/registry.py:13-41: a
model is published per engine id, not owned (weak reference), and a second
different model for the same engine is an error.  The store registry lets the
scheduler-side connector of a single-process deployment reach the workers'
stores for lookup without the reference's ZeroMQ control plane.
"""

from __future__ import annotations

import threading
import weakref

_lock = threading.Lock()
_models: dict[str, weakref.ref] = {}
_stores: dict[tuple[str, int], object] = {}


def register_model(engine_id: str, model) -> None:
    with _lock:
        current = _models.get(engine_id)
        existing = current() if current is not None else None
        if existing is not None and existing is not model:
            raise RuntimeError(f"a different model is already registered for engine {engine_id}")
        _models[engine_id] = weakref.ref(model)


def get_model(engine_id: str):
    with _lock:
        ref = _models.get(engine_id)
        model = ref() if ref is not None else None
    if model is None:
        raise RuntimeError(f"model for engine {engine_id} is not registered")
    return model


def register_store(engine_id: str, rank: int, store) -> None:
    with _lock:
        _stores[(engine_id, rank)] = store


def stores(engine_id: str) -> list:
    with _lock:
        return [store for (engine, _), store in sorted(_stores.items()) if engine == engine_id]


def unregister_store(engine_id: str, rank: int) -> None:
    with _lock:
        _stores.pop((engine_id, rank), None)


def clear_for_test() -> None:
    with _lock:
        _models.clear()
        _stores.clear()
