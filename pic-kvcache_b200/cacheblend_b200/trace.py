"""Opt-in JSONL pipeline tracing (``CACHEBLEND_TRACE_DIR``).

Event names and the record fields (``timestamp_ns``, ``monotonic_ns``,
``pid``, ``thread_id``, ``component``, ``event``, ``request_id``) match
cacheblend_vllm/trace.py:19-64 so existing trace analysis keeps working.
Host enqueue times only; device timings come from CUDA events in bench.py.
"""

from __future__ import annotations

import json
import os
import threading
import time
from pathlib import Path
from typing import Any


class PipelineTracer:
    def __init__(self, component: str):
        self.component = component
        self._lock = threading.Lock()
        self._file = None
        directory = os.getenv("CACHEBLEND_TRACE_DIR")
        if directory:
            root = Path(directory)
            root.mkdir(parents=True, exist_ok=True)
            self._file = (root / f"{component}-pid-{os.getpid()}.jsonl").open(
                "a", encoding="utf-8", buffering=1
            )
            self.emit("trace_started")

    @property
    def enabled(self) -> bool:
        return self._file is not None

    def emit(self, event: str, request_id: str | None = None, **fields: Any) -> None:
        if self._file is None:
            return
        record: dict[str, Any] = {
            "timestamp_ns": time.time_ns(),
            "monotonic_ns": time.monotonic_ns(),
            "pid": os.getpid(),
            "thread_id": threading.get_ident(),
            "component": self.component,
            "event": event,
        }
        if request_id is not None:
            record["request_id"] = request_id
        record.update(fields)
        line = json.dumps(record, sort_keys=True, separators=(",", ":"))
        with self._lock:
            if self._file is not None:
                self._file.write(line + "\n")

    def close(self) -> None:
        with self._lock:
            handle, self._file = self._file, None
        if handle is not None:
            handle.close()
