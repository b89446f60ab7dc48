"""Opt-in JSONL pipeline tracing, enabled by ``CACHEBLEND_TRACE_DIR``.

Compatibility contract with the reference's trace files
(cacheblend_vllm/trace.py:19-64), so existing analysis scripts read these:
one file per component and process, ``<dir>/<component>-pid-<pid>.jsonl``;
one JSON object per line with sorted keys and compact separators; fields
``timestamp_ns``, ``monotonic_ns``, ``pid``, ``thread_id``, ``component``,
``event``, ``request_id`` (when given) plus the event's own fields; a
``trace_started`` record when the file opens.

Design here: the file is opened with ``O_APPEND`` and every record is a single
``os.write`` of a complete line, so concurrent writers (the forward thread and
the Store publisher threads) never interleave inside a line; the lock only
orders a write against ``close``.  Records carry host enqueue times; device
timings come from CUDA events (bench.py).
"""

from __future__ import annotations

import json
import os
import threading
import time
from typing import Any

TRACE_DIR_ENV = "CACHEBLEND_TRACE_DIR"


def _open_trace_file(component: str) -> int | None:
    directory = os.environ.get(TRACE_DIR_ENV)
    if not directory:
        return None
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{component}-pid-{os.getpid()}.jsonl")
    return os.open(path, os.O_WRONLY | os.O_CREAT | os.O_APPEND, 0o644)


class PipelineTracer:
    """Appends trace records for one component; a no-op when tracing is off."""

    def __init__(self, component: str):
        self.component = component
        self._fd = _open_trace_file(component)
        self._close_lock = threading.Lock()
        if self._fd is not None:
            self.emit("trace_started")

    @property
    def enabled(self) -> bool:
        return self._fd is not None

    def emit(self, event: str, request_id: str | None = None, **fields: Any) -> None:
        if self._fd is None:
            return
        fields.update(
            timestamp_ns=time.time_ns(),
            monotonic_ns=time.monotonic_ns(),
            pid=os.getpid(),
            thread_id=threading.get_ident(),
            component=self.component,
            event=event,
        )
        if request_id is not None:
            fields["request_id"] = request_id
        line = (json.dumps(fields, sort_keys=True, separators=(",", ":")) + "\n").encode()
        with self._close_lock:
            if self._fd is not None:
                os.write(self._fd, line)

    def close(self) -> None:
        with self._close_lock:
            fd, self._fd = self._fd, None
        if fd is not None:
            os.close(fd)
