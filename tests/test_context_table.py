"""The per-context address table behind cb_sparse_q_scores_static
(pic-kvcache_b200/csrc/cb_context_cache.h), checked on the CPU: values are
keyed by the CUDA context handle, a second context on the same device gets its
own entry, a handle that comes back (a context destroyed and created again)
takes the newly looked-up address, and a full table refuses new contexts."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include <cstdio>
#include "cb_context_cache.h"

int main() {
  cb::ContextTable<void*, 3> table;
  int a = 0, b = 0, c = 0, d = 0;  // stand-ins for context handles
  char x = 0, y = 0, z = 0;        // stand-ins for device addresses
  if (table.find(&a, nullptr) != nullptr) return 1;
  if (!table.store(&a, &x) || table.find(&a, nullptr) != &x) return 2;
  // another context (e.g. an FFI host's own on the same device) has its own entry
  if (!table.store(&b, &y) || table.find(&b, nullptr) != &y || table.find(&a, nullptr) != &x) return 3;
  // a context handle reused after a reset: the new lookup replaces the old address
  if (!table.store(&a, &z) || table.find(&a, nullptr) != &z || table.size() != 2) return 4;
  if (!table.store(&c, &x) || table.size() != 3) return 5;
  if (table.store(&d, &y) || table.find(&d, nullptr) != nullptr) return 6;  // full
  std::puts("ok");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_context_table_follows_the_context(tmp_path):
    source = tmp_path / "table.cc"
    binary = tmp_path / "table"
    source.write_text(PROGRAM)
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(REPO / "pic-kvcache_b200" / "csrc"),
                    str(source), "-o", str(binary)], check=True)
    result = subprocess.run([str(binary)], capture_output=True, text=True)
    assert result.returncode == 0, result.returncode
    assert result.stdout.strip() == "ok"
