"""Pinned host arena for the Store path's entries.

The reference keeps one CPU tensor per published layer of every entry
(cacheblend_vllm/storage.py:35-294); here the Store path publishes views into
one pinned arena instead:

* an entry slot holds every layer of one chunk, ``[num_layers][2, chunk, H, D]``,
  so a Store batch (one layer of consecutive chunks) lands with one strided
  copy (row pitch = the entry size) when its entries are consecutive slots;
* pinned memory is taken in segments of about ``segment_bytes`` as slots are
  first needed, never beyond ``max_bytes``: the byte budget is a hard bound on
  pinned memory, whatever the eviction pattern (views of per-batch buffers
  keep a whole batch alive while any of its chunks survives);
* slots come from a next-fit cursor, so entries begun together and freed in
  LRU order stay contiguous.

All methods are called under the store's lock.
"""

from __future__ import annotations

import numpy as np
import torch


class PinnedArena:
    def __init__(self, layer_bytes: int, num_layers: int, max_bytes: int,
                 segment_bytes: int = 1 << 30, pin_memory: bool = True):
        if layer_bytes <= 0 or num_layers <= 0:
            raise ValueError("layer_bytes and num_layers must be positive")
        self.layer_bytes = int(layer_bytes)
        self.num_layers = int(num_layers)
        self.entry_bytes = self.layer_bytes * self.num_layers
        self.capacity = int(max_bytes) // self.entry_bytes
        if self.capacity <= 0:
            raise ValueError("max_bytes is smaller than one entry")
        self.slots_per_segment = max(1, min(self.capacity, int(segment_bytes) // self.entry_bytes))
        self.pin_memory = pin_memory
        self._segments: list[torch.Tensor] = []
        self._free = np.zeros(self.capacity, dtype=bool)  # slots of allocated segments that are free
        self._allocated = 0  # slots backed by segments
        self._used = 0
        self._cursor = 0
        # per (segment, layer shape, dtype): the segment as [slots, layers, *shape], so a
        # run of consecutive slots yields its views with one slice and one unbind
        self._shaped: dict[tuple[int, tuple[int, ...], torch.dtype], torch.Tensor] = {}

    # ---- introspection --------------------------------------------------------
    @property
    def used_slots(self) -> int:
        return self._used

    @property
    def pinned_bytes(self) -> int:
        return sum(seg.numel() for seg in self._segments)

    # ---- slots ----------------------------------------------------------------
    def alloc(self) -> int | None:
        """A free slot (next fit from the cursor), growing by one segment when every
        backed slot is taken; None when the budget is exhausted."""
        if self._used == self._allocated and not self._grow():
            return None
        free = self._free[: self._allocated]
        hit = np.flatnonzero(free[self._cursor:])
        if hit.size:
            slot = self._cursor + int(hit[0])
        else:
            slot = int(np.flatnonzero(free[: self._cursor])[0])
        self._free[slot] = False
        self._used += 1
        self._cursor = slot + 1 if slot + 1 < self._allocated else 0
        return slot

    def free(self, slot: int) -> None:
        if not 0 <= slot < self._allocated or self._free[slot]:
            raise ValueError(f"slot {slot} is not allocated")
        self._free[slot] = True
        self._used -= 1

    def _grow(self) -> bool:
        if self._allocated >= self.capacity:
            return False
        count = min(self.slots_per_segment, self.capacity - self._allocated)
        segment = torch.empty(count * self.entry_bytes, dtype=torch.uint8, pin_memory=self.pin_memory)
        self._segments.append(segment)
        self._free[self._allocated : self._allocated + count] = True
        if self._used == self._allocated:
            self._cursor = self._allocated
        self._allocated += count
        return True

    def _locate(self, slot: int) -> tuple[torch.Tensor, int]:
        index, offset = divmod(slot, self.slots_per_segment)
        return self._segments[index], offset * self.entry_bytes

    # ---- addressing -----------------------------------------------------------
    def layer_view(self, slot: int, layer: int, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        """The bytes of ``layer`` in ``slot`` as a contiguous tensor of ``shape``."""
        segment, base = self._locate(slot)
        start = base + layer * self.layer_bytes
        return segment[start : start + self.layer_bytes].view(dtype).view(shape)

    def _shaped_segment(self, index: int, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        key = (index, shape, dtype)
        view = self._shaped.get(key)
        if view is None:
            segment = self._segments[index]
            view = segment.view(dtype).view(segment.numel() // self.entry_bytes, self.num_layers, *shape)
            self._shaped[key] = view
        return view

    def layer_views(self, slots: list[int], layer: int, shape: tuple[int, ...],
                    dtype: torch.dtype) -> list[torch.Tensor]:
        """``layer_view`` of every slot in ``slots``, built per run of consecutive slots of
        one segment with a single slice (the Store path publishes a batch at a time)."""
        shape = tuple(shape)
        out: list[torch.Tensor] = []
        i = 0
        while i < len(slots):
            index, first = divmod(slots[i], self.slots_per_segment)
            j = i + 1
            while (j < len(slots) and slots[j] == slots[j - 1] + 1
                   and slots[j] // self.slots_per_segment == index):
                j += 1
            view = self._shaped_segment(index, shape, dtype)
            out.extend(view[first : first + (j - i), layer].unbind(0))
            i = j
        return out

    def layer_ptr(self, slot: int, layer: int) -> int:
        segment, base = self._locate(slot)
        return segment.data_ptr() + base + layer * self.layer_bytes
