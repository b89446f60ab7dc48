"""The TP score reduction over NVLink peer memory, fused into the selection.

With tensor parallelism every rank scores its share of the KV heads and the
ranks' fp32 partial scores are summed before ``_select``
(cacheblend_vllm/ascend.py:764-770: ``tensor_model_parallel_all_reduce``,
then 771-796).  ``PeerScoreExchange.select`` does both in one kernel
(``cb_select_topk_peer``): each rank stores its partial scores straight into
every rank's exchange buffer over NVLink, waits for the others' (bounded), sums
them in rank order and selects.  No NCCL call sits between the deviation and
the selection, so the whole check layer -- and with it the whole step -- fits
in one CUDA graph on every rank.

The exchange buffers are plain ``cudaMalloc`` allocations shared through CUDA
IPC handles, which the ranks swap once over the process group (any backend).
Every rank must make the same sequence of ``select`` calls with the same
token count, budget and base mask; calls on one rank must run in order (one
stream, or streams ordered by events).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native

IPC_HANDLE_BYTES = 64
MAX_PEERS = 8
# exchange protocols of cb_select_topk_peer: fp32 rows + one fence + flags, or
# 64-bit (call number, score) words polled by the reader
PROTOCOLS = {"flags": 0, "low_latency": 1}
MAX_TOKENS = 8 * 42 * 1024  # one 8-CTA cluster's shared memory holds the scores' order keys
DEVICE_ERROR_PEER_WAIT = 5


class PeerExchangeUnavailable(RuntimeError):
    """Some rank could not create or map an exchange buffer (raised on every rank)."""


def default_protocol() -> str:
    """CACHEBLEND_B200_PEER_PROTOCOL (flags | low_latency), flags by default."""
    import os

    name = os.environ.get("CACHEBLEND_B200_PEER_PROTOCOL", "flags")
    if name not in PROTOCOLS:
        raise ValueError(f"CACHEBLEND_B200_PEER_PROTOCOL must be one of {sorted(PROTOCOLS)}, not {name!r}")
    return name


def _group_rank_world(group) -> tuple[int, int, object]:
    """(rank, world, torch process group) of a torch group or a vLLM GroupCoordinator."""
    import torch.distributed as dist

    if hasattr(group, "device_group") and hasattr(group, "rank_in_group"):
        return int(group.rank_in_group), int(group.world_size), group.cpu_group
    return dist.get_rank(group), dist.get_world_size(group), group


class PeerScoreExchange:
    """Exchange buffers of one TP group for selections over at most ``max_tokens`` tokens."""

    def __init__(self, group, max_tokens: int, device: torch.device | int | str,
                 protocol: str | None = None):
        import torch.distributed as dist

        self.protocol = default_protocol() if protocol is None else protocol
        if self.protocol not in PROTOCOLS:
            raise ValueError(f"protocol must be one of {sorted(PROTOCOLS)}, not {self.protocol!r}")
        self.device = torch.device(device)
        self.rank, self.world, self._group = _group_rank_world(group)
        if not 1 <= self.world <= MAX_PEERS:
            raise ValueError(f"peer exchange supports 1..{MAX_PEERS} ranks, not {self.world}")
        self.max_tokens = int(max_tokens)
        size = ctypes.c_int64(0)
        _native.call("cb_peer_select_buffer_size", self.world, self.max_tokens, ctypes.addressof(size))
        self.buffer_bytes = size.value
        index = self.device.index
        if index is None:
            index = torch.cuda.current_device() if self.device.type == "cuda" else 0
        self._index = index
        self._own = 0
        self._opened: list[int] = []
        self._closed = True
        # Every rank learns whether every other rank mapped everything, so that all
        # of them either use the exchange or raise PeerExchangeUnavailable together.
        failure = ""
        handle = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
        try:
            own = ctypes.c_void_p(0)
            _native.call("cb_peer_buffer_create", index, self.buffer_bytes, ctypes.addressof(own),
                         ctypes.addressof(handle))
            self._own = own.value
        except (RuntimeError, ValueError) as error:
            failure = f"rank {self.rank}: {error}"
        handles: list = [None] * self.world
        dist.all_gather_object(handles, None if failure else bytes(handle), group=self._group)
        addresses = [0] * self.world
        addresses[self.rank] = self._own
        if not failure and all(h is not None for h in handles):
            for r, h in enumerate(handles):
                if r == self.rank:
                    continue
                raw = (ctypes.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(h)
                mapped = ctypes.c_void_p(0)
                try:
                    _native.call("cb_peer_buffer_open", index, ctypes.addressof(raw), ctypes.addressof(mapped))
                except (RuntimeError, ValueError) as error:
                    failure = f"rank {self.rank} mapping rank {r}: {error}"
                    break
                addresses[r] = mapped.value
                self._opened.append(mapped.value)
        elif not failure:
            failure = "another rank could not create its exchange buffer"
        failures: list = [None] * self.world
        dist.all_gather_object(failures, failure, group=self._group)
        if any(failures):
            opened, self._opened = self._opened, []
            for mapped in opened:
                _native.call("cb_peer_buffer_close", self._index, mapped)
            dist.barrier(group=self._group)  # every mapping of this rank's buffer is gone
            self._release()
            raise PeerExchangeUnavailable("; ".join(f for f in failures if f))
        self._addresses = (ctypes.c_uint64 * self.world)(*addresses)
        self.device_error = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._closed = False

    def _release(self) -> None:
        """Free this rank's buffer once no rank maps it any more."""
        if self._own:
            _native.call("cb_peer_buffer_destroy", self._index, self._own)
            self._own = 0

    def select(
        self,
        partial: torch.Tensor,
        base_mask_device: torch.Tensor,
        k: int,
        capacity: int,
        stream: torch.cuda.Stream | None = None,
        summed: torch.Tensor | None = None,
        out: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Ascending indices of the base mask united with the top-``k`` non-base
        entries of the rank-ordered sum of every rank's ``partial`` scores
        (``capacity`` int64 entries, in ``out`` when given)."""
        if self._closed:
            raise RuntimeError("peer exchange is closed")
        _native.require_cuda(partial, base_mask_device)
        n = partial.numel()
        if partial.dtype != torch.float32 or not partial.is_contiguous():
            raise ValueError("partial scores must be a contiguous fp32 vector")
        if base_mask_device.dtype != torch.uint8 or base_mask_device.numel() != n:
            raise ValueError("base mask must be a uint8 vector shaped like the scores")
        if n > self.max_tokens:
            raise ValueError(f"{n} tokens exceed the exchange's {self.max_tokens}")
        if summed is not None and (summed.dtype != torch.float32 or summed.numel() < n):
            raise ValueError("summed must be an fp32 vector of at least n entries")
        if out is None:
            selected = torch.empty(capacity, dtype=torch.long, device=partial.device)
        else:
            if out.dtype != torch.long or out.numel() < capacity or not out.is_contiguous():
                raise ValueError("out must be a contiguous int64 vector of at least capacity entries")
            selected = out
        _native.call(
            "cb_select_topk_peer", partial.data_ptr(), base_mask_device.data_ptr(), n, k, selected.data_ptr(),
            capacity, ctypes.addressof(self._addresses), self.rank, self.world, self.max_tokens,
            PROTOCOLS[self.protocol], 0 if summed is None else summed.data_ptr(), self.device_error.data_ptr(),
            _native.stream_handle(stream),
        )
        return selected

    def _sync(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def check(self) -> None:
        """Raise if a call's wait for another rank gave up (synchronises the device)."""
        code = int(self.device_error.item())
        if code:
            raise RuntimeError(f"peer score exchange: a rank's scores did not arrive (device error {code})")

    def reset(self) -> None:
        """Zero the call counters of every rank (all ranks call this together)."""
        import torch.distributed as dist

        self._sync()
        dist.barrier(group=self._group)
        _native.call("cb_peer_buffer_reset", self._own, self.world, self.max_tokens, 0)
        self.device_error.zero_()
        self._sync()
        dist.barrier(group=self._group)

    def close(self) -> None:
        """Unmap the peers' buffers, then (after every rank did) free this rank's."""
        import torch.distributed as dist

        if self._closed:
            return
        self._closed = True
        self._sync()
        dist.barrier(group=self._group)
        opened, self._opened = self._opened, []
        for mapped in opened:
            _native.call("cb_peer_buffer_close", self._index, mapped)
        dist.barrier(group=self._group)  # every rank unmapped this rank's buffer
        self._release()


class AllRanksExchange:
    """Every rank of a ``world``-rank exchange played by one launch on one GPU
    (``cb_select_topk_peer_all_ranks``; cluster r is rank r, every buffer local):
    the single-GPU check of the protocol, call after call."""

    def __init__(self, world: int, max_tokens: int, device: torch.device | int | str,
                 protocol: str = "flags"):
        if protocol not in PROTOCOLS:
            raise ValueError(f"protocol must be one of {sorted(PROTOCOLS)}, not {protocol!r}")
        self.protocol = protocol
        self.world = int(world)
        self.max_tokens = int(max_tokens)
        self.device = torch.device(device)
        size = ctypes.c_int64(0)
        _native.call("cb_peer_select_buffer_size", self.world, self.max_tokens, ctypes.addressof(size))
        step = (size.value + 255) // 256 * 256  # each rank's buffer 256-byte aligned
        self._buffers = torch.zeros(self.world * step, dtype=torch.uint8, device=self.device)
        base = self._buffers.data_ptr()
        self._addresses = (ctypes.c_uint64 * self.world)(*[base + r * step for r in range(self.world)])
        self.device_error = torch.zeros(1, dtype=torch.int32, device=self.device)

    def select(self, partials: torch.Tensor, base_mask_device: torch.Tensor, k: int,
               capacity: int) -> tuple[torch.Tensor, torch.Tensor]:
        """([world, capacity] selections, [world, n] summed scores) of one call."""
        _native.require_cuda(partials, base_mask_device)
        world, n = partials.shape
        if world != self.world or n > self.max_tokens:
            raise ValueError("partials must be [world, n <= max_tokens]")
        partials = partials.to(torch.float32).contiguous()
        selected = torch.empty(world, capacity, dtype=torch.long, device=self.device)
        summed = torch.empty(world, n, dtype=torch.float32, device=self.device)
        _native.call(
            "cb_select_topk_peer_all_ranks", partials.data_ptr(), base_mask_device.data_ptr(), n, k,
            selected.data_ptr(), capacity, ctypes.addressof(self._addresses), world, self.max_tokens,
            PROTOCOLS[self.protocol], summed.data_ptr(), self.device_error.data_ptr(), 0,
        )
        return selected, summed
