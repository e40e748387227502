"""GPU adapter slots: one pinned staging block and one host-to-device copy per load.

Drop-in for ``loraforge.runtime.GPUAdapterSlots`` (src/loraforge/runtime/gpu.py:25-186):
same constructor, ``load`` / ``borrow`` / ``evict`` / ``collect`` / ``tensor_bytes``,
lease rules and error messages.  The B200 form differs in how a load moves bytes:
every factor of the adapter is packed into ONE pinned host block at 256-byte
aligned offsets and crosses PCIe in ONE ``cudaMemcpyAsync`` into ONE device
allocation, of which the returned modules are views (the reference issues two
copies per module into separate allocations).  A 1024-slot pool of 200-module
adapters therefore pays one copy launch per adapter instead of 400, and a lease
records the consumer stream on one allocation.

Ordering and lifetime:

* the copy is enqueued on the pool device's current stream and an event is
  recorded after it; ``borrow`` makes the borrowing stream wait on that event;
* ``borrow`` records the borrowing stream on the device allocation, so the caching
  allocator keeps it alive for work enqueued during the lease even after the slot
  is replaced or evicted;
* a slot with an active lease cannot be replaced or evicted;
* the pinned block is kept until its copy has completed (``collect`` and every
  later pool call release finished ones without waiting);
* nothing runs under CUDA graph capture.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass
from pathlib import Path

from loraforge_b200.adapters import AdapterModule, load_peft_adapter

from .slots import SlotHandle, SlotTable, payload_bytes

_ALIGN = 256


@dataclass
class _Resident:
    modules: tuple[AdapterModule, ...]
    device_block: object
    staging: object
    ready: object
    readers: int = 0


def pack_layout(modules) -> tuple[list[tuple[int, int]], int]:
    """(byte offset, byte length) of each module's A then B in one block, and its size."""
    spans, cursor = [], 0
    for m in modules:
        for t in (m.a, m.b):
            n = t.numel() * t.element_size()
            spans.append((cursor, n))
            cursor += (n + _ALIGN - 1) // _ALIGN * _ALIGN
    return spans, max(cursor, _ALIGN)


def _view(block, span, like):
    offset, nbytes = span
    return block[offset : offset + nbytes].view(like.dtype).view(like.shape)


class GPUAdapterSlots:
    """Explicit GPU slots; use the factors only inside ``borrow`` on its current stream."""

    def __init__(self, capacity: int, *, device: str, max_tensor_bytes: int | None = None):
        import torch

        self._table = SlotTable(capacity, max_tensor_bytes)
        selected = torch.device(device)
        if selected.type != "cuda" or selected.index is None:
            raise ValueError("device must explicitly select a CUDA/ROCm GPU index")
        self.device = selected
        self._stream()
        self._entries: dict[int, _Resident] = {}
        self._pending: list[_Resident] = []

    def _stream(self):
        import torch

        with torch.cuda.device(self.device):
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("GPU slots do not support graph capture")
            return torch.cuda.current_stream(self.device)

    def _reap(self) -> None:
        self._pending = [e for e in self._pending if not e.ready.query()]
        for entry in self._entries.values():
            if entry.staging is not None and entry.ready.query():
                entry.staging = None

    @property
    def tensor_bytes(self) -> int:
        """Committed factor bytes, excluding alignment padding, staging and retired blocks."""
        with self._table.lock:
            return sum(payload_bytes(e.modules) for e in self._entries.values())

    def load(self, source: str | Path, slot: int) -> SlotHandle:
        """Parse and pin on the host, then enqueue one H2D copy on the current stream.

        The returned handle can be borrowed at once from another stream (``borrow``
        inserts the event wait).  A failure leaves the previous occupant, its
        handle and the byte budget unchanged.
        """
        import torch

        table = self._table
        with table.lock:
            table.check_slot(slot)
            stream = self._stream()
            self._reap()
            old = self._entries.get(slot)
            if old is not None and old.readers:
                raise RuntimeError("slot has active leases")
            adapter = load_peft_adapter(source)
            table.check_budget(
                self.tensor_bytes - (payload_bytes(old.modules) if old else 0),
                payload_bytes(adapter.modules),
            )
            spans, total = pack_layout(adapter.modules)
            staging = torch.empty(total, dtype=torch.uint8, pin_memory=True)
            sources = [t for m in adapter.modules for t in (m.a, m.b)]
            for span, tensor in zip(spans, sources):
                _view(staging, span, tensor).copy_(tensor)
            try:
                with torch.cuda.device(self.device), torch.cuda.stream(stream):
                    block = torch.empty(total, dtype=torch.uint8, device=self.device)
                    block.copy_(staging, non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(stream)
            except BaseException:
                # Keep the pinned block alive until any copy already enqueued ends.
                stream.synchronize()
                raise
            views = iter(_view(block, span, t) for span, t in zip(spans, sources))
            modules = tuple(
                AdapterModule(m.name, next(views), next(views), m.alpha, m.use_rslora)
                for m in adapter.modules
            )
            if old is not None and old.staging is not None:
                self._pending.append(old)
            self._entries[slot] = _Resident(modules, block, staging, ready)
            return table.issue(slot)

    @contextmanager
    def borrow(self, handle: SlotHandle):
        """Lease the read-only factors for work enqueued on the current pool-device stream.

        Every launch that reads them must be enqueued inside the lease, on that
        stream; keep no references past it.  Scaling stays with the caller
        (``module.scaling``).
        """
        with self._table.lock:
            stream = self._stream()
            self._reap()
            self._table.check_handle(handle, self._entries)
            entry = self._entries[handle.slot]
            stream.wait_event(entry.ready)
            entry.device_block.record_stream(stream)
            entry.readers += 1
        try:
            yield entry.modules
        finally:
            with self._table.lock:
                entry.readers -= 1

    def evict(self, handle: SlotHandle) -> None:
        """Invalidate the occupant; stream records protect work already enqueued on it."""
        with self._table.lock:
            self._stream()
            self._reap()
            self._table.check_handle(handle, self._entries)
            entry = self._entries[handle.slot]
            if entry.readers:
                raise RuntimeError("slot has active leases")
            if entry.staging is not None:
                self._pending.append(entry)
            del self._entries[handle.slot]
            self._table.retire(handle.slot)

    def collect(self) -> None:
        """Release pinned staging blocks whose copies have finished, without waiting."""
        with self._table.lock:
            self._stream()
            self._reap()
