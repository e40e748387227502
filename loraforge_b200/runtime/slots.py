"""Generation-checked adapter slots: the handle type and the synchronous CPU pool.

Drop-in for ``loraforge.runtime.slots`` (src/loraforge/runtime/slots.py:15-111):
same constructor checks, handle semantics and error messages.  A slot holds the
modules of one PEFT adapter; replacing or evicting its occupant bumps the slot's
generation, which invalidates every handle issued before.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from threading import RLock
from uuid import uuid4

from loraforge_b200.adapters import AdapterModule, load_peft_adapter


@dataclass(frozen=True)
class SlotHandle:
    """Ownership token: valid only for its pool and the slot generation it names."""

    pool: str
    slot: int
    generation: int


def payload_bytes(modules) -> int:
    """Bytes of the A and B factors of ``modules`` (no padding or staging)."""
    return sum(t.numel() * t.element_size() for m in modules for t in (m.a, m.b))


class SlotTable:
    """Capacity, byte budget, generations and handle checks shared by both pools."""

    def __init__(self, capacity: int, max_tensor_bytes: int | None):
        if type(capacity) is not int or capacity <= 0:
            raise ValueError("capacity must be a positive integer")
        if max_tensor_bytes is not None and (type(max_tensor_bytes) is not int or max_tensor_bytes < 0):
            raise ValueError("max_tensor_bytes must be a nonnegative integer")
        self.capacity = capacity
        self.limit = max_tensor_bytes
        self.pool_id = uuid4().hex
        self.generations = [0] * capacity
        self.lock = RLock()

    def check_slot(self, slot) -> None:
        if type(slot) is not int or not 0 <= slot < self.capacity:
            raise ValueError("slot outside pool capacity")

    def check_handle(self, handle, occupied) -> None:
        if not isinstance(handle, SlotHandle) or handle.pool != self.pool_id:
            raise ValueError("handle belongs to a different pool")
        self.check_slot(handle.slot)
        if handle.generation != self.generations[handle.slot] or handle.slot not in occupied:
            raise ValueError("stale or evicted slot handle")

    def check_budget(self, resident_other: int, incoming: int) -> None:
        if self.limit is not None and resident_other + incoming > self.limit:
            raise ValueError("resident tensor byte limit exceeded")

    def issue(self, slot: int) -> SlotHandle:
        self.generations[slot] += 1
        return SlotHandle(self.pool_id, slot, self.generations[slot])

    def retire(self, slot: int) -> None:
        self.generations[slot] += 1


def _detached(modules) -> tuple[AdapterModule, ...]:
    return tuple(
        AdapterModule(m.name, m.a.detach().clone().contiguous(), m.b.detach().clone().contiguous(),
                      m.alpha, m.use_rslora)
        for m in modules
    )


class AdapterSlots:
    """Compact CPU snapshots in a fixed number of explicitly managed slots.

    ``load`` clones the factors into contiguous storage; a failed load leaves the
    previous occupant and its handle valid.  ``resolve`` returns fresh clones, so
    callers cannot modify pool storage.  No automatic eviction; one lock per pool.
    """

    def __init__(self, capacity: int, *, max_tensor_bytes: int | None = None):
        self._table = SlotTable(capacity, max_tensor_bytes)
        self._entries: dict[int, tuple[AdapterModule, ...]] = {}

    @property
    def tensor_bytes(self) -> int:
        """Resident factor bytes (excluding Python objects and transient copies)."""
        with self._table.lock:
            return sum(payload_bytes(m) for m in self._entries.values())

    def load(self, source: str | Path, slot: int) -> SlotHandle:
        """Read a local PEFT directory and atomically replace one slot's occupant."""
        table = self._table
        with table.lock:
            table.check_slot(slot)
            modules = _detached(load_peft_adapter(source).modules)
            table.check_budget(self.tensor_bytes - payload_bytes(self._entries.get(slot, ())),
                               payload_bytes(modules))
            self._entries[slot] = modules
            return table.issue(slot)

    def resolve(self, handle: SlotHandle) -> tuple[AdapterModule, ...]:
        """Detached copies of the occupant's modules (rank and scaling preserved)."""
        with self._table.lock:
            self._table.check_handle(handle, self._entries)
            return _detached(self._entries[handle.slot])

    def evict(self, handle: SlotHandle) -> None:
        """Drop the occupant and invalidate its handle; earlier copies stay valid."""
        with self._table.lock:
            self._table.check_handle(handle, self._entries)
            del self._entries[handle.slot]
            self._table.retire(handle.slot)
