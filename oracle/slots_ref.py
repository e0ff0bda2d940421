"""Slot-policy oracle: restatement of src/polylora/cache.py:60-84 and 97-117
(ensure_resident / _allocate_or_evict / _touch) over plain Python state.

Iteration over the batch's ``needed`` set follows the reference (a set), so
LRU ties depend on the string hash seed exactly as in the reference; fixtures
are produced and checked with PYTHONHASHSEED=0.
"""

from __future__ import annotations

from collections import OrderedDict


class SlotPolicy:
    def __init__(self, known: set[str], max_gpu_adapters: int, base: str = "__base__") -> None:
        self.known = set(known)
        self.base = base
        self.max_gpu = max_gpu_adapters
        self.num_slots = max_gpu_adapters + 1
        self.adapter_to_slot = {base: 0}
        self.slot_to_adapter: list[str | None] = [base] + [None] * max_gpu_adapters
        self.lru: OrderedDict[str, None] = OrderedDict()
        self.loads: list[tuple[str, int]] = []

    def ensure_resident(self, adapter_ids: list[str]) -> list[int]:
        needed = {a for a in adapter_ids if a != self.base}
        unknown = [a for a in needed if a not in self.known and a != self.base]
        if unknown:
            raise KeyError(f"Unknown LoRA adapter id(s): {unknown}")
        if len(needed) > self.max_gpu:
            raise RuntimeError("Batch needs more adapters than GPU cache capacity")
        for a in sorted(needed):  # cache.py:68-70
            if a not in self.adapter_to_slot:
                slot = self._allocate_or_evict(needed)
                self.adapter_to_slot[a] = slot
                self.slot_to_adapter[slot] = a
                self.loads.append((a, slot))
                self._touch(a)
        for a in needed:  # cache.py:72-73
            self._touch(a)
        return [0 if a == self.base else self.adapter_to_slot[a] for a in adapter_ids]

    def _allocate_or_evict(self, needed: set[str]) -> int:
        for slot in range(1, self.num_slots):  # cache.py:98-100
            if self.slot_to_adapter[slot] is None:
                return slot
        for a in list(self.lru.keys()):  # cache.py:102-116
            if a in needed:
                continue
            slot = self.adapter_to_slot.pop(a)
            self.lru.pop(a, None)
            self.slot_to_adapter[slot] = None
            return slot
        raise RuntimeError("No evictable LoRA adapter slot is available")

    def _touch(self, a: str) -> None:  # cache.py:152-157
        if a == self.base:
            return
        self.lru.pop(a, None)
        self.lru[a] = None
