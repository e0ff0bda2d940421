"""GPU adapter slots: dense per-module tensors indexed by slot.

Same public state and slot policy as the reference's ``GpuAdapterCache``
(src/polylora/cache.py:19-162): ``A[module]`` (num_slots, in, max_rank),
``B[module]`` (num_slots, max_rank, out), ``ranks`` / ``scales``, slot 0
reserved for ``__base__`` (rank 0, scale 0), ``adapter_to_slot``,
``slot_to_adapter``, ``lru``; non-resident adapters of a batch are placed in
``sorted()`` order into the first free slot, else the least recently used
slot not needed by the batch.

What changes is the refill (cache.py:97-150).  On a CUDA device a refill is
one pinned host-to-device copy of the adapter's packed image plus one scatter
kernel (``plora_slot_fill``) on a side stream; the side stream waits only for
the last forward that read the slot, and the forward that needs the slot
waits on the refill's event, so refills overlap with unrelated compute.  The
scatter rewrites the whole slot (zero padding past the rank, rank/scale of
absent modules set to 0), which covers the reference's zero-on-evict.
"""

from __future__ import annotations

import contextlib

from collections import OrderedDict
from dataclasses import dataclass

import torch

from . import _native
from .config import PolyLoraConfig
from .sgmv import dtype_code
from .store import CpuAdapterStore


@dataclass(frozen=True)
class ModuleSpec:
    name: str
    in_features: int
    out_features: int


class GpuAdapterCache:
    def __init__(
        self,
        store: CpuAdapterStore,
        module_specs: list[ModuleSpec],
        config: PolyLoraConfig,
        device: torch.device,
        dtype: torch.dtype,
    ) -> None:
        self.store = store
        self.config = config
        self.device = torch.device(device)
        self.dtype = dtype
        self.num_slots = config.max_gpu_adapters + 1
        base = config.base_adapter_id
        self.adapter_to_slot: dict[str, int] = {base: 0}
        self.slot_to_adapter: list[str | None] = [base] + [None] * config.max_gpu_adapters
        self.lru: OrderedDict[str, None] = OrderedDict()
        self.module_specs = {spec.name: spec for spec in module_specs}
        self.module_names = [spec.name for spec in module_specs]
        self.stats = {"hits": 0, "misses": 0, "evictions": 0, "h2d_bytes": 0}
        self._refill_stream: torch.cuda.Stream | None = None
        self._staging: torch.Tensor | None = None
        self._inflight: list[tuple[torch.cuda.Event, torch.Tensor]] = []
        self._slot_last_use: dict[int, torch.cuda.Event] = {}
        self.ready_event: torch.cuda.Event | None = None
        self._allocate(self.device, self.dtype)
        self._publish_image_spec()

    # ------------------------------------------------------------------ storage
    def _allocate(self, device: torch.device, dtype: torch.dtype, src: "GpuAdapterCache | None" = None) -> None:
        ns, r = self.num_slots, self.config.max_rank
        n_mod = len(self.module_names)
        old = (self.A, self.B, self._ranks2d, self._scales2d) if src is not None else None
        self.A = {}
        self.B = {}
        for spec in self.module_specs.values():
            if old is None:
                self.A[spec.name] = torch.zeros(ns, spec.in_features, r, device=device, dtype=dtype)
                self.B[spec.name] = torch.zeros(ns, r, spec.out_features, device=device, dtype=dtype)
            else:
                self.A[spec.name] = old[0][spec.name].to(device=device, dtype=dtype).contiguous()
                self.B[spec.name] = old[1][spec.name].to(device=device, dtype=dtype).contiguous()
        if old is None:
            self._ranks2d = torch.zeros(n_mod, ns, device=device, dtype=torch.int32)
            self._scales2d = torch.zeros(n_mod, ns, device=device, dtype=torch.float32)
        else:
            self._ranks2d = old[2].to(device=device).contiguous()
            self._scales2d = old[3].to(device=device).contiguous()
        self.ranks = {name: self._ranks2d[i] for i, name in enumerate(self.module_names)}
        self.scales = {name: self._scales2d[i] for i, name in enumerate(self.module_names)}
        # per-slot max rank over modules: rows of a slot are active in the
        # forward's segment table when any module gives them work
        self.table_ranks = (
            self._ranks2d.amax(dim=0).to(torch.int32).contiguous()
            if n_mod
            else torch.zeros(ns, device=device, dtype=torch.int32)
        )
        self._module_table = None
        if device.type == "cuda":
            mods = (_native.SlotModule * max(n_mod, 1))()
            for i, name in enumerate(self.module_names):
                spec = self.module_specs[name]
                mods[i].lora_a = self.A[name].data_ptr()
                mods[i].lora_b = self.B[name].data_ptr()
                mods[i].ranks = self.ranks[name].data_ptr()
                mods[i].scales = self.scales[name].data_ptr()
                mods[i].in_features = spec.in_features
                mods[i].out_features = spec.out_features
            raw = torch.frombuffer(bytearray(bytes(mods)), dtype=torch.uint8)
            self._module_table = raw.to(device)

    def to(self, device: torch.device, dtype: torch.dtype) -> None:
        device = torch.device(device)
        if self.device == device and self.dtype == dtype:
            return
        self.synchronize()
        self._allocate(device, dtype, src=self)
        self.device = device
        self.dtype = dtype
        self._publish_image_spec()
        self._staging = None
        self._slot_last_use.clear()
        self.ready_event = None

    def _publish_image_spec(self) -> None:
        """Tells the CPU tier the layout of this cache's slot images (CUDA only)."""
        setter = getattr(self.store, "set_image_spec", None)
        if setter is not None:
            cuda = self.device.type == "cuda"
            setter(self.module_names if cuda else None, self.dtype if cuda else None)

    # ------------------------------------------------------------------ slot policy
    def ensure_resident(self, adapter_ids: list[str]) -> torch.Tensor:
        base = self.config.base_adapter_id
        needed = {a for a in adapter_ids if a != base}
        unknown = [a for a in needed if a not in self.store]
        if unknown:
            raise KeyError(f"Unknown LoRA adapter id(s): {unknown}")
        if len(needed) > self.config.max_gpu_adapters:
            raise RuntimeError("Batch needs more adapters than GPU cache capacity")
        for adapter_id in sorted(needed):
            if adapter_id in self.adapter_to_slot:
                self.stats["hits"] += 1
            else:
                self.stats["misses"] += 1
                self._load_adapter_into_slot(adapter_id, self._allocate_or_evict(needed))
        for adapter_id in needed:  # same (set) order as the reference: LRU ties follow it
            self._touch(adapter_id)
        self._sync_cpu_eviction_exclusions()
        slots = [0 if a == base else self.adapter_to_slot[a] for a in adapter_ids]
        host = torch.tensor(slots, dtype=torch.int64)
        if self.device.type == "cuda":
            return host.pin_memory().to(self.device, non_blocking=True)
        return host.to(self.device)

    def _allocate_or_evict(self, needed: set[str]) -> int:
        for slot in range(1, self.num_slots):
            if self.slot_to_adapter[slot] is None:
                return slot
        for adapter_id in list(self.lru.keys()):
            if adapter_id in needed:
                continue
            slot = self.adapter_to_slot.pop(adapter_id)
            self.lru.pop(adapter_id, None)
            self.slot_to_adapter[slot] = None
            self.stats["evictions"] += 1
            return slot
        raise RuntimeError("No evictable LoRA adapter slot is available")

    def _validate(self, adapter_id: str, adapter) -> None:
        for name, spec in self.module_specs.items():
            w = adapter.layers.get(name)
            if w is None:
                continue
            if w.rank > self.config.max_rank:
                raise ValueError(f"Adapter {adapter_id!r} rank {w.rank} exceeds max_rank {self.config.max_rank}")
            if tuple(w.A.shape) != (spec.in_features, w.rank):
                raise ValueError(f"LoRA A shape mismatch for adapter {adapter_id!r}, module {name!r}")
            if tuple(w.B.shape) != (w.rank, spec.out_features):
                raise ValueError(f"LoRA B shape mismatch for adapter {adapter_id!r}, module {name!r}")

    def _load_adapter_into_slot(self, adapter_id: str, slot: int) -> None:
        # one critical section against the CPU tier's prefetch workers: the
        # adapter stays in the tier and its image's slab is not reused until
        # the copy reading it has been recorded (note_image_use)
        lock = getattr(self.store, "locked", None)
        with lock() if lock is not None else contextlib.nullcontext():
            # A failure anywhere before the slot is filled (the CPU or disk tier
            # cannot produce the adapter, its weights do not fit the modules, its
            # image cannot be built) leaves the slot free with rank 0 and scale 0
            # in every module, the state the reference's zero-on-evict leaves
            # (cache.py:97-150), and the error propagates.
            try:
                adapter = self.store.get(adapter_id)
                self._validate(adapter_id, adapter)
                if self.device.type == "cuda":
                    self._fill_slot_native(adapter_id, slot)
                else:
                    self._fill_slot_host(adapter, slot)
            except BaseException:
                self._clear_slot(slot)
                raise
            self.adapter_to_slot[adapter_id] = slot
            self.slot_to_adapter[slot] = adapter_id
            self._touch(adapter_id)
            self._sync_cpu_eviction_exclusions()

    def _touch(self, adapter_id: str) -> None:
        if adapter_id == self.config.base_adapter_id:
            return
        self.lru.pop(adapter_id, None)
        self.lru[adapter_id] = None
        self.store.touch(adapter_id)

    def _sync_cpu_eviction_exclusions(self) -> None:
        self.store.set_eviction_exclusions({a for a in self.slot_to_adapter[1:] if a is not None})

    # ------------------------------------------------------------------ refills
    def refill_stream(self) -> torch.cuda.Stream:
        if self._refill_stream is None:
            self._refill_stream = torch.cuda.Stream(device=self.device)
        return self._refill_stream

    def _fill_slot_native(self, adapter_id: str, slot: int) -> None:
        image, ranks = self.store.slot_image(adapter_id, self.module_names, self.dtype)
        stream = self.refill_stream()
        compute = torch.cuda.current_stream(self.device)
        last = self._slot_last_use.pop(slot, None)
        if last is not None:
            stream.wait_event(last)  # the previous reader of this slot is done
        else:
            stream.wait_stream(compute)
        nbytes = image.numel()
        if self._staging is None or self._staging.numel() < nbytes:
            self._staging = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
            self._staging.record_stream(stream)
        _native.call(
            "plora_slot_fill",
            self._module_table.data_ptr(), len(self.module_names), slot, self.num_slots,
            self.config.max_rank, dtype_code(self.dtype), image.data_ptr(), nbytes,
            self._staging.data_ptr(), self._staging.numel(), stream.cuda_stream,
        )
        with torch.cuda.stream(stream):
            self.table_ranks[slot].fill_(max(ranks) if ranks else 0)
        event = torch.cuda.Event()
        event.record(stream)
        self.ready_event = event
        self.stats["h2d_bytes"] += nbytes
        self.store.note_image_use(adapter_id, self.module_names, self.dtype, event)
        self._inflight = [(e, t) for e, t in self._inflight if not e.query()]
        self._inflight.append((event, image))

    def _fill_slot_host(self, adapter, slot: int) -> None:
        # Host-memory bookkeeping path for caches placed on a CPU device (the
        # LoRA kernels themselves only run on CUDA).
        best = 0
        for i, name in enumerate(self.module_names):
            self.A[name][slot].zero_()
            self.B[name][slot].zero_()
            w = adapter.layers.get(name)
            if w is None:
                self._ranks2d[i, slot] = 0
                self._scales2d[i, slot] = 0.0
                continue
            self.A[name][slot, :, : w.rank].copy_(w.A.to(self.dtype))
            self.B[name][slot, : w.rank, :].copy_(w.B.to(self.dtype))
            self._ranks2d[i, slot] = int(w.rank)
            self._scales2d[i, slot] = float(w.scale)
            best = max(best, int(w.rank))
        self.table_ranks[slot] = best

    def _clear_slot(self, slot: int) -> None:
        if self.device.type == "cuda":
            stream = self.refill_stream()
            stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(stream):
                self._ranks2d[:, slot].zero_()
                self._scales2d[:, slot].zero_()
                self.table_ranks[slot].zero_()
            event = torch.cuda.Event()
            event.record(stream)
            self.ready_event = event
        else:
            self._ranks2d[:, slot].zero_()
            self._scales2d[:, slot].zero_()
            self.table_ranks[slot] = 0

    def mark_slots_used(self, slots: set[int]) -> None:
        """Records that work enqueued so far on the current stream reads `slots`."""
        if self.device.type != "cuda" or not slots:
            return
        event = torch.cuda.Event()
        event.record(torch.cuda.current_stream(self.device))
        for slot in slots:
            self._slot_last_use[slot] = event

    def wait_ready(self, stream: torch.cuda.Stream | None = None) -> None:
        """Makes `stream` (default: current) wait for the pending refills.

        Not during stream capture: a captured forward (``GraphedForward``)
        orders the refills before each replay, outside the graph."""
        if self.ready_event is not None and not torch.cuda.is_current_stream_capturing():
            (stream or torch.cuda.current_stream(self.device)).wait_event(self.ready_event)

    def synchronize(self) -> None:
        if self._refill_stream is not None:
            self._refill_stream.synchronize()
        self._inflight.clear()


__all__ = ["GpuAdapterCache", "ModuleSpec"]
