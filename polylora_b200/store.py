"""CPU and disk adapter tiers and PEFT LoRA loading.

API-compatible with the reference's ``src/polylora/store.py``:

* :class:`DiskAdapterCache` — store.py:36-148.  Bounded copy of PEFT adapter
  directories with a ``manifest.json`` (same file name, JSON layout
  ``{"adapters": [{"adapter_id", "path", "peft_adapter_name"}]}`` written with
  ``indent=2, sort_keys=True``, same directory naming) so existing caches load.
* :class:`CpuAdapterStore` — store.py:160-436.  LRU of per-module
  ``(A^T, B^T, rank, alpha/rank)``, PEFT validation with the same exception
  types and messages, eviction that skips GPU-resident adapters.

Added for the GPU tier: :meth:`CpuAdapterStore.slot_image` packs every module
of an adapter into one pinned buffer laid out for ``plora_slot_fill`` so a
GPU slot refill is a single host-to-device copy plus one scatter kernel (the
per-module tensors themselves stay in pageable memory).
:meth:`CpuAdapterStore.prefetch` parses disk adapters and builds their images
on worker threads ahead of use (prefetch from queued batches); the LRU and the
disk tier are guarded by one lock.
"""

from __future__ import annotations

import ctypes
import json
import shutil
import threading
from collections import OrderedDict
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from hashlib import sha256
from pathlib import Path
from typing import Any

import torch

from ._native import SlotRecord

_SUPPORTED_OPTIONS = ("use_dora", "lora_bias", "use_rslora")


def _load_safetensors(path: Path) -> dict[str, torch.Tensor]:
    try:
        from safetensors.torch import load_file
    except ImportError as exc:
        raise ImportError("safetensors is required to load adapter_model.safetensors") from exc
    return load_file(str(path), device="cpu")


def _load_torch_bin(path: Path) -> dict[str, torch.Tensor]:
    return torch.load(path, map_location="cpu")


_PEFT_WEIGHT_FILES = (("adapter_model.safetensors", _load_safetensors), ("adapter_model.bin", _load_torch_bin))

# adapter_config.json rules, checked in this order: (refuses the config, error message)
_CONFIG_RULES = (
    (lambda c: c.get("peft_type") not in (None, "LORA"), lambda c: f"Unsupported PEFT adapter type: {c.get('peft_type')!r}"),
    (lambda c: bool(c.get("use_dora", False)), lambda c: "DoRA adapters are not supported"),
    (lambda c: bool(c.get("use_rslora", False)), lambda c: "RS-LoRA adapters are not supported"),
    (lambda c: bool(c.get("lora_bias", False)), lambda c: "LoRA bias is not supported"),
    (lambda c: float(c.get("lora_dropout", 0.0)) != 0.0, lambda c: "LoRA dropout is not supported by the inference runtime"),
    (lambda c: "lora_alpha" not in c, lambda c: "adapter_config.json is missing lora_alpha"),
)


def _capacity(max_adapters: int | None) -> int | None:
    """An LRU tier's bound: None (unbounded) or a positive count."""
    if max_adapters is None or max_adapters >= 1:
        return max_adapters
    raise ValueError("max_adapters must be at least 1")


@dataclass(frozen=True)
class CpuLayerWeights:
    A: torch.Tensor  # (in_features, rank)
    B: torch.Tensor  # (rank, out_features)
    rank: int
    scale: float


@dataclass(frozen=True)
class CpuAdapter:
    adapter_id: str
    config: dict[str, Any]
    layers: dict[str, CpuLayerWeights]


@dataclass(frozen=True)
class DiskAdapterEntry:
    adapter_id: str
    path: Path
    peft_adapter_name: str


def _entry_dirname(adapter_id: str) -> str:
    safe = "".join(ch if (ch.isalnum() or ch in "-_.") else "_" for ch in adapter_id)
    return f"{safe or 'adapter'}-{sha256(adapter_id.encode('utf-8')).hexdigest()[:12]}"


class DiskAdapterCache:
    """Bounded LRU of PEFT adapter directories with a JSON manifest."""

    _MANIFEST_NAME = "manifest.json"

    def __init__(self, cache_dir: str | Path, max_adapters: int | None = None) -> None:
        # entries in LRU order (most recent last); the manifest on disk mirrors them
        self.max_adapters = _capacity(max_adapters)
        self.cache_dir = Path(cache_dir)
        self.entries: OrderedDict[str, DiskAdapterEntry] = OrderedDict()
        self._json_blocks: dict[str, str] = {}  # adapter_id -> its manifest entry, serialised
        self.cache_dir.mkdir(parents=True, exist_ok=True)
        self._load_manifest()
        self._evict_if_needed()  # a manifest written under a larger bound

    def __contains__(self, adapter_id: str) -> bool:
        return adapter_id in self.entries

    @property
    def manifest_path(self) -> Path:
        return self.cache_dir / self._MANIFEST_NAME

    def get(self, adapter_id: str) -> DiskAdapterEntry:
        """The entry of a registered adapter, which becomes the most recently used."""
        entry = self.entries.get(adapter_id)
        if entry is None:
            raise KeyError(f"Unknown disk LoRA adapter id: {adapter_id}")
        self.touch(adapter_id)
        return entry

    def touch(self, adapter_id: str) -> None:
        """Marks an entry most recently used; unknown ids are ignored."""
        if adapter_id not in self.entries:
            return
        self.entries.move_to_end(adapter_id)
        self._write_manifest()

    def add_adapter(self, adapter_id: str, adapter_path: str | Path, peft_adapter_name: str = "default") -> Path:
        source = Path(adapter_path)
        _validate_adapter_dir(source)
        target = self.cache_dir / _entry_dirname(adapter_id)
        if source.resolve() != target.resolve():
            if target.exists():
                shutil.rmtree(target)
            shutil.copytree(source, target)
        self.entries[adapter_id] = DiskAdapterEntry(adapter_id, target, peft_adapter_name)
        self._json_blocks.pop(adapter_id, None)
        self.entries.move_to_end(adapter_id)
        self._evict_if_needed(exclude={adapter_id})
        self._write_manifest()
        return target

    def _load_manifest(self) -> None:
        if not self.manifest_path.exists():
            return
        data = json.loads(self.manifest_path.read_text(encoding="utf-8"))
        for item in data.get("adapters", []):
            path = self.cache_dir / str(item["path"])
            if path.exists():  # entries whose directory vanished are dropped
                adapter_id = str(item["adapter_id"])
                self.entries[adapter_id] = DiskAdapterEntry(
                    adapter_id, path, str(item.get("peft_adapter_name", "default"))
                )

    def _json_block(self, e: DiskAdapterEntry) -> str:
        block = self._json_blocks.get(e.adapter_id)
        if block is None:
            fields = {"adapter_id": e.adapter_id, "path": e.path.name, "peft_adapter_name": e.peft_adapter_name}
            body = ",\n".join(f"      {json.dumps(k)}: {json.dumps(fields[k])}" for k in sorted(fields))
            block = "    {\n" + body + "\n    }"
            self._json_blocks[e.adapter_id] = block
        return block

    def _write_manifest(self) -> None:
        """The LRU order, written on every change as the reference does
        (store.py:60-63, 101-114): the bytes of ``json.dump(..., indent=2,
        sort_keys=True)``, assembled from cached per-entry blocks so that a
        touch of a large catalog costs a string join, not a re-serialisation."""
        if self.entries:
            text = '{\n  "adapters": [\n' + ",\n".join(self._json_block(e) for e in self.entries.values()) + "\n  ]\n}"
        else:
            text = '{\n  "adapters": []\n}'
        self.manifest_path.write_text(text, encoding="utf-8")

    def _evict_if_needed(self, exclude: set[str] | None = None) -> None:
        if self.max_adapters is None:
            return
        exclude = exclude or set()
        evicted = False
        while len(self.entries) > self.max_adapters:
            victim = next((a for a in self.entries if a not in exclude), None)
            if victim is None:
                raise RuntimeError("No evictable disk LoRA adapter is available")
            entry = self.entries.pop(victim)
            self._json_blocks.pop(victim, None)
            if entry.path.exists():
                shutil.rmtree(entry.path)
            evicted = True
        if evicted:
            self._write_manifest()

    # kept for callers of the reference's private helpers
    _entry_dirname = staticmethod(_entry_dirname)


def _validate_adapter_dir(adapter_path: Path) -> None:
    config = adapter_path / "adapter_config.json"
    if not config.exists():
        raise FileNotFoundError(f"PEFT adapter config not found: {config}")
    if not (adapter_path / "adapter_model.safetensors").exists() and not (adapter_path / "adapter_model.bin").exists():
        raise FileNotFoundError(f"No PEFT adapter weights found in {adapter_path}")


def _matches_module_name(module_name: str, allowed: list[str]) -> bool:
    return any(module_name == a or module_name.endswith(f".{a}") for a in allowed)


_LORA_MARKERS = (".lora_A.", ".lora_B.", ".lora_A.weight", ".lora_B.weight")


def _state_dict_lora_module_names(state_dict: dict[str, torch.Tensor]) -> set[str]:
    found: set[str] = set()
    for key in state_dict:
        for marker in _LORA_MARKERS:
            if marker in key:
                found.add(key.split(marker, 1)[0])
                break
    return found


def _find_lora_key(state_dict: dict[str, torch.Tensor], module_name: str, side: str, peft_adapter_name: str) -> str | None:
    suffixes = (f"{module_name}.{side}.{peft_adapter_name}.weight", f"{module_name}.{side}.weight")
    return next((k for k in state_dict if k.endswith(suffixes)), None)


def _lora_key_index(state_dict: dict[str, torch.Tensor], module_names: list[str],
                    peft_adapter_name: str) -> dict[tuple[str, str], str]:
    """(module, side) -> the key :func:`_find_lora_key` returns, in one pass.

    A key ``<prefix>.<side>[.<name>].weight`` matches every module whose name is
    a string suffix of ``<prefix>``; each key is filed under all such module
    names, and the first key in ``state_dict`` order wins, as in the scan."""
    wanted = set(module_names)
    index: dict[tuple[str, str], str] = {}
    for key in state_dict:
        for side in ("lora_A", "lora_B"):
            prefix = None
            for suffix in (f".{side}.{peft_adapter_name}.weight", f".{side}.weight"):
                if key.endswith(suffix):
                    prefix = key[: -len(suffix)]
                    break
            if prefix is None:
                continue
            for i in range(len(prefix)):
                tail = prefix[i:]
                if tail in wanted and (tail, side) not in index:
                    index[(tail, side)] = key
    return index


class PinnedSlabPool:
    """Page-locked slabs of one size for slot images.

    One large pinned arena is carved into slabs, so that building an image
    costs no page-locking call.  A released slab is reused only once the GPU
    copy that last read it (:meth:`note_use`) has completed.  Safe to use from
    several threads (prefetch workers release slabs outside the store's lock)."""

    def __init__(self, slab_bytes: int, slabs_per_arena: int = 32) -> None:
        self.slab_bytes = slab_bytes
        self.slabs_per_arena = slabs_per_arena
        self.arenas: list[torch.Tensor] = []
        self.free: list[torch.Tensor] = []
        self.retired: list[tuple[torch.Tensor, Any]] = []  # (slab, event of its last copy)
        self.last_use: dict[int, Any] = {}                 # slab data_ptr -> event
        self._mutex = threading.Lock()

    def acquire(self) -> torch.Tensor:
        with self._mutex:
            if not self.free and self.retired:
                still = []
                for slab, ev in self.retired:
                    (self.free.append(slab) if ev.query() else still.append((slab, ev)))
                self.retired = still
            if not self.free:
                arena = torch.empty(self.slabs_per_arena * self.slab_bytes, dtype=torch.uint8, pin_memory=True)
                self.arenas.append(arena)
                self.free.extend(arena[i * self.slab_bytes:(i + 1) * self.slab_bytes]
                                 for i in range(self.slabs_per_arena))
            return self.free.pop()

    def note_use(self, slab: torch.Tensor, event: Any) -> None:
        with self._mutex:
            self.last_use[slab.data_ptr()] = event

    def release(self, slab: torch.Tensor) -> None:
        with self._mutex:
            ev = self.last_use.pop(slab.data_ptr(), None)
            if ev is None or ev.query():
                self.free.append(slab)
            else:
                self.retired.append((slab, ev))


class CpuAdapterStore:
    """LRU of adapters in host memory, refilled from the disk tier on a miss."""

    def __init__(
        self,
        base_adapter_id: str = "__base__",
        max_adapters: int | None = None,
        disk_cache: DiskAdapterCache | None = None,
        module_names: list[str] | None = None,
        prefetch_workers: int | None = None,
    ) -> None:
        self.max_adapters = _capacity(max_adapters)
        self.base_adapter_id = base_adapter_id
        self.disk_cache = disk_cache
        self.module_names = module_names
        # resident adapters in LRU order (most recent last), and the ids the GPU
        # tier holds, which this tier must not evict
        self.adapters: OrderedDict[str, CpuAdapter] = OrderedDict()
        self.eviction_exclusions: set[str] = set()
        self._images: dict[tuple, tuple[torch.Tensor, list]] = {}
        self._slabs: dict[tuple, tuple[PinnedSlabPool, torch.Tensor]] = {}  # image key -> its slab
        self._pools: dict[int, PinnedSlabPool] = {}  # slab size class -> pool
        # (module_names, dtype) of the GPU cache's slot images, set by the cache:
        # disk loads then place safetensors bytes straight into the image
        self._image_spec: tuple[tuple[str, ...], torch.dtype] | None = None
        self._c_names: dict[tuple[str, ...], Any] = {}   # module names as a C string array
        self._pack_bytes: dict[tuple[str, ...], int] = {}  # largest packed image seen (slab sizing)
        # guards adapters / _images / _loading / the disk tier (reentrant: get -> load -> add)
        self._lock = threading.RLock()
        self._loading: dict[str, Future] = {}  # adapter id -> in-flight prefetch
        # one worker by default: parsing holds the GIL for most of its time, so the
        # gain is overlap with the serving thread, not parallel parsing
        self.prefetch_workers = prefetch_workers or 1
        self._pool: ThreadPoolExecutor | None = None

    # ------------------------------------------------------------------ LRU
    def __contains__(self, adapter_id: str) -> bool:
        if adapter_id == self.base_adapter_id or adapter_id in self.adapters:
            return True
        return self.disk_cache is not None and adapter_id in self.disk_cache

    def get(self, adapter_id: str) -> CpuAdapter:
        if adapter_id == self.base_adapter_id:
            raise KeyError(f"Base adapter {adapter_id!r} has no LoRA weights")
        pending = self._loading.get(adapter_id)
        if pending is not None and not self._lock._is_owned():
            # a prefetch is loading it: wait (its error is raised here).  A caller
            # holding the lock must not wait (the worker needs the lock to insert):
            # it loads synchronously below and the worker discards its copy.
            pending.result()
        with self._lock:
            if adapter_id not in self.adapters:
                if self.disk_cache is None or adapter_id not in self.disk_cache:
                    raise KeyError(f"Unknown LoRA adapter id: {adapter_id}")
                self._load_adapter_from_disk_cache(adapter_id)
            self.touch(adapter_id)
            return self.adapters[adapter_id]

    def touch(self, adapter_id: str) -> None:
        with self._lock:
            if adapter_id in self.adapters:
                self.adapters.move_to_end(adapter_id)

    def set_eviction_exclusions(self, adapter_ids: set[str]) -> None:
        with self._lock:
            self.eviction_exclusions = {a for a in adapter_ids if a != self.base_adapter_id}

    def set_image_spec(self, module_names: list[str] | None, dtype: torch.dtype | None) -> None:
        """Module order and dtype of the GPU cache's slot images (None: no GPU
        cache).  With a spec, an adapter read from a safetensors file whose LoRA
        tensors already have that dtype is loaded by copying the file's bytes
        into its slot image, the per-module weights being views of the image."""
        with self._lock:
            self._image_spec = (tuple(module_names), dtype) if module_names is not None and dtype is not None else None

    def locked(self):
        """The tier's lock, for a caller that must keep an adapter (and its
        image's slab) in place across several calls, e.g. a GPU slot refill
        while prefetch workers insert and evict."""
        return self._lock

    # ------------------------------------------------------------------ prefetch
    def wait_prefetches(self) -> None:
        """Waits for every prefetch started so far (errors are left to get())."""
        for fut in list(self._loading.values()):
            try:
                fut.result()
            except Exception:  # noqa: BLE001 - surfaced again by get()
                pass

    def prefetch(self, adapter_ids, image_dtype: torch.dtype | None = None,
                 module_names: list[str] | None = None) -> list[Future]:
        """Starts loading the listed adapters that are only on the disk tier.

        Worker threads parse each adapter (and, with ``image_dtype``, build its
        pinned slot image for ``module_names``) and insert it into the LRU, so
        that a later :meth:`get` / :meth:`slot_image` finds it resident; a
        :meth:`get` of an adapter still loading waits for it.  Returns the
        futures of the loads started (errors surface there and in :meth:`get`).
        No counterpart in the reference, which loads on first use."""
        started: list[Future] = []
        with self._lock:
            for aid in dict.fromkeys(adapter_ids):
                if (aid == self.base_adapter_id or aid in self.adapters or aid in self._loading
                        or self.disk_cache is None or aid not in self.disk_cache):
                    continue
                if self._pool is None:
                    self._pool = ThreadPoolExecutor(self.prefetch_workers, thread_name_prefix="plora-prefetch")
                fut = self._pool.submit(self._prefetch_one, aid, image_dtype, module_names)
                self._loading[aid] = fut
                started.append(fut)
        return started

    def _prefetch_one(self, adapter_id: str, image_dtype: torch.dtype | None,
                      module_names: list[str] | None) -> None:
        try:
            with self._lock:
                if adapter_id in self.adapters:
                    return
                if self.module_names is None:
                    raise RuntimeError("module_names must be configured before loading adapters from disk cache")
                entry = self.disk_cache.get(adapter_id)
                names = list(self.module_names)
            fast = self._load_direct(adapter_id, Path(entry.path), names, entry.peft_adapter_name)
            if fast is not None:
                with self._lock:
                    if adapter_id not in self.adapters:  # a synchronous load may have won the race
                        self._insert_loaded(adapter_id, *fast)
                    elif fast[3] is not None:
                        fast[3][0].release(fast[3][1])
                return
            config, state_dict = self._read_peft_dir(Path(entry.path))  # outside the lock: file I/O, parsing
            layers = self._layers_from_peft_state_dict(adapter_id, state_dict, names, float(config["lora_alpha"]),
                                                       entry.peft_adapter_name)
            adapter = CpuAdapter(adapter_id, config, layers)
            image = slab = None
            if image_dtype is not None and module_names is not None:
                slab = self._acquire_slab(_slot_image_bytes(adapter, module_names, image_dtype))
                image = _build_slot_image(adapter, module_names, image_dtype, slab)
            with self._lock:
                if adapter_id not in self.adapters:  # a synchronous load may have won the race
                    self.add_adapter(adapter_id, layers, config)
                    if image is not None:
                        key = (adapter_id, image_dtype, tuple(module_names))
                        self._images[key] = image
                        if slab is not None:
                            self._slabs[key] = slab
                elif slab is not None:
                    slab[0].release(slab[1])
        finally:
            with self._lock:
                self._loading.pop(adapter_id, None)

    def set_module_names(self, module_names: list[str]) -> None:
        self.module_names = list(module_names)

    def add_adapter(self, adapter_id: str, layers: dict[str, CpuLayerWeights], config: dict[str, Any] | None = None) -> None:
        if adapter_id == self.base_adapter_id:
            raise ValueError(f"{self.base_adapter_id!r} is reserved for base-only rows")
        if not layers:
            raise ValueError("Adapter must contain at least one target layer")
        with self._lock:
            self._drop_images(adapter_id)
            self.adapters[adapter_id] = CpuAdapter(adapter_id, config or {}, layers)
            self.adapters.move_to_end(adapter_id)
            self._evict_if_needed(exclude={adapter_id})

    def _evict_if_needed(self, exclude: set[str] | None = None) -> None:
        if self.max_adapters is None:
            return
        keep = (exclude or set()) | self.eviction_exclusions
        while len(self.adapters) > self.max_adapters:
            victim = next((a for a in self.adapters if a not in keep), None)
            if victim is None:
                raise RuntimeError("No evictable CPU LoRA adapter is available")
            self.adapters.pop(victim)
            self._drop_images(victim)

    # ------------------------------------------------------------------ PEFT parsing
    def add_adapter_from_peft_state_dict(
        self,
        adapter_id: str,
        state_dict: dict[str, torch.Tensor],
        module_names: list[str],
        lora_alpha: float,
        peft_adapter_name: str = "default",
        config: dict[str, Any] | None = None,
    ) -> None:
        layers = self._layers_from_peft_state_dict(adapter_id, state_dict, module_names, lora_alpha, peft_adapter_name)
        self.add_adapter(adapter_id, layers, config)

    def _layers_from_peft_state_dict(
        self,
        adapter_id: str,
        state_dict: dict[str, torch.Tensor],
        module_names: list[str],
        lora_alpha: float,
        peft_adapter_name: str = "default",
        index: dict[tuple[str, str], str] | None = None,
    ) -> dict[str, CpuLayerWeights]:
        """Per-module weights of a PEFT state dict (store.py:260-291); no state
        changes.  ``index``: the state dict's :func:`_lora_key_index`, if built."""
        self._validate_lora_keys_within_modules(adapter_id, state_dict, module_names)
        if index is None:
            index = _lora_key_index(state_dict, module_names, peft_adapter_name)
        layers: dict[str, CpuLayerWeights] = {}
        for module_name in module_names:
            key_a = index.get((module_name, "lora_A"))
            key_b = index.get((module_name, "lora_B"))
            if key_a is None and key_b is None:
                continue  # module absent: a rank-0 no-op for this adapter
            if key_a is None or key_b is None:
                raise ValueError(f"Adapter {adapter_id!r} has incomplete LoRA weights for {module_name!r}")
            lora_a = state_dict[key_a].detach().to("cpu").contiguous()  # (r, in)
            lora_b = state_dict[key_b].detach().to("cpu").contiguous()  # (out, r)
            rank = int(lora_a.shape[0])
            if rank <= 0:
                raise ValueError(f"Adapter {adapter_id!r} has non-positive rank for {module_name!r}")
            if int(lora_b.shape[1]) != rank:
                raise ValueError(f"LoRA A/B rank mismatch for adapter {adapter_id!r}, module {module_name!r}")
            # (in, r) and (r, out) as transposed views: the one copy is the packed slot
            # image (slot_image), the only thing sent to the GPU, which is pinned
            layers[module_name] = CpuLayerWeights(
                A=lora_a.t(),
                B=lora_b.t(),
                rank=rank,
                scale=float(lora_alpha) / rank,
            )
        return layers

    def add_adapter_from_peft_model(
        self,
        adapter_id: str,
        peft_model: torch.nn.Module,
        module_names: list[str],
        peft_adapter_name: str | None = None,
    ) -> None:
        # the PEFT model names its adapters; ours default to the same name
        name = peft_adapter_name or adapter_id
        configs = getattr(peft_model, "peft_config", {})
        if name not in configs or configs[name] is None:
            raise ValueError(f"PEFT model does not contain adapter {name!r}")
        peft_cfg = configs[name]
        self._validate_peft_config(peft_cfg)
        alpha = float(getattr(peft_cfg, "lora_alpha"))
        self.add_adapter_from_peft_state_dict(adapter_id, peft_model.state_dict(), module_names, alpha,
                                              peft_adapter_name=name, config=self._config_to_dict(peft_cfg))

    def load_adapter_from_disk(
        self,
        adapter_id: str,
        adapter_path: str | Path,
        module_names: list[str],
        peft_adapter_name: str = "default",
    ) -> None:
        with self._lock:
            if self.disk_cache is not None:
                adapter_path = self.disk_cache.add_adapter(adapter_id, adapter_path, peft_adapter_name)
            self._load_adapter_from_disk_path(adapter_id, adapter_path, module_names, peft_adapter_name)

    def _load_adapter_from_disk_cache(self, adapter_id: str) -> None:
        if self.disk_cache is None:
            raise KeyError(f"Unknown LoRA adapter id: {adapter_id}")
        if self.module_names is None:
            raise RuntimeError("module_names must be configured before loading adapters from disk cache")
        entry = self.disk_cache.get(adapter_id)
        fast = self._load_direct(adapter_id, Path(entry.path), list(self.module_names), entry.peft_adapter_name)
        if fast is not None:
            self._insert_loaded(adapter_id, *fast)
            return
        self._load_adapter_from_disk_path(adapter_id, entry.path, self.module_names, entry.peft_adapter_name)

    def _insert_loaded(self, adapter_id, config, layers, image, slab, key) -> None:
        with self._lock:
            self.add_adapter(adapter_id, layers, config)
            self._images[key] = image
            if slab is not None:
                self._slabs[key] = slab

    def _load_direct(self, adapter_id: str, path: Path, names: list[str], peft_adapter_name: str):
        """Loads an adapter by packing its safetensors file straight into its slot image.

        Applies when the GPU cache's image spec is set and matches ``names``:
        the native packer (``plora_peft_pack``, no interpreter lock) fills a
        pinned slab, and the per-module weights are views of that image.  Returns
        None when the packer declines the file (a tensor of another dtype,
        missing, malformed, of inconsistent rank or outside the modules); the
        caller then takes the general path, which raises the reference's errors."""
        spec = self._image_spec
        st_path = path / "adapter_model.safetensors"
        if spec is None or tuple(names) != spec[0] or not st_path.exists():
            return None
        dtype = spec[1]
        code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}.get(dtype)
        if code is None:
            return None
        config, _ = self._read_peft_dir_config(path)
        alpha = float(config["lora_alpha"])
        try:
            from . import _native

            lib = _native.load()
        except Exception:  # noqa: BLE001 - no library: the general path still works
            return None
        key_names = tuple(names)
        c_names = self._c_names.get(key_names)
        if c_names is None:
            c_names = self._c_names[key_names] = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        n = len(names)
        dims = (ctypes.c_int64 * (3 * n))()
        nbytes = ctypes.c_size_t(0)
        need = self._pack_bytes.get(key_names, 1 << 20)
        for _ in range(2):
            slab = self._acquire_slab(need)
            buf = slab[1] if slab is not None else torch.empty(need, dtype=torch.uint8)
            status = lib.plora_peft_pack(str(st_path).encode(), c_names, n, peft_adapter_name.encode(), code, alpha,
                                         buf.data_ptr(), buf.numel(), ctypes.byref(nbytes), dims)
            if status == 0:
                break
            if slab is not None:
                slab[0].release(slab[1])
            if status != 4:  # anything but "image too small": the general path decides
                return None
            need = int(nbytes.value)
        else:
            return None
        size = int(nbytes.value)
        with self._lock:
            self._pack_bytes[key_names] = max(size, self._pack_bytes.get(key_names, 0))
        image = buf[:size]
        typed = image.view(dtype)
        base = typed.storage_offset()
        esize = typed.element_size()
        recs = (SlotRecord * n).from_buffer_copy(image[: n * ctypes.sizeof(SlotRecord)].numpy().tobytes())
        layers: dict[str, CpuLayerWeights] = {}
        ranks: list[int] = []
        for i, name in enumerate(names):
            r, k_in, n_out = int(dims[3 * i]), int(dims[3 * i + 1]), int(dims[3 * i + 2])
            ranks.append(r)
            if r == 0:
                continue
            # (in, r) and (r, out): transposed views of the image's (r, in) and (out, r) blocks
            a = torch.as_strided(typed, (k_in, r), (1, k_in), base + recs[i].a_offset // esize)
            b = torch.as_strided(typed, (r, n_out), (1, r), base + recs[i].b_offset // esize)
            layers[name] = CpuLayerWeights(A=a, B=b, rank=r, scale=alpha / r)
        if not layers:  # the general path raises the reference's error for this
            if slab is not None:
                slab[0].release(slab[1])
            return None
        key = (adapter_id, dtype, key_names)
        return config, layers, (image, ranks), slab, key

    def _load_adapter_from_disk_path(
        self,
        adapter_id: str,
        adapter_path: str | Path,
        module_names: list[str],
        peft_adapter_name: str = "default",
    ) -> None:
        config, weights = self._read_peft_dir(Path(adapter_path))
        self.add_adapter_from_peft_state_dict(adapter_id, weights, module_names, float(config["lora_alpha"]),
                                              peft_adapter_name=peft_adapter_name, config=config)

    def _read_peft_dir(self, adapter_path: Path) -> tuple[dict[str, Any], dict[str, torch.Tensor]]:
        """Validated adapter_config.json and the weights of a PEFT directory."""
        config, _ = self._read_peft_dir_config(adapter_path)
        return config, self._load_peft_state_dict(adapter_path)

    def _read_peft_dir_config(self, adapter_path: Path) -> tuple[dict[str, Any], None]:
        config_path = adapter_path / "adapter_config.json"
        if not config_path.exists():
            raise FileNotFoundError(f"PEFT adapter config not found: {config_path}")
        config = json.loads(config_path.read_text(encoding="utf-8"))
        self._validate_peft_config_dict(config)
        return config, None

    _find_lora_key = staticmethod(_find_lora_key)
    _state_dict_lora_module_names = staticmethod(_state_dict_lora_module_names)
    _matches_module_name = staticmethod(_matches_module_name)

    @classmethod
    def _validate_lora_keys_within_modules(
        cls, adapter_id: str, state_dict: dict[str, torch.Tensor], module_names: list[str]
    ) -> None:
        outside = sorted(m for m in _state_dict_lora_module_names(state_dict) if not _matches_module_name(m, module_names))
        if outside:
            raise ValueError(
                f"Adapter {adapter_id!r} contains LoRA weights outside the configured module set: {outside}"
            )

    @staticmethod
    def _load_peft_state_dict(adapter_path: Path) -> dict[str, torch.Tensor]:
        """The adapter's weights: adapter_model.safetensors if present, else
        adapter_model.bin (the order PEFT's own loader prefers)."""
        for filename, load in _PEFT_WEIGHT_FILES:
            path = adapter_path / filename
            if path.exists():
                return load(path)
        raise FileNotFoundError(f"No PEFT adapter weights found in {adapter_path}")

    @staticmethod
    def _validate_peft_config(config: Any) -> None:
        """A PEFT LoraConfig object: the options the runtime cannot apply are refused."""
        for option in _SUPPORTED_OPTIONS:
            value = getattr(config, option, False)
            if value != False:  # noqa: E712  (the reference compares with != False)
                raise ValueError(f"Unsupported PEFT LoRA option: {option}={value!r}")
        if getattr(config, "lora_dropout", 0.0) not in (0, 0.0):
            raise ValueError("LoRA dropout is not supported by the inference runtime")

    @staticmethod
    def _validate_peft_config_dict(config: dict[str, Any]) -> None:
        """adapter_config.json: the first failing rule of _CONFIG_RULES raises."""
        for refused, message in _CONFIG_RULES:
            if refused(config):
                raise ValueError(message(config))

    @staticmethod
    def _config_to_dict(config: Any) -> dict[str, Any]:
        """A plain dict of a PEFT config object (to_dict() when it has one)."""
        to_dict = getattr(config, "to_dict", None)
        if to_dict is not None:
            return dict(to_dict())
        return dict(vars(config)) if hasattr(config, "__dict__") else {}

    # ------------------------------------------------------------------ GPU refill images
    def slot_image(self, adapter_id: str, module_names: list[str], dtype: torch.dtype) -> tuple[torch.Tensor, list]:
        """Packed pinned image of an adapter for ``plora_slot_fill``.

        Layout: one ``plora_slot_record`` per module in ``module_names`` order
        (absent modules have rank 0), then the A block (r, in) and the B block
        (out, r) in ``dtype`` -- the factors as PEFT stores them, so that an
        adapter loaded from PEFT needs no transposes on the host (the fill
        kernel transposes) -- each 256-byte aligned.  Returns the uint8 image
        and the per-module ranks.  Cached until the adapter leaves this tier.
        """
        key = (adapter_id, dtype, tuple(module_names))
        with self._lock:
            cached = self._images.get(key)
            if cached is None:
                adapter = self.adapters[adapter_id]
                slab = self._acquire_slab(_slot_image_bytes(adapter, module_names, dtype))
                cached = _build_slot_image(adapter, module_names, dtype, slab)
                self._images[key] = cached
                if slab is not None:
                    self._slabs[key] = slab
            return cached

    def note_image_use(self, adapter_id: str, module_names: list[str], dtype: torch.dtype, event: Any) -> None:
        """Records the event of a GPU copy that reads this image: its slab is not
        reused (after the adapter leaves the tier) before the event completes."""
        with self._lock:
            slab = self._slabs.get((adapter_id, dtype, tuple(module_names)))
            if slab is not None:
                slab[0].note_use(slab[1], event)

    def _acquire_slab(self, nbytes: int) -> tuple[PinnedSlabPool, torch.Tensor] | None:
        """A pinned slab of at least ``nbytes`` (None without a CUDA device)."""
        if not torch.cuda.is_available():
            return None
        size = _align(nbytes, 1 << 18)  # 256 KB size classes
        with self._lock:
            pool = self._pools.get(size)
            if pool is None:
                pool = self._pools[size] = PinnedSlabPool(size)
            return pool, pool.acquire()

    def _drop_images(self, adapter_id: str) -> None:
        for key in [k for k in self._images if k[0] == adapter_id]:
            del self._images[key]
            slab = self._slabs.pop(key, None)
            if slab is not None:
                slab[0].release(slab[1])


def _slot_image_bytes(adapter: CpuAdapter, module_names: list[str], dtype: torch.dtype) -> int:
    esize = torch.empty((), dtype=dtype).element_size()
    offset = _align(len(module_names) * _ctypes_sizeof(SlotRecord))
    for name in module_names:
        w = adapter.layers.get(name)
        if w is not None:
            offset = _align(offset + w.A.numel() * esize)
            offset = _align(offset + w.B.numel() * esize)
    return offset


def _build_slot_image(adapter: CpuAdapter, module_names: list[str], dtype: torch.dtype,
                      slab: tuple[PinnedSlabPool, torch.Tensor] | None = None) -> tuple[torch.Tensor, list]:
    """The packed image of :meth:`CpuAdapterStore.slot_image`, in ``slab`` (a
    pinned pool slab) when given; no state changes."""
    esize = torch.empty((), dtype=dtype).element_size()
    records = (SlotRecord * len(module_names))()
    blocks: list[tuple[int, torch.Tensor]] = []
    offset = _align(len(module_names) * _ctypes_sizeof(SlotRecord))
    ranks: list[int] = []
    for i, name in enumerate(module_names):
        w = adapter.layers.get(name)
        if w is None:
            ranks.append(0)
            continue
        a_t, b_t = w.A.t(), w.B.t()  # (r, in), (out, r): contiguous for PEFT-loaded adapters
        records[i].a_offset = offset
        blocks.append((offset, a_t))
        offset = _align(offset + a_t.numel() * esize)
        records[i].b_offset = offset
        blocks.append((offset, b_t))
        offset = _align(offset + b_t.numel() * esize)
        records[i].rank = int(w.rank)
        records[i].scale = float(w.scale)
        ranks.append(int(w.rank))
    if slab is not None:
        image = slab[1][:offset]
        image.zero_()
    else:
        image = torch.zeros(offset, dtype=torch.uint8)
    header = bytes(records)
    image[: len(header)] = torch.frombuffer(bytearray(header), dtype=torch.uint8)
    for off, t in blocks:  # one converting copy per block
        image[off : off + t.numel() * esize].view(dtype).view(t.shape).copy_(t)
    return image, ranks


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


def _ctypes_sizeof(t: type) -> int:
    import ctypes

    return ctypes.sizeof(t)
