"""CPU and disk adapter tiers and PEFT LoRA loading.

API-compatible with the reference's ``src/polylora/store.py``:

* :class:`DiskAdapterCache` — store.py:36-148.  Bounded copy of PEFT adapter
  directories with a ``manifest.json`` (same file name, JSON layout
  ``{"adapters": [{"adapter_id", "path", "peft_adapter_name"}]}`` written with
  ``indent=2, sort_keys=True``, same directory naming) so existing caches load.
* :class:`CpuAdapterStore` — store.py:160-436.  LRU of per-module
  ``(A^T, B^T, rank, alpha/rank)`` in pinned memory, PEFT validation with the
  same exception types and messages, eviction that skips GPU-resident
  adapters.

Added for the GPU tier: :meth:`CpuAdapterStore.slot_image` packs every module
of an adapter into one pinned buffer laid out for ``plora_slot_fill`` so a
GPU slot refill is a single host-to-device copy plus one scatter kernel.
"""

from __future__ import annotations

import json
import shutil
from collections import OrderedDict
from dataclasses import dataclass
from hashlib import sha256
from pathlib import Path
from typing import Any

import torch

from ._native import SlotRecord

_SUPPORTED_OPTIONS = ("use_dora", "lora_bias", "use_rslora")


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
        if max_adapters is not None and max_adapters < 1:
            raise ValueError("max_adapters must be at least 1")
        self.cache_dir = Path(cache_dir)
        self.max_adapters = max_adapters
        self.cache_dir.mkdir(parents=True, exist_ok=True)
        self.entries: OrderedDict[str, DiskAdapterEntry] = OrderedDict()
        self._json_blocks: dict[str, str] = {}  # adapter_id -> its manifest entry, serialised
        self._load_manifest()
        self._evict_if_needed()

    def __contains__(self, adapter_id: str) -> bool:
        return adapter_id in self.entries

    @property
    def manifest_path(self) -> Path:
        return self.cache_dir / self._MANIFEST_NAME

    def get(self, adapter_id: str) -> DiskAdapterEntry:
        if adapter_id not in self.entries:
            raise KeyError(f"Unknown disk LoRA adapter id: {adapter_id}")
        self.touch(adapter_id)
        return self.entries[adapter_id]

    def touch(self, adapter_id: str) -> None:
        if adapter_id in self.entries:
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


class CpuAdapterStore:
    """LRU of adapters in host memory, refilled from the disk tier on a miss."""

    def __init__(
        self,
        base_adapter_id: str = "__base__",
        max_adapters: int | None = None,
        disk_cache: DiskAdapterCache | None = None,
        module_names: list[str] | None = None,
    ) -> None:
        if max_adapters is not None and max_adapters < 1:
            raise ValueError("max_adapters must be at least 1")
        self.base_adapter_id = base_adapter_id
        self.max_adapters = max_adapters
        self.disk_cache = disk_cache
        self.module_names = module_names
        self.adapters: OrderedDict[str, CpuAdapter] = OrderedDict()
        self.eviction_exclusions: set[str] = set()
        self._images: dict[tuple, tuple[torch.Tensor, list]] = {}

    # ------------------------------------------------------------------ LRU
    def __contains__(self, adapter_id: str) -> bool:
        if adapter_id == self.base_adapter_id or adapter_id in self.adapters:
            return True
        return self.disk_cache is not None and adapter_id in self.disk_cache

    def get(self, adapter_id: str) -> CpuAdapter:
        if adapter_id == self.base_adapter_id:
            raise KeyError(f"Base adapter {adapter_id!r} has no LoRA weights")
        if adapter_id not in self.adapters:
            if self.disk_cache is None or adapter_id not in self.disk_cache:
                raise KeyError(f"Unknown LoRA adapter id: {adapter_id}")
            self._load_adapter_from_disk_cache(adapter_id)
        self.touch(adapter_id)
        return self.adapters[adapter_id]

    def touch(self, adapter_id: str) -> None:
        if adapter_id in self.adapters:
            self.adapters.move_to_end(adapter_id)

    def set_eviction_exclusions(self, adapter_ids: set[str]) -> None:
        self.eviction_exclusions = {a for a in adapter_ids if a != self.base_adapter_id}

    def set_module_names(self, module_names: list[str]) -> None:
        self.module_names = list(module_names)

    def add_adapter(self, adapter_id: str, layers: dict[str, CpuLayerWeights], config: dict[str, Any] | None = None) -> None:
        if adapter_id == self.base_adapter_id:
            raise ValueError(f"{self.base_adapter_id!r} is reserved for base-only rows")
        if not layers:
            raise ValueError("Adapter must contain at least one target layer")
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
        self._validate_lora_keys_within_modules(adapter_id, state_dict, module_names)
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
        self.add_adapter(adapter_id, layers, config)

    def add_adapter_from_peft_model(
        self,
        adapter_id: str,
        peft_model: torch.nn.Module,
        module_names: list[str],
        peft_adapter_name: str | None = None,
    ) -> None:
        name = peft_adapter_name or adapter_id
        adapter_config = getattr(peft_model, "peft_config", {}).get(name)
        if adapter_config is None:
            raise ValueError(f"PEFT model does not contain adapter {name!r}")
        self._validate_peft_config(adapter_config)
        self.add_adapter_from_peft_state_dict(
            adapter_id=adapter_id,
            state_dict=peft_model.state_dict(),
            module_names=module_names,
            lora_alpha=float(getattr(adapter_config, "lora_alpha")),
            peft_adapter_name=name,
            config=self._config_to_dict(adapter_config),
        )

    def load_adapter_from_disk(
        self,
        adapter_id: str,
        adapter_path: str | Path,
        module_names: list[str],
        peft_adapter_name: str = "default",
    ) -> None:
        if self.disk_cache is not None:
            adapter_path = self.disk_cache.add_adapter(adapter_id, adapter_path, peft_adapter_name)
        self._load_adapter_from_disk_path(adapter_id, adapter_path, module_names, peft_adapter_name)

    def _load_adapter_from_disk_cache(self, adapter_id: str) -> None:
        if self.disk_cache is None:
            raise KeyError(f"Unknown LoRA adapter id: {adapter_id}")
        if self.module_names is None:
            raise RuntimeError("module_names must be configured before loading adapters from disk cache")
        entry = self.disk_cache.get(adapter_id)
        self._load_adapter_from_disk_path(adapter_id, entry.path, self.module_names, entry.peft_adapter_name)

    def _load_adapter_from_disk_path(
        self,
        adapter_id: str,
        adapter_path: str | Path,
        module_names: list[str],
        peft_adapter_name: str = "default",
    ) -> None:
        adapter_path = Path(adapter_path)
        config_path = adapter_path / "adapter_config.json"
        if not config_path.exists():
            raise FileNotFoundError(f"PEFT adapter config not found: {config_path}")
        config = json.loads(config_path.read_text(encoding="utf-8"))
        self._validate_peft_config_dict(config)
        self.add_adapter_from_peft_state_dict(
            adapter_id=adapter_id,
            state_dict=self._load_peft_state_dict(adapter_path),
            module_names=module_names,
            lora_alpha=float(config["lora_alpha"]),
            peft_adapter_name=peft_adapter_name,
            config=config,
        )

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
        st_path = adapter_path / "adapter_model.safetensors"
        bin_path = adapter_path / "adapter_model.bin"
        if st_path.exists():
            try:
                from safetensors.torch import load_file
            except ImportError as exc:
                raise ImportError("safetensors is required to load adapter_model.safetensors") from exc
            return load_file(str(st_path), device="cpu")
        if bin_path.exists():
            return torch.load(bin_path, map_location="cpu")
        raise FileNotFoundError(f"No PEFT adapter weights found in {adapter_path}")

    @staticmethod
    def _validate_peft_config(config: Any) -> None:
        for name in _SUPPORTED_OPTIONS:
            if hasattr(config, name) and getattr(config, name) != False:  # noqa: E712
                raise ValueError(f"Unsupported PEFT LoRA option: {name}={getattr(config, name)!r}")
        if getattr(config, "lora_dropout", 0.0) not in (0, 0.0):
            raise ValueError("LoRA dropout is not supported by the inference runtime")

    @staticmethod
    def _validate_peft_config_dict(config: dict[str, Any]) -> None:
        if config.get("peft_type") not in (None, "LORA"):
            raise ValueError(f"Unsupported PEFT adapter type: {config.get('peft_type')!r}")
        for key, label in (("use_dora", "DoRA adapters"), ("use_rslora", "RS-LoRA adapters"), ("lora_bias", "LoRA bias")):
            if config.get(key, False):
                raise ValueError(f"{label} {'is' if key == 'lora_bias' else 'are'} not supported")
        if float(config.get("lora_dropout", 0.0)) != 0.0:
            raise ValueError("LoRA dropout is not supported by the inference runtime")
        if "lora_alpha" not in config:
            raise ValueError("adapter_config.json is missing lora_alpha")

    @staticmethod
    def _config_to_dict(config: Any) -> dict[str, Any]:
        if hasattr(config, "to_dict"):
            return dict(config.to_dict())
        if hasattr(config, "__dict__"):
            return dict(config.__dict__)
        return {}

    # ------------------------------------------------------------------ GPU refill images
    def slot_image(self, adapter_id: str, module_names: list[str], dtype: torch.dtype) -> tuple[torch.Tensor, list]:
        """Packed pinned image of an adapter for ``plora_slot_fill``.

        Layout: one ``plora_slot_record`` per module in ``module_names`` order
        (absent modules have rank 0), then the A block (r, in) and the B block
        (out, r) in ``dtype`` -- the factors as PEFT stores them, so that an
        adapter loaded from PEFT needs no transposes on the host (the fill
        kernel transposes) -- each 256-byte aligned.  Returns the uint8 image and the
        per-module ranks.  Cached until the adapter leaves this tier.
        """
        key = (adapter_id, dtype, tuple(module_names))
        cached = self._images.get(key)
        if cached is not None:
            return cached
        adapter = self.adapters[adapter_id]
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
        # page-locked from the start when a CUDA device exists (torch's pinned block cache)
        image = torch.zeros(offset, dtype=torch.uint8, pin_memory=torch.cuda.is_available())
        header = bytes(records)
        image[: len(header)] = torch.frombuffer(bytearray(header), dtype=torch.uint8)
        for off, t in blocks:  # one converting copy per block
            image[off : off + t.numel() * esize].view(dtype).view(t.shape).copy_(t)
        self._images[key] = (image, ranks)
        return image, ranks

    def _drop_images(self, adapter_id: str) -> None:
        for key in [k for k in self._images if k[0] == adapter_id]:
            del self._images[key]


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


def _ctypes_sizeof(t: type) -> int:
    import ctypes

    return ctypes.sizeof(t)
