"""``PolyLoraModel``: wraps a model and routes each batch row to its adapter.

The public surface is the reference's (src/polylora/model.py:15-166): the
constructor, ``target_module_names``, ``add_adapter_from_peft_model``,
``load_adapter_from_disk``, ``forward(..., adapter_ids=...)``,
``prepare_lora_context`` and the ``CustomPeftModel`` alias, with the same
target-matching rule, shape-inference order and error messages.

``forward(..., adapter_ids=...)`` makes the batch's adapters resident (refills
overlap on a side stream), derives ``seq_lens`` from the attention mask, and
runs the base model with the batch context installed; every wrapped Linear
then adds its LoRA delta with the native kernels.
"""

from __future__ import annotations

from typing import Any, Iterator

import torch
from torch import nn

from .cache import GpuAdapterCache, ModuleSpec
from .config import PolyLoraConfig
from . import _native
from .context import RIGHT_PADDING_ERROR, LoraBatchContext, assert_right_padded, use_lora_context
from .layers import MultiLoraLinear
from .store import CpuAdapterStore, DiskAdapterCache

_NO_TARGETS = "No nn.Linear modules matched the PolyLoRA module selection"
_NO_BATCH_TENSOR = "Cannot infer batch size without input_ids, inputs_embeds, or a tensor positional arg"
_NOT_BATCHED = "Input tensor must have batch and sequence dimensions"


def _is_target(name: str, targets: list[str] | None) -> bool:
    """A module is targeted when its dotted name is a target or ends in
    ``.<target>`` (targets may themselves be dotted); None targets every Linear."""
    if targets is None:
        return True
    dotted = "." + name
    return any(dotted.endswith("." + t) for t in targets)


def _linear_targets(model: nn.Module, targets: list[str] | None) -> Iterator[tuple[str, nn.Linear]]:
    for name, module in model.named_modules():
        if isinstance(module, nn.Linear) and _is_target(name, targets):
            yield name, module


def _parent_and_attr(model: nn.Module, dotted: str) -> tuple[nn.Module, str]:
    prefix, _, attr = dotted.rpartition(".")
    return (model.get_submodule(prefix) if prefix else model), attr


def _param_device_dtype(model: nn.Module) -> tuple[torch.device, torch.dtype]:
    first = next(model.parameters(), None)
    if first is None:
        return torch.device("cpu"), torch.float32
    return first.device, first.dtype


def _batch_tensor(args: tuple, kwargs: dict) -> torch.Tensor:
    """input_ids, else inputs_embeds, else the first tensor positional argument."""
    for key in ("input_ids", "inputs_embeds"):
        if kwargs.get(key) is not None:
            return kwargs[key]
    for arg in args:
        if torch.is_tensor(arg):
            return arg
    raise ValueError(_NO_BATCH_TENSOR)


class PolyLoraModel(nn.Module):
    def __init__(self, base_model: nn.Module, config: PolyLoraConfig,
                 adapter_store: CpuAdapterStore | None = None) -> None:
        super().__init__()
        self.base_model = base_model
        self.config = config
        self.module_specs = self._collect_module_specs(base_model, config.target_modules)
        if not self.module_specs:
            raise ValueError(_NO_TARGETS)
        names = self.target_module_names
        if adapter_store is None:
            disk = None
            if config.disk_cache_dir is not None:
                disk = DiskAdapterCache(config.disk_cache_dir, config.max_disk_adapters)
            adapter_store = CpuAdapterStore(config.base_adapter_id, config.max_cpu_adapters, disk_cache=disk,
                                            module_names=names, prefetch_workers=config.prefetch_workers)
        self.adapter_store = adapter_store
        self.adapter_store.set_module_names(names)
        device, dtype = _param_device_dtype(base_model)
        self.adapter_cache = GpuAdapterCache(self.adapter_store, self.module_specs, config, device, dtype)
        self._replace_target_modules(self.base_model)

    @property
    def target_module_names(self) -> list[str]:
        return [spec.name for spec in self.module_specs]

    def prefetch(self, adapter_ids: list[str]):
        """Starts loading, on worker threads, the adapters of a queued batch that
        are only on the disk tier, with their slot images in this model's cache
        dtype, so that the batch's forward finds them in the CPU tier.  Returns
        the futures of the loads started.  No counterpart in the reference."""
        cache = self.adapter_cache
        return self.adapter_store.prefetch(adapter_ids, image_dtype=cache.dtype, module_names=cache.module_names)

    # adapter registration: the store parses and validates; the model supplies its module names
    def add_adapter_from_peft_model(self, adapter_id: str, peft_model: nn.Module,
                                    peft_adapter_name: str | None = None) -> None:
        self.adapter_store.add_adapter_from_peft_model(adapter_id=adapter_id, peft_model=peft_model,
                                                       module_names=self.target_module_names,
                                                       peft_adapter_name=peft_adapter_name)

    def load_adapter_from_disk(self, adapter_id: str, adapter_path: str,
                               peft_adapter_name: str = "default") -> None:
        self.adapter_store.load_adapter_from_disk(adapter_id=adapter_id, adapter_path=adapter_path,
                                                  module_names=self.target_module_names,
                                                  peft_adapter_name=peft_adapter_name)

    def forward(self, *args: Any, adapter_ids: list[str] | None = None, **kwargs: Any) -> Any:
        if adapter_ids is None:
            return self.base_model(*args, **kwargs)
        batch_size, seq_len, device, _ = self._infer_forward_shape(*args, **kwargs)
        self.adapter_cache.to(device, _param_device_dtype(self.base_model)[1])
        ctx = self.prepare_lora_context(adapter_ids, kwargs.get("attention_mask"), batch_size, seq_len, device)
        with use_lora_context(ctx):
            out = self.base_model(*args, **kwargs)
        # the slots this batch read may be refilled only after the work enqueued so far
        cache = self.adapter_cache
        cache.mark_slots_used({cache.adapter_to_slot[a] for a in set(adapter_ids) if a != self.config.base_adapter_id})
        return out

    def prepare_lora_context(self, adapter_ids: list[str], attention_mask: torch.Tensor | None, batch_size: int,
                             seq_len: int, device: torch.device) -> LoraBatchContext:
        if len(adapter_ids) != batch_size:
            raise ValueError("adapter_ids length must match batch size")
        weight_indices = self.adapter_cache.ensure_resident(adapter_ids)
        if attention_mask is not None:
            mask = attention_mask.to(device)
            seq_lens = mask.to(torch.int32).sum(dim=-1)  # int64, as torch sums integers
            if self.config.enforce_right_padding:
                if self.config.right_padding_check == "device" and mask.is_cuda:
                    if mask.dim() != 2:
                        raise ValueError("attention_mask must be a 2D batch mask")
                    _native.check_right_padded(mask, seq_lens)  # no wait; see raise_for_device_status
                else:
                    assert_right_padded(mask, seq_lens)
        else:
            seq_lens = torch.full((batch_size,), seq_len, dtype=torch.int32, device=device)
        return LoraBatchContext(adapter_ids=list(adapter_ids), weight_indices=weight_indices, seq_lens=seq_lens,
                                attention_mask=attention_mask, table_ranks=self.adapter_cache.table_ranks,
                                ready_event=self.adapter_cache.ready_event)

    def raise_for_device_status(self) -> None:
        """Waits for the device and raises for what the library's kernels
        recorded since the last read: the reference's right-padding ValueError
        for a mask checked on the device (``right_padding_check="device"``),
        a ``PloraError`` for any other status bit.  Reading clears the word.
        No counterpart in the reference, whose check raises in the forward."""
        status = _native.device_status(clear=True)
        if status & _native.DEV_PADDING:
            raise ValueError(RIGHT_PADDING_ERROR)
        if status:
            raise _native.PloraError("device status", _native.ERR_DEVICE, f"status word 0x{status:x}")

    # ------------------------------------------------------------------ module surgery
    @staticmethod
    def _matches_target(name: str, target_modules: list[str]) -> bool:
        return _is_target(name, target_modules)

    @classmethod
    def _collect_module_specs(cls, model: nn.Module, target_modules: list[str] | None) -> list[ModuleSpec]:
        return [ModuleSpec(name, lin.in_features, lin.out_features) for name, lin in _linear_targets(model, target_modules)]

    def _replace_target_modules(self, model: nn.Module) -> None:
        for name in self.target_module_names:
            parent, attr = _parent_and_attr(model, name)
            linear = getattr(parent, attr)
            if not isinstance(linear, nn.Linear):
                raise TypeError(f"Expected nn.Linear at {name!r}, found {type(linear).__name__}")
            setattr(parent, attr, MultiLoraLinear(linear, name, self.adapter_cache))

    @staticmethod
    def _get_parent(model: nn.Module, module_name: str) -> tuple[nn.Module, str]:
        return _parent_and_attr(model, module_name)

    @staticmethod
    def _infer_device_dtype(model: nn.Module) -> tuple[torch.device, torch.dtype]:
        return _param_device_dtype(model)

    @staticmethod
    def _infer_forward_shape(*args: Any, **kwargs: Any) -> tuple[int, int, torch.device, torch.dtype]:
        tensor = _batch_tensor(args, kwargs)
        if tensor.dim() < 2:
            raise ValueError(_NOT_BATCHED)
        batch_size, seq_len = (int(d) for d in tensor.shape[:2])
        return batch_size, seq_len, tensor.device, (tensor.dtype if tensor.is_floating_point() else torch.float32)


CustomPeftModel = PolyLoraModel
