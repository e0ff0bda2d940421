"""``PolyLoraModel``: wraps a model and routes each batch row to its adapter.

Same constructor, methods, target matching and shape inference as the
reference's src/polylora/model.py:15-166.  ``forward(..., adapter_ids=...)``
makes the batch's adapters resident (refills overlap on a side stream),
derives ``seq_lens`` from the attention mask, and runs the base model with
the batch context installed; every wrapped Linear then adds its LoRA delta
with the native kernels.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import nn

from .cache import GpuAdapterCache, ModuleSpec
from .config import PolyLoraConfig
from .context import LoraBatchContext, assert_right_padded, use_lora_context
from .layers import MultiLoraLinear
from .store import CpuAdapterStore, DiskAdapterCache


class PolyLoraModel(nn.Module):
    def __init__(self, base_model: nn.Module, config: PolyLoraConfig, adapter_store: CpuAdapterStore | None = None) -> None:
        super().__init__()
        self.base_model = base_model
        self.config = config
        self.module_specs = self._collect_module_specs(base_model, config.target_modules)
        if not self.module_specs:
            raise ValueError("No nn.Linear modules matched the PolyLoRA module selection")
        disk_cache = (
            DiskAdapterCache(config.disk_cache_dir, config.max_disk_adapters)
            if config.disk_cache_dir is not None
            else None
        )
        self.adapter_store = adapter_store or CpuAdapterStore(
            config.base_adapter_id,
            config.max_cpu_adapters,
            disk_cache=disk_cache,
            module_names=self.target_module_names,
            prefetch_workers=config.prefetch_workers,
        )
        self.adapter_store.set_module_names(self.target_module_names)
        device, dtype = self._infer_device_dtype(base_model)
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

    def add_adapter_from_peft_model(self, adapter_id: str, peft_model: nn.Module, peft_adapter_name: str | None = None) -> None:
        self.adapter_store.add_adapter_from_peft_model(
            adapter_id=adapter_id,
            peft_model=peft_model,
            module_names=self.target_module_names,
            peft_adapter_name=peft_adapter_name,
        )

    def load_adapter_from_disk(self, adapter_id: str, adapter_path: str, peft_adapter_name: str = "default") -> None:
        self.adapter_store.load_adapter_from_disk(
            adapter_id=adapter_id,
            adapter_path=adapter_path,
            module_names=self.target_module_names,
            peft_adapter_name=peft_adapter_name,
        )

    def forward(self, *args: Any, adapter_ids: list[str] | None = None, **kwargs: Any) -> Any:
        if adapter_ids is None:
            return self.base_model(*args, **kwargs)
        batch_size, seq_len, device, _ = self._infer_forward_shape(*args, **kwargs)
        _, dtype = self._infer_device_dtype(self.base_model)
        self.adapter_cache.to(device, dtype)
        ctx = self.prepare_lora_context(adapter_ids, kwargs.get("attention_mask"), batch_size, seq_len, device)
        with use_lora_context(ctx):
            out = self.base_model(*args, **kwargs)
        slots = {self.adapter_cache.adapter_to_slot[a] for a in set(adapter_ids) if a != self.config.base_adapter_id}
        self.adapter_cache.mark_slots_used(slots)
        return out

    def prepare_lora_context(
        self,
        adapter_ids: list[str],
        attention_mask: torch.Tensor | None,
        batch_size: int,
        seq_len: int,
        device: torch.device,
    ) -> LoraBatchContext:
        if len(adapter_ids) != batch_size:
            raise ValueError("adapter_ids length must match batch size")
        weight_indices = self.adapter_cache.ensure_resident(adapter_ids)
        if attention_mask is None:
            seq_lens = torch.full((batch_size,), seq_len, dtype=torch.int32, device=device)
        else:
            seq_lens = attention_mask.to(device=device, dtype=torch.int32).sum(dim=-1)
            if self.config.enforce_right_padding:
                assert_right_padded(attention_mask.to(device), seq_lens)
        return LoraBatchContext(
            adapter_ids=list(adapter_ids),
            weight_indices=weight_indices,
            seq_lens=seq_lens,
            attention_mask=attention_mask,
            table_ranks=self.adapter_cache.table_ranks,
            ready_event=self.adapter_cache.ready_event,
        )

    @staticmethod
    def _matches_target(name: str, target_modules: list[str]) -> bool:
        return any(name == t or name.endswith(f".{t}") for t in target_modules)

    @classmethod
    def _collect_module_specs(cls, model: nn.Module, target_modules: list[str] | None) -> list[ModuleSpec]:
        return [
            ModuleSpec(name, module.in_features, module.out_features)
            for name, module in model.named_modules()
            if isinstance(module, nn.Linear) and (target_modules is None or cls._matches_target(name, target_modules))
        ]

    def _replace_target_modules(self, model: nn.Module) -> None:
        for module_name in self.target_module_names:
            parent, child_name = self._get_parent(model, module_name)
            child = getattr(parent, child_name)
            if not isinstance(child, nn.Linear):
                raise TypeError(f"Expected nn.Linear at {module_name!r}, found {type(child).__name__}")
            setattr(parent, child_name, MultiLoraLinear(child, module_name, self.adapter_cache))

    @staticmethod
    def _get_parent(model: nn.Module, module_name: str) -> tuple[nn.Module, str]:
        *path, leaf = module_name.split(".")
        parent = model
        for part in path:
            parent = getattr(parent, part)
        return parent, leaf

    @staticmethod
    def _infer_device_dtype(model: nn.Module) -> tuple[torch.device, torch.dtype]:
        for param in model.parameters():
            return param.device, param.dtype
        return torch.device("cpu"), torch.float32

    @staticmethod
    def _infer_forward_shape(*args: Any, **kwargs: Any) -> tuple[int, int, torch.device, torch.dtype]:
        tensor = kwargs.get("input_ids")
        if tensor is None:
            tensor = kwargs.get("inputs_embeds")
        if tensor is None:
            tensor = next((a for a in args if torch.is_tensor(a)), None)
        if tensor is None:
            raise ValueError("Cannot infer batch size without input_ids, inputs_embeds, or a tensor positional arg")
        if tensor.dim() < 2:
            raise ValueError("Input tensor must have batch and sequence dimensions")
        dtype = tensor.dtype if tensor.is_floating_point() else torch.float32
        return int(tensor.shape[0]), int(tensor.shape[1]), tensor.device, dtype


CustomPeftModel = PolyLoraModel
