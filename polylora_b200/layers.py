"""The wrapped ``nn.Linear``: base GEMM, then fused LoRA shrink/expand.

Mirrors ``MultiLoraLinear`` of src/polylora/layers.py:18-134: same
constructor, the same three accepted input layouts (``_prepare_batched_inputs``,
layers.py:82-110) and in-place add-back into the base output.  The LoRA part
runs only on the native sm_100a kernels; the slot-grouped segment table is
built once per forward (per layout) and shared by every wrapped layer.
"""

from __future__ import annotations

import torch
from torch import nn

from .cache import GpuAdapterCache
from .context import LoraBatchContext, get_lora_context
from .sgmv import SegmentTable, build_segments, sgmv_shrink_expand


class MultiLoraLinear(nn.Module):
    def __init__(self, base_layer: nn.Linear, module_name: str, cache: GpuAdapterCache) -> None:
        super().__init__()
        self.base_layer = base_layer
        self.module_name = module_name
        self.cache = cache

    @property
    def in_features(self) -> int:
        return self.base_layer.in_features

    @property
    def out_features(self) -> int:
        return self.base_layer.out_features

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        base = self.base_layer(x)
        ctx = get_lora_context()
        if ctx is None:
            return base
        original_shape = base.shape
        x_3d, base_3d, seq_lens, weight_indices, key = self._prepare_batched_inputs(x, base, ctx)
        self._check_native(x_3d)
        table = self._segment_table(ctx, key, weight_indices, seq_lens, x_3d.shape[1])
        self.cache.wait_ready()
        name = self.module_name
        ranks = self.cache.ranks[name]
        # layers.py:42-58 of the reference: shrink then expand, issued as one call
        out = sgmv_shrink_expand(
            x_3d, self.cache.A[name], self.cache.B[name], base_3d, table, ranks, self.cache.scales[name]
        )
        return out.reshape(original_shape)

    def _check_native(self, x: torch.Tensor) -> None:
        if not self.cache.config.use_triton_kernels:
            raise RuntimeError(
                "use_triton_kernels=False selects the reference's PyTorch path, which polylora_b200 "
                "does not ship; the LoRA kernels here are the native sm_100a ones"
            )
        if not x.is_cuda:
            raise RuntimeError(
                f"polylora_b200 runs the LoRA path on CUDA only; module {self.module_name!r} got {x.device}"
            )

    @staticmethod
    def _as_3d(x: torch.Tensor) -> torch.Tensor:
        if x.dim() == 2:
            return x.unsqueeze(1)
        if x.dim() == 3:
            return x
        if x.dim() > 3:
            return x.reshape(x.shape[0], -1, x.shape[-1])
        raise ValueError("MultiLoraLinear expects a batched tensor")

    def _prepare_batched_inputs(self, x: torch.Tensor, base: torch.Tensor, ctx: LoraBatchContext):
        rows = ctx.weight_indices.shape[0]
        if x.shape[0] == rows:  # (B, ..., K): one batch row per leading index
            x_3d = self._as_3d(x).contiguous()
            return x_3d, self._as_3d(base).contiguous(), ctx.seq_lens, ctx.weight_indices, ("rows", x_3d.shape[1])
        if x.dim() == 3 and x.shape[0] == 1:  # (1, M, K): the reference uses row 0 only
            return x.contiguous(), base.contiguous(), ctx.seq_lens[:1], ctx.weight_indices[:1], ("row0", x.shape[1])
        if x.dim() == 2 and x.shape[0] % rows == 0:  # (B*S, K) flattened tokens
            seq = x.shape[0] // rows
            return (
                x.reshape(rows, seq, x.shape[-1]).contiguous(),
                base.reshape(rows, seq, base.shape[-1]).contiguous(),
                ctx.seq_lens,  # clamped to `seq` by the segment builder
                ctx.weight_indices,
                ("rows", seq),
            )
        raise ValueError("LoRA batch context batch size does not match layer input batch size")

    def _segment_table(self, ctx: LoraBatchContext, key, weight_indices, seq_lens, max_seq: int) -> SegmentTable:
        table = ctx.segments.get(key)
        if table is None:
            ranks = ctx.table_ranks if ctx.table_ranks is not None else self.cache.table_ranks
            self.cache.wait_ready()
            table = build_segments(weight_indices, seq_lens, ranks, max_seq)
            ctx.segments[key] = table
        return table
