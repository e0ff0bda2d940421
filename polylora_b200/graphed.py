"""One ``PolyLoraModel`` forward of fixed shapes replayed as a CUDA graph.

A forward of the wrapped model is a host part, the slot policy
(``ensure_resident``: which adapter sits in which GPU slot, refills on a side
stream), and a device part: the segment table, the base model and, in every
wrapped Linear, the shrink and expand kernels, none of which needs the host.
At decode sizes the device part is a few microseconds of GPU work per layer
but a Python layer and a C call each, so the forward is bound by launches.
``GraphedForward`` captures the device part once and, per call, runs the host
part, copies the batch's slot indices into the captured input buffers and
replays the graph.  Adapter assignments may change between calls (refills
included); the shapes, the input tensors' shapes and the model may not.

The reference has no counterpart (its forward syncs with the host in every
layer, src/polylora/sgmv.py:51,59).

Attention masks under capture: transformers' mask helpers treat CUDA stream
capture like tracing and then build an explicit causal mask even for an
unpadded batch whose causal mask eager mode skips (one query token, or as
many queries as keys).  SDPA cannot use its flash kernel with an explicit
mask, so a captured Llama-shaped decode step ran the memory-efficient kernel
at ~230 us per layer instead of ~40.  A graph is replayed only with the
shapes it was captured with, so the eager decision holds for it when the
positions are the model's own; captures given neither ``attention_mask`` nor
``position_ids`` therefore take it (``eager_mask_decisions``).
"""

from __future__ import annotations

import contextlib
from typing import Any

import torch

from .context import LoraBatchContext, use_lora_context


@contextlib.contextmanager
def eager_mask_decisions():
    """Within the block, while a CUDA stream captures, transformers' mask
    helpers decide as in eager mode for a batch given neither a padding mask
    nor position ids: the positions are the model's own aranges (no packed
    sequences), and the causal mask is skipped for one query token or as many
    queries as keys, so that SDPA applies ``is_causal`` itself.  Eager mode
    reaches the same decisions by reading tensor values, which a capture cannot
    do.  Outside a capture, under other tracing, with a padding mask, or on
    XPU devices the helpers run unchanged.  The two helpers are replaced in
    transformers' module for the duration of the block, so a capture on
    another thread at the same time gets the same decisions.  A no-op without
    transformers or when its helpers have other names."""
    try:
        from transformers import masking_utils
        from transformers.utils import import_utils
    except ImportError:
        yield
        return
    packed = getattr(masking_utils, "find_packed_sequence_indices", None)
    skip = getattr(masking_utils, "_ignore_causal_mask_sdpa", None)
    compiling = getattr(import_utils, "is_torchdynamo_compiling", None)
    jit_tracing = getattr(import_utils, "is_jit_tracing", None)
    capturing = getattr(import_utils, "is_cuda_stream_capturing", None)  # False where CUDA is absent
    if None in (packed, skip, compiling, jit_tracing, capturing) or getattr(masking_utils, "_is_torch_xpu_available",
                                                                           True):
        yield
        return

    def capturing_only() -> bool:
        return capturing() and not compiling() and not jit_tracing()

    def packed_eager(position_ids):
        return None if capturing_only() else packed(position_ids)

    def skip_eager(padding_mask, query_length, kv_length, kv_offset, local_attention_size=None):
        if padding_mask is None and capturing_only():
            return (query_length == 1 or kv_length == query_length) and (
                local_attention_size is None or kv_length < local_attention_size)
        return skip(padding_mask, query_length, kv_length, kv_offset, local_attention_size)

    masking_utils.find_packed_sequence_indices = packed_eager
    masking_utils._ignore_causal_mask_sdpa = skip_eager
    try:
        yield
    finally:
        masking_utils.find_packed_sequence_indices = packed
        masking_utils._ignore_causal_mask_sdpa = skip


class GraphedForward:
    """Captures ``model.base_model(**inputs)`` under a LoRA batch context.

    ``inputs`` are example keyword tensors (on the model's GPU) whose shapes
    every call must keep; ``output`` picks the tensor to return from the base
    model's output (default: ``last_hidden_state`` when present).  Pass no
    ``attention_mask`` for unpadded batches: mask helpers of some models sync
    with the host, which a capture cannot contain.  Given neither a mask nor
    position ids, the capture takes the eager mode's attention-mask decisions
    (``eager_mask_decisions``).
    """

    def __init__(self, model: Any, adapter_ids: list[str], warmup: int = 2, output=None, **inputs: torch.Tensor):
        self.model = model
        self.static = {k: v.clone() for k, v in inputs.items()}
        self.output = output or (lambda out: getattr(out, "last_hidden_state", out))
        batch, seq, device, _ = model._infer_forward_shape(**self.static)
        self.batch, self.seq, self.device = batch, seq, device
        _, dtype = model._infer_device_dtype(model.base_model)
        model.adapter_cache.to(device, dtype)
        ctx = self._host_part(adapter_ids)
        self.weight_indices = ctx.weight_indices.clone()
        self.seq_lens = ctx.seq_lens.clone()
        torch.cuda.synchronize(device)  # refills of the example batch are done

        def device_part():
            gctx = LoraBatchContext(
                adapter_ids=list(adapter_ids), weight_indices=self.weight_indices, seq_lens=self.seq_lens,
                attention_mask=self.static.get("attention_mask"), table_ranks=ctx.table_ranks, ready_event=None,
            )
            with use_lora_context(gctx):
                return self.output(model.base_model(**self.static))

        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.inference_mode(), torch.cuda.stream(side):
            for _ in range(max(warmup, 1)):
                device_part()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        own_positions = "attention_mask" not in self.static and "position_ids" not in self.static
        with torch.inference_mode(), (eager_mask_decisions() if own_positions else contextlib.nullcontext()), \
                torch.cuda.graph(self.graph):
            self.out = device_part()
        torch.cuda.synchronize(device)

    def _host_part(self, adapter_ids: list[str]) -> LoraBatchContext:
        return self.model.prepare_lora_context(
            adapter_ids, self.static.get("attention_mask"), self.batch, self.seq, self.device
        )

    def __call__(self, adapter_ids: list[str], **inputs: torch.Tensor) -> torch.Tensor:
        """Runs one forward with new inputs (same shapes) and adapter ids; the
        returned tensor is the graph's output buffer, overwritten by the next call."""
        for k, v in inputs.items():
            self.static[k].copy_(v, non_blocking=True)
        ctx = self._host_part(adapter_ids)
        stream = torch.cuda.current_stream(self.device)
        if ctx.ready_event is not None:
            stream.wait_event(ctx.ready_event)
        self.weight_indices.copy_(ctx.weight_indices, non_blocking=True)
        self.seq_lens.copy_(ctx.seq_lens, non_blocking=True)
        self.graph.replay()
        cache = self.model.adapter_cache
        slots = {cache.adapter_to_slot[a] for a in set(adapter_ids) if a != self.model.config.base_adapter_id}
        cache.mark_slots_used(slots)
        return self.out
