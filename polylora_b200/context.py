"""Per-forward batch context shared by every wrapped Linear.

Mirrors src/polylora/context.py:11-45: a ContextVar carries the slot of each
row (``weight_indices``) and its valid length (``seq_lens``) so that it is
local to the thread / async task running the forward.  In addition the
context caches the device segment tables built for this batch (one per
layer layout) and the event that orders slot refills before the first LoRA
kernel.
"""

from __future__ import annotations

from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass, field
from typing import Any, Iterator

import torch


@dataclass(frozen=True)
class LoraBatchContext:
    adapter_ids: list[str]
    weight_indices: torch.Tensor
    seq_lens: torch.Tensor
    attention_mask: torch.Tensor | None = None
    # slot ranks used to build segment tables (max over modules, per slot)
    table_ranks: torch.Tensor | None = None
    # event recorded after this batch's slot refills (None: nothing pending)
    ready_event: Any = None
    # (row_slice, max_seq) -> SegmentTable, filled lazily by the layers
    segments: dict = field(default_factory=dict, compare=False, repr=False)


_CURRENT: ContextVar[LoraBatchContext | None] = ContextVar("polylora_b200_lora_context", default=None)


def get_lora_context() -> LoraBatchContext | None:
    return _CURRENT.get()


@contextmanager
def use_lora_context(ctx: LoraBatchContext | None) -> Iterator[None]:
    token = _CURRENT.set(ctx)
    try:
        yield
    finally:
        _CURRENT.reset(token)


RIGHT_PADDING_ERROR = "Custom multi-LoRA runtime currently requires right-padded attention_mask"


def assert_right_padded(attention_mask: torch.Tensor, seq_lens: torch.Tensor) -> None:
    """Raises unless every mask row is ones followed by zeros (context.py:37-45).
    Compares on the host, so it waits for the device."""
    if attention_mask.dim() != 2:
        raise ValueError("attention_mask must be a 2D batch mask")
    width = attention_mask.shape[1]
    expected = torch.arange(width, device=attention_mask.device)[None, :] < seq_lens[:, None]
    if not torch.equal(attention_mask.bool(), expected):
        raise ValueError(RIGHT_PADDING_ERROR)
