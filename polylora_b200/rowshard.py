"""Row data-parallel execution of a mixed-adapter batch over the GPUs of a node.

Batch rows are independent on the LoRA path: a row reads only its own
adapter's slot and the (replicated) base weights.  So a batch is cut into
contiguous row shards balanced by valid tokens, every rank runs its shard
through its own ``PolyLoraModel`` (own GPU slot cache), and one all-gather of
the padded shard outputs rebuilds the full batch on every rank.  This is the
only collective of the path; nothing else crosses GPUs.

The reference has no multi-GPU code; this module implements the row
partitioning the build adds on top of it.
"""

from __future__ import annotations

from typing import Any, Callable, Sequence

import torch
import torch.distributed as dist


def partition_rows(
    seq_lens: Sequence[int], world_size: int, row_cost: Callable[[int], float] | None = None
) -> list[tuple[int, int]]:
    """Contiguous row ranges ``[start, end)`` per rank, balanced by cost.

    A row costs ``row_cost(seq_len)``; the default is its valid tokens (at
    least 1: an empty row still occupies the batch).  A model that computes
    every row at the padded length (eager attention over the whole padded
    sequence) costs the same per row: pass ``lambda n: 1`` to balance rows.
    Cuts are placed where the running cost crosses k/world_size of the total;
    every range is non-empty when there are at least ``world_size`` rows
    (otherwise the trailing ranks get empty ranges).  Deterministic, so every
    rank computes the same partition from the same ``seq_lens``.
    """
    if world_size < 1:
        raise ValueError("world_size must be at least 1")
    lens = [max(int(v), 0) for v in seq_lens]
    rows = len(lens)
    cost = row_cost if row_cost is not None else (lambda n: max(n, 1))
    weights = [float(cost(v)) for v in lens]
    total = sum(weights)
    bounds: list[tuple[int, int]] = []
    start = 0
    acc = 0
    for k in range(world_size):
        remaining_ranks = world_size - k - 1
        end = start
        if k == world_size - 1:
            end = rows
        else:
            target = total * (k + 1) / world_size
            # take at least one row, leave at least one per remaining rank
            while end < rows - remaining_ranks and (end == start or acc + weights[end] / 2 <= target):
                acc += weights[end]
                end += 1
        bounds.append((start, end))
        start = end
    return bounds


def all_gather_rows(local: torch.Tensor, bounds: list[tuple[int, int]], group=None) -> torch.Tensor:
    """Concatenates every rank's row shard (shapes may differ only in dim 0)."""
    world = len(bounds)
    rows = [e - s for s, e in bounds]
    max_rows = max(max(rows), 1)
    pad = torch.zeros((max_rows,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    if local.shape[0]:
        pad[: local.shape[0]] = local
    out = torch.empty((world * max_rows,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    parts = [out[r * max_rows : r * max_rows + rows[r]] for r in range(world)]
    return torch.cat(parts, dim=0)


class RowParallel:
    """Runs ``fn(**row_shard_kwargs, adapter_ids=shard_ids)`` on this rank's rows.

    ``fn`` is typically a ``PolyLoraModel`` (or a lambda extracting
    ``.last_hidden_state`` from it).  Batch tensors are the keyword arguments
    whose first dimension equals the number of rows; they are sliced, other
    arguments are passed through.  Returns the full-batch output (all-gathered).

    The partition needs each row's length on the host.  With
    ``row_cost=RowParallel.EQUAL_ROWS`` (every row costs the same: models that
    compute every row at the padded length) it needs none; otherwise it takes
    ``host_seq_lens`` (a list the caller already holds, e.g. from its
    tokenizer) or, failing that, reads the attention mask back from the
    device, which waits for the work queued before it.
    """

    EQUAL_ROWS = object()  # row_cost: balance rows, no lengths needed

    def __init__(self, fn: Callable[..., torch.Tensor], group=None,
                 row_cost: Callable[[int], float] | object | None = None) -> None:
        self.fn = fn
        self.group = group
        self.row_cost = row_cost  # see partition_rows, or EQUAL_ROWS

    def _seq_lens(self, rows: int, host_seq_lens, batch: dict) -> list[int]:
        if host_seq_lens is not None:
            return [int(v) for v in host_seq_lens]
        mask = batch.get("attention_mask")
        if mask is not None:
            return mask.sum(-1).tolist()  # device -> host read
        ref = batch.get("input_ids", batch.get("inputs_embeds"))
        return [int(ref.shape[1])] * rows

    def __call__(self, adapter_ids: list[str], host_seq_lens: Sequence[int] | None = None,
                 **batch: Any) -> torch.Tensor:
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        rows = len(adapter_ids)
        if self.row_cost is RowParallel.EQUAL_ROWS:
            bounds = partition_rows([1] * rows, world, lambda n: 1)
        else:
            bounds = partition_rows(self._seq_lens(rows, host_seq_lens, batch), world, self.row_cost)
        start, end = bounds[rank]
        if end == start:  # fewer rows than ranks: run a copy of the last row, drop it
            start, end = rows - 1, rows
            keep = 0
        else:
            keep = end - start
        shard = {
            k: (v[start:end] if torch.is_tensor(v) and v.dim() and v.shape[0] == rows else v)
            for k, v in batch.items()
        }
        out = self.fn(adapter_ids=list(adapter_ids[start:end]), **shard)
        out = out[:keep]
        if world == 1:
            return out
        return all_gather_rows(out, bounds, self.group)
