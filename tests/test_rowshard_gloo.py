"""Row data-parallel partitioning and output gather, on CPU with gloo ranks
(world size 2 and 3); the LoRA forward is replaced by a row-local function so
no GPU is needed."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from polylora_b200.rowshard import RowParallel, all_gather_rows, partition_rows


@pytest.mark.parametrize("lens,world", [
    ([5] * 8, 2), ([1, 100, 1, 1, 100, 3], 2), ([7, 3, 9, 1, 0, 4, 4, 4], 3),
    ([2, 2], 4), ([10], 1), (list(range(1, 65)), 8),
])
def test_partition_is_contiguous_covering_and_balanced(lens, world):
    b = partition_rows(lens, world)
    assert len(b) == world and b[0][0] == 0 and b[-1][1] == len(lens)
    assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
    if len(lens) >= world:
        assert all(e > s for s, e in b)
        loads = [sum(max(v, 1) for v in lens[s:e]) for s, e in b]
        assert max(loads) <= sum(max(v, 1) for v in lens) / world + max(max(v, 1) for v in lens)


def test_row_cost_balances_padded_rows():
    """With a per-row cost of 1 (a model that computes every row at the padded
    length), shards get equal row counts whatever the valid lengths."""
    lens = [64] * 48 + [512] * 16  # token balancing would give the short rows' rank 3x the rows
    b = partition_rows(lens, 4, row_cost=lambda n: 1)
    assert [e - s for s, e in b] == [16, 16, 16, 16]
    bt = partition_rows(lens, 4)
    assert max(e - s for s, e in bt) > 16


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _row_fn(adapter_ids, input_ids, attention_mask):
    # row-local stand-in for PolyLoraModel: depends only on the row's own data
    salt = torch.tensor([sum(map(ord, a)) for a in adapter_ids], dtype=torch.float32)
    return input_ids.float() * 2 + attention_mask.float() + salt[:, None]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        rows = 7
        ids = torch.randint(0, 50, (rows, 6), generator=g)
        mask = torch.ones(rows, 6, dtype=torch.long)
        for r, L in enumerate([6, 2, 4, 6, 1, 3, 5]):
            mask[r, L:] = 0
        adapters = ["a", "b", "__base__", "a", "c", "b", "a"]
        got = RowParallel(_row_fn)(adapter_ids=adapters, input_ids=ids, attention_mask=mask)
        want = _row_fn(adapters, ids, mask)
        results[rank] = bool(torch.equal(got, want))
        # uneven shards gather back in order
        bounds = [(0, 3), (3, 4)] + [(4, 4)] * (world - 2)
        s, e = bounds[rank]
        full = torch.arange(8).reshape(4, 2).float()
        results[world + rank] = bool(torch.equal(all_gather_rows(full[s:e], bounds), full))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_parallel_matches_single_process(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert all(results[i] for i in range(2 * world)), dict(results)


def _failing_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        if rank == 1:
            return  # this rank leaves between steps and never joins the gather
        try:
            all_gather_rows(torch.ones(2, 2), [(0, 2), (2, 4)])
            results[rank] = "no error"
        except Exception as exc:  # noqa: BLE001 - any collective failure is the signal
            results[rank] = type(exc).__name__
    finally:
        if rank == 0:
            dist.destroy_process_group()


def test_missing_rank_surfaces_as_collective_error():
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert results.get(0) not in (None, "no error")
