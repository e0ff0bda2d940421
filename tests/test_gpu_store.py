"""The CPU tier's pinned slab pool and disk prefetch on a CUDA host."""

import pytest
import torch

from polylora_b200.store import PinnedSlabPool

pytestmark = pytest.mark.gpu


def test_pinned_slab_is_reused_only_after_its_copy_completes():
    pool = PinnedSlabPool(1 << 18, slabs_per_arena=2)
    a, b = pool.acquire(), pool.acquire()
    assert a.is_pinned() and b.is_pinned() and a.numel() == 1 << 18
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        torch.cuda._sleep(100_000_000)  # bounded busy kernel standing in for a long copy
        ev = torch.cuda.Event()
        ev.record(side)
    pool.note_use(a, ev)
    pool.release(a)
    assert len(pool.retired) == 1 and not pool.free  # its copy may still read it
    c = pool.acquire()  # a fresh arena, not the retired slab
    assert c.data_ptr() not in (a.data_ptr(), b.data_ptr()) and len(pool.arenas) == 2
    ev.synchronize()
    pool.release(b)
    pool.release(c)
    got = {pool.acquire().data_ptr() for _ in range(4)}
    assert a.data_ptr() in got  # reclaimed once its event completed
