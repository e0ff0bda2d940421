"""GpuAdapterCache's slot policy against the oracle's restatement of the
reference (src/polylora/cache.py:60-117) on random batch sequences: returned
slot indices, errors, slot contents and LRU order after every batch.

Both sides build the batch's ``needed`` set the same way in one process, so
they see the same set iteration order whatever the hash seed; the fixed
reference sequences (PYTHONHASHSEED=0) are checked against goldens elsewhere."""

import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle.slots_ref import SlotPolicy
from polylora_b200 import PolyLoraConfig
from polylora_b200.cache import GpuAdapterCache, ModuleSpec
from polylora_b200.store import CpuAdapterStore, CpuLayerWeights

KNOWN = [f"a{i}" for i in range(8)]
IDS = KNOWN + ["__base__", "__base__", "unknown"]


@st.composite
def sequences(draw):
    capacity = draw(st.integers(1, 4))
    batches = draw(st.lists(st.lists(st.sampled_from(IDS), min_size=1, max_size=6), min_size=1, max_size=12))
    return capacity, batches


def _outcome(fn):
    try:
        return ("ok", fn())
    except (KeyError, RuntimeError) as exc:
        return (type(exc).__name__, str(exc))


@settings(max_examples=300, deadline=None, derandomize=True, suppress_health_check=list(HealthCheck))
@given(sequences())
def test_slot_policy_matches_the_oracle(case):
    capacity, batches = case
    store = CpuAdapterStore()
    for a in KNOWN:
        store.add_adapter(a, {"m": CpuLayerWeights(torch.ones(4, 2), torch.ones(2, 4), 2, 1.0)})
    cache = GpuAdapterCache(store, [ModuleSpec("m", 4, 4)], PolyLoraConfig(max_gpu_adapters=capacity, max_rank=2),
                            torch.device("cpu"), torch.float32)
    ref = SlotPolicy(set(KNOWN), capacity)
    for batch in batches:
        got = _outcome(lambda: cache.ensure_resident(batch).tolist())
        want = _outcome(lambda: ref.ensure_resident(batch))
        assert got == want, (batch, got, want)
        assert list(cache.slot_to_adapter) == ref.slot_to_adapter
        assert list(cache.lru) == list(ref.lru)
        # a resident adapter's slot holds its rank; free slots hold rank 0
        for slot, a in enumerate(cache.slot_to_adapter):
            assert int(cache.ranks["m"][slot]) == (2 if a not in (None, "__base__") else 0)
