"""CpuAdapterStore's in-memory LRU against the oracle's restatement of the
reference (oracle/store_ref.py) on random operation sequences: adds, gets,
touches and eviction exclusions; the resident order and every error must
match after each operation."""

import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle.store_ref import CpuLru
from polylora_b200.store import CpuAdapterStore, CpuLayerWeights

IDS = [f"a{i}" for i in range(6)] + ["__base__"]

op = st.one_of(
    st.tuples(st.just("add"), st.sampled_from(IDS)),
    st.tuples(st.just("get"), st.sampled_from(IDS)),
    st.tuples(st.just("touch"), st.sampled_from(IDS)),
    st.tuples(st.just("exclude"), st.frozensets(st.sampled_from(IDS), max_size=4)),
)


def _outcome(fn):
    try:
        fn()
        return ("ok",)
    except (KeyError, ValueError, RuntimeError) as exc:
        return (type(exc).__name__, str(exc))


@settings(max_examples=300, deadline=None, derandomize=True, suppress_health_check=list(HealthCheck))
@given(st.one_of(st.none(), st.integers(1, 4)), st.lists(op, min_size=1, max_size=25))
def test_cpu_lru_matches_the_oracle(max_adapters, ops):
    store = CpuAdapterStore(max_adapters=max_adapters)
    ref = CpuLru(max_adapters)
    layers = {"m": CpuLayerWeights(torch.ones(4, 2), torch.ones(2, 4), 2, 1.0)}
    for kind, arg in ops:
        if kind == "add":
            got = _outcome(lambda: store.add_adapter(arg, layers))
            want = _outcome(lambda: ref.add_adapter(arg))
        elif kind == "get":
            got = _outcome(lambda: store.get(arg))
            want = _outcome(lambda: ref.get(arg))
        elif kind == "touch":
            got = _outcome(lambda: store.touch(arg))
            want = _outcome(lambda: ref.touch(arg))
        else:
            got = _outcome(lambda: store.set_eviction_exclusions(set(arg)))
            want = _outcome(lambda: ref.set_eviction_exclusions(set(arg)))
        assert got == want, (kind, arg, got, want)
        assert list(store.adapters) == list(ref.adapters), (kind, arg)
