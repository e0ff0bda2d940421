"""The CPU oracle pinned against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  No GPU needed."""

import json
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import schedule_ref, sgmv_ref

# Tolerances of the north star: fp32 <= 1e-5, bf16 <= 2e-2 max relative error
# against an fp32-accumulated reference, measured by oracle.sgmv_ref.lora_err
# (error beyond one output ulp, relative to the largest LoRA delta).
TOL = {"float32": 1e-5, "bfloat16": 2e-2}


def _cases(npz):
    names = sorted({k.split("__")[0] for k in npz.files})
    return names


def test_flat_schedule_oracle_matches_reference(golden_dir):
    g = np.load(golden_dir / "flat_schedule.npz")
    for name in _cases(g):
        bm, bn = g[f"{name}__blocks"].tolist()
        cum, nn, total = schedule_ref.flat_schedule(g[f"{name}__seq"], g[f"{name}__neff"], bm, bn)
        np.testing.assert_array_equal(cum, g[f"{name}__cum"], err_msg=name)
        np.testing.assert_array_equal(nn, g[f"{name}__nn"], err_msg=name)
        assert total == int(g[f"{name}__total"][0])


@pytest.mark.parametrize("case", ["cfg1_rows_f32", "tokens_f32", "odd_rank_f32",
                                  "rows_bf16", "tokens_bf16", "rank64_bf16"])
def test_lora_oracle_matches_reference_forward(golden_dir, case):
    g = np.load(golden_dir / "reference_forward.npz")
    get = lambda k: g[f"{case}__{k}"]  # noqa: E731
    dtype = str(get("dtype")[0])
    ref = get("out")
    ours = sgmv_ref.lora_forward_fp32(get("x"), get("A"), get("B"), get("seq"), get("wi"),
                                      get("ranks"), get("scales"), get("y"))
    # the reference stores in `dtype`; the oracle is the fp32-accumulated form
    err = sgmv_ref.lora_err(ref, ours, get("y"), dtype)
    assert err <= TOL[dtype], f"{case}: {err}"
    assert sgmv_ref.rel_err(ref, ours) <= TOL[dtype]
    # tokens the reference leaves alone (rank-0 slot / padding) are identical
    inactive = _inactive_mask(get("x").shape[1], get("seq"), get("wi"), get("ranks"))
    assert np.array_equal(ref[inactive], get("y")[inactive])
    assert np.array_equal(ours[inactive], get("y")[inactive])


def _inactive_mask(M, seq, wi, ranks):
    m = np.arange(M)[None, :]
    active = (m < np.minimum(seq, M)[:, None]) & (ranks[wi] > 0)[:, None]
    return ~active


@pytest.mark.parametrize("case", ["rows_bf16", "tokens_bf16", "rank64_bf16"])
def test_shrink_expand_oracle_composes_to_forward(golden_dir, case):
    g = np.load(golden_dir / "reference_forward.npz")
    get = lambda k: g[f"{case}__{k}"]  # noqa: E731
    tmp, written = sgmv_ref.shrink(get("x"), get("A"), get("seq"), get("wi"), get("ranks"), 1, "bfloat16")
    out = sgmv_ref.expand(tmp, get("B"), get("seq"), get("wi"), get("ranks"), get("scales"), get("y"), "bfloat16")
    ref = sgmv_ref.lora_forward_fp32(get("x"), get("A"), get("B"), get("seq"), get("wi"),
                                     get("ranks"), get("scales"), get("y"))
    assert sgmv_ref.lora_err(out, ref, get("y"), "bfloat16") <= TOL["bfloat16"]
    assert sgmv_ref.lora_err(get("out"), ref, get("y"), "bfloat16") <= TOL["bfloat16"]


def test_round_to_bf16_is_nearest_even():
    vals = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-9, -2.5, 3.14159, 1e-40, np.inf], dtype=np.float32)
    got = sgmv_ref.round_to(vals, "bfloat16")
    import torch

    want = torch.from_numpy(vals).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(got, want)


def test_segments_oracle_properties():
    rng = np.random.default_rng(0)
    for _ in range(20):
        B, M, ns = int(rng.integers(0, 50)), int(rng.integers(1, 9)), int(rng.integers(1, 12))
        wi = rng.integers(0, ns, size=B)
        sl = rng.integers(-1, M + 3, size=B)
        rk = rng.choice([0, 4, 8, 16], size=ns)
        start, tok = schedule_ref.segments(wi, sl, rk, M, ns)
        assert start[0] == 0 and np.all(np.diff(start) >= 0) and start[-1] == len(tok)
        for s in range(ns):
            part = tok[start[s]:start[s + 1]]
            assert np.all(np.diff(part) > 0)
            assert np.all(wi[part // M] == s)
            assert len(part) == 0 or rk[s] > 0
        expect = sum(min(max(int(sl[b]), 0), M) for b in range(B) if rk[wi[b]] > 0)
        assert len(tok) == expect


_SLOT_CHECK = r"""
import json, sys
sys.path.insert(0, sys.argv[1])
from oracle.slots_ref import SlotPolicy
data = json.load(open(sys.argv[2]))
for sc in data["scenarios"]:
    pol = SlotPolicy(set(sc["ids"]), sc["max_gpu"])
    for step in sc["steps"]:
        wi = pol.ensure_resident(step["adapter_ids"])
        assert wi == step["weight_indices"], (wi, step)
        assert pol.slot_to_adapter == step["slot_to_adapter"], (pol.slot_to_adapter, step)
        assert list(pol.lru) == step["lru"], (list(pol.lru), step)
for label, ids in (("unknown", ["zz"]), ("capacity", ["a", "b"])):
    pol = SlotPolicy({"a", "b"}, 1)
    try:
        pol.ensure_resident(ids)
        raise SystemExit("no error for " + label)
    except (KeyError, RuntimeError) as exc:
        assert [type(exc).__name__, str(exc)] == data["errors"][label], (label, exc)
print("ok")
"""


def test_slot_policy_oracle_matches_reference_sequences(golden_dir):
    root = golden_dir.parents[1]
    env = dict(os.environ, PYTHONHASHSEED="0")
    res = subprocess.run([sys.executable, "-c", _SLOT_CHECK, str(root), str(golden_dir / "slot_sequences.json")],
                         capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stderr + res.stdout
    assert json.loads((golden_dir / "slot_sequences.json").read_text())["hashseed"] == 0


def _replay_lru(make, seq):
    store = make(seq["max_adapters"])
    for step in seq["steps"]:
        try:
            if step["op"] == "add":
                store.add(step["arg"])
            elif step["op"] == "get":
                store.get(step["arg"])
            elif step["op"] == "touch":
                store.touch(step["arg"])
            else:
                store.exclude(set(step["arg"]))
            outcome = ["ok"]
        except (KeyError, ValueError, RuntimeError) as exc:
            outcome = [type(exc).__name__, str(exc)]
        assert outcome == step["outcome"], step
        assert store.resident() == step["resident"], step


def test_cpu_lru_oracle_and_store_match_reference_sequences(golden_dir):
    """The CPU tier's LRU (oracle/store_ref.py, and CpuAdapterStore itself)
    replays the reference's recorded operation sequences exactly."""
    import torch

    from oracle.store_ref import CpuLru
    from polylora_b200.store import CpuAdapterStore, CpuLayerWeights

    layers = {"m": CpuLayerWeights(torch.ones(4, 2), torch.ones(2, 4), 2, 1.0)}

    class OracleView:
        def __init__(self, cap):
            self.s = CpuLru(cap)
            self.add, self.get, self.touch = self.s.add_adapter, self.s.get, self.s.touch
            self.exclude = self.s.set_eviction_exclusions

        def resident(self):
            return list(self.s.adapters)

    class StoreView:
        def __init__(self, cap):
            self.s = CpuAdapterStore(max_adapters=cap)
            self.get, self.touch, self.exclude = self.s.get, self.s.touch, self.s.set_eviction_exclusions

        def add(self, a):
            self.s.add_adapter(a, layers)

        def resident(self):
            return list(self.s.adapters)

    sequences = json.loads((golden_dir / "cpu_lru_sequences.json").read_text())
    assert len(sequences) == 60
    for seq in sequences:
        _replay_lru(OracleView, seq)
        _replay_lru(StoreView, seq)


def test_strict_error_catches_a_delta_lost_on_large_outputs():
    """A planted mistake (30% of the LoRA delta dropped on the elements whose
    base output is large) hides under the one-ulp allowance of lora_err but
    not under the half-ulp allowance of lora_err_strict: the rounding of
    y + delta into bf16 costs at most half an output ulp."""
    rng = np.random.default_rng(5)
    y = sgmv_ref.round_to(rng.normal(0, 1, size=(4096,)).astype(np.float32) * 4, "bfloat16")
    delta = rng.normal(0, 0.03, size=y.shape)
    ref = (y.astype(np.float64) + delta).astype(np.float32)
    big = np.abs(y) > 3.0
    planted = y.astype(np.float64) + np.where(big, 0.7 * delta, delta)
    out = sgmv_ref.round_to(planted.astype(np.float32), "bfloat16")
    good = sgmv_ref.round_to(ref, "bfloat16")
    assert sgmv_ref.lora_err_strict(good, ref, y, "bfloat16") <= 1e-6  # correct rounding passes exactly
    assert sgmv_ref.lora_err_strict(out, ref, y, "bfloat16") > 0.05
    # the loose form lets part of the planted error through
    assert sgmv_ref.lora_err(out, ref, y, "bfloat16") < sgmv_ref.lora_err_strict(out, ref, y, "bfloat16")
