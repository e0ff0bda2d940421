"""Host-side logic of the API mirror (config, PEFT parsing, disk tier, slot
policy bookkeeping) on CPU, against the reference's golden outputs."""

import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from polylora_b200 import CpuAdapterStore, DiskAdapterCache, PolyLoraConfig
from polylora_b200.cache import GpuAdapterCache, ModuleSpec
from polylora_b200.context import LoraBatchContext, assert_right_padded, get_lora_context, use_lora_context
from polylora_b200.store import CpuLayerWeights

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("kwargs,msg", [
    (dict(max_gpu_adapters=0, max_rank=4), "max_gpu_adapters must be at least 1"),
    (dict(max_gpu_adapters=2, max_rank=4, max_cpu_adapters=1), "max_cpu_adapters must be at least max_gpu_adapters"),
    (dict(max_gpu_adapters=1, max_rank=4, max_disk_adapters=0, disk_cache_dir="x"), "max_disk_adapters must be at least 1"),
    (dict(max_gpu_adapters=1, max_rank=4, max_disk_adapters=2), "disk_cache_dir must be set"),
    (dict(max_gpu_adapters=1, max_rank=0), "max_rank must be at least 1"),
    (dict(max_gpu_adapters=1, max_rank=4, target_modules=[]), "target_modules must not be empty"),
])
def test_config_validation_messages(kwargs, msg):
    with pytest.raises(ValueError, match=msg):
        PolyLoraConfig(**kwargs)


def test_peft_state_dict_parsing_matches_reference(golden_dir):
    g = np.load(golden_dir / "peft_store.npz")
    sd = {k[4:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("sd__")}
    modules = ["encoder.layer.0.attention.self.query_proj", "encoder.layer.0.attention.self.value_proj",
               "encoder.layer.0.output.dense", "encoder.layer.0.attention.self.key_proj"]
    store = CpuAdapterStore()
    store.add_adapter_from_peft_state_dict("adp", sd, modules, 6.0, "adp")
    layers = store.adapters["adp"].layers
    assert set(layers) == {m for m in modules if f"{m}__A" in g.files}
    assert "encoder.layer.0.attention.self.key_proj" not in layers  # absent -> rank-0 no-op
    for m, w in layers.items():
        np.testing.assert_array_equal(w.A.numpy(), g[f"{m}__A"])
        np.testing.assert_array_equal(w.B.numpy(), g[f"{m}__B"])
        assert w.rank == int(g[f"{m}__rank"][0]) and w.scale == float(g[f"{m}__scale"][0])


def test_rejects_outside_module_set_and_incomplete_pair():
    store = CpuAdapterStore()
    sd = {"base_model.model.q.lora_A.weight": torch.zeros(2, 4), "base_model.model.q.lora_B.weight": torch.zeros(4, 2),
          "base_model.model.v.lora_A.weight": torch.zeros(2, 4), "base_model.model.v.lora_B.weight": torch.zeros(4, 2)}
    with pytest.raises(ValueError, match="outside the configured module set"):
        store.add_adapter_from_peft_state_dict("a", sd, ["v"], 4.0)
    del sd["base_model.model.v.lora_B.weight"]
    with pytest.raises(ValueError, match="incomplete LoRA weights"):
        store.add_adapter_from_peft_state_dict("a", sd, ["q", "v"], 4.0)


@pytest.mark.parametrize("cfg,msg", [
    ({"peft_type": "IA3", "lora_alpha": 2}, "Unsupported PEFT adapter type"),
    ({"use_dora": True, "lora_alpha": 2}, "DoRA adapters are not supported"),
    ({"use_rslora": True, "lora_alpha": 2}, "RS-LoRA adapters are not supported"),
    ({"lora_bias": True, "lora_alpha": 2}, "LoRA bias is not supported"),
    ({"lora_dropout": 0.1, "lora_alpha": 2}, "LoRA dropout is not supported"),
    ({"r": 2}, "missing lora_alpha"),
])
def test_peft_config_validation(cfg, msg):
    with pytest.raises(ValueError, match=msg):
        CpuAdapterStore._validate_peft_config_dict(cfg)


def _adapter_dir(path: Path):
    path.mkdir(parents=True)
    (path / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 4, "r": 2}))
    torch.save({}, path / "adapter_model.bin")
    return path


def test_disk_manifest_matches_reference_bytes(tmp_path, golden_dir):
    cache = DiskAdapterCache(tmp_path / "cache", max_adapters=2)
    for name in ("alpha", "b/eta", "gamma"):
        cache.add_adapter(name, _adapter_dir(tmp_path / f"src_{name.replace('/', '_')}"), "default")
    cache.get("b/eta")
    assert (tmp_path / "cache" / "manifest.json").read_text() == (golden_dir / "manifest.json").read_text()
    # restart: the manifest is reloaded, missing dirs are skipped
    again = DiskAdapterCache(tmp_path / "cache", max_adapters=2)
    assert list(again.entries) == ["gamma", "b/eta"]


def test_manifest_bytes_equal_json_dump_for_any_ids(tmp_path):
    """The manifest is assembled from cached per-entry blocks; its bytes must be
    those of json.dump(indent=2, sort_keys=True) of the LRU order, whatever the
    ids hold (quotes, backslashes, non-ASCII) and after touches and evictions."""
    cache = DiskAdapterCache(tmp_path / "cache", max_adapters=4)
    ids = ['plain', 'qu"ote', "back\\slash", "ünïcode/ß", "tab\tid", "x" * 40]
    for i, a in enumerate(ids):
        cache.add_adapter(a, _adapter_dir(tmp_path / f"src{i}"), "default" if i % 2 else "named")
        if i >= 2:
            cache.get(ids[1]) if ids[1] in cache else None

        payload = {"adapters": [{"adapter_id": e.adapter_id, "path": e.path.name,
                                 "peft_adapter_name": e.peft_adapter_name} for e in cache.entries.values()]}
        assert cache.manifest_path.read_text(encoding="utf-8") == json.dumps(payload, indent=2, sort_keys=True)
    empty = DiskAdapterCache(tmp_path / "empty")
    empty._write_manifest()
    assert empty.manifest_path.read_text() == json.dumps({"adapters": []}, indent=2, sort_keys=True)


def test_disk_cache_evicts_oldest_directory(tmp_path):
    cache = DiskAdapterCache(tmp_path / "c", max_adapters=2)
    srcs = {a: _adapter_dir(tmp_path / f"s_{a}") for a in "abc"}
    for a, p in srcs.items():
        cache.add_adapter(a, p)
    assert list(cache.entries) == ["b", "c"]
    dirs = [p for p in (tmp_path / "c").iterdir() if p.is_dir()]
    assert len(dirs) == 2 and all(p.name.startswith(("b-", "c-")) for p in dirs)


def test_cpu_lru_skips_gpu_resident_adapters():
    store = CpuAdapterStore(max_adapters=1)
    w = {"m": CpuLayerWeights(torch.zeros(4, 1), torch.zeros(1, 4), 1, 1.0)}
    store.add_adapter("a", w)
    store.set_eviction_exclusions({"a"})
    with pytest.raises(RuntimeError, match="No evictable CPU LoRA adapter"):
        store.add_adapter("b", w)
    assert "__base__" in store and "zz" not in store
    with pytest.raises(KeyError):
        store.get("__base__")


_CACHE_CHECK = r"""
import json, sys, torch
sys.path.insert(0, sys.argv[1])
from polylora_b200 import PolyLoraConfig, CpuAdapterStore
from polylora_b200.cache import GpuAdapterCache, ModuleSpec
from polylora_b200.store import CpuLayerWeights
data = json.load(open(sys.argv[2]))
for sc in data["scenarios"]:
    cfg = PolyLoraConfig(max_gpu_adapters=sc["max_gpu"], max_rank=4)
    store = CpuAdapterStore()
    for i, a in enumerate(sc["ids"]):
        r = 1 + i % 4
        store.add_adapter(a, {"m": CpuLayerWeights(torch.zeros(8, r), torch.zeros(r, 8), r, 1.0)})
    cache = GpuAdapterCache(store, [ModuleSpec("m", 8, 8)], cfg, torch.device("cpu"), torch.float32)
    for step in sc["steps"]:
        wi = cache.ensure_resident(step["adapter_ids"]).tolist()
        assert wi == step["weight_indices"], (wi, step)
        assert cache.slot_to_adapter == step["slot_to_adapter"]
        assert list(cache.lru) == step["lru"]
        assert cache.ranks["m"].tolist() == step["ranks"]
cfg = PolyLoraConfig(max_gpu_adapters=1, max_rank=4)
store = CpuAdapterStore()
for a in ("a", "b"):
    store.add_adapter(a, {"m": CpuLayerWeights(torch.zeros(8, 2), torch.zeros(2, 8), 2, 1.0)})
cache = GpuAdapterCache(store, [ModuleSpec("m", 8, 8)], cfg, torch.device("cpu"), torch.float32)
for label, ids in (("unknown", ["zz"]), ("capacity", ["a", "b"])):
    try:
        cache.ensure_resident(ids)
        raise SystemExit("no error")
    except (KeyError, RuntimeError) as exc:
        assert [type(exc).__name__, str(exc)] == data["errors"][label]
print("ok")
"""


def test_slot_bookkeeping_matches_reference_sequences(golden_dir):
    env = dict(os.environ, PYTHONHASHSEED="0")
    res = subprocess.run([sys.executable, "-c", _CACHE_CHECK, str(ROOT), str(golden_dir / "slot_sequences.json")],
                         capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stderr + res.stdout


def test_base_slot_is_zero_rank_zero_on_host_cache():
    cfg = PolyLoraConfig(max_gpu_adapters=2, max_rank=4)
    store = CpuAdapterStore()
    store.add_adapter("a", {"m": CpuLayerWeights(torch.ones(8, 2), torch.ones(2, 8), 2, 2.0)})
    cache = GpuAdapterCache(store, [ModuleSpec("m", 8, 8), ModuleSpec("n", 8, 8)], cfg, torch.device("cpu"), torch.float32)
    wi = cache.ensure_resident(["__base__", "a"])
    assert wi.tolist() == [0, 1] and cache.adapter_to_slot["__base__"] == 0
    for name in ("m", "n"):
        assert int(cache.ranks[name][0]) == 0 and float(cache.scales[name][0]) == 0.0
    assert int(cache.ranks["n"][1]) == 0  # module absent from the adapter -> rank 0
    assert int(cache.ranks["m"][1]) == 2 and float(cache.scales["m"][1]) == 2.0
    assert cache.table_ranks.tolist() == [0, 2, 0]


def test_rank_above_max_rank_is_rejected():
    cfg = PolyLoraConfig(max_gpu_adapters=1, max_rank=2)
    store = CpuAdapterStore()
    store.add_adapter("a", {"m": CpuLayerWeights(torch.ones(8, 3), torch.ones(3, 8), 3, 1.0)})
    cache = GpuAdapterCache(store, [ModuleSpec("m", 8, 8)], cfg, torch.device("cpu"), torch.float32)
    with pytest.raises(ValueError, match="exceeds max_rank"):
        cache.ensure_resident(["a"])
    assert cache.slot_to_adapter[1] is None


def test_lora_key_index_matches_the_scan():
    """The one-pass key index returns what the per-module suffix scan returns,
    including modules that are string suffixes of others and named adapters."""
    from polylora_b200.store import _find_lora_key, _lora_key_index

    mods = ["layer.1.dense", "encoder.layer.1.dense", "layer.11.dense", "q", "attn.q", "missing"]
    keys = ["base_model.model.encoder.layer.11.dense.lora_A.weight", "base_model.model.encoder.layer.1.dense.lora_A.weight",
            "base_model.model.encoder.layer.1.dense.lora_B.default.weight", "x.attn.q.lora_A.other.weight",
            "x.attn.q.lora_A.weight", "x.attn.q.lora_B.weight", "encoder.layer.11.dense.lora_B.weight", "unrelated.weight"]
    sd = {k: torch.zeros(1) for k in keys}
    for name in ("default", "other"):
        index = _lora_key_index(sd, mods, name)
        for m in mods:
            for side in ("lora_A", "lora_B"):
                assert index.get((m, side)) == _find_lora_key(sd, m, side, name), (name, m, side)


def test_slot_image_layout():
    from polylora_b200._native import SlotRecord

    store = CpuAdapterStore()
    a = torch.arange(12, dtype=torch.float32).reshape(6, 2)
    b = torch.arange(10, dtype=torch.float32).reshape(2, 5)
    store.add_adapter("x", {"m2": CpuLayerWeights(a, b, 2, 0.5)})
    image, ranks = store.slot_image("x", ["m1", "m2"], torch.bfloat16)
    assert ranks == [0, 2]
    recs = (SlotRecord * 2).from_buffer_copy(image[:48].numpy().tobytes())
    assert recs[0].rank == 0 and recs[1].rank == 2 and recs[1].scale == 0.5
    # blocks as PEFT stores them: A (r, in), B (out, r)
    got_a = image[recs[1].a_offset: recs[1].a_offset + 24].view(torch.bfloat16).float().reshape(2, 6)
    got_b = image[recs[1].b_offset: recs[1].b_offset + 20].view(torch.bfloat16).float().reshape(5, 2)
    assert torch.equal(got_a, a.t()) and torch.equal(got_b, b.t())
    assert recs[1].a_offset % 256 == 0 and recs[1].b_offset % 256 == 0


def test_context_var_and_right_padding():
    ctx = LoraBatchContext(["a"], torch.zeros(1, dtype=torch.int64), torch.ones(1, dtype=torch.int32))
    assert get_lora_context() is None
    with use_lora_context(ctx):
        assert get_lora_context() is ctx
    assert get_lora_context() is None
    mask = torch.tensor([[1, 1, 0], [1, 1, 1]])
    assert_right_padded(mask, mask.sum(-1))
    with pytest.raises(ValueError, match="right-padded"):
        bad = torch.tensor([[0, 1, 1]])
        assert_right_padded(bad, bad.sum(-1))
