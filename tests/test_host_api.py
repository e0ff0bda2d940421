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
    (dict(max_gpu_adapters=1, max_rank=4, right_padding_check="gpu"), 'right_padding_check must be "host" or "device"'),
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


# ---------------------------------------------------------------- prefetch (CPU tier)
def _peft_dir(path: Path, mods, r, seed):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    path.mkdir(parents=True)
    (path / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 2 * r, "r": r}))
    sd = {}
    for m, (k, n) in mods.items():
        sd[f"base_model.model.{m}.lora_A.weight"] = torch.randn(r, k, generator=g)
        sd[f"base_model.model.{m}.lora_B.weight"] = torch.randn(n, r, generator=g)
    save_file(sd, str(path / "adapter_model.safetensors"))
    return path


def _disk_store(tmp_path, n=4, **kw):
    mods = {"enc.q": (6, 4), "enc.dense": (4, 8)}
    disk = DiskAdapterCache(tmp_path / "disk")
    for i in range(n):
        disk.add_adapter(f"ad{i}", _peft_dir(tmp_path / f"src{i}", mods, 2 + i % 2, i))
    return CpuAdapterStore(disk_cache=disk, module_names=list(mods), **kw), list(mods)


@pytest.mark.parametrize("workers", [1, 4])
@pytest.mark.parametrize("direct", [False, True], ids=["general", "native_packer"])
def test_prefetch_loads_the_same_weights_as_a_synchronous_get(tmp_path, workers, direct):
    """One or several workers, through the Python parser or the native packer
    (image spec published), while the main thread reads other adapters."""
    store, mods = _disk_store(tmp_path, n=6, prefetch_workers=workers)
    ref, _ = _disk_store(tmp_path / "ref", n=6)
    dt = torch.float32 if direct else torch.bfloat16  # the files hold fp32: the packer takes fp32 images only
    if direct:
        store.set_image_spec(mods, dt)
    wanted = ["ad1", "ad2", "ad3", "ad4", "ad5"]
    futs = store.prefetch(wanted[:2] + ["__base__", "unknown", "ad1"] + wanted[2:],
                          image_dtype=dt, module_names=mods)
    assert len(futs) == 5
    store.get("ad0")  # a synchronous load while the workers run
    for f in futs:
        f.result(timeout=30)
    assert set(wanted) <= set(store.adapters)
    for aid in wanted:
        got, want = store.get(aid), ref.get(aid)
        for m in mods:
            assert torch.equal(got.layers[m].A, want.layers[m].A) and torch.equal(got.layers[m].B, want.layers[m].B)
            assert got.layers[m].scale == want.layers[m].scale
        # the image was built by the worker and is what slot_image returns
        key = (aid, dt, tuple(mods))
        assert key in store._images
        image, ranks = store.slot_image(aid, mods, dt)
        assert torch.equal(image, ref.slot_image(aid, mods, dt)[0]) and ranks == [got.layers[m].rank for m in mods]
        # the native packer's weights are views of the packed image
        shares = got.layers[mods[0]].A.untyped_storage().data_ptr() == image.untyped_storage().data_ptr()
        assert shares == direct
    assert store.prefetch(["ad1"]) == []  # resident: nothing to start


def test_get_waits_for_an_inflight_prefetch_instead_of_loading_twice(tmp_path, monkeypatch):
    import threading
    import time

    store, mods = _disk_store(tmp_path)
    calls, gate = [], threading.Event()
    orig = store._read_peft_dir

    def slow_read(path):
        calls.append(path)
        gate.wait(5)
        return orig(path)

    monkeypatch.setattr(store, "_read_peft_dir", slow_read)
    (fut,) = store.prefetch(["ad3"])
    time.sleep(0.05)
    threading.Timer(0.2, gate.set).start()
    adapter = store.get("ad3")  # blocks until the worker has inserted it
    assert fut.done() and adapter is store.adapters["ad3"] and len(calls) == 1


def test_prefetch_errors_reach_the_future_and_get(tmp_path):
    store, mods = _disk_store(tmp_path, n=1)
    bad = tmp_path / "bad"
    bad.mkdir()
    (bad / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 2, "r": 2, "use_dora": True}))
    torch.save({}, bad / "adapter_model.bin")
    store.disk_cache.add_adapter("bad", bad)
    (fut,) = store.prefetch(["bad"])
    with pytest.raises(ValueError, match="DoRA"):
        fut.result(timeout=30)
    with pytest.raises(ValueError, match="DoRA"):
        store.get("bad")


def test_get_under_the_tier_lock_does_not_wait_for_a_prefetch(tmp_path, monkeypatch):
    """A GPU refill holds the tier's lock around get(); a prefetch of the same
    adapter in flight must not deadlock it (the worker needs the lock)."""
    import threading

    store, mods = _disk_store(tmp_path)
    gate = threading.Event()
    orig = store._read_peft_dir

    def gated_read(path):
        gate.wait(5)
        return orig(path)

    monkeypatch.setattr(store, "_read_peft_dir", gated_read)
    (fut,) = store.prefetch(["ad2"])
    result = {}

    def refill():
        with store.locked():
            monkeypatch.setattr(store, "_read_peft_dir", orig)  # the synchronous load is not gated
            result["adapter"] = store.get("ad2")
        gate.set()

    t = threading.Thread(target=refill)
    t.start()
    t.join(timeout=20)
    gate.set()
    assert not t.is_alive(), "get() under the lock waited for the prefetch"
    fut.result(timeout=20)
    assert store.adapters["ad2"] is result["adapter"]  # the worker discarded its copy


def _peft_dir_dtype(path: Path, mods, r, seed, dtype, tamper=None):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    path.mkdir(parents=True)
    (path / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 2 * r, "r": r}))
    sd = {}
    for m, (k, n) in mods.items():
        sd[f"base_model.model.{m}.lora_A.weight"] = torch.randn(r, k, generator=g).to(dtype)
        sd[f"base_model.model.{m}.lora_B.weight"] = torch.randn(n, r, generator=g).to(dtype)
    if tamper:
        tamper(sd)
    save_file(sd, str(path / "adapter_model.safetensors"))
    return path


@pytest.mark.parametrize("file_dtype", [torch.bfloat16, torch.float32])
def test_direct_safetensors_load_equals_the_general_path(tmp_path, file_dtype):
    mods = {"enc.q": (6, 4), "enc.dense": (4, 8), "enc.absent": (3, 3)}
    names = list(mods)
    disk = DiskAdapterCache(tmp_path / "disk")
    for i in range(3):
        disk.add_adapter(f"ad{i}", _peft_dir_dtype(tmp_path / f"s{i}", {m: mods[m] for m in names[:2]}, 2 + i, i, file_dtype))
    fast = CpuAdapterStore(disk_cache=disk, module_names=names)
    fast.set_image_spec(names, torch.bfloat16)
    slow = CpuAdapterStore(disk_cache=disk, module_names=names)
    for i in range(3):
        aid = f"ad{i}"
        a, b = fast.get(aid), slow.get(aid)
        # with bf16 files the image is written while loading (no second build)
        assert ((aid, torch.bfloat16, tuple(names)) in fast._images) == (file_dtype == torch.bfloat16)
        assert a.layers.keys() == b.layers.keys() and "enc.absent" not in a.layers
        for m in a.layers:
            la, lb = a.layers[m], b.layers[m]
            assert la.rank == lb.rank and la.scale == lb.scale and la.A.dtype == lb.A.dtype == file_dtype
            assert torch.equal(la.A, lb.A) and torch.equal(la.B, lb.B)
            assert tuple(la.A.shape) == (mods[m][0], la.rank) and tuple(la.B.shape) == (la.rank, mods[m][1])
        img_a, ranks_a = fast.slot_image(aid, names, torch.bfloat16)
        img_b, ranks_b = slow.slot_image(aid, names, torch.bfloat16)
        assert ranks_a == ranks_b and torch.equal(img_a, img_b)


@pytest.mark.parametrize("tamper,msg", [
    (lambda sd: sd.update({"base_model.model.enc.q.lora_B.weight": torch.zeros(4, 3, dtype=torch.bfloat16)}), "rank mismatch"),
    (lambda sd: sd.pop("base_model.model.enc.dense.lora_B.weight"), "incomplete LoRA weights"),
    (lambda sd: sd.update({"base_model.model.other.lora_A.weight": torch.zeros(2, 2, dtype=torch.bfloat16)}),
     "outside the configured module set"),
])
def test_direct_load_raises_the_general_paths_errors(tmp_path, tamper, msg):
    mods = {"enc.q": (6, 4), "enc.dense": (4, 8)}
    disk = DiskAdapterCache(tmp_path / "disk")
    disk.add_adapter("bad", _peft_dir_dtype(tmp_path / "s", mods, 2, 0, torch.bfloat16, tamper))
    for spec in (True, False):
        store = CpuAdapterStore(disk_cache=disk, module_names=list(mods))
        if spec:
            store.set_image_spec(list(mods), torch.bfloat16)
        with pytest.raises(ValueError, match=msg):
            store.get("bad")
        assert "bad" not in store.adapters


def test_native_packer_follows_the_reference_key_rules(tmp_path):
    """Module names that are string suffixes of others, adapter-named keys,
    __metadata__ and unrelated tensors: the packed load equals the general one."""
    from safetensors.torch import save_file

    mods = {"layer.1.dense": (4, 6), "encoder.layer.1.dense": (4, 6), "layer.11.dense": (5, 3), "q": (3, 3),
            "attn.q": (3, 3)}
    g = torch.Generator().manual_seed(7)
    t = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)  # noqa: E731
    sd = {
        "base_model.model.encoder.layer.11.dense.lora_A.weight": t(2, 5),
        "base_model.model.encoder.layer.11.dense.lora_B.weight": t(3, 2),
        "base_model.model.encoder.layer.1.dense.lora_A.default.weight": t(3, 4),
        "base_model.model.encoder.layer.1.dense.lora_B.default.weight": t(6, 3),
        "x.attn.q.lora_A.weight": t(2, 3),
        "x.attn.q.lora_B.weight": t(3, 2),
        "x.attn.q.lora_A.other.weight": t(4, 3),
        "unrelated.weight": t(2, 2),
    }
    path = tmp_path / "src"
    path.mkdir()
    (path / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 8, "r": 2}))
    save_file(sd, str(path / "adapter_model.safetensors"), metadata={"format": "pt", "note": 'é "q" \\ x'})
    names = list(mods)
    disk = DiskAdapterCache(tmp_path / "disk")
    disk.add_adapter("a", path)
    fast = CpuAdapterStore(disk_cache=disk, module_names=names)
    fast.set_image_spec(names, torch.bfloat16)
    slow = CpuAdapterStore(disk_cache=disk, module_names=names)
    a, b = fast.get("a"), slow.get("a")
    assert ("a", torch.bfloat16, tuple(names)) in fast._images  # packed natively
    assert a.layers.keys() == b.layers.keys()
    for m in a.layers:
        assert torch.equal(a.layers[m].A, b.layers[m].A) and torch.equal(a.layers[m].B, b.layers[m].B)
        assert a.layers[m].rank == b.layers[m].rank and a.layers[m].scale == b.layers[m].scale
    assert torch.equal(fast.slot_image("a", names, torch.bfloat16)[0], slow.slot_image("a", names, torch.bfloat16)[0])


def _raw_safetensors(path: Path, header: bytes, data: bytes = b"", declared_len: int | None = None) -> Path:
    n = len(header) if declared_len is None else declared_len
    path.write_bytes(n.to_bytes(8, "little") + header + data)
    return path


def test_native_packer_declines_hostile_headers(tmp_path):
    """The packer reads untrusted files: shapes whose byte count overflows,
    over-deep JSON, a header longer than the file and offsets past the data are
    declined (PLORA_ERR_UNSUPPORTED) with nothing written."""
    import ctypes

    from polylora_b200 import _native

    lib = _native.load()
    mods = (ctypes.c_char_p * 1)(b"enc.q")
    dims = (ctypes.c_int64 * 3)()
    nbytes = ctypes.c_size_t(0)
    image = torch.full((4096,), 0xAB, dtype=torch.uint8)

    def pack(path):
        return lib.plora_peft_pack(str(path).encode(), mods, 1, b"default", 2, 8.0, image.data_ptr(), image.numel(),
                                   ctypes.byref(nbytes), dims)

    huge = 1 << 62  # 2^62 x 4 bf16 elements: the byte count wraps to 0 in 64 bits
    overflow = {"base_model.model.enc.q.lora_A.weight": {"dtype": "BF16", "shape": [huge, 4], "data_offsets": [0, 0]},
                "base_model.model.enc.q.lora_B.weight": {"dtype": "BF16", "shape": [4, huge], "data_offsets": [0, 0]}}
    past_end = {"base_model.model.enc.q.lora_A.weight": {"dtype": "BF16", "shape": [2, 4], "data_offsets": [0, 16]},
                "base_model.model.enc.q.lora_B.weight": {"dtype": "BF16", "shape": [4, 2], "data_offsets": [16, 4096]}}
    cases = {
        "overflow": _raw_safetensors(tmp_path / "o.safetensors", json.dumps(overflow).encode()),
        "deep": _raw_safetensors(tmp_path / "d.safetensors", b"[" * 200 + b"]" * 200),
        "long_header": _raw_safetensors(tmp_path / "h.safetensors", b'{"a": 1}', declared_len=1 << 20),
        "past_end": _raw_safetensors(tmp_path / "p.safetensors", json.dumps(past_end).encode(), bytes(32)),
    }
    for name, path in cases.items():
        assert pack(path) == _native.ERR_UNSUPPORTED, name
        assert bool((image == 0xAB).all()), f"{name}: image written"
    assert pack(tmp_path / "missing.safetensors") == _native.ERR_INVALID_ARGUMENT


def test_disk_cache_replays_reference_sequences(tmp_path, golden_dir):
    """DiskAdapterCache on operation sequences recorded from the reference
    (adds, invalid sources, gets, touches, reopening from the manifest): the
    outcome, entry order, directories on disk and manifest text match after
    every step."""
    ids = ["a", "b", "c/d", "e f", "ünï", "__x"]
    sequences = json.loads((golden_dir / "disk_sequences.json").read_text())
    for n, seq in enumerate(sequences):
        root = tmp_path / f"s{n}"
        srcs = []
        for i in range(4):  # three valid PEFT directories and one without weights
            d = root / "sources" / f"src{i}"
            d.mkdir(parents=True)
            (d / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 4, "r": 2}))
            if i < 3:
                (d / "adapter_model.bin").write_bytes(b"weights-%d" % i)
            srcs.append(d)
        cache_dir = root / "cache"
        cache = DiskAdapterCache(cache_dir, max_adapters=seq["max_adapters"])
        for step in seq["steps"]:
            try:
                if step["op"] == "add":
                    cache.add_adapter(ids[step["id"]], srcs[step["src"]], step["name"])
                elif step["op"] == "get":
                    cache.get(ids[step["id"]])
                elif step["op"] == "touch":
                    cache.touch(ids[step["id"]])
                else:
                    cache = DiskAdapterCache(cache_dir, max_adapters=seq["max_adapters"])
                outcome = ["ok"]
            except (KeyError, FileNotFoundError, RuntimeError) as exc:
                outcome = [type(exc).__name__, str(exc).replace(str(srcs[step["src"]]), "<src>")]
            manifest = cache_dir / "manifest.json"
            assert outcome == step["outcome"], (n, step)
            assert list(cache.entries) == step["entries"], (n, step)
            assert sorted(p.name for p in cache_dir.iterdir() if p.is_dir()) == step["dirs"], (n, step)
            assert (manifest.read_text() if manifest.exists() else None) == step["manifest"], (n, step)
