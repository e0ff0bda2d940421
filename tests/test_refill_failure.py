"""Failures of the CPU / disk tier in the middle of a GPU-slot refill.

The reference evicts a slot (zeroing it in every module) before it asks the
CPU tier for the incoming adapter (src/polylora/cache.py:97-150); when that
request fails the batch raises and the slot stays free at rank 0 / scale 0.
Here the failure is made on the host: the store's ``get`` raises for one
adapter (a lost CPU-tier entry), or the adapter's files on the disk tier are
corrupted after registration.  The cache is placed on the CPU device, whose
bookkeeping path is the one the CUDA path shares; the GPU version of the
same sequence is in test_gpu_model.py.
"""

import json

import pytest
import torch

from polylora_b200 import CpuAdapterStore, DiskAdapterCache, PolyLoraConfig
from polylora_b200.cache import GpuAdapterCache, ModuleSpec
from polylora_b200.store import CpuLayerWeights

MODS = [ModuleSpec("q", 8, 6), ModuleSpec("v", 8, 6)]


def _weights(seed, r):
    g = torch.Generator().manual_seed(seed)
    return {m.name: CpuLayerWeights(torch.randn(m.in_features, r, generator=g), torch.randn(r, m.out_features, generator=g),
                                    r, 2.0) for m in MODS}


def _store_and_cache(ids, max_gpu=2):
    store = CpuAdapterStore()
    for i, a in enumerate(ids):
        store.add_adapter(a, _weights(i, 1 + i % 4))
    cfg = PolyLoraConfig(max_gpu_adapters=max_gpu, max_rank=4)
    return store, GpuAdapterCache(store, MODS, cfg, torch.device("cpu"), torch.float32)


def _assert_slot_holds(cache, store, adapter_id):
    slot = cache.adapter_to_slot[adapter_id]
    w = store.get(adapter_id).layers
    for i, m in enumerate(MODS):
        r = w[m.name].rank
        assert int(cache.ranks[m.name][slot]) == r
        assert float(cache.scales[m.name][slot]) == float(w[m.name].scale)
        assert torch.equal(cache.A[m.name][slot, :, :r], w[m.name].A)
        assert torch.equal(cache.B[m.name][slot, :r, :], w[m.name].B)


def test_store_get_failure_after_eviction_leaves_slot_free_and_zeroed(monkeypatch):
    store, cache = _store_and_cache(["a", "b", "c", "d"])
    cache.ensure_resident(["a", "b"])  # both slots used; "a" is now the LRU victim
    victim_slot = cache.adapter_to_slot["a"]
    assert int(cache.ranks["q"][victim_slot]) > 0

    real_get = store.get

    def failing_get(adapter_id):
        if adapter_id == "c":
            raise OSError("adapter files unreadable")
        return real_get(adapter_id)

    monkeypatch.setattr(store, "get", failing_get)
    with pytest.raises(OSError, match="unreadable"):
        cache.ensure_resident(["b", "c"])
    # the victim was evicted, the incoming adapter never became resident, and
    # the freed slot reads rank 0 / scale 0 in every module
    assert "a" not in cache.adapter_to_slot and "c" not in cache.adapter_to_slot
    assert cache.slot_to_adapter[victim_slot] is None
    for m in MODS:
        assert int(cache.ranks[m.name][victim_slot]) == 0
        assert float(cache.scales[m.name][victim_slot]) == 0.0
    assert int(cache.table_ranks[victim_slot]) == 0

    # later batches are served correctly, the freed slot reused first
    monkeypatch.setattr(store, "get", real_get)
    wi = cache.ensure_resident(["d", "b", "__base__"])
    assert cache.adapter_to_slot["d"] == victim_slot
    assert wi.tolist() == [victim_slot, cache.adapter_to_slot["b"], 0]
    for a in ("b", "d"):
        _assert_slot_holds(cache, store, a)
    wi = cache.ensure_resident(["c", "d"])  # and the adapter that failed loads now
    _assert_slot_holds(cache, store, "c")


def _peft_dir(path, r, seed):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    path.mkdir(parents=True)
    (path / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 2 * r, "r": r}))
    sd = {}
    for m in MODS:
        sd[f"base_model.model.{m.name}.lora_A.weight"] = torch.randn(r, m.in_features, generator=g)
        sd[f"base_model.model.{m.name}.lora_B.weight"] = torch.randn(m.out_features, r, generator=g)
    save_file(sd, str(path / "adapter_model.safetensors"))
    return path


def test_corrupt_disk_adapter_mid_refill(tmp_path):
    """The disk tier holds an adapter whose safetensors file was truncated after
    registration; the CPU tier has never loaded it, so the refill reads the
    disk."""
    disk = DiskAdapterCache(tmp_path / "disk")
    for i, a in enumerate(("a", "b", "c")):
        disk.add_adapter(a, _peft_dir(tmp_path / f"src_{a}", 2, i))
    store = CpuAdapterStore(disk_cache=disk, max_adapters=2, module_names=[m.name for m in MODS])
    cfg = PolyLoraConfig(max_gpu_adapters=1, max_rank=4)
    cache = GpuAdapterCache(store, MODS, cfg, torch.device("cpu"), torch.float32)
    cache.ensure_resident(["a"])
    slot = cache.adapter_to_slot["a"]
    # truncate c's weights on disk
    path = disk.get("c").path
    f = next(p for p in path.iterdir() if p.suffix == ".safetensors")
    f.write_bytes(f.read_bytes()[:40])
    with pytest.raises(Exception):
        cache.ensure_resident(["c"])
    assert cache.slot_to_adapter[slot] is None and "a" not in cache.adapter_to_slot
    for m in MODS:
        assert int(cache.ranks[m.name][slot]) == 0 and float(cache.scales[m.name][slot]) == 0.0
    # an intact adapter still loads into the freed slot with its own weights
    wi = cache.ensure_resident(["b"])
    assert wi.tolist() == [slot]
    _assert_slot_holds(cache, store, "b")
