"""Generates the golden fixtures of tests/golden/ by running the REFERENCE.

Run in a container where the reference checkout is available:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py <reference>/src

It imports the reference package ``polylora`` and records, on seeded inputs,
the outputs of:

* ``_build_flat_schedule`` (src/polylora/sgmv.py:29-61)      -> flat_schedule.npz
* ``MultiLoraLinear._reference_forward`` (layers.py:112-134) -> reference_forward.npz
* ``GpuAdapterCache.ensure_resident`` sequences (cache.py)    -> slot_sequences.json
  (run with PYTHONHASHSEED=0; the script re-executes itself to set it)
* PEFT parsing + disk manifest (store.py)                     -> peft_store.npz / manifest.json
* CpuAdapterStore's in-memory LRU sequences (store.py)        -> cpu_lru_sequences.json
* DiskAdapterCache operation sequences (store.py)             -> disk_sequences.json
* a tiny DeBERTa ``PolyLoraModel`` CPU forward (model.py)     -> model_tiny.pt

Nothing under tests/ reads the reference at run time; only these files.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _import_reference(src: str):
    sys.path.insert(0, src)
    import polylora  # noqa: F401
    from polylora import cache, layers, model, sgmv, store  # noqa: F401

    return polylora


# ------------------------------------------------------------------ schedule
def gen_flat_schedule(sgmv) -> None:
    rng = np.random.default_rng(1)
    cases = {}
    specs = [
        ("tokens", 64, 1, 16, 256),
        ("rows", 33, 200, 16, 256),
        ("rows_a", 17, 77, 16, 16),
        ("unit", 9, 9, 1, 1),
        ("big", 3000, 40, 16, 256),
    ]
    for name, B, max_len, bm, bn in specs:
        seq = rng.integers(0, max_len + 1, size=B).astype(np.int32)
        n_eff = np.where(rng.random(B) < 0.3, 0, rng.choice([16, 256, 4096, 300], size=B)).astype(np.int32)
        cum, nn, total = sgmv._build_flat_schedule(torch.from_numpy(seq), torch.from_numpy(n_eff), bm, bn)
        cases[f"{name}__seq"] = seq
        cases[f"{name}__neff"] = n_eff
        cases[f"{name}__blocks"] = np.array([bm, bn], dtype=np.int32)
        cases[f"{name}__cum"] = cum.numpy()
        cases[f"{name}__nn"] = nn.numpy()
        cases[f"{name}__total"] = np.array([total], dtype=np.int64)
    np.savez_compressed(OUT / "flat_schedule.npz", **cases)


# ------------------------------------------------------------------ _reference_forward
class _FakeCache:
    def __init__(self, A, B, ranks, scales, use_triton=False):
        self.A = {"m": A}
        self.B = {"m": B}
        self.ranks = {"m": ranks}
        self.scales = {"m": scales}


def _lora_case(rng, B, M, K, N, ns, R, rank_choices, dtype, base_frac=0.2, min_len=0):
    ranks = np.array([0] + list(rng.choice(rank_choices, size=ns - 1)), dtype=np.int32)
    A = np.zeros((ns, K, R), dtype=np.float32)
    Bw = np.zeros((ns, R, N), dtype=np.float32)
    for s in range(1, ns):
        r = int(ranks[s])
        A[s, :, :r] = rng.uniform(-1 / 64, 1 / 64, size=(K, r))
        Bw[s, :r, :] = rng.normal(0, 0.02, size=(r, N))
    scales = np.array([0.0] + [16.0 / r if r else 0.0 for r in ranks[1:]], dtype=np.float32)
    x = rng.normal(0, 1, size=(B, M, K)).astype(np.float32)
    y = rng.normal(0, 1, size=(B, M, N)).astype(np.float32)
    seq = rng.integers(min_len, M + 1, size=B).astype(np.int32)
    wi = rng.integers(1, ns, size=B).astype(np.int64)
    wi[rng.random(B) < base_frac] = 0
    tdt = {"float32": torch.float32, "bfloat16": torch.bfloat16}[dtype]
    cast = lambda a: torch.from_numpy(a).to(tdt)  # noqa: E731
    return dict(x=cast(x), y=cast(y), A=cast(A), B=cast(Bw), ranks=torch.from_numpy(ranks),
                scales=torch.from_numpy(scales), seq=torch.from_numpy(seq), wi=torch.from_numpy(wi))


def gen_reference_forward(layers) -> None:
    rng = np.random.default_rng(2)
    specs = [
        # name, B, M, K, N, num_slots, R, ranks, dtype
        ("cfg1_rows_f32", 8, 32, 64, 48, 5, 16, [4, 8, 8, 16], "float32"),
        ("tokens_f32", 64, 1, 128, 96, 9, 16, [0, 4, 8, 16], "float32"),
        ("odd_rank_f32", 6, 7, 40, 24, 4, 3, [1, 2, 3], "float32"),
        ("rows_bf16", 8, 32, 256, 128, 5, 16, [4, 8, 16], "bfloat16"),
        ("tokens_bf16", 96, 1, 512, 256, 17, 16, [0, 4, 8, 16], "bfloat16"),
        ("rank64_bf16", 12, 8, 256, 192, 7, 64, [8, 16, 32, 64], "bfloat16"),
    ]
    out = {}
    for name, B, M, K, N, ns, R, rc, dt in specs:
        c = _lora_case(rng, B, M, K, N, ns, R, rc, dt)
        lin = layers.MultiLoraLinear(torch.nn.Linear(K, N), "m", _FakeCache(c["A"], c["B"], c["ranks"], c["scales"]))
        res = lin._reference_forward(c["x"], c["y"], c["seq"], c["wi"])
        for key in ("x", "y", "A", "B"):
            out[f"{name}__{key}"] = c[key].float().numpy()
        out[f"{name}__ranks"] = c["ranks"].numpy()
        out[f"{name}__scales"] = c["scales"].numpy()
        out[f"{name}__seq"] = c["seq"].numpy()
        out[f"{name}__wi"] = c["wi"].numpy()
        out[f"{name}__out"] = res.float().numpy()
        out[f"{name}__dtype"] = np.array([dt])
    np.savez_compressed(OUT / "reference_forward.npz", **out)


# ------------------------------------------------------------------ slot sequences
def gen_slot_sequences(polylora) -> None:
    if os.environ.get("PYTHONHASHSEED") != "0":
        env = dict(os.environ, PYTHONHASHSEED="0")
        subprocess.run([sys.executable, __file__, sys.argv[1], "--slots-only"], check=True, env=env)
        return
    from polylora.cache import GpuAdapterCache, ModuleSpec
    from polylora.config import PolyLoraConfig
    from polylora.store import CpuAdapterStore, CpuLayerWeights

    rng = np.random.default_rng(3)
    scenarios = []
    for sc, (n_adapters, max_gpu, n_batches, batch) in enumerate([(6, 3, 40, 4), (12, 4, 60, 6), (3, 1, 12, 2)]):
        cfg = PolyLoraConfig(max_gpu_adapters=max_gpu, max_rank=4, use_triton_kernels=False)
        store = CpuAdapterStore()
        ids = [f"ad{i:02d}" for i in range(n_adapters)]
        for i, a in enumerate(ids):
            r = 1 + i % 4
            store.add_adapter(a, {"m": CpuLayerWeights(torch.zeros(8, r), torch.zeros(r, 8), r, 1.0)})
        cache = GpuAdapterCache(store, [ModuleSpec("m", 8, 8)], cfg, torch.device("cpu"), torch.float32)
        steps = []
        for _ in range(n_batches):
            k = int(rng.integers(1, max_gpu + 1))
            pool = list(rng.choice(ids, size=k, replace=False))
            row_ids = [str(pool[j]) if rng.random() > 0.25 else "__base__" for j in rng.integers(0, k, size=batch)]
            wi = cache.ensure_resident(row_ids).tolist()
            steps.append({
                "adapter_ids": row_ids,
                "weight_indices": wi,
                "slot_to_adapter": list(cache.slot_to_adapter),
                "lru": list(cache.lru.keys()),
                "ranks": cache.ranks["m"].tolist(),
            })
        scenarios.append({"n_adapters": n_adapters, "max_gpu": max_gpu, "ids": ids, "steps": steps})
    # error messages
    cfg = PolyLoraConfig(max_gpu_adapters=1, max_rank=4, use_triton_kernels=False)
    store = CpuAdapterStore()
    for a in ("a", "b"):
        store.add_adapter(a, {"m": CpuLayerWeights(torch.zeros(8, 2), torch.zeros(2, 8), 2, 1.0)})
    cache = GpuAdapterCache(store, [ModuleSpec("m", 8, 8)], cfg, torch.device("cpu"), torch.float32)
    errors = {}
    for label, ids in (("unknown", ["zz"]), ("capacity", ["a", "b"])):
        try:
            cache.ensure_resident(ids)
        except Exception as exc:  # noqa: BLE001
            errors[label] = [type(exc).__name__, str(exc)]
    (OUT / "slot_sequences.json").write_text(json.dumps({"hashseed": 0, "scenarios": scenarios, "errors": errors}, indent=1))


# ------------------------------------------------------------------ PEFT store + manifest
def gen_peft_store(polylora) -> None:
    from polylora.store import CpuAdapterStore, DiskAdapterCache

    g = torch.Generator().manual_seed(4)
    modules = ["encoder.layer.0.attention.self.query_proj", "encoder.layer.0.attention.self.value_proj",
               "encoder.layer.0.output.dense"]
    sd = {}
    for m, (inn, out, r) in zip(modules, [(32, 32, 2), (32, 32, 3), (64, 32, 2)]):
        sd[f"base_model.model.{m}.lora_A.adp.weight"] = torch.randn(r, inn, generator=g)
        sd[f"base_model.model.{m}.lora_B.adp.weight"] = torch.randn(out, r, generator=g)
    store = CpuAdapterStore()
    store.add_adapter_from_peft_state_dict("adp", sd, modules + ["encoder.layer.0.attention.self.key_proj"], 6.0, "adp")
    out = {}
    for m, w in store.adapters["adp"].layers.items():
        out[f"{m}__A"] = w.A.numpy()
        out[f"{m}__B"] = w.B.numpy()
        out[f"{m}__rank"] = np.array([w.rank])
        out[f"{m}__scale"] = np.array([w.scale])
    for k, v in sd.items():
        out[f"sd__{k}"] = v.numpy()
    np.savez_compressed(OUT / "peft_store.npz", **out)
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        cache = DiskAdapterCache(tmp / "cache", max_adapters=2)
        for name in ("alpha", "b/eta", "gamma"):
            d = tmp / f"src_{name.replace('/', '_')}"
            d.mkdir()
            (d / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 4, "r": 2}))
            torch.save({}, d / "adapter_model.bin")
            cache.add_adapter(name, d, "default")
        cache.get("b/eta")
        (OUT / "manifest.json").write_text((tmp / "cache" / "manifest.json").read_text())


# ------------------------------------------------------------------ tiny model
def _tiny_deberta(seed: int):
    from transformers import DebertaV2Config, DebertaV2Model

    torch.manual_seed(seed)
    cfg = DebertaV2Config(vocab_size=97, hidden_size=32, num_hidden_layers=1, num_attention_heads=4,
                          intermediate_size=64, hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0,
                          max_position_embeddings=32, relative_attention=False, type_vocab_size=0)
    return DebertaV2Model(cfg).eval(), cfg.to_dict()


def _write_adapter_dir(path: Path, modules, r: int, alpha: float, seed: int, fmt: str, subset=None):
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for name, (inn, out) in modules.items():
        if subset is not None and not any(name.endswith(s) for s in subset):
            continue
        sd[f"base_model.model.{name}.lora_A.weight"] = torch.randn(r, inn, generator=g) * 0.3
        sd[f"base_model.model.{name}.lora_B.weight"] = torch.randn(out, r, generator=g) * 0.3
    path.mkdir(parents=True)
    (path / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "r": r, "lora_alpha": alpha,
                                                          "lora_dropout": 0.0}))
    if fmt == "safetensors":
        from safetensors.torch import save_file

        save_file(sd, str(path / "adapter_model.safetensors"))
    else:
        torch.save(sd, path / "adapter_model.bin")
    return sd


def gen_model_tiny(polylora) -> None:
    from polylora import PolyLoraConfig, PolyLoraModel

    base, cfg_dict = _tiny_deberta(0)
    targets = ["query_proj", "key_proj", "value_proj", "dense"]
    modules = {n: (m.in_features, m.out_features) for n, m in base.named_modules()
               if isinstance(m, torch.nn.Linear) and any(n.endswith("." + t) for t in targets)}
    input_ids = torch.tensor([[1, 5, 6, 7, 2, 0], [1, 8, 9, 4, 3, 2], [1, 11, 12, 13, 14, 2], [1, 3, 3, 2, 0, 0]])
    attention_mask = torch.tensor([[1, 1, 1, 1, 1, 0], [1, 1, 1, 1, 1, 1], [1, 1, 1, 1, 1, 1], [1, 1, 1, 1, 0, 0]])
    adapter_ids = ["a", "b", "__base__", "c"]
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        sds = {
            "a": _write_adapter_dir(tmp / "a", modules, 2, 8.0, 10, "bin"),
            "b": _write_adapter_dir(tmp / "b", modules, 3, 6.0, 11, "safetensors"),
            "c": _write_adapter_dir(tmp / "c", modules, 4, 8.0, 12, "bin", subset=["value_proj"]),
        }
        model = PolyLoraModel(_tiny_deberta(0)[0], PolyLoraConfig(max_gpu_adapters=3, max_rank=4,
                                                                  target_modules=targets,
                                                                  use_triton_kernels=False)).eval()
        for a in ("a", "b", "c"):
            model.load_adapter_from_disk(a, str(tmp / a))
        with torch.inference_mode():
            lora_out = model(input_ids=input_ids, attention_mask=attention_mask, adapter_ids=adapter_ids).last_hidden_state
            base_out = base(input_ids=input_ids, attention_mask=attention_mask).last_hidden_state
    torch.save({
        "config": cfg_dict,
        "state_dict": base.state_dict(),
        "targets": targets,
        "modules": modules,
        "adapters": {k: {"sd": v, "r": r, "alpha": al} for (k, v), (r, al) in zip(sds.items(), [(2, 8.0), (3, 6.0), (4, 8.0)])},
        "input_ids": input_ids,
        "attention_mask": attention_mask,
        "adapter_ids": adapter_ids,
        "lora_out": lora_out,
        "base_out": base_out,
        "target_module_names": list(model.target_module_names),
    }, OUT / "model_tiny.pt")


def gen_cpu_lru_sequences(polylora) -> None:
    """CpuAdapterStore's in-memory LRU (store.py:184-219, 425-436) on seeded
    random operation sequences: outcome and resident order after each op."""
    from polylora.store import CpuAdapterStore, CpuLayerWeights

    rng = np.random.default_rng(11)
    ids = [f"a{i}" for i in range(6)] + ["__base__"]
    layers = {"m": CpuLayerWeights(torch.ones(4, 2), torch.ones(2, 4), 2, 1.0)}
    sequences = []
    for _ in range(60):
        cap = [None, 1, 2, 3, 4][int(rng.integers(0, 5))]
        store = CpuAdapterStore(max_adapters=cap)
        steps = []
        for _ in range(int(rng.integers(1, 26))):
            kind = ["add", "get", "touch", "exclude"][int(rng.integers(0, 4))]
            arg = sorted({ids[int(i)] for i in rng.integers(0, len(ids), int(rng.integers(0, 5)))}) if kind == "exclude" \
                else ids[int(rng.integers(0, len(ids)))]
            try:
                if kind == "add":
                    store.add_adapter(arg, layers)
                elif kind == "get":
                    store.get(arg)
                elif kind == "touch":
                    store.touch(arg)
                else:
                    store.set_eviction_exclusions(set(arg))
                outcome = ["ok"]
            except (KeyError, ValueError, RuntimeError) as exc:
                outcome = [type(exc).__name__, str(exc)]
            steps.append({"op": kind, "arg": arg, "outcome": outcome, "resident": list(store.adapters)})
        sequences.append({"max_adapters": cap, "steps": steps})
    (OUT / "cpu_lru_sequences.json").write_text(json.dumps(sequences, separators=(",", ":")))


DISK_IDS = ["a", "b", "c/d", "e f", "ünï", "__x"]


def make_disk_sources(root: Path) -> list[Path]:
    """Three valid PEFT directories and one without weights."""
    srcs = []
    for i in range(4):
        d = root / f"src{i}"
        d.mkdir(parents=True, exist_ok=True)
        (d / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "lora_alpha": 4, "r": 2}))
        if i < 3:
            (d / "adapter_model.bin").write_bytes(b"weights-%d" % i)
        srcs.append(d)
    return srcs


def gen_disk_sequences(polylora) -> None:
    """DiskAdapterCache (store.py:36-148) on seeded random operation sequences:
    outcome, entry order, directories on disk and manifest text after each op
    ("reopen" builds a new cache over the same directory)."""
    from polylora.store import DiskAdapterCache

    rng = np.random.default_rng(12)
    sequences = []
    for _ in range(30):
        cap = [None, 1, 2, 3][int(rng.integers(0, 4))]
        with tempfile.TemporaryDirectory() as tmp:
            srcs = make_disk_sources(Path(tmp) / "sources")
            cache_dir = Path(tmp) / "cache"
            cache = DiskAdapterCache(cache_dir, max_adapters=cap)
            steps = []
            for _ in range(int(rng.integers(1, 16))):
                kind = ["add", "add", "get", "touch", "reopen"][int(rng.integers(0, 5))]
                ident = int(rng.integers(0, len(DISK_IDS)))
                src = int(rng.integers(0, len(srcs)))
                name = ["default", "other"][int(rng.integers(0, 2))]
                try:
                    if kind == "add":
                        cache.add_adapter(DISK_IDS[ident], srcs[src], name)
                    elif kind == "get":
                        cache.get(DISK_IDS[ident])
                    elif kind == "touch":
                        cache.touch(DISK_IDS[ident])
                    else:
                        cache = DiskAdapterCache(cache_dir, max_adapters=cap)
                    outcome = ["ok"]
                except (KeyError, FileNotFoundError, RuntimeError) as exc:
                    outcome = [type(exc).__name__, str(exc).replace(str(srcs[src]), "<src>")]
                manifest = cache_dir / "manifest.json"
                steps.append({"op": kind, "id": ident, "src": src, "name": name, "outcome": outcome,
                              "entries": list(cache.entries),
                              "dirs": sorted(p.name for p in cache_dir.iterdir() if p.is_dir()),
                              "manifest": manifest.read_text() if manifest.exists() else None})
            sequences.append({"max_adapters": cap, "steps": steps})
    (OUT / "disk_sequences.json").write_text(json.dumps(sequences, separators=(",", ":")))


def main() -> None:
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("POLYLORA_REFERENCE_SRC", "")
    polylora = _import_reference(src)
    if "--slots-only" in sys.argv:
        gen_slot_sequences(polylora)
        return
    if "--lru-only" in sys.argv:
        gen_cpu_lru_sequences(polylora)
        return
    if "--disk-only" in sys.argv:
        gen_disk_sequences(polylora)
        return
    from polylora import layers, sgmv

    gen_flat_schedule(sgmv)
    gen_reference_forward(layers)
    gen_slot_sequences(polylora)
    gen_peft_store(polylora)
    gen_cpu_lru_sequences(polylora)
    gen_disk_sequences(polylora)
    gen_model_tiny(polylora)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
