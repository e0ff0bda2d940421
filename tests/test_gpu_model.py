"""Model-level behaviour on the GPU, re-expressing the reference's PEFT-parity
tests (tests/test_polylora_peft.py of the reference) without PEFT: adapters are
written as PEFT-format directories, and outputs are compared with the
reference's own CPU forward (golden model_tiny.pt) and with the closed form.

Base-model arithmetic differs between CPU (golden) and GPU, so the golden
comparison uses atol = rtol = 1e-4; comparisons made on the same device use
the reference tests' 1e-5.
"""

import copy
import json
from pathlib import Path

import pytest
import torch

from polylora_b200 import PolyLoraConfig, PolyLoraModel

pytestmark = pytest.mark.gpu

TARGETS = ["query_proj", "key_proj", "value_proj", "dense"]


def _tiny_deberta(seed: int, vocab: int = 97):
    from transformers import DebertaV2Config, DebertaV2Model

    torch.manual_seed(seed)
    cfg = DebertaV2Config(vocab_size=vocab, hidden_size=32, num_hidden_layers=1, num_attention_heads=4,
                          intermediate_size=64, hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0,
                          max_position_embeddings=32, relative_attention=False, type_vocab_size=0)
    return DebertaV2Model(cfg).eval()


def _linear_modules(model, targets=None):
    return {n: (m.in_features, m.out_features) for n, m in model.named_modules()
            if isinstance(m, torch.nn.Linear) and (targets is None or any(n == t or n.endswith("." + t) for t in targets))}


def _write_adapter(path: Path, sd: dict, r: int, alpha: float, fmt: str = "bin") -> Path:
    path.mkdir(parents=True, exist_ok=True)
    (path / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "r": r, "lora_alpha": alpha, "lora_dropout": 0.0}))
    if fmt == "safetensors":
        from safetensors.torch import save_file

        save_file(sd, str(path / "adapter_model.safetensors"))
    else:
        torch.save(sd, path / "adapter_model.bin")
    return path


def _random_adapter(modules, r, seed, subset=None, scale=0.3):
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for name, (inn, out) in modules.items():
        if subset is not None and not any(name.endswith(s) for s in subset):
            continue
        sd[f"base_model.model.{name}.lora_A.weight"] = torch.randn(r, inn, generator=g) * scale
        sd[f"base_model.model.{name}.lora_B.weight"] = torch.randn(out, r, generator=g) * scale
    return sd


def _closed_form_model(base, adapters_by_row, x_kwargs):
    """Runs `base` with forward hooks adding (alpha/r) x A^T B^T per row — the
    PEFT arithmetic restated — on the same device, to the valid (unpadded)
    tokens of each row as the reference does (layers.py:127-133)."""
    hooks = []
    mask = x_kwargs.get("attention_mask")
    lens = mask.sum(-1).tolist() if mask is not None else None

    def make_hook(name):
        def hook(mod, inp, out):
            x = inp[0]
            out = out.clone()
            for b, ad in enumerate(adapters_by_row):
                if ad is None or name not in ad["layers"]:
                    continue
                A, B, s = ad["layers"][name]
                L = x.shape[1] if lens is None else int(lens[b])
                out[b, :L] = out[b, :L] + s * (x[b, :L] @ A.t().to(x) @ B.t().to(x))
            return out
        return hook

    for name, mod in base.named_modules():
        if isinstance(mod, torch.nn.Linear):
            hooks.append(mod.register_forward_hook(make_hook(name)))
    try:
        with torch.inference_mode():
            return base(**x_kwargs).last_hidden_state
    finally:
        for h in hooks:
            h.remove()


def _layers_from_sd(sd, alpha):
    layers = {}
    for k, v in sd.items():
        if ".lora_A." in k:
            name = k.split(".lora_A.")[0].replace("base_model.model.", "")
            b = sd[k.replace(".lora_A.", ".lora_B.")]
            layers[name] = (v, b, alpha / v.shape[0])
    return {"layers": layers}


def test_mixed_batch_matches_reference_golden(golden_dir, tmp_path, cuda_status_clean):
    from transformers import DebertaV2Config, DebertaV2Model

    g = torch.load(golden_dir / "model_tiny.pt", weights_only=False)
    base = DebertaV2Model(DebertaV2Config.from_dict(g["config"])).eval()
    base.load_state_dict(g["state_dict"])
    base = base.cuda()
    model = PolyLoraModel(copy.deepcopy(base), PolyLoraConfig(max_gpu_adapters=3, max_rank=4, target_modules=g["targets"])).eval()
    assert model.target_module_names == g["target_module_names"]
    for name, ad in g["adapters"].items():
        fmt = "safetensors" if name == "b" else "bin"
        model.load_adapter_from_disk(name, str(_write_adapter(tmp_path / name, ad["sd"], ad["r"], ad["alpha"], fmt)))
    inputs = dict(input_ids=g["input_ids"].cuda(), attention_mask=g["attention_mask"].cuda())
    with torch.inference_mode():
        out = model(**inputs, adapter_ids=g["adapter_ids"]).last_hidden_state
        base_out = base(**inputs).last_hidden_state
    torch.testing.assert_close(out.cpu(), g["lora_out"], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(out[2], base_out[2], atol=1e-5, rtol=1e-5)  # __base__ row
    # same-device closed form at the reference tests' tolerance
    rows = [_layers_from_sd(g["adapters"][a]["sd"], g["adapters"][a]["alpha"]) if a != "__base__" else None
            for a in g["adapter_ids"]]
    rows = [None if r is None else {"layers": {k: tuple(t.cuda() if torch.is_tensor(t) else t for t in v)
                                               for k, v in r["layers"].items()}} for r in rows]
    expected = _closed_form_model(copy.deepcopy(base), rows, inputs)
    torch.testing.assert_close(out, expected, atol=1e-5, rtol=1e-5)


def test_gpu_cache_reloads_from_cpu_cache(cuda_status_clean):
    base = _tiny_deberta(1).cuda()
    modules = _linear_modules(base, TARGETS)
    model = PolyLoraModel(copy.deepcopy(base), PolyLoraConfig(target_modules=TARGETS, max_gpu_adapters=1,
                                                               max_cpu_adapters=2, max_rank=2)).eval()
    for name, seed in (("a", 5), ("b", 6)):
        model.adapter_store.add_adapter_from_peft_state_dict(name, _random_adapter(modules, 2, seed), model.target_module_names, 4.0)
    sample = dict(input_ids=torch.tensor([[1, 5, 6, 2]]).cuda(), attention_mask=torch.ones(1, 4, dtype=torch.long).cuda())
    with torch.inference_mode():
        out_a1 = model(**sample, adapter_ids=["a"]).last_hidden_state.clone()
        assert model.adapter_cache.slot_to_adapter[1] == "a"
        out_b = model(**sample, adapter_ids=["b"]).last_hidden_state.clone()
        assert model.adapter_cache.slot_to_adapter[1] == "b"
        out_a2 = model(**sample, adapter_ids=["a"]).last_hidden_state.clone()
        assert model.adapter_cache.slot_to_adapter[1] == "a"
    assert "a" in model.adapter_store and "b" in model.adapter_store
    assert not torch.allclose(out_a1, out_b, atol=1e-5, rtol=1e-5)
    assert torch.equal(out_a1, out_a2)
    assert model.adapter_cache.stats["evictions"] == 2


def test_base_adapter_uses_slot_zero_rank_zero(cuda_status_clean):
    base = _tiny_deberta(2).cuda()
    modules = _linear_modules(base, TARGETS)
    model = PolyLoraModel(copy.deepcopy(base), PolyLoraConfig(target_modules=TARGETS, max_gpu_adapters=1, max_rank=2)).eval()
    model.adapter_store.add_adapter_from_peft_state_dict("a", _random_adapter(modules, 2, 7), model.target_module_names, 4.0)
    sample = dict(input_ids=torch.tensor([[1, 5, 6, 2], [1, 8, 9, 2]]).cuda(), attention_mask=torch.ones(2, 4, dtype=torch.long).cuda())
    with torch.inference_mode():
        mixed = model(**sample, adapter_ids=["__base__", "a"]).last_hidden_state
        plain = base(**sample).last_hidden_state
    assert model.adapter_cache.adapter_to_slot["__base__"] == 0
    for name in model.target_module_names:
        assert int(model.adapter_cache.ranks[name][0].item()) == 0
        assert float(model.adapter_cache.scales[name][0].item()) == 0.0
    torch.testing.assert_close(mixed[0], plain[0], atol=1e-5, rtol=1e-5)
    assert not torch.allclose(mixed[1], plain[1], atol=1e-5, rtol=1e-5)


def test_missing_layer_weights_are_rank_zero(cuda_status_clean):
    base = _tiny_deberta(4).cuda()
    modules = _linear_modules(base)  # target_modules=None wraps every Linear
    model = PolyLoraModel(copy.deepcopy(base), PolyLoraConfig(max_gpu_adapters=1, max_rank=2)).eval()
    sd = _random_adapter(modules, 2, 8, subset=["value_proj"])
    model.adapter_store.add_adapter_from_peft_state_dict("sparse", sd, model.target_module_names, 4.0)
    sample = dict(input_ids=torch.tensor([[1, 5, 6, 2], [1, 8, 9, 2]]).cuda(), attention_mask=torch.ones(2, 4, dtype=torch.long).cuda())
    with torch.inference_mode():
        actual = model(**sample, adapter_ids=["sparse", "sparse"]).last_hidden_state
    q = next(n for n in model.target_module_names if n.endswith("query_proj"))
    v = next(n for n in model.target_module_names if n.endswith("value_proj"))
    slot = model.adapter_cache.adapter_to_slot["sparse"]
    assert int(model.adapter_cache.ranks[q][slot].item()) == 0
    assert float(model.adapter_cache.scales[q][slot].item()) == 0.0
    assert int(model.adapter_cache.ranks[v][slot].item()) == 2
    ad = _layers_from_sd({k: t.cuda() for k, t in sd.items()}, 4.0)
    expected = _closed_form_model(copy.deepcopy(base), [ad, ad], sample)
    torch.testing.assert_close(actual, expected, atol=1e-5, rtol=1e-5)


def test_cpu_miss_reloads_adapter_from_disk_cache(tmp_path, cuda_status_clean):
    base = _tiny_deberta(7).cuda()
    modules = _linear_modules(base, TARGETS)
    model = PolyLoraModel(copy.deepcopy(base), PolyLoraConfig(target_modules=TARGETS, max_gpu_adapters=1, max_cpu_adapters=1,
                                                               disk_cache_dir=tmp_path / "disk", max_disk_adapters=2,
                                                               max_rank=2)).eval()
    sds = {a: _random_adapter(modules, 2, 20 + i) for i, a in enumerate("ab")}
    for a, sd in sds.items():
        model.load_adapter_from_disk(a, str(_write_adapter(tmp_path / f"src_{a}", sd, 2, 4.0)))
    assert "a" not in model.adapter_store.adapters and "a" in model.adapter_store
    sample = dict(input_ids=torch.tensor([[1, 5, 6, 2]]).cuda(), attention_mask=torch.ones(1, 4, dtype=torch.long).cuda())
    with torch.inference_mode():
        actual = model(**sample, adapter_ids=["a"]).last_hidden_state
    assert "a" in model.adapter_store.adapters
    assert model.adapter_cache.slot_to_adapter[1] == "a"
    ad = _layers_from_sd({k: t.cuda() for k, t in sds["a"].items()}, 4.0)
    torch.testing.assert_close(actual, _closed_form_model(copy.deepcopy(base), [ad], sample), atol=1e-5, rtol=1e-5)


def test_three_disk_adapters_batched_equal_per_row(tmp_path, cuda_status_clean):
    """Three PEFT adapters saved as adapter_model.bin (ranks 2/3/4, alpha
    4/9/8, as the reference's disk test): a right-padded mixed batch equals
    each row run alone with its adapter, and the closed form, at 1e-5."""
    base = _tiny_deberta(11).cuda()
    modules = _linear_modules(base, TARGETS)
    model = PolyLoraModel(copy.deepcopy(base), PolyLoraConfig(target_modules=TARGETS, max_gpu_adapters=3,
                                                               max_rank=4)).eval()
    spec = {"a": (2, 4.0), "b": (3, 9.0), "c": (4, 8.0)}
    sds = {a: _random_adapter(modules, r, 40 + i) for i, (a, (r, _)) in enumerate(spec.items())}
    for a, (r, alpha) in spec.items():
        model.load_adapter_from_disk(a, str(_write_adapter(tmp_path / a, sds[a], r, alpha, "bin")))
    ids = torch.randint(1, 97, (5, 9), generator=torch.Generator().manual_seed(3))
    mask = torch.ones(5, 9, dtype=torch.long)
    mask[1, 6:] = 0
    mask[3, 2:] = 0
    rows = ["c", "a", "b", "__base__", "a"]
    sample = dict(input_ids=ids.cuda(), attention_mask=mask.cuda())
    with torch.inference_mode():
        out = model(**sample, adapter_ids=rows).last_hidden_state
        for i, a in enumerate(rows):
            one = model(input_ids=ids[i:i + 1].cuda(), attention_mask=mask[i:i + 1].cuda(),
                        adapter_ids=[a]).last_hidden_state
            valid = mask[i].bool().cuda()
            torch.testing.assert_close(out[i][valid], one[0][valid], atol=1e-5, rtol=1e-5)
    ads = {a: _layers_from_sd({k: t.cuda() for k, t in sds[a].items()}, spec[a][1]) for a in spec}
    expected = _closed_form_model(copy.deepcopy(base), [ads.get(r) for r in rows], sample)
    valid = mask.bool().cuda()
    torch.testing.assert_close(out[valid], expected[valid], atol=1e-5, rtol=1e-5)


def test_bf16_model_matches_closed_form(cuda_status_clean):
    """bf16 weights take the tensor-core kernels (max_rank 16)."""
    base = _tiny_deberta(9).cuda().to(torch.bfloat16)
    modules = _linear_modules(base, TARGETS)
    model = PolyLoraModel(copy.deepcopy(base), PolyLoraConfig(target_modules=TARGETS, max_gpu_adapters=2, max_rank=16)).eval()
    sds = {"a": _random_adapter(modules, 8, 30, scale=0.1), "b": _random_adapter(modules, 16, 31, scale=0.1)}
    for a, sd in sds.items():
        model.adapter_store.add_adapter_from_peft_state_dict(a, sd, model.target_module_names, 16.0)
    ids = torch.randint(1, 97, (6, 16))
    mask = torch.ones(6, 16, dtype=torch.long)
    mask[1, 10:] = 0
    mask[4, 3:] = 0
    sample = dict(input_ids=ids.cuda(), attention_mask=mask.cuda())
    rows = ["a", "b", "__base__", "b", "a", "__base__"]
    with torch.inference_mode():
        out = model(**sample, adapter_ids=rows).last_hidden_state.float()
    ads = {a: _layers_from_sd({k: t.cuda().to(torch.bfloat16) for k, t in sd.items()}, 16.0) for a, sd in sds.items()}
    expected = _closed_form_model(copy.deepcopy(base), [ads.get(r) for r in rows], sample).float()
    plain = _closed_form_model(copy.deepcopy(base), [None] * 6, sample).float()
    valid = mask.bool().cuda()
    delta_scale = (expected - plain)[valid].abs().max()
    assert ((out - expected)[valid].abs().max() / delta_scale) < 0.1  # bf16 through 1 layer + norms
    assert torch.equal(out[2], plain[2]) or torch.allclose(out[2], plain[2], atol=1e-2)


def test_layouts_flattened_and_row0(cuda_status_clean):
    """The three input layouts of MultiLoraLinear (layers.py:82-110)."""
    from polylora_b200.cache import GpuAdapterCache, ModuleSpec
    from polylora_b200.context import LoraBatchContext, use_lora_context
    from polylora_b200.layers import MultiLoraLinear
    from polylora_b200.store import CpuAdapterStore, CpuLayerWeights

    torch.manual_seed(0)
    lin = torch.nn.Linear(64, 48).cuda()
    cfg = PolyLoraConfig(max_gpu_adapters=2, max_rank=16)
    store = CpuAdapterStore()
    A = torch.randn(64, 8) * 0.1
    B = torch.randn(8, 48) * 0.1
    store.add_adapter("a", {"m": CpuLayerWeights(A, B, 8, 2.0)})
    cache = GpuAdapterCache(store, [ModuleSpec("m", 64, 48)], cfg, torch.device("cuda"), torch.float32)
    layer = MultiLoraLinear(lin, "m", cache)
    wi = cache.ensure_resident(["a", "__base__", "a"])
    seq = torch.tensor([5, 5, 2], dtype=torch.int32, device="cuda")
    ctx = LoraBatchContext(["a", "__base__", "a"], wi, seq, table_ranks=cache.table_ranks, ready_event=cache.ready_event)
    x = torch.randn(3, 5, 64, device="cuda")
    delta = 2.0 * (x @ A.cuda() @ B.cuda())
    with torch.inference_mode(), use_lora_context(ctx):
        out3 = layer(x)
        out2 = layer(x.reshape(15, 64)).reshape(3, 5, 48)
        out1 = layer(x[:1])
    want = lin(x).detach().clone()
    want[0] += delta[0]
    want[2, :2] += delta[2, :2]
    for got in (out3, out2):
        torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(out1[0], want[0], atol=1e-5, rtol=1e-5)
