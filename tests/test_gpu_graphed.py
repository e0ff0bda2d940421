"""GraphedForward: a PolyLoraModel decode forward captured once and replayed
with new inputs and adapter assignments gives the eager forward's output."""

import pytest
import torch

from polylora_b200 import PolyLoraConfig, PolyLoraModel
from polylora_b200.graphed import GraphedForward
from polylora_b200.store import CpuLayerWeights

pytestmark = pytest.mark.gpu

TARGETS = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


def _small_llama(dev):
    from transformers import LlamaConfig, LlamaModel

    cfg = LlamaConfig(vocab_size=1000, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64, use_cache=False)
    torch.manual_seed(0)
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            return LlamaModel(cfg).eval()
    finally:
        torch.set_default_dtype(torch.float32)


def _model(dev, adapters=4, slots=3):
    base = _small_llama(dev)
    shapes = {n: (m.in_features, m.out_features) for n, m in base.named_modules()
              if isinstance(m, torch.nn.Linear) and any(n.endswith("." + t) for t in TARGETS)}
    model = PolyLoraModel(base, PolyLoraConfig(max_gpu_adapters=slots, max_rank=16, target_modules=TARGETS,
                                               enforce_right_padding=False))
    g = torch.Generator().manual_seed(1)
    for a in range(adapters):
        r = [4, 8, 16, 16][a % 4]
        layers = {name: CpuLayerWeights(A=torch.randn(k, r, generator=g) * 0.1, B=torch.randn(r, n, generator=g) * 0.1,
                                        rank=r, scale=2.0)
                  for name, (k, n) in shapes.items()}
        model.adapter_store.add_adapter(f"a{a}", layers)
    return model


def test_graphed_decode_matches_eager_across_refills(cuda_status_clean):
    dev = torch.device("cuda")
    model = _model(dev)
    g = torch.Generator(device=dev).manual_seed(2)
    ids1 = ["a0", "a1", "__base__", "a2", "a0", "a1", "a2", "__base__"]
    x1 = torch.randint(0, 1000, (8, 1), device=dev, generator=g)
    with torch.inference_mode():
        graphed = GraphedForward(model, ids1, input_ids=x1)
        got1 = graphed(ids1, input_ids=x1).clone()
        ref1 = model(input_ids=x1, adapter_ids=ids1).last_hidden_state
    torch.testing.assert_close(got1, ref1, rtol=0, atol=0)
    # a3 is not resident: the call evicts one slot and refills it before the replay
    ids2 = ["a3", "__base__", "a1", "a3", "a1", "a3", "__base__", "a1"]
    x2 = torch.randint(0, 1000, (8, 1), device=dev, generator=g)
    with torch.inference_mode():
        got2 = graphed(ids2, input_ids=x2).clone()
        ref2 = model(input_ids=x2, adapter_ids=ids2).last_hidden_state
        base2 = model.base_model(input_ids=x2).last_hidden_state
    torch.testing.assert_close(got2, ref2, rtol=0, atol=0)
    assert not torch.equal(got2, base2)  # the adapters did act


def test_graphed_unpadded_prefill_matches_eager(cuda_status_clean):
    """Several tokens per row, no attention mask: the capture skips the causal
    mask as eager mode does (SDPA's own causal path, not an explicit mask), so
    replay and eager agree bit for bit."""
    dev = torch.device("cuda")
    model = _model(dev)
    g = torch.Generator(device=dev).manual_seed(3)
    ids = ["a0", "__base__", "a1", "a2"]
    x = torch.randint(0, 1000, (4, 16), device=dev, generator=g)
    with torch.inference_mode():
        graphed = GraphedForward(model, ids, input_ids=x)
        ref = model(input_ids=x, adapter_ids=ids).last_hidden_state
        for _ in range(2):
            got = graphed(ids, input_ids=x).clone()
            torch.testing.assert_close(got, ref, rtol=0, atol=0)
