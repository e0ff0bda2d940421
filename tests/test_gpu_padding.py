"""The device-side right-padding check (plora_check_right_padded and
PolyLoraConfig(right_padding_check="device")).

The reference checks the attention mask with a host comparison
(src/polylora/context.py:37-45), which makes every forward wait for the
device.  The device check enqueues a kernel instead and records a violation in
the library's device status word.  These tests compare it with the host check
(assert_right_padded) on the same masks: every dtype a mask comes in, holes,
values other than 0/1, negative zeros, and rows of length 0 and width.
"""

import copy

import numpy as np
import pytest
import torch

from polylora_b200 import PolyLoraConfig, PolyLoraModel
from polylora_b200 import _native
from polylora_b200.context import assert_right_padded

pytestmark = pytest.mark.gpu

DTYPES = [torch.bool, torch.uint8, torch.int32, torch.int64, torch.float16, torch.bfloat16, torch.float32,
          torch.float64]


def _masks(seed, rows=37, width=53):
    """Right-padded rows, then the same rows with one defect each."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, width + 1, size=rows)
    lens[0], lens[1] = 0, width
    good = (np.arange(width)[None, :] < lens[:, None]).astype(np.int64)
    bad = []
    for kind in ("hole", "left", "two", "tail"):
        m = good.copy()
        r = int(rng.integers(2, rows))
        if kind == "hole" and lens[r] >= 2:
            m[r, int(rng.integers(0, lens[r] - 1))] = 0
        elif kind == "left":
            m[r] = m[r][::-1]
            if lens[r] in (0, width):
                m[r, 0], m[r, -1] = 0, 1
        elif kind == "two":
            m[r, 0] = 2  # bool() is true, but the row sum counts it twice
        else:
            m[r, -1] = 1 if lens[r] < width - 1 else m[r, -1]
        bad.append(m)
    return good, bad


def _host_ok(mask):
    try:
        assert_right_padded(mask, mask.to(torch.int32).sum(-1))
        return True
    except ValueError:
        return False


def _device_flag(mask):
    _native.device_status(clear=True)
    _native.check_right_padded(mask, mask.to(torch.int32).sum(-1))
    return bool(_native.device_status(clear=True) & _native.DEV_PADDING)


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
def test_device_check_matches_host_check(dtype):
    good, bad = _masks(DTYPES.index(dtype))
    for m in [good] + bad:
        mask = torch.from_numpy(m).to("cuda").to(dtype)
        assert _device_flag(mask) == (not _host_ok(mask)), (dtype, m.tolist())
    assert not _device_flag(torch.from_numpy(good).to("cuda").to(dtype))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32, torch.float64], ids=str)
def test_negative_zero_counts_as_padding(dtype):
    mask = torch.tensor([[1.0, 1.0, -0.0, -0.0], [1.0, -0.0, 0.0, 0.0]], dtype=dtype, device="cuda")
    assert _host_ok(mask) and not _device_flag(mask)


def test_empty_and_degenerate_shapes():
    assert not _device_flag(torch.zeros(0, 5, dtype=torch.int64, device="cuda"))
    assert not _device_flag(torch.zeros(3, 0, dtype=torch.int64, device="cuda"))
    assert not _device_flag(torch.zeros(3, 4, dtype=torch.int64, device="cuda"))
    with pytest.raises(ValueError, match="2D"):
        _native.check_right_padded(torch.ones(2, 2, 2, device="cuda"), torch.ones(2, device="cuda"))


def _tiny_model(check):
    from transformers import DebertaV2Config, DebertaV2Model

    torch.manual_seed(0)
    cfg = DebertaV2Config(vocab_size=50, hidden_size=32, num_hidden_layers=1, num_attention_heads=4,
                          intermediate_size=64, hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0,
                          max_position_embeddings=32, relative_attention=False, type_vocab_size=0)
    base = DebertaV2Model(cfg).eval().cuda()
    model = PolyLoraModel(copy.deepcopy(base), PolyLoraConfig(target_modules=["query_proj", "value_proj"],
                                                              max_gpu_adapters=2, max_rank=4,
                                                              right_padding_check=check)).eval()
    return model


def test_model_device_check_defers_the_reference_error():
    model = _tiny_model("device")
    ids = torch.tensor([[1, 5, 6, 2], [1, 8, 9, 2]], device="cuda")
    good = torch.tensor([[1, 1, 1, 0], [1, 1, 0, 0]], device="cuda")
    left = torch.tensor([[0, 1, 1, 1], [1, 1, 0, 0]], device="cuda")
    _native.device_status(clear=True)
    with torch.inference_mode():
        model(input_ids=ids, attention_mask=good, adapter_ids=["__base__", "__base__"])
        model.raise_for_device_status()  # nothing recorded
        model(input_ids=ids, attention_mask=left, adapter_ids=["__base__", "__base__"])  # does not raise here
    with pytest.raises(ValueError, match="right-padded attention_mask"):
        model.raise_for_device_status()
    model.raise_for_device_status()  # the read cleared the word


def test_model_host_check_raises_in_the_forward():
    model = _tiny_model("host")
    ids = torch.tensor([[1, 5, 6, 2]], device="cuda")
    with torch.inference_mode(), pytest.raises(ValueError, match="right-padded attention_mask"):
        model(input_ids=ids, attention_mask=torch.tensor([[0, 1, 1, 1]], device="cuda"), adapter_ids=["__base__"])
