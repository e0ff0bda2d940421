"""eager_mask_decisions: while a CUDA stream captures a batch given neither a
padding mask nor position ids, transformers' mask helpers reach the decisions
eager mode reaches by reading tensor values (no packed sequences; the causal
mask skipped for one query or as many queries as keys).  Everything else runs
the helpers unchanged, and they are restored afterwards.  Capture is simulated
here by making torch's capture test answer yes (no GPU)."""

import pytest
import torch

masking_utils = pytest.importorskip("transformers.masking_utils")
import_utils = pytest.importorskip("transformers.utils.import_utils")

from polylora_b200.graphed import eager_mask_decisions  # noqa: E402

ARANGE = torch.arange(8)[None, :].expand(3, -1)
PACKED = torch.tensor([[0, 1, 2, 0, 1, 2, 3, 4]] * 3)


def _skips(q_len, kv_len, padding_mask=None, local=None):
    return bool(masking_utils._ignore_causal_mask_sdpa(padding_mask, q_len, kv_len, 0, local))


@pytest.fixture
def capturing(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)


def test_eager_mode_decisions_for_reference():
    assert _skips(1, 1) and _skips(16, 16) and not _skips(4, 16)
    assert masking_utils.find_packed_sequence_indices(ARANGE) is None
    assert masking_utils.find_packed_sequence_indices(PACKED) is not None


def test_capture_takes_the_eager_decisions(capturing):
    packed, skip = masking_utils.find_packed_sequence_indices, masking_utils._ignore_causal_mask_sdpa
    assert not _skips(1, 1) and not _skips(16, 16)  # unchanged helpers: capture counts as tracing
    assert masking_utils.find_packed_sequence_indices(ARANGE) is not None
    with eager_mask_decisions():
        assert _skips(1, 1) and _skips(16, 16) and not _skips(4, 16)
        assert _skips(8, 8, local=16) and not _skips(8, 8, local=8)
        assert masking_utils.find_packed_sequence_indices(ARANGE) is None
    assert masking_utils.find_packed_sequence_indices is packed
    assert masking_utils._ignore_causal_mask_sdpa is skip
    assert not _skips(1, 1)


def test_padding_mask_and_other_tracing_keep_the_helpers(capturing, monkeypatch):
    pad = torch.ones(2, 4, dtype=torch.bool)
    with eager_mask_decisions():
        assert not _skips(4, 4, padding_mask=pad)  # the unchanged helper, as under any capture
    monkeypatch.setattr(import_utils, "is_jit_tracing", lambda: True)
    with eager_mask_decisions():
        assert not _skips(1, 1)
        assert masking_utils.find_packed_sequence_indices(ARANGE) is not None


def test_outside_a_capture_nothing_changes():
    with eager_mask_decisions():
        assert _skips(1, 1) and not _skips(4, 16)
        assert masking_utils.find_packed_sequence_indices(PACKED) is not None


def test_restored_after_an_error(capturing):
    skip = masking_utils._ignore_causal_mask_sdpa
    with pytest.raises(RuntimeError):
        with eager_mask_decisions():
            raise RuntimeError("capture failed")
    assert masking_utils._ignore_causal_mask_sdpa is skip
