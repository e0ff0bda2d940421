"""Device segment table and flat schedule: bit-exact against the oracle and
the reference's golden schedule."""

import numpy as np
import pytest
import torch

from oracle import schedule_ref
from polylora_b200.sgmv import build_flat_schedule, build_segments

pytestmark = pytest.mark.gpu


def _run(wi, sl, rk, M):
    dev = torch.device("cuda")
    t = build_segments(torch.as_tensor(wi, dtype=torch.int64, device=dev),
                       torch.as_tensor(sl, dtype=torch.int32, device=dev),
                       torch.as_tensor(rk, dtype=torch.int32, device=dev), M)
    start = t.slot_start.cpu().numpy()
    return start, t.token_index[: int(start[-1])].cpu().numpy()


CASES = [
    # B, M, num_slots, base fraction, rank choices
    (16384, 1, 65, 0.2, [0, 4, 8, 16]),
    (256, 512, 33, 0.25, [0, 4, 8, 16]),
    (64, 1024, 129, 0.0, [8, 16, 32, 64]),
    (3000, 7, 1000, 0.1, [0, 4]),
    (1, 1, 1, 0.0, [0]),
    (37, 5, 2, 0.5, [16]),
    (255, 3, 17, 0.3, [0, 16]),
    (257, 3, 17, 0.3, [0, 16]),
    # the one-launch builder's limits (rows <= 1024, slots <= 256, tokens <= 16384) and just past each
    (1024, 16, 256, 0.2, [0, 4, 8, 16]),
    (1000, 16, 200, 0.1, [0, 8]),
    (1024, 17, 65, 0.2, [0, 4, 8, 16]),
    (1025, 1, 65, 0.2, [0, 4, 8, 16]),
    (1024, 1, 257, 0.2, [0, 4, 8, 16]),
    # larger batches (three kernels): many blocks of rows, all slots in one block, long rows
    (1025, 3, 9, 0.2, [0, 4, 8, 16]),
    (2048, 1, 1, 0.0, [0]),
    (4097, 2, 256, 0.1, [0, 16]),
    (32768, 1, 65, 0.2, [0, 4, 8, 16]),
    (32769, 1, 65, 0.2, [0, 4, 8, 16]),
    (8192, 1, 257, 0.2, [0, 4, 8, 16]),
    (4096, 1025, 9, 0.0, [16]),
]


@pytest.mark.parametrize("B,M,ns,base,rc", CASES)
def test_segments_bit_exact(B, M, ns, base, rc, cuda_status_clean):
    rng = np.random.default_rng(B * 7 + M)
    wi = rng.integers(0, ns, size=B)
    wi[rng.random(B) < base] = 0
    sl = rng.integers(-2, M + 3, size=B)
    rk = np.array([0] + list(rng.choice(rc, size=ns - 1)), dtype=np.int32) if ns > 1 else np.zeros(1, np.int32)
    start, tok = _run(wi, sl, rk, M)
    ref_start, ref_tok = schedule_ref.segments(wi, sl, rk, M, ns)
    np.testing.assert_array_equal(start, ref_start)
    np.testing.assert_array_equal(tok, ref_tok)


def test_segments_empty_and_all_base(cuda_status_clean):
    start, tok = _run(np.zeros(0, np.int64), np.zeros(0, np.int32), np.array([0, 4]), 8)
    assert start.tolist() == [0, 0, 0] and tok.size == 0
    start, tok = _run(np.zeros(10, np.int64), np.full(10, 3), np.array([0, 4]), 8)
    assert start.tolist() == [0, 0, 0] and tok.size == 0


def test_out_of_range_slot_is_skipped_and_reported(native):
    native.device_status(clear=True)
    wi = np.array([1, 9, 1, -1], dtype=np.int64)
    start, tok = _run(wi, np.array([2, 2, 1, 2]), np.array([0, 4, 8]), 4)
    assert start.tolist() == [0, 0, 3, 3]
    assert tok.tolist() == [0, 1, 8]
    assert native.device_status(clear=True) & native.DEV_SLOT_RANGE


def test_flat_schedule_matches_reference_golden(golden_dir, cuda_status_clean):
    g = np.load(golden_dir / "flat_schedule.npz")
    names = sorted({k.split("__")[0] for k in g.files})
    for name in names:
        bm, bn = g[f"{name}__blocks"].tolist()
        cum, nn, total = build_flat_schedule(torch.from_numpy(g[f"{name}__seq"]).cuda(),
                                             torch.from_numpy(g[f"{name}__neff"]).cuda(), bm, bn)
        np.testing.assert_array_equal(cum.cpu().numpy(), g[f"{name}__cum"], err_msg=name)
        np.testing.assert_array_equal(nn.cpu().numpy(), g[f"{name}__nn"], err_msg=name)
        assert total == int(g[f"{name}__total"][0])
