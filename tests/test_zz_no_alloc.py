"""The allocation-free shrink entry point, plora_sgmv_a_fwd_noalloc.

Some callers cannot allocate device memory when they invoke the kernel: a
serving loop running inside a region where cudaMalloc's implicit device
synchronisation is not allowed, an embedding runtime that hands out memory
only from its own fixed pool, or a foreign-language host that owns no CUDA
allocator.  For them this entry point takes only inputs and outputs and keeps
its segment scratch in a static device array inside the library.

The tests drive it through the C ABI (ctypes), twice in a row on different
batches so the second call runs over the scratch the first one left behind,
and check each result against the workspace entry point plora_sgmv_a_fwd on
every active token and against the CPU oracle, within the bf16 tolerance the
other GPU tests use: small batches, batches past the one-launch segment
builder (whose scratch then lives in the array too), and batches whose
scratch nearly fills the array.  They also check that the size limit is
enforced before any work is enqueued.
"""

import numpy as np
import pytest
import torch

from oracle import sgmv_ref
from polylora_b200 import _native
from polylora_b200.sgmv import sgmv_lora_a_fwd

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2  # normwise max relative error, as in test_gpu_sgmv.py


def _batch(seed, B, M, K, ns, R, dev):
    g = torch.Generator().manual_seed(seed)
    ranks = torch.tensor([0] + [int(r) for r in torch.tensor([4, 8, 16])[torch.randint(0, 3, (ns - 1,), generator=g)]],
                         dtype=torch.int32)
    A = (torch.rand(ns, K, R, generator=g) * 2 - 1) / 64
    A *= (torch.arange(R)[None, :] < ranks[:, None]).float()[:, None, :]
    x = torch.randn(B, M, K, generator=g)
    seq = torch.randint(0, M + 1, (B,), generator=g, dtype=torch.int32)
    wi = torch.randint(0, ns, (B,), generator=g, dtype=torch.int64)
    to = lambda t, dt=None: t.to(dev, dt) if dt else t.to(dev)  # noqa: E731
    return to(x, torch.bfloat16), to(A, torch.bfloat16), to(seq), to(wi), to(ranks)


def _active(seq, wi, ranks, M):
    m = torch.arange(M, device=seq.device)[None, :]
    return (m < seq.clamp(max=M)[:, None]) & (ranks[wi] > 0)[:, None]


def _noalloc(lib, x, A, seq, wi, ranks, out):
    B, M, K = x.shape
    ns, _, R = A.shape
    return lib.plora_sgmv_a_fwd_noalloc(
        x.data_ptr(), A.data_ptr(), out.data_ptr(), seq.data_ptr(), wi.data_ptr(), ranks.data_ptr(),
        B, M, K, R, ns, 1, _native.DTYPE_BF16, torch.cuda.current_stream().cuda_stream)


def _check_against_oracle(x, A, seq, wi, ranks, got, rows=None):
    """The shrink of the given rows (all by default) against oracle.sgmv_ref.shrink."""
    sel = slice(None) if rows is None else rows
    xs = x[sel].float().cpu().numpy()
    ref, written = sgmv_ref.shrink(xs, A.float().cpu().numpy(), seq[sel].cpu().numpy(), wi[sel].cpu().numpy(),
                                   ranks.cpu().numpy(), 1, "bfloat16")
    g = got[sel].float().cpu().numpy()
    if written.any():
        assert sgmv_ref.rel_err(g[written], ref[written]) <= TOL_BF16


def _two_calls(lib, cases, dev, K=1024, ns=9, oracle_rows=None):
    """Runs each batch through the no-alloc entry point, in order, each one over
    the scratch the previous call left; checks it against the workspace entry
    point on every active token and against the oracle."""
    for call, (seed, B, M) in enumerate(cases):
        x, A, seq, wi, ranks = _batch(seed, B, M, K, ns, 16, dev)
        want = sgmv_lora_a_fwd(x, A, seq, wi, ranks)
        got = torch.full_like(want, float("nan"))
        st = _noalloc(lib, x, A, seq, wi, ranks, got)
        assert st == _native.OK, _native.last_error()
        torch.cuda.synchronize()
        assert _native.device_status(clear=True) == 0
        act = _active(seq, wi, ranks, M)
        w = want[act].float().cpu().numpy()
        g = got[act].float().cpu().numpy()
        assert np.all(np.isfinite(g)), f"call {call}: active entries left unwritten"
        assert sgmv_ref.rel_err(g, w) <= TOL_BF16, f"call {call}"
        rows = None
        if oracle_rows is not None and B > oracle_rows:
            rows = torch.from_numpy(np.sort(np.random.default_rng(seed).choice(B, oracle_rows, replace=False)))
        _check_against_oracle(x, A, seq, wi, ranks, got, rows)


def test_no_alloc_shrink_matches_workspace_entry_point():
    """Batches small enough for the one-launch segment builder."""
    _two_calls(_native.load(), [(0, 300, 3), (1, 64, 17)], torch.device("cuda"))


def test_no_alloc_shrink_above_the_one_launch_builder():
    """More than 1024 rows: the three-pass segment builder carves its per-block
    counts and row offsets out of the static scratch too."""
    _two_calls(_native.load(), [(2, 2048, 4), (3, 3000, 2)], torch.device("cuda"))


def test_no_alloc_shrink_near_the_scratch_limit():
    """Single-token rows whose scratch (plora_workspace_size) is just under
    PLORA_NOALLOC_SCRATCH_BYTES, twice in a row; one row more than fits is
    refused before any work is enqueued."""
    lib = _native.load()
    ns = 9
    lo, hi = 1, 4 << 20
    while lo < hi:  # largest row count whose scratch fits
        mid = (lo + hi + 1) // 2
        if _native.workspace_size(mid, 1, ns) <= _native.NOALLOC_SCRATCH_BYTES:
            lo = mid
        else:
            hi = mid - 1
    rows = lo
    assert _native.workspace_size(rows, 1, ns) > 0.98 * _native.NOALLOC_SCRATCH_BYTES
    _two_calls(lib, [(4, rows, 1), (5, rows - 777, 1)], torch.device("cuda"), K=256, ns=ns, oracle_rows=4096)
    st = lib.plora_sgmv_a_fwd_noalloc(None, None, None, None, None, None, rows + 256, 1, 256, 16, ns, 1,
                                      _native.DTYPE_BF16, None)
    assert st == _native.ERR_UNSUPPORTED and "static scratch" in _native.last_error()


def test_no_alloc_rejects_batches_beyond_its_scratch():
    lib = _native.load()
    rows = _native.NOALLOC_SCRATCH_BYTES // 4  # the token table alone would overflow
    st = lib.plora_sgmv_a_fwd_noalloc(None, None, None, None, None, None, rows, 2, 64, 16, 5, 1,
                                      _native.DTYPE_BF16, None)
    assert st == _native.ERR_UNSUPPORTED
    assert "static scratch" in _native.last_error()
