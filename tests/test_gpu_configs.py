"""Parity at the shapes the benches run (3 and 4), every
active token checked against the CPU oracle.

* Config 2 at every T of its sweep (1 .. 16384 tokens, K = N = 4096, 64 slots
  + __base__, max_rank 16).
* Config 3's three Linear shapes of a DeBERTa-v3-large layer (1024 -> 1024,
  1024 -> 4096, 4096 -> 1024) on 256 rows x 512 right-padded tokens, 33 slots,
  max_rank 16.
* Config 4's q / gate / down projections of a Llama-3-8B layer (4096 -> 4096,
  4096 -> 14336, 14336 -> 4096), max_rank 64, 128 adapters with Zipf(1.1)
  popularity: prefill rows of 1024 tokens and a 256 x 1 decode batch.

Every case runs under each kernel family (stream, windowed token split, slot
grid) through the two operators, and through the combined call that the
layers make (sgmv_shrink_expand: the fused stream kernel where it applies);
the oracle is computed once per case.  Checks: tmp against the oracle
shrink, the output against the fp32-accumulated forward with the one-ulp
error measure and, on a second run over a zero base output, the delta itself
element-wise (half an ulp of allowance: oracle.sgmv_ref.lora_err_strict);
tokens the reference leaves alone stay bit-identical.  The oracle is compared
in row chunks to bound host memory.
"""

import numpy as np
import pytest
import torch

from oracle import sgmv_ref
from polylora_b200 import _native
from polylora_b200.sgmv import build_segments, sgmv_lora_a_fwd, sgmv_lora_b_fwd, sgmv_shrink_expand

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16, north star
MODES = ("stream", "token_split", "weight_split", "combined")


def _set_mode(mode):
    prev = (_native.weight_split_tokens_per_sm(), _native.stream_kernels())
    _native.weight_split_tokens_per_sm(1 << 40 if mode == "weight_split" else 0)
    _native.stream_kernels({"token_split": 0, "combined": 2}.get(mode, 1))
    return prev


def _restore(prev):
    _native.weight_split_tokens_per_sm(prev[0])
    _native.stream_kernels(prev[1])


def _case(seed, rows, seq, K, N, ns, R, rank_choices, base_frac, popularity=None, lens=None):
    """Seeded bf16 case on the GPU (host copies for the oracle are made per chunk)."""
    rng = np.random.default_rng(seed)
    ranks = np.array([0] + list(rng.choice(rank_choices, size=ns - 1)), dtype=np.int32)
    d = torch.device("cuda")
    g = torch.Generator(device=d).manual_seed(seed)
    colmask = torch.arange(R, device=d)[None, :] < torch.from_numpy(ranks).to(d)[:, None]
    A = ((torch.rand(ns, K, R, device=d, generator=g) * 2 - 1) / np.sqrt(K) * colmask[:, None, :]).to(torch.bfloat16)
    Bw = (torch.randn(ns, R, N, device=d, generator=g) * 0.02 * colmask[:, :, None]).to(torch.bfloat16)
    x = torch.randn(rows, seq, K, device=d, generator=g).to(torch.bfloat16)
    y = torch.randn(rows, seq, N, device=d, generator=g).to(torch.bfloat16)
    if popularity is None:
        wi = rng.integers(1, ns, size=rows).astype(np.int64)
    else:
        wi = (1 + rng.choice(ns - 1, size=rows, p=popularity)).astype(np.int64)
    wi[rng.random(rows) < base_frac] = 0
    sl = np.full(rows, seq, np.int32) if lens is None else np.asarray(lens, np.int32)
    scales = np.array([0.0] + [16.0 / int(r) if r else 0.0 for r in ranks[1:]], np.float32)  # alpha 16
    return dict(x=x, y=y, A=A, B=Bw, ranks=ranks, scales=scales, wi=wi, seq=sl)


def _run(c, y, combined=False):
    d = torch.device("cuda")
    seq = torch.from_numpy(c["seq"]).to(d)
    wi = torch.from_numpy(c["wi"]).to(d)
    ranks = torch.from_numpy(c["ranks"]).to(d)
    scales = torch.from_numpy(c["scales"]).to(d)
    out = y.clone()
    if combined:
        x = c["x"]
        table = build_segments(wi, seq, ranks, x.shape[1])
        tmp = torch.empty(x.shape[0], x.shape[1], c["A"].shape[2], device=d, dtype=x.dtype)
        sgmv_shrink_expand(x, c["A"], c["B"], out, table, ranks, scales, tmp=tmp)
    else:
        tmp = sgmv_lora_a_fwd(c["x"], c["A"], seq, wi, ranks)
        sgmv_lora_b_fwd(tmp, c["B"], seq, wi, ranks, scales, out)
    torch.cuda.synchronize()
    return tmp, out


def _oracle_chunks(c, chunk_rows):
    """Yields (row slice, oracle tmp, written mask, fp32 forward over y, over zeros)."""
    A = c["A"].float().cpu().numpy()
    Bw = c["B"].float().cpu().numpy()
    rows = c["x"].shape[0]
    for r0 in range(0, rows, chunk_rows):
        sl = slice(r0, min(rows, r0 + chunk_rows))
        x = c["x"][sl].float().cpu().numpy()
        y = c["y"][sl].float().cpu().numpy()
        seq, wi = c["seq"][sl], c["wi"][sl]
        tmp, written = sgmv_ref.shrink(x, A, seq, wi, c["ranks"], 1, "bfloat16")
        fwd = sgmv_ref.lora_forward_fp32(x, A, Bw, seq, wi, c["ranks"], c["scales"], y)
        fwd0 = sgmv_ref.lora_forward_fp32(x, A, Bw, seq, wi, c["ranks"], c["scales"], np.zeros_like(y))
        yield sl, tmp, written, fwd, fwd0, y


def _inactive(c, sl):
    M = c["x"].shape[1]
    m = np.arange(M)[None, :]
    seq, wi = c["seq"][sl], c["wi"][sl]
    active = (m < np.minimum(np.maximum(seq, 0), M)[:, None]) & (c["ranks"][wi] > 0)[:, None]
    return ~active


def _check_case(c, chunk_rows, modes=MODES):
    outs = {}
    for mode in modes:
        prev = _set_mode(mode)
        try:
            _native.device_status(clear=True)
            tmp, out = _run(c, c["y"], mode == "combined")
            _, out0 = _run(c, torch.zeros_like(c["y"]), mode == "combined")
            assert _native.device_status(clear=True) == 0, mode
        finally:
            _restore(prev)
        outs[mode] = (tmp, out, out0)
    for sl, ref_tmp, written, fwd, fwd0, y in _oracle_chunks(c, chunk_rows):
        inact = _inactive(c, sl)
        for mode, (tmp, out, out0) in outs.items():
            got_tmp = tmp[sl].float().cpu().numpy()
            if written.any():
                assert sgmv_ref.rel_err(got_tmp[written], ref_tmp[written]) <= TOL, mode
            got = out[sl].float().cpu().numpy()
            assert sgmv_ref.lora_err(got, fwd, y, "bfloat16") <= TOL, mode
            got0 = out0[sl].float().cpu().numpy()
            assert sgmv_ref.lora_err_strict(got0, fwd0, np.zeros_like(got0), "bfloat16") <= TOL, mode
            assert np.array_equal(got[inact], y[inact]), f"{mode}: inactive tokens changed"
            assert np.all(got0[inact] == 0), f"{mode}: inactive tokens changed (zero base)"


@pytest.mark.parametrize("T", [1, 16, 256, 4096, 16384])
def test_config2_sweep_every_token(T, cuda_status_clean):
    c = _case(100 + T, T, 1, 4096, 4096, 65, 16, [0, 4, 8, 16], 0.2)
    _check_case(c, chunk_rows=4096)


@pytest.mark.parametrize("K,N", [(1024, 1024), (1024, 4096), (4096, 1024)], ids=["attn", "ffn_in", "ffn_out"])
def test_config3_layer_shapes(K, N, cuda_status_clean):
    rng = np.random.default_rng(7)
    lens = rng.integers(64, 513, size=256)
    c = _case(200 + K + N, 256, 512, K, N, 33, 16, [4, 8, 16], 0.25, lens=lens)
    _check_case(c, chunk_rows=32)


def _zipf(n, s):
    p = 1.0 / np.arange(1, n + 1) ** s
    return p / p.sum()


@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 14336), (14336, 4096)], ids=["q_proj", "gate_proj", "down_proj"])
@pytest.mark.parametrize("step", ["prefill", "decode"])
def test_config4_layer_shapes(K, N, step, cuda_status_clean):
    rows, seq = (16, 1024) if step == "prefill" else (256, 1)
    c = _case(300 + K + N, rows, seq, K, N, 129, 64, [8, 16, 32, 64], 0.0, popularity=_zipf(128, 1.1))
    _check_case(c, chunk_rows=4 if step == "prefill" else 256)


@pytest.mark.parametrize("ns,rows", [(601, 2048), (4096, 1500)], ids=["601_slots", "4096_slots"])
def test_slot_grid_later_tiles_many_slots(ns, rows, cuda_status_clean):
    """The slot grid's later-tile rows (slots holding more than 16 tokens get
    one grid row per further 16-token tile) when the slot table spans several
    256-slot rounds of the row search: Zipf popularity puts hundreds of tokens
    on the first slots and one or none on the rest."""
    c = _case(400 + ns, rows, 1, 1024, 1024, ns, 16, [4, 8, 16], 0.1, popularity=_zipf(ns - 1, 1.1))
    _check_case(c, chunk_rows=rows, modes=("weight_split", "combined"))

