"""SGMV shrink / expand through the C-ABI (drop-in sgmv_lora_a_fwd /
sgmv_lora_b_fwd) against the CPU oracle and the reference's golden outputs.

Tolerances (north star): bf16 / fp16 <= 2e-2, fp32 <= 1e-5, measured by
oracle.sgmv_ref.lora_err against the fp32-accumulated oracle (error beyond one
output ulp, relative to the largest LoRA delta).  Inactive tokens (rank-0
slot, padding, __base__) must stay bit-identical."""

import numpy as np
import pytest
import torch

from oracle import sgmv_ref
from polylora_b200.sgmv import (build_segments, sgmv_expand, sgmv_lora_a_fwd, sgmv_lora_b_fwd,
                                sgmv_shrink, sgmv_shrink_expand)

pytestmark = pytest.mark.gpu

TOL = {"bfloat16": 2e-2, "float16": 2e-2, "float32": 1e-5}


@pytest.fixture(params=["stream", "stream_separate", "token_split", "weight_split"])
def split_mode(request):
    """Runs the test under each kernel family of the tensor-core path: every
    CTA a share of the tokens, with rank-16 calls on the stream kernels (rows
    by bulk copies, weights in registers; the combined call as one fused
    kernel, or with "stream_separate" as the two) or on the windowed kernels;
    or each slot's weights spread over the grid (slot grid)."""
    from polylora_b200 import _native

    prev = _native.weight_split_tokens_per_sm(1 << 40 if request.param == "weight_split" else 0)
    prev_stream = _native.stream_kernels({"token_split": 0, "stream_separate": 1}.get(request.param, 2))
    yield request.param
    _native.weight_split_tokens_per_sm(prev)
    _native.stream_kernels(prev_stream)
TORCH = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def make_case(seed, B, M, K, N, ns, R, rank_choices, dtype, base_frac=0.2, stack_num=1, seq=None):
    rng = np.random.default_rng(seed)
    ranks = np.array([0] + list(rng.choice(rank_choices, size=ns - 1)), dtype=np.int32)
    A = np.zeros((ns, K, R), dtype=np.float32)
    Bw = np.zeros((ns, R // stack_num, N), dtype=np.float32)
    for s in range(1, ns):
        r = int(ranks[s])
        A[s, :, : r * stack_num] = rng.uniform(-1 / 64, 1 / 64, size=(K, r * stack_num))
        Bw[s, :r, :] = rng.normal(0, 0.02, size=(r, N))
    scales = np.array([0.0] + [16.0 / r if r else 0.0 for r in ranks[1:]], dtype=np.float32)
    x = rng.normal(0, 1, size=(B, M, K)).astype(np.float32)
    y = rng.normal(0, 1, size=(B, M, N)).astype(np.float32)
    sl = rng.integers(0, M + 2, size=B).astype(np.int32) if seq is None else np.asarray(seq, np.int32)
    wi = rng.integers(1, ns, size=B).astype(np.int64) if ns > 1 else np.zeros(B, np.int64)
    wi[rng.random(B) < base_frac] = 0
    r = lambda a: sgmv_ref.round_to(a, dtype)  # noqa: E731
    return dict(x=r(x), y=r(y), A=r(A), B=r(Bw), ranks=ranks, scales=scales, seq=sl, wi=wi, dtype=dtype)


def to_dev(c):
    t = TORCH[c["dtype"]]
    d = torch.device("cuda")
    return dict(
        x=torch.from_numpy(c["x"]).to(d, t), y=torch.from_numpy(c["y"]).to(d, t),
        A=torch.from_numpy(c["A"]).to(d, t), B=torch.from_numpy(c["B"]).to(d, t),
        ranks=torch.from_numpy(c["ranks"]).to(d), scales=torch.from_numpy(c["scales"]).to(d),
        seq=torch.from_numpy(c["seq"]).to(d), wi=torch.from_numpy(c["wi"]).to(d),
    )


def inactive_mask(c):
    M = c["x"].shape[1]
    m = np.arange(M)[None, :]
    active = (m < np.minimum(np.maximum(c["seq"], 0), M)[:, None]) & (c["ranks"][c["wi"]] > 0)[:, None]
    return ~active


def run_and_check(c):
    d = to_dev(c)
    tmp = sgmv_lora_a_fwd(d["x"], d["A"], d["seq"], d["wi"], d["ranks"])
    out = d["y"].clone()
    sgmv_lora_b_fwd(tmp, d["B"], d["seq"], d["wi"], d["ranks"], d["scales"], out)
    torch.cuda.synchronize()
    dt = c["dtype"]
    # shrink vs oracle on the entries the reference defines
    ref_tmp, written = sgmv_ref.shrink(c["x"], c["A"], c["seq"], c["wi"], c["ranks"], 1, dt)
    got_tmp = tmp.float().cpu().numpy()
    if written.any():
        assert sgmv_ref.rel_err(got_tmp[written], ref_tmp[written]) <= TOL[dt]
    # padded columns of active tokens are written as zeros
    active_tok = ~inactive_mask(c)
    pad = active_tok[:, :, None] & ~written
    assert np.all(got_tmp[pad] == 0)
    # full LoRA output vs the fp32-accumulated oracle
    got = out.float().cpu().numpy()
    ref = sgmv_ref.lora_forward_fp32(c["x"], c["A"], c["B"], c["seq"], c["wi"], c["ranks"], c["scales"], c["y"])
    err = sgmv_ref.lora_err(got, ref, c["y"], dt)
    assert err <= TOL[dt], err
    inact = inactive_mask(c)
    assert np.array_equal(got[inact], c["y"][inact]), "inactive tokens changed"
    return got, err


TC_CASES = [
    # seed, B, M, K, N, slots, R, ranks, dtype
    (1, 1, 1, 4096, 4096, 65, 16, [0, 4, 8, 16], "bfloat16"),
    (2, 16, 1, 4096, 4096, 65, 16, [0, 4, 8, 16], "bfloat16"),
    (3, 256, 1, 4096, 4096, 65, 16, [0, 4, 8, 16], "bfloat16"),
    (4, 1000, 1, 4096, 4096, 65, 16, [0, 4, 8, 16], "bfloat16"),
    (5, 8, 128, 768, 3072, 5, 16, [4, 8, 16], "bfloat16"),
    (6, 8, 128, 3072, 768, 5, 16, [4, 8, 16], "bfloat16"),
    (7, 6, 64, 1024, 1024, 9, 32, [8, 16, 32], "bfloat16"),
    (8, 4, 300, 512, 1536, 7, 64, [8, 16, 32, 64], "bfloat16"),
    (9, 300, 1, 200, 200, 11, 16, [0, 16], "bfloat16"),
    (10, 64, 3, 1024, 2048, 17, 16, [4, 16], "float16"),
    (11, 2, 1000, 256, 128, 3, 16, [16], "bfloat16"),
    (12, 40, 2, 800, 640, 6, 16, [4, 8, 16], "bfloat16"),  # K = 3 x 256 + 32: single-block tail boxes
    (13, 50, 1, 224, 96, 4, 32, [8, 32], "bfloat16"),  # K = 7 x 32: tail boxes only
]


@pytest.mark.parametrize("case", TC_CASES, ids=[f"tc{c[0]}" for c in TC_CASES])
def test_tensor_core_path_matches_oracle(case, split_mode, cuda_status_clean):
    seed, B, M, K, N, ns, R, rc, dt = case
    run_and_check(make_case(seed, B, M, K, N, ns, R, rc, dt))


SIMT_CASES = [
    (20, 8, 32, 64, 48, 5, 16, [4, 8, 16], "float32"),
    (21, 64, 1, 768, 768, 9, 16, [0, 4, 8, 16], "float32"),
    (22, 6, 7, 40, 24, 4, 3, [1, 2, 3], "float32"),
    (23, 9, 5, 100, 72, 5, 16, [4, 16], "bfloat16"),  # K % 8 != 0
    (24, 9, 5, 128, 96, 5, 8, [4, 8], "bfloat16"),    # max_rank 8
    (25, 9, 5, 128, 96, 5, 3, [1, 3], "float16"),     # odd max_rank
]


@pytest.mark.parametrize("case", SIMT_CASES, ids=[f"simt{c[0]}" for c in SIMT_CASES])
def test_cuda_core_path_matches_oracle(case, cuda_status_clean):
    seed, B, M, K, N, ns, R, rc, dt = case
    run_and_check(make_case(seed, B, M, K, N, ns, R, rc, dt))


def test_stack_num_two(split_mode, cuda_status_clean):
    c = make_case(30, 12, 4, 256, 128, 5, 32, [4, 8, 16], "bfloat16", stack_num=2)
    d = to_dev(c)
    tmp = sgmv_lora_a_fwd(d["x"], d["A"], d["seq"], d["wi"], d["ranks"], 2)
    ref_tmp, written = sgmv_ref.shrink(c["x"], c["A"], c["seq"], c["wi"], c["ranks"], 2, "bfloat16")
    got = tmp.float().cpu().numpy()
    assert sgmv_ref.rel_err(got[written], ref_tmp[written]) <= 2e-2
    # columns beyond rank * stack_num of active tokens are written as zeros
    pad = (~inactive_mask(c))[:, :, None] & ~written
    assert np.all(got[pad] == 0)


def test_all_base_rows_are_untouched(cuda_status_clean):
    c = make_case(31, 64, 4, 512, 256, 5, 16, [4, 16], "bfloat16", base_frac=1.0)
    got, _ = run_and_check(c)
    assert np.array_equal(got, c["y"])


def test_empty_batch(cuda_status_clean):
    d = torch.device("cuda")
    x = torch.zeros(0, 4, 64, device=d, dtype=torch.bfloat16)
    A = torch.zeros(3, 64, 16, device=d, dtype=torch.bfloat16)
    tmp = sgmv_lora_a_fwd(x, A, torch.zeros(0, dtype=torch.int32, device=d),
                          torch.zeros(0, dtype=torch.int64, device=d), torch.zeros(3, dtype=torch.int32, device=d))
    assert tmp.shape == (0, 4, 16)
    y = sgmv_lora_b_fwd(tmp, torch.zeros(3, 16, 32, device=d, dtype=torch.bfloat16), torch.zeros(0, dtype=torch.int32, device=d),
                        torch.zeros(0, dtype=torch.int64, device=d), torch.zeros(3, dtype=torch.int32, device=d),
                        torch.zeros(3, device=d))
    assert y.shape == (0, 4, 32)


@pytest.mark.parametrize("case", ["cfg1_rows_f32", "tokens_f32", "odd_rank_f32", "rows_bf16", "tokens_bf16", "rank64_bf16"])
def test_reference_golden_through_kernels(golden_dir, case, split_mode, cuda_status_clean):
    g = np.load(golden_dir / "reference_forward.npz")
    get = lambda k: g[f"{case}__{k}"]  # noqa: E731
    dt = str(get("dtype")[0])
    c = dict(x=get("x"), y=get("y"), A=get("A"), B=get("B"), ranks=get("ranks"), scales=get("scales"),
             seq=get("seq"), wi=get("wi"), dtype=dt)
    got, _ = run_and_check(c)
    # and against the reference's own output (which rounds in `dt` itself)
    tol = TOL[dt] if dt != "float32" else 1e-5
    assert sgmv_ref.lora_err(got, get("out"), get("y"), dt) <= max(tol, 2 * sgmv_ref.ULP[dt])


def test_segment_table_reuse_across_modules(cuda_status_clean):
    """One table (built with the max rank over modules) serves modules whose
    own ranks are 0 for some slots: those tokens are skipped."""
    c = make_case(40, 200, 1, 512, 512, 9, 16, [4, 8, 16], "bfloat16", base_frac=0.1)
    d = to_dev(c)
    union = d["ranks"].clone()
    module_ranks = d["ranks"].clone()
    module_ranks[1::2] = 0  # this module has no weights in odd slots
    cm = dict(c, ranks=module_ranks.cpu().numpy())
    table = build_segments(d["wi"], d["seq"], union, 1)
    tmp = sgmv_shrink(d["x"], d["A"], table, module_ranks)
    out = d["y"].clone()
    sgmv_expand(tmp, d["B"], out, table, module_ranks, d["scales"])
    ref = sgmv_ref.lora_forward_fp32(cm["x"], cm["A"], cm["B"], cm["seq"], cm["wi"], cm["ranks"], cm["scales"], cm["y"])
    got = out.float().cpu().numpy()
    assert sgmv_ref.lora_err(got, ref, c["y"], "bfloat16") <= 2e-2
    inact = inactive_mask(cm)
    assert np.array_equal(got[inact], c["y"][inact])


@pytest.mark.parametrize("R,rc,dt", [(16, [0, 4, 8, 16], "bfloat16"), (64, [8, 64], "float16"), (32, [8, 32], "bfloat16")])
def test_combined_entry_matches_separate_calls(R, rc, dt, split_mode, cuda_status_clean):
    """plora_sgmv_shrink_expand (expand launched to overlap the shrink's end)
    gives bit-identical tmp and y to plora_sgmv_shrink + plora_sgmv_expand,
    repeated back to back on one stream."""
    c = make_case(50 + R, 600, 1, 1024, 2048, 17, R, rc, dt, base_frac=0.2)
    d = to_dev(c)
    table = build_segments(d["wi"], d["seq"], d["ranks"], 1)
    # rows of inactive tokens are never written: both tmp buffers start at zero
    tmp_sep = torch.zeros(d["x"].shape[:2] + (R,), device="cuda", dtype=d["x"].dtype)
    tmp_comb = torch.zeros_like(tmp_sep)
    y_sep = d["y"].clone()
    y_comb = d["y"].clone()
    for _ in range(3):  # back to back: each call must see the previous one's y
        sgmv_shrink_expand(d["x"], d["A"], d["B"], y_comb, table, d["ranks"], d["scales"], tmp=tmp_comb)
        sgmv_shrink(d["x"], d["A"], table, d["ranks"], out=tmp_sep)
        sgmv_expand(tmp_sep, d["B"], y_sep, table, d["ranks"], d["scales"])
    torch.cuda.synchronize()
    assert torch.equal(tmp_comb, tmp_sep)
    assert torch.equal(y_comb, y_sep)


def test_full_size_cfg2_sampled_parity_and_determinism(cuda_status_clean):
    """BASELINE config 2 at its largest size (T=16384, K=N=4096, 64 slots):
    a sample of tokens against the oracle, inactive tokens bit-identical, and
    two runs bit-identical (no atomics decide any sum)."""
    T, K, N, ns, R = 16384, 4096, 4096, 65, 16
    g = torch.Generator(device="cuda").manual_seed(0)
    d = torch.device("cuda")
    ranks = torch.tensor([0] + list(np.random.default_rng(0).choice([0, 4, 8, 16], size=ns - 1)), dtype=torch.int32, device=d)
    A = (torch.rand(ns, K, R, device=d, generator=g) * 2 - 1) / 64
    Bw = torch.randn(ns, R, N, device=d, generator=g) * 0.02
    colmask = torch.arange(R, device=d)[None, :] < ranks[:, None]
    A = (A * colmask[:, None, :]).to(torch.bfloat16)
    Bw = (Bw * colmask[:, :, None]).to(torch.bfloat16)
    scales = torch.where(ranks > 0, 16.0 / ranks.clamp(min=1).float(), torch.zeros_like(ranks, dtype=torch.float32))
    x = torch.randn(T, 1, K, device=d, generator=g).to(torch.bfloat16)
    y = torch.randn(T, 1, N, device=d, generator=g).to(torch.bfloat16)
    wi = torch.randint(1, ns, (T,), device=d, generator=g)
    wi[torch.rand(T, device=d, generator=g) < 0.2] = 0
    seq = torch.ones(T, dtype=torch.int32, device=d)
    outs = []
    for _ in range(2):
        tmp = sgmv_lora_a_fwd(x, A, seq, wi, ranks)
        o = y.clone()
        sgmv_lora_b_fwd(tmp, Bw, seq, wi, ranks, scales, o)
        outs.append(o)
    assert torch.equal(outs[0], outs[1])
    rows = np.random.default_rng(1).choice(T, size=384, replace=False)
    sub = dict(x=x[rows].float().cpu().numpy(), y=y[rows].float().cpu().numpy(), A=A.float().cpu().numpy(),
               B=Bw.float().cpu().numpy(), ranks=ranks.cpu().numpy(), scales=scales.cpu().numpy(),
               seq=np.ones(len(rows), np.int32), wi=wi[rows].cpu().numpy(), dtype="bfloat16")
    ref = sgmv_ref.lora_forward_fp32(sub["x"], sub["A"], sub["B"], sub["seq"], sub["wi"], sub["ranks"], sub["scales"], sub["y"])
    got = outs[0][rows].float().cpu().numpy()
    assert sgmv_ref.lora_err(got, ref, sub["y"], "bfloat16") <= 2e-2
    inactive = (ranks[wi] == 0)
    assert torch.equal(outs[0][inactive], y[inactive])
