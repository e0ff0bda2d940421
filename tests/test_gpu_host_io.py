"""HostLoraPipeline: the LoRA op on host buffers, row-chunked over copy streams.

Checked against the fp32 oracle and, token for token,
against the single-shot device call: a token's result must not depend on the
chunking, and back-to-back calls on reused buffers must not race."""

import numpy as np
import pytest
import torch

from oracle import sgmv_ref
from polylora_b200.host_io import HostLoraPipeline
from polylora_b200.sgmv import build_segments, sgmv_shrink_expand
from test_gpu_sgmv import TOL, TORCH, inactive_mask, make_case

pytestmark = pytest.mark.gpu


def _host(c, key):
    return torch.from_numpy(c[key]).to(TORCH[c["dtype"]]).pin_memory()


def _single_shot(c, d_a, d_b, ranks, scales):
    x = _host(c, "x").cuda()
    y = _host(c, "y").cuda()
    wi = torch.from_numpy(c["wi"]).cuda()
    seq = torch.from_numpy(c["seq"]).cuda()
    table = build_segments(wi, seq, ranks, x.shape[1])
    sgmv_shrink_expand(x, d_a, d_b, y, table, ranks, scales)
    return y.cpu()


@pytest.mark.parametrize("chunks", [1, 3, 4, 64])
@pytest.mark.parametrize("shape", [(37, 5, 256, 384, 6, 16, [0, 8, 16], "bfloat16"),
                                   (2000, 1, 1024, 2048, 17, 16, [4, 8, 16], "bfloat16"),
                                   (9, 40, 512, 768, 4, 32, [8, 32], "float16")],
                         ids=["ragged", "decode", "prefill"])
def test_pipeline_matches_oracle_and_single_shot(shape, chunks, cuda_status_clean):
    B, M, K, N, ns, R, rc, dt = shape
    c = make_case(900 + B + chunks, B, M, K, N, ns, R, rc, dt, base_frac=0.2)
    t = TORCH[dt]
    d_a = torch.from_numpy(c["A"]).to("cuda", t)
    d_b = torch.from_numpy(c["B"]).to("cuda", t)
    ranks = torch.from_numpy(c["ranks"]).cuda()
    scales = torch.from_numpy(c["scales"]).cuda()
    x_h, y_h = _host(c, "x"), _host(c, "y")
    seq_h, wi_h = torch.from_numpy(c["seq"]).pin_memory(), torch.from_numpy(c["wi"]).pin_memory()
    out_h = torch.empty_like(y_h).pin_memory()
    pipe = HostLoraPipeline("cuda", chunks=chunks)
    pipe(x_h, d_a, d_b, seq_h, wi_h, ranks, scales, y_h, out_h)
    torch.cuda.current_stream().synchronize()
    got = out_h.float().numpy()
    ref = sgmv_ref.lora_forward_fp32(c["x"], c["A"], c["B"], c["seq"], c["wi"], c["ranks"], c["scales"], c["y"])
    assert sgmv_ref.lora_err(got, ref, c["y"], dt) <= TOL[dt]
    inact = inactive_mask(c)
    assert np.array_equal(got[inact], c["y"][inact]), "inactive tokens changed"
    assert torch.equal(out_h, _single_shot(c, d_a, d_b, ranks, scales))


def test_pipeline_back_to_back_reuses_buffers(cuda_status_clean):
    """Five calls queued without a sync, alternating two input sets and two
    output buffers, the last one in place (out is the base output): every
    result equals its single-shot value."""
    sets = [make_case(950 + i, 700, 2, 1024, 1536, 9, 16, [0, 4, 16], "bfloat16") for i in range(2)]
    t = torch.bfloat16
    d_a = torch.from_numpy(sets[0]["A"]).to("cuda", t)
    d_b = torch.from_numpy(sets[0]["B"]).to("cuda", t)
    ranks = torch.from_numpy(sets[0]["ranks"]).cuda()
    scales = torch.from_numpy(sets[0]["scales"]).cuda()
    for c in sets[1:]:  # one slot state for both input sets
        c.update(A=sets[0]["A"], B=sets[0]["B"], ranks=sets[0]["ranks"], scales=sets[0]["scales"])
    host = [(_host(c, "x"), _host(c, "y"), torch.from_numpy(c["seq"]).pin_memory(),
             torch.from_numpy(c["wi"]).pin_memory()) for c in sets]
    outs = [torch.empty_like(host[0][1]).pin_memory() for _ in range(2)]
    pipe = HostLoraPipeline("cuda", chunks=4)
    for i in range(4):
        x_h, y_h, seq_h, wi_h = host[i % 2]
        pipe(x_h, d_a, d_b, seq_h, wi_h, ranks, scales, y_h, outs[i % 2])
    torch.cuda.current_stream().synchronize()
    expect = [_single_shot(c, d_a, d_b, ranks, scales) for c in sets]
    for i in range(2):
        assert torch.equal(outs[i], expect[i])
    x_h, y_h, seq_h, wi_h = host[0]
    pipe(x_h, d_a, d_b, seq_h, wi_h, ranks, scales, y_h, y_h)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(y_h, expect[0])


def test_pipeline_rejects_device_inputs_and_empty_batch(cuda_status_clean):
    c = make_case(990, 4, 1, 64, 64, 3, 16, [16], "bfloat16")
    t = torch.bfloat16
    d_a = torch.from_numpy(c["A"]).to("cuda", t)
    d_b = torch.from_numpy(c["B"]).to("cuda", t)
    ranks = torch.from_numpy(c["ranks"]).cuda()
    scales = torch.from_numpy(c["scales"]).cuda()
    pipe = HostLoraPipeline("cuda")
    x_h, y_h = _host(c, "x"), _host(c, "y")
    seq_h, wi_h = torch.from_numpy(c["seq"]), torch.from_numpy(c["wi"])
    with pytest.raises(ValueError, match="host tensor"):
        pipe(x_h.cuda(), d_a, d_b, seq_h, wi_h, ranks, scales, y_h, y_h.clone())
    empty_x, empty_y = x_h[:0], y_h[:0]
    out = torch.empty_like(empty_y)
    assert pipe(empty_x, d_a, d_b, seq_h[:0], wi_h[:0], ranks, scales, empty_y, out).shape == empty_y.shape


def _slot_state(c):
    t = TORCH[c["dtype"]]
    return (torch.from_numpy(c["A"]).to("cuda", t), torch.from_numpy(c["B"]).to("cuda", t),
            torch.from_numpy(c["ranks"]).cuda(), torch.from_numpy(c["scales"]).cuda())


@pytest.mark.parametrize("chunks", [1, 4])
@pytest.mark.parametrize("shape", [(37, 5, 256, 384, 6, 16, [0, 8, 16], "bfloat16"),
                                   (2000, 1, 1024, 2048, 17, 16, [0, 4, 8, 16], "bfloat16"),
                                   (9, 40, 512, 768, 4, 32, [8, 32], "float16")],
                         ids=["ragged", "decode", "prefill"])
def test_in_place_moves_active_rows_only(shape, chunks, cuda_status_clean):
    """In place with pinned buffers the pipeline gathers and scatters only the
    segment table's rows (plora_gather_token_rows / plora_scatter_token_rows):
    the result equals the all-rows path and the single-shot call bit for bit,
    and rows of __base__ / rank-0 tokens and padding keep their bytes."""
    B, M, K, N, ns, R, rc, dt = shape
    c = make_case(1200 + B + chunks, B, M, K, N, ns, R, rc, dt, base_frac=0.2)
    d_a, d_b, ranks, scales = _slot_state(c)
    x_h = _host(c, "x")
    seq_h, wi_h = torch.from_numpy(c["seq"]).pin_memory(), torch.from_numpy(c["wi"]).pin_memory()
    y_active, y_all = _host(c, "y"), _host(c, "y")
    HostLoraPipeline("cuda", chunks=chunks)(x_h, d_a, d_b, seq_h, wi_h, ranks, scales, y_active, y_active)
    HostLoraPipeline("cuda", chunks=chunks, active_rows=False)(x_h, d_a, d_b, seq_h, wi_h, ranks, scales, y_all,
                                                               y_all)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(y_active, y_all)
    assert torch.equal(y_active, _single_shot(c, d_a, d_b, ranks, scales))
    inact = torch.from_numpy(inactive_mask(c))
    assert torch.equal(y_active[inact], _host(c, "y")[inact])


def test_in_place_back_to_back_accumulates(cuda_status_clean):
    """Four in-place calls queued without a sync over two input sets: each
    adds its delta to the same host rows; the active-rows path ends where the
    all-rows path does."""
    sets = [make_case(1300 + i, 600, 2, 1024, 1536, 9, 16, [0, 4, 16], "bfloat16") for i in range(2)]
    for c in sets[1:]:
        c.update(A=sets[0]["A"], B=sets[0]["B"], ranks=sets[0]["ranks"], scales=sets[0]["scales"])
    d_a, d_b, ranks, scales = _slot_state(sets[0])
    results = []
    for active in (True, False):
        pipe = HostLoraPipeline("cuda", chunks=3, active_rows=active)
        ys = [_host(c, "y") for c in sets]
        ins = [(_host(c, "x"), torch.from_numpy(c["seq"]).pin_memory(), torch.from_numpy(c["wi"]).pin_memory())
               for c in sets]
        for i in range(4):
            x_h, seq_h, wi_h = ins[i % 2]
            pipe(x_h, d_a, d_b, seq_h, wi_h, ranks, scales, ys[i % 2], ys[i % 2])
        torch.cuda.current_stream().synchronize()
        results.append(ys)
    for a, b in zip(*results):
        assert torch.equal(a, b)
    assert not torch.equal(results[0][0], _host(sets[0], "y"))  # the deltas did land


def test_token_rows_refuses_pageable_memory_and_flags_bad_tokens(cuda_status_clean):
    from polylora_b200 import _native
    from polylora_b200.sgmv import SegmentTable

    dev_rows = torch.zeros(4, 1, 16, dtype=torch.bfloat16, device="cuda")
    pageable = torch.arange(64, dtype=torch.float32).to(torch.bfloat16).reshape(4, 1, 16)
    table = SegmentTable(torch.tensor([0, 3], dtype=torch.int32, device="cuda"),
                         torch.tensor([0, 99, 2], dtype=torch.int32, device="cuda"), 4, 1, 1)
    with pytest.raises(ValueError, match="pinned"):
        _native.token_rows(pageable, dev_rows, table, to_host=False)
    lib = _native.load()
    st = lib.plora_gather_token_rows(pageable.data_ptr(), dev_rows.data_ptr(), 32, 4, table.slot_start.data_ptr(),
                                     table.token_index.data_ptr(), 1, torch.cuda.current_stream().cuda_stream)
    assert st == _native.ERR_INVALID_ARGUMENT and "page-locked" in _native.last_error()
    pinned = pageable.pin_memory()
    _native.device_status(clear=True)
    _native.token_rows(pinned, dev_rows, table, to_host=False)
    status = _native.device_status(clear=True)
    assert status == _native.DEV_TOKEN_RANGE  # token 99 skipped
    assert torch.equal(dev_rows[0].cpu(), pinned[0]) and torch.equal(dev_rows[2].cpu(), pinned[2])
    assert not dev_rows[1].any() and not dev_rows[3].any()


def test_paths_alternate_on_one_pipeline(cuda_status_clean):
    """In-place (active rows) and out-of-place (all rows) calls queued on one
    pipeline without a sync share its buffers and events: each result equals
    its single-shot value."""
    sets = [make_case(1400 + i, 500, 3, 512, 768, 7, 16, [0, 8, 16], "bfloat16") for i in range(2)]
    for c in sets[1:]:
        c.update(A=sets[0]["A"], B=sets[0]["B"], ranks=sets[0]["ranks"], scales=sets[0]["scales"])
    d_a, d_b, ranks, scales = _slot_state(sets[0])
    pipe = HostLoraPipeline("cuda", chunks=3)
    ins = [(_host(c, "x"), torch.from_numpy(c["seq"]).pin_memory(), torch.from_numpy(c["wi"]).pin_memory())
           for c in sets]
    y_in_place = _host(sets[0], "y")
    y_base, out = _host(sets[1], "y"), torch.empty_like(_host(sets[1], "y")).pin_memory()
    pipe(*ins[0][:1], d_a, d_b, *ins[0][1:], ranks, scales, y_in_place, y_in_place)
    pipe(*ins[1][:1], d_a, d_b, *ins[1][1:], ranks, scales, y_base, out)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(y_in_place, _single_shot(sets[0], d_a, d_b, ranks, scales))
    assert torch.equal(out, _single_shot(sets[1], d_a, d_b, ranks, scales))
