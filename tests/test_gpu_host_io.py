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
