"""The bounded pipeline waits give up and report instead of spinning.

Every mbarrier wait of the tensor-core kernels is bounded (1 s by default);
on expiry the kernel sets PLORA_DEV_WAIT_TIMEOUT in the device status word,
the warps leave their loops, the CTA waits (with its own fixed bound) for
the copies it already issued, and the kernel returns.  The test shortens the
limit to zero through plora_set_wait_limit_ns, so that a wait whose phase is
not already complete when first polled runs out (a ring stage just issued is
never complete that soon); no fault, trap or endless loop is involved.  It
then checks that the status bit was raised, that the context is still
usable, and that with the limit restored the same call gives the oracle's
result again.
"""

import numpy as np
import pytest
import torch

from oracle import sgmv_ref
from polylora_b200 import _native
from polylora_b200.sgmv import build_segments, sgmv_expand, sgmv_shrink, sgmv_shrink_expand

pytestmark = pytest.mark.gpu


def _config2_like(dev, T=8192, K=4096, N=4096, ns=65, R=16, seed=11):
    rng = np.random.default_rng(seed)
    ranks = torch.tensor([0] + list(rng.choice([4, 8, 16], size=ns - 1)), dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    colmask = torch.arange(R, device=dev)[None, :] < ranks[:, None]
    A = ((torch.rand(ns, K, R, device=dev, generator=g) * 2 - 1) / 64 * colmask[:, None, :]).to(torch.bfloat16)
    Bw = (torch.randn(ns, R, N, device=dev, generator=g) * 0.02 * colmask[:, :, None]).to(torch.bfloat16)
    x = torch.randn(T, 1, K, device=dev, generator=g).to(torch.bfloat16)
    y = torch.randn(T, 1, N, device=dev, generator=g).to(torch.bfloat16)
    wi = torch.randint(1, ns, (T,), device=dev, generator=g)
    scales = torch.where(ranks > 0, 16.0 / ranks.clamp(min=1).float(), torch.zeros(ns, device=dev))
    return x, y, A, Bw, ranks, scales, wi, torch.ones(T, dtype=torch.int32, device=dev)


# kernel families whose waits are driven out: the stream shrink and expand as
# two launches, the fused stream kernel (combined call), the windowed kernels
FAMILIES = {"stream": 1, "fused": 2, "windowed": 0}


@pytest.fixture(params=list(FAMILIES))
def family(request):
    prev = (_native.weight_split_tokens_per_sm(0), _native.stream_kernels(FAMILIES[request.param]))
    yield request.param
    _native.weight_split_tokens_per_sm(prev[0])
    _native.stream_kernels(prev[1])


def _lora(family, x, A, Bw, table, ranks, scales, tmp, out):
    if family == "fused":
        sgmv_shrink_expand(x, A, Bw, out, table, ranks, scales, tmp=tmp)
    else:
        sgmv_shrink(x, A, table, ranks, out=tmp)
        sgmv_expand(tmp, Bw, out, table, ranks, scales)


def test_expired_waits_report_and_leave_the_context_usable(family):
    dev = torch.device("cuda")
    x, y, A, Bw, ranks, scales, wi, seq = _config2_like(dev)
    table = build_segments(wi, seq, ranks, 1)
    tmp = torch.zeros(x.shape[0], 1, 16, device=dev, dtype=torch.bfloat16)
    torch.cuda.synchronize()
    _native.device_status(clear=True)
    prev = _native.set_wait_limit_ns(0)
    try:
        raised = 0
        for _ in range(3):
            _lora(family, x, A, Bw, table, ranks, scales, tmp, y.clone())
            status = _native.device_status(clear=True)  # synchronises: every kernel returned
            raised += bool(status & _native.DEV_WAIT_TIMEOUT)
            assert status & ~_native.DEV_WAIT_TIMEOUT == 0, f"unexpected status {status:#x}"
        # a launch runs out at its first ring wait that is not already complete:
        # the token stage issued just before the loop starts has not landed then
        assert raised >= 1, "a zero wait limit must expire a ring wait"
    finally:
        assert _native.set_wait_limit_ns(prev) == 0
    # limit restored: the same calls are correct again and raise nothing
    out = y.clone()
    _lora(family, x, A, Bw, table, ranks, scales, tmp, out)
    assert _native.device_status(clear=True) == 0
    rows = np.random.default_rng(0).choice(x.shape[0], size=512, replace=False)
    ref = sgmv_ref.lora_forward_fp32(
        x[rows].float().cpu().numpy(), A.float().cpu().numpy(), Bw.float().cpu().numpy(), np.ones(len(rows), np.int32),
        wi[rows].cpu().numpy(), ranks.cpu().numpy(), scales.cpu().numpy(), y[rows].float().cpu().numpy())
    err = sgmv_ref.lora_err(out[rows].float().cpu().numpy(), ref, y[rows].float().cpu().numpy(), "bfloat16")
    assert err <= 2e-2, err
