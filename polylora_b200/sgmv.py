"""SGMV operators over the C-ABI library (no Triton, no CPU fallback).

Drop-in for the reference operators in ``src/polylora/sgmv.py``:

* :func:`sgmv_lora_a_fwd` — sgmv.py:141-175 (shrink, x·A[slot])
* :func:`sgmv_lora_b_fwd` — sgmv.py:278-328 (expand, fused scale + add-back)
* :func:`build_flat_schedule` — sgmv.py:29-61 (the reference's tile schedule,
  computed on the device)

plus the segment-table API the wrapped layers use: the table that groups the
active tokens of a batch by slot is built once per forward on the device
(:func:`build_segments`) and shared by every wrapped Linear
(:func:`sgmv_shrink`, :func:`sgmv_expand`).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native

_DTYPES = {
    torch.float32: _native.DTYPE_F32,
    torch.float16: _native.DTYPE_F16,
    torch.bfloat16: _native.DTYPE_BF16,
}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise TypeError(f"polylora_b200 kernels support float32/float16/bfloat16, got {dtype}") from None


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise RuntimeError(
            "polylora_b200 runs its LoRA kernels on CUDA devices only "
            f"(got a tensor on {dev}); there is no CPU fallback"
        )
    for t in tensors[1:]:
        if t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _as(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return t if t.dtype == dtype and t.is_contiguous() else t.to(dtype).contiguous()


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


@dataclass
class SegmentTable:
    """Active tokens of a batch grouped by slot (device tensors).

    ``slot_start`` (num_slots + 1,) int32 is the exclusive prefix of active
    tokens per slot; ``token_index`` holds the active token ids
    ``row * max_seq + m`` in (slot, row, m) order.
    """

    slot_start: torch.Tensor
    token_index: torch.Tensor
    num_rows: int
    max_seq: int
    num_slots: int

    @property
    def num_tokens(self) -> int:
        return self.num_rows * self.max_seq


def build_segments(
    weight_indices: torch.Tensor,
    seq_lens: torch.Tensor,
    lora_ranks: torch.Tensor,
    max_seq: int,
) -> SegmentTable:
    """Builds the slot-grouped token table on the device (no host sync)."""
    dev = _require_cuda(weight_indices, seq_lens, lora_ranks)
    wi = _as(weight_indices, torch.int64)
    sl = _as(seq_lens, torch.int32)
    rk = _as(lora_ranks, torch.int32)
    num_rows = int(wi.shape[0])
    num_slots = int(rk.shape[0])
    slot_start = torch.empty(num_slots + 1, dtype=torch.int32, device=dev)
    token_index = torch.empty(max(num_rows * max_seq, 1), dtype=torch.int32, device=dev)
    ws = _workspace(dev, _native.workspace_size(num_rows, max_seq, num_slots))
    _native.call(
        "plora_build_segments",
        wi.data_ptr(), sl.data_ptr(), rk.data_ptr(), num_rows, max_seq, num_slots,
        slot_start.data_ptr(), token_index.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev),
    )
    return SegmentTable(slot_start, token_index, num_rows, max_seq, num_slots)


def sgmv_shrink(
    x: torch.Tensor,
    weights: torch.Tensor,
    table: SegmentTable,
    lora_ranks: torch.Tensor,
    stack_num: int = 1,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """tmp = x · A[slot] over a prebuilt table; x (B, M, K), weights (NS, K, R)."""
    dev = _require_cuda(x, weights, lora_ranks)
    B, M, K = x.shape
    ns, kw, R = weights.shape
    if kw != K:
        raise ValueError(f"K mismatch: x={K}, weights={kw}")
    if (B, M) != (table.num_rows, table.max_seq) or ns != table.num_slots:
        raise ValueError("segment table does not match the input shape")
    if out is None:
        out = torch.empty((B, M, R), device=dev, dtype=x.dtype)
    if B == 0 or M == 0:
        return out
    xc = x.contiguous()
    w = weights.contiguous()
    if w.dtype != xc.dtype:
        raise TypeError(f"dtype mismatch: x={xc.dtype}, weights={w.dtype}")
    rk = _as(lora_ranks, torch.int32)
    _native.call(
        "plora_sgmv_shrink",
        xc.data_ptr(), w.data_ptr(), out.data_ptr(), rk.data_ptr(),
        table.slot_start.data_ptr(), table.token_index.data_ptr(), table.num_tokens,
        K, R, ns, stack_num, dtype_code(xc.dtype), _stream(dev),
    )
    return out


def sgmv_expand(
    tmp: torch.Tensor,
    weights: torch.Tensor,
    y: torch.Tensor,
    table: SegmentTable,
    lora_ranks: torch.Tensor,
    scalings: torch.Tensor,
) -> torch.Tensor:
    """y += scale · tmp · B[slot] in place over a prebuilt table; y (B, M, N)."""
    dev = _require_cuda(tmp, weights, y, lora_ranks, scalings)
    B, M, R = tmp.shape
    ns, rw, N = weights.shape
    if rw != R:
        raise ValueError(f"K mismatch: x={R}, weights={rw}")
    if tuple(y.shape) != (B, M, N):
        raise ValueError(f"base_output shape {tuple(y.shape)} != {(B, M, N)}")
    if not y.is_contiguous():
        raise ValueError("base_output must be contiguous (it is updated in place)")
    if B == 0 or M == 0:
        return y
    t = tmp.contiguous()
    w = weights.contiguous()
    if not (t.dtype == w.dtype == y.dtype):
        raise TypeError(f"dtype mismatch: tmp={t.dtype}, weights={w.dtype}, out={y.dtype}")
    rk = _as(lora_ranks, torch.int32)
    sc = _as(scalings, torch.float32)
    _native.call(
        "plora_sgmv_expand",
        t.data_ptr(), w.data_ptr(), y.data_ptr(), rk.data_ptr(), sc.data_ptr(),
        table.slot_start.data_ptr(), table.token_index.data_ptr(), table.num_tokens,
        R, N, ns, dtype_code(y.dtype), _stream(dev),
    )
    return y


def sgmv_shrink_expand(
    x: torch.Tensor,
    weights_a: torch.Tensor,
    weights_b: torch.Tensor,
    y: torch.Tensor,
    table: SegmentTable,
    lora_ranks: torch.Tensor,
    scalings: torch.Tensor,
    tmp: torch.Tensor | None = None,
) -> torch.Tensor:
    """y += scale · (x · A[slot]) · B[slot] in place: :func:`sgmv_shrink` then
    :func:`sgmv_expand` in one call, the expand overlapping the shrink's end.

    x (B, M, K), weights_a (NS, K, R), weights_b (NS, R, N), y (B, M, N)."""
    dev = _require_cuda(x, weights_a, weights_b, y, lora_ranks, scalings)
    B, M, K = x.shape
    ns, kw, R = weights_a.shape
    nsb, rw, N = weights_b.shape
    if kw != K or rw != R or nsb != ns:
        raise ValueError(f"weight shapes {tuple(weights_a.shape)} / {tuple(weights_b.shape)} do not match x")
    if (B, M) != (table.num_rows, table.max_seq) or ns != table.num_slots:
        raise ValueError("segment table does not match the input shape")
    if tuple(y.shape) != (B, M, N):
        raise ValueError(f"base_output shape {tuple(y.shape)} != {(B, M, N)}")
    if not y.is_contiguous():
        raise ValueError("base_output must be contiguous (it is updated in place)")
    if tmp is None:
        tmp = torch.empty((B, M, R), device=dev, dtype=x.dtype)
    if B == 0 or M == 0:
        return y
    xc = x.contiguous()
    wa = weights_a.contiguous()
    wb = weights_b.contiguous()
    if not (xc.dtype == wa.dtype == wb.dtype == y.dtype == tmp.dtype):
        raise TypeError("x, weights, tmp and base_output must share one dtype")
    rk = _as(lora_ranks, torch.int32)
    sc = _as(scalings, torch.float32)
    _native.call(
        "plora_sgmv_shrink_expand",
        xc.data_ptr(), wa.data_ptr(), tmp.data_ptr(), wb.data_ptr(), y.data_ptr(),
        rk.data_ptr(), sc.data_ptr(), table.slot_start.data_ptr(), table.token_index.data_ptr(),
        table.num_tokens, K, R, N, ns, dtype_code(xc.dtype), _stream(dev),
    )
    return y


def sgmv_lora_a_fwd(
    x: torch.Tensor,
    weights: torch.Tensor,
    seq_lens: torch.Tensor,
    weight_indices: torch.Tensor,
    lora_ranks: torch.Tensor,
    stack_num: int = 1,
) -> torch.Tensor:
    """LoRA-A shrink with the reference signature (src/polylora/sgmv.py:141-175).

    Returns ``(B, M, N_max)`` in ``x.dtype``; entries of inactive tokens are
    left uninitialised exactly as in the reference.
    """
    assert x.is_contiguous() and weights.is_contiguous()
    assert x.dim() == 3 and weights.dim() == 3
    B, M, K = x.shape
    ns, kw, n_max = weights.shape
    assert kw == K, f"K mismatch: x={K}, weights={kw}"
    output = torch.empty((B, M, n_max), device=x.device, dtype=x.dtype)
    if B == 0 or M == 0 or n_max == 0:
        return output
    dev = _require_cuda(x, weights, seq_lens, weight_indices, lora_ranks)
    if weights.dtype != x.dtype:
        raise TypeError(f"dtype mismatch: x={x.dtype}, weights={weights.dtype}")
    sl = _as(seq_lens, torch.int32)
    wi = _as(weight_indices, torch.int64)
    rk = _as(lora_ranks, torch.int32)
    ws = _workspace(dev, _native.workspace_size(B, M, ns))
    _native.call(
        "plora_sgmv_a_fwd",
        x.data_ptr(), weights.data_ptr(), output.data_ptr(), sl.data_ptr(), wi.data_ptr(),
        rk.data_ptr(), B, M, K, n_max, ns, stack_num, dtype_code(x.dtype),
        ws.data_ptr(), ws.numel(), _stream(dev),
    )
    return output


def sgmv_lora_b_fwd(
    x: torch.Tensor,
    weights: torch.Tensor,
    seq_lens: torch.Tensor,
    weight_indices: torch.Tensor,
    lora_ranks: torch.Tensor,
    scalings: torch.Tensor,
    base_output: torch.Tensor | None = None,
) -> torch.Tensor:
    """LoRA-B expand with the reference signature (src/polylora/sgmv.py:278-328).

    Adds ``scalings[slot] * x · B[slot]`` into ``base_output`` in place and
    returns it (a zero tensor is allocated when it is None, as the reference
    does).
    """
    assert x.is_contiguous() and weights.is_contiguous()
    assert x.dim() == 3 and weights.dim() == 3
    B, M, k_max = x.shape
    ns, kw, N = weights.shape
    assert kw == k_max, f"K mismatch: x={k_max}, weights={kw}"
    if base_output is None:
        output = torch.zeros((B, M, N), device=x.device, dtype=x.dtype)
    else:
        assert base_output.shape == (B, M, N)
        output = base_output
    if B == 0 or M == 0:
        return output
    dev = _require_cuda(x, weights, seq_lens, weight_indices, lora_ranks, scalings, output)
    if not output.is_contiguous():
        raise ValueError("base_output must be contiguous (it is updated in place)")
    if not (x.dtype == weights.dtype == output.dtype):
        raise TypeError(f"dtype mismatch: x={x.dtype}, weights={weights.dtype}, out={output.dtype}")
    sl = _as(seq_lens, torch.int32)
    wi = _as(weight_indices, torch.int64)
    rk = _as(lora_ranks, torch.int32)
    sc = _as(scalings, torch.float32)
    ws = _workspace(dev, _native.workspace_size(B, M, ns))
    _native.call(
        "plora_sgmv_b_fwd",
        x.data_ptr(), weights.data_ptr(), output.data_ptr(), sl.data_ptr(), wi.data_ptr(),
        rk.data_ptr(), sc.data_ptr(), B, M, k_max, N, ns, dtype_code(x.dtype),
        ws.data_ptr(), ws.numel(), _stream(dev),
    )
    return output


def build_flat_schedule(
    seq_lens: torch.Tensor,
    n_eff_per_batch: torch.Tensor,
    block_m: int,
    block_n: int,
) -> tuple[torch.Tensor, torch.Tensor, int]:
    """The reference's flat tile schedule (src/polylora/sgmv.py:29-61), on device.

    Returns ``(cum_tiles, num_n_tiles, total_tiles)`` like the reference; the
    total is read back with one ``.item()`` to keep the reference signature.
    """
    dev = _require_cuda(seq_lens, n_eff_per_batch)
    sl = _as(seq_lens, torch.int32)
    ne = _as(n_eff_per_batch, torch.int32)
    B = int(sl.shape[0])
    cum_tiles = torch.empty(B + 1, dtype=torch.int32, device=dev)
    num_n_tiles = torch.empty(B, dtype=torch.int32, device=dev)
    _native.call(
        "plora_flat_schedule",
        sl.data_ptr(), ne.data_ptr(), B, block_m, block_n,
        cum_tiles.data_ptr(), num_n_tiles.data_ptr() if B else 0, _stream(dev),
    )
    return cum_tiles, num_n_tiles, int(cum_tiles[-1].item())
