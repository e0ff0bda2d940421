"""LoRA op on HOST buffers: x and the base output in pinned host memory, the
result written back to host memory.

The reference operators take device tensors (src/polylora/sgmv.py:141-175 and
278-328); a caller holding host buffers copies in, calls them, and copies out,
one direction at a time.  :class:`HostLoraPipeline` runs the same op
(``out = base + scale[slot] * (x . A[slot]) . B[slot]`` per active token) over
row chunks instead: chunk c+1's host-to-device copy runs on one copy stream
while chunk c is computed and chunk c-1 is copied back on another, so the two
PCIe directions overlap each other and the kernels.  Each chunk builds its own
segment table on the device and runs :func:`sgmv_shrink_expand`; a token's
result does not depend on the chunking.

Adapter slot state (weights, ranks, scalings) stays on the device, as in the
GPU cache; per-row metadata (``seq_lens``, ``weight_indices``) travels with
the rows.

In place (``out_host`` is ``base_output_host``) with pinned host buffers, only
the rows the op reads and writes cross the bus: after a chunk's segment table
is built, a kernel reads x and the base output of the table's tokens from the
mapped host memory (``plora_gather_token_rows``), and after the op another
writes those output rows back (``plora_scatter_token_rows``).  Rows of
``__base__`` or rank-0 tokens, and padding, stay in host memory untouched,
which is their result (the op leaves them unchanged, as the reference's
in-place expand does).
"""

from __future__ import annotations

import torch

from . import _native
from .sgmv import _require_cuda, build_segments, sgmv_shrink_expand


class HostLoraPipeline:
    """Row-chunked host -> device -> host pipeline for the batched LoRA op.

    ``chunks`` row groups per call (at most one per row).  Device staging
    buffers are kept between calls of the same shape; events order a call's
    copies into a chunk's buffers after the previous call's copy out of them.
    The results are in ``out`` once the caller's current stream reaches the
    point after the call (e.g. ``torch.cuda.current_stream().synchronize()``).
    """

    def __init__(self, device: torch.device | int | str, chunks: int = 4, active_rows: bool = True) -> None:
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("HostLoraPipeline needs a CUDA device; there is no CPU fallback")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if chunks < 1:
            raise ValueError(f"chunks must be >= 1, got {chunks}")
        self.chunks = int(chunks)
        self.active_rows = bool(active_rows)  # in-place pinned calls move the table's rows only
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self._key = None
        self._bufs: dict[str, torch.Tensor] = {}
        self._out_free: list[torch.cuda.Event] = []
        self._in_ready: list[torch.cuda.Event] = []
        self._done: list[torch.cuda.Event] = []
        self._tables_built: list[torch.cuda.Event] = []

    def _buffers(self, x_host, base_host, weights_a, seq_host, wi_host):
        B, M, K = x_host.shape
        N = base_host.shape[2]
        R = weights_a.shape[2]
        key = (B, M, K, N, R, x_host.dtype, seq_host.dtype, wi_host.dtype)
        if key != self._key:
            torch.cuda.current_stream(self.device).synchronize()
            self.h2d.synchronize()
            self.d2h.synchronize()
            dev, dt = self.device, x_host.dtype
            self._bufs = {
                "x": torch.empty((B, M, K), dtype=dt, device=dev),
                "y": torch.empty((B, M, N), dtype=dt, device=dev),
                "tmp": torch.empty((B, M, R), dtype=dt, device=dev),
                "seq": torch.empty(B, dtype=seq_host.dtype, device=dev),
                "wi": torch.empty(B, dtype=wi_host.dtype, device=dev),
            }
            self._out_free = [torch.cuda.Event() for _ in range(self.chunks)]
            self._in_ready = [torch.cuda.Event() for _ in range(self.chunks)]
            self._done = [torch.cuda.Event() for _ in range(self.chunks)]
            self._tables_built = [torch.cuda.Event() for _ in range(self.chunks)]
            self._key = key
        return self._bufs

    def __call__(
        self,
        x_host: torch.Tensor,
        weights_a: torch.Tensor,
        weights_b: torch.Tensor,
        seq_lens_host: torch.Tensor,
        weight_indices_host: torch.Tensor,
        lora_ranks: torch.Tensor,
        scalings: torch.Tensor,
        base_output_host: torch.Tensor,
        out_host: torch.Tensor,
    ) -> torch.Tensor:
        """``out_host = base_output_host + LoRA(x_host)``; returns ``out_host``.

        x_host (B, M, K) and base_output_host / out_host (B, M, N) are host
        tensors (pinned, or the copies are not asynchronous); weights_a
        (NS, K, R), weights_b (NS, R, N), lora_ranks and scalings (NS,) are on
        the pipeline's device; seq_lens_host and weight_indices_host (B,) are
        host tensors.  ``out_host`` may be ``base_output_host``.  The host
        inputs must be complete when the call is made (the copies in start at
        once, not after work queued on the caller's stream), and no host buffer
        may be rewritten before the results are ready."""
        _require_cuda(weights_a, weights_b, lora_ranks, scalings)
        if weights_a.device != self.device:
            raise ValueError(f"weights on {weights_a.device}, pipeline on {self.device}")
        for name, t in (("x", x_host), ("base_output", base_output_host), ("out", out_host),
                        ("seq_lens", seq_lens_host), ("weight_indices", weight_indices_host)):
            if t.device.type != "cpu":
                raise ValueError(f"{name} must be a host tensor, got one on {t.device}")
            if not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
        B, M, K = x_host.shape
        if base_output_host.shape[:2] != (B, M) or out_host.shape != base_output_host.shape:
            raise ValueError(f"base_output {tuple(base_output_host.shape)} / out {tuple(out_host.shape)} "
                             f"do not match x {tuple(x_host.shape)}")
        if tuple(seq_lens_host.shape) != (B,) or tuple(weight_indices_host.shape) != (B,):
            raise ValueError("seq_lens and weight_indices must have one entry per row")
        if not (x_host.dtype == base_output_host.dtype == out_host.dtype == weights_a.dtype == weights_b.dtype):
            raise TypeError("x, base_output, out and the weights must share one dtype")
        if B == 0 or M == 0:
            out_host.copy_(base_output_host)
            return out_host
        bufs = self._buffers(x_host, base_output_host, weights_a, seq_lens_host, weight_indices_host)
        compute = torch.cuda.current_stream(self.device)
        in_place = out_host.data_ptr() == base_output_host.data_ptr()
        if self.active_rows and in_place and x_host.is_pinned() and base_output_host.is_pinned():
            return self._active_rows(x_host, weights_a, weights_b, seq_lens_host, weight_indices_host, lora_ranks,
                                     scalings, out_host, bufs, compute)
        n = min(self.chunks, B)
        bounds = [B * c // n for c in range(n + 1)]
        for c in range(n):
            r0, r1 = bounds[c], bounds[c + 1]
            if r1 == r0:
                continue
            xs, ys, ts = bufs["x"][r0:r1], bufs["y"][r0:r1], bufs["tmp"][r0:r1]
            ss, ws = bufs["seq"][r0:r1], bufs["wi"][r0:r1]
            with torch.cuda.stream(self.h2d):
                self.h2d.wait_event(self._out_free[c])  # the previous call's copy out of these rows
                xs.copy_(x_host[r0:r1], non_blocking=True)
                ys.copy_(base_output_host[r0:r1], non_blocking=True)
                ss.copy_(seq_lens_host[r0:r1], non_blocking=True)
                ws.copy_(weight_indices_host[r0:r1], non_blocking=True)
            self._in_ready[c].record(self.h2d)
            compute.wait_event(self._in_ready[c])
            table = build_segments(ws, ss, lora_ranks, M)
            self._tables_built[c].record(compute)  # the metadata buffers are free again
            sgmv_shrink_expand(xs, weights_a, weights_b, ys, table, lora_ranks, scalings, tmp=ts)
            self._done[c].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self._done[c])
                out_host[r0:r1].copy_(ys, non_blocking=True)
                self._out_free[c].record(self.d2h)
        compute.wait_stream(self.d2h)
        return out_host

    def _active_rows(self, x_host, weights_a, weights_b, seq_host, wi_host, lora_ranks, scalings, y_host, bufs,
                     compute):
        """The in-place call moving only the segment table's rows.  Per chunk:
        on the copy stream the metadata and the chunk's segment table (so that
        it is built while the previous chunk's rows move); on the compute
        stream the gather of the table's x and y rows from mapped host memory
        (after the previous call's scatter of those rows) and the op; on the
        second stream the scatter of its y rows back."""
        B, M, _ = x_host.shape
        n = min(self.chunks, B)
        bounds = [B * c // n for c in range(n + 1)]
        # the tables read lora_ranks on the copy stream: after the caller's work on it
        self.h2d.wait_stream(compute)
        for c in range(n):
            r0, r1 = bounds[c], bounds[c + 1]
            if r1 == r0:
                continue
            xs, ys, ts = bufs["x"][r0:r1], bufs["y"][r0:r1], bufs["tmp"][r0:r1]
            ss, ws = bufs["seq"][r0:r1], bufs["wi"][r0:r1]
            with torch.cuda.stream(self.h2d):
                self.h2d.wait_event(self._tables_built[c])  # the previous call's table read these
                ss.copy_(seq_host[r0:r1], non_blocking=True)
                ws.copy_(wi_host[r0:r1], non_blocking=True)
                table = build_segments(ws, ss, lora_ranks, M)
                self._tables_built[c].record(self.h2d)
            compute.wait_event(self._tables_built[c])
            compute.wait_event(self._out_free[c])  # the previous call's scatter out of these rows
            for t in (table.slot_start, table.token_index):
                t.record_stream(compute)
                t.record_stream(self.d2h)
            _native.token_rows(x_host[r0:r1], xs, table, to_host=False)
            _native.token_rows(y_host[r0:r1], ys, table, to_host=False)
            sgmv_shrink_expand(xs, weights_a, weights_b, ys, table, lora_ranks, scalings, tmp=ts)
            self._done[c].record(compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self._done[c])
                _native.token_rows(y_host[r0:r1], ys, table, to_host=True, stream=self.d2h.cuda_stream)
                self._out_free[c].record(self.d2h)
        compute.wait_stream(self.d2h)
        return y_host
