"""Float oracle of the SGMV shrink / expand and the LoRA forward (numpy).

Arrays are float32 holding values already representable in the tensor dtype
(bf16 / fp16 inputs are passed upcast).  ``dtype`` names the rounding applied
where the reference stores in the tensor dtype.
"""

from __future__ import annotations

import numpy as np


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round-to-nearest-even of float32 values to bf16/fp16/fp32, kept as float32."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "float32":
        return a.copy()
    if dtype == "float16":
        return a.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        u = a.view(np.uint32).astype(np.uint64)
        nan = np.isnan(a)
        rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        out = rounded.astype(np.uint32).view(np.float32)
        return np.where(nan, a, out).astype(np.float32)
    raise ValueError(dtype)


def active_rows(seq_lens, weight_indices, ranks, max_seq):
    """Per row: (slot, valid tokens, rank).  Mirrors the masks of
    src/polylora/sgmv.py:92-97 (seq_len == 0 / rank-0 rows do nothing) and
    layers.py:127-131 of the torch path."""
    out = []
    for b, slot in enumerate(np.asarray(weight_indices).tolist()):
        rank = int(ranks[slot])
        length = int(min(max(int(seq_lens[b]), 0), max_seq))
        out.append((int(slot), length, rank))
    return out


def shrink(x, A, seq_lens, weight_indices, ranks, stack_num=1, dtype="bfloat16"):
    """src/polylora/sgmv.py:63-138 — tmp[b,m,n] = sum_k x[b,m,k] A[w_b,k,n] for
    m < seq_len, n < rank*stack_num (fp32 accumulate, stored in ``dtype``).

    Returns (tmp, written) where ``written`` marks the entries the reference
    defines (everything else is uninitialised memory there)."""
    B, M, K = x.shape
    n_max = A.shape[2]
    tmp = np.zeros((B, M, n_max), dtype=np.float32)
    written = np.zeros((B, M, n_max), dtype=bool)
    for b, (slot, length, rank) in enumerate(active_rows(seq_lens, weight_indices, ranks, M)):
        n_eff = min(rank * stack_num, n_max)
        if length == 0 or n_eff <= 0:
            continue
        acc = x[b, :length].astype(np.float64) @ A[slot, :, :n_eff].astype(np.float64)
        tmp[b, :length, :n_eff] = round_to(acc.astype(np.float32), dtype)
        written[b, :length, :n_eff] = True
    return tmp, written


def expand(tmp, Bw, seq_lens, weight_indices, ranks, scales, y, dtype="bfloat16"):
    """src/polylora/sgmv.py:178-275 — y[b,m,:] += scale[w] * sum_{k<min(K,rank)}
    tmp[b,m,k] B[w,k,:] for m < seq_len and rank > 0, other rows untouched.
    One rounding of (y + scale*acc) into ``dtype`` (the reference rounds the
    product first; both are within the stated tolerance of the fp32 form)."""
    B, M, k_max = tmp.shape
    out = np.array(y, dtype=np.float32, copy=True)
    for b, (slot, length, rank) in enumerate(active_rows(seq_lens, weight_indices, ranks, M)):
        kr = min(k_max, rank)
        if length == 0 or kr <= 0:
            continue
        acc = tmp[b, :length, :kr].astype(np.float64) @ Bw[slot, :kr, :].astype(np.float64)
        out[b, :length] = round_to((out[b, :length] + np.float32(scales[slot]) * acc).astype(np.float32), dtype)
    return out


def lora_forward_fp32(x, A, Bw, seq_lens, weight_indices, ranks, scales, y):
    """fp32-accumulated form of src/polylora/layers.py:127-133:
    y[b,:L] + scale * (x[b,:L] @ A[s,:,:r]) @ B[s,:r,:], no intermediate rounding."""
    B, M, _ = x.shape
    out = np.array(y, dtype=np.float64, copy=True)
    for b, (slot, length, rank) in enumerate(active_rows(seq_lens, weight_indices, ranks, M)):
        if rank == 0 or length == 0:
            continue
        r = min(rank, A.shape[2])
        t = x[b, :length].astype(np.float64) @ A[slot, :, :r].astype(np.float64)
        out[b, :length] += float(scales[slot]) * (t @ Bw[slot, :r, :].astype(np.float64))
    return out.astype(np.float32)


def lora_forward_grouped(x, A, Bw, seq_lens, weight_indices, ranks, scales, y):
    """Same math as :func:`lora_forward_fp32` with rows of one slot batched into
    one matmul pair (fp32, BLAS threads).  The timed CPU baseline."""
    B, M, K = x.shape
    out = np.array(y, dtype=np.float32, copy=True)
    rows = active_rows(seq_lens, weight_indices, ranks, M)
    by_slot: dict[int, list[int]] = {}
    for b, (slot, length, rank) in enumerate(rows):
        if rank > 0 and length > 0:
            by_slot.setdefault(slot, []).append(b)
    for slot, members in by_slot.items():
        r = min(int(ranks[slot]), A.shape[2])
        if M == 1:
            xs = x[members, 0, :]
            out[members, 0, :] += np.float32(scales[slot]) * ((xs @ A[slot, :, :r]) @ Bw[slot, :r, :])
        else:
            for b in members:
                length = rows[b][1]
                out[b, :length] += np.float32(scales[slot]) * ((x[b, :length] @ A[slot, :, :r]) @ Bw[slot, :r, :])
    return out


# One unit in the last place, relative, of each storage type: outputs are
# rounded once (or, in the reference's bf16 path, twice) into this type.
ULP = {"float32": 2.0**-23, "float16": 2.0**-10, "bfloat16": 2.0**-7}


def lora_err(out, ref, y, dtype: str) -> float:
    """Error of a LoRA output against an fp32-accumulated reference, relative to
    the size of the LoRA delta: max over elements of
    max(0, |out - ref| - ULP[dtype]*|ref|) / max|ref - y|.
    The ULP allowance absorbs rounding the output ``y + delta`` into ``dtype``;
    what remains is error in the delta itself."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    if ref.size == 0:
        return 0.0
    scale = max(float(np.max(np.abs(ref - y))), 1e-30)
    excess = np.maximum(np.abs(out - ref) - ULP[dtype] * np.abs(ref), 0.0)
    return float(np.max(excess)) / scale


def lora_err_strict(out, ref, y, dtype: str) -> float:
    """As :func:`lora_err`, with half an output ulp of allowance instead of
    one: max over elements of max(0, |out - ref| - ULP[dtype]/2 * |ref|) /
    max|ref - y|.  Half an ulp is exactly the rounding of ``y + delta`` into
    ``dtype``, so what remains is the error of the LoRA delta itself (its
    accumulation and its own rounding).  With ``y = 0`` the output is the
    delta and this is an element-wise check of it."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    if ref.size == 0:
        return 0.0
    scale = max(float(np.max(np.abs(ref - y))), 1e-30)
    excess = np.maximum(np.abs(out - ref) - 0.5 * ULP[dtype] * np.abs(ref), 0.0)
    return float(np.max(excess)) / scale


def rel_err(out, ref) -> float:
    """Normwise max relative error: max|out - ref| / max|ref|."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = max(float(np.max(np.abs(ref))) if ref.size else 0.0, 1e-30)
    return float(np.max(np.abs(out - ref))) / denom if ref.size else 0.0
