"""Integer oracle: the reference flat tile schedule and the slot-grouped
segment table (numpy / plain Python; bit-exact targets)."""

from __future__ import annotations

import numpy as np


def flat_schedule(seq_lens, n_eff, block_m, block_n):
    """src/polylora/sgmv.py:29-61 (_build_flat_schedule):
    cum_tiles (B+1,) int32, num_n_tiles (B,) int32, total_tiles int."""
    seq_lens = np.asarray(seq_lens, dtype=np.int64)
    n_eff = np.asarray(n_eff, dtype=np.int64)
    num_m = (seq_lens + block_m - 1) // block_m
    num_n = (n_eff + block_n - 1) // block_n
    tiles = (num_m * num_n).astype(np.int32)
    tiles = np.where((seq_lens == 0) | (n_eff == 0), 0, tiles).astype(np.int32)
    cum = np.zeros(len(seq_lens) + 1, dtype=np.int32)
    cum[1:] = np.cumsum(tiles, dtype=np.int64).astype(np.int32)
    return cum, num_n.astype(np.int32), int(cum[-1])


def n_eff_expand(ranks_per_row, out_features):
    """src/polylora/sgmv.py:304-309: N for rows with rank > 0, else 0."""
    r = np.asarray(ranks_per_row)
    return np.where(r > 0, out_features, 0).astype(np.int32)


def segments(weight_indices, seq_lens, ranks, max_seq, num_slots):
    """Slot-grouped table of the active tokens (definition of the device table).

    A token (row, m) is active when m < min(seq_lens[row], max_seq) and
    ranks[weight_indices[row]] > 0 — the work predicate of the reference
    kernels (sgmv.py:92-97, 226-231) and of layers.py:127-131.  Tokens are
    ordered by (slot, row, m); slot_start is the exclusive prefix of counts.
    """
    wi = np.asarray(weight_indices, dtype=np.int64)
    sl = np.asarray(seq_lens, dtype=np.int64)
    rk = np.asarray(ranks, dtype=np.int64)
    per_slot: list[list[int]] = [[] for _ in range(num_slots)]
    for row in range(len(wi)):
        slot = int(wi[row])
        if slot < 0 or slot >= num_slots:
            continue
        length = int(min(max(sl[row], 0), max_seq))
        if rk[slot] <= 0 or length == 0:
            continue
        per_slot[slot].extend(row * max_seq + m for m in range(length))
    slot_start = np.zeros(num_slots + 1, dtype=np.int32)
    slot_start[1:] = np.cumsum([len(p) for p in per_slot])
    token_index = np.array([t for p in per_slot for t in p], dtype=np.int32)
    return slot_start, token_index
