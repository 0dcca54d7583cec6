"""Sequence split of decode / verify attention across the GPUs of one node.

Each rank holds one contiguous range of every layer's KV cells, computes unnormalised partials of the
attention over its range (kb_flash_attn_ext_partial), and the partials of all ranks are merged with the
log-sum-exp rule (kb_lse_combine) after an all-gather — the split-KV decomposition ggml applies across CPU
threads (ops.cpp:9489-9520 + reduce_partials :9370-9438), applied across devices.

The range arithmetic here is plain integer work shared by bench.py and the tests.
"""
from __future__ import annotations

TILE = 64  # keys per pipeline stage of the streaming kernel: ranges start on a tile boundary


def kv_range(n_kv: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) cells of `rank`; ranges are contiguous, cover [0, n_kv), and start on a TILE boundary."""
    per = (n_kv + world - 1) // world
    per = (per + TILE - 1) // TILE * TILE
    lo = min(rank * per, n_kv)
    hi = min(lo + per, n_kv)
    return lo, hi


def local_bounds(lo: int, pos0: int, kv_lo: int) -> tuple[int, int]:
    """Causal bounds of a part in its own coordinates (cell 0 = global cell lo)."""
    return pos0 - lo, max(kv_lo - lo, 0)


def packed_part_floats(rows: int, head_dim: int) -> int:
    """Floats of one rank's packed partial: o [rows][head_dim] followed by (m, l) [rows][2], padded to a
    multiple of 4 floats so that every part of an all-gathered buffer stays 16-byte aligned."""
    return rows * head_dim + (rows * 2 + 3) // 4 * 4
