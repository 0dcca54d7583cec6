"""Sequence split of decode / verify attention across the GPUs of one node, and the head shards of DeltaNet and
prefill attention.

Each rank holds one contiguous range of every layer's KV cells, computes unnormalised partials of the
attention over its range (kb_flash_attn_ext_partial), and the partials of all ranks are merged with the
log-sum-exp rule (kb_lse_combine) after an all-gather — the split-KV decomposition ggml applies across CPU
threads (ops.cpp:9489-9520 + reduce_partials :9370-9438), applied across devices.

DeltaNet and prefill attention shard by heads instead, with no exchange: each rank calls the same op on its
slice of heads (gdn_head_shard, fa_head_shard), choosing the key / KV heads so that the op's own head mapping on
the slice is the reference's mapping on the whole.

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


def head_range(n_heads: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) heads of `rank`: contiguous, ceil(n_heads / world) per rank, covering [0, n_heads)."""
    per = (n_heads + world - 1) // world
    lo = min(rank * per, n_heads)
    return lo, min(lo + per, n_heads)


def gdn_head_shard(H_k: int, H_v: int, world: int, rank: int) -> tuple[int, int, list[int]]:
    """DeltaNet value heads [lo, hi) of `rank` and the key head each of them reads: h % H_k (ops.cpp:11199,
    gated_delta_net.cu). The rank gathers q and k heads in that order and calls the op with H_k = H_v = hi - lo,
    so its local head j reads local key head j; state, snapshots and outputs are the [lo, hi) slices of the
    whole op's."""
    lo, hi = head_range(H_v, world, rank)
    return lo, hi, [h % H_k for h in range(lo, hi)]


def fa_head_shard(H: int, H_kv: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """Query heads [q_lo, q_hi) and KV heads [kv_lo, kv_hi) of `rank` for head-sharded attention. The op maps local
    query head j to local KV head j // ((q_hi - q_lo) / (kv_hi - kv_lo)); that equals the global mapping
    h // (H / H_kv) (ggml's GQA rule) when each rank's heads cover whole GQA groups or part of one group
    (qwen35's 24 / 4 heads at 1, 2, 4, 8 ranks). Other splits raise ValueError."""
    G = H // H_kv
    lo, hi = head_range(H, world, rank)
    if lo == hi:
        return lo, hi, 0, 0
    kv_lo, kv_hi = lo // G, (hi - 1) // G + 1
    n, nk = hi - lo, kv_hi - kv_lo
    if n % nk or any((lo + j) // G - kv_lo != j // (n // nk) for j in range(n)):
        raise ValueError(f"{H} query / {H_kv} KV heads over {world} ranks split a GQA group unevenly")
    return lo, hi, kv_lo, kv_hi
