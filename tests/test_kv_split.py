"""Host logic of the multi-GPU sequence split, on CPU: range arithmetic, and a 2-rank gloo run in which
each rank computes its part's (o, m, l) partial with the oracle, the parts are all-gathered, and the
restated log-sum-exp merge (oracle.rs_lse_combine, ops.cpp:9370-9438) reproduces the full attention."""
import os
import socket

import numpy as np
import pytest

import oracle as O
from klein_b200.kv_split import TILE, kv_range, local_bounds, packed_part_floats


@pytest.mark.parametrize("n_kv,world", [(262144, 1), (262144, 2), (262144, 8), (1000, 3), (65, 4), (64, 8), (1, 2)])
def test_kv_range_partition(n_kv, world):
    prev = 0
    for r in range(world):
        lo, hi = kv_range(n_kv, world, r)
        assert lo == prev and lo <= hi
        assert lo % TILE == 0 or lo == n_kv
        prev = hi
    assert prev == n_kv


def partial_f64(q, kd, vd, mask, scale):
    """(o, m, l) of one part in the layout of kb_flash_attn_ext_partial: m in log2 units."""
    n_q, H, D = q.shape
    G = H // kd.shape[1]
    o = np.zeros((n_q, H, D))
    ml = np.zeros((n_q, H, 2))
    for h in range(H):
        s = (q[:, h].astype(np.float64) @ kd[:, h // G].T.astype(np.float64)) * scale * np.log2(np.e)
        s = s + np.where(np.isfinite(mask), 0.0, -np.inf)
        m = s.max(1)
        ok = np.isfinite(m)
        mm = np.where(ok, m, 0.0)
        p = np.exp2(s - mm[:, None])
        o[:, h] = p @ vd[:, h // G].astype(np.float64)
        ml[:, h, 0] = mm
        ml[:, h, 1] = p.sum(1)
    return o, ml


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_q, n_kv, result_path):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, kc, vc, kd, vd = O.make_fa_inputs(2024, n_q, n_kv, H=24, H_kv=4, D=64)
    lo, hi = kv_range(n_kv, world, rank)
    pos0, kv_lo = local_bounds(lo, n_kv - n_q, 0)
    mask = O.rs_visible_mask(n_q, hi - lo, pos0, kv_lo=kv_lo)
    o, ml = partial_f64(O.q_round_f16(q), kd[lo:hi], vd[lo:hi], mask, 1 / 8)
    rows = n_q * 24
    part = torch.zeros(packed_part_floats(rows, 64), dtype=torch.float64)
    part[: rows * 64] = torch.from_numpy(o.reshape(-1))
    part[rows * 64:] = torch.from_numpy(ml.reshape(-1))
    gathered = [torch.zeros_like(part) for _ in range(world)]
    dist.all_gather(gathered, part)
    if rank == 0:
        g = torch.stack(gathered).numpy()
        o_parts = g[:, : rows * 64].reshape(world, rows, 64)
        ml_parts = g[:, rows * 64:].reshape(world, rows, 2)
        # kb partials carry the max in log2 units; the restated merge (like ggml's) works in natural units
        merged = O.rs_lse_combine(o_parts, ml_parts[..., 0] * np.log(2.0), ml_parts[..., 1])
        np.save(result_path, merged)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_two_rank_split_matches_full(tmp_path, world):
    """world ranks (2, or 4 with a ragged last range) each attend over their cells; the merge equals the whole."""
    import torch.multiprocessing as mp

    n_q, n_kv = 4, 1000
    out = str(tmp_path / "merged.npy")
    mp.start_processes(_worker, args=(world, _free_port(), n_q, n_kv, out), nprocs=world, start_method="spawn")
    merged = np.load(out).reshape(n_q, 24, 64)
    q, kc, vc, kd, vd = O.make_fa_inputs(2024, n_q, n_kv, H=24, H_kv=4, D=64)
    full = O.rs_flash_attn_f64(O.q_round_f16(q), kd, vd, mask=O.rs_visible_mask(n_q, n_kv, n_kv - n_q), scale=1 / 8)
    assert np.abs(merged - full).max() <= 1e-5 * np.abs(full).max()
