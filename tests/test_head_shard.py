"""Head sharding of DeltaNet and prefill attention across ranks, on CPU: every rank runs the restated op on its
slice of heads (gdn_head_shard / fa_head_shard choose the key and KV heads), and the slices put together equal
the whole op, exactly; plus a 2-rank gloo run that all-gathers the DeltaNet slices."""
import os
import socket

import numpy as np
import pytest

import oracle as O
from klein_b200.kv_split import fa_head_shard, gdn_head_shard, head_range


@pytest.mark.parametrize("n,world", [(48, 1), (48, 2), (48, 8), (48, 5), (24, 8), (3, 4)])
def test_head_range_partition(n, world):
    prev = 0
    for r in range(world):
        lo, hi = head_range(n, world, r)
        assert lo == prev and lo <= hi
        prev = hi
    assert prev == n


def gdn_slice(q, k, v, g, beta, s0, K, lo, hi, kidx):
    """The op on value heads [lo, hi) with key heads kidx, unpacked to (attn [T][n][S], states [K][n][S][S])."""
    T, S = q.shape[1], q.shape[3]
    n = hi - lo
    out = O.rs_gated_delta_net_f64(q[:, :, kidx], k[:, :, kidx], v[:, :, lo:hi], g[:, :, lo:hi], beta[:, :, lo:hi],
                                   s0[:, lo:hi], K)
    attn = out[: T * n * S].reshape(T, n, S)
    states = out[T * n * S:].reshape(K, n, S, S)
    return attn, states


@pytest.mark.parametrize("world", [2, 3, 8])
def test_gdn_head_shards_equal_whole(world):
    H_k, H_v, S, T, K = 4, 12, 16, 3, 2
    q, k, v, g, beta, s0 = O.make_gdn_inputs(11, T, H_k=H_k, H_v=H_v, S=S)
    attn, states = gdn_slice(q, k, v, g, beta, s0, K, 0, H_v, list(range(H_v)) if H_k == H_v else
                             [h % H_k for h in range(H_v)])
    # the whole op itself, as the reference runs it (H_k key heads broadcast over H_v)
    whole = O.rs_gated_delta_net_f64(q, k, v, g, beta, s0, K)
    assert np.array_equal(whole[: T * H_v * S].reshape(T, H_v, S), attn)
    for r in range(world):
        lo, hi, kidx = gdn_head_shard(H_k, H_v, world, r)
        if lo == hi:
            continue
        a, st = gdn_slice(q, k, v, g, beta, s0, K, lo, hi, kidx)
        assert np.array_equal(a, attn[:, lo:hi])
        assert np.array_equal(st, states[:, lo:hi])


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_fa_head_shards_equal_whole(world):
    n_q, n_kv = 8, 96
    q, kc, vc, kd, vd = O.make_fa_inputs(5, n_q, n_kv, H=24, H_kv=4, D=64)
    mask = O.rs_visible_mask(n_q, n_kv, 0)  # causal prefill of 8 tokens over their own 96-cell prefix
    whole = O.rs_flash_attn_f64(q, kd, vd, mask=mask, scale=1 / 8)
    for r in range(world):
        lo, hi, kv_lo, kv_hi = fa_head_shard(24, 4, world, r)
        part = O.rs_flash_attn_f64(q[:, lo:hi], kd[:, kv_lo:kv_hi], vd[:, kv_lo:kv_hi], mask=mask, scale=1 / 8)
        assert np.array_equal(part, whole[:, lo:hi])


def test_fa_head_shard_rejects_uneven_groups():
    with pytest.raises(ValueError):
        fa_head_shard(24, 4, 5, 1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    H_k, H_v, S, T, K = 4, 12, 16, 3, 2
    q, k, v, g, beta, s0 = O.make_gdn_inputs(12, T, H_k=H_k, H_v=H_v, S=S)
    lo, hi, kidx = gdn_head_shard(H_k, H_v, world, rank)
    a, st = gdn_slice(q, k, v, g, beta, s0, K, lo, hi, kidx)
    # equal slices here (12 heads over 2 ranks), so a plain all-gather suffices
    parts = [torch.zeros(a.size + st.size, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(np.concatenate([a.reshape(-1), st.reshape(-1)])))
    if rank == 0:
        n = hi - lo
        attn = np.concatenate([p[: T * n * S].numpy().reshape(T, n, S) for p in parts], axis=1)
        states = np.concatenate([p[T * n * S:].numpy().reshape(K, n, S, S) for p in parts], axis=1)
        np.savez(result_path, attn=attn, states=states)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gdn_heads_all_gathered(tmp_path):
    import torch.multiprocessing as mp

    out = str(tmp_path / "gdn.npz")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    got = np.load(out)
    H_k, H_v, S, T, K = 4, 12, 16, 3, 2
    whole = O.rs_gated_delta_net_f64(*O.make_gdn_inputs(12, T, H_k=H_k, H_v=H_v, S=S), K)
    assert np.array_equal(got["attn"], whole[: T * H_v * S].reshape(T, H_v, S))
    assert np.array_equal(got["states"], whole[T * H_v * S:].reshape(K, H_v, S, S))
