"""GPU parity of the gated DeltaNet kernels, the snapshot/rollback path and the KV-cache write, against the
CPU oracle (restated f64 recurrence, ggml's own CPU op, restated set_rows/rollback)."""
import numpy as np
import pytest

import oracle as O
from parity import DELTANET_TOL, rel_err

pytestmark = pytest.mark.gpu


def to_dev(cuda, *arrays):
    import torch

    return [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in arrays]


def split_packed(out, S, H, T, n_seqs, K):
    attn = out[: S * H * T * n_seqs].reshape(n_seqs, T, H, S)
    slots = out[S * H * T * n_seqs:].reshape(K, n_seqs, H, S, S)
    return attn, slots


@pytest.mark.parametrize("kda", [False, True])
def test_config1_verify_step(kb, cuda, kda):
    """config[1]: 16 key heads x3 -> 48 value heads, d 128, 4 tokens, K = 4 snapshot slots."""
    import torch

    T, K = 4, 4
    q, k, v, g, beta, s0 = O.make_gdn_inputs(101 + kda, T, kda=kda)
    out = kb.gated_delta_net(*to_dev(cuda, q, k, v, g, beta[..., None], s0), K)
    torch.cuda.synchronize()
    gpu = out.cpu().numpy()
    exact = O.rs_gated_delta_net_f64(q, k, v, g, beta, s0, K)
    assert rel_err(gpu, exact) <= 1e-5
    if O.ref_available():
        ggml = O.ref_gated_delta_net(q, k, v, g, beta, s0, K, n_threads=4)
        assert rel_err(gpu, ggml, np.abs(exact).max()) <= 1e-5


@pytest.mark.parametrize("T,K", [(1, 4), (2, 4), (4, 1), (6, 4)])
def test_slot_rules(kb, cuda, T, K):
    """Only slots < min(T, K) are written (ggml.h:2649-2651); the others keep the caller's contents."""
    import torch

    q, k, v, g, beta, s0 = O.make_gdn_inputs(7 + T, T, H_k=4, H_v=8)
    S, H = 128, 8
    n = S * H * T + K * S * S * H
    out = torch.full((n,), float("nan"), device=cuda)
    dt = kb.kb_tensor(out.data_ptr(), kb.F32, [S * H, T + K * S, 1, 1], [4, S * H * 4])
    args = [kb.from_torch(x) for x in to_dev(cuda, q, k, v, g, beta[..., None], s0)]
    import ctypes

    assert kb.lib().kb_gated_delta_net(*[ctypes.byref(a) for a in args], K, ctypes.byref(dt), None, 0, None) == 0
    torch.cuda.synchronize()
    attn, slots = split_packed(out.cpu().numpy(), S, H, T, 1, K)
    ex_attn, ex_slots = split_packed(O.rs_gated_delta_net_f64(q, k, v, g, beta, s0, K), S, H, T, 1, K)
    assert rel_err(attn, ex_attn) <= 1e-5
    for s in range(K):
        if s < min(T, K):
            assert rel_err(slots[s], ex_slots[s]) <= 1e-5
        else:
            assert np.isnan(slots[s]).all()


def test_multi_sequence_broadcast(kb, cuda):
    """n_seqs = 2 with q/k of one sequence broadcast (ne3 % q.ne3 == 0)."""
    import torch

    T, K = 3, 2
    q, k, v, g, beta, s0 = O.make_gdn_inputs(55, T, H_k=2, H_v=6, n_seqs=2)
    q1, k1 = q[:1], k[:1]
    out = kb.gated_delta_net(*to_dev(cuda, q1, k1, v, g, beta[..., None], s0), K)
    torch.cuda.synchronize()
    exact = O.rs_gated_delta_net_f64(np.repeat(q1, 2, 0), np.repeat(k1, 2, 0), v, g, beta, s0, K)
    assert rel_err(out.cpu().numpy(), exact) <= 1e-5


@pytest.mark.parametrize("snap_dtype", ["float16", "bfloat16", "float32"])
def test_cache_form_snapshots_and_rollback(kb, cuda, snap_dtype):
    """klein's fused form: slot 0 overwrites the f32 state, slots 1..3 land in the snapshot rows; rolling back
    s tokens restores snapshot row s-1 exactly and conv slot s byte for byte (state.cpp:162-183)."""
    import torch

    T, K, S, H = 4, 4, 128, 48
    q, k, v, g, beta, s0 = O.make_gdn_inputs(303, T)
    tq, tk, tv, tg, tb, ts = to_dev(cuda, q, k, v, g, beta[..., None], s0)
    packed = kb.gated_delta_net(tq, tk, tv, tg, tb, ts, K)
    dt = getattr(torch, snap_dtype)
    snap = torch.zeros(K - 1, S * S * H, dtype=dt, device=cuda)
    state = ts.clone()
    attn = kb.gated_delta_net_cache(tq, tk, tv, tg, tb, state, snap, K)
    torch.cuda.synchronize()
    p_attn, p_slots = split_packed(packed.cpu().numpy(), S, H, T, 1, K)
    assert np.array_equal(attn.cpu().numpy(), p_attn)
    assert np.array_equal(state.cpu().numpy().reshape(-1), p_slots[0].reshape(-1))
    want = torch.from_numpy(p_slots[1:].reshape(K - 1, -1)).to(dt)
    assert torch.equal(snap.cpu(), want)
    # rollback over 3 layers that share the same snapshot rows
    rng = np.random.default_rng(4)
    conv_row = 3 * 10240
    convs = [torch.from_numpy(rng.standard_normal((K, conv_row)).astype(np.float32)).to(cuda) for _ in range(3)]
    ssms = [torch.zeros(S * S * H, device=cuda) for _ in range(3)]
    snaps = [snap] * 3
    code = {"float16": kb.F16, "bfloat16": kb.BF16, "float32": kb.F32}[snap_dtype]
    for s in (0, 1, 3):
        before = [c.clone() for c in convs]
        kb.rollback_recurrent(convs, snaps, ssms, code, s, K)
        torch.cuda.synchronize()
        for c, b0, m in zip(convs, before, ssms):
            if s == 0:
                assert torch.equal(c, b0)
                continue
            assert torch.equal(c[0], b0[s])
            assert torch.equal(m, snap[s - 1].float())


def test_rollback_rejects_bad_slot(kb, cuda):
    import torch

    c = [torch.zeros(4, 64, device=cuda)]
    m = [torch.zeros(64, device=cuda)]
    sn = [torch.zeros(3, 64, dtype=torch.float16, device=cuda)]
    with pytest.raises(kb.KbError):
        kb.rollback_recurrent(c, sn, m, kb.F16, 4, 4)


def test_state_drift_4096_steps(kb, cuda):
    """The recurrence over 4096 tokens (recurrent decode path): state within 1e-3 of f64."""
    import torch

    T, K = 4096, 1
    q, k, v, g, beta, s0 = O.make_gdn_inputs(4096, T, H_k=2, H_v=6)
    out = kb.gated_delta_net(*to_dev(cuda, q, k, v, g, beta[..., None], s0), K)
    torch.cuda.synchronize()
    S, H = 128, 6
    attn, slots = split_packed(out.cpu().numpy(), S, H, T, 1, K)
    ex_attn, ex_slots = split_packed(O.rs_gated_delta_net_f64(q, k, v, g, beta, s0, K), S, H, T, 1, K)
    e_state = rel_err(slots[0], ex_slots[0])
    assert e_state <= DELTANET_TOL
    assert e_state <= 1e-5  # measured headroom: f32 stays close to f64 over 4096 steps
    assert rel_err(attn, ex_attn) <= 1e-4


# ---------------------------------------------------------------------------------------------- KV write

@pytest.mark.parametrize("dst_type", ["f16", "q8_0", "bf16", "f32"])
def test_set_rows_bit_exact(kb, cuda, dst_type):
    import torch

    rng = np.random.default_rng(12)
    n_rows, n_src, row = 40, 6, 1024
    src = (rng.standard_normal((n_src, row)) * 3).astype(np.float32)
    src[0, :32] = 0.0                                  # zero block: d = 0
    src[1, :32] = np.arange(32) - 15.5                 # values on .5 steps of the block scale
    idx = np.array([5, 39, 0, 17, 6, 22], dtype=np.int64)
    code = {"f16": O.GGML_F16, "q8_0": O.GGML_Q8_0, "bf16": O.GGML_BF16, "f32": O.GGML_F32}[dst_type]
    row_bytes = {"f16": 2048, "q8_0": 1088, "bf16": 2048, "f32": 4096}[dst_type]
    host = rng.integers(0, 255, size=(n_rows, row_bytes), dtype=np.uint8)
    dev = torch.from_numpy(host.copy()).to(cuda)
    es = {"f16": 2, "q8_0": 34, "bf16": 2, "f32": 4}[dst_type]
    dst = kb.kb_tensor(dev.data_ptr(), code, [row, n_rows, 1, 1], [es, row_bytes])
    st, it = to_dev(cuda, src, idx)
    kb.set_rows(dst, st, it)
    torch.cuda.synchronize()
    got = dev.cpu().numpy()
    want = host.copy()
    if dst_type == "bf16":
        b = torch.from_numpy(src).to(torch.bfloat16).view(torch.uint8).numpy().reshape(n_src, -1)
        want[idx] = b
    else:
        assert O.rs_set_rows(want, code, row, src, idx) == 0
    assert np.array_equal(got, want)


def test_set_rows_i32_broadcast_and_bad_index(kb, cuda):
    import torch

    rng = np.random.default_rng(13)
    ne0, n_src, ne2, n_rows = 64, 3, 2, 8
    src = rng.standard_normal((1, ne2, n_src, ne0)).astype(np.float32)
    idx = np.array([[[1, 6, 3]]], dtype=np.int32)   # [ne12=1][ne11=1][n_src], broadcast over ne2
    cache = torch.zeros(1, ne2, n_rows, ne0, dtype=torch.float16, device=cuda)
    dst = kb.from_torch(cache)
    st, it = to_dev(cuda, src, idx)
    kb.device_error(clear=True)
    kb.set_rows(dst, st, it)
    torch.cuda.synchronize()
    got = cache.cpu().numpy()
    for i2 in range(ne2):
        for r, row in enumerate(idx[0, 0]):
            assert np.array_equal(got[0, i2, row], src[0, i2, r].astype(np.float16))
    assert kb.device_error() == 0
    bad = torch.tensor([1, 99, 3], dtype=torch.int32, device=cuda)
    kb.set_rows(dst, st, bad.reshape(1, 1, 3))
    torch.cuda.synchronize()
    assert kb.device_error(clear=True) != 0


@pytest.mark.parametrize("T", [4, 130])
def test_head_shards_equal_whole(kb, cuda, T):
    """Head sharding (8 ranks' slices of 48 value heads, key heads gathered by gdn_head_shard): each slice through
    the op equals the same heads of the whole op, for the recurrent verify (T = 4) and the chunked prefill."""
    import torch

    from klein_b200.kv_split import gdn_head_shard

    K = 4
    q, k, v, g, beta, s0 = O.make_gdn_inputs(303, T)
    whole = kb.gated_delta_net(*to_dev(cuda, q, k, v, g, beta[..., None], s0), K)
    torch.cuda.synchronize()
    attn, slots = split_packed(whole.cpu().numpy(), 128, 48, T, 1, K)
    for r in range(8):
        lo, hi, kidx = gdn_head_shard(16, 48, 8, r)
        part = kb.gated_delta_net(*to_dev(cuda, q[:, :, kidx], k[:, :, kidx], v[:, :, lo:hi], g[:, :, lo:hi],
                                          beta[:, :, lo:hi, None], s0[:, lo:hi]), K)
        torch.cuda.synchronize()
        a, s = split_packed(part.cpu().numpy(), 128, hi - lo, T, 1, K)
        scale = np.abs(attn).max()
        assert np.abs(a - attn[:, :, lo:hi]).max() <= 1e-6 * scale
        assert np.abs(s - slots[:, :, lo:hi]).max() <= 1e-6 * np.abs(slots).max()
