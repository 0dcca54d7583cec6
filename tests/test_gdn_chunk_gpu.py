"""GPU parity of the chunked DeltaNet prefill (config[2]: 4,096 tokens in 64-token chunks from a zero state) against
the f64 restatement of the recurrence (ops.cpp:11123-11275) and ggml's own CPU op, and of the dispatch around it:
the last min(T, K) - 1 tokens run token by token so every snapshot slot is a per-token state, ragged chunks,
broadcast q/k over sequences, klein's cache form, and the multi-pass split when scratch is short."""
import ctypes

import numpy as np
import pytest

import oracle as O
from parity import DELTANET_TOL, rel_err

pytestmark = pytest.mark.gpu

S = 128


def to_dev(cuda, *arrays):
    import torch

    return [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in arrays]


def split_packed(out, H, T, n_seqs, K):
    attn = out[: S * H * T * n_seqs].reshape(n_seqs, T, H, S)
    slots = out[S * H * T * n_seqs:].reshape(K, n_seqs, H, S, S)
    return attn, slots


def scratch_bytes(kb, v, g, K):
    return kb.lib().kb_gated_delta_net_scratch_bytes(ctypes.byref(kb.from_torch(v)), ctypes.byref(kb.from_torch(g)), K)


def test_config2_prefill_4096(kb, cuda):
    """48 value heads, 4,096 tokens, K = 4 snapshot slots, s0 = 0: state after 4,096 steps within 1e-3 of f64."""
    import torch

    T, K, H = 4096, 4, 48
    q, k, v, g, beta, s0 = O.make_gdn_inputs(2024, T, s0_std=0.0)
    args = to_dev(cuda, q, k, v, g, beta[..., None], s0)
    assert scratch_bytes(kb, args[2], args[3], K) == 48 * 64 * 65792  # the chunked form runs
    kb.device_error(clear=True)
    out = kb.gated_delta_net(*args, K)
    rec = kb.gated_delta_net(*args, K, scratch=False)  # recurrent kernel for every token
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    attn, slots = split_packed(out.cpu().numpy(), H, T, 1, K)
    r_attn, r_slots = split_packed(rec.cpu().numpy(), H, T, 1, K)
    # the f64 recurrence for value heads 32..47 (their key heads h % 16 are unchanged by the slice)
    sub = slice(32, 48)
    ex = O.rs_gated_delta_net_f64(q, k, v[:, :, sub], g[:, :, sub], beta[:, :, sub], s0[:, sub], K)
    ex_attn, ex_slots = split_packed(ex, 16, T, 1, K)
    e_state = rel_err(slots[0][:, sub], ex_slots[0])
    assert e_state <= DELTANET_TOL
    assert e_state <= 1e-4  # measured headroom of the split-f16 products
    for s in range(1, K):
        assert rel_err(slots[s][:, sub], ex_slots[s]) <= 1e-4
    assert rel_err(attn[:, :, sub], ex_attn) <= 1e-4
    # every head against the recurrent kernel (itself within 1e-5 of f64)
    assert rel_err(slots, r_slots) <= 1e-4
    assert rel_err(attn, r_attn) <= 1e-4


def test_against_ggml(kb, cuda):
    """Three-way rule against ggml's CPU op at 256 tokens, 48 heads, s0 ~ N(0, 0.02)."""
    import torch

    T, K, H = 256, 4, 48
    q, k, v, g, beta, s0 = O.make_gdn_inputs(77, T)
    out = kb.gated_delta_net(*to_dev(cuda, q, k, v, g, beta[..., None], s0), K)
    torch.cuda.synchronize()
    gpu = out.cpu().numpy()
    exact = O.rs_gated_delta_net_f64(q, k, v, g, beta, s0, K)
    e_gpu = rel_err(gpu, exact)
    assert e_gpu <= 1e-4
    if O.ref_available():
        ggml = O.ref_gated_delta_net(q, k, v, g, beta, s0, K, n_threads=4)
        e_cpu = rel_err(ggml, exact)
        assert rel_err(gpu, ggml, np.abs(exact).max()) <= e_cpu + DELTANET_TOL


@pytest.mark.parametrize("T,K", [(200, 4), (64, 1), (67, 4), (130, 2)])
def test_ragged_multiseq(kb, cuda, T, K):
    """Chunk boundaries that do not divide T, two sequences sharing broadcast q/k, slots from both paths."""
    import torch

    H_k, H_v, n_seqs = 4, 8, 2
    q, k, v, g, beta, s0 = O.make_gdn_inputs(300 + T, T, H_k=H_k, H_v=H_v, n_seqs=n_seqs)
    q1, k1 = q[:1], k[:1]
    dev = to_dev(cuda, q1, k1, v, g, beta[..., None], s0)
    assert scratch_bytes(kb, dev[2], dev[3], K) > 0
    out = kb.gated_delta_net(*dev, K)
    torch.cuda.synchronize()
    exact = O.rs_gated_delta_net_f64(np.repeat(q1, 2, 0), np.repeat(k1, 2, 0), v, g, beta, s0, K)
    attn, slots = split_packed(out.cpu().numpy(), H_v, T, n_seqs, K)
    ex_attn, ex_slots = split_packed(exact, H_v, T, n_seqs, K)
    assert rel_err(attn, ex_attn) <= 1e-4
    for s in range(min(T, K)):
        assert rel_err(slots[s], ex_slots[s]) <= 1e-4


@pytest.mark.parametrize("snap_dtype", ["float16", "bfloat16"])
def test_cache_form_matches_packed(kb, cuda, snap_dtype):
    """klein's fused form runs the same kernels: attention and slot 0 bit-identical to the packed result, the
    snapshot rows its rounding (slot 3 comes from the chunked kernel, slots 1-2 from the recurrent tail)."""
    import torch

    T, K, H = 300, 4, 48
    q, k, v, g, beta, s0 = O.make_gdn_inputs(41, T)
    tq, tk, tv, tg, tb, ts = to_dev(cuda, q, k, v, g, beta[..., None], s0)
    packed = kb.gated_delta_net(tq, tk, tv, tg, tb, ts, K)
    dt = getattr(torch, snap_dtype)
    snap = torch.zeros(K - 1, S * S * H, dtype=dt, device=cuda)
    state = ts.clone()
    attn = kb.gated_delta_net_cache(tq, tk, tv, tg, tb, state, snap, K)
    torch.cuda.synchronize()
    p_attn, p_slots = split_packed(packed.cpu().numpy(), H, T, 1, K)
    assert np.array_equal(attn.cpu().numpy(), p_attn)
    assert np.array_equal(state.cpu().numpy().reshape(-1), p_slots[0].reshape(-1))
    want = torch.from_numpy(p_slots[1:].reshape(K - 1, -1)).to(dt)
    assert torch.equal(snap.cpu(), want)


def test_multipass_bit_identical(kb, cuda):
    """Scratch for 3 chunks runs 640 tokens in 4 passes; the state carried in f32 between passes gives the same
    bits as one pass."""
    import torch

    T, K, H_k, H_v = 640, 4, 4, 8
    q, k, v, g, beta, s0 = O.make_gdn_inputs(9, T, H_k=H_k, H_v=H_v)
    dev = to_dev(cuda, q, k, v, g, beta[..., None], s0)
    full = kb.gated_delta_net(*dev, K)
    small = torch.empty(3 * H_v * 65792, dtype=torch.uint8, device=cuda)
    multi = kb.gated_delta_net(*dev, K, scratch=small)
    torch.cuda.synchronize()
    assert torch.equal(full, multi)
    too_small = torch.empty(H_v * 65792 - 16, dtype=torch.uint8, device=cuda)  # below one chunk: recurrent kernel
    rec = kb.gated_delta_net(*dev, K, scratch=too_small)
    ref = kb.gated_delta_net(*dev, K, scratch=False)
    torch.cuda.synchronize()
    assert torch.equal(rec, ref)
