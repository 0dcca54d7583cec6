"""A whole DeltaNet layer of the decode / verify step in one launch (kb_gdn_step) against the three calls it fuses
(kb_gdn_input, kb_gated_delta_net_cache, kb_gdn_gated_norm — each parity-tested against the reference elsewhere):
bit for bit, over consecutive steps on the same state (the per-key-head counters leave themselves at zero), for 1-4
tokens and every snapshot type; and against the exact float64 composition of the reference's ops
(graph.cpp:136-190: the conv input side, GGML_OP_GATED_DELTA_NET, the gated norm)."""
import numpy as np
import pytest

import oracle as O
from parity import DELTANET_TOL

pytestmark = pytest.mark.gpu

S, HK, HV, KC = 128, 16, 48, 4
CH = 2 * S * HK + S * HV
EPS = 1e-6


def make_layer(torch, dev, K, snap_dtype, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w = {
        "conv_w": 0.5 * torch.randn(CH, KC, device=dev, generator=g),
        "dt": torch.randn(HV, device=dev, generator=g),
        "a": -torch.rand(HV, device=dev, generator=g) - 0.1,
        "norm_w": 1 + 0.1 * torch.randn(S, device=dev, generator=g),
    }
    conv = 0.5 * torch.randn(K, (KC - 1) * CH, device=dev, generator=g)
    ssm = 0.05 * torch.randn(1, HV, S, S, device=dev, generator=g)
    snap = torch.full((K - 1, S * S * HV), 7.0, device=dev).to(snap_dtype) if K > 1 else None
    return g, w, conv, ssm, snap


def step_inputs(torch, dev, g, T):
    return (torch.randn(T, CH, device=dev, generator=g), torch.randn(T, HV * S, device=dev, generator=g),
            torch.randn(T, HV, device=dev, generator=g), torch.randn(T, HV, device=dev, generator=g))


def chain(kb, T, K, w, conv, ssm, snap, qkv, z, br, al):
    q, k, v, beta, gg = kb.gdn_input(qkv, conv, w["conv_w"], S, HK, EPS, beta_raw=br, alpha=al, dt_bias=w["dt"], a=w["a"])
    attn = kb.gated_delta_net_cache(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), gg.view(1, T, HV, 1),
                                    beta.view(1, T, HV), ssm, snap, K)
    return kb.gdn_gated_norm(attn.view(T, HV, S), z, w["norm_w"], EPS).view(T, HV * S)


@pytest.mark.parametrize("T", [1, 2, 3, 4])
@pytest.mark.parametrize("snap", ["f16", "bf16", "f32"])
def test_step_matches_three_calls_bitwise(kb, cuda, T, snap):
    import torch

    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[snap]
    K = 4
    g, w, conv, ssm, sn = make_layer(torch, cuda, K, dt, 300 + T)
    f = [conv.clone(), ssm.clone(), sn.clone()]
    c = [conv.clone(), ssm.clone(), sn.clone()]
    sync = torch.zeros(HK, dtype=torch.int32, device=cuda)
    for _ in range(3):
        qkv, z, br, al = step_inputs(torch, cuda, g, T)
        out = kb.gdn_step(qkv, f[0], w["conv_w"], br, al, w["dt"], w["a"], f[1], f[2], K, z, w["norm_w"], EPS, sync)
        want = chain(kb, T, K, w, c[0], c[1], c[2], qkv, z, br, al)
        torch.cuda.synchronize()
        assert kb.device_error() == 0
        assert torch.equal(out, want)
        for a, b in zip(f, c):
            assert torch.equal(a, b)
    assert int(sync.abs().sum()) == 0


@pytest.mark.parametrize("T,K", [(1, 1), (4, 1), (3, 2)])
def test_step_fewer_snapshots(kb, cuda, T, K):
    """n_snapshots 1 (no snapshot rows) and 2 (one row, fewer than the tokens): only the slots below K are written."""
    import torch

    g, w, conv, ssm, sn = make_layer(torch, cuda, K, torch.float16, 400 + 10 * T + K)
    f = [conv.clone(), ssm.clone(), sn.clone() if sn is not None else None]
    c = [conv.clone(), ssm.clone(), sn.clone() if sn is not None else None]
    sync = torch.zeros(HK, dtype=torch.int32, device=cuda)
    qkv, z, br, al = step_inputs(torch, cuda, g, T)
    out = kb.gdn_step(qkv, f[0], w["conv_w"], br, al, w["dt"], w["a"], f[1], f[2], K, z, w["norm_w"], EPS, sync)
    want = chain(kb, T, K, w, c[0], c[1], c[2], qkv, z, br, al)
    torch.cuda.synchronize()
    assert torch.equal(out, want) and torch.equal(f[0], c[0]) and torch.equal(f[1], c[1])
    if sn is not None:
        assert torch.equal(f[2], c[2])


def test_step_against_f64(kb, cuda):
    """The verify step (4 tokens, 4 snapshots, f32 rows) against the float64 composition of the reference's ops."""
    import torch

    T, K = 4, 4
    g, w, conv, ssm, sn = make_layer(torch, cuda, K, torch.float32, 77)
    qkv, z, br, al = step_inputs(torch, cuda, g, T)
    host = lambda x: x.detach().cpu().numpy().astype(np.float32)
    conv0, s0 = host(conv), host(ssm)
    sync = torch.zeros(HK, dtype=torch.int32, device=cuda)
    out = kb.gdn_step(qkv, conv, w["conv_w"], br, al, w["dt"], w["a"], ssm, sn, K, z, w["norm_w"], EPS, sync)
    torch.cuda.synchronize()
    q, k, v, beta, gg, conv_x = O.rs_gdn_input(host(qkv), conv0, host(w["conv_w"]), host(br), host(al), host(w["dt"]),
                                               host(w["a"]), S, HK, EPS)
    packed = O.rs_gated_delta_net_f64(q[None], k[None], v[None], gg[None, ..., None], beta[None, ..., None], s0, K)
    attn = packed[:S * HV * T].reshape(T, HV, S)
    slots = packed[S * HV * T:].reshape(K, -1)
    out_x = O.rs_gdn_gated_norm(attn, host(z), host(w["norm_w"]), EPS).reshape(T, -1)
    assert np.abs(host(out) - out_x).max() <= DELTANET_TOL * np.abs(out_x).max()
    assert np.abs(host(ssm).reshape(-1) - slots[0]).max() <= DELTANET_TOL * np.abs(slots[0]).max()
    for s in range(1, K):
        assert np.abs(host(sn[s - 1]) - slots[s]).max() <= DELTANET_TOL * np.abs(slots[s]).max()
    assert np.array_equal(host(conv), conv_x)  # the conv slots are copies of stored inputs
