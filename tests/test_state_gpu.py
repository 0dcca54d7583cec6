"""GPU checks of klein's State in HBM and the layer compositions bound to it (kb_state_*, kb_layer_attention,
kb_layer_deltanet): a 4-layer qwen35 stack (3 DeltaNet + 1 full attention) with the MTP layer, driven through a
prompt pass, a 4-token verify pass, the accept / rollback of Engine::generate and MTP passes around the ring. Every
output, cache row and recurrent state must equal (bit for bit) the same ops called one by one on separate buffers —
those ops are parity-tested against the reference elsewhere — and the rollback must restore the snapshot exactly."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HD, NH, NKV, S, HK, HV, KC = 256, 24, 4, 128, 16, 48, 4
CH = 2 * S * HK + S * HV
EPS = 1e-6


@pytest.fixture(scope="module")
def setup(kb, cuda):
    import torch

    from klein_b200.state import State

    dims = kb.qwen35_dims(n_layer=4, with_mtp=1)
    cfg = kb.state_config(4096, kb.Q8_0, kb.Q8_0, 4, kb.F16, mtp_window=1024)
    st = State(dims, cfg, cuda)
    g = torch.Generator(device=cuda)
    g.manual_seed(11)
    w = {
        "q_norm": 1 + 0.1 * torch.randn(HD, device=cuda, generator=g),
        "k_norm": 1 + 0.1 * torch.randn(HD, device=cuda, generator=g),
        "conv_w": 0.5 * torch.randn(CH, KC, device=cuda, generator=g),
        "dt": torch.randn(HV, device=cuda, generator=g),
        "a": -torch.rand(HV, device=cuda, generator=g) - 0.1,
        "ssm_norm": 1 + 0.1 * torch.randn(S, device=cuda, generator=g),
    }
    rp = kb.KbRopeParams(64, (ctypes.c_int32 * 4)(11, 11, 10, 0), 40, 1e7, 1.0, 1.0)
    # the same state kept by hand: caches per attention layer, conv / ssm / snapshots per DeltaNet layer
    ref = {"k": {}, "v": {}, "conv": {}, "ssm": {}, "snap": {}}
    for il in (3, 4):
        cells = 4096 if il == 3 else 1024
        ref["k"][il] = torch.zeros(cells, NKV * HD // 32 * 34, dtype=torch.uint8, device=cuda)
        ref["v"][il] = torch.zeros_like(ref["k"][il])
    for il in (0, 1, 2):
        ref["conv"][il] = torch.zeros(4, (KC - 1) * CH, device=cuda)
        ref["ssm"][il] = torch.zeros(1, HV, S, S, device=cuda)
        ref["snap"][il] = torch.zeros(3, S * S * HV, dtype=torch.float16, device=cuda)
    yield kb, torch, st, w, rp, ref, g
    st.close()


def attn_pass(setup, il, n, kv_lo, mtp, cell0=None):
    kb, torch, st, w, rp, ref, g = setup
    dev = st.device
    p, idx = st.plan(n, kv_lo=kv_lo, mtp=mtp, cell0=cell0)
    qfull = torch.randn(n, NH * 2 * HD, device=dev, generator=g)
    kcur = torch.randn(n, NKV * HD, device=dev, generator=g)
    vcur = torch.randn(n, NKV * HD, device=dev, generator=g)
    posv = torch.arange(n, dtype=torch.int32, device=dev) + int(p.cell0)
    pos = torch.cat([posv, posv, posv, torch.zeros_like(posv)])
    kv_idx = torch.from_numpy(idx).to(dev)
    out = torch.empty(n, NH * HD, device=dev)
    scratch = torch.empty(st.attention_scratch_bytes(il, p), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    st.attention(il, p, qfull, kcur, vcur, pos, kv_idx, w["q_norm"], w["k_norm"], EPS, rp, out, scratch, stream)
    # the same ops one by one on the hand-kept cache
    kc, vc = kb.cache_rows(ref["k"][il], kb.Q8_0), kb.cache_rows(ref["v"][il], kb.Q8_0)
    q, gate = kb.attn_prologue(qfull, kcur, vcur, pos, kv_idx, w["q_norm"], w["k_norm"], EPS, 64, [11, 11, 10, 0], 40,
                               1e7, kc, vc)
    kview = kb.kv_cache_view(ref["k"][il], kb.Q8_0, NKV, HD, n_kv=int(p.n_kv))
    vview = kb.kv_cache_view(ref["v"][il], kb.Q8_0, NKV, HD, n_kv=int(p.n_kv))
    want = kb.flash_attn_ext(q.unsqueeze(0), kview, vview, p.fa.scale, causal=True, pos0=int(p.fa.pos0),
                             kv_lo=int(p.fa.kv_lo), ring=int(p.fa.ring), gate=gate.view(1, n, NH, HD))
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    lay = st.layer(il)
    assert torch.equal(st.view(lay.k), ref["k"][il]) and torch.equal(st.view(lay.v), ref["v"][il])
    assert torch.equal(out, want.view(n, NH * HD))
    return p


def gdn_pass(setup, il, n):
    kb, torch, st, w, rp, ref, g = setup
    dev = st.device
    qkv = torch.randn(n, CH, device=dev, generator=g)
    z = torch.randn(n, HV * S, device=dev, generator=g)
    br = torch.randn(n, HV, device=dev, generator=g)
    al = torch.randn(n, HV, device=dev, generator=g)
    out = torch.empty(n, HV * S, device=dev)
    scratch = torch.empty(st.deltanet_scratch_bytes(il, n), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    st.deltanet(il, n, qkv, z, br, al, w["dt"], w["a"], w["conv_w"], w["ssm_norm"], EPS, out, scratch, stream)
    q, k, v, beta, gg = kb.gdn_input(qkv, ref["conv"][il], w["conv_w"], S, HK, EPS, beta_raw=br, alpha=al, dt_bias=w["dt"],
                                     a=w["a"])
    attn = kb.gated_delta_net_cache(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), gg.view(1, n, HV, 1), beta.view(1, n, HV),
                                    ref["ssm"][il], ref["snap"][il], 4)
    want = kb.gdn_gated_norm(attn.view(n, HV, S), z, w["ssm_norm"], EPS)
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    lay = st.layer(il)
    assert torch.equal(out, want.view(n, HV * S))
    assert torch.equal(st.view(lay.conv), ref["conv"][il].view(torch.uint8).view(4, -1))
    assert torch.equal(st.view(lay.ssm), ref["ssm"][il].view(torch.uint8).view(1, -1))
    assert torch.equal(st.view(lay.ssm_snap), ref["snap"][il].view(torch.uint8).view(3, -1))


def test_state_layout(setup):
    kb, torch, st, w, rp, ref, g = setup
    lay3, lay0, mtp = st.layer(3), st.layer(0), st.layer(4)
    assert (lay3.k.type, lay3.k.ne[0], lay3.k.ne[1], lay3.k.nb[1]) == (kb.Q8_0, NKV * HD, 4096, 1088)
    assert (mtp.k.ne[1], lay3.conv.data, lay0.k.data) == (1024, None, None)
    assert (lay0.conv.ne[0], lay0.conv.ne[1], lay0.ssm.ne[0], lay0.ssm_snap.ne[1], lay0.ssm_snap.type) == \
        ((KC - 1) * CH, 4, S * S * HV, 3, kb.F16)
    assert int(st.buf.abs().sum()) == 0  # zeroed at creation


def test_prompt_verify_accept_rollback_and_mtp_ring(setup):
    kb, torch, st, w, rp, ref, g = setup
    # a 300-token prompt pass through every layer, the MTP layer from cell 1 (kv_lo = 1, engine.cpp:431)
    for il in (0, 1, 2):
        gdn_pass(setup, il, 300)
    attn_pass(setup, 3, 300, 0, False)
    attn_pass(setup, 4, 299, 1, True, cell0=1)
    st.n_past = 300
    # a verify pass of 4 cells from n_past
    base = st.n_past
    for il in (0, 1, 2):
        gdn_pass(setup, il, 4)
    p = attn_pass(setup, 3, 4, 0, False)
    assert (p.cell0, p.n_kv) == (300, 512)
    # accept one draft: 2 rejected -> every DeltaNet layer back to the state 2 tokens before the end
    conv_before = {il: st.view(st.layer(il).conv).clone() for il in (0, 1, 2)}
    snap_before = {il: ref["snap"][il][1].clone() for il in (0, 1, 2)}
    st.accept(base, 4, 1, torch.cuda.current_stream(st.device).cuda_stream)
    torch.cuda.synchronize()
    assert st.n_past == base + 2
    for il in (0, 1, 2):
        lay = st.layer(il)
        assert torch.equal(st.view(lay.ssm).view(torch.float32).view(-1), snap_before[il].float())
        cv = st.view(lay.conv)
        assert torch.equal(cv[0], conv_before[il][2])
        ref["ssm"][il].copy_(snap_before[il].float().view_as(ref["ssm"][il]))
        ref["conv"][il][0].copy_(conv_before[il][2].view(torch.float32))
    # MTP passes that wrap the 1,024-cell ring
    attn_pass(setup, 4, 4, 1, True, cell0=2000)
    p = attn_pass(setup, 4, 1, 1, True, cell0=3000)
    assert (p.ring, p.n_kv) == (1024, 1024)


def test_clear_zeroes_recurrent_state(setup):
    kb, torch, st, w, rp, ref, g = setup
    st.n_past = 17
    st.clear(torch.cuda.current_stream(st.device).cuda_stream)
    torch.cuda.synchronize()
    assert st.n_past == 0
    for il in (0, 1, 2):
        lay = st.layer(il)
        for t in (lay.conv, lay.ssm, lay.ssm_snap):
            assert int(st.view(t).abs().sum()) == 0
