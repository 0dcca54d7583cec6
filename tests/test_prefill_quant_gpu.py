"""GPU parity of prompt-length attention over klein's quantised caches (q8_0, and q4_0 beyond 131K cells):
kb_flash_attn_ext with >= 128 query tokens widens the visible cells to f16 in the scratch and runs the
tensor-core prefill kernel with Q rounded to q8_0 (ggml rounds Q to the vec_dot type of a q8_0 / q4_0 K,
ops.cpp:8960). klein attends each 2,048-token prompt chunk over the cache it has just written
(graph.cpp:111-121, engine.cpp:479-523). Also the long-prompt cases: the 16,384-token prefill and the MTP
head's 16,384-cell ring (state.cpp:17, engine.cpp:317-322).

Reference values: exact f64 attention on the same cache contents (the whole output where that is cheap, a
spread of query rows at prompt lengths) and, at moderate sizes, ggml's own CPU op (three-way rule,
tests/parity.py)."""
import numpy as np
import pytest

import oracle as O
from parity import check_attention

pytestmark = pytest.mark.gpu

H, H_KV, D = 24, 4, 256


def exact_rows(q, kd, vd, rows, pos0, kv_lo=0, ring=0, n_q=None, scale=1.0 / 16):
    """f64 attention of the query rows `rows` (indices into q) under klein's causal / ring rule."""
    n_q = q.shape[0] if n_q is None else n_q
    mask = O.rs_visible_mask(n_q, kd.shape[0], pos0, kv_lo=kv_lo, ring=ring)[rows].astype(np.float64)
    G = q.shape[1] // kd.shape[1]
    out = np.zeros((len(rows), q.shape[1], q.shape[2]))
    for h in range(q.shape[1]):
        s = (q[rows, h].astype(np.float64) @ kd[:, h // G].T.astype(np.float64)) * scale + mask
        m = s.max(1, keepdims=True)
        m = np.where(np.isfinite(m), m, 0.0)
        p = np.exp(s - m)
        l = p.sum(1, keepdims=True)
        out[:, h] = np.where(l > 0, (p @ vd[:, h // G].astype(np.float64)) / np.where(l > 0, l, 1.0), 0.0)
    return out


def spread_rows(n_q, n=192):
    """about n query rows spread over the prompt, with the first and last 16 rows"""
    r = set(range(min(16, n_q))) | set(range(max(0, n_q - 16), n_q)) | set(np.linspace(0, n_q - 1, n).astype(int))
    return np.array(sorted(r))


def run(kb, cuda, q, kc, vc, kv_type, mask=None, **kw):
    import torch

    kt, vt = torch.from_numpy(kc).to(cuda), torch.from_numpy(vc).to(cuda)
    mt = None if mask is None else torch.from_numpy(mask.astype(np.float16)).to(cuda)
    out = kb.flash_attn_ext(torch.from_numpy(q).to(cuda), kb.kv_cache_view(kt, kv_type, H_KV, D),
                            kb.kv_cache_view(vt, kv_type, H_KV, D), 1 / 16, mask=mt, **kw)
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    return out[0].cpu().numpy()


TYPES = [("q8_0", O.GGML_Q8_0), ("q4_0", O.GGML_Q4_0)]


def kb_type(kb, name):
    return kb.Q8_0 if name == "q8_0" else kb.Q4_0


@pytest.mark.parametrize("name,gt", TYPES, ids=[t[0] for t in TYPES])
def test_prefill_quant_vs_ggml(kb, cuda, name, gt):
    """256 new tokens over a 1,024-cell cache: every output row against f64 and ggml's CPU op."""
    n_q, n_kv = 256, 1024
    pos0 = n_kv - n_q
    q, kc, vc, kd, vd = O.make_fa_inputs(500 + gt, n_q, n_kv, kv_type=gt)
    gpu = run(kb, cuda, q, kc, vc, kb_type(kb, name), causal=True, pos0=pos0)
    mask = O.rs_visible_mask(n_q, n_kv, pos0)
    ggml = O.ref_flash_attn_ext(q, kc, vc, gt, H_KV, mask=mask.astype(np.float16), n_threads=8, use_ref=False) \
        if O.ref_available() else None
    check_attention(gpu, exact_rows(O.q_round_q8_0(q), kd, vd, np.arange(n_q), pos0), ggml)


@pytest.mark.parametrize("name,gt", TYPES, ids=[t[0] for t in TYPES])
def test_prefill_quant_chunk_2048(kb, cuda, name, gt):
    """klein's prompt chunk: 2,048 tokens attending over the 4,096-cell cache they were just written into."""
    n_q, n_kv = 2048, 4096
    pos0 = n_kv - n_q
    q, kc, vc, kd, vd = O.make_fa_inputs(600 + gt, n_q, n_kv, kv_type=gt)
    gpu = run(kb, cuda, q, kc, vc, kb_type(kb, name), causal=True, pos0=pos0)
    rows = spread_rows(n_q)
    check_attention(gpu[rows], exact_rows(O.q_round_q8_0(q), kd, vd, rows, pos0))


@pytest.mark.parametrize("pair", ["0", "1"], ids=["one_cta", "cta_pairs"])
@pytest.mark.parametrize("n_q,n_kv,pos0,kv_lo", [(300, 1300, 1000, 37), (128, 4000, 3872, 0), (640, 700, 60, 0)])
def test_prefill_quant_ragged(kb, cuda, monkeypatch, pair, n_q, n_kv, pos0, kv_lo):
    """ragged tiles, a kv_lo window that starts inside a 64-cell block, and cells past the last query's position; on
    one CTA per tile and on CTA pairs (KB_PREFILL_PAIR=1)"""
    monkeypatch.setenv("KB_PREFILL_PAIR", pair)
    q, kc, vc, kd, vd = O.make_fa_inputs(700 + n_q + n_kv, n_q, n_kv, kv_type=O.GGML_Q8_0)
    gpu = run(kb, cuda, q, kc, vc, kb.Q8_0, causal=True, pos0=pos0, kv_lo=kv_lo)
    check_attention(gpu, exact_rows(O.q_round_q8_0(q), kd, vd, np.arange(n_q), pos0, kv_lo=kv_lo))


def test_prefill_quant_dense_mask(kb, cuda):
    """klein's dense f16 mask over a q4_0 cache (every cell widened) against the analytic bounds. The two visit
    different numbers of 64-cell blocks per tile, so their block order (and with it the stale maximum that P is
    rounded to f16 against) differs: they agree within the parity bound, not bit for bit."""
    n_q, n_kv, pos0 = 384, 512, 100
    q, kc, vc, kd, vd = O.make_fa_inputs(801, n_q, n_kv, kv_type=O.GGML_Q4_0)
    mask = O.rs_visible_mask(n_q, n_kv, pos0)
    dense = run(kb, cuda, q, kc, vc, kb.Q4_0, mask=mask)
    anal = run(kb, cuda, q, kc, vc, kb.Q4_0, causal=True, pos0=pos0)
    exact = exact_rows(O.q_round_q8_0(q), kd, vd, np.arange(n_q), pos0)
    check_attention(dense, exact)
    check_attention(anal, exact)
    assert np.abs(dense - anal).max() <= 2e-3 * np.abs(exact).max()


@pytest.mark.parametrize("name,gt", TYPES, ids=[t[0] for t in TYPES])
def test_prefill_quant_without_view_scratch_runs_streaming(kb, cuda, name, gt):
    """Given no room for the f16 views, the same call runs on the streaming kernel: both within the bound."""
    n_q, n_kv = 512, 2048
    pos0 = n_kv - n_q
    q, kc, vc, kd, vd = O.make_fa_inputs(900 + gt, n_q, n_kv, kv_type=gt)
    t = kb_type(kb, name)
    tc = run(kb, cuda, q, kc, vc, t, causal=True, pos0=pos0)
    st = run(kb, cuda, q, kc, vc, t, causal=True, pos0=pos0, scratch_bytes=0)
    exact = exact_rows(O.q_round_q8_0(q), kd, vd, np.arange(n_q), pos0)
    check_attention(tc, exact)
    check_attention(st, exact)


def test_prefill_quant_gated(kb, cuda):
    """the fused output gate on the widened-cache prefill path"""
    import torch

    n_q, n_kv = 256, 512
    q, kc, vc, kd, vd = O.make_fa_inputs(1001, n_q, n_kv, kv_type=O.GGML_Q8_0)
    gate = np.random.default_rng(3).standard_normal((1, n_q, H, D)).astype(np.float32) * 3
    plain = run(kb, cuda, q, kc, vc, kb.Q8_0, causal=True, pos0=n_kv - n_q)
    gated = run(kb, cuda, q, kc, vc, kb.Q8_0, causal=True, pos0=n_kv - n_q, gate=torch.from_numpy(gate).to(cuda))
    want = plain * (1.0 / (1.0 + np.exp(-gate[0].astype(np.float64))))
    assert np.abs(gated - want).max() <= 1e-6 * np.abs(want).max()


@pytest.mark.parametrize("kv", ["f16", "q8_0"])
def test_prefill_16384_tokens(kb, cuda, kv):
    """the 16,384-token prefill of the whole-stack workload (3.30 TFLOP per layer), a spread of rows vs f64"""
    n_q = n_kv = 16384
    gt = O.GGML_F16 if kv == "f16" else O.GGML_Q8_0
    q, kc, vc, kd, vd = O.make_fa_inputs(16384 + gt, n_q, n_kv, kv_type=gt)
    gpu = run(kb, cuda, q, kc, vc, kb.F16 if kv == "f16" else kb.Q8_0, causal=True, pos0=0)
    rows = spread_rows(n_q, 160)
    qr = O.q_round_f16(q) if kv == "f16" else O.q_round_q8_0(q)
    check_attention(gpu[rows], exact_rows(qr, kd, vd, rows, 0))


@pytest.mark.parametrize("kv,n_q", [("f16", 4), ("f16", 1), ("q8_0", 4)])
def test_mtp_ring_16384(kb, cuda, kv, n_q):
    """The MTP head's window at its real size: a 16,384-cell ring (min(n_ctx, 16384), state.cpp:17) at a position
    far past one wrap, analytic ring bounds and klein's dense ring mask against f64."""
    ring, pos0 = 16384, 70001
    gt = O.GGML_F16 if kv == "f16" else O.GGML_Q8_0
    q, kc, vc, kd, vd = O.make_fa_inputs(1600 + n_q + gt, n_q, ring, kv_type=gt)
    t = kb.F16 if kv == "f16" else kb.Q8_0
    mask = O.rs_visible_mask(n_q, ring, pos0, ring=ring)
    anal = run(kb, cuda, q, kc, vc, t, causal=True, pos0=pos0, ring=ring)
    dense = run(kb, cuda, q, kc, vc, t, mask=mask)
    qr = O.q_round_f16(q) if kv == "f16" else O.q_round_q8_0(q)
    exact = exact_rows(qr, kd, vd, np.arange(n_q), pos0, ring=ring)
    check_attention(anal, exact)
    check_attention(dense, exact)
