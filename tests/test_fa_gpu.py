"""GPU parity of kb_flash_attn_ext (decode / verify streaming kernel) against the CPU oracle.

Every case runs the CUDA path through the C ABI and compares it with the exact f64 restatement on the same
cache contents and, at sizes ggml finishes quickly, with the reference's own ggml CPU op (three-way rule in
tests/parity.py).
"""
import numpy as np
import pytest

import oracle as O
from parity import check_attention

pytestmark = pytest.mark.gpu


def exact_np(q, kd, vd, mask=None, scale=1.0 / 16, softcap=0.0):
    """f64 attention with numpy matmuls (same definition as oracle.rs_flash_attn_f64, faster at large n_kv)."""
    n_q, H, D = q.shape
    H_kv = kd.shape[1]
    G = H // H_kv
    out = np.zeros((n_q, H, D))
    for h in range(H):
        hk = h // G
        s = (q[:, h, :].astype(np.float64) @ kd[:, hk, :].T.astype(np.float64)) * scale
        if softcap:
            s = softcap * np.tanh(s / softcap)
        if mask is not None:
            s = s + mask.astype(np.float64)
        m = s.max(1, keepdims=True)
        ok = np.isfinite(m)
        m = np.where(ok, m, 0.0)
        p = np.exp(s - m)
        l = p.sum(1, keepdims=True)
        o = (p @ vd[:, hk, :].astype(np.float64))
        out[:, h, :] = np.where(l > 0, o / np.where(l > 0, l, 1.0), 0.0)
    return out


def run_gpu(kb, cuda, q, kc, vc, H_kv, scale=1.0 / 16, mask=None, **kw):
    import torch

    D = q.shape[-1]
    qt = torch.from_numpy(q).to(cuda)
    kt = torch.from_numpy(kc).to(cuda)
    vt = torch.from_numpy(vc).to(cuda)
    kv_type = kb.F16 if kc.dtype == np.float16 else kb.Q8_0 if kc.shape[-1] % 34 == 0 and kc.shape[-1] % 18 != 0 else kb.Q4_0
    kview = kb.kv_cache_view(kt, kv_type, H_kv, D)
    vview = kb.kv_cache_view(vt, kv_type, H_kv, D)
    mt = None if mask is None else torch.from_numpy(mask.astype(np.float16)).to(cuda)
    out = kb.flash_attn_ext(qt, kview, vview, scale, mask=mt, **kw)
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    return out[0].cpu().numpy()


@pytest.mark.parametrize("n_q,n_kv", [(1, 4096), (4, 4096), (1, 1), (1, 17), (4, 63), (4, 64), (4, 65), (1, 1000),
                                      (4, 4099), (2, 777), (3, 2048), (5, 513), (8, 300)])
def test_f16_causal_analytic(kb, cuda, n_q, n_kv):
    q, kc, vc, kd, vd = O.make_fa_inputs(1000 + n_q * 7 + n_kv, n_q, n_kv)
    pos0 = max(n_kv - n_q, 0)
    mask = O.rs_visible_mask(n_q, n_kv, pos0)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=pos0)
    exact = exact_np(O.q_round_f16(q), kd, vd, mask)
    ggml = O.ref_flash_attn_ext(q, kc, vc, O.GGML_F16, 4, mask=mask.astype(np.float16), n_threads=4, use_ref=False) \
        if O.ref_available() and n_kv <= 4099 else None
    check_attention(gpu, exact, ggml)


def test_f16_decode_config0(kb, cuda):
    """config[0]: 1 token, 4096 cells, 24/4 heads, D 256, scale 1/16, no mask."""
    q, kc, vc, kd, vd = O.make_fa_inputs(1234, 1, 4096)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4)
    exact = O.rs_flash_attn_f64(O.q_round_f16(q), kd, vd)
    ggml = O.ref_flash_attn_ext(q, kc, vc, O.GGML_F16, 4, n_threads=8, use_ref=False) if O.ref_available() else None
    e_gpu, e_cpu, _ = check_attention(gpu, exact, ggml)
    assert e_gpu < 1e-3


def test_f16_dense_mask_matches_analytic(kb, cuda):
    """klein's dense mask (padded n_kv, engine.cpp:308-326) and the analytic bounds give the same output."""
    n_q, n_past = 4, 4100
    n_kv = (n_past + n_q + 255) // 256 * 256  # padded_n_kv
    q, kc, vc, kd, vd = O.make_fa_inputs(77, n_q, n_kv)
    mask = O.rs_visible_mask(n_q, n_kv, n_past)
    g_dense = run_gpu(kb, cuda, q, kc, vc, 4, mask=mask)
    g_anal = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=n_past)
    exact = exact_np(O.q_round_f16(q), kd, vd, mask)
    check_attention(g_dense, exact)
    check_attention(g_anal, exact)
    assert np.abs(g_dense - g_anal).max() <= 1e-6 * np.abs(exact).max()


def test_f16_fully_masked_rows_are_zero(kb, cuda):
    q, kc, vc, kd, vd = O.make_fa_inputs(5, 4, 512)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=100, kv_lo=200)
    assert np.all(gpu == 0.0)


def test_f16_kv_lo_window(kb, cuda):
    n_q, n_kv = 4, 3000
    q, kc, vc, kd, vd = O.make_fa_inputs(6, n_q, n_kv)
    mask = O.rs_visible_mask(n_q, n_kv, n_kv - n_q, kv_lo=1234)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=n_kv - n_q, kv_lo=1234)
    check_attention(gpu, exact_np(O.q_round_f16(q), kd, vd, mask))


def test_f16_ring_window(kb, cuda):
    """The MTP head's sliding window: a ring of `ring` cells (engine.cpp:304, :317-322)."""
    ring, n_q, pos0 = 1024, 4, 5000
    q, kc, vc, kd, vd = O.make_fa_inputs(8, n_q, ring)
    mask = O.rs_visible_mask(n_q, ring, pos0, ring=ring)
    g_anal = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=pos0, ring=ring)
    g_dense = run_gpu(kb, cuda, q, kc, vc, 4, mask=mask)
    exact = exact_np(O.q_round_f16(q), kd, vd, mask)
    check_attention(g_anal, exact)
    check_attention(g_dense, exact)


def test_f16_softcap(kb, cuda):
    q, kc, vc, kd, vd = O.make_fa_inputs(9, 4, 2048)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, softcap=2.0)
    exact = exact_np(O.q_round_f16(q), kd, vd, softcap=2.0)
    ggml = O.ref_flash_attn_ext(q, kc, vc, O.GGML_F16, 4, softcap=2.0, n_threads=4, use_ref=True) if O.ref_available() else None
    check_attention(gpu, exact, ggml)


def test_f16_alibi(kb, cuda):
    n_q, n_kv = 4, 1024
    q, kc, vc, kd, vd = O.make_fa_inputs(10, n_q, n_kv)
    rng = np.random.default_rng(3)
    mask = (rng.standard_normal((n_q, n_kv)) * 0.5).astype(np.float16).astype(np.float32)
    mask[:, 700:] = -np.inf
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, mask=mask, max_bias=8.0)
    exact = O.rs_flash_attn_f64(O.q_round_f16(q), kd, vd, mask=mask, max_bias=8.0)
    ggml = O.ref_flash_attn_ext(q, kc, vc, O.GGML_F16, 4, mask=mask.astype(np.float16), max_bias=8.0, n_threads=4) \
        if O.ref_available() else None
    check_attention(gpu, exact, ggml)


@pytest.mark.parametrize("H,H_kv", [(8, 8), (32, 4), (16, 2)])
def test_f16_gqa_shapes(kb, cuda, H, H_kv):
    q, kc, vc, kd, vd = O.make_fa_inputs(11 + H, 4, 1500, H=H, H_kv=H_kv)
    gpu = run_gpu(kb, cuda, q, kc, vc, H_kv)
    check_attention(gpu, exact_np(O.q_round_f16(q), kd, vd))


def test_f16_long_verify_262144(kb, cuda):
    """config[3] shape (f16): 4 tokens, causal among the last 4, 262,144 cells."""
    n_q, n_kv = 4, 262144
    q, kc, vc, kd, vd = O.make_fa_inputs(31337, n_q, n_kv)
    mask = O.rs_visible_mask(n_q, n_kv, n_kv - n_q)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=n_kv - n_q)
    check_attention(gpu, exact_np(O.q_round_f16(q), kd, vd, mask))


def test_scratch_too_small_is_rejected(kb, cuda):
    import ctypes
    import torch

    q, kc, vc, kd, vd = O.make_fa_inputs(12, 4, 8192)
    qt = torch.from_numpy(q).to(cuda).unsqueeze(0)
    kt = torch.from_numpy(kc).to(cuda)
    vt = torch.from_numpy(vc).to(cuda)
    kv = kb.kv_cache_view(kt, kb.F16, 4, 256)
    vv = kb.kv_cache_view(vt, kb.F16, 4, 256)
    qv = kb.kb_tensor(qt.data_ptr(), kb.F32, [256, 4, 24, 1], [4, 24 * 256 * 4, 256 * 4, 4 * 24 * 256 * 4])
    out = torch.zeros((4, 24, 256), device=cuda)
    dv = kb.from_torch(out.reshape(1, 4, 24, 256))
    prm = kb.fa_params(1 / 16)
    need = kb.lib().kb_flash_attn_ext_scratch_bytes(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(prm))
    assert need > 0
    rc = kb.lib().kb_flash_attn_ext(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), None, ctypes.byref(prm),
                                    ctypes.byref(dv), None, 0, None)
    assert rc == kb.KB_ERR_SCRATCH
    torch.cuda.synchronize()
    assert float(out.abs().max()) == 0.0


def test_partials_and_lse_combine(kb, cuda):
    """Two parts of the KV sequence computed with kb_flash_attn_ext_partial and merged with kb_lse_combine
    give the full attention (the per-GPU step of the sequence split, run on one GPU)."""
    import ctypes
    import torch

    from klein_b200.kv_split import kv_range, local_bounds, packed_part_floats

    n_q, n_kv, world, D, H = 4, 5000, 3, 256, 24
    q, kc, vc, kd, vd = O.make_fa_inputs(99, n_q, n_kv)
    qt = torch.from_numpy(q).to(cuda).unsqueeze(0)
    rows = n_q * H
    pf = packed_part_floats(rows, D)
    parts = torch.zeros(world, pf, device=cuda)
    L = kb.lib()
    qv = kb.kb_tensor(qt.data_ptr(), kb.F32, [D, n_q, H, 1], [4, H * D * 4, D * 4, n_q * H * D * 4])
    for r in range(world):
        lo, hi = kv_range(n_kv, world, r)
        kt = torch.from_numpy(kc[lo:hi].copy()).to(cuda)
        vt = torch.from_numpy(vc[lo:hi].copy()).to(cuda)
        kv, vv = kb.kv_cache_view(kt, kb.F16, 4, D), kb.kv_cache_view(vt, kb.F16, 4, D)
        pos0, kv_lo = local_bounds(lo, n_kv - n_q, 0)
        prm = kb.fa_params(1 / 16, causal=True, pos0=pos0, kv_lo=kv_lo)
        ov = kb.kb_tensor(parts[r].data_ptr(), kb.F32, [D, H, n_q, 1], [4, D * 4, H * D * 4, rows * D * 4])
        need = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(prm))
        scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=cuda)
        rc = L.kb_flash_attn_ext_partial(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), None, ctypes.byref(prm),
                                         ctypes.byref(ov), ctypes.c_void_p(parts[r].data_ptr() + rows * D * 4),
                                         ctypes.c_void_p(scratch.data_ptr()), need, None)
        assert rc == 0
        torch.cuda.synchronize()
    out = torch.empty(rows, D, device=cuda)
    rc = L.kb_lse_combine(ctypes.c_void_p(parts.data_ptr()), ctypes.c_void_p(parts.data_ptr() + rows * D * 4),
                          pf, world, rows, D, ctypes.c_void_p(out.data_ptr()), None)
    assert rc == 0
    torch.cuda.synchronize()
    mask = O.rs_visible_mask(n_q, n_kv, n_kv - n_q)
    check_attention(out.cpu().numpy().reshape(n_q, H, D), exact_np(O.q_round_f16(q), kd, vd, mask))


# ---------------------------------------------------------------------------------------------- q8_0 cache

@pytest.mark.parametrize("n_q,n_kv", [(1, 4096), (4, 4096), (4, 65), (1, 1000), (3, 777), (8, 300)])
def test_q8_0_causal_analytic(kb, cuda, n_q, n_kv):
    q, kc, vc, kd, vd = O.make_fa_inputs(2000 + n_q * 7 + n_kv, n_q, n_kv, kv_type=O.GGML_Q8_0)
    pos0 = n_kv - n_q
    mask = O.rs_visible_mask(n_q, n_kv, pos0)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=pos0)
    exact = exact_np(O.q_round_q8_0(q), kd, vd, mask)
    ggml = O.ref_flash_attn_ext(q, kc, vc, O.GGML_Q8_0, 4, mask=mask.astype(np.float16), n_threads=4, use_ref=False) \
        if O.ref_available() else None
    check_attention(gpu, exact, ggml)


def test_q8_0_dense_mask_and_ring(kb, cuda):
    ring, n_q, pos0 = 2048, 4, 9000
    q, kc, vc, kd, vd = O.make_fa_inputs(31, n_q, ring, kv_type=O.GGML_Q8_0)
    mask = O.rs_visible_mask(n_q, ring, pos0, ring=ring)
    exact = exact_np(O.q_round_q8_0(q), kd, vd, mask)
    check_attention(run_gpu(kb, cuda, q, kc, vc, 4, mask=mask), exact)
    check_attention(run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=pos0, ring=ring), exact)


def test_q8_0_long_verify_262144(kb, cuda):
    """config[3] shape (q8_0): 4 tokens, causal among the last 4, 262,144 cells."""
    n_q, n_kv = 4, 262144
    q, kc, vc, kd, vd = O.make_fa_inputs(4711, n_q, n_kv, kv_type=O.GGML_Q8_0)
    mask = O.rs_visible_mask(n_q, n_kv, n_kv - n_q)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=n_kv - n_q)
    check_attention(gpu, exact_np(O.q_round_q8_0(q), kd, vd, mask))


# ---------------------------------------------------------------------------------------------- q4_0 cache
# klein's cache type beyond 131K cells; ggml's vec_dot type for q4_0 K is q8_0, so Q is rounded as for q8_0

@pytest.mark.parametrize("n_q,n_kv", [(1, 4096), (4, 4096), (4, 65), (3, 777)])
def test_q4_0_causal_analytic(kb, cuda, n_q, n_kv):
    q, kc, vc, kd, vd = O.make_fa_inputs(3000 + n_q * 7 + n_kv, n_q, n_kv, kv_type=O.GGML_Q4_0)
    pos0 = n_kv - n_q
    mask = O.rs_visible_mask(n_q, n_kv, pos0)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=pos0)
    exact = exact_np(O.q_round_q8_0(q), kd, vd, mask)
    ggml = O.ref_flash_attn_ext(q, kc, vc, O.GGML_Q4_0, 4, mask=mask.astype(np.float16), n_threads=4, use_ref=False) \
        if O.ref_available() else None
    check_attention(gpu, exact, ggml)


def test_q4_0_dense_mask_and_ring(kb, cuda):
    ring, n_q, pos0 = 2048, 4, 9000
    q, kc, vc, kd, vd = O.make_fa_inputs(37, n_q, ring, kv_type=O.GGML_Q4_0)
    mask = O.rs_visible_mask(n_q, ring, pos0, ring=ring)
    exact = exact_np(O.q_round_q8_0(q), kd, vd, mask)
    check_attention(run_gpu(kb, cuda, q, kc, vc, 4, mask=mask), exact)
    check_attention(run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=pos0, ring=ring), exact)


def test_q4_0_long_verify_262144(kb, cuda):
    """config[3] shape over a q4_0 cache: 4 tokens, causal among the last 4, 262,144 cells."""
    n_q, n_kv = 4, 262144
    q, kc, vc, kd, vd = O.make_fa_inputs(4713, n_q, n_kv, kv_type=O.GGML_Q4_0)
    mask = O.rs_visible_mask(n_q, n_kv, n_kv - n_q)
    gpu = run_gpu(kb, cuda, q, kc, vc, 4, causal=True, pos0=n_kv - n_q)
    check_attention(gpu, exact_np(O.q_round_q8_0(q), kd, vd, mask))


# ---------------------------------------------------------------------------------------------- output gate

@pytest.mark.parametrize("kvt,n_q,n_kv", [("f16", 4, 8192), ("f16", 1, 100), ("q8_0", 4, 8192), ("bf16", 256, 512)])
def test_output_gate_fused(kb, cuda, kvt, n_q, n_kv):
    """kb_flash_attn_ext_gated = kb_flash_attn_ext * sigmoid(gate) (graph.cpp:124) on the split-combine path, the
    single-split store, the q8_0 kernel and the prefill kernel."""
    import torch

    g = torch.Generator(device=cuda)
    g.manual_seed(n_q * 7 + n_kv)
    H, H_kv, D = 24, 4, 256
    q = torch.randn(1, n_q, H, D, device=cuda, generator=g)
    if kvt == "bf16":
        q = q.bfloat16().float()
    kf = torch.randn(n_kv, H_kv * D, device=cuda, generator=g)
    vf = torch.randn(n_kv, H_kv * D, device=cuda, generator=g)
    if kvt == "q8_0":
        kc = torch.from_numpy(O.rs_quantize_q8_0(kf.cpu().numpy())).to(cuda)
        vc = torch.from_numpy(O.rs_quantize_q8_0(vf.cpu().numpy())).to(cuda)
        t = kb.Q8_0
    elif kvt == "bf16":
        kc, vc, t = kf.bfloat16(), vf.bfloat16(), kb.BF16
    else:
        kc, vc, t = kf.half(), vf.half(), kb.F16
    kv, vv = kb.kv_cache_view(kc, t, H_kv, D), kb.kv_cache_view(vc, t, H_kv, D)
    gate = torch.randn(1, n_q, H, D, device=cuda, generator=g) * 3
    plain = kb.flash_attn_ext(q, kv, vv, 1 / 16, causal=True, pos0=n_kv - n_q)
    gated = kb.flash_attn_ext(q, kv, vv, 1 / 16, causal=True, pos0=n_kv - n_q, gate=gate)
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    want = plain * (1.0 / (1.0 + torch.exp(-gate)))
    assert float((gated - want).abs().max()) <= 1e-6 * float(want.abs().max()) + 1e-30


# ---------------------------------------------------------------------------------------------- golden fixtures
# the reference's own ggml CPU outputs, committed (tests/golden/make_golden.py): the GPU path against them with the
# three-way rule, with no reference build needed on the GPU machine

@pytest.mark.parametrize("name", ["fa_decode_f16", "fa_verify_f16", "fa_verify_q8_0", "fa_verify_q4_0"])
def test_golden_fixture(kb, cuda, name):
    import os

    g = dict(np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", name + ".npz")))
    kvt = int(g["kv_type"])
    n_kv = g["k"].shape[0]
    if kvt == O.GGML_F16:
        kd, vd = (g[x].astype(np.float32).reshape(n_kv, 4, 256) for x in ("k", "v"))
        q = O.q_round_f16(g["q"])
    else:
        deq = O.rs_dequantize_q8_0 if kvt == O.GGML_Q8_0 else O.rs_dequantize_q4_0
        kd, vd = (deq(g[x]).reshape(n_kv, 4, 256) for x in ("k", "v"))
        q = O.q_round_q8_0(g["q"])
    mask = g["mask"] if g["mask"].size else None
    gpu = run_gpu(kb, cuda, g["q"], g["k"], g["v"], 4, mask=mask)
    check_attention(gpu, exact_np(q, kd, vd, mask=mask), g["out"])


# ---------------------------------------------------------------------------------------------- in-kernel exchange
# kb_flash_attn_ext_exchange with one rank: the same kernel path the N-GPU sequence split runs (grid barrier, split
# merge, stores into the gather buffer, per-slot release flags, bounded waits, final merge, device-side epochs), with
# every peer being this GPU itself

@pytest.mark.parametrize("kvt,n_q,n_kv,gated", [("f16", 4, 262144, False), ("f16", 1, 4096, False),
                                                ("f16", 4, 9000, True), ("q8_0", 4, 70001, False),
                                                ("q4_0", 4, 20000, False)])
def test_exchange_single_rank(kb, cuda, kvt, n_q, n_kv, gated):
    import ctypes
    import torch

    from klein_b200.kv_split import packed_part_floats

    gt = {"f16": O.GGML_F16, "q8_0": O.GGML_Q8_0, "q4_0": O.GGML_Q4_0}[kvt]
    t = {"f16": kb.F16, "q8_0": kb.Q8_0, "q4_0": kb.Q4_0}[kvt]
    q, kc, vc, kd, vd = O.make_fa_inputs(4242 + n_q + n_kv, n_q, n_kv, kv_type=gt)
    H, D = 24, 256
    kt, vt = torch.from_numpy(kc).to(cuda), torch.from_numpy(vc).to(cuda)
    kv, vv = kb.kv_cache_view(kt, t, 4, D), kb.kv_cache_view(vt, t, 4, D)
    qd = torch.from_numpy(q).to(cuda).unsqueeze(0)
    qt = kb.kb_tensor(qd.data_ptr(), kb.F32, [D, n_q, H, 1], [4, H * D * 4, D * 4, n_q * H * D * 4])
    prm = kb.fa_params(1 / 16, causal=True, pos0=n_kv - n_q)
    gate = torch.randn(1, n_q, H, D, device=cuda) * 2 if gated else None
    rows = n_q * H
    xchg = kb.PeerExchange(0, 1, packed_part_floats(rows, D), lambda obj: [obj])
    L = kb.lib()
    nb = L.kb_flash_attn_ext_push_scratch_bytes(ctypes.byref(qt), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(prm))
    scratch = torch.empty(max(nb, 1), dtype=torch.uint8, device=cuda)
    outs = [torch.full((1, n_q, H, D), float("nan"), device=cuda) for _ in range(4)]
    dts = [kb.from_torch(o.view(1, n_q, H, D)) for o in outs]
    for dt in dts:
        dt.ne[:] = [D, H, n_q, 1]
        dt.nb[:] = [4, D * 4, H * D * 4, n_q * H * D * 4]
    gt_t = None
    if gated:
        gt_t = kb.from_torch(gate)
        gt_t.ne[:] = [D, H, n_q, 1]
        gt_t.nb[:] = [4, D * 4, H * D * 4, n_q * H * D * 4]
    kb.device_error(clear=True)
    st = torch.cuda.current_stream(cuda).cuda_stream
    # two eager calls, then two replays of a captured call (the epoch lives on the device)
    for i in range(2):
        xchg.attend_exchange(qt, kv, vv, prm, scratch.data_ptr(), nb, dts[i], st, gate=gt_t)
    torch.cuda.synchronize()
    graphs = []
    for i in (2, 3):
        side = torch.cuda.Stream(cuda)
        side.wait_stream(torch.cuda.current_stream(cuda))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            xchg.attend_exchange(qt, kv, vv, prm, scratch.data_ptr(), nb, dts[i], side.cuda_stream, gate=gt_t)
        torch.cuda.current_stream(cuda).wait_stream(side)
        graphs.append(g)
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    plain = kb.flash_attn_ext(qd, kv, vv, 1 / 16, causal=True, pos0=n_kv - n_q, gate=gate)
    torch.cuda.synchronize()
    mask = O.rs_visible_mask(n_q, n_kv, n_kv - n_q)
    qr = O.q_round_f16(q) if kvt == "f16" else O.q_round_q8_0(q)
    exact = exact_np(qr, kd, vd, mask)
    if gated:
        exact = exact / (1.0 + np.exp(-gate[0].double().cpu().numpy()))
    ref = plain[0].cpu().numpy()
    for o in outs:
        got = o[0].cpu().numpy()
        check_attention(got, exact)
        # the same merge arithmetic as the split combine, in another order: f32 rounding differences only
        assert np.abs(got - ref).max() <= 1e-5 * np.abs(exact).max()
    del graphs
    xchg.close()
