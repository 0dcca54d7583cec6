"""CPU checks of the State-side entry points: the byte counts of klein's state_kv_bytes / state_mtp_kv_bytes /
state_recurrent_bytes (state.cpp:20-35) and Engine::run's pass indexing (engine.cpp:254-326), restated here from
the reference and compared with kb_state_sizes / kb_plan_pass (no device needed)."""
import ctypes

import numpy as np
import pytest

import klein_b200 as kb
import oracle as O

BLOCK = {kb.F16: (1, 2), kb.BF16: (1, 2), kb.Q8_0: (32, 34), kb.Q4_0: (32, 18), kb.F32: (1, 4)}


def row_size(t, n):  # ggml_row_size
    blk, sz = BLOCK[t]
    return n // blk * sz


def ref_sizes(d, c):
    """state.cpp:20-35 with klein's HParams helpers (model.h:39-42)"""
    kv_row = d.n_head_kv * d.head_dim
    n_attn = d.n_layer // d.full_attn_interval
    row = row_size(c.type_k, kv_row) + row_size(c.type_v, kv_row)
    kv = n_attn * row * c.n_ctx
    mtp = row * min(c.n_ctx, c.mtp_window) if d.with_mtp else 0
    ch = d.ssm_dt_rank * d.ssm_d_state + 2 * d.ssm_n_group * d.ssm_d_state
    conv_row = (d.ssm_conv_kernel - 1) * ch
    ssm_row = d.ssm_d_state ** 2 * d.ssm_dt_rank
    n_rec = d.n_layer - n_attn
    rec = n_rec * (conv_row * 4 * c.n_snapshots + ssm_row * (4 + row_size(c.snap_type, 1) * (c.n_snapshots - 1)))
    return kv, mtp, rec


@pytest.mark.parametrize("n_ctx,tk,snaps,st", [(262144, kb.Q4_0, 4, kb.F16), (131072, kb.Q8_0, 4, kb.F16),
                                                (4096, kb.F16, 1, kb.F16), (8192, kb.Q8_0, 3, kb.F32),
                                                (10000, kb.BF16, 2, kb.BF16)])
def test_state_sizes_match_reference(kb, n_ctx, tk, snaps, st):
    d = kb.qwen35_dims()
    c = kb.state_config(n_ctx, tk, tk, snaps, st)
    a, b, r = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    assert kb.lib().kb_state_sizes(ctypes.byref(d), ctypes.byref(c), ctypes.byref(a), ctypes.byref(b), ctypes.byref(r)) == 0
    assert (a.value, b.value, r.value) == ref_sizes(d, c)
    assert kb.lib().kb_state_required_bytes(ctypes.byref(d), ctypes.byref(c)) >= a.value + b.value + r.value


def ref_pass(n_ctx, mtp_cells, mtp, n, cell0, kv_lo):
    """Engine::run (engine.cpp:254-257, 304) and graph.cpp:16-19"""
    ring = mtp_cells if mtp and mtp_cells < n_ctx else 0
    padded = min(n_ctx, (cell0 + n + 255) // 256 * 256)
    n_kv = min(ring, padded) if ring else padded
    idx = [(cell0 + i) % ring if ring > 0 else cell0 + i for i in range(n)]
    return ring, n_kv, idx


def ref_mask(n, n_kv, cell0, kv_lo, ring):
    """the dense mask loop of Engine::run (engine.cpp:308-326): True where visible"""
    m = np.zeros((n, n_kv), dtype=bool)
    end = cell0 + n - 1
    for i in range(n):
        p = cell0 + i
        for j in range(n_kv):
            if ring == 0:
                m[i, j] = kv_lo <= j <= p
            else:
                q = end - ((end - j) % ring + ring) % ring
                m[i, j] = kv_lo <= q <= p and q > p - ring
    return m


@pytest.mark.parametrize("mtp,n,cell0,kv_lo", [(0, 4, 0, 0), (0, 4, 300, 0), (0, 1, 4095, 0), (0, 256, 1000, 0),
                                              (1, 4, 1, 1), (1, 1, 20000, 1), (1, 4, 40000, 1), (1, 3, 16383, 1)])
def test_plan_pass_matches_engine_run(kb, mtp, n, cell0, kv_lo):
    n_ctx, window = 65536, 16384
    d = kb.qwen35_dims(n_layer=8)
    c = kb.state_config(n_ctx, mtp_window=window)
    p = kb.KbPass()
    idx = np.zeros(n, dtype=np.int64)
    assert kb.lib().kb_plan_pass(ctypes.byref(d), ctypes.byref(c), mtp, n, cell0, kv_lo, ctypes.byref(p),
                                 ctypes.c_void_p(idx.ctypes.data)) == 0
    ring, n_kv, ridx = ref_pass(n_ctx, window, mtp, n, cell0, kv_lo)
    assert (p.ring, p.n_kv) == (ring, n_kv)
    assert list(idx) == ridx
    assert (p.fa.causal, p.fa.pos0, p.fa.kv_lo, p.fa.ring) == (1, cell0, kv_lo, ring)
    assert abs(p.fa.scale - 1 / 16) < 1e-9
    # the analytic bounds admit exactly the cells of klein's dense mask
    vis = np.isfinite(O.rs_visible_mask(n, n_kv, p.fa.pos0, kv_lo=p.fa.kv_lo, ring=p.fa.ring))
    assert np.array_equal(vis, ref_mask(n, n_kv, cell0, kv_lo, ring))


def test_plan_pass_rejects_full_context(kb):
    d = kb.qwen35_dims(n_layer=8)
    c = kb.state_config(4096)
    p = kb.KbPass()
    assert kb.lib().kb_plan_pass(ctypes.byref(d), ctypes.byref(c), 0, 4, 4093, 0, ctypes.byref(p), None) == kb.KB_ERR_ARG
    assert kb.lib().kb_plan_pass(ctypes.byref(d), ctypes.byref(c), 0, 4, 4092, 0, ctypes.byref(p), None) == 0


def test_state_rejects_bad_configs(kb):
    d = kb.qwen35_dims()
    out = ctypes.c_void_p()
    for c in (kb.state_config(0), kb.state_config(4096, n_snapshots=0), kb.state_config(4096, type_k=kb.F32),
              kb.state_config(4096, snap_type=kb.Q8_0)):
        assert kb.lib().kb_state_create(ctypes.byref(d), ctypes.byref(c), ctypes.byref(out)) == kb.KB_ERR_ARG
        assert not out.value
