"""The CPU oracle is pinned to the reference: the C restatement (oracle/restate.c) against the committed
golden fixtures generated from ggml's CPU ops (tests/golden/make_golden.py), and — where the reference build
oracle/_ref is present — against the live reference library on fresh seeded inputs."""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ref_only = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


def gold(name):
    return dict(np.load(os.path.join(GOLD, name + ".npz")))


# ---------------------------------------------------------------------------------------------- fixtures

def test_golden_q8_0_bit_exact():
    g = gold("q8_0")
    assert np.array_equal(O.rs_quantize_q8_0(g["x"]), g["y"])


def test_golden_set_rows_bit_exact():
    g = gold("set_rows")
    c16 = np.zeros_like(g["cache_f16"])
    assert O.rs_set_rows(c16, O.GGML_F16, 256, g["src"], g["idx"]) == 0
    assert np.array_equal(c16, g["cache_f16"])
    c8 = np.zeros_like(g["cache_q8_0"])
    assert O.rs_set_rows(c8, O.GGML_Q8_0, 256, g["src"], g["idx"]) == 0
    assert np.array_equal(c8, g["cache_q8_0"])


def test_golden_q4_0_set_rows_bit_exact():
    g = gold("q4_0")
    c4 = np.zeros_like(g["cache_q4_0"])
    assert O.rs_set_rows(c4, O.GGML_Q4_0, 256, g["src"], g["idx"]) == 0
    assert np.array_equal(c4, g["cache_q4_0"])
    rows = O.rs_quantize_q4_0(g["src"])
    assert np.array_equal(rows, g["cache_q4_0"][g["idx"]])


def test_golden_f16_conversion_bit_exact():
    g = gold("cpy_f32_f16")
    with np.errstate(over="ignore"):  # the fixture holds values beyond f16's range on purpose (they become inf)
        assert np.array_equal(g["x"].astype(np.float16).view(np.uint16), g["y"])
    h = np.array([O.restate().rs_fp32_to_fp16(O.ctypes_float(x)) for x in g["x"]], dtype=np.uint16)
    assert np.array_equal(h, g["y"])


@pytest.mark.parametrize("name", ["fa_decode_f16", "fa_verify_f16", "fa_verify_q8_0", "fa_verify_q4_0"])
def test_golden_flash_attention(name):
    g = gold(name)
    kvt = int(g["kv_type"])
    n_kv = g["k"].shape[0]
    if kvt == O.GGML_F16:
        kd = g["k"].astype(np.float32).reshape(n_kv, 4, 256)
        vd = g["v"].astype(np.float32).reshape(n_kv, 4, 256)
        q = O.q_round_f16(g["q"])
        tol = 2e-2  # ggml accumulates V*softmax in fp16 for f16 V (ops.cpp:8992-9007)
    else:
        deq = O.rs_dequantize_q8_0 if kvt == O.GGML_Q8_0 else O.rs_dequantize_q4_0
        kd = deq(g["k"]).reshape(n_kv, 4, 256)
        vd = deq(g["v"]).reshape(n_kv, 4, 256)
        q = O.q_round_q8_0(g["q"])  # q8_0 is the vec_dot type of both q8_0 and q4_0 K
        tol = 1e-5  # f32 accumulation: only summation order differs
    mask = g["mask"].astype(np.float32) if g["mask"].size else None
    exact = O.rs_flash_attn_f64(q, kd, vd, mask=mask)
    err = np.abs(exact - g["out"]).max() / np.abs(exact).max()
    assert err <= tol, err


@pytest.mark.parametrize("name", ["gdn_verify", "gdn_verify_kda"])
def test_golden_gated_delta_net(name):
    g = gold(name)
    exact = O.rs_gated_delta_net_f64(g["q"], g["k"], g["v"], g["g"], g["beta"], g["s0"], int(g["K"]))
    err = np.abs(exact - g["out"]).max() / np.abs(exact).max()
    assert err <= 1e-6, err


def test_mask_rule_matches_engine_loop():
    """rs_visible_mask against a direct transcription of klein's host loop (engine.cpp:308-326)."""
    for n_q, n_kv, cell0, kv_lo, ring in [(4, 512, 300, 0, 0), (4, 256, 1000, 0, 256), (3, 128, 130, 20, 128),
                                          (1, 64, 10, 0, 0)]:
        want = np.full((n_q, n_kv), -np.inf, np.float32)
        end = cell0 + n_q - 1
        for i in range(n_q):
            p = cell0 + i
            for j in range(n_kv):
                if ring == 0:
                    vis = kv_lo <= j <= p
                else:
                    c = end - ((end - j) % ring + ring) % ring
                    vis = kv_lo <= c <= p and c > p - ring
                if vis:
                    want[i, j] = 0.0
        assert np.array_equal(O.rs_visible_mask(n_q, n_kv, cell0, kv_lo=kv_lo, ring=ring), want)
        for i in range(n_q):
            for j in range(0, n_kv, 7):
                assert O.restate().rs_visible(j, i, cell0, n_q, kv_lo, ring) == (want[i, j] == 0.0)


def test_lse_combine_of_split_equals_whole():
    """Splitting the cells in parts, computing (o, m, l) per part, and merging gives the full attention."""
    q, kc, vc, kd, vd = O.make_fa_inputs(3, 2, 700, H=6, H_kv=1, D=64)
    scale = 0.125
    full = O.rs_flash_attn_f64(q, kd, vd, scale=scale)
    parts = [(0, 100), (100, 101), (101, 700)]
    o_p, m_p, l_p = [], [], []
    for lo, hi in parts:
        s = np.einsum("qhd,kd->qhk", q.astype(np.float64), kd[lo:hi, 0].astype(np.float64)) * scale
        m = s.max(-1)
        p = np.exp(s - m[..., None])
        o_p.append(np.einsum("qhk,kd->qhd", p, vd[lo:hi, 0].astype(np.float64)).reshape(-1, 64))
        m_p.append(m.reshape(-1))
        l_p.append(p.sum(-1).reshape(-1))
    merged = O.rs_lse_combine(np.stack(o_p), np.stack(m_p), np.stack(l_p)).reshape(full.shape)
    assert np.abs(merged - full).max() <= 1e-6 * np.abs(full).max()


def test_rollback_restores_snapshot_bit_exact():
    rng = np.random.default_rng(1)
    conv = rng.standard_normal((4, 96)).astype(np.float32)
    snap = (rng.standard_normal((3, 500)) * 0.02).astype(np.float16)
    for s in (1, 2, 3):
        c = conv.copy()
        ssm = np.zeros(500, np.float32)
        O.rs_rollback(c, snap.view(np.uint16), ssm, s)
        assert np.array_equal(c[0], conv[s])
        assert np.array_equal(ssm, snap[s - 1].astype(np.float32))


# ---------------------------------------------------------------------------------------------- live reference

@ref_only
def test_live_q8_0_bit_exact():
    x = np.random.default_rng(11).standard_normal((128, 1024)).astype(np.float32) * 3
    assert np.array_equal(O.rs_quantize_q8_0(x), O.ref_quantize_q8_0(x))
    y = O.ref_quantize_q8_0(x)
    assert np.array_equal(O.rs_dequantize_q8_0(y).reshape(-1), O.ref_dequantize(O.GGML_Q8_0, y, x.size))


@ref_only
def test_live_q4_0_bit_exact():
    x = np.random.default_rng(12).standard_normal((128, 1024)).astype(np.float32) * 3
    y = np.zeros((128, 1024 // 32 * 18), np.uint8)
    O.ref_set_rows(y, O.GGML_Q4_0, 1024, x, np.arange(128, dtype=np.int64))
    assert np.array_equal(O.rs_quantize_q4_0(x), y)
    assert np.array_equal(O.rs_dequantize_q4_0(y).reshape(-1), O.ref_dequantize(O.GGML_Q4_0, y, x.size))


@ref_only
@pytest.mark.parametrize("kvt,n_q,n_kv", [(O.GGML_F16, 1, 4096), (O.GGML_F16, 4, 1000), (O.GGML_Q8_0, 1, 4096),
                                          (O.GGML_Q8_0, 4, 1000), (O.GGML_Q4_0, 1, 4096), (O.GGML_Q4_0, 4, 1000)])
def test_live_flash_attention(kvt, n_q, n_kv):
    q, kc, vc, kd, vd = O.make_fa_inputs(900 + n_q + n_kv, n_q, n_kv, kv_type=kvt)
    mask = O.rs_visible_mask(n_q, n_kv, n_kv - n_q)
    ref = O.ref_flash_attn_ext(q, kc, vc, kvt, 4, mask=mask.astype(np.float16), n_threads=2, use_ref=True)
    qr = O.q_round_f16(q) if kvt == O.GGML_F16 else O.q_round_q8_0(q)
    exact = O.rs_flash_attn_f64(qr, kd, vd, mask=mask)
    err = np.abs(exact - ref).max() / np.abs(exact).max()
    assert err <= (2.5e-2 if kvt == O.GGML_F16 else 1e-5), err


@ref_only
def test_live_gated_delta_net_config1():
    """config[1]: 48 value heads, 16 key heads, d 128, 4 tokens, K = 4 snapshot slots."""
    q, k, v, g, beta, s0 = O.make_gdn_inputs(21, T=4)
    ref = O.ref_gated_delta_net(q, k, v, g, beta, s0, 4, n_threads=4)
    exact = O.rs_gated_delta_net_f64(q, k, v, g, beta, s0, 4)
    assert np.abs(exact - ref).max() / np.abs(exact).max() <= 1e-6


@ref_only
def test_live_set_rows_f16_bit_exact():
    rng = np.random.default_rng(8)
    src = rng.standard_normal((5, 1024)).astype(np.float32)
    idx = np.array([3, 9, 0, 31, 17], np.int64)
    a = np.zeros((32, 2048), np.uint8)
    b = np.zeros((32, 2048), np.uint8)
    assert O.ref_set_rows(a, O.GGML_F16, 1024, src, idx) == 0
    assert O.rs_set_rows(b, O.GGML_F16, 1024, src, idx) == 0
    assert np.array_equal(a, b)


@ref_only
def test_live_set_rows_q8_0_matches_cpu_path():
    """ggml's CPU set_rows quantises with its SIMD quantize_row_q8_0 (127/amax, round-half-even); the
    restatement follows quantize_row_q8_0_ref (1/d, roundf), as ggml-cuda's set_rows does. They agree except
    at rounding ties, which differ by one quantum."""
    rng = np.random.default_rng(9)
    src = rng.standard_normal((64, 1024)).astype(np.float32)
    idx = np.arange(64, dtype=np.int64)[::-1].copy()
    a = np.zeros((64, 1088), np.uint8)
    b = np.zeros((64, 1088), np.uint8)
    O.ref_set_rows(a, O.GGML_Q8_0, 1024, src, idx)
    O.rs_set_rows(b, O.GGML_Q8_0, 1024, src, idx)
    da = O.rs_dequantize_q8_0(a)
    db = O.rs_dequantize_q8_0(b)
    assert (a != b).mean() < 1e-3
    d = a.reshape(64, 32, 34)[:, :, :2].copy().view(np.float16).astype(np.float32)
    assert np.all(np.abs(da - db).reshape(64, 32, 32) <= d + 1e-12)


# ---------------------------------------------------------------------------------------------- attention prologue

def assert_f16_near(cache_f16, x64):
    """K rows in f16 against the float64 restatement: the reference rounds its float32 value, so the two can sit on
    either side of an f16 rounding boundary (one f16 ulp apart), rarely."""
    a = cache_f16.astype(np.float64)
    b = x64.astype(np.float32).astype(np.float16).astype(np.float64)
    ulp = np.spacing(np.abs(b).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(a - b) <= ulp)
    assert np.mean(a != b) < 1e-2


def test_golden_attn_prologue():
    """RMS norm * weight and interleaved M-RoPE (64 of 256 dims, base 1e7) of the restatement against the
    reference's graph (graph.cpp:94-112) on positions up to 262,143; the gate and V rows pass through."""
    g = gold("attn_prologue")
    q, k, gate = O.rs_attn_prologue(g["qfull"], g["kcur"], g["pos"], g["q_norm"], g["k_norm"], 1e-6, 64,
                                    [11, 11, 10, 0], 40, 1e7)
    assert np.abs(q - g["q"]).max() <= 1e-6 * np.abs(g["q"]).max()
    assert np.array_equal(gate.astype(np.float32), g["gate"])
    kc = g["k_cache"].view(np.float16).reshape(64, -1, 256)[g["kv_idx"]]
    assert_f16_near(kc, k)
    vc = g["v_cache"].view(np.float16).reshape(64, -1)[g["kv_idx"]]
    assert np.array_equal(vc, g["vcur"].astype(np.float16))


@ref_only
def test_live_attn_prologue_qwen35_shapes():
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import PROLOGUE_ROPE, make_prologue_inputs

    qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm = make_prologue_inputs(12, 5)
    kc = np.zeros((64, 4 * 256 * 2), np.uint8)
    vc = np.zeros_like(kc)
    q_ref, gate_ref = O.ref_attn_prologue(qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm, 1e-6, k_cache=kc, v_cache=vc,
                                          cache_type=O.GGML_F16, **PROLOGUE_ROPE)
    q, k, gate = O.rs_attn_prologue(qfull, kcur, pos, q_norm, k_norm, 1e-6, **PROLOGUE_ROPE)
    assert np.abs(q - q_ref).max() <= 1e-6 * np.abs(q_ref).max()
    assert np.array_equal(gate.astype(np.float32), gate_ref)
    assert_f16_near(kc.view(np.float16).reshape(64, 4, 256)[kv_idx], k)


@ref_only
@pytest.mark.parametrize("cache_type", [O.GGML_Q8_0, O.GGML_Q4_0])
def test_live_attn_prologue_quantised_caches(cache_type):
    """The reference's quantised cache writes after the prologue: V rows are the restated quantisation of the input
    rows, bit for bit; K rows that of the restated normed, roped rows, within one quantisation step."""
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import PROLOGUE_ROPE, make_prologue_inputs

    qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm = make_prologue_inputs(13, 6)
    bb = 34 if cache_type == O.GGML_Q8_0 else 18
    kc = np.zeros((64, 4 * 8 * bb), np.uint8)
    vc = np.zeros_like(kc)
    O.ref_attn_prologue(qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm, 1e-6, k_cache=kc, v_cache=vc,
                        cache_type=cache_type, **PROLOGUE_ROPE)
    quant = O.rs_quantize_q8_0 if cache_type == O.GGML_Q8_0 else O.rs_quantize_q4_0
    deq = O.rs_dequantize_q8_0 if cache_type == O.GGML_Q8_0 else O.rs_dequantize_q4_0
    assert np.array_equal(vc[kv_idx], quant(vcur))
    _, k, _ = O.rs_attn_prologue(qfull, kcur, pos, q_norm, k_norm, 1e-6, **PROLOGUE_ROPE)
    a = deq(kc[kv_idx].reshape(-1, bb)).reshape(-1, 32)
    b = deq(quant(k.reshape(len(kv_idx), -1).astype(np.float32)).reshape(-1, bb)).reshape(-1, 32)
    d = np.abs(kc[kv_idx].reshape(-1, bb)[:, :2].copy().view(np.float16).astype(np.float32))
    assert np.all(np.abs(a - b) <= 1.01 * d + 1e-30)
    assert np.mean(a != b) < 1e-2


# ---------------------------------------------------------------------------------------------- DeltaNet input / output sides

def test_golden_gdn_io():
    """conv + silu + l2 norms, the gates, the conv-state snapshot rule and the gated output norm of the
    restatement against the reference's graph (graph.cpp:136-165, 186-190)."""
    g = gold("gdn_io")
    q, k, v, beta, gg, state = O.rs_gdn_input(g["qkv"], g["conv_state"], g["conv_w"], g["beta_raw"], g["alpha"],
                                              g["dt_bias"], g["a"], 64, 2, 1e-6)
    for a, b in ((q, g["q"]), (k, g["k"]), (v, g["v"]), (beta, g["beta"]), (gg, g["g"])):
        assert np.abs(a - b).max() <= 1e-6 * np.abs(b).max()
    assert np.array_equal(state, g["conv_state_out"])
    o = O.rs_gdn_gated_norm(g["x"], g["z"], g["norm_w"], 1e-6)
    assert np.abs(o - g["o"]).max() <= 1e-6 * np.abs(g["o"]).max()


@ref_only
@pytest.mark.parametrize("n", [1, 2, 5])
def test_live_gdn_input_qwen35_shapes(n):
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import make_gdn_io_inputs

    qkv, cs, w, br, al, dt, a = make_gdn_io_inputs(30 + n, n)
    cs_ref = cs.copy()
    ref = O.ref_gdn_input(qkv, cs_ref, w, br, al, dt, a, 128, 16, 1e-6)
    rs = O.rs_gdn_input(qkv, cs, w, br, al, dt, a, 128, 16, 1e-6)
    for x, y in zip(rs[:5], ref):
        assert np.abs(x - y).max() <= 1e-6 * np.abs(y).max()
    assert np.array_equal(rs[5], cs_ref)
