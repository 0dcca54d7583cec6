"""Generates the golden fixtures in this directory from the reference's own ggml CPU ops.

    python tests/golden/make_golden.py [attn_prologue | gdn_io | q4_0 | fa_verify_q4_0 | ...]   (one fixture only with its name)

Needs oracle/_ref (built by `make -C oracle ref` from the reference sources). Every fixture holds seeded
inputs and the reference's outputs for them; tests/test_oracle.py checks the C restatement against them
(so the restatement stays pinned where the reference tree is absent) and the GPU tests reuse them.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402


def q8_edge_rows():
    """Rows that exercise q8_0 rounding: an all-zero block, exact half steps, tiny and large magnitudes."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((6, 256)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, :32] = np.linspace(-127, 127, 32).astype(np.float32) / 127.0 * 3.0
    x[2, :32] = (np.arange(32) - 16 + 0.5).astype(np.float32)  # x*id lands on .5 boundaries
    x[3, :32] = 1e-30
    x[4, :32] = 6e4
    return x


# qwen35 full-attention rope: 64 of 256 dims rotated, interleaved M-RoPE sections, theta base 1e7
PROLOGUE_ROPE = dict(n_rot=64, sections=[11, 11, 10, 0], mode=40, freq_base=1e7)


def make_prologue_inputs(seed, n, nh=24, nkv=4, hd=256, max_pos=262143):
    """Seeded inputs of the attention prologue: projections ~N(0, 1), norm weights ~1 + N(0, 0.1), text positions
    (t = h = w, extra 0) spread up to max_pos, distinct cache cells of a 64-cell ring (n <= 64)."""
    rng = np.random.default_rng(seed)
    qfull = rng.standard_normal((n, nh * 2 * hd)).astype(np.float32)
    kcur = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    vcur = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    p = np.sort(rng.integers(0, max_pos + 1, n)).astype(np.int32)
    pos = np.concatenate([p, p, p, np.zeros(n, np.int32)]).astype(np.int32)
    kv_idx = (np.arange(n, dtype=np.int64) + seed) % 64  # distinct cells (a token owns its cell)
    q_norm = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    k_norm = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    return qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm


def prologue_fixture():
    qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm = make_prologue_inputs(11, 3, nh=4, nkv=2)
    kv_idx = np.array([5, 17, 63], dtype=np.int64)
    c16k = np.zeros((64, 2 * 256 * 2), np.uint8)
    c16v = np.zeros_like(c16k)
    q, gate = O.ref_attn_prologue(qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm, 1e-6, k_cache=c16k, v_cache=c16v,
                                  cache_type=O.GGML_F16, **PROLOGUE_ROPE)
    return dict(qfull=qfull, kcur=kcur, vcur=vcur, pos=pos, kv_idx=kv_idx, q_norm=q_norm, k_norm=k_norm, q=q,
                gate=gate, k_cache=c16k, v_cache=c16v)


def make_gdn_io_inputs(seed, n, S=128, H_k=16, H_v=48, K=4, kc=4):
    """Seeded inputs of the DeltaNet input / output sides: projections ~N(0, 1), conv weights ~N(0, 0.5),
    a stored conv state ~N(0, 1) in slot 0 (older slots hold a sentinel), gate inputs ~N(0, 1), a < 0."""
    rng = np.random.default_rng(seed)
    ch = 2 * S * H_k + S * H_v
    qkv = rng.standard_normal((n, ch)).astype(np.float32)
    conv_state = np.full((K, (kc - 1) * ch), 7.0, np.float32)
    conv_state[0] = rng.standard_normal((kc - 1) * ch).astype(np.float32)
    conv_w = (0.5 * rng.standard_normal((ch, kc))).astype(np.float32)
    beta_raw = rng.standard_normal((n, H_v)).astype(np.float32)
    alpha = rng.standard_normal((n, H_v)).astype(np.float32)
    dt_bias = rng.standard_normal(H_v).astype(np.float32)
    a = -np.exp(rng.standard_normal(H_v)).astype(np.float32)
    return qkv, conv_state, conv_w, beta_raw, alpha, dt_bias, a


def gdn_io_fixture():
    qkv, cs, w, br, al, dt, a = make_gdn_io_inputs(21, 3, S=64, H_k=2, H_v=4)
    cs_out = cs.copy()
    q, k, v, beta, g = O.ref_gdn_input(qkv, cs_out, w, br, al, dt, a, 64, 2, 1e-6)
    rng = np.random.default_rng(22)
    x = rng.standard_normal((3, 4, 64)).astype(np.float32)
    z = rng.standard_normal((3, 4, 64)).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(64)).astype(np.float32)
    o = O.ref_gdn_gated_norm(x, z, nw, 1e-6)
    return dict(qkv=qkv, conv_state=cs, conv_w=w, beta_raw=br, alpha=al, dt_bias=dt, a=a, q=q, k=k, v=v, beta=beta,
                g=g, conv_state_out=cs_out, x=x, z=z, norm_w=nw, o=o)


def q4_0_fixture():
    """set_rows into a q4_0 cache (quantize_row_q4_0_ref): the q8_0 edge rows plus a block whose largest magnitude
    appears twice with opposite signs (the first one sets the scale) and one of values that land on x * id + 8.5
    integer boundaries."""
    x = q8_edge_rows()
    x[5, :32] = np.linspace(-1, 1, 32).astype(np.float32)
    x[5, 3], x[5, 9] = -2.0, 2.0
    x[5, 32:64] = (np.arange(32) % 16 - 8).astype(np.float32) / 4.0
    idx = np.array([5, 0, 3, 1, 7, 2], dtype=np.int64)
    cache = np.zeros((8, 256 // 32 * 18), dtype=np.uint8)
    O.ref_set_rows(cache, O.GGML_Q4_0, 256, x, idx)
    return dict(src=x, idx=idx, cache_q4_0=cache)


def fa_fixture(n_q, n_kv, kvt):
    q, kc, vc, kd, vd = O.make_fa_inputs(4242 + n_kv, n_q, n_kv, kv_type=kvt)
    mask = None if n_q == 1 else O.rs_visible_mask(n_q, n_kv, n_kv - n_q).astype(np.float16)
    ref = O.ref_flash_attn_ext(q, kc, vc, kvt, 4, mask=mask, n_threads=1, use_ref=True)
    return dict(q=q, k=kc, v=vc, mask=np.zeros((0, 0), np.float16) if mask is None else mask, out=ref,
                kv_type=np.int32(kvt))


# flash attention: decode f16, verify f16 with klein's causal mask, verify q8_0 / q4_0 with mask
FA_FIXTURES = {"fa_decode_f16": (1, 64, O.GGML_F16), "fa_verify_f16": (4, 48, O.GGML_F16),
               "fa_verify_q8_0": (4, 80, O.GGML_Q8_0), "fa_verify_q4_0": (4, 72, O.GGML_Q4_0)}

FIXTURES = {"attn_prologue": lambda: prologue_fixture(), "gdn_io": lambda: gdn_io_fixture(),
            "q4_0": lambda: q4_0_fixture()}
FIXTURES.update({name: (lambda a=args: fa_fixture(*a)) for name, args in FA_FIXTURES.items()})


def main(only=None):
    out = {}
    if only in FIXTURES:
        out[only] = FIXTURES[only]()
        for name, arrays in out.items():
            np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)
            print(name, sum(a.nbytes for a in arrays.values()))
        return
    for name, (n_q, n_kv, kvt) in FA_FIXTURES.items():
        out[name] = fa_fixture(n_q, n_kv, kvt)
    # gated delta net (small heads so the fixture stays small): scalar gate and KDA vector gate
    for name, kda in [("gdn_verify", False), ("gdn_verify_kda", True)]:
        q, k, v, g, beta, s0 = O.make_gdn_inputs(77 + kda, T=4, H_k=2, H_v=6, S=32, kda=kda)
        ref = O.ref_gated_delta_net(q, k, v, g, beta, s0, K=4)
        out[name] = dict(q=q, k=k, v=v, g=g, beta=beta, s0=s0, K=np.int32(4), out=ref)
    # q8_0 quantisation (ggml_quantize_chunk -> quantize_row_q8_0_ref)
    x = q8_edge_rows()
    out["q8_0"] = dict(x=x, y=O.ref_quantize_q8_0(x))
    # set_rows into f16 and q8_0 caches
    rng = np.random.default_rng(5)
    src = rng.standard_normal((3, 256)).astype(np.float32)
    idx = np.array([7, 0, 12], dtype=np.int64)
    c16 = np.zeros((16, 512), dtype=np.uint8)
    O.ref_set_rows(c16, O.GGML_F16, 256, src, idx)
    c8 = np.zeros((16, 256 // 32 * 34), dtype=np.uint8)
    O.ref_set_rows(c8, O.GGML_Q8_0, 256, src, idx)
    out["set_rows"] = dict(src=src, idx=idx, cache_f16=c16, cache_q8_0=c8)
    # f32 -> f16 snapshot conversion (ggml_cpy), including overflow and subnormal values
    xs = np.concatenate([rng.standard_normal(64).astype(np.float32) * 0.02,
                         np.array([7e4, -7e4, 1e-8, -3e-6, 65504.0, 65519.0, 65520.0, 0.0], np.float32)])
    h = np.zeros(xs.size, dtype=np.uint16)
    O.ref_cpy(xs, O.GGML_F32, h, O.GGML_F16)
    out["cpy_f32_f16"] = dict(x=xs, y=h)
    out["attn_prologue"] = prologue_fixture()
    out["gdn_io"] = gdn_io_fixture()
    out["q4_0"] = q4_0_fixture()
    for name, arrays in out.items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)
        print(name, sum(a.nbytes for a in arrays.values()))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else None)
