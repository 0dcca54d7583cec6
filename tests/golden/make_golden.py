"""Generates the golden fixtures in this directory from the reference's own ggml CPU ops.

    python tests/golden/make_golden.py

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


def main():
    out = {}
    # flash attention: decode f16, verify f16 with klein's causal mask, verify q8_0 with mask
    for name, n_q, n_kv, kvt in [("fa_decode_f16", 1, 64, O.GGML_F16), ("fa_verify_f16", 4, 48, O.GGML_F16),
                                 ("fa_verify_q8_0", 4, 80, O.GGML_Q8_0)]:
        q, kc, vc, kd, vd = O.make_fa_inputs(4242 + n_kv, n_q, n_kv, kv_type=kvt)
        mask = None if n_q == 1 else O.rs_visible_mask(n_q, n_kv, n_kv - n_q).astype(np.float16)
        ref = O.ref_flash_attn_ext(q, kc, vc, kvt, 4, mask=mask, n_threads=1, use_ref=True)
        out[name] = dict(q=q, k=kc, v=vc, mask=np.zeros((0, 0), np.float16) if mask is None else mask, out=ref,
                         kv_type=np.int32(kvt))
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
    for name, arrays in out.items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)
        print(name, sum(a.nbytes for a in arrays.values()))


if __name__ == "__main__":
    main()
