"""The attention prologue (kb_attn_prologue: Q/gate split, RMS norms, interleaved M-RoPE, KV-cache writes) against
the reference's own ggml graph for it (graph.cpp:94-112) on the same seeded inputs, f16 and q8_0 caches."""
import os
import sys

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLD)
from make_golden import PROLOGUE_ROPE, make_prologue_inputs  # noqa: E402

ref_only = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


def run(kb, cuda, inputs, cache_type, n_cells=64, offset=0):
    """offset: qfull placed one float past a 16-byte boundary (offset 1) takes the 4-byte gate copy."""
    import torch

    qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm = [torch.from_numpy(x).to(cuda) for x in inputs]
    if offset:
        buf = torch.zeros(qfull.numel() + offset, dtype=torch.float32, device=cuda)
        buf[offset:] = qfull.reshape(-1)
        qfull = buf[offset:].view(qfull.shape)
    row = {kb.F16: 4 * 256 * 2, kb.Q8_0: 4 * 8 * 34, kb.Q4_0: 4 * 8 * 18}[cache_type]
    kc = torch.zeros((n_cells, row), dtype=torch.uint8, device=cuda)
    vc = torch.zeros_like(kc)
    q, gate = kb.attn_prologue(qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm, 1e-6, k_cache=kb.cache_rows(kc, cache_type),
                               v_cache=kb.cache_rows(vc, cache_type), **PROLOGUE_ROPE)
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    return q.cpu().numpy(), gate.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy()


@ref_only
@pytest.mark.parametrize("n,offset", [(1, 0), (4, 0), (37, 0), (4, 1)])
def test_prologue_f16_cache_matches_reference(kb, cuda, n, offset):
    inputs = make_prologue_inputs(100 + n, n)
    q, gate, kc, vc = run(kb, cuda, inputs, kb.F16, offset=offset)
    rk = np.zeros((64, 4 * 256 * 2), np.uint8)
    rv = np.zeros_like(rk)
    q_ref, gate_ref = O.ref_attn_prologue(*inputs, 1e-6, k_cache=rk, v_cache=rv, cache_type=O.GGML_F16, **PROLOGUE_ROPE)
    # float32 math on both sides; the GPU's cosf / sinf and fused multiply-adds differ from glibc's by ulps
    assert np.abs(q - q_ref).max() <= 2e-6 * np.abs(q_ref).max()
    assert np.array_equal(gate.reshape(gate_ref.shape), gate_ref)
    assert np.array_equal(vc, rv)
    # K rows: identical f16 except where the float value sits on a rounding boundary (one ulp at most)
    a, b = kc.view(np.float16).astype(np.float32), rk.view(np.float16).astype(np.float32)
    ulp = np.spacing(np.abs(b).astype(np.float16)).astype(np.float32)  # one f16 ulp at each value
    assert np.all(np.abs(a - b) <= ulp)
    assert np.mean(a != b) < 1e-3


@ref_only
def test_prologue_q8_0_cache_matches_reference(kb, cuda):
    inputs = make_prologue_inputs(7, 9)
    _, _, kc, vc = run(kb, cuda, inputs, kb.Q8_0)
    rk = np.zeros((64, 4 * 8 * 34), np.uint8)
    rv = np.zeros_like(rk)
    O.ref_attn_prologue(*inputs, 1e-6, k_cache=rk, v_cache=rv, cache_type=O.GGML_Q8_0, **PROLOGUE_ROPE)
    assert np.array_equal(vc, rv)  # V rows: the same f32 input, the same quantisation rule
    a = O.rs_dequantize_q8_0(kc.reshape(-1, 34)).reshape(64, -1)
    b = O.rs_dequantize_q8_0(rk.reshape(-1, 34)).reshape(64, -1)
    d = np.abs(rk.reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float32)).reshape(64, -1)
    # a K value may land on the other side of a quantisation step: at most one step (d) apart
    assert np.all(np.abs(a - b).reshape(64, -1, 32) <= 1.01 * d[:, :, None] + 1e-30)


def test_prologue_rejects_bad_cell(kb, cuda):
    import torch

    inputs = list(make_prologue_inputs(3, 2))
    inputs[4] = np.array([0, 99], dtype=np.int64)  # cell 99 of a 64-cell cache
    kb.device_error(clear=True)
    t = [torch.from_numpy(x).to(cuda) for x in inputs]
    kc = torch.zeros((64, 4 * 256 * 2), dtype=torch.uint8, device=cuda)
    kb.attn_prologue(*t, 1e-6, k_cache=kb.cache_rows(kc, kb.F16), v_cache=kb.cache_rows(kc.clone(), kb.F16), **PROLOGUE_ROPE)
    torch.cuda.synchronize()
    assert kb.device_error(clear=True) != 0


@ref_only
def test_prologue_q4_0_cache_matches_reference(kb, cuda):
    inputs = make_prologue_inputs(8, 9)
    _, _, kc, vc = run(kb, cuda, inputs, kb.Q4_0)
    rk = np.zeros((64, 4 * 8 * 18), np.uint8)
    rv = np.zeros_like(rk)
    O.ref_attn_prologue(*inputs, 1e-6, k_cache=rk, v_cache=rv, cache_type=O.GGML_Q4_0, **PROLOGUE_ROPE)
    assert np.array_equal(vc, rv)  # V rows: the same f32 input, quantize_row_q4_0_ref's rule
    a = O.rs_dequantize_q4_0(kc.reshape(-1, 18)).reshape(64, -1)
    b = O.rs_dequantize_q4_0(rk.reshape(-1, 18)).reshape(64, -1)
    d = np.abs(rk.reshape(-1, 18)[:, :2].copy().view(np.float16).astype(np.float32)).reshape(64, -1)
    assert np.all(np.abs(a - b).reshape(64, -1, 32) <= 1.01 * d[:, :, None] + 1e-30)


def test_set_rows_q4_0_bit_exact(kb, cuda):
    """kb_set_rows into a q4_0 cache equals ggml's set_rows (quantize_row_q4_0_ref) on the golden rows: an all-zero
    block, a tie of opposite-signed maxima (the first sets the scale), .5 boundaries, tiny and large magnitudes."""
    import torch

    g = dict(np.load(os.path.join(GOLD, "q4_0.npz")))
    cache = torch.zeros(g["cache_q4_0"].shape, dtype=torch.uint8, device=cuda)
    kb.set_rows(kb.cache_rows(cache, kb.Q4_0), torch.from_numpy(g["src"]).to(cuda), torch.from_numpy(g["idx"]).to(cuda))
    torch.cuda.synchronize()
    assert np.array_equal(cache.cpu().numpy(), g["cache_q4_0"])
