"""klein's own graph nodes through ggml's graph API on ggml's CUDA backend, built with klein_b200 in place of its
attention and DeltaNet kernels (klein_b200/ggml: kb_ggml_cuda.cu and the build recipe), against ggml's CPU backend
(the reference) and the exact f64 attention / DeltaNet restatement:
  - Builder::attention's attention node (graph.cpp:113-121) over f16, q8_0 and q4_0 caches with klein's dense mask
    (engine.cpp:308-326) and padded n_kv (graph.cpp:16-19): decode, the 4-token verify and a prompt chunk; the graph
    is computed several times in a row, so the CUDA backend replays it as a CUDA graph (ggml-cuda.cu:4347)
  - Builder::deltanet's recurrence with its state and snapshot copies (graph.cpp:166-184): the decode step (where
    ggml-cuda fuses the slot-0 copy into the op, ggml-cuda.cu:3609-3620) and the verify step with f16 snapshots
  - State::rollback_recurrent's copies (state.cpp:162-183)
The library is built from the reference tree (make -C klein_b200/ggml); without it the tests skip."""
import ctypes
import os

import numpy as np
import pytest

import oracle as O
from parity import DELTANET_TOL, check_attention

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "klein_b200", "ggml", "_build",
                   "libkbggml.so")
HD, NH, NKV = 256, 24, 4
P = ctypes.c_void_p


@pytest.fixture(scope="module")
def gg(kb, cuda):
    if not os.path.exists(LIB):
        pytest.skip("klein_b200/ggml/_build/libkbggml.so not built (make -C klein_b200/ggml needs the reference tree)")
    L = ctypes.CDLL(LIB)
    L.kbggml_attention.restype = ctypes.c_int
    L.kbggml_attention.argtypes = [ctypes.c_int] * 8 + [P] * 5 + [ctypes.c_int, ctypes.c_int]
    L.kbggml_deltanet.restype = ctypes.c_int
    L.kbggml_deltanet.argtypes = [ctypes.c_int] * 7 + [P] * 8 + [ctypes.c_int, ctypes.c_int]
    L.kbggml_rollback.restype = ctypes.c_int
    L.kbggml_rollback.argtypes = [ctypes.c_int] * 3 + [ctypes.c_int64] * 2 + [ctypes.c_int, P, P, P, ctypes.c_int]
    return L


def ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


def padded(n, n_ctx):  # graph.cpp:16-19
    return min(n_ctx, (n + 255) // 256 * 256)


@pytest.mark.parametrize("kvt", ["f16", "q8_0", "q4_0"])
@pytest.mark.parametrize("n_q,n_past", [(1, 3000), (4, 4000), (256, 768)])
def test_attention_node(gg, kvt, n_q, n_past):
    n_ctx = 8192
    gt = {"f16": O.GGML_F16, "q8_0": O.GGML_Q8_0, "q4_0": O.GGML_Q4_0}[kvt]
    q, kc, vc, kd, vd = O.make_fa_inputs(77 + n_q + gt, n_q, n_ctx, kv_type=gt)
    n_kv = padded(n_past + n_q, n_ctx)
    mask = O.rs_visible_mask(n_q, n_kv, n_past)
    m16 = mask.astype(np.float16)
    outs = {}
    for use_cuda in (1, 0):
        out = np.zeros((n_q, NH, HD), dtype=np.float32)
        rc = gg.kbggml_attention(use_cuda, gt, n_q, n_ctx, n_kv, HD, NH, NKV, ptr(q), ptr(kc), ptr(vc), ptr(m16), ptr(out),
                                 3 if use_cuda else 1, 8)
        assert rc == 0
        outs[use_cuda] = out
    qr = O.q_round_f16(q) if kvt == "f16" else O.q_round_q8_0(q)
    exact = O.rs_flash_attn_f64(qr, kd[:n_kv], vd[:n_kv], mask=mask)
    check_attention(outs[1], exact, outs[0])


def gdn_inputs(T, seed):
    q, k, v, g, beta, s0 = O.make_gdn_inputs(seed, T)
    return [np.ascontiguousarray(x, dtype=np.float32) for x in (q[0], k[0], v[0], g[0], beta[0], s0[0])]


@pytest.mark.parametrize("T,snap", [(1, "f32"), (4, "f16"), (4, "f32")])
def test_deltanet_node(gg, T, snap):
    S, HK, HV, K = 128, 16, 48, 4
    q, k, v, g, beta, s0 = gdn_inputs(T, 900 + T)
    D = S * S * HV
    st = O.GGML_F32 if snap == "f32" else O.GGML_F16
    res = {}
    for use_cuda in (1, 0):
        state = s0.reshape(-1).copy()
        sn = np.full((K - 1, D), 7.0, dtype=np.float32 if snap == "f32" else np.float16)
        attn = np.zeros(S * HV * T, dtype=np.float32)
        rc = gg.kbggml_deltanet(use_cuda, S, HK, HV, T, K, st, ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), ptr(state),
                                ptr(sn), ptr(attn), 1, 8)
        assert rc == 0
        res[use_cuda] = (attn, state, sn.astype(np.float32))
    # the exact recurrence: ggml's packed result of attention then K slots, newest first (ops.cpp:11123-11275)
    packed = O.rs_gated_delta_net_f64(q[None], k[None], v[None], g[None], beta[None, ..., None], s0[None], K).reshape(-1)
    attn_x = packed[:S * HV * T]
    slots = packed[S * HV * T:].reshape(K, D)
    for use_cuda in (1, 0):
        attn, state, sn = res[use_cuda]
        assert np.abs(attn - attn_x).max() <= DELTANET_TOL * np.abs(attn_x).max()
        assert np.abs(state - slots[0]).max() <= DELTANET_TOL * np.abs(slots[0]).max()
        for s in range(1, min(T, K)):
            tol = DELTANET_TOL if snap == "f32" else 2e-3  # f16 snapshots: one f16 rounding
            assert np.abs(sn[s - 1] - slots[s]).max() <= tol * np.abs(slots[s]).max()
        for s in range(min(T, K), K):
            assert np.all(sn[s - 1] == 7.0)  # slots past the batch are not written (ggml.h:2649-2651)
    # CUDA (klein_b200) against the CPU backend: f32 results within f32 rounding; f16 snapshot rows within one f16 step
    # (both round the same f32 state, which differs in its last bits between the two summation orders)
    names = ("attention", "state", "snapshots")
    for name, a, b in zip(names, res[1], res[0]):
        tol = 1e-3 if (name == "snapshots" and snap == "f16") else 1e-5
        assert np.abs(a - b).max() <= tol * max(np.abs(b).max(), 1e-30), name


def test_rollback_copies(gg):
    conv_row, ssm_row, K, s = 3 * 10240, 128 * 128 * 48, 4, 2
    rng = np.random.default_rng(5)
    conv0 = rng.standard_normal((K, conv_row), dtype=np.float32)
    snap = rng.standard_normal((K - 1, ssm_row), dtype=np.float32).astype(np.float16)
    ssm0 = rng.standard_normal(ssm_row, dtype=np.float32)
    outs = {}
    for use_cuda in (1, 0):
        conv, ssm = conv0.copy(), ssm0.copy()
        assert gg.kbggml_rollback(use_cuda, s, K, conv_row, ssm_row, O.GGML_F16, ptr(conv), ptr(snap), ptr(ssm), 8) == 0
        outs[use_cuda] = (conv, ssm)
    for use_cuda in (1, 0):
        conv, ssm = outs[use_cuda]
        assert np.array_equal(conv[0], conv0[s]) and np.array_equal(ssm, snap[s - 1].astype(np.float32))
