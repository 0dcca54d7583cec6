"""CPU oracle for the attention hot path — TEST INFRASTRUCTURE ONLY.

Two libraries live here:

* ``librestate.so`` — the C restatement in ``restate.c`` (f64 exact attention, GDN recurrence, q8_0
  rounding, set_rows, LSE combine, rollback), each function citing the reference code it follows.
* ``_ref/libggml_ref_v{3,4}.so`` — the reference's own ggml CPU implementation of the ops, compiled from
  the reference sources by ``Makefile`` plus the harness ``ref_harness.cpp``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (cpu_baseline leg and ``--impl reference``)
may import this package, and only as the checker or the timed CPU baseline. The ``klein_b200`` product
never imports it.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_double, c_int, c_int64, c_size_t, c_uint16, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_I64, GGML_BF16 = 0, 1, 2, 8, 27, 30
Q8_0_BLOCK = 34


def _ptr(a):
    return None if a is None else c_void_p(a.ctypes.data)


def ctypes_float(x) -> c_float:
    return c_float(float(x))


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return all(x in flags for x in ("avx512f", "avx512bw", "avx512vl", "avx512dq"))
    except OSError:
        return False


_restate = None
_ref = None


def restate():
    """ctypes handle of librestate.so (built by ``make -C oracle restate``)."""
    global _restate
    if _restate is None:
        path = os.path.join(HERE, "librestate.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run `make -C oracle restate`")
        lib = ctypes.CDLL(path)
        lib.rs_fp32_to_fp16.restype = c_uint16
        lib.rs_fp32_to_fp16.argtypes = [c_float]
        lib.rs_fp16_to_fp32.restype = c_float
        lib.rs_visible.restype = c_int
        lib.rs_visible.argtypes = [c_int64] * 6
        lib.rs_set_rows.restype = c_int
        _restate = lib
    return _restate


def ref_available() -> bool:
    return any(os.path.exists(os.path.join(REF_DIR, f"libggml_ref_{v}.so")) for v in ("v3", "v4"))


def ref():
    """ctypes handle of the reference ggml CPU library (prebuilt into oracle/_ref)."""
    global _ref
    if _ref is None:
        order = ("v4", "v3") if _cpu_has_avx512() else ("v3",)
        for v in order:
            path = os.path.join(REF_DIR, f"libggml_ref_{v}.so")
            if os.path.exists(path):
                lib = ctypes.CDLL(path)
                break
        else:
            raise RuntimeError("reference ggml CPU library missing: run `make -C oracle ref` where the reference tree exists")
        lib.kbref_flash_attn_ext.restype = c_int
        lib.kbref_flash_attn_ext.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int64, c_int,
                                             c_size_t, c_void_p, c_float, c_float, c_float, c_void_p, c_int, c_int]
        lib.kbref_gated_delta_net.restype = c_int
        lib.kbref_gated_delta_net.argtypes = [c_void_p] * 6 + [c_int] * 7 + [c_void_p, c_int]
        lib.kbref_quantize_q8_0.restype = c_size_t
        lib.kbref_quantize_q8_0.argtypes = [c_void_p, c_void_p, c_int64, c_int64]
        lib.kbref_dequantize.argtypes = [c_int, c_void_p, c_void_p, c_int64]
        lib.kbref_set_rows.restype = c_int
        lib.kbref_set_rows.argtypes = [c_void_p, c_int, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int]
        lib.kbref_cpy.restype = c_int
        lib.kbref_cpy.argtypes = [c_void_p, c_int, c_void_p, c_int, c_int64]
        lib.kbref_gdn_input.restype = c_int
        lib.kbref_gdn_input.argtypes = [c_void_p] * 7 + [c_int] * 6 + [c_float] + [c_void_p] * 5 + [c_int]
        lib.kbref_gdn_gated_norm.restype = c_int
        lib.kbref_gdn_gated_norm.argtypes = [c_void_p] * 3 + [c_int] * 3 + [c_float, c_void_p, c_int]
        lib.kbref_attn_prologue.restype = c_int
        lib.kbref_attn_prologue.argtypes = [c_void_p] * 7 + [c_int] * 4 + [c_float, c_int, c_void_p, c_int, c_float, c_int] + \
            [c_void_p] * 4 + [c_int, c_int64, c_int]
        _ref = lib
    return _ref


# ----------------------------------------------------------------------------------------------------------
# restatement wrappers (numpy in, numpy out)

def rs_quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """f32 [..., n] (n % 32 == 0) -> uint8 [..., n/32*34] in ggml's block_q8_0 layout."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    out = np.empty(x.shape[:-1] + (n // 32 * Q8_0_BLOCK,), dtype=np.uint8)
    restate().rs_quantize_row_q8_0(_ptr(x), _ptr(out), c_int64(x.size))
    return out


def rs_dequantize_q8_0(y: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(y, dtype=np.uint8)
    nb = y.shape[-1] // Q8_0_BLOCK
    out = np.empty(y.shape[:-1] + (nb * 32,), dtype=np.float32)
    restate().rs_dequantize_row_q8_0(_ptr(y), _ptr(out), c_int64(out.size))
    return out


def rs_quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """f32 [..., n] (n % 32 == 0) -> uint8 [..., n/32*18] in ggml's block_q4_0 layout."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    out = np.empty(x.shape[:-1] + (n // 32 * 18,), dtype=np.uint8)
    restate().rs_quantize_row_q4_0(_ptr(x), _ptr(out), c_int64(x.size))
    return out


def rs_dequantize_q4_0(y: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(y, dtype=np.uint8)
    nb = y.shape[-1] // 18
    out = np.empty(y.shape[:-1] + (nb * 32,), dtype=np.float32)
    restate().rs_dequantize_row_q4_0(_ptr(y), _ptr(out), c_int64(out.size))
    return out


def rs_visible_mask(n_q: int, n_kv: int, pos0: int, kv_lo: int = 0, ring: int = 0) -> np.ndarray:
    """klein's dense mask as f32 [n_q][n_kv] (0 visible, -inf hidden)."""
    j = np.arange(n_kv, dtype=np.int64)[None, :]
    i = np.arange(n_q, dtype=np.int64)[:, None]
    p = pos0 + i
    if ring == 0:
        vis = (j >= kv_lo) & (j <= p)
    else:
        end = pos0 + n_q - 1
        c = end - (((end - j) % ring) + ring) % ring
        vis = (c >= kv_lo) & (c <= p) & (c > p - ring)
    return np.where(vis, 0.0, -np.inf).astype(np.float32)


def rs_flash_attn_f64(q, k, v, mask=None, scale=1.0 / 16, max_bias=0.0, softcap=0.0) -> np.ndarray:
    """Exact attention. q f32 [n_q][H][D]; k, v f32 [n_kv][H_kv][D]; mask f32 [n_q][n_kv] or None."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    n_q, H, D = q.shape
    n_kv, H_kv, _ = k.shape
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    out = np.empty((n_q, H, D), dtype=np.float64)
    restate().rs_flash_attn_f64(_ptr(q), c_int(n_q), c_int(H), c_int(D), _ptr(k), _ptr(v), c_int64(n_kv), c_int(H_kv),
                                _ptr(m), c_float(scale), c_float(max_bias), c_float(softcap), _ptr(out))
    return out


def rs_lse_combine(o_part, m, l) -> np.ndarray:
    o_part = np.ascontiguousarray(o_part, dtype=np.float32)
    m = np.ascontiguousarray(m, dtype=np.float32)
    l = np.ascontiguousarray(l, dtype=np.float32)
    P, R, D = o_part.shape
    out = np.empty((R, D), dtype=np.float32)
    restate().rs_lse_combine(_ptr(o_part), _ptr(m), _ptr(l), c_int(P), c_int(R), c_int(D), _ptr(out))
    return out


def rs_gated_delta_net_f64(q, k, v, g, beta, s0, K: int) -> np.ndarray:
    """Shapes as ``ref_gated_delta_net``; returns the packed f64 output."""
    q, k, v, g, beta, s0 = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, g, beta, s0))
    n_seqs, T, H_k, S = q.shape
    H_v = v.shape[2]
    kda = int(g.shape[-1] == S and g.ndim == 4)
    n_out = S * H_v * T * n_seqs + K * S * S * H_v * n_seqs
    out = np.zeros(n_out, dtype=np.float64)
    restate().rs_gated_delta_net_f64(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(s0), c_int(S), c_int(H_k),
                                     c_int(H_v), c_int(T), c_int(n_seqs), c_int(kda), c_int(K), _ptr(out))
    return out


def rs_set_rows(cache: np.ndarray, dst_type: int, row_elems: int, src: np.ndarray, idx: np.ndarray) -> int:
    """In-place cache row write; cache uint8 [n_rows][row_bytes]."""
    src = np.ascontiguousarray(src, dtype=np.float32)
    idx = np.ascontiguousarray(idx, dtype=np.int64)
    return restate().rs_set_rows(_ptr(cache), c_int(dst_type), c_int64(row_elems), c_size_t(cache.shape[1]),
                                 c_int64(cache.shape[0]), _ptr(src), c_int64(src.shape[0]), _ptr(idx))


def rs_rollback(conv: np.ndarray, snap: np.ndarray, ssm: np.ndarray, s: int) -> None:
    """conv f32 [n_snap][conv_row], snap f16 [n_snap-1][ssm_row] (as uint16 or float16), ssm f32 [ssm_row]."""
    restate().rs_rollback(_ptr(conv), c_int64(conv.shape[1]), _ptr(snap), _ptr(ssm), c_int64(ssm.shape[-1]), c_int(s))


# ----------------------------------------------------------------------------------------------------------
# reference (ggml CPU) wrappers

def ref_flash_attn_ext(q, k_cache, v_cache, kv_type, n_head_kv, mask=None, scale=1.0 / 16, max_bias=0.0, softcap=0.0,
                       n_threads=1, use_ref=True) -> np.ndarray:
    """ggml_flash_attn_ext on ggml's CPU backend with klein's views.

    q: f32 [n_q][H][D]; k_cache/v_cache: raw rows (f16 as uint16/float16 [n_kv][H_kv*D], q8_0 as uint8
    [n_kv][H_kv*D/32*34]); mask: f16 [n_q][n_kv] or None. Returns f32 [n_q][H][D].
    """
    q = np.ascontiguousarray(q, dtype=np.float32)
    n_q, H, D = q.shape
    n_kv = k_cache.shape[0]
    row_bytes = k_cache.strides[0]
    assert k_cache.flags.c_contiguous and v_cache.flags.c_contiguous
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float16)
    out = np.empty((n_q, H, D), dtype=np.float32)
    rc = ref().kbref_flash_attn_ext(_ptr(q), n_q, H, D, _ptr(k_cache), _ptr(v_cache), kv_type, n_kv, n_head_kv, row_bytes,
                                    _ptr(m), scale, max_bias, softcap, _ptr(out), n_threads, int(use_ref))
    assert rc == 0
    return out


def ref_gated_delta_net(q, k, v, g, beta, s0, K: int, n_threads=1) -> np.ndarray:
    """q, k f32 [n_seqs][T][H_k][S]; v [n_seqs][T][H_v][S]; g [n_seqs][T][H_v][1 or S]; beta [n_seqs][T][H_v];
    s0 [n_seqs][H_v][S][S]. Returns ggml's packed f32 output (attn, then K state slots)."""
    q, k, v, g, beta, s0 = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, g, beta, s0))
    n_seqs, T, H_k, S = q.shape
    H_v = v.shape[2]
    kda = int(g.shape[-1] == S)
    n_out = S * H_v * T * n_seqs + K * S * S * H_v * n_seqs
    out = np.zeros(n_out, dtype=np.float32)
    rc = ref().kbref_gated_delta_net(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(s0), S, H_k, H_v, T, n_seqs,
                                     kda, K, _ptr(out), n_threads)
    assert rc == 0
    return out


def ref_quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    nrows = x.size // n
    out = np.empty(x.shape[:-1] + (n // 32 * Q8_0_BLOCK,), dtype=np.uint8)
    ref().kbref_quantize_q8_0(_ptr(x), _ptr(out), nrows, n)
    return out


def ref_dequantize(type_: int, y: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    ref().kbref_dequantize(type_, _ptr(np.ascontiguousarray(y)), _ptr(out), n)
    return out


def ref_set_rows(cache: np.ndarray, dst_type: int, row_elems: int, src: np.ndarray, idx: np.ndarray, n_threads=1) -> int:
    src = np.ascontiguousarray(src, dtype=np.float32)
    idx = np.ascontiguousarray(idx, dtype=np.int64)
    return ref().kbref_set_rows(_ptr(cache), dst_type, row_elems, cache.shape[0], _ptr(src), src.shape[0], _ptr(idx),
                                n_threads)


def ref_attn_prologue(qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm, eps, n_rot, sections, mode, freq_base,
                      k_cache, v_cache, cache_type, n_ctx_orig=262144, n_threads=1):
    """Builder::attention's prologue on the reference ggml CPU ops (graph.cpp:94-112). qfull f32 [n][nh * 2 hd],
    kcur / vcur f32 [n][nkv * hd], pos i32 [4 n], kv_idx i64 [n], q_norm / k_norm f32 [hd]; the caches (numpy
    byte or f16 arrays [n_cells][row]) are written in place. Returns (q [n][nh][hd], gate [n][nh * hd])."""
    qfull = np.ascontiguousarray(qfull, dtype=np.float32)
    kcur = np.ascontiguousarray(kcur, dtype=np.float32)
    vcur = np.ascontiguousarray(vcur, dtype=np.float32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    kv_idx = np.ascontiguousarray(kv_idx, dtype=np.int64)
    q_norm = np.ascontiguousarray(q_norm, dtype=np.float32)
    k_norm = np.ascontiguousarray(k_norm, dtype=np.float32)
    hd = q_norm.shape[0]
    n = qfull.shape[0]
    nh = qfull.shape[1] // (2 * hd)
    nkv = kcur.shape[1] // hd
    sec = np.ascontiguousarray(sections, dtype=np.int32)
    q_out = np.zeros((n, nh, hd), np.float32)
    gate = np.zeros((n, nh * hd), np.float32)
    rc = ref().kbref_attn_prologue(_ptr(qfull), _ptr(kcur), _ptr(vcur), _ptr(pos), _ptr(kv_idx), _ptr(q_norm),
                                   _ptr(k_norm), hd, nh, nkv, n, eps, n_rot, _ptr(sec), mode, freq_base, n_ctx_orig,
                                   _ptr(q_out), _ptr(gate), _ptr(k_cache), _ptr(v_cache), cache_type, k_cache.shape[0],
                                   n_threads)
    assert rc == 0
    return q_out, gate


def ref_gdn_input(qkv, conv_state, conv_w, beta_raw, alpha, dt_bias, a, S, H_k, eps, n_threads=1):
    """Builder::deltanet's input side on the reference ggml CPU ops (graph.cpp:136-165). qkv f32 [n][ch],
    conv_state f32 [K][(kc - 1) ch] (written in place), conv_w f32 [ch][kc], beta_raw / alpha f32 [n][H_v],
    dt_bias / a f32 [H_v]. Returns (q [n][H_k][S], k, v [n][H_v][S], beta [n][H_v], g [n][H_v])."""
    f = lambda x: np.ascontiguousarray(x, dtype=np.float32)
    qkv, conv_w, beta_raw, alpha, dt_bias, a = map(f, (qkv, conv_w, beta_raw, alpha, dt_bias, a))
    assert conv_state.dtype == np.float32 and conv_state.flags.c_contiguous
    n, ch = qkv.shape
    H_v = (ch - 2 * S * H_k) // S
    kc = conv_w.shape[1]
    K = conv_state.shape[0]
    q = np.zeros((n, H_k, S), np.float32)
    k = np.zeros_like(q)
    v = np.zeros((n, H_v, S), np.float32)
    beta = np.zeros((n, H_v), np.float32)
    g = np.zeros_like(beta)
    rc = ref().kbref_gdn_input(_ptr(qkv), _ptr(conv_state), _ptr(conv_w), _ptr(beta_raw), _ptr(alpha), _ptr(dt_bias),
                               _ptr(a), S, H_k, H_v, kc, K, n, eps, _ptr(q), _ptr(k), _ptr(v), _ptr(beta), _ptr(g),
                               n_threads)
    assert rc == 0
    return q, k, v, beta, g


def ref_gdn_gated_norm(x, z, w, eps, n_threads=1):
    """rms_norm(x, eps) * w * silu(z) on the reference's ops (graph.cpp:186-190); x, z f32 [n][H][S], w f32 [S]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    z = np.ascontiguousarray(z, dtype=np.float32).reshape(x.shape)
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, H, S = x.shape
    dst = np.zeros_like(x)
    assert ref().kbref_gdn_gated_norm(_ptr(x), _ptr(z), _ptr(w), S, H, n, eps, _ptr(dst), n_threads) == 0
    return dst


def ref_cpy(src: np.ndarray, src_type: int, dst: np.ndarray, dst_type: int) -> int:
    return ref().kbref_cpy(_ptr(src), src_type, _ptr(dst), dst_type, src.size)


# ----------------------------------------------------------------------------------------------------------
# seeded synthetic inputs (the BASELINE configurations' distributions)

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """IEEE f32 -> bf16 bit patterns, round to nearest even (ggml's GGML_FP32_TO_BF16 for finite values)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def q_round_bf16(q: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(q)).reshape(q.shape)


def make_fa_inputs(seed: int, n_q: int, n_kv: int, H=24, H_kv=4, D=256, kv_type=GGML_F16):
    """Q f32 [n_q][H][D] ~N(0,1); K, V cache rows ~N(0,1) stored as kv_type. Returns (q, k_cache, v_cache,
    k_deq, v_deq) where *_deq are the exact f32 values the cache holds."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_q, H, D), dtype=np.float32)
    kf = rng.standard_normal((n_kv, H_kv * D), dtype=np.float32)
    vf = rng.standard_normal((n_kv, H_kv * D), dtype=np.float32)
    if kv_type == GGML_F16:
        kc, vc = kf.astype(np.float16), vf.astype(np.float16)
        kd, vd = kc.astype(np.float32), vc.astype(np.float32)
    elif kv_type == GGML_Q8_0:
        kc, vc = rs_quantize_q8_0(kf), rs_quantize_q8_0(vf)
        kd, vd = rs_dequantize_q8_0(kc), rs_dequantize_q8_0(vc)
    elif kv_type == GGML_Q4_0:
        kc, vc = rs_quantize_q4_0(kf), rs_quantize_q4_0(vf)
        kd, vd = rs_dequantize_q4_0(kc), rs_dequantize_q4_0(vc)
    elif kv_type == GGML_BF16:
        kc, vc = f32_to_bf16_bits(kf), f32_to_bf16_bits(vf)
        kd, vd = bf16_bits_to_f32(kc).reshape(kf.shape), bf16_bits_to_f32(vc).reshape(vf.shape)
    else:
        raise ValueError(kv_type)
    return q, kc, vc, kd.reshape(n_kv, H_kv, D), vd.reshape(n_kv, H_kv, D)


def make_gdn_inputs(seed: int, T: int, H_k=16, H_v=48, S=128, n_seqs=1, s0_std=0.02, kda=False):
    """config[1] distributions: q, k ~N(0,1) then L2-normalised; v ~N(0,1); beta = sigmoid(N(0,1));
    g = -softplus(N(0,1)); s0 ~N(0, s0_std)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_seqs, T, H_k, S), dtype=np.float32)
    k = rng.standard_normal((n_seqs, T, H_k, S), dtype=np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((n_seqs, T, H_v, S), dtype=np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((n_seqs, T, H_v))))).astype(np.float32)
    graw = rng.standard_normal((n_seqs, T, H_v, S if kda else 1))
    g = (-np.logaddexp(0.0, graw)).astype(np.float32)
    s0 = (rng.standard_normal((n_seqs, H_v, S, S)) * s0_std).astype(np.float32)
    return q, k, v, g, beta, s0


def q_round_f16(q: np.ndarray) -> np.ndarray:
    """Q as ggml's f16 K dot type sees it (ops.cpp:8960 with vec_dot_type f16)."""
    return q.astype(np.float16).astype(np.float32)


def q_round_q8_0(q: np.ndarray) -> np.ndarray:
    """Q as the q8_0 K dot type sees it, with quantize_row_q8_0_ref rounding."""
    return rs_dequantize_q8_0(rs_quantize_q8_0(q))


def rs_attn_prologue(qfull, kcur, pos, q_norm, k_norm, eps, n_rot, sections, mode, freq_base):
    """Restatement of the attention prologue's arithmetic (TEST INFRASTRUCTURE): RMS norm with weight
    (ggml-cpu/ops.cpp:4107-4167) and ggml_rope_multi (ops.cpp:6219-6306, 6376-6450) on q and k. The rope angles
    follow ggml's running f32 product theta_{i+1} = theta_i * theta_scale; the rest is float64.
    Returns (q [n][nh][hd], k [n][nkv][hd], gate [n][nh * hd])."""
    hd = q_norm.shape[0]
    n = qfull.shape[0]
    nh = qfull.shape[1] // (2 * hd)
    nkv = kcur.shape[1] // hd
    qg = qfull.reshape(n, nh, 2, hd).astype(np.float64)
    q, gate = qg[:, :, 0, :], qg[:, :, 1, :].reshape(n, nh * hd)
    k = kcur.reshape(n, nkv, hd).astype(np.float64)

    def rms(x, w):
        ms = (x * x).mean(-1, keepdims=True)
        return x / np.sqrt(ms + eps) * w.astype(np.float64)

    q, k = rms(q, q_norm), rms(k, k_norm)
    half = n_rot // 2
    sect = sum(sections)
    theta_scale = np.float32(np.power(np.float32(freq_base), np.float32(-2.0) / np.float32(n_rot)))
    cos = np.zeros((n, half))
    sin = np.zeros((n, half))
    for t in range(n):
        th = [np.float32(pos[c * n + t]) for c in range(4)]
        for i in range(half):
            sector = i % sect
            if mode == 40:
                if sector % 3 == 1 and sector < 3 * sections[1]:
                    c = 1
                elif sector % 3 == 2 and sector < 3 * sections[2]:
                    c = 2
                elif sector % 3 == 0 and sector < 3 * sections[0]:
                    c = 0
                else:
                    c = 3
            else:
                sw = sections[0] + sections[1]
                c = 1 if sections[0] <= sector < sw else 2 if sw <= sector < sw + sections[2] else 3 if sector >= sw + sections[2] else 0
            cos[t, i] = np.cos(np.float64(th[c]))
            sin[t, i] = np.sin(np.float64(th[c]))
            th = [np.float32(x * theta_scale) for x in th]

    def rope(x):
        y = x.copy()
        x0, x1 = x[..., :half], x[..., half:n_rot]
        c, s_ = cos[:, None, :], sin[:, None, :]
        y[..., :half] = x0 * c - x1 * s_
        y[..., half:n_rot] = x0 * s_ + x1 * c
        return y

    return rope(q), rope(k), gate


def rs_gdn_input(qkv, conv_state, conv_w, beta_raw, alpha, dt_bias, a, S, H_k, eps):
    """Restatement of the DeltaNet input side (TEST INFRASTRUCTURE; graph.cpp:136-165 with ggml's ops):
    float64 conv over [state | batch] (ops.cpp:9931-9982), silu, l2 = rms_norm(eps / S) / sqrt(S), the gates,
    and the conv-state snapshot rule. Returns (q, k, v, beta, g, new_state)."""
    n, ch = qkv.shape
    H_v = (ch - 2 * S * H_k) // S
    kc = conv_w.shape[1]
    K = conv_state.shape[0]
    old = conv_state[0].reshape(ch, kc - 1).astype(np.float64)
    seq = np.concatenate([old, qkv.T.astype(np.float64)], axis=1)  # [ch][kc - 1 + n]
    w = conv_w.astype(np.float64)
    conv = np.stack([(seq[:, t:t + kc] * w).sum(1) for t in range(n)], 0)  # [n][ch]
    conv = conv / (1.0 + np.exp(-conv))
    q = conv[:, :S * H_k].reshape(n, H_k, S)
    k = conv[:, S * H_k:2 * S * H_k].reshape(n, H_k, S)
    v = conv[:, 2 * S * H_k:].reshape(n, H_v, S)

    def l2(x):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps / S) / np.sqrt(S)

    beta = 1.0 / (1.0 + np.exp(-beta_raw.astype(np.float64)))
    xg = alpha.astype(np.float64) + dt_bias.astype(np.float64)
    g = np.where(xg > 20.0, xg, np.log1p(np.exp(np.minimum(xg, 20.0)))) * a.astype(np.float64)
    state = conv_state.copy()
    for s_ in range(K):
        if s_ >= n and s_ > 0:
            continue
        start = max(0, n - s_)
        state[s_] = seq[:, start:start + kc - 1].astype(np.float32).reshape(-1)
    return l2(q), l2(k), v, beta, g, state


def rs_gdn_gated_norm(x, z, w, eps):
    """rms_norm(x, eps) * w * silu(z) in float64 (graph.cpp:186-190)."""
    x = x.astype(np.float64)
    z = z.astype(np.float64).reshape(x.shape)
    y = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w.astype(np.float64)
    return y * z / (1.0 + np.exp(-z))
