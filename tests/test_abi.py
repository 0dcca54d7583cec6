"""The C-ABI library loads, exports every symbol include/klein_b200.h declares, and rejects malformed
descriptors before touching the device (runs without a GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    with open(os.path.join(ROOT, "include", "klein_b200.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_declared_symbols(kb):
    L = kb.lib()
    decl = declared_symbols()
    assert decl, "no kb_* declarations found"
    for name in decl:
        assert hasattr(L, name), f"{name} declared in include/klein_b200.h but not exported"
    assert sorted(kb.EXPORTED) == decl


def test_version(kb):
    assert kb.lib().kb_version().startswith(b"klein_b200")


def _fa_args(kb, **over):
    D, n_q, H, n_kv, H_kv = 256, 4, 24, 1024, 4
    fake = 1 << 20  # never dereferenced: validation fails first
    q = kb.kb_tensor(fake, kb.F32, [D, n_q, H, 1], [4, H * D * 4, D * 4, n_q * H * D * 4])
    k = kb.kb_tensor(fake, kb.F16, [D, n_kv, H_kv, 1], [2, 2048, 512, 2048 * n_kv])
    v = kb.kb_tensor(fake, kb.F16, [D, n_kv, H_kv, 1], [2, 2048, 512, 2048 * n_kv])
    dst = kb.kb_tensor(fake, kb.F32, [D, H, n_q, 1], [4, D * 4, H * D * 4, n_q * H * D * 4])
    args = dict(q=q, k=k, v=v, dst=dst)
    args.update(over)
    return args


def _call(kb, a):
    prm = kb.fa_params(1 / 16)
    return kb.lib().kb_flash_attn_ext(ctypes.byref(a["q"]), ctypes.byref(a["k"]), ctypes.byref(a["v"]), None,
                                      ctypes.byref(prm), ctypes.byref(a["dst"]), None, 0, None)


def test_fa_rejects_bad_descriptors(kb):
    a = _fa_args(kb)
    a["q"].type = kb.F16
    assert _call(kb, a) == kb.KB_ERR_UNSUPPORTED
    a = _fa_args(kb)
    a["k"].ne[0] = 128
    assert _call(kb, a) == kb.KB_ERR_BAD_SHAPE
    a = _fa_args(kb)
    a["v"].type = kb.Q8_0
    assert _call(kb, a) == kb.KB_ERR_UNSUPPORTED
    a = _fa_args(kb)
    a["k"].ne[2] = 5  # 24 % 5 != 0
    a["v"].ne[2] = 5
    assert _call(kb, a) == kb.KB_ERR_BAD_SHAPE
    a = _fa_args(kb)
    a["dst"].ne[1] = 23
    assert _call(kb, a) == kb.KB_ERR_BAD_SHAPE
    a = _fa_args(kb)
    a["k"].nb[1] = 2040  # TMA needs 16-byte strides
    assert _call(kb, a) == kb.KB_ERR_UNSUPPORTED
    assert kb.lib().kb_flash_attn_ext(None, None, None, None, None, None, None, 0, None) == kb.KB_ERR_ARG


no_gpu = pytest.mark.skipif(__import__("torch").cuda.is_available(),
                            reason="passing validation would launch on host pointers")


@no_gpu
def test_gdn_descriptors_validate(kb):
    """Operands shaped like klein's DeltaNet node pass validation (the call then fails only for lack of a GPU),
    malformed ones are rejected."""
    import numpy as np
    import torch

    import oracle as O

    q, k, v, g, beta, s0 = O.make_gdn_inputs(1, 4)
    ts = [torch.from_numpy(np.ascontiguousarray(a)) for a in (q, k, v, g, beta[..., None], s0)]
    args = [kb.from_torch(t) for t in ts]
    S, H, T, K = 128, 48, 4, 4
    out = torch.zeros(S * H * T + K * S * S * H)
    dt = kb.kb_tensor(out.data_ptr(), kb.F32, [S * H, T + K * S, 1, 1], [4, S * H * 4])
    call = lambda a, d=dt, K_=K: kb.lib().kb_gated_delta_net(*[ctypes.byref(x) for x in a], K_, ctypes.byref(d), None, 0,
                                                             None)
    assert call(args) == kb.KB_ERR_CUDA  # validation passed; no device here
    bad = list(args)
    bad[3] = kb.from_torch(torch.zeros(1, T, H, 7))  # gate neither scalar nor per-channel
    assert call(bad) == kb.KB_ERR_BAD_SHAPE
    assert call(args, K_=0) == kb.KB_ERR_BAD_SHAPE
    small = kb.kb_tensor(out.data_ptr(), kb.F32, [S * H, T + K * S - 1, 1, 1], [4, S * H * 4])
    assert call(args, d=small) == kb.KB_ERR_BAD_SHAPE
    snap = torch.zeros(K - 1, S * S * H, dtype=torch.float16)
    attn = torch.zeros(1, T, H, S)
    rc = kb.lib().kb_gated_delta_net_cache(*[ctypes.byref(x) for x in args], ctypes.byref(kb.from_torch(snap)), K,
                                           ctypes.byref(kb.from_torch(attn)), None, 0, None)
    assert rc == kb.KB_ERR_CUDA


@no_gpu
def test_set_rows_and_rollback_validate(kb):
    import torch

    cache = torch.zeros(16, 1024, dtype=torch.float16)
    src = torch.zeros(1, 1, 3, 1024)
    idx = torch.zeros(3, dtype=torch.int64)
    L = kb.lib()
    d, s_, i_ = kb.from_torch(cache), kb.from_torch(src), kb.from_torch(idx)
    assert L.kb_set_rows(ctypes.byref(d), ctypes.byref(s_), ctypes.byref(i_), None) == kb.KB_ERR_CUDA
    odd = kb.from_torch(torch.zeros(1, 1, 3, 1000))
    assert L.kb_set_rows(ctypes.byref(d), ctypes.byref(odd), ctypes.byref(i_), None) == kb.KB_ERR_BAD_SHAPE
    f = ctypes.c_void_p * 1
    assert L.kb_rollback_recurrent(1, f(64), 64, f(64), kb.F16, f(64), 64, 0, 4, None) == kb.KB_OK  # s = 0: no-op
    assert L.kb_rollback_recurrent(1, f(64), 64, f(64), kb.F16, f(64), 64, 4, 4, None) == kb.KB_ERR_ARG
    assert L.kb_rollback_recurrent(1, f(64), 64, f(64), 99, f(64), 64, 1, 4, None) == kb.KB_ERR_UNSUPPORTED
