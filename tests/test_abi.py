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
