"""kb_flash_attn_ext_noalloc: the attention entry point for callers that cannot allocate device memory.

Some callers of this library have no way to hand it scratch memory: code that runs while a CUDA graph is
being captured (cudaMalloc is not allowed there), hosts that give the whole GPU to their own memory pools
at start-up, and foreign-language bindings that only pass raw pointers. For them the library keeps the
split-KV partials in a fixed device buffer of its own. This test calls that entry point through the C ABI
and checks that it gives the same output as kb_flash_attn_ext (with caller scratch), on two calls in a
row, the second on different inputs so that leftovers of the first call in the shared buffer would show.

The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from parity import ATTN_TOL, rel_err

pytestmark = pytest.mark.gpu


def _inputs(kb, cuda, seed, n_q, n_kv):
    import torch

    q, kc, vc, kd, vd = O.make_fa_inputs(seed, n_q, n_kv)
    qt = torch.from_numpy(q).to(cuda).unsqueeze(0)
    kt, vt = torch.from_numpy(kc).to(cuda), torch.from_numpy(vc).to(cuda)
    qv = kb.kb_tensor(qt.data_ptr(), kb.F32, [256, n_q, 24, 1], [4, 24 * 256 * 4, 256 * 4, n_q * 24 * 256 * 4])
    return (qt, kt, vt), qv, kb.kv_cache_view(kt, kb.F16, 4, 256), kb.kv_cache_view(vt, kb.F16, 4, 256)


def _out(kb, cuda, n_q):
    import torch

    o = torch.full((1, n_q, 24, 256), float("nan"), device=cuda)
    return o, kb.kb_tensor(o.data_ptr(), kb.F32, [256, 24, n_q, 1], [4, 256 * 4, 24 * 256 * 4, n_q * 24 * 256 * 4])


def test_noalloc_matches_allocating_entry_point_twice(kb, cuda):
    import torch

    L = kb.lib()
    for call, (seed, n_q, n_kv) in enumerate([(501, 4, 262144), (502, 4, 70001)]):
        keep, qv, kv, vv = _inputs(kb, cuda, seed, n_q, n_kv)
        prm = kb.fa_params(1 / 16, causal=True, pos0=n_kv - n_q)
        need = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(prm))
        assert 0 < need <= kb.NOALLOC_SCRATCH_BYTES
        scratch = torch.empty(need, dtype=torch.uint8, device=cuda)
        ref_o, ref_t = _out(kb, cuda, n_q)
        rc = L.kb_flash_attn_ext(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), None, ctypes.byref(prm),
                                 ctypes.byref(ref_t), ctypes.c_void_p(scratch.data_ptr()), need, None)
        assert rc == kb.KB_OK
        na_o, na_t = _out(kb, cuda, n_q)
        rc = L.kb_flash_attn_ext_noalloc(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), None, ctypes.byref(prm),
                                         ctypes.byref(na_t), None)
        assert rc == kb.KB_OK, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        a, b = na_o.cpu().numpy(), ref_o.cpu().numpy()
        assert np.isfinite(a).all()
        assert rel_err(a, b) <= ATTN_TOL, f"call {call}: no-alloc vs allocating entry point {rel_err(a, b):.3e}"
        del keep


def test_noalloc_buffer_covers_every_split_plan(kb, cuda):
    """The split plan keeps the partials of one call at most (SM count x 32 rows x (256 + 2) floats), so the
    built-in buffer covers every shape on this GPU; a 64-token call (many row chunks) matches the allocating
    entry point."""
    import torch

    L = kb.lib()
    for n_q, n_kv, H in [(1, 262144, 24), (4, 262144, 24), (16, 262144, 24), (64, 8192, 24), (4, 1 << 20, 32)]:
        q = torch.zeros(1, n_q, H, 256, device=cuda)
        k = torch.zeros(64, 4 * 256, dtype=torch.float16, device=cuda)
        qv = kb.kb_tensor(q.data_ptr(), kb.F32, [256, n_q, H, 1], [4, H * 256 * 4, 256 * 4, n_q * H * 256 * 4])
        kv = kb.kb_tensor(k.data_ptr(), kb.F16, [256, n_kv, 4, 1], [2, 2048, 512, 2048 * n_kv])
        prm = kb.fa_params(1 / 16)
        need = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(kv), ctypes.byref(prm))
        assert need <= kb.NOALLOC_SCRATCH_BYTES, (n_q, n_kv, H, need)
    n_q, n_kv = 64, 9000
    keep, qv, kv, vv = _inputs(kb, cuda, 503, n_q, n_kv)
    prm = kb.fa_params(1 / 16, causal=True, pos0=n_kv - n_q)
    need = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(prm))
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=cuda)
    ref_o, ref_t = _out(kb, cuda, n_q)
    assert L.kb_flash_attn_ext(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), None, ctypes.byref(prm),
                               ctypes.byref(ref_t), ctypes.c_void_p(scratch.data_ptr()), need, None) == kb.KB_OK
    na_o, na_t = _out(kb, cuda, n_q)
    assert L.kb_flash_attn_ext_noalloc(ctypes.byref(qv), ctypes.byref(kv), ctypes.byref(vv), None, ctypes.byref(prm),
                                       ctypes.byref(na_t), None) == kb.KB_OK
    torch.cuda.synchronize()
    assert rel_err(na_o.cpu().numpy(), ref_o.cpu().numpy()) <= ATTN_TOL
