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


def test_gated_and_push_reject_bad_arguments(kb):
    L = kb.lib()
    prm = kb.fa_params(1 / 16)
    a = _fa_args(kb)
    by = ctypes.byref
    gate = kb.kb_tensor(1 << 20, kb.F32, [256, 24, 4, 1], [4, 256 * 4, 24 * 256 * 4, 4 * 24 * 256 * 4])
    call = lambda g: L.kb_flash_attn_ext_gated(by(a["q"]), by(a["k"]), by(a["v"]), None, by(prm), g, by(a["dst"]),
                                               None, 0, None)
    assert call(None) == kb.KB_ERR_ARG
    bad = kb.kb_tensor(1 << 20, kb.F32, [256, 24, 3, 1], [4, 256 * 4, 24 * 256 * 4, 3 * 24 * 256 * 4])
    assert call(by(bad)) == kb.KB_ERR_BAD_SHAPE  # gate must have the output's shape
    gate.type = kb.F16
    assert call(by(gate)) == kb.KB_ERR_BAD_SHAPE
    # push: peers, ranks and the packed partial size are checked first
    rows, D = 4 * 24, 256
    pf = rows * D + rows * 2
    ptrs = (ctypes.POINTER(ctypes.c_float) * 2)()
    flags = (ctypes.POINTER(ctypes.c_int32) * 2)()
    push = lambda part, rank, n: L.kb_flash_attn_ext_push(by(a["q"]), by(a["k"]), by(a["v"]), None, by(prm), part, ptrs,
                                                         2 * pf, flags, rank, n, None, 0, None)
    assert push(pf, 2, 2) == kb.KB_ERR_ARG  # rank out of range
    assert push(pf - 4, 0, 2) == kb.KB_ERR_BAD_SHAPE  # part smaller than o + (m, l)
    assert push(pf, 0, 2) == kb.KB_ERR_ARG  # null gather buffers
    assert L.kb_flash_attn_ext_push_scratch_bytes(by(a["q"]), by(a["k"]), by(a["v"]), by(prm)) >= \
        L.kb_flash_attn_ext_scratch_bytes(by(a["q"]), by(a["k"]), by(a["v"]), by(prm))


def _prologue_args(torch, kb, n=2, nh=24, nkv=4, hd=256, cache_dtype=None, cache_type=None):
    qfull, kcur, vcur = torch.zeros(n, nh * 2 * hd), torch.zeros(n, nkv * hd), torch.zeros(n, nkv * hd)
    pos, kv_idx = torch.zeros(4 * n, dtype=torch.int32), torch.arange(n, dtype=torch.int64)
    qn = torch.ones(hd)
    cache = torch.zeros(8, nkv * hd, dtype=cache_dtype or torch.float16)
    c = kb.cache_rows(cache, cache_type if cache_type is not None else kb.F16)
    return [qfull, kcur, vcur, pos, kv_idx, qn, qn], c, cache


@no_gpu
def test_prologue_validates(kb):
    import torch

    def status(args, c, n_rot=64, mode=40, vc=None):
        try:
            kb.attn_prologue(*args, 1e-6, n_rot, [11, 11, 10, 0], mode, 1e7, c, vc or c, stream=0)
        except kb.KbError as e:
            return e.status
        return kb.KB_OK

    args, c, _keep = _prologue_args(torch, kb)
    assert status(args, c) == kb.KB_ERR_CUDA  # validation passed; no device here
    assert status(args, c, n_rot=32) == kb.KB_ERR_UNSUPPORTED  # pairs must fill whole warps
    assert status(args, c, mode=0) == kb.KB_ERR_UNSUPPORTED  # M-RoPE modes only
    bad = list(args)
    bad[3] = torch.zeros(8, dtype=torch.int64)  # positions are i32
    assert status(bad, c) == kb.KB_ERR_UNSUPPORTED
    bad = list(args)
    bad[1] = torch.zeros(2, 1000)  # K width not a multiple of the head dim
    assert status(bad, c) == kb.KB_ERR_BAD_SHAPE
    _, c32, _k32 = _prologue_args(torch, kb, cache_dtype=torch.float32, cache_type=kb.F32)
    assert status(args, c32) == kb.KB_ERR_UNSUPPORTED  # caches are f16, q8_0 or q4_0
    q4 = torch.zeros(8, 4 * 8 * 18, dtype=torch.uint8)
    assert status(args, c, vc=kb.cache_rows(q4, kb.Q4_0)) == kb.KB_ERR_UNSUPPORTED  # K and V of one type
    assert status(args, kb.cache_rows(q4, kb.Q4_0)) == kb.KB_ERR_CUDA


@no_gpu
def test_gdn_io_validates(kb):
    import torch

    S, H_k, H_v, n = 128, 16, 48, 2
    ch = 2 * S * H_k + S * H_v
    qkv, state, w = torch.zeros(n, ch), torch.zeros(4, 3 * ch), torch.zeros(ch, 4)

    def status(fn):
        try:
            fn()
        except kb.KbError as e:
            return e.status
        return kb.KB_OK

    assert status(lambda: kb.gdn_input(qkv, state, w, S, H_k, 1e-6, stream=0)) == kb.KB_ERR_CUDA
    assert status(lambda: kb.gdn_input(qkv, state, torch.zeros(ch, 3), S, H_k, 1e-6, stream=0)) == \
        kb.KB_ERR_UNSUPPORTED  # conv kernel width 4 only
    assert status(lambda: kb.gdn_input(qkv, torch.zeros(4, 3 * ch - 3), w, S, H_k, 1e-6, stream=0)) == \
        kb.KB_ERR_BAD_SHAPE
    # 40 key heads leave no value heads: rejected before the device (the empty v output is refused first)
    assert status(lambda: kb.gdn_input(qkv, state, w, S, 40, 1e-6, stream=0)) in (kb.KB_ERR_BAD_SHAPE,
                                                                                 kb.KB_ERR_UNSUPPORTED)
    x = torch.zeros(n, H_v, S)
    assert status(lambda: kb.gdn_gated_norm(x, x, torch.ones(S), 1e-6, stream=0)) == kb.KB_ERR_CUDA
    assert status(lambda: kb.gdn_gated_norm(x, x, torch.ones(96), 1e-6, stream=0)) == kb.KB_ERR_UNSUPPORTED
    y = torch.zeros(n, H_v, 64)
    assert status(lambda: kb.gdn_gated_norm(y, y, torch.ones(S), 1e-6, stream=0)) == kb.KB_ERR_BAD_SHAPE


def test_scratch_bytes_cover_the_prefill_mask_table(kb):
    """For prompt chunks the scratch a caller sizes with kb_flash_attn_ext_scratch_bytes holds the dense mask's class
    table (one byte per 128-query tile and 64-cell block, rounded up to 256 bytes), and for a quantised cache the two
    f16 views before it; the verify shape keeps its split partials."""
    D, H, H_kv = 256, 24, 4
    L = kb.lib()
    by = ctypes.byref
    prm = kb.fa_params(1 / 16)
    for n_q, n_kv in ((4096, 8192), (2048, 4096), (300, 1000)):
        q = kb.kb_tensor(1 << 20, kb.F32, [D, n_q, H, 1], [4, H * D * 4, D * 4, n_q * H * D * 4])
        table = -(-(-(-n_q // 128) * -(-n_kv // 64)) // 256) * 256
        k = kb.kb_tensor(1 << 20, kb.F16, [D, n_kv, H_kv, 1], [2, 2048, 512, 2048 * n_kv])
        assert L.kb_flash_attn_ext_scratch_bytes(by(q), by(k), by(k), by(prm)) >= table
        kq = kb.kb_tensor(1 << 20, kb.Q8_0, [D, n_kv, H_kv, 1], [34, 1088, 272, 1088 * n_kv])
        views = 2 * n_kv * H_kv * D * 2
        assert L.kb_flash_attn_ext_scratch_bytes(by(q), by(kq), by(kq), by(prm)) >= views + table
    q = kb.kb_tensor(1 << 20, kb.F32, [D, 4, H, 1], [4, H * D * 4, D * 4, 4 * H * D * 4])
    k = kb.kb_tensor(1 << 20, kb.F16, [D, 262144, H_kv, 1], [2, 2048, 512, 2048 * 262144])
    assert L.kb_flash_attn_ext_scratch_bytes(by(q), by(k), by(k), by(prm)) > 0


def test_gdn_step_validates(kb):
    """kb_gdn_step refuses malformed layers before touching the device; a well-formed one reaches the launch, which
    fails without a GPU."""
    import torch

    S, H_k, H_v, KC = 128, 16, 48, 4
    ch = 2 * S * H_k + S * H_v

    def layer(n=4, K=4, conv_w_width=KC, conv_rows=None, snap_dtype=torch.float16, snap_rows=None):
        return dict(qkv=torch.zeros(n, ch), conv_state=torch.zeros(K, conv_rows or (KC - 1) * ch),
                    conv_w=torch.zeros(ch, conv_w_width), beta_raw=torch.zeros(n, H_v), alpha=torch.zeros(n, H_v),
                    dt_bias=torch.zeros(H_v), a=torch.zeros(H_v), ssm=torch.zeros(H_v, S, S),
                    snap=torch.zeros(snap_rows if snap_rows is not None else K - 1, S * S * H_v, dtype=snap_dtype)
                    if K > 1 else None,
                    n_snapshots=K, z=torch.zeros(n, H_v * S), ssm_norm=torch.ones(S), rms_eps=1e-6,
                    sync=torch.zeros(H_k, dtype=torch.int32))

    def status(**kw):
        try:
            kb.gdn_step(**kw, stream=0)
        except kb.KbError as e:
            return e.status
        return kb.KB_OK

    assert status(**layer()) == kb.KB_ERR_CUDA  # well-formed: fails only at the launch
    assert status(**layer(n=1, K=1)) == kb.KB_ERR_CUDA
    assert status(**layer(n=5)) == kb.KB_ERR_UNSUPPORTED  # 1-4 tokens per launch
    assert status(**layer(conv_w_width=3)) == kb.KB_ERR_UNSUPPORTED  # conv kernel width 4 only
    assert status(**layer(conv_rows=3 * ch - 4)) == kb.KB_ERR_BAD_SHAPE
    assert status(**dict(layer(), n_snapshots=0)) == kb.KB_ERR_ARG
    assert status(**dict(layer(), snap=None)) == kb.KB_ERR_ARG  # 4 snapshots need the snapshot rows
    assert status(**layer(n=2, snap_rows=1)) == kb.KB_ERR_CUDA  # 2 tokens write slots 0 and 1 only
    assert status(**layer(snap_rows=2)) == kb.KB_ERR_BAD_SHAPE  # 4 tokens write 3 snapshot rows
    assert status(**layer(snap_dtype=torch.int32)) == kb.KB_ERR_UNSUPPORTED  # f32 / f16 / bf16 snapshots only
    odd = torch.zeros(4 * H_k + 4, dtype=torch.uint8)[1:]  # a counter array off its 4-byte alignment
    assert status(**dict(layer(), sync=odd)) == kb.KB_ERR_ARG
    bad_z = layer()
    bad_z["z"] = torch.zeros(4, H_v * S - 4)
    assert status(**bad_z) == kb.KB_ERR_BAD_SHAPE


def test_plain_c_caller(tmp_path):
    """tests/abi_check.c: the header compiles as C11 with warnings as errors, links against the library, and the
    calls' validation answers a C caller without a device."""
    import shutil
    import subprocess

    lib_dir = os.path.join(ROOT, "klein_b200")
    if not shutil.which("gcc") or not os.path.exists(os.path.join(lib_dir, "libklein_b200.so")):
        pytest.skip("gcc or the built library is missing")
    exe = str(tmp_path / "abi_check")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "abi_check.c"), "-L", lib_dir, "-lklein_b200",
                    "-Wl,-rpath," + lib_dir, "-o", exe], check=True)
    r = subprocess.run([exe], stdout=subprocess.PIPE, text=True, timeout=60)
    assert r.returncode == 0, r.stdout
    assert "abi_check: ok" in r.stdout
