"""klein_b200 — B200 (sm_100a) kernels for klein's qwen35 attention hot path.

The product is the C-ABI library ``libklein_b200.so`` declared in ``include/klein_b200.h``. This module
loads it with ctypes and offers thin torch-facing wrappers with the operator names and argument meaning
of the ggml nodes klein builds (``flash_attn_ext`` = ``ggml_flash_attn_ext``, ...), so tests and the
benchmark call exactly the entry points a patched ggml-cuda backend would call.

There is no fallback: when the library is missing, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int32, c_int64, c_size_t, c_uint64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libklein_b200.so")

# element types (numbered as enum ggml_type)
F32, F16, Q4_0, Q8_0, I32, I64, BF16 = 0, 1, 2, 8, 26, 27, 30
TYPE_SIZE = {F32: 4, F16: 2, I32: 4, I64: 8, BF16: 2}
Q8_0_BLOCK_BYTES = 34
Q4_0_BLOCK_BYTES = 18
BLOCK_BYTES = {Q8_0: Q8_0_BLOCK_BYTES, Q4_0: Q4_0_BLOCK_BYTES}

NOALLOC_SCRATCH_BYTES = 8 << 20  # KB_NOALLOC_SCRATCH_BYTES

KB_OK, KB_ERR_ARG, KB_ERR_BAD_SHAPE, KB_ERR_UNSUPPORTED, KB_ERR_SCRATCH, KB_ERR_CUDA, KB_ERR_TIMEOUT = range(7)
STATUS_NAMES = ["OK", "ERR_ARG", "ERR_BAD_SHAPE", "ERR_UNSUPPORTED", "ERR_SCRATCH", "ERR_CUDA", "ERR_TIMEOUT"]

# every symbol include/klein_b200.h declares (checked by tests/test_abi.py)
EXPORTED = [
    "kb_flash_attn_ext",
    "kb_flash_attn_ext_partial",
    "kb_lse_combine",
    "kb_gated_delta_net",
    "kb_gated_delta_net_cache",
    "kb_gated_delta_net_scratch_bytes",
    "kb_rollback_recurrent",
    "kb_set_rows",
    "kb_flash_attn_ext_scratch_bytes",
    "kb_flash_attn_ext_noalloc",
    "kb_device_error",
    "kb_version",
    "kb_peer_alloc",
    "kb_peer_open",
    "kb_peer_close",
    "kb_peer_free",
    "kb_partials_push",
    "kb_lse_combine_wait",
    "kb_attn_prologue",
    "kb_flash_attn_ext_gated",
    "kb_gdn_input",
    "kb_gdn_gated_norm",
    "kb_gdn_step_sync_bytes",
    "kb_gdn_step",
    "kb_flash_attn_ext_push",
    "kb_flash_attn_ext_push_scratch_bytes",
    "kb_flash_attn_ext_exchange",
    "kb_exchange_flag_bytes",
    "kb_flash_attn_ext_supported",
    "kb_state_sizes",
    "kb_state_create",
    "kb_state_required_bytes",
    "kb_state_create_in",
    "kb_state_destroy",
    "kb_state_device_bytes",
    "kb_state_get_layer",
    "kb_state_n_past",
    "kb_state_set_n_past",
    "kb_state_clear",
    "kb_state_rollback",
    "kb_plan_pass",
    "kb_state_plan_pass",
    "kb_state_accept",
    "kb_layer_attention_scratch_bytes",
    "kb_layer_attention",
    "kb_layer_deltanet_scratch_bytes",
    "kb_layer_deltanet",
]


class KbError(RuntimeError):
    def __init__(self, fn, status):
        super().__init__(f"{fn} returned {STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else status}")
        self.status = status


class KbTensor(ctypes.Structure):
    _fields_ = [("type", c_int32), ("ne", c_int64 * 4), ("nb", c_size_t * 4), ("data", c_void_p)]


class KbRopeParams(ctypes.Structure):
    """kb_rope_params: M-RoPE of ggml_rope_multi (mode 40 = IMROPE, 8 = MROPE)."""
    _fields_ = [("n_rot", c_int32), ("sections", c_int32 * 4), ("mode", c_int32), ("freq_base", ctypes.c_float),
                ("freq_scale", ctypes.c_float), ("attn_factor", ctypes.c_float)]


class KbFaParams(ctypes.Structure):
    _fields_ = [("scale", c_float), ("max_bias", c_float), ("logit_softcap", c_float), ("prec", c_int32),
                ("causal", c_int32), ("pos0", c_int64), ("kv_lo", c_int64), ("ring", c_int64)]


class KbQwen35Dims(ctypes.Structure):
    _fields_ = [("n_layer", c_int32), ("full_attn_interval", c_int32), ("n_head", c_int32), ("n_head_kv", c_int32),
                ("head_dim", c_int32), ("ssm_conv_kernel", c_int32), ("ssm_d_state", c_int32), ("ssm_n_group", c_int32),
                ("ssm_dt_rank", c_int32), ("with_mtp", c_int32)]


class KbStateConfig(ctypes.Structure):
    _fields_ = [("n_ctx", c_int32), ("type_k", c_int32), ("type_v", c_int32), ("n_snapshots", c_int32),
                ("snap_type", c_int32), ("mtp_window", c_int32)]


class KbStateLayer(ctypes.Structure):
    _fields_ = [("k", KbTensor), ("v", KbTensor), ("conv", KbTensor), ("ssm", KbTensor), ("ssm_snap", KbTensor)]


class KbPass(ctypes.Structure):
    _fields_ = [("n_tokens", c_int32), ("mtp", c_int32), ("cell0", c_int64), ("kv_lo", c_int64), ("ring", c_int64),
                ("n_kv", c_int64), ("fa", KbFaParams)]


def qwen35_dims(n_layer=64, with_mtp=1, full_attn_interval=4, n_head=24, n_head_kv=4, head_dim=256, conv_kernel=4,
                d_state=128, n_group=16, dt_rank=48) -> KbQwen35Dims:
    """qwen35 27B's attention shapes (model.h HParams; 64 decoder layers, every 4th full attention, 24 / 4 heads of
    256, DeltaNet 16 key / 48 value heads of 128, conv kernel 4) unless given otherwise."""
    return KbQwen35Dims(n_layer, full_attn_interval, n_head, n_head_kv, head_dim, conv_kernel, d_state, n_group, dt_rank,
                        with_mtp)


def state_config(n_ctx, type_k=None, type_v=None, n_snapshots=4, snap_type=None, mtp_window=16384) -> KbStateConfig:
    return KbStateConfig(n_ctx, Q8_0 if type_k is None else type_k, Q8_0 if type_v is None else type_v, n_snapshots,
                         F16 if snap_type is None else snap_type, mtp_window)


_lib = None


def lib():
    """The loaded C-ABI library; raises when it has not been built (there is no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m klein_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER
        L.kb_flash_attn_ext.restype = c_int32
        L.kb_flash_attn_ext.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams), P(KbTensor),
                                        c_void_p, c_size_t, c_void_p]
        L.kb_flash_attn_ext_partial.restype = c_int32
        L.kb_flash_attn_ext_partial.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams),
                                                P(KbTensor), c_void_p, c_void_p, c_size_t, c_void_p]
        L.kb_lse_combine.restype = c_int32
        L.kb_lse_combine.argtypes = [c_void_p, c_void_p, c_int64, c_int32, c_int64, c_int32, c_void_p, c_void_p]
        L.kb_flash_attn_ext_scratch_bytes.restype = c_size_t
        L.kb_flash_attn_ext_scratch_bytes.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams)]
        L.kb_flash_attn_ext_noalloc.restype = c_int32
        L.kb_flash_attn_ext_noalloc.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams),
                                                P(KbTensor), c_void_p]
        T4 = [P(KbTensor)] * 6
        L.kb_gated_delta_net.restype = c_int32
        L.kb_gated_delta_net.argtypes = T4 + [c_int32, P(KbTensor), c_void_p, c_size_t, c_void_p]
        L.kb_gated_delta_net_cache.restype = c_int32
        L.kb_gated_delta_net_cache.argtypes = T4 + [P(KbTensor), c_int32, P(KbTensor), c_void_p, c_size_t, c_void_p]
        L.kb_gated_delta_net_scratch_bytes.restype = c_size_t
        L.kb_gated_delta_net_scratch_bytes.argtypes = [P(KbTensor), P(KbTensor), c_int32]
        L.kb_rollback_recurrent.restype = c_int32
        L.kb_rollback_recurrent.argtypes = [c_int32, c_void_p, c_int64, c_void_p, c_int32, c_void_p, c_int64, c_int32,
                                            c_int32, c_void_p]
        L.kb_set_rows.restype = c_int32
        L.kb_set_rows.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), c_void_p]
        L.kb_flash_attn_ext_gated.restype = c_int32
        L.kb_flash_attn_ext_gated.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams),
                                              P(KbTensor), P(KbTensor), c_void_p, c_size_t, c_void_p]
        L.kb_flash_attn_ext_push.restype = c_int32
        L.kb_flash_attn_ext_push.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams), c_int64,
                                             c_void_p, c_int64, c_void_p, c_int32, c_int32, c_void_p, c_size_t, c_void_p]
        L.kb_flash_attn_ext_push_scratch_bytes.restype = c_size_t
        L.kb_flash_attn_ext_push_scratch_bytes.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams)]
        L.kb_flash_attn_ext_exchange.restype = c_int32
        L.kb_flash_attn_ext_exchange.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams),
                                                 P(KbTensor), c_int64, c_void_p, c_int64, c_void_p, c_int32, c_int32,
                                                 P(KbTensor), c_void_p, c_size_t, c_void_p]
        L.kb_flash_attn_ext_supported.restype = c_int32
        L.kb_flash_attn_ext_supported.argtypes = [P(KbTensor), P(KbTensor), P(KbTensor), P(KbTensor), P(KbFaParams)]
        L.kb_exchange_flag_bytes.restype = c_size_t
        L.kb_exchange_flag_bytes.argtypes = [c_int32]
        L.kb_state_sizes.restype = c_int32
        L.kb_state_sizes.argtypes = [P(KbQwen35Dims), P(KbStateConfig), P(c_size_t), P(c_size_t), P(c_size_t)]
        L.kb_state_create.restype = c_int32
        L.kb_state_create.argtypes = [P(KbQwen35Dims), P(KbStateConfig), P(c_void_p)]
        L.kb_state_required_bytes.restype = c_size_t
        L.kb_state_required_bytes.argtypes = [P(KbQwen35Dims), P(KbStateConfig)]
        L.kb_state_create_in.restype = c_int32
        L.kb_state_create_in.argtypes = [P(KbQwen35Dims), P(KbStateConfig), c_void_p, c_size_t, P(c_void_p)]
        L.kb_state_destroy.restype = c_int32
        L.kb_state_destroy.argtypes = [c_void_p]
        L.kb_state_device_bytes.restype = c_size_t
        L.kb_state_device_bytes.argtypes = [c_void_p]
        L.kb_state_get_layer.restype = c_int32
        L.kb_state_get_layer.argtypes = [c_void_p, c_int32, P(KbStateLayer)]
        L.kb_state_n_past.restype = c_int64
        L.kb_state_n_past.argtypes = [c_void_p, c_int32]
        L.kb_state_set_n_past.restype = c_int32
        L.kb_state_set_n_past.argtypes = [c_void_p, c_int32, c_int64]
        L.kb_state_clear.restype = c_int32
        L.kb_state_clear.argtypes = [c_void_p, c_void_p]
        L.kb_state_rollback.restype = c_int32
        L.kb_state_rollback.argtypes = [c_void_p, c_int32, c_void_p]
        L.kb_plan_pass.restype = c_int32
        L.kb_plan_pass.argtypes = [P(KbQwen35Dims), P(KbStateConfig), c_int32, c_int32, c_int64, c_int64, P(KbPass),
                                   c_void_p]
        L.kb_state_plan_pass.restype = c_int32
        L.kb_state_plan_pass.argtypes = [c_void_p, c_int32, c_int32, c_int64, P(KbPass), c_void_p]
        L.kb_state_accept.restype = c_int32
        L.kb_state_accept.argtypes = [c_void_p, c_int64, c_int32, c_int32, c_void_p]
        L.kb_layer_attention_scratch_bytes.restype = c_size_t
        L.kb_layer_attention_scratch_bytes.argtypes = [c_void_p, c_int32, P(KbPass)]
        L.kb_layer_attention.restype = c_int32
        L.kb_layer_attention.argtypes = [c_void_p, c_int32, P(KbPass)] + [P(KbTensor)] * 7 + \
            [ctypes.c_float, P(KbRopeParams), P(KbTensor), c_void_p, c_size_t, c_void_p]
        L.kb_layer_deltanet_scratch_bytes.restype = c_size_t
        L.kb_layer_deltanet_scratch_bytes.argtypes = [c_void_p, c_int32, c_int32]
        L.kb_layer_deltanet.restype = c_int32
        L.kb_layer_deltanet.argtypes = [c_void_p, c_int32, c_int32] + [P(KbTensor)] * 8 + \
            [ctypes.c_float, P(KbTensor), c_void_p, c_size_t, c_void_p]
        L.kb_gdn_input.restype = c_int32
        L.kb_gdn_input.argtypes = [P(KbTensor)] * 7 + [c_int32, c_int32, ctypes.c_float] + [P(KbTensor)] * 5 + [c_void_p]
        L.kb_gdn_gated_norm.restype = c_int32
        L.kb_gdn_gated_norm.argtypes = [P(KbTensor)] * 3 + [ctypes.c_float, P(KbTensor), c_void_p]
        L.kb_gdn_step_sync_bytes.restype = ctypes.c_size_t
        L.kb_gdn_step_sync_bytes.argtypes = [c_int32]
        L.kb_gdn_step.restype = c_int32
        L.kb_gdn_step.argtypes = [P(KbTensor)] * 9 + [c_int32] + [P(KbTensor)] * 2 + [ctypes.c_float, c_void_p,
                                                                                       P(KbTensor), c_void_p]
        L.kb_attn_prologue.restype = c_int32
        L.kb_attn_prologue.argtypes = [P(KbTensor)] * 7 + [ctypes.c_float, P(KbRopeParams)] + [P(KbTensor)] * 4 + [c_void_p]
        L.kb_device_error.restype = c_int32
        L.kb_device_error.argtypes = [P(c_int32), c_int32]
        L.kb_version.restype = ctypes.c_char_p
        L.kb_peer_alloc.restype = c_int32
        L.kb_peer_alloc.argtypes = [c_size_t, P(c_void_p), c_void_p]
        L.kb_peer_open.restype = c_int32
        L.kb_peer_open.argtypes = [c_void_p, P(c_void_p)]
        L.kb_peer_close.restype = c_int32
        L.kb_peer_close.argtypes = [c_void_p]
        L.kb_peer_free.restype = c_int32
        L.kb_peer_free.argtypes = [c_void_p]
        L.kb_partials_push.restype = c_int32
        L.kb_partials_push.argtypes = [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int32, c_int32, c_void_p]
        L.kb_lse_combine_wait.restype = c_int32
        L.kb_lse_combine_wait.argtypes = [c_void_p, c_int64, c_int64, c_int32, c_int64, c_int32, c_void_p, c_void_p,
                                          c_void_p]
        _lib = L
    return _lib


def check(fn: str, status: int) -> None:
    if status != KB_OK:
        raise KbError(fn, status)


# ------------------------------------------------------------------------------------------------ tensors

def kb_tensor(data_ptr: int, type_: int, ne, nb) -> KbTensor:
    """A kb_tensor from ggml-order extents ne[0..3] (innermost first) and byte strides nb[0..3]."""
    ne = list(ne) + [1] * (4 - len(ne))
    nb = list(nb)
    while len(nb) < 4:
        nb.append(nb[-1] * ne[len(nb) - 1])
    t = KbTensor()
    t.type = type_
    for i in range(4):
        t.ne[i] = int(ne[i])
        t.nb[i] = int(nb[i])
    t.data = data_ptr
    return t


def from_torch(x, type_: int | None = None) -> KbTensor:
    """kb_tensor view of a torch tensor (ggml order: reversed shape and strides)."""
    import torch

    if type_ is None:
        type_ = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int32: I32, torch.int64: I64}[x.dtype]
    es = x.element_size()
    ne = list(reversed(x.shape)) + [1] * (4 - x.dim())
    nb = [s * es for s in reversed(x.stride())]
    while len(nb) < 4:
        nb.append(nb[-1] * ne[len(nb) - 1] if nb else es)
    # a size-1 dimension gets ggml's packed stride (its stride is arbitrary in torch/numpy, e.g. 0 for None axes)
    for i in range(4):
        if ne[i] == 1:
            nb[i] = es if i == 0 else nb[i - 1] * ne[i - 1]
    return kb_tensor(x.data_ptr(), type_, ne, nb)


def kv_cache_view(cache, kv_type: int, n_head_kv: int, head_dim: int, n_kv: int | None = None) -> KbTensor:
    """klein's K or V view of a cache [n_ctx rows][n_head_kv * head_dim elements] (graph.cpp:114-117):
    ggml tensor [head_dim, n_kv, n_head_kv] with nb1 = row bytes, nb2 = one head's bytes."""
    rows = cache.shape[0] if n_kv is None else n_kv
    row_bytes = cache.stride(0) * cache.element_size()
    if kv_type in BLOCK_BYTES:
        head_bytes = head_dim // 32 * BLOCK_BYTES[kv_type]
        es = BLOCK_BYTES[kv_type]  # nb0 of a block-quantised tensor is the block size
    else:
        es = TYPE_SIZE[kv_type]
        head_bytes = head_dim * es
    return kb_tensor(cache.data_ptr(), kv_type, [head_dim, rows, n_head_kv, 1],
                     [es, row_bytes, head_bytes, row_bytes * cache.shape[0]])


# ------------------------------------------------------------------------------------------------ ops

def fa_params(scale: float, max_bias=0.0, softcap=0.0, causal=False, pos0=0, kv_lo=0, ring=0) -> KbFaParams:
    p = KbFaParams()
    p.scale, p.max_bias, p.logit_softcap, p.prec = scale, max_bias, softcap, 10
    p.causal, p.pos0, p.kv_lo, p.ring = int(causal), pos0, kv_lo, ring
    return p


def flash_attn_ext(q, k: KbTensor, v: KbTensor, scale: float, mask=None, max_bias=0.0, softcap=0.0, causal=False,
                   pos0=0, kv_lo=0, ring=0, out=None, stream=None, gate=None, scratch_bytes=None):
    """GGML_OP_FLASH_ATTN_EXT through kb_flash_attn_ext.

    q: torch f32 on the GPU, token-major [ne3][n_q][H][D] (or [n_q][H][D]); passed as klein's permuted
    view [D, n_q, H, ne3]. k, v: kb_tensor cache views (kv_cache_view). mask: torch f16 [n_q'][n_kv] or
    None. Returns f32 [ne3][n_q][H][D] (ggml's permuted result [D, H, n_q, ne3]). gate: torch f32 of the output's
    shape, or None; with a gate the result is o * sigmoid(gate) (kb_flash_attn_ext_gated). scratch_bytes: the
    scratch to pass (default: kb_flash_attn_ext_scratch_bytes).
    """
    import torch

    if q.dim() == 3:
        q = q.unsqueeze(0)
    ne3, n_q, H, D = q.shape
    es = 4
    qt = kb_tensor(q.data_ptr(), F32, [D, n_q, H, ne3],
                   [es, q.stride(1) * es, q.stride(2) * es, q.stride(0) * es])
    if out is None:
        out = torch.empty((ne3, n_q, H, D), dtype=torch.float32, device=q.device)
    dt = kb_tensor(out.data_ptr(), F32, [D, H, n_q, ne3], [4, D * 4, H * D * 4, n_q * H * D * 4])
    mt = None
    if mask is not None:
        m = mask if mask.dim() == 4 else mask.reshape((1, 1) + tuple(mask.shape[-2:]))
        mt = from_torch(m, F16)
    prm = fa_params(scale, max_bias, softcap, causal, pos0, kv_lo, ring)
    L = lib()
    nbytes = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qt), ctypes.byref(k), ctypes.byref(v), ctypes.byref(prm))
    if scratch_bytes is not None:
        nbytes = scratch_bytes
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    st = torch.cuda.current_stream(q.device).cuda_stream if stream is None else stream
    if gate is not None:
        g = gate if gate.dim() == 4 else gate.reshape((ne3, n_q, H, D))
        gt = from_torch(g)
        rc = L.kb_flash_attn_ext_gated(ctypes.byref(qt), ctypes.byref(k), ctypes.byref(v),
                                       ctypes.byref(mt) if mt is not None else None, ctypes.byref(prm), ctypes.byref(gt),
                                       ctypes.byref(dt), c_void_p(scratch.data_ptr()), c_size_t(nbytes), c_void_p(st))
        check("kb_flash_attn_ext_gated", rc)
    else:
        rc = L.kb_flash_attn_ext(ctypes.byref(qt), ctypes.byref(k), ctypes.byref(v),
                                 ctypes.byref(mt) if mt is not None else None, ctypes.byref(prm), ctypes.byref(dt),
                                 c_void_p(scratch.data_ptr()), c_size_t(nbytes), c_void_p(st))
        check("kb_flash_attn_ext", rc)
    out._kb_scratch = scratch  # keep alive until the stream has used it
    return out


def flash_attn_ext_partial(q, k: KbTensor, v: KbTensor, scale: float, part, causal=False, pos0=0, kv_lo=0, ring=0,
                           stream=None):
    """kb_flash_attn_ext_partial into `part`, a flat f32 torch tensor of kv_split.packed_part_floats(n_q*H, D):
    the unnormalised output rows [n_q*H][D] followed by (m, l) per row. q as for flash_attn_ext (ne3 = 1)."""
    import torch

    if q.dim() == 3:
        q = q.unsqueeze(0)
    _, n_q, H, D = q.shape
    qt = kb_tensor(q.data_ptr(), F32, [D, n_q, H, 1], [4, q.stride(1) * 4, q.stride(2) * 4, q.stride(0) * 4])
    pt = kb_tensor(part.data_ptr(), F32, [D, H, n_q, 1], [4, D * 4, H * D * 4, n_q * H * D * 4])
    prm = fa_params(scale, causal=causal, pos0=pos0, kv_lo=kv_lo, ring=ring)
    L = lib()
    nbytes = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qt), ctypes.byref(k), ctypes.byref(v), ctypes.byref(prm))
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    st = torch.cuda.current_stream(q.device).cuda_stream if stream is None else stream
    rc = L.kb_flash_attn_ext_partial(ctypes.byref(qt), ctypes.byref(k), ctypes.byref(v), None, ctypes.byref(prm),
                                     ctypes.byref(pt), c_void_p(part.data_ptr() + n_q * H * D * 4),
                                     c_void_p(scratch.data_ptr()), c_size_t(nbytes), c_void_p(st))
    check("kb_flash_attn_ext_partial", rc)
    part._kb_scratch = scratch
    return part


def device_error(clear: bool = True) -> int:
    code = c_int32(0)
    check("kb_device_error", lib().kb_device_error(ctypes.byref(code), int(clear)))
    return code.value


def _stream(x, stream):
    import torch

    return torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream


def gdn_scratch(v, g, K: int, scratch=None):
    """(pointer, bytes) of DeltaNet scratch: `scratch` if given (a torch uint8 tensor, or False for none), else a
    new buffer of kb_gated_delta_net_scratch_bytes (none when the call does not use it)."""
    import torch

    if scratch is False:
        return None, 0
    if scratch is None:
        n = lib().kb_gated_delta_net_scratch_bytes(ctypes.byref(from_torch(v)), ctypes.byref(from_torch(g)), K)
        if n == 0:
            return None, 0
        scratch = torch.empty(n, dtype=torch.uint8, device=v.device)
    return scratch, scratch.numel()


def gated_delta_net(q, k, v, g, beta, state, K: int, scratch=None, stream=None):
    """GGML_OP_GATED_DELTA_NET through kb_gated_delta_net. Torch f32 tensors in ggml order reversed:
    q, k [n_seqs][T][H_k][S]; v [n_seqs][T][H_v][S]; g [n_seqs][T][H_v][1 or S]; beta [n_seqs][T][H_v][1];
    state [n_seqs][H_v][S][S]. Returns ggml's packed f32 result as a flat tensor. scratch: see gdn_scratch
    (False forces the recurrent kernel for every token)."""
    import torch

    n_seqs, T, H_v, S = v.shape
    n = S * H_v * T * n_seqs + K * S * S * H_v * n_seqs
    out = torch.empty(n, dtype=torch.float32, device=v.device)
    dt = kb_tensor(out.data_ptr(), F32, [S * H_v, T * n_seqs + K * S * n_seqs, 1, 1], [4, S * H_v * 4])
    args = [from_torch(x) for x in (q, k, v, g, beta.reshape(n_seqs, T, H_v, 1), state)]
    buf, nbytes = gdn_scratch(v, g, K, scratch)
    rc = lib().kb_gated_delta_net(*[ctypes.byref(a) for a in args], K, ctypes.byref(dt),
                                  c_void_p(buf.data_ptr() if buf is not None else None), nbytes,
                                  c_void_p(_stream(v, stream)))
    check("kb_gated_delta_net", rc)
    return out


def gated_delta_net_cache(q, k, v, g, beta, state, snap, K: int, attn=None, scratch=None, stream=None):
    """klein's fused form through kb_gated_delta_net_cache: state (f32 [n_seqs][H_v][S][S]) is updated in place
    to slot 0; snap (f16/bf16/f32 [K-1][S*S*H_v*n_seqs] or None) receives slots 1..min(T,K)-1.
    Returns the attention output f32 [n_seqs][T][H_v][S]."""
    import torch

    n_seqs, T, H_v, S = v.shape
    if attn is None:
        attn = torch.empty(n_seqs, T, H_v, S, dtype=torch.float32, device=v.device)
    args = [from_torch(x) for x in (q, k, v, g, beta.reshape(n_seqs, T, H_v, 1), state)]
    st = from_torch(snap) if snap is not None else None
    at = from_torch(attn)
    buf, nbytes = gdn_scratch(v, g, K, scratch)
    rc = lib().kb_gated_delta_net_cache(*[ctypes.byref(a) for a in args], ctypes.byref(st) if st is not None else None, K,
                                        ctypes.byref(at), c_void_p(buf.data_ptr() if buf is not None else None), nbytes,
                                        c_void_p(_stream(v, stream)))
    check("kb_gated_delta_net_cache", rc)
    return attn


def set_rows(dst: KbTensor, src, idx, stream=None):
    """ggml_set_rows through kb_set_rows: src torch f32 [n_src][ne0] (or 4-d), idx torch i64/i32 [n_src]."""
    s4 = src if src.dim() == 4 else src.reshape((1,) * (4 - src.dim()) + tuple(src.shape))
    st = from_torch(s4)
    it = from_torch(idx)
    rc = lib().kb_set_rows(ctypes.byref(dst), ctypes.byref(st), ctypes.byref(it), c_void_p(_stream(src, stream)))
    check("kb_set_rows", rc)


def attn_prologue(qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm, rms_eps: float, n_rot: int, sections, mode: int,
                  freq_base: float, k_cache: KbTensor, v_cache: KbTensor, freq_scale: float = 1.0,
                  attn_factor: float = 1.0, stream=None):
    """klein's attention prologue (graph.cpp:94-112) through kb_attn_prologue. qfull torch f32 [n][nh * 2 hd], kcur /
    vcur f32 [n][nkv * hd], pos i32 [4 n], kv_idx i64 [n], q_norm / k_norm f32 [hd]; k_cache / v_cache: kb_tensor
    views [nkv * hd, n_cells] (cache_rows). Returns (q f32 [n][nh][hd], gate f32 [n][nh * hd])."""
    import torch

    hd = q_norm.shape[-1]
    n = qfull.shape[0]
    nh = qfull.shape[1] // (2 * hd)
    q = torch.empty((n, nh, hd), dtype=torch.float32, device=qfull.device)
    gate = torch.empty((n, nh * hd), dtype=torch.float32, device=qfull.device)
    rp = KbRopeParams(n_rot, (c_int32 * 4)(*sections), mode, freq_base, freq_scale, attn_factor)
    ts = [from_torch(x) for x in (qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm)]
    rc = lib().kb_attn_prologue(*[ctypes.byref(t) for t in ts], ctypes.c_float(rms_eps), ctypes.byref(rp),
                                ctypes.byref(from_torch(q)), ctypes.byref(from_torch(gate)), ctypes.byref(k_cache),
                                ctypes.byref(v_cache), c_void_p(_stream(qfull, stream)))
    check("kb_attn_prologue", rc)
    return q, gate


def gdn_input(qkv, conv_state, conv_w, S: int, H_k: int, rms_eps: float, beta_raw=None, alpha=None, dt_bias=None,
              a=None, stream=None):
    """klein's DeltaNet input side (graph.cpp:136-165) through kb_gdn_input. qkv torch f32 [n][ch], conv_state
    f32 [K][(kc - 1) ch] (updated in place), conv_w f32 [ch][kc]; beta_raw / alpha f32 [n][H_v] and dt_bias / a
    f32 [H_v] optional. Returns (q [n][H_k][S], k [n][H_k][S], v [n][H_v][S], beta [n][H_v] | None, g | None)."""
    import torch

    n, ch = qkv.shape
    H_v = (ch - 2 * S * H_k) // S
    dev = qkv.device
    q = torch.empty((n, H_k, S), dtype=torch.float32, device=dev)
    k = torch.empty_like(q)
    v = torch.empty((n, H_v, S), dtype=torch.float32, device=dev)
    beta = g = None
    gate_args = [None, None, None, None]
    if beta_raw is not None:
        beta = torch.empty((n, H_v), dtype=torch.float32, device=dev)
        g = torch.empty_like(beta)
        gate_args = [ctypes.byref(from_torch(x)) for x in (beta_raw, alpha, dt_bias, a)]
    rc = lib().kb_gdn_input(ctypes.byref(from_torch(qkv)), ctypes.byref(from_torch(conv_state)),
                            ctypes.byref(from_torch(conv_w)), *gate_args, S, H_k, ctypes.c_float(rms_eps),
                            ctypes.byref(from_torch(q)), ctypes.byref(from_torch(k)), ctypes.byref(from_torch(v)),
                            ctypes.byref(from_torch(beta)) if beta is not None else None,
                            ctypes.byref(from_torch(g)) if g is not None else None, c_void_p(_stream(qkv, stream)))
    check("kb_gdn_input", rc)
    return q, k, v, beta, g


def gdn_gated_norm(x, z, w, rms_eps: float, stream=None):
    """klein's DeltaNet output norm (graph.cpp:186-190) through kb_gdn_gated_norm: rms_norm(x) * w * silu(z)."""
    import torch

    dst = torch.empty_like(x)
    rc = lib().kb_gdn_gated_norm(ctypes.byref(from_torch(x)), ctypes.byref(from_torch(z.reshape(x.shape))),
                                 ctypes.byref(from_torch(w)), ctypes.c_float(rms_eps), ctypes.byref(from_torch(dst)),
                                 c_void_p(_stream(x, stream)))
    check("kb_gdn_gated_norm", rc)
    return dst


def gdn_step(qkv, conv_state, conv_w, beta_raw, alpha, dt_bias, a, ssm, snap, n_snapshots: int, z, ssm_norm,
             rms_eps: float, sync, out=None, stream=None):
    """A whole DeltaNet layer of a decode / verify pass (1..4 tokens) in one launch through kb_gdn_step: the input
    side on conv_state (f32 [n_snapshots][3 ch], updated in place), the recurrence into ssm (f32, H_v S S values,
    slot 0 in place) and snap (f16 / bf16 / f32 [n_snapshots - 1][S S H_v] or None), and the gated norm with z
    (f32 [n][H_v S]). sync: torch int32 [H_k] of zeros on the device (left zero). Returns out f32 [n][H_v S]."""
    import torch

    n = qkv.shape[0]
    if out is None:
        out = torch.empty(z.shape, dtype=torch.float32, device=qkv.device)
    tensors = [from_torch(x) for x in (qkv, conv_state, conv_w, beta_raw, alpha, dt_bias, a)]
    ssm_t = from_torch(ssm.reshape(-1))
    snap_t = from_torch(snap.reshape(snap.shape[0], -1)) if snap is not None else None
    rc = lib().kb_gdn_step(*[ctypes.byref(t) for t in tensors], ctypes.byref(ssm_t),
                           ctypes.byref(snap_t) if snap_t is not None else None, n_snapshots,
                           ctypes.byref(from_torch(z.reshape(n, -1))), ctypes.byref(from_torch(ssm_norm)),
                           ctypes.c_float(rms_eps), c_void_p(sync.data_ptr()), ctypes.byref(from_torch(out.view(n, -1))),
                           c_void_p(_stream(qkv, stream)))
    check("kb_gdn_step", rc)
    return out


def cache_rows(cache, kv_type: int) -> KbTensor:
    """kb_tensor of a whole cache as ggml's 2-d rows tensor [row elements, n_cells] (the set_rows destination)."""
    row_bytes = cache.stride(0) * cache.element_size()
    if kv_type in BLOCK_BYTES:
        bb = BLOCK_BYTES[kv_type]
        return kb_tensor(cache.data_ptr(), kv_type, [row_bytes // bb * 32, cache.shape[0], 1, 1],
                         [bb, row_bytes, row_bytes * cache.shape[0], row_bytes * cache.shape[0]])
    es = TYPE_SIZE[kv_type]
    return kb_tensor(cache.data_ptr(), kv_type, [row_bytes // es, cache.shape[0], 1, 1],
                     [es, row_bytes, row_bytes * cache.shape[0], row_bytes * cache.shape[0]])


def rollback_recurrent(convs, snaps, ssms, snap_type: int, s: int, n_snapshots: int, stream=None):
    """State::rollback_recurrent through kb_rollback_recurrent; lists of torch tensors, one entry per layer."""
    n = len(convs)
    P = c_void_p * max(n, 1)
    conv_p = P(*[c.data_ptr() for c in convs])
    snap_p = P(*[x.data_ptr() for x in snaps])
    ssm_p = P(*[x.data_ptr() for x in ssms])
    rc = lib().kb_rollback_recurrent(n, conv_p, convs[0].shape[-1], snap_p, snap_type, ssm_p, ssms[0].numel(), s,
                                     n_snapshots, c_void_p(_stream(convs[0], stream)))
    check("kb_rollback_recurrent", rc)


# ------------------------------------------------------------------------------------------------ peers

IPC_HANDLE_BYTES = 64


def peer_alloc(nbytes: int):
    """(device pointer, 64-byte IPC handle) of a zeroed buffer other processes can map (kb_peer_alloc)."""
    ptr = c_void_p()
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    check("kb_peer_alloc", lib().kb_peer_alloc(nbytes, ctypes.byref(ptr), h))
    return ptr.value, h.raw


def peer_open(handle: bytes) -> int:
    ptr = c_void_p()
    check("kb_peer_open", lib().kb_peer_open(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(ptr)))
    return ptr.value


class PeerExchange:
    """The all-gather of split partials over NVLink (kb_partials_push + kb_lse_combine_wait) for one process per
    GPU. `exchange_handles(obj) -> list` gathers a picklable object from every rank (e.g. a gloo / NCCL process
    group's all_gather_object). part_floats: packed partial size (kv_split.packed_part_floats). The epochs live on
    the device, so exchange_and_combine can be captured in a CUDA graph."""

    def __init__(self, rank: int, n_ranks: int, part_floats: int, exchange_handles):
        self.rank, self.n, self.pf = rank, n_ranks, part_floats
        self.set_floats = n_ranks * part_floats
        self.gbuf, gh = peer_alloc(2 * self.set_floats * 4)  # two slot sets
        # flag words of both exchanges (push / wait: n_ranks + 2; in-kernel: kb_exchange_flag_bytes)
        self.fbuf, fh = peer_alloc(max(256, (n_ranks + 2) * 4, lib().kb_exchange_flag_bytes(n_ranks)))
        handles = exchange_handles((gh, fh))
        self.gather = [self.gbuf if r == rank else peer_open(handles[r][0]) for r in range(n_ranks)]
        self.flags = [self.fbuf if r == rank else peer_open(handles[r][1]) for r in range(n_ranks)]
        self._g = (c_void_p * n_ranks)(*self.gather)
        self._f = (c_void_p * n_ranks)(*self.flags)

    def exchange_and_combine(self, part_ptr: int, rows: int, head_dim: int, dst_ptr: int, stream: int) -> None:
        """Push this rank's packed partial to every rank, wait for all of them, merge into dst (rows x head_dim)."""
        L = lib()
        check("kb_partials_push", L.kb_partials_push(c_void_p(part_ptr), self.pf, self._g, self.set_floats, self._f,
                                                     self.rank, self.n, c_void_p(stream)))
        check("kb_lse_combine_wait", L.kb_lse_combine_wait(c_void_p(self.gbuf), self.pf, self.set_floats, self.n, rows,
                                                           head_dim, c_void_p(self.fbuf), c_void_p(dst_ptr),
                                                           c_void_p(stream)))

    def attend_and_combine(self, qt, k: KbTensor, v: KbTensor, prm, scratch_ptr: int, scratch_bytes: int, rows: int,
                           head_dim: int, dst_ptr: int, stream: int) -> None:
        """kb_flash_attn_ext_push (this rank's partial attention, its rows written straight into every rank's gather
        buffer) then kb_lse_combine_wait into dst: the whole sequence-split attention of one layer in two kernels of
        this library plus the attention's own. qt / prm: kb_tensor q and KbFaParams as for kb_flash_attn_ext."""
        L = lib()
        check("kb_flash_attn_ext_push", L.kb_flash_attn_ext_push(ctypes.byref(qt), ctypes.byref(k), ctypes.byref(v), None,
                                                                 ctypes.byref(prm), self.pf, self._g, self.set_floats,
                                                                 self._f, self.rank, self.n, c_void_p(scratch_ptr),
                                                                 c_size_t(scratch_bytes), c_void_p(stream)))
        check("kb_lse_combine_wait", L.kb_lse_combine_wait(c_void_p(self.gbuf), self.pf, self.set_floats, self.n, rows,
                                                           head_dim, c_void_p(self.fbuf), c_void_p(dst_ptr),
                                                           c_void_p(stream)))

    def attend_exchange(self, qt, k: KbTensor, v: KbTensor, prm, scratch_ptr: int, scratch_bytes: int, dt, stream: int,
                        gate=None) -> None:
        """kb_flash_attn_ext_exchange: this rank's partial attention, the exchange and the final merge into dt (a
        kb_tensor [D, H, n_q, 1]) in one launch. gate: a kb_tensor of dt's shape, or None."""
        L = lib()
        check("kb_flash_attn_ext_exchange",
              L.kb_flash_attn_ext_exchange(ctypes.byref(qt), ctypes.byref(k), ctypes.byref(v), None, ctypes.byref(prm),
                                           ctypes.byref(gate) if gate is not None else None, self.pf, self._g,
                                           self.set_floats, self._f, self.rank, self.n, ctypes.byref(dt),
                                           c_void_p(scratch_ptr), c_size_t(scratch_bytes), c_void_p(stream)))

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank has finished its last exchange)."""
        L = lib()
        for r in range(self.n):
            if r != self.rank:
                L.kb_peer_close(c_void_p(self.gather[r]))
                L.kb_peer_close(c_void_p(self.flags[r]))
        L.kb_peer_free(c_void_p(self.gbuf))
        L.kb_peer_free(c_void_p(self.fbuf))
