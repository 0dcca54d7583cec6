"""klein's per-sequence State in HBM and the layer compositions bound to it, through the C ABI (kb_state_*,
kb_plan_pass, kb_layer_attention, kb_layer_deltanet). The state lives in one torch uint8 buffer handed to
kb_state_create_in, so its tensors can also be read as torch views (tests, diagnostics)."""
from __future__ import annotations

import ctypes
from ctypes import c_int64, c_size_t, c_void_p

import numpy as np

from . import (F16, F32, KbPass, KbRopeParams, KbStateLayer, check, from_torch, lib, qwen35_dims,  # noqa: F401
               state_config)


class State:
    def __init__(self, dims, cfg, device):
        import torch

        L = lib()
        self.dims, self.cfg, self.device = dims, cfg, device
        n = L.kb_state_required_bytes(ctypes.byref(dims), ctypes.byref(cfg))
        if n == 0:
            raise ValueError("kb_state_required_bytes rejected the shapes")
        self.buf = torch.empty(n, dtype=torch.uint8, device=device)
        self.h = c_void_p()
        check("kb_state_create_in", L.kb_state_create_in(ctypes.byref(dims), ctypes.byref(cfg), c_void_p(self.buf.data_ptr()),
                                                         c_size_t(n), ctypes.byref(self.h)))

    def close(self):
        if self.h:
            lib().kb_state_destroy(self.h)
            self.h = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------------------------------- tensors
    def layer(self, il: int) -> KbStateLayer:
        out = KbStateLayer()
        check("kb_state_get_layer", lib().kb_state_get_layer(self.h, il, ctypes.byref(out)))
        return out

    def view(self, t) -> "torch.Tensor":  # noqa: F821
        """A 2-d uint8 torch view [ne1][row bytes] of a state tensor."""
        off = t.data - self.buf.data_ptr()
        rows, row = t.ne[1], t.nb[1]
        return self.buf[off:off + rows * row].view(rows, row)

    @property
    def n_past(self) -> int:
        return lib().kb_state_n_past(self.h, 0)

    @n_past.setter
    def n_past(self, n: int):
        check("kb_state_set_n_past", lib().kb_state_set_n_past(self.h, 0, n))

    # ------------------------------------------------------------------------------------------- passes
    def plan(self, n_tokens: int, kv_lo: int = 0, mtp: bool = False, cell0: int | None = None):
        """(KbPass, kv_idx int64 numpy) of a pass of n_tokens from the state's n_past (or from cell0)."""
        p = KbPass()
        idx = np.zeros(n_tokens, dtype=np.int64)
        L = lib()
        if cell0 is None:
            rc = L.kb_state_plan_pass(self.h, int(mtp), n_tokens, kv_lo, ctypes.byref(p), c_void_p(idx.ctypes.data))
        else:
            rc = L.kb_plan_pass(ctypes.byref(self.dims), ctypes.byref(self.cfg), int(mtp), n_tokens, cell0, kv_lo,
                                ctypes.byref(p), c_void_p(idx.ctypes.data))
        check("kb_plan_pass", rc)
        return p, idx

    def accept(self, base: int, n_batch: int, accepted: int, stream: int = 0):
        check("kb_state_accept", lib().kb_state_accept(self.h, base, n_batch, accepted, c_void_p(stream)))

    def rollback(self, s: int, stream: int = 0):
        check("kb_state_rollback", lib().kb_state_rollback(self.h, s, c_void_p(stream)))

    def clear(self, stream: int = 0):
        check("kb_state_clear", lib().kb_state_clear(self.h, c_void_p(stream)))

    # ------------------------------------------------------------------------------------------- layers
    def attention_scratch_bytes(self, il: int, p) -> int:
        return lib().kb_layer_attention_scratch_bytes(self.h, il, ctypes.byref(p))

    def attention(self, il, p, qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm, eps, rope: KbRopeParams, out, scratch,
                  stream: int):
        """kb_layer_attention; tensors are torch tensors (qfull [n][2 hd nh], kcur / vcur [n][hd nkv], pos i32 [4 n],
        kv_idx i64 [n], norms [hd], out [n][hd nh]); scratch a torch uint8 tensor."""
        T = [from_torch(x) for x in (qfull, kcur, vcur, pos, kv_idx, q_norm, k_norm)]
        o = from_torch(out)
        check("kb_layer_attention",
              lib().kb_layer_attention(self.h, il, ctypes.byref(p), *[ctypes.byref(t) for t in T], ctypes.c_float(eps),
                                       ctypes.byref(rope), ctypes.byref(o), c_void_p(scratch.data_ptr()),
                                       c_size_t(scratch.numel()), c_void_p(stream)))

    def deltanet_scratch_bytes(self, il: int, n_tokens: int) -> int:
        return lib().kb_layer_deltanet_scratch_bytes(self.h, il, n_tokens)

    def deltanet(self, il, n, qkv, z, beta_raw, alpha, dt_bias, a, conv_w, ssm_norm, eps, out, scratch, stream: int):
        """kb_layer_deltanet; qkv [n][ch], z [n][S Hv], beta_raw / alpha [n][Hv], dt_bias / a [Hv], conv_w [ch][kc],
        ssm_norm [S], out [n][S Hv] (torch f32)."""
        T = [from_torch(x) for x in (qkv, z, beta_raw, alpha, dt_bias, a, conv_w, ssm_norm)]
        o = from_torch(out)
        check("kb_layer_deltanet",
              lib().kb_layer_deltanet(self.h, il, n, *[ctypes.byref(t) for t in T], ctypes.c_float(eps), ctypes.byref(o),
                                      c_void_p(scratch.data_ptr()), c_size_t(scratch.numel()), c_void_p(stream)))
