"""The DeltaNet input side (kb_gdn_input: conv, SiLU, L2 norms, gates, conv-state snapshots) and output norm
(kb_gdn_gated_norm) against the reference's own ggml graph for them (graph.cpp:136-165, 186-190)."""
import os
import sys

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLD)
from make_golden import make_gdn_io_inputs  # noqa: E402

ref_only = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@ref_only
@pytest.mark.parametrize("n,offset", [(1, 0), (2, 0), (4, 0), (37, 0), (4, 1), (37, 1)])
def test_gdn_input_matches_reference(kb, cuda, n, offset):
    """16-byte aligned buffers take the vector-access kernel; qkv offset by one float takes the strided one."""
    import torch

    qkv, cs, w, br, al, dt, a = make_gdn_io_inputs(50 + n, n)
    cs_ref = cs.copy()
    ref = O.ref_gdn_input(qkv, cs_ref, w, br, al, dt, a, 128, 16, 1e-6)

    def t(x, off=0):
        buf = torch.zeros(x.size + off, dtype=torch.float32, device=cuda)
        buf[off:] = torch.from_numpy(np.ascontiguousarray(x).reshape(-1)).to(cuda)
        return buf[off:].view(x.shape)

    cs_gpu = t(cs)
    qkv_gpu = t(qkv, offset)
    q, k, v, beta, g = kb.gdn_input(qkv_gpu, cs_gpu, t(w), 128, 16, 1e-6, beta_raw=t(br), alpha=t(al), dt_bias=t(dt),
                                    a=t(a))
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    for x, y in zip((q, k, v, beta, g), ref):
        x = x.cpu().numpy()
        # float32 on both sides; expf / logf and the conv's multiply-adds differ by ulps
        assert np.abs(x - y).max() <= 2e-6 * np.abs(y).max()
    # the snapshot slots are copies of stored inputs: bit-exact, untouched slots keep their old contents
    assert np.array_equal(cs_gpu.cpu().numpy(), cs_ref)


@ref_only
@pytest.mark.parametrize("n,H,S,offset", [(6, 48, 128, 0), (5, 3, 128, 0), (7, 5, 64, 0), (5, 3, 128, 1), (4, 6, 64, 1)])
def test_gdn_gated_norm_matches_reference(kb, cuda, n, H, S, offset):
    """Rows of 16-byte aligned buffers take the vectorised kernel (2 rows per warp: odd row counts leave a warp
    with one row); buffers offset by one float take the one-row-per-warp kernel."""
    import torch

    rng = np.random.default_rng(9 + n + S)
    x = rng.standard_normal((n, H, S)).astype(np.float32)
    z = rng.standard_normal((n, H, S)).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(S)).astype(np.float32)
    ref = O.ref_gdn_gated_norm(x, z, w, 1e-6)

    def dev(a):
        buf = torch.zeros(a.size + offset, dtype=torch.float32, device=cuda)
        buf[offset:] = torch.from_numpy(a.reshape(-1)).to(cuda)
        return buf[offset:].view(a.shape)

    out = kb.gdn_gated_norm(dev(x), dev(z), dev(w), 1e-6)
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - ref).max() <= 2e-6 * np.abs(ref).max()


def test_gdn_io_golden_fixture_s64(kb, cuda):
    """The committed reference outputs (S 64, 2 key / 4 value heads, 3 tokens): the input side and the gated norm."""
    import torch

    g = dict(np.load(os.path.join(GOLD, "gdn_io.npz")))
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
    cs = t(g["conv_state"])
    q, k, v, beta, gg = kb.gdn_input(t(g["qkv"]), cs, t(g["conv_w"]), 64, 2, 1e-6, beta_raw=t(g["beta_raw"]),
                                     alpha=t(g["alpha"]), dt_bias=t(g["dt_bias"]), a=t(g["a"]))
    o = kb.gdn_gated_norm(t(g["x"]), t(g["z"]), t(g["norm_w"]), 1e-6)
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    for x, name in ((q, "q"), (k, "k"), (v, "v"), (beta, "beta"), (gg, "g"), (o, "o")):
        y = g[name]
        assert np.abs(x.cpu().numpy().reshape(y.shape) - y).max() <= 2e-6 * np.abs(y).max(), name
    assert np.array_equal(cs.cpu().numpy(), g["conv_state_out"])
