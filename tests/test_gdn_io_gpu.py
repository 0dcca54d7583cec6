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
@pytest.mark.parametrize("n", [1, 2, 4, 37])
def test_gdn_input_matches_reference(kb, cuda, n):
    import torch

    qkv, cs, w, br, al, dt, a = make_gdn_io_inputs(50 + n, n)
    cs_ref = cs.copy()
    ref = O.ref_gdn_input(qkv, cs_ref, w, br, al, dt, a, 128, 16, 1e-6)
    t = lambda x: torch.from_numpy(x).to(cuda)
    cs_gpu = t(cs)
    q, k, v, beta, g = kb.gdn_input(t(qkv), cs_gpu, t(w), 128, 16, 1e-6, beta_raw=t(br), alpha=t(al), dt_bias=t(dt),
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
def test_gdn_gated_norm_matches_reference(kb, cuda):
    import torch

    rng = np.random.default_rng(9)
    x = rng.standard_normal((6, 48, 128)).astype(np.float32)
    z = rng.standard_normal((6, 48, 128)).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    ref = O.ref_gdn_gated_norm(x, z, w, 1e-6)
    out = kb.gdn_gated_norm(torch.from_numpy(x).to(cuda), torch.from_numpy(z).to(cuda), torch.from_numpy(w).to(cuda), 1e-6)
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - ref).max() <= 2e-6 * np.abs(ref).max()
