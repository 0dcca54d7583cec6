"""GPU parity of the tcgen05 causal-prefill kernel (kb_flash_attn_ext with >= 128 query tokens over an f16 or
bf16 cache) against the exact f64 attention and, at moderate sizes, ggml's own CPU op."""
import numpy as np
import pytest

import oracle as O
from parity import check_attention

pytestmark = pytest.mark.gpu


def exact_np(q, kd, vd, mask, scale=1.0 / 16):
    n_q, H, D = q.shape
    G = H // kd.shape[1]
    out = np.zeros((n_q, H, D))
    for h in range(H):
        s = (q[:, h].astype(np.float64) @ kd[:, h // G].T.astype(np.float64)) * scale + mask
        m = s.max(1, keepdims=True)
        m = np.where(np.isfinite(m), m, 0.0)
        p = np.exp(s - m)
        l = p.sum(1, keepdims=True)
        out[:, h] = np.where(l > 0, (p @ vd[:, h // G].astype(np.float64)) / np.where(l > 0, l, 1.0), 0.0)
    return out


def run(kb, cuda, q, kc, vc, kv_type, H_kv, mask=None, **kw):
    import torch

    qt = torch.from_numpy(q).to(cuda)
    if kv_type == kb.BF16:
        kt = torch.from_numpy(kc).to(cuda).view(torch.bfloat16)
        vt = torch.from_numpy(vc).to(cuda).view(torch.bfloat16)
    else:
        kt, vt = torch.from_numpy(kc).to(cuda), torch.from_numpy(vc).to(cuda)
    mt = None if mask is None else torch.from_numpy(mask.astype(np.float16)).to(cuda)
    out = kb.flash_attn_ext(qt, kb.kv_cache_view(kt, kv_type, H_kv, 256), kb.kv_cache_view(vt, kv_type, H_kv, 256),
                            1 / 16, mask=mt, **kw)
    torch.cuda.synchronize()
    assert kb.device_error() == 0
    return out[0].cpu().numpy()


def case(kb, cuda, kvt, n_q, n_kv, pos0, H=24, H_kv=4, seed=0, dense=False, ggml=False):
    ggml_t = O.GGML_F16 if kvt == kb.F16 else O.GGML_BF16
    q, kc, vc, kd, vd = O.make_fa_inputs(seed + n_q + n_kv, n_q, n_kv, H=H, H_kv=H_kv, kv_type=ggml_t)
    mask = O.rs_visible_mask(n_q, n_kv, pos0)
    gpu = run(kb, cuda, q, kc, vc, kvt, H_kv, mask=mask if dense else None, causal=not dense, pos0=pos0)
    qr = O.q_round_f16(q) if kvt == kb.F16 else O.q_round_bf16(q)
    ref = None
    if ggml and O.ref_available():
        ref = O.ref_flash_attn_ext(q, kc, vc, ggml_t, H_kv, mask=mask.astype(np.float16), n_threads=8, use_ref=False)
    return check_attention(gpu, exact_np(qr, kd, vd, mask), ref)


@pytest.mark.parametrize("kvt_name", ["F16", "BF16"])
def test_prefill_one_tile(kb, cuda, kvt_name):
    case(kb, cuda, getattr(kb, kvt_name), 128, 128, 0, H=6, H_kv=1)


@pytest.mark.parametrize("kvt_name", ["F16", "BF16"])
def test_prefill_small_vs_ggml(kb, cuda, kvt_name):
    case(kb, cuda, getattr(kb, kvt_name), 256, 256, 0, ggml=True)


@pytest.mark.parametrize("n_q,n_kv,pos0", [(300, 300, 0), (256, 1256, 1000), (128, 4000, 3872), (640, 700, 60)])
def test_prefill_ragged_and_chunked(kb, cuda, n_q, n_kv, pos0):
    case(kb, cuda, kb.F16, n_q, n_kv, pos0)


def test_prefill_dense_mask_matches_analytic(kb, cuda):
    case(kb, cuda, kb.F16, 384, 512, 100, dense=True)


def test_prefill_config2_bf16_4096(kb, cuda):
    """config[2]: 4,096-token causal prefill, 24 Q / 4 KV heads, D 256, bf16 Q/K/V."""
    case(kb, cuda, kb.BF16, 4096, 4096, 0, seed=2)


@pytest.fixture
def pair_mode(monkeypatch):
    """The CTA-pair form of the prefill kernel (cta_group::2: two heads of a GQA group on one query tile, each CTA
    loading half of every K / V tile), selected per call by KB_PREFILL_PAIR=1."""
    monkeypatch.setenv("KB_PREFILL_PAIR", "1")


@pytest.mark.parametrize("kvt_name", ["F16", "BF16"])
@pytest.mark.parametrize("n_q,n_kv,pos0", [(128, 128, 0), (300, 300, 0), (256, 1256, 1000), (640, 700, 60)])
def test_prefill_pairs(kb, cuda, pair_mode, kvt_name, n_q, n_kv, pos0):
    case(kb, cuda, getattr(kb, kvt_name), n_q, n_kv, pos0, seed=11)


def test_prefill_pairs_dense_mask_and_config2(kb, cuda, pair_mode):
    case(kb, cuda, kb.F16, 256, 700, 444, dense=True)
    case(kb, cuda, kb.BF16, 4096, 4096, 0)


@pytest.mark.parametrize("kvt_name", ["F16", "BF16"])
def test_prefill_mask_classes(kb, cuda, kvt_name):
    """A dense mask whose 64-cell blocks are, per 128-query tile, all 0 (computed as unmasked), all -inf (the leading
    and trailing ones skipped, those in between computed), or mixed, plus finite nonzero values: every class of the
    mask classification against the exact f64 attention with the same mask."""
    kvt = getattr(kb, kvt_name)
    n_q, n_kv, H_kv = 384, 1000, 4
    ggml_t = O.GGML_F16 if kvt == kb.F16 else O.GGML_BF16
    q, kc, vc, kd, vd = O.make_fa_inputs(4242, n_q, n_kv, H_kv=H_kv, kv_type=ggml_t)
    rng = np.random.default_rng(7)
    mask = np.zeros((n_q, n_kv), dtype=np.float32)
    mask[:, :128] = -np.inf                      # hidden leading blocks (every tile)
    mask[:128, 640:] = -np.inf                   # hidden trailing blocks of the first tile
    mask[128:256, 320:384] = -np.inf             # a hidden block between visible ones
    mask[256:, 448:512] = rng.choice([0.0, -np.inf, -0.5], size=(128, 64))  # mixed values
    mask[:, 900:] = -rng.random((n_q, 100)).astype(np.float32)  # finite, nonzero
    mask = mask.astype(np.float16).astype(np.float32)
    gpu = run(kb, cuda, q, kc, vc, kvt, H_kv, mask=mask)
    qr = O.q_round_f16(q) if kvt == kb.F16 else O.q_round_bf16(q)
    check_attention(gpu, exact_np(qr, kd, vd, mask), None)
