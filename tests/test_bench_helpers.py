"""CPU checks of bench.py's own helpers: the f64 checker of its sequence-split parity run against the oracle's
restatement, the host-CPU description behind cpu_baseline.cores, and the clock sampler without a GPU."""
import numpy as np

import bench
import oracle as O


def test_bench_exact_attention_matches_restatement():
    n_q, n_kv = 4, 700
    q, kc, vc, kd, vd = O.make_fa_inputs(42, n_q, n_kv)
    qr = O.q_round_f16(q)
    got = bench.exact_attention_f64(qr, kd, vd, n_kv - n_q)
    want = O.rs_flash_attn_f64(qr, kd, vd, mask=O.rs_visible_mask(n_q, n_kv, n_kv - n_q))
    assert np.abs(got - want).max() <= 1e-12 * np.abs(want).max()


def test_host_cpu_counts_physical_cores():
    physical, logical, model = bench.host_cpu()
    assert 1 <= physical <= logical
    assert isinstance(model, str) and model


def test_clock_sampler_without_gpu_reports_no_samples():
    with bench.ClockSampler(0) as clk:
        pass
    s = clk.summary()
    assert "reasons" in s


def test_every_committed_profile_traffic_line_parses():
    """bench.py reads `traffic_bytes:` from each profile summary it cites; a note after the number must not break it."""
    import glob
    import os

    for path in glob.glob(os.path.join(os.path.dirname(bench.__file__), "profiles", "*.md")):
        name = os.path.splitext(os.path.basename(path))[0]
        with open(path) as f:
            has = any(line.startswith("traffic_bytes:") for line in f)
        if has:
            v = bench.ncu_traffic(name)
            assert isinstance(v, int) and v > 0, name
