#!/usr/bin/env python
"""Benchmark of klein's attention hot path on B200.

Headline (BASELINE.json metric "verify-step attention us/layer @262K KV"): the MTP verify step of
config[3] — 4 query tokens per layer, causal among the 4 new cells, over a 262,144-cell KV cache
(4 KV heads x 256, f16) in each of 16 full-attention layers. One step = the 16 layers. value = us per
layer of the whole job (max over ranks), lower is better. With --gpus N the KV sequence of every layer is
split into N contiguous ranges, one per rank (strong scaling); each rank computes unnormalised partials
(o, m, l) of its range, and the attention kernel itself exchanges them over NVLink and merges them with a
log-sum-exp combine (one launch per layer and rank).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

--impl reference times the reference's own ggml CPU implementation of the same op (oracle/_ref, built
from the reference sources) on the host cores, one layer per step, and prints the same JSON line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_KV = 262144
N_Q = 4
H, H_KV, D = 24, 4, 256
LAYERS = 16
SCALE = 1.0 / 16
METRIC = "verify-step attention us/layer @262K KV"
UNIT = "us/layer"


def kv_bytes_per_layer(n_kv: int, kv_type: str) -> int:
    row = {"f16": H_KV * D * 2, "q8_0": H_KV * D // 32 * 34, "q4_0": H_KV * D // 32 * 18}[kv_type]
    return 2 * n_kv * row


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def ncu_traffic(name: str):
    """dram bytes per launch recorded in a committed ncu summary (profiles/<name>.md, line 'traffic_bytes: N')."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes:"):
                    return int(float(line.split(":", 1)[1].split()[0]))  # the number; a note may follow it
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs. The sampler is started and its
    first sample awaited before the timed region begins (nvidia-smi takes ~0.5 s to start), then it samples
    every 20 ms until the region ends."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def _reader(self):
        for line in self.proc.stdout:
            if line.strip():
                self.lines.append(line)

    def __enter__(self):
        import threading

        # nvidia-smi numbers the GPUs physically; map this process's device through CUDA_VISIBLE_DEVICES
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = str(self.gpu)
        if vis:
            ids = [x.strip() for x in vis.split(",") if x.strip()]
            if self.gpu < len(ids):
                idx = ids[self.gpu]
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", idx, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._reader, daemon=True)
        self.thread.start()
        t_end = time.time() + 5.0
        while not self.lines and time.time() < t_end and self.proc.poll() is None:
            time.sleep(0.01)
        self.skip = len(self.lines)  # samples taken before the timed region
        return self

    def __exit__(self, *a):
        if self.proc is None:
            return
        time.sleep(0.05)  # one more sample at the end of the region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.thread.join(timeout=5)
        # keep the last pre-region sample too when the region was shorter than the sampling period
        self.lines = self.lines[max(0, getattr(self, "skip", 0) - 1):]

    def summary(self):
        rows = []
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 10:
                continue
            try:
                rows.append({"sm": float(f[1]), "max": float(f[2]), "util": float(f[4]), "hw": f[6], "hwt": f[7],
                             "swt": f[8], "pcap": f[9]})
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        load = [r for r in rows if r["util"] > 0] or rows
        reasons = set()
        for r in load:
            if r["hw"] == "Active":
                reasons.add("hw_slowdown")
            if r["hwt"] == "Active":
                reasons.add("hw_thermal_slowdown")
            if r["swt"] == "Active":
                reasons.add("sw_thermal_slowdown")
            if r["pcap"] == "Active":
                reasons.add("sw_power_cap")
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["max"] for r in load),
                "reasons": sorted(reasons), "samples": len(load)}


# ------------------------------------------------------------------------------------------------ CPU arm

def host_cpu():
    """(physical cores, logical CPUs, model name) of this host from /proc/cpuinfo."""
    logical = os.cpu_count() or 1
    model, cores, phys, core = None, set(), None, None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                k, _, v = line.partition(":")
                k, v = k.strip(), v.strip()
                if k == "model name" and model is None:
                    model = v
                elif k == "physical id":
                    phys = v
                elif k == "core id":
                    core = v
                elif not k and phys is not None and core is not None:
                    cores.add((phys, core))
                    phys = core = None
        if phys is not None and core is not None:
            cores.add((phys, core))
    except OSError:
        pass
    try:
        avail = len(os.sched_getaffinity(0))
    except AttributeError:
        avail = logical
    physical = len(cores) if cores else logical
    return min(physical, avail), logical, model or "unknown"


def cpu_verify_sample(kv_type: str, threads: int, budget_s: float, min_reps: int = 2):
    """Times ggml's CPU flash attention (the reference build in oracle/_ref) on one layer of the headline
    workload: 4 tokens over 262,144 cells. Returns (us per layer, reps)."""
    import numpy as np

    import oracle as O

    rng = np.random.default_rng(7)
    q = rng.standard_normal((N_Q, H, D), dtype=np.float32)
    if kv_type == "f16":
        kc = rng.standard_normal((N_KV, H_KV * D), dtype=np.float32).astype(np.float16)
        vc = rng.standard_normal((N_KV, H_KV * D), dtype=np.float32).astype(np.float16)
        t = O.GGML_F16
    else:
        kc = O.rs_quantize_q8_0(rng.standard_normal((N_KV, H_KV * D), dtype=np.float32))
        vc = O.rs_quantize_q8_0(rng.standard_normal((N_KV, H_KV * D), dtype=np.float32))
        t = O.GGML_Q8_0
    mask = O.rs_visible_mask(N_Q, N_KV, N_KV - N_Q).astype(np.float16)
    O.ref_flash_attn_ext(q, kc, vc, t, H_KV, mask=mask, n_threads=threads, use_ref=False)  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < min_reps or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        O.ref_flash_attn_ext(q, kc, vc, t, H_KV, mask=mask, n_threads=threads, use_ref=False)
        times.append(time.perf_counter() - t0)
    return statistics.median(times) * 1e6, len(times)


def run_reference(args, rank: int):
    """--impl reference: the reference's ggml CPU op on the host cores, one layer per step."""
    if rank != 0:
        return
    import oracle as O

    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built (reference tree absent at build time)"}))
        return
    import numpy as np

    threads, logical, model = host_cpu()  # ggml's CPU backend on every physical core
    rng = np.random.default_rng(7)
    q = rng.standard_normal((N_Q, H, D), dtype=np.float32)
    kc = rng.standard_normal((N_KV, H_KV * D), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((N_KV, H_KV * D), dtype=np.float32).astype(np.float16)
    mask = O.rs_visible_mask(N_Q, N_KV, N_KV - N_Q).astype(np.float16)
    for _ in range(args.warmup):
        O.ref_flash_attn_ext(q, kc, vc, O.GGML_F16, H_KV, mask=mask, n_threads=threads, use_ref=False)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.ref_flash_attn_ext(q, kc, vc, O.GGML_F16, H_KV, mask=mask, n_threads=threads, use_ref=False)
    dt = time.perf_counter() - t0
    us = dt * 1e6 / args.steps
    line = {
        "impl": "reference", "metric": METRIC, "value": round(us, 2), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "config[3] long verify, one layer per step: 4 tokens, causal among the last 4, "
                               "262144-cell f16 KV cache, 24 Q / 4 KV heads, D 256 (ggml CPU flash_attn_ext)",
                   "n_kv": N_KV, "kv_type": "f16", "layers_per_step": 1},
        "cpu_baseline": {"value": round(us, 2), "unit": UNIT, "cores": threads, "kind": "reference",
                         "logical_cpus": logical, "cpu_model": model,
                         "sample": f"{args.steps} layers of the headline workload on ggml's CPU backend, "
                                   f"{threads} threads (one per physical core)"},
        "e2e": {"value": round(us, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ GPU arm

def quantize_q8_0_rows(torch, x):
    """Device-side q8_0 quantisation of f32 rows [n, k] (k % 32 == 0) with quantize_row_q8_0_ref's rule
    (d = amax/127 stored as f16, q = round(x / d)); builds the synthetic q8_0 caches of the benchmark."""
    n, k = x.shape
    blk = x.view(n, k // 32, 32)
    d = blk.abs().amax(-1) / 127.0
    inv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    qv = torch.round(blk * inv.unsqueeze(-1)).clamp(-127, 127).to(torch.int8)
    out = torch.empty(n, k // 32, 34, dtype=torch.uint8, device=x.device)
    out[:, :, :2] = d.to(torch.float16).view(torch.uint8).view(n, k // 32, 2)
    out[:, :, 2:] = qv.view(torch.uint8)
    return out.view(n, k // 32 * 34)


def quantize_q4_0_rows(torch, x):
    """Device-side q4_0 quantisation of f32 rows [n, k] with quantize_row_q4_0_ref's rule (max = the first value of
    largest magnitude, d = max / -8 stored as f16, q = min(15, trunc(x / d + 8.5)), byte j = q_j | q_{j+16} << 4);
    builds the synthetic q4_0 caches of the benchmark."""
    n, k = x.shape
    blk = x.view(n, k // 32, 32)
    mx = torch.gather(blk, -1, blk.abs().argmax(-1, keepdim=True)).squeeze(-1)
    d = mx / -8.0
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    qv = torch.clamp(torch.trunc(blk * inv.unsqueeze(-1) + 8.5), max=15).to(torch.uint8)
    out = torch.empty(n, k // 32, 18, dtype=torch.uint8, device=x.device)
    out[:, :, :2] = d.to(torch.float16).view(torch.uint8).view(n, k // 32, 2)
    out[:, :, 2:] = qv[:, :, :16] | (qv[:, :, 16:] << 4)
    return out.view(n, k // 32 * 18)


def bench_prefill(kb, torch, dev, steps, warmup, kv="bf16", T=4096, n_kv=4096):
    """Causal prefill through kb_flash_attn_ext (tcgen05 kernel): T new tokens at positions [n_kv - T, n_kv) over an
    n_kv-cell cache, 24 Q / 4 KV heads, D 256. bf16 Q/K/V: config[2] (T = n_kv = 4,096). q8_0: klein's 2,048-token
    prompt chunk over the 4,096-cell cache it has just written, the call widening the visible cells to f16 in its
    scratch first (timed as part of the call). Two independent input sets alternate so inputs exceed L2."""
    import ctypes

    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    sets = []
    for _ in range(2):
        q = torch.randn(1, T, H, D, device=dev, generator=gen)
        kf = torch.randn(n_kv, H_KV * D, device=dev, generator=gen)
        vf = torch.randn(n_kv, H_KV * D, device=dev, generator=gen)
        if kv == "bf16":
            q = q.bfloat16().float()
            k, v, t = kf.bfloat16(), vf.bfloat16(), kb.BF16
        else:
            k, v, t = quantize_q8_0_rows(torch, kf), quantize_q8_0_rows(torch, vf), kb.Q8_0
        sets.append((q, k, v, kb.kv_cache_view(k, t, H_KV, D), kb.kv_cache_view(v, t, H_KV, D)))
    pos0 = n_kv - T
    out = torch.empty(1, T, H, D, device=dev)
    L = kb.lib()
    q0 = sets[0][0]
    qt = kb.kb_tensor(q0.data_ptr(), kb.F32, [D, T, H, 1], [4, H * D * 4, D * 4, T * H * D * 4])
    prm = kb.fa_params(SCALE, causal=True, pos0=pos0)
    need = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qt), ctypes.byref(sets[0][3]), ctypes.byref(sets[0][4]),
                                             ctypes.byref(prm))
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    dt = kb.kb_tensor(out.data_ptr(), kb.F32, [D, H, T, 1], [4, D * 4, H * D * 4, T * H * D * 4])
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def call(i):
        q, _, _, kv_, vv_ = sets[i % 2]
        qt.data = q.data_ptr()
        rc = L.kb_flash_attn_ext(ctypes.byref(qt), ctypes.byref(kv_), ctypes.byref(vv_), None, ctypes.byref(prm),
                                 ctypes.byref(dt), ctypes.c_void_p(scratch.data_ptr()), ctypes.c_size_t(need), st)
        if rc != 0:
            raise kb.KbError("kb_flash_attn_ext", rc)

    for i in range(warmup):
        call(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        call(i)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    pairs = T * pos0 + T * (T + 1) // 2  # (query, visible cell) pairs
    flops = 4.0 * D * H * pairs  # QK^T and PV over the causal pairs only
    tf = flops / (us * 1e-6) / 1e12
    pk, kind = measured_peaks()
    name = "fa_prefill_bf16_4096" if kv == "bf16" else f"fa_prefill_{kv}_{T}"
    wl = (f"config[2] causal prefill, {T} tokens, 24 Q / 4 KV heads, D 256, bf16" if kv == "bf16" else
          f"prompt chunk: {T} new tokens over a {n_kv}-cell {kv} cache (widened to f16 in the call), 24 Q / 4 KV "
          f"heads, D 256")
    return {"value": round(tf, 1), "unit": "TFLOP/s", "us_per_layer": round(us, 2), "kv_type": kv, "workload": wl,
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(tf / pk["bf16_tflops"], 4), "peak_kind": kind + " burst",
                         "frac_of_sustained": round(tf / pk.get("bf16_tflops_sustained", pk["bf16_tflops"]), 4),
                         "algorithmic_flops_per_launch": flops, "traffic": ncu_traffic(name)}}


def bench_gdn(kb, torch, dev, steps, warmup):
    """config[1]: gated DeltaNet 4-token verify step with K = 4 snapshots (48 value / 16 key heads, d 128), in
    klein's cache form (state updated in place, f16 snapshots), over 48 layers so the states exceed L2."""
    L_, T, K, S, Hv, Hk = 48, 4, 4, 128, 48, 16
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    q = torch.nn.functional.normalize(torch.randn(1, T, Hk, S, device=dev, generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(1, T, Hk, S, device=dev, generator=gen), dim=-1)
    v = torch.randn(1, T, Hv, S, device=dev, generator=gen)
    g = -torch.nn.functional.softplus(torch.randn(1, T, Hv, 1, device=dev, generator=gen))
    beta = torch.sigmoid(torch.randn(1, T, Hv, 1, device=dev, generator=gen))
    states = [torch.randn(1, Hv, S, S, device=dev, generator=gen) * 0.02 for _ in range(L_)]
    snaps = [torch.zeros(K - 1, S * S * Hv, dtype=torch.float16, device=dev) for _ in range(L_)]
    attn = torch.empty(1, T, Hv, S, device=dev)
    import ctypes

    L = kb.lib()
    ins = [kb.from_torch(x) for x in (q, k, v, g, beta)]
    outs = [(kb.from_torch(states[l]), kb.from_torch(snaps[l])) for l in range(L_)]
    at = kb.from_torch(attn)

    def step(stream):
        for l in range(L_):
            rc = L.kb_gated_delta_net_cache(*[ctypes.byref(x) for x in ins], ctypes.byref(outs[l][0]),
                                            ctypes.byref(outs[l][1]), K, ctypes.byref(at), None, 0,
                                            ctypes.c_void_p(stream))
            if rc != 0:
                raise kb.KbError("kb_gated_delta_net_cache", rc)

    # the 48-layer step as one CUDA graph (klein's ggml-cuda backend replays its step graphs the same way)
    side = torch.cuda.Stream(dev)
    with torch.cuda.stream(side):
        step(side.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(torch.cuda.current_stream(dev).cuda_stream)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    us = e0.elapsed_time(e1) * 1e3 / (steps * L_)
    nbytes = S * S * Hv * 4 * 2 + (K - 1) * S * S * Hv * 2 + (2 * T * Hk * S + 2 * T * Hv * S + 2 * T * Hv) * 4
    gbs = nbytes / (us * 1e-6) / 1e9
    pk, _ = measured_peaks()
    return {"value": round(us, 2), "unit": "us/layer",
            "workload": "config[1] DeltaNet verify step: 4 tokens, K = 4 f16 snapshots, 48/16 heads, d 128",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / pk["hbm_gbs"], 4), "algorithmic_bytes_per_launch": nbytes,
                         "traffic": ncu_traffic("gdn_recurrent_verify")}}


def bench_gdn_layer(kb, torch, dev, steps, warmup):
    """A whole DeltaNet layer of the decode step (1 token) and the 4-token verify step between its GEMMs — conv input
    side, recurrence with K = 4 f16 snapshots in klein's cache form, gated norm — as kb_gdn_step's single launch and
    as the three calls it replaces (kb_gdn_input, kb_gated_delta_net_cache, kb_gdn_gated_norm), each over 48 layers
    with their own states in one CUDA graph (the states, 151 MB, exceed L2)."""
    L_, K, S, Hv, Hk = 48, 4, 128, 48, 16
    ch = 2 * S * Hk + S * Hv
    gen = torch.Generator(device=dev)
    gen.manual_seed(9)
    pk, _ = measured_peaks()
    conv_w = torch.randn(ch, 4, device=dev, generator=gen) * 0.5
    dt, aa = torch.randn(Hv, device=dev, generator=gen), -torch.rand(Hv, device=dev, generator=gen) - 0.1
    nw = 1 + 0.1 * torch.randn(S, device=dev, generator=gen)
    convs = [torch.randn(K, 3 * ch, device=dev, generator=gen) * 0.5 for _ in range(L_)]
    ssms = [torch.randn(1, Hv, S, S, device=dev, generator=gen) * 0.02 for _ in range(L_)]
    snaps = [torch.zeros(K - 1, S * S * Hv, dtype=torch.float16, device=dev) for _ in range(L_)]
    sync = torch.zeros(L_, Hk, dtype=torch.int32, device=dev)
    res = {}
    for T in (1, 4):
        qkv = torch.randn(T, ch, device=dev, generator=gen)
        z = torch.randn(T, Hv * S, device=dev, generator=gen)
        br, al = torch.randn(T, Hv, device=dev, generator=gen), torch.randn(T, Hv, device=dev, generator=gen)
        out = torch.empty(T, Hv * S, device=dev)

        def fused():
            for l in range(L_):
                kb.gdn_step(qkv, convs[l], conv_w, br, al, dt, aa, ssms[l], snaps[l], K, z, nw, 1e-6, sync[l], out=out)

        def chain():
            for l in range(L_):
                q, k, v, beta, g = kb.gdn_input(qkv, convs[l], conv_w, S, Hk, 1e-6, beta_raw=br, alpha=al, dt_bias=dt, a=aa)
                attn = kb.gated_delta_net_cache(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), g.view(1, T, Hv, 1),
                                                beta.view(1, T, Hv), ssms[l], snaps[l], K)
                kb.gdn_gated_norm(attn.view(T, Hv, S), z, nw, 1e-6)

        times = {}
        for name, fn in (("fused", fused), ("chain", chain)):
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            for _ in range(warmup):
                graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            del graph
            times[name] = e0.elapsed_time(e1) * 1e3 / (steps * L_)
        # bytes one layer must move: the state read and written back, the T - 1 f16 snapshots, the conv state slots
        # (read slot 0, write min(T, K) slots), the T rows of qkv, z, beta, alpha and the output
        nbytes = (S * S * Hv * 4 * 2 + (min(T, K) - 1) * S * S * Hv * 2 + 3 * ch * 4 * (1 + min(T, K)) +
                  T * (ch + 2 * Hv * S + 2 * Hv) * 4)
        gbs = nbytes / (times["fused"] * 1e-6) / 1e9
        res[f"gdn_layer_{T}"] = {
            "value": round(times["fused"], 2), "unit": "us/layer", "tokens": T, "three_calls_us": round(times["chain"], 2),
            "workload": f"one DeltaNet layer between its GEMMs, {T} token(s): conv input side, recurrence with K = 4 "
                        "f16 snapshots, gated norm (48/16 heads, d 128), 48 layers per CUDA graph",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / pk["hbm_gbs"], 4), "algorithmic_bytes_per_launch": nbytes,
                         "traffic": ncu_traffic(f"gdn_step_{T}")}}
    return res


def bench_dense_mask(kb, torch, dev, steps, warmup):
    """The two attention kernels with klein's dense f16 mask (engine.cpp:308-326, what klein's graph passes through
    ggml) instead of the analytic bounds: the 4-token verify step over 262,144 f16 cells (4 layers, inputs > L2) and a
    2,048-token bf16 prompt chunk over 4,096 cells, each beside the same call with analytic bounds."""
    def causal_mask(n_q, n_kv, pos0):
        # klein's mask for a prompt chunk at positions pos0 .. pos0 + n_q - 1 (engine.cpp:308-326): 0 where the cell is
        # at or before the row's position, -inf after it
        c = torch.arange(n_kv, device=dev)[None, :]
        p = pos0 + torch.arange(n_q, device=dev)[:, None]
        return torch.where(c <= p, 0.0, float("-inf")).half()

    gen = torch.Generator(device=dev)
    gen.manual_seed(17)
    pk, _ = measured_peaks()

    def time_calls(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / steps

    res = {}
    n_kv, n_q, n_layers = N_KV, N_Q, 4
    layers = []
    for _ in range(n_layers):
        kc = torch.randn(n_kv, H_KV * D, device=dev, generator=gen).half()
        vc = torch.randn(n_kv, H_KV * D, device=dev, generator=gen).half()
        layers.append((kc, vc, kb.kv_cache_view(kc, kb.F16, H_KV, D), kb.kv_cache_view(vc, kb.F16, H_KV, D)))
    q = torch.randn(1, n_q, H, D, device=dev, generator=gen)
    mask = causal_mask(n_q, n_kv, n_kv - n_q)
    t = {}
    for name, kw in (("analytic", dict(causal=True, pos0=n_kv - n_q)), ("dense", dict(mask=mask))):
        t[name] = time_calls(lambda: [kb.flash_attn_ext(q, l[2], l[3], SCALE, **kw) for l in layers]) / n_layers
    gbs = 2 * n_kv * H_KV * D * 2 / (t["dense"] * 1e-6) / 1e9
    res["verify_f16_dense_mask"] = {
        "value": round(t["dense"], 2), "unit": "us/layer", "analytic_bounds_us": round(t["analytic"], 2),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / pk["hbm_gbs"], 4)}}
    del layers, mask
    torch.cuda.empty_cache()
    T, n_kv = 2048, 4096
    q = torch.randn(1, T, H, D, device=dev, generator=gen).bfloat16().float()
    k = torch.randn(n_kv, H_KV * D, device=dev, generator=gen).bfloat16()
    v = torch.randn(n_kv, H_KV * D, device=dev, generator=gen).bfloat16()
    kv, vv = kb.kv_cache_view(k, kb.BF16, H_KV, D), kb.kv_cache_view(v, kb.BF16, H_KV, D)
    mask = causal_mask(T, n_kv, n_kv - T)
    t = {}
    for name, kw in (("analytic", dict(causal=True, pos0=n_kv - T)), ("dense", dict(mask=mask))):
        t[name] = time_calls(lambda: kb.flash_attn_ext(q, kv, vv, SCALE, **kw))
    flops = 4 * D * H * (T * (T + 1) // 2 + T * (n_kv - T))
    tf = flops / (t["dense"] * 1e-6) / 1e12
    res["prefill_bf16_2048_dense_mask"] = {
        "value": round(tf, 1), "unit": "TFLOP/s", "us": round(t["dense"], 1), "analytic_bounds_us": round(t["analytic"], 1),
        "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(tf / pk["bf16_tflops"], 4)}}
    return res


def bench_io_ops(kb, torch, dev, steps, warmup):
    """The ops around the two attention kinds at config[2]'s 4,096-token prefill (qwen35 shapes, f16 cache):
    kb_attn_prologue (Q/gate split, RMS norms, M-RoPE, K/V cache writes), kb_gdn_input (conv, SiLU, L2 norms, gates,
    conv-state snapshots) and kb_gdn_gated_norm; plus the same three at the 4-token verify (positions at the end of a
    262,144-cell context). HBM-bound: bytes = what
    each op must read and write once. Timed with CUDA events, each op alone in a loop (inputs > L2 at 4,096 tokens)."""
    import ctypes  # noqa: F401

    g = torch.Generator(device=dev)
    g.manual_seed(3)
    hd, nh, nkv, S, Hk, Hv = D, H, H_KV, 128, 16, 48
    ch = 2 * S * Hk + S * Hv
    pk, _ = measured_peaks()
    res = {}
    for T in (4096, 4):
        qfull = torch.randn(T, nh * 2 * hd, device=dev, generator=g)
        kcur = torch.randn(T, nkv * hd, device=dev, generator=g)
        vcur = torch.randn(T, nkv * hd, device=dev, generator=g)
        # the prefill from position 0; the verify step at the end of a 262,144-cell context (long-context angles)
        p = torch.arange(T, dtype=torch.int32, device=dev) + (0 if T > 4 else 262144 - T)
        pos = torch.cat([p, p, p, torch.zeros_like(p)])
        kv_idx = torch.arange(T, dtype=torch.int64, device=dev)  # cells of a T-cell cache
        qn = torch.ones(hd, device=dev)
        kcache = torch.zeros(T, nkv * hd, dtype=torch.float16, device=dev)
        vcache = torch.zeros_like(kcache)
        kc, vc = kb.cache_rows(kcache, kb.F16), kb.cache_rows(vcache, kb.F16)
        qkv = torch.randn(T, ch, device=dev, generator=g)
        state = torch.randn(4, 3 * ch, device=dev, generator=g)
        cw = torch.randn(ch, 4, device=dev, generator=g) * 0.5
        br = torch.randn(T, Hv, device=dev, generator=g)
        al = torch.randn(T, Hv, device=dev, generator=g)
        dt = torch.randn(Hv, device=dev, generator=g)
        aa = -torch.rand(Hv, device=dev, generator=g) - 0.1
        x = torch.randn(T, Hv, S, device=dev, generator=g)
        z = torch.randn(T, Hv, S, device=dev, generator=g)
        nw = torch.ones(S, device=dev)
        ops = {
            "attn_prologue": (lambda: kb.attn_prologue(qfull, kcur, vcur, pos, kv_idx, qn, qn, 1e-6, 64, [11, 11, 10, 0], 40,
                                                       1e7, kc, vc),
                              T * (nh * 2 * hd + 2 * nkv * hd) * 4 + T * (2 * nh * hd * 4 + 2 * nkv * hd * 2)),
            "gdn_input": (lambda: kb.gdn_input(qkv, state, cw, S, Hk, 1e-6, beta_raw=br, alpha=al, dt_bias=dt, a=aa),
                          T * ch * 4 * 2 + T * Hv * 4 * 4 + 4 * 3 * ch * 4),
            "gdn_gated_norm": (lambda: kb.gdn_gated_norm(x, z, nw, 1e-6), T * Hv * S * 4 * 3),
        }
        for name, (fn, nbytes) in ops.items():
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            # 10 calls per CUDA graph (as a captured forward launches them), so host overhead is not timed
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(torch.cuda.current_stream(dev))
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=cap):
                for _ in range(10):
                    fn()
            torch.cuda.current_stream(dev).wait_stream(cap)
            graph.replay()
            torch.cuda.synchronize()
            reps = max(2, steps // 10)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            del graph
            us = e0.elapsed_time(e1) * 1e3 / (reps * 10)
            gbs = nbytes / (us * 1e-6) / 1e9
            res[f"{name}_{T}"] = {"value": round(us, 2), "unit": "us", "tokens": T,
                                  "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"],
                                               "unit": "GB/s", "frac": round(gbs / pk["hbm_gbs"], 4),
                                               "algorithmic_bytes_per_launch": nbytes,
                                               "traffic": ncu_traffic(f"{name}_{T}")}}
    return res


def bench_gdn_prefill(kb, torch, dev, steps, warmup):
    """config[2] DeltaNet half: 4,096 tokens in 64-token chunks from a zero state (48 value / 16 key heads, d 128,
    K = 4 slots) through kb_gated_delta_net with scratch (tcgen05 prep + state kernels, the last 3 tokens
    recurrent). Two input sets alternate; the records (202 MB) exceed L2 as well."""
    import ctypes

    import numpy as np

    T, K = 4096, 4
    rng = np.random.default_rng(4096)
    sets = []
    for _ in range(2):
        q = rng.standard_normal((1, T, 16, 128), dtype=np.float32)
        k = rng.standard_normal((1, T, 16, 128), dtype=np.float32)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        v = rng.standard_normal((1, T, 48, 128), dtype=np.float32)
        beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((1, T, 48, 1))))).astype(np.float32)
        g = (-np.logaddexp(0.0, rng.standard_normal((1, T, 48, 1)))).astype(np.float32)
        s0 = np.zeros((1, 48, 128, 128), dtype=np.float32)
        sets.append([torch.from_numpy(a).to(dev) for a in (q, k, v, g, beta, s0)])
    nbytes = kb.lib().kb_gated_delta_net_scratch_bytes(ctypes.byref(kb.from_torch(sets[0][2])),
                                                      ctypes.byref(kb.from_torch(sets[0][3])), K)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    for i in range(warmup):
        kb.gated_delta_net(*sets[i % 2], K, scratch=scratch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        kb.gated_delta_net(*sets[i % 2], K, scratch=scratch)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    C, d, H = 64, 128, 48
    flops = T * H * (10 * C * d + 6 * d * d)  # chunked-form algorithmic count (35.4 GFLOP)
    tf = flops / (us * 1e-6) / 1e12
    pk, kind = measured_peaks()
    return {"value": round(us, 1), "unit": "us/layer", "tflops_algorithmic": round(tf, 2),
            "workload": "config[2] gated DeltaNet prefill, 4096 tokens, chunk 64, 48 value / 16 key heads, d 128",
            "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(tf / pk["bf16_tflops"], 4), "peak_kind": kind + " burst (f16 operands)",
                         "algorithmic_flops_per_launch": flops, "traffic": ncu_traffic("gdn_chunk_prefill_4096")}}


# ------------------------------------------------------------------------------------------------ head shards

def bench_head_shards(kb, torch, dev, steps, warmup, rank, world, dist):
    """N > 1: the paths that shard by heads with no collective (kv_split.gdn_head_shard / fa_head_shard), each rank
    running the single-GPU op on its heads: config[1]'s DeltaNet verify step (48 layers per CUDA graph), config[2]'s
    4,096-token prefill attention (bf16) and its chunked DeltaNet prefill. Strong scaling: the whole op's work is split
    over the N ranks; the time is the max over ranks (device events), throughput = the whole op's work / that time."""
    import ctypes

    import numpy as np

    from klein_b200.kv_split import fa_head_shard, gdn_head_shard

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def time_graph(fn, reps):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(max(1, warmup)):
            g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) * 1e3 / reps

    pk, kind = measured_peaks()
    res = {}
    gen = torch.Generator(device=dev)
    gen.manual_seed(55)
    # DeltaNet verify step on this rank's value heads (key heads gathered, H_k = H_v = local heads)
    L_, T, K, S = 48, 4, 4, 128
    lo, hi, kidx = gdn_head_shard(16, 48, world, rank)
    n = hi - lo
    q = torch.nn.functional.normalize(torch.randn(1, T, 16, S, device=dev, generator=gen), dim=-1)[:, :, kidx].contiguous()
    k = torch.nn.functional.normalize(torch.randn(1, T, 16, S, device=dev, generator=gen), dim=-1)[:, :, kidx].contiguous()
    v = torch.randn(1, T, n, S, device=dev, generator=gen)
    g = -torch.nn.functional.softplus(torch.randn(1, T, n, 1, device=dev, generator=gen))
    beta = torch.sigmoid(torch.randn(1, T, n, 1, device=dev, generator=gen))
    states = [torch.randn(1, n, S, S, device=dev, generator=gen) * 0.02 for _ in range(L_)]
    snaps = [torch.zeros(K - 1, S * S * n, dtype=torch.float16, device=dev) for _ in range(L_)]
    attn = torch.empty(1, T, n, S, device=dev)
    L = kb.lib()
    ins = [kb.from_torch(x) for x in (q, k, v, g, beta)]
    outs = [(kb.from_torch(states[l]), kb.from_torch(snaps[l])) for l in range(L_)]
    at = kb.from_torch(attn)

    def gdn_step():
        st = torch.cuda.current_stream(dev).cuda_stream
        for l in range(L_):
            rc = L.kb_gated_delta_net_cache(*[ctypes.byref(x) for x in ins], ctypes.byref(outs[l][0]),
                                            ctypes.byref(outs[l][1]), K, ctypes.byref(at), None, 0, ctypes.c_void_p(st))
            if rc != 0:
                raise kb.KbError("kb_gated_delta_net_cache", rc)

    us = max_over_ranks(time_graph(gdn_step, max(3, steps)) / L_)
    nbytes = S * S * 48 * 4 * 2 + (K - 1) * S * S * 48 * 2 + (2 * T * 16 * S + 2 * T * 48 * S + 2 * T * 48) * 4
    res["gdn_verify_heads"] = {"value": round(us, 2), "unit": "us/layer", "heads_per_rank": n,
                               "workload": "config[1] DeltaNet verify step (48 layers per graph), value heads split "
                                           "over the ranks, max over ranks",
                               "roofline": {"bound": "hbm", "achieved": round(nbytes / (us * 1e-6) / 1e9, 1),
                                            "peak": pk["hbm_gbs"] * world, "unit": "GB/s (all ranks)",
                                            "frac": round(nbytes / (us * 1e-6) / 1e9 / (pk["hbm_gbs"] * world), 4)}}
    del states, snaps, q, k, v, g, beta, attn
    # prefill attention (config[2], bf16) on this rank's query heads and the KV heads they read
    TT = 4096
    q_lo, q_hi, kv_lo, kv_hi = fa_head_shard(H, H_KV, world, rank)
    nq, nkv = q_hi - q_lo, kv_hi - kv_lo
    qp = torch.randn(1, TT, nq, D, device=dev, generator=gen).bfloat16().float()
    kk = torch.randn(TT, nkv * D, device=dev, generator=gen).bfloat16()
    vv = torch.randn(TT, nkv * D, device=dev, generator=gen).bfloat16()
    kv_, vv_ = kb.kv_cache_view(kk, kb.BF16, nkv, D), kb.kv_cache_view(vv, kb.BF16, nkv, D)
    outp = torch.empty(1, TT, nq, D, device=dev)

    def prefill():
        kb.flash_attn_ext(qp, kv_, vv_, SCALE, causal=True, pos0=0, out=outp,
                          stream=torch.cuda.current_stream(dev).cuda_stream)

    us = max_over_ranks(time_graph(prefill, max(3, steps // 4)))
    flops = 2.0 * D * H * TT * (TT + 1)
    tf = flops / (us * 1e-6) / 1e12
    res["prefill_bf16_4096_heads"] = {"value": round(tf, 1), "unit": "TFLOP/s (all ranks)", "us_per_layer": round(us, 2),
                                      "q_heads_per_rank": nq, "kv_heads_per_rank": nkv,
                                      "roofline": {"bound": "tensor", "achieved": round(tf, 1),
                                                   "peak": pk["bf16_tflops"] * world, "unit": "TFLOP/s (all ranks)",
                                                   "frac": round(tf / (pk["bf16_tflops"] * world), 4)}}
    del qp, kk, vv, outp
    # chunked DeltaNet prefill (config[2]) on this rank's value heads
    rng = np.random.default_rng(4096)
    qn = rng.standard_normal((1, TT, 16, S), dtype=np.float32)
    kn = rng.standard_normal((1, TT, 16, S), dtype=np.float32)
    qn /= np.linalg.norm(qn, axis=-1, keepdims=True)
    kn /= np.linalg.norm(kn, axis=-1, keepdims=True)
    vn = rng.standard_normal((1, TT, 48, S), dtype=np.float32)
    bn = (1.0 / (1.0 + np.exp(-rng.standard_normal((1, TT, 48, 1))))).astype(np.float32)
    gn = (-np.logaddexp(0.0, rng.standard_normal((1, TT, 48, 1)))).astype(np.float32)
    args = [torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in
            (qn[:, :, kidx], kn[:, :, kidx], vn[:, :, lo:hi], gn[:, :, lo:hi], bn[:, :, lo:hi],
             np.zeros((1, n, S, S), dtype=np.float32))]
    nb = L.kb_gated_delta_net_scratch_bytes(ctypes.byref(kb.from_torch(args[2])), ctypes.byref(kb.from_torch(args[3])), 4)
    scratch = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)

    def gdn_prefill():
        kb.gated_delta_net(*args, 4, scratch=scratch, stream=torch.cuda.current_stream(dev).cuda_stream)

    us = max_over_ranks(time_graph(gdn_prefill, max(3, steps // 4)))
    flops = TT * 48 * (10 * 64 * S + 6 * S * S)
    tf = flops / (us * 1e-6) / 1e12
    res["gdn_prefill_4096_heads"] = {"value": round(us, 1), "unit": "us/layer", "heads_per_rank": n,
                                     "tflops_algorithmic": round(tf, 2),
                                     "roofline": {"bound": "tensor", "achieved": round(tf, 2),
                                                  "peak": pk["bf16_tflops"] * world, "unit": "TFLOP/s (all ranks)",
                                                  "frac": round(tf / (pk["bf16_tflops"] * world), 4)}}
    return res


# ------------------------------------------------------------------------------------------------ whole stack

HIDDEN = 5120  # qwen35 27B n_embd


def bench_stack(kb, torch, dev, steps, warmup, contexts=(4096, 32768, 131072, 262144)):
    """config[4]: the whole 64-layer attention stack of a 27B qwen35 model (48 gated DeltaNet + 16 GQA full-attention
    layers, hidden 5120; random-init bf16 projections, 7.25 B parameters, distinct per layer; the FFN blocks are not
    part of the attention stack and are left out) over klein's State in HBM (kb_state, caches of klein's --kv auto type:
    q8_0 up to 131,072 cells, q4_0 beyond, engine.cpp:114; 4 recurrent slots, f16 snapshots). Per context: batch-1
    decode and the 4-token verify step, each one CUDA graph of 64 layers (RMS norm, projections by cuBLAS through
    torch, kb_layer_attention / kb_layer_deltanet, output projection, residual), timed whole and with the projections
    and norms removed (the attention-path ops alone, fed by fixed projection outputs). Plus the MTP head's attention
    over its full 16,384-cell ring and the 16,384-token prefill in klein's 2,048-token chunks."""
    import ctypes  # noqa: F401

    from klein_b200.state import State

    HD, NH, NKV, S, HK, HV = D, H, H_KV, 128, 16, 48
    CH = 2 * S * HK + S * HV
    eps = 1e-6
    dims = kb.qwen35_dims()
    n_layer = dims.n_layer
    attn_layer = [((il + 1) % dims.full_attn_interval) == 0 for il in range(n_layer)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(27)
    bf = torch.bfloat16

    def randw(i, o):
        return (torch.randn(i, o, device=dev, generator=gen) * (i ** -0.5)).to(bf)

    W = []
    for il in range(n_layer + 1):  # + the MTP block's attention (index n_layer)
        if il == n_layer or attn_layer[il]:
            W.append({"wq": randw(HIDDEN, 2 * NH * HD), "wk": randw(HIDDEN, NKV * HD), "wv": randw(HIDDEN, NKV * HD),
                      "wo": randw(NH * HD, HIDDEN), "norm": torch.ones(HIDDEN, device=dev),
                      "q_norm": torch.ones(HD, device=dev), "k_norm": torch.ones(HD, device=dev)})
        else:
            W.append({"wqkv": randw(HIDDEN, CH), "wz": randw(HIDDEN, HV * S), "wb": randw(HIDDEN, HV),
                      "wa": randw(HIDDEN, HV), "wout": randw(HV * S, HIDDEN), "norm": torch.ones(HIDDEN, device=dev),
                      "conv_w": torch.randn(CH, 4, device=dev, generator=gen) * 0.5,
                      "dt": torch.randn(HV, device=dev, generator=gen), "a": -torch.rand(HV, device=dev, generator=gen) - 0.1,
                      "ssm_norm": torch.ones(S, device=dev)})
    n_params = sum(t.numel() for w in W[:n_layer] for t in w.values() if t.dtype == bf)
    rope = kb.KbRopeParams(64, (ctypes.c_int32 * 4)(11, 11, 10, 0), 40, 1e7, 1.0, 1.0)

    def rms(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def timed(fn, reps):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(max(1, warmup)):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) * 1e3 / reps

    def fill_caches(st, n_cells, kv_type):
        # ~N(0,1) rows quantised once (klein's set_rows rounding), copied into every attention layer's K and V
        rows = torch.randn(min(n_cells, 65536), NKV * HD, device=dev, generator=gen)
        qr = quantize_q8_0_rows(torch, rows) if kv_type == kb.Q8_0 else quantize_q4_0_rows(torch, rows)
        del rows
        for il in range(n_layer + 1):
            if il < n_layer and not attn_layer[il]:
                continue
            lay = st.layer(il)
            for t in (lay.k, lay.v):
                view = st.view(t)
                for c0 in range(0, view.shape[0], qr.shape[0]):
                    c1 = min(view.shape[0], c0 + qr.shape[0])
                    view[c0:c1].copy_(qr[:c1 - c0])
        del qr

    def layer_ops(st, n, p, pos, kv_idx, scratch_a, scratch_g, proj, outs, mtp=False):
        """the attention-path ops of every layer for one pass, fed by proj[il] (the projection outputs)"""
        stream = torch.cuda.current_stream(dev).cuda_stream
        for il in ([n_layer] if mtp else range(n_layer)):
            w, pr = W[il], proj[il]
            if il == n_layer or attn_layer[il]:
                st.attention(il, p, pr["qfull"], pr["kcur"], pr["vcur"], pos, kv_idx, w["q_norm"], w["k_norm"], eps, rope,
                             outs["attn"], scratch_a, stream)
            else:
                st.deltanet(il, n, pr["qkv"], pr["z"], pr["b"], pr["a"], w["dt"], w["a"], w["conv_w"], w["ssm_norm"], eps,
                            outs["gdn"], scratch_g, stream)

    def full_step(st, n, p, pos, kv_idx, scratch_a, scratch_g, x, outs, mtp=False):
        """one forward pass of n tokens through the stack: norms, projections, the layer ops, output projections and
        residuals (x updated in place)"""
        stream = torch.cuda.current_stream(dev).cuda_stream
        for il in ([n_layer] if mtp else range(n_layer)):
            w = W[il]
            hb = rms(x, w["norm"]).to(bf)
            if il == n_layer or attn_layer[il]:
                qfull = (hb @ w["wq"]).float()
                kcur, vcur = (hb @ w["wk"]).float(), (hb @ w["wv"]).float()
                st.attention(il, p, qfull, kcur, vcur, pos, kv_idx, w["q_norm"], w["k_norm"], eps, rope, outs["attn"],
                             scratch_a, stream)
                x.add_((outs["attn"].to(bf) @ w["wo"]).float())
            else:
                qkv, z = (hb @ w["wqkv"]).float(), (hb @ w["wz"]).float()
                br, al = (hb @ w["wb"]).float(), (hb @ w["wa"]).float()
                st.deltanet(il, n, qkv, z, br, al, w["dt"], w["a"], w["conv_w"], w["ssm_norm"], eps, outs["gdn"],
                            scratch_g, stream)
                x.add_((outs["gdn"].to(bf) @ w["wout"]).float())

    def proj_inputs(n):
        pr = []
        for il in range(n_layer + 1):
            if il == n_layer or attn_layer[il]:
                pr.append({"qfull": torch.randn(n, 2 * NH * HD, device=dev, generator=gen),
                           "kcur": torch.randn(n, NKV * HD, device=dev, generator=gen),
                           "vcur": torch.randn(n, NKV * HD, device=dev, generator=gen)})
            else:
                pr.append({"qkv": torch.randn(n, CH, device=dev, generator=gen),
                           "z": torch.randn(n, HV * S, device=dev, generator=gen),
                           "b": torch.randn(n, HV, device=dev, generator=gen),
                           "a": torch.randn(n, HV, device=dev, generator=gen)})
        return pr

    def pass_inputs(st, n, mtp=False, cell0=None, kv_lo=0):
        p, idx = st.plan(n, kv_lo=kv_lo, mtp=mtp, cell0=cell0)
        posv = torch.arange(n, dtype=torch.int32, device=dev) + int(p.cell0)
        pos = torch.cat([posv, posv, posv, torch.zeros_like(posv)])
        return p, pos, torch.from_numpy(idx).to(dev)

    pk, _ = measured_peaks()
    res = {"workload": "config[4] whole attention stack, qwen35 27B shapes: 48 gated DeltaNet + 16 GQA layers (24 / 4 "
                       "heads x 256), hidden 5120, random-init bf16 projections (FFN blocks excluded), klein's State in "
                       "HBM with --kv auto cache types, 4 recurrent slots",
           "projection_params": n_params, "decode": {}, "verify": {}}
    reps = max(3, steps)
    for ctx_len in contexts:
        kv_type = kb.Q8_0 if ctx_len <= 131072 else kb.Q4_0
        cfg = kb.state_config(ctx_len, kv_type, kv_type, 4, kb.F16, 16384)
        st = State(dims, cfg, dev)
        fill_caches(st, ctx_len, kv_type)
        for mode, n in (("decode", 1), ("verify", 4)):
            st.n_past = ctx_len - n  # the pass writes the last n cells of the context
            p, pos, kv_idx = pass_inputs(st, n)
            scratch_a = torch.empty(max(st.attention_scratch_bytes(n_layer - 1, p), 1), dtype=torch.uint8, device=dev)
            scratch_g = torch.empty(max(st.deltanet_scratch_bytes(0, n), 1), dtype=torch.uint8, device=dev)
            outs = {"attn": torch.empty(n, NH * HD, device=dev), "gdn": torch.empty(n, HV * S, device=dev)}
            x = torch.randn(n, HIDDEN, device=dev, generator=gen)
            proj = proj_inputs(n)
            t_full = timed(lambda: full_step(st, n, p, pos, kv_idx, scratch_a, scratch_g, x, outs), reps)
            t_attn = timed(lambda: layer_ops(st, n, p, pos, kv_idx, scratch_a, scratch_g, proj, outs), reps)
            kvb = kv_bytes_per_layer(int(p.n_kv), "q8_0" if kv_type == kb.Q8_0 else "q4_0")
            gdn_b = S * S * HV * 4 * 2 + 3 * S * S * HV * 2  # state read + slot 0 write + 3 f16 snapshots
            att_bytes = 16 * kvb + 48 * gdn_b
            res[mode][str(ctx_len)] = {
                "kv_type": "q8_0" if kv_type == kb.Q8_0 else "q4_0", "step_us": round(t_full, 1),
                "attention_us": round(t_attn, 1), "projections_and_norms_us": round(t_full - t_attn, 1),
                "attention_bytes": att_bytes,
                "attention_hbm_frac": round(att_bytes / (t_attn * 1e-6) / 1e9 / pk["hbm_gbs"], 4)}
            del proj, outs, scratch_a, scratch_g
        st.close()
        del st
        torch.cuda.empty_cache()

    # the MTP head's attention: decode over its full 16,384-cell ring at a position past several wraps
    cfg = kb.state_config(131072, kb.Q8_0, kb.Q8_0, 4, kb.F16, 16384)
    st = State(dims, cfg, dev)
    fill_caches(st, 16384, kb.Q8_0)
    p, pos, kv_idx = pass_inputs(st, 1, mtp=True, cell0=70001, kv_lo=1)
    scratch_a = torch.empty(st.attention_scratch_bytes(n_layer, p), dtype=torch.uint8, device=dev)
    outs = {"attn": torch.empty(1, NH * HD, device=dev), "gdn": torch.empty(1, HV * S, device=dev)}
    x = torch.randn(1, HIDDEN, device=dev, generator=gen)
    proj = proj_inputs(1)
    t_full = timed(lambda: full_step(st, 1, p, pos, kv_idx, scratch_a, None, x, outs, mtp=True), reps)
    t_attn = timed(lambda: layer_ops(st, 1, p, pos, kv_idx, scratch_a, None, proj, outs, mtp=True), reps)
    res["mtp_16k"] = {"ring_cells": int(p.ring), "n_kv": int(p.n_kv), "layer_us": round(t_full, 1),
                      "attention_us": round(t_attn, 1), "kv_type": "q8_0"}
    st.close()
    del st, proj, outs, scratch_a
    torch.cuda.empty_cache()

    # the 16,384-token prefill: 8 chunks of 2,048 (klein's n_ubatch) through the 64 layers, q8_0 caches
    T, CHUNK = 16384, 2048
    cfg = kb.state_config(T, kb.Q8_0, kb.Q8_0, 4, kb.F16, 16384)
    st = State(dims, cfg, dev)
    x = torch.randn(CHUNK, HIDDEN, device=dev, generator=gen)
    outs = {"attn": torch.empty(CHUNK, NH * HD, device=dev), "gdn": torch.empty(CHUNK, HV * S, device=dev)}
    passes = []
    for c in range(T // CHUNK):
        st.n_past = c * CHUNK
        passes.append(pass_inputs(st, CHUNK))
    sa = max(st.attention_scratch_bytes(n_layer - 1, pp[0]) for pp in passes)
    scratch_a = torch.empty(sa, dtype=torch.uint8, device=dev)
    scratch_g = torch.empty(st.deltanet_scratch_bytes(0, CHUNK), dtype=torch.uint8, device=dev)
    proj = proj_inputs(CHUNK)

    def prefill(attn_only):
        st.clear(torch.cuda.current_stream(dev).cuda_stream)
        for p, pos, kv_idx in passes:
            if attn_only:
                layer_ops(st, CHUNK, p, pos, kv_idx, scratch_a, scratch_g, proj, outs)
            else:
                full_step(st, CHUNK, p, pos, kv_idx, scratch_a, scratch_g, x, outs)

    times = {}
    for attn_only in (False, True):
        prefill(attn_only)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        prefill(attn_only)
        e1.record()
        torch.cuda.synchronize()
        times[attn_only] = e0.elapsed_time(e1)
    flops = 16 * 4.0 * D * H * T * (T + 1) / 2 + 48 * T * HV * (10 * 64 * S + 6 * S * S)
    res["prefill_16384"] = {"chunk": CHUNK, "kv_type": "q8_0", "total_ms": round(times[False], 2),
                            "attention_ms": round(times[True], 2),
                            "projections_and_norms_ms": round(times[False] - times[True], 2),
                            "attention_algorithmic_tflop": round(flops / 1e12, 2),
                            "attention_tflops": round(flops / (times[True] * 1e-3) / 1e12, 1)}
    st.close()
    del st, proj, outs, scratch_a, scratch_g, W
    torch.cuda.empty_cache()
    return res


def make_layers(kb, torch, dev, gen, n_kv, kv_type):
    layers = []
    for _ in range(LAYERS):
        kf = torch.randn(n_kv, H_KV * D, device=dev, generator=gen)
        vf = torch.randn(n_kv, H_KV * D, device=dev, generator=gen)
        if kv_type == "f16":
            kc, vc, t = kf.half(), vf.half(), kb.F16
        elif kv_type == "q8_0":
            kc, vc, t = quantize_q8_0_rows(torch, kf), quantize_q8_0_rows(torch, vf), kb.Q8_0
        else:
            kc, vc, t = quantize_q4_0_rows(torch, kf), quantize_q4_0_rows(torch, vf), kb.Q4_0
        del kf, vf
        layers.append((kc, vc, kb.kv_cache_view(kc, t, H_KV, D), kb.kv_cache_view(vc, t, H_KV, D)))
    return layers


PARITY_N_KV = 32768  # cells of the sequence-split parity check (4,096 per rank at N = 8)


def exact_attention_f64(q, k, v, pos0, scale=SCALE):
    """Exact causal attention in float64 (numpy): q [n_q][H][D], k / v [n_kv][H_kv][D], query i sees cells
    [0, pos0 + i]. The checker of the sequence-split parity run (ggml's flash-attention semantics, ops.cpp:8842-9078,
    with Q rounded to f16 beforehand by the caller)."""
    import numpy as np

    n_q, h, d = q.shape
    g = h // k.shape[1]
    out = np.zeros((n_q, h, d))
    vis = np.arange(k.shape[0])[None, :] <= (pos0 + np.arange(n_q))[:, None]
    for hh in range(h):
        s = (q[:, hh].astype(np.float64) @ k[:, hh // g].T.astype(np.float64)) * scale
        s = np.where(vis, s, -np.inf)
        p = np.exp(s - s.max(1, keepdims=True))
        out[:, hh] = (p @ v[:, hh // g].astype(np.float64)) / p.sum(1, keepdims=True)
    return out


def split_parity(kb, torch, dev, args, rank, world, xchg, dist):
    """Correctness of the timed path at this N, before timing: the same per-rank calls and the same exchange
    (push kernel, fused push or NCCL) on a PARITY_N_KV-cell f16 cache split the same way; every rank's merged
    output must be identical, and rank 0's is compared with exact attention over the whole cache."""
    import ctypes

    import numpy as np

    from klein_b200.kv_split import kv_range, local_bounds, packed_part_floats

    n_kv = PARITY_N_KV
    rng = np.random.default_rng(2024)  # the same cache and queries on every rank
    q = rng.standard_normal((N_Q, H, D), dtype=np.float32)
    kc = rng.standard_normal((n_kv, H_KV * D), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((n_kv, H_KV * D), dtype=np.float32).astype(np.float16)
    lo, hi = kv_range(n_kv, world, rank)
    kt = torch.from_numpy(kc[lo:hi].copy()).to(dev)
    vt = torch.from_numpy(vc[lo:hi].copy()).to(dev)
    kv, vv = kb.kv_cache_view(kt, kb.F16, H_KV, D), kb.kv_cache_view(vt, kb.F16, H_KV, D)
    pos0, kv_lo = local_bounds(lo, n_kv - N_Q, 0)
    qd = torch.from_numpy(q).to(dev).unsqueeze(0)
    out = torch.zeros(1, N_Q, H, D, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    rows = N_Q * H
    kb.device_error(clear=True)
    if world == 1:
        kb.flash_attn_ext(qd, kv, vv, SCALE, causal=True, pos0=pos0, out=out)
    elif args.exchange in ("fused", "kernel"):
        L = kb.lib()
        qt = kb.kb_tensor(qd.data_ptr(), kb.F32, [D, N_Q, H, 1], [4, H * D * 4, D * 4, N_Q * H * D * 4])
        prm = kb.fa_params(SCALE, causal=True, pos0=pos0, kv_lo=kv_lo)
        nb = L.kb_flash_attn_ext_push_scratch_bytes(ctypes.byref(qt), ctypes.byref(kv), ctypes.byref(vv),
                                                    ctypes.byref(prm))
        scratch = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
        if args.exchange == "kernel":
            xchg.attend_exchange(qt, kv, vv, prm, scratch.data_ptr(), nb, kb.from_torch(out), st)
        else:
            xchg.attend_and_combine(qt, kv, vv, prm, scratch.data_ptr(), nb, rows, D, out.data_ptr(), st)
    else:
        part = torch.empty(packed_part_floats(rows, D), device=dev)
        kb.flash_attn_ext_partial(qd, kv, vv, SCALE, part, causal=True, pos0=pos0, kv_lo=kv_lo)
        if xchg is not None:
            xchg.exchange_and_combine(part.data_ptr(), rows, D, out.data_ptr(), st)
        else:
            gathered = torch.empty(world * part.numel(), device=dev)
            dist.all_gather_into_tensor(gathered, part)
            rc = kb.lib().kb_lse_combine(ctypes.c_void_p(gathered.data_ptr()),
                                         ctypes.c_void_p(gathered.data_ptr() + rows * D * 4), ctypes.c_int64(part.numel()),
                                         world, ctypes.c_int64(rows), D, ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(st))
            if rc != 0:
                raise kb.KbError("kb_lse_combine", rc)
    torch.cuda.synchronize()
    code = kb.device_error(clear=True)
    spread = 0.0
    if world > 1:
        ref = out.clone()
        dist.broadcast(ref, src=0)
        d = torch.tensor([float((out - ref).abs().max())], device=dev)
        dist.all_reduce(d, op=dist.ReduceOp.MAX)
        c = torch.tensor([float(code)], device=dev)
        dist.all_reduce(c, op=dist.ReduceOp.MAX)
        spread, code = float(d.item()), int(c.item())
    res = {"n": world, "n_kv": n_kv, "exchange": args.exchange if world > 1 else "none",
           "ranks_max_abs_diff": spread, "device_error": code}
    if rank == 0:
        qr = q.astype(np.float16).astype(np.float32)  # Q as the f16 K dot type sees it (ops.cpp:8960)
        exact = exact_attention_f64(qr, kc.astype(np.float32).reshape(n_kv, H_KV, D),
                                    vc.astype(np.float32).reshape(n_kv, H_KV, D), n_kv - N_Q)
        gpu = out[0].cpu().numpy().astype(np.float64)
        res["e_gpu"] = float(np.abs(gpu - exact).max() / np.abs(exact).max())
        res["ok"] = bool(res["e_gpu"] <= 2e-3 and code == 0 and spread == 0.0)
    return res


def run_gpu(args, rank: int, world: int, local_rank: int):
    import ctypes

    import torch
    import torch.distributed as dist

    import klein_b200 as kb

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep NCCL's version banner off stdout (one JSON line)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
        if args.exchange == "nccl":
            args.eager = True  # NCCL collectives stay out of the step graphs
    kb.lib()

    from klein_b200.kv_split import kv_range, local_bounds, packed_part_floats

    lo, hi = kv_range(N_KV, world, rank)  # this rank's contiguous KV range (strong scaling)
    n_kv = hi - lo
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    layers = make_layers(kb, torch, dev, gen, n_kv, "f16")
    q = torch.randn(1, N_Q, H, D, device=dev, generator=gen)
    out = torch.empty(1, N_Q, H, D, device=dev)
    stream = torch.cuda.current_stream(dev)

    # causal among the 4 new cells, which sit at the end of the last rank's range
    pos0, kv_lo = local_bounds(lo, N_KV - N_Q, 0)

    qt = kb.kb_tensor(q.data_ptr(), kb.F32, [D, N_Q, H, 1], [4, H * D * 4, D * 4, N_Q * H * D * 4])
    dt = kb.kb_tensor(out.data_ptr(), kb.F32, [D, H, N_Q, 1], [4, D * 4, H * D * 4, N_Q * H * D * 4])
    prm = kb.fa_params(SCALE, causal=True, pos0=pos0, kv_lo=kv_lo)
    L = kb.lib()
    need = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qt), ctypes.byref(layers[0][2]), ctypes.byref(layers[0][3]),
                                             ctypes.byref(prm))
    if world > 1:  # the fused exchange needs its counter as well
        need = max(need, L.kb_flash_attn_ext_push_scratch_bytes(ctypes.byref(qt), ctypes.byref(layers[0][2]),
                                                                ctypes.byref(layers[0][3]), ctypes.byref(prm)))
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    sp = ctypes.c_void_p(scratch.data_ptr())
    st = ctypes.c_void_p(stream.cuda_stream)

    rows = N_Q * H
    xchg = None
    if world > 1:
        # per-rank packed partial [o rows x D | (m, l) rows x 2], exchanged over NVLink (kb_partials_push into every
        # rank's gather buffer + kb_lse_combine_wait), or all-gathered over NCCL and merged by kb_lse_combine
        pf = packed_part_floats(rows, D)
        part = torch.empty(pf, device=dev)
        gathered = torch.empty(world * pf, device=dev)
        if args.exchange in ("p2p", "fused", "kernel"):
            def all_gather_obj(obj):
                objs = [None] * world
                dist.all_gather_object(objs, obj)
                return objs
            xchg = kb.PeerExchange(rank, world, pf, all_gather_obj)
        pt = kb.kb_tensor(part.data_ptr(), kb.F32, [D, H, N_Q, 1], [4, D * 4, H * D * 4, N_Q * H * D * 4])
        ml_ptr = ctypes.c_void_p(part.data_ptr() + rows * D * 4)
        g_o = ctypes.c_void_p(gathered.data_ptr())
        g_ml = ctypes.c_void_p(gathered.data_ptr() + rows * D * 4)

    def layer_call(l, st, qx=None, dx=None):
        qx, dx = qx or qt, dx or dt
        if world == 1:
            rc = L.kb_flash_attn_ext(ctypes.byref(qx), ctypes.byref(layers[l][2]), ctypes.byref(layers[l][3]), None,
                                     ctypes.byref(prm), ctypes.byref(dx), sp, ctypes.c_size_t(need), st)
            if rc != 0:
                raise kb.KbError("kb_flash_attn_ext", rc)
            return
        if xchg is not None and args.exchange == "kernel":
            # the partial attention, the exchange over NVLink and the final merge in one launch
            xchg.attend_exchange(qx, layers[l][2], layers[l][3], prm, sp.value, need, dx, st.value)
            return
        if xchg is not None and args.exchange == "fused":
            # the partial attention writes its rows straight into every rank's gather buffer, then the merge
            xchg.attend_and_combine(qt, layers[l][2], layers[l][3], prm, sp.value, need, rows, D, out.data_ptr(),
                                    st.value)
            return
        rc = L.kb_flash_attn_ext_partial(ctypes.byref(qt), ctypes.byref(layers[l][2]), ctypes.byref(layers[l][3]), None,
                                         ctypes.byref(prm), ctypes.byref(pt), ml_ptr, sp, ctypes.c_size_t(need), st)
        if rc != 0:
            raise kb.KbError("kb_flash_attn_ext_partial", rc)
        if xchg is not None:
            # kb_partials_push into every rank's gather buffer, then kb_lse_combine_wait
            xchg.exchange_and_combine(part.data_ptr(), rows, D, out.data_ptr(), st.value)
            return
        dist.all_gather_into_tensor(gathered, part)
        rc = L.kb_lse_combine(g_o, g_ml, ctypes.c_int64(pf), world, ctypes.c_int64(rows), D,
                              ctypes.c_void_p(out.data_ptr()), st)
        if rc != 0:
            raise kb.KbError("kb_lse_combine", rc)

    def step(st):
        for l in range(LAYERS):
            layer_call(l, st)

    def graphed(fn):
        # one step captured as a CUDA graph (as ggml-cuda runs klein's forward); replays on the current stream
        if args.eager:
            return lambda: fn(st)
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            fn(ctypes.c_void_p(cap.cuda_stream))
        stream.wait_stream(cap)
        graphs.append(g)
        return g.replay

    parity = split_parity(kb, torch, dev, args, rank, world, xchg, dist if world > 1 else None)

    graphs = []
    for _ in range(args.warmup):
        step(st)
    torch.cuda.synchronize()
    run_step = graphed(step)
    for _ in range(2):
        run_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            run_step()
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    us_per_layer = ms_per_step * 1e3 / LAYERS
    # this library's kernels per layer: attention (+ split combine when the plan splits the cells), then at N > 1
    # push + merge-wait (p2p), merge-wait (fused: the combine pushes), merge (nccl; NCCL's own kernel not counted);
    # the in-kernel exchange is one launch
    combine = 1 if need > 0 else 0
    kernels_per_call = {1: 1 + combine}.get(world) if world == 1 else \
        {"kernel": 1, "p2p": 1 + combine + 2, "fused": 3, "nccl": 1 + combine + 1}[args.exchange]
    launches = args.steps * LAYERS * kernels_per_call

    # end to end through the C ABI: per layer, pinned host Q -> device, attention, output -> pinned host. The
    # copies run on streams of their own (one for each direction), so that layer l + 1's Q arrives and layer l's
    # output leaves while layer l computes; every copy is inside the timed step.
    q_host = torch.randn(LAYERS, N_Q, H, D).pin_memory()
    o_host = torch.empty(LAYERS, N_Q, H, D).pin_memory()
    q_dev = torch.empty(LAYERS, N_Q, H, D, device=dev)
    o_dev = torch.empty(LAYERS, N_Q, H, D, device=dev)  # [token][head][dim]: dst's [D, H, n_q] layout
    q_ts = [kb.kb_tensor(q_dev[l].data_ptr(), kb.F32, [D, N_Q, H, 1], [4, H * D * 4, D * 4, N_Q * H * D * 4])
            for l in range(LAYERS)]
    o_ts = [kb.kb_tensor(o_dev[l].data_ptr(), kb.F32, [D, H, N_Q, 1], [4, D * 4, H * D * 4, N_Q * H * D * 4])
            for l in range(LAYERS)]
    overlap = world == 1 or (xchg is not None and args.exchange == "kernel")
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_step(st):
        cs = torch.cuda.ExternalStream(st.value, device=dev) if st.value else torch.cuda.current_stream(dev)
        if not overlap:
            with torch.cuda.stream(cs):
                for l in range(LAYERS):
                    q_dev[l].copy_(q_host[l], non_blocking=True)
                    layer_call(l, st, q_ts[l], o_ts[l])
                    o_host[l].copy_(o_dev[l], non_blocking=True)
            return
        ev_in = [torch.cuda.Event() for _ in range(LAYERS)]
        ev_out = [torch.cuda.Event() for _ in range(LAYERS)]
        h2d_s.wait_stream(cs)
        d2h_s.wait_stream(cs)
        with torch.cuda.stream(h2d_s):
            for l in range(LAYERS):
                q_dev[l].copy_(q_host[l], non_blocking=True)
                ev_in[l].record(h2d_s)
        for l in range(LAYERS):
            cs.wait_event(ev_in[l])
            layer_call(l, st, q_ts[l], o_ts[l])
            ev_out[l].record(cs)
            d2h_s.wait_event(ev_out[l])
            with torch.cuda.stream(d2h_s):
                o_host[l].copy_(o_dev[l], non_blocking=True)
        cs.wait_stream(d2h_s)

    for _ in range(max(1, args.warmup)):
        e2e_step(st)
    torch.cuda.synchronize()
    run_e2e = graphed(e2e_step)
    run_e2e()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    f0.record(stream)
    for _ in range(args.steps):
        run_e2e()
    f1.record(stream)
    torch.cuda.synchronize()
    t_wall = time.perf_counter() - t_wall
    e2e_ms = max(f0.elapsed_time(f1), t_wall * 1e3)

    # secondary: the same verify step over q8_0 and q4_0 caches (config[3]'s other variant; klein's type beyond
    # 131K cells)
    secondary = {}
    if not args.no_secondary:
        for kvt in ("q8_0", "q4_0"):
            graphs.clear()  # the previous graphs refer to the cache about to be freed
            del layers[:]
            torch.cuda.empty_cache()
            layers.extend(make_layers(kb, torch, dev, gen, n_kv, kvt))
            # the quantised kernels plan their own row chunks and splits: size the scratch for them
            need = L.kb_flash_attn_ext_scratch_bytes(ctypes.byref(qt), ctypes.byref(layers[0][2]),
                                                     ctypes.byref(layers[0][3]), ctypes.byref(prm))
            if world > 1:
                need = max(need, L.kb_flash_attn_ext_push_scratch_bytes(ctypes.byref(qt), ctypes.byref(layers[0][2]),
                                                                        ctypes.byref(layers[0][3]), ctypes.byref(prm)))
            del scratch
            scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
            sp = ctypes.c_void_p(scratch.data_ptr())
            for _ in range(args.warmup):
                step(st)
            torch.cuda.synchronize()
            run_q = graphed(step)  # a new capture: the earlier graphs refer to freed caches
            run_q()
            torch.cuda.synchronize()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            for _ in range(args.steps):
                run_q()
            g1.record(stream)
            torch.cuda.synchronize()
            qms = g0.elapsed_time(g1)
            if world > 1:
                t = torch.tensor([qms], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                qms = float(t.item())
            q_us = qms * 1e3 / (args.steps * LAYERS)
            qbytes = kv_bytes_per_layer(n_kv, kvt)
            pk, _ = measured_peaks()
            secondary["verify_" + kvt] = {
                "value": round(q_us, 2), "unit": UNIT, "kv_type": kvt,
                "roofline": {"bound": "hbm", "achieved": round(qbytes / (q_us * 1e-6) / 1e9, 1), "peak": pk["hbm_gbs"],
                             "unit": "GB/s", "frac": round(qbytes / (q_us * 1e-6) / 1e9 / pk["hbm_gbs"], 4),
                             "algorithmic_bytes_per_launch": qbytes,
                             # ncu DRAM bytes of one full-cache launch; a rank of an N-way split streams 1/N of it
                             "traffic": (lambda t: None if t is None else int(t / world))(
                                 ncu_traffic(f"fa_stream_{kvt}_verify262k"))}}

    if not args.no_secondary and world > 1:
        graphs.clear()
        del layers[:]
        torch.cuda.empty_cache()
        secondary.update(bench_head_shards(kb, torch, dev, args.steps, args.warmup, rank, world, dist))

    peaks, peak_kind = measured_peaks()
    bytes_layer = kv_bytes_per_layer(n_kv, "f16")
    achieved = bytes_layer / (us_per_layer * 1e-6) / 1e9
    line = {
        "metric": METRIC, "value": round(us_per_layer, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "config[3] long verify: 4 query tokens per layer, causal among the last 4, "
                               "262144-cell f16 KV cache (4 KV heads x 256), 24 Q heads, 16 layers per step",
                   "n_kv": N_KV, "kv_type": "f16", "layers_per_step": LAYERS,
                   "parallelism": f"kv-split{world}-{args.exchange}" if world > 1 else "single",
                   "l2": "inputs larger than L2: each layer streams 1.07 GB of KV"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_kind": peak_kind,
                     # ncu DRAM bytes of one full-cache launch; a rank of an N-way split streams 1/N of the cells
                     "traffic": (lambda t: None if t is None else int(t / world))(ncu_traffic("fa_stream_f16_verify262k")),
                     "algorithmic_bytes_per_launch": bytes_layer},
        "gpu_launches": launches,
        "parity": parity,
        "e2e": {"value": round(e2e_ms * 1e3 / (args.steps * LAYERS), 2), "unit": UNIT,
                "h2d_bytes_per_step": LAYERS * N_Q * H * D * 4, "d2h_bytes_per_step": LAYERS * N_Q * H * D * 4},
        "clocks": clk.summary(),
    }
    if not args.no_secondary and world == 1:
        graphs.clear()  # the f16 graphs refer to the cache about to be freed
        del layers[:]
        torch.cuda.empty_cache()
        secondary["prefill_bf16_4096"] = bench_prefill(kb, torch, dev, max(3, args.steps // 20), args.warmup)
        secondary["prefill_q8_0_2048"] = bench_prefill(kb, torch, dev, max(3, args.steps // 20), args.warmup,
                                                       kv="q8_0", T=2048, n_kv=4096)
        secondary["gdn_verify"] = bench_gdn(kb, torch, dev, max(3, args.steps // 20), args.warmup)
        secondary.update(bench_gdn_layer(kb, torch, dev, max(3, args.steps // 20), args.warmup))
        secondary.update(bench_dense_mask(kb, torch, dev, max(3, args.steps // 20), args.warmup))
        secondary["gdn_prefill_4096"] = bench_gdn_prefill(kb, torch, dev, max(3, args.steps // 20), args.warmup)
        secondary["io_ops"] = bench_io_ops(kb, torch, dev, max(20, args.steps // 2), args.warmup)
        if not args.no_stack:
            secondary["stack_27b"] = bench_stack(kb, torch, dev, max(3, args.steps // 4), args.warmup)
    if secondary:
        line["secondary"] = secondary
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle as O

        if O.ref_available():
            threads, logical, model = host_cpu()  # one thread per physical core
            us_cpu, reps = cpu_verify_sample("f16", threads, args.cpu_budget)
            line["cpu_baseline"] = {"value": round(us_cpu, 1), "unit": UNIT, "cores": threads, "kind": "reference",
                                    "logical_cpus": logical, "cpu_model": model,
                                    "sample": f"{reps} single layers of the headline workload (ggml CPU flash_attn_ext, "
                                              f"262144 f16 cells, 4 tokens), median, {threads} threads"}
        else:
            line["cpu_baseline"] = None
    if rank == 0:
        print(json.dumps(line), flush=True)
    graphs.clear()  # graphs that hold collective calls go before the process group
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()  # every rank's last exchange has landed before peer buffers go away
        if xchg is not None:
            xchg.close()
        dist.barrier()
        dist.destroy_process_group()


def run_case(case: str):
    """One small, untimed invocation of a workload for profiler captures: three calls of the same operation
    (capture the third with ncu -s <2 x kernels per call> -c <kernels per call>)."""
    import numpy as np
    import torch

    import klein_b200 as kb

    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(1)
    if case == "prefill_bf16_4096":
        T = 4096
        q = torch.randn(1, T, H, D, device=dev, generator=gen).bfloat16().float()
        k = torch.randn(T, H_KV * D, device=dev, generator=gen).bfloat16()
        v = torch.randn(T, H_KV * D, device=dev, generator=gen).bfloat16()
        kv, vv = kb.kv_cache_view(k, kb.BF16, H_KV, D), kb.kv_cache_view(v, kb.BF16, H_KV, D)
        run = lambda: kb.flash_attn_ext(q, kv, vv, SCALE, causal=True, pos0=0)
    elif case == "prefill_q8_0_2048":
        T, n_kv = 2048, 4096
        q = torch.randn(1, T, H, D, device=dev, generator=gen)
        k = quantize_q8_0_rows(torch, torch.randn(n_kv, H_KV * D, device=dev, generator=gen))
        v = quantize_q8_0_rows(torch, torch.randn(n_kv, H_KV * D, device=dev, generator=gen))
        kv, vv = kb.kv_cache_view(k, kb.Q8_0, H_KV, D), kb.kv_cache_view(v, kb.Q8_0, H_KV, D)
        run = lambda: kb.flash_attn_ext(q, kv, vv, SCALE, causal=True, pos0=n_kv - T)
    elif case in ("gdn_prefill_4096", "gdn_verify"):
        T = 4096 if case == "gdn_prefill_4096" else 4
        rng = np.random.default_rng(3)
        q = rng.standard_normal((1, T, 16, 128), dtype=np.float32)
        k = rng.standard_normal((1, T, 16, 128), dtype=np.float32)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        v = rng.standard_normal((1, T, 48, 128), dtype=np.float32)
        beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((1, T, 48, 1))))).astype(np.float32)
        g = (-np.logaddexp(0.0, rng.standard_normal((1, T, 48, 1)))).astype(np.float32)
        s0 = (rng.standard_normal((1, 48, 128, 128)) * (0.0 if T > 4 else 0.02)).astype(np.float32)
        args = [torch.from_numpy(a).to(dev) for a in (q, k, v, g, beta, s0)]
        run = lambda: kb.gated_delta_net(*args, 4)
    elif case in ("verify_f16", "verify_q8_0", "verify_q4_0"):
        n_kv = 262144
        global LAYERS
        LAYERS = 1
        # keep the cache tensors (the first two entries) alive: the views only hold their pointers
        kc, vc, kv, vv = make_layers(kb, torch, dev, gen, n_kv, case[len("verify_"):])[0]
        q = torch.randn(1, 4, H, D, device=dev, generator=gen)
        run = lambda: kb.flash_attn_ext(q, kv, vv, SCALE, causal=True, pos0=n_kv - 4)
    elif case in ("verify_f16_dense_mask", "prefill_bf16_2048_dense_mask"):
        # klein's dense f16 mask instead of the analytic bounds (0 at or before the row's position, -inf after)
        T, n_kv = (4, 262144) if case.startswith("verify") else (2048, 4096)
        bf = case.startswith("prefill")
        k = torch.randn(n_kv, H_KV * D, device=dev, generator=gen)
        v = torch.randn(n_kv, H_KV * D, device=dev, generator=gen)
        k, v = (k.bfloat16(), v.bfloat16()) if bf else (k.half(), v.half())
        t = kb.BF16 if bf else kb.F16
        kv, vv = kb.kv_cache_view(k, t, H_KV, D), kb.kv_cache_view(v, t, H_KV, D)
        q = torch.randn(1, T, H, D, device=dev, generator=gen)
        if bf:
            q = q.bfloat16().float()
        c = torch.arange(n_kv, device=dev)[None, :]
        pos = n_kv - T + torch.arange(T, device=dev)[:, None]
        mask = torch.where(c <= pos, 0.0, float("-inf")).half()
        run = lambda: kb.flash_attn_ext(q, kv, vv, SCALE, mask=mask)
    elif case in ("gdn_step_1", "gdn_step_4"):
        # one DeltaNet layer of the decode / verify step in one launch (kb_gdn_step), K = 4 f16 snapshots
        T, S, Hk, Hv = int(case[-1]), 128, 16, 48
        ch = 2 * S * Hk + S * Hv
        conv = torch.randn(4, 3 * ch, device=dev, generator=gen)
        ssm = torch.randn(1, Hv, S, S, device=dev, generator=gen) * 0.02
        snap = torch.zeros(3, S * S * Hv, dtype=torch.float16, device=dev)
        cw = torch.randn(ch, 4, device=dev, generator=gen) * 0.5
        qkv, z = torch.randn(T, ch, device=dev, generator=gen), torch.randn(T, Hv * S, device=dev, generator=gen)
        br, al = torch.randn(T, Hv, device=dev, generator=gen), torch.randn(T, Hv, device=dev, generator=gen)
        dt, aa = torch.randn(Hv, device=dev, generator=gen), -torch.rand(Hv, device=dev, generator=gen) - 0.1
        nw, sync = torch.ones(S, device=dev), torch.zeros(Hk, dtype=torch.int32, device=dev)
        run = lambda: kb.gdn_step(qkv, conv, cw, br, al, dt, aa, ssm, snap, 4, z, nw, 1e-6, sync)
    elif case == "gdn_input_4096":
        # the DeltaNet input side at config[2]'s 4,096 tokens (qwen35: 16 key / 48 value heads, S 128)
        T, S, Hk, Hv = 4096, 128, 16, 48
        ch = 2 * S * Hk + S * Hv
        qkv = torch.randn(T, ch, device=dev, generator=gen)
        state = torch.randn(4, 3 * ch, device=dev, generator=gen)
        cw = torch.randn(ch, 4, device=dev, generator=gen) * 0.5
        br, al = torch.randn(T, Hv, device=dev, generator=gen), torch.randn(T, Hv, device=dev, generator=gen)
        dt, aa = torch.randn(Hv, device=dev, generator=gen), -torch.rand(Hv, device=dev, generator=gen) - 0.1
        run = lambda: kb.gdn_input(qkv, state, cw, S, Hk, 1e-6, beta_raw=br, alpha=al, dt_bias=dt, a=aa)[0]
    else:
        raise SystemExit(f"unknown case {case}")
    for _ in range(3):
        out = run()
    torch.cuda.synchronize()
    print(case, "ok", float(out.float().abs().sum()))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kb", choices=["kb", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU timing for cpu_baseline")
    ap.add_argument("--layers", type=int, default=16, help="full-attention layers per step (16 = the headline)")
    ap.add_argument("--no-secondary", action="store_true", help="skip the secondary measurements (q8_0 / q4_0 caches, prefill, DeltaNet, I/O ops)")
    ap.add_argument("--no-stack", action="store_true", help="skip the whole-stack (config[4]) secondary")
    ap.add_argument("--stack-only", action="store_true", help="run only the whole-stack (config[4]) measurement")
    ap.add_argument("--eager", action="store_true", help="launch every layer from Python instead of a CUDA graph per step")
    ap.add_argument("--exchange", default="kernel", choices=["kernel", "p2p", "fused", "nccl"],
                    help="N > 1: the partials exchange over NVLink inside the attention kernel (kernel, default: one "
                         "launch per layer), by a push kernel after the split combine (p2p), by the split combine "
                         "itself (fused), or an NCCL all-gather")
    ap.add_argument("--case", default=None,
                    choices=["prefill_bf16_4096", "prefill_q8_0_2048", "gdn_prefill_4096", "gdn_verify", "verify_f16", "verify_q8_0",
                             "verify_q4_0", "gdn_input_4096", "gdn_step_1", "gdn_step_4", "verify_f16_dense_mask",
                             "prefill_bf16_2048_dense_mask"],
                    help="run one small untimed invocation of a workload (for profiler captures) and exit")
    args = ap.parse_args()
    if args.case:
        run_case(args.case)
        return
    if args.stack_only:
        import torch

        import klein_b200 as kb

        dev = torch.device("cuda:0")
        torch.cuda.set_device(dev)
        print(json.dumps({"stack_27b": bench_stack(kb, torch, dev, max(3, args.steps // 4), max(args.warmup, 3))}), flush=True)
        return
    global LAYERS
    LAYERS = args.layers
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_gpu(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
