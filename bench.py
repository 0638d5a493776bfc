#!/usr/bin/env python
"""Per-frame AR decode benchmark (RCuteTTS hot path on B200).

Headline workload (config[3]): batched serving, bf16 weights / fp32
accumulate, the config[2] model (12-layer Qwen3-style LM 768/12Q/4KV/d64/FFN
2048 + 32000x768 embedding, 4-layer DiT head 512/8 heads/FFN 1536, 10 Euler
steps) at 64 utterances per GPU with text lengths U[20,120], 150-frame
speaker prompts and 500 generated frames each.  Utterances are sharded over
ranks (weak scaling, no collective on the data path).  One bench step = one
latent frame for every utterance on the GPU (stop head, DiT sample, feedback
projection, LM decode step), replayed as one CUDA graph.  The timed window
sits in the middle of the 500-frame generation so the KV context is the
run's mean.  Synthetic random-init weights (N(0,0.02), seed 3) and inputs.

Also reported: the batch-1 fp32 decode step of config[2] (`b1`), the
roofline of the dominant kernel, the CPU restatement timed on the host
cores (`cpu_baseline`), the end-to-end figure through the host C-ABI call
(`e2e`), and SM clocks sampled during the timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "latent frames/s (batched AR decode step, LM+DiT)"
UNIT = "frames/s"
FRAME_HZ = 75.0  # 24 kHz / hop 320 (config[4] decoder topology)
B_PER_GPU = 64
GEN_FRAMES = 500
PROMPT_FRAMES = 150
L2_BYTES = 126 * 1024 * 1024  # fallback when the device does not report its L2 size
# DRAM bytes (read + write) of one DiT Euler-loop launch at the benchmark
# shape, from the ncu capture summarised in the file named below (ncu cannot
# run inside the timed bench; the figure is profile-derived, not measured live)
DIT_TRAFFIC_BYTES = 31.0e6
DIT_TRAFFIC_SOURCE = ("profile-derived: profiles/dit_cluster_kernel_b64.md, ncu dram__bytes_read.sum + "
                      "dram__bytes_write.sum of one launch (weights L2-resident)")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clocks and throttle reasons sampled while the timed region runs:
    NVML every ~2 ms from a host thread, with one sample taken before the
    region starts (the timed region of a short run lasts tens of ms);
    nvidia-smi -lms 200 when NVML is missing.  Reads only."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int):
        self.index = index
        self.rows = []  # (sm MHz, max sm MHz, [reason names])
        self.proc = None
        self.nv = None
        self.halt = threading.Event()

    def _nvml_handle(self, nv):
        try:  # the CUDA device's UUID names the same board for NVML
            import torch
            u = str(torch.cuda.get_device_properties(self.index).uuid)
            return nv.nvmlDeviceGetHandleByUUID(u if u.startswith("GPU-") else "GPU-" + u)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.h = self._nvml_handle(nv)
            self.nv = nv
            self.bits = [getattr(nv, "nvmlClocksEventReason" + n, 0) for n in
                         ("HwSlowdown", "HwThermalSlowdown", "SwThermalSlowdown", "SwPowerCap")]
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.rows and self.t.is_alive() and time.time() - t0 < 2.0:
                time.sleep(0.0005)
            return self
        except Exception:
            self.nv = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _poll(self):
        nv = self.nv
        while not self.halt.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                return
            self.rows.append((float(sm), float(mx), [n for n, b in zip(self.NAMES, self.bits) if b and rs & b]))
            time.sleep(0.002)

    def _read(self):
        for line in self.proc.stdout:
            r = [c.strip() for c in line.split(",")]
            if len(r) >= 9 and r[1].replace(".", "").isdigit() and r[2].replace(".", "").isdigit():
                self.rows.append((float(r[1]), float(r[2]),
                                  [n for n, v in zip(self.NAMES, r[5:9]) if v.strip().lower() == "active"]))

    def stop(self):
        if self.nv is not None:
            self.halt.set()
            self.t.join(timeout=2)
            src = "nvml"
        elif self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)
            src = "nvidia-smi"
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml and nvidia-smi unavailable"], "samples": 0}
        sm = [r[0] for r in self.rows]
        mx = [r[1] for r in self.rows]
        reasons = sorted({n for r in self.rows for n in r[2]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm), "source": src}


# ----------------------------------------------------------------- workload
def make_models(dtype: str, seed: int, device: int):
    from rcutetts_b200 import synth
    from rcutetts_b200.config import DiTConfig, LMConfig
    from rcutetts_b200.model import DitW, QwenW

    lcfg, dcfg = LMConfig(), DiTConfig()
    lw = synth.lm_weights(lcfg, seed=seed, with_embed=True)
    dw = synth.dit_weights(dcfg, seed=seed + 10)
    hw = synth.frame_weights(lcfg.hidden, dcfg.latent, seed=seed + 20)
    lm = QwenW(lcfg, dtype, device).set_weights(lw)
    dit = DitW(dcfg, dtype, device).set_weights(dw)
    return lcfg, dcfg, lw, dw, hw, lm, dit


def utterances(n_total: int, seed: int, vocab: int):
    rng = np.random.default_rng(seed)
    lens = rng.integers(20, 121, n_total)
    return [(rng.integers(0, vocab, lens[u]), rng.standard_normal((PROMPT_FRAMES, 64), dtype=np.float32))
            for u in range(n_total)]


def shard(n_total: int, rank: int, world: int):
    """Contiguous utterance shard of this rank (utterances are independent:
    no collective on the data path)."""
    per = n_total // world
    return range(rank * per, (rank + 1) * per)


def rank_workload(rank: int, world: int, vocab: int, seed: int = 3):
    """The utterances (text ids, prompt latents) rank `rank` decodes: its
    contiguous shard of the B_PER_GPU * world utterances of the seeded
    batch, in batch order (every rank draws the same batch, so no data moves
    between ranks)."""
    allu = utterances(B_PER_GPU * world, seed=seed, vocab=vocab)
    return [allu[i] for i in shard(B_PER_GPU * world, rank, world)]


def max_over_ranks(values, world: int, device=None):
    """Element-wise max of per-rank timings (the slowest rank defines the
    job's time).  torch.distributed plumbing only."""
    if world <= 1:
        return list(values)
    import torch

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]


def prefix_rows(lm, hw, ids, prompt):
    emb = lm.embed_lookup(ids)
    pr = prompt @ hw["latent_proj.weight"].T + hw["latent_proj.bias"]
    return np.concatenate([emb, pr.astype(np.float32)], 0)


def algorithmic_bytes_per_step(lcfg, dcfg, B, ctx_mean, wbytes, kvbytes, steps=10):
    """Bytes one frame step must move (the reference's own traffic model,
    PERF_PLAN.md:39-50: each weight byte once per pass that streams it, plus
    the KV cache read)."""
    H, F, L = lcfg.hidden, lcfg.ffn, lcfg.n_layers
    lm_params = L * (H * (lcfg.q_dim + 2 * lcfg.kv_dim) + H * lcfg.q_dim + 3 * H * F)
    Hd, Fd, Ld = dcfg.hidden, dcfg.ffn, dcfg.n_layers
    dit_step = Ld * (4 * Hd * Hd + 3 * Hd * Fd) + 2 * Hd * Hd + 2 * Hd * 64 + 64 * Hd
    once = Ld * 6 * Hd * dcfg.spk_dim + Hd * dcfg.cond_dim + 2 * Hd * Hd + H * 64 + 2 * H
    kv = 2 * L * lcfg.kv_dim * ctx_mean * kvbytes * B
    return (lm_params + steps * dit_step + once) * wbytes + kv


# ------------------------------------------------------------- our arm
def run_ours(args, rank, world, local):
    import torch

    from rcutetts_b200.model import FrameEngine

    torch.cuda.set_device(local)
    dev = local
    hbm, bf16_tf, peak_kind = peaks()
    lcfg, dcfg, lw, dw, hw, lm, dit = make_models("bf16", seed=3, device=dev)
    B = B_PER_GPU
    utts = rank_workload(rank, world, lcfg.vocab)
    K, W = args.steps, args.warmup
    # timed frames end near the middle of the run unless a start frame is given
    start = args.start_frame if args.start_frame >= 0 else max(0, GEN_FRAMES // 2 - W - K)
    total = start + W + 2 * K + 2
    max_prefix = max(len(ids) for ids, _ in utts) + PROMPT_FRAMES
    cap = max_prefix + max(total, GEN_FRAMES) + 16
    eng = FrameEngine(lm, dit, hw, batch=B, capacity=cap, euler_steps=10, groups=args.groups)
    ctx0 = []
    for b, (ids, prompt) in enumerate(utts):
        rows = prefix_rows(lm, hw, ids, prompt)
        ctx0.append(rows.shape[0])
        eng.prefill(b, rows, prompt[-1])
    # everything runs on the engine's own stream; events are recorded there
    stream = torch.cuda.ExternalStream(eng.stream_ptr)
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    noise = torch.randn((total, B, 64), device="cuda", generator=g)
    lat = torch.empty((total, B, 64), device="cuda")
    torch.cuda.synchronize()
    for f in range(start):
        eng.step_dev(noise[f], lat[f], None)
    for f in range(start, start + W):
        eng.step_dev(noise[f], lat[f], None)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(dev).start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()  # profiler window = the timed frames (ncu --profile-from-start off)
    e0.record(stream)
    for f in range(start + W, start + W + K):
        eng.step_dev(noise[f], lat[f], None)
    e1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    clocks = clk.stop()
    ms = e0.elapsed_time(e1)
    # e2e: the host C-ABI call (pinned H2D of the step's noise, graph replay,
    # D2H of the latents and stop logits, sync) -- ctts_engine_step.
    noise_h = noise[start + W + K:start + W + 2 * K].cpu().numpy()
    es = torch.cuda.ExternalStream(eng.stream_ptr)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(es)
    for k in range(K):
        eng.step(noise_h[k])
    x1.record(es)
    torch.cuda.synchronize()
    ms_e2e = x0.elapsed_time(x1)
    ms, ms_e2e = max_over_ranks([ms, ms_e2e], world, device="cuda")
    phases = profile_phases(eng, noise[start + W:start + W + 10], lat[start + W:start + W + 10])
    launches = eng.launches_per_step
    ctx_mean = float(np.mean(ctx0)) + start + W + K / 2
    step_bytes = algorithmic_bytes_per_step(lcfg, dcfg, B, ctx_mean, 2, 2)
    res = {
        "ms": ms, "ms_e2e": ms_e2e, "launches": launches, "clocks": clocks, "ctx_mean": ctx_mean,
        "step_bytes": step_bytes, "start": start, "peak": (hbm, bf16_tf, peak_kind),
        "finite": bool(torch.isfinite(lat[:start + W + K]).all().item()), "phases": phases,
    }
    del eng
    return res, (lm, dit, lcfg, dcfg, hw)


def profile_phases(eng, noise, lat):
    """Per-phase device times of a few extra frames in the engine's
    profiling mode (the --profile-steps timers of bin/cutetts.rs:328-350):
    eager frames with CUDA events between the stop head, DiT sample,
    feedback projection and LM step (no graph replay, so the phases add up
    to more than a replayed frame)."""
    eng.set_profile(True)
    for f in range(noise.shape[0]):
        eng.step_dev(noise[f], lat[f], None)
    st = eng.profile_stats()
    eng.set_profile(False)
    return {k: {"p50_ms": round(v["p50_ms"], 4), "p99_ms": round(v["p99_ms"], 4), "n": v["n"]} for k, v in st.items()}


def run_b1(args, dev):
    """config[2]: batch 1, fp32, 200 frames; one step = one frame."""
    import torch

    from rcutetts_b200.model import FrameEngine

    lcfg, dcfg, lw, dw, hw, lm, dit = make_models("f32", seed=2, device=dev)
    rng = np.random.default_rng(2)
    ids = rng.integers(0, lcfg.vocab, 40)
    prompt = rng.standard_normal((PROMPT_FRAMES, 64), dtype=np.float32)
    eng = FrameEngine(lm, dit, hw, batch=1, capacity=40 + PROMPT_FRAMES + 210, euler_steps=10)
    eng.prefill(0, prefix_rows(lm, hw, ids, prompt), prompt[-1])
    frames = 200
    noise = torch.from_numpy(rng.standard_normal((frames, 1, 64), dtype=np.float32)).cuda()
    lat = torch.empty_like(noise)
    stream = torch.cuda.ExternalStream(eng.stream_ptr)
    torch.cuda.synchronize()
    W = 3
    for f in range(W):
        eng.step_dev(noise[f], lat[f], None)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()
    e0.record(stream)
    for f in range(W, W + args.b1_frames):
        eng.step_dev(noise[f], lat[f], None)
    e1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1) / args.b1_frames
    # five more frames in the profiling mode (the cache has 210 rows past
    # the prefix; noise rows are reused)
    phases = profile_phases(eng, noise[:5], lat[:5])
    ctx_mean = 40 + PROMPT_FRAMES + frames / 2
    step_bytes = algorithmic_bytes_per_step(lcfg, dcfg, 1, ctx_mean, 4, 4)
    hbm, _, kind = peaks()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    out = {"config": "config[2] B=1 fp32, 40 text + 150 prompt rows, 200 frames",
           "us_per_step": round(ms * 1e3, 2), "frames_per_s": round(1e3 / ms, 2),
           "rtf": round((ms * 1e-3) * FRAME_HZ, 4),
           "step_roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(gbs / hbm, 4), "bytes_per_step": int(step_bytes),
                             "of": kind},
           "launches_per_step": eng.launches_per_step, "phases": phases}
    del eng
    return out


def dit_kernel_roofline(dit, dcfg, lcfg, dev, tc_probe=None):
    """Roofline of the dominant kernel of the batched frame: the DiT head's
    cluster-resident Euler loop (dit_cluster_kernel, about 60% of the frame
    in the ncu launch list), run alone through ctts_dit_euler_sample_dev at
    the benchmark's 64 utterances x 10 Euler steps, timed with CUDA events
    on the launching stream.  The timed call also holds the once-per-frame
    prologue (AdaLN, cond/mu projections, time embeddings: 6 small
    launches).  Algorithmic flops = 2 x 192 token rows x the DiT layer
    parameters x 10 steps + the prologue GEMMs; its weights are
    L2-resident, so the bound is the tensor pipe (measured bf16 peak, burst)."""
    import ctypes as C

    import torch

    from rcutetts_b200 import _lib

    lib = _lib.load()
    hbm, bf16_tf, kind = peaks()
    B, steps = B_PER_GPU, 10
    g = torch.Generator(device="cuda").manual_seed(7)
    x0 = torch.randn((B, dcfg.latent), device="cuda", generator=g)
    z = torch.randn((B, lcfg.hidden), device="cuda", generator=g)
    cond = torch.randn((B, dcfg.latent), device="cuda", generator=g)
    out = torch.empty((B, dcfg.latent), device="cuda")
    # a stream of our own: a null stream handle would select the head's
    # internal stream, which the events below would not see
    st = torch.cuda.Stream()
    torch.cuda.synchronize()

    def call():
        rc = lib.ctts_dit_euler_sample_dev(dit.h, B, x0.data_ptr(), z.data_ptr(), cond.data_ptr(), z.data_ptr(),
                                           steps, C.c_float(0.0), out.data_ptr(), st.cuda_stream)
        assert rc == 0, lib.ctts_last_error()

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    n = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(n):
        call()
    e1.record(st)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / n * 1e-3
    Hd, Fd, L = dcfg.hidden, dcfg.ffn, dcfg.n_layers
    layer_params = L * (4 * Hd * Hd + 3 * Hd * Fd)
    flops = 2 * 3 * B * layer_params * steps + 2 * B * (L * 6 * Hd * dcfg.spk_dim + Hd * dcfg.cond_dim)
    tf = flops / t / 1e12
    res = {"bound": "tensor", "achieved": round(tf, 2), "peak": bf16_tf, "unit": "TFLOP/s",
           "frac": round(tf / bf16_tf, 4), "traffic": DIT_TRAFFIC_BYTES, "of": kind,
           "kernel": "dit_cluster_kernel (tcgen05, 16-CTA clusters) + DiT prologue via ctts_dit_euler_sample_dev, "
                     "64 utterances x 10 Euler steps",
           "flops_per_launch": flops, "us_per_launch": round(t * 1e6, 2),
           "traffic_source": DIT_TRAFFIC_SOURCE}
    if tc_probe is not None:
        res["others"] = tc_probe
    return res


def dominant_kernel_roofline(lm, dit, lcfg, dcfg, dev):
    """Average device time of the LM's tensor-core linear (tc_linear_kernel,
    the second kernel class of the batched frame), replayed alone through
    ctts_op_linear with CUDA events on the launching stream: the LM down and
    gate/up shapes of the batched step (M = 64 rows, bf16 weights streamed
    from HBM; L2 flushed between launches).  Algorithmic bytes = weights +
    activation in + output out."""
    import ctypes as C

    import torch

    from rcutetts_b200 import _lib, synth

    lib = _lib.load()
    hbm, _, kind = peaks()
    out = {}
    for name, M, K, N in (("lm_down", 64, 2048, 768), ("lm_gate_up", 64, 768, 4096)):
        rng = np.random.default_rng(0)
        W = synth.to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * 0.02).view(np.int16)
        wdev = torch.from_numpy(W).cuda()
        x = torch.randn(M, K, device="cuda")
        g = torch.ones(K, device="cuda")
        y = torch.empty(M, N, device="cuda")
        flush = torch.empty(2 * l2_bytes() // 4, device="cuda")
        st = torch.cuda.current_stream()
        times = []
        torch.cuda.profiler.start()
        for it in range(23):
            flush.add_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            rc = lib.ctts_op_linear(x.data_ptr(), M, K, wdev.data_ptr(), 1, N, g.data_ptr(), C.c_float(1e-6),
                                    None, y.data_ptr(), st.cuda_stream)
            e1.record(st)
            assert rc == 0
            torch.cuda.synchronize()
            if it >= 3:
                times.append(e0.elapsed_time(e1))
        torch.cuda.profiler.stop()
        t = statistics.mean(times) * 1e-3
        algo = N * K * 2 + M * K * 4 + M * N * 4
        out[name] = {"us": round(t * 1e6, 2), "bytes": algo, "gbs": algo / t / 1e9}
    d = out["lm_gate_up"]
    return {"bound": "hbm", "achieved": round(d["gbs"], 1), "peak": hbm, "unit": "GB/s",
            "frac": round(d["gbs"] / hbm, 4), "traffic": None, "of": kind,
            "kernel": "tc_linear_kernel (tcgen05, bf16) via ctts_op_linear: LM gate/up shape M=64 K=768 N=4096, L2 flushed",
            "bytes_per_launch": d["bytes"], "us_per_launch": d["us"],
            "others": {k: {"us": v["us"], "gbs": round(v["gbs"], 1)} for k, v in out.items()}}


# ------------------------------------------- config[0], config[1], config[4]
def dev_time(fn, n, stream, flush=None):
    """Mean device time in seconds of fn() over n calls, each bracketed by
    CUDA events on `stream` (the stream fn launches on); with `flush`, a
    buffer larger than L2 is rewritten before every call."""
    import torch

    ts = []
    for _ in range(n):
        if flush is not None:
            flush.add_(1.0)
            torch.cuda.synchronize()  # the flush (torch's stream) ends before the timed call starts
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e-3)
    return statistics.mean(ts)


def l2_bytes():
    import torch

    return int(getattr(torch.cuda.get_device_properties(torch.cuda.current_device()), "L2_cache_size", L2_BYTES))


def bench_c0(dev):
    """config[0]: one fp32 decoder layer at batch 1 -- a 64-row prefill, then
    32 single-token decode steps against the growing cache, each timed on the
    device (us per layer step; weights 25.2 MB fp32 streamed per step).  The
    CPU restatement times the same decode steps beside it."""
    import torch

    from oracle import oracle as orc
    from rcutetts_b200 import synth
    from rcutetts_b200.config import LMConfig
    from rcutetts_b200.model import QwenCache, QwenW, decode_step_dev, prefill

    cfg = LMConfig(n_layers=1)
    w = synth.lm_weights(cfg, seed=0)
    m = QwenW(cfg, "f32", dev).set_weights(w)
    rng = np.random.default_rng(0)
    xp = rng.standard_normal((64, cfg.hidden), dtype=np.float32)
    xd = rng.standard_normal((32, cfg.hidden), dtype=np.float32)
    cache = QwenCache(m, batch=1, capacity=128)
    prefill(m, xp, cache)
    xdd = torch.from_numpy(xd).cuda()
    out = torch.empty_like(xdd)
    st = torch.cuda.Stream()
    torch.cuda.synchronize()
    flush = torch.empty(2 * l2_bytes() // 4, device="cuda")
    ts = []
    for i in range(32):
        ts.append(dev_time(lambda: decode_step_dev(m, xdd[i:i + 1], cache, out[i:i + 1], st), 1, st, flush))
    us = statistics.median(ts) * 1e6
    wbytes = 4 * (cfg.hidden * (cfg.q_dim + 2 * cfg.kv_dim) + cfg.hidden * cfg.q_dim + 3 * cfg.hidden * cfg.ffn)
    kv = 2 * cfg.kv_dim * 4 * (64 + 16)
    hbm, _, kind = peaks()
    lm_o = orc.LM(cfg, w)
    oc = lm_o.new_cache(128)
    lm_o.forward(xp, oc)
    cts = []
    for i in range(32):
        t0 = time.perf_counter()
        lm_o.forward(xd[i:i + 1], oc)
        cts.append(time.perf_counter() - t0)
    gbs = (wbytes + kv) / (us * 1e-6) / 1e9
    return {"workload": "config[0]: one fp32 Qwen3 layer (768, 12/4 heads, FFN 2048), batch 1, 64-row prefill + "
                        "32 decode steps, L2 flushed before each step",
            "us_per_layer_step": round(us, 2), "gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4), "of": kind,
            "bytes_per_step": wbytes + kv,
            "cpu_us_per_layer_step": round(statistics.median(cts) * 1e6, 1), "cpu_cores": orc.get_threads()}


def bench_c1(dev):
    """config[1]: y = RMSNorm(x) W^T + residual through ctts_op_linear at
    every (M, K, N, dtype) point, L2 flushed before every launch (device
    time, CUDA events on the launching stream), the CPU restatement beside
    each point; plus RoPE on [256, 12, 64] at positions 0..255 + the 4096
    sweep, SwiGLU on [256, 2x2048] and the 32000x768 embedding gather."""
    import ctypes as C

    import torch

    from oracle import oracle as orc
    from rcutetts_b200 import _lib, synth

    lib = _lib.load()
    hbm, _, kind = peaks()
    st = torch.cuda.current_stream()
    flush = torch.empty(2 * l2_bytes() // 4, device="cuda")
    rows = []
    rng = np.random.default_rng(1)
    for dtype in ("f32", "bf16"):
        for K, N in ((768, 768), (768, 2048), (2048, 768), (768, 2304)):
            W = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
            if dtype == "bf16":
                W = synth.bf16_round(W)
                wd = torch.from_numpy(synth.to_bf16_bits(W).view(np.int16)).cuda()
            else:
                wd = torch.from_numpy(W).cuda()
            g = torch.ones(K, device="cuda")
            for M in (1, 8, 64, 256):
                x = rng.standard_normal((M, K), dtype=np.float32)
                res = rng.standard_normal((M, N), dtype=np.float32)
                xd, rd = torch.from_numpy(x).cuda(), torch.from_numpy(res).cuda()
                y = torch.empty((M, N), device="cuda")

                def call():
                    rc = lib.ctts_op_linear(xd.data_ptr(), M, K, wd.data_ptr(), 1 if dtype == "bf16" else 0, N,
                                            g.data_ptr(), C.c_float(1e-6), rd.data_ptr(), y.data_ptr(),
                                            st.cuda_stream)
                    assert rc == 0, lib.ctts_last_error()

                for _ in range(3):
                    call()
                t = dev_time(call, 10, st, flush)
                algo = N * K * (2 if dtype == "bf16" else 4) + M * K * 4 + 2 * M * N * 4
                t0 = time.perf_counter()
                orc.linear(orc.rms_norm(x, np.ones(K, np.float32), 1e-6), W)
                ct = time.perf_counter() - t0
                rows.append({"M": M, "K": K, "N": N, "dtype": dtype, "us": round(t * 1e6, 2),
                             "gbs": round(algo / t / 1e9, 1), "hbm_frac": round(algo / t / 1e9 / hbm, 4),
                             "cpu_us": round(ct * 1e6, 1)})
    out = {"workload": "config[1] op sweep: RMSNorm + linear + residual, M x (K,N) x {fp32, bf16 weights}, "
                       "L2 flushed before every launch", "of": kind, "linear": rows}
    # RoPE over positions 0..4095, SwiGLU, embedding gather
    M = 4096
    xr = torch.randn((M, 12, 64), device="cuda")
    pos = torch.arange(M, dtype=torch.int32, device="cuda")
    t = dev_time(lambda: lib.ctts_op_rope(xr.data_ptr(), M, 12, 64, pos.data_ptr(), C.c_float(1e6),
                                          st.cuda_stream), 10, st, flush)
    out["rope"] = {"shape": "[4096, 12, 64], positions 0..4095", "us": round(t * 1e6, 2),
                   "gbs": round(2 * xr.numel() * 4 / t / 1e9, 1)}
    gu = torch.randn((256, 4096), device="cuda")
    so = torch.empty((256, 2048), device="cuda")
    t = dev_time(lambda: lib.ctts_op_swiglu(gu.data_ptr(), 256, 2048, so.data_ptr(), st.cuda_stream), 10, st, flush)
    out["swiglu"] = {"shape": "[256, 2x2048]", "us": round(t * 1e6, 2),
                     "gbs": round((gu.numel() + so.numel()) * 4 / t / 1e9, 1)}
    table = torch.randn((32000, 768), device="cuda")
    ids = torch.from_numpy(rng.integers(0, 32000, 256)).cuda()
    eo = torch.empty((256, 768), device="cuda")
    t = dev_time(lambda: lib.ctts_op_embed_gather(table.data_ptr(), 32000, 768, ids.data_ptr(), 256, eo.data_ptr(),
                                                  None, st.cuda_stream), 10, st, flush)
    out["embed_gather"] = {"shape": "32000x768 table, 256 uniform ids", "us": round(t * 1e6, 2),
                           "gbs": round(2 * eo.numel() * 4 / t / 1e9, 1)}
    return out


def vae_flops(cfg, T):
    """Dense conv flops of one utterance through the config[4] decoder."""
    C, L = cfg.channels, cfg.latent
    f = 2 * C * L * 7 * T
    t = T
    for si, s in enumerate(cfg.strides):
        cin, cout = C >> si, C >> (si + 1)
        f += 2 * cout * cin * 2 * t * s  # transposed conv: 2 taps per output sample
        t *= s
        f += 3 * (2 * cout * cout * 7 * t + 2 * cout * cout * t)
    f += 2 * (C >> len(cfg.strides)) * 7 * t
    return f


def bench_c4(dev, cpu=True, B=32, T=400, dtypes=("bf16", "f32")):
    """config[4]: the causal VAE decoder on latents [32, 64, 400] (bf16 on the
    tensor cores, fp32 on the CUDA cores), ms per batch with CUDA events, RTF
    against the 170.7 s of audio, TFLOP/s; the CPU restatement decodes one
    utterance of the batch (extrapolated to 32, stated as such).  Protocol of
    decode_bench.rs:41-72: warm-up, then repeated timed decodes."""
    import torch

    from oracle import oracle as orc
    from rcutetts_b200 import synth
    from rcutetts_b200.config import VAEConfig
    from rcutetts_b200.model import DecoderW

    cfg = VAEConfig()
    w = synth.vae_weights(cfg, seed=4)
    lat = torch.randn((B, cfg.latent, T), device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    wav = torch.empty((B, T * cfg.hop), device="cuda")
    audio_s = B * T * cfg.hop / 24000.0
    flops = vae_flops(cfg, T) * B
    _, bf16_tf, kind = peaks()
    out = {"workload": f"config[4]: causal VAE decoder, latents [{B}, 64, {T}] -> {B} x {T * cfg.hop} samples",
           "flops_per_batch": flops, "audio_s": audio_s}
    for dtype, n in (("bf16", 5), ("f32", 2)):
        if dtype not in dtypes:
            continue
        m = DecoderW(cfg, dtype, dev).set_weights(w)
        st = torch.cuda.Stream()
        m.decode_dev(lat, wav, st)
        torch.cuda.synchronize()
        t = dev_time(lambda: m.decode_dev(lat, wav, st), n, st)
        tf = flops / t / 1e12
        row = {"ms_per_batch": round(t * 1e3, 2), "rtf": round(t / audio_s, 6), "tflops": round(tf, 1)}
        if dtype == "bf16":
            row.update({"tensor_frac": round(tf / bf16_tf, 4), "of": kind,
                        "kernel": "vae_tc_conv_kernel (tcgen05) for every dense conv; final 64->1 conv on CUDA cores"})
        else:
            row["kernel"] = "conv_kernel (CUDA-core FFMA, fp32 weights)"
        out[dtype] = row
        del m
    if cpu:
        o = orc.VAE(cfg, w)
        one = lat[0].cpu().numpy()
        t0 = time.perf_counter()
        o.decode(one)
        ct = time.perf_counter() - t0
        out["cpu"] = {"s_per_utterance": round(ct, 3), "ms_per_batch_extrapolated": round(ct * B * 1e3, 1),
                      "rtf": round(ct * B / audio_s, 4), "cores": orc.get_threads(),
                      "sample": f"one utterance of the batch (T={T}, fp32) decoded by the CPU restatement; "
                                f"batch time extrapolated x{B}"}
    return out


# -------------------------------------------------------------- CPU side
class CpuRef:
    """The oracle (C restatement of the reference CPU path) on the host
    cores, on config[3]'s own workload: utterances 0..n-1 of the benchmark
    batch (bf16-rounded weights widened to fp32, as the reference loads bf16
    checkpoints), each prefilled untimed with its text + prompt rows and
    `ctx_frames` feedback rows so the KV context matches the GPU's timed
    window.  The reference decodes one utterance at a time (decode_step is
    batch-1, qwen.rs:395-397), so a batch is advanced round-robin, one frame
    of one utterance per iteration; run() advances frames for a time budget
    and returns (frames, seconds)."""

    def __init__(self, threads: int | None = None, n_utts: int = 4, ctx_frames: int | None = None):
        from oracle import oracle as orc
        from rcutetts_b200 import synth
        from rcutetts_b200.config import DiTConfig, LMConfig

        self.orc = orc
        self.threads = threads or os.cpu_count() or 1
        orc.set_threads(self.threads)
        lcfg, dcfg = LMConfig(), DiTConfig()
        lw = {k: synth.bf16_round(v) if v.ndim > 1 else v for k, v in synth.lm_weights(lcfg, 3).items()}
        dw = {k: synth.bf16_round(v) if v.ndim > 1 else v for k, v in synth.dit_weights(dcfg, 13).items()}
        self.hw = synth.frame_weights(lcfg.hidden, dcfg.latent, 23)
        self.lm, self.dit = orc.LM(lcfg, lw), orc.DiT(dcfg, dw)
        self.ctx_frames = GEN_FRAMES // 2 - 10 if ctx_frames is None else ctx_frames
        rng = np.random.default_rng(5)
        self.rng = rng
        self.utts = []
        for ids, prompt in utterances(B_PER_GPU, 3, lcfg.vocab)[:n_utts]:
            fb = orc.linear(rng.standard_normal((self.ctx_frames, 64), dtype=np.float32),
                            self.hw["latent_proj.weight"], self.hw["latent_proj.bias"])
            pre = np.concatenate([orc.embed_lookup(lw["embed_tokens.weight"], ids),
                                  orc.linear(prompt, self.hw["latent_proj.weight"], self.hw["latent_proj.bias"]),
                                  fb], 0)
            cache = self.lm.new_cache(pre.shape[0] + GEN_FRAMES + 8)
            z = self.lm.forward(pre, cache)[-1].copy()
            self.utts.append({"cache": cache, "z": z, "cond": prompt[-1].copy(), "frames": 0})
        self.ctx_mean = float(np.mean([u["cache"]["len"] for u in self.utts]))
        self.next = 0

    def run(self, seconds: float):
        orc, hw = self.orc, self.hw
        n = 0
        t0 = time.perf_counter()
        while True:
            u = self.utts[self.next % len(self.utts)]
            self.next += 1
            if u["frames"] >= GEN_FRAMES // 2:
                break
            orc.stop_logits(hw["stop_predictor.weight"], hw["stop_predictor.bias"], u["z"])
            x = self.dit.euler_sample(self.rng.standard_normal(64, dtype=np.float32), u["z"], u["cond"], u["z"], 10)
            u["cond"] = x
            fb = orc.linear(x[None], hw["latent_proj.weight"], hw["latent_proj.bias"])
            u["z"] = self.lm.forward(fb, u["cache"])[0].copy()
            u["frames"] += 1
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
        return n, time.perf_counter() - t0

    def describe(self, frames: int, seconds: float) -> str:
        return (f"{frames} frames in {seconds:.1f}s: config[3] utterances 0..{len(self.utts) - 1} of the batch "
                f"advanced round-robin (the reference is batch-1), KV context ~{self.ctx_mean:.0f} like the GPU's "
                "timed window, untimed prefill; CPU restatement on all host threads (Rust crate unbuildable "
                "here: no cargo)")


def run_reference(args, rank, world):
    if rank != 0:
        return
    K, W = args.steps, args.warmup
    # each step: a bounded sample of the workload (about 1 s of frames of the
    # round-robin batch sample) on every host core
    budget = float(os.environ.get("CTTS_REF_STEP_S", "1.0"))
    ref = CpuRef()
    frames, secs = 0, 0.0
    for i in range(W + K):
        n, el = ref.run(budget)
        if i >= W:
            frames, secs = frames + n, secs + el
    fps = frames / secs
    line = {"impl": "reference", "metric": METRIC, "value": round(fps, 3), "unit": UNIT, "n_gpus": args.gpus,
            "steps": K, "warmup": W, "ms_per_step": round(1e3 / fps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16-rounded weights)",
            "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) random-init weights)",
            "config": {"workload": "config[3]: batched AR decode, config[2] model, 64 utterances/GPU, "
                                   "text U[20,120] + 150 prompt frames, 500 frames each",
                       "utterances_sampled": len(ref.utts), "kv_ctx_mean": round(ref.ctx_mean, 1),
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": round(fps, 3), "unit": UNIT, "cores": ref.threads, "kind": "port",
                             "sample": ref.describe(frames, secs) + f"; {K} steps of ~{budget:.0f}s"},
            "e2e": {"value": round(fps, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-b1", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--only", default="", choices=["", "c2", "probe", "c0", "c1", "c4"],
                    help="c2: only the batch-1 fp32 config[2] measurement; probe: only the roofline probe; "
                         "c0 / c1 / c4: only that configuration's measurement")
    ap.add_argument("--b1-frames", type=int, default=197, help="timed frames of the batch-1 run (<= 197)")
    ap.add_argument("--c4-batch", type=int, default=32, help="config[4] batch (profiling: smaller)")
    ap.add_argument("--c4-frames", type=int, default=400, help="config[4] latent frames (profiling: fewer)")
    ap.add_argument("--c4-dtypes", default="bf16,f32", help="config[4] weight dtypes to time")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the config[0] / config[1] / config[4] measurements")
    ap.add_argument("--groups", type=int, default=1,
                    help="sub-batches of the 64 utterances run as parallel branches of the frame graph")
    ap.add_argument("--start-frame", type=int, default=-1,
                    help="first warm-up frame (default: timed window centred on the run)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch

    if args.only == "probe":
        torch.cuda.set_device(local)
        print(json.dumps({"roofline": dominant_kernel_roofline(None, None, None, None, local)}), flush=True)
        return
    if args.only in ("c0", "c1", "c4"):
        torch.cuda.set_device(local)
        if args.only == "c4":
            res = bench_c4(local, cpu=not args.no_cpu, B=args.c4_batch, T=args.c4_frames,
                           dtypes=tuple(args.c4_dtypes.split(",")))
        else:
            res = {"c0": bench_c0, "c1": bench_c1}[args.only](local)
        print(json.dumps({args.only: res}), flush=True)
        return
    if args.only == "c2":
        torch.cuda.set_device(local)
        out = run_b1(args, local)
        out.update({"metric": "us per decode step (config[2], batch 1, fp32)", "n_gpus": 1})
        print(json.dumps(out), flush=True)
        return
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                             device_id=torch.device("cuda", local))
    res, keep = run_ours(args, rank, world, local)
    K, W = args.steps, args.warmup
    B = B_PER_GPU
    total_frames = B * world * K
    value = total_frames / (res["ms"] * 1e-3)
    e2e = total_frames / (res["ms_e2e"] * 1e-3)
    hbm, bf16_tf, kind = res["peak"]
    step_gbs = res["step_bytes"] / (res["ms"] / K * 1e-3) / 1e9
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(res["ms"] / K, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 weights/KV, fp32 accumulate",
        "data": "synthetic (seeded N(0,1) inputs and noise, N(0,0.02) random-init weights)",
        "config": {"workload": "config[3]: batched AR decode, config[2] model, 64 utterances/GPU, "
                               "text U[20,120] + 150 prompt frames, 500 frames each",
                   "global_batch": B * world, "utterances_per_gpu": B, "euler_steps": 10,
                   "sub_batch_groups": args.groups,
                   "timed_frames": f"{res['start'] + W}..{res['start'] + W + K - 1} of 500",
                   "kv_ctx_mean": round(res["ctx_mean"], 1), "parallelism": f"utterance-sharded x{world}",
                   "l2": f"per-step working set (weights+KV) > {l2_bytes() >> 20} MB L2; no flush"},
        "rtf": round((res["ms"] / K * 1e-3) * FRAME_HZ, 4),
        "us_per_step": round(res["ms"] / K * 1e3, 2),
        "step_roofline": {"bound": "hbm", "achieved": round(step_gbs, 1), "peak": hbm, "unit": "GB/s",
                          "frac": round(step_gbs / hbm, 4), "bytes_per_step": int(res["step_bytes"]),
                          "of": kind},
        "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": B * 64 * 4,
                "d2h_bytes_per_step": B * 64 * 4 + B * 2 * 4},
        "gpu_launches": res["launches"] * K,
        "launches_per_step": res["launches"],
        "clocks": res["clocks"],
        "outputs_finite": res["finite"],
        "phases": res["phases"],
    }
    if rank == 0 and world == 1:
        lm, dit, lcfg, dcfg, hw = keep
        try:
            tc = dominant_kernel_roofline(lm, dit, lcfg, dcfg, local)
            out["roofline"] = dit_kernel_roofline(dit, dcfg, lcfg, local, tc_probe={"tc_linear": tc})
        except Exception as ex:  # report, do not hide
            out["roofline"] = {"error": repr(ex)}
        if not args.no_b1:
            out["b1"] = run_b1(args, local)
        if not args.no_configs:
            for name, fn in (("c0", bench_c0), ("c1", bench_c1), ("c4", bench_c4)):
                try:
                    out[name] = fn(local)
                except Exception as ex:  # report, do not hide
                    out[name] = {"error": repr(ex)}
        if not args.no_cpu:
            ref = CpuRef()
            n, el = ref.run(15.0)
            out["cpu_baseline"] = {"value": round(n / el, 3), "unit": UNIT, "cores": ref.threads,
                                   "kind": "port", "sample": ref.describe(n, el)}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
