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
L2_BYTES = 126 * 1024 * 1024


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            if len(r) >= 9:
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


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
    allu = utterances(B * world, seed=3, vocab=lcfg.vocab)
    utts = [allu[i] for i in shard(B * world, rank, world)]
    K, W = args.steps, args.warmup
    # timed frames end near the middle of the run unless a start frame is given
    start = args.start_frame if args.start_frame >= 0 else max(0, GEN_FRAMES // 2 - W - K)
    total = start + W + 2 * K + 2
    max_prefix = max(len(ids) for ids, _ in utts) + PROMPT_FRAMES
    cap = max_prefix + max(total, GEN_FRAMES) + 4
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
    launches = eng.launches_per_step
    ctx_mean = float(np.mean(ctx0)) + start + W + K / 2
    step_bytes = algorithmic_bytes_per_step(lcfg, dcfg, B, ctx_mean, 2, 2)
    res = {
        "ms": ms, "ms_e2e": ms_e2e, "launches": launches, "clocks": clocks, "ctx_mean": ctx_mean,
        "step_bytes": step_bytes, "start": start, "peak": (hbm, bf16_tf, peak_kind),
        "finite": bool(torch.isfinite(lat[:start + W + K]).all().item()),
    }
    del eng
    return res, (lm, dit, lcfg, dcfg, hw)


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
           "launches_per_step": eng.launches_per_step}
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
           "frac": round(tf / bf16_tf, 4), "traffic": 31.0e6, "of": kind,
           "kernel": "dit_cluster_kernel (tcgen05, 16-CTA clusters) + DiT prologue via ctts_dit_euler_sample_dev, "
                     "64 utterances x 10 Euler steps",
           "flops_per_launch": flops, "us_per_launch": round(t * 1e6, 2),
           "traffic_note": "ncu dram__bytes_read+write of one dit_cluster_kernel launch in the bench frame "
                           "(weights L2-resident; 1.94 GB of L2->SMEM TMA traffic per launch)"}
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
        flush = torch.empty(2 * L2_BYTES // 4, device="cuda")
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


# -------------------------------------------------------------- CPU side
class CpuRef:
    """The oracle (C restatement of the reference CPU path) on the host
    cores: one utterance of the config[3] model (bf16-rounded weights widened
    to fp32, as the reference loads bf16 checkpoints), prefill untimed; run()
    advances frames for a time budget and returns (frames, seconds)."""

    def __init__(self, threads: int | None = None):
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
        ids, prompt = utterances(1, 3, lcfg.vocab)[0]
        pre = np.concatenate([orc.embed_lookup(lw["embed_tokens.weight"], ids),
                              orc.linear(prompt, self.hw["latent_proj.weight"], self.hw["latent_proj.bias"])], 0)
        self.cache = self.lm.new_cache(pre.shape[0] + GEN_FRAMES + 8)
        self.z = self.lm.forward(pre, self.cache)[-1].copy()
        self.cond = prompt[-1].copy()
        self.rng = np.random.default_rng(5)
        self.frames = 0

    def run(self, seconds: float):
        orc, hw = self.orc, self.hw
        n = 0
        t0 = time.perf_counter()
        while self.frames < GEN_FRAMES:
            orc.stop_logits(hw["stop_predictor.weight"], hw["stop_predictor.bias"], self.z)
            x = self.dit.euler_sample(self.rng.standard_normal(64, dtype=np.float32), self.z, self.cond,
                                      self.z, 10)
            self.cond = x
            fb = orc.linear(x[None], hw["latent_proj.weight"], hw["latent_proj.bias"])
            self.z = self.lm.forward(fb, self.cache)[0].copy()
            n += 1
            self.frames += 1
            if time.perf_counter() - t0 >= seconds:
                break
        return n, time.perf_counter() - t0


def run_reference(args, rank, world):
    if rank != 0:
        return
    K, W = args.steps, args.warmup
    # each step: a bounded sample of the workload (about 1 s of frames of one
    # utterance) on every host core
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
            "config": {"workload": "config[3] model, one utterance, CPU restatement of the reference path",
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": round(fps, 3), "unit": UNIT, "cores": ref.threads, "kind": "port",
                             "sample": f"{frames} frames of one utterance over {K} steps of ~{budget:.0f}s "
                                       "after an untimed prefill (Rust crate unbuildable here: no cargo)"},
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
    ap.add_argument("--only", default="", choices=["", "c2", "probe"],
                    help="c2: only the batch-1 fp32 config[2] measurement; probe: only the roofline probe")
    ap.add_argument("--b1-frames", type=int, default=197, help="timed frames of the batch-1 run (<= 197)")
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
                   "l2": "per-step working set (weights+KV) > 126 MB L2; no flush"},
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
        if not args.no_cpu:
            ref = CpuRef()
            n, el = ref.run(15.0)
            out["cpu_baseline"] = {"value": round(n / el, 3), "unit": UNIT, "cores": ref.threads,
                                   "kind": "port",
                                   "sample": f"{n} frames of one config[3]-model utterance in {el:.1f}s "
                                             "after an untimed prefill (CPU restatement, all host threads)"}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
