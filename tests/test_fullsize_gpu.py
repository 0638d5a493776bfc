"""Parity at the sizes the benchmark runs, against the oracle on identical
seeded inputs (flow-ODE noise passed in).

Policy of the reference's end-to-end test (rust-codec/tests/e2e_tts.rs:84-127):
teacher-forced per-frame gates over a whole run, then the decoded result.
Teacher forcing here: the oracle recomputes every frame from the device's own
history (the device latents are fed back on both sides), so a gate measures
one frame's error, not the drift of two free-running trajectories.

* config[2] (batch 1, fp32, 12+4 layers): all 200 frames teacher-forced at
  1e-4 (latents and stop logits), and the free-running run against the
  oracle's own free-running loop at cosine >= 0.9999 on the final latents.
* config[3] (bench.py's workload: 64 utterances, bf16 weights and KV, ragged
  170-270-row prefixes, 7 DiT clusters with 4 utterances in the last): the
  frames of bench.py's timed window (KV context ~ 450), teacher-forced, for
  8 utterances spread over all 7 clusters, cosine >= 0.999.
* config[4] (VAE, T = 400): 2 utterances against the oracle, fp32 within
  1e-4 and cosine >= 0.9999, bf16 cosine >= 0.999.
"""
import numpy as np
import pytest

import bench
from conftest import cosine, rel_err
from helpers import bf16_weights
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def feedback(hw, lat):
    """latent_proj(latent) rows (the engine's feedback projection)."""
    return orc.linear(np.ascontiguousarray(lat, np.float32).reshape(-1, 64), hw["latent_proj.weight"],
                      hw["latent_proj.bias"])


def teacher_forced(lm_o, dit_o, hw, prefix, cond0, noise, dev_lat, frames):
    """Oracle frames `frames` (consecutive) of one utterance, each computed
    from the device's history: the LM consumes the prefix and the feedback
    rows of dev_lat[:frames[0]] in one prefill, then per frame the stop
    logits and the DiT sample from the current LM state and the previous
    device latent, after which the device latent of that frame is fed back.
    Returns (latents [n, 64], stop logits [n, 2])."""
    f0 = frames[0]
    rows = prefix if f0 == 0 else np.concatenate([prefix, feedback(hw, dev_lat[:f0])], 0)
    cache = lm_o.new_cache(rows.shape[0] + len(frames) + 1)
    z = lm_o.forward(rows, cache)[-1].copy()
    cond = np.asarray(cond0 if f0 == 0 else dev_lat[f0 - 1], np.float32).copy()
    lats, stops = [], []
    for f in frames:
        stops.append(orc.stop_logits(hw["stop_predictor.weight"], hw["stop_predictor.bias"], z))
        lats.append(dit_o.euler_sample(noise[f], z, cond, z, 10))
        cond = np.asarray(dev_lat[f], np.float32).copy()
        z = lm_o.forward(feedback(hw, cond), cache)[0].copy()
    return np.stack(lats), np.stack(stops)


def test_config2_all_200_frames():
    """config[2] end to end on the frame engine: batch 1, fp32, 40 text ids +
    150 prompt latents, 200 frames (bench.py's batch-1 workload)."""
    from rcutetts_b200.model import FrameEngine

    lcfg, dcfg, lw, dw, hw, lm, dit = bench.make_models("f32", seed=2, device=0)
    rng = np.random.default_rng(2)
    ids = rng.integers(0, lcfg.vocab, 40)
    prompt = rng.standard_normal((bench.PROMPT_FRAMES, 64), dtype=np.float32)
    F = 200
    noise = rng.standard_normal((F, 64), dtype=np.float32)
    pre = bench.prefix_rows(lm, hw, ids, prompt)
    eng = FrameEngine(lm, dit, hw, batch=1, capacity=pre.shape[0] + F + 4, euler_steps=10)
    eng.prefill(0, pre, prompt[-1])
    lat, stop = np.empty((F, 64), np.float32), np.empty((F, 2), np.float32)
    for f in range(F):
        lv, sv = eng.step(noise[f:f + 1])
        lat[f], stop[f] = lv[0], sv[0]
    lm_o, dit_o = orc.LM(lcfg, lw), orc.DiT(dcfg, dw)
    ref, ref_stop = teacher_forced(lm_o, dit_o, hw, pre, prompt[-1], noise, lat, list(range(F)))
    errs = [rel_err(lat[f], ref[f]) for f in range(F)]
    serrs = [rel_err(stop[f], ref_stop[f]) for f in range(F)]
    assert max(errs) < 1e-4, (int(np.argmax(errs)), max(errs))
    assert max(serrs) < 1e-4, (int(np.argmax(serrs)), max(serrs))
    # free running on both sides from the same prefix and noise
    free, free_stop, _ = orc.generate(lm_o, dit_o, hw, pre, noise, prompt[-1], 10)
    assert cosine(lat, free) >= 0.9999
    assert cosine(lat[-1], free[-1]) >= 0.9999
    assert cosine(stop, free_stop) >= 0.9999


# utterances of every DiT cluster (10 per cluster; cluster 6 holds 60..63)
C3_UTTS = [0, 9, 10, 21, 32, 43, 54, 63]


def test_config3_bench_workload_full_size():
    """bench.py's headline workload at full size: 64 utterances, the 12-layer
    bf16 LM, the 4-layer DiT on 7 clusters.  The engine generates through the
    timed window of the benchmark (frames 230..233, KV context ~ 450) and 8
    utterances spread over every cluster are checked frame by frame."""
    from rcutetts_b200.model import FrameEngine

    lcfg, dcfg, lw, dw, hw, lm, dit = bench.make_models("bf16", seed=3, device=0)
    B = bench.B_PER_GPU
    utts = bench.utterances(B, seed=3, vocab=lcfg.vocab)
    F0, NF = 230, 4
    pres = [bench.prefix_rows(lm, hw, ids, prompt) for ids, prompt in utts]
    eng = FrameEngine(lm, dit, hw, batch=B, capacity=max(p.shape[0] for p in pres) + F0 + NF + 4,
                      euler_steps=10)
    for b, (ids, prompt) in enumerate(utts):
        eng.prefill(b, pres[b], prompt[-1])
    rng = np.random.default_rng(33)
    noise = rng.standard_normal((F0 + NF, B, 64), dtype=np.float32)
    lat = np.empty((F0 + NF, B, 64), np.float32)
    stop = np.empty((F0 + NF, B, 2), np.float32)
    for f in range(F0 + NF):
        lat[f], stop[f] = eng.step(noise[f])
    assert np.isfinite(lat).all()
    ctx = [pres[u].shape[0] + F0 for u in C3_UTTS]
    assert min(ctx) >= 400, ctx
    lm_o, dit_o = orc.LM(lcfg, bf16_weights(lw)), orc.DiT(dcfg, bf16_weights(dw))
    frames = list(range(F0, F0 + NF))
    dev_stops, ref_stops = [], []
    for u in C3_UTTS:
        ref, ref_stop = teacher_forced(lm_o, dit_o, hw, pres[u], utts[u][1][-1], noise[:, u], lat[:, u], frames)
        for i, f in enumerate(frames):
            assert cosine(lat[f, u], ref[i]) >= 0.999, (u, f, cosine(lat[f, u], ref[i]))
        dev_stops.append(stop[F0:F0 + NF, u])
        ref_stops.append(ref_stop)
    # two logits per frame: gate them together over every checked frame
    assert cosine(np.stack(dev_stops), np.stack(ref_stops)) >= 0.999


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_config4_full_length_vs_oracle(dtype):
    """VAE decoder of config[4] at full length (T = 400 frames -> 128,000
    samples), two utterances, against the oracle."""
    from rcutetts_b200 import synth
    from rcutetts_b200.config import VAEConfig
    from rcutetts_b200.model import DecoderW

    cfg = VAEConfig()
    w = synth.vae_weights(cfg, seed=4)
    m = DecoderW(cfg, dtype).set_weights(w)
    lat = np.random.default_rng(4).standard_normal((2, 64, 400), dtype=np.float32)
    wav = m.decode(lat)
    assert wav.shape == (2, 400 * cfg.hop)
    o = orc.VAE(cfg, w if dtype == "f32" else bf16_weights(w))
    for b in range(2):
        ref = o.decode(lat[b])
        if dtype == "f32":
            assert rel_err(wav[b], ref) < 1e-4, b
            assert cosine(wav[b], ref) >= 0.9999, b
        else:
            assert cosine(wav[b], ref) >= 0.999, b
