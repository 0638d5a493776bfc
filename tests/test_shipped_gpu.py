"""The shipped model's LM and DiT head shapes on the GPU (qwen.rs:17-24:
hidden 1024, 7 layers, 16/8 heads of 128, FFN 3072, vocab 16385; dit.rs:16-26:
hidden 1024, FFN 4096, 16/2 heads of 64, patch 2, speaker AdaLN width 256,
mu_proj Identity), against golden vectors made with HF Qwen3Model and the
reference AudioDiTHead (tests/golden/make_golden.py shipped; synthetic
weights, there is no checkpoint here), and against the oracle in bf16 and
at a 16-utterance batch (tensor-core paths); the frame engine at these
shapes with a per-utterance speaker vector conditioning AdaLN."""
import numpy as np
import pytest

from conftest import cosine, rel_err
from helpers import bf16_weights, dit_model, lm_model, rnd
from oracle import oracle as orc
from rcutetts_b200 import synth
from rcutetts_b200.config import DiTConfig, LMConfig

pytestmark = pytest.mark.gpu

LM_SHIPPED = LMConfig(hidden=1024, n_layers=7, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072, vocab=16385)
DIT_SHIPPED = DiTConfig(hidden=1024, n_heads=16, n_kv_heads=2, head_dim=64, ffn=4096, n_layers=4, patch=2,
                        cond_dim=1024, spk_dim=256)


def run_device(m, xp, xd, capacity=64):
    from rcutetts_b200.model import QwenCache, decode_step, prefill

    cache = QwenCache(m, batch=1, capacity=capacity)
    outs = [prefill(m, xp, cache)]
    for i in range(xd.shape[0]):
        outs.append(decode_step(m, xd[i:i + 1], cache))
    return np.concatenate(outs, 0)


def test_lm_shipped_fp32_vs_golden(golden):
    g = golden("lm_shipped.npz")
    m, _ = lm_model(LM_SHIPPED, seed=30)
    got = run_device(m, g["x_prefill"], g["x_decode"])
    for i in range(got.shape[0]):
        assert rel_err(got[i], g["final_out"][i]) < 1e-4, i


def test_lm_shipped_bf16_batch_vs_oracle():
    """16 utterances with ragged prefills: the bf16 tensor-core linears and
    the head_dim-128 decode attention against the oracle on bf16 weights."""
    from rcutetts_b200.model import QwenCache, decode_step, prefill

    m, w = lm_model(LM_SHIPPED, seed=32, dtype="bf16")
    o = orc.LM(LM_SHIPPED, bf16_weights(w))
    B = 16
    lens = [3 + (5 * b) % 11 for b in range(B)]
    cache = QwenCache(m, batch=B, capacity=32)
    pre = [rnd(600 + b, (lens[b], LM_SHIPPED.hidden)) for b in range(B)]
    dec = rnd(650, (3, B, LM_SHIPPED.hidden))
    for b in range(B):
        prefill(m, pre[b], cache, b)
    outs = [decode_step(m, dec[s], cache) for s in range(3)]
    for b in (0, 7, 15):
        oc = o.new_cache(32)
        o.forward(pre[b], oc)
        for s in range(3):
            ref = o.forward(dec[s, b:b + 1], oc)[0]
            assert cosine(outs[s][b], ref) >= 0.999, (b, s)


def test_dit_shipped_fp32_vs_golden(golden):
    g = golden("dit_shipped.npz")
    m, _ = dit_model(DIT_SHIPPED, seed=31)
    v = m.predict(g["x0"], float(g["t"]), g["z"], g["cond"], spk=g["spk"])
    for b in range(2):
        assert rel_err(v[b], g["predict_out"][b]) < 1e-4
    x = m.euler_sample(g["x0"], g["z"], g["cond"], g["spk"], 10)
    for b in range(2):
        assert rel_err(x[b], g["euler10_out"][b]) < 1e-4
        assert cosine(x[b], g["euler10_out"][b]) >= 0.9999


def test_dit_shipped_bf16_batch_vs_oracle():
    m, w = dit_model(DIT_SHIPPED, seed=33, dtype="bf16")
    o = orc.DiT(DIT_SHIPPED, bf16_weights(w))
    B, P = 16, DIT_SHIPPED.patch * DIT_SHIPPED.latent
    x0, z, c, spk = rnd(700, (B, P)), rnd(701, (B, 1024)), rnd(702, (B, P)), rnd(703, (B, 256))
    x = m.euler_sample(x0, z, c, spk, 10)
    for b in (0, 5, 15):
        ref = o.euler_sample(x0[b], z[b], c[b], spk[b], 10)
        assert cosine(x[b], ref) >= 0.999, b


@pytest.mark.parametrize("distill", [False, True])
def test_engine_shipped_frames_vs_oracle(distill):
    """The frame engine at the shipped shapes (7-layer LM, patch-2 DiT whose
    AdaLN is conditioned on a 256-wide speaker vector set per utterance):
    4 utterances x 3 frames in bf16 against the oracle's AR loop on the same
    bf16 weights.  distill: the distill checkpoint's head (step-size and
    cfg-strength embeddings, dit_manifest.json) sampled in 4 Euler steps with
    the distilled guidance strength 2.0 as its condition (bin/cutetts.rs:460-461)."""
    from dataclasses import replace

    from rcutetts_b200._lib import ERR_STATE, CttsError
    from rcutetts_b200.model import DitW, FrameEngine, QwenW

    lcfg = LM_SHIPPED
    dcfg = replace(DIT_SHIPPED, step_emb=True, cfg_emb=True) if distill else DIT_SHIPPED
    steps, strength = (4, 2.0) if distill else (10, 0.0)
    PL = dcfg.latent * dcfg.patch
    lw = synth.lm_weights(lcfg, seed=34, with_embed=True)
    dw = synth.dit_weights(dcfg, seed=35)
    hw = synth.frame_weights(lcfg.hidden, PL, seed=36)
    lm = QwenW(lcfg, "bf16").set_weights(lw)
    dit = DitW(dcfg, "bf16").set_weights(dw)
    B = 4
    eng = FrameEngine(lm, dit, hw, batch=B, capacity=64, euler_steps=steps, cfg_strength=strength)
    pres = [rnd(800 + b, (6 + 3 * b, lcfg.hidden)) for b in range(B)]
    conds, spks = rnd(810, (B, PL)), rnd(811, (B, dcfg.spk_dim))
    noise = rnd(812, (3, B, PL))
    for b in range(B):
        eng.prefill(b, pres[b], conds[b])
    with pytest.raises(CttsError) as e:  # the speaker vectors are required
        eng.step(noise[0])
    assert e.value.code == ERR_STATE
    for b in range(B):
        eng.set_speaker(b, spks[b])
    lat = np.stack([eng.step(noise[f])[0] for f in range(3)])
    lm_o, dit_o = orc.LM(lcfg, bf16_weights(lw)), orc.DiT(dcfg, bf16_weights(dw))
    for b in (0, 3):
        ref, _, _ = orc.generate(lm_o, dit_o, hw, pres[b], noise[:, b, :], conds[b], steps, spk=spks[b],
                                 cfg_w=strength)
        for f in range(3):
            assert cosine(lat[f, b], ref[f]) >= 0.999, (b, f)
