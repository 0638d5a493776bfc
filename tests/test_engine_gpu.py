"""The per-frame engine (stop head -> DiT Euler sample -> latent out ->
feedback projection -> LM decode step, one CUDA graph per frame) against
the oracle's AR loop on identical seeded inputs (noise passed in)."""
import numpy as np
import pytest

from conftest import cosine, rel_err
from helpers import bf16_weights, rnd
from oracle import oracle as orc
from rcutetts_b200 import synth
from rcutetts_b200.config import DiTConfig, LMConfig

pytestmark = pytest.mark.gpu


def build(lcfg, dcfg, seed, dtype, batch, capacity, use_graph=True):
    from rcutetts_b200.model import DitW, FrameEngine, QwenW

    lw = synth.lm_weights(lcfg, seed=seed, with_embed=True)
    dw = synth.dit_weights(dcfg, seed=seed + 10)
    hw = synth.frame_weights(lcfg.hidden, dcfg.latent, seed=seed + 20)
    lm = QwenW(lcfg, dtype).set_weights(lw)
    dit = DitW(dcfg, dtype).set_weights(dw)
    eng = FrameEngine(lm, dit, hw, batch=batch, capacity=capacity, euler_steps=10, use_graph=use_graph)
    return eng, (lm, dit), lw, dw, hw


def prefix_rows(lw, hw, ids, prompt):
    """[embed(text ids); latent_proj(prompt latents)] -- the config[2] prefix."""
    emb = orc.embed_lookup(lw["embed_tokens.weight"], ids)
    pr = orc.linear(prompt, hw["latent_proj.weight"], hw["latent_proj.bias"])
    return np.concatenate([emb, pr], 0)


def test_b1_fp32_frames_vs_oracle():
    lcfg, dcfg = LMConfig(), DiTConfig()
    eng, keep, lw, dw, hw = build(lcfg, dcfg, seed=2, dtype="f32", batch=1, capacity=256)
    rng = np.random.default_rng(2)
    ids = rng.integers(0, lcfg.vocab, 40)
    prompt = rng.standard_normal((150, 64), dtype=np.float32)
    noise = rng.standard_normal((5, 64), dtype=np.float32)
    pre = prefix_rows(lw, hw, ids, prompt)
    eng.prefill(0, pre, prompt[-1])
    lats, stops = [], []
    for f in range(5):
        lat, st = eng.step(noise[f:f + 1])
        lats.append(lat[0])
        stops.append(st[0])
    ref_lat, ref_stop, _ = orc.generate(orc.LM(lcfg, lw), orc.DiT(dcfg, dw), hw, pre, noise, prompt[-1], 10)
    for f in range(5):
        assert rel_err(lats[f], ref_lat[f]) < 1e-4, f
        assert cosine(lats[f], ref_lat[f]) >= 0.9999, f
        assert rel_err(stops[f], ref_stop[f]) < 1e-4, f
    assert eng.launches_per_step > 0


def test_graph_replay_matches_eager():
    lcfg, dcfg = LMConfig(n_layers=2), DiTConfig(n_layers=2)
    outs = []
    for use_graph in (True, False):
        eng, keep, lw, dw, hw = build(lcfg, dcfg, seed=3, dtype="f32", batch=2, capacity=64,
                                      use_graph=use_graph)
        for b in range(2):
            eng.prefill(b, rnd(30 + b, (7 + 3 * b, lcfg.hidden)), rnd(40 + b, (64,)))
        noise = rnd(50, (4, 2, 64))
        outs.append(np.stack([eng.step(noise[f])[0] for f in range(4)]))
        del eng
    assert np.array_equal(outs[0], outs[1])


def test_batched_bf16_ragged_vs_oracle():
    """config[3] in miniature: bf16 weights, ragged prefixes, batch 3."""
    lcfg, dcfg = LMConfig(n_layers=4), DiTConfig()
    eng, keep, lw, dw, hw = build(lcfg, dcfg, seed=4, dtype="bf16", batch=3, capacity=96)
    rng = np.random.default_rng(4)
    lens = [20, 33, 27]
    pres, conds = [], []
    lwb, dwb, hwb = bf16_weights(lw), bf16_weights(dw), hw
    for b in range(3):
        ids = rng.integers(0, lcfg.vocab, lens[b])
        prompt = rng.standard_normal((12, 64), dtype=np.float32)
        # the device embeds with its bf16 table: build the prefix from the same rounded table
        pres.append(prefix_rows(lwb, hw, ids, prompt))
        conds.append(prompt[-1])
        eng.prefill(b, pres[-1], conds[-1])
    noise = rng.standard_normal((4, 3, 64), dtype=np.float32)
    lat = np.stack([eng.step(noise[f])[0] for f in range(4)])
    lm_o, dit_o = orc.LM(lcfg, lwb), orc.DiT(dcfg, dwb)
    for b in range(3):
        ref, _, _ = orc.generate(lm_o, dit_o, hwb, pres[b], noise[:, b, :], conds[b], 10)
        for f in range(4):
            assert cosine(lat[f, b], ref[f]) >= 0.999, (b, f)


def test_step_requires_prefill():
    from rcutetts_b200._lib import ERR_STATE, CttsError

    lcfg, dcfg = LMConfig(n_layers=1), DiTConfig(n_layers=1)
    eng, keep, lw, dw, hw = build(lcfg, dcfg, seed=5, dtype="f32", batch=2, capacity=16)
    eng.prefill(0, rnd(1, (3, lcfg.hidden)), rnd(2, (64,)))
    with pytest.raises(CttsError) as e:
        eng.step(rnd(3, (2, 64)))
    assert e.value.code == ERR_STATE


def test_batched_bf16_tensor_core_path_vs_oracle():
    """16 utterances: the LM decode step and the DiT linears run on the
    tcgen05 tensor cores (>= 16 rows); prefill rows too."""
    lcfg, dcfg = LMConfig(n_layers=2), DiTConfig(n_layers=2)
    B = 16
    eng, keep, lw, dw, hw = build(lcfg, dcfg, seed=6, dtype="bf16", batch=B, capacity=64)
    rng = np.random.default_rng(6)
    lwb, dwb = bf16_weights(lw), bf16_weights(dw)
    pres, conds = [], []
    for b in range(B):
        ids = rng.integers(0, lcfg.vocab, 10 + (7 * b) % 23)
        prompt = rng.standard_normal((6, 64), dtype=np.float32)
        pres.append(prefix_rows(lwb, hw, ids, prompt))
        conds.append(prompt[-1])
        eng.prefill(b, pres[-1], conds[-1])
    noise = rng.standard_normal((3, B, 64), dtype=np.float32)
    lat = np.stack([eng.step(noise[f])[0] for f in range(3)])
    lm_o, dit_o = orc.LM(lcfg, lwb), orc.DiT(dcfg, dwb)
    for b in range(B):
        ref, _, _ = orc.generate(lm_o, dit_o, hw, pres[b], noise[:, b, :], conds[b], 10)
        for f in range(3):
            assert cosine(lat[f, b], ref[f]) >= 0.999, (b, f)


def test_sub_batch_groups_match_single_group():
    """groups=4 splits 32 utterances into 4 chains of 8 (own KV cache, DiT
    workspace and stream, parallel graph branches); every utterance's latents
    match the single-chain engine and the oracle, and graph replay equals
    eager execution bit for bit."""
    lcfg, dcfg = LMConfig(n_layers=2), DiTConfig(n_layers=2)
    B = 32
    rng = np.random.default_rng(7)
    lens = [5 + (11 * b) % 29 for b in range(B)]
    pres = [rnd(100 + b, (lens[b], lcfg.hidden)) for b in range(B)]
    conds = [rnd(200 + b, (64,)) for b in range(B)]
    noise = rng.standard_normal((3, B, 64), dtype=np.float32)
    outs = {}
    for groups, use_graph in ((1, True), (4, True), (4, False), (2, True)):
        from rcutetts_b200.model import DitW, FrameEngine, QwenW

        lw = synth.lm_weights(lcfg, seed=8, with_embed=False)
        dw = synth.dit_weights(dcfg, seed=18)
        hw = synth.frame_weights(lcfg.hidden, dcfg.latent, seed=28)
        lm = QwenW(lcfg, "bf16").set_weights(lw)
        dit = DitW(dcfg, "bf16").set_weights(dw)
        eng = FrameEngine(lm, dit, hw, batch=B, capacity=64, euler_steps=10, use_graph=use_graph,
                          groups=groups)
        for b in range(B):
            eng.prefill(b, pres[b], conds[b])
        outs[(groups, use_graph)] = np.stack([eng.step(noise[f])[0] for f in range(3)])
        del eng
    assert np.array_equal(outs[(4, True)], outs[(4, False)])
    for key in ((4, True), (2, True)):
        for b in range(B):
            for f in range(3):
                assert cosine(outs[key][f, b], outs[(1, True)][f, b]) >= 0.9999, (key, b, f)
    lwb, dwb = bf16_weights(lw), bf16_weights(dw)
    lm_o, dit_o = orc.LM(lcfg, lwb), orc.DiT(dcfg, dwb)
    for b in (0, 9, 31):
        ref, _, _ = orc.generate(lm_o, dit_o, hw, pres[b], noise[:, b, :], conds[b], 10)
        for f in range(3):
            assert cosine(outs[(4, True)][f, b], ref[f]) >= 0.999, (b, f)


def test_groups_must_divide_batch():
    from rcutetts_b200._lib import ERR_ARG, CttsError
    from rcutetts_b200.model import DitW, FrameEngine, QwenW

    lcfg, dcfg = LMConfig(n_layers=1), DiTConfig(n_layers=1)
    lm = QwenW(lcfg, "f32").set_weights(synth.lm_weights(lcfg, seed=9, with_embed=False))
    dit = DitW(dcfg, "f32").set_weights(synth.dit_weights(dcfg, seed=19))
    hw = synth.frame_weights(lcfg.hidden, dcfg.latent, seed=29)
    with pytest.raises(CttsError) as e:
        FrameEngine(lm, dit, hw, batch=6, capacity=16, groups=4)
    assert e.value.code == ERR_ARG


def test_cluster_dit_path_is_one_launch(monkeypatch):
    """bf16 engine at the benchmark DiT shape: the whole Euler loop of a
    frame is one launch (CTTS_DIT_CLUSTER unset) instead of the per-step
    chain, with the same latents."""
    lcfg, dcfg = LMConfig(n_layers=1), DiTConfig()
    B = 16
    res = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("CTTS_DIT_CLUSTER", flag)
        eng, keep, lw, dw, hw = build(lcfg, dcfg, seed=11, dtype="bf16", batch=B, capacity=32)
        for b in range(B):
            eng.prefill(b, rnd(300 + b, (4 + b % 5, lcfg.hidden)), rnd(400 + b, (64,)))
        noise = rnd(500, (2, B, 64))
        lat = np.stack([eng.step(noise[f])[0] for f in range(2)])
        res[flag] = (lat, eng.launches_per_step)
        del eng
    assert res["1"][1] + 200 < res["0"][1], (res["1"][1], res["0"][1])
    for f in range(2):
        for b in range(B):
            assert cosine(res["1"][0][f, b], res["0"][0][f, b]) >= 0.9999, (f, b)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_cfg_frames_vs_oracle(dtype):
    """Base-variant CFG frames (bin/cutetts.rs:440-456, 474-509): an
    unconditional LM branch per utterance with its own KV cache, fed the
    same latent; the DiT runs euler_sample_cfg on the sway grid with the
    unconditional rows' AdaLN zeroed.  Against the oracle's composition of
    the same loop."""
    from rcutetts_b200.model import DitW, FrameEngine, QwenW

    lcfg, dcfg = LMConfig(n_layers=2), DiTConfig(n_layers=2)
    lw = synth.lm_weights(lcfg, seed=31, with_embed=False)
    dw = synth.dit_weights(dcfg, seed=32)
    hw = synth.frame_weights(lcfg.hidden, dcfg.latent, seed=33)
    lm = QwenW(lcfg, dtype).set_weights(lw)
    dit = DitW(dcfg, dtype).set_weights(dw)
    B, F, cfg_s, coeff = 2, 3, 2.0, -1.0
    eng = FrameEngine(lm, dit, hw, batch=B, capacity=48, euler_steps=10, cfg_strength=cfg_s, sway_coeff=coeff)
    pres_c = [rnd(40 + b, (6 + 3 * b, lcfg.hidden)) for b in range(B)]
    pres_u = [rnd(50 + b, (2 + b, lcfg.hidden)) for b in range(B)]
    conds = [rnd(60 + b, (64,)) for b in range(B)]
    unconds = [rnd(70 + b, (64,)) for b in range(B)]
    for b in range(B):
        eng.prefill(b, pres_c[b], conds[b])
        eng.prefill_uncond(b, pres_u[b], unconds[b])
    noise = rnd(80, (F, B, 64))
    lat = np.stack([eng.step(noise[f])[0] for f in range(F)])
    lwo, dwo = (bf16_weights(lw), bf16_weights(dw)) if dtype == "bf16" else (lw, dw)
    lm_o, dit_o = orc.LM(lcfg, lwo), orc.DiT(dcfg, dwo)
    for b in range(B):
        cc, cu = lm_o.new_cache(48), lm_o.new_cache(48)
        zc = lm_o.forward(pres_c[b], cc)[-1].copy()
        zu = lm_o.forward(pres_u[b], cu)[-1].copy()
        cond, uncond = conds[b], unconds[b]
        for f in range(F):
            x = dit_o.euler_sample_cfg(noise[f, b], zc, zu, cond, uncond, zc, 10, coeff, cfg_s)
            if dtype == "f32":
                assert rel_err(lat[f, b], x) < 1e-4, (b, f)
            else:
                assert cosine(lat[f, b], x) >= 0.999, (b, f)
            x = lat[f, b] if dtype == "bf16" else x  # bf16: follow the device trajectory
            cond = uncond = x
            fb = orc.linear(x[None], hw["latent_proj.weight"], hw["latent_proj.bias"])
            zc = lm_o.forward(fb, cc)[0].copy()
            zu = lm_o.forward(fb, cu)[0].copy()


def test_phase_timers():
    """Per-frame phase timers (--profile-steps, bin/cutetts.rs:328-350): the
    profiled frames produce the same latents as graph replay, and every
    phase collects one positive device time per frame."""
    lcfg, dcfg = LMConfig(n_layers=2), DiTConfig(n_layers=2)
    outs = []
    for profile in (False, True):
        eng, keep, lw, dw, hw = build(lcfg, dcfg, seed=9, dtype="f32", batch=2, capacity=64)
        for b in range(2):
            eng.prefill(b, rnd(90 + b, (6 + b, lcfg.hidden)), rnd(95 + b, (64,)))
        noise = rnd(99, (5, 2, 64))
        lat = [eng.step(noise[0])[0]]  # the first frame runs eagerly in both modes
        if profile:
            eng.set_profile(True)
        lat += [eng.step(noise[f])[0] for f in range(1, 5)]
        outs.append(np.stack(lat))
        if profile:
            st = eng.profile_stats()
            rep = eng.profile_report()
        del eng
    assert np.array_equal(outs[0], outs[1])
    for name in ("stop", "dit", "feedback", "lm"):
        assert st[name]["n"] == 4, st
        assert 0.0 < st[name]["p50_ms"] <= st[name]["p99_ms"] + 1e-9
        assert f"{name}: n=4 mean=" in rep, rep


def test_dit_fp16_range_error_moves_head_to_launch_chain(monkeypatch):
    """A DiT head whose split-K partials leave the fp16 exchange range of
    the cluster loop (down projections scaled by 1e8): the frame step
    reports CTTS_ERR_RANGE (its latents, and the LM state they fed, are
    invalid); an engine built again on the same head runs the fp32-partial
    launch chain, bit for bit like a CTTS_DIT_CLUSTER=0 head."""
    from rcutetts_b200._lib import ERR_RANGE, CttsError
    from rcutetts_b200.model import DitW, FrameEngine, QwenW

    lcfg, dcfg = LMConfig(n_layers=1), DiTConfig()
    B = 16
    lw = synth.lm_weights(lcfg, seed=11, with_embed=True)
    dw = synth.dit_weights(dcfg, seed=21)
    for i in range(dcfg.n_layers):
        k = f"decoder.layers.{i}.mlp.down_proj.weight"
        dw[k] = dw[k] * np.float32(1e8)
    hw = synth.frame_weights(lcfg.hidden, dcfg.latent, seed=31)
    lm = QwenW(lcfg, "bf16").set_weights(lw)

    def engine(dit):
        eng = FrameEngine(lm, dit, hw, batch=B, capacity=32, euler_steps=10)
        for b in range(B):
            eng.prefill(b, rnd(300 + b, (4 + b % 5, lcfg.hidden)), rnd(400 + b, (64,)))
        return eng

    noise = rnd(500, (3, B, 64))
    dit = DitW(dcfg, "bf16").set_weights(dw)
    eng = engine(dit)
    with pytest.raises(CttsError) as e:
        eng.step(noise[0])
    assert e.value.code == ERR_RANGE
    del eng
    eng = engine(dit)
    lat = np.stack([eng.step(noise[f])[0] for f in range(3)])
    monkeypatch.setenv("CTTS_DIT_CLUSTER", "0")
    eng0 = engine(DitW(dcfg, "bf16").set_weights(dw))
    lat0 = np.stack([eng0.step(noise[f])[0] for f in range(3)])
    assert np.isfinite(lat).all()
    assert np.array_equal(lat, lat0)
    assert eng.launches_per_step == eng0.launches_per_step


def test_two_engines_from_two_host_threads():
    """Two bf16 engines (own handles, streams and workspaces; the benchmark
    DiT shape) stepped at the same time from two host threads -- the C calls
    release the GIL.  Each gives bit for bit what the same engine gives
    stepped alone, and matches the oracle."""
    import threading

    lcfg, dcfg = LMConfig(n_layers=2), DiTConfig()
    B, F = 16, 3

    def setup(k):
        eng, keep, lw, dw, hw = build(lcfg, dcfg, seed=40 + k, dtype="bf16", batch=B, capacity=48)
        rng = np.random.default_rng(40 + k)
        lwb = bf16_weights(lw)
        pres, conds = [], []
        for b in range(B):
            ids = rng.integers(0, lcfg.vocab, 8 + b % 5)
            prompt = rng.standard_normal((4, 64), dtype=np.float32)
            pres.append(prefix_rows(lwb, hw, ids, prompt))
            conds.append(prompt[-1])
            eng.prefill(b, pres[-1], conds[-1])
        noise = rng.standard_normal((F, B, 64), dtype=np.float32)
        return dict(eng=eng, keep=keep, lw=lw, dw=dw, hw=hw, pres=pres, conds=conds, noise=noise)

    def frames(st):
        return np.stack([st["eng"].step(st["noise"][f])[0] for f in range(F)])

    alone = []
    for k in range(2):
        st = setup(k)
        alone.append(frames(st))
        del st
    setups = [setup(k) for k in range(2)]
    out, errs = [None, None], []
    start = threading.Barrier(2)

    def run(k):
        try:
            start.wait(timeout=60)
            out[k] = frames(setups[k])
        except Exception as e:  # reported below
            errs.append(e)

    th = [threading.Thread(target=run, args=(k,)) for k in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join(300)
    assert not any(t.is_alive() for t in th)
    assert not errs, errs
    for k in range(2):
        st = setups[k]
        assert np.array_equal(out[k], alone[k]), k
        lm_o, dit_o = orc.LM(lcfg, bf16_weights(st["lw"])), orc.DiT(dcfg, bf16_weights(st["dw"]))
        for b in (0, B - 1):
            ref, _, _ = orc.generate(lm_o, dit_o, st["hw"], st["pres"][b], st["noise"][:, b, :], st["conds"][b], 10)
            for f in range(F):
                assert cosine(out[k][f, b], ref[f]) >= 0.999, (k, b, f)
