"""DiT flow head on the GPU against the torch-made golden vectors
(AudioDiTHead at the config[2] shape) and the oracle."""
import numpy as np
import pytest

from conftest import cosine, rel_err
from helpers import bf16_weights, dit_model, rnd
from oracle import oracle as orc
from rcutetts_b200.config import DiTConfig

pytestmark = pytest.mark.gpu


def test_predict_and_euler_config2(golden):
    g = golden("dit_c2.npz")
    cfg = DiTConfig()
    m, w = dit_model(cfg, seed=12)
    v = m.predict(g["x0"], float(g["t"]), g["z"], g["cond"], spk=g["z"])
    for b in range(2):
        assert rel_err(v[b], g["predict_out"][b]) < 1e-4
    x = m.euler_sample(g["x0"], g["z"], g["cond"], g["z"], 10)
    for b in range(2):
        assert rel_err(x[b], g["euler10_out"][b]) < 1e-4
        assert cosine(x[b], g["euler10_out"][b]) >= 0.9999


def test_plain_predict_and_cfg(golden):
    g, gc = golden("dit_plain.npz"), golden("dit_c2.npz")
    cfg = DiTConfig(adaln=False, n_layers=2)
    m, w = dit_model(cfg, seed=13)
    v = m.predict(gc["x0"], 0.7, gc["z"], gc["cond"])
    assert rel_err(v, g["predict_out"]) < 1e-4
    x = m.euler_sample_cfg(gc["x0"], gc["z"], g["z_uncond"], gc["cond"], g["uncond"], None, 10, -0.8, 2.0)
    assert rel_err(x, g["cfg_out"]) < 1e-4


def test_cfg_with_adaln_vs_oracle():
    """CFG with AdaLN: the uncond branch feeds zero AdaLN rows (dit.rs:878-887)."""
    cfg = DiTConfig(n_layers=2)
    m, w = dit_model(cfg, seed=14)
    o = orc.DiT(cfg, w)
    x0, zc, zu = rnd(1, (2, 64)), rnd(2, (2, 768)), rnd(3, (2, 768))
    c, u, spk = rnd(4, (2, 64)), rnd(5, (2, 64)), rnd(6, (2, 768))
    x = m.euler_sample_cfg(x0, zc, zu, c, u, spk, 6, -0.8, 2.0)
    for b in range(2):
        ref = o.euler_sample_cfg(x0[b], zc[b], zu[b], c[b], u[b], spk[b], 6, -0.8, 2.0)
        assert rel_err(x[b], ref) < 1e-4


def test_bf16_vs_oracle():
    cfg = DiTConfig()
    m, w = dit_model(cfg, seed=15, dtype="bf16")
    o = orc.DiT(cfg, bf16_weights(w))
    x0, z, c = rnd(7, (3, 64)), rnd(8, (3, 768)), rnd(9, (3, 64))
    x = m.euler_sample(x0, z, c, z, 10)
    for b in range(3):
        ref = o.euler_sample(x0[b], z[b], c[b], z[b], 10)
        assert cosine(x[b], ref) >= 0.999
        assert rel_err(x[b], ref) < 2e-3  # bf16 operands: rounding points differ by path


def test_batch_matches_single():
    cfg = DiTConfig()
    m, _ = dit_model(cfg, seed=16)
    x0, z, c = rnd(10, (5, 64)), rnd(11, (5, 768)), rnd(12, (5, 64))
    xb = m.euler_sample(x0, z, c, z, 4)
    for b in range(5):
        xs = m.euler_sample(x0[b:b + 1], z[b:b + 1], c[b:b + 1], z[b:b + 1], 4)
        assert rel_err(xs[0], xb[b]) < 1e-6


def test_distill_embeddings_vs_oracle():
    """Step-size and cfg-strength embeddings (distill checkpoint layout,
    diffusion_head.py:451-542) with hidden == cond_dim (mu_proj Identity)."""
    cfg = DiTConfig(hidden=256, cond_dim=256, spk_dim=128, n_heads=4, n_kv_heads=2, ffn=512,
                    n_layers=2, patch=2, step_emb=True, cfg_emb=True)
    m, w = dit_model(cfg, seed=17)
    o = orc.DiT(cfg, w)
    x0, z, c, spk = rnd(13, (2, 128)), rnd(14, (2, 256)), rnd(15, (2, 128)), rnd(16, (2, 128))
    x = m.euler_sample(x0, z, c, spk, 4, cfg_w=2.0)
    for b in range(2):
        ref = o.euler_sample(x0[b], z[b], c[b], spk[b], 4, cfg_w=2.0)
        assert rel_err(x[b], ref) < 1e-4


def test_bf16_tensor_core_batch_vs_oracle():
    """48 sequence rows (16 utterances x 3 tokens): tcgen05 linears incl. the
    AdaLN projection, gated residual epilogues and the SwiGLU tile pairing."""
    cfg = DiTConfig()
    m, w = dit_model(cfg, seed=18, dtype="bf16")
    o = orc.DiT(cfg, bf16_weights(w))
    B = 16
    x0, z, c = rnd(20, (B, 64)), rnd(21, (B, 768)), rnd(22, (B, 64))
    x = m.euler_sample(x0, z, c, z, 10)
    for b in range(B):
        ref = o.euler_sample(x0[b], z[b], c[b], z[b], 10)
        assert cosine(x[b], ref) >= 0.999, b


@pytest.mark.parametrize("adaln", [True, False])
def test_cluster_euler_loop_matches_launch_chain(monkeypatch, adaln):
    """bf16, 23 utterances (three 16-CTA clusters of 10 utterances, the last
    one partly filled): the cluster-resident Euler loop (one launch for all
    10 steps) against the per-step launch chain (CTTS_DIT_CLUSTER=0) and
    the oracle."""
    cfg = DiTConfig(adaln=adaln)
    B = 23
    x0, z, c = rnd(21, (B, 64)), rnd(22, (B, 768)), rnd(23, (B, 64))
    spk = z if adaln else None
    outs = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("CTTS_DIT_CLUSTER", flag)
        m, w = dit_model(cfg, seed=16, dtype="bf16")
        outs[flag] = m.euler_sample(x0, z, c, spk, 10)
        del m
    for b in range(B):
        assert cosine(outs["1"][b], outs["0"][b]) >= 0.9999, b
    o = orc.DiT(cfg, bf16_weights(w))
    for b in (0, 9, 10, 22):
        ref = o.euler_sample(x0[b], z[b], c[b], spk[b] if adaln else None, 10)
        assert cosine(outs["1"][b], ref) >= 0.999, b
        assert rel_err(outs["1"][b], ref) < 2e-3, b


@pytest.mark.parametrize("adaln,B", [(True, 1), (False, 3), (True, 4)])
def test_grid_euler_loop_matches_launch_chain(monkeypatch, adaln, B):
    """fp32, small batch: the grid-persistent Euler loop (one launch for all
    10 steps, CTTS_DIT_GRID unset) against the per-step launch chain
    (CTTS_DIT_GRID=0) and the oracle, twice in a row (the second launch
    must not take the first one's exchange words for its own)."""
    cfg = DiTConfig(adaln=adaln)
    x0, z, c = rnd(31, (B, 64)), rnd(32, (B, 768)), rnd(33, (B, 64))
    spk = z if adaln else None
    outs = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("CTTS_DIT_GRID", flag)
        m, w = dit_model(cfg, seed=26)
        outs[flag] = [m.euler_sample(x0, z, c, spk, 10) for _ in range(2)]
        del m
    assert np.array_equal(outs["1"][0], outs["1"][1])
    o = orc.DiT(cfg, w)
    for b in range(B):
        assert rel_err(outs["1"][0][b], outs["0"][0][b]) < 1e-5, b
        ref = o.euler_sample(x0[b], z[b], c[b], spk[b] if adaln else None, 10)
        assert rel_err(outs["1"][0][b], ref) < 1e-4, b


def test_grid_euler_loop_alternating_batches(monkeypatch):
    """One model, grid-persistent loop launches of batch 3, 1, 3, 2 in turn:
    each batch size lays out its exchange words differently in the shared
    workspace, so words left by the previous launch sit where the next one
    polls; their older generation tag must keep them from being taken.
    Every launch matches the per-utterance oracle (1e-4)."""
    monkeypatch.delenv("CTTS_DIT_GRID", raising=False)
    cfg = DiTConfig(adaln=True)
    m, w = dit_model(cfg, seed=27)
    o = orc.DiT(cfg, w)
    x0, z, c = rnd(41, (3, 64)), rnd(42, (3, 768)), rnd(43, (3, 64))
    refs = [o.euler_sample(x0[b], z[b], c[b], z[b], 10) for b in range(3)]
    for B in (3, 1, 3, 2):
        out = m.euler_sample(x0[:B], z[:B], c[:B], z[:B], 10)
        for b in range(B):
            assert rel_err(out[b], refs[b]) < 1e-4, (B, b)


def _scaled_down(cfg, seed, scale):
    from rcutetts_b200 import synth

    w = synth.dit_weights(cfg, seed=seed)
    for i in range(cfg.n_layers):
        w[f"decoder.layers.{i}.mlp.down_proj.weight"] = w[f"decoder.layers.{i}.mlp.down_proj.weight"] * np.float32(scale)
    return w


def test_cluster_fp16_partial_range_falls_back(monkeypatch):
    """Down-projection weights scaled by 1e8: the split-K partials of the
    cluster loop (exchanged as fp16) leave the fp16 range.  The loop flags
    it, the call reruns on the fp32-partial launch chain (bit for bit what
    a CTTS_DIT_CLUSTER=0 handle gives) and later calls of the handle stay on
    the chain."""
    from rcutetts_b200.model import DitW

    cfg = DiTConfig()
    w = _scaled_down(cfg, 16, 1e8)
    B = 12
    x0, z, c = rnd(31, (B, 64)), rnd(32, (B, 768)), rnd(33, (B, 64))
    monkeypatch.setenv("CTTS_DIT_CLUSTER", "0")
    ref = DitW(cfg, "bf16").set_weights(w).euler_sample(x0, z, c, z, 10)
    monkeypatch.setenv("CTTS_DIT_CLUSTER", "1")
    m = DitW(cfg, "bf16").set_weights(w)
    out = m.euler_sample(x0, z, c, z, 10)
    assert np.isfinite(out).all()
    assert np.array_equal(out, ref)
    assert np.array_equal(m.euler_sample(x0, z, c, z, 10), ref)
    o = orc.DiT(cfg, bf16_weights(w))
    for b in (0, 11):
        assert rel_err(out[b], o.euler_sample(x0[b], z[b], c[b], z[b], 10)) < 2e-3, b


def test_cluster_repacks_after_upload():
    """New weights uploaded to a handle whose cluster loop already ran (and
    packed its copy) are what the next run uses: the result equals a fresh
    handle's, bit for bit."""
    from rcutetts_b200 import synth
    from rcutetts_b200.model import DitW

    cfg = DiTConfig()
    w1, w2 = synth.dit_weights(cfg, seed=16), synth.dit_weights(cfg, seed=17)
    B = 12
    x0, z, c = rnd(34, (B, 64)), rnd(35, (B, 768)), rnd(36, (B, 64))
    m = DitW(cfg, "bf16").set_weights(w1)
    first = m.euler_sample(x0, z, c, z, 10)
    m.set_weights(w2)
    again = m.euler_sample(x0, z, c, z, 10)
    fresh = DitW(cfg, "bf16").set_weights(w2).euler_sample(x0, z, c, z, 10)
    assert not np.array_equal(first, again)
    assert np.array_equal(again, fresh)
