"""The CPU restatement (oracle/) against the reference's golden vectors.

Two kinds of pins: the reference crate's own weight-free fixtures
(rust-codec/testdata/m1_*, base_sway; gates from tests/m1_ops.rs and
tests/dit_base.rs) and fixtures made by running the reference's torch
modules at the benchmark shapes (tests/golden/make_golden.py).
"""
import numpy as np
import pytest

from conftest import cosine, rel_err
from oracle import oracle as orc
from rcutetts_b200 import synth
from rcutetts_b200.config import DiTConfig, LMConfig, VAEConfig


def maxabs(a, b):
    return float(np.max(np.abs(np.asarray(a) - np.asarray(b))))


# ------------------------------------------------- reference m1 fixtures
def test_m1_conv_d3(golden):
    x, w, b = golden("ref/m1_conv_d3_in.npy"), golden("ref/m1_conv_d3_w.npy"), golden("ref/m1_conv_d3_b.npy")
    y = orc.causal_conv1d(x, w, b, dilation=3, groups=1, pad=9)
    assert maxabs(y, golden("ref/m1_conv_d3_out.npy")) < 1e-4


def test_m1_conv_dw9(golden):
    x, w, b = golden("ref/m1_conv_dw9_in.npy"), golden("ref/m1_conv_dw9_w.npy"), golden("ref/m1_conv_dw9_b.npy")
    y = orc.causal_conv1d(x, w, b, dilation=9, groups=8, pad=27)
    assert maxabs(y, golden("ref/m1_conv_dw9_out.npy")) < 1e-4


def test_m1_transpose_s16(golden):
    x, w, b = golden("ref/m1_trans_s16_in.npy"), golden("ref/m1_trans_s16_w.npy"), golden("ref/m1_trans_s16_b.npy")
    y = orc.causal_transpose_conv1d(x, w, b, stride=16, groups=1, pad=8, out_pad=0)
    assert maxabs(y, golden("ref/m1_trans_s16_out.npy")) < 1e-4


def test_m1_transpose_s3(golden):
    x, w, b = golden("ref/m1_trans_s3_in.npy"), golden("ref/m1_trans_s3_w.npy"), golden("ref/m1_trans_s3_b.npy")
    y = orc.causal_transpose_conv1d(x, w, b, stride=3, groups=1, pad=2, out_pad=1)
    assert maxabs(y, golden("ref/m1_trans_s3_out.npy")) < 1e-4


def test_m1_residual_unit(golden):
    x = golden("ref/m1_resunit_d3_in.npy")
    ones = np.ones(x.shape[0], np.float32)
    h = orc.snake(x, ones)
    h = orc.causal_conv1d(h, golden("ref/m1_resunit_d3_w0.npy"), golden("ref/m1_resunit_d3_b0.npy"), 3, 1, 9)
    h = orc.snake(h, ones)
    h = orc.causal_conv1d(h, golden("ref/m1_resunit_d3_w1.npy"), golden("ref/m1_resunit_d3_b1.npy"), 1, 1, 0)
    assert maxabs(x + h, golden("ref/m1_resunit_d3_out.npy")) < 1e-4


def test_m1_snake(golden):
    y = orc.snake(golden("ref/m1_snake_in.npy"), golden("ref/m1_snake_alpha.npy"))
    assert maxabs(y, golden("ref/m1_snake_out.npy")) < 1e-6


def test_sway_grid(golden):
    got = orc.sway_timesteps(10, -0.8)
    ref = golden("ref/base_sway.npy")
    assert abs(got[0]) < 1e-6 and abs(got[10] - 1) < 1e-6
    assert maxabs(got, ref) < 1e-6


def test_weight_norm_fuse(golden):
    g = golden("weight_norm.npz")
    assert maxabs(orc.fuse_weight_norm(g["g"], g["v"]), g["w"]) < 1e-6


# ------------------------------------------- torch modules at BASELINE shape
def test_lm_layer_config0(golden):
    """config[0]: one fp32 layer, 64-row prefill + 32 single-row decodes,
    every step's output against HF Qwen3 (gate 1e-4 rel, per layer)."""
    g = golden("lm_layer_c0.npz")
    cfg = LMConfig(n_layers=1)
    lm = orc.LM(cfg, synth.lm_weights(cfg, seed=0, with_embed=False))
    cache = lm.new_cache(128)
    outs = [lm.layer(0, g["x_prefill"], cache["k"][0], cache["v"][0], 0)]
    n = 64
    for i in range(32):
        outs.append(lm.layer(0, g["x_decode"][i:i + 1], cache["k"][0], cache["v"][0], n))
        n += 1
    got = np.concatenate(outs, 0)
    ref = g["layer_out"]
    for i in range(got.shape[0]):
        assert rel_err(got[i], ref[i]) < 1e-4, i
    # whole-stack entry (layer + final norm) against HF last_hidden_state
    cache = lm.new_cache(128)
    fin = [lm.forward(g["x_prefill"], cache)]
    for i in range(32):
        fin.append(lm.forward(g["x_decode"][i:i + 1], cache))
    assert rel_err(np.concatenate(fin, 0), g["final_out"]) < 1e-4


def test_lm_stack_config2(golden):
    g = golden("lm_stack_c2.npz")
    cfg = LMConfig()
    lm = orc.LM(cfg, synth.lm_weights(cfg, seed=2))
    cache = lm.new_cache(32)
    outs = [lm.forward(g["x_prefill"], cache)]
    for i in range(g["x_decode"].shape[0]):
        outs.append(lm.forward(g["x_decode"][i:i + 1], cache))
    got = np.concatenate(outs, 0)
    for i in range(got.shape[0]):
        assert rel_err(got[i], g["final_out"][i]) < 1e-4, i
    assert np.array_equal(lm.embed(g["ids"]), g["embed_out"])


def test_embed_out_of_range():
    table = np.zeros((4, 3), np.float32)
    with pytest.raises(IndexError):
        orc.embed_lookup(table, np.array([4]))


def test_dit_config2(golden):
    g = golden("dit_c2.npz")
    cfg = DiTConfig()
    dit = orc.DiT(cfg, synth.dit_weights(cfg, seed=12))
    for b in range(2):
        v = dit.predict(g["x0"][b], float(g["t"]), g["z"][b], g["cond"][b], spk=g["z"][b])
        assert rel_err(v, g["predict_out"][b]) < 1e-4
        x = dit.euler_sample(g["x0"][b], g["z"][b], g["cond"][b], g["z"][b], 10)
        assert rel_err(x, g["euler10_out"][b]) < 1e-4
        assert cosine(x, g["euler10_out"][b]) > 0.9999


# The shipped model's shapes (qwen.rs:17-24, dit.rs:16-26)
LM_SHIPPED = LMConfig(hidden=1024, n_layers=7, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072, vocab=16385)
DIT_SHIPPED = DiTConfig(hidden=1024, n_heads=16, n_kv_heads=2, head_dim=64, ffn=4096, n_layers=4, patch=2,
                        cond_dim=1024, spk_dim=256)


def test_lm_shipped_shape(golden):
    """7 layers, 16/8 heads of 128, FFN 3072 against HF Qwen3Model."""
    g = golden("lm_shipped.npz")
    lm = orc.LM(LM_SHIPPED, synth.lm_weights(LM_SHIPPED, seed=30, with_embed=False))
    cache = lm.new_cache(16)
    outs = [lm.forward(g["x_prefill"], cache)]
    for i in range(g["x_decode"].shape[0]):
        outs.append(lm.forward(g["x_decode"][i:i + 1], cache))
    got = np.concatenate(outs, 0)
    for i in range(got.shape[0]):
        assert rel_err(got[i], g["final_out"][i]) < 1e-4, i


def test_dit_shipped_shape(golden):
    """hidden 1024, 16/2 heads, FFN 4096, patch 2, speaker AdaLN (256),
    mu_proj Identity: predict and the 10-step Euler sample against the
    reference AudioDiTHead."""
    g = golden("dit_shipped.npz")
    dit = orc.DiT(DIT_SHIPPED, synth.dit_weights(DIT_SHIPPED, seed=31))
    for b in range(2):
        v = dit.predict(g["x0"][b], float(g["t"]), g["z"][b], g["cond"][b], spk=g["spk"][b])
        assert rel_err(v, g["predict_out"][b]) < 1e-4
        x = dit.euler_sample(g["x0"][b], g["z"][b], g["cond"][b], g["spk"][b], 10)
        assert rel_err(x, g["euler10_out"][b]) < 1e-4
        assert cosine(x, g["euler10_out"][b]) > 0.9999


def test_dit_plain_and_cfg(golden):
    g, gc = golden("dit_plain.npz"), golden("dit_c2.npz")
    cfg = DiTConfig(adaln=False, n_layers=2)
    dit = orc.DiT(cfg, synth.dit_weights(cfg, seed=13))
    for b in range(2):
        v = dit.predict(gc["x0"][b], 0.7, gc["z"][b], gc["cond"][b])
        assert rel_err(v, g["predict_out"][b]) < 1e-4
        x = dit.euler_sample_cfg(gc["x0"][b], gc["z"][b], g["z_uncond"][b], gc["cond"][b],
                                 g["uncond"][b], None, 10, -0.8, 2.0)
        assert rel_err(x, g["cfg_out"][b]) < 1e-4


def test_vae_config4(golden):
    g = golden("vae_c4.npz")
    cfg = VAEConfig()
    vae = orc.VAE(cfg, synth.vae_weights(cfg, seed=4))
    for b in range(g["latent"].shape[0]):
        wav = vae.decode(g["latent"][b])
        assert rel_err(wav, g["wav"][b]) < 1e-4
        assert cosine(wav, g["wav"][b]) > 0.9999


@pytest.mark.parametrize("name,cfg,seed", [
    ("vae_dw_small", VAEConfig(latent=64, channels=96, strides=(4, 3, 2), depthwise=True), 8),
    ("vae_dw_shipped", VAEConfig(latent=64, channels=1536, strides=(16, 8, 5, 3), depthwise=True), 9),
])
def test_vae_depthwise(golden, name, cfg, seed):
    """The shipped depthwise topology (audio_vae.py:255-280, decode.rs:94-136)
    against the reference CausalDecoder(depthwise=True)."""
    g = golden(name + ".npz")
    vae = orc.VAE(cfg, synth.vae_weights(cfg, seed=seed, fan_in=0.8))
    for b in range(g["latent"].shape[0]):
        wav = vae.decode(g["latent"][b])
        assert rel_err(wav, g["wav"][b]) < 1e-4
        assert cosine(wav, g["wav"][b]) > 0.9999


def test_vae_causal_prefix():
    """Causality: the first T1*hop samples depend only on the first T1 frames
    (a size-independent property also used at full size on the GPU)."""
    cfg = VAEConfig(channels=64, strides=(4, 2))
    vae = orc.VAE(cfg, synth.vae_weights(cfg, seed=5))
    lat = np.random.default_rng(5).standard_normal((64, 7), dtype=np.float32)
    full = vae.decode(lat)
    part = vae.decode(lat[:, :4])
    assert np.array_equal(full[:4 * cfg.hop], part)


@pytest.mark.parametrize("rows", [3, 37])
def test_linear_threads_bitwise(rows):
    """Few rows (eight-output FMA panels) and many rows (16 rows side by
    side): bitwise the same for any thread count, and the many-row path
    bitwise equal to running its rows one at a time."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((rows, 700), dtype=np.float32)
    W = rng.standard_normal((2000, 700), dtype=np.float32)
    b = rng.standard_normal(2000, dtype=np.float32)
    prev = orc.get_threads()
    try:
        orc.set_threads(1)
        one = orc.linear(x, W, b)
        orc.set_threads(4)
        four = orc.linear(x, W, b)
    finally:
        orc.set_threads(prev)
    assert np.array_equal(one, four)
    by_row = np.concatenate([orc.linear(x[i:i + 1], W, b) for i in range(rows)])
    assert np.array_equal(one, by_row)
    ref = (x.astype(np.float64) @ W.T.astype(np.float64)) + b
    assert rel_err(one, ref) < 1e-5


def test_locenc_vs_torch_module(golden):
    """The LocEnc restatement (locenc.rs:222-255 + locenc_to_lm_proj) against
    the reference's AudioLocEnc torch module (tests/golden/make_golden.py),
    at a small shape and at the shipped shape (hidden 1024, 16/2 heads)."""
    from rcutetts_b200 import synth
    from rcutetts_b200.config import LocEncConfig

    g = golden("locenc.npz")
    for tag, cfg, seed in (("small", LocEncConfig(hidden=256, n_heads=4, n_kv_heads=2, ffn=512, out_dim=128), 17),
                           ("shipped", LocEncConfig(), 18)):
        o = orc.LocEnc(cfg, synth.locenc_weights(cfg, seed))
        got = o.embed(g[f"{tag}_x"])
        ref = g[f"{tag}_out"].reshape(got.shape)
        assert rel_err(got, ref) < 1e-4, tag
