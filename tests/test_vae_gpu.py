"""VAE decoder (config[4] topology) on the GPU against the torch golden
vectors and the oracle; causality at full size; the reference's ffi.rs
entry points with weight-norm checkpoints."""
import ctypes as C

import numpy as np
import pytest

from conftest import cosine, rel_err
from helpers import bf16_weights, rnd
from oracle import oracle as orc
from rcutetts_b200 import synth
from rcutetts_b200.config import VAEConfig

pytestmark = pytest.mark.gpu


def vae(cfg, seed, dtype="f32"):
    from rcutetts_b200.model import DecoderW

    w = synth.vae_weights(cfg, seed=seed)
    return DecoderW(cfg, dtype).set_weights(w), w


def test_config4_vs_golden(golden):
    g = golden("vae_c4.npz")
    m, w = vae(VAEConfig(), 4)
    wav = m.decode(g["latent"])
    for b in range(wav.shape[0]):
        assert rel_err(wav[b], g["wav"][b]) < 1e-4
        assert cosine(wav[b], g["wav"][b]) >= 0.9999


def test_bf16_vs_oracle():
    cfg = VAEConfig()
    m, w = vae(cfg, 4, "bf16")
    o = orc.VAE(cfg, bf16_weights(w))
    lat = rnd(5, (64, 5))
    assert cosine(m.decode(lat), o.decode(lat)) >= 0.999


def test_causal_prefix_full_size():
    """config[4] size (T=400, hop 320): the first 200 frames' samples do not
    depend on later frames, bit for bit; batch rows are independent."""
    m, _ = vae(VAEConfig(), 4)
    lat = rnd(6, (2, 64, 400))
    full = m.decode(lat)
    half = m.decode(lat[:, :, :200])
    assert full.shape == (2, 400 * 320)
    assert np.array_equal(full[:, :200 * 320], half)
    one = m.decode(lat[1:2])
    assert np.array_equal(one[0], full[1])
    assert np.all(np.abs(full) <= 1.0)


def test_reference_ffi_with_weight_norm(tmp_path):
    """cutetts_vae_load/decode (ffi.rs:19-65) on a checkpoint that stores
    weight_g/weight_v pairs under decoder.*; fused at load (conv.rs:12-30)."""
    from safetensors.numpy import save_file

    from rcutetts_b200 import _lib

    cfg = VAEConfig(channels=64, strides=(4, 2))
    w = synth.vae_weights(cfg, seed=7)
    st = {}
    rng = np.random.default_rng(7)
    fused = {}
    for k, v in w.items():
        if k.endswith(".weight"):
            g = (rng.random((v.shape[0], 1, 1), dtype=np.float32) + 0.5).astype(np.float32)
            st["decoder." + k[:-len("weight")] + "weight_g"] = g
            st["decoder." + k[:-len("weight")] + "weight_v"] = v
            fused[k] = orc.fuse_weight_norm(g, v)
        else:
            st["decoder." + k] = v
            fused[k] = v
    path = str(tmp_path / "vae.safetensors")
    save_file(st, path)
    lib = _lib.load()
    h = lib.cutetts_vae_load(path.encode())
    assert h
    lat = rnd(8, (64, 9))
    wav = np.empty(9 * cfg.hop, np.float32)
    assert lib.cutetts_vae_decode(h, lat.ctypes.data_as(C.POINTER(C.c_float)), 9,
                                  wav.ctypes.data_as(C.POINTER(C.c_float))) == 0
    assert lib.cutetts_vae_decode(h, lat.ctypes.data_as(C.POINTER(C.c_float)), 0,
                                  wav.ctypes.data_as(C.POINTER(C.c_float))) == -1
    lib.cutetts_vae_free(h)
    ref = orc.VAE(cfg, fused).decode(lat)
    assert rel_err(wav, ref) < 1e-4


def test_stage_profile_env(capfd, monkeypatch):
    """CUTETTS_PROFILE=1 prints one "[prof]" line per decoder stage
    (decode.rs:12-24) without changing the waveform."""
    cfg = VAEConfig(channels=128, strides=(4, 2))
    m, _ = vae(cfg, 8, "bf16")
    lat = rnd(9, (2, 64, 6))
    ref = m.decode(lat)
    monkeypatch.setenv("CUTETTS_PROFILE", "1")
    got = m.decode(lat)
    err = capfd.readouterr().err
    assert np.array_equal(got, ref)
    for name in ("front conv", "stage 0 snake+transpose", "stage 1 resunit d9", "final snake+conv+tanh"):
        assert f"[prof] {name}" in err, err
