"""Checkpoint layouts of the shipped model (the crate's manifests, copied to
tests/golden/ref/manifests.json by import_reference_fixtures.py): the
synthetic weight generators produce exactly the shipped tensor names and
shapes at the shipped configurations, so the loaders that the GPU tests
feed with manifest-shaped checkpoints see the real file's layout
(qwen.rs:75-120, dit.rs:27-159, locenc.rs:88, weights.rs:98-186)."""
import json
import os
from dataclasses import replace

import pytest

from rcutetts_b200 import synth
from rcutetts_b200.config import DiTConfig, LMConfig, LocEncConfig, VAEConfig

HERE = os.path.dirname(os.path.abspath(__file__))

LM_SHIPPED = LMConfig(hidden=1024, n_layers=7, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072, vocab=16385)
DIT_DISTILL = DiTConfig(hidden=1024, n_heads=16, n_kv_heads=2, head_dim=64, ffn=4096, n_layers=4, patch=2,
                        cond_dim=1024, spk_dim=256, step_emb=True, cfg_emb=True)
LOCENC_SHIPPED = replace(LocEncConfig(), out_dim=1024)
VAE_SHIPPED = VAEConfig(latent=64, channels=1536, strides=(16, 8, 5, 3), depthwise=True)


def manifests():
    with open(os.path.join(HERE, "golden", "ref", "manifests.json")) as f:
        return json.load(f)


def checkpoint_tensors(tag, w):
    """Our generator's tensors under the names the shipped file uses (the
    VAE's conv weights as their weight-norm pairs, g = 1 per channel)."""
    import numpy as np

    if tag == "lm":
        return {"qwen_backbone." + k: v for k, v in w.items()}
    if tag == "locenc":
        return {(k if k.startswith("locenc_to_lm_proj") else "locenc." + k): v for k, v in w.items()}
    if tag == "vae":
        out = {}
        for k, v in w.items():
            if k.endswith(".weight"):
                out["decoder." + k + "_g"] = np.ones((v.shape[0], 1, 1), np.float32)
                out["decoder." + k + "_v"] = v
            else:
                out["decoder." + k] = v
        return out
    return dict(w)


def checkpoint_names(tag, w):
    return {k: list(v.shape) for k, v in checkpoint_tensors(tag, w).items()}


@pytest.mark.parametrize("tag", ["lm", "dit", "locenc", "vae"])
def test_synth_matches_shipped_manifest(tag):
    gen = {"lm": lambda: synth.lm_weights(LM_SHIPPED, seed=1, with_embed=True),
           "dit": lambda: synth.dit_weights(DIT_DISTILL, seed=1),
           "locenc": lambda: synth.locenc_weights(LOCENC_SHIPPED, seed=1),
           "vae": lambda: synth.vae_weights(VAE_SHIPPED, seed=1)}[tag]
    ours = checkpoint_names(tag, gen())
    man = manifests()[tag]
    assert sorted(ours) == sorted(man)
    for name, (shape, _) in man.items():
        assert ours[name] == shape, name


def test_manifest_dtypes():
    """bf16 LM and LocEnc, fp32 DiT head and VAE (dit.rs:1-3, weights.rs:3)."""
    m = manifests()
    assert {d for _, d in m["lm"].values()} == {"bfloat16"}
    assert {d for _, d in m["locenc"].values()} == {"bfloat16"}
    assert {d for _, d in m["dit"].values()} == {"float32"}
    assert {d for _, d in m["vae"].values()} == {"float32"}
