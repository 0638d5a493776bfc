"""Shared builders for the parity tests (device models from synth weights)."""
import numpy as np

from rcutetts_b200 import synth


def lm_model(cfg, seed, dtype="f32", with_embed=False):
    from rcutetts_b200.model import QwenW

    w = synth.lm_weights(cfg, seed=seed, with_embed=with_embed)
    m = QwenW(cfg, dtype).set_weights(w)
    return m, w


def dit_model(cfg, seed, dtype="f32"):
    from rcutetts_b200.model import DitW

    w = synth.dit_weights(cfg, seed=seed)
    return DitW(cfg, dtype).set_weights(w), w


def bf16_weights(w: dict) -> dict:
    """The weights the bf16 device path stores (norm gains stay float32)."""
    out = {}
    for k, v in w.items():
        is_norm = k.endswith("norm.weight") or "layernorm" in k or k.endswith("q_norm.weight") \
            or k.endswith("k_norm.weight") or k.endswith(".bias") or "cfg_strength_embedding.0" in k
        out[k] = v if is_norm else synth.bf16_round(v)
    return out


def rnd(seed, shape, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(scale))
