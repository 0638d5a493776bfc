"""Seeded random-init weights with the reference checkpoint's tensor names.

There are no checkpoints on this machine, so tests and the benchmark use
N(0, 0.02) weights (norm gains 1, Snake alpha 1) drawn from numpy's PCG64 in a
fixed order.  Names follow the reference safetensors layout
(rust-codec/qwen_manifest.json, dit_manifest.json, weights_manifest.json) so
the same dictionaries can be written to a .safetensors file and read by the
C ABI loader.
"""
from __future__ import annotations

import numpy as np

from .config import DiTConfig, LMConfig, VAEConfig

STD = 0.02


def _normal(rng: np.random.Generator, shape, std=STD) -> np.ndarray:
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def lm_weights(cfg: LMConfig, seed: int, with_embed: bool = True) -> dict:
    """Qwen3 backbone tensors, names without the `qwen_backbone.` prefix."""
    rng = np.random.default_rng(seed)
    H, F = cfg.hidden, cfg.ffn
    w = {}
    if with_embed:
        w["embed_tokens.weight"] = _normal(rng, (cfg.vocab, H))
    for i in range(cfg.n_layers):
        p = f"layers.{i}."
        w[p + "input_layernorm.weight"] = np.ones(H, np.float32)
        w[p + "post_attention_layernorm.weight"] = np.ones(H, np.float32)
        w[p + "self_attn.q_proj.weight"] = _normal(rng, (cfg.q_dim, H))
        w[p + "self_attn.k_proj.weight"] = _normal(rng, (cfg.kv_dim, H))
        w[p + "self_attn.v_proj.weight"] = _normal(rng, (cfg.kv_dim, H))
        w[p + "self_attn.o_proj.weight"] = _normal(rng, (H, cfg.q_dim))
        w[p + "self_attn.q_norm.weight"] = np.ones(cfg.head_dim, np.float32)
        w[p + "self_attn.k_norm.weight"] = np.ones(cfg.head_dim, np.float32)
        w[p + "mlp.gate_proj.weight"] = _normal(rng, (F, H))
        w[p + "mlp.up_proj.weight"] = _normal(rng, (F, H))
        w[p + "mlp.down_proj.weight"] = _normal(rng, (H, F))
    w["norm.weight"] = np.ones(H, np.float32)
    return w


def locenc_weights(cfg, seed: int) -> dict:
    """AudioLocEnc tensors (names of the module, without `locenc.`) plus
    locenc_to_lm_proj.*; norm gains 1."""
    rng = np.random.default_rng(seed)
    H, F = cfg.hidden, cfg.ffn
    qd, kvd = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    w = {"special_token": rng.standard_normal((1, 1, 1, H), dtype=np.float32),
         "in_proj.weight": _normal(rng, (H, cfg.latent)), "in_proj.bias": _normal(rng, (H,))}
    for i in range(cfg.n_layers):
        p = f"encoder.layers.{i}."
        w[p + "input_layernorm.weight"] = np.ones(H, np.float32)
        w[p + "post_attention_layernorm.weight"] = np.ones(H, np.float32)
        w[p + "self_attn.q_proj.weight"] = _normal(rng, (qd, H))
        w[p + "self_attn.k_proj.weight"] = _normal(rng, (kvd, H))
        w[p + "self_attn.v_proj.weight"] = _normal(rng, (kvd, H))
        w[p + "self_attn.o_proj.weight"] = _normal(rng, (H, qd))
        w[p + "mlp.gate_proj.weight"] = _normal(rng, (F, H))
        w[p + "mlp.up_proj.weight"] = _normal(rng, (F, H))
        w[p + "mlp.down_proj.weight"] = _normal(rng, (H, F))
    w["encoder.norm.weight"] = np.ones(H, np.float32)
    w["locenc_to_lm_proj.weight"] = _normal(rng, (cfg.out_dim, H))
    w["locenc_to_lm_proj.bias"] = _normal(rng, (cfg.out_dim,))
    return w


def dit_weights(cfg: DiTConfig, seed: int) -> dict:
    """AudioDiTHead tensors, names without the `head.` prefix."""
    rng = np.random.default_rng(seed)
    H, L, F = cfg.hidden, cfg.latent, cfg.ffn
    kvd = cfg.n_kv_heads * cfg.head_dim
    w = {}
    w["in_proj.weight"] = _normal(rng, (H, L))
    w["in_proj.bias"] = _normal(rng, (H,))
    w["cond_proj.weight"] = _normal(rng, (H, L))
    w["cond_proj.bias"] = _normal(rng, (H,))
    if cfg.has_mu_proj:
        w["mu_proj.weight"] = _normal(rng, (H, cfg.cond_dim))
        w["mu_proj.bias"] = _normal(rng, (H,))
    w["out_proj.weight"] = _normal(rng, (L, H))
    w["out_proj.bias"] = _normal(rng, (L,))
    for m in ("time_mlp", "delta_time_mlp") + (("step_size_embedding",) if cfg.step_emb else ()):
        w[f"{m}.linear_1.weight"] = _normal(rng, (H, H))
        w[f"{m}.linear_1.bias"] = _normal(rng, (H,))
        w[f"{m}.linear_2.weight"] = _normal(rng, (H, H))
        w[f"{m}.linear_2.bias"] = _normal(rng, (H,))
    if cfg.cfg_emb:
        w["cfg_strength_embedding.0.weight"] = _normal(rng, (H, 1))
        w["cfg_strength_embedding.2.weight"] = _normal(rng, (H, H))
    for i in range(cfg.n_layers):
        p = f"decoder.layers.{i}."
        w[p + "input_layernorm.weight"] = np.ones(H, np.float32)
        w[p + "post_attention_layernorm.weight"] = np.ones(H, np.float32)
        w[p + "self_attn.q_proj.weight"] = _normal(rng, (cfg.n_heads * cfg.head_dim, H))
        w[p + "self_attn.k_proj.weight"] = _normal(rng, (kvd, H))
        w[p + "self_attn.v_proj.weight"] = _normal(rng, (kvd, H))
        w[p + "self_attn.o_proj.weight"] = _normal(rng, (H, cfg.n_heads * cfg.head_dim))
        w[p + "mlp.gate_proj.weight"] = _normal(rng, (F, H))
        w[p + "mlp.up_proj.weight"] = _normal(rng, (F, H))
        w[p + "mlp.down_proj.weight"] = _normal(rng, (H, F))
        if cfg.adaln:
            w[p + "speaker_adaln.weight"] = _normal(rng, (6 * H, cfg.spk_dim))
    w["decoder.norm.weight"] = np.ones(H, np.float32)
    return w


def frame_weights(lm_hidden: int, latent: int, seed: int) -> dict:
    """Stop head (e2e.rs:83-92) and the latent->LM feedback projection.

    The reference feeds each predicted patch back through AudioLocEnc +
    locenc_to_lm_proj (locenc.rs:222-255); the benchmark model replaces that
    with one Linear(latent -> LM hidden), stored as `latent_proj`.
    """
    rng = np.random.default_rng(seed)
    return {
        "stop_predictor.weight": _normal(rng, (2, lm_hidden)),
        "stop_predictor.bias": _normal(rng, (2,)),
        "latent_proj.weight": _normal(rng, (lm_hidden, latent)),
        "latent_proj.bias": _normal(rng, (lm_hidden,)),
    }


def vae_weights(cfg: VAEConfig, seed: int, fan_in: float = 0.0) -> dict:
    """CausalDecoder tensors with weight norm already fused (`.weight`),
    names without the `decoder.` prefix.  Biases are zero, as the
    reference's init_weights (audio_vae.py:90-95) leaves them.  fan_in > 0
    draws every conv weight with std fan_in / sqrt(in_per_group * k) instead
    of the fixed init std, so the signal keeps its scale through deep
    (depthwise) stacks."""
    rng = np.random.default_rng(seed)
    C, L = cfg.channels, cfg.latent

    def _normal(rng, shape):
        std = fan_in / np.sqrt(shape[1] * shape[2]) if fan_in > 0 else STD
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    w = {}
    idx = 0
    if cfg.depthwise:
        w["model.0.weight"] = _normal(rng, (L, 1, 7))
        w["model.0.bias"] = np.zeros(L, np.float32)
        w["model.1.weight"] = _normal(rng, (C, L, 1))
        w["model.1.bias"] = np.zeros(C, np.float32)
        idx = 2
    else:
        w["model.0.weight"] = _normal(rng, (C, L, 7))
        w["model.0.bias"] = np.zeros(C, np.float32)
        idx = 1
    ch = C
    for si, s in enumerate(cfg.strides):
        cin, cout = C >> si, C >> (si + 1)
        b = f"model.{idx}.block."
        w[b + "0.alpha"] = np.ones((1, cin, 1), np.float32)
        w[b + "1.weight"] = _normal(rng, (cin, cout, 2 * s))
        w[b + "1.bias"] = np.zeros(cout, np.float32)
        g = cout if cfg.depthwise else 1
        for r in range(3):
            rb = f"{b}{2 + r}.block."
            w[rb + "0.alpha"] = np.ones((1, cout, 1), np.float32)
            w[rb + "1.weight"] = _normal(rng, (cout, cout // g, 7))
            w[rb + "1.bias"] = np.zeros(cout, np.float32)
            w[rb + "2.alpha"] = np.ones((1, cout, 1), np.float32)
            w[rb + "3.weight"] = _normal(rng, (cout, cout, 1))
            w[rb + "3.bias"] = np.zeros(cout, np.float32)
        idx += 1
        ch = cout
    w[f"model.{idx}.alpha"] = np.ones((1, ch, 1), np.float32)
    w[f"model.{idx + 1}.weight"] = _normal(rng, (1, ch, 7))
    w[f"model.{idx + 1}.bias"] = np.zeros(1, np.float32)
    return w


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16 and widen back to f32 (exact widening,
    simd.rs:283-319).  Used to give the oracle the same weights the bf16
    device path stores."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    r = ((u + rounding) & np.uint32(0xFFFF0000)).astype(np.uint32)
    return r.view(np.float32)


def to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) of round-to-nearest-even(a)."""
    return (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)
