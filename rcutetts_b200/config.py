"""Model dimensions of the per-frame decode path.

The reference crate hard-codes its shipped shapes as constants
(rust-codec/src/qwen.rs:17-24, dit.rs:16-25, decoder.rs:10-16); this package
is shape-generic and carries them as configs.  The defaults are the synthetic
shapes the benchmark configurations are quoted on.
"""
from __future__ import annotations

from dataclasses import dataclass, field

# dtype codes shared with the C ABI (include/cutetts_b200.h)
DTYPE_F32 = 0
DTYPE_BF16 = 1


@dataclass(frozen=True)
class LMConfig:
    """Qwen3-style decoder stack (qwen.rs:17-24 at generic shape)."""

    hidden: int = 768
    n_layers: int = 12
    n_heads: int = 12
    n_kv_heads: int = 4
    head_dim: int = 64
    ffn: int = 2048
    vocab: int = 32000
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    qk_norm: bool = True

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim


@dataclass(frozen=True)
class DiTConfig:
    """AudioDiTHead (diffusion_head.py:381-445) at generic shape.

    spk_dim is the width of the AdaLN conditioning vector; the benchmark
    model conditions AdaLN on the LM hidden state (spk_dim == LM hidden).
    """

    latent: int = 64
    hidden: int = 512
    n_heads: int = 8
    n_kv_heads: int = 8
    head_dim: int = 64
    ffn: int = 1536
    n_layers: int = 4
    patch: int = 1
    cond_dim: int = 768
    spk_dim: int = 768
    rms_eps: float = 1e-6
    rope_theta: float = 1e4
    adaln: bool = True
    step_emb: bool = False
    cfg_emb: bool = False

    @property
    def seq(self) -> int:
        return 1 + 2 * self.patch

    @property
    def has_mu_proj(self) -> bool:
        return self.cond_dim != self.hidden


@dataclass(frozen=True)
class LocEncConfig:
    """AudioLocEnc (diffusion_head.py:334-378) + locenc_to_lm_proj
    (model.py:55) at generic shape; the shipped model is hidden 1024,
    ffn 4096, 16 heads / 2 KV heads, 2 layers, patch 2 (locenc.rs:22-24)."""

    latent: int = 64
    hidden: int = 1024
    n_heads: int = 16
    n_kv_heads: int = 2
    head_dim: int = 64
    ffn: int = 4096
    n_layers: int = 2
    patch: int = 2
    out_dim: int = 768
    rms_eps: float = 1e-6
    rope_theta: float = 1e4


@dataclass(frozen=True)
class VAEConfig:
    """CausalDecoder (audio_vae.py:243-292) at generic shape."""

    latent: int = 64
    channels: int = 1024
    strides: tuple = (8, 5, 4, 2)
    depthwise: bool = False

    @property
    def hop(self) -> int:
        h = 1
        for s in self.strides:
            h *= s
        return h


@dataclass(frozen=True)
class FrameConfig:
    """Per-frame AR loop constants (bin/cutetts.rs:429-523 at generic shape)."""

    lm: LMConfig = field(default_factory=LMConfig)
    dit: DiTConfig = field(default_factory=DiTConfig)
    euler_steps: int = 10
    latent_scale: float = 1.0
    latent_bias: float = 0.0
