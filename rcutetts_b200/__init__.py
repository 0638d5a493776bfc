"""rcutetts_b200 -- B200 (sm_100a) per-frame decode path of RCuteTTS.

The compute lives in libcutetts_b200.so (hand-written CUDA behind the C ABI
of include/cutetts_b200.h); this package is the host-side mirror of the
reference crate's model API (see rcutetts_b200.model).
"""
from .config import DiTConfig, FrameConfig, LMConfig, VAEConfig  # noqa: F401

_MODEL_NAMES = {
    "QwenW", "QwenCache", "load_qwen_weights", "prefill", "decode_step", "decode_step_dev",
    "embed_lookup", "DitW", "load_dit_weights", "sway_timesteps", "FrameEngine", "DecoderW",
    "load_decoder_weights", "decode",
}

__all__ = ["LMConfig", "DiTConfig", "VAEConfig", "FrameConfig"] + sorted(_MODEL_NAMES)


def __getattr__(name):
    # Model classes need the CUDA library; import them lazily so config and
    # synth stay importable while the library is being built.
    if name in _MODEL_NAMES:
        from . import model

        return getattr(model, name)
    raise AttributeError(name)
