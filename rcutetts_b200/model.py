"""Host-side mirror of the reference crate's model API over the C ABI.

Names follow rust-codec/src: load_qwen_weights / QwenCache / prefill /
decode_step / embed_lookup (qwen.rs), load_dit_weights / predict /
euler_sample / euler_sample_cfg / sway_timesteps (dit.rs), load_decoder_weights
/ decode (weights.rs, decode.rs), stop_logits (e2e.rs).  Arrays are numpy
float32 on the host; the *_dev methods take torch CUDA tensors.  All compute
runs in libcutetts_b200.so on the GPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import check
from .config import DiTConfig, LMConfig, VAEConfig

fp = C.POINTER(C.c_float)


def _f(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return None if a is None else a.ctypes.data_as(fp)


def _shape(a):
    return (C.c_int64 * a.ndim)(*a.shape), a.ndim


def _dtype_code(dtype) -> int:
    if dtype in (_lib.F32, "f32", "fp32", "float32"):
        return _lib.F32
    if dtype in (_lib.BF16, "bf16", "bfloat16"):
        return _lib.BF16
    raise ValueError(f"unknown dtype {dtype}")


def _stream(stream):
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream  # torch.cuda.Stream


def _tensor_ptr(t):
    assert t.is_cuda and t.is_contiguous(), "expected a contiguous CUDA tensor"
    return t.data_ptr()


class _Handle:
    _free = None

    def __init__(self):
        self.h = C.c_void_p()

    def close(self):
        if self.h and self.h.value:
            getattr(_lib.load(), self._free)(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _set_tensor(fn, h, name, arr):
    a = _f(arr)
    shp, nd = _shape(a)
    check(fn(h, name.encode(), a.ctypes.data_as(C.c_void_p), _lib.F32, shp, nd))


# ------------------------------------------------------------------- LM
class QwenW(_Handle):
    """Device-resident Qwen3 stack (QwenW, qwen.rs:26-44)."""

    _free = "ctts_lm_free"

    def __init__(self, cfg: LMConfig, dtype="f32", device: int = 0):
        super().__init__()
        self.cfg = cfg
        self.dtype = _dtype_code(dtype)
        c = _lib.LMConfigC(cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                           cfg.ffn, cfg.vocab, cfg.rms_eps, cfg.rope_theta, int(cfg.qk_norm),
                           self.dtype)
        check(_lib.load().ctts_lm_create(C.byref(c), device, C.byref(self.h)))

    def set_tensor(self, name: str, arr) -> None:
        _set_tensor(_lib.load().ctts_lm_set_tensor, self.h, name, arr)

    def set_weights(self, weights: dict) -> "QwenW":
        for k, v in weights.items():
            self.set_tensor(k, v)
        return self

    def load(self, path: str, prefix: str = "qwen_backbone.") -> "QwenW":
        check(_lib.load().ctts_lm_load(self.h, path.encode(), prefix.encode()))
        return self

    @property
    def missing(self) -> int:
        return _lib.load().ctts_lm_missing(self.h)

    def embed_lookup(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int64)
        out = np.empty((ids.size, self.cfg.hidden), np.float32)
        check(_lib.load().ctts_lm_embed_lookup(self.h, ids.ctypes.data_as(C.POINTER(C.c_int64)),
                                               ids.size, _p(out)))
        return out


def load_qwen_weights(path: str, cfg: LMConfig, dtype="f32", device: int = 0,
                      prefix: str = "qwen_backbone.") -> QwenW:
    """load_qwen_weights (qwen.rs:75-120) at generic shape."""
    return QwenW(cfg, dtype, device).load(path, prefix)


class QwenCache(_Handle):
    """Batched KV cache (QwenCache, qwen.rs:139-149)."""

    _free = "ctts_kv_free"

    def __init__(self, lm: QwenW, batch: int = 1, capacity: int = 1024):
        super().__init__()
        self.lm = lm
        self.batch = batch
        self.capacity = capacity
        check(_lib.load().ctts_kv_alloc(lm.h, batch, capacity, C.byref(self.h)))

    def len(self, b: int = 0) -> int:
        r = _lib.load().ctts_kv_len(self.h, b)
        if r < 0:
            check(r)
        return r

    def set_len(self, b: int, n: int) -> None:
        check(_lib.load().ctts_kv_set_len(self.h, b, n))

    def reset(self) -> None:
        check(_lib.load().ctts_kv_reset(self.h))


def prefill(w: QwenW, x, cache: QwenCache, b: int = 0) -> np.ndarray:
    """prefill (qwen.rs:379-391): rows x [T, H] of utterance b -> [T, H]."""
    x = _f(x)
    out = np.empty_like(x)
    check(_lib.load().ctts_lm_prefill(w.h, cache.h, b, _p(x), x.shape[0], _p(out)))
    return out


def decode_step(w: QwenW, x, cache: QwenCache) -> np.ndarray:
    """decode_step (qwen.rs:394-406) for every utterance: x [B, H] -> [B, H]."""
    x = _f(x).reshape(cache.batch, w.cfg.hidden)
    out = np.empty_like(x)
    check(_lib.load().ctts_lm_decode_step(w.h, cache.h, _p(x), _p(out)))
    return out


def decode_step_dev(w: QwenW, x, cache: QwenCache, out, stream=None) -> None:
    check(_lib.load().ctts_lm_decode_step_dev(w.h, cache.h, _tensor_ptr(x), _tensor_ptr(out),
                                              _stream(stream)))


def embed_lookup(w: QwenW, ids) -> np.ndarray:
    return w.embed_lookup(ids)


# ------------------------------------------------------------------- DiT
class DitW(_Handle):
    """Device-resident AudioDiTHead (DitW, dit.rs:27-68)."""

    _free = "ctts_dit_free"

    def __init__(self, cfg: DiTConfig, dtype="f32", device: int = 0):
        super().__init__()
        self.cfg = cfg
        self.dtype = _dtype_code(dtype)
        c = _lib.DiTConfigC(cfg.latent, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                            cfg.ffn, cfg.n_layers, cfg.patch, cfg.cond_dim, cfg.spk_dim,
                            cfg.rms_eps, cfg.rope_theta, int(cfg.adaln), int(cfg.step_emb),
                            int(cfg.cfg_emb), self.dtype)
        check(_lib.load().ctts_dit_create(C.byref(c), device, C.byref(self.h)))

    def set_tensor(self, name: str, arr) -> None:
        _set_tensor(_lib.load().ctts_dit_set_tensor, self.h, name, arr)

    def set_weights(self, weights: dict) -> "DitW":
        for k, v in weights.items():
            self.set_tensor(k, v)
        return self

    def load(self, path: str, prefix: str = "head.") -> "DitW":
        check(_lib.load().ctts_dit_load(self.h, path.encode(), prefix.encode()))
        return self

    @property
    def missing(self) -> int:
        return _lib.load().ctts_dit_missing(self.h)

    def _pl(self):
        return self.cfg.patch * self.cfg.latent

    def predict(self, x, t, z, cond, dt=0.0, spk=None, cfg_w=0.0) -> np.ndarray:
        x, z, cond = _f(x), _f(z), _f(cond)
        B = x.size // self._pl()
        v = np.empty((B, self._pl()), np.float32)
        spk = _f(spk) if spk is not None else None
        check(_lib.load().ctts_dit_predict(self.h, B, _p(x), t, _p(z), _p(cond), dt, _p(spk), cfg_w,
                                           _p(v)))
        return v

    def euler_sample(self, x0, z, cond, spk, steps, cfg_w=0.0) -> np.ndarray:
        x0, z, cond = _f(x0), _f(z), _f(cond)
        B = x0.size // self._pl()
        x = np.empty((B, self._pl()), np.float32)
        spk = _f(spk) if spk is not None else None
        check(_lib.load().ctts_dit_euler_sample(self.h, B, _p(x0), _p(z), _p(cond), _p(spk), steps,
                                                cfg_w, _p(x)))
        return x

    def euler_sample_cfg(self, x0, z_c, z_u, cond, uncond, spk, steps, coeff, cfg) -> np.ndarray:
        a = [_f(v) for v in (x0, z_c, z_u, cond, uncond)]
        B = a[0].size // self._pl()
        x = np.empty((B, self._pl()), np.float32)
        spk = _f(spk) if spk is not None else None
        check(_lib.load().ctts_dit_euler_sample_cfg(self.h, B, *[_p(v) for v in a], _p(spk), steps,
                                                    coeff, cfg, _p(x)))
        return x


def load_dit_weights(path: str, cfg: DiTConfig, dtype="f32", device: int = 0,
                     prefix: str = "head.") -> DitW:
    return DitW(cfg, dtype, device).load(path, prefix)


def sway_timesteps(steps: int, coeff: float) -> np.ndarray:
    out = np.empty(steps + 1, np.float32)
    check(_lib.load().ctts_sway_timesteps(steps, coeff, _p(out)))
    return out


# ------------------------------------------------------------- engine
class FrameEngine(_Handle):
    """Per-frame AR loop body (bin/cutetts.rs:429-523) for a batch of
    utterances; one frame = one CUDA-graph replay."""

    _free = "ctts_engine_free"

    def __init__(self, lm: QwenW, dit: DitW, heads: dict, batch: int, capacity: int,
                 euler_steps: int = 10, latent_scale: float = 1.0, latent_bias: float = 0.0,
                 use_graph: bool = True, groups: int = 1, cfg_strength: float = 0.0,
                 sway_coeff: float = 0.0):
        super().__init__()
        self.lm, self.dit = lm, dit
        self.batch = batch
        c = _lib.EngineConfigC(batch, capacity, euler_steps, latent_scale, latent_bias, int(use_graph),
                               groups, cfg_strength, sway_coeff)
        check(_lib.load().ctts_engine_create(lm.h, dit.h, C.byref(c), C.byref(self.h)))
        sw, sb = _f(heads["stop_predictor.weight"]), _f(heads["stop_predictor.bias"])
        pw, pb = _f(heads["latent_proj.weight"]), _f(heads["latent_proj.bias"])
        check(_lib.load().ctts_engine_set_heads(self.h, _p(sw), _p(sb), _p(pw), _p(pb)))
        self.pl = dit.cfg.patch * dit.cfg.latent

    def prefill(self, b: int, x, cond0) -> None:
        x, cond0 = _f(x), _f(cond0)
        check(_lib.load().ctts_engine_prefill(self.h, b, _p(x), x.shape[0], _p(cond0)))

    def prefill_uncond(self, b: int, x, cond0) -> None:
        """CFG mode: the unconditional branch of utterance b."""
        x, cond0 = _f(x), _f(cond0)
        check(_lib.load().ctts_engine_prefill_uncond(self.h, b, _p(x), x.shape[0], _p(cond0)))

    def set_speaker(self, b: int, spk) -> None:
        """AdaLN speaker embedding [spk_dim] of utterance b (required when the
        DiT's spk_dim differs from the LM hidden width)."""
        spk = np.ascontiguousarray(spk, dtype=np.float32).reshape(-1)
        check(_lib.load().ctts_engine_set_speaker(self.h, b, _p(spk)))

    def step(self, noise):
        noise = _f(noise).reshape(self.batch, self.pl)
        lat = np.empty_like(noise)
        stop = np.empty((self.batch, 2), np.float32)
        check(_lib.load().ctts_engine_step(self.h, _p(noise), _p(lat), _p(stop)))
        return lat, stop

    def step_dev(self, noise, lat=None, stop=None, stream=None) -> None:
        check(_lib.load().ctts_engine_step_dev(
            self.h, _tensor_ptr(noise), _tensor_ptr(lat) if lat is not None else None,
            _tensor_ptr(stop) if stop is not None else None, _stream(stream)))

    @property
    def launches_per_step(self) -> int:
        return _lib.load().ctts_engine_launches_per_step(self.h)

    # per-frame phase timers (--profile-steps, bin/cutetts.rs:328-350)
    PHASES = ("stop", "dit", "feedback", "lm")

    def set_profile(self, on: bool) -> None:
        check(_lib.load().ctts_engine_set_profile(self.h, int(bool(on))))

    def profile_stats(self) -> dict:
        """{phase: {"n", "mean_ms", "p50_ms", "p99_ms"}} over the profiled frames."""
        out = {}
        for i, name in enumerate(self.PHASES):
            st = (C.c_float * 3)()
            n = C.c_int()
            check(_lib.load().ctts_engine_profile_stats(self.h, i, st, C.byref(n)))
            out[name] = {"n": n.value, "mean_ms": st[0], "p50_ms": st[1], "p99_ms": st[2]}
        return out

    def profile_report(self) -> str:
        buf = C.create_string_buffer(1024)
        n = _lib.load().ctts_engine_profile_report(self.h, buf, 1024)
        if n < 0:
            check(n)
        return buf.value.decode()

    @property
    def stream_ptr(self) -> int:
        return _lib.load().ctts_engine_stream(self.h) or 0


# ------------------------------------------------------------------- VAE
class DecoderW(_Handle):
    """Device-resident CausalDecoder (DecoderW, weights.rs:34-44)."""

    _free = "ctts_vae_free"

    def __init__(self, cfg: VAEConfig, dtype="f32", device: int = 0):
        super().__init__()
        self.cfg = cfg
        st = (C.c_int * 8)(*(list(cfg.strides) + [0] * (8 - len(cfg.strides))))
        c = _lib.VAEConfigC(cfg.latent, cfg.channels, len(cfg.strides), int(cfg.depthwise), st,
                            _dtype_code(dtype))
        check(_lib.load().ctts_vae_create(C.byref(c), device, C.byref(self.h)))

    def set_tensor(self, name: str, arr) -> None:
        _set_tensor(_lib.load().ctts_vae_set_tensor, self.h, name, arr)

    def set_weights(self, weights: dict) -> "DecoderW":
        for k, v in weights.items():
            self.set_tensor(k, v)
        return self

    def load(self, path: str, prefix: str = "decoder.") -> "DecoderW":
        check(_lib.load().ctts_vae_load_file(self.h, path.encode(), prefix.encode()))
        return self

    @property
    def missing(self) -> int:
        return _lib.load().ctts_vae_missing(self.h)

    def decode(self, latent) -> np.ndarray:
        """latent [latent, T] or [B, latent, T] -> wav [T*hop] / [B, T*hop]."""
        lat = _f(latent)
        single = lat.ndim == 2
        if single:
            lat = lat[None]
        B, _, T = lat.shape
        wav = np.empty((B, T * self.cfg.hop), np.float32)
        check(_lib.load().ctts_vae_decode_batch(self.h, B, _p(lat), T, _p(wav)))
        return wav[0] if single else wav

    def decode_dev(self, latent, wav, stream=None) -> None:
        B, _, T = latent.shape
        check(_lib.load().ctts_vae_decode_batch_dev(self.h, B, _tensor_ptr(latent), T,
                                                    _tensor_ptr(wav), _stream(stream)))


class LocEncW(_Handle):
    """Device-resident LocEnc + locenc_to_lm_proj (LocencW, locenc.rs:36-44;
    embed = locenc_embed, locenc.rs:222-255 / model.py:128-130)."""

    _free = "ctts_locenc_free"

    def __init__(self, cfg, dtype="f32", device: int = 0):
        super().__init__()
        self.cfg = cfg
        c = _lib.LocEncConfigC(cfg.latent, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn,
                               cfg.n_layers, cfg.patch, cfg.out_dim, cfg.rms_eps, cfg.rope_theta,
                               _dtype_code(dtype))
        check(_lib.load().ctts_locenc_create(C.byref(c), device, C.byref(self.h)))

    def set_tensor(self, name: str, arr) -> None:
        _set_tensor(_lib.load().ctts_locenc_set_tensor, self.h, name, arr)

    def set_weights(self, weights: dict) -> "LocEncW":
        for k, v in weights.items():
            self.set_tensor(k, v)
        return self

    def load(self, path: str, prefix: str = "locenc.") -> "LocEncW":
        check(_lib.load().ctts_locenc_load(self.h, path.encode(), prefix.encode()))
        return self

    @property
    def missing(self) -> int:
        return _lib.load().ctts_locenc_missing(self.h)

    def embed(self, x) -> np.ndarray:
        """x [n, patch, latent] (or [B, T, patch, latent]) -> [n, out_dim]."""
        a = _f(x).reshape(-1, self.cfg.patch, self.cfg.latent)
        out = np.empty((a.shape[0], self.cfg.out_dim), np.float32)
        check(_lib.load().ctts_locenc_embed(self.h, _p(a), a.shape[0], _p(out)))
        return out


def locenc_embed(w: LocEncW, x, b: int | None = None, t: int | None = None, nth: int = 0) -> np.ndarray:
    """locenc_embed(w, x, b, t, nth) (locenc.rs:222): x [B, T, patch, 64]
    flattened -> [B*T, out_dim]; nth is accepted and ignored."""
    return w.embed(x)


class StreamingDecoder(_Handle):
    """Chunked VAE decode with the convs' left histories carried across
    chunks (StreamingDecoder, stream.rs:62-139): decode_chunk output equals
    the matching slice of the offline decode."""

    _free = "ctts_vae_stream_free"

    def __init__(self, w: DecoderW, batch: int = 1):
        super().__init__()
        self.w = w  # keeps the weights alive
        self.batch = batch
        check(_lib.load().ctts_vae_stream_create(w.h, batch, C.byref(self.h)))

    def reset(self) -> None:
        check(_lib.load().ctts_vae_stream_reset(self.h))

    def decode_chunk(self, latent) -> np.ndarray:
        """latent [latent, F] or [B, latent, F] -> wav [F*hop] / [B, F*hop]."""
        lat = _f(latent)
        single = lat.ndim == 2
        if single:
            lat = lat[None]
        B, _, F = lat.shape
        if B != self.batch:
            raise ValueError(f"stream holds {self.batch} utterances, chunk has {B}")
        wav = np.empty((B, F * self.w.cfg.hop), np.float32)
        check(_lib.load().ctts_vae_stream_decode_chunk(self.h, _p(lat), F, _p(wav)))
        return wav[0] if single else wav


def load_decoder_weights(path: str, cfg: VAEConfig, dtype="f32", device: int = 0,
                         prefix: str = "decoder.") -> DecoderW:
    return DecoderW(cfg, dtype, device).load(path, prefix)


def decode(w: DecoderW, latent, frames: int | None = None) -> np.ndarray:
    """decode (decode.rs:90-92): latent [latent, frames] -> wav [frames*hop]."""
    return w.decode(latent)
