"""ctypes binding of libcutetts_b200.so (the C ABI in include/cutetts_b200.h).

The library is built in-tree by rcutetts_b200.build; importing this module
loads it and fails loudly if it is missing -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcutetts_b200.so")

OK = 0
ERR_ARG, ERR_CUDA, ERR_TIMEOUT, ERR_STATE, ERR_IO, ERR_NOMEM, ERR_RANGE = -1, -2, -3, -4, -5, -6, -7
F32, BF16 = 0, 1

vp = C.c_void_p
fp = C.POINTER(C.c_float)
i64p = C.POINTER(C.c_int64)


class LMConfigC(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("ffn", C.c_int),
                ("vocab", C.c_int), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("qk_norm", C.c_int), ("weight_dtype", C.c_int)]


class DiTConfigC(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("latent", "hidden", "n_heads", "n_kv_heads", "head_dim",
                                       "ffn", "n_layers", "patch", "cond_dim", "spk_dim")] + \
               [("rms_eps", C.c_float), ("rope_theta", C.c_float), ("adaln", C.c_int),
                ("step_emb", C.c_int), ("cfg_emb", C.c_int), ("weight_dtype", C.c_int)]


class EngineConfigC(C.Structure):
    _fields_ = [("batch", C.c_int), ("capacity", C.c_int), ("euler_steps", C.c_int),
                ("latent_scale", C.c_float), ("latent_bias", C.c_float), ("use_graph", C.c_int),
                ("groups", C.c_int), ("cfg_strength", C.c_float), ("sway_coeff", C.c_float)]


class LocEncConfigC(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("latent", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn",
                                       "n_layers", "patch", "out_dim")] + \
               [("rms_eps", C.c_float), ("rope_theta", C.c_float), ("weight_dtype", C.c_int)]


class VAEConfigC(C.Structure):
    _fields_ = [("latent", C.c_int), ("channels", C.c_int), ("n_stages", C.c_int),
                ("depthwise", C.c_int), ("strides", C.c_int * 8), ("weight_dtype", C.c_int)]


# name -> (restype, argtypes)
SIGNATURES = {
    "ctts_last_error": (C.c_char_p, []),
    "ctts_version": (C.c_char_p, []),
    "ctts_debug_inject_wait_fault": (C.c_int, [C.c_int, C.c_uint]),
    "ctts_lm_create": (C.c_int, [C.POINTER(LMConfigC), C.c_int, C.POINTER(vp)]),
    "ctts_lm_set_tensor": (C.c_int, [vp, C.c_char_p, vp, C.c_int, i64p, C.c_int]),
    "ctts_lm_load": (C.c_int, [vp, C.c_char_p, C.c_char_p]),
    "ctts_lm_missing": (C.c_int, [vp]),
    "ctts_lm_free": (None, [vp]),
    "ctts_kv_alloc": (C.c_int, [vp, C.c_int, C.c_int, C.POINTER(vp)]),
    "ctts_kv_reset": (C.c_int, [vp]),
    "ctts_kv_len": (C.c_int, [vp, C.c_int]),
    "ctts_kv_set_len": (C.c_int, [vp, C.c_int, C.c_int]),
    "ctts_kv_free": (None, [vp]),
    "ctts_lm_prefill": (C.c_int, [vp, vp, C.c_int, fp, C.c_int, fp]),
    "ctts_lm_prefill_dev": (C.c_int, [vp, vp, C.c_int, vp, C.c_int, vp, vp]),
    "ctts_lm_decode_step": (C.c_int, [vp, vp, fp, fp]),
    "ctts_lm_decode_step_dev": (C.c_int, [vp, vp, vp, vp, vp]),
    "ctts_lm_embed_lookup": (C.c_int, [vp, i64p, C.c_int, fp]),
    "ctts_dit_create": (C.c_int, [C.POINTER(DiTConfigC), C.c_int, C.POINTER(vp)]),
    "ctts_dit_set_tensor": (C.c_int, [vp, C.c_char_p, vp, C.c_int, i64p, C.c_int]),
    "ctts_dit_load": (C.c_int, [vp, C.c_char_p, C.c_char_p]),
    "ctts_dit_missing": (C.c_int, [vp]),
    "ctts_dit_free": (None, [vp]),
    "ctts_dit_predict": (C.c_int, [vp, C.c_int, fp, C.c_float, fp, fp, C.c_float, fp, C.c_float, fp]),
    "ctts_dit_euler_sample": (C.c_int, [vp, C.c_int, fp, fp, fp, fp, C.c_int, C.c_float, fp]),
    "ctts_dit_euler_sample_dev": (C.c_int, [vp, C.c_int, vp, vp, vp, vp, C.c_int, C.c_float, vp, vp]),
    "ctts_dit_euler_sample_cfg": (C.c_int, [vp, C.c_int, fp, fp, fp, fp, fp, fp, C.c_int, C.c_float,
                                            C.c_float, fp]),
    "ctts_sway_timesteps": (C.c_int, [C.c_int, C.c_float, fp]),
    "ctts_engine_create": (C.c_int, [vp, vp, C.POINTER(EngineConfigC), C.POINTER(vp)]),
    "ctts_engine_set_heads": (C.c_int, [vp, fp, fp, fp, fp]),
    "ctts_engine_prefill": (C.c_int, [vp, C.c_int, fp, C.c_int, fp]),
    "ctts_engine_prefill_uncond": (C.c_int, [vp, C.c_int, fp, C.c_int, fp]),
    "ctts_engine_set_speaker": (C.c_int, [vp, C.c_int, fp]),
    "ctts_engine_step": (C.c_int, [vp, fp, fp, fp]),
    "ctts_engine_step_dev": (C.c_int, [vp, vp, vp, vp, vp]),
    "ctts_engine_set_profile": (C.c_int, [vp, C.c_int]),
    "ctts_engine_profile_stats": (C.c_int, [vp, C.c_int, fp, C.POINTER(C.c_int)]),
    "ctts_engine_profile_report": (C.c_int, [vp, C.c_char_p, C.c_int]),
    "ctts_engine_launches_per_step": (C.c_int, [vp]),
    "ctts_engine_stream": (vp, [vp]),
    "ctts_engine_free": (None, [vp]),
    "ctts_vae_create": (C.c_int, [C.POINTER(VAEConfigC), C.c_int, C.POINTER(vp)]),
    "ctts_vae_set_tensor": (C.c_int, [vp, C.c_char_p, vp, C.c_int, i64p, C.c_int]),
    "ctts_vae_load_file": (C.c_int, [vp, C.c_char_p, C.c_char_p]),
    "ctts_vae_missing": (C.c_int, [vp]),
    "ctts_vae_free": (None, [vp]),
    "ctts_vae_decode_batch": (C.c_int, [vp, C.c_int, fp, C.c_int, fp]),
    "ctts_vae_decode_batch_dev": (C.c_int, [vp, C.c_int, vp, C.c_int, vp, vp]),
    "ctts_vae_stream_create": (C.c_int, [vp, C.c_int, C.POINTER(vp)]),
    "ctts_vae_stream_reset": (C.c_int, [vp]),
    "ctts_vae_stream_decode_chunk": (C.c_int, [vp, fp, C.c_int, fp]),
    "ctts_vae_stream_decode_chunk_dev": (C.c_int, [vp, vp, C.c_int, vp, vp]),
    "ctts_vae_stream_free": (None, [vp]),
    "ctts_locenc_create": (C.c_int, [C.POINTER(LocEncConfigC), C.c_int, C.POINTER(vp)]),
    "ctts_locenc_set_tensor": (C.c_int, [vp, C.c_char_p, vp, C.c_int, i64p, C.c_int]),
    "ctts_locenc_load": (C.c_int, [vp, C.c_char_p, C.c_char_p]),
    "ctts_locenc_missing": (C.c_int, [vp]),
    "ctts_locenc_free": (None, [vp]),
    "ctts_locenc_embed": (C.c_int, [vp, fp, C.c_int, fp]),
    "ctts_locenc_embed_dev": (C.c_int, [vp, vp, C.c_int, vp, vp]),
    "cutetts_vae_load": (vp, [C.c_char_p]),
    "cutetts_vae_free": (None, [vp]),
    "cutetts_vae_decode": (C.c_int, [vp, fp, C.c_ulong, fp]),
    "ctts_op_linear": (C.c_int, [vp, C.c_int, C.c_int, vp, C.c_int, C.c_int, vp, C.c_float, vp, vp, vp]),
    "ctts_op_linear_noalloc": (C.c_int, [vp, C.c_int, C.c_int, vp, C.c_int, C.c_int, vp, C.c_float, vp, vp,
                                         vp]),
    "ctts_op_rope": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, vp, C.c_float, vp]),
    "ctts_op_swiglu": (C.c_int, [vp, C.c_int, C.c_int, vp, vp]),
    "ctts_op_causal_conv1d": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, vp, C.c_int, vp, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_int, vp, vp]),
    "ctts_op_embed_gather": (C.c_int, [vp, C.c_int, C.c_int, vp, C.c_int, vp, vp, vp]),
}

_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m rcutetts_b200.build` "
            "(there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _lib = lib
    return lib


class CttsError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != OK:
        msg = load().ctts_last_error().decode(errors="replace")
        raise CttsError(rc, msg)
