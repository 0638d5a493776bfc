"""ctypes front end of the CPU restatement (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  The shipped package never
imports it.  Weight dictionaries use the reference checkpoint names produced
by rcutetts_b200.synth.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

fp = C.POINTER(C.c_float)


def build() -> str:
    """Compile liboracle.so with the committed Makefile."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _lib.orc_embed_lookup.restype = C.c_int
        _lib.orc_get_threads.restype = C.c_int
        # every output is computed by one thread in a fixed order, so the
        # results are bitwise the same for any thread count: use them all
        _lib.orc_set_threads(int(os.cpu_count() or 1))
    return _lib


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def get_threads() -> int:
    return int(lib().orc_get_threads())


def _p(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(fp)


def _f(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------------ structs
class LMDims(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_heads", C.c_int), ("n_kv", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("eps", C.c_float),
                ("rope_theta", C.c_float), ("qk_norm", C.c_int)]


class LMLayerW(C.Structure):
    _fields_ = [(n, fp) for n in ("norm1", "norm2", "wq", "wk", "wv", "wo", "qn", "kn",
                                  "wg", "wu", "wd")]


class DiTDims(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("latent", "hidden", "n_heads", "n_kv", "head_dim",
                                       "ffn", "n_layers", "patch", "cond_dim", "spk_dim")] + \
               [("eps", C.c_float), ("rope_theta", C.c_float)]


class DiTLayerW(C.Structure):
    _fields_ = [(n, fp) for n in ("norm1", "norm2", "wq", "wk", "wv", "wo", "wg", "wu",
                                  "wd", "adaln")]


class DiTW(C.Structure):
    _fields_ = [(n, fp) for n in (
        "in_w", "in_b", "cond_w", "cond_b", "mu_w", "mu_b", "out_w", "out_b",
        "t1_w", "t1_b", "t2_w", "t2_b", "dt1_w", "dt1_b", "dt2_w", "dt2_b",
        "st1_w", "st1_b", "st2_w", "st2_b", "cfg0_w", "cfg2_w", "final_norm")] + \
        [("layers", C.POINTER(DiTLayerW))]


class LocEncW(C.Structure):
    _fields_ = [(n, fp) for n in ("in_w", "in_b", "special", "final_norm", "proj_w", "proj_b")] + \
               [("layers", C.POINTER(DiTLayerW)), ("out_dim", C.c_int)]


class ResW(C.Structure):
    _fields_ = [(n, fp) for n in ("a0", "w0", "b0", "a1", "w1", "b1")]


class StageW(C.Structure):
    _fields_ = [("alpha", fp), ("tw", fp), ("tb", fp), ("res", ResW * 3)]


class VAEW(C.Structure):
    _fields_ = [("latent", C.c_int), ("channels", C.c_int), ("n_stages", C.c_int),
                ("depthwise", C.c_int), ("strides", C.c_int * 8),
                ("front_w", fp), ("front_b", fp), ("front_pw_w", fp), ("front_pw_b", fp),
                ("stages", C.POINTER(StageW)),
                ("final_alpha", fp), ("final_w", fp), ("final_b", fp)]


# --------------------------------------------------------------- primitives
def linear(x, W, b=None):
    x, W = _f(x), _f(W)
    S, I = x.reshape(-1, x.shape[-1]).shape
    O = W.shape[0]
    y = np.empty((S, O), np.float32)
    bb = _f(b) if b is not None else None
    lib().orc_linear(_p(x), S, I, _p(W), _p(bb), O, _p(y))
    return y.reshape(x.shape[:-1] + (O,))


def rms_norm(x, w, eps=1e-6):
    x, w = _f(x), _f(w)
    out = np.empty_like(x)
    n = x.shape[-1]
    xr, orr = x.reshape(-1, n), out.reshape(-1, n)
    for i in range(xr.shape[0]):
        lib().orc_rms_norm_row(_p(xr[i]), _p(w), n, C.c_float(eps), _p(orr[i]))
    return out


def rope(v, pos, theta):
    """v [..., d] rotated at positions pos (broadcast over leading dims)."""
    v = _f(v)
    d = v.shape[-1]
    out = np.empty_like(v)
    vr, orr = v.reshape(-1, d), out.reshape(-1, d)
    pos = np.broadcast_to(np.asarray(pos, np.int64), v.shape[:-1]).reshape(-1)
    for i in range(vr.shape[0]):
        lib().orc_rope(_p(vr[i]), d, int(pos[i]), C.c_float(theta), _p(orr[i]))
    return out


def swiglu(g, u):
    g, u = _f(g), _f(u)
    out = np.empty_like(g)
    lib().orc_swiglu(_p(g), _p(u), g.size, _p(out))
    return out


def embed_lookup(table, ids):
    table = _f(table)
    ids = np.ascontiguousarray(ids, np.int64)
    out = np.empty((ids.size, table.shape[1]), np.float32)
    rc = lib().orc_embed_lookup(_p(table), table.shape[0], table.shape[1],
                                ids.ctypes.data_as(C.POINTER(C.c_int64)), ids.size, _p(out))
    if rc != 0:
        raise IndexError("token id out of range")
    return out


def sin_emb(x, dim):
    out = np.empty(dim, np.float32)
    lib().orc_sin_emb(C.c_float(x), dim, _p(out))
    return out


def sway_timesteps(steps, coeff):
    out = np.empty(steps + 1, np.float32)
    lib().orc_sway_timesteps(steps, C.c_float(coeff), _p(out))
    return out


def stop_logits(w, b, h):
    w, b, h = _f(w), _f(b), _f(h)
    out = np.empty(2, np.float32)
    lib().orc_stop_logits(_p(w), _p(b), h.size, _p(h), _p(out))
    return out


# ------------------------------------------------------------------------ LM
class LM:
    """Restated Qwen3 stack over host float32 weights + per-utterance cache."""

    def __init__(self, cfg, weights: dict, n_layers: int | None = None):
        self.cfg = cfg
        self.n_layers = cfg.n_layers if n_layers is None else n_layers
        self.w = {k: _f(v) for k, v in weights.items()}
        self.dims = LMDims(cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn,
                           cfg.rms_eps, cfg.rope_theta, int(cfg.qk_norm))
        g = lambda n: _p(self.w[n])
        self.layers = (LMLayerW * self.n_layers)()
        for i in range(self.n_layers):
            p = f"layers.{i}."
            L = self.layers[i]
            L.norm1, L.norm2 = g(p + "input_layernorm.weight"), g(p + "post_attention_layernorm.weight")
            L.wq, L.wk = g(p + "self_attn.q_proj.weight"), g(p + "self_attn.k_proj.weight")
            L.wv, L.wo = g(p + "self_attn.v_proj.weight"), g(p + "self_attn.o_proj.weight")
            L.qn, L.kn = g(p + "self_attn.q_norm.weight"), g(p + "self_attn.k_norm.weight")
            L.wg, L.wu = g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")
            L.wd = g(p + "mlp.down_proj.weight")

    def new_cache(self, capacity):
        kv = self.cfg.kv_dim
        return {"k": [np.zeros((capacity, kv), np.float32) for _ in range(self.n_layers)],
                "v": [np.zeros((capacity, kv), np.float32) for _ in range(self.n_layers)],
                "len": 0}

    def layer(self, i, h, cache_k, cache_v, length, pos0=None):
        """One layer; appends to cache_k/cache_v [cap, kv_dim]."""
        h = _f(h)
        T = h.shape[0]
        out = np.empty_like(h)
        lib().orc_lm_layer(C.byref(self.dims), C.byref(self.layers[i]), _p(h), T,
                           length if pos0 is None else pos0, _p(cache_k), _p(cache_v),
                           length, _p(out))
        return out

    def forward(self, x, cache, pos0=None):
        """All layers + final norm over T new rows; advances cache['len']."""
        x = _f(x)
        T = x.shape[0]
        n = self.n_layers
        kp = (fp * n)(*[_p(a) for a in cache["k"]])
        vp = (fp * n)(*[_p(a) for a in cache["v"]])
        out = np.empty_like(x)
        L = cache["len"]
        lib().orc_lm_forward(C.byref(self.dims), n, self.layers, _p(self.w["norm.weight"]),
                             _p(x), T, L if pos0 is None else pos0, kp, vp, L, _p(out))
        cache["len"] = L + T
        return out

    def embed(self, ids):
        return embed_lookup(self.w["embed_tokens.weight"], ids)


# ----------------------------------------------------------------------- DiT
class DiT:
    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        self.w = {k: _f(v) for k, v in weights.items()}
        self.dims = DiTDims(cfg.latent, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                            cfg.ffn, cfg.n_layers, cfg.patch, cfg.cond_dim, cfg.spk_dim,
                            cfg.rms_eps, cfg.rope_theta)
        g = lambda n: _p(self.w[n]) if n in self.w else None
        self.layers = (DiTLayerW * cfg.n_layers)()
        for i in range(cfg.n_layers):
            p = f"decoder.layers.{i}."
            L = self.layers[i]
            L.norm1, L.norm2 = g(p + "input_layernorm.weight"), g(p + "post_attention_layernorm.weight")
            L.wq, L.wk = g(p + "self_attn.q_proj.weight"), g(p + "self_attn.k_proj.weight")
            L.wv, L.wo = g(p + "self_attn.v_proj.weight"), g(p + "self_attn.o_proj.weight")
            L.wg, L.wu = g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")
            L.wd, L.adaln = g(p + "mlp.down_proj.weight"), g(p + "speaker_adaln.weight")
        W = DiTW()
        names = {"in_w": "in_proj.weight", "in_b": "in_proj.bias", "cond_w": "cond_proj.weight",
                 "cond_b": "cond_proj.bias", "mu_w": "mu_proj.weight", "mu_b": "mu_proj.bias",
                 "out_w": "out_proj.weight", "out_b": "out_proj.bias",
                 "t1_w": "time_mlp.linear_1.weight", "t1_b": "time_mlp.linear_1.bias",
                 "t2_w": "time_mlp.linear_2.weight", "t2_b": "time_mlp.linear_2.bias",
                 "dt1_w": "delta_time_mlp.linear_1.weight", "dt1_b": "delta_time_mlp.linear_1.bias",
                 "dt2_w": "delta_time_mlp.linear_2.weight", "dt2_b": "delta_time_mlp.linear_2.bias",
                 "st1_w": "step_size_embedding.linear_1.weight",
                 "st1_b": "step_size_embedding.linear_1.bias",
                 "st2_w": "step_size_embedding.linear_2.weight",
                 "st2_b": "step_size_embedding.linear_2.bias",
                 "cfg0_w": "cfg_strength_embedding.0.weight",
                 "cfg2_w": "cfg_strength_embedding.2.weight",
                 "final_norm": "decoder.norm.weight"}
        for field, name in names.items():
            setattr(W, field, g(name))
        W.layers = self.layers
        self.W = W

    def predict(self, x, t, z, cond, dt=0.0, spk=None, cfg_w=0.0):
        x, z, cond = _f(x).reshape(-1), _f(z).reshape(-1), _f(cond).reshape(-1)
        v = np.empty_like(x)
        spk = _f(spk).reshape(-1) if spk is not None else None
        lib().orc_dit_predict(C.byref(self.dims), C.byref(self.W), _p(x), C.c_float(t), _p(z),
                              _p(cond), C.c_float(dt), _p(spk), C.c_float(cfg_w), _p(v))
        return v

    def euler_sample(self, x0, z, cond, spk, steps, cfg_w=0.0):
        x0, z, cond = _f(x0).reshape(-1), _f(z).reshape(-1), _f(cond).reshape(-1)
        spk = _f(spk).reshape(-1) if spk is not None else None
        x = np.empty_like(x0)
        lib().orc_dit_euler_sample(C.byref(self.dims), C.byref(self.W), _p(x0), _p(z), _p(cond),
                                   _p(spk), steps, C.c_float(cfg_w), _p(x))
        return x

    def euler_sample_cfg(self, x0, z_c, z_u, cond, uncond, spk, steps, coeff, cfg):
        a = [_f(v).reshape(-1) for v in (x0, z_c, z_u, cond, uncond)]
        spk = _f(spk).reshape(-1) if spk is not None else None
        x = np.empty_like(a[0])
        lib().orc_dit_euler_sample_cfg(C.byref(self.dims), C.byref(self.W), *[_p(v) for v in a],
                                       _p(spk), steps, C.c_float(coeff), C.c_float(cfg), _p(x))
        return x


class LocEnc:
    """locenc_embed + locenc_to_lm_proj (locenc.rs:222-255, model.py:128-130)."""

    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        self.w = {k: _f(v) for k, v in weights.items()}
        self.dims = DiTDims(cfg.latent, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn,
                            cfg.n_layers, cfg.patch, 0, 0, cfg.rms_eps, cfg.rope_theta)
        g = lambda n: _p(self.w[n])
        self.layers = (DiTLayerW * cfg.n_layers)()
        for i in range(cfg.n_layers):
            p = f"encoder.layers.{i}."
            L = self.layers[i]
            L.norm1, L.norm2 = g(p + "input_layernorm.weight"), g(p + "post_attention_layernorm.weight")
            L.wq, L.wk = g(p + "self_attn.q_proj.weight"), g(p + "self_attn.k_proj.weight")
            L.wv, L.wo = g(p + "self_attn.v_proj.weight"), g(p + "self_attn.o_proj.weight")
            L.wg, L.wu = g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")
            L.wd, L.adaln = g(p + "mlp.down_proj.weight"), None
        W = LocEncW()
        W.in_w, W.in_b, W.special = g("in_proj.weight"), g("in_proj.bias"), g("special_token")
        W.final_norm, W.proj_w, W.proj_b = g("encoder.norm.weight"), g("locenc_to_lm_proj.weight"), \
            g("locenc_to_lm_proj.bias")
        W.layers, W.out_dim = self.layers, cfg.out_dim
        self.W = W

    def embed(self, x):
        """x [n, patch, latent] -> [n, out_dim]"""
        x = _f(x).reshape(-1, self.cfg.patch, self.cfg.latent)
        out = np.empty((x.shape[0], self.cfg.out_dim), np.float32)
        lib().orc_locenc_embed(C.byref(self.dims), C.byref(self.W), _p(x), x.shape[0], _p(out))
        return out


# ----------------------------------------------------------------------- VAE
def snake(x, alpha):
    x = _f(x).copy()
    Cc, T = x.shape
    lib().orc_snake(_p(x), Cc, T, _p(_f(alpha).reshape(-1)))
    return x


def fuse_weight_norm(g, v):
    g, v = _f(g).reshape(-1), _f(v)
    w = np.empty_like(v)
    lib().orc_fuse_weight_norm(_p(g), _p(v), v.shape[0], int(np.prod(v.shape[1:])), _p(w))
    return w


def causal_conv1d(x, w, b, dilation=1, groups=1, pad=0):
    x, w, b = _f(x), _f(w), _f(b)
    c_in, T = x.shape
    c_out, _, k = w.shape
    out = np.empty((c_out, T), np.float32)
    lib().orc_causal_conv1d(_p(x), c_in, T, _p(w), _p(b), c_out, k, dilation, groups, pad, _p(out))
    return out


def causal_transpose_conv1d(x, w, b, stride, groups=1, pad=0, out_pad=0):
    x, w, b = _f(x), _f(w), _f(b)
    c_in, T = x.shape
    _, cog, k = w.shape
    c_out = cog * groups
    out_t = (T - 1) * stride + k - (2 * pad - out_pad)
    out = np.empty((c_out, out_t), np.float32)
    lib().orc_causal_transpose_conv1d(_p(x), c_in, T, _p(w), _p(b), c_out, k, stride, groups,
                                      pad, out_pad, _p(out))
    return out


class VAE:
    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        self.w = {k: _f(v) for k, v in weights.items()}
        g = lambda n: _p(self.w[n])
        n = len(cfg.strides)
        self.stages = (StageW * n)()
        V = VAEW()
        V.latent, V.channels, V.n_stages, V.depthwise = cfg.latent, cfg.channels, n, int(cfg.depthwise)
        for i, s in enumerate(cfg.strides):
            V.strides[i] = s
        if cfg.depthwise:
            V.front_w, V.front_b = g("model.0.weight"), g("model.0.bias")
            V.front_pw_w, V.front_pw_b = g("model.1.weight"), g("model.1.bias")
            idx = 2
        else:
            V.front_w, V.front_b = g("model.0.weight"), g("model.0.bias")
            idx = 1
        for si in range(n):
            b = f"model.{idx + si}.block."
            st = self.stages[si]
            st.alpha, st.tw, st.tb = g(b + "0.alpha"), g(b + "1.weight"), g(b + "1.bias")
            for r in range(3):
                rb = f"{b}{2 + r}.block."
                st.res[r] = ResW(g(rb + "0.alpha"), g(rb + "1.weight"), g(rb + "1.bias"),
                                 g(rb + "2.alpha"), g(rb + "3.weight"), g(rb + "3.bias"))
        fi = idx + n
        V.stages = self.stages
        V.final_alpha, V.final_w, V.final_b = g(f"model.{fi}.alpha"), g(f"model.{fi + 1}.weight"), g(f"model.{fi + 1}.bias")
        self.V = V

    def decode(self, latent):
        latent = _f(latent)
        T = latent.shape[1]
        wav = np.empty(T * self.cfg.hop, np.float32)
        lib().orc_vae_decode(C.byref(self.V), _p(latent), T, _p(wav))
        return wav


# ------------------------------------------------------------- frame loop
def generate(lm: LM, dit: DiT, fw: dict, prefix: np.ndarray, noise: np.ndarray,
             cond0: np.ndarray, euler_steps: int, capacity: int | None = None, spk=None, cfg_w=0.0):
    """Per-frame AR loop (bin/cutetts.rs:429-523 / generation.py:931-1087)
    for one utterance: prefill the prefix rows, then for every frame: stop
    logits, Euler-sample the DiT from the supplied noise conditioned on the
    last LM hidden state (AdaLN conditioned on it too), feed the raw latent
    back through latent_proj into one LM decode step.  Returns latents
    [F, latent], stop logits [F, 2] and the final LM hidden state.  spk, if
    given, conditions AdaLN instead of the LM state (a speaker embedding);
    cfg_w is the distilled guidance strength of a head with a cfg-strength
    embedding (bin/cutetts.rs:460-461)."""
    F = noise.shape[0]
    T = prefix.shape[0]
    cache = lm.new_cache(capacity or (T + F + 1))
    h = lm.forward(prefix, cache)
    z = h[-1].copy()
    cond = _f(cond0).reshape(-1).copy()
    lat = np.empty((F, dit.cfg.latent * dit.cfg.patch), np.float32)
    stops = np.empty((F, 2), np.float32)
    for f in range(F):
        stops[f] = stop_logits(fw["stop_predictor.weight"], fw["stop_predictor.bias"], z)
        ad = (z if spk is None else _f(spk).reshape(-1)) if dit.cfg.adaln else None
        x = dit.euler_sample(noise[f], z, cond, ad, euler_steps, cfg_w=cfg_w)
        lat[f] = x
        cond = x
        fb = linear(x[None, :], fw["latent_proj.weight"], fw["latent_proj.bias"])
        z = lm.forward(fb, cache)[0].copy()
    return lat, stops, z
