"""Loading checkpoints laid out like the shipped ones (tensor names, shapes
and dtypes from the crate's manifests: one tts file with qwen_backbone.*
bf16, head.* fp32 and locenc.* bf16, and the VAE file with weight-norm pairs
under decoder.*) through the device loaders (ctts_lm_load, ctts_dit_load,
ctts_locenc_load, cutetts_vae_load; qwen.rs:75-120, dit.rs:27-159,
locenc.rs:88, weights.rs:98-186).  Synthetic values, there is no checkpoint
here: every loaded model must report no missing tensor and compute exactly
what the same weights uploaded tensor by tensor compute."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err
from helpers import rnd
from oracle import oracle as orc
from rcutetts_b200 import synth
from test_manifests import DIT_DISTILL, LM_SHIPPED, LOCENC_SHIPPED, VAE_SHIPPED, checkpoint_tensors, manifests

pytestmark = pytest.mark.gpu


def save(path, tensors, man):
    """tensors: checkpoint name -> numpy array; stored in the manifest's dtype."""
    import torch
    from safetensors.torch import save_file

    assert sorted(tensors) == sorted(man)
    out = {}
    for name, arr in tensors.items():
        shape, dt = man[name]
        assert list(arr.shape) == shape, name
        out[name] = torch.from_numpy(np.ascontiguousarray(arr)).to(getattr(torch, dt))
    save_file(out, str(path))


@pytest.fixture(scope="module")
def tts_file(tmp_path_factory):
    """One file like model/CuteTTS-distill/weights/tts/model.safetensors:
    qwen_backbone.* and locenc.* in bf16, the DiT head under head.* in fp32."""
    m = manifests()
    lw = synth.lm_weights(LM_SHIPPED, seed=41, with_embed=True)
    dw = synth.dit_weights(DIT_DISTILL, seed=42)
    le = synth.locenc_weights(LOCENC_SHIPPED, seed=43)
    tensors, man = {}, {}
    for tag, w, prefix in (("lm", lw, ""), ("dit", dw, "head."), ("locenc", le, "")):
        for name, arr in checkpoint_tensors(tag, w).items():
            tensors[prefix + name] = arr
            man[prefix + name] = m[tag][name]
    path = tmp_path_factory.mktemp("ckpt") / "model.safetensors"
    save(path, tensors, man)
    return str(path), lw, dw, le


def test_lm_from_checkpoint(tts_file):
    from rcutetts_b200.model import QwenCache, QwenW, decode_step, prefill

    path, lw, _, _ = tts_file
    a = QwenW(LM_SHIPPED, "bf16").load(path, "qwen_backbone.")
    assert a.missing == 0
    # the same values at the file's precision (norm gains included)
    b = QwenW(LM_SHIPPED, "bf16").set_weights({k: synth.bf16_round(v) for k, v in lw.items()})
    xp, xd = rnd(900, (9, 1024)), rnd(901, (2, 1024))
    outs = []
    for m in (a, b):
        cache = QwenCache(m, batch=1, capacity=16)
        o = [prefill(m, xp, cache)] + [decode_step(m, xd[i:i + 1], cache) for i in range(2)]
        outs.append(np.concatenate(o, 0))
    assert np.array_equal(outs[0], outs[1])
    ids = np.array([0, 5, 16384], np.int64)
    assert np.array_equal(a.embed_lookup(ids), b.embed_lookup(ids))


def test_dit_from_checkpoint(tts_file):
    """The distill head (step-size and cfg-strength embeddings, speaker
    AdaLN) stored in fp32 under head.*, sampled in 4 steps at strength 2."""
    from rcutetts_b200.model import DitW

    path, _, dw, _ = tts_file
    a = DitW(DIT_DISTILL, "f32").load(path, "head.")
    assert a.missing == 0
    b = DitW(DIT_DISTILL, "f32").set_weights(dw)
    x0, z, c, spk = rnd(910, (3, 128)), rnd(911, (3, 1024)), rnd(912, (3, 128)), rnd(913, (3, 256))
    xa = a.euler_sample(x0, z, c, spk, 4, cfg_w=2.0)
    assert np.array_equal(xa, b.euler_sample(x0, z, c, spk, 4, cfg_w=2.0))
    ref = orc.DiT(DIT_DISTILL, dw).euler_sample(x0[1], z[1], c[1], spk[1], 4, cfg_w=2.0)
    assert rel_err(xa[1], ref) < 1e-4


def test_locenc_from_checkpoint(tts_file):
    from rcutetts_b200.model import LocEncW

    path, _, _, le = tts_file
    a = LocEncW(LOCENC_SHIPPED, "bf16").load(path, "locenc.")
    assert a.missing == 0
    b = LocEncW(LOCENC_SHIPPED, "bf16").set_weights({k: synth.bf16_round(v) for k, v in le.items()})
    x = rnd(920, (4, LOCENC_SHIPPED.patch, 64))
    assert np.array_equal(a.embed(x), b.embed(x))


def test_vae_from_checkpoint(tmp_path):
    """The shipped depthwise decoder with weight-norm pairs, through the
    reference's ffi.rs entry points (the topology is read from the shapes)."""
    from rcutetts_b200 import _lib

    m = manifests()["vae"]
    w = synth.vae_weights(VAE_SHIPPED, seed=44, fan_in=0.8)
    rng = np.random.default_rng(44)
    st, fused = {}, {}
    for k, v in w.items():
        if k.endswith(".weight"):
            # g near each channel's ||v|| (x 0.9..1.1): the fused weights keep
            # the fan-in scale, so the deep stack stays out of saturation
            norm = np.sqrt((v.astype(np.float64) ** 2).reshape(v.shape[0], -1).sum(1)).reshape(-1, 1, 1)
            g = (norm * (0.9 + 0.2 * rng.random((v.shape[0], 1, 1)))).astype(np.float32)
            st["decoder." + k + "_g"], st["decoder." + k + "_v"] = g, v
            fused[k] = orc.fuse_weight_norm(g, v)
        else:
            st["decoder." + k] = v
            fused[k] = v
    path = tmp_path / "audio_vae.safetensors"
    save(path, st, m)
    lib = _lib.load()
    h = lib.cutetts_vae_load(str(path).encode())
    assert h
    lat = rnd(930, (64, 3))
    wav = np.empty(3 * VAE_SHIPPED.hop, np.float32)
    assert lib.cutetts_vae_decode(h, lat.ctypes.data_as(C.POINTER(C.c_float)), 3,
                                  wav.ctypes.data_as(C.POINTER(C.c_float))) == 0
    lib.cutetts_vae_free(h)
    assert rel_err(wav, orc.VAE(VAE_SHIPPED, fused).decode(lat)) < 1e-4
