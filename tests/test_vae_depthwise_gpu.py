"""The shipped depthwise VAE topology on the GPU (audio_vae.py:255-280
CausalDecoder(depthwise=True); decode.rs:94-136, weights.rs:98-186): the
depthwise k7 + pointwise front and the depthwise dilated k7 residual convs,
against the reference's torch module (golden fixtures at a small shape and
at the shipped shape: 1536 channels, rates 16/8/5/3, hop 1920), the oracle
in bf16, the reference's conv fixtures (m1_conv_dw9, m1_conv_d3), causality,
streaming bit-identity and the ffi.rs loader on a weight-norm checkpoint
with the shipped tensor names."""
import ctypes as C

import numpy as np
import pytest

from conftest import cosine, rel_err
from helpers import bf16_weights, rnd
from oracle import oracle as orc
from rcutetts_b200 import synth
from rcutetts_b200.config import VAEConfig

pytestmark = pytest.mark.gpu

SMALL = VAEConfig(latent=64, channels=96, strides=(4, 3, 2), depthwise=True)
SHIPPED = VAEConfig(latent=64, channels=1536, strides=(16, 8, 5, 3), depthwise=True)
GAIN = 0.8  # tests/golden/make_golden.py VAE_DW_GAIN


def model(cfg, seed, dtype="f32"):
    from rcutetts_b200.model import DecoderW

    w = synth.vae_weights(cfg, seed=seed, fan_in=GAIN)
    return DecoderW(cfg, dtype).set_weights(w), w


@pytest.mark.parametrize("name,cfg,seed", [("vae_dw_small", SMALL, 8), ("vae_dw_shipped", SHIPPED, 9)])
def test_depthwise_vs_golden(golden, name, cfg, seed):
    g = golden(name + ".npz")
    m, _ = model(cfg, seed)
    assert m.missing == 0
    wav = m.decode(g["latent"])
    assert wav.shape == (g["latent"].shape[0], g["latent"].shape[2] * cfg.hop)
    for b in range(wav.shape[0]):
        assert rel_err(wav[b], g["wav"][b]) < 1e-4
        assert cosine(wav[b], g["wav"][b]) >= 0.9999


def test_depthwise_bf16_vs_oracle():
    m, w = model(SHIPPED, 9, "bf16")
    o = orc.VAE(SHIPPED, bf16_weights(w))
    lat = rnd(11, (64, 3))
    assert cosine(m.decode(lat), o.decode(lat)) >= 0.999


@pytest.mark.parametrize("tag,dil,groups,pad", [("dw9", 9, 8, 27), ("d3", 3, 1, 9)])
def test_conv_reference_fixtures(golden, tag, dil, groups, pad):
    """The reference's conv fixtures (tests/m1_ops.rs conv_depthwise_d9:
    8 channels, k7, dilation 9, pad 27, groups 8; conv_dilated_d3: dense,
    dilation 3, pad 9) through ctts_op_causal_conv1d on the device, gate
    1e-4 as in m1_ops.rs."""
    import torch

    from rcutetts_b200 import _lib

    x, w, b = (golden(f"ref/m1_conv_{tag}_{n}.npy") for n in ("in", "w", "b"))
    ref = golden(f"ref/m1_conv_{tag}_out.npy")
    c_in, T = x.shape
    c_out, _, k = w.shape
    xd, wd, bd = (torch.from_numpy(np.ascontiguousarray(v, np.float32)).cuda() for v in (x, w, b))
    yd = torch.empty((c_out, T), device="cuda")
    lib = _lib.load()
    rc = lib.ctts_op_causal_conv1d(xd.data_ptr(), 1, c_in, T, wd.data_ptr(), 0, bd.data_ptr(), c_out, k, dil, groups,
                                   pad, yd.data_ptr(), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert np.max(np.abs(yd.cpu().numpy() - ref)) < 1e-4
    # groupings other than dense / depthwise are refused
    assert lib.ctts_op_causal_conv1d(xd.data_ptr(), 1, c_in, T, wd.data_ptr(), 0, bd.data_ptr(), c_out, k, dil, 2,
                                     pad, yd.data_ptr(), None) != 0


def test_depthwise_causal_prefix_and_batch():
    m, _ = model(SMALL, 8)
    lat = rnd(12, (3, 64, 40))
    full = m.decode(lat)
    half = m.decode(lat[:, :, :17])
    assert np.array_equal(full[:, :17 * SMALL.hop], half)
    assert np.array_equal(m.decode(lat[2:3])[0], full[2])


@pytest.mark.parametrize("cfg,seed", [(SMALL, 8), (SHIPPED, 9)])
def test_depthwise_stream_matches_offline(cfg, seed):
    from rcutetts_b200.model import StreamingDecoder

    m, _ = model(cfg, seed)
    T = 12 if cfg is SHIPPED else 30
    lat = rnd(13, (2, 64, T))
    full = m.decode(lat)
    dec = StreamingDecoder(m, batch=2)
    out, f = [], 0
    for n in ([2] * (T // 2)):
        out.append(dec.decode_chunk(lat[:, :, f:f + n]))
        f += n
    assert np.array_equal(np.concatenate(out, 1), full)
    dec.reset()
    out, f = [], 0
    for n in [1, 4, 3, T - 8]:
        out.append(dec.decode_chunk(lat[:, :, f:f + n]))
        f += n
    assert np.array_equal(np.concatenate(out, 1), full)


def test_reference_ffi_depthwise_checkpoint(tmp_path):
    """cutetts_vae_load (ffi.rs) on a checkpoint with the shipped names
    (decoder.model.0 depthwise [64,1,7], decoder.model.1 pointwise, stages
    at model.2..) stored as weight_g/weight_v pairs: the topology is read
    from the tensor shapes and the weights fused at load (conv.rs:12-30)."""
    from safetensors.numpy import save_file

    from rcutetts_b200 import _lib

    cfg = SMALL
    w = synth.vae_weights(cfg, seed=14, fan_in=GAIN)
    st, fused = {}, {}
    rng = np.random.default_rng(14)
    for k, v in w.items():
        if k.endswith(".weight"):
            g = (rng.random((v.shape[0], 1, 1), dtype=np.float32) + 0.5).astype(np.float32)
            st["decoder." + k[:-len("weight")] + "weight_g"] = g
            st["decoder." + k[:-len("weight")] + "weight_v"] = v
            fused[k] = orc.fuse_weight_norm(g, v)
        else:
            st["decoder." + k] = v
            fused[k] = v
    path = str(tmp_path / "vae_dw.safetensors")
    save_file(st, path)
    lib = _lib.load()
    h = lib.cutetts_vae_load(path.encode())
    assert h
    lat = rnd(15, (64, 7))
    wav = np.empty(7 * cfg.hop, np.float32)
    assert lib.cutetts_vae_decode(h, lat.ctypes.data_as(C.POINTER(C.c_float)), 7,
                                  wav.ctypes.data_as(C.POINTER(C.c_float))) == 0
    lib.cutetts_vae_free(h)
    ref = orc.VAE(cfg, fused).decode(lat)
    assert rel_err(wav, ref) < 1e-4
