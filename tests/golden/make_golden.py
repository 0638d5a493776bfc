"""Generate golden vectors from the reference's own torch modules.

Runs the upstream CuteTTS torch code (src/cutetts/modeling/diffusion_head.py,
src/cutetts/audio_codec/model/audio_vae.py) and the HF Qwen3Model the
reference builds its LM from (src/cutetts/modeling/model.py:83-89) at the
benchmark shapes, on seeded synthetic weights (rcutetts_b200.synth) and seeded
inputs, and stores inputs + outputs as small .npz fixtures.  Weights are not
stored: they are regenerated from their seed by rcutetts_b200.synth.

The reference package cannot be imported as `cutetts` here (its __init__
pulls soundfile), so the two module files are loaded by path under stub
parent packages.  Needs the reference tree; run once in the build container:

    python tests/golden/make_golden.py [REFERENCE_ROOT]
"""
import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from rcutetts_b200 import synth  # noqa: E402
from rcutetts_b200.config import DiTConfig, LMConfig, LocEncConfig, VAEConfig  # noqa: E402

torch.set_grad_enabled(False)


def load_reference(root):
    src = os.path.join(root, "src", "cutetts")
    for name in ("cutetts", "cutetts.modeling", "cutetts.audio_codec", "cutetts.audio_codec.model"):
        m = types.ModuleType(name)
        m.__path__ = [os.path.join(src, *name.split(".")[1:])]
        sys.modules[name] = m

    def load(modname, rel):
        spec = importlib.util.spec_from_file_location(modname, os.path.join(src, rel))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[modname] = mod
        spec.loader.exec_module(mod)
        return mod

    load("cutetts.modeling.sampling", "modeling/sampling.py")
    dh = load("cutetts.modeling.diffusion_head", "modeling/diffusion_head.py")
    load("cutetts.audio_codec.model.vae", "audio_codec/model/vae.py")
    av = load("cutetts.audio_codec.model.audio_vae", "audio_codec/model/audio_vae.py")
    return dh, av


def rnd(seed, shape):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)


# ----------------------------------------------------------------------- LM
def hf_qwen(cfg: LMConfig, n_layers: int, w: dict):
    from transformers import Qwen3Config, Qwen3Model

    kw = dict(hidden_size=cfg.hidden, intermediate_size=cfg.ffn, num_hidden_layers=n_layers,
              num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.n_kv_heads,
              head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_eps, vocab_size=cfg.vocab,
              max_position_embeddings=8192, attention_bias=False, tie_word_embeddings=False)
    c = Qwen3Config(**kw)
    # transformers 4.x: rope_theta attribute; 5.x: rope_parameters dict
    if hasattr(c, "rope_parameters") and isinstance(getattr(c, "rope_parameters"), dict):
        c.rope_parameters["rope_theta"] = cfg.rope_theta
    c.rope_theta = cfg.rope_theta
    c._attn_implementation = "eager"
    m = Qwen3Model(c).float().eval()
    sd = {k: torch.from_numpy(v) for k, v in w.items()
          if not k.startswith("layers.") or int(k.split(".")[1]) < n_layers}
    if "embed_tokens.weight" not in sd:
        sd["embed_tokens.weight"] = m.embed_tokens.weight.detach().clone()
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in k for k in missing), missing
    return m


def run_hf(m, x_prefill, x_decode, capture_layer=None):
    """Prefill rows then decode rows one at a time.  Returns final-normed
    outputs and (optionally) the raw output of layer `capture_layer`."""
    from transformers import DynamicCache

    grabbed = []
    hook = None
    if capture_layer is not None:
        def _h(mod, inp, out):
            grabbed.append((out[0] if isinstance(out, tuple) else out).detach().clone())
        hook = m.layers[capture_layer].register_forward_hook(_h)
    cache = DynamicCache()
    T = x_prefill.shape[0]
    o = m(inputs_embeds=torch.from_numpy(x_prefill)[None], past_key_values=cache, use_cache=True,
          position_ids=torch.arange(T)[None])
    outs = [o.last_hidden_state[0]]
    for i in range(x_decode.shape[0]):
        o = m(inputs_embeds=torch.from_numpy(x_decode[i:i + 1])[None], past_key_values=cache,
              use_cache=True, position_ids=torch.tensor([[T + i]]))
        outs.append(o.last_hidden_state[0])
    if hook:
        hook.remove()
    final = torch.cat(outs, 0).numpy()
    layer = torch.cat([g[0] for g in grabbed], 0).numpy() if grabbed else None
    return final, layer


# ---------------------------------------------------------------------- DiT
def torch_dit(dh, cfg: DiTConfig, w: dict):
    m = dh.AudioDiTHead(latent_dim=cfg.latent, cond_dim=cfg.cond_dim, hidden_dim=cfg.hidden,
                        ffn_dim=cfg.ffn, num_layers=cfg.n_layers, num_heads=cfg.n_heads,
                        num_kv_heads=cfg.n_kv_heads, patch_size=cfg.patch,
                        rms_norm_eps=cfg.rms_eps, rope_theta=cfg.rope_theta,
                        speaker_adaln_zero_enabled=cfg.adaln, speaker_embedding_dim=cfg.spk_dim,
                        step_size_embedding_enabled=cfg.step_emb,
                        cfg_strength_embedding_enabled=cfg.cfg_emb).float().eval()
    sd = {k: torch.from_numpy(v) for k, v in w.items()}
    m.load_state_dict(sd, strict=True)
    return m


# ---------------------------------------------------------------------- VAE
def torch_vae(av, cfg: VAEConfig, w: dict):
    m = av.CausalDecoder(cfg.latent, cfg.channels, list(cfg.strides), depthwise=cfg.depthwise).float().eval()
    for mod in m.modules():
        if hasattr(mod, "weight_g"):
            torch.nn.utils.remove_weight_norm(mod)
    sd = {k: torch.from_numpy(v) for k, v in w.items()}
    m.load_state_dict(sd, strict=True)
    return m


# -------------------------------------------------------------------- LocEnc
LOCENC_SMALL = LocEncConfig(hidden=256, n_heads=4, n_kv_heads=2, ffn=512, out_dim=128)
LOCENC_SHIPPED = LocEncConfig()  # hidden 1024, ffn 4096, 16/2 heads, 2 layers, patch 2


def torch_locenc(dh, cfg: LocEncConfig, w: dict):
    """AudioLocEnc (diffusion_head.py:334-378) + locenc_to_lm_proj (model.py:55)."""
    enc = dh.AudioLocEnc(input_dim=cfg.latent, hidden_dim=cfg.hidden, ffn_dim=cfg.ffn, num_layers=cfg.n_layers,
                         num_heads=cfg.n_heads, num_kv_heads=cfg.n_kv_heads, patch_size=cfg.patch,
                         rms_norm_eps=cfg.rms_eps, use_rope=True, rope_theta=cfg.rope_theta).float().eval()
    enc.load_state_dict({k: torch.from_numpy(v) for k, v in w.items() if not k.startswith("locenc_to_lm_proj")},
                        strict=True)
    proj = torch.nn.Linear(cfg.hidden, cfg.out_dim).float().eval()
    proj.weight.copy_(torch.from_numpy(w["locenc_to_lm_proj.weight"]))
    proj.bias.copy_(torch.from_numpy(w["locenc_to_lm_proj.bias"]))
    return lambda x: proj(enc(x))


def make_locenc(root):
    """locenc.npz: x [B, T, patch, 64] and proj(locenc(x)) [B, T, out_dim] for
    the small config (weights synth.locenc_weights(seed 17)) and the shipped
    shape (seed 18, one utterance-step pair)."""
    dh, _ = load_reference(root)
    out = {}
    for tag, cfg, seed, shape in (("small", LOCENC_SMALL, 17, (2, 3)), ("shipped", LOCENC_SHIPPED, 18, (1, 2))):
        w = synth.locenc_weights(cfg, seed)
        x = rnd(seed + 100, shape + (cfg.patch, cfg.latent))
        y = torch_locenc(dh, cfg, w)(torch.from_numpy(x)).numpy()
        out[f"{tag}_x"], out[f"{tag}_out"] = x, y
    np.savez_compressed(os.path.join(HERE, "locenc.npz"), **out)
    print({k: v.shape for k, v in out.items()})


def main(root):
    dh, av = load_reference(root)
    out = {}

    # config[0]: one fp32 layer, weights seed 0, 64-row prefill + 32 decodes.
    lcfg = LMConfig(n_layers=1)
    w0 = synth.lm_weights(lcfg, seed=0, with_embed=False)
    xp, xd = rnd(100, (64, lcfg.hidden)), rnd(101, (32, lcfg.hidden))
    m = hf_qwen(lcfg, 1, w0)
    final, layer = run_hf(m, xp, xd, capture_layer=0)
    np.savez_compressed(os.path.join(HERE, "lm_layer_c0.npz"), x_prefill=xp, x_decode=xd,
                        layer_out=layer, final_out=final)
    out["lm_layer_c0"] = layer.shape

    # config[2] LM stack (12 layers, seed 2): short prefill + 3 decodes.
    l2 = LMConfig()
    w2 = synth.lm_weights(l2, seed=2)
    m2 = hf_qwen(l2, l2.n_layers, w2)
    xp2, xd2 = rnd(200, (12, l2.hidden)), rnd(201, (3, l2.hidden))
    final2, _ = run_hf(m2, xp2, xd2)
    ids = np.random.default_rng(202).integers(0, l2.vocab, 16)
    emb = m2.embed_tokens(torch.from_numpy(ids))[None].numpy()[0]
    np.savez_compressed(os.path.join(HERE, "lm_stack_c2.npz"), x_prefill=xp2, x_decode=xd2,
                        final_out=final2, ids=ids, embed_out=emb)
    out["lm_stack_c2"] = final2.shape

    # config[2] DiT head (seed 2 via dit seed 12): predict + 10-step Euler, batch 2.
    dcfg = DiTConfig()
    wd = synth.dit_weights(dcfg, seed=12)
    md = torch_dit(dh, dcfg, wd)
    B = 2
    x0, z = rnd(300, (B, dcfg.latent)), rnd(301, (B, dcfg.cond_dim))
    cond = rnd(302, (B, dcfg.latent))
    tx, tz, tc = torch.from_numpy(x0), torch.from_numpy(z), torch.from_numpy(cond)
    v = md._predict(tx, torch.full((B,), 0.3), tz, tc, speaker_embedding=tz).numpy()
    xs = md._euler_sample_core(tx, tz, tc, tz, None, 0.0, 10).numpy()
    np.savez_compressed(os.path.join(HERE, "dit_c2.npz"), x0=x0, z=z, cond=cond, t=np.float32(0.3),
                        predict_out=v, euler10_out=xs)
    out["dit_c2"] = xs.shape

    # Plain (no AdaLN) DiT variant + sway grid + CFG euler (base variant).
    dplain = DiTConfig(adaln=False, n_layers=2)
    wdp = synth.dit_weights(dplain, seed=13)
    mp = torch_dit(dh, dplain, wdp)
    vp = mp._predict(tx, torch.full((B,), 0.7), tz, tc).numpy()
    times = dh.sway_timesteps(10, -0.8).numpy()
    zu = rnd(303, (B, dplain.cond_dim))
    condu = rnd(304, (B, dplain.latent))

    def fwd(xc, tb, cnd):
        return mp._predict(xc, tb, cnd[:, :dplain.cond_dim], cnd[:, dplain.cond_dim:])
    # CFG combine over the sway grid (diffusion_head.py:58-97) with explicit x0.
    x = tx.clone()
    for s in range(10):
        tb = torch.full((2 * B,), float(times[s]))
        zz = torch.cat([tz, torch.from_numpy(zu)], 0)
        cc = torch.cat([tc, torch.from_numpy(condu)], 0)
        vel = mp._predict(torch.cat([x, x], 0), tb, zz, cc).float()
        vc, vu = torch.chunk(vel, 2, 0)
        vel = vc + 2.0 * (vc - vu)
        x = x + vel * (times[s + 1] - times[s])
    np.savez_compressed(os.path.join(HERE, "dit_plain.npz"), predict_out=vp, sway=times,
                        z_uncond=zu, uncond=condu, cfg_out=x.numpy())
    out["dit_plain"] = vp.shape

    # config[4] VAE decoder (seed 4) on a short latent.
    vcfg = VAEConfig()
    wv = synth.vae_weights(vcfg, seed=4)
    mv = torch_vae(av, vcfg, wv)
    lat = rnd(400, (2, vcfg.latent, 6))
    wav = mv(torch.from_numpy(lat)).numpy()[:, 0, :]
    np.savez_compressed(os.path.join(HERE, "vae_c4.npz"), latent=lat, wav=wav)
    out["vae_c4"] = wav.shape

    # Weight-norm fuse KAT from the torch parametrisation (conv.rs:12-30).
    conv = av.WNCausalConv1d(6, 4, kernel_size=3, padding=1)
    g = conv.weight_g.detach().numpy() * 1.7
    vv = conv.weight_v.detach().numpy()
    conv.weight_g.data = torch.from_numpy(g)
    fused = torch._weight_norm(conv.weight_v, conv.weight_g, 0).detach().numpy()
    np.savez_compressed(os.path.join(HERE, "weight_norm.npz"), g=g, v=vv, w=fused)

    for k, v in out.items():
        print(k, v)


# The shipped model's LM and DiT head shapes (qwen.rs:17-24, dit.rs:16-26):
# LM hidden 1024, 7 layers, 16/8 heads of 128, FFN 3072, vocab 16385; DiT
# hidden 1024, FFN 4096, 16/2 heads of 64, patch 2, speaker AdaLN width 256,
# mu_proj Identity (cond_dim == hidden).
LM_SHIPPED = LMConfig(hidden=1024, n_layers=7, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072, vocab=16385)
DIT_SHIPPED = DiTConfig(hidden=1024, n_heads=16, n_kv_heads=2, head_dim=64, ffn=4096, n_layers=4, patch=2,
                        cond_dim=1024, spk_dim=256)


def make_shipped(root):
    """lm_shipped.npz (synth weights seed 30: 10-row prefill + 3 decodes,
    final-normed outputs) and dit_shipped.npz (seed 31: predict at t=0.4 and
    a 10-step Euler sample for 2 utterances with speaker AdaLN)."""
    dh, _ = load_reference(root)
    wl = synth.lm_weights(LM_SHIPPED, seed=30, with_embed=False)
    m = hf_qwen(LM_SHIPPED, LM_SHIPPED.n_layers, wl)
    xp, xd = rnd(500, (10, LM_SHIPPED.hidden)), rnd(501, (3, LM_SHIPPED.hidden))
    final, _ = run_hf(m, xp, xd)
    np.savez_compressed(os.path.join(HERE, "lm_shipped.npz"), x_prefill=xp, x_decode=xd, final_out=final)
    print("lm_shipped", final.shape)
    cfg = DIT_SHIPPED
    wd = synth.dit_weights(cfg, seed=31)
    md = torch_dit(dh, cfg, wd)
    B, P = 2, cfg.patch * cfg.latent
    x0, z = rnd(510, (B, P)), rnd(511, (B, cfg.cond_dim))
    cond, spk = rnd(512, (B, P)), rnd(513, (B, cfg.spk_dim))
    tx, tz, tc, ts = (torch.from_numpy(a) for a in (x0, z, cond, spk))
    with torch.no_grad():
        # [N, P, D] inputs: a flat [N, P*D] input makes _predict return patch 0 only
        v3 = md._predict(tx.reshape(B, cfg.patch, cfg.latent), torch.full((B,), 0.4), tz,
                         tc.reshape(B, cfg.patch, cfg.latent), speaker_embedding=ts)
        v = v3.reshape(B, P).numpy()
        xs = md._euler_sample_core(tx, tz, tc, ts, None, 0.0, 10).numpy()
    np.savez_compressed(os.path.join(HERE, "dit_shipped.npz"), x0=x0, z=z, cond=cond, spk=spk, t=np.float32(0.4),
                        predict_out=v, euler10_out=xs)
    print("dit_shipped", xs.shape)


VAE_DW_GAIN = 0.8  # fan-in weight scale: waveform std well inside tanh's range
VAE_DW_SMALL = VAEConfig(latent=64, channels=96, strides=(4, 3, 2), depthwise=True)
VAE_DW_SHIPPED = VAEConfig(latent=64, channels=1536, strides=(16, 8, 5, 3), depthwise=True)


def make_vae_dw(root):
    """Depthwise CausalDecoder (the shipped topology, audio_vae.py:255-280):
    a small shape and the shipped shape (1536 channels, rates 16/8/5/3,
    hop 1920), synth weights with fan-in scaling (seed 8 / 9), two short
    latents each."""
    _, av = load_reference(root)
    for name, cfg, seed, T in (("vae_dw_small", VAE_DW_SMALL, 8, 9), ("vae_dw_shipped", VAE_DW_SHIPPED, 9, 3)):
        w = synth.vae_weights(cfg, seed=seed, fan_in=VAE_DW_GAIN)
        m = torch_vae(av, cfg, w)
        lat = rnd(410 + seed, (2, cfg.latent, T))
        with torch.no_grad():
            wav = m(torch.from_numpy(lat)).numpy()[:, 0, :]
        np.savez_compressed(os.path.join(HERE, name + ".npz"), latent=lat, wav=wav)
        print(name, wav.shape)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if a not in ("locenc", "vae_dw", "shipped")]
    root = args[0] if args else os.environ.get("RCUTETTS_REFERENCE", "")
    if not root:
        sys.exit("usage: make_golden.py <RCuteTTS checkout> [locenc|vae_dw|shipped] "
                 "(or set RCUTETTS_REFERENCE)")
    if "locenc" in sys.argv[1:]:
        make_locenc(root)  # only the LocEnc fixture
    elif "vae_dw" in sys.argv[1:]:
        make_vae_dw(root)  # only the depthwise VAE fixtures
    elif "shipped" in sys.argv[1:]:
        make_shipped(root)  # only the shipped-shape LM / DiT fixtures
    else:
        main(root)
        make_locenc(root)
