"""LocEnc feedback encoder + locenc_to_lm_proj on the GPU (locenc.rs:222-255
locenc_embed, model.py:128-130) against the reference's AudioLocEnc torch
module (golden fixture) and the oracle; fp32 and bf16; loading from a
combined checkpoint under the `locenc.` prefix."""
import numpy as np
import pytest

from conftest import cosine, rel_err
from helpers import bf16_weights, rnd
from oracle import oracle as orc
from rcutetts_b200 import synth
from rcutetts_b200.config import LocEncConfig

pytestmark = pytest.mark.gpu

SMALL = LocEncConfig(hidden=256, n_heads=4, n_kv_heads=2, ffn=512, out_dim=128)


def model(cfg, seed, dtype="f32"):
    from rcutetts_b200.model import LocEncW

    w = synth.locenc_weights(cfg, seed)
    return LocEncW(cfg, dtype).set_weights(w), w


@pytest.mark.parametrize("tag,cfg,seed", [("small", SMALL, 17), ("shipped", LocEncConfig(), 18)])
def test_fp32_vs_torch_golden(golden, tag, cfg, seed):
    g = golden("locenc.npz")
    m, _ = model(cfg, seed)
    got = m.embed(g[f"{tag}_x"])
    ref = g[f"{tag}_out"].reshape(got.shape)
    assert rel_err(got, ref) < 1e-4
    assert cosine(got, ref) >= 0.9999


def test_bf16_vs_oracle_and_batch_independence():
    cfg = LocEncConfig()
    m, w = model(cfg, 21, "bf16")
    x = rnd(22, (20, cfg.patch, cfg.latent))
    got = m.embed(x)
    ref = orc.LocEnc(cfg, bf16_weights(w)).embed(x)
    for i in range(x.shape[0]):
        assert cosine(got[i], ref[i]) >= 0.999, i
    assert np.array_equal(m.embed(x[7:8])[0], got[7])


def test_load_combined_checkpoint(tmp_path):
    """load_locenc_weights (locenc.rs:88-143): encoder tensors under
    `locenc.`, the projection beside it as `locenc_to_lm_proj.*`."""
    import torch
    from safetensors.torch import save_file

    from rcutetts_b200.model import LocEncW

    m, w = model(SMALL, 23)
    st = {("" if k.startswith("locenc_to_lm_proj") else "locenc.") + k: torch.from_numpy(v) for k, v in w.items()}
    st["head.other"] = torch.zeros(2)
    path = str(tmp_path / "m.safetensors")
    save_file(st, path)
    m2 = LocEncW(SMALL).load(path)
    assert m2.missing == 0
    x = rnd(24, (3, SMALL.patch, SMALL.latent))
    assert np.array_equal(m2.embed(x), m.embed(x))
