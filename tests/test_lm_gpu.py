"""LM stack on the GPU through the C ABI against the oracle and the golden
vectors made from HF Qwen3 (config[0], config[2] stack)."""
import numpy as np
import pytest

from conftest import cosine, rel_err
from helpers import bf16_weights, lm_model, rnd
from oracle import oracle as orc
from rcutetts_b200 import synth
from rcutetts_b200.config import LMConfig

pytestmark = pytest.mark.gpu


def run_device(m, xp, xd, capacity=128):
    from rcutetts_b200.model import QwenCache, decode_step, prefill

    cache = QwenCache(m, batch=1, capacity=capacity)
    outs = [prefill(m, xp, cache)]
    for i in range(xd.shape[0]):
        outs.append(decode_step(m, xd[i:i + 1], cache))
    assert cache.len(0) == xp.shape[0] + xd.shape[0]
    return np.concatenate(outs, 0)


def run_oracle(cfg, w, xp, xd, capacity=128):
    lm = orc.LM(cfg, w)
    cache = lm.new_cache(capacity)
    outs = [lm.forward(xp, cache)]
    for i in range(xd.shape[0]):
        outs.append(lm.forward(xd[i:i + 1], cache))
    return np.concatenate(outs, 0)


def test_layer_config0_fp32(golden):
    """config[0]: 64-row prefill + 32 decodes; every step within 1e-4."""
    g = golden("lm_layer_c0.npz")
    cfg = LMConfig(n_layers=1)
    m, w = lm_model(cfg, seed=0)
    got = run_device(m, g["x_prefill"], g["x_decode"])
    ref = run_oracle(cfg, w, g["x_prefill"], g["x_decode"])
    for i in range(got.shape[0]):
        assert rel_err(got[i], g["final_out"][i]) < 1e-4, i
        assert rel_err(got[i], ref[i]) < 1e-4, i


def test_layer_config0_bf16(golden):
    g = golden("lm_layer_c0.npz")
    cfg = LMConfig(n_layers=1)
    m, w = lm_model(cfg, seed=0, dtype="bf16")
    got = run_device(m, g["x_prefill"], g["x_decode"])
    ref = run_oracle(cfg, bf16_weights(w), g["x_prefill"], g["x_decode"])
    for i in range(got.shape[0]):
        assert cosine(got[i], ref[i]) >= 0.999, i


def test_stack_config2(golden):
    g = golden("lm_stack_c2.npz")
    cfg = LMConfig()
    m, w = lm_model(cfg, seed=2, with_embed=True)
    got = run_device(m, g["x_prefill"], g["x_decode"], capacity=32)
    for i in range(got.shape[0]):
        assert rel_err(got[i], g["final_out"][i]) < 1e-4, i
    assert np.array_equal(m.embed_lookup(g["ids"]), g["embed_out"])


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_batched_ragged_decode(dtype):
    """Three utterances with different prefill lengths advance together."""
    from rcutetts_b200.model import QwenCache, decode_step, prefill

    cfg = LMConfig(n_layers=2)
    m, w = lm_model(cfg, seed=5, dtype=dtype)
    wo = bf16_weights(w) if dtype == "bf16" else w
    lens = [5, 9, 2]
    cache = QwenCache(m, batch=3, capacity=40)
    pre = [rnd(50 + b, (lens[b], cfg.hidden)) for b in range(3)]
    dec = rnd(60, (4, 3, cfg.hidden))
    for b in range(3):
        prefill(m, pre[b], cache, b)
    outs = [decode_step(m, dec[s], cache) for s in range(4)]
    for b in range(3):
        assert cache.len(b) == lens[b] + 4
        ref = run_oracle(cfg, wo, pre[b], dec[:, b, :], capacity=40)[lens[b]:]
        for s in range(4):
            if dtype == "f32":
                assert rel_err(outs[s][b], ref[s]) < 1e-4
            else:
                assert cosine(outs[s][b], ref[s]) >= 0.999


def test_long_context_positions():
    """Decode at positions beyond one attention split (128 keys) and far
    into the RoPE range."""
    cfg = LMConfig(n_layers=1)
    m, w = lm_model(cfg, seed=7)
    xp = rnd(70, (300, cfg.hidden))
    xd = rnd(71, (3, cfg.hidden))
    got = run_device(m, xp, xd, capacity=400)
    ref = run_oracle(cfg, w, xp, xd, capacity=400)
    assert rel_err(got[-3:], ref[-3:]) < 1e-4
    assert rel_err(got[:300], ref[:300]) < 1e-4


def test_kv_capacity_and_embed_range():
    from rcutetts_b200._lib import ERR_RANGE, CttsError
    from rcutetts_b200.model import QwenCache, decode_step, prefill

    cfg = LMConfig(n_layers=1, vocab=100)
    m, w = lm_model(cfg, seed=8, with_embed=True)
    cache = QwenCache(m, batch=1, capacity=4)
    prefill(m, rnd(1, (4, cfg.hidden)), cache)
    with pytest.raises(CttsError) as e:
        decode_step(m, rnd(2, (1, cfg.hidden)), cache)
    assert e.value.code == ERR_RANGE
    with pytest.raises(CttsError) as e:
        m.embed_lookup(np.array([3, 100]))
    assert e.value.code == ERR_RANGE
    cache.reset()
    assert cache.len(0) == 0


def test_missing_weights_rejected():
    from rcutetts_b200._lib import ERR_STATE, CttsError
    from rcutetts_b200.model import QwenCache, QwenW, prefill

    cfg = LMConfig(n_layers=1)
    m = QwenW(cfg)
    w = synth.lm_weights(cfg, seed=0, with_embed=False)
    for k in list(w)[:-2]:
        m.set_tensor(k, w[k])
    assert m.missing == 2
    cache = QwenCache(m, 1, 8)
    with pytest.raises(CttsError) as e:
        prefill(m, rnd(1, (2, cfg.hidden)), cache)
    assert e.value.code == ERR_STATE


def test_safetensors_loader(tmp_path):
    """load_qwen_weights from a combined checkpoint (qwen_backbone.* names,
    bf16 storage, qwen.rs:75-120) equals uploading the rounded tensors."""
    import torch
    from safetensors.torch import save_file

    from rcutetts_b200.model import QwenCache, load_qwen_weights, prefill

    cfg = LMConfig(n_layers=1, vocab=64)
    w = synth.lm_weights(cfg, seed=9, with_embed=True)
    st = {"qwen_backbone." + k: torch.from_numpy(v).to(torch.bfloat16) for k, v in w.items()}
    st["head.other"] = torch.zeros(3)  # tensors of other modules are skipped
    path = str(tmp_path / "m.safetensors")
    save_file(st, path)
    m2 = load_qwen_weights(path, cfg)
    assert m2.missing == 0
    m3, _ = lm_model(cfg, seed=9, with_embed=True)
    m3.set_weights(bf16_weights(w))
    x = rnd(3, (5, cfg.hidden))
    a = prefill(m2, x, QwenCache(m2, 1, 8))
    b = prefill(m3, x, QwenCache(m3, 1, 8))
    assert np.array_equal(a, b)


def test_tensor_core_decode_batch16():
    """Batched decode with 16 utterances uses the tcgen05 linears."""
    from rcutetts_b200.model import QwenCache, decode_step, prefill

    cfg = LMConfig(n_layers=2)
    m, w = lm_model(cfg, seed=10, dtype="bf16")
    wo = bf16_weights(w)
    B = 16
    cache = QwenCache(m, batch=B, capacity=48)
    pre = [rnd(100 + b, (3 + b, cfg.hidden)) for b in range(B)]
    for b in range(B):
        prefill(m, pre[b], cache, b)
    dec = rnd(200, (3, B, cfg.hidden))
    outs = [decode_step(m, dec[s], cache) for s in range(3)]
    for b in range(B):
        ref = run_oracle(cfg, wo, pre[b], dec[:, b, :], capacity=48)[3 + b:]
        for s in range(3):
            assert cosine(outs[s][b], ref[s]) >= 0.999, (b, s)


@pytest.mark.parametrize("dtype,B", [("bf16", 40), ("f32", 32)])
def test_large_batch_decode_stage_boundaries(dtype, B):
    """Enough utterances that the decode attention runs one CTA per
    (utterance, kv head) walking 128-key stages: ragged contexts that cross
    stage boundaries, and steps whose new key opens a stage (position 128,
    256), against the oracle."""
    from rcutetts_b200.model import QwenCache, decode_step, prefill

    cfg = LMConfig(n_layers=2)
    m, w = lm_model(cfg, seed=12, dtype=dtype)
    wo = bf16_weights(w) if dtype == "bf16" else w
    special = [126, 255, 1, 127, 300, 128, 254]
    lens = [special[b] if b < len(special) else 1 + (37 * b) % 290 for b in range(B)]
    cap = 312
    cache = QwenCache(m, batch=B, capacity=cap)
    pre = [rnd(300 + b, (lens[b], cfg.hidden)) for b in range(B)]
    for b in range(B):
        prefill(m, pre[b], cache, b)
    dec = rnd(400, (4, B, cfg.hidden))
    outs = [decode_step(m, dec[s], cache) for s in range(4)]
    for b in list(range(len(special))) + [B - 1]:
        ref = run_oracle(cfg, wo, pre[b], dec[:, b, :], capacity=cap)[lens[b]:]
        for s in range(4):
            if dtype == "f32":
                assert rel_err(outs[s][b], ref[s]) < 1e-4, (b, s)
            else:
                assert cosine(outs[s][b], ref[s]) >= 0.999, (b, s)


@pytest.mark.parametrize("batch,cfg", [
    (1, LMConfig()),
    (3, LMConfig(n_layers=4)),
    (2, LMConfig(hidden=768, n_layers=2, n_heads=8, n_kv_heads=4, head_dim=128, ffn=1536)),
])
def test_grid_decode_matches_launch_chain(monkeypatch, batch, cfg):
    """Small-batch fp32 decode as one grid-persistent launch (lm_grid.cu)
    against the per-layer launch chain (CTTS_LM_GRID=0): ragged prefills in
    both length orders, several steps, the cache lengths left behind, and the
    oracle per utterance."""
    from rcutetts_b200.model import QwenCache, decode_step, prefill

    m, w = lm_model(cfg, seed=70)
    for lens in ([4 + 5 * b for b in range(batch)], [14 - 5 * b for b in range(batch)]):
        pre = [rnd(700 + b, (lens[b], cfg.hidden)) for b in range(batch)]
        dec = rnd(720, (4, batch, cfg.hidden))
        outs = {}
        for grid in ("1", "0"):
            monkeypatch.setenv("CTTS_LM_GRID", grid)
            cache = QwenCache(m, batch=batch, capacity=40)
            for b in range(batch):
                prefill(m, pre[b], cache, b)
            outs[grid] = np.stack([decode_step(m, dec[s], cache) for s in range(4)])
            for b in range(batch):
                assert cache.len(b) == lens[b] + 4
        assert np.isfinite(outs["1"]).all()
        assert rel_err(outs["1"], outs["0"]) < 1e-4
        for b in range(batch):
            ref = run_oracle(cfg, w, pre[b], dec[:, b, :], capacity=40)[lens[b]:]
            for s in range(4):
                assert rel_err(outs["1"][s, b], ref[s]) < 1e-4, (lens, b, s)
