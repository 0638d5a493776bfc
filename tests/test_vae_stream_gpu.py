"""Streaming VAE decoder (stream.rs:62-139 StreamingDecoder) on the GPU:
decoding an utterance chunk by chunk, with each conv's left history carried
across chunks, gives exactly the samples of the offline decode (the
reference's stream_chunks_match_offline property, tests/stream.rs:31-76:
same taps => bit-identical), for AR-patch chunks of 2 frames, ragged chunk
sizes, after a reset, in fp32 and bf16, and at the config[4] length."""
import numpy as np
import pytest

from conftest import rel_err
from helpers import rnd
from oracle import oracle as orc
from rcutetts_b200 import synth
from rcutetts_b200.config import VAEConfig

pytestmark = pytest.mark.gpu


def model(dtype, seed=4):
    from rcutetts_b200.model import DecoderW

    cfg = VAEConfig()
    w = synth.vae_weights(cfg, seed=seed)
    return DecoderW(cfg, dtype).set_weights(w), w, cfg


def chunked(dec, lat, sizes):
    out, f = [], 0
    for n in sizes:
        out.append(dec.decode_chunk(lat[:, :, f:f + n]))
        f += n
    assert f == lat.shape[2]
    return np.concatenate(out, axis=1)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_chunks_match_offline_bit_for_bit(dtype):
    from rcutetts_b200.model import StreamingDecoder

    m, w, cfg = model(dtype)
    lat = rnd(40, (2, 64, 24))
    full = m.decode(lat)
    dec = StreamingDecoder(m, batch=2)
    assert np.array_equal(chunked(dec, lat, [2] * 12), full)
    dec.reset()
    assert np.array_equal(chunked(dec, lat, [1, 3, 2, 5, 4, 1, 8]), full)
    if dtype == "f32":
        o = orc.VAE(cfg, w)
        assert rel_err(full[0], o.decode(lat[0])) < 1e-4


def test_streams_are_independent_and_resumable():
    """Two streams over the same weights keep their own histories; a stream
    fed the second half after the first equals one fed everything."""
    from rcutetts_b200.model import StreamingDecoder

    m, _, _ = model("f32", seed=7)
    a, b = rnd(41, (1, 64, 10)), rnd(42, (1, 64, 10))
    s1, s2 = StreamingDecoder(m, 1), StreamingDecoder(m, 1)
    w1 = s1.decode_chunk(a[:, :, :6])
    w2 = s2.decode_chunk(b[:, :, :6])
    w1b = s1.decode_chunk(a[:, :, 6:])
    w2b = s2.decode_chunk(b[:, :, 6:])
    assert np.array_equal(np.concatenate([w1, w1b], 1), m.decode(a))
    assert np.array_equal(np.concatenate([w2, w2b], 1), m.decode(b))


def test_config4_length_in_ar_patches():
    """config[4] topology and length (T=400 frames, hop 320) in 2-frame
    patches, four utterances."""
    from rcutetts_b200.model import StreamingDecoder

    m, _, cfg = model("f32")
    lat = rnd(43, (4, 64, 400))
    full = m.decode(lat)
    dec = StreamingDecoder(m, batch=4)
    got = chunked(dec, lat, [2] * 200)
    assert got.shape == (4, 400 * cfg.hop)
    assert np.array_equal(got, full)
