"""config[1]: the fused layer kernels on their own, through the op-level
C-ABI entry points, against the oracle (seed 1, N(0,1) inputs, N(0,0.02)
weights)."""
import ctypes as C

import numpy as np
import pytest

from conftest import cosine, rel_err
from helpers import rnd
from oracle import oracle as orc
from rcutetts_b200 import synth

pytestmark = pytest.mark.gpu

SHAPES = [(768, 768), (768, 2048), (2048, 768), (768, 2304)]


def lib():
    from rcutetts_b200 import _lib

    return _lib.load()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("KN", SHAPES)
@pytest.mark.parametrize("M", [1, 8, 64, 256])
def test_linear_rmsnorm_residual(M, KN, dtype):
    import torch

    K, N = KN
    rng = np.random.default_rng(1)
    x = rng.standard_normal((M, K), dtype=np.float32)
    W = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    res = rng.standard_normal((M, N), dtype=np.float32)
    g = np.ones(K, np.float32)
    if dtype == "bf16":
        W = synth.bf16_round(W)
        wdev = torch.from_numpy(synth.to_bf16_bits(W).view(np.int16)).cuda()
    else:
        wdev = torch.from_numpy(W).cuda()
    xd, rd, gd = (torch.from_numpy(a).cuda() for a in (x, res, g))
    y = torch.empty((M, N), device="cuda")
    rc = lib().ctts_op_linear(xd.data_ptr(), M, K, wdev.data_ptr(), 1 if dtype == "bf16" else 0, N,
                              gd.data_ptr(), C.c_float(1e-6), rd.data_ptr(), y.data_ptr(), None)
    assert rc == 0
    torch.cuda.synchronize()
    ref = orc.linear(orc.rms_norm(x, g, 1e-6), W) + res
    got = y.cpu().numpy()
    if dtype == "bf16" and M >= 16:
        # tensor-core path: activations rounded to bf16 for the MMA
        assert cosine(got - res, ref - res) >= 0.9999
        assert rel_err(got, ref) < 1e-2
    else:
        assert rel_err(got, ref) < 1e-4


def test_rope_positions_0_4095():
    import torch

    M = 4096
    x = rnd(1, (M, 12, 64))
    pos = np.arange(M, dtype=np.int32)
    xd, pd = torch.from_numpy(x).cuda(), torch.from_numpy(pos).cuda()
    assert lib().ctts_op_rope(xd.data_ptr(), M, 12, 64, pd.data_ptr(), C.c_float(1e6), None) == 0
    torch.cuda.synchronize()
    ref = orc.rope(x, pos[:, None], 1e6)
    assert rel_err(xd.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("M", [1, 64])
def test_swiglu(M):
    import torch

    gu = rnd(2, (M, 2 * 2048))
    gd = torch.from_numpy(gu).cuda()
    out = torch.empty((M, 2048), device="cuda")
    assert lib().ctts_op_swiglu(gd.data_ptr(), M, 2048, out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    ref = orc.swiglu(gu[:, :2048], gu[:, 2048:])
    assert rel_err(out.cpu().numpy(), ref) < 1e-6


def test_embed_gather_bit_exact():
    import torch

    table = rnd(3, (32000, 768), 0.02)
    ids = np.random.default_rng(1).integers(0, 32000, 512)
    ids_bad = ids.copy()
    ids_bad[[5, 77]] = [-1, 32000]
    td = torch.from_numpy(table).cuda()
    for arr, nbad in ((ids, 0), (ids_bad, 2)):
        idd = torch.from_numpy(arr.astype(np.int64)).cuda()
        out = torch.empty((arr.size, 768), device="cuda")
        bad = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert lib().ctts_op_embed_gather(td.data_ptr(), 32000, 768, idd.data_ptr(), arr.size,
                                          out.data_ptr(), bad.data_ptr(), None) == 0
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        ok = (arr >= 0) & (arr < 32000)
        assert np.array_equal(o[ok], table[arr[ok]])
        assert np.all(o[~ok] == 0)
        assert int(bad.item()) == nbad
