"""ctts_op_linear_noalloc: the op-level linear for callers that cannot
allocate device memory (their device heap is owned by a pool, or a serving
loop must not allocate after set-up because cudaMalloc synchronizes the
device).  It keeps the bf16 tensor-core operand in a fixed static device
array instead of a cudaMalloc'd buffer.  Checked through the C ABI against
ctts_op_linear, on two calls in a row (the array keeps the previous call's
contents), with the device's free memory unchanged across a repeated call.
This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err
from rcutetts_b200 import synth

pytestmark = pytest.mark.gpu


def _lib():
    from rcutetts_b200 import _lib

    return _lib.load()


def _run(fn, x, wdev, g, res, M, K, N):
    import torch

    y = torch.empty((M, N), device="cuda")
    rc = fn(x.data_ptr(), M, K, wdev.data_ptr(), 1, N, g.data_ptr(), C.c_float(1e-6), res.data_ptr(),
            y.data_ptr(), None)
    assert rc == 0, _lib().ctts_last_error()
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_noalloc_matches_allocating_linear_twice():
    import torch

    lib = _lib()
    rng = np.random.default_rng(11)
    cases = [(64, 768, 2048), (192, 512, 1536)]  # different shapes: the array is reused
    for M, K, N in cases:
        x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
        W = synth.to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * 0.02).view(np.int16)
        wdev = torch.from_numpy(W).cuda()
        g = torch.ones(K, device="cuda")
        res = torch.from_numpy(rng.standard_normal((M, N), dtype=np.float32)).cuda()
        ref = _run(lib.ctts_op_linear, x, wdev, g, res, M, K, N)
        for _ in range(2):
            got = _run(lib.ctts_op_linear_noalloc, x, wdev, g, res, M, K, N)
            assert rel_err(got, ref) < 1e-4
        # a repeated call takes no device memory (the output is allocated
        # beforehand; the driver's free-memory count must not move)
        y = torch.empty((M, N), device="cuda")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = lib.ctts_op_linear_noalloc(x.data_ptr(), M, K, wdev.data_ptr(), 1, N, g.data_ptr(), C.c_float(1e-6),
                                        res.data_ptr(), y.data_ptr(), None)
        torch.cuda.synchronize()
        assert rc == 0 and torch.cuda.mem_get_info()[0] == free0
        assert rel_err(y.cpu().numpy(), ref) < 1e-4


def test_noalloc_rejects_oversize():
    import torch

    lib = _lib()
    M, K, N = 1024, 2048, 128  # M*K = 2^21 > 2^20
    x = torch.zeros((M, K), device="cuda")
    w = torch.zeros((N, K), dtype=torch.int16, device="cuda")
    y = torch.empty((M, N), device="cuda")
    rc = lib.ctts_op_linear_noalloc(x.data_ptr(), M, K, w.data_ptr(), 1, N, None, C.c_float(1e-6), None,
                                    y.data_ptr(), None)
    assert rc == -7
    assert b"exceeds the static operand" in lib.ctts_last_error()
