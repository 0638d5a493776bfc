"""Failure detection on the device without a GPU fault: a bounded wait that
runs out ends in an error status the host reads, and the device stays usable.

The reference's contract is the panic -> -1 of its FFI
(rust-codec/src/ffi.rs:51-64); here every spin in a kernel is bounded and
records an error word instead of hanging.  The test switches on the
host-set fault of the small-batch DiT grid loop (CTA 0 leaves its QKV
exchange words unwritten, so the attention phase polls words no producer
writes) with a short poll limit, expects CTTS_ERR_TIMEOUT from the host call
within seconds, then switches it off and checks that the same handle gives
the fault-free result bit for bit, against the oracle."""
import time

import numpy as np
import pytest

from conftest import rel_err
from helpers import dit_model, rnd
from oracle import oracle as orc
from rcutetts_b200.config import DiTConfig

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_device_recovers():
    from rcutetts_b200 import _lib

    lib = _lib.load()
    cfg = DiTConfig()
    m, w = dit_model(cfg, seed=12)  # fp32, batch 2: the grid-persistent Euler loop
    x0, z, c = rnd(61, (2, 64)), rnd(62, (2, 768)), rnd(63, (2, 64))
    good = m.euler_sample(x0, z, c, z, 10)
    assert lib.ctts_debug_inject_wait_fault(1, 1 << 14) == 0
    try:
        t0 = time.time()
        with pytest.raises(_lib.CttsError) as e:
            m.euler_sample(x0, z, c, z, 10)
        took = time.time() - t0
    finally:
        assert lib.ctts_debug_inject_wait_fault(0, 0) == 0
    assert e.value.code == _lib.ERR_TIMEOUT, e.value
    assert took < 30.0, took
    again = m.euler_sample(x0, z, c, z, 10)
    assert np.array_equal(again, good)
    o = orc.DiT(cfg, w)
    for b in range(2):
        assert rel_err(again[b], o.euler_sample(x0[b], z[b], c[b], z[b], 10)) < 1e-4
