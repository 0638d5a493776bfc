"""C-ABI surface checks that need no GPU: the library loads, exports every
entry point include/cutetts_b200.h declares, and rejects bad arguments."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def lib():
    from rcutetts_b200 import build, _lib

    if not os.path.exists(_lib.LIB_PATH):
        build.build()
    return _lib.load()


def declared_symbols():
    names = []
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            src = open(os.path.join(ROOT, "include", f)).read()
            names += re.findall(r"^CTTS_API[^(]*?\b(\w+)\(", src, re.M)
    return names


def test_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 45
    for n in names:
        assert hasattr(lib, n), n


def test_binding_table_matches_header(lib):
    from rcutetts_b200 import _lib

    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_version(lib):
    assert b"sm_100a" in lib.ctts_version()


def test_sway_timesteps_host(lib, golden):
    out = np.empty(11, np.float32)
    assert lib.ctts_sway_timesteps(10, C.c_float(-0.8), out.ctypes.data_as(C.POINTER(C.c_float))) == 0
    assert np.max(np.abs(out - golden("ref/base_sway.npy"))) < 1e-6
    # coefficient outside [-1, 2/(pi-2)] is rejected like diffusion_head.py:40-45
    assert lib.ctts_sway_timesteps(10, C.c_float(-1.5), out.ctypes.data_as(C.POINTER(C.c_float))) == -1


def test_null_arguments_rejected(lib):
    h = C.c_void_p()
    assert lib.ctts_lm_create(None, 0, C.byref(h)) == -1
    assert b"null" in lib.ctts_last_error()
    assert lib.ctts_dit_create(None, 0, C.byref(h)) == -1
    assert lib.ctts_vae_create(None, 0, C.byref(h)) == -1
    assert lib.ctts_lm_missing(None) == -1
    assert lib.ctts_kv_len(None, 0) < 0
    assert lib.ctts_engine_step(None, None, None, None) == -1


def test_reference_ffi_error_contract(lib, tmp_path):
    # ffi.rs:19-65: null on a failed load, -1 on a bad decode call
    assert lib.cutetts_vae_load(None) is None
    assert lib.cutetts_vae_load(str(tmp_path / "missing.safetensors").encode()) is None
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(b"\x04\x00\x00\x00\x00\x00\x00\x00{}  ")
    assert lib.cutetts_vae_load(str(bad).encode()) is None
    assert lib.cutetts_vae_decode(None, None, 8, None) == -1
    lib.cutetts_vae_free(None)


def test_bad_config_rejected_before_device(lib):
    from rcutetts_b200._lib import LMConfigC

    h = C.c_void_p()
    c = LMConfigC(768, 12, 12, 5, 64, 2048, 32000, 1e-6, 1e6, 1, 0)  # 12 % 5 != 0
    assert lib.ctts_lm_create(C.byref(c), 0, C.byref(h)) == -1
    c = LMConfigC(768, 12, 12, 4, 48, 2048, 32000, 1e-6, 1e6, 1, 0)  # head_dim 48
    assert lib.ctts_lm_create(C.byref(c), 0, C.byref(h)) == -1
