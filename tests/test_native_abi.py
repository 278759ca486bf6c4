"""The C-ABI library loads and exports every function include/gemma_b200.h declares.

These run without a GPU: no compute call is made; gg_create must fail cleanly with an
error code and a message when no CUDA device is present.
"""
import ctypes
import os
import re

import pytest

from conftest import ROOT, has_gpu


def declared_functions():
    src = open(os.path.join(ROOT, "include", "gemma_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gg_[a-z_0-9]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from gemma_b200 import native
    if not os.path.exists(native.LIB_PATH):
        import subprocess, sys
        subprocess.check_call([sys.executable, os.path.join(ROOT, "webgpu-gemma_b200", "build.py")])
    return native.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    from gemma_b200 import native
    assert set(names) <= set(native.SIGNATURES)


def test_version_string(lib):
    assert b"sm_100a" in lib.gg_version()


@pytest.mark.skipif(has_gpu(), reason="checks the no-device error path")
def test_create_without_gpu_fails_cleanly(lib):
    from gemma_b200.config import to_cconfig
    from gemma_b200.synth import SHAPES
    h = ctypes.c_void_p()
    rc = lib.gg_create(ctypes.byref(to_cconfig(SHAPES["tiny"].config())), 0, ctypes.byref(h))
    assert rc < 0 and not h.value
    assert lib.gg_last_error(None)


def test_bad_config_rejected(lib):
    from gemma_b200.config import to_cconfig
    from gemma_b200.synth import SHAPES
    c = to_cconfig(SHAPES["tiny"].config())
    c.hidden_size = 100  # not a multiple of 32
    h = ctypes.c_void_p()
    assert lib.gg_create(ctypes.byref(c), 0, ctypes.byref(h)) == -1
    assert b"config" in lib.gg_last_error(None)


def test_noalloc_sampler_rejects_oversize_vocab(lib):
    """The size check comes before any CUDA call, so it runs without a GPU."""
    from gemma_b200.native import GGSample
    s = GGSample(0.0, 0.9, 1.0)
    out = ctypes.c_int32()
    rc = lib.gg_sample_logits_noalloc(ctypes.c_void_p(16), 524289, None, ctypes.byref(s), 0.0,
                                      ctypes.byref(out), None)
    assert rc == -1
    assert b"524288" in lib.gg_last_error(None)
    assert lib.gg_sample_logits_noalloc(None, 1000, None, ctypes.byref(s), 0.0, ctypes.byref(out), None) == -1
