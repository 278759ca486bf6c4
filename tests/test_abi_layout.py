"""The ctypes view of the C-ABI matches include/gemma_b200.h byte for byte (CPU only).

A small C program built with gcc against the header prints the size and every field offset of
gg_config and gg_sample and the values of the GG_* constants; the ctypes structures and Python
constants the binding passes to the library must agree, or every call would read shifted fields.
"""
import ctypes
import os
import subprocess

import pytest

from conftest import ROOT

CONFIG_FIELDS = ["hidden_size", "q_dim", "kv_dim", "num_q_heads", "num_kv_heads", "head_dim",
                 "intermediate_size", "vocab_size", "num_layers", "context_length", "rms_norm_eps",
                 "rope_theta_global", "rope_theta_swa", "swa_period", "max_seqs", "flags", "sliding_window"]
SAMPLE_FIELDS = ["temperature", "top_p", "rep_penalty"]
CONSTANTS = ["GG_OK", "GG_E_ARG", "GG_E_CUDA", "GG_E_STATE", "GG_E_DEVICE", "GG_E_NOMEM",
             "GG_FLAG_SERIAL_PREFILL", "GG_FLAG_KV_BF16"]


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    d = tmp_path_factory.mktemp("abi")
    lines = ["#include <stddef.h>", "#include <stdio.h>", "#include <stdint.h>", '#include "gemma_b200.h"',
             "int main(void) {",
             '  printf("sizeof gg_config %zu\\n", sizeof(gg_config));',
             '  printf("sizeof gg_sample %zu\\n", sizeof(gg_sample));']
    lines += [f'  printf("gg_config.{f} %zu\\n", offsetof(gg_config, {f}));' for f in CONFIG_FIELDS]
    lines += [f'  printf("gg_sample.{f} %zu\\n", offsetof(gg_sample, {f}));' for f in SAMPLE_FIELDS]
    lines += [f'  printf("{c} %d\\n", (int)({c}));' for c in CONSTANTS]
    lines += ["  return 0;", "}"]
    src = d / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = d / "layout"
    subprocess.check_call(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)])
    out = subprocess.check_output([str(exe)], text=True)
    return {k: int(v) for k, v in (ln.rsplit(" ", 1) for ln in out.strip().splitlines())}


def test_config_layout(c_layout):
    from gemma_b200.config import CConfig
    assert [f for f, _ in CConfig._fields_] == CONFIG_FIELDS
    assert ctypes.sizeof(CConfig) == c_layout["sizeof gg_config"]
    for f in CONFIG_FIELDS:
        assert getattr(CConfig, f).offset == c_layout[f"gg_config.{f}"], f


def test_sample_layout(c_layout):
    from gemma_b200.native import GGSample
    assert [f for f, _ in GGSample._fields_] == SAMPLE_FIELDS
    assert ctypes.sizeof(GGSample) == c_layout["sizeof gg_sample"]
    for f in SAMPLE_FIELDS:
        assert getattr(GGSample, f).offset == c_layout[f"gg_sample.{f}"], f


def test_constants(c_layout):
    from gemma_b200 import config, native
    assert (native.GG_OK, native.GG_E_ARG, native.GG_E_CUDA, native.GG_E_STATE, native.GG_E_DEVICE,
            native.GG_E_NOMEM) == tuple(c_layout[c] for c in CONSTANTS[:6])
    assert native.GG_FLAG_SERIAL_PREFILL == c_layout["GG_FLAG_SERIAL_PREFILL"]
    assert config.GG_FLAG_KV_BF16 == c_layout["GG_FLAG_KV_BF16"]
