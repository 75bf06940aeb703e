"""CPU checks of the C-ABI library: it builds for sm_100a, loads without a GPU, exports every
entry point declared in include/pulsar_b200.h, and rejects bad arguments with the
reference's messages before touching the device."""

from __future__ import annotations

import ctypes as C
import os
import re

import pytest

from conftest import REPO
from pulsar_b200 import _lib, build

HEADER = os.path.join(REPO, "include", "pulsar_b200.h")


def _declared():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(pulsar_[a-z0-9_]+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_expected_entry_points():
    names = _declared()
    assert "pulsar_engine_create" in names and "pulsar_op_moe_router_topk" in names
    assert set(names) == set(_lib.PROTOTYPES), "ctypes prototypes and header disagree"


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, f"symbols declared in the header but not exported: {missing}"


def test_abi_version(lib):
    assert lib.pulsar_abi_version() >= 100


def test_argument_errors_are_reported_without_a_gpu(lib):
    st = lib.pulsar_op_moe_router_topk(None, 0, None, 4, 33, 2, 0.0, None, None, None, None, None, None)
    assert st == -1
    assert "E <= 32" in _lib.last_error()
    st = lib.pulsar_op_moe_router_topk(None, 0, None, 4, 16, 9, 0.0, None, None, None, None, None, None)
    assert st == -1 and "top_k must be in" in _lib.last_error()
    st = lib.pulsar_op_moe_dispatch(None, None, None, None, 4, 2, 4, 8, 12, None, None)
    assert st == -1 and "multiple of 8" in _lib.last_error()
    # empty inputs are a no-op, as in the reference (csrc/kernels.cu:232-234)
    assert lib.pulsar_op_rmsnorm(None, None, 0, 64, 1e-6, None, None, None) == 0
    assert lib.pulsar_op_rope(None, None, None, 0, 1, 64, None, None) == 0


def test_engine_config_is_validated(lib):
    ec = _lib.EngineConfig(vocab_size=1000, max_pulses=8, loop_lora_rank=8, loop_lora_alpha=16.0, rms_eps=1e-6,
                           logit_softcap=30.0, base_seq_len=1024, use_canon_conv=1, per_pulse_bias=1, max_batch=1,
                           max_seq_len=256, max_prefill=128, kv_fp32=0, device=0)
    h = C.c_void_p()
    assert lib.pulsar_engine_create(C.byref(ec), C.byref(h)) == -1
    assert "multiple of 256" in _lib.last_error()
    ec.vocab_size = 32768
    ec.max_batch = 0
    assert lib.pulsar_engine_create(C.byref(ec), C.byref(h)) == -1
    assert "max_batch" in _lib.last_error()


def test_engine_calls_on_null_handle(lib):
    assert lib.pulsar_engine_finalize(None) == -1
    n = C.c_int32()
    assert lib.pulsar_engine_get_length(None, 0, C.byref(n)) == -1
    assert lib.pulsar_engine_destroy(None) == 0
