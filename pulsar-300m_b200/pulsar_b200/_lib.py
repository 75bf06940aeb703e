"""ctypes binding of ``libpulsar_b200.so`` (the C ABI in ``include/pulsar_b200.h``).

The library is built in-tree by ``pulsar_b200.build``. There is no fallback: if the
library is missing or a call fails, a ``RuntimeError`` is raised with the library's own
error text (the same exception type ``TORCH_CHECK`` raises in the reference extension).
"""

from __future__ import annotations

import ctypes as C
import os

from .build import LIB

_lib = None

PULSAR_OK = 0
ERR_NAMES = {-1: "INVALID", -2: "CUDA", -3: "OOM", -4: "STATE", -5: "UNSUPPORTED", -6: "CAPACITY"}

c_void_p, c_int, c_int64, c_float, c_char_p = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_char_p


class EngineConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32), ("max_pulses", C.c_int32), ("loop_lora_rank", C.c_int32),
        ("loop_lora_alpha", C.c_float), ("rms_eps", C.c_float), ("logit_softcap", C.c_float),
        ("base_seq_len", C.c_int32), ("use_canon_conv", C.c_int32), ("per_pulse_bias", C.c_int32),
        ("max_batch", C.c_int32), ("max_seq_len", C.c_int32), ("max_prefill", C.c_int32),
        ("kv_fp32", C.c_int32), ("device", C.c_int32),
    ]


# name -> (restype, argtypes); every exported symbol of include/pulsar_b200.h
PROTOTYPES = {
    "pulsar_last_error": (c_char_p, []),
    "pulsar_abi_version": (c_int, []),
    "pulsar_op_rmsnorm": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p, c_void_p, c_void_p]),
    "pulsar_op_rope": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "pulsar_op_swiglu": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "pulsar_op_moe_router_topk": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int64, c_int64, c_float, c_void_p,
                                          c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "pulsar_op_moe_router_topk_noalloc": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int64, c_int64, c_float,
                                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "pulsar_op_qk_rmsnorm_rope": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                          c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p]),
    "pulsar_op_attn_gate": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "pulsar_op_conv1d_k4": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "pulsar_op_moe_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                      c_int64, c_int64, c_void_p, c_void_p]),
    "pulsar_op_moe_dispatch": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                       c_int64, c_void_p, c_void_p]),
    "pulsar_engine_create": (c_int, [C.POINTER(EngineConfig), C.POINTER(c_void_p)]),
    "pulsar_engine_destroy": (c_int, [c_void_p]),
    "pulsar_engine_set_tensor": (c_int, [c_void_p, c_char_p, c_void_p, c_int64]),
    "pulsar_engine_finalize": (c_int, [c_void_p]),
    "pulsar_engine_memory": (c_int, [c_void_p, C.POINTER(c_int64), C.POINTER(c_int64), C.POINTER(c_int64)]),
    "pulsar_engine_prefill": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "pulsar_engine_pulse": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p]),
    "pulsar_engine_get_length": (c_int, [c_void_p, c_int, C.POINTER(C.c_int32)]),
    "pulsar_engine_set_length": (c_int, [c_void_p, c_int, c_int]),
    "pulsar_engine_read_kv": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "pulsar_engine_forward": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "pulsar_engine_prefill_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p]),
    "pulsar_engine_decode_attention": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int,
                                               c_void_p]),
    "pulsar_engine_generate_greedy": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p,
                                              C.POINTER(c_int64), c_void_p]),
    "pulsar_engine_generate_sampled": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                               C.c_float, C.c_float, C.c_uint64, c_void_p, C.POINTER(c_int64),
                                               c_void_p]),
    "pulsar_engine_set_early_exit": (c_int, [c_void_p, c_int, C.c_float]),
    "pulsar_engine_early_exit_counts": (c_int, [c_void_p, C.POINTER(c_int64)]),
    "pulsar_engine_set_repetition_penalty": (c_int, [c_void_p, C.c_float]),
    "pulsar_engine_arena_count": (c_int, [c_void_p, C.POINTER(C.c_int32)]),
    "pulsar_engine_arena_info": (c_int, [c_void_p, c_int, C.POINTER(c_char_p), C.POINTER(c_int64)]),
    "pulsar_engine_arena_read": (c_int, [c_void_p, c_char_p, c_void_p, c_int64]),
    "pulsar_engine_arena_write": (c_int, [c_void_p, c_char_p, c_void_p, c_int64]),
    "pulsar_engine_set_option": (c_int, [c_void_p, c_char_p, c_int64]),
    "pulsar_engine_get_option": (c_int, [c_void_p, c_char_p, C.POINTER(c_int64)]),
    "pulsar_engine_read_trace": (c_int, [c_void_p, c_void_p, c_int64]),
}


def lib_path() -> str:
    return os.environ.get("PULSAR_B200_LIB", LIB)


def load():
    """Load the library (once) and attach prototypes. Raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise RuntimeError(f"libpulsar_b200.so not built at {path}: run `python -m pulsar_b200.build` "
                           f"(or __graft_entry__.build()); there is no CPU fallback")
    lib = C.CDLL(path)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    return load().pulsar_last_error().decode(errors="replace")


def check(status: int, what: str = "") -> None:
    if status != PULSAR_OK:
        raise RuntimeError(f"{what or 'pulsar_b200'} failed ({ERR_NAMES.get(status, status)}): {last_error()}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
