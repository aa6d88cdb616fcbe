"""ctypes binding of the C ABI in include/tgsample.h (libtgsample.so, in-tree).

There is no fallback: if the library is missing or fails to load, every entry
point raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("TGSAMPLE_LIB", os.path.join(HERE, "libtgsample.so"))

TG_OK = 0
TG_ERR_INVALID_ARG = -1
TG_ERR_CUDA = -2
TG_ERR_UNSUPPORTED = -3
TG_ERR_NO_DEVICE = -4
TG_ERR_DEVICE_STATUS = -5
TG_ERR_COLLECTIVE = -6
TG_DTYPE_F32 = 0
TG_DTYPE_BF16 = 1
TG_MAX_VOCAB = 1 << 20
TG_MAX_HISTORY = 4096
TG_STATIC_SPEC_MAX_ROWS = 8192
TG_SHARD_CAP = 1280
TG_GRAMMAR_JSON_SCHEMA = 0
TG_GRAMMAR_TOOL_TAGS = 1
SHARD_RECORD_BYTES = 16 + 8 * TG_SHARD_CAP

ROW_PARAMS_DTYPE = np.dtype([
    ("temperature", np.float32), ("top_p", np.float32), ("min_p", np.float32),
    ("repetition_penalty", np.float32), ("presence_penalty", np.float32),
    ("frequency_penalty", np.float32), ("top_k", np.int32), ("flags", np.int32),
])

EXPORTED = ["tg_abi_version", "tg_last_error_string", "tg_sampler_create", "tg_sampler_destroy",
            "tg_sample", "tg_sample_host", "tg_spec_verify", "tg_sampler_device_status", "tg_sampler_path_counters",
            "tg_spec_verify_static", "tg_sample_shard_local", "tg_sample_shard_merge", "tg_sampler_profile", "tg_spec_verify_masked", "tg_sample_sharded",
            "tg_sampler_reserve", "tg_sampler_set_collective_timeout", "tg_spec_verify_static_status",
            "tg_grammar_last_error", "tg_grammar_create", "tg_grammar_destroy",
            "tg_grammar_state_create", "tg_grammar_state_destroy", "tg_grammar_accept_bytes",
            "tg_grammar_kind", "tg_grammar_state_clone",
            "tg_grammar_commit", "tg_grammar_is_complete", "tg_grammar_mask",
            "tg_grammar_state_row", "tg_grammar_table"]


class TGError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"tgsample error {code}: {msg}")
        self.code = code


_LIB = None


def load(path: str = LIB_PATH):
    """Load libtgsample.so and declare every exported symbol's signature."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: run `python -m tinygpt_b200.build` "
                          "(the CUDA library is required; there is no CPU fallback)")
    L = ctypes.CDLL(path)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    L.tg_abi_version.argtypes = []
    L.tg_abi_version.restype = i32
    L.tg_last_error_string.argtypes = []
    L.tg_last_error_string.restype = ctypes.c_char_p
    L.tg_sampler_create.argtypes = [i32, i32, i32, ctypes.POINTER(vp)]
    L.tg_sampler_create.restype = i32
    L.tg_sampler_destroy.argtypes = [vp]
    L.tg_sampler_destroy.restype = i32
    L.tg_sample.argtypes = [vp, vp, i32, i64, i32, vp, vp, vp, i32, vp, i32, vp, vp, vp, vp, vp]
    L.tg_sample.restype = i32
    L.tg_sample_host.argtypes = [vp, vp, i32, i64, i32, vp, vp, vp, i32, vp, i32, vp, vp, vp, vp]
    L.tg_sample_host.restype = i32
    L.tg_spec_verify.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]
    L.tg_spec_verify.restype = i32
    L.tg_spec_verify_masked.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp, i32, vp, vp, vp, vp]
    L.tg_spec_verify_masked.restype = i32
    L.tg_sampler_device_status.argtypes = [vp, ctypes.POINTER(ctypes.c_uint32)]
    L.tg_sampler_device_status.restype = i32
    L.tg_sampler_path_counters.argtypes = [vp, vp, i32, i32]
    L.tg_sampler_path_counters.restype = i32
    L.tg_spec_verify_static.argtypes = [i32, i32, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp]
    L.tg_spec_verify_static.restype = i32
    L.tg_sample_shard_local.argtypes = [vp, i32, i32, vp, i32, i64, i32, vp, vp, vp, i32, vp, i32,
                                        vp, vp, vp]
    L.tg_sample_shard_local.restype = i32
    L.tg_sample_shard_merge.argtypes = [vp, vp, i32, i32, i32, vp, vp, vp, vp, vp]
    L.tg_sample_shard_merge.restype = i32
    L.tg_sample_sharded.argtypes = [vp, vp, i32, i32, i32, vp, i32, i64, i32, vp, vp, vp, i32, vp, i32, vp,
                                    vp, vp, vp, vp]
    L.tg_sample_sharded.restype = i32
    L.tg_sampler_reserve.argtypes = [vp, i32, i32]
    L.tg_sampler_reserve.restype = i32
    L.tg_sampler_set_collective_timeout.argtypes = [vp, i32]
    L.tg_sampler_set_collective_timeout.restype = i32
    L.tg_spec_verify_static_status.argtypes = [i32, ctypes.POINTER(ctypes.c_uint32)]
    L.tg_spec_verify_static_status.restype = i32
    L.tg_sampler_profile.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(i32)]
    L.tg_sampler_profile.restype = i32
    L.tg_grammar_last_error.argtypes = []
    L.tg_grammar_last_error.restype = ctypes.c_char_p
    L.tg_grammar_create.argtypes = [ctypes.c_char_p, i64, i32, vp, vp, i32, ctypes.POINTER(vp)]
    L.tg_grammar_destroy.argtypes = [vp]
    L.tg_grammar_state_create.argtypes = [vp, ctypes.POINTER(vp)]
    L.tg_grammar_state_destroy.argtypes = [vp]
    L.tg_grammar_kind.argtypes = [vp, ctypes.POINTER(i32)]
    L.tg_grammar_state_clone.argtypes = [vp, ctypes.POINTER(vp)]
    L.tg_grammar_accept_bytes.argtypes = [vp, ctypes.c_char_p, i64, ctypes.POINTER(i32)]
    L.tg_grammar_commit.argtypes = [vp, i32, ctypes.POINTER(i32)]
    L.tg_grammar_is_complete.argtypes = [vp, ctypes.POINTER(i32)]
    L.tg_grammar_mask.argtypes = [vp, vp]
    L.tg_grammar_state_row.argtypes = [vp, ctypes.POINTER(i32), ctypes.POINTER(i32)]
    L.tg_grammar_table.argtypes = [vp, ctypes.POINTER(ctypes.POINTER(ctypes.c_uint32)),
                                   ctypes.POINTER(i32)]
    for name in ("tg_grammar_create", "tg_grammar_destroy", "tg_grammar_state_create",
                 "tg_grammar_kind", "tg_grammar_state_clone",
                 "tg_grammar_state_destroy", "tg_grammar_accept_bytes", "tg_grammar_commit",
                 "tg_grammar_is_complete", "tg_grammar_mask", "tg_grammar_state_row",
                 "tg_grammar_table"):
        getattr(L, name).restype = i32
    _LIB = L
    return L


def check(rc: int) -> None:
    if rc != TG_OK:
        msg = load().tg_last_error_string().decode(errors="replace")
        raise TGError(rc, msg)
