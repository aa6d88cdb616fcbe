"""ctypes binding of oracle/libtgs_oracle.so -- TEST INFRASTRUCTURE ONLY.

The C restatement in oracle/tgs_oracle.c is the checker for the CUDA path.
Each wrapper takes numpy arrays laid out exactly like the device arrays of
include/tgsample.h and returns numpy outputs.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

ROW_PARAMS_DTYPE = np.dtype([
    ("temperature", np.float32), ("top_p", np.float32), ("min_p", np.float32),
    ("repetition_penalty", np.float32), ("presence_penalty", np.float32),
    ("frequency_penalty", np.float32), ("top_k", np.int32), ("flags", np.int32),
])


def build() -> None:
    """Compile the oracle (and the reference harness when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libtgs_oracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        L.tgo_sample.argtypes = [vp, i32, i64, i32, i32, vp, vp, vp, i32, vp, i32, vp, vp, vp, vp]
        L.tgo_sample.restype = i32
        L.tgo_spec_verify.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]
        L.tgo_spec_verify.restype = i32
        L.tgo_spec_verify_masked.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, i32, vp, vp, vp]
        L.tgo_spec_verify_masked.restype = i32
        L.tgo_exp.argtypes = [ctypes.c_float]
        L.tgo_exp.restype = ctypes.c_float
        L.tgo_qmass.argtypes = [ctypes.c_float]
        L.tgo_qmass.restype = ctypes.c_uint64
        L.tgo_sample_row_detail.argtypes = [vp, i32, i32, vp, vp, i32, vp, ctypes.c_float,
                                            vp, vp, vp, vp]
        L.tgo_sample_row_detail.restype = i32
        _LIB = L
    return _LIB


def ref_lib():
    """The reference's own C++ sampler harness (oracle/_ref/libtgref.so) or None."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "libtgref.so")
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        L.tgref_generate_fixed_logits.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_float,
                                                  ctypes.c_int, ctypes.c_uint, ctypes.c_int,
                                                  ctypes.c_void_p]
        L.tgref_generate_fixed_logits.restype = ctypes.c_int
        L.tgref_canonical_uniforms.argtypes = [ctypes.c_uint, ctypes.c_int, ctypes.c_void_p]
        L.tgref_canonical_uniforms.restype = None
        _REF = L
    return _REF


def _p(a):
    return None if a is None else a.ctypes.data


def dtype_code(logits: np.ndarray) -> int:
    if logits.dtype == np.float32:
        return 0
    if logits.dtype == np.uint16:  # bf16 bit patterns
        return 1
    raise TypeError(f"logits must be float32 or uint16 (bf16 bits), got {logits.dtype}")


def sample(logits, params, history=None, history_len=None, mask_table=None, state_id=None,
           uniforms=None, vocab=None):
    """Oracle tg_sample.  logits [B, stride] float32 or uint16 (bf16 bits)."""
    logits = np.ascontiguousarray(logits)
    B, stride = logits.shape
    V = stride if vocab is None else vocab
    params = np.ascontiguousarray(params, dtype=ROW_PARAMS_DTYPE)
    hstride = 0
    if history is not None:
        history = np.ascontiguousarray(history, dtype=np.int32)
        hstride = history.shape[1]
        history_len = np.ascontiguousarray(history_len, dtype=np.int32)
    nstates = 0
    if mask_table is not None:
        mask_table = np.ascontiguousarray(mask_table, dtype=np.uint32)
        nstates = mask_table.shape[0]
        state_id = np.ascontiguousarray(state_id, dtype=np.int32)
    if uniforms is not None:
        uniforms = np.ascontiguousarray(uniforms, dtype=np.float32)
    out = np.empty(B, np.int32)
    probs = np.empty(B, np.float32)
    rc = lib().tgo_sample(_p(logits), dtype_code(logits), stride, B, V, _p(params), _p(history),
                          _p(history_len), hstride, _p(mask_table), nstates, _p(state_id),
                          _p(uniforms), _p(out), _p(probs))
    if rc != 0:
        raise RuntimeError(f"tgo_sample failed: {rc}")
    return out, probs


def sample_row_detail(logits_row, params_row, history=None, mask=None, u=0.0):
    """One row with per-token detail: (id, prob, y, stage bits, masses)."""
    logits_row = np.ascontiguousarray(logits_row)
    V = logits_row.shape[0]
    p = np.ascontiguousarray(np.array([params_row], dtype=ROW_PARAMS_DTYPE))
    hist = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint32)
    y = np.empty(V, np.float32)
    st = np.empty(V, np.uint8)
    q = np.empty(V, np.uint64)
    prob = ctypes.c_float(0)
    i = lib().tgo_sample_row_detail(_p(logits_row), dtype_code(logits_row), V, _p(p), _p(hist),
                                    0 if hist is None else len(hist), _p(m), float(u),
                                    ctypes.addressof(prob), _p(y), _p(st), _p(q))
    return i, prob.value, y, st, q


def spec_verify(target, draft, draft_ids, temperature, u_accept, u_draw):
    """Oracle tg_spec_verify.  target [B,K+1,V], draft [B,K,V] float32 or bf16 bits."""
    target = np.ascontiguousarray(target)
    B, K1, V = target.shape
    K = K1 - 1
    draft = np.ascontiguousarray(draft) if draft is not None else None
    draft_ids = np.ascontiguousarray(draft_ids, dtype=np.int32)
    temperature = np.ascontiguousarray(temperature, dtype=np.float32)
    u_accept = np.ascontiguousarray(u_accept, dtype=np.float32)
    u_draw = np.ascontiguousarray(u_draw, dtype=np.float32)
    out = np.empty((B, K + 1), np.int32)
    n = np.empty(B, np.int32)
    rc = lib().tgo_spec_verify(_p(target), _p(draft), dtype_code(target), B, K, V, _p(draft_ids),
                               _p(temperature), _p(u_accept), _p(u_draw), _p(out), _p(n))
    if rc != 0:
        raise RuntimeError(f"tgo_spec_verify failed: {rc}")
    return out, n


def spec_verify_masked(target, draft, draft_ids, temperature, u_accept, u_draw, mask_table, state_ids):
    """Oracle tg_spec_verify_masked: mask_table [S, ceil(V/32)] uint32, state_ids [B, K+1]."""
    target = np.ascontiguousarray(target)
    B, K1, V = target.shape
    K = K1 - 1
    draft = np.ascontiguousarray(draft) if draft is not None else None
    args = [np.ascontiguousarray(draft_ids, dtype=np.int32), np.ascontiguousarray(temperature, dtype=np.float32),
            np.ascontiguousarray(u_accept, dtype=np.float32), np.ascontiguousarray(u_draw, dtype=np.float32)]
    mask_table = np.ascontiguousarray(mask_table, dtype=np.uint32)
    state_ids = np.ascontiguousarray(state_ids, dtype=np.int32)
    out = np.empty((B, K + 1), np.int32)
    n = np.empty(B, np.int32)
    rc = lib().tgo_spec_verify_masked(_p(target), _p(draft), dtype_code(target), B, K, V,
                                      *[_p(x) for x in args], _p(mask_table), mask_table.shape[0],
                                      _p(state_ids), _p(out), _p(n))
    if rc != 0:
        raise RuntimeError(f"tgo_spec_verify_masked failed: {rc}")
    return out, n


def exp32(x: float) -> float:
    return lib().tgo_exp(float(x))


def qmass(d: float) -> int:
    return lib().tgo_qmass(float(d))
