"""Host API over the C ABI, with the reference sampler's parameter names.

Reference call sites this mirrors (sarthak-fleet/tinygpt):
  sample_next(logits, temperature, top_k, generator)
      <- the sampling block of TinyGPT.generate, python_ref/model.py:213-224
         (temperature <= 0 is greedy; top_k None disables top-k)
  Sampler.sample(...)  <- batched form with per-row penalties, top-p, min-p and
      grammar-state masks (ModelController.swift:262-304, Serve.swift:1483-1506)
  SpecVerifier.verify(...) <- SpeculativeDecode.stepStochastic / step,
      native-mac/Sources/TinyGPT/SpeculativeDecode.swift:41-210

Device arrays are torch CUDA tensors (torch is only the allocator and stream
provider here); every call goes through libtgsample.so.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import ROW_PARAMS_DTYPE, TGError, check  # noqa: F401

try:
    import torch
except ImportError:  # pragma: no cover - the host API needs torch for device memory
    torch = None


def row_params(batch: int, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0,
               repetition_penalty=1.0, presence_penalty=0.0, frequency_penalty=0.0) -> np.ndarray:
    """Per-row parameter records (tg_row_params); scalars broadcast to every row."""
    p = np.zeros(batch, ROW_PARAMS_DTYPE)
    p["temperature"] = temperature
    p["top_k"] = 0 if top_k is None else top_k
    p["top_p"] = top_p
    p["min_p"] = min_p
    p["repetition_penalty"] = repetition_penalty
    p["presence_penalty"] = presence_penalty
    p["frequency_penalty"] = frequency_penalty
    return p


def _dtype_code(t) -> int:
    if t.dtype == torch.float32:
        return _lib.TG_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return _lib.TG_DTYPE_BF16
    raise TypeError(f"logits must be float32 or bfloat16, got {t.dtype}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream_ptr(stream):
    if stream is None:
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


def params_to_device(params: np.ndarray, device) -> "torch.Tensor":
    p = np.ascontiguousarray(params, dtype=ROW_PARAMS_DTYPE)
    return torch.from_numpy(p.view(np.int32).reshape(len(p), 8).copy()).to(device)


class Sampler:
    """A tg_sampler handle on one CUDA device (one handle per device and thread)."""

    def __init__(self, vocab: int, max_batch: int, device: int = 0):
        self._L = _lib.load()
        self.vocab = int(vocab)
        self.max_batch = int(max_batch)
        self.device = int(device)
        h = ctypes.c_void_p()
        check(self._L.tg_sampler_create(self.device, self.vocab, self.max_batch, ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def reserve(self, max_K: int = 0, max_ranks: int = 0) -> None:
        """tg_sampler_reserve: buffers for tg_spec_verify of up to max_K proposals
        and tg_sample_sharded of up to max_ranks ranks at max_batch rows.  The
        wrappers below call it when a call needs more than was reserved; call it
        up front to keep every later call allocation-free."""
        k = max(max_K, getattr(self, "_res_K", -1))
        r = max(max_ranks, getattr(self, "_res_ranks", 0))
        if k == getattr(self, "_res_K", -1) and r == getattr(self, "_res_ranks", 0):
            return
        check(self._L.tg_sampler_reserve(self._h, max(k, 0), r))
        self._res_K, self._res_ranks = max(k, 0), r

    def set_collective_timeout(self, ms: int) -> None:
        """Deadline of tg_sample_sharded's all-gather (0: no host wait)."""
        check(self._L.tg_sampler_set_collective_timeout(self._h, int(ms)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.tg_sampler_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def sample(self, logits, params, *, history=None, history_len=None, mask_table=None,
               state_id=None, uniforms=None, out=None, out_probs=None, stream=None):
        """tg_sample on device tensors.  logits [B, stride] fp32/bf16; params is a
        device int32 [B, 8] tensor (params_to_device) or a numpy record array.
        Returns (ids int32 [B], probs float32 [B] or None)."""
        B, stride = logits.shape
        if logits.stride(1) != 1:
            raise ValueError("logits rows must be contiguous")
        dev = logits.device
        if isinstance(params, np.ndarray):
            params = params_to_device(params, dev)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=dev)
        hstride = 0
        if history is not None:
            hstride = history.shape[1]
        nstates = 0
        if mask_table is not None:
            nstates = mask_table.shape[0]
        check(self._L.tg_sample(self._h, _ptr(logits), _dtype_code(logits), logits.stride(0), B,
                                _ptr(params), _ptr(history), _ptr(history_len), hstride,
                                _ptr(mask_table), nstates, _ptr(state_id), _ptr(uniforms),
                                _ptr(out), _ptr(out_probs), _stream_ptr(stream)))
        return out, out_probs

    def sample_host(self, logits: np.ndarray, params: np.ndarray, *, history=None,
                    history_len=None, mask_table=None, state_id=None, uniforms=None,
                    want_probs: bool = False):
        """tg_sample_host on numpy arrays (logits float32, or uint16 bf16 bit patterns)."""
        logits = np.ascontiguousarray(logits)
        B, stride = logits.shape
        code = _lib.TG_DTYPE_F32 if logits.dtype == np.float32 else _lib.TG_DTYPE_BF16
        if logits.dtype not in (np.float32, np.uint16):
            raise TypeError("logits must be float32 or uint16 (bf16 bits)")
        params = np.ascontiguousarray(params, dtype=ROW_PARAMS_DTYPE)
        hstride = 0
        if history is not None:
            history = np.ascontiguousarray(history, dtype=np.int32)
            history_len = np.ascontiguousarray(history_len, dtype=np.int32)
            hstride = history.shape[1]
        nstates = 0
        if mask_table is not None:
            mask_table = np.ascontiguousarray(mask_table, dtype=np.uint32)
            state_id = np.ascontiguousarray(state_id, dtype=np.int32)
            nstates = mask_table.shape[0]
        if uniforms is not None:
            uniforms = np.ascontiguousarray(uniforms, dtype=np.float32)
        out = np.empty(B, np.int32)
        probs = np.empty(B, np.float32) if want_probs else None
        p = lambda a: None if a is None else ctypes.c_void_p(a.ctypes.data)  # noqa: E731
        check(self._L.tg_sample_host(self._h, p(logits), code, stride, B, p(params), p(history),
                                     p(history_len), hstride, p(mask_table), nstates,
                                     p(state_id), p(uniforms), p(out), p(probs)))
        return out, probs

    def spec_verify(self, target_logits, draft_logits, draft_ids, temperature, u_accept, u_draw,
                    *, out=None, out_n=None, stream=None):
        """tg_spec_verify on device tensors.  target [B, K+1, V], draft [B, K, V]
        (draft_logits and u_accept None: greedy verification without a draft,
        Medusa / EAGLE style)."""
        B, K1, V = target_logits.shape
        K = K1 - 1
        if V != self.vocab:
            raise ValueError("vocab mismatch")
        dev = target_logits.device
        if out is None:
            out = torch.empty((B, K + 1), dtype=torch.int32, device=dev)
        if out_n is None:
            out_n = torch.empty(B, dtype=torch.int32, device=dev)
        self.reserve(max_K=K)
        check(self._L.tg_spec_verify(self._h, _ptr(target_logits), _ptr(draft_logits),
                                     _dtype_code(target_logits), B, K, _ptr(draft_ids),
                                     _ptr(temperature), _ptr(u_accept), _ptr(u_draw), _ptr(out),
                                     _ptr(out_n), _stream_ptr(stream)))
        return out, out_n

    def spec_verify_masked(self, target_logits, draft_logits, draft_ids, temperature, u_accept,
                           u_draw, mask_table, state_ids, *, out=None, out_n=None, stream=None):
        """tg_spec_verify_masked: mask_table int32/uint32 [S, ceil(V/32)] and
        state_ids int32 [B, K+1] device tensors (the grammar state before each
        position's token)."""
        B, K1, V = target_logits.shape
        K = K1 - 1
        dev = target_logits.device
        if out is None:
            out = torch.empty((B, K + 1), dtype=torch.int32, device=dev)
        if out_n is None:
            out_n = torch.empty(B, dtype=torch.int32, device=dev)
        self.reserve(max_K=K)
        check(self._L.tg_spec_verify_masked(self._h, _ptr(target_logits), _ptr(draft_logits),
                                            _dtype_code(target_logits), B, K, _ptr(draft_ids),
                                            _ptr(temperature), _ptr(u_accept), _ptr(u_draw),
                                            _ptr(mask_table), mask_table.shape[0], _ptr(state_ids),
                                            _ptr(out), _ptr(out_n), _stream_ptr(stream)))
        return out, out_n

    def sample_shard_local(self, logits, params, vocab_offset: int, full_vocab: int, *,
                           history=None, history_len=None, mask_table=None, state_id=None,
                           out_records=None, stream=None):
        """tg_sample_shard_local: this handle's vocab slice [vocab_offset, +vocab) of
        every row -> one record per row (uint8 [B, SHARD_RECORD_BYTES])."""
        B, stride = logits.shape
        dev = logits.device
        if isinstance(params, np.ndarray):
            params = params_to_device(params, dev)
        if out_records is None:
            out_records = torch.empty((B, _lib.SHARD_RECORD_BYTES), dtype=torch.uint8, device=dev)
        hstride = history.shape[1] if history is not None else 0
        nstates = mask_table.shape[0] if mask_table is not None else 0
        check(self._L.tg_sample_shard_local(self._h, vocab_offset, full_vocab, _ptr(logits),
                                            _dtype_code(logits), logits.stride(0), B, _ptr(params),
                                            _ptr(history), _ptr(history_len), hstride,
                                            _ptr(mask_table), nstates, _ptr(state_id),
                                            _ptr(out_records), _stream_ptr(stream)))
        return out_records

    def sample_shard_merge(self, records, full_vocab: int, params, *, uniforms=None, out=None,
                           out_probs=None, stream=None):
        """tg_sample_shard_merge over gathered records uint8 [nshards, B, RECORD]."""
        nshards, B, _ = records.shape
        dev = records.device
        if isinstance(params, np.ndarray):
            params = params_to_device(params, dev)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=dev)
        check(self._L.tg_sample_shard_merge(self._h, _ptr(records), nshards, full_vocab, B,
                                            _ptr(params), _ptr(uniforms), _ptr(out),
                                            _ptr(out_probs), _stream_ptr(stream)))
        return out, out_probs

    def sample_sharded(self, nccl_comm, nranks: int, logits, params, vocab_offset: int, full_vocab: int, *,
                       history=None, history_len=None, mask_table=None, state_id=None, uniforms=None,
                       out=None, out_probs=None, stream=None):
        """tg_sample_sharded: this rank's vocab slice of every row, the record
        all-gather over the NCCL communicator (an ncclComm_t pointer, see
        tinygpt_b200.dist.NcclComm) and the merge; ids for the whole rows."""
        B, _ = logits.shape
        dev = logits.device
        if isinstance(params, np.ndarray):
            params = params_to_device(params, dev)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=dev)
        hstride = history.shape[1] if history is not None else 0
        nstates = mask_table.shape[0] if mask_table is not None else 0
        self.reserve(max_ranks=nranks)
        check(self._L.tg_sample_sharded(self._h, ctypes.c_void_p(int(nccl_comm)), nranks, vocab_offset,
                                        full_vocab, _ptr(logits), _dtype_code(logits), logits.stride(0), B,
                                        _ptr(params), _ptr(history), _ptr(history_len), hstride,
                                        _ptr(mask_table), nstates, _ptr(state_id), _ptr(uniforms),
                                        _ptr(out), _ptr(out_probs), _stream_ptr(stream)))
        return out, out_probs

    def path_counters(self, reset: bool = True) -> dict:
        """Row counts per sampling path since the last reset (see tgsample.h)."""
        buf = (ctypes.c_uint64 * 8)()
        check(self._L.tg_sampler_path_counters(self._h, buf, 8, int(reset)))
        keys = ["candidate", "overflow", "short", "threshold", "full_row", "candidates", "warp_finished",
                "pool_full"]
        return {k: int(buf[i]) for i, k in enumerate(keys)}

    def profile(self, enable: bool = True):
        """Kernel times (ms) of the last tg_sample call recorded while profiling
        was on: (stream, finish) in the two-kernel mode, (whole call,) otherwise;
        then switches recording on or off (tg_sampler_profile)."""
        ms = (ctypes.c_float * 2)()
        n = ctypes.c_int32(0)
        check(self._L.tg_sampler_profile(self._h, int(enable), ms, ctypes.byref(n)))
        return tuple(ms[i] for i in range(n.value))

    def device_status(self) -> int:
        bits = ctypes.c_uint32(0)
        check(self._L.tg_sampler_device_status(self._h, ctypes.byref(bits)))
        return bits.value


class SpecVerifier:
    """SpeculativeDecode-style wrapper: verify(target, draft, ids, temperature, ...)."""

    def __init__(self, vocab: int, max_batch: int, device: int = 0):
        self.s = Sampler(vocab, max_batch, device)

    def verify(self, target_logits, draft_logits, draft_ids, temperature, u_accept, u_draw):
        return self.s.spec_verify(target_logits, draft_logits, draft_ids, temperature, u_accept,
                                  u_draw)


_SAMPLERS: dict = {}


def sample_next(logits, temperature: float = 1.0, top_k=None, generator=None, *,
                top_p: float = 1.0, min_p: float = 0.0, uniforms=None):
    """Drop-in for the sampling block of TinyGPT.generate (python_ref/model.py:213-224).

    logits: [B, V] CUDA tensor (fp32 or bf16).  temperature <= 0 is greedy;
    top_k None disables top-k.  One uniform per row is drawn from `generator`
    (torch.rand on the generator's device) unless `uniforms` is given.
    Returns next ids as int64 [B, 1], like the reference.
    """
    B, V = logits.shape
    key = (logits.device.index or 0, V)
    s = _SAMPLERS.get(key)
    if s is None or s.max_batch < B:
        s = Sampler(V, max(B, 64), logits.device.index or 0)
        _SAMPLERS[key] = s
    params = row_params(B, temperature=temperature, top_k=top_k, top_p=top_p, min_p=min_p)
    if uniforms is None:
        gdev = generator.device if generator is not None else torch.device("cpu")
        uniforms = torch.rand(B, generator=generator, device=gdev, dtype=torch.float32)
    uniforms = uniforms.to(logits.device, torch.float32).contiguous()
    ids, _ = s.sample(logits.contiguous(), params, uniforms=uniforms)
    return ids.to(torch.int64).view(B, 1)
