"""The allocation-free speculative verification entry point (tg_spec_verify_static).

Some callers of this library cannot call cudaMalloc: a serving process that has
reserved all free HBM for its KV cache, or a decode loop that must not take the
device-wide synchronization an allocation can cause.  tg_spec_verify_static
keeps its scratch in a fixed array inside the library instead.  This test calls
it through the C ABI twice in a row (the array keeps the previous call's
contents) and checks both results against tg_spec_verify, bit for bit -- the
tolerance every parity test here uses -- and against the CPU oracle, at a
small and at the full vocabulary, in fp32 and bf16.  The file is named to be
collected last.
"""
import ctypes

import numpy as np
import pytest

from tinygpt_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_static_scratch_entry_matches_allocating_entry(cuda_lib):
    import torch
    from tinygpt_b200 import _lib
    from tinygpt_b200.sampler import Sampler

    V = 5003
    s = Sampler(V, 64, 0)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    for seed, B in ((21, 24), (22, 40)):  # two calls in a row, different shapes
        w = W.make(5, seed=seed, batch=B, vocab=V)
        w["temperature"][::4] = 0.0  # some greedy rows too
        dev = {k: torch.from_numpy(np.ascontiguousarray(w[k])).cuda()
               for k in ("target", "draft", "draft_ids", "temperature", "u_accept", "u_draw")}
        K = w["draft_ids"].shape[1]
        ref_ids, ref_n = s.spec_verify(dev["target"], dev["draft"], dev["draft_ids"],
                                       dev["temperature"], dev["u_accept"], dev["u_draw"])
        ids = torch.full((B, K + 1), -7, dtype=torch.int32, device="cuda:0")
        n = torch.full((B,), -7, dtype=torch.int32, device="cuda:0")
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = cuda_lib.tg_spec_verify_static(0, V, P(dev["target"]), P(dev["draft"]),
                                            _lib.TG_DTYPE_F32, B, K, P(dev["draft_ids"]),
                                            P(dev["temperature"]), P(dev["u_accept"]),
                                            P(dev["u_draw"]), P(ids), P(n), stream)
        assert rc == _lib.TG_OK, cuda_lib.tg_last_error_string()
        torch.cuda.synchronize()
        assert torch.equal(n, ref_n)
        assert torch.equal(ids, ref_ids)
    # beyond the static scratch: rejected with a clear error, nothing launched
    rc = cuda_lib.tg_spec_verify_static(0, V, P(dev["target"]), P(dev["draft"]),
                                        _lib.TG_DTYPE_F32, _lib.TG_STATIC_SPEC_MAX_ROWS, K,
                                        P(dev["draft_ids"]), P(dev["temperature"]),
                                        P(dev["u_accept"]), P(dev["u_draw"]), P(ids), P(n), stream)
    assert rc == _lib.TG_ERR_UNSUPPORTED
    assert b"TG_STATIC_SPEC_MAX_ROWS" in cuda_lib.tg_last_error_string()


@pytest.mark.parametrize("V,dtype", [(5003, "bf16"), (128256, "f32"), (128256, "bf16")])
def test_static_scratch_entry_matches_oracle(cuda_lib, oracle_mod, V, dtype):
    import torch
    from tinygpt_b200 import _lib
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    B = 16
    w = W.make(5, seed=41, batch=B, vocab=V)
    w["temperature"][::5] = 0.0
    if dtype == "bf16":  # the oracle sees the same bf16 values
        w["target"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["target"]))
        w["draft"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["draft"]))
    cv = (lambda a: torch.from_numpy(W.to_bf16_bits(a)).view(torch.int16).view(torch.bfloat16)) \
        if dtype == "bf16" else torch.from_numpy
    dev = {k: cv(w[k]).cuda() for k in ("target", "draft")}
    dev.update({k: torch.from_numpy(np.ascontiguousarray(w[k])).cuda()
                for k in ("draft_ids", "temperature", "u_accept", "u_draw")})
    K = w["draft_ids"].shape[1]
    code = _lib.TG_DTYPE_BF16 if dtype == "bf16" else _lib.TG_DTYPE_F32
    oo, on = oracle_mod.spec_verify(w["target"], w["draft"], w["draft_ids"], w["temperature"],
                                    w["u_accept"], w["u_draw"])
    for _ in range(2):  # twice in a row: the array keeps the previous call's contents
        ids = torch.full((B, K + 1), -7, dtype=torch.int32, device="cuda:0")
        n = torch.full((B,), -7, dtype=torch.int32, device="cuda:0")
        rc = cuda_lib.tg_spec_verify_static(0, V, P(dev["target"]), P(dev["draft"]), code, B, K,
                                            P(dev["draft_ids"]), P(dev["temperature"]), P(dev["u_accept"]),
                                            P(dev["u_draw"]), P(ids), P(n), None)
        assert rc == _lib.TG_OK, cuda_lib.tg_last_error_string()
        torch.cuda.synchronize()
        assert np.array_equal(n.cpu().numpy(), on)
        assert np.array_equal(ids.cpu().numpy(), oo)
        bits = ctypes.c_uint32(99)
        assert cuda_lib.tg_spec_verify_static_status(0, ctypes.byref(bits)) == _lib.TG_OK
        assert bits.value == 0
