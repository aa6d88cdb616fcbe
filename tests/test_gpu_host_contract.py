"""Host-side contract of the C ABI on a GPU handle: argument checks that run
before any launch, the reservation of buffers (hot calls allocate nothing), and
greedy verification without a draft distribution (Medusa / EAGLE heads,
MedusaHeads.swift:186-265, EagleDraft.swift:216-290)."""
import ctypes

import numpy as np
import pytest

from tinygpt_b200 import _lib
from tinygpt_b200 import workloads as W

pytestmark = pytest.mark.gpu

P = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731


def test_sharded_rejects_bad_slice_before_launch(cuda_lib):
    from tinygpt_b200.sampler import Sampler
    s = Sampler(1000, 8, 0)
    fake_comm = ctypes.c_void_p(1)  # never used: the slice check comes first
    for off, full in ((-1, 2000), (1500, 2000), (0, _lib.TG_MAX_VOCAB + 1), (0, 999)):
        rc = cuda_lib.tg_sample_sharded(s.handle, fake_comm, 2, off, full, None, 0, 1000, 1, None, None,
                                        None, 0, None, 0, None, None, None, None, None)
        assert rc == _lib.TG_ERR_INVALID_ARG, (off, full)
        assert b"vocab_offset" in cuda_lib.tg_last_error_string()


def test_verification_needs_reserved_statistics(cuda_lib):
    import torch
    from tinygpt_b200.sampler import Sampler
    V, B, K = 4099, 4, 3
    s = Sampler(V, 8, 0)
    w = W.make(5, seed=9, batch=B, vocab=V)
    d = {k: torch.from_numpy(np.ascontiguousarray(w[k][:, :K + 1] if k == "target" else w[k])).cuda()
         for k in ("target", "draft", "draft_ids", "temperature", "u_accept", "u_draw")}
    K = d["draft"].shape[1]
    out = torch.empty((B, K + 1), dtype=torch.int32, device="cuda:0")
    n = torch.empty(B, dtype=torch.int32, device="cuda:0")
    args = (P(d["target"]), P(d["draft"]), _lib.TG_DTYPE_F32, B, K, P(d["draft_ids"]), P(d["temperature"]),
            P(d["u_accept"]), P(d["u_draw"]), P(out), P(n), None)
    assert cuda_lib.tg_spec_verify(s.handle, *args) == _lib.TG_ERR_UNSUPPORTED
    assert b"tg_sampler_reserve" in cuda_lib.tg_last_error_string()
    assert cuda_lib.tg_sampler_reserve(s.handle, K, 0) == _lib.TG_OK
    assert cuda_lib.tg_spec_verify(s.handle, *args) == _lib.TG_OK
    torch.cuda.synchronize()


def test_hot_calls_allocate_nothing_after_reserve(sampler_factory):
    """cudaMemGetInfo is unchanged across reserved-size tg_sample (two-kernel
    mode) and tg_spec_verify calls."""
    import torch
    from tinygpt_b200.sampler import params_to_device
    w = W.make(4, seed=3, batch=2048)
    s = sampler_factory(w["vocab"])
    logits = torch.from_numpy(w["logits"]).view(torch.int16).view(torch.bfloat16).cuda()
    params = params_to_device(w["params"], "cuda:0")
    hist = torch.from_numpy(w["history"]).cuda()
    hlen = torch.from_numpy(w["history_len"]).cuda()
    u = torch.from_numpy(w["uniforms"]).cuda()
    out = torch.empty(2048, dtype=torch.int32, device="cuda:0")
    sp = W.make(5, seed=4, batch=16)
    tgt, drf = torch.from_numpy(sp["target"]).cuda(), torch.from_numpy(sp["draft"]).cuda()
    sv = sampler_factory(sp["vocab"])
    K = sp["draft_ids"].shape[1]
    sv.reserve(max_K=K)
    ids = torch.from_numpy(sp["draft_ids"]).cuda()
    T = torch.from_numpy(sp["temperature"]).cuda()
    ua, ud = torch.from_numpy(sp["u_accept"]).cuda(), torch.from_numpy(sp["u_draw"]).cuda()
    vo = torch.empty((16, K + 1), dtype=torch.int32, device="cuda:0")
    vn = torch.empty(16, dtype=torch.int32, device="cuda:0")

    def calls():
        s.sample(logits, params, history=hist, history_len=hlen, uniforms=u, out=out)
        sv.spec_verify(tgt, drf, ids, T, ua, ud, out=vo, out_n=vn)
        torch.cuda.synchronize()

    calls()  # first calls: lazily initialised CUDA state, kernel modules
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        calls()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_draft_free_greedy_verification(oracle_mod, sampler_factory, dtype):
    """Without draft logits every greedy row verifies exactly as with them (the
    greedy rule never reads the draft); a stochastic row ends without a token
    and sets device status bit 4."""
    import torch
    V, B = 5003, 12
    w = W.make(5, seed=31, batch=B, vocab=V)
    K = w["draft_ids"].shape[1]
    w["temperature"][:] = 0.0
    ids = w["draft_ids"].copy()
    am = np.argmax(w["target"], axis=2)  # proposals matching the target argmax for a while
    for b in range(B):
        m = b % (K + 1)
        ids[b, :m] = am[b, :m]
    w["draft_ids"] = ids
    if dtype == "bf16":
        w["target"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["target"]))
    cv = (lambda a: torch.from_numpy(W.to_bf16_bits(a)).view(torch.int16).view(torch.bfloat16)) \
        if dtype == "bf16" else torch.from_numpy
    s = sampler_factory(V)
    tgt = cv(w["target"]).cuda()
    T = torch.from_numpy(w["temperature"]).cuda()
    o, n = s.spec_verify(tgt, None, torch.from_numpy(ids).cuda(), T, None,
                         torch.from_numpy(w["u_draw"]).cuda())
    torch.cuda.synchronize()
    oo, on = oracle_mod.spec_verify(w["target"], w["draft"], ids, w["temperature"], w["u_accept"], w["u_draw"])
    assert np.array_equal(n.cpu().numpy(), on)
    assert np.array_equal(o.cpu().numpy(), oo)
    assert s.device_status() == 0
    T[3] = 0.8  # one stochastic row: no draft to test it against
    o, n = s.spec_verify(tgt, None, torch.from_numpy(ids).cuda(), T, None, torch.from_numpy(w["u_draw"]).cuda())
    torch.cuda.synchronize()
    assert int(n[3]) == 0 and (o[3] == -1).all()
    assert s.device_status() & 16
    keep = np.arange(B) != 3
    assert np.array_equal(n.cpu().numpy()[keep], on[keep])
