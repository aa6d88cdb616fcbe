"""Shared helpers of the GPU parity tests: run one input set through the CUDA
path (C ABI via tinygpt_b200.sampler) and through the oracle."""
import numpy as np


def logits_to_dev(x, stride=None):
    import torch
    x = np.ascontiguousarray(x)
    B, V = x.shape
    if stride is not None and stride != V:
        pad = np.zeros((B, stride), x.dtype)
        pad[:, :V] = x
        x = pad
    t = torch.from_numpy(x)
    if x.dtype == np.uint16:
        t = t.view(torch.int16).view(torch.bfloat16)
    return t.to("cuda:0")


def gpu_sample(sampler, w, stride=None):
    import torch
    x = w["logits"]
    B, V = x.shape
    L = logits_to_dev(x, stride)
    params = torch.from_numpy(np.ascontiguousarray(w["params"]).view(np.int32).reshape(B, 8).copy()).cuda()
    hist = hl = mt = sid = None
    if w.get("history") is not None:
        hist = torch.from_numpy(w["history"]).cuda()
        hl = torch.from_numpy(w["history_len"]).cuda()
    if w.get("mask_table") is not None:
        mt = torch.from_numpy(w["mask_table"].view(np.int32)).cuda()
        sid = torch.from_numpy(w["state_id"]).cuda()
    u = torch.from_numpy(w["uniforms"]).cuda()
    probs = torch.empty(B, dtype=torch.float32, device="cuda:0")
    ids, _ = sampler.sample(L, params, history=hist, history_len=hl, mask_table=mt, state_id=sid,
                            uniforms=u, out_probs=probs)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), probs.cpu().numpy()


def oracle_sample(oracle, w):
    return oracle.sample(w["logits"], w["params"], w.get("history"), w.get("history_len"),
                         w.get("mask_table"), w.get("state_id"), w["uniforms"])


def assert_same(oracle, sampler, w, stride=None, what=""):
    gi, gp = gpu_sample(sampler, w, stride)
    oi, op = oracle_sample(oracle, w)
    bad = np.nonzero(gi != oi)[0]
    assert bad.size == 0, f"{what}: {bad.size} id mismatches, first rows {bad[:8]} gpu {gi[bad[:8]]} oracle {oi[bad[:8]]}"
    badp = np.nonzero(gp.view(np.uint32) != op.view(np.uint32))[0]
    assert badp.size == 0, f"{what}: prob mismatch rows {badp[:8]} gpu {gp[badp[:8]]} oracle {op[badp[:8]]}"
    return gi, gp
