"""Vocab-sharded mode on one GPU: the shards of every row are processed by
separate handles (as separate ranks would), their records stacked as an
all-gather would, and the merge must equal the oracle on whole rows, ids and
probabilities bit for bit."""
import numpy as np
import pytest
import torch

from tinygpt_b200 import workloads as W
from tests.gpu_helpers import logits_to_dev, oracle_sample

pytestmark = pytest.mark.gpu


def run_sharded(sampler_factory, w, cuts):
    V = w["logits"].shape[1]
    B = w["logits"].shape[0]
    params = np.ascontiguousarray(w["params"])
    recs = []
    kw = {}
    if w.get("history") is not None:
        kw.update(history=torch.from_numpy(w["history"]).cuda(), history_len=torch.from_numpy(w["history_len"]).cuda())
    if w.get("mask_table") is not None:
        kw.update(mask_table=torch.from_numpy(w["mask_table"].view(np.int32)).cuda(),
                  state_id=torch.from_numpy(w["state_id"]).cuda())
    bounds = [0] + list(cuts) + [V]
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        s = sampler_factory(hi - lo)
        L = logits_to_dev(np.ascontiguousarray(w["logits"][:, lo:hi]))
        recs.append(s.sample_shard_local(L, params, lo, V, **kw))
    gathered = torch.stack(recs)
    m = sampler_factory(V)
    probs = torch.empty(B, dtype=torch.float32, device="cuda:0")
    ids, _ = m.sample_shard_merge(gathered, V, params, uniforms=torch.from_numpy(w["uniforms"]).cuda(),
                                  out_probs=probs)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), probs.cpu().numpy(), m


@pytest.mark.parametrize("cuts", [[64128], [40001, 90000], [1000, 64128, 100003], [8 * 16032 * i // 8 for i in range(1, 8)]])
def test_sharded_config4_equals_whole_rows(oracle_mod, sampler_factory, cuts):
    w = W.make(4, seed=7, batch=96)
    gi, gp, _ = run_sharded(sampler_factory, w, cuts)
    oi, op = oracle_sample(oracle_mod, w)
    assert np.array_equal(gi, oi)
    assert np.array_equal(gp.view(np.uint32), op.view(np.uint32))


def test_sharded_greedy_masks_and_unsupported_rows(oracle_mod, sampler_factory):
    w = W.make(3, seed=2, batch=40)  # fp32, grammar masks, half greedy / half k=50
    w["params"]["top_k"][5] = 0       # no top-k, not greedy: unsupported in sharded mode
    w["params"]["temperature"][5] = 1.0
    gi, gp, m = run_sharded(sampler_factory, w, [33333, 77777])
    oi, op = oracle_sample(oracle_mod, w)
    ok = np.arange(40) != 5
    assert np.array_equal(gi[ok], oi[ok])
    assert np.array_equal(gp[ok].view(np.uint32), op[ok].view(np.uint32))
    assert gi[5] == -1 and m.device_status() & 4


def test_sample_sharded_one_rank_communicator(oracle_mod, sampler_factory):
    """tg_sample_sharded on a one-rank NCCL communicator (local records, all-gather,
    merge in one call) equals the oracle on whole rows."""
    import torch
    from tinygpt_b200.dist import NcclComm
    from tests.gpu_helpers import logits_to_dev, oracle_sample
    w = W.make(4, seed=13, batch=48)
    V = w["vocab"]
    s = sampler_factory(V)
    comm = NcclComm(0, 1, 0)
    try:
        ids, _ = s.sample_sharded(comm.ptr, 1, logits_to_dev(w["logits"]), w["params"], 0, V,
                                  uniforms=torch.from_numpy(w["uniforms"]).cuda(),
                                  history=torch.from_numpy(w["history"]).cuda(),
                                  history_len=torch.from_numpy(w["history_len"]).cuda())
        torch.cuda.synchronize()
    finally:
        comm.close()
    want, _ = oracle_sample(oracle_mod, w)
    assert np.array_equal(ids.cpu().numpy(), want)
