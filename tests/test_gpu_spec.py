"""Speculative verification on the GPU vs the oracle (bit-exact ids and counts)."""
import numpy as np
import pytest

from tinygpt_b200 import workloads as W

pytestmark = pytest.mark.gpu


def run(sampler, w, dtype="f32"):
    import torch
    cv = (lambda a: torch.from_numpy(W.to_bf16_bits(a)).view(torch.int16).view(torch.bfloat16)) \
        if dtype == "bf16" else torch.from_numpy
    tgt = cv(w["target"]).cuda()
    drf = cv(w["draft"]).cuda()
    o, n = sampler.spec_verify(tgt, drf, torch.from_numpy(w["draft_ids"]).cuda(),
                               torch.from_numpy(w["temperature"]).cuda(),
                               torch.from_numpy(w["u_accept"]).cuda(),
                               torch.from_numpy(w["u_draw"]).cuda())
    torch.cuda.synchronize()
    return o.cpu().numpy(), n.cpu().numpy()


@pytest.mark.parametrize("seed", [0, 1])
def test_spec_config5_full(oracle_mod, sampler_factory, seed):
    w = W.make(5, seed=seed)
    s = sampler_factory(w["vocab"])
    o, n = run(s, w)
    oo, on = oracle_mod.spec_verify(w["target"], w["draft"], w["draft_ids"], w["temperature"],
                                    w["u_accept"], w["u_draw"])
    assert np.array_equal(n, on)
    assert np.array_equal(o, oo)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_spec_mixed_modes(oracle_mod, sampler_factory, dtype):
    V, K, B = 5003, 4, 24
    w = W.make(5, seed=3, batch=B, vocab=V)
    w["target"] = w["target"][:, :K + 1].copy() if w["target"].shape[1] > K + 1 else w["target"]
    g = W.rng(4)
    K = w["draft"].shape[1]
    T = g.choice([0.0, -1.0, 1e-7, 0.3, 1.0, 2.0], size=B).astype(np.float32)
    w["temperature"] = T
    ids = w["draft_ids"].copy()
    ids[::5, 0] = np.argmax(w["target"][::5, 0], axis=1)  # greedy accepts
    ids[1, 1] = -3  # invalid proposal -> reject
    w["draft_ids"] = ids
    w["u_accept"][2] = 0.0
    w["u_accept"][3] = 1.0
    if dtype == "bf16":  # the oracle sees the same bf16 values
        w["target"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["target"]))
        w["draft"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["draft"]))
    s = sampler_factory(V)
    o, n = run(s, w, dtype)
    oo, on = oracle_mod.spec_verify(w["target"], w["draft"], w["draft_ids"], w["temperature"],
                                    w["u_accept"], w["u_draw"])
    assert np.array_equal(n, on)
    assert np.array_equal(o, oo)


@pytest.mark.parametrize("V,dtype", [(128256, "bf16"), (50257, "f32"), (50257, "bf16"), (32000, "bf16")])
def test_spec_vocab_shapes(oracle_mod, sampler_factory, V, dtype):
    """Config-5 rows at the configurations' vocabularies, f32 and bf16: whole and
    partial tiles of the draw pass, rows on and off 16-byte boundaries
    (V=50257 in f32 or bf16 leaves every row but the first unaligned)."""
    B = 32
    w = W.make(5, seed=11, batch=B, vocab=V)
    w["temperature"][::6] = 0.0  # some greedy rows
    if dtype == "bf16":  # the oracle sees the same bf16 values
        w["target"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["target"]))
        w["draft"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["draft"]))
    s = sampler_factory(V)
    o, n = run(s, w, dtype)
    oo, on = oracle_mod.spec_verify(w["target"], w["draft"], w["draft_ids"], w["temperature"],
                                    w["u_accept"], w["u_draw"])
    assert np.array_equal(n, on)
    assert np.array_equal(o, oo)
