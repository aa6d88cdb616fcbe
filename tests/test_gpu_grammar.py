"""Constrained generation end to end on the GPU: grammar automaton (host) ->
mask table rows (device) -> tg_sample -> commit, checked against the oracle
sampler on the same table every step, and every sampled token against the
automaton (the mask guarantees acceptance, LogitsMasker.commit's contract,
ConstrainedGen.swift:824-830)."""
from __future__ import annotations

import json
import random

import numpy as np
import pytest

from tests.gpu_helpers import oracle_sample

pytestmark = pytest.mark.gpu


def _vocab(V, seed):
    rng = random.Random(seed)
    toks = {bytes([i]) for i in range(1, 256)}
    frags = ['{"', '":', '",', '"}', "},", "[{", "]}", '":"', "true", "false", "null",
             "name", "age", "kind", "alpha", "beta", "tags", "x", "12", "3.5", "-1", "e+"]
    toks.update(f.encode() for f in frags)
    alpha = "abcdefghijklmnopqrstuvwxyz"
    while len(toks) < V - 1:
        r = rng.random()
        if r < 0.6:
            t = (" " if rng.random() < 0.5 else "") + "".join(rng.choice(alpha) for _ in range(rng.randint(2, 8)))
        else:
            t = "".join(rng.choice('{}[]",:0123456789-.e ' + alpha) for _ in range(rng.randint(1, 4)))
        toks.add(t.encode())
    vocab = sorted(toks)[: V - 1]
    vocab.append(b"\x00<eos>")  # EOS: never accepted by the automaton itself
    return vocab


SCHEMA = {"type": "object", "properties": {
    "name": {"type": "string", "maxLength": 12},
    "age": {"type": "integer"},
    "kind": {"enum": ["alpha", "beta"]},
    "tags": {"type": "array", "items": {"type": "string", "maxLength": 5}}},
    "required": ["name", "kind"]}

TAGS = 'root ::= response\nresponse ::= sentence " " tag\ntag ::= "[POINT:" coords "]"\n'


@pytest.mark.parametrize("spec", [json.dumps(SCHEMA), TAGS])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_constrained_generation_matches_oracle(oracle_mod, sampler_factory, spec, dtype):
    import torch
    from tinygpt_b200 import workloads as W
    from tinygpt_b200.grammar import Grammar, MaskTableBatch
    from tinygpt_b200.sampler import row_params

    V, B, steps = 8192, 12, 40
    vocab = _vocab(V, 3)
    eos = V - 1
    g = Grammar(spec, vocab, eos_id=eos)
    batch = MaskTableBatch(g, B, device="cuda:0", capacity=4)  # small capacity: exercises growth
    s = sampler_factory(V)
    rng = np.random.default_rng(17)
    params = row_params(B, temperature=np.where(np.arange(B) % 3 == 0, 0.0, 0.9),
                        top_k=np.where(np.arange(B) % 4 == 1, 40, 0),
                        top_p=np.where(np.arange(B) % 4 == 2, 0.9, 1.0))
    pdev = torch.from_numpy(params.view(np.int32).reshape(B, 8).copy()).cuda()
    dead = np.zeros(B, bool)
    for step in range(steps):
        table, n_states, sid = batch.prepare()
        x = rng.standard_normal((B, V)).astype(np.float32) * 3
        if dtype == "bf16":
            x = W.to_bf16_bits(x)
        w = {"logits": x, "params": params, "uniforms": rng.random(B, dtype=np.float32),
             "mask_table": g.table(), "state_id": sid.cpu().numpy()}
        assert w["mask_table"].shape[0] == n_states
        L = torch.from_numpy(x)
        if dtype == "bf16":
            L = L.view(torch.int16).view(torch.bfloat16)
        ids, _ = s.sample(L.cuda(), pdev, mask_table=table[:n_states], state_id=sid,
                          uniforms=torch.from_numpy(w["uniforms"]).cuda())
        torch.cuda.synchronize()
        gi = ids.cpu().numpy()
        oi, _ = oracle_sample(oracle_mod, w)
        assert np.array_equal(gi, oi), (step, gi, oi)
        for r in range(B):
            st = batch.states[r]
            if st.is_complete:
                assert gi[r] == eos
                continue
            if gi[r] < 0:
                # a dead end of the reference automaton (e.g. '\\' taken at maxLength: every
                # escape then overflows); its mask is empty and it stays so
                assert st.allowed().size == 0
                dead[r] = True
                continue
            assert not dead[r] and gi[r] != eos
            assert st.commit(int(gi[r])), (r, vocab[gi[r]])
    assert s.device_status() == 0
