"""Grammar-masked speculative verification (tg_spec_verify_masked) on the GPU
vs the oracle: bit-exact ids and counts; all -1 states equal tg_spec_verify;
with a compiled grammar every emitted token is accepted by the automaton."""
import json

import numpy as np
import pytest

from tinygpt_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _dev(a, dtype):
    import torch
    if dtype == "bf16":
        return torch.from_numpy(W.to_bf16_bits(a)).view(torch.int16).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _run(s, w, table, sids, dtype):
    import torch
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    o, n = s.spec_verify_masked(_dev(w["target"], dtype), _dev(w["draft"], dtype), t(w["draft_ids"]),
                                t(w["temperature"]), t(w["u_accept"]), t(w["u_draw"]),
                                t(table.view(np.int32)), t(sids))
    torch.cuda.synchronize()
    return o.cpu().numpy(), n.cpu().numpy()


def _case(V, B, seed, dtype):
    w = W.make(5, seed=seed, batch=B, vocab=V)
    K = w["draft"].shape[1]
    g = W.rng(100 + seed)
    S = 8
    bits = g.random((S, ((V + 31) // 32) * 32)) < g.uniform(0.02, 0.3, size=S)[:, None]
    bits[:, V:] = False
    bits[5] = False                      # a dead state: nothing allowed
    bits[6] = False
    bits[6, g.integers(V)] = True        # exactly one token
    bits[7, :V] = True                   # everything allowed
    table = W.pack_mask(bits)
    sids = g.integers(-1, S, size=(B, K + 1)).astype(np.int32)
    ids = w["draft_ids"].copy()
    for b in range(B):                   # half the proposals drawn from the allowed set
        for i in range(K):
            if g.random() < 0.5 and sids[b, i] >= 0:
                allowed = np.flatnonzero(bits[sids[b, i], :V])
                if allowed.size:
                    ids[b, i] = g.choice(allowed)
    w["draft_ids"] = ids
    w["temperature"] = g.choice([0.0, 0.5, 1.0, 1.5], size=B).astype(np.float32)
    w["u_accept"][0] = 0.0
    if dtype == "bf16":
        w["target"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["target"]))
        w["draft"] = W.bf16_bits_to_f32(W.to_bf16_bits(w["draft"]))
    return w, table, sids


@pytest.mark.parametrize("V,dtype", [(5003, "f32"), (5003, "bf16"), (128256, "f32")])
def test_masked_matches_oracle(oracle_mod, sampler_factory, V, dtype):
    B = 24 if V < 10000 else 8
    w, table, sids = _case(V, B, 7, dtype)
    s = sampler_factory(V)
    s.device_status()
    o, n = _run(s, w, table, sids, dtype)
    oo, on = oracle_mod.spec_verify_masked(w["target"], w["draft"], w["draft_ids"], w["temperature"],
                                           w["u_accept"], w["u_draw"], table, sids)
    assert np.array_equal(n, on)
    assert np.array_equal(o, oo)
    assert s.device_status() == 0
    # every emitted id is allowed at its position
    for b in range(B):
        for i in range(n[b]):
            if o[b, i] < 0:  # greedy row at a state that allows nothing
                assert w["temperature"][b] <= 0 and sids[b, i] == 5
                continue
            if sids[b, i] >= 0:
                assert (table[sids[b, i], o[b, i] >> 5] >> (o[b, i] & 31)) & 1


def test_unmasked_states_equal_plain_verify(oracle_mod, sampler_factory):
    import torch
    V = 5003
    w, table, _ = _case(V, 16, 9, "f32")
    sids = np.full((16, w["draft"].shape[1] + 1), -1, np.int32)
    s = sampler_factory(V)
    o, n = _run(s, w, table, sids, "f32")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    po, pn = s.spec_verify(t(w["target"]), t(w["draft"]), t(w["draft_ids"]), t(w["temperature"]),
                           t(w["u_accept"]), t(w["u_draw"]))
    torch.cuda.synchronize()
    assert np.array_equal(n, pn.cpu().numpy())
    assert np.array_equal(o, po.cpu().numpy())


def test_out_of_range_state_sets_status(oracle_mod, sampler_factory):
    V = 5003
    w, table, sids = _case(V, 4, 11, "f32")
    sids[1, 0] = table.shape[0] + 3
    s = sampler_factory(V)
    s.device_status()
    o, n = _run(s, w, table, sids, "f32")
    assert s.device_status() & 1
    sids2 = sids.copy()
    sids2[1, 0] = -1  # the documented behaviour: that position unmasked
    oo, on = oracle_mod.spec_verify_masked(w["target"], w["draft"], w["draft_ids"], w["temperature"],
                                           w["u_accept"], w["u_draw"], table, sids2)
    assert np.array_equal(n, on) and np.array_equal(o, oo)


def test_grammar_driven_verification(oracle_mod, sampler_factory):
    """Drafts verified under a compiled JSON schema: the emitted tokens always
    advance the automaton."""
    from tinygpt_b200.grammar import Grammar, draft_state_rows
    V, B, K = 4096, 6, 4
    vocab = [bytes([i]) for i in range(1, 256)]
    frags = [b'{"', b'":', b'",', b'"}', b"name", b"age", b"12", b"3", b'":"', b"ab"]
    vocab += frags
    rng = np.random.default_rng(3)
    while len(vocab) < V:
        vocab.append(bytes(rng.integers(97, 123, size=rng.integers(2, 6)).tolist()))
    schema = {"type": "object", "properties": {"name": {"type": "string"}, "age": {"type": "integer"}},
              "required": ["name", "age"]}
    g = Grammar(json.dumps(schema), vocab)
    states = [g.state() for _ in range(B)]
    for st in states[3:]:
        assert st.accept_bytes(b'{"name":"')
    w = W.make(5, seed=2, batch=B, vocab=V)
    w["target"] = w["target"][:, :K + 1].copy()
    w["draft"] = w["draft"][:, :K].copy()
    ids = np.empty((B, K), np.int32)
    for b in range(B):  # proposals: allowed tokens mostly, a disallowed one sometimes
        c = states[b].clone()
        for i in range(K):
            al = c.allowed()
            tok = int(rng.choice(al)) if (al.size and rng.random() < 0.8) else int(rng.integers(V))
            ids[b, i] = tok
            c.commit(tok)
    w["draft_ids"] = ids
    w["u_accept"] = w["u_accept"][:, :K].copy()
    w["temperature"] = np.array([0.0, 0.7, 1.0, 0.0, 0.7, 1.2], np.float32)
    rows = draft_state_rows(states, ids)
    table = g.table()
    o, n = _run(sampler_factory(V), w, table, rows, "f32")
    oo, on = oracle_mod.spec_verify_masked(w["target"], w["draft"], ids, w["temperature"],
                                           w["u_accept"], w["u_draw"], table, rows)
    assert np.array_equal(n, on) and np.array_equal(o, oo)
    for b in range(B):
        c = states[b].clone()
        for i in range(n[b]):
            assert c.commit(int(o[b, i])), (b, i, o[b, i])
