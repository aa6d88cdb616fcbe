"""JSON-Schema constrained generation: host grammar compiler -> device mask table.

Mirrors the reference's constrained-generation API
(native-mac/Sources/TinyGPTModel/ConstrainedGen.swift:35-837, JSONSchema.swift:1-117):

    JSONSchemaFSM(schema)          -> Grammar(schema, vocab_tokens, eos_id).state()
    fsm.acceptBytes(b)             -> GrammarState.accept_bytes(b)
    fsm.isComplete                 -> GrammarState.is_complete
    LogitsMasker.computeMask(fsm)  -> GrammarState.mask()  (bitmask words)

and adds what the device sampler needs: `GrammarState.row()` gives the row of
the grammar's mask table for the state (computed once per distinct automaton
state), `Grammar.table()` the table to pass as tg_sample's mask_table, and
`MaskTableBatch` keeps a device copy in step with a batch of sequences.
All automaton work is native (libtgsample.so); nothing here runs on the GPU.
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from . import _lib


def _gcheck(rc: int) -> None:
    if rc != _lib.TG_OK:
        msg = _lib.load().tg_grammar_last_error().decode(errors="replace")
        raise _lib.TGError(rc, msg)


class Grammar:
    """A compiled grammar over a token vocabulary (list of bytes per token id).

    `spec` is a JSON Schema (dict or text) or the tool-tag GBNF text, chosen as
    ServeGrammarSpec.parse does (Serve.swift:1929-1941).
    """

    def __init__(self, spec, vocab_tokens, eos_id: int = -1):
        schema = spec
        L = _lib.load()
        text = schema if isinstance(schema, str) else json.dumps(schema)
        raw = text.encode()
        toks = [bytes(t) if not isinstance(t, str) else t.encode() for t in vocab_tokens]
        self.vocab = len(toks)
        self.eos_id = eos_id
        self.words = (self.vocab + 31) // 32
        offs = np.zeros(self.vocab + 1, np.int64)
        offs[1:] = np.cumsum([len(t) for t in toks])
        blob = np.frombuffer(b"".join(toks) or b"\0", np.uint8).copy()
        h = ctypes.c_void_p()
        _gcheck(L.tg_grammar_create(raw, len(raw), self.vocab, blob.ctypes.data,
                                    offs.ctypes.data, eos_id, ctypes.byref(h)))
        self._h = h
        self._L = L

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._L.tg_grammar_destroy(h)
            self._h = None

    @property
    def kind(self) -> int:
        v = ctypes.c_int32()
        _gcheck(self._L.tg_grammar_kind(self._h, ctypes.byref(v)))
        return v.value

    def state(self) -> "GrammarState":
        return GrammarState(self)

    def table(self) -> np.ndarray:
        """The mask table so far: [rows, ceil(vocab/32)] uint32 (a copy)."""
        p = ctypes.POINTER(ctypes.c_uint32)()
        n = ctypes.c_int32()
        _gcheck(self._L.tg_grammar_table(self._h, ctypes.byref(p), ctypes.byref(n)))
        if n.value == 0:
            return np.zeros((0, self.words), np.uint32)
        return np.ctypeslib.as_array(p, shape=(n.value * self.words,)).reshape(
            n.value, self.words).copy()


class GrammarState:
    """One sequence's automaton (the reference's JSONSchemaFSM instance)."""

    def __init__(self, g: Grammar, _handle=None):
        self.g = g
        h = _handle if _handle is not None else ctypes.c_void_p()
        if _handle is None:
            _gcheck(g._L.tg_grammar_state_create(g._h, ctypes.byref(h)))
        self._h = h

    def clone(self) -> "GrammarState":
        h = ctypes.c_void_p()
        _gcheck(self.g._L.tg_grammar_state_clone(self._h, ctypes.byref(h)))
        return GrammarState(self.g, h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self.g._L.tg_grammar_state_destroy(h)
            self._h = None

    def accept_bytes(self, data) -> bool:
        if isinstance(data, str):
            data = data.encode()
        ok = ctypes.c_int32()
        _gcheck(self.g._L.tg_grammar_accept_bytes(self._h, bytes(data), len(data), ctypes.byref(ok)))
        return bool(ok.value)

    def commit(self, token: int) -> bool:
        ok = ctypes.c_int32()
        _gcheck(self.g._L.tg_grammar_commit(self._h, int(token), ctypes.byref(ok)))
        return bool(ok.value)

    @property
    def is_complete(self) -> bool:
        v = ctypes.c_int32()
        _gcheck(self.g._L.tg_grammar_is_complete(self._h, ctypes.byref(v)))
        return bool(v.value)

    def mask(self) -> np.ndarray:
        out = np.zeros(self.g.words, np.uint32)
        _gcheck(self.g._L.tg_grammar_mask(self._h, out.ctypes.data))
        return out

    def allowed(self) -> np.ndarray:
        """Token ids the mask allows (ascending)."""
        bits = np.unpackbits(self.mask().view(np.uint8), bitorder="little")[: self.g.vocab]
        return np.flatnonzero(bits)

    def row(self) -> int:
        r = ctypes.c_int32()
        _gcheck(self.g._L.tg_grammar_state_row(self._h, ctypes.byref(r), None))
        return r.value


class MaskTableBatch:
    """Device mask table + per-row state ids for a batch of constrained sequences.

    `prepare()` returns (mask_table, num_states, state_id) for tg_sample; it
    uploads only the table rows added since the previous call (the table grows
    as new automaton states are met and is kept on the device with spare
    capacity).  `commit(ids)` advances every sequence by its sampled token.
    """

    def __init__(self, grammar: Grammar, batch: int, device="cuda", capacity: int = 256):
        import torch
        self.g = grammar
        self.states = [grammar.state() for _ in range(batch)]
        self.device = device
        self._torch = torch
        self._dev = torch.zeros((capacity, grammar.words), dtype=torch.int32, device=device)
        self._uploaded = 0
        self._sid = torch.zeros(batch, dtype=torch.int32, device=device)

    def prepare(self):
        torch = self._torch
        rows = np.array([s.row() for s in self.states], np.int32)
        tab = self.g.table()
        n = tab.shape[0]
        if n > self._dev.shape[0]:
            cap = max(n, 2 * self._dev.shape[0])
            new = torch.zeros((cap, self.g.words), dtype=torch.int32, device=self.device)
            new[: self._uploaded] = self._dev[: self._uploaded]
            self._dev = new
        if n > self._uploaded:
            self._dev[self._uploaded:n] = torch.from_numpy(tab[self._uploaded:n].view(np.int32)).to(self.device)
            self._uploaded = n
        self._sid.copy_(torch.from_numpy(rows))
        return self._dev, n, self._sid

    def commit(self, ids) -> list[bool]:
        ids = np.asarray(ids.cpu() if hasattr(ids, "cpu") else ids).reshape(-1)
        return [s.commit(int(t)) for s, t in zip(self.states, ids)]


def draft_state_rows(states, draft_ids) -> np.ndarray:
    """State rows [B, K+1] for tg_spec_verify_masked: entry i is the mask-table
    row of the grammar state before draft token i of the row (state after
    tokens 0..i-1, computed on a clone; the live states are not advanced).
    After a proposal the grammar rejects, the later positions keep the state
    before it (verification stops at that proposal anyway)."""
    draft_ids = np.asarray(draft_ids.cpu() if hasattr(draft_ids, "cpu") else draft_ids)
    B, K = draft_ids.shape
    rows = np.empty((B, K + 1), np.int32)
    for b, st in enumerate(states):
        c = st.clone()
        ok = True
        for i in range(K + 1):
            rows[b, i] = c.row()
            if i < K and ok:
                ok = c.commit(int(draft_ids[b, i]))
    return rows
