"""Grammar compiler (tg_grammar_*): known-answer tests and differential checks.

CPU only.  Three layers:
  1. The reference's own known-answer tests, restated
     (native-mac/Tests/TinyGPTModelTests/ConstrainedGenTests.swift:12-270), run
     against the native library AND the Python oracle (pins both).
  2. Native vs oracle on generated documents, their prefixes and single-byte
     mutations (accept / complete) and on token masks over a multi-byte
     vocabulary (the native trie walk vs the oracle's per-token probe).
  3. Mask-table rows: every state's row equals its directly computed mask
     (checks that states sharing a row have equal futures).
"""
from __future__ import annotations

import json
import os
import random
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(__file__), ".."))

from oracle import grammar_oracle as go  # noqa: E402
from tinygpt_b200 import _lib  # noqa: E402
from tinygpt_b200.grammar import Grammar  # noqa: E402

BYTE_VOCAB = [bytes([i]) for i in range(256)]


def native(schema, vocab=BYTE_VOCAB, eos=-1):
    return Grammar(schema, vocab, eos_id=eos)


def both(schema):
    """(native state, oracle fsm) at the document start."""
    text = schema if isinstance(schema, str) else json.dumps(schema)
    return native(text).state(), go.compile_schema(text)


def check_both(schema, steps):
    """steps: list of (bytes, expected_accept); checks accept and completion on both."""
    n, o = both(schema)
    for data, want in steps:
        data = data.encode() if isinstance(data, str) else data
        assert n.accept_bytes(data) == want, (schema, data)
        assert o.accept_bytes(data) == want, (schema, data)
    return n, o


# ------------------------------------------------------------------ 1. reference KATs

def test_parse_object_required_properties():  # ConstrainedGenTests.swift:12-31
    node = go.parse_schema(json.loads(
        '{"type":"object","required":["name"],"properties":{"name":{"type":"string"}}}'))
    assert node[0] == "object" and [k for k, _ in node[1]] == ["name"] and "name" in node[2]


def test_parse_enum_string():  # ConstrainedGenTests.swift:33-44
    assert go.parse_schema({"type": "string", "enum": ["a", "b", "c"]})[:2] == ("string", ["a", "b", "c"])


SIMPLE = {"type": "object", "properties": {"name": {"type": "string"}, "age": {"type": "integer"}},
          "required": ["name", "age"]}
X_INT = {"type": "object", "properties": {"x": {"type": "integer"}}, "required": ["x"]}


def test_accepts_simple_object():  # :48-67
    n, o = check_both(SIMPLE, [('{"name":"Alice","age":42}', True)])
    assert n.is_complete and o.is_complete


def test_rejects_inter_token_whitespace():  # :69-78
    check_both(X_INT, [('  {"x":1}', False)])


def test_string_allows_whitespace_in_content():  # :80-85
    n, o = check_both({"type": "string"}, [('"hello world"', True)])
    assert n.is_complete and o.is_complete


def test_rejects_invalid_json():  # :87-96
    n, o = check_both(X_INT, [("garbage", False)])
    assert not n.is_complete and not o.is_complete


def test_rejects_undeclared_key():  # :98-111
    check_both({"type": "object", "properties": {"x": {"type": "integer"}}, "required": []},
               [('{"', True), ("y", False)])


def test_enum_restricts_content():  # :113-122
    n, o = check_both({"type": "string", "enum": ["foo", "bar"]}, [('"foo"', True)])
    assert n.is_complete and o.is_complete


def test_enum_rejects_non_member():  # :124-136
    n, o = check_both({"type": "string", "enum": ["foo", "bar"]},
                      [('"', True), ("f", True), ("x", False), ('oo"', True)])
    assert n.is_complete and o.is_complete


def test_accepts_array():  # :138-147
    n, o = check_both({"type": "array", "items": {"type": "integer"}}, [("[1,2,3]", True)])
    assert n.is_complete and o.is_complete


NESTED = {"type": "object", "properties": {
    "tool_name": {"type": "string", "enum": ["read_file", "run_test"]},
    "arguments": {"type": "object", "properties": {"path": {"type": "string"}}}},
    "required": ["tool_name", "arguments"]}


def test_accepts_nested_object():  # :149-168
    n, o = check_both(NESTED, [('{"tool_name":"read_file","arguments":{"path":"/etc/passwd"}}', True)])
    assert n.is_complete and o.is_complete


@pytest.mark.parametrize("schema,text", [({"type": "boolean"}, "true"), ({"type": "boolean"}, "false"),
                                         ({"type": "null"}, "null")])
def test_accepts_booleans_and_null(schema, text):  # :170-180
    n, o = check_both(schema, [(text, True)])
    assert n.is_complete and o.is_complete


AB = {"type": "object", "properties": {"a": {"type": "integer"}, "b": {"type": "integer"}}, "required": []}


def test_rejects_trailing_comma_object():  # :182-192
    check_both(AB, [('{"a":1', True), (",", True), ("}", False)])


def test_rejects_trailing_comma_array():  # :194-203
    check_both({"type": "array", "items": {"type": "integer"}}, [("[1,2", True), (",", True), ("]", False)])


def test_requires_all_required_keys():  # :205-224
    schema = dict(AB, required=["a", "b"])
    n, o = check_both(schema, [('{"a":1', True), ("}", False), (',"b":2}', True)])
    assert n.is_complete and o.is_complete


def test_masker_only_open_brace_at_start():  # :228-245
    g = native({"type": "object", "properties": {}, "required": []})
    assert list(g.state().allowed()) == [ord("{")]
    assert go.mask_ids(go.compile_schema('{"type":"object","properties":{},"required":[]}'), BYTE_VOCAB) == [ord("{")]


def test_masker_complete_masks_all():  # :247-259
    s = native({"type": "boolean"}).state()
    assert s.accept_bytes("true") and s.is_complete
    assert s.allowed().size == 0


def test_masker_eos_allowed_when_complete():  # :261-270
    s = native({"type": "boolean"}, eos=42).state()
    assert s.accept_bytes("true")
    assert list(s.allowed()) == [42]


# ------------------------------------------------------------------ grammar selection

def test_grammar_kind_and_unsupported():
    assert native(json.dumps(SIMPLE)).kind == _lib.TG_GRAMMAR_JSON_SCHEMA
    assert native("  \n" + json.dumps(SIMPLE) + "\n").kind == _lib.TG_GRAMMAR_JSON_SCHEMA
    gbnf = 'root ::= response\ntag ::= "[POINT:" coords "]"\n'
    assert native(gbnf).kind == _lib.TG_GRAMMAR_TOOL_TAGS
    with pytest.raises(_lib.TGError) as e:
        native("root ::= foo")
    assert e.value.code == _lib.TG_ERR_UNSUPPORTED
    with pytest.raises(_lib.TGError) as e:
        native('{"type": ')
    assert e.value.code == _lib.TG_ERR_INVALID_ARG


# ------------------------------------------------------------------ edge semantics (pinned to the oracle)

EDGE_CASES = [
    ({"type": "string", "maxLength": 3}, ['"abc"', '"abcd"', '"a\\n"', '"a\\nb"', '"\\u0041"']),
    ({"type": "string", "minLength": 2}, ['""', '"a"', '"ab"', '"\\n"']),
    ({"type": "string", "maxLength": -1}, ['""', '"a"']),
    ({"type": "integer"}, ["0", "-", "-0", "01", "12", "1.5", "1e3", "12,"]),
    ({"type": "array", "items": {"type": "number"}}, ["[0.5,-1e-3,2E+7]", "[1.]", "[01]", "[-]", "[1 ]", "[]"]),
    ({"type": "array", "items": {}}, ['[{"a":[1,"x"]},null,true]', '[{"a":1,}]', "[[],[[]]]"]),
    ({"type": "object", "properties": {}, "required": ["k"]}, ['{}', '{"k":1}', '{"j":1,"k":2}', '{"k":1,"k":2}']),
    ({"type": "object", "required": ["a"], "properties": {"a": {"type": "null"}}},
     ['{"a":null}', '{}', '{"a":nul}', '{"a":null,"a":null}']),
    ({"enum": ["x", "xy", "café", "中"]},
     ['"x"', '"xy"', '"xz"', '"café"', '"cafÃ©"', '"中"', '"\\u0078"']),
    ({"type": "object", "properties": {"été": {"type": "boolean"}}}, ['{"été":true}']),
    ({"type": "string"}, ['"\x01"', '"tab\there"', '"\\x"', '"\\uZZZZ"', '"\\u00e9"']),
    ({"type": "object", "properties": {"a": {"type": "integer"}}, "required": [1]}, ['{}', '{"a":1}']),
    ({"type": "number"}, ["3", "3 ", "-0.0e-0"]),
    ({"type": "strange"}, ['"s"', "1", "{}", "tru", "[1,[2]]"]),
]


@pytest.mark.parametrize("schema,docs", EDGE_CASES)
def test_edge_cases_match_oracle(schema, docs):
    text = json.dumps(schema)
    g = native(text)
    for d in docs:
        raw = d.encode("latin-1") if all(ord(c) < 256 for c in d) else d.encode()
        for variant in (raw, d.encode()):
            n, o = g.state(), go.compile_schema(text)
            a_n, a_o = n.accept_bytes(variant), o.accept_bytes(variant)
            assert a_n == a_o, (schema, variant)
            assert n.is_complete == o.is_complete, (schema, variant)
            # byte by byte (the reference's acceptByte path restores nothing, acceptBytes does)
            n, o = g.state(), go.compile_schema(text)
            for b in variant:
                assert n.accept_bytes(bytes([b])) == o.accept_bytes(bytes([b])), (schema, variant, b)
            assert n.is_complete == o.is_complete


# ------------------------------------------------------------------ 2. random documents

SCHEMAS = [
    SIMPLE, NESTED, AB,
    {"type": "object", "properties": {
        "id": {"type": "integer"},
        "tags": {"type": "array", "items": {"type": "string", "maxLength": 6}},
        "kind": {"enum": ["alpha", "alps", "beta"]},
        "score": {"type": "number"},
        "ok": {"type": "boolean"},
        "note": {"type": "null"},
        "meta": {}},
     "required": ["id", "kind"]},
    {"type": "array", "items": {"type": "object", "properties": {
        "k": {"type": "string", "minLength": 1, "maxLength": 4}}, "required": ["k"]}},
    {"type": "object", "properties": {}},
]


def gen_value(node, rng, depth=0):
    k = node[0]
    if k == "any":
        choice = rng.choice(["obj", "arr", "str", "num", "lit"] if depth < 3 else ["str", "num", "lit"])
        if choice == "obj":
            return gen_value(go.EMPTY_OBJECT, rng, depth + 1)
        if choice == "arr":
            return gen_value(("array", go.ANY), rng, depth + 1)
        return gen_value({"str": ("string", None, None, None), "num": ("number", False),
                          "lit": ("boolean",)}[choice], rng, depth + 1)
    if k == "object":
        props, req = node[1], node[2]
        if props:
            names = [n for n, _ in props]
            chosen = [n for n in names if n in req or rng.random() < 0.6]
            rng.shuffle(chosen)
            items = [(n, dict(props)[n]) for n in chosen]
        else:
            items = [(n, go.ANY) for n in sorted(req)] + \
                [("k%d" % i, go.ANY) for i in range(rng.randint(0, 2))]
        return "{" + ",".join(json.dumps(n) + ":" + gen_value(v, rng, depth + 1) for n, v in items) + "}"
    if k == "array":
        return "[" + ",".join(gen_value(node[1], rng, depth + 1) for _ in range(rng.randint(0, 3))) + "]"
    if k == "string":
        if node[1] is not None:
            return json.dumps(rng.choice(node[1]))
        lo = node[2] or 0
        hi = node[3] if node[3] is not None else lo + 8
        n = rng.randint(lo, max(lo, hi))
        return '"' + "".join(rng.choice("abc xyz_-.") for _ in range(n)) + '"'
    if k == "number":
        if node[1]:
            return str(rng.randint(-500, 500))
        return rng.choice([str(rng.randint(-9, 99)), "%.3f" % rng.uniform(-5, 5), "1e%d" % rng.randint(-3, 3)])
    if k == "boolean":
        return rng.choice(["true", "false"])
    if k == "null":
        return "null"
    raise AssertionError(k)


@pytest.mark.parametrize("si", range(len(SCHEMAS)))
def test_random_documents_and_mutations(si):
    rng = random.Random(1000 + si)
    text = json.dumps(SCHEMAS[si])
    g = native(text)
    node = go.parse_schema(SCHEMAS[si])
    alphabet = b'{}[]",:0123456789-.eE+ abxyz\\ntfu'
    for _ in range(25):
        doc = gen_value(node, rng).encode()
        n, o = g.state(), go.compile_schema(text)
        assert n.accept_bytes(doc) and o.accept_bytes(doc), doc
        assert n.is_complete == o.is_complete
        for _ in range(6):
            cut = rng.randint(0, len(doc))
            mut = bytearray(doc[:cut])
            if rng.random() < 0.7 or not mut:
                mut.append(rng.choice(alphabet))
            else:
                mut[rng.randrange(len(mut))] = rng.choice(alphabet)
            n, o = g.state(), go.compile_schema(text)
            assert n.accept_bytes(bytes(mut)) == o.accept_bytes(bytes(mut)), (doc, bytes(mut))
            assert n.is_complete == o.is_complete, bytes(mut)


def synthetic_vocab(rng, n=600):
    """Single bytes plus multi-byte pieces that straddle JSON structure."""
    pieces = set(BYTE_VOCAB)
    frags = ['{"', '":', '",', '"}', "},", "[{", "]}", '":"', "true", "false", "null", "tr", "ue",
             "name", "age", "Alice", "tool_name", "read_file", "run_", "arguments", "path", "/etc",
             "alpha", "al", "alps", "beta", "id", "tags", "kind", "score", "ok", "note", "meta",
             '":[', '"]', "12", "3.", "e-", "-1", " ", "  ", "\\n", "\\u00", "k", '"k"', ':"']
    pieces.update(f.encode() for f in frags)
    while len(pieces) < n:
        m = rng.randint(2, 5)
        pieces.add(bytes(rng.choice(b'{}[]",:0123456789-.eabnrstu lkpm_') for _ in range(m)))
    vocab = sorted(pieces)
    vocab.insert(7, b"")  # an empty token: never allowed
    return vocab


@pytest.mark.parametrize("si", [0, 1, 3, 4, 5])
def test_masks_match_oracle_probe(si):
    rng = random.Random(77 + si)
    vocab = synthetic_vocab(rng)
    text = json.dumps(SCHEMAS[si])
    g = Grammar(text, vocab, eos_id=3)
    node = go.parse_schema(SCHEMAS[si])
    for _ in range(4):
        doc = gen_value(node, rng).encode()
        for cut in sorted(set([0, len(doc)] + [rng.randint(0, len(doc)) for _ in range(5)])):
            n, o = g.state(), go.compile_schema(text)
            assert n.accept_bytes(doc[:cut]) and o.accept_bytes(doc[:cut])
            assert list(n.allowed()) == go.mask_ids(o, vocab, eos_id=3), (doc[:cut])


# ------------------------------------------------------------------ 3. mask-table rows

def test_rows_share_only_equal_masks():
    rng = random.Random(5)
    vocab = synthetic_vocab(rng, 400)
    for schema in SCHEMAS:
        g = Grammar(json.dumps(schema), vocab)
        node = go.parse_schema(schema)
        seen = {}
        for _ in range(6):
            doc = gen_value(node, rng).encode()
            s = g.state()
            for b in doc:
                r = s.row()
                m = s.mask()
                if r in seen:
                    assert np.array_equal(seen[r], m)
                seen[r] = m
                assert s.accept_bytes(bytes([b]))
        tab = g.table()
        assert tab.shape == (len(seen), (len(vocab) + 31) // 32)
        for r, m in seen.items():
            assert np.array_equal(tab[r], m)


def test_rows_bounded_for_free_strings():
    """An unconstrained string's content does not create new rows."""
    g = native({"type": "object", "properties": {"t": {"type": "string"}}, "required": ["t"]})
    s = g.state()
    assert s.accept_bytes('{"t":"')
    rows = set()
    for ch in "the quick brown fox jumps over the lazy dog" * 3:
        assert s.accept_bytes(ch)
        rows.add(s.row())
    assert len(rows) == 1


def test_commit_and_clone():
    vocab = [b'{"', b"name", b'":"', b"Al", b"ice", b'",', b'"age', b'":', b"42", b"}", b"x"]
    g = Grammar(SIMPLE, vocab, eos_id=10)
    s = g.state()
    for t in [0, 1, 2, 3]:
        assert s.commit(t)
    c = s.clone()
    assert s.commit(9)  # '}' inside a string value is content; the clone must not see it
    for t in [4, 5, 6, 7, 8, 9]:
        assert c.commit(t), t
    assert c.is_complete and list(c.allowed()) == [10]
    assert not c.commit(-1) and not c.commit(len(vocab))


# ------------------------------------------------------------------ tool tags

TAG_GRAMMAR = 'root ::= response\nresponse ::= sentence " " tag\ntag ::= point-tag\npoint-tag ::= "[POINT:" ( coords ":" label | "none" ) "]"\n'

TAG_DOCS = ["Look here [POINT:12,340:Save button]", "ok [POINT:none]", "Click it [CLICK:1,2:A]",
            "typing [TYPE:Hello, world! it's \"fine\"]", "scroll [SCROLL:down:120]", "[KEY:cmd+s]",
            "open [OPEN_APP:Safari 2]", "bad [POINT:12345,1:x]", "bad [POINT:1,2:]", "bad [TYPE:]",
            "x [SCROLL:sideways:1]", "[KEY:" + "a" * 31 + "]", "[POINT:none] trailing", "café [KEY:a]",
            "two [KEY:a][KEY:b]", "[OPEN_APP:1abc]", "[POINT:1,2:a" + "b" * 40 + "]", "[POINT:1,2:a" + "b" * 41 + "]",
            "line\nbreak", "[CLICK:0000,9999:Z_-z]", "[SCROLL:up:]", "[SCROLL:up:12345]", "[POINT:nonE]"]


@pytest.mark.parametrize("doc", TAG_DOCS)
def test_tool_tags_match_oracle(doc):
    g = native(TAG_GRAMMAR)
    raw = doc.encode()
    for cut in range(len(raw) + 1):
        n, o = g.state(), go.PaceToolTagFSM()
        assert n.accept_bytes(raw[:cut]) == o.accept_bytes(raw[:cut]), raw[:cut]
        assert n.is_complete == o.is_complete, raw[:cut]


def test_tool_tags_fuzz_and_masks():
    rng = random.Random(11)
    g_bytes = native(TAG_GRAMMAR)
    alphabet = b"[]:,0123456789POINTCLICKTYPESCROLLKEYOPEN_APPnoneupdownleftright aZz+-_.!?'\"\n\xc3"
    heads = [b"[POINT:", b"[POINT:none]", b"[CLICK:", b"[TYPE:", b"[SCROLL:", b"[KEY:", b"[OPEN_APP:"]
    for _ in range(400):
        s = bytearray(b"hi " if rng.random() < 0.5 else b"")
        s += rng.choice(heads) if rng.random() < 0.8 else b""
        for _ in range(rng.randint(0, 12)):
            s.append(rng.choice(alphabet))
        n, o = g_bytes.state(), go.PaceToolTagFSM()
        for b in bytes(s):
            a_n, a_o = n.accept_bytes(bytes([b])), o.accept_bytes(bytes([b]))
            assert a_n == a_o, bytes(s)
            assert n.is_complete == o.is_complete, bytes(s)
            if not a_n:
                break
    vocab = sorted(set(BYTE_VOCAB) | {h for h in heads} | {b"none]", b"up:", b"12", b",3", b"ab]", b"Safari"})
    g = Grammar(TAG_GRAMMAR, vocab)
    for prefix in [b"", b"Hi ", b"Hi [", b"Hi [POINT:", b"Hi [POINT:1", b"[SCROLL:up", b"[TYPE:x", b"[KEY:a]"]:
        n, o = g.state(), go.PaceToolTagFSM()
        assert n.accept_bytes(prefix) and o.accept_bytes(prefix)
        assert list(n.allowed()) == go.mask_ids(o, vocab), prefix


def test_draft_state_rows():
    """State rows for masked verification: row i is the state after drafts 0..i-1;
    after a rejected draft the state stays; the live states are not advanced."""
    from tinygpt_b200.grammar import draft_state_rows
    vocab = [b'{"', b"name", b'":"', b"Al", b'"', b"x", b"}"]
    g = Grammar(SIMPLE, vocab)
    s0, s1 = g.state(), g.state()
    drafts = np.array([[0, 1, 2, 3], [0, 6, 1, 2]], np.int32)  # row 1: '}' is rejected at i=1
    rows = draft_state_rows([s0, s1], drafts)
    ref = g.state()
    expect0 = []
    for t in [None, 0, 1, 2, 3]:
        if t is not None:
            assert ref.commit(t)
        expect0.append(ref.row())
    assert list(rows[0]) == expect0
    assert rows[1, 0] == expect0[0] and rows[1, 1] == expect0[1]
    assert list(rows[1, 2:]) == [rows[1, 1]] * 3
    assert s0.row() == expect0[0] and s1.row() == expect0[0]


# ------------------------------------------------------------------ the reference's own grammars
# tests/golden/grammars/ holds the grammars the reference serves (its grammars/
# directory: the pace-fm-* JSON Schemas and pace-tool-tags.gbnf), as fixtures.

REF_GRAMMARS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "grammars")
REF_SCHEMAS = sorted(f for f in os.listdir(REF_GRAMMARS) if f.endswith(".schema.json"))


def schema_vocab(rng, schema: dict, n=700):
    """synthetic_vocab plus the schema's own key names, enum members and their
    quoted forms, so multi-byte tokens cross the structure of its documents."""
    pieces = set(synthetic_vocab(rng, n))

    def walk(node):
        if isinstance(node, dict):
            for k, v in node.get("properties", {}).items():
                pieces.update({k.encode(), ('"' + k + '"').encode(), ('"' + k + '":').encode()})
                walk(v)
            for e in node.get("enum", []):
                if isinstance(e, str):
                    pieces.update({e.encode(), ('"' + e + '"').encode(), e[:3].encode()})
            if "items" in node:
                walk(node["items"])
    walk(schema)
    pieces.discard(b"")
    vocab = sorted(pieces)
    vocab.insert(5, b"")
    return vocab


@pytest.mark.parametrize("name", REF_SCHEMAS)
def test_reference_schemas_documents_and_masks(name):
    text = open(os.path.join(REF_GRAMMARS, name)).read()
    schema = json.loads(text)
    node = go.parse_schema(schema)
    rng = random.Random(sum(name.encode()))
    g = native(text)
    for _ in range(12):  # documents: acceptance and completion agree byte for byte
        doc = gen_value(node, rng).encode()
        n, o = g.state(), go.compile_schema(text)
        assert n.accept_bytes(doc) and o.accept_bytes(doc), doc
        assert n.is_complete and o.is_complete
        cut = rng.randint(0, len(doc))
        mut = doc[:cut] + bytes([rng.choice(b'{}[]",:0123456789ax ')])
        n, o = g.state(), go.compile_schema(text)
        assert n.accept_bytes(mut) == o.accept_bytes(mut), mut
    vocab = schema_vocab(rng, schema)
    gv = Grammar(text, vocab, eos_id=3)
    for _ in range(3):  # masks over a multi-byte vocabulary along valid documents
        doc = gen_value(node, rng).encode()
        for cut in sorted({0, len(doc)} | {rng.randint(0, len(doc)) for _ in range(4)}):
            n, o = gv.state(), go.compile_schema(text)
            assert n.accept_bytes(doc[:cut]) and o.accept_bytes(doc[:cut])
            assert list(n.allowed()) == go.mask_ids(o, vocab, eos_id=3), (name, doc[:cut])


def test_reference_tool_tag_grammar():
    text = open(os.path.join(REF_GRAMMARS, "pace-tool-tags.gbnf")).read()
    g = native(text)
    assert g.kind == 1  # the tool-tag grammar
    for doc in TAG_DOCS:
        raw = doc.encode()
        n, o = g.state(), go.PaceToolTagFSM()
        assert n.accept_bytes(raw) == o.accept_bytes(raw), raw
        assert n.is_complete == o.is_complete, raw
    heads = [b"[POINT:", b"[POINT:none]", b"[CLICK:", b"[TYPE:", b"[SCROLL:", b"[KEY:", b"[OPEN_APP:"]
    vocab = sorted(set(BYTE_VOCAB) | set(heads) | {b"none]", b"up:", b"12", b",3", b"ab]", b"Safari", b"Look ",
                                                     b"here ", b"the ", b"button"})
    gv = Grammar(text, vocab)
    for prefix in [b"", b"Look here ", b"Look here [", b"Look here [CLICK:12,3", b"ok [SCROLL:up:1",
                   b"typing [TYPE:Hi", b"go [OPEN_APP:Saf"]:
        n, o = gv.state(), go.PaceToolTagFSM()
        assert n.accept_bytes(prefix) == o.accept_bytes(prefix), prefix
        assert list(n.allowed()) == go.mask_ids(o, vocab), prefix
