"""CPU oracle for the grammar compiler -- TEST INFRASTRUCTURE ONLY.

Only tests/ may import this module; the product path (libtgsample.so's
tg_grammar_* entry points) never calls it.

A plain restatement of the reference's constrained-decoding automata, kept in
the reference's own shape (a frame stack driven by per-frame actions; masks by
probing every token on a copy) so that it is independent of the native
implementation, which walks a vocabulary trie and caches rows by state:

  schema parse     native-mac/Sources/TinyGPTModel/JSONSchema.swift:71-116
  JSONSchemaFSM    native-mac/Sources/TinyGPTModel/ConstrainedGen.swift:160-749
  LogitsMasker     ConstrainedGen.swift:775-837
  PaceToolTagFSM   native-mac/Sources/TinyGPTServe/Serve.swift:2057-2233 (string
                   re-check of the whole output on every byte, as there)

Strings are handled as the reference handles them: content grows by one
Unicode scalar per byte (`String(UnicodeScalar(b))`, ConstrainedGen.swift:597),
i.e. Latin-1 decoding, and lengths count those characters.

Parity pins: tests/test_grammar.py holds the reference's own known-answer
tests (native-mac/Tests/TinyGPTModelTests/ConstrainedGenTests.swift) and checks
this oracle and the native library against them.
"""
from __future__ import annotations

import copy
import json
import re

# ----------------------------------------------------------------- schema
# node: ("any",) | ("object", [(name, node)], set(required)) |
#       ("string", enum|None, min|None, max|None) | ("number", integer) |
#       ("boolean",) | ("null",) | ("array", node)


def _as_int(v):
    # `as? Int` on a JSONSerialization number: integral values only (bools excluded here)
    if isinstance(v, bool):
        return None
    if isinstance(v, int):
        return v
    if isinstance(v, float) and v == int(v):
        return int(v)
    return None


def parse_schema(d):
    """JSONSchema.swift:71-116."""
    if not isinstance(d, dict):
        return ("any",)
    en = d.get("enum")
    if isinstance(en, list):
        strings = [x for x in en if isinstance(x, str)]
        if strings:
            return ("string", strings, _as_int(d.get("minLength")), _as_int(d.get("maxLength")))
    t = d.get("type")
    if not isinstance(t, str):
        return ("any",)
    if t == "object":
        props = d.get("properties")
        props = props if isinstance(props, dict) else {}
        req = d.get("required")
        req = set(req) if isinstance(req, list) and all(isinstance(x, str) for x in req) else set()
        return ("object", [(k, parse_schema(props[k])) for k in sorted(props)], req)
    if t == "string":
        return ("string", None, _as_int(d.get("minLength")), _as_int(d.get("maxLength")))
    if t in ("number", "integer"):
        return ("number", t == "integer")
    if t == "boolean":
        return ("boolean",)
    if t == "null":
        return ("null",)
    if t == "array":
        return ("array", parse_schema(d.get("items")))
    return ("any",)


ANY = ("any",)
EMPTY_OBJECT = ("object", [], set())

# ----------------------------------------------------------------- automaton
# frames are dicts; actions are tuples as in ConstrainedGen.swift:120-158


class JSONSchemaFSM:
    def __init__(self, root):
        self.stack = [{"k": "value", "schema": root, "done": False}]
        self.last_key = None

    def clone(self):
        c = JSONSchemaFSM(ANY)
        c.stack = copy.deepcopy(self.stack)
        c.last_key = self.last_key
        return c

    @property
    def is_complete(self):
        return len(self.stack) == 1 and self.stack[0]["k"] == "value" and self.stack[0]["done"]

    def accept_bytes(self, bs):
        snap, key = copy.deepcopy(self.stack), self.last_key
        for b in bs:
            if not self._drive(b, 0):
                self.stack, self.last_key = snap, key
                return False
        return True

    # ConstrainedGen.swift:214-276
    def _drive(self, b, depth):
        if depth > 64 or not self.stack:
            return False
        top = self.stack[-1]
        act = self._transition(top, b)
        kind = act[0]
        if kind == "reject":
            return False
        if kind == "replace":
            self.stack[-1] = act[1]
            return True
        if kind == "push":
            self.stack.append(act[1])
            return True
        if kind == "replace_push":
            self.stack[-1] = act[1]
            self.stack.append(act[2])
            return True
        if kind == "push_retry":
            self.stack.append(act[1])
            ok = self._drive(b, depth + 1)
            if not ok:
                self.stack.pop()
            return ok
        if kind == "pop":
            if top["k"] == "string" and top["is_key"]:
                self.last_key = top["content"]
            self.stack.pop()
            self._advance()
            return True
        if kind == "pop_retry":
            self.stack.pop()
            self._advance()
            return self._drive(b, depth + 1)
        raise AssertionError(kind)

    # ConstrainedGen.swift:294-352
    def _advance(self):
        while self.stack:
            p = self.stack[-1]
            if p["k"] == "object":
                if p["phase"] in ("afterOpen", "afterComma"):
                    key = self.last_key if self.last_key is not None else ""
                    self.last_key = None
                    p["phase"] = ("afterKey", key)
                elif isinstance(p["phase"], tuple) and p["phase"][0] == "insideValue":
                    p["emitted"].add(p["phase"][1])
                    p["phase"] = "afterValue"
                return
            if p["k"] == "array":
                p["phase"] = "afterItem"
                return
            if p["k"] == "value":
                if len(self.stack) == 1:
                    p["done"] = True
                    return
                self.stack.pop()
                continue
            return

    def _transition(self, top, b):
        k = top["k"]
        if k == "value":
            return ("reject",) if top["done"] else self._open(top["schema"], b)
        if k == "object":
            return self._object(top, b)
        if k == "array":
            return self._array(top, b)
        if k == "string":
            return self._string(top, b)
        if k == "number":
            return self._number(top, b)
        if k == "literal":
            lit, pos = top["lit"], top["pos"]
            if pos >= len(lit) or ord(lit[pos]) != b:
                return ("reject",)
            if pos + 1 == len(lit):
                return ("pop",)
            return ("replace", dict(top, pos=pos + 1))
        raise AssertionError(k)

    @staticmethod
    def _str(enum, mn, mx, is_key=False):
        return {"k": "string", "state": "body", "enum": enum, "min": mn, "max": mx,
                "content": "", "is_key": is_key}

    @staticmethod
    def _num(b, integer):
        st = "sign" if b == ord("-") else ("intZero" if b == ord("0") else "intDigits")
        return {"k": "number", "state": st, "integer": integer}

    # ConstrainedGen.swift:372-459
    def _open(self, s, b):
        c = chr(b)
        if s[0] == "any":
            if c == "{":
                return ("push", {"k": "object", "schema": EMPTY_OBJECT, "emitted": set(), "phase": "afterOpen"})
            if c == "[":
                return ("push", {"k": "array", "items": ANY, "phase": "afterOpen"})
            if c == '"':
                return ("push", self._str(None, None, None))
            if c == "-" or c.isdigit() and b < 128:
                return ("push", self._num(b, False))
            if c in "tfn":
                return ("push", {"k": "literal", "lit": {"t": "true", "f": "false", "n": "null"}[c], "pos": 1})
            return ("reject",)
        if s[0] == "object":
            return ("push", {"k": "object", "schema": s, "emitted": set(), "phase": "afterOpen"}) if c == "{" else ("reject",)
        if s[0] == "array":
            return ("push", {"k": "array", "items": s[1], "phase": "afterOpen"}) if c == "[" else ("reject",)
        if s[0] == "string":
            return ("push", self._str(s[1], s[2], s[3])) if c == '"' else ("reject",)
        if s[0] == "number":
            if c == "-" or (48 <= b <= 57):
                return ("push", self._num(b, s[1]))
            return ("reject",)
        if s[0] == "boolean":
            if c == "t":
                return ("push", {"k": "literal", "lit": "true", "pos": 1})
            if c == "f":
                return ("push", {"k": "literal", "lit": "false", "pos": 1})
            return ("reject",)
        if s[0] == "null":
            return ("push", {"k": "literal", "lit": "null", "pos": 1}) if c == "n" else ("reject",)
        raise AssertionError(s)

    @staticmethod
    def _unemitted(schema, emitted):
        if schema[0] == "object":
            if not schema[1]:
                return None
            return [k for k, _ in schema[1] if k not in emitted]
        return None

    @staticmethod
    def _schema_for(key, schema):
        if schema[0] == "object":
            for k, v in schema[1]:
                if k == key:
                    return v
        return ANY

    # ConstrainedGen.swift:463-527
    def _object(self, of, b):
        c, ph = chr(b), of["phase"]
        schema = of["schema"]
        if ph in ("afterOpen", "afterComma"):
            if c == "}" and ph == "afterOpen":
                return ("pop",) if schema[2] <= of["emitted"] else ("reject",)
            if c == '"':
                keys = self._unemitted(schema, of["emitted"])
                if keys is not None and not keys:
                    return ("reject",)
                return ("push", self._str(keys, None, None, is_key=True))
            return ("reject",)
        if isinstance(ph, tuple) and ph[0] == "afterKey":
            if c == ":":
                nf = dict(of, phase=("insideValue", ph[1]))
                return ("replace_push", nf, {"k": "value", "schema": self._schema_for(ph[1], schema), "done": False})
            return ("reject",)
        if ph == "afterValue":
            if c == ",":
                rem = self._unemitted(schema, of["emitted"])
                if rem is not None and not rem:
                    return ("reject",)
                return ("replace", dict(of, phase="afterComma"))
            if c == "}":
                return ("pop",) if schema[2] <= of["emitted"] else ("reject",)
        return ("reject",)

    # ConstrainedGen.swift:543-573
    def _array(self, af, b):
        c, ph = chr(b), af["phase"]
        if ph == "afterOpen":
            if c == "]":
                return ("pop",)
            return ("push_retry", {"k": "value", "schema": af["items"], "done": False})
        if ph == "afterComma":
            return ("push_retry", {"k": "value", "schema": af["items"], "done": False})
        if ph == "afterItem":
            if c == ",":
                return ("replace", dict(af, phase="afterComma"))
            if c == "]":
                return ("pop",)
        return ("reject",)

    # ConstrainedGen.swift:577-643
    def _string(self, sf, b):
        c, st = chr(b), sf["state"]  # chr(b): the byte as a Unicode scalar
        if st == "body":
            if c == '"':
                if sf["enum"] is not None and sf["content"] not in sf["enum"]:
                    return ("reject",)
                if sf["min"] is not None and len(sf["content"]) < sf["min"]:
                    return ("reject",)
                return ("pop",)
            if c == "\\":
                if sf["enum"] is not None:
                    return ("reject",)
                return ("replace", dict(sf, state="escape"))
            if b < 0x20:
                return ("reject",)
            new = sf["content"] + c
            if sf["max"] is not None and len(new) > sf["max"]:
                return ("reject",)
            if sf["enum"] is not None and not any(e.startswith(new) for e in sf["enum"]):
                return ("reject",)
            return ("replace", dict(sf, content=new))
        if st == "escape":
            if c in '"\\/bfnrt':
                new = sf["content"] + "\\" + c
                if sf["max"] is not None and len(new) > sf["max"]:
                    return ("reject",)
                return ("replace", dict(sf, state="body", content=new))
            if c == "u":
                new = sf["content"] + "\\u"
                if sf["max"] is not None and len(new) > sf["max"]:
                    return ("reject",)
                return ("replace", dict(sf, state=("u", 0), content=new))
            return ("reject",)
        if isinstance(st, tuple):
            if c in "0123456789abcdefABCDEF":
                new = sf["content"] + c
                if sf["max"] is not None and len(new) > sf["max"]:
                    return ("reject",)
                n = st[1] + 1
                return ("replace", dict(sf, content=new, state="body" if n == 4 else ("u", n)))
            return ("reject",)
        return ("reject",)

    # ConstrainedGen.swift:646-705
    def _number(self, nf, b):
        c, st = chr(b), nf["state"]
        if c in ",}] \t\n\r":
            return ("pop_retry",) if st in ("intZero", "intDigits", "frac", "expDigits") else ("reject",)
        dig = "0" <= c <= "9"
        nxt = None
        if st == "sign":
            nxt = ("intZero" if c == "0" else "intDigits") if dig else None
        elif st == "intZero":
            nxt = None if dig else ("afterPoint" if c == "." and not nf["integer"] else
                                   "afterExp" if c in "eE" and not nf["integer"] else None)
        elif st == "intDigits":
            nxt = "intDigits" if dig else ("afterPoint" if c == "." and not nf["integer"] else
                                           "afterExp" if c in "eE" and not nf["integer"] else None)
        elif st == "afterPoint":
            nxt = "frac" if dig else None
        elif st == "frac":
            nxt = "frac" if dig else ("afterExp" if c in "eE" else None)
        elif st == "afterExp":
            nxt = "expSign" if c in "+-" else ("expDigits" if dig else None)
        elif st == "expSign":
            nxt = "expDigits" if dig else None
        elif st == "expDigits":
            nxt = "expDigits" if dig else None
        return ("replace", dict(nf, state=nxt)) if nxt else ("reject",)


def compile_schema(text: str) -> JSONSchemaFSM:
    return JSONSchemaFSM(parse_schema(json.loads(text)))


# ----------------------------------------------------------------- tool tags
# Serve.swift:2057-2233: the whole output is re-checked on every byte.

def _text_scalar(ch):
    v = ord(ch)
    if v in (0x0A, 0x0D, 0x09) or ch in "[]":
        return False
    return 0x20 <= v <= 0x7E


def _digit(ch):
    return "0" <= ch <= "9"


def _alpha(ch):
    return "A" <= ch <= "Z" or "a" <= ch <= "z"


def _key(ch):
    return _alpha(ch) or ch == "+"


def _app(ch):
    return _alpha(ch) or _digit(ch) or ch == " "


def _label(ch):
    return _alpha(ch) or _digit(ch) or ch in " _-"


def _type(ch):
    return _alpha(ch) or _digit(ch) or ch in " _-.,!?'\""


def _body_prefix(s, mn, mx, first, rest):
    count = 0
    for idx, ch in enumerate(s):
        if ch == "]":
            return idx == len(s) - 1 and count >= mn
        if not (first(ch) if count == 0 else rest(ch)):
            return False
        count += 1
        if count > mx:
            return False
    return True


def _consume_digits(s, i, mx):
    count = 0
    while i < len(s) and _digit(s[i]):
        count += 1
        if count > mx:
            return count, i
        i += 1
    return count, i


def _coords_label_prefix(s):
    x, i = _consume_digits(s, 0, 4)
    if i == len(s):
        return x <= 4
    if not (x >= 1 and s[i] == ","):
        return False
    i += 1
    y, i = _consume_digits(s, i, 4)
    if i == len(s):
        return y <= 4
    if not (y >= 1 and s[i] == ":"):
        return False
    i += 1
    return _body_prefix(s[i:], 1, 41, _alpha, _label)


def _scroll_prefix(s):
    for d in ("up", "down", "left", "right"):
        if d.startswith(s):
            return True
        if s.startswith(d + ":"):
            return _body_prefix(s[len(d) + 1:], 1, 4, _digit, _digit)
    return False


def _tag_prefix(tag):
    if "[POINT:none]".startswith(tag):
        return True
    for head, fn in (("[POINT:", _coords_label_prefix), ("[CLICK:", _coords_label_prefix),
                     ("[TYPE:", lambda s: _body_prefix(s, 1, 200, _type, _type)),
                     ("[SCROLL:", _scroll_prefix),
                     ("[KEY:", lambda s: _body_prefix(s, 1, 30, _key, _key)),
                     ("[OPEN_APP:", lambda s: _body_prefix(s, 1, 31, _alpha, _app))):
        if tag.startswith(head):
            return fn(tag[len(head):])
        if head.startswith(tag):
            return True
    return False


_COMPLETE = re.compile(
    r"^\[(POINT:none|POINT:[0-9]{1,4},[0-9]{1,4}:[A-Za-z][A-Za-z0-9 _-]{0,40}|"
    r"CLICK:[0-9]{1,4},[0-9]{1,4}:[A-Za-z][A-Za-z0-9 _-]{0,40}|TYPE:[A-Za-z0-9 _.,!?'\"-]{1,200}|"
    r"SCROLL:(up|down|left|right):[0-9]{1,4}|KEY:[A-Za-z+]{1,30}|"
    r"OPEN_APP:[A-Za-z][A-Za-z0-9 ]{0,30})\]\Z")


def _viable(bs: bytes) -> bool:
    try:
        text = bs.decode("utf-8")
    except UnicodeDecodeError:
        return False
    i = text.find("[")
    if i < 0:
        return all(_text_scalar(ch) for ch in text)
    if not all(_text_scalar(ch) for ch in text[:i]):
        return False
    return _tag_prefix(text[i:])


class PaceToolTagFSM:
    def __init__(self):
        self.bytes = b""

    def clone(self):
        c = PaceToolTagFSM()
        c.bytes = self.bytes
        return c

    @property
    def is_complete(self):
        try:
            text = self.bytes.decode("utf-8")
        except UnicodeDecodeError:
            return False
        i = text.find("[")
        return i >= 0 and _COMPLETE.match(text[i:]) is not None

    def accept_bytes(self, bs):
        cand = self.bytes
        for b in bs:
            cand += bytes([b])
            if not _viable(cand):
                return False
        self.bytes = cand
        return True


# ----------------------------------------------------------------- masker

def mask_ids(fsm, tokens, eos_id=None):
    """LogitsMasker.mask (ConstrainedGen.swift:805-822) as a list of allowed ids."""
    if fsm.is_complete:
        return [eos_id] if eos_id is not None and 0 <= eos_id < len(tokens) else []
    out = []
    for i, t in enumerate(tokens):
        if t and fsm.clone().accept_bytes(t):
            out.append(i)
    return out
