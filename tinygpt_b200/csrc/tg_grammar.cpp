// tg_grammar.cpp -- host-side grammar compiler: JSON Schema -> byte-level
// pushdown automaton -> per-state token bitmasks for the device mask table.
//
// Reference behaviour restated (sarthak-fleet/tinygpt):
//   schema subset      native-mac/Sources/TinyGPTModel/JSONSchema.swift:1-117
//                      (enum of strings first; object properties sorted by key;
//                      required; string min/maxLength; number / integer;
//                      boolean; null; array items; anything else = any)
//   automaton          native-mac/Sources/TinyGPTModel/ConstrainedGen.swift:35-749
//                      (minified JSON only -- no whitespace between tokens;
//                      object keys restricted to the declared, not yet emitted
//                      properties; no trailing commas; required keys before
//                      '}'; numbers end on , } ] or whitespace and a bare
//                      top-level number never completes; escapes count as
//                      their source characters in string lengths)
//   masker             ConstrainedGen.swift:775-837 (a token is allowed iff all
//                      its bytes are accepted from the current state; empty
//                      tokens never; a complete automaton allows only EOS)
// Lengths are counted in bytes (the reference counts characters of a
// byte-per-character view; identical for ASCII).
//
// The mask of a state is computed by a depth-first walk of a byte trie of the
// vocabulary, carrying the automaton state down the trie: tokens sharing a
// prefix share the work and a rejected byte prunes its whole subtree.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/tgsample.h"

namespace tgg {

// ---------------------------------------------------------------- JSON values
struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  bool is_int = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* e;
  std::string err;
  void ws() { while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++; }
  bool fail(const char* m) { if (err.empty()) err = m; return false; }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if (static_cast<size_t>(e - p) < n || memcmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  static void utf8(std::string& o, uint32_t c) {
    if (c < 0x80) o += static_cast<char>(c);
    else if (c < 0x800) { o += static_cast<char>(0xC0 | (c >> 6)); o += static_cast<char>(0x80 | (c & 63)); }
    else if (c < 0x10000) { o += static_cast<char>(0xE0 | (c >> 12)); o += static_cast<char>(0x80 | ((c >> 6) & 63)); o += static_cast<char>(0x80 | (c & 63)); }
    else { o += static_cast<char>(0xF0 | (c >> 18)); o += static_cast<char>(0x80 | ((c >> 12) & 63)); o += static_cast<char>(0x80 | ((c >> 6) & 63)); o += static_cast<char>(0x80 | (c & 63)); }
  }
  bool hex4(uint32_t& v) {
    if (e - p < 4) return false;
    v = 0;
    for (int i = 0; i < 4; i++) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else return false;
    }
    return true;
  }
  bool string(std::string& o) {
    if (p >= e || *p != '"') return fail("expected string");
    p++;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        p++;
        if (p >= e) return fail("bad escape");
        const char c = *p++;
        switch (c) {
          case '"': o += '"'; break;
          case '\\': o += '\\'; break;
          case '/': o += '/'; break;
          case 'b': o += '\b'; break;
          case 'f': o += '\f'; break;
          case 'n': o += '\n'; break;
          case 'r': o += '\r'; break;
          case 't': o += '\t'; break;
          case 'u': {
            uint32_t v;
            if (!hex4(v)) return fail("bad \\u escape");
            if (v >= 0xD800 && v < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
              p += 2;
              uint32_t w;
              if (!hex4(w)) return fail("bad \\u escape");
              v = 0x10000 + ((v - 0xD800) << 10) + (w - 0xDC00);
            }
            utf8(o, v);
            break;
          }
          default: return fail("bad escape");
        }
      } else {
        o += *p++;
      }
    }
    if (p >= e) return fail("unterminated string");
    p++;
    return true;
  }
  bool value(JVal& v, int depth = 0) {
    if (depth > 256) return fail("nesting too deep");
    ws();
    if (p >= e) return fail("unexpected end");
    if (*p == '{') {
      p++;
      v.kind = JVal::Obj;
      ws();
      if (p < e && *p == '}') { p++; return true; }
      for (;;) {
        ws();
        std::string k;
        if (!string(k)) return false;
        ws();
        if (p >= e || *p != ':') return fail("expected ':'");
        p++;
        JVal x;
        if (!value(x, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (p < e && *p == ',') { p++; continue; }
        if (p < e && *p == '}') { p++; return true; }
        return fail("expected ',' or '}'");
      }
    }
    if (*p == '[') {
      p++;
      v.kind = JVal::Arr;
      ws();
      if (p < e && *p == ']') { p++; return true; }
      for (;;) {
        JVal x;
        if (!value(x, depth + 1)) return false;
        v.arr.push_back(std::move(x));
        ws();
        if (p < e && *p == ',') { p++; continue; }
        if (p < e && *p == ']') { p++; return true; }
        return fail("expected ',' or ']'");
      }
    }
    if (*p == '"') { v.kind = JVal::Str; return string(v.str); }
    if (lit("true")) { v.kind = JVal::Bool; v.b = true; return true; }
    if (lit("false")) { v.kind = JVal::Bool; v.b = false; return true; }
    if (lit("null")) { v.kind = JVal::Null; return true; }
    const char* s = p;
    if (p < e && *p == '-') p++;
    bool frac = false;
    while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-')) {
      if (*p == '.' || *p == 'e' || *p == 'E') frac = true;
      p++;
    }
    if (p == s) return fail("unexpected character");
    v.kind = JVal::Num;
    v.num = strtod(std::string(s, p).c_str(), nullptr);
    v.is_int = !frac;
    return true;
  }
};

// ---------------------------------------------------------------- schema
// A schema string (enum value, property name, required name) as the byte
// string the automaton can produce for it.  The automaton builds string
// content one byte at a time, each byte read as the Unicode scalar of the same
// value (ConstrainedGen.swift:597, `String(UnicodeScalar(b))`), so a schema
// character <= U+00FF corresponds to the single byte of that value and a
// character above U+00FF can never be produced: the string is reachable only
// up to it (`full` false).  Canonical-equivalence cases (decomposed accents)
// are not modelled.
struct Lit {
  std::string b;
  bool full = true;
};

static Lit latin1(const std::string& u) {
  Lit r;
  size_t i = 0;
  while (i < u.size()) {
    const uint8_t c = static_cast<uint8_t>(u[i]);
    uint32_t cp;
    size_t n;
    if (c < 0x80) { cp = c; n = 1; }
    else if ((c & 0xE0) == 0xC0 && i + 1 < u.size()) { cp = ((c & 0x1F) << 6) | (u[i + 1] & 0x3F); n = 2; }
    else { r.full = false; return r; }  // three- and four-byte sequences are above U+00FF
    if (cp > 0xFF) { r.full = false; return r; }
    r.b.push_back(static_cast<char>(cp));
    i += n;
  }
  return r;
}

struct Node {
  enum Kind { Any, Object, String, Number, Boolean, Null, Array } kind = Any;
  std::vector<std::pair<Lit, std::unique_ptr<Node>>> props;  // sorted by name
  std::vector<Lit> required;
  bool has_enum = false;
  std::vector<Lit> enum_values;
  bool has_min = false, has_max = false;
  int64_t min_len = 0, max_len = 0;
  bool integer = false;
  std::unique_ptr<Node> items;
};

// `dict[k] as? Int` on a JSONSerialization number: integral values only.
static bool json_int(const JVal* v, int64_t* out) {
  if (!v || v->kind != JVal::Num) return false;
  if (!(v->num == static_cast<double>(static_cast<int64_t>(v->num)))) return false;
  if (v->num > 9.2e18 || v->num < -9.2e18) return false;
  *out = static_cast<int64_t>(v->num);
  return true;
}

static void lengths(const JVal& v, Node* n) {
  n->has_min = json_int(v.get("minLength"), &n->min_len);
  n->has_max = json_int(v.get("maxLength"), &n->max_len);
}

// JSONSchema.swift:71-116.
static std::unique_ptr<Node> parse_schema(const JVal& v) {
  auto n = std::make_unique<Node>();
  if (v.kind != JVal::Obj) return n;  // any
  if (const JVal* en = v.get("enum")) {
    if (en->kind == JVal::Arr) {
      for (auto& x : en->arr)
        if (x.kind == JVal::Str) n->enum_values.push_back(latin1(x.str));
      if (!n->enum_values.empty()) {
        n->kind = Node::String;
        n->has_enum = true;
        lengths(v, n.get());
        return n;
      }
    }
  }
  const JVal* ty = v.get("type");
  if (!ty || ty->kind != JVal::Str) return n;
  const std::string& t = ty->str;
  if (t == "object") {
    n->kind = Node::Object;
    const JVal* ps = v.get("properties");
    if (ps && ps->kind == JVal::Obj) {
      // keys sorted by code point (UTF-8 byte order); a repeated key keeps its last value
      std::map<std::string, const JVal*> byname;
      for (auto& kv : ps->obj) byname[kv.first] = &kv.second;
      for (auto& kv : byname) n->props.emplace_back(latin1(kv.first), parse_schema(*kv.second));
    }
    const JVal* rq = v.get("required");
    if (rq && rq->kind == JVal::Arr) {
      bool all_str = true;
      for (auto& x : rq->arr) all_str = all_str && x.kind == JVal::Str;
      if (all_str)  // `as? [String]` fails as a whole on any other element
        for (auto& x : rq->arr) n->required.push_back(latin1(x.str));
    }
  } else if (t == "string") {
    n->kind = Node::String;
    lengths(v, n.get());
  } else if (t == "number" || t == "integer") {
    n->kind = Node::Number;
    n->integer = t == "integer";
  } else if (t == "boolean") {
    n->kind = Node::Boolean;
  } else if (t == "null") {
    n->kind = Node::Null;
  } else if (t == "array") {
    const JVal* it = v.get("items");
    n->kind = Node::Array;
    n->items = it ? parse_schema(*it) : std::make_unique<Node>();
  }
  return n;
}

// ---------------------------------------------------------------- automaton
// Frames (ConstrainedGen.swift:35-158).  A value slot opens its concrete
// frame on top of itself; when the concrete frame pops, nested slots pop too
// and the root slot stays, marked done (ConstrainedGen.swift:318-352).
enum : uint8_t { kValue, kObject, kArray, kString, kNumber, kLiteral };
enum : uint8_t { OAfterOpen, OAfterComma, OAfterKey, OInsideValue, OAfterValue };
enum : uint8_t { AAfterOpen, AAfterComma, AAfterItem };
enum : uint8_t { SBody, SEscape, SUnicode };
enum : uint8_t { NSign, NIntZero, NIntDigits, NAfterPoint, NFrac, NAfterExp, NExpSign, NExpDigits };

struct Frame {
  uint8_t kind = kValue;
  uint8_t phase = 0;     // value: 0 start / 1 done; otherwise the frame's phase
  uint8_t aux = 0;       // string: \u digits seen; literal: bytes matched
  bool is_key = false;   // string frame of an object key
  bool integer = false;  // number frame
  const Node* node = nullptr;  // value slot / object / array items / string schema
  const char* lit = nullptr;   // "true", "false" or "null"
  std::string text;            // string: content so far; object: the current key
  std::vector<std::string> emitted;  // object: keys whose values completed (a set)
};

struct Anyish {
  Node any_node;
  Node empty_object;
  Anyish() { empty_object.kind = Node::Object; }
};
static const Anyish& anyish() {
  static Anyish a;
  return a;
}

static bool is_digit(uint8_t b) { return b >= '0' && b <= '9'; }
static bool is_hex(uint8_t b) { return is_digit(b) || (b >= 'a' && b <= 'f') || (b >= 'A' && b <= 'F'); }
static bool has(const std::vector<std::string>& set, const std::string& k) {
  return std::find(set.begin(), set.end(), k) != set.end();
}
static bool lit_eq(const Lit& l, const std::string& s) { return l.full && l.b == s; }
static bool lit_prefix(const Lit& l, const std::string& p) {
  return p.size() <= l.b.size() && l.b.compare(0, p.size(), p) == 0;
}

struct Machine {
  std::vector<Frame> st;
  std::string last_key;
  bool has_last_key = false;

  bool complete() const { return st.size() == 1 && st[0].kind == kValue && st[0].phase == 1; }

  // Declared property names not yet emitted (ConstrainedGen.swift:531-541);
  // an object without declared properties takes any key (no list).
  static bool key_list(const Frame& of, std::vector<const Lit*>* out) {
    const Node* n = of.node;
    if (n->props.empty()) return false;
    out->clear();
    for (auto& p : n->props)
      if (!(p.first.full && has(of.emitted, p.first.b))) out->push_back(&p.first);
    return true;
  }
  static bool keys_exhausted(const Frame& of) {
    std::vector<const Lit*> ks;
    return key_list(of, &ks) && ks.empty();
  }
  static bool required_done(const Frame& of) {
    for (auto& r : of.node->required)
      if (!(r.full && has(of.emitted, r.b))) return false;
    return true;
  }
  static const Node* prop_schema(const Node* n, const std::string& key) {
    for (auto& p : n->props)
      if (lit_eq(p.first, key)) return p.second.get();
    return &anyish().any_node;
  }

  // After the top frame popped: advance the parent, cascading through value
  // slots (ConstrainedGen.swift:294-352).
  void after_pop() {
    while (!st.empty()) {
      Frame& p = st.back();
      if (p.kind == kObject) {
        if (p.phase == OAfterOpen || p.phase == OAfterComma) {
          p.text = has_last_key ? last_key : std::string();
          has_last_key = false;
          last_key.clear();
          p.phase = OAfterKey;
        } else if (p.phase == OInsideValue) {
          if (!has(p.emitted, p.text)) p.emitted.push_back(p.text);
          p.text.clear();
          p.phase = OAfterValue;
        }
        return;
      }
      if (p.kind == kArray) { p.phase = AAfterItem; return; }
      if (p.kind == kValue) {
        if (st.size() == 1) { p.phase = 1; return; }
        st.pop_back();
        continue;
      }
      return;
    }
  }

  void push_literal(const char* l) {
    Frame f;
    f.kind = kLiteral;
    f.lit = l;
    f.aux = 1;
    st.push_back(std::move(f));
  }
  void push_number(uint8_t b, bool integer) {
    Frame f;
    f.kind = kNumber;
    f.phase = b == '-' ? NSign : b == '0' ? NIntZero : NIntDigits;
    f.integer = integer;
    st.push_back(std::move(f));
  }
  void push_string(const Node* n, bool key) {
    Frame f;
    f.kind = kString;
    f.phase = SBody;
    f.node = n;
    f.is_key = key;
    st.push_back(std::move(f));
  }
  void push_object(const Node* n) {
    Frame f;
    f.kind = kObject;
    f.phase = OAfterOpen;
    f.node = n;
    st.push_back(std::move(f));
  }
  void push_array(const Node* items) {
    Frame f;
    f.kind = kArray;
    f.phase = AAfterOpen;
    f.node = items;
    st.push_back(std::move(f));
  }

  // ConstrainedGen.swift:372-459.
  bool open_value(const Node* n, uint8_t b) {
    switch (n->kind) {
      case Node::Any:
        if (b == '{') { push_object(&anyish().empty_object); return true; }
        if (b == '[') { push_array(&anyish().any_node); return true; }
        if (b == '"') { push_string(&anyish().any_node, false); return true; }
        if (b == '-' || is_digit(b)) { push_number(b, false); return true; }
        if (b == 't') { push_literal("true"); return true; }
        if (b == 'f') { push_literal("false"); return true; }
        if (b == 'n') { push_literal("null"); return true; }
        return false;
      case Node::Object:
        if (b != '{') return false;
        push_object(n);
        return true;
      case Node::Array:
        if (b != '[') return false;
        push_array(n->items.get());
        return true;
      case Node::String:
        if (b != '"') return false;
        push_string(n, false);
        return true;
      case Node::Number:
        if (b != '-' && !is_digit(b)) return false;
        push_number(b, n->integer);
        return true;
      case Node::Boolean:
        if (b == 't') { push_literal("true"); return true; }
        if (b == 'f') { push_literal("false"); return true; }
        return false;
      case Node::Null:
        if (b != 'n') return false;
        push_literal("null");
        return true;
    }
    return false;
  }

  // The enum list of a string frame: the schema's enum, or for a key the
  // parent object's open keys.  False when the string is unconstrained.
  bool enum_list(const Frame& sf, std::vector<const Lit*>* out) const {
    if (sf.is_key) return key_list(st[st.size() - 2], out);
    if (!sf.node->has_enum) return false;
    out->clear();
    for (auto& e : sf.node->enum_values) out->push_back(&e);
    return true;
  }

  // ConstrainedGen.swift:577-643.
  bool step_string(Frame& top, uint8_t b) {
    const Node* n = top.node;
    std::vector<const Lit*> en;
    switch (top.phase) {
      case SBody: {
        if (b == '"') {
          if (enum_list(top, &en)) {
            bool ok = false;
            for (auto* l : en) ok = ok || lit_eq(*l, top.text);
            if (!ok) return false;
          }
          if (n->has_min && static_cast<int64_t>(top.text.size()) < n->min_len) return false;
          if (top.is_key) { last_key = top.text; has_last_key = true; }
          st.pop_back();
          after_pop();
          return true;
        }
        if (b == '\\') {
          if (enum_list(top, &en)) return false;
          top.phase = SEscape;
          return true;
        }
        if (b < 0x20) return false;
        if (n->has_max && static_cast<int64_t>(top.text.size() + 1) > n->max_len) return false;
        top.text.push_back(static_cast<char>(b));
        if (enum_list(top, &en)) {
          bool ok = false;
          for (auto* l : en) ok = ok || lit_prefix(*l, top.text);
          if (!ok) { top.text.pop_back(); return false; }
        }
        return true;
      }
      case SEscape:
        switch (b) {
          case '"': case '\\': case '/': case 'b': case 'f': case 'n': case 'r': case 't': case 'u':
            if (n->has_max && static_cast<int64_t>(top.text.size() + 2) > n->max_len) return false;
            top.text.push_back('\\');
            top.text.push_back(static_cast<char>(b));
            top.phase = b == 'u' ? SUnicode : SBody;
            top.aux = 0;
            return true;
          default:
            return false;
        }
      case SUnicode:
        if (!is_hex(b)) return false;
        if (n->has_max && static_cast<int64_t>(top.text.size() + 1) > n->max_len) return false;
        top.text.push_back(static_cast<char>(b));
        if (++top.aux == 4) top.phase = SBody;
        return true;
      default:
        return false;
    }
  }

  // ConstrainedGen.swift:463-527.
  bool step_object(Frame& top, uint8_t b) {
    switch (top.phase) {
      case OAfterOpen:
      case OAfterComma:
        if (b == '}' && top.phase == OAfterOpen) {
          if (!required_done(top)) return false;
          st.pop_back();
          after_pop();
          return true;
        }
        if (b != '"' || keys_exhausted(top)) return false;
        push_string(&anyish().any_node, true);
        return true;
      case OAfterKey: {
        if (b != ':') return false;
        top.phase = OInsideValue;
        const Node* vs = prop_schema(top.node, top.text);
        Frame f;
        f.kind = kValue;
        f.node = vs;
        st.push_back(std::move(f));
        return true;
      }
      case OAfterValue:
        if (b == ',') {
          if (keys_exhausted(top)) return false;
          top.phase = OAfterComma;
          return true;
        }
        if (b == '}') {
          if (!required_done(top)) return false;
          st.pop_back();
          after_pop();
          return true;
        }
        return false;
      default:
        return false;
    }
  }

  // ConstrainedGen.swift:646-705 (numbers end on , } ] or whitespace, which
  // the parent then consumes).
  bool step_number(Frame& top, uint8_t b, int depth) {
    const bool term = b == ',' || b == '}' || b == ']' || b == ' ' || b == '\t' || b == '\n' || b == '\r';
    if (term) {
      const uint8_t s = top.phase;
      if (!(s == NIntZero || s == NIntDigits || s == NFrac || s == NExpDigits)) return false;
      st.pop_back();
      after_pop();
      return step(b, depth + 1);  // callers restore the snapshot on failure
    }
    switch (top.phase) {
      case NSign:
        if (!is_digit(b)) return false;
        top.phase = b == '0' ? NIntZero : NIntDigits;
        return true;
      case NIntZero:
      case NIntDigits:
        if (top.phase == NIntDigits && is_digit(b)) return true;
        if (top.integer) return false;
        if (b == '.') { top.phase = NAfterPoint; return true; }
        if (b == 'e' || b == 'E') { top.phase = NAfterExp; return true; }
        return false;
      case NAfterPoint:
        if (!is_digit(b)) return false;
        top.phase = NFrac;
        return true;
      case NFrac:
        if (is_digit(b)) return true;
        if (b == 'e' || b == 'E') { top.phase = NAfterExp; return true; }
        return false;
      case NAfterExp:
        if (b == '+' || b == '-') { top.phase = NExpSign; return true; }
        if (!is_digit(b)) return false;
        top.phase = NExpDigits;
        return true;
      case NExpSign:
        if (!is_digit(b)) return false;
        top.phase = NExpDigits;
        return true;
      case NExpDigits:
        return is_digit(b);
      default:
        return false;
    }
  }

  // One byte (ConstrainedGen.swift:214-276).  A false return may leave the
  // machine changed; accept() restores its snapshot.
  bool step(uint8_t b, int depth = 0) {
    if (depth > 64 || st.empty()) return false;
    Frame& top = st.back();
    switch (top.kind) {
      case kValue:
        return top.phase == 0 && open_value(top.node, b);
      case kObject:
        return step_object(top, b);
      case kArray:
        if (top.phase == AAfterItem) {
          if (b == ',') { top.phase = AAfterComma; return true; }
          if (b == ']') { st.pop_back(); after_pop(); return true; }
          return false;
        }
        if (top.phase == AAfterOpen && b == ']') { st.pop_back(); after_pop(); return true; }
        {
          Frame f;
          f.kind = kValue;
          f.node = top.node;
          st.push_back(std::move(f));
        }
        if (step(b, depth + 1)) return true;
        st.pop_back();
        return false;
      case kString:
        return step_string(top, b);
      case kNumber:
        return step_number(top, b, depth);
      case kLiteral: {
        const size_t len = strlen(top.lit);
        if (top.aux >= len || static_cast<uint8_t>(top.lit[top.aux]) != b) return false;
        if (++top.aux == len) { st.pop_back(); after_pop(); }
        return true;
      }
    }
    return false;
  }

  // All or nothing (ConstrainedGen.swift:188-199).
  bool accept(const uint8_t* bytes, size_t n) {
    Machine saved = *this;
    for (size_t i = 0; i < n; i++) {
      if (!step(bytes[i])) { *this = std::move(saved); return false; }
    }
    return true;
  }

  // A canonical byte string of the state: equal keys <=> equal futures, so
  // one mask row serves every state with the key.  Contents that cannot
  // influence what is accepted later are dropped: the text of an
  // unconstrained string beyond what its length limits observe, and object
  // keys that are neither declared nor required (they only ever reach the
  // emitted set, which is consulted for declared and required names).
  static bool names_key(const Node* n, const std::string& k) {
    for (auto& p : n->props)
      if (lit_eq(p.first, k)) return true;
    for (auto& r : n->required)
      if (lit_eq(r, k)) return true;
    return false;
  }
  static bool prefixes_required(const Node* n, const std::string& t) {
    for (auto& r : n->required)
      if (lit_prefix(r, t)) return true;
    return false;
  }
  std::string key() const {
    std::string k;
    auto put32 = [&](uint32_t v) { k.append(reinterpret_cast<const char*>(&v), 4); };
    auto put_str = [&](const std::string& v) { put32(static_cast<uint32_t>(v.size())); k += v; };
    for (size_t i = 0; i < st.size(); i++) {
      const Frame& f = st[i];
      k.push_back(static_cast<char>(f.kind));
      k.push_back(static_cast<char>(f.phase));
      k.push_back(static_cast<char>(f.aux));
      k.push_back(static_cast<char>(f.is_key | (f.integer << 1)));
      k.append(reinterpret_cast<const char*>(&f.node), sizeof(f.node));
      k.append(reinterpret_cast<const char*>(&f.lit), sizeof(f.lit));
      if (f.kind == kString) {
        const Node* n = f.node;
        if (f.is_key) {
          const Node* obj = st[i - 1].node;
          if (!obj->props.empty() || prefixes_required(obj, f.text)) put_str(f.text);
          else k.push_back('~');
        } else if (n->has_enum) {
          put_str(f.text);
        } else {
          const uint64_t len = f.text.size();
          const uint64_t seen = n->has_max ? len
                                : n->has_min ? std::min<uint64_t>(len, static_cast<uint64_t>(std::max<int64_t>(n->min_len, 0)))
                                : 0;
          put32(static_cast<uint32_t>(seen));
        }
      } else if (f.kind == kObject) {
        if (names_key(f.node, f.text)) put_str(f.text);
        else k.push_back('~');
        std::vector<std::string> em;
        for (auto& e : f.emitted)
          if (names_key(f.node, e)) em.push_back(e);
        std::sort(em.begin(), em.end());
        put32(static_cast<uint32_t>(em.size()));
        for (auto& e : em) put_str(e);
      }
    }
    return k;
  }
};

// ---------------------------------------------------------------- tool tags
// The tool-tag grammar of the serve path (Serve.swift:2057-2233,
// grammars/pace-tool-tags.gbnf): printable ASCII text without brackets, then
// exactly one tag, nothing after it.  The reference re-checks the whole
// output on every byte (isViable / isCompleteTag); this is the same language
// as an incremental automaton with a small state:
//   [POINT:none]   [POINT:x,y:label]   [CLICK:x,y:label]   [TYPE:text]
//   [SCROLL:up|down|left|right:n]      [KEY:keys]          [OPEN_APP:name]
// x, y, n: 1-4 digits; label: letter then [A-Za-z0-9 _-], 1-41 in all;
// text: [A-Za-z0-9 _-.,!?'"] 1-200; keys: [A-Za-z+] 1-30;
// name: letter then [A-Za-z0-9 ], 1-31 in all.
struct PaceTags {
  enum Mode : uint8_t { Text, Head, Body, CoordX, CoordY, Dir, Done };
  enum Tag : uint8_t { Point, Click, Type, Scroll, Key, OpenApp, PointNone };
  enum Cls : uint8_t { CDigit, CAlpha, CKey, CApp, CLabel, CType };
  Mode mode = Text;
  uint8_t tag = 0;
  uint8_t dir = 0;     // Dir: candidate direction (0 none yet)
  uint16_t pos = 0;    // Head / Dir / PointNone: bytes matched; Body / Coord: count
  // Body parameters
  uint8_t first_cls = 0, rest_cls = 0;
  uint16_t bmin = 0, bmax = 0;

  static const char* head(uint8_t t) {
    static const char* h[] = {"POINT:", "CLICK:", "TYPE:", "SCROLL:", "KEY:", "OPEN_APP:", "none]"};
    return h[t];
  }
  static bool alpha(uint8_t b) { return (b >= 'A' && b <= 'Z') || (b >= 'a' && b <= 'z'); }
  static bool cls(uint8_t c, uint8_t b) {
    const bool d = b >= '0' && b <= '9';
    switch (c) {
      case CDigit: return d;
      case CAlpha: return alpha(b);
      case CKey: return alpha(b) || b == '+';
      case CApp: return alpha(b) || d || b == ' ';
      case CLabel: return alpha(b) || d || b == ' ' || b == '_' || b == '-';
      case CType:
        return alpha(b) || d || b == ' ' || b == '_' || b == '-' || b == '.' || b == ',' ||
               b == '!' || b == '?' || b == '\'' || b == '"';
    }
    return false;
  }
  void body(uint8_t f, uint8_t r, uint16_t mn, uint16_t mx) {
    mode = Body; pos = 0; first_cls = f; rest_cls = r; bmin = mn; bmax = mx;
  }
  void enter(uint8_t t) {
    switch (t) {
      case Point: case Click: mode = CoordX; pos = 0; break;
      case Type: body(CType, CType, 1, 200); break;
      case Scroll: mode = Dir; dir = 0; pos = 0; break;
      case Key: body(CKey, CKey, 1, 30); break;
      case OpenApp: body(CAlpha, CApp, 1, 31); break;
      default: mode = Done; break;  // PointNone matched in full
    }
  }
  bool complete() const { return mode == Done; }

  bool step(uint8_t b) {
    switch (mode) {
      case Text:
        if (b == '[') { mode = Head; tag = 0xFF; pos = 0; return true; }
        return b >= 0x20 && b <= 0x7E && b != ']';
      case Head: {
        if (tag == 0xFF) {  // first byte after '[' picks the tag (initials are distinct)
          for (uint8_t t = 0; t <= OpenApp; t++)
            if (head(t)[0] == b) { tag = t; pos = 1; return true; }
          return false;
        }
        const char* h = head(tag);
        if (static_cast<uint8_t>(h[pos]) != b) return false;
        pos++;
        if (h[pos] == 0) {
          if (tag == PointNone) { mode = Done; return true; }
          enter(tag);
        }
        return true;
      }
      case CoordX:
        if (b >= '0' && b <= '9') {
          if (pos >= 4) return false;
          pos++;
          return true;
        }
        if (pos == 0 && tag == Point && b == 'n') { mode = Head; tag = PointNone; pos = 1; return true; }
        if (b == ',' && pos >= 1) { mode = CoordY; pos = 0; return true; }
        return false;
      case CoordY:
        if (b >= '0' && b <= '9') {
          if (pos >= 4) return false;
          pos++;
          return true;
        }
        if (b == ':' && pos >= 1) { body(CAlpha, CLabel, 1, 41); return true; }
        return false;
      case Dir: {
        static const char* dirs[] = {"up", "down", "left", "right"};
        if (dir == 0) {
          for (uint8_t d = 0; d < 4; d++)
            if (dirs[d][0] == b) { dir = static_cast<uint8_t>(d + 1); pos = 1; return true; }
          return false;
        }
        const char* dn = dirs[dir - 1];
        if (dn[pos] != 0) {
          if (static_cast<uint8_t>(dn[pos]) != b) return false;
          pos++;
          return true;
        }
        if (b != ':') return false;
        body(CDigit, CDigit, 1, 4);
        return true;
      }
      case Body:
        if (b == ']') {
          if (pos < bmin) return false;
          mode = Done;
          return true;
        }
        if (!cls(pos == 0 ? first_cls : rest_cls, b)) return false;
        if (pos + 1 > bmax) return false;
        pos++;
        return true;
      case Done:
        return false;
    }
    return false;
  }

  bool accept(const uint8_t* bytes, size_t n) {
    PaceTags saved = *this;
    for (size_t i = 0; i < n; i++)
      if (!step(bytes[i])) { *this = saved; return false; }
    return true;
  }

  std::string key() const {
    std::string k(12, '\0');
    k[0] = static_cast<char>(mode);
    k[1] = static_cast<char>(tag);
    k[2] = static_cast<char>(dir);
    memcpy(&k[3], &pos, 2);
    k[5] = static_cast<char>(first_cls);
    k[6] = static_cast<char>(rest_cls);
    memcpy(&k[7], &bmin, 2);
    memcpy(&k[9], &bmax, 2);
    return k;
  }
};

// ---------------------------------------------------------------- vocab trie
struct Trie {
  // node: children as (byte, node) sorted; token ids ending here
  struct TNode {
    std::vector<std::pair<uint8_t, int>> kids;
    std::vector<int> ends;
  };
  std::vector<TNode> nodes;
  Trie() { nodes.emplace_back(); }
  void add(const uint8_t* s, size_t n, int id) {
    int cur = 0;
    for (size_t i = 0; i < n; i++) {
      auto& kids = nodes[cur].kids;
      int nxt = -1;
      for (auto& kv : kids)
        if (kv.first == s[i]) { nxt = kv.second; break; }
      if (nxt < 0) {
        nxt = static_cast<int>(nodes.size());
        nodes[cur].kids.emplace_back(s[i], nxt);
        nodes.emplace_back();
      }
      cur = nxt;
    }
    nodes[cur].ends.push_back(id);
  }
};

}  // namespace tgg

struct tg_grammar {
  int32_t kind = TG_GRAMMAR_JSON_SCHEMA;
  std::unique_ptr<tgg::Node> root;
  int32_t vocab = 0;
  int32_t eos = -1;
  int32_t words = 0;
  std::vector<std::vector<uint8_t>> tokens;
  tgg::Trie trie;
  std::mutex mu;
  std::unordered_map<std::string, int32_t> rows;  // state key -> mask table row
  std::vector<uint32_t> table;                    // rows * words
};

struct tg_grammar_state {
  tg_grammar* g;
  tgg::Machine json;
  tgg::PaceTags tags;

  bool complete() const { return g->kind == TG_GRAMMAR_TOOL_TAGS ? tags.complete() : json.complete(); }
  bool accept(const uint8_t* b, size_t n) {
    return g->kind == TG_GRAMMAR_TOOL_TAGS ? tags.accept(b, n) : json.accept(b, n);
  }
  std::string key() const {
    return g->kind == TG_GRAMMAR_TOOL_TAGS ? "T" + tags.key() : "J" + json.key();
  }
};

namespace {
thread_local std::string g_gerr;
int32_t gfail(int32_t code, const std::string& m) {
  g_gerr = m;
  return code;
}

// Depth-first walk of the vocabulary trie carrying the automaton: a token is
// allowed iff every byte is accepted (ConstrainedGen.swift:805-822); a byte
// the automaton rejects prunes every token below it.
template <class M>
void walk_mask(const tgg::Trie& trie, const M& start, uint32_t* out) {
  struct Item { int node; M m; };
  std::vector<Item> stack;
  stack.push_back({0, start});
  while (!stack.empty()) {
    Item it = std::move(stack.back());
    stack.pop_back();
    const auto& nd = trie.nodes[it.node];
    for (size_t c = 0; c < nd.kids.size(); c++) {
      const int child = nd.kids[c].second;
      M probe = it.m;
      if (!probe.step(nd.kids[c].first)) continue;
      for (int id : trie.nodes[child].ends) out[id >> 5] |= 1u << (id & 31);
      if (!trie.nodes[child].kids.empty()) stack.push_back({child, std::move(probe)});
    }
  }
}

// JSON fast path.  Below a state whose top frame is the body of a string
// without enum or key constraint, a byte either stays in that frame (only the
// length and the escape phase change) or closes the string.  The walk carries
// just (length, phase, \u digits) there, and builds a full automaton copy only
// at a closing quote.  Same decisions as Machine::step_string.
struct JsonWalk {
  const tgg::Trie& trie;
  uint32_t* out;

  static bool plain_string(const tgg::Machine& m) {
    if (m.st.empty()) return false;
    const tgg::Frame& f = m.st.back();
    return f.kind == tgg::kString && !f.is_key && !f.node->has_enum;
  }
  void mark(int node) {
    for (int id : trie.nodes[node].ends) out[id >> 5] |= 1u << (id & 31);
  }

  void generic(int node, const tgg::Machine& m) {
    if (plain_string(m)) {
      const tgg::Frame& f = m.st.back();
      string_body(node, m, static_cast<int64_t>(f.text.size()), f.phase, f.aux);
      return;
    }
    const auto& nd = trie.nodes[node];
    for (auto& kv : nd.kids) {
      tgg::Machine probe = m;
      if (!probe.step(kv.first)) continue;
      mark(kv.second);
      if (!trie.nodes[kv.second].kids.empty()) generic(kv.second, probe);
    }
  }

  // `base` is the automaton at the string's start of this walk; its top frame
  // is the string (text of length len0 there); len/phase/aux the current values.
  void string_body(int node, const tgg::Machine& base, int64_t len, uint8_t phase, uint8_t aux) {
    const tgg::Node* sn = base.st.back().node;
    const bool hmax = sn->has_max;
    const int64_t mx = sn->max_len;
    const auto& nd = trie.nodes[node];
    for (auto& kv : nd.kids) {
      const uint8_t b = kv.first;
      const int child = kv.second;
      int64_t nlen = len;
      uint8_t nph = phase, naux = aux;
      if (phase == tgg::SBody) {
        if (b == '"') {
          tgg::Machine probe = base;
          tgg::Frame& f = probe.st.back();
          f.text.assign(static_cast<size_t>(len), 'a');  // content beyond its length is not consulted
          f.phase = tgg::SBody;
          if (!probe.step(b)) continue;
          mark(child);
          if (!trie.nodes[child].kids.empty()) generic(child, probe);
          continue;
        }
        if (b == '\\') {
          nph = tgg::SEscape;
        } else {
          if (b < 0x20) continue;
          if (hmax && len + 1 > mx) continue;
          nlen = len + 1;
        }
      } else if (phase == tgg::SEscape) {
        if (!(b == '"' || b == '\\' || b == '/' || b == 'b' || b == 'f' || b == 'n' || b == 'r' ||
              b == 't' || b == 'u'))
          continue;
        if (hmax && len + 2 > mx) continue;
        nlen = len + 2;
        nph = b == 'u' ? tgg::SUnicode : tgg::SBody;
        naux = 0;
      } else {
        if (!tgg::is_hex(b)) continue;
        if (hmax && len + 1 > mx) continue;
        nlen = len + 1;
        if (++naux == 4) nph = tgg::SBody;
      }
      mark(child);
      if (!trie.nodes[child].kids.empty()) string_body(child, base, nlen, nph, naux);
    }
  }
};

void compute_mask(const tg_grammar_state& s, uint32_t* out) {
  const tg_grammar& g = *s.g;
  std::fill(out, out + g.words, 0u);
  if (s.complete()) {
    if (g.eos >= 0 && g.eos < g.vocab) out[g.eos >> 5] |= 1u << (g.eos & 31);
    return;
  }
  if (g.kind == TG_GRAMMAR_TOOL_TAGS) walk_mask(g.trie, s.tags, out);
  else JsonWalk{g.trie, out}.generic(0, s.json);
}

// ServeGrammarSpec.parse (Serve.swift:1929-1941): text starting with '{'
// after trimming is a JSON Schema; a GBNF text with a `root ::=` rule naming
// the [POINT: tag is the tool-tag grammar; anything else is unsupported.
int32_t grammar_kind(const std::string& text, std::string* trimmed) {
  size_t a = 0, b = text.size();
  auto ws = [](char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\v' || c == '\f'; };
  while (a < b && ws(text[a])) a++;
  while (b > a && ws(text[b - 1])) b--;
  *trimmed = text.substr(a, b - a);
  if (!trimmed->empty() && (*trimmed)[0] == '{') return TG_GRAMMAR_JSON_SCHEMA;
  if (trimmed->find("root ::=") != std::string::npos && trimmed->find("[POINT:") != std::string::npos)
    return TG_GRAMMAR_TOOL_TAGS;
  return -1;
}
}  // namespace

extern "C" {

const char* tg_grammar_last_error(void) { return g_gerr.c_str(); }

int32_t tg_grammar_create(const char* grammar_text, int64_t text_len, int32_t vocab,
                          const uint8_t* token_bytes, const int64_t* token_offsets,
                          int32_t eos_id, tg_grammar** out) {
  if (!out) return gfail(TG_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  if (!grammar_text || text_len < 0) return gfail(TG_ERR_INVALID_ARG, "grammar text is NULL");
  if (vocab <= 0 || vocab > TG_MAX_VOCAB || !token_offsets || (!token_bytes && token_offsets[vocab] > 0))
    return gfail(TG_ERR_INVALID_ARG, "bad vocabulary");
  std::string trimmed;
  const int32_t kind = grammar_kind(std::string(grammar_text, static_cast<size_t>(text_len)), &trimmed);
  if (kind < 0)
    return gfail(TG_ERR_UNSUPPORTED, "unsupported grammar: pass a JSON Schema or the tool-tag GBNF grammar");
  auto g = std::make_unique<tg_grammar>();
  g->kind = kind;
  if (kind == TG_GRAMMAR_JSON_SCHEMA) {
    tgg::JParser jp{trimmed.data(), trimmed.data() + trimmed.size(), {}};
    tgg::JVal v;
    if (!jp.value(v)) return gfail(TG_ERR_INVALID_ARG, "schema is not valid JSON: " + jp.err);
    jp.ws();
    if (jp.p != jp.e) return gfail(TG_ERR_INVALID_ARG, "schema is not valid JSON: trailing characters");
    g->root = tgg::parse_schema(v);
  }
  g->vocab = vocab;
  g->eos = eos_id;
  g->words = (vocab + 31) / 32;
  g->tokens.resize(vocab);
  for (int32_t i = 0; i < vocab; i++) {
    const int64_t a = token_offsets[i], b = token_offsets[i + 1];
    if (a < 0 || b < a) return gfail(TG_ERR_INVALID_ARG, "token offsets must not decrease");
    g->tokens[i].assign(token_bytes + a, token_bytes + b);
    if (b > a) g->trie.add(token_bytes + a, static_cast<size_t>(b - a), i);
  }
  *out = g.release();
  return TG_OK;
}

int32_t tg_grammar_destroy(tg_grammar* g) {
  delete g;
  return TG_OK;
}

int32_t tg_grammar_kind(tg_grammar* g, int32_t* kind) {
  if (!g || !kind) return gfail(TG_ERR_INVALID_ARG, "NULL argument");
  *kind = g->kind;
  return TG_OK;
}

int32_t tg_grammar_state_create(tg_grammar* g, tg_grammar_state** out) {
  if (!g || !out) return gfail(TG_ERR_INVALID_ARG, "NULL argument");
  auto* s = new tg_grammar_state{g, {}, {}};
  if (g->kind == TG_GRAMMAR_JSON_SCHEMA) {
    tgg::Frame f;
    f.kind = tgg::kValue;
    f.node = g->root.get();
    s->json.st.push_back(std::move(f));
  }
  *out = s;
  return TG_OK;
}

int32_t tg_grammar_state_clone(const tg_grammar_state* s, tg_grammar_state** out) {
  if (!s || !out) return gfail(TG_ERR_INVALID_ARG, "NULL argument");
  *out = new tg_grammar_state(*s);
  return TG_OK;
}

int32_t tg_grammar_state_destroy(tg_grammar_state* s) {
  delete s;
  return TG_OK;
}

int32_t tg_grammar_accept_bytes(tg_grammar_state* s, const uint8_t* bytes, int64_t n,
                                int32_t* accepted) {
  if (!s || !accepted || n < 0 || (n > 0 && !bytes)) return gfail(TG_ERR_INVALID_ARG, "bad argument");
  *accepted = s->accept(bytes, static_cast<size_t>(n)) ? 1 : 0;
  return TG_OK;
}

int32_t tg_grammar_commit(tg_grammar_state* s, int32_t token, int32_t* accepted) {
  if (!s || !accepted) return gfail(TG_ERR_INVALID_ARG, "NULL argument");
  if (token < 0 || token >= s->g->vocab) { *accepted = 0; return TG_OK; }
  const auto& t = s->g->tokens[token];
  *accepted = s->accept(t.data(), t.size()) ? 1 : 0;
  return TG_OK;
}

int32_t tg_grammar_is_complete(const tg_grammar_state* s, int32_t* out) {
  if (!s || !out) return gfail(TG_ERR_INVALID_ARG, "NULL argument");
  *out = s->complete() ? 1 : 0;
  return TG_OK;
}

int32_t tg_grammar_mask(const tg_grammar_state* s, uint32_t* out_words) {
  if (!s || !out_words) return gfail(TG_ERR_INVALID_ARG, "NULL argument");
  compute_mask(*s, out_words);
  return TG_OK;
}

int32_t tg_grammar_state_row(const tg_grammar_state* s, int32_t* row, int32_t* is_new) {
  if (!s || !row) return gfail(TG_ERR_INVALID_ARG, "NULL argument");
  tg_grammar* g = s->g;
  const std::string k = s->key();
  std::lock_guard<std::mutex> lk(g->mu);
  auto it = g->rows.find(k);
  if (it != g->rows.end()) {
    *row = it->second;
    if (is_new) *is_new = 0;
    return TG_OK;
  }
  const int32_t r = static_cast<int32_t>(g->rows.size());
  g->table.resize(static_cast<size_t>(r + 1) * g->words);
  compute_mask(*s, g->table.data() + static_cast<size_t>(r) * g->words);
  g->rows.emplace(k, r);
  *row = r;
  if (is_new) *is_new = 1;
  return TG_OK;
}

int32_t tg_grammar_table(tg_grammar* g, const uint32_t** words, int32_t* rows) {
  if (!g || !words || !rows) return gfail(TG_ERR_INVALID_ARG, "NULL argument");
  std::lock_guard<std::mutex> lk(g->mu);
  *words = g->table.data();
  *rows = static_cast<int32_t>(g->rows.size());
  return TG_OK;
}

}  // extern "C"
