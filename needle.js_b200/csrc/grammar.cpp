// grammar.cpp -- the constrained tool-call grammar on the host, behind the C-ABI of
// include/needle_grammar.h.
//
//   JsonSchemaGrammar  JsonSchemaGrammar  packages/needle.js/src/tools/grammar.ts:258-627
//   ToolCallGrammar    ToolCallGrammar    grammar.ts:655-797
//   normalize_tools    normalizeTools     packages/needle.js/src/tools/schema.ts:124-204
//   allowed tokens     the constrained loop's vocabulary scan (packages/needle.js/src/tools/agent.ts:
//                      165-176), as a walk of a byte trie of the pieces
//
// Both grammars are byte automata over compact JSON driven by a JSON Schema; they restate the
// reference's frame stack, phases and checks byte for byte (the same bytes are accepted or
// rejected, the same values produced), in C++ with explicit value types.  Strings are kept as
// UTF-8 (escapes of lone surrogates as their 3-byte forms), so code-point lengths and JSON.stringify
// equality behave as in JavaScript.  Schema `pattern`s run through std::regex's ECMAScript grammar
// (a JavaScript RegExp without the u / v / s flags).
//
// Allowed tokens.  The reference clones the grammar and feeds every piece of the vocabulary at
// every step.  Here the pieces form a byte trie: a clone is fed one trie edge at a time and a
// rejected byte prunes the whole subtree, so the work is the number of trie nodes the grammar
// accepts rather than the vocabulary times the piece length.  Inside a string's content every byte
// other than a quote, a backslash or a control byte is accepted and only appended, so those
// subtrees are walked without copying the grammar at all (most steps of a tool call are spent in
// argument strings, where nearly the whole vocabulary is allowed).  The result is the same id list
// (ascending, as the reference's Map of candidates).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <regex>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/needle_cuda.h"
#include "../../include/needle_grammar.h"

namespace needle {
void set_last_error(const char* msg);
}

namespace {

struct SchemaError : std::runtime_error {
  explicit SchemaError(const std::string& m) : std::runtime_error(m) {}
};

// ------------------------------------------------------------------ JSON values

struct Json {
  enum Kind : uint8_t { Null, Bool, Number, String, Array, Object };
  Kind kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;                                   // UTF-8
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;    // insertion order (JavaScript object key order)

  const Json* get(const std::string& key) const {
    if (kind != Object) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  // obj[key] = v: an existing key keeps its position
  void set(const std::string& key, Json v) {
    for (auto& kv : obj)
      if (kv.first == key) {
        kv.second = std::move(v);
        return;
      }
    obj.emplace_back(key, std::move(v));
  }
};

void append_utf8(std::string& out, uint32_t cp) {
  if (cp < 0x80) {
    out += (char)cp;
  } else if (cp < 0x800) {
    out += (char)(0xC0 | (cp >> 6));
    out += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {  // includes lone surrogates (their 3-byte forms)
    out += (char)(0xE0 | (cp >> 12));
    out += (char)(0x80 | ((cp >> 6) & 0x3F));
    out += (char)(0x80 | (cp & 0x3F));
  } else {
    out += (char)(0xF0 | (cp >> 18));
    out += (char)(0x80 | ((cp >> 12) & 0x3F));
    out += (char)(0x80 | ((cp >> 6) & 0x3F));
    out += (char)(0x80 | (cp & 0x3F));
  }
}

// Code points of a UTF-8 string: the length of Array.from(string) in JavaScript.
size_t code_points(const std::string& s) {
  size_t n = 0;
  for (unsigned char c : s)
    if ((c & 0xC0) != 0x80) n++;
  return n;
}

// Strict UTF-8 check (TextDecoder with fatal: true): no overlong forms, surrogates or code points
// above U+10FFFF, no truncated sequences.
bool valid_utf8(const std::string& s) {
  size_t i = 0;
  const size_t n = s.size();
  while (i < n) {
    const unsigned char c = (unsigned char)s[i];
    if (c < 0x80) {
      i++;
      continue;
    }
    int len;
    uint32_t cp, min;
    if (c >= 0xC2 && c <= 0xDF) len = 2, cp = c & 0x1F, min = 0x80;
    else if (c >= 0xE0 && c <= 0xEF) len = 3, cp = c & 0x0F, min = 0x800;
    else if (c >= 0xF0 && c <= 0xF4) len = 4, cp = c & 0x07, min = 0x10000;
    else return false;
    if (i + len > n) return false;
    for (int k = 1; k < len; k++) {
      const unsigned char d = (unsigned char)s[i + k];
      if ((d & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (d & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
  }
  return true;
}

// valid_utf8 one byte at a time: ok() after the last byte tells whether the whole input was valid.
struct Utf8Check {
  int need = 0;  // continuation bytes still expected
  uint32_t cp = 0, min = 0;
  bool bad = false;
  void feed(uint8_t c) {
    if (bad) return;
    if (need > 0) {
      if ((c & 0xC0) != 0x80) {
        bad = true;
        return;
      }
      cp = (cp << 6) | (c & 0x3F);
      if (--need == 0 && (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))) bad = true;
      return;
    }
    if (c < 0x80) return;
    if (c >= 0xC2 && c <= 0xDF) need = 1, cp = c & 0x1F, min = 0x80;
    else if (c >= 0xE0 && c <= 0xEF) need = 2, cp = c & 0x0F, min = 0x800;
    else if (c >= 0xF0 && c <= 0xF4) need = 3, cp = c & 0x07, min = 0x10000;
    else bad = true;
  }
  bool ok() const { return !bad && need == 0; }
};

// Number::toString (ECMA-262 6.1.6.1.20): the shortest decimal that reads back as the same double.
std::string js_number(double x) {
  if (std::isnan(x) || std::isinf(x)) return "null";  // JSON.stringify
  if (x == 0.0) return "0";
  std::string sign = x < 0 ? "-" : "";
  const double a = std::fabs(x);
  char buf[64];
  int k = 1;
  for (; k <= 17; k++) {
    snprintf(buf, sizeof buf, "%.*e", k - 1, a);
    if (strtod(buf, nullptr) == a) break;
  }
  // buf = d[.ddd]e[+-]XX
  std::string digits;
  const char* p = buf;
  for (; *p && *p != 'e'; p++)
    if (*p != '.') digits += *p;
  const int e = atoi(p + 1);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  const int nd = (int)digits.size(), n = e + 1;
  std::string out;
  if (nd <= n && n <= 21) {
    out = digits + std::string(n - nd, '0');
  } else if (0 < n && n <= 21) {
    out = digits.substr(0, n) + "." + digits.substr(n);
  } else if (-6 < n && n <= 0) {
    out = "0." + std::string(-n, '0') + digits;
  } else {
    out = digits.substr(0, 1);
    if (nd > 1) out += "." + digits.substr(1);
    out += "e";
    out += (n - 1 > 0) ? "+" : "-";
    out += std::to_string(std::abs(n - 1));
  }
  return sign + out;
}

void stringify_string(const std::string& s, std::string& out) {
  out += '"';
  for (size_t i = 0; i < s.size(); i++) {
    const unsigned char c = (unsigned char)s[i];
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          char b[8];
          snprintf(b, sizeof b, "\\u%04x", c);
          out += b;
        } else if (c == 0xED && i + 2 < s.size() && ((unsigned char)s[i + 1] & 0xE0) == 0xA0) {
          // a lone surrogate (3-byte form): JSON.stringify escapes it
          const uint32_t cp = 0xD000 | (((unsigned char)s[i + 1] & 0x3F) << 6) | ((unsigned char)s[i + 2] & 0x3F);
          char b[8];
          snprintf(b, sizeof b, "\\u%04x", cp);
          out += b;
          i += 2;
        } else {
          out += (char)c;
        }
    }
  }
  out += '"';
}

// JSON.stringify without indentation.
void stringify(const Json& v, std::string& out) {
  switch (v.kind) {
    case Json::Null: out += "null"; break;
    case Json::Bool: out += v.b ? "true" : "false"; break;
    case Json::Number: out += js_number(v.num); break;
    case Json::String: stringify_string(v.str, out); break;
    case Json::Array:
      out += '[';
      for (size_t i = 0; i < v.arr.size(); i++) {
        if (i) out += ',';
        stringify(v.arr[i], out);
      }
      out += ']';
      break;
    case Json::Object:
      out += '{';
      for (size_t i = 0; i < v.obj.size(); i++) {
        if (i) out += ',';
        stringify_string(v.obj[i].first, out);
        out += ':';
        stringify(v.obj[i].second, out);
      }
      out += '}';
      break;
  }
}

std::string stringify(const Json& v) {
  std::string out;
  stringify(v, out);
  return out;
}

bool deep_equal(const Json& a, const Json& b) { return stringify(a) == stringify(b); }

// Minimal JSON parser (JSON.parse): objects keep key order, a repeated key keeps its first
// position and takes the last value.  Throws SchemaError on malformed input.
struct Parser {
  std::string s;
  size_t i = 0;
  explicit Parser(std::string text) : s(std::move(text)) {}
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) i++;
  }
  [[noreturn]] void fail(const char* what) { throw SchemaError(std::string("malformed JSON: ") + what); }
  uint32_t hex4() {
    if (i + 4 > s.size()) fail("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; k++) {
      const char c = s[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string_body() {  // after the opening quote
    std::string out;
    for (;;) {
      if (i >= s.size()) fail("unterminated string");
      const unsigned char c = (unsigned char)s[i++];
      if (c == '"') return out;
      if (c < 0x20) fail("control character in string");
      if (c != '\\') {
        out += (char)c;
        continue;
      }
      if (i >= s.size()) fail("unterminated escape");
      const char e = s[i++];
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp <= 0xDBFF && i + 6 <= s.size() && s[i] == '\\' && s[i + 1] == 'u') {
            const size_t save = i;
            i += 2;
            const uint32_t lo = hex4();
            if (lo >= 0xDC00 && lo <= 0xDFFF) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            else i = save;
          }
          append_utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
  }
  Json value() {
    ws();
    if (i >= s.size()) fail("unexpected end");
    Json v;
    const char c = s[i];
    if (c == '{') {
      i++;
      v.kind = Json::Object;
      ws();
      if (i < s.size() && s[i] == '}') {
        i++;
        return v;
      }
      for (;;) {
        ws();
        if (i >= s.size() || s[i] != '"') fail("expected key");
        i++;
        std::string key = string_body();
        ws();
        if (i >= s.size() || s[i] != ':') fail("expected ':'");
        i++;
        v.set(key, value());
        ws();
        if (i < s.size() && s[i] == ',') {
          i++;
          continue;
        }
        if (i < s.size() && s[i] == '}') {
          i++;
          return v;
        }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      i++;
      v.kind = Json::Array;
      ws();
      if (i < s.size() && s[i] == ']') {
        i++;
        return v;
      }
      for (;;) {
        v.arr.push_back(value());
        ws();
        if (i < s.size() && s[i] == ',') {
          i++;
          continue;
        }
        if (i < s.size() && s[i] == ']') {
          i++;
          return v;
        }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      i++;
      v.kind = Json::String;
      v.str = string_body();
      return v;
    }
    if (s.compare(i, 4, "true") == 0) {
      i += 4;
      v.kind = Json::Bool;
      v.b = true;
      return v;
    }
    if (s.compare(i, 5, "false") == 0) {
      i += 5;
      v.kind = Json::Bool;
      return v;
    }
    if (s.compare(i, 4, "null") == 0) {
      i += 4;
      return v;
    }
    const size_t start = i;
    if (i < s.size() && s[i] == '-') i++;
    while (i < s.size() && (isdigit((unsigned char)s[i]) || s[i] == '.' || s[i] == 'e' || s[i] == 'E' ||
                            s[i] == '+' || s[i] == '-'))
      i++;
    if (i == start) fail("unexpected character");
    v.kind = Json::Number;
    v.num = strtod(s.substr(start, i - start).c_str(), nullptr);
    return v;
  }
  Json document() {
    Json v = value();
    ws();
    if (i != s.size()) fail("trailing characters");
    return v;
  }
};

// ------------------------------------------------------------------ schema helpers

using SchemaPtr = std::shared_ptr<const Json>;

const Json& empty_schema() {
  static const Json e = [] {
    Json j;
    j.kind = Json::Object;
    return j;
  }();
  return e;
}

// A schema inside `owner` (a subschema, or `{}` when absent), sharing owner's lifetime instead of
// copying it.
SchemaPtr subschema(const SchemaPtr& owner, const Json* child) {
  if (child) return SchemaPtr(owner, child);
  static const SchemaPtr empty(std::shared_ptr<const Json>(), &empty_schema());
  return empty;
}

// resolveReference (grammar.ts:121-144): a local "#/..." ref, merged as { ...target, ...local }.
SchemaPtr resolve_reference(const SchemaPtr& schema, const Json& root) {
  const Json* ref = schema->get("$ref");
  if (!ref) return schema;
  if (ref->kind != Json::String || ref->str.compare(0, 2, "#/") != 0)
    throw SchemaError("Only local JSON Schema refs are supported");
  const Json* current = &root;
  size_t pos = 2;
  const std::string& path = ref->str;
  for (;;) {
    const size_t slash = path.find('/', pos);
    std::string part = path.substr(pos, slash == std::string::npos ? std::string::npos : slash - pos);
    for (size_t k; (k = part.find("~1")) != std::string::npos;) part.replace(k, 2, "/");
    for (size_t k; (k = part.find("~0")) != std::string::npos;) part.replace(k, 2, "~");
    const Json* next = nullptr;
    if (current->kind == Json::Object) next = current->get(part);
    else if (current->kind == Json::Array) {
      char* end = nullptr;
      const long idx = strtol(part.c_str(), &end, 10);
      if (end && *end == 0 && idx >= 0 && (size_t)idx < current->arr.size()) next = &current->arr[idx];
    }
    if (!next) throw SchemaError("Unresolved JSON Schema ref " + path);
    current = next;
    if (slash == std::string::npos) break;
    pos = slash + 1;
  }
  if (current->kind != Json::Object) throw SchemaError("JSON Schema ref " + path + " does not point to a schema");
  auto merged = std::make_shared<Json>(*current);
  for (const auto& kv : schema->obj)
    if (kv.first != "$ref") merged->set(kv.first, kv.second);
  return merged;
}

void schema_alternatives(const SchemaPtr& schema, const Json& root, std::vector<SchemaPtr>& out) {
  const SchemaPtr resolved = resolve_reference(schema, root);
  const Json* choices = resolved->get("oneOf");
  if (!choices || choices->kind == Json::Null) choices = resolved->get("anyOf");
  if (!choices || choices->kind == Json::Null) {
    out.push_back(resolved);
    return;
  }
  if (choices->kind != Json::Array) throw SchemaError("oneOf / anyOf must be an array");
  for (const Json& c : choices->arr) schema_alternatives(subschema(resolved, &c), root, out);
}

const char* json_type(const Json& v) {
  switch (v.kind) {
    case Json::Null: return "null";
    case Json::Bool: return "boolean";
    case Json::Number: return "number";
    case Json::String: return "string";
    case Json::Array: return "array";
    default: return "object";
  }
}

std::vector<std::string> possible_types(const Json& schema) {
  const Json* type = schema.get("type");
  if (type && type->kind == Json::Array) {
    std::vector<std::string> t;
    for (const Json& e : type->arr) t.push_back(e.kind == Json::String ? e.str : std::string());
    return t;
  }
  if (type && type->kind == Json::String) return {type->str};
  if (schema.get("properties")) return {"object"};
  if (schema.get("items")) return {"array"};
  if (const Json* c = schema.get("const")) return {json_type(*c)};
  if (const Json* e = schema.get("enum"); e && e->kind == Json::Array && !e->arr.empty()) {
    std::vector<std::string> t;
    for (const Json& v : e->arr) {
      const std::string ty = json_type(v);
      if (std::find(t.begin(), t.end(), ty) == t.end()) t.push_back(ty);
    }
    return t;
  }
  return {"string"};
}

bool type_starts_with(const std::string& type, int byte) {
  if (type == "string") return byte == 0x22;
  if (type == "object") return byte == 0x7b;
  if (type == "array") return byte == 0x5b;
  if (type == "boolean") return byte == 0x74 || byte == 0x66;
  if (type == "null") return byte == 0x6e;
  if (type == "number" || type == "integer") return byte == 0x2d || (byte >= 0x30 && byte <= 0x39);
  return false;
}

bool has_number(const Json& schema, const char* key, double& v) {
  const Json* j = schema.get(key);
  if (!j || j->kind != Json::Number) return false;
  v = j->num;
  return true;
}

bool validate_enum(const Json& value, const Json& schema) {
  if (const Json* c = schema.get("const"); c && !deep_equal(value, *c)) return false;
  if (const Json* e = schema.get("enum")) {
    bool any = false;
    if (e->kind == Json::Array)
      for (const Json& cand : e->arr)
        if (deep_equal(value, cand)) {
          any = true;
          break;
        }
    if (!any) return false;
  }
  return true;
}

bool is_email(const std::string& s) {  // /^[^\s@]+@[^\s@]+\.[^\s@]+$/
  static const std::regex re("^[^\\s@]+@[^\\s@]+\\.[^\\s@]+$", std::regex::ECMAScript);
  return std::regex_search(s, re);
}

bool is_uuid(const std::string& s) {  // /^[0-9a-f]{8}-[0-9a-f]{4}-[1-8][0-9a-f]{3}-[89ab][0-9a-f]{3}-[0-9a-f]{12}$/i
  static const std::regex re("^[0-9a-f]{8}-[0-9a-f]{4}-[1-8][0-9a-f]{3}-[89ab][0-9a-f]{3}-[0-9a-f]{12}$",
                             std::regex::ECMAScript | std::regex::icase);
  return std::regex_search(s, re);
}

bool validate_string(const std::string& value, const Json& schema) {
  const double length = (double)code_points(value);
  double v;
  if (has_number(schema, "minLength", v) && length < v) return false;
  if (has_number(schema, "maxLength", v) && length > v) return false;
  if (const Json* p = schema.get("pattern"); p && p->kind == Json::String) {
    try {
      const std::regex re(p->str, std::regex::ECMAScript);
      if (!std::regex_search(value, re)) return false;
    } catch (const std::regex_error&) {
      throw SchemaError("Invalid JSON Schema pattern " + p->str);
    }
  }
  if (const Json* f = schema.get("format"); f && f->kind == Json::String) {
    if (f->str == "email" && !is_email(value)) return false;
    if (f->str == "uuid" && !is_uuid(value)) return false;
  }
  Json j;
  j.kind = Json::String;
  j.str = value;
  return validate_enum(j, schema);
}

bool validate_number(double value, const Json& schema) {
  if (!std::isfinite(value)) return false;
  const auto types = possible_types(schema);
  const bool has_int = std::find(types.begin(), types.end(), "integer") != types.end();
  const bool has_num = std::find(types.begin(), types.end(), "number") != types.end();
  if (has_int && !has_num && std::trunc(value) != value) return false;
  double v;
  if (has_number(schema, "minimum", v) && value < v) return false;
  if (has_number(schema, "maximum", v) && value > v) return false;
  if (has_number(schema, "exclusiveMinimum", v) && value <= v) return false;
  if (has_number(schema, "exclusiveMaximum", v) && value >= v) return false;
  if (has_number(schema, "multipleOf", v)) {
    const double quotient = value / v;
    if (std::fabs(quotient - std::round(quotient)) > 1e-9 * std::max(1.0, std::fabs(quotient))) return false;
  }
  Json j;
  j.kind = Json::Number;
  j.num = value;
  return validate_enum(j, schema);
}

// isNumberPrefix (grammar.ts:222-245): a JSON number, or a prefix that can still become one.
bool is_number_prefix(const std::string& t) {
  size_t i = 0;
  auto digit = [&](size_t k) { return k < t.size() && t[k] >= '0' && t[k] <= '9'; };
  if (i < t.size() && t[i] == '-') i++;
  if (i == t.size()) return true;
  if (t[i] == '0') {
    i++;
    if (digit(i)) return false;
  } else if (t[i] >= '1' && t[i] <= '9') {
    while (digit(i)) i++;
  } else {
    return false;
  }
  if (i < t.size() && t[i] == '.') {
    i++;
    while (digit(i)) i++;
  }
  if (i < t.size() && (t[i] == 'e' || t[i] == 'E')) {
    i++;
    if (i < t.size() && (t[i] == '+' || t[i] == '-')) i++;
    while (digit(i)) i++;
  }
  return i == t.size();
}

// /^-?(?:0|[1-9]\d*)(?:\.\d+)?(?:[eE][+-]?\d+)?$/
bool is_complete_number(const std::string& t) {
  size_t i = 0;
  auto digit = [&](size_t k) { return k < t.size() && t[k] >= '0' && t[k] <= '9'; };
  if (i < t.size() && t[i] == '-') i++;
  if (i < t.size() && t[i] == '0') i++;
  else if (i < t.size() && t[i] >= '1' && t[i] <= '9') {
    while (digit(i)) i++;
  } else return false;
  if (i < t.size() && t[i] == '.') {
    i++;
    if (!digit(i)) return false;
    while (digit(i)) i++;
  }
  if (i < t.size() && (t[i] == 'e' || t[i] == 'E')) {
    i++;
    if (i < t.size() && (t[i] == '+' || t[i] == '-')) i++;
    if (!digit(i)) return false;
    while (digit(i)) i++;
  }
  return i == t.size();
}

// JSON.parse of the bytes of a string literal (quotes included), with the fatal UTF-8 decoder.
bool parse_string_literal(const std::string& bytes, std::string& out) {
  if (!valid_utf8(bytes)) return false;
  try {
    Parser p(bytes);
    const Json v = p.document();
    if (v.kind != Json::String) return false;
    out = v.str;
    return true;
  } catch (const SchemaError&) {
    return false;
  }
}

// ------------------------------------------------------------------ JsonSchemaGrammar

// State keys (the allowed-token mask cache): fixed-width integers and length-prefixed strings, so
// that distinct field sequences never concatenate to the same bytes.
void key_int(std::string& k, int64_t v) { k.append(reinterpret_cast<const char*>(&v), sizeof v); }
void key_str(std::string& k, const std::string& s) {
  key_int(k, (int64_t)s.size());
  k += s;
}

struct Candidate {
  std::string bytes;  // choice: JSON text of the value; key: the property name
  Json value;
  int offset = 0;
};

struct Frame {
  enum Kind : uint8_t { Value, String, Number, Literal, Choice, Array, Object, Key } kind = Value;
  SchemaPtr schema;
  // string
  std::string bytes;
  bool started = false, escaped = false;
  int unicode_remaining = 0;
  Utf8Check utf8;  // over `bytes` so far (the state key needs it without rescanning them)
  // number
  std::string text;
  // literal
  std::string literal;
  Json value;  // literal value; array values (Array) and object value (Object)
  int offset = 0;
  // choice / key
  std::vector<Candidate> candidates;
  // array / object
  enum Phase : uint8_t { Open, FirstOrEnd, InValue, AfterValue, KeyOrEnd, KeyRequired, InKey, Colon } phase = Open;
  std::vector<std::string> used;
  std::string current_key;
  bool has_key = false;
};

class SchemaGrammar {
 public:
  explicit SchemaGrammar(SchemaPtr root) : root_(std::move(root)) {
    Frame f;
    f.kind = Frame::Value;
    f.schema = root_;
    stack_.push_back(std::move(f));
  }

  bool complete() const {
    if (complete_) return true;
    if (stack_.size() == 1 && stack_[0].kind == Frame::Choice)
      for (const auto& c : stack_[0].candidates)
        if (c.offset == (int)c.bytes.size()) return true;
    return false;
  }

  // The parsed value once complete (nullptr before).
  const Json* value() const {
    if (complete_) return &value_;
    if (stack_.size() == 1 && stack_[0].kind == Frame::Choice)
      for (const auto& c : stack_[0].candidates)
        if (c.offset == (int)c.bytes.size()) return &c.value;
    return nullptr;
  }

  // True while the next byte goes to the content of a started string (not after a backslash, not
  // inside the hex digits of \u): every byte >= 0x20 other than '"' and '\\' is then accepted and
  // only appended to the string's bytes, which the allowed-token walk exploits.
  bool in_string_content() const {
    if (complete_ || stack_.empty()) return false;
    const Frame& f = stack_.back();
    return f.kind == Frame::String && f.started && !f.escaped && f.unicode_remaining == 0;
  }

  // True when feed_byte(byte) would certainly return false, decided from the top frame without
  // changing anything; false means "feed a copy to find out".  Each case restates the first check
  // feed_byte makes for that frame.
  bool rejects(int byte) const {
    if (complete_ || stack_.empty()) return true;
    const Frame& f = stack_.back();
    switch (f.kind) {
      case Frame::String:
        if (!f.started) return byte != 0x22;
        if (f.unicode_remaining > 0)
          return !((byte >= 0x30 && byte <= 0x39) || (byte >= 0x41 && byte <= 0x46) || (byte >= 0x61 && byte <= 0x66));
        if (f.escaped) {
          static const int ok[] = {0x22, 0x5c, 0x2f, 0x62, 0x66, 0x6e, 0x72, 0x74, 0x75};
          return std::find(std::begin(ok), std::end(ok), byte) == std::end(ok);
        }
        return byte < 0x20;
      case Frame::Number: {
        const char c = (char)byte;
        if ((c >= '0' && c <= '9') || c == 'e' || c == 'E' || c == '+' || c == '-' || c == '.')
          return !is_number_prefix(f.text + c);
        return !is_complete_number(f.text);
      }
      case Frame::Literal:
        return byte != (unsigned char)f.literal[f.offset];
      case Frame::Choice:
        for (const auto& c : f.candidates)
          if (c.offset == (int)c.bytes.size() || (unsigned char)c.bytes[c.offset] == byte) return false;
        return true;
      case Frame::Key:
        for (const auto& c : f.candidates)
          if (byte == 0x22 ? c.offset == (int)c.bytes.size()
                           : c.offset < (int)c.bytes.size() && (unsigned char)c.bytes[c.offset] == byte)
            return false;
        return true;
      case Frame::Array:
        if (f.phase == Frame::Open) return byte != 0x5b;
        if (f.phase == Frame::AfterValue) return byte != 0x2c && byte != 0x5d;
        return false;
      case Frame::Object:
        if (f.phase == Frame::Open) return byte != 0x7b;
        if (f.phase == Frame::KeyOrEnd) return byte != 0x22 && byte != 0x7d;
        if (f.phase == Frame::KeyRequired) return byte != 0x22;
        if (f.phase == Frame::Colon) return byte != 0x3a;
        if (f.phase == Frame::AfterValue) return byte != 0x2c && byte != 0x7d;
        return false;
      case Frame::Value:
        return false;
    }
    return false;
  }

  // True while the top frame is a number that is not the whole document.  A byte of the number's
  // charset then only extends number_text() (when the result is still a number prefix); any other
  // byte ends the number (end_number) and goes to the frame below.
  bool in_number() const { return !complete_ && stack_.size() >= 2 && stack_.back().kind == Frame::Number; }
  const std::string& number_text() const { return stack_.back().text; }
  void append_number(const char* bytes, size_t n) { stack_.back().text.append(bytes, n); }

  // Ends the number on top of the stack as a following byte outside its charset does: false when
  // the text is not a complete number or the value fails the schema.
  bool end_number() {
    const Frame& frame = stack_.back();
    if (!is_complete_number(frame.text)) return false;
    const double value = strtod(frame.text.c_str(), nullptr);
    if (!validate_number(value, *frame.schema)) return false;
    Json v;
    v.kind = Json::Number;
    v.num = value;
    finish(std::move(v));
    return true;
  }

  // Closing the current string (in_string_content) after more content bytes, decided without
  // feeding: prepared once for a state, then asked about many byte runs.  The literal's bytes so far
  // hold no unescaped quote and end outside an escape, and the run holds only content bytes, so
  // JSON.parse of the closed literal is the content decoded so far followed by the run, and the UTF-8
  // check continues from where the bytes so far left it.
  struct StringClose {
    Utf8Check utf8;
    std::string decoded;
    const Json* schema = nullptr;
    bool constrained = false;  // the schema checks strings beyond their type
    bool usable = false;
    // Whether feeding `bytes` and then '"' is accepted.
    bool accepts(const char* bytes, size_t n) const {
      Utf8Check u = utf8;
      for (size_t k = 0; k < n; k++) u.feed((uint8_t)bytes[k]);
      u.feed(0x22);
      if (!u.ok()) return false;
      if (!constrained) return true;
      std::string value = decoded;
      value.append(bytes, n);
      return validate_string(value, *schema);
    }
  };

  StringClose string_close() const {
    StringClose c;
    const Frame& f = stack_.back();
    c.utf8 = f.utf8;
    try {
      Parser p{f.bytes + "\""};
      Json v = p.document();
      if (v.kind != Json::String) return c;
      c.decoded = std::move(v.str);
    } catch (const SchemaError&) {
      return c;
    }
    c.schema = f.schema.get();
    for (const char* key : {"minLength", "maxLength", "pattern", "format", "enum", "const"})
      if (f.schema->get(key)) c.constrained = true;
    c.usable = true;
    return c;
  }

  // The bytes feed_byte could accept next, as a 256-bit set: exact when the top frame is a value
  // whose type is not chosen yet (the bytes that start one of its enum candidates or one of its
  // types, as feed_byte's Value case decides), every byte otherwise (rejects() covers the rest).
  void first_bytes(uint64_t (&set)[4]) const {
    set[0] = set[1] = set[2] = set[3] = ~0ull;
    if (complete_ || stack_.empty() || stack_.back().kind != Frame::Value) return;
    try {
      const Frame& frame = stack_.back();
      std::vector<SchemaPtr> alternatives;
      schema_alternatives(frame.schema, *root_, alternatives);
      bool all_enum = true, any_enum = false;
      uint64_t enum_set[4] = {0, 0, 0, 0}, type_set[4] = {0, 0, 0, 0};
      for (const auto& a : alternatives) {
        const SchemaPtr r = resolve_reference(a, *root_);
        const Json* c = r->get("const");
        const Json* e = r->get("enum");
        if (c) {
          const std::string t = stringify(*c);
          enum_set[(uint8_t)t[0] >> 6] |= 1ull << ((uint8_t)t[0] & 63);
          any_enum = true;
        } else if (e && e->kind == Json::Array) {
          for (const Json& v : e->arr) {
            const std::string t = stringify(v);
            enum_set[(uint8_t)t[0] >> 6] |= 1ull << ((uint8_t)t[0] & 63);
            any_enum = true;
          }
        }
        if (!c && !e) all_enum = false;
        for (const auto& t : possible_types(*r))
          for (int b = 0; b < 256; b++)
            if (type_starts_with(t, b)) type_set[b >> 6] |= 1ull << (b & 63);
      }
      const uint64_t* chosen = any_enum && all_enum ? enum_set : type_set;
      for (int k = 0; k < 4; k++) set[k] = chosen[k];
    } catch (const SchemaError&) {  // feed_byte reports it
    }
  }

  // The same as feeding `bytes` one at a time (each >= 0x20, none '"' or '\\') while
  // in_string_content().
  void append_string_content(const char* bytes, size_t n) {
    Frame& f = stack_.back();
    f.bytes.append(bytes, n);
    for (size_t k = 0; k < n; k++) f.utf8.feed((uint8_t)bytes[k]);
  }

  // Appends a key of this state.  Two grammars cloned from one template whose keys are equal accept
  // the same byte strings from here on, so they allow the same tokens.  The key keeps what
  // feed_byte can still read -- each frame's kind, schema, phase and progress -- and drops what no
  // later check reads: the content of a string or an array whose value nothing inspects any more
  // (no enum, const or uniqueItems on it or around it, and for a string no constraint of its own)
  // shrinks to the UTF-8 decoder's state or the item count.  A string's close then depends only on
  // that state: JSON.parse of bytes that feed_byte accepted fails only on invalid UTF-8 (lone
  // surrogate escapes decode).  Schemas inside the template's document are named by address (the
  // cache keeps the template alive); a schema outside it (a $ref merged into a new object) by its
  // JSON text.
  void state_key(std::string& k) const {
    if (complete_) {
      k += 'C';
      k += (char)value_.kind;
      return;
    }
    key_int(k, (int64_t)stack_.size());
    bool read_later = false;  // an enclosing value's content is checked when it closes
    for (const Frame& f : stack_) {
      k += (char)f.kind;
      key_schema(k, f.schema);
      const Json* s = f.schema.get();
      const bool checked = s && (s->get("enum") || s->get("const") || (f.kind == Frame::Array && s->get("uniqueItems")));
      switch (f.kind) {
        case Frame::Value:
          break;
        case Frame::String: {
          k += (char)((f.started ? 1 : 0) | (f.escaped ? 2 : 0));
          key_int(k, f.unicode_remaining);
          bool content = read_later;
          for (const char* key : {"minLength", "maxLength", "pattern", "format", "enum", "const"})
            if (s && s->get(key)) content = true;
          if (content) {
            key_str(k, f.bytes);
          } else {
            k += (char)(f.utf8.bad ? 1 : 0);
            key_int(k, f.utf8.need);
            if (f.utf8.need > 0) {
              key_int(k, f.utf8.cp);
              key_int(k, f.utf8.min);
            }
          }
          break;
        }
        case Frame::Number:
          key_str(k, f.text);
          break;
        case Frame::Literal:
          key_str(k, f.literal);
          key_int(k, f.offset);
          break;
        case Frame::Choice:
        case Frame::Key:
          key_int(k, (int64_t)f.candidates.size());
          for (const auto& c : f.candidates) {
            key_str(k, c.bytes);
            key_int(k, c.offset);
          }
          break;
        case Frame::Array:
          k += (char)f.phase;
          key_int(k, (int64_t)f.value.arr.size());
          if (read_later || checked) key_str(k, stringify(f.value));
          break;
        case Frame::Object: {
          k += (char)f.phase;
          k += (char)(f.has_key ? 1 : 0);
          key_str(k, f.current_key);
          std::vector<std::string> used(f.used);  // only membership is read
          std::sort(used.begin(), used.end());
          key_int(k, (int64_t)used.size());
          for (const auto& u : used) key_str(k, u);
          if (read_later || checked) key_str(k, stringify(f.value));
          break;
        }
      }
      read_later = read_later || checked;
    }
  }

  // The template this grammar was cloned from (shared by all its clones).
  const void* template_id() const { return root_.get(); }

  bool feed_byte(int byte) {
    if (complete_) return false;
    for (int retry = 0; retry < 16; retry++) {
      if (stack_.empty()) return false;
      Frame& frame = stack_.back();
      switch (frame.kind) {
        case Frame::Value: {
          std::vector<SchemaPtr> alternatives;
          schema_alternatives(frame.schema, *root_, alternatives);
          std::vector<SchemaPtr> resolved;
          for (const auto& a : alternatives) resolved.push_back(resolve_reference(a, *root_));
          std::vector<Json> enum_values;
          bool all_enum = true;
          for (const auto& r : resolved) {
            const Json* c = r->get("const");
            const Json* e = r->get("enum");
            if (c) enum_values.push_back(*c);
            else if (e && e->kind == Json::Array)
              for (const Json& v : e->arr) enum_values.push_back(v);
            if (!c && !e) all_enum = false;
          }
          if (!enum_values.empty() && all_enum) {
            Frame choice;
            choice.kind = Frame::Choice;
            for (Json& v : enum_values) {
              Candidate cand;
              cand.bytes = stringify(v);
              cand.value = std::move(v);
              choice.candidates.push_back(std::move(cand));
            }
            stack_.back() = std::move(choice);
            continue;
          }
          SchemaPtr matching;
          for (const auto& a : alternatives) {
            const auto types = possible_types(*resolve_reference(a, *root_));
            bool ok = false;
            for (const auto& t : types) ok = ok || type_starts_with(t, byte);
            if (ok) {
              matching = a;
              break;
            }
          }
          if (!matching) return false;
          const SchemaPtr schema = resolve_reference(matching, *root_);
          const auto types = possible_types(*schema);
          std::string selected;
          for (const auto& t : types)
            if (type_starts_with(t, byte)) {
              selected = t;
              break;
            }
          if (selected.empty()) return false;
          Frame f;
          f.schema = schema;
          if (selected == "string") {
            f.kind = Frame::String;
          } else if (selected == "number" || selected == "integer") {
            f.kind = Frame::Number;
          } else if (selected == "boolean") {
            const bool v = byte == 0x74;
            f.kind = Frame::Literal;
            f.literal = v ? "true" : "false";
            f.value.kind = Json::Bool;
            f.value.b = v;
          } else if (selected == "null") {
            f.kind = Frame::Literal;
            f.literal = "null";
          } else if (selected == "array") {
            f.kind = Frame::Array;
            f.phase = Frame::Open;
            f.value.kind = Json::Array;
          } else if (selected == "object") {
            f.kind = Frame::Object;
            f.phase = Frame::Open;
            f.value.kind = Json::Object;
          } else {
            return false;
          }
          stack_.back() = std::move(f);
          continue;
        }
        case Frame::String: {
          if (!frame.started) {
            if (byte != 0x22) return false;
            frame.started = true;
            frame.bytes += (char)byte;
            frame.utf8.feed((uint8_t)byte);
            return true;
          }
          if (frame.unicode_remaining > 0) {
            if (!((byte >= 0x30 && byte <= 0x39) || (byte >= 0x41 && byte <= 0x46) || (byte >= 0x61 && byte <= 0x66)))
              return false;
            frame.unicode_remaining--;
            frame.bytes += (char)byte;
            frame.utf8.feed((uint8_t)byte);
            return true;
          }
          if (frame.escaped) {
            static const int ok[] = {0x22, 0x5c, 0x2f, 0x62, 0x66, 0x6e, 0x72, 0x74, 0x75};
            if (std::find(std::begin(ok), std::end(ok), byte) == std::end(ok)) return false;
            frame.escaped = false;
            if (byte == 0x75) frame.unicode_remaining = 4;
            frame.bytes += (char)byte;
            frame.utf8.feed((uint8_t)byte);
            return true;
          }
          if (byte == 0x5c) {
            frame.escaped = true;
            frame.bytes += (char)byte;
            frame.utf8.feed((uint8_t)byte);
            return true;
          }
          if (byte < 0x20) return false;
          frame.bytes += (char)byte;
          frame.utf8.feed((uint8_t)byte);
          if (byte != 0x22) return true;
          std::string value;
          if (!parse_string_literal(frame.bytes, value)) return false;
          if (!validate_string(value, *frame.schema)) return false;
          Json v;
          v.kind = Json::String;
          v.str = std::move(value);
          finish(std::move(v));
          return true;
        }
        case Frame::Number: {
          const char c = (char)byte;
          if ((c >= '0' && c <= '9') || c == 'e' || c == 'E' || c == '+' || c == '-' || c == '.') {
            std::string next = frame.text + c;
            if (!is_number_prefix(next)) return false;
            frame.text = std::move(next);
            return true;
          }
          if (!end_number()) return false;
          continue;
        }
        case Frame::Literal: {
          if (byte != (unsigned char)frame.literal[frame.offset]) return false;
          frame.offset++;
          if (frame.offset == (int)frame.literal.size()) finish(Json(frame.value));
          return true;
        }
        case Frame::Choice: {
          std::vector<Candidate> continuing;
          for (const auto& c : frame.candidates)
            if (c.offset < (int)c.bytes.size() && (unsigned char)c.bytes[c.offset] == byte) continuing.push_back(c);
          if (!continuing.empty()) {
            for (auto& c : continuing) c.offset++;
            frame.candidates = std::move(continuing);
            return true;
          }
          const Candidate* completed = nullptr;
          for (const auto& c : frame.candidates)
            if (c.offset == (int)c.bytes.size()) {
              completed = &c;
              break;
            }
          if (!completed) return false;
          finish(Json(completed->value));
          continue;
        }
        case Frame::Array: {
          if (frame.phase == Frame::Open) {
            if (byte != 0x5b) return false;
            frame.phase = Frame::FirstOrEnd;
            return true;
          }
          double minimum = 0, maximum = 32, v;
          if (has_number(*frame.schema, "minItems", v)) minimum = v;
          if (has_number(*frame.schema, "maxItems", v)) maximum = v;
          const double count = (double)frame.value.arr.size();
          const Json* items = frame.schema->get("items");
          if (frame.phase == Frame::FirstOrEnd) {
            if (byte == 0x5d) {
              if (count < minimum) return false;
              if (!validate_enum(frame.value, *frame.schema)) return false;
              finish(Json(frame.value));
              return true;
            }
            if (count >= maximum) return false;
            frame.phase = Frame::InValue;
            push_value(subschema(frame.schema, items));
            continue;
          }
          if (frame.phase == Frame::AfterValue) {
            if (byte == 0x2c && count < maximum) {
              frame.phase = Frame::InValue;
              push_value(subschema(frame.schema, items));
              return true;
            }
            if (byte == 0x5d && count >= minimum) {
              const Json* unique = frame.schema->get("uniqueItems");
              if (unique && unique->kind != Json::Null && !(unique->kind == Json::Bool && !unique->b) &&
                  !(unique->kind == Json::Number && unique->num == 0) &&
                  !(unique->kind == Json::String && unique->str.empty())) {
                std::vector<std::string> seen;
                for (const Json& e : frame.value.arr) {
                  const std::string s = stringify(e);
                  if (std::find(seen.begin(), seen.end(), s) != seen.end()) return false;
                  seen.push_back(s);
                }
              }
              if (!validate_enum(frame.value, *frame.schema)) return false;
              finish(Json(frame.value));
              return true;
            }
            return false;
          }
          return false;
        }
        case Frame::Object: {
          if (frame.phase == Frame::Open) {
            if (byte != 0x7b) return false;
            frame.phase = Frame::KeyOrEnd;
            return true;
          }
          const Json* properties = frame.schema->get("properties");
          const Json* required = frame.schema->get("required");
          double minimum = 0, v;
          double maximum = properties && properties->kind == Json::Object ? (double)properties->obj.size() : 0.0;
          if (has_number(*frame.schema, "minProperties", v)) minimum = v;
          if (has_number(*frame.schema, "maxProperties", v)) maximum = v;
          auto all_required_used = [&]() {
            if (!required || required->kind != Json::Array) return true;
            for (const Json& r : required->arr)
              if (r.kind != Json::String || std::find(frame.used.begin(), frame.used.end(), r.str) == frame.used.end())
                return false;
            return true;
          };
          const double used = (double)frame.used.size();
          if (frame.phase == Frame::KeyOrEnd || frame.phase == Frame::KeyRequired) {
            if (byte == 0x7d && frame.phase == Frame::KeyOrEnd) {
              if (used < minimum || !all_required_used()) return false;
              if (!validate_enum(frame.value, *frame.schema)) return false;
              finish(Json(frame.value));
              return true;
            }
            if (byte != 0x22 || used >= maximum) return false;
            Frame key;
            key.kind = Frame::Key;
            if (properties && properties->kind == Json::Object)
              for (const auto& kv : properties->obj)
                if (std::find(frame.used.begin(), frame.used.end(), kv.first) == frame.used.end()) {
                  Candidate c;
                  c.bytes = kv.first;
                  key.candidates.push_back(std::move(c));
                }
            if (key.candidates.empty()) return false;
            frame.phase = Frame::InKey;
            stack_.push_back(std::move(key));
            return true;
          }
          if (frame.phase == Frame::Colon) {
            if (byte != 0x3a || !frame.has_key) return false;
            frame.phase = Frame::InValue;
            const Json* p = properties ? properties->get(frame.current_key) : nullptr;
            const Json* extra = frame.schema->get("additionalProperties");
            SchemaPtr child = subschema(frame.schema, p ? p : (extra && extra->kind == Json::Object ? extra : nullptr));
            push_value(std::move(child));
            return true;
          }
          if (frame.phase == Frame::AfterValue) {
            if (byte == 0x2c && used < maximum) {
              frame.phase = Frame::KeyRequired;
              return true;
            }
            if (byte == 0x7d && used >= minimum && all_required_used()) {
              if (!validate_enum(frame.value, *frame.schema)) return false;
              finish(Json(frame.value));
              return true;
            }
            return false;
          }
          return false;
        }
        case Frame::Key: {
          if (byte == 0x22) {
            const Candidate* done = nullptr;
            for (const auto& c : frame.candidates)
              if (c.offset == (int)c.bytes.size()) {
                done = &c;
                break;
              }
            if (!done) return false;
            const std::string name = done->bytes;
            stack_.pop_back();
            if (stack_.empty() || stack_.back().kind != Frame::Object) return false;
            stack_.back().current_key = name;
            stack_.back().has_key = true;
            stack_.back().phase = Frame::Colon;
            return true;
          }
          std::vector<Candidate> continuing;
          for (const auto& c : frame.candidates)
            if (c.offset < (int)c.bytes.size() && (unsigned char)c.bytes[c.offset] == byte) continuing.push_back(c);
          if (continuing.empty()) return false;
          for (auto& c : continuing) c.offset++;
          frame.candidates = std::move(continuing);
          return true;
        }
      }
    }
    return false;
  }

 private:
  void push_value(SchemaPtr schema) {
    Frame f;
    f.kind = Frame::Value;
    f.schema = std::move(schema);
    stack_.push_back(std::move(f));
  }

  void key_schema(std::string& k, const SchemaPtr& s) const {
    if (!s) {
      k += 'N';
    } else if (s.get() == &empty_schema()) {
      k += 'E';
    } else if (!s.owner_before(root_) && !root_.owner_before(s)) {
      k += 'P';
      key_int(k, (int64_t)(uintptr_t)s.get());
    } else {
      k += 'J';
      key_str(k, stringify(*s));
    }
  }

  void finish(Json value) {
    stack_.pop_back();
    if (stack_.empty()) {
      complete_ = true;
      value_ = std::move(value);
      return;
    }
    Frame& parent = stack_.back();
    if (parent.kind == Frame::Array && parent.phase == Frame::InValue) {
      parent.value.arr.push_back(std::move(value));
      parent.phase = Frame::AfterValue;
      return;
    }
    if (parent.kind == Frame::Object && parent.phase == Frame::InValue && parent.has_key) {
      parent.value.set(parent.current_key, std::move(value));
      parent.used.push_back(parent.current_key);
      parent.has_key = false;
      parent.current_key.clear();
      parent.phase = Frame::AfterValue;
      return;
    }
    throw SchemaError("Internal JSON Schema grammar stack is inconsistent");
  }

  SchemaPtr root_;
  std::vector<Frame> stack_;
  bool complete_ = false;
  Json value_;
};

// ------------------------------------------------------------------ ToolCallGrammar

struct Tool {
  std::string name;
  SchemaPtr parameters;
};

bool unsafe_name(const std::string& s) {
  for (unsigned char c : s)
    if (c == '"' || c == '\\' || c < 0x20) return true;
  return false;
}

// UTF-16 length of a UTF-8 string (JavaScript string length).
size_t utf16_length(const std::string& s) {
  size_t n = 0;
  for (size_t i = 0; i < s.size(); i++) {
    const unsigned char c = (unsigned char)s[i];
    if ((c & 0xC0) == 0x80) continue;
    n += c >= 0xF0 ? 2 : 1;
  }
  return n;
}

// normalizeTools (schema.ts:124-204) over a JSON array of tools ({name, description?,
// parameters?} or {type: "function", function: {...}}).
std::vector<Tool> normalize_tools(const Json& input) {
  if (input.kind != Json::Array) throw SchemaError("Tools must be a JSON array");
  std::vector<Tool> tools;
  for (const Json& t : input.arr) {
    const Json* src = &t;
    if (const Json* fn = t.get("function"); fn && fn->kind == Json::Object) src = fn;
    const Json* name = src->get("name");
    if (!name || name->kind != Json::String || name->str.empty() || utf16_length(name->str) > 128)
      throw SchemaError("A tool name must contain 1\xe2\x80\x93" "128 characters");
    if (unsafe_name(name->str))
      throw SchemaError("Tool name " + stringify(*name) + " contains characters that cannot be constrained safely");
    Json parameters;
    if (const Json* p = src->get("parameters"); p && p->kind != Json::Null) {
      parameters = *p;
    } else {
      parameters.kind = Json::Object;
      Json ty;
      ty.kind = Json::String;
      ty.str = "object";
      parameters.set("type", ty);
      Json props;
      props.kind = Json::Object;
      parameters.set("properties", props);
    }
    if (parameters.kind != Json::Object) throw SchemaError("Tool " + name->str + " parameters must be an object schema");
    const Json* type = parameters.get("type");
    if (type && !(type->kind == Json::String && type->str == "object"))
      throw SchemaError("Tool " + name->str + " parameters must be an object schema");
    Json properties;
    properties.kind = Json::Object;
    if (const Json* p = parameters.get("properties"); p && p->kind != Json::Null) properties = *p;
    for (const auto& kv : properties.obj) {
      if (kv.first.empty() || unsafe_name(kv.first))
        throw SchemaError("Tool " + name->str + " has an invalid parameter name");
      if (kv.second.kind != Json::Object && kv.second.kind != Json::Array)
        throw SchemaError("Tool " + name->str + " parameter " + kv.first + " has no schema");
    }
    if (const Json* r = parameters.get("required"); r && r->kind == Json::Array)
      for (const Json& n : r->arr)
        if (n.kind != Json::String || !properties.get(n.str))
          throw SchemaError("Tool " + name->str + " requires unknown parameter");
    Json ty;
    ty.kind = Json::String;
    ty.str = "object";
    parameters.set("type", ty);
    parameters.set("properties", properties);
    for (const Tool& other : tools)
      if (other.name == name->str) throw SchemaError("Duplicate tool name " + name->str);
    tools.push_back({name->str, std::make_shared<Json>(std::move(parameters))});
  }
  return tools;
}

struct ToolCall {
  std::string name;
  Json arguments;
};

class ToolGrammar {
 public:
  ToolGrammar(std::shared_ptr<const std::vector<Tool>> tools, int maximum_calls)
      : tools_(std::move(tools)), maximum_calls_(std::max(1, maximum_calls)) {
    if (tools_->empty()) throw SchemaError("Tool-call grammar needs at least one tool");
  }

  bool complete() const { return phase_ == Done; }
  const std::vector<ToolCall>& calls() const { return calls_; }
  bool in_string_content() const { return phase_ == Arguments && arguments_ && arguments_->in_string_content(); }

  // As SchemaGrammar::rejects: feed_byte's first check for the current phase, without feeding.
  bool rejects(int byte) const {
    switch (phase_) {
      case ArrayOpen: return byte != 0x5b;
      case CallOpen: return byte != 0x7b;
      case NameLiteral: return byte != (unsigned char)kName[literal_offset_];
      case ToolName:
        for (const auto& c : names_) {
          const std::string& n = (*tools_)[c.first].name;
          if (byte == 0x22 ? c.second == (int)n.size() : c.second < (int)n.size() && (unsigned char)n[c.second] == byte)
            return false;
        }
        return true;
      case ArgumentsLiteral: return byte != (unsigned char)kArguments[literal_offset_];
      case Arguments:
        if (!arguments_) return true;
        if (arguments_->complete()) return byte != 0x7d;
        return arguments_->rejects(byte);
      case CallClose: return byte != 0x7d;
      case AfterCall: return byte != 0x5d && byte != 0x2c;
      case Done: return true;
    }
    return false;
  }
  void append_string_content(const char* bytes, size_t n) { arguments_->append_string_content(bytes, n); }
  SchemaGrammar::StringClose string_close() const { return arguments_->string_close(); }
  void first_bytes(uint64_t (&set)[4]) const {
    if (phase_ == Arguments && arguments_ && !arguments_->complete()) {
      arguments_->first_bytes(set);
      return;
    }
    set[0] = set[1] = set[2] = set[3] = ~0ull;
  }
  bool in_number() const { return phase_ == Arguments && arguments_ && arguments_->in_number(); }
  const std::string& number_text() const { return arguments_->number_text(); }
  void append_number(const char* bytes, size_t n) { arguments_->append_number(bytes, n); }
  bool end_number() { return arguments_->end_number(); }

  // As SchemaGrammar::state_key.  The calls made so far are read only through the tools they used
  // (a used tool's name is not offered again; their number bounds further calls); the arguments
  // grammar is keyed while it is being fed or checked.
  void state_key(std::string& k) const {
    k += (char)phase_;
    std::vector<int> used(used_);
    std::sort(used.begin(), used.end());
    key_int(k, (int64_t)used.size());
    for (int u : used) key_int(k, u);
    switch (phase_) {
      case NameLiteral:
        key_int(k, literal_offset_);
        break;
      case ToolName:
        key_int(k, (int64_t)names_.size());
        for (const auto& c : names_) {
          key_int(k, c.first);
          key_int(k, c.second);
        }
        break;
      case ArgumentsLiteral:
        key_int(k, literal_offset_);
        key_int(k, current_);
        break;
      case Arguments:
      case CallClose:
        key_int(k, current_);
        if (arguments_) arguments_->state_key(k);
        else k += 'X';
        break;
      default:
        break;
    }
  }
  const void* template_id() const { return tools_.get(); }
  int maximum_calls() const { return maximum_calls_; }

  bool feed_byte(int byte) {
    for (int retry = 0; retry < 8; retry++) {
      switch (phase_) {
        case ArrayOpen:
          if (byte != 0x5b) return false;
          phase_ = CallOpen;
          return true;
        case CallOpen:
          if (byte != 0x7b) return false;
          phase_ = NameLiteral;
          literal_offset_ = 0;
          return true;
        case NameLiteral:
          if (byte != (unsigned char)kName[literal_offset_]) return false;
          literal_offset_++;
          if (literal_offset_ == kNameLength) {
            phase_ = ToolName;
            names_.clear();
            for (int k = 0; k < (int)tools_->size(); k++)
              if (std::find(used_.begin(), used_.end(), k) == used_.end()) names_.push_back({k, 0});
          }
          return true;
        case ToolName: {
          if (byte == 0x22) {
            int found = -1;
            for (const auto& c : names_)
              if (c.second == (int)(*tools_)[c.first].name.size()) {
                found = c.first;
                break;
              }
            if (found < 0) return false;
            current_ = found;
            phase_ = ArgumentsLiteral;
            literal_offset_ = 0;
            return true;
          }
          std::vector<std::pair<int, int>> continuing;
          for (const auto& c : names_) {
            const std::string& n = (*tools_)[c.first].name;
            if (c.second < (int)n.size() && (unsigned char)n[c.second] == byte) continuing.push_back({c.first, c.second + 1});
          }
          if (continuing.empty()) return false;
          names_ = std::move(continuing);
          return true;
        }
        case ArgumentsLiteral:
          if (byte != (unsigned char)kArguments[literal_offset_]) return false;
          literal_offset_++;
          if (literal_offset_ == kArgumentsLength) {
            if (current_ < 0 || current_ >= (int)tools_->size()) return false;
            arguments_ = std::make_unique<SchemaGrammar>((*tools_)[current_].parameters);
            phase_ = Arguments;
          }
          return true;
        case Arguments:
          if (!arguments_) return false;
          if (arguments_->complete()) {
            phase_ = CallClose;
            continue;
          }
          return arguments_->feed_byte(byte);
        case CallClose: {
          if (byte != 0x7d) return false;
          const Json* args = arguments_ ? arguments_->value() : nullptr;
          if (current_ < 0 || !args || args->kind != Json::Object) return false;
          calls_.push_back({(*tools_)[current_].name, *args});
          used_.push_back(current_);
          phase_ = AfterCall;
          return true;
        }
        case AfterCall:
          if (byte == 0x5d) {
            phase_ = Done;
            return true;
          }
          if (byte == 0x2c && (int)calls_.size() < maximum_calls_ && used_.size() < tools_->size()) {
            phase_ = CallOpen;
            return true;
          }
          return false;
        case Done:
          return false;
      }
    }
    return false;
  }

  ToolGrammar(const ToolGrammar& o)
      : tools_(o.tools_), maximum_calls_(o.maximum_calls_), phase_(o.phase_), literal_offset_(o.literal_offset_),
        names_(o.names_), current_(o.current_), used_(o.used_),
        arguments_(o.arguments_ ? std::make_unique<SchemaGrammar>(*o.arguments_) : nullptr), calls_(o.calls_) {}

  // Copy-assignment keeps this object's buffers (strings, vectors, the argument grammar) and only
  // overwrites their contents, which is what the allowed-token walk's per-depth scratch relies on.
  ToolGrammar& operator=(const ToolGrammar& o) {
    if (this == &o) return *this;
    tools_ = o.tools_;
    maximum_calls_ = o.maximum_calls_;
    phase_ = o.phase_;
    literal_offset_ = o.literal_offset_;
    names_ = o.names_;
    current_ = o.current_;
    used_ = o.used_;
    if (!o.arguments_) arguments_.reset();
    else if (arguments_) *arguments_ = *o.arguments_;
    else arguments_ = std::make_unique<SchemaGrammar>(*o.arguments_);
    calls_ = o.calls_;
    return *this;
  }

 private:
  static constexpr const char kName[] = "\"name\":\"";
  static constexpr int kNameLength = sizeof(kName) - 1;
  static constexpr const char kArguments[] = ",\"arguments\":";
  static constexpr int kArgumentsLength = sizeof(kArguments) - 1;
  enum Phase : uint8_t { ArrayOpen, CallOpen, NameLiteral, ToolName, ArgumentsLiteral, Arguments, CallClose, AfterCall, Done };
  std::shared_ptr<const std::vector<Tool>> tools_;
  int maximum_calls_;
  Phase phase_ = ArrayOpen;
  int literal_offset_ = 0;
  std::vector<std::pair<int, int>> names_;  // (tool index, offset)
  int current_ = -1;
  std::vector<int> used_;
  std::unique_ptr<SchemaGrammar> arguments_;
  std::vector<ToolCall> calls_;
};

// ------------------------------------------------------------------ vocabulary trie

struct Trie {
  struct Node {
    std::vector<std::pair<uint8_t, int32_t>> children;  // sorted by byte
    std::vector<uint32_t> ids;                           // pieces ending here
  };
  std::vector<Node> nodes{1};
  int32_t max_len = 0;

  void insert(const uint8_t* bytes, int32_t n, uint32_t id) {
    int32_t cur = 0;
    for (int32_t k = 0; k < n; k++) {
      auto& ch = nodes[cur].children;
      auto it = std::lower_bound(ch.begin(), ch.end(), std::make_pair(bytes[k], (int32_t)-1));
      if (it != ch.end() && it->first == bytes[k]) {
        cur = it->second;
      } else {
        const int32_t next = (int32_t)nodes.size();
        ch.insert(it, {bytes[k], next});
        nodes.emplace_back();
        cur = next;
      }
    }
    nodes[cur].ids.push_back(id);
    max_len = std::max(max_len, n);
  }

  // String content.  Inside a string every byte >= 0x20 other than '"' and '\\' is accepted and
  // only appended, so from a string state at the root: every piece made only of such bytes is
  // accepted (`plain`), a piece with a control byte before any quote or backslash is rejected, and
  // the rest depend on the grammar from their first quote or backslash on (`exits`: the node below
  // that byte, the byte, its depth and the plain bytes before it in `exit_bytes`).
  struct Exit {
    int32_t node, depth, prefix_offset, prefix_length;
    uint8_t byte;
  };
  std::vector<uint8_t> plain;
  std::vector<Exit> exits;
  std::string exit_bytes;

  void index_string_content(int32_t vocab_size) {
    plain.assign(vocab_size, 0);
    exits.clear();
    exit_bytes.clear();
    std::string path;
    index_from(0, path);
  }

 private:
  void index_from(int32_t node, std::string& path) {
    for (uint32_t id : nodes[node].ids) plain[id] = 1;
    for (const auto& edge : nodes[node].children) {
      const uint8_t b = edge.first;
      if (b < 0x20) continue;
      if (b == 0x22 || b == 0x5c) {
        exits.push_back({edge.second, (int32_t)path.size() + 1, (int32_t)exit_bytes.size(), (int32_t)path.size(), b});
        exit_bytes += path;
        continue;
      }
      path.push_back((char)b);
      index_from(edge.second, path);
      path.pop_back();
    }
  }
};

}  // namespace

// ------------------------------------------------------------------ C-ABI

struct needle_grammar {
  std::unique_ptr<SchemaGrammar> schema;
  std::unique_ptr<ToolGrammar> tools;
  bool feed_byte(int b) { return schema ? schema->feed_byte(b) : tools->feed_byte(b); }
  bool complete() const { return schema ? schema->complete() : tools->complete(); }
};

struct needle_vocab {
  Trie trie;
  int32_t size = 0;  // ids are below this
};

// Allowed-token masks per grammar state (needle_mask_cache_*): a fixed table of `capacity` bit
// masks, reused least-recently-used first, indexed by the state key of the grammar and the walk's
// length limit.
struct needle_mask_cache {
  std::unique_ptr<needle_grammar> keep;  // a clone of the template: keeps its schemas alive
  const void* template_id = nullptr;
  int maximum_calls = 0;
  const needle_vocab* vocab = nullptr;
  int32_t capacity = 0, words = 0;
  std::vector<uint32_t> table;   // [capacity][words]
  std::vector<int32_t> count;    // ids set in each mask
  std::vector<std::string> key;  // "" = free
  std::vector<int32_t> prev, next;
  int32_t head = -1, tail = -1;  // most / least recently used
  std::vector<uint64_t> used_in;  // the lookup that last used each slot
  uint64_t lookups = 0;
  std::unordered_map<std::string, int32_t> index;
  int64_t hits = 0, misses = 0, evictions = 0;
};

namespace {

int fail(int code, const std::string& msg) {
  needle::set_last_error(msg.c_str());
  return code;
}

// The trie walk.  `mark` collects accepted ids; `pending` holds the string-content bytes fed since
// walk_string's `base`, `number` the whole text of the number walk_number is extending.
struct Walk {
  const Trie& trie;
  int32_t limit;
  std::vector<uint8_t>& mark;
  std::string pending;
  std::string number;
};

inline void mark_ids(Walk& w, int32_t node) {
  for (uint32_t id : w.trie.nodes[node].ids) w.mark[id] = 1;
}

inline bool number_byte(uint8_t c) {
  return (c >= '0' && c <= '9') || c == 'e' || c == 'E' || c == '+' || c == '-' || c == '.';
}

// Grammars per trie depth, per thread, kept across calls: copying a state into one by assignment
// reuses its buffers instead of allocating a new copy for every trie edge.  Tag 0 holds the state
// after an edge, tag 1 the state after a number ended at a node.
template <class G, int Tag>
G& scratch(int32_t depth, const G& from) {
  thread_local std::vector<std::unique_ptr<G>> slots;
  if ((int32_t)slots.size() <= depth) slots.resize(depth + 1);
  if (!slots[depth]) slots[depth] = std::make_unique<G>(from);
  else *slots[depth] = from;
  return *slots[depth];
}

template <class G>
void descend(Walk& w, int32_t node, const G& g, int32_t depth);

// The general case: every edge the grammar does not reject outright is fed to a copy.
template <class G>
void walk(Walk& w, int32_t node, const G& g, int32_t depth) {
  uint64_t first[4];
  g.first_bytes(first);
  for (const auto& edge : w.trie.nodes[node].children) {
    if (depth + 1 > w.limit) break;
    if (!((first[edge.first >> 6] >> (edge.first & 63)) & 1) || g.rejects(edge.first)) continue;
    G& next = scratch<G, 0>(depth + 1, g);
    if (!next.feed_byte(edge.first)) continue;
    mark_ids(w, edge.second);
    descend(w, edge.second, next, depth + 1);
  }
}

// `base` is inside a string's content and the bytes on the path since then are in w.pending.
// Content bytes (>= 0x20, not '"' or '\\') are accepted without looking at the grammar, so the
// subtree below them is walked without copying it; a quote or backslash edge applies the pending
// bytes to a copy and continues from there.  Control bytes are rejected in a string.
template <class G>
void walk_string(Walk& w, int32_t node, const G& base, int32_t depth) {
  if (node == 0 && w.limit >= w.trie.max_len) {  // from the root: the index built at vocab open
    for (size_t id = 0; id < w.mark.size(); id++) w.mark[id] |= w.trie.plain[id];
    // A closing quote is decided by StringClose; what follows it in the piece goes to the frame
    // below the string, whose first check does not depend on the string's value, so `closed` (the
    // state after any accepted close) rejects most continuations without a copy.
    const auto close = base.string_close();
    const G* closed = nullptr;
    for (const auto& e : w.trie.exits) {
      const char* prefix = w.trie.exit_bytes.data() + e.prefix_offset;
      const auto& children = w.trie.nodes[e.node].children;
      if (e.byte == 0x22 && close.usable) {
        if (!close.accepts(prefix, e.prefix_length)) continue;
        mark_ids(w, e.node);
        bool more = false;
        for (const auto& c : children)
          if (!closed || !closed->rejects(c.first)) {
            more = true;
            break;
          }
        if (!more) continue;
      }
      G& next = scratch<G, 0>(e.depth, base);
      next.append_string_content(prefix, e.prefix_length);
      if (!next.feed_byte(e.byte)) continue;
      mark_ids(w, e.node);
      if (e.byte == 0x22 && !closed) closed = &scratch<G, 2>(0, next);
      descend(w, e.node, next, e.depth);
    }
    return;
  }
  for (const auto& edge : w.trie.nodes[node].children) {
    if (depth + 1 > w.limit) break;
    const uint8_t b = edge.first;
    if (b < 0x20) continue;
    if (b != 0x22 && b != 0x5c) {
      mark_ids(w, edge.second);
      w.pending.push_back((char)b);
      walk_string(w, edge.second, base, depth + 1);
      w.pending.pop_back();
      continue;
    }
    G& next = scratch<G, 0>(depth + 1, base);
    next.append_string_content(w.pending.data(), w.pending.size());
    if (!next.feed_byte(b)) continue;
    mark_ids(w, edge.second);
    descend(w, edge.second, next, depth + 1);
  }
}

// `base` is inside a number whose text, with the path's bytes since `base`, is w.number (the first
// `base_length` bytes are base's own).  A number byte is accepted when the text stays a number
// prefix, with no copy; the other bytes end the number once per node, on a copy, and are fed to
// what lies below it.
template <class G>
void walk_number(Walk& w, int32_t node, const G& base, size_t base_length, int32_t depth) {
  const G* ended = nullptr;
  bool tried = false;
  for (const auto& edge : w.trie.nodes[node].children) {
    if (depth + 1 > w.limit) break;
    const uint8_t b = edge.first;
    if (number_byte(b)) {
      w.number.push_back((char)b);
      if (is_number_prefix(w.number)) {
        mark_ids(w, edge.second);
        walk_number(w, edge.second, base, base_length, depth + 1);
      }
      w.number.pop_back();
      continue;
    }
    if (!tried) {
      tried = true;
      if (is_complete_number(w.number)) {
        G& e = scratch<G, 1>(depth, base);
        e.append_number(w.number.data() + base_length, w.number.size() - base_length);
        if (e.end_number()) ended = &e;
      }
    }
    if (!ended || ended->rejects(b)) continue;
    G& next = scratch<G, 0>(depth + 1, *ended);
    if (!next.feed_byte(b)) continue;
    mark_ids(w, edge.second);
    descend(w, edge.second, next, depth + 1);
  }
}

// Walks the subtree below `node` from grammar state `g` with the walk that suits the state.
template <class G>
void descend(Walk& w, int32_t node, const G& g, int32_t depth) {
  if (g.in_string_content()) {
    std::string saved;
    saved.swap(w.pending);
    walk_string(w, node, g, depth);
    w.pending.swap(saved);
  } else if (g.in_number()) {
    std::string saved(g.number_text());
    saved.swap(w.number);
    walk_number(w, node, g, w.number.size(), depth);
    w.number.swap(saved);
  } else {
    walk(w, node, g, depth);
  }
}

// The longest piece the walk may take: agent.ts:171 keeps the output within 64 KiB; 0 when no piece
// fits.
int32_t walk_limit(const needle_vocab& v, int64_t output_bytes) {
  const int64_t room = 65536 - output_bytes;
  return room <= 0 ? 0 : (int32_t)std::min<int64_t>(room, v.trie.max_len);
}

// mark[id] = 1 for each id whose piece the grammar accepts; `mark` is resized to the vocabulary.
void mark_allowed(const needle_grammar& g, const needle_vocab& v, int64_t output_bytes, std::vector<uint8_t>& mark) {
  mark.assign(v.size, 0);
  const int32_t limit = walk_limit(v, output_bytes);
  if (limit == 0) return;
  Walk w{v.trie, limit, mark, {}, {}};
  if (g.schema) descend(w, 0, *g.schema, 0);
  else descend(w, 0, *g.tools, 0);
}

// Ascending ids whose piece the grammar accepts; `mark` is scratch of the vocabulary's size.
void allowed(const needle_grammar& g, const needle_vocab& v, int64_t output_bytes, std::vector<uint8_t>& mark,
             std::vector<uint32_t>& out) {
  out.clear();
  mark_allowed(g, v, output_bytes, mark);
  for (int32_t id = 0; id < v.size; id++)
    if (mark[id]) out.push_back((uint32_t)id);
}

std::string grammar_key(const needle_grammar& g, int32_t limit) {
  std::string k;
  key_int(k, limit);
  if (limit > 0) {
    if (g.schema) g.schema->state_key(k);
    else g.tools->state_key(k);
  }
  return k;
}

bool same_template(const needle_grammar& g, const needle_mask_cache& c) {
  if (g.schema) return g.schema->template_id() == c.template_id;
  return g.tools->template_id() == c.template_id && g.tools->maximum_calls() == c.maximum_calls;
}

void lru_unlink(needle_mask_cache& c, int32_t s) {
  if (c.prev[s] >= 0) c.next[c.prev[s]] = c.next[s];
  else c.head = c.next[s];
  if (c.next[s] >= 0) c.prev[c.next[s]] = c.prev[s];
  else c.tail = c.prev[s];
  c.prev[s] = c.next[s] = -1;
}

void lru_front(needle_mask_cache& c, int32_t s) {
  if (c.head == s) return;
  if (c.prev[s] >= 0) lru_unlink(c, s);  // linked (every linked slot but the head has a prev)
  c.next[s] = c.head;
  if (c.head >= 0) c.prev[c.head] = s;
  c.head = s;
  if (c.tail < 0) c.tail = s;
}

// Empties slots whose key was taken but whose mask was not written.
void drop_slots(needle_mask_cache& c, const std::vector<int32_t>& slots) {
  for (int32_t s : slots) {
    c.index.erase(c.key[s]);
    c.key[s].clear();
    c.count[s] = 0;
  }
}

}  // namespace

extern "C" {

int needle_mask_cache_open(const needle_grammar* template_grammar, const needle_vocab* vocab, int32_t capacity,
                           needle_mask_cache** out) {
  if (!template_grammar || !vocab || !out) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  if (capacity < 1) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "mask cache capacity must be positive");
  auto c = std::make_unique<needle_mask_cache>();
  c->keep = std::make_unique<needle_grammar>();
  if (template_grammar->schema) {
    c->keep->schema = std::make_unique<SchemaGrammar>(*template_grammar->schema);
    c->template_id = c->keep->schema->template_id();
  } else {
    c->keep->tools = std::make_unique<ToolGrammar>(*template_grammar->tools);
    c->template_id = c->keep->tools->template_id();
    c->maximum_calls = c->keep->tools->maximum_calls();
  }
  c->vocab = vocab;
  c->capacity = capacity;
  c->words = (vocab->size + 31) / 32;
  c->table.assign((size_t)capacity * c->words, 0u);
  c->count.assign(capacity, 0);
  c->key.assign(capacity, std::string());
  c->prev.assign(capacity, -1);
  c->next.assign(capacity, -1);
  c->used_in.assign(capacity, 0);
  for (int32_t s = 0; s < capacity; s++) lru_front(*c, s);  // slot 0 ends last: taken first
  *out = c.release();
  return NEEDLE_OK;
}

void needle_mask_cache_free(needle_mask_cache* cache) { delete cache; }

int needle_mask_cache_table(const needle_mask_cache* cache, const uint32_t** table, int32_t* words) {
  if (!cache || !table || !words) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  *table = cache->table.data();
  *words = cache->words;
  return NEEDLE_OK;
}

int needle_mask_cache_stats(const needle_mask_cache* cache, int64_t* hits, int64_t* misses, int64_t* evictions) {
  if (!cache || !hits || !misses || !evictions) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  *hits = cache->hits;
  *misses = cache->misses;
  *evictions = cache->evictions;
  return NEEDLE_OK;
}

int needle_mask_cache_lookup(needle_mask_cache* cache, const needle_grammar* const* grammars,
                             const int64_t* output_bytes, int32_t n, int32_t threads, int32_t* slots,
                             int32_t* counts, int32_t* filled, int32_t* n_filled) {
  if (!cache || !n_filled || n < 0 || (n > 0 && (!grammars || !output_bytes || !slots || !counts || !filled)))
    return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  needle_mask_cache& c = *cache;
  *n_filled = 0;
  for (int32_t k = 0; k < n; k++)
    if (grammars[k] && !same_template(*grammars[k], c))
      return fail(NEEDLE_INVALID_TOOL_SCHEMA, "grammar is not a clone of the mask cache's template");
  std::vector<int32_t> fill_slot, fill_from;
  const uint64_t lookup = ++c.lookups;
  try {
    for (int32_t k = 0; k < n; k++) {
      if (!grammars[k]) {
        slots[k] = -1;
        counts[k] = 0;
        continue;
      }
      std::string key = grammar_key(*grammars[k], walk_limit(*c.vocab, output_bytes[k]));
      int32_t slot;
      if (auto it = c.index.find(key); it != c.index.end()) {
        slot = it->second;
        c.hits++;
      } else {
        slot = c.tail;
        if (slot < 0 || c.used_in[slot] == lookup) {
          drop_slots(c, fill_slot);
          return fail(NEEDLE_INVALID_TOOL_SCHEMA, "mask cache capacity is below the distinct states of one lookup");
        }
        if (!c.key[slot].empty()) {
          c.index.erase(c.key[slot]);
          c.evictions++;
        }
        c.key[slot] = key;
        c.index.emplace(std::move(key), slot);
        c.misses++;
        fill_slot.push_back(slot);
        fill_from.push_back(k);
      }
      c.used_in[slot] = lookup;
      lru_front(c, slot);
      slots[k] = slot;
    }
  } catch (const std::exception& e) {
    drop_slots(c, fill_slot);
    return fail(NEEDLE_INVALID_TOOL_SCHEMA, e.what());
  }
  std::atomic<int> next{0};
  std::atomic<bool> bad{false};
  auto work = [&]() {
    std::vector<uint8_t> mark;
    for (int j; (j = next.fetch_add(1)) < (int)fill_slot.size();) {
      try {
        const int32_t k = fill_from[j], slot = fill_slot[j];
        mark_allowed(*grammars[k], *c.vocab, output_bytes[k], mark);
        uint32_t* w = c.table.data() + (size_t)slot * c.words;
        std::fill(w, w + c.words, 0u);
        int32_t set = 0;
        for (int32_t id = 0; id < c.vocab->size; id++)
          if (mark[id]) {
            w[id >> 5] |= 1u << (id & 31);
            set++;
          }
        c.count[slot] = set;
      } catch (const std::exception&) {
        bad.store(true);
      }
    }
  };
  const int t = std::max(1, std::min<int>(threads, (int)fill_slot.size()));
  std::vector<std::thread> pool;
  for (int k = 1; k < t; k++) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
  if (bad.load()) {
    drop_slots(c, fill_slot);
    return fail(NEEDLE_INVALID_TOOL_SCHEMA, "grammar enumeration failed (schema error)");
  }
  for (int32_t k = 0; k < n; k++) counts[k] = slots[k] < 0 ? 0 : c.count[slots[k]];
  for (size_t j = 0; j < fill_slot.size(); j++) filled[j] = fill_slot[j];
  *n_filled = (int32_t)fill_slot.size();
  return NEEDLE_OK;
}

int needle_grammar_tools(const char* tools_json, int32_t maximum_calls, needle_grammar** out) {
  if (!tools_json || !out) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  try {
    Parser p{std::string(tools_json)};
    const Json doc = p.document();
    auto tools = std::make_shared<const std::vector<Tool>>(normalize_tools(doc));
    auto g = std::make_unique<needle_grammar>();
    g->tools = std::make_unique<ToolGrammar>(tools, maximum_calls);
    *out = g.release();
    return NEEDLE_OK;
  } catch (const std::exception& e) {
    return fail(NEEDLE_INVALID_TOOL_SCHEMA, e.what());
  }
}

int needle_grammar_schema(const char* schema_json, needle_grammar** out) {
  if (!schema_json || !out) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  try {
    Parser p{std::string(schema_json)};
    auto root = std::make_shared<const Json>(p.document());
    auto g = std::make_unique<needle_grammar>();
    g->schema = std::make_unique<SchemaGrammar>(root);
    *out = g.release();
    return NEEDLE_OK;
  } catch (const std::exception& e) {
    return fail(NEEDLE_INVALID_TOOL_SCHEMA, e.what());
  }
}

int needle_grammar_clone(const needle_grammar* g, needle_grammar** out) {
  if (!g || !out) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  auto c = std::make_unique<needle_grammar>();
  if (g->schema) c->schema = std::make_unique<SchemaGrammar>(*g->schema);
  else c->tools = std::make_unique<ToolGrammar>(*g->tools);
  *out = c.release();
  return NEEDLE_OK;
}

void needle_grammar_free(needle_grammar* g) { delete g; }

int needle_grammar_feed(needle_grammar* g, const uint8_t* bytes, int32_t n, int32_t* accepted) {
  if (!g || !accepted || (n > 0 && !bytes)) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  try {
    int ok = 1;
    for (int32_t k = 0; k < n && ok; k++) ok = g->feed_byte(bytes[k]) ? 1 : 0;
    *accepted = ok;
    return NEEDLE_OK;
  } catch (const std::exception& e) {
    return fail(NEEDLE_INVALID_TOOL_SCHEMA, e.what());
  }
}

int needle_grammar_complete(const needle_grammar* g, int32_t* complete) {
  if (!g || !complete) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  *complete = g->complete() ? 1 : 0;
  return NEEDLE_OK;
}

int needle_grammar_result(const needle_grammar* g, char* buf, int32_t capacity, int32_t* length) {
  if (!g || !length) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  std::string text;
  if (g->schema) {
    const Json* v = g->schema->value();
    text = v ? stringify(*v) : std::string();
  } else {
    Json arr;
    arr.kind = Json::Array;
    for (const auto& c : g->tools->calls()) {
      Json call;
      call.kind = Json::Object;
      Json name;
      name.kind = Json::String;
      name.str = c.name;
      call.set("name", name);
      call.set("arguments", c.arguments);
      arr.arr.push_back(std::move(call));
    }
    text = stringify(arr);
  }
  *length = (int32_t)text.size();
  if (buf && capacity > 0) {
    const int32_t n = std::min<int32_t>(capacity - 1, (int32_t)text.size());
    memcpy(buf, text.data(), n);
    buf[n] = 0;
  }
  return NEEDLE_OK;
}

int needle_vocab_open(const uint8_t* bytes, const int32_t* offsets, int32_t n, needle_vocab** out) {
  if (!out || n < 0 || (n > 0 && (!bytes || !offsets))) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  auto v = std::make_unique<needle_vocab>();
  v->size = n;
  for (int32_t id = 0; id < n; id++) {
    const int32_t len = offsets[id + 1] - offsets[id];
    if (len < 0) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "offsets must not decrease");
    if (len > 0) v->trie.insert(bytes + offsets[id], len, (uint32_t)id);
  }
  v->trie.index_string_content(n);
  *out = v.release();
  return NEEDLE_OK;
}

void needle_vocab_free(needle_vocab* v) { delete v; }

int needle_grammar_allowed(const needle_grammar* g, const needle_vocab* v, int64_t output_bytes, uint32_t* ids,
                           int32_t capacity, int32_t* count) {
  if (!g || !v || !count) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  try {
    std::vector<uint8_t> mark;
    std::vector<uint32_t> out;
    allowed(*g, *v, output_bytes, mark, out);
    *count = (int32_t)out.size();
    if ((int32_t)out.size() > capacity) return fail(NEEDLE_INVALID_TOOL_SCHEMA, "id buffer too small");
    if (!out.empty()) memcpy(ids, out.data(), out.size() * sizeof(uint32_t));
    return NEEDLE_OK;
  } catch (const std::exception& e) {
    return fail(NEEDLE_INVALID_TOOL_SCHEMA, e.what());
  }
}

int needle_grammar_allowed_batch(const needle_grammar* const* grammars, const int64_t* output_bytes, int32_t n,
                                 const needle_vocab* v, int32_t threads, uint32_t* ids, int32_t capacity_each,
                                 int32_t* counts) {
  if ((n > 0 && (!grammars || !output_bytes || !ids || !counts)) || !v)
    return fail(NEEDLE_INVALID_TOOL_SCHEMA, "null argument");
  std::atomic<int> next{0};
  std::atomic<int> status{NEEDLE_OK};
  std::string message;
  auto work = [&]() {
    std::vector<uint8_t> mark;
    std::vector<uint32_t> out;
    for (int k; (k = next.fetch_add(1)) < n;) {
      try {
        if (!grammars[k]) {
          counts[k] = 0;
          continue;
        }
        allowed(*grammars[k], *v, output_bytes[k], mark, out);
        counts[k] = (int32_t)out.size();
        if ((int32_t)out.size() > capacity_each) {
          status.store(NEEDLE_INVALID_TOOL_SCHEMA);
          continue;
        }
        if (!out.empty()) memcpy(ids + (int64_t)k * capacity_each, out.data(), out.size() * sizeof(uint32_t));
      } catch (const std::exception&) {
        status.store(NEEDLE_INVALID_TOOL_SCHEMA);
      }
    }
  };
  const int t = std::max(1, std::min<int>(threads, n));
  std::vector<std::thread> pool;
  for (int k = 1; k < t; k++) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
  if (status.load() != NEEDLE_OK) return fail(status.load(), "grammar enumeration failed (schema error or id buffer too small)");
  return NEEDLE_OK;
}

}  // extern "C"
