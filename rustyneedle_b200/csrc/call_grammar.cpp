// call_grammar.cpp — compiles a tool-call grammar into the byte automaton the
// device grammar kernels run (grammar.cu).
//
// The reference builds a CallGrammar from the tools JSON
// (CallGrammar::from_tools_json, crates/grammar/src/call.rs:16-61; the schema
// compiler is schema.rs:29-141) and, inside every constrained step, clones the
// live CallMachine once per vocabulary piece and steps it byte by byte
// (TokenBytes::allowed, mask.rs:28-42). Here the machine's reachable states are
// explored once on the host, breadth first from CallMachine::start: every
// state is a value (its stage, nested machines and counters) with a canonical
// key, and each of the 256 bytes either moves it to another state, rejects it
// leaving it as it was, or rejects it and still changes it (an array item or
// an object value that can finish hands the byte to the next stage, which
// rejects it: machine.rs:357-364, 444-451, 495-505). The table entry is the
// next state, 0, or the changed state with the top bit set.
//
// A key must decide every future step, and the state space must stay finite,
// so counters that matter only against a bound are saturated:
//   text     the character count above min_chars when there is no max_chars
//            (only `count < min_chars` is asked, machine.rs:113-119)
//   number   without bounds, only the text's shape (length, sign, the integer
//            part empty / "0" / other, the dot, an empty fraction) is asked;
//            with bounds, an integer part whose magnitude is at least
//            2·max|bound| + 2 decides every comparison the same way, and a
//            text with a fraction is its length and whether it can finish,
//            unless some bound lies between its extensions' values (then it
//            is kept exactly: one or two such texts per length and bound)
//   calls    only whether a call has completed (AfterOpen's `completed == 0`)
//   done     a finished text, array or object rejects every byte
// Grammars whose exploration passes `max_states` (long arrays of nested
// objects, for instance) fail with NB_ERR_UNSUPPORTED.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <limits>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "needle_b200.h"

namespace {

struct GrammarError : std::runtime_error {
  nb_status status;
  GrammarError(nb_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

// ------------------------------------------------------------------ JSON
// A JSON value as serde_json holds it (with preserve_order: objects keep their
// key order). Numbers without '.', 'e' or 'E' that fit 64 bits are integers.
struct Json {
  enum Kind { Null, Bool, Int, Uint, Float, String, Array, Object } kind = Null;
  bool b = false;
  int64_t i = 0;
  uint64_t u = 0;
  double f = 0.0;
  std::string s;
  std::vector<Json> items;
  std::vector<std::pair<std::string, Json>> fields;

  const Json* get(const std::string& key) const {
    if (kind != Object) return nullptr;
    for (const auto& kv : fields)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  std::optional<double> as_f64() const {
    if (kind == Int) return (double)i;
    if (kind == Uint) return (double)u;
    if (kind == Float) return f;
    return std::nullopt;
  }
  std::optional<uint64_t> as_u64() const {
    if (kind == Uint) return u;
    if (kind == Int && i >= 0) return (uint64_t)i;
    return std::nullopt;
  }
  const std::string* as_str() const { return kind == String ? &s : nullptr; }
};

class Parser {
 public:
  explicit Parser(const std::string& text) : t_(text) {}
  Json parse() {
    Json v = value(0);
    ws();
    if (p_ != t_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& t_;
  size_t p_ = 0;
  [[noreturn]] void fail(const std::string& why) {
    throw GrammarError(NB_ERR_ARGUMENT, "tools JSON: " + why + " at byte " + std::to_string(p_));
  }
  void ws() {
    while (p_ < t_.size() && (t_[p_] == ' ' || t_[p_] == '\t' || t_[p_] == '\n' || t_[p_] == '\r')) ++p_;
  }
  bool eat(char c) {
    ws();
    if (p_ < t_.size() && t_[p_] == c) {
      ++p_;
      return true;
    }
    return false;
  }
  void expect(char c) {
    if (!eat(c)) fail(std::string("expected '") + c + "'");
  }
  Json value(int depth) {
    if (depth > 256) fail("nesting too deep");
    ws();
    if (p_ >= t_.size()) fail("unexpected end");
    const char c = t_[p_];
    Json v;
    if (c == '{') {
      ++p_;
      v.kind = Json::Object;
      if (eat('}')) return v;
      do {
        ws();
        if (p_ >= t_.size() || t_[p_] != '"') fail("expected a key");
        std::string key = string();
        expect(':');
        Json item = value(depth + 1);
        bool replaced = false;  // a repeated key keeps its first position and the last value
        for (auto& kv : v.fields)
          if (kv.first == key) {
            kv.second = std::move(item);
            replaced = true;
            break;
          }
        if (!replaced) v.fields.emplace_back(std::move(key), std::move(item));
      } while (eat(','));
      expect('}');
    } else if (c == '[') {
      ++p_;
      v.kind = Json::Array;
      if (eat(']')) return v;
      do v.items.push_back(value(depth + 1));
      while (eat(','));
      expect(']');
    } else if (c == '"') {
      v.kind = Json::String;
      v.s = string();
    } else if (t_.compare(p_, 4, "true") == 0) {
      p_ += 4;
      v.kind = Json::Bool;
      v.b = true;
    } else if (t_.compare(p_, 5, "false") == 0) {
      p_ += 5;
      v.kind = Json::Bool;
    } else if (t_.compare(p_, 4, "null") == 0) {
      p_ += 4;
    } else {
      v = number();
    }
    return v;
  }
  static void utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
      out += (char)cp;
    } else if (cp < 0x800) {
      out += (char)(0xC0 | (cp >> 6));
      out += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
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
  uint32_t hex4() {
    if (p_ + 4 > t_.size()) fail("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char h = t_[p_++];
      v <<= 4;
      if (h >= '0' && h <= '9') v |= (uint32_t)(h - '0');
      else if (h >= 'a' && h <= 'f') v |= (uint32_t)(h - 'a' + 10);
      else if (h >= 'A' && h <= 'F') v |= (uint32_t)(h - 'A' + 10);
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string() {
    ++p_;  // the opening quote
    std::string out;
    while (true) {
      if (p_ >= t_.size()) fail("unterminated string");
      const unsigned char c = (unsigned char)t_[p_++];
      if (c == '"') break;
      if (c < 0x20) fail("control character in a string");
      if (c != '\\') {
        out += (char)c;
        continue;
      }
      if (p_ >= t_.size()) fail("unterminated escape");
      const char e = t_[p_++];
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
          if (cp >= 0xD800 && cp < 0xDC00) {
            if (p_ + 6 > t_.size() || t_[p_] != '\\' || t_[p_ + 1] != 'u') fail("lone surrogate");
            p_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            fail("lone surrogate");
          }
          utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return out;
  }
  Json number() {
    const size_t start = p_;
    if (p_ < t_.size() && t_[p_] == '-') ++p_;
    bool integral = true;
    auto digits = [&] {
      const size_t d = p_;
      while (p_ < t_.size() && t_[p_] >= '0' && t_[p_] <= '9') ++p_;
      return p_ - d;
    };
    if (digits() == 0) fail("bad value");
    if (p_ < t_.size() && t_[p_] == '.') {
      ++p_;
      integral = false;
      if (digits() == 0) fail("bad number");
    }
    if (p_ < t_.size() && (t_[p_] == 'e' || t_[p_] == 'E')) {
      ++p_;
      integral = false;
      if (p_ < t_.size() && (t_[p_] == '+' || t_[p_] == '-')) ++p_;
      if (digits() == 0) fail("bad exponent");
    }
    const std::string text = t_.substr(start, p_ - start);
    Json v;
    if (integral) {
      errno = 0;
      if (text[0] == '-') {
        char* end = nullptr;
        const long long x = std::strtoll(text.c_str(), &end, 10);
        if (errno == 0) {
          v.kind = Json::Int;
          v.i = x;
          return v;
        }
      } else {
        char* end = nullptr;
        const unsigned long long x = std::strtoull(text.c_str(), &end, 10);
        if (errno == 0) {
          v.kind = Json::Uint;
          v.u = x;
          return v;
        }
      }
    }
    v.kind = Json::Float;
    v.f = std::strtod(text.c_str(), nullptr);
    return v;
  }
};

// serde_json::to_string of a value: compact, strings escaped as serde_json
// escapes them, floats in the shortest round-trip form laid out as ryu does
// (decimal notation for exponents in [-5, 16), otherwise d.ddde±x).
std::string quote(const std::string& s) {
  std::string out = "\"";
  for (unsigned char c : s) {
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
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          out += buf;
        } else {
          out += (char)c;
        }
    }
  }
  return out + "\"";
}

std::string shortest_float(double x) {
  if (!std::isfinite(x)) return "null";
  if (x == 0.0) return std::signbit(x) ? "-0.0" : "0.0";
  char buf[40];
  int prec = 1;
  for (; prec <= 17; ++prec) {
    std::snprintf(buf, sizeof buf, "%.*e", prec - 1, x);
    if (std::strtod(buf, nullptr) == x) break;
  }
  // buf = [-]d.ddde±XX: the digits and the decimal exponent
  std::string s(buf);
  const bool neg = s[0] == '-';
  if (neg) s.erase(0, 1);
  const size_t epos = s.find('e');
  const int exp10 = std::atoi(s.c_str() + epos + 1);
  std::string digits = s.substr(0, epos);
  digits.erase(std::remove(digits.begin(), digits.end(), '.'), digits.end());
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  const int point = exp10 + 1;  // value = 0.digits × 10^point
  const int n = (int)digits.size();
  std::string out = neg ? "-" : "";
  if (point > 0 && point <= 16) {
    if (n <= point) return out + digits + std::string(point - n, '0') + ".0";
    return out + digits.substr(0, point) + "." + digits.substr(point);
  }
  if (point > -5 && point <= 0) return out + "0." + std::string(-point, '0') + digits;
  out += digits.substr(0, 1);
  if (n > 1) out += "." + digits.substr(1);
  return out + "e" + std::to_string(point - 1);
}

std::string to_text(const Json& v) {
  switch (v.kind) {
    case Json::Null: return "null";
    case Json::Bool: return v.b ? "true" : "false";
    case Json::Int: return std::to_string(v.i);
    case Json::Uint: return std::to_string(v.u);
    case Json::Float: return shortest_float(v.f);
    case Json::String: return quote(v.s);
    case Json::Array: {
      std::string out = "[";
      for (size_t k = 0; k < v.items.size(); ++k) out += (k ? "," : "") + to_text(v.items[k]);
      return out + "]";
    }
    case Json::Object: {
      std::string out = "{";
      for (size_t k = 0; k < v.fields.size(); ++k) out += (k ? "," : "") + quote(v.fields[k].first) + ":" + to_text(v.fields[k].second);
      return out + "}";
    }
  }
  return "null";
}

// ---------------------------------------------------------------- schema
constexpr int MAX_SCHEMA_DEPTH = 12;   // schema.rs:5
constexpr size_t MAX_ARRAY_ITEMS = 64;  // schema.rs:6-7
constexpr size_t MAX_NUMBER_CHARS = 20;  // machine.rs:5

struct Node;
using NodeP = std::shared_ptr<const Node>;
struct Property {
  std::string name;
  NodeP node;
  bool required;
};
struct Node {
  enum Kind { Text, Integer, Number, Literals, Array, Object, Choice } kind = Text;
  uint32_t id = 0;  // distinct per node of a grammar: machines of different nodes never share a key
  size_t min_chars = 0;
  std::optional<size_t> max_chars;
  std::optional<double> lo, hi;  // number bounds (integer bounds converted as `i64 as f64`)
  std::vector<std::string> options;  // Literals (Boolean and Null become Literals, machine.rs:25-26)
  NodeP items;
  size_t min_items = 0, max_items = MAX_ARRAY_ITEMS;
  std::vector<Property> properties;
  std::vector<std::string> keys;  // "\"name\"" per property (machine.rs:413-414)
  std::vector<NodeP> alternatives;
};

int64_t saturate_i64(double x) {
  if (std::isnan(x)) return 0;
  if (x >= 9.223372036854775807e18) return std::numeric_limits<int64_t>::max();
  if (x <= -9.223372036854775808e18) return std::numeric_limits<int64_t>::min();
  return (int64_t)x;
}

const Json* resolve(const Json* schema, const Json& root) {
  const Json* current = schema;
  for (int k = 0; k < MAX_SCHEMA_DEPTH; ++k) {
    const Json* ref = current->get("$ref");
    if (!ref || !ref->as_str() || ref->s.compare(0, 2, "#/") != 0) return current;
    const Json* target = &root;
    size_t at = 2;
    while (true) {
      const size_t slash = ref->s.find('/', at);
      const std::string part = ref->s.substr(at, slash == std::string::npos ? std::string::npos : slash - at);
      target = target->get(part);
      if (!target) return current;
      if (slash == std::string::npos) break;
      at = slash + 1;
    }
    current = target;
  }
  return current;
}

thread_local uint32_t t_next_node = 0;

NodeP make_text(size_t min_chars, std::optional<size_t> max_chars) {
  auto n = std::make_shared<Node>();
  n->id = ++t_next_node;
  n->kind = Node::Text;
  n->min_chars = min_chars;
  n->max_chars = max_chars;
  return n;
}

NodeP make_literals(std::vector<std::string> options) {
  auto n = std::make_shared<Node>();
  n->id = ++t_next_node;
  n->kind = Node::Literals;
  n->options = std::move(options);
  return n;
}

NodeP compile(const Json* schema, const Json& root, int depth) {
  schema = resolve(schema, root);
  if (depth > MAX_SCHEMA_DEPTH) return make_text(0, std::nullopt);
  if (const Json* c = schema->get("const")) return make_literals({to_text(*c)});
  if (const Json* e = schema->get("enum"); e && e->kind == Json::Array) {
    std::vector<std::string> options;
    for (const Json& v : e->items) options.push_back(to_text(v));
    return make_literals(std::move(options));
  }
  for (const char* key : {"anyOf", "oneOf"}) {
    const Json* variants = schema->get(key);
    if (variants && variants->kind == Json::Array) {
      std::vector<NodeP> nodes;
      for (const Json& v : variants->items) nodes.push_back(compile(&v, root, depth + 1));
      if (nodes.size() == 1) return nodes[0];
      auto n = std::make_shared<Node>();
      n->id = ++t_next_node;
      n->kind = Node::Choice;
      n->alternatives = std::move(nodes);
      return n;
    }
  }
  const Json* type = schema->get("type");
  if (type && type->kind == Json::Array) {
    auto n = std::make_shared<Node>();
    n->id = ++t_next_node;
    n->kind = Node::Choice;
    for (const Json& kind : type->items) {
      if (!kind.as_str()) continue;
      Json single = *schema;
      for (auto& kv : single.fields)
        if (kv.first == "type") kv.second = kind;
      n->alternatives.push_back(compile(&single, root, depth + 1));
    }
    return n;
  }
  const std::string kind = type && type->as_str() ? type->s : "string";
  auto num = [&](const char* key) -> std::optional<double> {
    const Json* v = schema->get(key);
    return v ? v->as_f64() : std::nullopt;
  };
  auto count = [&](const char* key) -> std::optional<uint64_t> {
    const Json* v = schema->get(key);
    return v ? v->as_u64() : std::nullopt;
  };
  auto n = std::make_shared<Node>();
  n->id = ++t_next_node;
  if (kind == "integer") {
    // schema.rs:97-104: inclusive bounds rounded inward, exclusive ones moved one past, the tighter of each pair
    std::optional<int64_t> lower, upper, lx, ux;
    if (auto v = num("minimum")) lower = saturate_i64(std::ceil(*v));
    if (auto v = num("maximum")) upper = saturate_i64(std::floor(*v));
    // `floor(v) as i64 + 1` (and `- 1`): kept at the i64 limits instead of wrapping
    if (auto v = num("exclusiveMinimum")) {
      const int64_t x = saturate_i64(std::floor(*v));
      lx = x == std::numeric_limits<int64_t>::max() ? x : x + 1;
    }
    if (auto v = num("exclusiveMaximum")) {
      const int64_t x = saturate_i64(std::ceil(*v));
      ux = x == std::numeric_limits<int64_t>::min() ? x : x - 1;
    }
    std::optional<int64_t> mn = lower && lx ? std::max(*lower, *lx) : (lower ? lower : lx);
    std::optional<int64_t> mx = upper && ux ? std::min(*upper, *ux) : (upper ? upper : ux);
    n->kind = Node::Integer;
    if (mn) n->lo = (double)*mn;
    if (mx) n->hi = (double)*mx;
  } else if (kind == "number") {
    n->kind = Node::Number;
    n->lo = num("minimum") ? num("minimum") : num("exclusiveMinimum");
    n->hi = num("maximum") ? num("maximum") : num("exclusiveMaximum");
  } else if (kind == "boolean") {
    return make_literals({"true", "false"});
  } else if (kind == "null") {
    return make_literals({"null"});
  } else if (kind == "array") {
    n->kind = Node::Array;
    const Json* items = schema->get("items");
    n->items = items ? compile(items, root, depth + 1) : make_text(0, std::nullopt);
    n->min_items = (size_t)count("minItems").value_or(0);
    if (auto mx = count("maxItems")) n->max_items = (size_t)std::min<uint64_t>(*mx, MAX_ARRAY_ITEMS);
  } else if (kind == "object") {
    n->kind = Node::Object;
    std::vector<std::string> required;
    if (const Json* r = schema->get("required"); r && r->kind == Json::Array)
      for (const Json& v : r->items)
        if (v.as_str()) required.push_back(v.s);
    if (const Json* props = schema->get("properties"); props && props->kind == Json::Object)
      for (const auto& kv : props->fields) {
        const bool req = std::find(required.begin(), required.end(), kv.first) != required.end();
        n->properties.push_back({kv.first, compile(&kv.second, root, depth + 1), req});
        n->keys.push_back("\"" + kv.first + "\"");
      }
  } else {
    auto mx = count("maxLength");
    return make_text((size_t)count("minLength").value_or(0), mx ? std::optional<size_t>((size_t)*mx) : std::nullopt);
  }
  return n;
}

// --------------------------------------------------------------- machines
// One machine value; `kids` holds the nested machine of an array item or an
// object value (0 or 1) and the alternatives of a choice.
struct M {
  const Node* node = nullptr;
  // text
  size_t count = 0;
  bool opened = false, closed = false;
  uint8_t escape = 0, unicode_left = 0, continuation = 0;  // escape: 0 none, 1 slash, 2 \u
  // number
  std::string text;
  // literals (and an object's key literal)
  std::vector<uint32_t> alive;
  size_t position = 0;
  // array / object
  uint8_t stage = 0;
  bool done = false, first = false;
  size_t next = 0, property = 0;
  std::vector<M> kids;
};

enum : uint8_t { A_START, A_AFTER_OPEN, A_ITEM, A_AFTER_ITEM, A_AFTER_COMMA };
enum : uint8_t { O_START, O_BEFORE_KEY, O_KEY, O_COLON, O_VALUE, O_AFTER_VALUE };

M make(const Node* n) {
  M m;
  m.node = n;
  if (n->kind == Node::Literals)
    for (uint32_t i = 0; i < n->options.size(); ++i) m.alive.push_back(i);
  if (n->kind == Node::Choice)
    for (const NodeP& a : n->alternatives) m.kids.push_back(make(a.get()));
  return m;
}

bool literal_step(const std::vector<std::string>& options, std::vector<uint32_t>& alive, size_t& position, uint8_t b) {
  std::vector<uint32_t> survivors;
  for (uint32_t i : alive)
    if (position < options[i].size() && (uint8_t)options[i][position] == b) survivors.push_back(i);
  if (survivors.empty()) return false;
  alive.swap(survivors);
  ++position;
  return true;
}

int literal_chosen(const std::vector<std::string>& options, const std::vector<uint32_t>& alive, size_t position) {
  for (uint32_t i : alive)
    if (options[i].size() == position) return (int)i;
  return -1;
}

bool is_hex(uint8_t b) { return (b >= '0' && b <= '9') || (b >= 'a' && b <= 'f') || (b >= 'A' && b <= 'F'); }

bool text_step(M& m, uint8_t b) {
  const Node& n = *m.node;
  const bool room = !n.max_chars || m.count < *n.max_chars;
  if (m.closed) return false;
  if (!m.opened) return m.opened = b == '"';
  if (m.continuation > 0) {
    if ((b & 0xC0) != 0x80) return false;
    --m.continuation;
    return true;
  }
  if (m.escape == 1) {
    if (b == '"' || b == '\\' || b == '/' || b == 'b' || b == 'f' || b == 'n' || b == 'r' || b == 't') {
      m.escape = 0;
      ++m.count;
      return true;
    }
    if (b == 'u') {
      m.escape = 2;
      m.unicode_left = 4;
      return true;
    }
    return false;
  }
  if (m.escape == 2) {
    if (!is_hex(b)) return false;
    if (m.unicode_left == 1) {
      m.escape = 0;
      m.unicode_left = 0;
      ++m.count;
    } else {
      --m.unicode_left;
    }
    return true;
  }
  if (b == '"') {
    if (m.count < n.min_chars) return false;
    m.closed = true;
    return true;
  }
  if (b == '\\') {
    if (!room) return false;
    m.escape = 1;
    return true;
  }
  if (b <= 0x1F) return false;
  int cont = -1;
  if (b <= 0x7F) cont = 0;
  else if (b >= 0xC2 && b <= 0xDF) cont = 1;
  else if (b >= 0xE0 && b <= 0xEF) cont = 2;
  else if (b >= 0xF0 && b <= 0xF4) cont = 3;
  if (cont < 0 || !room) return false;
  ++m.count;
  m.continuation = (uint8_t)cont;
  return true;
}

struct NumberParts {
  bool negative;
  std::string integer;
  bool has_fraction;
  std::string fraction;
};

NumberParts split(const std::string& text) {
  NumberParts p{};
  p.negative = !text.empty() && text[0] == '-';
  const std::string body = p.negative ? text.substr(1) : text;
  const size_t dot = body.find('.');
  if (dot == std::string::npos) {
    p.integer = body;
  } else {
    p.integer = body.substr(0, dot);
    p.has_fraction = true;
    p.fraction = body.substr(dot + 1);
  }
  return p;
}

bool all_digits(const std::string& s) {
  return std::all_of(s.begin(), s.end(), [](char c) { return c >= '0' && c <= '9'; });
}

bool number_viable(const std::string& text, const Node& n, bool fractional) {
  const NumberParts p = split(text);
  for (size_t k = 0; k < text.size(); ++k) {
    const char c = text[k];
    if (!((c >= '0' && c <= '9') || (c == '-' && k == 0) || (c == '.' && fractional))) return false;
  }
  if (std::count(text.begin(), text.end(), '.') > 1) return false;
  if (p.integer.size() > 1 && p.integer[0] == '0') return false;
  if (p.has_fraction && (p.integer.empty() || !all_digits(p.fraction))) return false;
  if (p.negative && n.lo && *n.lo >= 0.0) return false;
  if (p.integer.empty()) return true;
  const double value = std::strtod(p.integer.c_str(), nullptr);
  const double lower = n.lo ? *n.lo : -INFINITY, upper = n.hi ? *n.hi : INFINITY;
  if (p.has_fraction) {
    const double low = p.negative ? -value - 1.0 : value, high = p.negative ? -value : value + 1.0;
    return high >= lower && low <= upper;
  }
  const size_t remaining = text.size() >= MAX_NUMBER_CHARS ? 0 : MAX_NUMBER_CHARS - text.size();
  double scale = 1.0;
  for (size_t extra = 0; extra <= std::min<size_t>(remaining, 18); ++extra) {
    if (extra > 0) scale *= 10.0;  // 10^extra, exact up to 10^22
    const double low = value * scale;
    const double high = low + scale - 1.0;
    const double span_low = p.negative ? -high : low, span_high = p.negative ? -low : high;
    if (span_high >= lower && span_low <= upper) return true;
    if (fractional && extra == 0) {
      const double fl = p.negative ? -value - 1.0 : value, fh = p.negative ? -value : value + 1.0;
      if (fh >= lower && fl <= upper) return true;
    }
  }
  return false;
}

bool number_step(M& m, uint8_t b) {
  const bool fractional = m.node->kind == Node::Number;
  if (m.text.size() >= MAX_NUMBER_CHARS) return false;
  m.text.push_back((char)b);
  if (number_viable(m.text, *m.node, fractional)) return true;
  m.text.pop_back();
  return false;
}

bool number_can_finish(const M& m) {
  const NumberParts p = split(m.text);
  if (p.integer.empty() || (p.has_fraction && p.fraction.empty())) return false;
  const double value = std::strtod(m.text.c_str(), nullptr);
  return (!m.node->lo || value >= *m.node->lo) && (!m.node->hi || value <= *m.node->hi);
}

bool step(M& m, uint8_t b);
bool can_finish(const M& m);

bool array_begin(M& m, uint8_t b) {
  if (m.count >= m.node->max_items) return false;
  M item = make(m.node->items.get());
  if (!step(item, b)) return false;
  ++m.count;
  m.stage = A_ITEM;
  m.kids.assign(1, std::move(item));
  return true;
}

bool array_step(M& m, uint8_t b) {
  if (m.done) return false;
  switch (m.stage) {
    case A_START:
      if (b != '[') return false;
      m.stage = A_AFTER_OPEN;
      return true;
    case A_AFTER_OPEN:
      if (b == ']' && m.node->min_items == 0) return m.done = true;
      return array_begin(m, b);
    case A_ITEM:
      if (step(m.kids[0], b)) return true;
      if (!can_finish(m.kids[0])) return false;
      m.stage = A_AFTER_ITEM;
      m.kids.clear();
      return array_step(m, b);
    case A_AFTER_ITEM:
      if (b == ',' && m.count < m.node->max_items) {
        m.stage = A_AFTER_COMMA;
        return true;
      }
      if (b == ']' && m.count >= m.node->min_items) return m.done = true;
      return false;
    default:
      return array_begin(m, b);
  }
}

bool object_can_close(const M& m) {
  for (size_t k = m.next; k < m.node->properties.size(); ++k)
    if (m.node->properties[k].required) return false;
  return true;
}

bool object_step(M& m, uint8_t b) {
  const Node& n = *m.node;
  if (m.done) return false;
  switch (m.stage) {
    case O_START:
      if (b != '{') return false;
      m.stage = O_BEFORE_KEY;
      m.first = true;
      return true;
    case O_BEFORE_KEY: {
      if (b == '}' && m.first && object_can_close(m)) return m.done = true;
      std::vector<uint32_t> candidates;
      for (size_t k = m.next; k < n.properties.size(); ++k) {
        candidates.push_back((uint32_t)k);
        if (n.properties[k].required) break;
      }
      if (candidates.empty()) return false;
      size_t position = 0;
      if (!literal_step(n.keys, candidates, position, b)) return false;
      m.stage = O_KEY;
      m.alive = std::move(candidates);
      m.position = position;
      return true;
    }
    case O_KEY: {
      if (literal_step(n.keys, m.alive, m.position, b)) return true;
      const int chosen = literal_chosen(n.keys, m.alive, m.position);
      if (chosen < 0) return false;
      m.stage = O_COLON;
      m.property = (size_t)chosen;
      m.alive.clear();
      m.position = 0;
      return object_step(m, b);
    }
    case O_COLON:
      if (b != ':') return false;
      m.stage = O_VALUE;
      m.kids.clear();
      return true;
    case O_VALUE: {
      if (m.kids.empty()) {
        M fresh = make(n.properties[m.property].node.get());
        if (!step(fresh, b)) return false;
        m.kids.assign(1, std::move(fresh));
        return true;
      }
      if (step(m.kids[0], b)) return true;
      if (!can_finish(m.kids[0])) return false;
      m.next = m.property + 1;
      m.stage = O_AFTER_VALUE;
      m.kids.clear();
      m.property = 0;
      return object_step(m, b);
    }
    default:
      if (b == ',' && m.next < n.properties.size()) {
        m.stage = O_BEFORE_KEY;
        m.first = false;
        return true;
      }
      if (b == '}' && object_can_close(m)) return m.done = true;
      return false;
  }
}

bool step(M& m, uint8_t b) {
  switch (m.node->kind) {
    case Node::Text: return text_step(m, b);
    case Node::Integer:
    case Node::Number: return number_step(m, b);
    case Node::Literals: return literal_step(m.node->options, m.alive, m.position, b);
    case Node::Array: return array_step(m, b);
    case Node::Object: return object_step(m, b);
    case Node::Choice: {
      std::vector<M> survivors;
      for (const M& alt : m.kids) {
        M candidate = alt;
        if (step(candidate, b)) survivors.push_back(std::move(candidate));
      }
      if (survivors.empty()) return false;
      m.kids.swap(survivors);
      return true;
    }
  }
  return false;
}

bool can_finish(const M& m) {
  switch (m.node->kind) {
    case Node::Text: return m.closed;
    case Node::Integer:
    case Node::Number: return number_can_finish(m);
    case Node::Literals: return literal_chosen(m.node->options, m.alive, m.position) >= 0;
    case Node::Array:
    case Node::Object: return m.done;
    case Node::Choice:
      for (const M& alt : m.kids)
        if (can_finish(alt)) return true;
      return false;
  }
  return false;
}

// The canonical key of a machine value (see the file comment).
void put(std::string& k, uint64_t v) {
  do {
    k += (char)(0x80 | (v & 0x7F));
    v >>= 7;
  } while (v);
  k += '.';
}

void number_key(std::string& k, const M& m) {
  const Node& n = *m.node;
  const NumberParts p = split(m.text);
  put(k, m.text.size());
  put(k, p.negative);
  put(k, p.has_fraction);
  put(k, !p.fraction.empty());
  if (!n.lo && !n.hi) {  // shape only
    put(k, p.integer.empty() ? 0 : p.integer == "0" ? 1 : 2);
    return;
  }
  if (p.has_fraction) {
    // Every extension of a text with a fraction is viable while it has room
    // (its integer part decides viability), so it behaves as its can_finish
    // outcomes do. The extensions' values lie between the text's own and the
    // text padded with 9s (parsing is monotone): each bound comparison is
    // either the same for all of them, or the text is one of the few prefixes
    // that follow the bound's decimal expansion and is kept exactly.
    const std::string body = p.integer + "." + p.fraction;
    const double first = std::strtod(body.c_str(), nullptr);
    const double last = m.text.size() < MAX_NUMBER_CHARS
                            ? std::strtod((body + std::string(MAX_NUMBER_CHARS - m.text.size(), '9')).c_str(), nullptr)
                            : first;
    const double low = p.negative ? -last : first, high = p.negative ? -first : last;
    const int above_min = !n.lo ? 1 : low >= *n.lo ? 1 : high < *n.lo ? 0 : 2;
    const int below_max = !n.hi ? 1 : high <= *n.hi ? 1 : low > *n.hi ? 0 : 2;
    if (above_min != 2 && below_max != 2) {
      k += 'F';
      put(k, above_min && below_max);
      return;
    }
  } else if (!p.integer.empty()) {
    const double value = std::strtod(p.integer.c_str(), nullptr);
    double bound = 0.0;
    if (n.lo) bound = std::max(bound, std::fabs(*n.lo));
    if (n.hi) bound = std::max(bound, std::fabs(*n.hi));
    if (value >= 2.0 * bound + 2.0) {  // every comparison decided the same way for every extension
      k += 'S';
      return;
    }
  }
  k += 'X';
  k += m.text;
  k += '.';
}

void key(std::string& k, const M& m) {
  const Node& n = *m.node;
  put(k, n.id);
  switch (n.kind) {
    case Node::Text:
      if (m.closed) {
        k += 'c';
        return;
      }
      k += 't';
      put(k, m.opened);
      put(k, m.escape);
      put(k, m.unicode_left);
      put(k, m.continuation);
      put(k, n.max_chars ? m.count : std::min(m.count, n.min_chars));
      return;
    case Node::Integer:
    case Node::Number:
      k += 'n';
      number_key(k, m);
      return;
    case Node::Literals:
      k += 'l';
      put(k, m.position);
      put(k, m.alive.size());
      for (uint32_t i : m.alive) put(k, i);
      return;
    case Node::Array:
      if (m.done) {
        k += 'D';
        return;
      }
      k += 'a';
      put(k, m.count);
      put(k, m.stage);
      if (m.stage == A_ITEM) key(k, m.kids[0]);
      return;
    case Node::Object:
      if (m.done) {
        k += 'D';
        return;
      }
      k += 'o';
      put(k, m.next);
      put(k, m.stage);
      if (m.stage == O_BEFORE_KEY) put(k, m.first);
      if (m.stage == O_KEY) {
        put(k, m.position);
        put(k, m.alive.size());
        for (uint32_t i : m.alive) put(k, i);
      }
      if (m.stage == O_COLON || m.stage == O_VALUE) put(k, m.property);
      if (m.stage == O_VALUE) {
        put(k, m.kids.size());
        if (!m.kids.empty()) key(k, m.kids[0]);
      }
      return;
    case Node::Choice:
      k += 'h';
      put(k, m.kids.size());
      for (const M& alt : m.kids) key(k, alt);
      return;
  }
}

// -------------------------------------------------------------- the call
const std::string NAME_PREFIX = "{\"name\":\"";         // call.rs:8
const std::string ARGUMENTS_PREFIX = ",\"arguments\":";  // call.rs:9

enum : uint8_t { C_OPEN, C_AFTER_OPEN, C_PREFIX, C_NAME, C_MIDDLE, C_ARGUMENTS, C_CLOSE, C_AFTER_CALL, C_DONE };

struct Grammar {
  std::vector<std::string> names;  // each tool's name and its closing quote (call.rs:43-44)
  std::vector<NodeP> arguments;
  bool allow_empty = true;
  std::vector<uint32_t> permitted;  // the Name stage's options (all tools unless restricted)
};

struct Call {
  uint8_t stage = C_OPEN;
  bool completed = false;  // only `completed == 0` is ever asked (call.rs:101)
  size_t position = 0;
  uint32_t tool = 0;
  std::vector<uint32_t> alive;  // the name literal
  std::vector<M> arguments;     // 0 or 1
};

bool call_step(const Grammar& g, Call& c, uint8_t b) {
  switch (c.stage) {
    case C_OPEN:
      if (b != '[') return false;
      c.stage = C_AFTER_OPEN;
      return true;
    case C_AFTER_OPEN:
      if (b == ']' && g.allow_empty && !c.completed) {
        c.stage = C_DONE;
        return true;
      }
      if (b != (uint8_t)NAME_PREFIX[0]) return false;
      c.stage = C_PREFIX;
      c.position = 1;
      return true;
    case C_PREFIX:
      if (c.position >= NAME_PREFIX.size() || (uint8_t)NAME_PREFIX[c.position] != b) return false;
      if (++c.position == NAME_PREFIX.size()) {
        c.stage = C_NAME;
        c.alive = g.permitted;
        c.position = 0;
      }
      return true;
    case C_NAME: {
      if (!literal_step(g.names, c.alive, c.position, b)) return false;
      const int chosen = literal_chosen(g.names, c.alive, c.position);
      if (chosen >= 0) {
        c.stage = C_MIDDLE;
        c.tool = (uint32_t)chosen;
        c.position = 0;
        c.alive.clear();
      }
      return true;
    }
    case C_MIDDLE:
      if (c.position >= ARGUMENTS_PREFIX.size() || (uint8_t)ARGUMENTS_PREFIX[c.position] != b) return false;
      if (++c.position == ARGUMENTS_PREFIX.size()) {
        c.stage = C_ARGUMENTS;
        c.position = 0;
        c.arguments.assign(1, make(g.arguments[c.tool].get()));
      }
      return true;
    case C_ARGUMENTS:
      if (!step(c.arguments[0], b)) return false;
      if (can_finish(c.arguments[0])) {
        c.stage = C_CLOSE;
        c.arguments.clear();
      }
      return true;
    case C_CLOSE:
      if (b != '}') return false;
      c.completed = true;
      c.stage = C_AFTER_CALL;
      return true;
    case C_AFTER_CALL:
      if (b == ',') {
        c.stage = C_PREFIX;
        c.position = 0;
        return true;
      }
      if (b == ']') {
        c.stage = C_DONE;
        return true;
      }
      return false;
    default:
      return false;
  }
}

std::string call_key(const Call& c) {
  std::string k;
  put(k, c.stage);
  if (c.stage == C_DONE) return k;
  put(k, c.completed);
  put(k, c.position);
  if (c.stage == C_NAME) {
    put(k, c.alive.size());
    for (uint32_t i : c.alive) put(k, i);
  }
  if (c.stage == C_MIDDLE) put(k, c.tool);
  if (c.stage == C_ARGUMENTS) key(k, c.arguments[0]);
  return k;
}

}  // namespace

struct nb_call_grammar {
  std::vector<uint32_t> transitions;  // [states][256]
  std::vector<uint8_t> complete;
  uint32_t start = 1;
};

namespace nbr {
extern thread_local std::string g_error;  // nb_last_error's message (runtime.cu)
}

extern "C" {

nb_status nb_call_grammar_compile(const char* tools_json, int require_call, const uint32_t* permitted, size_t permitted_count,
                                  uint32_t max_states, nb_call_grammar** out) {
  if (!tools_json || !out || (permitted_count && !permitted) || (permitted && !require_call)) return NB_ERR_ARGUMENT;
  *out = nullptr;
  if (max_states == 0 || max_states > NB_AUTOMATON_MAX_STATES) max_states = NB_AUTOMATON_MAX_STATES;
  try {
    const std::string text(tools_json);
    const Json tools = Parser(text).parse();
    Grammar g;
    // tool_specs (call.rs:16-31): every tool (or its "function") with a string name
    if (tools.kind == Json::Array) {
      for (const Json& entry : tools.items) {
        const Json* tool = entry.get("function");
        if (!tool) tool = &entry;
        const Json* name = tool->get("name");
        if (!name || !name->as_str()) continue;
        Json parameters;
        if (const Json* p = tool->get("parameters")) {
          parameters = *p;
        } else {
          parameters.kind = Json::Object;
          Json object;
          object.kind = Json::String;
          object.s = "object";
          Json empty;
          empty.kind = Json::Object;
          parameters.fields = {{"type", object}, {"properties", empty}};
        }
        g.names.push_back(name->s + "\"");
        g.arguments.push_back(compile(&parameters, parameters, 0));
      }
    }
    g.allow_empty = !require_call;
    if (permitted) {
      for (size_t k = 0; k < permitted_count; ++k) {
        if (permitted[k] >= g.names.size())
          throw GrammarError(NB_ERR_ARGUMENT, "permitted tool " + std::to_string(permitted[k]) + " is not among the " +
                                                  std::to_string(g.names.size()) + " tools");
        g.permitted.push_back(permitted[k]);
      }
    } else {
      for (uint32_t k = 0; k < g.names.size(); ++k) g.permitted.push_back(k);
    }

    auto result = std::make_unique<nb_call_grammar>();
    std::unordered_map<std::string, uint32_t> ids;
    std::vector<Call> states(1);  // state 0: no call machine
    std::deque<uint32_t> queue;
    auto intern = [&](Call&& c) -> uint32_t {
      std::string k = call_key(c);
      auto it = ids.find(k);
      if (it != ids.end()) return it->second;
      if (states.size() >= max_states)
        throw GrammarError(NB_ERR_UNSUPPORTED, "the call grammar has more than " + std::to_string(max_states - 1) +
                                                   " machine states; constrain it with host masks");
      const uint32_t id = (uint32_t)states.size();
      ids.emplace(std::move(k), id);
      states.push_back(std::move(c));
      queue.push_back(id);
      return id;
    };
    result->start = intern(Call{});
    result->transitions.assign(256, 0u);
    result->complete.assign(1, 0);
    while (!queue.empty()) {
      const uint32_t s = queue.front();
      queue.pop_front();
      const std::string own = call_key(states[s]);
      uint32_t row[256];
      for (int b = 0; b < 256; ++b) {
        Call c = states[s];
        const bool accepted = call_step(g, c, (uint8_t)b);
        if (accepted) {
          row[b] = intern(std::move(c));
        } else {
          const std::string k = call_key(c);
          row[b] = k == own ? 0u : (0x80000000u | intern(std::move(c)));
        }
      }
      if (result->transitions.size() < (size_t)(s + 1) * 256) result->transitions.resize((size_t)(s + 1) * 256, 0u);
      std::memcpy(&result->transitions[(size_t)s * 256], row, sizeof row);
      if (result->complete.size() < (size_t)s + 1) result->complete.resize((size_t)s + 1, 0);
      result->complete[s] = states[s].stage == C_DONE ? 1 : 0;
    }
    result->transitions.resize(states.size() * 256, 0u);
    result->complete.resize(states.size(), 0);
    *out = result.release();
    return NB_OK;
  } catch (const GrammarError& e) {
    nbr::g_error = e.what();
    return e.status;
  } catch (const std::bad_alloc&) {
    nbr::g_error = "out of host memory compiling the call grammar";
    return NB_ERR_UNSUPPORTED;
  }
}

uint32_t nb_call_grammar_states(const nb_call_grammar* grammar) {
  return grammar ? (uint32_t)grammar->complete.size() : 0;
}

nb_status nb_call_grammar_tables(const nb_call_grammar* grammar, uint32_t* transitions, uint8_t* complete,
                                 uint32_t* start_state) {
  if (!grammar || !transitions || !complete || !start_state) return NB_ERR_ARGUMENT;
  std::memcpy(transitions, grammar->transitions.data(), grammar->transitions.size() * sizeof(uint32_t));
  std::memcpy(complete, grammar->complete.data(), grammar->complete.size());
  *start_state = grammar->start;
  return NB_OK;
}

void nb_call_grammar_release(nb_call_grammar* grammar) { delete grammar; }

}  // extern "C"
