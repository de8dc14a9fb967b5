// Tokeniser and operation splitter for the textual MLIR subset read by the
// B200 target (see mlir_text.h).
#include "mlir_text.h"

#include <cctype>
#include <cstdlib>
#include <sstream>

namespace hxbc {
namespace {

bool id_char(char c) {
  return std::isalnum((unsigned char)c) || c == '_' || c == '$' || c == '.' || c == '-';
}

// Angle-bracketed constructs lexed as one token: their text is kept whole.
bool angle_keyword(const std::string& s) {
  return s == "tensor" || s == "vector" || s == "memref" || s == "affine_map" ||
         s == "dense" || s == "complex" || s == "array" || s == "dense_resource";
}

bool tokenize(const std::string& t, std::vector<Tok>* out, std::string* err) {
  size_t i = 0;
  int line = 1;
  bool bol = true;
  auto push = [&](Tok::Kind k, std::string s) {
    out->push_back(Tok{k, std::move(s), line, bol});
    bol = false;
  };
  while (i < t.size()) {
    const char c = t[i];
    if (c == '\n') {
      ++line;
      bol = true;
      ++i;
      continue;
    }
    if (std::isspace((unsigned char)c)) {
      ++i;
      continue;
    }
    if (c == '/' && i + 1 < t.size() && t[i + 1] == '/') {
      while (i < t.size() && t[i] != '\n') ++i;
      continue;
    }
    if (c == '%') {
      size_t j = i + 1;
      while (j < t.size() && (id_char(t[j]) && t[j] != '.')) ++j;
      // %17#0: a use of result 0 of a multi-result op
      if (j < t.size() && t[j] == '#') {
        size_t k = j + 1;
        while (k < t.size() && std::isdigit((unsigned char)t[k])) ++k;
        if (k > j + 1) j = k;
      }
      push(Tok::kSsa, t.substr(i, j - i));
      i = j;
      continue;
    }
    if (c == '@') {
      size_t j = i + 1;
      if (j < t.size() && t[j] == '"') {  // @"quoted"
        size_t k = t.find('"', j + 1);
        if (k == std::string::npos) break;
        push(Tok::kSym, t.substr(j + 1, k - j - 1));
        i = k + 1;
        continue;
      }
      while (j < t.size() && (id_char(t[j]) && t[j] != '-')) ++j;
      push(Tok::kSym, t.substr(i + 1, j - i - 1));
      i = j;
      continue;
    }
    if (c == '#' || c == '^') {
      size_t j = i + 1;
      while (j < t.size() && id_char(t[j]) && t[j] != '-') ++j;
      // a dialect attribute, #dialect.attr<...>: one token with its body
      if (c == '#' && j < t.size() && t[j] == '<') {
        int depth = 0;
        while (j < t.size()) {
          if (t[j] == '\n') ++line;
          if (t[j] == '<') ++depth;
          if (t[j] == '>' && t[j - 1] != '-' && --depth == 0) {
            ++j;
            break;
          }
          ++j;
        }
      }
      push(c == '#' ? Tok::kHash : Tok::kCaret, t.substr(i, j - i));
      i = j;
      continue;
    }
    if (c == '!') {  // dialect type, e.g. !hal.buffer_view
      size_t j = i + 1;
      while (j < t.size() && id_char(t[j]) && t[j] != '-') ++j;
      if (j < t.size() && t[j] == '<') {
        int depth = 0;
        while (j < t.size()) {
          if (t[j] == '<') ++depth;
          if (t[j] == '>' && --depth == 0) {
            ++j;
            break;
          }
          ++j;
        }
      }
      push(Tok::kBang, t.substr(i, j - i));
      i = j;
      continue;
    }
    if (c == '"') {
      size_t j = i + 1;
      while (j < t.size() && t[j] != '"') {
        if (t[j] == '\\') ++j;
        ++j;
      }
      if (j >= t.size()) {
        *err = "line " + std::to_string(line) + ": unterminated string";
        return false;
      }
      push(Tok::kStr, t.substr(i + 1, j - i - 1));
      i = j + 1;
      continue;
    }
    if (std::isdigit((unsigned char)c) ||
        (c == '-' && i + 1 < t.size() && std::isdigit((unsigned char)t[i + 1]))) {
      size_t j = i + 1;
      if (c == '0' && j < t.size() && (t[j] == 'x' || t[j] == 'X')) {
        j++;
        while (j < t.size() && std::isxdigit((unsigned char)t[j])) ++j;
      } else {
        while (j < t.size() && std::isdigit((unsigned char)t[j])) ++j;
        if (j < t.size() && t[j] == '.') {
          ++j;
          while (j < t.size() && std::isdigit((unsigned char)t[j])) ++j;
        }
        if (j < t.size() && (t[j] == 'e' || t[j] == 'E') && j + 1 < t.size() &&
            (std::isdigit((unsigned char)t[j + 1]) || t[j + 1] == '+' || t[j + 1] == '-')) {
          j += 2;
          while (j < t.size() && std::isdigit((unsigned char)t[j])) ++j;
        }
      }
      push(Tok::kNum, t.substr(i, j - i));
      i = j;
      continue;
    }
    if (std::isalpha((unsigned char)c) || c == '_') {
      size_t j = i + 1;
      while (j < t.size() && id_char(t[j]) && t[j] != '-') ++j;
      std::string word = t.substr(i, j - i);
      if (angle_keyword(word) && j < t.size() && t[j] == '<') {
        int depth = 0;
        size_t k = j;
        while (k < t.size()) {
          if (t[k] == '<') ++depth;
          if (t[k] == '>' && t[k - 1] != '-' && --depth == 0) {
            ++k;
            break;
          }
          if (t[k] == '\n') ++line;
          ++k;
        }
        push(Tok::kAngle, t.substr(i, k - i));
        i = k;
        continue;
      }
      push(Tok::kIdent, word);
      i = j;
      continue;
    }
    if (c == '-' && i + 1 < t.size() && t[i + 1] == '>') {
      push(Tok::kPunct, "->");
      i += 2;
      continue;
    }
    push(Tok::kPunct, std::string(1, c));
    ++i;
  }
  out->push_back(Tok{Tok::kEnd, "", line, true});
  return true;
}

bool is_open(const Tok& t) {
  return t.k == Tok::kPunct && (t.s == "(" || t.s == "[" || t.s == "{");
}
bool is_close(const Tok& t) {
  return t.k == Tok::kPunct && (t.s == ")" || t.s == "]" || t.s == "}");
}
bool is_punct(const Tok& t, const char* s) { return t.k == Tok::kPunct && t.s == s; }

bool dotted(const Tok& t) { return t.k == Tok::kIdent && t.s.find('.') != std::string::npos; }

class Parser {
 public:
  Parser(std::vector<Tok> toks) : t_(std::move(toks)) {}

  bool module(Module* m, std::string* err) {
    err_ = err;
    // top level: aliases, then `module [@name] [attributes {...}] { ... }`
    // or bare functions
    while (cur().k != Tok::kEnd) {
      if (cur().k == Tok::kHash && is_punct(peek(1), "=")) {
        const std::string name = cur().s;
        pos_ += 2;
        m->aliases[name] = cur().s;
        ++pos_;
        continue;
      }
      if (cur().k == Tok::kIdent && (cur().s == "module" || cur().s == "builtin.module")) {
        ++pos_;
        while (cur().k != Tok::kEnd && !is_punct(cur(), "{")) {
          if (cur().k == Tok::kIdent && cur().s == "attributes") {
            ++pos_;
            if (!skip_balanced()) return false;
            continue;
          }
          ++pos_;
        }
        if (!expect("{")) return false;
        if (!module_body(m)) return false;
        if (!expect("}")) return false;
        continue;
      }
      if (cur().k == Tok::kIdent && (cur().s == "func.func" || cur().s == "util.func")) {
        if (!module_body(m)) return false;
        continue;
      }
      return fail(cur(), "unexpected '" + cur().s + "' at module level");
    }
    return true;
  }

 private:
  std::vector<Tok> t_;
  size_t pos_ = 0;
  std::string* err_ = nullptr;

  const Tok& cur() const { return t_[pos_]; }
  const Tok& peek(size_t n) const { return t_[pos_ + n < t_.size() ? pos_ + n : t_.size() - 1]; }

  bool fail(const Tok& at, const std::string& msg) {
    *err_ = "line " + std::to_string(at.line) + ": " + msg;
    return false;
  }
  bool expect(const char* p) {
    if (!is_punct(cur(), p)) return fail(cur(), std::string("expected '") + p + "', got '" + cur().s + "'");
    ++pos_;
    return true;
  }
  // Skips one balanced (...), [...] or {...} starting at the current token.
  bool skip_balanced() {
    if (!is_open(cur())) return fail(cur(), "expected a bracket");
    int depth = 0;
    do {
      if (is_open(cur())) ++depth;
      if (is_close(cur())) --depth;
      if (cur().k == Tok::kEnd) return fail(cur(), "unbalanced brackets");
      ++pos_;
    } while (depth > 0);
    return true;
  }

  bool module_body(Module* m) {
    while (cur().k != Tok::kEnd && !is_punct(cur(), "}")) {
      if (cur().k == Tok::kIdent && (cur().s == "func.func" || cur().s == "util.func")) {
        Func f;
        if (!func(&f)) return false;
        m->funcs.push_back(std::move(f));
        continue;
      }
      if (cur().k == Tok::kHash && is_punct(peek(1), "=")) {
        const std::string name = cur().s;
        pos_ += 2;
        m->aliases[name] = cur().s;
        ++pos_;
        continue;
      }
      // other module-level ops (globals, declarations): skip to the next line
      const int line = cur().line;
      ++pos_;
      while (cur().k != Tok::kEnd && !(cur().bol && cur().line != line)) {
        if (is_open(cur())) {
          if (!skip_balanced()) return false;
        } else {
          ++pos_;
        }
      }
    }
    return true;
  }

  bool func(Func* f) {
    f->line = cur().line;
    ++pos_;  // func.func / util.func
    while (cur().k == Tok::kIdent && (cur().s == "public" || cur().s == "private" ||
                                      cur().s == "nested"))
      ++pos_;
    if (cur().k != Tok::kSym) return fail(cur(), "expected a function symbol");
    f->name = cur().s;
    ++pos_;
    if (!expect("(")) return false;
    while (!is_punct(cur(), ")")) {
      if (cur().k != Tok::kSsa) return fail(cur(), "expected an argument");
      f->arg_names.push_back(cur().s);
      ++pos_;
      if (!expect(":")) return false;
      f->arg_types.push_back(cur().s);
      ++pos_;
      if (is_open(cur()) && is_punct(cur(), "{")) {  // argument attributes
        if (!skip_balanced()) return false;
      }
      if (is_punct(cur(), ",")) ++pos_;
      if (cur().k == Tok::kEnd) return fail(cur(), "unterminated argument list");
    }
    ++pos_;
    if (is_punct(cur(), "->")) {
      ++pos_;
      if (is_punct(cur(), "(")) {
        ++pos_;
        while (!is_punct(cur(), ")")) {
          if (cur().k == Tok::kEnd) return fail(cur(), "unterminated result list");
          if (!is_punct(cur(), ",")) f->result_types.push_back(cur().s);
          ++pos_;
          if (is_punct(cur(), "{") && !skip_balanced()) return false;
        }
        ++pos_;
      } else {
        f->result_types.push_back(cur().s);
        ++pos_;
      }
    }
    if (cur().k == Tok::kIdent && cur().s == "attributes") {
      ++pos_;
      if (!skip_balanced()) return false;
    }
    if (!expect("{")) return false;
    Block b;
    if (!block_ops(&b)) return false;
    f->ops = std::move(b.ops);
    return expect("}");
  }

  // True if the token at the current position starts a new operation.
  bool starts_op() const {
    const Tok& t = cur();
    if (t.k == Tok::kSsa) {
      // %a = ..., %a, %b = ..., %a:2 = ...
      size_t j = pos_ + 1;
      while (j < t_.size() && (is_punct(t_[j], ",") || t_[j].k == Tok::kSsa ||
                               is_punct(t_[j], ":") || t_[j].k == Tok::kNum))
        ++j;
      return j < t_.size() && is_punct(t_[j], "=");
    }
    return dotted(t) || (t.k == Tok::kIdent && t.s == "return");
  }

  bool block_ops(Block* b) {
    while (cur().k != Tok::kEnd && !is_punct(cur(), "}")) {
      if (!starts_op()) return fail(cur(), "expected an operation, got '" + cur().s + "'");
      Op op;
      if (!operation(&op)) return false;
      b->ops.push_back(std::move(op));
    }
    return true;
  }

  bool operation(Op* op) {
    op->line = cur().line;
    if (cur().k == Tok::kSsa) {
      while (true) {
        std::string name = cur().s;
        ++pos_;
        int count = 1;
        if (is_punct(cur(), ":") && peek(1).k == Tok::kNum) {
          count = std::atoi(peek(1).s.c_str());
          pos_ += 2;
        }
        if (count == 1) {
          op->results.push_back(name);
        } else {
          for (int i = 0; i < count; ++i) op->results.push_back(name + "#" + std::to_string(i));
        }
        if (is_punct(cur(), ",")) {
          ++pos_;
          continue;
        }
        break;
      }
      if (!expect("=")) return false;
    }
    if (cur().k != Tok::kIdent) return fail(cur(), "expected an operation name");
    op->name = cur().s;
    ++pos_;
    int depth = 0;
    while (cur().k != Tok::kEnd) {
      const Tok& t = cur();
      if (depth == 0) {
        if (is_punct(t, "}")) break;  // end of the enclosing block
        if (t.bol && t.line != op->line && starts_op()) break;
        if (is_punct(t, "{") && region_follows()) {
          if (!region(op)) return false;
          continue;
        }
      }
      if (is_open(t)) ++depth;
      if (is_close(t)) --depth;
      op->toks.push_back(t);
      ++pos_;
    }
    return true;
  }

  // At a depth-0 '{': a region (block label or operations follow) rather
  // than an attribute dictionary (`key = value`).
  bool region_follows() const {
    const Tok& n = peek(1);
    if (n.k == Tok::kCaret) return true;
    if (is_punct(n, "}")) return false;
    if ((n.k == Tok::kIdent || n.k == Tok::kStr) && is_punct(peek(2), "=")) return false;
    return n.bol;
  }

  bool region(Op* op) {
    ++pos_;  // '{'
    Block b;
    if (cur().k == Tok::kCaret) {
      ++pos_;
      if (is_punct(cur(), "(")) {
        ++pos_;
        while (!is_punct(cur(), ")")) {
          if (cur().k != Tok::kSsa) return fail(cur(), "expected a block argument");
          b.args.push_back(cur().s);
          ++pos_;
          if (!expect(":")) return false;
          b.arg_types.push_back(cur().s);
          ++pos_;
          if (is_punct(cur(), ",")) ++pos_;
        }
        ++pos_;
      }
      if (!expect(":")) return false;
    }
    if (!block_ops(&b)) return false;
    if (!expect("}")) return false;
    op->region.push_back(std::move(b));
    return true;
  }
};

}  // namespace

bool parse_module(const std::string& text, Module* out, std::string* error) {
  std::vector<Tok> toks;
  if (!tokenize(text, &toks, error)) return false;
  Parser p(std::move(toks));
  return p.module(out, error);
}

// ------------------------------------------------------------------ queries

bool op_group(const Op& op, const std::string& kw, std::vector<std::string>* names,
              std::vector<std::string>* types) {
  names->clear();
  types->clear();
  const auto& t = op.toks;
  for (size_t i = 0; i + 1 < t.size(); ++i) {
    if (t[i].k == Tok::kIdent && t[i].s == kw && is_punct(t[i + 1], "(")) {
      size_t j = i + 2;
      bool after_colon = false;
      int depth = 1;
      for (; j < t.size() && depth > 0; ++j) {
        if (is_open(t[j])) ++depth;
        if (is_close(t[j]) && --depth == 0) break;
        if (depth != 1) continue;
        if (is_punct(t[j], ":")) {
          after_colon = true;
          continue;
        }
        if (is_punct(t[j], ",")) continue;
        if (!after_colon && t[j].k == Tok::kSsa) names->push_back(t[j].s);
        if (after_colon) types->push_back(t[j].s);
      }
      return true;
    }
  }
  return false;
}

std::vector<std::string> op_operands(const Op& op) {
  std::vector<std::string> out;
  const auto& t = op.toks;
  int depth = 0;
  for (size_t i = 0; i < t.size(); ++i) {
    if (is_open(t[i])) {
      // keyword groups and attribute dictionaries are not plain operands
      ++depth;
      continue;
    }
    if (is_close(t[i])) {
      --depth;
      continue;
    }
    if (depth == 0 && is_punct(t[i], ":")) break;  // the type list follows
    if (depth == 0 && t[i].k == Tok::kSsa) out.push_back(t[i].s);
  }
  return out;
}

std::vector<std::string> op_result_types(const Op& op) {
  std::vector<std::string> out;
  const auto& t = op.toks;
  int depth = 0;
  long arrow = -1, colon = -1;
  for (size_t i = 0; i < t.size(); ++i) {
    if (is_open(t[i])) ++depth;
    if (is_close(t[i])) --depth;
    if (depth == 0 && is_punct(t[i], "->")) arrow = (long)i;
    if (depth == 0 && is_punct(t[i], ":")) colon = (long)i;
  }
  long from = arrow >= 0 ? arrow : colon;
  if (from < 0) return out;
  size_t i = (size_t)from + 1;
  if (i < t.size() && is_punct(t[i], "(")) {
    for (++i; i < t.size() && !is_punct(t[i], ")"); ++i)
      if (!is_punct(t[i], ",")) out.push_back(t[i].s);
    return out;
  }
  // `: f16 to f32` (casts) -> the type after `to`; otherwise the last type
  std::string last;
  for (; i < t.size(); ++i) {
    if (is_punct(t[i], ",")) continue;
    if (t[i].k == Tok::kIdent && (t[i].s == "to" || t[i].s == "into")) continue;
    if (t[i].k == Tok::kAngle || t[i].k == Tok::kIdent || t[i].k == Tok::kBang) last = t[i].s;
  }
  if (!last.empty()) out.push_back(last);
  return out;
}

std::vector<Tok> op_attr(const Op& op, const std::string& key) {
  std::vector<Tok> out;
  const auto& t = op.toks;
  for (size_t i = 0; i + 2 < t.size(); ++i) {
    if ((t[i].k == Tok::kIdent || t[i].k == Tok::kStr) && t[i].s == key && is_punct(t[i + 1], "=")) {
      size_t j = i + 2;
      int depth = 0;
      for (; j < t.size(); ++j) {
        if (depth == 0 && (is_punct(t[j], ",") || is_close(t[j]))) break;
        if (is_open(t[j])) ++depth;
        if (is_close(t[j])) --depth;
        out.push_back(t[j]);
        if (depth == 0 && !is_open(t[j]) && j > i + 2 && t[j].k != Tok::kAngle) {
          // scalar value: one token
        }
      }
      return out;
    }
  }
  return out;
}

std::string op_constant_text(const Op& op) {
  for (const Tok& t : op.toks) {
    if (t.k == Tok::kNum || t.k == Tok::kAngle) return t.s;
    if (t.k == Tok::kIdent && (t.s == "true" || t.s == "false")) return t.s;
    if (is_punct(t, ":")) break;
  }
  return "";
}

TensorType parse_type(const std::string& t) {
  TensorType r;
  if (t.rfind("tensor<", 0) == 0 && t.back() == '>') {
    const std::string body = t.substr(7, t.size() - 8);
    std::stringstream ss(body);
    std::string part;
    std::vector<std::string> parts;
    while (std::getline(ss, part, 'x')) parts.push_back(part);
    if (parts.empty()) return r;
    r.elem = parts.back();
    parts.pop_back();
    for (const std::string& p : parts) {
      if (p.empty() || p == "?") return r;  // dynamic dims are not supported
      char* end = nullptr;
      const long long v = std::strtoll(p.c_str(), &end, 10);
      if (*end != '\0' || v < 0) return r;
      r.dims.push_back(v);
    }
    r.tensor = true;
    r.ok = true;
    return r;
  }
  if (t == "f16" || t == "f32" || t == "f64" || t == "i8" || t == "i1" || t == "i32" ||
      t == "i64" || t == "index" || t == "bf16") {
    r.elem = t;
    r.ok = true;
  }
  return r;
}

AffineMap parse_affine_map(const std::string& text) {
  AffineMap m;
  // affine_map<(d0, d1, d2) -> (d0, d1, 0)>
  const size_t a = text.find('(');
  const size_t arrow = text.find("->");
  if (a == std::string::npos || arrow == std::string::npos) return m;
  const size_t b = text.find(')', a);
  const size_t c = text.find('(', arrow);
  const size_t d = text.rfind(')');
  if (b == std::string::npos || c == std::string::npos || d == std::string::npos || d < c)
    return m;
  auto split = [](const std::string& s) {
    std::vector<std::string> out;
    std::string cur;
    for (char ch : s) {
      if (ch == ',') {
        out.push_back(cur);
        cur.clear();
      } else if (!std::isspace((unsigned char)ch)) {
        cur += ch;
      }
    }
    if (!cur.empty()) out.push_back(cur);
    return out;
  };
  const auto dims = split(text.substr(a + 1, b - a - 1));
  const auto res = split(text.substr(c + 1, d - c - 1));
  m.num_dims = (int)dims.size();
  for (const std::string& r : res) {
    if (r == "0") {
      m.results.push_back(-1);
      continue;
    }
    bool found = false;
    for (int i = 0; i < m.num_dims; ++i)
      if (dims[i] == r) {
        m.results.push_back(i);
        found = true;
      }
    if (!found) return m;  // non-trivial expression
  }
  m.ok = true;
  return m;
}

}  // namespace hxbc
