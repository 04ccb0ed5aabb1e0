// json.cpp -- dump/parse of the tuner's JSON value type.
#include "json.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>

namespace kernscope::db::json {

const Value *Value::find(std::string_view key) const {
  if (kind_ != Kind::Object) return nullptr;
  for (const auto &[k, v] : object_)
    if (k == key) return &v;
  return nullptr;
}

void Value::set(std::string key, Value v) {
  if (kind_ != Kind::Object) {
    *this = Value(std::vector<Member>{});
  }
  for (auto &[k, old] : object_)
    if (k == key) {
      old = std::move(v);
      return;
    }
  object_.emplace_back(std::move(key), std::move(v));
}

double Value::number_or(std::string_view key, double dflt) const {
  const Value *v = find(key);
  return v && v->is_number() ? v->as_number() : dflt;
}

std::string Value::string_or(std::string_view key, std::string dflt) const {
  const Value *v = find(key);
  return v && v->is_string() ? v->as_string() : dflt;
}

bool Value::operator==(const Value &o) const {
  if (kind_ != o.kind_) return false;
  switch (kind_) {
    case Kind::Null: return true;
    case Kind::Bool: return bool_ == o.bool_;
    case Kind::Number: return number_ == o.number_;
    case Kind::String: return string_ == o.string_;
    case Kind::Array: return array_ == o.array_;
    case Kind::Object: return object_ == o.object_;
  }
  return false;
}

static void dump_string(std::string &out, const std::string &s) {
  out += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", c);
          out += buf;
        } else {
          out += static_cast<char>(c);
        }
    }
  }
  out += '"';
}

void Value::dump_to(std::string &out) const {
  switch (kind_) {
    case Kind::Null: out += "null"; break;
    case Kind::Bool: out += bool_ ? "true" : "false"; break;
    case Kind::Number: {
      char buf[40];
      if (!std::isfinite(number_)) {
        out += "null";
      } else if (number_ == std::floor(number_) && std::fabs(number_) < 9.007199254740992e15) {
        std::snprintf(buf, sizeof(buf), "%lld", static_cast<long long>(number_));
        out += buf;
      } else {
        std::snprintf(buf, sizeof(buf), "%.17g", number_);
        out += buf;
      }
      break;
    }
    case Kind::String: dump_string(out, string_); break;
    case Kind::Array:
      out += '[';
      for (std::size_t i = 0; i < array_.size(); ++i) {
        if (i) out += ',';
        array_[i].dump_to(out);
      }
      out += ']';
      break;
    case Kind::Object:
      out += '{';
      for (std::size_t i = 0; i < object_.size(); ++i) {
        if (i) out += ',';
        dump_string(out, object_[i].first);
        out += ':';
        object_[i].second.dump_to(out);
      }
      out += '}';
      break;
  }
}

std::string Value::dump() const {
  std::string s;
  dump_to(s);
  return s;
}

namespace {
struct Parser {
  std::string_view t;
  std::size_t i = 0;
  std::string err;

  void ws() {
    while (i < t.size() && (t[i] == ' ' || t[i] == '\n' || t[i] == '\r' || t[i] == '\t')) ++i;
  }
  bool fail(const char *m) {
    if (err.empty()) err = std::string(m) + " at offset " + std::to_string(i);
    return false;
  }
  bool lit(std::string_view w) {
    if (t.substr(i, w.size()) != w) return false;
    i += w.size();
    return true;
  }
  bool str(std::string *out) {
    if (i >= t.size() || t[i] != '"') return fail("expected string");
    ++i;
    out->clear();
    while (i < t.size() && t[i] != '"') {
      char c = t[i++];
      if (c == '\\') {
        if (i >= t.size()) return fail("bad escape");
        char e = t[i++];
        switch (e) {
          case '"': out->push_back('"'); break;
          case '\\': out->push_back('\\'); break;
          case '/': out->push_back('/'); break;
          case 'b': out->push_back('\b'); break;
          case 'f': out->push_back('\f'); break;
          case 'n': out->push_back('\n'); break;
          case 'r': out->push_back('\r'); break;
          case 't': out->push_back('\t'); break;
          case 'u': {
            if (i + 4 > t.size()) return fail("bad \\u escape");
            unsigned cp = std::strtoul(std::string(t.substr(i, 4)).c_str(), nullptr, 16);
            i += 4;
            if (cp < 0x80) {
              out->push_back(static_cast<char>(cp));
            } else if (cp < 0x800) {
              out->push_back(static_cast<char>(0xc0 | (cp >> 6)));
              out->push_back(static_cast<char>(0x80 | (cp & 0x3f)));
            } else {
              out->push_back(static_cast<char>(0xe0 | (cp >> 12)));
              out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3f)));
              out->push_back(static_cast<char>(0x80 | (cp & 0x3f)));
            }
            break;
          }
          default: return fail("bad escape");
        }
      } else {
        out->push_back(c);
      }
    }
    if (i >= t.size()) return fail("unterminated string");
    ++i;
    return true;
  }
  bool value(Value *out) {
    ws();
    if (i >= t.size()) return fail("unexpected end");
    const char c = t[i];
    if (c == '{') {
      ++i;
      std::vector<Value::Member> m;
      ws();
      if (i < t.size() && t[i] == '}') {
        ++i;
        *out = Value(std::move(m));
        return true;
      }
      while (true) {
        ws();
        std::string k;
        if (!str(&k)) return false;
        ws();
        if (i >= t.size() || t[i] != ':') return fail("expected ':'");
        ++i;
        Value v;
        if (!value(&v)) return false;
        m.emplace_back(std::move(k), std::move(v));
        ws();
        if (i < t.size() && t[i] == ',') {
          ++i;
          continue;
        }
        if (i < t.size() && t[i] == '}') {
          ++i;
          break;
        }
        return fail("expected ',' or '}'");
      }
      *out = Value(std::move(m));
      return true;
    }
    if (c == '[') {
      ++i;
      std::vector<Value> a;
      ws();
      if (i < t.size() && t[i] == ']') {
        ++i;
        *out = Value(std::move(a));
        return true;
      }
      while (true) {
        Value v;
        if (!value(&v)) return false;
        a.push_back(std::move(v));
        ws();
        if (i < t.size() && t[i] == ',') {
          ++i;
          continue;
        }
        if (i < t.size() && t[i] == ']') {
          ++i;
          break;
        }
        return fail("expected ',' or ']'");
      }
      *out = Value(std::move(a));
      return true;
    }
    if (c == '"') {
      std::string s;
      if (!str(&s)) return false;
      *out = Value(std::move(s));
      return true;
    }
    if (lit("true")) {
      *out = Value(true);
      return true;
    }
    if (lit("false")) {
      *out = Value(false);
      return true;
    }
    if (lit("null")) {
      *out = Value();
      return true;
    }
    const std::size_t start = i;
    while (i < t.size() && (std::isdigit(static_cast<unsigned char>(t[i])) || t[i] == '-' || t[i] == '+' ||
                            t[i] == '.' || t[i] == 'e' || t[i] == 'E'))
      ++i;
    if (start == i) return fail("unexpected character");
    const std::string num(t.substr(start, i - start));
    char *end = nullptr;
    const double d = std::strtod(num.c_str(), &end);
    if (!end || *end != '\0') return fail("bad number");
    *out = Value(d);
    return true;
  }
};
}  // namespace

bool Value::parse(std::string_view text, Value *out, std::string *error) {
  Parser p{text, 0, {}};
  Value v;
  if (!p.value(&v)) {
    if (error) *error = p.err;
    return false;
  }
  p.ws();
  if (p.i != text.size()) {
    if (error) *error = "trailing characters at offset " + std::to_string(p.i);
    return false;
  }
  *out = std::move(v);
  return true;
}

}  // namespace kernscope::db::json
