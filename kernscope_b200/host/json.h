// json.h -- the JSON value type of the tuner's persistence (the role of
// kernscope::db::json::Value, libs/db/include/kernscope/db.h:74-135): null,
// bool, number, string, array and insertion-ordered object; dump() writes
// compact JSON, parse() reads it back.
#pragma once

#include <cstdint>
#include <initializer_list>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace kernscope::db::json {

class Value {
 public:
  enum class Kind : std::uint8_t { Null, Bool, Number, String, Array, Object };
  using Member = std::pair<std::string, Value>;

  Value() = default;
  Value(std::nullptr_t) {}
  Value(bool b) : kind_(Kind::Bool), bool_(b) {}
  Value(int v) : kind_(Kind::Number), number_(v) {}
  Value(std::int64_t v) : kind_(Kind::Number), number_(static_cast<double>(v)) {}
  Value(double v) : kind_(Kind::Number), number_(v) {}
  Value(const char *s) : kind_(Kind::String), string_(s) {}
  Value(std::string s) : kind_(Kind::String), string_(std::move(s)) {}
  Value(std::string_view s) : kind_(Kind::String), string_(s) {}
  Value(std::vector<Value> a) : kind_(Kind::Array), array_(std::move(a)) {}
  Value(std::vector<Member> o) : kind_(Kind::Object), object_(std::move(o)) {}

  Kind kind() const { return kind_; }
  bool is_null() const { return kind_ == Kind::Null; }
  bool is_number() const { return kind_ == Kind::Number; }
  bool is_string() const { return kind_ == Kind::String; }
  bool is_object() const { return kind_ == Kind::Object; }
  bool is_array() const { return kind_ == Kind::Array; }
  bool as_bool() const { return bool_; }
  double as_number() const { return number_; }
  const std::string &as_string() const { return string_; }
  const std::vector<Value> &as_array() const { return array_; }
  std::vector<Value> &as_array() { return array_; }
  const std::vector<Member> &as_object() const { return object_; }

  // Object access: find returns nullptr when absent; set replaces or appends.
  const Value *find(std::string_view key) const;
  void set(std::string key, Value v);
  // Convenience lookups with defaults.
  double number_or(std::string_view key, double dflt) const;
  std::string string_or(std::string_view key, std::string dflt) const;

  std::string dump() const;
  bool operator==(const Value &o) const;

  // Parse text; returns false (and *error) on malformed input.
  static bool parse(std::string_view text, Value *out, std::string *error);

 private:
  void dump_to(std::string &out) const;
  Kind kind_ = Kind::Null;
  bool bool_ = false;
  double number_ = 0.0;
  std::string string_;
  std::vector<Member> object_;
  std::vector<Value> array_;
};

inline Value object(std::initializer_list<Value::Member> members) {
  return Value(std::vector<Value::Member>(members.begin(), members.end()));
}
inline Value array(std::initializer_list<Value> elements) {
  return Value(std::vector<Value>(elements.begin(), elements.end()));
}

}  // namespace kernscope::db::json
