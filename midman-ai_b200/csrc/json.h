// A small JSON writer with the output conventions of the reference's
// crates/midman-api/src/json.rs: numbers in the shortest decimal form that reads
// back to the same double, without exponents; non-finite numbers as null.
#pragma once
#include <charconv>
#include <cmath>
#include <cstdint>
#include <string>
#include <vector>

namespace mm {

class JsonWriter {
 public:
  JsonWriter& begin_object() { before(); out_ += '{'; has_.push_back(false); return *this; }
  JsonWriter& end_object() { has_.pop_back(); out_ += '}'; return *this; }
  JsonWriter& begin_array() { before(); out_ += '['; has_.push_back(false); return *this; }
  JsonWriter& end_array() { has_.pop_back(); out_ += ']'; return *this; }
  JsonWriter& key(const std::string& k) {
    if (!has_.empty()) {
      if (has_.back()) out_ += ',';
      has_.back() = true;
    }
    escape(k);
    out_ += ':';
    after_key_ = true;
    return *this;
  }
  JsonWriter& string(const std::string& v) { before(); escape(v); return *this; }
  JsonWriter& integer(uint64_t v) { before(); out_ += std::to_string(v); return *this; }
  JsonWriter& boolean(bool v) { before(); out_ += v ? "true" : "false"; return *this; }
  JsonWriter& null() { before(); out_ += "null"; return *this; }
  JsonWriter& number(double v) {
    before();
    if (!std::isfinite(v)) {
      out_ += "null";
      return *this;
    }
    char buf[512];
    auto r = std::to_chars(buf, buf + sizeof(buf), v, std::chars_format::fixed);
    out_.append(buf, r.ptr);
    return *this;
  }
  JsonWriter& optional_number(bool present, double v) { return present ? number(v) : null(); }
  std::string finish() { return std::move(out_); }

 private:
  void before() {
    if (after_key_) {
      after_key_ = false;
    } else if (!has_.empty()) {
      if (has_.back()) out_ += ',';
      has_.back() = true;
    }
  }
  void escape(const std::string& s) {
    out_ += '"';
    for (unsigned char c : s) {
      switch (c) {
        case '"': out_ += "\\\""; break;
        case '\\': out_ += "\\\\"; break;
        case '\n': out_ += "\\n"; break;
        case '\r': out_ += "\\r"; break;
        case '\t': out_ += "\\t"; break;
        default:
          if (c < 0x20) {
            char b[8];
            std::snprintf(b, sizeof(b), "\\u%04x", c);
            out_ += b;
          } else {
            out_ += static_cast<char>(c);
          }
      }
    }
    out_ += '"';
  }
  std::string out_;
  std::vector<bool> has_;
  bool after_key_ = false;
};

}  // namespace mm
