// Training-state files: the safetensors container of
// crates/midman-checkpoint/src/safetensors.rs (with the header reader of json.rs)
// and the run state of crates/midman-training/src/state.rs. A file written here
// is byte-identical to the reference's for the same tensors and metadata, and a
// file is accepted or refused for the same reasons.
#include "state.h"

#include <algorithm>
#include <charconv>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <set>
#include <unistd.h>

namespace mm {

namespace {

constexpr uint64_t kMaxHeaderBytes = 100000000;  // safetensors.rs:39
constexpr int kMaxDepth = 8;                     // json.rs:18
constexpr const char* kMetadataKey = "__metadata__";

[[noreturn]] void fail(const std::string& what) { throw StateFormatError("safetensors file: " + what); }

// ---------------------------------------------------------------- header JSON
// Objects, arrays, strings and non-negative integers only (json.rs:5-9).
struct Json {
  enum Kind { Object, Array, String, Number } kind = Number;
  std::vector<std::pair<std::string, Json>> object;
  std::vector<Json> array;
  std::string text;
  uint64_t number = 0;
};

class JsonReader {
 public:
  explicit JsonReader(const std::string& s) : s_(s) {}
  Json parse() {
    skip();
    Json v = value(0);
    skip();
    if (pos_ != s_.size()) bad("unexpected data after the top-level value");
    return v;
  }

 private:
  [[noreturn]] void bad(const std::string& m) const {
    throw StateFormatError("safetensors header: " + m + " at byte " + std::to_string(pos_));
  }
  int peek() const { return pos_ < s_.size() ? static_cast<unsigned char>(s_[pos_]) : -1; }
  void skip() {
    while (pos_ < s_.size() && (s_[pos_] == ' ' || s_[pos_] == '\t' || s_[pos_] == '\n' || s_[pos_] == '\r')) ++pos_;
  }
  void expect(char c) {
    if (peek() != static_cast<unsigned char>(c)) bad(std::string("expected `") + c + "`");
    ++pos_;
  }
  Json value(int depth) {
    if (depth > kMaxDepth) bad("nesting is too deep");
    const int c = peek();
    if (c == '{') return object(depth);
    if (c == '[') return array(depth);
    Json v;
    if (c == '"') {
      v.kind = Json::String;
      v.text = string();
      return v;
    }
    if (c >= '0' && c <= '9') {
      v.kind = Json::Number;
      v.number = number();
      return v;
    }
    if (c == '-') bad("negative numbers are not allowed");
    if (c < 0) bad("unexpected end of the header");
    bad("unexpected character");
  }
  Json object(int depth) {
    expect('{');
    skip();
    Json v;
    v.kind = Json::Object;
    if (peek() == '}') {
      ++pos_;
      return v;
    }
    std::set<std::string> seen;
    for (;;) {
      skip();
      if (peek() != '"') bad("expected a string key");
      std::string key = string();
      if (!seen.insert(key).second) bad("duplicate key `" + key + "`");
      skip();
      expect(':');
      skip();
      Json item = value(depth + 1);
      v.object.emplace_back(std::move(key), std::move(item));
      skip();
      const int c = peek();
      if (c == ',') {
        ++pos_;
      } else if (c == '}') {
        ++pos_;
        return v;
      } else {
        bad("expected `,` or `}`");
      }
    }
  }
  Json array(int depth) {
    expect('[');
    skip();
    Json v;
    v.kind = Json::Array;
    if (peek() == ']') {
      ++pos_;
      return v;
    }
    for (;;) {
      skip();
      v.array.push_back(value(depth + 1));
      skip();
      const int c = peek();
      if (c == ',') {
        ++pos_;
      } else if (c == ']') {
        ++pos_;
        return v;
      } else {
        bad("expected `,` or `]`");
      }
    }
  }
  uint64_t number() {
    const size_t start = pos_;
    while (peek() >= '0' && peek() <= '9') ++pos_;
    if (pos_ - start > 1 && s_[start] == '0') bad("numbers must not have leading zeros");
    if (peek() == '.' || peek() == 'e' || peek() == 'E') bad("fractions and exponents are not allowed");
    uint64_t v = 0;
    for (size_t i = start; i < pos_; ++i) {
      const uint64_t d = static_cast<uint64_t>(s_[i] - '0');
      if (v > (UINT64_MAX - d) / 10) bad("number is too large");
      v = v * 10 + d;
    }
    return v;
  }
  unsigned hex4() {
    unsigned v = 0;
    for (int i = 0; i < 4; ++i) {
      const int c = peek();
      unsigned d;
      if (c >= '0' && c <= '9') d = c - '0';
      else if (c >= 'a' && c <= 'f') d = c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') d = c - 'A' + 10;
      else bad("expected four hex digits after `\\u`");
      ++pos_;
      v = v * 16 + d;
    }
    return v;
  }
  static void utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
      out += static_cast<char>(cp);
    } else if (cp < 0x800) {
      out += static_cast<char>(0xC0 | (cp >> 6));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += static_cast<char>(0xE0 | (cp >> 12));
      out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    } else {
      out += static_cast<char>(0xF0 | (cp >> 18));
      out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
      out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    }
  }
  std::string string() {
    expect('"');
    std::string out;
    for (;;) {
      const int c = peek();
      if (c < 0) bad("unterminated string");
      ++pos_;
      if (c == '"') break;
      if (c < 0x20) {
        --pos_;
        bad("control character in a string");
      }
      if (c != '\\') {
        out += static_cast<char>(c);
        continue;
      }
      const int e = peek();
      if (e < 0) bad("unterminated escape");
      ++pos_;
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
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            if (peek() != '\\' || pos_ + 1 >= s_.size() || s_[pos_ + 1] != 'u') bad("unpaired surrogate in an escape");
            pos_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo > 0xDFFF) bad("unpaired surrogate in an escape");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
            bad("unpaired surrogate in an escape");
          }
          utf8(out, cp);
          break;
        }
        default:
          --pos_;
          bad("unknown escape");
      }
    }
    return out;
  }

  const std::string& s_;
  size_t pos_ = 0;
};

// Quoted JSON string with serde_json's escapes (json.rs:51-70).
void write_string(std::string& out, const std::string& text) {
  out += '"';
  for (const char ch : text) {
    const unsigned char c = static_cast<unsigned char>(ch);
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case 0x08: out += "\\b"; break;
      case 0x0c: out += "\\f"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          out += buf;
        } else {
          out += ch;
        }
    }
  }
  out += '"';
}

bool valid_utf8(const uint8_t* p, size_t n) {
  size_t i = 0;
  while (i < n) {
    const uint8_t c = p[i];
    int len = c < 0x80 ? 1 : (c >> 5) == 0x6 ? 2 : (c >> 4) == 0xE ? 3 : (c >> 3) == 0x1E ? 4 : 0;
    if (len == 0 || i + len > n) return false;
    uint32_t cp = len == 1 ? c : len == 2 ? (c & 0x1F) : len == 3 ? (c & 0x0F) : (c & 0x07);
    for (int k = 1; k < len; ++k) {
      if ((p[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i + k] & 0x3F);
    }
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && (cp < 0x10000 || cp > 0x10FFFF)) ||
        (cp >= 0xD800 && cp <= 0xDFFF))
      return false;
    i += len;
  }
  return true;
}

std::string dims_text(const std::vector<uint64_t>& shape) {
  std::string s = "[";
  for (size_t i = 0; i < shape.size(); ++i) s += (i ? ", " : "") + std::to_string(shape[i]);
  return s + "]";
}

// safetensors.rs:379-443
SafeTensor read_entry(const std::string& name, const Json& v) {
  if (v.kind != Json::Object) fail("the entry for `" + name + "` must be an object");
  const Json *dtype = nullptr, *shape = nullptr, *offsets = nullptr;
  for (const auto& [k, f] : v.object) {
    if (k == "dtype") dtype = &f;
    else if (k == "shape") shape = &f;
    else if (k == "data_offsets") offsets = &f;
    else fail("the entry for `" + name + "` has an unknown field `" + k + "`");
  }
  if (!dtype || !shape || !offsets) fail("the entry for `" + name + "` must have `dtype`, `shape` and `data_offsets`");
  if (dtype->kind != Json::String) fail("the dtype of `" + name + "` must be a string");
  if (dtype->text != "F32") fail("tensor `" + name + "` has dtype `" + dtype->text + "`; only F32 is supported");
  if (shape->kind != Json::Array) fail("the shape of `" + name + "` must be an array");
  SafeTensor t;
  t.name = name;
  for (const Json& d : shape->array) {
    if (d.kind != Json::Number) fail("the shape of `" + name + "` must hold only integers");
    t.shape.push_back(d.number);
  }
  if (offsets->kind != Json::Array || offsets->array.size() != 2 || offsets->array[0].kind != Json::Number ||
      offsets->array[1].kind != Json::Number)
    fail("the data_offsets of `" + name + "` must be two integers");
  t.begin = offsets->array[0].number;
  t.end = offsets->array[1].number;
  uint64_t count = 1;
  bool overflow = false;
  for (uint64_t d : t.shape) {
    if (d != 0 && count > UINT64_MAX / d) overflow = true;
    count *= d;
  }
  if (overflow || count > UINT64_MAX / 4) fail("the shape of `" + name + "` is too large");
  const uint64_t bytes = count * 4;
  if (t.end < t.begin || t.end - t.begin != bytes)
    fail("tensor `" + name + "` has shape " + dims_text(t.shape) + ", which needs " + std::to_string(bytes) +
         " bytes, but its data_offsets [" + std::to_string(t.begin) + ", " + std::to_string(t.end) +
         "] do not span that");
  return t;
}

}  // namespace

// ---------------------------------------------------------------- container

const SafeTensor* SafeFile::find(const std::string& name) const {
  for (const SafeTensor& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}

void SafeFile::copy_values(const SafeTensor& t, float* out) const {
  // little-endian f32 on a little-endian host: the bytes are the values
  std::memcpy(out, bytes.data() + data_offset + t.begin, t.end - t.begin);
}

SafeFile parse_safetensors(std::vector<uint8_t> bytes) {
  if (bytes.size() < 8) fail("the file is shorter than its 8-byte length prefix");
  uint64_t header_len = 0;
  for (int i = 7; i >= 0; --i) header_len = (header_len << 8) | bytes[i];
  if (header_len > kMaxHeaderBytes)
    fail("the header claims " + std::to_string(header_len) + " bytes, over the format's limit of " +
         std::to_string(kMaxHeaderBytes));
  if (header_len > bytes.size() - 8)
    fail("the header claims " + std::to_string(header_len) + " bytes but the file has only " +
         std::to_string(bytes.size() - 8) + " after the prefix");
  if (header_len == 0 || bytes[8] != '{') fail("the header must start with `{`");
  if (!valid_utf8(bytes.data() + 8, header_len)) fail("the header is not valid UTF-8");
  const std::string text(reinterpret_cast<const char*>(bytes.data() + 8), header_len);
  const Json root = JsonReader(text).parse();
  if (root.kind != Json::Object) fail("the header must be a JSON object");

  SafeFile f;
  for (const auto& [key, value] : root.object) {
    if (key == kMetadataKey) {
      if (value.kind != Json::Object) fail("`__metadata__` must be an object of strings");
      for (const auto& [mk, mv] : value.object) {
        if (mv.kind != Json::String) fail("metadata value for `" + mk + "` must be a string");
        f.metadata[mk] = mv.text;
      }
    } else {
      f.tensors.push_back(read_entry(key, value));
    }
  }
  std::stable_sort(f.tensors.begin(), f.tensors.end(), [](const SafeTensor& a, const SafeTensor& b) {
    return a.begin != b.begin ? a.begin < b.begin : a.end < b.end;
  });
  const uint64_t data_len = bytes.size() - 8 - header_len;
  uint64_t expected = 0;
  for (const SafeTensor& t : f.tensors) {
    if (t.begin != expected)
      fail("tensor `" + t.name + "` starts at byte " + std::to_string(t.begin) + " where byte " +
           std::to_string(expected) + " was expected: the data ranges must tile the data with no gap or overlap");
    expected = t.end;
  }
  if (expected != data_len)
    fail("the tensors cover " + std::to_string(expected) + " bytes but the data section has " +
         std::to_string(data_len));
  f.data_offset = 8 + header_len;
  f.bytes = std::move(bytes);
  return f;
}

SafeFile load_safetensors(const std::string& path) {
  std::ifstream in(path, std::ios::binary | std::ios::ate);
  if (!in) throw StateFormatError(path + ": cannot open the file");
  const std::streamsize n = in.tellg();
  in.seekg(0);
  std::vector<uint8_t> bytes(static_cast<size_t>(n));
  if (n > 0 && !in.read(reinterpret_cast<char*>(bytes.data()), n))
    throw StateFormatError(path + ": cannot read the file");
  return parse_safetensors(std::move(bytes));
}

void save_safetensors(const std::string& path, const std::map<std::string, std::string>& metadata,
                      std::vector<WriteTensor> tensors,
                      const std::function<void(const WriteTensor&, std::vector<float>&)>& fill) {
  std::sort(tensors.begin(), tensors.end(), [](const WriteTensor& a, const WriteTensor& b) { return a.name < b.name; });
  std::string header = "{";
  bool first = true;
  if (!metadata.empty()) {
    header += "\"__metadata__\":{";
    bool f2 = true;
    for (const auto& [k, v] : metadata) {
      if (!f2) header += ',';
      f2 = false;
      write_string(header, k);
      header += ':';
      write_string(header, v);
    }
    header += '}';
    first = false;
  }
  uint64_t begin = 0;
  for (const WriteTensor& t : tensors) {
    if (t.name == kMetadataKey) throw StateError("`__metadata__` is reserved and cannot name a tensor");
    const uint64_t end = begin + t.count * 4;
    if (!first) header += ',';
    first = false;
    write_string(header, t.name);
    header += ":{\"dtype\":\"F32\",\"shape\":[";
    for (size_t i = 0; i < t.shape.size(); ++i) header += (i ? "," : "") + std::to_string(t.shape[i]);
    header += "],\"data_offsets\":[" + std::to_string(begin) + "," + std::to_string(end) + "]}";
    begin = end;
  }
  header += '}';
  header.append((8 - header.size() % 8) % 8, ' ');
  if (header.size() > kMaxHeaderBytes)
    throw StateError("the header is " + std::to_string(header.size()) + " bytes, over the format's limit");

  const std::string tmp = path + ".tmp";
  FILE* fp = std::fopen(tmp.c_str(), "wb");
  if (!fp) throw StateFormatError(path + ": cannot create " + tmp);
  bool ok = true;
  uint8_t prefix[8];
  for (int i = 0; i < 8; ++i) prefix[i] = static_cast<uint8_t>(static_cast<uint64_t>(header.size()) >> (8 * i));
  ok = ok && std::fwrite(prefix, 1, 8, fp) == 8;
  ok = ok && std::fwrite(header.data(), 1, header.size(), fp) == header.size();
  std::vector<float> buf;
  for (const WriteTensor& t : tensors) {
    if (!ok) break;
    buf.assign(t.count, 0.0f);
    fill(t, buf);
    ok = std::fwrite(buf.data(), 4, t.count, fp) == t.count;
  }
  ok = ok && std::fflush(fp) == 0 && ::fsync(fileno(fp)) == 0;
  ok = (std::fclose(fp) == 0) && ok;
  if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) {
    std::remove(tmp.c_str());
    throw StateFormatError(path + ": writing the file failed");
  }
}

std::string rust_f32(float v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "inf" : "-inf";
  char buf[128];
  // shortest round-trip digits, in positional notation
  const auto r = std::to_chars(buf, buf + sizeof buf, v, std::chars_format::fixed);
  return std::string(buf, r.ptr);
}

// ---------------------------------------------------------------- training state

namespace {
constexpr const char* kFormat = "midman-training-state";  // state.rs:15
constexpr uint64_t kVersion = 1;                          // state.rs:18
const std::string kParam = "param/", kM = "adamw.m/", kV = "adamw.v/";

std::string list_names(const std::vector<std::string>& names) {  // state.rs:290-298
  std::string text;
  for (size_t i = 0; i < names.size() && i < 5; ++i) text += (i ? ", `" : "`") + names[i] + "`";
  if (names.size() > 5) text += " and " + std::to_string(names.size() - 5) + " more";
  return text;
}
}  // namespace

std::vector<std::pair<std::string, std::string>> settings_entries(const TrainSettings& s) {
  return {{"train.batch_size", std::to_string(s.batch_size)},
          {"train.seq_len", std::to_string(s.seq_len)},
          {"train.seed", std::to_string(s.seed)},
          {"train.max_lr", rust_f32(s.max_lr)},
          {"train.min_lr", rust_f32(s.min_lr)},
          {"train.warmup_steps", std::to_string(s.warmup_steps)},
          {"train.total_steps", std::to_string(s.total_steps)},
          {"train.beta1", rust_f32(s.beta1)},
          {"train.beta2", rust_f32(s.beta2)},
          {"train.eps", rust_f32(s.eps)},
          {"train.weight_decay", rust_f32(s.weight_decay)},
          {"train.clip_norm", rust_f32(s.clip_norm)}};
}

Progress progress_of(const std::map<std::string, std::string>& md) {
  const auto fmt = md.find("format");
  if (fmt == md.end())
    throw StateFormatError(std::string("training state: the file has no `format` entry, so it is not a ") + kFormat +
                     " file");
  if (fmt->second != kFormat)
    throw StateFormatError("training state: `format` is `" + fmt->second + "`, not `" + kFormat + "`");
  auto number = [&](const char* key) -> uint64_t {
    const auto it = md.find(key);
    if (it == md.end()) throw StateFormatError(std::string("training state: the file has no `") + key + "` entry");
    const std::string& t = it->second;
    // u64::from_str: decimal digits, optionally after one `+`
    const char* b = t.data() + (!t.empty() && t[0] == '+' ? 1 : 0);
    const char* e = t.data() + t.size();
    uint64_t v = 0;
    const auto r = std::from_chars(b, e, v);
    if (b == e || r.ec != std::errc() || r.ptr != e)
      throw StateFormatError(std::string("training state: `") + key + "` is `" + t + "`, not a whole number");
    return v;
  };
  const uint64_t version = number("state_version");
  if (version != kVersion)
    throw StateFormatError("training state: version " + std::to_string(version) + " is not supported (this build reads " +
                     std::to_string(kVersion) + ")");
  const uint64_t position = number("position");
  Progress p;
  p.step = number("step");
  p.epoch = number("epoch");
  p.position = position;
  return p;
}

void check_settings(const TrainSettings& s, const std::map<std::string, std::string>& md) {
  std::string problems;
  for (const auto& [key, now] : settings_entries(s)) {
    const auto it = md.find(key);
    std::string p;
    if (it == md.end()) p = "`" + key + "` is missing from the saved run";
    else if (it->second != now) p = "`" + key + "` was " + it->second + " and is now " + now;
    if (!p.empty()) problems += (problems.empty() ? "" : "; ") + p;
  }
  if (!problems.empty()) throw StateError("the saved run was made with other settings: " + problems);
}

void save_state(const std::string& path, const std::vector<StateParam>& params, const Progress& progress,
                const TrainSettings& settings, const std::function<void(int, uint64_t, uint64_t, float*)>& read) {
  std::set<std::string> names;
  for (const StateParam& p : params)
    if (!names.insert(p.name).second) throw StateError("two parameters are named `" + p.name + "`");
  std::map<std::string, std::string> md;
  for (const auto& [k, v] : settings_entries(settings)) md[k] = v;
  md["format"] = kFormat;
  md["state_version"] = std::to_string(kVersion);
  md["step"] = std::to_string(progress.step);
  md["epoch"] = std::to_string(progress.epoch);
  md["position"] = std::to_string(progress.position);
  struct Src {
    int which;
    uint64_t offset;
  };
  std::map<std::string, Src> src;
  std::vector<WriteTensor> tensors;
  for (const StateParam& p : params) {
    tensors.push_back({kParam + p.name, p.shape, p.count});
    src[kParam + p.name] = {0, p.offset};
    if (progress.step > 0) {  // the moments exist once a step has been taken
      tensors.push_back({kM + p.name, p.shape, p.count});
      tensors.push_back({kV + p.name, p.shape, p.count});
      src[kM + p.name] = {2, p.offset};
      src[kV + p.name] = {3, p.offset};
    }
  }
  save_safetensors(path, md, std::move(tensors), [&](const WriteTensor& t, std::vector<float>& out) {
    const Src& s = src.at(t.name);
    read(s.which, s.offset, t.count, out.data());
  });
}

LoadedState load_state(const std::string& path, const std::vector<StateParam>& params, uint64_t total,
                       const TrainSettings& settings) {
  const SafeFile file = load_safetensors(path);
  LoadedState out;
  out.progress = progress_of(file.metadata);
  check_settings(settings, file.metadata);
  std::set<std::string> wanted;
  for (const StateParam& p : params)
    if (!wanted.insert(p.name).second) throw StateError("two parameters are named `" + p.name + "`");
  // every tensor of the file is one of the three kinds, for a parameter of this model
  std::vector<std::string> unexpected;
  for (const SafeTensor& t : file.tensors) {
    bool known = false;
    for (const std::string* prefix : {&kParam, &kM, &kV})
      if (t.name.compare(0, prefix->size(), *prefix) == 0 && wanted.count(t.name.substr(prefix->size()))) known = true;
    if (!known) unexpected.push_back(t.name);
  }
  if (!unexpected.empty())
    throw StateError("the saved run holds " + std::to_string(unexpected.size()) +
                     " tensor(s) this model does not have: " + list_names(unexpected));
  const bool with_moments = out.progress.step > 0;
  std::vector<std::string> missing;
  for (const StateParam& p : params) {
    std::vector<const std::string*> kinds{&kParam};
    if (with_moments) {
      kinds.push_back(&kM);
      kinds.push_back(&kV);
    }
    for (const std::string* prefix : kinds) {
      const std::string key = *prefix + p.name;
      const SafeTensor* t = file.find(key);
      if (!t) {
        missing.push_back(key);
      } else if (t->shape != p.shape) {
        throw StateShapeError("load_state: `" + key + "` has shape " + dims_text(t->shape) +
                         " in the saved run but the parameter has " + dims_text(p.shape));
      }
    }
  }
  if (!missing.empty())
    throw StateError("the saved run is missing " + std::to_string(missing.size()) +
                     " tensor(s): " + list_names(missing));
  if (!with_moments)
    for (const SafeTensor& t : file.tensors)
      if (t.name.compare(0, kParam.size(), kParam) != 0)
        throw StateError("the saved run has taken no step and yet holds optimizer moments");

  out.params.assign(total, 0.0f);
  if (with_moments) {
    out.m.assign(total, 0.0f);
    out.v.assign(total, 0.0f);
  }
  for (const StateParam& p : params) {
    file.copy_values(*file.find(kParam + p.name), out.params.data() + p.offset);
    if (!with_moments) continue;
    float* m = out.m.data() + p.offset;
    float* v = out.v.data() + p.offset;
    file.copy_values(*file.find(kM + p.name), m);
    file.copy_values(*file.find(kV + p.name), v);
    // AdamW::restore (adamw.rs:95-130)
    for (uint64_t i = 0; i < p.count; ++i)
      if (!std::isfinite(m[i])) throw StateError("adamw: first moment of '" + p.name + "' is not finite");
    for (uint64_t i = 0; i < p.count; ++i)
      if (!(std::isfinite(v[i]) && v[i] >= 0.0f))
        throw StateError("adamw: second moment of '" + p.name + "' is negative or not finite");
  }
  return out;
}

}  // namespace mm
