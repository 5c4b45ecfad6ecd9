// Token shards (crates/midman-data/src/shard.rs) and the SHA-256 their files end
// with (crates/midman-data/src/hash.rs restates FIPS 180-4; so does this file).
#include "shard.h"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <unistd.h>

namespace mm {

namespace {

// FIPS 180-4 section 4.2.2 / 5.3.3: the round constants are the first 32 bits of
// the fractional parts of the cube roots of the first 64 primes, the initial hash
// those of the square roots of the first 8 primes. Computed here from that
// definition with exact integer roots: floor(root(p) * 2^32) mod 2^32.
struct Sha256Constants {
  uint32_t k[64];
  uint32_t h0[8];
  Sha256Constants() {
    int primes[64];
    int n = 0;
    for (int c = 2; n < 64; ++c) {
      bool prime = true;
      for (int d = 2; d * d <= c; ++d)
        if (c % d == 0) prime = false;
      if (prime) primes[n++] = c;
    }
    using u128 = unsigned __int128;
    for (int i = 0; i < 64; ++i) {  // largest x with x^3 <= p * 2^96
      const u128 target = static_cast<u128>(primes[i]) << 96;
      uint64_t lo = 0, hi = uint64_t(1) << 40;
      while (lo < hi) {
        const uint64_t mid = lo + (hi - lo + 1) / 2;
        if (static_cast<u128>(mid) * mid * mid <= target) lo = mid;
        else hi = mid - 1;
      }
      k[i] = static_cast<uint32_t>(lo);
    }
    for (int i = 0; i < 8; ++i) {  // largest x with x^2 <= p * 2^64
      const u128 target = static_cast<u128>(primes[i]) << 64;
      uint64_t lo = 0, hi = uint64_t(1) << 40;
      while (lo < hi) {
        const uint64_t mid = lo + (hi - lo + 1) / 2;
        if (static_cast<u128>(mid) * mid <= target) lo = mid;
        else hi = mid - 1;
      }
      h0[i] = static_cast<uint32_t>(lo);
    }
  }
};

const Sha256Constants& constants() {
  static const Sha256Constants c;
  return c;
}

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void compress(uint32_t h[8], const uint8_t block[64], const uint32_t k[64]) {
  uint32_t w[64];
  for (int t = 0; t < 16; ++t)
    w[t] = (uint32_t(block[4 * t]) << 24) | (uint32_t(block[4 * t + 1]) << 16) | (uint32_t(block[4 * t + 2]) << 8) |
           uint32_t(block[4 * t + 3]);
  for (int t = 16; t < 64; ++t) {
    const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
    const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
    w[t] = w[t - 16] + s0 + w[t - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
  for (int t = 0; t < 64; ++t) {
    const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[t] + w[t];
    const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
    hh = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

constexpr size_t kHeaderBytes = 8 + 4 + 4 + 4 + 4 + 8;  // shard.rs:22
constexpr size_t kChecksumBytes = 32;
constexpr uint32_t kVersion = 1;

size_t width_for(uint32_t vocab) { return vocab <= 65536 ? 2 : 4; }  // shard.rs:28-34

[[noreturn]] void fail(const std::string& m) { throw ShardError("token shard: " + m); }

uint32_t word(const uint8_t* p) { return uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24; }

}  // namespace

std::array<uint8_t, 32> sha256(const uint8_t* data, size_t n) {
  const Sha256Constants& c = constants();
  uint32_t h[8];
  std::memcpy(h, c.h0, sizeof h);
  size_t i = 0;
  for (; i + 64 <= n; i += 64) compress(h, data + i, c.k);
  // padding: 0x80, zeros, the bit length as a 64-bit big-endian integer
  uint8_t tail[128] = {};
  const size_t rest = n - i;
  std::memcpy(tail, data + i, rest);
  tail[rest] = 0x80;
  const size_t blocks = rest + 1 + 8 <= 64 ? 1 : 2;
  const uint64_t bits = static_cast<uint64_t>(n) * 8;
  for (int b = 0; b < 8; ++b) tail[blocks * 64 - 1 - b] = static_cast<uint8_t>(bits >> (8 * b));
  for (size_t b = 0; b < blocks; ++b) compress(h, tail + 64 * b, c.k);
  std::array<uint8_t, 32> out;
  for (int j = 0; j < 8; ++j)
    for (int b = 0; b < 4; ++b) out[4 * j + b] = static_cast<uint8_t>(h[j] >> (24 - 8 * b));
  return out;
}

TokenShard parse_token_shard(const std::vector<uint8_t>& bytes) {
  if (bytes.size() < kHeaderBytes + kChecksumBytes)
    fail(std::to_string(bytes.size()) + " bytes is shorter than the smallest shard, " +
         std::to_string(kHeaderBytes + kChecksumBytes));
  if (std::memcmp(bytes.data(), "MMTOKENS", 8) != 0) fail("the file does not start with `MMTOKENS`");
  const uint32_t version = word(bytes.data() + 8);
  if (version != kVersion)
    fail("version " + std::to_string(version) + " is not supported (this build reads " + std::to_string(kVersion) +
         ")");
  const size_t width = word(bytes.data() + 12);
  TokenShard s;
  s.vocab_size = word(bytes.data() + 16);
  s.eos = word(bytes.data() + 20);
  uint64_t count = 0;
  for (int b = 7; b >= 0; --b) count = (count << 8) | bytes[24 + b];
  if (s.vocab_size == 0) fail("the vocabulary size is 0");
  if (width != width_for(s.vocab_size))
    fail("token width " + std::to_string(width) + " is not the one for a vocabulary of " +
         std::to_string(s.vocab_size) + " ids (" + std::to_string(width_for(s.vocab_size)) + ")");
  if (s.eos >= s.vocab_size)
    fail("the end-of-text id " + std::to_string(s.eos) + " is not below the vocabulary size " +
         std::to_string(s.vocab_size));
  const bool fits = count <= (UINT64_MAX - kHeaderBytes - kChecksumBytes) / width;
  if (!fits || count * width + kHeaderBytes + kChecksumBytes != bytes.size())
    fail(std::to_string(count) + " tokens of " + std::to_string(width) + " bytes do not make a file of " +
         std::to_string(bytes.size()) + " bytes");
  const size_t body = bytes.size() - kChecksumBytes;
  const std::array<uint8_t, 32> digest = sha256(bytes.data(), body);
  if (std::memcmp(digest.data(), bytes.data() + body, kChecksumBytes) != 0)
    fail("the checksum does not match: the file is damaged");
  s.tokens.resize(count);
  const uint8_t* p = bytes.data() + kHeaderBytes;
  for (uint64_t i = 0; i < count; ++i)
    s.tokens[i] = width == 2 ? uint32_t(p[2 * i]) | uint32_t(p[2 * i + 1]) << 8 : word(p + 4 * i);
  for (uint64_t i = 0; i < count; ++i)
    if (s.tokens[i] >= s.vocab_size)
      fail("token " + std::to_string(s.tokens[i]) + " at position " + std::to_string(i) +
           " is not below the vocabulary size " + std::to_string(s.vocab_size));
  return s;
}

TokenShard load_token_shard(const std::string& path) {
  std::ifstream in(path, std::ios::binary | std::ios::ate);
  if (!in) throw ShardError(path + ": cannot open the file");
  const std::streamsize n = in.tellg();
  in.seekg(0);
  std::vector<uint8_t> bytes(static_cast<size_t>(n));
  if (n > 0 && !in.read(reinterpret_cast<char*>(bytes.data()), n)) throw ShardError(path + ": cannot read the file");
  return parse_token_shard(bytes);
}

void check_token_shard(uint32_t vocab_size, uint32_t eos, const uint32_t* tokens, size_t n) {
  if (vocab_size == 0) throw std::invalid_argument("the vocabulary size is 0");
  if (eos >= vocab_size)
    throw std::invalid_argument("the end-of-text id " + std::to_string(eos) + " is not below the vocabulary size " +
                                std::to_string(vocab_size));
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] >= vocab_size)
      throw std::invalid_argument("token " + std::to_string(tokens[i]) + " at position " + std::to_string(i) +
                                  " is not below the vocabulary size " + std::to_string(vocab_size));
}

std::vector<uint8_t> token_shard_bytes(uint32_t vocab_size, uint32_t eos, const uint32_t* tokens, size_t n) {
  check_token_shard(vocab_size, eos, tokens, n);
  const size_t width = width_for(vocab_size);
  std::vector<uint8_t> out(kHeaderBytes + n * width + kChecksumBytes);
  uint8_t* p = out.data();
  std::memcpy(p, "MMTOKENS", 8);
  const uint32_t words[4] = {kVersion, static_cast<uint32_t>(width), vocab_size, eos};
  for (int w = 0; w < 4; ++w)
    for (int b = 0; b < 4; ++b) p[8 + 4 * w + b] = static_cast<uint8_t>(words[w] >> (8 * b));
  for (int b = 0; b < 8; ++b) p[24 + b] = static_cast<uint8_t>(static_cast<uint64_t>(n) >> (8 * b));
  uint8_t* q = p + kHeaderBytes;
  for (size_t i = 0; i < n; ++i)
    for (size_t b = 0; b < width; ++b) *q++ = static_cast<uint8_t>(tokens[i] >> (8 * b));
  const size_t body = out.size() - kChecksumBytes;
  const std::array<uint8_t, 32> digest = sha256(p, body);
  std::memcpy(p + body, digest.data(), kChecksumBytes);
  return out;
}

void save_token_shard(const std::string& path, uint32_t vocab_size, uint32_t eos, const uint32_t* tokens, size_t n) {
  const std::vector<uint8_t> bytes = token_shard_bytes(vocab_size, eos, tokens, n);
  const std::string tmp = path + ".tmp";
  FILE* fp = std::fopen(tmp.c_str(), "wb");
  if (!fp) throw ShardError(path + ": cannot create " + tmp);
  bool ok = std::fwrite(bytes.data(), 1, bytes.size(), fp) == bytes.size();
  ok = std::fflush(fp) == 0 && ok;
  ok = fsync(fileno(fp)) == 0 && ok;
  ok = std::fclose(fp) == 0 && ok;
  if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) {
    std::remove(tmp.c_str());
    throw ShardError(path + ": cannot write the file");
  }
}

}  // namespace mm
