// Token shards (crates/midman-data/src/shard.rs): the `.mmtokens` files the
// training data comes in. A shard is a 32-byte header (the magic `MMTOKENS`,
// version, token width, vocabulary size, end-of-text id, token count), the ids as
// little-endian integers of 2 bytes (vocabularies of up to 65,536 ids) or 4, and
// a SHA-256 of everything before it.
#pragma once
#include <array>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace mm {

// A file the reader refuses (the reference's Error::Parse / UnsupportedVersion /
// Io for shards, MIDMAN_ERR_OTHER at the C ABI).
struct ShardError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

struct TokenShard {
  uint32_t vocab_size = 0, eos = 0;
  std::vector<uint32_t> tokens;
};

// SHA-256 (FIPS 180-4) of `n` bytes.
std::array<uint8_t, 32> sha256(const uint8_t* data, size_t n);

// TokenShard::from_bytes (shard.rs:137-219): the magic, the version, the width for
// the vocabulary, the end-of-text id, the exact length, the checksum and every id.
TokenShard parse_token_shard(const std::vector<uint8_t>& bytes);
TokenShard load_token_shard(const std::string& path);

// TokenShard::new (shard.rs:59-82): throws std::invalid_argument for a vocabulary of
// 0, an end-of-text id or a token not below the vocabulary size.
void check_token_shard(uint32_t vocab_size, uint32_t eos, const uint32_t* tokens, size_t n);
// TokenShard::to_bytes (shard.rs:113-135).
std::vector<uint8_t> token_shard_bytes(uint32_t vocab_size, uint32_t eos, const uint32_t* tokens, size_t n);
// TokenShard::save (shard.rs:221-253): written to `path`.tmp, flushed to disk, then
// renamed over `path`; the temporary file is removed on failure (ShardError).
void save_token_shard(const std::string& path, uint32_t vocab_size, uint32_t eos, const uint32_t* tokens, size_t n);

}  // namespace mm
