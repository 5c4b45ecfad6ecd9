// The state of a training run in one safetensors file, readable and writable by
// the reference: crates/midman-checkpoint/src/safetensors.rs (the container) and
// crates/midman-training/src/state.rs + config.rs (what a run stores in it).
#pragma once
#include <cstdint>
#include <functional>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace mm {

// The reference's error kinds for state files, which its C ABI reports as
// MIDMAN_ERR_ARGUMENT (Error::InvalidArgument: a state that does not fit the
// run), MIDMAN_ERR_OTHER (Error::Parse / Io / UnsupportedVersion: a file that is
// not a valid state file) and MIDMAN_ERR_SHAPE (Error::Shape).
struct StateError : std::invalid_argument {
  using std::invalid_argument::invalid_argument;
};
struct StateFormatError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct StateShapeError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// ---------------------------------------------------------------- container

struct SafeTensor {
  std::string name;
  std::vector<uint64_t> shape;
  uint64_t begin = 0, end = 0;  // byte range inside the data section
};

// A parsed file: every check of safetensors.rs:270-353 passed.
struct SafeFile {
  std::map<std::string, std::string> metadata;
  std::vector<SafeTensor> tensors;  // in the order of their data
  std::vector<uint8_t> bytes;       // the whole file
  uint64_t data_offset = 0;         // start of the data section in `bytes`
  const SafeTensor* find(const std::string& name) const;
  // The tensor's values (little-endian f32) copied out of the file.
  void copy_values(const SafeTensor& t, float* out) const;
};

SafeFile parse_safetensors(std::vector<uint8_t> bytes);
SafeFile load_safetensors(const std::string& path);

// One tensor to write; `fill` produces its values when its turn comes, so a
// file larger than host memory needs only one tensor in memory at a time.
struct WriteTensor {
  std::string name;
  std::vector<uint64_t> shape;
  uint64_t count;
};
// Writes `<path>.tmp`, flushes it to disk and renames it over `path`
// (safetensors.rs:224-253). Layout as safetensors.rs:139-222: the metadata
// object first, then tensors sorted by name with consecutive byte ranges; the
// header is padded with spaces to a multiple of eight bytes.
void save_safetensors(const std::string& path, const std::map<std::string, std::string>& metadata,
                      std::vector<WriteTensor> tensors,
                      const std::function<void(const WriteTensor&, std::vector<float>&)>& fill);

// Rust's `Display` of an f32 (the shortest decimal that reads back as the same
// value, never in exponent form), which the reference uses for settings.
std::string rust_f32(float v);

// ---------------------------------------------------------------- training state

// TrainConfig (crates/midman-training/src/config.rs:16-41).
struct TrainSettings {
  uint64_t batch_size = 0, seq_len = 0, seed = 0;
  float max_lr = 0, min_lr = 0;
  uint64_t warmup_steps = 0, total_steps = 0;
  float beta1 = 0, beta2 = 0, eps = 0, weight_decay = 0, clip_norm = 0;
};
// The twelve `train.*` metadata entries (config.rs:113-131).
std::vector<std::pair<std::string, std::string>> settings_entries(const TrainSettings& s);

// Progress (state.rs:34-43).
struct Progress {
  uint64_t step = 0, epoch = 0, position = 0;
};

// Reads and checks the header entries of a state file (state.rs:125-173).
Progress progress_of(const std::map<std::string, std::string>& metadata);

// Every setting must be present and equal (config.rs:138-157).
void check_settings(const TrainSettings& s, const std::map<std::string, std::string>& metadata);

// A parameter of the run: its name and shape (MidManModel::parameters order).
struct StateParam {
  std::string name;
  std::vector<uint64_t> shape;
  uint64_t offset, count;  // in the flat parameter vector
};

// Writes the state: `param/<name>` for every parameter and, after the first
// step, `adamw.m/<name>` and `adamw.v/<name>` (state.rs:45-116). read(which,
// offset, count, out) fetches values: which 0 = parameters, 2 = m, 3 = v.
void save_state(const std::string& path, const std::vector<StateParam>& params, const Progress& progress,
                const TrainSettings& settings,
                const std::function<void(int, uint64_t, uint64_t, float*)>& read);

// Reads a state file into flat host vectors (params, m, v; m and v empty for a
// run with no step) after every check of state.rs:176-288 and adamw.rs:95-130,
// so that the caller changes nothing unless this returns.
struct LoadedState {
  Progress progress;
  std::vector<float> params, m, v;
};
LoadedState load_state(const std::string& path, const std::vector<StateParam>& params, uint64_t total,
                       const TrainSettings& settings);

}  // namespace mm
