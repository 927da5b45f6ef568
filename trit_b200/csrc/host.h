// Host-side helpers of libtrit_cuda: errors, f16 bits, a small JSON reader,
// and a GGUF v3 reader/writer (the container that Trit reads in
// src/models/gguf/mod.rs:147-215).
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "types.h"

namespace trit {

struct Error : std::runtime_error {
  explicit Error(const std::string& s) : std::runtime_error(s) {}
};

// IEEE f32 -> f16 bits, nearest with ties to even, subnormals kept; the
// conversion of src/cpu/tensors.rs:542-580.
uint16_t f32_to_f16(float value);
float f16_to_f32(uint16_t half);

// ---------------------------------------------------------------- JSON ----
// Objects, arrays, strings, numbers, true/false/null. Enough for
// config.json and the option strings of the C ABI.
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> items;
  std::vector<std::pair<std::string, Json>> fields;

  static Json parse(const std::string& text);
  const Json* get(const std::string& key) const;  // dotted path a.b.c
  bool has(const std::string& key) const { return get(key) != nullptr; }
  double number(const std::string& key, double dflt) const;
  long integer(const std::string& key) const;  // throws when missing
  std::string string_or(const std::string& key, const std::string& dflt) const;
  bool flag(const std::string& key, bool dflt) const;
};

// ---------------------------------------------------------------- GGUF ----
enum GgmlType : uint32_t { F32 = 0, F16 = 1, Q8_0 = 8, I8 = 24, I32 = 26 };
size_t ggml_size(uint32_t type, uint64_t count);

struct GgufTensor {
  std::string name;
  uint32_t type = 0;
  std::vector<uint64_t> dims;  // ne[0] innermost
  uint64_t offset = 0;         // from the start of the data section
  const uint8_t* data = nullptr;
  size_t bytes = 0;
  uint64_t count() const {
    uint64_t c = 1;
    for (auto d : dims) c *= d;
    return c;
  }
};

class GgufFile {
 public:
  explicit GgufFile(const std::string& path);
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;
  const GgufTensor* find(const std::string& name) const;
  const GgufTensor& at(const std::string& name) const;
  const std::map<std::string, std::string>& strings() const { return strings_; }

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, GgufTensor> tensors_;
  std::map<std::string, std::string> strings_;
};

// Streams a GGUF file: declare every tensor (`add`), then `open` writes the
// header and the tensor list, then `put` writes each tensor's bytes in the
// order of the declarations.
class GgufWriter {
 public:
  ~GgufWriter();
  void meta(const std::string& key, const std::string& value) { meta_.emplace_back(key, value); }
  void add(const std::string& name, uint32_t type, std::vector<uint64_t> dims);
  void open(const std::string& path);
  void put(const void* bytes, size_t size);
  void close();

 private:
  std::vector<std::pair<std::string, std::string>> meta_;
  std::vector<GgufTensor> infos_;
  size_t next_ = 0;
  uint64_t written_ = 0;
  std::FILE* file_ = nullptr;
};

// The decoder settings of a model folder's config.json, as Config::parse
// (causal_lm.rs:41-77) reads them: key and value heads, widths, head_dim
// (default hidden / heads), eps (1e-6), rope_theta (1e6), the Granite
// multipliers, tie_word_embeddings, and q/k norms iff model_type is
// "qwen3". Throws for a model this engine does not run.
struct ModelConfig {
  DConfig cfg;
  std::string type;
  bool qk_norm = false;
  bool tied = false;
  float rope_base = 1e6f;
  float attention_multiplier = 1.0f;  // when cfg.has_q_scale
};
// `at` is the key path the settings sit under ("" or, in Qwen3-ASR,
// "thinker_config.text_config.").
ModelConfig parse_model_config(const std::string& json_text, const std::string& at = "");
ModelConfig read_model_config(const std::string& dir, const std::string& at = "");

// A JSON description of a model folder without touching a GPU: its
// settings, the storage of its products and token tables, and the bytes a
// greedy step reads from device memory.
// `prefix` starts every tensor name ("", "thinker.", "llm." ...).
std::string describe_model(const std::string& dir, const std::string& at = "", const std::string& prefix = "");

}  // namespace trit
