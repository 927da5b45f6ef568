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
enum GgmlType : uint32_t { F32 = 0, F16 = 1, Q8_0 = 8, I8 = 24, I32 = 26, BF16 = 30 };
size_t ggml_size(uint32_t type, uint64_t count);
float bf16_to_f32(uint16_t bits);

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

// The tensors of a model's files, mapped read-only: one GGUF file (ggml's
// container, src/models/gguf/mod.rs:147-215) or safetensors files (an
// 8-byte header length, a JSON header of dtype / shape / byte range per
// tensor, the data; src/cpu/tensors.rs:155-180,263-305). Safetensors dtypes
// F32, F16, BF16, I8, U8 and I32 are held under the ggml type codes.
class TensorFiles {
 public:
  static std::unique_ptr<TensorFiles> gguf(const std::string& path);
  static std::unique_ptr<TensorFiles> safetensors(const std::vector<std::string>& paths);
  ~TensorFiles();
  TensorFiles(const TensorFiles&) = delete;
  TensorFiles& operator=(const TensorFiles&) = delete;
  const GgufTensor* find(const std::string& name) const;
  const GgufTensor& at(const std::string& name) const;
  // GGUF metadata: strings, and every scalar (integers, floats, bools) as a double.
  const std::map<std::string, std::string>& strings() const { return strings_; }
  bool number(const std::string& key, double* out) const;
  // Renames every tensor: map(name) is the new name, or "" to drop it.
  template <class F>
  void rename(F map) {
    std::map<std::string, GgufTensor> out;
    for (auto& kv : tensors_) {
      std::string to = map(kv.first);
      if (to.empty()) continue;
      GgufTensor t = kv.second;
      t.name = to;
      out[to] = t;
    }
    tensors_.swap(out);
  }
  const std::vector<std::string>& paths() const { return paths_; }
  const std::string& what() const { return what_; }  // "model.gguf", ... for messages

 private:
  TensorFiles() = default;
  void map_file(const std::string& path, const uint8_t** base, size_t* size);
  std::vector<std::pair<void*, size_t>> maps_;
  std::vector<std::string> paths_;
  std::string what_;
  std::map<std::string, GgufTensor> tensors_;
  std::map<std::string, std::string> strings_;
  std::map<std::string, double> numbers_;
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

// A decoder's settings and tensors from a model folder, in one of three
// forms:
//   - config.json (settings under `at`) + model.gguf with Hugging Face
//     tensor names under `prefix`;
//   - config.json + safetensors files (model.safetensors, the shards of
//     model.safetensors.index.json, or every *.safetensors);
//   - one GGUF file as transcribe.cpp writes it, no config.json: the
//     settings come from its metadata (stt.<arch>.decoder.*, as
//     src/models/gguf/blocks.rs:25-45 reads them) and its `dec.*` tensor
//     names are mapped to Hugging Face names under the family's prefix
//     (src/models/gguf/qwen3_asr.rs:103-136); `at` and `prefix` are not
//     used, the file says where its decoder is.
struct ModelSource {
  ModelConfig mc;
  std::unique_ptr<TensorFiles> files;
  std::string prefix;  // the start of the decoder's tensor names
  std::string format;  // "gguf", "gguf-transcribe" or "safetensors"
};
ModelSource open_model(const std::string& dir, const std::string& at = "", const std::string& prefix = "");

// The tensor-parallel shard of rank `rank` of `size` (the optional 2/4-way
// split of the largest decoder): its query heads (with the key/value heads
// they share, whole GQA groups), its FFN units (gate and up rows kept
// paired) and its rows of the output table. The q/k/v and gate/up products
// split their output rows, o_proj and down_proj their input columns (a
// partial sum per rank, then a sum across the ranks), the token table its
// vocabulary rows (a best token per rank, then the best of those).
struct TpShard {
  int rank = 0, size = 1;
  int heads0 = 0, heads = 0;  // query heads [heads0, heads0 + heads)
  int kv0 = 0, kv = 0;        // key/value heads
  int ffn0 = 0, ffn = 0;      // FFN units
  int vocab0 = 0, vocab = 0;  // output-table rows
};
TpShard tp_shard(const DConfig& full, int rank, int size);

// ggml's quantize_row_q8_0_ref for one block of 32 (Blocks::quantize,
// src/cpu/gemm.rs:53-76): d = max|x| / 127, codes round(x * (1 / d)) half
// away from zero, d stored as f16; out = 2 bytes of d, 32 codes.
void q8_0_quantize_block(const float* v, uint8_t* out);

// A JSON description of a model folder without touching a GPU: its
// settings, the storage of its products and token tables, and the bytes a
// greedy step reads from device memory.
// `prefix` starts every tensor name ("", "thinker.", "llm." ...).
// With tp_size > 1, also the shard of tp_rank ("tp": heads, kv_heads,
// ffn_units, vocab_rows as [first, end) ranges).
std::string describe_model(const std::string& dir, const std::string& at = "", const std::string& prefix = "",
                           int tp_rank = 0, int tp_size = 1);

}  // namespace trit
