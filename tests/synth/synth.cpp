// Seeded synthetic decoder models for the benchmarks and tests (test
// infrastructure, built into tests/synth/libtrit_synth.so, not into the
// product library): a model
// folder (config.json + model.gguf) with the tensor names of a Hugging
// Face Qwen3/Llama checkpoint, which trit_lm_load and the CPU oracle read.
//
// Weights are N(0, std) from a 64-bit xorshift* stream per (tensor, row)
// (the generator of the reference's kernel bench, src/cpu/v2/bench.rs:14-30)
// through Box-Muller; RMSNorm weights are 1. Formats:
//   q8_0    : every matrix as ggml Q8_0 blocks (quantize_row_q8_0_ref,
//             src/cpu/gemm.rs:53-76); token table Q8_0.
//   int8    : per-output-row symmetric int8 (scale = absmax/127, codes
//             round-half-even, src/cpu/int8.rs:176-186) as `.weight` (I8)
//             + `.scales` (F32, one per row); token table int8 with one f32
//             scale per 32 values (Q8::quantize, src/cpu/gemm.rs:116-150).
//   ternary : codes {-1,0,+1} with P(0)=0.4, P(+-1)=0.3, five base-3 digits
//             a byte (`.qweight`, src/cpu/kernels.rs:91-130) + `.scales`
//             (F32, [rows][k/128], the row's mean |w| of an N(0,std) draw);
//             token table Q8_0, as Dense::table keeps it (never ternary).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>

#include "../../trit_b200/csrc/host.h"
#include "trit_synth.h"

namespace trit {
namespace {

uint64_t splitmix(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

uint64_t fnv1a(const std::string& s) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (unsigned char c : s) {
    h ^= c;
    h *= 0x100000001b3ull;
  }
  return h;
}

struct Xorshift {
  uint64_t s;
  uint64_t next() {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s * 0x2545F4914F6CDD1Dull;
  }
  double unit() { return (double)(next() >> 11) * 0x1p-53; }  // [0, 1)
};

Xorshift stream(uint64_t seed, const std::string& name, uint64_t row) {
  Xorshift r{splitmix(seed ^ fnv1a(name) ^ splitmix(row + 1))};
  if (!r.s) r.s = 1;
  return r;
}

void normal_row(uint64_t seed, const std::string& name, uint64_t row, size_t k, float sd, float* out) {
  Xorshift r = stream(seed, name, row);
  for (size_t i = 0; i < k; i += 2) {
    double u1 = ((double)(r.next() >> 11) + 1.0) * 0x1p-53;  // (0, 1]
    double u2 = r.unit();
    double rad = std::sqrt(-2.0 * std::log(u1));
    double z0 = rad * std::cos(2.0 * M_PI * u2), z1 = rad * std::sin(2.0 * M_PI * u2);
    out[i] = (float)(sd * z0);
    if (i + 1 < k) out[i + 1] = (float)(sd * z1);
  }
}

template <class F>
void parallel_rows(size_t n, F f) {
  unsigned threads = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
  std::vector<std::thread> pool;
  for (unsigned t = 0; t < threads; ++t)
    pool.emplace_back([&, t]() {
      for (size_t r = t; r < n; r += threads) f(r);
    });
  for (auto& th : pool) th.join();
}

// ggml quantize_row_q8_0_ref: d = max|x|/127, codes round-half-away(x/d... * 1/d).
void q8_0_block(const float* v, uint8_t* out) {
  float max = 0.0f;
  for (int i = 0; i < 32; ++i) max = std::max(max, std::fabs(v[i]));
  float d = max / 127.0f;
  float inv = d != 0.0f ? 1.0f / d : 0.0f;
  uint16_t h = f32_to_f16(d);
  out[0] = (uint8_t)(h & 0xff);
  out[1] = (uint8_t)(h >> 8);
  for (int i = 0; i < 32; ++i) {
    float c = std::round(v[i] * inv);
    c = std::min(std::max(c, -128.0f), 127.0f);
    out[2 + i] = (uint8_t)(int8_t)c;
  }
}

float row_scale(float max) { return max > 0.0f ? max / 127.0f : 1.0f; }
int8_t code_of(float v, float scale) {
  float c = std::nearbyint(v / scale);
  return (int8_t)std::min(std::max(c, -127.0f), 127.0f);
}

// A model file being written: declare every tensor (`add`, with ggml type
// codes and dims innermost first), then `open` writes the header and `put`
// writes each tensor's bytes in the order of the declarations.
class Writer {
 public:
  virtual ~Writer() = default;
  virtual void add(const std::string& name, uint32_t type, std::vector<uint64_t> dims) = 0;
  virtual void open(const std::string& path) = 0;
  virtual void put(const void* bytes, size_t size) = 0;
  virtual void close() = 0;
};

struct Declared {
  std::string name;
  uint32_t type;
  std::vector<uint64_t> dims;
  size_t bytes;
};

// GGUF v3 (src/models/gguf/mod.rs:147-215 reads it): typed metadata, then
// the tensor list, then the data, each tensor 32-byte aligned.
class GgufOut : public Writer {
 public:
  ~GgufOut() override {
    if (file_) std::fclose(file_);
  }
  void meta_str(const std::string& key, const std::string& v) { meta_.push_back({key, 8, v, 0}); }
  void meta_u32(const std::string& key, uint32_t v) { meta_.push_back({key, 4, "", (double)v}); }
  void meta_f32(const std::string& key, float v) { meta_.push_back({key, 6, "", (double)v}); }
  void meta_bool(const std::string& key, bool v) { meta_.push_back({key, 7, "", v ? 1.0 : 0.0}); }
  void add(const std::string& name, uint32_t type, std::vector<uint64_t> dims) override {
    uint64_t count = 1;
    for (auto d : dims) count *= d;
    infos_.push_back({name, type, std::move(dims), ggml_size(type, count)});
  }
  void open(const std::string& path) override {
    file_ = std::fopen(path.c_str(), "wb");
    if (!file_) throw Error("cannot write " + path);
    auto w32 = [&](uint32_t v) { w(&v, 4); };
    auto w64 = [&](uint64_t v) { w(&v, 8); };
    auto ws = [&](const std::string& s) { w64(s.size()); w(s.data(), s.size()); };
    w("GGUF", 4);
    w32(3);
    w64(infos_.size());
    w64(meta_.size() + 1);
    ws("general.alignment");
    w32(4);
    w32(32);
    for (auto& m : meta_) {
      ws(m.key);
      w32(m.type);
      if (m.type == 8) ws(m.str);
      else if (m.type == 4) w32((uint32_t)m.num);
      else if (m.type == 6) { float f = (float)m.num; w(&f, 4); }
      else { uint8_t b = m.num != 0; w(&b, 1); }
    }
    uint64_t offset = 0;
    for (auto& t : infos_) {
      ws(t.name);
      w32((uint32_t)t.dims.size());
      for (auto d : t.dims) w64(d);
      w32(t.type);
      w64(offset);
      offset = (offset + t.bytes + 31) / 32 * 32;
    }
    static const uint8_t zeros[32] = {0};
    w(zeros, (32 - written_ % 32) % 32);
    written_ = 0;
  }
  void put(const void* bytes, size_t size) override {
    if (next_ >= infos_.size() || size != infos_[next_].bytes) throw Error("GGUF writer: tensor size mismatch");
    static const uint8_t zeros[32] = {0};
    w(bytes, size);
    w(zeros, (32 - written_ % 32) % 32);
    ++next_;
  }
  void close() override {
    if (next_ != infos_.size()) throw Error("GGUF writer: not every tensor was written");
    if (file_ && std::fclose(file_) != 0) {
      file_ = nullptr;
      throw Error("GGUF writer: close failed");
    }
    file_ = nullptr;
  }

 private:
  struct Meta {
    std::string key;
    uint32_t type;
    std::string str;
    double num;
  };
  void w(const void* p, size_t n) {
    if (n && std::fwrite(p, 1, n, file_) != n) throw Error("GGUF writer: write failed");
    written_ += n;
  }
  std::vector<Meta> meta_;
  std::vector<Declared> infos_;
  size_t next_ = 0;
  uint64_t written_ = 0;
  std::FILE* file_ = nullptr;
};

// One safetensors file: an 8-byte header length, a JSON header with each
// tensor's dtype, shape (outermost first) and byte range, then the data.
class SafetensorsOut : public Writer {
 public:
  ~SafetensorsOut() override {
    if (file_) std::fclose(file_);
  }
  void add(const std::string& name, uint32_t type, std::vector<uint64_t> dims) override {
    uint64_t count = 1;
    for (auto d : dims) count *= d;
    infos_.push_back({name, type, std::move(dims), ggml_size(type, count)});
  }
  void open(const std::string& path) override {
    std::string h = "{\"__metadata__\": {\"format\": \"pt\"}";
    uint64_t at = 0;
    for (auto& t : infos_) {
      const char* dtype = t.type == F32 ? "F32" : t.type == F16 ? "F16" : t.type == BF16 ? "BF16" : t.type == I8 ? "I8" : "I32";
      h += ", \"" + t.name + "\": {\"dtype\": \"" + dtype + "\", \"shape\": [";
      for (size_t i = t.dims.size(); i-- > 0;) h += std::to_string(t.dims[i]) + (i ? ", " : "");
      h += "], \"data_offsets\": [" + std::to_string(at) + ", " + std::to_string(at + t.bytes) + "]}";
      at += t.bytes;
    }
    h += "}";
    while (h.size() % 8) h += ' ';
    file_ = std::fopen(path.c_str(), "wb");
    if (!file_) throw Error("cannot write " + path);
    uint64_t n = h.size();
    if (std::fwrite(&n, 8, 1, file_) != 1 || std::fwrite(h.data(), 1, h.size(), file_) != h.size())
      throw Error("safetensors writer: write failed");
  }
  void put(const void* bytes, size_t size) override {
    if (next_ >= infos_.size() || size != infos_[next_].bytes) throw Error("safetensors writer: tensor size mismatch");
    if (size && std::fwrite(bytes, 1, size, file_) != size) throw Error("safetensors writer: write failed");
    ++next_;
  }
  void close() override {
    if (next_ != infos_.size()) throw Error("safetensors writer: not every tensor was written");
    if (file_ && std::fclose(file_) != 0) {
      file_ = nullptr;
      throw Error("safetensors writer: close failed");
    }
    file_ = nullptr;
  }

 private:
  std::vector<Declared> infos_;
  size_t next_ = 0;
  std::FILE* file_ = nullptr;
};

struct Spec {
  Json config;
  std::string format;
  uint64_t seed = 0;
  float sd = 0.02f;
  size_t d = 0, ffn = 0, layers = 0, heads = 0, kv_heads = 0, hd = 0, vocab = 0;
  bool tied = true;
  std::string prefix;     // start of every tensor name ("thinker." ...)
  std::string config_at;  // key path the settings are nested under ("a.b.")
  std::string dtype = "f32";  // the float format's element type: f32, f16 or bf16
  std::string names = "hf";   // "hf", or "transcribe": dec.* names under the file's arch
  // The name a tensor's values are drawn for: its Hugging Face name without
  // the model's prefix, so one seed gives the same weights under any
  // prefix and any file form.
  std::string seed_name(const std::string& hf) const {
    return hf.compare(0, prefix.size(), prefix) == 0 ? hf.substr(prefix.size()) : hf;
  }
  // The transcribe.cpp name of a Hugging Face tensor name (its inverse is
  // hf_decoder_name in the product's host.cpp).
  std::string out_name(const std::string& hf) const {
    if (names != "transcribe") return hf;
    std::string n = hf.substr(prefix.size());
    auto starts = [&](const char* p) { return n.compare(0, std::strlen(p), p) == 0; };
    if (starts("model.embed_tokens.")) return "dec.token_embd." + n.substr(19);
    if (starts("model.norm.")) return "dec.output_norm." + n.substr(11);
    if (starts("lm_head.")) return "dec.output." + n.substr(8);
    n = n.substr(std::strlen("model.layers."));
    const size_t dot = n.find('.');
    const std::string layer = n.substr(0, dot), part = n.substr(dot + 1);
    static const char* table[][2] = {
        {"input_layernorm.", "norm_attn."},   {"post_attention_layernorm.", "norm_ffn."},
        {"self_attn.q_norm.", "attn.q_norm."}, {"self_attn.k_norm.", "attn.k_norm."},
        {"self_attn.q_proj.", "attn.q."},      {"self_attn.k_proj.", "attn.k."},
        {"self_attn.v_proj.", "attn.v."},      {"self_attn.o_proj.", "attn.o."},
        {"mlp.gate_proj.", "ffn.gate."},       {"mlp.up_proj.", "ffn.up."},
        {"mlp.down_proj.", "ffn.down."},
    };
    for (auto& row : table)
      if (part.compare(0, std::strlen(row[0]), row[0]) == 0)
        return "dec.blocks." + layer + "." + row[1] + part.substr(std::strlen(row[0]));
    throw Error("no transcribe.cpp name for " + hf);
  }
};

// Float rows in the spec's element type.
void put_float_rows(Writer* w, const Spec& s, const std::vector<float>& v) {
  if (s.dtype == "f32") return w->put(v.data(), v.size() * 4);
  std::vector<uint16_t> h(v.size());
  for (size_t i = 0; i < v.size(); ++i) {
    if (s.dtype == "f16") {
      h[i] = f32_to_f16(v[i]);
    } else {
      uint32_t u;
      std::memcpy(&u, &v[i], 4);
      u += 0x7fff + ((u >> 16) & 1);  // bf16, nearest even (these values are finite)
      h[i] = (uint16_t)(u >> 16);
    }
  }
  w->put(h.data(), h.size() * 2);
}
uint32_t float_type(const Spec& s) { return s.dtype == "f32" ? F32 : s.dtype == "f16" ? F16 : BF16; }

void write_matrix(Writer* w, const Spec& s, const std::string& hf, size_t n, size_t k, bool declare) {
  const std::string name = s.out_name(hf + ".weight");
  const std::string base = name.substr(0, name.size() - 7);  // without ".weight"
  if (s.format == "float") {
    if (declare) return w->add(name, float_type(s), {k, n});
    std::vector<float> all(n * k);
    parallel_rows(n, [&](size_t r) { normal_row(s.seed, s.seed_name(hf), r, k, s.sd, all.data() + r * k); });
    return put_float_rows(w, s, all);
  }
  if (s.format == "q8_0") {
    if (k % 32) throw Error("q8_0 needs k to be a multiple of 32");
    if (declare) return w->add(base + ".weight", Q8_0, {k, n});
    std::vector<uint8_t> bytes(n * (k / 32) * 34);
    parallel_rows(n, [&](size_t r) {
      std::vector<float> row(k);
      normal_row(s.seed, s.seed_name(hf), r, k, s.sd, row.data());
      for (size_t b = 0; b < k / 32; ++b) q8_0_block(row.data() + b * 32, bytes.data() + (r * (k / 32) + b) * 34);
    });
    w->put(bytes.data(), bytes.size());
  } else if (s.format == "int8") {
    if (declare) {
      w->add(base + ".weight", I8, {k, n});
      w->add(base + ".scales", F32, {n});
      return;
    }
    std::vector<int8_t> codes(n * k);
    std::vector<float> scales(n);
    parallel_rows(n, [&](size_t r) {
      std::vector<float> row(k);
      normal_row(s.seed, s.seed_name(hf), r, k, s.sd, row.data());
      float max = 0.0f;
      for (float v : row) max = std::max(max, std::fabs(v));
      scales[r] = row_scale(max);
      for (size_t i = 0; i < k; ++i) codes[r * k + i] = code_of(row[i], scales[r]);
    });
    w->put(codes.data(), codes.size());
    w->put(scales.data(), scales.size() * 4);
  } else if (s.format == "ternary") {
    if (k % 128) throw Error("ternary needs k to be a multiple of 128");
    size_t row_bytes = (k + 4) / 5;
    if (declare) {
      w->add(base + ".qweight", I8, {row_bytes, n});
      w->add(base + ".scales", F32, {k / 128, n});
      return;
    }
    std::vector<uint8_t> packed(n * row_bytes);
    std::vector<float> scales(n * (k / 128));
    parallel_rows(n, [&](size_t r) {
      std::vector<float> row(k);
      normal_row(s.seed, s.seed_name(hf), r, k, s.sd, row.data());
      double sum = 0;
      for (float v : row) sum += std::fabs(v);
      float absmean = (float)(sum / (double)k);
      for (size_t g = 0; g < k / 128; ++g) scales[r * (k / 128) + g] = absmean;
      Xorshift codes = stream(s.seed, s.seed_name(hf) + ".codes", r);
      uint8_t* dst = packed.data() + r * row_bytes;
      for (size_t b = 0; b < row_bytes; ++b) {
        unsigned byte = 0, place = 1;
        for (int dd = 0; dd < 5; ++dd) {
          unsigned code = 1;  // a code past k pads the last byte with zeros (code 1)
          if (b * 5 + dd < k) {
            double u = codes.unit();
            code = u < 0.4 ? 1 : (u < 0.7 ? 2 : 0);
          }
          byte += code * place;
          place *= 3;
        }
        dst[b] = (uint8_t)byte;
      }
    });
    w->put(packed.data(), packed.size());
    w->put(scales.data(), scales.size() * 4);
  } else {
    throw Error("synthetic format must be q8_0, float, int8 or ternary, not " + s.format);
  }
}

void write_table(Writer* w, const Spec& s, const std::string& hf, size_t n, size_t k, bool declare) {
  const std::string name = s.out_name(hf + ".weight");
  const std::string base = name.substr(0, name.size() - 7);
  if (s.format == "float") return write_matrix(w, s, hf, n, k, declare);
  if (s.format == "int8") {
    if (k % 32) throw Error("an int8 table needs k to be a multiple of 32");
    if (declare) {
      w->add(base + ".weight", I8, {k, n});
      w->add(base + ".scales", F32, {k / 32, n});
      return;
    }
    std::vector<int8_t> codes(n * k);
    std::vector<float> scales(n * (k / 32));
    parallel_rows(n, [&](size_t r) {
      std::vector<float> row(k);
      normal_row(s.seed, s.seed_name(hf), r, k, s.sd, row.data());
      for (size_t g = 0; g < k / 32; ++g) {
        float max = 0.0f;
        for (int i = 0; i < 32; ++i) max = std::max(max, std::fabs(row[g * 32 + i]));
        float sc = row_scale(max);
        scales[r * (k / 32) + g] = sc;
        for (int i = 0; i < 32; ++i) codes[r * k + g * 32 + i] = code_of(row[g * 32 + i], sc);
      }
    });
    w->put(codes.data(), codes.size());
    w->put(scales.data(), scales.size() * 4);
    return;
  }
  Spec q = s;
  q.format = "q8_0";
  write_matrix(w, q, hf, n, k, declare);
}

void write_norm(Writer* w, const Spec& s, const std::string& hf, size_t n, bool declare) {
  if (declare) return w->add(s.out_name(hf), F32, {n});
  std::vector<float> ones(n, 1.0f);
  w->put(ones.data(), n * 4);
}

void walk(Writer* w, const Spec& s, bool declare) {
  bool qk_norm = s.config.string_or("model_type", "qwen3") == "qwen3";
  for (size_t l = 0; l < s.layers; ++l) {
    std::string p = s.prefix + "model.layers." + std::to_string(l);
    write_norm(w, s, p + ".input_layernorm.weight", s.d, declare);
    write_matrix(w, s, p + ".self_attn.q_proj", s.heads * s.hd, s.d, declare);
    write_matrix(w, s, p + ".self_attn.k_proj", s.kv_heads * s.hd, s.d, declare);
    write_matrix(w, s, p + ".self_attn.v_proj", s.kv_heads * s.hd, s.d, declare);
    if (qk_norm) {
      write_norm(w, s, p + ".self_attn.q_norm.weight", s.hd, declare);
      write_norm(w, s, p + ".self_attn.k_norm.weight", s.hd, declare);
    }
    write_matrix(w, s, p + ".self_attn.o_proj", s.d, s.heads * s.hd, declare);
    write_norm(w, s, p + ".post_attention_layernorm.weight", s.d, declare);
    write_matrix(w, s, p + ".mlp.gate_proj", s.ffn, s.d, declare);
    write_matrix(w, s, p + ".mlp.up_proj", s.ffn, s.d, declare);
    write_matrix(w, s, p + ".mlp.down_proj", s.d, s.ffn, declare);
  }
  write_norm(w, s, s.prefix + "model.norm.weight", s.d, declare);
  write_table(w, s, s.prefix + "model.embed_tokens", s.vocab, s.d, declare);
  if (!s.tied) write_table(w, s, s.prefix + "lm_head", s.vocab, s.d, declare);
}

std::string config_text(const Spec& s) {
  const Json& c = s.config;
  char buf[1024];
  snprintf(buf, sizeof buf,
           "{\n  \"model_type\": \"%s\",\n  \"hidden_size\": %zu,\n  \"intermediate_size\": %zu,\n"
           "  \"num_hidden_layers\": %zu,\n  \"num_attention_heads\": %zu,\n  \"num_key_value_heads\": %zu,\n"
           "  \"head_dim\": %zu,\n  \"vocab_size\": %zu,\n  \"rms_norm_eps\": %.9g,\n  \"rope_theta\": %.9g,\n"
           "  \"tie_word_embeddings\": %s",
           c.string_or("model_type", "qwen3").c_str(), s.d, s.ffn, s.layers, s.heads, s.kv_heads, s.hd, s.vocab,
           c.number("rms_norm_eps", 1e-6), c.number("rope_theta", 1e6), s.tied ? "true" : "false");
  std::string out = buf;
  // Granite's multipliers, when the spec gives them.
  for (const char* key : {"embedding_multiplier", "attention_multiplier", "residual_multiplier", "logits_scaling"})
    if (c.has(key)) {
      snprintf(buf, sizeof buf, ",\n  \"%s\": %.9g", key, c.number(key, 1.0));
      out += buf;
    }
  out += "\n}";
  // Nest the settings under config_at ("thinker_config.text_config.").
  std::vector<std::string> parts;
  for (size_t from = 0; from < s.config_at.size();) {
    size_t dot = s.config_at.find('.', from);
    if (dot == std::string::npos) dot = s.config_at.size();
    if (dot > from) parts.push_back(s.config_at.substr(from, dot - from));
    from = dot + 1;
  }
  std::string tail;
  for (size_t i = parts.size(); i-- > 0;) {
    out = "{\"" + parts[i] + "\": " + out;
    tail += "}";
  }
  snprintf(buf, sizeof buf, "\"trit_synthetic\": {\"format\": \"%s\", \"seed\": %llu, \"std\": %.9g}",
           s.format.c_str(), (unsigned long long)s.seed, (double)s.sd);
  if (tail.empty()) out = out.substr(0, out.size() - 2) + ",\n  " + buf + "\n}\n";
  else out += tail + "\n";
  return out;
}

}  // namespace

void synthesize(const std::string& dir, const std::string& spec_json) {
  Json spec = Json::parse(spec_json);
  Spec s;
  const Json* c = spec.get("config");
  if (!c) throw Error("synthetic spec: no config");
  s.config = *c;
  s.format = spec.string_or("format", "q8_0");
  s.seed = (uint64_t)spec.number("seed", 0);
  s.sd = (float)spec.number("std", 0.02);
  s.d = s.config.integer("hidden_size");
  s.ffn = s.config.integer("intermediate_size");
  s.layers = s.config.integer("num_hidden_layers");
  s.heads = s.config.integer("num_attention_heads");
  s.kv_heads = s.config.integer("num_key_value_heads");
  s.hd = s.config.has("head_dim") ? s.config.integer("head_dim") : s.d / std::max<size_t>(1, s.heads);
  s.vocab = s.config.integer("vocab_size");
  s.tied = s.config.flag("tie_word_embeddings", true);
  s.prefix = spec.string_or("prefix", "");
  s.config_at = spec.string_or("config_at", "");
  if (!s.heads || !s.kv_heads || s.heads % s.kv_heads) throw Error("synthetic spec: heads must share kv heads evenly");
  std::string type = s.config.string_or("model_type", "qwen3");
  if (type != "qwen3" && type != "llama" && type != "mistral" && type != "granite")
    throw Error("synthetic spec: model_type " + type);
  s.dtype = spec.string_or("dtype", "f32");
  s.names = spec.string_or("names", "hf");
  const std::string container = spec.string_or("container", "gguf");
  if (s.format == "float" && s.dtype != "f32" && s.dtype != "f16" && s.dtype != "bf16")
    throw Error("synthetic spec: dtype must be f32, f16 or bf16");
  if (s.names == "transcribe") {
    // One GGUF file as transcribe.cpp writes it: no config.json, the
    // decoder's settings in metadata under stt.<arch>.decoder, dec.* names.
    const std::string arch = spec.string_or("arch", "qwen3_asr");
    const std::string meta = "stt." + (arch == "granite_speech" ? std::string("granite") : arch) + ".decoder";
    s.prefix = arch == "qwen3_asr" ? "thinker." : (arch == "funasr_nano" || arch == "canary_qwen") ? "llm."
                                                                                                     : "language_model.";
    if (container != "gguf") throw Error("synthetic spec: transcribe names come in a GGUF file");
    GgufOut w;
    w.meta_str("general.architecture", arch);
    w.meta_str("trit.synthetic", spec_json);
    w.meta_str(meta + ".hidden_act", "silu");
    w.meta_u32(meta + ".hidden_size", (uint32_t)s.d);
    w.meta_u32(meta + ".intermediate_size", (uint32_t)s.ffn);
    w.meta_u32(meta + ".n_layers", (uint32_t)s.layers);
    w.meta_u32(meta + ".n_heads", (uint32_t)s.heads);
    w.meta_u32(meta + ".n_kv_heads", (uint32_t)s.kv_heads);
    w.meta_u32(meta + ".head_dim", (uint32_t)s.hd);
    w.meta_u32(meta + ".vocab_size", (uint32_t)s.vocab);
    w.meta_f32(meta + ".rms_norm_eps", (float)s.config.number("rms_norm_eps", 1e-6));
    w.meta_f32(meta + ".rope_theta", (float)s.config.number("rope_theta", 1e6));
    w.meta_bool(meta + ".tie_word_embeddings", s.tied);
    walk(&w, s, true);
    w.add("enc.blocks.0.attn.q.weight", F32, {8, 8});  // an encoder tensor the decoder does not read
    w.open(dir + "/" + arch + ".gguf");
    walk(&w, s, false);
    std::vector<float> enc(64, 0.5f);
    w.put(enc.data(), enc.size() * 4);
    w.close();
    return;
  }
  std::string cfg = config_text(s);
  FILE* f = fopen((dir + "/config.json").c_str(), "wb");
  if (!f) throw Error("cannot write " + dir + "/config.json (does the folder exist?)");
  fwrite(cfg.data(), 1, cfg.size(), f);
  fclose(f);
  if (container == "safetensors") {
    SafetensorsOut w;
    walk(&w, s, true);
    w.open(dir + "/model.safetensors");
    walk(&w, s, false);
    w.close();
    return;
  }
  if (container != "gguf") throw Error("synthetic spec: container must be gguf or safetensors");
  GgufOut w;
  w.meta_str("general.architecture", type);
  w.meta_str("trit.synthetic", spec_json);
  walk(&w, s, true);
  w.open(dir + "/model.gguf");
  walk(&w, s, false);
  w.close();
}

}  // namespace trit

namespace {
thread_local std::string g_synth_error;
}  // namespace

extern "C" {

const char* trit_synth_last_error(void) { return g_synth_error.c_str(); }

int trit_synth_model(const char* dir, const char* spec_json) {
  g_synth_error.clear();
  try {
    if (!dir || !spec_json) throw trit::Error("dir or spec_json is NULL");
    trit::synthesize(dir, spec_json);
    return 0;
  } catch (const std::exception& e) {
    g_synth_error = e.what();
  } catch (...) {
    g_synth_error = "internal error in trit_synth";
  }
  return -1;
}

void trit_synth_normal_row(uint64_t seed, const char* name, uint64_t row, size_t k, float sd, float* out) {
  if (name && out) trit::normal_row(seed, name, row, k, sd, out);
}

}  // extern "C"
