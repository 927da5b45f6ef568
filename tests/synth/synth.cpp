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

struct Spec {
  Json config;
  std::string format;
  uint64_t seed = 0;
  float sd = 0.02f;
  size_t d = 0, ffn = 0, layers = 0, heads = 0, kv_heads = 0, hd = 0, vocab = 0;
  bool tied = true;
  std::string prefix;     // start of every tensor name ("thinker." ...)
  std::string config_at;  // key path the settings are nested under ("a.b.")
};

void write_matrix(GgufWriter* w, const Spec& s, const std::string& name, size_t n, size_t k, bool declare) {
  if (s.format == "q8_0") {
    if (k % 32) throw Error("q8_0 needs k to be a multiple of 32");
    if (declare) return w->add(name + ".weight", Q8_0, {k, n});
    std::vector<uint8_t> bytes(n * (k / 32) * 34);
    parallel_rows(n, [&](size_t r) {
      std::vector<float> row(k);
      normal_row(s.seed, name, r, k, s.sd, row.data());
      for (size_t b = 0; b < k / 32; ++b) q8_0_block(row.data() + b * 32, bytes.data() + (r * (k / 32) + b) * 34);
    });
    w->put(bytes.data(), bytes.size());
  } else if (s.format == "int8") {
    if (declare) {
      w->add(name + ".weight", I8, {k, n});
      w->add(name + ".scales", F32, {n});
      return;
    }
    std::vector<int8_t> codes(n * k);
    std::vector<float> scales(n);
    parallel_rows(n, [&](size_t r) {
      std::vector<float> row(k);
      normal_row(s.seed, name, r, k, s.sd, row.data());
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
      w->add(name + ".qweight", I8, {row_bytes, n});
      w->add(name + ".scales", F32, {k / 128, n});
      return;
    }
    std::vector<uint8_t> packed(n * row_bytes);
    std::vector<float> scales(n * (k / 128));
    parallel_rows(n, [&](size_t r) {
      std::vector<float> row(k);
      normal_row(s.seed, name, r, k, s.sd, row.data());
      double sum = 0;
      for (float v : row) sum += std::fabs(v);
      float absmean = (float)(sum / (double)k);
      for (size_t g = 0; g < k / 128; ++g) scales[r * (k / 128) + g] = absmean;
      Xorshift codes = stream(s.seed, name + ".codes", r);
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
    throw Error("synthetic format must be q8_0, int8 or ternary, not " + s.format);
  }
}

void write_table(GgufWriter* w, const Spec& s, const std::string& name, size_t n, size_t k, bool declare) {
  if (s.format == "int8") {
    if (k % 32) throw Error("an int8 table needs k to be a multiple of 32");
    if (declare) {
      w->add(name + ".weight", I8, {k, n});
      w->add(name + ".scales", F32, {k / 32, n});
      return;
    }
    std::vector<int8_t> codes(n * k);
    std::vector<float> scales(n * (k / 32));
    parallel_rows(n, [&](size_t r) {
      std::vector<float> row(k);
      normal_row(s.seed, name, r, k, s.sd, row.data());
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
  write_matrix(w, q, name, n, k, declare);
}

void write_norm(GgufWriter* w, const std::string& name, size_t n, bool declare) {
  if (declare) return w->add(name, F32, {n});
  std::vector<float> ones(n, 1.0f);
  w->put(ones.data(), n * 4);
}

void walk(GgufWriter* w, const Spec& s, bool declare) {
  bool qk_norm = s.config.string_or("model_type", "qwen3") == "qwen3";
  for (size_t l = 0; l < s.layers; ++l) {
    std::string p = s.prefix + "model.layers." + std::to_string(l);
    write_norm(w, p + ".input_layernorm.weight", s.d, declare);
    write_matrix(w, s, p + ".self_attn.q_proj", s.heads * s.hd, s.d, declare);
    write_matrix(w, s, p + ".self_attn.k_proj", s.kv_heads * s.hd, s.d, declare);
    write_matrix(w, s, p + ".self_attn.v_proj", s.kv_heads * s.hd, s.d, declare);
    if (qk_norm) {
      write_norm(w, p + ".self_attn.q_norm.weight", s.hd, declare);
      write_norm(w, p + ".self_attn.k_norm.weight", s.hd, declare);
    }
    write_matrix(w, s, p + ".self_attn.o_proj", s.d, s.heads * s.hd, declare);
    write_norm(w, p + ".post_attention_layernorm.weight", s.d, declare);
    write_matrix(w, s, p + ".mlp.gate_proj", s.ffn, s.d, declare);
    write_matrix(w, s, p + ".mlp.up_proj", s.ffn, s.d, declare);
    write_matrix(w, s, p + ".mlp.down_proj", s.d, s.ffn, declare);
  }
  write_norm(w, s.prefix + "model.norm.weight", s.d, declare);
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
  std::string cfg = config_text(s);
  FILE* f = fopen((dir + "/config.json").c_str(), "wb");
  if (!f) throw Error("cannot write " + dir + "/config.json (does the folder exist?)");
  fwrite(cfg.data(), 1, cfg.size(), f);
  fclose(f);
  GgufWriter w;
  w.meta("general.architecture", type);
  w.meta("trit.synthetic", spec_json);
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
