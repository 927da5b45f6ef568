#include "host.h"

#include <cmath>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <dirent.h>

#include <algorithm>
#include <set>

namespace trit {

// ------------------------------------------------------------------ f16 --
uint16_t f32_to_f16(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, 4);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
  int32_t exponent = (int32_t)((bits >> 23) & 0xff);
  uint32_t mantissa = bits & 0x7fffff;
  if (exponent == 0xff) return sign | 0x7c00 | (mantissa ? 0x200 : 0);
  int32_t e = exponent - 127 + 15;
  if (e >= 0x1f) return sign | 0x7c00;
  if (e <= 0) {
    if (e < -10) return sign;
    uint32_t full = mantissa | 0x800000;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half = full >> shift, rest = full & ((1u << shift) - 1), mid = 1u << (shift - 1);
    return sign | (uint16_t)(half + ((rest > mid || (rest == mid && (half & 1))) ? 1 : 0));
  }
  uint32_t half = ((uint32_t)e << 10) | (mantissa >> 13), rest = mantissa & 0x1fff;
  return sign | (uint16_t)(half + ((rest > 0x1000 || (rest == 0x1000 && (half & 1))) ? 1 : 0));
}

float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, exponent = (h >> 10) & 0x1f, mantissa = h & 0x3ff, bits;
  if (exponent == 0 && mantissa == 0) {
    bits = sign;
  } else if (exponent == 0) {
    uint32_t e = 113, m = mantissa;
    while (!(m & 0x400)) {
      m <<= 1;
      --e;
    }
    bits = sign | (e << 23) | ((m & 0x3ff) << 13);
  } else if (exponent == 0x1f) {
    bits = sign | 0x7f800000 | (mantissa << 13);
  } else {
    bits = sign | ((exponent + 112) << 23) | (mantissa << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// ----------------------------------------------------------------- JSON --
namespace {
struct Parser {
  const char* p;
  const char* end;
  [[noreturn]] void fail(const char* what) { throw Error(std::string("JSON: ") + what); }
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  std::string str() {
    if (p >= end || *p != '"') fail("expected a string");
    ++p;
    std::string s;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) fail("unterminated escape");
        switch (*p) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u': {
            if (end - p < 5) fail("bad \\u escape");
            unsigned code = (unsigned)std::stoul(std::string(p + 1, 4), nullptr, 16);
            p += 4;
            if (code < 0x80) s += (char)code;
            else if (code < 0x800) { s += (char)(0xc0 | (code >> 6)); s += (char)(0x80 | (code & 0x3f)); }
            else { s += (char)(0xe0 | (code >> 12)); s += (char)(0x80 | ((code >> 6) & 0x3f)); s += (char)(0x80 | (code & 0x3f)); }
            break;
          }
          default: s += *p;
        }
        ++p;
      } else {
        s += *p++;
      }
    }
    if (p >= end) fail("unterminated string");
    ++p;
    return s;
  }
  Json value(int depth) {
    if (depth > 64) fail("nested too deeply");
    ws();
    if (p >= end) fail("ends early");
    Json j;
    if (*p == '{') {
      j.kind = Json::Object;
      ++p;
      ws();
      if (p < end && *p == '}') { ++p; return j; }
      while (true) {
        ws();
        std::string key = str();
        ws();
        if (p >= end || *p != ':') fail("expected ':'");
        ++p;
        j.fields.emplace_back(key, value(depth + 1));
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') { ++p; return j; }
        fail("expected ',' or '}'");
      }
    }
    if (*p == '[') {
      j.kind = Json::Array;
      ++p;
      ws();
      if (p < end && *p == ']') { ++p; return j; }
      while (true) {
        j.items.push_back(value(depth + 1));
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') { ++p; return j; }
        fail("expected ',' or ']'");
      }
    }
    if (*p == '"') {
      j.kind = Json::String;
      j.str = str();
      return j;
    }
    if (end - p >= 4 && !strncmp(p, "true", 4)) { j.kind = Json::Bool; j.b = true; p += 4; return j; }
    if (end - p >= 5 && !strncmp(p, "false", 5)) { j.kind = Json::Bool; p += 5; return j; }
    if (end - p >= 4 && !strncmp(p, "null", 4)) { p += 4; return j; }
    std::string digits;
    while (p < end && (isdigit((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.' || *p == 'e' || *p == 'E'))
      digits += *p++;
    if (digits.empty()) fail("bad value");
    j.kind = Json::Number;
    char* stop = nullptr;
    j.num = strtod(digits.c_str(), &stop);
    if (*stop) fail("bad number");
    return j;
  }
};
}  // namespace

Json Json::parse(const std::string& text) {
  Parser parser{text.data(), text.data() + text.size()};
  Json j = parser.value(0);
  parser.ws();
  if (parser.p != parser.end) throw Error("JSON: text after the value");
  return j;
}

const Json* Json::get(const std::string& key) const {
  const Json* at = this;
  size_t start = 0;
  while (start <= key.size()) {
    size_t dot = key.find('.', start);
    std::string part = key.substr(start, dot == std::string::npos ? std::string::npos : dot - start);
    if (at->kind != Object) return nullptr;
    const Json* next = nullptr;
    for (auto& f : at->fields)
      if (f.first == part) next = &f.second;
    if (!next) return nullptr;
    at = next;
    if (dot == std::string::npos) break;
    start = dot + 1;
  }
  return at->kind == Null ? nullptr : at;
}

double Json::number(const std::string& key, double dflt) const {
  const Json* j = get(key);
  if (!j) return dflt;
  if (j->kind != Number) throw Error("JSON: " + key + " is not a number");
  return j->num;
}

long Json::integer(const std::string& key) const {
  const Json* j = get(key);
  if (!j || j->kind != Number) throw Error("config.json: no " + key);
  if (j->num < 0 || j->num != std::floor(j->num)) throw Error("config.json: " + key + " is not a count");
  return (long)j->num;
}

std::string Json::string_or(const std::string& key, const std::string& dflt) const {
  const Json* j = get(key);
  if (!j) return dflt;
  if (j->kind != String) throw Error("JSON: " + key + " is not a string");
  return j->str;
}

bool Json::flag(const std::string& key, bool dflt) const {
  const Json* j = get(key);
  if (!j) return dflt;
  if (j->kind != Bool) throw Error("JSON: " + key + " is not true or false");
  return j->b;
}

// ----------------------------------------------------------------- GGUF --
size_t ggml_size(uint32_t type, uint64_t count) {
  switch (type) {
    case F32: return count * 4;
    case F16: return count * 2;
    case Q8_0:
      if (count % 32) throw Error("GGUF: a Q8_0 tensor is not whole blocks");
      return count / 32 * 34;
    case I8: return count;
    case I32: return count * 4;
    case BF16: return count * 2;
    default: throw Error("GGUF: ggml type " + std::to_string(type) + " is not read (F32, F16, BF16, Q8_0, I8, I32 are)");
  }
}

void TensorFiles::map_file(const std::string& path, const uint8_t** base, size_t* size) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw Error("cannot open " + path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    throw Error("cannot stat " + path);
  }
  const size_t n = (size_t)st.st_size;
  void* m = n ? mmap(nullptr, n, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
  ::close(fd);
  if (m == MAP_FAILED) throw Error("cannot map " + path);
  maps_.emplace_back(m, n);
  paths_.push_back(path);
  *base = (const uint8_t*)m;
  *size = n;
}

std::unique_ptr<TensorFiles> TensorFiles::gguf(const std::string& path) {
  std::unique_ptr<TensorFiles> f(new TensorFiles());
  f->what_ = path.substr(path.find_last_of('/') + 1);
  const uint8_t* base = nullptr;
  size_t size_ = 0;
  f->map_file(path, &base, &size_);
  auto& strings_ = f->strings_;
  auto& numbers_ = f->numbers_;
  auto& tensors_ = f->tensors_;
  size_t at = 0;
  auto need = [&](uint64_t n) {
    if (n > size_ || at > size_ - n) throw Error(path + ": the header runs past the end of the file");
  };
  auto u32 = [&]() { need(4); uint32_t v; std::memcpy(&v, base + at, 4); at += 4; return v; };
  auto u64 = [&]() { need(8); uint64_t v; std::memcpy(&v, base + at, 8); at += 8; return v; };
  auto gstr = [&]() {
    uint64_t n = u64();
    need(n);
    std::string s((const char*)base + at, n);
    at += n;
    return s;
  };
  if (size_ < 4 || std::memcmp(base, "GGUF", 4) != 0) throw Error(path + ": not a GGUF file");
  at = 4;
  uint32_t version = u32();
  if (version < 2 || version > 3) throw Error(path + ": GGUF version " + std::to_string(version));
  uint64_t tensor_count = u64(), kv_count = u64();
  if (tensor_count > size_ / 24 || kv_count > size_ / 12) throw Error(path + ": the lists run past the end of the file");
  uint64_t alignment = 32;
  static const size_t scalar[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
  for (uint64_t i = 0; i < kv_count; ++i) {
    std::string key = gstr();
    uint32_t type = u32();
    if (type == 8) {
      strings_[key] = gstr();
    } else if (type == 9) {
      uint32_t et = u32();
      uint64_t n = u64();
      if (et == 8) {
        for (uint64_t e = 0; e < n; ++e) gstr();
      } else if (et < 13 && et != 9 && scalar[et]) {
        need(n * scalar[et]);
        at += n * scalar[et];
      } else {
        throw Error(path + ": an array of arrays in the metadata");
      }
    } else if (type < 13 && scalar[type]) {
      need(scalar[type]);
      const uint8_t* v = base + at;
      double num = 0;
      switch (type) {
        case 0: num = v[0]; break;
        case 1: num = (int8_t)v[0]; break;
        case 2: { uint16_t x; std::memcpy(&x, v, 2); num = x; break; }
        case 3: { int16_t x; std::memcpy(&x, v, 2); num = x; break; }
        case 4: { uint32_t x; std::memcpy(&x, v, 4); num = x; break; }
        case 5: { int32_t x; std::memcpy(&x, v, 4); num = x; break; }
        case 6: { float x; std::memcpy(&x, v, 4); num = x; break; }
        case 7: num = v[0] ? 1 : 0; break;
        case 10: { uint64_t x; std::memcpy(&x, v, 8); num = (double)x; break; }
        case 11: { int64_t x; std::memcpy(&x, v, 8); num = (double)x; break; }
        case 12: { double x; std::memcpy(&x, v, 8); num = x; break; }
      }
      at += scalar[type];
      numbers_[key] = num;
      if (key == "general.alignment" && (type == 4 || type == 10)) alignment = (uint64_t)num;
    } else {
      throw Error(path + ": metadata value type " + std::to_string(type));
    }
  }
  if (alignment == 0) throw Error(path + ": general.alignment is 0");
  std::vector<GgufTensor> infos;
  for (uint64_t i = 0; i < tensor_count; ++i) {
    GgufTensor t;
    t.name = gstr();
    uint32_t nd = u32();
    if (nd > 4) throw Error(path + ": tensor " + t.name + " has " + std::to_string(nd) + " dimensions");
    for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(u64());
    t.type = u32();
    t.offset = u64();
    infos.push_back(t);
  }
  uint64_t data = (at + alignment - 1) / alignment * alignment;
  for (auto& t : infos) {
    uint64_t count = 1;
    for (auto d : t.dims) {
      if (d && count > UINT64_MAX / d) throw Error(path + ": tensor " + t.name + " is too large");
      count *= d;
    }
    t.bytes = ggml_size(t.type, count);
    if (data > size_ || t.offset > size_ - data || t.bytes > size_ - data - t.offset)
      throw Error(path + ": tensor " + t.name + " runs past the end of the file");
    t.data = base + data + t.offset;
    tensors_[t.name] = t;
  }
  return f;
}

std::unique_ptr<TensorFiles> TensorFiles::safetensors(const std::vector<std::string>& paths) {
  std::unique_ptr<TensorFiles> f(new TensorFiles());
  f->what_ = paths.size() == 1 ? paths[0].substr(paths[0].find_last_of('/') + 1) : "the safetensors files";
  for (const std::string& path : paths) {
    const uint8_t* base = nullptr;
    size_t size = 0;
    f->map_file(path, &base, &size);
    uint64_t header = 0;
    if (size < 8) throw Error(path + ": not a safetensors file");
    std::memcpy(&header, base, 8);
    if (header > size - 8) throw Error(path + ": the safetensors header runs past the end of the file");
    const size_t data = 8 + (size_t)header;
    Json j = Json::parse(std::string((const char*)base + 8, (size_t)header));
    if (j.kind != Json::Object) throw Error(path + ": the safetensors header is not an object");
    for (auto& kv : j.fields) {
      if (kv.first == "__metadata__") continue;
      const Json& e = kv.second;
      const std::string dtype = e.string_or("dtype", "");
      GgufTensor t;
      t.name = kv.first;
      if (dtype == "F32") t.type = F32;
      else if (dtype == "F16") t.type = F16;
      else if (dtype == "BF16") t.type = BF16;
      else if (dtype == "I8" || dtype == "U8") t.type = I8;
      else if (dtype == "I32") t.type = I32;
      else throw Error(path + ": tensor " + t.name + " has dtype " + dtype + " (F32, F16, BF16, I8, U8, I32 are read)");
      const Json* shape = e.get("shape");
      const Json* offs = e.get("data_offsets");
      if (!shape || shape->kind != Json::Array || !offs || offs->kind != Json::Array || offs->items.size() != 2)
        throw Error(path + ": tensor " + t.name + " has no shape or data_offsets");
      // Innermost dimension first, as GGUF lists them.
      for (size_t i = shape->items.size(); i-- > 0;) t.dims.push_back((uint64_t)shape->items[i].num);
      const uint64_t b = (uint64_t)offs->items[0].num, en = (uint64_t)offs->items[1].num;
      t.bytes = ggml_size(t.type, t.count());
      if (en < b || en - b != t.bytes || en > size - data)
        throw Error(path + ": tensor " + t.name + " has a byte range that does not fit its shape or the file");
      t.offset = b;
      t.data = base + data + b;
      f->tensors_[t.name] = t;
    }
  }
  return f;
}

TensorFiles::~TensorFiles() {
  for (auto& m : maps_) munmap(m.first, m.second);
}

bool TensorFiles::number(const std::string& key, double* out) const {
  auto it = numbers_.find(key);
  if (it == numbers_.end()) return false;
  *out = it->second;
  return true;
}

const GgufTensor* TensorFiles::find(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

const GgufTensor& TensorFiles::at(const std::string& name) const {
  const GgufTensor* t = find(name);
  if (!t) throw Error(what_ + " has no tensor " + name);
  return *t;
}

float bf16_to_f32(uint16_t bits) {
  uint32_t u = (uint32_t)bits << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

void q8_0_quantize_block(const float* v, uint8_t* out) {
  float max = 0.0f;
  for (int i = 0; i < 32; ++i) max = std::max(max, std::fabs(v[i]));
  const float d = max / 127.0f;
  const float inverse = d != 0.0f ? 1.0f / d : 0.0f;
  const uint16_t h = f32_to_f16(d);
  std::memcpy(out, &h, 2);
  for (int i = 0; i < 32; ++i) out[2 + i] = (uint8_t)(int8_t)std::round(v[i] * inverse);
}


}  // namespace trit

namespace trit {

ModelConfig parse_model_config(const std::string& text, const std::string& at) {
  Json j = Json::parse(text);
  auto key = [&](const char* name) { return at + name; };
  ModelConfig m;
  m.type = j.string_or(key("model_type"), "");
  if (m.type == "qwen3") m.qk_norm = true;
  else if (m.type == "llama" || m.type == "mistral" || m.type == "granite") m.qk_norm = false;
  else throw Error("config.json does not describe a language model this engine runs");
  DConfig& c = m.cfg;
  c.heads = (int)j.integer(key("num_attention_heads"));
  c.kv_heads = (int)j.integer(key("num_key_value_heads"));
  if (c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads)
    throw Error("config.json: the query heads do not share the key heads evenly");
  c.d = (int)j.integer(key("hidden_size"));
  c.embedding_multiplier = (float)j.number(key("embedding_multiplier"), 1.0);
  c.has_q_scale = j.has(key("attention_multiplier"));
  c.residual_multiplier = (float)j.number(key("residual_multiplier"), 1.0);
  c.logits_scaling = (float)j.number(key("logits_scaling"), 1.0);
  c.ffn = (int)j.integer(key("intermediate_size"));
  c.layers = (int)j.integer(key("num_hidden_layers"));
  c.hd = j.has(key("head_dim")) ? (int)j.integer(key("head_dim")) : c.d / c.heads;
  c.vocab = (int)j.integer(key("vocab_size"));
  c.eps = (float)j.number(key("rms_norm_eps"), 1e-6);
  m.rope_base = (float)j.number(key("rope_theta"), 1e6);
  // `attention` divides by sqrt(head_dim); Granite's multiplier replaces
  // that (causal_lm.rs:416-419), so the kernels scale q by it times sqrt(hd).
  m.attention_multiplier = (float)j.number(key("attention_multiplier"), 1.0);
  c.q_scale = c.has_q_scale ? m.attention_multiplier * std::sqrt((float)c.hd) : 1.0f;
  m.tied = j.flag(key("tie_word_embeddings"), false);
  return m;
}

ModelConfig read_model_config(const std::string& dir, const std::string& at) {
  std::string text;
  FILE* f = std::fopen((dir + "/config.json").c_str(), "rb");
  if (!f) throw Error("cannot read " + dir + "/config.json");
  char buf[65536];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
  std::fclose(f);
  return parse_model_config(text, at);
}

namespace {

bool is_file(const std::string& path) {
  struct stat st;
  return ::stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

// The files of `dir` that end in `suffix`, sorted.
std::vector<std::string> files_ending(const std::string& dir, const std::string& suffix) {
  std::vector<std::string> out;
  DIR* d = ::opendir(dir.c_str());
  if (!d) throw Error("cannot list " + dir);
  while (dirent* e = ::readdir(d)) {
    std::string n = e->d_name;
    if (n.size() > suffix.size() && n.compare(n.size() - suffix.size(), suffix.size(), suffix) == 0 &&
        is_file(dir + "/" + n))
      out.push_back(dir + "/" + n);
  }
  ::closedir(d);
  std::sort(out.begin(), out.end());
  return out;
}

std::string read_text(const std::string& path) {
  std::string text;
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) throw Error("cannot read " + path);
  char buf[65536];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
  std::fclose(f);
  return text;
}

// The GGUF architectures whose language model is a CausalLm decoder
// (src/models/gguf/mod.rs:61-103): the metadata prefix of its settings,
// its model_type, the tie of its head when the file does not say, and the
// prefix of its tensors' Hugging Face names (qwen3_asr.rs:58,69;
// moss.rs:50,64; fun_asr.rs:49,60; canary_qwen.rs:39,50; voxtral.rs:41,54;
// voxtral_realtime.rs:25,85; granite_speech.rs:32-36,94).
struct DecoderArch {
  const char* arch;
  const char* meta;
  const char* model_type;
  bool tie;
  const char* prefix;
};
const DecoderArch kDecoderArchs[] = {
    {"qwen3_asr", "stt.qwen3_asr.decoder", "qwen3", true, "thinker."},
    {"moss", "stt.moss.decoder", "qwen3", true, "language_model."},
    {"funasr_nano", "stt.funasr_nano.decoder", "qwen3", true, "llm."},
    {"canary_qwen", "stt.canary_qwen.decoder", "qwen3", true, "llm."},
    {"voxtral", "stt.voxtral.decoder", "mistral", false, "language_model."},
    {"voxtral_realtime", "stt.voxtral_realtime.decoder", "mistral", true, "language_model."},
    {"granite_speech", "stt.granite.decoder", "granite", false, "language_model."},
};

// A transcribe.cpp decoder tensor name (`dec.*`) as the Hugging Face
// checkpoint names it under `prefix` (language_model_name,
// src/models/gguf/qwen3_asr.rs:103-136; the untied head, voxtral.rs:50-52),
// or "" for a tensor of another part (the audio encoder).
std::string hf_decoder_name(const std::string& name, const std::string& prefix) {
  auto starts = [&](const std::string& s, const char* p) { return s.compare(0, std::strlen(p), p) == 0; };
  if (starts(name, "dec.token_embd.")) return prefix + "model.embed_tokens." + name.substr(15);
  if (starts(name, "dec.output_norm.")) return prefix + "model.norm." + name.substr(16);
  if (starts(name, "dec.output.")) return prefix + "lm_head." + name.substr(11);
  std::string rest;
  if (starts(name, "dec.blocks.")) rest = name.substr(11);
  else if (starts(name, "dec.layers.")) rest = name.substr(11);  // Fun-ASR files
  else return "";
  const size_t dot = rest.find('.');
  if (dot == std::string::npos) return "";
  const std::string layer = rest.substr(0, dot), part = rest.substr(dot + 1);
  // A longer source comes before a shorter one it starts with.
  static const char* table[][2] = {
      {"norm_attn.", "input_layernorm."},   {"norm_ffn.", "post_attention_layernorm."},
      {"attn.q_norm.", "self_attn.q_norm."}, {"attn.k_norm.", "self_attn.k_norm."},
      {"attn.q.", "self_attn.q_proj."},      {"attn.k.", "self_attn.k_proj."},
      {"attn.v.", "self_attn.v_proj."},      {"attn.o.", "self_attn.o_proj."},
      {"ffn.gate.", "mlp.gate_proj."},       {"ffn.up.", "mlp.up_proj."},
      {"ffn.down.", "mlp.down_proj."},
  };
  for (auto& row : table)
    if (starts(part, row[0])) return prefix + "model.layers." + layer + "." + row[1] + part.substr(std::strlen(row[0]));
  return "";
}

// The config.json block of a transcribe.cpp decoder (src/models/gguf/
// blocks.rs:25-45 `llm`, with Granite's multipliers, granite_speech.rs:33-36).
std::string decoder_config(const TensorFiles& g, const DecoderArch& a) {
  auto num = [&](const char* key) {
    double v;
    if (!g.number(std::string(a.meta) + "." + key, &v))
      throw Error(g.what() + ": no " + std::string(a.meta) + "." + key);
    return v;
  };
  auto opt = [&](const char* key, double* v) { return g.number(std::string(a.meta) + "." + key, v); };
  char buf[1024];
  double eps = 1e-6, theta = 1e6, tie = a.tie ? 1 : 0;
  opt("rms_norm_eps", &eps);
  opt("rope_theta", &theta);
  opt("tie_word_embeddings", &tie);
  std::snprintf(buf, sizeof buf,
                "{\"model_type\": \"%s\", \"hidden_size\": %.0f, \"intermediate_size\": %.0f, "
                "\"num_hidden_layers\": %.0f, \"num_attention_heads\": %.0f, \"num_key_value_heads\": %.0f, "
                "\"head_dim\": %.0f, \"vocab_size\": %.0f, \"rms_norm_eps\": %.9g, \"rope_theta\": %.9g, "
                "\"tie_word_embeddings\": %s",
                a.model_type, num("hidden_size"), num("intermediate_size"), num("n_layers"), num("n_heads"),
                num("n_kv_heads"), num("head_dim"), num("vocab_size"), eps, theta, tie != 0 ? "true" : "false");
  std::string out = buf;
  for (const char* key : {"embedding_multiplier", "attention_multiplier", "residual_multiplier", "logits_scaling"}) {
    double v;
    if (opt(key, &v)) {
      std::snprintf(buf, sizeof buf, ", \"%s\": %.9g", key, v);
      out += buf;
    }
  }
  return out + "}";
}

}  // namespace

ModelSource open_model(const std::string& dir, const std::string& at, const std::string& prefix) {
  ModelSource src;
  struct stat st;
  if (::stat(dir.c_str(), &st) != 0 || !S_ISDIR(st.st_mode))
    throw Error(dir + " is not a model folder (config.json with model.gguf or .safetensors files, or one .gguf file)");
  if (is_file(dir + "/config.json")) {
    src.mc = read_model_config(dir, at);
    src.prefix = prefix;
    if (is_file(dir + "/model.gguf")) {
      src.files = TensorFiles::gguf(dir + "/model.gguf");
      src.format = "gguf";
      return src;
    }
    std::vector<std::string> shards;
    if (is_file(dir + "/model.safetensors.index.json")) {
      Json idx = Json::parse(read_text(dir + "/model.safetensors.index.json"));
      const Json* map = idx.get("weight_map");
      if (!map || map->kind != Json::Object) throw Error(dir + "/model.safetensors.index.json has no weight_map");
      std::set<std::string> files;
      for (auto& kv : map->fields) files.insert(dir + "/" + kv.second.str);
      shards.assign(files.begin(), files.end());
    } else if (is_file(dir + "/model.safetensors")) {
      shards.push_back(dir + "/model.safetensors");
    } else {
      shards = files_ending(dir, ".safetensors");
    }
    if (shards.empty()) throw Error(dir + " has config.json but no model.gguf or .safetensors files");
    src.files = TensorFiles::safetensors(shards);
    src.format = "safetensors";
    return src;
  }
  std::vector<std::string> ggufs = files_ending(dir, ".gguf");
  if (ggufs.size() != 1)
    throw Error(dir + ": no config.json, and " + std::to_string(ggufs.size()) + " .gguf files (one is read alone)");
  src.files = TensorFiles::gguf(ggufs[0]);
  auto arch_it = src.files->strings().find("general.architecture");
  const std::string arch = arch_it == src.files->strings().end() ? "" : arch_it->second;
  const DecoderArch* a = nullptr;
  for (auto& row : kDecoderArchs)
    if (arch == row.arch) a = &row;
  if (!a) {
    std::string names;
    for (auto& row : kDecoderArchs) names += (names.empty() ? "" : ", ") + std::string(row.arch);
    throw Error(src.files->what() + ": GGUF architecture " + (arch.empty() ? "(none)" : arch) +
                " has no decoder this library runs (" + names + " do)");
  }
  src.mc = parse_model_config(decoder_config(*src.files, *a), "");
  src.prefix = a->prefix;
  const std::string pre = a->prefix;
  src.files->rename([&](const std::string& n) { return hf_decoder_name(n, pre); });
  src.format = "gguf-transcribe";
  return src;
}

TpShard tp_shard(const DConfig& c, int rank, int size) {
  if (size < 1 || rank < 0 || rank >= size) throw Error("tensor parallelism: rank " + std::to_string(rank) + " of " +
                                                        std::to_string(size));
  if (c.kv_heads % size || c.heads % size)
    throw Error("tensor parallelism: " + std::to_string(c.kv_heads) + " key/value heads do not split " +
                std::to_string(size) + " ways");
  // Whole 128-value groups of FFN units per rank (the activation groups
  // of int8 and ternary products and the tensor cores' K step).
  if (c.ffn % (128 * size)) throw Error("tensor parallelism: intermediate_size does not split into 128-wide shards");
  if (c.vocab % size) throw Error("tensor parallelism: vocab_size does not split evenly");
  TpShard t;
  t.rank = rank;
  t.size = size;
  t.kv = c.kv_heads / size;
  t.kv0 = rank * t.kv;
  t.heads = c.heads / size;
  t.heads0 = rank * t.heads;  // query heads follow their key/value heads
  t.ffn = c.ffn / size;
  t.ffn0 = rank * t.ffn;
  t.vocab = c.vocab / size;
  t.vocab0 = rank * t.vocab;
  return t;
}

namespace {

// The storage of the product `name` (without .weight): its kind and the
// bytes of its codes and scales as the device holds them. Float weights
// (safetensors, or F32 / F16 / BF16 in GGUF) are quantized to Q8_0 at load.
std::string product_kind(const TensorFiles& g, const std::string& name, uint64_t* bytes) {
  const GgufTensor* w = g.find(name + ".weight");
  if (w && (w->type == Q8_0 || w->type == F32 || w->type == F16 || w->type == BF16)) {
    *bytes = w->count() + w->count() / 32 * 2;
    return "q8_0";
  }
  if (w && w->type == I8 && g.find(name + ".scales")) {
    *bytes = w->count() + g.at(name + ".scales").count() * 4;
    return "int8";
  }
  const GgufTensor* q = g.find(name + ".qweight");
  if (q) {
    const GgufTensor& s = g.at(name + ".scales");
    // 5 codes a byte in the file, 2 bits a code on the device.
    *bytes = s.count() * 128 / 4 + s.count() * 4;
    return "ternary";
  }
  throw Error(g.what() + ": no Q8_0, float, int8 or ternary weights for " + name);
}

}  // namespace

std::string describe_model(const std::string& dir, const std::string& at, const std::string& prefix_in, int tp_rank,
                           int tp_size) {
  ModelSource src = open_model(dir, at, prefix_in);
  const ModelConfig& m = src.mc;
  const DConfig& c = m.cfg;
  const TensorFiles& g = *src.files;
  const std::string& prefix = src.prefix;
  std::map<std::string, int> kinds;
  uint64_t layer_bytes = 0, b = 0;
  const char* parts[] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                         "mlp.gate_proj",    "mlp.up_proj",      "mlp.down_proj"};
  for (int l = 0; l < c.layers; ++l)
    for (const char* p : parts) {
      kinds[product_kind(g, prefix + "model.layers." + std::to_string(l) + "." + p, &b)]++;
      layer_bytes += b;
    }
  auto table_kind = [&](const std::string& name, uint64_t* bytes) -> std::string {
    const GgufTensor& t = g.at(name);
    if (t.type == Q8_0 || t.type == F32 || t.type == F16 || t.type == BF16) {
      *bytes = t.count() + t.count() / 32 * 2;
      return "q8_0";
    }
    if (t.type == I8) {
      *bytes = t.count() + t.count() / 32 * 4;
      return "int8";
    }
    throw Error(g.what() + ": " + name + " is neither Q8_0, float nor int8 with per-32 scales");
  };
  uint64_t embed_bytes = 0, head_bytes = 0;
  std::string embed = table_kind(prefix + "model.embed_tokens.weight", &embed_bytes);
  bool has_head = !m.tied && g.find(prefix + "lm_head.weight");
  std::string head = has_head ? table_kind(prefix + "lm_head.weight", &head_bytes) : embed;
  if (!has_head) head_bytes = embed_bytes;
  std::string weights;
  for (auto& k : kinds) weights += (weights.empty() ? "" : "+") + k.first;
  char q_mult[64] = "null";
  if (c.has_q_scale) std::snprintf(q_mult, sizeof q_mult, "%.9g", (double)m.attention_multiplier);
  char buf[2048];
  std::snprintf(buf, sizeof buf,
                "{\"model_type\": \"%s\", \"hidden_size\": %d, \"intermediate_size\": %d, \"num_hidden_layers\": %d, "
                "\"num_attention_heads\": %d, \"num_key_value_heads\": %d, \"head_dim\": %d, \"vocab_size\": %d, "
                "\"rms_norm_eps\": %.9g, \"rope_theta\": %.9g, \"qk_norm\": %s, \"tie_word_embeddings\": %s, "
                "\"embedding_multiplier\": %.9g, \"attention_multiplier\": %s, \"residual_multiplier\": %.9g, "
                "\"logits_scaling\": %.9g, \"products\": \"%s\", \"token_table\": \"%s\", \"output_table\": \"%s\", "
                "\"separate_head\": %s, \"product_bytes\": %llu, \"output_table_bytes\": %llu, "
                "\"source\": \"%s\", \"tensor_prefix\": \"%s\"}",
                m.type.c_str(), c.d, c.ffn, c.layers, c.heads, c.kv_heads, c.hd, c.vocab, (double)c.eps,
                (double)m.rope_base, m.qk_norm ? "true" : "false", m.tied ? "true" : "false",
                (double)c.embedding_multiplier,
                q_mult,
                (double)c.residual_multiplier, (double)c.logits_scaling, weights.c_str(), embed.c_str(),
                head.c_str(), has_head ? "true" : "false", (unsigned long long)layer_bytes,
                (unsigned long long)head_bytes, src.format.c_str(), prefix.c_str());
  std::string out = buf;
  if (tp_size > 1) {
    const TpShard t = tp_shard(c, tp_rank, tp_size);
    std::snprintf(buf, sizeof buf,
                  ", \"tp\": {\"rank\": %d, \"size\": %d, \"heads\": [%d, %d], \"kv_heads\": [%d, %d], "
                  "\"ffn_units\": [%d, %d], \"vocab_rows\": [%d, %d]}}",
                  t.rank, t.size, t.heads0, t.heads0 + t.heads, t.kv0, t.kv0 + t.kv, t.ffn0, t.ffn0 + t.ffn, t.vocab0,
                  t.vocab0 + t.vocab);
    out = out.substr(0, out.size() - 1) + buf;
  }
  return out;
}

}  // namespace trit
