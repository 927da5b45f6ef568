#include "host.h"

#include <cmath>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

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
    default: throw Error("GGUF: ggml type " + std::to_string(type) + " is not read (F32, F16, Q8_0, I8, I32 are)");
  }
}

GgufFile::GgufFile(const std::string& path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw Error("cannot open " + path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    throw Error("cannot stat " + path);
  }
  size_ = (size_t)st.st_size;
  map_ = size_ ? mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    throw Error("cannot map " + path);
  }
  const uint8_t* base = (const uint8_t*)map_;
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
      if (key == "general.alignment" && type == 4) {
        alignment = u32();
      } else {
        need(scalar[type]);
        at += scalar[type];
      }
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
}

GgufFile::~GgufFile() {
  if (map_) munmap(map_, size_);
}

const GgufTensor* GgufFile::find(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

const GgufTensor& GgufFile::at(const std::string& name) const {
  const GgufTensor* t = find(name);
  if (!t) throw Error("model.gguf has no tensor " + name);
  return *t;
}

GgufWriter::~GgufWriter() {
  if (file_) std::fclose(file_);
}

void GgufWriter::add(const std::string& name, uint32_t type, std::vector<uint64_t> dims) {
  GgufTensor t;
  t.name = name;
  t.type = type;
  t.dims = std::move(dims);
  t.bytes = ggml_size(type, t.count());
  infos_.push_back(t);
}

void GgufWriter::open(const std::string& path) {
  file_ = std::fopen(path.c_str(), "wb");
  if (!file_) throw Error("cannot write " + path);
  auto w = [&](const void* p, size_t n) {
    if (std::fwrite(p, 1, n, file_) != n) throw Error("write failed: " + path);
    written_ += n;
  };
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
    ws(m.first);
    w32(8);
    ws(m.second);
  }
  uint64_t offset = 0;
  for (auto& t : infos_) {
    t.offset = offset;
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

void GgufWriter::put(const void* bytes, size_t size) {
  if (next_ >= infos_.size() || size != infos_[next_].bytes) throw Error("GGUF writer: tensor size mismatch");
  static const uint8_t zeros[32] = {0};
  if (std::fwrite(bytes, 1, size, file_) != size) throw Error("GGUF writer: write failed");
  written_ += size;
  size_t pad = (32 - written_ % 32) % 32;
  if (pad && std::fwrite(zeros, 1, pad, file_) != pad) throw Error("GGUF writer: write failed");
  written_ += pad;
  ++next_;
}

void GgufWriter::close() {
  if (next_ != infos_.size()) throw Error("GGUF writer: not every tensor was written");
  if (file_ && std::fclose(file_) != 0) {
    file_ = nullptr;
    throw Error("GGUF writer: close failed");
  }
  file_ = nullptr;
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

// The storage of the product `name` (without .weight): its kind and the
// bytes of its codes and scales as the device holds them.
std::string product_kind(const GgufFile& g, const std::string& name, uint64_t* bytes) {
  const GgufTensor* w = g.find(name + ".weight");
  if (w && w->type == Q8_0) {
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
  throw Error("model.gguf: no Q8_0, int8 or ternary weights for " + name);
}

}  // namespace

std::string describe_model(const std::string& dir, const std::string& at, const std::string& prefix) {
  ModelConfig m = read_model_config(dir, at);
  const DConfig& c = m.cfg;
  GgufFile g(dir + "/model.gguf");
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
    if (t.type == Q8_0) {
      *bytes = t.count() + t.count() / 32 * 2;
      return "q8_0";
    }
    if (t.type == I8) {
      *bytes = t.count() + t.count() / 32 * 4;
      return "int8";
    }
    throw Error("model.gguf: " + name + " is neither Q8_0 nor int8 with per-32 scales");
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
                "\"separate_head\": %s, \"product_bytes\": %llu, \"output_table_bytes\": %llu}",
                m.type.c_str(), c.d, c.ffn, c.layers, c.heads, c.kv_heads, c.hd, c.vocab, (double)c.eps,
                (double)m.rope_base, m.qk_norm ? "true" : "false", m.tied ? "true" : "false",
                (double)c.embedding_multiplier,
                q_mult,
                (double)c.residual_multiplier, (double)c.logits_scaling, weights.c_str(), embed.c_str(),
                head.c_str(), has_head ? "true" : "false", (unsigned long long)layer_bytes,
                (unsigned long long)head_bytes);
  return buf;
}

}  // namespace trit
