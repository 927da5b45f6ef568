// Loading a decoder into device memory and running CausalLm's generation
// flows (src/models/parts/causal_lm.rs:141-302) on one GPU.
#include "engine.h"
#include "nccl_link.h"

#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <thread>

namespace trit {

void CudaCheck::ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(std::string("CUDA: ") + cudaGetErrorString(e) + " (" + what + ")");
}

Options Options::parse(const char* text, bool lenient) {
  Options o;
  if (!text || !*text) return o;
  Json j = Json::parse(text);
  if (j.kind != Json::Object) throw Error("options: not a JSON object");
  for (auto& f : j.fields) {
    const std::string& k = f.first;
    const Json& v = f.second;
    if (lenient && k != "config_at" && k != "prefix" && k != "tp_size" && k != "tp_rank") continue;
    auto count = [&](int lo, int hi) {
      if (v.kind != Json::Number || v.num != std::floor(v.num) || v.num < lo || v.num > hi)
        throw Error("options: " + k + " must be a whole number from " + std::to_string(lo) + " to " + std::to_string(hi));
      return (int)v.num;
    };
    if (k == "device") o.device = count(0, 63);
    else if (k == "kv") {
      if (v.kind != Json::String || (v.str != "f16" && v.str != "f32")) throw Error("options: kv is \"f16\" or \"f32\"");
      o.kv_f16 = v.str == "f16";
    } else if (k == "max_context") o.max_context = count(1, 1 << 20);
    else if (k == "max_streams") o.max_streams = count(1, 4096);
    else if (k == "page_tokens") o.page_tokens = count(1, 4096);
    else if (k == "prefill_rows") o.prefill_rows = count(1, 65536);
    else if (k == "prefix_pages") o.prefix_pages = count(0, 1 << 20);
    else if (k == "decode") {
      if (v.kind != Json::String || (v.str != "persistent" && v.str != "layered"))
        throw Error("options: decode is \"persistent\" or \"layered\"");
      o.decode = v.str;
    } else if (k == "tensor_cores") {
      if (v.kind != Json::Bool) throw Error("options: tensor_cores is true or false");
      o.tensor_cores = v.b;
    } else if (k == "tc_rows") {
      o.tc_rows = count(1, 1 << 20);
    } else if (k == "tp_size") {
      o.tp_size = count(1, 64);
    } else if (k == "tp_rank") {
      o.tp_rank = count(0, 63);
    } else if (k == "tc_attention") {
      if (v.kind != Json::Bool) throw Error("options: tc_attention must be true or false");
      o.tc_attention = v.b;
    } else if (k == "tc_f16") {
      if (v.kind != Json::Bool) throw Error("options: tc_f16 must be true or false");
      o.tc_f16 = v.b;
    } else if (k == "tp_timeout_s") {
      if (v.kind != Json::Number || v.num <= 0) throw Error("options: tp_timeout_s must be a positive number");
      o.tp_timeout_s = v.num;
    } else if (k == "tp_id") {
      if (v.kind != Json::String) throw Error("options: tp_id must be a string");
      o.tp_id = v.str;
    } else if (k == "weight_cache") {
      if (v.kind != Json::Bool) throw Error("options: weight_cache is true or false");
      o.weight_cache = v.b;
    } else if (k == "cache_dir") {
      if (v.kind != Json::String) throw Error("options: cache_dir must be a string");
      o.cache_dir = v.str;
    } else if (k == "exact") {
      if (v.kind != Json::Bool) throw Error("options: exact is true or false");
      o.exact = v.b;
    } else if (k == "config_at" || k == "prefix") {
      if (v.kind != Json::String) throw Error("options: " + k + " must be a string");
      (k == "config_at" ? o.config_at : o.prefix) = v.str;
    } else {
      throw Error("options: unknown key " + k);
    }
  }
  if (o.tc_attention && o.exact) throw Error("options: tc_attention needs \"exact\": false (it is not the reference's arithmetic)");
  return o;
}

PrefixState::~PrefixState() {
  if (owner) {
    std::lock_guard<std::mutex> lock(owner->mutex());
    owner->release_prefix(this);
  }
  if (partial) cudaFree(partial);
}

void Lm::release_prefix(PrefixState* p) {
  prefix_free_.insert(prefix_free_.end(), p->pages.begin(), p->pages.end());
  p->pages.clear();
  p->owner = nullptr;
  prefixes_.erase(p);
}

void Lm::map_slot(int slot, const PrefixState* prefix) {
  const int pps = cache_.pages_per_stream;
  int* row = table_host_.data() + (size_t)slot * pps;
  bool changed = false;
  for (int i = 0; i < pps; ++i) {
    const int want = (prefix && i < (int)prefix->pages.size()) ? prefix->pages[i] : slot * pps + i;
    changed |= row[i] != want;
    row[i] = want;
  }
  if (changed)
    TRIT_CUDA(cudaMemcpyAsync(page_table_ + (size_t)slot * pps, row, (size_t)pps * 4, cudaMemcpyHostToDevice, stream_));
  if (prefix && prefix->partial) {
    char* own = (char*)pool_ + ((size_t)slot * pps + prefix->pages.size()) * page_bytes_;
    TRIT_CUDA(cudaMemcpyAsync(own, prefix->partial, page_bytes_, cudaMemcpyDeviceToDevice, stream_));
  }
}

namespace {

// Two passes over the weights: the first sizes the arena, the second
// copies every tensor into it.
struct Arena {
  char* base = nullptr;
  size_t used = 0;
  bool fill = false;
  size_t take(size_t n) {
    size_t at = (used + 255) / 256 * 256;
    used = at + n;
    return at;
  }
  void put(size_t at, const void* src, size_t n) {
    if (fill) TRIT_CUDA(cudaMemcpy(base + at, src, n, cudaMemcpyHostToDevice));
  }
  const void* ptr(size_t at) const { return base ? base + at : nullptr; }
};

std::vector<float> f32_of(const TensorFiles& g, const std::string& name, size_t len) {
  const GgufTensor& t = g.at(name);
  if (t.count() != len) throw Error("tensor " + name + " has " + std::to_string(t.count()) + " values, expected " + std::to_string(len));
  std::vector<float> out(len);
  if (t.type == F32) {
    std::memcpy(out.data(), t.data, len * 4);
  } else if (t.type == F16 || t.type == BF16) {
    for (size_t i = 0; i < len; ++i) {
      uint16_t h;
      std::memcpy(&h, t.data + 2 * i, 2);
      out[i] = t.type == F16 ? f16_to_f32(h) : bf16_to_f32(h);
    }
  } else {
    throw Error("tensor " + name + " is not F32, F16 or BF16");
  }
  return out;
}

bool is_float(uint32_t type) { return type == F32 || type == F16 || type == BF16; }


const float* load_vector(const TensorFiles& g, Arena& A, const std::string& name, size_t len) {
  size_t at = A.take(len * 4);
  if (A.fill) {
    std::vector<float> v = f32_of(g, name, len);
    A.put(at, v.data(), len * 4);
  }
  return (const float*)A.ptr(at);
}

// One source matrix's rows [row0, row0 + rows) in a stacked product.
struct Part {
  std::string name;
  int row0, rows;
};

// Dense::load (src/cpu/gemm.rs:254-343) of parts stacked by output rows,
// in the device layout: Q8_0 blocks split into a codes plane and an f16
// scale plane (34-byte blocks are not 16-byte aligned; float weights are
// quantized to Q8_0 first); per-row int8 codes and row scales; ternary
// base-3 bytes (src/cpu/kernels.rs:91-130) repacked 16 codes a word in the
// pack_span order (kernels.rs:618-628). Of each source row of kfull inputs
// the columns [c0, c0 + k) are kept (a tensor-parallel shard of the inputs;
// c0 and k are whole activation groups, so every group stays whole).
DMat load_mat(const TensorFiles& g, Arena& A, const std::vector<Part>& parts, int k, int c0 = 0, int kfull = 0) {
  if (!kfull) kfull = k;
  DMat m;
  m.k = k;
  for (auto& p : parts) m.n += p.rows;
  const std::string& first = parts[0].name;
  const GgufTensor* w = g.find(first + ".weight");
  if (w && (w->type == Q8_0 || is_float(w->type))) {
    m.kind = kQ8_0;  // float weights are quantized to Q8_0 here
    m.agroup = 32;
    m.half = 1;
  } else if (w && w->type == I8 && g.find(first + ".scales")) {
    m.kind = kInt8Row;
    m.agroup = 128;
  } else if (g.find(first + ".qweight")) {
    m.kind = kTernary;
    m.agroup = 128;
  } else {
    throw Error(g.what() + ": no Q8_0, float, int8 or ternary weights for " + first);
  }
  if (k % m.agroup != 0 || c0 % m.agroup != 0)
    throw Error(first + ": the input width is not whole groups of " + std::to_string(m.agroup));
  if (m.n % 32 != 0) throw Error(first + ": the output rows are not a multiple of 32");
  size_t codes_bytes = (m.kind == kTernary) ? (size_t)m.n * k / 4 : (size_t)m.n * k;
  size_t scale_bytes = m.kind == kQ8_0 ? (size_t)m.n * (k / 32) * 2 : m.kind == kInt8Row ? (size_t)m.n * 4
                                                                                         : (size_t)m.n * (k / 128) * 4;
  size_t co = A.take(codes_bytes), so = A.take(scale_bytes);
  m.codes = A.ptr(co);
  m.scales = A.ptr(so);
  if (!A.fill) return m;
  std::vector<uint8_t> codes(codes_bytes), scales(scale_bytes);
  size_t out = 0;  // rows written so far
  for (auto& p : parts) {
    const size_t rows = (size_t)p.rows, r0 = (size_t)p.row0;
    auto source_rows = [&](const GgufTensor& t, size_t per_row) {
      if (t.count() % per_row || t.count() / per_row < r0 + rows)
        throw Error("tensor " + t.name + ": expected rows of " + std::to_string(per_row) + " values, " +
                    std::to_string(r0 + rows) + " at least");
    };
    if (m.kind == kQ8_0 && is_float(g.at(p.name + ".weight").type)) {
      const GgufTensor& t = g.at(p.name + ".weight");
      source_rows(t, kfull);
      std::vector<float> v = f32_of(g, p.name + ".weight", t.count());
      uint8_t blk[34];
      for (size_t r = 0; r < rows; ++r)
        for (int b = 0; b < k / 32; ++b) {
          q8_0_quantize_block(v.data() + (r0 + r) * kfull + c0 + b * 32, blk);
          std::memcpy(scales.data() + ((out + r) * (k / 32) + b) * 2, blk, 2);
          std::memcpy(codes.data() + (out + r) * k + b * 32, blk + 2, 32);
        }
    } else if (m.kind == kQ8_0) {
      const GgufTensor& t = g.at(p.name + ".weight");
      if (t.type != Q8_0) throw Error("tensor " + p.name + ".weight: expected Q8_0");
      source_rows(t, kfull);
      for (size_t r = 0; r < rows; ++r)
        for (int b = 0; b < k / 32; ++b) {
          const uint8_t* blk = t.data + ((r0 + r) * (kfull / 32) + c0 / 32 + b) * 34;
          std::memcpy(scales.data() + ((out + r) * (k / 32) + b) * 2, blk, 2);
          std::memcpy(codes.data() + (out + r) * k + b * 32, blk + 2, 32);
        }
    } else if (m.kind == kInt8Row) {
      const GgufTensor& t = g.at(p.name + ".weight");
      if (t.type != I8) throw Error("tensor " + p.name + ".weight: expected I8");
      source_rows(t, kfull);
      for (size_t r = 0; r < rows; ++r) std::memcpy(codes.data() + (out + r) * k, t.data + (r0 + r) * kfull + c0, k);
      const GgufTensor& st = g.at(p.name + ".scales");
      std::vector<float> s = f32_of(g, p.name + ".scales", st.count());
      if (s.size() < r0 + rows) throw Error("tensor " + p.name + ".scales: too few rows");
      std::memcpy(scales.data() + out * 4, s.data() + r0, rows * 4);
    } else {
      const GgufTensor& t = g.at(p.name + ".qweight");
      const size_t row_bytes = ((size_t)kfull + 4) / 5;
      source_rows(t, row_bytes);
      std::vector<uint8_t> digits((size_t)kfull + 5);
      for (size_t r = 0; r < rows; ++r) {
        const uint8_t* src = t.data + (r0 + r) * row_bytes;
        for (size_t b = 0; b < row_bytes; ++b) {
          unsigned v = src[b];
          if (v >= 243) throw Error("ternary byte above 242 in row " + std::to_string(r0 + r) + " of " + p.name);
          for (int dd = 0; dd < 5; ++dd) {
            digits[b * 5 + dd] = (uint8_t)(v % 3);
            v /= 3;
          }
        }
        uint32_t* dst = (uint32_t*)(codes.data()) + (out + r) * (k / 16);
        for (int w16 = 0; w16 < k / 16; ++w16) {
          uint32_t word = 0;
          for (int s4 = 0; s4 < 4; ++s4)
            for (int j = 0; j < 4; ++j) word |= (uint32_t)digits[c0 + w16 * 16 + 4 * s4 + j] << (8 * j + 2 * s4);
          dst[w16] = word;
        }
      }
      const GgufTensor& st = g.at(p.name + ".scales");
      std::vector<float> s = f32_of(g, p.name + ".scales", st.count());
      const size_t gfull = kfull / 128, gk = k / 128;
      if (s.size() < (r0 + rows) * gfull) throw Error("tensor " + p.name + ".scales: too few rows");
      for (size_t r = 0; r < rows; ++r)
        std::memcpy(scales.data() + ((out + r) * gk) * 4, s.data() + (r0 + r) * gfull + c0 / 128, gk * 4);
    }
    out += rows;
  }
  A.put(co, codes.data(), codes_bytes);
  A.put(so, scales.data(), scale_bytes);
  return m;
}

// Dense::table (src/cpu/gemm.rs:383-409): Q8_0 blocks (f16 scales) or int8
// codes with one f32 scale per 32 values, f32 math.
DTable load_table(const TensorFiles& g, Arena& A, const std::string& name, int rows, int cols, int row0 = 0,
                  int rows_full = 0) {
  if (!rows_full) rows_full = rows;
  DTable t;
  t.n = rows;
  t.k = cols;
  if (cols % 32) throw Error(name + ": the width is not whole blocks of 32");
  const GgufTensor& w = g.at(name + ".weight");
  if (w.count() != (uint64_t)rows_full * cols) throw Error(name + ".weight has the wrong size");
  t.scale_f16 = w.type == Q8_0 || is_float(w.type);  // float tables are quantized to Q8_0
  if (!t.scale_f16 && w.type != I8) throw Error(name + ".weight is neither Q8_0, float nor I8");
  size_t co = A.take((size_t)rows * cols), so = A.take((size_t)rows * (cols / 32) * (t.scale_f16 ? 2 : 4));
  t.codes = (const int8_t*)A.ptr(co);
  t.scales = A.ptr(so);
  if (!A.fill) return t;
  const size_t n = (size_t)rows * cols, first = (size_t)row0 * cols;
  if (is_float(w.type)) {
    std::vector<float> v = f32_of(g, name + ".weight", (size_t)rows_full * cols);
    std::vector<uint8_t> codes(n), scales(n / 32 * 2);
    uint8_t blk[34];
    for (size_t b = 0; b < n / 32; ++b) {
      q8_0_quantize_block(v.data() + first + b * 32, blk);
      std::memcpy(scales.data() + b * 2, blk, 2);
      std::memcpy(codes.data() + b * 32, blk + 2, 32);
    }
    A.put(co, codes.data(), codes.size());
    A.put(so, scales.data(), scales.size());
  } else if (w.type == Q8_0) {
    std::vector<uint8_t> codes(n), scales(n / 32 * 2);
    for (size_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = w.data + (first / 32 + b) * 34;
      std::memcpy(scales.data() + b * 2, blk, 2);
      std::memcpy(codes.data() + b * 32, blk + 2, 32);
    }
    A.put(co, codes.data(), codes.size());
    A.put(so, scales.data(), scales.size());
  } else {
    A.put(co, w.data + first, n);
    std::vector<float> s = f32_of(g, name + ".scales", (size_t)rows_full * (cols / 32));
    A.put(so, s.data() + first / 32, n / 32 * 4);
  }
  return t;
}

}  // namespace

Lm::Lm(const std::string& dir, const Options& o) : opt_(o) {
  int count = 0;
  TRIT_CUDA(cudaGetDeviceCount(&count));
  if (opt_.device >= count) throw Error("options: device " + std::to_string(opt_.device) + " of " + std::to_string(count));
  TRIT_CUDA(cudaSetDevice(opt_.device));
  TRIT_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  for (auto& e : ev_) TRIT_CUDA(cudaEventCreate(&e));
  try {
    if (opt_.tp_size > 1) {
      // The ranks' communicator, from the unique id rank 0 made.
      if (opt_.tp_id.size() != 2 * sizeof(ncclUniqueId)) throw Error("options: tp_id must be trit_cuda_tp_id's text");
      ncclUniqueId id;
      for (size_t i = 0; i < sizeof id; ++i) id.internal[i] = (char)std::stoi(opt_.tp_id.substr(2 * i, 2), nullptr, 16);
      comm_ = nccl_join(id, opt_.tp_size, opt_.tp_rank, opt_.device, opt_.tp_timeout_s);
      if (opt_.decode == "persistent") opt_.decode = "layered";  // the persistent kernel runs a whole model
    }
    load(dir);
    alloc_buffers();
    setup_tensor_cores();
  } catch (...) {
    release();
    throw;
  }
}

Lm::~Lm() { release(); }

// TRIT_KERNEL_CLOCK=1: CUDA events between the steps of hidden() and the
// table; report() prints each step's total device time to stderr (a
// measurement aid; the batched decode then runs without its graph).
KernelClock::KernelClock() {
  const char* v = getenv("TRIT_KERNEL_CLOCK");
  on = v && *v == '1';
}
KernelClock::~KernelClock() {
  for (auto& e : pool) cudaEventDestroy(e);
}
void KernelClock::mark(const char* name, cudaStream_t s) {
  if (!on) return;
  if (used == pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return;
    pool.push_back(e);
  }
  cudaEventRecord(pool[used], s);
  names.push_back(name);
  ++used;
}
void KernelClock::report(const char* what) {
  if (!on || used < 2) {
    used = 0;
    names.clear();
    return;
  }
  cudaEventSynchronize(pool[used - 1]);
  std::map<std::string, double> total;
  double all = 0;
  for (size_t i = 0; i + 1 < used; ++i) {
    if (!names[i]) continue;
    float ms = 0;
    cudaEventElapsedTime(&ms, pool[i], pool[i + 1]);
    total[names[i]] += ms;
    all += ms;
  }
  fprintf(stderr, "kernel clock (%s): %.3f ms in marked steps\n", what, all);
  for (auto& kv : total) fprintf(stderr, "  %-26s %9.3f ms  %5.1f%%\n", kv.first.c_str(), kv.second, 100 * kv.second / all);
  used = 0;
  names.clear();
}

// Frees every device and pinned buffer; safe to call twice.
void Lm::release() {
  for (PrefixState* p : prefixes_) p->owner = nullptr;  // their pages go with the pool
  prefixes_.clear();
  cudaSetDevice(opt_.device);
  if (stream_) {
    try {
      wait();
    } catch (const std::exception&) {  // the communicator is aborted; the stream has drained
    }
  }
  void* bufs[] = {arena_, d_layers_, pool_, page_table_, x_, qkv_, att_, h_, xn_, xq_, xs_, row_stream_, row_pos_, ids_,
                  best_val_, best_idx_, tokens_, logits_, stop_, positions_, dll_, dstatus_, dcount_,
                  trace_, rope_};
  for (void* b : bufs)
    if (b) cudaFree(b);
  if (host_rows_) cudaFreeHost(host_rows_);
  if (batch_host_) cudaFreeHost(batch_host_);
  if (tiles_pinned_) cudaFreeHost(tiles_pinned_);
  if (tiles_dev_) cudaFree(tiles_dev_);
  tiles_pinned_ = nullptr;
  tiles_dev_ = nullptr;
  if (tc_w16_buf_) cudaFree(tc_w16_buf_);
  if (xq16_) cudaFree(xq16_);
  tc_w16_buf_ = nullptr;
  xq16_ = nullptr;
  tc_f16_ = false;
  void* batch[] = {batch_last_, batch_cur_, batch_step_, batch_tok_, tc_expanded_, gu_, tc_status_, ffn_scales_, audio_,
                   part_, keys_};
  for (void* b : batch)
    if (b) cudaFree(b);
  if (batch_graph_) cudaGraphExecDestroy(batch_graph_);
  batch_host_ = nullptr;
  batch_last_ = nullptr;
  batch_cur_ = batch_step_ = batch_tok_ = nullptr;
  tc_expanded_ = nullptr;
  ffn_scales_ = nullptr;
  audio_ = nullptr;
  part_ = nullptr;
  keys_ = nullptr;
  gu_ = nullptr;
  tc_status_ = nullptr;
  tc_ready_ = false;
  batch_graph_ = nullptr;
  // After the graph that holds its collectives.
  if (comm_) nccl().CommDestroy((ncclComm_t)comm_);
  comm_ = nullptr;
  batch_ready_ = false;
  if (ev_rows_) cudaEventDestroy(ev_rows_);
  ev_rows_ = nullptr;
  for (auto& e : ev_)
    if (e) cudaEventDestroy(e);
  if (stream_) cudaStreamDestroy(stream_);
  arena_ = pool_ = nullptr;
  d_layers_ = nullptr;
  page_table_ = nullptr;
  stream_ = nullptr;
  host_rows_ = nullptr;
  for (auto& e : ev_) e = nullptr;
  x_ = qkv_ = att_ = h_ = xn_ = nullptr;
  xq_ = nullptr; xs_ = nullptr; row_stream_ = row_pos_ = ids_ = nullptr; best_val_ = nullptr; best_idx_ = nullptr;
  tokens_ = nullptr; logits_ = nullptr; stop_ = nullptr; positions_ = nullptr; dll_ = nullptr;
  dstatus_ = nullptr;
  dcount_ = nullptr; trace_ = nullptr; rope_ = nullptr;
}

// ------------------------------------------------------------ weight cache --
// The arena's bytes (every weight in its device layout) in one file, so a
// later load reads them straight into device memory with no parsing or
// conversion (the weight store of src/cpu/store.rs:1-16,369-428, for the
// device layout). The file is named by a hash of what made it: the cache
// version, the source files' paths, sizes and modification times, the
// tensor prefix and the arena size. A file that does not match byte for
// byte (its header, its length, or the hash of its contents) is ignored
// and rewritten: the cache never changes a result, it only saves time.
namespace {

constexpr char kCacheMagic[8] = {'T', 'R', 'I', 'T', 'C', 'U', 'D', 'A'};
constexpr uint32_t kCacheVersion = 1;  // the arena layout; bump when it changes
constexpr size_t kCacheChunk = 64u << 20;

uint64_t mix64(uint64_t h, uint64_t w) {
  h ^= w + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
  return h * 0xff51afd7ed558ccdull;
}
uint64_t hash_bytes(uint64_t h, const uint8_t* p, size_t n) {
  size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    uint64_t w;
    std::memcpy(&w, p + i, 8);
    h = mix64(h, w);
  }
  for (; i < n; ++i) h = mix64(h, p[i]);
  return h;
}

struct CacheHeader {
  char magic[8];
  uint32_t version;
  uint32_t identity_bytes;
  uint64_t arena_bytes;
  uint64_t content_hash;
};

struct Pinned {
  void* p = nullptr;
  explicit Pinned(size_t n) { TRIT_CUDA(cudaMallocHost(&p, n)); }
  ~Pinned() {
    if (p) cudaFreeHost(p);
  }
};

}  // namespace

std::string Lm::weight_cache_identity(const ModelSource& src) const {
  std::string id = "trit-cuda weights v" + std::to_string(kCacheVersion) + "\n" + src.format + "\n" + src.prefix +
                   "\n" + std::to_string(arena_bytes_) + "\ntp " + std::to_string(tp_.rank) + "/" +
                   std::to_string(tp_.size) + "\n";
  for (const std::string& p : src.files->paths()) {
    struct stat st;
    if (::stat(p.c_str(), &st) != 0) throw Error("cannot stat " + p);
    id += p + " " + std::to_string((long long)st.st_size) + " " + std::to_string((long long)st.st_mtim.tv_sec) + "." +
          std::to_string((long long)st.st_mtim.tv_nsec) + "\n";
  }
  return id;
}

std::string Lm::weight_cache_path(const std::string& dir, const ModelSource& src) const {
  const std::string id = weight_cache_identity(src);
  char name[64];
  std::snprintf(name, sizeof name, "%016llx.bin", (unsigned long long)hash_bytes(1469598103934665603ull,
                                                                                    (const uint8_t*)id.data(), id.size()));
  const std::string folder = opt_.cache_dir.empty() ? dir + "/.trit_cuda" : opt_.cache_dir;
  return folder + "/" + name;
}

bool Lm::read_weight_cache(const std::string& path, void* arena, size_t bytes, cudaStream_t s) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  bool ok = false;
  try {
    CacheHeader h{};
    std::string want_id;
    if (std::fread(&h, sizeof h, 1, f) == 1 && std::memcmp(h.magic, kCacheMagic, 8) == 0 &&
        h.version == kCacheVersion && h.arena_bytes == bytes && h.identity_bytes < (1u << 20)) {
      std::string id(h.identity_bytes, '\0');
      if (std::fread(&id[0], 1, id.size(), f) == id.size()) {
        // Two pinned buffers: one fills from the file while the other copies.
        Pinned buf(2 * kCacheChunk);
        uint64_t hash = 1469598103934665603ull;
        size_t done = 0;
        int which = 0;
        bool short_read = false;
        while (done < bytes) {
          const size_t n = std::min(kCacheChunk, bytes - done);
          uint8_t* b = (uint8_t*)buf.p + which * kCacheChunk;
          TRIT_CUDA(cudaStreamSynchronize(s));  // the copy that used this half two chunks ago
          if (std::fread(b, 1, n, f) != n) {
            short_read = true;
            break;
          }
          hash = hash_bytes(hash, b, n);
          TRIT_CUDA(cudaMemcpyAsync((char*)arena + done, b, n, cudaMemcpyHostToDevice, s));
          done += n;
          which ^= 1;
        }
        TRIT_CUDA(cudaStreamSynchronize(s));
        ok = !short_read && hash == h.content_hash && std::fgetc(f) == EOF;
      }
    }
  } catch (...) {
    ok = false;
  }
  std::fclose(f);
  return ok;
}

void Lm::write_weight_cache(const std::string& path, const void* arena, size_t bytes, cudaStream_t s) {
  // Best effort: a folder that cannot be written leaves the load as it is.
  const std::string folder = path.substr(0, path.find_last_of('/'));
  ::mkdir(folder.c_str(), 0755);
  const std::string tmp = path + "." + std::to_string((long long)::getpid()) + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) return;
  bool ok = true;
  try {
    const std::string id = cache_identity_;
    CacheHeader h{};
    std::memcpy(h.magic, kCacheMagic, 8);
    h.version = kCacheVersion;
    h.identity_bytes = (uint32_t)id.size();
    h.arena_bytes = bytes;
    ok = std::fwrite(&h, sizeof h, 1, f) == 1 && std::fwrite(id.data(), 1, id.size(), f) == id.size();
    Pinned buf(kCacheChunk);
    uint64_t hash = 1469598103934665603ull;
    for (size_t done = 0; ok && done < bytes;) {
      const size_t n = std::min(kCacheChunk, bytes - done);
      TRIT_CUDA(cudaMemcpyAsync(buf.p, (const char*)arena + done, n, cudaMemcpyDeviceToHost, s));
      TRIT_CUDA(cudaStreamSynchronize(s));
      hash = hash_bytes(hash, (const uint8_t*)buf.p, n);
      ok = std::fwrite(buf.p, 1, n, f) == n;
      done += n;
    }
    h.content_hash = hash;
    ok = ok && std::fseek(f, 0, SEEK_SET) == 0 && std::fwrite(&h, sizeof h, 1, f) == 1;
  } catch (...) {
    ok = false;
  }
  ok = (std::fclose(f) == 0) && ok;
  if (ok) ok = std::rename(tmp.c_str(), path.c_str()) == 0;
  if (!ok) std::remove(tmp.c_str());
}

std::string Lm::status() const {
  auto quote = [](const std::string& v) {
    std::string o = "\"";
    for (char c : v) {
      if (c == '"' || c == '\\') o += '\\';
      o += c;
    }
    return o + "\"";
  };
  char buf[512];
  std::snprintf(buf, sizeof buf,
                "\"arena_bytes\": %zu, \"device\": %d, \"kv\": \"%s\", \"decode\": \"%s\", \"exact\": %s, "
                "\"prefix_pages\": [%d, %d], \"max_streams\": %d, \"max_context\": %d",
                arena_bytes_, opt_.device, opt_.kv_f16 ? "f16" : "f32", opt_.decode.c_str(),
                opt_.exact ? "true" : "false", prefix_pages_used(), prefix_pages_total(), opt_.max_streams,
                opt_.max_context);
  return "{\"source\": " + quote(source_) + ", \"weights_from\": " + quote(weights_from_) +
         ", \"weight_cache\": " + (cache_file_.empty() ? std::string("null") : quote(cache_file_)) + ", " + buf + "}";
}

// Config::parse (causal_lm.rs:41-77) and CausalLm::from_tensors (:141-198).
void Lm::load(const std::string& dir) {
  ModelSource src = open_model(dir, opt_.config_at, opt_.prefix);
  const ModelConfig& mc = src.mc;
  const std::string& prefix = src.prefix;
  source_ = src.format;
  cfg_ = mc.cfg;
  const bool qk_norm = mc.qk_norm;
  const float rope_base = mc.rope_base;
  tied_ = mc.tied;
  if (cfg_.hd != 128) throw Error("head_dim " + std::to_string(cfg_.hd) + ": the CUDA kernels take head_dim 128");
  // A tensor-parallel rank runs its shard: its heads, kv heads and FFN
  // units are the model's, as far as the kernels see.
  const DConfig full = cfg_;
  tp_ = tp_shard(full, opt_.tp_rank, opt_.tp_size);
  if (tp_.size > 1) {
    if (full.residual_multiplier != 1.0f) throw Error("tensor parallelism takes residual_multiplier 1");
    cfg_.heads = tp_.heads;
    cfg_.kv_heads = tp_.kv;
    cfg_.ffn = tp_.ffn;
  }
  if (cfg_.d % 128 || cfg_.ffn % 128) throw Error("hidden and intermediate sizes must be multiples of 128");

  const TensorFiles& g = *src.files;
  const int hd = cfg_.hd, qd = cfg_.heads * hd, kvd = cfg_.kv_heads * hd;
  bool has_head = !tied_ && g.find(prefix + "lm_head.weight");
  // Pass 0 sizes the arena; pass 1 lays the weights out in it, converting
  // them from the files, or only naming their places when the weight cache
  // already put the arena's bytes there.
  bool from_cache = false;
  std::string cache_file;
  for (int pass = 0; pass < 2; ++pass) {
    Arena A;
    A.fill = pass == 1 && !from_cache;
    A.base = (char*)arena_;
    layers_.assign(cfg_.layers, DLayer{});
    for (int l = 0; l < cfg_.layers; ++l) {
      std::string p = prefix + "model.layers." + std::to_string(l);
      DLayer& L = layers_[l];
      L.norm_attn = load_vector(g, A, p + ".input_layernorm.weight", cfg_.d);
      L.qkv = load_mat(g, A, {{p + ".self_attn.q_proj", tp_.heads0 * hd, qd}, {p + ".self_attn.k_proj", tp_.kv0 * hd, kvd},
                              {p + ".self_attn.v_proj", tp_.kv0 * hd, kvd}}, cfg_.d);
      if (qk_norm) {
        L.q_norm = load_vector(g, A, p + ".self_attn.q_norm.weight", hd);
        L.k_norm = load_vector(g, A, p + ".self_attn.k_norm.weight", hd);
      }
      L.out = load_mat(g, A, {{p + ".self_attn.o_proj", 0, cfg_.d}}, qd, tp_.heads0 * hd, full.heads * hd);
      L.norm_mlp = load_vector(g, A, p + ".post_attention_layernorm.weight", cfg_.d);
      L.gate_up = load_mat(g, A, {{p + ".mlp.gate_proj", tp_.ffn0, cfg_.ffn}, {p + ".mlp.up_proj", tp_.ffn0, cfg_.ffn}},
                           cfg_.d);
      L.down = load_mat(g, A, {{p + ".mlp.down_proj", 0, cfg_.d}}, cfg_.ffn, tp_.ffn0, full.ffn);
    }
    final_norm_ = load_vector(g, A, prefix + "model.norm.weight", cfg_.d);
    embed_ = load_table(g, A, prefix + "model.embed_tokens", cfg_.vocab, cfg_.d);
    head_ = has_head ? load_table(g, A, prefix + "lm_head", tp_.vocab, cfg_.d, tp_.vocab0, cfg_.vocab) : embed_;
    if (!has_head && tp_.size > 1) {
      // Tied: this rank's rows of the token table are the output table.
      const size_t sb = embed_.scale_f16 ? 2 : 4;
      head_.n = tp_.vocab;
      head_.codes = embed_.codes ? embed_.codes + (size_t)tp_.vocab0 * cfg_.d : nullptr;
      head_.scales = embed_.scales ? (const char*)embed_.scales + (size_t)tp_.vocab0 * (cfg_.d / 32) * sb : nullptr;
    }
    if (pass == 0) {
      arena_bytes_ = A.used;
      TRIT_CUDA(cudaMalloc(&arena_, arena_bytes_));
      if (opt_.weight_cache) {
        cache_identity_ = weight_cache_identity(src);
        cache_file = weight_cache_path(dir, src);
        from_cache = read_weight_cache(cache_file, arena_, arena_bytes_, stream_);
      }
    }
  }
  weights_from_ = from_cache ? "cache" : "files";
  cache_file_ = opt_.weight_cache ? cache_file : "";
  if (opt_.weight_cache && !from_cache) write_weight_cache(cache_file, arena_, arena_bytes_, stream_);
  TRIT_CUDA(cudaMalloc(&d_layers_, sizeof(DLayer) * cfg_.layers));
  TRIT_CUDA(cudaMemcpy(d_layers_, layers_.data(), sizeof(DLayer) * cfg_.layers, cudaMemcpyHostToDevice));

  // Rotary::halves (layers.rs:276-300): inv_freq = base^(-2i/hd) in f32, and
  // (position * f).sin_cos() in f32, here once per position: [pos][sin | cos].
  std::vector<float> inv(hd / 2);
  for (int i = 0; i < hd / 2; ++i) inv[i] = powf(rope_base, -((float)(2 * i)) / (float)hd);
  std::vector<float> table((size_t)opt_.max_context * hd);
  for (int p = 0; p < opt_.max_context; ++p)
    for (int i = 0; i < hd / 2; ++i) {
      float a = (float)p * inv[i];
      table[(size_t)p * hd + i] = sinf(a);
      table[(size_t)p * hd + hd / 2 + i] = cosf(a);
    }
  TRIT_CUDA(cudaMalloc(&rope_, table.size() * 4));
  TRIT_CUDA(cudaMemcpy(rope_, table.data(), table.size() * 4, cudaMemcpyHostToDevice));
}

void Lm::alloc_buffers() {
  const int d = cfg_.d, hd = cfg_.hd, qd = cfg_.heads * hd, kvd = cfg_.kv_heads * hd;
  // The paged cache: every stream slot owns pages_per_stream pages.
  cache_.f16 = opt_.kv_f16;
  cache_.page_tokens = opt_.page_tokens;
  cache_.pages_per_stream = (opt_.max_context + opt_.page_tokens - 1) / opt_.page_tokens;
  page_bytes_ = (size_t)cfg_.layers * 2 * cfg_.kv_heads * opt_.page_tokens * hd * (opt_.kv_f16 ? 2 : 4);
  // Then the pages kept for prefixes, which any slot's table row may name.
  size_t pages = (size_t)opt_.max_streams * cache_.pages_per_stream;
  prefix_pages_total_ = opt_.prefix_pages >= 0 ? opt_.prefix_pages : cache_.pages_per_stream;
  pool_pages_ = (size_t)pages + prefix_pages_total_;
  TRIT_CUDA(cudaMalloc(&pool_, pool_pages_ * page_bytes_));
  // Zeroed: positions past a stream's end are read (and masked) by the
  // tensor-core prompt attention, which must see finite values there.
  TRIT_CUDA(cudaMemset(pool_, 0, pool_pages_ * page_bytes_));
  cache_.pool = pool_;
  table_host_.resize(pages);
  for (size_t i = 0; i < pages; ++i) table_host_[i] = (int)i;
  prefix_free_.clear();
  for (int i = prefix_pages_total_ - 1; i >= 0; --i) prefix_free_.push_back((int)pages + i);
  TRIT_CUDA(cudaMalloc(&page_table_, pages * sizeof(int)));
  TRIT_CUDA(cudaMemcpy(page_table_, table_host_.data(), pages * sizeof(int), cudaMemcpyHostToDevice));
  cache_.page_table = page_table_;

  rows_cap_ = std::max(opt_.prefill_rows, opt_.max_streams);
  int kmax = std::max(std::max(d, qd), cfg_.ffn);
  TRIT_CUDA(cudaMalloc(&x_, (size_t)rows_cap_ * d * 4));
  TRIT_CUDA(cudaMalloc(&qkv_, (size_t)rows_cap_ * (qd + 2 * kvd) * 4));
  TRIT_CUDA(cudaMalloc(&att_, (size_t)rows_cap_ * qd * 4));
  TRIT_CUDA(cudaMalloc(&h_, (size_t)rows_cap_ * cfg_.ffn * 4));
  // Whole 64-row tiles: the tensor-core products read frames in tiles.
  TRIT_CUDA(cudaMalloc(&xq_, (size_t)((rows_cap_ + 63) / 64 * 64) * kmax));
  TRIT_CUDA(cudaMalloc(&xs_, (size_t)rows_cap_ * (kmax / 32) * 4));
  TRIT_CUDA(cudaMalloc(&row_stream_, (size_t)rows_cap_ * 4));
  TRIT_CUDA(cudaMalloc(&row_pos_, (size_t)rows_cap_ * 4));
  TRIT_CUDA(cudaMalloc(&ids_, (size_t)rows_cap_ * 4));
  TRIT_CUDA(cudaMalloc(&xn_, (size_t)opt_.max_streams * d * 4));
  if (tp_.size > 1) {
    TRIT_CUDA(cudaMalloc(&part_, (size_t)rows_cap_ * d * 4));
    TRIT_CUDA(cudaMalloc(&keys_, (size_t)std::max(rows_cap_, opt_.max_streams) * 8));
  }
  TRIT_CUDA(cudaMalloc(&best_val_, (size_t)opt_.max_streams * table_blocks(cfg_.vocab) * 4));
  TRIT_CUDA(cudaMalloc(&best_idx_, (size_t)opt_.max_streams * table_blocks(cfg_.vocab) * 4));
  TRIT_CUDA(cudaMalloc(&logits_, (size_t)cfg_.vocab * 4));
  TRIT_CUDA(cudaMalloc(&stop_, 256 * 4));
  TRIT_CUDA(cudaMallocHost(&host_rows_, ((size_t)2 * rows_cap_ + opt_.max_context + 16) * 4));
  TRIT_CUDA(cudaMalloc(&positions_, (size_t)opt_.max_context * std::max(1, opt_.max_streams) * 4));
  TRIT_CUDA(cudaMallocHost(&tiles_pinned_, (size_t)rows_cap_ * 8));
  TRIT_CUDA(cudaMalloc(&tiles_dev_, (size_t)rows_cap_ * 8));
}

void Lm::check_ids(const int* ids, size_t n) const {
  for (size_t i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= cfg_.vocab)
      throw Error("token id " + std::to_string(ids[i]) + " is outside the vocabulary of " + std::to_string(cfg_.vocab));
}

// CausalLm::hidden (causal_lm.rs:410-481) for the rows in x_, whose stream
// and position are in row_stream_ / row_pos_.
void Lm::final_rows(const float* x, int ldx, int nb, float* logits, int* tokens) {
  if (tp_.size == 1) {
    TRIT_CUDA(launch_final(x, ldx, nb, final_norm_, cfg_, head_, xn_, logits, best_val_, best_idx_, tokens, stream_));
    return;
  }
  // Each rank's best among its vocabulary rows, as argmax-ordered keys; the
  // largest key over the ranks is the first strict maximum of all rows.
  if (logits) throw Error("logit traces are not kept with tensor parallelism");
  if (!comm_) throw Error("tensor parallelism: this rank's communicator was aborted; load the model again");
  TRIT_CUDA(launch_final(x, ldx, nb, final_norm_, cfg_, head_, xn_, nullptr, best_val_, best_idx_, tokens, stream_,
                         keys_, tp_.vocab0));
  nccl_check(nccl().AllReduce(keys_, keys_, (size_t)nb, ncclUint64, ncclMax, (ncclComm_t)comm_, stream_),
             "argmax keys");
  TRIT_CUDA(launch_key_tokens(keys_, nb, tokens, stream_));
  timing_.gpu_launches += 1;
}

void Lm::wait() {
  if (!comm_) {
    if (tp_lost_) throw Error("tensor parallelism: this rank's communicator was aborted; load the model again");
    TRIT_CUDA(cudaStreamSynchronize(stream_));
    return;
  }
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(stream_);
    if (e == cudaSuccess) return;
    if (e != cudaErrorNotReady) TRIT_CUDA(e);
    ncclResult_t async = ncclSuccess;
    nccl().CommGetAsyncError((ncclComm_t)comm_, &async);
    const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if ((async != ncclSuccess && async != ncclInProgress) || waited > opt_.tp_timeout_s) {
      // Aborting ends the collectives in flight; the stream then drains.
      nccl().CommAbort((ncclComm_t)comm_);
      comm_ = nullptr;
      tp_lost_ = true;
      cudaStreamSynchronize(stream_);
      cudaGetLastError();
      if (async != ncclSuccess && async != ncclInProgress)
        throw Error(std::string("tensor parallelism: NCCL reported ") + nccl().GetErrorString(async));
      throw Error("tensor parallelism: the other ranks did not answer within " +
                  std::to_string((int)opt_.tp_timeout_s) + " s (a rank failed or left); the communicator is aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void Lm::reduce_into_x(int m) {
  if (!comm_) throw Error("tensor parallelism: this rank's communicator was aborted; load the model again");
  const size_t n = (size_t)m * cfg_.d;
  nccl_check(nccl().AllReduce(part_, part_, n, ncclFloat32, ncclSum, (ncclComm_t)comm_, stream_), "partial sums");
  TRIT_CUDA(launch_add(x_, part_, n, stream_));
  timing_.gpu_launches += 1;
}

void Lm::hidden(int m, int max_tk, const std::vector<std::pair<int, int>>* runs) {
  const int d = cfg_.d, qd = cfg_.heads * cfg_.hd, kvd = cfg_.kv_heads * cfg_.hd;
  cudaStream_t s = stream_;
  // Prompt tiles: a run of one stream's rows is cut into tiles whose rows
  // share the keys they read (the exact kernel's size, or 128 query rows of
  // the tensor-core kernel when "exact" is off).
  int ntiles = 0, rows_max = 0;
  const bool tc_attention = attention_tc_ && runs && causal_;
  if (runs && causal_ && !runs->empty()) {
    const int R = tc_attention ? attention_tc_rows(cfg_) : attention_tile_rows(cfg_, (max_tk + 3) / 4 * 4, cache_.f16);
    for (const auto& run : *runs)
      for (int r = 0; r < run.second; r += R) {
        tiles_pinned_[2 * ntiles] = run.first + r;
        tiles_pinned_[2 * ntiles + 1] = std::min(R, run.second - r);
        rows_max = std::max(rows_max, tiles_pinned_[2 * ntiles + 1]);
        ++ntiles;
      }
    TRIT_CUDA(cudaMemcpyAsync(tiles_dev_, tiles_pinned_, (size_t)ntiles * 8, cudaMemcpyHostToDevice, s));
  }
  const bool tc = tc_ready_ && m >= opt_.tc_rows;
  // One product: the tensor-core kernel for enough rows, else the GEMV.
  // xi: the width of the product's input (0: d, 1: heads * hd, 2: ffn).
  bool h_quantized = false;  // the tensor-core gate_up quantized h for the down product already
  auto product = [&](int l, int which, const DMat& W, int xi, int mode, float* y, int ldy, float mult) {
    if (!tc) {
      TRIT_CUDA(launch_gemv(W, xq_, xs_, m, mode, y, ldy, mult, s));
      return;
    }
    // Q8_0 layers with an f16 copy of their codes: the frames' codes as f16
    // too, and the exact f16 MMA.
    const bool f16 = tc_f16_ && W.kind == kQ8_0;
    if (f16) {
      TRIT_CUDA(launch_codes_f16(xq_, (size_t)m * W.k, xq16_, s));
      timing_.gpu_launches += 1;
    }
    const TcMap& wmap = f16 ? tc_w16_[(size_t)l * 4 + which] : tc_w_[(size_t)l * 4 + which];
    const TcMap& xmap = f16 ? tc_x16_[xi] : tc_x_[xi];
    if (mode == kEpSilu) {
      // h = silu(gate) * up, quantized straight into the down product's
      // input (h itself is needed by nothing else).
      TRIT_CUDA(launch_gemm_tc(wmap, xmap, W, xs_, m, kEpOut, gu_, W.n, 1.0f, tc_status_, s, f16));
      const DMat& D = layers_[l].down;
      TRIT_CUDA(launch_silu_quant(gu_, m, W.n / 2, D.agroup, D.half, xq_, xs_, s));
      timing_.gpu_launches += 1;
      h_quantized = true;
    } else {
      TRIT_CUDA(launch_gemm_tc(wmap, xmap, W, xs_, m, mode, y, ldy, mult, tc_status_, s, f16));
    }
  };
  if (cfg_.embedding_multiplier != 1.0f) TRIT_CUDA(launch_scale(x_, (size_t)m * d, cfg_.embedding_multiplier, s));
  for (int l = 0; l < cfg_.layers; ++l) {
    const DLayer& L = layers_[l];
    clock_.mark("norm+quant", s);
    TRIT_CUDA(launch_norm_quant(x_, m, d, L.norm_attn, cfg_.eps, L.qkv.agroup, L.qkv.half, xq_, xs_, s));
    clock_.mark("qkv", s);
    product(l, 0, L.qkv, 0, kEpOut, qkv_, qd + 2 * kvd, 1.0f);
    clock_.mark("qk norm+rope+append", s);
    TRIT_CUDA(launch_qk_rope_append(qkv_, m, cfg_, L.q_norm, L.k_norm, rope_, opt_.max_context, cache_, row_stream_,
                                    row_pos_, l, s));
    clock_.mark("attention", s);
    if (ntiles && tc_attention)
      TRIT_CUDA(launch_attention_tc(kv_map_, qkv_, (const int2*)tiles_dev_, ntiles, cfg_, cache_, row_stream_, row_pos_,
                                    l, att_, tc_status_, s));
    else if (ntiles)
      TRIT_CUDA(launch_attention_rows(qkv_, (const int2*)tiles_dev_, ntiles, rows_max, cfg_, cache_, row_stream_,
                                      row_pos_, l, max_tk, att_, s));
    else
      TRIT_CUDA(launch_attention_rows(qkv_, nullptr, m, 1, cfg_, cache_, row_stream_, row_pos_, l, max_tk, att_, s,
                                      causal_ ? 0 : max_tk));
    clock_.mark("norm+quant", s);
    TRIT_CUDA(launch_norm_quant(att_, m, qd, nullptr, cfg_.eps, L.out.agroup, L.out.half, xq_, xs_, s));
    clock_.mark("o", s);
    if (tp_.size > 1) {
      // A rank's heads give a partial sum of o; the ranks' sum joins x.
      product(l, 1, L.out, 1, kEpOut, part_, d, 1.0f);
      reduce_into_x(m);
    } else {
      product(l, 1, L.out, 1, kEpResid, x_, d, cfg_.residual_multiplier);
    }
    clock_.mark("norm+quant", s);
    TRIT_CUDA(launch_norm_quant(x_, m, d, L.norm_mlp, cfg_.eps, L.gate_up.agroup, L.gate_up.half, xq_, xs_, s,
                                L.ffn_scale));
    clock_.mark("gate_up", s);
    h_quantized = false;
    product(l, 2, L.gate_up, 0, kEpSilu, h_, cfg_.ffn, 1.0f);
    clock_.mark("norm+quant", s);
    if (!h_quantized)
      TRIT_CUDA(launch_norm_quant(h_, m, cfg_.ffn, nullptr, cfg_.eps, L.down.agroup, L.down.half, xq_, xs_, s));
    clock_.mark("down", s);
    if (tp_.size > 1) {
      product(l, 3, L.down, 2, kEpOut, part_, d, 1.0f);
      reduce_into_x(m);
    } else {
      product(l, 3, L.down, 2, kEpResid, x_, d, cfg_.residual_multiplier);
    }
    clock_.mark(nullptr, s);
  }
  timing_.gpu_launches += cfg_.layers * 10 + (cfg_.embedding_multiplier != 1.0f ? 1 : 0);
}

// CausalLm::set_ffn_scales (causal_lm.rs:305-307): the normed MLP input of
// layer l times scales[l] (hidden, :458-463); null clears them.
void Lm::set_ffn_scales(const float* scales) {
  TRIT_CUDA(cudaSetDevice(opt_.device));
  wait();
  if (scales) {
    if (!ffn_scales_) TRIT_CUDA(cudaMalloc(&ffn_scales_, (size_t)cfg_.layers * cfg_.d * 4));
    TRIT_CUDA(cudaMemcpy(ffn_scales_, scales, (size_t)cfg_.layers * cfg_.d * 4, cudaMemcpyHostToDevice));
  }
  for (int l = 0; l < cfg_.layers; ++l) layers_[l].ffn_scale = scales ? ffn_scales_ + (size_t)l * cfg_.d : nullptr;
  TRIT_CUDA(cudaMemcpy(d_layers_, layers_.data(), sizeof(DLayer) * cfg_.layers, cudaMemcpyHostToDevice));
}

// CausalLm::generate_additive (causal_lm.rs:317-345), Voxtral Realtime's
// loop: the prompt's embeddings plus audio rows [0, n), then each new
// token's embedding plus the next audio row, until a stop token or the
// rows run out (at most rows - n + 1 tokens). Decoded with the layered
// kernels, one added row per step.
std::vector<int> Lm::generate_additive(const int* ids, size_t n, const float* audio, size_t rows, const int* stop,
                                       size_t nstop, float* logits) {
  if (tp_.size > 1) throw Error("generate_additive does not run with tensor parallelism");
  std::vector<int> out;
  if (n == 0 || rows < n) return out;
  check_ids(ids, n);
  if (rows + 1 > (size_t)opt_.max_context) throw Error("audio rows exceed max_context " + std::to_string(opt_.max_context));
  timing_ = Timing{};
  TRIT_CUDA(cudaSetDevice(opt_.device));
  const int d = cfg_.d;
  if (audio_cap_ < rows) {
    if (audio_) cudaFree(audio_);
    audio_ = nullptr;
    TRIT_CUDA(cudaMalloc(&audio_, rows * d * 4));
    audio_cap_ = rows;
  }
  int* staged = stage_ids(ids, n, nullptr, 0);
  TRIT_CUDA(cudaEventRecord(ev_[0], stream_));
  map_slot(0, nullptr);
  TRIT_CUDA(cudaMemcpyAsync(audio_, audio, rows * d * 4, cudaMemcpyHostToDevice, stream_));
  run_prompt(n, 0, 0, [&](size_t c0, size_t c1) {
    embed_rows(staged, c0, c1, x_);
    TRIT_CUDA(launch_add(x_, audio_ + c0 * d, (c1 - c0) * d, stream_));
    timing_.gpu_launches += 1;
  });
  const int max_new = (int)(rows - n + 1);
  if (tokens_cap_ < max_new + 1) {
    if (tokens_) cudaFree(tokens_);
    tokens_ = nullptr;
    tokens_cap_ = max_new + 1;
    TRIT_CUDA(cudaMalloc(&tokens_, (size_t)tokens_cap_ * std::max(1, opt_.max_streams) * 4));
  }
  final_rows(x_ + (size_t)(last_rows_ - 1) * d, d, 1, logits ? logits_ : nullptr, tokens_);
  if (logits) TRIT_CUDA(cudaMemcpyAsync(logits, logits_, (size_t)cfg_.vocab * 4, cudaMemcpyDeviceToHost, stream_));
  TRIT_CUDA(cudaEventRecord(ev_[1], stream_));
  wait();
  int* host = host_rows_;
  host[0] = 0;
  TRIT_CUDA(cudaMemcpyAsync(row_stream_, host, 4, cudaMemcpyHostToDevice, stream_));
  int* hp = host_rows_ + 2 * rows_cap_;
  const int steps = max_new - 1;
  for (int i = 0; i < steps; ++i) hp[i] = (int)n + i;
  TRIT_CUDA(cudaMemcpyAsync(positions_, hp, (size_t)steps * 4, cudaMemcpyHostToDevice, stream_));
  int* saved = row_pos_;
  for (int i = 0; i < steps; ++i) {
    TRIT_CUDA(launch_embed(embed_, tokens_ + i, 1, x_, 1.0f, stream_));
    TRIT_CUDA(launch_add(x_, audio_ + (n + i) * d, d, stream_));
    row_pos_ = positions_ + i;
    hidden(1, (int)n + i + 1);
    row_pos_ = saved;
    TRIT_CUDA(launch_final(x_, d, 1, final_norm_, cfg_, head_, xn_, logits ? logits_ : nullptr, best_val_, best_idx_,
                           tokens_ + i + 1, stream_));
    timing_.gpu_launches += 5;
    if (logits)
      TRIT_CUDA(cudaMemcpyAsync(logits + (size_t)(i + 1) * cfg_.vocab, logits_, (size_t)cfg_.vocab * 4,
                                cudaMemcpyDeviceToHost, stream_));
  }
  row_pos_ = saved;
  TRIT_CUDA(cudaEventRecord(ev_[2], stream_));
  std::vector<int> toks(max_new);
  TRIT_CUDA(cudaMemcpyAsync(toks.data(), tokens_, (size_t)max_new * 4, cudaMemcpyDeviceToHost, stream_));
  wait();
  check_tc_status();
  float ms = 0;
  TRIT_CUDA(cudaEventElapsedTime(&ms, ev_[0], ev_[1]));
  timing_.prefill_ms = ms;
  TRIT_CUDA(cudaEventElapsedTime(&ms, ev_[1], ev_[2]));
  timing_.decode_ms = ms;
  timing_.decode_tokens = steps;
  for (int t : toks) {
    bool stopped = false;
    for (size_t k = 0; k < nstop; ++k) stopped |= t == stop[k];
    if (stopped) break;
    out.push_back(t);
  }
  return out;
}

// CausalLm::bidirectional_tokens (causal_lm.rs:393-408), Granite Speech
// NAR's editor: one pass over all rows with no causal mask (every row sees
// every key), then the best token of each row from `from` on. The rows
// must fit one pass (prefill_rows).
std::vector<int> Lm::bidirectional_tokens(const float* rows, size_t m, size_t from) {
  if (tp_.size > 1) throw Error("bidirectional_tokens does not run with tensor parallelism");
  if (from > m) throw Error("from (" + std::to_string(from) + ") is past the rows (" + std::to_string(m) + ")");
  if (m == 0) return {};
  if (m > (size_t)rows_cap_)
    throw Error(std::to_string(m) + " rows do not fit one pass of prefill_rows " + std::to_string(rows_cap_));
  if (m > (size_t)opt_.max_context) throw Error("more rows than max_context");
  timing_ = Timing{};
  TRIT_CUDA(cudaSetDevice(opt_.device));
  const int d = cfg_.d;
  wait();
  int* host = host_rows_;
  for (size_t r = 0; r < m; ++r) {
    host[r] = 0;
    host[rows_cap_ + r] = (int)r;
  }
  TRIT_CUDA(cudaEventRecord(ev_[0], stream_));
  map_slot(0, nullptr);
  TRIT_CUDA(cudaMemcpyAsync(row_stream_, host, m * 4, cudaMemcpyHostToDevice, stream_));
  TRIT_CUDA(cudaMemcpyAsync(row_pos_, host + rows_cap_, m * 4, cudaMemcpyHostToDevice, stream_));
  TRIT_CUDA(cudaMemcpyAsync(x_, rows, m * d * 4, cudaMemcpyHostToDevice, stream_));
  causal_ = false;
  try {
    hidden((int)m, (int)m);
  } catch (...) {
    causal_ = true;
    throw;
  }
  causal_ = true;
  const size_t nb = m - from;
  if (tokens_cap_ < (int)nb + 1) {
    if (tokens_) cudaFree(tokens_);
    tokens_ = nullptr;
    tokens_cap_ = (int)nb + 1;
    TRIT_CUDA(cudaMalloc(&tokens_, (size_t)tokens_cap_ * std::max(1, opt_.max_streams) * 4));
  }
  const size_t chunk = (size_t)std::max(1, opt_.max_streams);
  for (size_t r0 = 0; r0 < nb; r0 += chunk) {
    int c = (int)std::min(chunk, nb - r0);
    TRIT_CUDA(launch_final(x_ + (from + r0) * d, d, c, final_norm_, cfg_, head_, xn_, nullptr, best_val_, best_idx_,
                           tokens_ + r0, stream_));
    timing_.gpu_launches += 3;
  }
  std::vector<int> out(nb);
  TRIT_CUDA(cudaMemcpyAsync(out.data(), tokens_, nb * 4, cudaMemcpyDeviceToHost, stream_));
  TRIT_CUDA(cudaEventRecord(ev_[1], stream_));
  wait();
  check_tc_status();
  float ms = 0;
  TRIT_CUDA(cudaEventElapsedTime(&ms, ev_[0], ev_[1]));
  timing_.prefill_ms = ms;
  return out;
}

// The tensor-core products (mma.cu) for prefill and batches: TMA maps of
// every product's int8 codes (ternary layers get an int8 copy of their
// codes, c - 1, beside the 2-bit one the GEMV reads) and of the quantized
// frames for each input width. Off on a GPU other than sm_100 or when the
// "tensor_cores" option is false.
void Lm::setup_tensor_cores() {
  if (!opt_.tensor_cores) return;
  cudaDeviceProp prop;
  TRIT_CUDA(cudaGetDeviceProperties(&prop, opt_.device));
  if (prop.major != 10) return;
  const int d = cfg_.d, qd = cfg_.heads * cfg_.hd;
  size_t expanded = 0;
  for (const DLayer& L : layers_)
    for (const DMat* W : {&L.qkv, &L.out, &L.gate_up, &L.down})
      if (W->kind == kTernary) expanded += (size_t)W->n * W->k;
  if (expanded) TRIT_CUDA(cudaMalloc(&tc_expanded_, expanded));
  size_t at = 0;
  tc_w_.assign((size_t)cfg_.layers * 4, TcMap{});
  for (int l = 0; l < cfg_.layers; ++l) {
    const DLayer& L = layers_[l];
    const DMat* mats[4] = {&L.qkv, &L.out, &L.gate_up, &L.down};
    for (int i = 0; i < 4; ++i) {
      const void* codes = mats[i]->codes;
      if (mats[i]->kind == kTernary) {
        int8_t* dst = tc_expanded_ + at;
        TRIT_CUDA(launch_expand_ternary(*mats[i], dst, stream_));
        at += (size_t)mats[i]->n * mats[i]->k;
        codes = dst;
      }
      TRIT_CUDA(make_tc_weight_map(&tc_w_[(size_t)l * 4 + i], *mats[i], codes));
    }
  }
  const size_t rows8 = (size_t)(rows_cap_ + 63) / 64 * 64;
  const int widths[3] = {d, qd, cfg_.ffn};
  for (int i = 0; i < 3; ++i) TRIT_CUDA(make_tc_frame_map(&tc_x_[i], xq_, rows8, (size_t)widths[i]));
  // The f16 form of the Q8_0 products (exact f32 dots from the tensor cores,
  // no integer bias in the fold): an f16 copy of each Q8_0 layer's codes,
  // and an f16 buffer for the frames' codes.
  if (opt_.tc_f16) {
    size_t bytes = 0;
    for (const DLayer& L : layers_)
      for (const DMat* W : {&L.qkv, &L.out, &L.gate_up, &L.down})
        if (W->kind == kQ8_0) bytes += (size_t)W->n * W->k * 2;
    if (bytes) {
      TRIT_CUDA(cudaMalloc(&tc_w16_buf_, bytes));
      tc_w16_.assign((size_t)cfg_.layers * 4, TcMap{});
      size_t at16 = 0;
      for (int l = 0; l < cfg_.layers; ++l) {
        const DLayer& L = layers_[l];
        const DMat* mats[4] = {&L.qkv, &L.out, &L.gate_up, &L.down};
        for (int i = 0; i < 4; ++i) {
          if (mats[i]->kind != kQ8_0) continue;
          char* dst = (char*)tc_w16_buf_ + at16;
          TRIT_CUDA(launch_codes_f16((const int8_t*)mats[i]->codes, (size_t)mats[i]->n * mats[i]->k, dst, stream_));
          TRIT_CUDA(make_tc_map_f16(&tc_w16_[(size_t)l * 4 + i], dst, (size_t)mats[i]->n, (size_t)mats[i]->k, 128));
          at16 += (size_t)mats[i]->n * mats[i]->k * 2;
        }
      }
      const int kmax = std::max(std::max(d, qd), cfg_.ffn);
      TRIT_CUDA(cudaMalloc(&xq16_, rows8 * kmax * 2));
      for (int i = 0; i < 3; ++i) TRIT_CUDA(make_tc_map_f16(&tc_x16_[i], xq16_, rows8, (size_t)widths[i], 16));
      tc_f16_ = true;
    }
  }
  TRIT_CUDA(cudaMalloc(&gu_, (size_t)rows_cap_ * 2 * cfg_.ffn * 4));
  TRIT_CUDA(cudaMalloc(&tc_status_, 4));
  TRIT_CUDA(cudaMemset(tc_status_, 0, 4));
  // "exact": false: prompt attention on the tensor cores (f16 cache, pages
  // of a multiple of 64 positions), over a TMA view of the whole pool.
  if (opt_.tc_attention && attention_tc_supported(cfg_, cache_)) {
    const size_t rows = pool_pages_ * (size_t)cfg_.layers * 2 * cfg_.kv_heads * cache_.page_tokens;
    TRIT_CUDA(make_kv_map(&kv_map_, pool_, rows));
    attention_tc_ = true;
  }
  wait();
  tc_ready_ = true;
}

// Throws if a tensor-core product gave up waiting (its status word).
void Lm::check_tc_status() {
  if (!tc_ready_) return;
  int st = 0;
  TRIT_CUDA(cudaMemcpy(&st, tc_status_, 4, cudaMemcpyDeviceToHost));
  if (st) {
    cudaMemset(tc_status_, 0, 4);
    throw Error("a tensor-core product gave up waiting for its pipeline (status " + std::to_string(st) + ")");
  }
}

// The prompt rows through every layer, prefill_rows at a time (causal
// attention sees the earlier chunks through the cache). `fill(c0, c1)`
// writes prompt rows c0..c1 into x_ (embedded, before the embedding
// multiplier). Leaves the last chunk in x_ and its row count in last_rows_.
void Lm::run_prompt(size_t m, int slot, int first, const std::function<void(size_t, size_t)>& fill) {
  int* host = host_rows_;
  for (size_t c0 = 0; c0 < m; c0 += rows_cap_) {
    int mc = (int)std::min<size_t>(rows_cap_, m - c0);
    wait();  // the pinned row metadata is reused per chunk
    for (int r = 0; r < mc; ++r) {
      host[r] = slot;
      host[rows_cap_ + r] = first + (int)c0 + r;
    }
    TRIT_CUDA(cudaMemcpyAsync(row_stream_, host, mc * 4, cudaMemcpyHostToDevice, stream_));
    TRIT_CUDA(cudaMemcpyAsync(row_pos_, host + rows_cap_, mc * 4, cudaMemcpyHostToDevice, stream_));
    fill(c0, c0 + mc);
    const int top = first + (int)c0 + mc;
    const std::vector<std::pair<int, int>> runs = {{0, mc}};  // one stream
    hidden(mc, top, &runs);
    last_rows_ = mc;
  }
}

// Token ids of the prompt, staged once in pinned memory: rows c0..c1 are
// embedded from there.
void Lm::embed_rows(const int* ids, size_t c0, size_t c1, float* x) {
  int* staged = host_rows_ + 2 * rows_cap_;
  if (ids != staged) throw Error("internal: ids are not staged");
  TRIT_CUDA(cudaMemcpyAsync(ids_ + c0 % rows_cap_, staged + c0, (c1 - c0) * 4, cudaMemcpyHostToDevice, stream_));
  TRIT_CUDA(launch_embed(embed_, ids_ + c0 % rows_cap_, (int)(c1 - c0), x, 1.0f, stream_));
  timing_.gpu_launches += 1;
}

int* Lm::stage_ids(const int* a, size_t na, const int* b, size_t nb) {
  if (na + nb > (size_t)opt_.max_context) throw Error("more prompt ids than max_context");
  wait();
  int* staged = host_rows_ + 2 * rows_cap_;
  if (na) std::memcpy(staged, a, na * 4);
  if (nb) std::memcpy(staged + na, b, nb * 4);
  return staged;
}

std::vector<int> Lm::generate(const PrefixState* prefix, const int* ids, size_t n, int max_new, const int* stop,
                              size_t nstop, float* logits) {
  if (n == 0) throw Error("the prompt is empty");
  check_ids(ids, n);
  bool use = prefix && n > prefix->tokens.size() && std::equal(prefix->tokens.begin(), prefix->tokens.end(), ids);
  size_t done = use ? prefix->tokens.size() : 0;
  if (n + (size_t)std::max(max_new, 0) > (size_t)opt_.max_context)
    throw Error("prompt plus max_new (" + std::to_string(n + max_new) + ") exceeds max_context " +
                std::to_string(opt_.max_context));
  timing_ = Timing{};
  TRIT_CUDA(cudaSetDevice(opt_.device));
  int* staged = stage_ids(ids + done, n - done, nullptr, 0);
  TRIT_CUDA(cudaEventRecord(ev_[0], stream_));
  map_slot(0, use ? prefix : nullptr);  // the prefix's pages, read in place
  run_prompt(n - done, 0, (int)done, [&](size_t c0, size_t c1) { embed_rows(staged, c0, c1, x_); });
  return finish(0, (int)n, max_new, stop, nstop, logits);
}

std::vector<int> Lm::generate_rows(const float* rows, size_t nrows, int max_new, const int* stop, size_t nstop,
                                   float* logits) {
  return answer(nullptr, 0, rows, nrows, nullptr, 0, max_new, stop, nstop, logits);
}

// CausalLm::answer (causal_lm.rs:264-282): [embed(head); audio; embed(tail)]
// as the prompt rows, then generate_rows (:251-262).
std::vector<int> Lm::answer(const int* head, size_t nhead, const float* audio, size_t naudio, const int* tail,
                            size_t ntail, int max_new, const int* stop, size_t nstop, float* logits,
                            cudaStream_t audio_stream, bool audio_on_device) {
  size_t m = nhead + naudio + ntail;
  if (m == 0) throw Error("no prompt rows");
  check_ids(head, nhead);
  check_ids(tail, ntail);
  if (m + (size_t)std::max(max_new, 0) > (size_t)opt_.max_context)
    throw Error("prompt plus max_new exceeds max_context " + std::to_string(opt_.max_context));
  timing_ = Timing{};
  TRIT_CUDA(cudaSetDevice(opt_.device));
  int* staged = stage_ids(head, nhead, tail, ntail);  // head ids then tail ids
  if (audio_on_device && naudio) {
    // Rows in device memory (an encoder's output on this GPU): check that
    // they are, then order their reads after the caller's stream.
    cudaPointerAttributes attr{};
    TRIT_CUDA(cudaPointerGetAttributes(&attr, audio));
    if ((attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) || attr.device != opt_.device)
      throw Error("the rows are not device memory of CUDA device " + std::to_string(opt_.device));
    if (!ev_rows_) TRIT_CUDA(cudaEventCreateWithFlags(&ev_rows_, cudaEventDisableTiming));
    TRIT_CUDA(cudaEventRecord(ev_rows_, audio_stream));
    TRIT_CUDA(cudaStreamWaitEvent(stream_, ev_rows_, 0));
  }
  const cudaMemcpyKind rows_kind = audio_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  TRIT_CUDA(cudaEventRecord(ev_[0], stream_));
  map_slot(0, nullptr);
  const int d = cfg_.d;
  run_prompt(m, 0, 0, [&](size_t c0, size_t c1) {
    for (size_t r = c0; r < c1;) {
      float* dst = x_ + (r - c0) * d;
      if (r < nhead) {
        size_t e = std::min(c1, nhead);
        embed_rows(staged, r, e, dst);
        r = e;
      } else if (r < nhead + naudio) {
        size_t e = std::min(c1, nhead + naudio);
        TRIT_CUDA(cudaMemcpyAsync(dst, audio + (r - nhead) * d, (e - r) * d * 4, rows_kind, stream_));
        r = e;
      } else {
        // Tail ids sit after the head ids in the staging area.
        size_t e = c1;
        size_t s0 = nhead + (r - nhead - naudio), s1 = s0 + (e - r);
        TRIT_CUDA(cudaMemcpyAsync(ids_, staged + s0, (s1 - s0) * 4, cudaMemcpyHostToDevice, stream_));
        TRIT_CUDA(launch_embed(embed_, ids_, (int)(s1 - s0), dst, 1.0f, stream_));
        timing_.gpu_launches += 1;
        r = e;
      }
    }
  });
  return finish(0, (int)m, max_new, stop, nstop, logits);
}

// After a prefill whose last chunk is in x_: the last row's logits, then
// greedy steps (CausalLm::greedy, causal_lm.rs:284-302). The forward after
// the last kept token changes no output and is not run.
std::vector<int> Lm::finish(int slot, int position, int max_new, const int* stop, size_t nstop, float* logits) {
  std::vector<int> out;
  clock_.report("prefill");
  if (max_new <= 0) {
    wait();
    check_tc_status();
    return out;
  }
  if (tokens_cap_ < max_new + 1) {
    if (tokens_) cudaFree(tokens_);
    tokens_ = nullptr;
    tokens_cap_ = max_new + 1;
    TRIT_CUDA(cudaMalloc(&tokens_, (size_t)tokens_cap_ * std::max(1, opt_.max_streams) * 4));
  }
  final_rows(x_ + (size_t)(last_rows_ - 1) * cfg_.d, cfg_.d, 1, logits ? logits_ : nullptr, tokens_);
  timing_.gpu_launches += 3;
  if (logits) TRIT_CUDA(cudaMemcpyAsync(logits, logits_, (size_t)cfg_.vocab * 4, cudaMemcpyDeviceToHost, stream_));
  TRIT_CUDA(cudaEventRecord(ev_[1], stream_));
  int steps = max_new - 1;  // forwards after the prompt's
  if (nstop > 256) throw Error("more than 256 stop ids");
  nstop_ = (int)nstop;
  if (nstop) TRIT_CUDA(cudaMemcpyAsync(stop_, stop, nstop * 4, cudaMemcpyHostToDevice, stream_));
  if (steps > 0) {
    if (opt_.decode == "persistent") decode_persistent(slot, position, steps, logits);
    else decode_layered(slot, position, steps, logits);
  }
  TRIT_CUDA(cudaEventRecord(ev_[2], stream_));
  clock_.report("generate");
  std::vector<int> toks(max_new);
  TRIT_CUDA(cudaMemcpyAsync(toks.data(), tokens_, (size_t)max_new * 4, cudaMemcpyDeviceToHost, stream_));
  wait();
  check_tc_status();
  float ms = 0;
  TRIT_CUDA(cudaEventElapsedTime(&ms, ev_[0], ev_[1]));
  timing_.prefill_ms = ms;
  TRIT_CUDA(cudaEventElapsedTime(&ms, ev_[1], ev_[2]));
  timing_.decode_ms = ms;
  timing_.decode_tokens = steps;
  for (int i = 0; i < max_new; ++i) {
    bool stopped = false;
    for (size_t s = 0; s < nstop; ++s) stopped |= toks[i] == stop[s];
    if (stopped) break;
    out.push_back(toks[i]);
  }
  return out;
}

// Batch-1 decode through the layered kernels: step i feeds tokens_[i] at
// position + i and writes tokens_[i + 1]; every step's position is in
// positions_ from the start, so no step waits for the host.
void Lm::decode_layered(int slot, int position, int steps, float* trace) {
  wait();
  int* host = host_rows_;
  host[0] = slot;
  int* hp = host_rows_ + 2 * rows_cap_;  // free again: the prompt is in
  for (int i = 0; i < steps; ++i) hp[i] = position + i;
  TRIT_CUDA(cudaMemcpyAsync(row_stream_, host, 4, cudaMemcpyHostToDevice, stream_));
  TRIT_CUDA(cudaMemcpyAsync(positions_, hp, (size_t)steps * 4, cudaMemcpyHostToDevice, stream_));
  int* saved = row_pos_;
  for (int i = 0; i < steps; ++i) {
    TRIT_CUDA(launch_embed(embed_, tokens_ + i, 1, x_, 1.0f, stream_));
    row_pos_ = positions_ + i;
    hidden(1, position + i + 1);
    row_pos_ = saved;
    final_rows(x_, cfg_.d, 1, trace ? logits_ : nullptr, tokens_ + i + 1);
    timing_.gpu_launches += 4;
    if (trace)
      TRIT_CUDA(cudaMemcpyAsync(trace + (size_t)(i + 1) * cfg_.vocab, logits_, (size_t)cfg_.vocab * 4,
                                cudaMemcpyDeviceToHost, stream_));
  }
  row_pos_ = saved;
}

// Batch-1 decode in one cooperative kernel (decode.cu): step i feeds
// tokens_[i] at position + i; the kernel stops at a stop token.
// Batch-1 decode in one cooperative kernel (decode.cu): step i feeds
// tokens_[i] at position + i; the kernel stops at a stop token.
void Lm::decode_persistent(int slot, int position, int steps, float* trace) {
  if (!decode_grid_) {
    decode_grid_ = decode_grid(opt_.device);
    if (decode_grid_ < cfg_.kv_heads) throw Error("too few SMs for the persistent decode");
    ll_words_ = std::max(decode_ll_words(cfg_, decode_grid_), decode_fast_ll_words(cfg_, decode_grid_));
    TRIT_CUDA(cudaMalloc(&dll_, ll_words_ * 8));
    TRIT_CUDA(cudaMalloc(&dstatus_, 4));
    TRIT_CUDA(cudaMalloc(&dcount_, 4));
  }
  // The default path sums in tree order (decode_fast.cu); "exact" keeps the
  // reference's order (decode.cu).
  const bool fast = !opt_.exact && decode_fast_supported(cfg_, head_, decode_grid_, cache_.f16);
  if (!fast && !decode_supported(cfg_))
    throw Error("the persistent decode takes widths up to 8192 in multiples of 128; use {\"decode\": \"layered\"}");
  float* dtrace = nullptr;
  if (trace) {
    size_t need = (size_t)(steps + 1) * cfg_.vocab;
    if (trace_cap_ < need) {
      if (trace_) cudaFree(trace_);
      trace_ = nullptr;
      TRIT_CUDA(cudaMalloc(&trace_, need * 4));
      trace_cap_ = need;
    }
    dtrace = trace_;
  }
  DecodeArgs a{};
  a.cfg = cfg_;
  a.layers = d_layers_;
  a.final_norm = final_norm_;
  a.table = head_;
  a.embed = embed_;
  a.cache = cache_;
  a.rope = rope_;
  a.rope_rows = opt_.max_context;
  a.stream = slot;
  a.first_pos = position;
  a.steps = steps;
  a.stop = stop_;
  a.nstop = nstop_;
  a.tokens = tokens_;
  a.count = dcount_;
  a.logits = dtrace;
  a.ll = dll_;
  a.status = dstatus_;
  // TRIT_PHASE_TRACE=1: stamp every phase of block 0 and print the mean time
  // of each phase kind to stderr (a measurement aid).
  static const bool trace_phases = getenv("TRIT_PHASE_TRACE") && *getenv("TRIT_PHASE_TRACE") == '1';
  const int per_layer = fast ? 4 : 5;
  const int marks = per_layer * cfg_.layers + 2;
  long long* dphase = nullptr;
  if (trace_phases) {
    TRIT_CUDA(cudaMallocAsync(&dphase, (size_t)steps * marks * 8, stream_));
    TRIT_CUDA(cudaMemsetAsync(dphase, 0, (size_t)steps * marks * 8, stream_));
  }
  a.phase_ns = dphase;
  // TRIT_PHASE_TRACE=3: per-block stamps of kEventSlots events a layer for one step.
  static const bool trace_events = getenv("TRIT_PHASE_TRACE") && *getenv("TRIT_PHASE_TRACE") == '3';
  long long* devents = nullptr;
  const size_t nev = (size_t)cfg_.layers * kEventSlots * decode_grid_;
  if (trace_events && steps > 3) {
    TRIT_CUDA(cudaMallocAsync(&devents, nev * 8, stream_));
    TRIT_CUDA(cudaMemsetAsync(devents, 0, nev * 8, stream_));
  }
  a.events = devents;
  a.event_step = 2;
  TRIT_CUDA(cudaMemsetAsync(dll_, 0, ll_words_ * 8, stream_));
  TRIT_CUDA(cudaMemsetAsync(dstatus_, 0, 4, stream_));
  TRIT_CUDA(fast ? launch_decode_fast(a, decode_grid_, stream_) : launch_decode(a, decode_grid_, stream_));
  timing_.gpu_launches += 1;
  int status = 0;
  TRIT_CUDA(cudaMemcpyAsync(&status, dstatus_, 4, cudaMemcpyDeviceToHost, stream_));
  if (trace)
    TRIT_CUDA(cudaMemcpyAsync(trace + cfg_.vocab, dtrace + cfg_.vocab, (size_t)steps * cfg_.vocab * 4,
                              cudaMemcpyDeviceToHost, stream_));
  wait();
  if (dphase) {
    std::vector<long long> t((size_t)steps * marks);
    TRIT_CUDA(cudaMemcpy(t.data(), dphase, t.size() * 8, cudaMemcpyDeviceToHost));
    TRIT_CUDA(cudaFree(dphase));
    // Stamps per step: start, then per layer the end of each phase (exact:
    // qkv, attention, o, gate_up, down; default: qkv, attention + o,
    // gate_up, down), then the argmax.
    double sum[7] = {0};
    int n[7] = {0};
    for (int st = 1; st < steps; ++st) {
      const long long* r = t.data() + (size_t)st * marks;
      if (!r[marks - 1]) continue;
      for (int l = 0; l < cfg_.layers; ++l)
        for (int p = 0; p < per_layer; ++p) {
          sum[p] += (double)(r[l * per_layer + p + 1] - r[l * per_layer + p]);
          n[p]++;
        }
      sum[5] += (double)(r[marks - 1] - r[marks - 2]);
      n[5]++;
      sum[6] += (double)(r[marks - 1] - r[0]);
      n[6]++;
    }
    const char* exact_names[7] = {"qkv", "attention", "o", "gate_up", "down", "table", "step"};
    const char* fast_names[7] = {"qkv", "attend+o", "gate_up", "down", "", "table", "step"};
    const char* const* names = fast ? fast_names : exact_names;
    for (int p = 0; p < 7; ++p)
      if (n[p]) fprintf(stderr, "phase %-9s %8.2f us\n", names[p], sum[p] / n[p] / 1e3);
  }
  if (devents) {
    std::vector<long long> t(nev);
    TRIT_CUDA(cudaMemcpy(t.data(), devents, nev * 8, cudaMemcpyDeviceToHost));
    TRIT_CUDA(cudaFree(devents));
    const char* fast_names[kEventSlots] = {"layer start", "P1 x arrived", "P1 norm+quant", "P1 qkv rows",
                                           "P1 published", "P2 qkv arrived", "P2 attention", "P2 quantize",
                                           "P2 o partial rows", "P2 published", "P4 partials arrived",
                                           "P4 norm+quant", "P4 gate_up rows", "P4 published", "P5 h arrived",
                                           "P5 quantize", "P5 down rows", "P5 published", "table x arrived",
                                           "table norm", "table rows", "argmax bests arrived", "", "", "", "", "",
                                           "", "", "", "", ""};
    const char* exact_names[kEventSlots] = {"layer start", "P1 x arrived", "P1 norm+quant", "P1 qkv rows", "P1 published",
                                      "P2 qkv arrived", "P2 attention", "P2 published", "P3 attq arrived", "P3 o rows",
                                      "P4 xa arrived", "P4 norm+quant", "P4 gate_up rows", "P5 h arrived",
                                      "P5 quantize", "P5 down rows", "P1 weights in smem", "P1 dots", "P1 chains",
                                      "P3 weights in smem", "P3 dots", "P3 chains", "P4 weights in smem", "P4 dots",
                                      "P4 chains", "P5 weights in smem", "P5 dots", "P5 chains", "P2 qk norm+rope",
                                      "", "", ""};
    const char* const* names = fast ? fast_names : exact_names;
    // Per block and layer: the stamps in time order; each interval is
    // charged to the stamp that ends it.
    const int G = decode_grid_;
    double sum[kEventSlots] = {0}, mx[kEventSlots] = {0};
    long cnt[kEventSlots] = {0};
    for (int l = 1; l < cfg_.layers; ++l)
      for (int c = 0; c < G; ++c) {
        std::vector<std::pair<long long, int>> st;
        for (int k = 0; k < kEventSlots; ++k) {
          long long v = t[((size_t)l * kEventSlots + k) * G + c];
          if (v) st.emplace_back(v, k);
        }
        std::sort(st.begin(), st.end());
        for (size_t i2 = 1; i2 < st.size(); ++i2) {
          double d = (double)(st[i2].first - st[i2 - 1].first) / 1e3;
          sum[st[i2].second] += d;
          mx[st[i2].second] = std::max(mx[st[i2].second], d);
          ++cnt[st[i2].second];
        }
      }
    for (int k = 1; k < kEventSlots; ++k)
      if (cnt[k])
        fprintf(stderr, "event %-20s mean %7.2f us  max %7.2f us  (%ld)\n", names[k], sum[k] / cnt[k], mx[k], cnt[k]);
  }
  if (status) throw Error("the persistent decode gave up waiting for another block (status " + std::to_string(status) + ")");
}

void Lm::embed(const int* ids, size_t n, float* out) {
  check_ids(ids, n);
  TRIT_CUDA(cudaSetDevice(opt_.device));
  for (size_t c0 = 0; c0 < n; c0 += rows_cap_) {
    size_t mc = std::min<size_t>(rows_cap_, n - c0);
    TRIT_CUDA(cudaMemcpyAsync(ids_, ids + c0, mc * 4, cudaMemcpyHostToDevice, stream_));
    TRIT_CUDA(launch_embed(embed_, ids_, (int)mc, x_, 1.0f, stream_));
    TRIT_CUDA(cudaMemcpyAsync(out + c0 * cfg_.d, x_, mc * cfg_.d * 4, cudaMemcpyDeviceToHost, stream_));
    wait();
  }
}

// CausalLm::prefix (causal_lm.rs:202-215): the prompt start through every
// layer; its pages are kept.
std::unique_ptr<PrefixState> Lm::prefix(const int* ids, size_t n) {
  check_ids(ids, n);
  if (n > (size_t)opt_.max_context) throw Error("the prefix is longer than max_context");
  auto p = std::make_unique<PrefixState>();
  p->tokens.assign(ids, ids + n);
  if (n == 0) return p;
  TRIT_CUDA(cudaSetDevice(opt_.device));
  // Its full pages take kept pages, and the prompt is run straight into
  // them through slot 0's table row; the partial page after them is run
  // into slot 0's own page and copied out.
  const size_t full = n / opt_.page_tokens;
  if (full > prefix_free_.size())
    throw Error("the prefix needs " + std::to_string(full) + " KV pages and " + std::to_string(prefix_free_.size()) +
                " of the kept pages are free (load option prefix_pages)");
  for (size_t i = 0; i < full; ++i) {
    p->pages.push_back(prefix_free_.back());
    prefix_free_.pop_back();
  }
  p->owner = this;
  prefixes_.insert(p.get());
  try {
    int* staged = stage_ids(ids, n, nullptr, 0);
    map_slot(0, p.get());
    run_prompt(n, 0, 0, [&](size_t c0, size_t c1) { embed_rows(staged, c0, c1, x_); });
    if (n % opt_.page_tokens) {
      TRIT_CUDA(cudaMalloc(&p->partial, page_bytes_));
      const char* own = (const char*)pool_ + full * page_bytes_;  // slot 0, logical page `full`
      TRIT_CUDA(cudaMemcpyAsync(p->partial, own, page_bytes_, cudaMemcpyDeviceToDevice, stream_));
    }
    wait();
    check_tc_status();
  } catch (...) {
    release_prefix(p.get());  // under the caller's lock already
    throw;
  }
  return p;
}

// Independent greedy generations decoded side by side: CausalLm::generate
// (causal_lm.rs:217-249) and greedy (:284-302) for every stream, each
// stream in its own KV slot. The prompts of all streams share prefill
// passes (every row carries its stream and position). Each greedy step runs
// the rows of all streams through the layered kernels; the step is captured
// once as a CUDA graph and replayed, since its kernels read the tokens and
// positions from device buffers that a small kernel advances. Every stream
// runs max_new steps; the host cuts each at its first stop token.
void Lm::generate_batch(size_t S, const int* const* prompts, const size_t* lens, int max_new, const int* stop,
                        size_t nstop, int* out, int64_t* counts, const PrefixState* prefix) {
  if (S == 0) return;
  if (S > (size_t)opt_.max_streams)
    throw Error(std::to_string(S) + " streams exceed max_streams " + std::to_string(opt_.max_streams));
  size_t total = 0, longest = 0;
  for (size_t s = 0; s < S; ++s) {
    if (!prompts[s]) throw Error("prompt " + std::to_string(s) + " is NULL");
    if (lens[s] == 0) throw Error("prompt " + std::to_string(s) + " is empty");
    check_ids(prompts[s], lens[s]);
    if (lens[s] + (size_t)std::max(max_new, 0) > (size_t)opt_.max_context)
      throw Error("stream " + std::to_string(s) + ": prompt plus max_new exceeds max_context " +
                  std::to_string(opt_.max_context));
    total += lens[s];
    longest = std::max(longest, lens[s]);
  }
  timing_ = Timing{};
  for (size_t s = 0; s < S; ++s) counts[s] = 0;
  if (max_new <= 0) return;
  TRIT_CUDA(cudaSetDevice(opt_.device));
  const int d = cfg_.d;
  if (!batch_ready_) {
    TRIT_CUDA(cudaMallocHost(&batch_host_, (size_t)3 * rows_cap_ * 4));
    TRIT_CUDA(cudaMalloc(&batch_last_, (size_t)opt_.max_streams * d * 4));
    TRIT_CUDA(cudaMalloc(&batch_cur_, (size_t)opt_.max_streams * 4));
    TRIT_CUDA(cudaMalloc(&batch_step_, 4));
    batch_ready_ = true;
  }
  if (batch_tok_cap_ < (size_t)max_new * S) {
    if (batch_tok_) cudaFree(batch_tok_);
    batch_tok_ = nullptr;
    TRIT_CUDA(cudaMalloc(&batch_tok_, (size_t)max_new * S * 4));
    batch_tok_cap_ = (size_t)max_new * S;
    if (batch_graph_) cudaGraphExecDestroy(batch_graph_);  // it holds the old buffer's address
    batch_graph_ = nullptr;
  }
  TRIT_CUDA(cudaEventRecord(ev_[0], stream_));
  // A stream whose prompt starts with the prefix (and is longer) points its
  // first pages at the prefix's and starts its prompt after it.
  std::vector<size_t> start(S, 0);
  const size_t plen = prefix ? prefix->tokens.size() : 0;
  for (size_t q = 0; q < S; ++q) {
    const bool use = prefix && lens[q] > plen && std::equal(prefix->tokens.begin(), prefix->tokens.end(), prompts[q]);
    map_slot((int)q, use ? prefix : nullptr);
    start[q] = use ? plen : 0;
  }
  // Prefill: rows of every stream in order, rows_cap_ at a time.
  int* hs = batch_host_;
  int* hp = batch_host_ + rows_cap_;
  int* hi = batch_host_ + 2 * rows_cap_;
  size_t s = 0, p = start[0];
  while (s < S) {
    wait();  // the pinned staging is reused per chunk
    int mc = 0, top = 0;
    std::vector<std::pair<int, int>> ends;  // (chunk row, stream) of each stream's last prompt row
    while (s < S && mc < rows_cap_) {
      hs[mc] = (int)s;
      hp[mc] = (int)p;
      hi[mc] = prompts[s][p];
      top = std::max(top, (int)p + 1);
      if (++p == lens[s]) {
        ends.emplace_back(mc, (int)s);
        ++s;
        p = s < S ? start[s] : 0;
      }
      ++mc;
    }
    TRIT_CUDA(cudaMemcpyAsync(row_stream_, hs, (size_t)mc * 4, cudaMemcpyHostToDevice, stream_));
    TRIT_CUDA(cudaMemcpyAsync(row_pos_, hp, (size_t)mc * 4, cudaMemcpyHostToDevice, stream_));
    TRIT_CUDA(cudaMemcpyAsync(ids_, hi, (size_t)mc * 4, cudaMemcpyHostToDevice, stream_));
    TRIT_CUDA(launch_embed(embed_, ids_, mc, x_, 1.0f, stream_));
    // Runs of consecutive rows of one stream.
    std::vector<std::pair<int, int>> runs;
    for (int r = 0; r < mc;) {
      int e = r + 1;
      while (e < mc && hs[e] == hs[r]) ++e;
      runs.emplace_back(r, e - r);
      r = e;
    }
    hidden(mc, top, &runs);
    timing_.gpu_launches += 1;
    for (auto& e : ends)
      TRIT_CUDA(cudaMemcpyAsync(batch_last_ + (size_t)e.second * d, x_ + (size_t)e.first * d, (size_t)d * 4,
                                cudaMemcpyDeviceToDevice, stream_));
  }
  // The first token of every stream, then the decode state: stream s sits
  // in slot s at position lens[s] with its last token in batch_cur_.
  clock_.report("batch prefill");
  wait();
  for (size_t i = 0; i < S; ++i) {
    hs[i] = (int)i;
    hp[i] = (int)lens[i];
  }
  TRIT_CUDA(cudaMemcpyAsync(row_stream_, hs, S * 4, cudaMemcpyHostToDevice, stream_));
  TRIT_CUDA(cudaMemcpyAsync(row_pos_, hp, S * 4, cudaMemcpyHostToDevice, stream_));
  TRIT_CUDA(cudaMemsetAsync(batch_step_, 0, 4, stream_));
  final_rows(batch_last_, d, (int)S, nullptr, batch_cur_);
  TRIT_CUDA(launch_batch_advance(batch_cur_, row_pos_, batch_step_, batch_tok_, (int)S, 0, stream_));
  timing_.gpu_launches += 4;
  TRIT_CUDA(cudaEventRecord(ev_[1], stream_));
  const int steps = max_new - 1;
  const int tmax = (int)(longest + max_new);
  int per_step = 0;
  auto step = [&]() {
    int before = timing_.gpu_launches;
    TRIT_CUDA(launch_embed(embed_, batch_cur_, (int)S, x_, 1.0f, stream_));
    hidden((int)S, tmax);
    clock_.mark("final norm+table+argmax", stream_);
    final_rows(x_, d, (int)S, nullptr, batch_cur_);
    clock_.mark(nullptr, stream_);
    TRIT_CUDA(launch_batch_advance(batch_cur_, row_pos_, batch_step_, batch_tok_, (int)S, 1, stream_));
    timing_.gpu_launches += 1 + 3 + 1;
    per_step = timing_.gpu_launches - before;
  };
  if (steps > 0) {
    step();  // eagerly once: sets up every kernel's attributes before a capture
    if (steps > 1 && clock_.on) {
      for (int i = 1; i < steps; ++i) step();  // per-kernel clocks: no graph
    } else if (steps > 1) {
      if (!batch_graph_ || batch_graph_streams_ != (int)S || batch_graph_tmax_ < tmax) {
        if (batch_graph_) cudaGraphExecDestroy(batch_graph_);
        batch_graph_ = nullptr;
        int counted = timing_.gpu_launches;
        cudaGraph_t g = nullptr;
        TRIT_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        try {
          step();
        } catch (...) {
          cudaStreamEndCapture(stream_, &g);
          if (g) cudaGraphDestroy(g);
          throw;
        }
        TRIT_CUDA(cudaStreamEndCapture(stream_, &g));
        cudaError_t e = cudaGraphInstantiate(&batch_graph_, g, 0);
        cudaGraphDestroy(g);
        TRIT_CUDA(e);
        timing_.gpu_launches = counted;  // captured, not run
        batch_graph_streams_ = (int)S;
        batch_graph_tmax_ = tmax;
      }
      for (int i = 1; i < steps; ++i) TRIT_CUDA(cudaGraphLaunch(batch_graph_, stream_));
      timing_.gpu_launches += per_step * (steps - 1);
    }
  }
  TRIT_CUDA(cudaEventRecord(ev_[2], stream_));
  clock_.report("generate_batch");
  std::vector<int> toks((size_t)max_new * S);
  TRIT_CUDA(cudaMemcpyAsync(toks.data(), batch_tok_, toks.size() * 4, cudaMemcpyDeviceToHost, stream_));
  wait();
  check_tc_status();
  float ms = 0;
  TRIT_CUDA(cudaEventElapsedTime(&ms, ev_[0], ev_[1]));
  timing_.prefill_ms = ms;
  TRIT_CUDA(cudaEventElapsedTime(&ms, ev_[1], ev_[2]));
  timing_.decode_ms = ms;
  timing_.decode_tokens = steps * (int)S;
  (void)total;
  for (size_t i = 0; i < S; ++i) {
    int64_t n = 0;
    for (int t = 0; t < max_new; ++t) {
      int tok = toks[(size_t)t * S + i];
      bool stopped = false;
      for (size_t k = 0; k < nstop; ++k) stopped |= tok == stop[k];
      if (stopped) break;
      out[i * (size_t)max_new + t] = tok;
      ++n;
    }
    counts[i] = n;
  }
}

// ------------------------------------------------------------ DenseOp ----
DenseOp::~DenseOp() {
  cudaSetDevice(device);
  void* bufs[] = {mem, xq, xs, xdev, ydev, best_val, best_idx, token, tc_status};
  for (void* b : bufs)
    if (b) cudaFree(b);
  if (stream) cudaStreamDestroy(stream);
}

std::unique_ptr<DenseOp> dense_q8_0(const void* blocks, size_t n, size_t k, int device, bool table) {
  if (k % 32) throw Error("Q8_0 rows are whole blocks of 32");
  if (!table && n % 32) throw Error("a W8A8 layer needs a multiple of 32 output rows");
  // The W8A8 products (k_gemv_slots, k_gemm_tc) take rows of whole
  // 128-value chunks; the table product takes any whole blocks.
  if (!table && k % 128) throw Error("a W8A8 layer needs k a multiple of 128");
  auto op = std::make_unique<DenseOp>();
  op->device = device;
  op->table = table;
  TRIT_CUDA(cudaSetDevice(device));
  TRIT_CUDA(cudaStreamCreateWithFlags(&op->stream, cudaStreamNonBlocking));
  size_t nb = n * (k / 32);
  std::vector<uint8_t> codes(n * k), scales(nb * 2);
  const uint8_t* src = (const uint8_t*)blocks;
  for (size_t b = 0; b < nb; ++b) {
    std::memcpy(scales.data() + b * 2, src + b * 34, 2);
    std::memcpy(codes.data() + b * 32, src + b * 34 + 2, 32);
  }
  size_t co = 0, so = (n * k + 255) / 256 * 256;
  TRIT_CUDA(cudaMalloc(&op->mem, so + scales.size()));
  TRIT_CUDA(cudaMemcpy(op->mem, codes.data(), codes.size(), cudaMemcpyHostToDevice));
  TRIT_CUDA(cudaMemcpy((char*)op->mem + so, scales.data(), scales.size(), cudaMemcpyHostToDevice));
  if (table) {
    op->tab.n = (int)n; op->tab.k = (int)k; op->tab.scale_f16 = 1;
    op->tab.codes = (const int8_t*)op->mem + co;
    op->tab.scales = (char*)op->mem + so;
  } else {
    op->mat.kind = kQ8_0; op->mat.n = (int)n; op->mat.k = (int)k; op->mat.agroup = 32; op->mat.half = 1;
    op->mat.codes = (char*)op->mem + co;
    op->mat.scales = (char*)op->mem + so;
    // The tensor-core product (64 rows or more) on sm_100.
    int major = 0;
    TRIT_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    TRIT_CUDA(cudaDeviceGetAttribute(&op->sm_count, cudaDevAttrMultiProcessorCount, device));
    if (major == 10 && k % 128 == 0 && make_tc_weight_map(&op->tc_w, op->mat, op->mat.codes) == cudaSuccess) {
      TRIT_CUDA(cudaMalloc(&op->tc_status, 4));
      TRIT_CUDA(cudaMemset(op->tc_status, 0, 4));
      op->tc_ok = true;
    }
  }
  return op;
}

void DenseOp::forward_device(const float* x, size_t m, float* y, cudaStream_t s) {
  if (m > rows_cap) {
    if (xq) cudaFree(xq);
    if (xs) cudaFree(xs);
    if (best_val) cudaFree(best_val);
    if (best_idx) cudaFree(best_idx);
    if (token) cudaFree(token);
    xq = nullptr; xs = nullptr; best_val = nullptr; best_idx = nullptr; token = nullptr;
    size_t k = table ? tab.k : mat.k;
    size_t n = table ? tab.n : mat.n;
    // Whole 64-row tiles: the tensor-core product reads frames in tiles.
    TRIT_CUDA(cudaMalloc(&xq, (m + 63) / 64 * 64 * k));
    tc_tried = false;  // the frame map names the old buffer
    TRIT_CUDA(cudaMalloc(&xs, m * (k / 32) * 4));
    TRIT_CUDA(cudaMalloc(&best_val, m * table_blocks((int)n) * 4));
    TRIT_CUDA(cudaMalloc(&best_idx, m * table_blocks((int)n) * 4));
    TRIT_CUDA(cudaMalloc(&token, m * 4));
    rows_cap = m;
  }
  if (table) {
    TRIT_CUDA(launch_table(tab, x, (int)m, 1.0f, y, best_val, best_idx, s));
  } else {
    TRIT_CUDA(launch_norm_quant(x, (int)m, mat.k, nullptr, 0.0f, mat.agroup, mat.half, xq, xs, s));
    // The tensor cores from 16 rows, from 4 on matrices of 6144 rows or
    // more, and always from 32768 rows (measured with the op sweep: below
    // that the dp4a GEMV wins).
    const bool use_tc = tc_ok && (m >= 16 || (m >= 4 && mat.n >= 6144) || mat.n >= 32768);
    if (use_tc && !tc_tried) {
      // The frame map of the current activation buffer (made again after
      // the buffer grows).
      tc_tried = true;
      tc_ok = make_tc_frame_map(&tc_x, xq, (rows_cap + 63) / 64 * 64, (size_t)mat.k) == cudaSuccess;
    }
    if (use_tc && tc_ok) TRIT_CUDA(launch_gemm_tc(tc_w, tc_x, mat, xs, (int)m, kEpOut, y, mat.n, 1.0f, tc_status, s));
    else TRIT_CUDA(launch_gemv(mat, xq, xs, (int)m, kEpOut, y, mat.n, 1.0f, s));
  }
}

}  // namespace trit
