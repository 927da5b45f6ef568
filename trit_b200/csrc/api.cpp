// The C ABI of include/trit_cuda.h. Every entry
// point runs its body under `guard`, which turns a C++ exception into the
// thread's error text and the failure value, as ffi/src/lib.rs:20-45 does
// for Rust panics.
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>

#include "../../include/trit_cuda.h"
#include "engine.h"
#include "nccl_link.h"

struct TritLm {
  std::unique_ptr<trit::Lm> lm;
};
struct TritLmPrefix {
  std::unique_ptr<trit::PrefixState> state;
  const TritLm* owner = nullptr;
};
struct TritDense {
  std::unique_ptr<trit::DenseOp> op;
  std::mutex mu;
};

namespace {
thread_local std::string g_error;
}  // namespace

namespace trit {
void set_last_error(const std::string& text) { g_error = text; }
}  // namespace trit

namespace {

template <class T, class F>
T guard(T failed, F body) {
  g_error.clear();
  try {
    return body();
  } catch (const std::exception& e) {
    g_error = e.what();
  } catch (...) {
    g_error = "internal error in trit_cuda";
  }
  return failed;
}

void need(const void* p, const char* what) {
  if (!p) throw trit::Error(std::string(what) + " is NULL");
}

int64_t copy_out(const std::vector<int>& toks, int32_t* out, size_t cap) {
  if (cap && !out) throw trit::Error("out is NULL");
  size_t n = std::min(cap, toks.size());
  for (size_t i = 0; i < n; ++i) out[i] = toks[i];
  return (int64_t)toks.size();
}

}  // namespace

extern "C" {

const char* trit_cuda_version(void) { return "0.1.0"; }

const char* trit_cuda_last_error(void) { return g_error.c_str(); }

char* trit_lm_inspect(const char* model_dir, const char* options_json) {
  return guard<char*>(nullptr, [&]() {
    need(model_dir, "model_dir");
    trit::Options o = trit::Options::parse(options_json, true);
    std::string text = trit::describe_model(model_dir, o.config_at, o.prefix, o.tp_rank, o.tp_size);
    char* out = (char*)std::malloc(text.size() + 1);
    if (!out) throw trit::Error("out of host memory");
    std::memcpy(out, text.c_str(), text.size() + 1);
    return out;
  });
}

void trit_cuda_free_text(char* text) { std::free(text); }

int trit_cuda_tp_id(char* out, size_t cap) {
  return guard<int>(-1, [&]() {
    need(out, "out");
    ncclUniqueId id;
    trit::nccl_check(trit::nccl().GetUniqueId(&id), "unique id");
    if (cap < 2 * sizeof id + 1) throw trit::Error("out holds fewer than 257 bytes");
    static const char hex[] = "0123456789abcdef";
    for (size_t i = 0; i < sizeof id; ++i) {
      out[2 * i] = hex[(uint8_t)id.internal[i] >> 4];
      out[2 * i + 1] = hex[(uint8_t)id.internal[i] & 15];
    }
    out[2 * sizeof id] = '\0';
    return 0;
  });
}

char* trit_lm_status(const TritLm* lm) {
  return guard<char*>(nullptr, [&]() {
    need(lm, "lm");
    std::string text;
    {
      std::lock_guard<std::mutex> lock(const_cast<TritLm*>(lm)->lm->mutex());
      text = lm->lm->status();
    }
    char* out = (char*)std::malloc(text.size() + 1);
    if (!out) throw trit::Error("out of host memory");
    std::memcpy(out, text.c_str(), text.size() + 1);
    return out;
  });
}

TritLm* trit_lm_load(const char* model_dir, const char* options_json) {
  return guard<TritLm*>(nullptr, [&]() {
    need(model_dir, "model_dir");
    trit::Options o = trit::Options::parse(options_json);
    auto h = std::make_unique<TritLm>();
    h->lm = std::make_unique<trit::Lm>(model_dir, o);
    return h.release();
  });
}

void trit_lm_free(TritLm* lm) { delete lm; }

int64_t trit_lm_width(const TritLm* lm) { return lm ? lm->lm->config().d : -1; }
int64_t trit_lm_layers(const TritLm* lm) { return lm ? lm->lm->config().layers : -1; }
int64_t trit_lm_vocab(const TritLm* lm) { return lm ? lm->lm->config().vocab : -1; }

TritLmPrefix* trit_lm_prefix(TritLm* lm, const int32_t* ids, size_t n) {
  return guard<TritLmPrefix*>(nullptr, [&]() {
    need(lm, "lm");
    if (n) need(ids, "ids");
    std::lock_guard<std::mutex> lock(lm->lm->mutex());
    auto p = std::make_unique<TritLmPrefix>();
    p->state = lm->lm->prefix(ids, n);
    p->owner = lm;
    return p.release();
  });
}

void trit_lm_prefix_free(TritLmPrefix* prefix) { delete prefix; }

static int64_t generate_impl(TritLm* lm, const TritLmPrefix* prefix, const int32_t* prompt, size_t n,
                             int32_t max_new, const int32_t* stop, size_t nstop, int32_t* out, size_t cap,
                             float* logits) {
  return guard<int64_t>(-1, [&]() {
    need(lm, "lm");
    need(prompt, "prompt");
    if (nstop) need(stop, "stop");
    if (max_new < 0) throw trit::Error("max_new is negative");
    if (prefix && prefix->owner != lm) throw trit::Error("the prefix belongs to another model");
    std::lock_guard<std::mutex> lock(lm->lm->mutex());
    auto toks = lm->lm->generate(prefix ? prefix->state.get() : nullptr, prompt, n, max_new, stop, nstop, logits);
    return copy_out(toks, out, cap);
  });
}

int64_t trit_lm_generate(TritLm* lm, const TritLmPrefix* prefix, const int32_t* prompt, size_t n, int32_t max_new,
                         const int32_t* stop, size_t nstop, int32_t* out, size_t cap) {
  return generate_impl(lm, prefix, prompt, n, max_new, stop, nstop, out, cap, nullptr);
}

int64_t trit_lm_generate_traced(TritLm* lm, const TritLmPrefix* prefix, const int32_t* prompt, size_t n,
                                int32_t max_new, const int32_t* stop, size_t nstop, int32_t* out, size_t cap,
                                float* logits) {
  if (!logits) {
    g_error = "logits is NULL";
    return -1;
  }
  return generate_impl(lm, prefix, prompt, n, max_new, stop, nstop, out, cap, logits);
}

static int64_t answer_impl(TritLm* lm, const int32_t* head, size_t nhead, const float* audio, size_t naudio,
                           const int32_t* tail, size_t ntail, int32_t max_new, const int32_t* stop, size_t nstop,
                           int32_t* out, size_t cap, float* logits, bool on_device = false,
                           void* cuda_stream = nullptr) {
  return guard<int64_t>(-1, [&]() {
    need(lm, "lm");
    if (nhead) need(head, "head");
    if (naudio) need(audio, "audio");
    if (ntail) need(tail, "tail");
    if (nstop) need(stop, "stop");
    if (max_new < 0) throw trit::Error("max_new is negative");
    std::lock_guard<std::mutex> lock(lm->lm->mutex());
    auto toks = lm->lm->answer(head, nhead, audio, naudio, tail, ntail, max_new, stop, nstop, logits,
                               (cudaStream_t)cuda_stream, on_device);
    return copy_out(toks, out, cap);
  });
}

int64_t trit_lm_generate_rows(TritLm* lm, const float* rows, size_t nrows, int32_t max_new, const int32_t* stop,
                              size_t nstop, int32_t* out, size_t cap) {
  return answer_impl(lm, nullptr, 0, rows, nrows, nullptr, 0, max_new, stop, nstop, out, cap, nullptr);
}

int64_t trit_lm_answer(TritLm* lm, const int32_t* head, size_t nhead, const float* audio, size_t naudio,
                       const int32_t* tail, size_t ntail, int32_t max_new, const int32_t* stop, size_t nstop,
                       int32_t* out, size_t cap) {
  return answer_impl(lm, head, nhead, audio, naudio, tail, ntail, max_new, stop, nstop, out, cap, nullptr);
}

int64_t trit_lm_generate_rows_device(TritLm* lm, const float* rows, size_t nrows, int32_t max_new,
                                     const int32_t* stop, size_t nstop, int32_t* out, size_t cap, void* cuda_stream) {
  return answer_impl(lm, nullptr, 0, rows, nrows, nullptr, 0, max_new, stop, nstop, out, cap, nullptr, true,
                     cuda_stream);
}

int64_t trit_lm_answer_device(TritLm* lm, const int32_t* head, size_t nhead, const float* audio, size_t naudio,
                              const int32_t* tail, size_t ntail, int32_t max_new, const int32_t* stop, size_t nstop,
                              int32_t* out, size_t cap, void* cuda_stream) {
  return answer_impl(lm, head, nhead, audio, naudio, tail, ntail, max_new, stop, nstop, out, cap, nullptr, true,
                     cuda_stream);
}

int64_t trit_lm_answer_traced(TritLm* lm, const int32_t* head, size_t nhead, const float* audio, size_t naudio,
                              const int32_t* tail, size_t ntail, int32_t max_new, const int32_t* stop, size_t nstop,
                              int32_t* out, size_t cap, float* logits) {
  if (!logits) {
    g_error = "logits is NULL";
    return -1;
  }
  return answer_impl(lm, head, nhead, audio, naudio, tail, ntail, max_new, stop, nstop, out, cap, logits);
}

int trit_lm_embed(TritLm* lm, const int32_t* ids, size_t n, float* out) {
  return guard<int>(-1, [&]() {
    need(lm, "lm");
    if (n) {
      need(ids, "ids");
      need(out, "out");
    }
    std::lock_guard<std::mutex> lock(lm->lm->mutex());
    lm->lm->embed(ids, n, out);
    return 0;
  });
}

int trit_lm_set_ffn_scales(TritLm* lm, const float* scales, size_t layers, size_t width) {
  return guard<int>(-1, [&]() {
    need(lm, "lm");
    const trit::DConfig& c = lm->lm->config();
    if (scales && (layers != (size_t)c.layers || width != (size_t)c.d))
      throw trit::Error("ffn scales are " + std::to_string(layers) + " x " + std::to_string(width) + ", the model has " +
                        std::to_string(c.layers) + " layers of width " + std::to_string(c.d));
    std::lock_guard<std::mutex> lock(lm->lm->mutex());
    lm->lm->set_ffn_scales(scales);
    return 0;
  });
}

int64_t trit_lm_generate_additive(TritLm* lm, const int32_t* prompt, size_t n, const float* audio, size_t rows,
                                  const int32_t* stop, size_t nstop, int32_t* out, size_t cap) {
  return guard<int64_t>(-1, [&]() {
    need(lm, "lm");
    if (n) need(prompt, "prompt");
    if (rows) need(audio, "audio");
    if (nstop) need(stop, "stop");
    std::lock_guard<std::mutex> lock(lm->lm->mutex());
    auto toks = lm->lm->generate_additive(prompt, n, audio, rows, stop, nstop, nullptr);
    return copy_out(toks, out, cap);
  });
}

int64_t trit_lm_bidirectional_tokens(TritLm* lm, const float* rows, size_t m, size_t from, int32_t* out) {
  return guard<int64_t>(-1, [&]() {
    need(lm, "lm");
    if (m) need(rows, "rows");
    if (m > from) need(out, "out");
    std::lock_guard<std::mutex> lock(lm->lm->mutex());
    auto toks = lm->lm->bidirectional_tokens(rows, m, from);
    for (size_t i = 0; i < toks.size(); ++i) out[i] = toks[i];
    return (int64_t)toks.size();
  });
}

static int batch_impl(TritLm* lm, const TritLmPrefix* prefix, size_t streams, const int32_t* const* prompts,
                      const size_t* lens, int32_t max_new, const int32_t* stop, size_t nstop, int32_t* out,
                      int64_t* counts) {
  return guard<int>(-1, [&]() {
    need(lm, "lm");
    need(prompts, "prompts");
    need(lens, "lens");
    need(out, "out");
    need(counts, "counts");
    if (nstop) need(stop, "stop");
    if (max_new < 0) throw trit::Error("max_new is negative");
    if (prefix && prefix->owner != lm) throw trit::Error("the prefix belongs to another model");
    std::lock_guard<std::mutex> lock(lm->lm->mutex());
    lm->lm->generate_batch(streams, prompts, lens, max_new, stop, nstop, out, counts,
                           prefix ? prefix->state.get() : nullptr);
    return 0;
  });
}

int trit_lm_generate_batch(TritLm* lm, size_t streams, const int32_t* const* prompts, const size_t* lens,
                           int32_t max_new, const int32_t* stop, size_t nstop, int32_t* out, int64_t* counts) {
  return batch_impl(lm, nullptr, streams, prompts, lens, max_new, stop, nstop, out, counts);
}

int trit_lm_generate_batch_prefix(TritLm* lm, const TritLmPrefix* prefix, size_t streams,
                                  const int32_t* const* prompts, const size_t* lens, int32_t max_new,
                                  const int32_t* stop, size_t nstop, int32_t* out, int64_t* counts) {
  return batch_impl(lm, prefix, streams, prompts, lens, max_new, stop, nstop, out, counts);
}

int trit_lm_prefix_pages(const TritLm* lm, int64_t* used, int64_t* total) {
  return guard<int>(-1, [&]() {
    need(lm, "lm");
    need(used, "used");
    need(total, "total");
    std::lock_guard<std::mutex> lock(const_cast<TritLm*>(lm)->lm->mutex());
    *used = lm->lm->prefix_pages_used();
    *total = lm->lm->prefix_pages_total();
    return 0;
  });
}

int trit_lm_last_timing(const TritLm* lm, double* prefill_ms, double* decode_ms, int64_t* decode_steps,
                        int64_t* launches) {
  return guard<int>(-1, [&]() {
    need(lm, "lm");
    const trit::Timing& t = lm->lm->timing();
    if (prefill_ms) *prefill_ms = t.prefill_ms;
    if (decode_ms) *decode_ms = t.decode_ms;
    if (decode_steps) *decode_steps = t.decode_tokens;
    if (launches) *launches = t.gpu_launches;
    return 0;
  });
}

TritDense* trit_dense_q8_0(const void* blocks, size_t n, size_t k, int table, int device) {
  return guard<TritDense*>(nullptr, [&]() {
    need(blocks, "blocks");
    auto h = std::make_unique<TritDense>();
    h->op = trit::dense_q8_0(blocks, n, k, device, table != 0);
    return h.release();
  });
}

int trit_dense_forward(TritDense* layer, const float* x, size_t rows, float* out) {
  return guard<int>(-1, [&]() {
    need(layer, "layer");
    need(x, "x");
    need(out, "out");
    std::lock_guard<std::mutex> lock(layer->mu);
    trit::DenseOp& op = *layer->op;
    TRIT_CUDA(cudaSetDevice(op.device));
    size_t k = op.table ? op.tab.k : op.mat.k, n = op.table ? op.tab.n : op.mat.n;
    float *dx = nullptr, *dy = nullptr;
    TRIT_CUDA(cudaMallocAsync(&dx, rows * k * 4, op.stream));
    TRIT_CUDA(cudaMallocAsync(&dy, rows * n * 4, op.stream));
    TRIT_CUDA(cudaMemcpyAsync(dx, x, rows * k * 4, cudaMemcpyHostToDevice, op.stream));
    op.forward_device(dx, rows, dy, op.stream);
    TRIT_CUDA(cudaMemcpyAsync(out, dy, rows * n * 4, cudaMemcpyDeviceToHost, op.stream));
    TRIT_CUDA(cudaFreeAsync(dx, op.stream));
    TRIT_CUDA(cudaFreeAsync(dy, op.stream));
    TRIT_CUDA(cudaStreamSynchronize(op.stream));
    if (op.tc_status) {  // did a wait in a tensor-core product run out?
      int st = 0;
      TRIT_CUDA(cudaMemcpyAsync(&st, op.tc_status, 4, cudaMemcpyDeviceToHost, op.stream));
      TRIT_CUDA(cudaStreamSynchronize(op.stream));
      if (st) throw trit::Error("the tensor-core product gave up waiting for its pipeline");
    }
    return 0;
  });
}

int trit_dense_forward_device(TritDense* layer, const float* x, size_t rows, float* out, void* cuda_stream) {
  return guard<int>(-1, [&]() {
    need(layer, "layer");
    need(x, "x");
    need(out, "out");
    std::lock_guard<std::mutex> lock(layer->mu);
    trit::DenseOp& op = *layer->op;
    TRIT_CUDA(cudaSetDevice(op.device));
    op.forward_device(x, rows, out, cuda_stream ? (cudaStream_t)cuda_stream : op.stream);
    return 0;
  });
}

void trit_dense_free(TritDense* layer) { delete layer; }

}  // extern "C"
