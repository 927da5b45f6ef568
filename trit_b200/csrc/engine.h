// The decoder engine behind the C ABI: one model on one GPU, its paged KV
// cache, and the generation flows of CausalLm
// (src/models/parts/causal_lm.rs:200-345).
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "host.h"
#include "kernels.h"

namespace trit {

struct Options {
  int device = 0;
  bool kv_f16 = true;            // the paged KV cache in f16 (f32: the reference's cache)
  int max_context = 4096;        // positions per stream
  int max_streams = 1;           // stream slots for generate_batch
  int page_tokens = 64;          // positions per KV page
  int prefill_rows = 512;        // rows per prefill pass
  int prefix_pages = -1;         // KV pages kept for prefixes (-1: one stream's worth)
  std::string decode = "persistent";  // "persistent" (one kernel per generation) or "layered"
  bool tensor_cores = true;      // tcgen05 products for prefill and batches of >= tc_rows rows
  int tc_rows = 64;
  // The f16 form of the Q8_0 tensor-core products (codes as f16, exact f32
  // dots, a fold without the integer bias); costs an f16 copy of the Q8_0
  // layers' codes. Measured slower on C5 (two 32-value groups a stage
  // instead of four: twice the stages and hand-offs), so off by default.
  bool tc_f16 = false;
  // true (default): every floating-point step in the reference's order
  // (logits bit for bit those of the CPU decoder). false: the batch-1
  // decode sums in tree order (decode_fast.cu); tokens stay the reference's
  // but, since a reordered sum can move an int8 activation code, logits
  // drift by up to ~5e-2.
  bool exact = true;
  // Prompt attention as f16 flash attention on the tensor cores (not the
  // reference's arithmetic; needs exact false, an f16 cache and pages of a
  // multiple of 64 positions).
  bool tc_attention = false;
  // Keep the weights' device layout in a cache file and read it on later
  // loads (cache_dir, default <model folder>/.trit_cuda).
  bool weight_cache = false;
  std::string cache_dir;
  // Tensor parallelism: this process's rank of tp_size, and the NCCL
  // unique id (hex, from trit_cuda_tp_id on rank 0) the ranks share.
  int tp_size = 1, tp_rank = 0;
  std::string tp_id;
  // Seconds a rank waits for the others (joining the group, or a step whose
  // collectives they must answer) before the communicator is aborted and
  // the call fails: a rank that failed or left ends the others' calls with
  // an error instead of a hang.
  double tp_timeout_s = 120.0;
  std::string config_at;         // key path of the settings in config.json (from_tensors' config_at)
  std::string prefix;            // start of every tensor name (from_tensors' prefix)
  // `lenient`: keys other than config_at and prefix are skipped unchecked.
  static Options parse(const char* json, bool lenient = false);
};

struct CudaCheck {
  static void ok(cudaError_t e, const char* what);
};
#define TRIT_CUDA(x) ::trit::CudaCheck::ok((x), #x)

class Lm;

// A prompt start that many calls share (Prefix, causal_lm.rs:118-122,
// 202-215): its tokens, the physical KV pages that hold its full pages
// (read-only once made; a stream's page table points at them), and a device
// copy of the page after them when the prefix ends inside a page (copied
// into the stream's own page on use, since the stream appends there).
struct PrefixState {
  std::vector<int> tokens;
  std::vector<int> pages;
  void* partial = nullptr;
  Lm* owner = nullptr;  // gets the pages back; null once the model is gone
  ~PrefixState();
};

struct Timing {
  double prefill_ms = 0, decode_ms = 0;
  int decode_tokens = 0;
  int gpu_launches = 0;
};

// Device time per step kind (TRIT_KERNEL_CLOCK=1), a measurement aid.
struct KernelClock {
  bool on = false;
  std::vector<cudaEvent_t> pool;
  std::vector<const char*> names;  // the step that starts at each mark (null: none)
  size_t used = 0;
  KernelClock();
  ~KernelClock();
  void mark(const char* name, cudaStream_t s);
  void report(const char* what);
};

class Lm {
 public:
  Lm(const std::string& dir, const Options& o);
  ~Lm();
  Lm(const Lm&) = delete;
  Lm& operator=(const Lm&) = delete;

  const DConfig& config() const { return cfg_; }
  const Options& options() const { return opt_; }
  std::mutex& mutex() { return mu_; }
  const Timing& timing() const { return timing_; }
  // What the load did, as JSON text (trit_lm_status).
  std::string status() const;

  // CausalLm::generate with an optional prefix; `logits` (host, may be
  // null) receives the logits of every kept or stopping token, [max_new][vocab].
  std::vector<int> generate(const PrefixState* prefix, const int* ids, size_t n, int max_new, const int* stop,
                            size_t nstop, float* logits);
  // CausalLm::generate_rows: the prompt as embeddings [nrows][d].
  std::vector<int> generate_rows(const float* rows, size_t nrows, int max_new, const int* stop, size_t nstop,
                                 float* logits);
  // CausalLm::answer: head ids, audio rows, tail ids. `audio_stream`
  // non-null: the rows are device memory of this model's GPU, written by
  // work queued on that stream (the rows never pass through the host).
  std::vector<int> answer(const int* head, size_t nhead, const float* audio, size_t naudio, const int* tail,
                          size_t ntail, int max_new, const int* stop, size_t nstop, float* logits,
                          cudaStream_t audio_stream = nullptr, bool audio_on_device = false);
  void embed(const int* ids, size_t n, float* out);
  std::unique_ptr<PrefixState> prefix(const int* ids, size_t n);
  // CausalLm::set_ffn_scales: [layers][d] host floats, or null to clear.
  void set_ffn_scales(const float* scales);
  // CausalLm::generate_additive: prompt ids plus audio rows [rows][d].
  std::vector<int> generate_additive(const int* ids, size_t n, const float* audio, size_t rows, const int* stop,
                                     size_t nstop, float* logits);
  // CausalLm::bidirectional_tokens: rows [m][d] without the causal mask.
  std::vector<int> bidirectional_tokens(const float* rows, size_t m, size_t from);
  // Independent streams, each with its own prompt: out [streams][max_new].
  // A stream whose prompt starts with `prefix` (and is longer) reads the
  // prefix's pages instead of recomputing them.
  void generate_batch(size_t streams, const int* const* prompts, const size_t* lens, int max_new, const int* stop,
                      size_t nstop, int* out, int64_t* counts, const PrefixState* prefix = nullptr);
  // Prefix pages in use and in all.
  int prefix_pages_used() const { return prefix_pages_total_ - (int)prefix_free_.size(); }
  int prefix_pages_total() const { return prefix_pages_total_; }
  // A prefix goes: its pages return to the free list (under mutex()).
  void release_prefix(PrefixState* p);

 private:
  void load(const std::string& dir);
  std::string weight_cache_identity(const ModelSource& src) const;
  std::string weight_cache_path(const std::string& dir, const ModelSource& src) const;
  bool read_weight_cache(const std::string& path, void* arena, size_t bytes, cudaStream_t s);
  void write_weight_cache(const std::string& path, const void* arena, size_t bytes, cudaStream_t s);
  void release();
  void alloc_buffers();
  // Points the page table row of `slot` at its own pages, or, with a
  // prefix, its first pages at the prefix's pages (and copies the prefix's
  // partial page into the slot's own page).
  void map_slot(int slot, const PrefixState* prefix);
  void check_ids(const int* ids, size_t n) const;
  // Runs rows x (device, [m][d]) through every layer at positions
  // first.. of stream `slot`; chunks of prefill_rows.
  void run_prompt(size_t m, int slot, int first, const std::function<void(size_t, size_t)>& fill);
  void embed_rows(const int* staged, size_t c0, size_t c1, float* x);
  int* stage_ids(const int* a, size_t na, const int* b, size_t nb);
  // `tiles`: {first row, rows} runs of one stream at consecutive positions
  // (prompt chunks), or null for one row per attention block.
  // `runs`: prompt rows as runs of consecutive positions of one stream
  // (first row, rows), cut into attention tiles here; null for decode rows.
  void hidden(int m, int max_tk, const std::vector<std::pair<int, int>>* runs = nullptr);
  void setup_tensor_cores();
  // The final norm, the output table and the best token of nb rows at x
  // (row stride ldx) into tokens; with tensor parallelism the ranks' best
  // tokens meet in one all-reduce. logits (device, [nb][vocab]) may be null.
  void final_rows(const float* x, int ldx, int nb, float* logits, int* tokens);
  // x[m][d] += the sum over ranks of part_[m][d].
  void reduce_into_x(int m);
  void check_tc_status();
  // Greedy decode for `slot` after a prefill that left its last row in x.
  std::vector<int> finish(int slot, int position, int max_new, const int* stop, size_t nstop, float* logits);
  void decode_layered(int slot, int position, int steps, float* trace);
  void decode_persistent(int slot, int position, int steps, float* trace);

  Options opt_;
  DConfig cfg_{};
  std::mutex mu_;
  Timing timing_;
  cudaStream_t stream_ = nullptr;
  cudaEvent_t ev_[4] = {};
  cudaEvent_t ev_rows_ = nullptr;  // the caller's device rows are written (answer on device rows)

  // weights
  std::string source_;          // the files' form (open_model)
  std::string weights_from_;    // "files" or "cache"
  std::string cache_file_;      // the weight cache file, or ""
  std::string cache_identity_;
  TpShard tp_;                  // this rank's shard (size 1: the whole model)
  void* comm_ = nullptr;        // ncclComm_t of the tensor-parallel ranks
  bool tp_lost_ = false;        // the communicator was aborted: the handle is unusable
  // Waits for stream_; with tensor parallelism a bounded wait that aborts
  // the communicator when the other ranks do not answer.
  void wait();
  float* part_ = nullptr;       // [rows][d] a rank's partial o / down sums
  unsigned long long* keys_ = nullptr;  // [rows] (value, index) keys of each row's best token
  void* arena_ = nullptr;
  size_t arena_bytes_ = 0;
  std::vector<DLayer> layers_;
  DLayer* d_layers_ = nullptr;
  const float* final_norm_ = nullptr;
  DTable embed_{}, head_{};
  bool tied_ = true;
  float* rope_ = nullptr;

  // cache
  DCache cache_{};
  void* pool_ = nullptr;
  size_t page_bytes_ = 0;
  int* page_table_ = nullptr;
  std::vector<int> table_host_;       // the page table as the device holds it
  std::vector<int> prefix_free_;      // free physical pages kept for prefixes
  int prefix_pages_total_ = 0;
  std::set<PrefixState*> prefixes_;   // live prefixes, detached when the model goes

  // scratch
  int rows_cap_ = 0;
  float *x_ = nullptr, *qkv_ = nullptr, *att_ = nullptr, *h_ = nullptr, *xn_ = nullptr;
  int8_t* xq_ = nullptr;
  float* xs_ = nullptr;
  int *row_stream_ = nullptr, *row_pos_ = nullptr, *ids_ = nullptr;
  float* best_val_ = nullptr;
  int* best_idx_ = nullptr;
  int* tokens_ = nullptr;       // device [(max_new + 1) * max_streams]
  int tokens_cap_ = 0;
  float* logits_ = nullptr;     // device [vocab] trace buffer (one step)
  int* stop_ = nullptr;
  int nstop_ = 0;
  int* host_rows_ = nullptr;    // pinned staging: [rows] streams, [rows] positions, [max_context] ids
  int* positions_ = nullptr;    // device positions of every decode step
  int last_rows_ = 0;           // rows of the last prompt chunk (in x_)
  // persistent decode scratch
  unsigned long long* dll_ = nullptr;
  size_t ll_words_ = 0;
  int* dstatus_ = nullptr;
  int* dcount_ = nullptr;
  int decode_grid_ = 0;
  float* trace_ = nullptr;      // device [max_new][vocab] for traced persistent decode
  size_t trace_cap_ = 0;
  // batched decode state
  bool batch_ready_ = false;
  int* batch_host_ = nullptr;   // pinned [3][rows_cap_]: streams, positions, ids of a prefill chunk
  float* batch_last_ = nullptr; // device [max_streams][d]: each stream's last prompt row
  int* batch_cur_ = nullptr;    // device [max_streams]: each stream's latest token
  int* batch_step_ = nullptr;   // device step counter
  int* batch_tok_ = nullptr;    // device [max_new][streams]
  size_t batch_tok_cap_ = 0;
  cudaGraphExec_t batch_graph_ = nullptr;  // one captured greedy step
  int batch_graph_streams_ = 0, batch_graph_tmax_ = 0;
  // tensor-core products
  bool tc_ready_ = false;
  std::vector<TcMap> tc_w_;     // [layer][qkv, out, gate_up, down]
  TcMap tc_x_[3] = {};          // quantized frames of width d, heads * hd, ffn
  TcMap kv_map_{};              // the KV pool for the tensor-core prompt attention
  std::vector<TcMap> tc_w16_;   // f16 codes of the Q8_0 layers, [layer][qkv, out, gate_up, down]
  TcMap tc_x16_[3] = {};        // the frames' codes as f16, widths d, heads * hd, ffn
  void* tc_w16_buf_ = nullptr;
  void* xq16_ = nullptr;
  bool tc_f16_ = false;
  bool attention_tc_ = false;   // "exact": false prompt attention on the tensor cores
  size_t pool_pages_ = 0;
  int8_t* tc_expanded_ = nullptr;  // int8 codes of ternary layers
  float* gu_ = nullptr;         // [rows][2 ffn] gate|up products before silu * up
  int* tc_status_ = nullptr;
  bool causal_ = true;
  KernelClock clock_;
  int* tiles_pinned_ = nullptr;  // pinned [rows_cap][2]
  int* tiles_dev_ = nullptr;     // device copy of the tiles of a prompt chunk          // false: attention sees every key (bidirectional_tokens)
  float* ffn_scales_ = nullptr; // device [layers][d]
  float* audio_ = nullptr;      // device rows of generate_additive
  size_t audio_cap_ = 0;
};

// A lone product layer for the op sweep (Dense::forward, gemm.rs:500-542).
struct DenseOp {
  int device = 0;
  bool table = false;
  DMat mat{};
  DTable tab{};
  void* mem = nullptr;
  int8_t* xq = nullptr;
  float *xs = nullptr, *xdev = nullptr, *ydev = nullptr, *best_val = nullptr;
  int* best_idx = nullptr;
  int* token = nullptr;
  size_t rows_cap = 0;
  cudaStream_t stream = nullptr;
  // The tensor-core product for 64 rows or more (sm_100 only).
  bool tc_tried = false, tc_ok = false;
  int sm_count = 148;
  TcMap tc_w{}, tc_x{};
  int* tc_status = nullptr;
  ~DenseOp();
  void forward_device(const float* x, size_t m, float* y, cudaStream_t s);
};

std::unique_ptr<DenseOp> dense_q8_0(const void* blocks, size_t n, size_t k, int device, bool table);

// The text trit_cuda_last_error() returns on this thread ("" clears it).
void set_last_error(const std::string& text);

}  // namespace trit
