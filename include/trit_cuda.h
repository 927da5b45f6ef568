/* trit_cuda: the greedy token loop of Trit's decoder language model
 * (CausalLm: Qwen3 / Llama / Mistral / Granite) on NVIDIA B200 (sm_100a).
 * C ABI of libtrit_cuda.so.
 *
 * It replaces the CPU decoder behind src/models/parts/causal_lm.rs of
 * Hi9841/trit; the entry points follow that interface (each cites the
 * function it stands for) and the rules of include/trit.h:7-18:
 * - Strings are UTF-8 and NUL-terminated.
 * - A call that fails returns NULL or -1; trit_cuda_last_error() then gives
 *   the reason, for the calling thread. No C++ exception crosses the ABI.
 * - Every exported name starts with trit_cuda_, trit_lm_ or trit_dense_, so
 *   the library can share a process with the reference's own libtrit,
 *   whose trit_last_error and trit_free_text (ffi/src/lib.rs:186,641) keep
 *   their meaning; nothing else is exported.
 * - One model handle may be used from several threads; calls on it take
 *   turns (a mutex), as calls on one Trit engine share one worker team.
 *   Do not free a handle while another thread is in a call on it.
 * - The caller owns every buffer it passes, for the length of the call;
 *   the library owns the device memory of a handle until trit_lm_free.
 * - There is no CPU fallback: without a usable GPU the load fails.
 *
 * A model is a folder in one of three forms (src/models/gguf/mod.rs,
 * src/cpu/tensors.rs):
 * - config.json (Hugging Face keys, as Config::parse reads them,
 *   causal_lm.rs:41-77) and model.gguf with the tensors under their
 *   Hugging Face names;
 * - config.json and safetensors files (model.safetensors, the shards of
 *   model.safetensors.index.json, or every *.safetensors);
 * - one GGUF file as transcribe.cpp writes it (no config.json): the decoder
 *   settings come from its stt.<arch>.decoder.* metadata and its dec.*
 *   tensor names are mapped as the reference maps them (architectures
 *   qwen3_asr, moss, funasr_nano, canary_qwen, voxtral, voxtral_realtime,
 *   granite_speech; src/models/gguf/qwen3_asr.rs:103-136).
 * Products are Q8_0 (ggml blocks of 32 codes and an f16 scale), float (F32,
 * F16, BF16: quantized to Q8_0 at load as ggml quantizes, gemm.rs:53-76),
 * per-row int8 (`.weight` I8 + `.scales` F32 per row), or ternary
 * (`.qweight`, five base-3 codes a byte, + `.scales` F32 per 128 inputs, as
 * src/models/parts/fastconformer.rs:440-452 reads them); norms F32/F16/BF16;
 * token tables Q8_0, float (quantized to Q8_0) or int8 with per-32 F32
 * scales.
 */
#ifndef TRIT_CUDA_H
#define TRIT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct TritLm TritLm;
typedef struct TritLmPrefix TritLmPrefix;
typedef struct TritDense TritDense;

/* A tensor-parallel group's id (NCCL's unique id as 256 hex characters
 * and a NUL, into out of cap >= 257 bytes), made once on one rank and
 * passed to every rank's trit_lm_load as "tp_id". Returns 0, or -1. No
 * counterpart in the reference, which runs on one CPU. */
int trit_cuda_tp_id(char *out, size_t cap);

/* The library version, for example "0.1.0". Static; do not free.
 * (trit_version, include/trit.h:41.) */
const char *trit_cuda_version(void);

/* The error of the last failed call on this thread, or "" after a success.
 * Valid until the next call on this thread; do not free.
 * (trit_last_error, include/trit.h:44-46; ffi/src/lib.rs:20-45,186.) */
const char *trit_cuda_last_error(void);

/* A model folder described without a GPU, as JSON text: its settings as
 * Config::parse reads them (causal_lm.rs:41-77: q/k norms iff model_type
 * is "qwen3", head_dim defaulting to hidden / heads, eps 1e-6, rope_theta
 * 1e6, the Granite multipliers, tie_word_embeddings), the storage of its
 * products and token tables, and the bytes a greedy step reads from device
 * memory for the products and the output table. `options_json` takes the
 * "config_at" and "prefix" keys of trit_lm_load (others are ignored).
 * Free the text with trit_cuda_free_text. NULL on failure. */
char *trit_lm_inspect(const char *model_dir, const char *options_json);

/* Frees text returned by this library (and only by it: the reference's
 * trit_free_text frees with its own allocator). NULL is a no-op.
 * (trit_free_text, include/trit.h:11; ffi/src/lib.rs:641.) */
void trit_cuda_free_text(char *text);

/* Loads a decoder onto a GPU. `options_json` is NULL, "" or an object;
 * every key is optional and an unknown key fails (as trit_load_json,
 * include/trit.h:76-87):
 *   "device":       CUDA device index (0)
 *   "kv":           "f16" (default) or "f32": the element type of the paged
 *                   KV cache; "f32" holds what the reference holds
 *   "max_context":  positions per stream (4096)
 *   "max_streams":  stream slots for trit_lm_generate_batch (1)
 *   "page_tokens":  positions per KV page (64)
 *   "prefill_rows": prompt rows per prefill pass (512)
 *   "prefix_pages": KV pages kept for trit_lm_prefix (max_context /
 *                   page_tokens: one stream's worth)
 *   "decode":       "persistent" (default: one kernel runs every greedy
 *                   step of a batch-1 generation) or "layered" (a kernel
 *                   per operation and step)
 *   "tensor_cores": true (default on sm_100) or false: products of
 *                   "tc_rows" rows or more on the tensor cores
 *   "tc_rows":      rows from which a product uses the tensor cores (64)
 *   "tc_f16":       false (default) or true: Q8_0 products on the tensor
 *                   cores take their codes as f16 (exact; the MMA makes the
 *                   group dots as exact f32), at the cost of an f16 copy of
 *                   the Q8_0 layers' codes (2 bytes a weight); measured
 *                   slower than the int8 MMA on C5 (5045 against 5268 tok/s)
 *   "tp_size", "tp_rank", "tp_id": tensor parallelism over tp_size ranks,
 *                   one process (or thread) and GPU each: every rank loads
 *                   with the same tp_id (trit_cuda_tp_id's text, made once
 *                   on one rank and shared) and its own tp_rank, and then
 *                   makes the same calls; a rank holds its query heads
 *                   with their key/value heads, its FFN units and its rows
 *                   of the output table, and the ranks sum the o_proj and
 *                   down_proj partials and take the best token of their
 *                   output rows through NCCL (all-reduce). Greedy steps run
 *                   the layered kernels; logit traces, generate_additive
 *                   and bidirectional_tokens are not available
 *   "tp_timeout_s": seconds a rank waits for the others (joining, or a call
 *                   whose collectives they must answer) before it aborts
 *                   the communicator and the call fails (120); the handle
 *                   is unusable afterwards
 *   "weight_cache": false (default) or true: keep the weights' device
 *                   layout in a file (in "cache_dir", default
 *                   <model_dir>/.trit_cuda) on the first load and read it
 *                   straight into device memory on later loads, with no
 *                   parsing or conversion; a file that does not match the
 *                   model's files byte for byte is rewritten, and one that
 *                   cannot be written is skipped (as src/cpu/store.rs:1-16)
 *   "cache_dir":    the folder of the weight cache
 *   "exact":        true (default) or false. true: every floating-point
 *                   step in the order of the reference's CPU decoder, so
 *                   logits equal its logits bit for bit. false: the batch-1
 *                   decode sums in tree order and splits attention and
 *                   o_proj by kv head; the int8 activation codes can then
 *                   move where a value sits on a rounding boundary, so
 *                   logits drift (measured up to 5e-2 max-abs, cosine
 *                   >= 0.9999; the reference restatement with only its
 *                   RmsNorm sum reordered drifts as much) while tokens
 *                   stayed the reference's on every tested config
 *   "tc_attention": false (default) or true (with "exact": false): prompt
 *                   attention as f16 flash attention on the tensor cores
 *                   (f16 cache, pages of a multiple of 64 positions); its
 *                   sums are not the reference's, so logits drift and a
 *                   token can differ where the reference's top two logits
 *                   are close
 *   "config_at":    key path of the decoder settings in config.json ("";
 *                   "thinker_config.text_config." in Qwen3-ASR)
 *   "prefix":       start of every tensor name ("", "thinker.", "llm.")
 * NULL on failure. (CausalLm::load / from_tensors, causal_lm.rs:124-198.) */
TritLm *trit_lm_load(const char *model_dir, const char *options_json);

/* Frees a model and its device memory. NULL is a no-op. (trit_free,
 * include/trit.h:115-116.) */
void trit_lm_free(TritLm *lm);

/* What a load did, as JSON text: "source" (the files' form: "gguf",
 * "gguf-transcribe" or "safetensors"), "weights_from" ("files", or "cache"
 * when the weight cache supplied the device layout), "weight_cache" (its
 * file, or null), "arena_bytes", the KV and decode settings and the
 * prefix pages in use. Free with trit_cuda_free_text. NULL on failure. */
char *trit_lm_status(const TritLm *lm);

/* hidden_size, num_hidden_layers, vocab_size; -1 for NULL.
 * (CausalLm::width / layers, causal_lm.rs:307-313,343-345.) */
int64_t trit_lm_width(const TritLm *lm);
int64_t trit_lm_layers(const TritLm *lm);
int64_t trit_lm_vocab(const TritLm *lm);

/* Runs a prompt start that many calls share (a system prompt) once; a
 * trit_lm_generate or trit_lm_generate_batch_prefix stream whose prompt
 * begins with it and is longer starts from its cache. The prefix's full KV
 * pages are kept read-only in pages the model holds for prefixes (load
 * option "prefix_pages") and every call reads them in place (the page
 * tables of its streams point at them); only the page the prefix ends
 * inside is copied, once per stream and call. NULL on failure (also when
 * the kept pages are used up). (CausalLm::prefix, causal_lm.rs:200-215.) */
TritLmPrefix *trit_lm_prefix(TritLm *lm, const int32_t *ids, size_t n);

/* Frees a prefix and returns its pages. NULL is a no-op. Not while a call
 * on its model uses it. */
void trit_lm_prefix_free(TritLmPrefix *prefix);

/* The KV pages kept for prefixes: in use (by live prefixes) and in all.
 * Returns 0, or -1. */
int trit_lm_prefix_pages(const TritLm *lm, int64_t *used, int64_t *total);

/* Greedy tokens after `prompt` (n ids), until a token of `stop` (nstop ids,
 * not kept) or `max_new` tokens; writes at most `cap` of them to `out`.
 * Returns the number of tokens made, or -1. `prefix` may be NULL.
 * (CausalLm::generate + greedy, causal_lm.rs:217-249,284-302.) */
int64_t trit_lm_generate(TritLm *lm, const TritLmPrefix *prefix, const int32_t *prompt, size_t n,
                         int32_t max_new, const int32_t *stop, size_t nstop, int32_t *out, size_t cap);

/* Greedy tokens after a prompt given as embeddings, `nrows` rows of
 * trit_lm_width() floats (some rows from another model, such as audio
 * frames). Returns the count, or -1. (CausalLm::generate_rows,
 * causal_lm.rs:251-262.) */
int64_t trit_lm_generate_rows(TritLm *lm, const float *rows, size_t nrows, int32_t max_new,
                              const int32_t *stop, size_t nstop, int32_t *out, size_t cap);

/* generate_rows after the prompt `head` (ids), the rows `audio` (naudio
 * rows of trit_lm_width() floats) and the prompt `tail` (ids). Returns the
 * count, or -1. (CausalLm::answer, causal_lm.rs:264-282.) */
int64_t trit_lm_answer(TritLm *lm, const int32_t *head, size_t nhead, const float *audio, size_t naudio,
                       const int32_t *tail, size_t ntail, int32_t max_new, const int32_t *stop,
                       size_t nstop, int32_t *out, size_t cap);

/* trit_lm_generate_rows and trit_lm_answer with the rows in device memory
 * of the model's GPU (an encoder's output that stays on the GPU: no copy
 * through the host). The rows are read after the work queued so far on
 * `cuda_stream` (a cudaStream_t; NULL: the legacy default stream), as
 * device-to-device copies; the call returns when the tokens are on the
 * host, so the caller may reuse the rows' memory then. Fails when the
 * pointer is not device memory of that GPU. Returns the count, or -1.
 * (CausalLm::generate_rows / answer, causal_lm.rs:251-282, fed by
 * Qwen3Asr's encoder rows, src/models/families/qwen3_asr.rs:321-372.) */
int64_t trit_lm_generate_rows_device(TritLm *lm, const float *rows_device, size_t nrows, int32_t max_new,
                                     const int32_t *stop, size_t nstop, int32_t *out, size_t cap,
                                     void *cuda_stream);
int64_t trit_lm_answer_device(TritLm *lm, const int32_t *head, size_t nhead, const float *audio_device,
                              size_t naudio, const int32_t *tail, size_t ntail, int32_t max_new,
                              const int32_t *stop, size_t nstop, int32_t *out, size_t cap, void *cuda_stream);

/* The embeddings of `n` ids, n x trit_lm_width() floats, into `out`.
 * Returns 0, or -1. (CausalLm::embed, causal_lm.rs:347-355.) */
int trit_lm_embed(TritLm *lm, const int32_t *ids, size_t n, float *out);

/* trit_lm_generate with the logits each token came from: `logits` holds
 * max_new x trit_lm_vocab() floats; row i is written for every token made
 * and for a stopping token. For parity checks; slower than
 * trit_lm_generate. (The logits of forward_rows, causal_lm.rs:366-389.) */
int64_t trit_lm_generate_traced(TritLm *lm, const TritLmPrefix *prefix, const int32_t *prompt, size_t n,
                                int32_t max_new, const int32_t *stop, size_t nstop, int32_t *out,
                                size_t cap, float *logits);

/* trit_lm_answer with the logits trace of trit_lm_generate_traced. */
int64_t trit_lm_answer_traced(TritLm *lm, const int32_t *head, size_t nhead, const float *audio,
                              size_t naudio, const int32_t *tail, size_t ntail, int32_t max_new,
                              const int32_t *stop, size_t nstop, int32_t *out, size_t cap,
                              float *logits);

/* Independent greedy generations, one per stream (at most "max_streams"),
 * decoded side by side: stream s starts from prompts[s] (lens[s] ids) and
 * writes its tokens to out[s * max_new ...] and their count to counts[s].
 * Returns 0, or -1. (CausalLm::generate for each stream; the streams share
 * the weights, as the reference's callers share one model.) */
int trit_lm_generate_batch(TritLm *lm, size_t streams, const int32_t *const *prompts, const size_t *lens,
                           int32_t max_new, const int32_t *stop, size_t nstop, int32_t *out,
                           int64_t *counts);

/* trit_lm_generate_batch where the streams whose prompt begins with
 * `prefix` (and is longer) read its pages and run only the rest of their
 * prompt, as S1-mini's cleanup calls share one system prompt
 * (src/cleanup.rs:208,297-299). `prefix` may be NULL. Returns 0, or -1. */
int trit_lm_generate_batch_prefix(TritLm *lm, const TritLmPrefix *prefix, size_t streams,
                                  const int32_t *const *prompts, const size_t *lens, int32_t max_new,
                                  const int32_t *stop, size_t nstop, int32_t *out, int64_t *counts);

/* CausalLm::set_ffn_scales (causal_lm.rs:305-307): the normed MLP input of
 * layer l is multiplied by scales[l * width ...] (layers x width floats,
 * copied); NULL clears the scales. Returns 0, or -1. */
int trit_lm_set_ffn_scales(TritLm *lm, const float *scales, size_t layers, size_t width);

/* CausalLm::generate_additive (causal_lm.rs:317-345), Voxtral Realtime's
 * loop: the prompt's embeddings plus audio rows 0..n, then each new token's
 * embedding plus the next row (`audio`: rows x width floats), until a token
 * of `stop` or the rows end; at most rows - n + 1 tokens, written to `out`
 * (cap of them). Returns the count, or -1. */
int64_t trit_lm_generate_additive(TritLm *lm, const int32_t *prompt, size_t n, const float *audio, size_t rows,
                                  const int32_t *stop, size_t nstop, int32_t *out, size_t cap);

/* CausalLm::bidirectional_tokens (causal_lm.rs:393-408), Granite Speech
 * NAR's editor: one pass over `m` rows (m x width floats) with no causal
 * mask, then the best token of each row from `from` on, m - from ids into
 * `out`. The rows must fit one prefill pass ("prefill_rows"). Returns
 * m - from, or -1. */
int64_t trit_lm_bidirectional_tokens(TritLm *lm, const float *rows, size_t m, size_t from, int32_t *out);

/* The device time of the last generation on this handle, from CUDA events:
 * the prompt (prefill) and the greedy steps after it, in ms, the number of
 * decode steps, and the kernel launches it made. Returns 0, or -1. */
int trit_lm_last_timing(const TritLm *lm, double *prefill_ms, double *decode_ms, int64_t *decode_steps,
                        int64_t *launches);

/* ---- single product layers (Dense, src/cpu/gemm.rs:14-542) ---- */

/* A layer from ggml Q8_0 blocks of an `n x k` row-major matrix (34 bytes a
 * block: f16 scale, 32 codes). table = 0: int8 activations in groups of 32
 * with f16-rounded scales, i8 x i8 products (Dense::q8_0 -> Int8::from_q8_0,
 * gemm.rs:212-231, int8.rs:234-289); table = 1: a token table, f32 math
 * (Dense::table -> Weights::Q8, gemm.rs:383-409). NULL on failure. */
TritDense *trit_dense_q8_0(const void *blocks, size_t n, size_t k, int table, int device);

/* out (rows x n) = x (rows x k) times the layer, both in host memory.
 * Returns 0, or -1. (Dense::forward, gemm.rs:500-542.) */
int trit_dense_forward(TritDense *layer, const float *x, size_t rows, float *out);

/* trit_dense_forward on device pointers, queued on `cuda_stream` (a
 * cudaStream_t, or NULL for the layer's own stream); does not wait. */
int trit_dense_forward_device(TritDense *layer, const float *x, size_t rows, float *out, void *cuda_stream);

/* Frees a layer. NULL is a no-op. */
void trit_dense_free(TritDense *layer);

/* A Q8_0 W8A8 product that allocates nothing, for callers that cannot
 * call cudaMalloc when they run it (inside another party's graph capture,
 * on a real-time thread, or with every byte of device memory owned by
 * their own pool). No counterpart in the reference: Trit runs on the CPU
 * and allocates freely. It computes what trit_dense_forward_device
 * computes, on device pointers: `codes` (n x k int8, row-major) and
 * `scales` (n x k/32 f16 bits) are the split form of ggml Q8_0 blocks
 * (block b of row r: scales[r * k/32 + b], codes[r * k + 32 b ...]); x is
 * rows x k f32; out is rows x n f32; k is a multiple of 128 from 128 to
 * 8192 and n a positive multiple of 32. Its scratch (the int8 activations and
 * their scales) is one 1 MiB device array that the library holds on every
 * GPU it is loaded on until the process exits, so rows * k * 9 / 8 must stay
 * within 1 MiB (larger calls fail). All calls share that array and leave
 * their contents in it: calls that overlap on the GPU (other streams,
 * other threads) race; order them on one stream. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture. Returns 0, or -1 with
 * trit_cuda_last_error(). Queued on `cuda_stream` (NULL: the default stream);
 * does not wait. */
int trit_dense_q8_0_forward_static(const void *codes, const void *scales, size_t n, size_t k, const float *x,
                                   size_t rows, float *out, void *cuda_stream);

#ifdef __cplusplus
}
#endif

#endif /* TRIT_CUDA_H */
