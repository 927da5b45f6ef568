// Launchers of the device kernels (host-callable, no templates).
#pragma once

#include <cuda_runtime.h>

#include <mutex>

#include "types.h"

namespace trit {

// One-time set-up per device (kernel attributes, device properties), safe
// when several host threads make their first call at once: f runs once per
// device index and its result is kept for later calls.
constexpr int kMaxDevices = 64;
struct DeviceOnce {
  std::once_flag flag[kMaxDevices];
  cudaError_t result[kMaxDevices] = {};
  template <class F>
  cudaError_t run(int dev, F f) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(flag[dev], [&] { result[dev] = f(); });
    return result[dev];
  }
};
// The SM count of the current device (148 on B200), looked up once.
int current_sm_count();

enum Epilogue : int { kEpOut = 0, kEpResid = 1, kEpSilu = 2 };

cudaError_t launch_embed(const DTable& T, const int* ids, int m, float* x, float mult, cudaStream_t s);
cudaError_t launch_scale(float* x, size_t n, float mult, cudaStream_t s);
// RmsNorm (weights w; null: none) of m rows, times `scale` (null: none),
// then the activation quantizer in groups of `group`.
cudaError_t launch_norm_quant(const float* x, int m, int d, const float* w, float eps, int group, int half,
                              int8_t* xq, float* xs, cudaStream_t s, const float* scale = nullptr);
cudaError_t launch_gemv(const DMat& W, const int8_t* xq, const float* xs, int m, int mode, float* y, int ldy,
                        float resid_mult, cudaStream_t s);
cudaError_t launch_qk_rope_append(float* qkv, int m, const DConfig& cfg, const float* q_norm, const float* k_norm,
                                  const float* rope, int rope_rows, const DCache& cache, const int* row_stream,
                                  const int* row_pos, int layer, cudaStream_t s);
// Attention of tiles of rows: tiles[b] = {first row, rows} of rows of one
// stream at consecutive positions, at most rows_max rows a tile
// (attention_tile_rows); tiles null: one row a block (ntiles rows).
// all_keys > 0: every row sees keys [0, all_keys) (no causal mask).
int attention_tile_rows(const DConfig& cfg, int tmax, int f16);
cudaError_t launch_attention_rows(const float* qkv, const int2* tiles, int ntiles, int rows_max, const DConfig& cfg,
                                  const DCache& cache, const int* row_stream, const int* row_pos, int layer,
                                  int max_tk, float* att, cudaStream_t s, int all_keys = 0);
// x[i] += a[i] for i < n.
cudaError_t launch_add(float* x, const float* a, size_t n, cudaStream_t s);
// RmsNorm of `nb` rows, the table product and each row's argmax. logits
// ([nb][vocab]) may be null; best_* hold [nb][table_blocks(vocab)].
// keys non-null (tensor parallelism, this rank's table rows from v0): each
// row's best as an argmax-ordered key (k_argmax_key) instead of a token;
// after the ranks' max-reduction, launch_key_tokens turns keys into tokens.
cudaError_t launch_final(const float* x, int ldx, int nb, const float* norm_w, const DConfig& cfg, const DTable& T,
                         float* xn, float* logits, float* best_val, int* best_idx, int* token, cudaStream_t s,
                         unsigned long long* keys = nullptr, int v0 = 0);
cudaError_t launch_key_tokens(const unsigned long long* keys, int nb, int* token, cudaStream_t s);
// The table product alone for `nb` rows already normed.
cudaError_t launch_table(const DTable& T, const float* xn, int nb, float mult, float* logits, float* best_val,
                         int* best_idx, cudaStream_t s);
int table_blocks(int n);
int table_max_streams();
// After a greedy step of a batch: tokens[step][s] = cur[s] for every stream,
// positions advance by one when `advance_pos`, and the step counter by one.
cudaError_t launch_batch_advance(const int* cur, int* pos, int* step, int* tokens, int streams, int advance_pos,
                                 cudaStream_t s);

// Tensor-core W8A8 products (mma.cu) for prefill and batches. A TcMap is an
// opaque TMA tensor map (CUtensorMap) of an int8 matrix [rows][k].
struct alignas(64) TcMap {
  unsigned long long opaque[16];
};
int tc_frames();  // frames (rows of x) per CTA: the frame map's row multiple
cudaError_t make_tc_weight_map(TcMap* out, const DMat& W, const void* codes8);
cudaError_t make_tc_frame_map(TcMap* out, const int8_t* xq, size_t rows_cap, size_t k);
// The f16 form of the Q8_0 products: codes as f16 (exact), so the tensor
// cores make exact f32 group dots and the fold needs no integer bias.
cudaError_t make_tc_map_f16(TcMap* out, const void* codes16, size_t rows, size_t k, int box_rows);
cudaError_t launch_codes_f16(const int8_t* in, size_t n, void* out, cudaStream_t s);
// y (m x ldy) from W times the quantized frames (xq via bmap, scales xs):
// kEpOut stores, kEpResid adds (times resid_mult). *status is set when a
// wait inside the kernel ran out.
// Prompt attention on the tensor cores ("exact": false; mma.cu): tiles of
// at most attention_tc_rows() rows of one stream, f16 cache, pages of a
// multiple of 64 positions.
bool attention_tc_supported(const DConfig& cfg, const DCache& cache);
int attention_tc_rows(const DConfig& cfg);
cudaError_t make_kv_map(TcMap* out, const void* pool, size_t rows);
cudaError_t launch_attention_tc(const TcMap& kvmap, const float* qkv, const int2* tiles, int ntiles,
                                const DConfig& cfg, const DCache& cache, const int* row_stream, const int* row_pos,
                                int layer, float* att, int* status, cudaStream_t s);
cudaError_t launch_gemm_tc(const TcMap& amap, const TcMap& bmap, const DMat& W, const float* xs, int m, int mode,
                           float* y, int ldy, float resid_mult, int* status, cudaStream_t s, bool f16 = false);
// h[m][units] = silu(g[.][u]) * g[.][units + u] for g = [m][2 units].
// silu(gate) * up of a stacked gate|up product, quantized in groups for the
// down product (the tensor-core path's h, never stored in f32).
cudaError_t launch_silu_quant(const float* g, int m, int units, int group, int half, int8_t* xq, float* xs,
                              cudaStream_t s);
// Ternary 2-bit words [n][k/16] -> int8 codes c - 1 in {-1, 0, 1}, [n][k].
cudaError_t launch_expand_ternary(const DMat& W, int8_t* out, cudaStream_t s);

// The persistent batch-1 decode (decode.cu).
constexpr int kEventSlots = 32;  // event stamps a layer (TRIT_PHASE_TRACE=3)
struct DecodeArgs {
  DConfig cfg;
  const DLayer* layers;  // device array [cfg.layers]
  const float* final_norm;
  DTable table;          // the output projection (the embedding when tied)
  DTable embed;
  DCache cache;
  const float* rope;
  int rope_rows;
  int stream;            // the stream slot whose pages this decode uses
  int first_pos;         // position of the first token fed
  int steps;             // forwards to run (each feeds the token before)
  const int* stop;       // device list of stop ids
  int nstop;
  int* tokens;           // [steps + 1]: tokens[0] is the token fed first; the rest are made
  int* count;            // how many tokens were made before a stop
  float* logits;         // optional [steps + 1][vocab] trace (row i + 1 from step i), or null
  unsigned long long* ll;   // [decode_ll_words] {data, tag} words, zeroed before the launch
  int* status;           // 0 ok; nonzero: a wait ran out (see decode.cu)
  long long* phase_ns;   // optional [steps][phases * layers + 2] globaltimer stamps of block 0, or null
                         // (5 phases a layer in decode.cu, 4 in decode_fast.cu)
  long long* events;     // optional [layers][kEventSlots][grid] per-block stamps of step event_step, or null
  int event_step;
  int key_tile;          // keys a staged attention tile (decode_fast.cu; set by its launcher)
  int table_stages;      // token-table rows in flight per warp (decode_fast.cu; set by its launcher)
};

// Whether the persistent decode takes this model (its product widths).
bool decode_supported(const DConfig& cfg);
cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t s);
int decode_grid(int device);
// LL words of the decode's hand-off buffers.
size_t decode_ll_words(const DConfig& cfg, int grid);

// The persistent batch-1 decode of the default path (decode_fast.cu): the
// reference's quantizers and integer products, floating-point sums in tree
// order, four hand-offs a layer. Whether it takes this model on `grid`
// blocks, its launch, and the LL words of its hand-off buffers.
bool decode_fast_supported(const DConfig& cfg, const DTable& table, int grid, int f16);
cudaError_t launch_decode_fast(const DecodeArgs& a, int grid, cudaStream_t s);
size_t decode_fast_ll_words(const DConfig& cfg, int grid);

}  // namespace trit
