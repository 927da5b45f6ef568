// Plain structs shared by host and device code: how the model's weights,
// configuration and KV cache are laid out in device memory.
#pragma once

#include <cstddef>
#include <cstdint>

namespace trit {

// How a product layer stores its weights (all row-major by output row).
enum WeightKind : int {
  kQ8_0 = 0,      // codes i8 [n][k], scales f16 [n][k/32]; activations per 32, f16 scales
  kInt8Row = 1,   // codes i8 [n][k], scales f32 [n];       activations per 128
  kTernary = 2,   // codes u32 [n][k/16] (2-bit, pack_span), scales f32 [n][k/128]; activations per 128
};

struct DMat {
  int kind = 0;
  int n = 0, k = 0;
  int agroup = 32;   // activation group
  int half = 0;      // activation scales rounded to f16
  const void* codes = nullptr;
  const void* scales = nullptr;
};

// A token table, f32 math (Dense::table / Weights::Q8): codes i8 [n][k],
// one scale per 32 values, f16 (Q8_0 file) or f32 (int8 table).
struct DTable {
  int n = 0, k = 0;
  int scale_f16 = 1;
  const int8_t* codes = nullptr;
  const void* scales = nullptr;
};

struct DLayer {
  const float* norm_attn = nullptr;
  const float* q_norm = nullptr;  // null: no qk norm (llama, mistral, granite)
  const float* k_norm = nullptr;
  const float* norm_mlp = nullptr;
  const float* ffn_scale = nullptr;  // set_ffn_scales: the normed MLP input times this [d], or null
  DMat qkv, out, gate_up, down;
};

struct DConfig {
  int d, ffn, layers, heads, kv_heads, hd, vocab;
  float eps;
  float embedding_multiplier, residual_multiplier, logits_scaling;
  float q_scale;     // Granite attention multiplier * sqrt(hd), else 1
  int has_q_scale;
};

// The paged KV cache: pool[page][layer][2][kv_heads][page_tokens][hd],
// f16 or f32. A stream's logical page p is physical page table[p].
struct DCache {
  void* pool = nullptr;
  int f16 = 1;
  int page_tokens = 64;
  int pages_per_stream = 0;     // the width of one page table row
  const int* page_table = nullptr;  // [streams][pages_per_stream]
};

}  // namespace trit
