/* Seeded synthetic decoder models for benchmarks and tests
 * (tests/synth/libtrit_synth.so, apart from the product library; host code
 * only, no GPU needed). The reference has no
 * counterpart: its benchmarks run downloaded checkpoints, which this build
 * replaces with seeded weights of the same shapes.
 */
#ifndef TRIT_SYNTH_H
#define TRIT_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Writes `dir`/config.json and `dir`/model.gguf (the folder must exist).
 * spec_json: {"config": {Hugging Face config keys: model_type,
 * hidden_size, intermediate_size, num_hidden_layers, num_attention_heads,
 * num_key_value_heads, head_dim, vocab_size, rms_norm_eps, rope_theta,
 * tie_word_embeddings, and Granite's embedding_multiplier,
 * attention_multiplier, residual_multiplier, logits_scaling},
 * "format": "q8_0" | "float" | "int8" | "ternary", "seed": N, "std": 0.02,
 * "dtype": "f32" | "f16" | "bf16" (the float format's elements),
 * "container": "gguf" (model.gguf) | "safetensors" (model.safetensors),
 * "names": "hf" | "transcribe" (one <arch>.gguf as transcribe.cpp writes
 * it: no config.json, the settings in stt.<arch>.decoder.* metadata, dec.*
 * tensor names), "arch": "qwen3_asr" (of a transcribe file),
 * "prefix": start of every tensor name (""), "config_at": key path the
 * settings are nested under in config.json ("", or for example
 * "thinker_config.text_config.")}. Returns 0, or -1 (trit_synth_last_error). */
int trit_synth_model(const char *dir, const char *spec_json);

/* The error of the last failed trit_synth_model on this thread. */
const char *trit_synth_last_error(void);

/* The f32 values of row `row` of tensor `name` (without ".weight") before
 * quantization: k values of N(0, sd) from the model's seed. */
void trit_synth_normal_row(uint64_t seed, const char *name, uint64_t row, size_t k, float sd, float *out);

#ifdef __cplusplus
}
#endif

#endif /* TRIT_SYNTH_H */
