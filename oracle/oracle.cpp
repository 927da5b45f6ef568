// TEST INFRASTRUCTURE ONLY. Nothing in the product (trit_b200/) links,
// loads or calls this file; tests/, __graft_entry__.smoke() and the CPU
// baseline legs of bench.py use it as the checker.
//
// A CPU restatement, in C++17, of the greedy token loop of Trit's decoder
// language model (Hi9841/trit 0.15.0, Rust). Every function names the
// reference lines it follows (paths relative to the reference project).
//
// Parity status: UNPINNED at the golden-vector level. The reference ships
// no unit tests and no golden vectors (AGENTS.md:92), and its Rust crates
// cannot be built in this image (no cargo, no network). The restatement is
// pinned by the self-checks that the reference implies (f16 conversion
// against IEEE round-to-nearest-even, ggml Q8_0 round trips, base-3 digit
// tables, the ggml quantizer rounding half away from zero) and by the
// committed fixtures in tests/golden/, which freeze its outputs.
//
// Arithmetic follows the reference's AVX-512 VNNI production path:
//   * W8A8 products: per (row, group) an exact i32 dot, then
//     acc = fma(f32(dot), w_scale * x_scale, acc) in group order
//     (src/cpu/int8.rs:560-570; ternary src/cpu/kernels.rs:395-405).
//   * f32 products (token tables): 16 lanes of fma over k, lane l taking
//     k = 16t + l in order, then the _mm512_reduce_add_ps tree
//     (src/cpu/fgemm.rs:380-430).
//   * attention products: one sequential fma chain per output
//     (src/cpu/fgemm.rs:700-860, matmul_nn / strips).
//   * exp: the Cephes polynomial in its AVX-512 form
//     (src/cpu/activation.rs:8-38,356-372).
// The source is built with -ffp-contract=off: every fma below is explicit.

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>
#include <omp.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace {

using std::size_t;
using std::string;
using std::vector;

thread_local string g_error;

// ---------------------------------------------------------------- f16 ----
// src/cpu/tensors.rs:542-580 (f32_to_f16: nearest, ties to even; subnormals).
uint16_t f32_to_f16(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, 4);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
  int32_t exponent = (int32_t)((bits >> 23) & 0xff);
  uint32_t mantissa = bits & 0x7fffff;
  if (exponent == 0xff) return sign | 0x7c00 | (mantissa != 0 ? 0x200 : 0);
  int32_t half_exponent = exponent - 127 + 15;
  if (half_exponent >= 0x1f) return sign | 0x7c00;
  if (half_exponent <= 0) {
    if (half_exponent < -10) return sign;
    uint32_t full = mantissa | 0x800000;
    uint32_t shift = (uint32_t)(14 - half_exponent);
    uint32_t half = full >> shift;
    uint32_t rest = full & ((1u << shift) - 1);
    uint32_t midpoint = 1u << (shift - 1);
    bool round = rest > midpoint || (rest == midpoint && (half & 1) == 1);
    return sign | (uint16_t)(half + (round ? 1 : 0));
  }
  uint32_t half = ((uint32_t)half_exponent << 10) | (mantissa >> 13);
  uint32_t rest = mantissa & 0x1fff;
  bool round = rest > 0x1000 || (rest == 0x1000 && (half & 1) == 1);
  return sign | (uint16_t)(half + (round ? 1 : 0));
}

// src/cpu/tensors.rs:582-595.
float f16_to_f32(uint16_t half) {
  uint32_t sign = (uint32_t)(half >> 15) << 31;
  uint32_t exponent = (half >> 10) & 0x1f;
  uint32_t mantissa = half & 0x3ff;
  uint32_t bits;
  if (exponent == 0 && mantissa == 0) {
    bits = sign;
  } else if (exponent == 0) {
    uint32_t exp = 127 - 15 + 1;
    uint32_t m = mantissa;
    while ((m & 0x400) == 0) {
      m <<= 1;
      exp -= 1;
    }
    bits = sign | (exp << 23) | ((m & 0x3ff) << 13);
  } else if (exponent == 0x1f) {
    bits = sign | 0x7f800000 | (mantissa << 13);
  } else {
    bits = sign | ((exponent + 127 - 15) << 23) | (mantissa << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

// ---------------------------------------------------------------- exp ----
// src/cpu/activation.rs:8-38 (constants) and :356-372 (the AVX-512 form).
const float LOG2E = 1.44269504088896340735992468100189214f;
const float LN2_HI = 0.6933594f;
const float LN2_LO = -2.1219444e-4f;
const float EXP_LOW = -87.3f;
const float EXP_HIGH = 88.0f;
const float POLY[6] = {1.9875691e-4f, 1.3981999e-3f, 8.333452e-3f,
                       4.1665796e-2f, 0.16666665f, 0.5f};

float cephes_exp(float x) {
  // _mm512_max_ps(x, LOW) returns LOW for a NaN x; min then caps at HIGH.
  x = (x > EXP_LOW) ? x : EXP_LOW;
  x = (x < EXP_HIGH) ? x : EXP_HIGH;
  float t = x * LOG2E;
  int32_t n_int = (int32_t)std::nearbyint(t);  // cvtps2dq: nearest, ties even
  float n = (float)n_int;
  float r = std::fma(-n, LN2_HI, x);
  r = std::fma(-n, LN2_LO, r);
  float p = 0.0f;
  for (float c : POLY) p = std::fma(p, r, c);
  float rr = r * r;
  float r1 = r + 1.0f;
  float y = std::fma(p, rr, r1);
  uint32_t two_bits = (uint32_t)(n_int + 127) << 23;
  float two_n;
  std::memcpy(&two_n, &two_bits, 4);
  return y * two_n;
}

// src/cpu/activation.rs:330 (AVX-512 Silu: v / (1 + exp(0 - v))).
float silu(float v) { return v / (1.0f + cephes_exp(0.0f - v)); }

// ------------------------------------------------------- quantizers ----
// src/cpu/int8.rs:176-186 (group_scale, quantize_code: weights).
float group_scale(float max) { return max > 0.0f ? max / 127.0f : 1.0f; }
int8_t quantize_code(float value, float scale) {
  float v = std::nearbyint(value / scale);
  v = std::min(std::max(v, -127.0f), 127.0f);
  return (int8_t)v;
}

// src/cpu/gemm.rs:53-76 (Blocks::quantize, ggml quantize_row_q8_0_ref):
// d = max|x| / 127, codes round(x * (1/d)) half away from zero, d as f16.
void q8_0_quantize(const float* values, size_t count, int8_t* codes, uint16_t* scales) {
  for (size_t b = 0; b < count / 32; ++b) {
    const float* block = values + b * 32;
    float max = 0.0f;
    for (int i = 0; i < 32; ++i) max = std::max(max, std::fabs(block[i]));
    float d = max / 127.0f;
    float inverse = d != 0.0f ? 1.0f / d : 0.0f;
    for (int i = 0; i < 32; ++i) {
      // `as i8` saturates in Rust.
      float v = std::round(block[i] * inverse);
      codes[b * 32 + i] = (int8_t)std::min(std::max(v, -128.0f), 127.0f);
    }
    scales[b] = f32_to_f16(d);
  }
}

// src/cpu/kernels.rs:646-737 (Quantized::grouped) with the values of
// quantize_scalar / quantize_avx512 (:769-807): scale = max|x|/127 (1 for
// an all-zero group), codes = clamp(round_ties_even(x * (1/scale)), +-127),
// the sum of the codes; Q8_0 rounds each scale to f16 after the codes.
struct Quantized {
  size_t m = 0, k = 0, group = 0;
  vector<int8_t> values;
  vector<float> scales;
  vector<int32_t> sums;
};

void quantize_group(const float* src, size_t n, int8_t* dst, float* scale_out, int32_t* sum_out) {
  float max = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float a = std::fabs(src[i]);
    max = (max > a) ? max : a;  // vmaxps(vmax, abs): keeps vmax for a NaN
  }
  float scale = group_scale(max);
  float inv = 1.0f / scale;
  int32_t sum = 0;
  for (size_t i = 0; i < n; ++i) {
    float v = std::nearbyint(src[i] * inv);
    v = std::min(std::max(v, -127.0f), 127.0f);
    dst[i] = (int8_t)v;
    sum += (int32_t)dst[i];
  }
  *scale_out = scale;
  *sum_out = sum;
}

Quantized quantize_grouped(const float* x, size_t m, size_t k, size_t group, bool half_scales) {
  Quantized q;
  q.m = m;
  q.k = k;
  q.group = group;
  size_t groups = k / group;
  q.values.resize(m * k);
  q.scales.resize(m * groups);
  q.sums.resize(m * groups);
#pragma omp parallel for schedule(static) if (m > 1)
  for (long row = 0; row < (long)m; ++row) {
    for (size_t g = 0; g < groups; ++g) {
      float scale;
      int32_t sum;
      quantize_group(x + row * k + g * group, group, q.values.data() + row * k + g * group,
                     &scale, &sum);
      q.scales[row * groups + g] = half_scales ? f16_to_f32(f32_to_f16(scale)) : scale;
      q.sums[row * groups + g] = sum;
    }
  }
  return q;
}

// --------------------------------------------------- W8A8 products ----
// An Int8 layer (src/cpu/int8.rs:190-240): row-major codes (ternary codes
// are held as code - 1, which gives the same integer dots as the
// reference's sum(c*q) - sum(q), src/cpu/kernels.rs:318-322), one f32
// scale per (row, weight group), activations quantized per `group`.
struct IntLayer {
  size_t n = 0, k = 0;
  size_t group = 0;          // activation group (32 Q8_0, 128 int8/ternary)
  size_t wgroup = 0;         // k values per weight scale
  bool half_scales = false;  // Q8_0 rounds activation scales to f16
  vector<int8_t> codes;      // [n][k]
  vector<float> scales;      // [n][k / wgroup]
  vector<int8_t> packed;     // VNNI layout [n/16][k/4][16][4], bytes flipped (+128)
};

bool cpu_has_vnni() {
#if defined(__x86_64__)
  static int has = -1;
  if (has < 0) {
    __builtin_cpu_init();
    has = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
          __builtin_cpu_supports("avx512vnni");
  }
  return has == 1;
#else
  return false;
#endif
}

bool g_force_scalar = false;

const char* isa_name() { return (cpu_has_vnni() && !g_force_scalar) ? "avx512-vnni" : "scalar"; }

// Path::at for Vnni512 (src/cpu/int8.rs:85-100) and the +128 flip (:101-106).
void pack_vnni(IntLayer& layer) {
  if (!cpu_has_vnni() || layer.n % 32 != 0 || layer.k % layer.group != 0) return;
  size_t n = layer.n, k = layer.k;
  layer.packed.resize(n * k);
#pragma omp parallel for schedule(static)
  for (long row = 0; row < (long)n; ++row) {
    size_t block = row / 16, r = row % 16;
    for (size_t kk = 0; kk < k; ++kk) {
      int8_t code = layer.codes[row * k + kk];
      layer.packed[((block * (k / 4) + kk / 4) * 16 + r) * 4 + kk % 4] = (int8_t)(code ^ (int8_t)0x80);
    }
  }
}

float w_scale(const IntLayer& L, size_t row, size_t g) {
  size_t wg = (g * L.group) / L.wgroup;
  return L.scales[row * (L.k / L.wgroup) + wg];
}

// One output: the group chain of src/cpu/int8.rs:560-570.
float int_row_scalar(const IntLayer& L, const Quantized& q, size_t frame, size_t row) {
  size_t groups = L.k / L.group;
  float acc = 0.0f;
  for (size_t g = 0; g < groups; ++g) {
    int32_t dot = 0;
    const int8_t* w = L.codes.data() + row * L.k + g * L.group;
    const int8_t* x = q.values.data() + frame * L.k + g * L.group;
    for (size_t i = 0; i < L.group; ++i) dot += (int32_t)w[i] * (int32_t)x[i];
    float scale = w_scale(L, row, g) * q.scales[frame * groups + g];
    acc = std::fma((float)dot, scale, acc);
  }
  return acc;
}

#if defined(__x86_64__)
// The VNNI tile of src/cpu/int8.rs:520-584: 32 outputs (two 16-row blocks)
// by F frames; the same f32 steps as int_row_scalar.
template <int F>
__attribute__((target("avx512f,avx512bw,avx512vnni"))) void vnni_tile(
    const IntLayer& L, const Quantized& q, size_t task, size_t frame0, float* out) {
  size_t k = L.k, k4s = k / 4, groups = k / L.group, quads = L.group / 4;
  size_t blocks[2] = {2 * task, 2 * task + 1};
  __m512 acc[2][F];
  for (int b = 0; b < 2; ++b)
    for (int f = 0; f < F; ++f) acc[b][f] = _mm512_setzero_ps();
  for (size_t g = 0; g < groups; ++g) {
    __m512i dots[2][F];
    for (int b = 0; b < 2; ++b)
      for (int f = 0; f < F; ++f) dots[b][f] = _mm512_setzero_si512();
    for (size_t k4 = g * quads; k4 < (g + 1) * quads; ++k4) {
      __m512i w0 = _mm512_loadu_si512(L.packed.data() + (blocks[0] * k4s + k4) * 64);
      __m512i w1 = _mm512_loadu_si512(L.packed.data() + (blocks[1] * k4s + k4) * 64);
      for (int f = 0; f < F; ++f) {
        int32_t four;
        std::memcpy(&four, q.values.data() + (frame0 + f) * k + k4 * 4, 4);
        __m512i x = _mm512_set1_epi32(four);
        dots[0][f] = _mm512_dpbusd_epi32(dots[0][f], w0, x);
        dots[1][f] = _mm512_dpbusd_epi32(dots[1][f], w1, x);
      }
    }
    for (int b = 0; b < 2; ++b) {
      float ws[16];
      for (int r = 0; r < 16; ++r) ws[r] = w_scale(L, blocks[b] * 16 + r, g);
      __m512 wscale = _mm512_loadu_ps(ws);
      for (int f = 0; f < F; ++f) {
        size_t index = (frame0 + f) * groups + g;
        __m512i corrected = _mm512_sub_epi32(dots[b][f], _mm512_set1_epi32(128 * q.sums[index]));
        __m512 scale = _mm512_mul_ps(wscale, _mm512_set1_ps(q.scales[index]));
        acc[b][f] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(corrected), scale, acc[b][f]);
      }
    }
  }
  for (int b = 0; b < 2; ++b)
    for (int f = 0; f < F; ++f) _mm512_storeu_ps(out + (frame0 + f) * L.n + blocks[b] * 16, acc[b][f]);
}

void vnni_task(const IntLayer& L, const Quantized& q, size_t task, float* out) {
  size_t frame = 0;
  while (frame + 6 <= q.m) {
    vnni_tile<6>(L, q, task, frame, out);
    frame += 6;
  }
  switch (q.m - frame) {
    case 1: vnni_tile<1>(L, q, task, frame, out); break;
    case 2: vnni_tile<2>(L, q, task, frame, out); break;
    case 3: vnni_tile<3>(L, q, task, frame, out); break;
    case 4: vnni_tile<4>(L, q, task, frame, out); break;
    case 5: vnni_tile<5>(L, q, task, frame, out); break;
    default: break;
  }
}
#endif

// Int8::forward_biased (src/cpu/int8.rs:425-483) with no bias.
vector<float> int_forward_q(const IntLayer& L, const Quantized& q) {
  vector<float> out(q.m * L.n);
#if defined(__x86_64__)
  if (!L.packed.empty() && !g_force_scalar) {
#pragma omp parallel for schedule(dynamic, 1)
    for (long task = 0; task < (long)(L.n / 32); ++task) vnni_task(L, q, task, out.data());
    return out;
  }
#endif
#pragma omp parallel for schedule(static)
  for (long row = 0; row < (long)L.n; ++row)
    for (size_t f = 0; f < q.m; ++f) out[f * L.n + row] = int_row_scalar(L, q, f, row);
  return out;
}

vector<float> int_forward(const IntLayer& L, const float* x, size_t m) {
  Quantized q = quantize_grouped(x, m, L.k, L.group, L.half_scales);
  return int_forward_q(L, q);
}

// ------------------------------------------ token table, f32 math ----
// Q8 (src/cpu/gemm.rs:37-187): int8 storage, one f32 scale per 32 values,
// widened to f32 (code * scale) and multiplied in f32 (Q8::matmul ->
// fgemm::matmul_widened, src/cpu/fgemm.rs:265-295; tile :380-430).
struct Table {
  size_t n = 0, k = 0;
  vector<int8_t> codes;  // [n][k]
  vector<float> scales;  // [n][k/32]
};

// _mm512_reduce_add_ps: halves, then quarters, then pairs.
float reduce16(const float* a) {
  float s8[8], s4[4];
  for (int i = 0; i < 8; ++i) s8[i] = a[i] + a[i + 8];
  for (int i = 0; i < 4; ++i) s4[i] = s8[i] + s8[i + 4];
  float s0 = s4[0] + s4[2], s1 = s4[1] + s4[3];
  return s0 + s1;
}

float table_dot(const Table& t, const float* x, size_t row) {
  float lanes[16] = {0};
  const int8_t* c = t.codes.data() + row * t.k;
  const float* s = t.scales.data() + row * (t.k / 32);
  size_t kk = 0;
  for (; kk + 16 <= t.k; kk += 16)
    for (int l = 0; l < 16; ++l) {
      float w = (float)c[kk + l] * s[(kk + l) / 32];
      lanes[l] = std::fma(x[kk + l], w, lanes[l]);
    }
  // A k tail (masked load: zeros beyond k) keeps the same lanes.
  for (int l = 0; kk + l < t.k; ++l) {
    float w = (float)c[kk + l] * s[(kk + l) / 32];
    lanes[l] = std::fma(x[kk + l], w, lanes[l]);
  }
  return reduce16(lanes);
}

#if defined(__x86_64__)
__attribute__((target("avx512f"))) float table_dot_avx512(const Table& t, const float* x,
                                                            size_t row) {
  const int8_t* c = t.codes.data() + row * t.k;
  const float* s = t.scales.data() + row * (t.k / 32);
  __m512 acc = _mm512_setzero_ps();
  for (size_t kk = 0; kk < t.k; kk += 16) {
    __m128i bytes = _mm_loadu_si128((const __m128i*)(c + kk));
    __m512 w = _mm512_mul_ps(_mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(bytes)),
                             _mm512_set1_ps(s[kk / 32]));
    acc = _mm512_fmadd_ps(_mm512_loadu_ps(x + kk), w, acc);
  }
  float lanes[16];
  _mm512_storeu_ps(lanes, acc);
  return reduce16(lanes);
}
#endif

vector<float> table_forward(const Table& t, const float* x, size_t m) {
  vector<float> out(m * t.n);
  bool fast = false;
#if defined(__x86_64__)
  fast = cpu_has_vnni() && !g_force_scalar && t.k % 16 == 0;
#endif
#pragma omp parallel for schedule(static)
  for (long j = 0; j < (long)t.n; ++j)
    for (size_t i = 0; i < m; ++i) {
#if defined(__x86_64__)
      out[i * t.n + j] = fast ? table_dot_avx512(t, x + i * t.k, j) : table_dot(t, x + i * t.k, j);
#else
      out[i * t.n + j] = table_dot(t, x + i * t.k, j);
#endif
    }
  return out;
}

// Dense::row (src/cpu/gemm.rs:412-429) for a Q8 table: code * scale.
void table_row(const Table& t, size_t index, float* out) {
  for (size_t kk = 0; kk < t.k; ++kk)
    out[kk] = (float)t.codes[index * t.k + kk] * t.scales[index * (t.k / 32) + kk / 32];
}

// ----------------------------------------------------------- layers ----
// RmsNorm::apply_in_place (src/layers.rs:135-144): a sequential f32 sum
// of squares, inv = 1 / sqrt(sum / d + eps), v *= inv * w.
void rms_in_place(float* row, const float* w, size_t d, float eps) {
  float sum = -0.0f;
  for (size_t i = 0; i < d; ++i) {
    float sq = row[i] * row[i];
    sum = sum + sq;
  }
  float inv = 1.0f / std::sqrt(sum / (float)d + eps);
  for (size_t i = 0; i < d; ++i) {
    float s = inv * w[i];
    row[i] = row[i] * s;
  }
}

// Rotary::halves + apply (src/layers.rs:276-335): inv_freq = base^(-2i/dims)
// in f32, (position * f).sin_cos() in f32, pairs (i, i + dims/2).
struct Rotary {
  size_t dims = 0;
  vector<float> inv_freq;
  void init(size_t d, float base) {
    dims = d;
    inv_freq.resize(d / 2);
    for (size_t i = 0; i < d / 2; ++i) inv_freq[i] = powf(base, -((float)(2 * i)) / (float)d);
  }
  void apply(float* x, size_t rows, size_t stride, size_t heads, size_t hd, size_t first) const {
    size_t half = dims / 2;
    vector<float> sn(half), cs(half);
    for (size_t r = 0; r < rows; ++r) {
      float position = (float)(first + r);
      for (size_t i = 0; i < half; ++i) {
        float a = position * inv_freq[i];
        sn[i] = sinf(a);
        cs[i] = cosf(a);
      }
      for (size_t h = 0; h < heads; ++h) {
        float* head = x + r * stride + h * hd;
        for (size_t i = 0; i < half; ++i) {
          float a = head[i], b = head[i + half];
          float ac = a * cs[i], bs = b * sn[i];
          float bc = b * cs[i], as = a * sn[i];
          head[i] = ac - bs;
          head[i + half] = bc + as;
        }
      }
    }
  }
};

// attention + HeadMajor + attention_with (src/layers.rs:343-504) and
// softmax_rows (:571-587): q scaled by 1/sqrt(hd); scores as sequential fma
// chains over the head dimension; keys beyond the causal limit set to -inf
// before the maximum; exp of (score - max) summed in key order; each
// probability times 1/sum; values as sequential fma chains over the keys.
void attention(const float* q, size_t qs, const float* k, const float* v, size_t kvs, size_t tq,
               size_t tk, size_t heads, size_t kv_heads, size_t hd, bool causal, float* out) {
  size_t d = heads * hd;
  size_t group = heads / kv_heads;
  float scale = 1.0f / std::sqrt((float)hd);
#pragma omp parallel for schedule(dynamic, 1) if (tq * tk > 4096)
  for (long task = 0; task < (long)(heads * tq); ++task) {
    size_t h = task / tq, i = task % tq;
    size_t g = h / group;
    vector<float> qh(hd), probs(tk);
    for (size_t e = 0; e < hd; ++e) qh[e] = q[i * qs + h * hd + e] * scale;
    for (size_t j = 0; j < tk; ++j) {
      float acc = 0.0f;
      const float* key = k + j * kvs + g * hd;
      for (size_t e = 0; e < hd; ++e) acc = std::fma(qh[e], key[e], acc);
      probs[j] = acc;
    }
    size_t visible = causal ? tk - tq + i + 1 : tk;
    for (size_t j = visible; j < tk; ++j) probs[j] = -INFINITY;
    float max = -INFINITY;
    for (size_t j = 0; j < tk; ++j) max = (probs[j] > max) ? probs[j] : max;
    float sum = 0.0f;
    for (size_t j = 0; j < tk; ++j) {
      probs[j] = cephes_exp(probs[j] - max);
      sum = sum + probs[j];
    }
    float inv = 1.0f / sum;
    for (size_t j = 0; j < tk; ++j) probs[j] = probs[j] * inv;
    for (size_t e = 0; e < hd; ++e) {
      float acc = 0.0f;
      for (size_t j = 0; j < tk; ++j) acc = std::fma(probs[j], v[j * kvs + g * hd + e], acc);
      out[i * d + h * hd + e] = acc;
    }
  }
}

// argmax (src/layers.rs:603-612): the first strict maximum wins.
size_t argmax(const float* values, size_t n) {
  size_t best = 0;
  for (size_t i = 0; i < n; ++i)
    if (values[i] > values[best]) best = i;
  return best;
}

// ------------------------------------------------------------ files ----
// A minimal JSON reader for config.json: numbers, strings, bools, null,
// nested objects (flattened to "a.b.c" keys), arrays skipped.
struct Json {
  std::map<string, string> strings;
  std::map<string, double> numbers;
  std::map<string, bool> flags;
  bool has_number(const string& key) const { return numbers.count(key) > 0; }
};

struct JsonParser {
  const char* p;
  const char* end;
  Json* out;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  string str() {
    if (*p != '"') throw std::runtime_error("config.json: expected a string");
    ++p;
    string s;
    while (p < end && *p != '"') {
      if (*p == '\\' && p + 1 < end) ++p;
      s += *p++;
    }
    ++p;
    return s;
  }
  void value(const string& key) {
    ws();
    if (p >= end) throw std::runtime_error("config.json ends early");
    if (*p == '{') {
      ++p;
      ws();
      if (*p == '}') {
        ++p;
        return;
      }
      while (true) {
        ws();
        string name = str();
        ws();
        if (*p != ':') throw std::runtime_error("config.json: expected ':'");
        ++p;
        value(key.empty() ? name : key + "." + name);
        ws();
        if (*p == ',') {
          ++p;
          continue;
        }
        if (*p == '}') {
          ++p;
          return;
        }
        throw std::runtime_error("config.json: expected ',' or '}'");
      }
    } else if (*p == '[') {
      int depth = 0;
      bool in_string = false;
      while (p < end) {
        char c = *p++;
        if (in_string) {
          if (c == '\\') ++p;
          else if (c == '"') in_string = false;
        } else if (c == '"') in_string = true;
        else if (c == '[') ++depth;
        else if (c == ']' && --depth == 0) return;
      }
    } else if (*p == '"') {
      out->strings[key] = str();
    } else if (!strncmp(p, "true", 4)) {
      out->flags[key] = true;
      p += 4;
    } else if (!strncmp(p, "false", 5)) {
      out->flags[key] = false;
      p += 5;
    } else if (!strncmp(p, "null", 4)) {
      p += 4;
    } else {
      char* stop = nullptr;
      double v = strtod(p, &stop);
      if (stop == p) throw std::runtime_error("config.json: bad value");
      out->numbers[key] = v;
      p = stop;
    }
  }
};

Json parse_json(const string& text) {
  Json j;
  JsonParser parser{text.data(), text.data() + text.size(), &j};
  parser.value("");
  return j;
}

string read_file(const string& path) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) throw std::runtime_error("cannot open " + path);
  string s;
  char buf[65536];
  size_t n;
  while ((n = fread(buf, 1, sizeof buf, f)) > 0) s.append(buf, n);
  fclose(f);
  return s;
}

// A GGUF v2/v3 reader (the layout that src/models/gguf/mod.rs:147-215 reads).
struct GgufTensor {
  uint32_t type = 0;
  vector<uint64_t> dims;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
  uint64_t count() const {
    uint64_t c = 1;
    for (uint64_t d : dims) c *= d;
    return c;
  }
};

struct Gguf {
  void* map = nullptr;
  size_t size = 0;
  std::map<string, GgufTensor> tensors;
  ~Gguf() {
    if (map) munmap(map, size);
  }
};

size_t ggml_bytes(uint32_t type, uint64_t count) {
  switch (type) {
    case 0: return count * 4;         // F32
    case 1: return count * 2;         // F16
    case 8: return count / 32 * 34;   // Q8_0
    case 24: return count;            // I8
    case 26: return count * 4;        // I32
    default: throw std::runtime_error("gguf: ggml type " + std::to_string(type) + " not read here");
  }
}

std::unique_ptr<Gguf> open_gguf(const string& path) {
  auto g = std::make_unique<Gguf>();
  int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("cannot open " + path);
  struct stat st;
  fstat(fd, &st);
  g->size = st.st_size;
  g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (g->map == MAP_FAILED) {
    g->map = nullptr;
    throw std::runtime_error("cannot map " + path);
  }
  const uint8_t* base = (const uint8_t*)g->map;
  size_t at = 0;
  auto need = [&](size_t n) {
    if (at + n > g->size) throw std::runtime_error("gguf: truncated file");
  };
  auto u32 = [&]() { need(4); uint32_t v; memcpy(&v, base + at, 4); at += 4; return v; };
  auto u64 = [&]() { need(8); uint64_t v; memcpy(&v, base + at, 8); at += 8; return v; };
  auto gstr = [&]() { uint64_t n = u64(); need(n); string s((const char*)base + at, n); at += n; return s; };
  if (g->size < 4 || memcmp(base, "GGUF", 4) != 0) throw std::runtime_error("not a GGUF file");
  at = 4;
  uint32_t version = u32();
  if (version < 2 || version > 3) throw std::runtime_error("gguf version");
  uint64_t tensor_count = u64(), kv_count = u64();
  uint64_t alignment = 32;
  std::function<void(uint32_t)> skip = [&](uint32_t type) {
    static const size_t sizes[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type == 8) { gstr(); return; }
    if (type == 9) {
      uint32_t et = u32();
      uint64_t n = u64();
      for (uint64_t i = 0; i < n; ++i) skip(et);
      return;
    }
    if (type > 12) throw std::runtime_error("gguf: bad value type");
    need(sizes[type]);
    at += sizes[type];
  };
  for (uint64_t i = 0; i < kv_count; ++i) {
    string key = gstr();
    uint32_t type = u32();
    if (key == "general.alignment" && type == 4) {
      alignment = u32();
    } else {
      skip(type);
    }
  }
  struct Info { string name; GgufTensor t; uint64_t offset; };
  vector<Info> infos;
  for (uint64_t i = 0; i < tensor_count; ++i) {
    Info info;
    info.name = gstr();
    uint32_t nd = u32();
    for (uint32_t d = 0; d < nd; ++d) info.t.dims.push_back(u64());
    info.t.type = u32();
    info.offset = u64();
    infos.push_back(info);
  }
  size_t data = (at + alignment - 1) / alignment * alignment;
  for (auto& info : infos) {
    info.t.bytes = ggml_bytes(info.t.type, info.t.count());
    if (data + info.offset + info.t.bytes > g->size)
      throw std::runtime_error("gguf: tensor " + info.name + " runs past the end");
    info.t.data = base + data + info.offset;
    g->tensors[info.name] = info.t;
  }
  return g;
}

// ------------------------------------------------------------ model ----
struct Config {
  bool qk_norm = true;
  float embedding_multiplier = 1.0f, residual_multiplier = 1.0f, logits_scaling = 1.0f;
  bool has_attention_multiplier = false;
  float attention_multiplier = 1.0f;
  size_t d = 0, ffn = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0;
  float eps = 1e-6f, rope_base = 1e6f;
  bool tied = false;
};

// Config::parse (src/models/parts/causal_lm.rs:41-77).
Config parse_config(const Json& j) {
  Config c;
  auto num = [&](const char* k) -> size_t {
    if (!j.has_number(k)) throw std::runtime_error(string("config.json: no ") + k);
    return (size_t)j.numbers.at(k);
  };
  auto it = j.strings.find("model_type");
  string type = it == j.strings.end() ? "" : it->second;
  if (type == "qwen3") c.qk_norm = true;
  else if (type == "llama" || type == "mistral" || type == "granite") c.qk_norm = false;
  else throw std::runtime_error("config.json does not describe a language model this engine runs");
  c.heads = num("num_attention_heads");
  c.kv_heads = num("num_key_value_heads");
  if (c.heads == 0 || c.kv_heads == 0 || c.heads % c.kv_heads)
    throw std::runtime_error("config.json: the query heads do not share the key heads evenly");
  c.d = num("hidden_size");
  auto fl = [&](const char* k, float dflt) { return j.has_number(k) ? (float)j.numbers.at(k) : dflt; };
  c.embedding_multiplier = fl("embedding_multiplier", 1.0f);
  c.has_attention_multiplier = j.has_number("attention_multiplier");
  c.attention_multiplier = fl("attention_multiplier", 1.0f);
  c.residual_multiplier = fl("residual_multiplier", 1.0f);
  c.logits_scaling = fl("logits_scaling", 1.0f);
  c.ffn = num("intermediate_size");
  c.layers = num("num_hidden_layers");
  c.head_dim = j.has_number("head_dim") ? num("head_dim") : c.d / c.heads;
  c.vocab = num("vocab_size");
  c.eps = fl("rms_norm_eps", 1e-6f);
  c.rope_base = fl("rope_theta", 1e6f);
  auto t = j.flags.find("tie_word_embeddings");
  c.tied = t != j.flags.end() && t->second;
  return c;
}

struct Layer {
  vector<float> norm_attn, q_norm, k_norm, norm_mlp;
  IntLayer qkv, out, gate_up, down;
};

struct Model {
  Config c;
  vector<Layer> layers;
  vector<float> norm;
  Table embed;
  bool has_head = false;
  Table head;
  Rotary rotary;
  bool kv_f16 = false;  // a documented variant: K and V rounded to f16 as stored
  vector<vector<float>> ffn_scales;  // set_ffn_scales: [layers][d], or empty
};

const GgufTensor& tensor(const Gguf& g, const string& name) {
  auto it = g.tensors.find(name);
  if (it == g.tensors.end()) throw std::runtime_error("model.gguf has no tensor " + name);
  return it->second;
}

vector<float> f32_tensor(const Gguf& g, const string& name, size_t len) {
  const GgufTensor& t = tensor(g, name);
  if (t.count() != len) throw std::runtime_error("tensor " + name + " has the wrong size");
  vector<float> out(len);
  if (t.type == 0) memcpy(out.data(), t.data, len * 4);
  else if (t.type == 1) {
    for (size_t i = 0; i < len; ++i) {
      uint16_t h;
      memcpy(&h, t.data + 2 * i, 2);
      out[i] = f16_to_f32(h);
    }
  } else throw std::runtime_error("tensor " + name + " is not f32/f16");
  return out;
}

// Tensors::q8_0 (src/cpu/tensors.rs:282-305): 34-byte blocks -> codes and
// the f16 scales widened to f32.
void q8_0_blocks(const GgufTensor& t, size_t len, int8_t* codes, float* scales) {
  for (size_t b = 0; b < len / 32; ++b) {
    const uint8_t* block = t.data + b * 34;
    uint16_t h = (uint16_t)(block[0] | (block[1] << 8));
    scales[b] = f16_to_f32(h);
    memcpy(codes + b * 32, block + 2, 32);
  }
}

// The base-3 digits of every packed byte (src/cpu/kernels.rs:624-643).
void base3_digits(uint8_t byte, uint8_t out[5]) {
  unsigned value = byte;
  for (int d = 0; d < 5; ++d) {
    out[d] = (uint8_t)(value % 3);
    value /= 3;
  }
}

// Dense::load (src/cpu/gemm.rs:254-343) for one stacked layer: parts with
// their output rows, stacked by output rows. Q8_0 parts give Int8::from_q8_0
// (group 32, f16 activation scales); I8 parts with per-row f32 `.scales`
// give an Int8 layer whose group scales are the row scale (group 128);
// ternary `.qweight` (base 3, 5 codes a byte) with `.scales` per 128 give
// Ternary::from_base3 (src/cpu/kernels.rs:91-130; fastconformer.rs:440-452).
IntLayer load_dense(const Gguf& g, const vector<std::pair<string, size_t>>& parts, size_t k) {
  IntLayer L;
  L.k = k;
  for (auto& p : parts) L.n += p.second;
  L.codes.resize(L.n * k);
  string first = parts[0].first;
  size_t row0 = 0;
  if (g.tensors.count(first + ".weight") && tensor(g, first + ".weight").type == 8) {
    L.group = 32;
    L.wgroup = 32;
    L.half_scales = true;
    L.scales.resize(L.n * (k / 32));
    for (auto& p : parts) {
      const GgufTensor& t = tensor(g, p.first + ".weight");
      if (t.type != 8 || t.count() != p.second * k) throw std::runtime_error("bad Q8_0 part " + p.first);
      q8_0_blocks(t, p.second * k, L.codes.data() + row0 * k, L.scales.data() + row0 * (k / 32));
      row0 += p.second;
    }
  } else if (g.tensors.count(first + ".weight") && tensor(g, first + ".weight").type == 24) {
    L.group = 128;
    L.wgroup = k;
    L.scales.resize(L.n);
    for (auto& p : parts) {
      const GgufTensor& t = tensor(g, p.first + ".weight");
      if (t.count() != p.second * k) throw std::runtime_error("bad int8 part " + p.first);
      memcpy(L.codes.data() + row0 * k, t.data, p.second * k);
      vector<float> s = f32_tensor(g, p.first + ".scales", p.second);
      memcpy(L.scales.data() + row0, s.data(), p.second * 4);
      row0 += p.second;
    }
  } else if (g.tensors.count(first + ".qweight")) {
    L.group = 128;
    L.wgroup = 128;
    L.scales.resize(L.n * (k / 128));
    size_t row_bytes = (k + 4) / 5;
    for (auto& p : parts) {
      const GgufTensor& t = tensor(g, p.first + ".qweight");
      if (t.count() != p.second * row_bytes) throw std::runtime_error("bad ternary part " + p.first);
      for (size_t r = 0; r < p.second; ++r) {
        const uint8_t* src = t.data + r * row_bytes;
        int8_t* dst = L.codes.data() + (row0 + r) * k;
        for (size_t b = 0; b < row_bytes; ++b) {
          if (src[b] >= 243) throw std::runtime_error("ternary byte above 242");
          uint8_t digits[5];
          base3_digits(src[b], digits);
          for (int dd = 0; dd < 5 && b * 5 + dd < k; ++dd) dst[b * 5 + dd] = (int8_t)(digits[dd] - 1);
        }
      }
      vector<float> s = f32_tensor(g, p.first + ".scales", p.second * (k / 128));
      memcpy(L.scales.data() + row0 * (k / 128), s.data(), s.size() * 4);
      row0 += p.second;
    }
  } else {
    throw std::runtime_error("model.gguf has no weights for " + first);
  }
  pack_vnni(L);
  return L;
}

// Dense::table (src/cpu/gemm.rs:383-409): Q8_0 blocks kept with f32 math,
// or int8 codes with one f32 scale per 32 values (Q8::quantize's layout).
Table load_table(const Gguf& g, const string& name, size_t rows, size_t cols) {
  Table t;
  t.n = rows;
  t.k = cols;
  t.codes.resize(rows * cols);
  t.scales.resize(rows * (cols / 32));
  const GgufTensor& w = tensor(g, name + ".weight");
  if (w.count() != rows * cols) throw std::runtime_error("table " + name + " has the wrong size");
  if (w.type == 8) {
    q8_0_blocks(w, rows * cols, t.codes.data(), t.scales.data());
  } else if (w.type == 24) {
    memcpy(t.codes.data(), w.data, rows * cols);
    vector<float> s = f32_tensor(g, name + ".scales", rows * (cols / 32));
    t.scales = s;
  } else {
    throw std::runtime_error("table " + name + " is neither Q8_0 nor int8");
  }
  return t;
}

// CausalLm::from_tensors (src/models/parts/causal_lm.rs:141-198).
std::unique_ptr<Model> load_model(const string& dir) {
  auto m = std::make_unique<Model>();
  m->c = parse_config(parse_json(read_file(dir + "/config.json")));
  auto g = open_gguf(dir + "/model.gguf");
  const Config& c = m->c;
  size_t hd = c.head_dim;
  m->layers.resize(c.layers);
  for (size_t i = 0; i < c.layers; ++i) {
    string p = "model.layers." + std::to_string(i);
    Layer& L = m->layers[i];
    L.norm_attn = f32_tensor(*g, p + ".input_layernorm.weight", c.d);
    L.qkv = load_dense(*g, {{p + ".self_attn.q_proj", c.heads * hd},
                            {p + ".self_attn.k_proj", c.kv_heads * hd},
                            {p + ".self_attn.v_proj", c.kv_heads * hd}}, c.d);
    if (c.qk_norm) {
      L.q_norm = f32_tensor(*g, p + ".self_attn.q_norm.weight", hd);
      L.k_norm = f32_tensor(*g, p + ".self_attn.k_norm.weight", hd);
    }
    L.out = load_dense(*g, {{p + ".self_attn.o_proj", c.d}}, c.heads * hd);
    L.norm_mlp = f32_tensor(*g, p + ".post_attention_layernorm.weight", c.d);
    L.gate_up = load_dense(*g, {{p + ".mlp.gate_proj", c.ffn}, {p + ".mlp.up_proj", c.ffn}}, c.d);
    L.down = load_dense(*g, {{p + ".mlp.down_proj", c.d}}, c.ffn);
  }
  m->norm = f32_tensor(*g, "model.norm.weight", c.d);
  m->embed = load_table(*g, "model.embed_tokens", c.vocab, c.d);
  if (!c.tied && g->tensors.count("lm_head.weight")) {
    m->has_head = true;
    m->head = load_table(*g, "lm_head", c.vocab, c.d);
  }
  m->rotary.init(hd, c.rope_base);
  return m;
}

struct Cache {
  vector<vector<float>> keys, values;  // per layer, [tokens][kv_heads * hd]
};

void scale_all(float* x, size_t n, float w) {
  if (w != 1.0f)
    for (size_t i = 0; i < n; ++i) x[i] = x[i] * w;
}

// CausalLm::hidden (src/models/parts/causal_lm.rs:410-481).
void hidden(const Model& M, vector<float>& x, size_t first, Cache& cache, bool causal) {
  const Config& c = M.c;
  size_t d = c.d, hd = c.head_dim, m = x.size() / d;
  size_t qd = c.heads * hd, kv = c.kv_heads * hd, stride = qd + 2 * kv;
  scale_all(x.data(), x.size(), c.embedding_multiplier);
  float q_scale = c.has_attention_multiplier ? c.attention_multiplier * std::sqrt((float)hd) : 1.0f;
  for (size_t l = 0; l < c.layers; ++l) {
    const Layer& L = M.layers[l];
    vector<float> normed = x;
    for (size_t r = 0; r < m; ++r) rms_in_place(normed.data() + r * d, L.norm_attn.data(), d, c.eps);
    vector<float> qkv = int_forward(L.qkv, normed.data(), m);
    if (c.qk_norm) {
      for (size_t r = 0; r < m; ++r) {
        float* row = qkv.data() + r * stride;
        for (size_t h = 0; h < c.heads; ++h) rms_in_place(row + h * hd, L.q_norm.data(), hd, c.eps);
        for (size_t h = 0; h < c.kv_heads; ++h) rms_in_place(row + qd + h * hd, L.k_norm.data(), hd, c.eps);
      }
    }
    M.rotary.apply(qkv.data(), m, stride, c.heads, hd, first);
    M.rotary.apply(qkv.data() + qd, m, stride, c.kv_heads, hd, first);
    if (q_scale != 1.0f)
      for (size_t r = 0; r < m; ++r)
        for (size_t i = 0; i < qd; ++i) qkv[r * stride + i] = qkv[r * stride + i] * q_scale;
    for (size_t r = 0; r < m; ++r) {
      const float* row = qkv.data() + r * stride;
      for (size_t i = 0; i < kv; ++i) {
        float kk = row[qd + i], vv = row[qd + kv + i];
        if (M.kv_f16) {
          kk = f16_to_f32(f32_to_f16(kk));
          vv = f16_to_f32(f32_to_f16(vv));
        }
        cache.keys[l].push_back(kk);
        cache.values[l].push_back(vv);
      }
    }
    size_t seen = first + m;
    vector<float> att(m * qd);
    attention(qkv.data(), stride, cache.keys[l].data(), cache.values[l].data(), kv, m, seen, c.heads,
              c.kv_heads, hd, causal, att.data());
    vector<float> o = int_forward(L.out, att.data(), m);
    for (size_t i = 0; i < x.size(); ++i)
      x[i] = (c.residual_multiplier == 1.0f) ? x[i] + o[i] : x[i] + c.residual_multiplier * o[i];
    normed = x;
    for (size_t r = 0; r < m; ++r) rms_in_place(normed.data() + r * d, L.norm_mlp.data(), d, c.eps);
    // set_ffn_scales (causal_lm.rs:305-307,458-463): the normed MLP input
    // times the layer's scale, element by element.
    if (!M.ffn_scales.empty())
      for (size_t r = 0; r < m; ++r)
        for (size_t i = 0; i < d; ++i) normed[r * d + i] = normed[r * d + i] * M.ffn_scales[l][i];
    vector<float> wide = int_forward(L.gate_up, normed.data(), m);
    vector<float> hbuf(m * c.ffn);
    for (size_t r = 0; r < m; ++r)
      for (size_t j = 0; j < c.ffn; ++j) {
        float g = silu(wide[r * 2 * c.ffn + j]);
        hbuf[r * c.ffn + j] = g * wide[r * 2 * c.ffn + c.ffn + j];
      }
    vector<float> down = int_forward(L.down, hbuf.data(), m);
    for (size_t i = 0; i < x.size(); ++i)
      x[i] = (c.residual_multiplier == 1.0f) ? x[i] + down[i] : x[i] + c.residual_multiplier * down[i];
  }
}

// CausalLm::forward_rows (src/models/parts/causal_lm.rs:366-389).
vector<float> forward_rows(const Model& M, vector<float> x, size_t first, Cache& cache) {
  const Config& c = M.c;
  size_t m = x.size() / c.d;
  hidden(M, x, first, cache, true);
  vector<float> last(x.begin() + (m - 1) * c.d, x.end());
  rms_in_place(last.data(), M.norm.data(), c.d, c.eps);
  vector<float> logits = table_forward(M.has_head ? M.head : M.embed, last.data(), 1);
  scale_all(logits.data(), logits.size(), 1.0f / c.logits_scaling);
  return logits;
}

vector<float> embed(const Model& M, const int32_t* ids, size_t n) {
  vector<float> x(n * M.c.d);
  for (size_t i = 0; i < n; ++i) {
    if (ids[i] < 0 || (size_t)ids[i] >= M.c.vocab) throw std::runtime_error("token id out of range");
    table_row(M.embed, (size_t)ids[i], x.data() + i * M.c.d);
  }
  return x;
}

struct Prefix {
  vector<int32_t> tokens;
  Cache cache;
};

struct Trace {
  float* logits = nullptr;   // [steps][vocab] or null: the logits each token came from
  float* gaps = nullptr;     // [steps] top1 - top2 of those logits, or null
  double* seconds = nullptr; // [steps] wall time of the forward that made them, or null
};

// The top-1 minus top-2 logit of a row.
float top_gap(const float* v, size_t n) {
  size_t best = argmax(v, n);
  float second = -INFINITY;
  for (size_t i = 0; i < n; ++i)
    if (i != best && v[i] > second) second = v[i];
  return v[best] - second;
}

// CausalLm::greedy (src/models/parts/causal_lm.rs:284-302). The forward
// after the last kept token changes no output and is skipped.
size_t greedy(const Model& M, vector<float> logits, size_t position, Cache& cache, size_t max_new,
              const int32_t* stop, size_t nstop, int32_t* out, Trace tr, double first_seconds) {
  size_t count = 0;
  double step_seconds = first_seconds;
  while (count < max_new) {
    size_t token = argmax(logits.data(), logits.size());
    if (tr.logits) memcpy(tr.logits + count * logits.size(), logits.data(), logits.size() * 4);
    if (tr.gaps) tr.gaps[count] = top_gap(logits.data(), logits.size());
    if (tr.seconds) tr.seconds[count] = step_seconds;
    bool stopped = false;
    for (size_t s = 0; s < nstop; ++s) stopped |= (size_t)stop[s] == token;
    if (stopped) break;
    out[count++] = (int32_t)token;
    if (count == max_new) break;
    int32_t id = (int32_t)token;
    auto t0 = std::chrono::steady_clock::now();
    logits = forward_rows(M, embed(M, &id, 1), position + count - 1, cache);
    step_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  }
  return count;
}

Cache empty_cache(const Model& M) {
  Cache c;
  c.keys.resize(M.c.layers);
  c.values.resize(M.c.layers);
  return c;
}

template <class F>
auto guarded(F f, decltype(f()) failed) -> decltype(f()) {
  g_error.clear();
  try {
    return f();
  } catch (const std::exception& e) {
    g_error = e.what();
    return failed;
  }
}

}  // namespace

// ------------------------------------------------------------ C ABI ----
extern "C" {

const char* oracle_last_error() { return g_error.c_str(); }
const char* oracle_isa() { return isa_name(); }
void oracle_force_scalar(int on) { g_force_scalar = on != 0; }
int oracle_threads() { return omp_get_max_threads(); }
void oracle_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

void* oracle_load(const char* dir, int kv_f16) {
  return guarded([&]() -> void* {
    auto m = load_model(dir);
    m->kv_f16 = kv_f16 != 0;
    return m.release();
  }, nullptr);
}
void oracle_free(void* h) { delete (Model*)h; }

int64_t oracle_vocab(void* h) { return (int64_t)((Model*)h)->c.vocab; }
int64_t oracle_width(void* h) { return (int64_t)((Model*)h)->c.d; }
int64_t oracle_layers(void* h) { return (int64_t)((Model*)h)->c.layers; }

// CausalLm::prefix (src/models/parts/causal_lm.rs:202-215).
void* oracle_prefix(void* h, const int32_t* ids, size_t n) {
  return guarded([&]() -> void* {
    const Model& M = *(Model*)h;
    auto p = std::make_unique<Prefix>();
    p->tokens.assign(ids, ids + n);
    p->cache = empty_cache(M);
    if (n) forward_rows(M, embed(M, ids, n), 0, p->cache);
    return p.release();
  }, nullptr);
}
void oracle_prefix_free(void* p) { delete (Prefix*)p; }

// CausalLm::generate (src/models/parts/causal_lm.rs:217-249).
int64_t oracle_generate(void* h, void* prefix, const int32_t* prompt, size_t n, int64_t max_new,
                        const int32_t* stop, size_t nstop, int32_t* out, float* logits, float* gaps,
                        double* seconds, double* prefill_seconds) {
  return guarded([&]() -> int64_t {
    const Model& M = *(Model*)h;
    if (n == 0) throw std::runtime_error("empty prompt");
    const Prefix* p = (const Prefix*)prefix;
    bool use = p && n > p->tokens.size() &&
               std::equal(p->tokens.begin(), p->tokens.end(), prompt);
    size_t done = use ? p->tokens.size() : 0;
    Cache cache = use ? p->cache : empty_cache(M);
    auto t0 = std::chrono::steady_clock::now();
    vector<float> lg = forward_rows(M, embed(M, prompt + done, n - done), done, cache);
    double pf = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (prefill_seconds) *prefill_seconds = pf;
    return (int64_t)greedy(M, lg, n, cache, (size_t)max_new, stop, nstop, out,
                           Trace{logits, gaps, seconds}, pf);
  }, -1);
}

// CausalLm::generate_rows (src/models/parts/causal_lm.rs:251-262).
int64_t oracle_generate_rows(void* h, const float* rows, size_t nrows, int64_t max_new,
                             const int32_t* stop, size_t nstop, int32_t* out, float* logits,
                             float* gaps) {
  return guarded([&]() -> int64_t {
    const Model& M = *(Model*)h;
    if (nrows == 0) throw std::runtime_error("no rows");
    Cache cache = empty_cache(M);
    vector<float> x(rows, rows + nrows * M.c.d);
    vector<float> lg = forward_rows(M, x, 0, cache);
    return (int64_t)greedy(M, lg, nrows, cache, (size_t)max_new, stop, nstop, out,
                           Trace{logits, gaps, nullptr}, 0.0);
  }, -1);
}

// CausalLm::answer (src/models/parts/causal_lm.rs:264-282).
int64_t oracle_answer(void* h, const int32_t* head, size_t nhead, const float* audio, size_t naudio,
                      const int32_t* tail, size_t ntail, int64_t max_new, const int32_t* stop,
                      size_t nstop, int32_t* out, float* logits, float* gaps) {
  return guarded([&]() -> int64_t {
    const Model& M = *(Model*)h;
    size_t d = M.c.d;
    vector<float> rows;
    vector<float> a = embed(M, head, nhead);
    rows.insert(rows.end(), a.begin(), a.end());
    rows.insert(rows.end(), audio, audio + naudio * d);
    vector<float> b = embed(M, tail, ntail);
    rows.insert(rows.end(), b.begin(), b.end());
    Cache cache = empty_cache(M);
    size_t length = rows.size() / d;
    if (!length) throw std::runtime_error("no rows");
    vector<float> lg = forward_rows(M, rows, 0, cache);
    return (int64_t)greedy(M, lg, length, cache, (size_t)max_new, stop, nstop, out,
                           Trace{logits, gaps, nullptr}, 0.0);
  }, -1);
}

// CausalLm::set_ffn_scales (causal_lm.rs:305-307): [layers][d], or NULL
// to clear.
void oracle_set_ffn_scales(void* h, const float* scales) {
  Model& M = *(Model*)h;
  M.ffn_scales.clear();
  if (!scales) return;
  for (size_t l = 0; l < M.c.layers; ++l) M.ffn_scales.emplace_back(scales + l * M.c.d, scales + (l + 1) * M.c.d);
}

// CausalLm::generate_additive (causal_lm.rs:317-345): the prompt's
// embeddings plus audio rows 0..n, then each new token's embedding plus
// the next row, until a stop token or the rows end.
int64_t oracle_generate_additive(void* h, const int32_t* prompt, size_t n, const float* audio, size_t rows,
                                 const int32_t* stop, size_t nstop, int32_t* out, float* logits) {
  return guarded([&]() -> int64_t {
    const Model& M = *(Model*)h;
    const size_t d = M.c.d, V = M.c.vocab;
    if (n == 0 || rows < n) return (int64_t)0;
    auto stopped = [&](size_t t) {
      for (size_t s = 0; s < nstop; ++s)
        if ((size_t)stop[s] == t) return true;
      return false;
    };
    Cache cache = empty_cache(M);
    vector<float> x = embed(M, prompt, n);
    for (size_t i = 0; i < n * d; ++i) x[i] = x[i] + audio[i];
    vector<float> lg = forward_rows(M, x, 0, cache);
    size_t token = argmax(lg.data(), V), count = 0;
    if (logits) memcpy(logits, lg.data(), V * 4);
    for (size_t position = n; position < rows; ++position) {
      if (stopped(token)) return (int64_t)count;
      out[count++] = (int32_t)token;
      int32_t id = (int32_t)token;
      vector<float> e = embed(M, &id, 1);
      for (size_t i = 0; i < d; ++i) e[i] = e[i] + audio[position * d + i];
      lg = forward_rows(M, e, position, cache);
      token = argmax(lg.data(), V);
      if (logits) memcpy(logits + count * V, lg.data(), V * 4);
    }
    if (!stopped(token)) out[count++] = (int32_t)token;
    return (int64_t)count;
  }, -1);
}

// CausalLm::bidirectional_tokens (causal_lm.rs:393-408): one pass over all
// rows without the causal mask, then the best token of each row from
// `from` on. out: rows - from tokens.
int64_t oracle_bidirectional_tokens(void* h, const float* rows, size_t m, size_t from, int32_t* out) {
  return guarded([&]() -> int64_t {
    const Model& M = *(Model*)h;
    const size_t d = M.c.d, V = M.c.vocab;
    if (from > m) throw std::runtime_error("from is past the rows");
    Cache cache = empty_cache(M);
    vector<float> x(rows, rows + m * d);
    hidden(M, x, 0, cache, false);
    const Table& T = M.has_head ? M.head : M.embed;
    for (size_t r = from; r < m; ++r) {
      vector<float> row(x.begin() + r * d, x.begin() + (r + 1) * d);
      rms_in_place(row.data(), M.norm.data(), d, M.c.eps);
      vector<float> lg = table_forward(T, row.data(), 1);
      out[r - from] = (int32_t)argmax(lg.data(), V);
    }
    return (int64_t)(m - from);
  }, -1);
}

// CausalLm::embed (src/models/parts/causal_lm.rs:347-355).
int oracle_embed(void* h, const int32_t* ids, size_t n, float* out) {
  return guarded([&]() -> int {
    vector<float> x = embed(*(Model*)h, ids, n);
    memcpy(out, x.data(), x.size() * 4);
    return 0;
  }, -1);
}

// ---- op-level entry points (the op sweep and the unit checks) ----
uint16_t oracle_f32_to_f16(float v) { return f32_to_f16(v); }
float oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
float oracle_exp(float v) { return cephes_exp(v); }
float oracle_silu(float v) { return silu(v); }
void oracle_base3(uint8_t byte, uint8_t* out5) { base3_digits(byte, out5); }

void oracle_q8_0_quantize(const float* values, size_t count, int8_t* codes, uint16_t* scales) {
  q8_0_quantize(values, count, codes, scales);
}

void oracle_quantize(const float* x, size_t m, size_t k, size_t group, int half, int8_t* codes,
                     float* scales, int32_t* sums) {
  Quantized q = quantize_grouped(x, m, k, group, half != 0);
  memcpy(codes, q.values.data(), m * k);
  memcpy(scales, q.scales.data(), q.scales.size() * 4);
  memcpy(sums, q.sums.data(), q.sums.size() * 4);
}

// A W8A8 layer from raw parts: codes [n][k], scales [n][k/wgroup].
void* oracle_int_layer(const int8_t* codes, const float* scales, size_t n, size_t k, size_t group,
                       size_t wgroup, int half) {
  return guarded([&]() -> void* {
    auto L = std::make_unique<IntLayer>();
    L->n = n; L->k = k; L->group = group; L->wgroup = wgroup; L->half_scales = half != 0;
    L->codes.assign(codes, codes + n * k);
    L->scales.assign(scales, scales + n * (k / wgroup));
    pack_vnni(*L);
    return L.release();
  }, nullptr);
}
void oracle_int_layer_free(void* L) { delete (IntLayer*)L; }
int oracle_int_forward(void* L, const float* x, size_t m, float* out) {
  return guarded([&]() -> int {
    vector<float> y = int_forward(*(IntLayer*)L, x, m);
    memcpy(out, y.data(), y.size() * 4);
    return 0;
  }, -1);
}

void* oracle_table(const int8_t* codes, const float* scales, size_t n, size_t k) {
  auto t = std::make_unique<Table>();
  t->n = n; t->k = k;
  t->codes.assign(codes, codes + n * k);
  t->scales.assign(scales, scales + n * (k / 32));
  return t.release();
}
void oracle_table_free(void* t) { delete (Table*)t; }
void oracle_table_forward(void* t, const float* x, size_t m, float* out) {
  vector<float> y = table_forward(*(Table*)t, x, m);
  memcpy(out, y.data(), y.size() * 4);
}

void oracle_rmsnorm(float* row, const float* w, size_t d, float eps) { rms_in_place(row, w, d, eps); }

void oracle_attention(const float* q, size_t qs, const float* k, const float* v, size_t kvs, size_t tq,
                      size_t tk, size_t heads, size_t kv_heads, size_t hd, int causal, float* out) {
  attention(q, qs, k, v, kvs, tq, tk, heads, kv_heads, hd, causal != 0, out);
}

void oracle_rope(float* x, size_t rows, size_t stride, size_t heads, size_t hd, size_t first, float base) {
  Rotary r;
  r.init(hd, base);
  r.apply(x, rows, stride, heads, hd, first);
}

}  // extern "C"
