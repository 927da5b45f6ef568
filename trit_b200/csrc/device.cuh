// Device-side types and helpers shared by the layered kernels (prefill,
// batched decode) and the persistent batch-1 decode kernel.
//
// Exactness: the helpers below use the *_rn intrinsics wherever the
// reference performs a separate multiply or add, so that nvcc cannot fuse
// them; every fused multiply-add is an explicit __fmaf_rn where the
// reference's AVX-512 path uses _mm512_fmadd_ps.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "types.h"

namespace trit {

__device__ __forceinline__ size_t kv_offset(const DCache& c, const DConfig& cfg, int page, int layer,
                                            int which, int head, int tok) {
  return ((((size_t)page * cfg.layers + layer) * 2 + which) * cfg.kv_heads + head) * (size_t)c.page_tokens * cfg.hd +
         (size_t)tok * cfg.hd;
}

// ------------------------------------------------------------ numbers ----
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

// The Cephes exp of src/cpu/activation.rs:356-372 (AVX-512 form), step for
// step: clamp, n = rint(x*log2e), two fused reductions, Horner by fma,
// y = fma(p, r*r, r+1), times 2^n.
__device__ __forceinline__ float cephes_exp(float x) {
  const float LOG2E = 1.44269504088896340735992468100189214f;
  const float LN2_HI = 0.6933594f, LN2_LO = -2.1219444e-4f;
  x = fmaxf(x, -87.3f);
  x = fminf(x, 88.0f);
  int n_int = __float2int_rn(__fmul_rn(x, LOG2E));
  float n = (float)n_int;
  float r = __fmaf_rn(-n, LN2_HI, x);
  r = __fmaf_rn(-n, LN2_LO, r);
  float p = 1.9875691e-4f;  // fma(0, r, c0) = c0
  p = __fmaf_rn(p, r, 1.3981999e-3f);
  p = __fmaf_rn(p, r, 8.333452e-3f);
  p = __fmaf_rn(p, r, 4.1665796e-2f);
  p = __fmaf_rn(p, r, 0.16666665f);
  p = __fmaf_rn(p, r, 0.5f);
  float y = __fmaf_rn(p, __fmul_rn(r, r), __fadd_rn(r, 1.0f));
  return __fmul_rn(y, __int_as_float((n_int + 127) << 23));
}

// SiLU of src/cpu/activation.rs:330: v / (1 + exp(0 - v)), IEEE division.
__device__ __forceinline__ float silu(float v) {
  return __fdiv_rn(v, __fadd_rn(1.0f, cephes_exp(__fsub_rn(0.0f, v))));
}

// RmsNorm's sum of squares in the reference's order (layers.rs:137): one
// thread, v[0]^2 + v[1]^2 + ... left to right, each square rounded.
__device__ __forceinline__ float seq_sum_squares(const float* v, int n) {
  float s = 0.0f;
#pragma unroll 8
  for (int i = 0; i < n; ++i) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
  return s;
}

// seq_sum_squares with the loads run ahead: the next 16 values are loaded
// while the current 16 are squared and added, so the adds wait only on
// each other. The same sum, in the same order. v is 16-byte aligned.
__device__ __forceinline__ float seq_sum_squares_ahead(const float* v, int n) {
  const float4* p = (const float4*)v;
  const int nb = n / 16;
  float s = 0.0f;
  float4 a[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) a[u] = nb > 0 ? p[u] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int b = 0; b < nb; ++b) {
    float4 c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) c[u] = a[u];
    if (b + 1 < nb) {
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = p[4 * (b + 1) + u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s = __fadd_rn(s, __fmul_rn(c[u].x, c[u].x));
      s = __fadd_rn(s, __fmul_rn(c[u].y, c[u].y));
      s = __fadd_rn(s, __fmul_rn(c[u].z, c[u].z));
      s = __fadd_rn(s, __fmul_rn(c[u].w, c[u].w));
    }
  }
  for (int i = nb * 16; i < n; ++i) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
  return s;
}

// seq_sum with the loads run ahead as above: the same sum, in the same
// order. v is 16-byte aligned.
__device__ __forceinline__ float seq_sum_ahead(const float* v, int n) {
  const float4* p = (const float4*)v;
  const int nb = n / 16;
  float s = 0.0f;
  float4 a[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) a[u] = nb > 0 ? p[u] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int b = 0; b < nb; ++b) {
    float4 c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) c[u] = a[u];
    if (b + 1 < nb) {
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = p[4 * (b + 1) + u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s = __fadd_rn(s, c[u].x);
      s = __fadd_rn(s, c[u].y);
      s = __fadd_rn(s, c[u].z);
      s = __fadd_rn(s, c[u].w);
    }
  }
  for (int i = nb * 16; i < n; ++i) s = __fadd_rn(s, v[i]);
  return s;
}

// A sum left to right (the reference's f32 `sum()`), reading 4 values at a
// time so that only the adds wait on each other. v is 16-byte aligned.
__device__ __forceinline__ float seq_sum(const float* v, int n) {
  float s = 0.0f;
  int i = 0;
#pragma unroll 8
  for (; i + 4 <= n; i += 4) {
    float4 q = *(const float4*)(v + i);
    s = __fadd_rn(s, q.x);
    s = __fadd_rn(s, q.y);
    s = __fadd_rn(s, q.z);
    s = __fadd_rn(s, q.w);
  }
  for (; i < n; ++i) s = __fadd_rn(s, v[i]);
  return s;
}

// inv = 1 / sqrt(sum / d + eps), each step rounded (layers.rs:137).
__device__ __forceinline__ float rms_inv(float sum, int d, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)d), eps)));
}

// Packed f32x2 arithmetic (sm_100): two lanes a instruction, each rounded
// as the scalar operation (IEEE round to nearest even).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// ------------------------------------------------------------- warps ----
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------- quantizer ----
// Quantized::grouped for one group (src/cpu/kernels.rs:769-807): scale =
// max|x|/127 (1 for a zero group), codes = clamp(rint(x * (1/scale)),
// +-127); Q8_0 then rounds the scale to f16 (kernels.rs:721-725).
__device__ __forceinline__ float group_scale(float max) { return max > 0.0f ? __fdiv_rn(max, 127.0f) : 1.0f; }
__device__ __forceinline__ int quantize_value(float v, float inv) {
  int c = __float2int_rn(__fmul_rn(v, inv));
  return max(-127, min(127, c));
}

// A warp quantizes one group of `G` values (32 or 128) held as `G/32`
// values per lane (lane l holds values l*(G/32) .. +G/32-1). Writes the
// codes, returns the (optionally f16-rounded) scale in every lane.
template <int G>
__device__ __forceinline__ float warp_quantize_group(const float (&v)[G / 32], int8_t* codes, bool half) {
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < G / 32; ++i) m = fmaxf(m, fabsf(v[i]));
  m = warp_max(m);
  float scale = group_scale(m);
  float inv = __fdiv_rn(1.0f, scale);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < G / 32; ++i) codes[lane * (G / 32) + i] = (int8_t)quantize_value(v[i], inv);
  return half ? round_f16(scale) : scale;
}

// Quantized::grouped of k values (kernels.rs:769-807) by a block of NT
// threads, every group at once: thread t takes VPT (4 or 8) consecutive
// values from VPT * t (then VPT * (t + NT) ...), and the G / VPT threads of
// a group (G = 32 or 128) share its max by shuffles. Each value is src[i],
// times inv * w[i] when w is given (RmsNorm, layers.rs:135-144), times sc[i]
// when sc is given. Codes to q, scales to s (f16-rounded when `half`). The
// max of a group does not depend on the order it is taken in, so the codes
// and scales are those of warp_quantize_group. src, q: 16- and VPT-byte
// aligned; k a multiple of G.
template <int NT, int VPT = 8>
__device__ __forceinline__ void quantize_groups(const float* src, int k, const float* w, const float* sc, float inv,
                                                int G, bool half, int8_t* q, float* s) {
  const int lanes = G / VPT;
  for (int base = 0; base < k; base += VPT * NT) {
    const int i0 = base + VPT * threadIdx.x;
    const bool live = i0 < k;
    float v[VPT];
    float m = 0.0f;
    if (live) {
#pragma unroll
      for (int j = 0; j < VPT; j += 4) {
        const float4 a = *(const float4*)(src + i0 + j);
        v[j] = a.x; v[j + 1] = a.y; v[j + 2] = a.z; v[j + 3] = a.w;
      }
      if (w) {
#pragma unroll
        for (int i = 0; i < VPT; ++i) v[i] = __fmul_rn(v[i], __fmul_rn(inv, w[i0 + i]));
      }
      if (sc) {
#pragma unroll
        for (int i = 0; i < VPT; ++i) v[i] = __fmul_rn(v[i], sc[i0 + i]);
      }
#pragma unroll
      for (int i = 0; i < VPT; ++i) m = fmaxf(m, fabsf(v[i]));
    }
    for (int o = 1; o < lanes; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (live) {
      const float scale = group_scale(m);
      const float r = __fdiv_rn(1.0f, scale);
#pragma unroll
      for (int j = 0; j < VPT; j += 4) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) word |= (uint32_t)(uint8_t)quantize_value(v[j + i], r) << (8 * i);
        *(uint32_t*)(q + i0 + j) = word;
      }
      if ((threadIdx.x & (lanes - 1)) == 0) s[i0 / G] = half ? round_f16(scale) : scale;
    }
  }
}

// ------------------------------------------------------------ loads ----
__device__ __forceinline__ int4 ld_stream(const void* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Hint the L2 to fetch [p, p+bytes): no completion, no visible effect.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  const char* c = (const char*)p;
  // The bulk prefetch wants 16-byte alignment and a multiple of 16 bytes.
  uintptr_t a = (uintptr_t)c;
  uintptr_t start = a & ~(uintptr_t)15;
  uintptr_t stop = (a + bytes + 15) & ~(uintptr_t)15;
  for (uintptr_t at = start; at < stop; at += 32768) {
    uint32_t n = (uint32_t)((stop - at) < 32768 ? (stop - at) : 32768);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(at), "r"(n) : "memory");
  }
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// The i32 dot of 16 weight bytes and 16 activation bytes (ternary: 16
// two-bit codes in one word, pack_span layout, minus one).
__device__ __forceinline__ int dot16(int4 w, int4 x) {
  int s = dp4a(w.x, x.x, 0);
  s = dp4a(w.y, x.y, s);
  s = dp4a(w.z, x.z, s);
  return dp4a(w.w, x.w, s);
}
__device__ __forceinline__ int dot16_ternary(uint32_t word, int4 x) {
  // Bits 2s..2s+1 of byte j hold the code of k = 4s + j (pack_span,
  // src/cpu/kernels.rs:618-628); codes 0..2 stand for -1..+1.
  int s = 0;
  s = dp4a((int)__vsub4(word & 0x03030303u, 0x01010101u), x.x, s);
  s = dp4a((int)__vsub4((word >> 2) & 0x03030303u, 0x01010101u), x.y, s);
  s = dp4a((int)__vsub4((word >> 4) & 0x03030303u, 0x01010101u), x.z, s);
  s = dp4a((int)__vsub4((word >> 6) & 0x03030303u, 0x01010101u), x.w, s);
  return s;
}

// The weight scale of output `row` for activation group `g`.
__device__ __forceinline__ float weight_scale(const DMat& W, int row, int g) {
  if (W.kind == kQ8_0) {
    const uint16_t* s = (const uint16_t*)W.scales;
    return f16_bits_to_f32(s[(size_t)row * (W.k / 32) + g]);
  }
  if (W.kind == kInt8Row) return ((const float*)W.scales)[row];
  return ((const float*)W.scales)[(size_t)row * (W.k / 128) + g];
}

__device__ __forceinline__ float table_scale(const DTable& T, int row, int g) {
  if (T.scale_f16) return f16_bits_to_f32(((const uint16_t*)T.scales)[(size_t)row * (T.k / 32) + g]);
  return ((const float*)T.scales)[(size_t)row * (T.k / 32) + g];
}

// Byte b of a word as an exact f32 (-128..127): 2^23 + (b ^ 0x80) built
// by a byte permute, minus 2^23 + 128.
__device__ __forceinline__ float byte_to_float(uint32_t word_xor80, int b) {
  uint32_t bits = __byte_perm(word_xor80, 0x4B000000u, 0x7650 + b - 0) ;
  return __fsub_rn(__uint_as_float(bits), 8388736.0f);
}

}  // namespace trit
