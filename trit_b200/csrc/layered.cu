// The layered path: one kernel per step of CausalLm::hidden
// (src/models/parts/causal_lm.rs:410-481) over `m` rows, each row with its
// own stream and position. It runs prefill (one stream, many positions),
// batched decode (many streams, one position each) and, as a fallback,
// batch-1 decode.
#include <algorithm>
#include <cstdio>

#include "attention.cuh"
#include "device.cuh"
#include "kernels.h"

namespace trit {

// --------------------------------------------------------- embedding ----
// Dense::row of a token table (src/cpu/gemm.rs:412-429): code * scale, then
// the embedding multiplier of CausalLm::hidden (causal_lm.rs:415).
__global__ void k_embed(DTable T, const int* ids, int m, float* x, float mult) {
  int r = blockIdx.x;
  if (r >= m) return;
  int id = ids[r];
  if (id < 0 || id >= T.n) id = 0;  // the host checks ids; this keeps the read in bounds
  for (int kk = threadIdx.x; kk < T.k; kk += blockDim.x) {
    float v = __fmul_rn((float)T.codes[(size_t)id * T.k + kk], table_scale(T, id, kk / 32));
    if (mult != 1.0f) v = __fmul_rn(v, mult);
    x[(size_t)r * T.k + kk] = v;
  }
}

__global__ void k_scale(float* x, size_t n, float mult) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = __fmul_rn(x[i], mult);
}

// ------------------------------------------------- norm + quantize ----
// Dynamic shared memory of the norm kernels: the 48 KB a launch may take
// without an opt-in, less room for their static shared variables.
constexpr size_t kNormSmem = 48 * 1024 - 256;

// RmsNorm::apply (src/layers.rs:135-153) then Quantized::grouped
// (src/cpu/kernels.rs:661-737) of the normed row. One thread of a block
// sums the row's squares in order, as the reference does, so the result is
// the reference's to the bit.
// With `squares`, the squares are formed by all threads into shared memory
// first (each rounded, as the reference rounds them), so the one thread's
// chain is adds only. A row's groups spread over `gridDim.y` blocks (decode
// batches: few rows); each block sums the whole row (the same chain, so the
// same inv) and quantizes its own groups. With `wstage`, the block's slice
// of the norm weights loads with the row, so its latency hides behind the
// sum.
template <int G>
__global__ void __launch_bounds__(256) k_norm_quant(const float* x, int d, const float* w, float eps, int half,
                                                    int8_t* xq, float* xs, const float* sc, int squares, int wstage) {
  extern __shared__ __align__(16) float rowv[];  // [d], then [d] squares, then the weights of the block's groups
  float* sq = rowv + d;
  float* wv = sq + (squares ? d : 0);
  const int r = blockIdx.x, groups = d / G;
  const int per = (groups + gridDim.y - 1) / gridDim.y;
  const int g0 = blockIdx.y * per, g1 = min(groups, g0 + per);
  const float* row = x + (size_t)r * d;
  __shared__ float s_inv;
  for (int i = threadIdx.x; i < d; i += 256) {
    const float v = row[i];
    rowv[i] = v;
    if (squares) sq[i] = __fmul_rn(v, v);
  }
  if (w && wstage)
    for (int i = g0 * G + threadIdx.x; i < g1 * G; i += 256) wv[i - g0 * G] = w[i];
  __syncthreads();
  if (threadIdx.x == 0)
    s_inv = !w ? 1.0f : rms_inv(squares ? seq_sum_ahead(sq, d) : seq_sum_squares_ahead(rowv, d), d, eps);
  __syncthreads();
  float inv = s_inv;
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int g = g0 + warp; g < g1; g += 8) {
    float v[G / 32];
#pragma unroll
    for (int i = 0; i < G / 32; ++i) {
      int kk = g * G + lane * (G / 32) + i;
      v[i] = w ? __fmul_rn(rowv[kk], __fmul_rn(inv, wstage ? wv[kk - g0 * G] : w[kk])) : rowv[kk];
      if (sc) v[i] = __fmul_rn(v[i], sc[kk]);
    }
    float scale = warp_quantize_group<G>(v, xq + (size_t)r * d + g * G, half);
    if (lane == 0) xs[(size_t)r * groups + g] = scale;
  }
}

// ------------------------------------------------------ W8A8 product ----
// Int8::forward_biased (src/cpu/int8.rs:425-483), VNNI float order
// (:560-570): per output and frame, acc = fma(f32(dot_g), ws_g * xs_g, acc)
// over the groups in order. The i32 group dots come from dp4a over
// coalesced 16-byte loads (a warp per output row); the group chain runs
// in order in one thread per (row, frame), so each output is the
// reference's value bit for bit.
//
// Units: OUT/RESID: a unit is one output row. SILU: a unit j is the pair of
// gate row j and up row ffn + j of a stacked gate_up layer, and the output
// is h[j] = silu(gate) * up (causal_lm.rs:464-474).
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_ROWS = 8;   // output rows per block
constexpr int GEMV_FRAMES = 8; // frames per pass

__device__ __forceinline__ int4 load_weights16(const DMat& W, int row, int chunk) {
  if (W.kind == kTernary) {
    uint32_t word = ((const uint32_t*)W.codes)[(size_t)row * (W.k / 16) + chunk];
    return make_int4((int)word, 0, 0, 0);
  }
  return __ldg((const int4*)((const int8_t*)W.codes + (size_t)row * W.k) + chunk);
}

__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(DMat W, const int8_t* xq, const float* xs, int m, int mode,
                                                        float* y, int ldy, float resid_mult, int units) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int k = W.k, groups = k / W.agroup;
  const int rows_per_unit = (mode == kEpSilu) ? 2 : 1;
  const int units_per_block = GEMV_ROWS / rows_per_unit;
  const int unit0 = blockIdx.x * units_per_block;
  const int nunits = min(units_per_block, units - unit0);
  int8_t* act = (int8_t*)smem;                                      // [F][k]
  float* act_s = (float*)(smem + GEMV_FRAMES * k);                  // [F][groups]
  int* part = (int*)(act_s + GEMV_FRAMES * groups);                 // [ROWS][F][groups]
  float* res = (float*)(part + GEMV_ROWS * GEMV_FRAMES * groups);   // [ROWS][F]
  float* wsc = res + GEMV_ROWS * GEMV_FRAMES;                        // [ROWS][groups]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = k / 16;            // 16 k-values per lane-load
  const int lanes_per_group = W.agroup / 16;
  // The weight scales of the block's rows, once (coalesced per row).
  for (int i = threadIdx.x; i < nunits * rows_per_unit * groups; i += GEMV_THREADS) {
    int lr = i / groups, g = i % groups;
    int u = unit0 + lr / rows_per_unit;
    int row = (mode == kEpSilu) ? u + (lr % 2) * units : u;
    wsc[i] = weight_scale(W, row, g);
  }
  for (int f0 = 0; f0 < m; f0 += GEMV_FRAMES) {
    const int nf = min(GEMV_FRAMES, m - f0);
    __syncthreads();
    for (int i = threadIdx.x; i < nf * k / 16; i += GEMV_THREADS)
      ((int4*)act)[i] = ((const int4*)(xq + (size_t)f0 * k))[i];
    for (int i = threadIdx.x; i < nf * groups; i += GEMV_THREADS) act_s[i] = xs[(size_t)f0 * groups + i];
    __syncthreads();
    // Group dots: warp w takes local rows w, w + 8, ...
    for (int lr = warp; lr < nunits * rows_per_unit; lr += GEMV_THREADS / 32) {
      int u = unit0 + lr / rows_per_unit;
      int row = (mode == kEpSilu) ? u + (lr % 2) * units : u;
      for (int c = lane; c < chunks + ((32 - chunks % 32) % 32); c += 32) {
        bool live = c < chunks;
        int4 w = live ? load_weights16(W, row, c) : make_int4(0, 0, 0, 0);
        for (int f = 0; f < nf; ++f) {
          int dot = 0;
          if (live) {
            int4 a = ((const int4*)(act + f * k))[c];
            dot = (W.kind == kTernary) ? dot16_ternary((uint32_t)w.x, a) : dot16(w, a);
          }
          for (int o = 1; o < lanes_per_group; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
          if (live && (lane % lanes_per_group) == 0) part[(lr * GEMV_FRAMES + f) * groups + c / lanes_per_group] = dot;
        }
      }
    }
    __syncthreads();
    // Chains: one thread per (local row, frame), groups in order.
    for (int t = threadIdx.x; t < nunits * rows_per_unit * nf; t += GEMV_THREADS) {
      int lr = t / nf, f = t % nf;
      const int* p = part + (lr * GEMV_FRAMES + f) * groups;
      const float* sx = act_s + f * groups;
      float acc = 0.0f;
      const float* wr = wsc + lr * groups;
      for (int g = 0; g < groups; ++g) acc = __fmaf_rn((float)p[g], __fmul_rn(wr[g], sx[g]), acc);
      res[lr * GEMV_FRAMES + f] = acc;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < nunits * nf; t += GEMV_THREADS) {
      int lu = t / nf, f = t % nf;
      int u = unit0 + lu;
      size_t at = (size_t)(f0 + f) * ldy + u;
      if (mode == kEpOut) {
        y[at] = res[lu * GEMV_FRAMES + f];
      } else if (mode == kEpResid) {
        float o = res[lu * GEMV_FRAMES + f];
        y[at] = (resid_mult == 1.0f) ? __fadd_rn(y[at], o) : __fadd_rn(y[at], __fmul_rn(resid_mult, o));
      } else {
        float g = res[(2 * lu) * GEMV_FRAMES + f], up = res[(2 * lu + 1) * GEMV_FRAMES + f];
        y[at] = __fmul_rn(silu(g), up);
      }
    }
  }
}

// The W8A8 product for decode-size batches (Int8::forward_biased,
// src/cpu/int8.rs:425-483, VNNI float order :560-570). A warp owns one
// output row; a row is cut into 32-byte slots (32 int8 codes, or 32
// two-bit ternary codes in two words), lane l taking slots l, l + 32, ...
// Each weight slot is loaded once and multiplied with the codes of every
// frame of the pass (FR frames, staged in shared memory). A Q8_0 group is
// one slot; a 128-value group is four slots of neighbouring lanes, summed
// with two shuffles. The exact i32 group dots go to shared memory as f32;
// then one thread per (row, frame) runs the chain acc = fma(f32(dot_g),
// ws_g * xs_g, acc) over the groups in order, so each output is the
// reference's value bit for bit.
constexpr int GS_WARPS = 8;

template <int FR>
__global__ void __launch_bounds__(GS_WARPS * 32) k_gemv_slots(DMat W, const int8_t* xq, const float* xs, int m,
                                                            int mode, float* y, int ldy, float resid_mult,
                                                            int units) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int k = W.k, G = W.agroup, groups = k / G, slots = k / 32;
  const int rows_per_unit = (mode == kEpSilu) ? 2 : 1;
  const int units_per_block = GS_WARPS / rows_per_unit;
  const int ntiles = (units + units_per_block - 1) / units_per_block;
  // Frames' codes as [FR][2][slots] 16-byte halves: the lanes of a warp
  // read consecutive 16-byte words (no bank conflicts). Group dots as
  // [GS_WARPS][FR][groups + 1]: the padding keeps both the writes (lanes
  // by group) and the chain reads (threads by frame) conflict-free.
  const int gp = groups + 1;
  int4* act = (int4*)smem;                                 // [FR][2][slots]
  float* axs = (float*)(smem + (size_t)FR * k);            // [FR][groups]
  float* pdot = axs + FR * groups;                         // [GS_WARPS][FR][gp]
  float* wsc = pdot + GS_WARPS * FR * gp;                  // [GS_WARPS][groups]
  float* res = wsc + GS_WARPS * groups;                    // [GS_WARPS][FR]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool ternary = W.kind == kTernary;
  for (int f0 = 0; f0 < m; f0 += FR) {
    const int nf = min(FR, m - f0);
    __syncthreads();
    for (int i = threadIdx.x; i < nf * k / 16; i += GS_WARPS * 32) {
      const int f = i / (k / 16), c = i - f * (k / 16);
      act[(f * 2 + (c & 1)) * slots + (c >> 1)] = ((const int4*)(xq + (size_t)f0 * k))[i];
    }
    for (int i = threadIdx.x; i < nf * groups; i += GS_WARPS * 32) axs[i] = xs[(size_t)f0 * groups + i];
    // The block's row tiles, the frames staged once for all of them.
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int unit0 = tile * units_per_block;
      const int nunits = min(units_per_block, units - unit0);
      const int nrows = nunits * rows_per_unit;
      auto row_of = [&](int lr) {
        const int u = unit0 + lr / rows_per_unit;
        return (mode == kEpSilu) ? u + (lr % 2) * units : u;
      };
      __syncthreads();  // the tile before is done with wsc, pdot and res
      for (int i = threadIdx.x; i < nrows * groups; i += GS_WARPS * 32)
        wsc[i] = weight_scale(W, row_of(i / groups), i % groups);
      if (warp < nrows) {
        const int row = row_of(warp);
        const int8_t* wrow = (const int8_t*)W.codes + (size_t)row * k;      // int8 codes
        const uint2* trow = (const uint2*)W.codes + (size_t)row * (k / 32);  // ternary: two words a slot
#pragma unroll 2
        for (int s0 = 0; s0 < slots; s0 += 32) {
          const int sl = s0 + lane;
          const bool live = sl < slots;
          int4 w0 = make_int4(0, 0, 0, 0), w1 = make_int4(0, 0, 0, 0);
          uint2 tw = make_uint2(0, 0);
          if (live) {
            if (ternary) tw = __ldg(trow + sl);
            else {
              w0 = __ldg((const int4*)(wrow + sl * 32));
              w1 = __ldg((const int4*)(wrow + sl * 32 + 16));
            }
          }
          int dot[FR];
#pragma unroll
          for (int f = 0; f < FR; ++f) {
            dot[f] = 0;
            if (live && f < nf) {
              const int4 a0 = act[(f * 2) * slots + sl];
              const int4 a1 = act[(f * 2 + 1) * slots + sl];
              dot[f] = ternary ? dot16_ternary(tw.x, a0) + dot16_ternary(tw.y, a1) : dot16(w0, a0) + dot16(w1, a1);
            }
          }
          if (G == 128) {
#pragma unroll
            for (int f = 0; f < FR; ++f) {
              dot[f] += __shfl_xor_sync(0xffffffffu, dot[f], 1);
              dot[f] += __shfl_xor_sync(0xffffffffu, dot[f], 2);
            }
          }
          if (live && (G == 32 || (lane & 3) == 0)) {
            const int g = (sl * 32) / G;
            float* pd = pdot + (size_t)warp * FR * gp + g;
#pragma unroll
            for (int f = 0; f < FR; ++f)
              if (f < nf) pd[f * gp] = __int2float_rn(dot[f]);
          }
        }
      }
      __syncthreads();
      // The chains: one thread per (row, frame), groups in order.
      for (int t = threadIdx.x; t < nrows * nf; t += GS_WARPS * 32) {
        const int lr = t / nf, f = t - lr * nf;
        const float* pd = pdot + ((size_t)lr * FR + f) * gp;
        const float* ws = wsc + lr * groups;
        const float* sx = axs + f * groups;
        float acc = 0.0f;
#pragma unroll 8
        for (int g = 0; g < groups; ++g) acc = __fmaf_rn(pd[g], __fmul_rn(ws[g], sx[g]), acc);
        res[lr * FR + f] = acc;
      }
      __syncthreads();
      for (int t = threadIdx.x; t < nunits * nf; t += GS_WARPS * 32) {
        const int lu = t / nf, f = t - lu * nf;
        const int u = unit0 + lu;
        const size_t at = (size_t)(f0 + f) * ldy + u;
        if (mode == kEpOut) {
          y[at] = res[lu * FR + f];
        } else if (mode == kEpResid) {
          const float o = res[lu * FR + f];
          y[at] = (resid_mult == 1.0f) ? __fadd_rn(y[at], o) : __fadd_rn(y[at], __fmul_rn(resid_mult, o));
        } else {
          const float g = res[(2 * lu) * FR + f], up = res[(2 * lu + 1) * FR + f];
          y[at] = __fmul_rn(silu(g), up);
        }
      }
    }
  }
}

size_t gemv_slots_smem(const DMat& W, int fr) {
  const size_t groups = W.k / W.agroup;
  return (size_t)fr * W.k + (size_t)fr * groups * 4 + (size_t)GS_WARPS * (groups + 1) * fr * 4 +
         GS_WARPS * groups * 4 + GS_WARPS * fr * 4;
}

size_t gemv_smem(const DMat& W) {
  size_t groups = W.k / W.agroup;
  return GEMV_FRAMES * (size_t)W.k + GEMV_FRAMES * groups * 4 + GEMV_ROWS * GEMV_FRAMES * groups * 4 +
         GEMV_ROWS * GEMV_FRAMES * 4 + GEMV_ROWS * groups * 4;
}

// ------------------------------------------- q/k norm, RoPE, KV append ----
// causal_lm.rs:428-446: per-head RMSNorm of q and k (Qwen3), the halves
// rotation of layers.rs:317-333 with the host's sin/cos table, Granite's
// q scale, then K and V appended to the stream's pages. One block per
// row, one warp per head; lane l holds values 4l..4l+3 of the head, so the
// rotation partner of value i (i + 64) sits in lane l ^ 16.
__global__ void __launch_bounds__(256) k_qk_rope_append(float* qkv, int m, DConfig cfg, const float* q_norm,
                                                        const float* k_norm, const float* rope, int rope_rows,
                                                        DCache cache, const int* row_stream, const int* row_pos,
                                                        int layer) {
  __shared__ __align__(16) float headv[8][128];
  int r = blockIdx.x;
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = cfg.heads * cfg.hd, kvd = cfg.kv_heads * cfg.hd, stride = qd + 2 * kvd;
  int pos = row_pos[r], stream = row_stream[r];
  float* row = qkv + (size_t)r * stride;
  const int half = cfg.hd / 2;
  const float* sn = rope + (size_t)min(pos, rope_rows - 1) * cfg.hd;  // [sin(half) | cos(half)]
  const float* cs = sn + half;
  for (int h = warp; h < cfg.heads + 2 * cfg.kv_heads; h += blockDim.x / 32) {
    bool is_q = h < cfg.heads, is_k = !is_q && h < cfg.heads + cfg.kv_heads;
    float* head = row + h * cfg.hd;  // q heads, then k heads, then v heads
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = head[lane * 4 + i];
    if (is_q || is_k) {
      const float* nw = is_q ? q_norm : k_norm;
      if (nw) {
        // The head's sum of squares in order (layers.rs:137), by lane 0.
#pragma unroll
        for (int i = 0; i < 4; ++i) headv[warp][lane * 4 + i] = v[i];
        __syncwarp();
        float inv = 0.0f;
        if (lane == 0) inv = rms_inv(seq_sum_squares_ahead(headv[warp], cfg.hd), cfg.hd, cfg.eps);
        inv = __shfl_sync(0xffffffffu, inv, 0);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], __fmul_rn(inv, nw[lane * 4 + i]));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
        int idx = (lane & 15) * 4 + i;  // pair index
        float c = cs[idx], s = sn[idx];
        if (lane < 16) v[i] = __fsub_rn(__fmul_rn(v[i], c), __fmul_rn(partner, s));
        else v[i] = __fadd_rn(__fmul_rn(v[i], c), __fmul_rn(partner, s));
      }
      if (is_q && cfg.has_q_scale) {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], cfg.q_scale);
      }
    }
    if (is_q) {
#pragma unroll
      for (int i = 0; i < 4; ++i) head[lane * 4 + i] = v[i];
    } else {
      int kvh = is_k ? h - cfg.heads : h - cfg.heads - cfg.kv_heads;
      int page = cache.page_table[(size_t)stream * cache.pages_per_stream + pos / cache.page_tokens];
      size_t off = kv_offset(cache, cfg, page, layer, is_k ? 0 : 1, kvh, pos % cache.page_tokens) + lane * 4;
      if (cache.f16) {
        __half* dst = (__half*)cache.pool + off;
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = __float2half_rn(v[i]);
      } else {
        float* dst = (float*)cache.pool + off;
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = v[i];
      }
      if (is_k) {
#pragma unroll
        for (int i = 0; i < 4; ++i) head[lane * 4 + i] = v[i];
      }
    }
  }
}

// ---------------------------------------------------------- attention ----
// Attention of a tile of rows of one stream at consecutive positions (a
// prompt chunk; a decode step is a tile of one row), every row and query
// head in the reference's order as Attention::run computes it: row i of the
// tile (position p0 + i) sees keys [0, p0 + i + 1), or [0, all_keys) when
// all_keys > 0 (no causal mask). Keys and values are staged once for all
// the tile's rows, 128 at a time. Scores: a thread keeps a QB x KB block of
// (query head, key) chains, each an fma chain over the head dimension in
// order; outputs: a thread keeps DW (query head, dimension) chains, each an
// fma chain over the keys in order. The scores of the tile's RQ query heads
// stay in shared memory, [RQ][tmax]. tiles[b] = {first row, rows}, or
// null for one row per block.
constexpr int AR_KT = 128;  // keys staged at a time

template <int QB, int KB, int DW>
__global__ void __launch_bounds__(256) k_attention_rows(const float* qkv, const int2* tiles, DConfig cfg, DCache cache,
                                                        const int* row_stream, const int* row_pos, int layer, int tmax,
                                                        int all_keys, float* att) {
  extern __shared__ __align__(16) float sm[];
  const int kvh = blockIdx.y, t = threadIdx.x;
  const int2 tile = tiles ? tiles[blockIdx.x] : make_int2(blockIdx.x, 1);
  const int r0 = tile.x, R = tile.y;
  const int qpk = cfg.heads / cfg.kv_heads, qd = cfg.heads * 128, stride = qd + 2 * cfg.kv_heads * 128;
  const int RQ = R * qpk;
  const bool f16 = cache.f16;
  const int pitch = f16 ? 68 : 132;           // floats a staged row (16-byte aligned, banks staggered)
  float* q = sm;                              // [RQ][128]
  float* sc = q + RQ * 128;                   // [RQ][tmax]
  float* kvb[2] = {sc + (size_t)RQ * tmax,   // [2][AR_KT][pitch]: tile t in buffer t % 2
                   sc + (size_t)RQ * tmax + AR_KT * pitch};
  float* inv = kvb[1] + AR_KT * pitch;        // [RQ]
  const int stream = row_stream[r0];
  const int p0 = row_pos[r0];
  const int T = all_keys > 0 ? all_keys : p0 + R;  // keys the last row sees
  auto visible = [&](int qh) { return all_keys > 0 ? all_keys : p0 + qh / qpk + 1; };
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
  for (int i = t; i < RQ * 128; i += 256) {
    int qh = i / 128, e = i % 128, r = qh / qpk, h = qh % qpk;
    q[i] = __fmul_rn(qkv[(size_t)(r0 + r) * stride + (kvh * qpk + h) * 128 + e], scale);
  }
  // Keys (which 0) or values (1) [j0, j0 + n) into kv, row pitch `pitch` floats.
  // Keys (which 0) or values (1) [j0, j0 + n) into dst (cp.async, one
  // commit group; the caller waits).
  // A thread's chunks walk the rows in order, so the page's base address
  // is worked out only when a row starts a new page.
  auto stage = [&](int which, int j0, int n, float* dst) {
    const int cshift = f16 ? 4 : 5;  // 16-byte chunks a row: 16 or 32
    const size_t row_bytes = f16 ? 256 : 512;
    int pg_start = 0, pg_end = -1;
    const char* base = nullptr;
    for (int ci = t; ci < (n << cshift); ci += 256) {
      const int jj = ci >> cshift, cc = ci & ((1 << cshift) - 1), j = j0 + jj;
      if (j >= pg_end) {
        const int pgi = j / cache.page_tokens;
        pg_start = pgi * cache.page_tokens;
        pg_end = pg_start + cache.page_tokens;
        const int page = cache.page_table[(size_t)stream * cache.pages_per_stream + pgi];
        const size_t off = kv_offset(cache, cfg, page, layer, which, kvh, 0);
        base = f16 ? (const char*)((const __half*)cache.pool + off) : (const char*)((const float*)cache.pool + off);
      }
      const int4* src = (const int4*)(base + (size_t)(j - pg_start) * row_bytes);
      cp_async16(dst + jj * pitch + cc * 4, src + cc);
    }
    cp_commit();
  };
  // Tile ti of keys or values: the next tile goes out before this one is
  // waited for (double buffering).
  const int ntile = (T + AR_KT - 1) / AR_KT;
  auto tile_ready = [&](int which, int ti) {
    if (ti + 1 < ntile) {
      stage(which, (ti + 1) * AR_KT, min(AR_KT, T - (ti + 1) * AR_KT), kvb[(ti + 1) & 1]);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      cp_wait_all();
    }
    __syncthreads();
  };
  // Eight consecutive dimensions of a staged row as floats (one 16-byte
  // load for f16 rows).
  const float* kv = kvb[0];  // the staged tile being read (set per tile)
  auto row8 = [&](int jj, int e, float (&o)[8]) {
    if (f16) {
      const uint4 raw = *(const uint4*)((const __half*)(kv + jj * pitch) + e);
      const __half2* h = (const __half2*)&raw;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        o[2 * i] = f.x;
        o[2 * i + 1] = f.y;
      }
    } else {
      const float4 a = *(const float4*)(kv + jj * pitch + e), b = *(const float4*)(kv + jj * pitch + e + 4);
      o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
      o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
  };
  // Scores.
  __syncthreads();
  stage(0, 0, min(AR_KT, T), kvb[0]);
  for (int ti = 0; ti < ntile; ++ti) {
    const int j0 = ti * AR_KT, n = min(AR_KT, T - j0);
    tile_ready(0, ti);
    kv = kvb[ti & 1];
    const int kg = (n + KB - 1) / KB, items = ((RQ + QB - 1) / QB) * kg;
    for (int it = t; it < items; it += 256) {
      // Keys jb, jb + kg, ...: neighbouring threads read neighbouring
      // staged rows (no shared-memory bank conflicts).
      const int qb = it / kg, jb = it % kg;
      float acc[QB][KB];
#pragma unroll
      for (int a = 0; a < QB; ++a)
#pragma unroll
        for (int b = 0; b < KB; ++b) acc[a][b] = 0.0f;
      for (int e = 0; e < 128; e += 8) {
        float kk[KB][8], qq[QB][8];
#pragma unroll
        for (int b = 0; b < KB; ++b) row8(min(jb + b * kg, n - 1), e, kk[b]);
#pragma unroll
        for (int a = 0; a < QB; ++a) {
          const float* qr = q + min(qb * QB + a, RQ - 1) * 128 + e;
          const float4 lo = *(const float4*)qr, hi = *(const float4*)(qr + 4);
          qq[a][0] = lo.x; qq[a][1] = lo.y; qq[a][2] = lo.z; qq[a][3] = lo.w;
          qq[a][4] = hi.x; qq[a][5] = hi.y; qq[a][6] = hi.z; qq[a][7] = hi.w;
        }
#pragma unroll
        for (int a = 0; a < QB; ++a)
#pragma unroll
          for (int b = 0; b < KB; ++b)
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[a][b] = __fmaf_rn(qq[a][c], kk[b][c], acc[a][b]);
      }
#pragma unroll
      for (int a = 0; a < QB; ++a)
#pragma unroll
        for (int b = 0; b < KB; ++b) {
          const int qh = qb * QB + a, jj = jb + b * kg, j = j0 + jj;
          if (qh < RQ && jj < n && j < visible(qh)) sc[(size_t)qh * tmax + j] = acc[a][b];
        }
    }
    __syncthreads();  // the buffer is refilled two tiles on
  }
  // Value tile 0 goes out before the softmax.
  stage(1, 0, min(AR_KT, T), kvb[0]);
  // Max and exp: a warp per query head; then the sums in key order, one
  // thread per query head (all heads at once); then the probabilities.
  const int warp = t >> 5, lane = t & 31;
  for (int qh = warp; qh < RQ; qh += 8) {
    const int vis = visible(qh);
    float* srow = sc + (size_t)qh * tmax;
    float mx = -INFINITY;
    for (int j = lane; j < vis; j += 32) mx = fmaxf(mx, srow[j]);
    mx = warp_max(mx);
    for (int j = lane; j < vis; j += 32) srow[j] = cephes_exp(__fsub_rn(srow[j], mx));
  }
  __syncthreads();
  if (t < RQ) {
    const int vis = visible(t);
    const float* srow = sc + (size_t)t * tmax;
    float sum = 0.0f;
#pragma unroll 8
    for (int j = 0; j < vis; ++j) sum = __fadd_rn(sum, srow[j]);
    inv[t] = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  for (int qh = warp; qh < RQ; qh += 8) {
    const int vis = visible(qh);
    float* srow = sc + (size_t)qh * tmax;
    const float iv = inv[qh];
    for (int j = lane; j < vis; j += 32) srow[j] = __fmul_rn(srow[j], iv);
  }
  // Values: a thread keeps DW chains (one query head, DW dimensions).
  constexpr int PER_HEAD = 128 / DW;
  const int items = RQ * PER_HEAD;
  constexpr int MAXI = 64 * PER_HEAD / 256;  // items a thread (RQ <= 64)
  float acc[MAXI][DW];
#pragma unroll
  for (int u = 0; u < MAXI; ++u)
#pragma unroll
    for (int c = 0; c < DW; ++c) acc[u][c] = 0.0f;
  for (int ti = 0; ti < ntile; ++ti) {
    const int j0 = ti * AR_KT, n = min(AR_KT, T - j0);
    tile_ready(1, ti);
    kv = kvb[ti & 1];
#pragma unroll
    for (int u = 0; u < MAXI; ++u) {
      const int it = t + u * 256;
      if (it < items) {
        const int qh = it / PER_HEAD, e = (it % PER_HEAD) * DW;
        const int lim = min(n, visible(qh) - j0);
        const float* pr = sc + (size_t)qh * tmax + j0;
#pragma unroll 4
        for (int jj = 0; jj < lim; ++jj) {
          const float p = pr[jj];
          float v[DW];
          if (DW == 2) {
            float2 f = f16 ? __half22float2(*((const __half2*)(kv + jj * pitch) + e / 2))
                           : *(const float2*)(kv + jj * pitch + e);
            v[0] = f.x;
            v[DW - 1] = f.y;
          } else {
#pragma unroll
            for (int c = 0; c < DW; c += 8) {
              float f[8];
              row8(jj, e + c, f);
#pragma unroll
              for (int i = 0; i < 8; ++i) v[c + i] = f[i];
            }
          }
#pragma unroll
          for (int c = 0; c < DW; ++c) acc[u][c] = __fmaf_rn(p, v[c], acc[u][c]);
        }
      }
    }
    __syncthreads();  // the buffer is refilled two tiles on
  }
#pragma unroll
  for (int u = 0; u < MAXI; ++u) {
    const int it = t + u * 256;
    if (it < items) {
      const int qh = it / PER_HEAD, e = (it % PER_HEAD) * DW, r = qh / qpk, h = qh % qpk;
      float* dst = att + (size_t)(r0 + r) * qd + (kvh * qpk + h) * 128 + e;
#pragma unroll
      for (int c = 0; c < DW; ++c) dst[c] = acc[u][c];
    }
  }
}

// ------------------------------------------- attention of decode rows ----
// One row (a stream's next position) per block and kv head: the row's QPK
// query heads over keys [0, T), with the same operations in the same order
// as k_attention_rows (each chain starts at 0 and takes its terms in
// order), laid out for one row so that a staged key or value is converted
// once for several chains and two chains share one packed f32x2 fma (each
// lane rounded as the scalar fma).
//   scores: a task keeps keys j and j + pairs (rows read by neighbouring
//           threads are neighbours: no bank conflicts) for HG query heads:
//           per dimension one converted key pair feeds HG packed fmas with
//           the head's q duplicated as (q, q) in shared memory;
//   softmax: max and exp a warp per head; the sum in key order by one
//           thread per head, its loads running ahead of the adds;
//   values: a task keeps one query head and dimensions (2d, 2d + 1), one
//           packed fma a key with the probability duplicated.
// Keys and values are staged KT at a time by cp.async into one buffer
// (two blocks an SM: while one waits for its tile the other computes;
// measured faster than two buffers of half the keys, which halve the
// score tasks a tile).
template <int QPK, bool F16>
struct StepShape {
  static constexpr int HG = QPK >= 2 ? 2 : 1;     // query heads a score task
  static constexpr int KT = F16 ? 256 : 128;      // keys a staged tile
  static constexpr int PITCH = F16 ? 68 : 132;    // floats a staged row (16-byte aligned, banks staggered)
  static size_t smem(int tmax) { return ((size_t)QPK * 256 + (size_t)QPK * tmax + (size_t)KT * PITCH + 8) * 4; }
};

template <int QPK, bool F16>
__global__ void __launch_bounds__(256, 2) k_attention_step(const float* qkv, DConfig cfg, DCache cache,
                                                           const int* row_stream, const int* row_pos, int layer,
                                                           int tmax, int all_keys, float* att) {
  using S = StepShape<QPK, F16>;
  constexpr int HG = S::HG, KT = S::KT, PITCH = S::PITCH;
  extern __shared__ __align__(16) float sm[];
  const int r = blockIdx.x, kvh = blockIdx.y, t = threadIdx.x;
  const int qd = cfg.heads * 128, stride = qd + 2 * cfg.kv_heads * 128;
  float2* qdup = (float2*)sm;
  float* sc = sm + QPK * 256;
  float* kv = sc + (size_t)QPK * tmax;
  float* inv = kv + KT * PITCH;
  const int stream = row_stream[r], pos = row_pos[r];
  const int T = all_keys > 0 ? all_keys : pos + 1;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
  for (int i = t; i < QPK * 128; i += 256) {
    const int h = i / 128, e = i % 128;
    const float v = __fmul_rn(qkv[(size_t)r * stride + (kvh * QPK + h) * 128 + e], scale);
    qdup[((h / HG) * 128 + e) * HG + h % HG] = make_float2(v, v);
  }
  auto stage = [&](int which, int j0, int n) {
    constexpr int cshift = F16 ? 4 : 5;
    constexpr size_t row_bytes = F16 ? 256 : 512;
    int pg_start = 0, pg_end = -1;
    const char* base = nullptr;
    for (int ci = t; ci < (n << cshift); ci += 256) {
      const int jj = ci >> cshift, cc = ci & ((1 << cshift) - 1), j = j0 + jj;
      if (j >= pg_end) {
        const int pgi = j / cache.page_tokens;
        pg_start = pgi * cache.page_tokens;
        pg_end = pg_start + cache.page_tokens;
        const int page = cache.page_table[(size_t)stream * cache.pages_per_stream + pgi];
        const size_t off = kv_offset(cache, cfg, page, layer, which, kvh, 0);
        base = F16 ? (const char*)((const __half*)cache.pool + off) : (const char*)((const float*)cache.pool + off);
      }
      cp_async16(kv + jj * PITCH + cc * 4, (const int4*)(base + (size_t)(j - pg_start) * row_bytes) + cc);
    }
    cp_commit();
  };
  auto row8 = [&](int jj, int e, float (&o)[8]) {
    if (F16) {
      const uint4 raw = *(const uint4*)((const __half*)(kv + jj * PITCH) + e);
      const __half2* h = (const __half2*)&raw;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        o[2 * i] = f.x;
        o[2 * i + 1] = f.y;
      }
    } else {
      const float4 a = *(const float4*)(kv + jj * PITCH + e), b = *(const float4*)(kv + jj * PITCH + e + 4);
      o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
      o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
  };
  const int ntile = (T + KT - 1) / KT;
  __syncthreads();
  for (int ti = 0; ti < ntile; ++ti) {
    const int j0 = ti * KT, n = min(KT, T - j0);
    stage(0, j0, n);
    cp_wait_all();
    __syncthreads();
    const int pairs = (n + 1) / 2, tasks = pairs * (QPK / HG);
    for (int it = t; it < tasks; it += 256) {
      const int g = it / pairs, ja = it % pairs, jb = min(ja + pairs, n - 1);
      float2 acc[HG];
#pragma unroll
      for (int h = 0; h < HG; ++h) acc[h] = make_float2(0.0f, 0.0f);
      const float2* qg = qdup + g * 128 * HG;
#pragma unroll 2
      for (int e = 0; e < 128; e += 8) {
        float ka[8], kb[8];
        row8(ja, e, ka);
        row8(jb, e, kb);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float2 kk = make_float2(ka[c], kb[c]);
          if (HG == 2) {
            const float4 qq = *(const float4*)(qg + (e + c) * 2);
            acc[0] = fma2(make_float2(qq.x, qq.y), kk, acc[0]);
            acc[HG - 1] = fma2(make_float2(qq.z, qq.w), kk, acc[HG - 1]);
          } else {
            acc[0] = fma2(qg[e + c], kk, acc[0]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        float* srow = sc + (size_t)(g * HG + h) * tmax + j0;
        srow[ja] = acc[h].x;
        if (ja + pairs < n) srow[ja + pairs] = acc[h].y;
      }
    }
    __syncthreads();
  }
  stage(1, 0, min(KT, T));
  const int warp = t >> 5, lane = t & 31;
  for (int h = warp; h < QPK; h += 8) {
    float* srow = sc + (size_t)h * tmax;
    float mx = -INFINITY;
    for (int j = lane; j < T; j += 32) mx = fmaxf(mx, srow[j]);
    mx = warp_max(mx);
    for (int j = lane; j < T; j += 32) srow[j] = cephes_exp(__fsub_rn(srow[j], mx));
  }
  __syncthreads();
  if (t < QPK) {
    inv[t] = __fdiv_rn(1.0f, seq_sum_ahead(sc + (size_t)t * tmax, T));
  }
  __syncthreads();
  for (int h = warp; h < QPK; h += 8) {
    float* srow = sc + (size_t)h * tmax;
    const float iv = inv[h];
    for (int j = lane; j < T; j += 32) srow[j] = __fmul_rn(srow[j], iv);
  }
  constexpr int TASKS = QPK * 64;
  constexpr int PER = (TASKS + 255) / 256;
  float2 acc[PER];
#pragma unroll
  for (int u = 0; u < PER; ++u) acc[u] = make_float2(0.0f, 0.0f);
  for (int ti = 0; ti < ntile; ++ti) {
    const int j0 = ti * KT, n = min(KT, T - j0);
    if (ti > 0) stage(1, j0, n);
    cp_wait_all();
    __syncthreads();
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int it = t + u * 256;
      if (it < TASKS) {
        const int h = it / 64, d = it % 64;
        const float* pr = sc + (size_t)h * tmax + j0;
        float2 a = acc[u];
        // Four probabilities a load (pr is 16-byte aligned: tmax and the
        // tile's first key are multiples of 4); the fmas stay in key order.
        int jj = 0;
#pragma unroll 2
        for (; jj + 4 <= n; jj += 4) {
          const float4 p4 = *(const float4*)(pr + jj);
          const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 v = F16 ? __half22float2(*((const __half2*)(kv + (jj + i) * PITCH) + d))
                                 : *(const float2*)(kv + (jj + i) * PITCH + 2 * d);
            a = fma2(make_float2(pv[i], pv[i]), v, a);
          }
        }
        for (; jj < n; ++jj) {
          const float p = pr[jj];
          const float2 v = F16 ? __half22float2(*((const __half2*)(kv + jj * PITCH) + d))
                               : *(const float2*)(kv + jj * PITCH + 2 * d);
          a = fma2(make_float2(p, p), v, a);
        }
        acc[u] = a;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int it = t + u * 256;
    if (it < TASKS) {
      const int h = it / 64, d = it % 64;
      *(float2*)(att + (size_t)r * qd + (kvh * QPK + h) * 128 + 2 * d) = acc[u];
    }
  }
}

template <int QPK, bool F16>
static cudaError_t step_attention(const float* qkv, int m, const DConfig& cfg, const DCache& cache,
                                  const int* row_stream, const int* row_pos, int layer, int tmax, int all_keys,
                                  float* att, cudaStream_t s) {
  static DeviceOnce once;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = once.run(dev, [] {
    return cudaFuncSetAttribute(k_attention_step<QPK, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (e != cudaSuccess) return e;
  k_attention_step<QPK, F16><<<dim3(m, cfg.kv_heads), 256, StepShape<QPK, F16>::smem(tmax), s>>>(
      qkv, cfg, cache, row_stream, row_pos, layer, tmax, all_keys, att);
  return cudaGetLastError();
}

// The decode-row kernel for this shape, or null when it does not apply
// (query heads a kv head other than 1, 2, 4, 8; shared memory too small).
using StepFn = cudaError_t (*)(const float*, int, const DConfig&, const DCache&, const int*, const int*, int, int, int,
                               float*, cudaStream_t);
template <bool F16>
static StepFn step_kernel(int qpk, int tmax) {
  const size_t limit = 227 * 1024;
  switch (qpk) {
    case 1: return StepShape<1, F16>::smem(tmax) <= limit ? step_attention<1, F16> : nullptr;
    case 2: return StepShape<2, F16>::smem(tmax) <= limit ? step_attention<2, F16> : nullptr;
    case 4: return StepShape<4, F16>::smem(tmax) <= limit ? step_attention<4, F16> : nullptr;
    case 8: return StepShape<8, F16>::smem(tmax) <= limit ? step_attention<8, F16> : nullptr;
    default: return nullptr;
  }
}

// ------------------------------------------ attention of prompt tiles ----
// k_attention_rows' work for tiles of 16 or more query heads on an f16
// cache with an even number of query heads a kv head, with the same
// operations in the same order, laid out so that each staged key or value
// is converted to f32 once for the whole tile and two chains share one
// packed f32x2 fma (each lane rounded as the scalar fma):
//   staging: a tile's keys (then values) are loaded into registers while
//            the tile before is used, and stored to shared memory as f32;
//   scores:  a thread keeps 4 query heads (two pairs, q interleaved by
//            pair in shared memory) x 4 keys; per dimension one packed fma
//            updates a pair's chains with the key duplicated;
//   values:  a thread keeps two query heads of one row (the same visible
//            keys) x 8 dimensions (4 and 4, 64 apart: conflict-free reads),
//            one packed fma per pair of dimensions and head.
constexpr int AT_PITCH = 132;  // floats a staged f32 row (16-byte aligned, rows 4 banks apart)
constexpr int AT_VI = 2;       // value items a thread at most (64 query heads)

__global__ void __launch_bounds__(256) k_attention_tile(const float* qkv, const int2* tiles, DConfig cfg, DCache cache,
                                                        const int* row_stream, const int* row_pos, int layer, int tmax,
                                                        int all_keys, float* att) {
  extern __shared__ __align__(16) float sm[];
  const int kvh = blockIdx.y, t = threadIdx.x;
  const int2 tile = tiles[blockIdx.x];
  const int r0 = tile.x, R = tile.y;
  const int qpk = cfg.heads / cfg.kv_heads, qd = cfg.heads * 128, stride = qd + 2 * cfg.kv_heads * 128;
  const int RQ = R * qpk;                // a multiple of 4 (qpk even, quad tiles)
  float* qp = sm;                        // [RQ / 2][128][2]: q of heads 2i and 2i + 1 per dimension
  float* sc = qp + (size_t)RQ * 128;     // [RQ][tmax]
  float* kv = sc + (size_t)RQ * tmax;    // [AR_KT][AT_PITCH]
  float* inv = kv + AR_KT * AT_PITCH;    // [RQ]
  const int stream = row_stream[r0], p0 = row_pos[r0];
  const int T = all_keys > 0 ? all_keys : p0 + R;
  auto visible = [&](int qh) { return all_keys > 0 ? all_keys : p0 + qh / qpk + 1; };
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
  for (int i = t; i < RQ * 128; i += 256) {
    const int qh = i / 128, e = i % 128, r = qh / qpk, h = qh % qpk;
    qp[((qh >> 1) * 128 + e) * 2 + (qh & 1)] = __fmul_rn(qkv[(size_t)(r0 + r) * stride + (kvh * qpk + h) * 128 + e], scale);
  }
  // Chunk u of a tile for this thread: chunk t + 256 u, row (t + 256 u) / 16
  // (rows 16 apart), 16 bytes = 8 values; neighbouring threads read a row's
  // neighbouring chunks.
  const int ntile = (T + AR_KT - 1) / AR_KT;
  uint4 pre[8];
  auto fetch = [&](int i) {
    const int which = i < ntile ? 0 : 1, j0 = (i % ntile) * AR_KT, n = min(AR_KT, T - j0);
    int pg_end = -1, pg_start = 0;
    const __half* base = nullptr;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int jj = (t >> 4) + 16 * u, cc = t & 15, j = j0 + jj;
      pre[u] = make_uint4(0, 0, 0, 0);
      if (jj < n) {
        if (j >= pg_end) {
          const int pgi = j / cache.page_tokens;
          pg_start = pgi * cache.page_tokens;
          pg_end = pg_start + cache.page_tokens;
          const int page = cache.page_table[(size_t)stream * cache.pages_per_stream + pgi];
          base = (const __half*)cache.pool + kv_offset(cache, cfg, page, layer, which, kvh, 0);
        }
        pre[u] = *(const uint4*)(base + (size_t)(j - pg_start) * 128 + cc * 8);
      }
    }
  };
  auto store = [&]() {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int jj = (t >> 4) + 16 * u, cc = t & 15;
      const __half2* h = (const __half2*)&pre[u];
      const float2 a = __half22float2(h[0]), b = __half22float2(h[1]), c = __half22float2(h[2]),
                   d = __half22float2(h[3]);
      *(float4*)(kv + jj * AT_PITCH + cc * 8) = make_float4(a.x, a.y, b.x, b.y);
      *(float4*)(kv + jj * AT_PITCH + cc * 8 + 4) = make_float4(c.x, c.y, d.x, d.y);
    }
  };
  const int warp = t >> 5, lane = t & 31;
  float2 vacc[AT_VI][2][4];
#pragma unroll
  for (int u = 0; u < AT_VI; ++u)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int k = 0; k < 4; ++k) vacc[u][h][k] = make_float2(0.0f, 0.0f);
  const int vitems = (RQ / 2) * 16;
  fetch(0);
  for (int i = 0; i < 2 * ntile; ++i) {
    __syncthreads();  // the tile before is used up
    store();
    __syncthreads();
    if (i + 1 < 2 * ntile) fetch(i + 1);  // in flight while this tile is used
    const int j0 = (i % ntile) * AR_KT, n = min(AR_KT, T - j0);
    if (i < ntile) {
      // Scores: 4 query heads x keys jb, jb + kg, jb + 2 kg, jb + 3 kg.
      // (The last group of a tile may hold one pair: RQ is even; the other
      // pair's q reads stay inside shared memory and its chains are dropped.)
      const int kg = (n + 3) / 4, items = ((RQ + 3) / 4) * kg;
      for (int it = t; it < items; it += 256) {
        const int qb = it / kg, jb = it % kg;
        float2 acc[2][4];
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int b = 0; b < 4; ++b) acc[p][b] = make_float2(0.0f, 0.0f);
        const float* kr[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) kr[b] = kv + min(jb + b * kg, n - 1) * AT_PITCH;
        const float* qa = qp + (size_t)(2 * qb) * 256;
        const float* qb2 = qa + 256;
#pragma unroll 2
        for (int e = 0; e < 128; e += 4) {
          float4 kk[4];
#pragma unroll
          for (int b = 0; b < 4; ++b) kk[b] = *(const float4*)(kr[b] + e);
          const float4 a0 = *(const float4*)(qa + 2 * e), a1 = *(const float4*)(qa + 2 * e + 4);
          const float4 c0 = *(const float4*)(qb2 + 2 * e), c1 = *(const float4*)(qb2 + 2 * e + 4);
          const float2 qx[2][4] = {{make_float2(a0.x, a0.y), make_float2(a0.z, a0.w), make_float2(a1.x, a1.y),
                                    make_float2(a1.z, a1.w)},
                                   {make_float2(c0.x, c0.y), make_float2(c0.z, c0.w), make_float2(c1.x, c1.y),
                                    make_float2(c1.z, c1.w)}};
#pragma unroll
          for (int d = 0; d < 4; ++d)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const float kd = d == 0 ? kk[b].x : d == 1 ? kk[b].y : d == 2 ? kk[b].z : kk[b].w;
              const float2 k2 = make_float2(kd, kd);
              acc[0][b] = fma2(qx[0][d], k2, acc[0][b]);
              acc[1][b] = fma2(qx[1][d], k2, acc[1][b]);
            }
        }
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int qh = 4 * qb + 2 * p + c;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const int jj = jb + b * kg, j = j0 + jj;
              if (qh < RQ && jj < n && j < visible(qh)) sc[(size_t)qh * tmax + j] = c ? acc[p][b].y : acc[p][b].x;
            }
          }
      }
      if (i == ntile - 1) {
        // Softmax: max and exp a warp per query head; the sums in key order,
        // one thread per query head, its loads ahead of the adds.
        __syncthreads();
        for (int qh = warp; qh < RQ; qh += 8) {
          const int vis = visible(qh);
          float* srow = sc + (size_t)qh * tmax;
          float mx = -INFINITY;
          for (int j = lane; j < vis; j += 32) mx = fmaxf(mx, srow[j]);
          mx = warp_max(mx);
          for (int j = lane; j < vis; j += 32) srow[j] = cephes_exp(__fsub_rn(srow[j], mx));
        }
        __syncthreads();
        if (t < RQ) inv[t] = __fdiv_rn(1.0f, seq_sum_ahead(sc + (size_t)t * tmax, visible(t)));
        __syncthreads();
        for (int qh = warp; qh < RQ; qh += 8) {
          const int vis = visible(qh);
          float* srow = sc + (size_t)qh * tmax;
          const float iv = inv[qh];
          for (int j = lane; j < vis; j += 32) srow[j] = __fmul_rn(srow[j], iv);
        }
      }
    } else {
      // Values: heads 2 pp and 2 pp + 1 (one row) x dimensions 4 dg.. and
      // 64 + 4 dg.., keys in order.
#pragma unroll
      for (int u = 0; u < AT_VI; ++u) {
        const int it = t + 256 * u;
        if (it < vitems) {
          const int pp = it >> 4, dg = it & 15, qh0 = 2 * pp;
          const int lim = min(n, visible(qh0) - j0);
          const float* pr0 = sc + (size_t)qh0 * tmax + j0;
          const float* pr1 = pr0 + tmax;
          const float* vr = kv + 4 * dg;
#pragma unroll 4
          for (int jj = 0; jj < lim; ++jj) {
            const float pa = pr0[jj], pb = pr1[jj];
            const float4 v0 = *(const float4*)(vr + jj * AT_PITCH), v1 = *(const float4*)(vr + jj * AT_PITCH + 64);
            const float2 vv[4] = {make_float2(v0.x, v0.y), make_float2(v0.z, v0.w), make_float2(v1.x, v1.y),
                                  make_float2(v1.z, v1.w)};
            const float2 p2a = make_float2(pa, pa), p2b = make_float2(pb, pb);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              vacc[u][0][k] = fma2(p2a, vv[k], vacc[u][0][k]);
              vacc[u][1][k] = fma2(p2b, vv[k], vacc[u][1][k]);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < AT_VI; ++u) {
    const int it = t + 256 * u;
    if (it < vitems) {
      const int pp = it >> 4, dg = it & 15;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int qh = 2 * pp + c, r = qh / qpk, h = qh % qpk;
        float* dst = att + (size_t)(r0 + r) * qd + (kvh * qpk + h) * 128;
        *(float4*)(dst + 4 * dg) = make_float4(vacc[u][c][0].x, vacc[u][c][0].y, vacc[u][c][1].x, vacc[u][c][1].y);
        *(float4*)(dst + 64 + 4 * dg) = make_float4(vacc[u][c][2].x, vacc[u][c][2].y, vacc[u][c][3].x, vacc[u][c][3].y);
      }
    }
  }
}

int attention_tile_rows(const DConfig& cfg, int tmax, int f16) {
  // A block's shared memory (220 KB): two staged K/V tiles, and for every
  // query head of the tile its q row and its scores; at most 16 rows and
  // 64 query heads a block, and whole groups of 4 query heads.
  const int qpk = cfg.heads / cfg.kv_heads;
  const long budget = 220L * 1024 / 4 - 2L * AR_KT * (f16 ? 68 : 132) - 64;
  const long rq = budget / (128L + std::max(tmax, 1));
  int r = (int)std::min<long>(std::min<long>(16, rq / qpk), 64 / std::max(qpk, 1));
  if (r * qpk >= 16) r = r / (4 / std::__gcd(qpk, 4)) * (4 / std::__gcd(qpk, 4));
  return std::max(r, 1);
}

cudaError_t launch_attention_rows(const float* qkv, const int2* tiles, int ntiles, int rows_max, const DConfig& cfg,
                                  const DCache& cache, const int* row_stream, const int* row_pos, int layer,
                                  int max_tk, float* att, cudaStream_t s, int all_keys) {
  const int qpk = cfg.heads / cfg.kv_heads;
  const int RQ = rows_max * qpk;
  if (RQ > 64 || all_keys > max_tk) return cudaErrorInvalidValue;
  const int tmax = (max_tk + 3) / 4 * 4;
  size_t smem = ((size_t)RQ * 128 + (size_t)RQ * tmax + (size_t)2 * AR_KT * (cache.f16 ? 68 : 132) + RQ) * 4;
  // One row a block (decode steps): the decode-row kernel where it applies.
  static const bool legacy_step = getenv("TRIT_ATTENTION_ROWS") != nullptr;  // the row-tile kernel instead
  if (!tiles && rows_max == 1 && !legacy_step) {
    StepFn fn = cache.f16 ? step_kernel<true>(qpk, tmax) : step_kernel<false>(qpk, tmax);
    if (fn) return fn(qkv, ntiles, cfg, cache, row_stream, row_pos, layer, tmax, all_keys, att, s);
  }
  if (smem > 220 * 1024) return cudaErrorInvalidValue;
  // Blocks of 4 query heads for tiles of 16 or more query heads.
  const bool quad = tiles && RQ >= 16;
  static const bool legacy_tile = getenv("TRIT_ATTENTION_ROWS") != nullptr;
  if (quad && cache.f16 && qpk % 2 == 0 && !legacy_tile) {
    const size_t tsmem = ((size_t)RQ * 128 + (size_t)RQ * tmax + (size_t)AR_KT * AT_PITCH + RQ) * 4;
    static DeviceOnce tonce;
    int tdev = 0;
    cudaError_t te = cudaGetDevice(&tdev);
    if (te != cudaSuccess) return te;
    te = tonce.run(tdev, [] {
      return cudaFuncSetAttribute(k_attention_tile, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
    });
    if (te != cudaSuccess) return te;
    if (tsmem <= 220 * 1024) {
      k_attention_tile<<<dim3(ntiles, cfg.kv_heads), 256, tsmem, s>>>(qkv, tiles, cfg, cache, row_stream, row_pos,
                                                                      layer, tmax, all_keys, att);
      return cudaGetLastError();
    }
  }
  static DeviceOnce once;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = once.run(dev, [] {
    cudaError_t r = cudaFuncSetAttribute(k_attention_rows<4, 4, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         220 * 1024);
    if (r != cudaSuccess) return r;
    return cudaFuncSetAttribute(k_attention_rows<1, 2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
  });
  if (e != cudaSuccess) return e;
  if (quad)
    k_attention_rows<4, 4, 8><<<dim3(ntiles, cfg.kv_heads), 256, smem, s>>>(qkv, tiles, cfg, cache, row_stream, row_pos,
                                                                      layer, tmax, all_keys, att);
  else
    k_attention_rows<1, 2, 2><<<dim3(ntiles, cfg.kv_heads), 256, smem, s>>>(qkv, tiles, cfg, cache, row_stream, row_pos,
                                                                      layer, tmax, all_keys, att);
  return cudaGetLastError();
}

// ------------------------------------------------ final norm + table ----
// forward_rows' last step (causal_lm.rs:384-388): RmsNorm of the row, then
// the token table in f32 math (Q8::matmul -> fgemm::matmul_widened). Each
// thread owns one vocabulary row and keeps the 16 lanes of the AVX-512 tile
// (lane l sums k = 16t + l in order with fma) and the _mm512_reduce_add_ps
// tree (fgemm.rs:380-430), so a logit is the reference's value bit for bit
// for the same normed row. The block's codes come through shared memory in
// slabs of 128 bytes a row.
constexpr int TABLE_ROWS = 64;   // vocabulary rows per block, 4 threads each
constexpr int TABLE_MAX_B = 16;  // streams per pass

// The token table for `nb` normed rows (streams) at once. Thread q of a
// vocabulary row holds lanes 4q..4q+3 of the reference's 16-lane
// accumulator: at step t it reads the 4 code bytes k = 16t + 4q .. +3 (a
// 32-bit load; the 4 threads of a row read 16 consecutive bytes), widens
// them (code * scale, exact in f32) and adds x * w into its lanes with
// fma. The reduce tree then runs across the 4 threads in the order of
// _mm512_reduce_add_ps.
template <int B>
__global__ void __launch_bounds__(256) k_table(DTable T, const float* xn, int nb, float logit_mult, float* logits,
                                               float* best_val, int* best_idx, int nblocks) {
  extern __shared__ __align__(16) float xt[];  // [k][B]: the rows side by side
  const int t = threadIdx.x, q = t & 3;
  const int row = blockIdx.x * TABLE_ROWS + (t >> 2);
  for (int i = t; i < T.k * B; i += 256) {
    int kk = i / B, b = i % B;
    xt[i] = (b < nb) ? xn[(size_t)b * T.k + kk] : 0.0f;
  }
  __syncthreads();
  float acc[B][4];
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int l = 0; l < 4; ++l) acc[b][l] = 0.0f;
  const bool live = row < T.n;
  if (live) {
    const uint32_t* codes = (const uint32_t*)(T.codes + (size_t)row * T.k) + q;
    const int steps = T.k / 16;
#pragma unroll 4
    for (int st = 0; st < steps; ++st) {
      uint32_t word = __ldg(codes + 4 * st) ^ 0x80808080u;
      float s = table_scale(T, row, st >> 1);
      int kk = 16 * st + 4 * q;
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        float w = __fmul_rn(byte_to_float(word, l), s);
#pragma unroll
        for (int b = 0; b < B; ++b) acc[b][l] = __fmaf_rn(xt[(kk + l) * B + b], w, acc[b][l]);
      }
    }
  }
  __shared__ float bv[B][8];
  __shared__ int bi[B][8];
  const int lane = t & 31, warp = t >> 5;
#pragma unroll
  for (int b = 0; b < B; ++b) {
    // s8[i] = a[i] + a[i + 8]: threads 0,1 take the lanes of threads 2,3.
    float s8[4];
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      float other = __shfl_down_sync(0xffffffffu, acc[b][l], 2);
      s8[l] = __fadd_rn(acc[b][l], other);
    }
    // s4[i] = s8[i] + s8[i + 4]: thread 0 takes thread 1's.
    float s4[4];
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      float other = __shfl_down_sync(0xffffffffu, s8[l], 1);
      s4[l] = __fadd_rn(s8[l], other);
    }
    float v = __fadd_rn(__fadd_rn(s4[0], s4[2]), __fadd_rn(s4[1], s4[3]));
    int idx = 0x7fffffff;
    if (q == 0 && live && b < nb) {
      if (logit_mult != 1.0f) v = __fmul_rn(v, logit_mult);
      if (logits) logits[(size_t)b * T.n + row] = v;
      idx = row;
      if (v != v) { v = -INFINITY; idx = 0x7fffffff; }  // a NaN never wins
    } else {
      v = -INFINITY;
    }
    // The largest value; the lowest index among equals (layers.rs:603-612).
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, v, o);
      int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
    }
    if (lane == 0) { bv[b][warp] = v; bi[b][warp] = idx; }
  }
  __syncthreads();
  if (t < nb && t < B) {
    float v = bv[t][0];
    int idx = bi[t][0];
    for (int i = 1; i < 8; ++i)
      if (bv[t][i] > v || (bv[t][i] == v && bi[t][i] < idx)) { v = bv[t][i]; idx = bi[t][i]; }
    best_val[(size_t)t * nblocks + blockIdx.x] = v;
    best_idx[(size_t)t * nblocks + blockIdx.x] = idx;
  }
}

// The token table for batches of streams: each thread keeps lane l of the
// reference's 16-lane accumulator (k = l mod 16) for 4 vocabulary rows and
// B streams, so every widened weight feeds B fma and every x pair 4 of
// them. A block owns TABLE_ROWS rows: 16 row groups x 16 lanes. The
// streams' rows come through shared memory in chunks of TB_KC values
// (cp.async, double-buffered), are turned k-major ([k][stream], pitch B + 2
// so that a half-warp's 8-byte reads of 16 consecutive k hit 32 distinct
// banks) and are read as stream pairs: one packed f32x2 fma (each lane
// rounded as the scalar fma) updates one row's chains of two streams.
// The block's codes and scales of each chunk come through shared memory
// with the chunk's x values (cp.async, double-buffered), so no thread
// waits on a global load in the fma loop. The 16 lanes of a row then
// reduce in the order of _mm512_reduce_add_ps, as k_table does.
constexpr int TB_KC = 256;
constexpr int TB_CPITCH = TB_KC + 16;  // bytes a staged code row (rows 4 apart land 16 banks apart)
constexpr int TB_SPITCH = 32;          // bytes a staged scale row (8 scales of a chunk, f16 or f32)

// Shared memory of k_table_rows<B>, in bytes.
constexpr size_t table_rows_smem(int B) {
  return ((size_t)2 * B * TB_KC + (size_t)TB_KC * (B + 2)) * 4 + (size_t)2 * TABLE_ROWS * (TB_CPITCH + TB_SPITCH);
}


template <int B>
__global__ void __launch_bounds__(256) k_table_rows(DTable T, const float* xn, int nb, float logit_mult,
                                                    float* logits, float* best_val, int* best_idx, int nblocks) {
  static_assert(B % 2 == 0, "stream pairs");
  constexpr int PB = B + 2;                    // k-major pitch
  extern __shared__ __align__(16) float xb[];  // [2][B][TB_KC] staged, then [TB_KC][PB] k-major
  float* xt = xb + 2 * B * TB_KC;
  uint8_t* cs = (uint8_t*)(xt + TB_KC * PB);           // [2][TABLE_ROWS][TB_CPITCH] codes
  uint8_t* ss = cs + 2 * TABLE_ROWS * TB_CPITCH;       // [2][TABLE_ROWS][TB_SPITCH] scales
  __shared__ float fin[B][TABLE_ROWS];
  const int t = threadIdx.x, l = t & 15, rg = t >> 4;
  const int blk0 = blockIdx.x * TABLE_ROWS;
  const int row0 = blk0 + rg * 4;
  const int k = T.k;
  const int sb = T.scale_f16 ? 2 : 4;  // bytes a scale
  auto stage = [&](int buf, int k0) {
    float* dst = xb + (size_t)buf * B * TB_KC;
    const int per = TB_KC / 4;  // 16-byte chunks a stream
    for (int i = t; i < B * per; i += 256) {
      int b = i / per, c = i % per;
      if (b < nb) cp_async16(dst + b * TB_KC + c * 4, xn + (size_t)b * k + k0 + c * 4);
      else *(float4*)(dst + b * TB_KC + c * 4) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    // The block's rows: TB_KC code bytes and TB_KC / 32 scales each (rows
    // past the table read row 0; their results are never kept).
    uint8_t* cdst = cs + (size_t)buf * TABLE_ROWS * TB_CPITCH;
    for (int i = t; i < TABLE_ROWS * (TB_KC / 16); i += 256) {
      const int r = i / (TB_KC / 16), c = i % (TB_KC / 16), row = blk0 + r < T.n ? blk0 + r : 0;
      cp_async16(cdst + r * TB_CPITCH + c * 16, T.codes + (size_t)row * k + k0 + c * 16);
    }
    uint8_t* sdst = ss + (size_t)buf * TABLE_ROWS * TB_SPITCH;
    const int sper = TB_KC / 32 * sb / 16;  // 16-byte chunks of a row's scales: 1 (f16) or 2 (f32)
    for (int i = t; i < TABLE_ROWS * sper; i += 256) {
      const int r = i / sper, c = i % sper, row = blk0 + r < T.n ? blk0 + r : 0;
      cp_async16(sdst + r * TB_SPITCH + c * 16,
                 (const uint8_t*)T.scales + ((size_t)row * (k / 32) + k0 / 32) * sb + c * 16);
    }
    cp_commit();
  };
  float2 acc[4][B / 2];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int p = 0; p < B / 2; ++p) acc[a][p] = make_float2(0.0f, 0.0f);
  bool live[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) live[a] = row0 + a < T.n;
  const int chunks = k / TB_KC;
  stage(0, 0);
  for (int c = 0; c < chunks; ++c) {
    if (c + 1 < chunks) stage((c + 1) & 1, (c + 1) * TB_KC);
    if (c + 1 < chunks) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else cp_wait_all();
    __syncthreads();
    {
      const float* xc = xb + (size_t)(c & 1) * B * TB_KC;
      for (int i = t; i < B * TB_KC; i += 256) {
        const int b = i / TB_KC, kk = i % TB_KC;
        xt[kk * PB + b] = xc[b * TB_KC + kk];
      }
    }
    __syncthreads();
    const int8_t* crow = (const int8_t*)cs + (size_t)(c & 1) * TABLE_ROWS * TB_CPITCH + rg * 4 * TB_CPITCH;
    const uint8_t* srow = ss + (size_t)(c & 1) * TABLE_ROWS * TB_SPITCH + rg * 4 * TB_SPITCH;
    for (int st = 0; st < TB_KC / 16; ++st) {
      const int kk = st * 16 + l;
      float2 w2[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const uint8_t* sp = srow + a * TB_SPITCH;
        const float scale = T.scale_f16 ? __half2float(((const __half*)sp)[st >> 1]) : ((const float*)sp)[st >> 1];
        const float w = __fmul_rn((float)crow[a * TB_CPITCH + kk], scale);
        w2[a] = make_float2(w, w);
      }
      const float2* xr = (const float2*)(xt + kk * PB);
#pragma unroll
      for (int p = 0; p < B / 2; ++p) {
        const float2 x2 = xr[p];
#pragma unroll
        for (int a = 0; a < 4; ++a) acc[a][p] = fma2(x2, w2[a], acc[a][p]);
      }
    }
    __syncthreads();
  }
  // Reduce the 16 lanes of each row: s8[i] = a[i] + a[i + 8], s4[i] =
  // s8[i] + s8[i + 4], then (s4[0] + s4[2]) + (s4[1] + s4[3]).
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float v = (b & 1) ? acc[a][b >> 1].y : acc[a][b >> 1].x;
      v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 8, 16));
      v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 16));
      v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 16));
      v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 16));
      if (l == 0) {
        if (logit_mult != 1.0f) v = __fmul_rn(v, logit_mult);
        if (logits && live[a] && b < nb) logits[(size_t)b * T.n + row0 + a] = v;
        fin[b][rg * 4 + a] = (live[a] && v == v) ? v : -INFINITY;  // a NaN never wins
      }
    }
  __syncthreads();
  // The block's best row per stream: the largest value, the lowest index
  // among equals (layers.rs:603-612).
  if (t < B && t < nb) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < TABLE_ROWS; ++r) {
      const int row = blockIdx.x * TABLE_ROWS + r;
      if (row < T.n && fin[t][r] > bv) {
        bv = fin[t][r];
        bi = row;
      }
    }
    best_val[(size_t)t * nblocks + blockIdx.x] = bv;
    best_idx[(size_t)t * nblocks + blockIdx.x] = bi;
  }
}

__global__ void k_argmax(const float* val, const int* idx, int n, int* token) {
  // One warp per stream (blockIdx.x): partials [stream][n].
  val += (size_t)blockIdx.x * n;
  idx += (size_t)blockIdx.x * n;
  float v = -INFINITY;
  int i = 0x7fffffff;
  for (int p = threadIdx.x; p < n; p += 32) {
    if (val[p] > v || (val[p] == v && idx[p] < i)) { v = val[p]; i = idx[p]; }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  if (threadIdx.x == 0) token[blockIdx.x] = (i == 0x7fffffff) ? 0 : i;
}

// The argmax of one stream's partials as a key whose unsigned order is the
// argmax order of layers.rs:603-612 across tensor-parallel ranks: the value
// (its bits mapped to an order-preserving unsigned) above the complement of
// its global index (rows v0 ..), so the larger value wins and, among equal
// values, the lower index. A row with no number (NaN everywhere) keys 0.
__global__ void k_argmax_key(const float* val, const int* idx, int n, int v0, unsigned long long* keys) {
  val += (size_t)blockIdx.x * n;
  idx += (size_t)blockIdx.x * n;
  float v = -INFINITY;
  int i = 0x7fffffff;
  for (int p = threadIdx.x; p < n; p += 32) {
    if (val[p] > v || (val[p] == v && idx[p] < i)) { v = val[p]; i = idx[p]; }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  if (threadIdx.x == 0) {
    unsigned long long key = 0;
    if (i != 0x7fffffff) {
      const uint32_t u = __float_as_uint(v);
      const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
      key = ((unsigned long long)ord << 32) | (uint32_t)~(uint32_t)(v0 + i);
    }
    keys[blockIdx.x] = key;
  }
}

__global__ void k_key_token(const unsigned long long* keys, int nb, int* token) {
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < nb; b += gridDim.x * blockDim.x)
    token[b] = keys[b] ? (int)~(uint32_t)keys[b] : 0;
}

// add_into (src/layers.rs): x[i] = x[i] + a[i].
__global__ void k_add(float* x, const float* a, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = __fadd_rn(x[i], a[i]);
}

// The bookkeeping between two greedy steps of a batch (one block).
__global__ void k_batch_advance(const int* cur, int* pos, int* step, int* tokens, int streams, int advance_pos) {
  const int at = *step;
  for (int s = threadIdx.x; s < streams; s += blockDim.x) {
    tokens[(size_t)at * streams + s] = cur[s];
    if (advance_pos) pos[s] += 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) *step = at + 1;
}

// ------------------------------------------------------------ launch ----
#define LAUNCH_CHECK()                                   \
  do {                                                   \
    cudaError_t e_ = cudaGetLastError();                 \
    if (e_ != cudaSuccess) return e_;                    \
  } while (0)

cudaError_t launch_embed(const DTable& T, const int* ids, int m, float* x, float mult, cudaStream_t s) {
  k_embed<<<m, 256, 0, s>>>(T, ids, m, x, mult);
  LAUNCH_CHECK();
  return cudaSuccess;
}

cudaError_t launch_batch_advance(const int* cur, int* pos, int* step, int* tokens, int streams, int advance_pos,
                                 cudaStream_t s) {
  k_batch_advance<<<1, 256, 0, s>>>(cur, pos, step, tokens, streams, advance_pos);
  LAUNCH_CHECK();
  return cudaSuccess;
}

cudaError_t launch_add(float* x, const float* a, size_t n, cudaStream_t s) {
  k_add<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, s>>>(x, a, n);
  LAUNCH_CHECK();
  return cudaSuccess;
}

cudaError_t launch_scale(float* x, size_t n, float mult, cudaStream_t s) {
  k_scale<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, s>>>(x, n, mult);
  LAUNCH_CHECK();
  return cudaSuccess;
}

// Quantized::grouped of rows with no norm and no scale (the attention
// output, h): the groups of a row are independent, so a row's groups spread
// over `gridDim.y` blocks (a warp a group, as k_norm_quant quantizes them).
template <int G>
__global__ void __launch_bounds__(256) k_quant_rows(const float* x, int d, int half, int8_t* xq, float* xs) {
  const int r = blockIdx.x, groups = d / G;
  const int per = (groups + gridDim.y - 1) / gridDim.y;
  const int g0 = blockIdx.y * per, g1 = min(groups, g0 + per);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* row = x + (size_t)r * d;
  for (int g = g0 + warp; g < g1; g += 8) {
    float v[G / 32];
#pragma unroll
    for (int i = 0; i < G / 32; ++i) v[i] = row[g * G + lane * (G / 32) + i];
    const float scale = warp_quantize_group<G>(v, xq + (size_t)r * d + g * G, half);
    if (lane == 0) xs[(size_t)r * groups + g] = scale;
  }
}

// h = silu(gate) * up of a stacked gate|up product (causal_lm.rs:464-474;
// g = [m][2 * units]), quantized as k_quant_rows quantizes h.
template <int G>
__global__ void __launch_bounds__(256) k_silu_quant(const float* g, int units, int half, int8_t* xq, float* xs) {
  const int r = blockIdx.x, groups = units / G;
  const int per = (groups + gridDim.y - 1) / gridDim.y;
  const int g0 = blockIdx.y * per, g1 = min(groups, g0 + per);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* row = g + (size_t)r * 2 * units;
  for (int gi = g0 + warp; gi < g1; gi += 8) {
    float v[G / 32];
#pragma unroll
    for (int i = 0; i < G / 32; ++i) {
      const int u = gi * G + lane * (G / 32) + i;
      v[i] = __fmul_rn(silu(row[u]), row[units + u]);
    }
    const float scale = warp_quantize_group<G>(v, xq + (size_t)r * units + gi * G, half);
    if (lane == 0) xs[(size_t)r * groups + gi] = scale;
  }
}

static int quant_splits(int m, int groups) {
  // Enough blocks for two an SM when the rows are few (decode batches):
  // each block of k_norm_quant runs the row's whole sum of squares.
  return std::max(1, std::min((groups + 7) / 8, (2 * current_sm_count() + m - 1) / m));
}

// Splits of the norm-free quantizers (k_quant_rows, k_silu_quant): a warp
// waits on its group's loads before it can quantize, so a block takes few
// groups a warp (up to eight blocks an SM when the rows are few).
static int free_quant_splits(int m, int groups) {
  return std::max(1, std::min((groups + 7) / 8, (8 * current_sm_count() + m - 1) / m));
}

cudaError_t launch_silu_quant(const float* g, int m, int units, int group, int half, int8_t* xq, float* xs,
                              cudaStream_t s) {
  if (units % group) return cudaErrorInvalidValue;
  const int splits = free_quant_splits(m, units / group);
  if (group == 32) k_silu_quant<32><<<dim3(m, splits), 256, 0, s>>>(g, units, half, xq, xs);
  else k_silu_quant<128><<<dim3(m, splits), 256, 0, s>>>(g, units, half, xq, xs);
  LAUNCH_CHECK();
  return cudaSuccess;
}

cudaError_t launch_norm_quant(const float* x, int m, int d, const float* w, float eps, int group, int half,
                              int8_t* xq, float* xs, cudaStream_t s, const float* scale) {
  if (!w && !scale) {
    const int splits = free_quant_splits(m, d / group);
    if (group == 32) k_quant_rows<32><<<dim3(m, splits), 256, 0, s>>>(x, d, half, xq, xs);
    else k_quant_rows<128><<<dim3(m, splits), 256, 0, s>>>(x, d, half, xq, xs);
    LAUNCH_CHECK();
    return cudaSuccess;
  }
  const int groups = d / group, splits = quant_splits(m, groups), per = (groups + splits - 1) / splits;
  const size_t row = (size_t)d * 4, wslice = w ? (size_t)per * group * 4 : 0;
  if (row > kNormSmem) return cudaErrorInvalidValue;           // d <= 12224
  const int wstage = row + wslice <= kNormSmem;                // room for the block's norm weights
  const size_t base = row + (wstage ? wslice : 0);
  const int squares = base + row <= kNormSmem;                 // room for the squares as well
  const size_t smem = base + (squares ? row : 0);
  const dim3 grid(m, splits);
  if (group == 32) k_norm_quant<32><<<grid, 256, smem, s>>>(x, d, w, eps, half, xq, xs, scale, squares, wstage);
  else k_norm_quant<128><<<grid, 256, smem, s>>>(x, d, w, eps, half, xq, xs, scale, squares, wstage);
  LAUNCH_CHECK();
  return cudaSuccess;
}

int current_sm_count() {
  static DeviceOnce once;
  static int sms[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (once.run(dev, [&] { return cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev); }) !=
      cudaSuccess)
    return 148;
  return std::max(sms[dev], 1);
}

// The shared-memory limits of every frame-count variant of k_gemv_slots,
// set on the first product on each device (whatever its row count), so a
// later call with another row count makes no driver calls.
static cudaError_t configure_gemv_slots() {
  static DeviceOnce once;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  return once.run(dev, [] {
    const void* fns[] = {(const void*)k_gemv_slots<1>, (const void*)k_gemv_slots<4>, (const void*)k_gemv_slots<8>,
                         (const void*)k_gemv_slots<16>};
    for (const void* f : fns) {
      cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (r != cudaSuccess) return r;
    }
    return cudaSuccess;
  });
}

template <int FR>
static cudaError_t gemv_slots_pass(const DMat& W, const int8_t* xq, const float* xs, int m, int mode, float* y,
                                   int ldy, float resid_mult, cudaStream_t s) {
  const int units = (mode == kEpSilu) ? W.n / 2 : W.n;
  const int per_block = (mode == kEpSilu) ? GS_WARPS / 2 : GS_WARPS;
  const size_t smem = gemv_slots_smem(W, FR);
  cudaError_t e = configure_gemv_slots();
  if (e != cudaSuccess) return e;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  // At most 8 blocks an SM; each loops over row tiles.
  const int ntiles = (units + per_block - 1) / per_block;
  const int grid = std::min(ntiles, 8 * current_sm_count());
  k_gemv_slots<FR><<<grid, GS_WARPS * 32, smem, s>>>(W, xq, xs, m, mode, y, ldy, resid_mult, units);
  return cudaGetLastError();
}

// Frames a pass: as many as the batch needs, up to 16, fewer when the
// shared memory of a wide input would not fit.
cudaError_t launch_gemv(const DMat& W, const int8_t* xq, const float* xs, int m, int mode, float* y, int ldy,
                        float resid_mult, cudaStream_t s) {
  if (W.k % 128) return cudaErrorInvalidValue;
  if (m <= 1) return gemv_slots_pass<1>(W, xq, xs, m, mode, y, ldy, resid_mult, s);
  if (m <= 4) return gemv_slots_pass<4>(W, xq, xs, m, mode, y, ldy, resid_mult, s);
  if (gemv_slots_smem(W, 16) <= 100 * 1024) return gemv_slots_pass<16>(W, xq, xs, m, mode, y, ldy, resid_mult, s);
  return gemv_slots_pass<8>(W, xq, xs, m, mode, y, ldy, resid_mult, s);
}

cudaError_t launch_qk_rope_append(float* qkv, int m, const DConfig& cfg, const float* q_norm, const float* k_norm,
                                  const float* rope, int rope_rows, const DCache& cache, const int* row_stream,
                                  const int* row_pos, int layer, cudaStream_t s) {
  k_qk_rope_append<<<m, 256, 0, s>>>(qkv, m, cfg, q_norm, k_norm, rope, rope_rows, cache, row_stream, row_pos,
                                     layer);
  LAUNCH_CHECK();
  return cudaSuccess;
}


// Final RmsNorm of `nb` rows (row stride `ldx`), then the table and the
// argmax of every row: token[b].
__global__ void __launch_bounds__(256) k_final_norm_rows(const float* x, int ldx, int d, const float* w, float eps,
                                                         float* xn, int squares) {
  extern __shared__ __align__(16) float rowv[];  // [d], then [d] squares (as k_norm_quant)
  float* sq = rowv + d;
  const float* row = x + (size_t)blockIdx.x * ldx;
  float* out = xn + (size_t)blockIdx.x * d;
  __shared__ float s_inv;
  for (int i = threadIdx.x; i < d; i += 256) {
    const float v = row[i];
    rowv[i] = v;
    if (squares) sq[i] = __fmul_rn(v, v);
  }
  __syncthreads();
  if (threadIdx.x == 0) s_inv = rms_inv(squares ? seq_sum_ahead(sq, d) : seq_sum_squares_ahead(rowv, d), d, eps);
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += 256) out[i] = __fmul_rn(rowv[i], __fmul_rn(s_inv, w[i]));
}

// The shared-memory limits of every variant of the table kernels, set once
// per device on its first table product.
static cudaError_t configure_tables() {
  static DeviceOnce once;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  return once.run(dev, [] {
    const void* fns[] = {(const void*)k_table<1>, (const void*)k_table<4>, (const void*)k_table<16>};
    for (const void* f : fns) {
      cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (r != cudaSuccess) return r;
    }
    return cudaFuncSetAttribute(k_table_rows<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)table_rows_smem(16));
  });
}

template <int B>
static cudaError_t table_pass(const DTable& T, const float* xn, int nb, float mult, float* logits, float* best_val,
                              int* best_idx, cudaStream_t s) {
  size_t smem = (size_t)T.k * B * 4;
  cudaError_t e = configure_tables();
  if (e != cudaSuccess) return e;
  int blocks = table_blocks(T.n);
  k_table<B><<<blocks, 256, smem, s>>>(T, xn, nb, mult, logits, best_val, best_idx, blocks);
  return cudaGetLastError();
}

template <int B>
static cudaError_t table_rows_pass(const DTable& T, const float* xn, int nb, float mult, float* logits,
                                   float* best_val, int* best_idx, cudaStream_t s) {
  size_t smem = table_rows_smem(B);
  cudaError_t e = configure_tables();
  if (e != cudaSuccess) return e;
  int blocks = table_blocks(T.n);
  k_table_rows<B><<<blocks, 256, smem, s>>>(T, xn, nb, mult, logits, best_val, best_idx, blocks);
  return cudaGetLastError();
}

cudaError_t launch_key_tokens(const unsigned long long* keys, int nb, int* token, cudaStream_t s) {
  k_key_token<<<(nb + 255) / 256, 256, 0, s>>>(keys, nb, token);
  LAUNCH_CHECK();
  return cudaSuccess;
}

cudaError_t launch_final(const float* x, int ldx, int nb, const float* norm_w, const DConfig& cfg, const DTable& T,
                         float* xn, float* logits, float* best_val, int* best_idx, int* token, cudaStream_t s,
                         unsigned long long* keys, int v0) {
  const int squares = (size_t)cfg.d * 8 <= kNormSmem;  // room for the squares (hidden size < 6144)
  k_final_norm_rows<<<nb, 256, (size_t)cfg.d * (squares ? 8 : 4), s>>>(x, ldx, cfg.d, norm_w, cfg.eps, xn, squares);
  LAUNCH_CHECK();
  float mult = (cfg.logits_scaling == 1.0f) ? 1.0f : 1.0f / cfg.logits_scaling;
  int blocks = table_blocks(T.n);
  cudaError_t e = launch_table(T, xn, nb, mult, logits, best_val, best_idx, s);
  if (e != cudaSuccess) return e;
  if (keys) k_argmax_key<<<nb, 32, 0, s>>>(best_val, best_idx, blocks, v0, keys);
  else k_argmax<<<nb, 32, 0, s>>>(best_val, best_idx, blocks, token);
  LAUNCH_CHECK();
  return cudaSuccess;
}

cudaError_t launch_table(const DTable& T, const float* xn, int nb, float mult, float* logits, float* best_val,
                         int* best_idx, cudaStream_t s) {
  int blocks = table_blocks(T.n);
  // Passes of up to 16 streams: two blocks an SM (k_table_rows<16> keeps
  // 64 f32 accumulators a thread), measured faster than passes of 32 at one
  // block an SM (C5 decode 5405 against 5265 tok/s) although the table is
  // read once per pass.
  const int pass = TABLE_MAX_B;
  for (int b0 = 0; b0 < nb; b0 += pass) {
    int n = std::min(pass, nb - b0);
    const float* xb = xn + (size_t)b0 * T.k;
    float* lg = logits ? logits + (size_t)b0 * T.n : nullptr;
    float* bv = best_val + (size_t)b0 * blocks;
    int* bi = best_idx + (size_t)b0 * blocks;
    cudaError_t e;
    if (n == 1) e = table_pass<1>(T, xb, n, mult, lg, bv, bi, s);
    else if (n <= 4) e = table_pass<4>(T, xb, n, mult, lg, bv, bi, s);
    else if (T.k % TB_KC) e = table_pass<16>(T, xb, n, mult, lg, bv, bi, s);
    else e = table_rows_pass<16>(T, xb, n, mult, lg, bv, bi, s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int table_blocks(int n) { return (n + TABLE_ROWS - 1) / TABLE_ROWS; }
int table_max_streams() { return TABLE_MAX_B; }

}  // namespace trit
