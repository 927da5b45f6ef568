// The persistent batch-1 decode: every greedy step of one generation in
// one cooperative kernel (one block per SM). A step runs the layers of
// CausalLm::hidden (src/models/parts/causal_lm.rs:410-481) as five phases
// separated by grid barriers:
//   P1 qkv      every block: RmsNorm + quantize of x (redundant, 4 KB), then
//               its slice of the stacked q/k/v rows
//   P2 attend   block (kv head, split): q/k norm, RoPE, K/V append (split 0),
//               a key range of GQA attention; the last split of a head joins
//               the splits and quantizes the head's output
//   P3 o        every block: its rows of o_proj, added to x (residual)
//   P4 gate_up  every block: RmsNorm + quantize of x, its units of gate/up,
//               h = silu(gate) * up
//   P5 down     every block: quantize h, its rows of down_proj, added to x
// then the final RmsNorm, the block's slice of the token table (f32 math),
// and a per-block argmax that every block reduces to the same token.
// Weights of the next phases are prefetched into L2 while a block waits.
//
// Waits are bounded: a barrier that does not complete within ~2^22 polls
// sets *status and every block returns; the host reports the error.
#include <cuda_runtime.h>

#include "device.cuh"
#include "kernels.h"

namespace trit {
namespace {

constexpr int DT = 512;          // threads per block
constexpr int DW = DT / 32;      // warps per block
constexpr int TAB_TILE = 128;    // table rows per tile (4 threads a row)
constexpr int TAB_SLAB = 128;    // bytes of a row per pipeline stage
constexpr int TAB_STAGES = 4;
constexpr int TAB_PITCH = TAB_SLAB + 16;
constexpr long long SPIN_LIMIT = 1ll << 22;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *(const volatile int*)p; }

// Grid barrier on a counter that only grows: barrier b of this launch
// waits for b * gridDim.x arrivals. Returns false when the wait ran out
// (or another block gave up): the caller returns at once.
__device__ bool grid_barrier(unsigned* counter, unsigned& target, int* status, volatile int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    __threadfence();
    atomicAdd(counter, 1u);
    long long spins = 0;
    int bad = 0;
    while (ld_acquire(counter) < target) {
      if (++spins > SPIN_LIMIT) {
        atomicCAS(status, 0, 1);
        bad = 1;
        break;
      }
      if ((spins & 1023) == 0 && ld_volatile(status) != 0) {
        bad = 1;
        break;
      }
    }
    __threadfence();
    *s_flag = bad;
  }
  __syncthreads();
  return *s_flag == 0;
}

__device__ __forceinline__ int split_at(int n, int part, int parts) { return (int)((long long)n * part / parts); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

struct Shared {
  float* xf;       // [d]: x, normed x (final), or h
  int8_t* xq;      // [kmax]
  float* xs;       // [kmax / 32]
  int* part;       // [rows][groups] group dots
  float* out;      // [rows]
  float* red;      // [64]
  float* att;      // attention scratch
  uint8_t* tab;    // table stages
  int* flag;       // [4]
};

// Block reductions over all DT threads.
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < DW; ++i) t = __fadd_rn(t, red[i]);
    red[DW] = t;
  }
  __syncthreads();
  return red[DW];
}

// RmsNorm (layers.rs:135-144) of src (d values) with weight w (null: no
// norm), then Quantized::grouped of the result into xq / xs.
__device__ void norm_quant(const float* src, int d, const float* w, float eps, int G, bool half, Shared& S) {
  if (src != S.xf) {
    for (int i = threadIdx.x; i < d; i += DT) S.xf[i] = src[i];
  }
  __syncthreads();
  float inv = 1.0f;
  if (w) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < d; i += DT) s = __fadd_rn(s, __fmul_rn(S.xf[i], S.xf[i]));
    float t = block_sum(s, S.red);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)d), eps)));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = d / G;
  for (int g = warp; g < groups; g += DW) {
    if (G == 32) {
      float v[1];
      int kk = g * 32 + lane;
      v[0] = w ? __fmul_rn(S.xf[kk], __fmul_rn(inv, w[kk])) : S.xf[kk];
      float sc = warp_quantize_group<32>(v, S.xq + g * 32, half);
      if (lane == 0) S.xs[g] = sc;
    } else {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int kk = g * 128 + lane * 4 + i;
        v[i] = w ? __fmul_rn(S.xf[kk], __fmul_rn(inv, w[kk])) : S.xf[kk];
      }
      float sc = warp_quantize_group<128>(v, S.xq + g * 128, half);
      if (lane == 0) S.xs[g] = sc;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ int4 load16(const DMat& W, int row, int chunk) {
  if (W.kind == kTernary) {
    uint32_t word = __ldg((const uint32_t*)W.codes + (size_t)row * (W.k / 16) + chunk);
    return make_int4((int)word, 0, 0, 0);
  }
  return ld_stream((const int8_t*)W.codes + (size_t)row * W.k + (size_t)chunk * 16);
}

// Group dots of `nrows` rows (row(lr) gives the weight row of local row
// lr) against the activations in S.xq, into S.part[lr][g]; then one
// thread per local row runs the group chain of int8.rs:560-570 in order
// and stores the output in S.out[lr].
template <class RowOf>
__device__ void gemv_rows(const DMat& W, int nrows, RowOf row_of, Shared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = W.k, chunks = k / 16, groups = k / W.agroup, lpg = W.agroup / 16;
  constexpr int MAXC = 8;
  for (int lr = warp; lr < nrows; lr += DW) {
    const int row = row_of(lr);
    for (int base = 0; base < chunks; base += 32 * MAXC) {
      int4 w[MAXC];
#pragma unroll
      for (int j = 0; j < MAXC; ++j) {
        int c = base + lane + 32 * j;
        w[j] = c < chunks ? load16(W, row, c) : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < MAXC; ++j) {
        int c = base + lane + 32 * j;
        if (base + 32 * j >= chunks) break;  // warp-uniform
        int dot = 0;
        if (c < chunks) {
          int4 a = ((const int4*)S.xq)[c];
          dot = (W.kind == kTernary) ? dot16_ternary((uint32_t)w[j].x, a) : dot16(w[j], a);
        }
        for (int o = 1; o < lpg; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (c < chunks && (lane % lpg) == 0) S.part[lr * groups + c / lpg] = dot;
      }
    }
  }
  __syncthreads();
  for (int lr = threadIdx.x; lr < nrows; lr += DT) {
    const int row = row_of(lr);
    const int* p = S.part + lr * groups;
    float acc = 0.0f;
    for (int g = 0; g < groups; ++g) acc = __fmaf_rn((float)p[g], __fmul_rn(weight_scale(W, row, g), S.xs[g]), acc);
    S.out[lr] = acc;
  }
  __syncthreads();
}

__device__ __forceinline__ void prefetch_rows(const DMat& W, int r0, int r1) {
  if (r1 <= r0) return;
  size_t code_row = (W.kind == kTernary) ? (size_t)W.k / 4 : (size_t)W.k;
  prefetch_l2((const int8_t*)W.codes + (size_t)r0 * code_row, (uint32_t)((r1 - r0) * code_row));
  size_t scale_row = W.kind == kQ8_0 ? (size_t)(W.k / 32) * 2 : W.kind == kInt8Row ? 4 : (size_t)(W.k / 128) * 4;
  prefetch_l2((const int8_t*)W.scales + (size_t)r0 * scale_row, (uint32_t)((r1 - r0) * scale_row));
}

// The slices of a layer's weights that block c reads, prefetched into L2.
__device__ void prefetch_layer(const DLayer& L, const DConfig& cfg, int c, int nb, bool qkv, bool rest) {
  if (threadIdx.x != 0) return;
  if (qkv) prefetch_rows(L.qkv, split_at(L.qkv.n, c, nb), split_at(L.qkv.n, c + 1, nb));
  if (rest) {
    prefetch_rows(L.out, split_at(L.out.n, c, nb), split_at(L.out.n, c + 1, nb));
    int u0 = split_at(cfg.ffn, c, nb), u1 = split_at(cfg.ffn, c + 1, nb);
    prefetch_rows(L.gate_up, u0, u1);
    prefetch_rows(L.gate_up, cfg.ffn + u0, cfg.ffn + u1);
    prefetch_rows(L.down, split_at(L.down.n, c, nb), split_at(L.down.n, c + 1, nb));
  }
}

// ------------------------------------------------------------ attention --
// Block (kvh, s) of the P2 phase. Scores are the reference's sequential fma
// chains; the softmax of the block's keys and the join across blocks run
// in another order than the reference's (tolerance).
__device__ void attend(const DecodeArgs& a, const DLayer& L, int layer, int pos, int kvh, int s, int S_splits,
                       unsigned* counters, Shared& S) {
  const DConfig& cfg = a.cfg;
  const int hd = 128, qpk = cfg.heads / cfg.kv_heads, qd = cfg.heads * hd, kvd = cfg.kv_heads * hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = pos + 1, len = (T + S_splits - 1) / S_splits;
  const int j0 = min(T, s * len), j1 = min(T, j0 + len), nk = j1 - j0;
  float* q = S.att;                 // [qpk][128]
  float* kf = q + qpk * hd;         // [128]
  float* vf = kf + hd;              // [128]
  float* sc = vf + hd;              // [qpk][len]
  const DCache& cache = a.cache;
  const float* sn = a.rope + (size_t)min(pos, a.rope_rows - 1) * hd;
  const float* cs = sn + hd / 2;
  // Warp 0: k, warp 1: v, warps 2..: q heads.
  for (int h = warp; h < 2 + qpk; h += DW) {
    const float* src = (h == 0) ? a.qkv + qd + kvh * hd : (h == 1) ? a.qkv + qd + kvd + kvh * hd
                                                                   : a.qkv + (kvh * qpk + h - 2) * hd;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = src[lane * 4 + i];
    if (h != 1) {
      const float* nw = (h == 0) ? L.k_norm : L.q_norm;
      if (nw) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        ss = warp_sum(ss);
        float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), cfg.eps)));
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], __fmul_rn(inv, nw[lane * 4 + i]));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
        int idx = (lane & 15) * 4 + i;
        float c = cs[idx], sgn = sn[idx];
        v[i] = (lane < 16) ? __fsub_rn(__fmul_rn(v[i], c), __fmul_rn(partner, sgn))
                           : __fadd_rn(__fmul_rn(v[i], c), __fmul_rn(partner, sgn));
      }
    }
    if (h >= 2) {
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float x = cfg.has_q_scale ? __fmul_rn(v[i], cfg.q_scale) : v[i];
        q[(h - 2) * hd + lane * 4 + i] = __fmul_rn(x, scale);
      }
    } else {
      float* dst = (h == 0) ? kf : vf;
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[lane * 4 + i] = cache.f16 ? round_f16(v[i]) : v[i];
      if (s == 0) {
        int page = cache.page_table[(size_t)a.stream * cache.pages_per_stream + pos / cache.page_tokens];
        size_t off = kv_offset(cache, cfg, page, layer, h, kvh, pos % cache.page_tokens) + lane * 4;
        if (cache.f16) {
#pragma unroll
          for (int i = 0; i < 4; ++i) ((__half*)cache.pool)[off + i] = __float2half_rn(v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) ((float*)cache.pool)[off + i] = v[i];
        }
      }
    }
  }
  __syncthreads();
  // Scores: one thread per (q head, key).
  for (int p = threadIdx.x; p < qpk * nk; p += DT) {
    int qh = p / nk, jj = p % nk, j = j0 + jj;
    const float* qv = q + qh * hd;
    float acc = 0.0f;
    if (j == pos) {
      for (int e = 0; e < hd; ++e) acc = __fmaf_rn(qv[e], kf[e], acc);
    } else {
      int page = cache.page_table[(size_t)a.stream * cache.pages_per_stream + j / cache.page_tokens];
      size_t off = kv_offset(cache, cfg, page, layer, 0, kvh, j % cache.page_tokens);
      if (cache.f16) {
        const int4* kp = (const int4*)((const __half*)cache.pool + off);
        for (int i = 0; i < 16; ++i) {
          int4 raw = kp[i];
          const __half2* h2 = (const __half2*)&raw;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float2 f = __half22float2(h2[t]);
            acc = __fmaf_rn(qv[8 * i + 2 * t], f.x, acc);
            acc = __fmaf_rn(qv[8 * i + 2 * t + 1], f.y, acc);
          }
        }
      } else {
        const float4* kp = (const float4*)((const float*)cache.pool + off);
        for (int i = 0; i < 32; ++i) {
          float4 f = kp[i];
          acc = __fmaf_rn(qv[4 * i], f.x, acc);
          acc = __fmaf_rn(qv[4 * i + 1], f.y, acc);
          acc = __fmaf_rn(qv[4 * i + 2], f.z, acc);
          acc = __fmaf_rn(qv[4 * i + 3], f.w, acc);
        }
      }
    }
    sc[qh * len + jj] = acc;
  }
  __syncthreads();
  // Softmax of the block's keys: warp qh takes head qh.
  float* stat = sc + qpk * len;  // [qpk][2]: max, sum
  if (warp < qpk) {
    float mx = -INFINITY;
    for (int jj = lane; jj < nk; jj += 32) mx = fmaxf(mx, sc[warp * len + jj]);
    mx = warp_max(mx);
    float sum = 0.0f;
    for (int jj = lane; jj < nk; jj += 32) {
      float e = cephes_exp(__fsub_rn(sc[warp * len + jj], mx));
      sc[warp * len + jj] = e;
      sum = __fadd_rn(sum, e);
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      stat[2 * warp] = nk ? mx : -INFINITY;
      stat[2 * warp + 1] = nk ? sum : 0.0f;
    }
  }
  __syncthreads();
  // Weighted V sums: one thread per (q head, dimension).
  float* part = a.att_part + ((size_t)(kvh * S_splits + s) * qpk) * (hd + 2);
  for (int p = threadIdx.x; p < qpk * hd; p += DT) {
    int qh = p / hd, e = p % hd;
    float acc = 0.0f;
    for (int jj = 0; jj < nk; ++jj) {
      int j = j0 + jj;
      float vv;
      if (j == pos) {
        vv = vf[e];
      } else {
        int page = cache.page_table[(size_t)a.stream * cache.pages_per_stream + j / cache.page_tokens];
        size_t off = kv_offset(cache, cfg, page, layer, 1, kvh, j % cache.page_tokens) + e;
        vv = cache.f16 ? __half2float(((const __half*)cache.pool)[off]) : ((const float*)cache.pool)[off];
      }
      acc = __fmaf_rn(sc[qh * len + jj], vv, acc);
    }
    part[qh * (hd + 2) + 2 + e] = acc;
    if (e == 0) {
      part[qh * (hd + 2)] = stat[2 * qh];
      part[qh * (hd + 2) + 1] = stat[2 * qh + 1];
    }
  }
  // The last block of this kv head to finish joins the splits.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned old = atomicAdd(&counters[kvh], 1u);
    S.flag[1] = (old == (unsigned)S_splits - 1);
  }
  __syncthreads();
  if (!S.flag[1]) return;
  __threadfence();
  const float* base = a.att_part + (size_t)kvh * S_splits * qpk * (hd + 2);
  float* outv = sc;  // [qpk][128], reuse
  for (int p = threadIdx.x; p < qpk * hd; p += DT) {
    int qh = p / hd, e = p % hd;
    float mx = -INFINITY;
    for (int t = 0; t < S_splits; ++t) {
      const float* pp = base + ((size_t)t * qpk + qh) * (hd + 2);
      if (pp[1] > 0.0f) mx = fmaxf(mx, pp[0]);
    }
    float l = 0.0f, acc = 0.0f;
    for (int t = 0; t < S_splits; ++t) {
      const float* pp = base + ((size_t)t * qpk + qh) * (hd + 2);
      if (!(pp[1] > 0.0f)) continue;
      float wgt = cephes_exp(__fsub_rn(pp[0], mx));
      l = __fmaf_rn(wgt, pp[1], l);
      acc = __fmaf_rn(wgt, pp[2 + e], acc);
    }
    outv[qh * hd + e] = __fdiv_rn(acc, l);
  }
  __syncthreads();
  // Quantize each head's output (groups of 32 or 128 lie inside a head).
  const DMat& O = L.out;
  const int G = O.agroup;
  for (int g = warp; g < qpk * hd / G; g += DW) {
    int qh0 = kvh * qpk;
    int8_t* dst = a.attq + qh0 * hd + g * G;
    float sc2;
    if (G == 32) {
      float v[1] = {outv[g * 32 + lane]};
      sc2 = warp_quantize_group<32>(v, dst, O.half);
    } else {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = outv[g * 128 + lane * 4 + i];
      sc2 = warp_quantize_group<128>(v, dst, O.half);
    }
    if (lane == 0) a.atts[(qh0 * hd) / G + g] = sc2;
  }
  if (threadIdx.x == 0) counters[kvh] = 0;
}

// ---------------------------------------------------------------- table --
// The block's slice of the token table (forward_rows' last product,
// causal_lm.rs:386-388) with f32 math in the lane order of the AVX-512
// tile, codes streamed through shared memory by cp.async, and the block's
// best (value, index).
__device__ void table_slice(const DecodeArgs& a, int v0, int v1, int step, Shared& S, float* best_v, int* best_i) {
  const DTable& T = a.table;
  const int t = threadIdx.x, q = t & 3, rl = t >> 2;
  const int slabs = T.k / TAB_SLAB;
  const int tiles = (v1 - v0 + TAB_TILE - 1) / TAB_TILE;
  const int items = tiles * slabs;
  const float mult = (a.cfg.logits_scaling == 1.0f) ? 1.0f : __fdiv_rn(1.0f, a.cfg.logits_scaling);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  auto issue = [&](int item) {
    if (item < items) {
      int tile = item / slabs, slab = item % slabs;
      uint8_t* stage = S.tab + (item % TAB_STAGES) * TAB_TILE * TAB_PITCH;
      // 128 rows x 128 bytes = 1024 chunks of 16 bytes: two a thread.
      for (int c = t; c < TAB_TILE * (TAB_SLAB / 16); c += DT) {
        int r = c / (TAB_SLAB / 16), cc = c % (TAB_SLAB / 16);
        int row = v0 + tile * TAB_TILE + r;
        if (row < v1) cp_async16(stage + r * TAB_PITCH + cc * 16, T.codes + (size_t)row * T.k + slab * TAB_SLAB + cc * 16);
      }
    }
    cp_commit();
  };
  for (int i = 0; i < TAB_STAGES - 1; ++i) issue(i);
  float lanes[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int item = 0; item < items; ++item) {
    issue(item + TAB_STAGES - 1);
    cp_wait<TAB_STAGES - 1>();
    __syncthreads();
    int tile = item / slabs, slab = item % slabs;
    int row = v0 + tile * TAB_TILE + rl;
    const uint8_t* stage = S.tab + (item % TAB_STAGES) * TAB_TILE * TAB_PITCH + rl * TAB_PITCH;
    if (row < v1) {
#pragma unroll
      for (int st = 0; st < TAB_SLAB / 16; ++st) {
        int kk = slab * TAB_SLAB + 16 * st + 4 * q;
        uint32_t word = *(const uint32_t*)(stage + 16 * st + 4 * q) ^ 0x80808080u;
        float s = table_scale(T, row, kk / 32);
        float4 xv = *(const float4*)(S.xf + kk);
        lanes[0] = __fmaf_rn(xv.x, __fmul_rn(byte_to_float(word, 0), s), lanes[0]);
        lanes[1] = __fmaf_rn(xv.y, __fmul_rn(byte_to_float(word, 1), s), lanes[1]);
        lanes[2] = __fmaf_rn(xv.z, __fmul_rn(byte_to_float(word, 2), s), lanes[2]);
        lanes[3] = __fmaf_rn(xv.w, __fmul_rn(byte_to_float(word, 3), s), lanes[3]);
      }
    }
    if (slab == slabs - 1) {
      // The row is done: _mm512_reduce_add_ps across the 4 threads.
      float s8[4], s4[4];
#pragma unroll
      for (int l = 0; l < 4; ++l) s8[l] = __fadd_rn(lanes[l], __shfl_down_sync(0xffffffffu, lanes[l], 2));
#pragma unroll
      for (int l = 0; l < 4; ++l) s4[l] = __fadd_rn(s8[l], __shfl_down_sync(0xffffffffu, s8[l], 1));
      float v = __fadd_rn(__fadd_rn(s4[0], s4[2]), __fadd_rn(s4[1], s4[3]));
      if (q == 0 && row < v1) {
        if (mult != 1.0f) v = __fmul_rn(v, mult);
        if (a.logits) a.logits[(size_t)step * T.n + row] = v;
        if (v > bv) { bv = v; bi = row; }  // rows rise: the first maximum stays
      }
#pragma unroll
      for (int l = 0; l < 4; ++l) lanes[l] = 0.0f;
    }
    __syncthreads();
  }
  cp_wait<0>();
  // Block best: the largest value, the lowest index among equals.
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  __syncthreads();
  if ((t & 31) == 0) {
    S.red[t >> 5] = bv;
    ((int*)S.red)[32 + (t >> 5)] = bi;
  }
  __syncthreads();
  if (t == 0) {
    for (int w = 1; w < DW; ++w) {
      float ov = S.red[w];
      int oi = ((int*)S.red)[32 + w];
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    *best_v = bv;
    *best_i = bi;
  }
}

__global__ void __launch_bounds__(DT, 1) k_decode(DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const DConfig& cfg = a.cfg;
  const int c = blockIdx.x, nb = gridDim.x;
  const int hd = 128, qd = cfg.heads * hd, kvd = cfg.kv_heads * hd, nqkv = qd + 2 * kvd;
  const int kmax = max(max(cfg.d, qd), cfg.ffn);
  const int S_splits = max(1, nb / cfg.kv_heads);
  // Shared memory plan (see decode_smem).
  Shared S;
  uint8_t* p = smem;
  S.flag = (int*)p; p += 64;
  S.red = (float*)p; p += 64 * 4;
  S.xf = (float*)p; p += (size_t)kmax * 4;
  S.xq = (int8_t*)p; p += (size_t)kmax;
  S.xs = (float*)p; p += (size_t)(kmax / 32) * 4;
  S.out = (float*)p; p += 512 * 4;
  S.part = (int*)p;          // union with attention and table scratch
  S.att = (float*)p;
  S.tab = p;
  unsigned* counter = a.sync;
  unsigned* att_counters = a.sync + 4;
  unsigned target = 0;
  if (threadIdx.x == 0) S.flag[0] = 0;
  __syncthreads();

  for (int i = 0; i < a.steps; ++i) {
    // Every block reduced the same token at the end of the last step.
    const int token = (i == 0) ? a.tokens[0] : S.flag[2];
    bool stopped = false;
    for (int s = 0; s < a.nstop; ++s) stopped |= a.stop[s] == token;
    if (stopped) {
      if (c == 0 && threadIdx.x == 0) *a.count = i;
      return;
    }
    const int pos = a.first_pos + i;
    // x = the token's embedding (causal_lm.rs:347-355, hidden :414), into
    // S.xf for layer 0's norm; block 0 also stores it as the residual.
    const DTable& E = a.embed;
    for (int kk = threadIdx.x; kk < cfg.d; kk += DT) {
      float v = __fmul_rn((float)E.codes[(size_t)token * E.k + kk], table_scale(E, token, kk / 32));
      if (cfg.embedding_multiplier != 1.0f) v = __fmul_rn(v, cfg.embedding_multiplier);
      if (c == 0) a.x[kk] = v;
      S.xf[kk] = v;
    }
    __syncthreads();
    for (int l = 0; l < cfg.layers; ++l) {
      const DLayer& L = a.layers[l];
      // P1: qkv.
      prefetch_layer(L, cfg, c, nb, false, true);
      if (l + 1 < cfg.layers) prefetch_layer(a.layers[l + 1], cfg, c, nb, true, false);
      norm_quant(l == 0 ? S.xf : a.x, cfg.d, L.norm_attn, cfg.eps, L.qkv.agroup, L.qkv.half, S);
      {
        int r0 = split_at(nqkv, c, nb), r1 = split_at(nqkv, c + 1, nb);
        gemv_rows(L.qkv, r1 - r0, [&](int lr) { return r0 + lr; }, S);
        for (int lr = threadIdx.x; lr < r1 - r0; lr += DT) a.qkv[r0 + lr] = S.out[lr];
      }
      if (!grid_barrier(counter, target, a.status, S.flag)) return;
      // P2: attention.
      if (c < cfg.kv_heads * S_splits) attend(a, L, l, pos, c / S_splits, c % S_splits, S_splits, att_counters, S);
      if (!grid_barrier(counter, target, a.status, S.flag)) return;
      // P3: o_proj + residual.
      {
        const int groups = qd / L.out.agroup;
        for (int j = threadIdx.x; j < qd / 16; j += DT) ((int4*)S.xq)[j] = ((const int4*)a.attq)[j];
        for (int j = threadIdx.x; j < groups; j += DT) S.xs[j] = a.atts[j];
        __syncthreads();
        int r0 = split_at(cfg.d, c, nb), r1 = split_at(cfg.d, c + 1, nb);
        gemv_rows(L.out, r1 - r0, [&](int lr) { return r0 + lr; }, S);
        for (int lr = threadIdx.x; lr < r1 - r0; lr += DT) {
          float o = S.out[lr];
          float xv = a.x[r0 + lr];
          a.x[r0 + lr] = (cfg.residual_multiplier == 1.0f) ? __fadd_rn(xv, o)
                                                           : __fadd_rn(xv, __fmul_rn(cfg.residual_multiplier, o));
        }
      }
      if (!grid_barrier(counter, target, a.status, S.flag)) return;
      // P4: gate_up, h = silu(gate) * up.
      norm_quant(a.x, cfg.d, L.norm_mlp, cfg.eps, L.gate_up.agroup, L.gate_up.half, S);
      {
        int u0 = split_at(cfg.ffn, c, nb), u1 = split_at(cfg.ffn, c + 1, nb), nu = u1 - u0;
        gemv_rows(L.gate_up, 2 * nu, [&](int lr) { return lr < nu ? u0 + lr : cfg.ffn + u0 + lr - nu; }, S);
        for (int lr = threadIdx.x; lr < nu; lr += DT) a.h[u0 + lr] = __fmul_rn(silu(S.out[lr]), S.out[nu + lr]);
      }
      if (!grid_barrier(counter, target, a.status, S.flag)) return;
      // P5: down + residual.
      norm_quant(a.h, cfg.ffn, nullptr, cfg.eps, L.down.agroup, L.down.half, S);
      {
        int r0 = split_at(cfg.d, c, nb), r1 = split_at(cfg.d, c + 1, nb);
        gemv_rows(L.down, r1 - r0, [&](int lr) { return r0 + lr; }, S);
        for (int lr = threadIdx.x; lr < r1 - r0; lr += DT) {
          float o = S.out[lr];
          float xv = a.x[r0 + lr];
          a.x[r0 + lr] = (cfg.residual_multiplier == 1.0f) ? __fadd_rn(xv, o)
                                                           : __fadd_rn(xv, __fmul_rn(cfg.residual_multiplier, o));
        }
      }
      if (!grid_barrier(counter, target, a.status, S.flag)) return;
    }
    // Final RmsNorm (f32, no quantization) into S.xf, then the table slice.
    {
      for (int kk = threadIdx.x; kk < cfg.d; kk += DT) S.xf[kk] = a.x[kk];
      __syncthreads();
      float ss = 0.0f;
      for (int kk = threadIdx.x; kk < cfg.d; kk += DT) ss = __fadd_rn(ss, __fmul_rn(S.xf[kk], S.xf[kk]));
      float tsum = block_sum(ss, S.red);
      float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tsum, (float)cfg.d), cfg.eps)));
      for (int kk = threadIdx.x; kk < cfg.d; kk += DT) S.xf[kk] = __fmul_rn(S.xf[kk], __fmul_rn(inv, a.final_norm[kk]));
      __syncthreads();
      int v0 = split_at(a.table.n, c, nb), v1 = split_at(a.table.n, c + 1, nb);
      table_slice(a, v0, v1, i + 1, S, a.best_val + c, a.best_idx + c);
    }
    if (!grid_barrier(counter, target, a.status, S.flag)) return;
    // Every block reduces the per-block bests to the same token.
    if (threadIdx.x < 32) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int b = threadIdx.x; b < nb; b += 32) {
        float v = a.best_val[b];
        int ix = a.best_idx[b];
        if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (threadIdx.x == 0) {
        int tok = (bi == 0x7fffffff) ? 0 : bi;
        S.flag[2] = tok;
        if (c == 0) a.tokens[i + 1] = tok;
      }
    }
    __syncthreads();
    // Every block has read best_* before any block writes them again: the
    // next write comes after 5 * layers more barriers.
  }
  if (c == 0 && threadIdx.x == 0) *a.count = a.steps;
}

size_t decode_smem(const DConfig& cfg) {
  const int hd = 128, qd = cfg.heads * hd, kvd = cfg.kv_heads * hd, nqkv = qd + 2 * kvd;
  const int kmax = std::max(std::max(cfg.d, qd), cfg.ffn);
  size_t head = 64 + 64 * 4 + (size_t)kmax * 4 + kmax + (size_t)(kmax / 32) * 4 + 512 * 4;
  (void)nqkv;
  return head;
}

}  // namespace

int decode_grid(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return 0;
  return prop.multiProcessorCount;
}

// Shared memory of the union region: the largest of the GEMV group dots,
// the attention scratch and the table stages.
static size_t union_smem(const DConfig& cfg, int grid) {
  const int hd = 128, qd = cfg.heads * hd, kvd = cfg.kv_heads * hd, nqkv = qd + 2 * kvd;
  auto rows = [&](int n) { return (n + grid - 1) / grid + 1; };
  size_t gemv = 0;
  gemv = std::max(gemv, (size_t)rows(nqkv) * (cfg.d / 32) * 4);
  gemv = std::max(gemv, (size_t)rows(cfg.d) * (qd / 32) * 4);
  gemv = std::max(gemv, (size_t)2 * rows(cfg.ffn) * (cfg.d / 32) * 4);
  gemv = std::max(gemv, (size_t)rows(cfg.d) * (cfg.ffn / 32) * 4);
  int qpk = cfg.heads / cfg.kv_heads;
  int splits = std::max(1, grid / cfg.kv_heads);
  (void)splits;
  size_t att_cap = 0;  // filled at launch (depends on the position)
  size_t tab = (size_t)TAB_STAGES * TAB_TILE * TAB_PITCH;
  (void)qpk;
  return std::max(std::max(gemv, tab), att_cap);
}

cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t s) {
  const int qpk = a.cfg.heads / a.cfg.kv_heads;
  const int splits = std::max(1, grid / a.cfg.kv_heads);
  const int max_pos = a.first_pos + a.steps;  // the last position fed
  const int len = (max_pos + 1 + splits - 1) / splits;
  size_t att = ((size_t)qpk * 128 + 2 * 128 + (size_t)qpk * len + 2 * qpk + (size_t)qpk * 128) * 4;
  size_t smem = decode_smem(a.cfg) + std::max(union_smem(a.cfg, grid), att);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode, DT, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
  DecodeArgs args = a;
  void* params[] = {&args};
  return cudaLaunchCooperativeKernel((const void*)k_decode, dim3(grid), dim3(DT), params, smem, s);
}

}  // namespace trit
