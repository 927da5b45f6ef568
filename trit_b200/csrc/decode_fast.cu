// The persistent batch-1 decode of the default ("exact": false) path: every
// greedy step of one generation in one cooperative kernel, one block per
// SM, computing what CausalLm::hidden and forward_rows compute
// (src/models/parts/causal_lm.rs:352-481) with the reference's quantizers
// and integer products, but with its floating-point sums in tree order.
// Tokens stay the reference's; logits move by rounding only.
//
// A layer takes four hand-offs between blocks instead of five:
//   P1 qkv       every block: RmsNorm + quantize of x, its rows of the
//                stacked q/k/v product
//   P2 attend+o  the blocks are split into one group per kv head; every
//                block of group g runs the whole attention of kv head g
//                (q/k norm, RoPE, the keys in tiles with an online
//                softmax), quantizes the heads' output (groups of 32 or
//                128 lie inside a head, so the codes are the reference's),
//                and multiplies it by its rows of o_proj restricted to the
//                group's columns: a partial sum of o per group
//   P4 gate_up   every block: x += the group partials (summed in group
//                order), RmsNorm + quantize, its gate/up units,
//                h = silu(gate) * up
//   P5 down      every block: quantize h, its rows of down_proj, added to x
// then the final RmsNorm, the block's slice of the token table (f32 math)
// and the argmax, which every block reduces from all blocks' bests.
//
// Values travel between blocks as 64-bit LL words {data, tag} (ll.cuh);
// every poll is bounded and reports through *status. Each block holds the
// whole residual stream x in shared memory. Weights are staged into shared
// memory by cp.async before the block waits for its input.
//
// KV cache: block 0 of group g appends the step's key and value; the other
// blocks of the group read them in later steps. The appending threads
// reach a fence before the block's next hand-off word, and every block
// fences at the start of each step, so the rows are visible when read.
#include <cuda_runtime.h>

#include <algorithm>

#include "device.cuh"
#include "kernels.h"
#include "ll.cuh"

namespace trit {
namespace {

constexpr int FT = 512;           // threads per block
constexpr int FW = FT / 32;       // warps per block
constexpr int FSTAGE = 40 * 1024; // bytes of one weight staging buffer
constexpr int FPASS = 8;          // LL words a thread keeps in flight (16 for the group partials)
constexpr int FOUT = 512;         // product rows of a block in one phase
constexpr int FPART = 512;        // slice partials of one weight batch
constexpr int TSTAGES = 6;        // the most token-table rows in flight per warp

struct FastLayout {
  int qkv, opart, h, xb, best, total;
  __host__ __device__ FastLayout(const DConfig& c, int grid) {
    const int nqkv = (c.heads + 2 * c.kv_heads) * 128;
    qkv = 0;
    opart = nqkv;
    h = opart + c.kv_heads * c.d;
    xb = h + c.ffn;
    best = xb + c.d;
    total = best + 2 * grid;
  }
};

__host__ __device__ inline int imax(int a, int b) { return a > b ? a : b; }
__host__ __device__ inline size_t zmax(size_t a, size_t b) { return a > b ? a : b; }
__host__ __device__ inline int kmax_of(const DConfig& c) { return imax(imax(c.d, c.heads * 128), c.ffn); }
// The table phase keeps the normed x with 4 floats of padding after every
// 16 (conflict-free 16-byte reads by lanes 16 values apart).
__host__ __device__ inline int xf_floats(const DConfig& c) { return imax(kmax_of(c), c.d + c.d / 4) + 16; }
__host__ __device__ inline int pad16(int v) { return (v + 15) / 16 * 16; }

// Bytes of the head region (everything outside the union).
__host__ __device__ inline size_t fast_head_bytes(const DConfig& c) {
  const int km = kmax_of(c);
  return 64 + 64 * 4 + (size_t)c.d * 4 * 3 + (size_t)xf_floats(c) * 4 + pad16(km) + (size_t)km / 32 * 4 +
         FOUT * 4 + FPART * 4;
}

// The attention scratch of P2 (inside the union, after the first staging
// buffer), as byte offsets.
struct AttLayout {
  int raw, qs, kn, sc, stat, oacc, pv, kt, vt, total, kpitch, vpitch;
  __host__ __device__ AttLayout(int qpk, int KT, int f16) {
    const int P = qpk * 128;
    kpitch = f16 ? 272 : 528;
    vpitch = f16 ? 256 : 512;
    int o = 0;
    raw = o; o += (qpk + 2) * 128 * 4;
    qs = o; o += P * 4;
    kn = o; o += 128 * 4;
    sc = o; o += qpk * KT * 4;
    stat = o; o += 3 * 16 * 4;
    oacc = o; o += P * 4;
    pv = o; o += imax(FT, P) * 4;
    o = pad16(o);
    kt = o; o += KT * kpitch;
    vt = o; o += KT * vpitch;
    total = o;
  }
};

__host__ __device__ inline size_t table_stage_bytes(const DTable& T) {
  return (size_t)T.k + pad16(T.k / 32 * (T.scale_f16 ? 2 : 4));
}

__host__ __device__ inline size_t fast_union_bytes(const DConfig& c, const DTable& table, int grid, int KT, int f16,
                                                   int ts) {
  const int qpk = c.heads / c.kv_heads;
  size_t u = 2 * (size_t)FSTAGE;
  u = zmax(u, (size_t)FSTAGE + AttLayout(qpk, KT, f16).total);
  u = zmax(u, 2 * (size_t)FSTAGE + (size_t)c.kv_heads * c.d * 4);
  u = zmax(u, (size_t)FW * ts * table_stage_bytes(table));
  u = zmax(u, (size_t)grid * 8);
  return u;
}

struct FS {
  int* flag;     // [16]
  float* red;    // [64]
  float* x;      // [d] the residual stream
  float* nw;     // [d] staged norm weights
  float* fsc;    // [d] staged ffn scales
  float* xf;     // [xf_floats] a phase's f32 input
  int8_t* xq;    // [kmax] quantized activations
  float* xs;     // [kmax / 32] their scales
  float* out;    // [FOUT] the block's product rows
  float* part;   // [FPART]
  uint8_t* u;    // union: weight stages | attention | group partials | table stages
};

// cp.async.wait_group with a count known only at run time (0 .. 5).
__device__ __forceinline__ void cp_wait_n(int n) {
  switch (n) {
    case 0: cp_wait<0>(); break;
    case 1: cp_wait<1>(); break;
    case 2: cp_wait<2>(); break;
    case 3: cp_wait<3>(); break;
    case 4: cp_wait<4>(); break;
    default: cp_wait<5>(); break;
  }
}

// ------------------------------------------------------------ reductions --
__device__ __forceinline__ float block_sum(float v, FS& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) S.red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float s = lane < FW ? S.red[lane] : 0.0f;
    s = warp_sum(s);
    if (lane == 0) S.red[32] = s;
  }
  __syncthreads();
  return S.red[32];
}

// The block waits until words addr(0) .. addr(n - 1) carry `tag`. Thread t
// takes words t, t + FT, ... in passes of FPASS, all loads of a pass in
// flight at once, and hands each word to take(i, data) as it arrives (so
// take must not depend on the order: the callers only store). False (in
// every thread) when a wait ran out.
template <int NP = FPASS, class Addr, class Take>
__device__ __forceinline__ bool ll_take(int n, uint32_t tag, int* status, Addr addr, Take take) {
  bool ok = true;
  const int t = threadIdx.x;
  for (int base = 0; base < n && ok; base += NP * FT) {
    uint32_t pending = 0;
#pragma unroll
    for (int j = 0; j < NP; ++j)
      if (base + t + FT * j < n) pending |= 1u << j;
    long long spins = 0;
    while (pending) {
      unsigned long long w[NP];
#pragma unroll
      for (int j = 0; j < NP; ++j)
        if (pending & (1u << j)) w[j] = ll_get(addr(base + t + FT * j));
#pragma unroll
      for (int j = 0; j < NP; ++j)
        if ((pending & (1u << j)) && (uint32_t)(w[j] >> 32) == tag) {
          take(base + t + FT * j, (uint32_t)w[j]);
          pending &= ~(1u << j);
        }
      if (pending) {
        if (++spins > kSpinLimit) {
          atomicCAS(status, 0, 2);
          ok = false;
          break;
        }
        if ((spins & 255) == 0 && ld_volatile(status) != 0) {
          ok = false;
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// ------------------------------------------------------------ quantizer --
__device__ __forceinline__ void quant_fast(const float* src, int k, const float* w, const float* sc, float inv, int G,
                                           bool half, int8_t* q, float* s) {
  quantize_groups<FT>(src, k, w, sc, inv, G, half, q, s);
}

// -------------------------------------------------------------- products --
// A product's rows restricted to the columns [col0, col0 + kc), as a block
// stages them: the codes, then the weight scales, each padded to 16 bytes.
struct Slice {
  int kind, k, col0, kc, agroup;
  const uint8_t* codes;
  const uint8_t* scales;
  int cbytes, sbytes, cpad, rbytes;
  int vpc, lpg, chunks;  // values a 16-byte code chunk covers, chunks a group, chunks a row

  __device__ Slice(const DMat& W, int c0, int kcols) {
    kind = W.kind;
    k = W.k;
    col0 = c0;
    kc = kcols;
    agroup = W.agroup;
    codes = (const uint8_t*)W.codes;
    scales = (const uint8_t*)W.scales;
    cbytes = kind == kTernary ? kc / 4 : kc;
    sbytes = kind == kQ8_0 ? kc / 32 * 2 : kind == kInt8Row ? 4 : kc / 128 * 4;
    cpad = pad16(cbytes);
    rbytes = cpad + pad16(sbytes);
    vpc = kind == kTernary ? 64 : 16;
    lpg = agroup / vpc;
    chunks = cbytes / 16;
  }
  __device__ const uint8_t* code_src(int row) const {
    return kind == kTernary ? codes + (size_t)row * (k / 4) + col0 / 4 : codes + (size_t)row * k + col0;
  }
  __device__ const uint8_t* scale_src(int row) const {
    if (kind == kQ8_0) return scales + ((size_t)row * (k / 32) + col0 / 32) * 2;
    if (kind == kInt8Row) return scales + (size_t)row * 4;
    return scales + ((size_t)row * (k / 128) + col0 / 128) * 4;
  }
  // The i32 dot of chunk c of a staged row with the block's activations.
  __device__ int dot(const uint8_t* rowp, int c, const int8_t* xq) const {
    if (kind == kTernary) {
      const uint4 w = ((const uint4*)rowp)[c];
      const int4* a = (const int4*)(xq + col0 + 64 * c);
      return dot16_ternary(w.x, a[0]) + dot16_ternary(w.y, a[1]) + dot16_ternary(w.z, a[2]) +
             dot16_ternary(w.w, a[3]);
    }
    return dot16(((const int4*)rowp)[c], ((const int4*)(xq + col0))[c]);
  }
  // ws * xs of the group that chunk c starts.
  __device__ float scale(const uint8_t* rowp, int c, const float* xs) const {
    const int gl = c * vpc / agroup;
    const float ws = kind == kQ8_0 ? f16_bits_to_f32(((const uint16_t*)(rowp + cpad))[gl])
                     : kind == kInt8Row ? ((const float*)(rowp + cpad))[0]
                                        : ((const float*)(rowp + cpad))[gl];
    return ws * xs[(col0 + c * vpc) / agroup];
  }
};

// The block's rows of W (row_of(lr) is the weight row of local row lr)
// times the activations in S.xq / S.xs, over columns [col0, col0 + kc):
// out[lr] = sum over groups of f32(i32 group dot) * ws * xs, summed in tree
// order. The first weight batch is staged before `ready()` (the block's
// wait for its input). Rows of at least 32 chunks are cut into segments of
// 32 * J chunks (a warp each, J chunks a lane); shorter rows of a power of
// two chunks share a warp.
template <class RowOf, class Ready>
__device__ __forceinline__ bool gemv_fast(const DMat& Wg, int col0, int kc, int nrows, RowOf row_of, FS& S, Ready ready) {
  const Slice W(Wg, col0, kc);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int per = max(1, min(nrows, FSTAGE / W.rbytes));
  const int nbatch = nrows > 0 ? (nrows + per - 1) / per : 0;
  uint8_t* buf0 = S.u;
  uint8_t* buf1 = S.u + FSTAGE;
  auto issue = [&](int b) {
    if (b < nbatch) {
      uint8_t* dst = (b & 1) ? buf1 : buf0;
      const int lr0 = b * per, n = min(per, nrows - lr0);
      const int swords = W.sbytes / 4;
      for (int r = warp; r < n; r += FW) {
        const uint8_t* cs = W.code_src(row_of(lr0 + r));
        const uint8_t* ss = W.scale_src(row_of(lr0 + r));
        uint8_t* d = dst + r * W.rbytes;
        for (int c = lane; c < W.chunks; c += 32) cp_async16(d + c * 16, cs + c * 16);
        for (int w4 = lane; w4 < swords; w4 += 32) cp_async4(d + W.cpad + w4 * 4, ss + w4 * 4);
      }
    }
    cp_commit();
  };
  issue(0);
  if (!ready()) {
    cp_wait<0>();
    return false;
  }
  const int C = W.chunks;
  const bool packed = C < 32 && (C & (C - 1)) == 0;  // 32 / C rows a warp
  const int nseg32 = (C + 31) / 32;
  for (int b = 0; b < nbatch; ++b) {
    issue(b + 1);
    cp_wait<1>();
    __syncthreads();
    const uint8_t* src = (b & 1) ? buf1 : buf0;
    const int lr0 = b * per, n = min(per, nrows - lr0);
    if (packed) {
      const int R = 32 / C;
      const int units = (n + R - 1) / R;
      for (int u = warp; u < units; u += FW) {
        const int r = u * R + lane / C, c = lane % C;
        const bool live = r < n;
        const uint8_t* rowp = src + r * W.rbytes;
        int dot = live ? W.dot(rowp, c, S.xq) : 0;
        for (int o = 1; o < W.lpg; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        float f = (live && (c & (W.lpg - 1)) == 0) ? (float)dot * W.scale(rowp, c, S.xs) : 0.0f;
        for (int o = 1; o < C; o <<= 1) f += __shfl_xor_sync(0xffffffffu, f, o);
        if (live && c == 0) S.part[r] = f;
      }
    } else {
      // J: the most chunks a lane that still gives every warp a segment.
      int J = nseg32;
      while (J > 1 && (nseg32 % J || n * (nseg32 / J) < FW)) --J;
      const int nseg = nseg32 / J, units = n * nseg;
      for (int u = warp; u < units; u += FW) {
        const int r = u / nseg, seg = u - r * nseg;
        const uint8_t* rowp = src + r * W.rbytes;
        float f = 0.0f;
        for (int j = 0; j < J; ++j) {
          const int c = (seg * J + j) * 32 + lane;
          const bool live = c < C;
          int dot = live ? W.dot(rowp, c, S.xq) : 0;
          for (int o = 1; o < W.lpg; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
          if (live && (c & (W.lpg - 1)) == 0) f += (float)dot * W.scale(rowp, c, S.xs);
        }
        f = warp_sum(f);
        if (lane == 0) S.part[u] = f;
      }
    }
    __syncthreads();
    if (packed) {
      for (int r = t; r < n; r += FT) S.out[lr0 + r] = S.part[r];
    } else {
      int J = nseg32;
      while (J > 1 && (nseg32 % J || n * (nseg32 / J) < FW)) --J;
      const int nseg = nseg32 / J;
      for (int r = t; r < n; r += FT) {
        float acc = 0.0f;
        for (int sg = 0; sg < nseg; ++sg) acc += S.part[r * nseg + sg];
        S.out[lr0 + r] = acc;
      }
    }
    __syncthreads();  // the buffer is refilled by issue(b + 2)
  }
  cp_wait<0>();
  return true;
}

// ------------------------------------------------------------- attention --
// Starts the copy of keys and values [j0, j0 + n) of kv head g (except
// position `skip`) into the staged tiles.
__device__ void stage_kv(const DecodeArgs& a, int layer, int g, int j0, int n, int skip, uint8_t* kt, uint8_t* vt,
                         const AttLayout& L) {
  const DCache& c = a.cache;
  const int esize = c.f16 ? 2 : 4;
  const int cpr = 128 * esize / 16;  // 16-byte chunks a row
  for (int ci = threadIdx.x; ci < 2 * n * cpr; ci += FT) {
    const int which = ci >= n * cpr;
    const int cc = ci - which * n * cpr;
    const int jj = cc / cpr, q = cc - jj * cpr, jpos = j0 + jj;
    if (jpos == skip) continue;
    const int page = c.page_table[(size_t)a.stream * c.pages_per_stream + jpos / c.page_tokens];
    const size_t off = kv_offset(c, a.cfg, page, layer, which, g, jpos % c.page_tokens);
    const uint8_t* src = (const uint8_t*)c.pool + off * esize + q * 16;
    uint8_t* dst = (which ? vt + jj * L.vpitch : kt + jj * L.kpitch) + q * 16;
    cp_async16(dst, src);
  }
  cp_commit();
}

// The attention of the qpk query heads of kv head g at position pos over
// keys [0, pos], in tiles of KT keys with an online softmax
// (src/layers.rs:343-504: scores of q / sqrt(hd), max, Cephes exp, sum,
// weighted values; sums in tree order). raw holds q heads, k and v as P1
// made them; tile 0 is already being staged. On return the heads' output
// is in the oacc region.
__device__ void attend_fast(const DecodeArgs& a, const DLayer& Lw, int layer, int pos, int g, bool append, int KT,
                            uint8_t* base) {
  const DConfig& cfg = a.cfg;
  const int qpk = cfg.heads / cfg.kv_heads, P = qpk * 128, T = pos + 1;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const DCache& cache = a.cache;
  const AttLayout L(qpk, KT, cache.f16);
  float* raw = (float*)(base + L.raw);
  float* qs = (float*)(base + L.qs);
  float* kn = (float*)(base + L.kn);
  float* sc = (float*)(base + L.sc);
  float* mrun = (float*)(base + L.stat);
  float* lrun = mrun + 16;
  float* corr = lrun + 16;
  float* oacc = (float*)(base + L.oacc);
  float* pv = (float*)(base + L.pv);
  uint8_t* kt = base + L.kt;
  uint8_t* vt = base + L.vt;
  const float* sn = a.rope + (size_t)min(pos, a.rope_rows - 1) * 128;
  const float* cs = sn + 64;
  // Warp 0: k (norm, RoPE), warp 1: v, warps 2..: q heads (causal_lm.rs:428-446).
  for (int h = warp; h < 2 + qpk; h += FW) {
    const float* src = (h == 0) ? raw + P : (h == 1) ? raw + P + 128 : raw + (h - 2) * 128;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = src[lane * 4 + i];
    if (h != 1) {
      const float* nw = (h == 0) ? Lw.k_norm : Lw.q_norm;
      if (nw) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) ss += v[i] * v[i];
        const float inv = rms_inv(warp_sum(ss), 128, cfg.eps);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], __fmul_rn(inv, nw[lane * 4 + i]));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
        const int idx = (lane & 15) * 4 + i;
        const float c = cs[idx], s = sn[idx];
        v[i] = (lane < 16) ? __fsub_rn(__fmul_rn(v[i], c), __fmul_rn(partner, s))
                           : __fadd_rn(__fmul_rn(v[i], c), __fmul_rn(partner, s));
      }
    }
    if (h >= 2) {
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = cfg.has_q_scale ? __fmul_rn(v[i], cfg.q_scale) : v[i];
        qs[(h - 2) * 128 + lane * 4 + i] = __fmul_rn(x, scale);
      }
    } else {
      // The key (normed, rotated) and the value as the cache holds them.
      float* dst = (h == 0) ? kn : raw + P + 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[lane * 4 + i] = cache.f16 ? round_f16(v[i]) : v[i];
      if (append) {
        const int page = cache.page_table[(size_t)a.stream * cache.pages_per_stream + pos / cache.page_tokens];
        const size_t off = kv_offset(cache, cfg, page, layer, h, g, pos % cache.page_tokens) + lane * 4;
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
  if (t < qpk) {
    mrun[t] = -INFINITY;
    lrun[t] = 0.0f;
  }
  for (int p = t; p < P; p += FT) oacc[p] = 0.0f;
  const float* vn = raw + P + 128;
  const int KS = max(1, FT / P);  // key splits of the value sums
  for (int j0 = 0; j0 < T; j0 += KT) {
    const int n = min(KT, T - j0);
    if (j0 > 0) {
      __syncthreads();  // the tiles are refilled
      stage_kv(a, layer, g, j0, n, pos, kt, vt, L);
    }
    cp_wait<0>();
    __syncthreads();  // the q/k/v rows above, the staged tile
    if (pos >= j0 && pos < j0 + n) {
      // The new position's key and value come from this step, not the cache.
      const int jj = pos - j0;
      for (int e = t; e < 256; e += FT) {
        const float v = e < 128 ? kn[e] : vn[e - 128];
        uint8_t* row = e < 128 ? kt + jj * L.kpitch : vt + jj * L.vpitch;
        const int ee = e & 127;
        if (cache.f16) ((__half*)row)[ee] = __float2half_rn(v);
        else ((float*)row)[ee] = v;
      }
      __syncthreads();
    }
    // Scores: a thread per (head, key).
    for (int p = t; p < qpk * n; p += FT) {
      const int h = p / n, jj = p - h * n;
      const float4* q4 = (const float4*)(qs + h * 128);
      float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
      if (cache.f16) {
        const int4* kr = (const int4*)(kt + jj * L.kpitch);
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const int4 rw = kr[i];
          const __half2* h2 = (const __half2*)&rw;
          const float4 qa = q4[2 * i], qb = q4[2 * i + 1];
          const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
          const float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
          s0 = fmaf(qa.x, f0.x, s0);
          s1 = fmaf(qa.y, f0.y, s1);
          s2 = fmaf(qa.z, f1.x, s2);
          s3 = fmaf(qa.w, f1.y, s3);
          s0 = fmaf(qb.x, f2.x, s0);
          s1 = fmaf(qb.y, f2.y, s1);
          s2 = fmaf(qb.z, f3.x, s2);
          s3 = fmaf(qb.w, f3.y, s3);
        }
      } else {
        const float4* kr = (const float4*)(kt + jj * L.kpitch);
#pragma unroll 4
        for (int i = 0; i < 32; ++i) {
          const float4 kv = kr[i], qv = q4[i];
          s0 = fmaf(qv.x, kv.x, s0);
          s1 = fmaf(qv.y, kv.y, s1);
          s2 = fmaf(qv.z, kv.z, s2);
          s3 = fmaf(qv.w, kv.w, s3);
        }
      }
      sc[h * KT + jj] = (s0 + s1) + (s2 + s3);
    }
    __syncthreads();
    // Online softmax: warp h takes head h.
    for (int h = warp; h < qpk; h += FW) {
      float mx = -INFINITY;
      for (int jj = lane; jj < n; jj += 32) mx = fmaxf(mx, sc[h * KT + jj]);
      mx = warp_max(mx);
      const float mold = mrun[h], mnew = fmaxf(mold, mx);
      float sum = 0.0f;
      for (int jj = lane; jj < n; jj += 32) {
        const float e = cephes_exp(sc[h * KT + jj] - mnew);
        sc[h * KT + jj] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float c = mold == -INFINITY ? 0.0f : cephes_exp(mold - mnew);
        corr[h] = c;
        lrun[h] = lrun[h] * c + sum;
        mrun[h] = mnew;
      }
    }
    __syncthreads();
    // Weighted values: a thread per (head, dimension, key split).
    for (int p0 = 0; p0 < P; p0 += FT) {
      const int pe = p0 + t % min(P, FT), ks = (P <= FT) ? t / P : 0;
      float acc0 = 0.0f, acc1 = 0.0f;
      if (pe < P && ks < KS) {
        const int h = pe >> 7, e = pe & 127;
        const float* pr = sc + h * KT;
        int jj = ks;
        if (cache.f16) {
          const __half* vh = (const __half*)vt;
          for (; jj + KS < n; jj += 2 * KS) {
            acc0 = fmaf(pr[jj], __half2float(vh[jj * 128 + e]), acc0);
            acc1 = fmaf(pr[jj + KS], __half2float(vh[(jj + KS) * 128 + e]), acc1);
          }
          if (jj < n) acc0 = fmaf(pr[jj], __half2float(vh[jj * 128 + e]), acc0);
        } else {
          const float* vf = (const float*)vt;
          for (; jj + KS < n; jj += 2 * KS) {
            acc0 = fmaf(pr[jj], vf[jj * 128 + e], acc0);
            acc1 = fmaf(pr[jj + KS], vf[(jj + KS) * 128 + e], acc1);
          }
          if (jj < n) acc0 = fmaf(pr[jj], vf[jj * 128 + e], acc0);
        }
      }
      if (KS > 1) {
        if (ks < KS) pv[ks * P + pe] = acc0 + acc1;
        __syncthreads();
        if (t < P) {
          float s = 0.0f;
          for (int k = 0; k < KS; ++k) s += pv[k * P + t];
          oacc[t] = oacc[t] * corr[t >> 7] + s;
        }
      } else if (pe < P) {
        oacc[pe] = oacc[pe] * corr[pe >> 7] + (acc0 + acc1);
      }
    }
  }
  __syncthreads();
  for (int p = t; p < P; p += FT) oacc[p] = oacc[p] * (1.0f / lrun[p >> 7]);
  __syncthreads();
}

// ---------------------------------------------------------------- table --
// The block's rows [v0, v1) of the token table (forward_rows' last product,
// causal_lm.rs:386-388): f32 x times f32(code) * scale, no activation
// quantization; within a row, lane l takes values [16(l + 32m), +16), a
// 16-value sum is scaled once, and the lanes' sums meet in a tree. Each
// warp streams its rows through TSTAGES cp.async stages; the first stages
// go out before `ready()` (the wait for the final hidden state).
template <class Ready>
__device__ __forceinline__ bool table_fast(const DecodeArgs& a, int v0, int v1, int step, FS& S, float* best_v, int* best_i,
                           Ready ready) {
  const DTable& T = a.table;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int sb = T.scale_f16 ? 2 : 4;
  const int stage = (int)table_stage_bytes(T);
  const int ts = a.table_stages;  // 2 .. TSTAGES
  uint8_t* wst = S.u + (size_t)warp * ts * stage;
  const int nrows = v1 - v0;
  const int mine = nrows > warp ? (nrows - warp + FW - 1) / FW : 0;
  const int chunks = T.k / 16, sbytes = T.k / 32 * sb;
  const float mult = (a.cfg.logits_scaling == 1.0f) ? 1.0f : __fdiv_rn(1.0f, a.cfg.logits_scaling);
  auto issue = [&](int it) {
    if (it < mine) {
      const int row = v0 + warp + FW * it;
      uint8_t* dst = wst + (it % ts) * stage;
      const uint8_t* cs = (const uint8_t*)T.codes + (size_t)row * T.k;
      const uint8_t* ss = (const uint8_t*)T.scales + (size_t)row * sbytes;
      for (int c = lane; c < chunks; c += 32) cp_async16(dst + c * 16, cs + c * 16);
      for (int c = lane; c < sbytes / 8; c += 32) cp_async8(dst + T.k + c * 8, ss + c * 8);
    }
    cp_commit();
  };
  for (int i = 0; i < ts - 1; ++i) issue(i);
  if (!ready()) {
    cp_wait<0>();
    return false;
  }
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int it = 0; it < mine; ++it) {
    issue(it + ts - 1);
    cp_wait_n(ts - 1);  // row it's group has landed
    __syncwarp();
    const int row = v0 + warp + FW * it;
    const uint8_t* st = wst + (it % ts) * stage;
    float acc = 0.0f;
    for (int c = lane; c < chunks; c += 32) {
      const int4 w = ((const int4*)st)[c];
      const uint32_t wd[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u, (uint32_t)w.z ^ 0x80808080u,
                              (uint32_t)w.w ^ 0x80808080u};
      const float* xp = S.xf + c * 20;  // 16 values + 4 padding a chunk
      float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 xv = *(const float4*)(xp + 4 * q);
        d0 = fmaf(xv.x, byte_to_float(wd[q], 0), d0);
        d1 = fmaf(xv.y, byte_to_float(wd[q], 1), d1);
        d0 = fmaf(xv.z, byte_to_float(wd[q], 2), d0);
        d1 = fmaf(xv.w, byte_to_float(wd[q], 3), d1);
      }
      const int gi = c >> 1;
      const float s = T.scale_f16 ? f16_bits_to_f32(((const uint16_t*)(st + T.k))[gi]) : ((const float*)(st + T.k))[gi];
      acc = fmaf(d0 + d1, s, acc);
    }
    acc = warp_sum(acc);
    if (mult != 1.0f) acc = acc * mult;
    if (lane == 0) {
      if (a.logits) a.logits[(size_t)step * T.n + row] = acc;
      if (acc > bv) {  // rows rise within a warp: the first of equals stays
        bv = acc;
        bi = row;
      }
    }
    __syncwarp();  // the stage is refilled by the next issue
  }
  cp_wait<0>();
  // Block best: the largest value, the lowest index among equals.
  if (lane == 0) {
    S.red[warp] = bv;
    ((int*)S.red)[32 + warp] = bi;
  }
  __syncthreads();
  if (t == 0) {
    for (int w = 1; w < FW; ++w) {
      const float ov = S.red[w];
      const int oi = ((int*)S.red)[32 + w];
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    *best_v = bv;
    *best_i = bi;
  }
  __syncthreads();
  return true;
}

// ----------------------------------------------------------------- kernel --
__global__ void __launch_bounds__(FT, 1) k_decode_fast(DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const DConfig& cfg = a.cfg;
  const int c = blockIdx.x, G = gridDim.x, t = threadIdx.x;
  const int d = cfg.d, qpk = cfg.heads / cfg.kv_heads, P = qpk * 128;
  const int qd = cfg.heads * 128, kvd = cfg.kv_heads * 128, nqkv = qd + 2 * kvd;
  const int L = cfg.layers, KV = cfg.kv_heads, KT = a.key_tile;
  const FastLayout ll(cfg, G);
  FS S;
  uint8_t* p = smem;
  S.flag = (int*)p; p += 64;
  S.red = (float*)p; p += 64 * 4;
  S.x = (float*)p; p += (size_t)d * 4;
  S.nw = (float*)p; p += (size_t)d * 4;
  S.fsc = (float*)p; p += (size_t)d * 4;
  S.xf = (float*)p; p += (size_t)xf_floats(cfg) * 4;
  S.xq = (int8_t*)p; p += pad16(kmax_of(cfg));
  S.xs = (float*)p; p += (size_t)kmax_of(cfg) / 32 * 4;
  S.out = (float*)p; p += FOUT * 4;
  S.part = (float*)p; p += FPART * 4;
  S.u = p;
  // This block's rows of each phase.
  const int q0 = split_at(nqkv, c, G), q1 = split_at(nqkv, c + 1, G);
  const int u0 = split_at(cfg.ffn, c, G), u1 = split_at(cfg.ffn, c + 1, G), nu = u1 - u0;
  const int r0 = split_at(d, c, G), r1 = split_at(d, c + 1, G), nown = r1 - r0;
  const int tv0 = split_at(a.table.n, c, G), tv1 = split_at(a.table.n, c + 1, G);
  // Its kv-head group, its place in the group, its rows of o_proj.
  int g = 0;
  while (g + 1 < KV && split_at(G, g + 1, KV) <= c) ++g;
  const int gstart = split_at(G, g, KV), nbg = split_at(G, g + 1, KV) - gstart, jg = c - gstart;
  const int o0 = split_at(d, jg, nbg), o1 = split_at(d, jg + 1, nbg);
  const bool appender = jg == 0;
  uint8_t* att = S.u + FSTAGE;
  float* gpart = (float*)(S.u + 2 * FSTAGE);  // [KV][d] group partials of o
  const AttLayout AL(qpk, KT, a.cache.f16);
  int mark_at = 0;
  auto mark = [&]() {
    if (a.phase_ns && c == 0 && t == 0) a.phase_ns[mark_at] = gtimer();
    ++mark_at;
  };
  // Optional per-block stamps of one step (TRIT_PHASE_TRACE=3): [layer][kEventSlots][grid].
  int cur_step = -1, cur_layer = 0;
  auto ev = [&](int k) {
    if (a.events && cur_step == a.event_step && t == 0)
      a.events[((size_t)cur_layer * kEventSlots + k) * G + c] = gtimer();
  };
  auto stage_vec = [&](float* dst, const float* src, int n) {
    for (int i = 4 * t; i < n; i += 4 * FT) cp_async16(dst + i, src + i);
  };
  int token = a.tokens[0];
  for (int i = 0; i < a.steps; ++i) {
    bool stopped = false;
    for (int s = 0; s < a.nstop; ++s) stopped |= a.stop[s] == token;
    if (stopped) {
      if (c == 0 && t == 0) *a.count = i;
      return;
    }
    // The cache rows that other blocks appended in earlier steps are
    // visible from here on.
    __threadfence();
    const int pos = a.first_pos + i;
    cur_step = i;
    const uint32_t base = (uint32_t)i * (uint32_t)(4 * L + 2) + 1;
    mark_at = i * (4 * L + 2);
    mark();
    // x = the token's embedding (causal_lm.rs:347-355).
    const DTable& E = a.embed;
    for (int kk = t; kk < d; kk += FT) {
      float v = __fmul_rn((float)E.codes[(size_t)token * E.k + kk], table_scale(E, token, kk / 32));
      if (cfg.embedding_multiplier != 1.0f) v = __fmul_rn(v, cfg.embedding_multiplier);
      S.x[kk] = v;
    }
    for (int l = 0; l < L; ++l) {
      cur_layer = l;
      ev(0);
      const DLayer& Lw = a.layers[l];
      const uint32_t t_qkv = base + 4 * l, t_att = t_qkv + 1, t_h = t_qkv + 2, t_xb = t_qkv + 3;
      // P1: qkv. Input: x (the embedding, or xb of the layer before).
      stage_vec(S.nw, Lw.norm_attn, d);
      cp_commit();
      bool ok = gemv_fast(Lw.qkv, 0, d, q1 - q0, [&](int lr) { return q0 + lr; }, S, [&]() {
        if (l > 0 && !ll_take(d, t_qkv - 1, a.status, [&](int k) { return a.ll + ll.xb + k; },
                              [&](int k, uint32_t v) { S.x[k] = __uint_as_float(v); }))
          return false;
        ev(1);
        // The thread's own words (the embedding's, or those it took).
        float ss = 0.0f;
        for (int kk = t; kk < d; kk += FT) ss += S.x[kk] * S.x[kk];
        cp_wait<1>();
        const float inv = rms_inv(block_sum(ss, S), d, cfg.eps);
        quant_fast(S.x, d, S.nw, nullptr, inv, Lw.qkv.agroup, Lw.qkv.half, S.xq, S.xs);
        __syncthreads();
        ev(2);
        return true;
      });
      if (!ok) return;
      ev(3);
      for (int lr = t; lr < q1 - q0; lr += FT) ll_put(a.ll + ll.qkv + q0 + lr, __float_as_uint(S.out[lr]), t_qkv);
      ev(4);
      mark();
      // P2: attention of kv head g, then o_proj over the group's columns.
      const int n0 = min(KT, pos + 1);
      stage_kv(a, l, g, 0, n0, pos, att + AL.kt, att + AL.vt, AL);
      const int col0 = g * P;
      ok = gemv_fast(Lw.out, col0, P, o1 - o0, [&](int lr) { return o0 + lr; }, S, [&]() {
        float* raw = (float*)(att + AL.raw);
        if (!ll_take(P + 256, t_qkv, a.status,
                     [&](int k) {
                       return a.ll + ll.qkv +
                              (k < P ? g * P + k : k < P + 128 ? qd + g * 128 + (k - P) : qd + kvd + g * 128 + (k - P - 128));
                     },
                     [&](int k, uint32_t v) { raw[k] = __uint_as_float(v); }))
          return false;
        ev(5);
        cp_wait<1>();
        __syncthreads();
        attend_fast(a, Lw, l, pos, g, appender, KT, att);
        ev(6);
        const float* o = (const float*)(att + AL.oacc);
        quant_fast(o, P, nullptr, nullptr, 1.0f, Lw.out.agroup, Lw.out.half, S.xq + col0, S.xs + col0 / Lw.out.agroup);
        __syncthreads();
        ev(7);
        return true;
      });
      if (!ok) return;
      ev(8);
      for (int lr = t; lr < o1 - o0; lr += FT)
        ll_put(a.ll + ll.opart + g * d + o0 + lr, __float_as_uint(S.out[lr]), t_att);
      ev(9);
      mark();
      // P4: x += o (the group partials in group order), gate_up, silu * up.
      stage_vec(S.nw, Lw.norm_mlp, d);
      if (Lw.ffn_scale) stage_vec(S.fsc, Lw.ffn_scale, d);
      cp_commit();
      ok = gemv_fast(Lw.gate_up, 0, d, 2 * nu, [&](int lr) { return lr < nu ? u0 + lr : cfg.ffn + u0 + lr - nu; }, S,
                     [&]() {
        if (appender) __threadfence();  // the cache rows this block appended, before its next words
        if (!ll_take<16>(KV * d, t_att, a.status, [&](int k) { return a.ll + ll.opart + k; },
                     [&](int k, uint32_t v) { gpart[k] = __uint_as_float(v); }))
          return false;
        ev(10);
        float ss = 0.0f;
        for (int r = t; r < d; r += FT) {
          float o = 0.0f;
          for (int gg = 0; gg < KV; ++gg) o += gpart[gg * d + r];
          const float xv = (cfg.residual_multiplier == 1.0f) ? __fadd_rn(S.x[r], o)
                                                             : __fadd_rn(S.x[r], __fmul_rn(cfg.residual_multiplier, o));
          S.x[r] = xv;
          ss += xv * xv;
        }
        cp_wait<1>();
        const float inv = rms_inv(block_sum(ss, S), d, cfg.eps);
        quant_fast(S.x, d, S.nw, Lw.ffn_scale ? S.fsc : nullptr, inv, Lw.gate_up.agroup, Lw.gate_up.half, S.xq,
                   S.xs);
        __syncthreads();
        ev(11);
        return true;
      });
      if (!ok) return;
      ev(12);
      for (int lr = t; lr < nu; lr += FT)
        ll_put(a.ll + ll.h + u0 + lr, __float_as_uint(__fmul_rn(silu(S.out[lr]), S.out[nu + lr])), t_h);
      ev(13);
      mark();
      // P5: down + residual. Input: h.
      ok = gemv_fast(Lw.down, 0, cfg.ffn, nown, [&](int lr) { return r0 + lr; }, S, [&]() {
        if (!ll_take(cfg.ffn, t_h, a.status, [&](int k) { return a.ll + ll.h + k; },
                     [&](int k, uint32_t v) { S.xf[k] = __uint_as_float(v); }))
          return false;
        ev(14);
        quant_fast(S.xf, cfg.ffn, nullptr, nullptr, 1.0f, Lw.down.agroup, Lw.down.half, S.xq, S.xs);
        __syncthreads();
        ev(15);
        return true;
      });
      if (!ok) return;
      ev(16);
      for (int lr = t; lr < nown; lr += FT) {
        const float o = S.out[lr];
        const float xv = (cfg.residual_multiplier == 1.0f) ? __fadd_rn(S.x[r0 + lr], o)
                                                           : __fadd_rn(S.x[r0 + lr], __fmul_rn(cfg.residual_multiplier, o));
        ll_put(a.ll + ll.xb + r0 + lr, __float_as_uint(xv), t_xb);
      }
      ev(17);
      mark();
    }
    // The final RmsNorm (f32, no quantization), the table slice, the argmax.
    const uint32_t t_final = base + 4 * L - 1, t_best = base + 4 * L;
    stage_vec(S.nw, a.final_norm, d);
    cp_commit();
    bool ok = table_fast(a, tv0, tv1, i + 1, S, (float*)(S.flag + 4), S.flag + 5, [&]() {
      if (!ll_take(d, t_final, a.status, [&](int k) { return a.ll + ll.xb + k; },
                   [&](int k, uint32_t v) { S.x[k] = __uint_as_float(v); }))
        return false;
      ev(18);
      float ss = 0.0f;
      for (int kk = t; kk < d; kk += FT) ss += S.x[kk] * S.x[kk];
      cp_wait_n(a.table_stages - 1);  // the final norm's weights (the table stages may still travel)
      const float inv = rms_inv(block_sum(ss, S), d, cfg.eps);
      for (int kk = t; kk < d; kk += FT) S.xf[kk + (kk >> 4) * 4] = __fmul_rn(S.x[kk], __fmul_rn(inv, S.nw[kk]));
      __syncthreads();
      ev(19);
      return true;
    });
    if (!ok) return;
    ev(20);
    if (t == 0) {
      ll_put(a.ll + ll.best + 2 * c, (uint32_t)S.flag[4], t_best);
      ll_put(a.ll + ll.best + 2 * c + 1, (uint32_t)S.flag[5], t_best);
    }
    float* bvals = (float*)S.u;
    int* bidx = (int*)S.u + G;
    ok = ll_take(2 * G, t_best, a.status, [&](int k) { return a.ll + ll.best + k; }, [&](int k, uint32_t v) {
      if (k & 1) bidx[k >> 1] = (int)v;
      else bvals[k >> 1] = __uint_as_float(v);
    });
    if (!ok) return;
    ev(21);
    mark();
    if (t < 32) {
      float b = -INFINITY;
      int ix = 0x7fffffff;
      for (int k = t; k < G; k += 32)
        if (bvals[k] > b || (bvals[k] == b && bidx[k] < ix)) {
          b = bvals[k];
          ix = bidx[k];
        }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, b, o);
        const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
        if (ob > b || (ob == b && oi < ix)) {
          b = ob;
          ix = oi;
        }
      }
      if (t == 0) S.flag[2] = (ix == 0x7fffffff) ? 0 : ix;
    }
    __syncthreads();
    token = S.flag[2];
    if (c == 0 && t == 0) a.tokens[i + 1] = token;
    __syncthreads();
  }
  if (c == 0 && t == 0) *a.count = a.steps;
}

// The key tile (the most keys of 256, 128, 64, 32) and then the table
// stages (the most of TSTAGES .. 2) whose shared memory fits; {0, 0} if none.
struct Tiles {
  int kt = 0, ts = 0;
};
Tiles pick_tiles(const DConfig& cfg, const DTable& table, int grid, int f16, size_t limit) {
  for (int kt = 256; kt >= 32; kt /= 2)
    for (int ts = TSTAGES; ts >= 2; --ts)
      if (fast_head_bytes(cfg) + fast_union_bytes(cfg, table, grid, kt, f16, ts) <= limit) return {kt, ts};
  return {};
}

}  // namespace

bool decode_fast_supported(const DConfig& cfg, const DTable& table, int grid, int f16) {
  const int qpk = cfg.heads / cfg.kv_heads;
  auto ok = [](int k) { return k % 128 == 0 && k <= 16384; };
  if (cfg.hd != 128 || !ok(cfg.d) || !ok(cfg.ffn) || !ok(cfg.heads * 128) || qpk * 128 > 2 * FT || qpk > 16) return false;
  if (cfg.kv_heads > grid || table.k != cfg.d) return false;
  // Rows a block takes in each phase.
  const int nqkv = (cfg.heads + 2 * cfg.kv_heads) * 128;
  const int min_group = grid / cfg.kv_heads;
  if ((nqkv + grid - 1) / grid > FOUT || 2 * ((cfg.ffn + grid - 1) / grid) > FOUT ||
      (cfg.d + grid - 1) / grid > FOUT || (cfg.d + min_group - 1) / min_group > FOUT)
    return false;
  // A staged row of any product fits a staging buffer (codes + scales).
  const int kmax = kmax_of(cfg);
  if (kmax + kmax / 16 + 32 > FSTAGE) return false;
  return pick_tiles(cfg, table, grid, f16, 227 * 1024).kt > 0;
}

size_t decode_fast_ll_words(const DConfig& cfg, int grid) { return (size_t)FastLayout(cfg, grid).total; }

cudaError_t launch_decode_fast(const DecodeArgs& a, int grid, cudaStream_t s) {
  if (!decode_fast_supported(a.cfg, a.table, grid, a.cache.f16)) return cudaErrorNotSupported;
  DecodeArgs args = a;
  const Tiles tl = pick_tiles(a.cfg, a.table, grid, a.cache.f16, 227 * 1024);
  args.key_tile = tl.kt;
  args.table_stages = tl.ts;
  const size_t smem =
      fast_head_bytes(a.cfg) + fast_union_bytes(a.cfg, a.table, grid, args.key_tile, a.cache.f16, args.table_stages);
  cudaError_t e = cudaFuncSetAttribute(k_decode_fast, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_fast, FT, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
  void* params[] = {&args};
  return cudaLaunchCooperativeKernel((const void*)k_decode_fast, dim3(grid), dim3(FT), params, smem, s);
}

}  // namespace trit
