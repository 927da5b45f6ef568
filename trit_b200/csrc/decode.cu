// The persistent batch-1 decode: every greedy step of one generation in
// one cooperative kernel (one block per SM). A step runs the layers of
// CausalLm::hidden (src/models/parts/causal_lm.rs:410-481) as five phases:
//   P1 qkv      every block: RmsNorm + quantize of x (redundant, 4 KB), then
//               its slice of the stacked q/k/v rows
//   P2 attend   block kvh (one per kv head): q/k norm, RoPE, K/V append,
//               the exact GQA attention of the kv head's query heads over
//               every key, and the quantized head outputs
//   P3 o        every block: its rows of o_proj, added to its residual rows
//   P4 gate_up  every block: RmsNorm + quantize of x, its units of gate/up,
//               h = silu(gate) * up
//   P5 down     every block: quantize h, its rows of down_proj, added to its
//               residual rows
// then the final RmsNorm, the block's slice of the token table (f32 math),
// and the argmax, which every block reduces from all blocks' bests.
//
// No grid barrier: a value that one block makes and another needs travels
// as a 64-bit word {data, tag} (the low-latency protocol of NCCL's LL
// transfers): the tag names the step and phase, and a consumer polls the
// words themselves, so the data and the "ready" signal arrive in one round
// trip. Each buffer is written once per layer; the all-to-all chain of
// phases guarantees that every reader of a word has read it before its
// writer can reach the next write of that word. A block issues its weight
// loads before it waits for its input. Each block keeps the residual rows
// it owns in shared memory.
//
// Waits are bounded: a poll that sees no data within ~2^22 rounds sets
// *status and every block returns; the host reports the error.
#include <cuda_runtime.h>

#include "attention.cuh"
#include "device.cuh"
#include "kernels.h"
#include "ll.cuh"

namespace trit {
namespace {

constexpr int DT = 512;          // threads per block
constexpr int DW = DT / 32;      // warps per block
constexpr int TAB_SLAB = 128;    // bytes of a table row per pipeline stage
constexpr int TAB_STAGES = 6;
constexpr int TAB_PITCH = TAB_SLAB + 16;
constexpr int TAB_ROWS_W = 8;    // table rows per warp group (4 threads a row)
constexpr long long SPIN_LIMIT = kSpinLimit;
constexpr int LLW = 4;           // LL words a thread polls at once

// The block waits until words [0, n) of `src` carry `tag` and hands each
// word's data to sink(i, data). Thread t polls words t, t + DT, ...: every
// load of a round goes out before any is checked. False when a wait ran
// out (the whole block then returns).
template <class Sink>
__device__ bool ll_wait(const unsigned long long* src, int n, uint32_t tag, int* status, Sink sink) {
  bool ok = true;
  // Passes of LLW words a thread (one pass for n <= LLW * DT).
  for (int base = 0; base < n && ok; base += LLW * DT) {
    uint32_t pending = 0;
#pragma unroll
    for (int j = 0; j < LLW; ++j)
      if (base + threadIdx.x + DT * j < n) pending |= 1u << j;
    long long spins = 0;
    while (pending) {
      unsigned long long v[LLW];
#pragma unroll
      for (int j = 0; j < LLW; ++j)
        if (pending & (1u << j)) v[j] = ll_get(src + base + threadIdx.x + DT * j);
#pragma unroll
      for (int j = 0; j < LLW; ++j)
        if ((pending & (1u << j)) && (uint32_t)(v[j] >> 32) == tag) {
          sink(base + threadIdx.x + DT * j, (uint32_t)v[j]);
          pending &= ~(1u << j);
        }
      if (pending) {
        if (++spins > SPIN_LIMIT) {
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

struct Shared {
  float* xf;       // [kmax]: the phase's f32 input (x or h), normed x for the table
  float* sq;       // [kmax]: squares for RmsNorm
  int8_t* xq;      // [kmax]
  float* xs;       // [kmax / 32]
  float* own;      // [512]: the residual rows this block owns
  float* out;      // [512]
  float* nw;       // [d]: the phase's RmsNorm weights, staged while the block waits
  float* red;      // [64]
  int* part;       // union: GEMV group dots ...
  float* att;      // ... attention scratch ...
  uint8_t* tab;    // ... table stages
  int* flag;       // [16]
  int gmax;        // the most activation groups of any product
};

// RmsNorm (layers.rs:135-144) of S.xf (d values) with weight w (null: no
// norm), then Quantized::grouped of the result into S.xq / S.xs.
// RmsNorm (weights w, or none) of S.xf, times sc (or none), then the
// activation quantizer in groups of G into S.xq / S.xs. A warp takes one
// group at a time. (Quantizing a warp's groups interleaved, with the norm
// weights loaded ahead, measured 8 % slower per token.)
__device__ void norm_quant(int d, const float* w, float eps, int G, bool half, Shared& S,
                           const float* sc = nullptr) {
  __syncthreads();
  float inv = 1.0f;
  if (w) {
    // The sum of squares in the reference's order: the squares in parallel
    // (each rounded, as the reference rounds them), then one thread adds
    // them left to right.
    for (int i = threadIdx.x; i < d; i += DT) S.sq[i] = __fmul_rn(S.xf[i], S.xf[i]);
    __syncthreads();
    if (threadIdx.x == 0) S.red[0] = rms_inv(seq_sum(S.sq, d), d, eps);
    __syncthreads();
    inv = S.red[0];
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = d / G;
  for (int g = warp; g < groups; g += DW) {
    if (G == 32) {
      float v[1];
      int kk = g * 32 + lane;
      v[0] = w ? __fmul_rn(S.xf[kk], __fmul_rn(inv, w[kk])) : S.xf[kk];
      if (sc) v[0] = __fmul_rn(v[0], sc[kk]);
      float s2 = warp_quantize_group<32>(v, S.xq + g * 32, half);
      if (lane == 0) S.xs[g] = s2;
    } else {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int kk = g * 128 + lane * 4 + i;
        v[i] = w ? __fmul_rn(S.xf[kk], __fmul_rn(inv, w[kk])) : S.xf[kk];
        if (sc) v[i] = __fmul_rn(v[i], sc[kk]);
      }
      float s2 = warp_quantize_group<128>(v, S.xq + g * 128, half);
      if (lane == 0) S.xs[g] = s2;
    }
  }
  __syncthreads();
}

// The layer's RmsNorm weights (d floats) into S.nw by cp.async, one commit
// group, issued before the product's first weight batch so that both travel
// while the block waits for its input; the norm waits for this group
// (cp_wait<1>: all but the batch after it). w and d * 4 are 16-byte
// multiples (arena vectors).
__device__ __forceinline__ void stage_norm(const float* w, int d, Shared& S) {
  for (int i = 4 * threadIdx.x; i < d; i += 4 * DT) cp_async16(S.nw + i, w + i);
  cp_commit();
}

// ------------------------------------------------------------- products --
constexpr int WSTAGE = 48 * 1024;  // bytes of one weight staging buffer (two of them): a block's C1 gate/up rows fit one

__host__ __device__ inline int code_row_bytes(const DMat& W) { return W.kind == kTernary ? W.k / 4 : W.k; }
__host__ __device__ inline int scale_row_bytes(const DMat& W) {
  return W.kind == kQ8_0 ? W.k / 32 * 2 : W.kind == kInt8Row ? 4 : W.k / 128 * 4;
}
__host__ __device__ inline int staged_row_bytes(const DMat& W) {
  return (code_row_bytes(W) + 15) / 16 * 16 + (scale_row_bytes(W) + 15) / 16 * 16;
}

// Rows of a W8A8 layer for this block (row_of(lr) is the weight row of
// local row lr). The rows' codes and scales stream into shared memory by
// cp.async in batches of up to WSTAGE bytes, double-buffered; the first
// batch is issued before `ready()` (the block's wait for its input and its
// quantization), so the weights travel while the block waits. A thread
// forms whole i32 group dots (a (row, group) pair at a time), then one
// thread a row runs the row's group chain of int8.rs:560-570 in order into
// S.out[lr].
// ev(evbase + 0..2): the first batch's weights in shared memory, its group
// dots, its chains (event trace only).
template <class RowOf, class Ready, class Ev>
__device__ bool gemv(const DMat& Wg, int nrows, RowOf row_of, Shared& S, Ready ready, Ev ev, int evbase) {
  const DMat W = Wg;  // in registers: the loops below store to shared memory, which would force reloads
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int k = W.k, groups = k / W.agroup, lpg = W.agroup / 16;  // 16-byte chunks a group: 2 or 8
  const int crow = code_row_bytes(W), srow = scale_row_bytes(W);
  const int cpad = (crow + 15) / 16 * 16, rbytes = staged_row_bytes(W);
  const int per = min(nrows, WSTAGE / rbytes);  // rows a batch (the host checks rbytes <= WSTAGE)
  const int nbatch = per > 0 ? (nrows + per - 1) / per : 0;
  uint8_t* buf0 = (uint8_t*)S.part;
  uint8_t* buf1 = buf0 + WSTAGE;
  // The batch's group dots (exact i32 values as f32, |dot| < 2^24) and
  // scale products, [group][row]: the chain threads (one a row) read
  // consecutive words.
  float* pdot = (float*)(buf1 + WSTAGE);
  float* pscl = pdot + WSTAGE / 32;  // per * groups <= WSTAGE / 32: a row takes >= 32 bytes a group
  // A warp per row: lanes take the row's 16-byte code chunks and 4-byte
  // scale words (no integer division in these loops).
  auto issue = [&](int b) {
    if (b < nbatch) {
      uint8_t* dst = (b & 1) ? buf1 : buf0;
      const int lr0 = b * per, n = min(per, nrows - lr0);
      const int cchunks = crow / 16, swords = srow / 4;
      for (int r = warp; r < n; r += DW) {
        const uint8_t* codes = (const uint8_t*)W.codes + (size_t)row_of(lr0 + r) * crow;
        const uint8_t* scales = (const uint8_t*)W.scales + (size_t)row_of(lr0 + r) * srow;
        uint8_t* d = dst + r * rbytes;
        for (int cc = lane; cc < cchunks; cc += 32) cp_async16(d + cc * 16, codes + cc * 16);
        for (int w4 = lane; w4 < swords; w4 += 32) cp_async4(d + cpad + w4 * 4, scales + w4 * 4);
      }
    }
    cp_commit();
  };
  issue(0);
  if (!ready()) {
    cp_wait<0>();
    return false;
  }
  for (int b = 0; b < nbatch; ++b) {
    issue(b + 1);
    cp_wait<1>();
    __syncthreads();
    if (b == 0) ev(evbase);
    const uint8_t* src = (b & 1) ? buf1 : buf0;
    const int lr0 = b * per, n = min(per, nrows - lr0);
    // The batch's group dots: thread t takes the (row, group) pairs t,
    // t + DT, ... of the batch, each a whole group (lpg 16-byte chunks), so
    // no lanes wait on each other and a thread's loads go out together.
    // Integer dots: the order of their terms changes nothing.
    {
      const int dr = DT / groups, dg = DT - dr * groups;
      int r = t / groups, g = t - r * groups;
      const int total = n * groups;
#pragma unroll 2
      for (int idx = t; idx < total; idx += DT) {
        const uint8_t* rowp = src + r * rbytes;
        int dot = 0;
        if (lpg == 2) {
          const int c = 2 * g;
          const int4 a0 = ((const int4*)S.xq)[c], a1 = ((const int4*)S.xq)[c + 1];
          if (W.kind == kTernary) {
            dot = dot16_ternary(((const uint32_t*)rowp)[c], a0) + dot16_ternary(((const uint32_t*)rowp)[c + 1], a1);
          } else {
            dot = dot16(((const int4*)rowp)[c], a0) + dot16(((const int4*)rowp)[c + 1], a1);
          }
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int c = 8 * g + u;
            const int4 a = ((const int4*)S.xq)[c];
            dot += W.kind == kTernary ? dot16_ternary(((const uint32_t*)rowp)[c], a) : dot16(((const int4*)rowp)[c], a);
          }
        }
        const float ws = W.kind == kQ8_0 ? f16_bits_to_f32(((const uint16_t*)(rowp + cpad))[g])
                         : W.kind == kInt8Row ? ((const float*)(rowp + cpad))[0]
                                              : ((const float*)(rowp + cpad))[g];
        pdot[g * per + r] = __int2float_rn(dot);
        pscl[g * per + r] = __fmul_rn(ws, S.xs[g]);
        g += dg;
        r += dr;
        if (g >= groups) {
          g -= groups;
          ++r;
        }
      }
    }
    __syncthreads();
    if (b == 0) ev(evbase + 1);
    // The group chains of the batch's rows, one thread a row, groups in order.
    for (int r = t; r < n; r += DT) {
      float acc = 0.0f;
#pragma unroll 8
      for (int g = 0; g < groups; ++g) acc = __fmaf_rn(pdot[g * per + r], pscl[g * per + r], acc);
      S.out[lr0 + r] = acc;
    }
    __syncthreads();  // the buffers are refilled by issue(b + 2) and the next batch's dots
    if (b == 0) ev(evbase + 2);
  }
  cp_wait<0>();
  return true;
}

// ------------------------------------------------------------ attention --
// LL word offsets of the decode buffers.
struct LlLayout {
  int qkv, attq, attq_scales, xa, h, xb, best, total;
  __host__ __device__ LlLayout(const DConfig& cfg, int grid) {
    const int qd = cfg.heads * 128, nqkv = qd + 2 * cfg.kv_heads * 128;
    qkv = 0;
    attq = nqkv;
    attq_scales = attq + qd / 4;
    xa = attq_scales + qd / 32;
    h = xa + cfg.d;
    xb = h + cfg.ffn;
    best = xb + cfg.d;
    total = best + 2 * grid;
  }
};

// The LL word of row `row` of the stacked q | k | v product: the words of
// each kv head's query heads, key and value lie together, [kv head][q heads
// of the group | k | v][128], so its attention block waits on one run.
__device__ __forceinline__ int qkv_slot(const DConfig& cfg, int row) {
  const int qpk = cfg.heads / cfg.kv_heads, qd = cfg.heads * 128, kvd = cfg.kv_heads * 128;
  const int run = (qpk + 2) * 128;
  if (row < qd) return (row / 128 / qpk) * run + row % (qpk * 128);
  if (row < qd + kvd) return ((row - qd) / 128) * run + qpk * 128 + row % 128;
  return ((row - qd - kvd) / 128) * run + (qpk + 1) * 128 + row % 128;
}

// Keys a staged attention tile: 256 (f16) or 128 (f32) when the shared
// memory has room (launch_decode picks it), so a short context is one tile.
__host__ __device__ inline int attend_kt(int f16, bool wide) { return (f16 ? 128 : 64) * (wide ? 2 : 1); }

// Shared memory of the attention phase, in floats.
__host__ __device__ inline size_t attend_smem_floats(int qpk, int tmax, int f16, int kt) {
  return (size_t)(qpk + 2) * 128 + (size_t)qpk * 128 + 2 * 128 + (size_t)qpk * 128 + (size_t)qpk * 4 +
         (size_t)qpk * 32 + 3 * 128 + attention_smem_floats(qpk, tmax, kt, f16);
}

// Block kvh of the P2 phase: the query heads of kv head kvh over keys
// 0..pos, exact (attention.cuh). Tile 0 of the cached keys and values goes
// out (cp.async) before the block waits for q, k and v; the block appends
// the new key and value to the cache and publishes the heads' quantized
// output as LL words.
template <class Ev>
__device__ bool attend(const DecodeArgs& a, const DLayer& L, int layer, int pos, int kvh, int tmax, uint32_t tag_in,
                       uint32_t tag_out, Shared& S, Ev ev) {
  const DConfig& cfg = a.cfg;
  const int hd = 128, qpk = cfg.heads / cfg.kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
  const int T = pos + 1;
  const DCache& cache = a.cache;
  const LlLayout ll(cfg, gridDim.x);
  const int nq = qpk * hd;
  float* raw = S.att;               // [(qpk + 2)][128]: q heads, k, v as P1 made them
  float* q = raw + nq + 2 * hd;     // [qpk][128]
  float* kf = q + nq;               // [128]
  float* vf = kf + hd;              // [128]
  float* out = vf + hd;             // [qpk][128]
  float* scales = out + nq;         // [qpk * 4]: one a group of 32 at most
  int8_t* codes = (int8_t*)(scales + qpk * 4);  // [qpk * 128] bytes
  float* nrm = scales + qpk * 4 + qpk * 32;  // [3][128]: q norm, k norm weights, the RoPE row (sin | cos)
  float* region = nrm + 3 * 128;
  const int kt = a.key_tile, row = cache.f16 ? 64 : 128;
  float* sc = region;
  float* ktl = sc + qpk * tmax;
  float* vtl = ktl + kt * (row + 4);
  float* stat = vtl + kt * row;
  Attention<DT> A{cache, cfg, a.stream, layer, kvh, qpk, kt, sc, ktl, vtl, stat, tmax};
  // The norm weights and the position's RoPE row go out with tile 0 of the
  // cached keys and values, before the wait for q, k and v.
  for (int i = 4 * t; i < 3 * hd; i += 4 * DT) {
    const float* src = i < hd ? L.q_norm : i < 2 * hd ? L.k_norm : a.rope + (size_t)min(pos, a.rope_rows - 1) * hd;
    if (src) cp_async16(nrm + i, src + i % hd);
  }
  A.preload(T, true);
  // q heads, k and v of this kv head, as P1 made them.
  // q heads, k and v of this kv head: one run of LL words (qkv_slot).
  bool ok = ll_wait(a.ll + ll.qkv + kvh * (nq + 2 * hd), nq + 2 * hd, tag_in, a.status,
                    [&](int i, uint32_t v) { raw[i] = __uint_as_float(v); });
  if (!ok) return false;
  ev(5);
  cp_wait_all();  // the staged norm weights and RoPE row (tile 0 as well)
  __syncthreads();
  const float* sn = nrm + 2 * hd;
  const float* cs = sn + hd / 2;
  // Warp 0: k, warp 1: v, warps 2..: q heads (causal_lm.rs:428-446).
  for (int h = warp; h < 2 + qpk; h += DW) {
    const float* src = (h == 0) ? raw + nq : (h == 1) ? raw + nq + hd : raw + (h - 2) * hd;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = src[lane * 4 + i];
    if (h != 1) {
      const float* nw = (h == 0) ? (L.k_norm ? nrm + hd : nullptr) : (L.q_norm ? nrm : nullptr);
      if (nw) {
        float inv = 0.0f;
        if (lane == 0) inv = rms_inv(seq_sum_squares(src, hd), hd, cfg.eps);
        inv = __shfl_sync(0xffffffffu, inv, 0);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], __fmul_rn(inv, nw[lane * 4 + i]));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
        int idx = (lane & 15) * 4 + i;
        float c = cs[idx], sg = sn[idx];
        v[i] = (lane < 16) ? __fsub_rn(__fmul_rn(v[i], c), __fmul_rn(partner, sg))
                           : __fadd_rn(__fmul_rn(v[i], c), __fmul_rn(partner, sg));
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
      for (int i = 0; i < 4; ++i) dst[lane * 4 + i] = v[i];
      int page = cache.page_table[(size_t)a.stream * cache.pages_per_stream + pos / cache.page_tokens];
      size_t off = kv_offset(cache, cfg, page, layer, h, kvh, pos % cache.page_tokens) + lane * 4;
      if (cache.f16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) ((__half*)cache.pool)[off + i] = __float2half_rn(v[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) ((float*)cache.pool)[off + i] = v[i];
      }
      // Only this block (the one of kv head kvh) reads the row in later
      // steps, after the __syncthreads below and its own later barriers;
      // other kernels read it after this kernel ends.
    }
  }
  __syncthreads();
  ev(28);
  A.run(q, T, kf, vf, true, out);
  ev(6);
  // Quantize each head's output (groups of 32 or 128 lie inside a head),
  // then publish codes (4 a word) and scales as LL words.
  const DMat& O = L.out;
  const int G = O.agroup;
  quantize_groups<DT, 4>(out, nq, nullptr, nullptr, 1.0f, G, O.half, codes, scales);
  __syncthreads();
  const int qh0 = kvh * qpk;
  for (int wd = t; wd < nq / 4; wd += DT) ll_put(a.ll + ll.attq + qh0 * hd / 4 + wd, ((const uint32_t*)codes)[wd], tag_out);
  for (int g = t; g < nq / G; g += DT) ll_put(a.ll + ll.attq_scales + qh0 * hd / G + g, __float_as_uint(scales[g]), tag_out);
  __syncthreads();  // the next phase stages weights over this scratch
  ev(7);
  return true;
}

// ---------------------------------------------------------------- table --
// The block's slice of the token table (forward_rows' last product,
// causal_lm.rs:386-388), f32 math in the lane order of the AVX-512 tile.
// Each warp streams its own groups of 8 rows through a private cp.async
// pipeline: a stage holds 128 code bytes of each row and, in the row's
// padding, the scales of those 4 groups of 32. The first stages are issued
// before `ready()` (the wait for the final hidden state and its norm).
template <class Ready>
__device__ bool table_slice(const DecodeArgs& a, int v0, int v1, int step, Shared& S, float* best_v, int* best_i,
                            Ready ready) {
  const DTable& T = a.table;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, q = lane & 3, rl = lane >> 2;
  const int slabs = T.k / TAB_SLAB;
  const int ngroups = (v1 - v0 + TAB_ROWS_W - 1) / TAB_ROWS_W;
  const int my_groups = ngroups > warp ? (ngroups - warp + DW - 1) / DW : 0;
  const int items = my_groups * slabs;
  const float mult = (a.cfg.logits_scaling == 1.0f) ? 1.0f : __fdiv_rn(1.0f, a.cfg.logits_scaling);
  uint8_t* wstage = S.tab + (size_t)warp * TAB_STAGES * TAB_ROWS_W * TAB_PITCH;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  auto issue = [&](int item) {
    if (item < items) {
      int g = warp + DW * (item / slabs), slab = item % slabs;
      uint8_t* stage = wstage + (item % TAB_STAGES) * TAB_ROWS_W * TAB_PITCH;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        int c = lane + 32 * u, r = c >> 3, cc = c & 7;
        int row = v0 + g * TAB_ROWS_W + r;
        if (row < v1) cp_async16(stage + r * TAB_PITCH + cc * 16, T.codes + (size_t)row * T.k + slab * TAB_SLAB + cc * 16);
      }
      if (lane < TAB_ROWS_W) {
        int row = v0 + g * TAB_ROWS_W + lane;
        if (row < v1) {
          const uint8_t* src = (const uint8_t*)T.scales + ((size_t)row * (T.k / 32) + slab * 4) * (T.scale_f16 ? 2 : 4);
          if (T.scale_f16) cp_async8(stage + lane * TAB_PITCH + TAB_SLAB, src);
          else cp_async16(stage + lane * TAB_PITCH + TAB_SLAB, src);
        }
      }
    }
    cp_commit();
  };
  for (int i = 0; i < TAB_STAGES - 1; ++i) issue(i);
  if (!ready()) {
    cp_wait<0>();
    return false;
  }
  // The thread's 4 lanes as two packed pairs: byte -> float, times the
  // scale, fma into the chain, each rounded as the scalar steps are.
  float2 l01 = make_float2(0.0f, 0.0f), l23 = make_float2(0.0f, 0.0f);
  const float2 bias = make_float2(8388736.0f, 8388736.0f);
  for (int item = 0; item < items; ++item) {
    issue(item + TAB_STAGES - 1);
    cp_wait<TAB_STAGES - 1>();
    __syncwarp();
    int g = warp + DW * (item / slabs), slab = item % slabs;
    int row = v0 + g * TAB_ROWS_W + rl;
    const uint8_t* srow = wstage + (item % TAB_STAGES) * TAB_ROWS_W * TAB_PITCH + rl * TAB_PITCH;
#pragma unroll
    for (int st = 0; st < TAB_SLAB / 16; ++st) {
      int kk = slab * TAB_SLAB + 16 * st + 4 * q;
      uint32_t word = *(const uint32_t*)(srow + 16 * st + 4 * q) ^ 0x80808080u;
      float s = T.scale_f16 ? f16_bits_to_f32(((const uint16_t*)(srow + TAB_SLAB))[st >> 1])
                            : ((const float*)(srow + TAB_SLAB))[st >> 1];
      float4 xv = *(const float4*)(S.xf + kk);
      const float2 c01 = sub2(make_float2(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650)),
                                          __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7651))), bias);
      const float2 c23 = sub2(make_float2(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7652)),
                                          __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7653))), bias);
      const float2 s2 = make_float2(s, s);
      l01 = fma2(make_float2(xv.x, xv.y), mul2(c01, s2), l01);
      l23 = fma2(make_float2(xv.z, xv.w), mul2(c23, s2), l23);
    }
    const float lanes[4] = {l01.x, l01.y, l23.x, l23.y};
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
        if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
      }
      l01 = make_float2(0.0f, 0.0f);
      l23 = make_float2(0.0f, 0.0f);
    }
    __syncwarp();  // the stage is refilled by the next issue
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
  if (lane == 0) {
    S.red[warp] = bv;
    ((int*)S.red)[32 + warp] = bi;
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
  __syncthreads();
  return true;
}

__global__ void __launch_bounds__(DT, 1) k_decode(DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const DConfig& cfg = a.cfg;
  const int c = blockIdx.x, nb = gridDim.x;
  const int hd = 128, qd = cfg.heads * hd, kvd = cfg.kv_heads * hd, nqkv = qd + 2 * kvd;
  const int kmax = max(max(cfg.d, qd), cfg.ffn);
  const int tmax = (a.first_pos + a.steps + 3) / 4 * 4;  // the most keys a step sees, rounded up
  const int L = cfg.layers;
  const LlLayout ll(cfg, nb);
  Shared S;
  uint8_t* p = smem;
  S.flag = (int*)p; p += 64;
  S.red = (float*)p; p += 64 * 4;
  S.xf = (float*)p; p += (size_t)kmax * 4;
  S.sq = (float*)p; p += (size_t)kmax * 4;
  S.xq = (int8_t*)p; p += (size_t)kmax;
  S.xs = (float*)p; p += (size_t)(kmax / 32) * 4;
  S.own = (float*)p; p += 512 * 4;
  S.out = (float*)p; p += 512 * 4;
  S.nw = (float*)p; p += (size_t)cfg.d * 4;
  S.gmax = kmax / 32;
  S.part = (int*)p;  // union with the attention and table scratch
  S.att = (float*)p;
  S.tab = p;
  // The rows this block owns: x rows (o_proj and down_proj), qkv rows, ffn units, table rows.
  const int r0 = split_at(cfg.d, c, nb), r1 = split_at(cfg.d, c + 1, nb), nown = r1 - r0;
  const int q0 = split_at(nqkv, c, nb), q1 = split_at(nqkv, c + 1, nb);
  const int u0 = split_at(cfg.ffn, c, nb), u1 = split_at(cfg.ffn, c + 1, nb), nu = u1 - u0;
  const int v0 = split_at(a.table.n, c, nb), v1 = split_at(a.table.n, c + 1, nb);
  int mark_at = 0;
  auto mark = [&]() {
    if (a.phase_ns && c == 0 && threadIdx.x == 0) a.phase_ns[mark_at] = gtimer();
    ++mark_at;
  };
  int token = a.tokens[0];
  int cur_step = -1, cur_layer = 0;
  // Optional per-block event stamps of one step: [layer][16][grid].
  auto ev = [&](int k) {
    if (a.events && cur_step == a.event_step && threadIdx.x == 0)
      a.events[((size_t)cur_layer * kEventSlots + k) * nb + c] = gtimer();
  };
  for (int i = 0; i < a.steps; ++i) {
    cur_step = i;
    bool stopped = false;
    for (int s = 0; s < a.nstop; ++s) stopped |= a.stop[s] == token;
    if (stopped) {
      if (c == 0 && threadIdx.x == 0) *a.count = i;
      return;
    }
    const int pos = a.first_pos + i;
    const uint32_t base = (uint32_t)i * (uint32_t)(5 * L + 2) + 1;  // tags of this step: base + phase
    mark_at = i * (5 * L + 2);
    mark();
    // x = the token's embedding (causal_lm.rs:347-355, hidden :414).
    const DTable& E = a.embed;
    for (int kk = threadIdx.x; kk < cfg.d; kk += DT) {
      float v = __fmul_rn((float)E.codes[(size_t)token * E.k + kk], table_scale(E, token, kk / 32));
      if (cfg.embedding_multiplier != 1.0f) v = __fmul_rn(v, cfg.embedding_multiplier);
      S.xf[kk] = v;
      if (kk >= r0 && kk < r1) S.own[kk - r0] = v;
    }
    for (int l = 0; l < L; ++l) {
      cur_layer = l;
      ev(0);
      const DLayer& Lw = a.layers[l];
      const uint32_t t_qkv = base + 5 * l, t_att = t_qkv + 1, t_xa = t_qkv + 2, t_h = t_qkv + 3, t_xb = t_qkv + 4;
      const uint32_t t_x_in = t_qkv - 1;  // xb of the layer before
      // P1: qkv. Input: x (the embedding, or xb of the layer before).
      stage_norm(Lw.norm_attn, cfg.d, S);
      bool ok = gemv(Lw.qkv, q1 - q0, [&](int lr) { return q0 + lr; }, S, [&]() {
        if (l > 0 && !ll_wait(a.ll + ll.xb, cfg.d, t_x_in, a.status,
                              [&](int k, uint32_t v) { S.xf[k] = __uint_as_float(v); }))
          return false;
        ev(1);
        cp_wait<1>();  // the norm weights (the group before the product's first weight batch)
        norm_quant(cfg.d, S.nw, cfg.eps, Lw.qkv.agroup, Lw.qkv.half, S);
        ev(2);
        return true;
      }, ev, 16);
      if (!ok) return;
      ev(3);
      for (int lr = threadIdx.x; lr < q1 - q0; lr += DT)
        ll_put(a.ll + ll.qkv + qkv_slot(cfg, q0 + lr), __float_as_uint(S.out[lr]), t_qkv);
      ev(4);
      mark();
      // P2: attention.
      if (c < cfg.kv_heads) {
        if (!attend(a, Lw, l, pos, c, tmax, t_qkv, t_att, S, ev)) return;
      }
      mark();
      // P3: o_proj + residual. Input: the quantized attention output.
      const int ncode = qd / 4, nsc = qd / Lw.out.agroup;
      ok = gemv(Lw.out, nown, [&](int lr) { return r0 + lr; }, S, [&]() {
        // The codes (4 a word) and then the scales: one run of LL words.
        if (!ll_wait(a.ll + ll.attq, ncode + nsc, t_att, a.status, [&](int k, uint32_t v) {
              if (k < ncode) ((uint32_t*)S.xq)[k] = v;
              else ((uint32_t*)S.xs)[k - ncode] = v;
            }))
          return false;
        ev(8);
        return true;
      }, ev, 19);
      if (!ok) return;
      ev(9);
      mark();
      for (int lr = threadIdx.x; lr < nown; lr += DT) {
        float o = S.out[lr];
        float xv = (cfg.residual_multiplier == 1.0f) ? __fadd_rn(S.own[lr], o)
                                                     : __fadd_rn(S.own[lr], __fmul_rn(cfg.residual_multiplier, o));
        S.own[lr] = xv;
        ll_put(a.ll + ll.xa + r0 + lr, __float_as_uint(xv), t_xa);
      }
      // P4: gate_up, h = silu(gate) * up. Input: xa.
      stage_norm(Lw.norm_mlp, cfg.d, S);
      ok = gemv(Lw.gate_up, 2 * nu, [&](int lr) { return lr < nu ? u0 + lr : cfg.ffn + u0 + lr - nu; }, S, [&]() {
        if (!ll_wait(a.ll + ll.xa, cfg.d, t_xa, a.status, [&](int k, uint32_t v) { S.xf[k] = __uint_as_float(v); }))
          return false;
        ev(10);
        cp_wait<1>();
        norm_quant(cfg.d, S.nw, cfg.eps, Lw.gate_up.agroup, Lw.gate_up.half, S, Lw.ffn_scale);
        ev(11);
        return true;
      }, ev, 22);
      if (!ok) return;
      ev(12);
      mark();
      for (int lr = threadIdx.x; lr < nu; lr += DT)
        ll_put(a.ll + ll.h + u0 + lr, __float_as_uint(__fmul_rn(silu(S.out[lr]), S.out[nu + lr])), t_h);
      // P5: down + residual. Input: h.
      ok = gemv(Lw.down, nown, [&](int lr) { return r0 + lr; }, S, [&]() {
        if (!ll_wait(a.ll + ll.h, cfg.ffn, t_h, a.status, [&](int k, uint32_t v) { S.xf[k] = __uint_as_float(v); }))
          return false;
        ev(13);
        // h, every group at once (no norm): the FFN width is long enough
        // that a warp per group takes several rounds.
        __syncthreads();
        quantize_groups<DT, 4>(S.xf, cfg.ffn, nullptr, nullptr, 1.0f, Lw.down.agroup, Lw.down.half, S.xq, S.xs);
        __syncthreads();
        ev(14);
        return true;
      }, ev, 25);
      if (!ok) return;
      ev(15);
      mark();
      for (int lr = threadIdx.x; lr < nown; lr += DT) {
        float o = S.out[lr];
        float xv = (cfg.residual_multiplier == 1.0f) ? __fadd_rn(S.own[lr], o)
                                                     : __fadd_rn(S.own[lr], __fmul_rn(cfg.residual_multiplier, o));
        S.own[lr] = xv;
        ll_put(a.ll + ll.xb + r0 + lr, __float_as_uint(xv), t_xb);
      }
    }
    // The final RmsNorm (f32, no quantization), the table slice, the argmax.
    const uint32_t t_final = base + 5 * L - 1, t_best = base + 5 * L;
    bool ok = table_slice(a, v0, v1, i + 1, S, (float*)(S.flag + 4), S.flag + 5, [&]() {
      if (!ll_wait(a.ll + ll.xb, cfg.d, t_final, a.status, [&](int k, uint32_t v) { S.xf[k] = __uint_as_float(v); }))
        return false;
      for (int kk = threadIdx.x; kk < cfg.d; kk += DT) S.sq[kk] = __fmul_rn(S.xf[kk], S.xf[kk]);
      __syncthreads();
      if (threadIdx.x == 0) S.red[0] = rms_inv(seq_sum(S.sq, cfg.d), cfg.d, cfg.eps);
      __syncthreads();
      const float inv = S.red[0];
      for (int kk = threadIdx.x; kk < cfg.d; kk += DT) S.xf[kk] = __fmul_rn(S.xf[kk], __fmul_rn(inv, a.final_norm[kk]));
      __syncthreads();
      return true;
    });
    if (!ok) return;
    if (threadIdx.x == 0) {
      ll_put(a.ll + ll.best + 2 * c, (uint32_t)S.flag[4], t_best);
      ll_put(a.ll + ll.best + 2 * c + 1, (uint32_t)S.flag[5], t_best);
    }
    // Every block reduces all blocks' bests to the same token.
    float* bvals = (float*)S.part;
    int* bidx = S.part + nb;
    ok = ll_wait(a.ll + ll.best, 2 * nb, t_best, a.status, [&](int k, uint32_t v) {
      if (k & 1) bidx[k >> 1] = (int)v;
      else bvals[k >> 1] = __uint_as_float(v);
    });
    if (!ok) return;
    mark();
    if (threadIdx.x < 32) {
      float b = -INFINITY;
      int ix = 0x7fffffff;
      for (int k = threadIdx.x; k < nb; k += 32)
        if (bvals[k] > b || (bvals[k] == b && bidx[k] < ix)) { b = bvals[k]; ix = bidx[k]; }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        float ob = __shfl_xor_sync(0xffffffffu, b, o);
        int oi = __shfl_xor_sync(0xffffffffu, ix, o);
        if (ob > b || (ob == b && oi < ix)) { b = ob; ix = oi; }
      }
      if (threadIdx.x == 0) S.flag[2] = (ix == 0x7fffffff) ? 0 : ix;
    }
    __syncthreads();
    token = S.flag[2];
    if (c == 0 && threadIdx.x == 0) a.tokens[i + 1] = token;
    __syncthreads();
  }
  if (c == 0 && threadIdx.x == 0) *a.count = a.steps;
}

size_t head_smem(const DConfig& cfg) {
  const int qd = cfg.heads * 128;
  const int kmax = std::max(std::max(cfg.d, qd), cfg.ffn);
  return 64 + 64 * 4 + (size_t)kmax * 8 + kmax + (size_t)(kmax / 32) * 4 + 512 * 4 + 512 * 4 + (size_t)cfg.d * 4;
}

// The union region: the largest of the GEMV group dots and scales, the
// attention scratch, the table stages and the argmax partials.
size_t union_smem(const DConfig& cfg, int grid, int f16, int tmax, int kt) {
  const int qd = cfg.heads * 128;
  size_t u = 0;
  const int kmax = std::max(std::max(cfg.d, qd), cfg.ffn);
  // Two staging buffers, then [group][row] dots and scale products for the
  // rows of a batch (at most WSTAGE / 32 group-row pairs: a staged row
  // takes at least 32 bytes a group).
  u = std::max(u, (size_t)2 * WSTAGE + (size_t)(WSTAGE / 32) * 8);
  u = std::max(u, (size_t)DW * TAB_STAGES * TAB_ROWS_W * TAB_PITCH);
  u = std::max(u, (size_t)grid * 8);
  u = std::max(u, attend_smem_floats(cfg.heads / cfg.kv_heads, tmax, f16, kt) * 4);
  return u;
}

}  // namespace

bool decode_supported(const DConfig& cfg) {
  auto ok = [](int k) { return k % 128 == 0 && k <= 8192; };
  int qpk = cfg.heads / cfg.kv_heads;
  return cfg.hd == 128 && ok(cfg.d) && ok(cfg.heads * 128) && ok(cfg.ffn) && qpk * 128 <= DT &&
         true;
}

int decode_grid(int device) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return 0;
  return prop.multiProcessorCount;
}

size_t decode_ll_words(const DConfig& cfg, int grid) { return (size_t)LlLayout(cfg, grid).total; }

cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t s) {
  if (!decode_supported(a.cfg)) return cudaErrorNotSupported;
  const int tmax = (a.first_pos + a.steps + 3) / 4 * 4;
  if ((a.cfg.heads / a.cfg.kv_heads) * 128 > 4 * DT || a.cfg.kv_heads > grid) return cudaErrorInvalidValue;
  // A staged weight row fits a staging buffer.
  for (int l = 0; l < 1; ++l) {
    const int kmax = std::max(std::max(a.cfg.d, a.cfg.heads * 128), a.cfg.ffn);
    if (kmax + kmax / 16 + 32 > WSTAGE) return cudaErrorInvalidValue;
  }
  // Per block: at most 512 own rows and 256 ffn units (S.own, S.out).
  if ((a.cfg.d + grid - 1) / grid > 512 || 2 * ((a.cfg.ffn + grid - 1) / grid) > 512) return cudaErrorInvalidValue;
  if (((a.cfg.heads * 128 + 2 * a.cfg.kv_heads * 128) + grid - 1) / grid > 512) return cudaErrorInvalidValue;
  int kt = attend_kt(a.cache.f16, true);
  size_t smem = head_smem(a.cfg) + union_smem(a.cfg, grid, a.cache.f16, tmax, kt);
  if (smem > 227 * 1024) {
    kt = attend_kt(a.cache.f16, false);
    smem = head_smem(a.cfg) + union_smem(a.cfg, grid, a.cache.f16, tmax, kt);
  }
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode, DT, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
  DecodeArgs args = a;
  args.key_tile = kt;
  void* params[] = {&args};
  return cudaLaunchCooperativeKernel((const void*)k_decode, dim3(grid), dim3(DT), params, smem, s);
}

}  // namespace trit
