// GQA softmax attention of one query position over its stream's keys, in
// the reference's arithmetic order (src/layers.rs:343-504 and
// softmax_rows :571-587, with the nn tiles of src/cpu/fgemm.rs:700-860):
//   score_j  = fma chain over the head dimension, e = 0..127, of q_e * k_je
//              (q already times 1/sqrt(hd))
//   max      = the largest score
//   e_j      = exp(score_j - max) (the Cephes polynomial)
//   sum      = e_0 + e_1 + ... in key order
//   p_j      = e_j * (1 / sum)
//   out_e    = fma chain over the keys in order of p_j * v_je
// so each output is the reference's value bit for bit (keys that the causal
// mask hides come after the visible ones and add less than an ulp; they
// are skipped). One block handles the `qpk` query heads of one kv head;
// keys and values come through shared memory in tiles of `kt` rows.
#pragma once

#include "device.cuh"

namespace trit {

// Shared memory of exact_attention, in floats.
__host__ __device__ inline size_t attention_smem_floats(int qpk, int tmax, int kt, int f16) {
  size_t row = f16 ? 64 : 128;  // a staged key or value row, as floats
  return (size_t)qpk * tmax + (size_t)kt * (row + 4) + (size_t)kt * row + 2 * (size_t)qpk + 64;
}

template <int NT>
struct Attention {
  const DCache& cache;
  const DConfig& cfg;
  int stream, layer, kvh, qpk, kt;
  float* sc;    // [qpk][tmax] scores, then probabilities
  float* ktl;   // [kt][row + 4] staged keys (pitch avoids bank conflicts)
  float* vtl;   // [kt][row] staged values
  float* stat;  // [2 * qpk + 64]
  int tmax;

  __device__ int row_floats() const { return cache.f16 ? 64 : 128; }

  // Starts the copy of keys (which 0) or values (which 1) [j0, j0 + n)
  // into dst (cp.async; run() waits for it); position `skip` (or -1) is
  // left for the caller to fill.
  __device__ void stage(int which, int j0, int n, int skip, float* dst, int pitch) {
    const int cpr = cache.f16 ? 16 : 32;  // 16-byte chunks a row
    for (int ci = threadIdx.x; ci < n * cpr; ci += NT) {
      int jj = ci / cpr, cc = ci % cpr, j = j0 + jj;
      if (j == skip) continue;
      int page = cache.page_table[(size_t)stream * cache.pages_per_stream + j / cache.page_tokens];
      size_t off = kv_offset(cache, cfg, page, layer, which, kvh, j % cache.page_tokens);
      const int4* src = cache.f16 ? (const int4*)((const __half*)cache.pool + off) : (const int4*)((const float*)cache.pool + off);
      cp_async16(dst + jj * pitch + cc * 4, src + cc);
    }
    cp_commit();
  }
  // Stages tile 0 of keys and values ([0, min(kt, T)), except T - 1).
  __device__ void preload(int T, bool skip_last) {
    int n = min(kt, T);
    stage(0, 0, n, skip_last ? T - 1 : -1, ktl, row_floats() + 4);
    stage(1, 0, n, skip_last ? T - 1 : -1, vtl, row_floats());
  }

  __device__ float dot_key(const float* q, const float* krow) const {
    float x = 0.0f;
    if (cache.f16) {
      const int4* kp = (const int4*)krow;
      for (int i = 0; i < 16; ++i) {
        int4 raw = kp[i];
        const __half2* h2 = (const __half2*)&raw;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float2 f = __half22float2(h2[u]);
          x = __fmaf_rn(q[8 * i + 2 * u], f.x, x);
          x = __fmaf_rn(q[8 * i + 2 * u + 1], f.y, x);
        }
      }
    } else {
      const float4* kp = (const float4*)krow;
      for (int i = 0; i < 32; ++i) {
        float4 f = kp[i];
        x = __fmaf_rn(q[4 * i], f.x, x);
        x = __fmaf_rn(q[4 * i + 1], f.y, x);
        x = __fmaf_rn(q[4 * i + 2], f.z, x);
        x = __fmaf_rn(q[4 * i + 3], f.w, x);
      }
    }
    return x;
  }

  // Writes a key or value row given as f32 (rounded to f16 for an f16
  // cache) into a staged row.
  __device__ void put_row(float* dst, const float* v) const {
    for (int e = threadIdx.x; e < 128; e += NT) {
      if (cache.f16) ((__half*)dst)[e] = __float2half_rn(v[e]);
      else dst[e] = v[e];
    }
  }

  // q: [qpk][128] in shared memory; keys [0, T). cur_k / cur_v (or null):
  // the key and value of position T - 1 from the caller, used instead of
  // the cache. `tile0_ready`: keys and values [0, min(kt, T)) other than
  // T - 1 are already staged. out: [qpk][128].
  __device__ void run(const float* q, int T, const float* cur_k, const float* cur_v, bool tile0_ready, float* out) {
    const int t = threadIdx.x;
    const int row = row_floats(), kpitch = row + 4;
    const int pos = T - 1;
    // Scores, tile by tile.
    for (int j0 = 0; j0 < T; j0 += kt) {
      const int n = min(kt, T - j0);
      if (!(j0 == 0 && tile0_ready)) {
        __syncthreads();
        stage(0, j0, n, cur_k ? pos : -1, ktl, kpitch);
      }
      if (cur_k && pos >= j0 && pos < j0 + n) put_row(ktl + (pos - j0) * kpitch, cur_k);
      cp_wait_all();
      __syncthreads();
      for (int p = t; p < qpk * n; p += NT) {
        int qh = p / n, jj = p % n;
        sc[qh * tmax + j0 + jj] = dot_key(q + qh * 128, ktl + jj * kpitch);
      }
    }
    __syncthreads();
    // Max, exp, the sum in key order, the probabilities.
    const int warp = t >> 5, lane = t & 31;
    for (int qh = warp; qh < qpk; qh += NT / 32) {
      float mx = -INFINITY;
      for (int j = lane; j < T; j += 32) mx = fmaxf(mx, sc[qh * tmax + j]);
      mx = warp_max(mx);
      for (int j = lane; j < T; j += 32) sc[qh * tmax + j] = cephes_exp(__fsub_rn(sc[qh * tmax + j], mx));
      __syncwarp();
      if (lane == 0) {
        // In key order; unrolled so that the loads run ahead of the adds.
        float sum = 0.0f;
#pragma unroll 8
        for (int j = 0; j < T; ++j) sum = __fadd_rn(sum, sc[qh * tmax + j]);
        stat[qh] = __fdiv_rn(1.0f, sum);
      }
      __syncwarp();
      float inv = stat[qh];
      for (int j = lane; j < T; j += 32) sc[qh * tmax + j] = __fmul_rn(sc[qh * tmax + j], inv);
    }
    // Values, tile by tile: one thread per (q head, dimension), keys in order.
    float acc[4];
    const int per = (qpk * 128 + NT - 1) / NT;  // (head, dim) pairs a thread (<= 4: the host checks)
    for (int u = 0; u < 4; ++u) acc[u] = 0.0f;
    for (int j0 = 0; j0 < T; j0 += kt) {
      const int n = min(kt, T - j0);
      __syncthreads();
      if (!(j0 == 0 && tile0_ready)) stage(1, j0, n, cur_v ? pos : -1, vtl, row);
      if (cur_v && pos >= j0 && pos < j0 + n) put_row(vtl + (pos - j0) * row, cur_v);
      cp_wait_all();
      __syncthreads();
      for (int u = 0; u < per; ++u) {
        int pe = t + u * NT;
        if (pe >= qpk * 128) break;
        int qh = pe / 128, e = pe % 128;
        const float* pr = sc + qh * tmax + j0;
        float x = acc[u];
        if (cache.f16) {
          const __half* vp = (const __half*)vtl;
#pragma unroll 8
          for (int jj = 0; jj < n; ++jj) x = __fmaf_rn(pr[jj], __half2float(vp[jj * 2 * row + e]), x);
        } else {
#pragma unroll 8
          for (int jj = 0; jj < n; ++jj) x = __fmaf_rn(pr[jj], vtl[jj * row + e], x);
        }
        acc[u] = x;
      }
    }
    for (int u = 0; u < per; ++u) {
      int pe = t + u * NT;
      if (pe < qpk * 128) out[pe] = acc[u];
    }
    __syncthreads();
  }
};

}  // namespace trit
