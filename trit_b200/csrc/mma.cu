// W8A8 products on the fifth-generation tensor cores (tcgen05.mma
// kind::i8) for prompt prefill and batches of streams: Int8::forward_biased
// (src/cpu/int8.rs:425-483) with the VNNI tile's float order (:560-570):
// for every output row and frame, acc = fma(f32(dot_g), ws_g * xs_g, acc)
// over the activation groups g in order, where dot_g is the exact i32 dot
// product of the group's codes. The tensor cores make each dot_g exactly;
// the CUDA cores run the f32 chain in order, so every output is the
// reference's value to the bit.
//
// One CTA owns 128 weight rows (the MMA's M, one TMEM lane each) and 64
// frames (N). Warp roles:
//   warp 0     TMA producer: a stage is 128 bytes of K for the CTA's weight
//              rows and frames, one 128-byte line per row with the 128-byte
//              swizzle (16-byte chunk c of row r at chunk c ^ (r % 8)), the
//              K-major SWIZZLE_128B layout of the tcgen05 shared-memory
//              descriptor, by one 2-D tensor copy each;
//   warp 1     allocates TMEM; lane 0 issues one MMA (K = 32) per step into
//              one of four TMEM accumulators and commits it to an mbarrier:
//              a 32-value group (Q8_0) is one MMA, a 128-value group
//              (per-row int8, ternary) four MMAs into the same accumulator;
//   warps 2-9  epilogue: per group, load the 128 x 64 accumulator from TMEM
//              (warp w: lanes 32 (w % 4).., columns 32 ((w - 2) / 4)..),
//              store the bias back (tcgen05.st), free the buffer, and fold
//              the group into 32 f32 chains per thread with packed f32x2
//              arithmetic (each lane rounds as the scalar instruction does).
//              Every accumulator starts at the bits of 1.5 * 2^23, so after
//              the MMAs it holds the float 1.5 * 2^23 + dot (|dot| < 2^22)
//              and one exact subtraction gives f32(dot). The epilogue warps
//              also stage the frames' activation scales while the first
//              stages load.
// Every wait is bounded in time; a wait that runs out sets the kernel's
// status, the CTA waits (bounded) for its copies and MMAs in flight, frees
// its TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "device.cuh"
#include "kernels.h"

namespace trit {
namespace {

constexpr int TC_M = 128;
constexpr int TC_N = 64;
constexpr int TC_KT = 128;  // K bytes a stage (four MMA steps of K = 32)
constexpr int TC_STAGES = 4;
constexpr int TC_BUFS = 4;
constexpr int TC_EPI_WARPS = 8;   // two per TMEM lane quarter, 32 columns each
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr int A_STAGE = TC_M * TC_KT;  // 16 KB
constexpr int B_STAGE = TC_N * TC_KT;  // 8 KB
constexpr int TC_TMEM_COLS = TC_BUFS * TC_N;  // 256 (a power of two >= 32)
constexpr long long TC_WAIT_NS = 2000000000ll;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return (long long)t;
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase of parity `parity` of *b; false when another role
// gave up (*abort) or the wait ran past TC_WAIT_NS (then it sets *abort).
__device__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort) {
  long long start = 0;
  for (uint32_t i = 0;; ++i) {
    if (mbar_test(b, parity)) return true;
    if ((i & 63) == 63) {
      if (*abort) return false;
      long long t = now_ns();
      if (!start) start = t;
      else if (t - start > TC_WAIT_NS) {
        *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor, K-major with the 128-byte swizzle: rows
// of 128 bytes, 8-row groups 1024 bytes apart (SBO); the leading offset is
// unused for this layout (encoded 1). `addr` may step through the 128-byte
// line in 32-byte K steps: the swizzle applies to the absolute address, and
// the stage bases are 1024-byte aligned (base offset 0). Bit 46 is the
// descriptor version of sm_100; bits 61-63 = 2 select SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor of kind::i8: D s32 (bits 4-5 = 2), A and B s8
// (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_N >> 3) << 17) |
                            ((uint32_t)(TC_M >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define TC_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                 "=r"(r[i + 6]), "=r"(r[i + 7])
// 32 consecutive TMEM columns of this warp's 32 lanes: r[j] = column j of
// the thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : TC_R8(0), TC_R8(8), TC_R8(16), TC_R8(24)
      : "r"(taddr));
}
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
// Every accumulator starts at the bits of 1.5 * 2^23 (kBias); after the
// MMAs add the i32 dot, the word is the float 1.5 * 2^23 + dot (ulp 1 for
// |dot| <= 2^22), and subtracting 1.5 * 2^23 gives f32(dot) exactly.
constexpr uint32_t kBias = 0x4B400000u;
__device__ __forceinline__ float2 biased_dots(uint32_t a, uint32_t b) {
  return add2(make_float2(__uint_as_float(a), __uint_as_float(b)), make_float2(-12582912.0f, -12582912.0f));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// kBias into 32 consecutive TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st32_bias(uint32_t taddr) {
  const uint32_t v = kBias;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}

struct TcSmem {
  uint64_t full[TC_STAGES], empty[TC_STAGES], tfull[TC_BUFS], tempty[TC_BUFS], drain;
  uint32_t tmem;
  int abort;
};

// y (m x ldy) <- the product of W (rows [0, n)) and the quantized frames
// xq / xs (m rows). mode kEpOut: y = acc; kEpResid: y += acc (times mult).
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, DMat W,
              const float* xs, int m, int mode, float* y, int ldy, float resid_mult, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* a_st = base;
  uint8_t* b_st = a_st + TC_STAGES * A_STAGE;
  const int G = W.agroup, groups = W.k / G;
  float* xs_s = (float*)(b_st + TC_STAGES * B_STAGE);  // [groups][TC_N]
  TcSmem* S = (TcSmem*)(xs_s + TC_N * groups);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TC_M, f0 = blockIdx.y * TC_N;
  const int ktiles = W.k / TC_KT;
  volatile int* abort = &S->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
    }
    for (int b = 0; b < TC_BUFS; ++b) {
      mbar_init(&S->tfull[b], 1);
      mbar_init(&S->tempty[b], 32 * TC_EPI_WARPS);
    }
    mbar_init(&S->drain, 1);
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S->tmem)),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S->tmem;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kt = 0; kt < ktiles; ++kt) {
        const int s = kt % TC_STAGES;
        if (!mbar_wait(&S->empty[s], ((kt / TC_STAGES) & 1) ^ 1, abort)) break;
        mbar_expect_tx(&S->full[s], A_STAGE + B_STAGE);
        tma_load_2d(a_st + s * A_STAGE, &amap, &S->full[s], kt * TC_KT, n0);
        tma_load_2d(b_st + s * B_STAGE, &bmap, &S->full[s], kt * TC_KT, f0);
        issued = kt + 1;
      }
      if (*abort) {
        // Let the copies in flight land before the CTA's memory is released.
        for (int kt = (issued > TC_STAGES ? issued - TC_STAGES : 0); kt < issued; ++kt) {
          long long t0 = now_ns();
          while (!mbar_test(&S->full[kt % TC_STAGES], (kt / TC_STAGES) & 1) && now_ns() - t0 < TC_WAIT_NS) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t a0 = smem_u32(a_st), b0 = smem_u32(b_st);
      bool ok = true;
      for (int kt = 0; kt < ktiles && ok; ++kt) {
        const int s = kt % TC_STAGES;
        if (!mbar_wait(&S->full[s], (kt / TC_STAGES) & 1, abort)) break;
        fence_after();
        for (int j = 0; j < TC_KT / 32; ++j) {
          const int step = kt * (TC_KT / 32) + j;  // K = 32 steps so far
          const int g = step * 32 / G;
          const bool first = (step * 32) % G == 0, last = ((step + 1) * 32) % G == 0;
          const int b = g % TC_BUFS;
          if (first) {
            if (!mbar_wait(&S->tempty[b], (g / TC_BUFS) & 1, abort)) {
              ok = false;
              break;
            }
            fence_after();
          }
          const uint64_t ad = smem_desc_sw128(a0 + s * A_STAGE + j * 32);
          const uint64_t bd = smem_desc_sw128(b0 + s * B_STAGE + j * 32);
          mma_i8(tmem + b * TC_N, ad, bd, 1u);
          if (last) mma_commit(&S->tfull[b]);
        }
        mma_commit(&S->empty[s]);
      }
      // Every MMA issued has finished once `drain` completes.
      mma_commit(&S->drain);
      long long t0 = now_ns();
      while (!mbar_test(&S->drain, 0) && now_ns() - t0 < TC_WAIT_NS) {
      }
    }
  } else {
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int lr = quarter * 32 + lane;
    const int row = n0 + lr;
    const bool live = row < W.n;
    const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16) + half * 32;  // + buffer * TC_N
    // Bias every accumulator, then hand all of them to the MMA thread.
    for (int b = 0; b < TC_BUFS; ++b) tmem_st32_bias(tl + b * TC_N);
    tmem_wait_st();
    fence_before();
    for (int b = 0; b < TC_BUFS; ++b) mbar_arrive(&S->tempty[b]);
    // Weight scales 8 groups ahead, so their loads overlap the MMAs.
    float wcur[8], wnxt[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) wcur[i] = (live && i < groups) ? weight_scale(W, row, i) : 0.0f;
    // The frames' activation scales, [group][frame] (frames past m read as
    // 0): coalesced reads of xs rows, eight in flight per thread, while the
    // first stages load and multiply.
    {
      const int total = TC_N * groups, t0 = threadIdx.x - 64, nt = 32 * TC_EPI_WARPS;
      for (int i0 = t0; i0 < total; i0 += 8 * nt) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * nt, f = i / groups, g = i - f * groups;
          v[u] = (i < total && f0 + f < m) ? __ldg(xs + (size_t)(f0 + f) * groups + g) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * nt, f = i / groups, g = i - f * groups;
          if (i < total) xs_s[g * TC_N + f] = v[u];
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(32 * TC_EPI_WARPS) : "memory");
    }
    float2 acc[16];  // frames 32 half + 2 i, + 1
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
    auto fetch = [&](int g, uint32_t (&r)[32]) -> bool {
      const int b = g % TC_BUFS;
      if (!mbar_wait(&S->tfull[b], (g / TC_BUFS) & 1, abort)) return false;
      fence_after();
      tmem_ld32(tl + b * TC_N, r);
      return true;
    };
    // One group: the next group's accumulator loads from TMEM while this
    // group's chains run; this group's buffer goes back to the MMA thread
    // once its bias store (issued a group earlier) has landed.
    auto step = [&](int g, float w, const uint32_t (&rc)[32], uint32_t (&rn)[32]) -> bool {
      const bool more = g + 1 < groups;
      if (more && !fetch(g + 1, rn)) return false;
      const float2 ws2 = make_float2(w, w);
      const float4* xg = (const float4*)(xs_s + g * TC_N + half * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 xv = xg[q];
        acc[2 * q] = fma2(biased_dots(rc[4 * q], rc[4 * q + 1]), mul2(ws2, make_float2(xv.x, xv.y)), acc[2 * q]);
        acc[2 * q + 1] =
            fma2(biased_dots(rc[4 * q + 2], rc[4 * q + 3]), mul2(ws2, make_float2(xv.z, xv.w)), acc[2 * q + 1]);
      }
      tmem_wait_ld();
      tmem_wait_st();
      fence_before();
      mbar_arrive(&S->tempty[g % TC_BUFS]);
      if (more) tmem_st32_bias(tl + ((g + 1) % TC_BUFS) * TC_N);
      return true;
    };
    uint32_t ra[32], rb[32];
    bool ok = fetch(0, ra);
    if (ok) {
      tmem_wait_ld();
      tmem_st32_bias(tl);
    }
    for (int gc = 0; gc < groups && ok; gc += 8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) wnxt[i] = (live && gc + 8 + i < groups) ? weight_scale(W, row, gc + 8 + i) : 0.0f;
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        if (gc + i >= groups) break;
        if (!step(gc + i, wcur[i], ra, rb)) {
          ok = false;
          break;
        }
        if (gc + i + 1 >= groups) break;
        if (!step(gc + i + 1, wcur[i + 1], rb, ra)) {
          ok = false;
          break;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) wcur[i] = wnxt[i];
    }
    tmem_wait_st();
    if (ok && live) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int f = f0 + half * 32 + j;
        const float v = (j & 1) ? acc[j >> 1].y : acc[j >> 1].x;
        if (f < m) {
          float* p = y + (size_t)f * ldy + row;
          if (mode == kEpOut) *p = v;
          else *p = (resid_mult == 1.0f) ? __fadd_rn(*p, v) : __fadd_rn(*p, __fmul_rn(resid_mult, v));
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
  }
  if (threadIdx.x == 0 && S->abort) atomicExch(status, 1);
}

// silu(gate) * up of a stacked gate|up product (causal_lm.rs:464-474):
// g = [m][2 * units], h = [m][units].
__global__ void k_silu_pairs(const float* g, int m, int units, float* h) {
  size_t total = (size_t)m * units;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    size_t r = i / units, u = i % units;
    const float* row = g + r * 2 * units;
    h[i] = __fmul_rn(silu(row[u]), row[units + u]);
  }
}

// Bits 2s..2s+1 of byte j of word w hold the code of k = 16 w + 4 s + j
// (pack_span, src/cpu/kernels.rs:624-628); the int8 value is code - 1.
__global__ void k_expand_ternary(const uint32_t* words, size_t n, int k, int8_t* out) {
  const int wpr = k / 16;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n * wpr; i += (size_t)gridDim.x * blockDim.x) {
    uint32_t w = words[i];
    size_t r = i / wpr;
    int c0 = (int)(i % wpr) * 16;
    int8_t v[16];
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * s + j] = (int8_t)(((w >> (8 * j + 2 * s)) & 3u) - 1);
    *(int4*)(out + r * k + c0) = *(const int4*)v;
  }
}

size_t tc_smem_bytes(const DMat& W) {
  size_t groups = W.k / W.agroup;
  return 1024 + (size_t)TC_STAGES * (A_STAGE + B_STAGE) + (size_t)TC_N * groups * 4 + sizeof(TcSmem);
}

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiled)p;
  });
  return fn;
}

}  // namespace

int tc_frames() { return TC_N; }

// A 2-D view (k bytes, rows) of a row-major int8 matrix [rows][k]; a box is
// one stage (TC_KT = 128 bytes of K) of `box_rows` rows, written to shared
// memory with the 128-byte swizzle. Rows past `rows` read as zero.
cudaError_t make_tc_map(TcMap* out, const void* base, size_t rows, size_t k, int box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return cudaErrorNotSupported;
  if (rows % 8 || k % TC_KT || ((uintptr_t)base & 15) || box_rows % 8 || box_rows > 256) return cudaErrorInvalidValue;
  static_assert(TC_KT == 128, "a stage's K is one 128-byte swizzle line");
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {k};
  cuuint32_t box[2] = {TC_KT, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  static_assert(sizeof(TcMap) == sizeof(CUtensorMap), "TcMap holds a CUtensorMap");
  CUresult r = enc((CUtensorMap*)out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_tc_weight_map(TcMap* out, const DMat& W, const void* codes8) {
  return make_tc_map(out, codes8, (size_t)W.n, (size_t)W.k, TC_M);
}
cudaError_t make_tc_frame_map(TcMap* out, const int8_t* xq, size_t rows_cap, size_t k) {
  return make_tc_map(out, xq, rows_cap, k, TC_N);
}

cudaError_t launch_gemm_tc(const TcMap& amap, const TcMap& bmap, const DMat& W, const float* xs, int m, int mode,
                           float* y, int ldy, float resid_mult, int* status, cudaStream_t s) {
  if (W.k % TC_KT || (W.agroup != 32 && W.agroup != 128) || m <= 0) return cudaErrorInvalidValue;
  size_t smem = tc_smem_bytes(W);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid((W.n + TC_M - 1) / TC_M, (m + TC_N - 1) / TC_N);
  k_gemm_tc<<<grid, TC_THREADS, smem, s>>>(*(const CUtensorMap*)&amap, *(const CUtensorMap*)&bmap, W, xs, m, mode, y,
                                            ldy, resid_mult, status);
  return cudaGetLastError();
}

cudaError_t launch_expand_ternary(const DMat& W, int8_t* out, cudaStream_t s) {
  if (W.kind != kTernary || W.k % 16) return cudaErrorInvalidValue;
  k_expand_ternary<<<148 * 8, 256, 0, s>>>((const uint32_t*)W.codes, (size_t)W.n, W.k, out);
  return cudaGetLastError();
}

cudaError_t launch_silu_pairs(const float* g, int m, int units, float* h, cudaStream_t s) {
  size_t total = (size_t)m * units;
  int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  k_silu_pairs<<<blocks, 256, 0, s>>>(g, m, units, h);
  return cudaGetLastError();
}

}  // namespace trit
