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

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "device.cuh"
#include "kernels.h"

namespace trit {
namespace {

constexpr int TC_M = 128;
constexpr int TC_NMAX = 64;  // frames a CTA at most: the frame buffers' row multiple
constexpr int TC_FBOX = 16;  // frame rows a TMA box (a CTA of N frames loads N / 16)
constexpr int TC_KT = 128;   // K bytes a stage (four MMA steps of K = 32)
constexpr int TC_GPS = TC_KT / 32;  // groups a stage holds at most (Q8_0)
constexpr int TC_STAGES = 4;
constexpr int TC_EPI_WARPS = 8;  // two per TMEM lane quarter, N / 2 columns each
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr int A_STAGE = TC_M * TC_KT;  // 16 KB
constexpr long long TC_WAIT_NS = 2000000000ll;  // 2 s

// A CTA's frame tile: N frames (the MMA's N). A TMEM buffer holds one
// stage's group accumulators side by side (TC_GPS x N columns).
// F16: the codes as f16 (exact: |code| <= 128), so a stage's 128 bytes
// hold 64 values, two 32-value groups, and the MMA (kind::f16, f32
// accumulators) makes each group's dot as an exact f32 (every partial sum
// is an integer below 2^24).
template <int N, bool F16 = false>
struct TcShape {
  static_assert(N == 16 || N == 32 || N == 64, "frame tiles of 16, 32 or 64");
  static constexpr int B_STAGE = N * TC_KT;
  static constexpr int GPS = F16 ? 2 : TC_GPS;       // 32-value groups a stage
  static constexpr int BUF_COLS = GPS * N;
  static constexpr int BUFS = F16 ? (N == 16 ? 8 : 4) : (N == 16 ? 4 : 2);
  static constexpr int TMEM_COLS = BUFS * BUF_COLS;  // 512, 256, 256: powers of two
  static_assert(BUFS <= 8, "TcSmem holds 8 buffer barriers");
  static constexpr int CW = N / 2;                   // columns an epilogue warp folds
  static constexpr int CTAS = N == 64 ? 1 : 2;       // CTAs an SM holds (TMEM, shared memory)
};

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
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
}

// Instruction descriptor of kind::f16: D f32 (bits 4-5 = 1), A and B f16
// (bits 7-9, 10-12 = 0), A K-major, B K-major or MN-major (bit 16), N >> 3
// at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_f16n(int n, bool b_mn_major = false) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
}

// D = A B (+ D when `accumulate`).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3));
}
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define TC_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                 "=r"(r[i + 6]), "=r"(r[i + 7])
// C consecutive TMEM columns of this warp's 32 lanes: r[j] = column j of
// the thread's lane.
template <int C>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[C]) {
  static_assert(C == 8 || C == 16 || C == 32, "8, 16 or 32 columns");
  if constexpr (C == 32) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : TC_R8(0), TC_R8(8), TC_R8(16), TC_R8(24)
        : "r"(taddr));
  } else if constexpr (C == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : TC_R8(0), TC_R8(8)
        : "r"(taddr));
  } else {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : TC_R8(0)
                 : "r"(taddr));
  }
}
// Two i32 dots as exact floats: the bits of 1.5 * 2^23 plus the dot are
// the float 1.5 * 2^23 + dot (ulp 1 for |dot| <= 2^22), and subtracting
// 1.5 * 2^23 gives f32(dot) exactly.
__device__ __forceinline__ float2 dots_to_float2(uint32_t a, uint32_t b) {
  return add2(make_float2(__int_as_float(0x4B400000 + (int)a), __int_as_float(0x4B400000 + (int)b)),
              make_float2(-12582912.0f, -12582912.0f));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The weight scales of 8 consecutive groups of one row, as loaded: Q8_0 f16
// (a: 8 halves), f32 per group (a, b: 8 floats) or one f32 per row (a.x).
struct Ws8 {
  uint4 a, b;
  __device__ float get(const DMat& W, int i) const {
    if (W.kind == kQ8_0) {
      const uint32_t w = (i < 2) ? a.x : (i < 4) ? a.y : (i < 6) ? a.z : a.w;
      return f16_bits_to_f32((i & 1) ? (w >> 16) : (w & 0xFFFF));
    }
    if (W.kind == kInt8Row) return __uint_as_float(a.x);
    const uint4 v = (i < 4) ? a : b;
    const int j = i & 3;
    return __uint_as_float(j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w);
  }
};
// Whether every row's chunks of 8 scales start 16-byte aligned.
__device__ __forceinline__ bool ws_vector_ok(const DMat& W, int groups) {
  if (W.kind == kQ8_0) return groups % 8 == 0 && ((uintptr_t)W.scales & 15) == 0;
  if (W.kind == kInt8Row) return true;
  return groups % 4 == 0 && ((uintptr_t)W.scales & 15) == 0;
}
__device__ __forceinline__ Ws8 load_ws8(const DMat& W, int row, bool live, int g0, int groups, bool vec) {
  Ws8 r{make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  if (!live || g0 >= groups) return r;
  if (W.kind == kInt8Row) {
    r.a.x = __float_as_uint(((const float*)W.scales)[row]);
    return r;
  }
  if (vec && g0 + 8 <= groups) {
    if (W.kind == kQ8_0) {
      r.a = __ldg((const uint4*)((const uint16_t*)W.scales + (size_t)row * groups + g0));
    } else {
      const uint4* p = (const uint4*)((const float*)W.scales + (size_t)row * groups + g0);
      r.a = __ldg(p);
      r.b = __ldg(p + 1);
    }
    return r;
  }
  // Unaligned rows or the last chunk: one scale at a time.
  uint32_t v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = 0;
  for (int i = 0; i < 8 && g0 + i < groups; ++i) {
    if (W.kind == kQ8_0) v[i] = ((const uint16_t*)W.scales)[(size_t)row * groups + g0 + i];
    else v[i] = __float_as_uint(((const float*)W.scales)[(size_t)row * groups + g0 + i]);
  }
  if (W.kind == kQ8_0) {
    r.a = make_uint4(v[0] | (v[1] << 16), v[2] | (v[3] << 16), v[4] | (v[5] << 16), v[6] | (v[7] << 16));
  } else {
    r.a = make_uint4(v[0], v[1], v[2], v[3]);
    r.b = make_uint4(v[4], v[5], v[6], v[7]);
  }
  return r;
}

struct TcSmem {
  uint64_t full[TC_STAGES], empty[TC_STAGES], tfull[8], tempty[8], drain;  // up to 8 TMEM buffers
  uint32_t tmem;
  int abort;
};

// y (m x ldy) <- the product of W (rows [0, n)) and the quantized frames
// xq / xs (m rows). mode kEpOut: y = acc; kEpResid: y += acc (times mult).
template <int N, bool F16>
__global__ void __launch_bounds__(TC_THREADS, TcShape<N, F16>::CTAS)
    k_gemm_tc(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, DMat W,
              const float* xs, int m, int mode, float* y, int ldy, float resid_mult, int* status) {
  using T = TcShape<N, F16>;
  constexpr int CW = T::CW;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* a_st = base;
  uint8_t* b_st = a_st + TC_STAGES * A_STAGE;
  const int G = W.agroup, groups = W.k / G;
  // A stage holds 4 groups of 32 (Q8_0) or one of 128; as f16, 2 of 32.
  const int gshift = (G == 32) ? (F16 ? 1 : 2) : 0, gmask = (1 << gshift) - 1;
  // 128-value groups with a multiple of 4 of them: four consecutive stages
  // (one group each) share a TMEM buffer, as a Q8_0 stage's four groups do.
  const bool quad128 = G == 128 && groups % 4 == 0;
  constexpr int XP = N + 4;  // xs_s row pitch: conflict-free staging, 16-byte rows
  float* xs_s = (float*)(b_st + TC_STAGES * T::B_STAGE);  // [groups][XP]
  TcSmem* S = (TcSmem*)(xs_s + XP * groups);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TC_M, f0 = blockIdx.y * N;
  const int ktiles = W.k * (F16 ? 2 : 1) / TC_KT;
  volatile int* abort = &S->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
    }
    for (int b = 0; b < T::BUFS; ++b) {
      mbar_init(&S->tfull[b], 1);
      mbar_init(&S->tempty[b], 32 * TC_EPI_WARPS);
    }
    mbar_init(&S->drain, 1);
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S->tmem)),
                 "r"(T::TMEM_COLS)
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
        mbar_expect_tx(&S->full[s], A_STAGE + T::B_STAGE);
        tma_load_2d(a_st + s * A_STAGE, &amap, &S->full[s], kt * TC_KT, n0);
#pragma unroll
        for (int i = 0; i < N / TC_FBOX; ++i)
          tma_load_2d(b_st + s * T::B_STAGE + i * TC_FBOX * TC_KT, &bmap, &S->full[s], kt * TC_KT, f0 + i * TC_FBOX);
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
      for (int kt = 0; kt < ktiles; ++kt) {
        // Buffer use u: a stage (Q8_0, other 128-value layers) or four
        // stages (quad128), each group in its own N columns of the buffer.
        const int u = quad128 ? kt >> 2 : kt, slot = quad128 ? kt & 3 : 0;
        const int s = kt % TC_STAGES, b = u % T::BUFS;
        if (!mbar_wait(&S->full[s], (kt / TC_STAGES) & 1, abort)) break;
        // The buffer's accumulators, read back by the epilogue.
        if (slot == 0 && !mbar_wait(&S->tempty[b], (u / T::BUFS) & 1, abort)) break;
        fence_after();
#pragma unroll
        for (int j = 0; j < TC_KT / 32; ++j) {
          const uint64_t ad = smem_desc_sw128(a0 + s * A_STAGE + j * 32);
          const uint64_t bd = smem_desc_sw128(b0 + s * T::B_STAGE + j * 32);
          if (F16) {
            // K = 16 values a step: two steps a 32-value group.
            mma_f16(tmem + b * T::BUF_COLS + (j >> 1) * N, ad, bd, idesc_f16n(N), (uint32_t)(j & 1));
          } else {
            const int gi = slot + (j * 32) / G;  // the group within the buffer
            mma_i8(tmem + b * T::BUF_COLS + gi * N, ad, bd, idesc_i8(N), (j * 32) % G ? 1u : 0u);
          }
        }
        if (slot == 3 || !quad128) mma_commit(&S->tfull[b]);
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
    const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16) + half * CW;
    // Every buffer starts free.
    for (int b = 0; b < T::BUFS; ++b) mbar_arrive(&S->tempty[b]);
    // Weight scales in chunks of 8 groups, loaded 3 chunks ahead.
    const bool wvec = ws_vector_ok(W, groups);
    Ws8 wq[4];
#pragma unroll
    for (int c = 0; c < 3; ++c) wq[c] = load_ws8(W, row, live, c * 8, groups, wvec);
    // The frames' activation scales, [group][frame] (frames past m read as
    // 0), while the first stages load and multiply. A warp moves blocks of
    // 8 groups x 4 frames: 32-byte pieces of 4 xs rows, stored at pitch
    // XP (XP % 32 is 4 or 20) on 32 distinct banks; eight in flight per
    // thread.
    {
      const int gblocks = (groups + 7) / 8, tasks = gblocks * (N / 4) * 32;
      const int t0 = threadIdx.x - 64, nt = 32 * TC_EPI_WARPS;
      for (int i0 = t0; i0 < tasks; i0 += 8 * nt) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * nt, b = i >> 5, l = i & 31;
          const int g = (b % gblocks) * 8 + (l >> 2), f = (b / gblocks) * 4 + (l & 3);
          v[u] = (i < tasks && g < groups && f0 + f < m) ? __ldg(xs + (size_t)(f0 + f) * groups + g) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = i0 + u * nt, b = i >> 5, l = i & 31;
          const int g = (b % gblocks) * 8 + (l >> 2), f = (b / gblocks) * 4 + (l & 3);
          if (i < tasks && g < groups) xs_s[g * XP + f] = v[u];
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(32 * TC_EPI_WARPS) : "memory");
    }
    float2 acc[CW / 2];  // frames CW half + 2 i, + 1
#pragma unroll
    for (int i = 0; i < CW / 2; ++i) acc[i] = make_float2(0.0f, 0.0f);
    // Group g: stage g >> gshift, TMEM buffer stage % BUFS, columns
    // (g & gmask) * N.. of it.
    auto col = [&](int g) -> uint32_t {
      return tl + ((g >> gshift) % T::BUFS) * T::BUF_COLS + (g & gmask) * N;
    };
    auto stage_ready = [&](int st) -> bool {
      if (!mbar_wait(&S->tfull[st % T::BUFS], (st / T::BUFS) & 1, abort)) return false;
      fence_after();
      return true;
    };
    // The f32 chains of group g from its dots.
    auto fold = [&](int g, float w, const uint32_t (&rc)[CW]) {
      const float2 ws2 = make_float2(w, w);
      const float4* xg = (const float4*)(xs_s + g * XP + half * CW);
#pragma unroll
      for (int q = 0; q < CW / 4; ++q) {
        const float4 xv = xg[q];
        const float2 d01 = F16 ? make_float2(__uint_as_float(rc[4 * q]), __uint_as_float(rc[4 * q + 1]))
                               : dots_to_float2(rc[4 * q], rc[4 * q + 1]);
        const float2 d23 = F16 ? make_float2(__uint_as_float(rc[4 * q + 2]), __uint_as_float(rc[4 * q + 3]))
                               : dots_to_float2(rc[4 * q + 2], rc[4 * q + 3]);
        acc[2 * q] = fma2(d01, mul2(ws2, make_float2(xv.x, xv.y)), acc[2 * q]);
        acc[2 * q + 1] = fma2(d23, mul2(ws2, make_float2(xv.z, xv.w)), acc[2 * q + 1]);
      }
    };
    bool ok = true;
    if (G == 32 || quad128) {
      // Four groups a buffer (a Q8_0 stage, or four 128-value stages):
      // the four accumulators load GB at a time (one TMEM wait
      // per batch and one hand-off per stage), then fold in order.
      constexpr int GPS = T::GPS;  // groups a buffer: 4 (int8 stage or quad128) or 2 (f16 stage)
      constexpr int GB = (CW <= 8 ? 4 : 2) < GPS ? (CW <= 8 ? 4 : 2) : GPS;
      auto chunk = [&](int gc, int c) -> bool {
        wq[(c + 3) & 3] = load_ws8(W, row, live, gc + 24, groups, wvec);
#pragma unroll
        for (int h2 = 0; h2 < 8 / GPS; ++h2) {
          const int g0 = gc + GPS * h2, st = g0 / GPS;
          if (g0 >= groups) return true;
          if (!stage_ready(st)) return false;
          const uint32_t base = tl + (st % T::BUFS) * T::BUF_COLS;
#pragma unroll
          for (int b0 = 0; b0 < GPS; b0 += GB) {
            uint32_t rs[GB][CW];
#pragma unroll
            for (int gi = 0; gi < GB; ++gi) tmem_ld<CW>(base + (b0 + gi) * N, rs[gi]);
            tmem_wait_ld();
            if (b0 + GB == GPS) {
              fence_before();
              mbar_arrive(&S->tempty[st % T::BUFS]);
            }
#pragma unroll
            for (int gi = 0; gi < GB; ++gi) fold(g0 + b0 + gi, wq[c].get(W, GPS * h2 + b0 + gi), rs[gi]);
          }
        }
        return true;
      };
      for (int gc = 0; gc < groups && ok; gc += 32) {
        ok = chunk(gc, 0) && chunk(gc + 8, 1) && chunk(gc + 16, 2) && chunk(gc + 24, 3);
      }
    } else {
      // One group: the next group's accumulator loads from TMEM while this
      // group's chains run; the last group of a stage hands the stage's
      // buffer back.
      auto step = [&](int g, float w, const uint32_t (&rc)[CW], uint32_t (&rn)[CW]) -> bool {
        const bool more = g + 1 < groups, ends = ((g + 1) & gmask) == 0;
        if (more) {
          if (ends && !stage_ready((g + 1) >> gshift)) return false;
          tmem_ld<CW>(col(g + 1), rn);
        }
        fold(g, w, rc);
        tmem_wait_ld();
        if (ends) {
          fence_before();
          mbar_arrive(&S->tempty[(g >> gshift) % T::BUFS]);
        }
        return true;
      };
      uint32_t ra[CW], rb[CW];
      ok = stage_ready(0);
      if (ok) {
        tmem_ld<CW>(col(0), ra);
        tmem_wait_ld();
      }
      // Eight groups with the scales of chunk buffer `c`; the buffer three
      // chunks on starts loading first.
      auto chunk = [&](int gc, int c) -> bool {
        wq[(c + 3) & 3] = load_ws8(W, row, live, gc + 24, groups, wvec);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          if (gc + i >= groups) return true;
          if (!step(gc + i, wq[c].get(W, i), ra, rb)) return false;
          if (gc + i + 1 >= groups) return true;
          if (!step(gc + i + 1, wq[c].get(W, i + 1), rb, ra)) return false;
        }
        return true;
      };
      for (int gc = 0; gc < groups && ok; gc += 32) {
        ok = chunk(gc, 0) && chunk(gc + 8, 1) && chunk(gc + 16, 2) && chunk(gc + 24, 3);
      }
    }
    if (ok && live) {
#pragma unroll
      for (int j = 0; j < CW; ++j) {
        const int f = f0 + half * CW + j;
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T::TMEM_COLS) : "memory");
  }
  if (threadIdx.x == 0 && S->abort) atomicExch(status, 1);
}

// ------------------------------------------ prompt attention, f16 MMA ----
// The `"tc_attention": true` prompt attention: causal GQA attention of a tile of
// 128 query rows (128 / qpk consecutive positions of one stream, each with
// the qpk query heads of one kv head) over the stream's paged f16 keys and
// values, flash-style on the tensor cores:
//   S = Q K^T   tcgen05.mma kind::f16 (M 128 rows, N 128 keys, K 128 dims),
//               f32 in one of two TMEM buffers;
//   softmax     a thread a row: running max and sum, exp2, P rounded to f16
//               into shared memory (K-major, 128-byte swizzle), O rescaled
//               in TMEM when its row's max grows;
//   O += P V    tcgen05.mma kind::f16 (N 128 dims, K 128 keys), V read
//               MN-major straight from the cache's layout.
// Warp 0 loads key/value tiles by TMA (two stages, one 64-row box per cache
// page and 64-dimension half), warp 1 issues the MMAs, warps 2-5 run the
// softmax. The sums' order differs from the reference's (the tensor cores'
// order, per-tile softmax, f16 P), so this path is not bit-exact. Every wait
// is bounded in time and reports through the status word.
constexpr int FA_ROWS = 128;                 // query rows a CTA (TMEM lanes)
constexpr int FA_KEYS = 128;                 // keys a tile (two cache pages of 64)
constexpr int FA_THREADS = 64 + 128;
constexpr int FA_TILE = FA_KEYS * 256;       // bytes of a K or V tile (f16, 128 dims)
constexpr int FA_HALF = FA_KEYS * 128;       // one 64-dimension half of it
constexpr uint32_t FA_TMEM_COLS = 512;       // S0 | S1 | O (128 columns each)
constexpr int FA_PAD = 4096;                 // slack after the last tile (shared memory)

struct FaSmem {
  uint64_t full[2], empty[2], sfull[2], sfree[2], qfull, pfull, ofull, drain;
  uint32_t tmem;
  int abort;
};

static_assert(FA_ROWS == TC_M, "the attention MMA's M is the products' M");
__host__ __device__ constexpr uint32_t idesc_f16(bool b_mn_major) { return idesc_f16n(FA_KEYS, b_mn_major); }
// MN-major operand with the 128-byte swizzle: 64-element atoms along MN
// (the leading offset between them), 8-row groups along K 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t addr, uint32_t mn_atom_bytes) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((mn_atom_bytes >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Row r (128 values, f32 -> f16) into a K-major, 128-byte-swizzled tile of
// 128 rows: values 64h.. of the row in half h, 16-byte chunk c of a row at
// chunk c ^ (r % 8).
__device__ __forceinline__ void put_row_f16(uint8_t* tile, int r, const float (&v)[128]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half2 p = __floats2half2_rn(v[64 * h + 8 * c + 2 * i], v[64 * h + 8 * c + 2 * i + 1]);
        w[i] = *(const uint32_t*)&p;
      }
      *(uint4*)(tile + h * FA_HALF + r * 128 + ((c ^ (r & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__global__ void __launch_bounds__(FA_THREADS, 1)
    k_attention_tc(const __grid_constant__ CUtensorMap kvmap, const float* qkv, const int2* tiles, DConfig cfg,
                   DCache cache, const int* row_stream, const int* row_pos, int layer, float* att, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* q_s = base;                 // [2 halves][128 rows][128 B]
  uint8_t* p_s = q_s + 2 * FA_HALF;    // the same layout for P
  uint8_t* kv_s = p_s + 2 * FA_HALF;   // [2 stages][K tile | V tile]
  FaSmem* S = (FaSmem*)(kv_s + 2 * 2 * FA_TILE + FA_PAD);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qpk = cfg.heads / cfg.kv_heads, kvh = blockIdx.y;
  const int2 tile = tiles[blockIdx.x];
  const int r0 = tile.x, R = tile.y;
  const int stream = row_stream[r0], p0 = row_pos[r0];
  const int nt = (p0 + R - 1) / FA_KEYS + 1;  // key tiles: keys [0, last position]
  volatile int* abort = &S->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
      mbar_init(&S->sfull[s], 1);
      mbar_init(&S->sfree[s], 128);
    }
    mbar_init(&S->qfull, 128);
    mbar_init(&S->pfull, 128);
    mbar_init(&S->ofull, 1);
    mbar_init(&S->drain, 1);
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S->tmem)),
                 "r"(FA_TMEM_COLS)
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
      for (int j = 0; j < nt; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&S->empty[s], ((j >> 1) & 1) ^ 1, abort)) break;
        mbar_expect_tx(&S->full[s], 2 * FA_TILE);
        uint8_t* kt = kv_s + s * 2 * FA_TILE;
        for (int pp = 0; pp < 2; ++pp) {
          const int key = j * FA_KEYS + pp * 64, pgi = key / cache.page_tokens, tok = key % cache.page_tokens;
          int page = pgi < cache.pages_per_stream ? cache.page_table[(size_t)stream * cache.pages_per_stream + pgi] : 0;
          if (page < 0) page = 0;
          for (int which = 0; which < 2; ++which) {
            const int row = (((page * cfg.layers + layer) * 2 + which) * cfg.kv_heads + kvh) * cache.page_tokens + tok;
            for (int h = 0; h < 2; ++h)
              tma_load_2d(kt + which * FA_TILE + h * FA_HALF + pp * 64 * 128, &kvmap, &S->full[s], h * 128, row);
          }
        }
        issued = j + 1;
      }
      if (*abort) {
        for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j) {
          long long t0 = now_ns();
          while (!mbar_test(&S->full[j & 1], (j >> 1) & 1) && now_ns() - t0 < TC_WAIT_NS) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t qa = smem_u32(q_s), pa = smem_u32(p_s), kva = smem_u32(kv_s);
      auto pv = [&](int j) -> bool {
        if (!mbar_wait(&S->pfull, j & 1, abort)) return false;
        fence_after();
        const uint32_t va = kva + (j & 1) * 2 * FA_TILE + FA_TILE;
#pragma unroll
        for (int i = 0; i < FA_KEYS / 16; ++i)
          mma_f16(tmem + 256, smem_desc_sw128(pa + (i >> 2) * FA_HALF + (i & 3) * 32),
                  smem_desc_sw128_mn(va + i * 2048, FA_HALF), idesc_f16(true), (j > 0 || i > 0) ? 1u : 0u);
        mma_commit(&S->ofull);
        mma_commit(&S->empty[j & 1]);
        return true;
      };
      bool ok = mbar_wait(&S->qfull, 0, abort);
      for (int j = 0; j < nt && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&S->full[s], (j >> 1) & 1, abort) || !mbar_wait(&S->sfree[s], ((j >> 1) & 1) ^ 1, abort)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t ka = kva + s * 2 * FA_TILE;
#pragma unroll
        for (int i = 0; i < 128 / 16; ++i)
          mma_f16(tmem + s * 128, smem_desc_sw128(qa + (i >> 2) * FA_HALF + (i & 3) * 32),
                  smem_desc_sw128(ka + (i >> 2) * FA_HALF + (i & 3) * 32), idesc_f16(false), i > 0 ? 1u : 0u);
        mma_commit(&S->sfull[s]);
        if (j > 0) ok = pv(j - 1);
      }
      if (ok) pv(nt - 1);
      mma_commit(&S->drain);
      long long t0 = now_ns();
      while (!mbar_test(&S->drain, 0) && now_ns() - t0 < TC_WAIT_NS) {
      }
    }
  } else {
    // Softmax: thread q is query row q (TMEM lane q).
    // A warp reaches the TMEM lanes of its quarter (warp % 4) only.
    const int q = (warp & 3) * 32 + lane, i = q / qpk, h = q % qpk;
    const bool valid = i < R;
    const int pos = valid ? row_pos[r0 + i] : p0;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int qd = cfg.heads * 128, stride = qd + 2 * cfg.kv_heads * 128;
    {
      float v[128];
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
      const float* src = qkv + (size_t)(r0 + (valid ? i : 0)) * stride + (kvh * qpk + h) * 128;
#pragma unroll
      for (int d = 0; d < 128; d += 4) {
        const float4 x = valid ? *(const float4*)(src + d) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        v[d] = __fmul_rn(x.x, scale);
        v[d + 1] = __fmul_rn(x.y, scale);
        v[d + 2] = __fmul_rn(x.z, scale);
        v[d + 3] = __fmul_rn(x.w, scale);
      }
      put_row_f16(q_s, q, v);
    }
    fence_async_smem();
    mbar_arrive(&S->qfull);
    const float log2e = 1.4426950408889634f;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nt && ok; ++j) {
      const int s = j & 1;
      // Warp-uniform waits: the TMEM loads and stores below are warp-wide.
      if (!__all_sync(0xffffffffu, mbar_wait(&S->sfull[s], (j >> 1) & 1, abort))) {
        ok = false;
        break;
      }
      fence_after();
      float v[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld<32>(lane_base + s * 128 + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 32; ++k) v[32 * c + k] = __uint_as_float(r[k]);
      }
      fence_before();
      mbar_arrive(&S->sfree[s]);
      // Causal mask, then the tile's max.
      float mt = -INFINITY;
#pragma unroll
      for (int k = 0; k < 128; ++k) {
        if (j * FA_KEYS + k > pos) v[k] = -INFINITY;
        mt = fmaxf(mt, v[k]);
      }
      const float mn = fmaxf(m, mt);
      const float alpha = exp2f((m - mn) * log2e);
      float sum = 0.0f;
#pragma unroll
      for (int k = 0; k < 128; ++k) {
        v[k] = exp2f((v[k] - mn) * log2e);
        sum += v[k];
      }
      l = l * alpha + sum;
      m = mn;
      if (j > 0) {
        // O holds tiles 0..j-1 once PV j-1 is done; it then scales by alpha.
        if (!__all_sync(0xffffffffu, mbar_wait(&S->ofull, (j - 1) & 1, abort))) {
          ok = false;
          break;
        }
        fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld<32>(lane_base + 256 + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) r[k] = __float_as_uint(__uint_as_float(r[k]) * alpha);
            tmem_st32(lane_base + 256 + c * 32, r);
          }
          tmem_wait_st();
        }
      }
      put_row_f16(p_s, q, v);
      fence_async_smem();
      fence_before();
      mbar_arrive(&S->pfull);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(&S->ofull, (nt - 1) & 1, abort))) {
      fence_after();
      const float inv = 1.0f / l;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld<32>(lane_base + 256 + c * 32, r);
        tmem_wait_ld();
        if (valid) {
          float* dst = att + (size_t)(r0 + i) * qd + (kvh * qpk + h) * 128 + c * 32;
#pragma unroll
          for (int k = 0; k < 32; k += 4)
            *(float4*)(dst + k) = make_float4(__uint_as_float(r[k]) * inv, __uint_as_float(r[k + 1]) * inv,
                                              __uint_as_float(r[k + 2]) * inv, __uint_as_float(r[k + 3]) * inv);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(FA_TMEM_COLS) : "memory");
  }
  if (threadIdx.x == 0 && S->abort) atomicExch(status, 1);
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

size_t tc_smem_bytes(const DMat& W, int n) {
  size_t groups = W.k / W.agroup;
  return 1024 + (size_t)TC_STAGES * (A_STAGE + (size_t)n * TC_KT) + (size_t)(n + 4) * groups * 4 + sizeof(TcSmem);
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

int tc_frames() { return TC_NMAX; }

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
  return make_tc_map(out, xq, rows_cap, k, TC_FBOX);
}

// The frame tile (16, 32 or 64 frames a CTA) for an n x k product of m
// frames: the fewest waves of CTAs, each wave weighted by the time a CTA
// of that tile takes per stage relative to a 64-frame CTA (measured).
int tc_frame_tile(int n, int m, int sms) {
  const int rows = (n + TC_M - 1) / TC_M;
  const int tiles[3] = {64, 32, 16}, per_sm[3] = {1, 2, 2};
  const double weight[3] = {1.0, 0.95, 0.6};
  int best = 64;
  double best_cost = 1e30;
  for (int i = 0; i < 3; ++i) {
    const long ctas = (long)rows * ((m + tiles[i] - 1) / tiles[i]);
    const long waves = (ctas + (long)sms * per_sm[i] - 1) / ((long)sms * per_sm[i]);
    const double cost = waves * weight[i];
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = tiles[i];
    }
  }
  return best;
}

// The shared-memory limit of every frame tile of k_gemm_tc, set once per
// device on its first tensor-core product.
static cudaError_t configure_gemm_tc(int dev) {
  static DeviceOnce once;
  return once.run(dev, [] {
    const void* fns[] = {(const void*)k_gemm_tc<16, false>, (const void*)k_gemm_tc<32, false>,
                         (const void*)k_gemm_tc<64, false>, (const void*)k_gemm_tc<16, true>,
                         (const void*)k_gemm_tc<32, true>, (const void*)k_gemm_tc<64, true>};
    for (const void* f : fns) {
      cudaError_t r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      if (r != cudaSuccess) return r;
    }
    return cudaSuccess;
  });
}

template <int N, bool F16>
cudaError_t launch_tc_n(const TcMap& amap, const TcMap& bmap, const DMat& W, const float* xs, int m, int mode,
                        float* y, int ldy, float resid_mult, int* status, cudaStream_t s, int dev) {
  size_t smem = tc_smem_bytes(W, N);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = configure_gemm_tc(dev);
  if (e != cudaSuccess) return e;
  dim3 grid((W.n + TC_M - 1) / TC_M, (m + N - 1) / N);
  k_gemm_tc<N, F16><<<grid, TC_THREADS, smem, s>>>(*(const CUtensorMap*)&amap, *(const CUtensorMap*)&bmap, W, xs, m,
                                                    mode, y, ldy, resid_mult, status);
  return cudaGetLastError();
}

// int8 codes as f16 (exact), for the f16 form of the products.
__global__ void k_codes_f16(const int8_t* in, size_t n, __half* out) {
  for (size_t i = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) * 8; i < n; i += (size_t)gridDim.x * blockDim.x * 8) {
    if (i + 8 <= n) {
      const int2 c = *(const int2*)(in + i);
      const int8_t* b = (const int8_t*)&c;
      __half2 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __halves2half2(__int2half_rn(b[2 * j]), __int2half_rn(b[2 * j + 1]));
      *(uint4*)(out + i) = *(const uint4*)h;
    } else {
      for (size_t j = i; j < n; ++j) out[j] = __int2half_rn(in[j]);
    }
  }
}

cudaError_t launch_codes_f16(const int8_t* in, size_t n, void* out, cudaStream_t s) {
  if (((uintptr_t)in & 7) || ((uintptr_t)out & 15)) return cudaErrorInvalidValue;
  const size_t threads = (n + 7) / 8;
  const int blocks = (int)std::min<size_t>((threads + 255) / 256, 148 * 16);
  k_codes_f16<<<std::max(blocks, 1), 256, 0, s>>>(in, n, (__half*)out);
  return cudaGetLastError();
}

// f16 codes of a [rows][k] matrix as a 2-D byte view (2k bytes a row) for
// the f16 products: boxes of 64 values (128 bytes) x box_rows.
cudaError_t make_tc_map_f16(TcMap* out, const void* codes16, size_t rows, size_t k, int box_rows) {
  return make_tc_map(out, codes16, rows, 2 * k, box_rows);
}

cudaError_t launch_gemm_tc(const TcMap& amap, const TcMap& bmap, const DMat& W, const float* xs, int m, int mode,
                           float* y, int ldy, float resid_mult, int* status, cudaStream_t s, bool f16) {
  if (W.k % TC_KT || (W.agroup != 32 && W.agroup != 128) || m <= 0) return cudaErrorInvalidValue;
  if (f16 && W.agroup != 32) return cudaErrorInvalidValue;
  int dev = 0;
  cudaGetDevice(&dev);
  // TRIT_TC_FRAMES=16, 32 or 64 fixes the frame tile (tests, tuning).
  static const int forced = [] {
    const char* e = getenv("TRIT_TC_FRAMES");
    const int v = e ? atoi(e) : 0;
    return (v == 16 || v == 32 || v == 64) ? v : 0;
  }();
  const int tile = forced ? forced : tc_frame_tile(W.n, m, current_sm_count());
  if (f16) {
    if (tile == 16) return launch_tc_n<16, true>(amap, bmap, W, xs, m, mode, y, ldy, resid_mult, status, s, dev);
    if (tile == 32) return launch_tc_n<32, true>(amap, bmap, W, xs, m, mode, y, ldy, resid_mult, status, s, dev);
    return launch_tc_n<64, true>(amap, bmap, W, xs, m, mode, y, ldy, resid_mult, status, s, dev);
  }
  if (tile == 16) return launch_tc_n<16, false>(amap, bmap, W, xs, m, mode, y, ldy, resid_mult, status, s, dev);
  if (tile == 32) return launch_tc_n<32, false>(amap, bmap, W, xs, m, mode, y, ldy, resid_mult, status, s, dev);
  return launch_tc_n<64, false>(amap, bmap, W, xs, m, mode, y, ldy, resid_mult, status, s, dev);
}

bool attention_tc_supported(const DConfig& cfg, const DCache& cache) {
  const int qpk = cfg.heads / cfg.kv_heads;
  return cache.f16 && cfg.hd == 128 && cache.page_tokens % 64 == 0 && (qpk == 1 || qpk == 2 || qpk == 4 || qpk == 8);
}

int attention_tc_rows(const DConfig& cfg) { return FA_ROWS / (cfg.heads / cfg.kv_heads); }

// The key/value pool as a 2-D byte view for TMA: rows of 256 bytes (one
// key or value, 128 f16), boxes of 64 rows x 128 bytes (one cache page's
// rows, one half of the dimensions), 128-byte swizzle.
cudaError_t make_kv_map(TcMap* out, const void* pool, size_t rows) { return make_tc_map(out, pool, rows, 256, 64); }

cudaError_t launch_attention_tc(const TcMap& kvmap, const float* qkv, const int2* tiles, int ntiles,
                                const DConfig& cfg, const DCache& cache, const int* row_stream, const int* row_pos,
                                int layer, float* att, int* status, cudaStream_t s) {
  if (!attention_tc_supported(cfg, cache) || ntiles <= 0) return cudaErrorInvalidValue;
  const size_t smem = 1024 + 4 * (size_t)FA_HALF + 4 * (size_t)FA_TILE + FA_PAD + sizeof(FaSmem);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static DeviceOnce once;
  e = once.run(dev, [smem] {
    return cudaFuncSetAttribute(k_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (e != cudaSuccess) return e;
  k_attention_tc<<<dim3(ntiles, cfg.kv_heads), FA_THREADS, smem, s>>>(*(const CUtensorMap*)&kvmap, qkv, tiles, cfg,
                                                                       cache, row_stream, row_pos, layer, att, status);
  return cudaGetLastError();
}

cudaError_t launch_expand_ternary(const DMat& W, int8_t* out, cudaStream_t s) {
  if (W.kind != kTernary || W.k % 16) return cudaErrorInvalidValue;
  k_expand_ternary<<<148 * 8, 256, 0, s>>>((const uint32_t*)W.codes, (size_t)W.n, W.k, out);
  return cudaGetLastError();
}


}  // namespace trit
