// Helpers of the persistent decode kernels (decode.cu, decode_fast.cu):
// the 64-bit {data, tag} words through which one block hands values to
// others (the low-latency protocol of NCCL's LL transfers: data and its
// "ready" signal arrive in one load), timers and cp.async forms.
#pragma once

#include <cstdint>

namespace trit {

// Polls of one wait before it gives up (~seconds): the kernel then sets a
// status word and returns instead of hanging.
constexpr long long kSpinLimit = 1ll << 22;

__device__ __forceinline__ int ld_volatile(const int* p) { return *(const volatile int*)p; }

__device__ __forceinline__ long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return (long long)t;
}

__host__ __device__ __forceinline__ int split_at(int n, int part, int parts) {
  return (int)((long long)n * part / parts);
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ll_put(unsigned long long* p, uint32_t data, uint32_t tag) {
  unsigned long long v = ((unsigned long long)tag << 32) | data;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ll_get(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace trit
