// A Q8_0 dense product for callers that cannot allocate device memory.
//
// Some hosts of this library may not call cudaMalloc at the point where
// they run a product: code that runs inside a CUDA graph being captured by
// someone else, real-time audio threads that must not take the driver's
// allocation locks, or embedders whose device memory is all handed out by
// their own pool. trit_dense_q8_0_forward_static runs the same W8A8 product
// as trit_dense_forward_device, but its one piece of scratch memory (the
// int8 activations and their scales) lives in the file-scope device array
// below, which every GPU that loads the library holds until the process
// exits. Nothing is allocated per call.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/trit_cuda.h"
#include "engine.h"
#include "kernels.h"

namespace {

// 1 MiB: rows * k activation codes plus rows * k / 32 scales must fit.
constexpr size_t kStaticScratchBytes = 1u << 20;
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// The device address of g_static_scratch, found once per device with that
// device current. Host code must not pass the symbol itself to a kernel:
// on the host it names a stand-in, not device memory.
std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

void* scratch_address(int device) {
  if (device < 0 || device >= 64) throw trit::Error("device index out of range for the static scratch");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) throw trit::Error(std::string("cudaGetSymbolAddress of the static scratch: ") + cudaGetErrorString(e));
    g_scratch_addr[device] = p;
  }
  return g_scratch_addr[device];
}

}  // namespace

extern "C" int trit_dense_q8_0_forward_static(const void* codes, const void* scales, size_t n, size_t k, const float* x,
                                              size_t rows, float* out, void* cuda_stream) {
  try {
    trit::set_last_error("");
    if (!codes || !scales || !x || !out) throw trit::Error("a pointer argument is NULL");
    // The W8A8 GEMV (k_gemv_slots) takes rows of whole 128-value chunks.
    if (k == 0 || k % 128 || k > 8192) throw trit::Error("k must be a multiple of 128 from 128 to 8192");
    if (n == 0 || n % 32) throw trit::Error("n must be a positive multiple of 32");
    if (rows == 0) return 0;
    const size_t codes_bytes = (rows * k + 255) / 256 * 256;
    const size_t need = codes_bytes + rows * (k / 32) * sizeof(float);
    if (rows > kStaticScratchBytes || need > kStaticScratchBytes)
      throw trit::Error("rows x k is too large for the static scratch: rows * k * 9 / 8 must stay within 1 MiB (" +
                        std::to_string(rows) + " x " + std::to_string(k) + " asks " + std::to_string(need) + " bytes)");
    int device = 0;
    TRIT_CUDA(cudaGetDevice(&device));
    unsigned char* base = (unsigned char*)scratch_address(device);
    int8_t* xq = (int8_t*)base;
    float* xs = (float*)(base + codes_bytes);
    trit::DMat W;
    W.kind = trit::kQ8_0;
    W.n = (int)n;
    W.k = (int)k;
    W.agroup = 32;
    W.half = 1;
    W.codes = codes;
    W.scales = scales;
    cudaStream_t s = (cudaStream_t)cuda_stream;
    TRIT_CUDA(trit::launch_norm_quant(x, (int)rows, (int)k, nullptr, 0.0f, 32, 1, xq, xs, s));
    TRIT_CUDA(trit::launch_gemv(W, xq, xs, (int)rows, trit::kEpOut, out, (int)n, 1.0f, s));
    return 0;
  } catch (const std::exception& e) {
    trit::set_last_error(e.what());
    return -1;
  }
}
