#include "nccl_link.h"

#include <dlfcn.h>
#include <stdlib.h>

#include <chrono>
#include <condition_variable>
#include <memory>
#include <mutex>
#include <string>
#include <thread>

#include <cuda_runtime.h>

#include "host.h"

namespace trit {

const Nccl& nccl() {
  static Nccl api;
  static std::string error;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      error = std::string("NCCL is needed for tensor parallelism: ") + dlerror();
      return;
    }
    auto bind = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn && error.empty()) error = std::string("libnccl.so.2 has no ") + name;
    };
    bind(api.GetUniqueId, "ncclGetUniqueId");
    bind(api.CommInitRank, "ncclCommInitRank");
    bind(api.CommDestroy, "ncclCommDestroy");
    bind(api.CommAbort, "ncclCommAbort");
    bind(api.CommGetAsyncError, "ncclCommGetAsyncError");
    bind(api.AllReduce, "ncclAllReduce");
    bind(api.GetErrorString, "ncclGetErrorString");
  });
  if (!error.empty()) throw Error(error);
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw Error(std::string("NCCL: ") + nccl().GetErrorString(r) + " (" + what + ")");
}

ncclComm_t nccl_join(const ncclUniqueId& id, int size, int rank, int device, double seconds) {
  // Unless the caller chose otherwise: connect every channel while joining
  // (a lazy connect would block the first collective's host call on a rank
  // that never makes it, out of reach of the bounded waits), and no NVLink
  // SHARP multicast (a rank that dies while bound to a multicast object can
  // fault the other ranks' GPUs; the all-reduces here are small).
  setenv("NCCL_RUNTIME_CONNECT", "0", 0);
  setenv("NCCL_NVLS_ENABLE", "0", 0);
  const Nccl& api = nccl();
  struct State {
    std::mutex m;
    std::condition_variable cv;
    bool done = false;
    ncclResult_t r = ncclSuccess;
    ncclComm_t comm = nullptr;
  };
  auto st = std::make_shared<State>();
  std::thread([st, id, size, rank, device, &api] {
    cudaSetDevice(device);
    ncclComm_t c = nullptr;
    ncclResult_t r = api.CommInitRank(&c, size, id, rank);
    std::lock_guard<std::mutex> g(st->m);
    st->r = r;
    st->comm = c;
    st->done = true;
    st->cv.notify_all();
  }).detach();
  std::unique_lock<std::mutex> g(st->m);
  if (!st->cv.wait_for(g, std::chrono::duration<double>(seconds), [&] { return st->done; }))
    throw Error("tensor parallelism: the " + std::to_string(size) + " ranks did not join within " +
                std::to_string((int)seconds) + " s (a rank failed, or was never started)");
  nccl_check(st->r, "communicator");
  return st->comm;
}

}  // namespace trit
