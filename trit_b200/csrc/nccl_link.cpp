#include "nccl_link.h"

#include <dlfcn.h>

#include <mutex>
#include <string>

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
    bind(api.AllReduce, "ncclAllReduce");
    bind(api.GetErrorString, "ncclGetErrorString");
  });
  if (!error.empty()) throw Error(error);
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw Error(std::string("NCCL: ") + nccl().GetErrorString(r) + " (" + what + ")");
}

}  // namespace trit
