#include "nccl_dl.h"

#include <dlfcn.h>

#include <mutex>

namespace sb {

const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, []() {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.error = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
#define SB_SYM(field, name)                                                   \
  api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name));          \
  if (!api.field) { api.error = std::string("NCCL symbol missing: ") + name; return; }
    SB_SYM(get_unique_id, "ncclGetUniqueId");
    SB_SYM(init_rank_config, "ncclCommInitRankConfig");
    SB_SYM(all_reduce, "ncclAllReduce");
    SB_SYM(group_start, "ncclGroupStart");
    SB_SYM(group_end, "ncclGroupEnd");
    SB_SYM(comm_abort, "ncclCommAbort");
    SB_SYM(comm_destroy, "ncclCommDestroy");
    SB_SYM(async_error, "ncclCommGetAsyncError");
    SB_SYM(error_string, "ncclGetErrorString");
#undef SB_SYM
    api.ok = true;
  });
  return api;
}

}  // namespace sb
