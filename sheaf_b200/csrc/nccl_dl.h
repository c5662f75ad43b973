// NCCL entry points resolved at run time (dlopen), so that the library loads on
// hosts without NCCL and binds to whichever libnccl.so.2 the process already
// uses (e.g. the one PyTorch ships).
#pragma once
#include <nccl.h>

#include <string>

namespace sb {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclCommAbort) comm_abort = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
  std::string error;
};

// Loads NCCL once per process; returns the table (check .ok).
const NcclApi& nccl_api();

}  // namespace sb
