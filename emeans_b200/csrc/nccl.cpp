// Multi-GPU groups: one engine per GPU joins an NCCL communicator, and the
// training loop splits each batch's top-1 across the ranks and all-gathers
// the labels and scores (the one exchange step of a data-parallel step).
//
// NCCL is loaded at run time, only when a group is formed: a process that
// already holds libnccl.so.2 (a PyTorch process does) keeps that copy, so
// the library never brings a second NCCL into it, and single-GPU use needs
// no NCCL at all.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "engine.h"

namespace eb {
namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  static std::string failure;
  std::call_once(once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) {
      failure = std::string("NCCL is not available: ") + dlerror();
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(lib, "ncclGetUniqueId"));
    api.init_rank = reinterpret_cast<decltype(api.init_rank)>(dlsym(lib, "ncclCommInitRank"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(lib, "ncclAllGather"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(lib, "ncclCommDestroy"));
    api.error_string =
        reinterpret_cast<decltype(api.error_string)>(dlsym(lib, "ncclGetErrorString"));
    if (!api.get_unique_id || !api.init_rank || !api.all_gather || !api.destroy ||
        !api.error_string)
      failure = "NCCL library lacks an entry point this engine needs";
  });
  if (!failure.empty()) throw Error(EB_ERROR, failure);
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw Error(EB_ERROR, std::string(what) + ": " + nccl().error_string(r));
}

}  // namespace

void group_allgather(eb_engine* e, uint32_t* buf, size_t words) {
  ensure(e->comm != nullptr, "engine is not in a group");
  nccl_check(nccl().all_gather(buf + (size_t)e->rank * words, buf, words, ncclUint32,
                               static_cast<ncclComm_t>(e->comm), e->stream),
             "ncclAllGather");
}

void group_leave(eb_engine* e) {
  if (e->comm) {
    nccl().destroy(static_cast<ncclComm_t>(e->comm));
    e->comm = nullptr;
  }
  e->rank = 0;
  e->world = 1;
}

}  // namespace eb

extern "C" int eb_group_unique_id(unsigned char* id) {
  try {
    eb::ensure(id != nullptr, "id is null");
    static_assert(sizeof(ncclUniqueId) == EB_GROUP_ID_BYTES, "NCCL id size");
    ncclUniqueId u;
    eb::nccl_check(eb::nccl().get_unique_id(&u), "ncclGetUniqueId");
    std::memcpy(id, &u, sizeof u);
    eb::set_last_error("");
    return EB_OK;
  } catch (const eb::Error& err) {
    eb::set_last_error(err.what());
    return err.code;
  }
}

extern "C" int eb_engine_join(eb_engine* e, int rank, int world, const unsigned char* id) {
  try {
    eb::ensure(e != nullptr && id != nullptr, "engine and id are required");
    eb::ensure(world >= 1 && rank >= 0 && rank < world, "rank must be in 0 .. world - 1");
    eb::ensure(e->comm == nullptr, "engine is already in a group");
    if (world > 1) {
      int prev = -1;
      cudaGetDevice(&prev);
      if (prev != e->device) EB_CUDA(cudaSetDevice(e->device));
      ncclUniqueId u;
      std::memcpy(&u, id, sizeof u);
      ncclComm_t comm = nullptr;
      const ncclResult_t r = eb::nccl().init_rank(&comm, world, u, rank);
      if (prev >= 0 && prev != e->device) cudaSetDevice(prev);
      eb::nccl_check(r, "ncclCommInitRank");
      e->comm = comm;
    }
    e->rank = rank;
    e->world = world;
    eb::set_last_error("");
    return EB_OK;
  } catch (const eb::Error& err) {
    eb::set_last_error(err.what());
    return err.code;
  }
}

extern "C" int eb_set_group_shard(eb_engine* e, int mode) {
  if (!e || mode < 0 || mode > 3) {
    eb::set_last_error("engine required; mode must be 0, 1, 2 or 3");
    return EB_INVALID_ARGUMENT;
  }
  e->group_shard = mode;
  return EB_OK;
}

extern "C" int eb_group_allgather(eb_engine* e, eb_buf* b, size_t words_per_rank) {
  try {
    eb::ensure(e != nullptr && b != nullptr, "engine and buffer are required");
    eb::ensure(b->len / (size_t)e->world >= words_per_rank,
               "the buffer holds fewer than world x words_per_rank elements");
    if (e->world > 1 && words_per_rank > 0) {
      int prev = -1;
      cudaGetDevice(&prev);
      if (prev != e->device) EB_CUDA(cudaSetDevice(e->device));
      try {
        eb::group_allgather(e, static_cast<uint32_t*>(b->ptr), words_per_rank);
      } catch (...) {
        if (prev >= 0 && prev != e->device) cudaSetDevice(prev);
        throw;
      }
      if (prev >= 0 && prev != e->device) cudaSetDevice(prev);
    }
    eb::set_last_error("");
    return EB_OK;
  } catch (const eb::Error& err) {
    eb::set_last_error(err.what());
    return err.code;
  }
}

extern "C" int eb_engine_group(eb_engine* e, int* rank, int* world) {
  if (!e || !rank || !world) {
    eb::set_last_error("engine, rank and world are required");
    return EB_INVALID_ARGUMENT;
  }
  *rank = e->rank;
  *world = e->world;
  return EB_OK;
}
