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

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

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

// The group's symmetric exchange region: on every rank one cudaMalloc of
// kPxFlagWords flag words and then the data, mapped on every other rank
// through CUDA IPC, so that a kernel can store into any rank's copy over
// NVLink (ops.cu's k_px_allgather).
struct PeerExchange {
  uint32_t* base = nullptr;       // this rank's region
  size_t words = 0;               // its data words
  std::vector<uint32_t*> peers;   // every rank's region as mapped here (own at rank)
  uint32_t** peers_d = nullptr;   // the same on the device
  uint32_t epoch = 0;             // calls so far (the flags' values)
};

namespace {

// The ranks' words w (one per rank) all-gathered; blocking.
std::vector<uint32_t> allgather_words(eb_engine* e, uint32_t w) {
  uint32_t* d = nullptr;
  EB_CUDA(cudaMalloc(&d, (size_t)e->world * 4));
  std::vector<uint32_t> all(e->world);
  try {
    EB_CUDA(cudaMemcpy(d + e->rank, &w, 4, cudaMemcpyHostToDevice));
    nccl_check(nccl().all_gather(d + e->rank, d, 1, ncclUint32, static_cast<ncclComm_t>(e->comm),
                                 e->stream),
               "ncclAllGather");
    EB_CUDA(cudaStreamSynchronize(e->stream));
    EB_CUDA(cudaMemcpy(all.data(), d, (size_t)e->world * 4, cudaMemcpyDeviceToHost));
  } catch (...) {
    cudaFree(d);
    throw;
  }
  cudaFree(d);
  return all;
}

// Closes and frees the region. Collective: every rank's stream has finished
// its calls and a round over the group has passed before any region goes,
// so no peer still stores into it.
void px_free(eb_engine* e) {
  PeerExchange* px = e->px;
  if (!px) return;
  e->px = nullptr;
  cudaStreamSynchronize(e->stream);
  try {
    allgather_words(e, 1);
  } catch (...) {
  }
  for (int q = 0; q < (int)px->peers.size(); q++)
    if (q != e->rank && px->peers[q]) cudaIpcCloseMemHandle(px->peers[q]);
  if (px->peers_d) cudaFree(px->peers_d);
  if (px->base) cudaFree(px->base);
  delete px;
}

// Exports this rank's region, maps every peer's and reports whether every
// rank mapped all of them (two rounds over the group; `why` says what failed
// here). Everything it opened or allocated is recorded in px.
bool px_setup(eb_engine* e, PeerExchange* px, size_t words, std::string& why) {
  px->words = words;
  px->peers.assign(e->world, nullptr);
  const size_t bytes = (kPxFlagWords + words) * 4;
  cudaIpcMemHandle_t h{};
  cudaError_t st = cudaMalloc(&px->base, bytes);
  if (st == cudaSuccess) st = cudaMemsetAsync(px->base, 0, bytes, e->stream);
  if (st == cudaSuccess) st = cudaStreamSynchronize(e->stream);
  if (st == cudaSuccess) st = cudaIpcGetMemHandle(&h, px->base);
  if (st != cudaSuccess) {
    why = std::string("exporting the region: ") + cudaGetErrorString(st);
    cudaGetLastError();
  }
  // Round 1: every rank's handle and whether it has one (32 words each).
  constexpr size_t kRec = 32;
  static_assert(sizeof(cudaIpcMemHandle_t) <= (kRec - 1) * 4, "IPC handle size");
  std::vector<uint32_t> rec(kRec, 0);
  std::memcpy(rec.data(), &h, sizeof h);
  rec[kRec - 1] = st == cudaSuccess ? 1u : 0u;
  uint32_t* d = nullptr;
  EB_CUDA(cudaMalloc(&d, kRec * 4 * (size_t)e->world));
  std::vector<uint32_t> all(kRec * (size_t)e->world);
  try {
    EB_CUDA(cudaMemcpy(d + kRec * (size_t)e->rank, rec.data(), kRec * 4, cudaMemcpyHostToDevice));
    nccl_check(nccl().all_gather(d + kRec * (size_t)e->rank, d, kRec, ncclUint32,
                                 static_cast<ncclComm_t>(e->comm), e->stream),
               "ncclAllGather");
    EB_CUDA(cudaStreamSynchronize(e->stream));
    EB_CUDA(cudaMemcpy(all.data(), d, all.size() * 4, cudaMemcpyDeviceToHost));
  } catch (...) {
    cudaFree(d);
    throw;
  }
  cudaFree(d);
  bool ok = true;
  for (int q = 0; q < e->world; q++) ok = ok && all[kRec * (size_t)q + kRec - 1] == 1u;
  if (!ok && why.empty()) why = "a peer could not export its region";
  // Round 2: whether every peer's region could be mapped here.
  uint32_t mapped = ok ? 1u : 0u;
  if (ok) {
    for (int q = 0; q < e->world; q++) {
      if (q == e->rank) {
        px->peers[q] = px->base;
        continue;
      }
      cudaIpcMemHandle_t hq;
      std::memcpy(&hq, all.data() + kRec * (size_t)q, sizeof hq);
      void* p = nullptr;
      const cudaError_t so = cudaIpcOpenMemHandle(&p, hq, cudaIpcMemLazyEnablePeerAccess);
      if (so != cudaSuccess) {
        why = "mapping rank " + std::to_string(q) + "'s region: " + cudaGetErrorString(so);
        cudaGetLastError();
        mapped = 0;
        break;
      }
      px->peers[q] = static_cast<uint32_t*>(p);
    }
  }
  if (mapped && cudaMalloc(&px->peers_d, sizeof(uint32_t*) * (size_t)e->world) == cudaSuccess) {
    if (cudaMemcpy(px->peers_d, px->peers.data(), sizeof(uint32_t*) * (size_t)e->world,
                   cudaMemcpyHostToDevice) != cudaSuccess)
      mapped = 0;
  } else {
    mapped = 0;
  }
  cudaGetLastError();
  std::vector<uint32_t> agree = allgather_words(e, mapped);
  bool all_mapped = true;
  for (uint32_t v : agree) all_mapped = all_mapped && v == 1u;
  return all_mapped;
}

// Sets up a region of `words` data words on every rank, or none (e->px stays
// null) when any rank cannot export or map one: the ranks agree on the
// outcome in two rounds over the group, so all take the same path.
void px_create(eb_engine* e, size_t words) {
  auto* px = new PeerExchange;
  std::string why;
  bool all_mapped = false;
  try {
    all_mapped = px_setup(e, px, words, why);
  } catch (...) {
    // An error before the ranks agreed: no kernel has stored into any
    // region, so this rank's mappings and memory go at once.
    for (int q = 0; q < (int)px->peers.size(); q++)
      if (q != e->rank && px->peers[q]) cudaIpcCloseMemHandle(px->peers[q]);
    if (px->peers_d) cudaFree(px->peers_d);
    if (px->base) cudaFree(px->base);
    delete px;
    cudaGetLastError();
    throw;
  }
  e->px = px;
  if (!all_mapped) {
    px_free(e);  // every rank frees: NCCL stays the path
    e->px_why = why.empty() ? "a peer could not map the regions" : why;
  } else {
    e->px_why.clear();
  }
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
    px_free(e);
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
        eb::PeerExchange* px = e->px;
        if (px && b->ptr == px->base + eb::kPxFlagWords && words_per_rank % 4 == 0 &&
            words_per_rank * (size_t)e->world <= px->words)
          eb::px_allgather(e, px->peers_d, e->world, e->rank, words_per_rank, ++px->epoch);
        else
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

extern "C" int eb_group_exchange(eb_engine* e, size_t words, eb_buf** out) {
  try {
    eb::ensure(e != nullptr && out != nullptr, "engine and out are required");
    eb::ensure(words > 0 && words < ((size_t)1 << 40), "words must be in 1 .. 2^40 - 1");
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != e->device) EB_CUDA(cudaSetDevice(e->device));
    struct Restore {
      int prev, dev;
      ~Restore() {
        if (prev >= 0 && prev != dev) cudaSetDevice(prev);
      }
    } restore{prev, e->device};
    // The flag words hold 64 ranks; larger groups take NCCL.
    if (e->world > 1 && e->world <= 64 && e->comm && (!e->px || e->px->words < words)) {
      eb::px_free(e);
      eb::px_create(e, words);
    }
    if (e->world > 1 && e->px) {
      auto* b = new eb_buf;
      b->ptr = e->px->base + eb::kPxFlagWords;
      b->len = words;
      b->dtype = EB_U32;
      b->owned = false;
      *out = b;
    } else {
      *out = eb::new_buf(e, EB_U32, words);
    }
    eb::set_last_error("");
    return EB_OK;
  } catch (const eb::Error& err) {
    eb::set_last_error(err.what());
    return err.code;
  }
}

extern "C" int eb_group_exchange_info(eb_engine* e, int* mapped, char* why, size_t cap) {
  if (!e || !mapped) {
    eb::set_last_error("engine and mapped are required");
    return EB_INVALID_ARGUMENT;
  }
  *mapped = e->px != nullptr ? 1 : 0;
  if (why && cap) {
    const std::string& w = e->px_why;
    const size_t len = std::min(cap - 1, w.size());
    std::memcpy(why, w.data(), len);
    why[len] = 0;
  }
  return EB_OK;
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
