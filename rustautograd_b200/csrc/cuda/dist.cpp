// NCCL communicator for the data-parallel step (one process per GPU over NVLink/NVSwitch).
#include "dist.h"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <thread>

#include "rgc.h"

namespace rgc {

namespace {

struct Nccl {
  void* lib = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

std::mutex g_mu;
Nccl g_nccl;
ncclComm_t g_comm = nullptr;
int g_rank = 0, g_world = 1;
bool g_aborted = false;

void load() {
  if (g_nccl.lib) return;
  // Prefer an NCCL that is already loaded (PyTorch's), then the default search path.
  void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) throw std::runtime_error("NCCL (libnccl.so.2) is not available");
  auto sym = [&](const char* n) {
    void* p = dlsym(lib, n);
    if (!p) throw std::runtime_error(std::string("NCCL symbol missing: ") + n);
    return p;
  };
  g_nccl.GetUniqueId = (decltype(g_nccl.GetUniqueId))sym("ncclGetUniqueId");
  g_nccl.CommInitRank = (decltype(g_nccl.CommInitRank))sym("ncclCommInitRank");
  g_nccl.AllReduce = (decltype(g_nccl.AllReduce))sym("ncclAllReduce");
  g_nccl.GroupStart = (decltype(g_nccl.GroupStart))sym("ncclGroupStart");
  g_nccl.GroupEnd = (decltype(g_nccl.GroupEnd))sym("ncclGroupEnd");
  g_nccl.CommDestroy = (decltype(g_nccl.CommDestroy))sym("ncclCommDestroy");
  g_nccl.CommAbort = (decltype(g_nccl.CommAbort))sym("ncclCommAbort");
  g_nccl.GetErrorString = (decltype(g_nccl.GetErrorString))sym("ncclGetErrorString");
  g_nccl.lib = lib;
}

void nck(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw std::runtime_error(std::string(what) + ": " + (g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "NCCL error"));
}

}  // namespace

bool dist_active() { return g_comm != nullptr && g_world > 1; }
bool dist_aborted() { return g_aborted; }
int dist_rank() { return g_rank; }
int dist_world() { return g_world; }

void dist_all_reduce(void* buf, size_t count, bool is_f64, cudaStream_t stream) {
  if (!dist_active()) return;
  nck(g_nccl.AllReduce(buf, buf, count, is_f64 ? ncclFloat64 : ncclFloat32, ncclSum, g_comm, stream), "ncclAllReduce");
}

void dist_all_reduce_into(void* dst, const void* src, size_t count, bool is_f64, cudaStream_t stream) {
  nck(g_nccl.AllReduce(src, dst, count, is_f64 ? ncclFloat64 : ncclFloat32, ncclSum, g_comm, stream), "ncclAllReduce");
}

cudaError_t dist_sync(cudaStream_t stream, std::string* why) {
  if (!dist_active()) return cudaStreamSynchronize(stream);
  double limit = 300.0;
  if (const char* e = std::getenv("RGC_COLLECTIVE_TIMEOUT_S")) limit = std::atof(e) > 0 ? std::atof(e) : limit;
  const auto t0 = std::chrono::steady_clock::now();
  auto pause = std::chrono::microseconds(20);
  for (;;) {
    cudaError_t q = cudaStreamQuery(stream);
    if (q != cudaErrorNotReady) return q;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit) break;
    std::this_thread::sleep_for(pause);
    if (pause < std::chrono::milliseconds(2)) pause *= 2;
  }
  // A collective has waited past the limit (another rank stopped or diverged): abort the
  // communicator so that its kernels return, then drain the stream.
  const bool trace = std::getenv("RGC_TRACE_DIST") != nullptr;
  if (trace) std::fprintf(stderr, "rgc dist: rank %d: stream still busy after %.1f s, aborting the communicator\n", g_rank, limit);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_comm) {
      g_nccl.CommAbort(g_comm);
      g_comm = nullptr;
      g_aborted = true;
    }
  }
  if (trace) std::fprintf(stderr, "rgc dist: rank %d: communicator aborted\n", g_rank);
  // The aborted collectives return; the drain is bounded as well.
  const auto t1 = std::chrono::steady_clock::now();
  while (cudaStreamQuery(stream) == cudaErrorNotReady &&
         std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count() < 30.0)
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  if (trace) std::fprintf(stderr, "rgc dist: rank %d: stream %s after the abort\n", g_rank, cudaStreamQuery(stream) == cudaErrorNotReady ? "still busy" : "drained");
  cudaGetLastError();
  if (why) *why = "a collective waited more than " + std::to_string((int)limit) + " s for another rank; the communicator was aborted";
  return cudaErrorLaunchTimeout;
}

void dist_group_start() {
  if (dist_active()) nck(g_nccl.GroupStart(), "ncclGroupStart");
}
void dist_group_end() {
  if (dist_active()) nck(g_nccl.GroupEnd(), "ncclGroupEnd");
}

}  // namespace rgc

using namespace rgc;

extern "C" {

__attribute__((visibility("default"))) int rgc_dist_unique_id(uint8_t id[128]) {
  try {
    std::lock_guard<std::mutex> lk(g_mu);
    load();
    ncclUniqueId u;
    nck(g_nccl.GetUniqueId(&u), "ncclGetUniqueId");
    static_assert(sizeof(u) == 128, "NCCL unique id is 128 bytes");
    std::memcpy(id, &u, 128);
    return RGC_OK;
  } catch (const std::exception&) {
    return RGC_ERR_UNAVAILABLE;
  }
}

__attribute__((visibility("default"))) int rgc_dist_init(int rank, int world, const uint8_t id[128]) {
  try {
    std::lock_guard<std::mutex> lk(g_mu);
    if (world <= 1) {
      g_rank = 0;
      g_world = 1;
      return RGC_OK;
    }
    load();
    ncclUniqueId u;
    std::memcpy(&u, id, 128);
    ncclComm_t comm;
    nck(g_nccl.CommInitRank(&comm, world, u, rank), "ncclCommInitRank");
    g_comm = comm;
    g_aborted = false;
    g_rank = rank;
    g_world = world;
    return RGC_OK;
  } catch (const std::exception&) {
    return RGC_ERR_UNAVAILABLE;
  }
}

__attribute__((visibility("default"))) int rgc_dist_finalize(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_comm) {
    cudaDeviceSynchronize();
    g_nccl.CommDestroy(g_comm);
    g_comm = nullptr;
  }
  g_rank = 0;
  g_world = 1;
  return RGC_OK;
}

}  // extern "C"
