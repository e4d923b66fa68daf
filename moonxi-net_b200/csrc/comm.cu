// comm.cu -- the data-parallel collective stubs of the C ABI
// (moonbit_nccl_*, include/mx_matmul.h): NCCL communicators over NVLink /
// NVSwitch, created, used, watched and torn down through plain pointers and
// sizes so that a host without torch (the reference's MoonBit train loop,
// moonxi-net-gpu/train/run.mbt:14-57) can run the data-parallel MLP step.
// The reference has no collectives at all; these stubs are new surface.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2): a process that
// already holds an NCCL (torch does) shares it, the library still loads on a
// machine without NCCL, and a missing NCCL is a status code, not a link
// error.  Host code only: the collectives' kernels are NCCL's own.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_set>

#include "../../include/mx_matmul.h"
#include "mx_internal.h"

#define MX_EXPORT extern "C" __attribute__((visibility("default")))

namespace mx {
namespace {

// The NCCL entry points this file uses, resolved once.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_version)(int*) = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  // optional (NCCL >= 2.14): communicator options such as the CTA cap
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int,
                                        ncclConfig_t*) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                 ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    auto sym = [h](const char* name) { return dlsym(h, name); };
#define MX_NCCL_SYM(field, name) \
  api.field = reinterpret_cast<decltype(api.field)>(sym(name))
    MX_NCCL_SYM(get_version, "ncclGetVersion");
    MX_NCCL_SYM(get_unique_id, "ncclGetUniqueId");
    MX_NCCL_SYM(comm_init_rank, "ncclCommInitRank");
    MX_NCCL_SYM(all_reduce, "ncclAllReduce");
    MX_NCCL_SYM(reduce_scatter, "ncclReduceScatter");
    MX_NCCL_SYM(all_gather, "ncclAllGather");
    MX_NCCL_SYM(broadcast, "ncclBroadcast");
    MX_NCCL_SYM(group_start, "ncclGroupStart");
    MX_NCCL_SYM(group_end, "ncclGroupEnd");
    MX_NCCL_SYM(get_async_error, "ncclCommGetAsyncError");
    MX_NCCL_SYM(comm_abort, "ncclCommAbort");
    MX_NCCL_SYM(comm_finalize, "ncclCommFinalize");
    MX_NCCL_SYM(comm_destroy, "ncclCommDestroy");
    api.comm_init_rank_config = reinterpret_cast<decltype(api.comm_init_rank_config)>(
        sym("ncclCommInitRankConfig"));
#undef MX_NCCL_SYM
    api.ok = api.get_version && api.get_unique_id && api.comm_init_rank && api.all_reduce &&
             api.reduce_scatter && api.all_gather && api.broadcast && api.group_start &&
             api.group_end && api.get_async_error && api.comm_abort && api.comm_destroy;
  });
  return api;
}

int nccl_status(ncclResult_t r) {
  if (r == ncclSuccess) return MX_OK;
  if (r == ncclInvalidArgument || r == ncclInvalidUsage) return MX_ERR_INVALID;
  return MX_ERR_COMM;
}

// One communicator handed out by moonbit_nccl_init*.  Handles are checked
// against this registry and never dereferenced when unknown.
struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
};
std::mutex g_mu;
std::unordered_set<Comm*> g_comms;

Comm* lookup(void* handle) {
  std::lock_guard<std::mutex> lk(g_mu);
  Comm* c = static_cast<Comm*>(handle);
  return (c && g_comms.count(c)) ? c : nullptr;
}

// Removes a handle from the registry (it is invalid from then on).
Comm* take(void* handle) {
  std::lock_guard<std::mutex> lk(g_mu);
  Comm* c = static_cast<Comm*>(handle);
  if (!c || !g_comms.count(c)) return nullptr;
  g_comms.erase(c);
  return c;
}

thread_local int t_last_status = MX_OK;

void* fail(int st) {
  t_last_status = st;
  return nullptr;
}

// The device current for the duration of a call, the caller's restored after.
struct DeviceScope {
  int prev = -1;
  bool ok = true;
  explicit DeviceScope(int dev) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) {
      ok = false;
      return;
    }
    if (cur != dev) {
      ok = cudaSetDevice(dev) == cudaSuccess;
      if (ok) prev = cur;
    }
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// max_ctas > 0: NCCL's kernels of this communicator take at most that many
// CTAs (SMs), launched without thread-block clusters, so that they fit beside
// GEMMs that leave that many SMs free.
void* init_with_id(const ncclUniqueId& id, int rank, int world, int device, int max_ctas = 0) {
  const NcclApi& api = nccl();
  if (!api.ok) return fail(MX_ERR_UNSUPPORTED);
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return fail(MX_ERR_NO_DEVICE);
  if (device < 0 || device >= count) return fail(MX_ERR_INVALID);
  DeviceScope ds(device);
  if (!ds.ok) return fail(MX_ERR_CUDA);
  ncclComm_t comm = nullptr;
  ncclResult_t r;
  if (max_ctas > 0 && api.comm_init_rank_config) {
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.minCTAs = 1;
    cfg.maxCTAs = max_ctas;
    // single-CTA launches: a cluster needs several SMs of one GPC free at
    // once, which SMs left over here and there beside a GEMM rarely are
    cfg.cgaClusterSize = 1;
    r = api.comm_init_rank_config(&comm, world, id, rank, &cfg);
  } else {
    if (max_ctas > 0) return fail(MX_ERR_UNSUPPORTED);
    r = api.comm_init_rank(&comm, world, id, rank);
  }
  if (r != ncclSuccess) return fail(nccl_status(r));
  Comm* c = new Comm();
  c->comm = comm;
  c->rank = rank;
  c->world = world;
  c->device = device;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    g_comms.insert(c);
  }
  t_last_status = MX_OK;
  return c;
}

bool count_ok(int64_t n) { return n >= 0 && static_cast<uint64_t>(n) <= (1ull << 40); }

}  // namespace
}  // namespace mx

using namespace mx;

MX_EXPORT int32_t moonbit_nccl_version(void) {
  const NcclApi& api = nccl();
  if (!api.ok) return -1;
  int v = 0;
  return api.get_version(&v) == ncclSuccess ? v : -1;
}

MX_EXPORT int32_t moonbit_nccl_get_unique_id(uint8_t* id) {
  if (!id) return MX_ERR_INVALID;
  const NcclApi& api = nccl();
  if (!api.ok) return MX_ERR_UNSUPPORTED;
  ncclUniqueId u;
  ncclResult_t r = api.get_unique_id(&u);
  if (r != ncclSuccess) return nccl_status(r);
  std::memcpy(id, u.internal, MX_NCCL_UNIQUE_ID_BYTES);
  return MX_OK;
}

MX_EXPORT void* moonbit_nccl_init(const uint8_t* id, int32_t rank, int32_t world,
                                  int32_t device) {
  if (!id || world < 1 || rank < 0 || rank >= world) return fail(MX_ERR_INVALID);
  ncclUniqueId u;
  std::memcpy(u.internal, id, MX_NCCL_UNIQUE_ID_BYTES);
  return init_with_id(u, rank, world, device);
}

MX_EXPORT void* moonbit_nccl_init_ex(const uint8_t* id, int32_t rank, int32_t world,
                                     int32_t device, int32_t max_ctas) {
  if (!id || world < 1 || rank < 0 || rank >= world || max_ctas < 0) return fail(MX_ERR_INVALID);
  ncclUniqueId u;
  std::memcpy(u.internal, id, MX_NCCL_UNIQUE_ID_BYTES);
  return init_with_id(u, rank, world, device, max_ctas);
}

MX_EXPORT void* moonbit_nccl_init_file(const char* path, int32_t rank, int32_t world,
                                       int32_t device, int32_t timeout_ms) {
  if (!path || !path[0] || world < 1 || rank < 0 || rank >= world || timeout_ms < 0)
    return fail(MX_ERR_INVALID);
  ncclUniqueId u;
  if (rank == 0) {
    const int st = moonbit_nccl_get_unique_id(reinterpret_cast<uint8_t*>(u.internal));
    if (st != MX_OK) return fail(st);
    // write-then-rename: a reader never sees a partial id
    const std::string tmp = std::string(path) + ".tmp." + std::to_string(getpid());
    FILE* f = std::fopen(tmp.c_str(), "wb");
    if (!f) return fail(MX_ERR_INVALID);
    const size_t w = std::fwrite(u.internal, 1, MX_NCCL_UNIQUE_ID_BYTES, f);
    const bool closed = std::fclose(f) == 0;
    if (w != MX_NCCL_UNIQUE_ID_BYTES || !closed || std::rename(tmp.c_str(), path) != 0) {
      std::remove(tmp.c_str());
      return fail(MX_ERR_INVALID);
    }
  } else {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
      struct stat sb;
      if (stat(path, &sb) == 0 && sb.st_size == MX_NCCL_UNIQUE_ID_BYTES) {
        FILE* f = std::fopen(path, "rb");
        if (f) {
          const size_t r = std::fread(u.internal, 1, MX_NCCL_UNIQUE_ID_BYTES, f);
          std::fclose(f);
          if (r == MX_NCCL_UNIQUE_ID_BYTES) break;
        }
      }
      const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                          std::chrono::steady_clock::now() - t0)
                          .count();
      if (ms >= timeout_ms) return fail(MX_ERR_TIMEOUT);
      std::this_thread::sleep_for(std::chrono::milliseconds(2));
    }
  }
  return init_with_id(u, rank, world, device);
}

MX_EXPORT int32_t moonbit_nccl_last_status(void) { return t_last_status; }

MX_EXPORT int32_t moonbit_nccl_comm_info(void* comm, int32_t* rank, int32_t* world,
                                         int32_t* device) {
  Comm* c = lookup(comm);
  if (!c) return MX_ERR_INVALID;
  if (rank) *rank = c->rank;
  if (world) *world = c->world;
  if (device) *device = c->device;
  return MX_OK;
}

MX_EXPORT int32_t moonbit_nccl_allreduce_sum_f32(void* comm, const float* send, float* recv,
                                                 int64_t count, void* stream) {
  Comm* c = lookup(comm);
  if (!c || !count_ok(count) || (count > 0 && (!send || !recv))) return MX_ERR_INVALID;
  if (count == 0) return MX_OK;
  DeviceScope ds(c->device);
  if (!ds.ok) return MX_ERR_CUDA;
  return nccl_status(nccl().all_reduce(send, recv, static_cast<size_t>(count), ncclFloat32,
                                       ncclSum, c->comm, static_cast<cudaStream_t>(stream)));
}

MX_EXPORT int32_t moonbit_nccl_reduce_scatter_sum_f32(void* comm, const float* send, float* recv,
                                                      int64_t recv_count, void* stream) {
  Comm* c = lookup(comm);
  if (!c || !count_ok(recv_count) || (recv_count > 0 && (!send || !recv))) return MX_ERR_INVALID;
  if (recv_count == 0) return MX_OK;
  DeviceScope ds(c->device);
  if (!ds.ok) return MX_ERR_CUDA;
  return nccl_status(nccl().reduce_scatter(send, recv, static_cast<size_t>(recv_count),
                                           ncclFloat32, ncclSum, c->comm,
                                           static_cast<cudaStream_t>(stream)));
}

MX_EXPORT int32_t moonbit_nccl_all_gather_f32(void* comm, const float* send, float* recv,
                                              int64_t send_count, void* stream) {
  Comm* c = lookup(comm);
  if (!c || !count_ok(send_count) || (send_count > 0 && (!send || !recv))) return MX_ERR_INVALID;
  if (send_count == 0) return MX_OK;
  DeviceScope ds(c->device);
  if (!ds.ok) return MX_ERR_CUDA;
  return nccl_status(nccl().all_gather(send, recv, static_cast<size_t>(send_count), ncclFloat32,
                                       c->comm, static_cast<cudaStream_t>(stream)));
}

MX_EXPORT int32_t moonbit_nccl_broadcast_f32(void* comm, const float* send, float* recv,
                                             int64_t count, int32_t root, void* stream) {
  Comm* c = lookup(comm);
  if (!c || !count_ok(count) || root < 0 || root >= c->world ||
      (count > 0 && (!recv || (c->rank == root && !send))))
    return MX_ERR_INVALID;
  if (count == 0) return MX_OK;
  DeviceScope ds(c->device);
  if (!ds.ok) return MX_ERR_CUDA;
  return nccl_status(nccl().broadcast(send, recv, static_cast<size_t>(count), ncclFloat32, root,
                                      c->comm, static_cast<cudaStream_t>(stream)));
}

MX_EXPORT int32_t moonbit_nccl_group_start(void) {
  const NcclApi& api = nccl();
  if (!api.ok) return MX_ERR_UNSUPPORTED;
  return nccl_status(api.group_start());
}

MX_EXPORT int32_t moonbit_nccl_group_end(void) {
  const NcclApi& api = nccl();
  if (!api.ok) return MX_ERR_UNSUPPORTED;
  return nccl_status(api.group_end());
}

MX_EXPORT int32_t moonbit_nccl_get_async_error(void* comm) {
  Comm* c = lookup(comm);
  if (!c) return MX_ERR_INVALID;
  ncclResult_t err = ncclSuccess;
  ncclResult_t r = nccl().get_async_error(c->comm, &err);
  if (r != ncclSuccess) return nccl_status(r);
  return (err == ncclSuccess || err == ncclInProgress) ? MX_OK : MX_ERR_COMM;
}

MX_EXPORT int32_t moonbit_nccl_abort(void* comm) {
  Comm* c = take(comm);
  if (!c) return MX_ERR_INVALID;
  DeviceScope ds(c->device);
  const ncclResult_t r = nccl().comm_abort(c->comm);
  delete c;
  return nccl_status(r);
}

MX_EXPORT int32_t moonbit_nccl_wait(void* comm, void* stream, int32_t timeout_ms) {
  Comm* c = lookup(comm);
  if (!c || timeout_ms < 0) return MX_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = MX_OK;
  {
    DeviceScope ds(c->device);
    if (!ds.ok) return MX_ERR_CUDA;
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
      const cudaError_t q = cudaStreamQuery(s);
      if (q == cudaSuccess) return MX_OK;
      if (q != cudaErrorNotReady) return cuda_status(q);
      if (moonbit_nccl_get_async_error(comm) != MX_OK) {
        st = MX_ERR_COMM;
        break;
      }
      const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                          std::chrono::steady_clock::now() - t0)
                          .count();
      if (ms >= timeout_ms) {
        st = MX_ERR_TIMEOUT;
        break;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
  // A failed or overdue communicator is aborted, so that its kernels stop
  // waiting for peers; the handle is invalid afterwards.
  moonbit_nccl_abort(comm);
  return st;
}

MX_EXPORT int32_t moonbit_nccl_destroy(void* comm) {
  Comm* c = take(comm);
  if (!c) return MX_ERR_INVALID;
  DeviceScope ds(c->device);
  ncclResult_t r = ncclSuccess;
  if (nccl().comm_finalize) r = nccl().comm_finalize(c->comm);
  const ncclResult_t r2 = nccl().comm_destroy(c->comm);
  delete c;
  return nccl_status(r != ncclSuccess ? r : r2);
}
