// Weight broadcast for data-parallel runs of the encoder policy: the C ABI
// block "weight broadcast over NCCL" of include/ow_policy.h.
//
// States are independent, so a multi-GPU run shards them with no exchange on
// the data path; the one exchange is the model itself. It moves as the
// handle's packed device weight arena (bf16 / e4m3 matrices with their
// scales, f32 vectors: exactly the bytes the kernels read), one ncclBroadcast
// over NVLink / NVSwitch from the root's arena into every other rank's. No
// host round trip and no re-conversion on the receivers; the receivers' arena
// layout, pointers and tensor maps stay as they are, because the layout is a
// function of the config alone.
//
// NCCL is resolved at run time (dlopen), so the library links no NCCL and a
// process that never broadcasts never loads it. Every wait is bounded: the
// communicator set-up polls ncclCommGetAsyncError, the broadcast polls its
// stream, and on expiry the communicator is aborted (which ends its kernels)
// and RUNTIME_ERROR comes back, so a rank that never joins cannot hang the
// others' GPUs.

#include "ow_policy.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>  // types and the config initialiser only; the functions come from dlsym

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace {

OwStatus ok() { return {OW_STATUS_OK, "ok"}; }
OwStatus bad(const char* m) { return {OW_STATUS_BAD_ARGUMENT, m}; }
OwStatus rt(const char* m) { return {OW_STATUS_RUNTIME_ERROR, m}; }

struct Nccl {
  bool loaded = false;
  const char* why = "NCCL not loaded";
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*init_all)(ncclComm_t*, int, const int*) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*count)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*version)(int*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

// The libnccl.so.2 already in the process (a framework's), else
// $ORBIT_WARS_NCCL_LIB, else libnccl.so.2 from the loader path.
Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) {
      const char* path = std::getenv("ORBIT_WARS_NCCL_LIB");
      if (path != nullptr && path[0] != '\0') h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    }
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) {
      n.why = "libnccl.so.2 not found (set ORBIT_WARS_NCCL_LIB)";
      return;
    }
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      all = all && fn != nullptr;
    };
    sym(n.get_unique_id, "ncclGetUniqueId");
    sym(n.init_rank_config, "ncclCommInitRankConfig");
    sym(n.init_all, "ncclCommInitAll");
    sym(n.async_error, "ncclCommGetAsyncError");
    sym(n.broadcast, "ncclBroadcast");
    sym(n.group_start, "ncclGroupStart");
    sym(n.group_end, "ncclGroupEnd");
    sym(n.destroy, "ncclCommDestroy");
    sym(n.abort, "ncclCommAbort");
    sym(n.count, "ncclCommCount");
    sym(n.version, "ncclGetVersion");
    sym(n.error_string, "ncclGetErrorString");
    if (!all) {
      n.why = "libnccl.so.2 lacks a needed symbol";
      return;
    }
    n.loaded = true;
  });
  return n;
}

double limit_seconds() {
  const char* e = std::getenv("ORBIT_WARS_COMM_TIMEOUT_S");
  const double v = e != nullptr ? std::atof(e) : 0.0;
  return v > 0.0 ? v : 120.0;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Waits for every stream, polling, at most `limit` seconds.
bool wait_streams(const std::vector<cudaStream_t>& s, double limit, cudaError_t* err) {
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<bool> done(s.size(), false);
  size_t left = s.size();
  while (left > 0) {
    for (size_t i = 0; i < s.size(); ++i) {
      if (done[i]) continue;
      const cudaError_t q = cudaStreamQuery(s[i]);
      if (q == cudaSuccess) {
        done[i] = true;
        --left;
      } else if (q != cudaErrorNotReady) {
        *err = q;
        return false;
      }
    }
    if (left == 0) break;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit) {
      *err = cudaErrorNotReady;
      return false;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  *err = cudaSuccess;
  return true;
}

// The device that owns `p` (the handle's weight arena).
int device_of(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess || a.type != cudaMemoryTypeDevice) return -1;
  return a.device;
}

}  // namespace

struct OwComm {
  ncclComm_t comm = nullptr;
  int rank = 0, nranks = 1, device = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  bool broken = false;  // aborted after an expired wait: only ow_comm_destroy is valid
};

namespace {

OwStatus comm_finish_setup(OwComm* c) {
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&c->t0) != cudaSuccess || cudaEventCreate(&c->t1) != cudaSuccess)
    return rt("stream or event creation failed");
  return ok();
}

void comm_release(OwComm* c) {
  if (c == nullptr) return;
  Nccl& n = nccl();
  DeviceGuard g(c->device);
  if (c->comm != nullptr && n.loaded) (c->broken ? n.abort : n.destroy)(c->comm);
  if (c->t0) cudaEventDestroy(c->t0);
  if (c->t1) cudaEventDestroy(c->t1);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

// Broadcasts the arenas of `pols` (one per comm) from `root` in one NCCL group.
OwStatus broadcast_group(OwPolicy* const* pols, OwComm* const* comms, int n, int root, float* elapsed_ms) {
  Nccl& nc = nccl();
  if (!nc.loaded) return rt(nc.why);
  std::vector<void*> arena(n);
  std::vector<size_t> bytes(n);
  for (int i = 0; i < n; ++i) {
    if (pols[i] == nullptr || comms[i] == nullptr) return bad("null handle or communicator");
    if (comms[i]->broken) return rt("communicator was aborted after an expired wait");
    OwStatus s = ow_policy_device_weights(pols[i], &arena[i], &bytes[i]);
    if (s.code != OW_STATUS_OK) return s;
    if (bytes[i] != bytes[0]) return bad("handles hold different weight layouts");
    if (device_of(arena[i]) != comms[i]->device) return bad("handle and communicator are on different devices");
    // forwards in flight read the arena: let them finish (and report their errors) first
    s = ow_policy_synchronize(pols[i]);
    if (s.code != OW_STATUS_OK) return s;
  }
  std::vector<cudaStream_t> streams(n);
  for (int i = 0; i < n; ++i) {
    DeviceGuard g(comms[i]->device);
    if (cudaEventRecord(comms[i]->t0, comms[i]->stream) != cudaSuccess) return rt("event record failed");
    streams[i] = comms[i]->stream;
  }
  ncclResult_t r = ncclSuccess;
  if (n > 1) r = nc.group_start();
  for (int i = 0; i < n && (r == ncclSuccess || r == ncclInProgress); ++i) {
    DeviceGuard g(comms[i]->device);
    r = nc.broadcast(arena[i], arena[i], bytes[i], ncclUint8, root, comms[i]->comm, comms[i]->stream);
  }
  if (n > 1 && (r == ncclSuccess || r == ncclInProgress)) r = nc.group_end();
  if (r != ncclSuccess && r != ncclInProgress) return rt(nc.error_string(r));
  // a non-blocking communicator may still be enqueuing: wait (bounded) until
  // the broadcast is on the streams before recording the closing events
  const auto t_enq = std::chrono::steady_clock::now();
  for (int i = 0; i < n; ++i) {
    for (;;) {
      ncclResult_t st = ncclSuccess;
      if (nc.async_error(comms[i]->comm, &st) != ncclSuccess) return rt("ncclCommGetAsyncError failed");
      if (st == ncclSuccess) break;
      if (st != ncclInProgress) return rt(nc.error_string(st));
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t_enq).count() > limit_seconds()) {
        for (int k = 0; k < n; ++k) {
          DeviceGuard g(comms[k]->device);
          nc.abort(comms[k]->comm);
          comms[k]->comm = nullptr;
          comms[k]->broken = true;
        }
        return rt("weight broadcast timed out while enqueuing (communicator aborted)");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
  for (int i = 0; i < n; ++i) {
    DeviceGuard g(comms[i]->device);
    if (cudaEventRecord(comms[i]->t1, comms[i]->stream) != cudaSuccess) return rt("event record failed");
  }
  cudaError_t e = cudaSuccess;
  if (!wait_streams(streams, limit_seconds(), &e)) {
    for (int i = 0; i < n; ++i) {
      DeviceGuard g(comms[i]->device);
      nc.abort(comms[i]->comm);
      comms[i]->comm = nullptr;
      comms[i]->broken = true;
    }
    return rt(e == cudaErrorNotReady ? "weight broadcast timed out (communicator aborted)"
                                     : "weight broadcast failed on the device");
  }
  for (int i = 0; i < n; ++i) {
    ncclResult_t ae = ncclSuccess;
    nc.async_error(comms[i]->comm, &ae);
    if (ae != ncclSuccess) return rt(nc.error_string(ae));
  }
  if (elapsed_ms != nullptr) {
    float worst = 0.0f;
    for (int i = 0; i < n; ++i) {
      float ms = 0.0f;
      DeviceGuard g(comms[i]->device);
      if (cudaEventElapsedTime(&ms, comms[i]->t0, comms[i]->t1) == cudaSuccess && ms > worst) worst = ms;
    }
    *elapsed_ms = worst;
  }
  return ok();
}

}  // namespace

extern "C" {

OwStatus ow_comm_unique_id(void* id, size_t id_bytes) {
  if (id == nullptr || id_bytes < sizeof(ncclUniqueId)) return bad("id buffer must hold 128 bytes");
  Nccl& nc = nccl();
  if (!nc.loaded) return rt(nc.why);
  ncclUniqueId u;
  const ncclResult_t r = nc.get_unique_id(&u);
  if (r != ncclSuccess) return rt(nc.error_string(r));
  std::memcpy(id, &u, sizeof(u));
  return ok();
}

OwStatus ow_comm_init_rank(const void* id, size_t id_bytes, int nranks, int rank, int device, OwComm** out) {
  if (id == nullptr || out == nullptr || id_bytes < sizeof(ncclUniqueId)) return bad("null argument or short id");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks) return bad("rank outside [0, nranks)");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return bad("device index out of range");
  Nccl& nc = nccl();
  if (!nc.loaded) return rt(nc.why);
  DeviceGuard g(device);
  auto* c = new OwComm();
  c->rank = rank;
  c->nranks = nranks;
  c->device = device;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // set-up polled below, bounded
  ncclResult_t r = nc.init_rank_config(&c->comm, nranks, u, rank, &cfg);
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress || r == ncclSuccess) {
    ncclResult_t st = ncclInProgress;
    if (c->comm == nullptr || nc.async_error(c->comm, &st) != ncclSuccess) {
      r = ncclInternalError;
      break;
    }
    if (st == ncclSuccess) {
      r = ncclSuccess;
      break;
    }
    if (st != ncclInProgress) {
      r = st;
      break;
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit_seconds()) {
      nc.abort(c->comm);
      c->comm = nullptr;
      comm_release(c);
      return rt("communicator set-up timed out (a rank did not join)");
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (r != ncclSuccess) {
    if (c->comm != nullptr) nc.abort(c->comm);
    c->comm = nullptr;
    comm_release(c);
    return rt(nc.error_string(r));
  }
  OwStatus s = comm_finish_setup(c);
  if (s.code != OW_STATUS_OK) {
    comm_release(c);
    return s;
  }
  *out = c;
  return ok();
}

OwStatus ow_comm_init_all(const int* devices, int n, OwComm** out) {
  if (devices == nullptr || out == nullptr || n < 1) return bad("null argument or n < 1");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess) return rt("no cuda devices");
  for (int i = 0; i < n; ++i) {
    out[i] = nullptr;
    if (devices[i] < 0 || devices[i] >= ndev) return bad("device index out of range");
    for (int j = 0; j < i; ++j)
      if (devices[j] == devices[i]) return bad("one communicator rank per device");
  }
  Nccl& nc = nccl();
  if (!nc.loaded) return rt(nc.why);
  std::vector<ncclComm_t> comms(n, nullptr);
  const ncclResult_t r = nc.init_all(comms.data(), n, devices);  // one process: every rank is local
  if (r != ncclSuccess) return rt(nc.error_string(r));
  for (int i = 0; i < n; ++i) {
    DeviceGuard g(devices[i]);
    auto* c = new OwComm();
    c->comm = comms[i];
    c->rank = i;
    c->nranks = n;
    c->device = devices[i];
    OwStatus s = comm_finish_setup(c);
    out[i] = c;
    if (s.code != OW_STATUS_OK) {
      for (int k = 0; k <= i; ++k) {
        comm_release(out[k]);
        out[k] = nullptr;
      }
      for (int k = i + 1; k < n; ++k) nc.destroy(comms[k]);
      return s;
    }
  }
  return ok();
}

OwStatus ow_comm_info(const OwComm* comm, int* rank, int* nranks, int* device) {
  if (comm == nullptr) return bad("null communicator");
  if (rank) *rank = comm->rank;
  if (nranks) *nranks = comm->nranks;
  if (device) *device = comm->device;
  return ok();
}

void ow_comm_destroy(OwComm* comm) { comm_release(comm); }

OwStatus ow_policy_broadcast_weights_comm(OwPolicy* policy, OwComm* comm, int root, float* elapsed_ms) {
  if (policy == nullptr || comm == nullptr) return bad("null argument");
  if (root < 0 || root >= comm->nranks) return bad("root outside [0, nranks)");
  OwPolicy* p[1] = {policy};
  OwComm* c[1] = {comm};
  return broadcast_group(p, c, 1, root, elapsed_ms);
}

OwStatus ow_policy_broadcast_weights(OwPolicy** handles, int n_gpus) {
  if (handles == nullptr || n_gpus < 1) return bad("null handles or n_gpus < 1");
  if (n_gpus == 1) return handles[0] != nullptr ? ok() : bad("null handle");
  std::vector<int> devs(n_gpus);
  for (int i = 0; i < n_gpus; ++i) {
    if (handles[i] == nullptr) return bad("null handle");
    void* a = nullptr;
    size_t b = 0;
    OwStatus s = ow_policy_device_weights(handles[i], &a, &b);
    if (s.code != OW_STATUS_OK) return s;
    devs[i] = device_of(a);
    if (devs[i] < 0) return rt("weight arena is not device memory");
  }
  std::vector<OwComm*> comms(n_gpus, nullptr);
  OwStatus s = ow_comm_init_all(devs.data(), n_gpus, comms.data());
  if (s.code != OW_STATUS_OK) return s;
  s = broadcast_group(handles, comms.data(), n_gpus, 0, nullptr);
  for (auto* c : comms) comm_release(c);
  return s;
}

OwStatus ow_nccl_version(int* version) {
  if (version == nullptr) return bad("null argument");
  Nccl& nc = nccl();
  if (!nc.loaded) return rt(nc.why);
  const ncclResult_t r = nc.version(version);
  return r == ncclSuccess ? ok() : rt(nc.error_string(r));
}

}  // extern "C"
