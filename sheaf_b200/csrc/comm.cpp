// Data-parallel gradient all-reduce over NCCL (NVLink / NVSwitch).
//
// The reference has no collectives ("NCCL all-reduce" is a roadmap item,
// docs/roadmap.md:61-62); value_and_grad shards along the batch, so the only
// exchange is the average of the per-rank loss and gradients (a mean over
// equal shards is the mean of the shard means).
//
// libnccl.so.2 is opened at run time (the one torch already loaded, if any),
// so the library itself carries no link-time NCCL dependency.
//
// What is bounded: communicators are created non-blocking, and the host-side
// waits of set-up and of enqueueing a collective poll with a limit (a rank
// that never joins turns into a DEADLINE_EXCEEDED status, not a hang). What
// is not: an all-reduce that has been enqueued (or captured into a step's
// CUDA graph) waits on the GPU for every peer with no limit, so a rank that
// leaves in the middle of a step leaves the other ranks' NCCL kernels waiting.
// A rank may therefore leave only between steps, with none of its
// collectives in flight; the others learn of it on the host (the process
// group's store or a heartbeat) before their next step and end their
// communicators with ncclCommAbort (sb_session_leave_group with abort).
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

#include "runtime.h"

namespace sb {

namespace {

struct NcclApi {
  void* handle = nullptr;
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRankConfig) initRankConfig = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommGetAsyncError) asyncError = nullptr;
  decltype(&ncclGetErrorString) errorString = nullptr;
  std::string load_error;
};

NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    for (const char* name : {"libnccl.so.2", "libnccl.so"}) {
      a.handle = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
      if (a.handle) break;
    }
    if (!a.handle) {
      a.load_error = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
#define SB_SYM(field, sym) a.field = reinterpret_cast<decltype(a.field)>(dlsym(a.handle, #sym))
    SB_SYM(getUniqueId, ncclGetUniqueId);
    SB_SYM(initRankConfig, ncclCommInitRankConfig);
    SB_SYM(allReduce, ncclAllReduce);
    SB_SYM(destroy, ncclCommDestroy);
    SB_SYM(abort, ncclCommAbort);
    SB_SYM(asyncError, ncclCommGetAsyncError);
    SB_SYM(errorString, ncclGetErrorString);
#undef SB_SYM
    if (!a.getUniqueId || !a.initRankConfig || !a.allReduce || !a.destroy || !a.abort || !a.asyncError)
      a.load_error = "libnccl.so.2 lacks a required symbol";
  });
  return a;
}

}  // namespace

struct Comm {
  ncclComm_t comm = nullptr;
};

sb_status comm_get_unique_id(void* out, size_t bytes) {
  NcclApi& a = api();
  SB_RETURN_IF(!a.load_error.empty(), SB_STATUS_UNAVAILABLE, a.load_error);
  SB_RETURN_IF(bytes < sizeof(ncclUniqueId), SB_STATUS_INVALID_ARGUMENT, "id buffer too small");
  ncclUniqueId id;
  ncclResult_t r = a.getUniqueId(&id);
  SB_RETURN_IF(r != ncclSuccess, SB_STATUS_INTERNAL, "ncclGetUniqueId failed");
  std::memcpy(out, &id, sizeof(id));
  return nullptr;
}

// Polls a non-blocking communicator until its pending operation settles.
static sb_status wait_comm_ready(NcclApi& a, ncclComm_t c, int64_t timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st = ncclInProgress;
    if (a.asyncError(c, &st) != ncclSuccess) return make_status(SB_STATUS_INTERNAL, "ncclCommGetAsyncError failed");
    if (st == ncclSuccess) return nullptr;
    if (st != ncclInProgress)
      return make_status(SB_STATUS_INTERNAL, std::string("nccl: ") + (a.errorString ? a.errorString(st) : "error"));
    if (std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
        timeout_ms)
      return make_status(SB_STATUS_DEADLINE_EXCEEDED, "nccl communicator did not become ready");
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}

sb_status comm_init(Session& s, const void* unique_id, size_t id_bytes, int rank, int world) {
  NcclApi& a = api();
  SB_RETURN_IF(!a.load_error.empty(), SB_STATUS_UNAVAILABLE, a.load_error);
  SB_RETURN_IF(id_bytes < sizeof(ncclUniqueId), SB_STATUS_INVALID_ARGUMENT, "id buffer too small");
  SB_RETURN_IF(world < 1 || rank < 0 || rank >= world, SB_STATUS_INVALID_ARGUMENT, "bad rank/world");
  if (s.comm) comm_destroy(s);
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  // The all-reduces run beside the step's persistent kernels (one CTA per
  // SM): every SM an all-reduce holds pushes CTAs of those kernels into a
  // second wave. At most kNcclMaxCtas CTAs per collective (measured on two
  // B200s: nanoGPT-char 2.564 -> 2.44 ms/step with 8 or 16, GPT-2-small 9.98
  // -> 10.11 ms at 16 and worse below, its 248 MB of gradients needing the
  // bandwidth). SHEAF_B200_NCCL_MAX_CTAS overrides it; 0 leaves NCCL's choice.
  constexpr int kNcclMaxCtas = 16;
  int max_ctas = kNcclMaxCtas;
  if (const char* e = std::getenv("SHEAF_B200_NCCL_MAX_CTAS")) max_ctas = std::atoi(e);
  if (max_ctas > 0) {
    cfg.minCTAs = 1;
    cfg.maxCTAs = max_ctas;
    cfg.nvlsCTAs = max_ctas;
  }
  auto* c = new Comm();
  cudaSetDevice(s.device);
  ncclResult_t r = a.initRankConfig(&c->comm, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return make_status(SB_STATUS_INTERNAL, "ncclCommInitRankConfig failed");
  }
  sb_status st = wait_comm_ready(a, c->comm, 120000);
  if (st) {
    a.abort(c->comm);
    delete c;
    return st;
  }
  s.comm = c;
  s.rank = rank;
  s.world = world;
  return nullptr;
}

sb_status comm_allreduce_avg(Session& s, void* data, size_t count, uint32_t elem, cudaStream_t stream) {
  NcclApi& a = api();
  SB_RETURN_IF(!s.comm, SB_STATUS_INVALID_ARGUMENT, "session has no group");
  ncclDataType_t t;
  switch (elem) {
    case SB_ELEM_F32: t = ncclFloat32; break;
    case SB_ELEM_BF16: t = ncclBfloat16; break;
    case SB_ELEM_F16: t = ncclFloat16; break;
    default: return make_status(SB_STATUS_INVALID_ARGUMENT, "all-reduce element type");
  }
  ncclResult_t r = a.allReduce(data, data, count, t, ncclAvg, s.comm->comm, stream);
  if (r == ncclInProgress) return wait_comm_ready(a, s.comm->comm, 120000);
  SB_RETURN_IF(r != ncclSuccess, SB_STATUS_INTERNAL, "ncclAllReduce failed");
  return nullptr;
}

void comm_destroy(Session& s, bool abort) {
  if (!s.comm) return;
  NcclApi& a = api();
  if (abort && a.abort)
    a.abort(s.comm->comm);
  else if (a.destroy)
    a.destroy(s.comm->comm);
  delete s.comm;
  s.comm = nullptr;
  s.world = 1;
  s.rank = 0;
}

}  // namespace sb

extern "C" {

sb_status sb_nccl_unique_id(void* out_id, size_t id_bytes) {
  SB_RETURN_IF(!out_id, SB_STATUS_INVALID_ARGUMENT, "null id");
  return sb::comm_get_unique_id(out_id, id_bytes);
}

sb_status sb_session_join_group(sb_session* session, const void* nccl_id, size_t id_bytes, int rank, int world) {
  SB_RETURN_IF(!session || !nccl_id, SB_STATUS_INVALID_ARGUMENT, "null argument");
  return sb::comm_init(*static_cast<sb::Session*>(session), nccl_id, id_bytes, rank, world);
}

sb_status sb_session_leave_group(sb_session* session, int abort) {
  SB_RETURN_IF(!session, SB_STATUS_INVALID_ARGUMENT, "null session");
  auto* s = static_cast<sb::Session*>(session);
  SB_RETURN_IF(!s->comm, SB_STATUS_FAILED_PRECONDITION, "session is not in a group");
  std::lock_guard<std::mutex> lk(s->mu);
  sb::comm_destroy(*s, abort != 0);
  return nullptr;
}

}  // extern "C"
