// tp.cu — the tensor-parallel communicator of a model: NCCL, loaded at run time (dlopen of libnccl.so.2, the copy the
// process already holds when torch has loaded one), so the library loads and runs single-device without it.
// The collectives of a decode step (two fp32 all-reduces per layer, one all-gather of the head's per-rank maxima) are
// enqueued on the model's stream and captured in its CUDA graph. A rank that never arrives would leave the others'
// collective kernels waiting; the host bounds every wait on a step (tp_wait) and aborts the communicator past it,
// which ends those kernels.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "common.cuh"
#include "internal.h"

namespace agxc {

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  std::string why;
};

const NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      a.why = std::string("libnccl.so.2 not loadable: ") + (e ? e : "?");
      return;
    }
    auto sym = [&](const char* name) -> void* {
      void* p = dlsym(h, name);
      if (!p && a.why.empty()) a.why = std::string("libnccl lacks ") + name;
      return p;
    };
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(sym("ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(sym("ncclCommInitRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(sym("ncclAllReduce"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(sym("ncclAllGather"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(sym("ncclCommDestroy"));
    a.comm_abort = reinterpret_cast<decltype(a.comm_abort)>(sym("ncclCommAbort"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(sym("ncclGetErrorString"));
    a.ok = a.why.empty();
  });
  return a;
}

int nccl_fail(ncclResult_t r, const char* what) {
  const NcclApi& a = api();
  return fail(AGXC_ENCCL, std::string(what) + ": " + (a.error_string ? a.error_string(r) : "nccl error") +
                              " (" + std::to_string(static_cast<int>(r)) + ")");
}

}  // namespace

struct TpComm {
  ncclComm_t comm = nullptr;
  int world = 1, rank = 0;
  bool aborted = false;
};

int tp_unique_id(void* out) {
  const NcclApi& a = api();
  if (!a.ok) return fail(AGXC_EUNSUPPORTED, a.why);
  ncclUniqueId id;
  if (ncclResult_t r = a.get_unique_id(&id)) return nccl_fail(r, "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == 128, "communicator id is 128 bytes");
  std::memcpy(out, &id, sizeof(id));
  return 0;
}

int tp_comm_create(int world, int rank, const void* id, TpComm** out) {
  const NcclApi& a = api();
  if (!a.ok) return fail(AGXC_EUNSUPPORTED, a.why);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  TpComm* c = new TpComm();
  c->world = world;
  c->rank = rank;
  if (ncclResult_t r = a.comm_init_rank(&c->comm, world, uid, rank)) {
    delete c;
    return nccl_fail(r, "ncclCommInitRank");
  }
  *out = c;
  return 0;
}

void tp_comm_free(TpComm* c) {
  if (!c) return;
  const NcclApi& a = api();
  if (c->comm) (c->aborted ? ncclSuccess : a.comm_destroy(c->comm));
  delete c;
}

int tp_allreduce_f32(TpComm* c, float* buf, size_t n, cudaStream_t s) {
  if (c->aborted) return fail(AGXC_ENCCL, "tensor parallel: the communicator was aborted");
  if (ncclResult_t r = api().all_reduce(buf, buf, n, ncclFloat32, ncclSum, c->comm, s))
    return nccl_fail(r, "ncclAllReduce");
  return 0;
}

int tp_allgather_u32(TpComm* c, const uint32_t* send, uint32_t* recv, size_t n, cudaStream_t s) {
  if (c->aborted) return fail(AGXC_ENCCL, "tensor parallel: the communicator was aborted");
  if (ncclResult_t r = api().all_gather(send, recv, n, ncclUint32, c->comm, s)) return nccl_fail(r, "ncclAllGather");
  return 0;
}

int tp_wait(TpComm* c, cudaEvent_t done, int timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaEventQuery(done);
    if (e == cudaSuccess) return 0;
    if (e != cudaErrorNotReady) return cuda_fail(e, "tensor parallel: step wait");
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > timeout_ms) {
      if (c && c->comm && !c->aborted) {
        api().comm_abort(c->comm);  // ends this rank's collective kernels still waiting for a peer
        c->aborted = true;
      }
      return fail(AGXC_ETIMEOUT, "tensor parallel: a step did not complete within " + std::to_string(timeout_ms) +
                                     " ms (a peer rank is missing); the communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace agxc

extern "C" int agxc_tp_unique_id(void* id128) {
  if (!id128) return agxc::fail(AGXC_EINVAL, "tp_unique_id: null buffer");
  return agxc::tp_unique_id(id128);
}
