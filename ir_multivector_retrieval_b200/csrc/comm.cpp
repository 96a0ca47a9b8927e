// comm.cpp — NCCL plumbing of a context; see comm.h.
#include "comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

namespace mvr {
namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.why = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    auto sym = [&](const char* n) { return dlsym(h, n); };
    a.GetUniqueId = (decltype(a.GetUniqueId))sym("ncclGetUniqueId");
    a.CommInitRank = (decltype(a.CommInitRank))sym("ncclCommInitRank");
    a.CommDestroy = (decltype(a.CommDestroy))sym("ncclCommDestroy");
    a.AllGather = (decltype(a.AllGather))sym("ncclAllGather");
    a.AllReduce = (decltype(a.AllReduce))sym("ncclAllReduce");
    a.Broadcast = (decltype(a.Broadcast))sym("ncclBroadcast");
    a.Send = (decltype(a.Send))sym("ncclSend");
    a.Recv = (decltype(a.Recv))sym("ncclRecv");
    a.GetErrorString = (decltype(a.GetErrorString))sym("ncclGetErrorString");
    a.GroupStart = (decltype(a.GroupStart))sym("ncclGroupStart");
    a.GroupEnd = (decltype(a.GroupEnd))sym("ncclGroupEnd");
    a.ok = a.GetUniqueId && a.CommInitRank && a.CommDestroy && a.AllGather && a.AllReduce && a.Broadcast &&
           a.Send && a.Recv && a.GetErrorString && a.GroupStart && a.GroupEnd;
    if (!a.ok) a.why = "libnccl.so.2 lacks a required symbol";
  });
  return a;
}

int nccl_fail(Ctx* ctx, ncclResult_t r, const char* what) {
  return fail(ctx, MVR_E_NCCL, std::string(what) + ": " + api().GetErrorString(r));
}

#define MVR_NCCL(ctx, call)                                  \
  do {                                                       \
    ncclResult_t _r = (call);                                \
    if (_r != ncclSuccess) return nccl_fail((ctx), _r, #call); \
  } while (0)

}  // namespace

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, size = 1;
};

bool comm_active(const Ctx* ctx) { return ctx && ctx->comm && ctx->comm->size > 1; }
int comm_rank(const Ctx* ctx) { return ctx && ctx->comm ? ctx->comm->rank : 0; }
int comm_size(const Ctx* ctx) { return ctx && ctx->comm ? ctx->comm->size : 1; }

void destroy_comm(Ctx* ctx) {
  if (!ctx->comm) return;
  if (ctx->comm->comm && api().ok) api().CommDestroy(ctx->comm->comm);
  delete ctx->comm;
  ctx->comm = nullptr;
}

int comm_allgather(Ctx* ctx, const void* send, void* recv, size_t bytes) {
  MVR_NCCL(ctx, api().AllGather(send, recv, bytes, ncclUint8, ctx->comm->comm, ctx->stream));
  return MVR_OK;
}
int comm_allreduce_sum_u32(Ctx* ctx, uint32_t* buf, size_t count) {
  MVR_NCCL(ctx, api().AllReduce(buf, buf, count, ncclUint32, ncclSum, ctx->comm->comm, ctx->stream));
  return MVR_OK;
}
int comm_allreduce_max_u64(Ctx* ctx, uint64_t* buf, size_t count) {
  MVR_NCCL(ctx, api().AllReduce(buf, buf, count, ncclUint64, ncclMax, ctx->comm->comm, ctx->stream));
  return MVR_OK;
}
int comm_broadcast(Ctx* ctx, void* buf, size_t bytes, int root) {
  MVR_NCCL(ctx, api().Broadcast(buf, buf, bytes, ncclUint8, root, ctx->comm->comm, ctx->stream));
  return MVR_OK;
}
int comm_send(Ctx* ctx, const void* buf, size_t bytes, int peer) {
  MVR_NCCL(ctx, api().Send(buf, bytes, ncclUint8, peer, ctx->comm->comm, ctx->stream));
  return MVR_OK;
}
int comm_recv(Ctx* ctx, void* buf, size_t bytes, int peer) {
  MVR_NCCL(ctx, api().Recv(buf, bytes, ncclUint8, peer, ctx->comm->comm, ctx->stream));
  return MVR_OK;
}
int comm_group_start(Ctx* ctx) {
  MVR_NCCL(ctx, api().GroupStart());
  return MVR_OK;
}
int comm_group_end(Ctx* ctx) {
  MVR_NCCL(ctx, api().GroupEnd());
  return MVR_OK;
}

}  // namespace mvr

using mvr::Ctx;

extern "C" {

int mvr_comm_unique_id(void* id_out, size_t id_bytes) {
  const auto& a = mvr::api();
  if (!id_out || id_bytes < sizeof(ncclUniqueId)) return MVR_E_INVALID_ARGUMENT;
  if (!a.ok) return MVR_E_NCCL;
  ncclUniqueId id;
  if (a.GetUniqueId(&id) != ncclSuccess) return MVR_E_NCCL;
  std::memcpy(id_out, &id, sizeof(id));
  return MVR_OK;
}

size_t mvr_comm_unique_id_bytes(void) { return sizeof(ncclUniqueId); }

int mvr_ctx_init_comm(mvr_ctx* h, int nranks, int rank, const void* id, size_t id_bytes) {
  if (!h || !id || id_bytes < sizeof(ncclUniqueId) || nranks < 1 || rank < 0 || rank >= nranks)
    return MVR_E_INVALID_ARGUMENT;
  Ctx* c = &h->impl;
  const auto& a = mvr::api();
  if (!a.ok) return mvr::fail(c, MVR_E_NCCL, a.why);
  mvr::destroy_comm(c);
  mvr::DeviceScope dev_scope(c);  // NCCL binds the communicator to the current device
  if (dev_scope.status != MVR_OK) return dev_scope.status;
  auto* cm = new (std::nothrow) mvr::Comm;
  if (!cm) return MVR_E_OUT_OF_MEMORY;
  cm->rank = rank;
  cm->size = nranks;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  const ncclResult_t r = a.CommInitRank(&cm->comm, nranks, uid, rank);
  if (r != ncclSuccess) {
    delete cm;
    return mvr::fail(c, MVR_E_NCCL, std::string("ncclCommInitRank: ") + a.GetErrorString(r));
  }
  c->comm = cm;
  return MVR_OK;
}

int mvr_ctx_comm_size(const mvr_ctx* h) { return h ? mvr::comm_size(&h->impl) : 0; }
int mvr_ctx_comm_rank(const mvr_ctx* h) { return h ? mvr::comm_rank(&h->impl) : 0; }

}  // extern "C"
