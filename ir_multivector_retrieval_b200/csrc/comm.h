// comm.h — NCCL communicator of a context (one process per GPU).
//
// NCCL is loaded at run time (dlopen "libnccl.so.2"): single-GPU entry
// points do not depend on it, and inside a PyTorch process the library that
// PyTorch already loaded is the one used. All collectives are enqueued on the
// context stream.
#pragma once
#include <cstddef>
#include <cstdint>

#include "mvr_internal.h"

namespace mvr {

struct Comm;  // opaque; owned by Ctx

bool comm_active(const Ctx* ctx);
int comm_rank(const Ctx* ctx);
int comm_size(const Ctx* ctx);
void destroy_comm(Ctx* ctx);

// recv = concat over ranks of each rank's `bytes` from send
int comm_allgather(Ctx* ctx, const void* send, void* recv, size_t bytes);
// in-place sum of `count` u32
int comm_allreduce_sum_u32(Ctx* ctx, uint32_t* buf, size_t count);
// in-place max of `count` u64
int comm_allreduce_max_u64(Ctx* ctx, uint64_t* buf, size_t count);
int comm_broadcast(Ctx* ctx, void* buf, size_t bytes, int root);
int comm_send(Ctx* ctx, const void* buf, size_t bytes, int peer);
int comm_recv(Ctx* ctx, void* buf, size_t bytes, int peer);
// bracket point-to-point calls that must progress together (an exchange)
int comm_group_start(Ctx* ctx);
int comm_group_end(Ctx* ctx);

}  // namespace mvr
