// shard_comm.h — NCCL communicator for the sample-sharded mode.
//
// In the sample-sharded mode every rank (one process per GPU) holds the whole population but
// only a slice of the samples. After each fused evaluation pass the per-tree sums (JtJ, Jtr,
// sum r^2) are all-reduced over NVLink, so every rank solves the same normal equations and
// takes the same steps; outputs are identical on every rank.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the library PyTorch or the system
// provides), so the engine loads where NCCL is absent and only this mode needs it. The
// communicator is non-blocking: every wait is bounded by a deadline, after which the
// communicator is aborted and the call returns CO_ERR_CUDA instead of hanging on a missing
// or failed peer.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>
#include <stddef.h>

namespace cusr {

struct ShardComm {
    ncclComm_t comm = nullptr;
    int nranks = 1, rank = 0;
    double timeout_s = 120.0;
    bool failed = false;
};

// 128-byte unique id for a new group (one rank creates it and shares it). CO_* code.
int shard_unique_id(unsigned char out[NCCL_UNIQUE_ID_BYTES]);
// Join the group on the current device. CO_* code.
int shard_init(ShardComm &sc, const unsigned char id[NCCL_UNIQUE_ID_BYTES], int nranks,
               int rank, double timeout_s);
// In-place sum all-reduce of `count` elements (float or double) on `stream`. CO_* code.
int shard_allreduce(ShardComm &sc, void *buf, size_t count, bool fp64, cudaStream_t stream);
// Wait for `ev` with the group's deadline, watching the communicator for errors. CO_* code.
int shard_wait_event(ShardComm &sc, cudaEvent_t ev);
void shard_destroy(ShardComm &sc);

}  // namespace cusr
