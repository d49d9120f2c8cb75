// Tensor-parallel groups: one NCCL communicator per rank, created from an id
// the ranks share, and the in-place all-gather the sharded session runs after
// every row-sharded op. The reference runs one process; its D1 contract
// (tests/sdk/llama_threads.cpp:32: any thread count gives the one-thread
// bits) is what the row sharding keeps across GPUs.
#include <cuda_runtime.h>
#include <nccl.h>

#include <cstring>
#include <string>

#include "../internal.h"
#include "synapse_b200.h"

struct syn_tp {
    int rank = 0, world = 1, device = 0;
    ncclComm_t comm = nullptr;
};

namespace {

int nccl(ncclResult_t r) {
    if (r == ncclSuccess) return SYN_OK;
    syn_set_error((std::string("nccl: ") + ncclGetErrorString(r)).c_str());
    return SYN_ERR_NCCL;
}

}  // namespace

void syn_tp_info(const syn_tp* tp, int* rank, int* world, int* device) {
    if (rank) *rank = tp ? tp->rank : 0;
    if (world) *world = tp ? tp->world : 1;
    if (device) *device = tp ? tp->device : -1;
}

static_assert(sizeof(ncclUniqueId) == SYN_TP_ID_BYTES, "SYN_TP_ID_BYTES is an ncclUniqueId");

extern "C" int syn_tp_unique_id(void* id_out) {
    if (!id_out) return SYN_ERR_INVALID;
    ncclUniqueId id;
    const int rc = nccl(ncclGetUniqueId(&id));
    if (!rc) std::memcpy(id_out, &id, sizeof id);
    return rc;
}

extern "C" int syn_tp_init(int rank, int world, const void* id, int device, syn_tp** out) {
    if (!id || !out || world < 1 || rank < 0 || rank >= world || device < 0) return SYN_ERR_INVALID;
    *out = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) {
        syn_set_error(cudaGetErrorString(cudaGetLastError()));
        return SYN_ERR_CUDA;
    }
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof u);
    syn_tp* tp = new syn_tp();
    tp->rank = rank;
    tp->world = world;
    tp->device = device;
    // Blocking init: it returns once every rank has joined (the caller's
    // launcher bounds how long ranks wait for one another).
    const int rc = nccl(ncclCommInitRank(&tp->comm, world, u, rank));
    if (rc) {
        delete tp;
        return rc;
    }
    *out = tp;
    return SYN_OK;
}

extern "C" void syn_tp_close(syn_tp* tp) {
    if (!tp) return;
    cudaSetDevice(tp->device);
    if (tp->comm) ncclCommDestroy(tp->comm);
    delete tp;
}

extern "C" int syn_allgather(syn_tp* tp, void* buf, size_t bytes_per_rank, void* stream) {
    if (!tp || !buf || !bytes_per_rank) return SYN_ERR_INVALID;
    char* b = static_cast<char*>(buf);
    return nccl(ncclAllGather(b + size_t(tp->rank) * bytes_per_rank, b, bytes_per_rank, ncclUint8, tp->comm,
                              static_cast<cudaStream_t>(stream)));
}

// Host bytes of every rank, gathered through the communicator on a private
// stream (a few hundred bytes at set-up: IPC handles).
int syn_tp_exchange(syn_tp* tp, const void* mine, void* all, size_t bytes) {
    if (!tp || !mine || !all || !bytes) return SYN_ERR_INVALID;
    if (cudaSetDevice(tp->device) != cudaSuccess) return SYN_ERR_CUDA;
    cudaStream_t st = nullptr;
    char* buf = nullptr;
    const size_t total = bytes * size_t(tp->world);
    int rc = SYN_OK;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&buf, total) != cudaSuccess ||
        cudaMemcpy(buf + bytes * size_t(tp->rank), mine, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        syn_set_error(cudaGetErrorString(cudaGetLastError()));
        rc = SYN_ERR_CUDA;
    }
    if (!rc) rc = nccl(ncclAllGather(buf + bytes * size_t(tp->rank), buf, bytes, ncclUint8, tp->comm, st));
    if (!rc && (cudaStreamSynchronize(st) != cudaSuccess || cudaMemcpy(all, buf, total, cudaMemcpyDeviceToHost) != cudaSuccess)) {
        syn_set_error(cudaGetErrorString(cudaGetLastError()));
        rc = SYN_ERR_CUDA;
    }
    if (buf) cudaFree(buf);
    if (st) cudaStreamDestroy(st);
    return rc;
}

int syn_tp_barrier(syn_tp* tp) {
    if (!tp) return SYN_ERR_INVALID;
    const int one = 1;
    std::string all(sizeof one * size_t(tp->world), '\0');
    return syn_tp_exchange(tp, &one, all.data(), sizeof one);
}
