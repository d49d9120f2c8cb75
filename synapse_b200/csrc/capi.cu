// Status plumbing of the C ABI: CUDA errors become syn_status values and the
// message is kept per thread for syn_last_error().
#include "common.cuh"

#include <cstdio>
#include <cstring>

namespace {
thread_local char g_last_error[256] = "";
thread_local int g_pdl = 0;
}

int syn_pdl_enabled() { return g_pdl; }
void syn_set_pdl(int on) { g_pdl = on; }
// For microbenchmarks that capture kernels as the session does.
extern "C" void syn_set_programmatic_launch(int on) { g_pdl = on; }

int syn_cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return SYN_OK;
    std::snprintf(g_last_error, sizeof g_last_error, "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? SYN_ERR_NO_MEMORY : SYN_ERR_CUDA;
}

int syn_check_launch() { return syn_cuda_status(cudaGetLastError()); }

void syn_set_error(const char* msg) { std::snprintf(g_last_error, sizeof g_last_error, "%s", msg); }

int syn_num_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

extern "C" const char* syn_build_info(void) { return "synapse_b200 0.1 sm_100a"; }

extern "C" const char* syn_last_error(void) { return g_last_error; }

extern "C" const char* syn_status_string(int status) {
    switch (status) {
    case SYN_OK: return "ok";
    case SYN_ERR_INVALID: return "invalid argument";
    case SYN_ERR_UNSUPPORTED: return "unsupported";
    case SYN_ERR_CUDA: return "cuda error";
    case SYN_ERR_NO_MEMORY: return "out of device memory";
    case SYN_ERR_TIMEOUT: return "timeout";
    case SYN_ERR_NCCL: return "nccl error";
    case SYN_ERR_FORMAT: return "bad format";
    case SYN_ERR_RANGE: return "out of range";
    default: return "unknown";
    }
}
