// Shared device helpers for the sm_100a decode path.
//
// Every file is compiled with --fmad=false: the reference builds with
// -ffp-contract=off (cmake/numerics.cmake:13), so a*b+c stays two roundings
// unless the code asks for fmaf() where the reference calls fma().
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/synapse_b200.h"

namespace syn {

constexpr int QK = 32;  // weights per Q4_0 / Q8_0 block (quant/blocks.hpp:31)

__host__ __device__ constexpr size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// ---- Q8_0 activation planes (see syn_q8_act_bytes) -------------------------
struct ActPlanes {
    int8_t* qs;      // [n_tok][cols]
    uint16_t* dh;    // [n_tok][nb] binary16 scale bits
    float* d;        // [n_tok][nb] decoded scale
    int32_t* sum;    // [n_tok][nb] sum of the block's quants
};

__host__ __device__ inline size_t act_qs_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * cols); }
__host__ __device__ inline size_t act_dh_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * (cols / QK) * 2); }
__host__ __device__ inline size_t act_d_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * (cols / QK) * 4); }

__host__ __device__ inline ActPlanes act_planes(void* act, int n_tok, int cols) {
    char* p = static_cast<char*>(act);
    ActPlanes a;
    a.qs = reinterpret_cast<int8_t*>(p);
    p += act_qs_bytes(n_tok, cols);
    a.dh = reinterpret_cast<uint16_t*>(p);
    p += act_dh_bytes(n_tok, cols);
    a.d = reinterpret_cast<float*>(p);
    p += act_d_bytes(n_tok, cols);
    a.sum = reinterpret_cast<int32_t*>(p);
    return a;
}

__host__ __device__ inline size_t act_bytes(int n_tok, int cols) {
    return act_qs_bytes(n_tok, cols) + act_dh_bytes(n_tok, cols) + 2 * act_d_bytes(n_tok, cols);
}

// ---- planar weight planes ----------------------------------------------------
__host__ __device__ inline int quant_bytes_per_block(int type) { return type == SYN_Q4_0 ? 16 : 32; }
__host__ __device__ inline int gguf_block_bytes(int type) { return type == SYN_Q4_0 ? 18 : 34; }
__host__ __device__ inline size_t planar_qs_bytes(int type, int rows, int cols) {
    return align256(size_t(rows) * (cols / QK) * quant_bytes_per_block(type));
}

// ---- binary16 ---------------------------------------------------------------
__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ uint16_t f16_bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
__device__ __forceinline__ float f16_from_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---- Q8_0 block quantizer: one block of 32 values, one per lane --------------
// quant/q8.hpp:54-69: amax, d = amax / 127 (float), id = d ? 1/d : 0 with the
// unrounded d, q = roundf(x * id), d stored as binary16 (RNE). IEEE division
// and round-half-away roundf make it bit-identical to the reference.
struct Q8Lane {
    int8_t q;
    uint16_t dh;
    float d;
    int32_t sum;
};

__device__ __forceinline__ Q8Lane quantize_q8_lane(float x) {
    const float ax = fabsf(x);
    // |x| as bits orders like the floats (non-negative); NaN inputs are outside
    // the reference's domain as well.
    const uint32_t amax_bits = __reduce_max_sync(0xffffffffu, __float_as_uint(ax));
    const float amax = __uint_as_float(amax_bits);
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    Q8Lane r;
    r.q = static_cast<int8_t>(roundf(__fmul_rn(x, id)));
    r.dh = f16_bits(d);
    r.d = f16_from_bits(r.dh);
    r.sum = __reduce_add_sync(0xffffffffu, static_cast<int>(r.q));
    return r;
}

// expf rounded once from double precision: the correctly rounded float in all
// but vanishingly rare cases, the closest a float result can be to the C
// runtime's expf that the reference calls (std::exp on float).
__device__ __forceinline__ float exp_rn(float x) { return float(exp(double(x))); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---- programmatic dependent launch ---------------------------------------
// griddepcontrol.wait: block until the grids this one depends on have
// completed and their memory is visible (a no-op without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// griddepcontrol.launch_dependents: let the next grid in the stream start
// its prologue early.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// L2 prefetch of [p, p + bytes) (16-byte aligned, bytes a multiple of 16) by
// the bulk-copy unit: weights the kernel will stream, requested before it
// waits on the previous kernel.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    if (bytes >= 16)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes & ~15u) : "memory");
}

}  // namespace syn

// Host-side error plumbing shared by the .cu files (defined in capi.cu).
int syn_cuda_status(cudaError_t e);
int syn_check_launch();
int syn_num_sms();
// Programmatic dependent launch for this thread's launches (the session turns
// it on while it enqueues a step; plain C-ABI calls launch without it).
int syn_pdl_enabled();
void syn_set_pdl(int on);

// Launch with the PDL attribute when enabled. Every kernel of this library
// calls griddepcontrol.wait before it reads a predecessor's output or writes
// any output, so a kernel may only start early, never read early.
template <typename... KArgs, typename... Args>
int syn_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (syn_pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return syn_cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}
