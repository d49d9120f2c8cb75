// Q8_0 activation quantizer and the weight repack the loader runs.
//
// syn_quantize_q8_0 replaces quantize_row_q8_0 (quant/q8.hpp:54-69) as
// prepare_activations calls it (kernels/gemv.hpp:72-116): one warp per
// 32-value block, bit-identical quants and binary16 scales, plus the decoded
// float scale and the block's quant sum that the GEMV consumes.
#include "common.cuh"
#include "internal.h"

#include <algorithm>

using namespace syn;

namespace {

__global__ void __launch_bounds__(256) quantize_q8_kernel(const float* __restrict__ x, int n_tok, int cols,
                                                          ActPlanes a) {
    pdl_launch_dependents();
    pdl_wait();
    const int nb = cols / QK;
    const long blk = (long(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (blk >= long(n_tok) * nb) return;
    const long t = blk / nb, b = blk % nb;
    const float v = x[t * cols + b * QK + lane];
    const Q8Lane r = quantize_q8_lane(v);
    a.qs[t * cols + b * QK + lane] = r.q;
    if (lane == 0) {
        a.dh[blk] = r.dh;
        a.d[blk] = r.d;
        a.sum[blk] = r.sum;
    }
}

__global__ void act_to_blocks_kernel(ActPlanes a, int n_tok, int cols, uint8_t* __restrict__ out) {
    const int nb = cols / QK;
    const long blk = long(blockIdx.x) * blockDim.x + threadIdx.x;
    if (blk >= long(n_tok) * nb) return;
    const long t = blk / nb, b = blk % nb;
    uint8_t* o = out + blk * 34;
    o[0] = a.dh[blk] & 0xff;
    o[1] = a.dh[blk] >> 8;
    for (int j = 0; j < QK; ++j) o[2 + j] = static_cast<uint8_t>(a.qs[t * cols + b * QK + j]);
}

// GGUF blocks [rows*nb] (18 / 34 B) -> quant plane (16 / 32 B per block) and
// binary16 scale plane. One thread per block; a one-time loader pass.
// GGUF blocks of rows [row0, row0 + rows) -> the planar matrix at dst (one
// thread per block; a one-time loader pass).
__global__ void repack_rows_kernel(int type, const uint8_t* __restrict__ src, int rows, int cols, uint8_t* dst,
                                   int row0, int row_step) {
    const int nb = cols / QK;
    const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= long(rows) * nb) return;
    const int bb = gguf_block_bytes(type), qb = quant_bytes_per_block(type);
    const uint8_t* s = src + i * bb;
    const size_t r = size_t(row0) + size_t(i / nb) * row_step, b = size_t(i % nb);
    uint8_t* q = dst + planar_quant_at(type, cols, r, b);
    for (int j = 0; j < qb; ++j) q[j] = s[2 + j];
    uint8_t* d = dst + planar_scale_at(type, cols, r, b);
    d[0] = s[0];
    d[1] = s[1];
}

// ---- seeded synthetic weights ---------------------------------------------
// A counter-based generator: splitmix64 of (seed, tensor, index) gives two
// uniforms, Box-Muller one normal. Independent of the launch shape.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t tensor, uint64_t idx) {
    const uint64_t h = mix64(seed ^ mix64(tensor * 0x100000001b3ull ^ mix64(idx)));
    const float u1 = (float(uint32_t(h >> 40)) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = float(uint32_t(h & 0xffffffu)) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// One thread per 32-weight block: generate, then ggml's reference quantizer
// (quantize_row_q4_0_ref / quantize_row_q8_0_ref; quant/q8.hpp:54-69).
__global__ void fill_random_q_kernel(int type, int rows, int cols, uint8_t* dst, int row0, int row_step,
                                     uint64_t seed, uint64_t tensor, float sigma, uint64_t first_block) {
    const int nb = cols / QK;
    const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= long(rows) * nb) return;
    float x[QK];
    float amax = 0.0f, mx = 0.0f;
    for (int j = 0; j < QK; ++j) {
        x[j] = __fmul_rn(normal_at(seed, tensor, (first_block + uint64_t(i)) * QK + j), sigma);
        const float a = fabsf(x[j]);
        if (amax < a) { amax = a; mx = x[j]; }
    }
    const size_t r = size_t(row0) + size_t(i / nb) * row_step, b = size_t(i % nb);
    uint16_t* dh = reinterpret_cast<uint16_t*>(dst + planar_scale_at(type, cols, r, b));
    if (type == SYN_Q4_0) {
        const float d = __fdiv_rn(mx, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        *dh = f16_bits(d);
        uint8_t* q = dst + planar_quant_at(type, cols, r, b);
        for (int j = 0; j < 16; ++j) {
            int lo = int(int8_t(__fadd_rn(__fmul_rn(x[j], id), 8.5f)));
            int hi = int(int8_t(__fadd_rn(__fmul_rn(x[16 + j], id), 8.5f)));
            lo = lo > 15 ? 15 : lo;
            hi = hi > 15 ? 15 : hi;
            q[j] = uint8_t(lo | (hi << 4));
        }
    } else {
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        *dh = f16_bits(d);
        int8_t* q = reinterpret_cast<int8_t*>(dst + planar_quant_at(type, cols, r, b));
        for (int j = 0; j < QK; ++j) q[j] = int8_t(roundf(__fmul_rn(x[j], id)));
    }
}

__global__ void fill_random_f_kernel(int type, size_t n, void* dst, uint64_t seed, uint64_t tensor, float sigma,
                                     uint64_t first) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        const float v = __fmul_rn(normal_at(seed, tensor, first + i), sigma);
        if (type == SYN_F32) static_cast<float*>(dst)[i] = v;
        else static_cast<uint16_t*>(dst)[i] = f16_bits(v);
    }
}

__global__ void fill_f32_kernel(float* dst, size_t n, float v) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        dst[i] = v;
}

bool quant_type(int type) { return type == SYN_Q4_0 || type == SYN_Q8_0; }

}  // namespace

int syn_planar_block_pos(int nb, size_t r, int b) { return planar_block_pos(nb, r, b); }

int syn_repack_rows(int type, const void* src, int rows, int cols, void* dst, int total_rows, int row0,
                    cudaStream_t s, int row_step) {
    if (!quant_type(type)) return SYN_ERR_UNSUPPORTED;
    if (row0 < 0 || row_step < 1 || long(row0) + long(rows - 1) * row_step >= total_rows) return SYN_ERR_INVALID;
    const long n = long(rows) * (cols / QK);
    repack_rows_kernel<<<(n + 255) / 256, 256, 0, s>>>(type, static_cast<const uint8_t*>(src), rows, cols,
                                                        static_cast<uint8_t*>(dst), row0, row_step);
    return syn_check_launch();
}

int syn_fill_random(int type, int rows, int cols, void* dst, int total_rows, int row0, uint64_t seed,
                    uint64_t tensor, float sigma, cudaStream_t s, int row_step, long first_row) {
    if (first_row < 0) return SYN_ERR_INVALID;
    if (quant_type(type)) {
        if (row0 < 0 || row_step < 1 || long(row0) + long(rows - 1) * row_step >= total_rows) return SYN_ERR_INVALID;
        const long n = long(rows) * (cols / QK);
        fill_random_q_kernel<<<(n + 127) / 128, 128, 0, s>>>(type, rows, cols, static_cast<uint8_t*>(dst), row0,
                                                              row_step, seed, tensor, sigma,
                                                              uint64_t(first_row) * (cols / QK));
    } else if (type == SYN_F32 || type == SYN_F16) {
        if (row0 < 0 || row_step != 1 || long(row0) + rows > total_rows) return SYN_ERR_INVALID;
        char* d = static_cast<char*>(dst) + size_t(row0) * cols * (type == SYN_F32 ? 4 : 2);
        fill_random_f_kernel<<<4096, 256, 0, s>>>(type, size_t(rows) * cols, d, seed, tensor, sigma,
                                                  uint64_t(first_row) * cols);
    } else {
        return SYN_ERR_UNSUPPORTED;
    }
    return syn_check_launch();
}

// Benchmark helper: a whole planar matrix of seeded N(0, 0.02) weights.
extern "C" int syn_fill_random_planar(int type, int rows, int cols, void* dst, uint64_t seed, void* stream) {
    if (!quant_type(type) || !dst || rows <= 0 || cols <= 0 || cols % QK) return SYN_ERR_INVALID;
    return syn_fill_random(type, rows, cols, dst, rows, 0, seed, 1, 0.02f, static_cast<cudaStream_t>(stream));
}

int syn_fill_f32(float* dst, size_t n, float v, cudaStream_t s) {
    fill_f32_kernel<<<(n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096, 256, 0, s>>>(dst, n, v);
    return syn_check_launch();
}

extern "C" size_t syn_q8_act_bytes(int n_tok, int cols) {
    if (n_tok <= 0 || cols <= 0 || cols % QK) return 0;
    return act_bytes(n_tok, cols);
}

extern "C" int syn_quantize_q8_0(const float* x, int n_tok, int cols, void* act, void* stream) {
    if (!x || !act || n_tok <= 0 || cols <= 0 || cols % QK) return SYN_ERR_INVALID;
    const long warps = long(n_tok) * (cols / QK);
    const int threads = 256;
    const long grid = (warps * 32 + threads - 1) / threads;
    return syn_launch(quantize_q8_kernel, unsigned(grid), threads, 0, static_cast<cudaStream_t>(stream), x, n_tok,
                      cols, act_planes(act, n_tok, cols));
}

extern "C" int syn_q8_act_to_blocks(const void* act, int n_tok, int cols, void* blocks, void* stream) {
    if (!act || !blocks || n_tok <= 0 || cols <= 0 || cols % QK) return SYN_ERR_INVALID;
    const long n = long(n_tok) * (cols / QK);
    act_to_blocks_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        act_planes(const_cast<void*>(act), n_tok, cols), n_tok, cols, static_cast<uint8_t*>(blocks));
    return syn_check_launch();
}

extern "C" size_t syn_weight_bytes(int type, int rows, int cols, int layout) {
    if (rows <= 0 || cols <= 0) return 0;
    switch (type) {
    case SYN_F32: return size_t(rows) * cols * 4;
    case SYN_F16: return size_t(rows) * cols * 2;
    case SYN_Q4_0:
    case SYN_Q8_0:
        if (cols % QK) return 0;
        if (layout == SYN_LAYOUT_GGUF) return size_t(rows) * (cols / QK) * gguf_block_bytes(type);
        return size_t(rows) * planar_row_bytes(type, cols);
    case SYN_Q4_K:
    case SYN_Q6_K: return syn_k_weight_bytes(type, rows, cols, layout);
    default: return 0;
    }
}

extern "C" int syn_repack_planar(int type, const void* src, int rows, int cols, void* dst, void* stream) {
    if (syn_k_type(type)) {
        if (!src || !dst || rows <= 0 || cols <= 0 || cols % 256) return SYN_ERR_INVALID;
        return syn_k_repack_rows(type, src, rows, cols, dst, static_cast<cudaStream_t>(stream));
    }
    if (!quant_type(type)) return SYN_ERR_UNSUPPORTED;
    if (!src || !dst || rows <= 0 || cols <= 0 || cols % QK) return SYN_ERR_INVALID;
    return syn_repack_rows(type, src, rows, cols, dst, rows, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int syn_upload_weight(int type, const void* host_src, int rows, int cols, void* dst, int layout,
                                 void* staging, size_t staging_bytes, void* stream) {
    if (!host_src || !dst || rows <= 0 || cols <= 0) return SYN_ERR_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t total = syn_weight_bytes(type, rows, cols, SYN_LAYOUT_GGUF);
    if (total == 0) return SYN_ERR_UNSUPPORTED;
    if ((!quant_type(type) && !syn_k_type(type)) || layout == SYN_LAYOUT_GGUF || type == SYN_Q4_K) {
        int st = syn_cuda_status(cudaMemcpyAsync(dst, host_src, total, cudaMemcpyHostToDevice, s));
        if (st) return st;
        return syn_cuda_status(cudaStreamSynchronize(s));
    }
    if (!staging || staging_bytes < (1u << 20)) return SYN_ERR_INVALID;
    if (syn_k_type(type)) {  // Q6_K: rows through the staging buffer, repacked into place
        const size_t row_g = total / size_t(rows), row_p = syn_k_weight_bytes(type, 1, cols, SYN_LAYOUT_PLANAR);
        if (row_g > staging_bytes) return SYN_ERR_INVALID;
        const int per = int(std::min<size_t>(size_t(rows), staging_bytes / row_g));
        const uint8_t* h = static_cast<const uint8_t*>(host_src);
        for (int r0 = 0; r0 < rows; r0 += per) {
            const int n = rows - r0 < per ? rows - r0 : per;
            int st = syn_cuda_status(cudaMemcpyAsync(staging, h + size_t(r0) * row_g, size_t(n) * row_g,
                                                     cudaMemcpyHostToDevice, s));
            if (st) return st;
            if ((st = syn_k_repack_rows(type, staging, n, cols, static_cast<uint8_t*>(dst) + size_t(r0) * row_p, s)))
                return st;
            if ((st = syn_cuda_status(cudaStreamSynchronize(s)))) return st;
        }
        return SYN_OK;
    }
    const size_t row_b = size_t(cols / QK) * gguf_block_bytes(type);
    const int per = int(std::max<size_t>(1, staging_bytes / row_b));
    if (row_b > staging_bytes) return SYN_ERR_INVALID;
    const uint8_t* h = static_cast<const uint8_t*>(host_src);
    for (int r0 = 0; r0 < rows; r0 += per) {
        const int n = rows - r0 < per ? rows - r0 : per;
        int st = syn_cuda_status(cudaMemcpyAsync(staging, h + size_t(r0) * row_b, size_t(n) * row_b,
                                                 cudaMemcpyHostToDevice, s));
        if (st) return st;
        if ((st = syn_repack_rows(type, staging, n, cols, dst, rows, r0, s))) return st;
        if ((st = syn_cuda_status(cudaStreamSynchronize(s)))) return st;
    }
    return SYN_OK;
}
