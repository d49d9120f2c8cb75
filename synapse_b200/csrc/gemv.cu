// mul_mat for decode: Y[t][r] = W[r,:] . X[t,:] (kernels/gemm.hpp:143-230,
// kernels/gemv.hpp:149-161).
//
// Quantized weights (Q4_0, Q8_0) meet Q8_0 activations. Each 32-weight
// block's dot is an exact integer -- four / eight dp4a per block, Q4_0's "- 8"
// folded out as 8 * (sum of the activation block's quants) -- exactly as the
// reference computes it (kernels/dot.hpp:103-164).
//
// The float accumulation reproduces the reference's order bit for bit in its
// portable configuration (dot.hpp:268-322, :398, :426): within each chunk of
// 32 blocks, acc = fma(float(isum_b), d_w*d_a, acc) in block order; the row
// result is ((0 + chunk_0) + chunk_1) + ... So the GPU output equals the
// oracle's exactly, and no 8-bit activation rounding downstream can flip
// because of a GEMV. The kernel streams the weights coalesced -- a warp takes
// one row, lane l the blocks l, l+32, ... (one 16/32-byte load each) -- and
// puts each block's (isum, scale) in shared memory; then one lane per chunk
// runs that chunk's fma chain, and one lane per token adds the chunks.
//
// Rows are split in contiguous ranges over a persistent grid (SMs x resident
// CTAs), so every SM streams the same number of bytes.
#include "common.cuh"

#include <algorithm>

using namespace syn;

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
// A whole row of per-block results is staged when it fits this budget per
// warp; otherwise one 32-block chunk at a time.
constexpr size_t kRowStageBytes = 16 * 1024;

struct GemvArgs {
    const uint8_t* w;    // GGUF rows, or the quant plane (planar)
    const uint16_t* dh;  // planar scale plane (planar only)
    int rows, cols, nb, n_tok;
    ActPlanes act;
    float* y;
    const float* residual;
};

// Block b of row r: its quants as 32-bit words and its decoded scale.
template <int TYPE, int LAYOUT>
__device__ __forceinline__ void load_block(const GemvArgs& p, int r, int b, uint32_t (&w)[8], float& dw) {
    const size_t i = size_t(r) * p.nb + b;
    if (LAYOUT == SYN_LAYOUT_PLANAR) {
        if (TYPE == SYN_Q4_0) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.w) + i);
            w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
        } else {
            const uint4* q = reinterpret_cast<const uint4*>(p.w) + 2 * i;
            const uint4 v0 = __ldg(q), v1 = __ldg(q + 1);
            w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w;
            w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
        }
        dw = f16_from_bits(__ldg(p.dh + i));
    } else {
        // GGUF AoS: 18 / 34-byte blocks, 2-byte aligned.
        const uint16_t* s = reinterpret_cast<const uint16_t*>(p.w + i * gguf_block_bytes(TYPE));
        dw = f16_from_bits(__ldg(s));
        constexpr int words = TYPE == SYN_Q4_0 ? 4 : 8;
#pragma unroll
        for (int k = 0; k < words; ++k) w[k] = uint32_t(__ldg(s + 1 + 2 * k)) | (uint32_t(__ldg(s + 2 + 2 * k)) << 16);
    }
}

template <int TYPE>
__device__ __forceinline__ int block_dot(const uint32_t (&w)[8], const int4 a0, const int4 a1, int asum) {
    int s = 0;
    if (TYPE == SYN_Q4_0) {
        // byte j: low nibble = weight j, high nibble = weight j + 16 (blocks.hpp:36-40)
        s = __dp4a(int(w[0] & 0x0f0f0f0fu), a0.x, s);
        s = __dp4a(int(w[1] & 0x0f0f0f0fu), a0.y, s);
        s = __dp4a(int(w[2] & 0x0f0f0f0fu), a0.z, s);
        s = __dp4a(int(w[3] & 0x0f0f0f0fu), a0.w, s);
        s = __dp4a(int((w[0] >> 4) & 0x0f0f0f0fu), a1.x, s);
        s = __dp4a(int((w[1] >> 4) & 0x0f0f0f0fu), a1.y, s);
        s = __dp4a(int((w[2] >> 4) & 0x0f0f0f0fu), a1.z, s);
        s = __dp4a(int((w[3] >> 4) & 0x0f0f0f0fu), a1.w, s);
        s -= 8 * asum;
    } else {
        s = __dp4a(int(w[0]), a0.x, s);
        s = __dp4a(int(w[1]), a0.y, s);
        s = __dp4a(int(w[2]), a0.z, s);
        s = __dp4a(int(w[3]), a0.w, s);
        s = __dp4a(int(w[4]), a1.x, s);
        s = __dp4a(int(w[5]), a1.y, s);
        s = __dp4a(int(w[6]), a1.z, s);
        s = __dp4a(int(w[7]), a1.w, s);
    }
    return s;
}

// Per warp shared memory: (isum, scale) per token per staged block (block b at
// index b + b/32, so the chunk chains of different lanes hit different banks),
// then one float per token per chunk.
__host__ __device__ inline int staged_blocks(int nb, bool whole_row) { return whole_row ? nb + nb / 32 : 33; }
// Rounded to 16 bytes so every warp's float2 staging area stays aligned.
__host__ __device__ inline size_t warp_stage_bytes(int nb, int nt, bool whole_row) {
    const int nch = (nb + 31) / 32;
    const size_t b = size_t(nt) * staged_blocks(nb, whole_row) * 8 + size_t(nt) * nch * 4;
    return (b + 15) & ~size_t(15);
}

// Warp w of W takes rows [rows*w/W, rows*(w+1)/W).
__device__ __forceinline__ void warp_rows(int rows, int& r0, int& r1) {
    const long gw = long(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const long nw = long(gridDim.x) * (blockDim.x >> 5);
    r0 = int(long(rows) * gw / nw);
    r1 = int(long(rows) * (gw + 1) / nw);
}

template <int TYPE, int LAYOUT, int NT, bool WHOLE_ROW>
__global__ void __launch_bounds__(kThreads) gemv_q_kernel(GemvArgs p) {
    extern __shared__ float2 stage_all[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = p.nb, nch = (nb + 31) / 32;
    const int SB = staged_blocks(nb, WHOLE_ROW);
    float2* stage = reinterpret_cast<float2*>(reinterpret_cast<char*>(stage_all) + warp * warp_stage_bytes(nb, NT, WHOLE_ROW));
    float* chunk_sum = reinterpret_cast<float*>(stage + NT * SB);
    int r0, r1;
    warp_rows(p.rows, r0, r1);
    pdl_launch_dependents();
    pdl_wait();  // activations (and the residual) come from the previous kernel

    for (int r = r0; r < r1; ++r) {
        float y[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) y[t] = 0.0f;
        const int c_end = WHOLE_ROW ? 1 : nch;
        for (int c = 0; c < c_end; ++c) {
            const int b_begin = WHOLE_ROW ? 0 : c * 32, b_end = WHOLE_ROW ? nb : min(nb, c * 32 + 32);
#pragma unroll 4
            for (int b = b_begin + lane; b < b_end; b += 32) {
                uint32_t w[8];
                float dw;
                load_block<TYPE, LAYOUT>(p, r, b, w, dw);
                const int sb = WHOLE_ROW ? b + (b >> 5) : b - b_begin;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const int4* aq = reinterpret_cast<const int4*>(p.act.qs + size_t(t) * p.cols + size_t(b) * QK);
                    const int4 a0 = __ldg(aq), a1 = __ldg(aq + 1);
                    const int asum = TYPE == SYN_Q4_0 ? __ldg(p.act.sum + size_t(t) * nb + b) : 0;
                    const int isum = block_dot<TYPE>(w, a0, a1, asum);
                    const float da = __ldg(p.act.d + size_t(t) * nb + b);
                    stage[t * SB + sb] = make_float2(float(isum), __fmul_rn(dw, da));
                }
            }
            __syncwarp();
            if (WHOLE_ROW) {
                // one lane per (token, chunk): the chunk's fma chain in block order
                for (int k = lane; k < NT * nch; k += 32) {
                    const int t = k / nch, ch = k % nch;
                    const float2* s = stage + t * SB + ch * 33;
                    const int n = min(32, nb - ch * 32);
                    float acc = 0.0f;
                    for (int i = 0; i < n; ++i) acc = fmaf(s[i].x, s[i].y, acc);
                    chunk_sum[t * nch + ch] = acc;
                }
                __syncwarp();
                if (lane < NT) {
                    float v = 0.0f;
                    for (int ch = 0; ch < nch; ++ch) v = __fadd_rn(v, chunk_sum[lane * nch + ch]);
#pragma unroll
                    for (int t = 0; t < NT; ++t)
                        if (t == lane) y[t] = v;
                }
            } else {
                if (lane < NT) {
                    const float2* s = stage + lane * SB;
                    const int n = b_end - b_begin;
                    float acc = 0.0f;
                    for (int i = 0; i < n; ++i) acc = fmaf(s[i].x, s[i].y, acc);
#pragma unroll
                    for (int t = 0; t < NT; ++t)
                        if (t == lane) y[t] = __fadd_rn(y[t], acc);
                }
            }
            __syncwarp();
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (lane == t) {
                const size_t o = size_t(t) * p.rows + r;
                p.y[o] = p.residual ? __fadd_rn(y[t], p.residual[o]) : y[t];
            }
        }
    }
}

// Plain F32 / F16 rows with float activations (dot.hpp:404-433), in the
// oracle's order: chunks of 256 columns; within a chunk eight lanes of fma
// (lane l over columns l, l+8, ...), reduced pairwise (4 then 2 then 1),
// plus a ragged tail in order; chunks added in order. One warp per row: lane
// group g (lanes 8g..8g+7) takes chunks g, g+4, ...
template <int TYPE, int NT>
__global__ void __launch_bounds__(kThreads) gemv_f_kernel(const void* __restrict__ wv, int rows, int cols,
                                                          const float* __restrict__ x, float* y,
                                                          const float* residual) {
    extern __shared__ float chunk_all[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nch = (cols + 255) / 256;
    float* chunk_sum = chunk_all + size_t(warp) * NT * nch;
    const int g = lane >> 3, l = lane & 7;
    int r0, r1;
    warp_rows(rows, r0, r1);
    pdl_launch_dependents();
    pdl_wait();
    for (int r = r0; r < r1; ++r) {
        for (int ch0 = 0; ch0 < nch; ch0 += 4) {
            const int ch = ch0 + g;
            const int c0 = ch * 256, len = ch < nch ? min(256, cols - c0) : 0;
            const int full = len / 8 * 8;
            float acc[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
            for (int j = l; j < full; j += 8) {
                const size_t wi = size_t(r) * cols + c0 + j;
                const float wf = TYPE == SYN_F32 ? __ldg(static_cast<const float*>(wv) + wi)
                                                 : f16_from_bits(__ldg(static_cast<const uint16_t*>(wv) + wi));
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[t] = fmaf(wf, __ldg(x + size_t(t) * cols + c0 + j), acc[t]);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                float v = acc[t];
                // pairwise: lane l + (l + 4), then + 2, then + 1, within the group of 8
                v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 8));
                v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 8));
                v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 8));
                if (l == 0 && ch < nch) {
                    for (int j = full; j < len; ++j) {
                        const size_t wi = size_t(r) * cols + c0 + j;
                        const float wf = TYPE == SYN_F32
                                             ? __ldg(static_cast<const float*>(wv) + wi)
                                             : f16_from_bits(__ldg(static_cast<const uint16_t*>(wv) + wi));
                        v = __fadd_rn(v, __fmul_rn(wf, __ldg(x + size_t(t) * cols + c0 + j)));
                    }
                    chunk_sum[t * nch + ch] = v;
                }
            }
        }
        __syncwarp();
        if (lane < NT) {
            float v = 0.0f;
            for (int ch = 0; ch < nch; ++ch) v = __fadd_rn(v, chunk_sum[lane * nch + ch]);
            const size_t o = size_t(lane) * rows + r;
            y[o] = residual ? __fadd_rn(v, residual[o]) : v;
        }
        __syncwarp();
    }
}

// Persistent grid: SMs x resident CTAs (from the occupancy of this kernel and
// shared memory size), capped by the work.
template <typename K>
int persistent_grid(K kernel, size_t smem, long work_warps) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const long want = (work_warps + kWarps - 1) / kWarps;
    const long cap = long(syn_num_sms()) * per_sm;
    return int(std::max<long>(1, std::min(want, cap)));
}

template <typename K>
int configure(K kernel, size_t smem) {
    if (smem > 48 * 1024)
        return syn_cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    return SYN_OK;
}

template <int TYPE, int LAYOUT, int NT>
int launch_q(const GemvArgs& p, cudaStream_t s) {
    const bool whole = warp_stage_bytes(p.nb, NT, true) <= kRowStageBytes;
    const size_t smem = size_t(kWarps) * warp_stage_bytes(p.nb, NT, whole);
    if (whole) {
        auto k = gemv_q_kernel<TYPE, LAYOUT, NT, true>;
        int st = configure(k, smem);
        if (st) return st;
        return syn_launch(k, persistent_grid(k, smem, p.rows), kThreads, smem, s, p);
    }
    auto k = gemv_q_kernel<TYPE, LAYOUT, NT, false>;
    int st = configure(k, smem);
    if (st) return st;
    return syn_launch(k, persistent_grid(k, smem, p.rows), kThreads, smem, s, p);
}

template <int TYPE, int LAYOUT>
int dispatch_q(const GemvArgs& p, int n, cudaStream_t s) {
    switch (n) {
    case 1: return launch_q<TYPE, LAYOUT, 1>(p, s);
    case 2: return launch_q<TYPE, LAYOUT, 2>(p, s);
    case 3: return launch_q<TYPE, LAYOUT, 3>(p, s);
    case 4: return launch_q<TYPE, LAYOUT, 4>(p, s);
    case 5: return launch_q<TYPE, LAYOUT, 5>(p, s);
    case 6: return launch_q<TYPE, LAYOUT, 6>(p, s);
    case 7: return launch_q<TYPE, LAYOUT, 7>(p, s);
    case 8: return launch_q<TYPE, LAYOUT, 8>(p, s);
    }
    return SYN_ERR_INVALID;
}

template <int TYPE, int NT>
int launch_f(const void* w, int rows, int cols, const float* x, float* y, const float* res, cudaStream_t s) {
    const size_t smem = size_t(kWarps) * NT * ((cols + 255) / 256) * 4;
    auto k = gemv_f_kernel<TYPE, NT>;
    int st = configure(k, smem);
    if (st) return st;
    return syn_launch(k, persistent_grid(k, smem, rows), kThreads, smem, s, w, rows, cols, x, y, res);
}

template <int TYPE>
int dispatch_f(const void* w, int rows, int cols, const float* x, int n, float* y, const float* res, cudaStream_t s) {
    switch (n) {
    case 1: return launch_f<TYPE, 1>(w, rows, cols, x, y, res, s);
    case 2: return launch_f<TYPE, 2>(w, rows, cols, x, y, res, s);
    case 3: return launch_f<TYPE, 3>(w, rows, cols, x, y, res, s);
    case 4: return launch_f<TYPE, 4>(w, rows, cols, x, y, res, s);
    case 5: return launch_f<TYPE, 5>(w, rows, cols, x, y, res, s);
    case 6: return launch_f<TYPE, 6>(w, rows, cols, x, y, res, s);
    case 7: return launch_f<TYPE, 7>(w, rows, cols, x, y, res, s);
    case 8: return launch_f<TYPE, 8>(w, rows, cols, x, y, res, s);
    }
    return SYN_ERR_INVALID;
}

}  // namespace

extern "C" int syn_gemv_q(int type, const void* w, int layout, int rows, int cols, const void* act, int n_tok,
                          float* y, const float* residual, void* stream) {
    if (type != SYN_Q4_0 && type != SYN_Q8_0) return SYN_ERR_UNSUPPORTED;
    if (layout != SYN_LAYOUT_GGUF && layout != SYN_LAYOUT_PLANAR) return SYN_ERR_INVALID;
    if (!w || !act || !y || rows <= 0 || cols <= 0 || cols % QK || n_tok <= 0) return SYN_ERR_INVALID;
    if (layout == SYN_LAYOUT_PLANAR && (reinterpret_cast<uintptr_t>(w) & 15)) return SYN_ERR_INVALID;
    if (layout == SYN_LAYOUT_GGUF && (reinterpret_cast<uintptr_t>(w) & 1)) return SYN_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(act) & 15) return SYN_ERR_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const ActPlanes all = act_planes(const_cast<void*>(act), n_tok, cols);
    const int nb = cols / QK;
    for (int t0 = 0; t0 < n_tok; t0 += 8) {
        const int n = n_tok - t0 < 8 ? n_tok - t0 : 8;
        GemvArgs p;
        p.w = static_cast<const uint8_t*>(w);
        p.dh = layout == SYN_LAYOUT_PLANAR
                   ? reinterpret_cast<const uint16_t*>(p.w + planar_qs_bytes(type, rows, cols))
                   : nullptr;
        p.rows = rows;
        p.cols = cols;
        p.nb = nb;
        p.n_tok = n;
        p.act.qs = all.qs + size_t(t0) * cols;
        p.act.dh = all.dh + size_t(t0) * nb;
        p.act.d = all.d + size_t(t0) * nb;
        p.act.sum = all.sum + size_t(t0) * nb;
        p.y = y + size_t(t0) * rows;
        p.residual = residual ? residual + size_t(t0) * rows : nullptr;
        int st;
        if (type == SYN_Q4_0)
            st = layout == SYN_LAYOUT_PLANAR ? dispatch_q<SYN_Q4_0, SYN_LAYOUT_PLANAR>(p, n, s)
                                             : dispatch_q<SYN_Q4_0, SYN_LAYOUT_GGUF>(p, n, s);
        else
            st = layout == SYN_LAYOUT_PLANAR ? dispatch_q<SYN_Q8_0, SYN_LAYOUT_PLANAR>(p, n, s)
                                             : dispatch_q<SYN_Q8_0, SYN_LAYOUT_GGUF>(p, n, s);
        if (st) return st;
    }
    return SYN_OK;
}

extern "C" int syn_gemv_f(int type, const void* w, int rows, int cols, const float* x, int n_tok, float* y,
                          const float* residual, void* stream) {
    if (type != SYN_F32 && type != SYN_F16) return SYN_ERR_UNSUPPORTED;
    if (!w || !x || !y || rows <= 0 || cols <= 0 || n_tok <= 0) return SYN_ERR_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int t0 = 0; t0 < n_tok; t0 += 8) {
        const int n = n_tok - t0 < 8 ? n_tok - t0 : 8;
        const float* xr = x + size_t(t0) * cols;
        float* yr = y + size_t(t0) * rows;
        const float* rr = residual ? residual + size_t(t0) * rows : nullptr;
        const int st = type == SYN_F32 ? dispatch_f<SYN_F32>(w, rows, cols, xr, n, yr, rr, s)
                                       : dispatch_f<SYN_F16>(w, rows, cols, xr, n, yr, rr, s);
        if (st) return st;
    }
    return SYN_OK;
}
