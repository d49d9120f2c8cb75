// mul_mat for decode: Y[t][r] = W[r,:] . X[t,:] (kernels/gemm.hpp:143-230,
// kernels/gemv.hpp:149-161).
//
// Quantized weights (Q4_0, Q8_0) meet Q8_0 activations. As in the reference
// (kernels/dot.hpp:103-164, :268-322), each 32-weight block's dot is an exact
// integer -- here four / eight dp4a per block -- and is accumulated in float
// as fmaf(float(isum), d_w * d_a, acc). Q4_0's "- 8" is folded out of the
// inner loop as 8 * (sum of the activation block's quants), which keeps the
// integer result identical. Only the float accumulation order across blocks
// differs from the reference (lanes over blocks, then a warp tree).
//
// The kernel is a bandwidth-bound stream: one warp per output row (grid-
// stride), each lane taking blocks lane, lane+32, ...; the planar layout makes
// a warp's 16-byte quant loads one contiguous 512-byte run per row step.
#include "common.cuh"

using namespace syn;

namespace {

struct GemvArgs {
    const uint8_t* w;    // GGUF rows, or the quant plane (planar)
    const uint16_t* dh;  // planar scale plane (planar only)
    int rows, cols, nb;
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

template <int TYPE, int LAYOUT, int NT>
__global__ void __launch_bounds__(256) gemv_q_kernel(GemvArgs p) {
    const int lane = threadIdx.x & 31;
    const int warp = int((size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    const int nwarps = int((size_t(gridDim.x) * blockDim.x) >> 5);
    for (int r = warp; r < p.rows; r += nwarps) {
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
#pragma unroll 4
        for (int b = lane; b < p.nb; b += 32) {
            uint32_t w[8];
            float dw;
            load_block<TYPE, LAYOUT>(p, r, b, w, dw);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int4* aq = reinterpret_cast<const int4*>(p.act.qs + size_t(t) * p.cols + size_t(b) * QK);
                const int4 a0 = __ldg(aq), a1 = __ldg(aq + 1);
                const int asum = TYPE == SYN_Q4_0 ? __ldg(p.act.sum + size_t(t) * p.nb + b) : 0;
                const int isum = block_dot<TYPE>(w, a0, a1, asum);
                const float da = __ldg(p.act.d + size_t(t) * p.nb + b);
                acc[t] = fmaf(float(isum), dw * da, acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float v = warp_sum(acc[t]);
            if (lane == 0) {
                const size_t o = size_t(t) * p.rows + r;
                p.y[o] = p.residual ? v + p.residual[o] : v;
            }
        }
    }
}

// Plain F32 / F16 rows with float activations (dot.hpp:404-433).
template <int TYPE, int NT>
__global__ void __launch_bounds__(256) gemv_f_kernel(const void* __restrict__ wv, int rows, int cols,
                                                     const float* __restrict__ x, float* y,
                                                     const float* residual) {
    const int lane = threadIdx.x & 31;
    const int warp = int((size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    const int nwarps = int((size_t(gridDim.x) * blockDim.x) >> 5);
    const bool vec = (cols & 3) == 0;
    for (int r = warp; r < rows; r += nwarps) {
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        int c0 = 0;
        if (vec) {
            for (int c = lane * 4; c < cols; c += 128) {
                float wf[4];
                if (TYPE == SYN_F32) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(wv) +
                                                                           size_t(r) * cols + c));
                    wf[0] = v.x; wf[1] = v.y; wf[2] = v.z; wf[3] = v.w;
                } else {
                    const uint2 v = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(wv) +
                                                                         size_t(r) * cols + c));
                    wf[0] = f16_from_bits(v.x & 0xffff); wf[1] = f16_from_bits(v.x >> 16);
                    wf[2] = f16_from_bits(v.y & 0xffff); wf[3] = f16_from_bits(v.y >> 16);
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const float4 xv = __ldg(reinterpret_cast<const float4*>(x + size_t(t) * cols + c));
                    acc[t] = fmaf(wf[0], xv.x, acc[t]);
                    acc[t] = fmaf(wf[1], xv.y, acc[t]);
                    acc[t] = fmaf(wf[2], xv.z, acc[t]);
                    acc[t] = fmaf(wf[3], xv.w, acc[t]);
                }
            }
            c0 = cols;
        }
        for (int c = c0 + lane; c < cols; c += 32) {
            const float wf = TYPE == SYN_F32 ? __ldg(static_cast<const float*>(wv) + size_t(r) * cols + c)
                                             : f16_from_bits(__ldg(static_cast<const uint16_t*>(wv) +
                                                                   size_t(r) * cols + c));
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] = fmaf(wf, __ldg(x + size_t(t) * cols + c), acc[t]);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float v = warp_sum(acc[t]);
            if (lane == 0) {
                const size_t o = size_t(t) * rows + r;
                y[o] = residual ? v + residual[o] : v;
            }
        }
    }
}

int grid_for_rows(int rows) {
    const long want = (long(rows) * 32 + 255) / 256;
    const long cap = long(syn_num_sms()) * 8;
    return int(want < cap ? want : cap);
}

template <int TYPE, int LAYOUT>
int launch_q(GemvArgs p, int n, cudaStream_t s) {
    const int grid = grid_for_rows(p.rows);
    switch (n) {
#define SYN_CASE(N) \
    case N: gemv_q_kernel<TYPE, LAYOUT, N><<<grid, 256, 0, s>>>(p); break;
        SYN_CASE(1) SYN_CASE(2) SYN_CASE(3) SYN_CASE(4) SYN_CASE(5) SYN_CASE(6) SYN_CASE(7) SYN_CASE(8)
#undef SYN_CASE
    default: return SYN_ERR_INVALID;
    }
    return syn_check_launch();
}

template <int TYPE>
int launch_f(const void* w, int rows, int cols, const float* x, int n, float* y, const float* res, cudaStream_t s) {
    const int grid = grid_for_rows(rows);
    switch (n) {
#define SYN_CASE(N) \
    case N: gemv_f_kernel<TYPE, N><<<grid, 256, 0, s>>>(w, rows, cols, x, y, res); break;
        SYN_CASE(1) SYN_CASE(2) SYN_CASE(3) SYN_CASE(4) SYN_CASE(5) SYN_CASE(6) SYN_CASE(7) SYN_CASE(8)
#undef SYN_CASE
    default: return SYN_ERR_INVALID;
    }
    return syn_check_launch();
}

}  // namespace

extern "C" int syn_gemv_q(int type, const void* w, int layout, int rows, int cols, const void* act, int n_tok,
                          float* y, const float* residual, void* stream) {
    if (type != SYN_Q4_0 && type != SYN_Q8_0) return SYN_ERR_UNSUPPORTED;
    if (layout != SYN_LAYOUT_GGUF && layout != SYN_LAYOUT_PLANAR) return SYN_ERR_INVALID;
    if (!w || !act || !y || rows <= 0 || cols <= 0 || cols % QK || n_tok <= 0) return SYN_ERR_INVALID;
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
        p.act.qs = all.qs + size_t(t0) * cols;
        p.act.dh = all.dh + size_t(t0) * nb;
        p.act.d = all.d + size_t(t0) * nb;
        p.act.sum = all.sum + size_t(t0) * nb;
        p.y = y + size_t(t0) * rows;
        p.residual = residual ? residual + size_t(t0) * rows : nullptr;
        int st;
        if (type == SYN_Q4_0)
            st = layout == SYN_LAYOUT_PLANAR ? launch_q<SYN_Q4_0, SYN_LAYOUT_PLANAR>(p, n, s)
                                             : launch_q<SYN_Q4_0, SYN_LAYOUT_GGUF>(p, n, s);
        else
            st = layout == SYN_LAYOUT_PLANAR ? launch_q<SYN_Q8_0, SYN_LAYOUT_PLANAR>(p, n, s)
                                             : launch_q<SYN_Q8_0, SYN_LAYOUT_GGUF>(p, n, s);
        if (st) return st;
    }
    return SYN_OK;
}

extern "C" int syn_gemv_f(int type, const void* w, int rows, int cols, const float* x, int n_tok, float* y,
                          const float* residual, void* stream) {
    if (type != SYN_F32 && type != SYN_F16) return SYN_ERR_UNSUPPORTED;
    if (!w || !x || !y || rows <= 0 || cols <= 0 || n_tok <= 0) return SYN_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15) return SYN_ERR_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int t0 = 0; t0 < n_tok; t0 += 8) {
        const int n = n_tok - t0 < 8 ? n_tok - t0 : 8;
        const float* xr = x + size_t(t0) * cols;
        float* yr = y + size_t(t0) * rows;
        const float* rr = residual ? residual + size_t(t0) * rows : nullptr;
        const int st = type == SYN_F32 ? launch_f<SYN_F32>(w, rows, cols, xr, n, yr, rr, s)
                                       : launch_f<SYN_F16>(w, rows, cols, xr, n, yr, rr, s);
        if (st) return st;
    }
    return SYN_OK;
}
