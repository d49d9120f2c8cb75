// Pieces of the one-token GEMV (gemv.cu): the exact block dot, the in-kernel Q8_0 quantization
// of the input (with or without rms_norm), and the staged batch: lane-parallel
// block dots staged in shared memory, then one fma chain per 32-block chunk in
// the reference's order, then the row sums.
#pragma once

#include "common.cuh"

namespace syn {

constexpr int kStageWarps = 8;
constexpr size_t kBatchBytes = 9728;  // target bytes of weights per batch

// dp4a of unsigned bytes (a) with signed bytes (b), plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <int TYPE>
__device__ __forceinline__ int block_dot(const uint32_t (&w)[8], const int4 a0, const int4 a1, int asum) {
    // two independent dp4a chains (an exact integer sum in any order)
    int s0 = 0, s1 = 0;
    if (TYPE == SYN_Q4_0) {
        // byte j: low nibble = weight j, high nibble = weight j + 16 (blocks.hpp:36-40).
        // The high nibbles stay in place (16 x their value), so s1 = 16 * their dot.
        s0 = __dp4a(int(w[0] & 0x0f0f0f0fu), a0.x, s0);
        s1 = dp4a_us(w[0] & 0xf0f0f0f0u, a1.x, s1);
        s0 = __dp4a(int(w[1] & 0x0f0f0f0fu), a0.y, s0);
        s1 = dp4a_us(w[1] & 0xf0f0f0f0u, a1.y, s1);
        s0 = __dp4a(int(w[2] & 0x0f0f0f0fu), a0.z, s0);
        s1 = dp4a_us(w[2] & 0xf0f0f0f0u, a1.z, s1);
        s0 = __dp4a(int(w[3] & 0x0f0f0f0fu), a0.w, s0);
        s1 = dp4a_us(w[3] & 0xf0f0f0f0u, a1.w, s1);
        return s0 + (s1 >> 4) - 8 * asum;  // s1 is a multiple of 16: the shift is exact
    }
    s0 = __dp4a(int(w[0]), a0.x, s0);
    s1 = __dp4a(int(w[4]), a1.x, s1);
    s0 = __dp4a(int(w[1]), a0.y, s0);
    s1 = __dp4a(int(w[5]), a1.y, s1);
    s0 = __dp4a(int(w[2]), a0.z, s0);
    s1 = __dp4a(int(w[6]), a1.z, s1);
    s0 = __dp4a(int(w[3]), a0.w, s0);
    s1 = __dp4a(int(w[7]), a1.w, s1);
    return s0 + s1;
}

__host__ __device__ inline size_t a16(size_t n) { return (n + 15) & ~size_t(15); }
__host__ __device__ inline size_t act_pad_off(int b) { return size_t(b) * QK + size_t(b >> 3) * 16; }
__host__ __device__ inline size_t act_pad_stride(int nb) { return a16(act_pad_off(nb)); }
// The staged kernel's activation layout: 16 bytes of padding after every 4 blocks.
__host__ __device__ inline size_t sact_off(int b) { return size_t(b) * QK + size_t(b >> 2) * 16; }
// Shared memory of the lane kernel: NT padded quant rows, then (d, sum) per token and block.
__host__ __device__ inline size_t lane_act_bytes(int nt, int nb) {
    return size_t(nt) * act_pad_stride(nb) + size_t(nt) * nb * 8;
}

// The activations made in the kernel: every CTA quantizes the float input
// (SYN_IN_F32), or its rms_norm (SYN_IN_RMSNORM), into shared memory with the
// exact arithmetic of syn_quantize_q8_0 / syn_rms_norm (quant/q8.hpp:54-69,
// elementwise.hpp:208-232), one 32-value block per thread.
// LAYOUT 1: the lane kernel's (16 bytes after every 8 blocks); 2: the staged
// kernel's (16 bytes after every 4 blocks).
// Every thread of the block calls it (it synchronizes the block).
template <int NT, int LAYOUT = 1>
__device__ void quantize_act(const float* x, const float* gamma, float eps, bool norm, int cols, uint8_t* aq,
                             float2* dsum) {
    __shared__ double red[NT * 32];
    __shared__ float scale_t[NT];
    const int nb = cols / QK, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t stride = act_pad_stride(nb);
    if (norm) {
        // Sum of squares per token: each thread's blocks with all eight
        // 16-byte loads of a block in flight at once, then one block reduction.
        double part[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) part[t] = 0.0;
        for (int blk = threadIdx.x; blk < NT * nb; blk += blockDim.x) {
            const int t = blk / nb, b = blk % nb;
            const float4* src = reinterpret_cast<const float4*>(x + size_t(t) * cols + size_t(b) * QK);
            float4 f[QK / 4];
#pragma unroll
            for (int k = 0; k < QK / 4; ++k) f[k] = src[k];
            double sum = 0.0;
#pragma unroll
            for (int k = 0; k < QK / 4; ++k) {
                sum += double(__fmul_rn(f[k].x, f[k].x));
                sum += double(__fmul_rn(f[k].y, f[k].y));
                sum += double(__fmul_rn(f[k].z, f[k].z));
                sum += double(__fmul_rn(f[k].w, f[k].w));
            }
#pragma unroll
            for (int tt = 0; tt < NT; ++tt)
                if (tt == t) part[tt] += sum;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const double w = warp_sum_d(part[t]);
            if (lane == 0) red[t * 32 + warp] = w;
        }
        __syncthreads();
        if (threadIdx.x < NT) {
            double tot = 0.0;
            for (int w = 0; w < int(blockDim.x >> 5); ++w) tot += red[threadIdx.x * 32 + w];
            const float mean = float(tot / double(cols));
            scale_t[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        }
        __syncthreads();
    }
    // Quantize one block per thread in two passes over its 32 values (the
    // second reads them again from L1), so few registers stay live.
    for (int blk = threadIdx.x; blk < NT * nb; blk += blockDim.x) {
        const int t = blk / nb, b = blk % nb;
        const float4* src = reinterpret_cast<const float4*>(x + size_t(t) * cols + size_t(b) * QK);
        const float4* g4 = reinterpret_cast<const float4*>(gamma + size_t(b) * QK);
        const float sc = norm ? scale_t[t] : 1.0f;
        auto value = [&](float x, float g) { return norm ? __fmul_rn(__fmul_rn(x, sc), g) : x; };
        float amax = 0.0f;
#pragma unroll
        for (int k = 0; k < QK / 4; ++k) {
            const float4 f = src[k];
            const float4 g = norm ? __ldg(g4 + k) : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
            amax = fmaxf(amax, fabsf(value(f.x, g.x)));
            amax = fmaxf(amax, fabsf(value(f.y, g.y)));
            amax = fmaxf(amax, fabsf(value(f.z, g.z)));
            amax = fmaxf(amax, fabsf(value(f.w, g.w)));
        }
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int qsum = 0;
        uint32_t* dst = reinterpret_cast<uint32_t*>(aq + size_t(t) * stride +
                                                    (LAYOUT == 1 ? act_pad_off(b) : sact_off(b)));
#pragma unroll
        for (int k = 0; k < QK / 4; ++k) {
            const float4 f = src[k];
            const float4 g = norm ? __ldg(g4 + k) : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
            const int q0 = int(roundf(__fmul_rn(value(f.x, g.x), id)));
            const int q1 = int(roundf(__fmul_rn(value(f.y, g.y), id)));
            const int q2 = int(roundf(__fmul_rn(value(f.z, g.z), id)));
            const int q3 = int(roundf(__fmul_rn(value(f.w, g.w), id)));
            qsum += q0 + q1 + q2 + q3;
            dst[k] = (uint32_t(q0) & 0xffu) | ((uint32_t(q1) & 0xffu) << 8) | ((uint32_t(q2) & 0xffu) << 16) |
                     ((uint32_t(q3) & 0xffu) << 24);
        }
        dsum[t * nb + b] = make_float2(f16_from_bits(f16_bits(d)), __int_as_float(qsum));
    }
}

// One token's input quantized into the staged layout by the whole block: each
// thread takes 16-value halves of blocks (lanes 2k, 2k+1 form one block, so the
// block's amax and sum meet by one shuffle), the loads of up to two halves in
// flight at once.
// The same arithmetic as quantize_act: rms_norm (double sum of float squares,
// mean, 1 / sqrt(mean + eps), (x * scale) * gamma), then quant/q8.hpp:54-69.
// Every thread of the block calls it (it synchronizes the block).
// WORDS: x is a gathered vector of tensor-parallel words ({float, epoch},
// TpSync); each value is read once its word carries this step's epoch.
template <bool WORDS = false>
__device__ inline void quantize_act1(const float* x, const float* gamma, float eps, bool norm, int cols, uint8_t* aq,
                              float2* dsum, const TpSync* tp = nullptr, unsigned epoch = 0,
                              const float4* gamma_first = nullptr) {
    __shared__ double red[32];
    constexpr int kIt = 2;  // half-blocks per thread whose loads are in flight together
    const int nh = cols / 16, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nt = int(blockDim.x);
    // the 16 values of half-block h
    auto load16 = [&](int h, float (&v)[16]) {
        if constexpr (WORDS) {
            tp_load_n(*tp, reinterpret_cast<const uint64_t*>(x) + size_t(h) * 16, epoch, v);
        } else {
            const float4* src = reinterpret_cast<const float4*>(x + size_t(h) * 16);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 f = src[k];
                v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
            }
        }
    };
    float scale = 1.0f;
    if (norm) {
        // thread t sums its half-blocks t, t + nt, ... in that order
        double sum = 0.0;
        for (int h0 = 0; h0 < nh; h0 += kIt * nt) {
            float v[kIt][16];
#pragma unroll
            for (int i = 0; i < kIt; ++i)
                if (h0 + i * nt + int(threadIdx.x) < nh) load16(h0 + i * nt + int(threadIdx.x), v[i]);
#pragma unroll
            for (int i = 0; i < kIt; ++i)
                if (h0 + i * nt + int(threadIdx.x) < nh) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) sum += double(__fmul_rn(v[i][j], v[i][j]));
                }
        }
        sum = warp_sum_d(sum);
        if (lane == 0) red[warp] = sum;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < int(blockDim.x >> 5); ++w) tot += red[w];
        const float mean = float(tot / double(cols));
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    for (int h0 = 0; h0 < nh; h0 += kIt * nt) {
        float vv[kIt][16];
#pragma unroll
        for (int i = 0; i < kIt; ++i)
            if (h0 + i * nt + int(threadIdx.x) < nh) load16(h0 + i * nt + int(threadIdx.x), vv[i]);
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
            const int hp = h0 + i * nt, h = hp + int(threadIdx.x);
            // lanes of this pass (a prefix of the warp; block pairs never straddle it)
            const int live = min(32, max(0, nh - (hp + warp * 32)));
            if (h >= nh) continue;
            const unsigned mask = live == 32 ? 0xffffffffu : ((1u << live) - 1u);
            float* v = vv[i];
            if (norm) {
                const float4* g4 = reinterpret_cast<const float4*>(gamma + size_t(h) * 16);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    // the first half-block's gamma may have been read before the kernel's wait
                    const float4 g = gamma_first && h == int(threadIdx.x) ? gamma_first[k] : __ldg(g4 + k);
                    v[4 * k] = __fmul_rn(__fmul_rn(v[4 * k], scale), g.x);
                    v[4 * k + 1] = __fmul_rn(__fmul_rn(v[4 * k + 1], scale), g.y);
                    v[4 * k + 2] = __fmul_rn(__fmul_rn(v[4 * k + 2], scale), g.z);
                    v[4 * k + 3] = __fmul_rn(__fmul_rn(v[4 * k + 3], scale), g.w);
                }
            }
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
            amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 1));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            int qsum = 0;
            uint32_t packed[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int q0 = int(roundf(__fmul_rn(v[4 * k], id)));
                const int q1 = int(roundf(__fmul_rn(v[4 * k + 1], id)));
                const int q2 = int(roundf(__fmul_rn(v[4 * k + 2], id)));
                const int q3 = int(roundf(__fmul_rn(v[4 * k + 3], id)));
                qsum += q0 + q1 + q2 + q3;
                packed[k] = (uint32_t(q0) & 0xffu) | ((uint32_t(q1) & 0xffu) << 8) | ((uint32_t(q2) & 0xffu) << 16) |
                            ((uint32_t(q3) & 0xffu) << 24);
            }
            qsum += __shfl_xor_sync(mask, qsum, 1);
            const int b = h >> 1;
            *reinterpret_cast<uint4*>(aq + sact_off(b) + 16 * (h & 1)) =
                make_uint4(packed[0], packed[1], packed[2], packed[3]);
            if ((h & 1) == 0) dsum[b] = make_float2(f16_from_bits(f16_bits(d)), __int_as_float(qsum));
        }
    }
}

struct StageShape {
    int nb, nch, R;                          // blocks, chunks per row; rows per batch
    size_t row_b, batch_bytes, act_bytes, stage_floats2, warp_bytes, smem;
};

__host__ __device__ inline StageShape stage_shape(int type, int cols, int warps = kStageWarps,
                                                  size_t batch_target = kBatchBytes, int nbuf = 2) {
    StageShape s;
    s.nb = cols / QK;
    s.nch = (s.nb + 31) / 32;
    s.row_b = planar_row_bytes(type, cols);
    int R = int(batch_target / s.row_b);
    if (R < 1) R = 1;
    const int rmax = s.nch >= 32 ? 1 : 32 / s.nch;  // every (row, chunk) chain gets a lane
    if (R > rmax) R = rmax;
    if (R > 1 && (R & 1)) --R;                       // even: gate/up pairs stay in one batch
    s.R = R;
    s.batch_bytes = size_t(R) * s.row_b;
    s.act_bytes = a16(a16(sact_off(s.nb)) + size_t(s.nb) * 8);
    s.stage_floats2 = size_t(R) * (s.nb + s.nch);    // one float2 of padding per chunk
    s.warp_bytes = 64 + size_t(nbuf) * s.batch_bytes + a16(s.stage_floats2 * 8) + a16(size_t(R) * s.nch * 4);
    s.smem = s.act_bytes + size_t(warps) * s.warp_bytes;
    return s;
}

// The blocks and chains of one batch of rows_k rows (bb: the rows, planar):
// chsum[r * nch + c] = chunk c of row r, by the reference's fma chain.
// The block dots of rows [0, R) of a batch (R fixed, 32-bit shared offsets).
template <int TYPE, int R>
__device__ __forceinline__ void stage_blocks(const unsigned char* bb, uint32_t row_b, uint32_t qbytes, int nb,
                                             const uint8_t* aq, const float2* dsum, float2* stage, int spr, int lane) {
    constexpr int QB = TYPE == SYN_Q4_0 ? 16 : 32;
    for (int b = lane; b < nb; b += 32) {
        const int4* ap = reinterpret_cast<const int4*>(aq + sact_off(b));
        const int4 a0 = ap[0], a1 = ap[1];
        const float2 ds = dsum[b];
        const int asum = TYPE == SYN_Q4_0 ? __float_as_int(ds.y) : 0;
        const uint32_t wo = uint32_t(b) * QB, so = qbytes + uint32_t(b) * 2;
        const int si = b + (b >> 5);
        uint4 v0[R], v1[R];
        uint16_t dwh[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const unsigned char* wr = bb + uint32_t(r) * row_b;
            v0[r] = *reinterpret_cast<const uint4*>(wr + wo);
            if (QB == 32) v1[r] = *reinterpret_cast<const uint4*>(wr + wo + 16);
            dwh[r] = *reinterpret_cast<const uint16_t*>(wr + so);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            uint32_t w[8];
            w[0] = v0[r].x; w[1] = v0[r].y; w[2] = v0[r].z; w[3] = v0[r].w;
            if (QB == 32) {
                w[4] = v1[r].x; w[5] = v1[r].y; w[6] = v1[r].z; w[7] = v1[r].w;
            }
            const int isum = block_dot<TYPE>(w, a0, a1, asum);
            stage[r * spr + si] = make_float2(float(isum), __fmul_rn(f16_from_bits(dwh[r]), ds.x));
        }
    }
}

template <int TYPE>
__device__ __forceinline__ void stage_batch(const unsigned char* bb, int rows_k, const StageShape& sh, size_t qbytes,
                                            const uint8_t* aq, const float2* dsum, float2* stage, float* chsum,
                                            int lane) {
    constexpr int QB = TYPE == SYN_Q4_0 ? 16 : 32;
    const int nb = sh.nb, nch = sh.nch, spr = nb + nch;
    // Block b's activations are read once and meet the batch's rows_k rows;
    // the rows' dots are independent, so their loads and dp4a chains overlap.
    const uint32_t rb = uint32_t(sh.row_b), qb = uint32_t(qbytes);
    if (rows_k == 4) {
        stage_blocks<TYPE, 4>(bb, rb, qb, nb, aq, dsum, stage, spr, lane);
    } else if (rows_k == 2) {
        stage_blocks<TYPE, 2>(bb, rb, qb, nb, aq, dsum, stage, spr, lane);
    } else if (rows_k == 1) {
        stage_blocks<TYPE, 1>(bb, rb, qb, nb, aq, dsum, stage, spr, lane);
    } else {
        for (int r = 0; r < rows_k; ++r)
            stage_blocks<TYPE, 1>(bb + uint32_t(r) * rb, rb, qb, nb, aq, dsum, stage + r * spr, spr, lane);
    }
    (void)QB;
    __syncwarp();
    for (int ch = lane; ch < rows_k * nch; ch += 32) {
        const int r = ch / nch, c = ch - r * nch;
        const int m = min(32, nb - 32 * c);
        const float2* sp = stage + r * spr + 33 * c;
        float acc = 0.0f;
        if (m == 32) {
#pragma unroll 8
            for (int j = 0; j < 32; ++j) {
                const float2 v = sp[j];
                acc = fmaf(v.x, v.y, acc);  // dot.hpp:286, in block order
            }
        } else {
            for (int j = 0; j < m; ++j) {
                const float2 v = sp[j];
                acc = fmaf(v.x, v.y, acc);
            }
        }
        chsum[ch] = acc;
    }
    __syncwarp();
}

// Row `lane` of the batch: ((0 + chunk 0) + chunk 1) + ... (dot.hpp:398).
__device__ __forceinline__ float stage_row(const float* chsum, int nch, int rows_k, int lane) {
    float y = 0.0f;
    if (lane < rows_k)
        for (int c = 0; c < nch; ++c) y = __fadd_rn(y, chsum[lane * nch + c]);
    return y;
}

#ifdef SYN_DEVICE_EXPF
// silu(gate) * up (elementwise.hpp:76, :50)
__device__ __forceinline__ float silu_mul1(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_rn(-g))), u);
}
#endif

}  // namespace syn
