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
#define SYN_DEVICE_EXPF  // softmax / silu: the device expf and its exception table
#include "gemv_core.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <utility>
#include <vector>

using namespace syn;

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
// A whole row of per-block results is staged when it fits this budget per
// warp; otherwise one 32-block chunk at a time.
constexpr size_t kRowStageBytes = 16 * 1024;

struct GemvArgs {
    const uint8_t* w;    // GGUF rows, or planar rows
    const uint16_t* dh;  // unused (kept for layout symmetry)
    int rows, cols, nb, n_tok;
    ActPlanes act;       // SYN_IN_Q8: the Q8_0 activations
    float* y;
    const float* residual;
    int in_mode;         // SYN_IN_Q8 / SYN_IN_F32 / SYN_IN_RMSNORM
    const float* x;      // SYN_IN_F32, SYN_IN_RMSNORM: [n_tok][cols] floats
    const float* gamma;  // SYN_IN_RMSNORM
    float eps;
    int out_mode;        // SYN_OUT_ROWS / SYN_OUT_SILU_PAIRS
    TpSync tp;           // staged kernel: gathered input / residual words, output pushed to every rank
};

// Block b of row r: its quants as 32-bit words and its decoded scale.
template <int TYPE, int LAYOUT>
__device__ __forceinline__ void load_block(const GemvArgs& p, int r, int b, uint32_t (&w)[8], float& dw) {
    const size_t i = size_t(r) * p.nb + b;
    if (LAYOUT == SYN_LAYOUT_PLANAR) {
        const uint4* q = reinterpret_cast<const uint4*>(p.w + planar_quant_at(TYPE, p.cols, r, b));
        if (TYPE == SYN_Q4_0) {
            const uint4 v = __ldg(q);
            w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
        } else {
            const uint4 v0 = __ldg(q), v1 = __ldg(q + 1);
            w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w;
            w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
        }
        dw = f16_from_bits(__ldg(reinterpret_cast<const uint16_t*>(p.w + planar_scale_at(TYPE, p.cols, r, b))));
    } else {
        // GGUF AoS: 18 / 34-byte blocks, 2-byte aligned.
        const uint16_t* s = reinterpret_cast<const uint16_t*>(p.w + i * gguf_block_bytes(TYPE));
        dw = f16_from_bits(__ldg(s));
        constexpr int words = TYPE == SYN_Q4_0 ? 4 : 8;
#pragma unroll
        for (int k = 0; k < words; ++k) w[k] = uint32_t(__ldg(s + 1 + 2 * k)) | (uint32_t(__ldg(s + 2 + 2 * k)) << 16);
    }
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

// One chunk's accumulation in block order: acc = fma(isum_b, scale_b, acc)
// (dot.hpp:277-287 with one lane). A full chunk is unrolled so its shared
// memory loads issue ahead of the dependent fma chain.
__device__ __forceinline__ float chunk_chain(const float2* s, int n) {
    float acc = 0.0f;
    if (n == 32) {
        float2 v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = s[i];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc = fmaf(v[i].x, v[i].y, acc);
    } else {
        for (int i = 0; i < n; ++i) acc = fmaf(s[i].x, s[i].y, acc);
    }
    return acc;
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
                    chunk_sum[t * nch + ch] = chunk_chain(s, n);
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
                    const float acc = chunk_chain(stage + lane * SB, b_end - b_begin);
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

// ---- lane-streamed variant (planar rows, 1-2 tokens) ----------------------------
// Each lane streams its own run of blocks straight from HBM into registers
// (16-byte loads, eight blocks in flight), so many warps per SM keep the
// memory system busy without any shared-memory staging of weights. Lane
// layout: a row's nch 32-block chunks are split over S lanes each (S = 1, 2
// or 4: 32 / S consecutive blocks per lane), nch * S lanes per row, 32 /
// (nch * S) rows per warp. Every lane forms (float(isum_b), d_w * d_a) for its
// blocks; a chunk's fma chain then runs in block order, sub-lane after
// sub-lane (the running sum moves one lane up by shuffle), and the row sum
// adds the chunks in order: the reference's float order exactly.
// The activations sit in shared memory with 16 bytes of padding after every
// 8 blocks, so the sub-lanes' 16-byte reads spread over the banks.
__device__ unsigned g_gemv_timeouts = 0;  // bounded waits that gave up (syn_device_errors; none here)

// S sub-lanes per chunk; BPL = 32 / S blocks per lane.
template <int TYPE, int NT, int S>
__global__ void __launch_bounds__(kThreads, 2) gemv_lane_kernel(GemvArgs p) {
    constexpr int BPL = 32 / S;
    constexpr int QB = TYPE == SYN_Q4_0 ? 16 : 32;  // quant bytes per block
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = p.nb, nch = (nb + 31) / 32, lpr = nch * S, rpw = 32 / lpr;
    const size_t stride = act_pad_stride(nb);
    uint8_t* aq = smem;
    float2* dsum = reinterpret_cast<float2*>(smem + size_t(NT) * stride);
    const int rl = lane / lpr, rem = lane % lpr, c = rem / S, s = rem % S;
    const int m = rl < rpw ? min(32, nb - 32 * c) : 0;  // blocks of this lane's chunk
    const int j0 = s * BPL, nblk = max(0, min(m, j0 + BPL) - j0);
    const int b0 = 32 * c + j0;  // this lane's first block
    const size_t row_b = planar_row_bytes(TYPE, p.cols), qbytes = planar_quant_bytes(TYPE, p.cols);
    const long n_groups = (p.rows + rpw - 1) / rpw;
    const long nw = long(gridDim.x) * (blockDim.x >> 5);
    const long gw0 = long(blockIdx.x) * (blockDim.x >> 5) + warp;

    pdl_launch_dependents();
    pdl_wait();  // the activations (and the residual) come from the previous kernel
    if (p.in_mode == SYN_IN_Q8) {
        for (int i = threadIdx.x; i < NT * nb * 2; i += blockDim.x) {
            const int t = i / (2 * nb), b = (i / 2) % nb, h = i & 1;
            reinterpret_cast<int4*>(aq + size_t(t) * stride + act_pad_off(b))[h] =
                __ldg(reinterpret_cast<const int4*>(p.act.qs + size_t(t) * p.cols + size_t(b) * QK) + h);
        }
        for (int i = threadIdx.x; i < NT * nb; i += blockDim.x)
            dsum[i] = make_float2(__ldg(p.act.d + i), __int_as_float(__ldg(p.act.sum + i)));
    } else {
        quantize_act<NT, 1>(p.x, p.gamma, p.eps, p.in_mode == SYN_IN_RMSNORM, p.cols, aq, dsum);
    }
    __syncthreads();

    for (long grp = gw0; grp < n_groups; grp += nw) {
        const long row = grp * rpw + rl;
        const bool live = nblk > 0 && row < p.rows;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        float px[S > 1 ? NT : 1][S > 1 ? BPL : 1], ps[S > 1 ? NT : 1][S > 1 ? BPL : 1];
        if (live) {
            const uint8_t* wrow = p.w + size_t(row) * row_b;
            // LD blocks per batch: 128 bytes of quants in flight per lane
            constexpr int LD = TYPE == SYN_Q4_0 ? 8 : 4;
#pragma unroll
            for (int k0 = 0; k0 < BPL; k0 += LD) {
                if (k0 < nblk) {
                    uint4 wv[LD][QB / 16];
#pragma unroll
                    for (int k = 0; k < LD; ++k)
                        if (k0 + k < nblk) {
#pragma unroll
                            for (int h = 0; h < QB / 16; ++h)
                                wv[k][h] = __ldg(reinterpret_cast<const uint4*>(
                                                     wrow + size_t(planar_block_pos(nb, size_t(row), b0 + k0 + k)) * QB) + h);
                        }
                    // the batch's binary16 scales (8-byte aligned: k0 is a multiple of 4)
                    const uint2 sv = __ldg(reinterpret_cast<const uint2*>(wrow + qbytes + size_t(b0 + k0) * 2));
                    uint2 sv2 = make_uint2(0u, 0u);
                    if (LD == 8) sv2 = __ldg(reinterpret_cast<const uint2*>(wrow + qbytes + size_t(b0 + k0 + 4) * 2));
                    const uint32_t sw[4] = {sv.x, sv.y, sv2.x, sv2.y};
#pragma unroll
                    for (int k = 0; k < LD; ++k) {
                        if (k0 + k < nblk) {
                            const int b = b0 + k0 + k;
                            uint32_t w[8];
                            w[0] = wv[k][0].x; w[1] = wv[k][0].y; w[2] = wv[k][0].z; w[3] = wv[k][0].w;
                            if (QB == 32) {
                                w[4] = wv[k][QB / 16 - 1].x; w[5] = wv[k][QB / 16 - 1].y;
                                w[6] = wv[k][QB / 16 - 1].z; w[7] = wv[k][QB / 16 - 1].w;
                            }
                            const float dw = f16_from_bits(uint16_t(sw[k >> 1] >> (16 * (k & 1))));
#pragma unroll
                            for (int t = 0; t < NT; ++t) {
                                const int4* ap = reinterpret_cast<const int4*>(aq + size_t(t) * stride + act_pad_off(b));
                                const float2 ds = dsum[t * nb + b];
                                const int isum = block_dot<TYPE>(w, ap[0], ap[1], TYPE == SYN_Q4_0 ? __float_as_int(ds.y) : 0);
                                const float sc = __fmul_rn(dw, ds.x);
                                if (S == 1) {
                                    acc[t] = fmaf(float(isum), sc, acc[t]);  // dot.hpp:286, in block order
                                } else {
                                    px[S > 1 ? t : 0][S > 1 ? k0 + k : 0] = float(isum);
                                    ps[S > 1 ? t : 0][S > 1 ? k0 + k : 0] = sc;
                                }
                            }
                        }
                    }
                }
            }
        }
        if (S > 1) {
            // the chunk's chain, sub-lane 0 first: each continues from the previous one's sum
#pragma unroll
            for (int st = 0; st < S; ++st) {
                if (live && s == st) {
#pragma unroll
                    for (int k = 0; k < BPL; ++k)
                        if (k < nblk) {
#pragma unroll
                            for (int t = 0; t < NT; ++t)
                                acc[t] = fmaf(px[S > 1 ? t : 0][S > 1 ? k : 0], ps[S > 1 ? t : 0][S > 1 ? k : 0], acc[t]);
                        }
                }
                if (st + 1 < S) {
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const float from = __shfl_up_sync(0xffffffffu, acc[t], 1);
                        if (s == st + 1) acc[t] = from;
                    }
                }
            }
        }
        // Row sums: ((0 + chunk 0) + chunk 1) + ... (dot.hpp:398); chunk c's sum is in its last sub-lane.
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float y = 0.0f;
            for (int cc = 0; cc < nch; ++cc)
                y = __fadd_rn(y, __shfl_sync(0xffffffffu, acc[t], (rl * lpr + cc * S + S - 1) & 31));
            if (p.out_mode == SYN_OUT_SILU_PAIRS) {
                // rows 2i (gate) and 2i+1 (up) are rows rl, rl + 1 of the warp's group:
                // out[i] = silu(gate) * up (elementwise.hpp:76, :50)
                const float up = __shfl_sync(0xffffffffu, y, ((rl + 1) * lpr) & 31);
                if (rem == 0 && (rl & 1) == 0 && rl < rpw && row < p.rows)
                    p.y[size_t(t) * (p.rows / 2) + size_t(row / 2)] =
                        __fmul_rn(__fdiv_rn(y, __fadd_rn(1.0f, exp_rn(-y))), up);
            } else if (rem == 0 && rl < rpw && row < p.rows) {
                const size_t o = size_t(t) * p.rows + size_t(row);
                p.y[o] = p.residual ? __fadd_rn(y, p.residual[o]) : y;
            }
        }
    }
}

// ---- staged kernel (planar rows, one token) -------------------------------------
// A warp takes batches of R consecutive rows. Each batch lands in one of the
// warp's two shared-memory buffers by one bulk copy (the first two are
// requested before the kernel waits on its predecessor: weights never depend
// on it). Then
//   blocks: lane l forms (float(isum_b), d_w * d_a) for blocks l, l+32, ...
//           of every row of the batch (consecutive lanes read consecutive
//           16-byte quants: no bank conflicts) and stages the pairs;
//   chains: one lane per (row, 32-block chunk) runs that chunk's fma chain in
//           block order over the staged pairs (dot.hpp:277-287);
//   rows:   one lane per row adds its chunks in order (dot.hpp:398) and
//           writes the row, its residual sum, or silu(gate) * up.
// The activations (Q8_0, padded 16 bytes per 4 blocks so consecutive lanes'
// 32-byte reads spread over the banks) sit in shared memory once per CTA.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// W warps per CTA, batches of about BB bytes of rows, NB batch buffers per warp
// (NB - 1 batches in flight while the warp works on one).
template <int TYPE, int W, int BB, int NB>
__global__ void __launch_bounds__(W * 32) gemv_stage_kernel(GemvArgs p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const StageShape sh = stage_shape(TYPE, p.cols, W, BB, NB);
    const int nb = sh.nb, nch = sh.nch, R = sh.R;
    const size_t row_b = sh.row_b, qbytes = planar_quant_bytes(TYPE, p.cols);
    uint8_t* aq = smem;
    float2* dsum = reinterpret_cast<float2*>(smem + a16(sact_off(nb)));
    unsigned char* wbase = smem + sh.act_bytes + size_t(warp) * sh.warp_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(wbase);
    unsigned char* buf = wbase + 64;
    float2* stage = reinterpret_cast<float2*>(buf + NB * sh.batch_bytes);
    float* chsum = reinterpret_cast<float*>(buf + NB * sh.batch_bytes + a16(sh.stage_floats2 * 8));
    const long n_batch = (p.rows + R - 1) / R;
    const long gw = long(blockIdx.x) * W + warp, nw = long(gridDim.x) * W;
    const long k0 = n_batch * gw / nw, k1 = n_batch * (gw + 1) / nw;
    const int nbatch = int(k1 - k0);
    auto batch_rows = [&](int k) { return int(min(long(R), long(p.rows) - (k0 + k) * R)); };
    auto issue = [&](int k) {
        const uint32_t bytes = uint32_t(size_t(batch_rows(k)) * row_b);
        mbar_expect_tx(&bars[k % NB], bytes);
        bulk_copy_g2s(buf + size_t(k % NB) * sh.batch_bytes, p.w + size_t((k0 + k) * R) * row_b, bytes,
                      &bars[k % NB]);
    };
    if (lane == 0) {
        for (int i = 0; i < NB; ++i) mbar_init(&bars[i], 1);
        mbar_init_fence();
        for (int k = 0; k < min(NB, nbatch); ++k) issue(k);
    }
    __syncwarp();
    // this thread's first half-block of gamma (a weight: read before the wait)
    float4 gpre[4];
    const bool pre = p.in_mode == SYN_IN_RMSNORM && int(threadIdx.x) < p.cols / 16;
    if (pre)
#pragma unroll
        for (int k = 0; k < 4; ++k) gpre[k] = __ldg(reinterpret_cast<const float4*>(p.gamma + size_t(threadIdx.x) * 16) + k);
    pdl_launch_dependents();
    pdl_wait();  // the activations (and the residual) come from the previous kernel
    const bool push = p.tp.peers && p.tp.out_ll;
    const unsigned ep = p.tp.peers ? *reinterpret_cast<const volatile unsigned*>(p.tp.epoch) : 0u;
    if (p.in_mode == SYN_IN_Q8) {
        for (int i = threadIdx.x; i < nb * 2; i += blockDim.x)
            reinterpret_cast<int4*>(aq + sact_off(i >> 1))[i & 1] =
                __ldg(reinterpret_cast<const int4*>(p.act.qs) + i);
        for (int i = threadIdx.x; i < nb; i += blockDim.x)
            dsum[i] = make_float2(__ldg(p.act.d + i), __int_as_float(__ldg(p.act.sum + i)));
    } else if (p.tp.peers && p.tp.in_ll) {  // a gathered vector: every rank's words of this step
        quantize_act1<true>(p.x, p.gamma, p.eps, p.in_mode == SYN_IN_RMSNORM, p.cols, aq, dsum, &p.tp, ep,
                            pre ? gpre : nullptr);
    } else {
        quantize_act1(p.x, p.gamma, p.eps, p.in_mode == SYN_IN_RMSNORM, p.cols, aq, dsum, nullptr, 0u, pre ? gpre : nullptr);
    }
    __syncthreads();

    int k = 0;
    bool ok = true;
    for (; k < nbatch; ++k) {
        const bool got = mbar_wait_bounded(&bars[k % NB], uint32_t((k / NB) & 1), kWaitLimitNs);
        if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
        }
        const int rows_k = batch_rows(k);
        stage_batch<TYPE>(buf + size_t(k % NB) * sh.batch_bytes, rows_k, sh, qbytes, aq, dsum, stage, chsum, lane);
        const float y = stage_row(chsum, nch, rows_k, lane);
        const long row = (k0 + k) * R + lane;
        if (p.out_mode == SYN_OUT_SILU_PAIRS) {
            // rows 2i (gate) and 2i+1 (up) are lanes l, l+1 of the batch: out[i] = silu(gate) * up
            const float up = __shfl_down_sync(0xffffffffu, y, 1);
            if (lane < rows_k && (lane & 1) == 0) {
                const float v = silu_mul1(y, up);
                if (push) tp_store(p.tp, size_t(row / 2), v, ep);
                else p.y[size_t(row / 2)] = v;
            }
        } else if (lane < rows_k) {
            float v = y;
            if (p.residual) {
                const float r = p.tp.res_ll ? word_value(reinterpret_cast<const uint64_t*>(p.residual)[row])
                                            : p.residual[row];
                v = __fadd_rn(y, r);
            }
            if (push) tp_store(p.tp, size_t(row), v, ep);
            else p.y[row] = v;
        }
        __syncwarp();
        if (lane == 0 && k + NB < nbatch) {
            fence_async_shared();  // the warp's reads of this buffer come before the copy that refills it
            issue(k + NB);
        }
    }
    if (!ok && lane == 0) {
        // record it, then let the copies still in flight into this warp's buffers land (bounded)
        atomicAdd(&g_gemv_timeouts, 1u);
        for (int q = k; q < min(nbatch, k + NB); ++q) mbar_wait_bounded(&bars[q % NB], uint32_t((q / NB) & 1), kWaitLimitNs);
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

// The shared memory opt-in of a kernel, set once per device (a per-device
// function attribute) to the most any shape of this library asks for.
int configure(const void* kernel, size_t smem) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, int>> done;
    if (smem <= 48 * 1024) return SYN_OK;
    int dev = 0;
    int st = syn_cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& d : done)
        if (d.first == kernel && d.second == dev) return SYN_OK;
    // the device's per-block opt-in less the kernel's static shared memory (the batched
    // kernel's Q8_0 x 16 tokens takes up to 222 KB)
    int optin = 0;
    cudaFuncAttributes fa{};
    st = syn_cuda_status(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (!st) st = syn_cuda_status(cudaFuncGetAttributes(&fa, kernel));
    if (st) return st;
    const size_t most = size_t(optin) - fa.sharedSizeBytes;
    if (smem > most) return SYN_ERR_UNSUPPORTED;
    st = syn_cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(most)));
    if (!st) done.push_back({kernel, dev});
    return st;
}

// Sub-lanes per chunk for the lane kernel: split chunks (S = 2, 4) only when
// there are too few (row, chunk) pairs to give every resident warp work; with
// two tokens S = 2 would hold too many pairs in registers. 0: not this kernel
// (a row of more than 32 chunks, or gate/up pairs that would straddle warps).
int lane_split(int nt, int rows, int cols, int out_mode) {
    const int nb = cols / QK, nch = (nb + 31) / 32;
    const long units = long(rows) * nch, target = long(syn_num_sms()) * 48 * 32;
    int order[3] = {1, 2, 4};
    if (units < target / 4) { order[0] = 4; order[1] = 2; order[2] = 1; }
    else if (units < target / 2) { order[0] = 2; order[1] = 4; order[2] = 1; }
    for (int S : order) {
        if (nt == 2 && S == 2) continue;
        const int lpr = nch * S;
        if (lpr > 32) continue;
        const int rpw = 32 / lpr;
        if (out_mode == SYN_OUT_SILU_PAIRS && (rpw % 2 || rows % 2)) continue;
        return S;
    }
    return 0;
}

template <int TYPE, int NT, int S>
int launch_lane_s(const GemvArgs& p, cudaStream_t s) {
    auto k = gemv_lane_kernel<TYPE, NT, S>;
    const size_t smem = lane_act_bytes(NT, p.nb);
    int st = configure(reinterpret_cast<const void*>(k), smem);
    if (st) return st;
    const int nch = (p.nb + 31) / 32, rpw = 32 / (nch * S);
    const long groups = (p.rows + rpw - 1) / rpw;
    return syn_launch(k, persistent_grid(k, smem, groups), kThreads, smem, s, p);
}

template <int TYPE, int NT>
int launch_lane(const GemvArgs& p, int S, cudaStream_t s) {
    switch (S) {
    case 1: return launch_lane_s<TYPE, NT, 1>(p, s);
    case 2: return launch_lane_s<TYPE, NT, 2>(p, s);
    case 4: return launch_lane_s<TYPE, NT, 4>(p, s);
    }
    return SYN_ERR_UNSUPPORTED;
}

// Configuration of the staged kernel per shape: warps per CTA and batch bytes.
struct StageCfg {
    int warps;
    int batch;
    int nbuf;
};
// The configurations the staged kernel is built for: warps per CTA, batch bytes.
constexpr StageCfg kStageCfgs[] = {{8, 9728, 2}, {8, 4864, 4}, {6, 9728, 3}, {8, 6400, 3}, {12, 4864, 3},
                                   {16, 4864, 2}};

StageCfg stage_cfg(int type, int rows, int cols) {
    (void)rows;
    // SYN_GEMV_CFG="warps,batch,buffers" picks a built configuration (tuning sweeps)
    static const StageCfg forced = [] {
        StageCfg c{0, 0, 0};
        if (const char* e = std::getenv("SYN_GEMV_CFG")) {
            int w = 0, b = 0, n = 0;
            if (std::sscanf(e, "%d,%d,%d", &w, &b, &n) == 3)
                for (const StageCfg& k : kStageCfgs)
                    if (k.warps == w && k.batch == b && k.nbuf == n) c = k;
        }
        return c;
    }();
    if (forced.warps) return forced;
    (void)type;
    (void)cols;
    return kStageCfgs[0];
}

// Whether the staged kernel takes this one-token shape (gate/up pairs need
// even batches).
bool stage_ok(int type, int rows, int cols, int out_mode) {
    const StageCfg cfg = stage_cfg(type, rows, cols);
    const StageShape sh = stage_shape(type, cols, cfg.warps, size_t(cfg.batch), cfg.nbuf);
    if (sh.smem > 200 * 1024) return false;
    if (out_mode == SYN_OUT_SILU_PAIRS && (sh.R % 2 || rows % 2)) return false;
    return true;
}

template <int TYPE, int W, int BB, int NB>
int launch_stage_cfg(const GemvArgs& p, cudaStream_t s) {
    auto k = gemv_stage_kernel<TYPE, W, BB, NB>;
    const StageShape sh = stage_shape(TYPE, p.cols, W, BB, NB);
    int st = configure(reinterpret_cast<const void*>(k), sh.smem);
    if (st) return st;
    // One CTA per SM (W warps streaming ~BB-byte batches of rows each).
    const long batches = (p.rows + sh.R - 1) / sh.R;
    const long grid = std::max<long>(1, std::min<long>(long(syn_num_sms()), (batches + W - 1) / W));
    return syn_launch(k, unsigned(grid), unsigned(W * 32), sh.smem, s, p);
}

template <int TYPE>
int launch_stage(const GemvArgs& p, cudaStream_t s) {
    const StageCfg c = stage_cfg(TYPE, p.rows, p.cols);
#define SYN_STAGE_CFG(w, b, n) \
    if (c.warps == w && c.batch == b && c.nbuf == n) return launch_stage_cfg<TYPE, w, b, n>(p, s);
    SYN_STAGE_CFG(8, 4864, 4)
    SYN_STAGE_CFG(6, 9728, 3)
    SYN_STAGE_CFG(8, 6400, 3)
    SYN_STAGE_CFG(12, 4864, 3)
    SYN_STAGE_CFG(16, 4864, 2)
#undef SYN_STAGE_CFG
    return launch_stage_cfg<TYPE, 8, 9728, 2>(p, s);
}

// ---- batched tokens on integer tensor cores --------------------------------------
// n_tok >= 3 tokens, planar Q4_0 / Q8_0 rows (gemm.hpp:143-221 gemm_rows, G1:
// every token's row equals the one-token GEMV's). mma.m16n8k32 .s8 takes one
// 32-weight block as its k-step: the int32 product of 16 rows x 8 tokens is
// each (row, token) block dot exactly (Q4_0 weights enter as q - 8, the value
// the reference multiplies). The lane holding C[row][token] then runs that
// pair's fma chain in block order, acc = fma(float(isum), d_w * d_a, acc),
// over one 32-block chunk (dot.hpp:277-287), and the chunk sums of a row are
// added in order (dot.hpp:398).
// Fragment layouts (PTX ISA, mma.m16n8k32 .s8): lane = 4 g + t;
//   A: a0 = A[g][4t..4t+3], a1 = A[g+8][4t..], a2 = A[g][16+4t..], a3 = A[g+8][16+4t..]
//   B: b0 = B[4t..4t+3][g], b1 = B[16+4t..16+4t+3][g]
//   C: c0, c1 = C[g][2t], C[g][2t+1]; c2, c3 = C[g+8][2t], C[g+8][2t+1]
// A Q4_0 block holds element j in the low nibble of byte j and element j+16 in
// its high nibble, so one 32-bit word of bytes 4t..4t+3 gives both a0 and a2.
__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16_g(void* smem, const void* gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

constexpr int kImmaWarps = 4;      // warps per CTA: the chunk slots of one 16-row tile
constexpr int kImmaChunk = 32;     // blocks per chunk (the reference's fma-chain unit)
constexpr int kImmaSeg = kImmaWarps * kImmaChunk;  // blocks of activations staged per pass: one chunk per warp
constexpr int kImmaTokPitch = kImmaSeg * 32 + 16;  // bytes per token: consecutive tokens 4 banks apart
__host__ __device__ constexpr int imma_chunk_bytes(int type) {
    return 16 * kImmaChunk * (type == SYN_Q4_0 ? 16 : 32) + 16 * kImmaChunk * 2;  // 16 rows' quants, then scales
}
__host__ __device__ constexpr size_t imma_act_bytes(int ntt) {
    return size_t(8 * ntt) * kImmaTokPitch + size_t(8 * ntt) * kImmaSeg * 4;  // quants, then the decoded scales
}
__host__ __device__ inline size_t imma_smem(int type, int ntt, int nch) {
    return imma_act_bytes(ntt) + size_t(nch) * 16 * 8 * ntt * 4 +  // chunk sums of the tile
           size_t(kImmaWarps) * 2 * imma_chunk_bytes(type);      // each warp's chunk, double-buffered
}

// CTA (x, y): the 16-row tile x for tokens 8 NTT y ..; warp w computes chunks
// w, w + 4, ... of every row of the tile (their weights requested one chunk
// ahead), against the tokens' activations the CTA stages one segment of four
// chunks at a time between two block barriers; the chunk sums then meet in
// shared memory and are added in chunk order.
template <int TYPE, int NTT>
__global__ void __launch_bounds__(kImmaWarps * 32) gemm_imma_kernel(GemvArgs p) {
    constexpr int QB = TYPE == SYN_Q4_0 ? 16 : 32;
    constexpr int QS = 16 * kImmaChunk * QB, CB = imma_chunk_bytes(TYPE), NTOK = 8 * NTT;
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int r0 = blockIdx.x * 16, tok0 = blockIdx.y * NTOK;
    const int nb = p.nb, nch = (nb + kImmaChunk - 1) / kImmaChunk, nseg = (nb + kImmaSeg - 1) / kImmaSeg;
    int8_t* sq = reinterpret_cast<int8_t*>(smem);                                  // [NTOK][kImmaTokPitch]
    float* sd = reinterpret_cast<float*>(smem + size_t(NTOK) * kImmaTokPitch);    // [NTOK][kImmaSeg]
    float* cs = reinterpret_cast<float*>(smem + imma_act_bytes(NTT));             // [nch][16 rows][NTOK]
    unsigned char* wbuf = smem + imma_act_bytes(NTT) + size_t(nch) * 16 * NTOK * 4 + size_t(warp) * 2 * CB;
    const size_t row_b = planar_row_bytes(TYPE, p.cols), qbytes = planar_quant_bytes(TYPE, p.cols);
    // chunk c of the tile's 16 rows into buffer k (rows past the matrix re-read its last row, never stored)
    auto issue_chunk = [&](int c, int k) {
        if (c < nch) {
            unsigned char* dst = wbuf + k * CB;
            const int b0 = c * kImmaChunk, cnt = min(kImmaChunk, nb - b0);
            const int qpr = cnt * QB / 16, spr = (cnt * 2 + 15) / 16;  // 16-byte pieces per row (scales padded)
            for (int i = lane; i < 16 * qpr; i += 32) {
                const int rr = i / qpr, q = i - rr * qpr;
                const size_t r = size_t(min(r0 + rr, p.rows - 1));
                cp_async16_g(dst + rr * (kImmaChunk * QB) + q * 16, p.w + r * row_b + size_t(b0) * QB + q * 16);
            }
            for (int i = lane; i < 16 * spr; i += 32) {
                const int rr = i / spr, q = i - rr * spr;
                const size_t r = size_t(min(r0 + rr, p.rows - 1));
                cp_async16_g(dst + QS + rr * (kImmaChunk * 2) + q * 16, p.w + r * row_b + qbytes + size_t(b0) * 2 + q * 16);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // activations of blocks [seg0, seg0 + kImmaSeg) for the CTA's tokens (zero past n_tok)
    auto stage_act = [&](int seg0) {
        const int nblk = min(kImmaSeg, nb - seg0);
        const int per_tok = nblk * 2;  // 16-byte pieces
        for (int i = threadIdx.x; i < NTOK * per_tok; i += kImmaWarps * 32) {
            const int tl = i / per_tok, c = i - tl * per_tok, tk = tok0 + tl;
            int4 v = make_int4(0, 0, 0, 0);
            if (tk < p.n_tok) v = __ldg(reinterpret_cast<const int4*>(p.act.qs + size_t(tk) * p.cols + size_t(seg0) * 32) + c);
            *reinterpret_cast<int4*>(sq + tl * kImmaTokPitch + c * 16) = v;
        }
        for (int i = threadIdx.x; i < NTOK * nblk; i += kImmaWarps * 32) {
            const int tl = i / nblk, j = i - tl * nblk, tk = tok0 + tl;
            sd[tl * kImmaSeg + j] = tk < p.n_tok ? __ldg(p.act.d + size_t(tk) * nb + seg0 + j) : 0.0f;
        }
    };
    issue_chunk(warp, 0);  // weights never depend on the previous kernel
    pdl_launch_dependents();
    pdl_wait();  // the activations do

    for (int seg = 0; seg < nseg; ++seg) {
        __syncthreads();  // every warp is done with the previous segment
        stage_act(seg * kImmaSeg);
        __syncthreads();
        const int c = seg * kImmaWarps + warp;
        issue_chunk(c + kImmaWarps, (seg + 1) & 1);  // this warp's next chunk, one segment ahead
        asm volatile("cp.async.wait_group 1;" ::: "memory");  // chunk c (the older group) is in
        __syncwarp();
        if (c >= nch) continue;
        const unsigned char* st = wbuf + (seg & 1) * CB;
        const int cnt = min(kImmaChunk, nb - c * kImmaChunk);
        float acc[NTT][4];
#pragma unroll
        for (int n = 0; n < NTT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
#pragma unroll 4
        for (int j = 0; j < cnt; ++j) {
            uint32_t a[4];
            const unsigned char* qlo = st + g * (kImmaChunk * QB) + j * QB;
            const unsigned char* qhi = qlo + 8 * (kImmaChunk * QB);
            if (TYPE == SYN_Q4_0) {
                const uint32_t wl = *reinterpret_cast<const uint32_t*>(qlo + 4 * t);
                const uint32_t wh = *reinterpret_cast<const uint32_t*>(qhi + 4 * t);
                a[0] = __vsub4(wl & 0x0f0f0f0fu, 0x08080808u);
                a[2] = __vsub4((wl >> 4) & 0x0f0f0f0fu, 0x08080808u);
                a[1] = __vsub4(wh & 0x0f0f0f0fu, 0x08080808u);
                a[3] = __vsub4((wh >> 4) & 0x0f0f0f0fu, 0x08080808u);
            } else {
                a[0] = *reinterpret_cast<const uint32_t*>(qlo + 4 * t);
                a[2] = *reinterpret_cast<const uint32_t*>(qlo + 16 + 4 * t);
                a[1] = *reinterpret_cast<const uint32_t*>(qhi + 4 * t);
                a[3] = *reinterpret_cast<const uint32_t*>(qhi + 16 + 4 * t);
            }
            const float dlo = f16_from_bits(*reinterpret_cast<const uint16_t*>(st + QS + g * (kImmaChunk * 2) + j * 2));
            const float dhi =
                f16_from_bits(*reinterpret_cast<const uint16_t*>(st + QS + (g + 8) * (kImmaChunk * 2) + j * 2));
            const int bs = warp * kImmaChunk + j;  // the block in the staged segment
#pragma unroll
            for (int n = 0; n < NTT; ++n) {
                // this lane's B column is local token 8n + g (zeros past n_tok)
                const int8_t* aq = sq + (8 * n + g) * kImmaTokPitch + bs * 32;
                const uint32_t bq0 = *reinterpret_cast<const uint32_t*>(aq + 4 * t);
                const uint32_t bq1 = *reinterpret_cast<const uint32_t*>(aq + 16 + 4 * t);
                int cc[4] = {0, 0, 0, 0};
                mma_s8(cc, a, bq0, bq1);
                const int tl = 8 * n + 2 * t;  // local tokens of c0 / c2 (c1 / c3: + 1)
                const float da0 = sd[tl * kImmaSeg + bs], da1 = sd[(tl + 1) * kImmaSeg + bs];
                acc[n][0] = fmaf(float(cc[0]), __fmul_rn(dlo, da0), acc[n][0]);
                acc[n][1] = fmaf(float(cc[1]), __fmul_rn(dlo, da1), acc[n][1]);
                acc[n][2] = fmaf(float(cc[2]), __fmul_rn(dhi, da0), acc[n][2]);
                acc[n][3] = fmaf(float(cc[3]), __fmul_rn(dhi, da1), acc[n][3]);
            }
        }
        float* cc_out = cs + size_t(c) * 16 * NTOK;  // [row][token]
#pragma unroll
        for (int n = 0; n < NTT; ++n) {
            const int tl = 8 * n + 2 * t;
            cc_out[g * NTOK + tl] = acc[n][0];
            cc_out[g * NTOK + tl + 1] = acc[n][1];
            cc_out[(g + 8) * NTOK + tl] = acc[n][2];
            cc_out[(g + 8) * NTOK + tl + 1] = acc[n][3];
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // nothing left in flight (trailing groups are empty)
    __syncthreads();
    // y = ((0 + chunk 0) + chunk 1) + ... (dot.hpp:398), plus the residual
    for (int i = threadIdx.x; i < 16 * NTOK; i += kImmaWarps * 32) {
        const int rr = i / NTOK, tl = i - rr * NTOK, r = r0 + rr, tk = tok0 + tl;
        if (r >= p.rows || tk >= p.n_tok) continue;
        float y = 0.0f;
        for (int c = 0; c < nch; ++c) y = __fadd_rn(y, cs[size_t(c) * 16 * NTOK + i]);
        const size_t o = size_t(tk) * p.rows + r;
        p.y[o] = p.residual ? __fadd_rn(y, p.residual[o]) : y;
    }
}

template <int TYPE>
int launch_imma(const GemvArgs& p, cudaStream_t s) {
    const int nch = (p.nb + kImmaChunk - 1) / kImmaChunk;
    const unsigned gx = unsigned((p.rows + 15) / 16);
    if (p.n_tok > 8) {
        auto k = gemm_imma_kernel<TYPE, 2>;
        const size_t smem = imma_smem(TYPE, 2, nch);
        int st = configure(reinterpret_cast<const void*>(k), smem);
        if (st) return st;
        return syn_launch(k, dim3(gx, (p.n_tok + 15) / 16, 1), unsigned(kImmaWarps * 32), smem, s, p);
    }
    auto k = gemm_imma_kernel<TYPE, 1>;
    const size_t smem = imma_smem(TYPE, 1, nch);
    int st = configure(reinterpret_cast<const void*>(k), smem);
    if (st) return st;
    return syn_launch(k, dim3(gx, 1, 1), unsigned(kImmaWarps * 32), smem, s, p);
}

template <int TYPE, int LAYOUT, int NT>
int launch_q(const GemvArgs& p, cudaStream_t s) {
    if (LAYOUT == SYN_LAYOUT_PLANAR && NT == 1 && stage_ok(TYPE, p.rows, p.cols, SYN_OUT_ROWS))
        return launch_stage<TYPE>(p, s);
    if (LAYOUT == SYN_LAYOUT_PLANAR && NT <= 2) {
        const int S = lane_split(NT, p.rows, p.cols, SYN_OUT_ROWS);
        if (S) return launch_lane<TYPE, NT <= 2 ? NT : 1>(p, S, s);
    }
    const bool whole = warp_stage_bytes(p.nb, NT, true) <= kRowStageBytes;
    const size_t smem = size_t(kWarps) * warp_stage_bytes(p.nb, NT, whole);
    if (whole) {
        auto k = gemv_q_kernel<TYPE, LAYOUT, NT, true>;
        int st = configure(reinterpret_cast<const void*>(k), smem);
        if (st) return st;
        return syn_launch(k, persistent_grid(k, smem, p.rows), kThreads, smem, s, p);
    }
    auto k = gemv_q_kernel<TYPE, LAYOUT, NT, false>;
    int st = configure(reinterpret_cast<const void*>(k), smem);
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
    int st = configure(reinterpret_cast<const void*>(k), smem);
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
    if (syn_k_type(type))
        return syn_gemv_k(type, w, layout, rows, cols, act, n_tok, y, residual, static_cast<cudaStream_t>(stream));
    if (type != SYN_Q4_0 && type != SYN_Q8_0) return SYN_ERR_UNSUPPORTED;
    if (layout != SYN_LAYOUT_GGUF && layout != SYN_LAYOUT_PLANAR) return SYN_ERR_INVALID;
    if (!w || !act || !y || rows <= 0 || cols <= 0 || cols % QK || n_tok <= 0) return SYN_ERR_INVALID;
    if (layout == SYN_LAYOUT_PLANAR && (reinterpret_cast<uintptr_t>(w) & 15)) return SYN_ERR_INVALID;
    if (layout == SYN_LAYOUT_GGUF && (reinterpret_cast<uintptr_t>(w) & 1)) return SYN_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(act) & 15) return SYN_ERR_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const ActPlanes all = act_planes(const_cast<void*>(act), n_tok, cols);
    const int nb = cols / QK;
    if (layout == SYN_LAYOUT_PLANAR && n_tok >= 3) {  // integer tensor cores, every token in one launch
        GemvArgs p{};
        p.w = static_cast<const uint8_t*>(w);
        p.rows = rows;
        p.cols = cols;
        p.nb = nb;
        p.n_tok = n_tok;
        p.act = all;
        p.y = y;
        p.residual = residual;
        p.in_mode = SYN_IN_Q8;
        p.out_mode = SYN_OUT_ROWS;
        const int st = type == SYN_Q4_0 ? launch_imma<SYN_Q4_0>(p, s) : launch_imma<SYN_Q8_0>(p, s);
        if (st != SYN_ERR_UNSUPPORTED) return st;  // else a row too wide for its shared memory: the lane kernels
    }
    for (int t0 = 0; t0 < n_tok; t0 += 8) {
        const int n = n_tok - t0 < 8 ? n_tok - t0 : 8;
        GemvArgs p{};
        p.w = static_cast<const uint8_t*>(w);
        p.dh = nullptr;
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
        p.in_mode = SYN_IN_Q8;
        p.out_mode = SYN_OUT_ROWS;
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

extern "C" int syn_gemv_fusable(int type, int layout, int rows, int cols, int n_tok, int out_mode) {
    if ((type != SYN_Q4_0 && type != SYN_Q8_0) || layout != SYN_LAYOUT_PLANAR) return 0;
    if (rows <= 0 || cols <= 0 || cols % QK || n_tok < 1 || n_tok > 2) return 0;
    if (n_tok == 1 && stage_ok(type, rows, cols, out_mode)) return 1;
    if (lane_split(n_tok, rows, cols, out_mode) == 0) return 0;
    return lane_act_bytes(n_tok, cols / QK) <= 200 * 1024;
}

namespace {

// The fused modes' checks and kernel arguments (syn_gemv, syn_gemv_tp).
int fused_args(const syn_gemv_args* a, GemvArgs& p) {
    if (a->in_mode != SYN_IN_Q8 && a->in_mode != SYN_IN_F32 && a->in_mode != SYN_IN_RMSNORM) return SYN_ERR_INVALID;
    if (a->out_mode != SYN_OUT_ROWS && a->out_mode != SYN_OUT_SILU_PAIRS) return SYN_ERR_INVALID;
    if (!a->w || !a->y) return SYN_ERR_INVALID;
    if (a->in_mode == SYN_IN_Q8 ? !a->act : !a->x) return SYN_ERR_INVALID;
    if (a->in_mode == SYN_IN_RMSNORM && !a->gamma) return SYN_ERR_INVALID;
    if (a->out_mode == SYN_OUT_SILU_PAIRS && a->residual) return SYN_ERR_INVALID;
    if (!syn_gemv_fusable(a->type, a->layout, a->rows, a->cols, a->n_tok, a->out_mode)) return SYN_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(a->w) | reinterpret_cast<uintptr_t>(a->x) |
         reinterpret_cast<uintptr_t>(a->act) | reinterpret_cast<uintptr_t>(a->gamma)) & 15)
        return SYN_ERR_INVALID;
    p = GemvArgs{};
    p.w = static_cast<const uint8_t*>(a->w);
    p.rows = a->rows;
    p.cols = a->cols;
    p.nb = a->cols / QK;
    p.n_tok = a->n_tok;
    if (a->in_mode == SYN_IN_Q8) p.act = act_planes(const_cast<void*>(a->act), a->n_tok, a->cols);
    p.y = a->y;
    p.residual = a->residual;
    p.in_mode = a->in_mode;
    p.x = a->x;
    p.gamma = a->gamma;
    p.eps = a->eps;
    p.out_mode = a->out_mode;
    return SYN_OK;
}

}  // namespace

int syn_gemv_tp(const syn_gemv_args* a, const TpSync& t, cudaStream_t s) {
    if (!a) return SYN_ERR_INVALID;
    if (t.peers && (t.world < 1 || t.world > kTpMaxWorld || t.rank < 0 || t.rank >= t.world || !t.epoch || !t.err))
        return SYN_ERR_INVALID;
    GemvArgs p;
    const int st = fused_args(a, p);
    if (st) return st;
    if (a->n_tok != 1 || !stage_ok(a->type, a->rows, a->cols, a->out_mode)) return SYN_ERR_UNSUPPORTED;
    p.tp = t;
    return a->type == SYN_Q4_0 ? launch_stage<SYN_Q4_0>(p, s) : launch_stage<SYN_Q8_0>(p, s);
}

extern "C" int syn_gemv(const syn_gemv_args* a, void* stream) {
    if (!a) return SYN_ERR_INVALID;
    if (a->in_mode == SYN_IN_Q8 && a->out_mode == SYN_OUT_ROWS)
        return syn_gemv_q(a->type, a->w, a->layout, a->rows, a->cols, a->act, a->n_tok, a->y, a->residual, stream);
    GemvArgs p;
    const int st = fused_args(a, p);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (a->n_tok == 1 && stage_ok(a->type, a->rows, a->cols, a->out_mode))
        return a->type == SYN_Q4_0 ? launch_stage<SYN_Q4_0>(p, s) : launch_stage<SYN_Q8_0>(p, s);
    const int S = lane_split(a->n_tok, a->rows, a->cols, a->out_mode);
    if (a->type == SYN_Q4_0)
        return a->n_tok == 1 ? launch_lane<SYN_Q4_0, 1>(p, S, s) : launch_lane<SYN_Q4_0, 2>(p, S, s);
    return a->n_tok == 1 ? launch_lane<SYN_Q8_0, 1>(p, S, s) : launch_lane<SYN_Q8_0, 2>(p, S, s);
}

unsigned* syn_gemv_timeout_word() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemv_timeouts) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return static_cast<unsigned*>(p);
}

namespace {
// 32 gathered words read as a GEMV input quantizer reads them (tp_load_n),
// awaiting an epoch they never carry: every read must give up, not hang.
__global__ void tp_wait_check_kernel(TpSync t, const uint64_t* words, float* out) {
    const unsigned ep = *t.epoch;
    float v[16];
    tp_load_n(t, words + 16 * (threadIdx.x & 1), ep, v);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) s += v[i];
    out[threadIdx.x] = s;
}
}  // namespace

extern "C" int syn_check_tp_wait(unsigned wait_us, int* errors) {
    if (!errors) return SYN_ERR_INVALID;
    char* buf = nullptr;
    int st = syn_cuda_status(cudaMalloc(&buf, 4096));
    if (st) return st;
    st = syn_cuda_status(cudaMemset(buf, 0, 4096));  // words of epoch 0; the reads await epoch 1
    unsigned one = 1;
    if (!st) st = syn_cuda_status(cudaMemcpy(buf + 256, &one, 4, cudaMemcpyHostToDevice));
    TpSync t;
    t.peers = reinterpret_cast<char* const*>(buf + 512);
    t.epoch = reinterpret_cast<const unsigned*>(buf + 256);
    t.err = reinterpret_cast<unsigned*>(buf + 260);
    t.world = 1;
    t.in_ll = 1;
    t.wait_ns = (unsigned long long)wait_us * 1000ull;
    if (!st) {
        tp_wait_check_kernel<<<1, 32>>>(t, reinterpret_cast<const uint64_t*>(buf + 1024), reinterpret_cast<float*>(buf + 2048));
        st = syn_check_launch();
    }
    if (!st) st = syn_cuda_status(cudaDeviceSynchronize());
    unsigned n = 0;
    if (!st) st = syn_cuda_status(cudaMemcpy(&n, buf + 260, 4, cudaMemcpyDeviceToHost));
    cudaFree(buf);
    *errors = int(n);
    return st;
}

extern "C" int syn_device_errors(void) {
    unsigned n = 0;
    if (cudaMemcpyFromSymbol(&n, g_gemv_timeouts, sizeof n) != cudaSuccess) return -1;
    const int a = syn_attn_timeouts();
    return a < 0 ? -1 : int(n) + a;
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
