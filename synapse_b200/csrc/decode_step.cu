// The whole decode step of a Llama model as one persistent kernel
// (models/llama.hpp:395-470 through graph::session::run): embedding, every
// layer (rms_norm -> fused QKV GEMV -> RoPE + KV append + attention -> O GEMV +
// residual -> rms_norm -> gate/up GEMV + silu*mul -> down GEMV + residual), the
// final rms_norm, the head GEMV and the argmax.
//
// One cooperative launch of one CTA per SM (8 warps). The phases are separated
// by grid barriers (an arrival counter; every wait bounded in time, after
// which the step aborts and records the error). What a separate kernel per op
// pays at every launch -- the first weight bytes arriving microseconds after
// the kernel starts -- disappears: a warp requests its first two batches of
// the next GEMV's weights as soon as it has finished its part of the current
// phase, before the barrier, so they stream in while the grid synchronizes.
//
// Arithmetic is that of the separate kernels, op for op: the same in-kernel
// Q8_0 quantization of each GEMV input (quantize_act), the same staged block
// dots and chunk chains (stage_batch), the same RoPE table and scores as
// syn_attention. Attention work: one CTA per (KV head, context chunk), the
// chunk's positions split over the CTA's warps, in two phases: scores with
// the chunk's max and sum of exponentials, then (after the barrier) the
// merged normaliser, p and p.V. A context of up to 256 positions is one chunk
// handled by one warp: the reference's max, normaliser and position order
// exactly.
#include "gemv_core.cuh"
#include "internal.h"

#include <algorithm>
#include <mutex>
#include <vector>

namespace syn {
namespace {

constexpr int kWarpsPerCta = kStageWarps;   // 8
constexpr int kThreadsPerCta = kWarpsPerCta * 32;
constexpr int kTileRows = 32;               // K or V rows per warp tile
constexpr int kExactCtx = 256;              // up to here one warp attends in position order
constexpr int kMaxChunkPerWarp = 256;       // score buffer per warp (positions)
constexpr uint64_t kStepWaitNs = 1000000000ull;

// Element c of row tok of the embedding table (kernels/quant dequantize_row),
// as syn_embed computes it.
__device__ __forceinline__ float embed_value(int type, int layout, const uint8_t* table, int cols, int tok, int c) {
    if (type == SYN_F32) return reinterpret_cast<const float*>(table)[size_t(tok) * cols + c];
    if (type == SYN_F16) return f16_from_bits(reinterpret_cast<const uint16_t*>(table)[size_t(tok) * cols + c]);
    const int nb = cols / QK, b = c / QK, j = c % QK;
    float dsc;
    int q;
    if (layout == SYN_LAYOUT_GGUF) {
        const uint8_t* p = table + (size_t(tok) * nb + b) * gguf_block_bytes(type);
        dsc = f16_from_bits(uint16_t(p[0] | (p[1] << 8)));
        if (type == SYN_Q4_0) q = j < 16 ? (p[2 + j] & 0x0f) - 8 : (p[2 + j - 16] >> 4) - 8;
        else q = int8_t(p[2 + j]);
    } else {
        dsc = f16_from_bits(*reinterpret_cast<const uint16_t*>(table + planar_scale_at(type, cols, tok, b)));
        const uint8_t* p = table + planar_quant_at(type, cols, tok, b);
        if (type == SYN_Q4_0) q = j < 16 ? (p[j] & 0x0f) - 8 : (p[j - 16] >> 4) - 8;
        else q = int8_t(p[j]);
    }
    return __fmul_rn(float(q), dsc);
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct Ctx {
    const StepPlan* P;
    unsigned target;      // barrier arrivals expected so far (thread 0)
    uint64_t* bars;       // this warp's two mbarriers
    unsigned char* wreg;  // this warp's region
    unsigned issued;      // batches this warp has requested (all jobs)
    unsigned done;        // batches this warp has consumed
    bool ok;
};

// Grid barrier: every CTA arrives once; waits are bounded, and a wait that
// runs out (or sees another CTA's abort) makes the whole step abort.
__device__ bool grid_sync(Ctx& c) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* arrive = c.P->sync;
        unsigned* abort_flag = c.P->sync + 1;
        c.target += gridDim.x;
        __threadfence();
        atomicAdd(arrive, 1u);
        int ok = 1;
        const uint64_t t0 = global_ns();
        while (ld_acquire(arrive) < c.target) {
            if (ld_acquire(abort_flag)) { ok = 0; break; }
            if (global_ns() - t0 > kStepWaitNs) {
                atomicExch(abort_flag, 1u);
                atomicAdd(c.P->err, 1u);
                ok = 0;
                break;
            }
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    c.ok = c.ok && s_ok;
    return s_ok != 0;
}

// ---- GEMV phases ------------------------------------------------------------

struct Job {
    const uint8_t* w;
    int rows, cols;
};

__device__ __forceinline__ void warp_batches(const StageShape& sh, int rows, long& k0, int& n) {
    const long n_batch = (rows + sh.R - 1) / sh.R;
    const long nw = long(gridDim.x) * kWarpsPerCta, gw = long(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
    k0 = n_batch * gw / nw;
    n = int(n_batch * (gw + 1) / nw - k0);
}

// Requests this warp's first two batches of job J (weights only: safe before the barrier).
template <int TYPE>
__device__ void gemv_prefetch(const Job& J, Ctx& c) {
    const StageShape sh = stage_shape(TYPE, J.cols);
    long k0;
    int n;
    warp_batches(sh, J.rows, k0, n);
    const int lane = threadIdx.x & 31;
    if (lane == 0) {
        fence_async_shared();  // earlier generic accesses of this region come before the copies
        for (int k = 0; k < min(2, n); ++k) {
            const unsigned g = c.issued + k;
            const int rows_k = int(min(long(sh.R), long(J.rows) - (k0 + k) * sh.R));
            const uint32_t bytes = uint32_t(size_t(rows_k) * sh.row_b);
            mbar_expect_tx(&c.bars[g & 1], bytes);
            bulk_copy_g2s(c.wreg + size_t(g & 1) * sh.batch_bytes, J.w + size_t((k0 + k) * sh.R) * sh.row_b, bytes,
                          &c.bars[g & 1]);
        }
    }
    c.issued += min(2, n);
}

// This warp's batches of job J (its first two already requested). out_mode:
// SYN_OUT_ROWS (y = W a (+ residual)) or SYN_OUT_SILU_PAIRS.
template <int TYPE>
__device__ void gemv_run(const Job& J, Ctx& c, const uint8_t* aq, const float2* dsum, int out_mode, float* y,
                         const float* residual) {
    const StageShape sh = stage_shape(TYPE, J.cols);
    long k0;
    int n;
    warp_batches(sh, J.rows, k0, n);
    const int lane = threadIdx.x & 31;
    const size_t qbytes = planar_quant_bytes(TYPE, J.cols);
    float2* stage = reinterpret_cast<float2*>(c.wreg + 2 * sh.batch_bytes);
    float* chsum = reinterpret_cast<float*>(c.wreg + 2 * sh.batch_bytes + a16(sh.stage_floats2 * 8));
    for (int k = 0; k < n; ++k) {
        const unsigned g = c.done;
        bool got = c.ok && mbar_wait_bounded(&c.bars[g & 1], (g >> 1) & 1, kStepWaitNs);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
            if (lane == 0 && c.ok) {
                atomicExch(c.P->sync + 1, 1u);
                atomicAdd(c.P->err, 1u);
            }
            c.ok = false;
            return;  // the copies still in flight are waited for at exit
        }
        ++c.done;
        const int rows_k = int(min(long(sh.R), long(J.rows) - (k0 + k) * sh.R));
        stage_batch<TYPE>(c.wreg + size_t(g & 1) * sh.batch_bytes, rows_k, sh, qbytes, aq, dsum, stage, chsum, lane);
        const float v = stage_row(chsum, sh.nch, rows_k, lane);
        const long row = (k0 + k) * sh.R + lane;
        if (out_mode == SYN_OUT_SILU_PAIRS) {
            const float up = __shfl_down_sync(0xffffffffu, v, 1);
            if (lane < rows_k && (lane & 1) == 0) y[row / 2] = silu_mul1(v, up);
        } else if (lane < rows_k) {
            y[row] = residual ? __fadd_rn(v, residual[row]) : v;
        }
        __syncwarp();
        if (lane == 0 && k + 2 < n) {
            fence_async_shared();  // this warp's reads of the buffer come before the copy that refills it
            const unsigned gi = c.issued;
            const int rk = int(min(long(sh.R), long(J.rows) - (k0 + k + 2) * sh.R));
            const uint32_t bytes = uint32_t(size_t(rk) * sh.row_b);
            mbar_expect_tx(&c.bars[gi & 1], bytes);
            bulk_copy_g2s(c.wreg + size_t(gi & 1) * sh.batch_bytes, J.w + size_t((k0 + k + 2) * sh.R) * sh.row_b,
                          bytes, &c.bars[gi & 1]);
        }
        if (k + 2 < n) ++c.issued;
    }
}

// ---- attention phases ---------------------------------------------------------

struct AttnShape {
    int G, C, chunk;  // query heads per KV head; CTAs per KV head; positions per CTA
};

__device__ __forceinline__ AttnShape attn_shape(const StepPlan& P, int L) {
    AttnShape a;
    a.G = P.n_head / P.n_kv;
    if (L <= kExactCtx) {
        a.C = 1;
    } else {
        const int most = max(1, int(gridDim.x) / P.n_kv);
        a.C = min(most, (L + kExactCtx - 1) / kExactCtx);
        a.C = max(a.C, (L + kWarpsPerCta * kMaxChunkPerWarp - 1) / (kWarpsPerCta * kMaxChunkPerWarp));
    }
    a.chunk = (L + a.C - 1) / a.C;
    return a;
}

// This warp's positions [w0, w1) of its CTA's chunk [t0, t1).
__device__ __forceinline__ void warp_positions(int L, int t0, int t1, int warp, int& w0, int& w1) {
    if (L <= kExactCtx) {  // one warp, the reference's order
        w0 = warp == 0 ? t0 : t1;
        w1 = t1;
        return;
    }
    const int per = (t1 - t0 + kWarpsPerCta - 1) / kWarpsPerCta;
    w0 = min(t1, t0 + warp * per);
    w1 = min(t1, w0 + per);
}

__device__ __forceinline__ void cp16(void* smem, const void* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Rows [tb, tb + m) of one head's K or V cache into a warp tile (row P, the
// appended one, is skipped: the caller writes it from registers).
__device__ __forceinline__ void load_tile(uint16_t* tile, const uint16_t* cache, size_t row, int hd, int tb, int m,
                                          int skip, int lane) {
    const int c8n = hd / 8, rowh = hd + 8;
    for (int i = lane; i < m * c8n; i += 32) {
        const int rr = i / c8n, c8 = i - rr * c8n;
        if (tb + rr != skip) cp16(tile + rr * rowh + c8 * 8, cache + size_t(tb + rr) * row + c8 * 8);
    }
    cp_commit();
}

struct AttnWarpMem {
    float* sc;     // [G][kMaxChunkPerWarp] scores, then e
    uint16_t* tile;// [kTileRows][hd + 8]
    float* part;   // [G][hd] this warp's p.V
};

__device__ __forceinline__ AttnWarpMem attn_warp_mem(unsigned char* wreg, int G, int hd) {
    AttnWarpMem m;
    m.sc = reinterpret_cast<float*>(wreg);
    m.tile = reinterpret_cast<uint16_t*>(wreg + size_t(G) * kMaxChunkPerWarp * 4);
    m.part = reinterpret_cast<float*>(wreg + size_t(G) * kMaxChunkPerWarp * 4 + size_t(kTileRows) * (hd + 8) * 2);
    return m;
}

__host__ __device__ inline size_t attn_warp_bytes(int G, int hd) {
    return size_t(G) * kMaxChunkPerWarp * 4 + size_t(kTileRows) * (hd + 8) * 2 + size_t(G) * hd * 4;
}

}  // namespace

// ---- the kernel ---------------------------------------------------------------

template <int LT, int HT>
__global__ void __launch_bounds__(kThreadsPerCta, 1) decode_step_kernel(const StepPlan* __restrict__ plan) {
    extern __shared__ __align__(128) unsigned char smem[];
    const StepPlan& P = *plan;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int d = P.d, G = P.n_head / P.n_kv, hd = P.hd;
    Ctx c;
    c.P = plan;
    c.target = 0;
    c.issued = 0;
    c.done = 0;
    c.ok = true;
    // shared memory: activations | barriers | CTA attention state | warp regions
    uint8_t* aq = smem;
    float2* dsum = reinterpret_cast<float2*>(smem + a16(sact_off(P.nb_max)));
    c.bars = reinterpret_cast<uint64_t*>(smem + P.act_bytes) + 2 * warp;
    float* qg = reinterpret_cast<float*>(smem + P.act_bytes + 16 * kWarpsPerCta);          // [G][hd]
    float* cta_f = qg + G * hd;                                                             // small reductions
    double* cta_d = reinterpret_cast<double*>(cta_f + 4 * 64);
    float* cs = reinterpret_cast<float*>(cta_d + 4 * 64);                                   // [hd] cos/sin
    unsigned char* wbase = smem + P.warp_base;
    c.wreg = wbase + size_t(warp) * P.warp_bytes;
    if (lane == 0) {
        mbar_init(&c.bars[0], 1);
        mbar_init(&c.bars[1], 1);
        mbar_init_fence();
    }
    __syncwarp();

    const int token = P.io[0], pos = P.io[1];
    const int L = pos + 1;
    const bool valid = token >= 0 && token < P.vocab && pos >= 0 && pos < P.max_ctx;

    if (!valid) return;  // the host checks token and position; every CTA sees the same io
    // embedding -> x (each CTA a slice), and the first layer's QKV weights on their way
    gemv_prefetch<LT>(Job{P.layers[0].qkv, P.qrows + 2 * P.kvrows, d}, c);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x)
        P.x[i] = embed_value(P.etype, P.elayout, P.embd, d, token, i);
    grid_sync(c);

    for (int l = 0; l < P.n_layer && c.ok; ++l) {
        const StepLayer& Lw = P.layers[l];
        // ---- QKV: rms_norm(x) quantized, one GEMV over the fused rows
        quantize_act1(P.x, Lw.attn_norm, P.eps, true, d, aq, dsum);
        __syncthreads();
        gemv_run<LT>(Job{Lw.qkv, P.qrows + 2 * P.kvrows, d}, c, aq, dsum, SYN_OUT_ROWS, P.qkv, nullptr);
        if (!grid_sync(c)) break;

        // ---- attention (one CTA per (KV head, chunk))
        const AttnShape A = attn_shape(P, L);
        const int items = P.n_kv * A.C;
        const bool att = int(blockIdx.x) < items;
        const int g = att ? int(blockIdx.x) / A.C : 0, jc = att ? int(blockIdx.x) % A.C : 0;
        const int t0 = min(L, jc * A.chunk), t1 = min(L, t0 + A.chunk);
        int w0, w1;
        warp_positions(L, t0, t1, warp, w0, w1);
        const int nw = w1 - w0;
        const size_t kvrow = size_t(P.n_kv) * hd;
        const bool owns = att && t0 <= pos && pos < t1;
        AttnWarpMem am = attn_warp_mem(c.wreg, G, hd);
        const int rowh = hd + 8;
        if (att) {
            // phase A: rotated q (binary16 values), the appended k / v, scores, chunk maxima
            for (int i = threadIdx.x; i < hd / 2; i += blockDim.x) {
                const float2 v = reinterpret_cast<const float2*>(P.rope_tab)[size_t(pos) * (hd / 2) + i];
                cs[2 * i] = v.x;
                cs[2 * i + 1] = v.y;
            }
            __syncthreads();
            const float* qb = P.qkv + size_t(g) * G * hd;
            for (int i = threadIdx.x; i < G * hd / 2; i += blockDim.x) {
                const int jh = i / (hd / 2), pi = i % (hd / 2);
                const float x0 = qb[jh * hd + 2 * pi], x1 = qb[jh * hd + 2 * pi + 1];
                qg[jh * hd + 2 * pi] = round_f16(__fsub_rn(__fmul_rn(x0, cs[2 * pi]), __fmul_rn(x1, cs[2 * pi + 1])));
                qg[jh * hd + 2 * pi + 1] = round_f16(__fadd_rn(__fmul_rn(x0, cs[2 * pi + 1]), __fmul_rn(x1, cs[2 * pi])));
            }
            if (owns) {
                const float* kb = P.qkv + P.qrows + size_t(g) * hd;
                const float* vb = P.qkv + P.qrows + P.kvrows + size_t(g) * hd;
                uint16_t* krow = Lw.kc + size_t(pos) * kvrow + size_t(g) * hd;
                uint16_t* vrow = Lw.vc + size_t(pos) * kvrow + size_t(g) * hd;
                for (int pi = threadIdx.x; pi < hd / 2; pi += blockDim.x) {
                    const float x0 = kb[2 * pi], x1 = kb[2 * pi + 1];
                    krow[2 * pi] = f16_bits(__fsub_rn(__fmul_rn(x0, cs[2 * pi]), __fmul_rn(x1, cs[2 * pi + 1])));
                    krow[2 * pi + 1] = f16_bits(__fadd_rn(__fmul_rn(x0, cs[2 * pi + 1]), __fmul_rn(x1, cs[2 * pi])));
                }
                for (int i = threadIdx.x; i < hd; i += blockDim.x) vrow[i] = f16_bits(vb[i]);
                __threadfence_block();
            }
            __syncthreads();  // q ready; row pos of K / V written (this CTA reads it back below)
        }
        float mloc[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) mloc[h] = -INFINITY;
        if (att && nw > 0) {
            const uint16_t* kc = Lw.kc + size_t(g) * hd;
            for (int tb = w0; tb < w1; tb += kTileRows) {
                const int m = min(kTileRows, w1 - tb);
                load_tile(am.tile, kc, kvrow, hd, tb, m, -1, lane);
                cp_wait_all();
                __syncwarp();
                // lane = position; all G heads in dimension order (attention.hpp:214-219)
                if (lane < m) {
                    const uint16_t* kt = am.tile + lane * rowh;
                    float acc[8];
#pragma unroll
                    for (int h = 0; h < 8; ++h) acc[h] = 0.0f;
                    for (int d8 = 0; d8 < hd; d8 += 8) {
                        const uint4 kv = *reinterpret_cast<const uint4*>(kt + d8);
                        const uint32_t wv[4] = {kv.x, kv.y, kv.z, kv.w};
                        float kf[8];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            kf[2 * e] = f16_from_bits(uint16_t(wv[e] & 0xffff));
                            kf[2 * e + 1] = f16_from_bits(uint16_t(wv[e] >> 16));
                        }
#pragma unroll
                        for (int h = 0; h < 8; ++h) {
                            if (h < G) {
                                const float4 q0 = *reinterpret_cast<const float4*>(qg + h * hd + d8);
                                const float4 q1 = *reinterpret_cast<const float4*>(qg + h * hd + d8 + 4);
                                float a = acc[h];
                                a = fmaf(q0.x, kf[0], a); a = fmaf(q0.y, kf[1], a);
                                a = fmaf(q0.z, kf[2], a); a = fmaf(q0.w, kf[3], a);
                                a = fmaf(q1.x, kf[4], a); a = fmaf(q1.y, kf[5], a);
                                a = fmaf(q1.z, kf[6], a); a = fmaf(q1.w, kf[7], a);
                                acc[h] = a;
                            }
                        }
                    }
#pragma unroll
                    for (int h = 0; h < 8; ++h) {
                        if (h < G) {
                            const float sv = __fmul_rn(acc[h], P.scale);
                            am.sc[h * kMaxChunkPerWarp + (tb - w0) + lane] = sv;
                            mloc[h] = fmaxf(mloc[h], sv);
                        }
                    }
                }
                __syncwarp();
            }
            // V of this warp's positions: requested now, needed after two barriers
            if (nw <= kTileRows) load_tile(am.tile, Lw.vc + size_t(g) * hd, kvrow, hd, w0, nw, -1, lane);
        }
        // the chunk's statistics per query head: max m over its positions, then
        // the double sum of expf(s - m) (the warps' parts in warp order)
#pragma unroll
        for (int h = 0; h < 8; ++h) mloc[h] = warp_max(mloc[h]);
        if (att && lane == 0)
            for (int h = 0; h < G; ++h) cta_f[h * 8 + warp] = mloc[h];
        __syncthreads();
        if (att) {
            if (threadIdx.x < G) {
                float mx = -INFINITY;
                for (int w = 0; w < kWarpsPerCta; ++w) mx = fmaxf(mx, cta_f[threadIdx.x * 8 + w]);
                cta_f[64 + threadIdx.x] = mx;
            }
            __syncthreads();
            double part[8];
#pragma unroll
            for (int h = 0; h < 8; ++h) part[h] = 0.0;
            for (int t = lane; t < nw; t += 32) {
#pragma unroll
                for (int h = 0; h < 8; ++h)
                    if (h < G) part[h] += double(exp_rn(__fsub_rn(am.sc[h * kMaxChunkPerWarp + t], cta_f[64 + h])));
            }
#pragma unroll
            for (int h = 0; h < 8; ++h) part[h] = warp_sum_d(part[h]);
            if (lane == 0)
                for (int h = 0; h < G; ++h) cta_d[h * 8 + warp] = part[h];
            __syncthreads();
            if (threadIdx.x < G) {
                double sum = 0.0;
                for (int w = 0; w < kWarpsPerCta; ++w) sum += cta_d[threadIdx.x * 8 + w];
                P.att_m[(g * G + threadIdx.x) * P.max_split + jc] = cta_f[64 + threadIdx.x];
                P.att_s[(g * G + threadIdx.x) * P.max_split + jc] = sum;
            }
        }
        if (!grid_sync(c)) break;

        // phase C: the context's max M and normaliser (elementwise.hpp:174-201;
        // merged over the chunks: sum_j s_j * exp(m_j - M), exact with one chunk),
        // p = binary16(expf(s - M) * (1 / sum)), p.V in position order per warp
        if (att) {
            if (threadIdx.x < G) {
                const float* mj = P.att_m + (g * G + threadIdx.x) * P.max_split;
                const double* sj = P.att_s + (g * G + threadIdx.x) * P.max_split;
                float M = -INFINITY;
                for (int j = 0; j < A.C; ++j) M = fmaxf(M, __ldcg(mj + j));
                double sum = 0.0;
                for (int j = 0; j < A.C; ++j) {
                    const double sv = __ldcg(sj + j);
                    if (sv > 0.0) sum += sv * exp(double(__ldcg(mj + j)) - double(M));
                }
                cta_f[64 + threadIdx.x] = M;
                cta_f[128 + threadIdx.x] = float(1.0 / sum);
            }
            __syncthreads();
            // lane owns columns 2 lane, 2 lane + 1 (+ 64, + 65, ...) of every head
            float acc[8][4];
#pragma unroll
            for (int h = 0; h < 8; ++h)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[h][q] = 0.0f;
            const uint16_t* vcache = Lw.vc + size_t(g) * hd;
            for (int tb = w0; tb < w1; tb += kTileRows) {
                const int m = min(kTileRows, w1 - tb);
                if (!(nw <= kTileRows)) load_tile(am.tile, vcache, kvrow, hd, tb, m, -1, lane);
                cp_wait_all();
                // p of the tile's rows, in place of the scores
                for (int i = lane; i < m * G; i += 32) {
                    const int h = i / m, r = i - h * m;
                    float* sp = am.sc + h * kMaxChunkPerWarp + (tb - w0) + r;
                    *sp = round_f16(__fmul_rn(exp_rn(__fsub_rn(*sp, cta_f[64 + h])), cta_f[128 + h]));
                }
                __syncwarp();
                for (int r = 0; r < m; ++r) {
                    const uint16_t* vr = am.tile + r * rowh;
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int col = 2 * lane + 64 * q;
                        if (col < hd) {
                            const uint32_t v2 = *reinterpret_cast<const uint32_t*>(vr + col);
                            const float va = f16_from_bits(uint16_t(v2 & 0xffff)), vb = f16_from_bits(uint16_t(v2 >> 16));
#pragma unroll
                            for (int h = 0; h < 8; ++h) {
                                if (h < G) {
                                    const float pp = am.sc[h * kMaxChunkPerWarp + (tb - w0) + r];
                                    acc[h][2 * q] = fmaf(pp, va, acc[h][2 * q]);  // exact products
                                    acc[h][2 * q + 1] = fmaf(pp, vb, acc[h][2 * q + 1]);
                                }
                            }
                        }
                    }
                }
                __syncwarp();
            }
#pragma unroll
            for (int h = 0; h < 8; ++h)
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int col = 2 * lane + 64 * q;
                    if (h < G && col < hd) {
                        am.part[h * hd + col] = acc[h][2 * q];
                        am.part[h * hd + col + 1] = acc[h][2 * q + 1];
                    }
                }
            __syncthreads();
            // the CTA's partial: its warps' partials in position order, to global
            float* gpart = P.att_part + (size_t(g) * P.max_split + jc) * G * hd;
            for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
                float s = 0.0f;
                for (int w = 0; w < kWarpsPerCta; ++w) {
                    const float* wp = reinterpret_cast<const float*>(wbase + size_t(w) * P.warp_bytes +
                                                                     size_t(G) * kMaxChunkPerWarp * 4 +
                                                                     size_t(kTileRows) * rowh * 2);
                    s = __fadd_rn(s, wp[i]);
                }
                gpart[i] = s;
            }
            // the last CTA of this KV head adds the chunks in order
            __threadfence();
            __syncthreads();
            __shared__ int s_last;
            if (threadIdx.x == 0) s_last = atomicAdd(P.sync + 2 + g, 1u) == unsigned(A.C - 1);
            __syncthreads();
            if (s_last) {
                __threadfence();
                float* ob = P.attn + size_t(g) * G * hd;
                for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
                    float s = 0.0f;
                    for (int j = 0; j < A.C; ++j)
                        s = __fadd_rn(s, __ldcg(P.att_part + (size_t(g) * P.max_split + j) * G * hd + i));
                    ob[i] = s;
                }
                if (threadIdx.x == 0) P.sync[2 + g] = 0u;  // ready for the next layer
            }
        }
        __syncthreads();
        gemv_prefetch<LT>(Job{Lw.o, d, P.qrows}, c);
        if (!grid_sync(c)) break;

        // ---- O: attention output quantized, + residual x -> x2
        quantize_act1(P.attn, nullptr, 0.0f, false, P.qrows, aq, dsum);
        __syncthreads();
        gemv_run<LT>(Job{Lw.o, d, P.qrows}, c, aq, dsum, SYN_OUT_ROWS, P.x2, P.x);
        gemv_prefetch<LT>(Job{Lw.gu, 2 * P.ff, d}, c);
        if (!grid_sync(c)) break;

        // ---- gate/up: rms_norm(x2) quantized; silu(gate) * up -> act
        quantize_act1(P.x2, Lw.ffn_norm, P.eps, true, d, aq, dsum);
        __syncthreads();
        gemv_run<LT>(Job{Lw.gu, 2 * P.ff, d}, c, aq, dsum, SYN_OUT_SILU_PAIRS, P.act, nullptr);
        gemv_prefetch<LT>(Job{Lw.down, d, P.ff}, c);
        if (!grid_sync(c)) break;

        // ---- down: act quantized, + residual x2 -> x
        quantize_act1(P.act, nullptr, 0.0f, false, P.ff, aq, dsum);
        __syncthreads();
        gemv_run<LT>(Job{Lw.down, d, P.ff}, c, aq, dsum, SYN_OUT_ROWS, P.x, P.x2);
        if (l + 1 < P.n_layer) gemv_prefetch<LT>(Job{P.layers[l + 1].qkv, P.qrows + 2 * P.kvrows, d}, c);
        else gemv_prefetch<HT>(Job{P.head, P.vocab, d}, c);
        if (!grid_sync(c)) break;
    }

    if (c.ok) {
        // ---- head: rms_norm(x) quantized -> logits
        quantize_act1(P.x, P.out_norm, P.eps, true, d, aq, dsum);
        __syncthreads();
        gemv_run<HT>(Job{P.head, P.vocab, d}, c, aq, dsum, SYN_OUT_ROWS, P.logits, nullptr);
        if (grid_sync(c)) {
            // ---- argmax (the first maximum, llama_decode.cpp:274): CTA slices, then CTA 0
            __shared__ float s_v[kWarpsPerCta];
            __shared__ int s_i[kWarpsPerCta];
            const int per = (P.vocab + gridDim.x - 1) / gridDim.x;
            const int lo = blockIdx.x * per, hi = min(P.vocab, lo + per);
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
                const float v = P.logits[i];
                if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
            }
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0) { s_v[warp] = bv; s_i[warp] = bi; }
            __syncthreads();
            if (threadIdx.x == 0) {
                for (int w = 1; w < kWarpsPerCta; ++w)
                    if (s_v[w] > bv || (s_v[w] == bv && s_i[w] < bi)) { bv = s_v[w]; bi = s_i[w]; }
                P.am_v[blockIdx.x] = bv;
                P.am_i[blockIdx.x] = bi;
            }
            if (grid_sync(c) && blockIdx.x == 0 && threadIdx.x == 0) {
                float v = -INFINITY;
                int idx = 0x7fffffff;
                for (int b = 0; b < int(gridDim.x); ++b) {
                    const float ov = __ldcg(P.am_v + b);
                    const int oi = __ldcg(P.am_i + b);
                    if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
                }
                P.io[2] = idx == 0x7fffffff ? 0 : idx;
            }
        }
    }
    // nothing may still be copying into this CTA's shared memory when it leaves
    if (lane == 0) {
        for (unsigned g = c.done; g < c.issued; ++g) mbar_wait_bounded(&c.bars[g & 1], (g >> 1) & 1, kStepWaitNs);
    }
    cp_wait_all();
    __syncwarp();
}

}  // namespace syn

using namespace syn;

namespace {

template <int LT, int HT>
int launch_step(const StepPlan* dplan, size_t smem, int grid, cudaStream_t s) {
    auto k = decode_step_kernel<LT, HT>;
    int st = syn_cuda_status(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    if (st) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreadsPerCta);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return syn_cuda_status(cudaLaunchKernelEx(&cfg, k, dplan));
}

template <int LT, int HT>
int max_blocks(size_t smem, int* per_sm) {
    auto k = decode_step_kernel<LT, HT>;
    int st = syn_cuda_status(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    if (st) return st;
    return syn_cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k, kThreadsPerCta, smem));
}

}  // namespace

// Shared memory layout of the step kernel for a plan (fills act_bytes,
// warp_base, warp_bytes, nb_max); 0 if the shapes need more than a CTA has.
size_t syn_step_smem(StepPlan* p, int ltype, int htype) {
    const int G = p->n_head / p->n_kv;
    const int cols_max = std::max(std::max(p->d, p->qrows), p->ff);
    p->nb_max = cols_max / QK;
    p->act_bytes = a16(a16(sact_off(p->nb_max)) + size_t(p->nb_max) * 8);
    size_t cta = 16 * kWarpsPerCta + size_t(G) * p->hd * 4 + 4 * 64 * 4 + 4 * 64 * 8 + size_t(p->hd) * 4;
    p->warp_base = a16(p->act_bytes + cta);
    size_t wb = attn_warp_bytes(G, p->hd);
    const int cols_of[4] = {p->d, p->qrows, p->d, p->ff};
    for (int i = 0; i < 4; ++i) {
        const StageShape sh = stage_shape(ltype, cols_of[i]);
        wb = std::max(wb, 2 * sh.batch_bytes + a16(sh.stage_floats2 * 8) + a16(size_t(sh.R) * sh.nch * 4));
    }
    {
        const StageShape sh = stage_shape(htype, p->d);
        wb = std::max(wb, 2 * sh.batch_bytes + a16(sh.stage_floats2 * 8) + a16(size_t(sh.R) * sh.nch * 4));
    }
    p->warp_bytes = a16(wb);
    const size_t total = p->warp_base + kWarpsPerCta * p->warp_bytes;
    return total <= 227 * 1024 ? total : 0;
}

int syn_step_grid(int ltype, int htype, size_t smem) {
    int per_sm = 0;
    int st;
    if (ltype == SYN_Q4_0) st = htype == SYN_Q4_0 ? max_blocks<SYN_Q4_0, SYN_Q4_0>(smem, &per_sm)
                                                 : max_blocks<SYN_Q4_0, SYN_Q8_0>(smem, &per_sm);
    else st = htype == SYN_Q4_0 ? max_blocks<SYN_Q8_0, SYN_Q4_0>(smem, &per_sm)
                                : max_blocks<SYN_Q8_0, SYN_Q8_0>(smem, &per_sm);
    if (st || per_sm < 1) return 0;
    return syn_num_sms();  // one CTA per SM (all resident: a cooperative launch)
}

int syn_step_launch(const StepPlan* dplan, int ltype, int htype, size_t smem, int grid, cudaStream_t s) {
    if (ltype == SYN_Q4_0)
        return htype == SYN_Q4_0 ? launch_step<SYN_Q4_0, SYN_Q4_0>(dplan, smem, grid, s)
                                 : launch_step<SYN_Q4_0, SYN_Q8_0>(dplan, smem, grid, s);
    return htype == SYN_Q4_0 ? launch_step<SYN_Q8_0, SYN_Q4_0>(dplan, smem, grid, s)
                             : launch_step<SYN_Q8_0, SYN_Q8_0>(dplan, smem, grid, s);
}
