// RoPE + F16 KV append + GQA decode attention (kernels/attention.hpp:89-269).
//
// Numerics follow attend_group (attention.hpp:185-244): q rounded to
// binary16; s_t = (q . K_t) * scale with the dot in dimension order (the
// binary16 products are exact in float, so each step is one fma); softmax
// with the float max M, e_t = expf(s_t - M), the normaliser summed in double
// and scale = float(1 / sum) (elementwise.hpp:174-201); p_t = binary16(e_t *
// scale), rounded after normalisation as the reference rounds it;
// out = sum_t p_t V_t.
//
// Two summation orders (syn_attention_args.order):
//
// SYN_ORDER_REFERENCE (the default): every float sum in the reference's order
// at any context length. Three stream-ordered kernels:
//   scores: one CTA per (chunk of kChunk positions, KV head, query); the
//           chunk's K rows land in shared memory by tensor copies; each
//           thread scores one position for the G query heads, every dot a
//           dimension-order chain of fmas on binary16 values (exact
//           products, one rounding per add, as the reference's); the
//           chunk's max per head;
//   exp:    the context's max M per head from the chunk maxima, e_t =
//           expf(s_t - M) in place of the scores, the chunk's double sum;
//   p.V:    one CTA per (query head, 32 output columns): a producer warp
//           streams V tiles and e_t through a shared-memory ring, a second
//           warp forms p_t, and a chain warp whose lanes each own one output
//           element adds p_t V_t in position order, one fma per position
//           (attention.hpp:231-243).
//           The normaliser is the chunks' double sums added in chunk order
//           (a re-association of double additions of float terms: exact
//           whenever every term is a multiple of 2^-53 of the sum, and
//           otherwise within a few double ulps, far inside one float ulp of
//           1 / sum).
//
// SYN_ORDER_SPLIT: the p.V sums split over 256-position chunks on tensor
// cores and re-associated (about 1e-6 relative from the reference past one
// chunk, bit-exact up to kChunk positions). Two kernels, one CTA per (chunk,
// KV head, query); each CTA reads its chunk's K (then V) rows from HBM once,
// for all G = n_head / n_kv query heads of the group, all requested at once.
//   scores kernel: rotates q (and appends the new K, V rows), scores the
//            chunk, and writes the scores and the chunk's statistics: the
//            max m_j and the double sum s_j of expf(s - m_j), per query head;
//   p.V kernel (its V rows requested before it waits on the scores kernel):
//            merges every chunk's statistics, M = max m_j and sum =
//            sum_j s_j * exp(m_j - M) (with one chunk, the reference's sum
//            of expf(s - M) exactly), forms p_t = binary16(expf(s_t - M) *
//            (1 / sum)) and the chunk's partial sum of p_t V_t in position
//            order; the group's last CTA to finish adds the partials in
//            chunk order (deterministic).
// Either way the split depends on the context only (fixed chunks), never on
// the grid or the device, so any caller (a tensor-parallel rank included)
// splits the same context the same way.
#define SYN_DEVICE_EXPF  // softmax / silu: the device expf and its exception table
#include "common.cuh"
#include "internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <array>
#include <mutex>
#include <vector>

using namespace syn;

namespace {

constexpr int kThreads = 128;      // RoPE / append kernels
constexpr int kAttnThreads = 256;  // the decode kernel
constexpr int kChunk = 256;        // positions per CTA: a context of up to kChunk is one chunk (exact order)
static_assert(kChunk == kAttnThreads, "the p.V kernel gives each thread one position of its chunk");
constexpr int kPwStride = kChunk + 4;  // floats per head in the p buffer: heads 4 banks apart
constexpr int kSlotPos = 128;          // the score scratch's rows are padded to a multiple of this
constexpr uint64_t kAttnWaitNs = 2000000000ull;  // bounded waits on bulk copies give up after 2 s

__device__ unsigned g_attn_timeouts = 0;  // bounded waits that gave up (syn_device_errors)

struct AttnParams {
    const float *q, *k, *v;
    uint16_t *kc, *vc;
    const int32_t* pos;
    float* out;
    float* scores;           // scratch: [n_q][n_head][ld] scores (the exact order: then expf(s - M))
    double* st_s;            // scratch: [n_q][n_head][nch] chunk sums
    float* st_m;             // scratch: [n_q][n_head][nch] chunk maxima
    float* parts;            // scratch: [n_q][n_kv][nch][G * head_dim] chunk partials of p.V
    unsigned* ctr;           // scratch: [n_q][n_kv] arrivals of the p.V kernel's CTAs
    int nch;                 // chunks at max_len
    int ld;                  // floats per head in the score scratch (max_len rounded up to 64)
    int order;               // SYN_ORDER_REFERENCE / SYN_ORDER_SPLIT
    int v3d;                 // the exact p.V kernel's V tensor map has a query dimension (cache_stride != 0)
    const float* rope_tab;   // [max_len][head_dim / 2] (cos, sin), or NULL: computed in the kernel
    size_t cache_stride;
    int n_q, n_head, n_kv, hd, max_len;
    int append, rope, rope_mode;
    float theta_scale, scale;
    const float* ff;
    float yarn[5];
    int has_yarn;
    TpSync tp;               // push the output to every rank (a tensor-parallel gather point)
};

// The caller's scratch: scores, chunk statistics, chunk partials, counters.
struct AttnScratch {
    size_t scores, st_s, st_m, parts, ctr, total;
};
__host__ __device__ inline int score_ld(int max_len) { return (max_len + kSlotPos - 1) / kSlotPos * kSlotPos; }
AttnScratch scratch_layout(int n_q, int n_head, int n_kv, int hd, int max_len) {
    AttnScratch l;
    const size_t nch = size_t(max_len + kChunk - 1) / kChunk;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off = align256(off + bytes);
        return o;
    };
    l.scores = take(size_t(n_q) * n_head * score_ld(max_len) * 4);
    l.st_s = take(size_t(n_q) * n_head * nch * 8);
    l.st_m = take(size_t(n_q) * n_head * nch * 4);
    l.parts = take(size_t(n_q) * n_head * nch * hd * 4);
    l.ctr = take(size_t(n_q) * n_kv * 4);
    l.total = off;
    return l;
}

// 16-byte asynchronous copy global -> shared (the copy engine; no register
// round trip), and its group fences.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// cos and sin of pair i at position p (attention.hpp:102-119): theta built by
// repeated float multiplication, divided by the frequency factor, then the
// YaRN ramp (when enabled) and the magnitude scale.
__device__ __forceinline__ void rope_cs(const AttnParams& a, int p, int i, float& c, float& s) {
    float theta = float(p);
    for (int k = 0; k < i; ++k) theta = __fmul_rn(theta, a.theta_scale);
    const float ff = a.ff ? a.ff[i] : 1.0f;
    const float fs = a.has_yarn ? a.yarn[0] : 1.0f;
    const float theta_extrap = __fdiv_rn(theta, ff);
    const float theta_interp = __fmul_rn(fs, theta_extrap);
    float t = theta_interp;
    float mscale = a.has_yarn ? a.yarn[2] : 1.0f;
    if (a.has_yarn && a.yarn[1] != 0.0f) {
        const float den = fmaxf(0.001f, __fsub_rn(a.yarn[4], a.yarn[3]));
        const float y = __fdiv_rn(__fsub_rn(float(i), a.yarn[3]), den);
        const float ramp = __fmul_rn(__fsub_rn(1.0f, fminf(1.0f, fmaxf(0.0f, y))), a.yarn[1]);
        t = __fadd_rn(__fmul_rn(theta_interp, __fsub_rn(1.0f, ramp)), __fmul_rn(theta_extrap, ramp));
        mscale = __fmul_rn(mscale, __fadd_rn(1.0f, __fmul_rn(0.1f, logf(__fdiv_rn(1.0f, fs)))));
    }
    // cos and sin rounded once from double precision: the correctly rounded
    // float in all but rare cases, as close to a C runtime's cosf/sinf as a
    // float result can be (the reference calls std::cos / std::sin on float).
    c = __fmul_rn(float(cos(double(t))), mscale);
    s = __fmul_rn(float(sin(double(t))), mscale);
}

// Element indices of pair i: normal (2i, 2i+1), neox (i, i + hd/2).
__device__ __forceinline__ void pair_index(int mode, int hd, int i, int& i0, int& i1) {
    if (mode == 0) { i0 = 2 * i; i1 = 2 * i + 1; }
    else { i0 = i; i1 = i + hd / 2; }
}

__device__ __forceinline__ void rotate(float x0, float x1, float c, float s, float& o0, float& o1) {
    o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    o1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = f16_from_bits(uint16_t(w[e] & 0xffff));
        f[2 * e + 1] = f16_from_bits(uint16_t(w[e] >> 16));
    }
}

// Dynamic shared memory of the two kernels: the chunk's K (V) rows padded to
// hd + 8 halves (16-byte reads stay conflict-free), and the chunk's scores
// (p) of the G query heads.
struct ScoreSmem {
    size_t cs, qg, krh, sc, kt, total;
};
__host__ __device__ inline ScoreSmem score_smem(int GT, int hd) {
    ScoreSmem l;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off = (off + bytes + 15) & ~size_t(15);
        return o;
    };
    l.cs = take(size_t(hd) * 4);                   // cos, sin of the hd / 2 pairs
    l.qg = take(size_t(GT) * hd * 4);              // rotated q of the group, binary16 values
    l.krh = take(size_t(hd) * 2);                  // appended K row (binary16)
    l.sc = take(size_t(GT) * kChunk * 4);          // the chunk's scores
    l.kt = take(size_t(kChunk) * (hd + 8) * 2);    // the chunk's K rows
    l.total = off;
    return l;
}
struct PvSmem {
    size_t pw, vt, total;
};
__host__ __device__ inline PvSmem pv_smem(int GT, int hd) {
    PvSmem l;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off = (off + bytes + 15) & ~size_t(15);
        return o;
    };
    l.pw = take(size_t(GT) * kPwStride * 4);       // the chunk's p
    l.vt = take(size_t(kChunk) * (hd + 8) * 2);    // the chunk's V rows
    l.total = off;
    return l;
}

// Rows [t0, t1) of KV head g of a cache (row = n_kv * hd halves) into rows
// 0.. of dst (pitch hd + 8), except row `skip` (-1: none), as one group of
// asynchronous 16-byte copies.
__device__ inline void copy_rows(uint16_t* dst, const uint16_t* cache, size_t row, int g, int hd, int t0, int t1,
                                 int skip) {
    const int c8n = hd / 8, rowh = hd + 8, m = t1 - t0;
    const uint16_t* src = cache + size_t(g) * hd;
    if (kAttnThreads % c8n == 0) {  // every thread copies one fixed 16-byte column of rows tid / c8n, + step, ...
        const int c8 = threadIdx.x % c8n, step = kAttnThreads / c8n;
        for (int rr = threadIdx.x / c8n; rr < m; rr += step)
            if (t0 + rr != skip) cp_async16(dst + rr * rowh + c8 * 8, src + size_t(t0 + rr) * row + c8 * 8);
    } else {
        for (int i = threadIdx.x; i < m * c8n; i += kAttnThreads) {
            const int rr = i / c8n, c8 = i - rr * c8n;
            if (t0 + rr != skip) cp_async16(dst + rr * rowh + c8 * 8, src + size_t(t0 + rr) * row + c8 * 8);
        }
    }
    cp_async_commit();
}

// Tensor-core tiles for contexts beyond kChunk (where the reference's
// summation order is re-associated over chunks anyway): m16n8k16, binary16
// inputs (q, K, p and V are binary16 values already), fp32 accumulation.
// Fragment layouts (PTX ISA, mma.m16n8k16 .f16): lane = 4 g + t;
//   A: a0 = A[g][2t..2t+1], a1 = A[g+8][2t..], a2 = A[g][2t+8..], a3 = A[g+8][2t+8..]
//   B: b0 = B[2t..2t+1][g], b1 = B[2t+8..2t+9][g]
//   C: c0, c1 = C[g][2t], C[g][2t+1]; c2, c3 = C[g+8][...]
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {  // exact: both are binary16 values
    return uint32_t(f16_bits(lo)) | (uint32_t(f16_bits(hi)) << 16);
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t& r0, uint32_t& r1, const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(static_cast<unsigned>(__cvta_generic_to_shared(row_addr))));
}

// Kernel 1: the chunk's scores and statistics. CTA (j, g, b): positions
// [j * kChunk, ...) of query b's context, KV head g and its G query heads.
template <int GT>
__global__ void __launch_bounds__(kAttnThreads) attn_scores_kernel(AttnParams a) {
    const int j = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int hd = a.hd, G = a.n_head / a.n_kv, H = a.n_head;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // pos (and the RoPE table) are written before the step's first kernel, or
    // by the caller, never by the kernel this one may overlap: read before the wait.
    const int P = a.pos[b], L = P + 1;
    if (P < 0 || L > a.max_len) return;
    const int t0 = j * kChunk;
    if (t0 >= L) return;  // past the context (the p.V kernel skips it too)
    const int t1 = min(L, t0 + kChunk), n = t1 - t0;
    const bool owns = a.append && P < t1;  // the chunk holds the appended row

    extern __shared__ __align__(16) unsigned char smem[];
    const ScoreSmem sl = score_smem(GT, hd);
    float* cs = reinterpret_cast<float*>(smem + sl.cs);
    float* qg = reinterpret_cast<float*>(smem + sl.qg);
    uint16_t* krh = reinterpret_cast<uint16_t*>(smem + sl.krh);
    float* sc = reinterpret_cast<float*>(smem + sl.sc);  // score of head h, chunk row r: sc[h * kChunk + r]
    uint16_t* kt = reinterpret_cast<uint16_t*>(smem + sl.kt);
    __shared__ float2 etab[64];  // 2^(j/64) for exp_rn_neg
    if (tid < 64) etab[tid] = kExp2J64[tid];
    const int rowh = hd + 8, c8n = hd / 8;
    const size_t row = size_t(a.n_kv) * hd;
    uint16_t* kcb = a.kc + size_t(b) * a.cache_stride;
    uint16_t* vcb = a.vc + size_t(b) * a.cache_stride;

    // With append, rows other than P were written by earlier calls: their
    // copies start before the wait. Without it the caller's previous kernel
    // may have written them (syn_rope_kv_append), so everything waits.
    if (!a.append) pdl_wait();
    float2 cs_v = make_float2(0.0f, 0.0f);  // this thread's (cos, sin), requested before the copies
    if (a.rope && a.rope_tab && tid < hd / 2)
        cs_v = reinterpret_cast<const float2*>(a.rope_tab)[size_t(P) * (hd / 2) + tid];
    copy_rows(kt, kcb, row, g, hd, t0, t1, owns ? P : -1);
    if (a.rope) {
        if (a.rope_tab) {
            for (int i = tid; i < hd / 2; i += kAttnThreads) {
                const float2 v = i == tid ? cs_v : reinterpret_cast<const float2*>(a.rope_tab)[size_t(P) * (hd / 2) + i];
                cs[2 * i] = v.x;
                cs[2 * i + 1] = v.y;
            }
        } else {
            for (int i = tid; i < hd / 2; i += kAttnThreads) rope_cs(a, P, i, cs[2 * i], cs[2 * i + 1]);
        }
    }
    pdl_launch_dependents();  // the p.V kernel may request its V rows now
    if (a.append) pdl_wait();  // q, k, v come from the previous kernel
    // the p.V kernel's arrivals for this group, re-armed here: the previous
    // call's p.V kernel has completed once the wait above has returned
    if (j == 0 && tid == 0) a.ctr[size_t(b) * a.n_kv + g] = 0u;
    __syncthreads();

    const float* qb = a.q + (size_t(b) * H + size_t(g) * G) * hd;
    if (a.rope) {
        for (int i = tid; i < G * hd / 2; i += kAttnThreads) {
            const int jh = i / (hd / 2), pi = i % (hd / 2);
            int i0, i1;
            pair_index(a.rope_mode, hd, pi, i0, i1);
            float o0, o1;
            rotate(qb[jh * hd + i0], qb[jh * hd + i1], cs[2 * pi], cs[2 * pi + 1], o0, o1);
            qg[jh * hd + i0] = round_f16(o0);
            qg[jh * hd + i1] = round_f16(o1);
        }
    } else {
        for (int i = tid; i < G * hd; i += kAttnThreads) qg[i] = round_f16(qb[i]);
    }
    if (owns) {
        const float* kb = a.k + size_t(b) * row + size_t(g) * hd;
        const float* vb = a.v + size_t(b) * row + size_t(g) * hd;
        uint16_t* krow = kcb + size_t(P) * row + size_t(g) * hd;
        uint16_t* vrow = vcb + size_t(P) * row + size_t(g) * hd;
        if (a.rope) {
            for (int pi = tid; pi < hd / 2; pi += kAttnThreads) {
                int i0, i1;
                pair_index(a.rope_mode, hd, pi, i0, i1);
                float o0, o1;
                rotate(kb[i0], kb[i1], cs[2 * pi], cs[2 * pi + 1], o0, o1);
                const uint16_t h0 = f16_bits(o0), h1 = f16_bits(o1);
                krow[i0] = h0;
                krow[i1] = h1;
                krh[i0] = h0;
                krh[i1] = h1;
            }
        } else {
            for (int d = tid; d < hd; d += kAttnThreads) krow[d] = krh[d] = f16_bits(kb[d]);
        }
        for (int d = tid; d < hd; d += kAttnThreads) vrow[d] = f16_bits(vb[d]);
    }
    __syncthreads();

    // The tensor-core path (a context of several chunks): q of head g as A
    // fragments, all head_dim / 16 k-steps.
    const bool tc = L > kChunk && hd % 16 == 0 && hd <= 128 && G <= 8;
    const int gq = lane >> 2, tq = lane & 3;
    uint32_t qa[16];  // per k-step (head_dim <= 128): a0 (row gq, k 2tq..), a2 (row gq, k 2tq+8..)
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        qa[2 * ks] = qa[2 * ks + 1] = 0u;
        if (tc && ks < hd / 16 && gq < G) {
            const float* qr = qg + gq * hd + 16 * ks + 2 * tq;
            qa[2 * ks] = pack_h2(qr[0], qr[1]);
            qa[2 * ks + 1] = pack_h2(qr[8], qr[9]);
        }
    }
    cp_async_wait_all();
    if (owns && tid < c8n)
        *reinterpret_cast<uint4*>(kt + (P - t0) * rowh + tid * 8) = *reinterpret_cast<const uint4*>(krh + tid * 8);
    __syncthreads();

    // Scores: the dot runs in dimension order (attention.hpp:214-219); the
    // tensor-core lanes keep the max of the scores they produce (lmx).
    float lmx = -INFINITY;
    if (tc) {
        // warp w scores rows 32w .. 32w + 31 as four tiles of 8 positions x all G heads,
        // interleaved (four independent accumulators): C[h][n] = sum_k q[h][k] K[n][k]
        float cacc[4][4];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) cacc[q4][0] = cacc[q4][1] = cacc[q4][2] = cacc[q4][3] = 0.0f;
        if (32 * warp < n) {
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                if (ks < hd / 16) {
                    const uint32_t af[4] = {qa[2 * ks], 0u, qa[2 * ks + 1], 0u};
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        // B: rows past n read stale data (inside the buffer), never stored
                        const uint16_t* krow = kt + (32 * warp + 8 * q4 + gq) * rowh + 2 * tq + 16 * ks;
                        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow);
                        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + 8);
                        mma16816(cacc[q4], af, b0, b1);
                    }
                }
            }
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            const int n0 = 32 * warp + 8 * q4;
            if (gq < G && n0 < n) {
                const int r0 = n0 + 2 * tq;
                const float v0 = __fmul_rn(cacc[q4][0], a.scale), v1 = __fmul_rn(cacc[q4][1], a.scale);
                if (r0 < n) {
                    sc[gq * kChunk + r0] = v0;
                    lmx = fmaxf(lmx, v0);
                }
                if (r0 + 1 < n) {
                    sc[gq * kChunk + r0 + 1] = v1;
                    lmx = fmaxf(lmx, v1);
                }
            }
        }
    } else {
        for (int i = tid; i < n * G; i += kAttnThreads) {
            const int jh = i / n, r = i % n;
            const uint16_t* kr = kt + r * rowh;
            const float4* qh = reinterpret_cast<const float4*>(qg + jh * hd);
            float dot = 0.0f;
#pragma unroll 4
            for (int d8 = 0; d8 < hd / 8; ++d8) {
                float kf[8];
                unpack8(*reinterpret_cast<const uint4*>(kr + 8 * d8), kf);
                const float4 q0 = qh[2 * d8], q1 = qh[2 * d8 + 1];
                dot = fmaf(q0.x, kf[0], dot);  // exact products: each fma is mul then add
                dot = fmaf(q0.y, kf[1], dot);
                dot = fmaf(q0.z, kf[2], dot);
                dot = fmaf(q0.w, kf[3], dot);
                dot = fmaf(q1.x, kf[4], dot);
                dot = fmaf(q1.y, kf[5], dot);
                dot = fmaf(q1.z, kf[6], dot);
                dot = fmaf(q1.w, kf[7], dot);
            }
            sc[jh * kChunk + r] = __fmul_rn(dot, a.scale);
        }
    }
    __syncthreads();

    // The chunk's statistics per query head (elementwise.hpp:174-201): the
    // max m_j, then the double sum s_j of expf(s - m_j) over positions
    // tid, + 256, ..., partials meeting in lane and warp order.
    __shared__ float red_mx[GT][kAttnThreads / 32];
    __shared__ double red_sm[GT][kAttnThreads / 32];
    __shared__ float m_loc[GT];
    if (tc) {
        float w = fmaxf(lmx, __shfl_xor_sync(0xffffffffu, lmx, 1));
        w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, 2));
        if (tq == 0 && gq < G) red_mx[gq][warp] = w;
    } else {
#pragma unroll 1
        for (int h = 0; h < G; ++h) {
            float mx = -INFINITY;
            for (int t = tid; t < n; t += kAttnThreads) mx = fmaxf(mx, sc[h * kChunk + t]);
            mx = warp_max(mx);
            if (lane == 0) red_mx[h][warp] = mx;
        }
    }
    __syncthreads();
    if (tid < G) {
        float m = -INFINITY;
        for (int w = 0; w < kAttnThreads / 32; ++w) m = fmaxf(m, red_mx[tid][w]);
        m_loc[tid] = m;
    }
    __syncthreads();
    {
        double acc[GT];
        float mh[GT];
#pragma unroll
        for (int h = 0; h < GT; ++h) {
            acc[h] = 0.0;
            mh[h] = h < G ? m_loc[h] : 0.0f;
        }
        for (int t = tid; t < n; t += kAttnThreads) {
#pragma unroll
            for (int h = 0; h < GT; ++h)
                if (h < G) acc[h] += double(exp_rn_neg(__fsub_rn(sc[h * kChunk + t], mh[h]), etab));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int h = 0; h < GT; ++h) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], o);
        }
        if (lane < G) {
            double v = 0.0;
#pragma unroll
            for (int h = 0; h < GT; ++h)
                if (h == lane) v = acc[h];
            red_sm[lane][warp] = v;
        }
    }
    __syncthreads();
    const size_t hb = size_t(b) * H + size_t(g) * G;  // first query head of the group
    if (tid < G) {
        double sum = 0.0;
        for (int w = 0; w < kAttnThreads / 32; ++w) sum += red_sm[tid][w];
        a.st_m[(hb + tid) * a.nch + j] = m_loc[tid];
        a.st_s[(hb + tid) * a.nch + j] = sum;
    }
#pragma unroll 1
    for (int h = 0; h < G; ++h)
        for (int t = tid; t < n; t += kAttnThreads) a.scores[(hb + h) * a.ld + t0 + t] = sc[h * kChunk + t];
}

// Kernel 2: p and p.V of the chunk, and the group's output.
template <int GT>
__global__ void __launch_bounds__(kAttnThreads) attn_pv_kernel(AttnParams a) {
    const int j = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int hd = a.hd, G = a.n_head / a.n_kv, H = a.n_head;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = a.pos[b], L = P + 1;
    if (P < 0 || L > a.max_len) return;
    const int t0 = j * kChunk;
    if (t0 >= L) return;
    const int t1 = min(L, t0 + kChunk), n = t1 - t0, nchk = (L + kChunk - 1) / kChunk;
    const bool owns = a.append && P < t1;

    extern __shared__ __align__(16) unsigned char smem[];
    const PvSmem sl = pv_smem(GT, hd);
    float* pw = reinterpret_cast<float*>(smem + sl.pw);  // p of head h, chunk row r: pw[h * kPwStride + r]
    uint16_t* vt = reinterpret_cast<uint16_t*>(smem + sl.vt);
    __shared__ float gm[GT], gscale[GT];
    __shared__ float2 etab[64];
    __shared__ bool last;
    if (tid < 64) etab[tid] = kExp2J64[tid];
    const int rowh = hd + 8, c8n = hd / 8;
    const size_t row = size_t(a.n_kv) * hd;
    const uint16_t* vcb = a.vc + size_t(b) * a.cache_stride;
    if (!a.append) pdl_wait();
    copy_rows(vt, vcb, row, g, hd, t0, t1, owns ? P : -1);  // row P comes from v below
    pdl_launch_dependents();
    pdl_wait();  // the scores kernel: scores, statistics, counters, cache rows

    // This thread's position t0 + tid: its scores, requested before the merge.
    const size_t hb = size_t(b) * H + size_t(g) * G;
    float sv[GT];
#pragma unroll
    for (int h = 0; h < GT; ++h)
        sv[h] = h < G && tid < n ? a.scores[(hb + h) * a.ld + t0 + tid] : 0.0f;

    // The context's max M and normaliser sum_j s_j * exp(m_j - M), one warp
    // per query head over the chunks (each lane loads its chunks' statistics
    // once). With one chunk the weight is exactly 1 and the sum is the
    // reference's sum of expf(s - M); with several, the chunks' weights and
    // their sum order are the approximation of the re-associated sum.
    for (int h = warp; h < G; h += kAttnThreads / 32) {
        const float* mj = a.st_m + (hb + h) * a.nch;
        const double* sj = a.st_s + (hb + h) * a.nch;
        constexpr int kHeld = 4;  // chunks per lane held in registers (all of them up to 128 chunks)
        float mr[kHeld];
        double sr[kHeld];
        float M = -INFINITY;
#pragma unroll
        for (int u = 0; u < kHeld; ++u) {
            const int r = lane + 32 * u;
            mr[u] = r < nchk ? mj[r] : -INFINITY;
            sr[u] = r < nchk ? sj[r] : 0.0;
        }
#pragma unroll
        for (int u = 0; u < kHeld; ++u) M = fmaxf(M, mr[u]);
        for (int r = lane + 32 * kHeld; r < nchk; r += 32) M = fmaxf(M, mj[r]);
        M = warp_max(M);
        double tot = 0.0;
#pragma unroll
        for (int u = 0; u < kHeld; ++u)
            if (sr[u] > 0.0) tot += sr[u] * double(mr[u] == M ? 1.0f : expf(__fsub_rn(mr[u], M)));
        for (int r = lane + 32 * kHeld; r < nchk; r += 32) {
            const float m = mj[r];
            const double sum = sj[r];
            if (sum > 0.0) tot += sum * double(m == M ? 1.0f : expf(__fsub_rn(m, M)));
        }
        tot = warp_sum_d(tot);
        if (lane == 0) {
            gm[h] = M;
            gscale[h] = float(1.0 / tot);
        }
    }
    __syncthreads();
    // p_t = binary16(expf(s_t - M) * (1 / sum)) of the chunk
    if (tid < n) {
#pragma unroll
        for (int h = 0; h < GT; ++h)
            if (h < G) pw[h * kPwStride + tid] = round_f16(__fmul_rn(exp_rn_neg(__fsub_rn(sv[h], gm[h]), etab), gscale[h]));
    }
    const bool tc = L > kChunk && hd % 16 == 0 && hd <= 128 && G <= 8;
    cp_async_wait_all();
    if (owns) {  // the appended row, rounded as the scores kernel stored it
        const float* vb = a.v + size_t(b) * row + size_t(g) * hd;
        for (int d = tid; d < hd; d += kAttnThreads) vt[(P - t0) * rowh + d] = f16_bits(vb[d]);
    }
    if (tc) {  // rows past n up to the next 16: V = 0 (stale bits could be a NaN; their p is 0)
        const int pad = ((n + 15) & ~15) - n;
        for (int i = tid; i < pad * c8n; i += kAttnThreads)
            *reinterpret_cast<uint4*>(vt + (n + i / c8n) * rowh + (i % c8n) * 8) = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();

    // The chunk's partial sum of p_t V_t.
    float* part = a.parts + ((size_t(b) * a.n_kv + g) * a.nch + j) * size_t(G) * hd;
    if (tc) {
        // warp w takes positions 32w .. 32w + 31 (two k-steps) of every head_dim column
        // (hd / 8 tiles of 8, independent accumulators): C[h][d] += sum_k p[h][k] V[k][d];
        // then the eight warps' sums are added in warp order through shared memory
        const int gq = lane >> 2, tq = lane & 3, r0 = 32 * warp;
        float vacc[16][4];
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) vacc[nt][0] = vacc[nt][1] = vacc[nt][2] = vacc[nt][3] = 0.0f;
#pragma unroll
        for (int ks2 = 0; ks2 < 2; ++ks2) {
            const int rk = r0 + 16 * ks2;
            if (rk < n) {  // rows past n up to the next 16 are zero; later k-steps are skipped
                uint32_t af[4] = {0u, 0u, 0u, 0u};
                if (gq < G) {
                    const int r = rk + 2 * tq;  // p past row n is 0
                    const float* pr = pw + gq * kPwStride + r;
                    af[0] = pack_h2(r < n ? pr[0] : 0.0f, r + 1 < n ? pr[1] : 0.0f);
                    af[2] = pack_h2(r + 8 < n ? pr[8] : 0.0f, r + 9 < n ? pr[9] : 0.0f);
                }
                // lanes 0-7: rows rk..rk+7 at column 8nt; lanes 8-15: rows rk+8..rk+15
                const uint16_t* vrow = vt + (rk + (lane & 15)) * rowh;
#pragma unroll
                for (int nt = 0; nt < 16; ++nt) {
                    if (nt < hd / 8) {
                        uint32_t b0, b1;
                        ldsm_x2_trans(b0, b1, vrow + 8 * nt);
                        mma16816(vacc[nt], af, b0, b1);
                    }
                }
            }
        }
        __syncthreads();  // every warp is done with the V rows: their buffer holds the warps' sums next
        float* red = reinterpret_cast<float*>(vt);  // [warp][G * hd]
        const int n_out = G * hd;
        if (gq < G) {
#pragma unroll
            for (int nt = 0; nt < 16; ++nt) {
                if (nt < hd / 8) {
                    const int o = gq * hd + 8 * nt + 2 * tq;
                    red[warp * n_out + o] = vacc[nt][0];
                    red[warp * n_out + o + 1] = vacc[nt][1];
                }
            }
        }
        __syncthreads();
        for (int o = tid; o < n_out; o += kAttnThreads) {
            float sum = 0.0f;
#pragma unroll
            for (int w = 0; w < kAttnThreads / 32; ++w) sum = __fadd_rn(sum, red[w * n_out + o]);
            part[o] = sum;
        }
    } else {
        // thread slot k owns the column pair (2 * (o % (hd / 2)), +1) of query head o / (hd / 2)
        constexpr int KO = GT >= 2 ? GT / 2 : 1;  // pairs per thread: G * hd / 2 <= GT * 128 pairs over 256 threads
        float acc0[KO], acc1[KO];
        int pcol[KO], prow[KO];
        const int n_pairs = G * hd / 2;
#pragma unroll
        for (int k = 0; k < KO; ++k) {
            const int o = tid + k * kAttnThreads;
            acc0[k] = acc1[k] = 0.0f;
            pcol[k] = o < n_pairs ? 2 * (o % (hd / 2)) : -1;
            prow[k] = o < n_pairs ? (o / (hd / 2)) * kPwStride : 0;
        }
#pragma unroll 4
        for (int r = 0; r < n; ++r) {
            const uint16_t* vr = vt + r * rowh;
#pragma unroll
            for (int k = 0; k < KO; ++k) {
                if (pcol[k] >= 0) {
                    const float p = pw[prow[k] + r];
                    const uint32_t v2 = *reinterpret_cast<const uint32_t*>(vr + pcol[k]);
                    acc0[k] = fmaf(p, f16_from_bits(uint16_t(v2 & 0xffff)), acc0[k]);  // exact products
                    acc1[k] = fmaf(p, f16_from_bits(uint16_t(v2 >> 16)), acc1[k]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < KO; ++k) {
            if (pcol[k] >= 0) {
                const int o = 2 * (tid + k * kAttnThreads);  // head * hd + pcol[k]
                part[o] = acc0[k];
                part[o + 1] = acc1[k];
            }
        }
    }

    // The group's last CTA to finish adds the chunks' partials in chunk order.
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&a.ctr[size_t(b) * a.n_kv + g], 1u) == unsigned(nchk - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int n_out = G * hd;
    const float* pb = a.parts + (size_t(b) * a.n_kv + g) * a.nch * size_t(n_out);
    float* ob = a.out + hb * hd;
    const unsigned ep = a.tp.peers ? *reinterpret_cast<const volatile unsigned*>(a.tp.epoch) : 0u;
    for (int i = tid; i < n_out; i += kAttnThreads) {
        float sum = 0.0f;
        int r = 0;
        for (; r + 16 <= nchk; r += 16) {  // sixteen loads in flight, added in chunk order
            float v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = __ldcg(pb + size_t(r + u) * n_out + i);
#pragma unroll
            for (int u = 0; u < 16; ++u) sum = __fadd_rn(sum, v[u]);
        }
        for (; r < nchk; ++r) sum = __fadd_rn(sum, __ldcg(pb + size_t(r) * n_out + i));
        if (a.tp.peers) tp_store(a.tp, hb * hd + i, sum, ep);
        else ob[i] = sum;
    }
}

// ---- the reference's order at any length (SYN_ORDER_REFERENCE) ------------------

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, bool three,
                                            uint64_t* bar) {
    if (three)
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
            "%4}], [%5];" ::"r"(smem_addr(dst)),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
            : "memory");
    else
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
            "%3}], [%4];" ::"r"(smem_addr(dst)),
            "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
            : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Shared memory of the exact scores kernel: cos/sin, the group's rotated q
// (binary16 values, held as floats), the appended K row, and the chunk's K rows: with SWZ (head_dim a
// multiple of 64) as tensor-TMA tiles of 64 rows x 64 columns in the 128-byte
// swizzle (16-byte piece c of row r at piece c ^ (r % 8), so consecutive
// threads' 16-byte reads of their own rows hit distinct banks), [quarter of 64
// rows][64-column box][row] x 128 bytes from a 1 KB boundary; otherwise rows
// of hd + 8 halves filled by 16-byte copies (the padding spreads the banks).
struct XsSmem {
    size_t cs, qh, krh, kt, total;
};
__host__ __device__ inline XsSmem xs_smem(int GT, int hd, bool swz) {
    XsSmem l;
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) {
        off = (off + align - 1) & ~(align - 1);
        const size_t o = off;
        off += bytes;
        return o;
    };
    l.cs = take(size_t(hd) * 4, 16);
    l.qh = take(size_t(GT) * hd * 4, 16);
    l.krh = take(size_t(hd) * 2, 16);
    l.kt = swz ? take(size_t(kChunk) * hd * 2, 1024) : take(size_t(kChunk) * (hd + 8) * 2, 16);
    l.total = ((off + 15) & ~size_t(15)) + (swz ? 1024 : 0);  // + the 1 KB alignment of the dynamic base
    return l;
}

// Exact scores of one chunk: CTA (j, g, b), thread r = position t0 + r.
template <int GT, bool SWZ>
__global__ void __launch_bounds__(kAttnThreads) attn_xs_kernel(AttnParams a, const __grid_constant__ CUtensorMap kmap) {
    const int j = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int hd = a.hd, G = a.n_head / a.n_kv, H = a.n_head;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = a.pos[b], L = P + 1;
    if (P < 0 || L > a.max_len) return;
    const int t0 = j * kChunk;
    if (t0 >= L) return;
    const int t1 = min(L, t0 + kChunk), n = t1 - t0;
    const bool owns = a.append && P < t1;  // the chunk holds the appended row

    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char* smem = SWZ ? smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u) : smem_raw;
    const XsSmem sl = xs_smem(GT, hd, SWZ);
    float* cs = reinterpret_cast<float*>(smem + sl.cs);
    float* qf = reinterpret_cast<float*>(smem + sl.qh);
    uint16_t* krh = reinterpret_cast<uint16_t*>(smem + sl.krh);
    uint16_t* kt = reinterpret_cast<uint16_t*>(smem + sl.kt);
    __shared__ __align__(8) uint64_t bar[kAttnThreads / 64];  // SWZ: one per 64 rows
    __shared__ float red[GT][kAttnThreads / 32];
    __shared__ int bad;
    const int rowh = hd + 8, nbx = hd / 64;
    const size_t row = size_t(a.n_kv) * hd;
    uint16_t* kcb = a.kc + size_t(b) * a.cache_stride;
    uint16_t* vcb = a.vc + size_t(b) * a.cache_stride;
    if (SWZ && tid < kAttnThreads / 64) mbar_init(&bar[tid], 1);
    if (tid == 0) bad = 0;
    mbar_init_fence();
    __syncthreads();

    // With append, rows other than P were written by earlier calls: their
    // copies start before the wait (row P's stale copy is overwritten below).
    // Without it the caller's previous kernel may have written them
    // (syn_rope_kv_append), so everything waits.
    if (!a.append) pdl_wait();
    float2 cs_v = make_float2(0.0f, 0.0f);
    if (a.rope && a.rope_tab && tid < hd / 2)
        cs_v = reinterpret_cast<const float2*>(a.rope_tab)[size_t(P) * (hd / 2) + tid];
    if (SWZ) {
        if (tid == 0)
            for (int q = 0; q * 64 < n; ++q) {
                mbar_expect_tx(&bar[q], uint32_t(nbx) * 64u * 128u);
                for (int bx = 0; bx < nbx; ++bx)
                    tma_load_3d(smem + sl.kt + (size_t(q) * nbx + bx) * 64 * 128, &kmap, g * hd + 64 * bx,
                                t0 + 64 * q, a.v3d ? b : 0, a.v3d != 0, &bar[q]);
            }
    } else {
        copy_rows(kt, kcb, row, g, hd, t0, t1, owns ? P : -1);
    }
    if (a.rope) {
        if (a.rope_tab) {
            for (int i = tid; i < hd / 2; i += kAttnThreads) {
                const float2 v = i == tid ? cs_v : reinterpret_cast<const float2*>(a.rope_tab)[size_t(P) * (hd / 2) + i];
                cs[2 * i] = v.x;
                cs[2 * i + 1] = v.y;
            }
        } else {
            for (int i = tid; i < hd / 2; i += kAttnThreads) rope_cs(a, P, i, cs[2 * i], cs[2 * i + 1]);
        }
    }
    pdl_launch_dependents();
    if (a.append) pdl_wait();  // q, k, v come from the previous kernel
    __syncthreads();

    // q of the group rotated and rounded to binary16 (attention.hpp:205-207)
    const float* qb = a.q + (size_t(b) * H + size_t(g) * G) * hd;
    if (a.rope) {
        for (int i = tid; i < G * hd / 2; i += kAttnThreads) {
            const int jh = i / (hd / 2), pi = i % (hd / 2);
            int i0, i1;
            pair_index(a.rope_mode, hd, pi, i0, i1);
            float o0, o1;
            rotate(qb[jh * hd + i0], qb[jh * hd + i1], cs[2 * pi], cs[2 * pi + 1], o0, o1);
            qf[jh * hd + i0] = round_f16(o0);
            qf[jh * hd + i1] = round_f16(o1);
        }
    } else {
        for (int i = tid; i < G * hd; i += kAttnThreads) qf[i] = round_f16(qb[i]);
    }
    if (owns) {  // kv_append (attention.hpp:165-175): the rotated k and v as binary16 into row P
        const float* kb = a.k + size_t(b) * row + size_t(g) * hd;
        const float* vb = a.v + size_t(b) * row + size_t(g) * hd;
        uint16_t* krow = kcb + size_t(P) * row + size_t(g) * hd;
        uint16_t* vrow = vcb + size_t(P) * row + size_t(g) * hd;
        if (a.rope) {
            for (int pi = tid; pi < hd / 2; pi += kAttnThreads) {
                int i0, i1;
                pair_index(a.rope_mode, hd, pi, i0, i1);
                float o0, o1;
                rotate(kb[i0], kb[i1], cs[2 * pi], cs[2 * pi + 1], o0, o1);
                const uint16_t h0 = f16_bits(o0), h1 = f16_bits(o1);
                krow[i0] = h0;
                krow[i1] = h1;
                krh[i0] = h0;
                krh[i1] = h1;
            }
        } else {
            for (int d = tid; d < hd; d += kAttnThreads) krow[d] = krh[d] = f16_bits(kb[d]);
        }
        for (int d = tid; d < hd; d += kAttnThreads) vrow[d] = f16_bits(vb[d]);
    }
    if (SWZ) {
        if (tid < n && !mbar_wait_bounded(&bar[tid >> 6], 0, kAttnWaitNs)) {
            atomicAdd(&g_attn_timeouts, 1u);
            bad = 1;
        }
    } else {
        cp_async_wait_all();
    }
    __syncthreads();
    if (bad) return;
    if (owns && tid < hd / 8) {  // the appended row over its stale copy
        const int r = P - t0;
        uint4* dst = SWZ ? reinterpret_cast<uint4*>(smem + sl.kt +
                                                    (((size_t(r >> 6) * nbx + (tid >> 3)) * 64 + (r & 63)) * 128) +
                                                    ((((tid & 7) ^ (r & 7))) << 4))
                         : reinterpret_cast<uint4*>(kt + r * rowh + tid * 8);
        *dst = *reinterpret_cast<const uint4*>(krh + tid * 8);
    }
    __syncthreads();

    // s_t = (q . K_t) * scale, each head's dot in dimension order (attention.hpp:214-220);
    // each K value widened once for the group's heads, every product exact
    const size_t hb = size_t(b) * H + size_t(g) * G;
    float acc[GT];
#pragma unroll
    for (int h = 0; h < GT; ++h) acc[h] = 0.0f;
    if (tid < n) {
        const uint4* kr = reinterpret_cast<const uint4*>(kt + tid * rowh);
        const unsigned char* ks = smem + sl.kt + ((size_t(tid >> 6) * nbx) * 64 + (tid & 63)) * 128;
#pragma unroll 2
        for (int d8 = 0; d8 < hd / 8; ++d8) {
            const uint4 kv = SWZ ? *reinterpret_cast<const uint4*>(ks + (d8 >> 3) * (64 * 128) +
                                                                   (((d8 & 7) ^ (tid & 7)) << 4))
                                 : kr[d8];
            float kf[8];
            unpack8(kv, kf);
#pragma unroll
            for (int h = 0; h < GT; ++h) {
                if (h < G) {
                    const float4 q0 = reinterpret_cast<const float4*>(qf + h * hd)[2 * d8];
                    const float4 q1 = reinterpret_cast<const float4*>(qf + h * hd)[2 * d8 + 1];
                    float c = acc[h];
                    c = fmaf(q0.x, kf[0], c);
                    c = fmaf(q0.y, kf[1], c);
                    c = fmaf(q0.z, kf[2], c);
                    c = fmaf(q0.w, kf[3], c);
                    c = fmaf(q1.x, kf[4], c);
                    c = fmaf(q1.y, kf[5], c);
                    c = fmaf(q1.z, kf[6], c);
                    c = fmaf(q1.w, kf[7], c);
                    acc[h] = c;
                }
            }
        }
    }
#pragma unroll
    for (int h = 0; h < GT; ++h) {
        if (h < G) {
            const float sv = __fmul_rn(acc[h], a.scale);
            if (tid < n) a.scores[(hb + h) * a.ld + t0 + tid] = sv;
            const float m = warp_max(tid < n ? sv : -INFINITY);
            if (lane == 0) red[h][warp] = m;
        }
    }
    __syncthreads();
    if (tid < G) {
        float m = -INFINITY;
        for (int w = 0; w < kAttnThreads / 32; ++w) m = fmaxf(m, red[tid][w]);
        a.st_m[(hb + tid) * a.nch + j] = m;
    }
}

// e_t = expf(s_t - M) of one chunk (in place) and the chunk's double sums:
// CTA (j, g, b), thread r = position t0 + r (elementwise.hpp:174-191).
template <int GT>
__global__ void __launch_bounds__(kAttnThreads) attn_xe_kernel(AttnParams a) {
    const int j = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int G = a.n_head / a.n_kv, H = a.n_head;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = a.pos[b], L = P + 1;
    if (P < 0 || L > a.max_len) return;
    const int t0 = j * kChunk;
    if (t0 >= L) return;
    const int n = min(L, t0 + kChunk) - t0, nchk = (L + kChunk - 1) / kChunk;
    __shared__ float gm[GT];
    __shared__ double red[GT][kAttnThreads / 32];
    __shared__ float2 etab[64];
    if (tid < 64) etab[tid] = kExp2J64[tid];
    pdl_launch_dependents();
    pdl_wait();  // the scores and chunk maxima
    const size_t hb = size_t(b) * H + size_t(g) * G;
    float sv[GT];
#pragma unroll
    for (int h = 0; h < GT; ++h) sv[h] = h < G && tid < n ? a.scores[(hb + h) * a.ld + t0 + tid] : 0.0f;
    for (int h = warp; h < G; h += kAttnThreads / 32) {  // M = the largest score (exact in any order)
        float m = -INFINITY;
        for (int c = lane; c < nchk; c += 32) m = fmaxf(m, a.st_m[(hb + h) * a.nch + c]);
        m = warp_max(m);
        if (lane == 0) gm[h] = m;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < GT; ++h) {
        if (h < G) {
            double e = 0.0;
            if (tid < n) {
                const float ev = exp_rn_neg(__fsub_rn(sv[h], gm[h]), etab);
                a.scores[(hb + h) * a.ld + t0 + tid] = ev;
                e = double(ev);
            }
            e = warp_sum_d(e);
            if (lane == 0) red[h][warp] = e;
        }
    }
    __syncthreads();
    if (tid < G) {
        double sum = 0.0;
        for (int w = 0; w < kAttnThreads / 32; ++w) sum += red[tid][w];
        a.st_s[(hb + tid) * a.nch + j] = sum;
    }
}

// Shared memory of the exact p.V kernel: a ring of kNr slots, each the V tile
// of kVSlot positions x 32 columns (binary16, as the tensor copy lands it),
// e_t and p_t of those positions; then the barriers.
constexpr int kVSlot = kSlotPos;  // positions per slot (128)
constexpr int kNr = 6;            // slots (768 positions in flight)
constexpr size_t kXvSmemMost = size_t(120) << 10;  // the p.V kernel's dynamic shared memory when it takes an SM alone
struct XvSmem {
    static constexpr size_t v16 = 0;                                // [kNr][kVSlot][32] binary16
    static constexpr size_t es = v16 + size_t(kNr) * kVSlot * 64;   // [kNr][kVSlot] e_t
    static constexpr size_t p32 = es + size_t(kNr) * kVSlot * 4;    // [kNr][kVSlot] p_t as floats
    static constexpr size_t bars = p32 + size_t(kNr) * kVSlot * 4;  // vfull, efull, pfull, empty: [kNr] each
    static constexpr size_t total = bars + size_t(4 * kNr) * 8 + 1024;  // + the ring's alignment
};

// p.V in position order over 32 output columns of one query head: CTA (h *
// ns + c, b), ns = ceil(head_dim / 32). Three warps:
//   warp 0, chain:    lane = output column 32 c + lane; acc = fma(p_t,
//                     V_t,d, acc) for t in order (attention.hpp:231-243;
//                     each product is exact, so the fma rounds exactly where
//                     the reference's add does). V comes straight from the
//                     ring as binary16, 16 positions loaded (and widened)
//                     ahead of the fmas;
//   warp 1, producer: one tensor copy of the V tile and one bulk copy of e_t
//                     per kVSlot positions;
//   warp 2, p:        p_t = binary16(e_t * scale) (elementwise.hpp:194-197,
//                     attention.hpp:224-227), scale = float(1 / sum) with sum
//                     the exp kernel's chunk sums added in chunk order
//                     (elementwise.hpp:190-193); p_t = 0 and V rows zeroed past
//                     the context, so that every slot runs whole (fma(0, 0,
//                     acc) = acc).
__global__ void __launch_bounds__(96) attn_xv_kernel(AttnParams a, const __grid_constant__ CUtensorMap vmap) {
    const int G = a.n_head / a.n_kv, H = a.n_head, hd = a.hd, ns = (hd + 31) / 32;
    const int h = blockIdx.x / ns, c = blockIdx.x % ns, g = h / G, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = a.pos[b], L = P + 1;
    if (P < 0 || L > a.max_len) return;
    const int nslot = (L + kVSlot - 1) / kVSlot, nchk = (L + kChunk - 1) / kChunk;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    // tensor copies land 128-byte aligned: the ring starts at the next 1 KB boundary
    unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint16_t* v16 = reinterpret_cast<uint16_t*>(smem + XvSmem::v16);
    float* es = reinterpret_cast<float*>(smem + XvSmem::es);
    float* p32 = reinterpret_cast<float*>(smem + XvSmem::p32);
    uint64_t* vfull = reinterpret_cast<uint64_t*>(smem + XvSmem::bars);
    uint64_t* efull = vfull + kNr;
    uint64_t* pfull = efull + kNr;
    uint64_t* empty = pfull + kNr;
    __shared__ int abort_flag, issued;
    if (tid < kNr) {
        mbar_init(&vfull[tid], 1);
        mbar_init(&efull[tid], 1);
        mbar_init(&pfull[tid], 1);
        mbar_init(&empty[tid], 1);
    }
    if (tid == 0) abort_flag = issued = 0;
    mbar_init_fence();
    __syncthreads();

    const size_t hb = size_t(b) * H + size_t(h);  // this CTA's query head
    const int vx = g * hd + 32 * c, vz = a.v3d ? b : 0;
    auto issue_v = [&](int k) {
        uint64_t* bar = &vfull[k % kNr];
        mbar_expect_tx(bar, uint32_t(kVSlot) * 64u);
        tma_load_3d(v16 + size_t(k % kNr) * kVSlot * 32, &vmap, vx, k * kVSlot, vz, a.v3d != 0, bar);
    };
    auto issue_e = [&](int k) {  // ld is a multiple of kVSlot: the slot's e_t lie inside the row
        uint64_t* bar = &efull[k % kNr];
        mbar_expect_tx(bar, kVSlot * 4u);
        bulk_copy_g2s(es + size_t(k % kNr) * kVSlot, a.scores + hb * a.ld + size_t(k) * kVSlot, kVSlot * 4u, bar);
    };
    // A wait that gives up after kAttnWaitNs, or at once when another warp gave up;
    // a waiting warp sleeps in the barrier (up to 1 us per try) instead of polling.
    auto wait = [&](uint64_t* bar, uint32_t par) -> bool {
        if (mbar_try_wait(bar, par)) return true;
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait_sleep(bar, par, 1000u)) {
            if (*reinterpret_cast<volatile int*>(&abort_flag)) return false;
            if (global_ns() - t0 > kAttnWaitNs) {
                if (atomicExch(&abort_flag, 1) == 0) atomicAdd(&g_attn_timeouts, 1u);
                return false;
            }
        }
        return true;
    };
    // V rows below P were written by earlier calls: their tiles start before the wait
    const int first = min(kNr, nslot);
    if (warp == 1 && lane == 0)
        for (int k = 0; k < first; ++k)
            if ((k + 1) * kVSlot <= P) issue_v(k);
    pdl_launch_dependents();
    pdl_wait();  // e_t, the chunk sums and the appended V row

    if (warp == 1) {
        if (lane == 0) {
            int k = 0;
            for (; k < first; ++k) {
                if ((k + 1) * kVSlot > P) issue_v(k);
                issue_e(k);
            }
            for (; k < nslot; ++k) {
                if (!wait(&empty[k % kNr], uint32_t((k / kNr - 1) & 1))) break;
                issue_v(k);
                issue_e(k);
            }
            issued = k;
        }
    } else if (warp == 2) {
        float scale = 0.0f;
        if (lane == 0) {
            double sum = 0.0;
            for (int j = 0; j < nchk; ++j) sum += a.st_s[hb * a.nch + j];
            scale = float(1.0 / sum);
        }
        scale = __shfl_sync(0xffffffffu, scale, 0);
        for (int k = 0; k < nslot; ++k) {
            const int slot = k % kNr;
            const uint32_t par = uint32_t((k / kNr) & 1);
            const int live = L - k * kVSlot;  // positions of this slot inside the context
            bool got = wait(&efull[slot], par);
            if (got && live < kVSlot) got = wait(&vfull[slot], par);  // its tile's rows past the context are zeroed
            if (!__all_sync(0xffffffffu, got)) break;
            static_assert(kVSlot == 128, "four positions per lane");
            const float4 e4 = reinterpret_cast<const float4*>(es + size_t(slot) * kVSlot)[lane];
            reinterpret_cast<float4*>(p32 + size_t(slot) * kVSlot)[lane] =
                make_float4(4 * lane < live ? round_f16(__fmul_rn(e4.x, scale)) : 0.0f,
                            4 * lane + 1 < live ? round_f16(__fmul_rn(e4.y, scale)) : 0.0f,
                            4 * lane + 2 < live ? round_f16(__fmul_rn(e4.z, scale)) : 0.0f,
                            4 * lane + 3 < live ? round_f16(__fmul_rn(e4.w, scale)) : 0.0f);
            if (live < kVSlot) {
                uint32_t* rows = reinterpret_cast<uint32_t*>(v16 + size_t(slot) * kVSlot * 32);  // 16 words per row
                for (int i = live * 16 + lane; i < kVSlot * 16; i += 32) rows[i] = 0u;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfull[slot]);
        }
    } else {
        // The chain: the slot's positions run as groups of 16 whose V (widened to
        // float) and p sit in registers; each group's loads are issued before the
        // previous group's fmas, so the chain does not wait on shared memory. The
        // next slot's barriers are tested early in each slot and waited on only
        // if they were not complete then.
        float acc = 0.0f;
        float va[16], vb[16];
        float4 pa[4], pb[4];
        auto load = [&](int slot, int i0, float (&v)[16], float4 (&p)[4]) {
            const uint16_t* vr = v16 + size_t(slot) * kVSlot * 32 + size_t(i0) * 32 + lane;
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = f16_from_bits(vr[j * 32]);
#pragma unroll
            for (int j = 0; j < 4; ++j) p[j] = reinterpret_cast<const float4*>(p32 + size_t(slot) * kVSlot + i0)[j];
        };
        auto run = [&](const float (&v)[16], const float4 (&p)[4]) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc = fmaf(p[j].x, v[4 * j + 0], acc);  // exact products: one rounding per add
                acc = fmaf(p[j].y, v[4 * j + 1], acc);
                acc = fmaf(p[j].z, v[4 * j + 2], acc);
                acc = fmaf(p[j].w, v[4 * j + 3], acc);
            }
        };
        // slot k is ready when its V tile has landed and its p is formed
        auto ready = [&](int k) {
            const uint32_t par = uint32_t((k / kNr) & 1);
            return __all_sync(0xffffffffu, wait(&vfull[k % kNr], par) && wait(&pfull[k % kNr], par));
        };
        constexpr int kGroups = kVSlot / 16;
        static_assert(kGroups % 2 == 0, "groups alternate between two register sets");
        bool ok = ready(0);
        if (ok) load(0, 0, va, pa);
        for (int k = 0; k < nslot && ok; ++k) {
            const int slot = k % kNr;
            const bool more = k + 1 < nslot;
            const uint32_t npar = uint32_t(((k + 1) / kNr) & 1);
            bool early = false;
#pragma unroll
            for (int gi = 0; gi < kGroups; gi += 2) {
                load(slot, 16 * (gi + 1), vb, pb);
                if (gi == 0 && more)
                    early = mbar_test_wait(&vfull[(k + 1) % kNr], npar) && mbar_test_wait(&pfull[(k + 1) % kNr], npar);
                run(va, pa);
                if (gi + 2 < kGroups) {
                    load(slot, 16 * (gi + 2), va, pa);
                } else if (more) {
                    ok = __all_sync(0xffffffffu, early) || ready(k + 1);
                    if (ok) load((k + 1) % kNr, 0, va, pa);
                }
                run(vb, pb);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        const int d = 32 * c + lane;
        if (d < hd && ok && !*reinterpret_cast<volatile int*>(&abort_flag)) {
            const size_t o = hb * hd + d;
            if (a.tp.peers) tp_store(a.tp, o, acc, *reinterpret_cast<const volatile unsigned*>(a.tp.epoch));
            else a.out[o] = acc;
        }
    }
    // A CTA that gave up lets its copies still in flight land before it leaves (bounded).
    __syncthreads();
    if (abort_flag && tid == 0) {
        for (int k = max(0, issued - kNr); k < issued; ++k) {
            mbar_wait_bounded(&vfull[k % kNr], uint32_t((k / kNr) & 1), kAttnWaitNs);
            mbar_wait_bounded(&efull[k % kNr], uint32_t((k / kNr) & 1), kAttnWaitNs);
        }
    }
}

// RoPE of k and F16 append of (k, v) at row pos[b], one CTA per token.
__global__ void __launch_bounds__(kThreads) rope_append_kernel(AttnParams a) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x, hd = a.hd, tid = threadIdx.x;
    const int P = a.pos[b];
    if (P < 0 || P >= a.max_len) return;  // outside the caller's bound
    extern __shared__ float cs[];
    if (a.rope)
        for (int i = tid; i < hd / 2; i += kThreads) rope_cs(a, P, i, cs[2 * i], cs[2 * i + 1]);
    __syncthreads();
    const size_t row = size_t(a.n_kv) * hd;
    uint16_t* krow = a.kc + size_t(b) * a.cache_stride + size_t(P) * row;
    uint16_t* vrow = a.vc + size_t(b) * a.cache_stride + size_t(P) * row;
    const float* kb = a.k + size_t(b) * row;
    const float* vb = a.v + size_t(b) * row;
    for (int i = tid; i < a.n_kv * hd / 2; i += kThreads) {
        const int h = i / (hd / 2), pi = i % (hd / 2);
        int i0, i1;
        pair_index(a.rope_mode, hd, pi, i0, i1);
        float o0 = kb[h * hd + i0], o1 = kb[h * hd + i1];
        if (a.rope) rotate(kb[h * hd + i0], kb[h * hd + i1], cs[2 * pi], cs[2 * pi + 1], o0, o1);
        krow[h * hd + i0] = f16_bits(o0);
        krow[h * hd + i1] = f16_bits(o1);
    }
    for (size_t i = tid; i < row; i += kThreads) vrow[i] = f16_bits(vb[i]);
}

// The (cos, sin) table of syn_rope_table: one CTA per position.
__global__ void __launch_bounds__(kThreads) rope_table_kernel(AttnParams a, float* table) {
    const int p = blockIdx.x, half = a.hd / 2;
    float2* row = reinterpret_cast<float2*>(table) + size_t(p) * half;
    for (int i = threadIdx.x; i < half; i += kThreads) {
        float c, s;
        rope_cs(a, p, i, c, s);
        row[i] = make_float2(c, s);
    }
}

// Plain RoPE of n rows (attention.hpp:89-129), one CTA per row.
__global__ void __launch_bounds__(kThreads) rope_kernel(AttnParams a, const float* x, float* out) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x, hd = a.hd, tid = threadIdx.x;
    const int P = a.pos[r];
    extern __shared__ float cs[];
    for (int i = tid; i < hd / 2; i += kThreads) rope_cs(a, P, i, cs[2 * i], cs[2 * i + 1]);
    __syncthreads();
    const size_t n = size_t(a.n_head) * hd;
    const float* xr = x + size_t(r) * n;
    float* orow = out + size_t(r) * n;
    for (int i = tid; i < a.n_head * hd / 2; i += kThreads) {
        const int h = i / (hd / 2), pi = i % (hd / 2);
        int i0, i1;
        pair_index(a.rope_mode, hd, pi, i0, i1);
        float o0, o1;
        rotate(xr[h * hd + i0], xr[h * hd + i1], cs[2 * pi], cs[2 * pi + 1], o0, o1);
        orow[h * hd + i0] = o0;
        orow[h * hd + i1] = o1;
    }
}

int group_tier(int G) {
    if (G <= 1) return 1;
    if (G <= 2) return 2;
    if (G <= 4) return 4;
    if (G <= 8) return 8;
    if (G <= 16) return 16;
    return 0;
}

AttnParams make_params(const syn_attention_args* x) {
    AttnParams a{};
    a.q = x->q; a.k = x->k; a.v = x->v;
    a.kc = x->k_cache; a.vc = x->v_cache;
    a.pos = x->pos; a.out = x->out;
    a.cache_stride = x->cache_stride;
    a.n_q = x->n_q; a.n_head = x->n_head; a.n_kv = x->n_kv; a.hd = x->head_dim; a.max_len = x->max_len;
    a.append = x->append; a.rope = x->rope; a.rope_mode = x->rope_mode;
    a.theta_scale = x->theta_scale; a.scale = x->scale;
    a.ff = x->freq_factors;
    a.rope_tab = x->rope_table;
    a.order = x->order;
    a.has_yarn = x->yarn != nullptr;
    for (int i = 0; i < 5; ++i) a.yarn[i] = x->yarn ? x->yarn[i] : 0.0f;
    return a;
}

int check_args(const syn_attention_args* x, bool need_scratch) {
    if (!x || !x->k_cache || !x->v_cache || !x->pos) return SYN_ERR_INVALID;
    if (x->n_q <= 0 || x->n_head <= 0 || x->n_kv <= 0 || x->n_head % x->n_kv) return SYN_ERR_INVALID;
    if (x->head_dim <= 0 || x->head_dim % 8 || x->head_dim > 256 || x->max_len <= 0) return SYN_ERR_INVALID;
    if (x->rope_mode != 0 && x->rope_mode != 1) return SYN_ERR_INVALID;
    if (!group_tier(x->n_head / x->n_kv)) return SYN_ERR_UNSUPPORTED;
    if (need_scratch && (!x->q || !x->out || !x->scratch)) return SYN_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x->k_cache) | reinterpret_cast<uintptr_t>(x->v_cache)) & 15)
        return SYN_ERR_INVALID;
    if (x->cache_stride % 8) return SYN_ERR_INVALID;  // rows stay 16-byte aligned
    if (reinterpret_cast<uintptr_t>(x->rope_table) & 7) return SYN_ERR_INVALID;
    if (x->order != SYN_ORDER_REFERENCE && x->order != SYN_ORDER_SPLIT) return SYN_ERR_INVALID;
    return SYN_OK;
}

// The dynamic shared memory opt-in of a kernel, set once per device to the
// most any head size (<= 256) asks for, so a smaller shape configured later
// never lowers it.
int opt_in(const void* kernel, size_t most) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, int>> done;
    int dev = 0;
    int st = syn_cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& d : done)
        if (d.first == kernel && d.second == dev) return SYN_OK;
    st = syn_cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(most)));
    if (!st) done.push_back({kernel, dev});
    return st;
}

// cuTensorMapEncodeTiled from the driver (looked up once; no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// A K or V cache as a tensor of binary16: x = column (n_kv * head_dim), y =
// position (max_len rows), z = query (cache_stride apart; absent when the
// queries share one cache); boxes of box_x columns x box_y positions, read
// into shared memory as they are (V) or in the 128-byte swizzle (K).
int cache_tensor_map(const AttnParams& a, const uint16_t* base, unsigned box_x, unsigned box_y, bool swizzle,
                     CUtensorMap* m) {
    const auto encode = tensor_map_encoder();
    if (!encode) {
        syn_set_error("cuTensorMapEncodeTiled is not available from the driver");
        return SYN_ERR_CUDA;
    }
    const cuuint64_t dims[3] = {cuuint64_t(a.n_kv) * a.hd, cuuint64_t(a.max_len), cuuint64_t(a.n_q)};
    const cuuint64_t strides[2] = {cuuint64_t(a.n_kv) * a.hd * 2, cuuint64_t(a.cache_stride) * 2};
    const cuuint32_t box[3] = {box_x, box_y, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.v3d ? 3 : 2, const_cast<uint16_t*>(base), dims,
                              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        syn_set_error("cuTensorMapEncodeTiled rejected the KV cache geometry");
        return SYN_ERR_INVALID;
    }
    return SYN_OK;
}

// The kernels of a call over grid (chunks at max_len, n_kv, n_q): a CTA whose
// chunk starts past its query's context leaves at once.
template <int GT>
int launch_attention(AttnParams a, void* scratch, cudaStream_t s) {
    const AttnScratch l = scratch_layout(a.n_q, a.n_head, a.n_kv, a.hd, a.max_len);
    char* base = static_cast<char*>(scratch);
    a.scores = reinterpret_cast<float*>(base + l.scores);
    a.st_s = reinterpret_cast<double*>(base + l.st_s);
    a.st_m = reinterpret_cast<float*>(base + l.st_m);
    a.parts = reinterpret_cast<float*>(base + l.parts);
    a.ctr = reinterpret_cast<unsigned*>(base + l.ctr);
    a.nch = (a.max_len + kChunk - 1) / kChunk;
    a.ld = score_ld(a.max_len);
    const dim3 grid(a.nch, a.n_kv, a.n_q);
    int st;
    if (a.order == SYN_ORDER_SPLIT) {
        st = opt_in(reinterpret_cast<const void*>(attn_scores_kernel<GT>), score_smem(GT, 256).total);
        if (!st) st = opt_in(reinterpret_cast<const void*>(attn_pv_kernel<GT>), pv_smem(GT, 256).total);
        if (st) return st;
        st = syn_launch(attn_scores_kernel<GT>, grid, kAttnThreads, score_smem(GT, a.hd).total, s, a);
        if (!st) st = syn_launch(attn_pv_kernel<GT>, grid, kAttnThreads, pv_smem(GT, a.hd).total, s, a);
        return st;
    }
    const bool swz = a.hd % 64 == 0;
    auto xs = swz ? attn_xs_kernel<GT, true> : attn_xs_kernel<GT, false>;
    st = opt_in(reinterpret_cast<const void*>(xs), xs_smem(GT, 256, swz).total);
    if (!st) st = opt_in(reinterpret_cast<const void*>(attn_xv_kernel), kXvSmemMost);
    if (st) return st;
    a.v3d = a.cache_stride != 0;
    CUtensorMap vmap, kmap;
    if ((st = cache_tensor_map(a, a.vc, 32, kVSlot, false, &vmap))) return st;
    if ((st = swz ? cache_tensor_map(a, a.kc, 64, 64, true, &kmap) : cache_tensor_map(a, a.kc, 32, kSlotPos, false, &kmap)))
        return st;
    const int ns = (a.hd + 31) / 32;
    st = syn_launch(xs, grid, kAttnThreads, xs_smem(GT, a.hd, swz).total, s, a, kmap);
    if (!st) st = syn_launch(attn_xe_kernel<GT>, grid, kAttnThreads, 0, s, a);
    if (!st) {
        // One p.V CTA per SM while the grid fits the device: each chain warp then has its
        // scheduler to itself (the kernel starts early, beside the previous kernels' CTAs,
        // and would otherwise stack several CTAs on the SMs that are free first).
        const unsigned ctas = unsigned(a.n_head * ns) * unsigned(a.n_q);
        size_t smem = XvSmem::total;
        int dev = 0, sms = 0, per_sm = 0;
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) == cudaSuccess &&
            ctas <= unsigned(sms))
            smem = std::min(std::max(smem, size_t(per_sm) / 2 + 1024), kXvSmemMost);
        st = syn_launch(attn_xv_kernel, dim3(unsigned(a.n_head * ns), unsigned(a.n_q)), 96u, smem, s, a, vmap);
    }
    return st;
}

}  // namespace

unsigned* syn_attn_timeout_word() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_timeouts) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return static_cast<unsigned*>(p);
}

// Bounded waits of the attention kernels that gave up on this device (syn_device_errors).
int syn_attn_timeouts() {
    unsigned n = 0;
    if (cudaMemcpyFromSymbol(&n, g_attn_timeouts, sizeof n) != cudaSuccess) return -1;
    return int(n);
}

extern "C" size_t syn_attention_scratch_bytes(int n_q, int n_head, int n_kv, int head_dim, int max_len) {
    if (n_q <= 0 || n_head <= 0 || n_kv <= 0 || head_dim <= 0 || max_len <= 0) return 0;
    return scratch_layout(n_q, n_head, n_kv, head_dim, max_len).total;
}

extern "C" int syn_attention(const syn_attention_args* x, void* stream) {
    int st = check_args(x, true);
    if (st) return st;
    if (x->append && x->cache_stride == 0 && x->n_q > 1) return SYN_ERR_INVALID;  // rows would race
    if (x->append && (!x->k || !x->v)) return SYN_ERR_INVALID;
    AttnParams a = make_params(x);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (group_tier(x->n_head / x->n_kv)) {
    case 1: return launch_attention<1>(a, x->scratch, s);
    case 2: return launch_attention<2>(a, x->scratch, s);
    case 4: return launch_attention<4>(a, x->scratch, s);
    case 8: return launch_attention<8>(a, x->scratch, s);
    case 16: return launch_attention<16>(a, x->scratch, s);
    }
    return SYN_ERR_UNSUPPORTED;
}

int syn_attention_tp(const syn_attention_args* x, const TpSync& t, cudaStream_t s) {
    int st = check_args(x, true);
    if (st) return st;
    if (x->append && x->cache_stride == 0 && x->n_q > 1) return SYN_ERR_INVALID;
    if (x->append && (!x->k || !x->v)) return SYN_ERR_INVALID;
    if (t.peers && (t.world < 1 || t.world > kTpMaxWorld || t.rank < 0 || t.rank >= t.world || !t.epoch || !t.out_ll))
        return SYN_ERR_INVALID;
    AttnParams a = make_params(x);
    a.tp = t;
    switch (group_tier(x->n_head / x->n_kv)) {
    case 1: return launch_attention<1>(a, x->scratch, s);
    case 2: return launch_attention<2>(a, x->scratch, s);
    case 4: return launch_attention<4>(a, x->scratch, s);
    case 8: return launch_attention<8>(a, x->scratch, s);
    case 16: return launch_attention<16>(a, x->scratch, s);
    }
    return SYN_ERR_UNSUPPORTED;
}

// ---- attention without caller scratch ---------------------------------------
// Some callers cannot allocate device memory: a host program that hands a
// plugin only the tensors it owns and keeps every other byte of the device
// budget to itself, or a real-time decode loop that has promised not to
// allocate once it is running (the reference's session::run makes the same
// promise). For them, syn_attention_noalloc keeps its scratch in this fixed
// array, which exists once per GPU that loads the library, until the process
// exits. Host code never touches the array by name: the device address comes
// from cudaGetSymbolAddress, looked up once per device.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// Device address of g_noalloc_scratch on the current device, looked up on the
// first call made with that device current (not inside a stream capture).
int noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* addr[64] = {};
    int dev = 0;
    int st = syn_cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    if (dev < 0 || dev >= 64) return SYN_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        st = syn_cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        if (st) return st;
        addr[dev] = p;
    }
    *out = addr[dev];
    return SYN_OK;
}

}  // namespace

extern "C" int syn_attention_noalloc(const syn_attention_args* x, void* stream) {
    if (!x) return SYN_ERR_INVALID;
    const size_t need = syn_attention_scratch_bytes(x->n_q, x->n_head, x->n_kv, x->head_dim, x->max_len);
    if (need == 0) return SYN_ERR_INVALID;
    if (need > kNoAllocScratchBytes) {
        syn_set_error("syn_attention_noalloc: this shape needs more scratch than the 16 MiB static array; "
                      "call syn_attention with caller scratch instead");
        return SYN_ERR_INVALID;
    }
    void* scratch = nullptr;
    const int st = noalloc_scratch(&scratch);
    if (st) return st;
    // The kernels write every score, statistic and partial they read later
    // in the same call, and the first re-arms the counters the second uses,
    // so nothing left from an earlier call needs clearing here.
    syn_attention_args a = *x;
    a.scratch = scratch;
    return syn_attention(&a, stream);
}

extern "C" int syn_rope_kv_append(const syn_attention_args* x, void* stream) {
    int st = check_args(x, false);
    if (st) return st;
    if (!x->k || !x->v) return SYN_ERR_INVALID;
    AttnParams a = make_params(x);
    return syn_launch(rope_append_kernel, x->n_q, kThreads, size_t(x->head_dim) * 4,
                      static_cast<cudaStream_t>(stream), a);
}

extern "C" int syn_rope_table(float* table, int max_len, int head_dim, float theta_scale, const float* freq_factors,
                              const float* yarn, void* stream) {
    if (!table || max_len <= 0 || head_dim <= 0 || head_dim % 2) return SYN_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(table) & 7) return SYN_ERR_INVALID;
    syn_attention_args args{};
    args.head_dim = head_dim;
    args.theta_scale = theta_scale;
    args.freq_factors = freq_factors;
    args.yarn = yarn;
    AttnParams a = make_params(&args);
    return syn_launch(rope_table_kernel, max_len, kThreads, 0, static_cast<cudaStream_t>(stream), a, table);
}

extern "C" int syn_rope(const float* x, float* out, int n, int n_heads, int head_dim, const int32_t* pos,
                        float theta_scale, const float* freq_factors, int rope_mode, const float* yarn,
                        void* stream) {
    if (!x || !out || !pos || n <= 0 || n_heads <= 0 || head_dim <= 0 || head_dim % 2) return SYN_ERR_INVALID;
    if (rope_mode != 0 && rope_mode != 1) return SYN_ERR_INVALID;
    syn_attention_args args{};
    args.n_head = n_heads;
    args.head_dim = head_dim;
    args.theta_scale = theta_scale;
    args.freq_factors = freq_factors;
    args.rope_mode = rope_mode;
    args.yarn = yarn;
    args.pos = pos;
    AttnParams a = make_params(&args);
    return syn_launch(rope_kernel, n, kThreads, size_t(head_dim) * 4, static_cast<cudaStream_t>(stream), a, x, out);
}
