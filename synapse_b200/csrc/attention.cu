// RoPE + F16 KV append + GQA decode attention (kernels/attention.hpp:89-269).
//
// Numerics follow attend_group (attention.hpp:185-244) step for step:
//   q rounded to binary16; s_t = (q . K_t) * scale; softmax with the float
//   max, e_t = expf(s_t - max), a double sum and scale = float(1 / sum)
//   (elementwise.hpp:174-201); p_t = binary16(e_t * scale); out = sum p_t V_t.
// Because p_t is rounded AFTER normalisation, the kernel runs in two passes
// over the cache, which still reads every K and V byte exactly once:
//   K-pass (grid: splits x KV heads x queries): rotates q (and k), appends
//     (k, v) as F16 at row pos, writes the scores of its positions and the
//     split's (max, double sum of expf(s - max)).
//   V-pass (same grid): merges the splits' statistics into the global max and
//     sum, forms p_t exactly as above, accumulates p_t V_t over its positions,
//     and the last split CTA of each (query, KV head) sums the partial outputs
//     in split order (deterministic).
// Each KV head's rows are read by one CTA per split for all G = n_head / n_kv
// query heads of its group (GQA sharing: K/V cross HBM once).
#include "common.cuh"
#include "internal.h"

#include <algorithm>
#include <mutex>

using namespace syn;

namespace {

constexpr int kThreads = 128;
constexpr int kMaxChunk = 1024;  // positions per split (bounds shared memory)
constexpr int kTile = 64;        // cached rows staged in shared memory at a time

struct AttnParams {
    const float *q, *k, *v;
    uint16_t *kc, *vc;
    const int32_t* pos;
    float* out;
    float* scores;    // [n_q][n_head][max_len]
    float* stat_m;    // [n_q][n_head][S]
    double* stat_s;   // [n_q][n_head][S]
    float* partial;   // [n_q][n_head][S][hd]
    unsigned* count;  // [n_q][n_kv]
    size_t cache_stride;
    int n_q, n_head, n_kv, hd, max_len, S;
    int append, rope, rope_mode;
    float theta_scale, scale;
    const float* ff;
    float yarn[5];
    int has_yarn;
};

struct ScratchLayout {
    int S;
    size_t scores, stat_m, stat_s, partial, count, total;
};

ScratchLayout scratch_layout(int n_q, int n_head, int n_kv, int hd, int max_len) {
    ScratchLayout l;
    const long units = long(n_q) * n_kv;
    long S = (512 + units - 1) / units;  // about 3-4 CTAs per SM of work per pass
    S = std::min<long>(S, (max_len + 31) / 32);
    S = std::max<long>(S, (max_len + kMaxChunk - 1) / kMaxChunk);
    S = std::max<long>(S, 1);
    l.S = int(S);
    size_t off = 0;
    l.scores = off;
    off += align256(size_t(n_q) * n_head * max_len * 4);
    l.stat_m = off;
    off += align256(size_t(n_q) * n_head * S * 4);
    l.stat_s = off;
    off += align256(size_t(n_q) * n_head * S * 8);
    l.partial = off;
    off += align256(size_t(n_q) * n_head * S * hd * 4);
    l.count = off;
    off += align256(size_t(n_q) * n_kv * 4);
    l.total = off;
    return l;
}

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

__device__ __forceinline__ void split_range(int L, int S, int j, int& t0, int& t1, int& n_active) {
    const int chunk = (L + S - 1) / S;
    t0 = j * chunk;
    t1 = min(L, t0 + chunk);
    n_active = (L + chunk - 1) / chunk;
}

__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        f[2 * e] = f16_from_bits(uint16_t(w[e] & 0xffff));
        f[2 * e + 1] = f16_from_bits(uint16_t(w[e] >> 16));
    }
}

template <int GT>
__global__ void __launch_bounds__(kThreads) attn_kpass(AttnParams a) {
    pdl_launch_dependents();
    pdl_wait();
    const int j = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int hd = a.hd, G = a.n_head / a.n_kv, H = a.n_head;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = a.pos[b], L = P + 1;
    if (P < 0 || L > a.max_len) return;  // outside the caller's bound: nothing is read or written
    int t0, t1, n_active;
    split_range(L, a.S, j, t0, t1, n_active);

    extern __shared__ float sm[];
    float* cs = sm;              // [hd/2][2]
    float* qg = cs + hd;         // [G][hd], rotated and rounded to binary16
    float* sc = qg + GT * hd;    // [G][chunk]
    uint16_t* krh = reinterpret_cast<uint16_t*>(sc + GT * kMaxChunk);  // [hd] the appended key, binary16
    uint16_t* tile = krh + hd;   // [kTile][hd + 8] cached K rows (16-byte padded)
    __shared__ float red_f[kThreads / 32];
    __shared__ double red_d[kThreads / 32];

    if (j == 0 && tid == 0) a.count[size_t(b) * a.n_kv + g] = 0u;
    const size_t stat0 = (size_t(b) * H + size_t(g) * G) * a.S + j;
    if (t0 >= L) {
        if (tid < G) {
            a.stat_m[stat0 + size_t(tid) * a.S] = -INFINITY;
            a.stat_s[stat0 + size_t(tid) * a.S] = 0.0;
        }
        return;
    }
    const int chunk = t1 - t0;

    if (a.rope)
        for (int i = tid; i < hd / 2; i += kThreads) rope_cs(a, P, i, cs[2 * i], cs[2 * i + 1]);
    __syncthreads();
    const float* qb = a.q + size_t(b) * H * hd + size_t(g) * G * hd;
    if (a.rope) {
        for (int i = tid; i < G * hd / 2; i += kThreads) {
            const int jh = i / (hd / 2), pi = i % (hd / 2);
            int i0, i1;
            pair_index(a.rope_mode, hd, pi, i0, i1);
            float o0, o1;
            rotate(qb[jh * hd + i0], qb[jh * hd + i1], cs[2 * pi], cs[2 * pi + 1], o0, o1);
            qg[jh * hd + i0] = round_f16(o0);
            qg[jh * hd + i1] = round_f16(o1);
        }
    } else {
        for (int i = tid; i < G * hd; i += kThreads) qg[i] = round_f16(qb[i]);
    }
    const bool owns_row = a.append && t0 <= P && P < t1;
    const size_t row = size_t(a.n_kv) * hd;
    uint16_t* kcb = a.kc + size_t(b) * a.cache_stride;
    uint16_t* vcb = a.vc + size_t(b) * a.cache_stride;
    if (owns_row) {
        const float* kb = a.k + size_t(b) * row + size_t(g) * hd;
        const float* vb = a.v + size_t(b) * row + size_t(g) * hd;
        uint16_t* krow = kcb + size_t(P) * row + size_t(g) * hd;
        uint16_t* vrow = vcb + size_t(P) * row + size_t(g) * hd;
        if (a.rope) {
            for (int pi = tid; pi < hd / 2; pi += kThreads) {
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
            for (int d = tid; d < hd; d += kThreads) {
                const uint16_t h = f16_bits(kb[d]);
                krow[d] = h;
                krh[d] = h;
            }
        }
        for (int d = tid; d < hd; d += kThreads) vrow[d] = f16_bits(vb[d]);
    }
    __syncthreads();

    // Scores, a tile of kTile positions at a time: the tile's K rows are loaded
    // coalesced into shared memory, then one thread per position runs the dot
    // in dimension order as attend_group sums it (attention.hpp:214-219);
    // binary16 products are exact in float, so each add is the reference's add.
    float* scores_b = a.scores + (size_t(b) * H + size_t(g) * G) * a.max_len;
    const int rowh = hd + 8, c8n = hd / 8;
    for (int tb = t0; tb < t1; tb += kTile) {
        const int n = min(kTile, t1 - tb);
        for (int i = tid; i < n * c8n; i += kThreads) {
            const int rr = i / c8n, c8 = i % c8n, t = tb + rr;
            const uint4 v = (owns_row && t == P)
                                ? *reinterpret_cast<const uint4*>(krh + c8 * 8)
                                : __ldg(reinterpret_cast<const uint4*>(kcb + size_t(t) * row + size_t(g) * hd + c8 * 8));
            *reinterpret_cast<uint4*>(tile + rr * rowh + c8 * 8) = v;
        }
        __syncthreads();
        if (tid < n) {
            const uint16_t* kt = tile + tid * rowh;
            float dot[GT];
#pragma unroll
            for (int jh = 0; jh < GT; ++jh) dot[jh] = 0.0f;
            for (int d8 = 0; d8 < hd; d8 += 8) {
                float kf[8];
                unpack8(*reinterpret_cast<const uint4*>(kt + d8), kf);
#pragma unroll
                for (int e = 0; e < 8; ++e)
#pragma unroll
                    for (int jh = 0; jh < GT; ++jh)
                        if (jh < G) dot[jh] = __fadd_rn(dot[jh], __fmul_rn(qg[jh * hd + d8 + e], kf[e]));
            }
            const int t = tb + tid;
#pragma unroll
            for (int jh = 0; jh < GT; ++jh) {
                if (jh < G) {
                    const float sv = __fmul_rn(dot[jh], a.scale);
                    sc[jh * chunk + (t - t0)] = sv;
                    scores_b[size_t(jh) * a.max_len + t] = sv;
                }
            }
        }
        __syncthreads();
    }

    // Split statistics per query head: max, then the double sum of expf(s - max).
    for (int jh = 0; jh < G; ++jh) {
        float m = -INFINITY;
        for (int t = tid; t < chunk; t += kThreads) m = fmaxf(m, sc[jh * chunk + t]);
        m = warp_max(m);
        if (lane == 0) red_f[warp] = m;
        __syncthreads();
        m = red_f[0];
        for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, red_f[w]);
        double s = 0.0;
        for (int t = tid; t < chunk; t += kThreads) s += double(exp_rn(__fsub_rn(sc[jh * chunk + t], m)));
        s = warp_sum_d(s);
        if (lane == 0) red_d[warp] = s;
        __syncthreads();
        if (tid == 0) {
            double tot = 0.0;
            for (int w = 0; w < kThreads / 32; ++w) tot += red_d[w];
            a.stat_m[stat0 + size_t(jh) * a.S] = m;
            a.stat_s[stat0 + size_t(jh) * a.S] = tot;
        }
        __syncthreads();
    }
}

template <int GT>
__global__ void __launch_bounds__(kThreads) attn_vpass(AttnParams a) {
    pdl_launch_dependents();
    pdl_wait();
    const int j = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int hd = a.hd, G = a.n_head / a.n_kv, H = a.n_head;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = a.pos[b], L = P + 1;
    if (P < 0 || L > a.max_len) return;
    int t0, t1, n_active;
    split_range(L, a.S, j, t0, t1, n_active);
    if (t0 >= L) return;
    const int chunk = t1 - t0;

    extern __shared__ float sm[];
    float* pw = sm;                                               // [G][chunk] probabilities
    uint16_t* tile = reinterpret_cast<uint16_t*>(pw + GT * kMaxChunk);  // [kTile][hd + 8] cached V rows
    __shared__ float gm[GT], gscale[GT];
    __shared__ int is_last;

    // Global max and sum of each query head from the splits' statistics.
    const size_t stat0 = (size_t(b) * H + size_t(g) * G) * a.S;
    for (int jh = warp; jh < G; jh += kThreads / 32) {
        const float* m = a.stat_m + stat0 + size_t(jh) * a.S;
        const double* s = a.stat_s + stat0 + size_t(jh) * a.S;
        float M = -INFINITY;
        for (int k = lane; k < n_active; k += 32) M = fmaxf(M, m[k]);
        M = warp_max(M);
        double tot = 0.0;
        for (int k = lane; k < n_active; k += 32) tot += s[k] * exp(double(m[k]) - double(M));
        tot = warp_sum_d(tot);
        if (lane == 0) {
            gm[jh] = M;
            gscale[jh] = float(1.0 / tot);
        }
    }
    __syncthreads();
    const float* scores_b = a.scores + (size_t(b) * H + size_t(g) * G) * a.max_len;
    for (int i = tid; i < G * chunk; i += kThreads) {
        const int jh = i / chunk, t = i % chunk;
        const float e = exp_rn(__fsub_rn(scores_b[size_t(jh) * a.max_len + t0 + t], gm[jh]));
        pw[jh * chunk + t] = round_f16(__fmul_rn(e, gscale[jh]));
    }
    __syncthreads();

    // p.V a tile of kTile cached V rows at a time (loaded coalesced into shared
    // memory); each thread owns outputs (head jh, dim d) and adds p_t * V_t,d
    // in position order (attention.hpp:231-243) over the split's positions.
    const size_t row = size_t(a.n_kv) * hd;
    const uint16_t* vcb = a.vc + size_t(b) * a.cache_stride + size_t(g) * hd;
    const int rowh = hd + 8, c8n = hd / 8;
    constexpr int kOut = (GT * 256 + kThreads - 1) / kThreads;  // outputs per thread, upper bound
    float acc[kOut];
#pragma unroll
    for (int k = 0; k < kOut; ++k) acc[k] = 0.0f;
    const int n_out = G * hd;
    for (int tb = t0; tb < t1; tb += kTile) {
        const int n = min(kTile, t1 - tb);
        for (int i = tid; i < n * c8n; i += kThreads) {
            const int rr = i / c8n, c8 = i % c8n;
            *reinterpret_cast<uint4*>(tile + rr * rowh + c8 * 8) =
                __ldg(reinterpret_cast<const uint4*>(vcb + size_t(tb + rr) * row + c8 * 8));
        }
        __syncthreads();
        for (int rr = 0; rr < n; ++rr) {
#pragma unroll
            for (int k = 0; k < kOut; ++k) {
                const int o = tid + k * kThreads;
                if (o < n_out) {
                    const int jh = o / hd, d = o % hd;  // fmaf: the products are exact
                    acc[k] = fmaf(pw[jh * chunk + (tb - t0) + rr], f16_from_bits(tile[rr * rowh + d]), acc[k]);
                }
            }
        }
        __syncthreads();
    }
    float* part = a.partial + (stat0 + j) * hd;  // + jh * S * hd
#pragma unroll
    for (int k = 0; k < kOut; ++k) {
        const int o = tid + k * kThreads;
        if (o < n_out) part[size_t(o / hd) * a.S * hd + o % hd] = acc[k];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&a.count[size_t(b) * a.n_kv + g], 1u) == unsigned(n_active - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const float* part0 = a.partial + stat0 * hd;
    float* ob = a.out + size_t(b) * H * hd + size_t(g) * G * hd;
    for (int i = tid; i < G * hd; i += kThreads) {
        const int jh = i / hd, d = i % hd;
        float s = 0.0f;
        for (int k = 0; k < n_active; ++k) s += __ldcg(part0 + (size_t(jh) * a.S + k) * hd + d);
        ob[i] = s;
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
    return SYN_OK;
}

template <int GT>
int launch_attention(AttnParams a, cudaStream_t s) {
    const dim3 grid(a.S, a.n_kv, a.n_q);
    const size_t tile_bytes = size_t(kTile) * (a.hd + 8) * 2;
    const size_t kshm = size_t(a.hd + GT * a.hd + GT * kMaxChunk) * 4 + size_t(a.hd) * 2 + tile_bytes;
    const size_t vshm = size_t(GT * kMaxChunk) * 4 + tile_bytes;
    // The opt-in above 48 KB is a per-device function attribute.
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        int st = syn_cuda_status(
            cudaFuncSetAttribute(attn_kpass<GT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        if (!st)
            st = syn_cuda_status(
                cudaFuncSetAttribute(attn_vpass<GT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        if (st) return st;
        configured[dev] = true;
    }
    int st = syn_launch(attn_kpass<GT>, grid, kThreads, kshm, s, a);
    if (st) return st;
    return syn_launch(attn_vpass<GT>, grid, kThreads, vshm, s, a);
}

}  // namespace

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
    const ScratchLayout l = scratch_layout(x->n_q, x->n_head, x->n_kv, x->head_dim, x->max_len);
    char* base = static_cast<char*>(x->scratch);
    a.scores = reinterpret_cast<float*>(base + l.scores);
    a.stat_m = reinterpret_cast<float*>(base + l.stat_m);
    a.stat_s = reinterpret_cast<double*>(base + l.stat_s);
    a.partial = reinterpret_cast<float*>(base + l.partial);
    a.count = reinterpret_cast<unsigned*>(base + l.count);
    a.S = l.S;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (group_tier(x->n_head / x->n_kv)) {
    case 1: return launch_attention<1>(a, s);
    case 2: return launch_attention<2>(a, s);
    case 4: return launch_attention<4>(a, s);
    case 8: return launch_attention<8>(a, s);
    case 16: return launch_attention<16>(a, s);
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
    // The kernels fully write every scratch value they read later in the same
    // call (scores, split statistics and partial outputs), and the first pass
    // zeroes the completion counters the second pass counts with, so nothing
    // left from an earlier call needs clearing here.
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
