/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY: a scalar C restatement of synapse's
 * CPU decode path, the parity checker for the CUDA kernels. See oracle.h for
 * what pins it. Build: -O2 -ffp-contract=off (the reference's numerics flag,
 * cmake/numerics.cmake:13), no fast-math.
 *
 * Citations are paths inside branes-ai/synapse v0.15.12, relative to
 * sdk/include/branes/synapse/ unless they start with tests/ or scripts/.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

_Static_assert(sizeof(orc_block_q4_k) == 144, "block_q4_k");
_Static_assert(sizeof(orc_block_q6_k) == 210, "block_q6_k");
_Static_assert(sizeof(orc_block_q8_k) == 292, "block_q8_k");

static int g_threads = 1;

void orc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }
int orc_get_threads(void) { return g_threads; }

/* body(i, ctx) for i in [0, n) on up to g_threads threads, contiguous pieces.
 * Each index is computed by exactly one call, so results do not depend on
 * the thread count (the reference's D1, tests/sdk/llama_threads.cpp:32-58). */
typedef void (*orc_body)(size_t i, void* ctx);
typedef struct { orc_body body; void* ctx; size_t begin, end; } orc_piece;

static void* orc_run_piece(void* p) {
    orc_piece* pc = (orc_piece*)p;
    for (size_t i = pc->begin; i < pc->end; ++i) pc->body(i, pc->ctx);
    return NULL;
}

static void orc_parallel_for(size_t n, size_t min_per_thread, orc_body body, void* ctx) {
    size_t team = (size_t)g_threads;
    if (min_per_thread == 0) min_per_thread = 1;
    if (team > n / min_per_thread) team = n / min_per_thread;
    if (team <= 1) {
        for (size_t i = 0; i < n; ++i) body(i, ctx);
        return;
    }
    pthread_t th[256];
    orc_piece pc[256];
    const size_t step = (n + team - 1) / team;
    size_t used = 0;
    for (size_t t = 0; t < team; ++t) {
        pc[t].body = body; pc[t].ctx = ctx;
        pc[t].begin = t * step < n ? t * step : n;
        pc[t].end = (t + 1) * step < n ? (t + 1) * step : n;
        if (t == 0) continue;
        if (pthread_create(&th[t], NULL, orc_run_piece, &pc[t]) != 0) { orc_run_piece(&pc[t]); th[t] = 0; }
        used = t;
    }
    orc_run_piece(&pc[0]);
    for (size_t t = 1; t <= used; ++t) if (th[t]) pthread_join(th[t], NULL);
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---- numeric/half.hpp:18-43: exact binary16 -> binary32 ---------------- */
float orc_fp16_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0x1fu) return u2f(sign | 0x7f800000u | (m << 13));
    if (e != 0) return u2f(sign | ((e + 112u) << 23) | (m << 13));
    if (m == 0) return u2f(sign);
    /* subnormal half: normalise into a binary32 normal */
    uint32_t exp32 = 113;
    while (!(m & 0x400u)) { m <<= 1; --exp32; }
    return u2f(sign | (exp32 << 23) | ((m & 0x3ffu) << 13));
}

/* ---- numeric/half.hpp:46-81: binary32 -> binary16, round to nearest even - */
uint16_t orc_float_to_fp16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) { /* inf / nan (quiet, top payload bits) */
        uint32_t nan = a > 0x7f800000u ? (0x200u | ((a >> 13) & 0x3ffu)) : 0u;
        return (uint16_t)(sign | 0x7c00u | nan);
    }
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds past 65504 */
    if (a < 0x38800000u) {                                      /* half subnormal or zero */
        if (a <= 0x33000000u) return sign;
        uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
        uint32_t sh = 126u - e;
        uint32_t h = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t r = a - 0x38000000u; /* rebias 127 -> 15 */
    uint32_t h = r >> 13, rem = r & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

static inline float round_f16(float f) { return orc_fp16_to_float(orc_float_to_fp16(f)); }

/* ---- quant/q8.hpp:54-69: quantize_row_q8_0 (ggml's _ref) --------------- */
void orc_quantize_row_q8_0(const float* x, size_t n, orc_block_q8_0* y) {
    for (size_t i = 0; i < n / ORC_QK; ++i) {
        const float* xb = x + i * ORC_QK;
        float amax = 0.0f;
        for (int j = 0; j < ORC_QK; ++j) {
            float a = fabsf(xb[j]);
            amax = amax < a ? a : amax; /* std::max(amax, a) */
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = orc_float_to_fp16(d);
        for (int j = 0; j < ORC_QK; ++j) y[i].qs[j] = (int8_t)roundf(xb[j] * id);
    }
}

/* ---- Q4_0 weight quantizer: ggml quantize_row_q4_0_ref, as gguf-py 0.19.0
 * gguf/quants.py Q4_0.quantize_blocks restates it (the reference only reads
 * weights; this makes synthetic models). ---------------------------------- */
void orc_quantize_row_q4_0(const float* x, size_t n, orc_block_q4_0* y) {
    for (size_t i = 0; i < n / ORC_QK; ++i) {
        const float* xb = x + i * ORC_QK;
        float amax = 0.0f, mx = 0.0f;
        for (int j = 0; j < ORC_QK; ++j) {
            float a = fabsf(xb[j]);
            if (amax < a) { amax = a; mx = xb[j]; }
        }
        const float d = mx / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = orc_float_to_fp16(d);
        for (int j = 0; j < 16; ++j) {
            int lo = (int)(int8_t)(xb[j] * id + 8.5f);
            int hi = (int)(int8_t)(xb[16 + j] * id + 8.5f);
            lo = lo > 15 ? 15 : lo;
            hi = hi > 15 ? 15 : hi;
            y[i].qs[j] = (uint8_t)(lo | (hi << 4));
        }
    }
}

/* ---- quant/q8.hpp:44-48 nearest_int: round half to even through the
 * 1.5 * 2^23 magic (valid for |v| <= 2^22) ----------------------------- */
static inline int nearest_int(float v) {
    const float t = v + 12582912.0f;
    return (int)(f2u(t) & 0x007fffffu) - 0x00400000;
}

/* ---- quant/q8.hpp:73-104: quantize_row_q8_k ------------------------------ */
void orc_quantize_row_q8_k(const float* x, size_t n, orc_block_q8_k* y) {
    for (size_t i = 0; i < n / ORC_QK_K; ++i) {
        const float* xb = x + i * ORC_QK_K;
        float max = 0.0f, amax = 0.0f; /* the first element of largest magnitude, signed */
        for (int j = 0; j < ORC_QK_K; ++j) {
            const float ax = fabsf(xb[j]);
            if (ax > amax) { amax = ax; max = xb[j]; }
        }
        if (amax == 0.0f) { memset(&y[i], 0, sizeof y[i]); continue; }
        const float iscale = -127.0f / max;
        for (int j = 0; j < ORC_QK_K; ++j) {
            const int q = nearest_int(iscale * xb[j]);
            y[i].qs[j] = (int8_t)(q < 127 ? q : 127);
        }
        for (int j = 0; j < ORC_QK_K / 16; ++j) {
            int sum = 0;
            for (int l = 0; l < 16; ++l) sum += y[i].qs[j * 16 + l];
            y[i].bsums[j] = (int16_t)sum;
        }
        y[i].d = 1.0f / iscale;
    }
}

/* ---- quant/blocks.hpp:114-124 get_scale_min_k4: the 6-bit scale and min of
 * sub-block j of a Q4_K block ------------------------------------------- */
static void q4_k_scale_min(int j, const uint8_t* q, int* sc, int* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

size_t orc_row_bytes(int type, size_t cols) {
    switch (type) {
    case ORC_F32: return cols * 4;
    case ORC_F16: return cols * 2;
    case ORC_Q4_0: return cols / ORC_QK * sizeof(orc_block_q4_0);
    case ORC_Q8_0: return cols / ORC_QK * sizeof(orc_block_q8_0);
    case ORC_Q4_K: return cols / ORC_QK_K * sizeof(orc_block_q4_k);
    case ORC_Q6_K: return cols / ORC_QK_K * sizeof(orc_block_q6_k);
    default: return 0;
    }
}

/* ---- quant/blocks.hpp:72-80 (Q4_0), :101-106 (Q8_0); scheme.hpp:76-107 -- */
void orc_dequantize_row(int type, const void* row, size_t n, float* y) {
    if (type == ORC_F32) { memcpy(y, row, n * 4); return; }
    if (type == ORC_F16) {
        const uint16_t* h = (const uint16_t*)row;
        for (size_t i = 0; i < n; ++i) y[i] = orc_fp16_to_float(h[i]);
        return;
    }
    if (type == ORC_Q4_0) {
        const orc_block_q4_0* b = (const orc_block_q4_0*)row;
        for (size_t i = 0; i < n / ORC_QK; ++i) {
            const float d = orc_fp16_to_float(b[i].d);
            for (int j = 0; j < 16; ++j) {
                y[i * 32 + j] = (float)((b[i].qs[j] & 0x0f) - 8) * d;
                y[i * 32 + j + 16] = (float)((b[i].qs[j] >> 4) - 8) * d;
            }
        }
        return;
    }
    if (type == ORC_Q8_0) {
        const orc_block_q8_0* b = (const orc_block_q8_0*)row;
        for (size_t i = 0; i < n / ORC_QK; ++i) {
            const float d = orc_fp16_to_float(b[i].d);
            for (int j = 0; j < 32; ++j) y[i * 32 + j] = (float)b[i].qs[j] * d;
        }
    }
    if (type == ORC_Q4_K) { /* quant/blocks.hpp:127-149 */
        for (size_t i = 0; i < n / ORC_QK_K; ++i) {
            orc_block_q4_k b;
            memcpy(&b, (const uint8_t*)row + i * sizeof b, sizeof b);
            const float d = orc_fp16_to_float(b.d), dmin = orc_fp16_to_float(b.dmin);
            float* o = y + i * ORC_QK_K;
            for (int k = 0; k < 4; ++k) { /* 32 bytes of qs: sub-block 2k low nibbles, 2k+1 high */
                int sc, m;
                q4_k_scale_min(2 * k, b.scales, &sc, &m);
                const float d1 = d * (float)sc, m1 = dmin * (float)m;
                q4_k_scale_min(2 * k + 1, b.scales, &sc, &m);
                const float d2 = d * (float)sc, m2 = dmin * (float)m;
                for (int l = 0; l < 32; ++l) o[64 * k + l] = d1 * (float)(b.qs[32 * k + l] & 0x0f) - m1;
                for (int l = 0; l < 32; ++l) o[64 * k + 32 + l] = d2 * (float)(b.qs[32 * k + l] >> 4) - m2;
            }
        }
    }
    if (type == ORC_Q6_K) { /* quant/blocks.hpp:152-174 */
        for (size_t i = 0; i < n / ORC_QK_K; ++i) {
            orc_block_q6_k b;
            memcpy(&b, (const uint8_t*)row + i * sizeof b, sizeof b);
            const float d = orc_fp16_to_float(b.d);
            for (int h = 0; h < 2; ++h) { /* halves of 128 */
                const uint8_t* ql = b.ql + 64 * h;
                const uint8_t* qh = b.qh + 32 * h;
                const int8_t* sc = b.scales + 8 * h;
                float* o = y + i * ORC_QK_K + 128 * h;
                for (int l = 0; l < 32; ++l) {
                    const int is = l / 16;
                    const int q1 = ((ql[l] & 0x0f) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    const int q2 = ((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    o[l] = d * (float)sc[is + 0] * (float)q1;
                    o[l + 32] = d * (float)sc[is + 2] * (float)q2;
                    o[l + 64] = d * (float)sc[is + 4] * (float)q3;
                    o[l + 96] = d * (float)sc[is + 6] * (float)q4;
                }
            }
        }
    }
}

/* ---- kernels/dot.hpp: one row dot ---------------------------------------
 * Quantized rows (dot.hpp:103-121 Q4_0, :147-164 Q8_0, :268-322, :327-402,
 * :424-442): chunks of chunk_elements = 1024 weights (32 blocks, :91). Each
 * block's integer sum is exact; within a chunk the float accumulator takes
 * fma(float(isum), d_w * d_a, acc) in block order (one lane: the portable
 * scalar configuration), and the chunk sum is added to the row result.
 * The activation scale d_a is the binary16 scale decoded once
 * (gemv.hpp:107-113). */
#define ORC_CHUNK_BLOCKS 32

static float row_dot_q(int type, const uint8_t* row, const orc_block_q8_0* act, const float* act_d, size_t nb) {
    float y = 0.0f;
    for (size_t b0 = 0; b0 < nb; b0 += ORC_CHUNK_BLOCKS) {
        size_t end = b0 + ORC_CHUNK_BLOCKS < nb ? b0 + ORC_CHUNK_BLOCKS : nb;
        float acc = 0.0f;
        for (size_t b = b0; b < end; ++b) {
            int32_t isum = 0;
            float dw;
            if (type == ORC_Q4_0) {
                orc_block_q4_0 w;
                memcpy(&w, row + b * sizeof(orc_block_q4_0), sizeof w);
                for (int j = 0; j < 16; ++j) {
                    isum += ((w.qs[j] & 0x0f) - 8) * act[b].qs[j];
                    isum += ((w.qs[j] >> 4) - 8) * act[b].qs[j + 16];
                }
                dw = orc_fp16_to_float(w.d);
            } else {
                orc_block_q8_0 w;
                memcpy(&w, row + b * sizeof(orc_block_q8_0), sizeof w);
                for (int j = 0; j < 32; ++j) isum += (int32_t)w.qs[j] * act[b].qs[j];
                dw = orc_fp16_to_float(w.d);
            }
            const float scale = dw * act_d[b]; /* dot_tile: c[r].s[b].d * act_scale (:369) */
            acc = fmaf((float)isum, scale, acc);
        }
        y += acc; /* dot_tile :398, y starts at 0 (row_dot :426) */
    }
    return y;
}

/* Plain rows (dot.hpp:404-433): chunks of plain_chunk = 256 decoded to float,
 * each chunk's dot (MTL5 reduce_dot) added to the row sum. reduce_dot is
 * restated in the configuration of the reference's published build (AVX2,
 * 8 float lanes): lane l takes fma(w, x, acc_l) over elements l, l+8, ...,
 * the lanes are reduced pairwise, and a ragged tail is added in order. */
#define ORC_PLAIN_CHUNK 256
#define ORC_LANES 8
static float reduce_dot8(const float* a, const float* b, size_t len) {
    float lane[ORC_LANES] = {0};
    size_t j = 0;
    for (; j + ORC_LANES <= len; j += ORC_LANES)
        for (int l = 0; l < ORC_LANES; ++l) lane[l] = fmaf(a[j + l], b[j + l], lane[l]);
    for (int w = ORC_LANES / 2; w >= 1; w /= 2)
        for (int l = 0; l < w; ++l) lane[l] += lane[l + w];
    float s = lane[0];
    for (; j < len; ++j) s += a[j] * b[j];
    return s;
}

static float row_dot_plain(int type, const uint8_t* row, const float* x, size_t cols) {
    float y = 0.0f;
    float buf[ORC_PLAIN_CHUNK];
    for (size_t i = 0; i < cols; i += ORC_PLAIN_CHUNK) {
        size_t len = cols - i < ORC_PLAIN_CHUNK ? cols - i : ORC_PLAIN_CHUNK;
        orc_dequantize_row(type, row + i * (type == ORC_F32 ? 4 : 2), len, buf);
        y += reduce_dot8(buf, x + i, len);
    }
    return y;
}

/* ---- K formats on Q8_K activations (dot.hpp:166-239 unpack, :359-399
 * dot_tile, :268-322 block_scaled_dots) --------------------------------------
 * Chunks of chunk_elements = 1024 weights are 4 super-blocks. Block b's
 * weight operand is sc_j * q (Q4_K) or sc_j * (q - 32) (Q6_K) per 32- or
 * 16-element sub-block j, so its dot with the Q8_K quants is one exact
 * integer; the chunk's float accumulator takes fma(float(isum_b), d_w * d_a,
 * acc) in block order. Q4_K also subtracts its min term: per block the exact
 * integer sum_j m_{j/2} * bsums_j (16 sub-block sums) accumulated as
 * fma(float(msum_b), dmin_w * d_a, acc_m); the chunk adds acc - acc_m to the
 * row result (:396 sums -= mins, then :398). One lane, as for Q4_0. */
#define ORC_CHUNK_SUPER 4

static int32_t q4_k_block_dot(const orc_block_q4_k* b, const orc_block_q8_k* a, int32_t* msum) {
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) q4_k_scale_min(j, b->scales, &sc[j], &m[j]);
    int32_t s = 0;
    for (int k = 0; k < 4; ++k)
        for (int l = 0; l < 32; ++l) {
            s += (int32_t)(sc[2 * k] * (b->qs[32 * k + l] & 0x0f)) * a->qs[64 * k + l];
            s += (int32_t)(sc[2 * k + 1] * (b->qs[32 * k + l] >> 4)) * a->qs[64 * k + 32 + l];
        }
    int32_t ms = 0;
    for (int j = 0; j < 16; ++j) ms += m[j / 2] * a->bsums[j];
    *msum = ms;
    return s;
}

static int32_t q6_k_block_dot(const orc_block_q6_k* b, const orc_block_q8_k* a) {
    int32_t s = 0;
    for (int h = 0; h < 2; ++h) {
        const uint8_t* ql = b->ql + 64 * h;
        const uint8_t* qh = b->qh + 32 * h;
        const int8_t* sc = b->scales + 8 * h;
        const int8_t* x = a->qs + 128 * h;
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q1 = ((ql[l] & 0x0f) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q2 = ((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            s += sc[is + 0] * q1 * x[l] + sc[is + 2] * q2 * x[l + 32] + sc[is + 4] * q3 * x[l + 64] +
                 sc[is + 6] * q4 * x[l + 96];
        }
    }
    return s;
}

static float row_dot_k(int type, const uint8_t* row, const orc_block_q8_k* act, size_t nb) {
    float y = 0.0f;
    for (size_t b0 = 0; b0 < nb; b0 += ORC_CHUNK_SUPER) {
        const size_t end = b0 + ORC_CHUNK_SUPER < nb ? b0 + ORC_CHUNK_SUPER : nb;
        float acc = 0.0f, accm = 0.0f;
        for (size_t b = b0; b < end; ++b) {
            if (type == ORC_Q4_K) {
                orc_block_q4_k w;
                memcpy(&w, row + b * sizeof w, sizeof w);
                int32_t ms;
                const int32_t s = q4_k_block_dot(&w, &act[b], &ms);
                acc = fmaf((float)s, orc_fp16_to_float(w.d) * act[b].d, acc);
                accm = fmaf((float)ms, orc_fp16_to_float(w.dmin) * act[b].d, accm);
            } else {
                orc_block_q6_k w;
                memcpy(&w, row + b * sizeof w, sizeof w);
                acc = fmaf((float)q6_k_block_dot(&w, &act[b]), orc_fp16_to_float(w.d) * act[b].d, acc);
            }
        }
        y += type == ORC_Q4_K ? acc - accm : acc;
    }
    return y;
}

typedef struct {
    int type;
    const uint8_t* W;
    size_t rb, nb, cols;
    const orc_block_q8_0* act;
    const float* ad;
    const float* x;
    float* y;
} orc_gemv_ctx;

static void gemv_k_row(size_t r, void* p) {
    orc_gemv_ctx* c = (orc_gemv_ctx*)p;
    c->y[r] = row_dot_k(c->type, c->W + r * c->rb, (const orc_block_q8_k*)c->act, c->nb);
}

void orc_gemv_q8k(int type, const void* w, size_t rows, size_t cols, const orc_block_q8_k* act, float* y) {
    orc_gemv_ctx c = {type, (const uint8_t*)w, orc_row_bytes(type, cols), cols / ORC_QK_K, cols,
                      (const orc_block_q8_0*)(const void*)act, NULL, NULL, y};
    orc_parallel_for(rows, 64, gemv_k_row, &c);
}

static void gemv_q_row(size_t r, void* p) {
    orc_gemv_ctx* c = (orc_gemv_ctx*)p;
    c->y[r] = row_dot_q(c->type, c->W + r * c->rb, c->act, c->ad, c->nb);
}
static void gemv_plain_row(size_t r, void* p) {
    orc_gemv_ctx* c = (orc_gemv_ctx*)p;
    c->y[r] = row_dot_plain(c->type, c->W + r * c->rb, c->x, c->cols);
}

void orc_gemv_q8act(int type, const void* w, size_t rows, size_t cols, const orc_block_q8_0* act, float* y) {
    const size_t nb = cols / ORC_QK;
    float* ad = (float*)malloc(nb * sizeof(float));
    for (size_t b = 0; b < nb; ++b) ad[b] = orc_fp16_to_float(act[b].d);
    orc_gemv_ctx c = {type, (const uint8_t*)w, orc_row_bytes(type, cols), nb, cols, act, ad, NULL, y};
    orc_parallel_for(rows, 64, gemv_q_row, &c);
    free(ad);
}

/* kernels/gemv.hpp:149-161 */
void orc_gemv(int type, const void* w, size_t rows, size_t cols, const float* x, float* y) {
    if (type == ORC_F32 || type == ORC_F16) {
        orc_gemv_ctx c = {type, (const uint8_t*)w, orc_row_bytes(type, cols), 0, cols, NULL, NULL, x, y};
        orc_parallel_for(rows, 64, gemv_plain_row, &c);
        return;
    }
    if (type == ORC_Q4_K || type == ORC_Q6_K) { /* gemv.hpp:149-161 with Q8_K activations */
        orc_block_q8_k* ak = (orc_block_q8_k*)malloc(cols / ORC_QK_K * sizeof(orc_block_q8_k));
        orc_quantize_row_q8_k(x, cols, ak);
        orc_gemv_q8k(type, w, rows, cols, ak, y);
        free(ak);
        return;
    }
    orc_block_q8_0* act = (orc_block_q8_0*)malloc(cols / ORC_QK * sizeof(orc_block_q8_0));
    orc_quantize_row_q8_0(x, cols, act);
    orc_gemv_q8act(type, w, rows, cols, act, y);
    free(act);
}

/* kernels/gemm.hpp:411-419: each token row exactly as gemv (G1). */
void orc_gemm(int type, const void* w, size_t rows, size_t cols, const float* x, size_t n, float* y) {
    for (size_t t = 0; t < n; ++t) orc_gemv(type, w, rows, cols, x + t * cols, y + t * rows);
}

/* ---- kernels/attention.hpp:47 ------------------------------------------- */
float orc_rope_theta_scale(float base, size_t head_dim) { return powf(base, -2.0f / (float)head_dim); }

/* ---- kernels/attention.hpp:89-129: rope --------------------------------- */
void orc_rope(const float* x, float* out, size_t n, size_t head_dim, uint32_t pos, float theta_scale,
              const float* ff, int neox, const orc_rope_scaling* sc) {
    const size_t stride = neox ? 1 : 2, offset = neox ? head_dim / 2 : 1;
    orc_rope_scaling none = {1.0f, 0.0f, 1.0f, 0.0f, 0.0f};
    if (!sc) sc = &none;
    float theta = (float)pos;
    for (size_t i = 0; i < head_dim / 2; ++i) {
        const float f = ff ? ff[i] : 1.0f;
        const float theta_extrap = theta / f;
        const float theta_interp = sc->freq_scale * theta_extrap;
        float t = theta_interp, mscale = sc->attn_factor;
        if (sc->ext_factor != 0.0f) {
            float den = sc->corr_high - sc->corr_low;
            den = den > 0.001f ? den : 0.001f;
            float yv = ((float)i - sc->corr_low) / den;
            yv = yv < 0.0f ? 0.0f : yv;
            yv = yv > 1.0f ? 1.0f : yv;
            const float ramp_mix = (1 - yv) * sc->ext_factor;
            t = theta_interp * (1 - ramp_mix) + theta_extrap * ramp_mix;
            mscale *= 1.0f + 0.1f * logf(1.0f / sc->freq_scale);
        }
        const float c = cosf(t) * mscale, s = sinf(t) * mscale;
        const size_t a = stride * i;
        for (size_t h = 0; h < n; h += head_dim) {
            const float x0 = x[h + a], x1 = x[h + a + offset];
            out[h + a] = x0 * c - x1 * s;
            out[h + a + offset] = x0 * s + x1 * c;
        }
        theta *= theta_scale;
    }
}

/* ---- kernels/attention.hpp:165-175 ---------------------------------------- */
void orc_kv_append(const float* k, const float* v, uint16_t* kc, uint16_t* vc, size_t max_ctx, size_t n_kv,
                   size_t head_dim, uint32_t pos) {
    (void)max_ctx;
    const size_t row = n_kv * head_dim;
    for (size_t i = 0; i < row; ++i) {
        kc[(size_t)pos * row + i] = orc_float_to_fp16(k[i]);
        vc[(size_t)pos * row + i] = orc_float_to_fp16(v[i]);
    }
}

size_t orc_attention_group_floats(size_t n_heads, size_t n_kv, size_t head_dim, size_t max_ctx) {
    return n_heads / n_kv * (max_ctx + head_dim); /* attention.hpp:147-152 */
}

/* std::exp on float as the reference calls it (elementwise.hpp:79, :188): the
 * host C library's expf, element by element. */
void orc_expf(const float* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = expf(x[i]);
}

/* ---- kernels/elementwise.hpp:174-201: softmax (float exp, double sum) ---- */
void orc_softmax(const float* x, float* out, size_t n) {
    float mx = x[0];
    for (size_t i = 0; i < n; ++i) mx = mx < x[i] ? x[i] : mx;
    for (size_t i = 0; i < n; ++i) out[i] = expf(x[i] - mx);
    double sum = 0.0;
    for (size_t i = 0; i < n; ++i) sum += out[i];
    const float scale = (float)(1.0 / sum);
    for (size_t i = 0; i < n; ++i) out[i] *= scale;
}

/* ---- kernels/attention.hpp:185-244: attend_group ------------------------- */
void orc_attend_group(const float* q, const uint16_t* kc, const uint16_t* vc, size_t max_ctx, size_t n_kv,
                      size_t hd, uint32_t pos, size_t n_heads, float scale, float* out, float* scores, size_t g) {
    const size_t row = n_kv * hd, group = n_heads / n_kv, n_pos = (size_t)pos + 1;
    float* qg = scores + group * max_ctx;
    float kv[256];
    for (size_t i = 0; i < group * hd; ++i) qg[i] = round_f16(q[g * group * hd + i]);
    for (size_t t = 0; t < n_pos; ++t) {
        const uint16_t* kt = kc + t * row + g * hd;
        for (size_t d = 0; d < hd; ++d) kv[d] = orc_fp16_to_float(kt[d]);
        for (size_t j = 0; j < group; ++j) {
            const float* qj = qg + j * hd;
            float dot = 0.0f;
            for (size_t d = 0; d < hd; ++d) dot += qj[d] * kv[d];
            scores[j * n_pos + t] = dot * scale;
        }
    }
    for (size_t j = 0; j < group; ++j) {
        float* s = scores + j * n_pos;
        orc_softmax(s, s, n_pos);
        for (size_t t = 0; t < n_pos; ++t) s[t] = round_f16(s[t]);
        memset(out + (g * group + j) * hd, 0, hd * sizeof(float));
    }
    for (size_t t = 0; t < n_pos; ++t) {
        const uint16_t* vt = vc + t * row + g * hd;
        for (size_t d = 0; d < hd; ++d) kv[d] = orc_fp16_to_float(vt[d]);
        for (size_t j = 0; j < group; ++j) {
            const float p = scores[j * n_pos + t];
            float* oj = out + (g * group + j) * hd;
            for (size_t d = 0; d < hd; ++d) oj[d] += p * kv[d];
        }
    }
}

/* ---- kernels/attention.hpp:254-269 (groups in parallel as session.hpp:360) */
typedef struct {
    const float* q;
    const uint16_t *kc, *vc;
    size_t max_ctx, n_kv, hd, n_heads, slot;
    uint32_t pos;
    float scale;
    float *out, *scratch;
} orc_attn_ctx;

static void attn_group_body(size_t g, void* p) {
    orc_attn_ctx* c = (orc_attn_ctx*)p;
    orc_attend_group(c->q, c->kc, c->vc, c->max_ctx, c->n_kv, c->hd, c->pos, c->n_heads, c->scale, c->out,
                     c->scratch + g * c->slot, g);
}

void orc_attention(const float* q, const float* k, const float* v, uint16_t* kc, uint16_t* vc, size_t max_ctx,
                   size_t n_kv, size_t hd, uint32_t pos, size_t n_heads, float scale, float* out, float* scratch) {
    orc_attn_ctx c = {q, kc, vc, max_ctx, n_kv, hd, n_heads, orc_attention_group_floats(n_heads, n_kv, hd, max_ctx),
                      pos, scale, out, scratch};
    orc_kv_append(k, v, kc, vc, max_ctx, n_kv, hd, pos);
    orc_parallel_for(n_kv, 1, attn_group_body, &c);
}

/* ---- kernels/elementwise.hpp:208-232: rms_norm (double sum of float squares) */
void orc_rms_norm(const float* x, const float* gamma, float eps, float* out, size_t n) {
    double sum = 0.0;
    for (size_t i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / (double)n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (size_t i = 0; i < n; ++i) out[i] = (x[i] * scale) * gamma[i];
}

/* elementwise.hpp:76-81, :50-55, :29-34 */
void orc_silu(const float* x, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = x[i] / (1.0f + expf(-x[i]));
}
void orc_mul(const float* a, const float* b, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = a[i] * b[i];
}
void orc_add(const float* a, const float* b, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* ---- models/llama.hpp:324-489 graph, executed as graph/session.hpp:133-374 */
struct orc_llama {
    orc_llama_config c;
    orc_tensor embd, out_norm, out;
    orc_layer* layers;
    float* ff;
    float theta_scale, scale;
    uint16_t* cache; /* per layer: K then V */
    float *x, *h, *q, *k, *v, *qr, *kr, *attn, *o, *g, *u, *act, *dn, *scores, *last;
};

orc_llama* orc_llama_create(const orc_llama_config* c, orc_tensor token_embd, orc_tensor output_norm,
                            orc_tensor output, const orc_layer* layers, const float* freq_factors) {
    orc_llama* m = (orc_llama*)calloc(1, sizeof *m);
    m->c = *c;
    m->embd = token_embd;
    m->out_norm = output_norm;
    m->out = output.data ? output : token_embd; /* llama.hpp:471-472: tied head */
    m->layers = (orc_layer*)malloc(c->n_layer * sizeof(orc_layer));
    memcpy(m->layers, layers, c->n_layer * sizeof(orc_layer));
    if (freq_factors) {
        m->ff = (float*)malloc(c->head_dim / 2 * sizeof(float));
        memcpy(m->ff, freq_factors, c->head_dim / 2 * sizeof(float));
    }
    m->theta_scale = orc_rope_theta_scale(c->rope_base, c->head_dim);
    m->scale = 1.0f / sqrtf((float)c->head_dim); /* llama.hpp:407 */
    const size_t kvrow = c->n_head_kv * c->head_dim, qrow = c->n_head * c->head_dim;
    m->cache = (uint16_t*)calloc(c->n_layer * 2 * c->max_ctx * kvrow, sizeof(uint16_t));
    size_t big = c->n_embd > c->n_ff ? c->n_embd : c->n_ff;
    big = big > qrow ? big : qrow;
#define ORC_ALLOC(p, n) m->p = (float*)calloc((n), sizeof(float))
    ORC_ALLOC(x, c->n_embd); ORC_ALLOC(h, c->n_embd); ORC_ALLOC(q, qrow); ORC_ALLOC(k, kvrow);
    ORC_ALLOC(v, kvrow); ORC_ALLOC(qr, qrow); ORC_ALLOC(kr, kvrow); ORC_ALLOC(attn, qrow);
    ORC_ALLOC(o, c->n_embd); ORC_ALLOC(g, c->n_ff); ORC_ALLOC(u, c->n_ff); ORC_ALLOC(act, c->n_ff);
    ORC_ALLOC(dn, c->n_embd); ORC_ALLOC(last, c->n_embd);
    ORC_ALLOC(scores, c->n_head_kv * orc_attention_group_floats(c->n_head, c->n_head_kv, c->head_dim, c->max_ctx));
#undef ORC_ALLOC
    return m;
}

void orc_llama_destroy(orc_llama* m) {
    if (!m) return;
    free(m->layers); free(m->ff); free(m->cache);
    free(m->x); free(m->h); free(m->q); free(m->k); free(m->v); free(m->qr); free(m->kr); free(m->attn);
    free(m->o); free(m->g); free(m->u); free(m->act); free(m->dn); free(m->scores); free(m->last);
    free(m);
}

void orc_llama_reset(orc_llama* m) {
    const orc_llama_config* c = &m->c;
    memset(m->cache, 0, c->n_layer * 2 * c->max_ctx * c->n_head_kv * c->head_dim * sizeof(uint16_t));
}

uint16_t* orc_llama_kcache(orc_llama* m, size_t l) {
    const size_t per = m->c.max_ctx * m->c.n_head_kv * m->c.head_dim;
    return m->cache + l * 2 * per;
}
uint16_t* orc_llama_vcache(orc_llama* m, size_t l) { return orc_llama_kcache(m, l) + m->c.max_ctx * m->c.n_head_kv * m->c.head_dim; }

static void matmul(const orc_tensor* w, size_t rows, size_t cols, const float* x, float* y) {
    orc_gemv(w->type, w->data, rows, cols, x, y);
}

int orc_llama_step(orc_llama* m, uint32_t token, uint32_t pos, float* logits) {
    return orc_llama_run(m, token, pos, 0, m->c.n_layer, 1, logits);
}

int orc_llama_run(orc_llama* m, uint32_t token, uint32_t pos, size_t l0, size_t l1, int embed, float* logits) {
    const orc_llama_config* c = &m->c;
    if (token >= c->n_vocab || pos >= c->max_ctx || l1 > c->n_layer) return 1; /* session::run returns false */
    const size_t d = c->n_embd, qrow = c->n_head * c->head_dim, kvrow = c->n_head_kv * c->head_dim;
    /* op_embed (session.hpp:331-336): decode_row of token_embd */
    if (embed)
        orc_dequantize_row(m->embd.type, (const uint8_t*)m->embd.data + token * orc_row_bytes(m->embd.type, d), d,
                           m->x);
    for (size_t l = l0; l < l1; ++l) {
        const orc_layer* L = &m->layers[l];
        orc_rms_norm(m->x, (const float*)L->attn_norm.data, c->rms_eps, m->h, d);
        matmul(&L->wq, qrow, d, m->h, m->q);
        matmul(&L->wk, kvrow, d, m->h, m->k);
        matmul(&L->wv, kvrow, d, m->h, m->v);
        orc_rope(m->q, m->qr, qrow, c->head_dim, pos, m->theta_scale, m->ff, 0, NULL);
        orc_rope(m->k, m->kr, kvrow, c->head_dim, pos, m->theta_scale, m->ff, 0, NULL);
        orc_attention(m->qr, m->kr, m->v, orc_llama_kcache(m, l), orc_llama_vcache(m, l), c->max_ctx, c->n_head_kv,
                      c->head_dim, pos, c->n_head, m->scale, m->attn, m->scores);
        matmul(&L->wo, d, qrow, m->attn, m->o);
        orc_add(m->o, m->x, m->x, d);
        orc_rms_norm(m->x, (const float*)L->ffn_norm.data, c->rms_eps, m->h, d);
        matmul(&L->gate, c->n_ff, d, m->h, m->g);
        matmul(&L->up, c->n_ff, d, m->h, m->u);
        orc_silu(m->g, m->g, c->n_ff);
        orc_mul(m->g, m->u, m->act, c->n_ff);
        matmul(&L->down, d, c->n_ff, m->act, m->dn);
        orc_add(m->dn, m->x, m->x, d);
    }
    if (logits) {
        orc_rms_norm(m->x, (const float*)m->out_norm.data, c->rms_eps, m->last, d);
        matmul(&m->out, c->n_vocab, d, m->last, logits);
    }
    return 0;
}

/* ---- synthetic weights (not part of the reference: it only reads files) ---- */
static uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

typedef struct {
    int type;
    size_t cols;
    uint64_t seed, tensor;
    float sigma;
    uint8_t* out;
} orc_fill_ctx;

static void fill_row(size_t r, void* p) {
    orc_fill_ctx* c = (orc_fill_ctx*)p;
    float buf[ORC_PLAIN_CHUNK];
    const size_t rb = orc_row_bytes(c->type, c->cols);
    for (size_t i = 0; i < c->cols; i += ORC_PLAIN_CHUNK) {
        const size_t len = c->cols - i < ORC_PLAIN_CHUNK ? c->cols - i : ORC_PLAIN_CHUNK;
        for (size_t j = 0; j < len; ++j) {
            const uint64_t idx = r * c->cols + i + j;
            const uint64_t h = mix64(c->seed ^ mix64(c->tensor * 0x100000001b3ull ^ mix64(idx)));
            const float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);
            const float u2 = (float)(uint32_t)(h & 0xffffffu) * (1.0f / 16777216.0f);
            buf[j] = sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2) * c->sigma;
        }
        uint8_t* row = c->out + r * rb;
        switch (c->type) {
        case ORC_F32: memcpy(row + i * 4, buf, len * 4); break;
        case ORC_F16:
            for (size_t j = 0; j < len; ++j) ((uint16_t*)row)[i + j] = orc_float_to_fp16(buf[j]);
            break;
        case ORC_Q4_0: orc_quantize_row_q4_0(buf, len, (orc_block_q4_0*)(row + i / ORC_QK * 18)); break;
        case ORC_Q8_0: orc_quantize_row_q8_0(buf, len, (orc_block_q8_0*)(row + i / ORC_QK * 34)); break;
        }
    }
}

void orc_fill_random(int type, size_t rows, size_t cols, uint64_t seed, uint64_t tensor, float sigma, void* out) {
    orc_fill_ctx c = {type, cols, seed, tensor, sigma, (uint8_t*)out};
    orc_parallel_for(rows, 1, fill_row, &c);
}
