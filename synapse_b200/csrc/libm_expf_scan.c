/* Build step: the inputs where the C runtime's expf rounds differently from
 * the library's device expf, as a hash table the device code includes.
 *
 * The reference computes exp on float with std::exp (kernels/elementwise.hpp:79
 * silu, :188 softmax), i.e. the host C library's expf. glibc's expf is
 * accurate to about 0.502 ulp, not correctly rounded: on some inputs whose
 * exact exp lies within a few thousandths of an ulp of a rounding midpoint it
 * returns the other neighbour. The device expf (common.cuh exp_rn) is
 * correctly rounded; with this table it returns the host library's value on
 * those inputs too, so device softmax and silu carry the reference's bits.
 *
 * The scan covers every float x in [-40, 88.72284]: below -40 exp(x) is under
 * 2^-57, which neither a softmax normaliser of at least 1 nor 1 + exp(x) in
 * silu can see. For each x it evaluates the device algorithm (ported op for
 * op below, in float with fused multiply-adds where the device uses them) and
 * the host expf; every x where they differ goes into an open-addressing hash
 * table (2^19 slots, multiplicative hash, linear probing). The output is a
 * C/CUDA include defining the table, the hash constants and the longest probe.
 *
 * Usage: libm_expf_scan OUT.inc   (compile with -O2 -ffp-contract=off -pthread)
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "exp_table.h"

typedef struct {
    float hi, lo;
} f2;
static const f2 kTab[64] = {SYN_EXP2_J64_TABLE};

static void two_sum(float a, float b, float* s, float* e) {
    *s = a + b;
    const float bb = *s - a;
    *e = (a - (*s - bb)) + (b - bb);
}

/* The device's exp_rn_core (common.cuh) for x in (-87, 88.72284]. */
static float device_exp(float x) {
    const float kf = rintf(x * 0x1.715476p+6f);
    const int k = (int)kf;
    const float c_hi = 0x1.62e430p-7f, c_lo = -0x1.05c610p-35f;
    const float p_hi = kf * c_hi;
    const float p_lo = fmaf(kf, c_hi, -p_hi);
    const float d = x - p_hi;
    const float q = fmaf(-kf, c_lo, -p_lo);
    float r_hi, r_lo;
    two_sum(d, q, &r_hi, &r_lo);
    const float sq = r_hi * r_hi;
    const float sq_lo = fmaf(r_hi, r_hi, -sq);
    const float tail = (sq * r_hi) * fmaf(r_hi, fmaf(r_hi, 1.0f / 120.0f, 1.0f / 24.0f), 1.0f / 6.0f);
    float s_hi, s_lo;
    two_sum(r_hi, sq * 0.5f, &s_hi, &s_lo);
    const float low = ((s_lo + r_lo) + sq_lo * 0.5f) + (tail + r_hi * r_lo);
    const f2 t = kTab[k & 63];
    const float m_hi = t.hi * s_hi;
    const float m_lo = fmaf(t.hi, s_hi, -m_hi);
    float a_hi, a_lo;
    two_sum(t.hi, m_hi, &a_hi, &a_lo);
    const float rest = (a_lo + m_lo) + fmaf(t.hi, low, fmaf(t.lo, s_hi, t.lo));
    const float y = a_hi + rest;
    const int e = k >> 6;
    if (e > 127) return (y * 0x1.p127f) * 2.0f;
    const uint32_t sb = (uint32_t)(e + 127) << 23;
    float sc;
    memcpy(&sc, &sb, 4);
    return y * sc;
}

enum { kBits = 19, kMul = 0x9E3779B1u };

typedef struct {
    uint32_t lo, hi;
    uint32_t* keys;
    size_t n, cap;
    long wider;  /* differences of more than one ulp (none expected) */
} job;

static void* scan(void* p) {
    job* j = (job*)p;
    for (uint64_t u = j->lo; u <= j->hi; ++u) {
        const uint32_t ub = (uint32_t)u;
        float x;
        memcpy(&x, &ub, 4);
        const float h = expf(x), g = device_exp(x);
        if (h == g) continue;
        uint32_t hb, gb;
        memcpy(&hb, &h, 4);
        memcpy(&gb, &g, 4);
        if ((hb > gb ? hb - gb : gb - hb) != 1) j->wider++;
        if (j->n == j->cap) {
            j->cap = j->cap ? 2 * j->cap : 4096;
            j->keys = (uint32_t*)realloc(j->keys, j->cap * sizeof(uint32_t));
        }
        j->keys[j->n++] = ub;
    }
    return NULL;
}

int main(int argc, char** argv) {
    if (argc != 2) {
        fprintf(stderr, "usage: %s OUT.inc\n", argv[0]);
        return 2;
    }
    const float lo_x = -40.0f, hi_x = 88.72284f;
    uint32_t nb, pb;
    memcpy(&nb, &lo_x, 4);
    memcpy(&pb, &hi_x, 4);
    /* negative floats 0x80000001 .. bits(-40), positive 0x00000001 .. bits(88.72284) */
    const uint64_t ranges[2][2] = {{0x80000001u, nb}, {0x00000001u, pb}};
    enum { kThreads = 32 };
    job jobs[2 * kThreads];
    pthread_t th[2 * kThreads];
    int nj = 0;
    for (int r = 0; r < 2; ++r) {
        const uint64_t lo = ranges[r][0], span = ranges[r][1] - lo + 1;
        for (int t = 0; t < kThreads; ++t) {
            job* j = &jobs[nj];
            memset(j, 0, sizeof *j);
            j->lo = (uint32_t)(lo + span * t / kThreads);
            j->hi = (uint32_t)(lo + span * (t + 1) / kThreads - 1);
            if (pthread_create(&th[nj], NULL, scan, j)) return 1;
            ++nj;
        }
    }
    size_t total = 0;
    long wider = 0;
    for (int i = 0; i < nj; ++i) {
        pthread_join(th[i], NULL);
        total += jobs[i].n;
        wider += jobs[i].wider;
    }
    if (wider) {
        fprintf(stderr, "libm_expf_scan: %ld inputs differ by more than one ulp\n", wider);
        return 1;
    }
    const size_t size = (size_t)1 << kBits;
    if (2 * total > size) {
        fprintf(stderr, "libm_expf_scan: %zu exceptions do not fit the table\n", total);
        return 1;
    }
    uint32_t* tab = (uint32_t*)calloc(size, sizeof(uint32_t));
    int longest = 1;
    for (int i = 0; i < nj; ++i)
        for (size_t k = 0; k < jobs[i].n; ++k) {
            const uint32_t key = jobs[i].keys[k];
            const uint32_t h = (uint32_t)(key * kMul) >> (32 - kBits);
            int probe = 0;
            while (tab[(h + probe) & (size - 1)]) ++probe;
            tab[(h + probe) & (size - 1)] = key;
            if (probe + 1 > longest) longest = probe + 1;
        }
    FILE* f = fopen(argv[1], "w");
    if (!f) return 1;
    fprintf(f, "// Generated by libm_expf_scan.c: %zu inputs where the host C library's expf\n"
               "// differs from the device expf by one ulp. Do not edit.\n", total);
    fprintf(f, "#define SYN_EXPF_EXC_COUNT %zu\n#define SYN_EXPF_EXC_BITS %d\n#define SYN_EXPF_EXC_MUL 0x%08xu\n"
               "#define SYN_EXPF_EXC_PROBES %d\n", total, (int)kBits, (unsigned)kMul, longest);
    fprintf(f, "static __device__ const uint32_t g_expf_exc[%zu] = {", size);
    for (size_t i = 0; i < size; ++i) {
        if (i % 16 == 0) fputc('\n', f);
        if (tab[i]) fprintf(f, "0x%x,", tab[i]);
        else fputs("0,", f);
    }
    fputs("\n};\n", f);
    fclose(f);
    printf("libm_expf_scan: %zu exceptions, longest probe %d\n", total, longest);
    return 0;
}
