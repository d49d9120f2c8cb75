// Shared device helpers for the sm_100a decode path.
//
// Every file is compiled with --fmad=false: the reference builds with
// -ffp-contract=off (cmake/numerics.cmake:13), so a*b+c stays two roundings
// unless the code asks for fmaf() where the reference calls fma().
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/synapse_b200.h"
#include "exp_table.h"
#include "internal.h"

namespace syn {

constexpr int QK = 32;  // weights per Q4_0 / Q8_0 block (quant/blocks.hpp:31)

__host__ __device__ constexpr size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// ---- Q8_0 activation planes (see syn_q8_act_bytes) -------------------------
struct ActPlanes {
    int8_t* qs;      // [n_tok][cols]
    uint16_t* dh;    // [n_tok][nb] binary16 scale bits
    float* d;        // [n_tok][nb] decoded scale
    int32_t* sum;    // [n_tok][nb] sum of the block's quants
};

__host__ __device__ inline size_t act_qs_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * cols); }
__host__ __device__ inline size_t act_dh_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * (cols / QK) * 2); }
__host__ __device__ inline size_t act_d_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * (cols / QK) * 4); }

__host__ __device__ inline ActPlanes act_planes(void* act, int n_tok, int cols) {
    char* p = static_cast<char*>(act);
    ActPlanes a;
    a.qs = reinterpret_cast<int8_t*>(p);
    p += act_qs_bytes(n_tok, cols);
    a.dh = reinterpret_cast<uint16_t*>(p);
    p += act_dh_bytes(n_tok, cols);
    a.d = reinterpret_cast<float*>(p);
    p += act_d_bytes(n_tok, cols);
    a.sum = reinterpret_cast<int32_t*>(p);
    return a;
}

__host__ __device__ inline size_t act_bytes(int n_tok, int cols) {
    return act_qs_bytes(n_tok, cols) + act_dh_bytes(n_tok, cols) + 2 * act_d_bytes(n_tok, cols);
}

// ---- planar (row-blocked) weights ---------------------------------------------
// Row r holds its quants (blocks x 16 bytes for Q4_0, x 32 for Q8_0) followed by
// its binary16 scales, padded to 16 bytes: one contiguous, 16-byte aligned run
// per row, so a lane reads eight blocks' quants and their scales with 16-byte
// loads.
__host__ __device__ inline int quant_bytes_per_block(int type) { return type == SYN_Q4_0 ? 16 : 32; }
__host__ __device__ inline int gguf_block_bytes(int type) { return type == SYN_Q4_0 ? 18 : 34; }
__host__ __device__ inline size_t planar_quant_bytes(int type, int cols) {
    return size_t(cols / QK) * quant_bytes_per_block(type);
}
__host__ __device__ inline size_t planar_row_bytes(int type, int cols) {
    return planar_quant_bytes(type, cols) + ((size_t(cols / QK) * 2 + 15) & ~size_t(15));
}
// Blocks sit in a row in order (every kernel and the host go through this map).
__host__ __device__ inline int planar_block_pos(int, size_t, int b) { return b; }
// Byte offsets of (logical) block b of row r: its quants, its binary16 scale.
__host__ __device__ inline size_t planar_quant_at(int type, int cols, size_t r, size_t b) {
    return r * planar_row_bytes(type, cols) + size_t(planar_block_pos(cols / QK, r, int(b))) * quant_bytes_per_block(type);
}
__host__ __device__ inline size_t planar_scale_at(int type, int cols, size_t r, size_t b) {
    return r * planar_row_bytes(type, cols) + planar_quant_bytes(type, cols) + b * 2;
}

// ---- binary16 ---------------------------------------------------------------
__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ uint16_t f16_bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
__device__ __forceinline__ float f16_from_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---- Q8_0 block quantizer: one block of 32 values, one per lane --------------
// quant/q8.hpp:54-69: amax, d = amax / 127 (float), id = d ? 1/d : 0 with the
// unrounded d, q = roundf(x * id), d stored as binary16 (RNE). IEEE division
// and round-half-away roundf make it bit-identical to the reference.
struct Q8Lane {
    int8_t q;
    uint16_t dh;
    float d;
    int32_t sum;
};

__device__ __forceinline__ Q8Lane quantize_q8_lane(float x) {
    const float ax = fabsf(x);
    // |x| as bits orders like the floats (non-negative); NaN inputs are outside
    // the reference's domain as well.
    const uint32_t amax_bits = __reduce_max_sync(0xffffffffu, __float_as_uint(ax));
    const float amax = __uint_as_float(amax_bits);
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    Q8Lane r;
    r.q = static_cast<int8_t>(roundf(__fmul_rn(x, id)));
    r.dh = f16_bits(d);
    r.d = f16_from_bits(r.dh);
    r.sum = __reduce_add_sync(0xffffffffu, static_cast<int>(r.q));
    return r;
}

// expf as the reference computes it (elementwise.hpp:79, :188 call std::exp
// on float, i.e. the host C library's expf). The evaluation is table-driven
// in float-float arithmetic (Tang's method: x = (64 e + j) ln2/64 + r, exp(x) =
// 2^e 2^(j/64) exp(r), |r| <= ln2/128), accurate to about 2^-44 relative, then
// rounded once to float: the correctly rounded result except within 2^-20 ulp
// of a rounding midpoint. The host library is not correctly rounded everywhere
// (glibc's expf: 0.502 ulp); on the inputs where it returns the other
// neighbour, all within 0.002 ulp of a midpoint, the result follows it: a
// result that lies within 0.004 ulp of a midpoint looks its input up in the
// table of those inputs (g_expf_exc, made at build time by
// libm_expf_scan.c from the host library over every float in [-40, 88.72]).
// Subnormal results, where the final scaling would round a second time, come
// from double precision.
// Table: 2^(j/64) split into a float and the float nearest the remainder,
// from the double 2^(j/64).
__device__ const float2 kExp2J64[64] = {SYN_EXP2_J64_TABLE};

// Translation units that evaluate exp define SYN_DEVICE_EXPF before including
// this header: the exception table is 2 MB of device data per unit.
#ifdef SYN_DEVICE_EXPF
#include "libm_expf_exc.inc"  // generated into the build directory (libm_expf_scan.c)

// The exception table's home slot of x and its first key, read at once (the
// load is issued where the exp starts, so that its latency hides behind the
// polynomial instead of following it).
static __device__ __forceinline__ uint32_t libm_expf_slot(uint32_t xb, uint32_t& h) {
    h = (xb * SYN_EXPF_EXC_MUL) >> (32 - SYN_EXPF_EXC_BITS);
    uint32_t k;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(k) : "l"(&g_expf_exc[h]));
    return k;
}
// Whether x is one of the inputs where the host library's expf is the other
// neighbour of the correctly rounded result (open addressing, bounded probes);
// k0 is the key in x's home slot h.
static __device__ __forceinline__ bool libm_expf_exception(uint32_t xb, uint32_t h, uint32_t k0) {
    if (k0 == xb) return true;
    if (k0 == 0u) return false;
    const uint32_t mask = (1u << SYN_EXPF_EXC_BITS) - 1u;
    for (int i = 1; i < SYN_EXPF_EXC_PROBES; ++i) {
        const uint32_t k = __ldg(&g_expf_exc[(h + uint32_t(i)) & mask]);
        if (k == xb) return true;
        if (k == 0u) return false;
    }
    return false;
}

__device__ __forceinline__ void two_sum(float a, float b, float& s, float& e) {
    s = __fadd_rn(a, b);
    const float bb = __fsub_rn(s, a);
    e = __fadd_rn(__fsub_rn(a, __fsub_rn(s, bb)), __fsub_rn(b, bb));
}

// exp_rn for x in (-87, 88.72]: the reduction, the polynomial and the
// reconstruction from 2^(j/64). tab is kExp2J64 in global memory (read
// through the read-only cache) or a shared-memory copy of it.
template <bool kSharedTab>
__device__ __forceinline__ float exp_rn_core(float x, const float2* tab) {
    uint32_t slot;
    const uint32_t key0 = libm_expf_slot(__float_as_uint(x), slot);
    const float kf = rintf(__fmul_rn(x, 0x1.715476p+6f));  // 64 / ln2
    const int k = int(kf);
    // r = x - k ln2/64 as r_hi + r_lo: k * C_hi exactly (product and its
    // error), x - p_hi exact by Sterbenz, then the low parts.
    const float c_hi = 0x1.62e430p-7f, c_lo = -0x1.05c610p-35f;
    const float p_hi = __fmul_rn(kf, c_hi);
    const float p_lo = __fmaf_rn(kf, c_hi, -p_hi);
    const float d = __fsub_rn(x, p_hi);
    const float q = __fmaf_rn(-kf, c_lo, -p_lo);
    float r_hi, r_lo;
    two_sum(d, q, r_hi, r_lo);
    // exp(r) - 1 = r + r^2/2 + r^3/6 + r^4/24 + r^5/120 (the next term < 2^-54)
    const float sq = __fmul_rn(r_hi, r_hi);
    const float sq_lo = __fmaf_rn(r_hi, r_hi, -sq);
    const float tail = __fmul_rn(__fmul_rn(sq, r_hi),
                                 __fmaf_rn(r_hi, __fmaf_rn(r_hi, 1.0f / 120.0f, 1.0f / 24.0f), 1.0f / 6.0f));
    float s_hi, s_lo;
    two_sum(r_hi, __fmul_rn(sq, 0.5f), s_hi, s_lo);
    const float low = __fadd_rn(__fadd_rn(__fadd_rn(s_lo, r_lo), __fmul_rn(sq_lo, 0.5f)),
                                __fadd_rn(tail, __fmul_rn(r_hi, r_lo)));
    // 2^(j/64) (1 + s): T_hi + T_hi s_hi + (T_hi low + T_lo (1 + s_hi))
    // lanes index freely (a constant-bank read would serialize)
    const float2 t = kSharedTab ? tab[k & 63] : __ldg(&tab[k & 63]);
    const float m_hi = __fmul_rn(t.x, s_hi);
    const float m_lo = __fmaf_rn(t.x, s_hi, -m_hi);
    float a_hi, a_lo;
    two_sum(t.x, m_hi, a_hi, a_lo);
    const float rest = __fadd_rn(__fadd_rn(a_lo, m_lo), __fmaf_rn(t.x, low, __fmaf_rn(t.y, s_hi, t.y)));
    const float y = __fadd_rn(a_hi, rest);
    // times 2^e, exact for a normal result (e in [-126, 128] here; 2^128 in two steps)
    const int e = k >> 6;
    float out = e > 127 ? __fmul_rn(__fmul_rn(y, 0x1.p127f), 2.0f) : __fmul_rn(y, __int_as_float((e + 127) << 23));
    // the unrounded value less y (exact - y to about 2^-44 relative), against the
    // ulp on its side of y (half of it below a power of two)
    const float res = __fadd_rn(__fsub_rn(a_hi, y), rest);
    const uint32_t yb = __float_as_uint(y);
    float ulp = __uint_as_float((yb & 0x7f800000u) - (23u << 23));
    if (res < 0.0f && (yb & 0x007fffffu) == 0u) ulp = __fmul_rn(ulp, 0.5f);
    if (fabsf(res) > __fmul_rn(0.496f, ulp) && libm_expf_exception(__float_as_uint(x), slot, key0))
        out = __uint_as_float(__float_as_uint(out) + (res > 0.0f ? 1u : 0xffffffffu));
    return out;
}

__device__ __forceinline__ float exp_rn(float x) {
    if (!(x > -87.0f)) return x != x ? x : float(exp(double(x)));  // NaN, subnormal or zero results
    if (x > 88.72284f) return __int_as_float(0x7f800000);
    return exp_rn_core<false>(x, kExp2J64);
}

// exp_rn for x <= 0 whose result is only added to a double sum that reaches
// at least 1 (a softmax denominator holds exp(0) = 1) or scaled by at most 1
// and rounded to binary16: a result below 2^-125 changes neither (it is under
// half an ulp of 1 in double, and under half the smallest binary16
// subnormal), so x <= -87 returns 0 without the double-precision tail. NaN
// propagates. tab: a shared-memory copy of kExp2J64.
__device__ __forceinline__ float exp_rn_neg(float x, const float2* tab) {
    if (!(x > -87.0f)) return x != x ? x : 0.0f;
    return exp_rn_core<true>(x, tab);
}
#endif  // SYN_DEVICE_EXPF

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---- programmatic dependent launch ---------------------------------------
// griddepcontrol.wait: block until the grids this one depends on have
// completed and their memory is visible (a no-op without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// griddepcontrol.launch_dependents: let the next grid in the stream start
// its prologue early.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// L2 prefetch of [p, p + bytes) (16-byte aligned, bytes a multiple of 16) by
// the bulk-copy unit: weights the kernel will stream, requested before it
// waits on the previous kernel.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    if (bytes >= 16)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes & ~15u) : "memory");
}

// ---- mbarrier + bulk async copy (global -> this CTA's shared memory) -------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
// Make barrier initialisation visible to the bulk-copy (async) proxy.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Order this thread's earlier generic accesses of shared memory before later
// bulk copies into it.
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// A non-multicast bulk copy of `bytes` (multiple of 16, both ends 16-byte
// aligned) completing on `bar`.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// As mbar_try_wait, but a thread whose phase is not complete sleeps in the
// barrier until it completes or about `hint_ns` pass (no polling of the
// shared-memory pipe meanwhile).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
// Whether phase `parity` of `bar` has completed, without waiting.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Wait for phase `parity` of `bar`, giving up after `limit_ns` of wall time
// (returns false then: the caller records the error and stops).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > limit_ns) return false;
        __nanosleep(32);  // back off: a waiting warp leaves the shared-memory pipe to the others
    }
    return true;
}

// ---- tensor-parallel gathers by peer stores (TpSync, internal.h) ---------------

__device__ __forceinline__ void st_word_sys(void* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_word_sys(const void* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Two words by one 16-byte load (each 8-byte word is written whole). No
// memory clobber: a thread's loads issue back to back and are checked after.
__device__ __forceinline__ void ld_words2_sys(const void* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p));
}
__device__ __forceinline__ uint64_t make_word(float v, unsigned epoch) {
    return (uint64_t(epoch) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ float word_value(uint64_t w) { return __uint_as_float(unsigned(w)); }

// Producer: output element i of this launch, as a word of this step's
// epoch, into every rank's copy.
__device__ __forceinline__ void tp_store(const TpSync& t, size_t i, float v, unsigned epoch) {
    const uint64_t w = make_word(v, epoch);
#pragma unroll
    for (int r = 0; r < kTpMaxWorld; ++r)
        if (r < t.world) st_word_sys(t.peers[r] + t.out_off + 8 * i, w);
}

// Consumer: n (even) words from p, 16-byte aligned, once each carries this
// step's epoch: all loads first, then the check, then a wait only for the
// words still behind.
template <int N>
__device__ __forceinline__ void tp_load_n(const TpSync& t, const uint64_t* p, unsigned epoch, float (&v)[N]);

// Consumer: the value of word p once it carries this step's epoch. A read
// that waits t.wait_ns (2 s unless the session sets it) is counted in *t.err
// and returns what is there; once one has given up, later reads do not wait
// (the host reads the count and fails the step).
__device__ inline float tp_load(const TpSync& t, const uint64_t* p, unsigned epoch) {
    uint64_t w = ld_word_sys(p);
    if (unsigned(w >> 32) == epoch) return word_value(w);
    const uint64_t t0 = global_ns();
    while (unsigned(w >> 32) != epoch) {
        if (*reinterpret_cast<const volatile unsigned*>(t.err) != 0) break;
        if (global_ns() - t0 > t.wait_ns) {
            atomicAdd(t.err, 1u);
            break;
        }
        __nanosleep(20);
        w = ld_word_sys(p);
    }
    return word_value(w);
}

template <int N>
__device__ __forceinline__ void tp_load_n(const TpSync& t, const uint64_t* p, unsigned epoch, float (&v)[N]) {
    static_assert(N % 2 == 0, "pairs of words");
    uint64_t w[N];
#pragma unroll
    for (int k = 0; k < N / 2; ++k) ld_words2_sys(p + 2 * k, w[2 * k], w[2 * k + 1]);
    bool ready = true;
#pragma unroll
    for (int j = 0; j < N; ++j) ready = ready && unsigned(w[j] >> 32) == epoch;
    if (!ready) {
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (unsigned(w[j] >> 32) != epoch) w[j] = __float_as_uint(tp_load(t, p + j, epoch)) | (uint64_t(epoch) << 32);
    }
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = word_value(w[j]);
}

}  // namespace syn

// Host-side error plumbing shared by the .cu files (defined in capi.cu).
int syn_cuda_status(cudaError_t e);
int syn_check_launch();
int syn_num_sms();
// Programmatic dependent launch for this thread's launches (the session turns
// it on while it enqueues a step; plain C-ABI calls launch without it).
int syn_pdl_enabled();
void syn_set_pdl(int on);

// Launch with the PDL attribute when enabled. Every kernel of this library
// calls griddepcontrol.wait before it reads a predecessor's output or writes
// any output, so a kernel may only start early, never read early.
template <typename... KArgs, typename... Args>
int syn_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (syn_pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return syn_cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}
