// Q4_K / Q6_K matrix-vector products on Q8_K activations: the K formats of
// GGUF files such as Q4_K_M (quant/blocks.hpp:56-70, quant/q8.hpp:33-104,
// kernels/dot.hpp:166-239 and :359-399).
//
// Numerics follow the reference's one-lane configuration, as the Q4_0 / Q8_0
// path does: a super-block's dot with the activation quants is one exact
// integer, sum_j sc_j * dot(q_j, a_j) (Q4_K) or sum_j sc_j * dot(q_j - 32,
// a_j) (Q6_K); a chunk of four super-blocks (chunk_elements 1024,
// dot.hpp:91) accumulates fma(float(isum), d_w * d_a, acc) in block order;
// Q4_K subtracts a second accumulator over its mins, fma(float(msum),
// dmin_w * d_a, acc_m) with msum = sum_j m_{j/2} * bsums_j; the chunk sums
// are added to the row in order. Integer order is free (sums are exact):
// gemv_kb_kernel gives each lane whole super-blocks and chains a chunk over
// four lanes; gemv_k_kernel (for rows too wide for the first's shared
// memory) splits each super-block across eight lanes and reduces their
// integers with shuffles before the float chain.
//
// Device layouts.
//   Q8_K activations, planar (16-byte loads): int8 quants [n_tok][cols], then
//     the float scales [n_tok][cols/256], then the int16 sub-block sums
//     [n_tok][cols/16], each plane 256-byte aligned. syn_q8k_act_to_blocks
//     writes ggml's block_q8_k bytes from them.
//   Q4_K weights: GGUF rows unchanged (144-byte blocks keep 16-byte alignment).
//   Q6_K weights, planar: a row's blocks as 208 bytes each (ql 128, qh 64,
//     scales 16: the GGUF block without its scale, so 16-byte aligned), then
//     the row's binary16 scales, padded to 16 bytes.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace syn {
namespace {

constexpr int QKK = 256;         // weights per super-block (quant/blocks.hpp:33)
constexpr int kChunkBlocks = 4;  // chunk_elements / 256 (kernels/dot.hpp:91)
constexpr int kQ4KBytes = 144;
constexpr int kQ6KBytes = 210;
constexpr int kQ6KQuant = 208;
constexpr int kMaxTok = 8;       // tokens per launch (weights read once for all of them)

struct KAct {
    int8_t* qs;      // [n_tok][cols]
    float* d;        // [n_tok][cols / 256]
    int16_t* bsums;  // [n_tok][cols / 16]
};

__host__ __device__ inline size_t kact_qs_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * cols); }
__host__ __device__ inline size_t kact_d_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * (cols / QKK) * 4); }
__host__ __device__ inline size_t kact_bs_bytes(int n_tok, int cols) { return align256(size_t(n_tok) * (cols / 16) * 2); }

inline KAct kact_planes(void* act, int n_tok, int cols) {
    char* p = static_cast<char*>(act);
    KAct a;
    a.qs = reinterpret_cast<int8_t*>(p);
    p += kact_qs_bytes(n_tok, cols);
    a.d = reinterpret_cast<float*>(p);
    p += kact_d_bytes(n_tok, cols);
    a.bsums = reinterpret_cast<int16_t*>(p);
    return a;
}

__host__ __device__ inline size_t k_gguf_row_bytes(int type, int cols) {
    return size_t(cols / QKK) * (type == SYN_Q4_K ? kQ4KBytes : kQ6KBytes);
}
__host__ __device__ inline size_t k_planar_row_bytes(int type, int cols) {
    const size_t nb = size_t(cols / QKK);
    if (type == SYN_Q4_K) return nb * kQ4KBytes;
    return (nb * kQ6KQuant + nb * 2 + 15) & ~size_t(15);
}

// ---- Q8_K activations (quant/q8.hpp:73-104) ---------------------------------
// One CTA per (token, super-block), one thread per value. The scale comes from
// the first value of largest magnitude (ties: the lower index); quants are
// nearest_int(iscale * x) capped at 127, through the 1.5 * 2^23 magic
// (q8.hpp:44-48), with every rounding explicit.
__global__ void __launch_bounds__(QKK) quantize_q8k_kernel(const float* __restrict__ x, int cols, KAct a) {
    __shared__ float xs[QKK];
    __shared__ float wkey[QKK / 32];
    __shared__ int widx[QKK / 32];
    const int nbk = cols / QKK;
    const int t = blockIdx.x / nbk, b = blockIdx.x % nbk, i = threadIdx.x;
    const size_t e = size_t(t) * cols + size_t(b) * QKK + i;
    const float v = x[e];
    xs[i] = v;
    const float ax = fabsf(v);
    float key = ax > 0.0f ? ax : 0.0f;  // a NaN never becomes the maximum (q8.hpp:83 ax > amax)
    int idx = i;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ok = __shfl_xor_sync(0xffffffffu, key, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ok > key || (ok == key && oi < idx)) {
            key = ok;
            idx = oi;
        }
    }
    if ((i & 31) == 0) {
        wkey[i >> 5] = key;
        widx[i >> 5] = idx;
    }
    __syncthreads();
    float amax = wkey[0];
    int imax = widx[0];
#pragma unroll
    for (int w = 1; w < QKK / 32; ++w)
        if (wkey[w] > amax) {  // warps in index order: equal keys keep the earlier warp
            amax = wkey[w];
            imax = widx[w];
        }
    int q = 0;
    float iscale = 0.0f;
    if (amax != 0.0f) {
        iscale = __fdiv_rn(-127.0f, xs[imax]);
        const float m = __fadd_rn(__fmul_rn(iscale, v), 12582912.0f);
        q = min(127, (__float_as_int(m) & 0x007fffff) - 0x00400000);
    }
    a.qs[e] = static_cast<int8_t>(q);
    int s = q;  // sums of 16 consecutive quants: half-warps
#pragma unroll
    for (int o = 8; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((i & 15) == 0) a.bsums[e / 16] = static_cast<int16_t>(s);
    if (i == 0) a.d[size_t(t) * nbk + b] = amax != 0.0f ? __fdiv_rn(1.0f, iscale) : 0.0f;
}

// planes -> ggml block_q8_k bytes (d, qs[256], bsums[16]; 292 bytes)
__global__ void q8k_to_blocks_kernel(KAct a, int cols, uint8_t* __restrict__ out) {
    const int nbk = cols / QKK;
    const int t = blockIdx.x / nbk, b = blockIdx.x % nbk, i = threadIdx.x;
    uint8_t* o = out + size_t(blockIdx.x) * 292;
    o[4 + i] = static_cast<uint8_t>(a.qs[size_t(t) * cols + size_t(b) * QKK + i]);
    if (i < 16) {
        const uint16_t s = static_cast<uint16_t>(a.bsums[(size_t(t) * cols + size_t(b) * QKK) / 16 + i]);
        o[260 + 2 * i] = uint8_t(s & 0xff);
        o[261 + 2 * i] = uint8_t(s >> 8);
    }
    if (i < 4) o[i] = uint8_t(__float_as_uint(a.d[size_t(t) * nbk + b]) >> (8 * i));
}

// GGUF Q6_K rows -> planar rows (layout above). One CTA per (row, block).
__global__ void repack_q6k_kernel(const uint8_t* __restrict__ src, int nb, size_t pitch, uint8_t* __restrict__ dst) {
    const size_t r = blockIdx.x / nb;
    const int b = blockIdx.x % nb;
    const uint8_t* s = src + (r * nb + b) * kQ6KBytes;
    uint8_t* row = dst + r * pitch;
    for (int i = threadIdx.x; i < kQ6KQuant; i += blockDim.x) row[size_t(b) * kQ6KQuant + i] = s[i];
    if (threadIdx.x < 2) row[size_t(nb) * kQ6KQuant + 2 * b + threadIdx.x] = s[kQ6KQuant + threadIdx.x];
    if (b == 0)  // the row's padding bytes, so the matrix is fully defined
        for (size_t p = size_t(nb) * (kQ6KQuant + 2) + threadIdx.x; p < pitch; p += blockDim.x) row[p] = 0;
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ int dot16(const uint4 w, const uint4 x) {
    int s = __dp4a(int(w.x), int(x.x), 0);
    s = __dp4a(int(w.y), int(x.y), s);
    s = __dp4a(int(w.z), int(x.z), s);
    return __dp4a(int(w.w), int(x.w), s);
}

__device__ __forceinline__ uint4 low_nibbles(uint4 v) {
    return {v.x & 0x0f0f0f0fu, v.y & 0x0f0f0f0fu, v.z & 0x0f0f0f0fu, v.w & 0x0f0f0f0fu};
}
__device__ __forceinline__ uint4 high_nibbles(uint4 v) {
    return {(v.x >> 4) & 0x0f0f0f0fu, (v.y >> 4) & 0x0f0f0f0fu, (v.z >> 4) & 0x0f0f0f0fu, (v.w >> 4) & 0x0f0f0f0fu};
}

// The 6-bit scale and min of sub-block j of a Q4_K block, from its 12 scale
// bytes held as three little-endian words (quant/blocks.hpp:114-124).
__device__ __forceinline__ void q4k_scale_min(int j, uint32_t s0, uint32_t s1, uint32_t s2, int& sc, int& m) {
    const auto byte = [&](int k) -> int {
        const uint32_t w = k < 4 ? s0 : (k < 8 ? s1 : s2);
        return int((w >> (8 * (k & 3))) & 0xff);
    };
    if (j < 4) {
        sc = byte(j) & 63;
        m = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 0x0f) | ((byte(j - 4) >> 6) << 4);
        m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

// One warp per row; lane = 8 * g + j takes part j of super-block 4c + g of
// each chunk c. Q4_K part j: qs bytes 16j..16j+15, i.e. 16 weights of
// sub-block 2k (low nibbles) and of 2k+1 (high), k = j/2, at element
// 64k + 16(j%2) (+32); and the min term of sub-block j. Q6_K part j: half
// h = j/4, quad pair p = (j/2)%2, positions ll = 16(j%2): ql bytes
// 64h + 32p + ll (low nibbles: quad p, high: quad p + 2) and qh bytes
// 32h + ll (bits 2p and 2p + 4).
// A lane's raw bytes of one super-block part, loaded a chunk ahead of use.
struct RawPart {
    uint4 a, b;      // Q4_K: header (d, dmin, scales), 16 quant bytes; Q6_K: 16 ql bytes, 16 qh bytes
    int sc_lo, sc_hi;  // Q6_K sub-block scales
    uint32_t dbits;    // Q6_K binary16 scale
};

template <int TYPE>
__device__ __forceinline__ RawPart load_part(const uint8_t* row, int nb, int b, int j) {
    RawPart p{};
    if (TYPE == SYN_Q4_K) {
        const uint8_t* blk = row + size_t(b) * kQ4KBytes;
        p.a = __ldg(reinterpret_cast<const uint4*>(blk));
        p.b = ld_stream(blk + 16 + 16 * j);
    } else {
        const uint8_t* blk = row + size_t(b) * kQ6KQuant;
        const int h = j >> 2, q = (j >> 1) & 1, ll = 16 * (j & 1);
        p.a = ld_stream(blk + 64 * h + 32 * q + ll);
        p.b = ld_stream(blk + 128 + 32 * h + ll);
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * h);
        p.sc_lo = __ldg(sc + (j & 1) + 2 * q);      // scales[is + 2q], is = ll / 16
        p.sc_hi = __ldg(sc + (j & 1) + 2 * q + 4);  // scales[is + 2q + 4]
        p.dbits = __ldg(reinterpret_cast<const unsigned short*>(row + size_t(nb) * kQ6KQuant) + b);
    }
    return p;
}

// One warp per row; lane = 8 * g + j takes part j of super-block 4c + g of
// each chunk c. Q4_K part j: qs bytes 16j..16j+15, i.e. 16 weights of
// sub-block 2k (low nibbles) and of 2k+1 (high), k = j/2, at element
// 64k + 16(j%2) (+32); and the min term of sub-block j. Q6_K part j: half
// h = j/4, quad pair p = (j/2)%2, positions ll = 16(j%2): ql bytes
// 64h + 32p + ll (low nibbles: quad p, high: quad p + 2) and qh bytes
// 32h + ll (bits 2p and 2p + 4). The next chunk's bytes are requested
// before this chunk is computed.
template <int TYPE>
__global__ void __launch_bounds__(256, 4) gemv_k_kernel(const uint8_t* __restrict__ w, size_t pitch, int rows, int cols,
                                                     KAct a, int n_tok, float* __restrict__ y,
                                                     const float* residual) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int g = lane >> 3, j = lane & 7;
    const int nb = cols / QKK;
    const uint8_t* row = w + size_t(r) * pitch;
    float yacc[kMaxTok];
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) yacc[t] = 0.0f;

    RawPart nxt{};
    if (g < nb) nxt = load_part<TYPE>(row, nb, g, j);
    for (int c = 0; c * kChunkBlocks < nb; ++c) {
        const int b = c * kChunkBlocks + g;
        const bool valid = b < nb;
        const RawPart raw = nxt;
        if (b + kChunkBlocks < nb) nxt = load_part<TYPE>(row, nb, b + kChunkBlocks, j);
        uint4 wlo = {0, 0, 0, 0}, whi = {0, 0, 0, 0};
        int sc_lo = 0, sc_hi = 0, mj = 0;
        float dw = 0.0f, dmin = 0.0f;
        int e_lo = 0, e_hi = 0;  // element offsets of this lane's two 16-value runs
        if (valid) {
            if (TYPE == SYN_Q4_K) {
                const uint4 hdr = raw.a;
                const int k = j >> 1;
                int m_unused;
                q4k_scale_min(2 * k, hdr.y, hdr.z, hdr.w, sc_lo, m_unused);
                q4k_scale_min(2 * k + 1, hdr.y, hdr.z, hdr.w, sc_hi, m_unused);
                int sc_unused;
                q4k_scale_min(j, hdr.y, hdr.z, hdr.w, sc_unused, mj);
                dw = __half2float(__ushort_as_half(uint16_t(hdr.x & 0xffff)));
                dmin = __half2float(__ushort_as_half(uint16_t(hdr.x >> 16)));
                wlo = low_nibbles(raw.b);
                whi = high_nibbles(raw.b);
                e_lo = 64 * k + 16 * (j & 1);
                e_hi = e_lo + 32;
            } else {
                const int h = j >> 2, p = (j >> 1) & 1, ll = 16 * (j & 1);
                sc_lo = raw.sc_lo;
                sc_hi = raw.sc_hi;
                dw = __half2float(__ushort_as_half(uint16_t(raw.dbits)));
                const uint32_t sh_lo = 2 * p, sh_hi = 2 * p + 4;
                const uint32_t* l4 = &raw.a.x;
                const uint32_t* h4 = &raw.b.x;
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    lo[i] = __vsub4((l4[i] & 0x0f0f0f0fu) | (((h4[i] >> sh_lo) & 0x03030303u) << 4), 0x20202020u);
                    hi[i] = __vsub4(((l4[i] >> 4) & 0x0f0f0f0fu) | (((h4[i] >> sh_hi) & 0x03030303u) << 4),
                                    0x20202020u);
                }
                wlo = {lo[0], lo[1], lo[2], lo[3]};
                whi = {hi[0], hi[1], hi[2], hi[3]};
                e_lo = 128 * h + 32 * p + ll;
                e_hi = e_lo + 64;
            }
        }
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
            if (t >= n_tok) break;
            int s = 0, ms = 0;
            float da = 0.0f;
            if (valid) {
                const int8_t* aq = a.qs + size_t(t) * cols + size_t(b) * QKK;
                const uint4 xlo = __ldg(reinterpret_cast<const uint4*>(aq + e_lo));
                const uint4 xhi = __ldg(reinterpret_cast<const uint4*>(aq + e_hi));
                s = sc_lo * dot16(wlo, xlo) + sc_hi * dot16(whi, xhi);
                if (TYPE == SYN_Q4_K) {
                    const uint32_t bs = __ldg(reinterpret_cast<const uint32_t*>(
                        a.bsums + (size_t(t) * cols + size_t(b) * QKK) / 16 + 2 * j));
                    ms = mj * (int(int16_t(bs & 0xffff)) + int(int16_t(bs >> 16)));
                }
                da = __ldg(a.d + size_t(t) * nb + b);
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                s += __shfl_xor_sync(0xffffffffu, s, o);
                if (TYPE == SYN_Q4_K) ms += __shfl_xor_sync(0xffffffffu, ms, o);
            }
            const float scl = __fmul_rn(dw, da);
            const float sclm = __fmul_rn(dmin, da);
            float acc = 0.0f, accm = 0.0f;
#pragma unroll
            for (int q = 0; q < kChunkBlocks; ++q) {
                const int sq = __shfl_sync(0xffffffffu, s, 8 * q);
                const float cq = __shfl_sync(0xffffffffu, scl, 8 * q);
                if (TYPE == SYN_Q4_K) {
                    const int mq = __shfl_sync(0xffffffffu, ms, 8 * q);
                    const float cm = __shfl_sync(0xffffffffu, sclm, 8 * q);
                    if (c * kChunkBlocks + q < nb) accm = fmaf(float(mq), cm, accm);
                }
                if (c * kChunkBlocks + q < nb) acc = fmaf(float(sq), cq, acc);
            }
            yacc[t] = __fadd_rn(yacc[t], TYPE == SYN_Q4_K ? __fsub_rn(acc, accm) : acc);
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
            if (t >= n_tok) break;
            const size_t o = size_t(t) * rows + r;
            y[o] = residual ? __fadd_rn(yacc[t], residual[o]) : yacc[t];
        }
    }
}

// ---- one lane per super-block ----------------------------------------------------
// Each lane owns whole 256-weight super-blocks, so a block's exact integer dot
// needs no cross-lane reduction; LPR lanes (a multiple of 4) cover LPR
// consecutive blocks of one row per pass, 32 / LPR rows per warp. The
// activation quants of every token of the launch are staged once per CTA in
// shared memory, transposed to [token][16-byte piece][block] so that lanes
// reading consecutive blocks hit consecutive banks; sub-block sums and scales
// likewise. The fma chain of a chunk runs over its four lanes by three
// shuffles (lane 4c + q adds block 4c + q), and the chunk sums of a row are
// broadcast and added in order, so every value is computed exactly as the
// reference's one-lane order computes it. A lane's 16-byte loads stride its
// block, so each load uses half of every 32-byte sector it touches: they
// allocate in L1, where the next load finds the other half.
constexpr int kKbSmemBudget = 96 * 1024;  // two CTAs per SM
constexpr int kKbBytesPerBlockTok = 256 + 32 + 4;

// The eight 6-bit scales and mins of a Q4_K block from its 12 scale bytes,
// as words s0 (bytes 0-3), s1 (4-7), s2 (8-11) (quant/blocks.hpp:114-124):
// byte j of sc_lo / m_lo is scale / min j, byte j of sc_hi / m_hi is j + 4.
__device__ __forceinline__ void q4k_scales_all(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t& sc_lo,
                                               uint32_t& sc_hi, uint32_t& m_lo, uint32_t& m_hi) {
    sc_lo = s0 & 0x3f3f3f3fu;
    m_lo = s1 & 0x3f3f3f3fu;
    sc_hi = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    m_hi = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
}

__device__ __forceinline__ int byte_at(uint32_t w, int i) { return int((w >> (8 * i)) & 0xffu); }
__device__ __forceinline__ int sbyte_at(uint32_t w, int i) { return int(int8_t((w >> (8 * i)) & 0xffu)); }

// MAXT: tokens per launch at most (1: the decode case, fewer live registers,
// three CTAs per SM; 8: the decoded weights are kept for every token).
template <int TYPE, int LPR, int MAXT>
__global__ void __launch_bounds__(256, MAXT == 1 ? 3 : 2) gemv_kb_kernel(const uint8_t* __restrict__ w, size_t pitch, int rows,
                                                         int cols, KAct a, int n_tok, float* __restrict__ y,
                                                         const float* residual) {
    extern __shared__ uint4 smem[];
    const int nb = cols / QKK;
    uint4* act_s = smem;                                                    // [(t * 16 + i) * nb + b]
    uint4* bs_s = act_s + size_t(n_tok) * 16 * nb;                         // [(t * 2 + j) * nb + b]
    float* d_s = reinterpret_cast<float*>(bs_s + size_t(n_tok) * 2 * nb);  // [t * nb + b]
    {
        const int nq = n_tok * nb * 16;
        const uint4* src = reinterpret_cast<const uint4*>(a.qs);  // [n_tok][cols] = [(t * nb + b) * 16 + i]
        for (int u = threadIdx.x; u < nq; u += blockDim.x) {
            const int i = u & 15, tb = u >> 4, t = tb / nb, b = tb - t * nb;
            act_s[(t * 16 + i) * nb + b] = __ldg(src + u);
        }
        const int ns = n_tok * nb * 2;
        const uint4* bsrc = reinterpret_cast<const uint4*>(a.bsums);  // [(t * nb + b) * 2 + j]
        for (int u = threadIdx.x; u < ns; u += blockDim.x) {
            const int j = u & 1, tb = u >> 1, t = tb / nb, b = tb - t * nb;
            bs_s[(t * 2 + j) * nb + b] = __ldg(bsrc + u);
        }
        for (int u = threadIdx.x; u < n_tok * nb; u += blockDim.x) d_s[u] = __ldg(a.d + u);
    }
    __syncthreads();

    constexpr int RPW = 32 / LPR;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane % LPR, q = lane & 3, rbase = lane & ~(LPR - 1);
    const int n_groups = (rows + 8 * RPW - 1) / (8 * RPW);
    for (int rg = blockIdx.x; rg < n_groups; rg += gridDim.x) {
        const int r = (rg * 8 + warp) * RPW + lane / LPR;
        const bool row_ok = r < rows;  // lanes of an absent row still take part in the shuffles
        const uint8_t* row = w + size_t(row_ok ? r : 0) * pitch;
        float yacc[MAXT];
#pragma unroll
        for (int t = 0; t < MAXT; ++t) yacc[t] = 0.0f;
        for (int b0 = 0; b0 < nb; b0 += LPR) {
            const int b = b0 + sub;
            const bool valid = row_ok && b < nb;
            const int bb = valid ? b : 0;
            // token-invariant weight operands
            // Q4_K: low nibbles (0..31), high nibbles (32..63); Q6_K: the unsigned 6-bit quants, quads 1..4 of halves 0, 1
            uint32_t wq[64];
            int sc[16];
            float dw = 0.0f, dmin = 0.0f;
            if (TYPE == SYN_Q4_K) {
                const uint8_t* blk = row + size_t(bb) * kQ4KBytes;
                uint4 hdr = {0, 0, 0, 0}, qv[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) qv[i] = {0, 0, 0, 0};
                if (valid) {
                    hdr = __ldg(reinterpret_cast<const uint4*>(blk));
#pragma unroll
                    for (int i = 0; i < 8; ++i) qv[i] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * i));
                }
                dw = __half2float(__ushort_as_half(uint16_t(hdr.x & 0xffff)));
                dmin = __half2float(__ushort_as_half(uint16_t(hdr.x >> 16)));
                uint32_t sc_lo, sc_hi, m_lo, m_hi;
                q4k_scales_all(hdr.y, hdr.z, hdr.w, sc_lo, sc_hi, m_lo, m_hi);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sc[j] = byte_at(sc_lo, j);
                    sc[j + 4] = byte_at(sc_hi, j);
                    sc[j + 8] = byte_at(m_lo, j);  // the mins ride in sc[8..15]
                    sc[j + 12] = byte_at(m_hi, j);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t* v = &qv[i].x;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        wq[4 * i + e] = v[e] & 0x0f0f0f0fu;
                        wq[32 + 4 * i + e] = (v[e] >> 4) & 0x0f0f0f0fu;
                    }
                }
            } else {
                const uint8_t* blk = row + size_t(bb) * kQ6KQuant;
                uint4 v[13];
#pragma unroll
                for (int i = 0; i < 13; ++i) v[i] = {0, 0, 0, 0};
                uint32_t dbits = 0;
                if (valid) {
#pragma unroll
                    for (int i = 0; i < 13; ++i) v[i] = __ldg(reinterpret_cast<const uint4*>(blk) + i);
                    dbits = __ldg(reinterpret_cast<const unsigned short*>(row + size_t(nb) * kQ6KQuant) + bb);
                }
                dw = __half2float(__ushort_as_half(uint16_t(dbits)));
                const uint32_t* sw = &v[12].x;
#pragma unroll
                for (int j = 0; j < 16; ++j) sc[j] = sbyte_at(sw[j >> 2], j & 3);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t* ql = &v[4 * h].x;    // 16 words: ql[64h .. 64h + 63]
                    const uint32_t* qh = &v[8 + 2 * h].x;  // 8 words: qh[32h .. 32h + 31]
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint32_t A = ql[k], B = ql[8 + k], H = qh[k];
                        wq[32 * h + k] = (A & 0x0f0f0f0fu) | ((H << 4) & 0x30303030u);
                        wq[32 * h + 8 + k] = (B & 0x0f0f0f0fu) | ((H << 2) & 0x30303030u);
                        wq[32 * h + 16 + k] = ((A >> 4) & 0x0f0f0f0fu) | (H & 0x30303030u);
                        wq[32 * h + 24 + k] = ((B >> 4) & 0x0f0f0f0fu) | ((H >> 2) & 0x30303030u);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                if (t >= n_tok) break;
                const uint4* at = act_s + size_t(t) * 16 * nb + bb;  // piece i at at[i * nb]
                int s = 0, ms = 0;
                if (TYPE == SYN_Q4_K) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint4 w0 = {wq[8 * k], wq[8 * k + 1], wq[8 * k + 2], wq[8 * k + 3]};
                        const uint4 w1 = {wq[8 * k + 4], wq[8 * k + 5], wq[8 * k + 6], wq[8 * k + 7]};
                        const uint4 h0 = {wq[32 + 8 * k], wq[33 + 8 * k], wq[34 + 8 * k], wq[35 + 8 * k]};
                        const uint4 h1 = {wq[36 + 8 * k], wq[37 + 8 * k], wq[38 + 8 * k], wq[39 + 8 * k]};
                        const int lo = dot16(w0, at[(4 * k) * nb]) + dot16(w1, at[(4 * k + 1) * nb]);
                        const int hi = dot16(h0, at[(4 * k + 2) * nb]) + dot16(h1, at[(4 * k + 3) * nb]);
                        s += sc[2 * k] * lo + sc[2 * k + 1] * hi;
                    }
                    const uint4 p0 = bs_s[size_t(t) * 2 * nb + bb], p1 = bs_s[(size_t(t) * 2 + 1) * nb + bb];
                    const uint32_t pw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        ms += sc[8 + j] * (int(int16_t(pw[j] & 0xffffu)) + (int(pw[j]) >> 16));
                } else {
                    // sum (q - 32) a = sum q a - 32 sum a, the second from the Q8_K sums of 16
                    const uint4 p0 = bs_s[size_t(t) * 2 * nb + bb], p1 = bs_s[(size_t(t) * 2 + 1) * nb + bb];
                    const uint32_t pw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int quad = 0; quad < 4; ++quad)
#pragma unroll
                            for (int is = 0; is < 2; ++is) {
                                const int o = 32 * h + 8 * quad + 4 * is;
                                const int j = 8 * h + 2 * quad + is;  // the sub-block of 16
                                const uint4 wv = {wq[o], wq[o + 1], wq[o + 2], wq[o + 3]};
                                const int bsum = j & 1 ? int(pw[j >> 1]) >> 16 : int(int16_t(pw[j >> 1] & 0xffffu));
                                s += sc[8 * h + is + 2 * quad] * (dot16(wv, at[j * nb]) - 32 * bsum);
                            }
                }
                const float da = d_s[t * nb + bb];
                const float scl = __fmul_rn(dw, da), sclm = __fmul_rn(dmin, da);
                float acc = q == 0 && valid ? fmaf(float(s), scl, 0.0f) : 0.0f;
                float accm = q == 0 && valid ? fmaf(float(ms), sclm, 0.0f) : 0.0f;
#pragma unroll
                for (int step = 1; step < 4; ++step) {
                    const float prev = __shfl_up_sync(0xffffffffu, acc, 1);
                    const float prevm = TYPE == SYN_Q4_K ? __shfl_up_sync(0xffffffffu, accm, 1) : 0.0f;
                    if (q == step) {
                        acc = valid ? fmaf(float(s), scl, prev) : prev;
                        if (TYPE == SYN_Q4_K) accm = valid ? fmaf(float(ms), sclm, prevm) : prevm;
                    }
                }
                const float chunk = TYPE == SYN_Q4_K ? __fsub_rn(acc, accm) : acc;  // at lane 4c + 3
#pragma unroll
                for (int c = 0; c < LPR / 4; ++c) {
                    const float v = __shfl_sync(0xffffffffu, chunk, rbase + 4 * c + 3);
                    if (b0 + 4 * c < nb) yacc[t] = __fadd_rn(yacc[t], v);
                }
            }
        }
        if (row_ok && sub == 0) {
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                if (t >= n_tok) break;
                const size_t o = size_t(t) * rows + r;
                y[o] = residual ? __fadd_rn(yacc[t], residual[o]) : yacc[t];
            }
        }
    }
}

template <int TYPE, int LPR, int MAXT>
int launch_kb(const uint8_t* w, size_t pitch, int rows, int cols, const KAct& a, int n, float* y, const float* res,
              size_t smem, cudaStream_t s) {
    static int per_sm = 0;  // resident CTAs per SM at the full budget (the opt-in is per kernel and process)
    static int sms = 0;
    auto kernel = gemv_kb_kernel<TYPE, LPR, MAXT>;
    if (!per_sm) {
        int st = syn_cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      kKbSmemBudget));
        if (st) return st;
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, 256, smem) != cudaSuccess || b < 1) b = 1;
        per_sm = b;
    }
    const int rpw = 32 / LPR;
    const int groups = (rows + 8 * rpw - 1) / (8 * rpw);
    const unsigned grid = unsigned(std::min(groups, per_sm * sms));
    kernel<<<grid, 256, smem, s>>>(w, pitch, rows, cols, a, n, y, res);
    return syn_cuda_status(cudaGetLastError());
}

template <int TYPE, int MAXT>
int launch_kb_lpr(int lpr, const uint8_t* w, size_t pitch, int rows, int cols, const KAct& a, int n, float* y,
                  const float* res, size_t smem, cudaStream_t s) {
    switch (lpr) {
    case 4: return launch_kb<TYPE, 4, MAXT>(w, pitch, rows, cols, a, n, y, res, smem, s);
    case 8: return launch_kb<TYPE, 8, MAXT>(w, pitch, rows, cols, a, n, y, res, smem, s);
    case 16: return launch_kb<TYPE, 16, MAXT>(w, pitch, rows, cols, a, n, y, res, smem, s);
    default: return launch_kb<TYPE, 32, MAXT>(w, pitch, rows, cols, a, n, y, res, smem, s);
    }
}

}  // namespace
}  // namespace syn

using namespace syn;

bool syn_k_type(int type) { return type == SYN_Q4_K || type == SYN_Q6_K; }

size_t syn_k_weight_bytes(int type, int rows, int cols, int layout) {
    if (!syn_k_type(type) || rows <= 0 || cols <= 0 || cols % QKK) return 0;
    return size_t(rows) * (layout == SYN_LAYOUT_GGUF ? k_gguf_row_bytes(type, cols) : k_planar_row_bytes(type, cols));
}

int syn_k_repack_rows(int type, const void* src, int rows, int cols, void* dst, cudaStream_t s) {
    if (type == SYN_Q4_K)
        return syn_cuda_status(cudaMemcpyAsync(dst, src, size_t(rows) * k_gguf_row_bytes(type, cols),
                                               cudaMemcpyDeviceToDevice, s));
    const int nb = cols / QKK;
    repack_q6k_kernel<<<unsigned(size_t(rows) * nb), 128, 0, s>>>(static_cast<const uint8_t*>(src), nb,
                                                                   k_planar_row_bytes(type, cols),
                                                                   static_cast<uint8_t*>(dst));
    return syn_cuda_status(cudaGetLastError());
}

int syn_gemv_k(int type, const void* w, int layout, int rows, int cols, const void* act, int n_tok, float* y,
               const float* residual, cudaStream_t s) {
    if (!syn_k_type(type)) return SYN_ERR_UNSUPPORTED;
    if (!w || !act || !y || rows <= 0 || cols <= 0 || cols % QKK || n_tok <= 0) return SYN_ERR_INVALID;
    if (type == SYN_Q6_K && layout != SYN_LAYOUT_PLANAR) return SYN_ERR_UNSUPPORTED;  // 210-byte blocks: repack first
    if (layout != SYN_LAYOUT_GGUF && layout != SYN_LAYOUT_PLANAR) return SYN_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(act) & 15)) return SYN_ERR_INVALID;
    const KAct all = kact_planes(const_cast<void*>(act), n_tok, cols);
    const size_t pitch = k_planar_row_bytes(type, cols);  // Q4_K: the GGUF pitch
    const unsigned grid = unsigned((rows + 7) / 8);
    const int nbk = cols / QKK;
    // one lane per super-block when a token's activations fit the shared-memory budget
    const int kb_tok = std::min(kMaxTok, kKbSmemBudget / (nbk * kKbBytesPerBlockTok));
    const char* env = std::getenv("SYN_GEMV_K_WARP");  // 1: the warp-per-row kernel only (comparisons)
    if (kb_tok >= 1 && !(env && env[0] == '1')) {
        const int lpr = nbk >= 24 ? 32 : nbk >= 12 ? 16 : nbk >= 6 ? 8 : 4;
        for (int t0 = 0; t0 < n_tok; t0 += kb_tok) {
            const int n = std::min(kb_tok, n_tok - t0);
            KAct a{all.qs + size_t(t0) * cols, all.d + size_t(t0) * nbk, all.bsums + size_t(t0) * (cols / 16)};
            const float* res = residual ? residual + size_t(t0) * rows : nullptr;
            const size_t smem = size_t(n) * nbk * kKbBytesPerBlockTok;
            const uint8_t* wp = static_cast<const uint8_t*>(w);
            float* yo = y + size_t(t0) * rows;
            int st;
            if (n == 1)
                st = type == SYN_Q4_K ? launch_kb_lpr<SYN_Q4_K, 1>(lpr, wp, pitch, rows, cols, a, n, yo, res, smem, s)
                                      : launch_kb_lpr<SYN_Q6_K, 1>(lpr, wp, pitch, rows, cols, a, n, yo, res, smem, s);
            else
                st = type == SYN_Q4_K
                         ? launch_kb_lpr<SYN_Q4_K, kMaxTok>(lpr, wp, pitch, rows, cols, a, n, yo, res, smem, s)
                         : launch_kb_lpr<SYN_Q6_K, kMaxTok>(lpr, wp, pitch, rows, cols, a, n, yo, res, smem, s);
            if (st) return st;
        }
        return SYN_OK;
    }
    for (int t0 = 0; t0 < n_tok; t0 += kMaxTok) {
        const int n = std::min(kMaxTok, n_tok - t0);
        KAct a{all.qs + size_t(t0) * cols, all.d + size_t(t0) * nbk, all.bsums + size_t(t0) * (cols / 16)};
        const float* res = residual ? residual + size_t(t0) * rows : nullptr;
        float* yo = y + size_t(t0) * rows;
        const uint8_t* wp = static_cast<const uint8_t*>(w);
        if (type == SYN_Q4_K)
            gemv_k_kernel<SYN_Q4_K><<<grid, 256, 0, s>>>(wp, pitch, rows, cols, a, n, yo, res);
        else
            gemv_k_kernel<SYN_Q6_K><<<grid, 256, 0, s>>>(wp, pitch, rows, cols, a, n, yo, res);
        const int st = syn_cuda_status(cudaGetLastError());
        if (st) return st;
    }
    return SYN_OK;
}

extern "C" size_t syn_q8k_act_bytes(int n_tok, int cols) {
    if (n_tok <= 0 || cols <= 0 || cols % QKK) return 0;
    return kact_qs_bytes(n_tok, cols) + kact_d_bytes(n_tok, cols) + kact_bs_bytes(n_tok, cols);
}

extern "C" int syn_quantize_q8_k(const float* x, int n_tok, int cols, void* act, void* stream) {
    if (!x || !act || n_tok <= 0 || cols <= 0 || cols % QKK) return SYN_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(act) & 15) return SYN_ERR_INVALID;
    const KAct a = kact_planes(act, n_tok, cols);
    quantize_q8k_kernel<<<unsigned(size_t(n_tok) * (cols / QKK)), QKK, 0, static_cast<cudaStream_t>(stream)>>>(
        x, cols, a);
    return syn_cuda_status(cudaGetLastError());
}

extern "C" int syn_q8k_act_to_blocks(const void* act, int n_tok, int cols, void* blocks, void* stream) {
    if (!act || !blocks || n_tok <= 0 || cols <= 0 || cols % QKK) return SYN_ERR_INVALID;
    const KAct a = kact_planes(const_cast<void*>(act), n_tok, cols);
    q8k_to_blocks_kernel<<<unsigned(size_t(n_tok) * (cols / QKK)), QKK, 0, static_cast<cudaStream_t>(stream)>>>(
        a, cols, static_cast<uint8_t*>(blocks));
    return syn_cuda_status(cudaGetLastError());
}
