// The element-wise ops of a decode step (kernels/elementwise.hpp), with the
// Q8_0 quantization of the next matmul's activations fused in where one
// follows (rms_norm -> Q/K/V and gate/up, silu*mul -> down).
#define SYN_DEVICE_EXPF  // softmax / silu: the device expf and its exception table
#include "common.cuh"
#include "internal.h"

#include <algorithm>
#include <mutex>

using namespace syn;

namespace {

constexpr int kNormThreads = 1024;

// rms_norm (elementwise.hpp:208-232): sum of float squares in double,
// mean = float(sum / n), scale = 1 / sqrtf(mean + eps) (IEEE), out = (x*scale)*g.
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ gamma, int cols,
                                                                float eps, float* out, ActPlanes act) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* xr = x + size_t(t) * cols;
    __shared__ double red[kNormThreads / 32];
    __shared__ float s_scale;
    double s = 0.0;
    for (int i = tid; i < cols; i += kNormThreads) {
        const float v = xr[i];
        s += double(__fmul_rn(v, v));
    }
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) {
        double tot = 0.0;
        for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
        const float mean = float(tot / double(cols));
        s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    __syncthreads();
    const float scale = s_scale;
    if (out) {
        for (int i = tid; i < cols; i += kNormThreads)
            out[size_t(t) * cols + i] = __fmul_rn(__fmul_rn(xr[i], scale), gamma[i]);
    }
    if (act.qs) {
        const int nb = cols / QK;
        for (int b = warp; b < nb; b += kNormThreads / 32) {
            const int i = b * QK + lane;
            const Q8Lane r = quantize_q8_lane(__fmul_rn(__fmul_rn(xr[i], scale), gamma[i]));
            act.qs[size_t(t) * cols + i] = r.q;
            if (lane == 0) {
                const size_t k = size_t(t) * nb + b;
                act.dh[k] = r.dh;
                act.d[k] = r.d;
                act.sum[k] = r.sum;
            }
        }
    }
}

// silu (elementwise.hpp:76-81) then mul (:50-55): out = (g / (1 + expf(-g))) * u.
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_rn(-g))), u);
}

// PAIRS: g and u interleaved by element (g at 2i, u at 2i + 1 of each token's
// 2 cols values: a GEMV over gate/up rows stored in pairs); else separate.
template <bool PAIRS>
__global__ void __launch_bounds__(256) silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                                       int n_tok, int cols, float* out, ActPlanes act) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    auto value = [&](size_t t, size_t c) {
        return PAIRS ? silu_mul(g[t * 2 * cols + 2 * c], g[t * 2 * cols + 2 * c + 1])
                     : silu_mul(g[t * cols + c], u[t * cols + c]);
    };
    if (act.qs) {
        // one warp per 32-value block: compute, then quantize it
        const int nb = cols / QK;
        const long blk = (long(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
        if (blk >= long(n_tok) * nb) return;
        const long t = blk / nb, b = blk % nb;
        const size_t i = size_t(t) * cols + size_t(b) * QK + lane;
        const float v = value(size_t(t), size_t(b) * QK + lane);
        if (out) out[i] = v;
        const Q8Lane r = quantize_q8_lane(v);
        act.qs[i] = r.q;
        if (lane == 0) {
            act.dh[blk] = r.dh;
            act.d[blk] = r.d;
            act.sum[blk] = r.sum;
        }
    } else {
        const size_t n = size_t(n_tok) * cols;
        for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
            out[i] = value(i / size_t(cols), i % size_t(cols));
    }
}

__global__ void add_kernel(const float* a, const float* b, float* out, size_t n) {
    pdl_launch_dependents();
    pdl_wait();
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

// op_embed (session.hpp:331-336): decode_row of the table (blocks.hpp:72-106).
__global__ void embed_kernel(int type, const uint8_t* __restrict__ table, int layout, int rows, int cols,
                             const int32_t* __restrict__ tokens, float* out) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.y;
    const int tok = tokens[t];
    float* o = out + size_t(t) * cols;
    const int c_begin = blockIdx.x * blockDim.x, c_step = gridDim.x * blockDim.x;
    if (tok < 0 || tok >= rows) {
        for (int c = c_begin + threadIdx.x; c < cols; c += c_step) o[c] = 0.0f;  // rejected on the host before launch
        return;
    }
    const int nb = cols / QK;
    for (int c = c_begin + threadIdx.x; c < cols; c += c_step) {
        float v;
        if (type == SYN_F32) {
            v = reinterpret_cast<const float*>(table)[size_t(tok) * cols + c];
        } else if (type == SYN_F16) {
            v = f16_from_bits(reinterpret_cast<const uint16_t*>(table)[size_t(tok) * cols + c]);
        } else {
            const int b = c / QK, j = c % QK;
            const size_t blk = size_t(tok) * nb + b;
            float d;
            int q;
            if (layout == SYN_LAYOUT_GGUF) {
                const uint8_t* p = table + blk * gguf_block_bytes(type);
                d = f16_from_bits(uint16_t(p[0] | (p[1] << 8)));
                if (type == SYN_Q4_0) q = j < 16 ? (p[2 + j] & 0x0f) - 8 : (p[2 + j - 16] >> 4) - 8;
                else q = int8_t(p[2 + j]);
            } else {
                d = f16_from_bits(*reinterpret_cast<const uint16_t*>(table + planar_scale_at(type, cols, tok, b)));
                const uint8_t* p = table + planar_quant_at(type, cols, tok, b);
                if (type == SYN_Q4_0) q = j < 16 ? (p[j] & 0x0f) - 8 : (p[j - 16] >> 4) - 8;
                else q = int8_t(p[j]);
            }
            v = __fmul_rn(float(q), d);
        }
        o[c] = v;
    }
}

// First index of the maximum (std::max_element, llama_decode.cpp:274): the
// larger value wins, equal values go to the lower index, so any split of the
// row gives the same answer.
__device__ __forceinline__ void argmax_merge(float& v, int& i, float ov, int oi, int n) {
    if (oi < n && (i >= n || ov > v || (ov == v && oi < i))) {
        v = ov;
        i = oi;
    }
}

// Grid (slices, n_tok): each CTA reduces a slice of its row into a partial;
// the last CTA of the row (atomic count) merges the partials and re-arms the
// counter for the next launch.
constexpr int kArgmaxThreads = 512;
constexpr int kArgmaxSlices = 64;

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ x, int n, int32_t* out,
                                                                float* part_v, int* part_i, unsigned* count,
                                                                TpSync tp, float* plain) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.y, tid = threadIdx.x, slices = gridDim.x;
    const float* xr = x + size_t(t) * n;
    const int per = (n + slices - 1) / slices;
    const int c0 = blockIdx.x * per, c1 = min(n, c0 + per);
    // tensor parallelism: x holds every rank's logits as words; read each
    // once it is this step's and keep the float in plain for the host
    const bool words = tp.peers && tp.in_ll;
    const unsigned ep = words ? *reinterpret_cast<const volatile unsigned*>(tp.epoch) : 0u;
    float best = -INFINITY;
    int bi = n;
    for (int c = c0 + tid; c < c1; c += kArgmaxThreads) {
        float v;
        if (words) {
            v = tp_load(tp, reinterpret_cast<const uint64_t*>(x) + c, ep);
            plain[c] = v;
        } else {
            v = xr[c];
        }
        if (bi >= n || v > best) { best = v; bi = c; }  // ascending c: ties keep the lower index
    }
    __shared__ float sv[kArgmaxThreads];
    __shared__ int si[kArgmaxThreads];
    __shared__ bool last;
    sv[tid] = best;
    si[tid] = bi;
    __syncthreads();
    for (int w = kArgmaxThreads / 2; w > 0; w >>= 1) {
        if (tid < w) argmax_merge(sv[tid], si[tid], sv[tid + w], si[tid + w], n);
        __syncthreads();
    }
    if (tid == 0) {
        part_v[size_t(t) * slices + blockIdx.x] = sv[0];
        part_i[size_t(t) * slices + blockIdx.x] = si[0];
        __threadfence();
        last = atomicAdd(&count[t], 1u) == unsigned(slices - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) {
        float v = -INFINITY;
        int i = n;
        for (int k = 0; k < slices; ++k)
            argmax_merge(v, i, __ldcg(part_v + size_t(t) * slices + k), __ldcg(part_i + size_t(t) * slices + k), n);
        out[t] = i >= n ? 0 : i;
        count[t] = 0u;
    }
}

// Scratch of syn_argmax for n_tok rows, in static device memory (partials
// plus the per-row completion counters, which start at zero and are re-armed
// by every launch).
constexpr int kArgmaxMaxTok = 64;
__device__ __align__(256) unsigned char g_argmax_ws[kArgmaxMaxTok * kArgmaxSlices * 8 + kArgmaxMaxTok * 4 + 256];

// io: [0] input token, [1] position, [2] argmax of this step, [3] steps done,
// [4] forced (prompt) tokens. After a step: history[step] = argmax, the
// position advances, and the next input is the next prompt token or the argmax.
__global__ void advance_kernel(int32_t* io, const int32_t* forced, int32_t* history) {
    pdl_launch_dependents();
    pdl_wait();
    const int step = io[3];
    history[step] = io[2];
    io[3] = step + 1;
    io[1] = io[1] + 1;
    io[0] = step + 1 < io[4] ? forced[step + 1] : io[2];
}

}  // namespace

int syn_advance(int32_t* io, const int32_t* forced, int32_t* history, cudaStream_t s) {
    return syn_launch(advance_kernel, 1, 1, 0, s, io, forced, history);
}

extern "C" int syn_rms_norm(const float* x, const float* gamma, int n_tok, int cols, float eps, float* out_f32,
                            void* act, void* stream) {
    if (!x || !gamma || n_tok <= 0 || cols <= 0 || (!out_f32 && !act)) return SYN_ERR_INVALID;
    if (act && cols % QK) return SYN_ERR_INVALID;
    ActPlanes a{};
    if (act) a = act_planes(act, n_tok, cols);
    return syn_launch(rms_norm_kernel, n_tok, kNormThreads, 0, static_cast<cudaStream_t>(stream), x, gamma, cols, eps,
                      out_f32, a);
}

namespace {
int launch_silu_mul(bool pairs, const float* g, const float* u, int n_tok, int cols, float* out_f32, void* act,
                    void* stream) {
    if (!g || (!pairs && !u) || n_tok <= 0 || cols <= 0 || (!out_f32 && !act)) return SYN_ERR_INVALID;
    if (act && cols % QK) return SYN_ERR_INVALID;
    ActPlanes a{};
    long grid;
    if (act) {
        a = act_planes(act, n_tok, cols);
        grid = (long(n_tok) * (cols / QK) * 32 + 255) / 256;
    } else {
        grid = (long(n_tok) * cols + 255) / 256;
        if (grid > 4096) grid = 4096;
    }
    return pairs ? syn_launch(silu_mul_kernel<true>, unsigned(grid), 256, 0, static_cast<cudaStream_t>(stream), g, u,
                              n_tok, cols, out_f32, a)
                 : syn_launch(silu_mul_kernel<false>, unsigned(grid), 256, 0, static_cast<cudaStream_t>(stream), g, u,
                              n_tok, cols, out_f32, a);
}
}  // namespace

extern "C" int syn_silu_mul(const float* g, const float* u, int n_tok, int cols, float* out_f32, void* act,
                            void* stream) {
    return launch_silu_mul(false, g, u, n_tok, cols, out_f32, act, stream);
}

int syn_silu_mul_pairs(const float* gu, int n_tok, int cols, float* out_f32, void* act, cudaStream_t stream) {
    return launch_silu_mul(true, gu, nullptr, n_tok, cols, out_f32, act, stream);
}

extern "C" int syn_add(const float* a, const float* b, float* out, size_t n, void* stream) {
    if (!a || !b || !out || n == 0) return SYN_ERR_INVALID;
    long grid = long((n + 255) / 256);
    if (grid > 4096) grid = 4096;
    return syn_launch(add_kernel, unsigned(grid), 256, 0, static_cast<cudaStream_t>(stream), a, b, out, n);
}

extern "C" int syn_embed(int type, const void* table, int layout, int rows, int cols, const int32_t* tokens,
                         int n_tok, float* out, void* stream) {
    if (type != SYN_F32 && type != SYN_F16 && type != SYN_Q4_0 && type != SYN_Q8_0) return SYN_ERR_UNSUPPORTED;
    if (!table || !tokens || !out || rows <= 0 || cols <= 0 || n_tok <= 0) return SYN_ERR_INVALID;
    if ((type == SYN_Q4_0 || type == SYN_Q8_0) && cols % QK) return SYN_ERR_INVALID;
    return syn_launch(embed_kernel, dim3((cols + 255) / 256, n_tok), 256, 0, static_cast<cudaStream_t>(stream), type,
                      static_cast<const uint8_t*>(table), layout, rows, cols, tokens, out);
}

size_t syn_argmax_ws_bytes(int n_tok) {
    return size_t(n_tok) * kArgmaxSlices * 8 + ((size_t(n_tok) * 4 + 255) & ~size_t(255));
}

// ws: partials then per-row counters (zero before the first launch; every
// launch leaves them zero again).
int syn_argmax_ws(const float* x, int n_tok, int n, int32_t* out, void* ws, cudaStream_t s) {
    if (!x || !out || !ws || n_tok <= 0 || n <= 0) return SYN_ERR_INVALID;
    const int slices = std::min(kArgmaxSlices, std::max(1, (n + 4095) / 4096));
    float* pv = static_cast<float*>(ws);
    int* pi = reinterpret_cast<int*>(pv + size_t(n_tok) * kArgmaxSlices);
    unsigned* pc = reinterpret_cast<unsigned*>(pi + size_t(n_tok) * kArgmaxSlices);
    return syn_launch(argmax_kernel, dim3(slices, n_tok), kArgmaxThreads, 0, s, x, n, out, pv, pi, pc, TpSync{},
                      static_cast<float*>(nullptr));
}

int syn_argmax_ws_tp(const void* words, int n, int32_t* out, float* plain, void* ws, const TpSync& t,
                     cudaStream_t s) {
    if (!words || !out || !plain || !ws || n <= 0 || !t.peers || !t.in_ll || !t.epoch || !t.err)
        return SYN_ERR_INVALID;
    const int slices = std::min(kArgmaxSlices, std::max(1, (n + 4095) / 4096));
    float* pv = static_cast<float*>(ws);
    int* pi = reinterpret_cast<int*>(pv + kArgmaxSlices);
    unsigned* pc = reinterpret_cast<unsigned*>(pi + kArgmaxSlices);
    return syn_launch(argmax_kernel, dim3(slices, 1), kArgmaxThreads, 0, s, static_cast<const float*>(words), n, out,
                      pv, pi, pc, t, plain);
}

namespace {
__global__ void tp_step_begin_kernel(unsigned* epoch) {
    pdl_launch_dependents();
    pdl_wait();
    *epoch += 1u;
}
}  // namespace

int syn_tp_step_begin(unsigned* epoch, cudaStream_t s) {
    if (!epoch) return SYN_ERR_INVALID;
    return syn_launch(tp_step_begin_kernel, 1, 1, 0, s, epoch);
}

extern "C" int syn_argmax(const float* x, int n_tok, int n, int32_t* out, void* stream) {
    if (!x || !out || n_tok <= 0 || n <= 0) return SYN_ERR_INVALID;
    if (n_tok > kArgmaxMaxTok) return SYN_ERR_UNSUPPORTED;
    static std::mutex mu;
    static void* ws[64] = {};
    int dev = 0;
    int st = syn_cuda_status(cudaGetDevice(&dev));
    if (st) return st;
    if (dev < 0 || dev >= 64) return SYN_ERR_UNSUPPORTED;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!ws[dev] && (st = syn_cuda_status(cudaGetSymbolAddress(&ws[dev], g_argmax_ws)))) return st;
    }
    return syn_argmax_ws(x, n_tok, n, out, ws[dev], static_cast<cudaStream_t>(stream));
}

namespace {
__global__ void check_exp_kernel(const float* x, float* y, float* y_ref, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        y[i] = exp_rn(x[i]);
        y_ref[i] = float(exp(double(x[i])));
    }
}
}  // namespace

extern "C" int syn_check_exp(const float* x, float* y, float* y_ref, int n, void* stream) {
    if (!x || !y || !y_ref || n <= 0) return SYN_ERR_INVALID;
    return syn_launch(check_exp_kernel, dim3(4 * syn_num_sms()), dim3(256), 0, static_cast<cudaStream_t>(stream), x,
                      y, y_ref, n);
}
