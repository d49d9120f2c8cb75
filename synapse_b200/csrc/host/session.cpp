// The Llama decode session on one B200 (models/llama.hpp:324-489 load_llama,
// graph/session.hpp:82-469 session).
//
// load: GGUF metadata is read with the reference's rules (llama.hpp:206-319),
//   every weight is bound with its shape checked (models/common.hpp:146-160),
//   and streamed into ONE device arena (pinned double buffers, host copies
//   overlapping the transfers and repacks): Q4_0/Q8_0/K matrices repacked to
//   the planar layout, Q/K/V (and gate/up) of equal type concatenated by rows so
//   one GEMV launch streams them together. The f16 KV cache and the step's
//   activations live in the same arena; activations are placed by the
//   reference's static planner (planner.hpp) over the step's node order.
// build: the step is the reference's graph (embed; per layer rms_norm, Q/K/V,
//   rope+attention, O + residual, rms_norm, gate/up, silu*mul, down +
//   residual; rms_norm, logits) with these fusions, none of which changes a
//   float operation: rms_norm / silu*mul quantize their output to Q8_0 in the
//   same kernel, matmul adds the residual in its epilogue, rope + kv_append
//   run inside the attention kernel.
// run: the step is captured once as a CUDA graph; position and token live in
//   device memory, so the same graph serves every position.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../internal.h"
#include "gguf.hpp"
#include "planner.hpp"
#include "synapse_b200.h"

namespace {

constexpr size_t kAlign = 256;

struct weight {
    int type = -1, layout = SYN_LAYOUT_PLANAR, rows = 0, cols = 0;
    size_t off = 0, bytes = 0;
    bool quant() const { return type == SYN_Q4_0 || type == SYN_Q8_0; }
    bool kquant() const { return type == SYN_Q4_K || type == SYN_Q6_K; }  // on Q8_K activations
};

// A file tensor (rows first .. first + rows - 1 of it) inside a (possibly
// fused) device matrix: its row first + i is the matrix's row row0 + i * step.
struct source {
    std::string name;
    const weight* w = nullptr;
    int row0 = 0, step = 1, rows = 0;
    int first = 0;
};

struct layer_w {
    weight attn_norm, ffn_norm;
    weight q, k, v;   // q holds k and v too when fused_qkv
    weight o;
    weight gate, up;  // gate holds up too when fused_gu
    weight down;
    bool fused_qkv = false, fused_gu = false;
    bool gu_pairs = false;  // gate/up rows interleaved (gate i at 2i, up i at 2i+1) for the silu-pair epilogue
};

enum class opk { embed, rms_norm, quantize, quantize_k, matmul, attention, silu_mul, argmax, allgather };

struct op {
    opk kind;
    const weight* w = nullptr;
    int in = -1, in2 = -1, out = -1, out2 = -1, res = -1, scratch = -1;  // tensor ids
    size_t in_off = 0, out_off = 0, in2_off = 0, res_off = 0;           // float offsets inside tensors
    int rows = 0, cols = 0;  // allgather: floats per rank at out_off = rank * cols
    int layer = 0;
    int in_mode = SYN_IN_Q8, out_mode = SYN_OUT_ROWS;  // matmul: fused input / output (syn_gemv)
    const weight* gamma = nullptr;                     // matmul with SYN_IN_RMSNORM
    bool in_words = false, res_words = false, out_words = false;  // peer gathers: words in / residual / out
};

struct tensor {
    size_t bytes = 0;
    size_t first = 0, last = 0;
    bool used = false;
    size_t off = 0;
};

}  // namespace

struct syn_session {
    syn_llama_config cfg{};
    int max_ctx = 0, device = 0;
    // run(batch): sequences with their own KV cache, and tokens one batched call carries
    int max_seqs = 1, max_batch = 1;
    struct batch_buffers {
        size_t tok, pos, arg, x, x2, q, k, v, attn, act, gu, g, u, logits, scratch, am_ws;
    } bo{};
    syn_tp* tp = nullptr;   // tensor-parallel group (not owned); NULL = one GPU
    syn_tp_layout part{};   // this rank's share (the whole model when world = 1)
    // Gathers by peer stores (world > 1): the producers store into every
    // rank's arena (mapped by CUDA IPC) and raise flags; else NCCL all-gathers.
    bool p2p = false;
    int n_gathers = 0;
    int logits_plain_t = -1;  // the logits as floats (the argmax unpacks the gathered words)
    size_t tp_off = 0;        // peers[8], epoch at +64, wait errors at +68
    std::vector<void*> peer_maps;
    cudaStream_t stream = nullptr;
    char* arena = nullptr;
    size_t arena_bytes = 0, weight_bytes = 0, kv_bytes = 0, act_bytes = 0;
    weight embd, out_norm, head;
    std::vector<layer_w> layers;
    std::vector<source> sources;
    size_t ff_off = 0;  // freq factors (floats), 0 = none
    bool has_ff = false;
    size_t kv_off = 0;
    size_t act_off = 0;
    size_t io_off = 0, forced_off = 0, hist_off = 0, argmax_ws_off = 0;
    size_t rope_tab_off = 0;  // (cos, sin) of every RoPE pair at every position < max_ctx
    std::vector<tensor> tensors;
    std::vector<op> ops;
    int logits_t = -1;
    float theta_scale = 0, scale = 0;
    int attn_order = SYN_ORDER_REFERENCE;  // SYN_ATTN_ORDER=split: the split p.V sums
    // host side
    int32_t* h_io = nullptr;   // pinned: token, pos
    float* h_logits = nullptr; // pinned
    int32_t* h_next = nullptr; // pinned
    // Health of the last step, copied out by the step graph: the peer word reads
    // that gave up (tensor parallelism) and the device's counters of bounded copy
    // waits that gave up (GEMV, attention), against their values at open.
    unsigned* h_status = nullptr;  // pinned: [0] peer wait errors, [1] GEMV, [2] attention
    unsigned* gemv_to = nullptr;
    unsigned* attn_to = nullptr;
    unsigned status_base[2] = {0, 0};
    unsigned long long tp_wait_ns = 2000000000ull;  // SYN_TP_WAIT_MS
    bool failed = false;  // a step found a wait that gave up: every later step fails too
    cudaGraphExec_t step_exec = nullptr, gen_exec = nullptr, prof_exec = nullptr;
    std::vector<cudaEvent_t> prof_events;
    bool use_graph = true;

    template <typename T>
    T* at(size_t off) { return reinterpret_cast<T*>(arena + off); }
    float* tf(int t, size_t off = 0) { return at<float>(act_off + tensors[t].off) + off; }
    float* logits() { return tf(p2p ? logits_plain_t : logits_t); }
    void* tb(int t) { return arena + act_off + tensors[t].off; }
    int32_t* io() { return at<int32_t>(io_off); }
    // halves of one sequence's cache of one layer (K or V); sequence i's rows follow sequence i - 1's
    size_t seq_halves() const { return size_t(max_ctx) * part.n_kv * cfg.head_dim; }
    uint16_t* kv(int layer, int which, int seq = 0) {
        return at<uint16_t>(kv_off) + ((size_t(layer) * 2 + which) * max_seqs + seq) * seq_halves();
    }
};

namespace {

int set_err(int st, const std::string& msg) {
    syn_set_error(msg.c_str());
    return st;
}

int cuda(cudaError_t e) {
    if (e == cudaSuccess) return SYN_OK;
    syn_set_error((std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e)).c_str());
    return e == cudaErrorMemoryAllocation ? SYN_ERR_NO_MEMORY : SYN_ERR_CUDA;
}

bool supported_type(int t) { return t == SYN_F32 || t == SYN_F16 || t == SYN_Q4_0 || t == SYN_Q8_0; }
// matrices that only multiply (not the embedding table): the K formats too
bool supported_matrix_type(int t) { return supported_type(t) || t == SYN_Q4_K || t == SYN_Q6_K; }
bool planar_type(int t) { return t == SYN_Q4_0 || t == SYN_Q8_0 || t == SYN_Q4_K || t == SYN_Q6_K; }

size_t weight_size(int type, int rows, int cols) {
    return syn_weight_bytes(type, rows, cols, planar_type(type) ? SYN_LAYOUT_PLANAR : SYN_LAYOUT_GGUF);
}

// ---- arena layout -------------------------------------------------------------

struct layout_builder {
    size_t off = 0;
    size_t take(size_t bytes) {
        const size_t o = off;
        off = (off + bytes + kAlign - 1) / kAlign * kAlign;
        return o;
    }
};

void define(weight& w, int type, int rows, int cols, layout_builder& lb) {
    w.type = type;
    w.rows = rows;
    w.cols = cols;
    w.layout = planar_type(type) ? SYN_LAYOUT_PLANAR : SYN_LAYOUT_GGUF;
    w.bytes = weight_size(type, rows, cols);
    w.off = lb.take(w.bytes);
}

// ---- the step graph --------------------------------------------------------

struct graph_builder {
    syn_session& s;
    int new_tensor(size_t bytes) {
        tensor t;
        t.bytes = bytes;
        s.tensors.push_back(t);
        return int(s.tensors.size() - 1);
    }
    void use(int t) {
        if (t < 0) return;
        tensor& x = s.tensors[t];
        const size_t i = s.ops.size();  // index of the op being added
        if (!x.used) { x.first = i; x.used = true; }
        x.last = i;
    }
    void add(op o) {
        use(o.in); use(o.in2); use(o.out); use(o.out2); use(o.res); use(o.scratch);
        s.ops.push_back(o);
    }
};

size_t act_bytes_for(int cols) { return syn_q8_act_bytes(1, cols); }

size_t act_k_bytes_for(int cols) { return syn_q8k_act_bytes(1, cols); }

// Activation input of a matmul: the Q8_0 form for Q4_0 / Q8_0 weights, the
// Q8_K form for the K formats (made from the floats on first use), else f32.
struct activation {
    int f32 = -1;  // tensor with float values
    int q8 = -1;   // tensor with Q8_0 activations
    int qk = -1;   // tensor with Q8_K activations
};

bool fusable(const weight& w, int out_mode = SYN_OUT_ROWS) {
    return w.quant() && syn_gemv_fusable(w.type, w.layout, w.rows, w.cols, 1, out_mode);
}

// The step as ops. Where the pipelined GEMV takes the shape, each matmul
// absorbs its neighbours: the rms_norm (and Q8_0 quantization) before it, the
// residual add after it, and for gate/up the silu * up epilogue, so a layer is
// four GEMVs and one attention launch.
//
// Sharded over world > 1 ranks, every matrix holds this rank's output rows,
// attention runs this rank's heads, and each op writes its slice in place
// into a whole-width tensor that an all-gather then completes on every rank:
// the attention output, the residual after O, silu * up, the residual after
// down, and the logits. Inputs (x, the gathered vectors) are whole on every
// rank, so each output element is computed exactly as on one GPU.
void build_step(syn_session& s) {
    const syn_llama_config& c = s.cfg;
    const syn_tp_layout& P = s.part;
    const bool tp = P.world > 1;
    graph_builder g{s};
    const int d = c.n_embd, hd = c.head_dim, ff = c.n_ff;
    const int qrows = P.n_head * hd, kvrows = P.n_kv * hd, qall = c.n_head * hd;  // rank's Q, K (V) rows; all heads
    const size_t x_off = size_t(P.embd0), a_off = size_t(P.head0) * hd, f_off = size_t(P.ff0);

    auto gather = [&](int t, int per_rank) {
        if (!tp) return;
        op o{opk::allgather};
        o.out = t;
        o.cols = per_rank;
        g.add(o);
    };
    int x = g.new_tensor(size_t(d) * 4);
    {
        op o{opk::embed};
        o.w = &s.embd;
        o.out = x;
        g.add(o);
    }
    auto norm = [&](int in, const weight& gamma, bool need_f32, bool need_q8) {
        activation a;
        op o{opk::rms_norm};
        o.w = &gamma;
        o.in = in;
        o.cols = d;
        if (need_f32) a.f32 = o.out = g.new_tensor(size_t(d) * 4);
        if (need_q8) a.q8 = o.out2 = g.new_tensor(act_bytes_for(d));
        g.add(o);
        return a;
    };
    auto matmul = [&](const weight& w, activation& a, int out, size_t out_off, int res, size_t res_off) {
        if (w.kquant() && a.qk < 0) {  // quantize_row_q8_k of the floats, once per activation
            op q{opk::quantize_k};
            q.in = a.f32;
            q.out = a.qk = g.new_tensor(act_k_bytes_for(w.cols));
            q.cols = w.cols;
            g.add(q);
        }
        op o{opk::matmul};
        o.w = &w;
        o.in = w.quant() ? a.q8 : w.kquant() ? a.qk : a.f32;
        o.out = out;
        o.out_off = out_off;
        o.res = res;
        o.res_off = res_off;
        o.rows = w.rows;
        o.cols = w.cols;
        g.add(o);
    };
    // y = W * prologue(in) (+ res), the input floats quantized inside the GEMV
    auto fused = [&](const weight& w, int in, const weight* gamma, int out, size_t out_off, int res, size_t res_off,
                     int out_mode) {
        op o{opk::matmul};
        o.w = &w;
        o.in = in;
        o.gamma = gamma;
        o.in_mode = gamma ? SYN_IN_RMSNORM : SYN_IN_F32;
        o.out_mode = out_mode;
        o.out = out;
        o.out_off = out_off;
        o.res = res;
        o.res_off = res_off;
        o.rows = w.rows;
        o.cols = w.cols;
        g.add(o);
    };
    auto quantize = [&](int in, int cols) {
        activation a;
        a.f32 = in;
        a.q8 = g.new_tensor(act_bytes_for(cols));
        op o{opk::quantize};
        o.in = in;
        o.out = a.q8;
        o.cols = cols;
        g.add(o);
        return a;
    };
    for (int l = 0; l < c.n_layer; ++l) {
        const layer_w& L = s.layers[l];
        const int qkv = g.new_tensor(size_t(qrows + 2 * kvrows) * 4);
        if (L.fused_qkv && fusable(L.q)) {
            fused(L.q, x, &L.attn_norm, qkv, 0, -1, 0, SYN_OUT_ROWS);
        } else {
            const bool qk_any = L.q.quant() || (!L.fused_qkv && (L.k.quant() || L.v.quant()));
            const bool qk_f = !L.q.quant() || (!L.fused_qkv && (!L.k.quant() || !L.v.quant()));
            activation h = norm(x, L.attn_norm, qk_f, qk_any);
            matmul(L.q, h, qkv, 0, -1, 0);
            if (!L.fused_qkv) {
                matmul(L.k, h, qkv, qrows, -1, 0);
                matmul(L.v, h, qkv, qrows + kvrows, -1, 0);
            }
        }
        const int attn = g.new_tensor(size_t(qall) * 4);
        {
            op o{opk::attention};
            o.in = qkv;
            o.out = attn;
            o.out_off = a_off;
            o.layer = l;
            o.scratch = g.new_tensor(syn_attention_scratch_bytes(1, P.n_head, P.n_kv, hd, s.max_ctx));
            g.add(o);
        }
        gather(attn, qrows);
        const int x2 = g.new_tensor(size_t(d) * 4);
        if (fusable(L.o)) {
            fused(L.o, attn, nullptr, x2, x_off, x, x_off, SYN_OUT_ROWS);
        } else {
            activation a;
            a.f32 = attn;
            if (L.o.quant()) a = quantize(attn, qall);
            matmul(L.o, a, x2, x_off, x, x_off);
        }
        gather(x2, P.n_embd);
        x = x2;
        const int x3 = g.new_tensor(size_t(d) * 4);
        if (L.gu_pairs) {  // fusable(L.gate, SYN_OUT_SILU_PAIRS) held when the rows were interleaved
            const int act = g.new_tensor(size_t(ff) * 4);
            fused(L.gate, x, &L.ffn_norm, act, f_off, -1, 0, SYN_OUT_SILU_PAIRS);
            gather(act, P.n_ff);
            if (fusable(L.down)) {
                fused(L.down, act, nullptr, x3, x_off, x, x_off, SYN_OUT_ROWS);
            } else {
                activation f;
                f.f32 = act;
                if (L.down.quant()) f = quantize(act, ff);
                matmul(L.down, f, x3, x_off, x, x_off);
            }
        } else {
            const bool gu_any = L.gate.quant() || (!L.fused_gu && L.up.quant());
            const bool gu_f = !L.gate.quant() || (!L.fused_gu && !L.up.quant());
            activation h2 = norm(x, L.ffn_norm, gu_f, gu_any);
            const int gu = g.new_tensor(size_t(2) * P.n_ff * 4);
            matmul(L.gate, h2, gu, 0, -1, 0);
            if (!L.fused_gu) matmul(L.up, h2, gu, size_t(P.n_ff), -1, 0);
            activation f;
            {
                op o{opk::silu_mul};
                o.in = gu;
                o.cols = P.n_ff;
                if (tp) {  // floats into the whole-width tensor, gathered, then quantized whole
                    f.f32 = o.out = g.new_tensor(size_t(ff) * 4);
                    o.out_off = f_off;
                } else if (L.down.quant()) {
                    f.q8 = o.out2 = g.new_tensor(act_bytes_for(ff));
                } else {
                    f.f32 = o.out = g.new_tensor(size_t(ff) * 4);
                }
                g.add(o);
            }
            if (tp) {
                gather(f.f32, P.n_ff);
                if (L.down.quant()) f = quantize(f.f32, ff);
            }
            matmul(L.down, f, x3, x_off, x, x_off);
        }
        gather(x3, P.n_embd);
        x = x3;
    }
    s.logits_t = g.new_tensor(size_t(c.n_vocab) * 4);
    if (fusable(s.head)) {
        fused(s.head, x, &s.out_norm, s.logits_t, size_t(P.vocab0), -1, 0, SYN_OUT_ROWS);
    } else {
        activation hl = norm(x, s.out_norm, !s.head.quant(), s.head.quant());
        matmul(s.head, hl, s.logits_t, size_t(P.vocab0), -1, 0);
    }
    gather(s.logits_t, P.n_vocab);
    {
        op o{opk::argmax};
        o.in = s.logits_t;
        g.add(o);
    }
    // the logits are the step's output: live to the end (planner.hpp liveness)
    s.tensors[s.logits_t].last = s.ops.size() - 1;
}

// Gathers by peer stores, when every gather's producer is the attention
// kernel or a staged GEMV and every reader of a gathered tensor (as input or
// residual) is a staged GEMV or the argmax (the Llama shapes), world <=
// kTpMaxWorld, and SYN_TP_P2P is not "0". A gathered tensor then holds words
// ({float, epoch}, twice the bytes) and lives for the whole step: peers write
// it while this rank may still run earlier ops, so no other tensor may share
// its bytes. Whether the peers' arenas can be mapped is settled later
// (map_peers); without it the NCCL all-gathers run on the same tensors.
void plan_p2p(syn_session& s) {
    s.n_gathers = 0;
    if (s.part.world <= 1 || s.part.world > kTpMaxWorld) return;
    const char* env = std::getenv("SYN_TP_P2P");
    if (env && env[0] == '0') return;
    auto staged = [](const op& o) {
        return o.kind == opk::matmul && o.in_mode != SYN_IN_Q8 && o.w->quant() &&
               syn_gemv_fusable(o.w->type, o.w->layout, o.rows, o.cols, 1, o.out_mode);
    };
    std::vector<op> ops = s.ops;
    std::vector<int> gathered;
    for (size_t i = 0; i < ops.size(); ++i) {
        if (ops[i].kind != opk::allgather) continue;
        const int t = ops[i].out;
        if (i == 0) return;
        op& prod = ops[i - 1];
        if (prod.out != t || !(prod.kind == opk::attention || staged(prod))) return;
        prod.out_words = true;
        for (size_t m = i + 1; m < ops.size(); ++m) {
            op& r = ops[m];
            if (r.in2 == t || ((r.in == t || r.res == t) && !(staged(r) || (r.kind == opk::argmax && r.in == t))))
                return;
            if (r.in == t) r.in_words = true;
            if (r.res == t) r.res_words = true;
        }
        gathered.push_back(t);
    }
    s.ops.swap(ops);
    s.n_gathers = int(gathered.size());
    for (int t : gathered) {
        s.tensors[t].bytes *= 2;
        s.tensors[t].first = 0;
        s.tensors[t].last = s.ops.size() - 1;
    }
    graph_builder g{s};
    s.logits_plain_t = g.new_tensor(size_t(s.cfg.n_vocab) * 4);
    s.tensors[s.logits_plain_t].used = true;
    s.tensors[s.logits_plain_t].first = 0;
    s.tensors[s.logits_plain_t].last = s.ops.size() - 1;
}

int plan_step(syn_session& s) {
    std::vector<syn::plan::tensor> ts;
    for (const tensor& t : s.tensors) ts.push_back({t.bytes, t.first, t.last});
    const syn::plan::result r = syn::plan::place(ts, kAlign);
    if (!syn::plan::valid(ts, r, kAlign)) return set_err(SYN_ERR_INVALID, "arena plan violates P1-P3");
    for (size_t i = 0; i < s.tensors.size(); ++i) s.tensors[i].off = r.offset[i];
    s.act_bytes = r.arena_bytes;
    return SYN_OK;
}

// ---- execution ---------------------------------------------------------------

int enqueue_ops(syn_session& s, cudaStream_t st);
TpSync tp_sync(syn_session& s, const op& o);

int enqueue_ops(syn_session& s, cudaStream_t st) {
    const syn_llama_config& c = s.cfg;
    const int qrows = s.part.n_head * c.head_dim, kvrows = s.part.n_kv * c.head_dim;  // this rank's heads
    int rc = SYN_OK;
    for (const op& o : s.ops) {
        switch (o.kind) {
        case opk::embed:
            if (s.p2p) rc = syn_tp_step_begin(s.at<unsigned>(s.tp_off + 64), st);  // this step's epoch
            if (!rc)
                rc = syn_embed(s.embd.type, s.arena + s.embd.off, s.embd.layout, s.embd.rows, s.embd.cols, s.io(), 1,
                               s.tf(o.out), st);
            break;
        case opk::rms_norm:
            rc = syn_rms_norm(s.tf(o.in), s.at<float>(o.w->off), 1, o.cols, c.rms_eps,
                              o.out >= 0 ? s.tf(o.out) : nullptr, o.out2 >= 0 ? s.tb(o.out2) : nullptr, st);
            break;
        case opk::quantize:
            rc = syn_quantize_q8_0(s.tf(o.in), 1, o.cols, s.tb(o.out), st);
            break;
        case opk::quantize_k:
            rc = syn_quantize_q8_k(s.tf(o.in), 1, o.cols, s.tb(o.out), st);
            break;
        case opk::matmul: {
            float* y = s.tf(o.out, o.out_off);
            const float* res = o.res < 0 ? nullptr
                               : o.res_words && s.p2p ? reinterpret_cast<const float*>(
                                                            static_cast<char*>(s.tb(o.res)) + o.res_off * 8)
                                                      : s.tf(o.res, o.res_off);
            if (o.in_mode != SYN_IN_Q8 || o.out_mode != SYN_OUT_ROWS) {
                syn_gemv_args a{};
                a.type = o.w->type;
                a.layout = o.w->layout;
                a.rows = o.rows;
                a.cols = o.cols;
                a.n_tok = 1;
                a.w = s.arena + o.w->off;
                a.in_mode = o.in_mode;
                a.x = s.tf(o.in);
                a.gamma = o.gamma ? s.at<float>(o.gamma->off) : nullptr;
                a.eps = c.rms_eps;
                a.out_mode = o.out_mode;
                a.y = y;
                a.residual = res;
                rc = s.p2p && (o.in_words || o.res_words || o.out_words) ? syn_gemv_tp(&a, tp_sync(s, o), st)
                                                                         : syn_gemv(&a, st);
            } else if (o.w->quant() || o.w->kquant())
                rc = syn_gemv_q(o.w->type, s.arena + o.w->off, o.w->layout, o.w->rows, o.w->cols, s.tb(o.in), 1, y,
                                res, st);
            else
                rc = syn_gemv_f(o.w->type, s.arena + o.w->off, o.w->rows, o.w->cols, s.tf(o.in), 1, y, res, st);
            break;
        }
        case opk::attention: {
            syn_attention_args a{};
            float* qkv = s.tf(o.in);
            a.q = qkv;
            a.k = qkv + qrows;
            a.v = qkv + qrows + kvrows;
            a.k_cache = s.kv(o.layer, 0);
            a.v_cache = s.kv(o.layer, 1);
            a.pos = s.io() + 1;
            a.out = s.tf(o.out, o.out_off);
            a.scratch = s.tb(o.scratch);
            a.cache_stride = 0;
            a.n_q = 1;
            a.n_head = s.part.n_head;
            a.n_kv = s.part.n_kv;
            a.head_dim = c.head_dim;
            a.max_len = s.max_ctx;
            a.append = 1;
            a.rope = 1;
            a.rope_mode = c.rope_mode;
            a.theta_scale = s.theta_scale;
            a.scale = s.scale;
            a.freq_factors = s.has_ff ? s.at<float>(s.ff_off) : nullptr;
            a.rope_table = s.at<float>(s.rope_tab_off);
            a.order = s.attn_order;
            rc = s.p2p && o.out_words ? syn_attention_tp(&a, tp_sync(s, o), st) : syn_attention(&a, st);
            break;
        }
        case opk::silu_mul:
            rc = syn_silu_mul(s.tf(o.in), s.tf(o.in, size_t(o.cols)), 1, o.cols,
                              o.out >= 0 ? s.tf(o.out, o.out_off) : nullptr, o.out2 >= 0 ? s.tb(o.out2) : nullptr, st);
            break;
        case opk::allgather:
            if (!s.p2p) rc = syn_allgather(s.tp, s.tf(o.out), size_t(o.cols) * 4, st);  // else the producer pushed it
            break;
        case opk::argmax:
            rc = s.p2p && o.in_words
                     ? syn_argmax_ws_tp(s.tb(o.in), c.n_vocab, s.io() + 2, s.tf(s.logits_plain_t),
                                        s.arena + s.argmax_ws_off, tp_sync(s, o), st)
                     : syn_argmax_ws(s.tf(o.in), 1, c.n_vocab, s.io() + 2, s.arena + s.argmax_ws_off, st);
            break;
        }
        if (rc) return rc;
    }
    return SYN_OK;
}

// The step's health words into the pinned status block (see syn_session).
int enqueue_status(syn_session& s, cudaStream_t st) {
    int rc = SYN_OK;
    if (s.p2p) rc = cuda(cudaMemcpyAsync(s.h_status, s.arena + s.tp_off + 68, 4, cudaMemcpyDeviceToHost, st));
    if (!rc && s.gemv_to) rc = cuda(cudaMemcpyAsync(s.h_status + 1, s.gemv_to, 4, cudaMemcpyDeviceToHost, st));
    if (!rc && s.attn_to) rc = cuda(cudaMemcpyAsync(s.h_status + 2, s.attn_to, 4, cudaMemcpyDeviceToHost, st));
    return rc;
}

// SYN_ERR_TIMEOUT once a bounded wait has given up (the session stays failed:
// a peer's words that never arrived leave later reads unwaited, and a copy
// that never landed leaves its kernel's output incomplete).
int check_status(syn_session& s) {
    if (!s.failed && (s.h_status[0] != 0 || s.h_status[1] != s.status_base[0] || s.h_status[2] != s.status_base[1])) {
        s.failed = true;
        char msg[160];
        std::snprintf(msg, sizeof msg, "a bounded wait gave up: %u peer word reads, %u GEMV and %u attention copies",
                      s.h_status[0], s.h_status[1] - s.status_base[0], s.h_status[2] - s.status_base[1]);
        syn_set_error(msg);
    }
    return s.failed ? SYN_ERR_TIMEOUT : SYN_OK;
}

int enqueue_step(syn_session& s, cudaStream_t st) {
    int rc = cuda(cudaMemcpyAsync(s.io(), s.h_io, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    if (!rc) rc = enqueue_ops(s, st);
    if (!rc) rc = cuda(cudaMemcpyAsync(s.h_logits, s.logits(), size_t(s.cfg.n_vocab) * 4,
                                       cudaMemcpyDeviceToHost, st));
    if (!rc) rc = cuda(cudaMemcpyAsync(s.h_next, s.io() + 2, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    if (!rc) rc = enqueue_status(s, st);
    return rc;
}

int enqueue_gen(syn_session& s, cudaStream_t st) {
    int rc = enqueue_ops(s, st);
    if (!rc) rc = syn_advance(s.io(), s.at<int32_t>(s.forced_off), s.at<int32_t>(s.hist_off), st);
    return rc;
}

// Programmatic dependent launch on for the launches of one scope.
struct pdl_scope {
    explicit pdl_scope(bool on) { syn_set_pdl(on ? 1 : 0); }
    ~pdl_scope() { syn_set_pdl(0); }
};

bool pdl_wanted() {
    const char* env = std::getenv("SYN_PDL");
    return !(env && env[0] == '0');
}

int capture(syn_session& s, int (*fn)(syn_session&, cudaStream_t), cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    int rc = cuda(cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal));
    if (rc) return rc;
    int body;
    {
        pdl_scope pdl(pdl_wanted());
        body = fn(s, s.stream);
    }
    rc = cuda(cudaStreamEndCapture(s.stream, &g));
    if (body) {
        if (g) cudaGraphDestroy(g);
        return body;
    }
    if (rc) return rc;
    rc = cuda(cudaGraphInstantiate(out, g, 0));
    cudaGraphDestroy(g);
    return rc;
}

// ---- config + weights ---------------------------------------------------------

int finish(syn_session& s, layout_builder& lb) {
    const syn_llama_config& c = s.cfg;
    s.weight_bytes = lb.off;
    s.kv_bytes = size_t(c.n_layer) * 2 * s.max_seqs * s.seq_halves() * 2;
    s.kv_off = lb.take(s.kv_bytes);
    build_step(s);
    plan_p2p(s);
    int rc = plan_step(s);
    if (rc) return rc;
    s.act_off = lb.take(s.act_bytes);
    s.io_off = lb.take(64);
    s.forced_off = lb.take(size_t(s.max_ctx) * 4);
    s.hist_off = lb.take(size_t(s.max_ctx) * 4);
    s.argmax_ws_off = lb.take(syn_argmax_ws_bytes(1));  // persistent: its counters must stay zero between steps
    s.rope_tab_off = lb.take(size_t(s.max_ctx) * c.head_dim * 4);
    if (s.n_gathers) s.tp_off = lb.take(128);  // peers[8], epoch at +64, wait errors at +68
    if (s.max_batch > 1 || s.max_seqs > 1) {  // run(batch) buffers: max_batch rows each
        const size_t B = size_t(s.max_batch), d = size_t(c.n_embd), hd = size_t(c.head_dim);
        const size_t qall = size_t(c.n_head) * hd, kvall = size_t(c.n_head_kv) * hd, ff = size_t(c.n_ff);
        const int widest = int(std::max({d, qall, ff}));
        s.bo.tok = lb.take(B * 4);
        s.bo.pos = lb.take(B * 4);
        s.bo.arg = lb.take(B * 4);
        s.bo.x = lb.take(B * d * 4);
        s.bo.x2 = lb.take(B * d * 4);
        s.bo.q = lb.take(B * qall * 4);
        s.bo.k = lb.take(B * kvall * 4);
        s.bo.v = lb.take(B * kvall * 4);
        s.bo.attn = lb.take(B * qall * 4);
        s.bo.act = lb.take(syn_q8_act_bytes(s.max_batch, widest));
        s.bo.gu = lb.take(B * 2 * ff * 4);
        s.bo.g = lb.take(B * ff * 4);
        s.bo.u = lb.take(B * ff * 4);
        s.bo.logits = lb.take(B * size_t(c.n_vocab) * 4);
        s.bo.scratch = lb.take(syn_attention_scratch_bytes(s.max_batch, c.n_head, c.n_head_kv, c.head_dim, s.max_ctx));
        s.bo.am_ws = lb.take(syn_argmax_ws_bytes(s.max_batch));
    }
    s.arena_bytes = lb.off;
    if (const char* e = std::getenv("SYN_ATTN_ORDER")) s.attn_order = std::strcmp(e, "split") == 0 ? SYN_ORDER_SPLIT : SYN_ORDER_REFERENCE;
    s.theta_scale = std::pow(c.rope_base, -2.0f / float(c.head_dim));  // attention.hpp:47
    s.scale = 1.0f / std::sqrt(float(c.head_dim));                      // llama.hpp:407
    if ((rc = cuda(cudaSetDevice(s.device)))) return rc;
    if ((rc = cuda(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking)))) return rc;
    if ((rc = cuda(cudaMalloc(&s.arena, s.arena_bytes)))) return rc;
    if ((rc = cuda(cudaMemset(s.arena + s.kv_off, 0, s.arena_bytes - s.kv_off)))) return rc;
    if ((rc = cuda(cudaMallocHost(&s.h_io, 64)))) return rc;
    if ((rc = cuda(cudaMallocHost(&s.h_logits, size_t(c.n_vocab) * 4 * std::max(1, s.max_batch))))) return rc;
    if ((rc = cuda(cudaMallocHost(&s.h_next, 64)))) return rc;
    if ((rc = cuda(cudaMallocHost(&s.h_status, 64)))) return rc;
    std::memset(s.h_status, 0, 64);
    if (const char* e = std::getenv("SYN_TP_WAIT_MS")) {
        const double ms = std::atof(e);
        if (ms > 0) s.tp_wait_ns = (unsigned long long)(ms * 1e6);
    }
    s.gemv_to = syn_gemv_timeout_word();
    s.attn_to = syn_attn_timeout_word();
    if (s.gemv_to && (rc = cuda(cudaMemcpy(&s.status_base[0], s.gemv_to, 4, cudaMemcpyDeviceToHost)))) return rc;
    if (s.attn_to && (rc = cuda(cudaMemcpy(&s.status_base[1], s.attn_to, 4, cudaMemcpyDeviceToHost)))) return rc;
    s.h_status[1] = s.status_base[0];
    s.h_status[2] = s.status_base[1];
    return SYN_OK;
}

// Map every peer's arena (CUDA IPC handles exchanged over the group) and put
// the bases in the arena for the kernels. Collective: every rank learns
// whether all ranks mapped theirs, and all use peer stores or none does.
int map_peers(syn_session& s) {
    s.p2p = false;
    if (!s.n_gathers) return SYN_OK;
    const int world = s.part.world, rank = s.part.rank;
    struct entry {
        cudaIpcMemHandle_t h;
        int ok;
    } mine{}, all[kTpMaxWorld];
    mine.ok = cudaIpcGetMemHandle(&mine.h, s.arena) == cudaSuccess;
    if (!mine.ok) cudaGetLastError();
    int rc = syn_tp_exchange(s.tp, &mine, all, sizeof(entry));
    if (rc) return rc;
    char* bases[kTpMaxWorld] = {};
    bool ok = true;
    for (int r = 0; r < world; ++r) ok = ok && all[r].ok;
    for (int r = 0; r < world && ok; ++r) {
        if (r == rank) {
            bases[r] = s.arena;
            continue;
        }
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[r].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
            break;
        }
        s.peer_maps.push_back(p);
        bases[r] = static_cast<char*>(p);
    }
    entry verdict{}, verdicts[kTpMaxWorld];
    verdict.ok = ok;
    if ((rc = syn_tp_exchange(s.tp, &verdict, verdicts, sizeof(entry)))) return rc;
    for (int r = 0; r < world; ++r) ok = ok && verdicts[r].ok;
    if (!ok) {
        for (void* p : s.peer_maps) cudaIpcCloseMemHandle(p);
        s.peer_maps.clear();
        return SYN_OK;  // NCCL all-gathers on every rank
    }
    rc = cuda(cudaMemcpy(s.arena + s.tp_off, bases, sizeof bases, cudaMemcpyHostToDevice));
    if (!rc) s.p2p = true;
    return rc;
}

// The gather hooks of op o (peers mapped).
TpSync tp_sync(syn_session& s, const op& o) {
    TpSync t;
    t.peers = s.at<char*>(s.tp_off);
    t.epoch = s.at<unsigned>(s.tp_off + 64);
    t.err = s.at<unsigned>(s.tp_off + 68);
    t.world = s.part.world;
    t.rank = s.part.rank;
    t.in_ll = o.in_words;
    t.res_ll = o.res_words;
    t.out_ll = o.out_words;
    t.wait_ns = s.tp_wait_ns;
    if (o.out_words) t.out_off = s.act_off + s.tensors[o.out].off + o.out_off * 8;
    return t;
}

// The RoPE table, one eager step at position 0 (sets per-device kernel
// attributes outside any capture), then the KV cache and io are cleared and
// both graphs captured.
int warm_and_capture(syn_session& s) {
    s.h_io[0] = 0;
    s.h_io[1] = 0;
    if (int rc = map_peers(s)) return rc;
    int rc = syn_rope_table(s.at<float>(s.rope_tab_off), s.max_ctx, s.cfg.head_dim, s.theta_scale,
                            s.has_ff ? s.at<float>(s.ff_off) : nullptr, nullptr, s.stream);
    if (!rc) rc = enqueue_step(s, s.stream);
    if (!rc) rc = cuda(cudaStreamSynchronize(s.stream));
    if (!rc) rc = cuda(cudaMemsetAsync(s.arena + s.kv_off, 0, s.kv_bytes, s.stream));
    if (!rc) rc = cuda(cudaMemsetAsync(s.io(), 0, 64, s.stream));
    if (!rc) rc = cuda(cudaStreamSynchronize(s.stream));
    if (rc) return rc;
    const char* env = std::getenv("SYN_NO_GRAPH");
    s.use_graph = !(env && env[0] == '1');
    if (s.use_graph) {
        if ((rc = capture(s, enqueue_step, &s.step_exec))) return rc;
        if ((rc = capture(s, enqueue_gen, &s.gen_exec))) return rc;
    }
    return SYN_OK;
}

// Each layer's matrices as this rank holds them (the whole model at world
// 1): Q/K/V rows of its heads (fused into one matrix when their types
// match), its rows of O, gate/up (interleaved in pairs for the silu epilogue
// when that kernel takes the shape) and down, and the norms whole.
void layer_layout(syn_session& s, const std::vector<std::vector<int>>& types, layout_builder& lb) {
    const syn_llama_config& c = s.cfg;
    const syn_tp_layout& P = s.part;
    const int d = c.n_embd, hd = c.head_dim, qall = c.n_head * hd;
    const int qrows = P.n_head * hd, kvrows = P.n_kv * hd, ff = P.n_ff;
    const int q0 = P.head0 * hd, kv0 = P.kv_head0 * hd;
    s.layers.resize(c.n_layer);
    for (int l = 0; l < c.n_layer; ++l) {
        layer_w& L = s.layers[l];
        const std::vector<int>& t = types[l];  // attn_norm, q, k, v, o, ffn_norm, gate, up, down
        const std::string p = "blk." + std::to_string(l) + ".";
        define(L.attn_norm, SYN_F32, 1, d, lb);
        L.fused_qkv = t[1] == t[2] && t[1] == t[3] && (t[1] == SYN_Q4_0 || t[1] == SYN_Q8_0);
        if (L.fused_qkv) {
            define(L.q, t[1], qrows + 2 * kvrows, d, lb);
            s.sources.push_back({p + "attn_q.weight", &L.q, 0, 1, qrows, q0});
            s.sources.push_back({p + "attn_k.weight", &L.q, qrows, 1, kvrows, kv0});
            s.sources.push_back({p + "attn_v.weight", &L.q, qrows + kvrows, 1, kvrows, kv0});
        } else {
            define(L.q, t[1], qrows, d, lb);
            define(L.k, t[2], kvrows, d, lb);
            define(L.v, t[3], kvrows, d, lb);
            s.sources.push_back({p + "attn_q.weight", &L.q, 0, 1, qrows, q0});
            s.sources.push_back({p + "attn_k.weight", &L.k, 0, 1, kvrows, kv0});
            s.sources.push_back({p + "attn_v.weight", &L.v, 0, 1, kvrows, kv0});
        }
        define(L.o, t[4], P.n_embd, qall, lb);
        s.sources.push_back({p + "attn_output.weight", &L.o, 0, 1, P.n_embd, P.embd0});
        define(L.ffn_norm, SYN_F32, 1, d, lb);
        L.fused_gu = t[6] == t[7] && (t[6] == SYN_Q4_0 || t[6] == SYN_Q8_0);
        if (L.fused_gu) {
            define(L.gate, t[6], 2 * ff, d, lb);
            L.gu_pairs = syn_gemv_fusable(t[6], SYN_LAYOUT_PLANAR, 2 * ff, d, 1, SYN_OUT_SILU_PAIRS) != 0;
            if (L.gu_pairs) {
                s.sources.push_back({p + "ffn_gate.weight", &L.gate, 0, 2, ff, P.ff0});
                s.sources.push_back({p + "ffn_up.weight", &L.gate, 1, 2, ff, P.ff0});
            } else {
                s.sources.push_back({p + "ffn_gate.weight", &L.gate, 0, 1, ff, P.ff0});
                s.sources.push_back({p + "ffn_up.weight", &L.gate, ff, 1, ff, P.ff0});
            }
        } else {
            define(L.gate, t[6], ff, d, lb);
            define(L.up, t[7], ff, d, lb);
            s.sources.push_back({p + "ffn_gate.weight", &L.gate, 0, 1, ff, P.ff0});
            s.sources.push_back({p + "ffn_up.weight", &L.up, 0, 1, ff, P.ff0});
        }
        define(L.down, t[8], P.n_embd, c.n_ff, lb);
        s.sources.push_back({p + "ffn_down.weight", &L.down, 0, 1, P.n_embd, P.embd0});
        s.sources.push_back({p + "attn_norm.weight", &L.attn_norm, 0, 1, 1});
        s.sources.push_back({p + "ffn_norm.weight", &L.ffn_norm, 0, 1, 1});
    }
}

// The output head as this rank holds it: its rows of output.weight, or of
// the token embedding when the two are tied (llama.hpp:471-472).
void head_layout(syn_session& s, layout_builder& lb) {
    const syn_llama_config& c = s.cfg;
    const syn_tp_layout& P = s.part;
    if (c.type_output >= 0) {
        define(s.head, c.type_output, P.n_vocab, c.n_embd, lb);
        s.sources.push_back({"output.weight", &s.head, 0, 1, P.n_vocab, P.vocab0});
    } else {
        s.head = s.embd;
        s.head.off += P.vocab0 ? weight_size(s.embd.type, P.vocab0, c.n_embd) : 0;
        s.head.rows = P.n_vocab;
        s.head.bytes = weight_size(s.embd.type, P.n_vocab, c.n_embd);
    }
}

// Rank's contiguous equal share of every sharded dimension.
int tp_layout(const syn_llama_config& c, int rank, int world, syn_tp_layout& L) {
    if (world < 1 || rank < 0 || rank >= world) return SYN_ERR_INVALID;
    if (c.n_head_kv % world || c.n_embd % world || c.n_ff % world || c.n_vocab % world || c.n_head % c.n_head_kv)
        return SYN_ERR_UNSUPPORTED;
    const int G = c.n_head / c.n_head_kv;
    L.rank = rank;
    L.world = world;
    L.n_kv = c.n_head_kv / world;
    L.kv_head0 = rank * L.n_kv;
    L.n_head = L.n_kv * G;  // the query heads of those KV groups
    L.head0 = L.kv_head0 * G;
    L.n_embd = c.n_embd / world;
    L.embd0 = rank * L.n_embd;
    L.n_ff = c.n_ff / world;
    L.ff0 = rank * L.n_ff;
    L.n_vocab = c.n_vocab / world;
    L.vocab0 = rank * L.n_vocab;
    return SYN_OK;
}

// The session's group and share; the device must be the group's.
int set_part(syn_session& s, syn_tp* tp, int device) {
    int rank = 0, world = 1, tdev = -1;
    syn_tp_info(tp, &rank, &world, &tdev);
    if (tp && tdev != device) return set_err(SYN_ERR_INVALID, "session device differs from the tp group's");
    s.tp = tp;
    const int rc = tp_layout(s.cfg, rank, world, s.part);
    if (rc) return set_err(rc, "tensor parallel: world must divide n_head_kv, n_embd, n_ff and n_vocab");
    return SYN_OK;
}

void destroy(syn_session* s) {
    if (!s) return;
    if (s->device >= 0) cudaSetDevice(s->device);
    if (s->step_exec) cudaGraphExecDestroy(s->step_exec);
    if (s->gen_exec) cudaGraphExecDestroy(s->gen_exec);
    if (s->prof_exec) cudaGraphExecDestroy(s->prof_exec);
    for (auto& e : s->prof_events) cudaEventDestroy(e);
    if (s->stream) cudaStreamSynchronize(s->stream);
    if (!s->peer_maps.empty()) {
        // no rank still stores into another's arena once all have drained (collective)
        syn_tp_barrier(s->tp);
        for (void* p : s->peer_maps) cudaIpcCloseMemHandle(p);
    }
    if (s->arena) cudaFree(s->arena);
    if (s->h_io) cudaFreeHost(s->h_io);
    if (s->h_logits) cudaFreeHost(s->h_logits);
    if (s->h_next) cudaFreeHost(s->h_next);
    if (s->h_status) cudaFreeHost(s->h_status);
    if (s->stream) cudaStreamDestroy(s->stream);
    delete s;
}

// Rows (ne[1]) and columns (ne[0]) of a 2-D GGUF tensor (tensor_view.hpp:5-8).
bool shape_is(const syn::gguf::tensor_info& t, uint64_t rows, uint64_t cols) {
    return t.ne[0] == cols && t.rows() == rows;
}

}  // namespace

// ---- streaming upload -------------------------------------------------------
// The file's bytes reach the arena through two pinned host buffers and two
// device staging buffers of kStageBytes: while the GPU copies piece k in and
// repacks it (planar rows, Q/K/V and gate/up placement), host threads copy
// piece k + 1 out of the mapped file into the other pinned buffer. A piece is
// up to kStageBytes of whole rows of one source; plain F32/F16 rows go from
// the pinned buffer straight to their place in the arena.
constexpr size_t kStageBytes = size_t(64) << 20;

struct upload_piece {
    const source* src;
    const uint8_t* data;  // host (mapped file)
    size_t bytes;
    int r0, n;  // rows of the source
};

// dst[0, n) = src[0, n) on up to `threads` host threads (page faults of a
// cold file are taken in parallel too).
void parallel_copy(void* dst, const void* src, size_t n, unsigned threads) {
    const size_t min_part = size_t(4) << 20;
    unsigned t = unsigned(std::min<size_t>(threads, std::max<size_t>(1, n / min_part)));
    if (t <= 1) {
        std::memcpy(dst, src, n);
        return;
    }
    const size_t part = (n + t - 1) / t;
    std::vector<std::thread> pool;
    pool.reserve(t - 1);
    for (unsigned i = 1; i < t; ++i) {
        const size_t b = std::min(n, size_t(i) * part), e = std::min(n, b + part);
        pool.emplace_back([=] { std::memcpy(static_cast<char*>(dst) + b, static_cast<const char*>(src) + b, e - b); });
    }
    std::memcpy(dst, src, std::min(n, part));
    for (auto& th : pool) th.join();
}

int upload_sources(syn_session& s, const syn::gguf::file& f) {
    std::vector<upload_piece> pieces;
    for (const auto& src : s.sources) {
        const syn::gguf::tensor_info* t = f.tensor(src.name);
        const size_t row_bytes = t->nbytes / size_t(t->rows());
        if (row_bytes > kStageBytes) return set_err(SYN_ERR_UNSUPPORTED, "row wider than the staging buffer: " + src.name);
        const uint8_t* data = f.data(*t) + size_t(src.first) * row_bytes;  // this rank's rows of the tensor
        const int per = int(kStageBytes / row_bytes);
        for (int r0 = 0; r0 < src.rows; r0 += per) {
            const int n = std::min(per, src.rows - r0);
            pieces.push_back({&src, data + size_t(r0) * row_bytes, size_t(n) * row_bytes, r0, n});
        }
    }
    const unsigned threads = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    void* host[2] = {nullptr, nullptr};
    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t free_ev[2] = {nullptr, nullptr};
    bool pending[2] = {false, false};
    int rc = SYN_OK;
    for (int b = 0; b < 2 && !rc; ++b) {
        rc = cuda(cudaHostAlloc(&host[b], kStageBytes, cudaHostAllocDefault));
        if (!rc) rc = cuda(cudaMalloc(&stage[b], kStageBytes));
        if (!rc) rc = cuda(cudaEventCreateWithFlags(&free_ev[b], cudaEventDisableTiming));
    }
    for (size_t k = 0; k < pieces.size() && !rc; ++k) {
        const int b = int(k & 1);
        const upload_piece& pc = pieces[k];
        const weight& w = *pc.src->w;
        if (pending[b] && (rc = cuda(cudaEventSynchronize(free_ev[b])))) break;  // piece k - 2 has left buffer b
        parallel_copy(host[b], pc.data, pc.bytes, threads);
        const int row = pc.src->row0 + pc.r0 * pc.src->step;  // first destination row
        if (w.kquant()) {  // src.step is 1: K matrices are never fused
            const size_t pitch = syn_weight_bytes(w.type, 1, w.cols, SYN_LAYOUT_PLANAR);
            rc = cuda(cudaMemcpyAsync(stage[b], host[b], pc.bytes, cudaMemcpyHostToDevice, s.stream));
            if (!rc) rc = syn_k_repack_rows(w.type, stage[b], pc.n, w.cols, s.arena + w.off + size_t(row) * pitch,
                                            s.stream);
        } else if (!w.quant()) {
            rc = cuda(cudaMemcpyAsync(s.arena + w.off + size_t(row) * w.cols * (w.type == SYN_F32 ? 4 : 2), host[b],
                                      pc.bytes, cudaMemcpyHostToDevice, s.stream));
        } else {
            rc = cuda(cudaMemcpyAsync(stage[b], host[b], pc.bytes, cudaMemcpyHostToDevice, s.stream));
            if (!rc) rc = syn_repack_rows(w.type, stage[b], pc.n, w.cols, s.arena + w.off, w.rows, row, s.stream,
                                          pc.src->step);
        }
        if (!rc) rc = cuda(cudaEventRecord(free_ev[b], s.stream));
        pending[b] = true;
    }
    const int sync_rc = cuda(cudaStreamSynchronize(s.stream));
    if (!rc) rc = sync_rc;
    for (int b = 0; b < 2; ++b) {
        if (free_ev[b]) cudaEventDestroy(free_ev[b]);
        if (stage[b]) cudaFree(stage[b]);
        if (host[b]) cudaFreeHost(host[b]);
    }
    return rc;
}

extern "C" int syn_session_open_gguf(const char* path, int max_ctx, int device, syn_session** out) {
    return syn_session_open_gguf_tp(path, max_ctx, device, nullptr, out);
}

namespace {
bool options_ok(const syn_session_options& o) {
    return o.max_ctx > 0 && o.max_seqs >= 1 && o.max_batch >= 1 && o.max_seqs <= 4096 && o.max_batch <= 64;
}
int open_gguf(const char* path, const syn_session_options& o, int device, syn_tp* tp, syn_session** out);
int open_synthetic(const syn_llama_config* cp, const syn_session_options& o, uint64_t seed, int device, syn_tp* tp,
                   syn_session** out);
}  // namespace

extern "C" int syn_session_open_gguf_tp(const char* path, int max_ctx, int device, syn_tp* tp, syn_session** out) {
    const syn_session_options o{max_ctx, 1, 1};
    return open_gguf(path, o, device, tp, out);
}

extern "C" int syn_session_open_gguf_ex(const char* path, const syn_session_options* o, int device,
                                        syn_session** out) {
    if (!o) return SYN_ERR_INVALID;
    return open_gguf(path, *o, device, nullptr, out);
}

namespace {
int open_gguf(const char* path, const syn_session_options& o, int device, syn_tp* tp, syn_session** out) {
    const int max_ctx = o.max_ctx;
    if (!path || !out || !options_ok(o)) return SYN_ERR_INVALID;
    *out = nullptr;
    std::unique_ptr<syn::gguf::file> f;
    std::string err;
    int rc = syn::gguf::file::open(path, f, &err);
    if (rc) return set_err(rc, err);
    // read_llama_config (llama.hpp:206-319)
    std::string_view arch;
    if (!f->get_string("general.architecture", arch) || arch != "llama")
        return set_err(SYN_ERR_UNSUPPORTED, "general.architecture: only llama");
    auto count = [&](const char* k, uint64_t& v, bool required, uint64_t dflt) {
        if (f->get_uint(std::string("llama.") + k, v)) return true;
        if (f->find(std::string("llama.") + k)) return false;  // present, wrong type
        v = dflt;
        return !required;
    };
    uint64_t n_layer, n_embd, n_ff, n_head, ctx_train, n_kv, hd, vlen, rot, experts;
    if (!count("block_count", n_layer, true, 0) || !count("embedding_length", n_embd, true, 0) ||
        !count("feed_forward_length", n_ff, true, 0) || !count("attention.head_count", n_head, true, 0) ||
        !count("context_length", ctx_train, true, 0) || !n_layer || !n_embd || !n_ff || !n_head || !ctx_train)
        return set_err(SYN_ERR_FORMAT, "missing or zero llama.* count");
    if (!count("attention.head_count_kv", n_kv, false, n_head) || !n_kv || n_head % n_kv)
        return set_err(SYN_ERR_FORMAT, "llama.attention.head_count_kv");
    if (!count("attention.key_length", hd, false, n_embd / n_head) || !hd)
        return set_err(SYN_ERR_FORMAT, "llama.attention.key_length");
    if (!count("attention.value_length", vlen, false, hd) || vlen != hd)
        return set_err(SYN_ERR_UNSUPPORTED, "llama.attention.value_length");
    if (!count("rope.dimension_count", rot, false, hd) || rot != hd)
        return set_err(SYN_ERR_UNSUPPORTED, "llama.rope.dimension_count");
    if (!count("expert_count", experts, false, 0) || experts)
        return set_err(SYN_ERR_UNSUPPORTED, "llama.expert_count");
    double eps, base = 10000.0;
    if (!f->get_float("llama.attention.layer_norm_rms_epsilon", eps) || !(eps > 0))
        return set_err(SYN_ERR_FORMAT, "llama.attention.layer_norm_rms_epsilon");
    if (f->find("llama.rope.freq_base") && (!f->get_float("llama.rope.freq_base", base) || !(base > 0)))
        return set_err(SYN_ERR_FORMAT, "llama.rope.freq_base");
    std::string_view rs_type;
    double rs_factor = 0;
    if ((f->get_string("llama.rope.scaling.type", rs_type) && rs_type != "none" && rs_type != "linear") ||
        (f->get_float("llama.rope.scaling.factor", rs_factor) && rs_factor != 0 && rs_factor != 1) ||
        f->find("llama.rope.scale_linear") || f->find("llama.attention.scale"))
        return set_err(SYN_ERR_UNSUPPORTED, "rope scaling / attention.scale");
    const syn::gguf::tensor_info* te = f->tensor("token_embd.weight");
    if (!te || te->ne[0] != n_embd || te->ne[2] != 1 || te->ne[3] != 1)
        return set_err(SYN_ERR_FORMAT, "token_embd.weight");
    if (hd % 8 || hd > 256 || n_embd % 32 || n_ff % 32 || (n_head * hd) % 32)
        return set_err(SYN_ERR_UNSUPPORTED, "head_dim / widths not multiples of 8 / 32");

    std::unique_ptr<syn_session, void (*)(syn_session*)> s(new syn_session(), destroy);
    s->device = device;
    s->max_ctx = max_ctx;
    s->max_seqs = o.max_seqs;
    s->max_batch = o.max_batch;
    syn_llama_config& c = s->cfg;
    c.n_layer = int(n_layer); c.n_embd = int(n_embd); c.n_ff = int(n_ff); c.n_head = int(n_head);
    c.n_head_kv = int(n_kv); c.head_dim = int(hd); c.n_vocab = int(te->ne[1]);
    c.rms_eps = float(eps); c.rope_base = float(base); c.rope_mode = 0;
    c.type_embd = int(te->type);
    const syn::gguf::tensor_info* tout = f->tensor("output.weight");
    c.type_output = tout ? int(tout->type) : -1;
    if (!supported_type(c.type_embd)) return set_err(SYN_ERR_UNSUPPORTED, "token_embd.weight type");

    // bind every weight with its shape (models/common.hpp:146-160)
    const uint64_t qrows = n_head * hd, kvrows = n_kv * hd;
    struct want { const char* suffix; uint64_t rows, cols; };
    const want layer_wants[9] = {{"attn_norm.weight", 1, n_embd}, {"attn_q.weight", qrows, n_embd},
                                 {"attn_k.weight", kvrows, n_embd}, {"attn_v.weight", kvrows, n_embd},
                                 {"attn_output.weight", n_embd, qrows}, {"ffn_norm.weight", 1, n_embd},
                                 {"ffn_gate.weight", n_ff, n_embd}, {"ffn_up.weight", n_ff, n_embd},
                                 {"ffn_down.weight", n_embd, n_ff}};
    std::vector<std::vector<int>> types(n_layer, std::vector<int>(9));
    for (uint64_t l = 0; l < n_layer; ++l) {
        for (int i = 0; i < 9; ++i) {
            const std::string name = "blk." + std::to_string(l) + "." + layer_wants[i].suffix;
            const syn::gguf::tensor_info* t = f->tensor(name);
            if (!t) return set_err(SYN_ERR_FORMAT, "missing " + name);
            const bool norm = i == 0 || i == 5;
            if (!(norm ? t->n_elements() == n_embd : shape_is(*t, layer_wants[i].rows, layer_wants[i].cols)))
                return set_err(SYN_ERR_FORMAT, "bad shape " + name);
            if (!supported_matrix_type(int(t->type)) || (norm && t->type != SYN_F32))
                return set_err(SYN_ERR_UNSUPPORTED, "type of " + name);
            types[l][i] = int(t->type);
        }
        for (const char* extra : {"attn_q.bias", "attn_k.bias", "attn_v.bias", "attn_output.bias", "ffn_gate.bias",
                                  "ffn_up.bias", "ffn_down.bias", "ffn_gate_inp.weight"})
            if (f->tensor("blk." + std::to_string(l) + "." + extra))
                return set_err(SYN_ERR_UNSUPPORTED, std::string("blk.N.") + extra);
    }
    const syn::gguf::tensor_info* on = f->tensor("output_norm.weight");
    if (!on || on->n_elements() != n_embd || on->type != SYN_F32) return set_err(SYN_ERR_FORMAT, "output_norm.weight");
    if (tout && (!shape_is(*tout, uint64_t(c.n_vocab), n_embd) || !supported_matrix_type(int(tout->type))))
        return set_err(SYN_ERR_UNSUPPORTED, "output.weight");
    if (f->tensor("output.bias")) return set_err(SYN_ERR_UNSUPPORTED, "output.bias");
    const syn::gguf::tensor_info* rf = f->tensor("rope_freqs.weight");
    if (rf && (rf->type != SYN_F32 || rf->n_elements() != hd / 2)) return set_err(SYN_ERR_FORMAT, "rope_freqs.weight");

    if ((rc = set_part(*s, tp, device))) return rc;
    layout_builder lb;
    define(s->embd, c.type_embd, c.n_vocab, c.n_embd, lb);
    s->sources.push_back({"token_embd.weight", &s->embd, 0, 1, c.n_vocab});
    layer_layout(*s, types, lb);
    define(s->out_norm, SYN_F32, 1, c.n_embd, lb);
    s->sources.push_back({"output_norm.weight", &s->out_norm, 0, 1, 1});
    head_layout(*s, lb);
    if (rf) {
        s->has_ff = true;
        s->ff_off = lb.take(size_t(hd / 2) * 4);
    }
    if ((rc = finish(*s, lb))) return rc;

    rc = upload_sources(*s, *f);
    if (!rc && rf)
        rc = cuda(cudaMemcpy(s->arena + s->ff_off, f->data(*rf), size_t(hd / 2) * 4, cudaMemcpyHostToDevice));
    if (rc) return rc;
    if ((rc = warm_and_capture(*s))) return rc;
    *out = s.release();
    return SYN_OK;
}
}  // namespace

extern "C" int syn_session_open_synthetic(const syn_llama_config* cp, int max_ctx, uint64_t seed, int device,
                                          syn_session** out) {
    return syn_session_open_synthetic_tp(cp, max_ctx, seed, device, nullptr, out);
}

extern "C" int syn_session_open_synthetic_tp(const syn_llama_config* cp, int max_ctx, uint64_t seed, int device,
                                             syn_tp* tp, syn_session** out) {
    const syn_session_options o{max_ctx, 1, 1};
    return open_synthetic(cp, o, seed, device, tp, out);
}

extern "C" int syn_session_open_synthetic_ex(const syn_llama_config* cp, const syn_session_options* o, uint64_t seed,
                                             int device, syn_session** out) {
    if (!o) return SYN_ERR_INVALID;
    return open_synthetic(cp, *o, seed, device, nullptr, out);
}

namespace {
int open_synthetic(const syn_llama_config* cp, const syn_session_options& o, uint64_t seed, int device, syn_tp* tp,
                   syn_session** out) {
    const int max_ctx = o.max_ctx;
    if (!cp || !out || !options_ok(o)) return SYN_ERR_INVALID;
    *out = nullptr;
    const syn_llama_config& c0 = *cp;
    if (c0.n_layer <= 0 || c0.n_embd <= 0 || c0.n_ff <= 0 || c0.n_head <= 0 || c0.n_head_kv <= 0 ||
        c0.head_dim <= 0 || c0.n_vocab <= 0 || c0.n_head % c0.n_head_kv || !(c0.rms_eps > 0) || !(c0.rope_base > 0))
        return SYN_ERR_INVALID;
    if (c0.head_dim % 8 || c0.head_dim > 256 || c0.n_embd % 32 || c0.n_ff % 32 || (c0.n_head * c0.head_dim) % 32)
        return SYN_ERR_UNSUPPORTED;
    if (!supported_type(c0.type_embd) || !supported_type(c0.type_layers) ||
        (c0.type_output != -1 && !supported_type(c0.type_output)))
        return SYN_ERR_UNSUPPORTED;
    std::unique_ptr<syn_session, void (*)(syn_session*)> s(new syn_session(), destroy);
    s->device = device;
    s->max_ctx = max_ctx;
    s->max_seqs = o.max_seqs;
    s->max_batch = o.max_batch;
    s->cfg = c0;
    s->cfg.rope_mode = 0;
    const syn_llama_config& c = s->cfg;
    int rc = set_part(*s, tp, device);
    if (rc) return rc;
    layout_builder lb;
    define(s->embd, c.type_embd, c.n_vocab, c.n_embd, lb);
    s->sources.push_back({"token_embd.weight", &s->embd, 0, 1, c.n_vocab});
    const int T = c.type_layers;
    layer_layout(*s, std::vector<std::vector<int>>(c.n_layer, {SYN_F32, T, T, T, T, SYN_F32, T, T, T}), lb);
    define(s->out_norm, SYN_F32, 1, c.n_embd, lb);
    s->sources.push_back({"output_norm.weight", &s->out_norm, 0, 1, 1});
    head_layout(*s, lb);
    rc = finish(*s, lb);
    if (rc) return rc;
    // Every matrix N(0, 0.02) (seeded per tensor name), norms 1.0.
    uint64_t tensor_id = 0;
    for (const auto& src : s->sources) {
        const weight& w = *src.w;
        ++tensor_id;
        if (src.name.find("norm") != std::string::npos)
            rc = syn_fill_f32(s->at<float>(w.off), size_t(w.cols), 1.0f, s->stream);
        else
            rc = syn_fill_random(w.type, src.rows, w.cols, s->arena + w.off, w.rows, src.row0, seed, tensor_id, 0.02f,
                                 s->stream, src.step, src.first);
        if (rc) return rc;
    }
    if ((rc = cuda(cudaStreamSynchronize(s->stream)))) return rc;
    if ((rc = warm_and_capture(*s))) return rc;
    *out = s.release();
    return SYN_OK;
}
}  // namespace

extern "C" void syn_session_close(syn_session* s) { destroy(s); }

extern "C" int syn_tp_layout_of(const syn_llama_config* c, int rank, int world, syn_tp_layout* out) {
    if (!c || !out || c->n_head_kv <= 0 || c->n_head <= 0) return SYN_ERR_INVALID;
    return tp_layout(*c, rank, world, *out);
}

extern "C" int syn_session_tp_layout(const syn_session* s, syn_tp_layout* out) {
    if (!s || !out) return SYN_ERR_INVALID;
    *out = s->part;
    return SYN_OK;
}

extern "C" int syn_session_tp_status(syn_session* s, int* peer_stores, int* wait_errors) {
    if (!s) return SYN_ERR_INVALID;
    if (peer_stores) *peer_stores = s->p2p ? 1 : 0;
    if (wait_errors) {
        unsigned n = 0;
        if (s->p2p) {
            int rc = cuda(cudaSetDevice(s->device));
            if (!rc) rc = cuda(cudaMemcpy(&n, s->arena + s->tp_off + 68, 4, cudaMemcpyDeviceToHost));
            if (rc) return rc;
        }
        *wait_errors = int(n);
    }
    return SYN_OK;
}

extern "C" int syn_session_config(const syn_session* s, syn_llama_config* out) {
    if (!s || !out) return SYN_ERR_INVALID;
    *out = s->cfg;
    return SYN_OK;
}

extern "C" int syn_session_memory(const syn_session* s, size_t* arena, size_t* weights, size_t* kv) {
    if (!s) return SYN_ERR_INVALID;
    if (arena) *arena = s->arena_bytes;
    if (weights) *weights = s->weight_bytes;
    if (kv) *kv = s->kv_bytes;
    return SYN_OK;
}

extern "C" int syn_session_reset(syn_session* s) {
    if (!s) return SYN_ERR_INVALID;
    int rc = cuda(cudaSetDevice(s->device));
    if (!rc) rc = cuda(cudaMemsetAsync(s->arena + s->kv_off, 0, s->kv_bytes, s->stream));
    if (!rc) rc = cuda(cudaStreamSynchronize(s->stream));
    return rc;
}

extern "C" int syn_session_step(syn_session* s, uint32_t token, uint32_t pos, float* host_logits,
                                int32_t* host_argmax) {
    if (!s) return SYN_ERR_INVALID;
    if (token >= uint32_t(s->cfg.n_vocab) || pos >= uint32_t(s->max_ctx)) return SYN_ERR_RANGE;
    if (s->failed) return SYN_ERR_TIMEOUT;
    int rc = cuda(cudaSetDevice(s->device));
    if (rc) return rc;
    s->h_io[0] = int32_t(token);
    s->h_io[1] = int32_t(pos);
    rc = s->use_graph ? cuda(cudaGraphLaunch(s->step_exec, s->stream)) : enqueue_step(*s, s->stream);
    if (!rc) rc = cuda(cudaStreamSynchronize(s->stream));
    if (!rc) rc = check_status(*s);
    if (rc) return rc;
    if (host_logits) std::memcpy(host_logits, s->h_logits, size_t(s->cfg.n_vocab) * 4);
    if (host_argmax) *host_argmax = s->h_next[0];
    return SYN_OK;
}

extern "C" int syn_session_generate(syn_session* s, const uint32_t* prompt, int n_prompt, uint32_t pos, int n_steps,
                                    int32_t* host_tokens) {
    if (!s || !prompt || n_prompt <= 0 || n_steps <= 0 || n_prompt > n_steps) return SYN_ERR_INVALID;
    if (uint64_t(pos) + uint64_t(n_steps) > uint64_t(s->max_ctx)) return SYN_ERR_RANGE;
    if (s->failed) return SYN_ERR_TIMEOUT;
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] >= uint32_t(s->cfg.n_vocab)) return SYN_ERR_RANGE;
    int rc = cuda(cudaSetDevice(s->device));
    if (rc) return rc;
    std::vector<int32_t> forced(prompt, prompt + n_prompt);
    int32_t io[5] = {int32_t(prompt[0]), int32_t(pos), 0, 0, n_prompt};
    rc = cuda(cudaMemcpyAsync(s->at<int32_t>(s->forced_off), forced.data(), forced.size() * 4, cudaMemcpyHostToDevice,
                              s->stream));
    if (!rc) rc = cuda(cudaMemcpyAsync(s->io(), io, sizeof io, cudaMemcpyHostToDevice, s->stream));
    for (int i = 0; i < n_steps && !rc; ++i)
        rc = s->use_graph ? cuda(cudaGraphLaunch(s->gen_exec, s->stream)) : enqueue_gen(*s, s->stream);
    if (!rc && host_tokens) {
        rc = cuda(cudaMemcpyAsync(host_tokens, s->at<int32_t>(s->hist_off), size_t(n_steps) * 4,
                                  cudaMemcpyDeviceToHost, s->stream));
        if (!rc) rc = enqueue_status(*s, s->stream);
        if (!rc) rc = cuda(cudaStreamSynchronize(s->stream));
        if (!rc) rc = check_status(*s);
    } else if (!rc) {
        rc = cuda(cudaGetLastError());
    }
    return rc;
}

// ---- run(batch): prefill chunks and batched decode --------------------------------

namespace {

// Whether the batched path takes this session: one GPU, Q4_0 / Q8_0 layer
// matrices (the integer tensor-core GEMV for 3+ rows), any head type but K.
bool batch_supported(const syn_session& s) {
    if (s.part.world != 1 || !(s.max_batch > 1 || s.max_seqs > 1)) return false;
    for (const layer_w& L : s.layers)
        for (const weight* w : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down})
            if (w->type >= 0 && !w->quant()) return false;
    return s.head.quant() || s.head.type == SYN_F32 || s.head.type == SYN_F16;
}

// Y[n][rows] = rows [row0, row0 + rows) of w times the Q8_0 activations (+ residual).
int batch_matmul(syn_session& s, const weight& w, int row0, int rows, const void* act, int n, float* y,
                 const float* residual) {
    const char* base = s.arena + w.off + syn_weight_bytes(w.type, row0, w.cols, w.layout);
    return syn_gemv_q(w.type, base, w.layout, rows, w.cols, act, n, y, residual, s.stream);
}

// run(batch) (session.hpp:143-156, the ops of session.hpp:287-374 over n rows),
// launched op by op on the session's stream.
//   prefill: rows are the tokens of sequence seq at positions pos[0], pos[0] + 1,
//            ...; all their K/V rows are appended first (session.hpp:349-356),
//            then every row attends over the shared cache up to its position;
//            the logits are the last row's (op_last_row).
//   decode:  row i is the next token of sequence i at pos[i]; logits of every row.
// Every row's arithmetic is the one-token step's: the GEMV and attention give
// each row the bits a single-token call gives it (the reference's G1).
int run_batch(syn_session& s, int n, bool prefill, int seq) {
    const syn_llama_config& c = s.cfg;
    cudaStream_t st = s.stream;
    const int d = c.n_embd, hd = c.head_dim, ff = c.n_ff;
    const int qrows = c.n_head * hd, kvrows = c.n_head_kv * hd;
    float *x = s.at<float>(s.bo.x), *x2 = s.at<float>(s.bo.x2), *q = s.at<float>(s.bo.q), *k = s.at<float>(s.bo.k),
          *v = s.at<float>(s.bo.v), *attn = s.at<float>(s.bo.attn), *gu = s.at<float>(s.bo.gu),
          *g = s.at<float>(s.bo.g), *u = s.at<float>(s.bo.u), *logits = s.at<float>(s.bo.logits);
    void* act = s.arena + s.bo.act;
    int32_t *tok = s.at<int32_t>(s.bo.tok), *pos = s.at<int32_t>(s.bo.pos), *arg = s.at<int32_t>(s.bo.arg);
    int rc = syn_embed(s.embd.type, s.arena + s.embd.off, s.embd.layout, s.embd.rows, s.embd.cols, tok, n, x, st);
    for (int l = 0; l < c.n_layer && !rc; ++l) {
        const layer_w& L = s.layers[l];
        rc = syn_rms_norm(x, s.at<float>(L.attn_norm.off), n, d, c.rms_eps, nullptr, act, st);
        if (!rc && L.fused_qkv) {
            rc = batch_matmul(s, L.q, 0, qrows, act, n, q, nullptr);
            if (!rc) rc = batch_matmul(s, L.q, qrows, kvrows, act, n, k, nullptr);
            if (!rc) rc = batch_matmul(s, L.q, qrows + kvrows, kvrows, act, n, v, nullptr);
        } else if (!rc) {
            rc = batch_matmul(s, L.q, 0, qrows, act, n, q, nullptr);
            if (!rc) rc = batch_matmul(s, L.k, 0, kvrows, act, n, k, nullptr);
            if (!rc) rc = batch_matmul(s, L.v, 0, kvrows, act, n, v, nullptr);
        }
        if (rc) break;
        syn_attention_args a{};
        a.q = q;
        a.k = k;
        a.v = v;
        a.k_cache = s.kv(l, 0, prefill ? seq : 0);
        a.v_cache = s.kv(l, 1, prefill ? seq : 0);
        a.pos = pos;
        a.out = attn;
        a.scratch = s.arena + s.bo.scratch;
        a.cache_stride = prefill ? 0 : s.seq_halves();
        a.n_q = n;
        a.n_head = c.n_head;
        a.n_kv = c.n_head_kv;
        a.head_dim = hd;
        a.max_len = s.max_ctx;
        a.append = prefill ? 0 : 1;
        a.rope = 1;
        a.rope_mode = c.rope_mode;
        a.theta_scale = s.theta_scale;
        a.scale = s.scale;
        a.freq_factors = s.has_ff ? s.at<float>(s.ff_off) : nullptr;
        a.rope_table = s.at<float>(s.rope_tab_off);
        a.order = s.attn_order;
        if (prefill) rc = syn_rope_kv_append(&a, st);  // every row's K/V before any row attends
        if (!rc) rc = syn_attention(&a, st);
        if (!rc) rc = syn_quantize_q8_0(attn, n, qrows, act, st);
        if (!rc) rc = batch_matmul(s, L.o, 0, d, act, n, x2, x);
        if (!rc) rc = syn_rms_norm(x2, s.at<float>(L.ffn_norm.off), n, d, c.rms_eps, nullptr, act, st);
        if (rc) break;
        if (L.gu_pairs) {  // gate i at row 2i, up i at 2i + 1
            rc = batch_matmul(s, L.gate, 0, 2 * ff, act, n, gu, nullptr);
            if (!rc) rc = syn_silu_mul_pairs(gu, n, ff, nullptr, act, st);
        } else {
            if (L.fused_gu) {
                rc = batch_matmul(s, L.gate, 0, ff, act, n, g, nullptr);
                if (!rc) rc = batch_matmul(s, L.gate, ff, ff, act, n, u, nullptr);
            } else {
                rc = batch_matmul(s, L.gate, 0, ff, act, n, g, nullptr);
                if (!rc) rc = batch_matmul(s, L.up, 0, ff, act, n, u, nullptr);
            }
            if (!rc) rc = syn_silu_mul(g, u, n, ff, nullptr, act, st);
        }
        if (!rc) rc = batch_matmul(s, L.down, 0, d, act, n, x, x2);
    }
    if (rc) return rc;
    // the output rows: the last one (prefill) or all of them
    const int rows = prefill ? 1 : n;
    const float* xo = prefill ? x + size_t(n - 1) * d : x;
    const bool quant_head = s.head.quant();
    rc = syn_rms_norm(xo, s.at<float>(s.out_norm.off), rows, d, c.rms_eps, quant_head ? nullptr : x2,
                      quant_head ? act : nullptr, st);
    if (!rc)
        rc = quant_head ? syn_gemv_q(s.head.type, s.arena + s.head.off, s.head.layout, s.head.rows, s.head.cols, act,
                                     rows, logits, nullptr, st)
                        : syn_gemv_f(s.head.type, s.arena + s.head.off, s.head.rows, s.head.cols, x2, rows, logits,
                                     nullptr, st);
    if (!rc) rc = syn_argmax_ws(logits, rows, c.n_vocab, arg, s.arena + s.bo.am_ws, st);
    return rc;
}

// Inputs to the device, run(batch), outputs back, the step's health.
int batch_call(syn_session& s, int n, const int32_t* tokens, const int32_t* positions, bool prefill, int seq,
               float* host_logits, int32_t* host_argmax) {
    const int rows = prefill ? 1 : n;
    int rc = cuda(cudaSetDevice(s.device));
    if (!rc) rc = cuda(cudaMemcpyAsync(s.arena + s.bo.tok, tokens, size_t(n) * 4, cudaMemcpyHostToDevice, s.stream));
    if (!rc) rc = cuda(cudaMemcpyAsync(s.arena + s.bo.pos, positions, size_t(n) * 4, cudaMemcpyHostToDevice, s.stream));
    if (!rc) rc = run_batch(s, n, prefill, seq);
    if (!rc && host_logits)
        rc = cuda(cudaMemcpyAsync(s.h_logits, s.arena + s.bo.logits, size_t(rows) * s.cfg.n_vocab * 4,
                                  cudaMemcpyDeviceToHost, s.stream));
    if (!rc) rc = cuda(cudaMemcpyAsync(s.h_next, s.arena + s.bo.arg, size_t(rows) * 4, cudaMemcpyDeviceToHost, s.stream));
    if (!rc) rc = enqueue_status(s, s.stream);
    if (!rc) rc = cuda(cudaStreamSynchronize(s.stream));
    if (!rc) rc = check_status(s);
    if (rc) return rc;
    if (host_logits) std::memcpy(host_logits, s.h_logits, size_t(rows) * s.cfg.n_vocab * 4);
    if (host_argmax) std::memcpy(host_argmax, s.h_next, size_t(rows) * 4);
    return SYN_OK;
}

}  // namespace

extern "C" int syn_session_prefill(syn_session* s, int seq, const uint32_t* tokens, int n, uint32_t pos,
                                   float* host_logits, int32_t* host_argmax) {
    if (!s || !tokens || n <= 0) return SYN_ERR_INVALID;
    if (!batch_supported(*s)) return SYN_ERR_UNSUPPORTED;
    if (n > s->max_batch || seq < 0 || seq >= s->max_seqs) return SYN_ERR_RANGE;
    if (uint64_t(pos) + uint64_t(n) > uint64_t(s->max_ctx)) return SYN_ERR_RANGE;
    if (s->failed) return SYN_ERR_TIMEOUT;
    std::vector<int32_t> t(n), p(n);
    for (int i = 0; i < n; ++i) {
        if (tokens[i] >= uint32_t(s->cfg.n_vocab)) return SYN_ERR_RANGE;
        t[i] = int32_t(tokens[i]);
        p[i] = int32_t(pos) + i;
    }
    return batch_call(*s, n, t.data(), p.data(), true, seq, host_logits, host_argmax);
}

extern "C" int syn_session_step_batch(syn_session* s, int n, const uint32_t* tokens, const uint32_t* pos,
                                      float* host_logits, int32_t* host_argmax) {
    if (!s || !tokens || !pos || n <= 0) return SYN_ERR_INVALID;
    if (!batch_supported(*s)) return SYN_ERR_UNSUPPORTED;
    if (n > s->max_batch || n > s->max_seqs) return SYN_ERR_RANGE;
    if (s->failed) return SYN_ERR_TIMEOUT;
    std::vector<int32_t> t(n), p(n);
    for (int i = 0; i < n; ++i) {
        if (tokens[i] >= uint32_t(s->cfg.n_vocab) || pos[i] >= uint32_t(s->max_ctx)) return SYN_ERR_RANGE;
        t[i] = int32_t(tokens[i]);
        p[i] = int32_t(pos[i]);
    }
    return batch_call(*s, n, t.data(), p.data(), false, 0, host_logits, host_argmax);
}

extern "C" int syn_session_fill_kv_random(syn_session* s, int n_pos, uint64_t seed) {
    if (!s || n_pos <= 0 || n_pos > s->max_ctx) return SYN_ERR_INVALID;
    int rc = cuda(cudaSetDevice(s->device));
    const int row = s->part.n_kv * s->cfg.head_dim;
    uint64_t id = 0;
    for (int l = 0; l < s->cfg.n_layer && !rc; ++l)
        for (int which = 0; which < 2 && !rc; ++which)
            for (int q = 0; q < s->max_seqs && !rc; ++q)
                rc = syn_fill_random(SYN_F16, n_pos, row, s->kv(l, which, q), n_pos, 0, seed, ++id, 1.0f, s->stream);
    if (!rc) rc = cuda(cudaStreamSynchronize(s->stream));
    return rc;
}

extern "C" int syn_session_launches_per_step(const syn_session* s) {
    if (!s) return 0;
    int n = 1 + (s->p2p ? 1 : 0);  // advance (and the epoch under peer gathers)
    // attention: scores, exp and p.V kernels in the reference order, two kernels split; NCCL's own kernels aside
    const int attn = s->attn_order == SYN_ORDER_SPLIT ? 2 : 3;
    for (const op& o : s->ops) n += o.kind == opk::attention ? attn : o.kind == opk::allgather ? 0 : 1;
    return n;
}

namespace {

// Algorithmic bytes of one op at position pos: every weight byte (with its
// scales), activation byte in and out, and KV row it must touch once.
double op_bytes(const syn_session& s, const op& o, uint32_t pos) {
    const syn_llama_config& c = s.cfg;
    switch (o.kind) {
    case opk::embed: return double(c.n_embd) * 4 * 2;
    case opk::rms_norm: return double(o.cols) * 4 * 3 + (o.out2 >= 0 ? double(o.cols) * 1.125 : 0);
    case opk::quantize: return double(o.cols) * (4 + 1.125);
    case opk::quantize_k: return double(o.cols) * (4 + 1 + 4.0 / 256 + 2.0 / 16);
    case opk::matmul: {
        const weight& w = *o.w;
        const double nb = double(w.cols) / 32;
        double wb = w.quant() ? double(w.rows) * nb * (w.type == SYN_Q4_0 ? 18 : 34)
                    : w.kquant() ? double(syn_weight_bytes(w.type, w.rows, w.cols, SYN_LAYOUT_GGUF))
                                 : double(w.rows) * w.cols * (w.type == SYN_F32 ? 4 : 2);
        double in = w.quant() ? double(w.cols) + nb * 8
                    : w.kquant() ? double(w.cols) * (1 + 4.0 / 256 + 2.0 / 16) : double(w.cols) * 4;
        if (o.in_mode != SYN_IN_Q8) in = double(w.cols) * 4 * (o.in_mode == SYN_IN_RMSNORM ? 2 : 1);  // x (+ gamma)
        const double out = o.out_mode == SYN_OUT_SILU_PAIRS ? double(w.rows) / 2 : double(w.rows);
        return wb + in + out * 4 * (o.res >= 0 ? 2 : 1);
    }
    case opk::attention: {
        const double L = double(pos) + 1, row = double(c.n_head_kv) * c.head_dim;
        return 2 * L * row * 2 + double(c.n_head) * c.head_dim * 4 * 2 + 2 * row * 4;
    }
    case opk::silu_mul: return double(o.cols) * (8 + 1.125);
    case opk::argmax: return double(c.n_vocab) * 4;
    case opk::allgather: return double(o.cols) * 4 * s.part.world;  // the whole vector lands on every rank
    }
    return 0;
}

int op_kind_code(opk k) {
    switch (k) {
    case opk::embed: return SYN_OP_EMBED;
    case opk::rms_norm: return SYN_OP_RMS_NORM;
    case opk::quantize:
    case opk::quantize_k: return SYN_OP_QUANTIZE;
    case opk::matmul: return SYN_OP_MATMUL;
    case opk::attention: return SYN_OP_ATTENTION;
    case opk::silu_mul: return SYN_OP_SILU_MUL;
    case opk::argmax: return SYN_OP_ARGMAX;
    case opk::allgather: return SYN_OP_ALLGATHER;
    }
    return -1;
}

}  // namespace

// The step with an event recorded between every two ops, captured once as a
// graph and replayed, so each op's time is the device's alone (no host gaps,
// no programmatic overlap between ops).
extern "C" int syn_session_profile(syn_session* s, uint32_t token, uint32_t pos, syn_op_profile* out, int max_ops,
                                   int* n_ops) {
    if (!s || !n_ops) return SYN_ERR_INVALID;
    if (token >= uint32_t(s->cfg.n_vocab) || pos >= uint32_t(s->max_ctx)) return SYN_ERR_RANGE;
    int rc = cuda(cudaSetDevice(s->device));
    if (rc) return rc;
    const size_t n = s->ops.size();
    *n_ops = int(n);
    if (!out) return SYN_OK;
    if (s->prof_events.empty()) {
        s->prof_events.resize(n + 1);
        for (auto& e : s->prof_events)
            if ((rc = cuda(cudaEventCreate(&e)))) return rc;
        cudaGraph_t g = nullptr;
        if ((rc = cuda(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal)))) return rc;
        int body = SYN_OK;
        std::vector<op> all;
        all.swap(s->ops);
        // External event records: timestamps readable after the replay (an
        // event recorded inside a capture is otherwise internal to the graph).
        for (size_t i = 0; i < n && !body; ++i) {
            body = cuda(cudaEventRecordWithFlags(s->prof_events[i], s->stream, cudaEventRecordExternal));
            s->ops.assign(1, all[i]);
            if (!body) body = enqueue_ops(*s, s->stream);
        }
        s->ops.swap(all);
        if (!body) body = cuda(cudaEventRecordWithFlags(s->prof_events[n], s->stream, cudaEventRecordExternal));
        rc = cuda(cudaStreamEndCapture(s->stream, &g));
        if (body || rc) {
            if (g) cudaGraphDestroy(g);
            return body ? body : rc;
        }
        rc = cuda(cudaGraphInstantiate(&s->prof_exec, g, 0));
        cudaGraphDestroy(g);
        if (rc) return rc;
    }
    int32_t io[2] = {int32_t(token), int32_t(pos)};
    rc = cuda(cudaMemcpyAsync(s->io(), io, sizeof io, cudaMemcpyHostToDevice, s->stream));
    if (!rc) rc = cuda(cudaGraphLaunch(s->prof_exec, s->stream));
    if (!rc) rc = cuda(cudaStreamSynchronize(s->stream));
    for (size_t i = 0; i < n && !rc && int(i) < max_ops; ++i) {
        const op& o = s->ops[i];
        syn_op_profile& p = out[i];
        p.kind = op_kind_code(o.kind);
        p.layer = o.kind == opk::attention ? o.layer : -1;
        p.type = o.w ? o.w->type : -1;
        p.rows = o.w ? o.w->rows : 0;
        p.cols = o.w ? o.w->cols : o.cols;
        rc = cuda(cudaEventElapsedTime(&p.ms, s->prof_events[i], s->prof_events[i + 1]));
        p.bytes = op_bytes(*s, o, pos);
    }
    return rc;
}

extern "C" int syn_copy_to_host(void* host_dst, const void* device_src, size_t bytes) {
    if (!host_dst || !device_src) return SYN_ERR_INVALID;
    return cuda(cudaMemcpy(host_dst, device_src, bytes, cudaMemcpyDeviceToHost));
}

extern "C" float* syn_session_logits(syn_session* s) { return s ? s->logits() : nullptr; }

extern "C" void* syn_session_stream(syn_session* s) { return s ? s->stream : nullptr; }

extern "C" uint16_t* syn_session_kv(syn_session* s, int layer, int which) {
    if (!s || layer < 0 || layer >= s->cfg.n_layer || (which != 0 && which != 1)) return nullptr;
    return s->kv(layer, which);
}

extern "C" int syn_session_weight(syn_session* s, const char* name, void* host_out, size_t bytes, int* type,
                                  int* rows, int* cols) {
    if (!s || !name) return SYN_ERR_INVALID;
    for (const auto& src : s->sources) {
        if (src.name != name) continue;
        const weight& w = *src.w;
        const int r = src.rows;
        if (type) *type = w.type;
        if (rows) *rows = r;
        if (cols) *cols = w.cols;
        const size_t need = syn_weight_bytes(w.type, r, w.cols, SYN_LAYOUT_GGUF);
        if (!host_out) return SYN_OK;
        if (bytes < need) return SYN_ERR_INVALID;
        int rc = cuda(cudaSetDevice(s->device));
        if (rc) return rc;
        if (w.kquant()) {  // planar rows -> GGUF blocks (Q6_K: each block's 208 quant bytes, then its scale)
            const int nb = w.cols / 256, bb = w.type == SYN_Q4_K ? 144 : 210;
            const size_t pitch = syn_weight_bytes(w.type, 1, w.cols, SYN_LAYOUT_PLANAR);
            std::vector<uint8_t> rowbuf(pitch);
            uint8_t* o = static_cast<uint8_t*>(host_out);
            for (int rr = 0; rr < r; ++rr) {
                const size_t dr = size_t(src.row0) + size_t(rr) * src.step;
                rc = cuda(cudaMemcpy(rowbuf.data(), s->arena + w.off + dr * pitch, pitch, cudaMemcpyDeviceToHost));
                if (rc) return rc;
                uint8_t* orow = o + size_t(rr) * nb * bb;
                if (w.type == SYN_Q4_K) {
                    std::memcpy(orow, rowbuf.data(), size_t(nb) * bb);
                    continue;
                }
                for (int b = 0; b < nb; ++b) {
                    std::memcpy(orow + size_t(b) * bb, rowbuf.data() + size_t(b) * 208, 208);
                    std::memcpy(orow + size_t(b) * bb + 208, rowbuf.data() + size_t(nb) * 208 + size_t(b) * 2, 2);
                }
            }
            return SYN_OK;
        }
        if (!w.quant()) {
            const size_t es = w.type == SYN_F32 ? 4 : 2;
            return cuda(cudaMemcpy(host_out, s->arena + w.off + size_t(src.row0) * w.cols * es, need,
                                   cudaMemcpyDeviceToHost));
        }
        // planar rows (quants, then binary16 scales, padded) -> GGUF blocks on the host
        const int nb = w.cols / 32, qb = w.type == SYN_Q4_0 ? 16 : 32, bb = qb + 2;
        const size_t row_b = size_t(nb) * qb + ((size_t(nb) * 2 + 15) & ~size_t(15));
        std::vector<uint8_t> rowbuf(row_b);
        uint8_t* o = static_cast<uint8_t*>(host_out);
        for (int rr = 0; rr < r; ++rr) {
            const size_t dr = size_t(src.row0) + size_t(rr) * src.step;
            rc = cuda(cudaMemcpy(rowbuf.data(), s->arena + w.off + dr * row_b, row_b, cudaMemcpyDeviceToHost));
            if (rc) return rc;
            for (int b = 0; b < nb; ++b) {
                uint8_t* blk = o + (size_t(rr) * nb + b) * bb;
                const size_t pos = size_t(syn_planar_block_pos(nb, dr, b));
                std::memcpy(blk, rowbuf.data() + size_t(nb) * qb + size_t(b) * 2, 2);
                std::memcpy(blk + 2, rowbuf.data() + pos * qb, qb);
            }
        }
        return SYN_OK;
    }
    return set_err(SYN_ERR_INVALID, std::string("no tensor ") + name);
}
