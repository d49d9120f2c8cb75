// Entry points shared inside the library (not part of the public C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "synapse_b200.h"

// GGUF blocks of `rows` rows (device) -> rows [row0, row0 + rows) of a planar
// matrix of `total_rows` rows at dst.
// Source row i lands on destination row row0 + i * row_step.
int syn_repack_rows(int type, const void* src, int rows, int cols, void* dst, int total_rows, int row0,
                    cudaStream_t s, int row_step = 1);

// Random N(0, sigma) values, seeded by (seed, tensor, element), quantized with
// ggml's reference quantizer (Q4_0 / Q8_0) into rows [row0, row0 + rows) of a
// planar matrix of total_rows, or written as F32 / F16 rows [row0, row0 + rows).
// Values are those of rows first_row .. of the tensor (seed, tensor), so a
// slice of a matrix holds the same weights as the whole matrix's rows.
int syn_fill_random(int type, int rows, int cols, void* dst, int total_rows, int row0, uint64_t seed,
                    uint64_t tensor, float sigma, cudaStream_t s, int row_step = 1, long first_row = 0);
// dst[i] = v for n floats.
int syn_fill_f32(float* dst, size_t n, float v, cudaStream_t s);

// Device-side greedy step bookkeeping (io layout in session.cpp): records the
// argmax, advances the position and picks the next input token.
int syn_advance(int32_t* io, const int32_t* forced, int32_t* history, cudaStream_t s);

// silu(gate) * up of n_tok tokens whose gate and up values are interleaved
// (gate i at 2i, up i at 2i + 1 of each token's 2 cols values), optionally
// quantized to Q8_0 activations (as syn_silu_mul).
int syn_silu_mul_pairs(const float* gu, int n_tok, int cols, float* out_f32, void* act, cudaStream_t stream);

// Argmax with a caller-owned persistent workspace of syn_argmax_ws_bytes
// (zeroed once; each launch leaves its counters zero again).
size_t syn_argmax_ws_bytes(int n_tok);
int syn_argmax_ws(const float* x, int n_tok, int n, int32_t* out, void* ws, cudaStream_t s);

// Physical position of logical block b in row r of a planar matrix of nb
// blocks per row (the loader's chunk rotation).
int syn_planar_block_pos(int nb, size_t r, int b);

// Q4_K / Q6_K (gemv_k.cu): bytes of a matrix in a layout (0 if not a K type
// or cols is not a multiple of 256), the GGUF -> planar repack of `rows`
// rows into dst, and the matrix-vector product on Q8_K activations.
bool syn_k_type(int type);
size_t syn_k_weight_bytes(int type, int rows, int cols, int layout);
int syn_k_repack_rows(int type, const void* src, int rows, int cols, void* dst, cudaStream_t s);
int syn_gemv_k(int type, const void* w, int layout, int rows, int cols, const void* act, int n_tok, float* y,
               const float* residual, cudaStream_t s);

// Programmatic dependent launch for this thread's launches.
void syn_set_pdl(int on);
// The same, exported for microbenchmarks that time kernels captured the way
// the session captures them.
extern "C" void syn_set_programmatic_launch(int on);

// Sets the thread's last error message.
void syn_set_error(const char* msg);

// Rank, world size and device of a tensor-parallel group (tp.cpp).
struct syn_tp;
void syn_tp_info(const syn_tp* tp, int* rank, int* world, int* device);
// Host helpers over the group's communicator (collective, synchronous):
// every rank's `bytes` of host data gathered in rank order, and a barrier.
int syn_tp_exchange(syn_tp* tp, const void* mine, void* all, size_t bytes);
int syn_tp_barrier(syn_tp* tp);

// ---- tensor-parallel gathers by peer stores ------------------------------------
// Every rank maps every other rank's arena (CUDA IPC); all arenas have the
// same layout. A gathered vector lives in every arena as 8-byte words, each
// {float bits, epoch}: a producer kernel stores each element of its slice,
// with the step's epoch, into every rank's copy by one 64-bit store; a
// consumer reads a word once its epoch is this step's (each word is written
// whole, so the value is the producer's). No flag and no fence is needed.
constexpr int kTpMaxWorld = 8;
struct TpSync {
    char* const* peers = nullptr;     // device array [world]: every rank's arena base; nullptr = no peer gathers
    size_t out_off = 0;               // producer: arena byte offset of the word of this launch's output element 0
    const unsigned* epoch = nullptr;  // this rank's step counter
    unsigned* err = nullptr;          // reads that gave up waiting (sticky count)
    int world = 1, rank = 0;
    int out_ll = 0;                   // the output goes to every rank as words
    int in_ll = 0;                    // the input vector is words (wait for this step's)
    int res_ll = 0;                   // the residual is words (this rank's slice: complete)
    unsigned long long wait_ns = 2000000000ull;  // a word read gives up after this long and counts an error
};
// syn_gemv / syn_attention / the session's argmax with a gather hook (the
// staged GEMV path only: SYN_ERR_UNSUPPORTED when the shape does not take it).
int syn_gemv_tp(const syn_gemv_args* a, const TpSync& t, cudaStream_t s);
int syn_attention_tp(const syn_attention_args* a, const TpSync& t, cudaStream_t s);
// The argmax of n gathered logits (words), which it also writes as floats to plain.
int syn_argmax_ws_tp(const void* words, int n, int32_t* out, float* plain, void* ws, const TpSync& t, cudaStream_t s);
// The step's first launch under peer gathers: epoch += 1.
int syn_tp_step_begin(unsigned* epoch, cudaStream_t s);

// Bounded waits of the attention kernels that gave up on the current device (-1: unreadable).
int syn_attn_timeouts();
// Device addresses (current device) of the counters of bounded copy waits that
// gave up in the GEMV and attention kernels, for a session to copy out after
// every step; NULL if they cannot be looked up.
unsigned* syn_gemv_timeout_word();
unsigned* syn_attn_timeout_word();

// Self-check of the bounded wait of a tensor-parallel word read: a kernel
// reads 32 gathered words that never carry the awaited step's epoch, with a
// limit of wait_us; *errors receives how many reads gave up (at least one when
// the wait ends as it must). The call allocates its own small buffers.
extern "C" int syn_check_tp_wait(unsigned wait_us, int* errors);

// Self-check of the library's expf (exp_rn): y = exp_rn(x) and, for
// comparison, y_ref = exp(double(x)) rounded to float, for n device floats.
extern "C" int syn_check_exp(const float* x, float* y, float* y_ref, int n, void* stream);

