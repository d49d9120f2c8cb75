/*
 * synapse_b200.h -- C ABI of the B200 (sm_100a) decode path.
 *
 * This is the drop-in boundary for branes-ai/synapse's Llama decode hot path:
 * the quantized matrix-vector products behind op_matmul, RoPE + KV append +
 * GQA decode attention behind op_rope / op_attention, the element-wise ops
 * around them, the device arena the GGUF loader and static planner fill, and
 * tensor parallelism over the GPUs of one NVLink box. Every comment cites the
 * reference interface (path:line inside branes-ai/synapse v0.15.12,
 * sdk/include/branes/synapse/) that the entry point replaces.
 *
 * Conventions (as the reference's kernels: no allocation, no throw):
 *   - every kernel entry point is asynchronous on the caller's stream
 *     (a cudaStream_t passed as void*; NULL = legacy default stream);
 *   - pointers are device pointers unless the name says host_;
 *   - scratch memory, where needed, is the caller's (a planned arena region);
 *   - the return value is a syn_status: 0 on success, never an abort.
 *
 * Tensor types are GGUF ggml_type tags (gguf/tensor_type.hpp:25-46).
 */
#ifndef SYNAPSE_B200_H
#define SYNAPSE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    SYN_OK = 0,
    SYN_ERR_INVALID = 1,      /* bad argument (a precondition the reference asserts) */
    SYN_ERR_UNSUPPORTED = 2,  /* a type / shape this build does not implement */
    SYN_ERR_CUDA = 3,         /* a CUDA runtime error (launch, copy, memory) */
    SYN_ERR_NO_MEMORY = 4,    /* device memory exhausted */
    SYN_ERR_TIMEOUT = 5,      /* a bounded wait gave up (multi-GPU flags) */
    SYN_ERR_NCCL = 6,         /* a collective failed */
    SYN_ERR_FORMAT = 7,       /* malformed GGUF / model metadata */
    SYN_ERR_RANGE = 8         /* token or position out of range: session::run returns false */
} syn_status;

/* GGUF tensor types (ggml_type values, gguf/tensor_type.hpp:25-46). */
enum { SYN_F32 = 0, SYN_F16 = 1, SYN_Q4_0 = 2, SYN_Q8_0 = 8, SYN_Q4_K = 12, SYN_Q6_K = 14 };

/* Weight layouts in device memory.
 *   SYN_LAYOUT_GGUF   : the GGUF bytes unchanged (rows of 18 B / 34 B blocks).
 *   SYN_LAYOUT_PLANAR : repacked for 16-byte coalesced loads, row after row:
 *                       a row's quants (blocks x 16 B for Q4_0, x 32 B for
 *                       Q8_0), then its binary16 scales, padded to 16 bytes.
 *                       A range of rows is one contiguous byte range.
 *                       Q4_K: the GGUF rows unchanged (144 B blocks).
 *                       Q6_K: a row's blocks as 208 B each (the GGUF block
 *                       without its binary16 scale), then its scales,
 *                       padded to 16 bytes.
 * Plain F32/F16 weights have one layout (row-major). Q6_K weights must be
 * planar for syn_gemv_q (GGUF Q6_K blocks are 210 B, not 16-byte aligned). */
enum { SYN_LAYOUT_GGUF = 0, SYN_LAYOUT_PLANAR = 1 };

/* Build-time identity: "sm_100a" and the library version. */
const char* syn_build_info(void);
/* Human-readable name of a status. */
const char* syn_status_string(int status);
/* The last CUDA error string seen by this thread (for SYN_ERR_CUDA). */
const char* syn_last_error(void);
/* How many bounded device-side waits on the current device gave up (a copy
 * that never arrived); 0 in a healthy run, -1 if it cannot be read. */
int syn_device_errors(void);

/* ------------------------------------------------------------------------
 * Q8_0 activations (quant/q8.hpp:54-69 quantize_row_q8_0; kernels/gemv.hpp:
 * 72-116 prepare_activations). The device form of n_tok rows of `cols` is
 * planar: int8 quants [n_tok][cols], then binary16 scales [n_tok][cols/32],
 * then the decoded float scales [n_tok][cols/32], then the int32 block sums
 * [n_tok][cols/32] (each plane 256-byte aligned). Quants and binary16 scales
 * are bit-identical to the reference's block_q8_0 (quant/blocks.hpp:49-53).
 * ---------------------------------------------------------------------- */
size_t syn_q8_act_bytes(int n_tok, int cols);
/* x: f32 [n_tok][cols] -> act. Replaces gemm_prepare_rows (gemm.hpp:111). */
int syn_quantize_q8_0(const float* x, int n_tok, int cols, void* act, void* stream);
/* act -> ggml block_q8_0 bytes [n_tok][cols/32][34] (checking / interchange). */
int syn_q8_act_to_blocks(const void* act, int n_tok, int cols, void* blocks, void* stream);

/* Q8_K activations for the K formats (quant/q8.hpp:73-104 quantize_row_q8_k):
 * planar int8 quants [n_tok][cols], float scales [n_tok][cols/256], int16
 * sums of 16 quants [n_tok][cols/16], each plane 256-byte aligned; cols a
 * multiple of 256. Bit-identical to the reference's block_q8_k
 * (quant/q8.hpp:33-38), which syn_q8k_act_to_blocks writes
 * ([n_tok][cols/256][292]). */
size_t syn_q8k_act_bytes(int n_tok, int cols);
int syn_quantize_q8_k(const float* x, int n_tok, int cols, void* act, void* stream);
int syn_q8k_act_to_blocks(const void* act, int n_tok, int cols, void* blocks, void* stream);

/* ------------------------------------------------------------------------
 * Weights: device bytes of a rows x cols matrix in a layout, and the
 * GGUF -> planar repack the loader runs once per tensor (gguf/tensor_view.hpp:
 * 33-40 view_as, where the reference views the mapped file in place).
 * ---------------------------------------------------------------------- */
size_t syn_weight_bytes(int type, int rows, int cols, int layout);
/* src (device, GGUF layout) -> dst (device, planar). src and dst must not overlap. */
int syn_repack_planar(int type, const void* src, int rows, int cols, void* dst, void* stream);
/* host GGUF bytes -> dst (device, `layout`), staged through the caller's device
 * buffer `staging` of `staging_bytes` (>= 1 MiB; unused for GGUF layout and
 * plain types). Synchronous with respect to the host buffer. */
int syn_upload_weight(int type, const void* host_src, int rows, int cols, void* dst, int layout, void* staging,
                      size_t staging_bytes, void* stream);

/* Seeded N(0, 0.02) weights quantized on the device (ggml's reference
 * quantizer) straight into a planar matrix: synthetic inputs for benchmarks
 * (the reference only reads weights from files; no counterpart). */
int syn_fill_random_planar(int type, int rows, int cols, void* dst, uint64_t seed, void* stream);

/* ------------------------------------------------------------------------
 * mul_mat: Y[t][r] = W[r,:] . X[t,:] for t < n_tok (kernels/gemm.hpp:143-230
 * gemm_rows, the n_tok = 1 case being kernels/gemv.hpp:149-161 gemv).
 *   Q4_0 / Q8_0 weights take Q8_0 activations (syn_quantize_q8_0); each block
 *   is an exact integer dot scaled by d_w * d_a (kernels/dot.hpp:103-164,
 *   :268-322); rows may be in either layout.
 *   Q4_K / Q6_K weights take Q8_K activations (syn_quantize_q8_k); each
 *   256-weight block is an exact integer dot with its sub-block scales folded
 *   in, less the Q4_K min term (kernels/dot.hpp:166-239, :359-399); Q6_K
 *   rows must be planar.
 *   F32 / F16 weights take float activations (kernels/dot.hpp:404-433).
 * residual (may be NULL): Y[t][r] += residual[t][r] after the dot, the
 *   reference's following op_add (elementwise.hpp:29); it may alias y.
 * ---------------------------------------------------------------------- */
int syn_gemv_q(int type, const void* w, int layout, int rows, int cols, const void* act, int n_tok, float* y,
               const float* residual, void* stream);
int syn_gemv_f(int type, const void* w, int rows, int cols, const float* x, int n_tok, float* y,
               const float* residual, void* stream);

/* mul_mat with its neighbours fused in (what the session runs): the input
 * quantized inside the kernel from floats (SYN_IN_F32: gemm_prepare_rows), or
 * from the rms_norm of the floats (SYN_IN_RMSNORM: op_rms_norm then
 * op_matmul, elementwise.hpp:208-232), and optionally rows taken in (gate, up)
 * pairs to give silu(gate) * up (SYN_OUT_SILU_PAIRS: op_silu then op_mul, the
 * output holding rows/2 values per token). Every value equals the separate
 * ops' bit for bit. The fused modes need planar weights, 1-2 tokens and a
 * shape the pipelined kernel takes (syn_gemv_fusable); SYN_IN_Q8 with
 * SYN_OUT_ROWS is syn_gemv_q. */
enum { SYN_IN_Q8 = 0, SYN_IN_F32 = 1, SYN_IN_RMSNORM = 2 };
enum { SYN_OUT_ROWS = 0, SYN_OUT_SILU_PAIRS = 1 };
typedef struct {
    int type, layout, rows, cols, n_tok;
    const void* w;
    int in_mode;
    const void* act;       /* SYN_IN_Q8 */
    const float* x;        /* SYN_IN_F32 / SYN_IN_RMSNORM, [n_tok][cols], 16-byte aligned */
    const float* gamma;    /* SYN_IN_RMSNORM: cols floats, 16-byte aligned */
    float eps;
    int out_mode;
    float* y;              /* [n_tok][rows] (SYN_OUT_ROWS) or [n_tok][rows/2] */
    const float* residual; /* SYN_OUT_ROWS only; may alias y */
} syn_gemv_args;
int syn_gemv(const syn_gemv_args* a, void* stream);
int syn_gemv_fusable(int type, int layout, int rows, int cols, int n_tok, int out_mode);

/* ------------------------------------------------------------------------
 * RoPE + KV append + GQA decode attention (kernels/attention.hpp:89-129 rope,
 * :165-175 kv_append, :185-244 attend_group, :254-269 attention), fused:
 * for each query b < n_q, with its position p = pos[b] (device int32):
 *   q_b and (if append) k_b are rotated at p; k_b, v_b are stored as F16 in
 *   row p of the cache; out_b = softmax(scale * q_b K^T) V over rows 0..p,
 *   query head h reading KV head h / (n_head / n_kv).
 * Caches: K and V of query b start at (k|v)_cache + b * cache_stride halves,
 *   rows of n_kv * head_dim halves (attention.hpp:133-143). cache_stride =
 *   max_ctx * n_kv * head_dim for independent sequences (batched decode), or 0
 *   for tokens of one sequence (then append must be 0: use syn_rope_kv_append
 *   first, as session.hpp:349-356 appends every token before attending).
 * max_len bounds pos[b] + 1 for every b (it sizes the grid and the score
 * scratch).
 * rope_mode: 0 normal (Llama), 1 neox. freq_factors: NULL or head_dim/2 floats
 * (device). yarn: NULL or 5 floats {freq_scale, ext_factor, attn_factor,
 * corr_low, corr_high} (host), attention.hpp:60-66.
 * order: SYN_ORDER_REFERENCE (0, the default) adds every float sum in the
 *   reference's order at any context length: the score dots in dimension
 *   order, the normaliser in double, and out = sum_t p_t V_t in position
 *   order, one fma per position and output element (attention.hpp:214-243);
 *   bit-identical to the reference's attend_group on the same binary16
 *   inputs. SYN_ORDER_SPLIT (1) splits the context over 256-position chunks
 *   whose partial p.V sums run on tensor cores and are added in chunk order:
 *   the same up to 256 positions, about 1e-6 relative beyond.
 * ---------------------------------------------------------------------- */
enum { SYN_ORDER_REFERENCE = 0, SYN_ORDER_SPLIT = 1 };
typedef struct {
    const float* q;        /* [n_q][n_head * head_dim], before RoPE */
    const float* k;        /* [n_q][n_kv * head_dim], before RoPE (append only) */
    const float* v;        /* [n_q][n_kv * head_dim] (append only) */
    uint16_t* k_cache;     /* binary16 bits */
    uint16_t* v_cache;
    const int32_t* pos;    /* [n_q] device */
    float* out;            /* [n_q][n_head * head_dim] */
    void* scratch;         /* syn_attention_scratch_bytes */
    size_t cache_stride;   /* halves between the caches of consecutive queries */
    int n_q, n_head, n_kv, head_dim, max_len;
    int append;            /* 1: rotate k and append (k, v) inside the kernel */
    int rope;              /* 1: rotate q (and k) at pos; 0: q, k already rotated */
    int rope_mode;
    float theta_scale;     /* rope_theta_scale(base, head_dim), attention.hpp:47 */
    float scale;           /* 1 / sqrt(head_dim), models/llama.hpp:407 */
    const float* freq_factors;
    const float* yarn;
    const float* rope_table; /* NULL, or syn_rope_table for these rope settings and max_len rows */
    int order;             /* SYN_ORDER_REFERENCE / SYN_ORDER_SPLIT */
} syn_attention_args;

size_t syn_attention_scratch_bytes(int n_q, int n_head, int n_kv, int head_dim, int max_len);
int syn_attention(const syn_attention_args* a, void* stream);
/* syn_attention for callers that cannot allocate device memory. It has no
 * counterpart in the reference; it exists for callers such as a host that
 * owns the whole device memory budget and passes a plugin only its tensors,
 * or a decode loop that must not allocate once running. a->scratch is
 * ignored: the scratch is a 16 MiB array in the library's own static device
 * memory, present on every GPU that loads the library until the process
 * exits. Shapes whose syn_attention_scratch_bytes exceed 16 MiB are rejected
 * with SYN_ERR_INVALID. The first call on a device looks up the array's device
 * address with that device current; make that first call before any stream
 * capture. No call allocates. Every call on a device uses the same array, so
 * calls whose GPU work overlaps (different streams, or different host
 * threads) race and must be serialised by the caller; the array keeps the
 * last call's contents, none of which a later call depends on. The device
 * address is cached per device for the life of the process: do not call it
 * again on a device after cudaDeviceReset there. */
int syn_attention_noalloc(const syn_attention_args* a, void* stream);
/* The (cos, sin) of every RoPE pair at every position p < max_len, as
 * table[p][i] = {cos, sin} of pair i (max_len * head_dim floats), with the
 * arithmetic of attention.hpp:102-119. An attention call given the table reads
 * it instead of evaluating the trigonometry for its position (a session builds
 * it once). Device table; freq_factors device, yarn host (as syn_attention). */
int syn_rope_table(float* table, int max_len, int head_dim, float theta_scale, const float* freq_factors,
                   const float* yarn, void* stream);
/* RoPE + F16 append only, for n_q tokens sharing one cache (prefill). */
int syn_rope_kv_append(const syn_attention_args* a, void* stream);
/* RoPE alone (attention.hpp:89): out[i] = rope(x[i], pos[i]) for n rows of
 * n_heads * head_dim floats. */
int syn_rope(const float* x, float* out, int n, int n_heads, int head_dim, const int32_t* pos, float theta_scale,
             const float* freq_factors, int rope_mode, const float* yarn, void* stream);

/* ------------------------------------------------------------------------
 * Element-wise ops (kernels/elementwise.hpp), each on n_tok rows.
 * ---------------------------------------------------------------------- */
/* out = x / rms(x) * gamma (elementwise.hpp:208-232), then optionally quantized
 * to Q8_0 activations; out_f32 and act may each be NULL. */
int syn_rms_norm(const float* x, const float* gamma, int n_tok, int cols, float eps, float* out_f32, void* act,
                 void* stream);
/* out = silu(g) * u (elementwise.hpp:76, :50), optionally quantized. */
int syn_silu_mul(const float* g, const float* u, int n_tok, int cols, float* out_f32, void* act, void* stream);
/* out = a + b (elementwise.hpp:29); out may alias a or b. */
int syn_add(const float* a, const float* b, float* out, size_t n, void* stream);
/* out[t] = row tokens[t] of the table (session.hpp:331-336 op_embed). */
int syn_embed(int type, const void* table, int layout, int rows, int cols, const int32_t* tokens, int n_tok,
              float* out, void* stream);
/* out[t] = first index of the largest of x[t][0..n) (llama_decode.cpp:274,
 * std::max_element: ties go to the lowest index). n_tok <= 64. Its partial
 * results live in a small static device array shared by every call on a
 * device, so calls that overlap on the GPU must be serialised by the caller
 * (a session uses its own workspace instead). The workspace's device address
 * is cached per device for the life of the process: do not call it again on
 * a device after cudaDeviceReset there. */
int syn_argmax(const float* x, int n_tok, int n, int32_t* out, void* stream);

/* ------------------------------------------------------------------------
 * Llama decode session (models/llama.hpp:324-489 load_llama + graph/
 * session.hpp:82-171): weights, activations and the F16 KV cache in one device
 * arena placed by the static planner (graph/planner.hpp:90-128); run() is a
 * captured CUDA graph per token.
 * ---------------------------------------------------------------------- */
typedef struct syn_session syn_session;

typedef struct {
    int n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab;
    float rms_eps, rope_base;
    int rope_mode;         /* 0 normal (llama) */
    int type_embd;         /* token_embd type */
    int type_layers;       /* attention + FFN matrices */
    int type_output;       /* output head; -1 = tied to token_embd */
} syn_llama_config;

/* What a session holds besides the model (graph/session.hpp:90-101 plans the
 * arena for max_batch rows and states for max_ctx positions):
 *   max_ctx   positions of each sequence's KV cache;
 *   max_seqs  sequences with their own KV cache (syn_session_step_batch decodes
 *             one token of each of the first n; the single-token calls use
 *             sequence 0);
 *   max_batch tokens one batched call may carry (a prefill chunk, or the
 *             sequences of a batched decode step). */
typedef struct {
    int max_ctx, max_seqs, max_batch;
} syn_session_options;

/* Open a GGUF Llama file (models/llama.hpp:206-319 read_llama_config rules). */
int syn_session_open_gguf(const char* path, int max_ctx, int device, syn_session** out);
/* A model of random N(0, 0.02) weights quantized on the device (seeded),
 * norm weights 1; for benchmarks at shapes no file exists for. */
int syn_session_open_synthetic(const syn_llama_config* c, int max_ctx, uint64_t seed, int device,
                               syn_session** out);
/* The same with options (one GPU). */
int syn_session_open_gguf_ex(const char* path, const syn_session_options* o, int device, syn_session** out);
int syn_session_open_synthetic_ex(const syn_llama_config* c, const syn_session_options* o, uint64_t seed, int device,
                                  syn_session** out);
void syn_session_close(syn_session* s);
int syn_session_config(const syn_session* s, syn_llama_config* out);
/* Bytes of the device arena, of the weights and of the KV cache. */
int syn_session_memory(const syn_session* s, size_t* arena, size_t* weights, size_t* kv);
/* Zero the KV cache (session.hpp:127 reset). */
int syn_session_reset(syn_session* s);
/* One token at pos (session.hpp:133 run(step)): host_logits (n_vocab floats)
 * and host_argmax may be NULL. Returns SYN_ERR_RANGE (running nothing) when
 * token >= n_vocab or pos >= max_ctx. Blocks until the outputs are on the host.
 * Returns SYN_ERR_TIMEOUT when a bounded device wait of the step gave up (a
 * tensor-parallel peer whose words never arrived, or a weight copy that never
 * landed on this device); the session then stays failed: every later step and
 * generate returns SYN_ERR_TIMEOUT until it is closed. */
int syn_session_step(syn_session* s, uint32_t token, uint32_t pos, float* host_logits, int32_t* host_argmax);
/* n_steps steps on the device from position pos, with no host round trip
 * between them: step i feeds prompt[i] while i < n_prompt, else the argmax of
 * step i - 1 (greedy decode, llama_decode.cpp:267-291); host_tokens (n_steps)
 * receives each step's argmax and the call returns when they are on the host;
 * with host_tokens NULL the call only enqueues the steps on the session's
 * stream (synchronise on syn_session_stream). 1 <= n_prompt <= n_steps. With
 * host_tokens, a wait that gave up returns SYN_ERR_TIMEOUT as syn_session_step
 * does. */
int syn_session_generate(syn_session* s, const uint32_t* prompt, int n_prompt, uint32_t pos, int n_steps,
                         int32_t* host_tokens);
/* run(batch) (session.hpp:143-156) for the tokens of one sequence: n <= max_batch
 * tokens at positions pos .. pos + n - 1 of sequence seq, their K/V rows
 * appended before any of them attends (session.hpp:349-356); host_logits
 * (n_vocab floats) and host_argmax receive the last token's (op_last_row). Each
 * token's arithmetic is a single-token step's, so a prompt in chunks gives the
 * logits and cache rows a token-by-token decode gives (the reference's G1,
 * tests/sdk/llama_prefill.cpp:20). Needs a session opened with max_batch > 1 or
 * max_seqs > 1 (SYN_ERR_UNSUPPORTED otherwise, and for K-format or float layer
 * matrices or tensor parallelism); SYN_ERR_RANGE for n, seq, pos or a token out
 * of range. Blocks until the outputs are on the host. */
int syn_session_prefill(syn_session* s, int seq, const uint32_t* tokens, int n, uint32_t pos, float* host_logits,
                        int32_t* host_argmax);
/* One decode token for each of sequences 0 .. n - 1 (n <= max_batch and
 * max_seqs): tokens[i] at pos[i] of sequence i; host_logits receives n x n_vocab
 * floats, host_argmax n tokens. The weights stream once for all n rows (the
 * integer tensor-core GEMV from 3 rows); every row's bits are those of that
 * sequence decoded alone. */
int syn_session_step_batch(syn_session* s, int n, const uint32_t* tokens, const uint32_t* pos, float* host_logits,
                           int32_t* host_argmax);
/* Fill positions 0 .. n_pos - 1 of every sequence's KV cache with seeded
 * N(0, 1) binary16 values: benchmark inputs at a long context without decoding
 * up to it (no counterpart in the reference). */
int syn_session_fill_kv_random(syn_session* s, int n_pos, uint64_t seed);

/* Kernel launches one step makes (each graph replay launches exactly these). */
int syn_session_launches_per_step(const syn_session* s);

/* One step at (token, pos) with CUDA events around every op on the session's
 * stream (captured once as its own graph, without programmatic overlap between
 * ops), for per-kernel timing. For each op: its kind
 * (SYN_OP_*), layer (-1 outside layers), weight type, rows, cols, device time
 * (ms) and algorithmic bytes (what the op must move at least once: weights
 * with their scales, activations in and out, KV rows 0..pos). Returns the op
 * count in *n_ops (at most max_ops records written). */
enum { SYN_OP_EMBED = 0, SYN_OP_RMS_NORM = 1, SYN_OP_QUANTIZE = 2, SYN_OP_MATMUL = 3, SYN_OP_ATTENTION = 4,
       SYN_OP_SILU_MUL = 5, SYN_OP_ARGMAX = 6, SYN_OP_ALLGATHER = 7 };
typedef struct {
    int kind, layer, type, rows, cols;
    float ms;
    double bytes;
} syn_op_profile;
int syn_session_profile(syn_session* s, uint32_t token, uint32_t pos, syn_op_profile* out, int max_ops, int* n_ops);

/* ------------------------------------------------------------------------
 * Tensor parallelism over the GPUs of one node, one process (or thread) per
 * GPU. The reference computes every output element of a GEMV with one
 * thread's arithmetic whatever the thread count (its D1 contract,
 * tests/sdk/llama_threads.cpp:32, over kernels/gemv.hpp:72-161 row ranges);
 * the sharding here keeps that across GPUs: attention by KV-head groups, every
 * matrix by output rows, and the four per-layer activations (attention output,
 * residual after O, silu*up, residual after down) plus the logits all-gathered
 * in place. Each rank's results are bit-identical to one GPU's.
 * ---------------------------------------------------------------------- */
typedef struct syn_tp syn_tp;
#define SYN_TP_ID_BYTES 128
/* A new communicator id (an ncclUniqueId) on the rank that creates it; every
 * rank passes the same id to syn_tp_init. */
int syn_tp_unique_id(void* id_out);
/* Join the group as rank of world on device (collective over all ranks). */
int syn_tp_init(int rank, int world, const void* id, int device, syn_tp** out);
void syn_tp_close(syn_tp* tp);
/* In-place all-gather on stream: rank r's bytes_per_rank bytes sit at
 * buf + r * bytes_per_rank; afterwards every rank holds all of them. */
int syn_allgather(syn_tp* tp, void* buf, size_t bytes_per_rank, void* stream);

/* A rank's share of a model (what it loads, computes and owns). */
typedef struct {
    int rank, world;
    int head0, n_head;    /* query heads (attn_q rows head0 * head_dim ..) */
    int kv_head0, n_kv;   /* KV heads: attn_k / attn_v rows and this rank's KV cache */
    int embd0, n_embd;    /* rows of attn_output and ffn_down: the residual slice */
    int ff0, n_ff;        /* rows of ffn_gate and ffn_up */
    int vocab0, n_vocab;  /* rows of output.weight: the logits slice */
} syn_tp_layout;
/* The layout of rank of world for config c (host only): contiguous equal
 * shares; SYN_ERR_UNSUPPORTED unless world divides n_head_kv, n_embd, n_ff
 * and n_vocab. */
int syn_tp_layout_of(const syn_llama_config* c, int rank, int world, syn_tp_layout* out);
/* Sessions sharded over tp (NULL = one GPU). All ranks open, step, generate,
 * reset and close together (each call runs the same collectives); logits and
 * tokens come back whole on every rank. */
int syn_session_open_gguf_tp(const char* path, int max_ctx, int device, syn_tp* tp, syn_session** out);
int syn_session_open_synthetic_tp(const syn_llama_config* c, int max_ctx, uint64_t seed, int device, syn_tp* tp,
                                  syn_session** out);
int syn_session_tp_layout(const syn_session* s, syn_tp_layout* out);
/* How a sharded session gathers: *peer_stores 1 when each producing kernel
 * stores its slice straight into every rank's memory (CUDA IPC over NVLink)
 * and the reading kernels wait on per-rank flags, 0 when NCCL all-gathers
 * run between the kernels (SYN_TP_P2P=0, or a peer could not be mapped);
 * *wait_errors counts peer word reads that gave up (0 in a healthy run); a read
 * gives up after 2 s, or SYN_TP_WAIT_MS milliseconds when that is set at open. */
int syn_session_tp_status(syn_session* s, int* peer_stores, int* wait_errors);

/* Copy device memory to the host (synchronous), e.g. a KV cache for checking. */
int syn_copy_to_host(void* host_dst, const void* device_src, size_t bytes);

/* Device pointers of the session's logits (n_vocab floats) and stream. */
float* syn_session_logits(syn_session* s);
void* syn_session_stream(syn_session* s);
/* Device pointer and geometry of a layer's KV cache (K then V, max_ctx rows of
 * n_head_kv * head_dim halves each) of sequence 0; with max_seqs > 1, sequence
 * i's rows follow at i * max_ctx * n_head_kv * head_dim halves. */
uint16_t* syn_session_kv(syn_session* s, int layer, int which /*0 K, 1 V*/);
/* Copy a tensor of the model to the host in GGUF layout (for checking). */
int syn_session_weight(syn_session* s, const char* name, void* host_out, size_t bytes, int* type, int* rows,
                       int* cols);

#ifdef __cplusplus
}
#endif
#endif
