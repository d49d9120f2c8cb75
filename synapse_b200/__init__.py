"""synapse_b200: B200 (sm_100a) implementation of synapse's Llama decode hot path.

Python mirror of the C ABI in include/synapse_b200.h, for tests, benchmarks
and Python callers. Device buffers are torch CUDA tensors (torch is only the
allocator and stream provider here); every computation runs in the in-tree
CUDA library libsynapse_b200.so. There is no CPU fallback: importing the
package on a machine without the built library raises, and calling a kernel
without a GPU raises.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsynapse_b200.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
LAYOUT_GGUF, LAYOUT_PLANAR = 0, 1
QK = 32
QK_K = 256

STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "cuda error", 4: "out of device memory",
          5: "timeout", 6: "nccl error", 7: "bad format", 8: "out of range"}


class SynapseError(RuntimeError):
    def __init__(self, status, where):
        self.status = status
        detail = _lib.syn_last_error().decode() if status == 3 and _lib is not None else ""
        super().__init__(f"{where}: {STATUS.get(status, status)}" + (f" ({detail})" if detail else ""))


_lib = None


class LlamaConfig(ctypes.Structure):
    """syn_llama_config (models/llama.hpp:93-109 llama_config, the decode subset)."""
    _fields_ = [(n, ctypes.c_int) for n in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim",
                                             "n_vocab")] + \
               [("rms_eps", ctypes.c_float), ("rope_base", ctypes.c_float), ("rope_mode", ctypes.c_int),
                ("type_embd", ctypes.c_int), ("type_layers", ctypes.c_int), ("type_output", ctypes.c_int)]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


class SessionOptions(ctypes.Structure):
    """syn_session_options: positions per sequence, sequences, tokens per batched call."""
    _fields_ = [("max_ctx", ctypes.c_int), ("max_seqs", ctypes.c_int), ("max_batch", ctypes.c_int)]


def build():
    from . import buildlib
    return buildlib.build()


def lib():
    """The loaded CUDA library; raises if it was not built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run synapse_b200.build() (nvcc, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        _declare(L)
        _lib = L
    return _lib


def _declare(L):
    vp, sz, i32, f32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
    sig = {
        "syn_build_info": (ctypes.c_char_p, []),
        "syn_status_string": (ctypes.c_char_p, [i32]),
        "syn_last_error": (ctypes.c_char_p, []),
        "syn_device_errors": (i32, []),
        "syn_q8_act_bytes": (sz, [i32, i32]),
        "syn_quantize_q8_0": (i32, [vp, i32, i32, vp, vp]),
        "syn_q8_act_to_blocks": (i32, [vp, i32, i32, vp, vp]),
        "syn_q8k_act_bytes": (sz, [i32, i32]),
        "syn_quantize_q8_k": (i32, [vp, i32, i32, vp, vp]),
        "syn_q8k_act_to_blocks": (i32, [vp, i32, i32, vp, vp]),
        "syn_weight_bytes": (sz, [i32, i32, i32, i32]),
        "syn_repack_planar": (i32, [i32, vp, i32, i32, vp, vp]),
        "syn_upload_weight": (i32, [i32, vp, i32, i32, vp, i32, vp, sz, vp]),
        "syn_gemv_q": (i32, [i32, vp, i32, i32, i32, vp, i32, vp, vp, vp]),
        "syn_gemv_f": (i32, [i32, vp, i32, i32, vp, i32, vp, vp, vp]),
        "syn_gemv": (i32, [vp, vp]),
        "syn_gemv_fusable": (i32, [i32, i32, i32, i32, i32, i32]),
        "syn_attention_scratch_bytes": (sz, [i32, i32, i32, i32, i32]),
        "syn_attention": (i32, [vp, vp]),
        "syn_attention_noalloc": (i32, [vp, vp]),
        "syn_rope_kv_append": (i32, [vp, vp]),
        "syn_rope": (i32, [vp, vp, i32, i32, i32, vp, f32, vp, i32, vp, vp]),
        "syn_rope_table": (i32, [vp, i32, i32, f32, vp, vp, vp]),
        "syn_rms_norm": (i32, [vp, vp, i32, i32, f32, vp, vp, vp]),
        "syn_silu_mul": (i32, [vp, vp, i32, i32, vp, vp, vp]),
        "syn_add": (i32, [vp, vp, vp, sz, vp]),
        "syn_embed": (i32, [i32, vp, i32, i32, i32, vp, i32, vp, vp]),
        "syn_argmax": (i32, [vp, i32, i32, vp, vp]),
    }
    sig.update({
        "syn_session_open_gguf": (i32, [ctypes.c_char_p, i32, i32, ctypes.POINTER(vp)]),
        "syn_session_open_synthetic": (i32, [ctypes.POINTER(LlamaConfig), i32, ctypes.c_uint64, i32,
                                             ctypes.POINTER(vp)]),
        "syn_session_close": (None, [vp]),
        "syn_session_config": (i32, [vp, ctypes.POINTER(LlamaConfig)]),
        "syn_session_memory": (i32, [vp, ctypes.POINTER(sz), ctypes.POINTER(sz), ctypes.POINTER(sz)]),
        "syn_session_reset": (i32, [vp]),
        "syn_session_step": (i32, [vp, ctypes.c_uint32, ctypes.c_uint32, vp, vp]),
        "syn_session_generate": (i32, [vp, vp, i32, ctypes.c_uint32, i32, vp]),
        "syn_session_logits": (vp, [vp]),
        "syn_session_stream": (vp, [vp]),
        "syn_session_kv": (vp, [vp, i32, i32]),
        "syn_session_weight": (i32, [vp, ctypes.c_char_p, vp, sz, ctypes.POINTER(i32), ctypes.POINTER(i32),
                                     ctypes.POINTER(i32)]),
        "syn_session_launches_per_step": (i32, [vp]),
        "syn_session_profile": (i32, [vp, ctypes.c_uint32, ctypes.c_uint32, vp, i32, ctypes.POINTER(i32)]),
        "syn_copy_to_host": (i32, [vp, vp, sz]),
        "syn_tp_unique_id": (i32, [vp]),
        "syn_tp_init": (i32, [i32, i32, vp, i32, ctypes.POINTER(vp)]),
        "syn_tp_close": (None, [vp]),
        "syn_allgather": (i32, [vp, vp, sz, vp]),
        "syn_tp_layout_of": (i32, [ctypes.POINTER(LlamaConfig), i32, i32, ctypes.POINTER(TPLayout)]),
        "syn_session_open_gguf_tp": (i32, [ctypes.c_char_p, i32, i32, vp, ctypes.POINTER(vp)]),
        "syn_session_open_synthetic_tp": (i32, [ctypes.POINTER(LlamaConfig), i32, ctypes.c_uint64, i32, vp,
                                                ctypes.POINTER(vp)]),
        "syn_session_tp_layout": (i32, [vp, ctypes.POINTER(TPLayout)]),
        "syn_session_tp_status": (i32, [vp, ctypes.POINTER(i32), ctypes.POINTER(i32)]),
        "syn_session_open_gguf_ex": (i32, [ctypes.c_char_p, ctypes.POINTER(SessionOptions), i32, ctypes.POINTER(vp)]),
        "syn_session_open_synthetic_ex": (i32, [ctypes.POINTER(LlamaConfig), ctypes.POINTER(SessionOptions),
                                                ctypes.c_uint64, i32, ctypes.POINTER(vp)]),
        "syn_session_prefill": (i32, [vp, i32, vp, i32, ctypes.c_uint32, vp, vp]),
        "syn_session_step_batch": (i32, [vp, i32, vp, vp, vp, vp]),
        "syn_session_fill_kv_random": (i32, [vp, i32, ctypes.c_uint64]),
    })
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype, fn.argtypes = res, args


def exported_symbols():
    """Names the header declares (for the ABI check)."""
    import re
    hdr = open(os.path.join(os.path.dirname(HERE), "include", "synapse_b200.h")).read()
    return sorted(set(re.findall(r"\b(syn_[a-z0-9_]+)\s*\(", hdr)))


def check(status, where):
    if status != 0:
        raise SynapseError(status, where)


# ---------------------------------------------------------------------------
# torch helpers (device memory and streams only)

def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("synapse_b200 needs a CUDA GPU (B200); there is no CPU path")
    return torch


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def empty_bytes(n, device="cuda"):
    torch = _torch()
    return torch.empty(max(int(n), 1), dtype=torch.uint8, device=device)


# ---------------------------------------------------------------------------
# Q8_0 activations

def q8_act_bytes(n_tok, cols):
    return lib().syn_q8_act_bytes(n_tok, cols)


def quantize_q8_0(x, act=None, stream=None):
    """x: (n_tok, cols) f32 CUDA tensor -> device Q8_0 activation buffer (uint8)."""
    x = x.contiguous()
    n_tok, cols = (1, x.numel()) if x.dim() == 1 else x.shape
    if act is None:
        act = empty_bytes(q8_act_bytes(n_tok, cols), x.device)
    check(lib().syn_quantize_q8_0(_ptr(x), n_tok, cols, _ptr(act), _stream(stream)), "syn_quantize_q8_0")
    return act


def act_to_blocks(act, n_tok, cols, stream=None):
    torch = _torch()
    out = torch.empty(n_tok * (cols // QK) * 34, dtype=torch.uint8, device=act.device)
    check(lib().syn_q8_act_to_blocks(_ptr(act), n_tok, cols, _ptr(out), _stream(stream)), "syn_q8_act_to_blocks")
    return out


# ---------------------------------------------------------------------------
# Q8_K activations (the K formats' activation blocks)

def q8k_act_bytes(n_tok, cols):
    return lib().syn_q8k_act_bytes(n_tok, cols)


def quantize_q8_k(x, act=None, stream=None):
    """x: (n_tok, cols) f32 CUDA tensor, cols a multiple of 256 -> device Q8_K activation buffer (uint8)."""
    x = x.contiguous()
    n_tok, cols = (1, x.numel()) if x.dim() == 1 else x.shape
    if act is None:
        act = empty_bytes(q8k_act_bytes(n_tok, cols), x.device)
    check(lib().syn_quantize_q8_k(_ptr(x), n_tok, cols, _ptr(act), _stream(stream)), "syn_quantize_q8_k")
    return act


def q8k_act_to_blocks(act, n_tok, cols, stream=None):
    """Device Q8_K activations -> ggml block_q8_k bytes (292 per 256 values)."""
    torch = _torch()
    out = torch.empty(n_tok * (cols // QK_K) * 292, dtype=torch.uint8, device=act.device)
    check(lib().syn_q8k_act_to_blocks(_ptr(act), n_tok, cols, _ptr(out), _stream(stream)), "syn_q8k_act_to_blocks")
    return out


# ---------------------------------------------------------------------------
# weights

def weight_bytes(type_, rows, cols, layout=LAYOUT_PLANAR):
    return lib().syn_weight_bytes(type_, rows, cols, layout)


def upload_weight(type_, host_bytes, rows, cols, layout=LAYOUT_PLANAR, device="cuda", stream=None):
    """GGUF row-major bytes (numpy) -> device tensor in `layout`."""
    host_bytes = np.ascontiguousarray(host_bytes).view(np.uint8)
    dst = empty_bytes(weight_bytes(type_, rows, cols, layout), device)
    staging = empty_bytes(1 << 22, device)
    check(lib().syn_upload_weight(type_, host_bytes.ctypes.data_as(ctypes.c_void_p), rows, cols, _ptr(dst), layout,
                                  _ptr(staging), staging.numel(), _stream(stream)), "syn_upload_weight")
    _torch().cuda.current_stream().synchronize()
    return dst


def gemv_q(type_, w, layout, rows, cols, act, n_tok, y=None, residual=None, stream=None):
    torch = _torch()
    if y is None:
        y = torch.empty((n_tok, rows), dtype=torch.float32, device=w.device)
    check(lib().syn_gemv_q(type_, _ptr(w), layout, rows, cols, _ptr(act), n_tok, _ptr(y), _ptr(residual),
                           _stream(stream)), "syn_gemv_q")
    return y


def gemv_f(type_, w, rows, cols, x, y=None, residual=None, stream=None):
    torch = _torch()
    x = x.contiguous()
    n_tok = 1 if x.dim() == 1 else x.shape[0]
    if y is None:
        y = torch.empty((n_tok, rows), dtype=torch.float32, device=w.device)
    check(lib().syn_gemv_f(type_, _ptr(w), rows, cols, _ptr(x), n_tok, _ptr(y), _ptr(residual), _stream(stream)),
          "syn_gemv_f")
    return y


IN_Q8, IN_F32, IN_RMSNORM = 0, 1, 2
OUT_ROWS, OUT_SILU_PAIRS = 0, 1


class GemvArgs(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int), ("layout", ctypes.c_int), ("rows", ctypes.c_int), ("cols", ctypes.c_int),
                ("n_tok", ctypes.c_int), ("w", ctypes.c_void_p), ("in_mode", ctypes.c_int), ("act", ctypes.c_void_p),
                ("x", ctypes.c_void_p), ("gamma", ctypes.c_void_p), ("eps", ctypes.c_float),
                ("out_mode", ctypes.c_int), ("y", ctypes.c_void_p), ("residual", ctypes.c_void_p)]


def gemv_fused(type_, w, rows, cols, x, in_mode=IN_F32, gamma=None, eps=1e-5, out_mode=OUT_ROWS, residual=None,
               act=None, stream=None):
    """syn_gemv: the matmul with its input quantization (and rms_norm) and its silu*mul fused in."""
    torch = _torch()
    n_tok = (1 if x.dim() == 1 else x.shape[0]) if x is not None else 1
    out_rows = rows // 2 if out_mode == OUT_SILU_PAIRS else rows
    y = torch.empty((n_tok, out_rows), dtype=torch.float32, device=w.device)
    a = GemvArgs(type_, LAYOUT_PLANAR, rows, cols, n_tok, w.data_ptr(), in_mode,
                 act.data_ptr() if act is not None else None, x.data_ptr() if x is not None else None,
                 gamma.data_ptr() if gamma is not None else None, eps, out_mode, y.data_ptr(),
                 residual.data_ptr() if residual is not None else None)
    check(lib().syn_gemv(ctypes.byref(a), _stream(stream)), "syn_gemv")
    return y


def mul_mat(type_, w, layout, rows, cols, x, stream=None):
    """Y = X W^T for float activations x (n_tok, cols): quantizes x for Q4_0/Q8_0."""
    if type_ in (F32, F16):
        return gemv_f(type_, w, rows, cols, x, stream=stream)
    x = x.contiguous()
    n_tok = 1 if x.dim() == 1 else x.shape[0]
    act = quantize_q8_0(x.reshape(n_tok, cols), stream=stream)
    return gemv_q(type_, w, layout, rows, cols, act, n_tok, stream=stream)


# ---------------------------------------------------------------------------
# attention

class AttentionArgs(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p), ("pos", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("scratch", ctypes.c_void_p), ("cache_stride", ctypes.c_size_t),
                ("n_q", ctypes.c_int), ("n_head", ctypes.c_int), ("n_kv", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("max_len", ctypes.c_int), ("append", ctypes.c_int), ("rope", ctypes.c_int),
                ("rope_mode", ctypes.c_int), ("theta_scale", ctypes.c_float), ("scale", ctypes.c_float),
                ("freq_factors", ctypes.c_void_p), ("yarn", ctypes.c_void_p), ("rope_table", ctypes.c_void_p),
                ("order", ctypes.c_int)]


ORDER_REFERENCE, ORDER_SPLIT = 0, 1


def attention_scratch_bytes(n_q, n_head, n_kv, head_dim, max_len):
    return lib().syn_attention_scratch_bytes(n_q, n_head, n_kv, head_dim, max_len)


def attention(q, k, v, k_cache, v_cache, pos, n_head, n_kv, head_dim, max_len, theta_scale, scale,
              cache_stride=None, append=True, rope=True, rope_mode=0, freq_factors=None, out=None, scratch=None,
              rope_table=None, order=ORDER_REFERENCE, stream=None):
    """Fused RoPE + F16 append + decode attention for n_q queries (see syn_attention); order:
    ORDER_REFERENCE (the reference's summation order) or ORDER_SPLIT (split p.V, re-associated)."""
    torch = _torch()
    n_q = pos.numel()
    if out is None:
        out = torch.empty((n_q, n_head * head_dim), dtype=torch.float32, device=q.device)
    if scratch is None:
        scratch = empty_bytes(attention_scratch_bytes(n_q, n_head, n_kv, head_dim, max_len), q.device)
    if cache_stride is None:
        cache_stride = k_cache.numel() // n_q
    a = AttentionArgs(q.data_ptr(), k.data_ptr() if k is not None else None,
                      v.data_ptr() if v is not None else None, k_cache.data_ptr(), v_cache.data_ptr(),
                      pos.data_ptr(), out.data_ptr(), scratch.data_ptr(), cache_stride, n_q, n_head, n_kv, head_dim,
                      max_len, int(append), int(rope), rope_mode, theta_scale, scale,
                      freq_factors.data_ptr() if freq_factors is not None else None, None,
                      rope_table.data_ptr() if rope_table is not None else None, int(order))
    check(lib().syn_attention(ctypes.byref(a), _stream(stream)), "syn_attention")
    return out


def rope_table(max_len, head_dim, theta_scale, freq_factors=None, device="cuda", stream=None):
    """(cos, sin) of every RoPE pair at every position: a [max_len, head_dim / 2, 2] float tensor."""
    torch = _torch()
    t = torch.empty((max_len, head_dim // 2, 2), dtype=torch.float32, device=device)
    check(lib().syn_rope_table(t.data_ptr(), max_len, head_dim, theta_scale,
                               freq_factors.data_ptr() if freq_factors is not None else None, None,
                               _stream(stream)), "syn_rope_table")
    return t


def rope_kv_append(k, v, k_cache, v_cache, pos, n_kv, head_dim, max_len, theta_scale, cache_stride=0,
                   rope=True, rope_mode=0, freq_factors=None, stream=None):
    n_q = pos.numel()
    a = AttentionArgs(None, k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), pos.data_ptr(),
                      None, None, cache_stride, n_q, n_kv, n_kv, head_dim, max_len, 1, int(rope), rope_mode,
                      theta_scale, 1.0, freq_factors.data_ptr() if freq_factors is not None else None, None)
    check(lib().syn_rope_kv_append(ctypes.byref(a), _stream(stream)), "syn_rope_kv_append")


def rope(x, pos, n_heads, head_dim, theta_scale, rope_mode=0, freq_factors=None, stream=None):
    torch = _torch()
    x = x.contiguous()
    n = pos.numel()
    out = torch.empty_like(x)
    check(lib().syn_rope(_ptr(x), _ptr(out), n, n_heads, head_dim, _ptr(pos), theta_scale, _ptr(freq_factors),
                         rope_mode, None, _stream(stream)), "syn_rope")
    return out


# ---------------------------------------------------------------------------
# element-wise

def rms_norm(x, gamma, eps, want_f32=True, want_act=False, stream=None):
    torch = _torch()
    x = x.contiguous()
    n_tok, cols = (1, x.numel()) if x.dim() == 1 else x.shape
    out = torch.empty((n_tok, cols), dtype=torch.float32, device=x.device) if want_f32 else None
    act = empty_bytes(q8_act_bytes(n_tok, cols), x.device) if want_act else None
    check(lib().syn_rms_norm(_ptr(x), _ptr(gamma), n_tok, cols, eps, _ptr(out), _ptr(act), _stream(stream)),
          "syn_rms_norm")
    return out, act


def silu_mul(g, u, want_f32=True, want_act=False, stream=None):
    torch = _torch()
    g, u = g.contiguous(), u.contiguous()
    n_tok, cols = (1, g.numel()) if g.dim() == 1 else g.shape
    out = torch.empty((n_tok, cols), dtype=torch.float32, device=g.device) if want_f32 else None
    act = empty_bytes(q8_act_bytes(n_tok, cols), g.device) if want_act else None
    check(lib().syn_silu_mul(_ptr(g), _ptr(u), n_tok, cols, _ptr(out), _ptr(act), _stream(stream)),
          "syn_silu_mul")
    return out, act


def add(a, b, out=None, stream=None):
    torch = _torch()
    if out is None:
        out = torch.empty_like(a)
    check(lib().syn_add(_ptr(a), _ptr(b), _ptr(out), a.numel(), _stream(stream)), "syn_add")
    return out


def embed(type_, table, layout, rows, cols, tokens, stream=None):
    torch = _torch()
    n = tokens.numel()
    out = torch.empty((n, cols), dtype=torch.float32, device=table.device)
    check(lib().syn_embed(type_, _ptr(table), layout, rows, cols, _ptr(tokens), n, _ptr(out), _stream(stream)),
          "syn_embed")
    return out


def argmax(x, stream=None):
    torch = _torch()
    x = x.contiguous()
    n_tok, n = (1, x.numel()) if x.dim() == 1 else x.shape
    out = torch.empty(n_tok, dtype=torch.int32, device=x.device)
    check(lib().syn_argmax(_ptr(x), n_tok, n, _ptr(out), _stream(stream)), "syn_argmax")
    return out


# ---------------------------------------------------------------------------
# the decode session (models/llama.hpp load_llama + graph/session.hpp session)

class OpProfile(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("layer", ctypes.c_int), ("type", ctypes.c_int), ("rows", ctypes.c_int),
                ("cols", ctypes.c_int), ("ms", ctypes.c_float), ("bytes", ctypes.c_double)]


OP_KINDS = {0: "embed", 1: "rms_norm", 2: "quantize", 3: "matmul", 4: "attention", 5: "silu_mul", 6: "argmax",
            7: "allgather"}


def copy_to_host(ptr, nbytes, dtype=np.uint8):
    out = np.empty(nbytes, dtype=np.uint8)
    check(lib().syn_copy_to_host(out.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(ptr), nbytes), "copy")
    return out.view(dtype)


class TPLayout(ctypes.Structure):
    """A rank's share of a model under tensor parallelism (syn_tp_layout)."""
    _fields_ = [(k, ctypes.c_int) for k in ("rank", "world", "head0", "n_head", "kv_head0", "n_kv", "embd0",
                                             "n_embd", "ff0", "n_ff", "vocab0", "n_vocab")]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


def tp_layout(cfg, rank, world):
    """The rows and heads rank of world holds for a model config (host only; no GPU needed)."""
    c = LlamaConfig(**{k: cfg[k] for k, _ in LlamaConfig._fields_ if k in cfg})
    out = TPLayout()
    check(lib().syn_tp_layout_of(ctypes.byref(c), int(rank), int(world), ctypes.byref(out)), "syn_tp_layout_of")
    return out.as_dict()


class TP:
    """A tensor-parallel group: one rank per GPU, joined through an id that rank 0 creates.

    share_id(id_bytes) -> id_bytes must give every rank rank 0's bytes (e.g. a
    torch.distributed broadcast); it is called on every rank."""

    def __init__(self, rank, world, device, share_id):
        import ctypes as C
        buf = (C.c_char * 128)()
        if rank == 0:
            check(lib().syn_tp_unique_id(buf), "syn_tp_unique_id")
        got = share_id(bytes(buf))
        if len(got) != 128:
            raise ValueError("tp id must be 128 bytes")
        buf = (C.c_char * 128).from_buffer_copy(got)
        self.h = ctypes.c_void_p()
        self.rank, self.world, self.device = int(rank), int(world), int(device)
        check(lib().syn_tp_init(self.rank, self.world, buf, self.device, ctypes.byref(self.h)), "syn_tp_init")

    @classmethod
    def from_torch_distributed(cls, device):
        """Join with the ranks of the default torch.distributed group (any backend)."""
        import torch.distributed as dist
        rank, world = dist.get_rank(), dist.get_world_size()

        def share(b):
            obj = [b]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]
        return cls(rank, world, device, share)

    def allgather(self, buf_ptr, bytes_per_rank, stream=None):
        check(lib().syn_allgather(self.h, buf_ptr, int(bytes_per_rank), stream), "syn_allgather")

    def close(self):
        if self.h:
            lib().syn_tp_close(self.h)
            self.h = None


class Session:
    """A Llama decode session on one GPU (or this rank's share of a
    tensor-parallel group): weights, activations and the F16 KV cache in one
    device arena; each step is a captured CUDA graph."""

    def __init__(self, handle, max_batch=1):
        self.h = handle
        self.max_batch = max_batch
        c = LlamaConfig()
        check(lib().syn_session_config(self.h, ctypes.byref(c)), "syn_session_config")
        self.config = c.as_dict()
        self.n_vocab = c.n_vocab
        self._logits = np.empty(self.n_vocab, dtype=np.float32)

    @classmethod
    def open(cls, path, max_ctx, device=0, tp=None):
        h = ctypes.c_void_p()
        check(lib().syn_session_open_gguf_tp(str(path).encode(), int(max_ctx), int(device), tp.h if tp else None,
                                             ctypes.byref(h)), f"syn_session_open_gguf({path})")
        return cls(h)

    @classmethod
    def open_ex(cls, path, max_ctx, max_seqs=1, max_batch=1, device=0):
        """A GGUF session holding max_seqs sequences' KV caches, taking up to max_batch tokens per batched call."""
        h = ctypes.c_void_p()
        o = SessionOptions(int(max_ctx), int(max_seqs), int(max_batch))
        check(lib().syn_session_open_gguf_ex(str(path).encode(), ctypes.byref(o), int(device), ctypes.byref(h)),
              f"syn_session_open_gguf_ex({path})")
        return cls(h, max_batch)

    @classmethod
    def synthetic_ex(cls, cfg, max_ctx, max_seqs=1, max_batch=1, seed=0, device=0):
        c = LlamaConfig(**{k: cfg[k] for k, _ in LlamaConfig._fields_ if k in cfg})
        h = ctypes.c_void_p()
        o = SessionOptions(int(max_ctx), int(max_seqs), int(max_batch))
        check(lib().syn_session_open_synthetic_ex(ctypes.byref(c), ctypes.byref(o), int(seed), int(device),
                                                  ctypes.byref(h)), "syn_session_open_synthetic_ex")
        return cls(h, max_batch)

    def prefill(self, tokens, pos, seq=0, logits=True):
        """run(batch): the tokens of sequence seq at positions pos, pos + 1, ...; (last logits, last argmax)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.n_vocab, dtype=np.float32) if logits else None
        nxt = ctypes.c_int32()
        check(lib().syn_session_prefill(self.h, int(seq), t.ctypes.data_as(ctypes.c_void_p), t.size, int(pos),
                                        out.ctypes.data_as(ctypes.c_void_p) if logits else None, ctypes.byref(nxt)),
              "syn_session_prefill")
        return out, int(nxt.value)

    def step_batch(self, tokens, positions, logits=True):
        """One token for each of sequences 0 .. n-1: (logits [n][vocab], argmax [n])."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint32)
        out = np.empty((t.size, self.n_vocab), dtype=np.float32) if logits else None
        nxt = np.empty(t.size, dtype=np.int32)
        check(lib().syn_session_step_batch(self.h, t.size, t.ctypes.data_as(ctypes.c_void_p),
                                           p.ctypes.data_as(ctypes.c_void_p),
                                           out.ctypes.data_as(ctypes.c_void_p) if logits else None,
                                           nxt.ctypes.data_as(ctypes.c_void_p)), "syn_session_step_batch")
        return out, nxt

    def fill_kv_random(self, n_pos, seed=0):
        check(lib().syn_session_fill_kv_random(self.h, int(n_pos), int(seed)), "syn_session_fill_kv_random")

    @classmethod
    def synthetic(cls, cfg, max_ctx, seed=0, device=0, tp=None):
        """cfg: dict with n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab, rms_eps, rope_base,
        type_embd, type_layers, type_output (-1 = tied). tp: a TP group (every rank opens together)."""
        c = LlamaConfig(**{k: cfg[k] for k, _ in LlamaConfig._fields_ if k in cfg})
        h = ctypes.c_void_p()
        check(lib().syn_session_open_synthetic_tp(ctypes.byref(c), int(max_ctx), int(seed), int(device),
                                                  tp.h if tp else None, ctypes.byref(h)),
              "syn_session_open_synthetic")
        return cls(h)

    def tp_layout(self):
        out = TPLayout()
        check(lib().syn_session_tp_layout(self.h, ctypes.byref(out)), "syn_session_tp_layout")
        return out.as_dict()

    def tp_status(self):
        """{'peer_stores': bool, 'wait_errors': int} of a sharded session."""
        p, e = ctypes.c_int(), ctypes.c_int()
        check(lib().syn_session_tp_status(self.h, ctypes.byref(p), ctypes.byref(e)), "syn_session_tp_status")
        return {"peer_stores": bool(p.value), "wait_errors": e.value}

    def step(self, token, pos, logits=True):
        """One token at pos: (logits copy or None, argmax)."""
        nxt = ctypes.c_int32()
        out = self._logits.ctypes.data_as(ctypes.c_void_p) if logits else None
        check(lib().syn_session_step(self.h, int(token), int(pos), out, ctypes.byref(nxt)), "syn_session_step")
        return (self._logits.copy() if logits else None), int(nxt.value)

    def generate(self, prompt, pos, n_steps, wait=True):
        """n_steps device-side steps: prompt tokens first, then greedy; returns each step's argmax.
        wait=False only enqueues them on the session stream (returns None)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(n_steps, dtype=np.int32) if wait else None
        check(lib().syn_session_generate(self.h, p.ctypes.data_as(ctypes.c_void_p), p.size, int(pos), int(n_steps),
                                         out.ctypes.data_as(ctypes.c_void_p) if wait else None),
              "syn_session_generate")
        return out

    def launches_per_step(self):
        return lib().syn_session_launches_per_step(self.h)

    def profile(self, token, pos):
        """Per-op CUDA-event times of one eager step: list of dicts."""
        n = ctypes.c_int()
        check(lib().syn_session_profile(self.h, int(token), int(pos), None, 0, ctypes.byref(n)), "profile")
        recs = (OpProfile * max(n.value, 1))()
        check(lib().syn_session_profile(self.h, int(token), int(pos), recs, n.value, ctypes.byref(n)), "profile")
        return [dict(kind=OP_KINDS[r.kind], layer=r.layer, type=r.type, rows=r.rows, cols=r.cols, ms=r.ms,
                     bytes=r.bytes) for r in recs]

    def reset(self):
        check(lib().syn_session_reset(self.h), "syn_session_reset")

    def memory(self):
        a, w, k = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        check(lib().syn_session_memory(self.h, ctypes.byref(a), ctypes.byref(w), ctypes.byref(k)), "memory")
        return {"arena": a.value, "weights": w.value, "kv": k.value}

    def weight(self, name):
        """(type, rows, cols, GGUF-layout bytes) of a tensor, copied from the device."""
        t, r, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(lib().syn_session_weight(self.h, name.encode(), None, 0, ctypes.byref(t), ctypes.byref(r),
                                       ctypes.byref(c)), f"weight {name}")
        n = weight_bytes(t.value, r.value, c.value, LAYOUT_GGUF)
        buf = np.empty(n, dtype=np.uint8)
        check(lib().syn_session_weight(self.h, name.encode(), buf.ctypes.data_as(ctypes.c_void_p), n, None, None,
                                       None), f"weight {name}")
        return t.value, r.value, c.value, buf

    def stream_handle(self):
        return lib().syn_session_stream(self.h)

    def logits_ptr(self):
        return lib().syn_session_logits(self.h)

    def kv_ptr(self, layer, which):
        return lib().syn_session_kv(self.h, layer, which)

    def close(self):
        if self.h:
            lib().syn_session_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
