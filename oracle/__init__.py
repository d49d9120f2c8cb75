"""ctypes binding of the C oracle -- TEST INFRASTRUCTURE ONLY.

The C restatement of synapse's CPU decode path (oracle.c) is the parity
checker for the CUDA kernels. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs import this package; the product (synapse_b200)
never does.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
QK = 32
QK_K = 256
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q4_K: 144, Q6_K: 210}
BLOCK_ELEMS = {Q4_0: QK, Q8_0: QK, Q4_K: QK_K, Q6_K: QK_K}
Q8_K_BYTES = 292

_lib = None


def build():
    """Compile oracle.c into _build/liboracle.so (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, sz, f32p = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p
        L.orc_fp16_to_float.restype = ctypes.c_float
        L.orc_fp16_to_float.argtypes = [ctypes.c_uint16]
        L.orc_float_to_fp16.restype = ctypes.c_uint16
        L.orc_float_to_fp16.argtypes = [ctypes.c_float]
        for name in ("orc_quantize_row_q8_0", "orc_quantize_row_q4_0", "orc_quantize_row_q8_k"):
            getattr(L, name).argtypes = [vp, sz, vp]
        L.orc_dequantize_row.argtypes = [ctypes.c_int, vp, sz, vp]
        L.orc_gemv.argtypes = [ctypes.c_int, vp, sz, sz, vp, vp]
        L.orc_gemv_q8act.argtypes = [ctypes.c_int, vp, sz, sz, vp, vp]
        L.orc_gemv_q8k.argtypes = [ctypes.c_int, vp, sz, sz, vp, vp]
        L.orc_gemm.argtypes = [ctypes.c_int, vp, sz, sz, vp, sz, vp]
        L.orc_rope_theta_scale.restype = ctypes.c_float
        L.orc_rope_theta_scale.argtypes = [ctypes.c_float, sz]
        L.orc_rope.argtypes = [vp, vp, sz, sz, ctypes.c_uint32, ctypes.c_float, vp, ctypes.c_int, vp]
        L.orc_kv_append.argtypes = [vp, vp, vp, vp, sz, sz, sz, ctypes.c_uint32]
        L.orc_attention_group_floats.restype = sz
        L.orc_attention_group_floats.argtypes = [sz, sz, sz, sz]
        L.orc_attention.argtypes = [vp, vp, vp, vp, vp, sz, sz, sz, ctypes.c_uint32, sz, ctypes.c_float, vp, vp]
        L.orc_attend_group.argtypes = [vp, vp, vp, sz, sz, sz, ctypes.c_uint32, sz, ctypes.c_float, vp, vp, sz]
        L.orc_softmax.argtypes = [vp, vp, sz]
        L.orc_expf.argtypes = [vp, vp, sz]
        L.orc_rms_norm.argtypes = [vp, vp, ctypes.c_float, vp, sz]
        for name in ("orc_silu",):
            getattr(L, name).argtypes = [vp, vp, sz]
        for name in ("orc_mul", "orc_add"):
            getattr(L, name).argtypes = [vp, vp, vp, sz]
        L.orc_llama_create.restype = vp
        L.orc_llama_create.argtypes = [vp, _Tensor, _Tensor, _Tensor, vp, vp]
        L.orc_llama_destroy.argtypes = [vp]
        L.orc_llama_reset.argtypes = [vp]
        L.orc_llama_step.argtypes = [vp, ctypes.c_uint32, ctypes.c_uint32, vp]
        L.orc_llama_step.restype = ctypes.c_int
        L.orc_llama_kcache.restype = vp
        L.orc_llama_kcache.argtypes = [vp, sz]
        L.orc_llama_vcache.restype = vp
        L.orc_llama_vcache.argtypes = [vp, sz]
        L.orc_llama_run.argtypes = [vp, ctypes.c_uint32, ctypes.c_uint32, sz, sz, ctypes.c_int, vp]
        L.orc_llama_run.restype = ctypes.c_int
        L.orc_fill_random.argtypes = [ctypes.c_int, sz, sz, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, vp]
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_get_threads.restype = ctypes.c_int
        _lib = L
    return _lib


class _Tensor(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int), ("data", ctypes.c_void_p)]


class _Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_size_t) for n in
                ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab", "max_ctx")] + \
               [("rms_eps", ctypes.c_float), ("rope_base", ctypes.c_float)]


class _Layer(ctypes.Structure):
    _fields_ = [(n, _Tensor) for n in
                ("attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "gate", "up", "down")]


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def set_threads(n):
    lib().orc_set_threads(int(n))


def fp16_to_float(h):
    return lib().orc_fp16_to_float(int(h))


def float_to_fp16(f):
    return lib().orc_float_to_fp16(float(f))


def row_bytes(type_, cols):
    if type_ == F32:
        return cols * 4
    if type_ == F16:
        return cols * 2
    return cols // BLOCK_ELEMS[type_] * BLOCK_BYTES[type_]


def quantize_q8_0(x):
    """x: (..., cols) f32 -> uint8 blocks (..., cols/32*34), ggml's Q8_0 layout."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    cols = x.shape[-1]
    out = np.empty(x.shape[:-1] + (cols // QK * 34,), dtype=np.uint8)
    xs, os_ = x.reshape(-1, cols), out.reshape(-1, cols // QK * 34)
    for i in range(xs.shape[0]):
        lib().orc_quantize_row_q8_0(_p(xs[i]), cols, _p(os_[i]))
    return out


def quantize_q8_k(x):
    """x: (..., cols) f32 -> uint8 blocks (..., cols/256*292), ggml's block_q8_k."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    cols = x.shape[-1]
    out = np.empty(x.shape[:-1] + (cols // QK_K * Q8_K_BYTES,), dtype=np.uint8)
    xs, os_ = x.reshape(-1, cols), out.reshape(-1, cols // QK_K * Q8_K_BYTES)
    for i in range(xs.shape[0]):
        lib().orc_quantize_row_q8_k(_p(xs[i]), cols, _p(os_[i]))
    return out


def random_k_blocks(type_, rows, cols, seed, log2_scale=(-14, -8)):
    """Seeded random Q4_K / Q6_K rows: every byte pattern of the quants and
    sub-block scales is a valid block; the binary16 super-block scales are
    drawn from [2^lo, 2^hi) of log2_scale so no value is inf or nan."""
    rng = np.random.default_rng(seed)
    nb = cols // QK_K
    out = rng.integers(0, 256, (rows, nb, BLOCK_BYTES[type_]), dtype=np.uint8)
    lo, hi = log2_scale
    scale = lambda n: (2.0 ** rng.uniform(lo, hi, n)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    if type_ == Q4_K:
        out[:, :, 0:2] = scale(rows * nb).reshape(rows, nb, 2)  # d
        out[:, :, 2:4] = scale(rows * nb).reshape(rows, nb, 2)  # dmin
    elif type_ == Q6_K:
        out[:, :, 208:210] = scale(rows * nb).reshape(rows, nb, 2)
    else:
        raise ValueError(type_)
    return out.reshape(rows, -1)


def quantize_q4_0(x):
    """Weights (rows, cols) f32 -> Q4_0 bytes (rows, cols/32*18), ggml's reference quantizer."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty((rows, cols // QK * 18), dtype=np.uint8)
    lib().orc_quantize_row_q4_0(_p(x), rows * cols, _p(out))
    return out


def quantize_weights(x, type_):
    x = np.ascontiguousarray(x, dtype=np.float32)
    if type_ == Q4_0:
        return quantize_q4_0(x)
    if type_ == Q8_0:
        return quantize_q8_0(x)
    if type_ == F32:
        return x.view(np.uint8).reshape(x.shape[0], -1).copy()
    if type_ == F16:
        h = np.array([float_to_fp16(v) for v in x.reshape(-1)], dtype=np.uint16)
        return h.view(np.uint8).reshape(x.shape[0], -1)
    raise ValueError(type_)


def random_weights(type_, rows, cols, seed, tensor, sigma=0.02):
    """Seeded N(0, sigma) weights in GGUF bytes (float32 array for F32), made on the oracle's threads."""
    if type_ == F32:
        out = np.empty((rows, cols), dtype=np.float32)
    else:
        out = np.empty((rows, row_bytes(type_, cols)), dtype=np.uint8)
    lib().orc_fill_random(type_, rows, cols, seed, tensor, sigma, _p(out))
    return out


def dequantize(type_, data, rows, cols):
    data = np.ascontiguousarray(data).view(np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    rb = row_bytes(type_, cols)
    d = data.reshape(-1)
    for r in range(rows):
        lib().orc_dequantize_row(type_, _p(d[r * rb:(r + 1) * rb]), cols, _p(out[r]))
    return out


def gemv(type_, w, rows, cols, x):
    w = np.ascontiguousarray(w).view(np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    lib().orc_gemv(type_, _p(w), rows, cols, _p(x), _p(y))
    return y


def gemv_q8act(type_, w, rows, cols, act):
    w = np.ascontiguousarray(w).view(np.uint8)
    act = np.ascontiguousarray(act, dtype=np.uint8)
    y = np.empty(rows, dtype=np.float32)
    lib().orc_gemv_q8act(type_, _p(w), rows, cols, _p(act), _p(y))
    return y


def gemv_q8k(type_, w, rows, cols, act):
    """Q4_K / Q6_K rows on ggml block_q8_k activations."""
    w = np.ascontiguousarray(w).view(np.uint8)
    act = np.ascontiguousarray(act, dtype=np.uint8)
    y = np.empty(rows, dtype=np.float32)
    lib().orc_gemv_q8k(type_, _p(w), rows, cols, _p(act), _p(y))
    return y


def gemm(type_, w, rows, cols, x):
    """x: (n, cols) -> (n, rows); every row as gemv (G1)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
    w = np.ascontiguousarray(w).view(np.uint8)
    y = np.empty((x.shape[0], rows), dtype=np.float32)
    lib().orc_gemm(type_, _p(w), rows, cols, _p(x), x.shape[0], _p(y))
    return y


def rope_theta_scale(base, head_dim):
    return lib().orc_rope_theta_scale(float(base), int(head_dim))


def rope(x, head_dim, pos, theta_scale, freq_factors=None, neox=False):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    ff = None if freq_factors is None else np.ascontiguousarray(freq_factors, dtype=np.float32)
    lib().orc_rope(_p(x), _p(out), x.size, head_dim, pos, theta_scale, _p(ff), int(neox), None)
    return out


def kv_append(k, v, kc, vc, max_ctx, n_kv, head_dim, pos):
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    lib().orc_kv_append(_p(k), _p(v), _p(kc), _p(vc), max_ctx, n_kv, head_dim, pos)


def attention(q, k, v, kc, vc, max_ctx, n_kv, head_dim, pos, n_heads, scale):
    """kv_append(k, v) at pos into the uint16 caches kc, vc (max_ctx*n_kv*hd), then attention."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty(n_heads * head_dim, dtype=np.float32)
    scratch = np.empty(n_kv * lib().orc_attention_group_floats(n_heads, n_kv, head_dim, max_ctx), dtype=np.float32)
    lib().orc_attention(_p(q), _p(k), _p(v), _p(kc), _p(vc), max_ctx, n_kv, head_dim, pos, n_heads, scale,
                        _p(out), _p(scratch))
    return out


def attend(q, kc, vc, max_ctx, n_kv, head_dim, pos, n_heads, scale):
    """Attention over rows 0..pos of the caches (no append); every KV group."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    out = np.empty(n_heads * head_dim, dtype=np.float32)
    slot = lib().orc_attention_group_floats(n_heads, n_kv, head_dim, max_ctx)
    scratch = np.empty(slot, dtype=np.float32)
    for g in range(n_kv):
        lib().orc_attend_group(_p(q), _p(kc), _p(vc), max_ctx, n_kv, head_dim, pos, n_heads, scale, _p(out),
                               _p(scratch), g)
    return out


def rms_norm(x, gamma, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    g = np.ascontiguousarray(gamma, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_rms_norm(_p(x), _p(g), eps, _p(out), x.size)
    return out


def silu(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_silu(_p(x), _p(out), x.size)
    return out


def expf(x):
    """The host C library's expf on each element (what the reference's std::exp on float gives)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_expf(_p(x), _p(out), x.size)
    return out


def softmax(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_softmax(_p(x), _p(out), x.size)
    return out


class Llama:
    """The reference's Llama decode graph on the CPU (one token per step).

    weights: dict with 'token_embd', 'output_norm', optional 'output', and
    per layer 'blk.{l}.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,
    ffn_gate,ffn_up,ffn_down}', each (type, numpy bytes or f32 array).
    """

    NAMES = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate", "ffn_up",
             "ffn_down")

    def __init__(self, cfg, weights, max_ctx, freq_factors=None):
        self.cfg = dict(cfg)
        self._keep = []

        def t(name):
            if name not in weights:
                return _Tensor(0, None)
            ty, arr = weights[name]
            arr = np.ascontiguousarray(arr)
            self._keep.append(arr)
            return _Tensor(ty, arr.ctypes.data)

        c = _Config(cfg["n_layer"], cfg["n_embd"], cfg["n_ff"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"],
                    cfg["n_vocab"], max_ctx, cfg["rms_eps"], cfg["rope_base"])
        layers = (_Layer * cfg["n_layer"])()
        for l in range(cfg["n_layer"]):
            for field, nm in zip(_Layer._fields_, self.NAMES):
                setattr(layers[l], field[0], t(f"blk.{l}.{nm}"))
        ff = None
        if freq_factors is not None:
            ff = np.ascontiguousarray(freq_factors, dtype=np.float32)
            self._keep.append(ff)
        self._c, self._layers = c, layers
        self.h = lib().orc_llama_create(ctypes.byref(c), t("token_embd"), t("output_norm"), t("output"), layers,
                                        _p(ff))
        self.max_ctx = max_ctx

    def step(self, token, pos):
        logits = np.empty(self.cfg["n_vocab"], dtype=np.float32)
        rc = lib().orc_llama_step(self.h, int(token), int(pos), _p(logits))
        if rc != 0:
            raise ValueError("oracle step rejected token/pos")
        return logits

    def run(self, token, pos, l0, l1, embed=True, logits=False):
        """Part of a step (embedding, layers [l0, l1), optionally the head)."""
        out = np.empty(self.cfg["n_vocab"], dtype=np.float32) if logits else None
        if lib().orc_llama_run(self.h, int(token), int(pos), l0, l1, int(embed), _p(out)) != 0:
            raise ValueError("oracle run rejected its arguments")
        return out

    def reset(self):
        lib().orc_llama_reset(self.h)

    def kcache(self, layer):
        n = self.max_ctx * self.cfg["n_head_kv"] * self.cfg["head_dim"]
        return np.ctypeslib.as_array(ctypes.cast(lib().orc_llama_kcache(self.h, layer),
                                                 ctypes.POINTER(ctypes.c_uint16)), shape=(n,))

    def vcache(self, layer):
        n = self.max_ctx * self.cfg["n_head_kv"] * self.cfg["head_dim"]
        return np.ctypeslib.as_array(ctypes.cast(lib().orc_llama_vcache(self.h, layer),
                                                 ctypes.POINTER(ctypes.c_uint16)), shape=(n,))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_llama_destroy(self.h)
            self.h = None
