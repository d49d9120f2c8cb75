"""Synthetic Llama models as GGUF files (the reference reads GGUF; it ships no
weights for the benchmark shapes, so benchmarks and tests make their own).

- quantize_q8_0 / quantize_q4_0: ggml's reference weight quantizers
  (quantize_row_q8_0_ref -- the same algorithm as the reference's activation
  quantizer, quant/q8.hpp:54-69 -- and quantize_row_q4_0_ref), vectorised in
  numpy with float32 arithmetic.
- write_gguf: a GGUF v3 writer (the layout gguf/reader.hpp:1-30 parses).
- random_llama_weights / write_llama_gguf: a seeded Llama of N(0, 0.02)
  matrices and unit norms, in the tensor names models/llama.hpp binds.
"""
import struct

import numpy as np

F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8
QK = 32
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34}

# GGUF metadata value types
_U32, _I32, _F32, _BOOL, _STR, _ARR, _U64 = 4, 5, 6, 7, 8, 9, 10


def _round_half_away(v):
    v = v.astype(np.float64)
    return np.sign(v) * np.floor(np.abs(v) + 0.5)


def quantize_q8_0(x):
    """(rows, cols) f32 -> (rows, cols/32*34) uint8 in ggml's block_q8_0 layout."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    b = x.reshape(rows, cols // QK, QK)
    amax = np.abs(b).max(axis=-1, keepdims=True)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = _round_half_away((b * inv).astype(np.float32)).astype(np.int8)
    out = np.empty((rows, cols // QK, 34), dtype=np.uint8)
    out[:, :, :2] = d.astype(np.float16).view(np.uint8).reshape(rows, cols // QK, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


def quantize_q4_0(x):
    """(rows, cols) f32 -> (rows, cols/32*18) uint8 in ggml's block_q4_0 layout."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    b = x.reshape(-1, QK)
    imax = np.abs(b).argmax(axis=-1)[:, None]
    mx = np.take_along_axis(b, imax, axis=-1)
    d = (mx / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.trunc((b * inv).astype(np.float32) + np.float32(8.5)).astype(np.int32)
    q = np.minimum(q, 15).astype(np.uint8)
    packed = q[:, :16] | (q[:, 16:] << 4)
    out = np.concatenate([d.astype(np.float16).view(np.uint8), packed], axis=1)
    return out.reshape(rows, -1)


def encode(x, type_):
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    if type_ == F32:
        return x
    if type_ == F16:
        return x.astype(np.float16).view(np.uint8).reshape(x.shape[0], -1)
    if type_ == Q8_0:
        return quantize_q8_0(x)
    if type_ == Q4_0:
        return quantize_q4_0(x)
    raise ValueError(f"unsupported type {type_}")


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key, value):
    if isinstance(value, bool):
        return _str(key) + struct.pack("<IB", _BOOL, int(value))
    if isinstance(value, int):
        return _str(key) + struct.pack("<II", _U32, value)
    if isinstance(value, float):
        return _str(key) + struct.pack("<If", _F32, value)
    if isinstance(value, str):
        return _str(key) + struct.pack("<I", _STR) + _str(value)
    if isinstance(value, (list, tuple)):
        return _str(key) + struct.pack("<IIQ", _ARR, _I32, len(value)) + struct.pack(f"<{len(value)}i", *value)
    raise TypeError(key)


def write_gguf(path, metadata, tensors, alignment=32):
    """tensors: list of (name, type, ne tuple (ne[0] innermost), bytes)."""
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(metadata))
    head += b"".join(_kv(k, v) for k, v in metadata.items())
    infos = b""
    offset = 0
    blobs = []
    for name, type_, ne, data in tensors:
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        infos += _str(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
        infos += struct.pack("<IQ", type_, offset)
        blobs.append((offset, data))
        offset = (offset + data.size + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head + infos)
        pos = f.tell()
        f.write(b"\0" * ((alignment - pos % alignment) % alignment))
        base = f.tell()
        for off, data in blobs:
            f.seek(base + off)
            f.write(data.tobytes())


LAYER_NAMES = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate", "ffn_up",
               "ffn_down")


def llama_shapes(cfg):
    d, ff = cfg["n_embd"], cfg["n_ff"]
    q, kv = cfg["n_head"] * cfg["head_dim"], cfg["n_head_kv"] * cfg["head_dim"]
    return {"attn_norm": (1, d), "attn_q": (q, d), "attn_k": (kv, d), "attn_v": (kv, d), "attn_output": (d, q),
            "ffn_norm": (1, d), "ffn_gate": (ff, d), "ffn_up": (ff, d), "ffn_down": (d, ff)}


def random_llama_weights(cfg, seed, type_layers=Q8_0, type_embd=F32, tied=True, type_output=Q8_0, sigma=0.02):
    """Seeded N(0, sigma) matrices (quantized to their types) and unit norm weights.
    Returns {name: (type, array)}: F32 arrays as float32, others as GGUF bytes."""
    rng = np.random.default_rng(seed)
    shapes = llama_shapes(cfg)
    w = {"token_embd": (type_embd, encode(rng.standard_normal((cfg["n_vocab"], cfg["n_embd"]), dtype=np.float32)
                                          * np.float32(sigma), type_embd))}
    for l in range(cfg["n_layer"]):
        for n in LAYER_NAMES:
            rows, cols = shapes[n]
            if n.endswith("norm"):
                w[f"blk.{l}.{n}"] = (F32, np.ones(cols, np.float32))
            else:
                m = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma)
                w[f"blk.{l}.{n}"] = (type_layers, encode(m, type_layers))
    w["output_norm"] = (F32, np.ones(cfg["n_embd"], np.float32))
    if not tied:
        m = rng.standard_normal((cfg["n_vocab"], cfg["n_embd"]), dtype=np.float32) * np.float32(sigma)
        w["output"] = (type_output, encode(m, type_output))
    return w


def write_llama_gguf(path, cfg, weights, context_length, freq_factors=None):
    meta = {
        "general.architecture": "llama",
        "general.name": "synapse_b200 synthetic llama",
        "llama.block_count": cfg["n_layer"],
        "llama.context_length": context_length,
        "llama.embedding_length": cfg["n_embd"],
        "llama.feed_forward_length": cfg["n_ff"],
        "llama.attention.head_count": cfg["n_head"],
        "llama.attention.head_count_kv": cfg["n_head_kv"],
        "llama.rope.freq_base": float(cfg["rope_base"]),
        "llama.attention.layer_norm_rms_epsilon": float(cfg["rms_eps"]),
        "llama.rope.dimension_count": cfg["head_dim"],
        "llama.vocab_size": cfg["n_vocab"],
    }
    if cfg["head_dim"] != cfg["n_embd"] // cfg["n_head"]:
        meta["llama.attention.key_length"] = cfg["head_dim"]
        meta["llama.attention.value_length"] = cfg["head_dim"]
    shapes = llama_shapes(cfg)
    tensors = []

    def add(name, type_, rows, cols, arr):
        ne = (cols,) if rows == 1 and name.endswith("norm.weight") else (cols, rows)
        tensors.append((name, type_, ne, arr))

    t, a = weights["token_embd"]
    add("token_embd.weight", t, cfg["n_vocab"], cfg["n_embd"], a)
    t, a = weights["output_norm"]
    add("output_norm.weight", t, 1, cfg["n_embd"], a)
    if "output" in weights:
        t, a = weights["output"]
        add("output.weight", t, cfg["n_vocab"], cfg["n_embd"], a)
    if freq_factors is not None:
        tensors.append(("rope_freqs.weight", F32, (len(freq_factors),), np.asarray(freq_factors, np.float32)))
    for l in range(cfg["n_layer"]):
        for n in LAYER_NAMES:
            if f"blk.{l}.{n}" not in weights:
                continue
            t, a = weights[f"blk.{l}.{n}"]
            rows, cols = shapes[n]
            add(f"blk.{l}.{n}.weight", t, rows, cols, a)
    for name, (t, a) in weights.items():  # extra tensors (biases, ...) as 1-D rows
        if name.startswith("blk.") and name.rsplit(".", 1)[-1] not in LAYER_NAMES and name.endswith("bias"):
            tensors.append((name + ".weight" if not name.endswith("bias") else name, t, (np.asarray(a).size,), a))
    write_gguf(path, meta, tensors)
