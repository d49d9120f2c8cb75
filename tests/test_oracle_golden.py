"""Pins the C oracle to the reference's own golden vectors and known answers.

Mirrors the reference's checks (branes-ai/synapse tests/sdk):
kernels_golden.cpp:81-156, quant_golden.cpp:66-87, kernels_gemv.cpp:65-118,
kernels_attention.cpp:37-77 and :178-240, llama_golden.cpp:70-83.
"""
import math
import os

import numpy as np
import pytest

import oracle as orc

from .conftest import GOLDEN


def load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.mark.parametrize("fmt,ty", [("q4_0", orc.Q4_0), ("q8_0", orc.Q8_0)])
def test_kernel_golden(fmt, ty):
    g = load("kernel_golden.npz")
    x = g["x"]
    rows, cols = (int(v) for v in g[fmt + "_shape"])
    # activations bit-identical to ggml's reference quantizer (kernels_golden.cpp:103)
    act = orc.quantize_q8_0(x)
    assert np.array_equal(act, g[fmt + "_act"])
    # y within 1e-5 relative of ggml's vec_dot (kernels_golden.cpp:114)
    y = orc.gemv(ty, g[fmt + "_w"], rows, cols, x)
    yg = g[fmt + "_y"]
    assert np.all(np.abs(y - yg) <= 1e-5 * np.maximum(1.0, np.abs(yg)))
    # within the activation-rounding bound of the float reference (:117-133)
    w = orc.dequantize(ty, g[fmt + "_w"], rows, cols).astype(np.float64)
    xq = orc.dequantize(orc.Q8_0, act, 1, cols)[0].astype(np.float64)
    ref = w @ x.astype(np.float64)
    bound = np.abs(w) @ np.abs(x.astype(np.float64) - xq)
    slack = 1e-6 * (np.abs(w) @ np.abs(xq))
    assert np.all(np.abs(y - ref) <= bound + slack)


def q8_k_values(act, cols):
    """ggml block_q8_k bytes -> the float values they stand for (q * d)."""
    b = np.ascontiguousarray(act, np.uint8).reshape(-1, orc.Q8_K_BYTES)
    d = b[:, 0:4].copy().view(np.float32)
    qs = b[:, 4:260].copy().view(np.int8).astype(np.float32)
    return (qs * d).reshape(-1)[:cols]


@pytest.mark.parametrize("fmt,ty", [("q4_K", orc.Q4_K), ("q6_K", orc.Q6_K)])
def test_kernel_golden_k_quants(fmt, ty):
    # kernels_golden.cpp:81-156 for the K formats: Q8_K activations
    g = load("kernel_golden.npz")
    x = g["x"]
    rows, cols = (int(v) for v in g[fmt + "_shape"])
    act = orc.quantize_q8_k(x)
    assert np.array_equal(act, g[fmt + "_act"])  # bit-identical, bsums included (:103)
    y = orc.gemv(ty, g[fmt + "_w"], rows, cols, x)
    assert np.array_equal(y.view(np.uint32), orc.gemv_q8k(ty, g[fmt + "_w"], rows, cols, act).view(np.uint32))
    yg = g[fmt + "_y"]
    assert np.all(np.abs(y - yg) <= 1e-5 * np.maximum(1.0, np.abs(yg)))  # (:114)
    w = orc.dequantize(ty, g[fmt + "_w"], rows, cols).astype(np.float64)
    xq = q8_k_values(act, cols).astype(np.float64)
    ref = w @ x.astype(np.float64)
    bound = np.abs(w) @ np.abs(x.astype(np.float64) - xq)
    slack = 1e-6 * (np.abs(w) @ np.abs(xq)) + 1e-6
    assert np.all(np.abs(y - ref) <= bound + slack)  # (:117-133)


def test_q8_k_edge_cases():
    # quant/q8.hpp:73-104: an all-zero block is all zero (bsums too); the
    # element of largest magnitude maps to -127 (never -128, :88), and of two
    # with equal magnitude the first one is that element
    x = np.zeros(512, np.float32)
    x[256 + 5], x[256 + 9] = -2.0, 2.0
    x[256 + 7] = 0.5
    b = orc.quantize_q8_k(x).reshape(2, orc.Q8_K_BYTES)
    assert not b[0].any()
    d = b[1, 0:4].copy().view(np.float32)[0]
    qs = b[1, 4:260].copy().view(np.int8)
    bsums = b[1, 260:292].copy().view(np.int16)
    assert d == np.float32(1.0) / (np.float32(-127.0) / np.float32(-2.0))
    assert qs[5] == -127 and qs[9] == 127 and qs[7] == 32  # iscale 63.5: 0.5 -> 31.75 -> 32
    assert bsums[0] == -127 + 127 + 32 and not bsums[1:].any()
    # iscale 1: halves round to even
    y = np.zeros(256, np.float32)
    y[0] = -127.0
    y[1], y[2], y[3] = 2.5, 3.5, -2.5
    q = orc.quantize_q8_k(y)[4:260].view(np.int8)
    assert q[0] == -127 and q[1] == 2 and q[2] == 4 and q[3] == -2


@pytest.mark.parametrize("fmt,ty", [("f16", orc.F16), ("q4_0", orc.Q4_0), ("q8_0", orc.Q8_0),
                                    ("q4_k", orc.Q4_K), ("q6_k", orc.Q6_K)])
def test_quant_golden_dequantize(fmt, ty):
    g = load("quant_golden.npz")
    rows, cols = (int(v) for v in g[fmt + "_shape"])
    got = orc.dequantize(ty, g[fmt + "_q"], rows, cols).reshape(-1)
    assert np.array_equal(got.view(np.uint32), g[fmt + "_expected"].view(np.uint32))


def test_fp16_roundtrip_all_patterns():
    # kernels_gemv.cpp:65-77
    lib = orc.lib()
    bad = 0
    for h in range(0, 0x10000, 7):
        f = lib.orc_fp16_to_float(h)
        if math.isnan(f):
            continue
        bad += lib.orc_float_to_fp16(f) != h
    assert bad == 0


def test_fp16_rne_against_numpy():
    # numpy's float16 cast is an independent round-to-nearest-even (kernels_gemv.cpp:79)
    rng = np.random.default_rng(7)
    bits = rng.integers(0, 0x477FEFFF, 20000, dtype=np.uint32) | (rng.integers(0, 2, 20000, dtype=np.uint32) << 31)
    f = bits.view(np.float32)
    ours = np.array([orc.float_to_fp16(v) for v in f], dtype=np.uint16)
    assert np.array_equal(ours, f.astype(np.float16).view(np.uint16))
    assert orc.float_to_fp16(1.0 + 2.0 ** -11) == 0x3C00
    assert orc.float_to_fp16(1.0 + 3 * 2.0 ** -11) == 0x3C02
    assert orc.float_to_fp16(65520.0) == 0x7C00
    assert orc.float_to_fp16(2.0 ** -25) == 0x0000


def test_q8_0_known_answer():
    # kernels_gemv.cpp:107-118
    x = np.arange(32, dtype=np.float32) - 16.0
    b = orc.quantize_q8_0(x)
    d = int(b[0]) | (int(b[1]) << 8)
    qs = b[2:].view(np.int8)
    assert d == orc.float_to_fp16(np.float32(16.0) / np.float32(127.0))
    assert qs[0] == -127 and qs[16] == 0 and qs[24] == 64


def test_q4_0_quantizer_matches_gguf_py_restatement():
    # ggml quantize_row_q4_0_ref as restated by gguf-py 0.19.0 Q4_0.quantize_blocks, in numpy
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((4, 256)) * 0.02).astype(np.float32)
    ours = orc.quantize_q4_0(w).reshape(-1, 18)
    blocks = w.reshape(-1, 32)
    imax = np.abs(blocks).argmax(axis=-1)[:, None]
    mx = np.take_along_axis(blocks, imax, axis=-1)
    d = mx / np.float32(-8)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    qs = np.trunc(blocks * inv + np.float32(8.5)).astype(np.uint8).clip(0, 15)
    packed = qs[:, :16] | (qs[:, 16:] << 4)
    ref = np.concatenate([d.astype(np.float16).view(np.uint8), packed], axis=1)
    assert np.array_equal(ours, ref)


def test_rope_against_double():
    # kernels_attention.cpp:37-77: tolerance 1e-5 * (1 + pos)
    rng = np.random.default_rng(1)
    hd = 64
    x = rng.standard_normal(4 * hd).astype(np.float32)
    ts = orc.rope_theta_scale(10000.0, hd)
    for pos in (0, 1, 17, 1000, 4095):
        out = orc.rope(x, hd, pos, ts)
        ref = np.empty_like(x, dtype=np.float64)
        for i in range(hd // 2):
            th = pos * (10000.0 ** (-2.0 * i / hd))
            c, s = math.cos(th), math.sin(th)
            for h in range(0, x.size, hd):
                x0, x1 = float(x[h + 2 * i]), float(x[h + 2 * i + 1])
                ref[h + 2 * i] = x0 * c - x1 * s
                ref[h + 2 * i + 1] = x0 * s + x1 * c
        assert np.max(np.abs(out - ref)) < 1e-5 * (1 + pos)


def test_attention_gqa_growing_cache():
    # kernels_attention.cpp:178-240
    n_heads, n_kv, hd, max_ctx = 4, 2, 16, 12
    row = n_kv * hd
    scale = np.float32(1.0) / np.float32(math.sqrt(hd))
    rng = np.random.default_rng(9)
    kc = np.zeros(max_ctx * row, np.uint16)
    vc = np.zeros(max_ctx * row, np.uint16)
    ks, vs = [], []
    r16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float64)
    for pos in range(max_ctx):
        q = rng.standard_normal(n_heads * hd).astype(np.float32)
        ks.append(rng.standard_normal(row).astype(np.float32))
        vs.append(rng.standard_normal(row).astype(np.float32))
        out = orc.attention(q, ks[-1], vs[-1], kc, vc, max_ctx, n_kv, hd, pos, n_heads, scale)
        assert np.array_equal(kc[pos * row:(pos + 1) * row], ks[-1].astype(np.float16).view(np.uint16))
        assert np.array_equal(vc[pos * row:(pos + 1) * row], vs[-1].astype(np.float16).view(np.uint16))
        for h in range(n_heads):
            g = h // (n_heads // n_kv)
            p = np.array([np.dot(r16(q[h * hd:(h + 1) * hd]), r16(ks[t][g * hd:(g + 1) * hd])) * float(scale)
                          for t in range(pos + 1)])
            p = np.exp(p - p.max())
            p /= p.sum()
            ref = sum(p[t] * r16(vs[t][g * hd:(g + 1) * hd]) for t in range(pos + 1))
            assert np.max(np.abs(out[h * hd:(h + 1) * hd] - ref)) < 2e-3
        if pos == 0:
            for h in range(n_heads):
                assert np.array_equal(out[h * hd:(h + 1) * hd], r16(vs[0][h // 2 * hd:(h // 2 + 1) * hd]))


def tiny_f32_model():
    g = load("llama_tiny_f32.npz")
    m = lambda k: int(g["meta.llama." + k])
    cfg = dict(n_layer=m("block_count"), n_embd=m("embedding_length"), n_ff=m("feed_forward_length"),
               n_head=m("attention.head_count"), n_head_kv=m("attention.head_count_kv"),
               n_vocab=m("vocab_size"), rms_eps=float(np.float32(g["meta.llama.attention.layer_norm_rms_epsilon"])),
               rope_base=float(g["meta.llama.rope.freq_base"]))
    cfg["head_dim"] = cfg["n_embd"] // cfg["n_head"]
    weights = {}
    for k in g.files:
        if k.startswith("t."):
            name = k[2:].replace(".weight", "")
            weights[name] = (orc.F32, g[k])
    return cfg, weights, g["t.rope_freqs.weight"], g["golden.tokens"], g["golden.logits"]


def test_llama_tiny_f32_golden():
    # llama_golden.cpp:70-83: every position within 1e-4 relative max of llama.cpp's logits
    cfg, weights, ff, tokens, golden = tiny_f32_model()
    m = orc.Llama(cfg, weights, max_ctx=len(tokens), freq_factors=ff)
    for i, tok in enumerate(tokens):
        logits = m.step(int(tok), i)
        ref = golden[i]
        rel = np.max(np.abs(logits.astype(np.float64) - ref)) / np.max(np.abs(ref))
        assert rel < 1e-4, (i, rel)
        assert int(np.argmax(logits)) == int(np.argmax(ref))


def test_oracle_thread_invariance():
    # D1 (llama_threads.cpp:32-58): results do not depend on the thread count
    rng = np.random.default_rng(5)
    rows, cols = 300, 1024
    w = orc.quantize_q4_0((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
    x = rng.standard_normal(cols).astype(np.float32)
    orc.set_threads(1)
    y1 = orc.gemv(orc.Q4_0, w, rows, cols, x)
    orc.set_threads(4)
    y4 = orc.gemv(orc.Q4_0, w, rows, cols, x)
    orc.set_threads(1)
    assert np.array_equal(y1.view(np.uint32), y4.view(np.uint32))
