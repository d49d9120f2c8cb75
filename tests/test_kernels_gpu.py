"""Parity of the sm_100a kernels with the C oracle, through the C ABI.

Tolerances are the north star's: GEMV and attention outputs within 1e-3
relative L2 of the oracle on identical inputs (the same Q8_0 activations);
the Q8_0 quantizer, the F16 cache rows and argmax are bit-exact.
"""
import ctypes
import math

import numpy as np
import pytest

import oracle as orc

from .helpers import act_planes_host, blocks_to_planes, random_weights, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

syn = pytest.importorskip("synapse_b200")


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.cuda() if dtype is None else t.to(dtype).cuda()


# ---------------------------------------------------------------- Q8_0 quantizer

@pytest.mark.parametrize("n_tok,cols", [(1, 32), (1, 1024), (3, 4096), (16, 14336), (2, 288)])
def test_quantize_q8_0_bit_exact(n_tok, cols):
    rng = np.random.default_rng(cols + n_tok)
    x = rng.standard_normal((n_tok, cols), dtype=np.float32)
    x[0, :32] = 0.0                                     # an all-zero block: d = 0, id = 0
    if cols >= 64:
        x[0, 32:64] = np.arange(32, dtype=np.float32) - 16.0  # the known answer (round half away)
    act = syn.quantize_q8_0(dev(x))
    qs, dh, d, s = act_planes_host(act.cpu().numpy(), n_tok, cols)
    ref_qs, ref_dh = blocks_to_planes(orc.quantize_q8_0(x), n_tok, cols)
    assert np.array_equal(qs, ref_qs)
    assert np.array_equal(dh, ref_dh)
    assert np.array_equal(d, ref_dh.view(np.float16).astype(np.float32))
    assert np.array_equal(s, ref_qs.reshape(n_tok, -1, 32).astype(np.int32).sum(-1))
    blocks = syn.act_to_blocks(act, n_tok, cols).cpu().numpy()
    assert np.array_equal(blocks, orc.quantize_q8_0(x).reshape(-1))


def test_quantize_golden_activations(golden_dir):
    g = np.load(golden_dir + "/kernel_golden.npz")
    act = syn.quantize_q8_0(dev(g["x"][None, :]))
    assert np.array_equal(syn.act_to_blocks(act, 1, 1024).cpu().numpy(), g["q4_0_act"])


# ---------------------------------------------------------------- GEMV

def check_gemv(ty, layout, rows, cols, n_tok, seed, row_subset=None):
    rng = np.random.default_rng(seed)
    w = orc.quantize_weights(random_weights(rng, rows, cols), ty)
    x = rng.standard_normal((n_tok, cols), dtype=np.float32)
    wd = syn.upload_weight(ty, w, rows, cols, layout)
    act = syn.quantize_q8_0(dev(x))
    y = syn.gemv_q(ty, wd, layout, rows, cols, act, n_tok).cpu().numpy()
    blocks = orc.quantize_q8_0(x)
    rs = np.arange(rows) if row_subset is None else row_subset
    wsub = w.reshape(rows, -1)[rs]
    for t in range(n_tok):
        ref = orc.gemv_q8act(ty, wsub, len(rs), cols, blocks[t])
        assert rel_l2(y[t, rs], ref) < 1e-3
        # the kernel keeps the reference's float order: bit-identical to the oracle
        assert np.array_equal(y[t, rs].view(np.uint32), ref.view(np.uint32)), (t, rel_l2(y[t, rs], ref))
    return y


@pytest.mark.parametrize("ty", [syn.Q4_0, syn.Q8_0])
@pytest.mark.parametrize("layout", [syn.LAYOUT_PLANAR, syn.LAYOUT_GGUF])
@pytest.mark.parametrize("rows,cols,n_tok", [(8, 1024, 1), (288, 288, 1), (768, 288, 2), (300, 4096, 4),
                                             (64, 14336, 16), (1000, 2048, 3), (300, 4096, 20), (37, 1056, 9)])
def test_gemv_small(ty, layout, rows, cols, n_tok):
    check_gemv(ty, layout, rows, cols, n_tok, seed=rows * 7 + cols + n_tok)


@pytest.mark.parametrize("ty", [syn.Q4_0, syn.Q8_0])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)])
def test_gemv_sweep_shapes(ty, rows, cols):
    # the BASELINE sweep shapes at batch 1, 4 and 16; the oracle checks a row sample of the largest
    subset = None if rows * cols <= 14336 * 4096 else np.random.default_rng(1).choice(rows, 512, replace=False)
    check_gemv(ty, syn.LAYOUT_PLANAR, rows, cols, 1, seed=rows + cols, row_subset=subset)
    check_gemv(ty, syn.LAYOUT_PLANAR, rows, cols, 4, seed=rows + cols + 1, row_subset=subset)
    check_gemv(ty, syn.LAYOUT_PLANAR, rows, cols, 16, seed=rows + cols + 2, row_subset=subset)


@pytest.mark.parametrize("fmt,ty", [("q4_0", syn.Q4_0), ("q8_0", syn.Q8_0)])
def test_gemv_golden(golden_dir, fmt, ty):
    # kernels_golden.cpp:114: y within 1e-5 relative of ggml's vec_dot
    g = np.load(golden_dir + "/kernel_golden.npz")
    rows, cols = (int(v) for v in g[fmt + "_shape"])
    for layout in (syn.LAYOUT_PLANAR, syn.LAYOUT_GGUF):
        wd = syn.upload_weight(ty, g[fmt + "_w"], rows, cols, layout)
        y = syn.mul_mat(ty, wd, layout, rows, cols, dev(g["x"][None, :])).cpu().numpy()[0]
        yg = g[fmt + "_y"]
        assert np.all(np.abs(y - yg) <= 1e-5 * np.maximum(1.0, np.abs(yg)))


def test_gemv_residual_epilogue():
    rng = np.random.default_rng(11)
    rows, cols = 512, 1024
    w = orc.quantize_weights(random_weights(rng, rows, cols), syn.Q4_0)
    x = rng.standard_normal((1, cols), dtype=np.float32)
    r = rng.standard_normal((1, rows), dtype=np.float32)
    wd = syn.upload_weight(syn.Q4_0, w, rows, cols)
    act = syn.quantize_q8_0(dev(x))
    y0 = syn.gemv_q(syn.Q4_0, wd, syn.LAYOUT_PLANAR, rows, cols, act, 1).cpu().numpy()
    rd = dev(r)
    y1 = syn.gemv_q(syn.Q4_0, wd, syn.LAYOUT_PLANAR, rows, cols, act, 1, y=rd, residual=rd).cpu().numpy()
    assert np.array_equal(y1, (y0 + r).astype(np.float32))  # in place, one float add as op_add


# ---------------------------------------------------------------- fused GEMV (syn_gemv)

FUSED_SHAPES = [(288, 288, 1), (768, 288, 2), (6144, 4096, 1), (4096, 4096, 2), (4096, 14336, 1), (1000, 2048, 2)]


def same_bits(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


@pytest.mark.parametrize("ty", [syn.Q4_0, syn.Q8_0])
@pytest.mark.parametrize("rows,cols,n_tok", FUSED_SHAPES)
def test_gemv_fused_f32_input_matches_separate_ops(ty, rows, cols, n_tok):
    # gemm_prepare_rows inside the GEMV, then op_add: bit-identical to quantize -> gemv_q -> add
    rng = np.random.default_rng(rows + cols + n_tok)
    w = orc.quantize_weights(random_weights(rng, rows, cols), ty)
    x = dev(rng.standard_normal((n_tok, cols), dtype=np.float32))
    r = dev(rng.standard_normal((n_tok, rows), dtype=np.float32))
    wd = syn.upload_weight(ty, w, rows, cols)
    want = syn.gemv_q(ty, wd, syn.LAYOUT_PLANAR, rows, cols, syn.quantize_q8_0(x), n_tok, residual=r)
    got = syn.gemv_fused(ty, wd, rows, cols, x, in_mode=syn.IN_F32, residual=r)
    assert same_bits(got.cpu().numpy(), want.cpu().numpy())
    # and the oracle's separate ops on the host
    blocks = orc.quantize_q8_0(x.cpu().numpy())
    for t in range(n_tok):
        ref = orc.gemv_q8act(ty, w, rows, cols, blocks[t]) + r.cpu().numpy()[t]
        assert same_bits(got.cpu().numpy()[t], ref.astype(np.float32))


@pytest.mark.parametrize("ty", [syn.Q4_0, syn.Q8_0])
@pytest.mark.parametrize("rows,cols,n_tok", FUSED_SHAPES)
def test_gemv_fused_rms_norm_matches_separate_ops(ty, rows, cols, n_tok):
    # op_rms_norm -> op_matmul in one kernel (every CTA normalizes the row it needs)
    rng = np.random.default_rng(3 * rows + cols + n_tok)
    w = orc.quantize_weights(random_weights(rng, rows, cols), ty)
    xh = (2.0 * rng.standard_normal((n_tok, cols))).astype(np.float32)
    gh = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    x, gamma = dev(xh), dev(gh)
    wd = syn.upload_weight(ty, w, rows, cols)
    _, act = syn.rms_norm(x, gamma, 1e-5, want_f32=False, want_act=True)
    want = syn.gemv_q(ty, wd, syn.LAYOUT_PLANAR, rows, cols, act, n_tok)
    got = syn.gemv_fused(ty, wd, rows, cols, x, in_mode=syn.IN_RMSNORM, gamma=gamma, eps=1e-5)
    assert same_bits(got.cpu().numpy(), want.cpu().numpy())
    for t in range(n_tok):
        h = orc.rms_norm(xh[t], gh, np.float32(1e-5))
        ref = orc.gemv_q8act(ty, w, rows, cols, orc.quantize_q8_0(h[None, :])[0])
        assert same_bits(got.cpu().numpy()[t], ref)


def interleave_rows(a, b, rows, cols, ty):
    """Rows of a and b alternating (a0, b0, a1, b1, ...) as GGUF bytes."""
    rb = (cols // 32) * (18 if ty == syn.Q4_0 else 34)
    out = np.empty((2 * rows, rb), np.uint8)
    out[0::2] = a.reshape(rows, rb)
    out[1::2] = b.reshape(rows, rb)
    return out.reshape(-1)


@pytest.mark.parametrize("ty", [syn.Q4_0, syn.Q8_0])
@pytest.mark.parametrize("ff,cols,n_tok", [(384, 288, 1), (768, 288, 2), (14336, 4096, 1), (2048, 4096, 2)])
def test_gemv_fused_silu_pairs_matches_separate_ops(ty, ff, cols, n_tok):
    # gate and up rows interleaved in one matrix: rms_norm -> matmul -> silu(gate) * up in one kernel
    rng = np.random.default_rng(ff + cols + n_tok)
    wg = orc.quantize_weights(random_weights(rng, ff, cols), ty)
    wu = orc.quantize_weights(random_weights(rng, ff, cols), ty)
    xh = rng.standard_normal((n_tok, cols), dtype=np.float32)
    gh = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    x, gamma = dev(xh), dev(gh)
    wgu = syn.upload_weight(ty, interleave_rows(wg, wu, ff, cols, ty), 2 * ff, cols)
    assert syn.lib().syn_gemv_fusable(ty, syn.LAYOUT_PLANAR, 2 * ff, cols, n_tok, syn.OUT_SILU_PAIRS) == 1
    got = syn.gemv_fused(ty, wgu, 2 * ff, cols, x, in_mode=syn.IN_RMSNORM, gamma=gamma, eps=1e-5,
                         out_mode=syn.OUT_SILU_PAIRS).cpu().numpy()
    _, act = syn.rms_norm(x, gamma, 1e-5, want_f32=False, want_act=True)
    g = syn.gemv_q(ty, syn.upload_weight(ty, wg, ff, cols), syn.LAYOUT_PLANAR, ff, cols, act, n_tok)
    u = syn.gemv_q(ty, syn.upload_weight(ty, wu, ff, cols), syn.LAYOUT_PLANAR, ff, cols, act, n_tok)
    want, _ = syn.silu_mul(g, u, want_f32=True, want_act=False)
    assert got.shape == (n_tok, ff)
    assert same_bits(got, want.cpu().numpy())


def test_gemv_fused_rejects_what_it_cannot_take():
    rows, cols = 64, 512
    wd = syn.empty_bytes(syn.weight_bytes(syn.Q4_0, rows, cols, syn.LAYOUT_GGUF))
    x = torch.zeros(1, cols, device="cuda")
    a = syn.GemvArgs(syn.Q4_0, syn.LAYOUT_GGUF, rows, cols, 1, wd.data_ptr(), syn.IN_F32, None, x.data_ptr(),
                     None, 1e-5, syn.OUT_ROWS, x.data_ptr(), None)
    assert syn.lib().syn_gemv(ctypes.byref(a), syn._stream()) == 2  # SYN_ERR_UNSUPPORTED: fused modes need planar rows
    assert syn.lib().syn_gemv_fusable(syn.Q4_0, syn.LAYOUT_PLANAR, 63, cols, 1, syn.OUT_SILU_PAIRS) == 0
    assert syn.lib().syn_gemv_fusable(syn.Q4_0, syn.LAYOUT_PLANAR, rows, cols, 3, syn.OUT_ROWS) == 0
    a.layout, a.in_mode = syn.LAYOUT_PLANAR, syn.IN_RMSNORM  # rms_norm without gamma
    assert syn.lib().syn_gemv(ctypes.byref(a), syn._stream()) == 1


@pytest.mark.parametrize("ty", [syn.F32, syn.F16])
@pytest.mark.parametrize("rows,cols,n_tok", [(32000, 288, 1), (128, 64, 1), (100, 130, 3), (512, 4096, 2)])
def test_gemv_plain(ty, rows, cols, n_tok):
    rng = np.random.default_rng(rows + cols)
    wf = random_weights(rng, rows, cols, 0.05)
    w = orc.quantize_weights(wf, ty)
    x = rng.standard_normal((n_tok, cols), dtype=np.float32)
    wd = syn.upload_weight(ty, w, rows, cols)
    y = syn.gemv_f(ty, wd, rows, cols, dev(x)).cpu().numpy()
    ref = orc.gemm(ty, w, rows, cols, x)
    assert rel_l2(y, ref) < 1e-3
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), rel_l2(y, ref)


def test_repack_matches_upload():
    rng = np.random.default_rng(2)
    rows, cols = 64, 512
    w = orc.quantize_weights(random_weights(rng, rows, cols), syn.Q4_0)
    g = syn.upload_weight(syn.Q4_0, w, rows, cols, syn.LAYOUT_GGUF)
    p = syn.upload_weight(syn.Q4_0, w, rows, cols, syn.LAYOUT_PLANAR)
    p2 = syn.empty_bytes(syn.weight_bytes(syn.Q4_0, rows, cols))
    p2.zero_()
    syn.check(syn.lib().syn_repack_planar(syn.Q4_0, syn._ptr(g), rows, cols, syn._ptr(p2), syn._stream()), "repack")
    assert torch.equal(p.cpu(), p2.cpu())


def test_gemv_rejects_bad_args():
    with pytest.raises(syn.SynapseError):
        syn.gemv_q(syn.Q4_0, syn.empty_bytes(1024), syn.LAYOUT_PLANAR, 4, 33, syn.empty_bytes(1024), 1)
    with pytest.raises(syn.SynapseError):
        syn.gemv_q(5, syn.empty_bytes(1024), syn.LAYOUT_PLANAR, 4, 32, syn.empty_bytes(1024), 1)


# ---------------------------------------------------------------- attention

def assert_f16_rows_close(got, want):
    """Equal F16 rows except rare one-ulp flips of rotated values (an ulp of cos/sin)."""
    g = got.view(np.uint16).astype(np.int32)
    w = want.view(np.uint16).astype(np.int32)
    diff = np.abs(g - w)
    assert diff.max() <= 1, diff.max()
    assert np.count_nonzero(diff) <= max(2, diff.size // 1000), np.count_nonzero(diff)


def fill_f16(rng, shape):
    """N(0, 1) values as binary16 bits, made a row block at a time (bounded host memory)."""
    out = np.empty(shape, np.uint16)
    flat = out.reshape(-1)
    step = 1 << 24
    for i in range(0, flat.size, step):
        n = min(step, flat.size - i)
        flat[i:i + n] = rng.standard_normal(n, dtype=np.float32).astype(np.float16).view(np.uint16)
    return out


def attention_case(n_head, n_kv, hd, L, n_q, seed, base=10000.0, freq_factors=None, fill=True,
                   order=0, rope=True):
    """Caches filled with N(0,1) F16 rows 0..L-2 per query, then one fused step at pos = L-1.

    rope=True: the kernel rotates q and k (its cos/sin may differ from the C runtime's by an ulp, so the
    check is a tolerance); rope=False: q and k arrive rotated by the oracle, so both sides hold the same
    binary16 inputs and the reference order must give the oracle's bits exactly."""
    rng = np.random.default_rng(seed)
    max_ctx = L
    row = n_kv * hd
    kc = np.zeros((n_q, max_ctx * row), np.uint16)
    vc = np.zeros((n_q, max_ctx * row), np.uint16)
    if fill and L > 1:
        for b in range(n_q):
            kc[b, :(L - 1) * row] = fill_f16(rng, (L - 1) * row)
            vc[b, :(L - 1) * row] = fill_f16(rng, (L - 1) * row)
    q = rng.standard_normal((n_q, n_head * hd), dtype=np.float32)
    k = rng.standard_normal((n_q, row), dtype=np.float32)
    v = rng.standard_normal((n_q, row), dtype=np.float32)
    pos = np.full(n_q, L - 1, np.int32)
    ts = orc.rope_theta_scale(base, hd)
    scale = np.float32(1.0) / np.float32(math.sqrt(hd))
    qr = np.stack([orc.rope(q[b], hd, L - 1, ts, freq_factors) for b in range(n_q)])
    kr = np.stack([orc.rope(k[b], hd, L - 1, ts, freq_factors) for b in range(n_q)])
    kcd, vcd = dev(kc), dev(vc)
    ffd = dev(np.asarray(freq_factors, np.float32)) if freq_factors is not None else None
    out = syn.attention(dev(q if rope else qr), dev(k if rope else kr), dev(v), kcd, vcd, dev(pos), n_head, n_kv,
                        hd, max_ctx, ts, float(scale), cache_stride=max_ctx * row, freq_factors=ffd, rope=rope,
                        order=order).cpu().numpy()
    kc_after, vc_after = kcd.cpu().numpy(), vcd.cpu().numpy()
    for b in range(n_q):
        kref, vref = kc[b], vc[b]  # the oracle appends into the host copies
        ref = orc.attention(qr[b], kr[b], v[b], kref, vref, max_ctx, n_kv, hd, L - 1, n_head, scale)
        if rope:
            assert_f16_rows_close(kc_after[b], kref)  # rotated: cos/sin may differ from the C runtime by an ulp
        else:
            assert np.array_equal(kc_after[b], kref), "K row appended bit-exactly"
        assert np.array_equal(vc_after[b], vref), "V row appended bit-exactly"
        err = rel_l2(out[b], ref)
        assert err < 1e-3, (b, err)  # the north star's bound
        if order == syn.ORDER_REFERENCE and not rope:
            assert np.array_equal(out[b].view(np.uint32), ref.view(np.uint32)), (b, err)
        else:
            assert err < 1e-4, (b, err)
    return out


SMALL_SHAPES = [(32, 8, 128), (6, 6, 48), (4, 2, 16), (64, 8, 128), (8, 2, 32)]
SMALL_L = [1, 2, 33, 63, 64, 65, 256, 257, 287, 1000, 1025]


@pytest.mark.parametrize("n_head,n_kv,hd", SMALL_SHAPES)
@pytest.mark.parametrize("L", SMALL_L)
def test_attention_reference_order_bit_exact(n_head, n_kv, hd, L):
    # attention.hpp:185-244 in its own summation order at every length: the oracle's bits
    attention_case(n_head, n_kv, hd, L, 1, seed=L * 13 + hd + n_head, rope=False, order=syn.ORDER_REFERENCE)


@pytest.mark.parametrize("order", [0, 1])
@pytest.mark.parametrize("n_head,n_kv,hd", SMALL_SHAPES)
@pytest.mark.parametrize("L", SMALL_L)
def test_attention_small(n_head, n_kv, hd, L, order):
    attention_case(n_head, n_kv, hd, L, 1, seed=L * 13 + hd + n_head + 7, order=order)


# 32 query / 8 KV heads of 128, theta 500000, contexts 1k-32k, batch 1, 8 and 32
CONFIG3 = [(1024, 1), (1024, 8), (1024, 32), (4096, 1), (4096, 3), (4096, 8), (4096, 32), (16384, 1), (16384, 8),
           (32768, 1), (32768, 8)]


@pytest.mark.parametrize("L,n_q", CONFIG3)
def test_attention_config3_reference_order(L, n_q):
    attention_case(32, 8, 128, L, n_q, seed=L + n_q, base=500000.0, rope=False, order=syn.ORDER_REFERENCE)


@pytest.mark.parametrize("L,n_q", [(1024, 8), (4096, 1), (4096, 32), (16384, 1), (32768, 8)])
def test_attention_config3_split_order(L, n_q):
    attention_case(32, 8, 128, L, n_q, seed=L + n_q + 1, base=500000.0, order=syn.ORDER_SPLIT)


def test_attention_rope_in_kernel_reference_order():
    # the kernel's own rotation at 4k context (the session's path): within 1e-4 of the oracle
    attention_case(32, 8, 128, 4096, 2, seed=77, base=500000.0, rope=True, order=syn.ORDER_REFERENCE)


def test_attention_pos0_is_v():
    # kernels_attention.cpp:231-238: one position -> softmax is exactly 1 -> out is V's F16 value
    out = attention_case(4, 2, 16, 1, 2, seed=5)
    assert out is not None


def test_attention_freq_factors():
    attention_case(4, 2, 16, 16, 1, seed=3, freq_factors=np.arange(1, 9, dtype=np.float32))


def test_attention_growing_cache_matches_oracle_sequence():
    # a sequence decoded position by position through the fused kernel (kernels_attention.cpp:178-240)
    n_head, n_kv, hd, max_ctx = 4, 2, 16, 12
    row = n_kv * hd
    rng = np.random.default_rng(9)
    kcd = torch.zeros(max_ctx * row, dtype=torch.int16, device="cuda")
    vcd = torch.zeros(max_ctx * row, dtype=torch.int16, device="cuda")
    kc = np.zeros(max_ctx * row, np.uint16)
    vc = np.zeros(max_ctx * row, np.uint16)
    scale = np.float32(1.0) / np.float32(4.0)
    ts = orc.rope_theta_scale(10000.0, hd)
    for pos in range(max_ctx):
        q = rng.standard_normal(n_head * hd, dtype=np.float32)
        k = rng.standard_normal(row, dtype=np.float32)
        v = rng.standard_normal(row, dtype=np.float32)
        out = syn.attention(dev(q[None]), dev(k[None]), dev(v[None]), kcd, vcd, dev(np.array([pos], np.int32)),
                            n_head, n_kv, hd, max_ctx, ts, float(scale), cache_stride=0).cpu().numpy()[0]
        ref = orc.attention(orc.rope(q, hd, pos, ts), orc.rope(k, hd, pos, ts), v, kc, vc, max_ctx, n_kv, hd, pos,
                            n_head, scale)
        assert_f16_rows_close(kcd.cpu().numpy().view(np.uint16), kc)
        assert rel_l2(out, ref) < 1e-4


def test_rope_kv_append_then_attend_prefill():
    # prefill: n tokens of one sequence share the cache; append all, then attend (session.hpp:349-373)
    n_head, n_kv, hd, max_ctx, n = 8, 2, 64, 40, 5
    row = n_kv * hd
    rng = np.random.default_rng(21)
    q = rng.standard_normal((n, n_head * hd), dtype=np.float32)
    k = rng.standard_normal((n, row), dtype=np.float32)
    v = rng.standard_normal((n, row), dtype=np.float32)
    p0 = 7
    kc = np.zeros(max_ctx * row, np.uint16)
    vc = np.zeros(max_ctx * row, np.uint16)
    kc[:p0 * row] = rng.standard_normal(p0 * row, dtype=np.float32).astype(np.float16).view(np.uint16)
    vc[:p0 * row] = rng.standard_normal(p0 * row, dtype=np.float32).astype(np.float16).view(np.uint16)
    kcd, vcd = dev(kc), dev(vc)
    pos = dev(np.arange(p0, p0 + n, dtype=np.int32))
    ts = orc.rope_theta_scale(10000.0, hd)
    scale = float(np.float32(1.0) / np.float32(8.0))
    syn.rope_kv_append(dev(k), dev(v), kcd, vcd, pos, n_kv, hd, max_ctx, ts)
    out = syn.attention(dev(q), None, None, kcd, vcd, pos, n_head, n_kv, hd, max_ctx, ts, scale, cache_stride=0,
                        append=False).cpu().numpy()
    for i in range(n):
        orc.kv_append(orc.rope(k[i], hd, p0 + i, ts), v[i], kc, vc, max_ctx, n_kv, hd, p0 + i)
    assert_f16_rows_close(kcd.cpu().numpy(), kc)
    assert np.array_equal(vcd.cpu().numpy(), vc)
    for i in range(n):
        ref = orc.attend(orc.rope(q[i], hd, p0 + i, ts), kc, vc, max_ctx, n_kv, hd, p0 + i, n_head, np.float32(scale))
        assert rel_l2(out[i], ref) < 1e-4


def test_rope_matches_oracle():
    rng = np.random.default_rng(4)
    hd, nh = 128, 32
    x = rng.standard_normal((3, nh * hd), dtype=np.float32)
    pos = np.array([0, 4095, 32767], np.int32)
    ts = orc.rope_theta_scale(500000.0, hd)
    got = syn.rope(dev(x), dev(pos), nh, hd, ts).cpu().numpy()
    for i in range(3):
        ref = orc.rope(x[i], hd, int(pos[i]), ts)
        assert np.max(np.abs(got[i] - ref)) <= 1e-5 * (1 + pos[i])
        assert np.max(np.abs(got[i] - ref)) <= 4e-6 * np.max(np.abs(ref))


# ---------------------------------------------------------------- expf

def libm_exceptions():
    """The inputs the build step found where the host expf differs from the correctly rounded one."""
    import os
    import re
    path = os.path.join(os.path.dirname(syn.__file__), "_build", "libm_expf_exc.inc")
    with open(path) as f:
        text = f.read()
    body = text[text.index("{") + 1:text.rindex("}")]
    keys = np.array([int(v, 16) for v in re.findall(r"0x[0-9a-f]+", body)], dtype=np.uint32)
    assert keys.size == int(re.search(r"SYN_EXPF_EXC_COUNT (\d+)", text).group(1))
    return keys.view(np.float32)


def test_device_expf_is_the_host_libraries():
    # the reference calls std::exp on float (elementwise.hpp:79 silu, :188 softmax): the device expf must give
    # the host C library's bits, which are correctly rounded except on the inputs of the build step's table
    rng = np.random.default_rng(5)
    exc = libm_exceptions()
    assert exc.size > 1000  # glibc's expf: ~6e-4 of the inputs with |x| >= 2^-8
    x = np.concatenate([exc, rng.uniform(-40.0, 0.0, 1 << 22), rng.uniform(0.0, 88.7, 1 << 21),
                        rng.uniform(-0.01, 0.01, 1 << 20),
                        np.float32([0.0, -0.0, 1e-30, -1e-30, 88.72, -39.99, 0.5, -0.5])]).astype(np.float32)
    xd = dev(x)
    y, yr = torch.empty_like(xd), torch.empty_like(xd)
    syn.lib().syn_check_exp.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p]
    assert syn.lib().syn_check_exp(xd.data_ptr(), y.data_ptr(), yr.data_ptr(), x.size, syn._stream()) == 0
    got = y.cpu().numpy()
    want = orc.expf(x)
    bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
    assert bad.size == 0, (bad.size, x[bad[:5]], got[bad[:5]], want[bad[:5]])
    # and the exceptions really are where the host library is not the correctly rounded value
    cr = yr.cpu().numpy()[:exc.size]
    assert np.count_nonzero(cr.view(np.uint32) != want[:exc.size].view(np.uint32)) >= 0.99 * exc.size


def test_attention_rope_table_matches_inline_rope():
    n_head, n_kv, hd, L = 32, 8, 128, 700
    ts = 500000.0 ** (-2.0 / hd)
    g = torch.Generator(device="cpu").manual_seed(4)
    row = n_kv * hd
    kc = torch.randn(L * row, generator=g).half().view(torch.int16).cuda()
    vc = torch.randn(L * row, generator=g).half().view(torch.int16).cuda()
    q, k, v = (torch.randn(1, n, generator=g).cuda() for n in (n_head * hd, row, row))
    pos = torch.full((1,), L - 1, dtype=torch.int32).cuda()
    kc2, vc2 = kc.clone(), vc.clone()
    tab = syn.rope_table(L, hd, ts)
    a = syn.attention(q, k, v, kc, vc, pos, n_head, n_kv, hd, L, ts, 1 / math.sqrt(hd))
    b = syn.attention(q, k, v, kc2, vc2, pos, n_head, n_kv, hd, L, ts, 1 / math.sqrt(hd), rope_table=tab)
    assert torch.equal(a, b) and torch.equal(kc, kc2) and torch.equal(vc, vc2)


# ---------------------------------------------------------------- element-wise

@pytest.mark.parametrize("n_tok,cols", [(1, 4096), (2, 288), (3, 8192)])
def test_rms_norm_and_quant(n_tok, cols):
    rng = np.random.default_rng(cols)
    x = rng.standard_normal((n_tok, cols), dtype=np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    out, act = syn.rms_norm(dev(x), dev(gamma), 1e-5, want_f32=True, want_act=True)
    out = out.cpu().numpy()
    for t in range(n_tok):
        ref = orc.rms_norm(x[t], gamma, np.float32(1e-5))
        assert np.array_equal(out[t], ref)
    qs, dh, _, _ = act_planes_host(act.cpu().numpy(), n_tok, cols)
    ref_qs, ref_dh = blocks_to_planes(orc.quantize_q8_0(out), n_tok, cols)
    assert np.array_equal(qs, ref_qs) and np.array_equal(dh, ref_dh)


@pytest.mark.parametrize("n_tok,cols", [(1, 14336), (2, 768)])
def test_silu_mul_and_quant(n_tok, cols):
    rng = np.random.default_rng(cols)
    g = (3 * rng.standard_normal((n_tok, cols))).astype(np.float32)
    u = rng.standard_normal((n_tok, cols), dtype=np.float32)
    out, act = syn.silu_mul(dev(g), dev(u), want_f32=True, want_act=True)
    out = out.cpu().numpy()
    ref = np.stack([orc.silu(g[t]) * u[t] for t in range(n_tok)]).astype(np.float32)
    # exp rounded once from double; the C runtime's expf agrees but for rare last-ulp cases
    assert np.max(np.abs(out - ref) / np.maximum(np.abs(ref), 1e-30)) < 1e-6
    assert np.count_nonzero(out != ref) <= out.size // 1000
    qs, dh, _, _ = act_planes_host(act.cpu().numpy(), n_tok, cols)
    ref_qs, ref_dh = blocks_to_planes(orc.quantize_q8_0(out), n_tok, cols)
    assert np.array_equal(qs, ref_qs) and np.array_equal(dh, ref_dh)


@pytest.mark.parametrize("ty", [syn.F32, syn.F16, syn.Q4_0, syn.Q8_0])
@pytest.mark.parametrize("layout", [syn.LAYOUT_PLANAR, syn.LAYOUT_GGUF])
def test_embed(ty, layout):
    rng = np.random.default_rng(ty)
    rows, cols = 100, 256
    w = orc.quantize_weights(random_weights(rng, rows, cols, 0.5), ty)
    wd = syn.upload_weight(ty, w, rows, cols, layout)
    toks = np.array([0, 99, 17, 17], np.int32)
    got = syn.embed(ty, wd, layout, rows, cols, dev(toks)).cpu().numpy()
    ref = orc.dequantize(ty, w, rows, cols)[toks]
    assert np.array_equal(got, ref)


def test_argmax_ties_lowest_index():
    x = np.zeros((3, 128256), np.float32)
    x[0, 5] = x[0, 70000] = 3.0
    x[1, :] = -1.0
    x[2, 128255] = 1e-30
    got = syn.argmax(dev(x)).cpu().numpy()
    assert list(got) == [5, 0, 128255]
    rng = np.random.default_rng(0)
    y = rng.standard_normal((4, 32000), dtype=np.float32)
    assert list(syn.argmax(dev(y)).cpu().numpy()) == list(np.argmax(y, axis=1))


def test_add():
    a = np.arange(1000, dtype=np.float32)
    b = np.float32(0.1) * np.ones(1000, np.float32)
    assert np.array_equal(syn.add(dev(a), dev(b)).cpu().numpy(), a + b)
