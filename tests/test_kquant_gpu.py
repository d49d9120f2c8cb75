"""Q4_K / Q6_K rows on Q8_K activations: the sm_100a kernels against the C
oracle, through the C ABI.

The Q8_K quantizer is bit-exact (ggml's block_q8_k bytes, sub-block sums
included), and so is every GEMV output: the kernel keeps the reference's
order of float operations (exact integer super-block dots, an fma chain per
chunk of four super-blocks, chunk sums in order). The reference's golden
vectors (kernels_golden.cpp:81-156 for q4_K / q6_K) are checked as there:
activations bit-identical, y within 1e-5 relative of ggml's vec_dot.
"""
import numpy as np
import pytest

import oracle as orc

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

syn = pytest.importorskip("synapse_b200")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def q8k_blocks(x):
    n_tok, cols = x.shape
    act = syn.quantize_q8_k(dev(x))
    return act, syn.q8k_act_to_blocks(act, n_tok, cols).cpu().numpy().reshape(n_tok, -1)


@pytest.mark.parametrize("n_tok,cols", [(1, 256), (1, 1024), (3, 4096), (9, 14336), (2, 1280)])
def test_quantize_q8_k_bit_exact(n_tok, cols):
    rng = np.random.default_rng(cols + n_tok)
    x = rng.standard_normal((n_tok, cols), dtype=np.float32)
    x[0, :256] = 0.0                                  # an all-zero block
    if cols >= 512:
        x[0, 256:512] = 0.25
        x[0, 256 + 7], x[0, 256 + 200] = -127.0, 127.0  # equal magnitudes: the first sets the sign (iscale 1)
        x[0, 256 + 9], x[0, 256 + 10] = 2.5, -3.5         # halves round to even
    _, got = q8k_blocks(x)
    assert np.array_equal(got, orc.quantize_q8_k(x))


def test_quantize_q8_k_golden(golden_dir):
    g = np.load(golden_dir + "/kernel_golden.npz")
    _, got = q8k_blocks(g["x"][None, :])
    assert np.array_equal(got[0], g["q4_K_act"])
    assert np.array_equal(got[0], g["q6_K_act"])


@pytest.mark.parametrize("fmt,ty", [("q4_K", syn.Q4_K), ("q6_K", syn.Q6_K)])
def test_gemv_k_golden(golden_dir, fmt, ty):
    g = np.load(golden_dir + "/kernel_golden.npz")
    rows, cols = (int(v) for v in g[fmt + "_shape"])
    wd = syn.upload_weight(ty, g[fmt + "_w"], rows, cols, syn.LAYOUT_PLANAR)
    act, blocks = q8k_blocks(g["x"][None, :])
    y = syn.gemv_q(ty, wd, syn.LAYOUT_PLANAR, rows, cols, act, 1).cpu().numpy()[0]
    assert same_bits(y, orc.gemv_q8k(ty, g[fmt + "_w"], rows, cols, blocks[0]))
    yg = g[fmt + "_y"]
    assert np.all(np.abs(y - yg) <= 1e-5 * np.maximum(1.0, np.abs(yg)))


K_SHAPES = [(8, 256, 1), (37, 1280, 1), (300, 4096, 3), (64, 14336, 2), (129, 768, 9), (4096, 4096, 1),
            (1000, 14336, 16)]


@pytest.mark.parametrize("kernel", ["lane", "warp"])
@pytest.mark.parametrize("ty", [syn.Q4_K, syn.Q6_K])
@pytest.mark.parametrize("rows,cols,n_tok", K_SHAPES)
def test_gemv_k_matches_oracle(ty, rows, cols, n_tok, kernel, monkeypatch):
    # lane: one lane per super-block (the default); warp: the warp-per-row kernel that
    # rows too wide for the lane kernel's shared memory take
    if kernel == "warp":
        monkeypatch.setenv("SYN_GEMV_K_WARP", "1")
    rng = np.random.default_rng(rows * 7 + cols + n_tok)
    w = orc.random_k_blocks(ty, rows, cols, seed=rows + cols)
    x = rng.standard_normal((n_tok, cols), dtype=np.float32)
    layouts = [syn.LAYOUT_PLANAR] + ([syn.LAYOUT_GGUF] if ty == syn.Q4_K else [])
    act, blocks = q8k_blocks(x)
    want = np.stack([orc.gemv_q8k(ty, w, rows, cols, blocks[t]) for t in range(n_tok)])
    for layout in layouts:
        wd = syn.upload_weight(ty, w, rows, cols, layout)
        y = syn.gemv_q(ty, wd, layout, rows, cols, act, n_tok).cpu().numpy()
        assert same_bits(y, want), (layout, np.flatnonzero(y.view(np.uint32) != want.view(np.uint32))[:8])
    # the float path: x quantized by the oracle as the reference's gemv does it
    assert same_bits(want[0], orc.gemv(ty, w, rows, cols, x[0]))


@pytest.mark.parametrize("ty", [syn.Q4_K, syn.Q6_K])
def test_gemv_k_residual(ty):
    rows, cols, n_tok = 512, 2048, 3
    rng = np.random.default_rng(5)
    w = orc.random_k_blocks(ty, rows, cols, seed=11)
    x = rng.standard_normal((n_tok, cols), dtype=np.float32)
    res = rng.standard_normal((n_tok, rows), dtype=np.float32)
    act, blocks = q8k_blocks(x)
    wd = syn.upload_weight(ty, w, rows, cols, syn.LAYOUT_PLANAR)
    y = syn.gemv_q(ty, wd, syn.LAYOUT_PLANAR, rows, cols, act, n_tok, residual=dev(res)).cpu().numpy()
    want = np.stack([orc.gemv_q8k(ty, w, rows, cols, blocks[t]) for t in range(n_tok)]) + res
    assert same_bits(y, want)


def test_q6_k_upload_through_staging_matches_device_repack():
    # 400 rows of 56 super-blocks (4.7 MB) take two passes of the 4 MiB staging buffer
    rows, cols = 400, 14336
    w = orc.random_k_blocks(syn.Q6_K, rows, cols, seed=3)
    up = syn.upload_weight(syn.Q6_K, w, rows, cols, syn.LAYOUT_PLANAR)
    src = dev(w.reshape(-1))
    dst = syn.empty_bytes(syn.weight_bytes(syn.Q6_K, rows, cols, syn.LAYOUT_PLANAR))
    syn.check(syn.lib().syn_repack_planar(syn.Q6_K, syn._ptr(src), rows, cols, syn._ptr(dst), syn._stream()),
              "syn_repack_planar")
    assert torch.equal(up, dst)
    # the planar row: 56 blocks of 208 bytes, then 56 scales
    pitch = syn.weight_bytes(syn.Q6_K, 1, cols, syn.LAYOUT_PLANAR)
    assert pitch == (56 * 208 + 112 + 15) // 16 * 16
    host = up.cpu().numpy().reshape(rows, pitch)
    blocks = w.reshape(rows, 56, 210)
    assert np.array_equal(host[:, :56 * 208].reshape(rows, 56, 208), blocks[:, :, :208])
    assert np.array_equal(host[:, 56 * 208:56 * 210].reshape(rows, 56, 2), blocks[:, :, 208:])


def test_gemv_k_rejects_bad_args():
    w = syn.empty_bytes(syn.weight_bytes(syn.Q6_K, 8, 256, syn.LAYOUT_PLANAR))
    act = syn.empty_bytes(syn.q8k_act_bytes(1, 256))
    y = torch.empty(8, dtype=torch.float32, device="cuda")
    L = syn.lib()
    # Q6_K in GGUF layout: 210-byte blocks are not 16-byte aligned
    assert L.syn_gemv_q(syn.Q6_K, syn._ptr(w), syn.LAYOUT_GGUF, 8, 256, syn._ptr(act), 1, syn._ptr(y), None,
                        syn._stream()) == 2
    # cols not a multiple of 256
    assert L.syn_gemv_q(syn.Q4_K, syn._ptr(w), syn.LAYOUT_PLANAR, 8, 288, syn._ptr(act), 1, syn._ptr(y), None,
                        syn._stream()) == 1
    assert L.syn_q8k_act_bytes(1, 288) == 0
    assert L.syn_weight_bytes(syn.Q4_K, 8, 288, syn.LAYOUT_GGUF) == 0


# ---------------------------------------------------------------- a K-format model end to end

KM_CFG = dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=64, n_vocab=512, rms_eps=1e-5,
              rope_base=10000.0)
KM_TYPES = {"attn_q": orc.Q4_K, "attn_k": orc.Q4_K, "attn_v": orc.Q6_K, "attn_output": orc.Q4_K,
            "ffn_gate": orc.Q4_K, "ffn_up": orc.Q4_K, "ffn_down": orc.Q6_K}


def q4_k_m_model(cfg, seed=21):
    """A Q4_K_M-style mix (Q4_K matrices, Q6_K for V, down and the head) with one
    Q8_0 matrix in the second layer, F32 embedding and norms."""
    from synapse_b200 import model
    rng = np.random.default_rng(seed)
    shapes = model.llama_shapes(cfg)
    w = {"token_embd": (model.F32, rng.standard_normal((cfg["n_vocab"], cfg["n_embd"]), dtype=np.float32) * 0.02)}
    for l in range(cfg["n_layer"]):
        for n in model.LAYER_NAMES:
            rows, cols = shapes[n]
            if n.endswith("norm"):
                w[f"blk.{l}.{n}"] = (model.F32, np.ones(cols, np.float32))
            elif l == 1 and n == "attn_k":
                w[f"blk.{l}.{n}"] = (model.Q8_0, model.encode(rng.standard_normal((rows, cols), dtype=np.float32)
                                                              * np.float32(0.02), model.Q8_0))
            else:
                w[f"blk.{l}.{n}"] = (KM_TYPES[n], orc.random_k_blocks(KM_TYPES[n], rows, cols, seed + l * 16 +
                                                                      len(n), log2_scale=(-18, -14)))
    w["output_norm"] = (model.F32, np.ones(cfg["n_embd"], np.float32))
    w["output"] = (orc.Q6_K, orc.random_k_blocks(orc.Q6_K, cfg["n_vocab"], cfg["n_embd"], seed + 99,
                                                 log2_scale=(-16, -12)))
    return w


def test_k_model_session_matches_oracle_bit_for_bit(tmp_path):
    from synapse_b200 import model
    cfg = KM_CFG
    w = q4_k_m_model(cfg)
    p = tmp_path / "q4_k_m.gguf"
    model.write_llama_gguf(str(p), cfg, w, context_length=64)
    sess = syn.Session.open(p, max_ctx=64)
    ref = orc.Llama(cfg, w, max_ctx=64)
    tok = 7
    for pos in range(40):  # one attention chunk: every op in the reference's order, so logits are identical
        got, nxt = sess.step(tok, pos)
        want = ref.step(tok, pos)
        assert np.all(np.isfinite(want)) and np.std(want) > 0
        assert same_bits(got, want), (pos, float(np.max(np.abs(got - want))))
        assert nxt == int(np.argmax(want))
        tok = nxt
    # the K matrices read back from the device as the file's GGUF bytes
    for name in ("blk.0.attn_q.weight", "blk.0.attn_v.weight", "blk.1.ffn_down.weight", "output.weight"):
        ty, rows, cols, data = sess.weight(name)
        key = name[:-len(".weight")]
        assert ty == w[key][0]
        assert np.array_equal(data, np.ascontiguousarray(w[key][1]).reshape(-1))
    sess.close()
