"""Extract the reference's golden vectors for this path into tests/golden/*.npz.

Runs where the reference checkout exists (pass its root as argv[1]); the
committed .npz files are what the tests read, so nothing at test time needs
the reference. Reads the GGUF fixtures with gguf-py (installed in the image).

Sources, all inside branes-ai/synapse v0.15.12 tests/data/ (generated there
by the reference's scripts/gen_*_fixture.py from ggml / llama.cpp @ e6f2ec01f):

- kernel_golden.gguf : x (1024 f32, N(0,1)), <fmt>.w (8 x 1024 weights),
  <fmt>.act (ggml's Q8_0 activation blocks), <fmt>.y (ggml's vec_dot);
  used by tests/sdk/kernels_golden.cpp:81-156.  Q4_0, Q8_0 (Q8_0 activations)
  and Q4_K, Q6_K (Q8_K activations) entries.
- quant_golden.gguf  : <fmt>.q blocks and gguf-py's dequantized .expected;
  used by tests/sdk/quant_golden.cpp:66-87.  F16, Q4_0, Q8_0, Q4_K, Q6_K entries.
- llama_tiny_f32.gguf + llama_tiny_f32_golden.gguf : a 2-layer all-F32 Llama
  (d 64, ff 128, 4 heads / 2 KV, hd 16, vocab 128, rope_freqs) and
  llama.cpp's logits after each of 16 tokens; tests/sdk/llama_golden.cpp:70-83.
"""
import os
import sys

import numpy as np


def raw(t):
    """The tensor's bytes exactly as stored (GGUF row-major)."""
    return np.ascontiguousarray(t.data).view(np.uint8).reshape(-1).copy()


def tensors(reader):
    return {t.name: t for t in reader.tensors}


def main(ref_root):
    import gguf

    data = os.path.join(ref_root, "tests", "data")
    out = os.path.dirname(os.path.abspath(__file__))

    # kernel_golden
    r = gguf.GGUFReader(os.path.join(data, "kernel_golden.gguf"))
    t = tensors(r)
    kg = {"x": np.asarray(t["x"].data, dtype=np.float32).reshape(-1).copy()}
    for fmt in ("q4_0", "q8_0", "q4_K", "q6_K"):
        w = t[fmt + ".w"]
        kg[fmt + "_w"] = raw(w)
        kg[fmt + "_shape"] = np.array([int(w.shape[1]), int(w.shape[0])], dtype=np.int64)  # rows, cols
        kg[fmt + "_act"] = raw(t[fmt + ".act"])
        kg[fmt + "_y"] = np.asarray(t[fmt + ".y"].data, dtype=np.float32).reshape(-1).copy()
    np.savez_compressed(os.path.join(out, "kernel_golden.npz"), **kg)

    # quant_golden
    r = gguf.GGUFReader(os.path.join(data, "quant_golden.gguf"))
    t = tensors(r)
    qg = {}
    for fmt in ("f16", "q4_0", "q8_0", "q4_k", "q6_k"):
        q = t[fmt + ".q"]
        qg[fmt + "_q"] = raw(q)
        qg[fmt + "_shape"] = np.array([int(q.shape[1]), int(q.shape[0])], dtype=np.int64)
        qg[fmt + "_expected"] = np.asarray(t[fmt + ".expected"].data, dtype=np.float32).reshape(-1).copy()
    np.savez_compressed(os.path.join(out, "quant_golden.npz"), **qg)

    # llama_tiny_f32 model + golden logits
    r = gguf.GGUFReader(os.path.join(data, "llama_tiny_f32.gguf"))
    lt = {}
    for k, f in r.fields.items():
        if k.startswith("llama."):
            lt["meta." + k] = np.array(f.contents())
    for tt in r.tensors:
        lt["t." + tt.name] = np.asarray(tt.data, dtype=np.float32).reshape(-1).copy()
        lt["shape." + tt.name] = np.array([int(s) for s in tt.shape], dtype=np.int64)
    g = gguf.GGUFReader(os.path.join(data, "llama_tiny_f32_golden.gguf"))
    lt["golden.tokens"] = np.array(g.fields["synapse.golden.tokens"].contents(), dtype=np.uint32)
    gt = tensors(g)
    lt["golden.logits"] = np.asarray(gt["logits"].data, dtype=np.float32).reshape(len(lt["golden.tokens"]), -1).copy()
    np.savez_compressed(os.path.join(out, "llama_tiny_f32.npz"), **lt)
    print("wrote", sorted(os.listdir(out)))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <checkout of the reference>")
    main(sys.argv[1])
