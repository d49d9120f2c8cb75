"""CPU-side checks of the boundary: the C-ABI library loads and exports every
symbol include/synapse_b200.h declares; GGUF validation rejects hostile files
before any device work (gguf/reader.hpp I1-I7, tests/sdk/gguf_reader.cpp:208-219,
tests/sdk/llama_loader.cpp:230-411); the planner keeps P1-P3
(tests/sdk/graph_planner.cpp:54); the synthetic-model quantizers equal the
oracle's."""
import ctypes
import os
import struct
import subprocess

import numpy as np
import pytest

import oracle as orc
import synapse_b200 as syn
from synapse_b200 import model

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_loads_and_exports_every_declared_symbol():
    L = syn.lib()
    assert syn.lib().syn_build_info().decode().endswith("sm_100a")
    missing = [n for n in syn.exported_symbols() if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", syn.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert set(syn.exported_symbols()) <= exported


def test_library_is_sm100a_only():
    out = subprocess.run(["cuobjdump", "--list-elf", syn.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = {tok for tok in out.stdout.split() if "sm_" in tok}
    assert arches and all("sm_100a" in a for a in arches), arches


def test_status_strings():
    L = syn.lib()
    assert L.syn_status_string(0) == b"ok"
    assert L.syn_status_string(8) == b"out of range"


def test_size_queries_without_gpu():
    assert syn.q8_act_bytes(1, 4096) == 4096 + 256 + 512 + 512
    assert syn.q8_act_bytes(1, 33) == 0
    assert syn.weight_bytes(syn.Q4_0, 4096, 4096, syn.LAYOUT_GGUF) == 4096 * 128 * 18
    # planar rows: quants, then binary16 scales padded to 16 bytes
    assert syn.weight_bytes(syn.Q4_0, 4096, 4096, syn.LAYOUT_PLANAR) == 4096 * (128 * 16 + 128 * 2)
    assert syn.weight_bytes(syn.Q8_0, 3, 64, syn.LAYOUT_PLANAR) == 3 * (2 * 32 + 16)
    assert syn.weight_bytes(syn.Q4_0, 2, 288, syn.LAYOUT_PLANAR) == 2 * (9 * 16 + 32)
    assert syn.attention_scratch_bytes(1, 32, 8, 128, 4096) >= 32 * 4096 * 4


@pytest.mark.parametrize("ty", [model.Q4_0, model.Q8_0])
def test_model_quantizers_match_oracle(ty):
    rng = np.random.default_rng(ty)
    w = (rng.standard_normal((16, 512)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0
    w[1, :32] = np.arange(32) - 16.0
    assert np.array_equal(model.encode(w, ty), orc.quantize_weights(w, ty))


def _open(path):
    h = ctypes.c_void_p()
    return syn.lib().syn_session_open_gguf(str(path).encode(), 16, 0, ctypes.byref(h))


def tiny_cfg():
    return dict(n_layer=1, n_embd=64, n_ff=128, n_head=4, n_head_kv=2, head_dim=16, n_vocab=64, rms_eps=1e-5,
                rope_base=10000.0)


def test_gguf_rejects_hostile_files(tmp_path):
    cfg = tiny_cfg()
    w = model.random_llama_weights(cfg, seed=0)
    good = tmp_path / "good.gguf"
    model.write_llama_gguf(str(good), cfg, w, context_length=16)
    data = good.read_bytes()
    # every truncation is rejected as a format error (gguf_reader.cpp:208)
    for n in (0, 3, 4, 20, 24, 100, len(data) // 2, len(data) - 1):
        p = tmp_path / f"t{n}.gguf"
        p.write_bytes(data[:n])
        assert _open(p) == 7, n
    # bad magic / version
    p = tmp_path / "magic.gguf"
    p.write_bytes(b"GGUX" + data[4:])
    assert _open(p) == 7
    p = tmp_path / "ver.gguf"
    p.write_bytes(data[:4] + struct.pack("<I", 9) + data[8:])
    assert _open(p) == 7
    # an oversized tensor count is rejected before allocating (gguf_reader.cpp:219)
    p = tmp_path / "count.gguf"
    p.write_bytes(data[:8] + struct.pack("<Q", 1 << 60) + data[16:])
    assert _open(p) == 7
    assert _open(tmp_path / "missing.gguf") == 1


def test_loader_rejects_bad_models(tmp_path):
    cfg = tiny_cfg()
    w = model.random_llama_weights(cfg, seed=0)
    # missing tensor (llama_loader.cpp: missing_tensor)
    w2 = dict(w)
    del w2["blk.0.ffn_up"]
    p = tmp_path / "missing_up.gguf"
    model.write_llama_gguf(str(p), cfg, w2, context_length=16)
    assert _open(p) == 7
    # a bias the Llama graph does not have is rejected, not ignored (llama.hpp:438-451)
    w3 = dict(w)
    w3["blk.0.attn_q.bias"] = (model.F32, np.zeros(64, np.float32))
    p = tmp_path / "bias.gguf"
    model.write_llama_gguf(str(p), cfg, w3, context_length=16)
    assert _open(p) == 2
    # wrong architecture
    p = tmp_path / "arch.gguf"
    model.write_gguf(str(p), {"general.architecture": "gpt2"}, [])
    assert _open(p) == 2
    # an unsupported weight type (K-quants are outside this path)
    meta = {"general.architecture": "llama", "llama.block_count": 1, "llama.context_length": 16,
            "llama.embedding_length": 64, "llama.feed_forward_length": 128, "llama.attention.head_count": 4,
            "llama.attention.layer_norm_rms_epsilon": 1e-5}
    p = tmp_path / "kquant.gguf"
    model.write_gguf(str(p), meta, [("token_embd.weight", 12, (256, 64), np.zeros(64 * 144, np.uint8))])
    assert _open(p) in (2, 7)
    # missing epsilon
    meta2 = dict(meta)
    del meta2["llama.attention.layer_norm_rms_epsilon"]
    p = tmp_path / "eps.gguf"
    model.write_gguf(str(p), meta2, [("token_embd.weight", 0, (64, 64), np.zeros(64 * 64, np.float32))])
    assert _open(p) == 7


def test_planner_invariants(tmp_path):
    # the header-only planner on random interval sets: P1-P3 and reuse
    src = tmp_path / "t.cpp"
    src.write_text(r'''
#include "planner.hpp"
#include <cstdio>
#include <random>
int main() {
    std::mt19937 rng(42);
    for (int g = 0; g < 200; ++g) {
        std::vector<syn::plan::tensor> ts(1 + rng() % 60);
        for (auto& t : ts) {
            t.bytes = rng() % 5000;
            t.first = rng() % 40;
            t.last = t.first + rng() % 10;
        }
        auto r = syn::plan::place(ts, 256);
        if (!syn::plan::valid(ts, r, 256)) { std::printf("invalid %d\n", g); return 1; }
        if (r.arena_bytes > r.naive_bytes) { std::printf("no reuse %d\n", g); return 1; }
    }
    // disjoint lifetimes share memory
    std::vector<syn::plan::tensor> ts = {{1000, 0, 1}, {1000, 2, 3}};
    auto r = syn::plan::place(ts, 256);
    if (r.arena_bytes != 1024 || r.offset[0] != r.offset[1]) return 2;
    std::printf("ok\n");
    return 0;
}
''')
    exe = tmp_path / "t"
    subprocess.run(["g++", "-std=c++20", "-O1", "-I", os.path.join(ROOT, "synapse_b200", "csrc", "host"), str(src),
                    "-o", str(exe)], check=True)
    assert subprocess.run([str(exe)], capture_output=True, text=True).stdout.strip() == "ok"
