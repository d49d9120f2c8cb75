"""Kernel microbenchmarks of the decode path (BASELINE configs 2 and 3).

  python -m synapse_b200.kernel_bench gemv [--type q4_0|q8_0] [--rows R --cols C] [--batch N] [--iters I]
  python -m synapse_b200.kernel_bench attention [--ctx L] [--batch B] [--iters I]

gemv: the quantized GEMV (syn_gemv_q, planar weights) at the sweep shapes
(4096x4096, 14336x4096, 4096x14336, 128256x4096) and batches 1/4/16, weights
N(0, 0.02) quantized on the device; enough weight copies rotate that their
total exceeds twice the 126 MB L2, so every launch streams from HBM.
attention: the fused RoPE + F16 append + split-KV attention (syn_attention)
with H 32 / KV 8 / hd 128, theta 500000, caches of N(0,1) F16 at context L,
batch 1/8/32.
Each line: JSON with the average CUDA-event time per launch, the algorithmic
bytes per launch and GB/s.
"""
import argparse
import ctypes
import json
import math

import numpy as np

from . import LAYOUT_PLANAR, Q4_0, Q8_0, _ptr, _stream, attention, attention_scratch_bytes, check, empty_bytes, \
    gemv_q, lib, q8_act_bytes, quantize_q8_0, weight_bytes

L2_BYTES = 126 << 20
TYPES = {"q4_0": Q4_0, "q8_0": Q8_0}


def _fill_random(type_, rows, cols, dst, seed):
    from ctypes import c_int, c_uint64, c_float, c_void_p
    L = lib()
    fn = getattr(L, "syn_fill_random_planar", None)
    if fn is None:
        raise RuntimeError("library lacks syn_fill_random_planar")
    fn.argtypes = [c_int, c_int, c_int, c_void_p, c_uint64, c_void_p]
    fn.restype = c_int
    check(fn(type_, rows, cols, ctypes.c_void_p(dst.data_ptr()), seed, _stream()), "fill")


def bench_gemv(type_name, rows, cols, batch, iters=50):
    import torch
    ty = TYPES[type_name]
    wb = weight_bytes(ty, rows, cols, LAYOUT_PLANAR)
    copies = max(1, math.ceil(2 * L2_BYTES / wb) + 1)
    ws = [empty_bytes(wb) for _ in range(copies)]
    for i, w in enumerate(ws):
        _fill_random(ty, rows, cols, w, 1000 + i)
    x = torch.randn(batch, cols, device="cuda")
    act = quantize_q8_0(x)
    y = torch.empty(batch, rows, device="cuda")
    for i in range(3 * copies):  # warm-up
        gemv_q(ty, ws[i % copies], LAYOUT_PLANAR, rows, cols, act, batch, y=y)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.synchronize()
    ev[0].record()
    for i in range(iters):
        gemv_q(ty, ws[i % copies], LAYOUT_PLANAR, rows, cols, act, batch, y=y)
    ev[1].record()
    ev[1].synchronize()
    ms = ev[0].elapsed_time(ev[1]) / iters
    nb = cols // 32
    alg = rows * nb * (18 if ty == Q4_0 else 34) + batch * (cols + nb * 8) + batch * rows * 4
    return {"kernel": "gemv_q", "type": type_name, "rows": rows, "cols": cols, "batch": batch,
            "us_per_launch": round(ms * 1e3, 3), "bytes_per_launch": alg, "GBps": round(alg / (ms * 1e-3) / 1e9, 1),
            "rotating_copies": copies}


def bench_attention(ctx, batch, iters=20, n_head=32, n_kv=8, hd=128):
    import torch
    row = n_kv * hd
    per_seq = ctx * row
    copies = max(1, math.ceil(2 * L2_BYTES / (2 * batch * per_seq * 2)) + 1)
    kcs, vcs = [], []
    for i in range(copies):
        kcs.append(torch.randn(batch * per_seq, device="cuda").half().view(torch.int16))
        vcs.append(torch.randn(batch * per_seq, device="cuda").half().view(torch.int16))
    q = torch.randn(batch, n_head * hd, device="cuda")
    k = torch.randn(batch, row, device="cuda")
    v = torch.randn(batch, row, device="cuda")
    pos = torch.full((batch,), ctx - 1, dtype=torch.int32, device="cuda")
    ts = 500000.0 ** (-2.0 / hd)
    scale = 1.0 / math.sqrt(hd)
    out = torch.empty(batch, n_head * hd, device="cuda")
    scratch = empty_bytes(attention_scratch_bytes(batch, n_head, n_kv, hd, ctx))
    for i in range(2 * copies):
        attention(q, k, v, kcs[i % copies], vcs[i % copies], pos, n_head, n_kv, hd, ctx, ts, scale,
                  cache_stride=per_seq, out=out, scratch=scratch)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.synchronize()
    ev[0].record()
    for i in range(iters):
        attention(q, k, v, kcs[i % copies], vcs[i % copies], pos, n_head, n_kv, hd, ctx, ts, scale,
                  cache_stride=per_seq, out=out, scratch=scratch)
    ev[1].record()
    ev[1].synchronize()
    ms = ev[0].elapsed_time(ev[1]) / iters
    alg = batch * (2 * ctx * row * 2 + n_head * hd * 8 + 2 * row * 4)
    return {"kernel": "attention", "ctx": ctx, "batch": batch, "heads": f"{n_head}/{n_kv}x{hd}",
            "us_per_launch": round(ms * 1e3, 3), "bytes_per_launch": alg, "GBps": round(alg / (ms * 1e-3) / 1e9, 1),
            "rotating_copies": copies}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("what", choices=["gemv", "attention", "all"])
    p.add_argument("--type", default=None)
    p.add_argument("--rows", type=int, default=None)
    p.add_argument("--cols", type=int, default=None)
    p.add_argument("--batch", type=int, default=None)
    p.add_argument("--ctx", type=int, default=None)
    p.add_argument("--iters", type=int, default=None)
    a = p.parse_args()
    if a.what in ("gemv", "all"):
        shapes = [(a.rows, a.cols)] if a.rows else [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
        for t in ([a.type] if a.type else ["q4_0", "q8_0"]):
            for r, c in shapes:
                for n in ([a.batch] if a.batch else [1, 4, 16]):
                    print(json.dumps(bench_gemv(t, r, c, n, a.iters or 50)), flush=True)
    if a.what in ("attention", "all"):
        for L in ([a.ctx] if a.ctx else [1024, 4096, 16384, 32768]):
            for b in ([a.batch] if a.batch else [1, 8, 32]):
                print(json.dumps(bench_attention(L, b, a.iters or 20)), flush=True)


if __name__ == "__main__":
    main()
