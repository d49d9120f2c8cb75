"""Kernel microbenchmarks of the decode path (BASELINE configs 2 and 3).

  python -m synapse_b200.kernel_bench gemv [--type q4_0|q8_0] [--rows R --cols C] [--batch N] [--iters I]
  python -m synapse_b200.kernel_bench attention [--ctx L] [--batch B] [--iters I] [--order reference|split|both]
  torchrun --nproc-per-node N -m synapse_b200.kernel_bench attention ...   (KV-head-sharded over N GPUs)
  python -m synapse_b200.kernel_bench gemv_k [--type q4_k|q6_k] [--rows R --cols C] [--batch N]
  python -m synapse_b200.kernel_bench load [--path DIR]
  python -m synapse_b200.kernel_bench llama70b [--batch B] [--ctx L] [--iters STEPS]
  python -m synapse_b200.kernel_bench excursions [--ctx L]
  python -m synapse_b200.kernel_bench decode [--ctx L] [--iters STEPS]

gemv: the quantized GEMV (syn_gemv_q, planar weights) at the sweep shapes
(4096x4096, 14336x4096, 4096x14336, 128256x4096) and batches 1/4/16, weights
N(0, 0.02) quantized on the device; enough weight copies rotate that their
total exceeds twice the 126 MB L2, so every launch streams from HBM.
gemv_k: the K-format GEMV (Q4_K / Q6_K on Q8_K activations) at the same
shapes, weights of random bytes with finite binary16 super-block scales.
load: a Llama-3-8B-shaped Q4_0 GGUF (Q8_0 head; 5.0 GB of tensor bytes with
valid block scales) written to DIR, then opened with syn_session_open_gguf
twice (the file is in the page cache both times); GB/s = tensor bytes over
the open time, beside the pinned host-to-device copy rate of this box.
attention: the fused RoPE + F16 append + attention (syn_attention) in either
summation order (--order), with H 32 / KV 8 / hd 128, theta 500000, caches of
N(0,1) F16 at context L, batch 1/8/32.
Each line: JSON with the average CUDA-event time per launch, the algorithmic
bytes per launch and GB/s. Launches are captured with programmatic dependent
launch as in the session's graphs (--no-pdl: without).
"""
import argparse
import ctypes
import json
import math
import os

import numpy as np

from . import IN_F32, IN_Q8, IN_RMSNORM, LAYOUT_PLANAR, OUT_ROWS, OUT_SILU_PAIRS, Q4_0, Q4_K, Q6_K, Q8_0, \
    GemvArgs, _ptr, _stream, attention, attention_scratch_bytes, check, empty_bytes, gemv_q, lib, q8_act_bytes, \
    quantize_q8_0, quantize_q8_k, rope_table, weight_bytes

L2_BYTES = 126 << 20
TYPES = {"q4_0": Q4_0, "q8_0": Q8_0}


PDL = True


def _graph_time(launch, iters):
    """Average device time per launch: `iters` launches captured in one CUDA graph, replayed
    twice (the second timed with CUDA events), so host launch overhead is not measured. With
    PDL the launches are captured with programmatic dependent launch, as the session's step
    graph captures them (a kernel's weight prefetch overlaps its predecessor's tail)."""
    import torch
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    L = lib()
    L.syn_set_programmatic_launch.argtypes = [ctypes.c_int]
    L.syn_set_programmatic_launch.restype = None
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
            L.syn_set_programmatic_launch(1 if PDL else 0)
            try:
                for i in range(iters):
                    launch(i)
            finally:
                L.syn_set_programmatic_launch(0)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.synchronize()
    ev[0].record()
    g.replay()
    ev[1].record()
    ev[1].synchronize()
    return ev[0].elapsed_time(ev[1]) / iters


def _fill_random(type_, rows, cols, dst, seed):
    from ctypes import c_int, c_uint64, c_float, c_void_p
    L = lib()
    fn = getattr(L, "syn_fill_random_planar", None)
    if fn is None:
        raise RuntimeError("library lacks syn_fill_random_planar")
    fn.argtypes = [c_int, c_int, c_int, c_void_p, c_uint64, c_void_p]
    fn.restype = c_int
    check(fn(type_, rows, cols, ctypes.c_void_p(dst.data_ptr()), seed, _stream()), "fill")


def bench_gemv(type_name, rows, cols, batch, iters=50, mode="q8"):
    """mode: q8 (syn_gemv_q on Q8_0 activations), f32 (floats quantized inside the kernel), rmsnorm
    (rms_norm + quantization inside), silu (rmsnorm input, rows taken as (gate, up) pairs)."""
    import torch
    ty = TYPES[type_name]
    wb = weight_bytes(ty, rows, cols, LAYOUT_PLANAR)
    copies = max(1, math.ceil(2 * L2_BYTES / wb) + 1)
    ws = [empty_bytes(wb) for _ in range(copies)]
    for i, w in enumerate(ws):
        _fill_random(ty, rows, cols, w, 1000 + i)
    x = torch.randn(batch, cols, device="cuda")
    gamma = torch.ones(cols, device="cuda")
    act = quantize_q8_0(x)
    out_rows = rows // 2 if mode == "silu" else rows
    y = torch.empty(batch, out_rows, device="cuda")
    if mode == "q8":
        def launch(i):
            gemv_q(ty, ws[i % copies], LAYOUT_PLANAR, rows, cols, act, batch, y=y)
    else:
        in_mode = IN_F32 if mode == "f32" else IN_RMSNORM
        out_mode = OUT_SILU_PAIRS if mode == "silu" else OUT_ROWS
        args = [GemvArgs(ty, LAYOUT_PLANAR, rows, cols, batch, w.data_ptr(), in_mode, None, x.data_ptr(),
                         gamma.data_ptr(), 1e-5, out_mode, y.data_ptr(), None) for w in ws]

        def launch(i):
            check(lib().syn_gemv(ctypes.byref(args[i % copies]), _stream()), "syn_gemv")
    for i in range(3 * copies):  # warm-up
        launch(i)
    ms = _graph_time(launch, iters)
    nb = cols // 32
    act_bytes = batch * (cols + nb * 8) if mode == "q8" else batch * cols * 4 * (2 if mode != "f32" else 1)
    alg = rows * nb * (18 if ty == Q4_0 else 34) + act_bytes + batch * out_rows * 4
    return {"kernel": "gemv_q" if mode == "q8" else "gemv_" + mode, "type": type_name, "rows": rows, "cols": cols,
            "batch": batch, "us_per_launch": round(ms * 1e3, 3), "bytes_per_launch": alg,
            "GBps": round(alg / (ms * 1e-3) / 1e9, 1), "rotating_copies": copies}


def bench_layers(type_name="q4_0", n_layer=32, iters=2):
    """The four fused GEMVs of each of n_layer distinct Llama-3-8B-shaped layers, captured back to back as the
    step graph runs them: qkv (rms_norm in), o (floats in, residual), gate/up pairs (rms_norm in, silu * up out),
    down (floats in, residual). Attention is left out, so this is the GEMV part of a decode step."""
    import torch
    ty = TYPES[type_name]
    d, ff, qkv_rows = 4096, 14336, 6144
    shapes = [(qkv_rows, d, IN_RMSNORM, OUT_ROWS), (d, d, IN_F32, OUT_ROWS), (2 * ff, d, IN_RMSNORM, OUT_SILU_PAIRS),
              (d, ff, IN_F32, OUT_ROWS)]
    x = torch.randn(d, device="cuda")
    qkv = torch.empty(qkv_rows, device="cuda")
    act = torch.randn(ff, device="cuda") * 0.1
    attn = torch.randn(d, device="cuda")
    gamma = torch.ones(d, device="cuda")
    keep, args = [], []
    weight_bytes_total = 0
    for l in range(n_layer):
        for j, (r, c, im, om) in enumerate(shapes):
            wb = weight_bytes(ty, r, c, LAYOUT_PLANAR)
            w = empty_bytes(wb)
            _fill_random(ty, r, c, w, 7000 + 10 * l + j)
            keep.append(w)
            weight_bytes_total += r * (c // 32) * (18 if ty == Q4_0 else 34)
            inp = {0: x, 1: attn, 2: x, 3: act}[j]
            out = {0: qkv, 1: x, 2: act, 3: x}[j]
            res = x.data_ptr() if j in (1, 3) else None
            args.append(GemvArgs(ty, LAYOUT_PLANAR, r, c, 1, w.data_ptr(), im, None, inp.data_ptr(),
                                 gamma.data_ptr() if im == IN_RMSNORM else None, 1e-5, om, out.data_ptr(), res))

    def launch(i):
        for a in args:
            check(lib().syn_gemv(ctypes.byref(a), _stream()), "syn_gemv")
    launch(0)
    ms = _graph_time(launch, iters) / 1.0
    return {"kernel": "gemv_layers", "type": type_name, "layers": n_layer, "us_per_layer": round(ms * 1e3 / n_layer, 2),
            "weight_bytes_per_layer": weight_bytes_total // n_layer,
            "GBps": round(weight_bytes_total / (ms * 1e-3) / 1e9, 1)}


LLAMA70B = dict(n_layer=80, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8, head_dim=128, n_vocab=128256,
                rms_eps=1e-5, rope_base=500000.0)


def bench_llama70b(batch, ctx=8192, steps=8, n_layer=80):
    """the Llama-3-70B-shaped decode (Q4_0 everywhere, F16 KV) at context ctx, batch 1
    (the captured step graph) or batch sequences per step (syn_session_step_batch: the weights stream once for
    all of them). The KV caches hold seeded N(0,1) values for positions 0 .. ctx - steps - 1, so the timed
    steps attend over ctx - steps .. ctx - 1 positions; weights random N(0, 0.02), quantized on the device."""
    import time
    import torch
    from . import Q4_0 as _Q4, Session
    cfg = dict(LLAMA70B, n_layer=n_layer, type_embd=_Q4, type_layers=_Q4, type_output=_Q4)
    t0 = time.perf_counter()
    if batch == 1:
        sess = Session.synthetic(cfg, max_ctx=ctx, seed=70)
    else:
        sess = Session.synthetic_ex(cfg, max_ctx=ctx, max_seqs=batch, max_batch=batch, seed=70)
    sess.fill_kv_random(ctx - steps, seed=71)
    open_s = time.perf_counter() - t0
    stream = torch.cuda.ExternalStream(sess.stream_handle())
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    pos0 = ctx - steps
    if batch == 1:
        sess.generate([1], pos0 - 2, 2)  # warm-up
        ev[0].record(stream)
        sess.generate([7], pos0, steps, wait=False)
        ev[1].record(stream)
        ev[1].synchronize()
    else:
        toks = [int(t) for t in np.random.default_rng(1).integers(0, LLAMA70B["n_vocab"], batch)]
        sess.step_batch(toks, [pos0 - 1] * batch, logits=False)  # warm-up
        ev[0].record(stream)
        for i in range(steps):
            _, nxt = sess.step_batch(toks, [pos0 + i] * batch, logits=False)
            toks = [int(t) for t in nxt]
        ev[1].record(stream)
        ev[1].synchronize()
    ms = ev[0].elapsed_time(ev[1]) / steps
    row = LLAMA70B["n_head_kv"] * LLAMA70B["head_dim"]
    weights = n_layer * ((8192 + 2 * 1024) * 8192 + 8192 * 8192 + 3 * 28672 * 8192) // 32 * 18 + 128256 * 8192 // 32 * 18
    kv = batch * n_layer * 2 * (pos0 + steps // 2) * row * 2
    sess.close()
    return {"kernel": "llama70b_decode", "batch": batch, "ctx": ctx, "layers": n_layer, "ms_per_step": round(ms, 3),
            "tok_s": round(batch / (ms * 1e-3), 2), "GBps": round((weights + kv) / (ms * 1e-3) / 1e9, 1),
            "bytes_per_step": weights + kv, "open_s": round(open_s, 1),
            "path": "step graph" if batch == 1 else "syn_session_step_batch (op by op)"}


def bench_decode(ctx=4096, steps=20):
    """One Llama-3-8B-shaped Q4_0 decode step (the captured step graph) at context ctx: the KV
    caches hold seeded values for positions 0 .. ctx - steps - 2, one untimed step warms up, then steps - 1
    timed device steps; the step at position ctx - 1 alone runs between cudaProfilerStart and cudaProfilerStop,
    so `ncu --profile-from-start off` lists exactly one step's launches."""
    import torch
    from . import Q4_0 as _Q4, Q8_0 as _Q8, Session
    cfg = dict(n_layer=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128, n_vocab=128256,
               rms_eps=1e-5, rope_base=500000.0, type_embd=_Q4, type_layers=_Q4, type_output=_Q8)
    sess = Session.synthetic(cfg, max_ctx=ctx, seed=1234)
    pos0 = ctx - steps - 1
    sess.fill_kv_random(pos0, seed=5)
    stream = torch.cuda.ExternalStream(sess.stream_handle())
    sess.generate([1], pos0, 1)  # warm-up
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    sess.generate([7], pos0 + 1, steps - 1, wait=False)
    ev[1].record(stream)
    ev[1].synchronize()
    torch.cuda.profiler.start()
    sess.generate([9], ctx - 1, 1)
    torch.cuda.profiler.stop()
    ms = ev[0].elapsed_time(ev[1]) / max(1, steps - 1)
    n = sess.launches_per_step()
    sess.close()
    return {"kernel": "decode_step", "ctx": ctx, "timed_steps": steps - 1, "ms_per_step": round(ms, 4),
            "tok_s": round(1e3 / ms, 2), "launches_per_step": n,
            "positions": f"{pos0 + 1}..{ctx - 2} timed, {ctx - 1} between the profiler marks"}


def bench_excursions(ctx=4096, seed=1234):
    """How often the split attention order moves the logits past the north-star tolerance: two sessions of the
    8B-shaped Q4_0 model with the same seeded weights, one with the attention sums in the reference's order
    (bit-identical to the oracle) and one with SYN_ATTN_ORDER=split, fed the same seeded random tokens at
    positions 0 .. ctx - 1 (teacher-forced). Per step: d = max |logit_split - logit_exact| / std(logit_exact)."""
    from . import Q4_0 as _Q4, Q8_0 as _Q8, Session
    cfg = dict(n_layer=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128, n_vocab=128256,
               rms_eps=1e-5, rope_base=500000.0, type_embd=_Q4, type_layers=_Q4, type_output=_Q8)
    prev = os.environ.pop("SYN_ATTN_ORDER", None)
    exact = Session.synthetic(cfg, max_ctx=ctx, seed=seed)
    os.environ["SYN_ATTN_ORDER"] = "split"
    split = Session.synthetic(cfg, max_ctx=ctx, seed=seed)
    if prev is None:
        os.environ.pop("SYN_ATTN_ORDER")
    else:
        os.environ["SYN_ATTN_ORDER"] = prev
    toks = np.random.default_rng(seed).integers(0, cfg["n_vocab"], ctx)
    d = np.zeros(ctx)
    argmax_diff = 0
    for pos in range(ctx):
        le, ae = exact.step(int(toks[pos]), pos)
        ls, as_ = split.step(int(toks[pos]), pos)
        d[pos] = float(np.max(np.abs(ls - le)) / np.std(le))
        argmax_diff += int(ae != as_)
    exact.close()
    split.close()
    past = d[256:]
    over = np.nonzero(d > 1e-2)[0]
    return {"kernel": "excursions", "ctx": ctx, "steps": ctx, "steps_past_256": int(past.size),
            "first_over_1e-2_std": int(over[0]) if over.size else None,
            "d_at_257_264": [float(x) for x in d[257:265]],
            "steps_differing": int(np.count_nonzero(d)), "steps_over_1e-2_std": int(np.count_nonzero(d > 1e-2)),
            "max_d": float(d.max()), "p99_d": float(np.percentile(past, 99)), "median_d": float(np.median(past)),
            "argmax_differs": argmax_diff,
            "note": "d = max|logit_split - logit_exact| / std(logit_exact) per step; positions <= 256 are one chunk "
                    "(both orders exact)"}


K_TYPES = {"q4_k": Q4_K, "q6_k": Q6_K}


def _random_k_weights(ty, rows, cols, seed):
    """Random bytes as planar K-format rows, every binary16 super-block scale set to 2^-10."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    wb = weight_bytes(ty, rows, cols, LAYOUT_PLANAR)
    w = torch.randint(0, 256, (wb,), dtype=torch.uint8, device="cuda", generator=g)
    nb = cols // 256
    scale = torch.tensor([0x00, 0x14], dtype=torch.uint8, device="cuda")  # 0x1400 little-endian
    if ty == Q4_K:
        blk = w.view(rows * nb, 144)
        blk[:, 0:2] = scale
        blk[:, 2:4] = scale
    else:
        r = w.view(rows, wb // rows)
        r[:, nb * 208:nb * 210] = scale.repeat(nb)
    return w


def bench_gemv_k(type_name, rows, cols, batch, iters=50):
    import torch
    ty = K_TYPES[type_name]
    wb = weight_bytes(ty, rows, cols, LAYOUT_PLANAR)
    copies = max(1, math.ceil(2 * L2_BYTES / wb) + 1)
    ws = [_random_k_weights(ty, rows, cols, 1000 + i) for i in range(copies)]
    x = torch.randn(batch, cols, device="cuda")
    act = quantize_q8_k(x)
    y = torch.empty(batch, rows, device="cuda")

    def launch(i):
        gemv_q(ty, ws[i % copies], LAYOUT_PLANAR, rows, cols, act, batch, y=y)
    for i in range(3 * copies):
        launch(i)
    ms = _graph_time(launch, iters)
    nb = cols // 256
    alg = rows * nb * (144 if ty == Q4_K else 210) + batch * (cols + nb * 4 + cols // 16 * 2) + batch * rows * 4
    return {"kernel": "gemv_k", "type": type_name, "rows": rows, "cols": cols, "batch": batch,
            "us_per_launch": round(ms * 1e3, 3), "bytes_per_launch": alg, "GBps": round(alg / (ms * 1e-3) / 1e9, 1),
            "rotating_copies": copies}


def _patterned(n_bytes, block, seed):
    """Random bytes laid out as `block`-byte GGUF blocks whose binary16 scale (the
    first two bytes) is 2^-10."""
    rng = np.random.default_rng(seed)
    n_blocks = -(-n_bytes // block)
    buf = rng.integers(0, 256, n_blocks * block, dtype=np.uint8)
    buf.reshape(n_blocks, block)[:, 0:2] = np.array([0x00, 0x14], np.uint8)
    return buf


def bench_load(directory=None, opens=2):
    """Load bandwidth of the session's GGUF loader on a synthetic 8B Q4_0 file."""
    import os
    import tempfile
    import time

    import torch

    from . import Session
    from . import model as m
    cfg = dict(n_layer=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128, n_vocab=128256,
               rms_eps=1e-5, rope_base=500000.0)
    shapes = m.llama_shapes(cfg)
    q4 = _patterned(cfg["n_vocab"] * cfg["n_embd"] // 32 * 18, 18, 1)
    q8 = _patterned(cfg["n_vocab"] * cfg["n_embd"] // 32 * 34, 34, 2)
    w = {"token_embd": (Q4_0, q4.reshape(cfg["n_vocab"], -1)),
         "output": (Q8_0, q8.reshape(cfg["n_vocab"], -1)),
         "output_norm": (m.F32, np.ones(cfg["n_embd"], np.float32))}
    total = q4.size + q8.size + cfg["n_embd"] * 4
    for l in range(cfg["n_layer"]):
        for n in m.LAYER_NAMES:
            rows, cols = shapes[n]
            if n.endswith("norm"):
                w[f"blk.{l}.{n}"] = (m.F32, np.ones(cols, np.float32))
                total += cols * 4
            else:
                nb = rows * cols // 32 * 18
                w[f"blk.{l}.{n}"] = (Q4_0, q4[:nb].reshape(rows, -1))
                total += nb
    d = directory or tempfile.mkdtemp(prefix="synload")
    path = os.path.join(d, "llama8b_q4_0.gguf")
    m.write_llama_gguf(path, cfg, w, context_length=4096)
    # the pinned host -> device rate of this box, for scale
    h = torch.empty(256 << 20, dtype=torch.uint8).pin_memory()
    dv = torch.empty_like(h, device="cuda")
    dv.copy_(h, non_blocking=True)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(4):
        dv.copy_(h, non_blocking=True)
    ev[1].record()
    ev[1].synchronize()
    h2d = 4 * h.numel() / (ev[0].elapsed_time(ev[1]) * 1e-3) / 1e9
    del h, dv
    times = []
    for _ in range(opens):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        sess = Session.open(path, max_ctx=4096)
        times.append(time.perf_counter() - t0)
        sess.close()
    os.remove(path)
    best = min(times)
    return {"kernel": "load", "file": "llama-3-8B-shaped Q4_0 (Q8_0 head)", "tensor_bytes": total,
            "open_s": [round(t, 3) for t in times], "GBps": round(total / best / 1e9, 2),
            "pinned_h2d_GBps": round(h2d, 1), "host_threads": os.cpu_count()}


def bench_attention(ctx, batch, iters=20, n_head=32, n_kv=8, hd=128, order=0):
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
    tab = rope_table(ctx, hd, ts)
    run = lambda i: attention(q, k, v, kcs[i % copies], vcs[i % copies], pos, n_head, n_kv, hd, ctx, ts, scale,
                              cache_stride=per_seq, out=out, scratch=scratch, rope_table=tab, order=order)
    for i in range(2 * copies):
        run(i)
    ms = _graph_time(run, iters)
    alg = batch * (2 * ctx * row * 2 + n_head * hd * 8 + 2 * row * 4)
    return {"kernel": "attention", "order": ["reference", "split"][order], "ctx": ctx, "batch": batch,
            "heads": f"{n_head}/{n_kv}x{hd}",
            "us_per_launch": round(ms * 1e3, 3), "bytes_per_launch": alg, "GBps": round(alg / (ms * 1e-3) / 1e9, 1),
            "rotating_copies": copies}


def bench_attention_sharded(a, world):
    """BASELINE config 3 KV-head-sharded (run under torchrun, one rank per GPU): rank r holds KV heads
    [r * 8 / world, (r + 1) * 8 / world) and their query heads, as the tensor-parallel session shards them, and
    times its own attention call; the line reports the slowest rank (the ranks meet in a gloo reduction of
    their times only: the attention itself exchanges nothing)."""
    import datetime
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", str(rank))))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    try:
        n_head, n_kv = 32 // world, 8 // world
        for L in ([a.ctx] if a.ctx else [1024, 4096, 16384, 32768]):
            for b in ([a.batch] if a.batch else [1, 8, 32]):
                for o in ({"reference": [0], "split": [1], "both": [0, 1]}[a.order]):
                    r = bench_attention(L, b, a.iters or 20, n_head=n_head, n_kv=n_kv, order=o)
                    t = torch.tensor([r["us_per_launch"]], dtype=torch.float64)
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                    if rank == 0:
                        alg = r["bytes_per_launch"] * world
                        print(json.dumps({"kernel": "attention_sharded", "order": r["order"], "ctx": L, "batch": b,
                                          "gpus": world, "heads_per_gpu": r["heads"],
                                          "us_per_launch_max_over_ranks": round(float(t.item()), 3),
                                          "bytes_all_gpus": alg,
                                          "GBps_all_gpus": round(alg / (float(t.item()) * 1e-6) / 1e9, 1)}),
                              flush=True)
    finally:
        dist.destroy_process_group()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("what", choices=["gemv", "gemv_k", "attention", "load", "llama70b", "excursions", "decode", "all"])
    p.add_argument("--path", default=None, help="load: directory for the synthetic GGUF file")
    p.add_argument("--type", default=None)
    p.add_argument("--rows", type=int, default=None)
    p.add_argument("--cols", type=int, default=None)
    p.add_argument("--batch", type=int, default=None)
    p.add_argument("--ctx", type=int, default=None)
    p.add_argument("--iters", type=int, default=None)
    p.add_argument("--no-pdl", action="store_true", help="capture without programmatic dependent launch")
    p.add_argument("--order", default="both", choices=["reference", "split", "both"],
                   help="attention: the summation order (syn_attention_args.order)")
    p.add_argument("--mode", default="q8", choices=["q8", "f32", "rmsnorm", "silu", "step", "layers"],
                   help="gemv input/output fusion; step: the four fused GEMVs of an 8B layer, each timed alone; "
                        "layers: those four GEMVs of 32 distinct layers back to back in one graph")
    a = p.parse_args()
    global PDL
    PDL = not a.no_pdl
    if a.what == "gemv" and a.mode == "layers":
        print(json.dumps(bench_layers(a.type or "q4_0", 32, a.iters or 2)), flush=True)
    elif a.what in ("gemv", "all") and a.mode == "step":
        # the fused GEMVs of one Llama-3-8B layer: qkv (rms_norm in), o (f32 in), gate/up pairs, down (f32 in)
        for t in ([a.type] if a.type else ["q4_0"]):
            for mode, r, c in (("rmsnorm", 6144, 4096), ("f32", 4096, 4096), ("silu", 28672, 4096),
                               ("f32", 4096, 14336)):
                print(json.dumps(bench_gemv(t, r, c, 1, a.iters or 50, mode)), flush=True)
    elif a.what in ("gemv", "all"):
        shapes = [(a.rows, a.cols)] if a.rows else [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
        for t in ([a.type] if a.type else ["q4_0", "q8_0"]):
            for r, c in shapes:
                for n in ([a.batch] if a.batch else [1, 4, 16]):
                    print(json.dumps(bench_gemv(t, r, c, n, a.iters or 50, a.mode)), flush=True)
    if a.what in ("gemv_k", "all"):
        shapes = [(a.rows, a.cols)] if a.rows else [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
        for t in ([a.type] if a.type else ["q4_k", "q6_k"]):
            for r, c in shapes:
                for n in ([a.batch] if a.batch else [1, 4, 16]):
                    print(json.dumps(bench_gemv_k(t, r, c, n, a.iters or 50)), flush=True)
    if a.what == "load":
        print(json.dumps(bench_load(a.path)), flush=True)
    if a.what == "decode":
        print(json.dumps(bench_decode(a.ctx or 4096, a.iters or 20)), flush=True)
    if a.what == "excursions":
        print(json.dumps(bench_excursions(a.ctx or 4096)), flush=True)
    if a.what == "llama70b":
        for b in ([a.batch] if a.batch else [1, 16]):
            print(json.dumps(bench_llama70b(b, a.ctx or 8192, a.iters or 8)), flush=True)
    if a.what in ("attention", "all"):
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if world > 1:
            bench_attention_sharded(a, world)
            return
        for L in ([a.ctx] if a.ctx else [1024, 4096, 16384, 32768]):
            for b in ([a.batch] if a.batch else [1, 8, 32]):
                for o in ({"reference": [0], "split": [1], "both": [0, 1]}[a.order]):
                    print(json.dumps(bench_attention(L, b, a.iters or 20, order=o)), flush=True)


if __name__ == "__main__":
    main()
