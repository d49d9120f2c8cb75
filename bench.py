#!/usr/bin/env python
"""Decode throughput of the Llama-3-8B-shaped Q4_0 model on B200 (the
reference's headline path: quantized GEMV + RoPE/KV-cache attention).

One step = one greedy decode token of the 32-layer model (Q4_0 layers and
embedding, Q8_0 head, F16 KV cache) at 4k context: a seeded 512-token prompt
and greedy decode to position 4095 - K run untimed on the device (W of those
steps are the warm-up), then the K timed steps decode positions 4096 - K ..
4095 ("at 4k context"). Weights are random N(0, 0.02),
quantized on the device (synthetic data of the named shape).

value : K / device time of the K steps (CUDA events on the session stream;
        the steps are CUDA-graph replays with the argmax fed back on the
        device). full_range: the same over every position 512 .. 4095.
e2e   : the same metric through the public step API over the same positions:
        per step the token and position go host->device from pinned memory
        and the logits + argmax come back device->host.
roofline : the dominant kernel (the quantized GEMV on the gate/up rows):
        algorithmic bytes per launch / its CUDA-event time inside one step at
        position 4095 (each op of the step captured between events), vs
        MEASURED_PEAKS hbm_gbs; traffic: DRAM bytes per launch of the same
        shape from ncu.
cpu_baseline : the C oracle (a restatement of the reference's CPU kernels) on
        this host's cores, a bounded sample (see `sample`), and on one core
        (cpu_baseline_1core).

--impl reference: the reference's CPU path (the oracle port; the reference's
own headers need MTL5, absent here) on all host cores, same metric and unit.

Multi-GPU (torchrun, N ranks), --parallel tp (default): one sequence,
tensor-parallel over the N GPUs (KV-head groups and GEMV output rows;
logits bit-identical to one GPU), strong scaling; value = tokens / max over
ranks of the device time. --parallel replicas: each GPU decodes its own
sequence (weak scaling); value = tokens of all ranks / max over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LLAMA8B = dict(n_layer=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128, n_vocab=128256,
               rms_eps=1e-5, rope_base=500000.0)
PROMPT = 512
CTX = 4096
METRIC = "decode tok/s (Llama-3-8B Q4_0 shape)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20, help="timed decode steps: positions 4096-K .. 4095")
    p.add_argument("--warmup", type=int, default=16)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--parallel", default="tp", choices=["tp", "replicas"],
                   help="N > 1: tensor-parallel one sequence (tp) or one sequence per GPU (replicas)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--profile-out", default=None, help="write the per-op device times of one step (JSON) here")
    p.add_argument("--ncu-step", type=int, default=0,
                   help="profiling mode: an 8-token prompt, then N graph steps inside the NVTX range decode_step")
    p.add_argument("--ncu-pos", type=int, default=8,
                   help="profiling mode: the position of the first profiled step (the cache rows before it hold zeros)")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- CPU (oracle) timing

class CpuDecoder:
    """The oracle (the reference's CPU path restated) on the 8B shape at position CTX-1.

    n_distinct distinct random Q4_0 layers (so no layer's weights sit in the CPU's caches), the Q4_0
    embedding, the Q8_0 head, and a KV cache filled with seeded F16 values for positions 0..CTX-2. A
    "layer-step" decodes one token through one layer (rotating layers); tok/s = 1 / (32 * mean
    layer-step + head)."""

    def __init__(self, threads, n_distinct=4, seed=7):
        import oracle as orc

        orc.set_threads(threads)
        self.threads, self.n = threads, n_distinct
        c = dict(LLAMA8B, n_layer=n_distinct)
        d, ff, q, kv = c["n_embd"], c["n_ff"], c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
        shapes = {"attn_q": (q, d), "attn_k": (kv, d), "attn_v": (kv, d), "attn_output": (d, q),
                  "ffn_gate": (ff, d), "ffn_up": (ff, d), "ffn_down": (d, ff)}
        w = {"token_embd": (orc.Q4_0, orc.random_weights(orc.Q4_0, c["n_vocab"], d, seed, 1)),
             "output": (orc.Q8_0, orc.random_weights(orc.Q8_0, c["n_vocab"], d, seed, 2)),
             "output_norm": (orc.F32, np.ones(d, np.float32))}
        tid = 3
        for l in range(n_distinct):
            w[f"blk.{l}.attn_norm"] = (orc.F32, np.ones(d, np.float32))
            w[f"blk.{l}.ffn_norm"] = (orc.F32, np.ones(d, np.float32))
            for n, (r, cc) in shapes.items():
                w[f"blk.{l}.{n}"] = (orc.Q4_0, orc.random_weights(orc.Q4_0, r, cc, seed, tid))
                tid += 1
        self.m = orc.Llama(c, w, max_ctx=CTX)
        rng = np.random.default_rng(seed)
        for l in range(n_distinct):
            for cache in (self.m.kcache(l), self.m.vcache(l)):
                cache[:] = rng.standard_normal(cache.size, dtype=np.float32).astype(np.float16).view(np.uint16)
        self.pos = CTX - 1
        self.m.run(1, self.pos, 0, 0, embed=True)
        self.i = 0
        self.times = []

    def layer_step(self, record=True):
        l = self.i % self.n
        t0 = time.perf_counter()
        self.m.run(1, self.pos, l, l + 1, embed=False)
        dt = time.perf_counter() - t0
        self.i += 1
        if record:
            self.times.append(dt)
        return dt

    def head(self):
        t0 = time.perf_counter()
        self.m.run(1, self.pos, 0, 0, embed=False, logits=True)
        return time.perf_counter() - t0

    def result(self, head_s):
        layer = statistics.mean(self.times)
        return 1.0 / (LLAMA8B["n_layer"] * layer + head_s), layer

    def sample(self, head_s, layer_s):
        return (f"oracle (reference CPU path restated, {self.threads} threads): {len(self.times)} timed layer-steps "
                f"of the 8B-shaped Q4_0 decode at position {self.pos} ({self.n} distinct random layers, KV "
                f"pre-filled) + the Q8_0 head once; tok/s = 1/(32*{layer_s * 1e3:.2f} ms + {head_s * 1e3:.2f} ms)")


def cpu_baselines(budget_all_s, budget_one_s):
    """The oracle timed on every host core, then on one core (the same decoder and position)."""
    import oracle as orc

    out = []
    dec = CpuDecoder(os.cpu_count() or 1)
    for threads, budget in ((os.cpu_count() or 1, budget_all_s), (1, budget_one_s)):
        orc.set_threads(threads)
        dec.threads, dec.times = threads, []
        dec.layer_step(record=False)
        t_end = time.perf_counter() + budget
        while time.perf_counter() < t_end or len(dec.times) < 2:
            dec.layer_step()
        head = dec.head()
        value, layer = dec.result(head)
        out.append({"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                    "sample": dec.sample(head, layer)})
    return out


def reference_arm(args, rank, world):
    """Rank 0 only: W warmup then exactly K timed layer-steps (each a bounded sample of one decode token)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    K = args.steps if args.steps is not None else 64
    t0 = time.perf_counter()
    dec = CpuDecoder(threads)
    for _ in range(max(3, args.warmup)):
        dec.layer_step(record=False)
    for _ in range(K):
        dec.layer_step()
    head = dec.head()
    value, layer = dec.result(head)
    print(json.dumps({
        "metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": world, "steps": K,
        "warmup": max(3, args.warmup), "ms_per_step": round(1000.0 / value, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_0/q8_0 weights x q8_0 activations (exact int dots), f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": "Llama-3-8B-shaped Q4_0 decode at 4k context (BASELINE config 4)", "global_batch": 1,
                   "seq_len": CTX, "parallelism": "cpu threads"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": dec.sample(head, layer)},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(time.perf_counter() - t0, 1),
    }))
    sys.stdout.flush()


# --------------------------------------------------------------------------- GPU arm

def ncu_step(args, local):
    """A short run for ncu launch lists: the 8B session, an 8-token prompt, then
    args.ncu_step graph steps from position args.ncu_pos inside the NVTX range "decode_step"."""
    import torch

    import synapse_b200 as syn

    cfg = dict(LLAMA8B, type_embd=syn.Q4_0, type_layers=syn.Q4_0, type_output=syn.Q8_0)
    sess = syn.Session.synthetic(cfg, max_ctx=CTX, seed=1234, device=local)
    toks = sess.generate(list(range(1, 9)), 0, 8)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("decode_step")
    pos = max(8, min(args.ncu_pos, CTX - args.ncu_step))
    out = sess.generate([int(toks[-1])], pos, args.ncu_step)
    torch.cuda.nvtx.range_pop()
    print(json.dumps({"ncu_step": args.ncu_step, "position": pos, "launches_per_step": sess.launches_per_step(),
                      "tokens": [int(t) for t in out]}))
    sess.close()


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist

    import synapse_b200 as syn

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    if args.ncu_step:
        return ncu_step(args, local)
    W = max(3, args.warmup)
    K = max(1, min(args.steps, CTX - PROMPT - W))
    start_pos = CTX - K  # the timed steps decode positions CTX-K .. CTX-1 (4k context)
    max_ctx = CTX
    cfg = dict(LLAMA8B, type_embd=syn.Q4_0, type_layers=syn.Q4_0, type_output=syn.Q8_0)
    tp_mode = world > 1 and args.parallel == "tp"
    tp = syn.TP.from_torch_distributed(device=local) if tp_mode else None
    seed_rank = 0 if tp_mode else rank  # tensor-parallel ranks share one model and one sequence
    sess = syn.Session.synthetic(cfg, max_ctx=max_ctx, seed=1234 + seed_rank, device=local, tp=tp)
    layout = sess.tp_layout()
    stream = torch.cuda.ExternalStream(sess.stream_handle(), device=torch.device("cuda", local))
    prompt = np.random.default_rng(42 + seed_rank).integers(0, LLAMA8B["n_vocab"], PROMPT)
    seqs = 1 if tp_mode else world  # sequences decoded by the whole job

    def device_max(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def to_start():
        """The prompt, then greedy decode to position start_pos - 1 (on the device, untimed); the last W of
        these steps are the warm-up. Returns the next input token and the device time of positions
        PROMPT .. start_pos - 1."""
        toks = sess.generate(prompt, 0, PROMPT)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        out = sess.generate([int(toks[-1])], PROMPT, start_pos - PROMPT)
        e1.record(stream)
        e1.synchronize()
        return int(out[-1]), e0.elapsed_time(e1)

    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clocks:  # the pre-decode runs the same step graph: the clocks under this load
        last, pre_ms = to_start()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        sess.generate([last], start_pos, K, wait=False)
        ev1.record(stream)
        ev1.synchronize()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_max = device_max(ev0.elapsed_time(ev1))
    value = seqs * K / (ms_max / 1e3)
    full_ms = device_max(pre_ms + ev0.elapsed_time(ev1))
    full_range = {"positions": f"{PROMPT}..{CTX - 1}", "value": round(seqs * (CTX - PROMPT) / (full_ms / 1e3), 2),
                  "unit": "tok/s"}

    # e2e through the public step API over the same positions (host round trip every step)
    sess.reset()
    last, _ = to_start()
    tok = last
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for i in range(K):
        _, tok = sess.step(tok, start_pos + i, logits=True)
    e1.record(stream)
    e1.synchronize()
    e2e = seqs * K / (device_max(e0.elapsed_time(e1)) / 1e3)

    # roofline of the dominant kernel: every op of one step at position CTX-1, timed op by op with CUDA events
    prof_pos = CTX - 1
    runs = [sess.profile(tok, prof_pos) for _ in range(3)]
    per_op = [min(r[i]["ms"] for r in runs) for i in range(len(runs[0]))]
    ops = runs[0]
    gemv_ms = sum(t for t, o in zip(per_op, ops) if o["kind"] == "matmul")
    gemv_bytes = sum(o["bytes"] for o in ops if o["kind"] == "matmul")
    attn_ms = sum(t for t, o in zip(per_op, ops) if o["kind"] == "attention")
    attn_bytes = sum(o["bytes"] for o in ops if o["kind"] == "attention")
    total_ms = sum(per_op)
    # the dominant kernel: the GEMV on the gate/up rows (the largest share of the step)
    gu = [(t, o) for t, o in zip(per_op, ops) if o["kind"] == "matmul" and o["rows"] == 2 * layout["n_ff"]]
    gather_ms = sum(t for t, o in zip(per_op, ops) if o["kind"] == "allgather")
    peer_stores = tp_mode and sess.tp_status()["peer_stores"]
    gu_ms = sum(t for t, _ in gu) / max(1, len(gu))
    gu_bytes = gu[0][1]["bytes"] if gu else 0.0
    peak, peak_kind = peaks()
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9 if gu else gemv_bytes / (gemv_ms / 1e3) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "gemv_traffic.json")) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    except Exception:
        pass
    step_bytes = sum(o["bytes"] for o in ops)
    if args.profile_out and rank == 0:
        with open(args.profile_out, "w") as f:
            json.dump([dict(o, ms=t, gbps=o["bytes"] / (t / 1e3) / 1e9 if t > 0 else None)
                       for o, t in zip(ops, per_op)], f, indent=0)

    cpu = cpu1 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu, cpu1 = cpu_baselines(12.0, 8.0)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms_max / K, 4), "higher_is_better": True,
            "scaling": "strong" if tp_mode else "weak",
            "vs_baseline": None, "dtype": "q4_0/q8_0 weights x q8_0 activations (exact int8 dots), f32 accum",
            "data": "synthetic",
            "config": {"workload": "Llama-3-8B-shaped Q4_0 decode at 4k context (BASELINE config 4): 512-token "
                                   f"prompt and greedy decode to position {start_pos - 1} untimed (the last {W} "
                                   f"steps the warm-up), then timed positions {start_pos}..{CTX - 1}",
                       "model": "llama3-8b-shape (32L, d4096, 32H/8KV, ff14336, V128256), Q4_0 + Q8_0 head",
                       "global_batch": seqs, "seq_len": CTX,
                       "parallelism": f"tp{world}" if tp_mode else ("replicas" if world > 1 else "single"),
                       "attention_order": "reference" if os.environ.get("SYN_ATTN_ORDER", "") != "split" else "split",
                       "l2": "weights 4.5 GB per step > 126 MB L2: streamed from HBM every step"},
            "full_range": full_range,
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": LLAMA8B["n_vocab"] * 4 + 4},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": f"gemv_stage_kernel<Q4_0> on the gate/up rows ({2 * layout['n_ff']}x4096 "
                                   f"per rank, rms_norm in, silu*up out), {len(gu)} launches of one step at pos "
                                   f"{prof_pos}, "
                                   f"{gu_bytes / 1e6:.2f} MB algorithmic per launch",
                         "all_gemv_gbs": round(gemv_bytes / (gemv_ms / 1e3) / 1e9, 1),
                         "peak_source": peak_kind,
                         "step_frac": round(step_bytes / (ms_max / K / 1e3) / 1e9 / peak, 4),
                         "attention_gbs": round(attn_bytes / (attn_ms / 1e3) / 1e9, 1),
                         "attention_us_per_layer": round(attn_ms * 1e3 / max(1, LLAMA8B["n_layer"]), 2),
                         "gemv_share_of_step": round(gemv_ms / total_ms, 3),
                         # NCCL all-gathers only: peer-store gathers run inside the producing and reading kernels
                         "allgather_ms_per_step": round(gather_ms, 4) if tp_mode and not peer_stores else None},
            "gpu_launches": sess.launches_per_step() * K,
            "clocks": clocks.summary(),
        }
        if cpu:
            line["cpu_baseline"] = cpu
            line["cpu_baseline_1core"] = cpu1
        print(json.dumps(line))
        sys.stdout.flush()
    sess.close()  # its graphs hold NCCL calls: released before the communicators
    if tp is not None:
        tp.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
