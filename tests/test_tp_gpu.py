"""Tensor parallelism on 2 or more GPUs of one node, through the session's C
ABI: each rank holds its heads and rows, NCCL all-gathers in place inside
the captured step graph, and the logits (and greedy tokens) equal one GPU's
bit for bit, the reference's D1 contract (tests/sdk/llama_threads.cpp:32)
across GPUs. Skipped on a box with fewer than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
syn = pytest.importorskip("synapse_b200")
torch = pytest.importorskip("torch")

from synapse_b200 import model  # noqa: E402

SHAPES = {
    # Llama-3-8B widths, two layers: the fused GEMV and fused attention paths
    "8b_2layer_q4_0": dict(n_layer=2, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128, n_vocab=128256,
                           rms_eps=1e-5, rope_base=500000.0, rope_mode=0, type_embd=model.F32,
                           type_layers=model.Q4_0, type_output=model.Q8_0),
    # BASELINE config 1's tiny model (Q8_0 layers, tied F32 embedding head): the unfused fallbacks
    "tiny_q8_0_tied": dict(n_layer=6, n_embd=288, n_ff=768, n_head=6, n_head_kv=6, head_dim=48, n_vocab=32000,
                           rms_eps=1e-5, rope_base=10000.0, rope_mode=0, type_embd=model.F32,
                           type_layers=model.Q8_0, type_output=-1),
}


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(cfg, n):
    return [int(t) for t in np.random.default_rng(11).integers(0, cfg["n_vocab"], n)]


def _rank_main(rank, world, port, shape, max_ctx, positions, mode, q, stop_after=None):
    import torch.distributed as dist
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["SYN_TP_P2P"] = "1" if mode == "peer_stores" else "0"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    tp = sess = None
    try:
        torch.cuda.set_device(rank)
        tp = syn.TP.from_torch_distributed(device=rank)
        cfg = SHAPES[shape]
        sess = syn.Session.synthetic(cfg, max_ctx=max_ctx, seed=5, device=rank, tp=tp)
        layout = sess.tp_layout()
        toks = _tokens(cfg, len(positions))
        if stop_after is not None:
            # every rank steps stop_after times; then rank 1 stops stepping (it stays up, runs nothing) and
            # rank 0 runs the next step, whose peer word reads must give up after SYN_TP_WAIT_MS
            import time
            for t, pos in list(zip(toks, positions))[:stop_after]:
                sess.step(t, pos)
            result = {}
            if rank == 0:
                t0 = time.perf_counter()
                try:
                    sess.step(toks[stop_after], positions[stop_after])
                    result["first"] = 0
                except syn.SynapseError as e:
                    result["first"] = e.status
                result["seconds"] = time.perf_counter() - t0
                try:
                    sess.step(toks[stop_after], positions[stop_after])
                    result["again"] = 0
                except syn.SynapseError as e:
                    result["again"] = e.status
                result["status"] = sess.tp_status()
            dist.barrier()  # rank 1 leaves the step loop only here, with nothing in flight
            q.put((rank, result))
            return
        logits, nxt = [], []
        for t, pos in zip(toks, positions):
            lg, n = sess.step(t, pos)
            logits.append(lg)
            nxt.append(n)
        sess.reset()
        gen = sess.generate(toks[:4], 0, 12)
        q.put((rank, dict(logits=np.stack(logits), next=nxt, gen=gen, layout=layout,
                          launches=sess.launches_per_step(), status=sess.tp_status())))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        if sess is not None:
            sess.close()
        if tp is not None:
            tp.close()
        dist.destroy_process_group()


def _run_world(world, shape, max_ctx, positions, mode, stop_after=None):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, shape, max_ctx, positions, mode, q, stop_after))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert not isinstance(got[r], str), f"rank {r}: {got[r]}"
    return got


def _one_gpu(shape, max_ctx, positions):
    cfg = SHAPES[shape]
    sess = syn.Session.synthetic(cfg, max_ctx=max_ctx, seed=5, device=0)
    toks = _tokens(cfg, len(positions))
    logits = np.stack([sess.step(t, pos)[0] for t, pos in zip(toks, positions)])
    sess.reset()
    gen = sess.generate(toks[:4], 0, 12)
    sess.close()
    return logits, gen


@pytest.mark.parametrize("mode", ["peer_stores", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("shape", list(SHAPES))
def test_tp_equals_one_gpu(world, shape, mode):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    cfg = SHAPES[shape]
    if cfg["n_head_kv"] % world or cfg["n_vocab"] % world or cfg["n_ff"] % world or cfg["n_embd"] % world:
        pytest.skip("world does not divide the model")
    max_ctx = 1024
    # single-chunk contexts, then positions past one 256-position chunk (several score CTAs per KV head)
    positions = list(range(8)) + [300, 301, 700, 1023]
    got = _run_world(world, shape, max_ctx, positions, mode)
    want, want_gen = _one_gpu(shape, max_ctx, positions)
    for r in range(world):
        g = got[r]
        assert g["layout"]["rank"] == r and g["layout"]["world"] == world
        # the 8B shape gathers by peer stores when asked; the tiny model's unfused ops always use NCCL
        want_p2p = mode == "peer_stores" and shape.startswith("8b")
        assert g["status"] == {"peer_stores": want_p2p, "wait_errors": 0}, g["status"]
        assert np.array_equal(g["logits"].view(np.uint32), want.view(np.uint32)), f"rank {r}"
        assert g["next"] == [int(np.argmax(x)) for x in want]
        assert np.array_equal(g["gen"], want_gen), f"rank {r} greedy tokens"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_long_context_equals_one_gpu(world):
    # positions past 4096 on the 8B-width model: every rank's logits and tokens are one GPU's bits
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    max_ctx = 4400
    positions = [0, 1, 2, 3, 2047, 4095, 4096, 4300]
    got = _run_world(world, "8b_2layer_q4_0", max_ctx, positions, "peer_stores")
    want, want_gen = _one_gpu("8b_2layer_q4_0", max_ctx, positions)
    for r in range(world):
        assert got[r]["status"] == {"peer_stores": True, "wait_errors": 0}, got[r]["status"]
        assert np.array_equal(got[r]["logits"].view(np.uint32), want.view(np.uint32)), f"rank {r}"
        assert np.array_equal(got[r]["gen"], want_gen), f"rank {r} greedy tokens"


def test_tp_rank_that_stops_stepping_fails_the_others_step(monkeypatch):
    # failure detection without a GPU fault: rank 1 stops between steps (alive, nothing in flight); rank 0's
    # next step gives up on rank 1's words after SYN_TP_WAIT_MS and returns SYN_ERR_TIMEOUT (5), and the
    # session stays failed; both ranks then close normally
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    monkeypatch.setenv("SYN_TP_WAIT_MS", "100")
    got = _run_world(2, "8b_2layer_q4_0", 64, [0, 1, 2, 3, 4], "peer_stores", stop_after=3)
    r0 = got[0]
    assert r0["first"] == 5 and r0["again"] == 5, r0
    assert r0["status"]["peer_stores"] and r0["status"]["wait_errors"] >= 1, r0
    assert r0["seconds"] < 30, r0


def test_tp_word_wait_gives_up_and_counts():
    # one GPU: a kernel reads gathered words whose epoch never arrives; every read gives up after the limit
    # and counts an error instead of waiting forever
    import ctypes
    import time
    L = syn.lib()
    L.syn_check_tp_wait.argtypes = [ctypes.c_uint, ctypes.POINTER(ctypes.c_int)]
    errors = ctypes.c_int(-1)
    t0 = time.perf_counter()
    assert L.syn_check_tp_wait(5000, ctypes.byref(errors)) == 0
    assert errors.value >= 1
    assert time.perf_counter() - t0 < 10
