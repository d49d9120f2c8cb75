"""Tensor-parallel sharding on the CPU (no GPU).

The product's rank layouts (syn_tp_layout_of, the same function the session
shards with) must partition every sharded dimension; and a gloo run over 2 or
4 ranks of the oracle's per-op functions over those shares, all-gathering at the five
points the sharded session gathers (attention output, residual after O,
silu * up, residual after down, logits), must reproduce the one-process
oracle's logits bit for bit. That is the reference's D1 contract
(tests/sdk/llama_threads.cpp:32) carried across ranks: row sharding never
changes how an output element is computed."""
import datetime
import os
import socket

import numpy as np
import pytest

import oracle as orc
import synapse_b200 as syn
from synapse_b200 import model

TINY = dict(n_layer=2, n_embd=64, n_ff=128, n_head=4, n_head_kv=2, head_dim=16, n_vocab=64, rms_eps=1e-5,
            rope_base=10000.0)
# four KV heads: shards over 2 and 4 ranks
TINY_KV4 = dict(n_layer=2, n_embd=64, n_ff=128, n_head=8, n_head_kv=4, head_dim=8, n_vocab=64, rms_eps=1e-5,
                rope_base=10000.0)
LLAMA_8B = dict(n_layer=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, head_dim=128, n_vocab=128256,
                rms_eps=1e-5, rope_base=500000.0)
LLAMA_70B = dict(n_layer=80, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8, head_dim=128, n_vocab=128256,
                 rms_eps=1e-5, rope_base=500000.0)


@pytest.mark.parametrize("cfg", [TINY, LLAMA_8B, LLAMA_70B], ids=["tiny", "8b", "70b"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_layouts_partition_every_dimension(cfg, world):
    if cfg["n_head_kv"] % world:
        pytest.skip("world does not divide the KV heads")
    parts = [syn.tp_layout(cfg, r, world) for r in range(world)]
    G = cfg["n_head"] // cfg["n_head_kv"]
    for key, total in (("head", cfg["n_head"]), ("kv_head", cfg["n_head_kv"]), ("embd", cfg["n_embd"]),
                       ("ff", cfg["n_ff"]), ("vocab", cfg["n_vocab"])):
        first = key + "0"
        count = "n_" + ("kv" if key == "kv_head" else key)
        nxt = 0
        for r, p in enumerate(parts):
            assert p["rank"] == r and p["world"] == world
            assert p[first] == nxt, (key, r)  # contiguous, in rank order (the all-gather's order)
            assert p[count] == total // world
            nxt += p[count]
        assert nxt == total
    for p in parts:  # a rank's query heads are exactly its KV heads' groups
        assert p["head0"] == p["kv_head0"] * G and p["n_head"] == p["n_kv"] * G


def test_layout_rejects_uneven_or_bad_worlds():
    with pytest.raises(syn.SynapseError) as e:
        syn.tp_layout(LLAMA_70B, 0, 3)  # 8 KV heads over 3 ranks
    assert e.value.status == 2
    for rank, world in ((0, 0), (2, 2), (-1, 2)):
        with pytest.raises(syn.SynapseError) as e:
            syn.tp_layout(TINY, rank, world)
        assert e.value.status == 1


def _rows(w, name, r0, n):
    ty, arr = w[name]
    return ty, np.ascontiguousarray(np.asarray(arr).reshape(np.asarray(arr).shape[0], -1)[r0:r0 + n])


def sharded_decode(cfg, w, tokens, max_ctx, rank, world, gather):
    """The session's sharded step with the oracle's ops: this rank's rows and
    heads (syn_tp_layout_of), whole inputs, gathers in rank order. Returns
    the gathered logits of every step."""
    P = syn.tp_layout(cfg, rank, world)
    d, hd, ff = cfg["n_embd"], cfg["head_dim"], cfg["n_ff"]
    qall = cfg["n_head"] * hd
    theta = orc.rope_theta_scale(cfg["rope_base"], hd)
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    e0, ne = P["embd0"], P["n_embd"]
    kc = [np.zeros(max_ctx * P["n_kv"] * hd, np.uint16) for _ in range(cfg["n_layer"])]
    vc = [np.zeros(max_ctx * P["n_kv"] * hd, np.uint16) for _ in range(cfg["n_layer"])]
    out = []
    for pos, tok in enumerate(tokens):
        x = np.asarray(w["token_embd"][1], np.float32).reshape(cfg["n_vocab"], d)[tok].copy()
        for l in range(cfg["n_layer"]):
            b = f"blk.{l}."
            h = orc.rms_norm(x, w[b + "attn_norm"][1], cfg["rms_eps"])
            q = orc.gemv(*_rows(w, b + "attn_q", P["head0"] * hd, P["n_head"] * hd), P["n_head"] * hd, d, h)
            k = orc.gemv(*_rows(w, b + "attn_k", P["kv_head0"] * hd, P["n_kv"] * hd), P["n_kv"] * hd, d, h)
            v = orc.gemv(*_rows(w, b + "attn_v", P["kv_head0"] * hd, P["n_kv"] * hd), P["n_kv"] * hd, d, h)
            qr = orc.rope(q, hd, pos, theta)
            kr = orc.rope(k, hd, pos, theta)
            a = orc.attention(qr, kr, v, kc[l], vc[l], max_ctx, P["n_kv"], hd, pos, P["n_head"], scale)
            attn = gather(a)
            assert attn.size == qall
            o = orc.gemv(*_rows(w, b + "attn_output", e0, ne), ne, qall, attn)
            x = gather(o + x[e0:e0 + ne])
            h = orc.rms_norm(x, w[b + "ffn_norm"][1], cfg["rms_eps"])
            g = orc.gemv(*_rows(w, b + "ffn_gate", P["ff0"], P["n_ff"]), P["n_ff"], d, h)
            u = orc.gemv(*_rows(w, b + "ffn_up", P["ff0"], P["n_ff"]), P["n_ff"], d, h)
            act = gather(orc.silu(g) * u)
            dn = orc.gemv(*_rows(w, b + "ffn_down", e0, ne), ne, ff, act)
            x = gather(dn + x[e0:e0 + ne])
        hl = orc.rms_norm(x, w["output_norm"][1], cfg["rms_eps"])
        out.append(gather(orc.gemv(*_rows(w, "output", P["vocab0"], P["n_vocab"]), P["n_vocab"], d, hl)))
    return out


def _model(cfg, type_layers):
    return model.random_llama_weights(cfg, seed=7, type_layers=type_layers, type_embd=model.F32, tied=False,
                                      type_output=model.Q8_0)


def _tokens(cfg, n):
    return [int(t) for t in np.random.default_rng(3).integers(0, cfg["n_vocab"], n)]


def _rank_main(rank, world, port, type_layers, n_steps, cfg_name, q):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        def gather(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            return torch.cat(parts).numpy()
        cfg = CONFIGS[cfg_name]
        w = _model(cfg, type_layers)
        logits = sharded_decode(cfg, w, _tokens(cfg, n_steps), n_steps, rank, world, gather)
        q.put((rank, np.stack(logits)))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CONFIGS = {"tiny": TINY, "tiny_kv4": TINY_KV4}


@pytest.mark.parametrize("world,cfg_name,type_layers", [(2, "tiny", model.Q8_0), (2, "tiny", model.Q4_0),
                                                        (4, "tiny_kv4", model.Q4_0)],
                         ids=["w2-q8_0", "w2-q4_0", "w4-q4_0"])
def test_sharded_logits_equal_one_process(world, cfg_name, type_layers):
    import torch.multiprocessing as mp
    n_steps = 6
    cfg = CONFIGS[cfg_name]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, type_layers, n_steps, cfg_name, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
    # every rank holds the same gathered logits
    for r in range(1, world):
        assert np.array_equal(got[0].view(np.uint32), got[r].view(np.uint32))
    w = _model(cfg, type_layers)
    ref = orc.Llama(cfg, w, max_ctx=n_steps)
    want = np.stack([ref.step(t, pos) for pos, t in enumerate(_tokens(cfg, n_steps))])
    assert np.array_equal(got[0].view(np.uint32), want.view(np.uint32))


def _leaving_rank_main(rank, world, port, n_steps, leave_after, q):
    """Rank 1 decodes leave_after steps of the sharded model and leaves (between steps: nothing of its own is in
    flight). Rank 0 carries on; its next gather must end with an error within the group's short timeout, not
    wait forever, and rank 0 must then leave cleanly."""
    import time

    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))

    def gather(a):
        t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return torch.cat(parts).numpy()

    cfg = TINY
    w = _model(cfg, model.Q8_0)
    toks = _tokens(cfg, n_steps)
    result = {"rank": rank}
    try:
        if rank == 1:
            sharded_decode(cfg, w, toks[:leave_after], n_steps, rank, world, gather)
            result["left_after"] = leave_after
            q.put((rank, result))
            return  # leaves the group between steps
        t0 = time.perf_counter()
        try:
            sharded_decode(cfg, w, toks, n_steps, rank, world, gather)
            result["error"] = None
        except Exception as e:  # the gather with the departed rank
            result["error"] = type(e).__name__
        result["seconds"] = time.perf_counter() - t0
        q.put((rank, result))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_leaving_between_steps_ends_the_others_next_gather_with_an_error():
    # failure detection on the host, without a GPU: the group's short timeout turns the departed rank into an
    # error on the next gather of every other rank
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_rank_main, args=(r, 2, port, 6, 2, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert got[1]["left_after"] == 2
    assert got[0]["error"] is not None, got[0]
    assert got[0]["seconds"] < 60, got[0]
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
