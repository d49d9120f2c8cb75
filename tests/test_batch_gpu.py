"""run(batch) through the session's C ABI: prefill chunks of one sequence and
one decode token for each of several sequences.

The reference's G1 contract (tests/sdk/llama_prefill.cpp:20): a prompt run in
chunks gives the logits (and KV rows) a token-by-token decode gives. Here the
batched GEMV (integer tensor cores from 3 rows) and the attention over several
queries give every row the bits of a single-token step, so chunked prefill and
batched decode must equal token-by-token decode bit for bit, and the oracle
within the north star's logit tolerance (1e-2 * std)."""
import numpy as np
import pytest

import oracle as orc
from synapse_b200 import model

pytestmark = pytest.mark.gpu
syn = pytest.importorskip("synapse_b200")
torch = pytest.importorskip("torch")

SMALL = dict(n_layer=2, n_embd=256, n_ff=768, n_head=8, n_head_kv=2, head_dim=32, n_vocab=3000, rms_eps=1e-5,
             rope_base=10000.0)
SMALL_CFG = dict(SMALL, type_embd=syn.Q4_0, type_layers=syn.Q4_0, type_output=syn.Q8_0)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_chunked_prefill_equals_token_by_token():
    # G1: 40 prompt tokens in chunks of 16, 16 and 8 against one token at a time (the step graph)
    prompt = np.random.default_rng(1).integers(0, SMALL["n_vocab"], 40)
    a = syn.Session.synthetic_ex(SMALL_CFG, max_ctx=128, max_batch=16, seed=3)
    b = syn.Session.synthetic(SMALL_CFG, max_ctx=128, seed=3)
    for p0 in (0, 16, 32):
        chunk = prompt[p0:p0 + 16]
        got, nxt = a.prefill(chunk, p0)
    for pos, t in enumerate(prompt):
        want, want_nxt = b.step(int(t), pos)
    assert np.array_equal(bits(got), bits(want))
    assert nxt == want_nxt
    row = SMALL["n_head_kv"] * SMALL["head_dim"]
    for layer in range(SMALL["n_layer"]):
        for which in (0, 1):
            ka = syn.copy_to_host(a.kv_ptr(layer, which), 40 * row * 2, np.uint16)
            kb = syn.copy_to_host(b.kv_ptr(layer, which), 40 * row * 2, np.uint16)
            assert np.array_equal(ka, kb), (layer, which)
    # and the next decode steps continue identically
    for pos in range(40, 44):
        la, na = a.prefill([nxt], pos)
        lb, nb = b.step(nxt, pos)
        assert np.array_equal(bits(la), bits(lb)) and na == nb
        nxt = na
    a.close()
    b.close()


def test_prefill_matches_the_oracle():
    cfg = dict(SMALL, n_layer=1)
    w = model.random_llama_weights(cfg, seed=5, type_layers=model.Q4_0, type_embd=model.Q4_0, tied=False,
                                   type_output=model.Q8_0)
    import os
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        model.write_llama_gguf(path, cfg, w, context_length=64)
        sess = syn.Session.open_ex(path, max_ctx=64, max_batch=12)
        prompt = [int(t) for t in np.random.default_rng(2).integers(0, cfg["n_vocab"], 12)]
        got, nxt = sess.prefill(prompt, 0)
        ref = orc.Llama(cfg, w, max_ctx=64)
        for pos, t in enumerate(prompt):
            want = ref.step(t, pos)
        assert np.max(np.abs(got - want)) <= 1e-2 * np.std(want)
        assert np.array_equal(bits(got), bits(want))  # the same arithmetic as the oracle's, token by token
        sess.close()


@pytest.mark.parametrize("n_seq", [2, 3, 8])
def test_batched_decode_equals_each_sequence_alone(n_seq):
    # one token for each of n sequences (different prompts and positions) in one call, against each sequence
    # decoded alone through the step graph
    rng = np.random.default_rng(n_seq)
    lens = [int(x) for x in rng.integers(5, 40, n_seq)]
    prompts = [rng.integers(0, SMALL["n_vocab"], L) for L in lens]
    batched = syn.Session.synthetic_ex(SMALL_CFG, max_ctx=64, max_seqs=n_seq, max_batch=max(n_seq, 16), seed=7)
    nexts = []
    for i, p in enumerate(prompts):
        for p0 in range(0, len(p), batched.max_batch):  # chunks of at most max_batch tokens
            _, nx = batched.prefill(p[p0:p0 + batched.max_batch], p0, seq=i)
        nexts.append(nx)
    toks, pos = list(nexts), list(lens)
    got_steps = []
    for step in range(3):
        lg, nx = batched.step_batch(toks, pos)
        got_steps.append(lg)
        toks, pos = [int(t) for t in nx], [p + 1 for p in pos]
    for i, p in enumerate(prompts):
        alone = syn.Session.synthetic(SMALL_CFG, max_ctx=64, seed=7)
        alone.generate(p, 0, len(p))
        t = nexts[i]
        for step in range(3):
            want, wn = alone.step(t, lens[i] + step)
            assert np.array_equal(bits(got_steps[step][i]), bits(want)), (i, step)
            t = wn
        alone.close()
    batched.close()


def test_batch_calls_reject_out_of_range():
    sess = syn.Session.synthetic_ex(SMALL_CFG, max_ctx=16, max_seqs=2, max_batch=4, seed=1)
    with pytest.raises(syn.SynapseError) as e:
        sess.prefill([1, 2, 3, 4, 5], 0)  # more tokens than max_batch
    assert e.value.status == 8
    with pytest.raises(syn.SynapseError) as e:
        sess.prefill([1, 2], 15)  # past max_ctx
    assert e.value.status == 8
    with pytest.raises(syn.SynapseError) as e:
        sess.step_batch([1, 2, 3], [0, 0, 0])  # more sequences than max_seqs
    assert e.value.status == 8
    one = syn.Session.synthetic(SMALL_CFG, max_ctx=16, seed=1)
    with pytest.raises(syn.SynapseError) as e:
        one.prefill([1, 2], 0)  # a session opened without batching
    assert e.value.status == 2
    one.close()
    sess.close()


LLAMA70B_1L = dict(n_layer=1, n_embd=8192, n_ff=28672, n_head=64, n_head_kv=8, head_dim=128, n_vocab=128256,
                   rms_eps=1e-5, rope_base=500000.0)


def test_config5_70b_shape_one_layer_against_oracle():
    # BASELINE config 5's widths (one of the 80 layers): Q4_0 everywhere, batched decode of 3 sequences
    cfg = dict(LLAMA70B_1L, type_embd=syn.Q4_0, type_layers=syn.Q4_0, type_output=syn.Q4_0)
    sess = syn.Session.synthetic_ex(cfg, max_ctx=32, max_seqs=3, max_batch=4, seed=70)
    weights = {}
    from .test_session_gpu import session_weights
    weights = session_weights(sess, 1)
    refs = [orc.Llama(LLAMA70B_1L, weights, max_ctx=32) for _ in range(3)]
    toks = [11, 22222, 120000]
    for pos in range(3):
        got, nxt = sess.step_batch(toks, [pos] * 3)
        for i in range(3):
            want = refs[i].step(toks[i], pos)
            assert np.max(np.abs(got[i] - want)) <= 1e-2 * np.std(want), (pos, i)
            if int(np.argmax(want)) != nxt[i]:
                gap = np.partition(want, -2)[-2:]
                assert gap[1] - gap[0] < 1e-2 * np.std(want)
        toks = [int(t) for t in nxt]
    sess.close()
