"""syn_attention_noalloc, the attention entry point for callers that cannot
allocate device memory (a host that owns the device memory budget and lends a
plugin only its tensors, or a decode loop that may not allocate once it runs).

It must give what syn_attention gives with caller scratch, on consecutive
calls that share its static scratch array. This file is named to be collected
last, so a run that stops at the first failure has run every other test first;
it also passes alone in a fresh process.
"""
import ctypes
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
syn = pytest.importorskip("synapse_b200")


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def make_case(seed, n_q, n_head, n_kv, hd, L):
    g = torch.Generator(device="cpu").manual_seed(seed)
    row = n_kv * hd
    kc = torch.randn(n_q, L * row, generator=g).half().view(torch.int16)
    vc = torch.randn(n_q, L * row, generator=g).half().view(torch.int16)
    q = torch.randn(n_q, n_head * hd, generator=g)
    k = torch.randn(n_q, row, generator=g)
    v = torch.randn(n_q, row, generator=g)
    pos = torch.full((n_q,), L - 1, dtype=torch.int32)
    return [t.cuda() for t in (q, k, v, kc, vc, pos)]


def call(fn_name, q, k, v, kc, vc, pos, n_head, n_kv, hd, L, scratch=None, order=0):
    out = torch.empty(q.shape[0], n_head * hd, device="cuda")
    a = syn.AttentionArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
                          out.data_ptr(), scratch.data_ptr() if scratch is not None else None, kc.shape[1],
                          q.shape[0], n_head, n_kv, hd, L, 1, 1, 0, 500000.0 ** (-2.0 / hd), 1.0 / math.sqrt(hd),
                          None, None, None, order)
    st = getattr(syn.lib(), fn_name)(ctypes.byref(a), syn._stream())
    return st, out


@pytest.mark.parametrize("order", [0, 1])
@pytest.mark.parametrize("n_q,n_head,n_kv,hd,L", [(1, 32, 8, 128, 4096), (3, 6, 6, 48, 256)])
def test_noalloc_matches_attention_on_consecutive_calls(n_q, n_head, n_kv, hd, L, order):
    for seed in (1, 2):  # two calls in a row share the static scratch
        q, k, v, kc, vc, pos = make_case(seed, n_q, n_head, n_kv, hd, L)
        kc2, vc2 = kc.clone(), vc.clone()
        scratch = syn.empty_bytes(syn.attention_scratch_bytes(n_q, n_head, n_kv, hd, L))
        st, want = call("syn_attention", q, k, v, kc, vc, pos, n_head, n_kv, hd, L, scratch, order)
        assert st == 0
        st, got = call("syn_attention_noalloc", q, k, v, kc2, vc2, pos, n_head, n_kv, hd, L, order=order)
        assert st == 0, syn.lib().syn_last_error()
        torch.cuda.synchronize()
        assert rel_l2(got.cpu().numpy(), want.cpu().numpy()) < 1e-3  # the north star's attention bound
        assert torch.equal(got, want)  # the same kernels on the same inputs: the same bits
        assert torch.equal(kc, kc2) and torch.equal(vc, vc2)  # the same rows appended


def test_noalloc_rejects_shapes_beyond_its_scratch():
    n_q, n_head, n_kv, hd, L = 32, 32, 8, 128, 32768
    assert syn.attention_scratch_bytes(n_q, n_head, n_kv, hd, L) > 16 << 20
    a = syn.AttentionArgs(0, 0, 0, 0, 0, 0, 0, None, 0, n_q, n_head, n_kv, hd, L, 1, 1, 0, 1.0, 1.0, None, None)
    assert syn.lib().syn_attention_noalloc(ctypes.byref(a), syn._stream()) == 1
    assert b"16 MiB" in syn.lib().syn_last_error()
