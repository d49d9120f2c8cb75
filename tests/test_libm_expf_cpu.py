"""The build step's table of expf exceptions (synapse_b200/csrc/libm_expf_scan.c)
against the host C library, on the CPU.

The reference calls std::exp on float (kernels/elementwise.hpp:79, :188), i.e.
the host library's expf, which is accurate to about 0.502 ulp rather than
correctly rounded. The device expf is correctly rounded except on the inputs of
this table, where it returns the host library's other neighbour instead. Here:
the table's inputs are (nearly all) where the host expf is not the correctly
rounded value, and random inputs outside it are where it is."""
import os
import re

import numpy as np
import pytest

import oracle as orc

INC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "synapse_b200", "_build",
                   "libm_expf_exc.inc")


def table():
    if not os.path.exists(INC):
        pytest.skip("the library has not been built (synapse_b200.buildlib.build())")
    with open(INC) as f:
        text = f.read()
    body = text[text.index("{") + 1:text.rindex("}")]
    keys = np.array([int(v, 16) for v in re.findall(r"0x[0-9a-f]+", body)], dtype=np.uint32)
    count = int(re.search(r"SYN_EXPF_EXC_COUNT (\d+)", text).group(1))
    probes = int(re.search(r"SYN_EXPF_EXC_PROBES (\d+)", text).group(1))
    return keys, count, probes, int(re.search(r"SYN_EXPF_EXC_BITS (\d+)", text).group(1))


def correctly_rounded(x):
    return np.exp(x.astype(np.float64)).astype(np.float32)  # exact but within ~2^-29 ulp of a midpoint


def test_table_inputs_are_where_the_host_expf_is_not_correctly_rounded():
    keys, count, probes, bits = table()
    assert keys.size == count > 0 and 2 * count <= 1 << bits
    x = keys.view(np.float32)
    assert np.all((x >= -40.0) & (x <= 88.72284))
    host, cr = orc.expf(x), correctly_rounded(x)
    diff = host.view(np.int32).astype(np.int64) - cr.view(np.int32).astype(np.int64)
    assert np.all(np.abs(diff) <= 1)
    assert np.count_nonzero(diff) >= 0.999 * x.size


def test_outside_the_table_the_host_expf_is_correctly_rounded():
    keys, _, _, _ = table()
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.uniform(-40.0, 0.0, 1 << 21), rng.uniform(0.0, 88.7, 1 << 20)]).astype(np.float32)
    x = x[~np.isin(x.view(np.uint32), keys)]
    host, cr = orc.expf(x), correctly_rounded(x)
    assert np.count_nonzero(host.view(np.uint32) != cr.view(np.uint32)) <= 2


def test_hash_table_probes_stay_within_the_bound():
    keys, count, probes, bits = table()
    with open(INC) as f:
        text = f.read()
    body = text[text.index("{") + 1:text.rindex("}")]
    slots = np.array([int(v, 0) for v in re.findall(r"0x[0-9a-f]+|0(?=,)", body)], dtype=np.uint64)
    assert slots.size == 1 << bits
    mask = (1 << bits) - 1
    for k in keys[::97].astype(np.uint64):
        h = int((k * 0x9E3779B1) & 0xffffffff) >> (32 - bits)
        assert any(int(slots[(h + i) & mask]) == int(k) for i in range(probes))
