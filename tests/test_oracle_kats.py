"""The CPU restatement (oracle/) pinned against the reference's own
known-answer tests (tests/golden/kats.json, transcribed from the reference's
test sources with file:line citations)."""
import json
import math
import os

import numpy as np
import pytest

import oracle as orc

HERE = os.path.dirname(os.path.abspath(__file__))
KATS = json.load(open(os.path.join(HERE, "golden", "kats.json")))


def _f(v):
    if v == "inf":
        return math.inf
    if v == "-inf":
        return -math.inf
    return v


def arr(v, dtype):
    return np.array([_f(x) for x in v], dtype=dtype)


def run_oracle(k):
    dt = np.float32 if k["dtype"] == "f32" else np.float64
    if k["kind"] == "copy_strided":
        return orc.copy_strided(arr(k["src"], dt), k["shape"], k["strides"], k["offset"]), None
    a, b = arr(k["a"], dt), arr(k["b"], dt)
    r = orc.contract(k["alg"], a, k["shape_a"], k["strides_a"], k["modes_a"], b, k["shape_b"],
                     k["strides_b"], k["modes_b"], k["shape_c"], k["modes_c"],
                     argmax=k.get("with_argmax", False))
    return r if isinstance(r, tuple) else (r, None)


def check_kat(k, c, am):
    """Shared by the oracle test here and the device test (test_gpu_contract.py::test_reference_kat_on_device)."""
    dt = np.float32 if k["dtype"] == "f32" else np.float64
    n = int(np.prod(k["shape_c"])) if k["kind"] == "contract" and k["shape_c"] else None
    if k["kind"] == "contract":
        assert c.shape == (max(n, 1) if n is not None else 1,)
    if k.get("expected") is not None:
        np.testing.assert_array_equal(c, arr(k["expected"], dt))
    if k.get("expected_partial"):
        for i, v in k["expected_partial"].items():
            assert c[int(i)] == v
    if k.get("expected_approx"):
        assert np.all(np.abs(c - np.array(k["expected_approx"], dtype=dt)) < 1e-6)
    if k.get("expected_argmax") is not None:
        np.testing.assert_array_equal(am, np.array(k["expected_argmax"], dtype=np.uint32))
    if k.get("with_argmax"):
        assert am is not None and am.shape == c.shape


@pytest.mark.parametrize("k", KATS, ids=[k["name"] for k in KATS])
def test_oracle_kat(k):
    c, am = run_oracle(k)
    check_kat(k, c, am)


def test_oracle_first_k_wins_and_nan_rule():
    # tropical.rs:57-63: acc >= p keeps acc -> first k wins on ties; a NaN
    # accumulator is replaced by the next product.
    a = np.array([1, 1, 1], dtype=np.float32)          # 1 x 3
    b = np.array([2, 2, 2], dtype=np.float32)          # 3 x 1
    c, am = orc.gemm("maxplus", a, b, 1, 3, 1, argmax=True)
    assert c[0] == 3 and am[0] == 0
    a = np.array([np.nan, 1, 0], dtype=np.float32)
    c, am = orc.gemm("maxplus", a, np.zeros(3, np.float32), 1, 3, 1, argmax=True)
    assert c[0] == 1 and am[0] == 1
    c, am = orc.gemm("minplus", np.array([5, 3, 3], np.float32), np.zeros(3, np.float32), 1, 3, 1,
                     argmax=True)
    assert c[0] == 3 and am[0] == 1


def test_oracle_unary_trace_and_argmax():
    # ii -> (trace) Standard; ij -> i MaxPlus with argmax = linear input index
    x = np.array([1, 2, 3, 4], dtype=np.float64)
    y = orc.unary("standard", x, [0, 0], [2, 2], [1, 2], [], {0: 2})
    assert y[0] == 5
    y, am = orc.unary("maxplus", np.array([1, 5, 7, 2], np.float32), [0, 1], [2, 2], [1, 2], [0],
                      {0: 2, 1: 2}, argmax=True)
    np.testing.assert_array_equal(y, [7, 5])
    np.testing.assert_array_equal(am, [2, 1])


def test_oracle_rng_is_deterministic():
    u = orc.uniform(0x5EED, 5000)
    assert u.dtype == np.float32 and u.min() >= -1 and u.max() < 1
    np.testing.assert_array_equal(u, orc.uniform(0x5EED, 5000))
    assert abs(float(u.mean())) < 0.05
