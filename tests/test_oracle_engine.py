"""The oracle's restated einsum engine and gradient tape (oracle/engine.py),
pinned against the reference's own engine-level known answers."""
import itertools

import numpy as np
import pytest

import engine as oe
from conftest import load_pkg



def _einsum_mod():
    load_pkg()
    import importlib
    return importlib.import_module("omeinsum_b200.einsum")


BW = "tests/suites/backward.rs"
# (cite, a, b, expected value, expected grad_a, expected grad_b)
TROPICAL_GRAD_KATS = [
    (BW + ":169-197", [1, 2, 3, 4], [1, 2, 3, 4], [5, 6, 7, 8], [0, 0, 2, 2], [0, 2, 0, 2]),
    (BW + ":199-227", [0, 10, 20, 0], [1, 1, 1, 1], [21, 11, 21, 11], [0, 2, 2, 0], None),
    (BW + ":229-258", [5, 1, 1, 5], [1, 5, 5, 1], [6, 10, 10, 6], [2, 1, 0, 1], [1, 1, 2, 0]),
]


@pytest.mark.parametrize("kat", TROPICAL_GRAD_KATS, ids=[k[0] for k in TROPICAL_GRAD_KATS])
def test_oracle_tropical_gradient_kats(kat):
    _, a, b, val, ga, gb = kat
    ts = [np.array(a, np.float32), np.array(b, np.float32)]
    cost, grads = oe.cost_and_gradient("maxplus", ts, [[0, 1], [1, 2]], [0, 2], {0: 2, 1: 2, 2: 2},
                                       [0, 1], [[0, 2]], np.ones(4, np.float32))
    np.testing.assert_array_equal(cost, val)
    np.testing.assert_array_equal(grads[0], ga)
    if gb is not None:
        np.testing.assert_array_equal(grads[1], gb)


def pentagon():
    # tests/suites/showcase.rs:1031-1173: weights [3,5,1,4,2], optimum 9 = {1,3}
    w = [3.0, 5.0, 1.0, 4.0, 2.0]
    edges = [(0, 1), (1, 2), (2, 3), (3, 4), (4, 0)]
    ixs = [[v] for v in range(5)] + [[u, v] for u, v in edges]
    ts = [np.array([0.0, x]) for x in w] + [np.array([0.0, 0.0, 0.0, -np.inf])] * 5
    return ixs, ts, edges


def test_oracle_mis_pentagon_value_and_configuration():
    E = _einsum_mod()
    ixs, ts, edges = pentagon()
    sizes = {v: 2 for v in range(5)}
    tree = E.greedy_tree(ixs, [], sizes)
    ch, niy = E.encode_tree(tree, ixs, [])
    cost, grads = oe.cost_and_gradient("maxplus", ts, ixs, [], sizes, ch, niy, np.ones(1))
    assert cost[0] == 9.0
    config = [int(np.argmax(g)) for g in grads[:5]]
    assert [v for v in range(5) if config[v]] == [1, 3]


def test_oracle_standard_gradient_matches_finite_difference():
    E = _einsum_mod()
    rng = np.random.default_rng(3)
    ixs = [[0, 1], [1, 2], [2, 0]]
    sizes = {0: 3, 1: 4, 2: 2}
    ts = [rng.standard_normal(int(np.prod([sizes[l] for l in ix]))) for ix in ixs]
    tree = E.greedy_tree(ixs, [], sizes)
    ch, niy = E.encode_tree(tree, ixs, [])
    cost, grads = oe.cost_and_gradient("standard", ts, ixs, [], sizes, ch, niy, np.ones(1))
    eps = 1e-6
    for t in range(3):
        for q in range(len(ts[t])):
            tp = [x.copy() for x in ts]
            tp[t][q] += eps
            cp = oe.einsum("standard", tp, ixs, [], sizes, ch, niy)
            assert abs((cp[0] - cost[0]) / eps - grads[t][q]) < 1e-4


def test_oracle_mis_small_graph_matches_enumeration():
    E = _einsum_mod()
    ixs, iy, sizes, ts, edges = E.mis_network(12, 5, np.float64)
    tree = E.greedy_tree(ixs, iy, sizes)
    ch, niy = E.encode_tree(tree, ixs, iy)
    cost, grads = oe.cost_and_gradient("maxplus", ts, ixs, iy, sizes, ch, niy, np.ones(1))
    best = 0
    for cfg in itertools.product([0, 1], repeat=12):
        if all(not (cfg[u] and cfg[v]) for u, v in edges):
            best = max(best, sum(cfg))
    assert cost[0] == best
    sel = [int(np.argmax(g)) for g in grads[:12]]
    assert sum(sel) == best and all(not (sel[u] and sel[v]) for u, v in edges)
