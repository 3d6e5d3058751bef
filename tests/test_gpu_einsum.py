"""The device einsum engine (om_b200_einsum / om_b200_einsum_backward)
against the oracle engine (oracle/engine.py) and the reference's engine-level
known answers.  Tropical values and gradients bit-exact; Standard within
relative 1e-12 (f64) / 1e-5 (f32) of the oracle."""
import itertools

import numpy as np
import pytest

import engine as oe
from conftest import load_pkg
from test_oracle_engine import TROPICAL_GRAD_KATS, pentagon

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    om = load_pkg()
    import importlib
    E = importlib.import_module("omeinsum_b200.einsum")
    be = om.B200(0)
    yield om, E, be
    be.close()


def run_both(E, be, alg, ixs, iy, sizes, ts, dy=None, tree=None):
    ein = E.Einsum(ixs, iy, sizes)
    if tree is not None:
        ein.set_contraction_tree(tree)
    ch, niy = ein.encoded()
    dev_ts = [be.from_slice(t) for t in ts]
    if dy is None:
        val = ein.execute(be, alg, dev_ts).to_vec()
        ref = oe.einsum(alg, ts, ixs, iy, sizes, ch, niy)
        return val, ref, None, None
    c, g = ein.cost_and_gradient(be, alg, dev_ts, dy=dy)
    rc, rg = oe.cost_and_gradient(alg, ts, ixs, iy, sizes, ch, niy, np.asarray(dy, ts[0].dtype))
    return c.to_vec(), rc, [x.to_vec() for x in g], rg


@pytest.mark.parametrize("kat", TROPICAL_GRAD_KATS, ids=[k[0] for k in TROPICAL_GRAD_KATS])
def test_tropical_gradient_kats_on_device(env, kat):
    om, E, be = env
    _, a, b, val, ga, gb = kat
    ts = [np.array(a, np.float32), np.array(b, np.float32)]
    c, rc, g, rg = run_both(E, be, "maxplus", [[0, 1], [1, 2]], [0, 2], {0: 2, 1: 2, 2: 2}, ts,
                            dy=np.ones(4, np.float32), tree=(0, 1))
    np.testing.assert_array_equal(c, val)
    np.testing.assert_array_equal(g[0], ga)
    if gb is not None:
        np.testing.assert_array_equal(g[1], gb)


def test_mis_pentagon_on_device(env):
    om, E, be = env
    ixs, ts, edges = pentagon()
    c, rc, g, rg = run_both(E, be, "maxplus", ixs, [], {v: 2 for v in range(5)}, ts, dy=[1.0])
    assert c[0] == 9.0
    assert [v for v in range(5) if g[v][1] > g[v][0]] == [1, 3]


@pytest.mark.parametrize("n,seed", [(10, 1), (20, 2), (40, 3)])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_mis_networks_match_oracle(env, n, seed, dtype):
    om, E, be = env
    ixs, iy, sizes, ts, edges = E.mis_network(n, seed, dtype)
    c, rc, g, rg = run_both(E, be, "maxplus", ixs, iy, sizes, ts, dy=[1.0])
    np.testing.assert_array_equal(c, rc)
    for x, y in zip(g, rg):
        np.testing.assert_array_equal(x, y)
    sel = [int(x[1] > x[0]) for x in g[:n]]
    assert sum(sel) == int(c[0]) and all(not (sel[u] and sel[v]) for u, v in edges)


@pytest.mark.parametrize("n,seed", [(10, 4), (24, 5)])
def test_ising_networks_match_oracle(env, n, seed):
    om, E, be = env
    ixs, iy, sizes, ts, edges = E.ising_network(n, seed)
    c, rc, g, rg = run_both(E, be, "standard", ixs, iy, sizes, ts, dy=[1.0])
    assert abs(c[0] - rc[0]) <= 1e-12 * abs(rc[0])
    for x, y in zip(g, rg):
        assert np.all(np.abs(x - y) <= 1e-12 * np.max(np.abs(y)) + 1e-300)


@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul", "standard"])
def test_engine_normalisation_cases(env, alg):
    # labels only in one operand (traced), repeated labels (diagonal), a
    # free output label, an outer product and a final permutation
    om, E, be = env
    rng = np.random.default_rng(11)
    ixs = [[0, 0, 1, 5], [1, 2, 6], [2, 3], [3, 4]]
    iy = [4, 0]
    sizes = {0: 3, 1: 4, 2: 2, 3: 5, 4: 3, 5: 2, 6: 3}
    ts = [np.abs(rng.standard_normal(int(np.prod([sizes[l] for l in ix])))).astype(np.float64)
          for ix in ixs]
    dy = np.ones(9)
    c, rc, g, rg = run_both(E, be, alg, ixs, iy, sizes, ts, dy=dy)
    if alg == "standard":
        np.testing.assert_allclose(c, rc, rtol=1e-12)
        for x, y in zip(g, rg):
            np.testing.assert_allclose(x, y, rtol=1e-12, atol=1e-300)
    else:
        np.testing.assert_array_equal(c, rc)
        for x, y in zip(g, rg):
            np.testing.assert_array_equal(x, y)


@pytest.mark.parametrize("alg", ["maxplus", "standard"])
def test_unary_only_einsum(env, alg):
    om, E, be = env
    x = np.arange(9, dtype=np.float64)
    c, rc, _, _ = run_both(E, be, alg, [[0, 0]], [], {0: 3}, [x])
    np.testing.assert_array_equal(c, rc)
    c, rc, _, _ = run_both(E, be, alg, [[0, 1]], [1], {0: 3, 1: 3}, [x])
    np.testing.assert_array_equal(c, rc)


def test_mis_150_config3(env):
    """MIS on a seeded 3-regular graph with 150 vertices,
    MaxPlus f32, greedy order, argmax backward recovers a configuration."""
    om, E, be = env
    ixs, iy, sizes, ts, edges = E.mis_network(150, 0x5EED)
    ein = E.Einsum(ixs, iy, sizes).optimize_greedy()
    ch, niy = ein.encoded()
    dev = [be.from_slice(t) for t in ts]
    c, g = ein.cost_and_gradient(be, "maxplus", dev, dy=[1.0])
    val = c.to_vec()[0]
    assert val == oe.einsum("maxplus", ts, ixs, iy, sizes, ch, niy)[0]
    sel = [int(x.to_vec()[1] > 0) for x in g[:150]]
    assert sum(sel) == int(val)
    assert all(not (sel[u] and sel[v]) for u, v in edges)


# ---- values-only tapes: the backward recomputes the argmax it needs ------
def both_tapes(E, be, alg, ixs, iy, sizes, ts, dy, tree=None):
    ein = E.Einsum(ixs, iy, sizes)
    if tree is not None:
        ein.set_contraction_tree(tree)
    else:
        ein.optimize_greedy()
    dev = [be.from_slice(t) for t in ts]
    c1, g1 = ein.cost_and_gradient(be, alg, dev, dy=dy)
    c2, g2 = ein.cost_and_gradient(be, alg, dev, dy=dy, values_only=True)
    return (c1.to_vec(), [x.to_vec() for x in g1]), (c2.to_vec(), [x.to_vec() for x in g2])


@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul"])
def test_values_only_tape_normalisation_cases(env, alg):
    om, E, be = env
    rng = np.random.default_rng(12)
    ixs = [[0, 0, 1, 5], [1, 2, 6], [2, 3], [3, 4]]
    iy = [4, 0]
    sizes = {0: 3, 1: 4, 2: 2, 3: 5, 4: 3, 5: 2, 6: 3}
    ts = [np.abs(rng.standard_normal(int(np.prod([sizes[l] for l in ix])))).astype(np.float64)
          for ix in ixs]
    (c1, g1), (c2, g2) = both_tapes(E, be, alg, ixs, iy, sizes, ts, np.arange(1.0, 10.0))
    np.testing.assert_array_equal(c1, c2)
    for x, y in zip(g1, g2):
        np.testing.assert_array_equal(x, y)


@pytest.mark.parametrize("kind", ["ties", "specials"])
@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul"])
def test_values_only_tape_ties_and_special_values(env, alg, kind):
    # integer-valued inputs (many equal maxima: first index must win) and
    # inputs with NaN / +-inf / -0 (the sequential rule decides)
    om, E, be = env
    rng = np.random.default_rng(13)
    ixs = [[0, 1], [1, 2, 3], [3, 4], [4, 0, 5], [5]]
    iy = [2]
    sizes = {0: 4, 1: 40, 2: 3, 3: 50, 4: 6, 5: 70}
    ts = []
    for ix in ixs:
        n = int(np.prod([sizes[l] for l in ix]))
        x = rng.integers(-2, 3, n).astype(np.float32)
        if kind == "specials":
            pick = rng.random(n)
            x[pick < 0.02] = np.nan
            x[(pick >= 0.02) & (pick < 0.05)] = -np.inf
            x[(pick >= 0.05) & (pick < 0.07)] = np.inf
            x[(pick >= 0.07) & (pick < 0.1)] = -0.0
        ts.append(x)
    (c1, g1), (c2, g2) = both_tapes(E, be, alg, ixs, iy, sizes, ts, np.ones(3, np.float32))
    np.testing.assert_array_equal(c1.view(np.uint32), c2.view(np.uint32))
    for x, y in zip(g1, g2):
        np.testing.assert_array_equal(x, y)


@pytest.mark.parametrize("n,seed", [(20, 2), (60, 7)])
def test_values_only_tape_mis(env, n, seed):
    om, E, be = env
    ixs, iy, sizes, ts, edges = E.mis_network(n, seed)
    (c1, g1), (c2, g2) = both_tapes(E, be, "maxplus", ixs, iy, sizes, ts, [1.0])
    np.testing.assert_array_equal(c1, c2)
    for x, y in zip(g1, g2):
        np.testing.assert_array_equal(x, y)


@pytest.mark.parametrize("kind", ["ties", "specials", "normal"])
@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul"])
def test_values_only_tape_long_contraction(env, alg, kind):
    # a node contracting 2^14 index values (the block-wide recomputation)
    om, E, be = env
    rng = np.random.default_rng(14)
    lab = list(range(14))
    ixs = [lab + [14], lab, [14]]
    iy = []
    sizes = {l: 2 for l in range(15)}
    ts = []
    for ix in ixs:
        n = 2 ** len(ix)
        x = (rng.integers(-3, 4, n) if kind != "normal" else rng.standard_normal(n)).astype(np.float32)
        if kind == "specials":
            pick = rng.random(n)
            x[pick < 0.001] = np.nan
            x[(pick >= 0.001) & (pick < 0.01)] = -np.inf
        ts.append(x)
    (c1, g1), (c2, g2) = both_tapes(E, be, alg, ixs, iy, sizes, ts, [1.0], tree=((0, 1), 2))
    np.testing.assert_array_equal(c1.view(np.uint32), c2.view(np.uint32))
    for x, y in zip(g1, g2):
        np.testing.assert_array_equal(x, y)
