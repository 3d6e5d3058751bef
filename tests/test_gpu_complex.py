"""Complex Standard contractions on the device (OM_C32 / OM_C64) against the
reference's complex known answers and the numpy restatement
(oracle/complex_ref.py).

Tolerances, per element: complex f64 |x - r| <= 1e-12 * max(|r|, ||r||_inf);
complex f32 |x - r| <= gamma_K * S with S = sum_k |a_k| |b_k| (the element's
sum of product moduli) and gamma_K = 4 K 2^-24, the classical forward error
bound of a length-K f32 dot product (Higham, Accuracy and Stability of
Numerical Algorithms, 3.1) with room for the complex multiply; the
reference's own Complex<f32> loops carry the same error.  r is computed in
complex128 from the same f32 inputs."""
import importlib

import numpy as np
import pytest

import complex_ref as cr
from conftest import load_pkg

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    om = load_pkg()
    E = importlib.import_module("omeinsum_b200.einsum")
    be = om.B200(0)
    yield om, E, be
    be.close()


def crandn(rng, n, dtype):
    return (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(dtype)


def check(x, r, dtype, K, S=None):
    x, r = np.asarray(x, np.complex128), np.asarray(r, np.complex128)
    inf = np.max(np.abs(r)) if r.size else 0.0
    if dtype == np.complex128:
        bound = 1e-12 * np.maximum(np.abs(r), inf) + 1e-300
    else:
        bound = 4 * K * 2.0 ** -24 * np.asarray(S) + 1e-30
    assert np.all(np.abs(x - r) <= bound), float(np.max(np.abs(x - r) / bound))


def col(shape):
    st, s = [], 1
    for d in shape:
        st.append(s)
        s *= d
    return st


# ---- the reference's complex known answers --------------------------------
C = complex


def test_kat_identity_times_b(env):
    """tests/suites/coverage.rs:486-510: identity (x) B = B."""
    om, E, be = env
    a = np.array([1, 0, 0, 1], np.complex128)
    b = np.array([C(1, 1), C(2, 0), C(0, 1), C(3, 0)])
    c = be.contract("standard", be.from_slice(a), [2, 2], [1, 2], [0, 1], be.from_slice(b),
                    [2, 2], [1, 2], [1, 2], [2, 2], [0, 2]).to_vec()
    np.testing.assert_allclose(c, b, atol=1e-10)


def test_kat_matmul_and_outer(env):
    """tests/suites/backward.rs:336-431: A @ I = A; outer product
    (1+i, 2-i) x (1, i) = [1+i, 2-i, -1+i, 1+2i]."""
    om, E, be = env
    a = np.array([C(1, 1), C(3, 0), C(2, 0), C(4, -1)])
    i2 = np.array([1, 0, 0, 1], np.complex128)
    ein = E.Einsum([[0, 1], [1, 2]], [0, 2], {0: 2, 1: 2, 2: 2})
    c, g = ein.cost_and_gradient(be, "standard", [be.from_slice(a), be.from_slice(i2)],
                                 dy=np.ones(4, np.complex128))
    np.testing.assert_allclose(c.to_vec(), a, atol=1e-10)
    u = np.array([C(1, 1), C(2, -1)])
    v = np.array([C(1, 0), C(0, 1)])
    ein = E.Einsum([[0, 1], [1, 2]], [0, 2], {0: 2, 1: 1, 2: 2})
    c, g = ein.cost_and_gradient(be, "standard", [be.from_slice(u), be.from_slice(v)],
                                 dy=np.ones(4, np.complex128))
    np.testing.assert_allclose(c.to_vec(), [C(1, 1), C(2, -1), C(-1, 1), C(1, 2)], atol=1e-10)
    assert len(g[0].to_vec()) == 2 and len(g[1].to_vec()) == 2


def test_kat_unary_trace_sum_transpose(env):
    """tests/suites/backward.rs:438-530: trace 5+0.5i with identity gradient;
    sum 10 with all-ones gradient; transpose with all-ones gradient."""
    om, E, be = env
    a = np.array([C(1, 1), C(2, -1), C(3, 0.5), C(4, -0.5)])
    A = be.from_slice(a)
    c, g = E.Einsum([[0, 0]], [], {0: 2}).cost_and_gradient(be, "standard", [A],
                                                            dy=np.ones(1, np.complex128))
    np.testing.assert_allclose(c.to_vec(), [C(5, 0.5)], atol=1e-10)
    np.testing.assert_allclose(g[0].to_vec(), [1, 0, 0, 1], atol=1e-10)
    c, g = E.Einsum([[0, 1]], [], {0: 2, 1: 2}).cost_and_gradient(be, "standard", [A],
                                                                 dy=np.ones(1, np.complex128))
    np.testing.assert_allclose(c.to_vec(), [C(10, 0)], atol=1e-10)
    np.testing.assert_allclose(g[0].to_vec(), np.ones(4), atol=1e-10)
    c, g = E.Einsum([[0, 1]], [1, 0], {0: 2, 1: 2}).cost_and_gradient(
        be, "standard", [A], dy=np.ones(4, np.complex128))
    np.testing.assert_allclose(c.to_vec(), a[[0, 2, 1, 3]], atol=1e-10)
    np.testing.assert_allclose(g[0].to_vec(), np.ones(4), atol=1e-10)


# ---- random contractions and networks against the restatement -------------
CASES = [
    # (modes_a, modes_b, modes_c, sizes)
    ([0, 1], [1, 2], [0, 2], {0: 64, 1: 96, 2: 80}),
    ([0, 1, 2], [2, 1, 3], [3, 0], {0: 33, 1: 7, 2: 20, 3: 45}),
    ([0, 1, 4], [1, 2, 4], [2, 4, 0], {0: 40, 1: 64, 2: 24, 4: 3}),       # batch
    ([0, 1, 2, 3], [3, 2, 4, 5], [0, 1, 5, 4], {0: 16, 1: 16, 2: 8, 3: 8, 4: 16, 5: 16}),
    ([0, 1], [1, 2], [0, 2], {0: 512, 1: 1024, 2: 512}),                 # tensor-core size
]


@pytest.mark.parametrize("dtype", [np.complex64, np.complex128])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_complex_contract_matches_restatement(env, dtype, case):
    om, E, be = env
    ma, mb, mc, sizes = CASES[case]
    rng = np.random.default_rng(100 + case)
    sa, sb, sc = ([sizes[l] for l in m] for m in (ma, mb, mc))
    a, b = crandn(rng, int(np.prod(sa)), dtype), crandn(rng, int(np.prod(sb)), dtype)
    c = be.contract("standard", be.from_slice(a), sa, col(sa), ma, be.from_slice(b), sb, col(sb),
                    mb, sc, mc).to_vec()
    r = cr.einsum([a, b], [ma, mb], mc, sizes)
    K = int(np.prod([sizes[l] for l in ma if l in mb and l not in mc]))
    S = cr.einsum([np.abs(a), np.abs(b)], [ma, mb], mc, sizes).real
    check(c, r, dtype, K, S)


def test_complex_strided_view_and_copy(env):
    om, E, be = env
    rng = np.random.default_rng(7)
    x = crandn(rng, 6 * 5 * 4, np.complex128)
    X = be.from_slice(x)
    # the [1:, ::2, :] -like view: shape (5, 3, 4) with offset 1
    v = be.copy_strided(X, [5, 3, 4], [1, 12, 30], 1).to_vec()
    r = x.reshape(6, 5, 4, order="F")[1:, ::2, :].reshape(-1, order="F")
    np.testing.assert_array_equal(v, r)
    # the contraction reads views through strides at offset 0 (the reference's
    # boundary passes no offset): the [:5, ::2, :] view
    y = be.contract("standard", X, [5, 3, 4], [1, 12, 30], [0, 1, 2], be.from_slice(
        np.ones(3, np.complex128)), [3], [1], [1], [4, 5], [2, 0]).to_vec()
    r0 = x.reshape(6, 5, 4, order="F")[:5, ::2, :].reshape(-1, order="F")
    check(y, cr.einsum([r0, np.ones(3)], [[0, 1, 2], [1]], [2, 0], {0: 5, 1: 3, 2: 4}),
          np.complex128, 3)


@pytest.mark.parametrize("dtype", [np.complex64, np.complex128])
def test_complex_network_value_and_gradients(env, dtype):
    """A tensor-train-like complex network with a trace and a free output:
    value and every input gradient against the restatement."""
    om, E, be = env
    rng = np.random.default_rng(21)
    ixs = [[0, 1], [1, 2, 3], [3, 4, 5], [5, 6, 0], [2, 4], [7, 7]]
    iy = [6]
    sizes = {0: 4, 1: 6, 2: 3, 3: 5, 4: 3, 5: 6, 6: 2, 7: 3}
    ts = [crandn(rng, int(np.prod([sizes[l] for l in ix])), dtype) for ix in ixs]
    ein = E.Einsum(ixs, iy, sizes).optimize_greedy()
    dy = crandn(rng, 2, dtype)
    c, g = ein.cost_and_gradient(be, "standard", [be.from_slice(t) for t in ts], dy=dy)
    r = cr.einsum(ts, ixs, iy, sizes)
    S = cr.einsum([np.abs(t) for t in ts], ixs, iy, sizes).real
    check(c.to_vec(), r, dtype, 64 * len(ixs), S)
    rg = cr.gradients(ts, ixs, iy, sizes, dy)
    Sg = cr.gradients([np.abs(t) for t in ts], ixs, iy, sizes, np.abs(dy))
    for x, y, s_ in zip(g, rg, Sg):
        check(x.to_vec(), y, dtype, 64 * len(ixs), np.abs(s_))


def test_complex_rejects_tropical(env):
    om, E, be = env
    x = be.from_slice(np.ones(4, np.complex64))
    with pytest.raises(om.OmError):
        be.contract("maxplus", x, [2, 2], [1, 2], [0, 1], x, [2, 2], [1, 2], [1, 2], [2, 2], [0, 2])
