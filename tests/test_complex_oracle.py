"""The complex restatement (oracle/complex_ref.py) pinned against the
reference's complex known answers (tests/suites/backward.rs:336-530,
tests/suites/coverage.rs:486-510) and a finite-difference check of its
holomorphic gradients."""
import numpy as np

import complex_ref as cr

C = complex


def test_kats():
    a = np.array([C(1, 1), C(3, 0), C(2, 0), C(4, -1)])
    i2 = np.array([1, 0, 0, 1], np.complex128)
    np.testing.assert_allclose(cr.einsum([a, i2], [[0, 1], [1, 2]], [0, 2], {0: 2, 1: 2, 2: 2}), a)
    np.testing.assert_allclose(cr.einsum([i2, np.array([C(1, 1), C(2, 0), C(0, 1), C(3, 0)])],
                                         [[0, 1], [1, 2]], [0, 2], {0: 2, 1: 2, 2: 2}),
                               [C(1, 1), C(2, 0), C(0, 1), C(3, 0)])
    u, v = np.array([C(1, 1), C(2, -1)]), np.array([C(1, 0), C(0, 1)])
    np.testing.assert_allclose(cr.einsum([u, v], [[0, 1], [1, 2]], [0, 2], {0: 2, 1: 1, 2: 2}),
                               [C(1, 1), C(2, -1), C(-1, 1), C(1, 2)])
    t = np.array([C(1, 1), C(2, -1), C(3, 0.5), C(4, -0.5)])
    np.testing.assert_allclose(cr.einsum([t], [[0, 0]], [], {0: 2}), [C(5, 0.5)])
    np.testing.assert_allclose(cr.gradients([t], [[0, 0]], [], {0: 2}, [1.0])[0], [1, 0, 0, 1])
    np.testing.assert_allclose(cr.einsum([t], [[0, 1]], [], {0: 2, 1: 2}), [C(10, 0)])
    np.testing.assert_allclose(cr.gradients([t], [[0, 1]], [1, 0], {0: 2, 1: 2}, np.ones(4))[0],
                               np.ones(4))


def test_gradients_are_holomorphic_derivatives():
    rng = np.random.default_rng(3)
    ixs, iy, sizes = [[0, 1], [1, 2], [2, 0]], [], {0: 3, 1: 4, 2: 2}
    ts = [rng.standard_normal(int(np.prod([sizes[l] for l in ix]))) +
          1j * rng.standard_normal(int(np.prod([sizes[l] for l in ix]))) for ix in ixs]
    g = cr.gradients(ts, ixs, iy, sizes, [1.0])
    h = 1e-7
    for t in range(3):
        for e in range(len(ts[t])):
            p = [x.copy() for x in ts]
            p[t][e] += h
            fd = (cr.einsum(p, ixs, iy, sizes)[0] - cr.einsum(ts, ixs, iy, sizes)[0]) / h
            assert abs(fd - g[t][e]) < 1e-5
