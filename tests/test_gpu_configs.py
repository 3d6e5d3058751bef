"""BASELINE configurations at their stated sizes, on the device through the
C ABI, against the oracle.

  config 2  'abcd,dcef->abfe', a=b=e=f=64, c=d=32, f32 N(0,1):
            MinPlus (with and without argmax): bit-exact on sampled output
            rows, and over the whole output every value is attained at its
            argmax;
            Standard: on sampled rows against an f64-accumulated sum, once
            for the tensor-core 3xTF32 path and once for the exact CUDA-core
            FMA path, each under the f32 rule
                |x - r| <= max(1e-5 |r|, ||r||_inf sqrt(K) 2^-23).
  config 5  Ising spin glass, n = 120, Standard f64, 8 slices (3 sliced
            labels) with gradients of every edge tensor, against the same
            sliced schedule on the oracle engine: Z and every gradient
            within 1e-12 relative.
  reference fixtures
            the reference's own network benchmarks (benches/network_*.json:
            graph + stored contraction tree, every edge tensor filled with
            0.5^0.4 as in benches/support/network.rs:44-100), Standard f32,
            on the stored tree, against the oracle engine on the same tree
            and against the closed form Z = 2^n * (2 * 0.5^0.4)^|E| / 2^|E|.
"""
import json
import os

import numpy as np
import pytest

import oracle as orc
from conftest import ROOT, load_pkg

pytestmark = pytest.mark.gpu

A_, C_ = 64, 32
SA, SB, SC = [A_, A_, C_, C_], [C_, C_, A_, A_], [A_] * 4
MA, MB, MC = [0, 1, 2, 3], [3, 2, 4, 5], [0, 1, 5, 4]
K2 = C_ * C_


@pytest.fixture(scope="module")
def env():
    om = load_pkg()
    be = om.B200(0)
    a = orc.normal(0x5EED + 2, A_ * A_ * C_ * C_)
    b = orc.normal(0x5EED + 3, C_ * C_ * A_ * A_)
    yield om, be, a, b, be.from_slice(a), be.from_slice(b)
    be.close()


def sampled_rows(seed=7, n=48):
    rng = np.random.default_rng(seed)
    rows = rng.choice(A_ * A_, size=n, replace=False)
    return np.sort(np.concatenate([[0, A_ * A_ - 1], rows]))


def oracle_rows(alg, a, b, rows, argmax):
    """The oracle's contraction restricted to output rows (a, b) in `rows`:
    A sliced to those rows as one mode p, same contracted order (c, d), so
    the argmax encoding is the full problem's."""
    sub = _rows_of(a, rows)  # [p, c, d] column-major
    sa = [len(rows), C_, C_]
    r = orc.contract(alg, sub, sa, orc.col_strides(sa), [100, 2, 3], b, SB, orc.col_strides(SB),
                     MB, [len(rows), A_, A_], [100, 5, 4], argmax=argmax)
    return r


def _rows_of(a, rows):
    # A is column-major [a, b, c, d] = flat index p + 4096 * (c + 32 d), p = a + 64 b
    m = a.reshape(K2, A_ * A_)  # row q = c + 32 d, column p
    return np.ascontiguousarray(m[:, rows].T).reshape(-1, order="F")


@pytest.mark.parametrize("argmax", [True, False])
def test_config2_minplus_full_size(env, argmax):
    om, be, a, b, A, B = env
    if argmax:
        C, AM = be.contract_with_argmax("minplus", A, SA, om.col_strides(SA), MA, B, SB,
                                        om.col_strides(SB), MB, SC, MC)
        am = AM.to_vec()
    else:
        C = be.contract("minplus", A, SA, om.col_strides(SA), MA, B, SB, om.col_strides(SB), MB,
                        SC, MC)
    c = C.to_vec()
    rows = sampled_rows()
    r = oracle_rows("minplus", a, b, rows, argmax)
    rc, ram = r if argmax else (r, None)
    # oracle output [p, f, e] column-major: flat = p' + R * (f + 64 e)
    got = c.reshape(A_ * A_, A_ * A_, order="F")[rows, :]
    want = rc.reshape(len(rows), A_ * A_, order="F")
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    if argmax:
        np.testing.assert_array_equal(am.reshape(A_ * A_, A_ * A_, order="F")[rows, :],
                                      ram.reshape(len(rows), A_ * A_, order="F"))
        # whole output: each value is attained at its argmax (k = c + 32 d)
        p = np.arange(A_ ** 4) % (A_ * A_)
        q = np.arange(A_ ** 4) // (A_ * A_)  # f + 64 e
        f, e = q % A_, q // A_
        k = am.astype(np.int64)
        cc, dd = k % C_, k // C_
        av = a[p + A_ * A_ * (cc + C_ * dd)]
        bv = b[dd + C_ * cc + K2 * (e + A_ * f)]
        np.testing.assert_array_equal((av + bv).view(np.uint32), c.view(np.uint32))


@pytest.mark.parametrize("mode", ["3xtf32", "exact"])
def test_config2_standard_full_size(env, mode):
    om, be, a, b, A, B = env
    be.set_f32_mode(mode)
    try:
        be.profile(True)
        c = be.contract("standard", A, SA, om.col_strides(SA), MA, B, SB, om.col_strides(SB), MB,
                        SC, MC).to_vec()
        kernels = be.profile_report()
        be.profile(False)
    finally:
        be.set_f32_mode("3xtf32")
    if mode == "3xtf32":
        assert any("tcgen05" in k for k in kernels), kernels
        # B's contracted pair (d, c) is decoded in the split pre-pass, not gathered
        assert "gather" not in kernels, kernels
    else:
        assert not any("tcgen05" in k for k in kernels), kernels
    rows = sampled_rows(seed=11)
    r = oracle_rows("standard", a.astype(np.float64), b.astype(np.float64), rows, False)
    got = c.reshape(A_ * A_, A_ * A_, order="F")[rows, :].astype(np.float64)
    want = r.reshape(len(rows), A_ * A_, order="F")
    err = np.abs(got - want)
    floor = np.max(np.abs(want)) * np.sqrt(K2) * 2.0 ** -23
    bound = np.maximum(1e-5 * np.abs(want), floor)
    worst = float(np.max(err / bound))
    print(f"\nconfig 2 Standard f32 [{mode}]: max |x-r| / bound = {worst:.3f}, "
          f"max rel (|r| > floor) = {float(np.max((err / np.abs(want))[np.abs(want) > floor])):.2e}")
    assert worst <= 1.0


def test_config5_ising_n120_sliced_gradients():
    """Config 5 at its stated size on one rank: 8 slices, Z and dZ/dT_e for
    every edge tensor against the oracle engine on the same schedule."""
    om = load_pkg()
    import importlib
    import engine as oe
    E = importlib.import_module("omeinsum_b200.einsum")
    N = importlib.import_module("omeinsum_b200.network")
    ixs, iy, sizes, ts, edges = E.ising_network(120, 0x5EED)
    tree = E.best_tree(ixs, iy, sizes, restarts=8)
    sliced = N.choose_slices(ixs, iy, sizes, tree, 3, E.tree_cost)
    be = om.B200(0)
    try:
        dv, dg, _ = N.run_sliced(N.DeviceExecutor(be, E, "standard", ixs, iy, sizes, ts, tree),
                                 "standard", ixs, sizes, sliced, 0, 1)
    finally:
        be.close()
    ov, og, _ = N.run_sliced(N.OracleExecutor(oe, E, "standard", ixs, iy, sizes, ts, tree),
                             "standard", ixs, sizes, sliced, 0, 1)
    assert len(dg) == len(edges) == 180
    assert abs(dv - ov) <= 1e-12 * abs(ov)
    for x, y in zip(dg, og):
        assert np.all(np.abs(x - y) <= 1e-12 * np.abs(y) + 1e-300), (x, y)
    # unsliced oracle value: slicing changes nothing
    ch, niy = E.encode_tree(tree, ixs, iy)
    z = oe.einsum("standard", ts, ixs, iy, sizes, ch, niy)[0]
    assert abs(dv - z) <= 1e-12 * abs(z)


FIXTURES = ["network_small", "network_medium", "network_large", "network_3reg_150"]


@pytest.mark.parametrize("name", FIXTURES)
def test_reference_network_fixture(name):
    om = load_pkg()
    import importlib
    import engine as oe
    E = importlib.import_module("omeinsum_b200.einsum")
    IO = importlib.import_module("omeinsum_b200.io")
    net = IO.read_network_json(os.path.join(ROOT, "tests", "golden", "networks", name + ".json"))
    ixs, iy, sizes, tree = net["ixs"], net["iy"], net["sizes"], net["tree"]
    fill = np.float32(0.5) ** np.float32(0.4)
    ts = [np.full(4, fill, np.float32) for _ in ixs]
    tc, sc = E.tree_cost(tree, ixs, iy, sizes)
    be = om.B200(0)
    try:
        ein = E.Einsum(ixs, iy, sizes).set_contraction_tree(tree)
        z = float(ein.execute(be, "standard", [be.from_slice(t) for t in ts]).to_vec()[0])
    finally:
        be.close()
    n, m = net["n_vertices"], len(ixs)
    closed = 2.0 ** n * float(fill) ** m  # every assignment has weight fill^|E|
    print(f"\n{name}: log2 tc {np.log2(tc):.2f} sc {np.log2(sc):.1f}, Z {z:.6e}, closed {closed:.6e}")
    assert abs(z - closed) <= 1e-4 * closed
    if sc <= 2 ** 22:  # the oracle engine in seconds
        ch, niy = E.encode_tree(tree, ixs, iy)
        r = float(oe.einsum("standard", ts, ixs, iy, sizes, ch, niy)[0])
        assert abs(z - r) <= 1e-5 * abs(r)
