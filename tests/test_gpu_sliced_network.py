"""Sliced network driver on the B200 (DeviceExecutor) against the same
sliced schedule restated on the CPU (OracleExecutor), single rank."""
import numpy as np
import pytest

from conftest import load_pkg

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,n", [("mis", 24), ("ising", 20)])
def test_device_slices_match_oracle_schedule(kind, n):
    om = load_pkg()
    import importlib
    import engine as oe
    E = importlib.import_module("omeinsum_b200.einsum")
    N = importlib.import_module("omeinsum_b200.network")
    if kind == "mis":
        ixs, iy, sizes, ts, edges = E.mis_network(n, 21)
        alg = "maxplus"
    else:
        ixs, iy, sizes, ts, edges = E.ising_network(n, 21)
        alg = "standard"
    tree = E.best_tree(ixs, iy, sizes, restarts=4)
    sliced = N.choose_slices(ixs, iy, sizes, tree, 3, E.tree_cost)
    be = om.B200(0)
    dv, dg, dw = N.run_sliced(N.DeviceExecutor(be, E, alg, ixs, iy, sizes, ts, tree), alg, ixs,
                              sizes, sliced, 0, 1)
    ov, og, ow = N.run_sliced(N.OracleExecutor(oe, E, alg, ixs, iy, sizes, ts, tree), alg, ixs,
                              sizes, sliced, 0, 1)
    if kind == "mis":
        assert dv == ov and dw == ow
        for x, y in zip(dg, og):
            np.testing.assert_array_equal(x, y)
        sel = [int(x[1] > x[0]) for x in dg[:n]]
        assert sum(sel) == int(dv) and all(not (sel[a] and sel[b]) for a, b in edges)
    else:
        assert abs(dv - ov) <= 1e-12 * abs(ov)
        for x, y in zip(dg, og):
            np.testing.assert_allclose(x, y, rtol=1e-11, atol=1e-300)
    be.close()
