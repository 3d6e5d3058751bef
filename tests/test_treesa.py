"""Contraction-order annealing (om_b200_optimize_tree, host code; the
replacement of omeco's optimize_treesa called at src/einsum/engine.rs:84-91)
against the reference's stored tree for its own benchmark network
(benches/network_3reg_150.json: log2 tc 34.6, log2 sc 27), and the trees it
returns checked for validity and value on the oracle engine.  CPU only."""
import importlib
import os

import numpy as np

import engine as oe
from conftest import ROOT, load_pkg


def mods():
    load_pkg()
    return (importlib.import_module("omeinsum_b200.einsum"),
            importlib.import_module("omeinsum_b200.io"))


def leaves(t):
    return [t] if isinstance(t, int) else leaves(t[0]) + leaves(t[1])


def test_treesa_beats_reference_stored_tree():
    E, IO = mods()
    net = IO.read_network_json(os.path.join(ROOT, "tests", "golden", "networks",
                                            "network_3reg_150.json"))
    ixs, iy, sizes = net["ixs"], net["iy"], net["sizes"]
    tc0, sc0 = (np.log2(float(x)) for x in E.tree_cost(net["tree"], ixs, iy, sizes))
    assert round(tc0, 1) == 34.6 and sc0 == 27.0
    # from random starting trees only: no help from another orderer
    tree, tc, sc = E.treesa_tree(ixs, iy, sizes, sc_target=sc0, ntrials=2, niters=10, seed=1)
    assert sorted(leaves(tree)) == list(range(len(ixs)))
    tcr, scr = (np.log2(float(x)) for x in E.tree_cost(tree, ixs, iy, sizes))
    assert abs(tcr - tc) < 1e-9 and scr == sc
    assert tc < tc0 - 5 and sc <= sc0


def test_treesa_never_worse_than_its_start():
    E, _ = mods()
    ixs, iy, sizes, ts, edges = E.mis_network(60, 3)
    g = E.greedy_tree(ixs, iy, sizes)
    tcg, scg = (np.log2(float(x)) for x in E.tree_cost(g, ixs, iy, sizes))
    tree, tc, sc = E.treesa_tree(ixs, iy, sizes, init=g, sc_target=scg, ntrials=1, niters=5)
    assert tc + max(0.0, sc - scg) <= tcg + 1e-9


def test_treesa_tree_gives_the_same_value():
    E, _ = mods()
    ixs, iy, sizes, ts, edges = E.mis_network(24, 5)
    g = E.greedy_tree(ixs, iy, sizes)
    tree, _, _ = E.treesa_tree(ixs, iy, sizes, sc_target=8, ntrials=2, niters=5, seed=7)
    ch1, n1 = E.encode_tree(g, ixs, iy)
    ch2, n2 = E.encode_tree(tree, ixs, iy)
    v1 = oe.einsum("maxplus", ts, ixs, iy, sizes, ch1, n1)
    v2 = oe.einsum("maxplus", ts, ixs, iy, sizes, ch2, n2)
    np.testing.assert_array_equal(v1, v2)


def test_decode_inverts_encode():
    E, _ = mods()
    ixs, iy, sizes, ts, edges = E.mis_network(12, 2)
    g = E.greedy_tree(ixs, iy, sizes)
    ch, _ = E.encode_tree(g, ixs, iy)
    assert E.decode_tree(ch, len(ixs)) == g
