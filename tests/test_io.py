"""CPU checks of the JSON wire formats (omeinsum-rs_b200/io.py) against the
reference CLI's own unit tests (omeinsum-cli/src/format.rs:162-244,
parse.rs tests) and its benchmark fixtures (benches/network_*.json)."""
import json
import os

import numpy as np
import pytest

from conftest import ROOT, load_pkg


def _io():
    load_pkg()
    import importlib
    return importlib.import_module("omeinsum_b200.io"), importlib.import_module("omeinsum_b200.einsum")


def test_row_col_major_conversions():
    IO, _ = _io()
    # format.rs: test_row_to_col_major_2x3, test_col_to_row_major_2x3, roundtrip, scalar, 1-d
    assert IO.row_to_col_major([1, 2, 3, 4, 5, 6], [2, 3]).tolist() == [1, 4, 2, 5, 3, 6]
    assert IO.col_to_row_major([1, 4, 2, 5, 3, 6], [2, 3]).tolist() == [1, 2, 3, 4, 5, 6]
    x = np.arange(1, 9, dtype=float)
    assert IO.col_to_row_major(IO.row_to_col_major(x, [2, 2, 2]), [2, 2, 2]).tolist() == x.tolist()
    assert IO.row_to_col_major([42.0], []).tolist() == [42.0]
    assert IO.row_to_col_major([1, 2, 3], [3]).tolist() == [1, 2, 3]


def test_tensors_file(tmp_path):
    IO, _ = _io()
    p = tmp_path / "t.json"
    p.write_text('{"dtype":"f64","tensors":[{"shape":[2],"data":[1.0,2.0]}]}')
    dt, order, arrs, shapes = IO.read_tensors(str(p))
    assert dt == "f64" and order == "col_major" and arrs[0].tolist() == [1.0, 2.0]
    # complex, row-major: interleaved pairs move together (common.rs:404-433)
    p.write_text(json.dumps({"dtype": "c64", "order": "row_major", "tensors": [
        {"shape": [2, 2], "data": [1.0, 1.0, 2.0, -1.0, 3.0, 0.0, 4.0, 2.0]}]}))
    dt, order, arrs, _ = IO.read_tensors(str(p))
    assert arrs[0].tolist() == [1 + 1j, 3 + 0j, 2 - 1j, 4 + 2j]
    assert IO.encode_data(arrs[0], [2, 2], "row_major") == [1.0, 1.0, 2.0, -1.0, 3.0, 0.0, 4.0, 2.0]
    p.write_text('{"dtype":"f64","order":"col_major","tensors":[{"shape":[2,3],"data":[1,2,3]}]}')
    with pytest.raises(IO.FormatError, match="doesn't match shape"):
        IO.read_tensors(str(p))


def test_parse_flat_cases():
    IO, _ = _io()
    ixs, iy, lm = IO.parse_flat("ij,jk->ik")
    assert ixs == [[0, 1], [1, 2]] and iy == [0, 2] and lm == {"i": 0, "j": 1, "k": 2}
    assert IO.parse_flat("ij,jk,kl->il")[:2] == ([[0, 1], [1, 2], [2, 3]], [0, 3])
    assert IO.parse_flat("ii->")[:2] == ([[0, 0]], [])
    assert IO.parse_flat("ij,ji->")[:2] == ([[0, 1], [1, 0]], [])
    assert IO.parse_flat("ij , jk -> ik")[:2] == ([[0, 1], [1, 2]], [0, 2])
    for bad in ["ij,jk", "iJ,jk->ik", "ij,jk->iz"]:
        with pytest.raises(IO.FormatError):
            IO.parse_flat(bad)


def test_parse_parenthesized_cases():
    IO, E = _io()
    ixs, iy, tree, _ = IO.parse_parenthesized("(ij,jk),kl->il")
    assert ixs == [[0, 1], [1, 2], [2, 3]] and iy == [0, 3] and tree == ((0, 1), 2)
    labels = E.tree_output_labels(tree, ixs, iy)
    assert set(labels[id(tree[0])]) == {0, 2}  # (ij,jk) keeps i and k, not j
    assert IO.parse_parenthesized("ij,jk->ik")[2] == (0, 1)
    assert IO.parse_parenthesized("ij->ji")[2] == 0
    for bad in ["(ij,jk->ik", "(,jk),kl->il", "ij,jk,kl->il"]:
        with pytest.raises(IO.FormatError):
            IO.parse_parenthesized(bad)


def test_topology_roundtrip_and_errors(tmp_path):
    IO, E = _io()
    ixs, iy, tree, lm = IO.parse_parenthesized("(ij,jk),kl->il")
    p = str(tmp_path / "topo.json")
    IO.write_topology(p, "ij,jk,kl->il", {0: 2, 1: 3, 2: 4, 3: 5}, tree, "greedy", ixs, iy, lm)
    assert IO.read_topology(p, 3) == (ixs, iy, {0: 2, 1: 3, 2: 4, 3: 5}, tree)
    d = json.load(open(p))
    leaf = {"Leaf": {"tensor_index": 0}}
    for change, msg in [({"schema_version": 99}, "schema_version"),
                        ({"tree": {"Leaf": {"tensor_index": 9}}}, "out of range"),
                        ({"size_dict": {}, "tree": leaf}, "Missing size for label index")]:
        e = dict(d)
        e.update(change)
        json.dump(e, open(p, "w"))
        with pytest.raises(IO.FormatError, match=msg):
            IO.read_topology(p, 3)
    e = dict(d)
    e["tree"] = {"Node": {"args": [{"Leaf": {"tensor_index": i}} for i in range(3)],
                          "eins": {"ixs": [[0], [1], [2]], "iy": [0]}}}
    json.dump(e, open(p, "w"))
    with pytest.raises(IO.FormatError, match="binary"):
        IO.read_topology(p, 3)


@pytest.mark.parametrize("name,log2_sc,log2_tc", [("network_small", 3, 7.29),
                                                  ("network_medium", 9, 12.76),
                                                  ("network_large", 14, 17.91),
                                                  ("network_3reg_150", 27, 34.60)])
def test_reference_network_fixtures_parse(name, log2_sc, log2_tc):
    """The stored trees load, their node labels equal the ones the engine
    derives, and their costs are the reference's (sc 2^27, tc 2^34.6 for the
    150-vertex graph)."""
    IO, E = _io()
    path = os.path.join(ROOT, "tests", "golden", "networks", name + ".json")
    net = IO.read_network_json(path)
    tc, sc = E.tree_cost(net["tree"], net["ixs"], net["iy"], net["sizes"])
    assert np.log2(sc) == log2_sc and abs(np.log2(tc) - log2_tc) < 0.01
    labels = E.tree_output_labels(net["tree"], net["ixs"], net["iy"])

    def walk(t, j):
        if isinstance(t, int):
            assert j["isleaf"] and j["tensorindex"] == t
            return
        assert set(labels[id(t)]) == set(j["eins"]["iy"])
        walk(t[0], j["args"][0])
        walk(t[1], j["args"][1])
    walk(net["tree"], json.load(open(path))["tree"])
