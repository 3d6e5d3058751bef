"""Copies the reference's network fixtures into tests/golden/networks/.

The reference benchmarks its network contraction on four JSON files
(tensor4all/omeinsum-rs benches/network_{small,medium,large,3reg_150}.json,
read by benches/support/network.rs:20-100): a 3-regular graph (n_vertices,
bond_dim, edges) and a stored binary contraction tree in omeco's
NestedEinsum serialisation (isleaf / tensorindex / eins{ixs, iy} / args).
They are data, copied unchanged (re-serialised without whitespace) so that
the tests can run them where the reference tree is absent.

    python tests/golden/make_network_fixtures.py [reference root]
"""
import json
import os
import sys

NAMES = ["network_small", "network_medium", "network_large", "network_3reg_150"]


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "networks")
    os.makedirs(out, exist_ok=True)
    for n in NAMES:
        with open(os.path.join(ref, "benches", n + ".json")) as f:
            d = json.load(f)
        with open(os.path.join(out, n + ".json"), "w") as f:
            json.dump(d, f, separators=(",", ":"))
        print(n, d["n_vertices"], len(d["edges"]))


if __name__ == "__main__":
    main()
