"""JSON wire formats of the reference, read and written for the B200 engine.

Two families of files (tensor4all/omeinsum-rs):

* omeinsum-cli (omeinsum-cli/src/format.rs:1-95, common.rs):
  - tensors file   {"dtype": "f32"|"f64"|"c32"|"c64", "order": "col_major"|
                    "row_major" (default col_major), "tensors": [{"shape",
                    "data"}]}, complex data interleaved (re, im);
  - topology file  {"schema_version": 1, "expression": "ij,jk->ik",
                    "label_map", "size_dict" (string keys), "method", "tree"}
                    with the tree in omeco's serde form
                    {"Leaf": {"tensor_index"}} / {"Node": {"args", "eins"}};
  - result file    {"dtype", "order", "shape", "data"};
  - autodiff file  {"dtype", "order", "result": {"shape", "data"},
                    "gradients": [{"input_index", "shape", "data"}]}.
* benchmark networks (benches/support/network.rs:20-100): {"n_vertices",
  "bond_dim", "edges", "tree"} with the tree in the OMEinsum.jl form
  {"isleaf": true, "tensorindex"} / {"isleaf": false, "eins": {"ixs", "iy"},
  "args"}; edge (u, v) is the tensor over labels [u, v].

Trees come back as nested pairs of leaf indices (the form einsum.py uses);
error messages follow the CLI's wording (common.rs:229-360), so callers see
the same failures.
"""
from __future__ import annotations

import json

import numpy as np

DTYPES = {"f32": np.float32, "f64": np.float64, "c32": np.complex64, "c64": np.complex128}


class FormatError(ValueError):
    """A file that does not follow the format (the CLI exits with this text)."""


# ---------------------------------------------------------------------------
# storage order (format.rs:96-160)
# ---------------------------------------------------------------------------
def row_to_col_major(data, shape):
    """Row-major flat data of `shape` -> column-major flat data."""
    data = np.asarray(data)
    if len(shape) <= 1:
        return data.copy()
    return np.ascontiguousarray(data.reshape(shape, order="C")).reshape(-1, order="F")


def col_to_row_major(data, shape):
    data = np.asarray(data)
    if len(shape) <= 1:
        return data.copy()
    return data.reshape(shape, order="F").reshape(-1, order="C")


# ---------------------------------------------------------------------------
# trees
# ---------------------------------------------------------------------------
def tree_from_json(node, ntensors=None, sizes=None):
    """Nested pairs from either tree form; checks what common.rs:314-360
    checks (binary nodes, leaf index range, known labels)."""
    if "isleaf" in node:  # OMEinsum.jl form
        if node["isleaf"]:
            return _leaf(node["tensorindex"], ntensors)
        args, eins = node["args"], node.get("eins")
    elif "Leaf" in node:
        return _leaf(node["Leaf"]["tensor_index"], ntensors)
    elif "Node" in node:
        args, eins = node["Node"]["args"], node["Node"].get("eins")
    else:
        raise FormatError("Failed to parse topology JSON: unknown tree node")
    if len(args) != 2:
        raise FormatError(f"Topology tree must be binary, found node with {len(args)} children")
    if sizes is not None and eins is not None:
        for l in [x for ix in eins["ixs"] for x in ix] + list(eins["iy"]):
            if l not in sizes:
                raise FormatError(f"Topology references unknown label index {l}")
    return (tree_from_json(args[0], ntensors, sizes), tree_from_json(args[1], ntensors, sizes))


def _leaf(i, ntensors):
    if ntensors is not None and not 0 <= i < ntensors:
        raise FormatError(f"Topology leaf tensor_index {i} out of range for {ntensors} tensors")
    return int(i)


def tree_to_json(tree, ixs, iy, julia=False):
    """omeco serde form (default) or OMEinsum.jl form of a nested-pair tree;
    node labels are those each subtree shares with the rest (and iy)."""
    from .einsum import tree_output_labels
    labels = tree_output_labels(tree, ixs, iy) if not isinstance(tree, int) else {}

    def out_of(t):
        return list(ixs[t]) if isinstance(t, int) else labels[id(t)]

    def rec(t):
        if isinstance(t, int):
            return {"isleaf": True, "tensorindex": t} if julia else {"Leaf": {"tensor_index": t}}
        eins = {"ixs": [out_of(t[0]), out_of(t[1])], "iy": list(out_of(t))}
        if julia:
            return {"isleaf": False, "eins": eins, "args": [rec(t[0]), rec(t[1])]}
        return {"Node": {"args": [rec(t[0]), rec(t[1])], "eins": eins}}

    return rec(tree)


# ---------------------------------------------------------------------------
# expressions (parse.rs)
# ---------------------------------------------------------------------------
def parse_flat(expr: str):
    """'ij,jk->ik' -> (ixs, iy, label_map); labels a-z numbered in order of
    first appearance (parse.rs:19-77)."""
    if "->" not in expr:
        raise FormatError("Missing '->' in expression")
    lhs, rhs = expr.split("->", 1)
    lm = {}

    def idx(ch):
        if not ("a" <= ch <= "z"):
            raise FormatError(f"Invalid label '{ch}': must be a-z")
        return lm.setdefault(ch, len(lm))

    ixs = []
    for part in lhs.split(","):
        part = part.strip()
        if not part:
            raise FormatError("Empty tensor label group")
        ixs.append([idx(c) for c in part])
    seen = {l for ix in ixs for l in ix}
    iy = []
    for c in rhs.strip():
        l = idx(c)
        if l not in seen:
            raise FormatError(f"Output label '{c}' not found in any input tensor")
        iy.append(l)
    return ixs, iy, lm


def parse_parenthesized(expr: str):
    """'(ij,jk),kl->il' -> (ixs, iy, tree, label_map): parentheses give the
    contraction order, leaves numbered left to right (parse.rs:89-170).
    Every group holds one or two members (parse.rs:268-274)."""
    if "->" not in expr:
        raise FormatError("Missing '->' in expression")
    lhs, rhs = (s.strip() for s in expr.split("->", 1))
    lm = {}
    for ch in lhs + rhs:
        if "a" <= ch <= "z":
            lm.setdefault(ch, len(lm))
        elif ch not in "(), ":
            raise FormatError(f"Invalid character '{ch}' in expression")
    ixs, pos = [], 0

    def group():
        nonlocal pos
        items = []
        while True:
            while pos < len(lhs) and lhs[pos] == " ":
                pos += 1
            if pos >= len(lhs) or lhs[pos] == ")":
                break
            if items:
                if lhs[pos] != ",":
                    raise FormatError(f"Unexpected character '{lhs[pos]}' at position {pos}")
                pos += 1
                while pos < len(lhs) and lhs[pos] == " ":
                    pos += 1
            if pos < len(lhs) and lhs[pos] == "(":
                pos += 1
                sub = group()
                if pos >= len(lhs) or lhs[pos] != ")":
                    raise FormatError("Unbalanced parentheses: missing ')'")
                pos += 1
                items.append(sub)
            else:
                start = pos
                while pos < len(lhs) and "a" <= lhs[pos] <= "z":
                    pos += 1
                if pos == start:
                    raise FormatError("Empty tensor label group")
                ixs.append([lm[c] for c in lhs[start:pos]])
                items.append(len(ixs) - 1)
        if not items:
            raise FormatError("Empty expression group")
        if len(items) > 2:
            raise FormatError(f"Node must have exactly 2 children, got {len(items)}")
        return items[0] if len(items) == 1 else (items[0], items[1])

    tree = group()
    if pos != len(lhs):
        raise FormatError(f"Unexpected character '{lhs[pos]}' at position {pos}")
    seen = {l for ix in ixs for l in ix}
    iy = []
    for c in rhs:
        if c not in lm or lm[c] not in seen:
            raise FormatError(f"Output label '{c}' not in any input tensor")
        iy.append(lm[c])
    return ixs, iy, tree, lm


# ---------------------------------------------------------------------------
# files
# ---------------------------------------------------------------------------
def _load(path, what):
    try:
        with open(path) as f:
            text = f.read()
    except OSError as e:
        raise FormatError(f"Failed to read '{path}': {e}")
    try:
        return json.loads(text)
    except json.JSONDecodeError as e:
        raise FormatError(f"Failed to parse {what} JSON: {e}")


def read_tensors(path):
    """(dtype name, order, [column-major numpy arrays], [shapes])."""
    d = _load(path, "tensors")
    dt = d.get("dtype")
    if dt not in DTYPES:
        raise FormatError(f"Failed to parse tensors JSON: unknown dtype {dt!r}")
    order = d.get("order", "col_major")
    if order not in ("col_major", "row_major"):
        raise FormatError(f"Failed to parse tensors JSON: unknown order {order!r}")
    arrs, shapes = [], []
    for t in d.get("tensors", []):
        shape = [int(x) for x in t["shape"]]
        arrs.append(decode_data(t["data"], shape, dt, order))
        shapes.append(shape)
    return dt, order, arrs, shapes


def decode_data(data, shape, dt, order):
    """Flat JSON numbers -> column-major array of dtype `dt` (common.rs:36-80)."""
    cplx = dt in ("c32", "c64")
    n = int(np.prod(shape)) if shape else 1
    want = 2 * n if cplx else n
    if len(data) != want:
        raise FormatError(f"Data length {len(data)} doesn't match shape {shape} "
                          f"(expected {want})")
    x = np.asarray(data, np.float64)
    if cplx:
        x = x[0::2] + 1j * x[1::2]
    if order == "row_major":
        x = row_to_col_major(x, shape)
    return np.ascontiguousarray(x.astype(DTYPES[dt]))


def encode_data(x, shape, order):
    """Column-major array -> flat JSON list in `order`, complex interleaved."""
    x = np.asarray(x).reshape(-1)
    if order == "row_major":
        x = col_to_row_major(x, shape)
    if np.iscomplexobj(x):
        out = np.empty(2 * x.size, np.float64)
        out[0::2], out[1::2] = x.real, x.imag
        return out.tolist()
    return x.astype(np.float64).tolist()


def read_topology(path, ntensors):
    """(ixs, iy, sizes, tree) of a topology file (common.rs:229-281)."""
    d = _load(path, "topology")
    if d.get("schema_version") != 1:
        raise FormatError(f"Unsupported schema_version {d.get('schema_version')}, expected 1")
    sizes = {}
    for k, v in d["size_dict"].items():
        try:
            sizes[int(k)] = int(v)
        except ValueError:
            raise FormatError(f"Invalid size_dict key '{k}'")
    tree = tree_from_json(d["tree"], ntensors, sizes)
    ixs, iy, _ = parse_flat(d["expression"])
    if len(ixs) != ntensors:
        raise FormatError(f"Expression expects {len(ixs)} tensors but received {ntensors}")
    for l in [x for ix in ixs for x in ix] + iy:
        if l not in sizes:
            raise FormatError(f"Missing size for label index {l} referenced by topology "
                              f"expression")
    return ixs, iy, sizes, tree


def write_topology(path, expression, sizes, tree, method, ixs, iy, label_map):
    d = {"schema_version": 1, "expression": expression,
         "label_map": {k: int(v) for k, v in label_map.items()},
         "size_dict": {str(k): int(v) for k, v in sizes.items()}, "method": method,
         "tree": tree_to_json(tree, ixs, iy)}
    return _dump(d, path)


def result_json(dtype, order, y, shape):
    return {"dtype": dtype, "order": order, "shape": list(shape),
            "data": encode_data(y, shape, order)}


def autodiff_json(dtype, order, y, shape, grads, grad_shapes):
    return {"dtype": dtype, "order": order,
            "result": {"shape": list(shape), "data": encode_data(y, shape, order)},
            "gradients": [{"input_index": i, "shape": list(s), "data": encode_data(g, s, order)}
                          for i, (g, s) in enumerate(zip(grads, grad_shapes))]}


def read_result(path):
    """(dtype, order, column-major array, shape) of a result file (grad_output)."""
    d = _load(path, "result")
    shape = [int(x) for x in d["shape"]]
    return d["dtype"], d["order"], decode_data(d["data"], shape, d["dtype"], d["order"]), shape


def _dump(d, path=None, pretty=False):
    text = json.dumps(d, indent=2 if pretty else None)
    if path:
        with open(path, "w") as f:
            f.write(text)
    return text


def read_network_json(path):
    """A benchmark network (benches/support/network.rs:20-100): edge tensors
    over [u, v], scalar output, the stored tree.  Returns a dict with ixs,
    iy, sizes, tree, n_vertices, bond_dim."""
    d = _load(path, "network")
    ixs = [[int(u), int(v)] for u, v in d["edges"]]
    sizes = {}
    for u, v in ixs:
        sizes[u] = sizes[v] = int(d["bond_dim"])
    tree = tree_from_json(d["tree"], len(ixs), sizes)
    return {"ixs": ixs, "iy": [], "sizes": sizes, "tree": tree,
            "n_vertices": int(d["n_vertices"]), "bond_dim": int(d["bond_dim"])}
