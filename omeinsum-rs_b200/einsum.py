"""Einsum front end of the B200 backend: contraction trees, a greedy order,
the engine call (om_b200_einsum) and its gradient (om_b200_einsum_backward).

Mirrors the reference's `Einsum` (src/einsum/engine.rs:37-110):
`Einsum(ixs, iy, size_dict)`, `optimize_greedy()`, `set_contraction_tree()`,
`execute(algebra, tensors)`, and `cost_and_gradient` (backward.rs:769-799).
Trees are nested pairs of leaf indices, e.g. ((0, 1), 2), each node carrying
its output labels; they are encoded in post order for the C ABI.

The greedy orderer replaces omeco's GreedyMethod (omeco 0.2.4 is not
available here); both the oracle and the device take the same tree.
"""
from __future__ import annotations

import ctypes
import itertools

import numpy as np

from . import B200, DTYPES, Storage, _alg, _check, _i32, _i64, _p, lib


def _bind():
    L = lib()
    if not getattr(L, "_einsum_bound", False):
        P, I = ctypes.c_void_p, ctypes.c_int
        L.om_b200_einsum.argtypes = [P, I, I, I, P, P, P, P, P, I, P, I, P, P, I, P, P, P, P,
                                     ctypes.POINTER(P)]
        L.om_b200_einsum_tape_values.argtypes = L.om_b200_einsum.argtypes
        L.om_b200_einsum_backward.argtypes = [P, P, P]
        L.om_b200_tape_free.argtypes = [P]
        L.om_b200_tape_release.argtypes = [P]
        L.om_b200_einsum_backward_linked.argtypes = [P, P, P, I, P, P, P]
        D = ctypes.c_double
        L.om_b200_optimize_tree.argtypes = [I, P, P, I, P, I, P, P, P, D, D, D, I, I, D, D, D,
                                            ctypes.c_uint64, P, ctypes.POINTER(D),
                                            ctypes.POINTER(D)]
        L._einsum_bound = True
    return L


# ---------------------------------------------------------------------------
# trees
# ---------------------------------------------------------------------------
def tree_output_labels(tree, ixs, iy):
    """Labels of every node: those of its subtree that appear outside it or
    in iy (what omeco's NestedEinsum stores per node), keyed by id(node)."""
    from collections import Counter
    total = Counter(l for ix in ixs for l in set(ix))
    final = set(iy)
    out = {}

    def rec(t):
        if isinstance(t, int):
            return list(dict.fromkeys(ixs[t])), Counter(set(ixs[t]))
        (a, ca), (b, cb) = rec(t[0]), rec(t[1])
        inside = ca + cb
        labels = [l for l in dict.fromkeys(a + b) if l in final or inside[l] < total[l]]
        out[id(t)] = labels
        return labels, inside

    rec(tree)
    return out


def encode_tree(tree, ixs, iy):
    """Post-order (children, node_iys) arrays for om_b200_einsum / the oracle."""
    n = len(ixs)
    labels = tree_output_labels(tree, ixs, iy)
    children, node_iys = [], []

    def rec(t):
        if isinstance(t, int):
            return t
        a, b = rec(t[0]), rec(t[1])
        children.extend([a, b])
        node_iys.append(labels[id(t)])
        return n + len(node_iys) - 1

    rec(tree)
    return children, node_iys


def greedy_tree(ixs, iy, sizes):
    """Greedy pairwise order: repeatedly contract the pair (sharing a label if
    any does) that minimises size(out) - size(a) - size(b); ties go to the
    lowest pair of positions.  Deterministic."""
    from collections import Counter
    final = set(iy)
    items = [(i, list(dict.fromkeys(ix))) for i, ix in enumerate(ixs)]
    count = Counter(l for _, ix in items for l in ix)

    def size(labels):
        s = 1
        for l in labels:
            s *= sizes[l]
        return s

    while len(items) > 1:
        best = None
        share_any = any(set(a[1]) & set(b[1]) for a, b in itertools.combinations(items, 2))
        for (pa, a), (pb, b) in itertools.combinations(enumerate(items), 2):
            if share_any and not (set(a[1]) & set(b[1])):
                continue
            both = Counter(a[1]) + Counter(b[1])
            out = [l for l in dict.fromkeys(a[1] + b[1]) if l in final or count[l] > both[l]]
            cost = size(out) - size(a[1]) - size(b[1])
            if best is None or cost < best[0]:
                best = (cost, pa, pb, out)
        _, pa, pb, out = best
        ta, tb = items[pa][0], items[pb][0]
        for l in items[pa][1] + items[pb][1]:
            count[l] -= 1
        for l in out:
            count[l] += 1
        items = [it for k, it in enumerate(items) if k not in (pa, pb)] + [((ta, tb), out)]
    return items[0][0]


def decode_tree(children, n):
    """Nested-tuple tree of a post-order children array (inverse of the
    children part of encode_tree)."""
    nodes = []
    for i in range(len(children) // 2):
        a, b = children[2 * i], children[2 * i + 1]
        nodes.append((a if a < n else nodes[a - n], b if b < n else nodes[b - n]))
    return nodes[-1] if nodes else 0


def treesa_tree(ixs, iy, sizes, init=None, sc_target=20.0, sc_weight=1.0, rw_weight=0.0,
                ntrials=4, niters=10, betas=(0.01, 15.0, 0.05), seed=0):
    """Tree simulated annealing (om_b200_optimize_tree, the replacement of
    omeco's optimize_treesa called at src/einsum/engine.rs:84-91): returns
    (tree, log2 tc, log2 sc).  init: a starting tree for the first trial
    (the others start from random trees)."""
    L = _bind()
    n = len(ixs)
    if n < 2:
        return 0, 0.0, 0.0
    nd = _i32([len(ix) for ix in ixs])
    flat = _i32([l for ix in ixs for l in ix])
    iya = _i32(list(iy))
    sl = _i32(list(sizes.keys()))
    sv = _i64(list(sizes.values()))
    ch0 = None
    if init is not None:
        ch0 = _i32(encode_tree(init, ixs, iy)[0])
    out = _i32([0] * (2 * (n - 1)))
    tc, sc = ctypes.c_double(), ctypes.c_double()
    _check(L.om_b200_optimize_tree(n, _p(nd), _p(flat), len(iya), _p(iya), len(sl), _p(sl),
                                   _p(sv), None if ch0 is None else _p(ch0), sc_target,
                                   sc_weight, rw_weight, ntrials, niters, betas[0], betas[1],
                                   betas[2], seed, _p(out), ctypes.byref(tc),
                                   ctypes.byref(sc)))
    return decode_tree([int(x) for x in out], n), tc.value, sc.value


def tree_cost(tree, ixs, iy, sizes):
    """(time complexity, space complexity) of a tree: sum over nodes of the
    product of all label extents involved, and the largest intermediate."""
    labels = tree_output_labels(tree, ixs, iy)
    tc, sc = 0, 0

    def rec(t):
        nonlocal tc, sc
        if isinstance(t, int):
            return list(dict.fromkeys(ixs[t]))
        a, b = rec(t[0]), rec(t[1])
        allv = list(dict.fromkeys(a + b))
        p = 1
        for l in allv:
            p *= sizes[l]
        tc += p
        o = 1
        for l in labels[id(t)]:
            o *= sizes[l]
        sc = max(sc, o)
        return labels[id(t)]

    rec(tree)
    return tc, sc


# ---------------------------------------------------------------------------
# engine calls
# ---------------------------------------------------------------------------
class Einsum:
    """Einsum{ixs, iy, size_dict, optimized} (engine.rs:37-110)."""

    def __init__(self, ixs, iy, size_dict):
        self.ixs = [list(ix) for ix in ixs]
        self.iy = list(iy)
        self.size_dict = dict(size_dict)
        self.tree = None

    def optimize_greedy(self):
        self.tree = greedy_tree(self.ixs, self.iy, self.size_dict) if len(self.ixs) > 1 else 0
        return self

    def set_contraction_tree(self, tree):
        self.tree = tree
        self._enc = None
        return self

    def set_encoded(self, children, node_iys):
        """Use an already encoded tree (post-order children and node labels)."""
        self._enc = (list(children), [list(x) for x in node_iys])
        return self

    def encoded(self):
        if getattr(self, "_enc", None) is not None:
            return self._enc
        if self.tree is None:
            self.optimize_greedy()
        if isinstance(self.tree, int):
            return [], []
        return encode_tree(self.tree, self.ixs, self.iy)

    def _call(self, be: B200, alg, tensors, out, tape, views=None, values_only=False):
        """views (optional): per tensor (element offset, shape, strides,
        labels) of a strided view into the tensor's storage.  values_only:
        keep a tropical tape of values without argmax
        (om_b200_einsum_tape_values)."""
        L = _bind()
        children, node_iys = self.encoded()
        dtype = tensors[0].dtype
        if views is None:
            views = [(0, [self.size_dict[l] for l in ix], _col([self.size_dict[l] for l in ix]), ix)
                     for ix in self.ixs]
        es = np.dtype(dtype).itemsize
        ptrs = (ctypes.c_void_p * len(tensors))(*[t.ptr + v[0] * es for t, v in zip(tensors, views)])
        nd = _i32([len(v[3]) for v in views])
        shapes = _i64([d for v in views for d in v[1]])
        strides = _i64([d for v in views for d in v[2]])
        ixs = _i32([l for v in views for l in v[3]])
        iy = _i32(self.iy)
        sl = _i32(list(self.size_dict.keys()))
        sv = _i64(list(self.size_dict.values()))
        ch = _i32(children)
        off = _i32(np.cumsum([0] + [len(x) for x in node_iys]))
        niy = _i32([l for x in node_iys for l in x])
        fn = L.om_b200_einsum_tape_values if values_only else L.om_b200_einsum
        _check(fn(be.h, _alg(alg), DTYPES[dtype], len(tensors), ptrs, _p(nd), _p(shapes),
                  _p(strides), _p(ixs), len(iy), _p(iy), len(sl), _p(sl), _p(sv), len(node_iys),
                  _p(ch), _p(off), _p(niy), out.ptr, tape))

    def out_size(self):
        return int(np.prod([self.size_dict[l] for l in self.iy])) if self.iy else 1

    def execute(self, be: B200, alg, tensors):
        """Einsum::execute (engine.rs:125-166); tensors are contiguous Storages."""
        out = be.alloc(self.out_size(), tensors[0].dtype)
        self._call(be, alg, tensors, out, None)
        return out

    def call_views(self, be: B200, alg, tensors, views, out, tape):
        self._call(be, alg, tensors, out, tape, views)

    def forward_tape_views(self, be: B200, alg, tensors, views, out) -> ctypes.c_void_p:
        """Forward over strided views keeping the gradient tape; returns the
        tape handle (free it with tape_free).  May be called while the
        backend records a graph: the tape then refers to the graph's buffers
        and stays valid across replays."""
        tape = ctypes.c_void_p()
        self._call(be, alg, tensors, out, ctypes.byref(tape), views)
        return tape

    def forward_values_tape_views(self, be: B200, alg, tensors, views, out) -> ctypes.c_void_p:
        """Tropical forward that keeps every intermediate but computes no
        argmax; backward_tape / backward_tape_linked then find the argmax of
        just the elements the gradient visits (outputs of at most 4096
        elements).  Costs what a plain forward costs, plus the memory of the
        intermediates."""
        tape = ctypes.c_void_p()
        self._call(be, alg, tensors, out, ctypes.byref(tape), views, values_only=True)
        return tape

    @staticmethod
    def backward_tape(tape, d: Storage, grads):
        ptrs = (ctypes.c_void_p * len(grads))(*[g.ptr for g in grads])
        _check(_bind().om_b200_einsum_backward(tape, d.ptr, ptrs))

    @staticmethod
    def linked_args(tape, d: Storage, grads, links):
        """The ctypes arguments of om_b200_einsum_backward_linked (see
        backward_tape_linked); a caller repeating the same backward keeps
        them and passes them to backward_linked_prepared."""
        P = ctypes.c_void_p
        ptrs = (P * len(grads))(*[g.ptr for g in grads])
        leaf = _i32([l[0] for l in links])
        tapes = (P * len(links))(*[l[1] for l in links])
        rows = [(P * len(l[2]))(*[g.ptr for g in l[2]]) for l in links]
        rowp = (P * len(links))(*[ctypes.cast(r, P) for r in rows])
        return (tape, d.ptr, ptrs, len(links), _p(leaf), tapes, rowp, leaf, rows)

    @staticmethod
    def backward_linked_prepared(args):
        _check(_bind().om_b200_einsum_backward_linked(*args[:7]))

    @staticmethod
    def backward_tape_linked(tape, d: Storage, grads, links):
        """links: [(leaf index of `tape`, tape of the contraction that made
        that leaf, grads of that contraction's inputs)]; one launch walks all
        tapes (tropical, small output only; raises OmError otherwise)."""
        Einsum.backward_linked_prepared(Einsum.linked_args(tape, d, grads, links))

    @staticmethod
    def tape_free(tape):
        _bind().om_b200_tape_free(tape)

    @staticmethod
    def tape_release(tape):
        _check(_bind().om_b200_tape_release(tape))

    def cost_and_gradient_views(self, be: B200, alg, tensors, views, dy):
        """cost_and_gradient over strided views; gradients are contiguous in
        each view's shape."""
        out = be.alloc(self.out_size(), tensors[0].dtype)
        tape = ctypes.c_void_p()
        self._call(be, alg, tensors, out, ctypes.byref(tape), views)
        try:
            d = be.from_slice(np.asarray(dy, tensors[0].dtype))
            grads = [be.alloc(max(1, int(np.prod(v[1]))), tensors[0].dtype) for v in views]
            ptrs = (ctypes.c_void_p * len(grads))(*[g.ptr for g in grads])
            _check(_bind().om_b200_einsum_backward(tape, d.ptr, ptrs))
        finally:
            _bind().om_b200_tape_free(tape)
        return out, grads

    def record_forward(self, be: B200, alg, tensors, values_only=False):
        """Records this einsum's forward with tape as a CUDA graph (the
        network's many small launches then cost one graph launch).  Returns
        (graph, out, tape): after every graph.launch() the output is in `out`
        and backward_tape(tape, dy, grads) gives the gradients; the tape and
        its buffers live as long as the graph (free the tape with tape_free
        when done).  values_only: a tropical tape without argmax."""
        out = be.alloc(self.out_size(), tensors[0].dtype)
        tape = ctypes.c_void_p()
        be.graph_begin()
        try:
            self._call(be, alg, tensors, out, ctypes.byref(tape), values_only=values_only)
        finally:
            graph = be.graph_end()
        return graph, out, tape

    def cost_and_gradient(self, be: B200, alg, tensors, dy=None, values_only=False):
        """cost_and_gradient (backward.rs:769-799).  dy defaults to the
        algebra's one() as in the reference (0 for MaxPlus/MinPlus, so pass
        dy = [1] to recover a tropical configuration).  values_only: tropical
        forward without argmax, the backward finding the argmax of the
        elements it visits (same gradient)."""
        out = be.alloc(self.out_size(), tensors[0].dtype)
        tape = ctypes.c_void_p()
        self._call(be, alg, tensors, out, ctypes.byref(tape), values_only=values_only)
        try:
            if dy is None:
                one = 1.0 if _alg(alg) in (0, 3) else 0.0
                dy = np.full(self.out_size(), one, dtype=tensors[0].dtype)
            d = dy if isinstance(dy, Storage) else be.from_slice(np.asarray(dy, tensors[0].dtype))
            grads = [be.alloc(t.n, t.dtype) for t in tensors]
            ptrs = (ctypes.c_void_p * len(grads))(*[g.ptr for g in grads])
            _check(_bind().om_b200_einsum_backward(tape, d.ptr, ptrs))
        finally:
            _bind().om_b200_tape_free(tape)
        return out, grads


def _col(shape):
    s, out = 1, []
    for d in shape:
        out.append(s)
        s *= d
    return out


# ---------------------------------------------------------------------------
# benchmark networks, seeded
# ---------------------------------------------------------------------------
def random_regular3(n: int, seed: int):
    """Seeded 3-regular graph by stub matching with rejection (the method of
    the reference's examples/profile_network.rs:75-106, with a seeded
    generator instead of the thread RNG).  Edges (u < v), sorted."""
    assert n % 2 == 0 and n >= 4
    rng = np.random.default_rng(seed)
    for _ in range(10000):
        stubs = np.repeat(np.arange(n), 3)
        rng.shuffle(stubs)
        pairs = stubs.reshape(-1, 2)
        if np.any(pairs[:, 0] == pairs[:, 1]):
            continue
        e = {(int(min(u, v)), int(max(u, v))) for u, v in pairs}
        if len(e) == len(pairs):
            return sorted(e)
    raise RuntimeError("failed to generate a 3-regular graph")


def mis_network(n: int, seed: int, dtype=np.float32):
    """Maximum-independent-set tropical network (MaxPlus): vertex tensors
    [0, 1] over label v, edge tensors [[0, 0], [0, -inf]] over (u, v)
    (tests/suites/showcase.rs:1031-1173 construction), output scalar."""
    edges = random_regular3(n, seed)
    ixs = [[v] for v in range(n)] + [[u, v] for u, v in edges]
    tensors = [np.array([0, 1], dtype)] * n + [np.array([0, 0, 0, -np.inf], dtype)] * len(edges)
    return ixs, [], {v: 2 for v in range(n)}, tensors, edges


def ising_network(n: int, seed: int, beta: float = 1.0):
    """Ising spin-glass partition function (Standard f64): edge tensors
    exp(beta*J*s_i*s_j), J ~ N(0,1), index 0 <-> s = +1; no vertex tensors."""
    edges = random_regular3(n, seed)
    rng = np.random.default_rng(seed + 1)
    J = rng.standard_normal(len(edges))
    tensors = []
    for j in J:
        t = np.exp(beta * j * np.array([[1.0, -1.0], [-1.0, 1.0]]))
        tensors.append(np.asfortranarray(t).reshape(-1, order="F"))
    ixs = [[u, v] for u, v in edges]
    return ixs, [], {v: 2 for v in range(n)}, tensors, edges


# ---------------------------------------------------------------------------
# elimination-order trees (stand-in for omeco's TreeSA on graph networks)
# ---------------------------------------------------------------------------
def min_fill_order(ixs, iy, seed=0, restarts=16):
    """Variable-elimination order by the min-fill heuristic with seeded random
    tie-breaks; of `restarts` orders, the one with the smallest largest
    elimination clique (then the smallest sum of 2^clique) is returned.
    Labels of iy are never eliminated."""
    rng = np.random.default_rng(seed)
    labels = sorted({l for ix in ixs for l in ix} - set(iy))
    base = {l: set() for l in labels}
    for ix in ixs:
        u = [l for l in set(ix) if l in base]
        for a in u:
            base[a].update(x for x in u if x != a)
    best = None
    for _ in range(restarts):
        adj = {l: set(v) for l, v in base.items()}
        order, width, total = [], 0, 0.0
        alive = set(labels)
        while alive:
            cand, bestfill = [], None
            for v in alive:
                nb = list(adj[v])
                fill = sum(1 for i in range(len(nb)) for j in range(i + 1, len(nb))
                           if nb[j] not in adj[nb[i]])
                if bestfill is None or fill < bestfill:
                    cand, bestfill = [v], fill
                elif fill == bestfill:
                    cand.append(v)
            cand.sort(key=lambda x: len(adj[x]))
            m = len(adj[cand[0]])
            cand = [c for c in cand if len(adj[c]) == m]
            v = cand[int(rng.integers(len(cand)))]
            nb = adj[v]
            width = max(width, len(nb))
            total += 2.0 ** len(nb)
            for a in nb:
                adj[a].update(x for x in nb if x != a)
                adj[a].discard(v)
            del adj[v]
            alive.discard(v)
            order.append(v)
        key = (width, total)
        if best is None or key < best[0]:
            best = (key, order)
    return best[1]


def elimination_tree(ixs, iy, sizes, order):
    """Binary contraction tree that follows an elimination order: eliminating
    label v contracts every current tensor holding v, smallest first; the
    remaining tensors are joined at the end."""
    items = [(i, list(dict.fromkeys(ix))) for i, ix in enumerate(ixs)]
    final = set(iy)

    def size(ls):
        s = 1
        for l in ls:
            s *= sizes[l]
        return s

    def join(a, b, rest):
        outside = {l for _, ix in rest for l in ix} | final
        out = [l for l in dict.fromkeys(a[1] + b[1]) if l in outside]
        return ((a[0], b[0]), out)

    for v in order:
        hold = [it for it in items if v in it[1]]
        if not hold:
            continue
        rest = [it for it in items if v not in it[1]]
        while len(hold) > 1:
            hold.sort(key=lambda it: size(it[1]))
            a, b = hold[0], hold[1]
            hold = hold[2:]
            hold.append(join(a, b, rest + hold))
        items = rest + hold
    while len(items) > 1:
        items.sort(key=lambda it: size(it[1]))
        a, b = items[0], items[1]
        items = items[2:] + [join(a, b, items[2:])]
    return items[0][0]


def best_tree(ixs, iy, sizes, seed=0, restarts=16):
    """The better (smaller space, then time) of the greedy tree and the
    min-fill elimination tree."""
    t1 = greedy_tree(ixs, iy, sizes)
    t2 = elimination_tree(ixs, iy, sizes, min_fill_order(ixs, iy, seed, restarts))
    c1, c2 = tree_cost(t1, ixs, iy, sizes), tree_cost(t2, ixs, iy, sizes)
    return t1 if (c1[1], c1[0]) <= (c2[1], c2[0]) else t2
