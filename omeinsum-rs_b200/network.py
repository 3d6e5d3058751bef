"""Sliced tensor-network driver over 1..N GPUs (one process per GPU).

The reference has no slicing or multi-GPU code; this is the driver that
`north_star` item 4 asks for, built on the engine (om_b200_einsum):

  * k labels are sliced: each of the 2^k assignments of their values is an
    independent sub-network (leaf tensors holding a sliced label become
    strided views with that label fixed -- no copy);
  * slice s runs on rank s mod N, contraction tree unchanged;
  * tropical (MaxPlus / MinPlus): every rank keeps its best slice; one
    all-reduce of a packed 64-bit key (order-preserving bits of the value,
    high; 0xffffffff - slice id, low) with MAX picks the global optimum, ties
    to the lowest slice id; the owner of that slice runs the argmax backward
    and broadcasts the gradient (the optimal configuration);
  * Standard: every rank sums its slices' values and gradients (gradients of
    sliced tensors are written at the fixed label values) and one SUM
    all-reduce combines them.

The per-slice executor is pluggable: DeviceExecutor (the B200 engine) is the
product path; tests pass the oracle engine to check the slicing and combine
logic on CPU ranks (gloo).
"""
from __future__ import annotations

import itertools

import numpy as np


def choose_slices(ixs, iy, sizes, tree, k, tree_cost):
    """Greedily picks k labels whose slicing most reduces the tree's space,
    then time, complexity."""
    chosen = []
    labels = sorted({l for ix in ixs for l in ix} - set(iy))
    for _ in range(k):
        best = None
        for l in labels:
            if l in chosen:
                continue
            s = dict(sizes)
            for c in chosen + [l]:
                s[c] = 1
            tc, sc = tree_cost(tree, ixs, iy, s)
            key = (sc, tc, l)
            if best is None or key < best[0]:
                best = (key, l)
        chosen.append(best[1])
    return chosen


def slice_assignments(sliced, sizes):
    """All assignments of the sliced labels, slice id = column-major index."""
    ranges = [range(sizes[l]) for l in sliced]
    out = []
    for vals in itertools.product(*reversed(ranges)):
        out.append(dict(zip(sliced, reversed(vals))))
    return out


def sliced_views(ixs, sizes, assign):
    """For each tensor: (element offset, shape, strides, labels) of its view
    with the sliced labels fixed (tensors contiguous column-major)."""
    views = []
    for ix in ixs:
        shape = [sizes[l] for l in ix]
        st, s = [], 1
        for d in shape:
            st.append(s)
            s *= d
        off = 0
        vs, vst, vix = [], [], []
        for l, d, t in zip(ix, shape, st):
            if l in assign:
                off += assign[l] * t
            else:
                vs.append(d)
                vst.append(t)
                vix.append(l)
        views.append((off, vs, vst, vix))
    return views


def order_key(value: float, minimize: bool) -> int:
    """Order-preserving unsigned 32-bit image of an f32 (inverted for min)."""
    u = int(np.array([value], np.float32).view(np.uint32)[0])
    k = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    return (~k & 0xFFFFFFFF) if minimize else k


class DeviceExecutor:
    """Runs one slice on this rank's GPU through om_b200_einsum.

    Subtrees none of whose leaves carries a sliced label give the same
    intermediate in every slice; value() contracts each such maximal subtree
    once, keeps the result on the device and feeds it to every slice as a
    leaf of a reduced tree, so a slice only runs the nodes that depend on
    the sliced labels.  value_and_grad() runs the full tree (its gradient
    flows to the original leaves)."""

    def __init__(self, be, E, alg, ixs, iy, sizes, tensors, tree):
        self.be, self.E, self.alg = be, E, alg
        self.ixs, self.iy, self.sizes, self.tree = ixs, iy, sizes, tree
        self.dev = [be.from_slice(t) for t in tensors]
        self.dtype = tensors[0].dtype
        self.enc = E.encode_tree(tree, ixs, iy) if not isinstance(tree, int) else ([], [])
        self._reduced = {}

    def _einsum(self, assign):
        views = sliced_views(self.ixs, self.sizes, assign)
        sizes = {l: v for l, v in self.sizes.items() if l not in assign}
        children, node_iys = self.enc
        node_iys = [[l for l in x if l not in assign] for x in node_iys]
        ein = self.E.Einsum([v[3] for v in views], self.iy, sizes).set_encoded(children, node_iys)
        return ein, views

    def _reduce(self, sliced):
        """(leaves, encoded reduced tree) for this set of sliced labels;
        leaves are ('leaf', i) or ('hoisted', Storage, labels)."""
        key = frozenset(sliced)
        if key in self._reduced:
            return self._reduced[key]
        E = self.E
        labels = E.tree_output_labels(self.tree, self.ixs, self.iy) \
            if not isinstance(self.tree, int) else {}
        leaves, ixs = [], []

        def leafset(t):
            return [t] if isinstance(t, int) else leafset(t[0]) + leafset(t[1])

        def invariant(t):
            return all(not (set(self.ixs[i]) & key) for i in leafset(t))

        def rec(t, root=False):
            if isinstance(t, int):
                leaves.append(("leaf", t))
                ixs.append(list(self.ixs[t]))
                return len(leaves) - 1
            if not root and invariant(t):
                sub = leafset(t)
                pos = {i: j for j, i in enumerate(sub)}

                def remap(u):
                    return pos[u] if isinstance(u, int) else (remap(u[0]), remap(u[1]))
                out_l = list(labels[id(t)])
                ein = E.Einsum([self.ixs[i] for i in sub], out_l, self.sizes)
                ein.set_contraction_tree(remap(t))
                val = ein.execute(self.be, self.alg, [self.dev[i] for i in sub])
                leaves.append(("hoisted", val, out_l))
                ixs.append(out_l)
                return len(leaves) - 1
            return (rec(t[0]), rec(t[1]))

        tree = rec(self.tree, root=True)
        enc = E.encode_tree(tree, ixs, self.iy) if not isinstance(tree, int) else ([], [])
        self._reduced[key] = (leaves, ixs, enc)
        return self._reduced[key]

    def value(self, assign):
        leaves, ixs, (children, node_iys) = self._reduce(assign.keys())
        full = sliced_views(self.ixs, self.sizes, assign)
        views, tensors = [], []
        for lf in leaves:
            if lf[0] == "leaf":
                views.append(full[lf[1]])
                tensors.append(self.dev[lf[1]])
            else:
                shape = [self.sizes[l] for l in lf[2]]
                st, s = [], 1
                for d in shape:
                    st.append(s)
                    s *= d
                views.append((0, shape, st, lf[2]))
                tensors.append(lf[1])
        sizes = {l: v for l, v in self.sizes.items() if l not in assign}
        node_iys = [[l for l in x if l not in assign] for x in node_iys]
        ein = self.E.Einsum([v[3] for v in views], self.iy, sizes).set_encoded(children, node_iys)
        out = self.be.alloc(ein.out_size(), self.dtype)
        ein.call_views(self.be, self.alg, tensors, views, out, None)
        return float(out.to_vec()[0])

    def value_and_grad(self, assign, dy=1.0):
        ein, views = self._einsum(assign)
        c, grads = ein.cost_and_gradient_views(self.be, self.alg, self.dev, views, [dy])
        return float(c.to_vec()[0]), [g.to_vec() for g in grads]


class OracleExecutor:
    """The same interface over the CPU restatement (test infrastructure)."""

    def __init__(self, oe, E, alg, ixs, iy, sizes, tensors, tree):
        self.oe, self.E, self.alg = oe, E, alg
        self.ixs, self.iy, self.sizes, self.tree, self.t = ixs, iy, sizes, tree, tensors

    def _args(self, assign):
        views = sliced_views(self.ixs, self.sizes, assign)
        ts = []
        for (off, vs, vst, vix), t in zip(views, self.t):
            idx = np.zeros(max(1, int(np.prod(vs))), dtype=np.int64) + off
            rem = np.arange(len(idx))
            for d, s in zip(vs, vst):
                idx += (rem % d) * s
                rem //= d
            ts.append(t[idx])
        ixs = [v[3] for v in views]
        sizes = {l: v for l, v in self.sizes.items() if l not in assign}
        ch, niy = self.E.encode_tree(self.tree, ixs, self.iy)
        return ts, ixs, sizes, ch, niy, views

    def value(self, assign):
        ts, ixs, sizes, ch, niy, _ = self._args(assign)
        return float(self.oe.einsum(self.alg, ts, ixs, self.iy, sizes, ch, niy)[0])

    def value_and_grad(self, assign, dy=1.0):
        ts, ixs, sizes, ch, niy, _ = self._args(assign)
        c, g = self.oe.cost_and_gradient(self.alg, ts, ixs, self.iy, sizes, ch, niy,
                                         np.array([dy], ts[0].dtype))
        return float(c[0]), g


def scatter_slice_grad(grad_view, ix, sizes, assign, full_size):
    """Place the gradient of a sliced view into its full (unsliced) tensor."""
    full = np.zeros(full_size, dtype=grad_view.dtype)
    shape = [sizes[l] for l in ix]
    st, s = [], 1
    for d in shape:
        st.append(s)
        s *= d
    off = sum(assign[l] * t for l, t in zip(ix, st) if l in assign)
    vs = [d for l, d in zip(ix, shape) if l not in assign]
    vst = [t for l, t in zip(ix, st) if l not in assign]
    idx = np.zeros(max(1, int(np.prod(vs))), dtype=np.int64) + off
    rem = np.arange(len(idx))
    for d, t in zip(vs, vst):
        idx += (rem % d) * t
        rem //= d
    full[idx] = grad_view
    return full


def run_sliced(executor, alg, ixs, sizes, sliced, rank, world, dist=None, device=None):
    """Contracts all 2^k slices over `world` ranks and combines them.

    Returns (value, gradients of every input tensor, winning slice id or -1).
    `dist` is torch.distributed (None for a single process); collectives run
    on `device` tensors (CUDA for NCCL, CPU for gloo)."""
    import torch
    assigns = slice_assignments(sliced, sizes)
    mine = [s for s in range(len(assigns)) if s % world == rank]
    full_sizes = [int(np.prod([sizes[l] for l in ix])) for ix in ixs]
    if alg in ("maxplus", "minplus"):
        minimize = alg == "minplus"
        best = None
        for s in mine:
            v = executor.value(assigns[s])
            key = (order_key(v, minimize) << 32) | (0xFFFFFFFF - s)
            if best is None or key > best:
                best = key
        # int64 MAX on the unsigned key: shift it into signed order first
        signed = (best - (1 << 63)) if best is not None else -(1 << 63)
        key = torch.tensor([signed], dtype=torch.int64, device=device)
        if dist is not None and world > 1:
            dist.all_reduce(key, op=dist.ReduceOp.MAX)
        k = int(key.item()) + (1 << 63)
        win = 0xFFFFFFFF - (k & 0xFFFFFFFF)
        owner = win % world
        grads = np.zeros(sum(full_sizes), dtype=np.float64)
        value = np.zeros(1)
        if owner == rank:
            v, g = executor.value_and_grad(assigns[win])
            value[0] = v
            parts = [scatter_slice_grad(gi, ix, sizes, assigns[win], n)
                     for gi, ix, n in zip(g, ixs, full_sizes)]
            grads = np.concatenate(parts).astype(np.float64)
        buf = torch.tensor(np.concatenate([value, grads]), dtype=torch.float64, device=device)
        if dist is not None and world > 1:
            dist.broadcast(buf, src=owner)
        out = buf.cpu().numpy()
        g = np.split(out[1:], np.cumsum(full_sizes)[:-1])
        return float(out[0]), g, win
    # Standard: sum of slices
    total = np.zeros(1 + sum(full_sizes), dtype=np.float64)
    for s in mine:
        v, g = executor.value_and_grad(assigns[s])
        parts = [scatter_slice_grad(gi, ix, sizes, assigns[s], n)
                 for gi, ix, n in zip(g, ixs, full_sizes)]
        total += np.concatenate([[v]] + parts)
    buf = torch.tensor(total, dtype=torch.float64, device=device)
    if dist is not None and world > 1:
        dist.all_reduce(buf, op=dist.ReduceOp.SUM)
    out = buf.cpu().numpy()
    return float(out[0]), np.split(out[1:], np.cumsum(full_sizes)[:-1]), -1
