"""CPU restatement of the reference's einsum engine and gradient tape.

TEST INFRASTRUCTURE ONLY (the checker for om_b200_einsum /
om_b200_einsum_backward).  Restates, over the oracle's contraction and unary
primitives (oracle/oracle.c):

  tape build               src/einsum/backward.rs:535-605 (build_tape_node_from_tree)
  operand normalisation    src/einsum/engine.rs:515-535 (compute_normalized_binary_indices),
                           backward.rs:607-642 (normalize_tape_operand)
  root finalisation        backward.rs:644-676 (finalize_tape_node)
  backward                 backward.rs:678-728 (backprop_tape_node), tropical scatter
                           :90-166, tropical unary :213-238, standard :287-332,
                           unary index exchange :183-195

The tree is the post-order encoding of include/omeinsum_b200.h: node i
contracts children[2i], children[2i+1] (c < ntensors: leaf c, else node
c - ntensors) into labels node_iys[i]; the last node is the root.
"""
from __future__ import annotations

import numpy as np

import oracle as orc


def _col(shape):
    return orc.col_strides(shape)


class _T:
    """A contiguous column-major tensor with labels."""

    def __init__(self, buf, ix, shape):
        self.buf = np.ascontiguousarray(buf.reshape(-1))
        self.ix = list(ix)
        self.shape = list(shape)


def normalized(ix, other, out):
    r = []
    for l in ix:
        if (l in other or l in out) and l not in r:
            r.append(l)
    return r


class Engine:
    def __init__(self, alg, sizes):
        self.alg = alg
        self.sizes = dict(sizes)
        self.tropical = alg != "standard"

    def shape_of(self, ix):
        return [self.sizes[l] for l in ix]

    def unary(self, x: _T, oix, argmax):
        r = orc.unary(self.alg, x.buf, x.ix, x.shape, _col(x.shape), oix, self.sizes, argmax=argmax)
        y, am = r if argmax else (r, None)
        return _T(y, oix, self.shape_of(oix)), am

    def contract(self, a: _T, b: _T, iy, argmax):
        r = orc.contract(self.alg, a.buf, a.shape, _col(a.shape), a.ix, b.buf, b.shape,
                         _col(b.shape), b.ix, self.shape_of(iy), iy, argmax=argmax)
        c, am = r if argmax else (r, None)
        return _T(c, iy, self.shape_of(iy)), am

    # ---- forward with tape ------------------------------------------------
    def forward(self, tensors, ixs, iy, children, node_iys, keep_tape=True):
        """tensors: flat column-major numpy buffers; returns (result, tape)."""
        n = len(tensors)
        for t, ix in zip(tensors, ixs):
            pass
        nodes = []  # dicts: op, content, argmax, children, ixs
        leaf = []
        for t in range(n):
            nodes.append(dict(op="leaf", t=t, content=_T(tensors[t], ixs[t],
                                                        self.shape_of(ixs[t])), am=None))
            leaf.append(len(nodes) - 1)
        track = keep_tape and self.tropical

        def push_unary(child, oix):
            c, am = self.unary(nodes[child]["content"], oix, track)
            nodes.append(dict(op="unary", content=c, am=am, child=child,
                              in_ix=nodes[child]["content"].ix, out_ix=list(oix)))
            return len(nodes) - 1

        def normalize(node, other, out):
            nix = normalized(nodes[node]["content"].ix, other, out)
            if nix == nodes[node]["content"].ix:
                return node
            return push_unary(node, nix)

        node_of = []
        for i in range(len(node_iys)):
            def res(c):
                return leaf[c] if c < n else node_of[c - n]
            l, r = res(children[2 * i]), res(children[2 * i + 1])
            niy = list(node_iys[i])
            l = normalize(l, nodes[r]["content"].ix, niy)
            r = normalize(r, nodes[l]["content"].ix, niy)
            c, am = self.contract(nodes[l]["content"], nodes[r]["content"], niy, track)
            nodes.append(dict(op="binary", content=c, am=am, l=l, r=r,
                              left_ix=nodes[l]["content"].ix, right_ix=nodes[r]["content"].ix,
                              out_ix=niy))
            node_of.append(len(nodes) - 1)
        cur = node_of[-1] if node_iys else leaf[0]
        if not node_iys or nodes[cur]["content"].ix != list(iy):
            cur = push_unary(cur, list(iy))
        self.nodes, self.root = nodes, cur
        return nodes[cur]["content"].buf

    # ---- backward -----------------------------------------------------------
    def backward(self, dy, ninputs):
        grads = [None] * ninputs
        self._bp(self.root, np.ascontiguousarray(dy.reshape(-1)), grads)
        return grads

    def _bp(self, idx, dy, grads):
        nd = self.nodes[idx]
        if nd["op"] == "leaf":
            grads[nd["t"]] = dy.copy()
            return
        if nd["op"] == "unary":
            child = self.nodes[nd["child"]]["content"]
            if self.tropical:
                g = np.zeros(int(np.prod(child.shape)) if child.shape else 1, dtype=dy.dtype)
                np.add.at(g, nd["am"].astype(np.int64), dy)
            else:
                out = _T(dy, nd["out_ix"], self.shape_of(nd["out_ix"]))
                g, _ = self.unary(out, nd["in_ix"], False)
                g = g.buf
            self._bp(nd["child"], g, grads)
            return
        lt, rt = self.nodes[nd["l"]]["content"], self.nodes[nd["r"]]["content"]
        ia, ib, iy = nd["left_ix"], nd["right_ix"], nd["out_ix"]
        if self.tropical:
            ga = np.zeros(max(1, int(np.prod(lt.shape))), dtype=dy.dtype)
            gb = np.zeros(max(1, int(np.prod(rt.shape))), dtype=dy.dtype)
            contracted = [l for l in ia if l in ib and l not in iy]
            cshape = self.shape_of(contracted)
            oshape = self.shape_of(iy)
            am = nd["am"].astype(np.int64)
            # every output element o routes dy[o] to the one element of each
            # operand that produced it; np.add.at applies the additions in
            # order of o, as the reference's loop over output elements does
            vals = {}
            rem = np.arange(len(dy), dtype=np.int64)
            for l, s in zip(iy, oshape):
                vals[l] = rem % s
                rem //= s
            w = am.copy()
            for l, s in zip(contracted, cshape):
                vals[l] = w % s
                w //= s
            pa = np.zeros(len(dy), dtype=np.int64)
            for l, st in zip(ia, _col(lt.shape)):
                pa += vals[l] * st
            pb = np.zeros(len(dy), dtype=np.int64)
            for l, st in zip(ib, _col(rt.shape)):
                pb += vals[l] * st
            np.add.at(ga, pa, dy)
            np.add.at(gb, pb, dy)
        else:
            d = _T(dy, iy, self.shape_of(iy))
            ga = self.contract(d, rt, ia, False)[0].buf
            gb = self.contract(lt, d, ib, False)[0].buf
        self._bp(nd["l"], ga, grads)
        self._bp(nd["r"], gb, grads)


def einsum(alg, tensors, ixs, iy, sizes, children, node_iys):
    return Engine(alg, sizes).forward(tensors, ixs, iy, children, node_iys, keep_tape=False)


def cost_and_gradient(alg, tensors, ixs, iy, sizes, children, node_iys, dy):
    e = Engine(alg, sizes)
    cost = e.forward(tensors, ixs, iy, children, node_iys, keep_tape=True)
    return cost, e.backward(np.asarray(dy, dtype=cost.dtype), len(tensors))
