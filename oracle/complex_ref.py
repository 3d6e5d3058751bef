"""Complex Standard contractions restated with numpy (complex128 accumulation).

TEST INFRASTRUCTURE ONLY: the checker for the device's OM_C32 / OM_C64 paths
(om_b200_contract, om_b200_unary, om_b200_einsum and its backward).  The
reference computes complex Standard contractions as plain (+, x) sums over
num_complex::Complex (src/algebra/standard.rs:26-116 over Complex32 /
Complex64, src/algebra/mod.rs:22,44-45) and its Standard backward is the
pair of contractions grad_a = dy (x) b, grad_b = a (x) dy with no
conjugation (src/einsum/backward.rs:287-332); the restatement below is the
same mathematics, labels as numpy einsum subscripts.
"""
from __future__ import annotations

import numpy as np

_LETTERS = "abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ"


def _sub(ix, names):
    return "".join(names.setdefault(l, _LETTERS[len(names)]) for l in ix)


def einsum(tensors, ixs, iy, sizes):
    """Value of the network, complex128, column-major output in iy order."""
    names = {}
    ops = [np.asarray(t, np.complex128).reshape([sizes[l] for l in ix], order="F")
           for t, ix in zip(tensors, ixs)]
    spec = ",".join(_sub(ix, names) for ix in ixs) + "->" + _sub(iy, names)
    return np.einsum(spec, *ops, optimize=True).reshape(-1, order="F")


def gradients(tensors, ixs, iy, sizes, dy):
    """d<dy, network>/d tensor_t for every t (holomorphic, no conjugation),
    column-major in each tensor's own shape; a tensor whose labels repeat
    receives its gradient on the diagonal (zeros elsewhere)."""
    names = {}
    out = []
    dyt = np.asarray(dy, np.complex128).reshape([sizes[l] for l in iy], order="F")
    for t, ix in enumerate(ixs):
        uniq = list(dict.fromkeys(ix))
        others = [(np.asarray(x, np.complex128).reshape([sizes[l] for l in jx], order="F"), jx)
                  for q, (x, jx) in enumerate(zip(tensors, ixs)) if q != t]
        # an all-ones factor over the tensor's own labels broadcasts the
        # gradient over labels no other operand carries
        ones = np.ones([sizes[l] for l in uniq])
        spec = ",".join([_sub(iy, names)] + [_sub(jx, names) for _, jx in others] +
                        [_sub(uniq, names)])
        g = np.einsum(spec + "->" + _sub(uniq, names), dyt, *[x for x, _ in others], ones,
                      optimize=True)
        full = np.zeros([sizes[l] for l in ix], np.complex128)
        idx = np.indices(full.shape)
        pos = {l: ix.index(l) for l in uniq}
        on_diag = np.ones(full.shape, bool)
        for k, l in enumerate(ix):
            on_diag &= idx[k] == idx[pos[l]]
        src = tuple(idx[pos[l]] for l in uniq)
        full[on_diag] = g[tuple(s[on_diag] for s in src)]
        out.append(full.reshape(-1, order="F"))
    return out
