"""numpy front end of the CPU restatement (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, always as the checker or the timed
CPU baseline, never as the product path.

All arrays are column-major (first axis fastest), as in omeinsum-rs
(src/tensor/mod.rs:533-546).  Helpers here take numpy arrays in Fortran order.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

STANDARD, MAXPLUS, MINPLUS, MAXMUL = 0, 1, 2, 3
ALGEBRAS = {"standard": STANDARD, "maxplus": MAXPLUS, "minplus": MINPLUS, "maxmul": MAXMUL}
F32, F64 = 0, 1

_lib = None


def build() -> str:
    """Compile the restatement with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I32, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int
        L.orc_gemm.argtypes = [I, I, P, I64, I64, P, I64, P, P, I]
        L.orc_gemm_batched.argtypes = [I, I, P, I64, I64, I64, P, I64, P, P]
        L.orc_copy_strided.argtypes = [I64, P, I, P, P, I64, P]
        L.orc_contract.argtypes = [I, I, P, I, P, P, P, P, I, P, P, P, I, P, P, P, P]
        L.orc_unary.argtypes = [I, I, P, I, P, P, P, I, P, P, P, P]
        L.orc_max_threads.restype = I
        _lib = L
    return _lib


def _alg(a) -> int:
    return ALGEBRAS[a] if isinstance(a, str) else int(a)


def _dt(x: np.ndarray) -> int:
    if x.dtype == np.float32:
        return F32
    if x.dtype == np.float64:
        return F64
    raise TypeError(f"oracle supports f32/f64, got {x.dtype}")


def _p(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def _i64(v):
    return np.ascontiguousarray(np.asarray(v, dtype=np.int64).reshape(-1))


def _i32(v):
    return np.ascontiguousarray(np.asarray(v, dtype=np.int32).reshape(-1))


def col_strides(shape):
    s, out = 1, []
    for d in shape:
        out.append(s)
        s *= d
    return out


def gemm(alg, a: np.ndarray, b: np.ndarray, m: int, k: int, n: int, argmax=False, threads=1):
    """generic_gemm(_with_argmax) on flat column-major buffers (cpu/mod.rs:862-920)."""
    a = np.ascontiguousarray(a.reshape(-1))
    b = np.ascontiguousarray(b.reshape(-1))
    c = np.empty(m * n, dtype=a.dtype)
    am = np.empty(m * n, dtype=np.uint32) if argmax else None
    rc = lib().orc_gemm(_alg(alg), _dt(a), _p(a), m, k, _p(b), n, _p(c), _p(am), threads)
    assert rc == 0
    return (c, am) if argmax else c


def contract(alg, a_buf, shape_a, strides_a, modes_a, b_buf, shape_b, strides_b, modes_b,
             shape_c, modes_c, argmax=False):
    """Backend::contract / contract_with_argmax on flat storage buffers.

    Returns the contiguous column-major output (and u32 argmax) as flat arrays,
    exactly like the reference's Storage return value (backend/traits.rs:147-199).
    """
    a_buf = np.ascontiguousarray(a_buf.reshape(-1))
    b_buf = np.ascontiguousarray(b_buf.reshape(-1))
    nc = int(np.prod(shape_c)) if len(shape_c) else 1
    c = np.empty(nc, dtype=a_buf.dtype)
    am = np.empty(nc, dtype=np.uint32) if argmax else None
    sa, ta, ma = _i64(shape_a), _i64(strides_a), _i32(modes_a)
    sb, tb, mb = _i64(shape_b), _i64(strides_b), _i32(modes_b)
    sc, mc = _i64(shape_c), _i32(modes_c)
    rc = lib().orc_contract(_alg(alg), _dt(a_buf), _p(a_buf), len(ma), _p(sa), _p(ta), _p(ma),
                            _p(b_buf), len(mb), _p(sb), _p(tb), _p(mb), len(mc), _p(sc), _p(mc),
                            _p(c), _p(am))
    assert rc == 0, rc
    return (c, am) if argmax else c


def copy_strided(src, shape, strides, offset=0):
    src = np.ascontiguousarray(src.reshape(-1))
    n = int(np.prod(shape)) if len(shape) else 1
    dst = np.empty(n, dtype=src.dtype)
    sh, st = _i64(shape), _i64(strides)
    lib().orc_copy_strided(src.itemsize, _p(src), len(sh), _p(sh), _p(st), offset, _p(dst))
    return dst


def unary(alg, x_buf, ix, shape_x, strides_x, iy, sizes: dict, argmax=False):
    """execute_unary_naive / execute_unary_with_argmax (engine.rs:752-926)."""
    x_buf = np.ascontiguousarray(x_buf.reshape(-1))
    maxl = max(list(ix) + list(iy) + [0]) + 1
    sz = np.zeros(maxl, dtype=np.int64)
    for k, v in sizes.items():
        if k < maxl:
            sz[k] = v
    ny = int(np.prod([sizes[l] for l in iy])) if len(iy) else 1
    y = np.empty(ny, dtype=x_buf.dtype)
    am = np.empty(ny, dtype=np.uint32) if argmax else None
    ixa, iya = _i32(ix), _i32(iy)
    sh, st = _i64(shape_x), _i64(strides_x)
    rc = lib().orc_unary(_alg(alg), _dt(x_buf), _p(x_buf), len(ixa), _p(ixa), _p(sh), _p(st),
                         len(iya), _p(iya), _p(sz), _p(y), _p(am))
    assert rc == 0
    return (y, am) if argmax else y


def max_threads() -> int:
    return int(lib().orc_max_threads())


# ---------------------------------------------------------------------------
# Seeded inputs shared by the oracle, the GPU tests and bench.py:
# splitmix64(seed) -> xoshiro256**, U[-1,1) = ((x >> 40) * 2^-24) * 2 - 1.
# ---------------------------------------------------------------------------
_M64 = (1 << 64) - 1


def _rotl(x, k):
    return ((x << k) | (x >> (64 - k))) & _M64


def _splitmix(seed, n):
    out = []
    z = seed & _M64
    for _ in range(n):
        z = (z + 0x9E3779B97F4A7C15) & _M64
        x = z
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _M64
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _M64
        out.append(x ^ (x >> 31))
    return out


def xoshiro_u64(seed: int, n: int) -> np.ndarray:
    """n outputs of xoshiro256** seeded by splitmix64(seed), vectorised over
    independent 1024 lanes (lane l seeded with seed + l) for speed."""
    lanes = min(1024, max(1, n))
    st = np.array([_splitmix(seed + l, 4) for l in range(lanes)], dtype=np.uint64).T.copy()
    s0, s1, s2, s3 = st[0], st[1], st[2], st[3]
    steps = (n + lanes - 1) // lanes
    out = np.empty((steps, lanes), dtype=np.uint64)
    with np.errstate(over="ignore"):
        for t in range(steps):
            r = s1 * np.uint64(5)
            r = ((r << np.uint64(7)) | (r >> np.uint64(57))) * np.uint64(9)
            out[t] = r
            tt = s1 << np.uint64(17)
            s2 ^= s0
            s3 ^= s1
            s1 ^= s2
            s0 ^= s3
            s2 ^= tt
            s3 = (s3 << np.uint64(45)) | (s3 >> np.uint64(19))
    return out.reshape(-1)[:n]


def uniform(seed: int, n: int, dtype=np.float32) -> np.ndarray:
    x = xoshiro_u64(seed, n)
    u = (x >> np.uint64(40)).astype(np.float64) * (2.0 ** -24)
    return (u * 2.0 - 1.0).astype(dtype)


def normal(seed: int, n: int, dtype=np.float32) -> np.ndarray:
    m = (n + 1) // 2
    x = xoshiro_u64(seed, 2 * m)
    u1 = ((x[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (2.0 ** -53)
    u2 = (x[1::2] >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.concatenate([r * np.cos(2 * np.pi * u2), r * np.sin(2 * np.pi * u2)])
    return z[:n].astype(dtype)


def ties(seed: int, n: int, lo=-8, hi=8, dtype=np.float32) -> np.ndarray:
    """Integers in [lo, hi]: many exact ties, to exercise the first-k rule."""
    x = xoshiro_u64(seed, n)
    return (lo + (x % np.uint64(hi - lo + 1)).astype(np.int64)).astype(dtype)
