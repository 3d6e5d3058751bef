"""omeinsum_b200 -- Python host binding of the B200 backend for omeinsum-rs.

The product is the C ABI in include/omeinsum_b200.h, implemented by
lib/libomeinsum_b200.so (hand-written sm_100a CUDA).  This module binds it
with ctypes and mirrors the reference's `Backend` / `Storage` interface
(tensor4all/omeinsum-rs src/backend/traits.rs:8-199), so tests read like the
reference's own backend tests:

    be = B200(0)
    a = be.from_slice(np.array([1, 2, 3, 4], np.float64))
    c = be.contract("standard", a, [2, 2], [1, 2], [0, 1], b, [2, 2], [1, 2], [1, 2],
                    [2, 2], [0, 2])
    c.to_vec()  # -> [23, 34, 31, 46]

There is no CPU fallback: if the shared library is missing this module
raises on first use.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libomeinsum_b200.so")

ALGEBRAS = {"standard": 0, "maxplus": 1, "minplus": 2, "maxmul": 3}
DTYPES = {np.dtype(np.float32): 0, np.dtype(np.float64): 1, np.dtype(np.uint32): 2,
          np.dtype(np.complex64): 3, np.dtype(np.complex128): 4}
NP_OF = {0: np.float32, 1: np.float64, 2: np.uint32, 3: np.complex64, 4: np.complex128}

# every symbol the header declares (checked by the CPU test suite)
EXPORTS = [
    "om_b200_name", "om_b200_last_error", "om_b200_create", "om_b200_destroy", "om_b200_stream",
    "om_b200_sync", "om_b200_alloc", "om_b200_free", "om_b200_upload", "om_b200_download",
    "om_b200_copy_strided", "om_b200_contract", "om_b200_unary", "om_b200_tropical_backward",
    "om_b200_launch_count", "om_b200_profile_enable", "om_b200_profile_query",
    "om_b200_tropical_matmul_argmax_noalloc", "om_b200_einsum", "om_b200_einsum_backward",
    "om_b200_tape_free", "om_b200_graph_begin", "om_b200_graph_end", "om_b200_graph_launch",
    "om_b200_graph_free", "om_b200_tape_release", "om_b200_einsum_backward_linked",
    "om_b200_set_f32_mode", "om_b200_scatter_index", "om_b200_gather_views", "om_b200_einsum_tape_values", "om_b200_optimize_tree", "om_b200_graph_branch", "om_b200_download_async",
]


class OmError(RuntimeError):
    """A non-zero status from the C ABI (the reference panics in these cases)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[om error {code}] {msg}")
        self.code = code


def build() -> str:
    """Compile libomeinsum_b200.so for sm_100a with the package Makefile."""
    subprocess.run(["make", "-s", "-j8", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OmError(-1, f"CUDA extension not built: {LIB_PATH} is missing "
                              "(run omeinsum_b200.build() or make -C omeinsum-rs_b200)")
        L = ctypes.CDLL(LIB_PATH)
        P, I, I64, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
        L.om_b200_name.restype = ctypes.c_char_p
        L.om_b200_last_error.argtypes = [ctypes.c_char_p, SZ]
        L.om_b200_create.argtypes = [I, ctypes.POINTER(P)]
        L.om_b200_destroy.argtypes = [P]
        L.om_b200_stream.argtypes = [P, ctypes.POINTER(P)]
        L.om_b200_sync.argtypes = [P]
        L.om_b200_alloc.argtypes = [P, SZ, ctypes.POINTER(P)]
        L.om_b200_free.argtypes = [P, P]
        L.om_b200_upload.argtypes = [P, P, P, SZ]
        L.om_b200_download.argtypes = [P, P, P, SZ]
        L.om_b200_download_async.argtypes = [P, P, P, SZ]
        L.om_b200_copy_strided.argtypes = [P, I, P, I, P, P, I64, P]
        L.om_b200_contract.argtypes = [P, I, I, P, I, P, P, P, P, I, P, P, P, I, P, P, P, P]
        L.om_b200_unary.argtypes = [P, I, I, P, I, P, P, P, I, P, P, P, P]
        L.om_b200_tropical_backward.argtypes = [P, I, P, P, I, P, P, I, P, P, I, P, P, P, P]
        L.om_b200_launch_count.restype = I64
        L.om_b200_graph_begin.argtypes = [P]
        L.om_b200_graph_branch.argtypes = [P, I]
        L.om_b200_graph_end.argtypes = [P, ctypes.POINTER(P)]
        L.om_b200_graph_launch.argtypes = [P, P]
        L.om_b200_graph_free.argtypes = [P]
        L.om_b200_profile_enable.argtypes = [P, I]
        L.om_b200_set_f32_mode.argtypes = [P, I]
        L.om_b200_scatter_index.argtypes = [P, I, P, I64, P, P, I]
        L.om_b200_gather_views.argtypes = [P, I, I, P, P, P, I64]
        L.om_b200_profile_query.argtypes = [P, I, ctypes.c_char_p, SZ,
                                            ctypes.POINTER(ctypes.c_double),
                                            ctypes.POINTER(ctypes.c_int64)]
        L.om_b200_tropical_matmul_argmax_noalloc.argtypes = [P, I, I64, I64, I64, P, I64, P, I64,
                                                             P, I64, P]
        _lib = L
    return _lib


def _check(rc: int):
    if rc != 0:
        buf = ctypes.create_string_buffer(1024)
        lib().om_b200_last_error(buf, 1024)
        raise OmError(rc, buf.value.decode(errors="replace"))


def _i64(v):
    return np.ascontiguousarray(np.asarray(list(v), dtype=np.int64))


def _i32(v):
    return np.ascontiguousarray(np.asarray(list(v), dtype=np.int32))


def _p(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def _alg(a) -> int:
    return ALGEBRAS[a.lower()] if isinstance(a, str) else int(a)


def col_strides(shape):
    s, out = 1, []
    for d in shape:
        out.append(s)
        s *= d
    return out


def launch_count() -> int:
    """Device kernels launched by this thread since the last call."""
    return int(lib().om_b200_launch_count())


class Graph:
    """Recorded stream work (om_b200_graph_*); launch() replays it."""

    def __init__(self, be, handle):
        self.be, self.h = be, handle

    def launch(self):
        _check(lib().om_b200_graph_launch(self.be.h, self.h))

    def __del__(self):
        if getattr(self, "h", None):
            try:
                lib().om_b200_graph_free(self.h)
            except Exception:
                pass
            self.h = None


class Storage:
    """Device buffer owned by a backend (the reference's `Storage<T>`)."""

    def __init__(self, backend: "B200", ptr: int, n: int, dtype):
        self.backend, self.ptr, self.n, self.dtype = backend, ptr, n, np.dtype(dtype)

    def __len__(self):
        return self.n

    @property
    def nbytes(self):
        return self.n * self.dtype.itemsize

    def to_vec(self) -> np.ndarray:
        out = np.empty(self.n, dtype=self.dtype)
        if self.n:
            _check(lib().om_b200_download(self.backend.h, _p(out), self.ptr, out.nbytes))
        return out

    def get(self, i: int):
        return self.to_vec()[i]

    def free(self):
        if self.ptr:
            _check(lib().om_b200_free(self.backend.h, self.ptr))
            self.ptr = None

    def __del__(self):
        try:
            if self.ptr and self.backend.h:
                lib().om_b200_free(self.backend.h, self.ptr)
        except Exception:
            pass


class View(Storage):
    """A non-owning window into another Storage (freed with its parent)."""

    def __init__(self, parent: Storage, offset: int, n: int):
        super().__init__(parent.backend, parent.ptr + offset * parent.dtype.itemsize, n,
                         parent.dtype)
        self.parent = parent

    def free(self):
        self.ptr = None

    def __del__(self):
        pass


class B200:
    """The B200 backend: `impl Backend for B200` in the reference's terms."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().om_b200_create(device, ctypes.byref(h)))
        self.h = h.value
        self.device = device

    @staticmethod
    def name() -> str:
        return lib().om_b200_name().decode()

    def close(self):
        if self.h:
            lib().om_b200_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synchronize(self):
        _check(lib().om_b200_sync(self.h))

    def stream(self) -> int:
        s = ctypes.c_void_p()
        _check(lib().om_b200_stream(self.h, ctypes.byref(s)))
        return s.value or 0

    def graph_begin(self):
        """Start recording the work issued on this backend's stream."""
        _check(lib().om_b200_graph_begin(self.h))

    def graph_branch(self, branch: int):
        """While recording: issue the following work on concurrent branch
        `branch` (-1: back to the backend's own stream)."""
        _check(lib().om_b200_graph_branch(self.h, branch))

    def graph_end(self) -> "Graph":
        """Stop recording; the recorded work as a replayable graph."""
        g = ctypes.c_void_p()
        _check(lib().om_b200_graph_end(self.h, ctypes.byref(g)))
        return Graph(self, g.value)

    def set_f32_mode(self, mode: str):
        """'3xtf32' (tensor cores, default) or 'exact' (f32 FMA on the CUDA
        cores) for Standard<f32> products."""
        _check(lib().om_b200_set_f32_mode(self.h, {"3xtf32": 0, "exact": 1}[mode]))

    def profile(self, on: bool = True):
        """Turn per-kernel CUDA-event timing on (clearing it) or off."""
        _check(lib().om_b200_profile_enable(self.h, 1 if on else 0))

    def profile_report(self) -> dict:
        """{kernel class: (total device ms, launches)} since profiling was enabled."""
        out, i = {}, 0
        name = ctypes.create_string_buffer(128)
        ms, n = ctypes.c_double(), ctypes.c_int64()
        while lib().om_b200_profile_query(self.h, i, name, 128, ctypes.byref(ms),
                                          ctypes.byref(n)) == 0:
            out[name.value.decode()] = (ms.value, n.value)
            i += 1
        return out

    def alloc(self, n: int, dtype=np.float32) -> Storage:
        p = ctypes.c_void_p()
        _check(lib().om_b200_alloc(self.h, n * np.dtype(dtype).itemsize, ctypes.byref(p)))
        return Storage(self, p.value, n, dtype)

    def from_slice(self, data) -> Storage:
        data = np.ascontiguousarray(np.asarray(data).reshape(-1))
        s = self.alloc(data.size, data.dtype)
        if data.size:
            _check(lib().om_b200_upload(self.h, s.ptr, _p(data), data.nbytes))
        return s

    def upload_into(self, s: Storage, data: np.ndarray):
        data = np.ascontiguousarray(data.reshape(-1))
        _check(lib().om_b200_upload(self.h, s.ptr, _p(data), data.nbytes))

    def copy_strided(self, src: Storage, shape, strides, offset=0) -> Storage:
        n = int(np.prod(shape)) if len(shape) else 1
        dst = self.alloc(n, src.dtype)
        self.copy_strided_into(src, shape, strides, offset, dst)
        return dst

    def copy_device(self, dst_ptr: int, src_ptr: int, nbytes: int):
        """Stream-ordered device-to-device copy of nbytes."""
        one = _i64([nbytes // 4])
        unit = _i64([1])
        _check(lib().om_b200_copy_strided(self.h, 2, src_ptr, 1, _p(one), _p(unit), 0, dst_ptr))

    def copy_strided_into(self, src: Storage, shape, strides, offset, dst: Storage):
        sh, st = _i64(shape), _i64(strides)
        _check(lib().om_b200_copy_strided(self.h, DTYPES[src.dtype], src.ptr, len(sh), _p(sh),
                                          _p(st), offset, dst.ptr))

    def contract_into(self, alg, a: Storage, shape_a, strides_a, modes_a, b: Storage, shape_b,
                      strides_b, modes_b, shape_c, modes_c, c: Storage, argmax: Storage | None):
        sa, ta, ma = _i64(shape_a), _i64(strides_a), _i32(modes_a)
        sb, tb, mb = _i64(shape_b), _i64(strides_b), _i32(modes_b)
        sc, mc = _i64(shape_c), _i32(modes_c)
        _check(lib().om_b200_contract(
            self.h, _alg(alg), DTYPES[a.dtype], a.ptr, len(ma), _p(sa), _p(ta), _p(ma),
            b.ptr, len(mb), _p(sb), _p(tb), _p(mb), len(mc), _p(sc), _p(mc),
            c.ptr, None if argmax is None else argmax.ptr))

    def contract(self, alg, a, shape_a, strides_a, modes_a, b, shape_b, strides_b, modes_b,
                 shape_c, modes_c) -> Storage:
        """Backend::contract (traits.rs:147-166)."""
        n = int(np.prod(shape_c)) if len(shape_c) else 1
        c = self.alloc(n, a.dtype)
        self.contract_into(alg, a, shape_a, strides_a, modes_a, b, shape_b, strides_b, modes_b,
                           shape_c, modes_c, c, None)
        return c

    def contract_with_argmax(self, alg, a, shape_a, strides_a, modes_a, b, shape_b, strides_b,
                             modes_b, shape_c, modes_c):
        """Backend::contract_with_argmax (traits.rs:180-199)."""
        n = int(np.prod(shape_c)) if len(shape_c) else 1
        c = self.alloc(n, a.dtype)
        am = self.alloc(n, np.uint32)
        self.contract_into(alg, a, shape_a, strides_a, modes_a, b, shape_b, strides_b, modes_b,
                           shape_c, modes_c, c, am)
        return c, am

    def unary(self, alg, x: Storage, ix, shape_x, strides_x, iy, sizes_y, argmax=False):
        """execute_unary_naive / execute_unary_with_argmax (engine.rs:752-926)."""
        n = int(np.prod(sizes_y)) if len(sizes_y) else 1
        y = self.alloc(n, x.dtype)
        am = self.alloc(n, np.uint32) if argmax else None
        ixa, sh, st = _i32(ix), _i64(shape_x), _i64(strides_x)
        iya, sy = _i32(iy), _i64(sizes_y)
        _check(lib().om_b200_unary(self.h, _alg(alg), DTYPES[x.dtype], x.ptr, len(ixa), _p(ixa),
                                   _p(sh), _p(st), len(iya), _p(iya), _p(sy), y.ptr,
                                   None if am is None else am.ptr))
        return (y, am) if argmax else y

    def tropical_backward(self, grad_c: Storage, argmax: Storage, shape_a, modes_a, shape_b,
                          modes_b, shape_c, modes_c, grad_a: Storage, grad_b: Storage):
        """Argmax-routed gradient scatter of one node (backward.rs:90-166)."""
        sa, ma, sb, mb = _i64(shape_a), _i32(modes_a), _i64(shape_b), _i32(modes_b)
        sc, mc = _i64(shape_c), _i32(modes_c)
        _check(lib().om_b200_tropical_backward(
            self.h, DTYPES[grad_c.dtype], grad_c.ptr, argmax.ptr, len(ma), _p(sa), _p(ma),
            len(mb), _p(sb), _p(mb), len(mc), _p(sc), _p(mc), grad_a.ptr, grad_b.ptr))
