"""The allocation-free entry point om_b200_tropical_matmul_argmax_noalloc.

It serves callers that may not allocate device memory during a call (an
application that owns all device memory through its own arena, or a
latency-critical path where an allocation could block or fail): its scratch
lives in fixed arrays inside the library.  This test calls it through the C
ABI and checks, on two calls in a row (so that state left in the shared
arrays by the first call cannot leak into the second), that values and argmax
equal those of om_b200_contract bit for bit, the tolerance every tropical
test here uses.  It lives in its own file, named to be collected last.
"""
import ctypes

import numpy as np
import pytest

import oracle as orc
from conftest import load_pkg

pytestmark = pytest.mark.gpu


def _noalloc(om, be, alg, A, B, C, AM, m, n, k):
    rc = om.lib().om_b200_tropical_matmul_argmax_noalloc(
        be.stream(), om.ALGEBRAS[alg], m, n, k, A.ptr, m, B.ptr, k, C.ptr, m, AM.ptr)
    om._check(rc)
    be.synchronize()


@pytest.fixture(scope="module")
def env():
    om = load_pkg()
    be = om.B200(0)
    yield om, be
    be.close()


CASES = [("maxplus", 512, 384, 640, 101), ("minplus", 256, 320, 96, 202),
         ("maxmul", 68, 70, 33, 303)]


def test_noalloc_matches_contract_twice(env):
    om, be = env
    for alg, m, n, k, seed in CASES:
        a = orc.uniform(seed, m * k)
        b = orc.uniform(seed + 1, k * n)
        if alg == "maxmul":
            a, b = np.abs(a), np.abs(b)
        A, B = be.from_slice(a), be.from_slice(b)
        ref_c, ref_am = be.contract_with_argmax(alg, A, [m, k], [1, m], [0, 1], B, [k, n], [1, k],
                                                [1, 2], [m, n], [0, 2])
        ref_c, ref_am = ref_c.to_vec(), ref_am.to_vec()
        C, AM = be.alloc(m * n, np.float32), be.alloc(m * n, np.uint32)
        for _ in range(2):
            _noalloc(om, be, alg, A, B, C, AM, m, n, k)
            np.testing.assert_array_equal(C.to_vec().view(np.uint32), ref_c.view(np.uint32))
            np.testing.assert_array_equal(AM.to_vec(), ref_am)


def test_noalloc_rejects_problems_beyond_its_workspace(env):
    om, be = env
    m = n = k = 8192  # 64 * 128 * 256 slab-tiles > 32768
    A = be.alloc(16, np.float32)
    with pytest.raises(om.OmError, match="static workspace"):
        rc = om.lib().om_b200_tropical_matmul_argmax_noalloc(
            be.stream(), 1, m, n, k, A.ptr, m, A.ptr, k, A.ptr, m, A.ptr)
        om._check(rc)
