"""Parity of the B200 contraction (through the C ABI) with the CPU restatement
of the reference (oracle/) and with the reference's own known answers.

Tropical algebras: values and argmax bit-exact.  Standard algebra: the
reference uses faer (summation order unknown), so Standard is checked
against the oracle's extended-precision sum with the GEMM error bound
    |x - r| <= tol * sum_k |a_ik| |b_kj|,   tol = 1e-5 (f32), 1e-12 (f64).
"""
import numpy as np
import pytest

import oracle as orc
from conftest import load_pkg
from test_oracle_kats import KATS, arr, check_kat

pytestmark = pytest.mark.gpu

TOL = {np.float32: 1e-5, np.float64: 1e-12}


@pytest.fixture(scope="module")
def be():
    om = load_pkg()
    b = om.B200(0)
    yield b
    b.close()


def dev_contract(be, alg, a, sa, ta, ma, b, sb, tb, mb, sc, mc, argmax):
    A, B = be.from_slice(a), be.from_slice(b)
    if argmax:
        c, am = be.contract_with_argmax(alg, A, sa, ta, ma, B, sb, tb, mb, sc, mc)
        return c.to_vec(), am.to_vec()
    return be.contract(alg, A, sa, ta, ma, B, sb, tb, mb, sc, mc).to_vec(), None


def bits_equal(x, y):
    """Bitwise equality, except that any NaN matches any NaN: the payload and
    sign of a NaN made by inf - inf or 0 * inf are set by the FPU (x86 gives
    0xffc00000, the GPU 0x7fffffff), not by the algorithm."""
    x, y = np.asarray(x), np.asarray(y)
    if x.dtype in (np.float32, np.float64):
        u = np.uint32 if x.dtype == np.float32 else np.uint64
        nx, ny = np.isnan(x), np.isnan(y)
        return np.array_equal(nx, ny) and np.array_equal(x[~nx].view(u), y[~ny].view(u))
    return np.array_equal(x, y)


def check_case(be, alg, a, sa, ta, ma, b, sb, tb, mb, sc, mc, argmax=True):
    c, am = dev_contract(be, alg, a, sa, ta, ma, b, sb, tb, mb, sc, mc, argmax)
    r = orc.contract(alg, a, sa, ta, ma, b, sb, tb, mb, sc, mc, argmax=argmax)
    rc, ram = (r if argmax else (r, None))
    if alg == "standard":
        bound = orc.contract("standard", np.abs(a), sa, ta, ma, np.abs(b), sb, tb, mb, sc, mc)
        tol = TOL[a.dtype.type]
        err = np.abs(c.astype(np.float64) - rc.astype(np.float64))
        assert np.all(err <= tol * bound + 1e-300), float(np.max(err / (bound + 1e-300)))
        if argmax:
            assert np.all(am == 0)
    else:
        if not bits_equal(c, rc):
            u = np.uint32 if c.dtype == np.float32 else np.uint64
            bad = np.nonzero((c.view(u) != rc.view(u)) & ~(np.isnan(c) & np.isnan(rc)))[0]
            raise AssertionError(f"{len(bad)} value mismatches, first at {bad[:5]}: "
                                 f"dev {c[bad[:5]]} ref {rc[bad[:5]]}")
        if argmax:
            bad = np.nonzero(am != ram)[0]
            assert len(bad) == 0, f"{len(bad)} argmax mismatches at {bad[:5]}: " \
                                  f"dev {am[bad[:5]]} ref {ram[bad[:5]]}"


def col(shape):
    return orc.col_strides(shape)


# ---------------------------------------------------------------------------
@pytest.mark.parametrize("k", KATS, ids=[k["name"] for k in KATS])
def test_reference_kat_on_device(be, k):
    dt = np.float32 if k["dtype"] == "f32" else np.float64
    if k["kind"] == "copy_strided":
        s = be.from_slice(arr(k["src"], dt))
        out = be.copy_strided(s, k["shape"], k["strides"], k["offset"]).to_vec()
        check_kat(k, out, None)
        return
    a, b = arr(k["a"], dt), arr(k["b"], dt)
    c, am = dev_contract(be, k["alg"], a, k["shape_a"], k["strides_a"], k["modes_a"], b,
                         k["shape_b"], k["strides_b"], k["modes_b"], k["shape_c"], k["modes_c"],
                         k.get("with_argmax", False))
    check_kat(k, c, am)
    # and the device agrees with the oracle on every KAT, asserted or not
    check_case(be, k["alg"], a, k["shape_a"], k["strides_a"], k["modes_a"], b, k["shape_b"],
               k["strides_b"], k["modes_b"], k["shape_c"], k["modes_c"],
               argmax=k.get("with_argmax", False) and k["alg"] != "standard")


MATMUL_SIZES = [(1, 1, 1), (3, 5, 7), (64, 32, 64), (130, 97, 129), (256, 512, 192),
                (128, 1000, 256)]


@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul", "standard"])
@pytest.mark.parametrize("mkn", MATMUL_SIZES, ids=[f"{m}x{k}x{n}" for m, k, n in MATMUL_SIZES])
@pytest.mark.parametrize("argmax", [True, False])
def test_matmul_uniform_f32(be, alg, mkn, argmax):
    m, k, n = mkn
    a = orc.uniform(11 + m, m * k)
    b = orc.uniform(977 + n, k * n)
    if alg == "maxmul":
        a, b = np.abs(a), np.abs(b)
    check_case(be, alg, a, [m, k], [1, m], [0, 1], b, [k, n], [1, k], [1, 2], [m, n], [0, 2],
               argmax=argmax and alg != "standard")


@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul"])
@pytest.mark.parametrize("mkn", [(64, 64, 64), (192, 256, 320), (257, 130, 131)])
def test_matmul_ties_first_k_wins(be, alg, mkn):
    m, k, n = mkn
    a = orc.ties(5, m * k, -2, 2)
    b = orc.ties(6, k * n, -2, 2)
    if alg == "maxmul":
        a, b = np.abs(a) + 1, np.abs(b)
    check_case(be, alg, a, [m, k], [1, m], [0, 1], b, [k, n], [1, k], [1, 2], [m, n], [0, 2])


@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul"])
@pytest.mark.parametrize("special", ["neg_inf_cols", "pos_inf", "nan", "neg_zero", "both_inf",
                                     "all_neg_inf"])
def test_special_values(be, alg, special):
    m, k, n = 128, 96, 136
    a = orc.uniform(1, m * k).reshape(k, m).T.copy()  # (m,k) then flatten col-major below
    b = orc.uniform(2, k * n).reshape(n, k).T.copy()
    if special == "neg_inf_cols":
        a[:, 3] = -np.inf
        a[:, 50:52] = -np.inf
        b[7, :] = -np.inf
    elif special == "pos_inf":
        a[5, :] = np.inf
        b[:, 9] = np.inf
    elif special == "nan":
        a[3, 4] = np.nan
        b[10, 17] = np.nan
    elif special == "neg_zero":
        a[:, :] = 0.0
        a[1::2, :] = -0.0
        b[:, :] = -0.0
    elif special == "both_inf":
        a[0, :] = np.inf
        b[:, 0] = -np.inf
    elif special == "all_neg_inf":
        a[:, :] = -np.inf
    af = np.asfortranarray(a).reshape(-1, order="F").astype(np.float32)
    bf = np.asfortranarray(b).reshape(-1, order="F").astype(np.float32)
    check_case(be, alg, af, [m, k], [1, m], [0, 1], bf, [k, n], [1, k], [1, 2], [m, n], [0, 2])


LAYOUTS = {
    # name: (modes_a, modes_b, modes_c) over labels i=0, j=1, k=2 with extents
    "ij,jk->ik": ([0, 1], [1, 2], [0, 2]),
    "ji,jk->ik": ([1, 0], [1, 2], [0, 2]),
    "ij,kj->ik": ([0, 1], [2, 1], [0, 2]),
    "ji,kj->ki": ([1, 0], [2, 1], [2, 0]),
    "ij,jk->ki": ([0, 1], [1, 2], [2, 0]),
}


@pytest.mark.parametrize("alg", ["maxplus", "minplus", "standard"])
@pytest.mark.parametrize("name", list(LAYOUTS))
def test_operand_orientations(be, alg, name):
    ext = {0: 96, 1: 160, 2: 128}
    ma, mb, mc = LAYOUTS[name]
    sa, sb, sc = [ext[x] for x in ma], [ext[x] for x in mb], [ext[x] for x in mc]
    a = orc.uniform(21, int(np.prod(sa)))
    b = orc.uniform(22, int(np.prod(sb)))
    check_case(be, alg, a, sa, col(sa), ma, b, sb, col(sb), mb, sc, mc,
               argmax=alg != "standard")


@pytest.mark.parametrize("alg", ["standard", "minplus", "maxplus"])
def test_permuted_config2_small(be, alg):
    # 'abcd,dcef->abfe' (the BASELINE Standard / MinPlus config) at a=b=e=f=8, c=d=4
    a_, c_ = 8, 4
    A = orc.normal(31, a_ * a_ * c_ * c_)
    B = orc.normal(32, c_ * c_ * a_ * a_)
    sa, sb = [a_, a_, c_, c_], [c_, c_, a_, a_]
    check_case(be, alg, A, sa, col(sa), [0, 1, 2, 3], B, sb, col(sb), [3, 2, 4, 5],
               [a_, a_, a_, a_], [0, 1, 5, 4], argmax=alg != "standard")


@pytest.mark.parametrize("alg", ["standard", "maxplus"])
def test_strided_views(be, alg):
    # sub-matrix views with padding between columns and a transposed B view
    m, k, n, lda, ldb = 70, 90, 80, 75, 100
    a = orc.uniform(41, lda * k)
    b = orc.uniform(42, ldb * k)
    check_case(be, alg, a, [m, k], [1, lda], [0, 1], b, [k, n], [ldb, 1], [1, 2], [m, n], [0, 2],
               argmax=alg != "standard")


@pytest.mark.parametrize("alg", ["standard", "maxplus", "minplus", "maxmul"])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_batched_and_trace(be, alg, dtype):
    # 'bijx,bjky->kib' : batch b, contracted j, traced x (A) and y (B)
    e = {0: 3, 1: 5, 2: 6, 3: 4, 4: 2, 5: 3}
    ma, mb, mc = [0, 1, 2, 4], [0, 2, 3, 5], [3, 1, 0]
    sa, sb, sc = [e[x] for x in ma], [e[x] for x in mb], [e[x] for x in mc]
    a = orc.uniform(51, int(np.prod(sa)), dtype)
    b = orc.uniform(52, int(np.prod(sb)), dtype)
    if alg == "maxmul":
        a, b = np.abs(a), np.abs(b)
    check_case(be, alg, a, sa, col(sa), ma, b, sb, col(sb), mb, sc, mc, argmax=alg != "standard")


@pytest.mark.parametrize("alg", ["standard", "maxplus", "minplus", "maxmul"])
def test_f64_matmul(be, alg):
    m, k, n = 100, 120, 90
    a = orc.uniform(61, m * k, np.float64)
    b = orc.uniform(62, k * n, np.float64)
    if alg == "maxmul":
        a, b = np.abs(a), np.abs(b)
    check_case(be, alg, a, [m, k], [1, m], [0, 1], b, [k, n], [1, k], [1, 2], [m, n], [0, 2],
               argmax=alg != "standard")


def test_network_like_hyperedges(be):
    # bond-dimension-2 node with many batch modes: 'abcdef,cdefgh->abgh' style
    ma, mb, mc = [0, 1, 2, 3, 4, 5, 6, 7], [2, 3, 4, 5, 6, 7, 8, 9], [0, 1, 4, 5, 8, 9]
    sa, sb = [2] * 8, [2] * 8
    a = orc.ties(71, 256, -3, 3)
    b = orc.ties(72, 256, -3, 3)
    a[::7] = -np.inf
    check_case(be, "maxplus", a, sa, col(sa), ma, b, sb, col(sb), mb, [2] * 6, mc)


def test_scalar_output_and_outer(be):
    a = orc.uniform(81, 300)
    b = orc.uniform(82, 300)
    check_case(be, "maxplus", a, [300], [1], [0], b, [300], [1], [0], [], [])
    check_case(be, "minplus", a[:40], [40], [1], [0], b[:30], [30], [1], [1], [40, 30], [0, 1])


def test_errors_are_status_codes(be):
    om = load_pkg()
    a = be.from_slice(np.ones(4, np.float32))
    with pytest.raises(om.OmError, match="extent"):
        be.contract("maxplus", a, [2, 2], [1, 2], [0, 1], a, [4], [1], [1], [2], [0])
    with pytest.raises(om.OmError, match="repeats"):
        be.contract("maxplus", a, [2, 2], [1, 2], [0, 0], a, [2, 2], [1, 2], [0, 1], [2], [1])


def test_headline_2048_maxplus_argmax(be):
    """BASELINE config 1 at full size: MaxPlus 'ij,jk->ik', 2048^3, argmax.
    Checked against the oracle on 48 sampled rows (all 2048 columns), plus
    size-independent properties over the whole output."""
    m = k = n = 2048
    a = orc.uniform(0x5EED, m * k)
    b = orc.uniform(0x5EED + 1, k * n)
    c, am = dev_contract(be, "maxplus", a, [m, k], [1, m], [0, 1], b, [k, n], [1, k], [1, 2],
                         [m, n], [0, 2], True)
    C = c.reshape(n, m).T
    AM = am.reshape(n, m).T
    Am = a.reshape(k, m).T
    Bm = b.reshape(n, k).T
    rows = np.linspace(0, m - 1, 48).astype(int)
    sub = np.asfortranarray(Am[rows, :]).reshape(-1, order="F")
    rc, ram = orc.gemm("maxplus", sub, b, len(rows), k, n, argmax=True, threads=orc.max_threads())
    assert bits_equal(C[rows, :].reshape(-1, order="F"), rc)
    np.testing.assert_array_equal(AM[rows, :].reshape(-1, order="F"), ram)
    # properties everywhere: the value is attained at the argmax, and argmax < k
    assert AM.max() < k
    jj = np.arange(n)[None, :]
    attained = (Am[np.arange(m)[:, None], AM] + Bm[AM, jj]).astype(np.float32)
    assert bits_equal(attained, C)


@pytest.mark.parametrize("shape", [(3, 200, 72, 96), (2, 130, 33, 257), (4, 64, 1000, 64)],
                         ids=["b3", "ragged", "deepk"])
def test_standard_f32_tensor_core_batched(be, shape):
    # 'bij,bjk->bik' with batch first (non-contiguous batch stride) through the
    # tcgen05 3xTF32 path; checked with the GEMM error bound
    bsz, m, k, n = shape
    sa, sb = [bsz, m, k], [bsz, k, n]
    a = orc.normal(91, bsz * m * k)
    b = orc.normal(92, bsz * k * n)
    check_case(be, "standard", a, sa, col(sa), [0, 1, 2], b, sb, col(sb), [0, 2, 3],
               [bsz, m, n], [0, 1, 3], argmax=False)


def test_standard_f32_tensor_core_padded_views(be):
    # sub-matrix views with padded leading dimensions, output transposed
    m, k, n, lda, ldb = 200, 150, 180, 208, 160
    a = orc.normal(93, lda * k)
    b = orc.normal(94, ldb * n)
    check_case(be, "standard", a, [m, k], [1, lda], [0, 1], b, [k, n], [1, ldb], [1, 2], [n, m],
               [2, 0], argmax=False)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("shape", [[2] * 14, [2] * 21, [3, 2, 5, 2, 2, 7, 2, 3, 2], [4, 2] * 6,
                                   [2, 2, 64, 2, 2, 2, 3]])
def test_copy_strided_dense_permutations(be, shape, dtype):
    """Permutations of dense tensors with short axes (the tiled permutation
    path of the gather: network intermediates of extent-2 modes), bit-exact
    against the oracle's restated copy_strided."""
    rng = np.random.default_rng(len(shape) * 7 + sum(shape))
    n = int(np.prod(shape))
    src = orc.normal(91 + len(shape), n).astype(dtype)
    s = be.from_slice(src)
    st = col(shape)
    for trial in range(4):
        perm = rng.permutation(len(shape)) if trial else np.arange(len(shape))[::-1]
        sh = [shape[i] for i in perm]
        sd = [st[i] for i in perm]
        got = be.copy_strided(s, sh, sd, 0).to_vec()
        want = orc.copy_strided(src, sh, sd, 0)
        assert np.array_equal(got.view(np.uint8), np.asarray(want, dtype).view(np.uint8)), (sh, sd)


@pytest.mark.gpu
@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul", "standard"])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_node_many_modes_permuted(be, alg, dtype, seed):
    """Tensor-network nodes with 10-22 extent-2 modes in scrambled orders
    (batch, free, contracted and trace modes mixed, more than 16 modes in a
    group): the in-place node kernel against the oracle, values and argmax."""
    rng = np.random.default_rng(100 + seed)
    nl = [10, 14, 18][seed]
    labels = list(range(nl))
    role = rng.integers(0, 5, nl)  # 0 batch, 1 left, 2 right, 3 contracted, 4 left trace
    ma = [l for l in labels if role[l] in (0, 1, 3, 4)]
    mb = [l for l in labels if role[l] in (0, 2, 3)]
    mc = [l for l in labels if role[l] in (0, 1, 2)]
    ma = list(rng.permutation(ma))
    mb = list(rng.permutation(mb))
    mc = list(rng.permutation(mc))
    sa, sb, sc = [2] * len(ma), [2] * len(mb), [2] * len(mc)
    a = orc.ties(300 + seed, 2 ** len(ma), -3, 3).astype(dtype)
    b = orc.ties(400 + seed, 2 ** len(mb), -3, 3).astype(dtype)
    if alg == "maxmul":
        a, b = np.abs(a), np.abs(b)
    check_case(be, alg, a, sa, col(sa), [int(x) for x in ma], b, sb, col(sb),
               [int(x) for x in mb], sc, [int(x) for x in mc], argmax=alg != "standard")


@pytest.mark.gpu
@pytest.mark.parametrize("alg", ["maxplus", "standard"])
def test_node_batched_tiny_k(be, alg):
    """K = 2 with large, non-flattenable M and N (the thread-per-output path
    for short contractions) and a long leading output mode."""
    ma, mb, mc = [0, 1, 2, 3], [2, 4, 3, 5], [5, 0, 4, 3, 1]
    sa, sb = [96, 3, 2, 40], [2, 64, 40, 3]
    sc = [3, 96, 64, 40, 3]
    a = orc.ties(501, int(np.prod(sa)), -4, 4)
    b = orc.ties(502, int(np.prod(sb)), -4, 4)
    check_case(be, alg, a, sa, col(sa), ma, b, sb, col(sb), mb, sc, mc, argmax=alg != "standard")
    # a long contiguous leading output mode (split into tile pieces)
    ma, mb, mc = [0, 1], [1, 2], [0, 2]
    check_case(be, alg, orc.ties(503, 4096 * 2, -4, 4), [4096, 2], [2, 1], ma,
               orc.ties(504, 2 * 3, -4, 4), [2, 3], [1, 2], mb, [4096, 3], mc,
               argmax=alg != "standard")


@pytest.mark.gpu
@pytest.mark.parametrize("alg", ["maxplus", "minplus", "standard"])
@pytest.mark.parametrize("big", ["a", "b"])
def test_node_rows_reordered_for_reuse(be, alg, big):
    """A large operand times a small one whose own modes sit above the large
    operand's in C (the tensor-network slice shape): the node kernel visits
    its rows with the small operand's modes fastest and writes each row at
    its place in C; values and argmax against the oracle."""
    ml, ms, mc = [0, 1, 2, 3], [3, 2, 4, 5], [0, 1, 4, 2, 5]
    sl, ss = [256, 96, 2, 8], [8, 2, 5, 3]
    sc = [256, 96, 5, 2, 3]
    lg = orc.ties(601, int(np.prod(sl)), -4, 4)
    sm = orc.ties(602, int(np.prod(ss)), -4, 4)
    if big == "a":
        check_case(be, alg, lg, sl, col(sl), ml, sm, ss, col(ss), ms, sc, mc,
                   argmax=alg != "standard")
    else:
        check_case(be, alg, sm, ss, col(ss), ms, lg, sl, col(sl), ml, sc, mc,
                   argmax=alg != "standard")


@pytest.mark.gpu
@pytest.mark.parametrize("alg", ["maxplus", "maxmul", "standard"])
@pytest.mark.parametrize("k", [1, 2, 4, 8])
@pytest.mark.parametrize("reps", [(5, 3), (5, 20)])
@pytest.mark.parametrize("big", ["a", "b"])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_node_register_reuse(be, alg, k, reps, big, dtype):
    """Short k (a compiled length) and modes of the small operand alone in
    C's rows: a thread keeps the large operand's values across those rows'
    combinations (at most 64 of them; the rest stay rows), with the large
    operand on either side; values and argmax against the oracle."""
    r4, r5 = reps
    ml, ms = [0, 1, 2], [2, 4, 5]
    sl, ss = [256, 48, k], [k, r4, r5]
    mc, sc = [0, 4, 1, 5], [256, r4, 48, r5]
    lg = orc.ties(611 + k, int(np.prod(sl)), -4, 4).astype(dtype)
    sm = orc.ties(612 + k, int(np.prod(ss)), -4, 4).astype(dtype)
    if alg == "maxmul":
        lg, sm = np.abs(lg), np.abs(sm)
    if big == "a":
        check_case(be, alg, lg, sl, col(sl), ml, sm, ss, col(ss), ms, sc, mc,
                   argmax=alg != "standard")
    else:
        check_case(be, alg, sm, ss, col(ss), ms, lg, sl, col(sl), ml, sc, mc,
                   argmax=alg != "standard")


@pytest.mark.gpu
@pytest.mark.parametrize("alg", ["maxplus", "standard"])
@pytest.mark.parametrize("k", [2, 8])
@pytest.mark.parametrize("lead", [[0, 6], [6, 0]])
def test_node_group_load_patterns(be, alg, k, lead):
    """Groups of four outputs over two extent-2 modes, one of which the small
    operand lacks: its four values are x x y y or x y x y (two loads)."""
    ml, ms = [0, 6, 1, 2], [2, 6, 4, 5]
    sl, ss = [2, 2, 96, k], [k, 2, 3, 5]
    mc = lead + [4, 1, 5]
    ext = {0: 2, 6: 2, 1: 96, 4: 3, 5: 5}
    sc = [ext[m] for m in mc]
    lg = orc.ties(621 + k, int(np.prod(sl)), -4, 4)
    sm = orc.ties(622 + k, int(np.prod(ss)), -4, 4)
    check_case(be, alg, lg, sl, col(sl), ml, sm, ss, col(ss), ms, sc, mc,
               argmax=alg != "standard")


@pytest.mark.gpu
def test_graph_replay_of_contractions(be):
    """om_b200_graph_*: contractions recorded once replay on new input data
    with the same results as eager calls (tropical bit-exact)."""
    m, k, n = 96, 70, 80
    A, B = be.alloc(m * k), be.alloc(k * n)
    C, AM = be.alloc(m * n), be.alloc(m * n, np.uint32)
    L = load_pkg().lib()

    def upload(dst, x):
        x = np.ascontiguousarray(x, np.float32)
        assert L.om_b200_upload(be.h, dst.ptr, x.ctypes.data, x.nbytes) == 0

    be.graph_begin()
    be.contract_into("maxplus", A, [m, k], [1, m], [0, 1], B, [k, n], [1, k], [1, 2], [m, n],
                     [0, 2], C, AM)
    g = be.graph_end()
    for seed in (5, 6, 7):
        a, b = orc.ties(seed, m * k, -5, 5), orc.ties(seed + 50, k * n, -5, 5)
        upload(A, a)
        upload(B, b)
        g.launch()
        rc, ram = orc.gemm("maxplus", a, b, m, k, n, argmax=True)
        assert bits_equal(C.to_vec(), rc) and np.array_equal(AM.to_vec(), ram)


@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul", "standard"])
@pytest.mark.parametrize("special", ["ties", "nan_inf", "normal"])
@pytest.mark.parametrize("nout", [1, 3, 700])
def test_long_k_few_outputs_split_k(be, alg, special, nout):
    """Nodes with a handful of outputs and a long contracted range (a
    network's root dot product) split k over a CTA; the tropical combine must
    reproduce the sequential first-k rule, NaN products included."""
    if alg == "standard" and special == "nan_inf":
        pytest.skip("the Standard bound is relative; NaN/inf sums are covered elsewhere")
    sa, sb = [8, 16, 32, nout], [32, 16, 8, nout]  # contracted (0,1,2): K = 4096
    n = int(np.prod(sa))
    if special == "ties":
        a, b = orc.ties(91, n), orc.ties(92, n)
    else:
        a, b = orc.uniform(93, n), orc.uniform(94, n)
    if special == "nan_inf":
        a[[5, 700, 3000]] = [np.nan, np.inf, -np.inf]
        b[[17, 2222]] = [np.nan, -np.inf]
    check_case(be, alg, a, sa, col(sa), [0, 1, 2, 3], b, sb, col(sb), [2, 1, 0, 3], [nout], [3],
               argmax=alg != "standard")


@pytest.mark.parametrize("alg", ["maxplus", "standard"])
def test_graph_branches_match_eager(be, alg):
    """Four contractions recorded on concurrent graph branches
    (om_b200_graph_branch) give the eager results; tropical ones take the
    exact path inside branches (bit-exact against the oracle)."""
    m, k, n = 192, 96, 160
    ins = [(orc.uniform(300 + 2 * i, m * k), orc.uniform(301 + 2 * i, k * n)) for i in range(4)]
    dev = [(be.from_slice(a), be.from_slice(b)) for a, b in ins]
    outs = [(be.alloc(m * n, np.float32), be.alloc(m * n, np.uint32)) for _ in ins]
    am = alg != "standard"
    be.graph_begin()
    for i, ((A, B), (C, AM)) in enumerate(zip(dev, outs)):
        be.graph_branch(i)
        be.contract_into(alg, A, [m, k], [1, m], [0, 1], B, [k, n], [1, k], [1, 2], [m, n],
                         [0, 2], C, AM if am else None)
    be.graph_branch(-1)
    g = be.graph_end()
    for _ in range(2):
        g.launch()
        for (a, b), (C, AM) in zip(ins, outs):
            if am:
                rc, ram = orc.gemm(alg, a, b, m, k, n, argmax=True)
                assert bits_equal(C.to_vec(), rc) and np.array_equal(AM.to_vec(), ram)
            else:
                ref = a.reshape(k, m).T.astype(np.float64) @ b.reshape(n, k).T.astype(np.float64)
                np.testing.assert_allclose(C.to_vec().reshape(n, m).T, ref, rtol=0, atol=1e-4)


@pytest.mark.parametrize("amc", [True, False])
@pytest.mark.parametrize("bkc", [True, False])
@pytest.mark.parametrize("shape", [(1100, 1200, 40, 1), (700, 900, 33, 2), (1302, 1000, 17, 1)])
def test_standard_f64_dfma_orientations(be, amc, bkc, shape):
    """Standard f64 GEMM shapes large enough for the DFMA kernel, every
    unit-stride orientation of A and B, ragged tiles and a batch, against
    numpy within 1e-12 of the largest output."""
    m, n, k, nb = shape
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal(m * k * nb)
    b = rng.standard_normal(k * n * nb)
    # A as [m, k, batch] (m fastest) or [k, m, batch]; B as [k, n, batch] or [n, k, batch]
    sa = [m, k, nb] if amc else [k, m, nb]
    ma = [0, 1, 9] if amc else [1, 0, 9]
    sb = [k, n, nb] if bkc else [n, k, nb]
    mb = [1, 2, 9] if bkc else [2, 1, 9]
    A, B = be.from_slice(a), be.from_slice(b)
    c = be.contract("standard", A, sa, col(sa), ma, B, sb, col(sb), mb, [m, n, nb],
                    [0, 2, 9]).to_vec().reshape(nb, n, m)
    at = a.reshape(nb, sa[1], sa[0])
    bt = b.reshape(nb, sb[1], sb[0])
    Am = np.transpose(at, (0, 2, 1)) if amc else at          # [batch, m, k]
    Bm = np.transpose(bt, (0, 2, 1)) if bkc else bt          # [batch, k, n]
    ref = np.einsum("bmk,bkn->bnm", Am, Bm)
    assert np.max(np.abs(c - ref)) <= 1e-12 * np.max(np.abs(ref))


@pytest.mark.parametrize("alg,dtype,argmax", [("minplus", np.float32, False),
                                              ("maxplus", np.float32, True),
                                              ("standard", np.float64, False)])
def test_two_level_contracted_group(be, alg, dtype, argmax):
    """A contracted group (c, d) laid out (c, d) in A and (d, c) in B: for
    Standard f64 the planner reorders it so B flattens and A's k is decoded
    in two levels inside the DFMA kernel (no gather); the tropical kernels
    gather B.  Same results either way."""
    m, c, d, n = 1024, 32, 32, 1280
    rng = np.random.default_rng(77)
    sa, sb = [m, c, d], [d, c, n]
    a = rng.uniform(-1, 1, m * c * d).astype(dtype)
    b = rng.uniform(-1, 1, d * c * n).astype(dtype)
    check_case(be, alg, a, sa, col(sa), [0, 1, 2], b, sb, col(sb), [2, 1, 3], [m, n], [0, 3],
               argmax=argmax)


@pytest.mark.parametrize("alg", ["maxplus", "minplus", "maxmul"])
@pytest.mark.parametrize("mnk", [(16, 2048, 512), (40, 96, 1000), (300, 20, 257), (8, 512, 64)])
def test_tropical_short_side_fast_path(be, alg, mnk):
    """Few rows (the operands swap so the tile's 64-wide side takes them) or
    a short N (16..63): the fast kernel with padding, bit-exact values and
    first-k argmax against the oracle, with ties."""
    m, n, k = mnk
    a, b = orc.ties(500 + m, m * k), orc.ties(600 + n, k * n)
    check_case(be, alg, a, [m, k], [1, m], [0, 1], b, [k, n], [1, k], [1, 2], [m, n], [0, 2],
               argmax=True)
