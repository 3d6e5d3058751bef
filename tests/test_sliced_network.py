"""Sliced network driver (omeinsum-rs_b200/network.py): slicing, per-rank
slice assignment and the combine step, on CPU ranks (gloo, world size 2)
with the oracle engine as the per-slice executor.  The GPU counterpart
(DeviceExecutor on the B200) is in test_gpu_sliced_network.py."""
import os

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT, load_pkg


def _mods():
    load_pkg()
    import importlib
    import engine as oe
    return (importlib.import_module("omeinsum_b200.einsum"),
            importlib.import_module("omeinsum_b200.network"), oe)


def _case(kind):
    E, N, oe = _mods()
    if kind == "mis":
        ixs, iy, sizes, ts, edges = E.mis_network(16, 9)
        alg = "maxplus"
    elif kind == "maxmul":
        # the same independent-set network in (max, x): vertex weights [1, 2],
        # forbidden edge state 0, so the value is 2^|MIS|
        ixs, iy, sizes, ts, edges = E.mis_network(16, 9)
        ts = [np.array([1.0, 2.0], np.float32)] * 16 + \
             [np.array([1.0, 1.0, 1.0, 0.0], np.float32)] * len(edges)
        alg = "maxmul"
    else:
        ixs, iy, sizes, ts, edges = E.ising_network(14, 9)
        alg = "standard"
    tree = E.greedy_tree(ixs, iy, sizes)
    sliced = N.choose_slices(ixs, iy, sizes, tree, 3, E.tree_cost)
    return E, N, oe, alg, ixs, iy, sizes, ts, edges, tree, sliced


def _worker(rank, world, init, kind, q):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    E, N, oe, alg, ixs, iy, sizes, ts, edges, tree, sliced = _case(kind)
    ex = N.OracleExecutor(oe, E, alg, ixs, iy, sizes, ts, tree)
    v, g, win = N.run_sliced(ex, alg, ixs, sizes, sliced, rank, world, dist=dist)
    q.put((rank, v, [x.tolist() for x in g], win))
    dist.barrier()
    dist.destroy_process_group()


def _init_file(tmp_path):
    """A rendezvous through a fresh file: no TCP port to race for between
    tests (a port found free can be taken again before the ranks bind it)."""
    return "file://" + str(tmp_path / "rendezvous")


@pytest.mark.parametrize("kind", ["mis", "maxmul", "ising"])
def test_two_gloo_ranks_match_single_rank_and_unsliced(kind, tmp_path):
    E, N, oe, alg, ixs, iy, sizes, ts, edges, tree, sliced = _case(kind)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init = _init_file(tmp_path)
    procs = [ctx.Process(target=_worker, args=(r, 2, init, kind, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # single rank, same sliced schedule
    ex = N.OracleExecutor(oe, E, alg, ixs, iy, sizes, ts, tree)
    v1, g1, w1 = N.run_sliced(ex, alg, ixs, sizes, sliced, 0, 1)
    ch, niy = E.encode_tree(tree, ixs, iy)
    unsliced = oe.einsum(alg, ts, ixs, iy, sizes, ch, niy)[0]
    for rank, v, g, win in res:
        if kind in ("mis", "maxmul"):
            assert v == v1 == unsliced and win == w1
            for x, y in zip(g, g1):
                np.testing.assert_array_equal(x, y)
            sel = [int(np.asarray(x)[1] != 0) for x in g[:16]]
            size = int(v) if kind == "mis" else int(round(np.log2(v)))
            assert sum(sel) == size and all(not (sel[a] and sel[b]) for a, b in edges)
        else:
            assert abs(v - unsliced) <= 1e-12 * abs(unsliced)
            for x, y in zip(g, g1):
                np.testing.assert_allclose(x, y, rtol=1e-12, atol=1e-300)


def test_order_key_is_monotone():
    _, N, _ = _mods()
    vals = [-np.inf, -3.5, -0.0, 0.0, 1e-30, 2.0, 7.0, np.inf]
    keys = [N.order_key(v, False) for v in vals]
    assert keys == sorted(keys)
    keys = [N.order_key(v, True) for v in vals]
    assert keys == sorted(keys, reverse=True)


def test_slice_grad_layout_matches_scatter():
    """The vectorised placement of sliced-view gradients equals the per-view
    scatter_slice_grad for every slice."""
    import importlib
    load_pkg()
    N = importlib.import_module("omeinsum_b200.network")
    ixs = [[0, 1, 2], [2, 3], [1], [3, 0]]
    sizes = {0: 2, 1: 3, 2: 2, 3: 4}
    sl = [1, 3]
    rng = np.random.default_rng(0)
    lay = N.SliceGradLayout(ixs, sizes, sl)
    for a in N.slice_assignments(sl, sizes):
        g = [rng.normal(size=int(np.prod([sizes[l] for l in ix if l not in sl]))) for ix in ixs]
        ref = np.concatenate([N.scatter_slice_grad(gi, ix, sizes, a,
                                                   int(np.prod([sizes[l] for l in ix])))
                              for gi, ix in zip(g, ixs)])
        assert np.array_equal(ref, lay.scatter(g, a))
        # device placement index: views concatenated in any order
        order = list(rng.permutation(len(ixs)))
        full = np.zeros(lay.total)
        full[lay.index_for(order, a)] = np.concatenate([g[v] for v in order])
        assert np.array_equal(full, ref)


def _leaving_worker(rank, world, init, q, dump):
    """Rank 1 computes its slices and leaves before the combine; rank 0 must
    get CombineError within the collective's time limit instead of hanging."""
    import faulthandler
    import sys
    import time
    # a stack dump of every thread if this rank is still alive after 60 s
    faulthandler.dump_traceback_later(60, exit=True, file=open(f"{dump}.{rank}", "w"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    E, N, oe, alg, ixs, iy, sizes, ts, edges, tree, sliced = _case("mis")
    ex = N.OracleExecutor(oe, E, alg, ixs, iy, sizes, ts, tree)
    if rank == 1:
        ex.value(N.slice_assignments(sliced, sizes)[1])
        os._exit(0)  # leaves between slices: no collective of its own in flight
    t0 = time.time()
    try:
        N.run_sliced(ex, alg, ixs, sizes, sliced, rank, world, dist=dist, timeout_s=5.0)
        q.put(("no error", time.time() - t0))
    except N.CombineError as e:
        q.put(("CombineError", time.time() - t0, str(e)[:200]))
    except BaseException as e:  # reported, so a failure says what happened
        q.put((type(e).__name__, time.time() - t0, str(e)[:200]))
    # the queue writes from a feeder thread: flush it before the hard exit
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_leaving_between_slices_gives_combine_error(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init = _init_file(tmp_path)
    dump = str(tmp_path / "stacks")
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, init, q, dump)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=120)
    except Exception:
        stacks = ""
        for r in range(2):
            if os.path.exists(f"{dump}.{r}"):
                stacks += f"--- rank {r}\n" + open(f"{dump}.{r}").read()
        raise AssertionError("no result from rank 0; stacks:\n" + stacks)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "CombineError", res
    assert res[1] < 60, res
