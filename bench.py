"""Benchmark of the hot path: the tropical binary contraction.

Workload (the config the target is quoted on):
MaxPlus<f32> 'ij,jk->ik' with i = j = k = 2048, argmax tracking on, inputs f32
U[-1,1) from the shared seeded generator.  One step = one
om_b200_contract call (the reference's Backend::contract_with_argmax).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints ONE JSON line (rank 0).  `value` is device-timed throughput with the
inputs resident in HBM (CUDA events on the backend's stream, L2 flushed by a
256 MiB write before every timed step); `e2e` is the same call made from
pinned host buffers with the host->device copies of A and B and the
device->host copies of C and argmax inside the timed region.  With N > 1 every
rank runs an independent replica (the binary contraction does not shard);
`value` is the sum over ranks using the max over ranks of the time.
`--impl reference` times the CPU restatement of the reference's
generic_gemm_with_argmax (oracle/) on all host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

M = N = K = 2048
SEED = 0x5EED
OPS = 2.0 * M * N * K  # one (x) and one (+) per (i, j, k)
METRIC = "tropical semiring GOP/s (binary contract)"
UNIT = "GOP/s"
WORKLOAD = "maxplus_f32_ij_jk_ik_2048x2048x2048_argmax"
# FP32 CUDA-core peak (MEASURED_PEAKS.json has no FP32 figure): 148 SMs x 128
# FP32 lanes x 2 (an FFMA counts as two operations) x 1965 MHz max SM clock.
FP32_PEAK_TOPS = 148 * 128 * 2 * 1.965e9 / 1e12
# Measured ceiling of the instruction pair the kernel is built on (one packed
# add.f32x2 + one 3-input max.f32 = 2 (+, max) steps = 4 operations) in a
# register-only loop: 39 pairs/clk/SM at 1965 MHz.
PAIR_CEILING_TOPS = 148 * 39 * 4 * 1.965e9 / 1e12
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant
# kernel, copied from an ncu capture of the same kernel and workload (ncu
# cannot run inside this process; the line labels the figure as copied).
NCU_TRAFFIC_BYTES = 48014336 + 53105920


def load_pkg():
    import importlib.util
    d = os.path.join(ROOT, "omeinsum-rs_b200")
    if "omeinsum_b200" in sys.modules:
        return sys.modules["omeinsum_b200"]
    spec = importlib.util.spec_from_file_location("omeinsum_b200", os.path.join(d, "__init__.py"),
                                                  submodule_search_locations=[d])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["omeinsum_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def inputs():
    import oracle as orc
    return orc.uniform(SEED, M * K), orc.uniform(SEED + 1, K * N)


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc = gpu, None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_sample(threads: int, rows: int):
    """Times the restated reference loop (generic_gemm_with_argmax) on the
    first `rows` rows of the workload (all columns, full k)."""
    import oracle as orc
    a, b = inputs()
    sub = np.ascontiguousarray(a.reshape(K, M)[:, :rows]).reshape(-1)
    t0 = time.perf_counter()
    orc.gemm("maxplus", sub, b, rows, K, N, argmax=True, threads=threads)
    dt = time.perf_counter() - t0
    return 2.0 * rows * N * K / dt / 1e9, dt


def run_reference(args, rank, world):
    import oracle as orc
    if rank != 0:
        return
    # every host core this process may run on (torchrun sets OMP_NUM_THREADS=1
    # for its ranks; the team size is passed explicitly instead)
    threads = max(orc.max_threads(), len(os.sched_getaffinity(0)))
    rows = max(8, min(M, int(os.environ.get("OM_BENCH_REF_ROWS", str(min(M, 32 * threads))))))
    for _ in range(args.warmup):
        cpu_sample(threads, max(8, rows // 8))
    vals, total = [], 0.0
    for _ in range(args.steps):
        v, dt = cpu_sample(threads, rows)
        vals.append(v)
        total += dt
    value = statistics.median(vals)
    sample = (f"rows 0..{rows - 1} of the {M}x{N}x{K} workload per step (all columns, full k), "
              f"oracle/ restatement of generic_gemm_with_argmax, OpenMP over columns")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded U[-1,1))",
        "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K, "algebra": "MaxPlus<f32>",
                   "argmax": True},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_permuted(be, om, local_rank):
    """'abcd,dcef->abfe', a=b=e=f=64, c=d=32, f32 N(0,1):
    Standard on the tensor cores (3xTF32) and on the CUDA cores (exact f32
    FMA), and MinPlus; plus the same contraction in Standard f64 (the DFMA
    kernel); device-timed per om_b200_contract call (kernels per
    class from the profiler), each output checked on sampled rows against
    the oracle first (Standard under the f32 rule, MinPlus bit-exact)."""
    import oracle as orc
    import torch
    a_, c_ = 64, 32
    sa, sb = [a_, a_, c_, c_], [c_, c_, a_, a_]
    ha, hb = orc.normal(SEED + 2, a_ * a_ * c_ * c_), orc.normal(SEED + 3, c_ * c_ * a_ * a_)
    A, B = be.from_slice(ha), be.from_slice(hb)
    C = be.alloc(a_ ** 4, np.float32)
    col = om.col_strides
    flops = 2.0 * 4096 * 4096 * 1024
    out = {"workload": "abcd,dcef->abfe a=b=e=f=64 c=d=32 f32 (and the same in f64)",
           "unit": "TFLOP/s (TOP/s)"}
    stream = torch.cuda.ExternalStream(be.stream(), device=local_rank)
    rows = np.array([0, 1, 777, 2048, 4095])
    sub = np.ascontiguousarray(ha.reshape(c_ * c_, a_ * a_)[:, rows].T).reshape(-1, order="F")
    ssub = [len(rows), c_, c_]
    A64, B64 = be.from_slice(ha.astype(np.float64)), be.from_slice(hb.astype(np.float64))
    C64 = be.alloc(a_ ** 4, np.float64)
    for alg, mode in (("standard", "3xtf32"), ("standard", "exact"), ("minplus", None),
                      ("standard", "f64")):
        if mode in ("3xtf32", "exact"):
            be.set_f32_mode(mode)
        f64 = mode == "f64"
        Ax, Bx, Cx = (A64, B64, C64) if f64 else (A, B, C)

        def call():
            be.contract_into(alg, Ax, sa, col(sa), [0, 1, 2, 3], Bx, sb, col(sb), [3, 2, 4, 5],
                             [a_] * 4, [0, 1, 5, 4], Cx, None)
        for _ in range(3):
            call()
        be.synchronize()
        # sampled-row check of this mode's output
        got = Cx.to_vec().reshape(a_ * a_, a_ * a_, order="F")[rows, :]
        if f64:
            r = orc.contract("standard", sub.astype(np.float64), ssub, col(ssub), [100, 2, 3],
                             hb.astype(np.float64), sb, col(sb), [3, 2, 4, 5],
                             [len(rows), a_, a_], [100, 5, 4]).reshape(len(rows), -1, order="F")
            bound = 1e-12 * np.maximum(np.abs(r), np.max(np.abs(r)))
            err = float(np.max(np.abs(got - r) / bound))
            check = {"rule": "|x-r| <= 1e-12 max(|r|, ||r||_inf)",
                     "max_err_over_bound": round(err, 4), "ok": err <= 1.0}
        elif alg == "standard":
            r = orc.contract("standard", sub.astype(np.float64), ssub, col(ssub), [100, 2, 3],
                             hb.astype(np.float64), sb, col(sb), [3, 2, 4, 5],
                             [len(rows), a_, a_], [100, 5, 4]).reshape(len(rows), -1, order="F")
            bound = np.maximum(1e-5 * np.abs(r), np.max(np.abs(r)) * 32 * 2.0 ** -23)
            err = float(np.max(np.abs(got - r) / bound))
            check = {"rule": "|x-r| <= max(1e-5|r|, ||r||_inf sqrt(K) 2^-23)",
                     "max_err_over_bound": round(err, 4), "ok": err <= 1.0}
        else:
            r = orc.contract("minplus", sub, ssub, col(ssub), [100, 2, 3], hb, sb, col(sb),
                             [3, 2, 4, 5], [len(rows), a_, a_], [100, 5, 4])
            ok = np.array_equal(got.view(np.uint32),
                                r.reshape(len(rows), -1, order="F").view(np.uint32))
            check = {"rule": "bit-exact", "ok": bool(ok)}
        be.profile(True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record(stream)
        for _ in range(reps):
            call()
        e1.record(stream)
        be.synchronize()
        ms = e0.elapsed_time(e1) / reps
        prof = be.profile_report()
        be.profile(False)
        key = alg if mode is None else f"{alg}_{mode}"
        out[key] = {"ms_per_call": round(ms, 4), "value": round(flops / (ms / 1e3) / 1e12, 2),
                    "kernels_ms": {k: round(v[0] / v[1], 4) for k, v in prof.items()},
                    "check_sampled_rows": check}
    be.set_f32_mode("3xtf32")
    return out


NET_N = 250
NET_SLICED = int(os.environ.get("OM_BENCH_NET_SLICED", "3"))
HBM_GBS = 6534.5  # MEASURED_PEAKS.json hbm_gbs (copy kernel, this pool's B200s)
# BASELINE config 4's order: tree annealing (om_b200_optimize_tree), seeded
TREESA = {"sc_target": 32.0, "ntrials": 4, "niters": 20, "seed": 2}
_NET_CACHE = {}


def config4_network(E, N, nsliced):
    """MIS on the seeded 3-regular graph with NET_N vertices, its annealed
    contraction tree and the nsliced labels the slicer picks (cached)."""
    key = nsliced
    if key not in _NET_CACHE:
        ixs, iy, sizes, ts, edges = E.mis_network(NET_N, SEED)
        if "tree" not in _NET_CACHE:
            _NET_CACHE["tree"] = E.treesa_tree(ixs, iy, sizes, **TREESA)[0]
        tree = _NET_CACHE["tree"]
        sliced = N.choose_slices(ixs, iy, sizes, tree, nsliced, E.tree_cost)
        _NET_CACHE[key] = (ixs, iy, sizes, ts, edges, tree, sliced)
    return _NET_CACHE[key]


def _events(torch, n):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def run_network(be, om, world, rank, local_rank, args, nsliced=None, cpu=False):
    """MIS on a seeded 3-regular graph with 250 vertices,
    MaxPlus f32, an annealed (TreeSA-method) contraction order, NET_SLICED
    sliced labels (2^NET_SLICED slices; 3 -> 8, config 4 as written) spread
    over the ranks, combined by an NCCL max-all-reduce carrying the slice id,
    then the argmax backward of the winning slice (the configuration)
    broadcast."""
    import importlib
    import torch
    E = importlib.import_module("omeinsum_b200.einsum")
    N = importlib.import_module("omeinsum_b200.network")
    nsliced = NET_SLICED if nsliced is None else nsliced
    ixs, iy, sizes, ts, edges, tree, sliced = config4_network(E, N, nsliced)
    tc, sc = E.tree_cost(tree, ixs, iy, sizes)
    s1 = dict(sizes)
    for l in sliced:
        s1[l] = 1
    tcs, scs = E.tree_cost(tree, ixs, iy, s1)
    ex = N.DeviceExecutor(be, E, "maxplus", ixs, iy, sizes, ts, tree)
    dist = torch.distributed if world > 1 else None
    dev = torch.device(f"cuda:{local_rank}")
    N.run_sliced(ex, "maxplus", ixs, sizes, sliced, rank, world, dist=dist, device=dev)  # warm-up
    assigns = N.slice_assignments(sliced, sizes)
    reps = 3
    stream = torch.cuda.ExternalStream(be.stream(), device=local_rank)
    t0, t1 = _events(torch, 2)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    be.synchronize()
    t0.record(stream)
    for _ in range(reps):
        v, g, win = N.run_sliced(ex, "maxplus", ixs, sizes, sliced, rank, world, dist=dist,
                                 device=dev)
    t1.record(stream)
    be.synchronize()
    torch.cuda.synchronize()
    ms = torch.tensor([t0.elapsed_time(t1) / reps], dtype=torch.float64, device=dev)
    # the two kinds of slice work, timed apart on this rank (diagnostic): a
    # slice at value cost (its intermediates kept) and the winner's backward
    layout = N._layout(ixs, sizes, sliced)
    gbuf = torch.zeros(1 + layout.total, dtype=torch.float32, device=dev)
    e0, e1, e2 = _events(torch, 3)
    e0.record(stream)
    _, bpos, slot = ex.best_of(assigns[:1], False)
    e1.record(stream)
    ex.grad_best_into(assigns[0], slot, layout, gbuf.data_ptr())
    e2.record(stream)
    be.synchronize()
    value_ms, grad_ms = e0.elapsed_time(e1), e1.elapsed_time(e2)
    if dist is not None:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    sel = [int(x[1] > x[0]) for x in g[:NET_N]]
    valid = sum(sel) == int(v) and all(not (sel[a] and sel[b]) for a, b in edges)
    nbytes = N.slice_node_bytes(tree, ixs, iy, sizes, sliced, 4, E.tree_output_labels)
    achieved = nbytes / (value_ms / 1e3) / 1e9
    out = {"workload": f"mis_3regular_n{NET_N}_maxplus_f32_{2 ** nsliced}_slices_argmax_backward",
           "metric": "network contract wall-time", "unit": "ms", "higher_is_better": False,
           "value": round(float(ms.item()), 3), "n_gpus": world, "scaling": "strong",
           "mis_size": v, "configuration_valid": bool(valid), "winning_slice": int(win),
           "log2_tc": round(float(np.log2(tc)), 2), "log2_sc": round(float(np.log2(sc)), 2),
           "per_slice_log2_tc": round(float(np.log2(tcs)), 2),
           "per_slice_log2_sc": round(float(np.log2(scs)), 2),
           "slices": 2 ** nsliced, "slice_value_ms": round(value_ms, 3),
           "winner_backward_ms": round(grad_ms, 3),
           "roofline": {"bound": "hbm", "bytes_per_slice": int(nbytes),
                        "achieved_gbs": round(achieved, 1), "peak_gbs": HBM_GBS,
                        "frac": round(achieved / HBM_GBS, 4),
                        "note": "operands read once + outputs written once over the nodes a "
                                "slice runs, / slice_value_ms; peak of measured (copy)"},
           "order": "tree annealing (om_b200_optimize_tree, TreeSA method) " + json.dumps(TREESA),
           "timing": "CUDA events on the backend stream around 3 full runs, max over ranks"}
    if cpu and rank == 0 and world == 1:
        # bounded CPU sample: one slice of the same tree cut into 64 slices
        # (per-slice log2 tc 3 lower; slicing adds no work on this tree, so
        # x64 is the whole network), checked against the device on that slice
        import engine as oe
        ixs6, iy6, sizes6, ts6, _, tree6, sliced6 = config4_network(E, N, 6)
        a6 = N.slice_assignments(sliced6, sizes6)
        ox = N.OracleExecutor(oe, E, "maxplus", ixs6, iy6, sizes6, ts6, tree6)
        t = time.perf_counter()
        ov = ox.value(a6[0])
        dt = time.perf_counter() - t
        dx = N.DeviceExecutor(be, E, "maxplus", ixs6, iy6, sizes6, ts6, tree6, use_graph=False)
        assert ov == dx.value(a6[0]), "network check"
        del dx
        out["cpu_baseline"] = {"value": round(dt * 1e3 * len(a6), 1), "unit": "ms",
                               "cores": 1, "kind": "port",
                               "sample": f"oracle engine, value of slice 0 of the same tree cut "
                                         f"into {len(a6)} slices ({dt:.1f} s) x {len(a6)}; "
                                         "the gradient is left out"}
    return out


def run_config3(be, om, local_rank, cpu=False):
    """MIS on a seeded 3-regular graph with 150 vertices,
    MaxPlus f32, greedy order, value and argmax backward (the configuration)
    on one GPU through the engine (om_b200_einsum + backward)."""
    import importlib
    import torch
    E = importlib.import_module("omeinsum_b200.einsum")
    ixs, iy, sizes, ts, edges = E.mis_network(150, SEED)
    ein = E.Einsum(ixs, iy, sizes).optimize_greedy()
    tc, sc = E.tree_cost(ein.tree, ixs, iy, sizes)
    dev = [be.from_slice(t) for t in ts]
    stream = torch.cuda.ExternalStream(be.stream(), device=local_rank)
    # the forward (values-only tape: no argmax in the nodes) recorded once as
    # a CUDA graph; each call replays it and runs the backward, which finds
    # the argmax of just the entries it visits
    graph, c, tape = ein.record_forward(be, "maxplus", dev, values_only=True)
    d = be.from_slice(np.ones(1, np.float32))
    g = [be.alloc(t.n, t.dtype) for t in dev]

    def call():
        graph.launch()
        E.Einsum.backward_tape(tape, d, g)

    for _ in range(2):
        call()
    be.synchronize()
    reps = 5
    e0, e1 = _events(torch, 2)
    e0.record(stream)
    for _ in range(reps):
        call()
    e1.record(stream)
    be.synchronize()
    ms = e0.elapsed_time(e1) / reps
    val = float(c.to_vec()[0])
    # the same answer as the engine's eager argmax-tape path, bit for bit
    c2, g2 = ein.cost_and_gradient(be, "maxplus", dev, dy=[1.0])
    assert c2.to_vec()[0] == val and all(np.array_equal(x.to_vec(), y.to_vec())
                                         for x, y in zip(g, g2)), "config 3 gradient check"
    E.Einsum.tape_free(tape)
    sel = [int(x.to_vec()[1] > 0) for x in g[:150]]
    valid = sum(sel) == int(val) and all(not (sel[u] and sel[v]) for u, v in edges)
    out = {"workload": "mis_3regular_n150_maxplus_f32_greedy_value_and_argmax_backward",
           "metric": "network contract wall-time", "unit": "ms", "higher_is_better": False,
           "value": round(ms, 3), "mis_size": val, "configuration_valid": bool(valid),
           "log2_tc": round(float(np.log2(tc)), 2), "log2_sc": round(float(np.log2(sc)), 2),
           "timing": "CUDA events on the backend stream around 5 value+gradient calls (forward "
                     "replayed from one recorded graph, backward eager)"}
    if cpu:
        import engine as oe
        ch, niy = ein.encoded()
        t = time.perf_counter()
        rc, _ = oe.cost_and_gradient("maxplus", ts, ixs, iy, sizes, ch, niy,
                                     np.ones(1, np.float32))
        dt = time.perf_counter() - t
        assert float(rc[0]) == val, "config 3 check"
        out["cpu_baseline"] = {"value": round(dt * 1e3, 1), "unit": "ms", "cores": 1,
                               "kind": "port",
                               "sample": "oracle engine, whole value + argmax backward, same tree"}
    return out


def run_config5(be, om, world, rank, local_rank, cpu=False):
    """Ising spin glass on a seeded 3-regular graph with
    120 vertices, Standard f64, beta = 1, J ~ N(0, 1), 3 sliced labels (8
    slices) over the ranks, Z and dZ/dT for every edge tensor, combined by an
    NCCL sum all-reduce on the device."""
    import importlib
    import torch
    E = importlib.import_module("omeinsum_b200.einsum")
    N = importlib.import_module("omeinsum_b200.network")
    ixs, iy, sizes, ts, edges = E.ising_network(120, SEED)
    tree = E.best_tree(ixs, iy, sizes, restarts=8)
    sliced = N.choose_slices(ixs, iy, sizes, tree, 3, E.tree_cost)
    tc, sc = E.tree_cost(tree, ixs, iy, sizes)
    ex = N.DeviceExecutor(be, E, "standard", ixs, iy, sizes, ts, tree)
    dist = torch.distributed if world > 1 else None
    dev = torch.device(f"cuda:{local_rank}")
    for _ in range(2):
        N.run_sliced(ex, "standard", ixs, sizes, sliced, rank, world, dist=dist, device=dev)
    stream = torch.cuda.ExternalStream(be.stream(), device=local_rank)
    reps = 5
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    be.synchronize()
    e0, e1 = _events(torch, 2)
    e0.record(stream)
    for _ in range(reps):
        z, g, _ = N.run_sliced(ex, "standard", ixs, sizes, sliced, rank, world, dist=dist,
                               device=dev)
    e1.record(stream)
    be.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    out = {"workload": "ising_3regular_n120_standard_f64_8_slices_z_and_edge_gradients",
           "metric": "network contract wall-time", "unit": "ms", "higher_is_better": False,
           "value": round(float(ms.item()), 3), "n_gpus": world, "scaling": "strong",
           "log_z": round(float(np.log(z)), 6), "edges_with_gradient": len(g),
           "log2_tc": round(float(np.log2(tc)), 2), "log2_sc": round(float(np.log2(sc)), 2),
           "timing": "CUDA events on the backend stream around 5 full runs, max over ranks"}
    if cpu and rank == 0 and world == 1:
        import engine as oe
        ox = N.OracleExecutor(oe, E, "standard", ixs, iy, sizes, ts, tree)
        t = time.perf_counter()
        oz, og, _ = N.run_sliced(ox, "standard", ixs, sizes, sliced, 0, 1)
        dt = time.perf_counter() - t
        assert abs(oz - z) <= 1e-12 * abs(oz), "config 5 check"
        out["cpu_baseline"] = {"value": round(dt * 1e3, 1), "unit": "ms", "cores": 1,
                               "kind": "port",
                               "sample": "oracle engine, all 8 slices with gradients, same tree"}
    return out


def run_b200(args, rank, world, local_rank):
    import torch
    om = load_pkg()
    torch.cuda.set_device(local_rank)
    be = om.B200(local_rank)
    a, b = inputs()
    A, B = be.from_slice(a), be.from_slice(b)
    C = be.alloc(M * N, np.float32)
    AM = be.alloc(M * N, np.uint32)
    stream = torch.cuda.ExternalStream(be.stream(), device=local_rank)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local_rank}")

    def step():
        be.contract_into("maxplus", A, [M, K], [1, M], [0, 1], B, [K, N], [1, K], [1, 2],
                         [M, N], [0, 2], C, AM)

    for _ in range(args.warmup):
        step()
    be.synchronize()

    # correctness guard on the benchmarked output (sampled rows vs the oracle)
    if rank == 0 and not args.no_check:
        import oracle as orc
        rows = [0, 777, 2047]
        cv, av = C.to_vec().reshape(N, M), AM.to_vec().reshape(N, M)
        sub = np.ascontiguousarray(a.reshape(K, M)[:, rows]).reshape(-1)
        rc, ram = orc.gemm("maxplus", sub, b, len(rows), K, N, argmax=True,
                           threads=orc.max_threads())
        assert np.array_equal(cv[:, rows].reshape(-1).view(np.uint32),
                              rc.reshape(N, len(rows)).reshape(-1).view(np.uint32)), "bench check"
        assert np.array_equal(av[:, rows].reshape(-1), ram.reshape(N, len(rows)).reshape(-1))

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        be.synchronize()

    # ---- device-timed region: inputs resident in HBM ----------------------
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    om.launch_count()
    be.profile(True)
    barrier()
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.fill_(i & 0xFF)  # L2 flush, outside the events
                ev[i][0].record(stream)
            step()
            with torch.cuda.stream(stream):
                ev[i][1].record(stream)
        barrier()
    launches = om.launch_count()
    prof = be.profile_report()
    be.profile(False)
    step_ms = [s.elapsed_time(e) for s, e in ev]
    total_ms = sum(step_ms)
    t_local = torch.tensor([total_ms], dtype=torch.float64, device=f"cuda:{local_rank}")
    if world > 1:
        torch.distributed.all_reduce(t_local, op=torch.distributed.ReduceOp.MAX)
    t_max = float(t_local.item())
    value = world * args.steps * OPS / (t_max / 1e3) / 1e9

    # ---- end-to-end: pinned host buffers through the C ABI ------------------
    # Every step uploads its inputs from pinned host memory, contracts and
    # reads back C and the argmax.  Several backends (streams; 4 by default)
    # take the steps in turn, so one step's copies run on the copy engines
    # while another step's contraction runs: the throughput a caller gets by
    # keeping that many steps in flight.
    L = om.lib()
    nlanes = int(os.environ.get("OM_BENCH_E2E_LANES", "4"))
    extra = [om.B200(local_rank) for _ in range(nlanes - 1)]
    ha = torch.from_numpy(a).pin_memory()
    hb = torch.from_numpy(b).pin_memory()
    lanes = []
    for bx in [be] + extra:
        lanes.append({"be": bx, "A": bx.alloc(M * K, np.float32), "B": bx.alloc(K * N, np.float32),
                      "C": bx.alloc(M * N, np.float32), "AM": bx.alloc(M * N, np.uint32),
                      "hc": torch.empty(M * N, dtype=torch.float32).pin_memory(),
                      "hm": torch.empty(M * N, dtype=torch.int32).pin_memory()})

    def e2e_step(i):
        ln = lanes[i % nlanes]
        bx = ln["be"]
        om._check(L.om_b200_upload(bx.h, ln["A"].ptr, ha.data_ptr(), ln["A"].nbytes))
        om._check(L.om_b200_upload(bx.h, ln["B"].ptr, hb.data_ptr(), ln["B"].nbytes))
        bx.contract_into("maxplus", ln["A"], [M, K], [1, M], [0, 1], ln["B"], [K, N], [1, K],
                         [1, 2], [M, N], [0, 2], ln["C"], ln["AM"])
        om._check(L.om_b200_download_async(bx.h, ln["hc"].data_ptr(), ln["C"].ptr, ln["C"].nbytes))
        om._check(L.om_b200_download_async(bx.h, ln["hm"].data_ptr(), ln["AM"].ptr,
                                           ln["AM"].nbytes))

    def e2e_sync():
        for ln in lanes:
            ln["be"].synchronize()

    for i in range(max(2, args.warmup)):
        e2e_step(i)
    e2e_sync()
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    e2e_sync()
    barrier()
    e2e_s = time.perf_counter() - t0
    # the read-back results are the benchmarked ones
    if rank == 0 and not args.no_check:
        assert np.array_equal(lanes[(args.steps - 1) % nlanes]["hc"].numpy().view(np.uint32),
                              C.to_vec().view(np.uint32)), "e2e check"
        assert np.array_equal(lanes[(args.steps - 1) % nlanes]["hm"].numpy().view(np.uint32), AM.to_vec())
    for bx in extra:
        bx.close()
    t_e2e = torch.tensor([e2e_s], dtype=torch.float64, device=f"cuda:{local_rank}")
    if world > 1:
        torch.distributed.all_reduce(t_e2e, op=torch.distributed.ReduceOp.MAX)
    e2e_value = world * args.steps * OPS / float(t_e2e.item()) / 1e9

    permuted = network = network64 = config5 = config3 = None
    if not args.headline_only:
        permuted = run_permuted(be, om, local_rank) if rank == 0 else None
        cpu_nets = world == 1 and not args.no_cpu
        # config 4 as written (3 sliced labels, 8 slices), and cut into 64
        network = run_network(be, om, world, rank, local_rank, args, cpu=cpu_nets)
        network64 = run_network(be, om, world, rank, local_rank, args, nsliced=6)
        config5 = run_config5(be, om, world, rank, local_rank, cpu=cpu_nets)
        config3 = run_config3(be, om, local_rank, cpu=cpu_nets) if rank == 0 else None
    if rank != 0:
        return
    # roofline of the dominant kernel (device time per launch from the events)
    top = max(prof.items(), key=lambda kv: kv[1][0]) if prof else ("?", (0.0, 1))
    kname, (kms, kn) = top
    achieved = OPS / (kms / kn / 1e3) / 1e12 if kn and kms else None
    threads_cpu = 1
    cpu_rows = int(os.environ.get("OM_BENCH_CPU_ROWS", str(M)))
    # the CPU baseline is an N = 1 figure; multi-GPU lines leave it out
    cpu_val, cpu_dt = cpu_sample(threads_cpu, cpu_rows) if world == 1 else (None, None)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded U[-1,1), splitmix64/xoshiro256**)",
        "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K, "algebra": "MaxPlus<f32>",
                   "argmax": True, "parallelism": f"replicas x{world}" if world > 1 else "single",
                   "l2": "flushed before each timed step (256 MiB write, untimed)"},
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": int(A.nbytes + B.nbytes),
                "d2h_bytes_per_step": int(C.nbytes + AM.nbytes),
                "pipelining": f"{nlanes} backends (streams) take the steps in turn; wall clock"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "fp32", "kernel": kname,
                     "achieved": None if achieved is None else round(achieved, 2),
                     "peak": round(FP32_PEAK_TOPS, 2), "unit": "TOP/s",
                     "frac": None if achieved is None else round(achieved / FP32_PEAK_TOPS, 4),
                     "peak_source": "computed: 148 SMs x 128 FP32 lanes x 2 x 1965 MHz "
                                    "(no FP32 figure in MEASURED_PEAKS.json)",
                     "instruction_ceiling": round(PAIR_CEILING_TOPS, 2),
                     "frac_of_instruction_ceiling": None if achieved is None
                     else round(achieved / PAIR_CEILING_TOPS, 4),
                     "traffic": NCU_TRAFFIC_BYTES,
                     "traffic_source": "copied from an ncu capture of this kernel on this "
                                       "workload (dram__bytes_read.sum + dram__bytes_write.sum)"},
        "kernels": {k: {"ms_total": round(v[0], 4), "launches": v[1]} for k, v in prof.items()},
        "cpu_baseline": None if cpu_val is None else {
            "value": round(cpu_val, 4), "unit": UNIT, "cores": threads_cpu, "kind": "port",
            "sample": f"rows 0..{cpu_rows - 1} of the workload (all columns, full k), "
                      f"reference loop order, {cpu_dt:.1f} s"},
        "clocks": clk.summary(),
        "network": network,
        "network_64_slices": network64,
        "ising_n120_f64_sliced_grad": config5,
        "config3_mis_n150": config3,
        "permuted": permuted,
    }
    print(json.dumps(line), flush=True)
    be.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-check", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="leave out the network CPU baselines")
    ap.add_argument("--headline-only", action="store_true",
                    help="only the headline contraction (no config-2 / network objects)")
    ap.add_argument("--case", default="headline", choices=["headline", "config2", "contract", "network", "slices",
                             "networks", "scaling", "f64"],
                    help="profiling cases: config2 = only the config-2 permuted "
                         "contraction; contract = only warmup + steps headline calls; "
                         "network = only the sliced MIS network, with its kernel breakdown; "
                         "slices = ten eager slice contractions of that network (profiling)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.case == "f64":  # profiling: Standard f64 config-2 shape, 5 calls
        om = load_pkg()
        be = om.B200(local_rank)
        import oracle as orc
        a_, c_ = 64, 32
        sa, sb = [a_, a_, c_, c_], [c_, c_, a_, a_]
        A = be.from_slice(orc.normal(SEED + 2, a_ ** 2 * c_ ** 2).astype(np.float64))
        B = be.from_slice(orc.normal(SEED + 3, a_ ** 2 * c_ ** 2).astype(np.float64))
        C = be.alloc(a_ ** 4, np.float64)
        for _ in range(5):
            be.contract_into("standard", A, sa, om.col_strides(sa), [0, 1, 2, 3], B, sb,
                             om.col_strides(sb), [3, 2, 4, 5], [a_] * 4, [0, 1, 5, 4], C, None)
        be.synchronize()
        print(json.dumps({"case": "f64", "calls": 5}), flush=True)
        be.close()
        return
    if args.case == "config2":
        import torch
        om = load_pkg()
        torch.cuda.set_device(local_rank)
        be = om.B200(local_rank)
        print(json.dumps(run_permuted(be, om, local_rank)), flush=True)
        be.close()
        return
    if args.case == "networks" and world == 1:
        import torch
        om = load_pkg()
        torch.cuda.set_device(local_rank)
        be = om.B200(local_rank)
        be.profile(True)
        out = {"config5": run_config5(be, om, 1, 0, local_rank),
               "config3": run_config3(be, om, local_rank)}
        prof = be.profile_report()
        be.profile(False)
        out["kernels_ms_total"] = {k: [round(v[0], 3), v[1]] for k, v in
                                   sorted(prof.items(), key=lambda kv: -kv[1][0])}
        print(json.dumps(out), flush=True)
        be.close()
        return
    if args.case == "network" and world == 1:
        import torch
        om = load_pkg()
        torch.cuda.set_device(local_rank)
        be = om.B200(local_rank)
        be.profile(True)
        net = run_network(be, om, 1, 0, local_rank, args)
        prof = be.profile_report()
        be.profile(False)
        net["kernels_ms_total"] = {k: [round(v[0], 3), v[1]] for k, v in
                                   sorted(prof.items(), key=lambda kv: -kv[1][0])}
        print(json.dumps(net), flush=True)
        be.close()
        return
    if args.case == "scaling":
        # the sliced networks alone, at N ranks (scaling runs of those objects)
        import torch
        om = load_pkg()
        torch.cuda.set_device(local_rank)
        if world > 1:
            torch.distributed.init_process_group("nccl", device_id=torch.device(f"cuda:{local_rank}"))
        be = om.B200(local_rank)
        out = {"network": run_network(be, om, world, rank, local_rank, args),
               "network_64_slices": run_network(be, om, world, rank, local_rank, args, nsliced=6),
               "config5": run_config5(be, om, world, rank, local_rank)}
        if rank == 0:
            print(json.dumps(out), flush=True)
        be.close()
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    if args.case == "slices" and world == 1:
        import importlib
        import torch
        om = load_pkg()
        torch.cuda.set_device(local_rank)
        be = om.B200(local_rank)
        E = importlib.import_module("omeinsum_b200.einsum")
        N = importlib.import_module("omeinsum_b200.network")
        ixs, iy, sizes, ts, _, tree, sliced = config4_network(E, N, NET_SLICED)
        ex = N.DeviceExecutor(be, E, "maxplus", ixs, iy, sizes, ts, tree, use_graph=False)
        assigns = N.slice_assignments(sliced, sizes)
        vals = [ex.value(assigns[q]) for q in range(min(4, len(assigns)))]
        print(json.dumps({"case": "slices", "values": vals}), flush=True)
        del ex
        be.close()
        return
    if args.case == "contract":
        import torch
        om = load_pkg()
        torch.cuda.set_device(local_rank)
        be = om.B200(local_rank)
        a, b = inputs()
        A, B = be.from_slice(a), be.from_slice(b)
        C, AM = be.alloc(M * N, np.float32), be.alloc(M * N, np.uint32)
        for _ in range(args.warmup + args.steps):
            be.contract_into("maxplus", A, [M, K], [1, M], [0, 1], B, [K, N], [1, K], [1, 2],
                             [M, N], [0, 2], C, AM)
        be.synchronize()
        print(json.dumps({"case": "contract", "calls": args.warmup + args.steps}), flush=True)
        be.close()
        return
    if world > 1:
        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", device_id=torch.device(f"cuda:{local_rank}"))
    try:
        run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
