"""Writes tests/golden/kats.json: known-answer vectors of the reference's own
tests for the binary-contraction path, transcribed from the test sources of
tensor4all/omeinsum-rs (the reference cannot be compiled here: no Rust
toolchain).  Each entry cites the test it comes from.  Expected arrays are the
reference's asserted values; entries whose reference test asserts only
lengths carry "expected": null and are checked device-vs-oracle instead.

Run:  python tests/golden/make_kats.py
"""
import json
import math
import os

INF = math.inf
FMAX = 3.4028234663852886e38  # f32::MAX

KATS = []


def contract(name, cite, alg, dtype, a, sa, ta, ma, b, sb, tb, mb, sc, mc,
             expected=None, argmax=None, with_argmax=False):
    KATS.append(dict(kind="contract", name=name, cite=cite, alg=alg, dtype=dtype,
                     a=a, shape_a=sa, strides_a=ta, modes_a=ma,
                     b=b, shape_b=sb, strides_b=tb, modes_b=mb,
                     shape_c=sc, modes_c=mc, expected=expected,
                     expected_argmax=argmax, with_argmax=with_argmax or argmax is not None))


# tests/suites/backend_contract.rs -------------------------------------------
BC = "tests/suites/backend_contract.rs"
contract("matmul", BC + ":7-33", "standard", "f64", [1, 2, 3, 4], [2, 2], [1, 2], [0, 1],
         [5, 6, 7, 8], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [23, 34, 31, 46])
contract("inner_product", BC + ":35-47", "standard", "f64", [1, 2, 3], [3], [1], [0],
         [4, 5, 6], [3], [1], [0], [], [], [32])
contract("outer_product", BC + ":49-63", "standard", "f64", [1, 2], [2], [1], [0],
         [3, 4, 5], [3], [1], [1], [2, 3], [0, 1], [3, 6, 4, 8, 5, 10])
contract("batched_batch_first", BC + ":65-89", "standard", "f64",
         [1, 5, 2, 6, 3, 7, 4, 8], [2, 2, 2], [1, 2, 4], [0, 1, 2],
         [1, 2, 0, 0, 0, 0, 1, 2], [2, 2, 2], [1, 2, 4], [0, 2, 3],
         [2, 2, 2], [0, 1, 3], [1, 10, 2, 12, 3, 14, 4, 16])
contract("maxplus_2x2", BC + ":91-126", "maxplus", "f64", [1, 2, 3, 4], [2, 2], [1, 2], [0, 1],
         [1, 2, 3, 4], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [5, 6, 7, 8])
contract("strided_input", BC + ":132-160", "standard", "f64", [1, 2, 3, 4, 5, 6, 7, 8, 9],
         [2, 2], [1, 3], [0, 1], [1, 0, 0, 1], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2],
         [1, 2, 4, 5])
contract("both_strided", BC + ":162-198", "standard", "f64", list(range(1, 17)),
         [2, 2], [1, 4], [0, 1], [9, 10, 11, 12, 13, 14, 15, 16, 1, 2, 3, 4, 5, 6, 7, 8],
         [2, 2], [1, 4], [1, 2], [2, 2], [0, 2], [59, 78, 83, 110])
contract("rhs_transpose_view", BC + ":200-233", "standard", "f64", [1, 2, 3, 4], [2, 2], [1, 2],
         [0, 1], [1, 2, 3, 4], [2, 2], [2, 1], [1, 2], [2, 2], [0, 2], [10, 14, 14, 20])
contract("output_permuted", BC + ":239-264", "standard", "f64", [1, 2, 3, 4], [2, 2], [1, 2],
         [0, 1], [5, 6, 7, 8], [2, 2], [1, 2], [1, 2], [2, 2], [2, 0], [23, 31, 34, 46])
contract("batched_output_permuted", BC + ":266-290", "standard", "f64",
         [1, 5, 2, 6, 3, 7, 4, 8], [2, 2, 2], [1, 2, 4], [0, 1, 2],
         [1, 1, 0, 0, 0, 0, 1, 1], [2, 2, 2], [1, 2, 4], [0, 2, 3],
         [2, 2, 2], [3, 1, 0], [1, 3, 2, 4, 5, 7, 6, 8])
contract("argmax_2x2", BC + ":296-326", "maxplus", "f64", [1, 2, 3, 4], [2, 2], [1, 2], [0, 1],
         [1, 2, 3, 4], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [5, 6, 7, 8], [1, 1, 1, 1])
contract("argmax_strided", BC + ":328-352 (length check)", "maxplus", "f64",
         [1, 2, 3, 4, 5, 6, 7, 8, 9], [2, 2], [1, 3], [0, 1], [1, 0, 0, 1], [2, 2], [1, 2],
         [1, 2], [2, 2], [0, 2], with_argmax=True)
contract("argmax_output_permuted", BC + ":354-382", "maxplus", "f64", [1, 2, 3, 4], [2, 2],
         [1, 2], [0, 1], [1, 2, 3, 4], [2, 2], [1, 2], [1, 2], [2, 2], [2, 0],
         [5, 7, 6, 8], with_argmax=True)
contract("argmax_batched", BC + ":384-412 (length check)", "maxplus", "f64",
         [1, 2, 3, 4, 5, 6, 7, 8], [2, 2, 2], [1, 2, 4], [0, 1, 2],
         [1, 2, 3, 4, 1, 2, 3, 4], [2, 2, 2], [1, 2, 4], [0, 2, 3], [2, 2, 2], [0, 1, 3],
         with_argmax=True)
contract("matmul_f32", BC + ":418-439", "standard", "f32", [1, 2, 3, 4], [2, 2], [1, 2], [0, 1],
         [5, 6, 7, 8], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [23, 34, 31, 46])

# src/backend/cpu/mod.rs unit tests ------------------------------------------
CM = "src/backend/cpu/mod.rs"
contract("gemm_standard", CM + ":1138-1147", "standard", "f32", [1, 2, 3, 4], [2, 2], [1, 2],
         [0, 1], [1, 2, 3, 4], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [7, 10, 15, 22])
contract("gemm_maxplus", CM + ":1256-1265", "maxplus", "f32", [1, 2, 3, 4], [2, 2], [1, 2],
         [0, 1], [1, 2, 3, 4], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [5, 6, 7, 8])
contract("gemm_with_argmax", CM + ":1268-1279", "maxplus", "f32", [1, 2, 3, 4], [2, 2], [1, 2],
         [0, 1], [1, 2, 3, 4], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [5, 6, 7, 8], [1, 1, 1, 1])
# gemm_batched_internal: A/B batch-last ([m,k,batch]) == modes [i,j,b],[j,k,b]->[i,k,b]
contract("gemm_batched_f32", CM + ":1240-1250", "standard", "f32", [1, 2, 3, 4, 5, 6, 7, 8],
         [2, 2, 2], [1, 2, 4], [0, 1, 9], [1, 2, 3, 4, 1, 0, 0, 1], [2, 2, 2], [1, 2, 4],
         [1, 2, 9], [2, 2, 2], [0, 2, 9], [7, 10, 15, 22, 5, 6, 7, 8])
KATS.append(dict(kind="copy_strided", name="copy_strided", cite=CM + ":1282-1290", dtype="f32",
                 src=[1, 2, 3, 4, 5, 6], shape=[3, 2], strides=[2, 1], offset=0,
                 expected=[1, 3, 5, 2, 4, 6]))

# tests/suites/tropical.rs (einsum-level pins that reduce to one contraction) --
TR = "tests/suites/tropical.rs"
# d2[0] = 0, d2[1] = 1, d2[2] = 3 (only those entries asserted); whole vector
# follows from the semiring rules with zero() = f32::MAX for MinPlus.
contract("minplus_shortest_path", TR + ":26-58", "minplus", "f32",
         [0, 1, INF, INF, 0, 2, INF, INF, 0], [3, 3], [1, 3], [0, 1],
         [0, 1, INF, INF, 0, 2, INF, INF, 0], [3, 3], [1, 3], [1, 2], [3, 3], [0, 2],
         None)
KATS[-1]["expected_partial"] = {"0": 0.0, "1": 1.0, "2": 3.0}
contract("maxplus_viterbi", TR + ":147-166", "maxplus", "f32", [-1, -2, -3, -1], [2, 2], [1, 2],
         [0, 1], [0, -1], [2, 1], [1, 2], [1, 2], [2, 1], [0, 2], [-1, -2])
contract("minplus_bellman_ford", TR + ":172-205", "minplus", "f32",
         [0, 4, 2, INF, 0, 3, INF, INF, 0], [3, 3], [1, 3], [0, 1],
         [0, INF, INF], [3, 1], [1, 3], [1, 2], [3, 1], [0, 2], [0, 4, 2])
contract("maxplus_identity", TR + ":61-70", "maxplus", "f32", [1, 2, 3, 4], [2, 2], [1, 2],
         [0, 1], [0, -INF, -INF, 0], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [1, 2, 3, 4])
contract("minplus_identity", TR + ":72-81", "minplus", "f32", [1, 2, 3, 4], [2, 2], [1, 2],
         [0, 1], [0, INF, INF, 0], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], [1, 2, 3, 4])
# semiring constants (tropical.rs:208-229): zero() of each algebra, seen through an
# all-(-inf) MaxPlus reduction (result f32::MIN) and an all-(+inf) MinPlus one.
contract("maxplus_all_neg_inf", TR + ":208-229 (zero = f32::MIN)", "maxplus", "f32",
         [-INF, -INF], [1, 2], [1, 1], [0, 1], [0, 0], [2, 1], [1, 2], [1, 2], [1, 1], [0, 2],
         [-FMAX], [0])
contract("minplus_all_pos_inf", TR + ":208-229 (zero = f32::MAX)", "minplus", "f32",
         [INF, INF], [1, 2], [1, 1], [0, 1], [0, 0], [2, 1], [1, 2], [1, 2], [1, 1], [0, 2],
         [FMAX], [0])
contract("maxmul_2x2", TR + ":86-109", "maxmul", "f32", [0.5, 0.3, 0.2, 0.8], [2, 2], [1, 2],
         [0, 1], [0.9, 0.1, 0.4, 0.6], [2, 2], [1, 2], [1, 2], [2, 2], [0, 2], None)
KATS[-1]["expected_approx"] = [0.45, 0.27, 0.20, 0.48]


def _clean(v):
    if isinstance(v, float) and math.isinf(v):
        return "inf" if v > 0 else "-inf"
    if isinstance(v, list):
        return [_clean(x) for x in v]
    if isinstance(v, dict):
        return {k: _clean(x) for k, x in v.items()}
    return v


if __name__ == "__main__":
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kats.json")
    with open(out, "w") as f:
        json.dump([_clean(k) for k in KATS], f, indent=1)
    print(f"wrote {len(KATS)} KATs to {out}")
