// Device-side semiring scalar operations.
//
// These restate the reference's scalar semantics exactly
// (tensor4all/omeinsum-rs src/algebra/tropical.rs:46-143,169-263,289-384 and
// src/algebra/standard.rs:26-116):
//   zero():  MaxPlus -FLT_MAX (f32::MIN), MinPlus +FLT_MAX, MaxMul 0, Standard 0
//   add(acc, p) keeps acc when acc >= p (max algebras) / acc <= p (MinPlus),
//   so the first index wins a tie and a NaN accumulator is replaced by p.
//   is_better is strict (>, <).
#pragma once

#include <cfloat>
#include <cstdint>

#include "omeinsum_b200.h"

namespace om {

template <typename T>
struct Lim;
template <>
struct Lim<float> {
  __host__ __device__ static constexpr float max() { return FLT_MAX; }
};
template <>
struct Lim<double> {
  __host__ __device__ static constexpr double max() { return DBL_MAX; }
};

template <int ALG, typename T>
struct Semi {
  __device__ __forceinline__ static T zero() {
    if (ALG == OM_MAXPLUS) return -Lim<T>::max();
    if (ALG == OM_MINPLUS) return Lim<T>::max();
    return T(0);
  }
  __device__ __forceinline__ static T mul(T a, T b) {
    if (ALG == OM_MAXPLUS || ALG == OM_MINPLUS) return a + b;
    return a * b;
  }
  // true when the accumulator is kept (Semiring::add / add_with_argmax)
  __device__ __forceinline__ static bool keep(T acc, T p) {
    if (ALG == OM_MINPLUS) return acc <= p;
    return acc >= p;
  }
  __device__ __forceinline__ static T add(T acc, T p) {
    if (ALG == OM_STANDARD) return acc + p;
    return keep(acc, p) ? acc : p;
  }
  // Algebra::is_better (strict)
  __device__ __forceinline__ static bool better(T v, T best) {
    if (ALG == OM_MINPLUS) return v < best;
    if (ALG == OM_STANDARD) return false;
    return v > best;
  }
};

// Special-value summary of the operands of a tropical GEMM, written by the
// scan kernel in front of the fast path.
enum : uint32_t {
  SV_NAN = 1u << 0,
  SV_A_PINF = 1u << 1,
  SV_A_NINF = 1u << 2,
  SV_B_PINF = 1u << 3,
  SV_B_NINF = 1u << 4,
  SV_NEGZERO = 1u << 5,
};

// The fast tropical GEMM computes max/min with 3-input max/min instructions,
// which drop NaN operands and may return either zero on a +0/-0 tie.  It is
// exact whenever no product can be NaN and no product can be -0; otherwise
// the exact compare-select kernel runs instead.
__host__ __device__ inline bool fast_path_ruled_out(uint32_t f, int alg) {
  if (f & SV_NAN) return true;
  if (alg == OM_MAXMUL) return (f & (SV_A_PINF | SV_A_NINF | SV_B_PINF | SV_B_NINF)) != 0;
  if (f & SV_NEGZERO) return true;
  return ((f & SV_A_PINF) && (f & SV_B_NINF)) || ((f & SV_A_NINF) && (f & SV_B_PINF));
}

}  // namespace om

// Dispatch a runtime algebra to a template parameter.
#define OM_DISPATCH_ALG(alg, ALGV, ...)                 \
  switch (alg) {                                        \
    case OM_STANDARD: { constexpr int ALGV = OM_STANDARD; __VA_ARGS__; break; } \
    case OM_MAXPLUS: { constexpr int ALGV = OM_MAXPLUS; __VA_ARGS__; break; }   \
    case OM_MINPLUS: { constexpr int ALGV = OM_MINPLUS; __VA_ARGS__; break; }   \
    case OM_MAXMUL: { constexpr int ALGV = OM_MAXMUL; __VA_ARGS__; break; }     \
    default: return ::om::set_error(OM_ERR_UNSUPPORTED, "unknown algebra");     \
  }
