// fpmod.cuh -- modular products on the FP64 pipe, and carry-free split
// products on the integer pipe.
//
// B200's FP64 pipe executes 64 operations per SM per cycle, while the
// 32 x 32 -> 64-bit integer multiply-add (IMAD.WIDE) that 64-bit modular
// products are built from runs at about a quarter of that.  So products of
// two residues of a prime below kFpPrime are formed exactly in float64
// (below).  For the larger primes (the 60-bit first and special primes),
// sums of products from 30-bit halves need no carry chain (SplitSums); they
// measured faster than 128-bit multiply-accumulates in the BSGS inner sums
// and no slower in the hoisted key products, and slower in the bulk key
// products and the basis conversions, which keep the 128-bit form.
#pragma once
#include <cstdint>

#include "modarith.cuh"

namespace ckks {

// Products of residues below kFpPrime are formed exactly in float64:
// with d, b < q < 2^50.6 both exact doubles,
//   hi = d*b (rounded), lo = fma(d, b, -hi)      d*b = hi + lo exactly, |lo| < 2^49
//   k  = rint(hi / q) via fma(hi, 1/q, 1.5*2^52)  |k - d*b/q| < 1.05
//   r  = fma(-k, q, hi) + lo                       exact, r = d*b mod q, |r| < 1.05 q
// and sums of four such r (|sum| < 4.75 q < 2^53) are exact; each four
// products the running sum is brought back to |acc| < 0.51 q the same way.
constexpr uint64_t kFpPrime = (1ull << 50) + (1ull << 49);
constexpr double kRoundMagic = 6755399441055744.0;  // 1.5 * 2^52

__device__ __forceinline__ double fp_mod_product(double d, double b, double q, double qinv) {
  const double hi = __dmul_rn(d, b);
  const double lo = __fma_rn(d, b, -hi);
  const double k = __dsub_rn(__fma_rn(hi, qinv, kRoundMagic), kRoundMagic);
  return __dadd_rn(__fma_rn(-k, q, hi), lo);
}

__device__ __forceinline__ double fp_center(double acc, double q, double qinv) {
  const double k = __dsub_rn(__fma_rn(acc, qinv, kRoundMagic), kRoundMagic);
  return __fma_rn(-k, q, acc);
}

// |acc| < 0.51 q -> canonical residue
__device__ __forceinline__ uint64_t fp_canonical(double acc, double q) {
  return __double2ull_rn(acc < 0.0 ? __dadd_rn(acc, q) : acc);
}

// residue (< 2^52) -> the same integer as a double
__device__ __forceinline__ double u2d(uint64_t v) {
  return __dsub_rn(__longlong_as_double((long long)(v | 0x4330000000000000ull)), 4503599627370496.0);
}

// Split products for primes below 2^60: with d = dh 2^30 + dl and
// b = bh 2^30 + bl (halves below 2^30), sum_j d_j b_j is kept as four 64-bit
// sums of partial products, dl bl, dl bh, dh bl and dh bh: up to 16 products
// stay below 2^64 (no carries), and the sums are recombined into a 128-bit
// value and Barrett-reduced once (below 64 q^2).
constexpr int kSplitBits = 30;

// sums of products of residues split into halves below 2^kSplitBits
struct SplitSums {
  uint64_t lo = 0, mid = 0, mid2 = 0, hi = 0;
  __device__ __forceinline__ void mac(uint32_t dl, uint32_t dh, uint32_t bl, uint32_t bh) {
    lo += (uint64_t)dl * bl;
    mid += (uint64_t)dl * bh;
    mid2 += (uint64_t)dh * bl;
    hi += (uint64_t)dh * bh;
  }
  __device__ __forceinline__ uint64_t reduce(const ckks::Mod& m) const {
    constexpr int SB = kSplitBits;
    ckks::U128 x{lo, 0};
    ckks::add_wide(x, ckks::U128{mid << SB, mid >> (64 - SB)});
    ckks::add_wide(x, ckks::U128{mid2 << SB, mid2 >> (64 - SB)});
    ckks::add_wide(x, ckks::U128{hi << (2 * SB), hi >> (64 - 2 * SB)});
    return ckks::reduce128(x, m);
  }
};

__device__ __forceinline__ void split_residue(uint64_t v, uint32_t& l, uint32_t& h) {
  l = (uint32_t)v & ((1u << kSplitBits) - 1u);
  h = (uint32_t)(v >> kSplitBits);
}

}  // namespace ckks
