// modarith.cuh -- 64-bit-word modular arithmetic for the integer pipes.
//
// Every residue lives in a 64-bit word below its prime q < 2^61.  Products
// are formed as 128-bit (hi, lo) pairs with mul.lo/mul.hi, and reduced with:
//   * Shoup multiplication by a constant w (precomputed w' = floor(w 2^64/q)):
//     three 64-bit multiplies, result in [0, 2q) before the final correction;
//   * a 128-bit Barrett reduction with floor(2^128/q) held as two words, for
//     products of two variable residues and for accumulated sums of up to
//     2^6 such products (the estimate is floor(x/q) or one less).
// Both give the canonical residue, so the results are identical to the CPU
// restatement's for the same inputs.
#pragma once
#include <cstdint>

namespace ckks {

struct Mod {
  uint64_t q;   // prime
  uint64_t r1;  // floor(2^128 / q), high word
  uint64_t r0;  // floor(2^128 / q), low word
};

struct U128 {
  uint64_t lo, hi;
};

__device__ __forceinline__ U128 mul_wide(uint64_t a, uint64_t b) {
  U128 r;
  r.lo = a * b;
  r.hi = __umul64hi(a, b);
  return r;
}

__device__ __forceinline__ void add_wide(U128& acc, U128 x) {
  asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(acc.lo), "+l"(acc.hi) : "l"(x.lo), "l"(x.hi));
}

// acc += a*b (128-bit) as one carry chain: mad.lo.cc + madc.hi
__device__ __forceinline__ void mac_wide(U128& acc, uint64_t a, uint64_t b) {
  asm("mad.lo.cc.u64 %0, %2, %3, %0;\n\tmadc.hi.u64 %1, %2, %3, %1;"
      : "+l"(acc.lo), "+l"(acc.hi)
      : "l"(a), "l"(b));
}

__device__ __forceinline__ uint64_t reduce128(U128 x, const Mod& m) {
  const uint64_t carry = __umul64hi(x.lo, m.r0);
  // a = x.lo * r1 + carry ; b = x.hi * r0 + lo(a) ; qe = x.hi * r1 + hi(a) + hi(b)
  uint64_t a_lo, a_hi, b_lo, b_hi;
  asm("mad.lo.cc.u64 %0, %2, %3, %4;\n\tmadc.hi.u64 %1, %2, %3, 0;"
      : "=l"(a_lo), "=l"(a_hi)
      : "l"(x.lo), "l"(m.r1), "l"(carry));
  asm("mad.lo.cc.u64 %0, %2, %3, %4;\n\tmadc.hi.u64 %1, %2, %3, 0;"
      : "=l"(b_lo), "=l"(b_hi)
      : "l"(x.hi), "l"(m.r0), "l"(a_lo));
  (void)b_lo;
  const uint64_t qe = x.hi * m.r1 + a_hi + b_hi;
  uint64_t r = x.lo - qe * m.q;
  return r >= m.q ? r - m.q : r;
}

__device__ __forceinline__ uint64_t mul_mod(uint64_t a, uint64_t b, const Mod& m) {
  return reduce128(mul_wide(a, b), m);
}

__device__ __forceinline__ uint64_t add_mod(uint64_t a, uint64_t b, uint64_t q) {
  uint64_t s = a + b;
  return s >= q ? s - q : s;
}

__device__ __forceinline__ uint64_t sub_mod(uint64_t a, uint64_t b, uint64_t q) {
  return a >= b ? a - b : a + q - b;
}

__device__ __forceinline__ uint64_t neg_mod(uint64_t a, uint64_t q) { return a ? q - a : 0; }

// a * w mod q with w' = floor(w 2^64 / q); exact for any a < 2^64
__device__ __forceinline__ uint64_t mul_shoup(uint64_t a, uint64_t w, uint64_t wp, uint64_t q) {
  const uint64_t h = __umul64hi(a, wp);
  const uint64_t r = a * w - h * q;
  return r >= q ? r - q : r;
}

// lazy variant: result in [0, 2q)
__device__ __forceinline__ uint64_t mul_shoup_lazy(uint64_t a, uint64_t w, uint64_t wp, uint64_t q) {
  const uint64_t h = __umul64hi(a, wp);
  return a * w - h * q;
}

__device__ __forceinline__ uint32_t bit_reverse(uint32_t x, int bits) { return __brev(x) >> (32 - bits); }

// NTT-domain automorphism X -> X^g for the bit-reversed evaluation order:
// output slot k holds input slot br(((2 br(k) + 1) g mod 2N - 1) / 2).
// An aligned group of 2^b consecutive k maps onto an aligned group of 2^b
// consecutive source slots, so warp gathers stay within one 256-byte span.
__device__ __forceinline__ uint32_t auto_index(uint32_t k, uint32_t g, int logN) {
  const uint32_t M = 2u << logN;
  const uint32_t e = 2u * bit_reverse(k, logN) + 1u;
  const uint32_t eg = (uint32_t)(((uint64_t)e * g) & (uint64_t)(M - 1));
  return bit_reverse((eg - 1u) >> 1, logN);
}

}  // namespace ckks
