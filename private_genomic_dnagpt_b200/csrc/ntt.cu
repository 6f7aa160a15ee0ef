// ntt.cu -- batched negacyclic NTT / inverse NTT over RNS limbs (sm_100a).
//
// A limb of N = 2^logN residues is transformed in two passes that split the
// logN butterfly stages as s1 = logN/2 (strided "row" stages) and
// s2 = logN - s1 (contiguous stages):
//   forward:  pass A over 2^s1-point sub-transforms at stride 2^s2 (global
//             stages 0..s1-1), then pass B over contiguous 2^s2-point blocks
//             (stages s1..logN-1);
//   inverse:  pass B' (stages logN-1..s1) then pass A' (stages s1-1..0), with
//             N^-1 folded into the last stage's twiddles.
// Inside a pass each thread keeps 8 or 16 residues in registers and applies
// up to three or four radix-2 stages to them before exchanging through shared
// memory: a 256-point sub-transform costs two exchanges in the contiguous
// pass (8 residues, 1024 resident threads per SM) and one in the strided pass
// (16 residues, 768 resident threads, whose column loads gain most from more
// loads in flight per thread).
// Twiddles are psi^bitrev in the Longa-Naehrig order, stored with their
// Shoup companions as (w, w') pairs; output order is bit-reversed (forward)
// and natural (inverse), identical to the CPU restatement.
#include <cstdio>

#include "ckks_internal.hpp"

namespace ckks {

namespace {

// threads per CTA and resident CTAs per SM, by residues per thread (2^R_LOG)
template <int R_LOG>
struct PassShape {
  static constexpr int kThreads = R_LOG >= 4 ? 256 : 512;
  static constexpr int kMinBlocks = R_LOG >= 4 ? 3 : 2;
};

struct PassArgs {
  const ulonglong2* tw;  // [P][N] (w, w'), forward or inverse table
  const double2* twd;    // [P][N] (w, fl(w / q)) as doubles, the same twiddles
  const Mod* mods;
  const ulonglong2* ninv_last;  // [P] (n^-1, shoup) ; inverse only
  const ulonglong2* w1_ninv;    // [P] (Winv[1] * n^-1, shoup) ; inverse only
  // optional per-batch-limb replacements of (n^-1, Winv[1] n^-1): the inverse
  // transform then returns x * c_l for a constant c_l folded into its last stage
  const ulonglong2* scale_a;
  const ulonglong2* scale_b;
  int scale_base;
  LimbMap map;
  int logN;
  int per_cta;  // columns (strided) or blocks (contiguous) per CTA
  bool has_src;  // the first pass reads `src` instead of the data array
  NttSource src;
};

// the array the first pass of limb `limb` reads
__device__ __forceinline__ const uint64_t* pass_input(const PassArgs& a, uint64_t* poly, int limb, bool first_pass) {
  if (!a.has_src || !first_pass) return poly;
  return a.src.item[limb / a.src.per_item] + (size_t)(limb % a.src.per_item) * a.src.limb_stride;
}

// Shared-memory slot of residue r in a contiguous block: the low four bits
// are XORed with a function of the next bits, so that each half-warp's
// 64-bit accesses of every register-group layout of a 256-point block fall in
// 16 distinct bank pairs (a bijection on every aligned 16 residues).  With 8
// residues per thread the function of bits 4-6 covers the three layouts;
// with 16 residues per thread the two layouts (r = u + 16 k and r = 16 u + k
// for thread u) are covered by XORing bits 4-7 themselves.
template <int R_LOG>
__device__ __forceinline__ int swizzle(int r) {
  const int h = r >> 4;
  if (R_LOG >= 4) return h & 15;
  return (h & 1) ^ (((h >> 1) & 1) * 6) ^ (((h >> 2) & 1) * 8);
}

template <int R_LOG>
__device__ __forceinline__ int group_size(int s_log, int gi) {
  const int rem = s_log - R_LOG * gi;
  return rem < R_LOG ? rem : R_LOG;
}

// Harvey butterflies.  Forward (Cooley-Tukey): values in [0, 4q);
// inverse (Gentleman-Sande): values in [0, 2q).  The last pass returns
// canonical residues in [0, q).
__device__ __forceinline__ void ct_bfly(uint64_t& x, uint64_t& y, ulonglong2 w, uint64_t q, uint64_t q2) {
  uint64_t a = x >= q2 ? x - q2 : x;
  const uint64_t t = mul_shoup_lazy(y, w.x, w.y, q);
  x = a + t;
  y = a + q2 - t;
}

__device__ __forceinline__ void gs_bfly(uint64_t& x, uint64_t& y, ulonglong2 w, uint64_t q, uint64_t q2) {
  uint64_t s = x + y;
  s = s >= q2 ? s - q2 : s;
  const uint64_t d = x + q2 - y;
  x = s;
  y = mul_shoup_lazy(d, w.x, w.y, q);
}

// Position of residue r of sub-transform `sub` inside a limb: strided
// sub-transforms are columns (r at stride N / S), contiguous ones blocks.
template <int S_LOG, bool STRIDED>
__device__ __forceinline__ size_t pass_gaddr(int logN, int sub, int r) {
  return STRIDED ? ((size_t)r << (logN - S_LOG)) + sub : ((size_t)sub << S_LOG) + r;
}
// Shared-memory slot of residue r of local sub-transform `lane` (the layout
// of the exchanges inside a pass and of the contiguous pass's staged side)
template <int S_LOG, bool STRIDED, int R_LOG>
__device__ __forceinline__ int pass_saddr(int per, int lane, int r) {
  return STRIDED ? r * per + lane : (lane << S_LOG) + (r ^ swizzle<R_LOG>(r));
}

// One pass: S-point sub-transforms of one limb, `per` of them per CTA
// starting at sub-transform sub_base.  load0(sub, lane, r) returns residue r
// of sub-transform sub (local index lane) as the pass starts;
// store_last(sub, lane, r, v) takes it as the pass ends, after every thread
// has called pre_store() once.
template <int S_LOG, bool INV, bool STRIDED, int R_LOG, class Load0, class StoreLast, class PreStore>
__device__ __forceinline__ void ntt_pass_body(const PassArgs& a, uint64_t* sm, int limb, int sub_base, Load0 load0,
                                              StoreLast store_last, PreStore pre_store) {
  constexpr int S = 1 << S_LOG;
  constexpr int R = 1 << R_LOG;                // residues per thread
  constexpr int T = S >= R ? S / R : 1;        // threads per sub-transform
  constexpr int NG = (S_LOG + R_LOG - 1) / R_LOG;  // register stage groups

  const int prime = a.map.prime(limb);
  const int N = 1 << a.logN;
  const uint64_t q = a.mods[prime].q;
  const uint64_t q2 = 2 * q;
  const ulonglong2* tw = a.tw + (size_t)prime * N;

  const int tid = threadIdx.x;
  const int per = a.per_cta;
  int sub_t, lane_idx;  // thread within sub-transform, sub-transform within CTA
  if (STRIDED) {
    lane_idx = tid % per;
    sub_t = tid / per;
  } else {
    lane_idx = tid / T;
    sub_t = tid % T;
  }
  const int sub_global = sub_base + lane_idx;  // column or block index
  const int gs0 = STRIDED ? 0 : (a.logN - S_LOG);
  const uint32_t prefix = STRIDED ? 0u : (uint32_t)sub_global;
  // the strided pass holds the first stages (forward) / the last stages
  // (inverse); the contiguous pass the others
  const bool first_pass = (STRIDED != INV);
  const bool last_pass = !first_pass;
  (void)N;

  auto saddr = [&](int r) -> int { return pass_saddr<S_LOG, STRIDED, R_LOG>(per, lane_idx, r); };

  uint64_t x[R];

#pragma unroll
  for (int step = 0; step < NG; ++step) {
    const int gi = INV ? (NG - 1 - step) : step;
    const int G = group_size<R_LOG>(S_LOG, gi);
    const int st0 = R_LOG * gi;
    const int D = S >> (st0 + G);  // smallest distance inside a unit
    const int units_per_thread = R >> G;
    const int usz = 1 << G;
    // load
#pragma unroll
    for (int j = 0; j < R; ++j) {
      if (j >= units_per_thread * usz) break;
      const int uj = j / usz, k = j % usz;
      const int u = sub_t + uj * T;
      const int r = (u / D) * (D << G) + (u % D) + k * D;
      x[j] = step > 0 ? sm[saddr(r)] : load0(sub_global, lane_idx, r);
    }
    // butterflies; the twiddle of pair (k, k+h) at stage st0+rr is
    // tw[2^(gs0+st) + prefix*2^st + B*2^rr + (k >> (G-rr))], B = u / D
#pragma unroll
    for (int uj = 0; uj < R; ++uj) {
      if (uj >= units_per_thread) break;
      const int u = sub_t + uj * T;
      const uint32_t B = (uint32_t)(u / D);
      uint64_t* xu = x + uj * usz;
#pragma unroll
      for (int it = 0; it < R_LOG; ++it) {
        if (it >= G) break;
        const int rr = INV ? (G - 1 - it) : it;
        const int st = st0 + rr;
        const int h = 1 << (G - 1 - rr);
        const bool final_stage = INV && STRIDED && st == 0;
        const uint32_t idx0 = (1u << (gs0 + st)) + (prefix << st) + (B << rr);
        // pairs (k, k + h) with k >> (G - rr) == jw share twiddle jw
#pragma unroll
        for (int jw = 0; jw < R / 2; ++jw) {
          if (jw >= (1 << rr)) break;
          ulonglong2 w{0, 0};
          if (!final_stage) w = __ldg(tw + idx0 + jw);
#pragma unroll
          for (int kk = 0; kk < R; ++kk) {
            if (kk >= (1 << (G - rr))) break;
            const int k = (jw << (G - rr)) + kk;
            if (k & h) continue;
            if (!INV) {
              ct_bfly(xu[k], xu[k + h], w, q, q2);
            } else if (!final_stage) {
              gs_bfly(xu[k], xu[k + h], w, q, q2);
            } else {
              const ulonglong2 c0 = a.scale_a ? __ldg(a.scale_a + (prime - a.scale_base)) : __ldg(a.ninv_last + prime);
              const ulonglong2 c1 = a.scale_b ? __ldg(a.scale_b + (prime - a.scale_base)) : __ldg(a.w1_ninv + prime);
              const uint64_t u0 = xu[k], v0 = xu[k + h];
              const uint64_t s0 = mul_shoup_lazy(u0 + v0, c0.x, c0.y, q);
              const uint64_t d0 = mul_shoup_lazy(u0 + q2 - v0, c1.x, c1.y, q);
              xu[k] = s0 >= q ? s0 - q : s0;
              xu[k + h] = d0 >= q ? d0 - q : d0;
            }
          }
        }
      }
    }
    // store
    if (step + 1 < NG) {
      if (step > 0) __syncthreads();  // everyone has read the previous layout
#pragma unroll
      for (int j = 0; j < R; ++j) {
        if (j >= units_per_thread * usz) break;
        const int uj = j / usz, k = j % usz;
        const int u = sub_t + uj * T;
        sm[saddr((u / D) * (D << G) + (u % D) + k * D)] = x[j];
      }
      __syncthreads();
    } else {
      pre_store();
#pragma unroll
      for (int j = 0; j < R; ++j) {
        if (j >= units_per_thread * usz) break;
        const int uj = j / usz, k = j % usz;
        const int u = sub_t + uj * T;
        uint64_t v = x[j];
        if (last_pass && !INV) {  // forward output: [0, 4q) -> [0, q)
          v = v >= q2 ? v - q2 : v;
          v = v >= q ? v - q : v;
        }
        // inverse output of the final stage is already canonical
        store_last(sub_global, lane_idx, (u / D) * (D << G) + (u % D) + k * D, v);
      }
    }
  }
}

// Float64 butterflies for primes below kFpNttPrime.  Residues are signed
// doubles; the twiddle product of y by (w, wq = fl(w/q)) is exact:
//   k = rint(y wq) (the 1.5 * 2^52 rounding, valid while |y wq| < 2^51),
//   r = fma(-k, q, y*w) + fma(y, w, -y*w)  = y w - k q,  |r| < 0.52 q,
// with |y| < 1.6 q; the bounds per stage within a register group of up to
// four stages, from inputs centred to |x| <= 0.51 q:
//   forward  x' = x + r, y' = x - r: the multiplied input of stages 1-3 is
//            below 0.51, 1.03, 1.55 q, and the fourth stage re-centres it
//            first; all values stay below 2.6 q;
//   inverse  x' = x + y, y' = (x - y) w: the difference is re-centred before
//            the product from the group's second stage on; the sums stay
//            below 4.1 q through three stages, and the fourth stage
//            re-centres both of its inputs first.
// All of these are below 2^53 for q < 1.25 * 2^50, so every sum is exact.
// Every group ends by re-centring all values (k = rint(x / q), x - k q), so
// each pass hands on |x| <= 0.51 q; the transform's output is the canonical
// residue, as on the integer path.
constexpr uint64_t kFpNttPrime = (1ull << 50) + (1ull << 48);
constexpr double kFpMagic = 6755399441055744.0;  // 1.5 * 2^52

__device__ __forceinline__ double fp_center(double x, double q, double qinv) {
  const double k = __dsub_rn(__fma_rn(x, qinv, kFpMagic), kFpMagic);
  return __fma_rn(-k, q, x);
}

__device__ __forceinline__ double fp_mulw(double y, double2 w, double q) {
  const double k = __dsub_rn(__fma_rn(y, w.y, kFpMagic), kFpMagic);
  const double hi = __dmul_rn(y, w.x);
  const double lo = __fma_rn(y, w.x, -hi);
  return __dadd_rn(__fma_rn(-k, q, hi), lo);
}

// |x| <= 0.51 q -> canonical residue
__device__ __forceinline__ uint64_t fp_to_residue(double x, double q) {
  return __double2ull_rn(x < 0.0 ? __dadd_rn(x, q) : x);
}

template <int S_LOG, bool INV, bool STRIDED, int R_LOG, class Load0, class StoreLast, class PreStore>
__device__ __forceinline__ void ntt_pass_body_fp(const PassArgs& a, uint64_t* sm, int limb, int sub_base,
                                                 Load0 load0, StoreLast store_last, PreStore pre_store) {
  constexpr int S = 1 << S_LOG;
  constexpr int R = 1 << R_LOG;
  constexpr int T = S >= R ? S / R : 1;
  constexpr int NG = (S_LOG + R_LOG - 1) / R_LOG;

  const int prime = a.map.prime(limb);
  const int N = 1 << a.logN;
  const uint64_t qi = a.mods[prime].q;
  const double q = (double)qi, qinv = 1.0 / q;
  const double2* tw = a.twd + (size_t)prime * N;

  const int tid = threadIdx.x;
  const int per = a.per_cta;
  int sub_t, lane_idx;
  if (STRIDED) {
    lane_idx = tid % per;
    sub_t = tid / per;
  } else {
    lane_idx = tid / T;
    sub_t = tid % T;
  }
  const int sub_global = sub_base + lane_idx;
  const int gs0 = STRIDED ? 0 : (a.logN - S_LOG);
  const uint32_t prefix = STRIDED ? 0u : (uint32_t)sub_global;
  const bool first_pass = (STRIDED != INV);

  auto saddr = [&](int r) -> int { return pass_saddr<S_LOG, STRIDED, R_LOG>(per, lane_idx, r); };

  double x[R];

#pragma unroll
  for (int step = 0; step < NG; ++step) {
    const int gi = INV ? (NG - 1 - step) : step;
    const int G = group_size<R_LOG>(S_LOG, gi);
    const int st0 = R_LOG * gi;
    const int D = S >> (st0 + G);
    const int units_per_thread = R >> G;
    const int usz = 1 << G;
    // load: the transform's input as residues, the first pass's output and
    // the exchanges as centred doubles
#pragma unroll
    for (int j = 0; j < R; ++j) {
      if (j >= units_per_thread * usz) break;
      const int uj = j / usz, k = j % usz;
      const int u = sub_t + uj * T;
      const int r = (u / D) * (D << G) + (u % D) + k * D;
      if (step > 0) {
        x[j] = __longlong_as_double((long long)sm[saddr(r)]);
      } else if (first_pass) {
        x[j] = fp_center(__ull2double_rn(load0(sub_global, lane_idx, r)), q, qinv);
      } else {
        x[j] = __longlong_as_double((long long)load0(sub_global, lane_idx, r));
      }
    }
    bool final_done = false;
#pragma unroll
    for (int uj = 0; uj < R; ++uj) {
      if (uj >= units_per_thread) break;
      const int u = sub_t + uj * T;
      const uint32_t B = (uint32_t)(u / D);
      double* xu = x + uj * usz;
#pragma unroll
      for (int it = 0; it < R_LOG; ++it) {
        if (it >= G) break;
        const int rr = INV ? (G - 1 - it) : it;
        const int st = st0 + rr;
        const int h = 1 << (G - 1 - rr);
        const bool final_stage = INV && STRIDED && st == 0;
        const uint32_t idx0 = (1u << (gs0 + st)) + (prefix << st) + (B << rr);
        // pairs (k, k + h) with k >> (G - rr) == jw share twiddle jw
#pragma unroll
        for (int jw = 0; jw < R / 2; ++jw) {
          if (jw >= (1 << rr)) break;
          double2 w{0.0, 0.0};
          if (!final_stage) w = __ldg(tw + idx0 + jw);
#pragma unroll
          for (int kk = 0; kk < R; ++kk) {
          if (kk >= (1 << (G - rr))) break;
          const int k = (jw << (G - rr)) + kk;
          if (k & h) continue;
          if (!INV) {
            const double y0 = it >= 3 ? fp_center(xu[k + h], q, qinv) : xu[k + h];
            const double t = fp_mulw(y0, w, q);
            const double x0 = xu[k];
            xu[k] = __dadd_rn(x0, t);
            xu[k + h] = __dsub_rn(x0, t);
          } else if (!final_stage) {
            double x0 = xu[k], y0 = xu[k + h], d;
            if (it >= 3) {
              x0 = fp_center(x0, q, qinv);
              y0 = fp_center(y0, q, qinv);
              d = __dsub_rn(x0, y0);
            } else {
              d = __dsub_rn(x0, y0);
              if (it > 0) d = fp_center(d, q, qinv);
            }
            xu[k] = __dadd_rn(x0, y0);
            xu[k + h] = fp_mulw(d, w, q);
          } else {
            // last inverse stage on canonical residues with the integer
            // Shoup constants (n^-1 or the caller's scale folded in)
            const ulonglong2 c0 = a.scale_a ? __ldg(a.scale_a + (prime - a.scale_base)) : __ldg(a.ninv_last + prime);
            const ulonglong2 c1 = a.scale_b ? __ldg(a.scale_b + (prime - a.scale_base)) : __ldg(a.w1_ninv + prime);
            const uint64_t u0 = fp_to_residue(fp_center(xu[k], q, qinv), q);
            const uint64_t v0 = fp_to_residue(fp_center(xu[k + h], q, qinv), q);
            const uint64_t s0 = mul_shoup_lazy(u0 + v0, c0.x, c0.y, qi);
            const uint64_t d0 = mul_shoup_lazy(u0 + 2 * qi - v0, c1.x, c1.y, qi);
            xu[k] = __longlong_as_double((long long)(s0 >= qi ? s0 - qi : s0));
            xu[k + h] = __longlong_as_double((long long)(d0 >= qi ? d0 - qi : d0));
            final_done = true;
          }
          }
        }
      }
    }
    // store
    if (step + 1 < NG) {
      if (step > 0) __syncthreads();
#pragma unroll
      for (int j = 0; j < R; ++j) {
        if (j >= units_per_thread * usz) break;
        const int uj = j / usz, k = j % usz;
        const int u = sub_t + uj * T;
        sm[saddr((u / D) * (D << G) + (u % D) + k * D)] = (uint64_t)__double_as_longlong(fp_center(x[j], q, qinv));
      }
      __syncthreads();
    } else {
      pre_store();
#pragma unroll
      for (int j = 0; j < R; ++j) {
        if (j >= units_per_thread * usz) break;
        const int uj = j / usz, k = j % usz;
        const int u = sub_t + uj * T;
        uint64_t v;
        if (final_done) {  // inverse: canonical residues already
          v = (uint64_t)__double_as_longlong(x[j]);
        } else {
          const double c = fp_center(x[j], q, qinv);
          v = first_pass ? (uint64_t)__double_as_longlong(c) : fp_to_residue(c, q);
        }
        store_last(sub_global, lane_idx, (u / D) * (D << G) + (u % D) + k * D, v);
      }
    }
  }
}

// One CTA of a pass.  The forward contiguous pass hands its output pairs
// (coefficients n, n + 1 of batch limb `limb`, n even) to staged_store.
template <int S_LOG, bool INV, bool STRIDED, int R_LOG, class StagedStore>
__device__ __forceinline__ void ntt_pass_run(uint64_t* __restrict__ data, const PassArgs& a, uint64_t* sm,
                                             StagedStore staged_store) {
  const int limb = blockIdx.y;
  if (a.map.skipped(limb)) return;
  const int prime = a.map.prime(limb);
  const Mod m = a.mods[prime];
  const int logN = a.logN;
  uint64_t* poly = data + ((size_t)limb << logN);
  const bool first_pass = (STRIDED != INV);
  const uint64_t* in = pass_input(a, poly, limb, first_pass);
  const bool reduce = first_pass && a.has_src && a.src.reduce;
  const int per = a.per_cta;
  const int sub_base = blockIdx.x * per;
  // A contiguous pass's CTA owns per * S consecutive words.  The forward's
  // output would leave a thread's registers at a 4-residue stride: it is
  // re-laid in shared memory and written in coalesced 16-byte stores.  (The
  // inverse's input, read at the same stride, gained nothing from staging:
  // the sectors of one load serve the next three from L1.)
  constexpr bool kStageOut = !STRIDED && !INV;
  const int W = per << S_LOG;
  const int nt = (int)blockDim.x;
  auto load0 = [&](int sub, int, int r) -> uint64_t {
    const uint64_t v = in[pass_gaddr<S_LOG, STRIDED>(logN, sub, r)];
    return reduce ? reduce128(U128{v, 0}, m) : v;
  };
  auto store_last = [&](int sub, int lane, int r, uint64_t v) {
    if (kStageOut)
      sm[pass_saddr<S_LOG, false, R_LOG>(per, lane, r)] = v;
    else
      poly[pass_gaddr<S_LOG, STRIDED>(logN, sub, r)] = v;
  };
  // the last step read shared memory: wait before overwriting it
  auto pre_store = [] {
    if (kStageOut) __syncthreads();
  };
  if (m.q < kFpNttPrime)
    ntt_pass_body_fp<S_LOG, INV, STRIDED, R_LOG>(a, sm, limb, sub_base, load0, store_last, pre_store);
  else
    ntt_pass_body<S_LOG, INV, STRIDED, R_LOG>(a, sm, limb, sub_base, load0, store_last, pre_store);
  if (kStageOut) {
    __syncthreads();
    const size_t n0 = (size_t)sub_base << S_LOG;
    for (int i = 2 * (int)threadIdx.x; i < W; i += 2 * nt) {
      const uint64_t x0 = sm[pass_saddr<S_LOG, false, R_LOG>(per, i >> S_LOG, i & ((1 << S_LOG) - 1))];
      const uint64_t x1 = sm[pass_saddr<S_LOG, false, R_LOG>(per, (i + 1) >> S_LOG, (i + 1) & ((1 << S_LOG) - 1))];
      staged_store(limb, poly, m, n0 + i, x0, x1);
    }
  }
}

template <int S_LOG, bool INV, bool STRIDED, int R_LOG>
__global__ void __launch_bounds__(PassShape<R_LOG>::kThreads, PassShape<R_LOG>::kMinBlocks)
    ntt_pass_kernel(uint64_t* __restrict__ data, PassArgs a) {
  extern __shared__ uint64_t sm[];
  CKKS_PDL_ENTRY();  // launched as a programmatic dependent (launch_pdl)
  ntt_pass_run<S_LOG, INV, STRIDED, R_LOG>(
      data, a, sm, [](int, uint64_t* poly, const Mod&, size_t n, uint64_t x0, uint64_t x1) {
        *reinterpret_cast<ulonglong2*>(poly + n) = make_ulonglong2(x0, x1);
      });
}

// The forward contiguous pass of ModDown's conversion with the combine step
// as its store: batch limb (2 m + p) limbs + t holds conv (item m, part p,
// limb t), and the pass writes (acc - conv) P^-1, plus the automorphism-
// permuted c0 addend (part 0) or the c1 addend (part 1), straight to the
// item's output instead of storing conv.
template <int S_LOG, int R_LOG>
__global__ void __launch_bounds__(PassShape<R_LOG>::kThreads, PassShape<R_LOG>::kMinBlocks)
    ntt_moddown_pass_kernel(uint64_t* __restrict__ data, PassArgs a, ModDownCombine mc) {
  extern __shared__ uint64_t sm[];
  CKKS_PDL_ENTRY();
  const int logN = a.logN;
  ntt_pass_run<S_LOG, false, false, R_LOG>(
      data, a, sm, [&](int limb, uint64_t*, const Mod& md, size_t n, uint64_t x0, uint64_t x1) {
        const int t = limb % mc.limbs, pm = limb / mc.limbs, p = pm & 1, m = pm >> 1;
        const size_t N = (size_t)1 << logN;
        const uint64_t q = md.q;
        const ulonglong2 pv = mc.pinv[t];
        const ulonglong2 av = *reinterpret_cast<const ulonglong2*>(mc.acc + ((size_t)(2 * m + p) * mc.E + t) * N + n);
        uint64_t r0 = mul_shoup(sub_mod(av.x, x0, q), pv.x, pv.y, q);
        uint64_t r1 = mul_shoup(sub_mod(av.y, x1, q), pv.x, pv.y, q);
        uint64_t* out;
        if (p == 0) {
          const uint64_t* add0 = mc.add0[m];
          if (add0) {
            const uint32_t g = mc.g[m];
            // the automorphism maps the aligned pair onto an aligned pair
            const uint32_t s = g == 1u ? (uint32_t)n : auto_index((uint32_t)n, g, logN);
            r0 = add_mod(r0, add0[(size_t)t * N + s], q);
            r1 = add_mod(r1, add0[(size_t)t * N + (s ^ 1u)], q);
          }
          out = mc.out0[m];
        } else {
          const uint64_t* add1 = mc.add1[m];
          if (add1) {
            const ulonglong2 bv = *reinterpret_cast<const ulonglong2*>(add1 + (size_t)t * N + n);
            r0 = add_mod(r0, bv.x, q);
            r1 = add_mod(r1, bv.y, q);
          }
          out = mc.out1[m];
        }
        *reinterpret_cast<ulonglong2*>(out + (size_t)t * N + n) = make_ulonglong2(r0, r1);
      });
}

template <int S_LOG, bool INV, bool STRIDED>
void launch_pass(uint64_t* data, int nlimbs, const PassArgs& a0, int sms, cudaStream_t st) {
  // strided passes: 16 residues per thread (four stages per register group,
  // twice the loads in flight per thread); contiguous passes, whose
  // shared-memory exchanges favour more resident warps: 8
  constexpr int R_LOG = (STRIDED && S_LOG >= 4) ? 4 : 3;
  constexpr int S = 1 << S_LOG;
  constexpr int T = S >= (1 << R_LOG) ? S / (1 << R_LOG) : 1;
  const int N = 1 << a0.logN;
  const int subs = N / S;  // sub-transforms per limb
  int per = PassShape<R_LOG>::kThreads / T;
  if (per > subs) per = subs;
  // small batches: smaller CTAs (fewer sub-transforms each, at least one
  // warp) until the grid holds four CTAs per SM, so the work spreads over
  // every SM instead of a partly filled second wave on a few of them
  while (per > 1 && per * T > 32 && (subs / per) * nlimbs < 4 * sms) per >>= 1;
  PassArgs a = a0;
  a.per_cta = per;
  const dim3 grid(subs / per, nlimbs);
  const int threads = per * T;
  const size_t smem = (size_t)S * per * sizeof(uint64_t);
  auto k = ntt_pass_kernel<S_LOG, INV, STRIDED, R_LOG>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // a programmatic dependent: its launch can overlap the previous kernel's
  // last wave (the kernel waits for that grid on the device)
  launch_pdl(k, grid, dim3(threads), smem, st, data, a);
}

template <int S_LOG>
void launch_moddown_pass(uint64_t* data, int nlimbs, const PassArgs& a0, const ModDownCombine& mc, int sms,
                         cudaStream_t st) {
  constexpr int R_LOG = 3;
  constexpr int S = 1 << S_LOG;
  constexpr int T = S >= (1 << R_LOG) ? S / (1 << R_LOG) : 1;
  const int subs = (1 << a0.logN) / S;
  int per = PassShape<R_LOG>::kThreads / T;
  if (per > subs) per = subs;
  while (per > 1 && per * T > 32 && (subs / per) * nlimbs < 4 * sms) per >>= 1;
  PassArgs a = a0;
  a.per_cta = per;
  const size_t smem = (size_t)S * per * sizeof(uint64_t);
  auto k = ntt_moddown_pass_kernel<S_LOG, R_LOG>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl(k, dim3(subs / per, nlimbs), dim3(per * T), smem, st, data, a, mc);
}

template <bool INV, bool STRIDED>
void dispatch_pass(int s_log, uint64_t* data, int nlimbs, const PassArgs& a, int sms, cudaStream_t st) {
  switch (s_log) {
    case 3: launch_pass<3, INV, STRIDED>(data, nlimbs, a, sms, st); break;
    case 4: launch_pass<4, INV, STRIDED>(data, nlimbs, a, sms, st); break;
    case 5: launch_pass<5, INV, STRIDED>(data, nlimbs, a, sms, st); break;
    case 6: launch_pass<6, INV, STRIDED>(data, nlimbs, a, sms, st); break;
    case 7: launch_pass<7, INV, STRIDED>(data, nlimbs, a, sms, st); break;
    case 8: launch_pass<8, INV, STRIDED>(data, nlimbs, a, sms, st); break;
    case 9: launch_pass<9, INV, STRIDED>(data, nlimbs, a, sms, st); break;
    default: break;
  }
}

}  // namespace

// limbs actually transformed (ModUp batches skip each digit's own limbs)
int live_limbs(const LimbMap& m, int nlimbs) {
  int n = 0;
  for (int l = 0; l < nlimbs; ++l) n += m.skipped(l) ? 0 : 1;
  return n;
}

void ntt_forward(const Context& c, uint64_t* data, int nlimbs, LimbMap map, cudaStream_t st, const NttSource* src) {
  if (nlimbs <= 0) return;
  // algorithmic traffic of a transform is one read + one write per limb;
  // each of the two passes is credited with half of it
  const double bytes = live_limbs(map, nlimbs) * c.limb_bytes();
  PassArgs a{};
  a.tw = c.d_tw;
  a.twd = c.d_twd;
  a.mods = c.d_mods;
  a.map = map;
  a.logN = c.logN;
  const int s1 = c.logN / 2, s2 = c.logN - s1;
  {
    ProfScope ps(c, "ntt_fwd_rows", bytes, st);
    PassArgs a1 = a;
    if (src) {
      a1.has_src = true;
      a1.src = *src;
    }
    dispatch_pass<false, true>(s1, data, nlimbs, a1, c.sms, st);
  }
  {
    ProfScope ps(c, "ntt_fwd_cols", bytes, st);
    dispatch_pass<false, false>(s2, data, nlimbs, a, c.sms, st);
  }
  CKKS_CUDA(cudaGetLastError());
}

void ntt_forward_moddown(const Context& c, uint64_t* conv, int items, const ModDownCombine& mc, cudaStream_t st) {
  const int nlimbs = items * 2 * mc.limbs;
  if (nlimbs <= 0) return;
  PassArgs a{};
  a.tw = c.d_tw;
  a.twd = c.d_twd;
  a.mods = c.d_mods;
  a.map = LimbMap::q(mc.limbs, c.L);
  a.logN = c.logN;
  const double lb = c.limb_bytes();
  const int s1 = c.logN / 2, s2 = c.logN - s1;
  {
    ProfScope ps(c, "ntt_fwd_rows", nlimbs * lb, st);
    dispatch_pass<false, true>(s1, conv, nlimbs, a, c.sms, st);
  }
  {
    // the pass's half of the transform, the accumulator read, the addends
    int adds = 0;
    for (int m = 0; m < items; ++m) adds += (mc.add0[m] ? 1 : 0) + (mc.add1[m] ? 1 : 0);
    ProfScope ps(c, "ntt_fwd_cols_moddown", (2.0 * nlimbs + (double)adds * mc.limbs) * lb, st);
    switch (s2) {
      case 3: launch_moddown_pass<3>(conv, nlimbs, a, mc, c.sms, st); break;
      case 4: launch_moddown_pass<4>(conv, nlimbs, a, mc, c.sms, st); break;
      case 5: launch_moddown_pass<5>(conv, nlimbs, a, mc, c.sms, st); break;
      case 6: launch_moddown_pass<6>(conv, nlimbs, a, mc, c.sms, st); break;
      case 7: launch_moddown_pass<7>(conv, nlimbs, a, mc, c.sms, st); break;
      case 8: launch_moddown_pass<8>(conv, nlimbs, a, mc, c.sms, st); break;
      case 9: launch_moddown_pass<9>(conv, nlimbs, a, mc, c.sms, st); break;
      default: throw Error(kErrArgument, "ring dimension outside 2^6 .. 2^17");
    }
  }
  CKKS_CUDA(cudaGetLastError());
}

void ntt_inverse(const Context& c, uint64_t* data, int nlimbs, LimbMap map, cudaStream_t st,
                 const ulonglong2* scale_a, const ulonglong2* scale_b, int scale_base, const NttSource* src) {
  if (nlimbs <= 0) return;
  const double bytes = live_limbs(map, nlimbs) * c.limb_bytes();
  PassArgs a{};
  a.tw = c.d_itw;
  a.twd = c.d_itwd;
  a.mods = c.d_mods;
  a.ninv_last = c.d_ninv;
  a.w1_ninv = c.d_w1ninv;
  a.scale_a = scale_a;
  a.scale_b = scale_b;
  a.scale_base = scale_base;
  a.map = map;
  a.logN = c.logN;
  const int s1 = c.logN / 2, s2 = c.logN - s1;
  {
    ProfScope ps(c, "ntt_inv_cols", bytes, st);
    PassArgs a1 = a;
    if (src) {
      a1.has_src = true;
      a1.src = *src;
    }
    dispatch_pass<true, false>(s2, data, nlimbs, a1, c.sms, st);
  }
  {
    ProfScope ps(c, "ntt_inv_rows", bytes, st);
    dispatch_pass<true, true>(s1, data, nlimbs, a, c.sms, st);
  }
  CKKS_CUDA(cudaGetLastError());
}

}  // namespace ckks
