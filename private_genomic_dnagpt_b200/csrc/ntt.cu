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
// Inside a pass each thread keeps 8 residues in registers and applies up to
// three radix-2 stages to them before exchanging through shared memory, so a
// 256-point sub-transform costs 2 shared-memory exchanges for 8 stages.
// Twiddles are psi^bitrev in the Longa-Naehrig order, stored with their
// Shoup companions as (w, w') pairs; output order is bit-reversed (forward)
// and natural (inverse), identical to the CPU restatement.
#include <cstdio>

#include "ckks_internal.hpp"

namespace ckks {

namespace {

// threads per CTA in both passes
constexpr int kThreads = 512;

struct PassArgs {
  const ulonglong2* tw;  // [P][N] (w, w'), forward or inverse table
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
};

__device__ __forceinline__ int group_size(int s_log, int gi) {
  const int rem = s_log - 3 * gi;
  return rem < 3 ? rem : 3;
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

// Lazy butterflies for primes below 2^kLazyBits: no correction inside a
// pass.  Forward: the Shoup product is in [0, 2q) for any 64-bit input, so
// every stage adds at most 2q to the bound (inputs < 4q: < 38q after 17
// stages).  Inverse: the sum doubles the bound each stage and the difference
// is offset by bq, a multiple of q at or above the current bound (inputs
// < 2q: < 2^10 q after 9 stages); each pass ends with one Shoup reduction by
// w = 1 (w' = floor(2^64/q), the high word of floor(2^128/q)) to [0, 2q).
// The results are the canonical residues of the exact transform, as with
// the corrected butterflies.
constexpr int kLazyBits = 52;

__device__ __forceinline__ void ct_bfly_lazy(uint64_t& x, uint64_t& y, ulonglong2 w, uint64_t q, uint64_t q2) {
  const uint64_t t = mul_shoup_lazy(y, w.x, w.y, q);
  const uint64_t a = x;
  x = a + t;
  y = a + q2 - t;
}

__device__ __forceinline__ void gs_bfly_lazy(uint64_t& x, uint64_t& y, ulonglong2 w, uint64_t q, uint64_t bq) {
  const uint64_t s = x + y;
  const uint64_t d = x + bq - y;
  x = s;
  y = mul_shoup_lazy(d, w.x, w.y, q);
}

// x mod q into [0, 2q) for any 64-bit x (Shoup product by 1)
__device__ __forceinline__ uint64_t reduce_2q(uint64_t x, uint64_t q, uint64_t w1) {
  return x - __umul64hi(x, w1) * q;
}

template <int S_LOG, bool INV, bool STRIDED, bool LAZY>
__device__ __forceinline__ void ntt_pass_body(uint64_t* __restrict__ data, const PassArgs& a, uint64_t* sm) {
  constexpr int S = 1 << S_LOG;
  constexpr int T = S >= 8 ? S / 8 : 1;  // threads per sub-transform
  constexpr int NG = (S_LOG + 2) / 3;     // register stage groups

  const int limb = blockIdx.y;
  const int prime = a.map.prime(limb);
  const int N = 1 << a.logN;
  uint64_t* poly = data + (size_t)limb * N;
  const uint64_t q = a.mods[prime].q;
  const uint64_t q2 = 2 * q;
  const uint64_t w1 = LAZY ? a.mods[prime].r1 : 0;  // floor(2^64 / q)
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
  const int sub_global = blockIdx.x * per + lane_idx;  // column or block index
  const int stride = N >> S_LOG;                         // strided: distance between rows
  const int gs0 = STRIDED ? 0 : (a.logN - S_LOG);
  const uint32_t prefix = STRIDED ? 0u : (uint32_t)sub_global;
  // the strided pass holds the first stages (forward) / the last stages
  // (inverse); the contiguous pass the others
  const bool first_pass = (STRIDED != INV);
  const bool last_pass = !first_pass;

  auto gaddr = [&](int r) -> size_t {
    return STRIDED ? (size_t)r * stride + sub_global : (size_t)sub_global * S + r;
  };
  auto saddr = [&](int r) -> int {
    return STRIDED ? r * per + lane_idx : lane_idx * (S + S / 16) + r + (r >> 4);
  };

  uint64_t x[8];
  int done = 0;  // stages of this pass already applied (inverse lazy bound)

#pragma unroll
  for (int step = 0; step < NG; ++step) {
    const int gi = INV ? (NG - 1 - step) : step;
    const int G = group_size(S_LOG, gi);
    const int st0 = 3 * gi;
    const int D = S >> (st0 + G);  // smallest distance inside a unit
    const int units_per_thread = 8 >> G;
    const int usz = 1 << G;
    // load
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= units_per_thread * usz) break;
      const int uj = j / usz, k = j % usz;
      const int u = sub_t + uj * T;
      const int r = (u / D) * (D << G) + (u % D) + k * D;
      x[j] = (step == 0) ? poly[gaddr(r)] : sm[saddr(r)];
    }
    // butterflies; the twiddle of pair (k, k+h) at stage st0+rr is
    // tw[2^(gs0+st) + prefix*2^st + B*2^rr + (k >> (G-rr))], B = u / D
#pragma unroll
    for (int uj = 0; uj < 8; ++uj) {
      if (uj >= units_per_thread) break;
      const int u = sub_t + uj * T;
      const uint32_t B = (uint32_t)(u / D);
      uint64_t* xu = x + uj * usz;
#pragma unroll
      for (int it = 0; it < 3; ++it) {
        if (it >= G) break;
        const int rr = INV ? (G - 1 - it) : it;
        const int st = st0 + rr;
        const int h = 1 << (G - 1 - rr);
        const bool final_stage = INV && STRIDED && st == 0;
        // inverse lazy bound: inputs of this stage < 2^(done+it+1) q
        const uint64_t bq = q2 << (done + it);
        const uint32_t idx0 = (1u << (gs0 + st)) + (prefix << st) + (B << rr);
        ulonglong2 w[4];
        if (!final_stage) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < (1 << rr)) w[j] = __ldg(tw + idx0 + j);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (k >= usz) break;
          if (k & h) continue;
          if (!INV) {
            if (LAZY)
              ct_bfly_lazy(xu[k], xu[k + h], w[k >> (G - rr)], q, q2);
            else
              ct_bfly(xu[k], xu[k + h], w[k >> (G - rr)], q, q2);
          } else if (!final_stage) {
            if (LAZY)
              gs_bfly_lazy(xu[k], xu[k + h], w[k >> (G - rr)], q, bq);
            else
              gs_bfly(xu[k], xu[k + h], w[k >> (G - rr)], q, q2);
          } else {
            const ulonglong2 c0 = a.scale_a ? __ldg(a.scale_a + (prime - a.scale_base)) : __ldg(a.ninv_last + prime);
            const ulonglong2 c1 = a.scale_b ? __ldg(a.scale_b + (prime - a.scale_base)) : __ldg(a.w1_ninv + prime);
            const uint64_t u0 = xu[k], v0 = xu[k + h];
            const uint64_t off = LAZY ? bq : q2;
            const uint64_t s0 = mul_shoup_lazy(u0 + v0, c0.x, c0.y, q);
            const uint64_t d0 = mul_shoup_lazy(u0 + off - v0, c1.x, c1.y, q);
            xu[k] = s0 >= q ? s0 - q : s0;
            xu[k + h] = d0 >= q ? d0 - q : d0;
          }
        }
      }
    }
    done += G;
    // store
    if (step + 1 < NG) {
      if (step > 0) __syncthreads();  // everyone has read the previous layout
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= units_per_thread * usz) break;
        const int uj = j / usz, k = j % usz;
        const int u = sub_t + uj * T;
        sm[saddr((u / D) * (D << G) + (u % D) + k * D)] = x[j];
      }
      __syncthreads();
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= units_per_thread * usz) break;
        const int uj = j / usz, k = j % usz;
        const int u = sub_t + uj * T;
        uint64_t v = x[j];
        if (last_pass && !INV) {  // forward output -> [0, q)
          if (LAZY) v = reduce_2q(v, q, w1);
          else v = v >= q2 ? v - q2 : v;
          v = v >= q ? v - q : v;
        } else if (LAZY && INV && !last_pass) {  // first inverse pass -> [0, 2q)
          v = reduce_2q(v, q, w1);
        }
        // inverse output of the final stage is already canonical; a forward
        // first pass hands values < 4q + 2q S_LOG to the second
        poly[gaddr((u / D) * (D << G) + (u % D) + k * D)] = v;
      }
    }
  }
}

template <int S_LOG, bool INV, bool STRIDED>
__global__ void __launch_bounds__(kThreads, 2) ntt_pass_kernel(uint64_t* __restrict__ data, PassArgs a) {
  extern __shared__ uint64_t sm[];
  const int limb = blockIdx.y;
  if (a.map.skipped(limb)) return;
  const uint64_t q = a.mods[a.map.prime(limb)].q;
  if (q < (1ull << kLazyBits))
    ntt_pass_body<S_LOG, INV, STRIDED, true>(data, a, sm);
  else
    ntt_pass_body<S_LOG, INV, STRIDED, false>(data, a, sm);
}

template <int S_LOG, bool INV, bool STRIDED>
void launch_pass(uint64_t* data, int nlimbs, const PassArgs& a0, cudaStream_t st) {
  constexpr int S = 1 << S_LOG;
  constexpr int T = S >= 8 ? S / 8 : 1;
  const int N = 1 << a0.logN;
  const int subs = N / S;  // sub-transforms per limb
  int per = kThreads / T;
  if (per > subs) per = subs;
  PassArgs a = a0;
  a.per_cta = per;
  const dim3 grid(subs / per, nlimbs);
  const int threads = per * T;
  const size_t smem = STRIDED ? (size_t)S * per * sizeof(uint64_t)
                              : (size_t)per * (S + S / 16) * sizeof(uint64_t);
  auto k = ntt_pass_kernel<S_LOG, INV, STRIDED>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k<<<grid, threads, smem, st>>>(data, a);
}

template <bool INV, bool STRIDED>
void dispatch_pass(int s_log, uint64_t* data, int nlimbs, const PassArgs& a, cudaStream_t st) {
  switch (s_log) {
    case 3: launch_pass<3, INV, STRIDED>(data, nlimbs, a, st); break;
    case 4: launch_pass<4, INV, STRIDED>(data, nlimbs, a, st); break;
    case 5: launch_pass<5, INV, STRIDED>(data, nlimbs, a, st); break;
    case 6: launch_pass<6, INV, STRIDED>(data, nlimbs, a, st); break;
    case 7: launch_pass<7, INV, STRIDED>(data, nlimbs, a, st); break;
    case 8: launch_pass<8, INV, STRIDED>(data, nlimbs, a, st); break;
    case 9: launch_pass<9, INV, STRIDED>(data, nlimbs, a, st); break;
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

void ntt_forward(const Context& c, uint64_t* data, int nlimbs, LimbMap map, cudaStream_t st) {
  if (nlimbs <= 0) return;
  // algorithmic traffic of a transform is one read + one write per limb;
  // each of the two passes is credited with half of it
  const double bytes = live_limbs(map, nlimbs) * c.limb_bytes();
  PassArgs a{};
  a.tw = c.d_tw;
  a.mods = c.d_mods;
  a.map = map;
  a.logN = c.logN;
  const int s1 = c.logN / 2, s2 = c.logN - s1;
  {
    ProfScope ps(c, "ntt_fwd_rows", bytes, st);
    dispatch_pass<false, true>(s1, data, nlimbs, a, st);
  }
  {
    ProfScope ps(c, "ntt_fwd_cols", bytes, st);
    dispatch_pass<false, false>(s2, data, nlimbs, a, st);
  }
  CKKS_CUDA(cudaGetLastError());
}

void ntt_inverse(const Context& c, uint64_t* data, int nlimbs, LimbMap map, cudaStream_t st,
                 const ulonglong2* scale_a, const ulonglong2* scale_b, int scale_base) {
  if (nlimbs <= 0) return;
  const double bytes = live_limbs(map, nlimbs) * c.limb_bytes();
  PassArgs a{};
  a.tw = c.d_itw;
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
    dispatch_pass<true, false>(s2, data, nlimbs, a, st);
  }
  {
    ProfScope ps(c, "ntt_inv_rows", bytes, st);
    dispatch_pass<true, true>(s1, data, nlimbs, a, st);
  }
  CKKS_CUDA(cudaGetLastError());
}

}  // namespace ckks
