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
  LimbMap map;
  int logN;
  int per_cta;  // columns (strided) or blocks (contiguous) per CTA
};

__device__ __forceinline__ int group_size(int s_log, int gi) {
  const int rem = s_log - 3 * gi;
  return rem < 3 ? rem : 3;
}

template <int S_LOG, bool INV, bool STRIDED>
__global__ void __launch_bounds__(kThreads) ntt_pass_kernel(uint64_t* __restrict__ data, PassArgs a) {
  constexpr int S = 1 << S_LOG;
  constexpr int T = S >= 8 ? S / 8 : 1;  // threads per sub-transform
  constexpr int NG = (S_LOG + 2) / 3;     // register stage groups
  extern __shared__ uint64_t sm[];

  const int limb = blockIdx.y;
  const int prime = a.map.prime(limb);
  if (a.map.skipped(limb)) return;
  const int N = 1 << a.logN;
  uint64_t* poly = data + (size_t)limb * N;
  const Mod md = a.mods[prime];
  const uint64_t q = md.q;
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
  // twiddle prefix: global stage offset and block index for contiguous passes
  const int gs0 = STRIDED ? 0 : (a.logN - S_LOG);
  const uint32_t prefix = STRIDED ? 0u : (uint32_t)sub_global;

  auto gaddr = [&](int r) -> size_t {
    return STRIDED ? (size_t)r * stride + sub_global : (size_t)sub_global * S + r;
  };
  auto saddr = [&](int r) -> int {
    return STRIDED ? r * per + lane_idx : lane_idx * (S + S / 16) + r + (r >> 4);
  };

  uint64_t x[8];

  auto tw_index = [&](int st, int r) -> uint32_t {
    return (1u << (gs0 + st)) + (prefix << st) + ((uint32_t)r >> (S_LOG - st));
  };

  // process stage group gi on registers; `first`/`last` select global I/O
#pragma unroll
  for (int step = 0; step < NG; ++step) {
    const int gi = INV ? (NG - 1 - step) : step;
    const int G = group_size(S_LOG, gi);
    const int st0 = 3 * gi;
    const int D = S >> (st0 + G);  // smallest distance (unit stride)
    const int units_per_thread = 8 >> G;
    const int usz = 1 << G;
    // load
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= units_per_thread * usz) break;
      const int uj = j / usz, k = j % usz;
      const int u = sub_t + uj * T;
      const int base = (u / D) * (D << G) + (u % D);
      const int r = base + k * D;
      if (step == 0)
        x[j] = poly[gaddr(r)];
      else
        x[j] = sm[saddr(r)];
    }
    // butterflies
#pragma unroll
    for (int uj = 0; uj < 8; ++uj) {
      if (uj >= units_per_thread) break;
      const int u = sub_t + uj * T;
      const int base = (u / D) * (D << G) + (u % D);
      uint64_t* xu = x + uj * usz;
      if (!INV) {
#pragma unroll
        for (int rr = 0; rr < 3; ++rr) {
          if (rr >= G) break;
          const int st = st0 + rr;
          const int h = 1 << (G - 1 - rr);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (k >= usz) break;
            if (k & h) continue;
            const int r = base + k * D;
            const ulonglong2 w = __ldg(tw + tw_index(st, r));
            const uint64_t u0 = xu[k];
            const uint64_t v0 = mul_shoup(xu[k + h], w.x, w.y, q);
            xu[k] = add_mod(u0, v0, q);
            xu[k + h] = sub_mod(u0, v0, q);
          }
        }
      } else {
#pragma unroll
        for (int rr = 2; rr >= 0; --rr) {
          if (rr >= G) continue;
          const int st = st0 + rr;
          const int h = 1 << (G - 1 - rr);
          const bool final_stage = STRIDED && st == 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (k >= usz) break;
            if (k & h) continue;
            const int r = base + k * D;
            const uint64_t u0 = xu[k], v0 = xu[k + h];
            if (final_stage) {
              const ulonglong2 ni = __ldg(a.ninv_last + prime);
              const ulonglong2 wn = __ldg(a.w1_ninv + prime);
              xu[k] = mul_shoup(add_mod(u0, v0, q), ni.x, ni.y, q);
              xu[k + h] = mul_shoup(sub_mod(u0, v0, q), wn.x, wn.y, q);
            } else {
              const ulonglong2 w = __ldg(tw + tw_index(st, r));
              xu[k] = add_mod(u0, v0, q);
              xu[k + h] = mul_shoup(sub_mod(u0, v0, q), w.x, w.y, q);
            }
          }
        }
      }
    }
    // store
    if (step + 1 < NG) {
      if (step > 0) __syncthreads();  // everyone has read the previous layout
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= units_per_thread * usz) break;
        const int uj = j / usz, k = j % usz;
        const int u = sub_t + uj * T;
        const int base = (u / D) * (D << G) + (u % D);
        sm[saddr(base + k * D)] = x[j];
      }
      __syncthreads();
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= units_per_thread * usz) break;
        const int uj = j / usz, k = j % usz;
        const int u = sub_t + uj * T;
        const int base = (u / D) * (D << G) + (u % D);
        poly[gaddr(base + k * D)] = x[j];
      }
    }
  }
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

void ntt_inverse(const Context& c, uint64_t* data, int nlimbs, LimbMap map, cudaStream_t st) {
  if (nlimbs <= 0) return;
  const double bytes = live_limbs(map, nlimbs) * c.limb_bytes();
  PassArgs a{};
  a.tw = c.d_itw;
  a.mods = c.d_mods;
  a.ninv_last = c.d_ninv;
  a.w1_ninv = c.d_w1ninv;
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
