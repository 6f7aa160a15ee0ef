// block.cu -- one encrypted DNAGPT transformer block (pre-LN, bias-free) on
// the engine: the server-side schedule of the reference's
// EncryptedEvaluator::evaluate with its client refreshes
// (fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_depth13_
//  digits3_ring65536_cpudiagcache_t123.cpp, "T123.cpp", :762-948 and :509-715).
//
// Layout: B tokens per ciphertext, lane-innermost,
//   slot(feature f, lane t) = f * B + t,  f < PW = N / (2B),
// so a rotation by B*k moves every token's features by k without crossing
// tokens (T123.cpp:419-426 with one copy; simd_layout.py:55-81).  With B = 32
// the T = 103 tokens take 4 ciphertexts (32, 32, 32, 7).
//
// Per token group, in order (T123.cpp:780-923):
//   LN1      AccumulateSum over features -> mean, centered, centered^2 ->
//            AccumulateSum -> variance; the client returns 1/sqrt(var + eps);
//            the LN gain is folded into the next weight matrix (x W^T with
//            W' = W diag(gamma)).
//   QKV      one hoisted baby-step set, three fused BSGS products (n1 = n2 = 32).
//   scores   for every causal (query group, key group, lane shift delta):
//            Q * lane_shift(K, delta), then a window sum over each head's 64
//            features (the AccumulateSum ladder, each step one hoisted
//            rotation sum); the client reads score(q, k, head) at feature
//            64*head and runs the exact float64 softmax (T123.cpp:629-665).
//   context  the client encrypts the weight tile of every alignment; the
//            server accumulates tile * lane_shift(V, delta).
//   O proj   BSGS; residual1 = x + O.
//   LN2      as LN1.
//   MLP      fc in PW-row chunks (BSGS each); the client applies exact
//            tanh-GELU (T123.cpp:190-194); down projection per chunk; sum;
//            block output = residual1 + MLP.
// Fresh ciphertexts (inputs and client refreshes) are encrypted at the level
// that leaves exactly the depth still needed plus two limbs at every
// decryption, so the key switches run on 3..11 limbs of the 24-limb chain.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <string>
#include <vector>

#include "../../include/ckks_b200.h"
#include "../../include/ckks_b200.hpp"
#include "capi_types.hpp"
#include "bulk.cuh"
#include "ckks_internal.hpp"
#include "fpmod.cuh"

using ckks_b200::Ciphertext;
using ckks_b200::Plaintext;

namespace blk {

constexpr int kThreads = 256;
constexpr int kMaxBaby = 32;

struct Shape {
  int T = 103, B = 32, D = 768, H = 12, HD = 64, MLP = 3072;
  int PW = 1024, n1 = 32, n2 = 32, groups = 4;
  int count(int g) const { return std::min(B, T - g * B); }
};

// lane shifts delta whose (query lane, key lane) pairs include a causal pair
// (simd_layout.py:386-406, T123.cpp:483-507)
std::vector<int> active_shifts(int T, int B, int qg, int kg) {
  const int qs = qg * B, ks = kg * B;
  const int qc = std::min(B, T - qs), kc = std::min(B, T - ks);
  std::vector<int> out;
  for (int d = 0; d < B; ++d) {
    for (int ql = 0; ql < qc; ++ql) {
      const int kl = (ql + d) % B;
      if (kl < kc && ks + kl <= qs + ql) {
        out.push_back(d);
        break;
      }
    }
  }
  return out;
}

// value of BSGS diagonal (g, j) at `feature`, pre-rotated by the giant step:
// W[rolled][(rolled + n1 g + j) mod PW] with rolled = (feature - n1 g) mod PW,
// zero outside the matrix (T123.cpp:1018-1046, simd_layout.py:161-178)
__host__ __device__ inline double diag_value(const double* W, int out_dim, int in_dim, int ld, int PW, int n1, int g,
                                             int j, int feature) {
  const int rolled = (feature + PW - (n1 * g) % PW) % PW;
  const int col = (rolled + n1 * g + j) % PW;
  return (rolled < out_dim && col < in_dim) ? W[(size_t)rolled * ld + col] : 0.0;
}

__global__ void __launch_bounds__(kThreads) diag_values_kernel(const double* __restrict__ W, int out_dim, int in_dim,
                                                               int ld, int PW, int B, int n1, int d0,
                                                               double* __restrict__ vals) {
  const int slots = PW * B;
  const int s = blockIdx.x * kThreads + threadIdx.x;
  if (s >= slots) return;
  const int d = d0 + blockIdx.y;
  vals[(size_t)blockIdx.y * slots + s] = diag_value(W, out_dim, in_dim, ld, PW, n1, d / n1, d % n1, s / B);
}

// token groups per BSGS launch.  Sharing one pass over a product's diagonals
// between groups (thread rows) did not pay: the kernel is bound by issue and
// load latency of its 128-bit multiply-accumulates, not by the diagonal
// traffic, so one group per launch keeps the most warps resident.
constexpr int kMaxGroups = 4;
struct BabyPtrs {
  const uint64_t* c0[kMaxGroups][kMaxBaby];
  const uint64_t* c1[kMaxGroups][kMaxBaby];
};
struct InnerPtrs {
  uint64_t* c0[kMaxGroups][kMaxBaby];
  uint64_t* c1[kMaxGroups][kMaxBaby];
};

using ckks::fp_canonical;
using ckks::fp_center;
using ckks::fp_mod_product;
using ckks::kFpPrime;
using ckks::u2d;

// Encoded diagonals are stored tile-major, [limb][tile of kDiagTile
// coefficients][diagonal][kDiagTile residues], so that the n1 diagonals of
// one giant step over the coefficients of one CTA of the product are one
// contiguous span (16 KiB at n1 = 32), streamed by a single bulk copy: this
// transposes a chunk of plaintext-major encodings into place.  Limbs whose
// prime is below kFpPrime hold their residues as doubles.
constexpr int kDiagTile = 64;

// word offset of diagonal d, coefficient n of limb l in the tile-major store
__host__ __device__ __forceinline__ size_t diag_offset(int l, int n, int d, int N, int ndiag) {
  return (((size_t)l * (N / kDiagTile) + n / kDiagTile) * ndiag + d) * kDiagTile + n % kDiagTile;
}

__global__ void __launch_bounds__(kThreads) diag_tile_kernel(const uint64_t* __restrict__ src, int cnt, int d0,
                                                             int ndiag, int limbs, int logN,
                                                             const ckks::Mod* __restrict__ mods,
                                                             uint64_t* __restrict__ dst) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x, l = blockIdx.y, dd = blockIdx.z;
  if (dd >= cnt) return;
  uint64_t v = src[((size_t)dd * limbs + l) * N + n];
  if (mods[l].q < kFpPrime) v = (uint64_t)__double_as_longlong((double)v);
  dst[diag_offset(l, n, d0 + dd, N, ndiag)] = v;
}

// inner_g = sum_j diag[g n1 + j] * baby_j.  One CTA = one giant step g, one
// 256-coefficient tile of one limb; each thread owns two adjacent
// coefficients (16-byte loads) and four 128-bit MAC chains, so the kernel
// runs at full occupancy.  Consecutive CTAs share the tile, so the baby
// residues they re-read stay in L2.
constexpr int kBsgsThreads = 128;

// inner sums of giant step g for `ng` token groups in one CTA of
// kBsgsThreads x ng threads: thread row q computes group q
__global__ void __launch_bounds__(kBsgsThreads * kMaxGroups) bsgs_inner_kernel(BabyPtrs babies, int ng, int n1,
                                                                               const uint64_t* __restrict__ diag,
                                                                               InnerPtrs out, int limbs, int logN,
                                                                               int n2, int l0, bool accumulate,
                                                                               const ckks::Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int g = blockIdx.x, tile = blockIdx.y, l = l0 + blockIdx.z;
  const int q = threadIdx.y;
  if (q >= ng) return;
  const int c = 2 * threadIdx.x;  // coefficient within the tile
  const size_t off = (size_t)l * N + (size_t)tile * kThreads + c;
  const int ndiag = n1 * n2;
  const uint64_t* dtile = diag + diag_offset(l, tile * kThreads + c, g * n1, N, ndiag);
  ckks::U128 a00{0, 0}, a01{0, 0}, a10{0, 0}, a11{0, 0};
  for (int j = 0; j < n1; ++j) {
    const ulonglong2 b0 = *reinterpret_cast<const ulonglong2*>(babies.c0[q][j] + off);
    const ulonglong2 b1 = *reinterpret_cast<const ulonglong2*>(babies.c1[q][j] + off);
    const ulonglong2 dv = __ldg(reinterpret_cast<const ulonglong2*>(dtile + (size_t)j * kDiagTile));
    ckks::mac_wide(a00, dv.x, b0.x);
    ckks::mac_wide(a01, dv.y, b0.y);
    ckks::mac_wide(a10, dv.x, b1.x);
    ckks::mac_wide(a11, dv.y, b1.y);
  }
  const ckks::Mod m = mods[l];
  ulonglong2 r0 = make_ulonglong2(ckks::reduce128(a00, m), ckks::reduce128(a01, m));
  ulonglong2 r1 = make_ulonglong2(ckks::reduce128(a10, m), ckks::reduce128(a11, m));
  if (accumulate) {
    const ulonglong2 p0 = *reinterpret_cast<const ulonglong2*>(out.c0[q][g] + off);
    const ulonglong2 p1 = *reinterpret_cast<const ulonglong2*>(out.c1[q][g] + off);
    r0 = make_ulonglong2(ckks::add_mod(r0.x, p0.x, m.q), ckks::add_mod(r0.y, p0.y, m.q));
    r1 = make_ulonglong2(ckks::add_mod(r1.x, p1.x, m.q), ckks::add_mod(r1.y, p1.y, m.q));
  }
  *reinterpret_cast<ulonglong2*>(out.c0[q][g] + off) = r0;
  *reinterpret_cast<ulonglong2*>(out.c1[q][g] + off) = r1;
}

// the same inner sums for a limb whose prime is below kFpPrime: diagonals
// stored as doubles, babies converted on load, float64 products
__global__ void __launch_bounds__(kBsgsThreads * kMaxGroups) bsgs_inner_fp_kernel(BabyPtrs babies, int ng, int n1,
                                                                                  const uint64_t* __restrict__ diag,
                                                                                  InnerPtrs out, int limbs, int logN,
                                                                                  int n2, int l0, bool accumulate,
                                                                                  const ckks::Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int g = blockIdx.x, tile = blockIdx.y, l = l0 + blockIdx.z;
  const int q = threadIdx.y;
  if (q >= ng) return;
  const int c = 2 * threadIdx.x;
  const size_t off = (size_t)l * N + (size_t)tile * kThreads + c;
  const int ndiag = n1 * n2;
  const double* dtile = reinterpret_cast<const double*>(diag) + diag_offset(l, tile * kThreads + c, g * n1, N, ndiag);
  const double qd = (double)mods[l].q, qinv = 1.0 / qd;
  double a00 = 0.0, a01 = 0.0, a10 = 0.0, a11 = 0.0;
  for (int j = 0; j < n1; ++j) {
    const ulonglong2 b0 = *reinterpret_cast<const ulonglong2*>(babies.c0[q][j] + off);
    const ulonglong2 b1 = *reinterpret_cast<const ulonglong2*>(babies.c1[q][j] + off);
    const double2 dv = __ldg(reinterpret_cast<const double2*>(dtile + (size_t)j * kDiagTile));
    a00 = __dadd_rn(a00, fp_mod_product(dv.x, u2d(b0.x), qd, qinv));
    a01 = __dadd_rn(a01, fp_mod_product(dv.y, u2d(b0.y), qd, qinv));
    a10 = __dadd_rn(a10, fp_mod_product(dv.x, u2d(b1.x), qd, qinv));
    a11 = __dadd_rn(a11, fp_mod_product(dv.y, u2d(b1.y), qd, qinv));
    if ((j & 3) == 3) {
      a00 = fp_center(a00, qd, qinv);
      a01 = fp_center(a01, qd, qinv);
      a10 = fp_center(a10, qd, qinv);
      a11 = fp_center(a11, qd, qinv);
    }
  }
  a00 = fp_center(a00, qd, qinv);
  a01 = fp_center(a01, qd, qinv);
  a10 = fp_center(a10, qd, qinv);
  a11 = fp_center(a11, qd, qinv);
  ulonglong2 r0 = make_ulonglong2(fp_canonical(a00, qd), fp_canonical(a01, qd));
  ulonglong2 r1 = make_ulonglong2(fp_canonical(a10, qd), fp_canonical(a11, qd));
  if (accumulate) {
    const uint64_t qi = mods[l].q;
    const ulonglong2 p0 = *reinterpret_cast<const ulonglong2*>(out.c0[q][g] + off);
    const ulonglong2 p1 = *reinterpret_cast<const ulonglong2*>(out.c1[q][g] + off);
    r0 = make_ulonglong2(ckks::add_mod(r0.x, p0.x, qi), ckks::add_mod(r0.y, p0.y, qi));
    r1 = make_ulonglong2(ckks::add_mod(r1.x, p1.x, qi), ckks::add_mod(r1.y, p1.y, qi));
  }
  *reinterpret_cast<ulonglong2*>(out.c0[q][g] + off) = r0;
  *reinterpret_cast<ulonglong2*>(out.c1[q][g] + off) = r1;
}

// Inner sums with the baby residues held in registers: SPLIT lanes share
// one coefficient of one token group and one limb, each holding n1 / SPLIT
// of the babies, looping over the n2 giant steps; the lanes' sums meet by
// shuffles once per giant step.  Each giant step's diagonals over the CTA's
// kDiagTile coefficients (one contiguous span of the tile-major store) come
// in one bulk copy into a two-stage shared-memory ring: thread 0 issues the
// copy of step g + 2 once every thread has passed step g's barrier, so the
// copy of step g + 1 lands while step g computes.  The CTAs of the token
// groups of one tile are adjacent in the grid, so each diagonal tile comes
// from HBM once and from L2 for the other groups, and no baby residue is
// read twice.
//
// On a limb whose prime is below kFpPrime every product is the exact
// float64 one (fp_mod_product), summed in CHAINS independent accumulators
// per output that are re-centred every four products.  On the 60-bit first
// prime the residues are split into 30-bit halves, d = dh 2^30 + dl: each
// product is four 32 x 32 -> 64-bit multiply-adds into four sums (dl bl,
// dl bh, dh bl, dh bh; 16 products of halves below 2^30 stay below 2^64, so
// no carries), recombined into a 128-bit value and Barrett-reduced once per
// giant step (a 64 x 64 -> 128-bit multiply-accumulate costs the same four
// partial products plus its carry chain).  The float64 and the integer
// instances are separate kernels, each with its own register budget.
constexpr int kBsgsRegThreads = 128;
template <int NB, int SPLIT>
struct BsgsShape {
  static constexpr int H = NB / SPLIT;                         // babies per lane
  static constexpr int kCoeffs = kBsgsRegThreads / SPLIT;      // coefficients per CTA
  static constexpr int kParts = kThreads / kCoeffs;            // CTAs per coefficient tile and group
};
constexpr int kRegSplit = 2, kFpChains = 2, kRegMinBlocks = 4;
using ckks::SplitSums;
using ckks::split_residue;

template <int NB, int SPLIT, int CHAINS, int MINB, bool FP>
__global__ void __launch_bounds__(kBsgsRegThreads, MINB)
    bsgs_inner_reg_kernel(BabyPtrs babies, int ng, const uint64_t* __restrict__ diag, InnerPtrs out, int logN, int n2,
                          int l0, bool accumulate, const ckks::Mod* __restrict__ mods,
                          unsigned int* __restrict__ faults) {
  using S = BsgsShape<NB, SPLIT>;
  constexpr int H = S::H;
  static_assert(FP || H <= 16, "at most 16 split products per sum");
  static_assert(!FP || (H % CHAINS == 0 && (H / CHAINS) % 4 == 0), "whole groups of four products per chain");
  static_assert(SPLIT >= 2, "one lane writes c0, another c1");
  static_assert(S::kCoeffs == kDiagTile, "one CTA per tile of the diagonal store");
  constexpr uint32_t kStepBytes = NB * kDiagTile * sizeof(uint64_t);
  __shared__ alignas(128) uint64_t sd[2][NB][kDiagTile];
  __shared__ alignas(8) uint64_t full[2];
  const int N = 1 << logN;
  const int l = l0 + blockIdx.z;
  const int q = blockIdx.x % ng, part = blockIdx.x / ng;
  const int tile = blockIdx.y;
  const int lane = threadIdx.x % SPLIT;
  const int cc = threadIdx.x / SPLIT;                   // coefficient within the CTA's diagonal tile
  const int c = part * S::kCoeffs + cc;                 // coefficient within the 256-coefficient tile
  const size_t off = (size_t)l * N + (size_t)tile * kThreads + c;
  // babies: doubles (FP) or 30-bit halves
  double b0d[FP ? H : 1], b1d[FP ? H : 1];
  uint32_t b0l[FP ? 1 : H], b0h[FP ? 1 : H], b1l[FP ? 1 : H], b1h[FP ? 1 : H];
#pragma unroll
  for (int j = 0; j < H; ++j) {
    const uint64_t v0 = babies.c0[q][lane * H + j][off], v1 = babies.c1[q][lane * H + j][off];
    if constexpr (FP) {
      b0d[j] = u2d(v0);
      b1d[j] = u2d(v1);
    } else {
      split_residue(v0, b0l[j], b0h[j]);
      split_residue(v1, b1l[j], b1h[j]);
    }
  }
  // giant step g's span: diagonals g NB .. g NB + NB - 1 of this tile
  const uint64_t* dt = diag + diag_offset(l, tile * kThreads + part * S::kCoeffs, 0, N, NB * n2);
  const uint32_t bar0 = ckks::smem_addr(&full[0]), bar1 = ckks::smem_addr(&full[1]);
  auto issue = [&](int g) {
    const uint32_t bar = (g & 1) ? bar1 : bar0;
    ckks::mbar_expect_tx(bar, kStepBytes);
    ckks::bulk_load(ckks::smem_addr(&sd[g & 1][0][0]), dt + (size_t)g * NB * kDiagTile, kStepBytes, bar);
  };
  if (threadIdx.x == 0) {
    ckks::mbar_init(bar0, 1);
    ckks::mbar_init(bar1, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    issue(0);
    if (n2 > 1) issue(1);
  }
  const ckks::Mod m = mods[l];
  const double qd = (double)m.q, qinv = 1.0 / qd;
  for (int g = 0; g < n2; ++g) {
    const int buf = g & 1;
    const bool arrived = ckks::mbar_wait_bounded(buf ? bar1 : bar0, (g >> 1) & 1);
    uint64_t r0 = 0, r1 = 0;
    if constexpr (FP) {
      double a0[CHAINS], a1[CHAINS];
#pragma unroll
      for (int k = 0; k < CHAINS; ++k) a0[k] = a1[k] = 0.0;
#pragma unroll
      for (int j = 0; j < H; ++j) {
        const int k = j % CHAINS;
        const double d = __longlong_as_double((long long)sd[buf][lane * H + j][cc]);
        a0[k] = __dadd_rn(a0[k], fp_mod_product(d, b0d[j], qd, qinv));
        a1[k] = __dadd_rn(a1[k], fp_mod_product(d, b1d[j], qd, qinv));
        if ((j / CHAINS) % 4 == 3) {  // four products since this chain's last re-centring
          a0[k] = fp_center(a0[k], qd, qinv);
          a1[k] = fp_center(a1[k], qd, qinv);
        }
      }
      // |a[k]| < 0.51 q: the chains and lanes add up to < 0.51 q CHAINS
      // SPLIT <= 4.1 q, exact
      double t0 = a0[0], t1 = a1[0];
#pragma unroll
      for (int k = 1; k < CHAINS; ++k) {
        t0 = __dadd_rn(t0, a0[k]);
        t1 = __dadd_rn(t1, a1[k]);
      }
#pragma unroll
      for (int sh = 1; sh < SPLIT; sh <<= 1) {
        t0 = __dadd_rn(t0, __shfl_xor_sync(0xffffffffu, t0, sh));
        t1 = __dadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, sh));
      }
      const double t = lane == 0 ? t0 : t1;
      r0 = r1 = fp_canonical(fp_center(t, qd, qinv), qd);
    } else {
      SplitSums s0, s1;
#pragma unroll
      for (int j = 0; j < H; ++j) {
        uint32_t dl, dh;
        split_residue(sd[buf][lane * H + j][cc], dl, dh);
        s0.mac(dl, dh, b0l[j], b0h[j]);
        s1.mac(dl, dh, b1l[j], b1h[j]);
      }
      r0 = s0.reduce(m);
      r1 = s1.reduce(m);
#pragma unroll
      for (int sh = 1; sh < SPLIT; sh <<= 1) {
        r0 = ckks::add_mod(r0, __shfl_xor_sync(0xffffffffu, r0, sh), m.q);
        r1 = ckks::add_mod(r1, __shfl_xor_sync(0xffffffffu, r1, sh), m.q);
      }
    }
    // every thread is done with this buffer: it takes step g + 2's copy
    if (!__syncthreads_and(arrived)) {
      // a copy did not arrive: count it, wait (bounded) for the copy still
      // in flight, and leave this CTA's remaining outputs unwritten
      if (threadIdx.x == 0) {
        atomicAdd(faults, 1u);
        if (g + 1 < n2) ckks::mbar_wait_bounded(buf ? bar0 : bar1, ((g + 1) >> 1) & 1);
      }
      return;
    }
    if (threadIdx.x == 0 && g + 2 < n2) issue(g + 2);
    if (lane < 2) {
      uint64_t* dst = lane == 0 ? out.c0[q][g] : out.c1[q][g];
      uint64_t r = lane == 0 ? r0 : r1;
      if (accumulate) r = ckks::add_mod(r, dst[off], m.q);
      dst[off] = r;
    }
  }
}

// Inner sums of one product term over limbs [0, limbs): each run of limbs
// whose primes allow float64 products goes to the FP instance, each other
// run (the 60-bit first prime) to the all-integer one.
template <int NB>
void launch_bsgs_inner_reg(const ckks::Context& C, const BabyPtrs& bp, int ng, const uint64_t* dg, const InnerPtrs& ip,
                           int limbs, int n2, bool acc) {
  using S = BsgsShape<NB, kRegSplit>;
  static_assert(kThreads % S::kCoeffs == 0, "a tile of whole CTAs");
  constexpr int CH = S::H / 4 < kFpChains ? S::H / 4 : kFpChains;
  for (int l0 = 0; l0 < limbs;) {
    const bool fp = C.moduli[l0] < kFpPrime;
    int l1 = l0 + 1;
    while (l1 < limbs && (C.moduli[l1] < kFpPrime) == fp) ++l1;
    const dim3 grid(ng * S::kParts, C.N / kThreads, l1 - l0);
    if (fp)
      bsgs_inner_reg_kernel<NB, kRegSplit, CH, kRegMinBlocks, true>
          <<<grid, kBsgsRegThreads, 0, C.stream>>>(bp, ng, dg, ip, C.logN, n2, l0, acc, C.d_mods, C.d_faults);
    else
      bsgs_inner_reg_kernel<NB, kRegSplit, CH, kRegMinBlocks, false>
          <<<grid, kBsgsRegThreads, 0, C.stream>>>(bp, ng, dg, ip, C.logN, n2, l0, acc, C.d_mods, C.d_faults);
    l0 = l1;
  }
}

// ---- client-side float64 transforms, on the device ------------------------
// (the reference computes these exactly in float64 on the host:
//  1/sqrt T123.cpp:514-538, tanh-GELU :190-194/:540-568, softmax :629-665)
__global__ void invsqrt_kernel(double* __restrict__ v, int n) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i < n) v[i] = 1.0 / sqrt(v[i]);
}

// GELU on features < odim of lanes < count, zero elsewhere; item m = blockIdx.y
__global__ void gelu_kernel(const double* __restrict__ in, double* __restrict__ out, int B, int odim, int count,
                            int slots) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= slots) return;
  const size_t o = (size_t)blockIdx.y * slots + i;
  const int f = i / B, t = i % B;
  double r = 0.0;
  if (f < odim && t < count) {
    const double u = in[o];
    r = 0.5 * u * (1.0 + tanh(0.7978845608028654 * (u + 0.044715 * u * u * u)));
  }
  out[o] = r;
}

// numerically stable SiLU on features < odim of lane 0, zero elsewhere (the
// head's single-token boundary, 12blocks_head..._t123_v3.cpp:536-542, 740-755)
__global__ void silu_kernel(const double* __restrict__ in, double* __restrict__ out, int B, int odim, int slots) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= slots) return;
  const int f = i / B, t = i % B;
  double r = 0.0;
  if (f < odim && t == 0) {
    const double u = in[i];
    if (u >= 0.0) {
      r = u / (1.0 + exp(-u));
    } else {
      const double e = exp(u);
      r = u * e / (1.0 + e);
    }
  }
  out[i] = r;
}

// x [T, D] -> group g slot vectors (feature f, lane t) = x[g B + t][f]
__global__ void pack_kernel(const double* __restrict__ x, double* __restrict__ vals, int T, int D, int B, int slots) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= slots) return;
  const int g = blockIdx.y, f = i / B, t = i % B, tok = g * B + t;
  vals[(size_t)g * slots + i] = (f < D && tok < T) ? x[(size_t)tok * D + f] : 0.0;
}

// token group g0 + blockIdx.y from slot vector blockIdx.y of vals
__global__ void unpack_kernel(const double* __restrict__ vals, double* __restrict__ y, int T, int D, int B,
                              int slots, int g0) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= slots) return;
  const int g = g0 + blockIdx.y, f = i / B, t = i % B, tok = g * B + t;
  if (f < D && tok < T) y[(size_t)tok * D + f] = vals[(size_t)blockIdx.y * slots + i];
}

struct TileTag {
  int qg, kg, d;
};

// score(q, k, head) from the head-window sums: feature head*HD, lane q - qg*B
// alignment (qg, kg, d) of a packed score tile (decrypted slot vector v)
struct ScoreTag {
  int qg, kg, d, v;
};

// score(q, k, head) from a packed tile: alignment d of head h sits at
// feature (h*HD - d) mod PW, lane q - qg*B (the isolation mask already applied
// the 1/sqrt(HD) scale)
__global__ void score_gather_kernel(const double* __restrict__ vals, const ScoreTag* __restrict__ tags, int T, int H,
                                    int HD, int B, int PW, int slots, double* __restrict__ scores) {
  const int ql = threadIdx.x;  // one lane per thread, B <= blockDim
  const int m = blockIdx.x, h = blockIdx.y;
  if (ql >= B) return;
  const ScoreTag tg = tags[m];
  const int kl = (ql + tg.d) % B;
  const int q = tg.qg * B + ql, k = tg.kg * B + kl;
  if (q >= T || k >= T || k > q) return;
  const int f = (h * HD - tg.d + PW) % PW;
  scores[((size_t)q * H + h) * T + k] = vals[(size_t)tg.v * slots + (size_t)f * B + ql];
}

// stable causal softmax of row (q, h) over k <= q; a missing score poisons the row
__global__ void softmax_kernel(const double* __restrict__ scores, double* __restrict__ prob, int T, int H,
                               int* __restrict__ bad) {
  const int r = blockIdx.x * kThreads + threadIdx.x;
  if (r >= T * H) return;
  const int q = r / H;
  const double* row = scores + (size_t)r * T;
  double* out = prob + (size_t)r * T;
  double mx = -INFINITY;
  for (int k = 0; k <= q; ++k) {
    if (!isfinite(row[k])) atomicExch(bad, 1);
    mx = fmax(mx, row[k]);
  }
  double den = 0.0;
  for (int k = 0; k <= q; ++k) den += exp(row[k] - mx);
  for (int k = 0; k < T; ++k) out[k] = k <= q ? exp(row[k] - mx) / den : 0.0;
}

// weight tile of alignment m: (feature f, lane ql) = prob[q][f / HD][k]
__global__ void weight_tile_kernel(const double* __restrict__ prob, const TileTag* __restrict__ tags, int T, int H,
                                   int HD, int D, int B, int slots, double* __restrict__ vals) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= slots) return;
  const int m = blockIdx.y;
  const TileTag tg = tags[m];
  const int f = i / B, ql = i % B;
  const int kl = (ql + tg.d) % B;
  const int q = tg.qg * B + ql, k = tg.kg * B + kl;
  double v = 0.0;
  if (f < D && q < T && k < T && k <= q) v = prob[((size_t)q * H + f / HD) * T + k];
  vals[(size_t)m * slots + i] = v;
}

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// All n1 * n2 BSGS diagonals of W ([out, in] float64 on the device, row
// stride ld) as plaintexts of `limbs` limbs at `scale`, in the tile-major
// layout the inner-sum kernels stream (the reference encodes them on the
// host, cached_diagonal_plains, T123.cpp:1005-1059).  Returns a buffer of
// n1 * n2 * limbs * N words from C.alloc.
uint64_t* encode_diagonals(ckks::Context& C, const double* W, int od, int idim, int ld, int PW, int B, int n1,
                           int n2, int limbs, double scale) {
  const int nd = n1 * n2, slots = PW * B;
  const size_t stride = (size_t)limbs * C.N;
  uint64_t* data = (uint64_t*)C.alloc(sizeof(uint64_t) * nd * stride);
  const int chunk = 128;
  double* vals = (double*)C.alloc(sizeof(double) * (size_t)chunk * slots);
  uint64_t* enc = (uint64_t*)C.alloc(sizeof(uint64_t) * (size_t)chunk * stride);
  for (int d0 = 0; d0 < nd; d0 += chunk) {
    const int cnt = std::min(chunk, nd - d0);
    {
      ckks::ProfScope ps(C, "diag_values", 8.0 * slots * cnt, C.stream);
      diag_values_kernel<<<dim3((slots + kThreads - 1) / kThreads, cnt), kThreads, 0, C.stream>>>(
          W, od, idim, ld, PW, B, n1, d0, vals);
    }
    CKKS_CUDA(cudaGetLastError());
    ckks::encode_batch(C, vals, cnt, limbs, scale, enc, stride, C.stream);
    {
      ckks::ProfScope ps(C, "diag_tile", 2.0 * cnt * stride * 8.0, C.stream);
      diag_tile_kernel<<<dim3(C.N / kThreads, limbs, cnt), kThreads, 0, C.stream>>>(enc, cnt, d0, nd, limbs, C.logN,
                                                                                     C.d_mods, data);
    }
    CKKS_CUDA(cudaGetLastError());
  }
  C.release(vals);
  C.release(enc);
  return data;
}

// encoded diagonals of one matrix term of a product
struct DiagRef {
  const uint64_t* data;
  int limbs;
  double scale;
};

// outs[q] = Rescale(sum_g rot(sum_t sum_j diag_t[g n1 + j] * babies[t][q][j],
// B n1 g)) for every token group q: the Halevi-Shoup product of
// matmul(BabyRotations, W) (T123.cpp:1264-1295) summed over the terms t (a
// sum of products x_t W_t^T whose giant-step rotations run once for the
// whole sum, rotation being linear).  babies[t][q] holds the n1 baby steps
// rot(x_{t,q}, B j); every term's diagonals are encoded at the babies'
// limbs.  The inner sums are fused kernels over all groups of a tile (up to
// kMaxGroups per launch); the giant steps of the groups are one rotation sum
// each, their key products sharing launches, then one batched rescale.
std::vector<Ciphertext> bsgs_products(ckks_b200::CryptoContextImpl& cc, ckks::Context& C,
                                      const std::vector<std::vector<std::vector<Ciphertext>>>& babies,
                                      const std::vector<DiagRef>& dgs, int n1, int n2, int B) {
  const int nt = (int)babies.size();
  const int G = nt ? (int)babies[0].size() : 0;
  std::vector<Ciphertext> outs(G);
  if (!G) return outs;
  if ((int)dgs.size() != nt) throw ckks::Error(CKKS_EARG, "one diagonal set per term");
  const int limbs = babies[0][0][0]->limbs();
  for (int t = 0; t < nt; ++t) {
    if ((int)babies[t].size() != G) throw ckks::Error(CKKS_EARG, "terms over different groups");
    if (dgs[t].limbs != limbs) throw ckks::Error(CKKS_ELEVEL, "diagonals at another level than the baby steps");
  }
  std::vector<int> gk(n2);
  for (int g = 0; g < n2; ++g) gk[g] = B * n1 * g;
  for (int q0 = 0; q0 < G; q0 += kMaxGroups) {
    const int ng = std::min(kMaxGroups, G - q0);
    InnerPtrs ip{};
    std::vector<std::vector<Ciphertext>> inner(ng, std::vector<Ciphertext>(n2));
    for (int q = 0; q < ng; ++q) {
      const double sc = babies[0][q0 + q][0]->scale() * dgs[0].scale;
      for (int t = 1; t < nt; ++t) {
        const double st_ = babies[t][q0 + q][0]->scale() * dgs[t].scale;
        if (std::fabs(st_ - sc) > 1e-9 * sc) throw ckks::Error(CKKS_ESCALE, "product terms at different scales");
      }
      for (int g = 0; g < n2; ++g) {
        inner[q][g] = cc.fresh();
        ckks::DevPoly& p = inner[q][g]->handle()->p;
        p.ensure(&C, 2, limbs);
        p.limbs = limbs;
        p.scale = sc;
        p.deg = babies[0][q0 + q][0]->noise_deg() + 1;
        ip.c0[q][g] = p.data;
        ip.c1[q][g] = p.data + (size_t)p.cap * C.N;
      }
    }
    for (int t = 0; t < nt; ++t) {
      BabyPtrs bp{};
      for (int q = 0; q < ng; ++q) {
        const auto& baby = babies[t][q0 + q];
        if ((int)baby.size() != n1) throw ckks::Error(CKKS_EARG, "baby-step count differs from n1");
        for (int j = 0; j < n1; ++j) {
          const ckks::DevPoly& p = baby[j]->handle()->p;
          if (p.limbs != limbs) throw ckks::Error(CKKS_ELEVEL, "baby steps at different levels");
          bp.c0[q][j] = p.data;
          bp.c1[q][j] = p.data + (size_t)p.cap * C.N;
        }
      }
      const uint64_t* dg = dgs[t].data;
      const bool acc = t > 0;
      ckks::ProfScope ps(
          C, "bsgs_inner",
          ((double)n1 * n2 * limbs + ng * (2.0 * n1 * limbs + (acc ? 4.0 : 2.0) * n2 * limbs)) * C.limb_bytes(),
          C.stream);
      // the split products of the integer instance need primes below 2^60
      bool reg = n1 == 32 || n1 == 16 || n1 == 8;
      for (int l = 0; l < limbs; ++l) reg = reg && C.moduli[l] < (1ull << 60);
      if (reg && n1 == 32)
        launch_bsgs_inner_reg<32>(C, bp, ng, dg, ip, limbs, n2, acc);
      else if (reg && n1 == 16)
        launch_bsgs_inner_reg<16>(C, bp, ng, dg, ip, limbs, n2, acc);
      else if (reg)
        launch_bsgs_inner_reg<8>(C, bp, ng, dg, ip, limbs, n2, acc);
      // generic n1: runs of limbs with primes below kFpPrime take the
      // float64 products, the others (the 60-bit first prime) the integer ones
      for (int l0 = 0; l0 < limbs && !reg;) {
        const bool fp = C.moduli[l0] < kFpPrime;
        int l1 = l0 + 1;
        while (l1 < limbs && (C.moduli[l1] < kFpPrime) == fp) ++l1;
        const dim3 grid(n2, C.N / kThreads, l1 - l0);
        if (fp) {
          bsgs_inner_fp_kernel<<<grid, dim3(kBsgsThreads, ng), 0, C.stream>>>(bp, ng, n1, dg, ip, limbs, C.logN, n2,
                                                                               l0, acc, C.d_mods);
        } else {
          bsgs_inner_kernel<<<grid, dim3(kBsgsThreads, ng), 0, C.stream>>>(bp, ng, n1, dg, ip, limbs, C.logN, n2, l0,
                                                                            acc, C.d_mods);
        }
        l0 = l1;
      }
      CKKS_CUDA(cudaGetLastError());
    }
    // giant steps: sum_g rot(inner_g, B n1 g), the key switches summed in the
    // extended basis with one ModDown (g = 0 is the identity); the groups'
    // sums share launches and each giant-step key is read once for them
    const auto sums = cc.RescaleBatch(cc.EvalRotateSumGroups(inner, gk));
    for (int q = 0; q < ng; ++q) outs[q0 + q] = sums[q];
  }
  return outs;
}

// mask plaintext of lane_shift by d: 1 on lanes t < B - d (lower) or t >=
// B - d (upper) of every feature, at `limbs` limbs
using LaneMask = std::function<Plaintext(int d, bool lower, int limbs)>;

// out[i][k] = lane_shift(in[i], ds[k]) for inputs at one limb count, with
// lane_shift(x, d)[f, t] = x[f, (t + d) mod B] = rot(x, d) * lower_d +
// rot(x, d - B) * upper_d, rescaled (simd_layout.py:142-158,
// T123.cpp:1297-1314).  The rotations of every input are one hoisted batch
// (each rotation key read once for all inputs), then batched masks, adds and
// rescales.
std::vector<std::vector<Ciphertext>> lane_shift_set(ckks_b200::CryptoContextImpl& cc, const std::vector<Ciphertext>& in,
                                                    const std::vector<int>& ds, int B, const LaneMask& mask) {
  std::vector<std::vector<Ciphertext>> out(in.size());
  if (in.empty() || ds.empty()) return out;
  const int l = in[0]->limbs();
  std::vector<int> idx;
  for (int d : ds) {
    if (d <= 0 || d >= B) throw ckks::Error(CKKS_EARG, "lane shift outside (0, batch)");
    idx.push_back(d);
    idx.push_back(d - B);
  }
  for (const auto& x : in)
    if (x->limbs() != l) throw ckks::Error(CKKS_ELEVEL, "lane shift inputs at different levels");
  const auto r = cc.EvalFastRotationBatch(in, idx);
  std::vector<Ciphertext> rot;
  std::vector<Plaintext> masks;
  for (size_t g = 0; g < in.size(); ++g)
    for (size_t k = 0; k < ds.size(); ++k) {
      rot.push_back(r[g][2 * k]);
      rot.push_back(r[g][2 * k + 1]);
      masks.push_back(mask(ds[k], true, l));
      masks.push_back(mask(ds[k], false, l));
    }
  const auto prod = cc.EvalMultPlainBatch(rot, masks);
  std::vector<Ciphertext> lo, hi;
  for (size_t j = 0; j < prod.size(); j += 2) {
    lo.push_back(prod[j]);
    hi.push_back(prod[j + 1]);
  }
  const auto rs_ = cc.RescaleBatch(cc.EvalAddBatch(lo, hi));
  for (size_t g = 0; g < in.size(); ++g)
    for (size_t k = 0; k < ds.size(); ++k) out[g].push_back(rs_[g * ds.size() + k]);
  return out;
}

// the slot values of lane_shift's mask: 1 where (t < B - d) == lower
std::vector<double> lane_mask_values(int PW, int B, int d, bool lower) {
  std::vector<double> v((size_t)PW * B, 0.0);
  for (int f = 0; f < PW; ++f)
    for (int t = 0; t < B; ++t) v[(size_t)f * B + t] = ((t < B - d) == lower) ? 1.0 : 0.0;
  return v;
}

}  // namespace blk

struct ckks_block {
  ckks_ctx* ctx;
  ckks_b200::CryptoContextImpl cc;
  ckks::Context& C;
  blk::Shape s;
  int LX = 11;  // limbs of the encrypted input; all other levels follow from it
  // device copies of the weights (gain folded), [out, in] row-major
  double* d_qkv = nullptr;
  double* d_proj = nullptr;
  double* d_fc = nullptr;
  double* d_proj2 = nullptr;
  // classifier head (a head object holds only these): D x D linear with the
  // final LN gain folded in, and the N - A readout with the head LN gain
  double* d_head = nullptr;
  std::vector<double> readout;
  int nfc = 3;
  struct Diag {
    uint64_t* data = nullptr;
    int limbs = 0;
    double scale = 0.0;
  };
  std::map<std::pair<int, int>, Diag> diags;  // (weight id, limbs) -> encoded diagonals
  std::map<std::pair<int, int>, Plaintext> masks;
  // counters (the reference pins the same kinds, T123.cpp:1698-1744)
  std::map<std::string, long> count;
  std::map<std::string, double> seconds;
  double client_seconds = 0.0;

  bool orphaned = false;

  ckks_block(ckks_ctx* c, const blk::Shape& shape) : ctx(c), cc(c), C(*c->c), s(shape) {}
  // device resources; called once, by the destructor or by the context's
  void release_device() {
    if (orphaned) return;
    for (auto& kv : diags) C.release(kv.second.data);
    diags.clear();
    masks.clear();
    cudaFree(d_qkv);
    cudaFree(d_proj);
    cudaFree(d_fc);
    cudaFree(d_proj2);
    cudaFree(d_head);
    d_qkv = d_proj = d_fc = d_proj2 = d_head = nullptr;
    st_x.clear();
    st_q.clear();
    st_k.clear();
    st_v.clear();
    st_ctx.clear();
    st_r1.clear();
    st_mlp.clear();
    C.release(st_prob);
    st_prob = nullptr;
    if (ev_in) cudaEventDestroy(ev_in);
    if (ev_out) cudaEventDestroy(ev_out);
    ev_in = ev_out = nullptr;
    orphaned = true;
  }
  // drop the encoded diagonals and masks (rebuilt on the next use); returns
  // the bytes released
  size_t release_cache() {
    size_t bytes = 0;
    for (auto& kv : diags) {
      bytes += sizeof(uint64_t) * (size_t)s.n1 * s.n2 * kv.second.limbs * C.N;
      C.release(kv.second.data);
    }
    diags.clear();
    masks.clear();
    return bytes;
  }
  size_t cache_bytes() const {
    size_t bytes = 0;
    for (auto& kv : diags) bytes += sizeof(uint64_t) * (size_t)s.n1 * s.n2 * kv.second.limbs * C.N;
    return bytes;
  }
  ~ckks_block() { release_device(); }

  double S(int limbs) const { return C.scales[limbs]; }

  // ---- client role (T123.cpp:509-715), batched on the device ---------------
  // encode + encrypt M slot vectors held on the device (M x N/2 doubles)
  std::vector<Ciphertext> client_encrypt(const double* dvals, int M, int limbs) {
    const double t0 = blk::now_s();
    const size_t stride = (size_t)limbs * C.N;
    uint64_t* pt = (uint64_t*)C.alloc(sizeof(uint64_t) * (size_t)M * stride);
    ckks::encode_batch(C, dvals, M, limbs, S(limbs), pt, stride, C.stream, /*ntt=*/false);
    std::vector<Ciphertext> out(M);
    std::vector<uint64_t*> c0(M), c1(M);
    for (int m = 0; m < M; ++m) {
      out[m] = cc.fresh();
      ckks::DevPoly& p = out[m]->handle()->p;
      p.ensure(&C, 2, limbs);
      p.limbs = limbs;
      p.scale = S(limbs);
      p.deg = 1;
      c0[m] = p.data;
      c1[m] = p.data + (size_t)p.cap * C.N;
    }
    ckks::encrypt_batch_coef(C, pt, limbs, M, c0.data(), c1.data(), C.stream);
    C.release(pt);
    client_seconds += blk::now_s() - t0;
    return out;
  }
  // decrypt + decode ciphertexts of one limb count into M x N/2 doubles (device)
  void client_decrypt(const std::vector<Ciphertext>& cts, double* dout) {
    const double t0 = blk::now_s();
    const int M = (int)cts.size();
    const int limbs = cts[0]->limbs();
    std::vector<const uint64_t*> c0(M), c1(M);
    std::vector<double> sc(M);
    for (int m = 0; m < M; ++m) {
      const ckks::DevPoly& p = cts[m]->handle()->p;
      if (p.limbs != limbs || p.deg != 1) throw ckks::Error(CKKS_ESTATE, "client batch needs rescaled ciphertexts");
      c0[m] = p.data;
      c1[m] = p.data + (size_t)p.cap * C.N;
      sc[m] = p.scale;
    }
    ckks::decrypt_decode_batch(C, c0.data(), c1.data(), limbs, M, sc.data(), dout, C.stream);
    client_seconds += blk::now_s() - t0;
  }
  double* dbuf(size_t n) { return (double*)C.alloc(sizeof(double) * n); }
  int slots() const { return s.PW * s.B; }

  // ---- server helpers -------------------------------------------------------
  Ciphertext rs(const Ciphertext& a) { return cc.Rescale(a); }
  Ciphertext mul_pt_rs(const Ciphertext& a, const Plaintext& p) {
    ++count["ct_plain"];
    return rs(cc.EvalMult(a, p));
  }
  Ciphertext mul_ct_rs(const Ciphertext& a, const Ciphertext& b) {
    ++count["ct_ct"];
    return rs(cc.EvalMult(a, b));
  }
  Ciphertext reduce_to(const Ciphertext& a, int limbs) {
    if (a->limbs() == limbs) return a;
    ++count["level_reduce"];
    return cc.LevelReduce(a, limbs);
  }
  // a at no more than `limbs` limbs: work whose result is next decrypted
  // runs at the fewest limbs that leave two at the decryption
  Ciphertext lower(const Ciphertext& a, int limbs) { return a->limbs() > limbs ? reduce_to(a, limbs) : a; }
  // reduce_to / lower of several ciphertexts, the rescales batched
  std::vector<Ciphertext> reduce_many(const std::vector<Ciphertext>& a, const std::vector<int>& limbs,
                                      bool only_lower = false) {
    std::vector<Ciphertext> out(a);
    std::vector<Ciphertext> xs;
    std::vector<int> ls;
    std::vector<size_t> idx;
    for (size_t i = 0; i < a.size(); ++i) {
      if (a[i]->limbs() == limbs[i] || (only_lower && a[i]->limbs() < limbs[i])) continue;
      ++count["level_reduce"];
      xs.push_back(a[i]);
      ls.push_back(limbs[i]);
      idx.push_back(i);
    }
    if (!xs.empty()) {
      const auto r = cc.LevelReduceBatch(xs, ls);
      for (size_t k = 0; k < idx.size(); ++k) out[idx[k]] = r[k];
    }
    return out;
  }
  // rescales of several ciphertexts, one batch per limb count
  std::vector<Ciphertext> rs_many(const std::vector<Ciphertext>& a) {
    std::vector<Ciphertext> out(a.size());
    std::vector<std::pair<int, std::vector<size_t>>> bins;
    for (size_t i = 0; i < a.size(); ++i) {
      size_t k = 0;
      while (k < bins.size() && bins[k].first != a[i]->limbs()) ++k;
      if (k == bins.size()) bins.push_back({a[i]->limbs(), {}});
      bins[k].second.push_back(i);
    }
    for (const auto& bin : bins) {
      std::vector<Ciphertext> xs;
      for (size_t i : bin.second) xs.push_back(a[i]);
      const auto r = cc.RescaleBatch(xs);
      for (size_t k = 0; k < bin.second.size(); ++k) out[bin.second[k]] = r[k];
    }
    return out;
  }
  Ciphertext rot(const Ciphertext& a, int k) {
    ++count["rotations"];
    return cc.EvalRotate(a, k);
  }
  Ciphertext add(const Ciphertext& a, const Ciphertext& b) { return cc.EvalAdd(a, b); }

  // plaintext of per-feature values, the same on every lane
  Plaintext feature_plain(int id, const std::vector<double>& per_feature, int limbs) {
    auto key = std::make_pair(id, limbs);
    auto it = masks.find(key);
    if (it != masks.end()) return it->second;
    std::vector<double> v((size_t)s.PW * s.B, 0.0);
    for (int f = 0; f < s.PW; ++f)
      for (int t = 0; t < s.B; ++t) v[(size_t)f * s.B + t] = per_feature[f];
    auto p = cc.MakePlaintextAt(v, limbs, S(limbs));
    masks[key] = p;
    return p;
  }
  Plaintext lane_plain(int delta, bool lower, int limbs) {
    auto key = std::make_pair(1000 + 2 * delta + (lower ? 1 : 0), limbs);
    auto it = masks.find(key);
    if (it != masks.end()) return it->second;
    auto p = cc.MakePlaintextAt(blk::lane_mask_values(s.PW, s.B, delta, lower), limbs, S(limbs));
    masks[key] = p;
    return p;
  }

  // isolation mask of alignment tg: `value` at feature h*HD (every head h)
  // of the lanes whose (query, key) pair is causal and inside the sequence
  Plaintext score_plain(const blk::TileTag& tg, int limbs, double value) {
    auto key = std::make_pair(100000 + (tg.qg * s.groups + tg.kg) * s.B + tg.d, limbs);
    auto it = masks.find(key);
    if (it != masks.end()) return it->second;
    std::vector<double> v((size_t)s.PW * s.B, 0.0);
    for (int ql = 0; ql < s.B; ++ql) {
      const int kl = (ql + tg.d) % s.B;
      const int q = tg.qg * s.B + ql, k = tg.kg * s.B + kl;
      if (q >= s.T || k >= s.T || k > q) continue;
      for (int h = 0; h < s.H; ++h) v[(size_t)(h * s.HD) * s.B + ql] = value;
    }
    auto p = cc.MakePlaintextAt(v, limbs, S(limbs));
    masks[key] = p;
    return p;
  }

  // sum over the PW features of every lane (the AccumulateSum ladder of
  // T123.cpp:1154-1159, each base-4 step one hoisted rotation sum), for a
  // batch of ciphertexts at one level
  std::vector<Ciphertext> feature_sums(const std::vector<Ciphertext>& xs) {
    count["accumulate_sum"] += (long)xs.size();
    for (long step = 1; step < s.PW; step *= 4)
      for (int m = 1; m < 4 && step * m < s.PW; ++m) count["rotations"] += (long)xs.size();
    return cc.WindowSumBatch(xs, s.PW, s.B);
  }
  Ciphertext feature_sum(const Ciphertext& x) { return feature_sums({x})[0]; }

  // LayerNorm without the gain (folded into the next product), for a batch of
  // token groups: the server computes centered and var + eps; the client
  // returns 1/sqrt for every slot in one device batch; the server multiplies
  // (T123.cpp:1168-1181).  Output at limbs(x) - 2.
  std::vector<Ciphertext> layernorm(const std::vector<Ciphertext>& xs, const std::vector<int>& active) {
    const int lx = xs[0]->limbs();
    std::vector<double> invd(s.PW, 0.0);
    for (int f = 0; f < s.D; ++f) invd[f] = 1.0 / s.D;
    std::vector<Ciphertext> centered, sqs;
    const auto sums = feature_sums(xs);
    std::vector<Ciphertext> prods;
    for (size_t i = 0; i < xs.size(); ++i) {
      ++count["ct_plain"];
      prods.push_back(cc.EvalMult(sums[i], feature_plain(1, invd, lx)));
    }
    const auto means = rs_many(prods);
    const auto xr = reduce_many(xs, std::vector<int>(xs.size(), lx - 1));
    for (size_t i = 0; i < xs.size(); ++i) centered.push_back(cc.EvalSub(xr[i], means[i]));
    // the variance is only decrypted: square at 4 limbs, sum and scale at 3,
    // decrypt at 2
    const auto low = reduce_many(centered, std::vector<int>(centered.size(), 4), true);
    count["ct_ct"] += (long)xs.size();
    sqs = cc.RescaleBatch(cc.EvalMultBatch(low, low));
    prods.clear();
    for (const auto& sq : feature_sums(sqs)) {
      ++count["ct_plain"];
      prods.push_back(cc.EvalMult(sq, feature_plain(1, invd, sq->limbs())));
    }
    std::vector<Ciphertext> var;
    for (const auto& v : rs_many(prods)) var.push_back(cc.EvalAdd(v, 1e-5));
    const int M = (int)xs.size();
    double* dv = dbuf((size_t)M * slots());
    client_decrypt(var, dv);
    blk::invsqrt_kernel<<<(M * slots() + blk::kThreads - 1) / blk::kThreads, blk::kThreads, 0, C.stream>>>(
        dv, M * slots());
    const auto inv = client_encrypt(dv, M, lx - 1);
    C.release(dv);
    count["client_round_trips"] += M;
    for (int a : active) count["client_logical_instances"] += a;
    return mul_ct_rs_batch(centered, inv);
  }

  // lane shifts of several inputs (xs[i] for every delta in needs[i], 0 ->
  // xs[i] brought to targets[i] limbs): inputs with the same deltas and level
  // share one hoisted batch (each rotation key read once for all of them),
  // then batched masks, adds and rescales (blk::lane_shift_set)
  std::vector<std::map<int, Ciphertext>> lane_shifts_batch(const std::vector<Ciphertext>& xs,
                                                           const std::vector<std::vector<int>>& needs,
                                                           const std::vector<int>& targets) {
    std::vector<std::map<int, Ciphertext>> out(xs.size());
    std::map<std::pair<std::vector<int>, int>, std::vector<size_t>> bins;  // (deltas, limbs) -> inputs
    for (size_t i = 0; i < xs.size(); ++i) {
      std::vector<int> ds;
      for (int d : needs[i]) {
        if (d == 0)
          out[i][0] = reduce_to(xs[i], targets[i]);
        else
          ds.push_back(d);
      }
      std::sort(ds.begin(), ds.end());
      ds.erase(std::unique(ds.begin(), ds.end()), ds.end());
      if (!ds.empty()) bins[{ds, xs[i]->limbs()}].push_back(i);
    }
    const blk::LaneMask mask = [this](int d, bool lower, int limbs) { return lane_plain(d, lower, limbs); };
    for (const auto& bin : bins) {
      const std::vector<int>& ds = bin.first.first;
      const std::vector<size_t>& mem = bin.second;
      std::vector<Ciphertext> in;
      for (size_t i : mem) in.push_back(xs[i]);
      count["rotations"] += 2 * (long)ds.size() * (long)mem.size();
      count["ct_plain"] += 2 * (long)ds.size() * (long)mem.size();
      const auto sh = blk::lane_shift_set(cc, in, ds, s.B, mask);
      for (size_t g = 0; g < mem.size(); ++g)
        for (size_t k = 0; k < ds.size(); ++k) out[mem[g]][ds[k]] = sh[g][k];
    }
    return out;
  }


  // products a[i] * b[i], rescaled, batched
  std::vector<Ciphertext> mul_ct_rs_batch(const std::vector<Ciphertext>& a, const std::vector<Ciphertext>& b) {
    count["ct_ct"] += (long)a.size();
    return cc.RescaleBatch(cc.EvalMultBatch(a, b));
  }

  // per head, the sum of its HD features at the head's first feature (and
  // window sums elsewhere): a base-8 ladder of hoisted rotation sums (two
  // steps for 64 features; at 2 limbs a step's ModUp and ModDown cost more
  // than its seven key products)
  static constexpr int kHeadRadix = 8;
  std::vector<Ciphertext> head_window_sums(const std::vector<Ciphertext>& h) {
    for (long step = 1; step < s.HD; step *= kHeadRadix)
      for (int m = 1; m < kHeadRadix && step * m < s.HD; ++m) count["rotations"] += (long)h.size();
    return cc.WindowSumBatch(h, s.HD, s.B, kHeadRadix);
  }

  // weight id -> (device matrix, out_dim, in_dim, leading dimension)
  void weight_view(int id, const double*& W, int& out_dim, int& in_dim, int& ld) const {
    const int D = s.D;
    if (id == kHeadLinear) {
      W = d_head;
      out_dim = in_dim = ld = D;
      return;
    }
    if (id < 3) {
      W = d_qkv + (size_t)id * D * D;
      out_dim = D;
      in_dim = D;
      ld = D;
    } else if (id == 3) {
      W = d_proj;
      out_dim = D;
      in_dim = D;
      ld = D;
    } else if (id < 4 + nfc) {
      const int c = id - 4;
      W = d_fc + (size_t)c * s.PW * D;
      out_dim = std::min(s.PW, s.MLP - c * s.PW);
      in_dim = D;
      ld = D;
    } else {
      const int c = id - 4 - nfc;
      W = d_proj2 + (size_t)c * s.PW;
      out_dim = D;
      in_dim = std::min(s.PW, s.MLP - c * s.PW);
      ld = s.MLP;
    }
  }

  // all n1 * n2 diagonals of weight `id`, encoded once per use level on the
  // device and kept (the reference encodes them on the host, T123.cpp:1005-1059)
  const Diag& diagonals(int id, int limbs) {
    auto key = std::make_pair(id, limbs);
    auto it = diags.find(key);
    if (it != diags.end()) {
      ++count["diagonal_cache_hits"];
      return it->second;
    }
    ++count["diagonal_cache_misses"];
    const double t0 = blk::now_s();
    const double* W;
    int od, id_, ld;
    weight_view(id, W, od, id_, ld);
    Diag dg;
    dg.limbs = limbs;
    dg.scale = S(limbs);
    dg.data = blk::encode_diagonals(C, W, od, id_, ld, s.PW, s.B, s.n1, s.n2, limbs, dg.scale);
    seconds["diagonal_encode"] += blk::now_s() - t0;
    return diags.emplace(key, dg).first->second;
  }

  std::vector<Ciphertext> babies_of(const Ciphertext& x) { return babies_of_batch({x})[0]; }
  // baby steps x, rot(x, B j) for j < n1 of every input, one hoisted batch
  // (each rotation key read once for all inputs)
  std::vector<std::vector<Ciphertext>> babies_of_batch(const std::vector<Ciphertext>& xs) {
    std::vector<int> idx;
    for (int j = 1; j < s.n1; ++j) idx.push_back(s.B * j);
    auto r = cc.EvalFastRotationBatch(xs, idx);
    count["rotations"] += (long)idx.size() * (long)xs.size();
    std::vector<std::vector<Ciphertext>> out(xs.size());
    for (size_t i = 0; i < xs.size(); ++i) {
      out[i].push_back(xs[i]);
      out[i].insert(out[i].end(), r[i].begin(), r[i].end());
    }
    return out;
  }

  // x_q W^T for weight `id` and every token group q from their baby-step
  // rotations (T123.cpp:1264-1295): fused diagonal x baby-step inner sums,
  // then the giant steps of each group as one rotation sum (one ModDown)
  std::vector<Ciphertext> bsgs_groups(const std::vector<std::vector<Ciphertext>>& babies, int id) {
    return bsgs_sum_groups({babies}, {id});
  }
  // sum_t x_{t,q} W_t^T for every token group q: the inner sums of all terms
  // t (weights ids[t] on baby steps babies[t][q]) accumulate into one set of
  // giant-step inputs, so the giant-step rotations run once per group for
  // the whole sum (rotation is linear)
  std::vector<Ciphertext> bsgs_sum_groups(const std::vector<std::vector<std::vector<Ciphertext>>>& babies,
                                          const std::vector<int>& ids) {
    const int nt = (int)babies.size();
    const int G = nt ? (int)babies[0].size() : 0;
    if (!G) return std::vector<Ciphertext>(G);
    const int limbs = babies[0][0][0]->limbs();
    std::vector<blk::DiagRef> dgs;
    for (int t = 0; t < nt; ++t) {
      const Diag& dg = diagonals(ids[t], limbs);
      dgs.push_back({dg.data, dg.limbs, dg.scale});
      count["matrix_products"] += G;
      count["ct_plain"] += (long)G * s.n1 * s.n2;
    }
    count["rotations"] += (long)G * (s.n2 - 1);
    return blk::bsgs_products(cc, C, babies, dgs, s.n1, s.n2, s.B);
  }
  Ciphertext bsgs(const std::vector<Ciphertext>& baby, int id) { return bsgs_groups({baby}, id)[0]; }

  static constexpr int kHeadLinear = 100;
  // evaluation state between the stages of one forward
  std::vector<Ciphertext> st_x, st_q, st_k, st_v, st_ctx, st_r1, st_mlp;
  double* st_prob = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  double t_start = 0.0, t_stage = 0.0, alloc_s0 = 0.0;
  long alloc_n0 = 0;
  void stamp(const char* k) {
    cc.Synchronize();
    const double n = blk::now_s();
    seconds[k] += n - t_stage;
    t_stage = n;
  }
  // every causal alignment (qg, kg, d) of the given (qg, kg) tiles
  std::vector<blk::TileTag> alignments(const std::vector<std::pair<int, int>>& pairs) const;
  static std::vector<blk::TileTag> tags_of(int kg, const std::vector<blk::TileTag>& tiles);
  void shard_inputs(const double* x, int T);
  // parts: bit 0 Q, bit 1 K, bit 2 V
  void shard_qkv(const std::vector<int>& groups, int parts);
  void shard_scores(const std::vector<blk::TileTag>& tiles, double* d_scores);
  void shard_softmax(const double* d_scores);
  void shard_context(const std::vector<blk::TileTag>& tiles);
  void shard_mlp(const std::vector<int>& groups, int c0, int c1);
  void shard_finish(const std::vector<int>& groups, double* y);
  void shard_output(const std::vector<int>& groups, double* y);
  void forward(const double* x, int T, double* y);
  double head_forward(const double* x_last);
  std::vector<int> rotation_indices() const;
};

std::vector<int> ckks_block::rotation_indices() const {
  const int slots = s.PW * s.B;
  auto canon = [&](long k) {
    long r = k % slots;
    if (r < 0) r += slots;
    if (r > slots / 2) r -= slots;
    return (int)r;
  };
  std::vector<int> v;
  for (int j = 1; j < s.n1; ++j) v.push_back(canon((long)s.B * j));
  for (int g = 1; g < s.n2; ++g) v.push_back(canon((long)s.B * s.n1 * g));
  for (long step = 1; step < s.PW; step *= 4)  // AccumulateSum ladder (T123.cpp:444-453)
    for (int m = 1; m < 4 && step * m < s.PW; ++m) v.push_back(canon((long)s.B * step * m));
  for (int d = 1; d < s.B; ++d) {
    v.push_back(canon(d));
    v.push_back(canon(d - s.B));
    v.push_back(canon((long)d * s.B));  // packing alignment d to feature h*HD - d (baby keys when n1 >= B)
  }
  for (long step = 1; step < s.HD; step *= kHeadRadix)  // head window sums: base-8 ladder over HD features
    for (int m = 1; m < kHeadRadix && step * m < s.HD; ++m) v.push_back(canon((long)s.B * step * m));
  std::sort(v.begin(), v.end());
  v.erase(std::unique(v.begin(), v.end()), v.end());
  v.erase(std::remove(v.begin(), v.end(), 0), v.end());
  return v;
}

// ---- stages of one block evaluation ---------------------------------------
// A forward is shard_inputs, shard_qkv(groups), shard_scores(tiles),
// shard_softmax, shard_context(tiles), shard_output(groups).  Run on every
// unit they give one block on one device; run on a subset of the token
// groups / (query group, key group) tiles by each rank, with the Q/K/V and
// partial-context ciphertexts and the score matrix exchanged between the
// stages, they shard one block over several devices.

std::vector<blk::TileTag> ckks_block::alignments(const std::vector<std::pair<int, int>>& pairs) const {
  std::vector<blk::TileTag> t;
  for (const auto& pr : pairs)
    for (int d : blk::active_shifts(s.T, s.B, pr.first, pr.second)) t.push_back({pr.first, pr.second, d});
  return t;
}

std::vector<blk::TileTag> ckks_block::tags_of(int kg, const std::vector<blk::TileTag>& tiles) {
  std::vector<blk::TileTag> t;
  for (const auto& tg : tiles)
    if (tg.kg == kg) t.push_back(tg);
  return t;
}

void ckks_block::shard_inputs(const double* x, int T) {
  C.prof.section = "encrypt_inputs";
  if (T != s.T) throw ckks::Error(CKKS_EARG, "token count differs from the block's");
  const int G = s.groups, D = s.D, SL = slots();
  const int nb = (SL + blk::kThreads - 1) / blk::kThreads;
  count.clear();
  seconds.clear();
  client_seconds = 0.0;
  alloc_s0 = C.alloc_seconds;
  alloc_n0 = C.alloc_calls;
  t_start = t_stage = blk::now_s();
  st_x.assign(G, Ciphertext());
  st_q.assign(G, Ciphertext());
  st_k.assign(G, Ciphertext());
  st_v.assign(G, Ciphertext());
  st_ctx.assign(G, Ciphertext());
  st_r1.assign(G, Ciphertext());
  st_mlp.assign(G, Ciphertext());
  // client: pack and encrypt the embeddings (T123.cpp:1642-1661)
  double* dx = dbuf((size_t)T * D);
  C.stage_upload(dx, x, sizeof(double) * T * D, C.stream);
  double* dvals = dbuf((size_t)G * SL);
  blk::pack_kernel<<<dim3(nb, G), blk::kThreads, 0, C.stream>>>(dx, dvals, T, D, s.B, SL);
  st_x = client_encrypt(dvals, G, LX);
  C.release(dvals);
  C.release(dx);
  stamp("encrypt_inputs");
  // device-timed span from encrypted inputs resident to encrypted outputs
  // resident (client refreshes included: the stream waits on them)
  if (!ev_in) CKKS_CUDA(cudaEventCreate(&ev_in));
  if (!ev_out) CKKS_CUDA(cudaEventCreate(&ev_out));
  CKKS_CUDA(cudaEventRecord(ev_in, C.stream));
}

// LN1 + QKV of the given token groups
void ckks_block::shard_qkv(const std::vector<int>& groups, int parts) {
  C.prof.section = "ln1_qkv";
  if (groups.empty() || !(parts & 7)) return;
  std::vector<Ciphertext> xs;
  std::vector<int> act;
  for (int g : groups) {
    if (g < 0 || g >= s.groups || !st_x[g]) throw ckks::Error(CKKS_ESTATE, "inputs not encrypted");
    xs.push_back(st_x[g]);
    act.push_back(s.count(g));
  }
  const auto nrm = layernorm(xs, act);
  const auto babies = babies_of_batch(nrm);
  std::vector<Ciphertext>* dst[3] = {&st_q, &st_k, &st_v};
  for (int w = 0; w < 3; ++w) {
    if (!(parts & (1 << w))) continue;
    const auto r = bsgs_groups(babies, w);
    for (size_t i = 0; i < groups.size(); ++i) (*dst[w])[groups[i]] = r[i];
  }
  stamp("ln1_qkv");
}

// scores of the given (query group, key group) tiles written into d_scores
// ([q][head][k] doubles on the device): server products and head-window sums,
// the client decrypts and gathers them on the device
void ckks_block::shard_scores(const std::vector<blk::TileTag>& tiles, double* d_scores) {
  C.prof.section = "scores";
  const int T = s.T, H = s.H, HD = s.HD, B = s.B, SL = slots();
  const double inv_sqrt_hd = 1.0 / std::sqrt((double)HD);
  // queries brought to the score level once per query group (a FLEXIBLEAUTO
  // level reduction is a scaled multiply and a rescale)
  std::map<int, Ciphertext> qr;
  // scores are only decrypted: keys shifted from 4 limbs, products of 3-limb
  // operands, head sums and decryption at 2; the key lane shifts of all key
  // groups in one batch
  std::vector<int> kgs, lks_of(s.groups, 0);
  std::vector<Ciphertext> kx;
  std::vector<std::vector<int>> kneed;
  std::vector<int> ktarget;
  for (int kg = 0; kg < s.groups; ++kg) {
    const auto tags = tags_of(kg, tiles);
    if (tags.empty()) continue;
    if (!st_k[kg]) throw ckks::Error(CKKS_ESTATE, "key group not evaluated");
    std::vector<int> need;
    for (const auto& tg : tags) {
      if (!st_q[tg.qg]) throw ckks::Error(CKKS_ESTATE, "query group not evaluated");
      if (std::find(need.begin(), need.end(), tg.d) == need.end()) need.push_back(tg.d);
    }
    lks_of[kg] = std::min(st_q[tags[0].qg]->limbs() - 1, 3);
    kgs.push_back(kg);
    kx.push_back(lower(st_k[kg], lks_of[kg] + 1));
    kneed.push_back(need);
    ktarget.push_back(lks_of[kg]);
  }
  auto kshift = lane_shifts_batch(kx, kneed, ktarget);
  kx.clear();
  for (size_t ki = 0; ki < kgs.size(); ++ki) {
    const int kg = kgs[ki];
    const auto tags = tags_of(kg, tiles);
    const int lks = lks_of[kg];
    auto ks = std::move(kshift[ki]);
    count["cached_key_lane_shifts"] += (long)ks.size() - (ks.count(0) ? 1 : 0);
    std::vector<Ciphertext> qa, kb;
    for (const auto& tg : tags) {
      auto it = qr.find(tg.qg);
      if (it == qr.end()) it = qr.emplace(tg.qg, reduce_to(st_q[tg.qg], lks)).first;
      qa.push_back(it->second);
      kb.push_back(ks[tg.d]);
    }
    const auto sums = head_window_sums(mul_ct_rs_batch(qa, kb));
    // isolate each head's score at its causal lanes (scaled by 1/sqrt(HD)),
    // move alignment d to feature h*HD - d (a rotation by d*B: the baby-step
    // keys) and pack every alignment of a (query group, key group) tile into
    // one ciphertext: one rotation sum, one client decryption per tile
    // (T123.cpp:803-833); distinct d < B <= HD never share a feature
    const int M = (int)sums.size();
    std::vector<Ciphertext> iso(M);
    {
      std::vector<Plaintext> pl;
      for (int i = 0; i < M; ++i) pl.push_back(score_plain(tags[i], sums[i]->limbs(), inv_sqrt_hd));
      iso = cc.EvalMultPlainBatch(sums, pl);
    }
    count["ct_plain"] += M;
    iso = cc.RescaleBatch(iso);
    std::vector<int> qgs;
    for (const auto& tg : tags)
      if (std::find(qgs.begin(), qgs.end(), tg.qg) == qgs.end()) qgs.push_back(tg.qg);
    std::vector<Ciphertext> packed;
    std::vector<blk::ScoreTag> st;
    for (size_t v = 0; v < qgs.size(); ++v) {
      std::vector<Ciphertext> parts;
      std::vector<int> rot;
      for (int i = 0; i < M; ++i)
        if (tags[i].qg == qgs[v]) {
          parts.push_back(iso[i]);
          rot.push_back(tags[i].d * B);
          st.push_back({tags[i].qg, kg, tags[i].d, (int)v});
        }
      count["rotations"] += (long)parts.size();
      packed.push_back(cc.EvalRotateSum(parts, rot));
    }
    const int P = (int)packed.size();
    double* dv = dbuf((size_t)P * SL);
    client_decrypt(packed, dv);
    blk::ScoreTag* dt = (blk::ScoreTag*)C.alloc(sizeof(blk::ScoreTag) * st.size());
    C.stage_upload(dt, st.data(), sizeof(blk::ScoreTag) * st.size(), C.stream);
    blk::score_gather_kernel<<<dim3((unsigned)st.size(), H), 32 * ((B + 31) / 32), 0, C.stream>>>(
        dv, dt, T, H, HD, B, s.PW, SL, d_scores);
    CKKS_CUDA(cudaGetLastError());
    C.release(dt);
    C.release(dv);
    count["score_tile_decryptions"] += P;
    count["client_round_trips"] += P;
  }
  stamp("scores");
}

// client: exact causal softmax in float64 (T123.cpp:629-665)
void ckks_block::shard_softmax(const double* d_scores) {
  C.prof.section = "softmax";
  const int T = s.T, H = s.H;
  if (!st_prob) st_prob = (double*)C.alloc(sizeof(double) * (size_t)T * H * T);
  int* bad = (int*)C.alloc(sizeof(int));
  CKKS_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), C.stream));
  blk::softmax_kernel<<<(T * H + blk::kThreads - 1) / blk::kThreads, blk::kThreads, 0, C.stream>>>(d_scores, st_prob,
                                                                                                     T, H, bad);
  int hbad = 0;
  CKKS_CUDA(cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, C.stream));
  CKKS_CUDA(cudaStreamSynchronize(C.stream));
  C.release(bad);
  if (hbad) throw ckks::Error(CKKS_ESTATE, "missing/non-finite causal attention score");
  count["client_logical_instances"] += (long)H * T * (T + 1) / 2;
}

// context of the given tiles: client weight tiles x shifted values, summed
// into per-query-group partial contexts (T123.cpp:838-860).  The products of
// a query group are only ever summed, so they are added as degree-2
// ciphertexts and relinearised once (EvalMultSum), then rescaled.
void ckks_block::shard_context(const std::vector<blk::TileTag>& tiles) {
  C.prof.section = "context";
  const int T = s.T, H = s.H, HD = s.HD, D = s.D, B = s.B, SL = slots();
  const int nb = (SL + blk::kThreads - 1) / blk::kThreads;
  if (!st_prob) throw ckks::Error(CKKS_ESTATE, "softmax not evaluated");
  std::vector<std::vector<Ciphertext>> lhs(s.groups), rhs(s.groups);  // per query group
  // the value lane shifts of all key groups in one batch
  std::vector<int> kgs;
  std::vector<Ciphertext> vx;
  std::vector<std::vector<int>> vneed;
  std::vector<int> vtarget;
  for (int kg = 0; kg < s.groups; ++kg) {
    const auto tags = tags_of(kg, tiles);
    if (tags.empty()) continue;
    if (!st_v[kg]) throw ckks::Error(CKKS_ESTATE, "value group not evaluated");
    std::vector<int> need;
    for (const auto& tg : tags)
      if (std::find(need.begin(), need.end(), tg.d) == need.end()) need.push_back(tg.d);
    kgs.push_back(kg);
    vx.push_back(st_v[kg]);
    vneed.push_back(need);
    vtarget.push_back(st_v[kg]->limbs() - 1);
  }
  auto vshift = lane_shifts_batch(vx, vneed, vtarget);
  vx.clear();
  for (size_t ki = 0; ki < kgs.size(); ++ki) {
    const int kg = kgs[ki];
    const auto tags = tags_of(kg, tiles);
    const int lk = st_v[kg]->limbs() - 1;
    auto vs = std::move(vshift[ki]);
    count["cached_value_lane_shifts"] += (long)vs.size() - (vs.count(0) ? 1 : 0);
    const int M = (int)tags.size();
    double* dv = dbuf((size_t)M * SL);
    blk::TileTag* dt = (blk::TileTag*)C.alloc(sizeof(blk::TileTag) * M);
    C.stage_upload(dt, tags.data(), sizeof(blk::TileTag) * M, C.stream);
    blk::weight_tile_kernel<<<dim3(nb, M), blk::kThreads, 0, C.stream>>>(st_prob, dt, T, H, HD, D, B, SL, dv);
    CKKS_CUDA(cudaGetLastError());
    const auto wa = client_encrypt(dv, M, lk);
    C.release(dt);
    C.release(dv);
    count["weight_tile_encryptions"] += M;
    count["client_round_trips"] += M;
    for (int i = 0; i < M; ++i) {
      lhs[tags[i].qg].push_back(wa[i]);
      rhs[tags[i].qg].push_back(vs[tags[i].d]);
    }
  }
  std::vector<Ciphertext> sums;
  std::vector<int> qgs;
  for (int qg = 0; qg < s.groups; ++qg) {
    if (lhs[qg].empty()) continue;
    count["ct_ct"] += (long)lhs[qg].size();
    sums.push_back(cc.EvalMultSum(lhs[qg], rhs[qg]));
    qgs.push_back(qg);
  }
  sums = rs_many(sums);
  for (size_t i = 0; i < qgs.size(); ++i) {
    const int qg = qgs[i];
    st_ctx[qg] = st_ctx[qg] ? add(st_ctx[qg], sums[i]) : sums[i];
  }
  stamp("context");
}

// O projection, residual, LN2, MLP of the given groups, then the client
// decrypts them into their rows of y ([T, D] host)
// O projection, residual, LN2 and the MLP chunks [c0, c1) of the given
// groups: the residual is kept in st_r1, the chunks' sum in st_mlp (the MLP
// of a group may be split over ranks and its partial sums added with EvalAdd,
// shard_layout.py stage 2)
void ckks_block::shard_mlp(const std::vector<int>& groups, int c0, int c1) {
  C.prof.section = "oproj_ln2_mlp";
  if (groups.empty()) return;
  c0 = std::max(0, c0);
  c1 = std::min(nfc, c1);
  const int B = s.B, PW = s.PW, SL = slots();
  const int nb = (SL + blk::kThreads - 1) / blk::kThreads;
  const int G = (int)groups.size();
  std::vector<Ciphertext> ctxs;
  std::vector<int> act;
  for (int g : groups) {
    if (!st_ctx[g] || !st_x[g]) throw ckks::Error(CKKS_ESTATE, "context of the group not complete");
    ctxs.push_back(st_ctx[g]);
    act.push_back(s.count(g));
  }
  auto ob = babies_of_batch(ctxs);
  const auto o = bsgs_groups(ob, 3);
  ob.clear();
  std::vector<Ciphertext> r1, xg;
  std::vector<int> lg;
  for (int i = 0; i < G; ++i) {
    xg.push_back(st_x[groups[i]]);
    lg.push_back(o[i]->limbs());
  }
  xg = reduce_many(xg, lg);
  for (int i = 0; i < G; ++i) r1.push_back(add(xg[i], o[i]));
  for (int i = 0; i < G; ++i) st_r1[groups[i]] = r1[i];
  if (c0 >= c1) {
    for (int g : groups) st_mlp[g] = Ciphertext();
    stamp("oproj_ln2_mlp");
    return;
  }
  const int nc = c1 - c0;
  const auto n2 = layernorm(r1, act);
  auto fb = babies_of_batch(n2);
  std::vector<std::vector<Ciphertext>> hc(nc);  // [chunk][group]
  for (int c = 0; c < nc; ++c) hc[c] = bsgs_groups(fb, 4 + c0 + c);
  fb.clear();
  // client: exact tanh-GELU on the active lanes of every group and chunk, one
  // device batch (T123.cpp:540-568); item i * nc + c
  const int gelu_limbs = 3;
  std::vector<Ciphertext> flat;
  for (int i = 0; i < G; ++i)
    for (int c = 0; c < nc; ++c) flat.push_back(hc[c][i]);
  hc.clear();
  double* dv = dbuf((size_t)G * nc * SL);
  client_decrypt(flat, dv);
  for (int i = 0; i < G; ++i)
    for (int c = 0; c < nc; ++c) {
      const int odim = std::min(PW, s.MLP - (c0 + c) * PW);
      double* v = dv + ((size_t)i * nc + c) * SL;
      blk::gelu_kernel<<<dim3(nb, 1), blk::kThreads, 0, C.stream>>>(v, v, B, odim, act[i], SL);
      count["client_logical_instances"] += (long)odim * act[i];
    }
  CKKS_CUDA(cudaGetLastError());
  const auto ge = client_encrypt(dv, G * nc, gelu_limbs);
  C.release(dv);
  count["client_round_trips"] += (long)G * nc;
  // down projection: the chunks' products summed before one set of giant
  // steps per group
  auto gb = babies_of_batch(ge);  // item i * nc + c
  std::vector<std::vector<std::vector<Ciphertext>>> db(nc);
  std::vector<int> dids;
  for (int c = 0; c < nc; ++c) {
    for (int i = 0; i < G; ++i) db[c].push_back(std::move(gb[(size_t)i * nc + c]));
    dids.push_back(4 + nfc + c0 + c);
  }
  const std::vector<Ciphertext> mlp = bsgs_sum_groups(db, dids);
  for (int i = 0; i < G; ++i) st_mlp[groups[i]] = mlp[i];
  stamp("oproj_ln2_mlp");
}

// block output r1 + MLP of the given groups, decrypted by the client into
// their rows of y ([T, D] host)
void ckks_block::shard_finish(const std::vector<int>& groups, double* y) {
  C.prof.section = "decrypt_outputs";
  if (groups.empty()) return;
  const int T = s.T, D = s.D, B = s.B, SL = slots();
  const int nb = (SL + blk::kThreads - 1) / blk::kThreads;
  const int G = (int)groups.size();
  std::vector<Ciphertext> out(G), rg;
  std::vector<int> lg;
  for (int i = 0; i < G; ++i) {
    const int g = groups[i];
    if (!st_r1[g] || !st_mlp[g]) throw ckks::Error(CKKS_ESTATE, "MLP of the group not complete");
    rg.push_back(st_r1[g]);
    lg.push_back(st_mlp[g]->limbs());
  }
  rg = reduce_many(rg, lg);
  for (int i = 0; i < G; ++i) out[i] = add(rg[i], st_mlp[groups[i]]);
  CKKS_CUDA(cudaEventRecord(ev_out, C.stream));
  // client: decrypt and unpack (T123.cpp:1675-1694)
  {
    double* dv = dbuf((size_t)G * SL);
    client_decrypt(out, dv);
    double* dy = dbuf((size_t)T * D);
    for (int i = 0; i < G; ++i) {
      const int g = groups[i];
      blk::unpack_kernel<<<dim3(nb, 1), blk::kThreads, 0, C.stream>>>(dv + (size_t)i * SL, dy, T, D, B, SL, g);
      const int r0 = g * B, r1_ = std::min(T, (g + 1) * B);
      CKKS_CUDA(cudaMemcpyAsync(y + (size_t)r0 * D, dy + (size_t)r0 * D, sizeof(double) * (size_t)(r1_ - r0) * D,
                                cudaMemcpyDeviceToHost, C.stream));
    }
    CKKS_CUDA(cudaGetLastError());
    CKKS_CUDA(cudaStreamSynchronize(C.stream));
    C.release(dv);
    C.release(dy);
    count["output_limbs"] = out[0]->limbs();
  }
  stamp("decrypt_outputs");
  seconds["total"] = blk::now_s() - t_start;
  seconds["client"] = client_seconds;
  seconds["alloc_host"] = C.alloc_seconds - alloc_s0;
  count["alloc_calls"] = C.alloc_calls - alloc_n0;
  count["input_limbs"] = LX;
  float ms = 0.f;
  CKKS_CUDA(cudaEventElapsedTime(&ms, ev_in, ev_out));
  seconds["evaluate_events"] = ms / 1e3;
}

void ckks_block::shard_output(const std::vector<int>& groups, double* y) {
  shard_mlp(groups, 0, nfc);
  shard_finish(groups, y);
}

void ckks_block::forward(const double* x, int T, double* y) {
  shard_inputs(x, T);
  std::vector<int> groups(s.groups);
  for (int g = 0; g < s.groups; ++g) groups[g] = g;
  std::vector<std::pair<int, int>> pairs;
  for (int kg = 0; kg < s.groups; ++kg)
    for (int qg = kg; qg < s.groups; ++qg) pairs.push_back({qg, kg});
  shard_qkv(groups, 7);
  const auto tiles = alignments(pairs);
  double* d_scores = dbuf((size_t)T * s.H * T);
  CKKS_CUDA(cudaMemsetAsync(d_scores, 0xFF, sizeof(double) * T * s.H * T, C.stream));  // NaN = missing
  shard_scores(tiles, d_scores);
  shard_softmax(d_scores);
  C.release(d_scores);
  shard_context(tiles);
  shard_output(groups, y);
}

// Classifier head on the last token's hidden state
// (12blocks_head_cpudiagcache_t123_v3.cpp:573-609, multiblock/manual.py:52-80):
// final LN -> head linear (BSGS) -> SiLU client boundary -> head LN -> dot
// with (readout_N - readout_A).  The token sits in lane 0 of one ciphertext;
// both LN gains are folded into the next linear map.  Levels: the input is
// encrypted at 5 limbs (LN 2, linear 1, decryption at 2), the SiLU output
// at 5 (LN 2, readout 1, decryption at 2).
double ckks_block::head_forward(const double* x_last) {
  C.prof.section = "head";
  const int D = s.D, B = s.B, SL = slots();
  const int nb = (SL + blk::kThreads - 1) / blk::kThreads;
  constexpr int kHeadLimbs = 5;
  if (C.L < kHeadLimbs) throw ckks::Error(CKKS_ELEVEL, "the head needs 5 Q limbs");
  const double t_start = blk::now_s();
  double* dx = dbuf(D);
  C.stage_upload(dx, x_last, sizeof(double) * D, C.stream);
  double* dv = dbuf(SL);
  blk::pack_kernel<<<dim3(nb, 1), blk::kThreads, 0, C.stream>>>(dx, dv, 1, D, B, SL);
  const auto xin = client_encrypt(dv, 1, kHeadLimbs);
  const std::vector<int> one{1};
  const Ciphertext fl = layernorm(xin, one)[0];
  const Ciphertext lin = bsgs(babies_of(fl), kHeadLinear);
  // client: SiLU on lane 0 (12blocks_head..._t123_v3.cpp:740-755)
  client_decrypt({lin}, dv);
  blk::silu_kernel<<<nb, blk::kThreads, 0, C.stream>>>(dv, dv, B, D, SL);
  CKKS_CUDA(cudaGetLastError());
  const auto act = client_encrypt(dv, 1, kHeadLimbs);
  count["client_round_trips"] += 1;
  count["client_logical_instances"] += 1;
  const Ciphertext hl = layernorm(act, one)[0];
  const Ciphertext margin = feature_sum(mul_pt_rs(hl, feature_plain(2, readout, hl->limbs())));
  client_decrypt({margin}, dv);
  double m = 0.0;
  CKKS_CUDA(cudaMemcpyAsync(&m, dv, sizeof(double), cudaMemcpyDeviceToHost, C.stream));
  CKKS_CUDA(cudaStreamSynchronize(C.stream));
  C.release(dv);
  C.release(dx);
  seconds["head_total"] = blk::now_s() - t_start;
  return m;
}

void ckks::block_orphan(ckks_block* b) { b->release_device(); }

namespace {
template <typename F>
int bguard(F&& f) {
  try {
    f();
    return CKKS_OK;
  } catch (const ckks::Error& e) {
    ckks::set_last_error(e.what());
    return e.code;
  } catch (const ckks_b200::Error& e) {
    ckks::set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    ckks::set_last_error(e.what());
    return CKKS_EARG;
  }
}

double* upload_matrix(const std::vector<double>& v) {
  double* d = nullptr;
  CKKS_CUDA(cudaMalloc(&d, sizeof(double) * v.size()));
  CKKS_CUDA(cudaMemcpy(d, v.data(), sizeof(double) * v.size(), cudaMemcpyHostToDevice));
  return d;
}
}  // namespace

extern "C" {

int ckks_block_create(ckks_ctx* ctx, const double* ln1, const double* attn_qkv, const double* attn_proj,
                      const double* ln2, const double* mlp_fc, const double* mlp_proj, int d_model, int heads,
                      int mlp_dim, int tokens, ckks_block** out) {
  return bguard([&] {
    if (!ctx || !ctx->c || !out) throw ckks::Error(CKKS_EARG, "null argument");
    if (!ln1 || !attn_qkv || !attn_proj || !ln2 || !mlp_fc || !mlp_proj) throw ckks::Error(CKKS_EARG, "null weight");
    ckks::Context& C = *ctx->c;
    blk::Shape s;
    s.D = d_model;
    s.H = heads;
    s.MLP = mlp_dim;
    s.T = tokens;
    if (d_model <= 0 || heads <= 0 || d_model % heads || mlp_dim <= 0 || tokens <= 0)
      throw ckks::Error(CKKS_EARG, "bad block shape");
    s.HD = d_model / heads;
    s.B = 32;
    s.PW = C.N / 2 / s.B;
    if (s.PW < d_model || (s.HD & (s.HD - 1)) || s.B > s.HD)
      throw ckks::Error(CKKS_EARG, "shape does not fit the slot layout");
    s.n1 = 32;
    while (s.n1 * s.n1 > s.PW) s.n1 >>= 1;
    s.n2 = s.PW / s.n1;
    if (s.n1 > blk::kMaxBaby) throw ckks::Error(CKKS_EARG, "too many baby steps");
    s.groups = (tokens + s.B - 1) / s.B;
    auto* b = new ckks_block(ctx, s);
    try {
      b->nfc = (mlp_dim + s.PW - 1) / s.PW;
      const int D = d_model;
      std::vector<double> qkv((size_t)3 * D * D), fc((size_t)mlp_dim * D);
      for (int r = 0; r < 3 * D; ++r)
        for (int c = 0; c < D; ++c) qkv[(size_t)r * D + c] = attn_qkv[(size_t)r * D + c] * ln1[c];
      for (int r = 0; r < mlp_dim; ++r)
        for (int c = 0; c < D; ++c) fc[(size_t)r * D + c] = mlp_fc[(size_t)r * D + c] * ln2[c];
      b->d_qkv = upload_matrix(qkv);
      b->d_proj = upload_matrix(std::vector<double>(attn_proj, attn_proj + (size_t)D * D));
      b->d_fc = upload_matrix(fc);
      b->d_proj2 = upload_matrix(std::vector<double>(mlp_proj, mlp_proj + (size_t)D * mlp_dim));
      if (C.L < b->LX) throw ckks::Error(CKKS_ELEVEL, "the block needs 11 Q limbs");
    } catch (...) {
      delete b;
      throw;
    }
    {
      std::lock_guard<std::mutex> lk(ctx->mu);
      ctx->blocks.insert(b);
    }
    *out = b;
  });
}

int ckks_head_create(ckks_ctx* ctx, const double* final_ln, const double* head_linear, const double* head_ln,
                     const double* readout, int d_model, ckks_block** out) {
  return bguard([&] {
    if (!ctx || !ctx->c || !out) throw ckks::Error(CKKS_EARG, "null argument");
    if (!final_ln || !head_linear || !head_ln || !readout) throw ckks::Error(CKKS_EARG, "null weight");
    ckks::Context& C = *ctx->c;
    blk::Shape s;
    s.D = d_model;
    s.H = 1;
    s.HD = d_model;
    s.MLP = d_model;
    s.T = 1;
    s.B = 32;
    s.PW = C.N / 2 / s.B;
    if (d_model <= 0 || s.PW < d_model) throw ckks::Error(CKKS_EARG, "shape does not fit the slot layout");
    s.n1 = 32;
    while (s.n1 * s.n1 > s.PW) s.n1 >>= 1;
    s.n2 = s.PW / s.n1;
    s.groups = 1;
    auto* b = new ckks_block(ctx, s);
    try {
      b->nfc = 0;
      const int D = d_model;
      std::vector<double> w((size_t)D * D);
      for (int r = 0; r < D; ++r)
        for (int c = 0; c < D; ++c) w[(size_t)r * D + c] = head_linear[(size_t)r * D + c] * final_ln[c];
      b->d_head = upload_matrix(w);
      b->readout.assign(b->s.PW, 0.0);
      for (int f = 0; f < D; ++f) b->readout[f] = readout[f] * head_ln[f];
    } catch (...) {
      delete b;
      throw;
    }
    {
      std::lock_guard<std::mutex> lk(ctx->mu);
      ctx->blocks.insert(b);
    }
    *out = b;
  });
}

int ckks_head_forward(ckks_block* h, const double* x_last, double* margin) {
  return bguard([&] {
    if (!h || !x_last || !margin) throw ckks::Error(CKKS_EARG, "null argument");
    if (h->orphaned) throw ckks::Error(CKKS_ESTATE, "the head's context was destroyed");
    if (!h->d_head) throw ckks::Error(CKKS_EARG, "not a head object");
    *margin = h->head_forward(x_last);
  });
}

int ckks_block_release_cache(ckks_block* b, size_t* released) {
  return bguard([&] {
    if (!b) throw ckks::Error(CKKS_EARG, "null argument");
    const size_t r = b->orphaned ? 0 : b->release_cache();
    if (released) *released = r;
  });
}

int ckks_model_forward(ckks_block* const* blocks, int nblocks, ckks_block* head, const double* x, int tokens,
                       int cached_blocks, double* hidden, double* margin) {
  return bguard([&] {
    if (!blocks || nblocks <= 0 || !x || !hidden) throw ckks::Error(CKKS_EARG, "null argument");
    for (int i = 0; i < nblocks; ++i) {
      if (!blocks[i] || blocks[i]->orphaned || blocks[i]->d_head) throw ckks::Error(CKKS_EARG, "bad block handle");
      if (blocks[i]->s.T != tokens || blocks[i]->ctx != blocks[0]->ctx)
        throw ckks::Error(CKKS_EARG, "blocks differ in token count or context");
    }
    if (head && (head->orphaned || !head->d_head || head->ctx != blocks[0]->ctx || head->s.D != blocks[0]->s.D))
      throw ckks::Error(CKKS_EARG, "bad head handle");
    if (head && !margin) throw ckks::Error(CKKS_EARG, "null margin");
    const size_t n = (size_t)tokens * blocks[0]->s.D;
    std::vector<double> cur(x, x + n), nxt(n);
    // each block decrypts its output and the next re-encrypts it: the
    // reference's full-hidden-state refresh between blocks
    // (12blocks_head..._t123_v3.cpp:452-470)
    for (int i = 0; i < nblocks; ++i) {
      blocks[i]->forward(cur.data(), tokens, nxt.data());
      for (size_t k = 0; k < n; ++k)
        if (!std::isfinite(nxt[k])) throw ckks::Error(CKKS_ESTATE, "non-finite hidden state at a block boundary");
      // blocks past the cache budget encode their diagonals again on each use
      if (i >= cached_blocks) blocks[i]->release_cache();
      cur.swap(nxt);
    }
    std::memcpy(hidden, cur.data(), sizeof(double) * n);
    // last-token refresh into the head (:480-510)
    if (head) *margin = head->head_forward(cur.data() + (size_t)(tokens - 1) * blocks[0]->s.D);
  });
}

// ---- sharded evaluation of one block (stages over unit subsets) ----------
namespace {
std::vector<int> group_list(const ckks_block* b, const int* groups, int n) {
  if (n < 0 || (n && !groups)) throw ckks::Error(CKKS_EARG, "bad group list");
  std::vector<int> v(groups, groups + n);
  for (int g : v)
    if (g < 0 || g >= b->s.groups) throw ckks::Error(CKKS_EARG, "group index out of range");
  return v;
}
std::vector<std::pair<int, int>> pair_list(const ckks_block* b, const int* pairs, int n) {
  if (n < 0 || (n && !pairs)) throw ckks::Error(CKKS_EARG, "bad tile list");
  std::vector<std::pair<int, int>> v;
  for (int i = 0; i < n; ++i) {
    const int qg = pairs[2 * i], kg = pairs[2 * i + 1];
    if (kg < 0 || qg < kg || qg >= b->s.groups) throw ckks::Error(CKKS_EARG, "tile (qg, kg) out of range");
    v.push_back({qg, kg});
  }
  return v;
}
// (qg, kg, d) alignment triples; each must be a causal alignment of its tile
std::vector<blk::TileTag> tile_list(const ckks_block* b, const int* t, int n) {
  if (n < 0 || (n && !t)) throw ckks::Error(CKKS_EARG, "bad alignment list");
  std::vector<blk::TileTag> v;
  for (int i = 0; i < n; ++i) {
    const int qg = t[3 * i], kg = t[3 * i + 1], d = t[3 * i + 2];
    if (kg < 0 || qg < kg || qg >= b->s.groups) throw ckks::Error(CKKS_EARG, "tile (qg, kg) out of range");
    const auto act = blk::active_shifts(b->s.T, b->s.B, qg, kg);
    if (std::find(act.begin(), act.end(), d) == act.end())
      throw ckks::Error(CKKS_EARG, "lane shift is not an alignment of the tile");
    v.push_back({qg, kg, d});
  }
  return v;
}

ckks_block* live(ckks_block* b) {
  if (!b) throw ckks::Error(CKKS_EARG, "null block");
  if (b->orphaned) throw ckks::Error(CKKS_ESTATE, "the block's context was destroyed");
  if (b->d_head) throw ckks::Error(CKKS_EARG, "not a block object");
  return b;
}
}  // namespace

int ckks_block_shard_inputs(ckks_block* b, const double* x, int tokens) {
  return bguard([&] {
    if (!x) throw ckks::Error(CKKS_EARG, "null input");
    live(b)->shard_inputs(x, tokens);
  });
}

int ckks_block_shard_qkv(ckks_block* b, const int* groups, int n) {
  return bguard([&] { live(b)->shard_qkv(group_list(b, groups, n), 7); });
}

int ckks_block_shard_qkv_parts(ckks_block* b, const int* groups, int n, int parts) {
  return bguard([&] {
    if (parts < 0 || parts > 7) throw ckks::Error(CKKS_EARG, "parts: bit 0 Q, bit 1 K, bit 2 V");
    live(b)->shard_qkv(group_list(b, groups, n), parts);
  });
}

int ckks_block_shard_mlp(ckks_block* b, const int* groups, int n, int chunk_begin, int chunk_end) {
  return bguard([&] { live(b)->shard_mlp(group_list(b, groups, n), chunk_begin, chunk_end); });
}

int ckks_block_shard_finish(ckks_block* b, const int* groups, int n, double* y) {
  return bguard([&] {
    if (!y) throw ckks::Error(CKKS_EARG, "null output");
    live(b)->shard_finish(group_list(b, groups, n), y);
  });
}

int ckks_block_mlp_chunks(const ckks_block* b) { return b ? b->nfc : -1; }

int ckks_block_shard_scores(ckks_block* b, const int* pairs, int n, double* d_scores) {
  return bguard([&] {
    if (!d_scores) throw ckks::Error(CKKS_EARG, "null score buffer");
    live(b)->shard_scores(b->alignments(pair_list(b, pairs, n)), d_scores);
  });
}

int ckks_block_shard_scores_tiles(ckks_block* b, const int* tiles, int n, double* d_scores) {
  return bguard([&] {
    if (!d_scores) throw ckks::Error(CKKS_EARG, "null score buffer");
    live(b)->shard_scores(tile_list(b, tiles, n), d_scores);
  });
}

int ckks_block_shard_softmax(ckks_block* b, const double* d_scores) {
  return bguard([&] {
    if (!d_scores) throw ckks::Error(CKKS_EARG, "null score buffer");
    live(b)->shard_softmax(d_scores);
  });
}

int ckks_block_shard_context(ckks_block* b, const int* pairs, int n) {
  return bguard([&] { live(b)->shard_context(b->alignments(pair_list(b, pairs, n))); });
}

int ckks_block_shard_context_tiles(ckks_block* b, const int* tiles, int n) {
  return bguard([&] { live(b)->shard_context(tile_list(b, tiles, n)); });
}

int ckks_block_shard_output(ckks_block* b, const int* groups, int n, double* y) {
  return bguard([&] {
    if (!y) throw ckks::Error(CKKS_EARG, "null output");
    live(b)->shard_output(group_list(b, groups, n), y);
  });
}

// kind: 0 Q, 1 K, 2 V, 3 context (partial sum), 4 encrypted input
int ckks_block_state_get(ckks_block* b, int kind, int group, ckks_ct* out) {
  return bguard([&] {
    live(b);
    if (!out || out->owner != b->ctx) throw ckks::Error(CKKS_EARG, "bad ciphertext handle");
    if (group < 0 || group >= b->s.groups) throw ckks::Error(CKKS_EARG, "group index out of range");
    std::vector<Ciphertext>* v[] = {&b->st_q, &b->st_k, &b->st_v, &b->st_ctx, &b->st_x, &b->st_mlp, &b->st_r1};
    if (kind < 0 || kind > 6) throw ckks::Error(CKKS_EARG, "bad state kind");
    if ((int)v[kind]->size() <= group || !(*v[kind])[group]) throw ckks::Error(CKKS_ESTATE, "state not present");
    const ckks::DevPoly& p = (*v[kind])[group]->handle()->p;
    ckks::Context& C = b->C;
    ckks::DevPoly tmp;
    tmp.ensure(&C, 2, p.limbs);
    for (int k = 0; k < 2; ++k)
      CKKS_CUDA(cudaMemcpyAsync(tmp.poly(k), p.poly(k), sizeof(uint64_t) * (size_t)p.limbs * C.N,
                                cudaMemcpyDeviceToDevice, C.stream));
    tmp.limbs = p.limbs;
    tmp.scale = p.scale;
    tmp.deg = p.deg;
    std::swap(out->p.data, tmp.data);
    std::swap(out->p.npolys, tmp.npolys);
    std::swap(out->p.cap, tmp.cap);
    std::swap(out->p.limbs, tmp.limbs);
    std::swap(out->p.scale, tmp.scale);
    std::swap(out->p.deg, tmp.deg);
    out->p.ctx = &C;
  });
}

// an empty ciphertext handle (no limbs) clears the entry
int ckks_block_state_set(ckks_block* b, int kind, int group, const ckks_ct* in) {
  return bguard([&] {
    live(b);
    if (!in || in->owner != b->ctx) throw ckks::Error(CKKS_EARG, "bad ciphertext handle");
    if (group < 0 || group >= b->s.groups) throw ckks::Error(CKKS_EARG, "group index out of range");
    std::vector<Ciphertext>* v[] = {&b->st_q, &b->st_k, &b->st_v, &b->st_ctx, &b->st_x, &b->st_mlp, &b->st_r1};
    if (kind < 0 || kind > 6) throw ckks::Error(CKKS_EARG, "bad state kind");
    if ((int)v[kind]->size() != b->s.groups) throw ckks::Error(CKKS_ESTATE, "inputs not encrypted");
    if (!in->p.data || in->p.limbs <= 0) {
      (*v[kind])[group] = Ciphertext();
      return;
    }
    Ciphertext c = b->cc.fresh();
    ckks::DevPoly& p = c->handle()->p;
    ckks::Context& C = b->C;
    p.ensure(&C, 2, in->p.limbs);
    for (int k = 0; k < 2; ++k)
      CKKS_CUDA(cudaMemcpyAsync(p.poly(k), in->p.poly(k), sizeof(uint64_t) * (size_t)in->p.limbs * C.N,
                                cudaMemcpyDeviceToDevice, C.stream));
    p.limbs = in->p.limbs;
    p.scale = in->p.scale;
    p.deg = in->p.deg;
    (*v[kind])[group] = c;
  });
}

int ckks_block_destroy(ckks_block* b) {
  return bguard([&] {
    if (!b) return;
    if (!b->orphaned) {
      std::lock_guard<std::mutex> lk(b->ctx->mu);
      b->ctx->blocks.erase(b);
    }
    delete b;
  });
}

int ckks_block_rotation_indices(const ckks_block* b, int* out, int cap) {
  if (!b) return -1;
  const auto v = b->rotation_indices();
  for (int i = 0; i < (int)v.size() && i < cap; ++i) out[i] = v[i];
  return (int)v.size();
}

int ckks_block_forward(ckks_block* b, const double* x, int tokens, double* y) {
  return bguard([&] {
    if (!b || !x || !y) throw ckks::Error(CKKS_EARG, "null argument");
    if (b->orphaned) throw ckks::Error(CKKS_ESTATE, "the block's context was destroyed");
    b->forward(x, tokens, y);
  });
}

int ckks_block_report(const ckks_block* b, char* buf, size_t size) {
  if (!b) return -1;
  std::string js = "{\"counts\": {";
  bool first = true;
  for (auto& kv : b->count) {
    js += (first ? "\"" : ", \"") + kv.first + "\": " + std::to_string(kv.second);
    first = false;
  }
  js += std::string(first ? "" : ", ") + "\"diagonal_cache_mib\": " + std::to_string(b->cache_bytes() >> 20);
  js += "}, \"seconds\": {";
  first = true;
  char tmp[64];
  for (auto& kv : b->seconds) {
    std::snprintf(tmp, sizeof tmp, "%.6f", kv.second);
    js += (first ? "\"" : ", \"") + kv.first + "\": " + tmp;
    first = false;
  }
  js += "}}";
  if (buf && size) {
    const size_t n = std::min(js.size(), size - 1);
    std::memcpy(buf, js.data(), n);
    buf[n] = 0;
  }
  return (int)js.size();
}

int ckks_schedule_active_shifts(int tokens, int batch, int qg, int kg, int* out, int cap) {
  if (tokens <= 0 || batch <= 0 || qg < kg || kg < 0 || qg * batch >= tokens) return -1;
  const auto v = blk::active_shifts(tokens, batch, qg, kg);
  for (int i = 0; i < (int)v.size() && i < cap; ++i) out[i] = v[i];
  return (int)v.size();
}

int ckks_schedule_diagonal(const double* W, int out_dim, int in_dim, int ld, int pack_width, int batch, int n1,
                           int g, int j, double* out_slots) {
  if (!W || !out_slots || out_dim > pack_width || in_dim > pack_width || n1 <= 0 || pack_width % n1) return CKKS_EARG;
  for (int f = 0; f < pack_width; ++f) {
    const double v = blk::diag_value(W, out_dim, in_dim, ld, pack_width, n1, g, j, f);
    for (int t = 0; t < batch; ++t) out_slots[(size_t)f * batch + t] = v;
  }
  return CKKS_OK;
}

}  // extern "C"

// ---- fused BSGS product and lane shift as entry points ---------------------
namespace {
// the caller's handle, viewed without taking ownership
Ciphertext view(ckks_ctx* ctx, const ckks_ct* h) {
  if (!h) throw ckks::Error(CKKS_EARG, "null ciphertext");
  if (h->owner != ctx) throw ckks::Error(CKKS_EARG, "ciphertext belongs to another context");
  if (!h->p.data || h->p.limbs <= 0) throw ckks::Error(CKKS_ESTATE, "ciphertext holds no data");
  return std::make_shared<ckks_b200::CiphertextImpl>(ctx, const_cast<ckks_ct*>(h));
}
// moves a computed ciphertext into the caller's output handle
void move_into(ckks_ctx* ctx, ckks_ct* dst, const Ciphertext& src) {
  if (!dst || dst->owner != ctx) throw ckks::Error(CKKS_EARG, "bad output handle");
  ckks::DevPoly& a = dst->p;
  ckks::DevPoly& b = src->handle()->p;
  std::swap(a.ctx, b.ctx);
  std::swap(a.data, b.data);
  std::swap(a.npolys, b.npolys);
  std::swap(a.cap, b.cap);
  std::swap(a.limbs, b.limbs);
  std::swap(a.scale, b.scale);
  std::swap(a.deg, b.deg);
}
}  // namespace

extern "C" {

int ckks_bsgs_diagonals_create(ckks_ctx* ctx, const double* W, int out_dim, int in_dim, int ld, int batch, int n1,
                               int limbs, ckks_diag** out) {
  return bguard([&] {
    if (!ctx || !ctx->c || !W || !out) throw ckks::Error(CKKS_EARG, "null argument");
    ckks::Context& C = *ctx->c;
    if (batch <= 0 || (batch & (batch - 1)) || 2 * batch > C.N)
      throw ckks::Error(CKKS_EARG, "batch must be a power of two dividing N/2");
    const int PW = C.N / 2 / batch;
    if (n1 <= 0 || n1 > blk::kMaxBaby || PW % n1 || PW / n1 > blk::kMaxBaby)
      throw ckks::Error(CKKS_EARG, "n1 must divide the pack width with n1, n2 <= 32");
    if (C.N < blk::kThreads) throw ckks::Error(CKKS_EARG, "ring too small for the tiled diagonal store");
    if (out_dim <= 0 || in_dim <= 0 || out_dim > PW || in_dim > PW || ld < in_dim)
      throw ckks::Error(CKKS_EARG, "matrix does not fit the pack width");
    if (limbs <= 0 || limbs > C.L) throw ckks::Error(CKKS_ELEVEL, "limb count outside the chain");
    const size_t words = (size_t)(out_dim - 1) * ld + in_dim;
    double* dW = (double*)C.alloc(sizeof(double) * words);
    CKKS_CUDA(cudaMemcpyAsync(dW, W, sizeof(double) * words, cudaMemcpyHostToDevice, C.stream));
    auto* d = new ckks_diag;
    d->owner = ctx;
    d->limbs = limbs;
    d->n1 = n1;
    d->n2 = PW / n1;
    d->batch = batch;
    d->scale = C.scales[limbs];
    try {
      d->data = blk::encode_diagonals(C, dW, out_dim, in_dim, ld, PW, batch, n1, d->n2, limbs, d->scale);
    } catch (...) {
      C.release(dW);
      delete d;
      throw;
    }
    C.release(dW);
    {
      std::lock_guard<std::mutex> lk(ctx->mu);
      ctx->diags.insert(d);
    }
    *out = d;
  });
}

int ckks_bsgs_diagonals_destroy(ckks_diag* d) {
  return bguard([&] {
    if (!d) return;
    if (d->owner) {
      std::lock_guard<std::mutex> lk(d->owner->mu);
      d->owner->diags.erase(d);
      if (d->data) d->owner->c->release(d->data);
    }
    delete d;
  });
}

int ckks_bsgs_matmul(ckks_ctx* ctx, const ckks_diag* const* diags, int terms, const ckks_ct* const* baby, int groups,
                     ckks_ct* const* outs) {
  return bguard([&] {
    if (!ctx || !ctx->c || !diags || !baby || !outs) throw ckks::Error(CKKS_EARG, "null argument");
    if (terms <= 0 || groups <= 0) throw ckks::Error(CKKS_EARG, "terms and groups must be positive");
    ckks::Context& C = *ctx->c;
    const ckks_diag* d0 = diags[0];
    std::vector<blk::DiagRef> dgs;
    for (int t = 0; t < terms; ++t) {
      const ckks_diag* d = diags[t];
      if (!d || d->owner != ctx || !d->data) throw ckks::Error(CKKS_EARG, "diagonals of another context or released");
      if (d->n1 != d0->n1 || d->batch != d0->batch || d->limbs != d0->limbs)
        throw ckks::Error(CKKS_EARG, "diagonal sets differ in shape or level");
      dgs.push_back({d->data, d->limbs, d->scale});
    }
    const int n1 = d0->n1;
    std::vector<std::vector<std::vector<Ciphertext>>> bb(terms, std::vector<std::vector<Ciphertext>>(groups));
    for (int t = 0; t < terms; ++t)
      for (int q = 0; q < groups; ++q)
        for (int j = 0; j < n1; ++j) {
          const ckks_ct* h = baby[((size_t)t * groups + q) * n1 + j];
          Ciphertext x = view(ctx, h);
          if (h->p.limbs != d0->limbs) throw ckks::Error(CKKS_ELEVEL, "baby step not at the diagonals' level");
          if (h->p.deg != 1) throw ckks::Error(CKKS_ESTATE, "baby steps must be rescaled (noise degree 1)");
          bb[t][q].push_back(std::move(x));
        }
    for (int q = 0; q < groups; ++q)
      if (!outs[q] || outs[q]->owner != ctx) throw ckks::Error(CKKS_EARG, "bad output handle");
    ckks_b200::CryptoContextImpl cc(ctx);
    const auto r = blk::bsgs_products(cc, C, bb, dgs, n1, d0->n2, d0->batch);
    for (int q = 0; q < groups; ++q) move_into(ctx, outs[q], r[q]);
  });
}

int ckks_lane_shift(ckks_ctx* ctx, const ckks_ct* const* in, int count, const int* deltas, int nd, int batch,
                    ckks_ct* const* outs) {
  return bguard([&] {
    if (!ctx || !ctx->c || !in || !deltas || !outs) throw ckks::Error(CKKS_EARG, "null argument");
    if (count <= 0 || nd <= 0) throw ckks::Error(CKKS_EARG, "count and nd must be positive");
    ckks::Context& C = *ctx->c;
    if (batch <= 1 || (batch & (batch - 1)) || 2 * batch > C.N)
      throw ckks::Error(CKKS_EARG, "batch must be a power of two dividing N/2");
    std::vector<int> ds(deltas, deltas + nd);
    std::vector<Ciphertext> xs;
    for (int i = 0; i < count; ++i) {
      Ciphertext x = view(ctx, in[i]);
      if (x->noise_deg() != 1) throw ckks::Error(CKKS_ESTATE, "lane shift input must be rescaled (noise degree 1)");
      if (x->limbs() < 2) throw ckks::Error(CKKS_ELEVEL, "lane shift needs two limbs (it rescales)");
      xs.push_back(std::move(x));
    }
    for (int i = 0; i < count * nd; ++i)
      if (!outs[i] || outs[i]->owner != ctx) throw ckks::Error(CKKS_EARG, "bad output handle");
    ckks_b200::CryptoContextImpl cc(ctx);
    const int PW = C.N / 2 / batch;
    std::map<std::pair<int, bool>, Plaintext> cache;
    const blk::LaneMask mask = [&](int d, bool lower, int limbs) {
      auto key = std::make_pair(d, lower);
      auto it = cache.find(key);
      if (it != cache.end()) return it->second;
      return cache[key] = cc.MakePlaintextAt(blk::lane_mask_values(PW, batch, d, lower), limbs, C.scales[limbs]);
    };
    const auto r = blk::lane_shift_set(cc, xs, ds, batch, mask);
    for (int i = 0; i < count; ++i)
      for (int k = 0; k < nd; ++k) move_into(ctx, outs[(size_t)i * nd + k], r[i][k]);
  });
}

}  // extern "C"
