// keyswitch.cu -- hybrid key switching (ModUp, key inner product, ModDown)
// and Rescale.
//
// Key switching of d (l limbs, NTT form) with dnum digits of alpha limbs:
//   ModUp:   iNTT(d); for digit j, every limb outside the digit receives
//            sum_i [d_i * Qhat_{j,i}^-1]_{q_i} * Qhat_{j,i} mod m_t (approximate
//            fast basis conversion), then NTT; the digit's own limbs are the
//            input limbs unchanged.  ext: beta x (l+K) limbs.
//   inner:   acc_{0,1}[t] = sum_j ext_j[t][pi_g(n)] * key_j^{b,a}[t][n] with
//            128-bit accumulation and one reduction; pi_g is the NTT-domain
//            automorphism (identity for relinearisation), so a hoisted set of
//            rotations shares one ModUp.
//   ModDown: iNTT of the K special limbs, conversion P -> Q_l, NTT, and
//            (acc - conv) * P^-1 (+ the permuted c0 for a rotation).
// The same steps, in the same order, are restated on the CPU by the oracle;
// every residue is canonical, so the limbs agree exactly.
#include "bulk.cuh"
#include "ckks_internal.hpp"
#include "fpmod.cuh"

namespace ckks {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxAlpha = 16;
constexpr int kMaxK = 16;

// ModUp conversion.  y holds [d_i * Qhat_{j,i}^-1]_{q_i} (the scaling is
// folded into the inverse NTT); each thread owns two adjacent coefficients
// and kTargets extended limbs of one digit, so the MAC chains of 2 x kTargets
// outputs interleave.  Chunk 0 also copies the digit's own NTT-form limbs.
constexpr int kTargets = 4;

template <int MAXA>
__global__ void __launch_bounds__(kThreads) modup_conv_kernel(const uint64_t* __restrict__ y,
                                                              const uint64_t* __restrict__ d_ntt,
                                                              uint64_t* __restrict__ ext, int limbs, int L, int K,
                                                              int alpha, int logN, int nchunks,
                                                              const Mod* __restrict__ mods,
                                                              const uint64_t* __restrict__ hat) {
  const int N = 1 << logN;
  const int n = 2 * (blockIdx.x * kThreads + threadIdx.x);
  if (n >= N) return;
  const int j = blockIdx.y / nchunks, chunk = blockIdx.y % nchunks;
  const int E = limbs + K;
  const int lo = j * alpha;
  const int hi = min(lo + alpha, limbs);
  const int cnt = hi - lo;
  uint64_t* ej = ext + (size_t)j * E * N;
  ulonglong2 yv[MAXA];
#pragma unroll
  for (int i = 0; i < MAXA; ++i)
    if (i < cnt) yv[i] = *reinterpret_cast<const ulonglong2*>(y + (size_t)(lo + i) * N + n);
  if (chunk == 0) {
    for (int i = lo; i < hi; ++i)
      *reinterpret_cast<ulonglong2*>(ej + (size_t)i * N + n) =
          *reinterpret_cast<const ulonglong2*>(d_ntt + (size_t)i * N + n);
  }
  const int others = E - cnt;
#pragma unroll
  for (int p = 0; p < kTargets; ++p) {
    const int tt = chunk * kTargets + p;
    if (tt >= others) break;
    const int t = tt < lo ? tt : tt + cnt;
    const int pt = t < limbs ? t : L + (t - limbs);
    const uint64_t* h = hat + (size_t)j * alpha * E + t;
    U128 a0{0, 0}, a1{0, 0};
#pragma unroll
    for (int i = 0; i < MAXA; ++i) {
      if (i < cnt) {
        const uint64_t hv = __ldg(h + (size_t)i * E);
        mac_wide(a0, yv[i].x, hv);
        mac_wide(a1, yv[i].y, hv);
      }
    }
    const Mod m = mods[pt];
    *reinterpret_cast<ulonglong2*>(ej + (size_t)t * N + n) = make_ulonglong2(reduce128(a0, m), reduce128(a1, m));
  }
}

__global__ void __launch_bounds__(kThreads) ks_inner_kernel(const uint64_t* __restrict__ ext,
                                                            const uint64_t* __restrict__ key,
                                                            uint64_t* __restrict__ acc, int limbs, int L, int K,
                                                            int P, int beta, uint32_t g, int logN,
                                                            const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int t = blockIdx.y;
  const int E = limbs + K;
  const int pt = t < limbs ? t : L + (t - limbs);
  const Mod m = mods[pt];
  const uint32_t src = (g == 1u) ? (uint32_t)n : auto_index((uint32_t)n, g, logN);
  U128 s0{0, 0}, s1{0, 0};
  for (int j = 0; j < beta; ++j) {
    const uint64_t v = ext[((size_t)j * E + t) * N + src];
    const uint64_t kb = key[((size_t)j * 2 * P + pt) * N + n];
    const uint64_t ka = key[((size_t)j * 2 * P + P + pt) * N + n];
    mac_wide(s0, v, kb);
    mac_wide(s1, v, ka);
  }
  acc[(size_t)t * N + n] = reduce128(s0, m);
  acc[((size_t)E + t) * N + n] = reduce128(s1, m);
}

// ModDown conversion: conv[p][t] = sum_k y_k * Phat_k mod q_t, where the K
// special limbs of acc_p already hold y_k = [x_k * Phat_k^-1]_{p_k} in
// coefficient form (scaling folded into their inverse NTT).
template <int MAXK>
__global__ void __launch_bounds__(kThreads) moddown_conv_kernel(const uint64_t* __restrict__ acc,
                                                                uint64_t* __restrict__ conv, int limbs, int L,
                                                                int K, int logN, int nchunks,
                                                                const Mod* __restrict__ mods,
                                                                const uint64_t* __restrict__ phat) {
  const int N = 1 << logN;
  const int n = 2 * (blockIdx.x * kThreads + threadIdx.x);
  if (n >= N) return;
  const int p = blockIdx.y / nchunks, chunk = blockIdx.y % nchunks;
  const int E = limbs + K;
  const uint64_t* xp = acc + ((size_t)p * E + limbs) * N;
  ulonglong2 yv[MAXK];
#pragma unroll
  for (int k = 0; k < MAXK; ++k)
    if (k < K) yv[k] = *reinterpret_cast<const ulonglong2*>(xp + (size_t)k * N + n);
  uint64_t* o = conv + (size_t)p * limbs * N;
#pragma unroll
  for (int pp = 0; pp < kTargets; ++pp) {
    const int t = chunk * kTargets + pp;
    if (t >= limbs) break;
    U128 a0{0, 0}, a1{0, 0};
#pragma unroll
    for (int k = 0; k < MAXK; ++k) {
      if (k < K) {
        const uint64_t hv = __ldg(phat + (size_t)k * limbs + t);
        mac_wide(a0, yv[k].x, hv);
        mac_wide(a1, yv[k].y, hv);
      }
    }
    const Mod m = mods[t];
    *reinterpret_cast<ulonglong2*>(o + (size_t)t * N + n) = make_ulonglong2(reduce128(a0, m), reduce128(a1, m));
  }
}

// out_p[t] = (acc_p[t] - conv_p[t]) * P^-1, plus add0[t][pi_g(n)] for p = 0
// and add1[t][n] for p = 1 when given
__global__ void __launch_bounds__(kThreads) moddown_combine_kernel(const uint64_t* __restrict__ acc,
                                                                   const uint64_t* __restrict__ conv,
                                                                   const uint64_t* __restrict__ add0, uint32_t g,
                                                                   const uint64_t* __restrict__ add1,
                                                                   uint64_t* __restrict__ out0,
                                                                   uint64_t* __restrict__ out1, int limbs, int K,
                                                                   int logN, const Mod* __restrict__ mods,
                                                                   const ulonglong2* __restrict__ pinv) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int t = blockIdx.y % limbs, p = blockIdx.y / limbs;
  const int E = limbs + K;
  const uint64_t q = mods[t].q;
  const ulonglong2 pv = pinv[t];
  const uint64_t a = acc[((size_t)p * E + t) * N + n];
  const uint64_t cv = conv[((size_t)p * limbs + t) * N + n];
  uint64_t r = mul_shoup(sub_mod(a, cv, q), pv.x, pv.y, q);
  if (p == 0) {
    if (add0) {
      const uint32_t src = (g == 1u) ? (uint32_t)n : auto_index((uint32_t)n, g, logN);
      r = add_mod(r, add0[(size_t)t * N + src], q);
    }
    out0[(size_t)t * N + n] = r;
  } else {
    if (add1) r = add_mod(r, add1[(size_t)t * N + n], q);
    out1[(size_t)t * N + n] = r;
  }
}

// tmp[p][i] = last_p mod q_i (coefficient form), i < limbs-1
__global__ void __launch_bounds__(kThreads) rescale_spread_kernel(const uint64_t* __restrict__ last,
                                                                  uint64_t* __restrict__ tmp, int limbs, int logN,
                                                                  const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int lo = limbs - 1;
  const int i = blockIdx.y % lo, p = blockIdx.y / lo;
  const uint64_t v = last[(size_t)p * N + n];
  tmp[((size_t)p * lo + i) * N + n] = reduce128(U128{v, 0}, mods[i]);
}

__global__ void __launch_bounds__(kThreads) rescale_combine_kernel(const uint64_t* __restrict__ x, size_t sx,
                                                                   const uint64_t* __restrict__ tmp,
                                                                   uint64_t* __restrict__ out, size_t so,
                                                                   int limbs, int logN,
                                                                   const Mod* __restrict__ mods,
                                                                   const ulonglong2* __restrict__ inv) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int lo = limbs - 1;
  const int i = blockIdx.y % lo, p = blockIdx.y / lo;
  const uint64_t q = mods[i].q;
  const ulonglong2 iv = inv[i];
  const uint64_t a = x[p * sx + (size_t)i * N + n];
  const uint64_t b = tmp[((size_t)p * lo + i) * N + n];
  out[p * so + (size_t)i * N + n] = mul_shoup(sub_mod(a, b, q), iv.x, iv.y, q);
}

}  // namespace

void modup(const Context& c, const uint64_t* d_ntt, int limbs, uint64_t* ext, cudaStream_t st) {
  if (c.alpha > kMaxAlpha) throw Error(kErrArgument, "alpha above 16 is not supported");
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  uint64_t* dc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)limbs * N);
  CKKS_CUDA(cudaMemcpyAsync(dc, d_ntt, sizeof(uint64_t) * (size_t)limbs * N, cudaMemcpyDeviceToDevice, st));
  ntt_inverse(c, dc, limbs, LimbMap::q(limbs, c.L), st, lt.d_up_scale_a, lt.d_up_scale_b);
  // the last digit may hold fewer than alpha limbs and so has the most targets
  const int min_cnt = limbs - (lt.beta - 1) * c.alpha;
  const int nchunks = (E - min_cnt + kTargets - 1) / kTargets;
  const dim3 grid((N / 2 + kThreads - 1) / kThreads, lt.beta * nchunks);
  {
    // reads the input limbs (coefficient form for the sources, NTT form for
    // the copied ones) and writes every extended limb of every digit
    ProfScope ps(c, "modup_conv", (2.0 * limbs + (double)lt.beta * E) * c.limb_bytes(), st);
    auto kern = c.alpha <= 4 ? modup_conv_kernel<4>
                : c.alpha <= 8 ? modup_conv_kernel<8>
                : c.alpha <= 12 ? modup_conv_kernel<12>
                                : modup_conv_kernel<16>;
    kern<<<grid, kThreads, 0, st>>>(dc, d_ntt, ext, limbs, c.L, c.Kx(limbs), c.alpha, c.logN, nchunks, c.d_mods,
                                    lt.d_up_hat);
  }
  CKKS_CUDA(cudaGetLastError());
  LimbMap m = LimbMap::ext(limbs, c.Kx(limbs), c.L);
  m.skip_alpha = c.alpha;
  ntt_forward(c, ext, lt.beta * E, m, st);
  c.release(dc);
}

void ks_inner(const Context& c, const uint64_t* ext, int limbs, const uint64_t* key, uint32_t g, uint64_t* acc,
              cudaStream_t st) {
  const LevelTables& lt = c.lt(limbs);
  const dim3 grid((c.N + kThreads - 1) / kThreads, limbs + c.Kx(limbs));
  const double E = limbs + c.Kx(limbs);
  ProfScope ps(c, "ks_inner", (3.0 * lt.beta * E + 2.0 * E) * c.limb_bytes(), st);
  ks_inner_kernel<<<grid, kThreads, 0, st>>>(ext, key, acc, limbs, c.L, c.Kx(limbs), c.P, lt.beta, g, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

void moddown2(const Context& c, uint64_t* acc, int limbs, const uint64_t* add0, uint32_t g_add0,
              const uint64_t* add1, uint64_t* out0, uint64_t* out1, cudaStream_t st) {
  if (c.Kx(limbs) > kMaxK) throw Error(kErrArgument, "more than 16 special primes is not supported");
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  // both polynomials' special limbs in one launch (the Q limbs are skipped)
  LimbMap pm = LimbMap::ext(limbs, c.Kx(limbs), c.L);
  pm.skip_q = 1;
  ntt_inverse(c, acc, 2 * E, pm, st, c.down_scale_a(limbs), c.down_scale_b(limbs), c.L);
  uint64_t* conv = (uint64_t*)c.alloc(sizeof(uint64_t) * 2 * (size_t)limbs * N);
  const int nchunks = (limbs + kTargets - 1) / kTargets;
  const dim3 g1((N / 2 + kThreads - 1) / kThreads, 2 * nchunks);
  {
    ProfScope ps1(c, "moddown_conv", (2.0 * c.Kx(limbs) + 2.0 * limbs) * c.limb_bytes(), st);
    auto kern = c.Kx(limbs) <= 4 ? moddown_conv_kernel<4>
                : c.Kx(limbs) <= 8 ? moddown_conv_kernel<8>
                : c.Kx(limbs) <= 12 ? moddown_conv_kernel<12>
                            : moddown_conv_kernel<16>;
    kern<<<g1, kThreads, 0, st>>>(acc, conv, limbs, c.L, c.Kx(limbs), c.logN, nchunks, c.d_mods, lt.d_down_phat);
  }
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, conv, 2 * limbs, LimbMap::q(limbs, c.L), st);
  const dim3 g2((N + kThreads - 1) / kThreads, 2 * limbs);
  {
    ProfScope ps2(c, "moddown_combine", ((add0 ? 1.0 : 0.0) + (add1 ? 1.0 : 0.0) + 6.0) * limbs * c.limb_bytes(),
                  st);
    moddown_combine_kernel<<<g2, kThreads, 0, st>>>(acc, conv, add0, g_add0, add1, out0, out1, limbs, c.Kx(limbs), c.logN,
                                                    c.d_mods, lt.d_down_pinv);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(conv);
}

void rescale(const Context& c, const uint64_t* x, size_t sx, int npolys, int limbs, uint64_t* out, size_t so,
             cudaStream_t st) {
  if (limbs < 2) throw Error(kErrLevel, "cannot rescale a single-limb ciphertext");
  const int N = c.N, lo = limbs - 1;
  const LevelTables& lt = c.lt(limbs);
  uint64_t* last = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)npolys * N);
  for (int p = 0; p < npolys; ++p)
    CKKS_CUDA(cudaMemcpyAsync(last + (size_t)p * N, x + p * sx + (size_t)lo * N, sizeof(uint64_t) * N,
                              cudaMemcpyDeviceToDevice, st));
  ntt_inverse(c, last, npolys, LimbMap::single(lo), st);
  uint64_t* tmp = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)npolys * lo * N);
  const dim3 g1((N + kThreads - 1) / kThreads, npolys * lo);
  {
    ProfScope ps1(c, "rescale_spread", (1.0 + lo) * npolys * c.limb_bytes(), st);
    rescale_spread_kernel<<<g1, kThreads, 0, st>>>(last, tmp, limbs, c.logN, c.d_mods);
  }
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, tmp, npolys * lo, LimbMap::q(lo, c.L), st);
  {
    ProfScope ps2(c, "rescale_combine", 3.0 * npolys * lo * c.limb_bytes(), st);
    rescale_combine_kernel<<<g1, kThreads, 0, st>>>(x, sx, tmp, out, so, limbs, c.logN, c.d_mods,
                                                    lt.d_rescale_inv);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(last);
  c.release(tmp);
}

// ModUp / ModDown with caller-provided scratch (limbs*N words for ModUp's
// transformed copy of d, 2*limbs*N words for ModDown's conversion output);
// same kernels and order as modup() / moddown2(), no allocation.
void modup_with(const Context& c, const uint64_t* d_ntt, int limbs, uint64_t* ext, uint64_t* dc, cudaStream_t st) {
  if (c.alpha > kMaxAlpha) throw Error(kErrArgument, "alpha above 16 is not supported");
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  CKKS_CUDA(cudaMemcpyAsync(dc, d_ntt, sizeof(uint64_t) * (size_t)limbs * N, cudaMemcpyDeviceToDevice, st));
  ntt_inverse(c, dc, limbs, LimbMap::q(limbs, c.L), st, lt.d_up_scale_a, lt.d_up_scale_b);
  // the last digit may hold fewer than alpha limbs and so has the most targets
  const int min_cnt = limbs - (lt.beta - 1) * c.alpha;
  const int nchunks = (E - min_cnt + kTargets - 1) / kTargets;
  const dim3 grid((N / 2 + kThreads - 1) / kThreads, lt.beta * nchunks);
  {
    ProfScope ps(c, "modup_conv", (2.0 * limbs + (double)lt.beta * E) * c.limb_bytes(), st);
    auto kern = c.alpha <= 4 ? modup_conv_kernel<4>
                : c.alpha <= 8 ? modup_conv_kernel<8>
                : c.alpha <= 12 ? modup_conv_kernel<12>
                                : modup_conv_kernel<16>;
    kern<<<grid, kThreads, 0, st>>>(dc, d_ntt, ext, limbs, c.L, c.Kx(limbs), c.alpha, c.logN, nchunks, c.d_mods,
                                    lt.d_up_hat);
  }
  CKKS_CUDA(cudaGetLastError());
  LimbMap m = LimbMap::ext(limbs, c.Kx(limbs), c.L);
  m.skip_alpha = c.alpha;
  ntt_forward(c, ext, lt.beta * E, m, st);
}

void moddown2_with(const Context& c, uint64_t* acc, int limbs, const uint64_t* add0, uint32_t g_add0,
                   const uint64_t* add1, uint64_t* out0, uint64_t* out1, uint64_t* conv, cudaStream_t st) {
  if (c.Kx(limbs) > kMaxK) throw Error(kErrArgument, "more than 16 special primes is not supported");
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  LimbMap pm = LimbMap::ext(limbs, c.Kx(limbs), c.L);
  pm.skip_q = 1;
  ntt_inverse(c, acc, 2 * E, pm, st, c.down_scale_a(limbs), c.down_scale_b(limbs), c.L);
  const int nchunks = (limbs + kTargets - 1) / kTargets;
  const dim3 g1((N / 2 + kThreads - 1) / kThreads, 2 * nchunks);
  {
    ProfScope ps1(c, "moddown_conv", (2.0 * c.Kx(limbs) + 2.0 * limbs) * c.limb_bytes(), st);
    auto kern = c.Kx(limbs) <= 4 ? moddown_conv_kernel<4>
                : c.Kx(limbs) <= 8 ? moddown_conv_kernel<8>
                : c.Kx(limbs) <= 12 ? moddown_conv_kernel<12>
                            : moddown_conv_kernel<16>;
    kern<<<g1, kThreads, 0, st>>>(acc, conv, limbs, c.L, c.Kx(limbs), c.logN, nchunks, c.d_mods, lt.d_down_phat);
  }
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, conv, 2 * limbs, LimbMap::q(limbs, c.L), st);
  const dim3 g2((N + kThreads - 1) / kThreads, 2 * limbs);
  {
    ProfScope ps2(c, "moddown_combine", ((add0 ? 1.0 : 0.0) + (add1 ? 1.0 : 0.0) + 6.0) * limbs * c.limb_bytes(),
                  st);
    moddown_combine_kernel<<<g2, kThreads, 0, st>>>(acc, conv, add0, g_add0, add1, out0, out1, limbs, c.Kx(limbs), c.logN,
                                                    c.d_mods, lt.d_down_pinv);
  }
  CKKS_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Batched key switching and rescale (one launch per stage for a whole batch)
// ---------------------------------------------------------------------------
namespace {

template <int MAXA>
__global__ void __launch_bounds__(kThreads) modup_conv_batch_kernel(KsBatch b, const uint64_t* __restrict__ y_all,
                                                                    uint64_t* __restrict__ ext_all, int limbs, int L,
                                                                    int K, int alpha, int beta, int logN, int nchunks,
                                                                    const Mod* __restrict__ mods,
                                                                    const uint64_t* __restrict__ hat) {
  CKKS_PDL_ENTRY();
  const int N = 1 << logN;
  const int n = 2 * (blockIdx.x * kThreads + threadIdx.x);
  if (n >= N) return;
  const int m = blockIdx.z;
  const int j = blockIdx.y / nchunks, chunk = blockIdx.y % nchunks;
  const int E = limbs + K;
  const int lo = j * alpha;
  const int hi = min(lo + alpha, limbs);
  const int cnt = hi - lo;
  const uint64_t* y = y_all + (size_t)m * limbs * N;
  const uint64_t* d_ntt = b.d[m];
  uint64_t* ej = ext_all + ((size_t)m * beta + j) * E * N;
  ulonglong2 yv[MAXA];
#pragma unroll
  for (int i = 0; i < MAXA; ++i)
    if (i < cnt) yv[i] = *reinterpret_cast<const ulonglong2*>(y + (size_t)(lo + i) * N + n);
  if (chunk == 0) {
    for (int i = lo; i < hi; ++i)
      *reinterpret_cast<ulonglong2*>(ej + (size_t)i * N + n) =
          *reinterpret_cast<const ulonglong2*>(d_ntt + (size_t)i * N + n);
  }
  const int others = E - cnt;
#pragma unroll
  for (int p = 0; p < kTargets; ++p) {
    const int tt = chunk * kTargets + p;
    if (tt >= others) break;
    const int t = tt < lo ? tt : tt + cnt;
    const int pt = t < limbs ? t : L + (t - limbs);
    const uint64_t* h = hat + (size_t)j * alpha * E + t;
    U128 a0{0, 0}, a1{0, 0};
#pragma unroll
    for (int i = 0; i < MAXA; ++i) {
      if (i < cnt) {
        const uint64_t hv = __ldg(h + (size_t)i * E);
        mac_wide(a0, yv[i].x, hv);
        mac_wide(a1, yv[i].y, hv);
      }
    }
    const Mod md = mods[pt];
    *reinterpret_cast<ulonglong2*>(ej + (size_t)t * N + n) = make_ulonglong2(reduce128(a0, md), reduce128(a1, md));
  }
}

// sum_j ext_j[src pair] * key_j for both key halves over the item's digits,
// two adjacent residues: every digit's loads are issued before any product
// when the digit count is a compile-time 1..4 (the runtime loop would wait
// one memory round trip per digit)
template <int BETA>
__device__ __forceinline__ void ks_digit_products(const uint64_t* __restrict__ ext, const uint64_t* __restrict__ key,
                                                  size_t E, size_t P, int t, int pt, int N, uint32_t src, int n,
                                                  U128& a0, U128& a1, U128& b0, U128& b1) {
  ulonglong2 v[BETA], k0[BETA], k1[BETA];
#pragma unroll
  for (int j = 0; j < BETA; ++j) {
    v[j] = *reinterpret_cast<const ulonglong2*>(ext + ((size_t)j * E + t) * N + (src & ~1u));
    k0[j] = *reinterpret_cast<const ulonglong2*>(key + ((size_t)j * 2 * P + pt) * N + n);
    k1[j] = *reinterpret_cast<const ulonglong2*>(key + ((size_t)j * 2 * P + P + pt) * N + n);
  }
  const bool swap = src & 1u;
#pragma unroll
  for (int j = 0; j < BETA; ++j) {
    const uint64_t v0 = swap ? v[j].y : v[j].x, v1 = swap ? v[j].x : v[j].y;
    mac_wide(a0, v0, k0[j].x);
    mac_wide(a1, v1, k0[j].y);
    mac_wide(b0, v0, k1[j].x);
    mac_wide(b1, v1, k1[j].y);
  }
}

__device__ __forceinline__ void ks_digits(const uint64_t* __restrict__ ext, const uint64_t* __restrict__ key, int beta,
                                          size_t E, size_t P, int t, int pt, int N, uint32_t src, int n, U128& a0,
                                          U128& a1, U128& b0, U128& b1) {
  switch (beta) {
    case 1: ks_digit_products<1>(ext, key, E, P, t, pt, N, src, n, a0, a1, b0, b1); return;
    case 2: ks_digit_products<2>(ext, key, E, P, t, pt, N, src, n, a0, a1, b0, b1); return;
    case 3: ks_digit_products<3>(ext, key, E, P, t, pt, N, src, n, a0, a1, b0, b1); return;
    case 4: ks_digit_products<4>(ext, key, E, P, t, pt, N, src, n, a0, a1, b0, b1); return;
    default: break;
  }
  const bool swap = src & 1u;
  for (int j = 0; j < beta; ++j) {
    const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(ext + ((size_t)j * E + t) * N + (src & ~1u));
    const uint64_t v0 = swap ? v.y : v.x, v1 = swap ? v.x : v.y;
    const ulonglong2 k0 = *reinterpret_cast<const ulonglong2*>(key + ((size_t)j * 2 * P + pt) * N + n);
    const ulonglong2 k1 = *reinterpret_cast<const ulonglong2*>(key + ((size_t)j * 2 * P + P + pt) * N + n);
    mac_wide(a0, v0, k0.x);
    mac_wide(a1, v1, k0.y);
    mac_wide(b0, v0, k1.x);
    mac_wide(b1, v1, k1.y);
  }
}

__global__ void __launch_bounds__(kThreads) ks_inner_batch_kernel(KsBatch b, const uint64_t* __restrict__ ext_all,
                                                                  bool shared, uint64_t* __restrict__ acc_all,
                                                                  int limbs, int L, int K, int P, int beta, int logN,
                                                                  const Mod* __restrict__ mods) {
  CKKS_PDL_ENTRY();
  // two adjacent residues per thread (src(n + 1) = src(n) ^ 1)
  const int N = 1 << logN;
  const int n = 2 * (blockIdx.x * kThreads + threadIdx.x);
  if (n >= N) return;
  const int t = blockIdx.y, m = blockIdx.z;
  const int E = limbs + K;
  const int pt = t < limbs ? t : L + (t - limbs);
  const Mod md = mods[pt];
  const uint32_t g = b.g[m];
  const uint64_t* ext = ext_all + (shared ? 0 : (size_t)m * beta * E * N);
  const uint64_t* key = b.key[m];
  const uint32_t src = (g == 1u) ? (uint32_t)n : auto_index((uint32_t)n, g, logN);
  U128 a0{0, 0}, a1{0, 0}, b0{0, 0}, b1{0, 0};
  ks_digits(ext, key, beta, E, P, t, pt, N, src, n, a0, a1, b0, b1);
  uint64_t* acc = acc_all + (size_t)m * 2 * E * N;
  *reinterpret_cast<ulonglong2*>(acc + (size_t)t * N + n) = make_ulonglong2(reduce128(a0, md), reduce128(a1, md));
  *reinterpret_cast<ulonglong2*>(acc + ((size_t)E + t) * N + n) =
      make_ulonglong2(reduce128(b0, md), reduce128(b1, md));
}

// inner products of every item summed: acc = sum_m sum_j ext_{m,j}[pi_m(n)] key_{m,j};
// the 128-bit accumulators are folded to a residue every `fold` items so that
// at most 63 products are ever summed unreduced
__global__ void __launch_bounds__(kThreads) ks_inner_sum_kernel(KsBatch b, const uint64_t* __restrict__ ext_all,
                                                                uint64_t* __restrict__ acc, int limbs, int L, int K,
                                                                int P, int beta, int logN, int fold,
                                                                const Mod* __restrict__ mods) {
  CKKS_PDL_ENTRY();
  // two adjacent residues per thread (src(n + 1) = src(n) ^ 1): 16-byte
  // loads and stores
  const int N = 1 << logN;
  const int n = 2 * (blockIdx.x * kThreads + threadIdx.x);
  if (n >= N) return;
  const int t = blockIdx.y;
  const int E = limbs + K;
  const int pt = t < limbs ? t : L + (t - limbs);
  const Mod md = mods[pt];
  U128 a0{0, 0}, a1{0, 0}, b0{0, 0}, b1{0, 0};
  for (int m = 0; m < b.M; ++m) {
    const uint32_t g = b.g[m];
    const uint32_t src = (g == 1u) ? (uint32_t)n : auto_index((uint32_t)n, g, logN);
    const uint64_t* ext = ext_all + (size_t)m * beta * E * N;
    ks_digits(ext, b.key[m], beta, E, P, t, pt, N, src, n, a0, a1, b0, b1);
    if ((m + 1) % fold == 0) {
      a0 = U128{reduce128(a0, md), 0};
      a1 = U128{reduce128(a1, md), 0};
      b0 = U128{reduce128(b0, md), 0};
      b1 = U128{reduce128(b1, md), 0};
    }
  }
  *reinterpret_cast<ulonglong2*>(acc + (size_t)t * N + n) = make_ulonglong2(reduce128(a0, md), reduce128(a1, md));
  *reinterpret_cast<ulonglong2*>(acc + ((size_t)E + t) * N + n) =
      make_ulonglong2(reduce128(b0, md), reduce128(b1, md));
}

// (acc - conv) P^-1 plus every item's automorphism-permuted c0 (output 0)
// or c1 addend (output 1)
__global__ void __launch_bounds__(kThreads) moddown_combine_sum_kernel(KsBatch b, const uint64_t* __restrict__ acc,
                                                                      const uint64_t* __restrict__ conv,
                                                                      uint64_t* __restrict__ out0,
                                                                      uint64_t* __restrict__ out1, int limbs, int K,
                                                                      int logN, const Mod* __restrict__ mods,
                                                                      const ulonglong2* __restrict__ pinv) {
  CKKS_PDL_ENTRY();
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int t = blockIdx.y % limbs, p = blockIdx.y / limbs;
  const int E = limbs + K;
  const uint64_t q = mods[t].q;
  const ulonglong2 pv = pinv[t];
  uint64_t r = mul_shoup(sub_mod(acc[((size_t)p * E + t) * N + n], conv[((size_t)p * limbs + t) * N + n], q), pv.x,
                         pv.y, q);
  for (int m = 0; m < b.M; ++m) {
    if (p == 0) {
      const uint64_t* a0 = b.add0[m];
      if (!a0) continue;
      const uint32_t g = b.g[m];
      const uint32_t src = (g == 1u) ? (uint32_t)n : auto_index((uint32_t)n, g, logN);
      r = add_mod(r, a0[(size_t)t * N + src], q);
    } else {
      const uint64_t* a1 = b.add1[m];
      if (a1) r = add_mod(r, a1[(size_t)t * N + n], q);
    }
  }
  (p == 0 ? out0 : out1)[(size_t)t * N + n] = r;
}

// giant-step sums of several groups: out0_g = ModDown(acc0_g) + sum_m
// pi_m(add0[g][m]) (+ id0_g), out1_g = ModDown(acc1_g) (+ id1_g)
__global__ void __launch_bounds__(kThreads) moddown_combine_groups_kernel(SumGroups s,
                                                                         const uint64_t* __restrict__ acc_all,
                                                                         const uint64_t* __restrict__ conv_all,
                                                                         int limbs, int K, int logN,
                                                                         const Mod* __restrict__ mods,
                                                                         const ulonglong2* __restrict__ pinv) {
  CKKS_PDL_ENTRY();
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int t = blockIdx.y % limbs, p = blockIdx.y / limbs, gi = blockIdx.z;
  const int E = limbs + K;
  const uint64_t q = mods[t].q;
  const ulonglong2 pv = pinv[t];
  const uint64_t a = acc_all[((size_t)(2 * gi + p) * E + t) * N + n];
  const uint64_t cv = conv_all[((size_t)(2 * gi + p) * limbs + t) * N + n];
  uint64_t r = mul_shoup(sub_mod(a, cv, q), pv.x, pv.y, q);
  if (p == 0) {
    for (int m = 0; m < s.M; ++m) {
      const uint32_t g = s.g[m];
      const uint32_t src = (g == 1u) ? (uint32_t)n : auto_index((uint32_t)n, g, logN);
      r = add_mod(r, s.add0[gi][m][(size_t)t * N + src], q);
    }
    if (s.id0[gi]) r = add_mod(r, s.id0[gi][(size_t)t * N + n], q);
    s.out0[gi][(size_t)t * N + n] = r;
  } else {
    if (s.id1[gi]) r = add_mod(r, s.id1[gi][(size_t)t * N + n], q);
    s.out1[gi][(size_t)t * N + n] = r;
  }
}

template <int MAXK>
__global__ void __launch_bounds__(kThreads) moddown_conv_batch_kernel(const uint64_t* __restrict__ acc_all,
                                                                      uint64_t* __restrict__ conv_all, int limbs,
                                                                      int L, int K, int logN, int nchunks,
                                                                      const Mod* __restrict__ mods,
                                                                      const uint64_t* __restrict__ phat) {
  CKKS_PDL_ENTRY();
  const int N = 1 << logN;
  const int n = 2 * (blockIdx.x * kThreads + threadIdx.x);
  if (n >= N) return;
  const int m = blockIdx.z;
  const int p = blockIdx.y / nchunks, chunk = blockIdx.y % nchunks;
  const int E = limbs + K;
  const uint64_t* xp = acc_all + ((size_t)(2 * m + p) * E + limbs) * N;
  ulonglong2 yv[MAXK];
#pragma unroll
  for (int k = 0; k < MAXK; ++k)
    if (k < K) yv[k] = *reinterpret_cast<const ulonglong2*>(xp + (size_t)k * N + n);
  uint64_t* o = conv_all + (size_t)(2 * m + p) * limbs * N;
#pragma unroll
  for (int pp = 0; pp < kTargets; ++pp) {
    const int t = chunk * kTargets + pp;
    if (t >= limbs) break;
    U128 a0{0, 0}, a1{0, 0};
#pragma unroll
    for (int k = 0; k < MAXK; ++k) {
      if (k < K) {
        const uint64_t hv = __ldg(phat + (size_t)k * limbs + t);
        mac_wide(a0, yv[k].x, hv);
        mac_wide(a1, yv[k].y, hv);
      }
    }
    const Mod md = mods[t];
    *reinterpret_cast<ulonglong2*>(o + (size_t)t * N + n) = make_ulonglong2(reduce128(a0, md), reduce128(a1, md));
  }
}

__global__ void __launch_bounds__(kThreads) rs_combine_batch_kernel(RsBatch b, const uint64_t* __restrict__ tmp,
                                                                    int limbs, int logN, const Mod* __restrict__ mods,
                                                                    const ulonglong2* __restrict__ inv) {
  CKKS_PDL_ENTRY();
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int lo = limbs - 1;
  const int i = blockIdx.y % lo, p = blockIdx.y / lo, m = blockIdx.z;
  const uint64_t q = mods[i].q;
  const ulonglong2 iv = inv[i];
  const uint64_t* x = p ? b.in1[m] : b.in0[m];
  uint64_t* o = p ? b.out1[m] : b.out0[m];
  const uint64_t a = x[(size_t)i * N + n];
  const uint64_t t = tmp[((size_t)(2 * m + p) * lo + i) * N + n];
  o[(size_t)i * N + n] = mul_shoup(sub_mod(a, t, q), iv.x, iv.y, q);
}

// hoisted sums: acc_m = sum_r sum_j ext_{m,j}[pi_r(n)] key_{r,j} -- the R
// rotations of item m share its ModUp.  A thread owns one residue (n, t) of
// kHoistItems items, so each key residue and automorphism index is loaded
// once for them.
constexpr int kHoistItems = 4;
// Item i of rotation r reads its extended digits at ext_all + i * istride +
// r * rstride: rstride = 0 for the rotations of one ModUp (hoisted sums),
// one digit set for the giant steps of several groups (one ModUp per
// rotated input).
// Products by the target prime: kHoistFp below kFpPrime (exact float64
// products, sums re-centred every four steps), kHoistSplit below 2^60
// (carry-free split products, reduced into a running residue every 16
// steps), kHoistWide otherwise (128-bit multiply-accumulates folded to a
// residue every `fold` rotations, so that at most 63 products are summed).
// Each mode is its own kernel, launched over the limbs of the extended basis
// whose primes take it (up to kTargetRuns runs of consecutive limbs, the
// blockIdx.y-th of them in order), so each keeps its own register budget.
enum { kHoistFp = 0, kHoistSplit = 1, kHoistWide = 2 };
constexpr int kTargetRuns = 4;
struct HoistTargets {
  int start[kTargetRuns], len[kTargetRuns];
  __device__ __forceinline__ int limb(int y) const {
    int t = start[0] + y;
#pragma unroll
    for (int r = 0; r + 1 < kTargetRuns; ++r) {
      if (y >= len[r]) {
        y -= len[r];
        t = start[r + 1] + y;
      } else {
        break;
      }
    }
    return t;
  }
};

template <int MODE>
__global__ void __launch_bounds__(kThreads, MODE == kHoistSplit ? 2 : 3)
    ks_inner_hoist_kernel(HoistKeys h, HoistTargets tl, const uint64_t* __restrict__ ext_all,
                          uint64_t* __restrict__ acc_all, int M, int limbs, int L, int K, int P, int beta, int logN,
                          int fold, const Mod* __restrict__ mods, size_t istride, size_t rstride) {
  CKKS_PDL_ENTRY();
  constexpr bool FP = MODE == kHoistFp;
  constexpr bool SPLIT = MODE == kHoistSplit;
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int t = tl.limb(blockIdx.y), m0 = blockIdx.z * kHoistItems;
  const int E = limbs + K;
  const int pt = t < limbs ? t : L + (t - limbs);
  const Mod md = mods[pt];
  const int cnt = min(kHoistItems, M - m0);
  const uint64_t* ext = ext_all + (size_t)m0 * istride + (size_t)t * N;
  const double qd = (double)md.q, qinv = 1.0 / qd;
  double f0[FP ? kHoistItems : 1], f1[FP ? kHoistItems : 1];
  SplitSums z0[SPLIT ? kHoistItems : 1], z1[SPLIT ? kHoistItems : 1];
  uint64_t r0[SPLIT ? kHoistItems : 1], r1[SPLIT ? kHoistItems : 1];
  U128 w0[MODE == kHoistWide ? kHoistItems : 1], w1[MODE == kHoistWide ? kHoistItems : 1];
#pragma unroll
  for (int i = 0; i < kHoistItems; ++i) {
    if constexpr (FP) {
      f0[i] = f1[i] = 0.0;
    } else if constexpr (SPLIT) {
      r0[i] = r1[i] = 0;
    } else {
      w0[i] = w1[i] = U128{0, 0};
    }
  }
  // the (rotation, digit) steps in order, the next step's key residues and
  // ModUp residues loaded while the current one's products run
  const int steps = h.R * beta;
  uint64_t k0 = 0, k1 = 0, v[kHoistItems];
  auto load = [&](int x, uint64_t& a0, uint64_t& a1, uint64_t* w) {
    const int r = x / beta, j = x - r * beta;
    const uint32_t src = auto_index((uint32_t)n, h.g[r], logN);
    const uint64_t* key = h.key[r];
    a0 = key[((size_t)j * 2 * P + pt) * N + n];
    a1 = key[((size_t)j * 2 * P + P + pt) * N + n];
    const uint64_t* ej = ext + (size_t)r * rstride + (size_t)j * E * N + src;
#pragma unroll
    for (int i = 0; i < kHoistItems; ++i) w[i] = i < cnt ? ej[(size_t)i * istride] : 0;
  };
  if (steps > 0) load(0, k0, k1, v);
  for (int x = 0; x < steps; ++x) {
    uint64_t nk0 = 0, nk1 = 0, nv[kHoistItems] = {};
    if (x + 1 < steps) load(x + 1, nk0, nk1, nv);
    if constexpr (FP) {
      const double kd0 = u2d(k0), kd1 = u2d(k1);
#pragma unroll
      for (int i = 0; i < kHoistItems; ++i) {
        if (i < cnt) {
          const double a = u2d(v[i]);
          f0[i] = __dadd_rn(f0[i], fp_mod_product(a, kd0, qd, qinv));
          f1[i] = __dadd_rn(f1[i], fp_mod_product(a, kd1, qd, qinv));
          if ((x & 3) == 3) {
            f0[i] = fp_center(f0[i], qd, qinv);
            f1[i] = fp_center(f1[i], qd, qinv);
          }
        }
      }
    } else if constexpr (SPLIT) {
      uint32_t kl0, kh0, kl1, kh1;
      split_residue(k0, kl0, kh0);
      split_residue(k1, kl1, kh1);
#pragma unroll
      for (int i = 0; i < kHoistItems; ++i) {
        if (i < cnt) {
          uint32_t vl, vh;
          split_residue(v[i], vl, vh);
          z0[i].mac(vl, vh, kl0, kh0);
          z1[i].mac(vl, vh, kl1, kh1);
          if ((x & 15) == 15) {
            r0[i] = add_mod(r0[i], z0[i].reduce(md), md.q);
            r1[i] = add_mod(r1[i], z1[i].reduce(md), md.q);
            z0[i] = SplitSums{};
            z1[i] = SplitSums{};
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < kHoistItems; ++i) {
        if (i < cnt) {
          mac_wide(w0[i], v[i], k0);
          mac_wide(w1[i], v[i], k1);
        }
      }
      const int r = x / beta;
      if (x - r * beta == beta - 1 && (r + 1) % fold == 0) {
#pragma unroll
        for (int i = 0; i < kHoistItems; ++i) {
          w0[i] = U128{reduce128(w0[i], md), 0};
          w1[i] = U128{reduce128(w1[i], md), 0};
        }
      }
    }
    k0 = nk0;
    k1 = nk1;
#pragma unroll
    for (int i = 0; i < kHoistItems; ++i) v[i] = nv[i];
  }
#pragma unroll
  for (int i = 0; i < kHoistItems; ++i) {
    if (i < cnt) {
      uint64_t* acc = acc_all + (size_t)(m0 + i) * 2 * E * N;
      uint64_t a, b;
      if constexpr (FP) {
        a = fp_canonical(fp_center(f0[i], qd, qinv), qd);
        b = fp_canonical(fp_center(f1[i], qd, qinv), qd);
      } else if constexpr (SPLIT) {
        a = add_mod(r0[i], z0[i].reduce(md), md.q);
        b = add_mod(r1[i], z1[i].reduce(md), md.q);
      } else {
        a = reduce128(w0[i], md);
        b = reduce128(w1[i], md);
      }
      acc[(size_t)t * N + n] = a;
      acc[((size_t)E + t) * N + n] = b;
    }
  }
}

// the hoisted key products of M items over every limb of the extended basis
// (Q_limbs and the K special primes), one launch per product mode
void launch_ks_inner_hoist(const Context& c, const HoistKeys& h, const uint64_t* ext, uint64_t* acc, int M,
                           int limbs, int beta, size_t istride, size_t rstride, cudaStream_t st) {
  const int K = c.Kx(limbs), E = limbs + K;
  HoistTargets tl[3]{};
  int cnt[3] = {0, 0, 0}, runs[3] = {0, 0, 0};
  for (int t = 0; t < E; ++t) {
    const uint64_t q = c.moduli[t < limbs ? t : c.L + (t - limbs)];
    const int mode = q < kFpPrime ? kHoistFp : q < (1ull << 60) ? kHoistSplit : kHoistWide;
    HoistTargets& x = tl[mode];
    int& r = runs[mode];
    if (r > 0 && x.start[r - 1] + x.len[r - 1] == t) {
      ++x.len[r - 1];
    } else {
      if (r == kTargetRuns) throw Error(kErrArgument, "prime sizes alternate too often along the extended basis");
      x.start[r] = t;
      x.len[r] = 1;
      ++r;
    }
    ++cnt[mode];
  }
  const int fold = 63 / beta;
  const int N = c.N;
  for (int mode = 0; mode < 3; ++mode) {
    if (!cnt[mode]) continue;
    const dim3 grid((N + kThreads - 1) / kThreads, cnt[mode], (M + kHoistItems - 1) / kHoistItems);
    auto kern = mode == kHoistFp      ? ks_inner_hoist_kernel<kHoistFp>
                : mode == kHoistSplit ? ks_inner_hoist_kernel<kHoistSplit>
                                      : ks_inner_hoist_kernel<kHoistWide>;
    launch_pdl(kern, grid, kThreads, 0, st, h, tl[mode], ext, acc, M, limbs, c.L, K, c.P, beta, c.logN, fold, c.d_mods, istride, rstride);
    CKKS_CUDA(cudaGetLastError());
  }
}

// (acc_m - conv_m) P^-1 plus sum_r pi_r(c0_m) (output 0), and the input
// itself when the identity is part of the sum
__global__ void __launch_bounds__(kThreads) moddown_combine_hoist_kernel(KsBatch b, HoistKeys h, bool identity,
                                                                        const uint64_t* __restrict__ acc_all,
                                                                        const uint64_t* __restrict__ conv_all,
                                                                        int limbs, int K, int logN,
                                                                        const Mod* __restrict__ mods,
                                                                        const ulonglong2* __restrict__ pinv) {
  CKKS_PDL_ENTRY();
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int t = blockIdx.y % limbs, p = blockIdx.y / limbs, m = blockIdx.z;
  const int E = limbs + K;
  const uint64_t q = mods[t].q;
  const ulonglong2 pv = pinv[t];
  const uint64_t a = acc_all[((size_t)(2 * m + p) * E + t) * N + n];
  const uint64_t cv = conv_all[((size_t)(2 * m + p) * limbs + t) * N + n];
  uint64_t r = mul_shoup(sub_mod(a, cv, q), pv.x, pv.y, q);
  if (p == 0) {
    const uint64_t* c0 = b.add0[m] + (size_t)t * N;
    if (identity) r = add_mod(r, c0[n], q);
    for (int k = 0; k < h.R; ++k) r = add_mod(r, c0[auto_index((uint32_t)n, h.g[k], logN)], q);
    b.out0[m][(size_t)t * N + n] = r;
  } else {
    if (identity) r = add_mod(r, b.d[m][(size_t)t * N + n], q);
    b.out1[m][(size_t)t * N + n] = r;
  }
}

// key products of (input, rotation) items, item m = blockIdx.x (fastest), so
// the CTAs of the items sharing one key and one residue range run together
// and its residues come from HBM once
__global__ void __launch_bounds__(kThreads) ks_inner_multi_kernel(KsBatch b, const uint64_t* __restrict__ ext_all,
                                                                  uint64_t* __restrict__ acc_all, int limbs, int L,
                                                                  int K, int P, int beta, int logN,
                                                                  const Mod* __restrict__ mods) {
  CKKS_PDL_ENTRY();
  // two adjacent residues n, n + 1 per thread: the automorphism maps the
  // aligned pair onto an aligned pair (src(n + 1) = src(n) ^ 1), so every
  // load and store is 16 bytes
  const int N = 1 << logN;
  const int m = blockIdx.x;
  const int n = 2 * (blockIdx.y * kThreads + threadIdx.x);
  if (n >= N) return;
  const int t = blockIdx.z;
  const int E = limbs + K;
  const int pt = t < limbs ? t : L + (t - limbs);
  const Mod md = mods[pt];
  const uint32_t g = b.g[m];
  const uint64_t* ext = ext_all + (size_t)b.src[m] * beta * E * N;
  const uint64_t* key = b.key[m];
  const uint32_t src = auto_index((uint32_t)n, g, logN);
  U128 a0{0, 0}, a1{0, 0}, b0{0, 0}, b1{0, 0};
  ks_digits(ext, key, beta, E, P, t, pt, N, src, n, a0, a1, b0, b1);
  uint64_t* acc = acc_all + (size_t)m * 2 * E * N;
  *reinterpret_cast<ulonglong2*>(acc + (size_t)t * N + n) = make_ulonglong2(reduce128(a0, md), reduce128(a1, md));
  *reinterpret_cast<ulonglong2*>(acc + ((size_t)E + t) * N + n) =
      make_ulonglong2(reduce128(b0, md), reduce128(b1, md));
}

// ---- key products with bulk-copied operands ---------------------------------
// The 2 kThreads outputs of one CTA read, per digit, 2 kThreads residues of
// each key half at the outputs' own positions and the ModUp residues at the
// automorphism's sources.  Those sources are one aligned span of the same
// size: with k = hi 2^9 + lo, the varying low bits lo of the output become
// the top bits of e = 2 bitrev(k) + 1, e g (g odd) runs over every value of
// those bits, and the bit reversal brings them back to the low bits of the
// source, while the high bits stay fixed by hi.  So one thread issues 3 beta
// contiguous 4 KiB copies (cp.async.bulk, completing on one mbarrier) and
// the products read shared memory only.
constexpr int kSpan = 2 * kThreads;
constexpr uint32_t kSpanBytes = kSpan * sizeof(uint64_t);
// BULK_MULTI false: item m = blockIdx.z, ModUp output per item unless
// `shared` (keyswitch_batch's grid); true: item m = blockIdx.x with the ModUp
// output of input b.src[m] (keyswitch_hoisted_multi's grid, the items of one
// key adjacent).
template <int BETA, bool BULK_MULTI>
__global__ void __launch_bounds__(kThreads) ks_inner_bulk_kernel(KsBatch b, const uint64_t* __restrict__ ext_all,
                                                                 bool shared, uint64_t* __restrict__ acc_all,
                                                                 int limbs, int L, int K, int P, int logN,
                                                                 const Mod* __restrict__ mods,
                                                                 unsigned int* __restrict__ faults) {
  CKKS_PDL_ENTRY();
  __shared__ alignas(128) uint64_t sx[BETA][kSpan];
  __shared__ alignas(128) uint64_t sk[BETA][2][kSpan];
  __shared__ alignas(8) uint64_t bar;
  const int N = 1 << logN;
  const int m = BULK_MULTI ? blockIdx.x : blockIdx.z;
  const int n0 = (BULK_MULTI ? blockIdx.y : blockIdx.x) * kSpan;
  const int t = BULK_MULTI ? blockIdx.z : blockIdx.y;
  const int E = limbs + K;
  const int pt = t < limbs ? t : L + (t - limbs);
  const uint32_t g = b.g[m];
  const uint64_t* ext =
      ext_all + (BULK_MULTI ? (size_t)b.src[m] * BETA * E * N : (shared ? 0 : (size_t)m * BETA * E * N));
  const uint64_t* key = b.key[m];
  const uint32_t s0 = g == 1u ? (uint32_t)n0 : auto_index((uint32_t)n0, g, logN) & ~(uint32_t)(kSpan - 1);
  const uint32_t mb = smem_addr(&bar);
  if (threadIdx.x == 0) mbar_init(mb, 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_expect_tx(mb, 3u * BETA * kSpanBytes);
#pragma unroll
    for (int j = 0; j < BETA; ++j) {
      bulk_load(smem_addr(sx[j]), ext + ((size_t)j * E + t) * N + s0, kSpanBytes, mb);
      bulk_load(smem_addr(sk[j][0]), key + ((size_t)j * 2 * P + pt) * N + n0, kSpanBytes, mb);
      bulk_load(smem_addr(sk[j][1]), key + ((size_t)j * 2 * P + P + pt) * N + n0, kSpanBytes, mb);
    }
  }
  if (!mbar_wait_bounded(mb, 0)) {
    // record it for the host, give the copies one more bounded wait, and
    // leave this CTA's outputs unwritten
    if (threadIdx.x == 0) atomicAdd(faults, 1u);
    mbar_wait_bounded(mb, 0);
    return;
  }
  const int i = 2 * threadIdx.x, n = n0 + i;
  const uint32_t src = g == 1u ? (uint32_t)n : auto_index((uint32_t)n, g, logN);
  const uint32_t so = (src & ~1u) & (uint32_t)(kSpan - 1);  // = (src & ~1) - s0
  const bool swap = src & 1u;
  const Mod md = mods[pt];
  ulonglong2 ra, rb;
  if (md.q < kFpPrime) {
    // exact float64 products: sums of at most three, |sum| < 3.2 q, exact
    // (the other primes keep 128-bit multiply-accumulates: 30-bit split
    // products measured slower here)
    const double qd = (double)md.q, qinv = 1.0 / qd;
    double a0 = 0.0, a1 = 0.0, b0 = 0.0, b1 = 0.0;
#pragma unroll
    for (int j = 0; j < BETA; ++j) {
      const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(&sx[j][so]);
      const ulonglong2 k0 = *reinterpret_cast<const ulonglong2*>(&sk[j][0][i]);
      const ulonglong2 k1 = *reinterpret_cast<const ulonglong2*>(&sk[j][1][i]);
      const double v0 = u2d(swap ? v.y : v.x), v1 = u2d(swap ? v.x : v.y);
      a0 = __dadd_rn(a0, fp_mod_product(v0, u2d(k0.x), qd, qinv));
      a1 = __dadd_rn(a1, fp_mod_product(v1, u2d(k0.y), qd, qinv));
      b0 = __dadd_rn(b0, fp_mod_product(v0, u2d(k1.x), qd, qinv));
      b1 = __dadd_rn(b1, fp_mod_product(v1, u2d(k1.y), qd, qinv));
    }
    ra = make_ulonglong2(fp_canonical(fp_center(a0, qd, qinv), qd), fp_canonical(fp_center(a1, qd, qinv), qd));
    rb = make_ulonglong2(fp_canonical(fp_center(b0, qd, qinv), qd), fp_canonical(fp_center(b1, qd, qinv), qd));
  } else {
    U128 a0{0, 0}, a1{0, 0}, b0{0, 0}, b1{0, 0};
#pragma unroll
    for (int j = 0; j < BETA; ++j) {
      const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(&sx[j][so]);
      const ulonglong2 k0 = *reinterpret_cast<const ulonglong2*>(&sk[j][0][i]);
      const ulonglong2 k1 = *reinterpret_cast<const ulonglong2*>(&sk[j][1][i]);
      const uint64_t v0 = swap ? v.y : v.x, v1 = swap ? v.x : v.y;
      mac_wide(a0, v0, k0.x);
      mac_wide(a1, v1, k0.y);
      mac_wide(b0, v0, k1.x);
      mac_wide(b1, v1, k1.y);
    }
    ra = make_ulonglong2(reduce128(a0, md), reduce128(a1, md));
    rb = make_ulonglong2(reduce128(b0, md), reduce128(b1, md));
  }
  uint64_t* acc = acc_all + (size_t)m * 2 * E * N;
  *reinterpret_cast<ulonglong2*>(acc + (size_t)t * N + n) = ra;
  *reinterpret_cast<ulonglong2*>(acc + ((size_t)E + t) * N + n) = rb;
}

// one CTA stages a span whose barrier expects `expect` bytes while `issue`
// bytes are copied: with expect > issue the wait runs out (the barrier is
// never completed) and the fault counter records it, which is how the
// bounded wait is tested without a fault
__global__ void bulk_wait_probe_kernel(const uint64_t* __restrict__ src, uint64_t* __restrict__ dst, uint32_t issue,
                                       uint32_t expect, unsigned int* __restrict__ faults) {
  __shared__ alignas(128) uint64_t sx[kSpan];
  __shared__ alignas(8) uint64_t bar;
  const uint32_t mb = smem_addr(&bar);
  if (threadIdx.x == 0) mbar_init(mb, 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_expect_tx(mb, expect);
    if (issue) bulk_load(smem_addr(sx), src, issue, mb);
  }
  if (!mbar_wait_bounded(mb, 0)) {
    if (threadIdx.x == 0) atomicAdd(faults, 1u);
    mbar_wait_bounded(mb, 0);
    return;
  }
  for (uint32_t k = threadIdx.x; k < issue / sizeof(uint64_t); k += blockDim.x) dst[k] = sx[k];
}

bool bulk_inner_fits(const Context& c, int beta) { return beta >= 1 && beta <= 3 && c.N >= 2 * kSpan; }

void launch_ks_inner_bulk(const Context& c, bool multi, dim3 grid, const KsBatch& b, const uint64_t* ext, bool shared,
                          uint64_t* acc, int limbs, int beta, cudaStream_t st) {
#define CKKS_BULK_LAUNCH(BETA)                                                                        \
  launch_pdl(multi ? ks_inner_bulk_kernel<BETA, true> : ks_inner_bulk_kernel<BETA, false>, grid, kThreads, 0, st, \
             b, ext, shared, acc, limbs, c.L, c.Kx(limbs), c.P, c.logN, c.d_mods, c.d_faults)
  switch (beta) {
    case 1: CKKS_BULK_LAUNCH(1); break;
    case 2: CKKS_BULK_LAUNCH(2); break;
    default: CKKS_BULK_LAUNCH(3); break;
  }
#undef CKKS_BULK_LAUNCH
}

}  // namespace

unsigned int take_device_faults(const Context& c) {
  unsigned int v = 0;
  CKKS_CUDA(cudaMemcpyAsync(&v, c.d_faults, sizeof(v), cudaMemcpyDeviceToHost, c.stream));
  CKKS_CUDA(cudaStreamSynchronize(c.stream));
  if (v) {
    CKKS_CUDA(cudaMemsetAsync(c.d_faults, 0, sizeof(unsigned int), c.stream));
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  }
  return v;
}

void bulk_wait_probe(const Context& c, const uint64_t* src, uint64_t* dst, bool starve, cudaStream_t st) {
  bulk_wait_probe_kernel<<<1, kThreads, 0, st>>>(src, dst, kSpanBytes, starve ? 2 * kSpanBytes : kSpanBytes,
                                                 c.d_faults);
  CKKS_CUDA(cudaGetLastError());
}

// ModDown's last two steps for the items of a batch: the forward transform
// of the converted limbs with the combine step as its store
void moddown_fused(const Context& c, const KsBatch& b, const uint64_t* acc, uint64_t* conv, int limbs,
                   const ulonglong2* pinv, cudaStream_t st) {
  ModDownCombine mc{};
  mc.acc = acc;
  mc.pinv = pinv;
  mc.limbs = limbs;
  mc.E = limbs + c.Kx(limbs);
  for (int m = 0; m < b.M; ++m) {
    mc.add0[m] = b.add0[m];
    mc.add1[m] = b.add1[m];
    mc.out0[m] = b.out0[m];
    mc.out1[m] = b.out1[m];
    mc.g[m] = b.g[m];
  }
  ntt_forward_moddown(c, conv, b.M, mc, st);
}

void keyswitch_batch(const Context& c, int limbs, const KsBatch& b, bool shared, cudaStream_t st) {
  if (c.alpha > kMaxAlpha || c.Kx(limbs) > kMaxK) throw Error(kErrArgument, "digit size above 16 is not supported");
  const int M = b.M;
  if (M <= 0) return;
  if (M > kKsBatch) throw Error(kErrArgument, "key-switch batch above 32");
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  const int Mu = shared ? 1 : M;  // ModUp inputs
  const double lb = c.limb_bytes();
  uint64_t* dc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)Mu * limbs * N);
  uint64_t* ext = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)Mu * lt.beta * E * N);
  uint64_t* acc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * 2 * E * N);
  uint64_t* conv = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * 2 * limbs * N);
  // ModUp
  {  // the inverse transform reads the inputs in place (no gather copy)
    NttSource src{};
    src.per_item = limbs;
    src.limb_stride = N;
    for (int m = 0; m < Mu; ++m) src.item[m] = b.d[m];
    ntt_inverse(c, dc, Mu * limbs, LimbMap::q(limbs, c.L), st, lt.d_up_scale_a, lt.d_up_scale_b, 0, &src);
  }
  const int min_cnt = limbs - (lt.beta - 1) * c.alpha;
  const int nch_up = (E - min_cnt + kTargets - 1) / kTargets;
  {
    ProfScope ps(c, "modup_conv", Mu * (2.0 * limbs + (double)lt.beta * E) * lb, st);
    auto kern = c.alpha <= 4 ? modup_conv_batch_kernel<4>
                : c.alpha <= 8 ? modup_conv_batch_kernel<8>
                : c.alpha <= 12 ? modup_conv_batch_kernel<12>
                                : modup_conv_batch_kernel<16>;
    launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, lt.beta * nch_up, Mu), kThreads, 0, st, b, dc, ext, limbs, c.L, c.Kx(limbs), c.alpha, lt.beta, c.logN, nch_up, c.d_mods, lt.d_up_hat);
  }
  CKKS_CUDA(cudaGetLastError());
  {
    LimbMap m = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    m.skip_alpha = c.alpha;
    m.skip_beta = lt.beta;
    ntt_forward(c, ext, Mu * lt.beta * E, m, st);
  }
  // key inner products
  {
    ProfScope ps(c, "ks_inner", M * (2.0 * lt.beta * E + 2.0 * E) * lb + Mu * (double)lt.beta * E * lb, st);
    if (bulk_inner_fits(c, lt.beta))
      launch_ks_inner_bulk(c, false, dim3(N / kSpan, E, M), b, ext, shared, acc, limbs, lt.beta, st);
    else
      launch_pdl(ks_inner_batch_kernel, dim3((N / 2 + kThreads - 1) / kThreads, E, M), kThreads, 0, st, b, ext, shared, acc, limbs, c.L, c.Kx(limbs), c.P, lt.beta, c.logN, c.d_mods);
  }
  CKKS_CUDA(cudaGetLastError());
  // ModDown
  {
    LimbMap pm = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    pm.skip_q = 1;
    ntt_inverse(c, acc, M * 2 * E, pm, st, c.down_scale_a(limbs), c.down_scale_b(limbs), c.L);
  }
  const int nch_dn = (limbs + kTargets - 1) / kTargets;
  {
    ProfScope ps(c, "moddown_conv", M * (2.0 * c.Kx(limbs) + 2.0 * limbs) * lb, st);
    auto kern = c.Kx(limbs) <= 4 ? moddown_conv_batch_kernel<4>
                : c.Kx(limbs) <= 8 ? moddown_conv_batch_kernel<8>
                : c.Kx(limbs) <= 12 ? moddown_conv_batch_kernel<12>
                            : moddown_conv_batch_kernel<16>;
    launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, 2 * nch_dn, M), kThreads, 0, st, acc, conv, limbs, c.L, c.Kx(limbs), c.logN, nch_dn, c.d_mods, lt.d_down_phat);
  }
  CKKS_CUDA(cudaGetLastError());
  moddown_fused(c, b, acc, conv, limbs, lt.d_down_pinv, st);
  c.release(dc);
  c.release(ext);
  c.release(acc);
  c.release(conv);
}

void keyswitch_hoisted_multi(const Context& c, int limbs, const uint64_t* const* d, const uint64_t* const* c0,
                             int G, const HoistKeys& h, uint64_t* const* out0, uint64_t* const* out1,
                             cudaStream_t st) {
  if (c.alpha > kMaxAlpha || c.Kx(limbs) > kMaxK) throw Error(kErrArgument, "digit size above 16 is not supported");
  if (G <= 0 || h.R <= 0) return;
  if (G > kKsBatch) throw Error(kErrArgument, "hoisted rotations of more than 32 inputs");
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  const double lb = c.limb_bytes();
  // one ModUp per input
  KsBatch bu{};
  bu.M = G;
  for (int g = 0; g < G; ++g) bu.d[g] = d[g];
  uint64_t* dc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)G * limbs * N);
  uint64_t* ext = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)G * lt.beta * E * N);
  {  // the inverse transform reads the inputs in place (no gather copy)
    NttSource src{};
    src.per_item = limbs;
    src.limb_stride = N;
    for (int m = 0; m < G; ++m) src.item[m] = bu.d[m];
    ntt_inverse(c, dc, G * limbs, LimbMap::q(limbs, c.L), st, lt.d_up_scale_a, lt.d_up_scale_b, 0, &src);
  }
  const int min_cnt = limbs - (lt.beta - 1) * c.alpha;
  const int nch_up = (E - min_cnt + kTargets - 1) / kTargets;
  {
    ProfScope ps(c, "modup_conv", G * (2.0 * limbs + (double)lt.beta * E) * lb, st);
    auto kern = c.alpha <= 4 ? modup_conv_batch_kernel<4>
                : c.alpha <= 8 ? modup_conv_batch_kernel<8>
                : c.alpha <= 12 ? modup_conv_batch_kernel<12>
                                : modup_conv_batch_kernel<16>;
    launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, lt.beta * nch_up, G), kThreads, 0, st, bu, dc, ext, limbs, c.L, c.Kx(limbs), c.alpha, lt.beta, c.logN, nch_up, c.d_mods, lt.d_up_hat);
  }
  CKKS_CUDA(cudaGetLastError());
  {
    LimbMap m = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    m.skip_alpha = c.alpha;
    m.skip_beta = lt.beta;
    ntt_forward(c, ext, G * lt.beta * E, m, st);
  }
  c.release(dc);
  // items (input g, rotation r), r-major so that a key's items are adjacent;
  // up to kKsBatch items per launch sequence
  const int per = std::max(1, kKsBatch / G);  // rotations per chunk
  uint64_t* acc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)kKsBatch * 2 * E * N);
  uint64_t* conv = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)kKsBatch * 2 * limbs * N);
  for (int r0 = 0; r0 < h.R; r0 += per) {
    const int r1 = std::min(h.R, r0 + per);
    KsBatch b{};
    for (int r = r0; r < r1; ++r)
      for (int g = 0; g < G; ++g) {
        const int m = b.M++;
        b.key[m] = h.key[r];
        b.g[m] = h.g[r];
        b.src[m] = (uint8_t)g;
        b.add0[m] = c0[g];
        b.add1[m] = nullptr;
        b.out0[m] = out0[(size_t)g * h.R + r];
        b.out1[m] = out1[(size_t)g * h.R + r];
      }
    const int M = b.M;
    {
      // acc writes, each key once, the gathered ext residues
      ProfScope ps(c, "ks_inner", (M * (2.0 * E + (double)lt.beta * E) + (r1 - r0) * 2.0 * lt.beta * E) * lb, st);
      if (bulk_inner_fits(c, lt.beta))
        launch_ks_inner_bulk(c, true, dim3(M, N / kSpan, E), b, ext, false, acc, limbs, lt.beta, st);
      else
        launch_pdl(ks_inner_multi_kernel, dim3(M, (N / 2 + kThreads - 1) / kThreads, E), kThreads, 0, st, b, ext, acc, limbs, c.L, c.Kx(limbs), c.P, lt.beta, c.logN, c.d_mods);
    }
    CKKS_CUDA(cudaGetLastError());
    {
      LimbMap pm = LimbMap::ext(limbs, c.Kx(limbs), c.L);
      pm.skip_q = 1;
      ntt_inverse(c, acc, M * 2 * E, pm, st, c.down_scale_a(limbs), c.down_scale_b(limbs), c.L);
    }
    const int nch_dn = (limbs + kTargets - 1) / kTargets;
    {
      ProfScope ps(c, "moddown_conv", M * (2.0 * c.Kx(limbs) + 2.0 * limbs) * lb, st);
      auto kern = c.Kx(limbs) <= 4 ? moddown_conv_batch_kernel<4>
                  : c.Kx(limbs) <= 8 ? moddown_conv_batch_kernel<8>
                  : c.Kx(limbs) <= 12 ? moddown_conv_batch_kernel<12>
                              : moddown_conv_batch_kernel<16>;
      launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, 2 * nch_dn, M), kThreads, 0, st, acc, conv, limbs, c.L, c.Kx(limbs), c.logN, nch_dn, c.d_mods, lt.d_down_phat);
    }
    CKKS_CUDA(cudaGetLastError());
    moddown_fused(c, b, acc, conv, limbs, lt.d_down_pinv, st);
  }
  c.release(ext);
  c.release(acc);
  c.release(conv);
}

void keyswitch_sum(const Context& c, int limbs, const KsBatch& b, uint64_t* out0, uint64_t* out1, cudaStream_t st) {
  if (c.alpha > kMaxAlpha || c.Kx(limbs) > kMaxK) throw Error(kErrArgument, "digit size above 16 is not supported");
  const int M = b.M;
  if (M <= 0 || M > kKsBatch) throw Error(kErrArgument, "key-switch sum of 1..32 items");
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  const double lb = c.limb_bytes();
  uint64_t* dc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * limbs * N);
  uint64_t* ext = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * lt.beta * E * N);
  uint64_t* acc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)2 * E * N);
  uint64_t* conv = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)2 * limbs * N);
  // ModUp of every item
  {  // the inverse transform reads the inputs in place (no gather copy)
    NttSource src{};
    src.per_item = limbs;
    src.limb_stride = N;
    for (int m = 0; m < M; ++m) src.item[m] = b.d[m];
    ntt_inverse(c, dc, M * limbs, LimbMap::q(limbs, c.L), st, lt.d_up_scale_a, lt.d_up_scale_b, 0, &src);
  }
  const int min_cnt = limbs - (lt.beta - 1) * c.alpha;
  const int nch_up = (E - min_cnt + kTargets - 1) / kTargets;
  {
    ProfScope ps(c, "modup_conv", M * (2.0 * limbs + (double)lt.beta * E) * lb, st);
    auto kern = c.alpha <= 4 ? modup_conv_batch_kernel<4>
                : c.alpha <= 8 ? modup_conv_batch_kernel<8>
                : c.alpha <= 12 ? modup_conv_batch_kernel<12>
                                : modup_conv_batch_kernel<16>;
    launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, lt.beta * nch_up, M), kThreads, 0, st, b, dc, ext, limbs, c.L, c.Kx(limbs), c.alpha, lt.beta, c.logN, nch_up, c.d_mods, lt.d_up_hat);
  }
  CKKS_CUDA(cudaGetLastError());
  {
    LimbMap m = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    m.skip_alpha = c.alpha;
    m.skip_beta = lt.beta;
    ntt_forward(c, ext, M * lt.beta * E, m, st);
  }
  // summed key inner products
  {
    const int fold = 63 / lt.beta;
    ProfScope ps(c, "ks_inner_sum", (M * 3.0 * lt.beta * E + 2.0 * E) * lb, st);
    launch_pdl(ks_inner_sum_kernel, dim3((N / 2 + kThreads - 1) / kThreads, E), kThreads, 0, st, b, ext, acc, limbs, c.L, c.Kx(limbs), c.P, lt.beta, c.logN, fold, c.d_mods);
  }
  CKKS_CUDA(cudaGetLastError());
  // one ModDown
  {
    LimbMap pm = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    pm.skip_q = 1;
    ntt_inverse(c, acc, 2 * E, pm, st, c.down_scale_a(limbs), c.down_scale_b(limbs), c.L);
  }
  const int nch_dn = (limbs + kTargets - 1) / kTargets;
  {
    ProfScope ps(c, "moddown_conv", (2.0 * c.Kx(limbs) + 2.0 * limbs) * lb, st);
    auto kern = c.Kx(limbs) <= 4 ? moddown_conv_batch_kernel<4>
                : c.Kx(limbs) <= 8 ? moddown_conv_batch_kernel<8>
                : c.Kx(limbs) <= 12 ? moddown_conv_batch_kernel<12>
                            : moddown_conv_batch_kernel<16>;
    launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, 2 * nch_dn, 1), kThreads, 0, st, acc, conv, limbs, c.L, c.Kx(limbs), c.logN, nch_dn, c.d_mods, lt.d_down_phat);
  }
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, conv, 2 * limbs, LimbMap::q(limbs, c.L), st);
  {
    ProfScope ps(c, "moddown_combine_sum", (6.0 + M) * limbs * lb, st);
    launch_pdl(moddown_combine_sum_kernel, dim3((N + kThreads - 1) / kThreads, 2 * limbs), kThreads, 0, st, b, acc, conv, out0, out1, limbs, c.Kx(limbs), c.logN, c.d_mods, lt.d_down_pinv);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(dc);
  c.release(ext);
  c.release(acc);
  c.release(conv);
}

void keyswitch_sum_groups(const Context& c, int limbs, const KsBatch* bs, SumGroups& s, int G, cudaStream_t st) {
  if (c.alpha > kMaxAlpha || c.Kx(limbs) > kMaxK) throw Error(kErrArgument, "digit size above 16 is not supported");
  if (G <= 0) return;
  if (G > kSumGroups) throw Error(kErrArgument, "key-switch sums of 1..4 groups");
  const int M = bs[0].M;
  if (M <= 0 || M > kKsBatch) throw Error(kErrArgument, "key-switch sum of 1..32 items");
  for (int gi = 1; gi < G; ++gi) {
    if (bs[gi].M != M) throw Error(kErrArgument, "groups of a key-switch sum differ in length");
    for (int m = 0; m < M; ++m)
      if (bs[gi].g[m] != bs[0].g[m] || bs[gi].key[m] != bs[0].key[m])
        throw Error(kErrArgument, "groups of a key-switch sum differ in their rotations");
  }
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  const double lb = c.limb_bytes();
  const size_t item = (size_t)lt.beta * E * N;
  uint64_t* dc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * limbs * N);
  uint64_t* ext = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)G * M * item);
  uint64_t* acc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)G * 2 * E * N);
  uint64_t* conv = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)G * 2 * limbs * N);
  // ModUp of every item of every group (one launch sequence per group)
  const int min_cnt = limbs - (lt.beta - 1) * c.alpha;
  const int nch_up = (E - min_cnt + kTargets - 1) / kTargets;
  for (int gi = 0; gi < G; ++gi) {
    const KsBatch& b = bs[gi];
    uint64_t* eg = ext + (size_t)gi * M * item;
    {
      NttSource src{};
      src.per_item = limbs;
      src.limb_stride = N;
      for (int m = 0; m < M; ++m) src.item[m] = b.d[m];
      ntt_inverse(c, dc, M * limbs, LimbMap::q(limbs, c.L), st, lt.d_up_scale_a, lt.d_up_scale_b, 0, &src);
    }
    {
      ProfScope ps(c, "modup_conv", M * (2.0 * limbs + (double)lt.beta * E) * lb, st);
      auto kern = c.alpha <= 4 ? modup_conv_batch_kernel<4>
                  : c.alpha <= 8 ? modup_conv_batch_kernel<8>
                  : c.alpha <= 12 ? modup_conv_batch_kernel<12>
                                  : modup_conv_batch_kernel<16>;
      launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, lt.beta * nch_up, M), kThreads, 0, st, b, dc, eg, limbs, c.L, c.Kx(limbs), c.alpha, lt.beta, c.logN, nch_up, c.d_mods, lt.d_up_hat);
    }
    CKKS_CUDA(cudaGetLastError());
    LimbMap m = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    m.skip_alpha = c.alpha;
    m.skip_beta = lt.beta;
    ntt_forward(c, eg, M * lt.beta * E, m, st);
  }
  // summed key inner products, each key residue loaded once for all groups
  {
    HoistKeys h{};
    h.R = M;
    for (int m = 0; m < M; ++m) {
      h.key[m] = bs[0].key[m];
      h.g[m] = bs[0].g[m];
    }
    ProfScope ps(c, "ks_inner_sum", ((double)G * M * lt.beta * E + 2.0 * M * lt.beta * E + 2.0 * G * E) * lb, st);
    launch_ks_inner_hoist(c, h, ext, acc, G, limbs, lt.beta, (size_t)M * item, item, st);
  }
  CKKS_CUDA(cudaGetLastError());
  // one ModDown per group
  {
    LimbMap pm = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    pm.skip_q = 1;
    ntt_inverse(c, acc, G * 2 * E, pm, st, c.down_scale_a(limbs), c.down_scale_b(limbs), c.L);
  }
  const int nch_dn = (limbs + kTargets - 1) / kTargets;
  {
    ProfScope ps(c, "moddown_conv", G * (2.0 * c.Kx(limbs) + 2.0 * limbs) * lb, st);
    auto kern = c.Kx(limbs) <= 4 ? moddown_conv_batch_kernel<4>
                : c.Kx(limbs) <= 8 ? moddown_conv_batch_kernel<8>
                : c.Kx(limbs) <= 12 ? moddown_conv_batch_kernel<12>
                            : moddown_conv_batch_kernel<16>;
    launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, 2 * nch_dn, G), kThreads, 0, st, acc, conv, limbs, c.L, c.Kx(limbs), c.logN, nch_dn, c.d_mods, lt.d_down_phat);
  }
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, conv, G * 2 * limbs, LimbMap::q(limbs, c.L), st);
  {
    s.M = M;
    for (int m = 0; m < M; ++m) s.g[m] = bs[0].g[m];
    for (int gi = 0; gi < G; ++gi)
      for (int m = 0; m < M; ++m) s.add0[gi][m] = bs[gi].add0[m];
    double extra = 0.0;
    for (int gi = 0; gi < G; ++gi) extra += (s.id0[gi] ? 1.0 : 0.0) + (s.id1[gi] ? 1.0 : 0.0);
    ProfScope ps(c, "moddown_combine_sum", (G * (6.0 + M) + extra) * limbs * lb, st);
    launch_pdl(moddown_combine_groups_kernel, dim3((N + kThreads - 1) / kThreads, 2 * limbs, G), kThreads, 0, st, s, acc, conv, limbs, c.Kx(limbs), c.logN, c.d_mods, lt.d_down_pinv);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(dc);
  c.release(ext);
  c.release(acc);
  c.release(conv);
}

void keyswitch_hoisted_sum(const Context& c, int limbs, const KsBatch& b, const HoistKeys& h, bool identity,
                           cudaStream_t st) {
  if (c.alpha > kMaxAlpha || c.Kx(limbs) > kMaxK) throw Error(kErrArgument, "digit size above 16 is not supported");
  const int M = b.M;
  if (M <= 0) return;
  if (M > kKsBatch) throw Error(kErrArgument, "hoisted-sum batch above 32");
  if (h.R < 1 || h.R > kKsBatch) throw Error(kErrArgument, "hoisted sum of 1..32 rotations");
  const int N = c.N, E = limbs + c.Kx(limbs);
  const LevelTables& lt = c.lt(limbs);
  const double lb = c.limb_bytes();
  uint64_t* dc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * limbs * N);
  uint64_t* ext = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * lt.beta * E * N);
  uint64_t* acc = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * 2 * E * N);
  uint64_t* conv = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * 2 * limbs * N);
  // one ModUp per item
  {  // the inverse transform reads the inputs in place (no gather copy)
    NttSource src{};
    src.per_item = limbs;
    src.limb_stride = N;
    for (int m = 0; m < M; ++m) src.item[m] = b.d[m];
    ntt_inverse(c, dc, M * limbs, LimbMap::q(limbs, c.L), st, lt.d_up_scale_a, lt.d_up_scale_b, 0, &src);
  }
  const int min_cnt = limbs - (lt.beta - 1) * c.alpha;
  const int nch_up = (E - min_cnt + kTargets - 1) / kTargets;
  {
    ProfScope ps(c, "modup_conv", M * (2.0 * limbs + (double)lt.beta * E) * lb, st);
    auto kern = c.alpha <= 4 ? modup_conv_batch_kernel<4>
                : c.alpha <= 8 ? modup_conv_batch_kernel<8>
                : c.alpha <= 12 ? modup_conv_batch_kernel<12>
                                : modup_conv_batch_kernel<16>;
    launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, lt.beta * nch_up, M), kThreads, 0, st, b, dc, ext, limbs, c.L, c.Kx(limbs), c.alpha, lt.beta, c.logN, nch_up, c.d_mods, lt.d_up_hat);
  }
  CKKS_CUDA(cudaGetLastError());
  {
    LimbMap m = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    m.skip_alpha = c.alpha;
    m.skip_beta = lt.beta;
    ntt_forward(c, ext, M * lt.beta * E, m, st);
  }
  // the R key inner products of each item, summed
  {
    ProfScope ps(c, "ks_inner_hoist", (M * (lt.beta * (1.0 + 2.0 * h.R) + 2.0) * E + 2.0 * h.R * lt.beta * E) * lb,
                 st);
    launch_ks_inner_hoist(c, h, ext, acc, M, limbs, lt.beta, (size_t)lt.beta * E * N, 0, st);
  }
  CKKS_CUDA(cudaGetLastError());
  // one ModDown per item
  {
    LimbMap pm = LimbMap::ext(limbs, c.Kx(limbs), c.L);
    pm.skip_q = 1;
    ntt_inverse(c, acc, M * 2 * E, pm, st, c.down_scale_a(limbs), c.down_scale_b(limbs), c.L);
  }
  const int nch_dn = (limbs + kTargets - 1) / kTargets;
  {
    ProfScope ps(c, "moddown_conv", M * (2.0 * c.Kx(limbs) + 2.0 * limbs) * lb, st);
    auto kern = c.Kx(limbs) <= 4 ? moddown_conv_batch_kernel<4>
                : c.Kx(limbs) <= 8 ? moddown_conv_batch_kernel<8>
                : c.Kx(limbs) <= 12 ? moddown_conv_batch_kernel<12>
                            : moddown_conv_batch_kernel<16>;
    launch_pdl(kern, dim3((N / 2 + kThreads - 1) / kThreads, 2 * nch_dn, M), kThreads, 0, st, acc, conv, limbs, c.L, c.Kx(limbs), c.logN, nch_dn, c.d_mods, lt.d_down_phat);
  }
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, conv, M * 2 * limbs, LimbMap::q(limbs, c.L), st);
  {
    ProfScope ps(c, "moddown_combine_hoist", M * (6.0 + h.R + (identity ? 2.0 : 0.0)) * limbs * lb, st);
    launch_pdl(moddown_combine_hoist_kernel, dim3((N + kThreads - 1) / kThreads, 2 * limbs, M), kThreads, 0, st, b, h, identity, acc, conv, limbs, c.Kx(limbs), c.logN, c.d_mods, lt.d_down_pinv);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(dc);
  c.release(ext);
  c.release(acc);
  c.release(conv);
}

void rescale_batch(const Context& c, int limbs, const RsBatch& b, cudaStream_t st) {
  if (limbs < 2) throw Error(kErrLevel, "cannot rescale a single-limb ciphertext");
  const int M = b.M;
  if (M <= 0) return;
  if (M > kKsBatch) throw Error(kErrArgument, "rescale batch above 32");
  const int N = c.N, lo = limbs - 1;
  const LevelTables& lt = c.lt(limbs);
  const double lb = c.limb_bytes();
  uint64_t* last = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)2 * M * N);
  uint64_t* tmp = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)2 * M * lo * N);
  {  // last limb of every polynomial (2m + p), read in place by the inverse transform
    NttSource src{};
    src.per_item = 1;
    src.limb_stride = 0;
    for (int m = 0; m < M; ++m) {
      src.item[2 * m] = b.in0[m] + (size_t)lo * N;
      src.item[2 * m + 1] = b.in1[m] + (size_t)lo * N;
    }
    ntt_inverse(c, last, 2 * M, LimbMap::single(lo), st, nullptr, nullptr, 0, &src);
  }
  {  // its coefficients reduced modulo every remaining prime as the forward transform reads them
    NttSource src{};
    src.per_item = lo;
    src.limb_stride = 0;
    src.reduce = true;
    for (int i = 0; i < 2 * M; ++i) src.item[i] = last + (size_t)i * N;
    ntt_forward(c, tmp, 2 * M * lo, LimbMap::q(lo, c.L), st, &src);
  }
  {
    ProfScope ps(c, "rescale_combine", 6.0 * M * lo * lb, st);
    launch_pdl(rs_combine_batch_kernel, dim3((N + kThreads - 1) / kThreads, 2 * lo, M), kThreads, 0, st, b, tmp, limbs, c.logN, c.d_mods, lt.d_rescale_inv);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(last);
  c.release(tmp);
}

}  // namespace ckks
