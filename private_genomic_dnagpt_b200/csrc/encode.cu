// encode.cu -- CKKS canonical embedding on the device: MakeCKKSPackedPlaintext
// (encode) and Decrypt's GetRealPackedValue (decode) for N/2 real slots.
//
// Slot j of a plaintext m(X) is m(zeta^(5^j)), zeta = exp(2 pi i / 2N).  The
// encoder runs the HEAAN "special" inverse FFT over the 5^j orbit, divides by
// n = N/2, multiplies by the scale and rounds half-to-even; coefficient i comes
// from the real part of entry i and coefficient i + n from its imaginary part.
// Every floating-point step is an explicit _rn intrinsic in a fixed order, the
// same order the CPU restatement uses, so encodings agree bit for bit.
// Stages whose butterfly span fits in 2048 entries run in shared memory; the
// wider ones run one launch per stage.
#include "ckks_internal.hpp"

namespace ckks {

namespace {

constexpr int kThreads = 256;
constexpr int kSmemLen = 2048;  // complex entries staged per CTA (32 KB)

__device__ __forceinline__ double2 cmul_rn(double2 a, double2 b) {
  const double t1 = __dmul_rn(a.x, b.x);
  const double t2 = __dmul_rn(a.y, b.y);
  const double t3 = __dmul_rn(a.x, b.y);
  const double t4 = __dmul_rn(a.y, b.x);
  return make_double2(__dsub_rn(t1, t2), __dadd_rn(t3, t4));
}

// Spans, the cyclotomic order M and the twiddle stride are powers of two:
// indices come from shifts and masks (lg = log2 span, lm = log2 M).
// inverse butterfly at (i, j) of span 2^lg: u = a + b, v = (a - b) * ksi[idx]
__device__ __forceinline__ void inv_bfly(double2& a, double2& b, const double2* ksi, uint32_t rg, int lg, int lm) {
  const uint32_t lenq = 4u << lg;
  const int idx = (int)((lenq - (rg & (lenq - 1u))) << (lm - lg - 2));
  const double2 u = make_double2(__dadd_rn(a.x, b.x), __dadd_rn(a.y, b.y));
  const double2 d = make_double2(__dsub_rn(a.x, b.x), __dsub_rn(a.y, b.y));
  a = u;
  b = cmul_rn(d, __ldg(ksi + idx));
}

// forward butterfly: t = b * ksi[idx]; a' = a + t; b' = a - t
__device__ __forceinline__ void fwd_bfly(double2& a, double2& b, const double2* ksi, uint32_t rg, int lg, int lm) {
  const uint32_t lenq = 4u << lg;
  const int idx = (int)((rg & (lenq - 1u)) << (lm - lg - 2));
  const double2 t = cmul_rn(b, __ldg(ksi + idx));
  const double2 u = a;
  a = make_double2(__dadd_rn(u.x, t.x), __dadd_rn(u.y, t.y));
  b = make_double2(__dsub_rn(u.x, t.x), __dsub_rn(u.y, t.y));
}

__global__ void __launch_bounds__(kThreads) fft_stage_kernel(double2* __restrict__ v, int n, int lg, bool inverse,
                                                             const double2* __restrict__ ksi,
                                                             const uint32_t* __restrict__ rot_group, int lm) {
  const int p = blockIdx.x * kThreads + threadIdx.x;
  if (p >= n / 2) return;
  const int lenh = 1 << (lg - 1);
  const int i = (p >> (lg - 1)) << lg, j = p & (lenh - 1);
  double2* vec = v + (size_t)blockIdx.y * n;
  double2 a = vec[i + j], b = vec[i + j + lenh];
  const uint32_t rg = __ldg(rot_group + j);
  if (inverse)
    inv_bfly(a, b, ksi, rg, lg, lm);
  else
    fwd_bfly(a, b, ksi, rg, lg, lm);
  vec[i + j] = a;
  vec[i + j + lenh] = b;
}

// The G stages with span above 2^lb (lg = lb+1 .. lb+G) in registers: they
// only combine entries whose indices differ in bits lb .. lb+G-1, so the
// 2^G entries lo + hi 2^lb (hi = 0 .. 2^G - 1) of each lo < 2^lb form a
// closed group.  One thread applies the G stages to its group in the
// stage kernel's order (inverse: largest span first), with the same
// butterflies and twiddles, so the results are those of G stage passes.
template <int G, bool INV>
__global__ void __launch_bounds__(kThreads) fft_outer_kernel(double2* __restrict__ v, int n, int lb,
                                                             const double2* __restrict__ ksi,
                                                             const uint32_t* __restrict__ rot_group, int lm) {
  constexpr int R = 1 << G;
  const int lo = blockIdx.x * kThreads + threadIdx.x;
  if (lo >= (1 << lb)) return;
  double2* vec = v + (size_t)blockIdx.y * n;
  double2 x[R];
#pragma unroll
  for (int h = 0; h < R; ++h) x[h] = vec[((size_t)h << lb) + lo];
#pragma unroll
  for (int it = 0; it < G; ++it) {
    const int s = INV ? (G - 1 - it) : it;  // stage lg = lb + 1 + s
    const int lg = lb + 1 + s;
#pragma unroll
    for (int h = 0; h < R; ++h) {
      if (h & (1 << s)) continue;
      const int j = ((h & ((1 << s) - 1)) << lb) + lo;  // index within the span
      const uint32_t rg = __ldg(rot_group + j);
      if constexpr (INV)
        inv_bfly(x[h], x[h | (1 << s)], ksi, rg, lg, lm);
      else
        fwd_bfly(x[h], x[h | (1 << s)], ksi, rg, lg, lm);
    }
  }
#pragma unroll
  for (int h = 0; h < R; ++h) vec[((size_t)h << lb) + lo] = x[h];
}

// all stages with span <= blk inside one aligned block of blk entries
__global__ void __launch_bounds__(kThreads) fft_smem_kernel(double2* __restrict__ v, int n, int lb, bool inverse,
                                                            const double2* __restrict__ ksi,
                                                            const uint32_t* __restrict__ rot_group, int lm) {
  __shared__ double2 s[kSmemLen];
  const int blk = 1 << lb;
  double2* vec = v + (size_t)blockIdx.y * n + (size_t)blockIdx.x * blk;
  for (int e = threadIdx.x; e < blk; e += kThreads) s[e] = vec[e];
  __syncthreads();
  if (inverse) {
    for (int lg = lb; lg >= 1; --lg) {
      const int lenh = 1 << (lg - 1);
      for (int p = threadIdx.x; p < blk / 2; p += kThreads) {
        const int i = (p >> (lg - 1)) << lg, j = p & (lenh - 1);
        inv_bfly(s[i + j], s[i + j + lenh], ksi, __ldg(rot_group + j), lg, lm);
      }
      __syncthreads();
    }
  } else {
    for (int lg = 1; lg <= lb; ++lg) {
      const int lenh = 1 << (lg - 1);
      for (int p = threadIdx.x; p < blk / 2; p += kThreads) {
        const int i = (p >> (lg - 1)) << lg, j = p & (lenh - 1);
        fwd_bfly(s[i + j], s[i + j + lenh], ksi, __ldg(rot_group + j), lg, lm);
      }
      __syncthreads();
    }
  }
  for (int e = threadIdx.x; e < blk; e += kThreads) vec[e] = s[e];
}

__global__ void __launch_bounds__(kThreads) load_real_kernel(const double* __restrict__ in, double2* __restrict__ v,
                                                             int n) {
  const int j = blockIdx.x * kThreads + threadIdx.x;
  if (j >= n) return;
  v[(size_t)blockIdx.y * n + j] = make_double2(in[(size_t)blockIdx.y * n + j], 0.0);
}

// residue of an integer-valued double: direct below 2^63, else mant * 2^e
__device__ uint64_t double_to_res(double r, const Mod& m) {
  const double ar = fabs(r);
  uint64_t v;
  if (ar < 9223372036854775808.0) {
    v = reduce128(U128{(uint64_t)ar, 0}, m);
  } else {
    const uint64_t bits = (uint64_t)__double_as_longlong(ar);
    const int e = (int)((bits >> 52) & 0x7FF) - 1075;
    const uint64_t mant = (bits & ((1ull << 52) - 1)) | (1ull << 52);
    uint64_t p2 = 1, base = 2 % m.q;
    for (int k = e; k; k >>= 1) {
      if (k & 1) p2 = mul_mod(p2, base, m);
      base = mul_mod(base, base, m);
    }
    v = mul_mod(reduce128(U128{mant, 0}, m), p2, m);
  }
  return (r < 0.0 && v) ? m.q - v : v;
}

// bit reversal, /n, *scale, round half-to-even, RNS residues (coefficient form)
__global__ void __launch_bounds__(kThreads) round_kernel(const double2* __restrict__ v, int n, int logn, double scale,
                                                         uint64_t* __restrict__ out, size_t out_stride, int limbs,
                                                         const Mod* __restrict__ mods) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= n) return;
  const int N = 2 * n;
  const double2 w = v[(size_t)blockIdx.y * n + bit_reverse((uint32_t)i, logn)];
  const double dn = (double)n;
  const double re = rint(__dmul_rn(__ddiv_rn(w.x, dn), scale));
  const double im = rint(__dmul_rn(__ddiv_rn(w.y, dn), scale));
  uint64_t* o = out + (size_t)blockIdx.y * out_stride;
  for (int l = 0; l < limbs; ++l) {
    const Mod m = mods[l];
    o[(size_t)l * N + i] = double_to_res(re, m);
    o[(size_t)l * N + i + n] = double_to_res(im, m);
  }
}

// centered CRT of the first one or two limbs -> double / scale, packed as
// w_j = (d_j, d_{j+n}) in bit-reversed position for the forward FFT
__global__ void __launch_bounds__(kThreads) crt_kernel(const uint64_t* __restrict__ x, int use, double scale,
                                                       double2* __restrict__ v, int n, int logn,
                                                       const Mod* __restrict__ mods, ulonglong2 q0inv1) {
  const int j = blockIdx.x * kThreads + threadIdx.x;
  if (j >= n) return;
  const int N = 2 * n;
  const Mod m0 = mods[0], m1 = mods[1];
  double d[2];
  for (int h = 0; h < 2; ++h) {
    const int i = j + h * n;
    U128 val, Q;
    if (use == 2) {
      const uint64_t x0 = x[i], x1 = x[(size_t)N + i];
      const uint64_t t = mul_shoup(sub_mod(x1, reduce128(U128{x0, 0}, m1), m1.q), q0inv1.x, q0inv1.y, m1.q);
      val = mul_wide(m0.q, t);
      const uint64_t lo = val.lo + x0;
      val.hi += lo < x0 ? 1ull : 0ull;
      val.lo = lo;
      Q = mul_wide(m0.q, m1.q);
    } else {
      val = U128{x[i], 0};
      Q = U128{m0.q, 0};
    }
    const U128 half{(Q.lo >> 1) | (Q.hi << 63), Q.hi >> 1};
    const bool neg = (val.hi > half.hi) || (val.hi == half.hi && val.lo > half.lo);
    U128 mag = val;
    if (neg) {
      mag.lo = Q.lo - val.lo;
      mag.hi = Q.hi - val.hi - (Q.lo < val.lo ? 1ull : 0ull);
    }
    double r = __dadd_rn(__dmul_rn(__ull2double_rn(mag.hi), 18446744073709551616.0), __ull2double_rn(mag.lo));
    if (neg) r = -r;
    d[h] = __ddiv_rn(r, scale);
  }
  v[bit_reverse((uint32_t)j, logn)] = make_double2(d[0], d[1]);
}

// batched form: item m reads x + m*use*N with scale scales[m] and writes
// v + m*n (bit-reversed positions)
__global__ void __launch_bounds__(kThreads) crt_batch_kernel(const uint64_t* __restrict__ x_all, int use,
                                                             const double* __restrict__ scales,
                                                             double2* __restrict__ v_all, int n, int logn,
                                                             const Mod* __restrict__ mods, ulonglong2 q0inv1) {
  const int j = blockIdx.x * kThreads + threadIdx.x;
  if (j >= n) return;
  const int m = blockIdx.y;
  const int N = 2 * n;
  const uint64_t* x = x_all + (size_t)m * use * N;
  const double scale = scales[m];
  const Mod m0 = mods[0], m1 = mods[1];
  double d[2];
  for (int h = 0; h < 2; ++h) {
    const int i = j + h * n;
    U128 val, Q;
    if (use == 2) {
      const uint64_t x0 = x[i], x1 = x[(size_t)N + i];
      const uint64_t t = mul_shoup(sub_mod(x1, reduce128(U128{x0, 0}, m1), m1.q), q0inv1.x, q0inv1.y, m1.q);
      val = mul_wide(m0.q, t);
      const uint64_t lo = val.lo + x0;
      val.hi += lo < x0 ? 1ull : 0ull;
      val.lo = lo;
      Q = mul_wide(m0.q, m1.q);
    } else {
      val = U128{x[i], 0};
      Q = U128{m0.q, 0};
    }
    const U128 half{(Q.lo >> 1) | (Q.hi << 63), Q.hi >> 1};
    const bool neg = (val.hi > half.hi) || (val.hi == half.hi && val.lo > half.lo);
    U128 mag = val;
    if (neg) {
      mag.lo = Q.lo - val.lo;
      mag.hi = Q.hi - val.hi - (Q.lo < val.lo ? 1ull : 0ull);
    }
    double r = __dadd_rn(__dmul_rn(__ull2double_rn(mag.hi), 18446744073709551616.0), __ull2double_rn(mag.lo));
    if (neg) r = -r;
    d[h] = __ddiv_rn(r, scale);
  }
  v_all[(size_t)m * n + bit_reverse((uint32_t)j, logn)] = make_double2(d[0], d[1]);
}

__global__ void __launch_bounds__(kThreads) take_real_batch_kernel(const double2* __restrict__ v,
                                                                   double* __restrict__ out, int n) {
  const int j = blockIdx.x * kThreads + threadIdx.x;
  if (j >= n) return;
  out[(size_t)blockIdx.y * n + j] = v[(size_t)blockIdx.y * n + j].x;
}

__global__ void __launch_bounds__(kThreads) take_real_kernel(const double2* __restrict__ v, double* __restrict__ out,
                                                             int n) {
  const int j = blockIdx.x * kThreads + threadIdx.x;
  if (j >= n) return;
  out[j] = v[j].x;
}

constexpr int kSmemLog = 11;  // log2 kSmemLen

// the stages with span above 2^lb: one register pass for up to 5 of them
// (logN <= 17), else one pass per stage
void fft_outer(const Context& c, double2* v, int batch, int lb, int ln, bool inverse, cudaStream_t st) {
  const int G = ln - lb, n = 1 << ln, lm = c.logN + 1;
  if (G <= 0) return;
  const dim3 grid(((1 << lb) + kThreads - 1) / kThreads, batch);
#define CKKS_FFT_OUTER(GG)                                                                           \
  (inverse ? fft_outer_kernel<GG, true> : fft_outer_kernel<GG, false>)<<<grid, kThreads, 0, st>>>( \
      v, n, lb, c.d_ksi, c.d_rot_group, lm)
  switch (G) {
    case 1: CKKS_FFT_OUTER(1); return;
    case 2: CKKS_FFT_OUTER(2); return;
    case 3: CKKS_FFT_OUTER(3); return;
    case 4: CKKS_FFT_OUTER(4); return;
    case 5: CKKS_FFT_OUTER(5); return;
    default: break;
  }
#undef CKKS_FFT_OUTER
  for (int k = 0; k < G; ++k) {
    const int lg = inverse ? ln - k : lb + 1 + k;
    fft_stage_kernel<<<dim3((n / 2 + kThreads - 1) / kThreads, batch), kThreads, 0, st>>>(v, n, lg, inverse, c.d_ksi,
                                                                                          c.d_rot_group, lm);
  }
}

void fft_inverse_batch(const Context& c, double2* v, int batch, cudaStream_t st) {
  const int ln = c.logN - 1, n = 1 << ln, lm = c.logN + 1;
  const int lb = ln < kSmemLog ? ln : kSmemLog;
  fft_outer(c, v, batch, lb, ln, true, st);
  fft_smem_kernel<<<dim3(n >> lb, batch), kThreads, 0, st>>>(v, n, lb, true, c.d_ksi, c.d_rot_group, lm);
  CKKS_CUDA(cudaGetLastError());
}

void fft_forward_batch(const Context& c, double2* v, int batch, cudaStream_t st) {
  const int ln = c.logN - 1, n = 1 << ln, lm = c.logN + 1;
  const int lb = ln < kSmemLog ? ln : kSmemLog;
  fft_smem_kernel<<<dim3(n >> lb, batch), kThreads, 0, st>>>(v, n, lb, false, c.d_ksi, c.d_rot_group, lm);
  fft_outer(c, v, batch, lb, ln, false, st);
  CKKS_CUDA(cudaGetLastError());
}

}  // namespace

// values: batch x n doubles (device); out: batch polys of `limbs` limbs at
// out_stride words apart, NTT form
void encode_batch(const Context& c, const double* d_values, int batch, int limbs, double scale, uint64_t* out,
                  size_t out_stride, cudaStream_t st, bool ntt) {
  const int n = c.N / 2;
  double2* v = (double2*)c.alloc(sizeof(double2) * (size_t)batch * n);
  const dim3 g((n + kThreads - 1) / kThreads, batch);
  {
    ProfScope ps(c, "encode_fft", 2.0 * 16.0 * n * batch, st);
    load_real_kernel<<<g, kThreads, 0, st>>>(d_values, v, n);
    fft_inverse_batch(c, v, batch, st);
  }
  {
    ProfScope ps(c, "encode_round", (16.0 * n + 8.0 * 2 * n * limbs) * batch, st);
    round_kernel<<<g, kThreads, 0, st>>>(v, n, c.logN - 1, scale, out, out_stride, limbs, c.d_mods);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(v);
  if (!ntt) return;  // coefficient form, for encrypt_batch_coef
  if (out_stride == (size_t)limbs * c.N) {
    ntt_forward(c, out, batch * limbs, LimbMap::q(limbs, c.L), st);  // one launch pair for the batch
  } else {
    for (int b = 0; b < batch; ++b) ntt_forward(c, out + (size_t)b * out_stride, limbs, LimbMap::q(limbs, c.L), st);
  }
}

void encode(const Context& c, const double* d_values, int limbs, double scale, uint64_t* out, cudaStream_t st) {
  encode_batch(c, d_values, 1, limbs, scale, out, (size_t)limbs * c.N, st);
}

void decode_contiguous_batch(const Context& c, uint64_t* pts, int use, int M, const double* scales, double* out,
                             cudaStream_t st) {
  const int n = c.N / 2;
  ntt_inverse(c, pts, M * use, LimbMap::q(use, c.L), st);
  double2* v = (double2*)c.alloc(sizeof(double2) * (size_t)M * n);
  const uint64_t q0 = c.moduli[0], q1 = c.moduli[1];
  unsigned __int128 inv = 1, b = q0 % q1;
  for (uint64_t e = q1 - 2; e; e >>= 1) {
    if (e & 1) inv = (inv * b) % q1;
    b = (b * b) % q1;
  }
  const uint64_t iv = (uint64_t)inv;
  const ulonglong2 q0inv1 = make_ulonglong2(iv, (uint64_t)(((unsigned __int128)iv << 64) / q1));
  const dim3 g((n + kThreads - 1) / kThreads, M);
  crt_batch_kernel<<<g, kThreads, 0, st>>>(pts, use, scales, v, n, c.logN - 1, c.d_mods, q0inv1);
  CKKS_CUDA(cudaGetLastError());
  fft_forward_batch(c, v, M, st);
  take_real_batch_kernel<<<g, kThreads, 0, st>>>(v, out, n);
  CKKS_CUDA(cudaGetLastError());
  c.release(v);
}

void decode(const Context& c, const uint64_t* pt, int limbs, double scale, double* d_values, cudaStream_t st) {
  const int n = c.N / 2, N = c.N;
  const int use = limbs >= 2 ? 2 : 1;
  uint64_t* x = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)use * N);
  CKKS_CUDA(cudaMemcpyAsync(x, pt, sizeof(uint64_t) * (size_t)use * N, cudaMemcpyDeviceToDevice, st));
  ntt_inverse(c, x, use, LimbMap::q(use, c.L), st);
  double2* v = (double2*)c.alloc(sizeof(double2) * (size_t)n);
  const uint64_t q0 = c.moduli[0], q1 = c.moduli[1];
  unsigned __int128 inv = 1, b = q0 % q1;
  for (uint64_t e = q1 - 2; e; e >>= 1) {
    if (e & 1) inv = (inv * b) % q1;
    b = (b * b) % q1;
  }
  const uint64_t iv = (uint64_t)inv;
  const ulonglong2 q0inv1 = make_ulonglong2(iv, (uint64_t)(((unsigned __int128)iv << 64) / q1));
  crt_kernel<<<(n + kThreads - 1) / kThreads, kThreads, 0, st>>>(x, use, scale, v, n, c.logN - 1, c.d_mods, q0inv1);
  CKKS_CUDA(cudaGetLastError());
  fft_forward_batch(c, v, 1, st);
  take_real_kernel<<<(n + kThreads - 1) / kThreads, kThreads, 0, st>>>(v, d_values, n);
  CKKS_CUDA(cudaGetLastError());
  c.release(x);
  c.release(v);
}

}  // namespace ckks
