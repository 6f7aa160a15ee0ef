// client.cu -- the client role of the reference driver, batched and kept on
// the device: Decrypt + GetRealPackedValue of many ciphertexts, and
// MakeCKKSPackedPlaintext + Encrypt of many slot vectors
// (fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_depth13_
//  digits3_ring65536_cpudiagcache_t123.cpp:509-715, where each refresh
// decrypts, transforms in float64 and re-encrypts one ciphertext at a time on
// the host).
//
// Item m of an encryption batch uses encryption counter c0 + m, so a batch
// produces exactly the ciphertexts of M successive single encryptions.
#include <vector>

#include "ckks_internal.hpp"

namespace ckks {

namespace {

constexpr int kThreads = 256;

uint64_t splitmix(uint64_t* x) {
  uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

struct Key8 {
  uint32_t k[8];
};

Key8 key_from_seed(uint64_t seed) {
  Key8 k;
  uint64_t s = seed;
  for (int i = 0; i < 4; ++i) {
    const uint64_t v = splitmix(&s);
    k.k[2 * i] = (uint32_t)v;
    k.k[2 * i + 1] = (uint32_t)(v >> 32);
  }
  return k;
}

__device__ __forceinline__ uint32_t rotl(uint32_t v, int n) { return (v << n) | (v >> (32 - n)); }

// the ChaCha20 block (RFC 7539 rounds, 64-bit counter in words 12-13 and
// 64-bit nonce in words 14-15) as eight 64-bit output words
__device__ void chacha_words8(const Key8& key, uint64_t nonce, uint64_t counter, uint64_t out[8]) {
  uint32_t st[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key.k[0], key.k[1], key.k[2], key.k[3],
                     key.k[4],    key.k[5],    key.k[6],    key.k[7],    (uint32_t)counter, (uint32_t)(counter >> 32),
                     (uint32_t)nonce, (uint32_t)(nonce >> 32)};
  uint32_t x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = st[i];
#define QR(a, b, c, d) \
  a += b;              \
  d ^= a;              \
  d = rotl(d, 16);     \
  c += d;              \
  b ^= c;              \
  b = rotl(b, 12);     \
  a += b;              \
  d ^= a;              \
  d = rotl(d, 8);      \
  c += d;              \
  b ^= c;              \
  b = rotl(b, 7);
#pragma unroll 1
  for (int r = 0; r < 10; ++r) {
    QR(x[0], x[4], x[8], x[12]);
    QR(x[1], x[5], x[9], x[13]);
    QR(x[2], x[6], x[10], x[14]);
    QR(x[3], x[7], x[11], x[15]);
    QR(x[0], x[5], x[10], x[15]);
    QR(x[1], x[6], x[11], x[12]);
    QR(x[2], x[7], x[8], x[13]);
    QR(x[3], x[4], x[9], x[14]);
  }
#undef QR
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = (uint64_t)(x[2 * i] + st[2 * i]) | ((uint64_t)(x[2 * i + 1] + st[2 * i + 1]) << 32);
}

// encryption randomness of item m: sub 0 ternary u, subs 1/2 centered
// binomial e0/e1 (nonce (0x20 << 56) | counter << 2 | sub, as single
// encryptions); coefficient n takes 64-bit word n % 8 of ChaCha block n / 8,
// so a thread computes one block for eight coefficients
__global__ void __launch_bounds__(kThreads) enc_sample_kernel(Key8 key, uint64_t counter0, int N,
                                                              int* __restrict__ out) {
  const int b = blockIdx.x * kThreads + threadIdx.x;
  if (b >= N / 8) return;
  const int m = blockIdx.y, sub = blockIdx.z;
  const uint64_t nonce = (0x20ull << 56) | ((counter0 + (uint64_t)m) << 2) | (uint64_t)sub;
  uint64_t w[8];
  chacha_words8(key, nonce, (uint64_t)b, w);
  int v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (sub == 0) {
      const uint64_t t = w[k] % 3ull;
      v[k] = t == 0 ? 0 : (t == 1 ? 1 : -1);
    } else {
      v[k] = __popcll(w[k] & 0x1FFFFFull) - __popcll((w[k] >> 21) & 0x1FFFFFull);
    }
  }
  int4* o = reinterpret_cast<int4*>(out + ((size_t)m * 3 + sub) * N + (size_t)8 * b);
  o[0] = make_int4(v[0], v[1], v[2], v[3]);
  o[1] = make_int4(v[4], v[5], v[6], v[7]);
}

__global__ void __launch_bounds__(kThreads) enc_spread_kernel(const int* __restrict__ v, uint64_t* __restrict__ out,
                                                              int limbs, int logN, const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int l = blockIdx.y % limbs, ms = blockIdx.y / limbs;  // ms = m * 3 + sub
  const uint64_t q = mods[l].q;
  const int x = v[(size_t)ms * N + n];
  out[((size_t)ms * limbs + l) * N + n] = x >= 0 ? (uint64_t)x : q - (uint64_t)(-x);
}

// u and e1 of item m into r ([m][2][limbs]); e0 added onto the item's
// coefficient-form plaintext
__global__ void __launch_bounds__(kThreads) enc_spread_coef_kernel(const int* __restrict__ v, uint64_t* __restrict__ r,
                                                                   uint64_t* __restrict__ pts, int limbs, int logN,
                                                                   const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int l = blockIdx.y % limbs, ms = blockIdx.y / limbs;  // ms = m * 3 + sub
  const int m = ms / 3, sub = ms % 3;
  const uint64_t q = mods[l].q;
  const int x = v[(size_t)ms * N + n];
  const uint64_t res = x >= 0 ? (uint64_t)x : q - (uint64_t)(-x);
  if (sub == 1) {
    uint64_t* p = pts + ((size_t)m * limbs + l) * N + n;
    *p = add_mod(*p, res, q);
  } else {
    r[((size_t)(2 * m + (sub >> 1)) * limbs + l) * N + n] = res;
  }
}

__global__ void __launch_bounds__(kThreads) enc_combine_coef_kernel(const uint64_t* __restrict__ pb,
                                                                    const uint64_t* __restrict__ pa,
                                                                    const uint64_t* __restrict__ r,
                                                                    const uint64_t* __restrict__ pts,
                                                                    uint64_t** c0s, uint64_t** c1s, int limbs,
                                                                    int logN, const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int l = blockIdx.y, m = blockIdx.z;
  const Mod md = mods[l];
  const size_t o_l = (size_t)l * N + n;
  const size_t S = (size_t)limbs * N;
  const uint64_t* rm = r + (size_t)m * 2 * S;  // u, e1
  const uint64_t uv = rm[o_l];
  c0s[m][o_l] = add_mod(mul_mod(pb[o_l], uv, md), pts[(size_t)m * S + o_l], md.q);
  c1s[m][o_l] = add_mod(mul_mod(pa[o_l], uv, md), rm[S + o_l], md.q);
}

struct OutPtrs {
  uint64_t** c0;
  uint64_t** c1;
};

__global__ void __launch_bounds__(kThreads) enc_combine_batch_kernel(const uint64_t* __restrict__ pb,
                                                                     const uint64_t* __restrict__ pa,
                                                                     const uint64_t* __restrict__ r,
                                                                     const uint64_t* __restrict__ pts, OutPtrs o,
                                                                     int limbs, int logN,
                                                                     const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int l = blockIdx.y, m = blockIdx.z;
  const Mod md = mods[l];
  const size_t o_l = (size_t)l * N + n;
  const size_t S = (size_t)limbs * N;
  const uint64_t* rm = r + (size_t)m * 3 * S;  // u, e0, e1
  const uint64_t uv = rm[o_l];
  o.c0[m][o_l] = add_mod(add_mod(mul_mod(pb[o_l], uv, md), rm[S + o_l], md.q), pts[(size_t)m * S + o_l], md.q);
  o.c1[m][o_l] = add_mod(mul_mod(pa[o_l], uv, md), rm[2 * S + o_l], md.q);
}

struct InPtrs {
  const uint64_t** c0;
  const uint64_t** c1;
};

// first `use` limbs of c0 + c1 * s
__global__ void __launch_bounds__(kThreads) dec_batch_kernel(InPtrs in, const uint64_t* __restrict__ s, int use,
                                                             int logN, const Mod* __restrict__ mods,
                                                             uint64_t* __restrict__ out) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int l = blockIdx.y, m = blockIdx.z;
  const Mod md = mods[l];
  const size_t o = (size_t)l * N + n;
  out[((size_t)m * use + l) * N + n] = add_mod(in.c0[m][o], mul_mod(in.c1[m][o], s[o], md), md.q);
}

template <typename T>
T* upload_async(const Context& c, const std::vector<T>& v, cudaStream_t st) {
  T* d = (T*)c.alloc(sizeof(T) * v.size());
  c.stage_upload(d, v.data(), sizeof(T) * v.size(), st);
  return d;
}

}  // namespace

// decode of `use` limbs per item from a contiguous [M][use][N] buffer of
// decrypted (NTT-form) plaintexts into M x N/2 doubles (device)
void decode_contiguous_batch(const Context& c, uint64_t* pts, int use, int M, const double* scales, double* out,
                             cudaStream_t st);

void encrypt_batch(Context& c, const uint64_t* pts, int limbs, int M, uint64_t* const* c0, uint64_t* const* c1,
                   cudaStream_t st) {
  if (!c.d_pk) throw Error(kErrState, "public key not generated");
  if (M <= 0) return;
  const int N = c.N;
  const size_t S = (size_t)limbs * N;
  int* small = (int*)c.alloc(sizeof(int) * (size_t)M * 3 * N);
  uint64_t* r = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * 3 * S);
  const uint64_t counter0 = c.enc_counter;
  c.enc_counter += (uint64_t)M;
  {
    ProfScope ps(c, "enc_sample", 12.0 * M * N, st);
    enc_sample_kernel<<<dim3((N / 8 + kThreads - 1) / kThreads, M, 3), kThreads, 0, st>>>(
        key_from_seed(c.params.seed), counter0, N, small);
    enc_spread_kernel<<<dim3((N + kThreads - 1) / kThreads, 3 * M * limbs), kThreads, 0, st>>>(small, r, limbs,
                                                                                               c.logN, c.d_mods);
  }
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, r, M * 3 * limbs, LimbMap::q(limbs, c.L), st);
  std::vector<uint64_t*> h0(c0, c0 + M), h1(c1, c1 + M);
  uint64_t** d0 = upload_async(c, h0, st);
  uint64_t** d1 = upload_async(c, h1, st);
  {
    ProfScope ps(c, "enc_combine", 7.0 * M * limbs * c.limb_bytes(), st);
    enc_combine_batch_kernel<<<dim3((N + kThreads - 1) / kThreads, limbs, M), kThreads, 0, st>>>(
        c.d_pk, c.d_pk + (size_t)c.L * N, r, pts, OutPtrs{d0, d1}, limbs, c.logN, c.d_mods);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(small);
  c.release(r);
  c.release(d0);
  c.release(d1);
}

void encrypt_batch_coef(Context& c, uint64_t* pts, int limbs, int M, uint64_t* const* c0, uint64_t* const* c1,
                        cudaStream_t st) {
  if (!c.d_pk) throw Error(kErrState, "public key not generated");
  if (M <= 0) return;
  const int N = c.N;
  const size_t S = (size_t)limbs * N;
  int* small = (int*)c.alloc(sizeof(int) * (size_t)M * 3 * N);
  uint64_t* r = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * 2 * S);
  const uint64_t counter0 = c.enc_counter;
  c.enc_counter += (uint64_t)M;
  {
    ProfScope ps(c, "enc_sample", 12.0 * M * N, st);
    enc_sample_kernel<<<dim3((N / 8 + kThreads - 1) / kThreads, M, 3), kThreads, 0, st>>>(
        key_from_seed(c.params.seed), counter0, N, small);
    enc_spread_coef_kernel<<<dim3((N + kThreads - 1) / kThreads, 3 * M * limbs), kThreads, 0, st>>>(
        small, r, pts, limbs, c.logN, c.d_mods);
  }
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, r, M * 2 * limbs, LimbMap::q(limbs, c.L), st);
  ntt_forward(c, pts, M * limbs, LimbMap::q(limbs, c.L), st);
  std::vector<uint64_t*> h0(c0, c0 + M), h1(c1, c1 + M);
  uint64_t** d0 = upload_async(c, h0, st);
  uint64_t** d1 = upload_async(c, h1, st);
  {
    ProfScope ps(c, "enc_combine", 6.0 * M * limbs * c.limb_bytes(), st);
    enc_combine_coef_kernel<<<dim3((N + kThreads - 1) / kThreads, limbs, M), kThreads, 0, st>>>(
        c.d_pk, c.d_pk + (size_t)c.L * N, r, pts, d0, d1, limbs, c.logN, c.d_mods);
  }
  CKKS_CUDA(cudaGetLastError());
  c.release(small);
  c.release(r);
  c.release(d0);
  c.release(d1);
}

void decrypt_decode_batch(const Context& c, const uint64_t* const* c0, const uint64_t* const* c1, int limbs, int M,
                          const double* scales_host, double* out, cudaStream_t st) {
  if (!c.d_sk) throw Error(kErrState, "secret key not generated");
  if (M <= 0) return;
  const int N = c.N;
  const int use = limbs >= 2 ? 2 : 1;
  uint64_t* pts = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)M * use * N);
  std::vector<const uint64_t*> h0(c0, c0 + M), h1(c1, c1 + M);
  const uint64_t** d0 = upload_async(c, h0, st);
  const uint64_t** d1 = upload_async(c, h1, st);
  {
    ProfScope ps(c, "dec_batch", 3.0 * M * use * c.limb_bytes(), st);
    dec_batch_kernel<<<dim3((N + kThreads - 1) / kThreads, use, M), kThreads, 0, st>>>(InPtrs{d0, d1}, c.d_sk, use,
                                                                                        c.logN, c.d_mods, pts);
  }
  CKKS_CUDA(cudaGetLastError());
  std::vector<double> hs(scales_host, scales_host + M);
  double* ds = upload_async(c, hs, st);
  decode_contiguous_batch(c, pts, use, M, ds, out, st);
  c.release(pts);
  c.release(d0);
  c.release(d1);
  c.release(ds);
}

}  // namespace ckks
