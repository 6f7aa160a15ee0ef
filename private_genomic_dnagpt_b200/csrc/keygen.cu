// keygen.cu -- seeded sampling, KeyGen / EvalMultKeyGen / EvalRotateKeyGen,
// Encrypt and Decrypt on the device.
//
// Restates the client/setup role of the reference driver
// (fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_depth13_
//  digits3_ring65536_cpudiagcache_t123.cpp:1622-1624 KeyGen/EvalMultKeyGen/
//  EvalRotateKeyGen, :514-531 Decrypt/Encrypt at the client boundary).
// Randomness: one ChaCha20 block (RFC 7539 block function, 64-bit counter and
// 64-bit nonce) per sampled element; the 256-bit key is expanded from the
// 64-bit context seed with splitmix64.  Secret and encryption masks are
// uniform ternary, errors centered binomial with 21+21 bits (sigma ~3.24),
// uniform residues use 128 random bits reduced mod q.  Nonces separate the
// streams: 1 secret, 2/3 public key a/e, (0x10<<36 | id<<8 | j<<1 | part) for
// switching-key digit j, (0x20<<56 | counter<<2 | sub) for the counter-th
// encryption.
#include "ckks_internal.hpp"

namespace ckks {

namespace {

constexpr int kThreads = 256;

struct ChachaKey {
  uint32_t k[8];
};

uint64_t splitmix(uint64_t* x) {
  uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

ChachaKey key_from_seed(uint64_t seed) {
  ChachaKey k;
  uint64_t s = seed;
  for (int i = 0; i < 4; ++i) {
    const uint64_t v = splitmix(&s);
    k.k[2 * i] = (uint32_t)v;
    k.k[2 * i + 1] = (uint32_t)(v >> 32);
  }
  return k;
}

__device__ __forceinline__ uint32_t rotl32(uint32_t v, int n) { return (v << n) | (v >> (32 - n)); }

#define CKKS_QR(a, b, c, d) \
  a += b;                   \
  d ^= a;                   \
  d = rotl32(d, 16);        \
  c += d;                   \
  b ^= c;                   \
  b = rotl32(b, 12);        \
  a += b;                   \
  d ^= a;                   \
  d = rotl32(d, 8);         \
  c += d;                   \
  b ^= c;                   \
  b = rotl32(b, 7);

__device__ void chacha_words(const ChachaKey& key, uint64_t nonce, uint64_t counter, uint64_t& w0, uint64_t& w1) {
  uint32_t st[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key.k[0], key.k[1], key.k[2], key.k[3],
                     key.k[4],    key.k[5],    key.k[6],    key.k[7],    (uint32_t)counter, (uint32_t)(counter >> 32),
                     (uint32_t)nonce, (uint32_t)(nonce >> 32)};
  uint32_t x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = st[i];
#pragma unroll 1
  for (int r = 0; r < 10; ++r) {
    CKKS_QR(x[0], x[4], x[8], x[12]);
    CKKS_QR(x[1], x[5], x[9], x[13]);
    CKKS_QR(x[2], x[6], x[10], x[14]);
    CKKS_QR(x[3], x[7], x[11], x[15]);
    CKKS_QR(x[0], x[5], x[10], x[15]);
    CKKS_QR(x[1], x[6], x[11], x[12]);
    CKKS_QR(x[2], x[7], x[8], x[13]);
    CKKS_QR(x[3], x[4], x[9], x[14]);
  }
  w0 = (uint64_t)(x[0] + st[0]) | ((uint64_t)(x[1] + st[1]) << 32);
  w1 = (uint64_t)(x[2] + st[2]) | ((uint64_t)(x[3] + st[3]) << 32);
}

// the whole block as eight 64-bit words (the encryption sampler's layout)
__device__ void chacha_words8(const ChachaKey& key, uint64_t nonce, uint64_t counter, uint64_t w[8]) {
  uint32_t st[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key.k[0], key.k[1], key.k[2], key.k[3],
                     key.k[4],    key.k[5],    key.k[6],    key.k[7],    (uint32_t)counter, (uint32_t)(counter >> 32),
                     (uint32_t)nonce, (uint32_t)(nonce >> 32)};
  uint32_t x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = st[i];
#pragma unroll 1
  for (int r = 0; r < 10; ++r) {
    CKKS_QR(x[0], x[4], x[8], x[12]);
    CKKS_QR(x[1], x[5], x[9], x[13]);
    CKKS_QR(x[2], x[6], x[10], x[14]);
    CKKS_QR(x[3], x[7], x[11], x[15]);
    CKKS_QR(x[0], x[5], x[10], x[15]);
    CKKS_QR(x[1], x[6], x[11], x[12]);
    CKKS_QR(x[2], x[7], x[8], x[13]);
    CKKS_QR(x[3], x[4], x[9], x[14]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = (uint64_t)(x[2 * i] + st[2 * i]) | ((uint64_t)(x[2 * i + 1] + st[2 * i + 1]) << 32);
}

constexpr uint64_t kNonceSk = 0x01ull;
constexpr uint64_t kNoncePkA = 0x02ull;
constexpr uint64_t kNoncePkE = 0x03ull;
inline uint64_t nonce_ksk(uint32_t id, int j, int part) {
  return (0x10ull << 36) | ((uint64_t)id << 8) | ((uint64_t)j << 1) | (uint64_t)part;
}
// switching keys over the reduced special-prime set
inline uint64_t nonce_ksk_low(uint32_t id, int part) {
  return (0x11ull << 36) | ((uint64_t)id << 8) | (uint64_t)part;
}
inline uint64_t nonce_enc(uint64_t cnt, int sub) { return (0x20ull << 56) | (cnt << 2) | (uint64_t)sub; }

// kind 0: uniform ternary from w0 mod 3; kind 1: centered binomial 21+21
__global__ void __launch_bounds__(kThreads) sample_small_kernel(int* __restrict__ out, ChachaKey key, uint64_t nonce,
                                                                int N, int kind) {
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  uint64_t w0, w1;
  chacha_words(key, nonce, (uint64_t)n, w0, w1);
  int v;
  if (kind == 0) {
    const uint64_t t = w0 % 3ull;
    v = t == 0 ? 0 : (t == 1 ? 1 : -1);
  } else {
    v = __popcll(w0 & 0x1FFFFFull) - __popcll((w0 >> 21) & 0x1FFFFFull);
  }
  out[n] = v;
}

// encryption randomness: coefficient n from 64-bit word n % 8 of block n / 8
// (the same sampling as the batched encryption, one thread per block)
__global__ void __launch_bounds__(kThreads) sample_small_wide_kernel(int* __restrict__ out, ChachaKey key,
                                                                     uint64_t nonce, int N, int kind) {
  const int b = blockIdx.x * kThreads + threadIdx.x;
  if (b >= N / 8) return;
  uint64_t w[8];
  chacha_words8(key, nonce, (uint64_t)b, w);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    int v;
    if (kind == 0) {
      const uint64_t t = w[k] % 3ull;
      v = t == 0 ? 0 : (t == 1 ? 1 : -1);
    } else {
      v = __popcll(w[k] & 0x1FFFFFull) - __popcll((w[k] >> 21) & 0x1FFFFFull);
    }
    out[8 * b + k] = v;
  }
}

__global__ void __launch_bounds__(kThreads) small_to_limbs_kernel(const int* __restrict__ v, uint64_t* __restrict__ out,
                                                                  LimbMap map, int logN,
                                                                  const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const uint64_t q = mods[map.prime(blockIdx.y)].q;
  const int x = v[n];
  out[(size_t)blockIdx.y * N + n] = x >= 0 ? (uint64_t)x : q - (uint64_t)(-x);
}

// uniform residue of prime(limb) with counter prime*N + n (NTT form directly)
__global__ void __launch_bounds__(kThreads) uniform_kernel(uint64_t* __restrict__ out, ChachaKey key, uint64_t nonce,
                                                           LimbMap map, int logN, const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int pr = map.prime(blockIdx.y);
  uint64_t w0, w1;
  chacha_words(key, nonce, (uint64_t)pr * N + n, w0, w1);
  out[(size_t)blockIdx.y * N + n] = reduce128(U128{w1, w0}, mods[pr]);
}

// b = e - a*s (+ P*s_from on the digit's Q limbs)
__global__ void __launch_bounds__(kThreads) rlwe_combine_kernel(const uint64_t* __restrict__ e,
                                                                const uint64_t* __restrict__ a,
                                                                const uint64_t* __restrict__ s,
                                                                const uint64_t* __restrict__ s_from,
                                                                const ulonglong2* __restrict__ pmod, int lo, int hi,
                                                                uint64_t* __restrict__ b, int logN,
                                                                const Mod* __restrict__ mods, int first) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int t = first + blockIdx.y;
  const Mod m = mods[t];
  const size_t o = (size_t)t * N + n;
  uint64_t bv = sub_mod(e[o], mul_mod(a[o], s[o], m), m.q);
  if (s_from && t >= lo && t < hi) {
    const ulonglong2 pm = pmod[t];
    bv = add_mod(bv, mul_shoup(s_from[o], pm.x, pm.y, m.q), m.q);
  }
  b[o] = bv;
}

__global__ void __launch_bounds__(kThreads) enc_combine_kernel(const uint64_t* __restrict__ pb,
                                                               const uint64_t* __restrict__ pa,
                                                               const uint64_t* __restrict__ u,
                                                               const uint64_t* __restrict__ e0,
                                                               const uint64_t* __restrict__ e1,
                                                               const uint64_t* __restrict__ pt,
                                                               uint64_t* __restrict__ c0, uint64_t* __restrict__ c1,
                                                               int logN, const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int l = blockIdx.y;
  const Mod m = mods[l];
  const size_t o = (size_t)l * N + n;
  const uint64_t uv = u[o];
  c0[o] = add_mod(add_mod(mul_mod(pb[o], uv, m), e0[o], m.q), pt[o], m.q);
  c1[o] = add_mod(mul_mod(pa[o], uv, m), e1[o], m.q);
}

__global__ void __launch_bounds__(kThreads) dec_kernel(const uint64_t* __restrict__ c0,
                                                       const uint64_t* __restrict__ c1,
                                                       const uint64_t* __restrict__ s, uint64_t* __restrict__ pt,
                                                       int logN, const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int n = blockIdx.x * kThreads + threadIdx.x;
  if (n >= N) return;
  const int l = blockIdx.y;
  const Mod m = mods[l];
  const size_t o = (size_t)l * N + n;
  pt[o] = add_mod(c0[o], mul_mod(c1[o], s[o], m), m.q);
}

dim3 grid_for(const Context& c, int limbs) { return dim3((c.N + kThreads - 1) / kThreads, limbs); }

// small polynomial sampled with (nonce, kind), spread over `limbs` primes
// (map) and transformed to NTT form
void small_ntt(const Context& c, uint64_t nonce, int kind, LimbMap map, int limbs, uint64_t* out, int* scratch,
               bool wide = false) {
  const ChachaKey key = key_from_seed(c.params.seed);
  if (wide)
    sample_small_wide_kernel<<<(c.N / 8 + kThreads - 1) / kThreads, kThreads, 0, c.stream>>>(scratch, key, nonce,
                                                                                             c.N, kind);
  else
    sample_small_kernel<<<(c.N + kThreads - 1) / kThreads, kThreads, 0, c.stream>>>(scratch, key, nonce, c.N, kind);
  small_to_limbs_kernel<<<grid_for(c, limbs), kThreads, 0, c.stream>>>(scratch, out, map, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
  ntt_forward(c, out, limbs, map, c.stream);
}

}  // namespace

void keygen_secret_public(Context& c) {
  const int N = c.N, P = c.P, L = c.L;
  const LimbMap all{P, P, L, 0, 0};
  int* scratch = (int*)c.alloc(sizeof(int) * N);
  if (!c.d_sk) CKKS_CUDA(cudaMalloc(&c.d_sk, sizeof(uint64_t) * (size_t)P * N));
  if (!c.d_pk) CKKS_CUDA(cudaMalloc(&c.d_pk, sizeof(uint64_t) * 2 * (size_t)L * N));
  small_ntt(c, kNonceSk, 0, all, P, c.d_sk, scratch);
  uint64_t* e = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)L * N);
  small_ntt(c, kNoncePkE, 1, LimbMap::q(L, L), L, e, scratch);
  uint64_t* a = c.d_pk + (size_t)L * N;
  const ChachaKey key = key_from_seed(c.params.seed);
  uniform_kernel<<<grid_for(c, L), kThreads, 0, c.stream>>>(a, key, kNoncePkA, LimbMap::q(L, L), c.logN, c.d_mods);
  rlwe_combine_kernel<<<grid_for(c, L), kThreads, 0, c.stream>>>(e, a, c.d_sk, nullptr, nullptr, 0, 0, c.d_pk,
                                                                 c.logN, c.d_mods, 0);
  CKKS_CUDA(cudaGetLastError());
  c.release(e);
  c.release(scratch);
  CKKS_CUDA(cudaStreamSynchronize(c.stream));
}

uint64_t* make_switch_key(Context& c, const uint64_t* s_from, uint32_t key_id) {
  if (!c.d_sk) throw Error(kErrState, "secret key not generated");
  const int N = c.N, P = c.P, L = c.L;
  const LimbMap all{P, P, L, 0, 0};
  uint64_t* key = nullptr;
  CKKS_CUDA(cudaMalloc(&key, sizeof(uint64_t) * c.key_words()));
  int* scratch = (int*)c.alloc(sizeof(int) * N);
  uint64_t* e = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)P * N);
  const ChachaKey ck = key_from_seed(c.params.seed);
  for (int j = 0; j < c.beta_top; ++j) {
    uint64_t* b = key + (size_t)j * 2 * P * N;
    uint64_t* a = b + (size_t)P * N;
    small_ntt(c, nonce_ksk(key_id, j, 1), 1, all, P, e, scratch);
    uniform_kernel<<<grid_for(c, P), kThreads, 0, c.stream>>>(a, ck, nonce_ksk(key_id, j, 0), all, c.logN, c.d_mods);
    const int lo = j * c.alpha, hi = std::min(lo + c.alpha, L);
    rlwe_combine_kernel<<<grid_for(c, P), kThreads, 0, c.stream>>>(e, a, c.d_sk, s_from, c.d_pmod, lo, hi, b, c.logN,
                                                                   c.d_mods, 0);
    CKKS_CUDA(cudaGetLastError());
  }
  c.release(e);
  c.release(scratch);
  CKKS_CUDA(cudaStreamSynchronize(c.stream));
  return key;
}

// One digit over Q primes 0..low_limbs-1 with P' = p_0 ... p_{K_low-1}:
// b = e - a s + P' s_from on those Q primes, e - a s on the K_low special
// primes; the other rows of the [2][P][N] layout stay zero.
uint64_t* make_switch_key_low(Context& c, const uint64_t* s_from, uint32_t key_id) {
  if (!c.d_sk) throw Error(kErrState, "secret key not generated");
  if (!c.low_limbs) throw Error(kErrState, "no reduced special-prime set for these parameters");
  const int N = c.N, P = c.P, L = c.L, lq = c.low_limbs, kp = c.K_low;
  uint64_t* key = nullptr;
  CKKS_CUDA(cudaMalloc(&key, sizeof(uint64_t) * c.low_key_words()));
  CKKS_CUDA(cudaMemsetAsync(key, 0, sizeof(uint64_t) * c.low_key_words(), c.stream));
  int* scratch = (int*)c.alloc(sizeof(int) * N);
  uint64_t* e = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)P * N);
  const ChachaKey ck = key_from_seed(c.params.seed);
  uint64_t* b = key;
  uint64_t* a = key + (size_t)P * N;
  for (int part = 0; part < 2; ++part) {
    const LimbMap m = part == 0 ? LimbMap::q(lq, L) : LimbMap::ponly(kp, L);
    const int rows = part == 0 ? lq : kp, first = part == 0 ? 0 : L;
    const size_t off = (size_t)first * N;
    small_ntt(c, nonce_ksk_low(key_id, 1), 1, m, rows, e + off, scratch);
    uniform_kernel<<<grid_for(c, rows), kThreads, 0, c.stream>>>(a + off, ck, nonce_ksk_low(key_id, 0), m, c.logN,
                                                                 c.d_mods);
    rlwe_combine_kernel<<<grid_for(c, rows), kThreads, 0, c.stream>>>(e, a, c.d_sk, s_from, c.d_pmod_low, 0, lq, b,
                                                                      c.logN, c.d_mods, first);
    CKKS_CUDA(cudaGetLastError());
  }
  c.release(e);
  c.release(scratch);
  CKKS_CUDA(cudaStreamSynchronize(c.stream));
  return key;
}

void encrypt(Context& c, const uint64_t* pt, int limbs, uint64_t counter, uint64_t* c0, uint64_t* c1) {
  if (!c.d_pk) throw Error(kErrState, "public key not generated");
  const int N = c.N, L = c.L;
  int* scratch = (int*)c.alloc(sizeof(int) * N);
  uint64_t* buf = (uint64_t*)c.alloc(sizeof(uint64_t) * 3 * (size_t)limbs * N);
  uint64_t *u = buf, *e0 = buf + (size_t)limbs * N, *e1 = buf + 2 * (size_t)limbs * N;
  const LimbMap m = LimbMap::q(limbs, L);
  small_ntt(c, nonce_enc(counter, 0), 0, m, limbs, u, scratch, true);
  small_ntt(c, nonce_enc(counter, 1), 1, m, limbs, e0, scratch, true);
  small_ntt(c, nonce_enc(counter, 2), 1, m, limbs, e1, scratch, true);
  enc_combine_kernel<<<grid_for(c, limbs), kThreads, 0, c.stream>>>(c.d_pk, c.d_pk + (size_t)L * N, u, e0, e1, pt, c0,
                                                                    c1, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
  c.release(buf);
  c.release(scratch);
}

void decrypt(const Context& c, const uint64_t* c0, const uint64_t* c1, int limbs, uint64_t* pt) {
  if (!c.d_sk) throw Error(kErrState, "secret key not generated");
  dec_kernel<<<grid_for(c, limbs), kThreads, 0, c.stream>>>(c0, c1, c.d_sk, pt, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

}  // namespace ckks
