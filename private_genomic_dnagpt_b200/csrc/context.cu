// context.cu -- CKKS context: parameter chain, device-resident tables,
// stream-ordered memory.  Restates the CCParams / GenCryptoContext /
// LoadContext step of the reference driver
// (fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_depth13_
//  digits3_ring65536_cpudiagcache_t123.cpp:1602-1626): FLEXIBLEAUTO scale
// chain, HYBRID key switching with dnum digits, ring dimension 2^log_n.
#include <chrono>
#include <cmath>
#include <cstring>

#include "ckks_internal.hpp"

namespace ckks {

using u128 = unsigned __int128;

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(kErrCuda, std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {

uint64_t powm(uint64_t b, uint64_t e, uint64_t q) {
  u128 r = 1, x = b % q;
  while (e) {
    if (e & 1) r = (r * x) % q;
    x = (x * x) % q;
    e >>= 1;
  }
  return (uint64_t)r;
}
uint64_t invm(uint64_t a, uint64_t q) { return powm(a % q, q - 2, q); }
uint64_t mulm(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)(((u128)a * b) % q); }
uint64_t shoup(uint64_t w, uint64_t q) { return (uint64_t)(((u128)w << 64) / q); }
ulonglong2 shoup_pair(uint64_t w, uint64_t q) { return make_ulonglong2(w, shoup(w, q)); }

bool is_prime64(uint64_t n) {
  static const uint64_t bases[12] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  if (n < 2) return false;
  for (uint64_t b : bases) {
    if (n == b) return true;
    if (n % b == 0) return false;
  }
  uint64_t d = n - 1;
  int s = 0;
  while (!(d & 1)) {
    d >>= 1;
    ++s;
  }
  for (uint64_t b : bases) {
    uint64_t x = powm(b, d, n);
    if (x == 1 || x == n - 1) continue;
    bool comp = true;
    for (int r = 1; r < s; ++r) {
      x = mulm(x, x, n);
      if (x == n - 1) {
        comp = false;
        break;
      }
    }
    if (comp) return false;
  }
  return true;
}

uint32_t bitrev(uint32_t x, int bits) {
  uint32_t r = 0;
  for (int i = 0; i < bits; ++i) {
    r = (r << 1) | (x & 1);
    x >>= 1;
  }
  return r;
}

bool contains(const std::vector<uint64_t>& v, uint64_t x) {
  for (uint64_t y : v)
    if (y == x) return true;
  return false;
}

// Prime chain: q_0 = largest prime < 2^first_bits with q = 1 mod 2N; the
// scaling primes alternate just below / just above 2^scale_bits; the special
// primes are the largest unused ones below 2^special_bits.
std::vector<uint64_t> prime_chain(int logN, int L, int K, int fb, int sb, int pb) {
  const uint64_t M = 2ull << logN;
  std::vector<uint64_t> q;
  {
    const uint64_t base = (1ull << fb) + 1;
    for (uint64_t m = 1;; ++m) {
      if (m * M >= base) throw Error(kErrArgument, "no first prime");
      const uint64_t c = base - m * M;
      if (is_prime64(c)) {
        q.push_back(c);
        break;
      }
    }
  }
  {
    const uint64_t base = (1ull << sb) + 1;
    uint64_t mlo = 1, mhi = 1;
    bool below = true;
    while ((int)q.size() < L) {
      uint64_t c = 0;
      if (below) {
        for (;; ++mlo) {
          if (mlo * M >= base) throw Error(kErrArgument, "scaling primes exhausted");
          c = base - mlo * M;
          if (is_prime64(c) && !contains(q, c)) {
            ++mlo;
            break;
          }
        }
      } else {
        for (;; ++mhi) {
          c = base + mhi * M;
          if (is_prime64(c) && !contains(q, c)) {
            ++mhi;
            break;
          }
        }
      }
      q.push_back(c);
      below = !below;
    }
  }
  {
    const uint64_t base = (1ull << pb) + 1;
    int k = 0;
    for (uint64_t m = 1; k < K; ++m) {
      if (m * M >= base) throw Error(kErrArgument, "special primes exhausted");
      const uint64_t c = base - m * M;
      if (is_prime64(c) && !contains(q, c)) {
        q.push_back(c);
        ++k;
      }
    }
  }
  return q;
}

uint64_t find_psi(uint64_t q, uint64_t twoN) {
  for (uint64_t x = 2;; ++x) {
    const uint64_t p = powm(x, (q - 1) / twoN, q);
    if (powm(p, twoN / 2, q) == q - 1) return p;
  }
}

template <typename T>
T* upload(const std::vector<T>& v) {
  T* d = nullptr;
  CKKS_CUDA(cudaMalloc(&d, sizeof(T) * (v.empty() ? 1 : v.size())));
  if (!v.empty()) CKKS_CUDA(cudaMemcpy(d, v.data(), sizeof(T) * v.size(), cudaMemcpyHostToDevice));
  return d;
}

}  // namespace

uint64_t host_int_to_res(int64_t k, uint64_t q) {
  if (k >= 0) return (uint64_t)k % q;
  const uint64_t m = (uint64_t)(-(k + 1)) % q;  // |k| - 1
  const uint64_t v = (m + 1) % q;
  return v ? q - v : 0;
}

uint64_t host_double_to_res(double r, uint64_t q) {
  const double ar = std::fabs(r);
  uint64_t v;
  if (ar < 9223372036854775808.0) {
    v = ((uint64_t)ar) % q;
  } else {
    uint64_t bits;
    std::memcpy(&bits, &ar, 8);
    const int e = (int)((bits >> 52) & 0x7FF) - 1075;
    const uint64_t mant = (bits & ((1ull << 52) - 1)) | (1ull << 52);
    v = mulm(mant % q, powm(2, (uint64_t)e, q), q);
  }
  return (r < 0 && v) ? q - v : v;
}

Context::Context(const Params& p) : params(p) {
  if (p.log_n < 6 || p.log_n > 17 || p.limbs < 2 || p.dnum < 1 || p.first_mod_bits > 61 ||
      p.scale_mod_bits > 61 || p.special_mod_bits > 61 || p.first_mod_bits <= p.log_n + 1 ||
      p.scale_mod_bits <= p.log_n + 1 || p.special_mod_bits <= p.log_n + 1)
    throw Error(kErrArgument, "parameters out of range (log_n 6..17, limbs >= 2, prime bits <= 61)");
  CKKS_CUDA(cudaSetDevice(p.device));
  CKKS_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p.device));
  logN = p.log_n;
  N = 1 << logN;
  L = p.limbs;
  alpha = (L + p.dnum - 1) / p.dnum;
  K = alpha;
  beta_top = (L + alpha - 1) / alpha;
  P = L + K;
  if (P > 96) throw Error(kErrArgument, "too many primes");
  moduli = prime_chain(logN, L, K, p.first_mod_bits, p.scale_mod_bits, p.special_mod_bits);
  CKKS_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));

  // scale chain (FLEXIBLEAUTO): s_L = q_{L-1}; s_{l-1} = s_l^2 / q_{l-1}
  scales.assign(L + 1, 0.0);
  scales[L] = (double)moduli[L - 1];
  for (int l = L; l >= 2; --l) scales[l - 1] = scales[l] * scales[l] / (double)moduli[l - 1];

  std::vector<Mod> mods(P);
  std::vector<ulonglong2> tw((size_t)P * N), itw((size_t)P * N), ninv(P), w1ninv(P), pmod(P);
  std::vector<double2> twd((size_t)P * N), itwd((size_t)P * N);
  psi.resize(P);
  for (int i = 0; i < P; ++i) {
    const uint64_t q = moduli[i];
    u128 r = (~(u128)0) / q;
    mods[i] = Mod{q, (uint64_t)(r >> 64), (uint64_t)r};
    const uint64_t s = find_psi(q, 2ull * N);
    psi[i] = s;
    const uint64_t si = invm(s, q);
    uint64_t pw = 1, pwi = 1;
    std::vector<uint64_t> w(N), wi(N);
    for (int j = 0; j < N; ++j) {
      const uint32_t rj = bitrev((uint32_t)j, logN);
      w[rj] = pw;
      wi[rj] = pwi;
      pw = mulm(pw, s, q);
      pwi = mulm(pwi, si, q);
    }
    for (int j = 0; j < N; ++j) {
      tw[(size_t)i * N + j] = shoup_pair(w[j], q);
      itw[(size_t)i * N + j] = shoup_pair(wi[j], q);
      // float64 twiddles (exact for the primes below 2^53 that use them)
      twd[(size_t)i * N + j] = make_double2((double)w[j], (double)w[j] / (double)q);
      itwd[(size_t)i * N + j] = make_double2((double)wi[j], (double)wi[j] / (double)q);
    }
    const uint64_t ni = invm((uint64_t)N, q);
    ninv[i] = shoup_pair(ni, q);
    w1ninv[i] = shoup_pair(mulm(wi[1], ni, q), q);
    uint64_t pm = 1;
    for (int k = 0; k < K; ++k) pm = mulm(pm, moduli[L + k] % q, q);
    pmod[i] = shoup_pair(i < L ? pm : 0, q);
  }
  d_mods = upload(mods);
  CKKS_CUDA(cudaMalloc(&d_faults, sizeof(unsigned int)));
  CKKS_CUDA(cudaMemset(d_faults, 0, sizeof(unsigned int)));
  d_tw = upload(tw);
  d_itw = upload(itw);
  d_twd = upload(twd);
  d_itwd = upload(itwd);
  d_ninv = upload(ninv);
  d_w1ninv = upload(w1ninv);
  d_pmod = upload(pmod);

  // reduced special-prime set for one-digit key switches at <= 3 limbs: the
  // fewest leading special primes whose product exceeds Q_3 by 2^19.5 (three
  // 60-bit primes over a 60 + 2 x 50-bit Q_3)
  {
    const int lo = std::min(3, alpha);
    double qbits = 0.0, pbits = 0.0;
    for (int i = 0; i < lo; ++i) qbits += std::log2((double)moduli[i]);
    int k = 0;
    while (k < K && pbits < qbits + 19.5) pbits += std::log2((double)moduli[L + k++]);
    if (L >= lo && lo >= 1 && pbits >= qbits + 19.5 && k < K) {
      low_limbs = lo;
      K_low = k;
    }
  }

  // (P/p_k)^-1 mod p_k over the first Kx special primes, with the ModDown
  // pre-scaling folded into the inverse NTT
  auto down_scales = [&](int Kx, ulonglong2*& da, ulonglong2*& db, std::vector<ulonglong2>* phat_out) {
    std::vector<ulonglong2> phatinv(K, make_ulonglong2(0, 0)), sa(K, make_ulonglong2(0, 0)),
        sb(K, make_ulonglong2(0, 0));
    for (int k = 0; k < Kx; ++k) {
      const uint64_t pk = moduli[L + k];
      uint64_t prod = 1;
      for (int k2 = 0; k2 < Kx; ++k2)
        if (k2 != k) prod = mulm(prod, moduli[L + k2] % pk, pk);
      phatinv[k] = shoup_pair(invm(prod, pk), pk);
      const uint64_t ni = invm((uint64_t)N, pk);
      const uint64_t w1 = mulm(ni, itw[(size_t)(L + k) * N + 1].x, pk);
      sa[k] = shoup_pair(mulm(phatinv[k].x, ni, pk), pk);
      sb[k] = shoup_pair(mulm(phatinv[k].x, w1, pk), pk);
    }
    if (phat_out) *phat_out = phatinv;
    da = upload(sa);
    db = upload(sb);
  };
  {
    std::vector<ulonglong2> phatinv;
    down_scales(K, d_down_scale_a, d_down_scale_b, &phatinv);
    d_phatinv = upload(phatinv);
    if (low_limbs) {
      down_scales(K_low, d_down_scale_low_a, d_down_scale_low_b, nullptr);
      std::vector<ulonglong2> pl(P);
      for (int i = 0; i < P; ++i) {
        const uint64_t q = moduli[i];
        uint64_t pm = 1;
        for (int k = 0; k < K_low; ++k) pm = mulm(pm, moduli[L + k] % q, q);
        pl[i] = shoup_pair(i < L ? pm : 0, q);
      }
      d_pmod_low = upload(pl);
    }
  }

  // canonical embedding tables
  {
    const int M = 2 * N;
    std::vector<double2> ksi(M + 1);
    for (int k = 0; k <= M; ++k) {
      const double ang = 2.0 * M_PI * (double)k / (double)M;
      ksi[k] = make_double2(std::cos(ang), std::sin(ang));
    }
    d_ksi = upload(ksi);
    std::vector<uint32_t> rg(N / 2);
    uint64_t g = 1;
    for (int j = 0; j < N / 2; ++j) {
      rg[j] = (uint32_t)g;
      g = (g * 5) % (uint64_t)M;
    }
    d_rot_group = upload(rg);
  }

  // per-level ModUp / ModDown / Rescale constants over the first Kx special primes
  auto level_tables = [&](int l, int Kx) {
    LevelTables t;
    t.limbs = l;
    t.beta = (l + alpha - 1) / alpha;
    const int E = l + Kx;
    std::vector<ulonglong2> hatinv((size_t)t.beta * alpha, make_ulonglong2(0, 0));
    std::vector<uint64_t> hat((size_t)t.beta * alpha * E, 0);
    for (int j = 0; j < t.beta; ++j) {
      const int lo = j * alpha, hi = std::min(lo + alpha, l);
      for (int i = lo; i < hi; ++i) {
        const uint64_t qi = moduli[i];
        uint64_t prod = 1;
        for (int i2 = lo; i2 < hi; ++i2)
          if (i2 != i) prod = mulm(prod, moduli[i2] % qi, qi);
        hatinv[(size_t)j * alpha + (i - lo)] = shoup_pair(invm(prod, qi), qi);
        for (int tt = 0; tt < E; ++tt) {
          const uint64_t mt = moduli[tt < l ? tt : L + (tt - l)];
          uint64_t h = 1;
          for (int i2 = lo; i2 < hi; ++i2)
            if (i2 != i) h = mulm(h, moduli[i2] % mt, mt);
          hat[((size_t)j * alpha + (i - lo)) * E + tt] = h;
        }
      }
    }
    t.d_up_hatinv = upload(hatinv);
    {
      std::vector<ulonglong2> sa(l), sb(l);
      for (int i = 0; i < l; ++i) {
        const int j = i / alpha;
        const uint64_t qi = moduli[i];
        const uint64_t hv = hatinv[(size_t)j * alpha + (i - j * alpha)].x;
        const uint64_t ni = invm((uint64_t)N, qi);
        sa[i] = shoup_pair(mulm(hv, ni, qi), qi);
        sb[i] = shoup_pair(mulm(hv, mulm(ni, itw[(size_t)i * N + 1].x, qi), qi), qi);
      }
      t.d_up_scale_a = upload(sa);
      t.d_up_scale_b = upload(sb);
    }
    t.d_up_hat = upload(hat);
    std::vector<uint64_t> phat((size_t)Kx * l);
    std::vector<ulonglong2> pinv(l);
    for (int tt = 0; tt < l; ++tt) {
      const uint64_t qt = moduli[tt];
      uint64_t pp = 1;
      for (int k = 0; k < Kx; ++k) {
        uint64_t h = 1;
        for (int k2 = 0; k2 < Kx; ++k2)
          if (k2 != k) h = mulm(h, moduli[L + k2] % qt, qt);
        phat[(size_t)k * l + tt] = h;
        pp = mulm(pp, moduli[L + k] % qt, qt);
      }
      pinv[tt] = shoup_pair(invm(pp, qt), qt);
    }
    t.d_down_phat = upload(phat);
    t.d_down_pinv = upload(pinv);
    std::vector<ulonglong2> rinv(l > 1 ? l - 1 : 1, make_ulonglong2(0, 0));
    for (int i = 0; i + 1 < l; ++i) rinv[i] = shoup_pair(invm(moduli[l - 1] % moduli[i], moduli[i]), moduli[i]);
    t.d_rescale_inv = upload(rinv);
    return t;
  };
  levels.resize(L + 1);
  for (int l = 1; l <= L; ++l) levels[l] = level_tables(l, K);
  levels_low.resize(low_limbs + 1);
  for (int l = 1; l <= low_limbs; ++l) levels_low[l] = level_tables(l, K_low);

  CKKS_CUDA(cudaDeviceSynchronize());
}

Context::~Context() {
  cudaSetDevice(params.device);
  cudaStreamSynchronize(stream);
  if (stage_) cudaFreeHost(stage_);
  drop_cache();
  for (auto& kv : size_of_) cudaFree(kv.first);  // blocks still held by live objects
  size_of_.clear();
  for (auto& kv : rot_keys) cudaFree(kv.second);
  cudaFree(d_sk);
  cudaFree(d_pk);
  cudaFree(d_rlk);
  for (auto& t : levels) {
    cudaFree(t.d_up_hatinv);
    cudaFree(t.d_up_hat);
    cudaFree(t.d_down_phat);
    cudaFree(t.d_down_pinv);
    cudaFree(t.d_rescale_inv);
    cudaFree(t.d_up_scale_a);
    cudaFree(t.d_up_scale_b);
  }
  cudaFree(d_down_scale_a);
  cudaFree(d_down_scale_b);
  for (auto& t : levels_low) {
    cudaFree(t.d_up_hatinv);
    cudaFree(t.d_up_hat);
    cudaFree(t.d_down_phat);
    cudaFree(t.d_down_pinv);
    cudaFree(t.d_rescale_inv);
    cudaFree(t.d_up_scale_a);
    cudaFree(t.d_up_scale_b);
  }
  cudaFree(d_down_scale_low_a);
  cudaFree(d_down_scale_low_b);
  cudaFree(d_pmod_low);
  for (auto& kv : rot_keys_low) cudaFree(kv.second);
  cudaFree(d_rlk_low);
  cudaFree(d_mods);
  cudaFree(d_faults);
  cudaFree(d_tw);
  cudaFree(d_itw);
  cudaFree(d_twd);
  cudaFree(d_itwd);
  cudaFree(d_ninv);
  cudaFree(d_w1ninv);
  cudaFree(d_pmod);
  cudaFree(d_ksi);
  cudaFree(d_rot_group);
  cudaFree(d_phatinv);
  cudaStreamDestroy(stream);
}

cudaEvent_t Profiler::get() {
  if (!pool_.empty()) {
    cudaEvent_t e = pool_.back();
    pool_.pop_back();
    return e;
  }
  cudaEvent_t e;
  CKKS_CUDA(cudaEventCreate(&e));
  return e;
}

size_t Profiler::begin(const char* name, double bytes, cudaStream_t st) {
  Rec r{name, bytes, get(), get(), section};
  CKKS_CUDA(cudaEventRecord(r.a, st));
  pending_.push_back(r);
  return pending_.size() - 1;
}

void Profiler::end(size_t idx, cudaStream_t st) {
  if (idx < pending_.size()) cudaEventRecord(pending_[idx].b, st);
}

std::map<std::string, Profiler::Totals> Profiler::report() {
  for (Rec& r : pending_) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.b) != cudaSuccess || cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) {
      cudaGetLastError();  // an unrecorded pair is dropped, not reported
      pool_.push_back(r.a);
      pool_.push_back(r.b);
      continue;
    }
    for (Totals* t : {&totals_[r.name], &by_section_[r.section.empty() ? "-" : r.section][r.name]}) {
      t->launches += 1;
      t->ms += ms;
      t->bytes += r.bytes;
    }
    auto& h = totals_[r.name].by_size[r.bytes >= 1.0 ? std::ilogb(r.bytes) : 0];
    h.first += 1;
    h.second += ms;
    pool_.push_back(r.a);
    pool_.push_back(r.b);
  }
  pending_.clear();
  return totals_;
}

void Profiler::reset() {
  report();
  totals_.clear();
  by_section_.clear();
}

Profiler::~Profiler() {
  for (Rec& r : pending_) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (cudaEvent_t e : pool_) cudaEventDestroy(e);
}

uint32_t Context::galois(int k) const {
  const int slots = N / 2;
  int r = k % slots;
  if (r < 0) r += slots;
  return (uint32_t)powm(5, (uint64_t)r, 2ull * N);
}

const uint64_t* Context::rot_key(uint32_t g) const {
  auto it = rot_keys.find(g);
  return it == rot_keys.end() ? nullptr : it->second;
}

void Context::install_key(int k, uint64_t* key, bool lowset) {
  uint64_t*& rlk = lowset ? d_rlk_low : d_rlk;
  auto& rot = lowset ? rot_keys_low : rot_keys;
  if (k == 0) {
    if (rlk) cudaFree(rlk);
    rlk = key;
    return;
  }
  const uint32_t g = galois(k);
  auto it = rot.find(g);
  if (it != rot.end()) cudaFree(it->second);
  rot[g] = key;
}

const uint64_t* Context::switch_key(uint32_t g, int limbs) const {
  if (low(limbs)) {
    if (g == 1u) return d_rlk_low;
    auto it = rot_keys_low.find(g);
    return it == rot_keys_low.end() ? nullptr : it->second;
  }
  if (g == 1u) return d_rlk;
  return rot_key(g);
}

namespace {
// bucket: powers of two up to 1 MiB, then multiples of 256 KiB
size_t bucket(size_t bytes) {
  if (bytes <= 256) return 256;
  if (bytes <= (1u << 20)) {
    size_t b = 256;
    while (b < bytes) b <<= 1;
    return b;
  }
  const size_t g = 256u << 10;
  return (bytes + g - 1) / g * g;
}
}  // namespace

void* Context::alloc(size_t bytes) const {
  const auto t0 = std::chrono::steady_clock::now();
  const size_t b = bucket(bytes);
  void* p = nullptr;
  {
    std::lock_guard<std::mutex> lk(mem_mu_);
    auto it = free_.find(b);
    if (it != free_.end() && !it->second.empty()) {
      p = it->second.back();
      it->second.pop_back();
    }
  }
  if (!p) {
    cudaError_t e = cudaMalloc(&p, b);
    if (e == cudaErrorMemoryAllocation) {  // give cached blocks back and retry once
      cudaGetLastError();
      CKKS_CUDA(cudaStreamSynchronize(stream));
      drop_cache();
      e = cudaMalloc(&p, b);
    }
    CKKS_CUDA(e);
    std::lock_guard<std::mutex> lk(mem_mu_);
    size_of_[p] = b;
  }
  alloc_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  ++alloc_calls;
  return p;
}

void Context::stage_upload(void* dst, const void* src, size_t bytes, cudaStream_t st) const {
  if (!bytes) return;
  const size_t span = (bytes + 255) & ~(size_t)255;
  if (span > kStageBytes) {
    CKKS_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st));
    return;
  }
  if (!stage_) CKKS_CUDA(cudaHostAlloc((void**)&stage_, kStageBytes, cudaHostAllocDefault));
  if (stage_off_ + span > kStageBytes) {
    // every copy out of the ring so far was issued on the context's stream
    CKKS_CUDA(cudaStreamSynchronize(st));
    stage_off_ = 0;
  }
  std::memcpy(stage_ + stage_off_, src, bytes);
  CKKS_CUDA(cudaMemcpyAsync(dst, stage_ + stage_off_, bytes, cudaMemcpyHostToDevice, st));
  stage_off_ += span;
}

void Context::release(void* p) const {
  if (!p) return;
  std::lock_guard<std::mutex> lk(mem_mu_);
  auto it = size_of_.find(p);
  if (it == size_of_.end()) return;
  free_[it->second].push_back(p);
}

void Context::drop_cache() const {
  std::lock_guard<std::mutex> lk(mem_mu_);
  for (auto& kv : free_)
    for (void* p : kv.second) {
      cudaFree(p);
      size_of_.erase(p);
    }
  free_.clear();
}

DevPoly::~DevPoly() {
  if (data && ctx) ctx->release(data);
}

void DevPoly::ensure(Context* c, int np, int need) {
  if (ctx && ctx != c) throw Error(kErrArgument, "object belongs to another context");
  if (data && np == npolys && need <= cap) {
    ctx = c;
    return;
  }
  if (data) c->release(data);
  ctx = c;
  npolys = np;
  cap = need;
  data = (uint64_t*)c->alloc(sizeof(uint64_t) * (size_t)np * need * c->N);
}

}  // namespace ckks
