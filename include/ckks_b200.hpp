// ckks_b200.hpp -- header-only C++ host layer over the C ABI (ckks_b200.h)
// with the OpenFHE/FIDESlib names the reference block driver programs
// against (fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_
// depth13_digits3_ring65536_cpudiagcache_t123.cpp, "T123.cpp").
//
//   auto cc = ckks_b200::GenCryptoContext(params);        // T123.cpp:1616
//   cc->KeyGen(); cc->EvalMultKeyGen(); cc->EvalRotateKeyGen(idx);
//   auto pt = cc->MakeCKKSPackedPlaintext(values, 1, level);
//   auto ct = cc->Encrypt(pt);  cc->Decrypt(ct)->GetRealPackedValue();
//   cc->EvalAdd / EvalSub / EvalMult / EvalRotate / EvalFastRotation /
//   cc->AccumulateSum / cc->Rescale / ct->GetLevel()
//
// Handles are shared_ptr like OpenFHE's.  Failures throw ckks_b200::Error
// carrying the ABI status (the reference maps exceptions to exit code 2,
// T123.cpp:1757-1761).  EvalMult follows FLEXIBLEAUTO: an operand carrying a
// product's scale is rescaled first, the operand with more limbs is brought
// down to the other's level, and the product is left unrescaled.
#pragma once

#include <cmath>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "ckks_b200.h"

namespace ckks_b200 {

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

inline void check(int rc) {
  if (rc != CKKS_OK) throw Error(rc, std::string("ckks: ") + ckks_last_error());
}

class CryptoContextImpl;

class PlaintextImpl {
 public:
  explicit PlaintextImpl(ckks_ctx* c) : ctx_(c) { check(ckks_pt_create(c, &h_)); }
  ~PlaintextImpl() { ckks_pt_destroy(h_); }
  PlaintextImpl(const PlaintextImpl&) = delete;
  PlaintextImpl& operator=(const PlaintextImpl&) = delete;
  ckks_pt* handle() const { return h_; }
  void SetLength(size_t n) { length_ = n; }
  std::vector<double> GetRealPackedValue() const {
    int n = 0;
    check(ckks_ctx_info(ctx_, &n, nullptr, nullptr, nullptr));
    const size_t len = length_ ? length_ : (size_t)n / 2;
    std::vector<double> out(len);
    check(ckks_decode(ctx_, h_, out.data(), (int)len));
    return out;
  }
  int limbs() const { return ckks_pt_limbs(h_); }
  double scale() const { return ckks_pt_scale(h_); }

 private:
  ckks_ctx* ctx_;
  ckks_pt* h_ = nullptr;
  size_t length_ = 0;
};

class CiphertextImpl {
 public:
  explicit CiphertextImpl(ckks_ctx* c) : ctx_(c) { check(ckks_ct_create(c, &h_)); }
  // non-owning view of a handle the caller keeps (not destroyed with the view)
  CiphertextImpl(ckks_ctx* c, ckks_ct* existing) : ctx_(c), h_(existing), owns_(false) {}
  ~CiphertextImpl() {
    if (owns_) ckks_ct_destroy(h_);
  }
  CiphertextImpl(const CiphertextImpl&) = delete;
  CiphertextImpl& operator=(const CiphertextImpl&) = delete;
  ckks_ct* handle() const { return h_; }
  uint32_t GetLevel() const { return (uint32_t)ckks_ct_level(h_); }
  int limbs() const { return ckks_ct_limbs(h_); }
  double scale() const { return ckks_ct_scale(h_); }
  int noise_deg() const { return ckks_ct_noise_deg(h_); }

 private:
  ckks_ctx* ctx_;
  ckks_ct* h_ = nullptr;
  bool owns_ = true;
};

using Plaintext = std::shared_ptr<PlaintextImpl>;
using Ciphertext = std::shared_ptr<CiphertextImpl>;

struct CCParams {
  int ring_dim_log = 16;
  int multiplicative_depth = 23;  // limbs = depth + 1
  int scaling_mod_size = 50;
  int first_mod_size = 60;
  int special_mod_size = 60;
  int num_large_digits = 3;
  uint64_t seed = 1;
  int device = 0;
};

class CryptoContextImpl {
 public:
  explicit CryptoContextImpl(const CCParams& p) {
    ckks_params q{p.ring_dim_log, p.multiplicative_depth + 1, p.num_large_digits, p.first_mod_size,
                  p.scaling_mod_size, p.special_mod_size, p.seed, p.device};
    check(ckks_ctx_create(&q, &h_));
    check(ckks_ctx_info(h_, &n_, &limbs_, &special_, &alpha_));
  }
  // non-owning view of an existing context
  explicit CryptoContextImpl(ckks_ctx* existing) : h_(existing), owns_(false) {
    check(ckks_ctx_info(h_, &n_, &limbs_, &special_, &alpha_));
  }
  ~CryptoContextImpl() {
    if (owns_) ckks_ctx_destroy(h_);
  }
  CryptoContextImpl(const CryptoContextImpl&) = delete;
  CryptoContextImpl& operator=(const CryptoContextImpl&) = delete;

  ckks_ctx* handle() const { return h_; }
  uint32_t GetRingDimension() const { return (uint32_t)n_; }
  uint32_t GetCyclotomicOrder() const { return 2u * (uint32_t)n_; }
  int limbs() const { return limbs_; }
  double ScaleAt(int level) const { return ckks_ctx_scale(h_, level); }
  void Synchronize() const { check(ckks_sync(h_)); }

  void KeyGen() { check(ckks_keygen(h_)); }
  void EvalMultKeyGen() { check(ckks_relin_keygen(h_)); }
  void EvalRotateKeyGen(const std::vector<int>& idx) { check(ckks_rotkey_gen(h_, idx.data(), (int)idx.size())); }

  Plaintext MakeCKKSPackedPlaintext(const std::vector<double>& v, int /*noise_scale_deg*/ = 1, uint32_t level = 0) {
    auto pt = std::make_shared<PlaintextImpl>(h_);
    check(ckks_encode(h_, v.data(), (int)v.size(), (int)level, pt->handle()));
    return pt;
  }
  Plaintext MakePlaintextAt(const std::vector<double>& v, int limbs, double scale) {
    auto pt = std::make_shared<PlaintextImpl>(h_);
    check(ckks_encode_at(h_, v.data(), (int)v.size(), limbs, scale, pt->handle()));
    return pt;
  }
  Ciphertext fresh() { return std::make_shared<CiphertextImpl>(h_); }
  Ciphertext Encrypt(const Plaintext& pt) {
    auto ct = fresh();
    check(ckks_encrypt(h_, pt->handle(), ct->handle()));
    return ct;
  }
  Plaintext Decrypt(const Ciphertext& ct) {
    const Ciphertext c1 = ct->noise_deg() >= 2 ? Rescale(ct) : ct;
    auto pt = std::make_shared<PlaintextImpl>(h_);
    check(ckks_decrypt(h_, c1->handle(), pt->handle()));
    return pt;
  }

  Ciphertext Rescale(const Ciphertext& a) {
    auto o = fresh();
    check(ckks_rescale(h_, a->handle(), o->handle()));
    return o;
  }
  Ciphertext EvalAdd(const Ciphertext& a, const Ciphertext& b) {
    auto [x, y] = align(a, b);
    auto o = fresh();
    check(ckks_add(h_, x->handle(), y->handle(), o->handle()));
    return o;
  }
  Ciphertext EvalSub(const Ciphertext& a, const Ciphertext& b) {
    auto [x, y] = align(a, b);
    auto o = fresh();
    check(ckks_sub(h_, x->handle(), y->handle(), o->handle()));
    return o;
  }
  Ciphertext EvalAdd(const Ciphertext& a, double v) {
    auto o = fresh();
    check(ckks_add_scalar(h_, a->handle(), v, o->handle()));
    return o;
  }
  Ciphertext EvalMult(const Ciphertext& a, const Ciphertext& b) {
    const Ciphertext a1 = deg1(a), b1 = deg1(b);
    auto [x, y] = align(a1, b1);
    auto o = fresh();
    check(ckks_mul_ct(h_, x->handle(), y->handle(), o->handle()));
    return o;
  }
  // the plaintext must carry at least the ciphertext's limbs (encode it at
  // the ciphertext's level, as T123.cpp:1053-1055 does)
  Ciphertext EvalMult(const Ciphertext& a, const Plaintext& p) {
    const Ciphertext a1 = deg1(a);
    auto o = fresh();
    check(ckks_mul_pt(h_, a1->handle(), p->handle(), o->handle()));
    return o;
  }
  Ciphertext EvalRotate(const Ciphertext& a, int k) {
    auto o = fresh();
    check(ckks_rotate(h_, a->handle(), k, o->handle()));
    return o;
  }
  // [[EvalFastRotation(x, k)] for x in a]: each key read once for all inputs
  std::vector<std::vector<Ciphertext>> EvalFastRotationBatch(const std::vector<Ciphertext>& a,
                                                             const std::vector<int>& k) {
    std::vector<std::vector<Ciphertext>> outs(a.size());
    std::vector<const ckks_ct*> in;
    std::vector<ckks_ct*> hs;
    for (size_t i = 0; i < a.size(); ++i) {
      in.push_back(a[i]->handle());
      for (size_t r = 0; r < k.size(); ++r) {
        outs[i].push_back(fresh());
        hs.push_back(outs[i].back()->handle());
      }
    }
    check(ckks_rotate_hoisted_batch(h_, in.data(), (int)a.size(), k.data(), (int)k.size(), hs.data()));
    return outs;
  }
  std::vector<Ciphertext> EvalFastRotation(const Ciphertext& a, const std::vector<int>& k) {
    std::vector<Ciphertext> outs;
    std::vector<ckks_ct*> hs;
    for (size_t i = 0; i < k.size(); ++i) {
      outs.push_back(fresh());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_rotate_hoisted(h_, a->handle(), k.data(), (int)k.size(), hs.data()));
    return outs;
  }
  // sum of many ciphertexts at one level and scale (EvalAddMany)
  Ciphertext EvalAddMany(const std::vector<Ciphertext>& a) {
    std::vector<const ckks_ct*> in;
    for (const auto& x : a) in.push_back(x->handle());
    auto o = fresh();
    check(ckks_add_many(h_, in.data(), (int)in.size(), o->handle()));
    return o;
  }
  std::vector<Ciphertext> EvalAddBatch(const std::vector<Ciphertext>& a, const std::vector<Ciphertext>& b) {
    std::vector<Ciphertext> outs;
    std::vector<const ckks_ct*> x, y;
    std::vector<ckks_ct*> hs;
    for (size_t i = 0; i < a.size(); ++i) {
      outs.push_back(fresh());
      x.push_back(a[i]->handle());
      y.push_back(b[i]->handle());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_add_batch(h_, x.data(), y.data(), (int)a.size(), hs.data()));
    return outs;
  }
  // independent rotations / products / rescales at one limb count, batched
  std::vector<Ciphertext> EvalRotateBatch(const std::vector<Ciphertext>& a, const std::vector<int>& k) {
    std::vector<Ciphertext> outs;
    std::vector<const ckks_ct*> in;
    std::vector<ckks_ct*> hs;
    for (size_t i = 0; i < a.size(); ++i) {
      outs.push_back(fresh());
      in.push_back(a[i]->handle());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_rotate_batch(h_, in.data(), k.data(), (int)a.size(), hs.data()));
    return outs;
  }
  // sum_i a[i] * b[i] with one relinearisation (not rescaled)
  Ciphertext EvalMultSum(const std::vector<Ciphertext>& a, const std::vector<Ciphertext>& b) {
    Ciphertext out = fresh();
    std::vector<const ckks_ct*> x, y;
    for (size_t i = 0; i < a.size(); ++i) {
      x.push_back(a[i]->handle());
      y.push_back(b[i]->handle());
    }
    check(ckks_mul_ct_sum(h_, x.data(), y.data(), (int)a.size(), out->handle()));
    return out;
  }
  // sum_i rot(a[i], k[i]) with one ModDown per 32 rotations
  Ciphertext EvalRotateSum(const std::vector<Ciphertext>& a, const std::vector<int>& k) {
    Ciphertext out = fresh();
    std::vector<const ckks_ct*> in;
    for (const auto& x : a) in.push_back(x->handle());
    check(ckks_rotate_sum(h_, in.data(), k.data(), (int)a.size(), out->handle()));
    return out;
  }
  // EvalRotateSum(a[g], k) for every group g (all groups of k.size() inputs)
  std::vector<Ciphertext> EvalRotateSumGroups(const std::vector<std::vector<Ciphertext>>& a,
                                              const std::vector<int>& k) {
    std::vector<Ciphertext> outs;
    std::vector<const ckks_ct*> in;
    std::vector<ckks_ct*> hs;
    for (const auto& grp : a) {
      if (grp.size() != k.size()) throw std::invalid_argument("EvalRotateSumGroups: group length differs from k");
      for (const auto& x : grp) in.push_back(x->handle());
      outs.push_back(fresh());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_rotate_sum_groups(h_, in.data(), (int)a.size(), k.data(), (int)k.size(), hs.data()));
    return outs;
  }
  std::vector<Ciphertext> EvalMultBatch(const std::vector<Ciphertext>& a, const std::vector<Ciphertext>& b) {
    std::vector<Ciphertext> outs;
    std::vector<const ckks_ct*> x, y;
    std::vector<ckks_ct*> hs;
    for (size_t i = 0; i < a.size(); ++i) {
      outs.push_back(fresh());
      x.push_back(a[i]->handle());
      y.push_back(b[i]->handle());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_mul_ct_batch(h_, x.data(), y.data(), (int)a.size(), hs.data()));
    return outs;
  }
  // [EvalMult(a[i], p[i])] for ciphertexts at one level, batched launches
  std::vector<Ciphertext> EvalMultPlainBatch(const std::vector<Ciphertext>& a, const std::vector<Plaintext>& p) {
    std::vector<Ciphertext> outs, in;
    std::vector<const ckks_ct*> x;
    std::vector<const ckks_pt*> y;
    std::vector<ckks_ct*> hs;
    for (size_t i = 0; i < a.size(); ++i) {
      outs.push_back(fresh());
      in.push_back(deg1(a[i]));
      x.push_back(in.back()->handle());
      y.push_back(p[i]->handle());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_mul_pt_batch(h_, x.data(), y.data(), (int)a.size(), hs.data()));
    return outs;
  }
  std::vector<Ciphertext> RescaleBatch(const std::vector<Ciphertext>& a) {
    std::vector<Ciphertext> outs;
    std::vector<const ckks_ct*> in;
    std::vector<ckks_ct*> hs;
    for (size_t i = 0; i < a.size(); ++i) {
      outs.push_back(fresh());
      in.push_back(a[i]->handle());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_rescale_batch(h_, in.data(), (int)a.size(), hs.data()));
    return outs;
  }
  Ciphertext AccumulateSum(const Ciphertext& a, int count, int stride) {
    auto o = fresh();
    check(ckks_accumulate_sum(h_, a->handle(), count, stride, o->handle()));
    return o;
  }
  // [sum_r rot(x, k[r]) for x in a]: one ModUp and one ModDown per input
  std::vector<Ciphertext> EvalRotateSumHoisted(const std::vector<Ciphertext>& a, const std::vector<int>& k) {
    std::vector<Ciphertext> outs;
    std::vector<const ckks_ct*> in;
    std::vector<ckks_ct*> hs;
    for (const auto& x : a) {
      outs.push_back(fresh());
      in.push_back(x->handle());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_rotate_sum_hoisted(h_, in.data(), (int)a.size(), k.data(), (int)k.size(), hs.data()));
    return outs;
  }
  // [sum_{j < window} rot(x, j * stride) for x in a]: the AccumulateSum
  // ladder with one ModDown per step
  std::vector<Ciphertext> WindowSumBatch(const std::vector<Ciphertext>& a, int window, int stride, int radix = 4) {
    std::vector<Ciphertext> outs;
    std::vector<const ckks_ct*> in;
    std::vector<ckks_ct*> hs;
    for (const auto& x : a) {
      outs.push_back(fresh());
      in.push_back(x->handle());
      hs.push_back(outs.back()->handle());
    }
    check(ckks_window_sum_batch_radix(h_, in.data(), (int)a.size(), window, stride, radix, hs.data()));
    return outs;
  }
  // degree-1 ciphertext at `limbs` limbs with that level's FLEXIBLEAUTO scale
  Ciphertext LevelReduce(const Ciphertext& a, int limbs) {
    Ciphertext x = deg1(a);
    if (x->limbs() == limbs) return x;
    const double target = ScaleAt(limbs_ - limbs);
    std::vector<uint64_t> q(limbs_);
    check(ckks_ctx_moduli(h_, q.data(), limbs_));
    const double ql = (double)q[x->limbs() - 1];
    const int64_t c = (int64_t)std::llround(target * ql / x->scale());
    auto t = fresh();
    check(ckks_mul_int(h_, x->handle(), c, t->handle()));
    check(ckks_ct_set_scale(t->handle(), x->scale() * (double)c, 2));
    auto r = Rescale(t);
    if (r->limbs() > limbs) {
      auto d = fresh();
      check(ckks_drop_limbs(h_, r->handle(), limbs, d->handle()));
      return d;
    }
    return r;
  }
  // LevelReduce(a[i], limbs[i]) for every input; the rescales of the scaled
  // inputs at one limb count run as one batch
  std::vector<Ciphertext> LevelReduceBatch(const std::vector<Ciphertext>& a, const std::vector<int>& limbs) {
    if (a.size() != limbs.size()) throw std::invalid_argument("LevelReduceBatch: one limb count per input");
    std::vector<Ciphertext> out(a.size()), scaled(a.size());
    std::vector<uint64_t> q(limbs_);
    check(ckks_ctx_moduli(h_, q.data(), limbs_));
    std::vector<std::pair<int, std::vector<size_t>>> bins;  // limb count -> inputs, first-seen order
    for (size_t i = 0; i < a.size(); ++i) {
      Ciphertext x = deg1(a[i]);
      if (x->limbs() == limbs[i]) {
        out[i] = x;
        continue;
      }
      const double target = ScaleAt(limbs_ - limbs[i]);
      const double ql = (double)q[x->limbs() - 1];
      const int64_t c = (int64_t)std::llround(target * ql / x->scale());
      auto t = fresh();
      check(ckks_mul_int(h_, x->handle(), c, t->handle()));
      check(ckks_ct_set_scale(t->handle(), x->scale() * (double)c, 2));
      scaled[i] = t;
      size_t k = 0;
      while (k < bins.size() && bins[k].first != t->limbs()) ++k;
      if (k == bins.size()) bins.push_back({t->limbs(), {}});
      bins[k].second.push_back(i);
    }
    for (const auto& bin : bins) {
      std::vector<Ciphertext> xs;
      for (size_t i : bin.second) xs.push_back(scaled[i]);
      const auto r = RescaleBatch(xs);
      for (size_t k = 0; k < bin.second.size(); ++k) {
        const size_t i = bin.second[k];
        if (r[k]->limbs() > limbs[i]) {
          auto d = fresh();
          check(ckks_drop_limbs(h_, r[k]->handle(), limbs[i], d->handle()));
          out[i] = d;
        } else {
          out[i] = r[k];
        }
      }
    }
    return out;
  }

 private:
  Ciphertext deg1(const Ciphertext& a) { return a->noise_deg() >= 2 ? Rescale(a) : a; }
  std::pair<Ciphertext, Ciphertext> align(Ciphertext a, Ciphertext b) {
    if (a->noise_deg() != b->noise_deg()) {
      a = deg1(a);
      b = deg1(b);
    }
    if (a->limbs() != b->limbs()) {
      a = deg1(a);
      b = deg1(b);
      const int lo = std::min(a->limbs(), b->limbs());
      a = LevelReduce(a, lo);
      b = LevelReduce(b, lo);
    }
    return {a, b};
  }

  ckks_ctx* h_ = nullptr;
  bool owns_ = true;
  int n_ = 0, limbs_ = 0, special_ = 0, alpha_ = 0;
};

using CryptoContext = std::shared_ptr<CryptoContextImpl>;

inline CryptoContext GenCryptoContext(const CCParams& p) { return std::make_shared<CryptoContextImpl>(p); }

}  // namespace ckks_b200
