// capi.cu -- the extern "C" boundary declared in include/ckks_b200.h.
// Each entry point validates its arguments, runs the device pipeline on the
// context's stream and converts C++ exceptions into status codes.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "../../include/ckks_b200.h"
#include "capi_types.hpp"
#include "ckks_internal.hpp"

using ckks::Context;
using ckks::DevPoly;
using ckks::Error;


namespace {

thread_local std::string g_error;

template <typename F>
int guard(F&& f) {
  try {
    f();
    return CKKS_OK;
  } catch (const Error& e) {
    g_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_error = e.what();
    return CKKS_EARG;
  } catch (...) {
    g_error = "unknown error";
    return CKKS_EARG;
  }
}

void need(bool ok, int code, const char* msg) {
  if (!ok) throw Error(code, msg);
}

Context& C(ckks_ctx* x) {
  need(x && x->c, CKKS_EARG, "null context");
  return *x->c;
}

void same_ctx(ckks_ctx* x, const ckks_ct* a) {
  need(a != nullptr, CKKS_EARG, "null ciphertext");
  need(a->owner == x, CKKS_EARG, "ciphertext belongs to another context");
  need(a->p.data != nullptr && a->p.limbs > 0, CKKS_ESTATE, "ciphertext holds no data");
}

void same_ctx(ckks_ctx* x, const ckks_pt* a) {
  need(a != nullptr, CKKS_EARG, "null plaintext");
  need(a->owner == x, CKKS_EARG, "plaintext belongs to another context");
  need(a->p.data != nullptr && a->p.limbs > 0, CKKS_ESTATE, "plaintext holds no data");
}

// moves a freshly computed object into the caller's handle
void take(DevPoly& dst, DevPoly& src) {
  std::swap(dst.ctx, src.ctx);
  std::swap(dst.data, src.data);
  std::swap(dst.npolys, src.npolys);
  std::swap(dst.cap, src.cap);
  std::swap(dst.limbs, src.limbs);
  std::swap(dst.scale, src.scale);
  std::swap(dst.deg, src.deg);
}

size_t stride(const DevPoly& p) { return (size_t)p.cap * p.ctx->N; }

void check_scales(double a, double b) {
  const double rel = std::fabs(a - b) / std::fmax(std::fabs(a), std::fabs(b));
  if (!(rel <= 1e-9)) throw Error(CKKS_ESCALE, "operand scales differ");
}

void ew_ct_ct(Context& c, ckks::EwOp op, const ckks_ct* a, const ckks_ct* b, ckks_ct* out) {
  need(a->p.limbs == b->p.limbs, CKKS_ELEVEL, "operands at different levels");
  need(a->p.deg == b->p.deg, CKKS_ESCALE, "operands with different noise degree");
  check_scales(a->p.scale, b->p.scale);
  const int limbs = a->p.limbs;
  DevPoly tmp;
  DevPoly* dst = &out->p;
  const bool alias_ok = (out == a || out == b) && out->p.cap >= limbs;
  if (!alias_ok) {
    tmp.ensure(&c, 2, limbs);
    dst = &tmp;
  }
  ckks::ew_binary(c, op, a->p.data, stride(a->p), b->p.data, stride(b->p), dst->data, stride(*dst), 2, limbs,
                  c.stream);
  dst->limbs = limbs;
  dst->scale = a->p.scale;
  dst->deg = a->p.deg;
  if (dst == &tmp) take(out->p, tmp);
}

// rotations of `a` by ks[0..n) into outs: one shared ModUp, then the inner
// products and ModDowns of up to 32 rotations per batched launch sequence
void rotate_many(Context& c, const ckks_ct* a, const int* ks, int n, ckks_ct* const* outs) {
  const int limbs = a->p.limbs;
  std::vector<uint32_t> gs(n);
  for (int r = 0; r < n; ++r) {
    gs[r] = c.galois(ks[r]);
    if (gs[r] != 1u && !c.switch_key(gs[r], limbs))
      throw Error(CKKS_EKEY, "rotation key not generated for index " + std::to_string(ks[r]));
  }
  std::vector<DevPoly> res(n);
  ckks::KsBatch b{};
  auto flush = [&] {
    if (b.M) ckks::keyswitch_batch(c, limbs, b, true, c.stream);
    b.M = 0;
  };
  for (int r = 0; r < n; ++r) {
    res[r].ensure(&c, 2, limbs);
    res[r].limbs = limbs;
    res[r].scale = a->p.scale;
    res[r].deg = a->p.deg;
    if (gs[r] == 1u) {
      ckks::ew_binary(c, ckks::EwOp::Copy, a->p.data, stride(a->p), nullptr, 0, res[r].data, stride(res[r]), 2,
                      limbs, c.stream);
      continue;
    }
    const int m = b.M++;
    b.d[m] = a->p.poly(1);
    b.key[m] = c.switch_key(gs[r], limbs);
    b.g[m] = gs[r];
    b.add0[m] = a->p.poly(0);
    b.add1[m] = nullptr;
    b.out0[m] = res[r].poly(0);
    b.out1[m] = res[r].poly(1);
    if (b.M == ckks::kKsBatch) flush();
  }
  flush();
  for (int r = 0; r < n; ++r) {
    outs[r]->owner = a->owner;
    take(outs[r]->p, res[r]);
  }
}

// rotations of every input in[g] by ks[0..nk) into outs[g * nk + r]: one
// ModUp per input; each key is read once for all inputs
void rotate_hoisted_batch(Context& c, const ckks_ct* const* in, int G, const int* ks, int nk,
                          ckks_ct* const* outs) {
  if (G <= 0 || nk <= 0) return;
  const int limbs = in[0]->p.limbs;
  std::vector<uint32_t> gs(nk);
  std::vector<int> live;  // non-identity rotations
  for (int r = 0; r < nk; ++r) {
    gs[r] = c.galois(ks[r]);
    if (gs[r] == 1u) continue;
    if (!c.switch_key(gs[r], limbs))
      throw Error(CKKS_EKEY, "rotation key not generated for index " + std::to_string(ks[r]));
    live.push_back(r);
  }
  std::vector<DevPoly> res((size_t)G * nk);
  for (int g = 0; g < G; ++g) {
    const ckks_ct* a = in[g];
    if (a->p.limbs != limbs) throw Error(CKKS_ELEVEL, "batched rotations need one limb count");
    for (int r = 0; r < nk; ++r) {
      DevPoly& o = res[(size_t)g * nk + r];
      o.ensure(&c, 2, limbs);
      o.limbs = limbs;
      o.scale = a->p.scale;
      o.deg = a->p.deg;
      if (gs[r] == 1u)
        ckks::ew_binary(c, ckks::EwOp::Copy, a->p.data, stride(a->p), nullptr, 0, o.data, stride(o), 2, limbs,
                        c.stream);
    }
  }
  for (int g0 = 0; g0 < G; g0 += ckks::kKsBatch) {
    const int gn = std::min(ckks::kKsBatch, G - g0);
    for (size_t r0 = 0; r0 < live.size(); r0 += ckks::kKsBatch) {
      const int rn = (int)std::min<size_t>(ckks::kKsBatch, live.size() - r0);
      ckks::HoistKeys h{};
      h.R = rn;
      for (int i = 0; i < rn; ++i) {
        h.key[i] = c.switch_key(gs[live[r0 + i]], limbs);
        h.g[i] = gs[live[r0 + i]];
      }
      std::vector<const uint64_t*> d(gn), c0(gn);
      std::vector<uint64_t*> o0((size_t)gn * rn), o1((size_t)gn * rn);
      for (int g = 0; g < gn; ++g) {
        d[g] = in[g0 + g]->p.poly(1);
        c0[g] = in[g0 + g]->p.poly(0);
        for (int i = 0; i < rn; ++i) {
          DevPoly& o = res[(size_t)(g0 + g) * nk + live[r0 + i]];
          o0[(size_t)g * rn + i] = o.poly(0);
          o1[(size_t)g * rn + i] = o.poly(1);
        }
      }
      ckks::keyswitch_hoisted_multi(c, limbs, d.data(), c0.data(), gn, h, o0.data(), o1.data(), c.stream);
    }
  }
  for (size_t i = 0; i < res.size(); ++i) {
    outs[i]->owner = in[i / nk]->owner;
    take(outs[i]->p, res[i]);
  }
}

// independent rotations in[i] by ks[i] (all at one limb count)
void rotate_batch(Context& c, const ckks_ct* const* in, const int* ks, int n, ckks_ct* const* outs) {
  if (n <= 0) return;
  const int limbs = in[0]->p.limbs;
  std::vector<DevPoly> res(n);
  ckks::KsBatch b{};
  auto flush = [&] {
    if (b.M) ckks::keyswitch_batch(c, limbs, b, false, c.stream);
    b.M = 0;
  };
  for (int r = 0; r < n; ++r) {
    const ckks_ct* a = in[r];
    if (a->p.limbs != limbs) throw Error(CKKS_ELEVEL, "batched rotations need one limb count");
    const uint32_t g = c.galois(ks[r]);
    res[r].ensure(&c, 2, limbs);
    res[r].limbs = limbs;
    res[r].scale = a->p.scale;
    res[r].deg = a->p.deg;
    if (g == 1u) {
      ckks::ew_binary(c, ckks::EwOp::Copy, a->p.data, stride(a->p), nullptr, 0, res[r].data, stride(res[r]), 2,
                      limbs, c.stream);
      continue;
    }
    if (!c.switch_key(g, limbs))
      throw Error(CKKS_EKEY, "rotation key not generated for index " + std::to_string(ks[r]));
    const int m = b.M++;
    b.d[m] = a->p.poly(1);
    b.key[m] = c.switch_key(g, limbs);
    b.g[m] = g;
    b.add0[m] = a->p.poly(0);
    b.add1[m] = nullptr;
    b.out0[m] = res[r].poly(0);
    b.out1[m] = res[r].poly(1);
    if (b.M == ckks::kKsBatch) flush();
  }
  flush();
  for (int r = 0; r < n; ++r) {
    outs[r]->owner = in[r]->owner;
    take(outs[r]->p, res[r]);
  }
}

// out[i] = sum_r rot(in[i], ks[r]) for every i (index 0 adds in[i] itself):
// the rotations of one input share its ModUp and one ModDown, and up to 32
// inputs go through each launch (all at one limb count; distinct indices)
void hoisted_sum_batch(Context& c, const ckks_ct* const* in, int n, const int* ks, int R, std::vector<DevPoly>& res) {
  res.assign(n, DevPoly());
  if (n <= 0) return;
  const int limbs = in[0]->p.limbs;
  ckks::HoistKeys h{};
  bool identity = false;
  std::vector<uint32_t> seen;
  for (int r = 0; r < R; ++r) {
    const uint32_t g = c.galois(ks[r]);
    if (std::find(seen.begin(), seen.end(), g) != seen.end())
      throw Error(CKKS_EARG, "rotation indices of a hoisted sum must be distinct");
    seen.push_back(g);
    if (g == 1u) {
      identity = true;
      continue;
    }
    if (!c.switch_key(g, limbs))
      throw Error(CKKS_EKEY, "rotation key not generated for index " + std::to_string(ks[r]));
    if (h.R == ckks::kKsBatch) throw Error(CKKS_EARG, "hoisted sum of more than 32 rotations");
    h.key[h.R] = c.switch_key(g, limbs);
    h.g[h.R] = g;
    ++h.R;
  }
  for (int i = 0; i < n; ++i) {
    if (in[i]->p.limbs != limbs) throw Error(CKKS_ELEVEL, "batched rotation sums need one limb count");
    res[i].ensure(&c, 2, limbs);
    res[i].limbs = limbs;
    res[i].scale = in[i]->p.scale;
    res[i].deg = in[i]->p.deg;
    if (!h.R) {
      if (identity)
        ckks::ew_binary(c, ckks::EwOp::Copy, in[i]->p.data, stride(in[i]->p), nullptr, 0, res[i].data,
                        stride(res[i]), 2, limbs, c.stream);
      else
        CKKS_CUDA(cudaMemsetAsync(res[i].data, 0, sizeof(uint64_t) * stride(res[i]) * 2, c.stream));
    }
  }
  if (!h.R) return;
  for (int i0 = 0; i0 < n; i0 += ckks::kKsBatch) {
    ckks::KsBatch b{};
    b.M = std::min(ckks::kKsBatch, n - i0);
    for (int m = 0; m < b.M; ++m) {
      const ckks_ct* a = in[i0 + m];
      b.d[m] = a->p.poly(1);
      b.add0[m] = a->p.poly(0);
      b.out0[m] = res[i0 + m].poly(0);
      b.out1[m] = res[i0 + m].poly(1);
    }
    ckks::keyswitch_hoisted_sum(c, limbs, b, h, identity, c.stream);
  }
}

// sum of polynomial pairs (c0, c1) at one limb count into `out` (up to 64
// addends per launch; later launches add onto the running sum)
void sum_pairs(Context& c, const std::vector<std::pair<const uint64_t*, const uint64_t*>>& terms, int limbs,
               DevPoly& out) {
  size_t i = 0;
  bool first = true;
  while (i < terms.size()) {
    ckks::SumPtrs sp{};
    int k = 0;
    if (!first) {
      sp.in0[k] = out.poly(0);
      sp.in1[k] = out.poly(1);
      ++k;
    }
    for (; i < terms.size() && k < ckks::kSumMax; ++i, ++k) {
      sp.in0[k] = terms[i].first;
      sp.in1[k] = terms[i].second;
    }
    sp.out0 = out.poly(0);
    sp.out1 = out.poly(1);
    ckks::add_many(c, sp, k, limbs, c.stream);
    first = false;
  }
}

// sum_r rot(in[r], ks[r]): the key switches of up to 32 non-identity
// rotations are summed in the extended basis with one ModDown per group of
// 32 (in input order); identity rotations and the groups' results are added
void rotate_sum(Context& c, const ckks_ct* const* in, const int* ks, int n, DevPoly& res) {
  const int limbs = in[0]->p.limbs;
  std::vector<std::unique_ptr<DevPoly>> parts;
  std::vector<std::pair<const uint64_t*, const uint64_t*>> terms;
  ckks::KsBatch b{};
  auto flush = [&] {
    if (!b.M) return;
    parts.emplace_back(new DevPoly);
    DevPoly& p = *parts.back();
    p.ensure(&c, 2, limbs);
    ckks::keyswitch_sum(c, limbs, b, p.poly(0), p.poly(1), c.stream);
    terms.push_back({p.poly(0), p.poly(1)});
    b.M = 0;
  };
  for (int r = 0; r < n; ++r) {
    const ckks_ct* a = in[r];
    const uint32_t g = c.galois(ks[r]);
    if (g == 1u) {
      terms.push_back({a->p.poly(0), a->p.poly(1)});
      continue;
    }
    if (!c.switch_key(g, limbs))
      throw Error(CKKS_EKEY, "rotation key not generated for index " + std::to_string(ks[r]));
    const int m = b.M++;
    b.d[m] = a->p.poly(1);
    b.key[m] = c.switch_key(g, limbs);
    b.g[m] = g;
    b.add0[m] = a->p.poly(0);
    b.add1[m] = nullptr;
    if (b.M == ckks::kKsBatch) flush();
  }
  flush();
  res.ensure(&c, 2, limbs);
  if (terms.size() == 1 && !parts.empty()) {
    std::swap(res.data, parts[0]->data);
    std::swap(res.cap, parts[0]->cap);
    std::swap(res.npolys, parts[0]->npolys);
  } else {
    sum_pairs(c, terms, limbs, res);
  }
  res.limbs = limbs;
  res.scale = in[0]->p.scale;
  res.deg = in[0]->p.deg;
}

// outs[g] = sum_r rot(in[g * n + r], ks[r]) for G groups: when the groups'
// rotations hold at most one identity and 32 others, the groups' giant-step
// sums run together, up to 4 groups per launch sequence
// (keyswitch_sum_groups); otherwise one rotate_sum per group
void rotate_sum_groups(Context& c, const ckks_ct* const* in, int G, const int* ks, int n, DevPoly* outs) {
  const int limbs = in[0]->p.limbs;
  int ident = -1, others = 0;
  bool shared = true;
  std::vector<uint32_t> gs(n);
  for (int r = 0; r < n; ++r) {
    gs[r] = c.galois(ks[r]);
    if (gs[r] == 1u) {
      if (ident >= 0) shared = false;
      ident = r;
    } else {
      ++others;
      if (!c.switch_key(gs[r], limbs))
        throw Error(CKKS_EKEY, "rotation key not generated for index " + std::to_string(ks[r]));
    }
  }
  if (others == 0 || others > ckks::kKsBatch) shared = false;
  if (!shared) {
    for (int gi = 0; gi < G; ++gi) rotate_sum(c, in + (size_t)gi * n, ks, n, outs[gi]);
    return;
  }
  for (int g0 = 0; g0 < G; g0 += ckks::kSumGroups) {
    const int k = std::min(ckks::kSumGroups, G - g0);
    std::vector<ckks::KsBatch> bs(k);
    ckks::SumGroups sg{};
    for (int i = 0; i < k; ++i) {
      const ckks_ct* const* gin = in + (size_t)(g0 + i) * n;
      ckks::KsBatch& b = bs[i];
      b = ckks::KsBatch{};
      for (int r = 0; r < n; ++r) {
        if (r == ident) continue;
        const int m = b.M++;
        b.d[m] = gin[r]->p.poly(1);
        b.key[m] = c.switch_key(gs[r], limbs);
        b.g[m] = gs[r];
        b.add0[m] = gin[r]->p.poly(0);
      }
      DevPoly& o = outs[g0 + i];
      o.ensure(&c, 2, limbs);
      o.limbs = limbs;
      o.scale = gin[0]->p.scale;
      o.deg = gin[0]->p.deg;
      sg.out0[i] = o.poly(0);
      sg.out1[i] = o.poly(1);
      if (ident >= 0) {
        sg.id0[i] = gin[ident]->p.poly(0);
        sg.id1[i] = gin[ident]->p.poly(1);
      }
    }
    ckks::keyswitch_sum_groups(c, limbs, bs.data(), sg, k, c.stream);
  }
}

// tensor + relinearisation of (a[i], b[i]) pairs at one limb count
void mul_ct_batch(Context& c, const ckks_ct* const* a, const ckks_ct* const* bb, int n, ckks_ct* const* outs) {
  if (n <= 0) return;
  const int limbs = a[0]->p.limbs, N = c.N;
  if (!c.switch_key(1u, limbs)) throw Error(CKKS_EKEY, "relinearisation key not generated");
  const size_t S = (size_t)limbs * N;
  std::vector<DevPoly> res(n);
  std::vector<uint64_t*> dbuf;
  ckks::KsBatch b{};
  ckks::TensorBatch tb{};
  tb.S = S;
  auto flush = [&] {
    ckks::tensor_batch(c, tb, limbs, c.stream);  // the batch's tensors in one launch
    if (b.M) ckks::keyswitch_batch(c, limbs, b, false, c.stream);
    b.M = 0;
    tb.M = 0;
    for (uint64_t* p : dbuf) c.release(p);
    dbuf.clear();
  };
  for (int r = 0; r < n; ++r) {
    if (a[r]->p.limbs != limbs || bb[r]->p.limbs != limbs)
      throw Error(CKKS_ELEVEL, "operands at different levels");
    uint64_t* d = (uint64_t*)c.alloc(sizeof(uint64_t) * 3 * S);
    dbuf.push_back(d);
    tb.a0[tb.M] = a[r]->p.poly(0);
    tb.a1[tb.M] = a[r]->p.poly(1);
    tb.b0[tb.M] = bb[r]->p.poly(0);
    tb.b1[tb.M] = bb[r]->p.poly(1);
    tb.d[tb.M] = d;
    ++tb.M;
    res[r].ensure(&c, 2, limbs);
    res[r].limbs = limbs;
    res[r].scale = a[r]->p.scale * bb[r]->p.scale;
    res[r].deg = a[r]->p.deg + bb[r]->p.deg;
    const int m = b.M++;
    b.d[m] = d + 2 * S;
    b.key[m] = c.switch_key(1u, limbs);
    b.g[m] = 1u;
    b.add0[m] = d;
    b.add1[m] = d + S;
    b.out0[m] = res[r].poly(0);
    b.out1[m] = res[r].poly(1);
    if (b.M == ckks::kKsBatch) flush();
  }
  flush();
  for (int r = 0; r < n; ++r) {
    outs[r]->owner = a[r]->owner;
    take(outs[r]->p, res[r]);
  }
}

// sum_r a[r] * b[r] with one relinearisation: the tensor products are
// summed as degree-2 ciphertexts (31 pairs per launch), then d2 is switched
// once
void mul_ct_sum(Context& c, const ckks_ct* const* a, const ckks_ct* const* bb, int n, DevPoly& res) {
  const int limbs = a[0]->p.limbs, N = c.N;
  if (!c.switch_key(1u, limbs)) throw Error(CKKS_EKEY, "relinearisation key not generated");
  const size_t S = (size_t)limbs * N;
  const double sc = a[0]->p.scale * bb[0]->p.scale;
  const int deg = a[0]->p.deg + bb[0]->p.deg;
  for (int r = 0; r < n; ++r) {
    if (a[r]->p.limbs != limbs || bb[r]->p.limbs != limbs) throw Error(CKKS_ELEVEL, "operands at different levels");
    if (a[r]->p.deg + bb[r]->p.deg != deg) throw Error(CKKS_ESCALE, "products of different noise degree");
    check_scales(sc, a[r]->p.scale * bb[r]->p.scale);
  }
  uint64_t* d = (uint64_t*)c.alloc(sizeof(uint64_t) * 3 * S);
  for (int r0 = 0; r0 < n; r0 += ckks::kTensorSum) {
    const int k = std::min(ckks::kTensorSum, n - r0);
    ckks::TensorPtrs tp{};
    for (int i = 0; i < k; ++i) {
      tp.a0[i] = a[r0 + i]->p.poly(0);
      tp.a1[i] = a[r0 + i]->p.poly(1);
      tp.b0[i] = bb[r0 + i]->p.poly(0);
      tp.b1[i] = bb[r0 + i]->p.poly(1);
    }
    ckks::tensor_sum(c, tp, k, r0 > 0, d, d + S, d + 2 * S, limbs, c.stream);
  }
  res.ensure(&c, 2, limbs);
  ckks::KsBatch b{};
  b.M = 1;
  b.d[0] = d + 2 * S;
  b.key[0] = c.switch_key(1u, limbs);
  b.g[0] = 1u;
  b.add0[0] = d;
  b.add1[0] = d + S;
  b.out0[0] = res.poly(0);
  b.out1[0] = res.poly(1);
  ckks::keyswitch_batch(c, limbs, b, false, c.stream);
  c.release(d);
  res.limbs = limbs;
  res.scale = sc;
  res.deg = deg;
}

void rescale_many(Context& c, const ckks_ct* const* in, int n, ckks_ct* const* outs) {
  if (n <= 0) return;
  const int limbs = in[0]->p.limbs;
  if (limbs < 2) throw Error(CKKS_ELEVEL, "no limb left to rescale");
  std::vector<DevPoly> res(n);
  ckks::RsBatch b{};
  auto flush = [&] {
    if (b.M) ckks::rescale_batch(c, limbs, b, c.stream);
    b.M = 0;
  };
  for (int r = 0; r < n; ++r) {
    if (in[r]->p.limbs != limbs) throw Error(CKKS_ELEVEL, "batched rescale needs one limb count");
    res[r].ensure(&c, 2, limbs - 1);
    res[r].limbs = limbs - 1;
    res[r].scale = in[r]->p.scale / (double)c.moduli[limbs - 1];
    res[r].deg = in[r]->p.deg > 1 ? in[r]->p.deg - 1 : 1;
    const int m = b.M++;
    b.in0[m] = in[r]->p.poly(0);
    b.in1[m] = in[r]->p.poly(1);
    b.out0[m] = res[r].poly(0);
    b.out1[m] = res[r].poly(1);
    if (b.M == ckks::kKsBatch) flush();
  }
  flush();
  for (int r = 0; r < n; ++r) {
    outs[r]->owner = in[r]->owner;
    take(outs[r]->p, res[r]);
  }
}

}  // namespace

void ckks::set_last_error(const std::string& msg) { g_error = msg; }

extern "C" {

const char* ckks_last_error(void) { return g_error.c_str(); }

int ckks_ctx_create(const ckks_params* params, ckks_ctx** out) {
  return guard([&] {
    need(params && out, CKKS_EARG, "null argument");
    ckks::Params p;
    p.log_n = params->log_n;
    p.limbs = params->limbs;
    p.dnum = params->dnum;
    p.first_mod_bits = params->first_mod_bits;
    p.scale_mod_bits = params->scale_mod_bits;
    p.special_mod_bits = params->special_mod_bits;
    p.seed = params->seed;
    p.device = params->device;
    auto* x = new ckks_ctx;
    try {
      x->c = std::make_unique<Context>(p);
    } catch (...) {
      delete x;
      throw;
    }
    *out = x;
  });
}

int ckks_ctx_destroy(ckks_ctx* ctx) {
  return guard([&] {
    if (!ctx) return;
    {
      std::lock_guard<std::mutex> lk(ctx->mu);
      // ciphertexts and plaintexts first: a block's cached plaintexts are
      // then already detached when the block releases them below
      for (ckks_ct* t : ctx->cts) {
        if (t->p.data && t->p.ctx) t->p.ctx->release(t->p.data);
        t->p.data = nullptr;
        t->p.ctx = nullptr;
        t->owner = nullptr;
      }
      for (ckks_pt* t : ctx->pts) {
        if (t->p.data && t->p.ctx) t->p.ctx->release(t->p.data);
        t->p.data = nullptr;
        t->p.ctx = nullptr;
        t->owner = nullptr;
      }
      for (ckks_diag* d : ctx->diags) {
        if (d->data) ctx->c->release(d->data);
        d->data = nullptr;
        d->owner = nullptr;
      }
      ctx->cts.clear();
      ctx->pts.clear();
      ctx->diags.clear();
      for (ckks_block* b : ctx->blocks) ckks::block_orphan(b);
      ctx->blocks.clear();
    }
    delete ctx;
  });
}

int ckks_ctx_info(const ckks_ctx* ctx, int* ring_dim, int* limbs, int* special, int* alpha) {
  return guard([&] {
    need(ctx && ctx->c, CKKS_EARG, "null context");
    const Context& c = *ctx->c;
    if (ring_dim) *ring_dim = c.N;
    if (limbs) *limbs = c.L;
    if (special) *special = c.K;
    if (alpha) *alpha = c.alpha;
  });
}

int ckks_ctx_low_set(const ckks_ctx* ctx, int* low_limbs, int* low_special) {
  return guard([&] {
    need(ctx && ctx->c, CKKS_EARG, "null context");
    if (low_limbs) *low_limbs = ctx->c->low_limbs;
    if (low_special) *low_special = ctx->c->K_low;
  });
}

int ckks_ctx_moduli(const ckks_ctx* ctx, uint64_t* out, int count) {
  return guard([&] {
    need(ctx && ctx->c && out, CKKS_EARG, "null argument");
    const Context& c = *ctx->c;
    need(count >= 0 && count <= c.P, CKKS_EARG, "count above L+K");
    std::memcpy(out, c.moduli.data(), sizeof(uint64_t) * count);
  });
}

double ckks_ctx_scale(const ckks_ctx* ctx, int level) {
  if (!ctx || !ctx->c) return 0.0;
  const Context& c = *ctx->c;
  const int limbs = c.L - level;
  if (limbs < 1 || limbs > c.L) return 0.0;
  return c.scales[limbs];
}

int ckks_sync(ckks_ctx* ctx) {
  return guard([&] {
    Context& c = C(ctx);
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
    const unsigned int f = ckks::take_device_faults(c);
    if (f)
      throw Error(CKKS_ECUDA, std::to_string(f) +
                                  " bounded device wait(s) gave up (a bulk copy into shared memory did not complete); "
                                  "the outputs since the last synchronisation are not valid");
  });
}

int ckks_selftest_bulk_wait(ckks_ctx* ctx, int starve) {
  return guard([&] {
    Context& c = C(ctx);
    constexpr int kWords = 512;
    std::vector<uint64_t> h(kWords), back(kWords, 0);
    for (int i = 0; i < kWords; ++i) h[i] = 0x9e3779b97f4a7c15ull * (uint64_t)(i + 1);
    uint64_t* d = (uint64_t*)c.alloc(2 * kWords * sizeof(uint64_t));
    CKKS_CUDA(cudaMemcpyAsync(d, h.data(), kWords * sizeof(uint64_t), cudaMemcpyHostToDevice, c.stream));
    CKKS_CUDA(cudaMemsetAsync(d + kWords, 0, kWords * sizeof(uint64_t), c.stream));
    ckks::bulk_wait_probe(c, d, d + kWords, starve != 0, c.stream);
    CKKS_CUDA(cudaMemcpyAsync(back.data(), d + kWords, kWords * sizeof(uint64_t), cudaMemcpyDeviceToHost, c.stream));
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
    c.release(d);
    const unsigned int f = ckks::take_device_faults(c);
    if (f) throw Error(CKKS_ECUDA, "bounded bulk-copy wait gave up");
    need(back == h, CKKS_ECUDA, "bulk copy through shared memory returned different data");
  });
}

void* ckks_ctx_stream(ckks_ctx* ctx) { return (ctx && ctx->c) ? (void*)ctx->c->stream : nullptr; }

int ckks_keygen(ckks_ctx* ctx) {
  return guard([&] { ckks::keygen_secret_public(C(ctx)); });
}

int ckks_relin_keygen(ckks_ctx* ctx) {
  return guard([&] {
    Context& c = C(ctx);
    need(c.d_sk != nullptr, CKKS_ESTATE, "secret key not generated");
    uint64_t* s2 = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)c.P * c.N);
    // s^2 over every prime (NTT form)
    ckks::ew_binary(c, ckks::EwOp::Mul, c.d_sk, 0, c.d_sk, 0, s2, 0, 1, c.P, c.stream);
    c.install_key(0, ckks::make_switch_key(c, s2, 1u));
    if (c.low_limbs) c.install_key(0, ckks::make_switch_key_low(c, s2, 1u), true);
    c.release(s2);
  });
}

int ckks_rotkey_gen(ckks_ctx* ctx, const int* indices, int count) {
  return guard([&] {
    Context& c = C(ctx);
    need(c.d_sk != nullptr, CKKS_ESTATE, "secret key not generated");
    need(count >= 0 && (count == 0 || indices), CKKS_EARG, "bad index list");
    uint64_t* sg = (uint64_t*)c.alloc(sizeof(uint64_t) * (size_t)c.P * c.N);
    for (int i = 0; i < count; ++i) {
      const uint32_t g = c.galois(indices[i]);
      if (g == 1u || c.rot_key(g)) continue;
      ckks::automorphism(c, c.d_sk, sg, c.P, g, c.stream);
      c.rot_keys[g] = ckks::make_switch_key(c, sg, 0x100u + g);
      if (c.low_limbs) {
        auto it = c.rot_keys_low.find(g);
        if (it != c.rot_keys_low.end()) cudaFree(it->second);
        c.rot_keys_low[g] = ckks::make_switch_key_low(c, sg, 0x100u + g);
      }
    }
    c.release(sg);
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  });
}

int ckks_key_export(ckks_ctx* ctx, int which, int k, uint64_t* host, size_t words) {
  return guard([&] {
    Context& c = C(ctx);
    need(host != nullptr, CKKS_EARG, "null buffer");
    const uint64_t* src = nullptr;
    size_t n = 0;
    switch (which) {
      case 0: src = c.d_sk; n = (size_t)c.P * c.N; break;
      case 1: src = c.d_pk; n = 2 * (size_t)c.L * c.N; break;
      case 2: src = c.d_rlk; n = c.key_words(); break;
      case 3: src = c.rot_key(c.galois(k)); n = c.key_words(); break;
      case 4: src = c.d_rlk_low; n = c.low_key_words(); break;
      case 5: {
        auto it = c.rot_keys_low.find(c.galois(k));
        src = it == c.rot_keys_low.end() ? nullptr : it->second;
        n = c.low_key_words();
        break;
      }
      default: throw Error(CKKS_EARG, "unknown key kind");
    }
    need(src != nullptr, CKKS_EKEY, "key not generated");
    need(words >= n, CKKS_EARG, "host buffer too small");
    CKKS_CUDA(cudaMemcpyAsync(host, src, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost, c.stream));
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  });
}

int ckks_ct_create(ckks_ctx* ctx, ckks_ct** out) {
  return guard([&] {
    C(ctx);
    need(out != nullptr, CKKS_EARG, "null argument");
    auto* t = new ckks_ct;
    t->owner = ctx;
    {
      std::lock_guard<std::mutex> lk(ctx->mu);
      ctx->cts.insert(t);
    }
    *out = t;
  });
}

int ckks_ct_destroy(ckks_ct* ct) {
  return guard([&] {
    if (!ct) return;
    if (ct->owner) {
      std::lock_guard<std::mutex> lk(ct->owner->mu);
      ct->owner->cts.erase(ct);
    }
    delete ct;
  });
}

int ckks_pt_create(ckks_ctx* ctx, ckks_pt** out) {
  return guard([&] {
    C(ctx);
    need(out != nullptr, CKKS_EARG, "null argument");
    auto* t = new ckks_pt;
    t->owner = ctx;
    {
      std::lock_guard<std::mutex> lk(ctx->mu);
      ctx->pts.insert(t);
    }
    *out = t;
  });
}

int ckks_pt_destroy(ckks_pt* pt) {
  return guard([&] {
    if (!pt) return;
    if (pt->owner) {
      std::lock_guard<std::mutex> lk(pt->owner->mu);
      pt->owner->pts.erase(pt);
    }
    delete pt;
  });
}

int ckks_ct_level(const ckks_ct* ct) {
  if (!ct || !ct->p.ctx) return -1;
  return ct->p.ctx->L - ct->p.limbs;
}
int ckks_ct_limbs(const ckks_ct* ct) { return ct ? ct->p.limbs : -1; }
double ckks_ct_scale(const ckks_ct* ct) { return ct ? ct->p.scale : 0.0; }
int ckks_ct_noise_deg(const ckks_ct* ct) { return ct ? ct->p.deg : -1; }
int ckks_pt_limbs(const ckks_pt* pt) { return pt ? pt->p.limbs : -1; }
double ckks_pt_scale(const ckks_pt* pt) { return pt ? pt->p.scale : 0.0; }

int ckks_ct_set_scale(ckks_ct* ct, double scale, int noise_deg) {
  return guard([&] {
    need(ct != nullptr && scale > 0.0 && noise_deg >= 1, CKKS_EARG, "bad scale");
    ct->p.scale = scale;
    ct->p.deg = noise_deg;
  });
}

int ckks_ct_export(ckks_ctx* ctx, const ckks_ct* ct, uint64_t* host, size_t words) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, ct);
    const size_t per = (size_t)ct->p.limbs * c.N;
    need(host && words >= 2 * per, CKKS_EARG, "host buffer too small");
    for (int p = 0; p < 2; ++p)
      CKKS_CUDA(cudaMemcpyAsync(host + p * per, ct->p.poly(p), sizeof(uint64_t) * per, cudaMemcpyDeviceToHost,
                                c.stream));
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  });
}

int ckks_ct_import(ckks_ctx* ctx, ckks_ct* ct, const uint64_t* host, int limbs, double scale, int noise_deg) {
  return guard([&] {
    Context& c = C(ctx);
    need(ct && ct->owner == ctx && host, CKKS_EARG, "bad argument");
    need(limbs >= 1 && limbs <= c.L, CKKS_EARG, "limb count outside 1..L");
    DevPoly tmp;
    tmp.ensure(&c, 2, limbs);
    const size_t per = (size_t)limbs * c.N;
    for (int p = 0; p < 2; ++p)
      CKKS_CUDA(cudaMemcpyAsync(tmp.poly(p), host + p * per, sizeof(uint64_t) * per, cudaMemcpyHostToDevice,
                                c.stream));
    tmp.limbs = limbs;
    tmp.scale = scale;
    tmp.deg = noise_deg;
    take(ct->p, tmp);
  });
}

int ckks_pt_export(ckks_ctx* ctx, const ckks_pt* pt, uint64_t* host, size_t words) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, pt);
    const size_t per = (size_t)pt->p.limbs * c.N;
    need(host && words >= per, CKKS_EARG, "host buffer too small");
    CKKS_CUDA(cudaMemcpyAsync(host, pt->p.data, sizeof(uint64_t) * per, cudaMemcpyDeviceToHost, c.stream));
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  });
}

int ckks_pt_import(ckks_ctx* ctx, ckks_pt* pt, const uint64_t* host, int limbs, double scale) {
  return guard([&] {
    Context& c = C(ctx);
    need(pt && pt->owner == ctx && host, CKKS_EARG, "bad argument");
    need(limbs >= 1 && limbs <= c.L, CKKS_EARG, "limb count outside 1..L");
    DevPoly tmp;
    tmp.ensure(&c, 1, limbs);
    CKKS_CUDA(cudaMemcpyAsync(tmp.data, host, sizeof(uint64_t) * (size_t)limbs * c.N, cudaMemcpyHostToDevice,
                              c.stream));
    tmp.limbs = limbs;
    tmp.scale = scale;
    take(pt->p, tmp);
  });
}

int ckks_ct_copy(ckks_ctx* ctx, const ckks_ct* src, ckks_ct* dst) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, src);
    need(dst && dst->owner == ctx, CKKS_EARG, "bad destination");
    if (src == dst) return;
    DevPoly tmp;
    tmp.ensure(&c, 2, src->p.limbs);
    ckks::ew_binary(c, ckks::EwOp::Copy, src->p.data, stride(src->p), nullptr, 0, tmp.data, stride(tmp), 2,
                    src->p.limbs, c.stream);
    tmp.limbs = src->p.limbs;
    tmp.scale = src->p.scale;
    tmp.deg = src->p.deg;
    take(dst->p, tmp);
  });
}

int ckks_encode_at(ckks_ctx* ctx, const double* values, int count, int limbs, double scale, ckks_pt* out) {
  return guard([&] {
    Context& c = C(ctx);
    need(out && out->owner == ctx, CKKS_EARG, "bad plaintext handle");
    need(values || count == 0, CKKS_EARG, "null values");
    need(count >= 0 && count <= c.N / 2, CKKS_EARG, "more values than slots");
    need(limbs >= 1 && limbs <= c.L, CKKS_EARG, "limb count outside 1..L");
    need(scale > 0.0 && std::isfinite(scale), CKKS_EARG, "bad scale");
    for (int i = 0; i < count; ++i) need(std::isfinite(values[i]), CKKS_EARG, "non-finite value");
    const int n = c.N / 2;
    double* dv = (double*)c.alloc(sizeof(double) * n);
    CKKS_CUDA(cudaMemsetAsync(dv, 0, sizeof(double) * n, c.stream));
    if (count) CKKS_CUDA(cudaMemcpyAsync(dv, values, sizeof(double) * count, cudaMemcpyHostToDevice, c.stream));
    DevPoly tmp;
    tmp.ensure(&c, 1, limbs);
    ckks::encode(c, dv, limbs, scale, tmp.data, c.stream);
    tmp.limbs = limbs;
    tmp.scale = scale;
    c.release(dv);
    CKKS_CUDA(cudaStreamSynchronize(c.stream));  // host values may be released on return
    take(out->p, tmp);
  });
}

int ckks_encode(ckks_ctx* ctx, const double* values, int count, int level, ckks_pt* out) {
  if (!ctx || !ctx->c) {
    g_error = "null context";
    return CKKS_EARG;
  }
  const Context& c = *ctx->c;
  const int limbs = c.L - level;
  if (limbs < 1 || limbs > c.L) {
    g_error = "level outside 0..L-1";
    return CKKS_EARG;
  }
  return ckks_encode_at(ctx, values, count, limbs, c.scales[limbs], out);
}

int ckks_decode(ckks_ctx* ctx, const ckks_pt* pt, double* out, int count) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, pt);
    need(out != nullptr && count >= 0 && count <= c.N / 2, CKKS_EARG, "bad output buffer");
    const int n = c.N / 2;
    double* dv = (double*)c.alloc(sizeof(double) * n);
    ckks::decode(c, pt->p.data, pt->p.limbs, pt->p.scale, dv, c.stream);
    if (count) CKKS_CUDA(cudaMemcpyAsync(out, dv, sizeof(double) * count, cudaMemcpyDeviceToHost, c.stream));
    c.release(dv);
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  });
}

int ckks_encrypt(ckks_ctx* ctx, const ckks_pt* pt, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, pt);
    need(out && out->owner == ctx, CKKS_EARG, "bad ciphertext handle");
    DevPoly tmp;
    tmp.ensure(&c, 2, pt->p.limbs);
    ckks::encrypt(c, pt->p.data, pt->p.limbs, c.enc_counter++, tmp.poly(0), tmp.poly(1));
    tmp.limbs = pt->p.limbs;
    tmp.scale = pt->p.scale;
    tmp.deg = 1;
    take(out->p, tmp);
  });
}

int ckks_decrypt(ckks_ctx* ctx, const ckks_ct* ct, ckks_pt* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, ct);
    need(out && out->owner == ctx, CKKS_EARG, "bad plaintext handle");
    DevPoly tmp;
    tmp.ensure(&c, 1, ct->p.limbs);
    ckks::decrypt(c, ct->p.poly(0), ct->p.poly(1), ct->p.limbs, tmp.data);
    tmp.limbs = ct->p.limbs;
    tmp.scale = ct->p.scale;
    take(out->p, tmp);
  });
}

int ckks_encrypt_batch(ckks_ctx* ctx, const ckks_pt* const* pts, int count, ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (pts && outs)), CKKS_EARG, "bad batch");
    if (!count) return;
    const int limbs = pts[0]->p.limbs;
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, pts[i]);
      need(pts[i]->p.limbs == limbs, CKKS_ELEVEL, "batched encryption needs one limb count");
      need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
    }
    const size_t S = (size_t)limbs * c.N;
    uint64_t* buf = (uint64_t*)c.alloc(sizeof(uint64_t) * S * count);
    for (int i = 0; i < count; ++i)
      CKKS_CUDA(cudaMemcpyAsync(buf + (size_t)i * S, pts[i]->p.data, sizeof(uint64_t) * S, cudaMemcpyDeviceToDevice,
                                c.stream));
    std::vector<DevPoly> res(count);
    std::vector<uint64_t*> c0(count), c1(count);
    for (int i = 0; i < count; ++i) {
      res[i].ensure(&c, 2, limbs);
      res[i].limbs = limbs;
      res[i].scale = pts[i]->p.scale;
      res[i].deg = 1;
      c0[i] = res[i].poly(0);
      c1[i] = res[i].poly(1);
    }
    ckks::encrypt_batch(c, buf, limbs, count, c0.data(), c1.data(), c.stream);
    c.release(buf);
    for (int i = 0; i < count; ++i) take(outs[i]->p, res[i]);
  });
}

int ckks_decrypt_decode_batch(ckks_ctx* ctx, const ckks_ct* const* cts, int count, double* out, int slots) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (cts && out)), CKKS_EARG, "bad batch");
    need(slots >= 0 && slots <= c.N / 2, CKKS_EARG, "more values than slots");
    if (!count) return;
    const int limbs = cts[0]->p.limbs;
    std::vector<const uint64_t*> c0(count), c1(count);
    std::vector<double> sc(count);
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, cts[i]);
      need(cts[i]->p.limbs == limbs, CKKS_ELEVEL, "batched decryption needs one limb count");
      c0[i] = cts[i]->p.poly(0);
      c1[i] = cts[i]->p.poly(1);
      sc[i] = cts[i]->p.scale;
    }
    const int n = c.N / 2;
    double* dv = (double*)c.alloc(sizeof(double) * (size_t)n * count);
    ckks::decrypt_decode_batch(c, c0.data(), c1.data(), limbs, count, sc.data(), dv, c.stream);
    if (slots)
      CKKS_CUDA(cudaMemcpy2DAsync(out, sizeof(double) * slots, dv, sizeof(double) * n, sizeof(double) * slots, count,
                                  cudaMemcpyDeviceToHost, c.stream));
    c.release(dv);
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  });
}

int ckks_set_encrypt_counter(ckks_ctx* ctx, uint64_t counter) {
  return guard([&] { C(ctx).enc_counter = counter; });
}

uint64_t ckks_get_encrypt_counter(const ckks_ctx* ctx) { return (ctx && ctx->c) ? ctx->c->enc_counter : 0; }

int ckks_add(ckks_ctx* ctx, const ckks_ct* a, const ckks_ct* b, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    same_ctx(ctx, b);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    ew_ct_ct(c, ckks::EwOp::Add, a, b, out);
  });
}

int ckks_sub(ckks_ctx* ctx, const ckks_ct* a, const ckks_ct* b, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    same_ctx(ctx, b);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    ew_ct_ct(c, ckks::EwOp::Sub, a, b, out);
  });
}

int ckks_add_many(ckks_ctx* ctx, const ckks_ct* const* in, int count, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 1 && in, CKKS_EARG, "empty sum");
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    const int limbs = in[0]->p.limbs;
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, in[i]);
      need(in[i]->p.limbs == limbs, CKKS_ELEVEL, "operands at different levels");
      need(in[i]->p.deg == in[0]->p.deg, CKKS_ESCALE, "operands with different noise degree");
      check_scales(in[0]->p.scale, in[i]->p.scale);
    }
    DevPoly tmp;
    tmp.ensure(&c, 2, limbs);
    // up to 64 inputs per launch; later launches add onto the running sum
    // (each thread reads and writes only its own residues)
    int i = 0;
    bool first = true;
    while (i < count) {
      ckks::SumPtrs sp{};
      int k = 0;
      if (!first) {
        sp.in0[k] = tmp.poly(0);
        sp.in1[k] = tmp.poly(1);
        ++k;
      }
      for (; i < count && k < ckks::kSumMax; ++i, ++k) {
        sp.in0[k] = in[i]->p.poly(0);
        sp.in1[k] = in[i]->p.poly(1);
      }
      sp.out0 = tmp.poly(0);
      sp.out1 = tmp.poly(1);
      ckks::add_many(c, sp, k, limbs, c.stream);
      first = false;
    }
    tmp.limbs = limbs;
    tmp.scale = in[0]->p.scale;
    tmp.deg = in[0]->p.deg;
    take(out->p, tmp);
  });
}

int ckks_add_batch(ckks_ctx* ctx, const ckks_ct* const* a, const ckks_ct* const* b, int count, ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (a && b && outs)), CKKS_EARG, "bad batch");
    if (!count) return;
    const int limbs = a[0]->p.limbs;
    std::vector<DevPoly> res(count);
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, a[i]);
      same_ctx(ctx, b[i]);
      need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
      need(a[i]->p.limbs == limbs && b[i]->p.limbs == limbs, CKKS_ELEVEL, "batched adds need one limb count");
      need(a[i]->p.deg == b[i]->p.deg, CKKS_ESCALE, "operands with different noise degree");
      check_scales(a[i]->p.scale, b[i]->p.scale);
      res[i].ensure(&c, 2, limbs);
      res[i].limbs = limbs;
      res[i].scale = a[i]->p.scale;
      res[i].deg = a[i]->p.deg;
    }
    for (int s0 = 0; s0 < count; s0 += 32) {
      ckks::PairPtrs pp{};
      const int M = std::min(32, count - s0);
      for (int m = 0; m < M; ++m) {
        pp.a0[m] = a[s0 + m]->p.poly(0);
        pp.a1[m] = a[s0 + m]->p.poly(1);
        pp.b0[m] = b[s0 + m]->p.poly(0);
        pp.b1[m] = b[s0 + m]->p.poly(1);
        pp.o0[m] = res[s0 + m].poly(0);
        pp.o1[m] = res[s0 + m].poly(1);
      }
      ckks::add_pairs(c, pp, M, limbs, c.stream);
    }
    for (int i = 0; i < count; ++i) take(outs[i]->p, res[i]);
  });
}

int ckks_add_pt(ckks_ctx* ctx, const ckks_ct* a, const ckks_pt* p, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    same_ctx(ctx, p);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    need(p->p.limbs >= a->p.limbs, CKKS_ELEVEL, "plaintext has fewer limbs than the ciphertext");
    check_scales(a->p.scale, p->p.scale);
    const int limbs = a->p.limbs;
    DevPoly tmp;
    tmp.ensure(&c, 2, limbs);
    ckks::ew_binary(c, ckks::EwOp::Add, a->p.data, 0, p->p.data, 0, tmp.data, 0, 1, limbs, c.stream);
    ckks::ew_binary(c, ckks::EwOp::Copy, a->p.poly(1), 0, nullptr, 0, tmp.poly(1), 0, 1, limbs, c.stream);
    tmp.limbs = limbs;
    tmp.scale = a->p.scale;
    tmp.deg = a->p.deg;
    take(out->p, tmp);
  });
}

int ckks_add_scalar(ckks_ctx* ctx, const ckks_ct* a, double value, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    need(std::isfinite(value), CKKS_EARG, "non-finite scalar");
    const int limbs = a->p.limbs;
    DevPoly tmp;
    tmp.ensure(&c, 2, limbs);
    ckks::ew_binary(c, ckks::EwOp::Copy, a->p.data, stride(a->p), nullptr, 0, tmp.data, stride(tmp), 2, limbs,
                    c.stream);
    const double r = std::rint(value * a->p.scale);
    std::vector<uint64_t> res(limbs);
    for (int l = 0; l < limbs; ++l) res[l] = ckks::host_double_to_res(r, c.moduli[l]);
    ckks::ew_add_const(c, tmp.data, limbs, res, c.stream);
    tmp.limbs = limbs;
    tmp.scale = a->p.scale;
    tmp.deg = a->p.deg;
    take(out->p, tmp);
  });
}

int ckks_mul_pt(ckks_ctx* ctx, const ckks_ct* a, const ckks_pt* p, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    same_ctx(ctx, p);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    need(p->p.limbs >= a->p.limbs, CKKS_ELEVEL, "plaintext has fewer limbs than the ciphertext");
    const int limbs = a->p.limbs;
    DevPoly tmp;
    DevPoly* dst = &out->p;
    if (!(out == a && out->p.cap >= limbs)) {
      tmp.ensure(&c, 2, limbs);
      dst = &tmp;
    }
    ckks::ew_mul_pt(c, a->p.data, stride(a->p), p->p.data, dst->data, stride(*dst), 2, limbs, c.stream);
    dst->limbs = limbs;
    dst->scale = a->p.scale * p->p.scale;
    dst->deg = a->p.deg + 1;
    if (dst == &tmp) take(out->p, tmp);
  });
}

int ckks_mul_pt_batch(ckks_ctx* ctx, const ckks_ct* const* a, const ckks_pt* const* p, int count,
                      ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (a && p && outs)), CKKS_EARG, "bad batch");
    if (!count) return;
    const int limbs = a[0]->p.limbs;
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, a[i]);
      same_ctx(ctx, p[i]);
      need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
      need(a[i]->p.limbs == limbs, CKKS_ELEVEL, "batched products need one limb count");
      need(p[i]->p.limbs >= limbs, CKKS_ELEVEL, "plaintext has fewer limbs than the ciphertext");
    }
    std::vector<DevPoly> res(count);
    for (int i0 = 0; i0 < count; i0 += ckks::kKsBatch) {
      ckks::MulPtBatch b{};
      b.M = std::min(ckks::kKsBatch, count - i0);
      for (int m = 0; m < b.M; ++m) {
        const int i = i0 + m;
        res[i].ensure(&c, 2, limbs);
        res[i].limbs = limbs;
        res[i].scale = a[i]->p.scale * p[i]->p.scale;
        res[i].deg = a[i]->p.deg + 1;
        b.a0[m] = a[i]->p.poly(0);
        b.a1[m] = a[i]->p.poly(1);
        b.pt[m] = p[i]->p.data;
        b.o0[m] = res[i].poly(0);
        b.o1[m] = res[i].poly(1);
      }
      ckks::ew_mul_pt_batch(c, b, limbs, c.stream);
    }
    for (int i = 0; i < count; ++i) take(outs[i]->p, res[i]);
  });
}

int ckks_mul_int(ckks_ctx* ctx, const ckks_ct* a, int64_t k, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    const int limbs = a->p.limbs;
    std::vector<uint64_t> res(limbs);
    for (int l = 0; l < limbs; ++l) res[l] = ckks::host_int_to_res(k, c.moduli[l]);
    DevPoly tmp;
    tmp.ensure(&c, 2, limbs);
    ckks::ew_mul_const(c, a->p.data, stride(a->p), tmp.data, stride(tmp), 2, limbs, res, c.stream);
    tmp.limbs = limbs;
    tmp.scale = a->p.scale;
    tmp.deg = a->p.deg;
    take(out->p, tmp);
  });
}

int ckks_mul_ct(ckks_ctx* ctx, const ckks_ct* a, const ckks_ct* b, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    same_ctx(ctx, b);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    need(c.switch_key(1u, a->p.limbs) != nullptr, CKKS_EKEY, "relinearisation key not generated");
    need(a->p.limbs == b->p.limbs, CKKS_ELEVEL, "operands at different levels");
    const ckks_ct* as[1] = {a};
    const ckks_ct* bs[1] = {b};
    ckks_ct* os[1] = {out};
    mul_ct_batch(c, as, bs, 1, os);
  });
}

int ckks_mul_ct_batch(ckks_ctx* ctx, const ckks_ct* const* a, const ckks_ct* const* b, int count,
                      ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (a && b && outs)), CKKS_EARG, "bad batch");
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, a[i]);
      same_ctx(ctx, b[i]);
      need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
    }
    mul_ct_batch(c, a, b, count, outs);
  });
}

int ckks_rotate_batch(ckks_ctx* ctx, const ckks_ct* const* in, const int* k, int count, ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (in && k && outs)), CKKS_EARG, "bad batch");
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, in[i]);
      need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
    }
    rotate_batch(c, in, k, count, outs);
  });
}

int ckks_mul_ct_sum(ckks_ctx* ctx, const ckks_ct* const* a, const ckks_ct* const* b, int count, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 1 && a && b, CKKS_EARG, "empty product sum");
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, a[i]);
      same_ctx(ctx, b[i]);
    }
    DevPoly tmp;
    mul_ct_sum(c, a, b, count, tmp);
    take(out->p, tmp);
  });
}

int ckks_rotate_sum_groups(ckks_ctx* ctx, const ckks_ct* const* in, int groups, const int* k, int count,
                           ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(groups >= 1 && count >= 1 && in && k && outs, CKKS_EARG, "empty rotation sum");
    for (int i = 0; i < groups * count; ++i) {
      same_ctx(ctx, in[i]);
      need(in[i]->p.limbs == in[0]->p.limbs, CKKS_ELEVEL, "operands at different levels");
      need(in[i]->p.deg == in[0]->p.deg, CKKS_ESCALE, "operands with different noise degree");
      check_scales(in[0]->p.scale, in[i]->p.scale);
    }
    for (int g = 0; g < groups; ++g) need(outs[g] && outs[g]->owner == ctx, CKKS_EARG, "bad output handle");
    std::vector<DevPoly> tmp(groups);
    rotate_sum_groups(c, in, groups, k, count, tmp.data());
    for (int g = 0; g < groups; ++g) take(outs[g]->p, tmp[g]);
  });
}

int ckks_rotate_sum(ckks_ctx* ctx, const ckks_ct* const* in, const int* k, int count, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 1 && in && k, CKKS_EARG, "empty rotation sum");
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, in[i]);
      need(in[i]->p.limbs == in[0]->p.limbs, CKKS_ELEVEL, "operands at different levels");
      need(in[i]->p.deg == in[0]->p.deg, CKKS_ESCALE, "operands with different noise degree");
      check_scales(in[0]->p.scale, in[i]->p.scale);
    }
    DevPoly tmp;
    rotate_sum(c, in, k, count, tmp);
    take(out->p, tmp);
  });
}

int ckks_rescale_batch(ckks_ctx* ctx, const ckks_ct* const* in, int count, ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (in && outs)), CKKS_EARG, "bad batch");
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, in[i]);
      need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
    }
    rescale_many(c, in, count, outs);
  });
}

int ckks_rescale(ckks_ctx* ctx, const ckks_ct* a, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    need(a->p.limbs >= 2, CKKS_ELEVEL, "no limb left to rescale");
    const ckks_ct* as[1] = {a};
    ckks_ct* os[1] = {out};
    rescale_many(c, as, 1, os);
  });
}

int ckks_drop_limbs(ckks_ctx* ctx, const ckks_ct* a, int limbs, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    need(limbs >= 1 && limbs <= a->p.limbs, CKKS_ELEVEL, "cannot add limbs");
    DevPoly tmp;
    tmp.ensure(&c, 2, limbs);
    ckks::ew_binary(c, ckks::EwOp::Copy, a->p.data, stride(a->p), nullptr, 0, tmp.data, stride(tmp), 2, limbs,
                    c.stream);
    tmp.limbs = limbs;
    tmp.scale = a->p.scale;
    tmp.deg = a->p.deg;
    take(out->p, tmp);
  });
}

int ckks_rotate(ckks_ctx* ctx, const ckks_ct* a, int k, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    ckks_ct* outs[1] = {out};
    rotate_many(c, a, &k, 1, outs);
  });
}

int ckks_rotate_hoisted(ckks_ctx* ctx, const ckks_ct* a, const int* k, int count, ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    need(count >= 0 && (count == 0 || (k && outs)), CKKS_EARG, "bad index list");
    for (int i = 0; i < count; ++i) need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
    rotate_many(c, a, k, count, outs);
  });
}

int ckks_rotate_sum_hoisted(ckks_ctx* ctx, const ckks_ct* const* in, int count, const int* k, int nk,
                            ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (in && outs)), CKKS_EARG, "bad batch");
    need(nk >= 1 && k, CKKS_EARG, "empty rotation list");
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, in[i]);
      need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
    }
    std::vector<DevPoly> res;
    hoisted_sum_batch(c, in, count, k, nk, res);
    for (int i = 0; i < count; ++i) take(outs[i]->p, res[i]);
  });
}

int ckks_window_sum_batch(ckks_ctx* ctx, const ckks_ct* const* in, int count, int window, int stride_,
                          ckks_ct* const* outs) {
  return ckks_window_sum_batch_radix(ctx, in, count, window, stride_, 4, outs);
}

int ckks_window_sum_batch_radix(ckks_ctx* ctx, const ckks_ct* const* in, int count, int window, int stride_,
                                int radix, ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && (count == 0 || (in && outs)), CKKS_EARG, "bad batch");
    need(window >= 1, CKKS_EARG, "window must be positive");
    need(radix >= 2 && radix <= ckks::kKsBatch + 1, CKKS_EARG, "radix must be 2..33");
    for (int i = 0; i < count; ++i) {
      same_ctx(ctx, in[i]);
      need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
    }
    if (!count) return;
    // base-r ladder: step s adds the rotations by stride * s * {1 .. r-1}
    // (those below the window) to the running sums, hoisted per ciphertext
    std::vector<ckks_ct> acc(count);
    std::vector<const ckks_ct*> cur(in, in + count);
    for (long step = 1; step < window; step *= radix) {
      std::vector<int> ks{0};
      for (int m = 1; m < radix && step * m < window; ++m) ks.push_back((int)(stride_ * step * m));
      const int nk = (int)ks.size();
      std::vector<DevPoly> res;
      hoisted_sum_batch(c, cur.data(), count, ks.data(), nk, res);
      for (int i = 0; i < count; ++i) {
        acc[i].owner = ctx;
        take(acc[i].p, res[i]);
        cur[i] = &acc[i];
      }
    }
    for (int i = 0; i < count; ++i) {
      if (cur[i] == in[i]) {  // window 1: a copy
        DevPoly cp;
        cp.ensure(&c, 2, in[i]->p.limbs);
        ckks::ew_binary(c, ckks::EwOp::Copy, in[i]->p.data, stride(in[i]->p), nullptr, 0, cp.data, stride(cp), 2,
                        in[i]->p.limbs, c.stream);
        cp.limbs = in[i]->p.limbs;
        cp.scale = in[i]->p.scale;
        cp.deg = in[i]->p.deg;
        take(outs[i]->p, cp);
      } else {
        take(outs[i]->p, acc[i].p);
      }
    }
  });
}

int ckks_rotate_hoisted_batch(ckks_ctx* ctx, const ckks_ct* const* in, int count, const int* k, int nk,
                              ckks_ct* const* outs) {
  return guard([&] {
    Context& c = C(ctx);
    need(count >= 0 && nk >= 0 && (count == 0 || nk == 0 || (in && k && outs)), CKKS_EARG, "bad batch");
    for (int i = 0; i < count; ++i) same_ctx(ctx, in[i]);
    for (long i = 0; i < (long)count * nk; ++i) need(outs[i] && outs[i]->owner == ctx, CKKS_EARG, "bad output handle");
    rotate_hoisted_batch(c, in, count, k, nk, outs);
  });
}

int ckks_accumulate_sum(ckks_ctx* ctx, const ckks_ct* a, int count, int stride_, ckks_ct* out) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, a);
    need(out && out->owner == ctx, CKKS_EARG, "bad output handle");
    need(count >= 1, CKKS_EARG, "count must be positive");
    const int limbs = a->p.limbs;
    ckks_ct acc;
    acc.owner = ctx;
    acc.p.ensure(&c, 2, limbs);
    ckks::ew_binary(c, ckks::EwOp::Copy, a->p.data, stride(a->p), nullptr, 0, acc.p.data, stride(acc.p), 2, limbs,
                    c.stream);
    acc.p.limbs = limbs;
    acc.p.scale = a->p.scale;
    acc.p.deg = a->p.deg;
    ckks_ct rots[3];
    ckks_ct* outs[3] = {&rots[0], &rots[1], &rots[2]};
    for (int i = 0; i < 3; ++i) rots[i].owner = ctx;
    for (long step = 1; step < count; step *= 4) {
      int ks[3], n = 0;
      for (int m = 1; m < 4 && step * m < count; ++m) ks[n++] = (int)(stride_ * step * m);
      rotate_many(c, &acc, ks, n, outs);
      for (int r = 0; r < n; ++r)
        ckks::ew_binary(c, ckks::EwOp::Add, acc.p.data, stride(acc.p), rots[r].p.data, stride(rots[r].p),
                        acc.p.data, stride(acc.p), 2, limbs, c.stream);
    }
    take(out->p, acc.p);
  });
}

int ckks_profile_enable(ckks_ctx* ctx, int on) {
  return guard([&] { C(ctx).prof.on = on != 0; });
}

int ckks_profile_only(ckks_ctx* ctx, const char* kernel) {
  return guard([&] { C(ctx).prof.only = kernel ? kernel : ""; });
}

int ckks_profile_reset(ckks_ctx* ctx) {
  return guard([&] { C(ctx).prof.reset(); });
}

int ckks_profile_sections(ckks_ctx* ctx, char* buf, size_t size) {
  std::string js;
  const int rc = guard([&] {
    ckks::Profiler& p = C(ctx).prof;
    p.report();
    js = "{";
    char tmp[256];
    bool fs = true;
    for (auto& sec : p.sections()) {
      js += (fs ? "\"" : ", \"") + sec.first + "\": {";
      fs = false;
      bool first = true;
      for (auto& kv : sec.second) {
        std::snprintf(tmp, sizeof tmp, "%s\"%s\": {\"launches\": %ld, \"ms\": %.6f}", first ? "" : ", ",
                      kv.first.c_str(), kv.second.launches, kv.second.ms);
        js += tmp;
        first = false;
      }
      js += "}";
    }
    js += "}";
  });
  if (rc != CKKS_OK) return -1;
  if (buf && size) {
    const size_t n = js.size() < size - 1 ? js.size() : size - 1;
    std::memcpy(buf, js.data(), n);
    buf[n] = 0;
  }
  return (int)js.size();
}

int ckks_profile_report(ckks_ctx* ctx, char* buf, size_t size) {
  std::string js;
  const int rc = guard([&] {
    auto t = C(ctx).prof.report();
    js = "{";
    bool first = true;
    char tmp[256];
    for (auto& kv : t) {
      std::snprintf(tmp, sizeof tmp, "%s\"%s\": {\"launches\": %ld, \"ms\": %.6f, \"bytes\": %.1f, \"by_size\": {",
                    first ? "" : ", ", kv.first.c_str(), kv.second.launches, kv.second.ms, kv.second.bytes);
      js += tmp;
      bool fh = true;
      for (auto& h : kv.second.by_size) {
        std::snprintf(tmp, sizeof tmp, "%s\"%d\": [%ld, %.6f]", fh ? "" : ", ", h.first, h.second.first, h.second.second);
        js += tmp;
        fh = false;
      }
      js += "}}";
      first = false;
    }
    js += "}";
  });
  if (rc != CKKS_OK) return -1;
  if (buf && size) {
    const size_t n = js.size() < size - 1 ? js.size() : size - 1;
    std::memcpy(buf, js.data(), n);
    buf[n] = 0;
  }
  return (int)js.size();
}

int ckks_ntt_forward_device(ckks_ctx* ctx, uint64_t* data, int nlimbs, int first_prime) {
  return guard([&] {
    Context& c = C(ctx);
    need(data && nlimbs >= 0 && first_prime >= 0 && first_prime + nlimbs <= c.P, CKKS_EARG, "bad limb range");
    ckks::LimbMap m{nlimbs, nlimbs, c.L, 0, first_prime};
    ckks::ntt_forward(c, data, nlimbs, m, c.stream);
    CKKS_CUDA(cudaGetLastError());
  });
}

int ckks_ntt_inverse_device(ckks_ctx* ctx, uint64_t* data, int nlimbs, int first_prime) {
  return guard([&] {
    Context& c = C(ctx);
    need(data && nlimbs >= 0 && first_prime >= 0 && first_prime + nlimbs <= c.P, CKKS_EARG, "bad limb range");
    ckks::LimbMap m{nlimbs, nlimbs, c.L, 0, first_prime};
    ckks::ntt_inverse(c, data, nlimbs, m, c.stream);
    CKKS_CUDA(cudaGetLastError());
  });
}

int ckks_ntt_forward_polys(ckks_ctx* ctx, uint64_t* data, int npolys, int limbs) {
  return guard([&] {
    Context& c = C(ctx);
    need(data && npolys >= 0 && limbs >= 1 && limbs <= c.L, CKKS_EARG, "bad polynomial shape");
    ckks::ntt_forward(c, data, npolys * limbs, ckks::LimbMap::q(limbs, c.L), c.stream);
    CKKS_CUDA(cudaGetLastError());
  });
}

int ckks_ntt_inverse_polys(ckks_ctx* ctx, uint64_t* data, int npolys, int limbs) {
  return guard([&] {
    Context& c = C(ctx);
    need(data && npolys >= 0 && limbs >= 1 && limbs <= c.L, CKKS_EARG, "bad polynomial shape");
    ckks::ntt_inverse(c, data, npolys * limbs, ckks::LimbMap::q(limbs, c.L), c.stream);
    CKKS_CUDA(cudaGetLastError());
  });
}

// ---- device-to-device limb transfer (NCCL exchanges between ranks) -------
int ckks_ct_export_device(ckks_ctx* ctx, const ckks_ct* ct, uint64_t* dev, size_t words) {
  return guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, ct);
    const size_t per = (size_t)ct->p.limbs * c.N;
    need(dev && words >= 2 * per, CKKS_EARG, "device buffer too small");
    for (int p = 0; p < 2; ++p)
      CKKS_CUDA(cudaMemcpyAsync(dev + p * per, ct->p.poly(p), sizeof(uint64_t) * per, cudaMemcpyDeviceToDevice,
                                c.stream));
  });
}

int ckks_ct_import_device(ckks_ctx* ctx, ckks_ct* ct, const uint64_t* dev, int limbs, double scale, int noise_deg) {
  return guard([&] {
    Context& c = C(ctx);
    need(ct && ct->owner == ctx && dev, CKKS_EARG, "bad argument");
    need(limbs >= 1 && limbs <= c.L, CKKS_EARG, "limb count outside 1..L");
    need(noise_deg == 1 || noise_deg == 2, CKKS_EARG, "noise degree must be 1 or 2");
    DevPoly tmp;
    tmp.ensure(&c, 2, limbs);
    const size_t per = (size_t)limbs * c.N;
    for (int p = 0; p < 2; ++p)
      CKKS_CUDA(cudaMemcpyAsync(tmp.poly(p), dev + p * per, sizeof(uint64_t) * per, cudaMemcpyDeviceToDevice,
                                c.stream));
    tmp.limbs = limbs;
    tmp.scale = scale;
    tmp.deg = noise_deg;
    take(ct->p, tmp);
  });
}

// ---- binary wire format ----------------------------------------------------
// Little-endian; header then the moduli of every limb, then the residues:
//   u32 magic 'CKB2', u32 version 1, u32 kind (1 ciphertext, 2 switching key),
//   u32 log2 N, u32 Q limbs, u32 special limbs, u32 polynomials, u32 noise
//   degree, f64 scale, i32 rotation index (keys; 0 = relinearisation key),
//   u32 digits (keys), then (Q limbs + special limbs) u64 moduli, then
//   polynomials x limbs x N u64 residues (a key: digits x 2 x (L + K) limbs).
// Readers check the magic, version, ring degree and every modulus against
// the context, so limbs never land under the wrong primes.
namespace {
constexpr uint32_t kWireMagic = 0x32424B43u;  // "CKB2"
struct WireHeader {
  uint32_t magic, version, kind, log_n, q_limbs, special, polys, deg;
  double scale;
  int32_t rot;
  uint32_t digits;
};
static_assert(sizeof(WireHeader) == 48, "wire header layout");

size_t wire_size(const WireHeader& h, int N) {
  const size_t P = h.q_limbs + h.special;
  const size_t words = h.kind == 1 ? (size_t)h.polys * h.q_limbs
                                   : (size_t)h.digits * 2 * P + (h.polys == 2 ? 2 * P : 0);
  return sizeof(WireHeader) + 8ull * P + 8ull * (size_t)N * words;
}

void check_header(const Context& c, const WireHeader& h, const uint8_t* buf, size_t size) {
  need(h.magic == kWireMagic && h.version == 1, CKKS_EARG, "not a ckks_b200 wire buffer");
  need((int)h.log_n == c.logN, CKKS_EARG, "ring degree differs from the context's");
  need(size >= wire_size(h, c.N), CKKS_EARG, "wire buffer truncated");
  const uint64_t* mod = (const uint64_t*)(buf + sizeof(WireHeader));
  for (uint32_t i = 0; i < h.q_limbs; ++i) need(mod[i] == c.moduli[i], CKKS_EARG, "Q modulus differs from the context's");
  for (uint32_t i = 0; i < h.special; ++i)
    need(mod[h.q_limbs + i] == c.moduli[c.L + i], CKKS_EARG, "special modulus differs from the context's");
}
}  // namespace

long long ckks_ct_serialize(ckks_ctx* ctx, const ckks_ct* ct, uint8_t* buf, size_t cap) {
  long long out = -1;
  const int rc = guard([&] {
    Context& c = C(ctx);
    same_ctx(ctx, ct);
    WireHeader h{kWireMagic, 1, 1, (uint32_t)c.logN, (uint32_t)ct->p.limbs, 0, 2, (uint32_t)ct->p.deg, ct->p.scale, 0, 0};
    const size_t n = wire_size(h, c.N);
    out = (long long)n;
    if (!buf) return;
    need(cap >= n, CKKS_EARG, "wire buffer too small");
    std::memcpy(buf, &h, sizeof h);
    std::memcpy(buf + sizeof h, c.moduli.data(), 8ull * h.q_limbs);
    uint64_t* data = (uint64_t*)(buf + sizeof h + 8ull * h.q_limbs);
    const size_t per = (size_t)ct->p.limbs * c.N;
    for (int p = 0; p < 2; ++p)
      CKKS_CUDA(cudaMemcpyAsync(data + p * per, ct->p.poly(p), 8 * per, cudaMemcpyDeviceToHost, c.stream));
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  });
  return rc == CKKS_OK ? out : -1;
}

int ckks_ct_deserialize(ckks_ctx* ctx, ckks_ct* ct, const uint8_t* buf, size_t size) {
  return guard([&] {
    Context& c = C(ctx);
    need(ct && ct->owner == ctx && buf && size >= sizeof(WireHeader), CKKS_EARG, "bad argument");
    WireHeader h;
    std::memcpy(&h, buf, sizeof h);
    need(h.kind == 1 && h.polys == 2 && h.special == 0, CKKS_EARG, "not a ciphertext");
    need(h.q_limbs >= 1 && (int)h.q_limbs <= c.L, CKKS_EARG, "limb count outside 1..L");
    need(h.deg == 1 || h.deg == 2, CKKS_EARG, "bad noise degree");
    check_header(c, h, buf, size);
    DevPoly tmp;
    tmp.ensure(&c, 2, (int)h.q_limbs);
    const uint64_t* data = (const uint64_t*)(buf + sizeof h + 8ull * h.q_limbs);
    const size_t per = (size_t)h.q_limbs * c.N;
    for (int p = 0; p < 2; ++p)
      CKKS_CUDA(cudaMemcpyAsync(tmp.poly(p), data + p * per, 8 * per, cudaMemcpyHostToDevice, c.stream));
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
    tmp.limbs = (int)h.q_limbs;
    tmp.scale = h.scale;
    tmp.deg = (int)h.deg;
    take(ct->p, tmp);
  });
}

long long ckks_key_serialize(ckks_ctx* ctx, int k, uint8_t* buf, size_t cap) {
  long long out = -1;
  const int rc = guard([&] {
    Context& c = C(ctx);
    const uint64_t* src = k == 0 ? c.d_rlk : c.rot_key(c.galois(k));
    need(src != nullptr, CKKS_EKEY, "key not generated");
    // the key over the reduced special-prime set, when the context has one,
    // follows the standard key (polys = 2, deg = its special-prime count)
    const uint64_t* low = nullptr;
    if (c.low_limbs) {
      low = k == 0 ? c.d_rlk_low : c.switch_key(c.galois(k), 1);
      need(low != nullptr, CKKS_EKEY, "reduced-set key not generated");
    }
    WireHeader h{kWireMagic, 1, 2, (uint32_t)c.logN, (uint32_t)c.L, (uint32_t)c.K, low ? 2u : 1u,
                 (uint32_t)(low ? c.K_low : 0), 1.0, k, (uint32_t)(c.key_words() / (2 * (size_t)c.P * c.N))};
    const size_t n = wire_size(h, c.N);
    out = (long long)n;
    if (!buf) return;
    need(cap >= n, CKKS_EARG, "wire buffer too small");
    std::memcpy(buf, &h, sizeof h);
    std::memcpy(buf + sizeof h, c.moduli.data(), 8ull * c.P);
    uint8_t* data = buf + sizeof h + 8ull * c.P;
    CKKS_CUDA(cudaMemcpyAsync(data, src, 8 * c.key_words(), cudaMemcpyDeviceToHost, c.stream));
    if (low)
      CKKS_CUDA(cudaMemcpyAsync(data + 8 * c.key_words(), low, 8 * c.low_key_words(), cudaMemcpyDeviceToHost,
                                c.stream));
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
  });
  return rc == CKKS_OK ? out : -1;
}

int ckks_key_deserialize(ckks_ctx* ctx, const uint8_t* buf, size_t size) {
  return guard([&] {
    Context& c = C(ctx);
    need(buf && size >= sizeof(WireHeader), CKKS_EARG, "bad argument");
    WireHeader h;
    std::memcpy(&h, buf, sizeof h);
    need(h.kind == 2, CKKS_EARG, "not a switching key");
    need((int)h.q_limbs == c.L && (int)h.special == c.K && (size_t)h.digits * 2 * c.P * c.N == c.key_words(),
         CKKS_EARG, "key shape differs from the context's");
    check_header(c, h, buf, size);
    need(h.polys == (c.low_limbs ? 2u : 1u) && h.deg == (uint32_t)(c.low_limbs ? c.K_low : 0), CKKS_EARG,
         "key's reduced special-prime set differs from the context's");
    const uint8_t* data = buf + sizeof h + 8ull * c.P;
    uint64_t* key = nullptr;
    CKKS_CUDA(cudaMalloc(&key, 8 * c.key_words()));
    CKKS_CUDA(cudaMemcpyAsync(key, data, 8 * c.key_words(), cudaMemcpyHostToDevice, c.stream));
    uint64_t* low = nullptr;
    if (h.polys == 2) {
      CKKS_CUDA(cudaMalloc(&low, 8 * c.low_key_words()));
      CKKS_CUDA(cudaMemcpyAsync(low, data + 8 * c.key_words(), 8 * c.low_key_words(), cudaMemcpyHostToDevice,
                                c.stream));
    }
    CKKS_CUDA(cudaStreamSynchronize(c.stream));
    c.install_key(h.rot, key);
    if (low) c.install_key(h.rot, low, true);
  });
}

}  // extern "C"
