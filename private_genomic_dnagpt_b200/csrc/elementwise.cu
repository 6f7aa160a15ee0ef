// elementwise.cu -- limb-wise ciphertext arithmetic in the NTT domain:
// EvalAdd / EvalSub / EvalMult(ct, pt) / constant products / the ct x ct
// tensor, and the NTT-domain automorphism.  All kernels move 16-byte
// vectors (two residues) per thread per operand; limb index comes from
// blockIdx.y so the modulus is uniform across a CTA.
#include "ckks_internal.hpp"

namespace ckks {

namespace {

constexpr int kEwThreads = 256;

struct ConstRes {
  uint64_t v[96];
};

__device__ __forceinline__ uint64_t apply(EwOp op, uint64_t a, uint64_t b, const Mod& m) {
  switch (op) {
    case EwOp::Add: return add_mod(a, b, m.q);
    case EwOp::Sub: return sub_mod(a, b, m.q);
    case EwOp::Mul: return mul_mod(a, b, m);
    case EwOp::Neg: return neg_mod(a, m.q);
    default: return a;
  }
}

template <EwOp OP>
__global__ void __launch_bounds__(kEwThreads) ew_binary_kernel(const uint64_t* __restrict__ a, size_t sa,
                                                               const uint64_t* __restrict__ b, size_t sb,
                                                               uint64_t* __restrict__ o, size_t so, int limbs,
                                                               int logN, const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int limb = blockIdx.y % limbs, p = blockIdx.y / limbs;
  const Mod m = mods[limb];
  const size_t i = ((size_t)blockIdx.x * kEwThreads + threadIdx.x) * 2;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(a + p * sa + off);
  ulonglong2 y = make_ulonglong2(0, 0);
  if (OP == EwOp::Add || OP == EwOp::Sub || OP == EwOp::Mul) y = *reinterpret_cast<const ulonglong2*>(b + p * sb + off);
  ulonglong2 r;
  r.x = apply(OP, x.x, y.x, m);
  r.y = apply(OP, x.y, y.y, m);
  *reinterpret_cast<ulonglong2*>(o + p * so + off) = r;
}

__global__ void __launch_bounds__(kEwThreads) mul_pt_kernel(const uint64_t* __restrict__ a, size_t sa,
                                                            const uint64_t* __restrict__ pt,
                                                            uint64_t* __restrict__ o, size_t so, int limbs,
                                                            int logN, const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int limb = blockIdx.y % limbs, p = blockIdx.y / limbs;
  const Mod m = mods[limb];
  const size_t i = ((size_t)blockIdx.x * kEwThreads + threadIdx.x) * 2;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(a + p * sa + off);
  const ulonglong2 y = *reinterpret_cast<const ulonglong2*>(pt + off);
  *reinterpret_cast<ulonglong2*>(o + p * so + off) = make_ulonglong2(mul_mod(x.x, y.x, m), mul_mod(x.y, y.y, m));
}

// item m = blockIdx.z: (c0, c1) of ciphertext m times plaintext m
__global__ void __launch_bounds__(kEwThreads) mul_pt_batch_kernel(MulPtBatch b, int limbs, int logN,
                                                                  const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int limb = blockIdx.y % limbs, p = blockIdx.y / limbs, mi = blockIdx.z;
  const Mod m = mods[limb];
  const size_t i = ((size_t)blockIdx.x * kEwThreads + threadIdx.x) * 2;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  const ulonglong2 x = *reinterpret_cast<const ulonglong2*>((p ? b.a1[mi] : b.a0[mi]) + off);
  const ulonglong2 y = *reinterpret_cast<const ulonglong2*>(b.pt[mi] + off);
  *reinterpret_cast<ulonglong2*>((p ? b.o1[mi] : b.o0[mi]) + off) =
      make_ulonglong2(mul_mod(x.x, y.x, m), mul_mod(x.y, y.y, m));
}

__global__ void __launch_bounds__(kEwThreads) mul_const_kernel(const uint64_t* __restrict__ a, size_t sa,
                                                               uint64_t* __restrict__ o, size_t so, int limbs,
                                                               int logN, const Mod* __restrict__ mods, ConstRes k) {
  const int N = 1 << logN;
  const int limb = blockIdx.y % limbs, p = blockIdx.y / limbs;
  const Mod m = mods[limb];
  const size_t i = ((size_t)blockIdx.x * kEwThreads + threadIdx.x) * 2;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  const uint64_t kv = k.v[limb];
  const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(a + p * sa + off);
  *reinterpret_cast<ulonglong2*>(o + p * so + off) = make_ulonglong2(mul_mod(x.x, kv, m), mul_mod(x.y, kv, m));
}

__global__ void __launch_bounds__(kEwThreads) add_const_kernel(uint64_t* __restrict__ a, int logN,
                                                               const Mod* __restrict__ mods, ConstRes k) {
  const int N = 1 << logN;
  const int limb = blockIdx.y;
  const uint64_t q = mods[limb].q;
  const size_t i = ((size_t)blockIdx.x * kEwThreads + threadIdx.x) * 2;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  const uint64_t kv = k.v[limb];
  ulonglong2 x = *reinterpret_cast<ulonglong2*>(a + off);
  x.x = add_mod(x.x, kv, q);
  x.y = add_mod(x.y, kv, q);
  *reinterpret_cast<ulonglong2*>(a + off) = x;
}

__global__ void __launch_bounds__(kEwThreads) tensor_kernel(const uint64_t* __restrict__ a0,
                                                            const uint64_t* __restrict__ a1,
                                                            const uint64_t* __restrict__ b0,
                                                            const uint64_t* __restrict__ b1, uint64_t* __restrict__ d0,
                                                            uint64_t* __restrict__ d1, uint64_t* __restrict__ d2,
                                                            int logN, const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int limb = blockIdx.y;
  const Mod m = mods[limb];
  const size_t i = (size_t)blockIdx.x * kEwThreads + threadIdx.x;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  const uint64_t x0 = a0[off], x1 = a1[off], y0 = b0[off], y1 = b1[off];
  U128 mid = mul_wide(x0, y1);
  mac_wide(mid, x1, y0);
  d0[off] = mul_mod(x0, y0, m);
  d1[off] = reduce128(mid, m);
  d2[off] = mul_mod(x1, y1, m);
}

// tensors of up to kKsBatch pairs, item m = blockIdx.z: d_m = (a0 b0, a0 b1 + a1 b0, a1 b1)
__global__ void __launch_bounds__(kEwThreads) tensor_batch_kernel(TensorBatch b, int logN,
                                                                  const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int limb = blockIdx.y, mi = blockIdx.z;
  const Mod m = mods[limb];
  const size_t i = (size_t)blockIdx.x * kEwThreads + threadIdx.x;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  const uint64_t x0 = b.a0[mi][off], x1 = b.a1[mi][off], y0 = b.b0[mi][off], y1 = b.b1[mi][off];
  U128 mid = mul_wide(x0, y1);
  mac_wide(mid, x1, y0);
  uint64_t* d = b.d[mi];
  d[off] = mul_mod(x0, y0, m);
  d[b.S + off] = reduce128(mid, m);
  d[2 * b.S + off] = mul_mod(x1, y1, m);
}

// sum_i a_i (x) b_i over up to kTensorSum pairs: d0 = sum a0 b0, d1 = sum
// (a0 b1 + a1 b0), d2 = sum a1 b1, 128-bit accumulation (at most 62 products
// of residues below 2^61 per accumulator)
__global__ void __launch_bounds__(kEwThreads) tensor_sum_kernel(TensorPtrs p, int n, bool accumulate,
                                                                uint64_t* __restrict__ d0, uint64_t* __restrict__ d1,
                                                                uint64_t* __restrict__ d2, int logN,
                                                                const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int limb = blockIdx.y;
  const Mod m = mods[limb];
  const size_t i = (size_t)blockIdx.x * kEwThreads + threadIdx.x;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  // accumulate: continue the sums already in d0, d1, d2 (residues)
  U128 s0{accumulate ? d0[off] : 0, 0}, s1{accumulate ? d1[off] : 0, 0}, s2{accumulate ? d2[off] : 0, 0};
  for (int k = 0; k < n; ++k) {
    const uint64_t x0 = p.a0[k][off], x1 = p.a1[k][off], y0 = p.b0[k][off], y1 = p.b1[k][off];
    mac_wide(s0, x0, y0);
    mac_wide(s1, x0, y1);
    mac_wide(s1, x1, y0);
    mac_wide(s2, x1, y1);
  }
  d0[off] = reduce128(s0, m);
  d1[off] = reduce128(s1, m);
  d2[off] = reduce128(s2, m);
}

// out[k] = in[auto_index(k)]: each warp reads one aligned 32-residue span
__global__ void __launch_bounds__(kEwThreads) automorphism_kernel(const uint64_t* __restrict__ a,
                                                                  uint64_t* __restrict__ o, uint32_t g, int logN) {
  const int N = 1 << logN;
  const size_t k = (size_t)blockIdx.x * kEwThreads + threadIdx.x;
  if (k >= (size_t)N) return;
  const size_t base = (size_t)blockIdx.y * N;
  o[base + k] = a[base + auto_index((uint32_t)k, g, logN)];
}

// out = sum of k inputs (EvalAddMany), per limb of both polynomials
__global__ void __launch_bounds__(kEwThreads) add_many_kernel(SumPtrs p, int k, int limbs, int logN,
                                                              const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int limb = blockIdx.y % limbs, poly = blockIdx.y / limbs;
  const uint64_t q = mods[limb].q;
  const size_t i = ((size_t)blockIdx.x * kEwThreads + threadIdx.x) * 2;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  ulonglong2 acc = make_ulonglong2(0, 0);
  for (int j = 0; j < k; ++j) {
    const ulonglong2 x = *reinterpret_cast<const ulonglong2*>((poly ? p.in1[j] : p.in0[j]) + off);
    acc.x = add_mod(acc.x, x.x, q);
    acc.y = add_mod(acc.y, x.y, q);
  }
  *reinterpret_cast<ulonglong2*>((poly ? p.out1 : p.out0) + off) = acc;
}

// out_m = a_m + b_m for a batch of independent pairs
__global__ void __launch_bounds__(kEwThreads) add_pairs_kernel(PairPtrs p, int limbs, int logN,
                                                               const Mod* __restrict__ mods) {
  const int N = 1 << logN;
  const int limb = blockIdx.y % limbs, poly = blockIdx.y / limbs, m = blockIdx.z;
  const uint64_t q = mods[limb].q;
  const size_t i = ((size_t)blockIdx.x * kEwThreads + threadIdx.x) * 2;
  if (i >= (size_t)N) return;
  const size_t off = (size_t)limb * N + i;
  const ulonglong2 x = *reinterpret_cast<const ulonglong2*>((poly ? p.a1[m] : p.a0[m]) + off);
  const ulonglong2 y = *reinterpret_cast<const ulonglong2*>((poly ? p.b1[m] : p.b0[m]) + off);
  *reinterpret_cast<ulonglong2*>((poly ? p.o1[m] : p.o0[m]) + off) =
      make_ulonglong2(add_mod(x.x, y.x, q), add_mod(x.y, y.y, q));
}

ConstRes pack(const std::vector<uint64_t>& v) {
  ConstRes c{};
  if (v.size() > 96) throw Error(kErrArgument, "too many limbs");
  for (size_t i = 0; i < v.size(); ++i) c.v[i] = v[i];
  return c;
}

}  // namespace

void ew_binary(const Context& c, EwOp op, const uint64_t* a, size_t sa, const uint64_t* b, size_t sb, uint64_t* o,
               size_t so, int npolys, int limbs, cudaStream_t st) {
  const dim3 grid((c.N / 2 + kEwThreads - 1) / kEwThreads, npolys * limbs);
  const int reads = (op == EwOp::Add || op == EwOp::Sub || op == EwOp::Mul) ? 2 : 1;
  ProfScope ps(c, "ew_binary", (reads + 1.0) * npolys * limbs * c.limb_bytes(), st);
  switch (op) {
    case EwOp::Add:
      ew_binary_kernel<EwOp::Add><<<grid, kEwThreads, 0, st>>>(a, sa, b, sb, o, so, limbs, c.logN, c.d_mods);
      break;
    case EwOp::Sub:
      ew_binary_kernel<EwOp::Sub><<<grid, kEwThreads, 0, st>>>(a, sa, b, sb, o, so, limbs, c.logN, c.d_mods);
      break;
    case EwOp::Mul:
      ew_binary_kernel<EwOp::Mul><<<grid, kEwThreads, 0, st>>>(a, sa, b, sb, o, so, limbs, c.logN, c.d_mods);
      break;
    case EwOp::Neg:
      ew_binary_kernel<EwOp::Neg><<<grid, kEwThreads, 0, st>>>(a, sa, b, sb, o, so, limbs, c.logN, c.d_mods);
      break;
    case EwOp::Copy:
      ew_binary_kernel<EwOp::Copy><<<grid, kEwThreads, 0, st>>>(a, sa, b, sb, o, so, limbs, c.logN, c.d_mods);
      break;
  }
  CKKS_CUDA(cudaGetLastError());
}

void ew_mul_pt(const Context& c, const uint64_t* a, size_t sa, const uint64_t* pt, uint64_t* o, size_t so,
               int npolys, int limbs, cudaStream_t st) {
  const dim3 grid((c.N / 2 + kEwThreads - 1) / kEwThreads, npolys * limbs);
  ProfScope ps(c, "mul_pt", (2.0 * npolys + 1.0) * limbs * c.limb_bytes(), st);
  mul_pt_kernel<<<grid, kEwThreads, 0, st>>>(a, sa, pt, o, so, limbs, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

void ew_mul_pt_batch(const Context& c, const MulPtBatch& b, int limbs, cudaStream_t st) {
  if (b.M <= 0) return;
  if (b.M > kKsBatch) throw Error(kErrArgument, "plaintext-product batch above 32");
  const dim3 grid((c.N / 2 + kEwThreads - 1) / kEwThreads, 2 * limbs, b.M);
  ProfScope ps(c, "mul_pt", 5.0 * b.M * limbs * c.limb_bytes(), st);
  mul_pt_batch_kernel<<<grid, kEwThreads, 0, st>>>(b, limbs, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

void ew_mul_const(const Context& c, const uint64_t* a, size_t sa, uint64_t* o, size_t so, int npolys, int limbs,
                  const std::vector<uint64_t>& k_res, cudaStream_t st) {
  const dim3 grid((c.N / 2 + kEwThreads - 1) / kEwThreads, npolys * limbs);
  ProfScope ps(c, "mul_const", 2.0 * npolys * limbs * c.limb_bytes(), st);
  mul_const_kernel<<<grid, kEwThreads, 0, st>>>(a, sa, o, so, limbs, c.logN, c.d_mods, pack(k_res));
  CKKS_CUDA(cudaGetLastError());
}

void ew_add_const(const Context& c, uint64_t* a, int limbs, const std::vector<uint64_t>& k_res, cudaStream_t st) {
  const dim3 grid((c.N / 2 + kEwThreads - 1) / kEwThreads, limbs);
  ProfScope ps(c, "add_const", 2.0 * limbs * c.limb_bytes(), st);
  add_const_kernel<<<grid, kEwThreads, 0, st>>>(a, c.logN, c.d_mods, pack(k_res));
  CKKS_CUDA(cudaGetLastError());
}

void tensor(const Context& c, const uint64_t* a0, const uint64_t* a1, const uint64_t* b0, const uint64_t* b1,
            uint64_t* d0, uint64_t* d1, uint64_t* d2, int limbs, cudaStream_t st) {
  const dim3 grid((c.N + kEwThreads - 1) / kEwThreads, limbs);
  ProfScope ps(c, "tensor", 7.0 * limbs * c.limb_bytes(), st);
  tensor_kernel<<<grid, kEwThreads, 0, st>>>(a0, a1, b0, b1, d0, d1, d2, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

void tensor_batch(const Context& c, const TensorBatch& b, int limbs, cudaStream_t st) {
  if (b.M <= 0) return;
  if (b.M > kKsBatch) throw Error(kErrArgument, "tensor batch above 32");
  const dim3 grid((c.N + kEwThreads - 1) / kEwThreads, limbs, b.M);
  ProfScope ps(c, "tensor", 7.0 * b.M * limbs * c.limb_bytes(), st);
  tensor_batch_kernel<<<grid, kEwThreads, 0, st>>>(b, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

void tensor_sum(const Context& c, const TensorPtrs& p, int n, bool accumulate, uint64_t* d0, uint64_t* d1,
                uint64_t* d2, int limbs, cudaStream_t st) {
  if (n < 1 || n > kTensorSum) throw Error(kErrArgument, "tensor sum of 1..31 pairs");
  const dim3 grid((c.N + kEwThreads - 1) / kEwThreads, limbs);
  ProfScope ps(c, "tensor_sum", (4.0 * n + 3.0) * limbs * c.limb_bytes(), st);
  tensor_sum_kernel<<<grid, kEwThreads, 0, st>>>(p, n, accumulate, d0, d1, d2, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

void add_many(const Context& c, const SumPtrs& p, int k, int limbs, cudaStream_t st) {
  const dim3 grid((c.N / 2 + kEwThreads - 1) / kEwThreads, 2 * limbs);
  ProfScope ps(c, "add_many", (k + 1.0) * 2 * limbs * c.limb_bytes(), st);
  add_many_kernel<<<grid, kEwThreads, 0, st>>>(p, k, limbs, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

void add_pairs(const Context& c, const PairPtrs& p, int M, int limbs, cudaStream_t st) {
  const dim3 grid((c.N / 2 + kEwThreads - 1) / kEwThreads, 2 * limbs, M);
  ProfScope ps(c, "add_pairs", 6.0 * M * limbs * c.limb_bytes(), st);
  add_pairs_kernel<<<grid, kEwThreads, 0, st>>>(p, limbs, c.logN, c.d_mods);
  CKKS_CUDA(cudaGetLastError());
}

void automorphism(const Context& c, const uint64_t* a, uint64_t* o, int nlimbs, uint32_t g, cudaStream_t st) {
  const dim3 grid((c.N + kEwThreads - 1) / kEwThreads, nlimbs);
  ProfScope ps(c, "automorphism", 2.0 * nlimbs * c.limb_bytes(), st);
  automorphism_kernel<<<grid, kEwThreads, 0, st>>>(a, o, g, c.logN);
  CKKS_CUDA(cudaGetLastError());
}

}  // namespace ckks
