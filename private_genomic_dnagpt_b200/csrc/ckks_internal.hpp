// ckks_internal.hpp -- engine-internal types shared by the CUDA translation
// units: the device-resident context (prime chain, NTT and conversion
// tables, keys), ciphertext/plaintext objects and the kernel launchers.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "modarith.cuh"

namespace ckks {

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// status codes returned through the C ABI
enum : int {
  kOk = 0,
  kErrArgument = 1,
  kErrState = 2,
  kErrCuda = 3,
  kErrKeyMissing = 4,
  kErrLevel = 5,
  kErrScale = 6,
  kErrCapacity = 7,
};

void cuda_check(cudaError_t e, const char* what);
#define CKKS_CUDA(x) ::ckks::cuda_check((x), #x)

// Programmatic dependent launch.  A kernel started by launch_pdl may begin
// while the previous kernel in its stream is still finishing, so it runs
// CKKS_PDL_ENTRY() before touching global memory: griddepcontrol.wait
// returns once the preceding grids have completed and their writes are
// visible; launch_dependents lets the next programmatic dependent start once
// every CTA of this grid has started (so its CTAs take the SMs that this
// grid's last wave frees).
#define CKKS_PDL_ENTRY()                                 \
  do {                                                   \
    asm volatile("griddepcontrol.wait;" ::: "memory");   \
    asm volatile("griddepcontrol.launch_dependents;");   \
  } while (0)

template <class... KArgs, class... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CKKS_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// Maps batch limb index -> global prime index.  A batch holds polynomials of
// `nper` limbs each; the first `lq` limbs of every polynomial are the Q primes
// 0..lq-1, the rest are the special primes L..L+nper-lq-1.  With
// skip_alpha > 0, polynomial p skips its limbs [p*skip_alpha, (p+1)*skip_alpha)
// that lie below lq (the ModUp digit's own limbs, already in NTT form).
struct LimbMap {
  int nper;
  int lq;
  int L;
  int skip_alpha;
  int q0 = 0;  // first Q prime of each polynomial (rescale transforms limb l-1 alone)
  int skip_q = 0;  // nonzero: skip every Q limb (transform only the special limbs)
  int skip_beta = 0;  // >0: polynomial p is digit p % skip_beta of its item (batched ModUp)
  __host__ __device__ int prime(int limb) const {
    const int t = limb % nper;
    return t < lq ? q0 + t : L + (t - lq);
  }
  __host__ __device__ bool skipped(int limb) const {
    if (skip_q && limb % nper < lq) return true;
    if (skip_alpha <= 0) return false;
    const int p = limb / nper, t = limb % nper;
    const int lo = (skip_beta > 0 ? p % skip_beta : p) * skip_alpha;
    const int hi = (lo + skip_alpha < lq) ? lo + skip_alpha : lq;
    return t >= lo && t < hi;
  }
  static LimbMap q(int lq, int L) { return {lq, lq, L, 0, 0, 0, 0}; }
  static LimbMap ext(int lq, int K, int L) { return {lq + K, lq, L, 0, 0, 0, 0}; }
  static LimbMap ponly(int K, int L) { return {K, 0, L, 0, 0, 0, 0}; }
  static LimbMap single(int prime) { return {1, 1, 0, 0, prime, 0, 0}; }
};

struct Params {
  int log_n = 16;
  int limbs = 24;  // L: Q primes at the top level
  int dnum = 3;
  int first_mod_bits = 60;
  int scale_mod_bits = 50;
  int special_mod_bits = 60;
  uint64_t seed = 1;
  int device = 0;
};

// constants of one level (number of Q limbs l) for ModUp / ModDown / Rescale
struct LevelTables {
  int limbs = 0;
  int beta = 0;
  // ModUp, per digit j and source i: (Qhat_{j,i})^-1 mod q_i as Shoup pair
  ulonglong2* d_up_hatinv = nullptr;  // [beta][alpha]
  // ModUp, per digit j, source i, extended target t: Qhat_{j,i} mod m_t
  uint64_t* d_up_hat = nullptr;  // [beta][alpha][l+K]
  // ModDown: Phat_k mod q_t
  uint64_t* d_down_phat = nullptr;  // [K][l]
  ulonglong2* d_down_pinv = nullptr;  // [l] P^-1 mod q_t
  // Rescale: q_{l-1}^-1 mod q_i, i < l-1
  ulonglong2* d_rescale_inv = nullptr;  // [l-1]
  // ModUp pre-scaling folded into the inverse NTT of d: limb i of digit j
  // leaves the transform multiplied by Qhat_{j,i}^-1
  ulonglong2* d_up_scale_a = nullptr;  // [l] Qhat^-1 * n^-1
  ulonglong2* d_up_scale_b = nullptr;  // [l] Qhat^-1 * Winv[1] * n^-1
};

// Per-context kernel timer: when enabled, every launch site records a CUDA
// event pair on the launching stream together with the launch's algorithmic
// bytes; report() folds them into per-kernel launch counts, device time and
// bytes.  Disabled, a scope costs one branch.
class Profiler {
 public:
  bool on = false;
  struct Totals {
    long launches = 0;
    double ms = 0.0;
    double bytes = 0.0;
    // launches and milliseconds by launch size: key e = floor(log2(bytes))
    std::map<int, std::pair<long, double>> by_size;
  };
  // launches are also totalled per section (a caller-named phase, e.g. a
  // stage of a block evaluation)
  std::string section;
  // when set, only launches of this kernel name are timed (two events per
  // launch cost host time; a filtered profile leaves the rest untouched)
  std::string only;
  bool wants(const char* name) const { return only.empty() || only == name; }
  size_t begin(const char* name, double bytes, cudaStream_t st);
  void end(size_t idx, cudaStream_t st);
  std::map<std::string, Totals> report();  // synchronises pending events
  // per section and kernel name; call after report()
  const std::map<std::string, std::map<std::string, Totals>>& sections() const { return by_section_; }
  void reset();
  ~Profiler();

 private:
  struct Rec {
    const char* name;
    double bytes;
    cudaEvent_t a, b;
    std::string section;
  };
  std::vector<Rec> pending_;
  std::vector<cudaEvent_t> pool_;
  std::map<std::string, Totals> totals_;
  std::map<std::string, std::map<std::string, Totals>> by_section_;
  cudaEvent_t get();
};

class Context;
struct ProfScope {
  Profiler& p;
  cudaStream_t st;
  bool on;
  size_t idx = 0;
  ProfScope(const Context& c, const char* name, double bytes, cudaStream_t s);
  ~ProfScope();
};

class Context {
 public:
  explicit Context(const Params& p);
  ~Context();
  Context(const Context&) = delete;
  Context& operator=(const Context&) = delete;

  Params params;
  int logN, N, L, K, alpha, beta_top, P;
  int sms = 148;  // multiprocessors of the context's device
  std::vector<uint64_t> moduli;  // L + K
  std::vector<uint64_t> psi;
  std::vector<double> scales;  // [limbs], 1..L
  cudaStream_t stream = nullptr;

  // device tables
  Mod* d_mods = nullptr;            // [P]
  unsigned int* d_faults = nullptr;  // bounded device waits that gave up (bulk copies)
  ulonglong2* d_tw = nullptr;       // [P][N] forward (w, w')
  ulonglong2* d_itw = nullptr;      // [P][N] inverse (w, w')
  double2* d_twd = nullptr;         // [P][N] forward (w, fl(w/q)) as doubles (primes below 2^50.3)
  double2* d_itwd = nullptr;        // [P][N] inverse, the same
  ulonglong2* d_ninv = nullptr;     // [P]
  ulonglong2* d_w1ninv = nullptr;   // [P]
  ulonglong2* d_pmod = nullptr;     // [P] P mod q_t (Shoup pair), 0 for special primes
  double2* d_ksi = nullptr;         // [2N+1]
  uint32_t* d_rot_group = nullptr;  // [N/2]
  ulonglong2* d_phatinv = nullptr;  // [K] (P/p_k)^-1 mod p_k
  ulonglong2* d_down_scale_a = nullptr;  // [K] Phat_k^-1 * n^-1 (ModDown pre-scaling)
  ulonglong2* d_down_scale_b = nullptr;  // [K] Phat_k^-1 * Winv[1] * n^-1
  std::vector<LevelTables> levels;  // index = limbs (1..L)

  // keys (device, NTT form)
  uint64_t* d_sk = nullptr;   // [P][N]
  uint64_t* d_pk = nullptr;   // [2][L][N]
  uint64_t* d_rlk = nullptr;  // [beta_top][2][P][N]
  std::map<uint32_t, uint64_t*> rot_keys;  // galois element -> key
  uint64_t enc_counter = 0;

  // Key switches at <= low_limbs limbs (one digit) use switching keys over
  // the first K_low special primes only, P' = p_0 ... p_{K_low-1}, with
  // log2 P' >= log2 Q_{low_limbs} + 20 so that the ModDown error stays below
  // 2^-20 of the digit bound.  Disabled (0) when that needs all K primes or
  // the digit is shorter than low_limbs.
  int low_limbs = 0, K_low = 0;
  ulonglong2* d_pmod_low = nullptr;          // [P] P' mod q_t, 0 for special primes
  ulonglong2* d_down_scale_low_a = nullptr;  // [K] (first K_low) P'hat_k^-1 * n^-1
  ulonglong2* d_down_scale_low_b = nullptr;  // [K] P'hat_k^-1 * Winv[1] * n^-1
  std::vector<LevelTables> levels_low;       // index = limbs (1..low_limbs)
  uint64_t* d_rlk_low = nullptr;             // [1][2][P][N], primes < low_limbs and the first K_low special
  std::map<uint32_t, uint64_t*> rot_keys_low;

  // the special-prime set of a key switch at `limbs` limbs
  bool low(int limbs) const { return low_limbs > 0 && limbs <= low_limbs; }
  int Kx(int limbs) const { return low(limbs) ? K_low : K; }
  const LevelTables& lt(int limbs) const { return low(limbs) ? levels_low[limbs] : levels[limbs]; }
  const ulonglong2* down_scale_a(int limbs) const { return low(limbs) ? d_down_scale_low_a : d_down_scale_a; }
  const ulonglong2* down_scale_b(int limbs) const { return low(limbs) ? d_down_scale_low_b : d_down_scale_b; }
  // switching key for a key switch at `limbs` limbs: rotation (g != 1) or,
  // with g == 1, relinearisation; null when not generated
  const uint64_t* switch_key(uint32_t g, int limbs) const;

  size_t key_words() const { return (size_t)beta_top * 2 * P * N; }
  size_t low_key_words() const { return (size_t)2 * P * N; }
  uint32_t galois(int k) const;
  const uint64_t* rot_key(uint32_t g) const;
  // takes ownership of a cudaMalloc'd switching key: relinearisation for
  // k == 0, else rotation by k (replaces a key already present); `low`
  // selects the reduced special-prime set
  void install_key(int k, uint64_t* key, bool low = false);

  void* alloc(size_t bytes) const;
  void release(void* p) const;
  // host -> device copy of a small host array on stream `st` through a
  // pinned staging ring, so that it does not synchronise the stream (a copy
  // from pageable memory would); the ring waits for the stream only when it
  // wraps.  Larger arrays are copied directly.
  void stage_upload(void* dst, const void* src, size_t bytes, cudaStream_t st) const;

  mutable Profiler prof;
  double limb_bytes() const { return 8.0 * N; }
  // host time spent in allocation calls (diagnostics)
  mutable double alloc_seconds = 0.0;
  mutable long alloc_calls = 0;

 private:
  // Size-bucketed cache of device blocks.  All work of a context runs on its
  // one stream, so a block released here may be handed to the next
  // allocation at once: kernels that use it later are ordered after every
  // kernel that used it before.  Misses fall back to cudaMalloc.
  mutable std::mutex mem_mu_;
  mutable std::unordered_map<size_t, std::vector<void*>> free_;
  mutable std::unordered_map<void*, size_t> size_of_;
  void drop_cache() const;
  static constexpr size_t kStageBytes = 8u << 20;
  mutable char* stage_ = nullptr;  // pinned host ring
  mutable size_t stage_off_ = 0;
};

inline ProfScope::ProfScope(const Context& c, const char* name, double bytes, cudaStream_t s)
    : p(c.prof), st(s), on(c.prof.on && c.prof.wants(name)) {
  if (on) idx = p.begin(name, bytes, s);
}
inline ProfScope::~ProfScope() {
  if (on) p.end(idx, st);
}

// A ciphertext or plaintext living in device memory.  c0 occupies limbs
// [0, cap) and c1 limbs [cap, 2 cap) of `data`; the first `limbs` of each are
// live (rescale shrinks `limbs` without moving data).
struct DevPoly {
  Context* ctx = nullptr;
  uint64_t* data = nullptr;
  int npolys = 0;
  int cap = 0;
  int limbs = 0;
  double scale = 1.0;
  int deg = 1;  // noise-scale degree (1 fresh, 2 after a product)
  ~DevPoly();
  void ensure(Context* c, int np, int limbs_needed);
  uint64_t* poly(int i) const { return data + (size_t)i * cap * ctx->N; }
};

// ---- kernel launchers ----------------------------------------------------
// Where a transform reads its input when that is not `data` itself (the
// result is still written to `data`): batch limb i reads item[i / per_item]
// + (i % per_item) * limb_stride words; with `reduce` each value is first
// reduced modulo the limb's prime (a residue of another prime spread over a
// set of primes).  Up to 64 items.
struct NttSource {
  const uint64_t* item[64];
  int per_item;
  int limb_stride;
  bool reduce;
};
void ntt_forward(const Context& c, uint64_t* data, int nlimbs, LimbMap map, cudaStream_t st,
                 const NttSource* src = nullptr);
// inverse transform; with scale_a/scale_b (indexed by prime - scale_base:
// c*n^-1 and c*Winv[1]*n^-1 as Shoup pairs) it returns the coefficients times c
void ntt_inverse(const Context& c, uint64_t* data, int nlimbs, LimbMap map, cudaStream_t st,
                 const ulonglong2* scale_a = nullptr, const ulonglong2* scale_b = nullptr, int scale_base = 0,
                 const NttSource* src = nullptr);

// element-wise over `limbs` Q limbs of `npolys` polynomials with strides
enum class EwOp : int { Add = 0, Sub = 1, Mul = 2, Neg = 3, Copy = 4 };
void ew_binary(const Context& c, EwOp op, const uint64_t* a, size_t sa, const uint64_t* b, size_t sb, uint64_t* o,
               size_t so, int npolys, int limbs, cudaStream_t st);
// o = a * pt (pt shared by both polys)
void ew_mul_pt(const Context& c, const uint64_t* a, size_t sa, const uint64_t* pt, uint64_t* o, size_t so,
               int npolys, int limbs, cudaStream_t st);
// o = a * k (per-limb constants given as host residues)
void ew_mul_const(const Context& c, const uint64_t* a, size_t sa, uint64_t* o, size_t so, int npolys, int limbs,
                  const std::vector<uint64_t>& k_res, cudaStream_t st);
void ew_add_const(const Context& c, uint64_t* a, int limbs, const std::vector<uint64_t>& k_res, cudaStream_t st);
// sums of up to 64 ciphertexts (both polynomials) and batches of up to 32 pairs
constexpr int kSumMax = 64;
struct SumPtrs {
  const uint64_t* in0[kSumMax];
  const uint64_t* in1[kSumMax];
  uint64_t* out0;
  uint64_t* out1;
};
struct PairPtrs {
  const uint64_t* a0[32];
  const uint64_t* a1[32];
  const uint64_t* b0[32];
  const uint64_t* b1[32];
  uint64_t* o0[32];
  uint64_t* o1[32];
};
void add_many(const Context& c, const SumPtrs& p, int k, int limbs, cudaStream_t st);
void add_pairs(const Context& c, const PairPtrs& p, int M, int limbs, cudaStream_t st);
void tensor(const Context& c, const uint64_t* a0, const uint64_t* a1, const uint64_t* b0, const uint64_t* b1,
            uint64_t* d0, uint64_t* d1, uint64_t* d2, int limbs, cudaStream_t st);
// items per batched launch sequence (key switches, rescales, products)
constexpr int kKsBatch = 32;
// sum_i a_i (x) b_i of n <= kTensorSum ciphertext pairs (degree-2 result)
constexpr int kTensorSum = 31;
// batched plaintext products: item m is (a0[m], a1[m]) * pt[m] -> (o0[m], o1[m])
struct MulPtBatch {
  const uint64_t* a0[kKsBatch];
  const uint64_t* a1[kKsBatch];
  const uint64_t* pt[kKsBatch];
  uint64_t* o0[kKsBatch];
  uint64_t* o1[kKsBatch];
  int M;
};
void ew_mul_pt_batch(const Context& c, const MulPtBatch& b, int limbs, cudaStream_t st);
// batched tensors: item m writes d0, d1, d2 at d[m], d[m] + S, d[m] + 2 S
struct TensorBatch {
  const uint64_t* a0[kKsBatch];
  const uint64_t* a1[kKsBatch];
  const uint64_t* b0[kKsBatch];
  const uint64_t* b1[kKsBatch];
  uint64_t* d[kKsBatch];
  size_t S;
  int M;
};
void tensor_batch(const Context& c, const TensorBatch& b, int limbs, cudaStream_t st);

struct TensorPtrs {
  const uint64_t* a0[kTensorSum];
  const uint64_t* a1[kTensorSum];
  const uint64_t* b0[kTensorSum];
  const uint64_t* b1[kTensorSum];
};
// accumulate: add onto the sums already in d0, d1, d2
void tensor_sum(const Context& c, const TensorPtrs& p, int n, bool accumulate, uint64_t* d0, uint64_t* d1,
                uint64_t* d2, int limbs, cudaStream_t st);

// key switching
void modup(const Context& c, const uint64_t* d_ntt, int limbs, uint64_t* ext, cudaStream_t st);
void ks_inner(const Context& c, const uint64_t* ext, int limbs, const uint64_t* key, uint32_t g, uint64_t* acc,
              cudaStream_t st);
// out_p = moddown(acc_p), plus add0 permuted by g (p = 0) and add1 (p = 1)
// when given; acc holds 2 polys of limbs+K limbs and is consumed
void moddown2(const Context& c, uint64_t* acc, int limbs, const uint64_t* add0, uint32_t g_add0,
              const uint64_t* add1, uint64_t* out0, uint64_t* out1, cudaStream_t st);
// Rotation keys of a hoisted sum (R non-identity Galois elements)
struct HoistKeys {
  const uint64_t* key[kKsBatch];
  uint32_t g[kKsBatch];
  int R;
};

// Batched key switching: up to kKsBatch independent switches at one limb
// count in one launch sequence (ModUp, inner product, ModDown each a single
// launch over the batch).  Item m switches d[m] with key[m]; the ModUp digits
// are permuted by g[m] on read (1 = none); out0[m] = ModDown(acc0) +
// add0[m][pi_g(n)], out1[m] = ModDown(acc1) + add1[m] (addends optional).
// With shared_input every item switches d[0] and one ModUp serves all
// (hoisted rotations).
struct KsBatch {
  const uint64_t* d[kKsBatch];
  const uint64_t* key[kKsBatch];
  const uint64_t* add0[kKsBatch];
  const uint64_t* add1[kKsBatch];
  uint64_t* out0[kKsBatch];
  uint64_t* out1[kKsBatch];
  uint32_t g[kKsBatch];
  uint8_t src[kKsBatch];  // keyswitch_hoisted_multi: the ModUp input of each item
  int M;
};

// ModDown's combine step fused into the forward transform of the converted
// limbs (batch limb (2 m + p) limbs + t = item m, part p, limb t): the last
// pass stores out_p[m][t] = (acc[m][p][t] - conv) P^-1, plus add0[m]
// permuted by the automorphism g[m] (part 0) or add1[m] (part 1), instead of
// the converted limb.
struct ModDownCombine {
  const uint64_t* acc;     // [item][2][E limbs][N]
  const ulonglong2* pinv;  // [limbs] P^-1 mod q_t as Shoup pairs
  const uint64_t* add0[kKsBatch];
  const uint64_t* add1[kKsBatch];
  uint64_t* out0[kKsBatch];
  uint64_t* out1[kKsBatch];
  uint32_t g[kKsBatch];
  int limbs, E;
};
void ntt_forward_moddown(const Context& c, uint64_t* conv, int items, const ModDownCombine& mc, cudaStream_t st);
void keyswitch_batch(const Context& c, int limbs, const KsBatch& b, bool shared_input, cudaStream_t st);
// Count of bounded device waits that gave up since the last call (each
// leaves its CTA's outputs unwritten), read after the stream drains and
// reset to zero.
unsigned int take_device_faults(const Context& c);
// One CTA stages 4 KiB of src through a bulk copy and writes it to dst;
// with `starve` its barrier expects twice the bytes copied, so its wait
// runs out and counts one fault (tests of the bounded wait).
void bulk_wait_probe(const Context& c, const uint64_t* src, uint64_t* dst, bool starve, cudaStream_t st);
// Hoisted rotations of G inputs (d = c1 pointers, c0 = their c0) by the same
// R rotations (h): one ModUp per input, then the key products and ModDowns of
// up to 32 (input, rotation) items per launch sequence, the items of one key
// adjacent in the grid so that its residues come from HBM once for all
// inputs.  out0/out1[g * R + r] = rotation r of input g.
void keyswitch_hoisted_multi(const Context& c, int limbs, const uint64_t* const* d, const uint64_t* const* c0,
                             int G, const HoistKeys& h, uint64_t* const* out0, uint64_t* const* out1,
                             cudaStream_t st);
// Sum of the M key switches of a batch with one ModDown: the key inner
// products are added in the extended basis Q_l P and divided by P once;
// out0 = ModDown(sum acc0) + sum_m auto_{g_m}(add0[m]), out1 = ModDown(sum
// acc1) + sum_m add1[m] (null addends skipped).  The giant steps of a BSGS
// product: sum_g rot(inner_g, k_g).
void keyswitch_sum(const Context& c, int limbs, const KsBatch& b, uint64_t* out0, uint64_t* out1, cudaStream_t st);
// keyswitch_sum of G <= 4 groups that rotate by the same keys (bs[g].key and
// .g equal across groups; bs[g].d/add0 the group's inputs): one ModUp per
// input, the key inner products of all groups in one launch (a key residue is
// loaded once for the groups), one batched ModDown.  out0_g = ModDown(sum
// acc0) + sum_m auto_{g_m}(add0[g][m]) + id0_g, out1_g = ModDown(sum acc1) +
// id1_g, the identity terms id0/id1 optional (null).  The caller fills s.id0,
// s.id1, s.out0, s.out1; add0, g and M are taken from bs.
constexpr int kSumGroups = 4;
struct SumGroups {
  const uint64_t* add0[kSumGroups][kKsBatch];
  const uint64_t* id0[kSumGroups];
  const uint64_t* id1[kSumGroups];
  uint64_t* out0[kSumGroups];
  uint64_t* out1[kSumGroups];
  uint32_t g[kKsBatch];
  int M;
};
void keyswitch_sum_groups(const Context& c, int limbs, const KsBatch* bs, SumGroups& s, int G, cudaStream_t st);
// For each of the M items (d = c1, add0 = c0, out0/out1): the sum of its R
// rotations by h (plus the item itself when `identity`), with one ModUp per
// item, the R key inner products added in the extended basis Q_l P and one
// ModDown per item -- a rotation sum of one ciphertext, evaluated once for
// a batch of ciphertexts.
void keyswitch_hoisted_sum(const Context& c, int limbs, const KsBatch& b, const HoistKeys& h, bool identity,
                           cudaStream_t st);

// Batched rescale of M ciphertexts (c0, c1 pointers per item, `limbs` limbs
// each) into outputs of limbs-1 limbs.
struct RsBatch {
  const uint64_t* in0[kKsBatch];
  const uint64_t* in1[kKsBatch];
  uint64_t* out0[kKsBatch];
  uint64_t* out1[kKsBatch];
  int M;
};
void rescale_batch(const Context& c, int limbs, const RsBatch& b, cudaStream_t st);

// the same with caller-provided scratch: dc holds limbs*N words, conv 2*limbs*N
void modup_with(const Context& c, const uint64_t* d_ntt, int limbs, uint64_t* ext, uint64_t* dc, cudaStream_t st);
void moddown2_with(const Context& c, uint64_t* acc, int limbs, const uint64_t* add0, uint32_t g_add0,
                   const uint64_t* add1, uint64_t* out0, uint64_t* out1, uint64_t* conv, cudaStream_t st);
void automorphism(const Context& c, const uint64_t* a, uint64_t* o, int nlimbs, uint32_t g, cudaStream_t st);
// rescale npolys polynomials (stride in words) of `limbs` limbs to limbs-1
void rescale(const Context& c, const uint64_t* x, size_t sx, int npolys, int limbs, uint64_t* out, size_t so,
             cudaStream_t st);

// keys / sampling / client
void keygen_secret_public(Context& c);
uint64_t* make_switch_key(Context& c, const uint64_t* s_from, uint32_t key_id);
// the same key over the reduced special-prime set (one digit covering the
// first low_limbs Q primes)
uint64_t* make_switch_key_low(Context& c, const uint64_t* s_from, uint32_t key_id);
void encrypt(Context& c, const uint64_t* pt, int limbs, uint64_t counter, uint64_t* c0, uint64_t* c1);
void decrypt(const Context& c, const uint64_t* c0, const uint64_t* c1, int limbs, uint64_t* pt);

// canonical embedding
void encode(const Context& c, const double* d_values, int limbs, double scale, uint64_t* out, cudaStream_t st);
// client role, batched on the device: M ciphertexts (c0/c1 pointers, one limb
// count) -> M x N/2 decoded doubles; M plaintexts [M][limbs][N] -> M fresh
// encryptions with counters enc_counter .. enc_counter + M - 1
void decrypt_decode_batch(const Context& c, const uint64_t* const* c0, const uint64_t* const* c1, int limbs, int M,
                          const double* scales_host, double* out, cudaStream_t st);
void encrypt_batch(Context& c, const uint64_t* pts, int limbs, int M, uint64_t* const* c0, uint64_t* const* c1,
                   cudaStream_t st);
// the same for plaintexts still in coefficient form ([M][limbs][N], consumed):
// e0 is added to them before their forward transform (NTT(m + e0) = NTT(m) +
// NTT(e0) exactly), so an encryption transforms three polynomials, not four;
// the ciphertexts equal encrypt_batch's on the transformed plaintexts
void encrypt_batch_coef(Context& c, uint64_t* pts_coef, int limbs, int M, uint64_t* const* c0, uint64_t* const* c1,
                        cudaStream_t st);
void decode_contiguous_batch(const Context& c, uint64_t* pts, int use, int M, const double* scales, double* out,
                             cudaStream_t st);
// batch x (N/2) device values -> batch plaintexts of `limbs` limbs, out_stride words apart
void encode_batch(const Context& c, const double* d_values, int batch, int limbs, double scale, uint64_t* out,
                  size_t out_stride, cudaStream_t st, bool ntt = true);
void decode(const Context& c, const uint64_t* pt, int limbs, double scale, double* d_values, cudaStream_t st);

// integer / double residues on the host
uint64_t host_double_to_res(double r, uint64_t q);
uint64_t host_int_to_res(int64_t k, uint64_t q);

}  // namespace ckks
