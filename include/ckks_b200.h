/*
 * ckks_b200.h -- C ABI of the B200 CKKS evaluation engine.
 *
 * This is the drop-in boundary for the server-side hot path of the encrypted
 * DNAGPT block driver.  The reference binds FIDESlib's OpenFHE-compatible C++
 * API (`#include <fideslib.hpp>`, `using namespace fideslib`) from
 *   fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_depth13_
 *   digits3_ring65536_cpudiagcache_t123.cpp            ("T123.cpp" below)
 * Every entry point names the reference call it replaces.  Plain pointers and
 * sizes only; no CUDA or torch types cross the boundary (device pointers are
 * passed as uint64_t* to device memory where stated).
 *
 * Conventions
 *  - Every function returns CKKS_OK (0) or a CKKS_E* status; the message of
 *    the last failure on the calling thread is ckks_last_error().  (The
 *    reference reports failures as C++ exceptions, mapped to exit code 2 in
 *    T123.cpp:1757-1761.)
 *  - Levels follow OpenFHE: level 0 is a fresh ciphertext with all Q limbs;
 *    each Rescale raises the level by one and drops one limb.
 *  - Operations are asynchronous on the context's CUDA stream; functions that
 *    return data to the host (export, decode) synchronise it.  A context is not
 *    thread-safe; use one context per host thread.
 *  - Output handles may alias inputs.
 *  - Multiplications do not rescale.  ckks_rescale is explicit; the FLEXIBLEAUTO
 *    behaviour of EvalMult (rescale-before-multiply, level alignment) is
 *    provided by the host-side evaluator above this ABI.
 */
#ifndef CKKS_B200_H
#define CKKS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CKKS_OK 0
#define CKKS_EARG 1      /* invalid argument / shape mismatch */
#define CKKS_ESTATE 2    /* missing prerequisite (e.g. no keys yet) */
#define CKKS_ECUDA 3     /* CUDA runtime error */
#define CKKS_EKEY 4      /* rotation / relinearisation key not generated */
#define CKKS_ELEVEL 5    /* no limb left to drop / level mismatch */
#define CKKS_ESCALE 6    /* operand scales differ */
#define CKKS_ECAPACITY 7 /* size above a fixed capacity */

typedef struct ckks_ctx ckks_ctx; /* CryptoContext<DCRTPoly> + keys */
typedef struct ckks_ct ckks_ct;   /* Ciphertext<DCRTPoly> (device resident) */
typedef struct ckks_pt ckks_pt;   /* Plaintext (device resident, NTT form) */

/* CCParams<CryptoContextCKKSRNS> (T123.cpp:1602-1614) */
typedef struct {
  int log_n;            /* SetRingDim(2^log_n), T123.cpp:1613 */
  int limbs;            /* Q limbs = SetMultiplicativeDepth(d) + 1, T123.cpp:1605 */
  int dnum;             /* SetNumLargeDigits, T123.cpp:1611 (HYBRID, :1610) */
  int first_mod_bits;   /* SetFirstModSize, T123.cpp:1607 */
  int scale_mod_bits;   /* SetScalingModSize, T123.cpp:1606 (FLEXIBLEAUTO, :1608) */
  int special_mod_bits; /* bit size of the HYBRID special primes */
  uint64_t seed;        /* seeds every sampler: keys and encryptions */
  int device;           /* SetDevices({gpu}), T123.cpp:1614 */
} ckks_params;

const char* ckks_last_error(void);

/* GenCryptoContext + Enable(PKE, KEYSWITCH, LEVELEDSHE, ADVANCEDSHE) (T123.cpp:1616-1620) */
int ckks_ctx_create(const ckks_params* params, ckks_ctx** out);
int ckks_ctx_destroy(ckks_ctx* ctx);
/* GetRingDimension (T123.cpp:1627); also Q limbs, special limbs K, digit size alpha */
int ckks_ctx_info(const ckks_ctx* ctx, int* ring_dim, int* limbs, int* special, int* alpha);
/* the prime chain: limbs Q primes then K special primes */
int ckks_ctx_moduli(const ckks_ctx* ctx, uint64_t* out, int count);
/* FLEXIBLEAUTO scaling factor of a fresh encoding at `level` */
double ckks_ctx_scale(const ckks_ctx* ctx, int level);
/* Synchronize() (T123.cpp:1626, 1662, 1671).  Also reports, as CKKS_ECUDA,
 * a bounded device wait that gave up since the last call (a bulk copy into
 * shared memory that did not complete within one second); the outputs of
 * the calls since then are not valid, and the context stays usable. */
int ckks_sync(ckks_ctx* ctx);
/* the cudaStream_t the context enqueues on (for event timing by callers) */
void* ckks_ctx_stream(ckks_ctx* ctx);

/* KeyGen + LoadContext(publicKey) (T123.cpp:1622, 1625) */
int ckks_keygen(ckks_ctx* ctx);
/* EvalMultKeyGen (T123.cpp:1623) */
int ckks_relin_keygen(ckks_ctx* ctx);
/* EvalRotateKeyGen(sk, indices) (T123.cpp:1624; index set :455-481) */
int ckks_rotkey_gen(ckks_ctx* ctx, const int* indices, int count);
/* Both generate, besides the key over all K special primes, a one-digit key
 * over the first K_low special primes when the parameters allow it
 * (log2(p_0 ... p_{K_low-1}) >= log2(q_0 q_1 q_2) + 19.5 with K_low < K and
 * alpha >= 3): key switches at <= 3 limbs then use it (fewer limbs to
 * extend, transform and divide).  ckks_ctx_low_set reports (3, K_low) or
 * (0, 0). */
int ckks_ctx_low_set(const ckks_ctx* ctx, int* low_limbs, int* low_special);
/* key material to host: which = 0 secret (P*N), 1 public (2*L*N),
 * 2 relinearisation key, 3 rotation key for index k (dnum*2*(L+K)*N words),
 * 4 / 5 the relinearisation / rotation key over the reduced special-prime
 * set (2*(L+K)*N words, rows of unused primes zero) */
int ckks_key_export(ckks_ctx* ctx, int which, int k, uint64_t* host, size_t words);

int ckks_ct_create(ckks_ctx* ctx, ckks_ct** out);
int ckks_ct_destroy(ckks_ct* ct);
int ckks_pt_create(ckks_ctx* ctx, ckks_pt** out);
int ckks_pt_destroy(ckks_pt* pt);
/* GetLevel (T123.cpp:787, 1367) and the scale / noise degree bookkeeping */
int ckks_ct_level(const ckks_ct* ct);
int ckks_ct_limbs(const ckks_ct* ct);
double ckks_ct_scale(const ckks_ct* ct);
int ckks_ct_noise_deg(const ckks_ct* ct);
int ckks_pt_limbs(const ckks_pt* pt);
double ckks_pt_scale(const ckks_pt* pt);
int ckks_ct_set_scale(ckks_ct* ct, double scale, int noise_deg);

/* limb import/export: host layout c0 limbs then c1 limbs, N words each.
 * (FIDESlib has no ciphertext serialization; docs/hybrid/tasks.md:2652-2706) */
int ckks_ct_export(ckks_ctx* ctx, const ckks_ct* ct, uint64_t* host, size_t words);
int ckks_ct_import(ckks_ctx* ctx, ckks_ct* ct, const uint64_t* host, int limbs, double scale, int noise_deg);
int ckks_pt_export(ckks_ctx* ctx, const ckks_pt* pt, uint64_t* host, size_t words);
int ckks_pt_import(ckks_ctx* ctx, ckks_pt* pt, const uint64_t* host, int limbs, double scale);
/* The same transfer between device buffers, enqueued on the context stream:
 * the exchange of ciphertexts between ranks (an NCCL all-gather of these
 * buffers on the same stream).  No counterpart in the reference, whose
 * shards exchange serialized files (shard_layout.py, docs/hybrid/tasks.md). */
int ckks_ct_export_device(ckks_ctx* ctx, const ckks_ct* ct, uint64_t* dev, size_t words);
int ckks_ct_import_device(ckks_ctx* ctx, ckks_ct* ct, const uint64_t* dev, int limbs, double scale, int noise_deg);

/* Binary wire format of ciphertexts and switching keys: a 48-byte header
 * (magic "CKB2", version 1, kind, log2 N, Q limbs, special limbs, polynomials,
 * noise degree, scale, rotation index, digits), the modulus of every limb,
 * then the residues.  Readers check magic, version, ring degree and every
 * modulus against their context.  Serialize returns the byte count (with
 * buf == NULL: the size needed) or -1; the reference's serialize_writer /
 * serialize_reader drivers use OpenFHE's own format instead. */
long long ckks_ct_serialize(ckks_ctx* ctx, const ckks_ct* ct, uint8_t* buf, size_t cap);
int ckks_ct_deserialize(ckks_ctx* ctx, ckks_ct* ct, const uint8_t* buf, size_t size);
/* k = 0: relinearisation key; else the rotation key of index k */
long long ckks_key_serialize(ckks_ctx* ctx, int k, uint8_t* buf, size_t cap);
int ckks_key_deserialize(ckks_ctx* ctx, const uint8_t* buf, size_t size);
int ckks_ct_copy(ckks_ctx* ctx, const ckks_ct* src, ckks_ct* dst);

/* MakeCKKSPackedPlaintext(values, 1, level, nullptr, N/2) (T123.cpp:955-960,
 * 1053-1055); count <= N/2 real slots, the rest zero */
int ckks_encode(ckks_ctx* ctx, const double* values, int count, int level, ckks_pt* out);
/* encoding at an explicit limb count and scale */
int ckks_encode_at(ckks_ctx* ctx, const double* values, int count, int limbs, double scale, ckks_pt* out);
/* GetRealPackedValue (T123.cpp:525-526); count <= N/2 */
int ckks_decode(ckks_ctx* ctx, const ckks_pt* pt, double* out, int count);
/* Encrypt(publicKey, pt) (T123.cpp:531, 1659) */
int ckks_encrypt(ckks_ctx* ctx, const ckks_pt* pt, ckks_ct* out);
/* Decrypt(secretKey, ct, &pt) (T123.cpp:523, 1680) */
int ckks_decrypt(ckks_ctx* ctx, const ckks_ct* ct, ckks_pt* out);
/* Batched client role: `count` Encrypts of plaintexts at one limb count in
 * one launch sequence (item i gets the counter the i-th of `count` successive
 * ckks_encrypt calls would get), and `count` Decrypt + GetRealPackedValue
 * into count x slots host doubles (the reference's client does these one
 * ciphertext at a time, T123.cpp:514-715) */
int ckks_encrypt_batch(ckks_ctx* ctx, const ckks_pt* const* pts, int count, ckks_ct* const* outs);
int ckks_decrypt_decode_batch(ckks_ctx* ctx, const ckks_ct* const* cts, int count, double* out, int slots);
/* the counter that selects the next encryption's randomness */
int ckks_set_encrypt_counter(ckks_ctx* ctx, uint64_t counter);
uint64_t ckks_get_encrypt_counter(const ckks_ctx* ctx);

/* EvalAdd / EvalSub (T123.cpp:820, 854, 872, 1171) */
int ckks_add(ckks_ctx* ctx, const ckks_ct* a, const ckks_ct* b, ckks_ct* out);
int ckks_sub(ckks_ctx* ctx, const ckks_ct* a, const ckks_ct* b, ckks_ct* out);
int ckks_add_pt(ckks_ctx* ctx, const ckks_ct* a, const ckks_pt* p, ckks_ct* out);
/* EvalAddMany: sum of `count` ciphertexts at one level and scale; and
 * `count` independent sums a[i] + b[i] in one launch sequence */
int ckks_add_many(ckks_ctx* ctx, const ckks_ct* const* in, int count, ckks_ct* out);
int ckks_add_batch(ckks_ctx* ctx, const ckks_ct* const* a, const ckks_ct* const* b, int count, ckks_ct* const* outs);
/* EvalAdd(ct, double) (T123.cpp:1173): adds round(value * scale) to every slot */
int ckks_add_scalar(ckks_ctx* ctx, const ckks_ct* a, double value, ckks_ct* out);
/* EvalMult(ct, pt) (T123.cpp:1149-1152), no rescale */
int ckks_mul_pt(ckks_ctx* ctx, const ckks_ct* a, const ckks_pt* p, ckks_ct* out);
/* EvalMult(ct, ct) = tensor + relinearisation (T123.cpp:1144-1147), no rescale */
int ckks_mul_ct(ckks_ctx* ctx, const ckks_ct* a, const ckks_ct* b, ckks_ct* out);
/* multiply by an integer constant (scale unchanged) */
int ckks_mul_int(ckks_ctx* ctx, const ckks_ct* a, int64_t k, ckks_ct* out);
/* Rescale (FLEXIBLEAUTO, implicit in T123.cpp:1608): divide by the last prime */
int ckks_rescale(ckks_ctx* ctx, const ckks_ct* a, ckks_ct* out);
/* drop limbs down to `limbs` without scaling (LevelReduce) */
int ckks_drop_limbs(ckks_ctx* ctx, const ckks_ct* a, int limbs, ckks_ct* out);
/* EvalRotate(ct, k), left rotation by k slots (T123.cpp:1286-1288, 1304-1309) */
int ckks_rotate(ckks_ctx* ctx, const ckks_ct* a, int k, ckks_ct* out);
/* EvalFastRotation(ct, k[], M, nullptr): one ModUp shared by `count`
 * rotations (T123.cpp:1183-1203, 1343-1362) */
int ckks_rotate_hoisted(ckks_ctx* ctx, const ckks_ct* a, const int* k, int count, ckks_ct* const* outs);
/* EvalFastRotation of `count` ciphertexts at one limb count by the same nk
 * indices: outs[i * nk + r] = rotation k[r] of in[i]; one ModUp per input and
 * each rotation key read from HBM once for all inputs (the baby steps of all
 * token groups of a BSGS product) */
int ckks_rotate_hoisted_batch(ckks_ctx* ctx, const ckks_ct* const* in, int count, const int* k, int nk,
                              ckks_ct* const* outs);
/* Batched forms: `count` independent operations at one limb count, run as
 * one launch sequence per stage (up to 32 per sequence).  They replace loops
 * of EvalRotate / EvalMult / Rescale calls over independent ciphertexts
 * (the reference issues them one at a time, T123.cpp:795-860). */
int ckks_rotate_batch(ckks_ctx* ctx, const ckks_ct* const* in, const int* k, int count, ckks_ct* const* outs);
/* out = sum_i EvalRotate(in[i], k[i]) (all inputs at one level and scale):
 * the giant-step sum of a BSGS product (T123.cpp:1283-1291).  The key
 * switches of up to 32 non-identity rotations are added in the extended
 * basis Q_l P and divided by P once (one ModDown per 32 rotations, in input
 * order, instead of one per rotation); identity rotations are added as is. */
int ckks_rotate_sum(ckks_ctx* ctx, const ckks_ct* const* in, const int* k, int count, ckks_ct* out);
/* outs[g] = sum_i EvalRotate(in[g * count + i], k[i]) for `groups` groups of
 * inputs (all at one level and scale): ckks_rotate_sum of every group, the
 * giant steps of one BSGS product for several token groups.  When k holds at
 * most one identity and at most 32 other indices, up to 4 groups share one
 * launch sequence: one ModUp per input, the key products of all groups in one
 * launch (each rotation key read once for them), one batched ModDown.  Equal
 * to ckks_rotate_sum per group, bit for bit. */
int ckks_rotate_sum_groups(ckks_ctx* ctx, const ckks_ct* const* in, int groups, const int* k, int count,
                           ckks_ct* const* outs);
/* out = sum_i EvalMult(a[i], b[i]) with one relinearisation: the tensor
 * products are summed as degree-2 ciphertexts and d2 is key-switched once
 * (the context accumulation of T123.cpp:838-860, where every weight tile x
 * shifted value product is only ever summed).  All products at one level,
 * scale and noise degree; the result is not rescaled. */
int ckks_mul_ct_sum(ckks_ctx* ctx, const ckks_ct* const* a, const ckks_ct* const* b, int count, ckks_ct* out);
int ckks_mul_ct_batch(ckks_ctx* ctx, const ckks_ct* const* a, const ckks_ct* const* b, int count,
                      ckks_ct* const* outs);
int ckks_rescale_batch(ckks_ctx* ctx, const ckks_ct* const* in, int count, ckks_ct* const* outs);
/* outs[i] = EvalMult(a[i], p[i]) (ciphertext x plaintext, T123.cpp:1149-1152) for ciphertexts at one
 * limb count, up to 32 products per launch */
int ckks_mul_pt_batch(ckks_ctx* ctx, const ckks_ct* const* a, const ckks_pt* const* p, int count,
                      ckks_ct* const* outs);
/* AccumulateSum(ct, count, stride) (T123.cpp:1154-1159; key ladder :444-453) */
int ckks_accumulate_sum(ckks_ctx* ctx, const ckks_ct* a, int count, int stride, ckks_ct* out);
/* outs[i] = sum_r EvalRotate(in[i], k[r]) for every input (k distinct; an
 * index 0 adds in[i] itself): the rotations of one input share its ModUp
 * (as EvalFastRotation) and their key switches are added in Q_l P and
 * divided by P once per input; up to 32 inputs per launch sequence, all at
 * one limb count.  Equal to ckks_rotate_sum over (in[i], k[r]) pairs. */
int ckks_rotate_sum_hoisted(ckks_ctx* ctx, const ckks_ct* const* in, int count, const int* k, int nk,
                            ckks_ct* const* outs);
/* outs[i] = sum_{j < window} EvalRotate(in[i], j * stride): the sums of the
 * AccumulateSum ladder (base 4, keys stride * 4^s * {1, 2, 3}) with every
 * step one hoisted rotation sum (one ModUp and one ModDown per step and
 * input, where AccumulateSum takes one ModDown per rotation) -- the same
 * slot values as AccumulateSum, different rounding noise. */
int ckks_window_sum_batch(ckks_ctx* ctx, const ckks_ct* const* in, int count, int window, int stride,
                          ckks_ct* const* outs);
/* the same with a base-r ladder (2 <= r <= 33; keys stride * r^s * {1 .. r-1}):
 * fewer ModUp/ModDown pairs (ceil(log_r window) per input) for more key products */
int ckks_window_sum_batch_radix(ckks_ctx* ctx, const ckks_ct* const* in, int count, int window, int stride,
                                int radix, ckks_ct* const* outs);

/* Kernel timer (the reference's per-call-site Profiler buckets,
 * fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_lintransform.cpp:627-629,
 * 797-824): when on, every kernel launch is bracketed by CUDA events on the
 * context stream.  The report is JSON text
 * {"<kernel>": {"launches": n, "ms": t, "bytes": algorithmic bytes,
 *               "by_size": {"<e>": [n_e, t_e], ...}}, ...}, where n_e and t_e
 * count the launches of 2^e to 2^(e+1) algorithmic bytes;
 * returns the length written (truncated to `size`) or -1. */
int ckks_profile_enable(ckks_ctx* ctx, int on);
int ckks_profile_reset(ckks_ctx* ctx);
/* time only the launches of one kernel name (NULL or "" = every kernel) */
int ckks_profile_only(ckks_ctx* ctx, const char* kernel);
int ckks_profile_report(ckks_ctx* ctx, char* buf, size_t size);
/* the same totals split by section (the block evaluation names its stages:
 * {"section": {"kernel": {"launches": n, "ms": t}}}), JSON text */
int ckks_profile_sections(ckks_ctx* ctx, char* buf, size_t size);

/* Limb-level kernels on caller-owned DEVICE buffers (uint64 residues,
 * limb-major, N words per limb), for parity checks and kernel benchmarks.
 * Limb i of `data` is taken modulo Q prime first_prime + i. */
int ckks_ntt_forward_device(ckks_ctx* ctx, uint64_t* data, int nlimbs, int first_prime);
int ckks_ntt_inverse_device(ckks_ctx* ctx, uint64_t* data, int nlimbs, int first_prime);
/* The same over `npolys` consecutive polynomials of `limbs` Q limbs each
 * (limb j of every polynomial modulo Q prime j), in one launch pair: the
 * batched shape the key switch uses. */
int ckks_ntt_forward_polys(ckks_ctx* ctx, uint64_t* data, int npolys, int limbs);
int ckks_ntt_inverse_polys(ckks_ctx* ctx, uint64_t* data, int npolys, int limbs);

/* ---- encrypted transformer block (the reference's EncryptedEvaluator and
 * Client, T123.cpp:509-948) ------------------------------------------------
 * Weights are float64 in PyTorch [out, in] layout, as the reference fixture
 * stores them (ln1/ln2 gains [D], attn_qkv [3D, D], attn_proj [D, D],
 * mlp_fc [MLP, D], mlp_proj [D, MLP]; bias-free, fhe/realweights/manual.py).
 * Tokens are packed 32 per ciphertext, lane-innermost. */
typedef struct ckks_block ckks_block;
int ckks_block_create(ckks_ctx* ctx, const double* ln1, const double* attn_qkv, const double* attn_proj,
                      const double* ln2, const double* mlp_fc, const double* mlp_proj, int d_model, int heads,
                      int mlp_dim, int tokens, ckks_block** out);
int ckks_block_destroy(ckks_block* b);
/* rotation indices the block needs (required_rotation_keys, T123.cpp:455-481);
 * returns the count, writes up to cap */
int ckks_block_rotation_indices(const ckks_block* b, int* out, int cap);
/* client encrypt -> server block evaluation with client refreshes -> client
 * decrypt; x and y are [tokens, d_model] float64 (T123.cpp:1642-1694) */
int ckks_block_forward(ckks_block* b, const double* x, int tokens, double* y);
/* operation counts and stage seconds of the last forward, JSON text */
int ckks_block_report(const ckks_block* b, char* buf, size_t size);
/* Stages of one block evaluation over unit subsets, for sharding one block
 * over several devices (one context per device, identical keys from the same
 * seed).  A forward is inputs -> qkv(groups) -> scores(tiles) -> softmax ->
 * context(tiles) -> output(groups); between stages the ranks exchange the
 * Q/K/V ciphertexts of their groups, the score matrix (disjoint entries:
 * a sum over ranks of zero-initialised buffers) and the partial contexts
 * (summed with EvalAdd).  Tiles are (query group, key group) pairs as 2n
 * ints.  d_scores: [tokens][heads][tokens] float64 on the device.  The units
 * follow the independent work of T123.cpp:780-790 (groups), :798-833 (tiles)
 * and shard_layout.py (exact EvalAdd merges of partial sums). */
int ckks_block_shard_inputs(ckks_block* b, const double* x, int tokens);
int ckks_block_shard_qkv(ckks_block* b, const int* groups, int n);
int ckks_block_shard_scores(ckks_block* b, const int* pairs, int n, double* d_scores);
int ckks_block_shard_softmax(ckks_block* b, const double* d_scores);
int ckks_block_shard_context(ckks_block* b, const int* pairs, int n);
/* the same two stages over explicit causal alignments (query group, key
 * group, lane shift d) as 3n ints: the finer units that balance many ranks
 * (each alignment is one score tile and one weight tile, T123.cpp:798-860) */
int ckks_block_shard_scores_tiles(ckks_block* b, const int* tiles, int n, double* d_scores);
int ckks_block_shard_context_tiles(ckks_block* b, const int* tiles, int n);
/* writes the rows of the given groups into y [tokens, d_model] (host) */
int ckks_block_shard_output(ckks_block* b, const int* groups, int n, double* y);
/* finer units for more ranks than token groups (shard_layout.py: Q/K/V
 * projections of a group on different devices, MLP partial sums merged by
 * EvalAdd).  qkv_parts: bit 0 Q, bit 1 K, bit 2 V.  shard_mlp: O projection,
 * residual (state 6), LN2 and the MLP chunks [chunk_begin, chunk_end) of the
 * groups, their sum kept as state 5 (the output stage = shard_mlp over all
 * chunks + shard_finish).  shard_finish: residual + MLP sum (states 6 and 5)
 * decrypted into the groups' rows of y.  mlp_chunks: the chunk count. */
int ckks_block_shard_qkv_parts(ckks_block* b, const int* groups, int n, int parts);
int ckks_block_shard_mlp(ckks_block* b, const int* groups, int n, int chunk_begin, int chunk_end);
int ckks_block_shard_finish(ckks_block* b, const int* groups, int n, double* y);
int ckks_block_mlp_chunks(const ckks_block* b);
/* state ciphertexts by kind (0 Q, 1 K, 2 V, 3 partial context, 4 encrypted
 * input, 5 MLP sum, 6 attention residual) and token group: get copies into
 * `out`; set copies from `in` (a handle without data clears the entry) */
int ckks_block_state_get(ckks_block* b, int kind, int group, ckks_ct* out);
int ckks_block_state_set(ckks_block* b, int kind, int group, const ckks_ct* in);

/* drop the block's encoded BSGS diagonals and masks (about 26 GB per block
 * at N = 2^16); the next forward encodes them again on the device */
int ckks_block_release_cache(ckks_block* b, size_t* released_bytes);

/* ---- classifier head and the multi-block model (the reference's
 * 12blocks_head_cpudiagcache_t123_v3.cpp:452-755, multiblock/manual.py:52-80)
 * A head object evaluates final LN -> head linear [D, D] -> SiLU (client)
 * -> head LN -> dot with readout (the N - A margin row) on one token; it is
 * a ckks_block handle released with ckks_block_destroy. */
int ckks_head_create(ckks_ctx* ctx, const double* final_ln, const double* head_linear, const double* head_ln,
                     const double* readout, int d_model, ckks_block** out);
/* encrypted margin of one hidden state x_last [d_model], decrypted */
int ckks_head_forward(ckks_block* head, const double* x_last, double* margin);
/* nblocks chained blocks with the full-hidden-state client refresh between
 * them, then the last-token refresh into `head` (may be NULL).  Blocks with
 * index >= cached_blocks release their diagonal cache after their forward.
 * hidden: [tokens, d_model] output of the last block. */
int ckks_model_forward(ckks_block* const* blocks, int nblocks, ckks_block* head, const double* x, int tokens,
                       int cached_blocks, double* hidden, double* margin);

/* ---- the block driver's fused matrix product and lane shift --------------
 * Slot layout slot(feature f, lane t) = f * batch + t with pack width
 * PW = N / (2 batch) features (T123.cpp:419-426 with one copy). */
typedef struct ckks_diag ckks_diag;
/* cached_diagonal_plains(W, level) (T123.cpp:1005-1059): the PW = n1 * n2
 * diagonals of the Halevi-Shoup product with W ([out_dim, in_dim] float64,
 * row stride ld, host; out_dim, in_dim <= PW), diagonal g * n1 + j holding
 * W[(f - n1 g) mod PW][(f + j) mod PW] at feature f of every lane (zero
 * outside the matrix, T123.cpp:1018-1046), encoded at `limbs` limbs with
 * that level's FLEXIBLEAUTO scale and kept on the device until destroyed
 * (n1, n2 <= 32). */
int ckks_bsgs_diagonals_create(ckks_ctx* ctx, const double* W, int out_dim, int in_dim, int ld, int batch, int n1,
                               int limbs, ckks_diag** out);
int ckks_bsgs_diagonals_destroy(ckks_diag* d);
/* matmul(BabyRotations, W) (T123.cpp:1264-1295) for `groups` token groups
 * and a sum of `terms` matrices: outs[q] = Rescale(sum_t sum_g rot(sum_j
 * diag_t[g n1 + j] * baby[(t * groups + q) * n1 + j], batch * n1 * g)),
 * where baby[... + j] = EvalRotate(x_{t,q}, batch * j) (j = 0: x itself) at
 * the diagonals' limbs and noise degree 1.  The inner sums of all groups of
 * a coefficient tile run in one fused kernel that reads each diagonal tile
 * from HBM once; the giant steps of a group are one rotation sum (one ModDown).
 * With terms > 1 the inner sums accumulate before the giant steps (the
 * summed MLP down projection).  Needs the rotation keys batch * n1 * g. */
int ckks_bsgs_matmul(ckks_ctx* ctx, const ckks_diag* const* diags, int terms, const ckks_ct* const* baby, int groups,
                     ckks_ct* const* outs);
/* lane_shift(x, d) (T123.cpp:1297-1314): out[f, t] = x[f, (t + d) mod batch]
 * = Rescale(rot(x, d) * [t < batch - d] + rot(x, d - batch) * [t >= batch - d])
 * for every input (one limb count, noise degree 1) and every d in
 * deltas (0 < d < batch): outs[i * nd + k] = lane_shift(in[i], deltas[k]).
 * The rotations of all inputs are one hoisted batch.  Needs the rotation
 * keys d and d - batch. */
int ckks_lane_shift(ckks_ctx* ctx, const ckks_ct* const* in, int count, const int* deltas, int nd, int batch,
                    ckks_ct* const* outs);

/* host-only schedule helpers: causal lane shifts of a (query group, key
 * group) tile (simd_layout.py:386-406) and one BSGS diagonal as slot values
 * (T123.cpp:1018-1046) */
int ckks_schedule_active_shifts(int tokens, int batch, int qg, int kg, int* out, int cap);
int ckks_schedule_diagonal(const double* W, int out_dim, int in_dim, int ld, int pack_width, int batch, int n1, int g,
                           int j, double* out_slots);

/* EvalRotate for callers that cannot allocate device memory (request
 * paths that must not enter the CUDA allocator, fixed memory budgets).  No
 * counterpart in the reference: it has no allocation-free entry point.
 * in_dev / out_dev: device buffers of 2*limbs*N words (c0 limbs then c1
 * limbs, NTT form), not overlapping.  Key-switching temporaries come from one
 * 128 MiB array compiled into the library (held by every GPU that loads it);
 * larger requests fail with CKKS_ECAPACITY.  No cudaMalloc/cudaFree.  The
 * first call on a device looks up the array's address (make it before any
 * stream capture); calls that overlap on the GPU race on the shared array. */
int ckks_rotate_noalloc(ckks_ctx* ctx, const uint64_t* in_dev, int limbs, int k, uint64_t* out_dev);

/* Diagnostic of the bounded waits: one CTA stages 4 KiB through a bulk copy
 * into shared memory and back.  starve = 0: CKKS_OK when the data came back
 * intact.  starve = 1: the barrier expects more bytes than are copied, the
 * wait gives up after one second, and ckks_sync's CKKS_ECUDA is returned. */
int ckks_selftest_bulk_wait(ckks_ctx* ctx, int starve);

#ifdef __cplusplus
}
#endif
#endif /* CKKS_B200_H */
