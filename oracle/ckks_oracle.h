/*
 * ckks_oracle.h -- CPU restatement of RNS-CKKS for the encrypted DNAGPT block
 * hot path.  TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and the
 * bench's cpu_baseline / reference arm may load it, as the checker and as the
 * timed CPU path; the product library never links it.
 *
 * What it restates (the reference delegates all of this to FIDESlib 786c760 +
 * the OpenFHE fork fideslib-ref-v1.5.1.1, neither of which is vendored):
 *   - CCParams/GenCryptoContext with FLEXIBLEAUTO + HYBRID
 *     (fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_
 *      depth13_digits3_ring65536_cpudiagcache_t123.cpp:1602-1621),
 *   - KeyGen / EvalMultKeyGen / EvalRotateKeyGen (same file :1622-1624),
 *   - MakeCKKSPackedPlaintext / Encrypt / Decrypt+GetRealPackedValue
 *     (:514-531, :1642-1661, :1675-1694),
 *   - EvalAdd / EvalSub / EvalMult(ct,pt) / EvalMult(ct,ct) / Rescale /
 *     EvalRotate / EvalFastRotation / AccumulateSum (:1144-1159, :1183-1203,
 *     :1286-1288).
 * Published algorithms followed: negacyclic NTT (Longa-Naehrig 2016 loop
 * order), HEAAN special FFT for the canonical embedding (Cheon-Kim-Kim-Song
 * 2017), hybrid key switching with dnum digits (Han-Ki 2020) and approximate
 * fast basis conversion (Halevi-Polyakov-Shoup 2019), ChaCha20 (RFC 7539) as
 * the seeded sampler, centered binomial errors.
 *
 * Parity with OpenFHE limbs is UNPINNED: OpenFHE is not available, so the
 * enforceable contract is limb-exact agreement between the CUDA engine and
 * this file given identical seeds, plus decrypted-value agreement with the
 * float64 plaintext block oracle.
 *
 * Layout: a polynomial with `limbs` RNS limbs is limbs*N uint64 words,
 * limb-major; limb i is reduced modulo moduli[i].  A ciphertext is two such
 * polynomials back to back (c0 then c1).  All polynomials handed across this
 * API are in NTT (evaluation) form, bit-reversed order, except where noted.
 */
#ifndef CKKS_ORACLE_H
#define CKKS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oc_ctx oc_ctx;

/* logN in [3,17]; L = Q limbs at the top level; dnum = number of digits
 * (alpha = ceil(L/dnum) limbs per digit, K = alpha special primes). */
oc_ctx* oc_create(int logN, int L, int dnum, int first_bits, int scale_bits,
                  int special_bits, uint64_t seed);
void oc_destroy(oc_ctx* c);
void oc_set_threads(int n);

int oc_N(const oc_ctx* c);
int oc_L(const oc_ctx* c);
int oc_K(const oc_ctx* c);
int oc_alpha(const oc_ctx* c);
void oc_moduli(const oc_ctx* c, uint64_t* out);      /* L+K words */
void oc_psi(const oc_ctx* c, uint64_t* out);         /* L+K primitive 2N-th roots */
double oc_scale(const oc_ctx* c, int limbs);          /* FLEXIBLEAUTO scale of a fresh encoding at `limbs` */

/* one limb, in place; prime_index in [0, L+K) */
void oc_ntt_fwd(const oc_ctx* c, int prime_index, uint64_t* a);
void oc_ntt_inv(const oc_ctx* c, int prime_index, uint64_t* a);

/* ChaCha20 block function (RFC 7539 rounds; words 12-13 counter, 14-15 nonce) */
void oc_chacha_block(const uint32_t key[8], uint64_t counter, uint64_t nonce, uint32_t out[16]);
/* 64-bit ChaCha20 sampler word pair for (seed, nonce, counter) */
void oc_chacha_words(uint64_t seed, uint64_t nonce, uint64_t counter, uint64_t out[2]);

/* values: N/2 real slots; out: limbs*N, NTT form.  Returns 0. */
int oc_encode(const oc_ctx* c, const double* values, int limbs, double scale, uint64_t* out);
/* count encodings at once (values count x N/2, out count x limbs x N), in parallel */
int oc_encode_batch(const oc_ctx* c, const double* values, int count, int limbs, double scale, uint64_t* out);
/* coefficient-form rounding only (no NTT); out: limbs*N */
int oc_encode_coeffs(const oc_ctx* c, const double* values, int limbs, double scale, uint64_t* out);
void oc_decode(const oc_ctx* c, const uint64_t* pt, int limbs, double scale, double* values);

/* keys (kept inside the context) */
void oc_keygen(oc_ctx* c);
void oc_relin_keygen(oc_ctx* c);
int oc_rot_keygen(oc_ctx* c, int k);                  /* rotation by k slots (left) */
void oc_secret_key(const oc_ctx* c, uint64_t* out);   /* (L+K)*N NTT form */
void oc_public_key(const oc_ctx* c, uint64_t* out);   /* 2*L*N */
/* key-switch key of a rotation (k) or relinearisation (k == 0):
 * dnum digits x 2 polys x (L+K) limbs x N */
int oc_switch_key(const oc_ctx* c, int k, uint64_t* out);
/* key switches at <= oc_low_limbs() limbs use keys over the first oc_K_low()
 * special primes (0: no such set); the key of index k (0 = relinearisation),
 * 2 x (L+K) x N words with the unused primes zero */
int oc_switch_key_low(const oc_ctx* c, int k, uint64_t* out);
int oc_low_limbs(const oc_ctx* c);
int oc_K_low(const oc_ctx* c);

void oc_encrypt(const oc_ctx* c, const uint64_t* pt, int limbs, uint64_t counter, uint64_t* ct);
void oc_decrypt(const oc_ctx* c, const uint64_t* ct, int limbs, uint64_t* pt);

/* element-wise; npolys polynomials of `limbs` limbs each */
void oc_add(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int npolys, int limbs, uint64_t* out);
void oc_sub(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int npolys, int limbs, uint64_t* out);
void oc_mul_pt(const oc_ctx* c, const uint64_t* ct, const uint64_t* pt, int limbs, uint64_t* out);
void oc_mul_int(const oc_ctx* c, const uint64_t* a, int npolys, int limbs, int64_t k, uint64_t* out);
void oc_add_int(const oc_ctx* c, const uint64_t* ct, int limbs, int64_t k, uint64_t* out);
/* d (coefficient form of k) added to c0: c0 += encode of constant k*scale
 * is done by callers through oc_add_const_scaled. */
void oc_add_const(const oc_ctx* c, const uint64_t* ct, int limbs, double value, double scale, uint64_t* out);

/* ct x ct: tensor then relinearise; out 2*limbs*N */
int oc_mul_ct(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int limbs, uint64_t* out);
void oc_tensor(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int limbs, uint64_t* out3);
/* hybrid key switch of d (limbs, NTT form) with key `ksk` (layout as oc_switch_key);
 * out: 2*limbs*N (delta c0, delta c1) */
void oc_keyswitch(const oc_ctx* c, const uint64_t* d, int limbs, const uint64_t* ksk, uint64_t* out);
/* sum_r a_r * b_r (n pairs, each 2*limbs*N) with one relinearisation */
int oc_mul_ct_sum(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int n, int limbs, uint64_t* out);
/* drop the last limb with division by it; out 2*(limbs-1)*N */
void oc_rescale(const oc_ctx* c, const uint64_t* ct, int limbs, uint64_t* out);
/* automorphism X -> X^g in NTT form on npolys polys */
void oc_automorphism(const oc_ctx* c, const uint64_t* a, int npolys, int limbs, uint32_t g, uint64_t* out);
uint32_t oc_galois_element(const oc_ctx* c, int k);
int oc_rotate(const oc_ctx* c, const uint64_t* ct, int limbs, int k, uint64_t* out);
int oc_rotate_hoisted(const oc_ctx* c, const uint64_t* ct, int limbs, const int* ks, int n, uint64_t* out);
/* sum_r rot(cts[r], ks[r]) with one ModDown per group of 32 non-identity rotations */
int oc_rotate_sum(const oc_ctx* c, const uint64_t* cts, int limbs, const int* ks, int n, uint64_t* out);
int oc_accumulate_sum(const oc_ctx* c, const uint64_t* ct, int limbs, int count, int stride, uint64_t* out);
/* the engine's window sums: the same ladder, one ModDown per step */
int oc_window_sum(const oc_ctx* c, const uint64_t* ct, int limbs, int window, int stride, uint64_t* out);
int oc_window_sum_radix(const oc_ctx* c, const uint64_t* ct, int limbs, int window, int stride, int radix,
                        uint64_t* out);

/* ModUp / ModDown exposed for limb-level parity of the key-switch stages.
 * modup: d in coefficient form (limbs) -> digits x (limbs+K) NTT form.
 * (takes NTT-form d, like the engine does) */
void oc_modup(const oc_ctx* c, const uint64_t* d_ntt, int limbs, uint64_t* ext);
void oc_moddown(const oc_ctx* c, const uint64_t* x_ntt, int limbs, uint64_t* out);

/* inner sums of the BSGS product (T123.cpp:1264-1295): out[g] (+)= sum_{j<n1}
 * diag[g*n1 + j] * baby[j] for g < n2; babies n1 x 2 x limbs x N, diags
 * (n1*n2) x limbs x N, out n2 x 2 x limbs x N */
int oc_bsgs_inner(const oc_ctx* c, const uint64_t* babies, int n1, const uint64_t* diags, int n2, int limbs,
                  int accumulate, uint64_t* out);

const char* oc_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
