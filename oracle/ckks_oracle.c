/*
 * ckks_oracle.c -- CPU restatement of RNS-CKKS (see ckks_oracle.h).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA engine and
 * the timed CPU baseline; the product never links it.  It is written from the
 * published algorithms named in the header, not from OpenFHE or FIDESlib
 * sources (neither is present).  Every function notes the reference call site
 * whose behaviour it restates; "T123" below is
 * fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_depth13_
 * digits3_ring65536_cpudiagcache_t123.cpp.
 *
 * Compile with -ffp-contract=off: the encoder's floating-point steps must be
 * performed one IEEE operation at a time, in the order written, because the
 * CUDA encoder performs the same operations with explicit _rn intrinsics and
 * the two must agree bit for bit.
 */
#include "ckks_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef unsigned __int128 u128;

#define OC_MAXP 80
#define OC_MAXROT 512

static __thread char g_err[256];
static void set_err(const char* m) { snprintf(g_err, sizeof g_err, "%s", m); }
const char* oc_last_error(void) { return g_err; }

void oc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------ */
/* modular arithmetic                                                  */
/* ------------------------------------------------------------------ */
typedef struct {
    uint64_t q, r1, r0; /* floor(2^128 / q) = r1*2^64 + r0 */
} modulus_t;

static modulus_t make_modulus(uint64_t q) {
    modulus_t m;
    m.q = q;
    /* floor((2^128 - 1) / q) equals floor(2^128 / q) because q is odd */
    u128 all = ~(u128)0;
    u128 r = all / q;
    m.r1 = (uint64_t)(r >> 64);
    m.r0 = (uint64_t)r;
    return m;
}

/* x mod q for any 128-bit x: quotient estimate floor(x * floor(2^128/q) / 2^128)
 * is floor(x/q) or one less, so one conditional subtraction finishes. */
static inline uint64_t reduce128(u128 x, const modulus_t* m) {
    uint64_t xl = (uint64_t)x, xh = (uint64_t)(x >> 64);
    uint64_t carry = (uint64_t)(((u128)xl * m->r0) >> 64);
    u128 a = (u128)xl * m->r1 + carry;
    u128 b = (u128)xh * m->r0 + (uint64_t)a;
    uint64_t qe = xh * m->r1 + (uint64_t)(a >> 64) + (uint64_t)(b >> 64);
    uint64_t r = xl - qe * m->q;
    return r >= m->q ? r - m->q : r;
}
static inline uint64_t mulm(uint64_t a, uint64_t b, const modulus_t* m) {
    return reduce128((u128)a * b, m);
}
static inline uint64_t addm(uint64_t a, uint64_t b, uint64_t q) {
    uint64_t s = a + b;
    return s >= q ? s - q : s;
}
static inline uint64_t subm(uint64_t a, uint64_t b, uint64_t q) {
    return a >= b ? a - b : a + q - b;
}
static inline uint64_t shoup_pre(uint64_t w, uint64_t q) {
    return (uint64_t)(((u128)w << 64) / q);
}
static inline uint64_t mul_shoup(uint64_t a, uint64_t w, uint64_t wp, uint64_t q) {
    uint64_t h = (uint64_t)(((u128)a * wp) >> 64);
    uint64_t r = a * w - h * q;
    return r >= q ? r - q : r;
}
static uint64_t powm(uint64_t b, uint64_t e, uint64_t q) {
    u128 r = 1, x = b % q;
    while (e) {
        if (e & 1) r = (r * x) % q;
        x = (x * x) % q;
        e >>= 1;
    }
    return (uint64_t)r;
}
static uint64_t invm(uint64_t a, uint64_t q) { return powm(a, q - 2, q); }

/* deterministic Miller-Rabin for 64-bit inputs (first 12 prime bases) */
static int is_prime64(uint64_t n) {
    static const uint64_t bases[12] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
    if (n < 2) return 0;
    for (int i = 0; i < 12; i++) {
        if (n == bases[i]) return 1;
        if (n % bases[i] == 0) return 0;
    }
    uint64_t d = n - 1;
    int s = 0;
    while (!(d & 1)) { d >>= 1; s++; }
    for (int i = 0; i < 12; i++) {
        uint64_t x = powm(bases[i], d, n);
        if (x == 1 || x == n - 1) continue;
        int comp = 1;
        for (int r = 1; r < s; r++) {
            x = (uint64_t)(((u128)x * x) % n);
            if (x == n - 1) { comp = 0; break; }
        }
        if (comp) return 0;
    }
    return 1;
}

static uint32_t bitrev(uint32_t x, int bits) {
    uint32_t r = 0;
    for (int i = 0; i < bits; i++) { r = (r << 1) | (x & 1); x >>= 1; }
    return r;
}

/* ------------------------------------------------------------------ */
/* context                                                             */
/* ------------------------------------------------------------------ */
typedef struct { double re, im; } cplx;

struct oc_ctx {
    int logN, N, L, K, dnum, alpha, beta;
    uint64_t seed;
    uint64_t q[OC_MAXP];
    modulus_t mod[OC_MAXP];
    uint64_t psi[OC_MAXP];
    uint64_t *w, *wp, *wi, *wip; /* (L+K)*N twiddle tables */
    uint64_t ninv[OC_MAXP], ninvp[OC_MAXP];
    double scales[OC_MAXP + 1];
    cplx* ksi;           /* M+1 roots of unity exp(2 pi i k / M), M = 2N */
    uint32_t* rot_group; /* 5^j mod M, j < N/2 */
    uint64_t* sk;        /* (L+K)*N */
    uint64_t* pk;        /* 2*L*N */
    uint64_t* rlk;       /* beta*2*(L+K)*N */
    int nrot;
    uint32_t rot_g[OC_MAXROT];
    uint64_t* rot_key[OC_MAXROT];
    /* one-digit key switches at <= low_limbs limbs use keys over the first
     * K_low special primes (log2 P' >= log2 Q_low + 20); 0 = none */
    int low_limbs, K_low;
    uint64_t* rlk_low;                 /* 2*(L+K)*N, unused primes zero */
    uint64_t* rot_key_low[OC_MAXROT];  /* parallel to rot_key */
};

static inline int is_low(const oc_ctx* c, int limbs) { return c->low_limbs > 0 && limbs <= c->low_limbs; }
static inline int kx(const oc_ctx* c, int limbs) { return is_low(c, limbs) ? c->K_low : c->K; }

int oc_N(const oc_ctx* c) { return c->N; }
int oc_L(const oc_ctx* c) { return c->L; }
int oc_K(const oc_ctx* c) { return c->K; }
int oc_alpha(const oc_ctx* c) { return c->alpha; }
void oc_moduli(const oc_ctx* c, uint64_t* out) { memcpy(out, c->q, sizeof(uint64_t) * (c->L + c->K)); }
void oc_psi(const oc_ctx* c, uint64_t* out) { memcpy(out, c->psi, sizeof(uint64_t) * (c->L + c->K)); }
double oc_scale(const oc_ctx* c, int limbs) {
    if (limbs < 1 || limbs > c->L) return 0.0;
    return c->scales[limbs];
}

static int used(const uint64_t* list, int n, uint64_t v) {
    for (int i = 0; i < n; i++)
        if (list[i] == v) return 1;
    return 0;
}

/* Prime chain, restating the parameter choice of T123.cpp:1602-1621
 * (SetFirstModSize, SetScalingModSize, HYBRID special primes):
 *   q_0            largest prime below 2^first_bits with q = 1 mod 2N,
 *   q_1..q_{L-1}   primes = 1 mod 2N taken alternately just below and just
 *                  above 2^scale_bits, so that consecutive scales stay close
 *                  to 2^scale_bits,
 *   p_0..p_{K-1}   largest unused primes below 2^special_bits, = 1 mod 2N. */
static int gen_primes(oc_ctx* c, int first_bits, int scale_bits, int special_bits) {
    const uint64_t M = 2ull * (uint64_t)c->N;
    int n = 0;
    uint64_t* q = c->q;
    {
        uint64_t base = (1ull << first_bits) + 1;
        for (uint64_t m = 1;; m++) {
            if (m * M >= base) return -1;
            uint64_t cand = base - m * M;
            if (is_prime64(cand)) { q[n++] = cand; break; }
        }
    }
    {
        uint64_t base = (1ull << scale_bits) + 1;
        uint64_t mlo = 1, mhi = 1;
        int below = 1;
        while (n < c->L) {
            uint64_t cand;
            if (below) {
                for (;; mlo++) {
                    if (mlo * M >= base) return -1;
                    cand = base - mlo * M;
                    if (is_prime64(cand) && !used(q, n, cand)) { mlo++; break; }
                }
            } else {
                for (;; mhi++) {
                    cand = base + mhi * M;
                    if (is_prime64(cand) && !used(q, n, cand)) { mhi++; break; }
                }
            }
            q[n++] = cand;
            below = !below;
        }
    }
    {
        uint64_t base = (1ull << special_bits) + 1;
        int k = 0;
        for (uint64_t m = 1; k < c->K; m++) {
            if (m * M >= base) return -1;
            uint64_t cand = base - m * M;
            if (is_prime64(cand) && !used(q, n, cand)) { q[n++] = cand; k++; }
        }
    }
    return 0;
}

/* smallest x >= 2 whose power x^((q-1)/2N) is a primitive 2N-th root */
static uint64_t find_psi(uint64_t q, uint64_t twoN) {
    for (uint64_t x = 2;; x++) {
        uint64_t p = powm(x, (q - 1) / twoN, q);
        if (powm(p, twoN / 2, q) == q - 1) return p;
    }
}

oc_ctx* oc_create(int logN, int L, int dnum, int first_bits, int scale_bits,
                  int special_bits, uint64_t seed) {
    if (logN < 3 || logN > 17 || L < 1 || dnum < 1 || L + (L + dnum - 1) / dnum > OC_MAXP ||
        first_bits > 61 || scale_bits > 61 || special_bits > 61 || first_bits <= logN + 1 ||
        scale_bits <= logN + 1 || special_bits <= logN + 1) {
        set_err("oc_create: parameters out of range");
        return NULL;
    }
    oc_ctx* c = (oc_ctx*)calloc(1, sizeof(oc_ctx));
    c->logN = logN;
    c->N = 1 << logN;
    c->L = L;
    c->dnum = dnum;
    c->alpha = (L + dnum - 1) / dnum;
    c->beta = (L + c->alpha - 1) / c->alpha;
    c->K = c->alpha;
    c->seed = seed;
    if (gen_primes(c, first_bits, scale_bits, special_bits)) {
        set_err("oc_create: prime search failed");
        free(c);
        return NULL;
    }
    const int P = L + c->K, N = c->N;
    c->w = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)P * N);
    c->wp = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)P * N);
    c->wi = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)P * N);
    c->wip = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)P * N);
    for (int i = 0; i < P; i++) {
        uint64_t q = c->q[i];
        c->mod[i] = make_modulus(q);
        uint64_t psi = find_psi(q, 2ull * N);
        c->psi[i] = psi;
        uint64_t psii = invm(psi, q);
        uint64_t *w = c->w + (size_t)i * N, *wi = c->wi + (size_t)i * N;
        uint64_t p = 1, pi = 1;
        /* psi^j stored at bit-reversed position: w[bitrev(j)] = psi^j */
        for (int j = 0; j < N; j++) {
            uint32_t r = bitrev((uint32_t)j, logN);
            w[r] = p;
            wi[r] = pi;
            p = (uint64_t)(((u128)p * psi) % q);
            pi = (uint64_t)(((u128)pi * psii) % q);
        }
        for (int j = 0; j < N; j++) {
            c->wp[(size_t)i * N + j] = shoup_pre(w[j], q);
            c->wip[(size_t)i * N + j] = shoup_pre(wi[j], q);
        }
        c->ninv[i] = invm((uint64_t)N, q);
        c->ninvp[i] = shoup_pre(c->ninv[i], q);
    }
    /* FLEXIBLEAUTO-style scale chain: fresh top-level scale is the last
     * scaling prime; each rescale by q_{l-1} maps s -> s*s/q_{l-1}. */
    c->scales[L] = (L >= 2) ? (double)c->q[L - 1] : ldexp(1.0, scale_bits);
    for (int l = L; l >= 2; l--) c->scales[l - 1] = c->scales[l] * c->scales[l] / (double)c->q[l - 1];
    /* reduced special-prime set for one-digit key switches at <= 3 limbs:
     * the fewest leading special primes with log2 P' >= log2 Q_3 + 19.5 */
    {
        const int lo = c->alpha < 3 ? c->alpha : 3;
        double qbits = 0.0, pbits = 0.0;
        for (int i = 0; i < lo; i++) qbits += log2((double)c->q[i]);
        int k = 0;
        while (k < c->K && pbits < qbits + 19.5) pbits += log2((double)c->q[L + k++]);
        if (L >= lo && lo >= 1 && pbits >= qbits + 19.5 && k < c->K) {
            c->low_limbs = lo;
            c->K_low = k;
        }
    }
    /* canonical-embedding tables (HEAAN special FFT) */
    const int M = 2 * N;
    c->ksi = (cplx*)malloc(sizeof(cplx) * (size_t)(M + 1));
    for (int k = 0; k <= M; k++) {
        double ang = 2.0 * M_PI * (double)k / (double)M;
        c->ksi[k].re = cos(ang);
        c->ksi[k].im = sin(ang);
    }
    c->rot_group = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(N / 2));
    uint64_t g = 1;
    for (int j = 0; j < N / 2; j++) {
        c->rot_group[j] = (uint32_t)g;
        g = (g * 5) % (uint64_t)M;
    }
    return c;
}

void oc_destroy(oc_ctx* c) {
    if (!c) return;
    free(c->w); free(c->wp); free(c->wi); free(c->wip);
    free(c->ksi); free(c->rot_group);
    free(c->sk); free(c->pk); free(c->rlk); free(c->rlk_low);
    for (int i = 0; i < c->nrot; i++) { free(c->rot_key[i]); free(c->rot_key_low[i]); }
    free(c);
}

/* ------------------------------------------------------------------ */
/* NTT: Cooley-Tukey forward (natural in, bit-reversed out) and        */
/* Gentleman-Sande inverse (bit-reversed in, natural out), negacyclic  */
/* twist folded into the bit-reversed psi tables.                      */
/* ------------------------------------------------------------------ */
void oc_ntt_fwd(const oc_ctx* c, int pi, uint64_t* a) {
    const uint64_t q = c->q[pi];
    const uint64_t* W = c->w + (size_t)pi * c->N;
    const uint64_t* Wp = c->wp + (size_t)pi * c->N;
    const int N = c->N;
    int t = N;
    for (int m = 1; m < N; m <<= 1) {
        t >>= 1;
        for (int i = 0; i < m; i++) {
            const int j1 = 2 * i * t;
            const uint64_t w = W[m + i], wp = Wp[m + i];
            for (int j = j1; j < j1 + t; j++) {
                uint64_t u = a[j];
                uint64_t v = mul_shoup(a[j + t], w, wp, q);
                a[j] = addm(u, v, q);
                a[j + t] = subm(u, v, q);
            }
        }
    }
}

void oc_ntt_inv(const oc_ctx* c, int pi, uint64_t* a) {
    const uint64_t q = c->q[pi];
    const uint64_t* W = c->wi + (size_t)pi * c->N;
    const uint64_t* Wp = c->wip + (size_t)pi * c->N;
    const int N = c->N;
    int t = 1;
    for (int m = N; m > 1; m >>= 1) {
        const int h = m >> 1;
        int j1 = 0;
        for (int i = 0; i < h; i++) {
            const uint64_t w = W[h + i], wp = Wp[h + i];
            for (int j = j1; j < j1 + t; j++) {
                uint64_t u = a[j], v = a[j + t];
                a[j] = addm(u, v, q);
                a[j + t] = mul_shoup(subm(u, v, q), w, wp, q);
            }
            j1 += 2 * t;
        }
        t <<= 1;
    }
    for (int j = 0; j < N; j++) a[j] = mul_shoup(a[j], c->ninv[pi], c->ninvp[pi], q);
}

/* ------------------------------------------------------------------ */
/* ChaCha20 sampler (RFC 7539 block function, 64-bit counter + nonce)  */
/* ------------------------------------------------------------------ */
#define ROTL32(v, n) (((v) << (n)) | ((v) >> (32 - (n))))
#define QR(a, b, c, d)                  \
    a += b; d ^= a; d = ROTL32(d, 16);  \
    c += d; b ^= c; b = ROTL32(b, 12);  \
    a += b; d ^= a; d = ROTL32(d, 8);   \
    c += d; b ^= c; b = ROTL32(b, 7);

static uint64_t splitmix(uint64_t* x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* RFC 7539 block function with a 64-bit counter (words 12-13) and a 64-bit
 * nonce (words 14-15); out = the 16 output words (state + input state). */
void oc_chacha_block(const uint32_t key[8], uint64_t counter, uint64_t nonce, uint32_t out[16]) {
    uint32_t st[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                       key[0], key[1], key[2], key[3], key[4], key[5], key[6], key[7],
                       (uint32_t)counter, (uint32_t)(counter >> 32),
                       (uint32_t)nonce, (uint32_t)(nonce >> 32)};
    uint32_t x[16];
    memcpy(x, st, sizeof x);
    for (int r = 0; r < 10; r++) {
        QR(x[0], x[4], x[8], x[12]);
        QR(x[1], x[5], x[9], x[13]);
        QR(x[2], x[6], x[10], x[14]);
        QR(x[3], x[7], x[11], x[15]);
        QR(x[0], x[5], x[10], x[15]);
        QR(x[1], x[6], x[11], x[12]);
        QR(x[2], x[7], x[8], x[13]);
        QR(x[3], x[4], x[9], x[14]);
    }
    for (int i = 0; i < 16; i++) out[i] = x[i] + st[i];
}

static void chacha_words(uint64_t seed, uint64_t nonce, uint64_t counter, uint64_t out[2]) {
    uint32_t key[8];
    uint64_t s = seed;
    for (int i = 0; i < 4; i++) {
        uint64_t k = splitmix(&s);
        key[2 * i] = (uint32_t)k;
        key[2 * i + 1] = (uint32_t)(k >> 32);
    }
    uint32_t st[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                       key[0], key[1], key[2], key[3], key[4], key[5], key[6], key[7],
                       (uint32_t)counter, (uint32_t)(counter >> 32),
                       (uint32_t)nonce, (uint32_t)(nonce >> 32)};
    uint32_t x[16];
    memcpy(x, st, sizeof x);
    for (int r = 0; r < 10; r++) {
        QR(x[0], x[4], x[8], x[12]);
        QR(x[1], x[5], x[9], x[13]);
        QR(x[2], x[6], x[10], x[14]);
        QR(x[3], x[7], x[11], x[15]);
        QR(x[0], x[5], x[10], x[15]);
        QR(x[1], x[6], x[11], x[12]);
        QR(x[2], x[7], x[8], x[13]);
        QR(x[3], x[4], x[9], x[14]);
    }
    for (int i = 0; i < 4; i++) x[i] += st[i];
    out[0] = (uint64_t)x[0] | ((uint64_t)x[1] << 32);
    out[1] = (uint64_t)x[2] | ((uint64_t)x[3] << 32);
}
void oc_chacha_words(uint64_t seed, uint64_t nonce, uint64_t counter, uint64_t out[2]) {
    chacha_words(seed, nonce, counter, out);
}

/* sampler domains (nonces) */
#define NONCE_SK 0x01ull
#define NONCE_PK_A 0x02ull
#define NONCE_PK_E 0x03ull
#define NONCE_KSK(id, j, part) ((0x10ull << 36) | ((uint64_t)(id) << 8) | ((uint64_t)(j) << 1) | (uint64_t)(part))
#define NONCE_KSK_LOW(id, part) ((0x11ull << 36) | ((uint64_t)(id) << 8) | (uint64_t)(part))
#define NONCE_ENC(cnt, sub) ((0x20ull << 56) | ((uint64_t)(cnt) << 2) | (uint64_t)(sub))
#define KEYID_RELIN 1u
#define KEYID_ROT(g) (0x100u + (uint32_t)(g))

/* ternary in {-1, 0, 1} and the centred binomial of 21 + 21 bits */
static int ternary_of(uint64_t w) {
    uint64_t t = w % 3;
    return t == 0 ? 0 : (t == 1 ? 1 : -1);
}
static int cbd_of(uint64_t w) {
    return __builtin_popcountll(w & 0x1FFFFFull) - __builtin_popcountll((w >> 21) & 0x1FFFFFull);
}
static int sample_ternary(uint64_t seed, uint64_t nonce, uint64_t n) {
    uint64_t w[2];
    chacha_words(seed, nonce, n, w);
    return ternary_of(w[0]);
}
static int sample_cbd(uint64_t seed, uint64_t nonce, uint64_t n) {
    uint64_t w[2];
    chacha_words(seed, nonce, n, w);
    return cbd_of(w[0]);
}
/* all 16 output words of block `counter` as eight 64-bit words: the
 * encryption sampler takes coefficient n from word n % 8 of block n / 8 */
static void chacha_words8(uint64_t seed, uint64_t nonce, uint64_t counter, uint64_t out[8]) {
    uint32_t key[8];
    uint64_t s = seed;
    for (int i = 0; i < 4; i++) {
        uint64_t k = splitmix(&s);
        key[2 * i] = (uint32_t)k;
        key[2 * i + 1] = (uint32_t)(k >> 32);
    }
    uint32_t w[16];
    oc_chacha_block(key, counter, nonce, w);
    for (int i = 0; i < 8; i++) out[i] = (uint64_t)w[2 * i] | ((uint64_t)w[2 * i + 1] << 32);
}
static uint64_t sample_uniform(uint64_t seed, uint64_t nonce, uint64_t counter, const modulus_t* m) {
    uint64_t w[2];
    chacha_words(seed, nonce, counter, w);
    return reduce128(((u128)w[0] << 64) | w[1], m);
}

static inline uint64_t small_to_res(int v, uint64_t q) {
    return v >= 0 ? (uint64_t)v : q - (uint64_t)(-v);
}

/* integer-valued small polynomial -> NTT form on the listed primes */
static void small_poly_ntt(const oc_ctx* c, const int* v, const int* primes, int nlimbs, uint64_t* out) {
    const int N = c->N;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < nlimbs; l++) {
        uint64_t q = c->q[primes[l]];
        uint64_t* o = out + (size_t)l * N;
        for (int n = 0; n < N; n++) o[n] = small_to_res(v[n], q);
        oc_ntt_fwd(c, primes[l], o);
    }
}

/* ------------------------------------------------------------------ */
/* canonical embedding: HEAAN special FFT over the 5^j orbit            */
/* ------------------------------------------------------------------ */
static inline cplx cmul(cplx a, cplx b) {
    cplx r;
    double t1 = a.re * b.re;
    double t2 = a.im * b.im;
    double t3 = a.re * b.im;
    double t4 = a.im * b.re;
    r.re = t1 - t2;
    r.im = t3 + t4;
    return r;
}
static void bit_reverse_cplx(cplx* v, int n) {
    int bits = 0;
    while ((1 << bits) < n) bits++;
    for (int i = 0; i < n; i++) {
        int j = (int)bitrev((uint32_t)i, bits);
        if (i < j) { cplx t = v[i]; v[i] = v[j]; v[j] = t; }
    }
}
/* z_j = sum_i v_i * zeta^(5^j * i), zeta = exp(2 pi i / 2N) */
static void fft_special(const oc_ctx* c, cplx* v, int n) {
    const int M = 2 * c->N;
    bit_reverse_cplx(v, n);
    for (int len = 2; len <= n; len <<= 1) {
        const int lenh = len >> 1, lenq = len << 2, gap = M / lenq;
        for (int i = 0; i < n; i += len) {
            for (int j = 0; j < lenh; j++) {
                int idx = (int)(c->rot_group[j] % (uint32_t)lenq) * gap;
                cplx u = v[i + j];
                cplx t = cmul(v[i + j + lenh], c->ksi[idx]);
                v[i + j].re = u.re + t.re;
                v[i + j].im = u.im + t.im;
                v[i + j + lenh].re = u.re - t.re;
                v[i + j + lenh].im = u.im - t.im;
            }
        }
    }
}
/* inverse of fft_special (without the 1/n, applied by the caller) */
static void ifft_special(const oc_ctx* c, cplx* v, int n) {
    const int M = 2 * c->N;
    for (int len = n; len >= 2; len >>= 1) {
        const int lenh = len >> 1, lenq = len << 2, gap = M / lenq;
        for (int i = 0; i < n; i += len) {
            for (int j = 0; j < lenh; j++) {
                int idx = (lenq - (int)(c->rot_group[j] % (uint32_t)lenq)) * gap;
                cplx a = v[i + j], b = v[i + j + lenh];
                cplx u, d;
                u.re = a.re + b.re;
                u.im = a.im + b.im;
                d.re = a.re - b.re;
                d.im = a.im - b.im;
                v[i + j] = u;
                v[i + j + lenh] = cmul(d, c->ksi[idx]);
            }
        }
    }
    bit_reverse_cplx(v, n);
}

/* residue of an integer-valued double, exact for every magnitude:
 * |r| < 2^63 converts directly; above, r = mant * 2^e with a 53-bit mant. */
static uint64_t double_to_res(double r, const modulus_t* m) {
    double ar = fabs(r);
    uint64_t v;
    if (ar < 9223372036854775808.0) {
        v = ((uint64_t)ar) % m->q;
    } else {
        uint64_t bits;
        memcpy(&bits, &ar, 8);
        int e = (int)((bits >> 52) & 0x7FF) - 1075;
        uint64_t mant = (bits & ((1ull << 52) - 1)) | (1ull << 52);
        v = mulm(mant % m->q, powm(2, (uint64_t)e, m->q), m);
    }
    return (r < 0 && v) ? m->q - v : v;
}

/* MakeCKKSPackedPlaintext(values, 1, level, nullptr, N/2), real slots
 * (T123.cpp:955-960): iFFT, /n, *scale, round half-to-even, RNS. */
int oc_encode_coeffs(const oc_ctx* c, const double* values, int limbs, double scale, uint64_t* out) {
    const int N = c->N, n = N / 2;
    if (limbs < 1 || limbs > c->L + c->K) { set_err("encode: bad limb count"); return -1; }
    cplx* v = (cplx*)malloc(sizeof(cplx) * (size_t)n);
    for (int j = 0; j < n; j++) { v[j].re = values[j]; v[j].im = 0.0; }
    ifft_special(c, v, n);
    double* coef = (double*)malloc(sizeof(double) * (size_t)N);
    const double dn = (double)n;
    for (int i = 0; i < n; i++) {
        double re = v[i].re / dn;
        double im = v[i].im / dn;
        coef[i] = rint(re * scale);
        coef[i + n] = rint(im * scale);
    }
    free(v);
#pragma omp parallel for schedule(static)
    for (int l = 0; l < limbs; l++) {
        for (int i = 0; i < N; i++) out[(size_t)l * N + i] = double_to_res(coef[i], &c->mod[l]);
    }
    free(coef);
    return 0;
}

int oc_encode(const oc_ctx* c, const double* values, int limbs, double scale, uint64_t* out) {
    if (limbs > c->L) { set_err("encode: more limbs than the Q chain"); return -1; }
    if (oc_encode_coeffs(c, values, limbs, scale, out)) return -1;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < limbs; l++) oc_ntt_fwd(c, l, out + (size_t)l * c->N);
    return 0;
}

/* `count` independent encodings (values: count x N/2, out: count x limbs x
 * N), spread over the threads: the reference encodes a product's diagonals
 * this way, one MakeCKKSPackedPlaintext per diagonal in an OpenMP loop
 * (T123.cpp:1048-1056). */
int oc_encode_batch(const oc_ctx* c, const double* values, int count, int limbs, double scale, uint64_t* out) {
    if (limbs > c->L) { set_err("encode: more limbs than the Q chain"); return -1; }
    int bad = 0;
#pragma omp parallel for schedule(dynamic) reduction(| : bad)
    for (int i = 0; i < count; i++)
        bad |= oc_encode(c, values + (size_t)i * (c->N / 2), limbs, scale, out + (size_t)i * limbs * c->N) != 0;
    return bad ? -1 : 0;
}

/* centered CRT over the first two limbs -> double, then /scale and FFT
 * (Decrypt + GetRealPackedValue, T123.cpp:523-531). */
void oc_decode(const oc_ctx* c, const uint64_t* pt, int limbs, double scale, double* values) {
    const int N = c->N, n = N / 2;
    const int use = limbs >= 2 ? 2 : 1;
    uint64_t* tmp = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)use * N);
    memcpy(tmp, pt, sizeof(uint64_t) * (size_t)use * N);
    for (int l = 0; l < use; l++) oc_ntt_inv(c, l, tmp + (size_t)l * N);
    double* d = (double*)malloc(sizeof(double) * (size_t)N);
    const uint64_t q0 = c->q[0], q1 = c->q[1];
    const uint64_t q0inv1 = use == 2 ? invm(q0 % q1, q1) : 0;
    const u128 Q = use == 2 ? (u128)q0 * q1 : (u128)q0;
    for (int i = 0; i < N; i++) {
        u128 x;
        if (use == 2) {
            uint64_t x0 = tmp[i], x1 = tmp[N + i];
            uint64_t t = mulm(subm(x1, x0 % q1, q1), q0inv1, &c->mod[1]);
            x = (u128)x0 + (u128)q0 * t;
        } else {
            x = tmp[i];
        }
        int neg = 0;
        u128 mag = x;
        if (x > Q / 2) { mag = Q - x; neg = 1; }
        double hi = (double)(uint64_t)(mag >> 64);
        double lo = (double)(uint64_t)mag;
        double val = hi * 18446744073709551616.0 + lo;
        if (neg) val = -val;
        d[i] = val / scale;
    }
    free(tmp);
    cplx* v = (cplx*)malloc(sizeof(cplx) * (size_t)n);
    for (int j = 0; j < n; j++) { v[j].re = d[j]; v[j].im = d[j + n]; }
    free(d);
    fft_special(c, v, n);
    for (int j = 0; j < n; j++) values[j] = v[j].re;
    free(v);
}

/* ------------------------------------------------------------------ */
/* keys: KeyGen / EvalMultKeyGen / EvalRotateKeyGen (T123.cpp:1622-1624) */
/* ------------------------------------------------------------------ */
static int* all_primes(const oc_ctx* c) {
    int* p = (int*)malloc(sizeof(int) * (size_t)(c->L + c->K));
    for (int i = 0; i < c->L + c->K; i++) p[i] = i;
    return p;
}

void oc_keygen(oc_ctx* c) {
    const int N = c->N, P = c->L + c->K;
    int* s = (int*)malloc(sizeof(int) * (size_t)N);
    for (int n = 0; n < N; n++) s[n] = sample_ternary(c->seed, NONCE_SK, (uint64_t)n);
    free(c->sk);
    c->sk = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)P * N);
    int* pr = all_primes(c);
    small_poly_ntt(c, s, pr, P, c->sk);
    /* public key over the Q limbs: b = -a*s + e, a uniform in NTT form */
    int* e = (int*)malloc(sizeof(int) * (size_t)N);
    for (int n = 0; n < N; n++) e[n] = sample_cbd(c->seed, NONCE_PK_E, (uint64_t)n);
    uint64_t* en = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)c->L * N);
    small_poly_ntt(c, e, pr, c->L, en);
    free(c->pk);
    c->pk = (uint64_t*)malloc(sizeof(uint64_t) * 2 * (size_t)c->L * N);
    uint64_t *b = c->pk, *a = c->pk + (size_t)c->L * N;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < c->L; l++) {
        const modulus_t* m = &c->mod[l];
        for (int n = 0; n < N; n++) {
            size_t o = (size_t)l * N + n;
            uint64_t av = sample_uniform(c->seed, NONCE_PK_A, o, m);
            a[o] = av;
            b[o] = subm(en[o], mulm(av, c->sk[o], m), m->q);
        }
    }
    free(s); free(e); free(en); free(pr);
}

void oc_secret_key(const oc_ctx* c, uint64_t* out) {
    memcpy(out, c->sk, sizeof(uint64_t) * (size_t)(c->L + c->K) * c->N);
}
void oc_public_key(const oc_ctx* c, uint64_t* out) {
    memcpy(out, c->pk, sizeof(uint64_t) * 2 * (size_t)c->L * c->N);
}

/* switching key from s_from to s: digit j encrypts P * [i in digit j] * s_from
 * modulo every Q prime i (the CRT idempotent of digit j times P), and 0
 * modulo the P primes. */
static uint64_t* make_switch_key(const oc_ctx* c, const uint64_t* s_from, uint32_t key_id) {
    const int N = c->N, P = c->L + c->K;
    uint64_t* key = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)c->beta * 2 * P * N);
    int* pr = all_primes(c);
    int* e = (int*)malloc(sizeof(int) * (size_t)N);
    uint64_t* en = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)P * N);
    for (int j = 0; j < c->beta; j++) {
        for (int n = 0; n < N; n++) e[n] = sample_cbd(c->seed, NONCE_KSK(key_id, j, 1), (uint64_t)n);
        small_poly_ntt(c, e, pr, P, en);
        uint64_t* b = key + (size_t)j * 2 * P * N;
        uint64_t* a = b + (size_t)P * N;
        const int lo = j * c->alpha, hi = (lo + c->alpha < c->L) ? lo + c->alpha : c->L;
#pragma omp parallel for schedule(static)
        for (int t = 0; t < P; t++) {
            const modulus_t* m = &c->mod[t];
            uint64_t pmod = 1;
            for (int k = 0; k < c->K; k++) pmod = mulm(pmod, c->q[c->L + k] % m->q, m);
            const int in_digit = (t >= lo && t < hi);
            for (int n = 0; n < N; n++) {
                size_t o = (size_t)t * N + n;
                uint64_t av = sample_uniform(c->seed, NONCE_KSK(key_id, j, 0), o, m);
                a[o] = av;
                uint64_t bv = subm(en[o], mulm(av, c->sk[o], m), m->q);
                if (in_digit) bv = addm(bv, mulm(pmod, s_from[o], m), m->q);
                b[o] = bv;
            }
        }
    }
    free(pr); free(e); free(en);
    return key;
}

/* the same key over the reduced special-prime set: one digit covering Q
 * primes 0..low_limbs-1 with P' = p_0 ... p_{K_low-1}; rows of the other
 * primes stay zero */
static uint64_t* make_switch_key_low(const oc_ctx* c, const uint64_t* s_from, uint32_t key_id) {
    const int N = c->N, P = c->L + c->K, lq = c->low_limbs, kp = c->K_low;
    uint64_t* key = (uint64_t*)calloc((size_t)2 * P * N, sizeof(uint64_t));
    int* e = (int*)malloc(sizeof(int) * (size_t)N);
    for (int n = 0; n < N; n++) e[n] = sample_cbd(c->seed, NONCE_KSK_LOW(key_id, 1), (uint64_t)n);
    uint64_t* b = key;
    uint64_t* a = key + (size_t)P * N;
    int rows[OC_MAXP], nr = 0;
    for (int t = 0; t < lq; t++) rows[nr++] = t;
    for (int k = 0; k < kp; k++) rows[nr++] = c->L + k;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < nr; r++) {
        const int t = rows[r];
        const modulus_t* m = &c->mod[t];
        uint64_t pmod = 1;
        for (int k = 0; k < kp; k++) pmod = mulm(pmod, c->q[c->L + k] % m->q, m);
        uint64_t* en = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)N);
        for (int n = 0; n < N; n++) en[n] = small_to_res(e[n], m->q);
        oc_ntt_fwd(c, t, en);
        for (int n = 0; n < N; n++) {
            size_t o = (size_t)t * N + n;
            uint64_t av = sample_uniform(c->seed, NONCE_KSK_LOW(key_id, 0), o, m);
            a[o] = av;
            uint64_t bv = subm(en[n], mulm(av, c->sk[o], m), m->q);
            if (t < lq) bv = addm(bv, mulm(pmod, s_from[o], m), m->q);
            b[o] = bv;
        }
        free(en);
    }
    free(e);
    return key;
}

void oc_relin_keygen(oc_ctx* c) {
    const int N = c->N, P = c->L + c->K;
    uint64_t* s2 = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)P * N);
    for (int t = 0; t < P; t++)
        for (int n = 0; n < N; n++) {
            size_t o = (size_t)t * N + n;
            s2[o] = mulm(c->sk[o], c->sk[o], &c->mod[t]);
        }
    free(c->rlk);
    c->rlk = make_switch_key(c, s2, KEYID_RELIN);
    if (c->low_limbs) {
        free(c->rlk_low);
        c->rlk_low = make_switch_key_low(c, s2, KEYID_RELIN);
    }
    free(s2);
}

uint32_t oc_galois_element(const oc_ctx* c, int k) {
    const int slots = c->N / 2;
    int r = k % slots;
    if (r < 0) r += slots;
    return c->rot_group[r];
}

/* NTT-domain automorphism: slot k of the output is evaluation point
 * psi^(2 br(k)+1) of a(X^g), i.e. input slot br(((2 br(k)+1) g mod 2N - 1)/2). */
static inline uint32_t auto_index(uint32_t k, uint32_t g, int logN) {
    const uint32_t M = 2u << logN;
    uint32_t e = 2 * bitrev(k, logN) + 1;
    uint32_t eg = (uint32_t)(((uint64_t)e * g) & (M - 1));
    return bitrev((eg - 1) >> 1, logN);
}

void oc_automorphism(const oc_ctx* c, const uint64_t* a, int npolys, int limbs, uint32_t g, uint64_t* out) {
    const int N = c->N;
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)N);
    for (int k = 0; k < N; k++) idx[k] = auto_index((uint32_t)k, g, c->logN);
    for (int p = 0; p < npolys * limbs; p++)
        for (int k = 0; k < N; k++) out[(size_t)p * N + k] = a[(size_t)p * N + idx[k]];
    free(idx);
}

static uint64_t* find_rot_key(const oc_ctx* c, uint32_t g) {
    for (int i = 0; i < c->nrot; i++)
        if (c->rot_g[i] == g) return c->rot_key[i];
    return NULL;
}

/* the switching key of a key switch at `limbs` limbs: rotation g, or the
 * relinearisation key for g == 1 */
static const uint64_t* key_for(const oc_ctx* c, uint32_t g, int limbs) {
    const int low = is_low(c, limbs);
    if (g == 1) return low ? c->rlk_low : c->rlk;
    for (int i = 0; i < c->nrot; i++)
        if (c->rot_g[i] == g) return low ? c->rot_key_low[i] : c->rot_key[i];
    return NULL;
}

int oc_rot_keygen(oc_ctx* c, int k) {
    uint32_t g = oc_galois_element(c, k);
    if (g == 1 || find_rot_key(c, g)) return 0;
    if (c->nrot >= OC_MAXROT) { set_err("too many rotation keys"); return -1; }
    const int N = c->N, P = c->L + c->K;
    uint64_t* sg = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)P * N);
    oc_automorphism(c, c->sk, 1, P, g, sg);
    c->rot_g[c->nrot] = g;
    c->rot_key[c->nrot] = make_switch_key(c, sg, KEYID_ROT(g));
    c->rot_key_low[c->nrot] = c->low_limbs ? make_switch_key_low(c, sg, KEYID_ROT(g)) : NULL;
    c->nrot++;
    free(sg);
    return 0;
}

int oc_switch_key_low(const oc_ctx* c, int k, uint64_t* out) {
    if (!c->low_limbs) { set_err("no reduced special-prime set"); return -1; }
    const uint32_t g = (k == 0) ? 1u : oc_galois_element(c, k);
    const uint64_t* key = key_for(c, g, 1);
    if (!key) { set_err("switch key not generated"); return -1; }
    memcpy(out, key, sizeof(uint64_t) * (size_t)2 * (c->L + c->K) * c->N);
    return 0;
}
int oc_low_limbs(const oc_ctx* c) { return c->low_limbs; }
int oc_K_low(const oc_ctx* c) { return c->K_low; }

int oc_switch_key(const oc_ctx* c, int k, uint64_t* out) {
    const size_t sz = sizeof(uint64_t) * (size_t)c->beta * 2 * (c->L + c->K) * c->N;
    const uint64_t* key = (k == 0) ? c->rlk : find_rot_key(c, oc_galois_element(c, k));
    if (!key) { set_err("switch key not generated"); return -1; }
    memcpy(out, key, sz);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Encrypt / Decrypt (client role, T123.cpp:514-531)                   */
/* ------------------------------------------------------------------ */
void oc_encrypt(const oc_ctx* c, const uint64_t* pt, int limbs, uint64_t counter, uint64_t* ct) {
    const int N = c->N;
    int* u = (int*)malloc(sizeof(int) * (size_t)N);
    int* e0 = (int*)malloc(sizeof(int) * (size_t)N);
    int* e1 = (int*)malloc(sizeof(int) * (size_t)N);
    for (int b = 0; b < N / 8; b++) {
        uint64_t wu[8], w0[8], w1[8];
        chacha_words8(c->seed, NONCE_ENC(counter, 0), (uint64_t)b, wu);
        chacha_words8(c->seed, NONCE_ENC(counter, 1), (uint64_t)b, w0);
        chacha_words8(c->seed, NONCE_ENC(counter, 2), (uint64_t)b, w1);
        for (int k = 0; k < 8; k++) {
            u[8 * b + k] = ternary_of(wu[k]);
            e0[8 * b + k] = cbd_of(w0[k]);
            e1[8 * b + k] = cbd_of(w1[k]);
        }
    }
    int* pr = all_primes(c);
    uint64_t* un = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)limbs * N);
    uint64_t* e0n = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)limbs * N);
    uint64_t* e1n = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)limbs * N);
    small_poly_ntt(c, u, pr, limbs, un);
    small_poly_ntt(c, e0, pr, limbs, e0n);
    small_poly_ntt(c, e1, pr, limbs, e1n);
    const uint64_t *pb = c->pk, *pa = c->pk + (size_t)c->L * N;
    uint64_t *c0 = ct, *c1 = ct + (size_t)limbs * N;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < limbs; l++) {
        const modulus_t* m = &c->mod[l];
        for (int n = 0; n < N; n++) {
            size_t o = (size_t)l * N + n;
            c0[o] = addm(addm(mulm(pb[o], un[o], m), e0n[o], m->q), pt[o], m->q);
            c1[o] = addm(mulm(pa[o], un[o], m), e1n[o], m->q);
        }
    }
    free(u); free(e0); free(e1); free(pr); free(un); free(e0n); free(e1n);
}

void oc_decrypt(const oc_ctx* c, const uint64_t* ct, int limbs, uint64_t* pt) {
    const int N = c->N;
    const uint64_t *c0 = ct, *c1 = ct + (size_t)limbs * N;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < limbs; l++) {
        const modulus_t* m = &c->mod[l];
        for (int n = 0; n < N; n++) {
            size_t o = (size_t)l * N + n;
            pt[o] = addm(c0[o], mulm(c1[o], c->sk[o], m), m->q);
        }
    }
}

/* ------------------------------------------------------------------ */
/* element-wise ops (EvalAdd/EvalSub/EvalMult(ct,pt), T123.cpp:1144-1173) */
/* ------------------------------------------------------------------ */
void oc_add(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int npolys, int limbs, uint64_t* out) {
    const int N = c->N;
    for (int p = 0; p < npolys; p++)
#pragma omp parallel for schedule(static)
        for (int l = 0; l < limbs; l++) {
            uint64_t q = c->q[l];
            size_t base = ((size_t)p * limbs + l) * N;
            for (int n = 0; n < N; n++) out[base + n] = addm(a[base + n], b[base + n], q);
        }
}
void oc_sub(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int npolys, int limbs, uint64_t* out) {
    const int N = c->N;
    for (int p = 0; p < npolys; p++)
#pragma omp parallel for schedule(static)
        for (int l = 0; l < limbs; l++) {
            uint64_t q = c->q[l];
            size_t base = ((size_t)p * limbs + l) * N;
            for (int n = 0; n < N; n++) out[base + n] = subm(a[base + n], b[base + n], q);
        }
}
void oc_mul_pt(const oc_ctx* c, const uint64_t* ct, const uint64_t* pt, int limbs, uint64_t* out) {
    const int N = c->N;
    for (int p = 0; p < 2; p++)
#pragma omp parallel for schedule(static)
        for (int l = 0; l < limbs; l++) {
            size_t base = ((size_t)p * limbs + l) * N;
            for (int n = 0; n < N; n++) out[base + n] = mulm(ct[base + n], pt[(size_t)l * N + n], &c->mod[l]);
        }
}
static uint64_t int_to_res(int64_t k, uint64_t q) {
    uint64_t v = (uint64_t)(k < 0 ? -(k + 1) : k) % q; /* avoid INT64_MIN overflow */
    if (k < 0) { v = (v + 1) % q; v = v ? q - v : 0; }
    return v;
}
void oc_mul_int(const oc_ctx* c, const uint64_t* a, int npolys, int limbs, int64_t k, uint64_t* out) {
    const int N = c->N;
    for (int p = 0; p < npolys; p++)
        for (int l = 0; l < limbs; l++) {
            uint64_t kr = int_to_res(k, c->q[l]);
            size_t base = ((size_t)p * limbs + l) * N;
            for (int n = 0; n < N; n++) out[base + n] = mulm(a[base + n], kr, &c->mod[l]);
        }
}
void oc_add_int(const oc_ctx* c, const uint64_t* ct, int limbs, int64_t k, uint64_t* out) {
    const int N = c->N;
    memcpy(out, ct, sizeof(uint64_t) * 2 * (size_t)limbs * N);
    for (int l = 0; l < limbs; l++) {
        uint64_t kr = int_to_res(k, c->q[l]);
        for (int n = 0; n < N; n++) out[(size_t)l * N + n] = addm(out[(size_t)l * N + n], kr, c->q[l]);
    }
}
/* EvalAdd(ct, double) (T123.cpp:1173): adds round(value*scale) to every slot */
void oc_add_const(const oc_ctx* c, const uint64_t* ct, int limbs, double value, double scale, uint64_t* out) {
    const int N = c->N;
    memcpy(out, ct, sizeof(uint64_t) * 2 * (size_t)limbs * N);
    double r = rint(value * scale);
    for (int l = 0; l < limbs; l++) {
        uint64_t kr = double_to_res(r, &c->mod[l]);
        for (int n = 0; n < N; n++) out[(size_t)l * N + n] = addm(out[(size_t)l * N + n], kr, c->q[l]);
    }
}

void oc_tensor(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int limbs, uint64_t* out3) {
    const int N = c->N;
    const size_t S = (size_t)limbs * N;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < limbs; l++) {
        const modulus_t* m = &c->mod[l];
        for (int n = 0; n < N; n++) {
            size_t o = (size_t)l * N + n;
            uint64_t a0 = a[o], a1 = a[S + o], b0 = b[o], b1 = b[S + o];
            out3[o] = mulm(a0, b0, m);
            out3[S + o] = reduce128((u128)a0 * b1 + (u128)a1 * b0, m);
            out3[2 * S + o] = mulm(a1, b1, m);
        }
    }
}

/* ------------------------------------------------------------------ */
/* hybrid key switching                                                 */
/* ------------------------------------------------------------------ */
/* extended limb t of a level-`limbs` computation -> global prime index */
static inline int ext_prime(const oc_ctx* c, int limbs, int t) { return t < limbs ? t : c->L + (t - limbs); }

/* ModUp of NTT-form d over `limbs` Q limbs: digit j keeps its own limbs
 * and receives the others by approximate basis conversion. */
void oc_modup(const oc_ctx* c, const uint64_t* d, int limbs, uint64_t* ext) {
    const int N = c->N, K = kx(c, limbs), E = limbs + K;
    const int beta = (limbs + c->alpha - 1) / c->alpha;
    uint64_t* dc = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)limbs * N);
    memcpy(dc, d, sizeof(uint64_t) * (size_t)limbs * N);
#pragma omp parallel for schedule(static)
    for (int l = 0; l < limbs; l++) oc_ntt_inv(c, l, dc + (size_t)l * N);
    for (int j = 0; j < beta; j++) {
        const int lo = j * c->alpha, hi = (lo + c->alpha < limbs) ? lo + c->alpha : limbs;
        const int cnt = hi - lo;
        uint64_t hatinv[OC_MAXP];
        for (int i = lo; i < hi; i++) {
            const modulus_t* m = &c->mod[i];
            uint64_t prod = 1;
            for (int i2 = lo; i2 < hi; i2++)
                if (i2 != i) prod = mulm(prod, c->q[i2] % m->q, m);
            hatinv[i - lo] = invm(prod, m->q);
        }
        uint64_t* y = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)cnt * N);
        for (int i = lo; i < hi; i++)
            for (int n = 0; n < N; n++)
                y[(size_t)(i - lo) * N + n] = mulm(dc[(size_t)i * N + n], hatinv[i - lo], &c->mod[i]);
        uint64_t* ej = ext + (size_t)j * E * N;
#pragma omp parallel for schedule(dynamic)
        for (int t = 0; t < E; t++) {
            uint64_t* o = ej + (size_t)t * N;
            if (t >= lo && t < hi) {
                memcpy(o, d + (size_t)t * N, sizeof(uint64_t) * N);
                continue;
            }
            const int pt = ext_prime(c, limbs, t);
            const modulus_t* m = &c->mod[pt];
            uint64_t hat[OC_MAXP];
            for (int i = lo; i < hi; i++) {
                uint64_t prod = 1;
                for (int i2 = lo; i2 < hi; i2++)
                    if (i2 != i) prod = mulm(prod, c->q[i2] % m->q, m);
                hat[i - lo] = prod;
            }
            for (int n = 0; n < N; n++) {
                u128 acc = 0;
                for (int i = 0; i < cnt; i++) acc += (u128)y[(size_t)i * N + n] * hat[i];
                o[n] = reduce128(acc, m);
            }
            oc_ntt_fwd(c, pt, o);
        }
        free(y);
    }
    free(dc);
}

/* ModDown: x over limbs+K extended limbs (NTT form) -> limbs Q limbs of
 * (x - conv_{P->Q}(x mod P)) * P^{-1}. */
void oc_moddown(const oc_ctx* c, const uint64_t* x, int limbs, uint64_t* out) {
    const int N = c->N, K = kx(c, limbs), L = c->L;
    uint64_t* xp = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)K * N);
    memcpy(xp, x + (size_t)limbs * N, sizeof(uint64_t) * (size_t)K * N);
#pragma omp parallel for schedule(static)
    for (int k = 0; k < K; k++) {
        oc_ntt_inv(c, L + k, xp + (size_t)k * N);
        const modulus_t* m = &c->mod[L + k];
        uint64_t prod = 1;
        for (int k2 = 0; k2 < K; k2++)
            if (k2 != k) prod = mulm(prod, c->q[L + k2] % m->q, m);
        uint64_t hinv = invm(prod, m->q);
        for (int n = 0; n < N; n++) xp[(size_t)k * N + n] = mulm(xp[(size_t)k * N + n], hinv, m);
    }
#pragma omp parallel for schedule(dynamic)
    for (int t = 0; t < limbs; t++) {
        const modulus_t* m = &c->mod[t];
        uint64_t hat[OC_MAXP];
        uint64_t pinv = 1;
        for (int k = 0; k < K; k++) {
            uint64_t prod = 1;
            for (int k2 = 0; k2 < K; k2++)
                if (k2 != k) prod = mulm(prod, c->q[L + k2] % m->q, m);
            hat[k] = prod;
            pinv = mulm(pinv, c->q[L + k] % m->q, m);
        }
        pinv = invm(pinv, m->q);
        uint64_t* conv = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)N);
        for (int n = 0; n < N; n++) {
            u128 acc = 0;
            for (int k = 0; k < K; k++) acc += (u128)xp[(size_t)k * N + n] * hat[k];
            conv[n] = reduce128(acc, m);
        }
        oc_ntt_fwd(c, t, conv);
        for (int n = 0; n < N; n++)
            out[(size_t)t * N + n] = mulm(subm(x[(size_t)t * N + n], conv[n], m->q), pinv, m);
        free(conv);
    }
    free(xp);
}

/* inner product of the ModUp digits (optionally permuted by the NTT-domain
 * automorphism g) with a switching key; acc: 2 x (limbs+K) limbs */
static void ks_inner(const oc_ctx* c, const uint64_t* ext, int limbs, const uint64_t* key, uint32_t g,
                     uint64_t* acc) {
    const int N = c->N, E = limbs + kx(c, limbs), P = c->L + c->K;
    const int beta = (limbs + c->alpha - 1) / c->alpha;
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)N);
    for (int k = 0; k < N; k++) idx[k] = (g == 1) ? (uint32_t)k : auto_index((uint32_t)k, g, c->logN);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < E; t++) {
        const int pt = ext_prime(c, limbs, t);
        const modulus_t* m = &c->mod[pt];
        for (int n = 0; n < N; n++) {
            u128 s0 = 0, s1 = 0;
            for (int j = 0; j < beta; j++) {
                uint64_t v = ext[((size_t)j * E + t) * N + idx[n]];
                const uint64_t* kb = key + ((size_t)j * 2 * P + pt) * N;
                const uint64_t* ka = key + ((size_t)j * 2 * P + P + pt) * N;
                s0 += (u128)v * kb[n];
                s1 += (u128)v * ka[n];
            }
            acc[(size_t)t * N + n] = reduce128(s0, m);
            acc[((size_t)E + t) * N + n] = reduce128(s1, m);
        }
    }
    free(idx);
}

void oc_keyswitch(const oc_ctx* c, const uint64_t* d, int limbs, const uint64_t* ksk, uint64_t* out) {
    const int N = c->N, E = limbs + kx(c, limbs);
    const int beta = (limbs + c->alpha - 1) / c->alpha;
    uint64_t* ext = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)beta * E * N);
    uint64_t* acc = (uint64_t*)malloc(sizeof(uint64_t) * 2 * (size_t)E * N);
    oc_modup(c, d, limbs, ext);
    ks_inner(c, ext, limbs, ksk, 1, acc);
    oc_moddown(c, acc, limbs, out);
    oc_moddown(c, acc + (size_t)E * N, limbs, out + (size_t)limbs * N);
    free(ext);
    free(acc);
}

/* EvalMult(ct, ct) = tensor + relinearisation of d2 (T123.cpp:1144-1147) */
int oc_mul_ct(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int limbs, uint64_t* out) {
    const uint64_t* rlk = key_for(c, 1, limbs);
    if (!rlk) { set_err("relinearisation key not generated"); return -1; }
    const int N = c->N;
    const size_t S = (size_t)limbs * N;
    uint64_t* d = (uint64_t*)malloc(sizeof(uint64_t) * 3 * S);
    uint64_t* ks = (uint64_t*)malloc(sizeof(uint64_t) * 2 * S);
    oc_tensor(c, a, b, limbs, d);
    oc_keyswitch(c, d + 2 * S, limbs, rlk, ks);
    oc_add(c, d, ks, 2, limbs, out);
    free(d);
    free(ks);
    return 0;
}

/* sum_r EvalMult(a_r, b_r) with one relinearisation: the tensor products are
 * summed as degree-2 ciphertexts and d2 is key-switched once (the context
 * accumulation of T123.cpp:838-860).  a, b: n x 2 x limbs x N. */
int oc_mul_ct_sum(const oc_ctx* c, const uint64_t* a, const uint64_t* b, int n, int limbs, uint64_t* out) {
    const uint64_t* rlk = key_for(c, 1, limbs);
    if (!rlk) { set_err("relinearisation key not generated"); return -1; }
    const int N = c->N;
    const size_t S = (size_t)limbs * N;
    uint64_t* d = (uint64_t*)calloc(3 * S, sizeof(uint64_t));
    uint64_t* t = (uint64_t*)malloc(sizeof(uint64_t) * 3 * S);
    uint64_t* ks = (uint64_t*)malloc(sizeof(uint64_t) * 2 * S);
    for (int r = 0; r < n; r++) {
        oc_tensor(c, a + (size_t)r * 2 * S, b + (size_t)r * 2 * S, limbs, t);
        oc_add(c, d, t, 3, limbs, d);
    }
    oc_keyswitch(c, d + 2 * S, limbs, rlk, ks);
    oc_add(c, d, ks, 2, limbs, out);
    free(d); free(t); free(ks);
    return 0;
}

/* Rescale (FLEXIBLEAUTO, T123.cpp:1608): x -> (x - [x]_{q_last}) / q_last */
void oc_rescale(const oc_ctx* c, const uint64_t* ct, int limbs, uint64_t* out) {
    const int N = c->N, lo = limbs - 1;
    for (int p = 0; p < 2; p++) {
        const uint64_t* x = ct + (size_t)p * limbs * N;
        uint64_t* o = out + (size_t)p * lo * N;
        uint64_t* last = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)N);
        memcpy(last, x + (size_t)lo * N, sizeof(uint64_t) * N);
        oc_ntt_inv(c, lo, last);
        const uint64_t ql = c->q[lo];
#pragma omp parallel for schedule(static)
        for (int i = 0; i < lo; i++) {
            const modulus_t* m = &c->mod[i];
            uint64_t* t = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)N);
            for (int n = 0; n < N; n++) t[n] = last[n] % m->q;
            oc_ntt_fwd(c, i, t);
            uint64_t inv = invm(ql % m->q, m->q);
            for (int n = 0; n < N; n++) o[(size_t)i * N + n] = mulm(subm(x[(size_t)i * N + n], t[n], m->q), inv, m);
            free(t);
        }
        free(last);
    }
}

/* EvalFastRotation (T123.cpp:1183-1203, 1343-1362): one ModUp of c1 shared by
 * every rotation; each rotation permutes the digits, takes the inner product
 * with its key, runs ModDown and adds the permuted c0.  EvalRotate is the
 * single-index case. */
int oc_rotate_hoisted(const oc_ctx* c, const uint64_t* ct, int limbs, const int* ks, int n, uint64_t* out) {
    const int N = c->N, E = limbs + kx(c, limbs);
    const int beta = (limbs + c->alpha - 1) / c->alpha;
    const size_t S = (size_t)limbs * N;
    for (int r = 0; r < n; r++) {
        uint32_t g = oc_galois_element(c, ks[r]);
        if (g != 1 && !key_for(c, g, limbs)) { set_err("rotation key not generated"); return -1; }
    }
    uint64_t* ext = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)beta * E * N);
    uint64_t* acc = (uint64_t*)malloc(sizeof(uint64_t) * 2 * (size_t)E * N);
    uint64_t* tmp = (uint64_t*)malloc(sizeof(uint64_t) * 2 * S);
    oc_modup(c, ct + S, limbs, ext);
    for (int r = 0; r < n; r++) {
        uint64_t* o = out + (size_t)r * 2 * S;
        uint32_t g = oc_galois_element(c, ks[r]);
        if (g == 1) { memcpy(o, ct, sizeof(uint64_t) * 2 * S); continue; }
        ks_inner(c, ext, limbs, key_for(c, g, limbs), g, acc);
        oc_moddown(c, acc, limbs, tmp);
        oc_moddown(c, acc + (size_t)E * N, limbs, tmp + S);
        oc_automorphism(c, ct, 1, limbs, g, o);
        oc_add(c, o, tmp, 1, limbs, o);
        memcpy(o + S, tmp + S, sizeof(uint64_t) * S);
    }
    free(ext); free(acc); free(tmp);
    return 0;
}

int oc_rotate(const oc_ctx* c, const uint64_t* ct, int limbs, int k, uint64_t* out) {
    return oc_rotate_hoisted(c, ct, limbs, &k, 1, out);
}

/* sum_r rot(ct_r, k_r), the giant-step sum of a BSGS product (T123.cpp:
 * 1283-1291), with the key switches of each group of up to 32 non-identity
 * rotations (in input order) added in the extended basis and one ModDown per
 * group; identity rotations are added as is.  cts: n x 2 x limbs x N. */
int oc_rotate_sum(const oc_ctx* c, const uint64_t* cts, int limbs, const int* ks, int n, uint64_t* out) {
    const int N = c->N, E = limbs + kx(c, limbs);
    const int beta = (limbs + c->alpha - 1) / c->alpha;
    const size_t S = (size_t)limbs * N;
    for (int r = 0; r < n; r++) {
        uint32_t g = oc_galois_element(c, ks[r]);
        if (g != 1 && !key_for(c, g, limbs)) { set_err("rotation key not generated"); return -1; }
    }
    uint64_t* ext = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)beta * E * N);
    uint64_t* acc = (uint64_t*)malloc(sizeof(uint64_t) * 2 * (size_t)E * N);
    uint64_t* accsum = (uint64_t*)malloc(sizeof(uint64_t) * 2 * (size_t)E * N);
    uint64_t* tmp = (uint64_t*)malloc(sizeof(uint64_t) * 2 * S);
    memset(out, 0, sizeof(uint64_t) * 2 * S);
    int in_group = 0;
    for (int r = 0; r <= n; r++) {
        const int last = (r == n);
        uint32_t g = last ? 0 : oc_galois_element(c, ks[r]);
        if (last || in_group == 32) {
            if (in_group) {  /* close the group: one ModDown of the summed products */
                oc_moddown(c, accsum, limbs, tmp);
                oc_moddown(c, accsum + (size_t)E * N, limbs, tmp + S);
                oc_add(c, out, tmp, 2, limbs, out);
            }
            in_group = 0;
            if (last) break;
        }
        const uint64_t* ct = cts + (size_t)r * 2 * S;
        if (g == 1) {
            oc_add(c, out, ct, 2, limbs, out);
            continue;
        }
        if (in_group == 0) memset(accsum, 0, sizeof(uint64_t) * 2 * (size_t)E * N);
        oc_modup(c, ct + S, limbs, ext);
        ks_inner(c, ext, limbs, key_for(c, g, limbs), g, acc);
        for (int p = 0; p < 2; p++)
            for (int t = 0; t < E; t++) {
                const uint64_t q = c->q[ext_prime(c, limbs, t)];
                uint64_t* a = accsum + ((size_t)p * E + t) * N;
                const uint64_t* b = acc + ((size_t)p * E + t) * N;
                for (int k = 0; k < N; k++) a[k] = addm(a[k], b[k], q);
            }
        oc_automorphism(c, ct, 1, limbs, g, tmp);
        oc_add(c, out, tmp, 1, limbs, out);
        in_group++;
    }
    free(ext); free(acc); free(accsum); free(tmp);
    return 0;
}

/* sum_{j < window} rot(ct, j * stride) by the AccumulateSum ladder with each
 * step's rotations {0, s, 2s, 3s} * stride summed as one rotation sum (the
 * key switches added in the extended basis, one ModDown per step) -- the
 * engine's hoisted window sums. */
int oc_window_sum(const oc_ctx* c, const uint64_t* ct, int limbs, int window, int stride, uint64_t* out) {
    return oc_window_sum_radix(c, ct, limbs, window, stride, 4, out);
}

/* the same with a base-r ladder: step s sums the rotations by
 * stride * s * {0 .. r-1} below the window as one rotation sum */
int oc_window_sum_radix(const oc_ctx* c, const uint64_t* ct, int limbs, int window, int stride, int radix,
                        uint64_t* out) {
    if (radix < 2 || radix > 33) { set_err("radix must be 2..33"); return -1; }
    const size_t S2 = 2 * (size_t)limbs * c->N;
    memcpy(out, ct, sizeof(uint64_t) * S2);
    uint64_t* rep = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)radix * S2);
    int* ks = (int*)malloc(sizeof(int) * (size_t)radix);
    for (long step = 1; step < window; step *= radix) {
        int n = 1;
        ks[0] = 0;
        for (int m = 1; m < radix && step * m < window; m++) ks[n++] = (int)(stride * step * m);
        for (int r = 0; r < n; r++) memcpy(rep + (size_t)r * S2, out, sizeof(uint64_t) * S2);
        if (oc_rotate_sum(c, rep, limbs, ks, n, out)) { free(rep); free(ks); return -1; }
    }
    free(rep);
    free(ks);
    return 0;
}

/* AccumulateSum(ct, count, stride) (T123.cpp:1154-1159, keys :444-453):
 * base-4 ladder; at step s the hoisted rotations by stride*s*{1,2,3}
 * (those with s*m < count) are added to the running sum. */
int oc_accumulate_sum(const oc_ctx* c, const uint64_t* ct, int limbs, int count, int stride, uint64_t* out) {
    const size_t S2 = 2 * (size_t)limbs * c->N;
    memcpy(out, ct, sizeof(uint64_t) * S2);
    uint64_t* rot = (uint64_t*)malloc(sizeof(uint64_t) * 3 * S2);
    for (long step = 1; step < count; step *= 4) {
        int ks[3], n = 0;
        for (int m = 1; m < 4 && step * m < count; m++) ks[n++] = (int)(stride * step * m);
        if (oc_rotate_hoisted(c, out, limbs, ks, n, rot)) { free(rot); return -1; }
        for (int r = 0; r < n; r++) oc_add(c, out, rot + (size_t)r * S2, 2, limbs, out);
    }
    free(rot);
    return 0;
}

/* Inner sums of the Halevi-Shoup product matmul(BabyRotations, W)
 * (T123.cpp:1264-1295, the loop over `small`): for every giant step g < n2,
 * out[g] (+)= sum_{j < n1} diag[g * n1 + j] * baby[j], both polynomials.
 * babies: n1 x 2 x limbs x N; diags: (n1 * n2) x limbs x N plaintexts;
 * out: n2 x 2 x limbs x N, added to when `accumulate` (a sum of products
 * whose giant steps run once).  Each output residue is the exact sum
 * reduced once (products below 2^120, at most 32 of them). */
int oc_bsgs_inner(const oc_ctx* c, const uint64_t* babies, int n1, const uint64_t* diags, int n2, int limbs,
                  int accumulate, uint64_t* out) {
    if (n1 <= 0 || n1 > 64 || n2 <= 0) { set_err("bsgs: n1 in 1..64, n2 > 0"); return -1; }
    const int N = c->N;
    const size_t S = (size_t)limbs * N;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int g = 0; g < n2; g++)
        for (int l = 0; l < limbs; l++) {
            const modulus_t* m = &c->mod[l];
            for (int p = 0; p < 2; p++) {
                uint64_t* o = out + (size_t)g * 2 * S + (size_t)p * S + (size_t)l * N;
                for (int n = 0; n < N; n++) {
                    u128 acc = 0;
                    for (int j = 0; j < n1; j++) {
                        const uint64_t b = babies[(size_t)j * 2 * S + (size_t)p * S + (size_t)l * N + n];
                        const uint64_t d = diags[((size_t)g * n1 + j) * S + (size_t)l * N + n];
                        acc += (u128)b * d;
                    }
                    const uint64_t r = reduce128(acc, m);
                    o[n] = accumulate ? addm(o[n], r, m->q) : r;
                }
            }
        }
    return 0;
}
