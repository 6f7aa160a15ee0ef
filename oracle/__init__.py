"""ctypes front-end of the CPU RNS-CKKS oracle (``ckks_oracle.c``).

TEST INFRASTRUCTURE ONLY.  ``tests/``, ``__graft_entry__.smoke()`` and the
bench's CPU-baseline / reference arm import this module as the checker and as
the timed CPU path; nothing in ``private_genomic_dnagpt_b200`` imports it.

Arrays are numpy uint64 in the layout documented in ``ckks_oracle.h``:
a polynomial is ``(limbs, N)``, a ciphertext ``(2, limbs, N)``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libckks_oracle.so")

_u64p = ctypes.POINTER(ctypes.c_uint64)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int)


def build() -> str:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oc_create.restype = ctypes.c_void_p
        L.oc_create.argtypes = [ctypes.c_int] * 6 + [ctypes.c_uint64]
        L.oc_destroy.argtypes = [ctypes.c_void_p]
        for name in ("oc_N", "oc_L", "oc_K", "oc_alpha", "oc_low_limbs", "oc_K_low"):
            getattr(L, name).argtypes = [ctypes.c_void_p]
            getattr(L, name).restype = ctypes.c_int
        L.oc_scale.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oc_scale.restype = ctypes.c_double
        L.oc_galois_element.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oc_galois_element.restype = ctypes.c_uint32
        L.oc_last_error.restype = ctypes.c_char_p
        L.oc_chacha_words.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _u64p]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    if a.dtype == np.uint64:
        return a.ctypes.data_as(_u64p)
    if a.dtype == np.float64:
        return a.ctypes.data_as(_f64p)
    if a.dtype == np.int32:
        return a.ctypes.data_as(_i32p)
    raise TypeError(a.dtype)


class OracleError(RuntimeError):
    pass


def diagonal_slots(W: np.ndarray, batch: int, pack_width: int, n1: int, g: int, j: int) -> np.ndarray:
    """Slot values of BSGS diagonal g * n1 + j of W ([out, in]) on the layout
    slot(feature f, lane t) = f * batch + t: the diagonal pre-rotated by the
    giant step, W[rolled][(rolled + n1 g + j) mod PW] at feature f with
    rolled = (f - n1 g) mod PW, zero outside W, the same on every lane
    (cached_diagonal_plains, T123.cpp:1018-1046)."""
    out_dim, in_dim = W.shape
    f = np.arange(pack_width)
    rolled = (f - n1 * g) % pack_width
    col = (rolled + n1 * g + j) % pack_width
    inside = (rolled < out_dim) & (col < in_dim)
    v = np.where(inside, W[np.minimum(rolled, out_dim - 1), np.minimum(col, in_dim - 1)], 0.0)
    return np.repeat(v, batch)


def lane_mask_slots(batch: int, pack_width: int, delta: int, no_wrap: bool) -> np.ndarray:
    """lane_mask_plain(delta, no_wrap) (T123.cpp:1076-1093): 1 on the lanes
    t < batch - delta (no_wrap) or t >= batch - delta (not no_wrap) of every
    feature."""
    t = np.arange(batch)
    lane = ((t < batch - delta) == no_wrap).astype(np.float64)
    return np.tile(lane, pack_width)


class Oracle:
    """One CPU CKKS context: parameters, tables and (after keygen) keys."""

    def __init__(self, logN=10, L=6, dnum=3, first_bits=60, scale_bits=50,
                 special_bits=60, seed=1, threads=0):
        self.L_ = lib()
        if threads:
            self.L_.oc_set_threads(int(threads))
        self.h = self.L_.oc_create(logN, L, dnum, first_bits, scale_bits, special_bits,
                                   ctypes.c_uint64(seed))
        if not self.h:
            raise OracleError(self.L_.oc_last_error().decode())
        self.logN = logN
        self.N = self.L_.oc_N(self.h)
        self.L = self.L_.oc_L(self.h)
        self.K = self.L_.oc_K(self.h)
        self.alpha = self.L_.oc_alpha(self.h)
        self.dnum = dnum
        self.beta = -(-self.L // self.alpha)
        self.seed = seed
        # one-digit key switches at <= low_limbs limbs use keys over the first
        # K_low special primes (0: no such set)
        self.low_limbs = self.L_.oc_low_limbs(self.h)
        self.K_low = self.L_.oc_K_low(self.h)
        q = np.zeros(self.L + self.K, np.uint64)
        self.L_.oc_moduli(ctypes.c_void_p(self.h), _p(q))
        self.moduli = q
        psi = np.zeros(self.L + self.K, np.uint64)
        self.L_.oc_psi(ctypes.c_void_p(self.h), _p(psi))
        self.psi = psi

    def __del__(self):
        try:
            if self.h:
                self.L_.oc_destroy(ctypes.c_void_p(self.h))
                self.h = None
        except Exception:
            pass

    # -- helpers ---------------------------------------------------------
    def _c(self):
        return ctypes.c_void_p(self.h)

    def _check(self, rc):
        if rc != 0:
            raise OracleError(self.L_.oc_last_error().decode())

    def scale(self, limbs: int) -> float:
        return self.L_.oc_scale(self._c(), limbs)

    def galois(self, k: int) -> int:
        return int(self.L_.oc_galois_element(self._c(), k))

    # -- NTT -------------------------------------------------------------
    def ntt(self, a: np.ndarray, prime_index: int) -> np.ndarray:
        a = np.ascontiguousarray(a, np.uint64).copy()
        self.L_.oc_ntt_fwd(self._c(), prime_index, _p(a))
        return a

    def intt(self, a: np.ndarray, prime_index: int) -> np.ndarray:
        a = np.ascontiguousarray(a, np.uint64).copy()
        self.L_.oc_ntt_inv(self._c(), prime_index, _p(a))
        return a

    # -- encode / decode -------------------------------------------------
    def encode(self, values, limbs: int, scale: float | None = None) -> np.ndarray:
        v = np.ascontiguousarray(values, np.float64)
        assert v.shape == (self.N // 2,)
        out = np.zeros((limbs, self.N), np.uint64)
        sc = self.scale(limbs) if scale is None else scale
        self._check(self.L_.oc_encode(self._c(), _p(v), limbs, ctypes.c_double(sc), _p(out)))
        return out

    def encode_batch(self, values: np.ndarray, limbs: int, scale: float, out: np.ndarray | None = None):
        """Encodings of the rows of `values` (count x N/2) at `limbs` limbs,
        computed in parallel; writes into `out` (count x limbs x N) if given."""
        v = np.ascontiguousarray(values, np.float64)
        count = v.shape[0]
        if out is None:
            out = np.zeros((count, limbs, self.N), np.uint64)
        assert out.flags["C_CONTIGUOUS"] and out.shape == (count, limbs, self.N)
        self._check(self.L_.oc_encode_batch(self._c(), _p(v), count, limbs, ctypes.c_double(scale), _p(out)))
        return out

    def decode(self, pt: np.ndarray, scale: float) -> np.ndarray:
        pt = np.ascontiguousarray(pt, np.uint64)
        out = np.zeros(self.N // 2, np.float64)
        self.L_.oc_decode(self._c(), _p(pt), pt.shape[0], ctypes.c_double(scale), _p(out))
        return out

    # -- keys --------------------------------------------------------------
    def keygen(self):
        self.L_.oc_keygen(self._c())

    def relin_keygen(self):
        self.L_.oc_relin_keygen(self._c())

    def rot_keygen(self, ks):
        for k in ks:
            self._check(self.L_.oc_rot_keygen(self._c(), int(k)))

    def secret_key(self) -> np.ndarray:
        out = np.zeros((self.L + self.K, self.N), np.uint64)
        self.L_.oc_secret_key(self._c(), _p(out))
        return out

    def public_key(self) -> np.ndarray:
        out = np.zeros((2, self.L, self.N), np.uint64)
        self.L_.oc_public_key(self._c(), _p(out))
        return out

    def switch_key(self, k: int) -> np.ndarray:
        out = np.zeros((self.beta, 2, self.L + self.K, self.N), np.uint64)
        self._check(self.L_.oc_switch_key(self._c(), int(k), _p(out)))
        return out

    def switch_key_low(self, k: int) -> np.ndarray:
        out = np.zeros((2, self.L + self.K, self.N), np.uint64)
        self._check(self.L_.oc_switch_key_low(self._c(), int(k), _p(out)))
        return out

    # -- client ------------------------------------------------------------
    def encrypt(self, pt: np.ndarray, counter: int) -> np.ndarray:
        pt = np.ascontiguousarray(pt, np.uint64)
        limbs = pt.shape[0]
        ct = np.zeros((2, limbs, self.N), np.uint64)
        self.L_.oc_encrypt(self._c(), _p(pt), limbs, ctypes.c_uint64(counter), _p(ct))
        return ct

    def decrypt(self, ct: np.ndarray) -> np.ndarray:
        ct = np.ascontiguousarray(ct, np.uint64)
        limbs = ct.shape[1]
        pt = np.zeros((limbs, self.N), np.uint64)
        self.L_.oc_decrypt(self._c(), _p(ct), limbs, _p(pt))
        return pt

    # -- evaluation --------------------------------------------------------
    def add(self, a, b):
        a = np.ascontiguousarray(a, np.uint64); b = np.ascontiguousarray(b, np.uint64)
        out = np.empty_like(a)
        npolys = a.shape[0] if a.ndim == 3 else 1
        self.L_.oc_add(self._c(), _p(a), _p(b), npolys, a.shape[-2], _p(out))
        return out

    def sub(self, a, b):
        a = np.ascontiguousarray(a, np.uint64); b = np.ascontiguousarray(b, np.uint64)
        out = np.empty_like(a)
        npolys = a.shape[0] if a.ndim == 3 else 1
        self.L_.oc_sub(self._c(), _p(a), _p(b), npolys, a.shape[-2], _p(out))
        return out

    def mul_pt(self, ct, pt):
        ct = np.ascontiguousarray(ct, np.uint64); pt = np.ascontiguousarray(pt, np.uint64)
        out = np.empty_like(ct)
        self.L_.oc_mul_pt(self._c(), _p(ct), _p(pt), ct.shape[1], _p(out))
        return out

    def mul_int(self, a, k: int):
        a = np.ascontiguousarray(a, np.uint64)
        out = np.empty_like(a)
        npolys = a.shape[0] if a.ndim == 3 else 1
        self.L_.oc_mul_int(self._c(), _p(a), npolys, a.shape[-2], ctypes.c_int64(k), _p(out))
        return out

    def add_const(self, ct, value: float, scale: float):
        ct = np.ascontiguousarray(ct, np.uint64)
        out = np.empty_like(ct)
        self.L_.oc_add_const(self._c(), _p(ct), ct.shape[1], ctypes.c_double(value),
                             ctypes.c_double(scale), _p(out))
        return out

    def tensor(self, a, b):
        a = np.ascontiguousarray(a, np.uint64); b = np.ascontiguousarray(b, np.uint64)
        out = np.zeros((3,) + a.shape[1:], np.uint64)
        self.L_.oc_tensor(self._c(), _p(a), _p(b), a.shape[1], _p(out))
        return out

    def mul_ct(self, a, b):
        a = np.ascontiguousarray(a, np.uint64); b = np.ascontiguousarray(b, np.uint64)
        out = np.empty_like(a)
        self._check(self.L_.oc_mul_ct(self._c(), _p(a), _p(b), a.shape[1], _p(out)))
        return out

    def keyswitch(self, d, ksk):
        d = np.ascontiguousarray(d, np.uint64); ksk = np.ascontiguousarray(ksk, np.uint64)
        limbs = d.shape[0]
        out = np.zeros((2, limbs, self.N), np.uint64)
        self.L_.oc_keyswitch(self._c(), _p(d), limbs, _p(ksk), _p(out))
        return out

    def modup(self, d):
        d = np.ascontiguousarray(d, np.uint64)
        limbs = d.shape[0]
        beta = -(-limbs // self.alpha)
        out = np.zeros((beta, limbs + self.K, self.N), np.uint64)
        self.L_.oc_modup(self._c(), _p(d), limbs, _p(out))
        return out

    def moddown(self, x):
        x = np.ascontiguousarray(x, np.uint64)
        limbs = x.shape[0] - self.K
        out = np.zeros((limbs, self.N), np.uint64)
        self.L_.oc_moddown(self._c(), _p(x), limbs, _p(out))
        return out

    def rescale(self, ct):
        ct = np.ascontiguousarray(ct, np.uint64)
        limbs = ct.shape[1]
        out = np.zeros((2, limbs - 1, self.N), np.uint64)
        self.L_.oc_rescale(self._c(), _p(ct), limbs, _p(out))
        return out

    def automorphism(self, a, g: int):
        a = np.ascontiguousarray(a, np.uint64)
        out = np.empty_like(a)
        npolys = a.shape[0] if a.ndim == 3 else 1
        self.L_.oc_automorphism(self._c(), _p(a), npolys, a.shape[-2], ctypes.c_uint32(g), _p(out))
        return out

    def rotate(self, ct, k: int):
        ct = np.ascontiguousarray(ct, np.uint64)
        out = np.empty_like(ct)
        self._check(self.L_.oc_rotate(self._c(), _p(ct), ct.shape[1], int(k), _p(out)))
        return out

    def rotate_hoisted(self, ct, ks):
        ct = np.ascontiguousarray(ct, np.uint64)
        kk = np.ascontiguousarray(ks, np.int32)
        out = np.zeros((len(kk),) + ct.shape, np.uint64)
        self._check(self.L_.oc_rotate_hoisted(self._c(), _p(ct), ct.shape[1], _p(kk), len(kk), _p(out)))
        return out

    def mul_ct_sum(self, a, b):
        a = np.ascontiguousarray(a, np.uint64)  # n x 2 x limbs x N
        b = np.ascontiguousarray(b, np.uint64)
        out = np.zeros(a.shape[1:], np.uint64)
        self._check(self.L_.oc_mul_ct_sum(self._c(), _p(a), _p(b), a.shape[0], a.shape[2], _p(out)))
        return out

    def rotate_sum(self, cts, ks):
        cts = np.ascontiguousarray(cts, np.uint64)  # n x 2 x limbs x N
        kk = np.ascontiguousarray(ks, np.int32)
        out = np.zeros(cts.shape[1:], np.uint64)
        self._check(self.L_.oc_rotate_sum(self._c(), _p(cts), cts.shape[2], _p(kk), len(kk), _p(out)))
        return out

    def window_sum(self, ct, window: int, stride: int, radix: int = 4):
        ct = np.ascontiguousarray(ct, np.uint64)
        out = np.empty_like(ct)
        self._check(self.L_.oc_window_sum_radix(self._c(), _p(ct), ct.shape[1], window, stride, radix, _p(out)))
        return out

    def accumulate_sum(self, ct, count: int, stride: int):
        ct = np.ascontiguousarray(ct, np.uint64)
        out = np.empty_like(ct)
        self._check(self.L_.oc_accumulate_sum(self._c(), _p(ct), ct.shape[1], count, stride, _p(out)))
        return out

    # -- block-driver compositions (T123.cpp:1005-1059, 1264-1314) ---------
    def bsgs_diagonals(self, W: np.ndarray, batch: int, n1: int, limbs: int) -> np.ndarray:
        """cached_diagonal_plains(W, level): every diagonal of the n1 x n2
        BSGS split encoded at `limbs` limbs and that level's scale,
        (n1 * n2, limbs, N)."""
        pw = self.N // 2 // batch
        nd = pw
        out = np.zeros((nd, limbs, self.N), np.uint64)
        for d0 in range(0, nd, 64):
            vals = np.stack([diagonal_slots(W, batch, pw, n1, d // n1, d % n1) for d in range(d0, min(nd, d0 + 64))])
            self.encode_batch(vals, limbs, self.scale(limbs), out[d0:d0 + len(vals)])
        return out

    def bsgs_inner(self, babies: np.ndarray, diags: np.ndarray, n1: int, out: np.ndarray | None = None):
        """out[g] (+)= sum_j diags[g n1 + j] * babies[j] (adds to `out` when
        given); babies (n1, 2, limbs, N), diags (n1 n2, limbs, N)."""
        babies = np.ascontiguousarray(babies, np.uint64)
        diags = np.ascontiguousarray(diags, np.uint64)
        n2 = diags.shape[0] // n1
        limbs = babies.shape[2]
        acc = out is not None
        if out is None:
            out = np.zeros((n2, 2, limbs, self.N), np.uint64)
        assert out.flags["C_CONTIGUOUS"] and out.dtype == np.uint64
        self._check(self.L_.oc_bsgs_inner(self._c(), _p(babies), n1, _p(diags), n2, limbs, int(acc), _p(out)))
        return out

    def bsgs_matmul(self, diags_terms, babies_terms, n1: int, batch: int):
        """matmul(BabyRotations, W) (T123.cpp:1264-1295) summed over matrix
        terms: for each group q, Rescale(sum_g rot(sum_t sum_j
        diag_t[g n1 + j] * babies_t[q][j], batch n1 g)), the giant steps as
        one rotation sum (one ModDown per 32 rotations, oc_rotate_sum)."""
        G = len(babies_terms[0])
        n2 = diags_terms[0].shape[0] // n1
        ks = [batch * n1 * g for g in range(n2)]
        outs = []
        for q in range(G):
            inner = None
            for t, diags in enumerate(diags_terms):
                inner = self.bsgs_inner(np.stack(babies_terms[t][q]), diags, n1, inner)
            outs.append(self.rescale(self.rotate_sum(inner, ks)))
        return outs

    def lane_shift(self, ct, delta: int, batch: int):
        """lane_shift(x, delta) (T123.cpp:1297-1314): rot(x, d) masked to
        the lanes t < batch - d plus rot(x, d - batch) masked to the others,
        rescaled; the two rotations share one ModUp (EvalFastRotation)."""
        limbs = ct.shape[1]
        pw = self.N // 2 // batch
        r = self.rotate_hoisted(ct, [delta, delta - batch])
        sc = self.scale(limbs)
        lo = self.mul_pt(r[0], self.encode(lane_mask_slots(batch, pw, delta, True), limbs, sc))
        hi = self.mul_pt(r[1], self.encode(lane_mask_slots(batch, pw, delta, False), limbs, sc))
        return self.rescale(self.add(lo, hi))

    @staticmethod
    def chacha(seed: int, nonce: int, counter: int):
        out = np.zeros(2, np.uint64)
        lib().oc_chacha_words(ctypes.c_uint64(seed), ctypes.c_uint64(nonce), ctypes.c_uint64(counter), _p(out))
        return out
