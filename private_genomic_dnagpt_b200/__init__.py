"""B200-native CKKS evaluation engine for the encrypted DNAGPT block hot path.

The compute path is ``libckks_b200.so`` (hand-written sm_100a CUDA behind the C
ABI in ``include/ckks_b200.h``).  This module binds that ABI with ctypes and
mirrors, for Python callers and tests, the OpenFHE-compatible surface the
reference block driver programs against
(fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_depth13_
digits3_ring65536_cpudiagcache_t123.cpp, "T123.cpp"):

    cc = GenCryptoContext(CCParams(...))          # T123.cpp:1602-1621
    cc.KeyGen(); cc.EvalMultKeyGen(); cc.EvalRotateKeyGen(idx)
    pt = cc.MakeCKKSPackedPlaintext(values, level=0)
    ct = cc.Encrypt(pt); cc.Decrypt(ct).GetRealPackedValue()
    cc.EvalAdd / EvalSub / EvalMult / EvalRotate / EvalFastRotation /
    cc.AccumulateSum / cc.Rescale / ct.GetLevel()

EvalMult follows FLEXIBLEAUTO: operands carrying a product's scale are
rescaled first and the operand with more limbs is brought down to the other's
level before the product; results are left unrescaled.  Errors surface as
``CKKSError`` (the reference raises C++ exceptions, T123.cpp:1757-1761).

There is no CPU fallback: importing works without a GPU, but creating a
context needs the CUDA library and a device, and fails loudly otherwise.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libckks_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "ckks_b200.h")

_u64p = ctypes.POINTER(ctypes.c_uint64)
_f64p = ctypes.POINTER(ctypes.c_double)
_vp = ctypes.c_void_p


class CKKSError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class ckks_params(ctypes.Structure):
    _fields_ = [
        ("log_n", ctypes.c_int),
        ("limbs", ctypes.c_int),
        ("dnum", ctypes.c_int),
        ("first_mod_bits", ctypes.c_int),
        ("scale_mod_bits", ctypes.c_int),
        ("special_mod_bits", ctypes.c_int),
        ("seed", ctypes.c_uint64),
        ("device", ctypes.c_int),
    ]


# (name, restype, argtypes) for every symbol of include/ckks_b200.h
_SIGS = [
    ("ckks_last_error", ctypes.c_char_p, []),
    ("ckks_ctx_create", ctypes.c_int, [ctypes.POINTER(ckks_params), ctypes.POINTER(_vp)]),
    ("ckks_ctx_destroy", ctypes.c_int, [_vp]),
    ("ckks_ctx_info", ctypes.c_int, [_vp] + [ctypes.POINTER(ctypes.c_int)] * 4),
    ("ckks_ctx_low_set", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    ("ckks_ctx_moduli", ctypes.c_int, [_vp, _u64p, ctypes.c_int]),
    ("ckks_ctx_scale", ctypes.c_double, [_vp, ctypes.c_int]),
    ("ckks_sync", ctypes.c_int, [_vp]),
    ("ckks_ctx_stream", _vp, [_vp]),
    ("ckks_keygen", ctypes.c_int, [_vp]),
    ("ckks_relin_keygen", ctypes.c_int, [_vp]),
    ("ckks_rotkey_gen", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    ("ckks_key_export", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _u64p, ctypes.c_size_t]),
    ("ckks_ct_create", ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    ("ckks_ct_destroy", ctypes.c_int, [_vp]),
    ("ckks_pt_create", ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    ("ckks_pt_destroy", ctypes.c_int, [_vp]),
    ("ckks_ct_level", ctypes.c_int, [_vp]),
    ("ckks_ct_limbs", ctypes.c_int, [_vp]),
    ("ckks_ct_scale", ctypes.c_double, [_vp]),
    ("ckks_ct_noise_deg", ctypes.c_int, [_vp]),
    ("ckks_pt_limbs", ctypes.c_int, [_vp]),
    ("ckks_pt_scale", ctypes.c_double, [_vp]),
    ("ckks_ct_set_scale", ctypes.c_int, [_vp, ctypes.c_double, ctypes.c_int]),
    ("ckks_ct_export", ctypes.c_int, [_vp, _vp, _u64p, ctypes.c_size_t]),
    ("ckks_ct_import", ctypes.c_int, [_vp, _vp, _u64p, ctypes.c_int, ctypes.c_double, ctypes.c_int]),
    ("ckks_pt_export", ctypes.c_int, [_vp, _vp, _u64p, ctypes.c_size_t]),
    ("ckks_pt_import", ctypes.c_int, [_vp, _vp, _u64p, ctypes.c_int, ctypes.c_double]),
    ("ckks_ct_copy", ctypes.c_int, [_vp, _vp, _vp]),
    ("ckks_encode", ctypes.c_int, [_vp, _f64p, ctypes.c_int, ctypes.c_int, _vp]),
    ("ckks_encode_at", ctypes.c_int, [_vp, _f64p, ctypes.c_int, ctypes.c_int, ctypes.c_double, _vp]),
    ("ckks_decode", ctypes.c_int, [_vp, _vp, _f64p, ctypes.c_int]),
    ("ckks_encrypt", ctypes.c_int, [_vp, _vp, _vp]),
    ("ckks_decrypt", ctypes.c_int, [_vp, _vp, _vp]),
    ("ckks_encrypt_batch", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.c_int, ctypes.POINTER(_vp)]),
    ("ckks_decrypt_decode_batch", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.c_int, _f64p, ctypes.c_int]),
    ("ckks_set_encrypt_counter", ctypes.c_int, [_vp, ctypes.c_uint64]),
    ("ckks_get_encrypt_counter", ctypes.c_uint64, [_vp]),
    ("ckks_add", ctypes.c_int, [_vp, _vp, _vp, _vp]),
    ("ckks_sub", ctypes.c_int, [_vp, _vp, _vp, _vp]),
    ("ckks_add_pt", ctypes.c_int, [_vp, _vp, _vp, _vp]),
    ("ckks_add_many", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.c_int, _vp]),
    ("ckks_add_batch", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.c_int,
                                      ctypes.POINTER(_vp)]),
    ("ckks_add_scalar", ctypes.c_int, [_vp, _vp, ctypes.c_double, _vp]),
    ("ckks_mul_pt", ctypes.c_int, [_vp, _vp, _vp, _vp]),
    ("ckks_mul_pt_batch", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, _vp]),
    ("ckks_rotate_hoisted_batch", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                                 _vp]),
    ("ckks_mul_ct", ctypes.c_int, [_vp, _vp, _vp, _vp]),
    ("ckks_mul_int", ctypes.c_int, [_vp, _vp, ctypes.c_int64, _vp]),
    ("ckks_rescale", ctypes.c_int, [_vp, _vp, _vp]),
    ("ckks_drop_limbs", ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    ("ckks_rotate", ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    ("ckks_rotate_hoisted", ctypes.c_int, [_vp, _vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                           ctypes.POINTER(_vp)]),
    ("ckks_rotate_batch", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                         ctypes.POINTER(_vp)]),
    ("ckks_rotate_sum", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(ctypes.c_int), ctypes.c_int, _vp]),
    ("ckks_mul_ct_sum", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.c_int, _vp]),
    ("ckks_mul_ct_batch", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.c_int,
                                         ctypes.POINTER(_vp)]),
    ("ckks_rescale_batch", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.c_int, ctypes.POINTER(_vp)]),
    ("ckks_accumulate_sum", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("ckks_rotate_sum_hoisted", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                               _vp]),
    ("ckks_window_sum_batch", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    ("ckks_window_sum_batch_radix", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                   _vp]),
    ("ckks_rotate_sum_groups", ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp]),
    ("ckks_profile_enable", ctypes.c_int, [_vp, ctypes.c_int]),
    ("ckks_profile_reset", ctypes.c_int, [_vp]),
    ("ckks_profile_report", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_size_t]),
    ("ckks_profile_sections", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_size_t]),
    ("ckks_profile_only", ctypes.c_int, [_vp, ctypes.c_char_p]),
    ("ckks_ntt_forward_device", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int]),
    ("ckks_rotate_noalloc", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("ckks_selftest_bulk_wait", ctypes.c_int, [_vp, ctypes.c_int]),
    ("ckks_block_create", ctypes.c_int, [_vp] + [_f64p] * 6 + [ctypes.c_int] * 4 + [ctypes.POINTER(_vp)]),
    ("ckks_block_destroy", ctypes.c_int, [_vp]),
    ("ckks_block_rotation_indices", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    ("ckks_block_forward", ctypes.c_int, [_vp, _f64p, ctypes.c_int, _f64p]),
    ("ckks_block_report", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_size_t]),
    ("ckks_block_release_cache", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_size_t)]),
    ("ckks_block_shard_inputs", ctypes.c_int, [_vp, _f64p, ctypes.c_int]),
    ("ckks_block_shard_qkv", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    ("ckks_block_shard_scores", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int, _vp]),
    ("ckks_block_shard_softmax", ctypes.c_int, [_vp, _vp]),
    ("ckks_block_shard_context", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    ("ckks_block_shard_scores_tiles", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int, _vp]),
    ("ckks_block_shard_context_tiles", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    ("ckks_block_shard_output", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int, _f64p]),
    ("ckks_block_shard_qkv_parts", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int]),
    ("ckks_block_shard_mlp", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int]),
    ("ckks_block_shard_finish", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int, _f64p]),
    ("ckks_block_mlp_chunks", ctypes.c_int, [_vp]),
    ("ckks_block_state_get", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("ckks_block_state_set", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    ("ckks_ct_export_device", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_size_t]),
    ("ckks_ct_import_device", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_double, ctypes.c_int]),
    ("ckks_ct_serialize", ctypes.c_longlong, [_vp, _vp, ctypes.c_char_p, ctypes.c_size_t]),
    ("ckks_ct_deserialize", ctypes.c_int, [_vp, _vp, ctypes.c_char_p, ctypes.c_size_t]),
    ("ckks_key_serialize", ctypes.c_longlong, [_vp, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]),
    ("ckks_key_deserialize", ctypes.c_int, [_vp, ctypes.c_char_p, ctypes.c_size_t]),
    ("ckks_head_create", ctypes.c_int, [_vp] + [_f64p] * 4 + [ctypes.c_int, ctypes.POINTER(_vp)]),
    ("ckks_head_forward", ctypes.c_int, [_vp, _f64p, _f64p]),
    ("ckks_model_forward", ctypes.c_int, [ctypes.POINTER(_vp), ctypes.c_int, _vp, _f64p, ctypes.c_int, ctypes.c_int,
                                          _f64p, _f64p]),
    ("ckks_schedule_active_shifts", ctypes.c_int, [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    ("ckks_schedule_diagonal", ctypes.c_int, [_f64p] + [ctypes.c_int] * 8 + [_f64p]),
    ("ckks_ntt_inverse_device", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int]),
    ("ckks_ntt_forward_polys", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int]),
    ("ckks_ntt_inverse_polys", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int]),
    ("ckks_bsgs_diagonals_create", ctypes.c_int, [_vp, _f64p] + [ctypes.c_int] * 6 + [ctypes.POINTER(_vp)]),
    ("ckks_bsgs_diagonals_destroy", ctypes.c_int, [_vp]),
    ("ckks_bsgs_matmul", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.c_int, ctypes.POINTER(_vp), ctypes.c_int,
                                        ctypes.POINTER(_vp)]),
    ("ckks_lane_shift", ctypes.c_int, [_vp, ctypes.POINTER(_vp), ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                       ctypes.c_int, ctypes.c_int, ctypes.POINTER(_vp)]),
]

_lib = None


def lib():
    """Loads libckks_b200.so (building it first if absent)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from .build import build
            build()
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return [s[0] for s in _SIGS]


def _check(rc: int):
    if rc != 0:
        raise CKKSError(rc, lib().ckks_last_error().decode())


def _u64(a: np.ndarray):
    assert a.dtype == np.uint64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_u64p)


@dataclass
class CCParams:
    """CCParams<CryptoContextCKKSRNS> fields used by T123.cpp:1602-1614."""
    ring_dim_log: int = 16
    limbs: int = 24            # multiplicative depth + 1
    dnum: int = 3              # SetNumLargeDigits
    first_mod_bits: int = 60   # SetFirstModSize
    scale_mod_bits: int = 50   # SetScalingModSize
    special_mod_bits: int = 60
    seed: int = 1
    device: int = 0


class Plaintext:
    def __init__(self, cc: "CryptoContext"):
        self.cc = cc
        h = _vp()
        _check(lib().ckks_pt_create(cc.h, ctypes.byref(h)))
        self.h = h

    def __del__(self):
        try:
            if self.h:
                lib().ckks_pt_destroy(self.h)
                self.h = None
        except Exception:
            pass

    @property
    def limbs(self) -> int:
        return lib().ckks_pt_limbs(self.h)

    @property
    def scale(self) -> float:
        return lib().ckks_pt_scale(self.h)

    def GetRealPackedValue(self, length: int | None = None) -> np.ndarray:
        n = self.cc.slots if length is None else length
        out = np.zeros(n, np.float64)
        _check(lib().ckks_decode(self.cc.h, self.h, out.ctypes.data_as(_f64p), n))
        return out

    def limbs_array(self) -> np.ndarray:
        out = np.zeros((self.limbs, self.cc.N), np.uint64)
        _check(lib().ckks_pt_export(self.cc.h, self.h, _u64(out), out.size))
        return out


class Ciphertext:
    def __init__(self, cc: "CryptoContext"):
        self.cc = cc
        h = _vp()
        _check(lib().ckks_ct_create(cc.h, ctypes.byref(h)))
        self.h = h

    def __del__(self):
        try:
            if self.h:
                lib().ckks_ct_destroy(self.h)
                self.h = None
        except Exception:
            pass

    def GetLevel(self) -> int:
        return lib().ckks_ct_level(self.h)

    @property
    def limbs(self) -> int:
        return lib().ckks_ct_limbs(self.h)

    @property
    def scale(self) -> float:
        return lib().ckks_ct_scale(self.h)

    @property
    def noise_deg(self) -> int:
        return lib().ckks_ct_noise_deg(self.h)

    def limbs_array(self) -> np.ndarray:
        out = np.zeros((2, self.limbs, self.cc.N), np.uint64)
        _check(lib().ckks_ct_export(self.cc.h, self.h, _u64(out), out.size))
        return out


class Diagonals:
    """cached_diagonal_plains of one matrix at one level (T123.cpp:1005-1059):
    the n1 * n2 encoded BSGS diagonals, kept on the device."""

    def __init__(self, cc: "CryptoContext", W: np.ndarray, batch: int, n1: int, limbs: int):
        self.cc = cc
        W = np.ascontiguousarray(W, np.float64)
        out_dim, in_dim = W.shape
        h = _vp()
        _check(lib().ckks_bsgs_diagonals_create(cc.h, W.ctypes.data_as(_f64p), out_dim, in_dim, in_dim, batch, n1,
                                                limbs, ctypes.byref(h)))
        self.h = h
        self.batch, self.n1, self.limbs = batch, n1, limbs
        self.n2 = cc.N // 2 // batch // n1

    def __del__(self):
        try:
            if self.h:
                lib().ckks_bsgs_diagonals_destroy(self.h)
                self.h = None
        except Exception:
            pass


class CryptoContext:
    """GenCryptoContext result: parameters, device tables and keys."""

    def __init__(self, params: CCParams):
        p = ckks_params(params.ring_dim_log, params.limbs, params.dnum, params.first_mod_bits,
                        params.scale_mod_bits, params.special_mod_bits, params.seed, params.device)
        h = _vp()
        _check(lib().ckks_ctx_create(ctypes.byref(p), ctypes.byref(h)))
        self.h = h
        self.params = params
        n, L, K, a = (ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int())
        _check(lib().ckks_ctx_info(h, ctypes.byref(n), ctypes.byref(L), ctypes.byref(K), ctypes.byref(a)))
        self.N, self.L, self.K, self.alpha = n.value, L.value, K.value, a.value
        self.slots = self.N // 2
        lo, kl = ctypes.c_int(0), ctypes.c_int(0)
        _check(lib().ckks_ctx_low_set(self.h, ctypes.byref(lo), ctypes.byref(kl)))
        self.low_limbs, self.K_low = lo.value, kl.value
        m = np.zeros(self.L + self.K, np.uint64)
        _check(lib().ckks_ctx_moduli(h, _u64(m), m.size))
        self.moduli = m

    def __del__(self):
        try:
            if self.h:
                lib().ckks_ctx_destroy(self.h)
                self.h = None
        except Exception:
            pass

    # -- setup -----------------------------------------------------------
    def GetRingDimension(self) -> int:
        return self.N

    def GetCyclotomicOrder(self) -> int:
        return 2 * self.N

    def scale_at(self, level: int) -> float:
        return lib().ckks_ctx_scale(self.h, level)

    def KeyGen(self):
        _check(lib().ckks_keygen(self.h))

    def EvalMultKeyGen(self):
        _check(lib().ckks_relin_keygen(self.h))

    def EvalRotateKeyGen(self, indices):
        idx = (ctypes.c_int * len(indices))(*[int(i) for i in indices])
        _check(lib().ckks_rotkey_gen(self.h, idx, len(indices)))

    def Synchronize(self):
        _check(lib().ckks_sync(self.h))

    def profile(self, on: bool = True):
        _check(lib().ckks_profile_enable(self.h, 1 if on else 0))

    def profile_reset(self):
        _check(lib().ckks_profile_reset(self.h))

    def profile_report(self) -> dict:
        import json
        n = lib().ckks_profile_report(self.h, None, 0)
        if n < 0:
            raise CKKSError(-1, lib().ckks_last_error().decode())
        buf = ctypes.create_string_buffer(n + 1)
        lib().ckks_profile_report(self.h, buf, n + 1)
        return json.loads(buf.value.decode())

    def profile_only(self, kernel: str | None):
        """Time only launches of `kernel` (None: every kernel)."""
        _check(lib().ckks_profile_only(self.h, (kernel or "").encode()))

    def profile_sections(self) -> dict:
        """Kernel totals per section (block stages) since the last reset."""
        import json
        n = lib().ckks_profile_sections(self.h, None, 0)
        if n < 0:
            raise CKKSError(-1, lib().ckks_last_error().decode())
        buf = ctypes.create_string_buffer(n + 1)
        lib().ckks_profile_sections(self.h, buf, n + 1)
        return json.loads(buf.value.decode())

    def stream_handle(self) -> int:
        return lib().ckks_ctx_stream(self.h) or 0

    def key_array(self, which: int, k: int = 0) -> np.ndarray:
        P = self.L + self.K
        beta = -(-self.L // self.alpha)
        # 4, 5: relinearisation / rotation key over the reduced special-prime set
        shapes = {0: (P, self.N), 1: (2, self.L, self.N), 2: (beta, 2, P, self.N), 3: (beta, 2, P, self.N),
                  4: (2, P, self.N), 5: (2, P, self.N)}
        out = np.zeros(shapes[which], np.uint64)
        _check(lib().ckks_key_export(self.h, which, k, _u64(out), out.size))
        return out

    # -- client ------------------------------------------------------------
    def MakeCKKSPackedPlaintext(self, values, level: int = 0, scale: float | None = None,
                                limbs: int | None = None) -> Plaintext:
        v = np.ascontiguousarray(values, np.float64)
        pt = Plaintext(self)
        if scale is None and limbs is None:
            _check(lib().ckks_encode(self.h, v.ctypes.data_as(_f64p), v.size, level, pt.h))
        else:
            lb = self.L - level if limbs is None else limbs
            sc = self.scale_at(self.L - lb) if scale is None else scale
            _check(lib().ckks_encode_at(self.h, v.ctypes.data_as(_f64p), v.size, lb, sc, pt.h))
        return pt

    def Encrypt(self, pt: Plaintext) -> Ciphertext:
        ct = Ciphertext(self)
        _check(lib().ckks_encrypt(self.h, pt.h, ct.h))
        return ct

    def Decrypt(self, ct: Ciphertext) -> Plaintext:
        pt = Plaintext(self)
        _check(lib().ckks_decrypt(self.h, ct.h, pt.h))
        return pt

    def EncryptBatch(self, pts) -> list[Ciphertext]:
        outs = [Ciphertext(self) for _ in pts]
        n = len(pts)
        _check(lib().ckks_encrypt_batch(self.h, (_vp * n)(*[p.h for p in pts]), n, (_vp * n)(*[o.h for o in outs])))
        return outs

    def DecryptDecodeBatch(self, cts, slots: int | None = None) -> np.ndarray:
        n = len(cts)
        k = self.slots if slots is None else slots
        out = np.zeros((n, k), np.float64)
        _check(lib().ckks_decrypt_decode_batch(self.h, (_vp * n)(*[c.h for c in cts]), n,
                                               out.ctypes.data_as(_f64p), k))
        return out

    def set_encrypt_counter(self, c: int):
        _check(lib().ckks_set_encrypt_counter(self.h, c))

    def import_ct(self, arr: np.ndarray, scale: float, deg: int = 1) -> Ciphertext:
        arr = np.ascontiguousarray(arr, np.uint64)
        ct = Ciphertext(self)
        _check(lib().ckks_ct_import(self.h, ct.h, _u64(arr), arr.shape[1], scale, deg))
        return ct

    def import_pt(self, arr: np.ndarray, scale: float) -> Plaintext:
        arr = np.ascontiguousarray(arr, np.uint64)
        pt = Plaintext(self)
        _check(lib().ckks_pt_import(self.h, pt.h, _u64(arr), arr.shape[0], scale))
        return pt

    # -- raw ops (no scale management) ------------------------------------
    def export_device(self, ct: Ciphertext, dev_ptr: int, words: int):
        """Copy ct's limbs (c0 then c1) into a device buffer, on the engine stream."""
        _check(lib().ckks_ct_export_device(self.h, ct.h, ctypes.c_void_p(dev_ptr), words))

    def import_device(self, dev_ptr: int, limbs: int, scale: float, deg: int = 1) -> Ciphertext:
        ct = self._new()
        _check(lib().ckks_ct_import_device(self.h, ct.h, ctypes.c_void_p(dev_ptr), limbs, scale, deg))
        return ct

    def serialize(self, ct: Ciphertext) -> bytes:
        """Binary wire format: header, moduli, residues (checked on load)."""
        n = lib().ckks_ct_serialize(self.h, ct.h, None, 0)
        if n < 0:
            _check(2)
        buf = ctypes.create_string_buffer(n)
        if lib().ckks_ct_serialize(self.h, ct.h, buf, n) != n:
            _check(1)
        return buf.raw

    def deserialize(self, data: bytes) -> Ciphertext:
        ct = self._new()
        _check(lib().ckks_ct_deserialize(self.h, ct.h, data, len(data)))
        return ct

    def serialize_key(self, k: int = 0) -> bytes:
        """Switching key in the wire format: relinearisation (k = 0) or rotation k."""
        n = lib().ckks_key_serialize(self.h, k, None, 0)
        if n < 0:
            _check(4)
        buf = ctypes.create_string_buffer(n)
        if lib().ckks_key_serialize(self.h, k, buf, n) != n:
            _check(1)
        return buf.raw

    def deserialize_key(self, data: bytes):
        _check(lib().ckks_key_deserialize(self.h, data, len(data)))

    def _new(self) -> Ciphertext:
        return Ciphertext(self)

    def add(self, a, b):
        o = self._new(); _check(lib().ckks_add(self.h, a.h, b.h, o.h)); return o

    def sub(self, a, b):
        o = self._new(); _check(lib().ckks_sub(self.h, a.h, b.h, o.h)); return o

    def mul_pt(self, a, p):
        o = self._new(); _check(lib().ckks_mul_pt(self.h, a.h, p.h, o.h)); return o

    def mul_pt_batch(self, cts, pts):
        """[mul_pt(a, p) for a, p in zip(cts, pts)], ciphertexts at one level."""
        n = len(cts)
        outs = [self._new() for _ in cts]
        _check(lib().ckks_mul_pt_batch(self.h, (_vp * max(1, n))(*[c.h for c in cts]),
                                       (_vp * max(1, n))(*[p.h for p in pts]), n,
                                       (_vp * max(1, n))(*[o.h for o in outs])))
        return outs

    def mul_ct(self, a, b):
        o = self._new(); _check(lib().ckks_mul_ct(self.h, a.h, b.h, o.h)); return o

    def mul_int(self, a, k: int):
        o = self._new(); _check(lib().ckks_mul_int(self.h, a.h, int(k), o.h)); return o

    def rescale(self, a):
        o = self._new(); _check(lib().ckks_rescale(self.h, a.h, o.h)); return o

    def drop_limbs(self, a, limbs: int):
        o = self._new(); _check(lib().ckks_drop_limbs(self.h, a.h, limbs, o.h)); return o

    # -- OpenFHE-named evaluation (FLEXIBLEAUTO) ----------------------------
    def Rescale(self, ct: Ciphertext) -> Ciphertext:
        return self.rescale(ct)

    def _to_deg1(self, ct: Ciphertext) -> Ciphertext:
        return self.rescale(ct) if ct.noise_deg >= 2 else ct

    def _level_reduce(self, ct: Ciphertext, limbs: int) -> Ciphertext:
        """Brings a degree-1 ciphertext down to `limbs` limbs at that level's scale."""
        if ct.limbs == limbs:
            return ct
        target = self.scale_at(self.L - limbs)
        ql = float(self.moduli[ct.limbs - 1])
        c = int(round(target * ql / ct.scale))
        t = self.mul_int(ct, c)
        _check(lib().ckks_ct_set_scale(t.h, ct.scale * c, 2))
        t = self.rescale(t)
        if t.limbs > limbs:
            t = self.drop_limbs(t, limbs)
        return t

    def _align(self, a: Ciphertext, b: Ciphertext):
        if a.noise_deg != b.noise_deg:
            a, b = self._to_deg1(a), self._to_deg1(b)
        if a.limbs != b.limbs:
            if a.noise_deg != 1:
                a, b = self._to_deg1(a), self._to_deg1(b)
            lo = min(a.limbs, b.limbs)
            a, b = self._level_reduce(a, lo), self._level_reduce(b, lo)
        return a, b

    def EvalAdd(self, a: Ciphertext, b) -> Ciphertext:
        if isinstance(b, (int, float)):
            o = self._new(); _check(lib().ckks_add_scalar(self.h, a.h, float(b), o.h)); return o
        if isinstance(b, Plaintext):
            o = self._new(); _check(lib().ckks_add_pt(self.h, a.h, b.h, o.h)); return o
        a, b = self._align(a, b)
        return self.add(a, b)

    def EvalSub(self, a: Ciphertext, b) -> Ciphertext:
        if isinstance(b, (int, float)):
            return self.EvalAdd(a, -float(b))
        a, b = self._align(a, b)
        return self.sub(a, b)

    def EvalMult(self, a: Ciphertext, b) -> Ciphertext:
        a = self._to_deg1(a)
        if isinstance(b, Plaintext):
            return self.mul_pt(a, b)
        if isinstance(b, (list, tuple, np.ndarray)):
            pt = self.MakeCKKSPackedPlaintext(b, level=a.GetLevel())
            return self.mul_pt(a, pt)
        b = self._to_deg1(b)
        a, b = self._align(a, b)
        return self.mul_ct(a, b)

    def EvalRotate(self, ct: Ciphertext, k: int) -> Ciphertext:
        o = self._new(); _check(lib().ckks_rotate(self.h, ct.h, int(k), o.h)); return o

    def EvalFastRotation(self, ct: Ciphertext, indices) -> list[Ciphertext]:
        outs = [self._new() for _ in indices]
        idx = (ctypes.c_int * len(indices))(*[int(i) for i in indices])
        hs = (_vp * len(indices))(*[o.h for o in outs])
        _check(lib().ckks_rotate_hoisted(self.h, ct.h, idx, len(indices), hs))
        return outs

    def EvalAddMany(self, cts) -> Ciphertext:
        o = self._new()
        n = len(cts)
        _check(lib().ckks_add_many(self.h, (_vp * n)(*[c.h for c in cts]), n, o.h))
        return o

    def add_batch(self, a, b) -> list[Ciphertext]:
        outs = [self._new() for _ in a]
        n = len(a)
        _check(lib().ckks_add_batch(self.h, (_vp * n)(*[c.h for c in a]), (_vp * n)(*[c.h for c in b]), n,
                                    (_vp * n)(*[o.h for o in outs])))
        return outs

    def rotate_batch(self, cts, ks) -> list[Ciphertext]:
        outs = [self._new() for _ in cts]
        n = len(cts)
        _check(lib().ckks_rotate_batch(self.h, (_vp * n)(*[c.h for c in cts]), (ctypes.c_int * n)(*ks), n,
                                       (_vp * n)(*[o.h for o in outs])))
        return outs

    def EvalMultSum(self, a, b) -> Ciphertext:
        """sum_i a[i] * b[i] with one relinearisation (not rescaled)."""
        out = self._new()
        n = len(a)
        _check(lib().ckks_mul_ct_sum(self.h, (_vp * n)(*[c.h for c in a]), (_vp * n)(*[c.h for c in b]), n, out.h))
        return out

    def EvalRotateSum(self, cts, ks) -> Ciphertext:
        """sum_i EvalRotate(cts[i], ks[i]) with one ModDown per 32 rotations."""
        out = self._new()
        n = len(cts)
        _check(lib().ckks_rotate_sum(self.h, (_vp * n)(*[c.h for c in cts]), (ctypes.c_int * n)(*ks), n, out.h))
        return out

    def EvalRotateSumGroups(self, groups, ks) -> list[Ciphertext]:
        """[EvalRotateSum(g, ks) for g in groups]: the groups' giant-step sums
        share launches (each rotation key read once for all groups)."""
        G, n = len(groups), len(ks)
        flat = [c.h for g in groups for c in g]
        if any(len(g) != n for g in groups):
            raise ValueError("every group needs one input per rotation index")
        outs = [self._new() for _ in range(G)]
        _check(lib().ckks_rotate_sum_groups(self.h, (_vp * len(flat))(*flat), G, (ctypes.c_int * n)(*ks), n,
                                            (_vp * G)(*[o.h for o in outs])))
        return outs

    def mul_ct_batch(self, a, b) -> list[Ciphertext]:
        outs = [self._new() for _ in a]
        n = len(a)
        _check(lib().ckks_mul_ct_batch(self.h, (_vp * n)(*[c.h for c in a]), (_vp * n)(*[c.h for c in b]), n,
                                       (_vp * n)(*[o.h for o in outs])))
        return outs

    def rescale_batch(self, cts) -> list[Ciphertext]:
        outs = [self._new() for _ in cts]
        n = len(cts)
        _check(lib().ckks_rescale_batch(self.h, (_vp * n)(*[c.h for c in cts]), n, (_vp * n)(*[o.h for o in outs])))
        return outs

    def AccumulateSum(self, ct: Ciphertext, count: int, stride: int) -> Ciphertext:
        o = self._new(); _check(lib().ckks_accumulate_sum(self.h, ct.h, count, stride, o.h)); return o

    def EvalFastRotationBatch(self, cts, ks) -> list[list[Ciphertext]]:
        """[[EvalFastRotation(ct, ks)] for ct in cts], each key read once."""
        n, nk = len(cts), len(ks)
        outs = [[self._new() for _ in ks] for _ in cts]
        flat = [o for row in outs for o in row]
        _check(lib().ckks_rotate_hoisted_batch(self.h, (_vp * max(1, n))(*[c.h for c in cts]), n,
                                               (ctypes.c_int * max(1, nk))(*ks), nk,
                                               (_vp * max(1, len(flat)))(*[o.h for o in flat])))
        return outs

    def EvalRotateSumHoisted(self, cts, ks) -> list[Ciphertext]:
        """[sum_r EvalRotate(ct, ks[r]) for ct in cts]: one ModUp and one
        ModDown per ciphertext."""
        n, nk = len(cts), len(ks)
        outs = [self._new() for _ in cts]
        _check(lib().ckks_rotate_sum_hoisted(self.h, (_vp * max(1, n))(*[c.h for c in cts]), n,
                                             (ctypes.c_int * nk)(*ks), nk, (_vp * max(1, n))(*[o.h for o in outs])))
        return outs

    def bsgs_diagonals(self, W: np.ndarray, batch: int, n1: int, limbs: int) -> Diagonals:
        """The encoded BSGS diagonals of W ([out, in]) at `limbs` limbs."""
        return Diagonals(self, W, batch, n1, limbs)

    def bsgs_babies(self, cts, batch: int, n1: int) -> list[list[Ciphertext]]:
        """Baby steps [x, rot(x, batch), ..., rot(x, batch (n1 - 1))] of every
        input, one hoisted batch (EvalFastRotation, T123.cpp:1190-1191)."""
        r = self.EvalFastRotationBatch(cts, [batch * j for j in range(1, n1)])
        return [[c] + row for c, row in zip(cts, r)]

    def bsgs_matmul(self, diags, babies) -> list[Ciphertext]:
        """matmul(BabyRotations, W) (T123.cpp:1264-1295): babies[t][q] are the
        n1 baby steps of token group q for matrix term t (diags[t]); returns
        one rescaled product per group, summed over the terms."""
        T, G = len(diags), len(babies[0])
        flat = [c.h for t in range(T) for q in range(G) for c in babies[t][q]]
        outs = [self._new() for _ in range(G)]
        _check(lib().ckks_bsgs_matmul(self.h, (_vp * T)(*[d.h for d in diags]), T, (_vp * len(flat))(*flat), G,
                                      (_vp * G)(*[o.h for o in outs])))
        return outs

    def lane_shift(self, cts, deltas, batch: int) -> list[list[Ciphertext]]:
        """lane_shift (T123.cpp:1297-1314) of every input by every delta:
        out[i][k][f, t] = cts[i][f, (t + deltas[k]) mod batch], rescaled."""
        n, nd = len(cts), len(deltas)
        outs = [[self._new() for _ in deltas] for _ in cts]
        flat = [o.h for row in outs for o in row]
        _check(lib().ckks_lane_shift(self.h, (_vp * n)(*[c.h for c in cts]), n, (ctypes.c_int * nd)(*deltas), nd,
                                     batch, (_vp * len(flat))(*flat)))
        return outs

    def WindowSumBatch(self, cts, window: int, stride: int, radix: int = 4) -> list[Ciphertext]:
        """[sum_{j < window} EvalRotate(ct, j * stride) for ct in cts]: a
        base-radix ladder (the AccumulateSum ladder for radix 4) with one
        ModDown per step."""
        n = len(cts)
        outs = [self._new() for _ in cts]
        _check(lib().ckks_window_sum_batch_radix(self.h, (_vp * max(1, n))(*[c.h for c in cts]), n, window, stride,
                                                 radix, (_vp * max(1, n))(*[o.h for o in outs])))
        return outs


def GenCryptoContext(params: CCParams) -> CryptoContext:
    return CryptoContext(params)


def _f64(a: np.ndarray):
    assert a.dtype == np.float64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f64p)


class EncryptedBlock:
    """One encrypted DNAGPT block (EncryptedEvaluator + Client of the
    reference driver) bound to a context.  ``forward(x)`` encrypts x
    ([tokens, D] float64), evaluates the block with client refreshes and
    returns the decrypted output."""

    def __init__(self, cc: CryptoContext, weights: dict, tokens: int, heads: int = 12):
        self.cc = cc
        self._w = {k: np.ascontiguousarray(weights[k], np.float64) for k in
                   ("ln1", "attn_qkv", "attn_proj", "ln2", "mlp_fc", "mlp_proj")}
        D = self._w["ln1"].shape[0]
        M = self._w["mlp_fc"].shape[0]
        self.D, self.tokens = D, tokens
        h = _vp()
        _check(lib().ckks_block_create(cc.h, _f64(self._w["ln1"]), _f64(self._w["attn_qkv"]),
                                       _f64(self._w["attn_proj"]), _f64(self._w["ln2"]), _f64(self._w["mlp_fc"]),
                                       _f64(self._w["mlp_proj"]), D, heads, M, tokens, ctypes.byref(h)))
        self.h = h

    def __del__(self):
        try:
            if self.h:
                lib().ckks_block_destroy(self.h)
                self.h = None
        except Exception:
            pass

    def rotation_indices(self) -> list[int]:
        n = lib().ckks_block_rotation_indices(self.h, None, 0)
        buf = (ctypes.c_int * n)()
        lib().ckks_block_rotation_indices(self.h, buf, n)
        return list(buf)

    def forward(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float64)
        y = np.zeros_like(x)
        _check(lib().ckks_block_forward(self.h, _f64(x), x.shape[0], _f64(y)))
        return y

    def report(self) -> dict:
        import json
        n = lib().ckks_block_report(self.h, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        lib().ckks_block_report(self.h, buf, n + 1)
        return json.loads(buf.value.decode())


    # ---- stages over unit subsets (sharding one block over ranks) ----
    def shard_inputs(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float64)
        _check(lib().ckks_block_shard_inputs(self.h, _f64(x), x.shape[0]))

    def shard_qkv(self, groups, parts: int = 7):
        """LN1 and the projections of `parts` (bit 0 Q, bit 1 K, bit 2 V)."""
        g = (ctypes.c_int * max(1, len(groups)))(*groups)
        _check(lib().ckks_block_shard_qkv_parts(self.h, g, len(groups), parts))

    @property
    def mlp_chunks(self) -> int:
        return lib().ckks_block_mlp_chunks(self.h)

    def shard_mlp(self, groups, chunk_begin: int, chunk_end: int):
        """O projection, residual, LN2 and MLP chunks [begin, end) of the
        groups; the chunks' sum is state 5, the residual state 6."""
        g = (ctypes.c_int * max(1, len(groups)))(*groups)
        _check(lib().ckks_block_shard_mlp(self.h, g, len(groups), chunk_begin, chunk_end))

    def shard_finish(self, groups, y: np.ndarray):
        assert y.dtype == np.float64 and y.flags["C_CONTIGUOUS"]
        g = (ctypes.c_int * max(1, len(groups)))(*groups)
        _check(lib().ckks_block_shard_finish(self.h, g, len(groups), _f64(y)))

    @staticmethod
    def _pairs(pairs):
        flat = [v for p in pairs for v in p]
        return (ctypes.c_int * max(1, len(flat)))(*flat), len(pairs)

    def shard_scores(self, pairs, d_scores_ptr: int):
        p, n = self._pairs(pairs)
        _check(lib().ckks_block_shard_scores(self.h, p, n, ctypes.c_void_p(d_scores_ptr)))

    def shard_softmax(self, d_scores_ptr: int):
        _check(lib().ckks_block_shard_softmax(self.h, ctypes.c_void_p(d_scores_ptr)))

    def shard_context(self, pairs):
        p, n = self._pairs(pairs)
        _check(lib().ckks_block_shard_context(self.h, p, n))

    def shard_scores_tiles(self, tiles, d_scores_ptr: int):
        """Scores of explicit alignments (qg, kg, d)."""
        p, n = self._pairs(tiles)
        _check(lib().ckks_block_shard_scores_tiles(self.h, p, n, ctypes.c_void_p(d_scores_ptr)))

    def shard_context_tiles(self, tiles):
        p, n = self._pairs(tiles)
        _check(lib().ckks_block_shard_context_tiles(self.h, p, n))

    def shard_output(self, groups, y: np.ndarray):
        assert y.dtype == np.float64 and y.flags["C_CONTIGUOUS"]
        g = (ctypes.c_int * max(1, len(groups)))(*groups)
        _check(lib().ckks_block_shard_output(self.h, g, len(groups), _f64(y)))

    def state_get(self, kind: int, group: int):
        """Copy of a state ciphertext (0 Q, 1 K, 2 V, 3 partial context,
        4 encrypted input, 5 MLP sum, 6 attention residual) of a token group,
        or None if absent."""
        out = self.cc._new()
        rc = lib().ckks_block_state_get(self.h, kind, group, out.h)
        if rc == 2:  # CKKS_ESTATE: not present
            return None
        _check(rc)
        return out

    def state_set(self, kind: int, group: int, ct):
        _check(lib().ckks_block_state_set(self.h, kind, group, ct.h))

    def release_cache(self) -> int:
        """Drop the encoded diagonals (re-encoded on the next forward);
        returns the bytes released."""
        n = ctypes.c_size_t(0)
        _check(lib().ckks_block_release_cache(self.h, ctypes.byref(n)))
        return n.value


class EncryptedHead:
    """The classifier head of the reference's 12-block driver
    (EncryptedHeadEvaluator): final LN, head linear, SiLU client boundary,
    head LN and the N - A readout margin, on one token.  ``weights`` holds
    final_ln [D], head_linear [D, D], head_ln [D] and readout [D] (the
    difference of the N and A rows of the readout matrix)."""

    def __init__(self, cc: CryptoContext, weights: dict):
        self.cc = cc
        self._w = {k: np.ascontiguousarray(weights[k], np.float64) for k in
                   ("final_ln", "head_linear", "head_ln", "readout")}
        D = self._w["final_ln"].shape[0]
        self.D = D
        h = _vp()
        _check(lib().ckks_head_create(cc.h, _f64(self._w["final_ln"]), _f64(self._w["head_linear"]),
                                      _f64(self._w["head_ln"]), _f64(self._w["readout"]), D, ctypes.byref(h)))
        self.h = h

    def __del__(self):
        try:
            if self.h:
                lib().ckks_block_destroy(self.h)
                self.h = None
        except Exception:
            pass

    def rotation_indices(self) -> list[int]:
        n = lib().ckks_block_rotation_indices(self.h, None, 0)
        buf = (ctypes.c_int * n)()
        lib().ckks_block_rotation_indices(self.h, buf, n)
        return list(buf)

    def forward(self, x_last: np.ndarray) -> float:
        x_last = np.ascontiguousarray(x_last, np.float64)
        assert x_last.shape == (self.D,)
        m = np.zeros(1, np.float64)
        _check(lib().ckks_head_forward(self.h, _f64(x_last), _f64(m)))
        return float(m[0])

    def report(self) -> dict:
        return EncryptedBlock.report(self)


class EncryptedModel:
    """Chained encrypted blocks with the full-hidden-state client refresh
    between them, then the last-token refresh into the classifier head (the
    reference's 12blocks_head_cpudiagcache_t123_v3.cpp driver).  Blocks with
    index >= ``cached_blocks`` release their encoded diagonals after each
    forward (about 26 GB per block at N = 2^16, so 12 blocks do not all fit
    one device); None keeps every block's cache."""

    def __init__(self, cc: CryptoContext, block_weights: list, head_weights: dict | None, tokens: int,
                 heads: int = 12, cached_blocks: int | None = None):
        self.cc = cc
        self.blocks = [EncryptedBlock(cc, w, tokens, heads) for w in block_weights]
        self.head = EncryptedHead(cc, head_weights) if head_weights is not None else None
        self.tokens = tokens
        self.cached_blocks = len(self.blocks) if cached_blocks is None else cached_blocks

    @classmethod
    def from_fixture(cls, cc: CryptoContext, directory, tokens: int | None = None, heads: int = 12,
                     cached_blocks: int | None = None, verify: bool = True):
        """Blocks and head from a fixture directory in the reference's float64
        format (`fixture.load_fixture`); tokens default to the fixture's
        `input.embeddings` rows."""
        from . import fixture as fx_mod
        fx = fx_mod.load_fixture(directory, verify)
        if tokens is None:
            tokens = fx.embeddings().shape[0]
        model = cls(cc, [fx.block_weights(b) for b in range(fx.num_blocks)], fx.head_weights(), tokens, heads,
                    cached_blocks)
        model.fixture = fx
        return model

    def rotation_indices(self) -> list[int]:
        s = set(self.blocks[0].rotation_indices())
        if self.head is not None:
            s |= set(self.head.rotation_indices())
        return sorted(s)

    def forward(self, x: np.ndarray):
        """Returns (hidden [tokens, D] of the last block, head margin or None)."""
        x = np.ascontiguousarray(x, np.float64)
        hidden = np.zeros_like(x)
        m = np.zeros(1, np.float64)
        n = len(self.blocks)
        hs = (_vp * n)(*[b.h for b in self.blocks])
        _check(lib().ckks_model_forward(hs, n, self.head.h if self.head is not None else None, _f64(x),
                                        x.shape[0], self.cached_blocks, _f64(hidden), _f64(m)))
        return hidden, (float(m[0]) if self.head is not None else None)


def schedule_active_shifts(tokens: int, batch: int, qg: int, kg: int) -> list[int]:
    buf = (ctypes.c_int * batch)()
    n = lib().ckks_schedule_active_shifts(tokens, batch, qg, kg, buf, batch)
    if n < 0:
        raise CKKSError(1, "bad tile")
    return list(buf)[:n]


def schedule_diagonal(W: np.ndarray, out_dim: int, in_dim: int, pack_width: int, batch: int, n1: int, g: int,
                      j: int) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float64)
    out = np.zeros(pack_width * batch, np.float64)
    _check(lib().ckks_schedule_diagonal(_f64(W), out_dim, in_dim, W.shape[1], pack_width, batch, n1, g, j,
                                        _f64(out)))
    return out
