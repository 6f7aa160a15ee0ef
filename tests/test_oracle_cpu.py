"""CPU checks of the RNS-CKKS oracle itself (no GPU).

The oracle cannot be pinned to OpenFHE limbs (OpenFHE is absent), so it is
pinned here against first principles and published known answers:
  * the NTT equals evaluation at psi^(2 bitrev(k) + 1) (naive O(N^2) sum);
  * the ChaCha20 block function reproduces RFC 7539 section 2.3.2;
  * encode/decode realises the slot semantics m(zeta^(5^j)) of the
    reference's MakeCKKSPackedPlaintext / GetRealPackedValue (T123.cpp:525-526,
    955-960), with the left-rotation convention of simd_layout.rotate_left
    (fhe/gpu_real_scheme_b/simd_layout.py:136-139);
  * every homomorphic operation decrypts to the plaintext operation.
"""

import ctypes

import numpy as np
import pytest

import oracle
from oracle import Oracle


def bitrev(x, bits):
    return int(format(x, f"0{bits}b")[::-1], 2)


def ladder_keys(count, stride):
    """Rotation indices of the base-4 AccumulateSum ladder (T123.cpp:444-453)."""
    keys, step = [], 1
    while step < count:
        keys += [stride * step * m for m in range(1, 4) if step * m < count]
        step *= 4
    return keys


ACC_CASES = [(64, 1), (32, 8), (8, 32), (2, 128)]


@pytest.fixture(scope="module")
def small():
    o = Oracle(logN=10, L=6, dnum=3, seed=11)
    o.keygen()
    o.relin_keygen()
    keys = [1, 2, 3, -1, 7, 8, 256] + [32 * m for m in range(1, 8)]  # + the base-8 ladder of 8 at stride 32
    for c, st in ACC_CASES:
        keys += ladder_keys(c, st)
    o.rot_keygen(sorted(set(keys)))
    return o


def test_prime_chain_properties():
    o = Oracle(logN=12, L=8, dnum=3, seed=1)
    q = [int(x) for x in o.moduli]
    assert len(q) == o.L + o.K and o.K == o.alpha == 3
    assert len(set(q)) == len(q)
    for x in q:
        assert x % (2 * o.N) == 1
        assert pow(2, x - 1, x) == 1
    assert q[0].bit_length() == 60
    assert all(x.bit_length() in (50, 51) for x in q[1:o.L])
    assert all(x.bit_length() == 60 for x in q[o.L:])
    # FLEXIBLEAUTO scale chain
    assert o.scale(o.L) == float(q[o.L - 1])
    for l in range(o.L, 1, -1):
        assert o.scale(l - 1) == o.scale(l) * o.scale(l) / float(q[l - 1])


@pytest.mark.parametrize("logN", [4, 6])
def test_ntt_is_negacyclic_evaluation(logN):
    o = Oracle(logN=logN, L=2, dnum=1, seed=3)
    N = o.N
    rng = np.random.default_rng(logN)
    for pi in range(o.L + o.K):
        q, psi = int(o.moduli[pi]), int(o.psi[pi])
        assert pow(psi, N, q) == q - 1
        a = rng.integers(0, q, N, dtype=np.uint64)
        ah = o.ntt(a, pi)
        for k in range(N):
            e = 2 * bitrev(k, logN) + 1
            s = sum(int(a[j]) * pow(psi, e * j, q) for j in range(N)) % q
            assert s == int(ah[k])
        assert np.array_equal(o.intt(ah, pi), a)


def test_ntt_convolution_is_negacyclic():
    o = Oracle(logN=6, L=2, dnum=1, seed=3)
    N, q = o.N, int(o.moduli[0])
    rng = np.random.default_rng(0)
    a = rng.integers(0, q, N, dtype=np.uint64)
    b = rng.integers(0, q, N, dtype=np.uint64)
    prod = o.intt(np.array([(int(x) * int(y)) % q for x, y in zip(o.ntt(a, 0), o.ntt(b, 0))], np.uint64), 0)
    ref = [0] * N
    for i in range(N):
        for j in range(N):
            k = i + j
            v = int(a[i]) * int(b[j])
            if k >= N:
                ref[k - N] -= v
            else:
                ref[k] += v
    assert [x % q for x in ref] == [int(x) for x in prod]


def test_chacha20_rfc7539_block():
    L = oracle.lib()
    key = (ctypes.c_uint32 * 8)(*[int.from_bytes(bytes(range(4 * i, 4 * i + 4)), "little") for i in range(8)])
    out = (ctypes.c_uint32 * 16)()
    # RFC 7539 2.3.2: block count 1, nonce 00:00:00:09:00:00:00:4a:00:00:00:00
    L.oc_chacha_block(key, ctypes.c_uint64(1 | (0x09000000 << 32)), ctypes.c_uint64(0x4A000000), out)
    expect = [0xE4E7F110, 0x15593BD1, 0x1FDD0F50, 0xC47120A3, 0xC7F4D1C7, 0x0368C033, 0x9AAA2204, 0x4E6CD4C3,
              0x466482D2, 0x09AA9F07, 0x05D7C214, 0xA2028BD9, 0xD19C12B5, 0xB94E16DE, 0xE883D0CB, 0x4E3C50A2]
    assert list(out) == expect


def test_encode_slot_semantics(small):
    o = small
    rng = np.random.default_rng(1)
    v = rng.standard_normal(o.N // 2)
    pt = o.encode(v, o.L)
    coef = o.intt(pt[0], 0)
    q0 = int(o.moduli[0])
    m = np.array([int(c) - q0 if int(c) > q0 // 2 else int(c) for c in coef], np.float64) / o.scale(o.L)
    M = 2 * o.N
    zeta = np.exp(2j * np.pi / M)
    for j in range(8):
        val = np.polyval(m[::-1], zeta ** pow(5, j, M))
        assert abs(val.real - v[j]) < 1e-9 and abs(val.imag) < 1e-9
    assert np.abs(o.decode(pt, o.scale(o.L)) - v).max() < 1e-9


def test_encode_large_values_exact_residues(small):
    """Values far above 2^63 after scaling go through the exact mant*2^e path."""
    o = small
    v = np.zeros(o.N // 2)
    v[0] = 3.0e6
    pt = o.encode(v, 2, scale=2.0 ** 60)
    back = o.decode(pt, 2.0 ** 60)
    assert abs(back[0] - 3.0e6) < 1e-3


def test_encrypt_decrypt_and_arithmetic(small):
    o = small
    rng = np.random.default_rng(2)
    x = rng.uniform(-1, 1, o.N // 2)
    y = rng.uniform(-1, 1, o.N // 2)
    L, S = o.L, o.scale(o.L)
    cx = o.encrypt(o.encode(x, L), 0)
    cy = o.encrypt(o.encode(y, L), 1)
    dec = lambda ct, s: o.decode(o.decrypt(ct), s)
    assert np.abs(dec(cx, S) - x).max() < 1e-8
    assert np.abs(dec(o.add(cx, cy), S) - (x + y)).max() < 1e-8
    assert np.abs(dec(o.sub(cx, cy), S) - (x - y)).max() < 1e-8
    assert np.abs(dec(o.mul_pt(cx, o.encode(y, L)), S * S) - x * y).max() < 1e-8
    prod = o.mul_ct(cx, cy)
    assert np.abs(dec(prod, S * S) - x * y).max() < 1e-8
    r = o.rescale(prod)
    assert r.shape[1] == L - 1
    assert np.abs(dec(r, S * S / float(o.moduli[L - 1])) - x * y).max() < 1e-8
    assert np.abs(dec(o.add_const(cx, 0.25, S), S) - (x + 0.25)).max() < 1e-8
    assert np.abs(dec(o.mul_int(cx, -3), S) - (-3 * x)).max() < 1e-8


@pytest.mark.parametrize("k", [1, 2, 3, -1, 7, 8, 256])
def test_rotation_is_left_roll(small, k):
    o = small
    x = np.random.default_rng(3).uniform(-1, 1, o.N // 2)
    S = o.scale(o.L)
    ct = o.encrypt(o.encode(x, o.L), 5)
    got = o.decode(o.decrypt(o.rotate(ct, k)), S)
    assert np.abs(got - np.roll(x, -k)).max() < 1e-8


def test_hoisted_equals_single_rotations(small):
    o = small
    x = np.random.default_rng(4).uniform(-1, 1, o.N // 2)
    ct = o.encrypt(o.encode(x, 4), 6)
    h = o.rotate_hoisted(ct, [1, 2, 3, 0])
    for i, k in enumerate([1, 2, 3]):
        assert np.array_equal(h[i], o.rotate(ct, k))
    assert np.array_equal(h[3], ct)


def test_rotate_sum_decrypts_to_the_sum_of_rotations(small):
    o = small
    rng = np.random.default_rng(41)
    xs = [rng.uniform(-1, 1, o.N // 2) for _ in range(4)]
    ks = [0, 1, 3, 7]
    S = o.scale(4)
    cts = np.stack([o.encrypt(o.encode(x, 4), 40 + i) for i, x in enumerate(xs)])
    got = o.decode(o.decrypt(o.rotate_sum(cts, ks)), S)
    ref = sum(np.roll(x, -k) for x, k in zip(xs, ks))
    assert np.abs(got - ref).max() < 1e-8
    # one ModDown for the group equals the separate rotations up to rounding
    sep = sum(o.decode(o.decrypt(o.rotate(ct, k)), S) for ct, k in zip(cts, ks))
    assert np.abs(got - sep).max() < 1e-9


def test_mul_ct_sum_decrypts_to_the_sum_of_products(small):
    o = small
    rng = np.random.default_rng(43)
    xs = [rng.uniform(-1, 1, o.N // 2) for _ in range(6)]
    S = o.scale(4)
    cts = np.stack([o.encrypt(o.encode(x, 4), 80 + i) for i, x in enumerate(xs)])
    got = o.decode(o.decrypt(o.mul_ct_sum(cts[:3], cts[3:])), S * S)
    assert np.abs(got - sum(xs[i] * xs[3 + i] for i in range(3))).max() < 1e-9


@pytest.mark.parametrize("count,stride", ACC_CASES)
def test_window_sum_equals_the_ladder_of_rotation_sums(small, count, stride):
    """The engine's window sums: the AccumulateSum slot values, each ladder
    step one rotation sum over (acc, acc, acc, acc) with one ModDown."""
    o = small
    x = np.random.default_rng(6).uniform(-1, 1, o.N // 2)
    S = o.scale(o.L)
    ct = o.encrypt(o.encode(x, o.L), 9)
    got = o.window_sum(ct, count, stride)
    ref = sum(np.roll(x, -stride * k) for k in range(count))
    assert np.abs(o.decode(o.decrypt(got), S) - ref).max() < 1e-7
    acc = ct
    step = 1
    while step < count:
        ks = [0] + [stride * step * m for m in range(1, 4) if step * m < count]
        acc = o.rotate_sum(np.stack([acc] * len(ks)), ks)
        step *= 4
    assert np.array_equal(got, acc)
    if count == 8:  # base 8: one step, the rotations by stride * {0 .. 7}
        got8 = o.window_sum(ct, count, stride, 8)
        ks = [stride * m for m in range(8)]
        assert np.array_equal(got8, o.rotate_sum(np.stack([ct] * 8), ks))
        assert np.abs(o.decode(o.decrypt(got8), S) - ref).max() < 1e-7


@pytest.mark.parametrize("count,stride", ACC_CASES)
def test_accumulate_sum(small, count, stride):
    o = small
    x = np.random.default_rng(5).uniform(-1, 1, o.N // 2)
    S = o.scale(o.L)
    ct = o.encrypt(o.encode(x, o.L), 7)
    got = o.decode(o.decrypt(o.accumulate_sum(ct, count, stride)), S)
    ref = sum(np.roll(x, -stride * k) for k in range(count))
    assert np.abs(got - ref).max() < 1e-7


def test_missing_rotation_key_raises(small):
    o = small
    ct = o.encrypt(o.encode(np.zeros(o.N // 2), 3), 8)
    with pytest.raises(oracle.OracleError):
        o.rotate(ct, 5 + o.N // 4)


def test_keyswitch_matches_definition(small):
    """KS(d) = (k0, k1) with k0 + k1*s = d*s^2 + small noise (relinearisation key)."""
    o = small
    s = o.secret_key()
    d = o.encrypt(o.encode(np.ones(o.N // 2), o.L), 9)[1]
    ks = o.keyswitch(d, o.switch_key(0))
    q = int(o.moduli[0])
    s0 = [int(v) for v in s[0]]
    lhs = [(int(a) + int(b) * c) % q for a, b, c in zip(ks[0][0], ks[1][0], s0)]
    rhs = [(int(a) * c * c) % q for a, c in zip(d[0], s0)]
    diff = o.intt(np.array([(a - b) % q for a, b in zip(lhs, rhs)], np.uint64), 0)
    centered = np.array([int(v) if int(v) <= q // 2 else int(v) - q for v in diff], dtype=np.float64)
    # ModDown leaves noise of a few hundred units, nowhere near q ~ 2^60
    assert np.abs(centered).max() < 2.0 ** 20


@pytest.fixture(scope="module")
def wide():
    """alpha = K = 8: key switches at <= 3 limbs use the 3-prime set."""
    o = Oracle(logN=10, L=8, dnum=1, seed=17)
    o.keygen()
    o.relin_keygen()
    o.rot_keygen([1, 3, 5, 32])
    return o


def test_reduced_special_prime_set_is_chosen_by_bits(wide):
    o = wide
    assert (o.low_limbs, o.K_low) == (3, 3) and o.K == 8
    q = o.moduli
    assert sum(np.log2(float(p)) for p in q[o.L:o.L + 3]) >= sum(np.log2(float(p)) for p in q[:3]) + 19.5
    key = o.switch_key_low(0)
    used = list(range(3)) + list(range(o.L, o.L + 3))
    unused = [t for t in range(o.L + o.K) if t not in used]
    assert not key[:, unused].any() and key[:, used].all(axis=-1).any()


@pytest.mark.parametrize("limbs", [1, 2, 3, 4, 5, 8])
def test_key_switches_on_both_prime_sets_decrypt(wide, limbs):
    o = wide
    rng = np.random.default_rng(limbs)
    x = rng.uniform(-1, 1, o.N // 2)
    y = rng.uniform(-1, 1, o.N // 2)
    S = o.scale(limbs)
    cx = o.encrypt(o.encode(x, limbs), 60 + limbs)
    cy = o.encrypt(o.encode(y, limbs), 70 + limbs)
    for k in (1, 5, 32):
        assert np.abs(o.decode(o.decrypt(o.rotate(cx, k)), S) - np.roll(x, -k)).max() < 1e-7
    h = o.rotate_hoisted(cx, [1, 3])
    assert np.abs(o.decode(o.decrypt(h[1]), S) - np.roll(x, -3)).max() < 1e-7
    if limbs >= 2:  # a product at scale S^2 needs more than the 60-bit first prime
        prod = o.decode(o.decrypt(o.mul_ct(cx, cy)), S * S)
        assert np.abs(prod - x * y).max() < 1e-7
    rs = o.decode(o.decrypt(o.rotate_sum(np.stack([cx, cy]), [1, 5])), S)
    assert np.abs(rs - np.roll(x, -1) - np.roll(y, -5)).max() < 1e-7
