"""Parity of the CUDA engine against the CPU oracle, through the C ABI.

Integer work is compared bit for bit (every limb of every key, plaintext and
ciphertext), floating-point decode within 1e-12 absolute on unit-range slots.
Same seeds, same parameters, same call order -> identical limbs.
"""

import numpy as np
import pytest

from oracle import Oracle

pytestmark = pytest.mark.gpu

import private_genomic_dnagpt_b200 as eng  # noqa: E402


def ladder_keys(count, stride):
    keys, step = [], 1
    while step < count:
        keys += [stride * step * m for m in range(1, 4) if step * m < count]
        step *= 4
    return keys


def make_pair(logN, L, dnum, seed, rot=(), relin=True):
    o = Oracle(logN=logN, L=L, dnum=dnum, seed=seed)
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=logN, limbs=L, dnum=dnum, seed=seed))
    o.keygen()
    cc.KeyGen()
    if relin:
        o.relin_keygen()
        cc.EvalMultKeyGen()
    if rot:
        o.rot_keygen(list(rot))
        cc.EvalRotateKeyGen(list(rot))
    return o, cc


ROT = ([1, 2, 3, 5, -1, -7, 8, 64, 100] + ladder_keys(64, 4) + ladder_keys(16, 32)
       + [4 * m for m in range(1, 8)] + [32 * m for m in range(1, 8)])  # base-8 ladder of 64 at stride 4


@pytest.fixture(scope="module")
def pair10():
    return make_pair(10, 6, 3, 21, rot=sorted(set(ROT)))


@pytest.mark.parametrize("logN,L,dnum", [(10, 6, 3), (12, 8, 4), (13, 5, 2), (16, 24, 3), (15, 16, 2), (17, 8, 4)])
def test_prime_chain_matches(logN, L, dnum):
    o = Oracle(logN=logN, L=L, dnum=dnum, seed=1)
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=logN, limbs=L, dnum=dnum, seed=1))
    assert np.array_equal(o.moduli, cc.moduli)
    assert cc.K == o.K and cc.alpha == o.alpha
    for lvl in range(L):
        assert cc.scale_at(lvl) == o.scale(L - lvl)


@pytest.mark.parametrize("logN", [6, 7, 10, 12, 15, 16, 17])
def test_ntt_bit_exact(logN):
    import torch
    L = 3
    o = Oracle(logN=logN, L=L, dnum=1, seed=2)
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=logN, limbs=L, dnum=1, seed=2))
    rng = np.random.default_rng(logN)
    P = L + o.K
    a = np.stack([rng.integers(0, int(o.moduli[i]), o.N, dtype=np.uint64) for i in range(P)])
    ref = np.stack([o.ntt(a[i], i) for i in range(P)])
    dev = torch.from_numpy(a.view(np.int64).copy()).cuda()
    torch.cuda.synchronize()
    eng._check(eng.lib().ckks_ntt_forward_device(cc.h, dev.data_ptr(), P, 0))
    cc.Synchronize()
    got = dev.cpu().numpy().view(np.uint64)
    assert np.array_equal(got, ref)
    eng._check(eng.lib().ckks_ntt_inverse_device(cc.h, dev.data_ptr(), P, 0))
    cc.Synchronize()
    assert np.array_equal(dev.cpu().numpy().view(np.uint64), a)
    # a sub-range starting at a later prime
    dev2 = torch.from_numpy(a[2:4].view(np.int64).copy()).cuda()
    torch.cuda.synchronize()
    eng._check(eng.lib().ckks_ntt_forward_device(cc.h, dev2.data_ptr(), 2, 2))
    cc.Synchronize()
    assert np.array_equal(dev2.cpu().numpy().view(np.uint64), ref[2:4])
    # three polynomials of L Q limbs each in one batched launch pair
    polys = np.concatenate([a[:L], a[:L][::-1] % o.moduli[:L, None], a[:L]])
    dev3 = torch.from_numpy(polys.view(np.int64).copy()).cuda()
    torch.cuda.synchronize()
    eng._check(eng.lib().ckks_ntt_forward_polys(cc.h, dev3.data_ptr(), 3, L))
    cc.Synchronize()
    want = np.stack([o.ntt(polys[i], i % L) for i in range(3 * L)])
    assert np.array_equal(dev3.cpu().numpy().view(np.uint64), want)
    eng._check(eng.lib().ckks_ntt_inverse_polys(cc.h, dev3.data_ptr(), 3, L))
    cc.Synchronize()
    assert np.array_equal(dev3.cpu().numpy().view(np.uint64), polys)


@pytest.mark.parametrize("logN", [10, 16])
def test_encode_bit_exact_and_decode(logN):
    L = 4
    o = Oracle(logN=logN, L=L, dnum=2, seed=3)
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=logN, limbs=L, dnum=2, seed=3))
    rng = np.random.default_rng(7)
    for vals in (rng.standard_normal(o.N // 2), rng.uniform(-4, 4, o.N // 2) * 1e3, np.zeros(o.N // 2)):
        for lvl in (0, 1, 3):
            pt = cc.MakeCKKSPackedPlaintext(vals, level=lvl)
            ref = o.encode(vals, L - lvl)
            assert np.array_equal(pt.limbs_array(), ref)
            dec = pt.GetRealPackedValue()
            dref = o.decode(ref, o.scale(L - lvl))
            assert np.abs(dec - dref).max() <= 1e-12 * max(1.0, np.abs(dref).max())
    # values above 2^63 after scaling (exact mantissa * 2^e path)
    big = np.zeros(o.N // 2)
    big[:3] = [3.0e6, -7.5e5, 1.25]
    pt = cc.MakeCKKSPackedPlaintext(big, limbs=2, scale=2.0 ** 60)
    assert np.array_equal(pt.limbs_array(), o.encode(big, 2, scale=2.0 ** 60))


def test_partial_slot_vector_is_zero_padded(pair10):
    o, cc = pair10
    vals = np.arange(5, dtype=np.float64)
    pt = cc.MakeCKKSPackedPlaintext(vals)
    full = np.zeros(o.N // 2)
    full[:5] = vals
    assert np.array_equal(pt.limbs_array(), o.encode(full, o.L))


def test_keys_bit_exact(pair10):
    o, cc = pair10
    assert np.array_equal(cc.key_array(0), o.secret_key())
    assert np.array_equal(cc.key_array(1), o.public_key())
    assert np.array_equal(cc.key_array(2), o.switch_key(0))
    for k in (1, -1, 64):
        assert np.array_equal(cc.key_array(3, k), o.switch_key(k))


def test_encrypt_decrypt_bit_exact(pair10):
    o, cc = pair10
    rng = np.random.default_rng(8)
    x = rng.uniform(-1, 1, o.N // 2)
    cc.set_encrypt_counter(40)
    for lvl in (0, 2):
        ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x, level=lvl))
        ref = o.encrypt(o.encode(x, o.L - lvl), 40 + lvl // 2)
        assert np.array_equal(ct.limbs_array(), ref)
        assert np.array_equal(cc.Decrypt(ct).limbs_array(), o.decrypt(ref))
        assert np.abs(cc.Decrypt(ct).GetRealPackedValue() - x).max() < 1e-8


def _fresh(o, cc, seed, limbs):
    x = np.random.default_rng(seed).uniform(-1, 1, o.N // 2)
    ref = o.encrypt(o.encode(x, limbs), 1000 + seed)
    return x, ref, cc.import_ct(ref, o.scale(limbs))


def test_elementwise_bit_exact(pair10):
    o, cc = pair10
    L = o.L
    x, rx, cx = _fresh(o, cc, 1, L)
    y, ry, cy = _fresh(o, cc, 2, L)
    assert np.array_equal(cc.add(cx, cy).limbs_array(), o.add(rx, ry))
    assert np.array_equal(cc.sub(cx, cy).limbs_array(), o.sub(rx, ry))
    p = o.encode(y, L)
    assert np.array_equal(cc.mul_pt(cx, cc.import_pt(p, o.scale(L))).limbs_array(), o.mul_pt(rx, p))
    assert np.array_equal(cc.mul_int(cx, -12345).limbs_array(), o.mul_int(rx, -12345))
    got = cc.EvalAdd(cx, 0.375).limbs_array()
    assert np.array_equal(got, o.add_const(rx, 0.375, o.scale(L)))


@pytest.mark.parametrize("limbs", [6, 4, 2, 1])
def test_mul_ct_relin_bit_exact(pair10, limbs):
    o, cc = pair10
    x, rx, cx = _fresh(o, cc, 3, limbs)
    y, ry, cy = _fresh(o, cc, 4, limbs)
    got = cc.mul_ct(cx, cy)
    ref = o.mul_ct(rx, ry)
    assert np.array_equal(got.limbs_array(), ref)
    if limbs >= 2:
        assert np.array_equal(cc.rescale(got).limbs_array(), o.rescale(ref))


@pytest.mark.parametrize("k", [1, 2, -1, 5, 100, -7])
@pytest.mark.parametrize("limbs", [6, 3])
def test_rotate_bit_exact(pair10, k, limbs):
    o, cc = pair10
    x, rx, cx = _fresh(o, cc, 5, limbs)
    got = cc.EvalRotate(cx, k)
    assert np.array_equal(got.limbs_array(), o.rotate(rx, k))
    dec = cc.Decrypt(got).GetRealPackedValue()
    assert np.abs(dec - np.roll(x, -k)).max() < 1e-8


def test_hoisted_and_inplace(pair10):
    o, cc = pair10
    x, rx, cx = _fresh(o, cc, 6, o.L)
    ks = [1, 2, 3, 0, 8]
    outs = cc.EvalFastRotation(cx, ks)
    ref = o.rotate_hoisted(rx, ks)
    for i in range(len(ks)):
        assert np.array_equal(outs[i].limbs_array(), ref[i])
    # output aliasing the input
    eng._check(eng.lib().ckks_rotate(cc.h, cx.h, 5, cx.h))
    assert np.array_equal(cx.limbs_array(), o.rotate(rx, 5))


@pytest.mark.parametrize("ks", [[0, 1, 2, 5, -7], [1] * 3 + [2, 3, 5, 8, 64, 100, -1, -7] * 4 + [0]])
def test_rotate_sum_bit_exact(pair10, ks):
    """Giant-step sums: one ModDown per group of 32 non-identity rotations
    (the second case spans two groups and an identity term)."""
    o, cc = pair10
    limbs = 5
    fr = [_fresh(o, cc, 50 + i, limbs) for i in range(len(ks))]
    got = cc.EvalRotateSum([f[2] for f in fr], ks)
    ref = o.rotate_sum(np.stack([f[1] for f in fr]), ks)
    assert np.array_equal(got.limbs_array(), ref)
    dec = cc.Decrypt(got).GetRealPackedValue()
    assert np.abs(dec - sum(np.roll(f[0], -k) for f, k in zip(fr, ks))).max() < 1e-7


@pytest.mark.parametrize("groups,ks,limbs", [
    (3, [0, 8, 16, 24], 5),             # identity + 3 giant steps, one launch sequence
    (5, [4, 8, -1], 4),                 # no identity; 4 + 1 groups
    (2, [0, 1, 0, 2], 3),               # two identities: one rotation sum per group
    (2, [0] + [1, 2, 3, 5, 8, 64, 100, -1, -7] * 4, 2),  # 36 others: per group
])
def test_rotate_sum_groups_bit_exact(pair10, groups, ks, limbs):
    """Giant-step sums of several groups sharing launches equal the oracle's
    rotation sum of each group."""
    o, cc = pair10
    fr = [[_fresh(o, cc, 500 + 40 * g + i, limbs) for i in range(len(ks))] for g in range(groups)]
    got = cc.EvalRotateSumGroups([[f[2] for f in grp] for grp in fr], ks)
    assert len(got) == groups
    for grp, out in zip(fr, got):
        assert out.limbs == limbs
        assert np.array_equal(out.limbs_array(), o.rotate_sum(np.stack([f[1] for f in grp]), ks))


@pytest.mark.parametrize("n,limbs", [(3, 6), (3, 2), (40, 4)])
def test_mul_ct_sum_bit_exact(pair10, n, limbs):
    """Products summed as degree-2 ciphertexts, one relinearisation (40
    pairs span two tensor-sum launches)."""
    o, cc = pair10
    fa = [_fresh(o, cc, 300 + i, limbs) for i in range(n)]
    fb = [_fresh(o, cc, 400 + i, limbs) for i in range(n)]
    got = cc.EvalMultSum([f[2] for f in fa], [f[2] for f in fb])
    ref = o.mul_ct_sum(np.stack([f[1] for f in fa]), np.stack([f[1] for f in fb]))
    assert np.array_equal(got.limbs_array(), ref)


@pytest.mark.parametrize("count,stride", [(64, 4), (16, 32)])
def test_accumulate_sum_bit_exact(pair10, count, stride):
    o, cc = pair10
    x, rx, cx = _fresh(o, cc, 7, o.L)
    got = cc.AccumulateSum(cx, count, stride)
    assert np.array_equal(got.limbs_array(), o.accumulate_sum(rx, count, stride))


@pytest.mark.parametrize("window,stride,limbs,radix", [(64, 4, None, 4), (16, 32, None, 4), (64, 4, 2, 4),
                                                        (1, 4, 3, 4), (64, 4, 2, 8), (64, 4, None, 8)])
def test_window_sums_bit_exact(pair10, window, stride, limbs, radix):
    """Batched hoisted window sums (three inputs per launch) against the
    oracle's ladder of rotation sums (base 4 and base 8)."""
    o, cc = pair10
    lv = o.L if limbs is None else limbs
    fs = [_fresh(o, cc, 40 + i, lv) for i in range(3)]
    got = cc.WindowSumBatch([f[2] for f in fs], window, stride, radix)
    for f, g in zip(fs, got):
        assert g.limbs == lv
        assert np.array_equal(g.limbs_array(), o.window_sum(f[1], window, stride, radix))


def test_hoisted_rotation_sum_equals_the_rotation_sum(pair10):
    o, cc = pair10
    x, rx, cx = _fresh(o, cc, 44, o.L)
    ks = [0, 4, 8, 12]
    h = cc.EvalRotateSumHoisted([cx], ks)[0]
    assert np.array_equal(h.limbs_array(), cc.EvalRotateSum([cx] * 4, ks).limbs_array())
    assert np.array_equal(h.limbs_array(), o.rotate_sum(np.stack([rx] * 4), ks))
    # without the identity
    h2 = cc.EvalRotateSumHoisted([cx], [4, 8])[0]
    assert np.array_equal(h2.limbs_array(), o.rotate_sum(np.stack([rx] * 2), [4, 8]))
    with pytest.raises(eng.CKKSError):
        cc.EvalRotateSumHoisted([cx], [4, 4])


@pytest.mark.parametrize("limbs", [None, 2])
def test_batched_hoisted_rotations_bit_exact(pair10, limbs):
    """Five inputs by the same indices (an identity among them), against
    the oracle's hoisted rotations of each input."""
    o, cc = pair10
    lv = o.L if limbs is None else limbs
    fs = [_fresh(o, cc, 70 + i, lv) for i in range(5)]
    ks = [1, 0, 3, -1, 8, 64]
    got = cc.EvalFastRotationBatch([f[2] for f in fs], ks)
    for f, row in zip(fs, got):
        ref = o.rotate_hoisted(f[1], ks)
        for r, g in enumerate(row):
            assert np.array_equal(g.limbs_array(), ref[r])


def test_batched_plaintext_products_bit_exact(pair10):
    """40 products (two launches) against the oracle's single products."""
    o, cc = pair10
    fs = [_fresh(o, cc, 60 + i, 4) for i in range(40)]
    pts = [o.encode(np.random.default_rng(90 + i).uniform(-1, 1, o.N // 2), 4) for i in range(40)]
    got = cc.mul_pt_batch([f[2] for f in fs], [cc.import_pt(p, o.scale(4)) for p in pts])
    for f, p, g in zip(fs, pts, got):
        assert np.array_equal(g.limbs_array(), o.mul_pt(f[1], p))


def test_errors_are_reported(pair10):
    o, cc = pair10
    x, rx, cx = _fresh(o, cc, 8, 3)
    y, ry, cy = _fresh(o, cc, 9, 2)
    with pytest.raises(eng.CKKSError) as e:
        cc.EvalRotate(cx, 77)
    assert e.value.code == 4
    with pytest.raises(eng.CKKSError) as e:
        cc.add(cx, cy)
    assert e.value.code == 5
    one = cc.import_ct(ry[:, :1], o.scale(1))
    with pytest.raises(eng.CKKSError) as e:
        cc.rescale(one)
    assert e.value.code == 5
    with pytest.raises(eng.CKKSError):
        cc.MakeCKKSPackedPlaintext(np.zeros(o.N))  # more values than slots


def test_flexibleauto_chain_accuracy(pair10):
    """(x*y + x) * y via EvalMult/EvalAdd with automatic rescale / level alignment."""
    o, cc = pair10
    rng = np.random.default_rng(10)
    x = rng.uniform(-1, 1, o.N // 2)
    y = rng.uniform(-1, 1, o.N // 2)
    cx = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cy = cc.Encrypt(cc.MakeCKKSPackedPlaintext(y))
    t = cc.EvalMult(cx, cy)
    t = cc.EvalAdd(t, cx)
    t = cc.EvalMult(t, cy)
    t = cc.Rescale(t)
    got = cc.Decrypt(t).GetRealPackedValue()
    assert np.abs(got - (x * y + x) * y).max() < 1e-6


@pytest.mark.parametrize("logN,L,dnum", [(12, 8, 3), (11, 7, 2), (11, 10, 4)])
def test_partial_last_digit_keyswitch_bit_exact(logN, L, dnum):
    """Digit sizes that do not divide the limb count (last digit shorter)."""
    o, cc = make_pair(logN, L, dnum, 9, rot=[1, -2], relin=True)
    for limbs in (L, L - 1, 2):
        x, rx, cx = _fresh(o, cc, 13, limbs)
        assert np.array_equal(cc.EvalRotate(cx, 1).limbs_array(), o.rotate(rx, 1))
        assert np.array_equal(cc.EvalRotate(cx, -2).limbs_array(), o.rotate(rx, -2))
        y, ry, cy = _fresh(o, cc, 14, limbs)
        assert np.array_equal(cc.mul_ct(cx, cy).limbs_array(), o.mul_ct(rx, ry))
        dec = cc.Decrypt(cc.EvalRotate(cx, 1)).GetRealPackedValue()
        assert np.abs(dec - np.roll(x, -1)).max() < 1e-7


def test_full_size_rotation_bit_exact():
    """N = 2^16, 24 limbs, dnum 3 (the block configuration)."""
    o, cc = make_pair(16, 24, 3, 5, rot=[1, 8], relin=False)
    assert np.array_equal(cc.key_array(3, 8), o.switch_key(8))
    x = np.random.default_rng(11).uniform(-1, 1, o.N // 2)
    cc.set_encrypt_counter(3)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    ref = o.encrypt(o.encode(x, 24), 3)
    assert np.array_equal(ct.limbs_array(), ref)
    got = cc.EvalRotate(ct, 8)
    assert np.array_equal(got.limbs_array(), o.rotate(ref, 8))
    dec = cc.Decrypt(got).GetRealPackedValue()
    assert np.abs(dec - np.roll(x, -8)).max() < 1e-6


def test_profiler_reports_every_rotation_kernel(pair10):
    o, cc = pair10
    x, rx, cx = _fresh(o, cc, 12, o.L)
    cc.profile(True)
    cc.profile_reset()
    for _ in range(3):
        cc.EvalRotate(cx, 1)
    rep = cc.profile_report()
    cc.profile(False)
    # ModDown's combine step is the store of the converted limbs' last pass
    for k in ("ntt_fwd_rows", "ntt_fwd_cols", "ntt_inv_cols", "ntt_inv_rows", "modup_conv", "ks_inner",
              "moddown_conv", "ntt_fwd_cols_moddown"):
        assert rep[k]["launches"] >= 3 and rep[k]["ms"] > 0 and rep[k]["bytes"] > 0
    assert rep["ks_inner"]["launches"] == 3
    # operations keep working after the profiler is switched off
    got = cc.EvalRotate(cx, 2)
    assert np.array_equal(got.limbs_array(), o.rotate(rx, 2))


def test_batched_rotations_products_rescales_bit_exact(pair10):
    """ckks_rotate_batch / ckks_mul_ct_batch / ckks_rescale_batch against the
    oracle, with more items than one launch sequence carries (32)."""
    o, cc = pair10
    limbs = 5
    keys = [1, 2, 3, 5, -1, -7, 8, 64, 100, 0]
    items = [_fresh(o, cc, 100 + i, limbs) for i in range(37)]
    ks = [keys[i % len(keys)] for i in range(37)]
    outs = cc.rotate_batch([it[2] for it in items], ks)
    for (x, rx, cx), k, out in zip(items, ks, outs):
        assert np.array_equal(out.limbs_array(), o.rotate(rx, k))
    prods = cc.mul_ct_batch([it[2] for it in items[:35]], [it[2] for it in items[1:36]])
    for i, p in enumerate(prods):
        assert np.array_equal(p.limbs_array(), o.mul_ct(items[i][1], items[i + 1][1]))
    rs = cc.rescale_batch(prods)
    for i, r in enumerate(rs):
        assert np.array_equal(r.limbs_array(), o.rescale(o.mul_ct(items[i][1], items[i + 1][1])))
    with pytest.raises(eng.CKKSError):  # one limb count per batch
        cc.rotate_batch([items[0][2], _fresh(o, cc, 300, 3)[2]], [1, 1])


def test_handles_survive_context_destruction_in_any_order():
    """Destroying a context first orphans its ciphertexts, plaintexts and
    blocks; releasing them afterwards (as a garbage collector may) is safe."""
    import ctypes
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=10, limbs=4, dnum=2, seed=3))
    cc.KeyGen()
    pt = cc.MakeCKKSPackedPlaintext(np.ones(8))
    ct = cc.Encrypt(pt)
    lib = eng.lib()
    eng._check(lib.ckks_ctx_destroy(cc.h))
    cc.h = None
    # orphaned handles: destroy is a host-only release
    assert lib.ckks_ct_destroy(ct.h) == 0
    ct.h = None
    assert lib.ckks_pt_destroy(pt.h) == 0
    pt.h = None


def test_batched_client_encrypt_decrypt(pair10):
    """ckks_encrypt_batch equals successive single encryptions of the oracle
    (counter i for item i); ckks_decrypt_decode_batch equals single decodes."""
    o, cc = pair10
    rng = np.random.default_rng(21)
    xs = [rng.uniform(-1, 1, o.N // 2) for _ in range(5)]
    pts = [cc.MakeCKKSPackedPlaintext(x, level=2) for x in xs]
    cc.set_encrypt_counter(500)
    cts = cc.EncryptBatch(pts)
    for i, (x, ct) in enumerate(zip(xs, cts)):
        assert np.array_equal(ct.limbs_array(), o.encrypt(o.encode(x, o.L - 2), 500 + i))
    dec = cc.DecryptDecodeBatch(cts)
    for i, ct in enumerate(cts):
        single = cc.Decrypt(ct).GetRealPackedValue()
        assert np.abs(dec[i] - single).max() <= 1e-12
        assert np.abs(dec[i] - xs[i]).max() < 1e-8


def test_add_many_and_add_batch_bit_exact(pair10):
    o, cc = pair10
    items = [_fresh(o, cc, 200 + i, 4) for i in range(70)]  # more than one launch of 64
    ref = items[0][1]
    for it in items[1:]:
        ref = o.add(ref, it[1])
    assert np.array_equal(cc.EvalAddMany([it[2] for it in items]).limbs_array(), ref)
    outs = cc.add_batch([it[2] for it in items[:35]], [it[2] for it in items[35:70]])
    for i, out in enumerate(outs):
        assert np.array_equal(out.limbs_array(), o.add(items[i][1], items[35 + i][1]))


# ---- key switches over the reduced special-prime set (alpha = K = 8) -------
WIDE_ROT = [1, 3, 5, 32, -7] + ladder_keys(16, 4)


@pytest.fixture(scope="module")
def pair_wide():
    return make_pair(12, 8, 1, 23, rot=sorted(set(WIDE_ROT)))


def test_reduced_set_keys_bit_exact(pair_wide):
    o, cc = pair_wide
    assert (cc.low_limbs, cc.K_low) == (o.low_limbs, o.K_low) == (3, 3)
    assert np.array_equal(cc.key_array(2), o.switch_key(0))
    assert np.array_equal(cc.key_array(4), o.switch_key_low(0))
    for k in (1, -7, 32):
        assert np.array_equal(cc.key_array(3, k), o.switch_key(k))
        assert np.array_equal(cc.key_array(5, k), o.switch_key_low(k))


@pytest.mark.parametrize("limbs", [1, 2, 3, 4, 5, 8])
def test_key_switches_across_the_reduced_set_boundary(pair_wide, limbs):
    o, cc = pair_wide
    x, rx, cx = _fresh(o, cc, 80 + limbs, limbs)
    y, ry, cy = _fresh(o, cc, 90 + limbs, limbs)
    for k in (1, -7, 32):
        assert np.array_equal(cc.EvalRotate(cx, k).limbs_array(), o.rotate(rx, k))
    outs = cc.EvalFastRotation(cx, [1, 3, 5])
    ref = o.rotate_hoisted(rx, [1, 3, 5])
    for i in range(3):
        assert np.array_equal(outs[i].limbs_array(), ref[i])
    assert np.array_equal(cc.mul_ct(cx, cy).limbs_array(), o.mul_ct(rx, ry))
    got = cc.EvalRotateSum([cx, cy, cx], [0, 3, 5])
    assert np.array_equal(got.limbs_array(), o.rotate_sum(np.stack([rx, ry, rx]), [0, 3, 5]))
    got = cc.EvalMultSum([cx, cy], [cy, cx])
    assert np.array_equal(got.limbs_array(), o.mul_ct_sum(np.stack([rx, ry]), np.stack([ry, rx])))
    rb = cc.rotate_batch([cx, cy], [5, -7])
    assert np.array_equal(rb[0].limbs_array(), o.rotate(rx, 5))
    assert np.array_equal(rb[1].limbs_array(), o.rotate(ry, -7))
    assert np.array_equal(cc.AccumulateSum(cx, 16, 4).limbs_array(), o.accumulate_sum(rx, 16, 4))
