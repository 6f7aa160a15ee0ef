"""Limb-level parity of the block driver's fused matrix product and lane shift.

The engine's BSGS product (``ckks_bsgs_matmul``: the fused diagonal x
baby-step inner-sum kernels, float64 products on the 50-bit limbs and 128-bit
integer chains on the 60-bit first limb, then the giant steps of all groups
as grouped rotation sums and one batched rescale) and its lane shift
(``ckks_lane_shift``) are compared bit for bit with the oracle's compositions
of the same algorithms (T123.cpp:1005-1059 diagonals, :1264-1295 matmul,
:1297-1314 lane_shift), through the C ABI.  The block evaluation uses the
same device functions for every one of its products and lane shifts.
Decrypted products are also checked against x W^T in float64.
"""

import numpy as np
import pytest

from oracle import Oracle

pytestmark = pytest.mark.gpu

import private_genomic_dnagpt_b200 as eng  # noqa: E402

B = 32


def make_pair(logN, L, dnum, seed, rot):
    o = Oracle(logN=logN, L=L, dnum=dnum, seed=seed)
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=logN, limbs=L, dnum=dnum, seed=seed))
    o.keygen()
    cc.KeyGen()
    o.relin_keygen()
    cc.EvalMultKeyGen()
    o.rot_keygen(list(rot))
    cc.EvalRotateKeyGen(list(rot))
    return o, cc


def bsgs_keys(N, n1):
    pw = N // 2 // B
    n2 = pw // n1
    return [B * j for j in range(1, n1)] + [B * n1 * g for g in range(1, n2)]


def token_rows(rng, pw, d):
    """slot vector of a token group: features < d of every lane, N(0, 1)"""
    x = np.zeros((pw, B))
    x[:d] = rng.standard_normal((d, B))
    return x


def encrypt_groups(o, cc, xs, limbs, counter):
    L = o.L
    cts, refs = [], []
    for i, x in enumerate(xs):
        cts.append(cc.Encrypt(cc.MakeCKKSPackedPlaintext(x.reshape(-1), level=L - limbs)))
        refs.append(o.encrypt(o.encode(x.reshape(-1), limbs), counter + i))
        assert np.array_equal(cts[-1].limbs_array(), refs[-1])
    return cts, refs


def check_products(o, cc, logN, limbs, n1, groups, terms, seed):
    rng = np.random.default_rng(seed)
    pw = o.N // 2 // B
    d = min(pw, 768)
    Ws = [rng.normal(0.0, 0.05, (d - 3 * t, d - t)) for t in range(terms)]  # ragged shapes
    xs = [[token_rows(rng, pw, W.shape[1]) for _ in range(groups)] for W in Ws]
    cts, refs = [], []
    for t in range(terms):
        c, r = encrypt_groups(o, cc, xs[t], limbs, counter=t * groups)
        cts.append(c)
        refs.append(r)
    # baby steps: one hoisted batch per term (the block's babies_of_batch)
    babies = [cc.bsgs_babies(cts[t], B, n1) for t in range(terms)]
    rb = [[[r] + list(o.rotate_hoisted(r, [B * j for j in range(1, n1)])) for r in refs[t]] for t in range(terms)]
    for t in range(terms):
        for q in range(groups):
            for j in (0, 1, n1 - 1):
                assert np.array_equal(babies[t][q][j].limbs_array(), rb[t][q][j])
    diags = [cc.bsgs_diagonals(W, B, n1, limbs) for W in Ws]
    rdiags = [o.bsgs_diagonals(W, B, n1, limbs) for W in Ws]
    got = cc.bsgs_matmul(diags, babies)
    want = o.bsgs_matmul(rdiags, rb, n1, B)
    for q in range(groups):
        assert got[q].limbs == limbs - 1
        assert np.array_equal(got[q].limbs_array(), want[q]), f"group {q} differs from the oracle"
    # the decrypted product is sum_t x_t W_t^T
    for q in (0, groups - 1):
        dec = cc.Decrypt(got[q]).GetRealPackedValue().reshape(pw, B)
        ref = np.zeros((pw, B))
        for t, W in enumerate(Ws):
            ref[:W.shape[0]] += W @ xs[t][q][:W.shape[1]]
        assert np.abs(dec - ref).max() < 1e-6 * max(1.0, np.abs(ref).max())


@pytest.fixture(scope="module")
def pair13():
    # 9 limbs: the 60-bit first prime (integer inner sums) and 8 primes of
    # ~50 bits (float64 inner sums); lane-shift keys for every delta
    rot = set(bsgs_keys(1 << 13, 8)) | set(bsgs_keys(1 << 13, 4)) | set(bsgs_keys(1 << 13, 16))
    for dl in range(1, B):
        rot |= {dl, dl - B}
    return make_pair(13, 9, 3, 41, sorted(rot))


def test_bsgs_matmul_five_groups_bit_exact(pair13):
    # n1 = 8, n2 = 16 (N = 2^13): five groups cross the four-group launch
    o, cc = pair13
    cc.set_encrypt_counter(0)
    check_products(o, cc, 13, limbs=9, n1=8, groups=5, terms=1, seed=1)


def test_bsgs_matmul_summed_terms_bit_exact(pair13):
    # three matrix terms whose inner sums accumulate before one set of giant
    # steps (the block's summed MLP down projection), at 7 limbs
    o, cc = pair13
    cc.set_encrypt_counter(0)
    check_products(o, cc, 13, limbs=7, n1=8, groups=4, terms=3, seed=2)


def test_bsgs_matmul_n1_16_bit_exact(pair13):
    # n1 = 16, n2 = 8: sixteen-baby register kernels, two summed terms
    o, cc = pair13
    cc.set_encrypt_counter(0)
    check_products(o, cc, 13, limbs=9, n1=16, groups=3, terms=2, seed=5)


def test_bsgs_matmul_generic_split_bit_exact(pair13):
    # n1 = 4 takes the generic inner-sum kernels (n2 = 32)
    o, cc = pair13
    cc.set_encrypt_counter(0)
    check_products(o, cc, 13, limbs=5, n1=4, groups=2, terms=1, seed=3)


def test_bsgs_matmul_full_ring_bit_exact():
    # the block's shape: N = 2^16, n1 = n2 = 32, 768 x 768, four token
    # groups sharing every diagonal tile, 9 limbs
    o, cc = make_pair(16, 9, 3, 43, bsgs_keys(1 << 16, 32))
    check_products(o, cc, 16, limbs=9, n1=32, groups=4, terms=1, seed=4)


@pytest.mark.parametrize("limbs", [3, 4, 6])
def test_lane_shift_bit_exact(pair13, limbs):
    # 3 and 4 limbs switch keys over the reduced special-prime set, 6 over all
    o, cc = pair13
    cc.set_encrypt_counter(0)
    rng = np.random.default_rng(limbs)
    pw = o.N // 2 // B
    xs = [rng.standard_normal((pw, B)) for _ in range(3)]
    cts, refs = encrypt_groups(o, cc, xs, limbs, 0)
    deltas = [1, 7, 16, 31]
    got = cc.lane_shift(cts, deltas, B)
    sc = None
    for i in range(len(xs)):
        for k, dl in enumerate(deltas):
            want = o.lane_shift(refs[i], dl, B)
            assert np.array_equal(got[i][k].limbs_array(), want), f"input {i} delta {dl}"
            if i == 0:
                dec = cc.Decrypt(got[i][k]).GetRealPackedValue().reshape(pw, B)
                sc = np.abs(dec - np.roll(xs[i], -dl, axis=1)).max()
                assert sc < 1e-6


def test_bsgs_and_lane_shift_reject_bad_arguments(pair13):
    o, cc = pair13
    W = np.zeros((8, 8))
    with pytest.raises(eng.CKKSError):
        cc.bsgs_diagonals(W, B, 3, 4)  # 3 does not divide the pack width
    with pytest.raises(eng.CKKSError):
        cc.bsgs_diagonals(np.zeros((200, 8)), B, 8, 4)  # more rows than the pack width
    pt = cc.MakeCKKSPackedPlaintext(np.ones(o.N // 2), level=o.L - 4)
    ct = cc.Encrypt(pt)
    with pytest.raises(eng.CKKSError):
        cc.lane_shift([ct], [0], B)
    with pytest.raises(eng.CKKSError):
        cc.lane_shift([ct], [B], B)
    dg = cc.bsgs_diagonals(W, B, 8, 5)  # diagonals at 5 limbs, babies at 4
    babies = cc.bsgs_babies([ct], B, 8)
    with pytest.raises(eng.CKKSError):
        cc.bsgs_matmul([dg], [babies])
