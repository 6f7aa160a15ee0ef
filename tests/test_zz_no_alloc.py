"""ckks_rotate_noalloc: rotation for callers that cannot allocate device memory.

Such callers (request paths that must not take the allocator's locks,
services on a fixed device-memory budget) pass their
own input and output device buffers; the key-switching temporaries come from
a fixed array inside the library.  These tests check, through the C ABI, that
two such calls in a row give exactly the limbs of the allocating ckks_rotate,
and that a request larger than the fixed array is refused.  The file is
named to be collected last and must also pass alone in a fresh process.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import private_genomic_dnagpt_b200 as eng  # noqa: E402


def _device_copy(arr):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(arr).reshape(-1).view(np.int64).copy()).cuda()
    torch.cuda.synchronize()
    return t


@pytest.mark.parametrize("dnum,levels", [(3, (8, 5)), (1, (8, 3))])
def test_noalloc_rotation_matches_allocating_rotation_twice(dnum, levels):
    import torch
    # dnum 1 (alpha = K = 8): the 3-limb case switches over the reduced set
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=13, limbs=8, dnum=dnum, seed=29))
    cc.KeyGen()
    ks = (1, -3)
    cc.EvalRotateKeyGen(list(ks))
    x = np.random.default_rng(3).uniform(-1, 1, cc.slots)
    for limbs in levels:
        ct = cc.drop_limbs(cc.Encrypt(cc.MakeCKKSPackedPlaintext(x)), limbs)
        src = ct.limbs_array()
        d_in = _device_copy(src)
        for i, k in enumerate(ks):  # two calls in a row through the shared array
            d_out = torch.zeros_like(d_in)
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info()[0]
            eng._check(eng.lib().ckks_rotate_noalloc(cc.h, d_in.data_ptr(), limbs, k, d_out.data_ptr()))
            cc.Synchronize()
            if i > 0:  # after the first call's address lookup, no device memory is taken
                assert torch.cuda.mem_get_info()[0] == free0
            got = d_out.cpu().numpy().view(np.uint64).reshape(src.shape)
            ref = cc.EvalRotate(ct, k).limbs_array()
            assert np.array_equal(got, ref)
            # and it decrypts to the rotated slots
            back = cc.Decrypt(cc.import_ct(got, ct.scale)).GetRealPackedValue()
            assert np.abs(back - np.roll(x, -k)).max() < 1e-6


def test_noalloc_refuses_oversized_and_overlapping_requests():
    import torch
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=13, limbs=8, dnum=3, seed=30))
    cc.KeyGen()
    cc.EvalRotateKeyGen([1])
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(np.ones(16)))
    d = _device_copy(ct.limbs_array())
    with pytest.raises(eng.CKKSError) as e:  # output aliasing the input
        eng._check(eng.lib().ckks_rotate_noalloc(cc.h, d.data_ptr(), 8, 1, d.data_ptr()))
    assert e.value.code == 1
    with pytest.raises(eng.CKKSError) as e:  # no key for this index
        out = torch.zeros_like(d)
        eng._check(eng.lib().ckks_rotate_noalloc(cc.h, d.data_ptr(), 8, 5, out.data_ptr()))
    assert e.value.code == 4
    # the identity is a copy: it needs no key and no scratch
    out = torch.zeros_like(d)
    eng._check(eng.lib().ckks_rotate_noalloc(cc.h, d.data_ptr(), 8, 0, out.data_ptr()))
    cc.Synchronize()
    assert torch.equal(out, d)
    # N = 2^17 with 24 limbs needs ~208 MiB of temporaries: above the fixed array
    big = eng.GenCryptoContext(eng.CCParams(ring_dim_log=17, limbs=24, dnum=3, seed=31))
    buf = torch.zeros(2 * 24 * (1 << 17), dtype=torch.int64, device="cuda")
    out = torch.zeros_like(buf)
    with pytest.raises(eng.CKKSError) as e:
        eng._check(eng.lib().ckks_rotate_noalloc(big.h, buf.data_ptr(), 24, 1, out.data_ptr()))
    assert e.value.code == 7 and "MiB" in str(e.value)
