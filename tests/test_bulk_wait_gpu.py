"""Bounded waits of the bulk-copy key products.

The key inner products stage their operands in shared memory with bulk
copies that complete on an mbarrier; every wait on it gives up after one
second, counts a fault on the device, and ckks_sync reports it.  These tests
run the diagnostic kernel through the C ABI: a complete copy comes back
intact, and a barrier that expects more bytes than are copied (a flag that
nothing sets) makes the wait run out, is reported as CKKS_ECUDA, and leaves
the context usable.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import private_genomic_dnagpt_b200 as eng  # noqa: E402


def _ctx():
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=12, limbs=6, dnum=3, seed=41))
    cc.KeyGen()
    cc.EvalRotateKeyGen([5])
    return cc


def test_bulk_copy_round_trip():
    cc = _ctx()
    eng._check(eng.lib().ckks_selftest_bulk_wait(cc.h, 0))
    cc.Synchronize()


def test_starved_wait_is_reported_and_context_stays_usable():
    import time
    cc = _ctx()
    x = np.random.default_rng(5).uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    before = cc.EvalRotate(ct, 5).limbs_array()
    t0 = time.time()
    with pytest.raises(eng.CKKSError) as e:
        eng._check(eng.lib().ckks_selftest_bulk_wait(cc.h, 1))
    assert e.value.code == 3 and "gave up" in str(e.value)
    assert time.time() - t0 < 30.0
    cc.Synchronize()  # the fault was taken by the call that saw it
    after = cc.EvalRotate(ct, 5).limbs_array()
    cc.Synchronize()
    assert np.array_equal(before, after)
    back = cc.Decrypt(cc.import_ct(after, ct.scale)).GetRealPackedValue()
    assert np.abs(back - np.roll(x, -5)).max() < 1e-6
