"""Host-side helpers of bench.py that shape its JSON line (no GPU)."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_keyswitch_bytes_is_the_algorithmic_figure(bench):
    # l + 2 beta (l + K) + 2 l limbs: 264 limbs of 512 KiB at l = 24, K = 8, alpha = 8
    assert bench.keyswitch_bytes(24, 8, 8, 1 << 16) == 264 * 8 * (1 << 16)
    # a partial last digit still counts as a digit (beta = ceil(l / alpha))
    assert bench.keyswitch_bytes(17, 8, 8, 1 << 16) == (17 + 2 * 3 * 25 + 34) * 8 * (1 << 16)


def test_ntt_launch_sizes_buckets_by_limbs(bench):
    limb = 19  # log2 of 8 * 2^16 bytes
    prof = {
        "ntt_fwd_rows": {"by_size": {str(limb + 3): [4, 1.0], str(limb + 7): [2, 5.0]}},
        "ntt_inv_cols": {"by_size": {str(limb + 3): [1, 0.5], str(limb - 2): [3, 0.3]}},
        "modup_conv": {"by_size": {str(limb + 3): [9, 9.0]}},  # not an NTT pass
    }
    got = bench.ntt_launch_sizes(prof, 16)
    assert got == {"2^0": [3, 0.3], "2^3": [5, 1.5], "2^7": [2, 5.0]}
    assert list(got) == ["2^0", "2^3", "2^7"]  # ascending limb buckets
    # the bucket offset follows the ring degree
    assert bench.ntt_launch_sizes({"ntt_fwd_cols": {"by_size": {"20": [1, 2.0]}}}, 13) == {"2^4": [1, 2.0]}
    assert bench.ntt_launch_sizes({}, 16) == {}


def test_traffic_per_limb_is_about_two_limbs(bench):
    # one read and one write of each limb per pass (512 KiB each), within 5 %
    for name, per_limb in bench.NCU_TRAFFIC_PER_LIMB.items():
        assert 0.95 * 2 * 8 * (1 << 16) < per_limb < 1.05 * 2 * 8 * (1 << 16), name
