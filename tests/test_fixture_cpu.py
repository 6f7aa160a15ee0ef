"""The reference's float64 fixture format (CPU only).

tests/golden/fixture_small/ was written by the reference's own array writer
(fhe/multiblock/export_fixture.py `_write_array`, generator
tests/golden/make_golden.py) from seeded synthetic weights, so reading it
back pins the loader to the reference's format; the package's writer must
produce directories the loader (and so the reference's readers) accept.
"""

import json
import os
import shutil

import numpy as np
import pytest

from oracle import plain_block
from private_genomic_dnagpt_b200 import fixture

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fixture_small")


def _expected():
    blocks = [plain_block.synthetic_weights(60 + b, d=16, mlp=64) for b in range(2)]
    head = plain_block.synthetic_head_weights(62, d=16)
    x = plain_block.synthetic_input(63, 3, d=16)
    return blocks, head, x


def test_loads_a_fixture_written_by_the_reference_writer():
    fx = fixture.load_fixture(GOLD)
    blocks, head, x = _expected()
    assert fx.num_blocks == 2
    for b in range(2):
        got = fx.block_weights(b)
        for f in fixture.BLOCK_FIELDS:
            assert got[f].shape == blocks[b][f].shape and np.array_equal(got[f], blocks[b][f]), (b, f)
    h = fx.head_weights()
    for k in ("final_ln", "head_linear", "head_ln", "readout"):
        assert np.array_equal(h[k], head[k]), k
    assert np.array_equal(fx.embeddings(), x)
    # the plaintext model runs from the loaded arrays (2 heads of 8 features)
    hid, m = plain_block.model(fx.embeddings(), [fx.block_weights(b) for b in range(2)], h, heads=2)
    ref_h, ref_m = plain_block.model(x, blocks, head, heads=2)
    assert np.array_equal(hid, ref_h) and m == ref_m


def test_writer_round_trip_and_format(tmp_path):
    blocks, head, x = _expected()
    d = tmp_path / "fx"
    fixture.export_fixture(d, fixture.model_arrays(blocks, head, x))
    fx = fixture.load_fixture(d)
    assert fx.num_blocks == 2 and np.array_equal(fx.embeddings(), x)
    mine = json.loads((d / "manifest.json").read_text())["arrays"]
    ref = json.loads(open(os.path.join(GOLD, "manifest.json")).read())["arrays"]
    assert set(mine) == set(ref)
    for name in ref:
        for key in ("file", "dtype", "endianness", "order", "shape", "elements", "bytes", "sha256"):
            assert mine[name][key] == ref[name][key], (name, key)
    with pytest.raises(fixture.FixtureError):
        fixture.export_fixture(d, {"a": np.ones(2)})  # manifest exists


def test_rejects_tampered_or_truncated_arrays(tmp_path):
    d = tmp_path / "fx"
    shutil.copytree(GOLD, d)
    path = d / fixture.array_filename("weights.block1.ln2")
    raw = bytearray(path.read_bytes())
    raw[3] ^= 0x40
    path.write_bytes(bytes(raw))
    with pytest.raises(fixture.FixtureError):
        fixture.load_fixture(d)
    fixture.load_fixture(d, verify=False)  # size still right
    path.write_bytes(bytes(raw[:-8]))
    with pytest.raises(fixture.FixtureError):
        fixture.load_fixture(d, verify=False)
