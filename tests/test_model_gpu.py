"""Chained encrypted blocks and the classifier head on the GPU against the
float64 plaintext model (the reference's 12-block + head driver,
real_dnagpt_fides_scheme_b_simd_full_t103_12blocks_head_cpudiagcache_t123_v3.cpp,
with fhe/multiblock/manual.py as its plaintext oracle).

Gates: hidden states within 1e-6 relative (max-norm) of the plaintext
model, as the single block; the N - A margin within 1e-6 of the plaintext
margin relative to the readout scale.
"""

import numpy as np
import pytest

from oracle import plain_block

pytestmark = pytest.mark.gpu

import private_genomic_dnagpt_b200 as eng  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=16, limbs=24, dnum=3, seed=43))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    return cc


def _margin_tol(hw, m_ref):
    # the margin is a dot product of a unit-variance vector with the readout
    return 1e-6 * max(abs(m_ref), float(np.abs(hw["readout"]).sum()) / 10)


def test_head_matches_plaintext(ctx):
    hw = plain_block.synthetic_head_weights(21)
    head = eng.EncryptedHead(ctx, hw)
    ctx.EvalRotateKeyGen(head.rotation_indices())
    rng = np.random.default_rng(22)
    for _ in range(2):
        h = rng.standard_normal(plain_block.D) * 3.0
        m = head.forward(h)
        m_ref = plain_block.head(h, hw)
        print(f"margin {m:.9f} plaintext {m_ref:.9f}")
        assert abs(m - m_ref) <= _margin_tol(hw, m_ref)


def test_two_chained_blocks_and_head(ctx):
    tokens = 40
    ws = [plain_block.synthetic_weights(31), plain_block.synthetic_weights(32)]
    hw = plain_block.synthetic_head_weights(33)
    x = plain_block.synthetic_input(34, tokens)
    # the second block releases its diagonal cache after each forward
    model = eng.EncryptedModel(ctx, ws, hw, tokens, cached_blocks=1)
    ctx.EvalRotateKeyGen(model.rotation_indices())
    h_ref, m_ref = plain_block.model(x, ws, hw)
    for _ in range(2):  # the second pass re-encodes block 1's diagonals
        h, m = model.forward(x)
        err = plain_block.rel_inf(h_ref, h)
        print(f"two blocks: hidden rel_inf {err:.3e} margin {m:.9f} plaintext {m_ref:.9f}")
        assert np.isfinite(h).all() and err < 1e-6
        assert abs(m - m_ref) <= _margin_tol(hw, m_ref)
    assert model.blocks[0].report()["counts"]["diagonal_cache_mib"] > 0
    assert model.blocks[1].report()["counts"]["diagonal_cache_mib"] == 0


def test_four_chained_blocks_past_the_cache_budget(ctx):
    """Three of four blocks lie past the diagonal-cache budget: they encode
    their diagonals inside every forward and release them after it (the
    12-block model's path for the blocks that do not fit beside the keys)."""
    tokens = 40
    ws = [plain_block.synthetic_weights(41 + b) for b in range(4)]
    hw = plain_block.synthetic_head_weights(45)
    x = plain_block.synthetic_input(46, tokens)
    model = eng.EncryptedModel(ctx, ws, hw, tokens, cached_blocks=1)
    ctx.EvalRotateKeyGen(model.rotation_indices())
    h_ref, m_ref = plain_block.model(x, ws, hw)
    for step in range(2):
        h, m = model.forward(x)
        err = plain_block.rel_inf(h_ref, h)
        print(f"four blocks, pass {step}: hidden rel_inf {err:.3e} margin {m:.9f} plaintext {m_ref:.9f}")
        assert np.isfinite(h).all() and err < 1e-6
        assert abs(m - m_ref) <= _margin_tol(hw, m_ref)
        for b, blk in enumerate(model.blocks):
            c = blk.report()["counts"]
            if b == 0:
                assert c["diagonal_cache_mib"] > 0
                assert c.get("diagonal_cache_misses", 0) == (10 if step == 0 else 0)
            else:  # re-encoded on every pass, released after it
                assert c["diagonal_cache_mib"] == 0
                assert c["diagonal_cache_misses"] == 10
