"""Encrypted DNAGPT block on the GPU against the float64 plaintext oracle.

North-star gate: decrypted block output within 1e-6 relative (max-norm) of
the plaintext block (the reference gates at 4e-2 and measures ~4.6e-9,
T123.cpp:1405-1440).  Shapes: D = 768, 12 heads, MLP 3072, N = 2^16 with the
24-limb chain and dnum = 3; seeded synthetic weights N(0, 0.02) and
embeddings N(0, 1) clipped to +-4.
"""

import numpy as np
import pytest

from oracle import plain_block

pytestmark = pytest.mark.gpu

import private_genomic_dnagpt_b200 as eng  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=16, limbs=24, dnum=3, seed=41))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    return cc


@pytest.mark.parametrize("tokens", [40, 103])
def test_block_matches_plaintext_oracle(ctx, tokens):
    w = plain_block.synthetic_weights(5)
    x = plain_block.synthetic_input(6, tokens)
    blk = eng.EncryptedBlock(ctx, w, tokens)
    ctx.EvalRotateKeyGen(blk.rotation_indices())
    y = blk.forward(x)
    ref = plain_block.block(x, w)
    err = plain_block.rel_inf(ref, y)
    worst = max(plain_block.rel_inf(ref[t], y[t]) for t in range(tokens))
    rep = blk.report()
    print(f"T={tokens} global rel_inf {err:.3e} worst-token {worst:.3e} {rep}")
    assert np.isfinite(y).all()
    assert err < 1e-6 and worst < 1e-6
    c = rep["counts"]
    groups = -(-tokens // 32)
    assert c["matrix_products"] == 10 * groups
    # one packed score tile per (query group, key group), one weight tile per
    # alignment: the reference's protocol counts (simd_layout.protocol_counts,
    # 10 and 295 at T = 103)
    assert c["score_tile_decryptions"] == groups * (groups + 1) // 2
    alignments = sum(len(eng.schedule_active_shifts(tokens, 32, q, k)) for q in range(groups)
                     for k in range(q + 1))
    assert c["weight_tile_encryptions"] == alignments
    if tokens == 103:
        assert (c["score_tile_decryptions"], c["weight_tile_encryptions"]) == (10, 295)


@pytest.mark.parametrize("log_n,d,heads,mlp", [(13, 128, 2, 256), (14, 256, 4, 512)])
def test_block_on_smaller_rings(log_n, d, heads, mlp):
    """Fewer slots per ciphertext: 8 (N = 2^13) and 16 (N = 2^14) baby steps
    per product instead of 32."""
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=log_n, limbs=24, dnum=3, seed=43))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    tokens = 40
    w = plain_block.synthetic_weights(7, d=d, mlp=mlp)
    x = plain_block.synthetic_input(8, tokens, d=d)
    blk = eng.EncryptedBlock(cc, w, tokens, heads=heads)
    cc.EvalRotateKeyGen(blk.rotation_indices())
    y = blk.forward(x)
    err = plain_block.rel_inf(plain_block.block(x, w, heads=heads), y)
    print(f"N=2^{log_n} D={d}: rel_inf {err:.3e}")
    assert np.isfinite(y).all() and err < 1e-6
