"""The CPU block schedule (oracle/cpu_block.py) on a small ring.

It is the checker of the engine's block stages and the timed CPU path of the
bench's reference arm, so it must evaluate the block: its decrypted output
matches the float64 plaintext block (itself pinned by fixtures from the
reference's manual.py), its stage count is what the bench slices by, and
its protocol counts are the reference's (one packed score tile per
(query group, key group), one weight tile per causal alignment,
simd_layout.protocol_counts).
"""

import numpy as np

from oracle import Oracle, plain_block
from oracle.cpu_block import CpuBlock


def test_cpu_block_schedule_matches_plaintext_block():
    o = Oracle(logN=12, L=24, dnum=3, seed=3)
    o.keygen()
    o.relin_keygen()
    w = plain_block.synthetic_weights(7, d=64, mlp=256)
    x = plain_block.synthetic_input(8, 103, d=64)
    cb = CpuBlock(o, w, 103, heads=1, threads=4, workers=2)
    o.rot_keygen(cb.rotation_indices())
    stages = list(cb.schedule(x))
    assert len(stages) == cb.n_stages()
    assert stages[0] == "encrypt_inputs" and stages[-1] == "decrypt_outputs"
    err = plain_block.rel_inf(plain_block.block(x, w, heads=1), cb.y)
    assert err < 1e-6, err
    # 4 token groups: 10 packed score tiles, 295 weight tiles (+ the client
    # refreshes: 4 inputs, 2 x 4 LayerNorm, 4 x 2 GELU chunks)
    assert cb.ops["score_tile_decryptions"] == 10
    assert cb.ops["client_encryptions"] == 4 + 8 + 295 + 4 * cb.nfc
    assert cb.ops["matrix_products"] == 4 * (3 + 1 + 2 * cb.nfc)
    assert np.isfinite(cb.scores[np.tril(np.ones((103, 103), bool))[:, None, :].repeat(1, axis=1)]).all()
