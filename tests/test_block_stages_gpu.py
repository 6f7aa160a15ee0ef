"""The engine's block evaluation against the CPU block schedule, stage by stage.

``oracle.cpu_block.CpuBlock`` restates the engine's block schedule (the
reference's EncryptedEvaluator::evaluate with its client refreshes,
T123.cpp:762-948) on the oracle.  With the same keys, the same encryption
counters and the same weights, every ciphertext up to the attention scores
is equal bit for bit: the encrypted inputs, LayerNorm (whose client 1/sqrt is
correctly rounded on both sides), the Q/K/V products, and the decrypted
score matrix.  After the softmax (exp differs in its last bits between
libraries) the outputs are compared after decryption.
"""

import numpy as np
import pytest

from oracle import Oracle, plain_block
from oracle.cpu_block import CpuBlock

pytestmark = pytest.mark.gpu

import private_genomic_dnagpt_b200 as eng  # noqa: E402


@pytest.mark.parametrize("log_n,d,heads,mlp,tokens", [(13, 128, 2, 256, 103), (14, 256, 4, 512, 40)])
def test_block_stages_match_cpu_schedule(log_n, d, heads, mlp, tokens):
    import torch
    seed = 61
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=log_n, limbs=24, dnum=3, seed=seed))
    o = Oracle(logN=log_n, L=24, dnum=3, seed=seed)
    cc.KeyGen(); cc.EvalMultKeyGen()
    o.keygen(); o.relin_keygen()
    w = plain_block.synthetic_weights(9, d=d, mlp=mlp)
    x = plain_block.synthetic_input(10, tokens, d=d)
    blk = eng.EncryptedBlock(cc, w, tokens, heads=heads)
    cb = CpuBlock(o, w, tokens, heads=heads)
    rot = blk.rotation_indices()
    assert rot == cb.rotation_indices()
    cc.EvalRotateKeyGen(rot)
    o.rot_keygen(rot)
    G = -(-tokens // 32)
    counter = eng.lib().ckks_get_encrypt_counter(cc.h)
    # engine: inputs, LN1 + Q/K/V, scores, stage by stage
    blk.shard_inputs(x)
    blk.shard_qkv(list(range(G)), 7)
    T, H = tokens, heads
    d_scores = torch.full((T * H * T,), float("nan"), dtype=torch.float64, device="cuda")
    torch.cuda.synchronize()
    blk.shard_scores([(qg, kg) for kg in range(G) for qg in range(kg, G)], d_scores.data_ptr())
    cc.Synchronize()
    gpu_scores = d_scores.cpu().numpy().reshape(T, H, T)
    # CPU schedule up to the softmax
    sched = cb.schedule(x, counter)
    for stage in sched:
        if stage == "softmax":
            break
    for g in range(G):
        xin = blk.state_get(4, g)
        assert xin is not None
        for kind, name in enumerate(("q", "k", "v")):
            got = blk.state_get(kind, g)
            want = cb.state[name][g]
            assert got.limbs == want.limbs and got.scale == want.scale
            assert np.array_equal(got.limbs_array(), want.data), f"{name} of group {g} differs"
    causal = np.tril(np.ones((T, T), bool))[:, None, :].repeat(H, axis=1)
    assert np.isfinite(gpu_scores[causal]).all()
    assert np.array_equal(gpu_scores[causal], cb.scores[causal]), "decrypted scores differ"
    for _ in sched:  # the rest of the CPU block
        pass
    # the engine's whole forward (fresh counters) against the CPU block's output
    y = blk.forward(x)
    ref = plain_block.block(x, w, heads=heads)
    assert plain_block.rel_inf(ref, y) < 1e-6
    assert plain_block.rel_inf(ref, cb.y) < 1e-6
    assert plain_block.rel_inf(cb.y, y) < 1e-6
    rep = blk.report()["counts"]
    assert rep["matrix_products"] == cb.ops["matrix_products"]
    assert rep["score_tile_decryptions"] == cb.ops["score_tile_decryptions"]
