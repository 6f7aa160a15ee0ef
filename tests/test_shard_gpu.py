"""Exchange paths on the GPU: device-to-device ciphertext transfer, the
binary wire format of ciphertexts and keys, block state access, and one
block sharded over two GPUs with NCCL (skipped with fewer than two GPUs).
"""

import os
import socket

import numpy as np
import pytest

from oracle import plain_block

pytestmark = pytest.mark.gpu

import private_genomic_dnagpt_b200 as eng  # noqa: E402


def _ctx(L=6, seed=7):
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=12, limbs=L, dnum=3, seed=seed))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    cc.EvalRotateKeyGen([1, 5])
    return cc


def test_device_transfer_and_wire_format_round_trip():
    import torch
    cc = _ctx()
    rng = np.random.default_rng(1)
    v = rng.uniform(-1, 1, cc.slots)
    ct = cc.EvalMult(cc.Encrypt(cc.MakeCKKSPackedPlaintext(v)), cc.Encrypt(cc.MakeCKKSPackedPlaintext(v)))
    ref = ct.limbs_array()
    # device buffer, on the engine stream
    buf = torch.zeros(2 * ct.limbs * cc.N, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    cc.export_device(ct, buf.data_ptr(), buf.numel())
    back = cc.import_device(buf.data_ptr(), ct.limbs, ct.scale, ct.noise_deg)
    assert np.array_equal(back.limbs_array(), ref) and back.scale == ct.scale
    assert back.noise_deg == ct.noise_deg
    # wire format: bytes survive, metadata checked
    data = cc.serialize(ct)
    ct2 = cc.deserialize(data)
    assert np.array_equal(ct2.limbs_array(), ref) and ct2.scale == ct.scale
    assert ct2.noise_deg == ct.noise_deg
    with pytest.raises(eng.CKKSError):
        cc.deserialize(data[:100])
    bad = bytearray(data)
    bad[48] ^= 1  # first modulus
    with pytest.raises(eng.CKKSError):
        cc.deserialize(bytes(bad))
    other = _ctx(L=5)  # same ring, different chain length: same first moduli
    ct3 = other.deserialize(data) if ct.limbs <= 5 else None
    if ct3 is not None:
        assert np.array_equal(ct3.limbs_array(), ref)
    big = eng.GenCryptoContext(eng.CCParams(ring_dim_log=13, limbs=6, dnum=3, seed=7))
    with pytest.raises(eng.CKKSError):
        big.deserialize(data)


def test_key_wire_format_moves_a_rotation_key_between_contexts():
    a = _ctx(seed=7)
    b = eng.GenCryptoContext(eng.CCParams(ring_dim_log=12, limbs=6, dnum=3, seed=7))
    b.KeyGen()  # same seed: same secret key, no switching keys yet
    b.deserialize_key(a.serialize_key(0))
    b.deserialize_key(a.serialize_key(5))
    rng = np.random.default_rng(2)
    v = rng.uniform(-1, 1, a.slots)
    ca = a.Encrypt(a.MakeCKKSPackedPlaintext(v))
    cb = b.import_ct(ca.limbs_array(), ca.scale)
    ra, rb = a.EvalRotate(ca, 5), b.EvalRotate(cb, 5)
    assert np.array_equal(ra.limbs_array(), rb.limbs_array())
    ma, mb = a.EvalMult(ca, ca), b.EvalMult(cb, cb)
    assert np.array_equal(ma.limbs_array(), mb.limbs_array())


def test_block_state_get_set_round_trip():
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=16, limbs=24, dnum=3, seed=51))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    tokens = 40
    w = plain_block.synthetic_weights(5)
    x = plain_block.synthetic_input(6, tokens)
    blk = eng.EncryptedBlock(cc, w, tokens)
    cc.EvalRotateKeyGen(blk.rotation_indices())
    blk.shard_inputs(x)
    blk.shard_qkv([0, 1])
    q0 = blk.state_get(0, 0)
    assert q0 is not None and blk.state_get(3, 0) is None
    blk.state_set(0, 1, q0)
    assert np.array_equal(blk.state_get(0, 1).limbs_array(), q0.limbs_array())
    # a full staged forward equals the plaintext block
    y = blk.forward(x)
    ref = plain_block.block(x, w)
    assert plain_block.rel_inf(ref, y) < 1e-6
    # the output stage split as an owner and a helper would: MLP chunks
    # [2, 3) and [0, 2) evaluated apart, their sums added with EvalAdd
    assert blk.mlp_chunks == 3
    blk.shard_mlp([0, 1], 2, 3)
    tail = [blk.state_get(5, g) for g in (0, 1)]
    blk.shard_mlp([0, 1], 0, 2)
    for g in (0, 1):
        blk.state_set(5, g, cc.EvalAdd(blk.state_get(5, g), tail[g]))
    y2 = np.zeros_like(y)
    blk.shard_finish([0, 1], y2)
    assert plain_block.rel_inf(ref, y2) < 1e-6
    # a projection evaluated alone equals the batched one (LN1 encrypts
    # fresh refreshes, so the ciphertexts differ in their noise)
    v_all = cc.DecryptDecodeBatch([blk.state_get(2, 1)])[0]
    blk.state_set(2, 1, cc._new())
    assert blk.state_get(2, 1) is None
    blk.shard_qkv([1], 4)
    assert blk.state_get(1, 1) is not None
    v_one = cc.DecryptDecodeBatch([blk.state_get(2, 1)])[0]
    assert np.abs(v_one - v_all).max() <= 1e-6 * np.abs(v_all).max()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, tokens, out):
    import datetime

    import torch
    import torch.distributed as dist
    from private_genomic_dnagpt_b200 import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", rank))
    try:
        cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=16, limbs=24, dnum=3, seed=61, device=rank))
        cc.KeyGen()
        cc.EvalMultKeyGen()
        w = plain_block.synthetic_weights(5)
        x = plain_block.synthetic_input(6, tokens)
        blk = eng.EncryptedBlock(cc, w, tokens)
        cc.EvalRotateKeyGen(blk.rotation_indices())
        sb = shard.ShardedBlock(shard.EngineIO(blk), tokens, 32, 12, plain_block.D, dist, "cuda")
        y = sb.forward(x)
        if rank == 0:
            np.save(out, y)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not __import__("torch").cuda.is_available() or __import__("torch").cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("tokens", [103, 32])
def test_block_sharded_over_two_gpus(tmp_path, tokens):
    """103 tokens: two owners of token groups; 32 tokens: one group, its
    owner (Q, K, MLP chunks 0-1) and a helper (V, MLP chunk 2)."""
    import torch.multiprocessing as mp
    out = str(tmp_path / "y.npy")
    mp.start_processes(_rank, args=(2, _free_port(), tokens, out), nprocs=2, join=True, start_method="spawn")
    y = np.load(out)
    ref = plain_block.block(plain_block.synthetic_input(6, tokens), plain_block.synthetic_weights(5))
    err = plain_block.rel_inf(ref, y)
    print(f"{tokens} tokens sharded over 2 GPUs: rel_inf {err:.3e}")
    assert err < 1e-6


def _model_rank(rank, world, port, tokens, out):
    import datetime

    import torch
    import torch.distributed as dist
    from private_genomic_dnagpt_b200 import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", rank))
    try:
        cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=16, limbs=24, dnum=3, seed=62, device=rank))
        cc.KeyGen()
        cc.EvalMultKeyGen()
        ws = [plain_block.synthetic_weights(30 + b) for b in range(2)]
        hw = plain_block.synthetic_head_weights(39)
        x = plain_block.synthetic_input(6, tokens)
        model = eng.EncryptedModel(cc, ws, hw, tokens, cached_blocks=1)
        cc.EvalRotateKeyGen(model.rotation_indices())
        sm = shard.ShardedModel([shard.EngineIO(b) for b in model.blocks], model.head, tokens, 32, 12, plain_block.D,
                                dist, "cuda", cached_blocks=1)
        h, m = sm.forward(x)
        np.save(out + f".{rank}.npy", np.concatenate([h.ravel(), [m]]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not __import__("torch").cuda.is_available() or __import__("torch").cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_block_model_sharded_over_two_gpus(tmp_path):
    """Two chained blocks (the second releasing its diagonals after use) and
    the head, sharded over two GPUs with NCCL."""
    import torch.multiprocessing as mp
    tokens = 70
    out = str(tmp_path / "m")
    mp.start_processes(_model_rank, args=(2, _free_port(), tokens, out), nprocs=2, join=True, start_method="spawn")
    ws = [plain_block.synthetic_weights(30 + b) for b in range(2)]
    h_ref, m_ref = plain_block.model(plain_block.synthetic_input(6, tokens), ws, plain_block.synthetic_head_weights(39))
    for r in range(2):
        got = np.load(out + f".{r}.npy")
        err = plain_block.rel_inf(h_ref, got[:-1].reshape(h_ref.shape))
        print(f"rank {r}: hidden rel_inf {err:.3e}, margin {got[-1]:.6f} vs {m_ref:.6f}")
        assert err < 1e-6 and abs(got[-1] - m_ref) < 1e-6
