"""Sharding one block over ranks: the unit plan and the exchange protocol on
CPU ranks (gloo, world size 2) over a float64 stand-in engine.

The stand-in evaluates each stage of the plaintext block (oracle/plain_block)
on exactly the units it is given, and keeps its per-group state (Q, K, V
rows, partial contexts, MLP partial sums) as tensors that the orchestration
exchanges; so the sharded output equals the unsharded block only if every
unit is evaluated once and every exchange (state broadcast, score
all-reduce, partial-context merge, MLP merge, output all-reduce) moves the
right data.
"""

import contextlib
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import plain_block
from private_genomic_dnagpt_b200 import shard

B = 32


def test_plan_covers_every_unit_once():
    for tokens in (1, 31, 40, 103, 256):
        groups = -(-tokens // B)
        want = {(qg, kg, d) for kg in range(groups) for qg in range(kg, groups)
                for d in shard.active_shifts(tokens, B, qg, kg)}
        for world in range(1, 9):
            plan = shard.shard_plan(tokens, B, world)
            assert len(plan) == world
            gs = [g for rp in plan for g in rp.groups]
            assert sorted(gs) == list(range(groups))
            ts = [t for rp in plan for t in rp.tiles]
            assert len(ts) == len(want) and set(ts) == want
            # a lane shift of a key group lives on one rank only
            owner = {}
            for r, rp in enumerate(plan):
                for qg, kg, d in rp.tiles:
                    assert owner.setdefault((kg, d), r) == r
            loads = [len(rp.tiles) for rp in plan]
            assert loads == [rp.load for rp in plan]
            assert max(loads) - min(loads) <= groups


def test_plan_splits_projections_and_mlp_chunks():
    for tokens in (1, 40, 103, 256):
        groups = -(-tokens // B)
        for world in range(1, 12):
            for chunks in (1, 2, 3, 4):
                plan = shard.shard_plan(tokens, B, world, chunks)
                for g in range(groups):
                    # each projection of each group on exactly one rank
                    for part in (shard.PART_Q, shard.PART_K, shard.PART_V):
                        assert sum(bool(rp.qkv.get(g, 0) & part) for rp in plan) == 1
                    # the chunk ranges tile [0, chunks), the owner's first
                    ranks = shard.mlp_ranks(plan, g)
                    assert ranks[0] == shard.group_owner(plan, g)
                    spans = sorted(plan[r].mlp[g] for r in ranks)
                    assert spans[0][0] == 0 and spans[-1][1] == chunks
                    assert all(a[1] == b[0] and a[0] < a[1] for a, b in zip(spans, spans[1:]))
                    assert plan[ranks[0]].mlp[g][0] == 0
                    helped = groups + g < world
                    assert len([rp for rp in plan if g in rp.qkv]) == (2 if helped else 1)


def test_plan_for_the_benchmark_shape():
    plan = shard.shard_plan(103, B, 8)
    assert [rp.groups for rp in plan] == [[0], [1], [2], [3], [], [], [], []]
    assert [rp.qkv for rp in plan] == [{0: 3}, {1: 3}, {2: 3}, {3: 3}, {0: 4}, {1: 4}, {2: 4}, {3: 4}]
    assert [rp.mlp for rp in plan] == [{0: (0, 2)}, {1: (0, 2)}, {2: (0, 2)}, {3: (0, 2)},
                                       {0: (2, 3)}, {1: (2, 3)}, {2: (2, 3)}, {3: (2, 3)}]
    total = sum(len(shard.active_shifts(103, B, qg, kg)) for kg in range(4) for qg in range(kg, 4))
    assert sum(rp.load for rp in plan) == total == 295
    assert max(rp.load for rp in plan) - min(rp.load for rp in plan) <= 4


class PlainIO:
    """Float64 stand-in engine: the plaintext block, stage by stage."""

    def __init__(self, w, tokens, heads=12):
        self.w, self.T, self.H = w, tokens, heads
        self.D = w["ln1"].shape[0]
        self.hd = self.D // heads
        self.state = {}

    def stream(self):
        return contextlib.nullcontext()

    def rows(self, g):
        return slice(g * B, min(self.T, (g + 1) * B))

    def inputs(self, x):
        self.x = np.asarray(x, np.float64)
        self.state = {}

    # MLP hidden units per chunk (one plaintext width of the engine)
    CHUNK = 1024

    @property
    def mlp_chunks(self):
        return -(-self.w["mlp_fc"].shape[0] // self.CHUNK)

    def qkv(self, groups, parts):
        D = self.D
        for g in groups:
            h1 = plain_block.layer_norm(self.x[self.rows(g)], self.w["ln1"])
            qkv = h1 @ self.w["attn_qkv"].T
            for kind in range(3):
                if parts & (1 << kind):
                    self.state[(kind, g)] = qkv[:, kind * D:(kind + 1) * D].copy()

    def _entries(self, qg, kg, d):
        """(query row in group, key row in group) of alignment (qg, kg, d):
        query lane ql meets key lane (ql + d) mod B, kept when causal."""
        for ql in range(B):
            kl = (ql + d) % B
            tq, tk = qg * B + ql, kg * B + kl
            if tq < self.T and tk < self.T and tk <= tq:
                yield ql, kl, tq, tk

    def scores(self, tiles, t):
        s = t.view(self.T, self.H, self.T)
        for qg, kg, d in tiles:
            q = self.state[(0, qg)].reshape(-1, self.H, self.hd)
            k = self.state[(1, kg)].reshape(-1, self.H, self.hd)
            for ql, kl, tq, tk in self._entries(qg, kg, d):
                s[tq, :, tk] = torch.from_numpy((q[ql] * k[kl]).sum(-1) / math.sqrt(self.hd))

    def softmax(self, t):
        s = t.view(self.T, self.H, self.T).numpy().transpose(1, 0, 2)
        mask = np.tril(np.ones((self.T, self.T), bool))
        s = np.where(mask[None], s, -np.inf)
        p = np.exp(s - s.max(-1, keepdims=True))
        self.p = p / p.sum(-1, keepdims=True)  # [H, T, T]

    def context(self, tiles):
        for qg, kg, d in tiles:
            v = self.state[(2, kg)].reshape(-1, self.H, self.hd)
            rq = self.rows(qg)
            part = np.zeros((rq.stop - rq.start, self.H, self.hd))
            for ql, kl, tq, tk in self._entries(qg, kg, d):
                part[ql] += self.p[:, tq, tk][:, None] * v[kl]
            key = (3, qg)
            self.state[key] = self.state.get(key, 0) + part.reshape(-1, self.D)

    def mlp(self, groups, c0, c1):
        for g in groups:
            r1 = self.x[self.rows(g)] + self.state[(3, g)] @ self.w["attn_proj"].T
            h2 = plain_block.layer_norm(r1, self.w["ln2"])
            cols = slice(c0 * self.CHUNK, c1 * self.CHUNK)
            hid = plain_block.gelu_tanh(h2 @ self.w["mlp_fc"][cols].T)
            self.state[(6, g)] = r1
            self.state[(5, g)] = hid @ self.w["mlp_proj"][:, cols].T

    def finish(self, groups, y):
        for g in groups:
            y[self.rows(g)] = self.state[(6, g)] + self.state[(5, g)]

    def release_cache(self):
        pass

    def state_meta(self, kind, g):
        a = self.state.get((kind, g))
        return None if a is None else (float(a.shape[0]), 1.0, 1.0)

    def state_buffer(self, meta):
        return torch.zeros(int(meta[0]) * self.D, dtype=torch.float64)

    def state_export(self, kind, g):
        a = self.state[(kind, g)]
        return torch.from_numpy(a.reshape(-1).copy()), (float(a.shape[0]), 1.0, 1.0)

    def state_import(self, kind, g, buf, meta):
        self.state[(kind, g)] = buf.numpy().reshape(int(meta[0]), self.D).copy()

    def state_sum(self, kind, g, bufs, meta):
        self.state[(kind, g)] = sum(b.numpy().reshape(int(meta[0]), self.D) for b in bufs)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, tokens, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = plain_block.synthetic_weights(3)
        x = plain_block.synthetic_input(4, tokens)
        sb = shard.ShardedBlock(PlainIO(w, tokens), tokens, B, 12, plain_block.D, dist, "cpu")
        y = sb.forward(x)
        if rank == 0:
            np.save(out_path, y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,tokens", [(2, 40), (2, 70), (3, 70), (5, 70), (6, 103), (8, 103)])
def test_sharded_block_over_gloo_ranks_equals_the_block(tmp_path, world, tokens):
    out = str(tmp_path / "y.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), tokens, out), nprocs=world, join=True,
                       start_method="spawn")
    y = np.load(out)
    ref = plain_block.block(plain_block.synthetic_input(4, tokens), plain_block.synthetic_weights(3))
    assert np.abs(y - ref).max() <= 1e-12 * np.abs(ref).max()


class PlainHead:
    def __init__(self, hw):
        self.hw = hw

    def forward(self, x_last):
        return plain_block.head(x_last, self.hw)


def _model_rank(rank, world, port, tokens, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ws = [plain_block.synthetic_weights(20 + b) for b in range(2)]
        hw = plain_block.synthetic_head_weights(29)
        x = plain_block.synthetic_input(4, tokens)
        m = shard.ShardedModel([PlainIO(w, tokens) for w in ws], PlainHead(hw), tokens, B, 12, plain_block.D,
                               dist, "cpu", cached_blocks=1)
        h, margin = m.forward(x)
        np.save(out_path + f".{rank}.npy", np.concatenate([h.ravel(), [margin]]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 5])
def test_sharded_two_block_model_with_head(tmp_path, world):
    """Two chained blocks sharded over the ranks with the refresh between
    them, and the head on rank 0: every rank ends with the plaintext
    model's hidden state and margin."""
    tokens = 70
    out = str(tmp_path / "m")
    mp.start_processes(_model_rank, args=(world, _free_port(), tokens, out), nprocs=world, join=True,
                       start_method="spawn")
    ws = [plain_block.synthetic_weights(20 + b) for b in range(2)]
    h_ref, m_ref = plain_block.model(plain_block.synthetic_input(4, tokens), ws, plain_block.synthetic_head_weights(29))
    for r in range(world):
        got = np.load(out + f".{r}.npy")
        assert np.abs(got[:-1] - h_ref.ravel()).max() <= 1e-12 * np.abs(h_ref).max()
        assert abs(got[-1] - m_ref) <= 1e-12 * max(1.0, abs(m_ref))


class MismatchedIO(PlainIO):
    """A helper whose partial MLP sum claims another scale than the owner's."""

    def state_export(self, kind, g):
        buf, meta = super().state_export(kind, g)
        return buf, (meta[0], 2.0 if kind == shard.KIND_MLP else meta[1], meta[2])


def _mismatch_rank(rank, world, port, tokens, out_path):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        w = plain_block.synthetic_weights(3)
        x = plain_block.synthetic_input(4, tokens)
        plan = shard.shard_plan(tokens, B, world)
        helper = any(len(shard.mlp_ranks(plan, g)) > 1 and rank in shard.mlp_ranks(plan, g)[1:]
                     for g in range(-(-tokens // B)))
        io = MismatchedIO(w, tokens) if helper else PlainIO(w, tokens)
        sb = shard.ShardedBlock(io, tokens, B, 12, plain_block.D, dist, "cpu")
        try:
            sb.forward(x)
            outcome = "finished"
        except RuntimeError as e:
            outcome = "raised" if "partial" in str(e) else f"other: {e}"
        with open(out_path + f".{rank}", "w") as f:
            f.write(outcome)
    finally:
        dist.destroy_process_group()


def test_mismatched_partial_sums_end_every_rank(tmp_path):
    """A partial MLP sum at another scale is found on its owner; every rank
    raises at the same collective step (none waits for the timeout)."""
    world, tokens = 5, 70
    out = str(tmp_path / "o")
    mp.start_processes(_mismatch_rank, args=(world, _free_port(), tokens, out), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        with open(out + f".{r}") as f:
            assert f.read() == "raised", r
