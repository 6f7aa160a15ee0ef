"""One encrypted block sharded over the ranks of a process group.

The reference evaluates a block on one GPU and models multi-GPU splits as
independent, exactly merged units (fhe/gpu_real_scheme_b/shard_layout.py:
Q/K/V per group, MLP partial sums merged by EvalAdd).  Here one block is
split into its independent units -- token groups (LN1 + QKV, and O + LN2 +
MLP, T123.cpp:780-790, 862-927) and the causal alignments (query group, key
group, lane shift) of the score and context tiles (T123.cpp:798-860) -- with
one process per GPU, identical keys
on every rank (same seed) and these exchanges between the stages:

  after QKV      each group's Q, K, V ciphertexts, broadcast by the rank that
                 evaluated the group (every tile needs K/V of its key group
                 and Q of its query group);
  after scores   the score matrix: every rank fills the entries of its
                 tiles into a zero-initialised buffer, an all-reduce sum
                 assembles it (entries are disjoint, so the sum is exact);
  after context  per query group, the partial context sums of all ranks,
                 all-gathered and added with EvalAdd (exact modular adds) by
                 the rank that owns the group;
  at the end     the output rows of every group (disjoint rows, all-reduce
                 sum).

``shard_plan`` is pure host logic; ``ShardedBlock`` drives a block through
an engine adapter, so the same orchestration runs on CPU ranks (gloo) over
a stand-in engine in the tests and on GPU ranks (NCCL) over the engine.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

KIND_Q, KIND_K, KIND_V, KIND_CTX = 0, 1, 2, 3


def active_shifts(tokens: int, batch: int, qg: int, kg: int) -> list[int]:
    """Lane shifts of the causal alignments of a (query group, key group)
    tile, from the engine's schedule (simd_layout.py:386-406)."""
    from . import schedule_active_shifts
    return schedule_active_shifts(tokens, batch, qg, kg)


@dataclass
class RankPlan:
    groups: list[int] = field(default_factory=list)
    # causal alignments (query group, key group, lane shift) of this rank
    tiles: list[tuple[int, int, int]] = field(default_factory=list)
    # alignments per key-group unit assigned (the load balanced)
    load: int = 0


def shard_plan(tokens: int, batch: int, world: int) -> list[RankPlan]:
    """Units of one block for each rank.  Token groups go round-robin.  The
    attention work is split into (key group, lane shift d) units -- every
    query group's alignment with that shift, which share one lane shift of
    the key and value ciphertexts -- assigned longest-processing-time-first by
    their alignment counts (ties to the lowest rank), so every alignment is
    evaluated exactly once and every lane shift on one rank only."""
    if world < 1:
        raise ValueError("world size must be positive")
    groups = -(-tokens // batch)
    plan = [RankPlan() for _ in range(world)]
    for g in range(groups):
        plan[g % world].groups.append(g)
    units: dict[tuple[int, int], list[tuple[int, int, int]]] = {}
    for kg in range(groups):
        for qg in range(kg, groups):
            for d in active_shifts(tokens, batch, qg, kg):
                units.setdefault((kg, d), []).append((qg, kg, d))
    for u in sorted(units, key=lambda u: (-len(units[u]), u)):
        r = min(range(world), key=lambda i: (plan[i].load, i))
        plan[r].tiles.extend(units[u])
        plan[r].load += len(units[u])
    for rp in plan:
        rp.tiles.sort(key=lambda t: (t[1], t[0], t[2]))
    return plan


def group_owner(plan: list[RankPlan], g: int) -> int:
    for r, rp in enumerate(plan):
        if g in rp.groups:
            return r
    raise ValueError(f"group {g} has no owner")


class ShardedBlock:
    """Drives one block through its stages on this rank's units and does the
    exchanges.  ``io`` is the engine adapter (``EngineIO`` for the CKKS
    engine); ``dist`` is torch.distributed with an initialised group."""

    def __init__(self, io, tokens: int, batch: int, heads: int, d_model: int, dist, device):
        self.io, self.dist, self.device = io, dist, device
        self.tokens, self.batch, self.heads, self.d_model = tokens, batch, heads, d_model
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.plan = shard_plan(tokens, batch, self.world)
        self.groups = -(-tokens // batch)

    def _broadcast_state(self, kind: int, g: int, src: int):
        import torch
        io, dist = self.io, self.dist
        if self.rank == src:
            buf, meta = io.state_export(kind, g)
            meta_t = torch.tensor(meta, dtype=torch.float64, device=self.device)
        else:
            meta_t = torch.zeros(3, dtype=torch.float64, device=self.device)
        dist.broadcast(meta_t, src=src)
        meta = tuple(float(v) for v in meta_t.cpu().tolist())
        if self.rank != src:
            buf = io.state_buffer(meta)
        dist.broadcast(buf, src=src)
        if self.rank != src:
            io.state_import(kind, g, buf, meta)

    def _merge_contexts(self, qg: int, owner: int):
        """All-gather every rank's partial context of query group qg (a flag
        and the limbs); the owner sums the present ones."""
        import torch
        io, dist = self.io, self.dist
        meta = io.state_meta(KIND_CTX, qg)  # (limbs, scale, deg) or None
        mt = torch.tensor([1.0, *meta] if meta is not None else [0.0, 0.0, 0.0, 0.0], dtype=torch.float64,
                          device=self.device)
        metas = [torch.zeros_like(mt) for _ in range(self.world)]
        dist.all_gather(metas, mt)
        metas = [tuple(m.cpu().tolist()) for m in metas]
        present = [m for m in metas if m[0] > 0]
        if not present:
            raise RuntimeError(f"no rank evaluated a context tile of query group {qg}")
        ref = present[0][1:]
        for m in present:
            # same limbs and degree; scales equal to the engine's tolerance
            # (a FLEXIBLEAUTO level reduction and a rescaled shift differ in
            # the last bits)
            if m[1] != ref[0] or m[3] != ref[2] or abs(m[2] - ref[1]) > 1e-9 * abs(ref[1]):
                raise RuntimeError("partial contexts at different levels or scales")
        buf = io.state_export(KIND_CTX, qg)[0] if meta is not None else io.state_buffer(ref)
        if meta is None:
            buf.zero_()
        bufs = [torch.empty_like(buf) for _ in range(self.world)]
        dist.all_gather(bufs, buf)
        if self.rank == owner:
            parts = [bufs[r] for r in range(self.world) if metas[r][0] > 0]
            io.state_sum(KIND_CTX, qg, parts, ref)

    def forward(self, x: np.ndarray) -> np.ndarray:
        with self.io.stream():
            return self._forward(x)

    def _forward(self, x: np.ndarray) -> np.ndarray:
        import torch
        io, dist = self.io, self.dist
        mine = self.plan[self.rank]
        io.inputs(x)
        io.qkv(mine.groups)
        for g in range(self.groups):
            src = group_owner(self.plan, g)
            for kind in (KIND_Q, KIND_K, KIND_V):
                self._broadcast_state(kind, g, src)
        scores = torch.zeros(self.tokens * self.heads * self.tokens, dtype=torch.float64, device=self.device)
        io.scores(mine.tiles, scores)
        dist.all_reduce(scores)
        io.softmax(scores)
        io.context(mine.tiles)
        for qg in range(self.groups):
            self._merge_contexts(qg, group_owner(self.plan, qg))
        y = np.zeros((self.tokens, self.d_model), np.float64)
        io.output(mine.groups, y)
        yt = torch.from_numpy(y).to(self.device)
        dist.all_reduce(yt)
        return yt.cpu().numpy()


class EngineIO:
    """Adapter from ShardedBlock to an EncryptedBlock on this rank's GPU: all
    device work on the engine stream, collectives on the same stream."""

    def __init__(self, block):
        self.b, self.cc = block, block.cc

    def stream(self):
        """Makes the engine stream torch's current stream, so buffers and
        collectives are ordered with the engine's kernels."""
        import torch
        return torch.cuda.stream(torch.cuda.ExternalStream(self.cc.stream_handle()))

    def inputs(self, x):
        self.b.shard_inputs(x)

    def qkv(self, groups):
        self.b.shard_qkv(groups)

    def scores(self, tiles, t):
        self.b.shard_scores_tiles(tiles, t.data_ptr())

    def softmax(self, t):
        self.b.shard_softmax(t.data_ptr())

    def context(self, tiles):
        self.b.shard_context_tiles(tiles)

    def output(self, groups, y):
        self.b.shard_output(groups, y)

    def state_meta(self, kind, g):
        ct = self.b.state_get(kind, g)
        return None if ct is None else (float(ct.limbs), float(ct.scale), float(ct.noise_deg))

    def state_buffer(self, meta):
        import torch
        return torch.empty(2 * int(meta[0]) * self.cc.N, dtype=torch.int64, device="cuda")

    def state_export(self, kind, g):
        ct = self.b.state_get(kind, g)
        if ct is None:
            raise RuntimeError(f"state {kind} of group {g} not present")
        meta = (float(ct.limbs), float(ct.scale), float(ct.noise_deg))
        buf = self.state_buffer(meta)
        self.cc.export_device(ct, buf.data_ptr(), buf.numel())
        return buf, meta

    def state_import(self, kind, g, buf, meta):
        ct = self.cc.import_device(buf.data_ptr(), int(meta[0]), meta[1], int(meta[2]))
        self.b.state_set(kind, g, ct)

    def state_sum(self, kind, g, bufs, meta):
        cts = [self.cc.import_device(b.data_ptr(), int(meta[0]), meta[1], int(meta[2])) for b in bufs]
        self.b.state_set(kind, g, cts[0] if len(cts) == 1 else self.cc.EvalAddMany(cts))
