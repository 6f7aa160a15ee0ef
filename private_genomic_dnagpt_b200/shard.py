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
                 evaluated them (every tile needs K/V of its key group and
                 Q of its query group);
  after scores   the score matrix: every rank fills the entries of its
                 tiles into a zero-initialised buffer, an all-reduce sum
                 assembles it (entries are disjoint, so the sum is exact);
  after context  per query group, the partial context sums of all ranks,
                 all-gathered and added with EvalAdd (exact modular adds) by
                 the ranks that evaluate the group's MLP;
  after the MLP  a helper's partial MLP sum, broadcast and added with
                 EvalAdd by the group's owner;
  at the end     the output rows of every group (disjoint rows, all-reduce
                 sum).

With more ranks than token groups, group g also gets a helper rank
(groups + g): the owner evaluates the Q and K projections and the first MLP
chunks, the helper the V projection and the remaining chunks (both evaluate
the O projection and LN2 the chunks need), as in shard_layout.py's split of
the projections and of the MLP into exactly merged partial sums.

``shard_plan`` is pure host logic; ``ShardedBlock`` drives a block through
an engine adapter, so the same orchestration runs on CPU ranks (gloo) over
a stand-in engine in the tests and on GPU ranks (NCCL) over the engine.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

KIND_Q, KIND_K, KIND_V, KIND_CTX, KIND_X, KIND_MLP, KIND_RES = 0, 1, 2, 3, 4, 5, 6
PART_Q, PART_K, PART_V = 1, 2, 4


def active_shifts(tokens: int, batch: int, qg: int, kg: int) -> list[int]:
    """Lane shifts of the causal alignments of a (query group, key group)
    tile, from the engine's schedule (simd_layout.py:386-406)."""
    from . import schedule_active_shifts
    return schedule_active_shifts(tokens, batch, qg, kg)


@dataclass
class RankPlan:
    # token groups this rank owns: their output rows are decrypted here
    groups: list[int] = field(default_factory=list)
    # causal alignments (query group, key group, lane shift) of this rank
    tiles: list[tuple[int, int, int]] = field(default_factory=list)
    # alignments per key-group unit assigned (the load balanced)
    load: int = 0
    # group -> projections evaluated here (PART_Q | PART_K | PART_V)
    qkv: dict[int, int] = field(default_factory=dict)
    # group -> MLP chunks [begin, end) evaluated here
    mlp: dict[int, tuple[int, int]] = field(default_factory=dict)


def shard_plan(tokens: int, batch: int, world: int, mlp_chunks: int = 3) -> list[RankPlan]:
    """Units of one block for each rank.  Token groups go round-robin to
    owners; with more ranks than groups, rank groups + g helps group g (V and
    the last floor(chunks / 2) MLP chunks; the owner keeps Q, K and the first
    chunks).  The attention work is split into (key group, lane shift d)
    units -- every query group's alignment with that shift, which share one
    lane shift of the key and value ciphertexts -- assigned
    longest-processing-time-first by their alignment counts (ties to the
    lowest rank), so every alignment is evaluated exactly once and every lane
    shift on one rank only."""
    if world < 1:
        raise ValueError("world size must be positive")
    if mlp_chunks < 1:
        raise ValueError("the MLP has at least one chunk")
    groups = -(-tokens // batch)
    plan = [RankPlan() for _ in range(world)]
    for g in range(groups):
        owner = plan[g % world]
        owner.groups.append(g)
        h = groups + g
        if h < world:
            split = mlp_chunks - mlp_chunks // 2
            owner.qkv[g] = PART_Q | PART_K
            owner.mlp[g] = (0, split)
            plan[h].qkv[g] = PART_V
            if split < mlp_chunks:
                plan[h].mlp[g] = (split, mlp_chunks)
        else:
            owner.qkv[g] = PART_Q | PART_K | PART_V
            owner.mlp[g] = (0, mlp_chunks)
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


def part_source(plan: list[RankPlan], g: int, part: int) -> int:
    """The rank that evaluates projection `part` of group g."""
    for r, rp in enumerate(plan):
        if rp.qkv.get(g, 0) & part:
            return r
    raise ValueError(f"projection {part} of group {g} is not assigned")


def mlp_ranks(plan: list[RankPlan], g: int) -> list[int]:
    """Ranks that evaluate MLP chunks of group g, the owner first."""
    owner = group_owner(plan, g)
    return [owner] + [r for r, rp in enumerate(plan) if g in rp.mlp and r != owner]


class ShardedBlock:
    """Drives one block through its stages on this rank's units and does the
    exchanges.  ``io`` is the engine adapter (``EngineIO`` for the CKKS
    engine); ``dist`` is torch.distributed with an initialised group."""

    def __init__(self, io, tokens: int, batch: int, heads: int, d_model: int, dist, device):
        self.io, self.dist, self.device = io, dist, device
        self.tokens, self.batch, self.heads, self.d_model = tokens, batch, heads, d_model
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.plan = shard_plan(tokens, batch, self.world, io.mlp_chunks)
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

    @staticmethod
    def _check_meta(present):
        ref = present[0]
        for m in present:
            # same limbs and degree; scales equal to the engine's tolerance
            # (a FLEXIBLEAUTO level reduction and a rescaled shift differ in
            # the last bits)
            if m[0] != ref[0] or m[2] != ref[2] or abs(m[1] - ref[1]) > 1e-9 * abs(ref[1]):
                raise RuntimeError("partial sums at different levels or scales")
        return ref

    def _merge_contexts(self, qg: int, sinks: list[int]):
        """All-gather every rank's partial context of query group qg (a flag
        and the limbs); the ranks in `sinks` sum the present ones."""
        import torch
        io, dist = self.io, self.dist
        meta = io.state_meta(KIND_CTX, qg)  # (limbs, scale, deg) or None
        mt = torch.tensor([1.0, *meta] if meta is not None else [0.0, 0.0, 0.0, 0.0], dtype=torch.float64,
                          device=self.device)
        metas = [torch.zeros_like(mt) for _ in range(self.world)]
        dist.all_gather(metas, mt)
        metas = [tuple(m.cpu().tolist()) for m in metas]
        present = [m[1:] for m in metas if m[0] > 0]
        if not present:
            raise RuntimeError(f"no rank evaluated a context tile of query group {qg}")
        ref = self._check_meta(present)
        buf = io.state_export(KIND_CTX, qg)[0] if meta is not None else io.state_buffer(ref)
        if meta is None:
            buf.zero_()
        bufs = [torch.empty_like(buf) for _ in range(self.world)]
        dist.all_gather(bufs, buf)
        if self.rank in sinks:
            parts = [bufs[r] for r in range(self.world) if metas[r][0] > 0]
            io.state_sum(KIND_CTX, qg, parts, ref)

    def _merge_mlp(self, g: int, ranks: list[int]):
        """Every helper in `ranks[1:]` broadcasts its partial MLP sum of
        group g; the owner ranks[0] adds them to its own with EvalAdd."""
        import torch
        io, dist = self.io, self.dist
        owner = ranks[0]
        parts = [io.state_export(KIND_MLP, g)] if self.rank == owner else []
        for src in ranks[1:]:
            if self.rank == src:
                buf, meta = io.state_export(KIND_MLP, g)
                meta_t = torch.tensor(meta, dtype=torch.float64, device=self.device)
            else:
                meta_t = torch.zeros(3, dtype=torch.float64, device=self.device)
            dist.broadcast(meta_t, src=src)
            meta = tuple(float(v) for v in meta_t.cpu().tolist())
            if self.rank != src:
                buf = io.state_buffer(meta)
            dist.broadcast(buf, src=src)
            if self.rank == owner:
                parts.append((buf, meta))
        # the owner checks that the parts add up and tells every rank, so
        # that a mismatch ends all ranks together instead of leaving the
        # others in their next collective until the timeout
        ok = torch.ones(1, dtype=torch.float64, device=self.device)
        err = None
        if self.rank == owner:
            try:
                ref = self._check_meta([m for _, m in parts])
            except RuntimeError as e:
                err = e
                ok.zero_()
        dist.broadcast(ok, src=owner)
        if err is not None:
            raise err
        if float(ok.cpu()[0]) == 0.0:
            raise RuntimeError(f"partial MLP sums of group {g} do not match on rank {owner}")
        if self.rank == owner:
            io.state_sum(KIND_MLP, g, [b for b, _ in parts], ref)

    def forward(self, x: np.ndarray) -> np.ndarray:
        with self.io.stream():
            return self._forward(x)

    def _forward(self, x: np.ndarray) -> np.ndarray:
        import torch
        io, dist = self.io, self.dist
        mine = self.plan[self.rank]
        io.inputs(x)
        by_parts: dict[int, list[int]] = {}
        for g, parts in sorted(mine.qkv.items()):
            by_parts.setdefault(parts, []).append(g)
        for parts, gs in sorted(by_parts.items()):
            io.qkv(gs, parts)
        for g in range(self.groups):
            for kind, part in ((KIND_Q, PART_Q), (KIND_K, PART_K), (KIND_V, PART_V)):
                self._broadcast_state(kind, g, part_source(self.plan, g, part))
        scores = torch.zeros(self.tokens * self.heads * self.tokens, dtype=torch.float64, device=self.device)
        io.scores(mine.tiles, scores)
        dist.all_reduce(scores)
        io.softmax(scores)
        io.context(mine.tiles)
        for qg in range(self.groups):
            self._merge_contexts(qg, mlp_ranks(self.plan, qg))
        by_chunks: dict[tuple[int, int], list[int]] = {}
        for g, chunks in sorted(mine.mlp.items()):
            by_chunks.setdefault(chunks, []).append(g)
        for (c0, c1), gs in sorted(by_chunks.items()):
            io.mlp(gs, c0, c1)
        for g in range(self.groups):
            ranks = mlp_ranks(self.plan, g)
            if len(ranks) > 1:
                self._merge_mlp(g, ranks)
        y = np.zeros((self.tokens, self.d_model), np.float64)
        io.finish(mine.groups, y)
        yt = torch.from_numpy(y).to(self.device)
        dist.all_reduce(yt)
        return yt.cpu().numpy()


class ShardedModel:
    """Chained blocks, each sharded over the ranks (``ShardedBlock``), with
    the client's full-hidden-state refresh between blocks -- the decrypted
    output of one block is the next block's input (the 12-block driver's
    refresh, 12blocks_head_cpudiagcache_t123_v3.cpp:452-470) -- and the
    classifier head on the last token, evaluated by rank 0 and broadcast
    (V3:480-510).  ``ios`` holds one engine adapter per block; blocks with
    index >= ``cached_blocks`` drop their encoded diagonals after each use
    (``io.release_cache()``)."""

    def __init__(self, ios, head, tokens: int, batch: int, heads: int, d_model: int, dist, device,
                 cached_blocks: int | None = None):
        self.blocks = [ShardedBlock(io, tokens, batch, heads, d_model, dist, device) for io in ios]
        self.head, self.dist, self.device = head, dist, device
        self.rank = dist.get_rank()
        self.cached_blocks = len(ios) if cached_blocks is None else cached_blocks

    def forward(self, x: np.ndarray):
        """Returns (hidden [tokens, D] of the last block, head margin or None)
        on every rank."""
        import torch
        h = np.asarray(x, np.float64)
        for i, sb in enumerate(self.blocks):
            h = sb.forward(h)
            if i >= self.cached_blocks:
                sb.io.release_cache()
        if self.head is None:
            return h, None
        m = torch.zeros(1, dtype=torch.float64, device=self.device)
        if self.rank == 0:
            m[0] = self.head.forward(h[-1])
        self.dist.broadcast(m, src=0)
        return h, float(m.cpu()[0])


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

    @property
    def mlp_chunks(self) -> int:
        return self.b.mlp_chunks

    def qkv(self, groups, parts):
        self.b.shard_qkv(groups, parts)

    def scores(self, tiles, t):
        self.b.shard_scores_tiles(tiles, t.data_ptr())

    def softmax(self, t):
        self.b.shard_softmax(t.data_ptr())

    def context(self, tiles):
        self.b.shard_context_tiles(tiles)

    def mlp(self, groups, chunk_begin, chunk_end):
        self.b.shard_mlp(groups, chunk_begin, chunk_end)

    def release_cache(self):
        self.b.release_cache()

    def finish(self, groups, y):
        self.b.shard_finish(groups, y)

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
