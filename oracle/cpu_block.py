"""The encrypted block's schedule on the CPU oracle.

TEST INFRASTRUCTURE AND TIMED CPU PATH ONLY: ``tests/`` use it as the checker
of the engine's block stages, ``bench.py`` times it as the CPU path of the
reference's algorithm (its ``--impl reference`` arm and ``cpu_baseline``).
Nothing in ``private_genomic_dnagpt_b200`` imports it.

It restates, operation by operation, the server schedule of the reference's
EncryptedEvaluator::evaluate with its client refreshes
(fhe/gpu_real_scheme_b/src/real_dnagpt_fides_scheme_b_simd_full_t103_depth13_
digits3_ring65536_cpudiagcache_t123.cpp, "T123.cpp", :762-948 and :509-715) in
the form the engine evaluates it:

- slot(feature f, lane t) = f * B + t, B = 32 tokens per ciphertext (T123.cpp
  :419-426 with one copy), PW = N / (2 B) features;
- LayerNorm (T123.cpp:1168-1181): the feature sums as base-4 window sums
  (the AccumulateSum ladder, :1154-1159, one rotation sum per step), the
  mean, the centered input, the variance at low level, the client's exact
  1/sqrt, the product; the gain folded into the next matrix;
- Q/K/V, O, MLP fc and down projections as BSGS products
  (matmul + cached_diagonal_plains, :1005-1059, :1264-1295), the diagonals
  encoded at the babies' level for every product (the reference encodes
  them inside its block evaluation too), the down projections' inner sums
  added before one set of giant steps;
- scores (:795-834): key lane shifts (:1297-1314), query x key products,
  head-window sums on a base-8 ladder, the causal isolation mask with
  1/sqrt(64), every alignment of a (query group, key group) tile packed into
  one ciphertext by a rotation sum and decrypted once; the client's exact
  causal softmax (:629-665);
- context (:838-860): value lane shifts, the client's weight tiles, the sum
  of tile x shifted value products with one relinearisation per query group;
- residuals, LN2, fc chunks, the client's exact tanh-GELU (:190-194), down
  projections, the output decryption.

Levels follow the engine (the input at 11 limbs, every refresh at the
fewest limbs its remaining depth needs), and every ciphertext of the server
schedule is the engine's bit for bit until the first client refresh whose
float64 function is not correctly rounded (softmax's exp, GELU's tanh):
LayerNorm's 1/sqrt and every integer operation are exact on both sides.

``CpuBlock.schedule(x)`` is a generator that yields after every operation
group, so that a caller can run the block in consecutive timed slices.
"""

from __future__ import annotations

import math
import os
import threading
from concurrent.futures import ThreadPoolExecutor
from decimal import ROUND_HALF_UP, Decimal

import numpy as np

from . import Oracle, lib

HEAD_RADIX = 8
EPS = 1e-5


class CT:
    """A ciphertext on the oracle: limbs (2, l, N), scale and noise degree."""

    __slots__ = ("data", "scale", "deg")

    def __init__(self, data: np.ndarray, scale: float, deg: int = 1):
        self.data = data
        self.scale = float(scale)
        self.deg = deg

    @property
    def limbs(self) -> int:
        return self.data.shape[1]


def llround(v: float) -> int:
    """C's llround: nearest integer, halves away from zero."""
    return int(Decimal(v).quantize(Decimal(1), rounding=ROUND_HALF_UP))


def gelu(u: np.ndarray) -> np.ndarray:
    """tanh-GELU (T123.cpp:190-194)."""
    return 0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u * u * u)))


class CpuBlock:
    """One DNAGPT block (pre-LN, bias-free) evaluated on the oracle with the
    engine's schedule.  weights: ln1, attn_qkv [3D, D], attn_proj [D, D],
    ln2, mlp_fc [MLP, D], mlp_proj [D, MLP] (PyTorch [out, in] layout)."""

    LX = 11  # limbs of the encrypted input

    def __init__(self, o: Oracle, weights: dict, tokens: int, heads: int = 12, batch: int = 32,
                 threads: int = 0, workers: int = 0):
        self.o = o
        # independent ciphertexts run on a pool of `workers` host threads, each
        # operation inside with threads // workers OpenMP threads (the oracle
        # parallelises over limbs only, and most of the block runs at 2..4)
        threads = threads or os.cpu_count() or 1
        workers = workers or max(1, threads // 4)
        per = max(1, threads // workers)
        self.threads, self.workers = threads, workers
        self.pool = ThreadPoolExecutor(workers, initializer=lambda: lib().oc_set_threads(per))
        D = weights["ln1"].shape[0]
        self.D, self.T, self.H = D, tokens, heads
        self.HD = D // heads
        self.MLP = weights["mlp_fc"].shape[0]
        self.B = batch
        self.PW = o.N // 2 // batch
        n1 = 32
        while n1 * n1 > self.PW:
            n1 //= 2
        self.n1, self.n2 = n1, self.PW // n1
        self.G = -(-tokens // batch)
        self.nfc = -(-self.MLP // self.PW)
        qkv = np.asarray(weights["attn_qkv"], np.float64) * np.asarray(weights["ln1"], np.float64)[None, :]
        fc = np.asarray(weights["mlp_fc"], np.float64) * np.asarray(weights["ln2"], np.float64)[None, :]
        proj2 = np.asarray(weights["mlp_proj"], np.float64)
        self.W = {0: qkv[:D], 1: qkv[D:2 * D], 2: qkv[2 * D:], 3: np.asarray(weights["attn_proj"], np.float64)}
        for c in range(self.nfc):
            self.W[4 + c] = fc[c * self.PW:min((c + 1) * self.PW, self.MLP)]
            self.W[4 + self.nfc + c] = proj2[:, c * self.PW:min((c + 1) * self.PW, self.MLP)]
        self.counter = 0
        self.ops = {}
        self._lock = threading.Lock()

    def pmap(self, fn, items):
        """[fn(x) for x in items], the items on the worker pool."""
        items = list(items)
        if len(items) <= 1:
            return [fn(x) for x in items]
        return list(self.pool.map(fn, items))

    # ---- primitives with the engine's scale bookkeeping --------------------
    def S(self, limbs: int) -> float:
        return self.o.scale(limbs)

    def _count(self, name: str, n: int = 1):
        with self._lock:
            self.ops[name] = self.ops.get(name, 0) + n

    def plain(self, values: np.ndarray, limbs: int) -> np.ndarray:
        return self.o.encode(values, limbs, self.S(limbs))

    def feature_plain(self, per_feature: np.ndarray, limbs: int) -> np.ndarray:
        return self.plain(np.repeat(per_feature, self.B), limbs)

    def mul_pt(self, a: CT, pt: np.ndarray, pt_scale: float) -> CT:
        self._count("ct_plain")
        return CT(self.o.mul_pt(a.data, pt), a.scale * pt_scale, a.deg + 1)

    def mul_ct(self, a: CT, b: CT) -> CT:
        self._count("ct_ct")
        return CT(self.o.mul_ct(a.data, b.data), a.scale * b.scale, a.deg + b.deg)

    def rescale(self, a: CT) -> CT:
        q = float(self.o.moduli[a.limbs - 1])
        return CT(self.o.rescale(a.data), a.scale / q, max(a.deg - 1, 1))

    def add(self, a: CT, b: CT) -> CT:
        assert a.limbs == b.limbs and a.deg == b.deg
        return CT(self.o.add(a.data, b.data), a.scale, a.deg)

    def sub(self, a: CT, b: CT) -> CT:
        assert a.limbs == b.limbs and a.deg == b.deg
        return CT(self.o.sub(a.data, b.data), a.scale, a.deg)

    def level_reduce(self, x: CT, limbs: int) -> CT:
        """FLEXIBLEAUTO level reduction: an integer multiply bringing the
        scale to the target level's, one rescale, dropped limbs."""
        if x.deg >= 2:
            x = self.rescale(x)
        if x.limbs == limbs:
            return x
        self._count("level_reduce")
        ql = float(self.o.moduli[x.limbs - 1])
        c = llround(self.S(limbs) * ql / x.scale)
        t = CT(self.o.mul_int(x.data, c), x.scale * float(c), 2)
        r = self.rescale(t)
        if r.limbs > limbs:
            r = CT(np.ascontiguousarray(r.data[:, :limbs]), r.scale, r.deg)
        return r

    def lower(self, x: CT, limbs: int) -> CT:
        return self.level_reduce(x, limbs) if x.limbs > limbs else x

    def window_sums(self, xs, window: int, radix: int):
        return self.pmap(lambda x: CT(self.o.window_sum(x.data, window, self.B, radix), x.scale, x.deg), xs)

    def babies(self, x: CT):
        """baby steps x, rot(x, B j) for j < n1 (one hoisted set)."""
        r = self.o.rotate_hoisted(x.data, [self.B * j for j in range(1, self.n1)])
        self._count("rotations", self.n1 - 1)
        return [x] + [CT(np.ascontiguousarray(r[j]), x.scale, x.deg) for j in range(self.n1 - 1)]

    def lane_shift(self, x: CT, d: int) -> CT:
        self._count("rotations", 2)
        self._count("ct_plain", 2)
        sc = self.S(x.limbs)
        return CT(self.o.lane_shift(x.data, d, self.B), x.scale * sc / float(self.o.moduli[x.limbs - 1]), 1)

    # ---- client role -----------------------------------------------------------
    def client_encrypt(self, vals: np.ndarray, limbs: int):
        """encode + encrypt every row of vals (M x N/2) at `limbs` limbs with
        the next M encryption counters."""
        sc = self.S(limbs)
        pts = self.o.encode_batch(vals, limbs, sc)
        c0 = self.counter
        self.counter += len(vals)
        self._count("client_encryptions", len(vals))
        return self.pmap(lambda m: CT(self.o.encrypt(pts[m], c0 + m), sc, 1), range(len(vals)))

    def client_decrypt(self, cts) -> np.ndarray:
        self._count("client_decryptions", len(cts))
        return np.stack(self.pmap(lambda c: self.o.decode(self.o.decrypt(c.data), c.scale), cts))

    # ---- compositions ------------------------------------------------------------
    def bsgs(self, babies_terms, ids):
        """sum_t x_{t,q} W_{ids[t]}^T for every group q from the baby steps
        babies_terms[t][q]: every term's diagonals encoded at the babies'
        level, the inner sums of all terms added, one set of giant steps."""
        limbs = babies_terms[0][0][0].limbs
        G = len(babies_terms[0])
        sc = self.S(limbs)
        diags = []
        for i in ids:
            diags.append(self.o.bsgs_diagonals(self.W[i], self.B, self.n1, limbs))
            self._count("matrix_products", G)
            self._count("ct_plain", G * self.n1 * self.n2)
            self._count("diagonal_encodes", self.n1 * self.n2)
            yield "diagonals"
        ks = [self.B * self.n1 * g for g in range(self.n2)]

        def group(q):
            inner = None
            for t, dg in enumerate(diags):
                inner = self.o.bsgs_inner(np.stack([b.data for b in babies_terms[t][q]]), dg, self.n1, inner)
            b0 = babies_terms[0][q][0]
            prod = CT(self.o.rotate_sum(inner, ks), b0.scale * sc, b0.deg + 1)
            self._count("rotations", self.n2 - 1)
            return self.rescale(prod)

        self._last = self.pmap(group, range(G))
        yield "bsgs_groups"

    def layernorm(self, xs, active):
        lx = xs[0].limbs
        invd = np.zeros(self.PW)
        invd[:self.D] = 1.0 / self.D
        sums = self.window_sums(xs, self.PW, 4)
        self._count("accumulate_sum", len(xs))
        yield "ln_sums"
        p = self.feature_plain(invd, lx)

        def center(i):  # x - mean, and its square at 4 limbs (only decrypted)
            mean = self.rescale(self.mul_pt(sums[i], p, self.S(lx)))
            c = self.sub(self.level_reduce(xs[i], lx - 1), mean)
            low = self.lower(c, 4)
            return c, self.rescale(self.mul_ct(low, low))

        cs = self.pmap(center, range(len(xs)))
        centered = [c for c, _ in cs]
        yield "ln_square"
        sqsum = self.window_sums([q for _, q in cs], self.PW, 4)
        self._count("accumulate_sum", len(xs))
        pv = self.feature_plain(invd, sqsum[0].limbs)

        def variance(s):
            v = self.rescale(self.mul_pt(s, pv, self.S(s.limbs)))
            return CT(self.o.add_const(v.data, EPS, v.scale), v.scale, v.deg)

        var = self.pmap(variance, sqsum)
        yield "ln_variance"
        dv = 1.0 / np.sqrt(self.client_decrypt(var))
        inv = self.client_encrypt(dv, lx - 1)
        self._count("client_round_trips", len(xs))
        self._last = self.pmap(lambda i: self.rescale(self.mul_ct(centered[i], inv[i])), range(len(xs)))
        yield "ln_product"

    def lane_shifts(self, x: CT, deltas, target: int):
        res = self.pmap(lambda d: self.level_reduce(x, target) if d == 0 else self.lane_shift(x, d), deltas)
        return dict(zip(deltas, res))

    def active_shifts(self, qg: int, kg: int):
        """lane shifts whose (query lane, key lane) pairs include a causal one
        (simd_layout.py:386-406)."""
        B, T = self.B, self.T
        qs, ks = qg * B, kg * B
        qc, kc = min(B, T - qs), min(B, T - ks)
        out = []
        for d in range(B):
            for ql in range(qc):
                kl = (ql + d) % B
                if kl < kc and ks + kl <= qs + ql:
                    out.append(d)
                    break
        return out

    def n_stages(self) -> int:
        """the number of stage names schedule() yields (its slices)"""
        return 26 + 5 * self.G + 3 * self.nfc

    def rotation_indices(self):
        """every rotation index the schedule uses (the block driver's
        required_rotation_keys, T123.cpp:455-481, for this layout)."""
        slots = self.PW * self.B

        def canon(k):
            r = k % slots
            return r - slots if r > slots // 2 else r

        v = [canon(self.B * j) for j in range(1, self.n1)]
        v += [canon(self.B * self.n1 * g) for g in range(1, self.n2)]
        step = 1
        while step < self.PW:
            v += [canon(self.B * step * m) for m in range(1, 4) if step * m < self.PW]
            step *= 4
        for d in range(1, self.B):
            v += [canon(d), canon(d - self.B), canon(d * self.B)]
        step = 1
        while step < self.HD:
            v += [canon(self.B * step * m) for m in range(1, HEAD_RADIX) if step * m < self.HD]
            step *= HEAD_RADIX
        return sorted(set(v) - {0})

    # ---- the block ---------------------------------------------------------------
    def schedule(self, x: np.ndarray, counter: int = 0):
        """Generator over the block evaluation of x ([T, D]); yields a stage
        name after every operation group; the output ([T, D], decrypted)
        is left in self.y and the Q/K/V ciphertexts in self.state."""
        B, D, T, G, PW, H, HD = self.B, self.D, self.T, self.G, self.PW, self.H, self.HD
        self.counter = counter
        self.ops = {}
        self.state = {}
        act = [min(B, T - g * B) for g in range(G)]
        # client: pack and encrypt the embeddings (T123.cpp:1642-1661)
        vals = np.zeros((G, PW, B))
        for g in range(G):
            rows = x[g * B:g * B + act[g]]
            vals[g, :D, :act[g]] = rows.T
        xs = self.client_encrypt(vals.reshape(G, -1), self.LX)
        yield "encrypt_inputs"
        # LN1 + Q/K/V (T123.cpp:780-790)
        yield from self.layernorm(xs, act)
        nrm = self._last
        bab = self.pmap(self.babies, nrm)
        yield "qkv_babies"
        qkv = []
        for w in range(3):
            yield from self.bsgs([bab], [w])
            qkv.append(self._last)
        del bab
        Q, K, V = qkv
        self.state = {"q": Q, "k": K, "v": V}
        # scores (T123.cpp:795-834)
        tiles = [(qg, kg, d) for kg in range(G) for qg in range(kg, G) for d in self.active_shifts(qg, kg)]
        scores = np.full((T, H, T), np.nan)
        inv_sqrt_hd = 1.0 / math.sqrt(HD)
        qr = {}
        for kg in range(G):
            tags = [t for t in tiles if t[1] == kg]
            if not tags:
                continue
            lks = min(Q[tags[0][0]].limbs - 1, 3)
            need = list(dict.fromkeys(t[2] for t in tags))
            ks = self.lane_shifts(self.lower(K[kg], lks + 1), need, lks)
            yield "key_lane_shifts"
            qgs = list(dict.fromkeys(t[0] for t in tags))
            new = [qg for qg in qgs if qg not in qr]
            qr.update(zip(new, self.pmap(lambda qg: self.level_reduce(Q[qg], lks), new)))

            def isolated(tag):
                # Q * shifted K, the head-window sums, the causal mask with
                # 1/sqrt(HD) at feature h*HD
                qg, _, d = tag
                prod = self.rescale(self.mul_ct(qr[qg], ks[d]))
                hs = CT(self.o.window_sum(prod.data, HD, B, HEAD_RADIX), prod.scale, prod.deg)
                v = np.zeros((PW, B))
                for ql in range(B):
                    q, k = qg * B + ql, kg * B + (ql + d) % B
                    if q < T and k < T and k <= q:
                        v[np.arange(H) * HD, ql] = inv_sqrt_hd
                return self.rescale(self.mul_pt(hs, self.plain(v.reshape(-1), hs.limbs), self.S(hs.limbs)))

            iso = self.pmap(isolated, tags)
            yield "score_products"
            st = []
            parts_of = []
            for vi, qg in enumerate(qgs):
                parts = [(iso[i], tags[i][2]) for i in range(len(tags)) if tags[i][0] == qg]
                st += [(qg, kg, d, vi) for (_, d) in parts]
                self._count("rotations", len(parts))
                parts_of.append(parts)

            def pack(parts):  # every alignment of the tile moved to h*HD - d, one ciphertext
                data = self.o.rotate_sum(np.stack([p[0].data for p in parts]), [d * B for (_, d) in parts])
                return CT(data, parts[0][0].scale, parts[0][0].deg)

            packed = self.pmap(pack, parts_of)
            dv = self.client_decrypt(packed).reshape(len(packed), PW, B)
            for (qg, kg_, d, vi) in st:
                for ql in range(B):
                    kl = (ql + d) % B
                    q, k = qg * B + ql, kg_ * B + kl
                    if q >= T or k >= T or k > q:
                        continue
                    f = (np.arange(H) * HD - d + PW) % PW
                    scores[q, :, k] = dv[vi, f, ql]
            self._count("score_tile_decryptions", len(packed))
            yield "score_tiles"
        self.scores = scores
        # client: exact causal softmax (T123.cpp:629-665)
        prob = np.zeros((T, H, T))
        for q in range(T):
            row = scores[q, :, :q + 1]
            assert np.isfinite(row).all(), "missing causal attention score"
            e = np.exp(row - row.max(axis=1, keepdims=True))
            prob[q, :, :q + 1] = e / e.sum(axis=1, keepdims=True)
        yield "softmax"
        # context (T123.cpp:838-860)
        lhs = [[] for _ in range(G)]
        rhs = [[] for _ in range(G)]
        for kg in range(G):
            tags = [t for t in tiles if t[1] == kg]
            if not tags:
                continue
            lk = V[kg].limbs - 1
            need = list(dict.fromkeys(t[2] for t in tags))
            vs = self.lane_shifts(V[kg], need, lk)
            yield "value_lane_shifts"
            w = np.zeros((len(tags), PW, B))
            for m, (qg, _, d) in enumerate(tags):
                for ql in range(B):
                    q, k = qg * B + ql, kg * B + (ql + d) % B
                    if q < T and k < T and k <= q:
                        w[m, :D, ql] = prob[q, np.arange(D) // HD, k]
            wa = self.client_encrypt(w.reshape(len(tags), -1), lk)
            for m, (qg, _, d) in enumerate(tags):
                lhs[qg].append(wa[m])
                rhs[qg].append(vs[d])
            yield "weight_tiles"
        def context(qg):  # sum of the tiles' products, one relinearisation
            a, b = lhs[qg], rhs[qg]
            data = self.o.mul_ct_sum(np.stack([c.data for c in a]), np.stack([c.data for c in b]))
            self._count("ct_ct", len(a))
            return self.rescale(CT(data, a[0].scale * b[0].scale, a[0].deg + b[0].deg))

        ctx = self.pmap(context, range(G))
        yield "context"
        # O projection, residual, LN2, MLP (T123.cpp:862-927)
        ob = self.pmap(self.babies, ctx)
        yield "o_babies"
        yield from self.bsgs([ob], [3])
        o_ = self._last
        del ob
        r1 = self.pmap(lambda g: self.add(self.level_reduce(xs[g], o_[g].limbs), o_[g]), range(G))
        yield from self.layernorm(r1, act)
        n2 = self._last
        fb = self.pmap(self.babies, n2)
        yield "fc_babies"
        hc = []
        for c in range(self.nfc):
            yield from self.bsgs([fb], [4 + c])
            hc.append(self._last)
        del fb
        flat = [hc[c][g] for g in range(G) for c in range(self.nfc)]
        dv = self.client_decrypt(flat).reshape(G, self.nfc, PW, B)
        out = np.zeros_like(dv)
        for g in range(G):
            for c in range(self.nfc):
                odim = min(PW, self.MLP - c * PW)
                out[g, c, :odim, :act[g]] = gelu(dv[g, c, :odim, :act[g]])
        ge = self.client_encrypt(out.reshape(G * self.nfc, -1), 3)
        self._count("client_round_trips", G * self.nfc)
        yield "gelu"
        gb = self.pmap(self.babies, ge)
        yield "down_babies"
        db = [[gb[g * self.nfc + c] for g in range(G)] for c in range(self.nfc)]
        yield from self.bsgs(db, [4 + self.nfc + c for c in range(self.nfc)])
        mlp = self._last
        del gb, db
        outs = self.pmap(lambda g: self.add(self.level_reduce(r1[g], mlp[g].limbs), mlp[g]), range(G))
        dv = self.client_decrypt(outs).reshape(G, PW, B)
        y = np.zeros((T, D))
        for g in range(G):
            y[g * B:g * B + act[g]] = dv[g, :D, :act[g]].T
        self.y = y
        yield "decrypt_outputs"

    def forward(self, x: np.ndarray, counter: int = 0) -> np.ndarray:
        for _ in self.schedule(x, counter):
            pass
        return self.y
