"""Benchmark of the encrypted DNAGPT block hot path on B200.

Headline (first part of the metric): encrypted block latency in seconds
for one DNAGPT-0.1B-shaped block at 103 tokens, N = 2^16, 24-limb chain
(60 + 23 x 50-bit primes), dnum = 3 -- the single-block configuration.  One
step is one block: client encryption of the 103 embeddings (32 tokens per
ciphertext), the server schedule with its client refreshes (LayerNorm
1/sqrt, softmax, GELU), client decryption.  Synthetic data: weights
N(0, 0.02) in [out, in] layout, unit LN gains, embeddings N(0,1) clipped to
+-4 (seeded; the real GSR fixture is not available).

  value      device-timed (CUDA events on the engine stream) span from
             encrypted inputs resident to encrypted outputs resident,
             seconds per block (lower is better), max over ranks;
  e2e        the whole C-ABI call with host buffers: host embeddings in,
             host outputs out, per block; e2e.cold_weights the same call
             with the weights' BSGS diagonals encoded inside it;
  roofline   the dominant kernel of the block (event-timed launches and
             their algorithmic bytes) against the measured HBM bandwidth;
             roofline.keyswitch: EvalRotate/s and key-switch GB/s on the
             primitive configuration (N = 2^16, 24 limbs, dnum 3, indices
             1..512);
  cpu_baseline  the same block on the CPU oracle (oracle/cpu_block.py, the
             engine's schedule restated on the CPU restatement of the
             reference's CKKS operations) on this host's cores, timed in
             full, once.
`--impl reference` times that CPU block as the reference arm (the
reference's own CPU path, OpenFHE under FIDESlib's API, is not in its tree;
the oracle port stands in): the whole block once, executed as --steps
consecutive slices of its stages, value = the sum of the slices.
Under torchrun the block is sharded over the ranks (token groups and
attention tiles split, NCCL exchanges between the stages; strong scaling,
`value` = latency of the one block); `--replicas` instead gives every rank
its own block (weak scaling).  `--blocks N [--head]` times chained blocks
(two-block and 12-block + head configurations), `--primitive` the primitive
operations of one (N, L, dnum) configuration.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LOG_N, LIMBS, DNUM, TOKENS = 16, 24, 3, 103
ROT_INDICES = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512]
METRIC = "encrypted block latency (s) @103 tok, N=2^16"
UNIT = "s"
WORKLOAD = ("one encrypted DNAGPT block, 103 tokens (32/ciphertext), D=768, 12 heads, MLP 3072, "
            "N=2^16, 24-limb chain (60+23x50-bit) and keys, dnum=3, block evaluated at 2..11 limbs "
            "(input encrypted at 11), client refresh at LN/softmax/GELU")
# the reference's published T123 block wall clock on one A100
# (docs/hybrid/t123_walkthrough.md:51, 668)
REF_A100_BLOCK_S = 663.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# DRAM bytes (read + write) per limb of one NTT pass, from an ncu capture of a
# 1536-limb forward transform (64 polynomials x 24 limbs, float64 butterflies
# on 23 of the 24 primes): ntt_fwd_rows is the strided pass, ntt_fwd_cols the
# contiguous one; the pass traffic grows in proportion to the limbs it
# transforms
NCU_TRAFFIC_PER_LIMB = {"ntt_fwd_rows": (805.841920 + 762.777088) * 1e6 / 1536,
                        "ntt_fwd_cols": (918.904576 + 755.164160) * 1e6 / 1536}


def keyswitch_bytes(limbs: int, K: int, alpha: int, N: int) -> float:
    beta = -(-limbs // alpha)
    return (limbs + 2 * beta * (limbs + K) + 2 * limbs) * 8.0 * N


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU path: the block schedule on the CPU oracle (oracle/cpu_block.py)
# ---------------------------------------------------------------------------
def block_shape(logn: int):
    """(d_model, heads, mlp) of the block at ring 2^logn: the real shape at
    2^16, shrunk to the slots of a smaller ring (D = N / 64) otherwise."""
    from oracle import plain_block
    if logn == LOG_N:
        return plain_block.D, plain_block.HEADS, plain_block.MLP
    d = min(plain_block.D, (1 << logn) // 64)
    return d, d // 64, 4 * d


def run_cpu_block(tokens: int, logn: int, threads: int, steps: int, warmup: int):
    """Times the whole block schedule on the CPU oracle once, executed as
    `steps` consecutive slices of its stages (the last one finishes it);
    `warmup` untimed warm-up samples (one encryption and one rotation of an
    input group each) come first.  Returns (seconds per block, seconds of
    every slice, rel_inf of the decrypted output against the float64 block,
    operation counts, cores used, workers)."""
    from oracle import Oracle, plain_block
    from oracle.cpu_block import CpuBlock
    d_model, heads, mlp = block_shape(logn)
    o = Oracle(logN=logn, L=LIMBS, dnum=DNUM, seed=7, threads=threads)
    o.keygen()
    o.relin_keygen()
    w = plain_block.synthetic_weights(5, d=d_model, mlp=mlp)
    x = plain_block.synthetic_input(6, tokens, d=d_model)
    cb = CpuBlock(o, w, tokens, heads=heads, threads=threads)
    o.rot_keygen(cb.rotation_indices())
    rng = np.random.default_rng(1)
    for i in range(warmup):
        ct = o.encrypt(o.encode(rng.uniform(-1, 1, o.N // 2), CpuBlock.LX), 1 << 40 | i)
        o.rotate(ct, 32)
    K = max(1, steps)
    Y = cb.n_stages()
    bounds = [(i * Y) // K for i in range(K + 1)]
    gen = cb.schedule(x)
    times = []
    for i in range(K):
        t0 = time.perf_counter()
        for _ in range(bounds[i + 1] - bounds[i]):
            next(gen, None)
        if i == K - 1:
            for _ in gen:
                pass
        times.append(time.perf_counter() - t0)
    err = plain_block.rel_inf(plain_block.block(x, w, heads=heads), cb.y)
    assert err < 1e-6, f"CPU block output error {err}"
    return sum(times), times, err, dict(cb.ops), threads, cb.workers


def cpu_sample_text(tokens, logn, steps, times, threads, workers):
    return (f"the whole {tokens}-token block schedule at N=2^{logn} on the CPU oracle (oracle/cpu_block.py: "
            f"the engine's schedule, OpenMP over limbs inside each operation, {workers} host threads over "
            f"independent ciphertexts, {threads} cores), executed once as {steps} consecutive slices of its "
            f"stages; value = the sum of the slices ({', '.join(f'{t:.1f}' for t in times[:40])} s)")


SHARD_PARALLELISM = "shard{} (token groups, Q/K/V and MLP chunks, attention tiles)"


def arm_config(world: int, tokens: int, logn: int, sharded: bool = False):
    """the workload description both arms print (the same for both)"""
    workload = WORKLOAD
    if tokens != TOKENS:
        workload = workload.replace(f"{TOKENS} tokens", f"{tokens} tokens")
    if logn != LOG_N:
        d, h, m = block_shape(logn)
        workload = (workload.replace(f"N=2^{LOG_N}", f"N=2^{logn}")
                    .replace("D=768, 12 heads, MLP 3072", f"D={d}, {h} heads, MLP {m}"))
    return {"workload": workload, "flush": "inputs > L2 (keys ~13 GB, diagonals ~26 GB)",
            "parallelism": SHARD_PARALLELISM.format(world) if sharded else f"replicas{world}", "input_limbs": 11}


def arm_metric(tokens: int, logn: int):
    m = METRIC
    if tokens != TOKENS:
        m = m.replace(f"@{TOKENS} tok", f"@{tokens} tok")
    if logn != LOG_N:
        m = m.replace(f"N=2^{LOG_N}", f"N=2^{logn}")
    return m


def run_reference(args):
    """The reference arm: the reference's algorithm for this path on the
    host's cores.  Its own CPU path (OpenFHE under FIDESlib's API) is not in
    the reference tree, so the arm runs the CPU restatement of the same
    block schedule (the oracle), timed in full: one block, split over the
    --steps timed steps."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    sharded = world > 1 and not args.replicas
    threads = os.cpu_count() or 1
    total, times, err, ops, cores, workers = run_cpu_block(args.tokens, args.logn, threads, args.steps, args.warmup)
    sample = cpu_sample_text(args.tokens, args.logn, len(times), times, cores, workers)
    line = {
        "impl": "reference", "metric": arm_metric(args.tokens, args.logn), "value": total, "unit": UNIT,
        "n_gpus": world, "steps": len(times), "warmup": args.warmup, "ms_per_step": total / len(times) * 1e3,
        "higher_is_better": False, "scaling": "strong" if sharded else "weak", "vs_baseline": total / REF_A100_BLOCK_S,
        "dtype": "u64", "data": "synthetic", "config": arm_config(world, args.tokens, args.logn, sharded),
        "cpu_baseline": {"value": total, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": total, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "accuracy": {"rel_inf_vs_plaintext": err}, "slice_s": [round(t, 3) for t in times], "ops": ops,
    }
    print(json.dumps(line), flush=True)


def ntt_launch_sizes(prof: dict, logn: int) -> dict:
    """The NTT passes' launches and milliseconds by limbs per launch (the
    profiler's size buckets are log2 of algorithmic bytes, 2^(logn+3) per limb)."""
    out = {}
    for name, v in prof.items():
        if not name.startswith("ntt_"):
            continue
        for e, (n, ms) in v.get("by_size", {}).items():
            cur = out.setdefault(max(int(e) - (logn + 3), 0), [0, 0.0])
            cur[0] += n
            cur[1] = round(cur[1] + ms, 3)
    return {f"2^{k}": out[k] for k in sorted(out)}


# (log N, limbs, dnum) points of the primitive sweep recorded beside the
# block: the ring sizes at 24 limbs, the limb counts at N = 2^16, the digit
# counts at 24 limbs
SWEEP = [(15, 24, 3), (17, 24, 3), (16, 8, 3), (16, 16, 3), (16, 32, 3), (16, 24, 2), (16, 24, 4)]


def rotation_rates(eng, torch, cc, R: int = 32, steps: int = 3):
    """Seconds per EvalRotate over R ciphertexts (indices 1..512, keys
    generated by the caller): batched (one ckks_rotate_batch call, the form
    the block uses for independent switches) and one ckks_rotate call each;
    event-timed on the engine stream after one untimed step."""
    stream = torch.cuda.ExternalStream(cc.stream_handle())
    rng = np.random.default_rng(cc.N + cc.L)
    cts = [cc.Encrypt(cc.MakeCKKSPackedPlaintext(rng.uniform(-1, 1, cc.slots))) for _ in range(R)]
    outs = [eng.Ciphertext(cc) for _ in range(R)]
    ks = [ROT_INDICES[r % len(ROT_INDICES)] for r in range(R)]
    lib = eng.lib()

    def single():
        for r in range(R):
            eng._check(lib.ckks_rotate(cc.h, cts[r].h, ks[r], outs[r].h))

    def batched():
        cc.rotate_batch(cts, ks)

    res = []
    for fn in (batched, single):
        fn()
        fn()  # the allocator's blocks of these sizes exist from here on
        cc.Synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        e1.synchronize()
        res.append(e0.elapsed_time(e1) / 1e3 / (R * steps))
    return res


def keyswitch_record(cc, per_batch: float, per_single: float, limbs: int, logn: int, dnum: int) -> dict:
    ks_b = keyswitch_bytes(limbs, cc.K, cc.alpha, cc.N)
    peak, kind = measured_peaks()
    return {"logN": logn, "limbs": limbs, "dnum": dnum, "EvalRotate/s": round(1.0 / per_batch, 1),
            "us_per_rotation": round(per_batch * 1e6, 2), "GBps": round(ks_b / per_batch / 1e9, 1),
            "frac": round(ks_b / per_batch / 1e9 / peak, 4), "peak_kind": kind,
            "us_per_rotation_single_call": round(per_single * 1e6, 2), "algorithmic_bytes": ks_b}


def keyswitch_point(eng, torch, logn: int, limbs: int, dnum: int, device: int):
    """The key-switch record at one (N, limbs, dnum) on a fresh context."""
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=logn, limbs=limbs, dnum=dnum, seed=3, device=device))
    cc.KeyGen()
    cc.EvalRotateKeyGen(ROT_INDICES)
    pb, ps = rotation_rates(eng, torch, cc)
    return keyswitch_record(cc, pb, ps, limbs, logn, dnum)


def run_engine(args):
    import torch
    import private_genomic_dnagpt_b200 as eng
    from oracle import plain_block

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    # a smaller ring only for profiler captures: the block shrunk to fit its
    # slots (D = N / 64 up to 768, 64-feature heads, MLP 4 D)
    d_model, heads, mlp = block_shape(args.logn)
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=args.logn, limbs=LIMBS, dnum=DNUM, seed=1 + rank,
                                           device=local))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    w = plain_block.synthetic_weights(5, d=d_model, mlp=mlp)
    x = plain_block.synthetic_input(6, args.tokens, d=d_model)
    block = eng.EncryptedBlock(cc, w, args.tokens, heads=heads)
    cc.EvalRotateKeyGen(sorted(set(block.rotation_indices()) | set(ROT_INDICES)))
    stream = torch.cuda.ExternalStream(cc.stream_handle())

    def barrier():
        cc.Synchronize()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    # warm-up (also encodes the diagonals at their use levels) + accuracy
    # check.  The last warm-up step times every kernel launch (per-kernel and
    # per-stage totals, the launch count and the dominant kernel); the timed
    # steps time only the dominant kernel's launches, for the roofline, so
    # that the per-launch event records of the others stay out of the
    # headline number.
    ref = plain_block.block(x, w, heads=heads)
    for i in range(args.warmup):
        if i == args.warmup - 1:
            barrier()
            cc.profile_reset()
            cc.profile_only(None)
            cc.profile(True)
        y = block.forward(x)
    err = plain_block.rel_inf(ref, y)
    assert err < 1e-6, f"block output error {err}"
    barrier()
    prof_all = cc.profile_report()
    sections = cc.profile_sections()
    dominant = max(prof_all.items(), key=lambda kv: kv[1]["ms"])[0] if prof_all else None
    cc.profile_reset()
    cc.profile_only(dominant)
    eval_s, e2e_ms_steps, diag_steps = [], [], []
    with ClockSampler(local) as clk:
        # profiler range: an ncu run with --profile-from-start off captures
        # exactly the timed steps
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(args.steps):
            start = torch.cuda.Event(enable_timing=True)
            stop = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            y = block.forward(x)
            stop.record(stream)
            stop.synchronize()
            e2e_ms_steps.append(start.elapsed_time(stop))
            r_ = block.report()
            eval_s.append(r_["seconds"]["evaluate_events"])
            diag_steps.append({"alloc_host_s": round(r_["seconds"].get("alloc_host", 0), 4),
                               "alloc_calls": r_["counts"].get("alloc_calls"),
                               "pool_reserved_mib": r_["counts"].get("pool_reserved_mib"),
                               "stages": {k: round(v, 3) for k, v in r_["seconds"].items()
                                          if k in ("ln1_qkv", "scores", "context", "oproj_ln2_mlp")}})
            prof = cc.profile_report()  # folds this step's kernel events (the GPU is idle here)
        barrier()
        torch.cuda.cudart().cudaProfilerStop()
    e2e_ms = float(np.mean(e2e_ms_steps))
    cc.profile(False)
    cc.profile_only(None)
    rep = block.report()
    value = float(np.mean(eval_s))
    if dist is not None:
        t = torch.tensor([value, e2e_ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        value, e2e_ms = float(t[0]), float(t[1])

    # the same block with cold weights: the diagonals encoded inside the
    # timed call (the reference encodes them inside its block evaluation)
    cold_s, cold_e2e = [], []
    for _ in range(2):
        block.release_cache()
        barrier()
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        block.forward(x)
        c1.record(stream)
        c1.synchronize()
        cold_e2e.append(c0.elapsed_time(c1) / 1e3)
        cold_s.append(block.report()["seconds"]["evaluate_events"])

    # EvalRotate/s and key-switch GB/s on the primitive configuration
    # (24 limbs, dnum 3), on this context and its keys
    pb, ps = rotation_rates(eng, torch, cc)
    keyswitch = keyswitch_record(cc, pb, ps, LIMBS, args.logn, DNUM)
    keyswitch["EvalRotate/s"] = round(keyswitch["EvalRotate/s"] * world, 1)  # all ranks
    keyswitch["config"] = (f"EvalRotate N=2^{args.logn}, {LIMBS} limbs, dnum={DNUM}, 32 ciphertexts x indices "
                           f"1..512: one ckks_rotate_batch call (us_per_rotation_single_call: one ckks_rotate each)")

    roof = None
    peak, peak_kind = measured_peaks()
    if dominant is not None and dominant in prof:
        name, d = dominant, prof[dominant]
        per_launch_ms = d["ms"] / d["launches"]
        achieved = (d["bytes"] / d["launches"]) / (per_launch_ms / 1e3) / 1e9
        traffic = None
        if name in NCU_TRAFFIC_PER_LIMB:  # limbs per launch x measured bytes per limb
            limbs_per_launch = d["bytes"] / d["launches"] / (8.0 * (1 << args.logn))
            traffic = NCU_TRAFFIC_PER_LIMB[name] * limbs_per_launch
        roof = {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                "launches": d["launches"], "ms_per_launch": per_launch_ms,
                # share of device time in the fully profiled warm-up step
                "share": prof_all[name]["ms"] / sum(v["ms"] for v in prof_all.values())}
    released_bytes = 0  # diagonal cache handed back to the context's allocator
    if roof is not None:
        # the metric's key-switch part (ks bytes = (l + 2 beta (l + K) + 2 l) limbs)
        roof["keyswitch"] = keyswitch
        if rank == 0 and not args.no_sweep:
            released_bytes += block.release_cache()  # room for the sweep's contexts
            roof["keyswitch_sweep"] = [keyswitch_point(eng, torch, *pt, device=local) for pt in SWEEP]

    # the 12-block + head model on one sequence (one sequence per GPU):
    # a warm-up pass, then one timed pass
    model_rec = None
    if rank == 0 and not args.no_model:
        released = released_bytes + block.release_cache()
        ws = [plain_block.synthetic_weights(100 + b, d=d_model, mlp=mlp) for b in range(12)]
        hw = plain_block.synthetic_head_weights(99, d=d_model)
        free, _ = torch.cuda.mem_get_info(local)
        cached = max(1, int(((free + released) / 2**30 - 70) // 27))
        model = eng.EncryptedModel(cc, ws, hw, args.tokens, heads=heads, cached_blocks=min(cached, 12))
        cc.EvalRotateKeyGen(sorted(set(model.rotation_indices()) - set(block.rotation_indices())))
        h_ref, m_ref = plain_block.model(x, ws, hw, heads=heads)
        model.forward(x)
        barrier()
        m0 = torch.cuda.Event(enable_timing=True)
        m1 = torch.cuda.Event(enable_timing=True)
        m0.record(stream)
        h, m = model.forward(x)
        m1.record(stream)
        m1.synchronize()
        dev = sum(b.report()["seconds"].get("evaluate_events", 0.0) for b in model.blocks)
        dev += model.head.report()["seconds"].get("head_total", 0.0)
        model_rec = {"workload": f"12 blocks + head (768 -> 2 readout margin), one sequence of {args.tokens} "
                                 "tokens, full-hidden-state client refresh between blocks",
                     "value": dev, "e2e": m0.elapsed_time(m1) / 1e3, "unit": UNIT, "steps": 1, "warmup": 1,
                     "cached_blocks": model.cached_blocks,
                     "rel_inf_vs_plaintext": plain_block.rel_inf(h_ref, h), "margin": m, "margin_plaintext": m_ref}
        del model

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        # the same block on the CPU oracle, timed in full (one run)
        total, times, cerr, _, cores, workers = run_cpu_block(args.tokens, args.logn, os.cpu_count() or 1, 1, 0)
        cpu = {"value": total, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": cpu_sample_text(args.tokens, args.logn, 1, times, cores, workers),
               "rel_inf_vs_plaintext": cerr}

    launches = sum(v["launches"] for v in prof_all.values())  # one block (the profiled warm-up step)
    if rank == 0:
        # host<->device traffic of one block: packed inputs and outputs plus
        # every client refresh (N/2 doubles per ciphertext each way)
        c = rep["counts"]
        groups = -(-args.tokens // 32)
        ct_bytes = cc.slots * 8
        h2d = (groups + 2 * groups + c.get("weight_tile_encryptions", 0) + 3 * groups) * ct_bytes
        d2h = (groups + 2 * groups + c.get("score_tile_decryptions", 0) + 3 * groups) * ct_bytes
        line = {
            "metric": arm_metric(args.tokens, args.logn), "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": e2e_ms, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": value / REF_A100_BLOCK_S, "dtype": "u64", "data": "synthetic",
            "config": arm_config(world, args.tokens, args.logn),
            "accuracy": {"rel_inf_vs_plaintext": err, "input_limbs": rep["counts"].get("input_limbs")},
            "e2e": {"value": e2e_ms / 1e3, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    # the same call with the weights' diagonals encoded inside it
                    "cold_weights": {"value": float(np.mean(cold_e2e)), "device_s": float(np.mean(cold_s)),
                                     "steps": len(cold_e2e)}},
            "roofline": roof,
            "block": {"counts": rep["counts"], "seconds": rep["seconds"],
                      "evaluate_s_per_step": [round(v, 4) for v in eval_s],
                      "e2e_s_per_step": [round(v / 1e3, 4) for v in e2e_ms_steps],
                      "host_per_step": diag_steps},
            # one block, every launch timed (the last warm-up step)
            "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 3),
                            "GBps": round(v["bytes"] / v["ms"] / 1e6, 1) if v["ms"] > 0 else None}
                        for k, v in prof_all.items()},
            # NTT passes by launch size: "2^k" = launches of 2^k to 2^(k+1) limbs: [launches, ms]
            "ntt_launch_sizes": ntt_launch_sizes(prof_all, args.logn),
            # per block stage: device ms of its kernels, the largest first
            "stage_kernels_ms": {
                sec: dict(sorted(((k, round(v["ms"], 2)) for k, v in ks.items()), key=lambda kv: -kv[1])[:8]) | {
                    "_total": round(sum(v["ms"] for v in ks.values()), 2)}
                for sec, ks in sections.items()},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "model_12_blocks_head": model_rec,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_shard(args):
    """One block sharded over the torchrun ranks (strong scaling): token
    groups (with more ranks than groups, their Q/K/V projections and MLP
    chunks) and attention alignments split across ranks, Q/K/V broadcasts, a
    score all-reduce, partial-context and MLP merges and an output all-reduce
    over NCCL between the stages (private_genomic_dnagpt_b200/shard.py).  Every
    rank holds the same keys (same seed).  value = device time of one block
    from the first stage to the assembled output, max over ranks."""
    import datetime

    import torch
    import torch.distributed as dist
    import private_genomic_dnagpt_b200 as eng
    from private_genomic_dnagpt_b200 import shard
    from oracle import plain_block

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=600),
                            device_id=torch.device("cuda", local))
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=LOG_N, limbs=LIMBS, dnum=DNUM, seed=1, device=local))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    w = plain_block.synthetic_weights(5)
    x = plain_block.synthetic_input(6, args.tokens)
    block = eng.EncryptedBlock(cc, w, args.tokens)
    cc.EvalRotateKeyGen(block.rotation_indices())
    io = shard.EngineIO(block)
    sb = shard.ShardedBlock(io, args.tokens, 32, 12, plain_block.D, dist, "cuda")
    stream = torch.cuda.ExternalStream(cc.stream_handle())
    ref = plain_block.block(x, w)
    for _ in range(args.warmup):
        y = sb.forward(x)
    err = plain_block.rel_inf(ref, y)
    assert err < 1e-6, f"sharded block output error {err}"
    cc.Synchronize()
    dist.barrier()
    steps, evals = [], []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            y = sb.forward(x)
            e1.record(stream)
            e1.synchronize()
            steps.append(e0.elapsed_time(e1) / 1e3)
            # this rank's span from encrypted inputs resident to encrypted
            # outputs resident (exchanges included); a helper rank owns no
            # token group and finishes none: the owners' spans, which wait
            # for the helpers' partial sums, carry the block's latency
            evals.append(block.report()["seconds"].get("evaluate_events", 0.0))
        cc.Synchronize()
        dist.barrier()
    t = torch.tensor([float(np.mean(evals)), float(np.mean(steps))], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    value, e2e = float(t[0]), float(t[1])
    if rank == 0:
        groups = -(-args.tokens // 32)
        line = {
            "metric": arm_metric(args.tokens, LOG_N), "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": e2e * 1e3, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": value / REF_A100_BLOCK_S, "dtype": "u64", "data": "synthetic",
            "config": arm_config(world, args.tokens, LOG_N, True),
            "accuracy": {"rel_inf_vs_plaintext": err},
            "shard": {"plan": [{"groups": rp.groups, "qkv": rp.qkv, "mlp": rp.mlp, "tiles": rp.tiles}
                               for rp in sb.plan],
                      "rank0_stage_s": {k: round(v, 4) for k, v in block.report().get("seconds", {}).items()}},
            # the whole sharded call: host embeddings in, host outputs out
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": groups * cc.slots * 8,
                    "d2h_bytes_per_step": groups * cc.slots * 8},
            "per_step_s": [round(v, 4) for v in steps],
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_model(args):
    """Chained blocks (the two-block and 12-block configurations) with the
    full-hidden-state client refresh between blocks and, with --head, the
    last-token refresh into the classifier head (N - A margin).  One step is
    one sequence through the whole model; under torchrun every rank runs its
    own sequence (replicas, weak scaling), or with --shard the ranks share one
    sequence, every block sharded over them (strong scaling, shard.py
    ShardedModel).  Blocks beyond the diagonal-cache budget of the device
    encode their diagonals again on every step."""
    import torch
    import private_genomic_dnagpt_b200 as eng
    from oracle import plain_block

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900))
    sharded = dist is not None and args.shard
    # sharded: identical keys (same seed) and one sequence on every rank
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=LOG_N, limbs=LIMBS, dnum=DNUM,
                                           seed=1 if sharded else 1 + rank, device=local))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    ws = [plain_block.synthetic_weights(100 + b) for b in range(args.blocks)]
    hw = plain_block.synthetic_head_weights(99) if args.head else None
    x = plain_block.synthetic_input(6 if sharded else 6 + rank, args.tokens)
    # diagonal caches: about 26 GB per block; keep what fits beside the keys
    free, _ = torch.cuda.mem_get_info(local)
    # headroom: one block re-encoding its diagonals (26 GB), keys (~8 GB) and
    # the evaluation's working set
    cached = args.cached_blocks if args.cached_blocks >= 0 else max(1, int((free / 2**30 - 70) // 27))
    model = eng.EncryptedModel(cc, ws, hw, args.tokens, cached_blocks=min(cached, args.blocks))
    cc.EvalRotateKeyGen(model.rotation_indices())
    stream = torch.cuda.ExternalStream(cc.stream_handle())
    h_ref, m_ref = plain_block.model(x, ws, hw)
    forward = model.forward
    if sharded:
        from private_genomic_dnagpt_b200 import shard
        sm = shard.ShardedModel([shard.EngineIO(b) for b in model.blocks], model.head, args.tokens, 32,
                                plain_block.HEADS, plain_block.D, dist, "cuda", cached_blocks=model.cached_blocks)
        forward = sm.forward

    def barrier():
        cc.Synchronize()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        h, m = forward(x)
    err = plain_block.rel_inf(h_ref, h)
    assert err < 1e-6, f"model hidden-state error {err}"
    barrier()
    steps_s, eval_s = [], []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            h, m = forward(x)
            e1.record(stream)
            e1.synchronize()
            steps_s.append(e0.elapsed_time(e1) / 1e3)
            if sharded:  # device time of the whole sharded sequence, exchanges included
                eval_s.append(steps_s[-1])
                continue
            ev = sum(b.report()["seconds"].get("evaluate_events", 0.0) for b in model.blocks)
            if model.head is not None:
                ev += model.head.report()["seconds"].get("head_total", 0.0)
            eval_s.append(ev)
        barrier()
    value, e2e = float(np.mean(eval_s)), float(np.mean(steps_s))
    if dist is not None:
        t = torch.tensor([value, e2e], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        value, e2e = float(t[0]), float(t[1])
    if rank == 0:
        name = f"{args.blocks} blocks" + (" + head" if args.head else "")
        groups = -(-args.tokens // 32)
        ct_bytes = cc.slots * 8
        line = {
            "metric": f"encrypted {name} latency (s) @{args.tokens} tok, N=2^16", "value": value, "unit": "s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": e2e * 1e3,
            "higher_is_better": False, "scaling": "strong" if sharded else "weak", "vs_baseline": None,
            "dtype": "u64", "data": "synthetic",
            "config": {"workload": f"{name}, " + ("one sequence sharded over the GPUs" if sharded else
                                                  "one sequence per GPU") +
                                   f", {args.tokens} tokens, D=768, 12 heads, MLP 3072, N=2^16, 24 limbs, dnum=3; "
                                   f"full-hidden-state client refresh between blocks",
                       "cached_blocks": model.cached_blocks,
                       "parallelism": f"shard{world}" if sharded else f"replicas{world}",
                       "flush": "inputs > L2 (keys, diagonals)",
                       "rel_inf_vs_plaintext": err,
                       "margin": m, "margin_plaintext": m_ref},
            "e2e": {"value": e2e, "unit": "s", "h2d_bytes_per_step": args.blocks * groups * ct_bytes,
                    "d2h_bytes_per_step": args.blocks * groups * ct_bytes},
            "per_step_s": [round(v, 4) for v in steps_s],
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_primitive(args):
    """Primitive operations on one configuration of the sweep (N, L, dnum):
    NTT, EvalRotate (single and batched), hoisted rotations, EvalMult+relin,
    Rescale, each timed with CUDA events on the engine stream over 32
    ciphertexts (> L2 at L >= 8).  The timed region is inside a profiler
    range, so `ncu --profile-from-start off` on this command captures the
    primitive kernels on a case of a few GB."""
    import torch
    import private_genomic_dnagpt_b200 as eng

    torch.cuda.set_device(0)
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=args.logn, limbs=args.limbs, dnum=args.dnum, seed=1))
    cc.KeyGen()
    cc.EvalMultKeyGen()
    cc.EvalRotateKeyGen(ROT_INDICES)
    stream = torch.cuda.ExternalStream(cc.stream_handle())
    lib = eng.lib()
    R, L, N = 32, args.limbs, cc.N
    rng = np.random.default_rng(3)
    cts = [cc.Encrypt(cc.MakeCKKSPackedPlaintext(rng.uniform(-1, 1, cc.slots))) for _ in range(R)]
    cts2 = [cc.Encrypt(cc.MakeCKKSPackedPlaintext(rng.uniform(-1, 1, cc.slots))) for _ in range(R)]
    outs = [eng.Ciphertext(cc) for _ in range(R)]
    # NTT input: R ciphertexts' worth of limbs (2 R L limbs), residues below 2^49
    ntt_buf = torch.randint(0, 1 << 49, (2 * R * L * N,), dtype=torch.int64, device="cuda")

    ops = {
        "ntt_fwd": lambda: eng._check(lib.ckks_ntt_forward_polys(cc.h, ntt_buf.data_ptr(), 2 * R, L)),
        "ntt_inv": lambda: eng._check(lib.ckks_ntt_inverse_polys(cc.h, ntt_buf.data_ptr(), 2 * R, L)),
        "rotate": lambda: [eng._check(lib.ckks_rotate(cc.h, cts[r].h, ROT_INDICES[r % len(ROT_INDICES)], outs[r].h))
                           for r in range(R)],
        "rotate_batch": lambda: cc.rotate_batch(cts, [ROT_INDICES[r % len(ROT_INDICES)] for r in range(R)]),
        "rotate_hoisted": lambda: [cc.EvalFastRotation(cts[r], ROT_INDICES[:4]) for r in range(R // 4)],
        "mul_relin_batch": lambda: cc.mul_ct_batch(cts, cts2),
        "rescale_batch": lambda: cc.rescale_batch(cts),
    }
    units = {"ntt_fwd": 2 * R * L, "ntt_inv": 2 * R * L, "rotate": R, "rotate_batch": R,
             "rotate_hoisted": (R // 4) * 4, "mul_relin_batch": R, "rescale_batch": R}
    res = {}
    torch.cuda.cudart().cudaProfilerStart()
    with ClockSampler(0) as clk:
        for name, fn in ops.items():
            for _ in range(args.warmup):
                fn()
            cc.Synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                fn()
            e1.record(stream)
            e1.synchronize()
            sec = e0.elapsed_time(e1) / 1e3 / args.steps
            res[name] = {"us_per_unit": sec / units[name] * 1e6, "units_per_step": units[name]}
    torch.cuda.cudart().cudaProfilerStop()
    peak, peak_kind = measured_peaks()
    ks_b = keyswitch_bytes(L, cc.K, cc.alpha, N)
    ntt_gbs = 2 * 8.0 * N / (res["ntt_fwd"]["us_per_unit"] * 1e-6) / 1e9
    rot_s = res["rotate_batch"]["us_per_unit"] * 1e-6
    line = {
        "metric": "EvalRotate/s", "value": 1.0 / rot_s, "unit": "rotations/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": rot_s * R * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u64", "data": "synthetic",
        "config": {"workload": f"primitive ops, N=2^{args.logn}, {L} limbs, dnum={args.dnum}, {R} ciphertexts",
                   "flush": "inputs > L2", "alpha": cc.alpha, "special": cc.K},
        "ops": res,
        "roofline": {"kernel": "ntt_fwd", "bound": "hbm", "achieved": ntt_gbs, "peak": peak, "unit": "GB/s",
                     "frac": ntt_gbs / peak, "peak_kind": peak_kind,
                     "keyswitch_GBps": ks_b / rot_s / 1e9, "keyswitch_frac": ks_b / rot_s / 1e9 / peak},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_bsgs(args):
    """One BSGS matrix product (T123.cpp:1264-1295) of a seeded 768 x 768
    weight over 4 token groups, n1 = n2 = 32, at the context's limbs: the
    diagonals are encoded once, the baby steps computed once, and each step
    is one ckks_bsgs_matmul (inner sums, grouped giant-step rotations,
    rescale).  The inner-sum kernel is timed from the engine's launch events.
    The baby steps, warm-up and timed products are inside a profiler range,
    so `ncu --profile-from-start off` on this command captures their kernels
    (about 2.5 GB on the device at 4 limbs, N = 2^16)."""
    import torch
    import private_genomic_dnagpt_b200 as eng

    torch.cuda.set_device(0)
    B, n1, n2, groups, D = 32, 32, 32, 4, 768
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=args.logn, limbs=args.limbs, dnum=args.dnum, seed=1))
    cc.KeyGen()
    cc.EvalRotateKeyGen([B * j for j in range(1, n1)] + [B * n1 * g for g in range(1, n2)])
    L, N = args.limbs, cc.N
    rng = np.random.default_rng(7)
    W = rng.normal(0.0, 0.02, (D, D))
    diags = cc.bsgs_diagonals(W, B, n1, L)
    x = [cc.Encrypt(cc.MakeCKKSPackedPlaintext(rng.uniform(-1, 1, cc.slots))) for _ in range(groups)]
    stream = torch.cuda.ExternalStream(cc.stream_handle())
    # the profiler range also holds the baby steps (hoisted rotations: the
    # key products of keyswitch_hoisted_multi) and the warm-up products
    torch.cuda.cudart().cudaProfilerStart()
    babies = [cc.bsgs_babies(x, B, n1)]
    for _ in range(args.warmup):
        cc.bsgs_matmul([diags], babies)
    cc.Synchronize()
    cc.profile_reset()
    cc.profile_only("bsgs_inner")
    cc.profile(True)
    with ClockSampler(0) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            cc.bsgs_matmul([diags], babies)
        e1.record(stream)
        e1.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    cc.Synchronize()
    prof = cc.profile_report()
    cc.profile(False)
    cc.profile_only(None)
    sec = e0.elapsed_time(e1) / 1e3 / args.steps
    inner = prof.get("bsgs_inner", {})
    inner_s = inner.get("ms", 0.0) / 1e3 / max(1, inner.get("launches", 1))
    peak, peak_kind = measured_peaks()
    lb = 8.0 * N
    # diagonals, baby residues, inner sums written (algorithmic bytes)
    inner_bytes = (n1 * n2 * L + groups * (2.0 * n1 * L + 2.0 * n2 * L)) * lb
    line = {
        "metric": "BSGS product latency (s)", "value": sec, "unit": "s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "u64/f64", "data": "synthetic",
        "config": {"workload": f"BSGS product, 768x768 weight, n1=n2=32, {groups} token groups, "
                               f"N=2^{args.logn}, {L} limbs, dnum={args.dnum}",
                   "flush": "diagonals > L2"},
        "inner": {"us_per_launch": inner_s * 1e6, "launches": inner.get("launches", 0),
                  "achieved_GBps": inner_bytes / inner_s / 1e9 if inner_s else None,
                  "frac": inner_bytes / inner_s / 1e9 / peak if inner_s else None, "peak": peak,
                  "peak_kind": peak_kind, "bytes": inner_bytes},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-model", action="store_true")
    # a smaller token count only for profiler captures (the benchmark is 103)
    ap.add_argument("--tokens", type=int, default=TOKENS)
    # primitive-operation sweep instead of the block (one configuration per run)
    ap.add_argument("--primitive", action="store_true")
    # one BSGS matrix product at --logn / --limbs instead of the block
    ap.add_argument("--bsgs", action="store_true")
    ap.add_argument("--logn", type=int, default=LOG_N)
    ap.add_argument("--limbs", type=int, default=LIMBS)
    ap.add_argument("--dnum", type=int, default=DNUM)
    # chained blocks (two-block / 12-block + head configurations)
    ap.add_argument("--blocks", type=int, default=1)
    ap.add_argument("--head", action="store_true")
    ap.add_argument("--cached-blocks", type=int, default=-1)
    # under torchrun (WORLD_SIZE > 1) one block is sharded over the ranks
    # (strong scaling); --replicas runs one independent block per rank instead
    ap.add_argument("--shard", action="store_true")
    ap.add_argument("--replicas", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.primitive:
        run_primitive(args)
    elif args.bsgs:
        run_bsgs(args)
    elif args.blocks > 1 or args.head:
        run_model(args)
    elif args.shard or (int(os.environ.get("WORLD_SIZE", "1")) > 1 and not args.replicas):
        run_shard(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
