"""Benchmark of the CKKS key-switching hot path on B200.

Workload (the primitive configuration of the benchmark set): EvalRotate on
ciphertexts at N = 2^16 with 24 Q limbs (60-bit first prime + 23 x 50-bit),
dnum = 3 (8 special primes), rotation indices 1, 2, 4, ..., 512.  One step
rotates R independent ciphertexts (R x 24 MiB of input, 10 x 96 MiB of
rotation keys, so every step streams more than the 126 MB L2 from HBM).

Reported (one JSON line on rank 0):
  value   rotations/s, inputs resident in HBM, device time (CUDA events on the
          engine's stream), summed over ranks / max time over ranks;
  e2e     the same through the C ABI with host buffers: per ciphertext a
          pinned host -> device import, the rotation, a device -> host export;
  roofline  the dominant kernel's algorithmic bytes / its event-timed
          duration against the measured HBM copy bandwidth, plus the
          composite key-switch bandwidth (ell + 2 beta (ell+K) + 2 ell limbs
          per rotation);
  cpu_baseline  the CPU oracle (restatement of the reference path) on a
          bounded sample on this host's cores.
`--impl reference` times that CPU path alone with every host thread.
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

LOG_N, LIMBS, DNUM = 16, 24, 3
ROT_INDICES = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512]
METRIC = "EvalRotate/s"
UNIT = "rotations/s"
WORKLOAD = "EvalRotate N=2^16, 24 limbs (60+23x50-bit), dnum=3, K=8, indices 1..512 pow2"


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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


class CpuPath:
    """CPU oracle EvalRotate at the benchmark parameters (keys made once)."""

    def __init__(self, threads: int):
        from oracle import Oracle
        self.o = Oracle(logN=LOG_N, L=LIMBS, dnum=DNUM, seed=7, threads=threads)
        self.o.keygen()
        self.ks = ROT_INDICES[:3]
        self.o.rot_keygen(self.ks)
        x = np.random.default_rng(1).uniform(-1, 1, self.o.N // 2)
        self.ct = self.o.encrypt(self.o.encode(x, LIMBS), 0)
        self.i = 0

    def rotations(self, n: int) -> float:
        t0 = time.perf_counter()
        for _ in range(n):
            self.o.rotate(self.ct, self.ks[self.i % len(self.ks)])
            self.i += 1
        return time.perf_counter() - t0


def cpu_rotations_per_s(budget_s: float, threads: int):
    """Bounded sample (about budget_s of CPU work): rotations/s and its description."""
    cp = CpuPath(threads)
    one = cp.rotations(1)
    n = max(2, min(200, int(budget_s / max(one, 1e-3))))
    dt = cp.rotations(n)
    return n / dt, f"{n} rotations of one 24-limb ciphertext (indices {cp.ks}), {dt:.2f} s"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cp = CpuPath(threads)
    one = cp.rotations(max(1, min(args.warmup, 3)))  # untimed warm-up
    per_step = max(1, int(6.0 / max(one, 1e-3)))     # ~6 s of CPU work per step
    total_t, total_n = 0.0, 0
    for _ in range(max(1, args.steps)):
        total_t += cp.rotations(per_step)
        total_n += per_step
    value = total_n / total_t
    sample = f"{args.steps} steps x {per_step} rotations of one 24-limb ciphertext, {total_t:.2f} s"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_t / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u64", "data": "synthetic",
        "config": {"workload": WORKLOAD, "flush": "inputs > L2"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_engine(args):
    import torch
    import private_genomic_dnagpt_b200 as eng

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))

    R = args.rotations
    cc = eng.GenCryptoContext(eng.CCParams(ring_dim_log=LOG_N, limbs=LIMBS, dnum=DNUM, seed=1 + rank,
                                           device=local))
    cc.KeyGen()
    cc.EvalRotateKeyGen(ROT_INDICES)
    rng = np.random.default_rng(rank)
    cts = []
    for r in range(R):
        cts.append(cc.Encrypt(cc.MakeCKKSPackedPlaintext(rng.uniform(-1, 1, cc.slots))))
    outs = [eng.Ciphertext(cc) for _ in range(R)]
    lib = eng.lib()
    stream = torch.cuda.ExternalStream(cc.stream_handle())

    def step():
        for r in range(R):
            eng._check(lib.ckks_rotate(cc.h, cts[r].h, ROT_INDICES[r % len(ROT_INDICES)], outs[r].h))

    # correctness spot check of the benchmarked path
    got = cc.Decrypt(cc.EvalRotate(cts[0], 1)).GetRealPackedValue()
    ref = np.roll(cc.Decrypt(cts[0]).GetRealPackedValue(), -1)
    assert np.abs(got - ref).max() < 1e-6

    def barrier():
        cc.Synchronize()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    barrier()
    cc.profile(True)
    cc.profile_reset()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        barrier()
    ms = start.elapsed_time(stop)
    prof = cc.profile_report()
    cc.profile(False)
    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    total_rot = R * args.steps * world
    value = total_rot / (ms_max / 1e3)

    # e2e: host buffers through the C ABI
    words = 2 * LIMBS * cc.N
    h_in = [torch.empty(words, dtype=torch.int64, pin_memory=True).numpy().view(np.uint64) for _ in range(R)]
    h_out = [torch.empty(words, dtype=torch.int64, pin_memory=True).numpy().view(np.uint64) for _ in range(R)]
    for r in range(R):
        h_in[r][:] = cts[r].limbs_array().reshape(-1)
    scale = cts[0].scale
    tmp_in = [eng.Ciphertext(cc) for _ in range(R)]
    u64p = eng._u64p

    def e2e_step():
        for r in range(R):
            eng._check(lib.ckks_ct_import(cc.h, tmp_in[r].h, h_in[r].ctypes.data_as(u64p), LIMBS, scale, 1))
            eng._check(lib.ckks_rotate(cc.h, tmp_in[r].h, ROT_INDICES[r % len(ROT_INDICES)], outs[r].h))
            eng._check(lib.ckks_ct_export(cc.h, outs[r].h, h_out[r].ctypes.data_as(u64p), words))

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e_ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_value = total_rot / (e_ms / 1e3)

    peak, peak_kind = measured_peaks()
    dom = max(prof.items(), key=lambda kv: kv[1]["ms"]) if prof else (None, None)
    roof = None
    if dom[0] is not None:
        name, d = dom
        per_launch_ms = d["ms"] / d["launches"]
        achieved = (d["bytes"] / d["launches"]) / (per_launch_ms / 1e3) / 1e9
        roof = {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                "launches": d["launches"], "ms_per_launch": per_launch_ms,
                "share": d["ms"] / sum(v["ms"] for v in prof.values())}
    ks_b = keyswitch_bytes(LIMBS, cc.K, cc.alpha, cc.N)
    per_rot_s = (ms_max / 1e3) / (R * args.steps)
    keyswitch = {"bytes_per_rotation": ks_b, "achieved_gbs": ks_b / per_rot_s / 1e9,
                 "frac_of_hbm": ks_b / per_rot_s / 1e9 / peak, "us_per_rotation": per_rot_s * 1e6}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        v, sample = cpu_rotations_per_s(args.cpu_budget, threads)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}

    launches = sum(v["launches"] for v in prof.values())
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "rotations_per_step": R, "flush": "inputs > L2 (keys 960 MiB)",
                       "parallelism": f"replicas{world}"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": R * words * 8,
                    "d2h_bytes_per_step": R * words * 8},
            "roofline": roof,
            "keyswitch": keyswitch,
            "kernels": {k: {"launches": v["launches"], "ms": round(v["ms"], 4)} for k, v in prof.items()},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--rotations", type=int, default=32)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
