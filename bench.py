"""Benchmark driver (one JSON line on rank 0).

Workload at N=1: BASELINE config 2 — batched forward + inverse negacyclic NTT,
N = 2^16, 36 RNS limbs of 59-bit NTT-friendly primes, 2 ciphertexts x 2 polys
(4 polys).  One step = forward NTT of the whole batch followed by the inverse
NTT of the whole batch.  Inputs are seeded uniform residues in [0, q_i).

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier
and torch.cuda.synchronize() on both sides; the device time is the max over
ranks.  Four rotating input batches (4 x 75.5 MB > 126 MB L2) keep each step's
input out of L2.  CUDA events on the context's stream time the forward
transform (the dominant kernel pair) for the roofline.

Multi-GPU (torchrun): each rank transforms its own independent batch (weak
scaling, no data-path collective); value = steps of all ranks / max time.

``--impl reference``: the reference's CKKS arithmetic lives in FIDESlib and
OpenFHE, which are not in the reference checkout and cannot be built here, so
the reference arm times the CPU oracle's restatement of OpenFHE's NTT on the
host cores (all threads), rank 0 only.
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

METRIC = "enc s/generated token (Mamba-2-130M shape); NTT+keyswitch % HBM roofline"
LOG_N, LIMBS, POLYS, BITS = 16, 36, 4, 59
UNIT = "batched fwd+inv NTT steps/s (4 polys x 36 limbs x 2^16)"
ALG_BYTES_PER_TRANSFORM = 16 * POLYS * LIMBS * (1 << LOG_N)  # read + write every word once
N_ROTATE = 4


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes of the forward transform from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "ntt_fwd_config2.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("traffic_bytes_per_forward_transform:"):
            try:
                return int(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def bench_primes():
    # The 36 largest primes below 2^59 that are 1 mod 2N (host-side, product code).
    from fhe_mamba_b200.params import ntt_primes
    return ntt_primes(LOG_N, BITS, LIMBS)


def make_batch(qs, seed):
    rng = np.random.default_rng(seed)
    n = 1 << LOG_N
    out = np.empty((POLYS, LIMBS, n), dtype=np.uint64)
    for l, q in enumerate(qs):
        out[:, l, :] = rng.integers(0, q, size=(POLYS, n), dtype=np.uint64)
    return out


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            if self.uuid and self.uuid not in f[1]:
                continue
            try:
                sm.append(float(f[2]))
                mx = float(f[3])
            except ValueError:
                continue
            for name, v in zip(names, f[6:10]):
                if v.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline(threads, sample_limbs=None):
    """Oracle NTT (restatement of OpenFHE's CPU NTT) on the host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    qs = O.ntt_primes(LOG_N, BITS, LIMBS)
    psis = [O.root_of_unity(2 << LOG_N, q) for q in qs]
    limbs = sample_limbs or LIMBS
    x = make_batch(qs, 1)[:, :limbs, :].copy()
    O.ntt_batch(x[:1, :1].copy(), qs[:1], psis[:1], False, 1)  # warm
    t0 = time.perf_counter()
    O.ntt_batch(x, qs[:limbs], psis[:limbs], False, threads)
    O.ntt_batch(x, qs[:limbs], psis[:limbs], True, threads)
    dt = time.perf_counter() - t0
    scale = LIMBS / limbs
    return 1.0 / (dt * scale), dt, f"fwd+inv of {POLYS} polys x {limbs} limbs x 2^16 (scaled x{scale:g})"


def measure_ckks(local, reps=10):
    """Key switching and the BSGS matvec at BASELINE config-3 shape
    (N=2^16, 2^15 slots, 20 limbs, dnum 3), timed with CUDA events on the
    context stream.  Returns the two report objects."""
    import torch
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.ckks import bsgs_diagonals
    cc = CryptoContext(CCParams(ring_dim=1 << 16, multiplicative_depth=19, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3, device=local))
    cc.KeyGen(7)
    stream = torch.cuda.ExternalStream(cc.stream_ptr(), device=torch.device("cuda", local))
    n, L, K = cc.n, cc.n_q, cc.n_p
    D = (L + cc.alpha - 1) // cc.alpha
    rng = np.random.default_rng(3)
    d3 = np.empty((3, L, n), dtype=np.uint64)
    for l, q in enumerate(cc.q):
        d3[:, l, :] = rng.integers(0, q, size=(3, n), dtype=np.uint64)
    ct3 = cc.upload(d3, noise_deg=2)
    for _ in range(3):
        cc.Relinearize(ct3)
    cc.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    outs = [cc.Relinearize(ct3) for _ in range(reps)]
    e1.record(stream)
    e1.synchronize()
    ks_ms = e0.elapsed_time(e1) / reps
    del outs
    ks_bytes = (L + 2 * L + 2 * L) * n * 8 + D * 2 * (L + K) * n * 8
    peak, kind = peaks()
    ks = {"workload": "relinearisation (HYBRID key switch), N=2^16, 20 Q limbs, 7 P limbs, dnum 3",
          "ms": ks_ms, "alg_bytes": ks_bytes, "achieved_gbs": ks_bytes / (ks_ms / 1e3) / 1e9,
          "frac": ks_bytes / (ks_ms / 1e3) / 1e9 / peak, "peak_gbs": peak, "peak_source": kind}

    m, k, baby, giant = 768, 1536, 32, 48
    W = rng.normal(0, 0.02, size=(m, k))
    x = rng.uniform(-1, 1, k)
    cc.EvalRotateKeyGen(list(range(1, baby)) + [g * baby for g in range(1, giant)])
    v = np.zeros(cc.slots)
    v[:k] = x
    v[k:2 * k] = x
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(v))
    pts = cc.MakeCKKSPackedPlaintexts(np.array([d for d in bsgs_diagonals(W, baby, giant, cc.slots)]))
    out = cc.EvalLinearTransform(ct, pts, baby, giant)
    cc.synchronize()
    e0.record(stream)
    for _ in range(3):
        out = cc.EvalLinearTransform(ct, pts, baby, giant)
    e1.record(stream)
    e1.synchronize()
    mv_ms = e0.elapsed_time(e1) / 3
    cc.RescaleInPlace(out)
    y = cc.Decrypt(out).GetRealPackedValue()
    err = float(np.max(np.abs(y[:m] - W @ x)))
    diag_bytes = k * L * n * 8
    mv = {"workload": "BASELINE configs[2]: 768x1536 BSGS matvec, N=2^16, 2^15 slots, 20 limbs, dnum 3, "
                      "baby 32 / giant 48, diagonals pre-encoded in HBM",
          "ms": mv_ms, "max_abs_err_vs_fp64": err, "rotations": (baby - 1) + (giant - 1),
          "diagonal_bytes": diag_bytes, "diagonal_stream_gbs": diag_bytes / (mv_ms / 1e3) / 1e9}
    del pts, ct, out, ct3
    cc.close()
    return ks, mv


def measure_bootstrap(local, reps=3):
    """One full-packing bootstrap at the reference's native parameters
    (N=2^16, 2^15 slots, multiplicative depth 44, 59-bit scaling / 60-bit
    first prime, dnum 3, level budget {4, 4}; packed_fideslib.cpp:1061-1089),
    timed with CUDA events on the context stream; the input has 2 limbs left."""
    import torch
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 16, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3, device=local))
    cc.KeyGen(11)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    stream = torch.cuda.ExternalStream(cc.stream_ptr(), device=torch.device("cuda", local))
    x = np.random.default_rng(5).uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 2)
    out = cc.EvalBootstrap(ct)  # first call encodes the SlotToCoeff diagonals
    cc.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        out = cc.EvalBootstrap(ct)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    err = float(np.max(np.abs(cc.Decrypt(out).GetRealPackedValue() - x)))
    info = cc.bootstrap_info()
    rep = {"workload": "full-packing bootstrap, N=2^16, 2^15 slots, depth 44 (45 Q limbs), 59/60-bit, dnum 3, "
                       "level budget {4,4}, uniform ternary secret",
           "ms": ms, "limbs_in": 2, "limbs_out": out.n_limbs(), "levels": cc.bootstrap_levels(),
           "max_abs_err": err, "correction": info["correction"], "chebyshev_degree": info["chebyshev_degree"],
           "rotation_keys": info["rotation_keys"]}
    del out, ct
    cc.close()
    return rep


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, rank):
    if rank != 0:
        return
    threads = host_threads()
    samples = []
    for _ in range(args.warmup):
        cpu_baseline(threads)
    for _ in range(args.steps):
        v, dt, sample = cpu_baseline(threads)
        samples.append(dt)
    mean = sum(samples) / len(samples)
    value = 1.0 / mean
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u64",
        "data": "synthetic", "config": config_dict(),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"fwd+inv of {POLYS} polys x {LIMBS} limbs x 2^16 per step; "
                                   "CPU oracle restating OpenFHE's NTT (OpenFHE/FIDESlib absent)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict():
    return {"workload": "BASELINE configs[1]: batched forward+inverse negacyclic NTT",
            "log_n": LOG_N, "limbs": LIMBS, "polys": POLYS, "prime_bits": BITS,
            "l2": f"{N_ROTATE} rotating input batches ({N_ROTATE * ALG_BYTES_PER_TRANSFORM // 2 / 1e6:.0f} MB) > L2",
            "parallelism": "independent batch per GPU"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ckks", action="store_true", help="skip the key-switch and matvec side measurements")
    ap.add_argument("--ckks-only", action="store_true",
                    help="print only the key-switch and matvec measurements (profiling runs)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if args.ckks_only:
        ks, mv = measure_ckks(local)
        bt = measure_bootstrap(local)
        print(json.dumps({"keyswitch": ks, "bsgs_matvec": mv, "bootstrap": bt}), flush=True)
        return
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    from fhe_mamba_b200 import NttContext
    from fhe_mamba_b200 import _lib

    qs = bench_primes()
    ctx = NttContext(LOG_N, qs, device=local)
    stream = torch.cuda.ExternalStream(ctx.stream_ptr(), device=torch.device("cuda", local))
    bufs = []
    for i in range(N_ROTATE):
        h = make_batch(qs, 1000 * rank + i)
        bufs.append(torch.from_numpy(h.view(np.int64)).cuda(local))
    torch.cuda.synchronize()

    def step(i, evs=None):
        b = bufs[i % N_ROTATE]
        if evs is not None:
            evs[0].record(stream)
        ctx.forward(b)
        if evs is not None:
            evs[1].record(stream)
        ctx.inverse(b)
        if evs is not None:
            evs[2].record(stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    time.sleep(0.5)

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(args.steps):
        step(i, evs[i])
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()

    total_ms = start.elapsed_time(end)
    fwd_ms = [e[0].elapsed_time(e[1]) for e in evs]
    inv_ms = [e[1].elapsed_time(e[2]) for e in evs]
    t = torch.tensor([total_ms], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    value = world * args.steps / (total_ms / 1e3)

    # End to end through the C ABI with pinned host buffers (copies inside the call).
    host = torch.empty((POLYS, LIMBS, 1 << LOG_N), dtype=torch.int64, pin_memory=True)
    host.copy_(bufs[0].cpu())
    hv = host.numpy().view(np.uint64)
    e2e_steps = max(3, min(args.steps, 20))
    ctx.forward(hv)
    ctx.inverse(hv)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        ctx.forward(hv)
        ctx.inverse(hv)
    e2e_dt = time.perf_counter() - t0
    te = torch.tensor([e2e_dt], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * e2e_steps / float(te.item())
    words = POLYS * LIMBS * (1 << LOG_N)

    fwd_avg = sum(fwd_ms) / len(fwd_ms)
    achieved = ALG_BYTES_PER_TRANSFORM / (fwd_avg / 1e3) / 1e9
    peak, peak_kind = peaks()
    traffic = ncu_traffic()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": config_dict(),
            "roofline": {"bound": "hbm", "kernel": "forward NTT (ntt_fwd_cols + ntt_fwd_rows)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "traffic": traffic,
                         "alg_bytes_per_launch": ALG_BYTES_PER_TRANSFORM,
                         "fwd_ms": fwd_avg, "inv_ms": sum(inv_ms) / len(inv_ms)},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 2 * 8 * words,
                    "d2h_bytes_per_step": 2 * 8 * words,
                    "path": "fhe_ntt + fhe_intt with FHE_MEM_HOST (pinned host buffer)"},
            "gpu_launches": 4 * args.steps,
            "clocks": clocks,
        }
        if not args.no_ckks and world == 1:
            ks, mv = measure_ckks(local)
            line["keyswitch"] = ks
            line["bsgs_matvec"] = mv
            line["bootstrap"] = measure_bootstrap(local)
        if not args.no_cpu_baseline and world == 1:
            v, dt, sample = cpu_baseline(host_threads())
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": host_threads(), "kind": "port",
                                    "sample": sample + "; CPU oracle restating OpenFHE's NTT"}
        print(json.dumps(line), flush=True)

    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
