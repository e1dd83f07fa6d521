"""Benchmark of the CKKS hot path on B200: HRotate key switching (headline),
with the NTT kernel's HBM roofline, an end-to-end number through the C ABI
with host buffers, and the CPU oracle timed on the host cores.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (the CKKS primitive microbench): N = 2^16,
l = 24 limbs of 50-bit NTT primes (q = 1 mod 2^17), dnum = 3 (alpha = 8,
beta = 3), K = 2 special primes, batches of 32 ciphertexts sharing one
rotation key, uniform residues from a seed.  One step = one HRotate of the
whole batch.  Inputs (768 MiB per batch) exceed the 126 MB L2, so no flush
is needed between steps.  Under torchrun every rank rotates its own batch
(independent ciphertexts, no collective on the data path: weak scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "easyfhe-llama3-8b_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "key-switches/s (HRotate, CKKS primitive microbench)"
UNIT = "key-switches/s"
N = 1 << 16
MiB = 1 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--limbs", type=int, default=24)
    ap.add_argument("--dnum", type=int, default=3)
    ap.add_argument("--special", type=int, default=2)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--rotation", type=int, default=1)
    ap.add_argument("--workload", default="hrotate", choices=["hrotate", "ntt"],
                    help="ntt: only the NTT kernel loop (for profiling)")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--cpu-sample", type=int, default=6,
                    help="rotations timed on the CPU oracle")
    return ap.parse_args()


def config(a) -> dict:
    return {
        "workload": (f"HRotate N=2^16 l={a.limbs} 50-bit primes dnum={a.dnum} "
                     f"K={a.special} batch={a.batch} ciphertexts/rank, shared key"),
        "log_n": 16, "limbs": a.limbs, "dnum": a.dnum, "special_primes": a.special,
        "batch_per_rank": a.batch, "rotation": a.rotation,
        "l2": "inputs larger than L2 (768 MiB per batch); no flush",
    }


def algorithmic_mib(a) -> float:
    """C * 2l MiB (ciphertexts in + out) + beta (l + K) MiB (key read once)."""

    beta = -(-a.limbs // -(-a.limbs // a.dnum))
    return a.batch * 2 * a.limbs + beta * (a.limbs + a.special)


class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, enabled: bool):
        self.proc = None
        self.path = None
        if not enabled:
            return
        try:
            out_dir = ROOT / "gpurun_out"
            out_dir.mkdir(exist_ok=True)
            self.path = out_dir / f"clocks_bench_{device_index}.csv"
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(device_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows)}


def cpu_oracle_rate(a, samples: int) -> dict:
    """Time HRotate on the CPU oracle (OpenMP over limbs, all host cores)."""

    import numpy as np

    from oracle import oracle as O

    O.build()
    allp = O.gen_primes(16, 50, a.limbs + a.special)
    q, p = allp[:a.limbs], allp[a.limbs:]
    orc = O.Oracle(16, q, p, a.dnum)
    s = O.sample_secret(16, 2024, 192)
    s_ntt = orc.secret_to_ntt(s)
    g = O.galois_element(16, a.rotation)
    key = orc.keygen_rotation(s_ntt, g, 7)
    rng = np.random.default_rng(5)
    ct = np.empty((2, a.limbs, N), dtype=np.uint64)
    for i, qi in enumerate(q):
        ct[:, i] = rng.integers(0, qi, (2, N), dtype=np.uint64)
    orc.rotate(ct, a.limbs, g, key)  # warm-up
    t0 = time.perf_counter()
    for _ in range(samples):
        orc.rotate(ct, a.limbs, g, key)
    dt = time.perf_counter() - t0
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": samples / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{samples} single-ciphertext HRotates at l={a.limbs}, "
                      f"dnum={a.dnum}, K={a.special} (C oracle, OpenMP over limbs)",
            "seconds": dt}


def run_reference(a) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = cpu_oracle_rate(a, max(1, a.steps))
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": 1000.0 / base["value"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
        "config": config(a),
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "reference EasyFHE is not in the reference tree; the arm times the CPU "
                "restatement of the same algorithm (oracle/), one ciphertext per step",
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    a = parse()
    if a.impl == "reference":
        run_reference(a)
        return

    import torch
    import torch.distributed as dist

    from easyfhe import core

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    params = core.Params.uniform(a.limbs, a.special, a.dnum, bits=50)
    ctx = core.NativeContext(params, dev)
    l, C = a.limbs, a.batch
    s_ntt = ctx.secret_to_ntt(core.sample_secret(2024 + rank, 192))
    g = core.galois_element(a.rotation)
    key = ctx.keygen_rotation(s_ntt, g, seed=7 + rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    ct = torch.empty(C, 2, l, N, dtype=torch.int64, device=dev)
    for i, q in enumerate(params.q):
        ct[:, :, i].random_(0, q, generator=gen)
    out = torch.empty_like(ct)
    ws = ctx.workspace(core.lib.b2f_rotate_workspace(ctx.handle, C, l))
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    from easyfhe import shard

    def max_over_ranks(x: float) -> float:
        return shard.max_over_ranks(x, dev)

    launches_per_rotate = 8  # iNTT, ModUp conv, NTT, inner product, iNTT(P), conv, NTT, combine

    # ---- NTT kernel loop (dominant kernel; roofline) ----
    ntt_buf = ct.view(-1, N)  # C*2*l limbs, 768 MiB
    ntt_limbs = C * 2 * l
    for _ in range(a.warmup):
        ctx.ntt(ntt_buf, l, 0, inverse=False)
        ctx.ntt(ntt_buf, l, 0, inverse=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(2, a.steps // 2)
    e0.record(stream)
    for _ in range(reps):
        ctx.ntt(ntt_buf, l, 0, inverse=False)
        ctx.ntt(ntt_buf, l, 0, inverse=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ntt_ms = e0.elapsed_time(e1) / (2 * reps)  # per launch (fwd and inv averaged)
    ntt_bytes = 16 * N * ntt_limbs
    ntt_gbs = ntt_bytes / (ntt_ms / 1e3) / 1e9
    if a.workload == "ntt":
        if rank == 0:
            print(json.dumps({"workload": "ntt", "limbs": ntt_limbs, "ms": ntt_ms,
                              "gbs": ntt_gbs}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    # ---- headline: HRotate batch, device-resident ----
    for _ in range(a.warmup):
        ctx.rotate(ct, l, g, key, out, ws)
    torch.cuda.synchronize()
    clocks = Clocks(local, not a.no_clocks)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(a.steps):
        ctx.rotate(ct, l, g, key, out, ws)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    value = world * C / (ms / 1e3)
    ntt_ms_max = max_over_ranks(ntt_ms)

    # ---- end to end through the C ABI with pinned host buffers ----
    host_in = torch.empty(ct.shape, dtype=torch.int64, pin_memory=True)
    host_in.copy_(ct)
    host_out = torch.empty(ct.shape, dtype=torch.int64, pin_memory=True)
    dev_in = torch.empty_like(ct)
    e2e_steps = max(2, min(a.steps, 5))
    for _ in range(2):
        dev_in.copy_(host_in, non_blocking=True)
        ctx.rotate(dev_in, l, g, key, out, ws)
        host_out.copy_(out, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    e0.record(stream)
    for _ in range(e2e_steps):
        dev_in.copy_(host_in, non_blocking=True)
        ctx.rotate(dev_in, l, g, key, out, ws)
        host_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    ct_bytes = ct.numel() * 8

    cpu = None
    if rank == 0 and world == 1:
        try:
            cpu = cpu_oracle_rate(a, a.cpu_sample)
            cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as exc:  # the oracle is a reported baseline only
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "port",
                   "sample": f"unavailable: {exc}"}

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    traffic = None
    tpath = ROOT / "profiles" / "ntt_traffic.json"
    if tpath.exists():
        try:
            t = json.loads(tpath.read_text())
            traffic = float(t["bytes_per_limb"]) * ntt_limbs
        except Exception:
            traffic = None

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u64", "data": "synthetic", "config": config(a),
            "roofline": {
                "bound": "hbm", "kernel": "ntt_fwd_kernel/ntt_inv_kernel",
                "achieved": ntt_gbs, "peak": hbm_peak, "unit": "GB/s",
                "frac": ntt_gbs / hbm_peak, "traffic": traffic,
                "peak_source": peak_src,
                "algorithmic_bytes_per_launch": ntt_bytes,
                "launch": f"{ntt_limbs} limbs of 2^16 words (16 N bytes per limb)",
            },
            "ntt_hbm_gbs": ntt_gbs,
            "keyswitch_hbm_gbs": algorithmic_mib(a) * MiB / (ms / 1e3) / 1e9,
            "cpu_baseline": cpu,
            "e2e": {"value": world * C / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": ct_bytes, "d2h_bytes_per_step": ct_bytes},
            "gpu_launches": launches_per_rotate * a.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
