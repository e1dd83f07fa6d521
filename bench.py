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
import math
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
    ap.add_argument("--batch", type=int, default=None,
                    help="ciphertexts per rank (hrotate 32, bootstrap 16, linear 16)")
    ap.add_argument("--rotation", type=int, default=1)
    ap.add_argument("--workload", default="hrotate",
                    choices=["hrotate", "ntt", "bootstrap", "linear"],
                    help="ntt: only the NTT kernel loop (for profiling); bootstrap: "
                         "BASELINE configs[3]; linear: BASELINE configs[2]")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--arith", default="auto", choices=["auto", "int64", "f64"],
                    help="butterfly arithmetic of the NTT kernels (auto: binary64 when "
                         "every prime is below 2^50)")
    ap.add_argument("--per-ct", action="store_true",
                    help="bootstrap/linear: one ciphertext per call (the reference's "
                         "calling pattern) instead of one batched call")
    ap.add_argument("--cpu-sample", type=int, default=6,
                    help="rotations timed on the CPU oracle")
    a = ap.parse_args()
    if a.batch is None:
        a.batch = {"hrotate": 32, "ntt": 32, "bootstrap": 16, "linear": 16}[a.workload]
    return a


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
            # the raw clock samples beside the JSON line's summary
            out_dir = Path(os.environ.get("B2F_BENCH_OUT", ROOT / "bench_out"))
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


def run_bootstrap(a, ctx_dev, rank: int, world: int, barrier, max_over_ranks) -> None:
    """full-slot bootstrapping at the layer parameters
    (logN 16, depth 37, dnum 5, 59/60-bit primes, BootstrapSpec(15, (4, 4),
    19)) of `batch` ciphertexts per rank with uniform complex slots in
    [-1, 1]^2.  One step bootstraps every ciphertext of the batch once."""

    import numpy as np
    import torch

    from easyfhe import fhe
    from easyfhe.bs import openfhe as bs

    dev = ctx_dev
    spec = bs.BootstrapSpec(log_slots=15, level_budget=(4, 4), output_levels=19)
    rots = bs.requirements((spec,), 16).rotations
    client, ctx = fhe.generate_client_context(
        fhe.CKKSContextSpec(depth=37, log_n=16, dnum=5, dcrt_bits=59, first_mod=60,
                            rotations=rots, seed=11 + rank), dev)
    program = bs.generate(ctx, spec)
    rng = np.random.default_rng(77 + rank)
    n = ctx.max_slots
    zs = [rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n) for _ in range(a.batch)]
    cts = [client.encrypt(z, slots=n, cur_limbs=2, scaling_factor=ctx.scale_at(2))
           for z in zs]
    stream = torch.cuda.current_stream()

    def step(inputs):
        if a.per_ct:
            return [bs.bootstrap(c, ctx, program) for c in inputs]
        out = bs.bootstrap(fhe.pack_cipher_batch(inputs), ctx, program)
        return list(fhe.unpack_cipher_batch(out))

    for _ in range(a.warmup):
        outs = step(cts)
    torch.cuda.synchronize()
    clocks = Clocks(dev.index or 0, not a.no_clocks)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(a.steps):
        outs = step(cts)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    err = max(float(np.max(np.abs(client.decrypt_complex(o) - z))) for o, z in zip(outs, zs))

    # end to end: pinned host limbs in, bootstrap, refreshed limbs back out
    host_in = [c.data.cpu().pin_memory() for c in cts]
    host_out = [torch.empty(o.data.shape, dtype=torch.int64, pin_memory=True) for o in outs]
    dev_in = [torch.empty_like(c.data) for c in cts]
    e2e_steps = max(1, min(a.steps, 3))
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        ins = []
        for h, d, c in zip(host_in, dev_in, cts):
            d.copy_(h, non_blocking=True)
            ins.append(fhe.Ciphertext(d, c.state, c.slots, ctx))
        res = step(ins)
        for h, o in zip(host_out, res):
            h.copy_(o.data, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    if rank == 0:
        unit = "bootstraps/s"
        line = {
            "metric": "bootstraps/s (full-slot CKKS bootstrapping, BASELINE configs[3])",
            "value": world * a.batch / (ms / 1e3), "unit": unit, "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u64", "data": "synthetic",
            "config": {"workload": (f"bootstrap N=2^16 depth 37 dnum 5 59/60-bit, "
                                    f"BootstrapSpec(15, (4, 4), 19), batch={a.batch} "
                                    "ciphertexts/rank at 2 limbs"),
                       "batch_per_rank": a.batch,
                       "calls": "one per ciphertext" if a.per_ct else "one batched call",
                       "l2": "working set (keys 29 x up to 230 MiB) larger than L2; no flush"},
            "ms_per_bootstrap": ms / a.batch,
            "precision_bits": -math.log2(err) if err > 0 else None,
            "max_abs_error": err,
            "output_limbs": int(outs[0].state.cur_limbs),
            "roofline": None,
            "cpu_baseline": None,
            "note": "the CPU oracle has no bootstrap; cpu_baseline and the kernel roofline "
                    "are reported on the hrotate line",
            "e2e": {"value": world * a.batch / (e2e_ms / 1e3), "unit": unit,
                    "h2d_bytes_per_step": sum(h.numel() * 8 for h in host_in),
                    "d2h_bytes_per_step": sum(h.numel() * 8 for h in host_out)},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)


def run_linear(a, dev, rank: int, world: int, barrier, max_over_ranks) -> None:
    """the QKV-shaped 4096 -> 4096 feature-major BSGS
    linear at l = 13 with the reference's production plan (B = 64 babies at
    offsets 8 b, giant offset 512, 8 chunks of 512 plaintext rows,
    llama3fhe/operators/linear/config.py:163-317), QuaRot-like synthetic
    weight W = G H (G ~ N(0, 1/sqrt(4096)), H a random-sign Hadamard /
    sqrt(4096)).  The 4096 diagonals are packed and encoded once (timed
    separately); one step runs LinearOperator.apply's call sequence
    (operator.py:320-394) on `batch` token-shard ciphertexts per rank."""

    import numpy as np
    import torch

    from easyfhe import fhe

    D, lanes, B, rows_per_chunk, level = 4096, 8, 64, 512, 13
    slots = 32768
    chunk_giants = rows_per_chunk // B
    G = D // B
    chunks = [(base, min(chunk_giants, G - base)) for base in range(0, G, chunk_giants)]
    giant_offset = B * lanes
    offsets = tuple(b * lanes for b in range(B))
    rotations = set(offsets[1:]) | {giant_offset} | {b * giant_offset for b, _ in chunks if b}
    client, ctx = fhe.generate_client_context(
        fhe.CKKSContextSpec(depth=37, log_n=16, dnum=5, dcrt_bits=59, first_mod=60,
                            rotations=tuple(sorted(rotations)), seed=21 + rank), dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    Gm = torch.randn(D, D, dtype=torch.float64, device=dev, generator=gen) / math.sqrt(D)
    H = torch.ones(1, 1, dtype=torch.float64, device=dev)
    while H.shape[0] < D:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    signs = torch.randint(0, 2, (D,), device=dev, generator=gen).to(torch.float64) * 2 - 1
    W = (Gm @ (H * signs[None, :])) / math.sqrt(D)
    del Gm, H
    scale = ctx.scale_at(level)
    # pack + encode every diagonal once at the working level (timed)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    pts = []
    for base, count in chunks:
        vals = ctx.native.pack_diagonals(W, D, lanes, B, base, count, slots)
        data = ctx.native.encode(vals, scale, level)
        pts.append(fhe.Plaintext(data, fhe.CipherState(level, 1, scale), slots, False))
        del vals
    torch.cuda.synchronize()
    encode_s = time.perf_counter() - t0
    rng = np.random.default_rng(5 + rank)
    tokens = [rng.normal(0, 1, (lanes, D)) for _ in range(a.batch)]

    def layout(t):
        return np.ascontiguousarray(t.T).reshape(-1)  # feature f at slots [8 f, 8 f + 8)

    cts = [client.encrypt(layout(t), slots=slots, cur_limbs=level, scaling_factor=scale)
           for t in tokens]
    stream = torch.cuda.current_stream()

    def apply(ct):
        # LinearOperator.apply's call sequence; ct may be a ciphertext batch
        babies = fhe.prepare_hoisted_baby_rotations(ct, offsets, ctx)
        acc = None
        for (base, count), pt in zip(chunks, pts):
            r = fhe.hoisted_mac_sum(ct, offsets, pt, giant_offset, count, ctx,
                                    baby_rotations=babies)
            if base:
                r = fhe.homo_rotate(r, base * giant_offset, ctx)
            acc = r if acc is None else fhe.homo_add(acc, r, ctx)
        return fhe.rescale(acc, ctx)

    def step(inputs):
        if a.per_ct:
            return [apply(c) for c in inputs]
        return list(fhe.unpack_cipher_batch(apply(fhe.pack_cipher_batch(inputs))))

    for _ in range(a.warmup):
        outs = step(cts)
    torch.cuda.synchronize()
    clocks = Clocks(dev.index or 0, not a.no_clocks)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(a.steps):
        outs = step(cts)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    Wn = W.cpu().numpy()
    err = max(float(np.max(np.abs(client.decrypt(o) - layout(t @ Wn.T))))
              for o, t in zip(outs[:2], tokens[:2]))

    host_in = [c.data.cpu().pin_memory() for c in cts]
    host_out = [torch.empty(o.data.shape, dtype=torch.int64, pin_memory=True) for o in outs]
    dev_in = [torch.empty_like(c.data) for c in cts]
    e2e_steps = max(1, min(a.steps, 3))
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        ins = []
        for h, d, c in zip(host_in, dev_in, cts):
            d.copy_(h, non_blocking=True)
            ins.append(fhe.Ciphertext(d, c.state, c.slots, ctx))
        res = step(ins)
        for h, o in zip(host_out, res):
            h.copy_(o.data, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    if rank == 0:
        peaks = {}
        try:
            peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        except Exception:
            pass
        hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
        # algorithmic bytes: the plaintext rows once per call (once per
        # ciphertext when called per ciphertext, as the reference does; once
        # per batch otherwise), babies and outputs once
        lim = N * 8
        pt_reads = a.batch if a.per_ct else 1
        alg = (pt_reads * D * level * lim
               + a.batch * (B * 2 * level * lim + 2 * level * lim))
        unit = "ciphertexts/s"
        line = {
            "metric": "linear-block ciphertexts/s (QKV-shaped 4096x4096 BSGS, BASELINE configs[2])",
            "value": world * a.batch / (ms / 1e3), "unit": unit, "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u64", "data": "synthetic",
            "config": {"workload": (f"QKV-shaped linear D=4096 l={level} B=64 G=64 in 8 chunks, "
                                    f"{a.batch} token-shard ciphertexts/rank, depth 37 dnum 5"),
                       "batch_per_rank": a.batch,
                       "calls": "one per ciphertext" if a.per_ct else "one batched call",
                       "l2": "plaintexts 26 GiB > L2; no flush"},
            "pt_x_ct_per_s": world * a.batch * D / (ms / 1e3),
            "encode_rows_per_s": D / encode_s,
            "max_abs_error": err,
            "roofline": {"bound": "hbm", "kernel": "whole step", "achieved":
                         alg / (ms / 1e3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                         "frac": alg / (ms / 1e3) / 1e9 / hbm_peak, "traffic": None},
            "cpu_baseline": None,
            "note": "cpu_baseline is reported on the hrotate line",
            "e2e": {"value": world * a.batch / (e2e_ms / 1e3), "unit": unit,
                    "h2d_bytes_per_step": sum(h.numel() * 8 for h in host_in),
                    "d2h_bytes_per_step": sum(h.numel() * 8 for h in host_out)},
            "clocks": clk,
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

    from easyfhe import shard

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        return shard.max_over_ranks(x, dev)

    if a.workload == "bootstrap":
        run_bootstrap(a, dev, rank, world, barrier, max_over_ranks)
        if world > 1:
            dist.destroy_process_group()
        return
    if a.workload == "linear":
        run_linear(a, dev, rank, world, barrier, max_over_ranks)
        if world > 1:
            dist.destroy_process_group()
        return

    params = core.Params.uniform(a.limbs, a.special, a.dnum, bits=50)
    ctx = core.NativeContext(params, dev)
    ctx.set_arith(a.arith)
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

    # iNTT, ModUp conversion, NTT, inner product, iNTT of the P part, ModDown
    # conversion, NTT + combine; binary64 with K <= 4 computes the ModDown
    # conversion inside its NTT (no separate conversion launch)
    launches_per_rotate = 6 if (ctx.arith == "f64" and a.special <= 4) else 7

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
    # the NTT is bound by 64-bit multiplies on CUDA cores: its butterfly rate
    # against the register-only rate of the same butterfly on this GPU
    ntt_bfly = ntt_limbs * (N // 2) * 16 / (ntt_ms / 1e3)
    bfly_peak = ctx.butterfly_peak()
    if a.workload == "ntt":
        if rank == 0:
            print(json.dumps({"workload": "ntt", "limbs": ntt_limbs, "ms": ntt_ms,
                              "us_per_limb": ntt_ms * 1e3 / ntt_limbs, "gbs": ntt_gbs,
                              "arith": ctx.arith,
                              "butterflies_per_s": ntt_bfly, "butterfly_peak": bfly_peak,
                              "frac": ntt_bfly / bfly_peak}), flush=True)
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
    # Three streams pipeline the steps: the upload of step i+1 and the
    # download of step i-1 overlap the rotation of step i (double-buffered
    # device inputs and outputs).  Every step still copies its whole batch
    # in and its whole result out; events bracket the first upload and the
    # last download.
    host_in = torch.empty(ct.shape, dtype=torch.int64, pin_memory=True)
    host_in.copy_(ct)
    host_out = [torch.empty(ct.shape, dtype=torch.int64, pin_memory=True) for _ in range(2)]
    dev_in = [torch.empty_like(ct) for _ in range(2)]
    dev_out = [torch.empty_like(ct) for _ in range(2)]
    s_up, s_rot, s_down = (torch.cuda.Stream(device=dev) for _ in range(3))
    e2e_steps = max(4, min(a.steps, 30))

    def e2e_run(steps: int) -> float:
        up_done = [torch.cuda.Event() for _ in range(steps)]
        rot_done = [torch.cuda.Event() for _ in range(steps)]
        down_done = [torch.cuda.Event() for _ in range(steps)]
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(s_up)
        for i in range(steps):
            b = i % 2
            with torch.cuda.stream(s_up):
                if i >= 2:
                    s_up.wait_event(rot_done[i - 2])  # dev_in[b] is free again
                dev_in[b].copy_(host_in, non_blocking=True)
                up_done[i].record(s_up)
            with torch.cuda.stream(s_rot):
                s_rot.wait_event(up_done[i])
                if i >= 2:
                    s_rot.wait_event(down_done[i - 2])  # dev_out[b] is free again
                ctx.rotate(dev_in[b], l, g, key, dev_out[b], ws)
                rot_done[i].record(s_rot)
            with torch.cuda.stream(s_down):
                s_down.wait_event(rot_done[i])
                host_out[b].copy_(dev_out[b], non_blocking=True)
                down_done[i].record(s_down)
        t1.record(s_down)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / steps

    e2e_run(2)  # warm-up
    barrier()
    e2e_ms = max_over_ranks(e2e_run(e2e_steps))
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
            "compute_roofline": {
                "bound": "fp64" if ctx.arith == "f64" else "imad",
                "kernel": "ntt_fwd_kernel/ntt_inv_kernel",
                "achieved": ntt_bfly, "peak": bfly_peak, "unit": "butterflies/s",
                "frac": ntt_bfly / bfly_peak,
                "peak_source": ("measured live: b2f_butterfly_peak (the NTT's lazy "
                                f"{ctx.arith} butterfly from registers, every SM full)"),
            },
            "arith": ctx.arith,
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
