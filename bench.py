"""Benchmark of the CKKS evaluation hot path of encrypted Llama-3-8B prefill on
B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload linear|hrotate|ntt|bootstrap|layer0]

Default workload: the encrypted linear block of a layer, the 4096 -> 4096
feature-major BSGS plaintext x ciphertext matmul at l = 13 with the
reference's production plan, over a fixed set of 16 token-shard ciphertexts
(N = 2^16, depth 37, dnum 5, 59/60-bit primes).  One step = the linear on
every ciphertext; under torchrun the ciphertexts are sharded by output
ciphertext over the ranks and the outputs are all-gathered over NCCL inside
the step (strong scaling).  At N = 1 the line also carries the HRotate
microbench (50-bit primes, l = 24, dnum 3, K = 2, 32 ciphertexts sharing one
key) with the NTT kernel's roofline, and one encrypted decoder layer through
the reference's own graph (s/layer).  Inputs exceed the 126 MB L2, so no
flush is needed between steps.
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
    ap.add_argument("--workload", default="linear",
                    choices=["linear", "hrotate", "ntt", "bootstrap", "layer0", "mac",
                             "prefill", "mlp"],
                    help="linear (default): the encrypted 4096x4096 linear block sharded "
                         "over the ranks with an all-gather; hrotate: the key-switching "
                         "microbench; ntt: only the NTT kernel loop (for profiling); "
                         "bootstrap: full-slot bootstrapping; layer0: one encrypted "
                         "decoder layer through the reference's graph")
    ap.add_argument("--layer-params", action="store_true",
                    help="hrotate/ntt: the layer's chain (depth 37, dnum 5, 59/60-bit "
                         "primes, K = 8) instead of 50-bit primes; --limbs picks the level")
    ap.add_argument("--linear-chunks", type=int, default=0,
                    help="linear: only the plan's first N chunks of 512 rows (a smaller "
                         "linear block, for profiling captures; 0 = all 8)")
    ap.add_argument("--no-extras", action="store_true",
                    help="linear at N = 1: skip the HRotate, Layer-0 and CPU attachments")
    ap.add_argument("--num-layers", type=int, default=32,
                    help="prefill: decoder layers through the reference's model loop")
    ap.add_argument("--no-check", action="store_true",
                    help="prefill: skip the fp64 check of the decrypted output")
    ap.add_argument("--no-layer", action="store_true",
                    help="skip the Layer-0 run the default line carries at N = 1")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--conv-path", default="auto", choices=["auto", "tcgen05", "mma_sync"],
                    help="key-switch base conversions: the faster kernel of each (auto), "
                         "tcgen05 or mma.sync for both")
    ap.add_argument("--giant-chain", default="extended", choices=["extended", "rotations"],
                    help="BSGS Horner chain over the giants: kept in Q_l u P with one "
                         "ModDown per chain (extended) or a full HRotate per giant")
    ap.add_argument("--hoist-strategy", default="normal",
                    choices=["normal", "ext_normal", "ext_double_hoist"],
                    help="linear and layer0: the hoisted-MAC schedule, as the reference's "
                         "--linear-hoist-strategy (normal: its production schedule; the "
                         "extended ones leave the babies in Q_l u P)")
    ap.add_argument("--mac-path", default="auto", choices=["auto", "cuda_cores"],
                    help="BSGS multiply-accumulate kernel: u8 tensor cores where exact "
                         "(auto) or the CUDA-core kernel")
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
        a.batch = {"hrotate": 32, "ntt": 32, "bootstrap": 16, "linear": 16,
                   "layer0": 16, "mac": 16, "prefill": 16, "mlp": 16}[a.workload]
    return a


def config(a) -> dict:
    if getattr(a, "layer_params", False):
        return {
            "workload": (f"HRotate N=2^16 at l={a.limbs} of the layer chain (depth 37, dnum 5, "
                         f"59/60-bit primes, K=8 special), batch={a.batch} ciphertexts/rank, "
                         "shared key"),
            "log_n": 16, "limbs": a.limbs, "dnum": 5, "special_primes": 8,
            "batch_per_rank": a.batch, "rotation": a.rotation,
            "l2": "inputs larger than L2; no flush",
        }
    return {
        "workload": (f"HRotate N=2^16 l={a.limbs} 50-bit primes dnum={a.dnum} "
                     f"K={a.special} batch={a.batch} ciphertexts/rank, shared key"),
        "log_n": 16, "limbs": a.limbs, "dnum": a.dnum, "special_primes": a.special,
        "batch_per_rank": a.batch, "rotation": a.rotation,
        "l2": "inputs larger than L2 (768 MiB per batch); no flush",
    }


def algorithmic_mib(l: int, batch: int, alpha: int, K: int) -> float:
    """C * 2l MiB (ciphertexts in + out) + beta (l + K) MiB (key read once),
    beta = ceil(l / alpha) digits."""

    return batch * 2 * l + (-(-l // alpha)) * (l + K)


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
    """The reference arm: the reference's implementation of the path, EasyFHE,
    is not in the reference tree (nor installable), so this times the CPU
    restatement of the same algorithm (oracle/, C with OpenMP) on the host
    cores for the same workload and metric.  Under torchrun rank 0 alone runs
    it; torchrun sets OMP_NUM_THREADS=1, so the thread count is set here to
    every host core before the oracle loads."""

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)
    samples = max(1, min(a.steps, 3))
    if a.workload in ("hrotate", "ntt"):
        base = cpu_oracle_rate(a, samples)
        metric, unit, cfg, scaling = METRIC, UNIT, config(a), "weak"
    elif a.workload == "linear":
        base = linear_cpu_rate(samples=samples)
        metric = ("encrypted linear-block ciphertexts/s (4096x4096 feature-major BSGS "
                  "plaintext x ciphertext matmul, l=13)")
        unit, scaling = "ciphertexts/s", "strong"
        cfg = {"workload": (f"linear 4096->4096 D=4096 l={LINEAR_LEVEL} B=64 babies, 64 giants "
                            "in 8 chunks of 512 rows, one ciphertext per sample"),
               "ciphertexts_total": a.batch}
    else:
        print(json.dumps({"impl": "reference", "unavailable":
                          f"no CPU restatement of the {a.workload} workload in the oracle"}))
        return
    line = {
        "impl": "reference", "metric": metric, "value": base["value"], "unit": unit,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": 1000.0 / base["value"], "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "u64", "data": "synthetic",
        "config": cfg,
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": ("reference EasyFHE is not in the reference tree; the arm times the CPU "
                 f"restatement of the same algorithm (oracle/), {samples} bounded samples "
                 f"on {base['cores']} host threads"),
    }
    print(json.dumps(line), flush=True)


def count_keyswitches(native, fn) -> dict:
    """Run fn() once with the context's key-switching entry points counted:
    {limbs: key switches at that level} (rotations, hoisted rotations,
    relinearisations, the Horner giants inside a BSGS multiply-accumulate)."""

    import collections

    counts = collections.Counter()
    orig = {}

    def wrap(name, how):
        f = getattr(native, name)
        orig[name] = f

        def w(*args, **kw):
            l, k = how(args, kw)
            counts[int(l)] += int(k)
            return f(*args, **kw)
        setattr(native, name, w)

    n = native.n
    wrap("rotate", lambda a, k: (a[1], a[0].numel() // (2 * a[1] * n)))
    wrap("rotate_hoisted", lambda a, k: (a[1], sum(g != 1 for g in a[3])
                                         * k.get("num_cts", 1)))
    wrap("rotate_hoisted_ext", lambda a, k: (a[1], sum(g != 1 for g in a[3])))
    wrap("relinearize", lambda a, k: (a[1], a[0].numel() // (3 * a[1] * n)))
    wrap("relinearize_rescale", lambda a, k: (a[1], a[0].numel() // (3 * a[1] * n)))
    wrap("bsgs_mac", lambda a, k: (a[4], (a[3] - 1) * k.get("num_cts", 1)))
    try:
        fn()
    finally:
        for name, f in orig.items():
            setattr(native, name, f)
    return dict(counts)


def keyswitch_cpu_seconds(params, counts: dict, samples: int = 1) -> tuple[float, str]:
    """CPU seconds of the counted key switches on the oracle: HRotate timed at
    the lowest, middle and highest level used, interpolated linearly in the
    limbs for the rest."""

    import numpy as np

    from oracle import oracle as O

    O.build()
    orc = O.Oracle(16, list(params.q), list(params.p), params.dnum)
    s_ntt = orc.secret_to_ntt(O.sample_secret(16, 2024, 192))
    g = O.galois_element(16, 1)
    key = orc.keygen_rotation(s_ntt, g, 7)
    rng = np.random.default_rng(3)
    levels = sorted(counts)
    probes = sorted({levels[0], levels[len(levels) // 2], levels[-1]})
    t = {}
    for l in probes:
        ct = np.empty((2, l, N), dtype=np.uint64)
        for i, qi in enumerate(params.q[:l]):
            ct[:, i] = rng.integers(0, qi, (2, N), dtype=np.uint64)
        t0 = time.perf_counter()
        for _ in range(samples):
            orc.rotate(ct, l, g, key)
        t[l] = (time.perf_counter() - t0) / samples
    xs = np.array(probes, dtype=np.float64)
    ys = np.array([t[l] for l in probes])
    total = float(sum(c * np.interp(l, xs, ys) for l, c in counts.items()))
    sample = (f"C oracle HRotate at l = {', '.join(str(l) for l in probes)} "
              f"({', '.join(f'{t[l]:.2f} s' for l in probes)}), interpolated over the "
              f"{sum(counts.values())} key switches one bootstrap issues; the rest of the "
              "bootstrap (NTT-free elementwise work, encoding) is not counted: a lower bound")
    return total, sample


def run_bootstrap(a, ctx_dev, rank: int, world: int, barrier, max_over_ranks) -> None:
    """Full-slot CKKS bootstrapping at the layer parameters
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
    ctx.native.set_giant_chain(a.giant_chain)
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
    boot_roofline = boot_cpu = ks_per_boot = None
    if rank == 0:
        # the dominant kernel: the NTT of the layer chain (integer arithmetic)
        # over the batch's polynomials at the full 38 limbs, timed live
        nat = ctx.native
        buf = torch.empty(a.batch * 2 * ctx.L, N, dtype=torch.int64, device=dev)
        for i, q in enumerate(ctx.params.q):
            buf.view(a.batch * 2, ctx.L, N)[:, i].random_(0, q)
        nat.ntt(buf, ctx.L)
        nat.ntt(buf, ctx.L, inverse=True)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 4
        t0.record(stream)
        for _ in range(reps):
            nat.ntt(buf, ctx.L)
            nat.ntt(buf, ctx.L, inverse=True)
        t1.record(stream)
        torch.cuda.synchronize()
        ntt_ms = t0.elapsed_time(t1) / (2 * reps)
        limbs = a.batch * 2 * ctx.L
        peaks = {}
        try:
            peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        except Exception:
            pass
        hbm = float(peaks.get("hbm_gbs", 6650.0))
        gbs = 16 * N * limbs / (ntt_ms / 1e3) / 1e9
        bfly = limbs * (N // 2) * 16 / (ntt_ms / 1e3)
        boot_roofline = {"bound": "hbm", "kernel": f"ntt_fwd_kernel/ntt_inv_kernel ({nat.arith})",
                         "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "traffic": None, "algorithmic_bytes_per_launch": 16 * N * limbs,
                         "launch": f"{limbs} limbs of 2^16 words, {ntt_ms:.3f} ms",
                         "compute_frac": bfly / nat.butterfly_peak()}
        del buf
        # CPU: the key switches of one bootstrap, priced on the oracle
        one = cts[0]
        counts = count_keyswitches(nat, lambda: bs.bootstrap(one, ctx, program))
        ks_per_boot = {"total": sum(counts.values()), "by_limbs": counts}
        try:
            os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
            sec, sample = keyswitch_cpu_seconds(ctx.params, counts)
            boot_cpu = {"value": 1.0 / sec, "unit": "bootstraps/s",
                        "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)),
                        "kind": "port", "sample": sample}
        except Exception as exc:  # a reported baseline only
            boot_cpu = {"value": None, "unit": "bootstraps/s", "cores": 0, "kind": "port",
                        "sample": f"unavailable: {exc}"}
    if rank == 0:
        unit = "bootstraps/s"
        line = {
            "metric": "bootstraps/s (full-slot CKKS bootstrapping, 2^15 slots, 16-112 ciphertexts)",
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
            "roofline": boot_roofline,
            "cpu_baseline": boot_cpu,
            "keyswitches_per_bootstrap": ks_per_boot,
            "note": ("roofline: the integer NTT (the bootstrap's dominant kernel) timed live "
                     "on this context over the batch's 38-limb polynomials"),
            "e2e": {"value": world * a.batch / (e2e_ms / 1e3), "unit": unit,
                    "h2d_bytes_per_step": sum(h.numel() * 8 for h in host_in),
                    "d2h_bytes_per_step": sum(h.numel() * 8 for h in host_out)},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)


LINEAR_D, LINEAR_LANES, LINEAR_B, LINEAR_ROWS, LINEAR_LEVEL = 4096, 8, 64, 512, 13


def linear_plan():
    """The production plan of the 4096 -> 4096 feature-major linear
    (llama3fhe/operators/linear/config.py:163-317): B = 64 babies at offsets
    8 b, giant offset 512, chunks of 512 plaintext rows (8 giants)."""

    D, lanes, B, rows = LINEAR_D, LINEAR_LANES, LINEAR_B, LINEAR_ROWS
    G = D // B
    per = rows // B
    chunks = [(base, min(per, G - base)) for base in range(0, G, per)]
    offsets = tuple(b * lanes for b in range(B))
    return chunks, offsets, B * lanes


def linear_cpu_rate(samples: int = 1, samples_rows: int = 64) -> dict:
    """The linear block on the CPU oracle, one token-shard ciphertext, from a
    bounded sample: the 63 hoisted baby rotations, then `samples_rows`
    plaintext rows of the multiply-accumulate and one giant rotation, scaled
    to the full 4096 rows, 56 Horner giant rotations and 7 chunk alignments
    (every rotation costs one key switch at l = 13)."""

    import numpy as np

    from oracle import oracle as O

    O.build()
    l, K, dnum = LINEAR_LEVEL, 8, 5
    allp = O.gen_primes(16, 59, l + K)
    q, p = allp[:l], allp[l:]
    orc = O.Oracle(16, q, p, dnum)
    s_ntt = orc.secret_to_ntt(O.sample_secret(16, 2024, 192))
    chunks, offsets, giant_offset = linear_plan()
    rng = np.random.default_rng(5)
    ct = np.empty((2, l, N), dtype=np.uint64)
    for i, qi in enumerate(q):
        ct[:, i] = rng.integers(0, qi, (2, N), dtype=np.uint64)
    gal = [O.galois_element(16, r) for r in offsets[1:]]
    keys = [orc.keygen_rotation(s_ntt, g, 40 + j) for j, g in enumerate(gal[:2])]
    pts = np.empty((samples_rows, l, N), dtype=np.uint64)
    for i, qi in enumerate(q):
        pts[:, i] = rng.integers(0, qi, (samples_rows, N), dtype=np.uint64)
    t_two = t_rot = t_mac = 0.0
    for _ in range(samples):
        # 63 babies share one ModUp: time two and scale the key switches
        t0 = time.perf_counter()
        babies2 = orc.rotate_hoisted(ct, l, gal[:2], keys)
        t_two += (time.perf_counter() - t0) / samples
        t0 = time.perf_counter()
        orc.rotate(ct, l, gal[0], keys[0])
        t_rot += (time.perf_counter() - t0) / samples
        babies = np.concatenate([ct[None], np.repeat(babies2[:1], samples_rows - 1, 0)])
        t0 = time.perf_counter()
        orc.bsgs_mac(babies, 1, samples_rows, pts, 1, l)
        t_mac += (time.perf_counter() - t0) / samples
    rotations = len(offsets) - 1
    giants = sum(c for _, c in chunks) - len(chunks)  # Horner steps
    align = len(chunks) - 1
    per_ct = (t_two * rotations / 2 + t_mac * LINEAR_D / samples_rows
              + t_rot * (giants + align))
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": 1.0 / per_ct, "unit": "ciphertexts/s", "cores": cores, "kind": "port",
            "sample": (f"C oracle (OpenMP over limbs) on one ciphertext at l={l}: 2 hoisted "
                       f"rotations ({t_two:.2f} s), one rotation ({t_rot:.2f} s), "
                       f"{samples_rows} of 4096 plaintext rows of the MAC ({t_mac:.2f} s), "
                       f"scaled to 63 babies + 4096 rows + {giants + align} rotations"),
            "seconds": t_two + t_rot + t_mac}


def run_linear(a, dev, rank: int, world: int, barrier, max_over_ranks) -> dict | None:
    """The encrypted linear block (the 4096 -> 4096 q/o shape) on a fixed
    set of token-shard ciphertexts, sharded by output ciphertext over the
    ranks: rank r runs LinearOperator.apply's call sequence
    (llama3fhe/operators/linear/operator.py:320-394) with the production plan
    on its 16/N ciphertexts as one batch, then the outputs are all-gathered
    over NCCL into every rank's HBM (the stage-boundary exchange).  The
    weight is QuaRot-like synthetic, W = G H (G ~ N(0, 1/sqrt(4096)), H a
    random-sign Hadamard / sqrt(4096)); its 4096 diagonals are packed and
    encoded once per rank, outside the timed step."""

    import numpy as np
    import torch
    import torch.distributed as dist

    from easyfhe import _native, fhe

    D, lanes, B, level = LINEAR_D, LINEAR_LANES, LINEAR_B, LINEAR_LEVEL
    slots = 32768
    total = a.batch
    strategy = a.hoist_strategy
    ext = strategy != "normal"
    if total % world:
        raise SystemExit(f"{total} ciphertexts do not split over {world} ranks")
    per = total // world
    chunks, offsets, giant_offset = linear_plan()
    if a.linear_chunks:
        chunks = chunks[: a.linear_chunks]
    rotations = set(offsets[1:]) | {giant_offset} | {b * giant_offset for b, _ in chunks if b}
    client, ctx = fhe.generate_client_context(
        fhe.CKKSContextSpec(depth=37, log_n=16, dnum=5, dcrt_bits=59, first_mod=60,
                            rotations=tuple(sorted(rotations)), seed=21), dev)
    ctx.native.set_mac_path(a.mac_path)
    ctx.native.set_conv_path(a.conv_path)
    ctx.native.set_giant_chain(a.giant_chain)
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
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    pts = []
    for base, count in chunks:
        vals = ctx.native.pack_diagonals(W, D, lanes, B, base, count, slots)
        data = ctx.native.encode(vals, scale, level, ctx.K if ext else 0)
        pts.append(fhe.Plaintext(data, fhe.CipherState(level, 1, scale), slots, ext))
        del vals
    torch.cuda.synchronize()
    encode_s = time.perf_counter() - t0
    rng = np.random.default_rng(5)
    tokens = [rng.normal(0, 1, (lanes, D)) for _ in range(total)]  # every rank: same set

    def layout(t):
        return np.ascontiguousarray(t.T).reshape(-1)  # feature f at slots [8 f, 8 f + 8)

    mine = range(rank * per, (rank + 1) * per)
    cts = [client.encrypt(layout(tokens[i]), slots=slots, cur_limbs=level, scaling_factor=scale)
           for i in mine]
    stream = torch.cuda.current_stream()
    gathered = torch.empty(total, 2, level - 1, N, dtype=torch.int64, device=dev)
    gather_ev = []

    def apply(ct):
        # LinearOperator.apply's call sequence; ct is this rank's batch
        babies = fhe.prepare_hoisted_baby_rotations(ct, offsets, ctx, strategy=strategy)
        acc = None
        for (base, count), pt in zip(chunks, pts):
            r = fhe.hoisted_mac_sum(ct, offsets, pt, giant_offset, count, ctx,
                                    strategy=strategy, baby_rotations=babies)
            if base:
                r = fhe.homo_rotate(r, base * giant_offset, ctx)
            acc = r if acc is None else fhe.homo_add(acc, r, ctx)
        return fhe.rescale(acc, ctx)

    out_state = {}

    def step(inputs, record=False):
        res = apply(fhe.pack_cipher_batch(inputs))
        out_state["state"] = res.state
        out = res.data.reshape(per, 2, level - 1, N)
        if world > 1:  # the stage-boundary exchange: every rank gets every output
            if record:
                e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                e[0].record(stream)
            dist.all_gather_into_tensor(gathered, out.contiguous())
            if record:
                e[1].record(stream)
                gather_ev.append(e)
            return gathered
        return out

    for _ in range(a.warmup):
        outs = step(cts)
    torch.cuda.synchronize()
    clocks = Clocks(dev.index or 0, not a.no_clocks)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    n0 = _native.lib.b2f_launch_count()
    e0.record(stream)
    for _ in range(a.steps):
        outs = step(cts, record=True)
    e1.record(stream)
    torch.cuda.synchronize()
    launches = (_native.lib.b2f_launch_count() - n0) // a.steps
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    gather_ms = max_over_ranks(sum(x.elapsed_time(y) for x, y in gather_ev) / a.steps
                               if gather_ev else 0.0)
    err = None
    if rank == 0 and not a.linear_chunks:  # first and last ciphertext of the gathered set
        Wn = W.cpu().numpy()
        err = max(float(np.max(np.abs(
            client.decrypt(fhe.Ciphertext(outs[j], out_state["state"], slots, ctx))
            - layout(tokens[j] @ Wn.T)))) for j in (0, total - 1))

    # ---- the MAC kernel alone: one chunk's launch on this rank's batch ----
    batch = fhe.pack_cipher_batch(cts)
    babies = tuple(fhe.prepare_hoisted_baby_rotations(batch, offsets, ctx,
                                                      strategy=strategy))[0]
    G0 = chunks[0][1]
    mac_reps = max(3, min(a.steps, 10))

    def mac_launch():
        if ext:  # over Q_l u P
            ctx.native.mac_ext(babies.data, B, pts[0].data, G0, level, num_cts=per)
        else:
            ctx.native.mac(babies.data, B, pts[0].data, G0, level, num_cts=per)

    mac_launch()
    torch.cuda.synchronize()
    m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    m0.record(stream)
    for _ in range(mac_reps):
        mac_launch()
    m1.record(stream)
    torch.cuda.synchronize()
    mac_ms = m0.elapsed_time(m1) / mac_reps
    mac_name = ctx.native.mac_kernel(B, level, ctx.K if ext else 0, num_cts=per,
                                     giant_count=G0)
    on_tc = mac_name == "mac_mma_kernel"
    mac_peak = ctx.native.mma_u8_peak() if on_tc else ctx.native.mac_peak()
    del babies, batch

    # ---- end to end: pinned host ciphertexts in, outputs out ----
    host_in = [c.data.cpu().pin_memory() for c in cts]
    host_out = torch.empty(tuple(outs.shape), dtype=torch.int64, pin_memory=True)
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
        if rank == 0:  # the job's result: every output ciphertext, on rank 0's host
            host_out.copy_(res, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    if rank != 0:
        return None
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    lim = N * 8
    # algorithmic bytes of one MAC launch (one chunk of G0 giants on `per`
    # ciphertexts): the plaintext rows once, the babies once, outputs
    lk = level + (ctx.K if ext else 0)  # limbs the MAC runs over
    mac_bytes = (G0 * B * lk + per * B * 2 * lk + per * G0 * 2 * lk) * lim
    macs = G0 * B * per * 2 * lk * N  # 64 x 64-bit products per launch
    traffic = None
    tpath = ROOT / "profiles" / f"{mac_name}_traffic.json"
    if tpath.exists() and not ext:  # captured over Q_l at l = 13
        try:
            t = json.loads(tpath.read_text())
            # DRAM bytes per launch scale with the ciphertexts of the launch
            traffic = float(t["bytes_fixed"]) + float(t["bytes_per_ct"]) * per
        except Exception:
            traffic = None
    unit = "ciphertexts/s"
    return {
        "metric": ("encrypted linear-block ciphertexts/s (4096x4096 feature-major BSGS "
                   "plaintext x ciphertext matmul, l=13)"),
        "value": total / (ms / 1e3), "unit": unit, "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u64", "data": "synthetic",
        "config": {"workload": (f"linear 4096->4096 D=4096 l={level} B=64 babies, 64 giants in "
                                f"8 chunks of 512 rows (the reference's production plan"
                                f"{'' if not ext else ', hoist strategy ' + strategy}), "
                                f"{total} token-shard ciphertexts sharded {per}/rank, outputs "
                                "all-gathered over NCCL in every step; logN 16 depth 37 dnum 5 "
                                "59/60-bit primes"),
                   "ciphertexts_total": total, "ciphertexts_per_rank": per,
                   "hoist_strategy": strategy,
                   "chunks": (len(chunks) if not a.linear_chunks else
                              f"{len(chunks)} of 8 (a smaller linear: --linear-chunks)"),
                   "parallelism": f"output-ciphertext sharding x{world} + all-gather",
                   "l2": "plaintexts 3.3 GB per chunk, babies 13.6 GB per 16 ciphertexts: "
                         "inputs far larger than L2; no flush"},
        "pt_x_ct_per_s": total * B * sum(c for _, c in chunks) / (ms / 1e3),
        "encode_rows_per_s": D / encode_s,
        "max_abs_error": err,
        "gather_ms_per_step": gather_ms,
        "gather_share": gather_ms / ms if ms else None,
        "roofline": {"bound": "hbm", "kernel": mac_name,
                     "achieved": mac_bytes / (mac_ms / 1e3) / 1e9, "peak": hbm_peak,
                     "unit": "GB/s", "frac": mac_bytes / (mac_ms / 1e3) / 1e9 / hbm_peak,
                     "traffic": traffic, "peak_source": "measured" if peaks else "fallback",
                     "algorithmic_bytes_per_launch": mac_bytes,
                     "launch": (f"one chunk: {G0} giants x {B} babies x {per} ciphertexts "
                                f"at l={level}; {mac_ms:.3f} ms per launch"),
                     "products_per_s": macs / (mac_ms / 1e3)},
        "compute_roofline": mac_compute_roofline(mac_name, macs, mac_ms, mac_peak),
        "gpu_launches": launches,
        "e2e": {"value": total / (e2e_ms / 1e3), "unit": unit,
                "h2d_bytes_per_step": sum(h.numel() * 8 for h in host_in) * world,
                "d2h_bytes_per_step": host_out.numel() * 8},
        "clocks": clk,
    }


def run_hrotate(a, dev, rank: int, world: int, barrier, max_over_ranks,
                with_cpu: bool = True) -> dict | None:
    """HRotate of `a.batch` ciphertexts per rank sharing one key (the CKKS
    primitive microbench): device-resident key-switches/s, the NTT kernel's
    roofline, and the same rotations end to end through the C ABI with
    pinned host buffers.  Returns rank 0's JSON line."""

    import torch

    from easyfhe import _native, core

    if getattr(a, "layer_params", False):  # the layer chain (assets/feature_major.json)
        params = core.Params.from_depth(37, 16, 5, 59, 60)
    else:
        params = core.Params.uniform(a.limbs, a.special, a.dnum, bits=50)
    ctx = core.NativeContext(params, dev)
    ctx.set_arith(a.arith)
    ctx.set_conv_path(a.conv_path)
    l, C = a.limbs, a.batch
    if not 1 <= l <= params.L:
        raise SystemExit(f"--limbs {l} outside the chain's 1..{params.L}")
    s_ntt = ctx.secret_to_ntt(core.sample_secret(2024 + rank, 192))
    g = core.galois_element(a.rotation)
    key = ctx.keygen_rotation(s_ntt, g, seed=7 + rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    ct = torch.empty(C, 2, l, N, dtype=torch.int64, device=dev)
    for i, q in enumerate(params.q[:l]):
        ct[:, :, i].random_(0, q, generator=gen)
    out = torch.empty_like(ct)
    ws = ctx.workspace(core.lib.b2f_rotate_workspace(ctx.handle, C, l))
    stream = torch.cuda.current_stream()

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
        return {"workload": "ntt", "limbs": ntt_limbs, "ms": ntt_ms,
                "us_per_limb": ntt_ms * 1e3 / ntt_limbs, "gbs": ntt_gbs, "arith": ctx.arith,
                "butterflies_per_s": ntt_bfly, "butterfly_peak": bfly_peak,
                "frac": ntt_bfly / bfly_peak} if rank == 0 else None

    # ---- headline: HRotate batch, device-resident ----
    for _ in range(a.warmup):
        ctx.rotate(ct, l, g, key, out, ws)
    torch.cuda.synchronize()
    clocks = Clocks(dev.index or 0, not a.no_clocks)
    barrier()
    torch.cuda.synchronize()
    n0 = _native.lib.b2f_launch_count()
    e0.record(stream)
    for _ in range(a.steps):
        ctx.rotate(ct, l, g, key, out, ws)
    e1.record(stream)
    torch.cuda.synchronize()
    launches = (_native.lib.b2f_launch_count() - n0) // a.steps
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
    if rank == 0 and world == 1 and with_cpu:
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
            # the capture is of one arithmetic's kernel: use it for that one only
            want = "FpArith" if ctx.arith == "f64" else "IntArith"
            for cap in t.get("captures", [t]):
                if want in cap["kernel"]:
                    traffic = float(cap["bytes_per_limb"]) * ntt_limbs
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
            "keyswitch_hbm_gbs": (algorithmic_mib(l, C, ctx.alpha, ctx.K) * MiB
                                  / (ms / 1e3) / 1e9),
            "cpu_baseline": cpu,
            "e2e": {"value": world * C / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": ct_bytes, "d2h_bytes_per_step": ct_bytes},
            "gpu_launches": launches,
            "clocks": clk,
        }
        return line
    return None




def mac_compute_roofline(kernel: str, macs: int, ms: float, peak: float) -> dict:
    """The MAC launch against the register-only rate of its own inner step:
    byte multiply-adds (64 per 64-bit product) against b2f_mma_u8_peak for
    the tensor-core kernel, 128-bit multiply-adds against b2f_mac_peak for the
    CUDA-core kernel."""

    if kernel == "mac_mma_kernel":
        achieved = 64 * macs / (ms / 1e3)
        return {"bound": "tensor (mma.sync m16n8k32 u8)", "kernel": kernel,
                "achieved": achieved, "peak": peak, "unit": "u8 multiply-adds/s",
                "frac": achieved / peak,
                "peak_source": "measured live: b2f_mma_u8_peak (32 independent u8 tiles "
                               "per warp from registers, every SM full)"}
    achieved = macs / (ms / 1e3)
    return {"bound": "imad", "kernel": kernel, "achieved": achieved, "peak": peak,
            "unit": "128-bit multiply-adds/s", "frac": achieved / peak,
            "peak_source": "measured live: b2f_mac_peak (mac_kernel's inner step from "
                           "registers, every SM full)"}


def run_mac(a, dev, rank: int, world: int, barrier, max_over_ranks) -> dict | None:
    """mac_kernel alone at the production chunk shape: 8 giants x 64 babies at
    l = 13 over `a.batch` ciphertexts, uniform residues of the layer's primes
    (the kernel is data-independent): one step = one chunk's launch.  For
    kernel profiling and the MAC's two rooflines."""

    import torch

    from easyfhe import _native, core

    params = core.Params.from_depth(37, 16, 5, 59, 60)
    ctx = core.NativeContext(params, dev)
    ctx.set_mac_path(a.mac_path)
    l, B, G, C = LINEAR_LEVEL, LINEAR_B, LINEAR_ROWS // LINEAR_B, a.batch
    gen = torch.Generator(device=dev)
    gen.manual_seed(7 + rank)
    babies = torch.empty(C * B, 2, l, N, dtype=torch.int64, device=dev)
    pts = torch.empty(G * B, l, N, dtype=torch.int64, device=dev)
    for i, q in enumerate(params.q[:l]):
        babies[:, :, i].random_(0, q, generator=gen)
        pts[:, i].random_(0, q, generator=gen)
    stream = torch.cuda.current_stream()
    for _ in range(a.warmup):
        ctx.mac(babies, B, pts, G, l, num_cts=C)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    n0 = _native.lib.b2f_launch_count()
    e0.record(stream)
    for _ in range(a.steps):
        ctx.mac(babies, B, pts, G, l, num_cts=C)
    e1.record(stream)
    torch.cuda.synchronize()
    launches = (_native.lib.b2f_launch_count() - n0) // a.steps
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    kernel = ctx.mac_kernel(B, l, num_cts=C, giant_count=G)
    peak = ctx.mma_u8_peak() if kernel == "mac_mma_kernel" else ctx.mac_peak()
    if rank:
        return None
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    alg = (G * B * l + C * B * 2 * l + C * G * 2 * l) * N * 8
    macs = G * B * C * 2 * l * N
    traffic = None
    tpath = ROOT / "profiles" / f"{kernel}_traffic.json"
    if tpath.exists():
        t = json.loads(tpath.read_text())
        traffic = float(t["bytes_fixed"]) + float(t["bytes_per_ct"]) * C
    return {"metric": "MAC launches/s (one BSGS chunk: 8 giants x 64 babies, l=13)",
            "value": world / (ms / 1e3), "unit": "launches/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u64", "data": "synthetic",
            "config": {"workload": f"{kernel}, {C} ciphertexts x 64 babies x 8 giants, l={l}",
                       "l2": "plaintext rows 3.3 GB: larger than L2; no flush"},
            "roofline": {"bound": "hbm", "kernel": kernel,
                         "achieved": alg / (ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": alg / (ms / 1e3) / 1e9 / hbm, "traffic": traffic,
                         "algorithmic_bytes_per_launch": alg},
            "compute_roofline": mac_compute_roofline(kernel, macs, ms, peak),
            "gpu_launches": launches}


def layer0_result(warmup: int = 1, repetitions: int = 1, extra_args=()) -> dict:
    """Layer-0 of encrypted Llama-3-8B through the reference's own llama3fhe
    (its runner's Layer-0 preset, unchanged) on this backend: s/layer from the
    runner's timed repetition, and the decrypted output against the fp64
    layer."""

    import llama3_layer

    from easyfhe import _native

    if llama3_layer.reference_root() is None:
        return {"unavailable": "the reference llama3fhe tree is not installed (baseline/_ref)"}
    n0 = _native.lib.b2f_launch_count()
    r = llama3_layer.run_layer0(warmup=warmup, repetitions=repetitions,
                                extra_args=extra_args)
    launches = _native.lib.b2f_launch_count() - n0
    perf = r["payload"]["performance"]
    return {
        "s_per_layer": r["s_per_layer"],
        "stage_seconds": perf["median_stage_seconds"],
        "context_keygen_seconds": perf["context_keygen_seconds"],
        "input_pack_encrypt_seconds": perf["input_pack_encrypt_seconds"],
        "bootstrap_prepare_seconds": perf["application_bootstrap_prepare_seconds"],
        "final_decrypt_seconds": perf["final_decrypt_seconds"],
        "warmup": warmup, "repetitions": repetitions,
        "cuda_allocator_peak_bytes": perf["cuda_allocator_peak_bytes"],
        "vs_fp64_exact": r["checks"]["vs_fp64_exact"],
        "vs_fp64_poly": r["checks"]["vs_fp64_poly"],
        "native_bootstrap_calls": r["payload"]["runtime"]["native_bootstrap_calls"],
        "linear_chunks_packed_by_cuda": r["pack_stats"],
        "gpu_launches_total": launches,
        "source": ("llama3fhe.application.runner.run, Layer-0 synthetic preset "
                   "(seed 26081461), unchanged, on this backend"),
        "runner_extra_args": list(extra_args),
    }


def single_gpu_extras(a, dev, barrier, max_over_ranks) -> dict:
    """At N = 1 the default line also carries the HRotate microbench (with the
    NTT roofline), the Layer-0 s/layer of the reference's own graph, and the
    CPU oracle's linear-block rate."""

    import copy
    import gc

    import torch

    out = {}
    h = copy.copy(a)
    h.workload, h.batch = "hrotate", 32
    try:
        line = run_hrotate(h, dev, 0, 1, barrier, max_over_ranks, with_cpu=False)
        out["hrotate"] = {k: line[k] for k in ("metric", "value", "unit", "ms_per_step",
                                               "config", "roofline", "compute_roofline",
                                               "keyswitch_hbm_gbs", "e2e", "gpu_launches")}
    except Exception as exc:  # reported, never fatal to the headline
        out["hrotate"] = {"error": repr(exc)}
    gc.collect()
    torch.cuda.empty_cache()
    # the same at the layer's parameters (integer arithmetic: 59/60-bit primes)
    out["hrotate_layer_params"] = []
    for limbs in (13, 38):
        h = copy.copy(a)
        h.workload, h.batch, h.limbs, h.layer_params = "hrotate", 16, limbs, True
        h.steps, h.warmup = min(a.steps, 20), min(a.warmup, 3)
        try:
            line = run_hrotate(h, dev, 0, 1, barrier, max_over_ranks, with_cpu=False)
            out["hrotate_layer_params"].append(
                {k: line[k] for k in ("value", "unit", "ms_per_step", "config", "roofline",
                                      "compute_roofline", "keyswitch_hbm_gbs", "arith",
                                      "gpu_launches")})
        except Exception as exc:
            out["hrotate_layer_params"].append({"limbs": limbs, "error": repr(exc)})
        gc.collect()
        torch.cuda.empty_cache()
    if not a.no_layer:
        try:
            out["layer0"] = layer0_result()
        except Exception as exc:
            out["layer0"] = {"error": repr(exc)}
        gc.collect()
        torch.cuda.empty_cache()
    try:
        cpu = linear_cpu_rate()
        out["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
    except Exception as exc:  # the oracle is a reported baseline only
        out["cpu_baseline"] = {"value": None, "unit": "ciphertexts/s", "cores": 0,
                               "kind": "port", "sample": f"unavailable: {exc}"}
    return out


def run_prefill(a, world: int) -> dict:
    """An encrypted prefill of --num-layers decoder layers through the
    reference's own model loop (Llama3Model.forward) on one GPU, seeded
    synthetic layers kept inside the reference's per-layer polynomial fits."""

    import llama3_layer

    from easyfhe import _native

    if llama3_layer.reference_root() is None:
        return {"metric": "encrypted Llama-3-8B prefill s/layer at seq128",
                "unavailable": "the reference llama3fhe tree is not installed (baseline/_ref)"}
    n0 = _native.lib.b2f_launch_count()
    r = llama3_layer.run_prefill(a.num_layers, check=not a.no_check)
    launches = _native.lib.b2f_launch_count() - n0
    r.pop("decoded", None)
    steady = r["per_layer_seconds"][1:] or r["per_layer_seconds"]
    return {"metric": f"encrypted Llama-3-8B prefill s/layer at seq128 ({a.num_layers} layers)",
            "value": r["s_per_layer"], "unit": "s/layer", "n_gpus": 1, "steps": 1,
            "warmup": 0, "ms_per_step": r["wall_seconds"] * 1e3,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "u64", "data": "synthetic",
            "config": {"workload": (f"{a.num_layers} Llama-3-8B decoder layers, seq 128, through "
                                    "the reference's Llama3Model.forward; seeded synthetic "
                                    "layers; logN 16 depth 37 dnum 5 59/60-bit primes")},
            "prefill_seconds": r["wall_seconds"],
            "steady_state_s_per_layer": sum(steady) / len(steady),
            "prefill": r, "gpu_launches_total": launches}


def run_mlp(a, dev, rank: int, world: int, barrier, max_over_ranks) -> dict | None:
    """The reference's own feature-major SwiGLU MLP block on this backend,
    sharded by token-shard ciphertext: ``mlp_fhe``
    (llama3fhe/operators/linear/mlp.py:524-1126: gate/up 4096 -> 14336 in
    four feature pages sharing one set of baby rotations, SiLU by the
    reference's Chebyshev PS evaluator, down 14336 -> 4096 over the four
    pages) with its production schedule, on a layout of 128/N tokens per rank
    (feature-major, 8 tokens per ciphertext: 16/N ciphertexts), then the
    outputs are all-gathered over NCCL inside the step.  Inputs: the Layer-0
    preset's weights and N(0, 1) activations encrypted at the MLP's entry
    level (11 limbs); the first step's outputs are decrypted against the
    reference's own NumPy MLP (mlp_packed_numpy) through its verify path."""

    import numpy as np
    import torch
    import torch.distributed as dist

    import llama3_layer

    from easyfhe import _native

    if llama3_layer.reference_root() is None:
        return ({"metric": "encrypted MLP block ciphertexts/s", "impl": "b200",
                 "unavailable": "the reference llama3fhe tree is not installed (baseline/_ref)"}
                if rank == 0 else None)
    llama3_layer.import_reference()
    from llama3fhe.application import session
    from llama3fhe.layouts import FeatureMajorPrefillLayout
    from llama3fhe.operators.linear.mlp import mlp_fhe

    total = a.batch
    if total % world or (total // world) % 2:
        raise SystemExit(f"{total} ciphertexts do not split over {world} ranks in pairs")
    per = total // world
    full = FeatureMajorPrefillLayout()
    tokens = per * full.tokens_per_cipher
    layout = FeatureMajorPrefillLayout(seq_len=tokens)
    s = llama3_layer.ReferenceSession()
    _, w, approx = llama3_layer.synthetic_layer()
    x = np.random.default_rng(6).normal(size=(total * full.tokens_per_cipher,
                                              full.hidden_dim)).astype(np.float32)
    x_r = x[rank * tokens:(rank + 1) * tokens]
    level = 11  # the MLP's entry level at Layer 0 (graph.py:1252-1259)
    cts = session._encrypt_hidden(x_r, context=s.context, layout=layout,
                                  input_level=int(s.context.context.L) - level)
    stream = torch.cuda.current_stream()
    gathered = None
    gather_ev = []
    info = {}

    def step(verify=False, record=False):
        nonlocal gathered
        r = mlp_fhe(x_r, w.gate_proj, w.up_proj, w.down_proj, silu_entry=approx.silu,
                    layout=layout, config=s.config, crypto_context=s.context,
                    input_ciphers=cts, verify=verify)
        out = torch.stack([c.data for c in r.ciphers])
        info["stages"] = r.stage_seconds
        if verify:
            info["check"] = {"max_abs": r.max_abs_diff, "mean_abs": r.mean_abs_diff,
                             "ref_max_abs": float(np.max(np.abs(r.expected)))}
        if world > 1:  # the stage-boundary exchange: every rank gets every output
            if gathered is None:
                gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype,
                                       device=out.device)
            if record:
                e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                e[0].record(stream)
            dist.all_gather_into_tensor(gathered, out.contiguous())
            if record:
                e[1].record(stream)
                gather_ev.append(e)
        return out

    step(verify=True)  # warm-up 1: keys generated on first use, outputs checked
    for _ in range(max(0, a.warmup - 1)):
        step()
    torch.cuda.synchronize()
    clocks = Clocks(dev.index or 0, not a.no_clocks)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    n0 = _native.lib.b2f_launch_count()
    e0.record(stream)
    for _ in range(a.steps):
        step(record=True)
    e1.record(stream)
    torch.cuda.synchronize()
    launches = (_native.lib.b2f_launch_count() - n0) // a.steps
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    gather_ms = max_over_ranks(sum(x.elapsed_time(y) for x, y in gather_ev) / a.steps
                               if gather_ev else 0.0)
    if rank != 0:
        return None
    return {
        "metric": ("encrypted MLP block ciphertexts/s (the reference's feature-major SwiGLU "
                   "mlp_fhe: gate/up 4096->14336, SiLU, down 14336->4096)"),
        "value": total / (ms / 1e3), "unit": "ciphertexts/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u64", "data": "synthetic",
        "config": {"workload": (f"llama3fhe mlp_fhe, unchanged, production schedule; "
                                f"{total} token-shard ciphertexts (8 tokens each) sharded "
                                f"{per}/rank, entry level {level} limbs, outputs all-gathered "
                                "over NCCL in every step; Layer-0 preset weights; logN 16 "
                                "depth 37 dnum 5 59/60-bit primes"),
                   "ciphertexts_total": total, "ciphertexts_per_rank": per,
                   "parallelism": f"token-shard sharding x{world} + all-gather",
                   "l2": "plaintexts of 512 rows per chunk (GBs): larger than L2; no flush"},
        "stage_seconds_rank0": info.get("stages"),
        "check_rank0": info.get("check"),
        "gather_ms_per_step": gather_ms,
        "gather_share": gather_ms / ms if ms else None,
        "gpu_launches": launches,
        "clocks": clk,
    }


def run_layer0(a, world: int) -> dict:
    """The Layer-0 workload as its own line: seconds per encrypted layer."""

    extra = (() if a.hoist_strategy == "normal"
             else ("--linear-hoist-strategy", a.hoist_strategy))
    r = layer0_result(warmup=max(1, min(a.warmup, 2)), repetitions=max(1, min(a.steps, 3)),
                      extra_args=extra)
    if "s_per_layer" not in r:
        return {"metric": "encrypted Llama-3-8B prefill s/layer at seq128", **r}
    return {"metric": "encrypted Llama-3-8B prefill s/layer at seq128 (Layer-0 preset)",
            "value": r["s_per_layer"], "unit": "s/layer", "n_gpus": 1,
            "steps": max(1, min(a.steps, 3)), "warmup": max(1, min(a.warmup, 2)),
            "ms_per_step": r["s_per_layer"] * 1e3, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": {"workload": ("one Llama-3-8B decoder layer, seq 128, hidden 4096, "
                                    "32/8 heads, SwiGLU 14336; logN 16 depth 37 dnum 5 "
                                    "59/60-bit primes; the reference's graph"),
                       "hoist_strategy": a.hoist_strategy},
            "layer0": r}


def main() -> None:
    a = parse()
    if a.impl == "reference":
        run_reference(a)
        return

    import torch
    import torch.distributed as dist

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

    try:
        if a.workload == "bootstrap":
            run_bootstrap(a, dev, rank, world, barrier, max_over_ranks)
        elif a.workload == "prefill":
            line = run_prefill(a, world) if rank == 0 else None
            if line:
                print(json.dumps(line), flush=True)
        elif a.workload == "layer0":
            line = run_layer0(a, world) if rank == 0 else None
            if line:
                print(json.dumps(line), flush=True)
        elif a.workload == "mlp":
            line = run_mlp(a, dev, rank, world, barrier, max_over_ranks)
            if line:
                print(json.dumps(line), flush=True)
        elif a.workload == "mac":
            line = run_mac(a, dev, rank, world, barrier, max_over_ranks)
            if line:
                print(json.dumps(line), flush=True)
        elif a.workload in ("hrotate", "ntt"):
            line = run_hrotate(a, dev, rank, world, barrier, max_over_ranks)
            if line:
                print(json.dumps(line), flush=True)
        else:
            line = run_linear(a, dev, rank, world, barrier, max_over_ranks)
            if rank == 0 and world == 1 and not a.no_extras:
                line.update(single_gpu_extras(a, dev, barrier, max_over_ranks))
            if line:
                print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
