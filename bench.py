"""Benchmark: batched n=4 Birkhoff projection, forward + backward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one rank per GPU)

One step is one pass of the hot path over one batch: the Newton forward
(mhc_proj.torch.birkhoff_proj_n4, tol 1e-6) then the implicit-function-theorem
backward (mhc_proj.torch.birkhoff_proj_n4_backward) on 2^24 matrices per GPU
with logits x ~ N(0,1) and upstream gradient G ~ N(0,1) (seeded synthetic
inputs of the workload's shape and distribution).  The batch is sharded
across GPUs with no collective on the data path, so per-GPU work is fixed as
N grows (weak scaling); the value is the whole job's matrices per second over
the slowest rank's device time.

Printed (rank 0): one JSON line with the metric, the roofline of the dominant
kernel, the end-to-end number through the public API with host buffers, the
CPU baseline (the oracle's C port on the host's cores) and the SM clocks seen
during the timed region.

`--impl reference` times the reference algorithm on the host CPU instead (the
reference's only CPU implementation of this path is its algorithm itself; the
C port in oracle/ runs it on every host thread) and prints the same line with
"impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "mhc-proj_b200")]

METRIC = "fwd+bwd matrices/s and % HBM roofline at N=2^24 fp32, 1/2/4/8 B200"
UNIT = "matrices/s"
BYTES_FWD = 128      # R in (64 B) + T out (64 B) per matrix
BYTES_BWD = 192      # G, T in + D out per matrix
BYTES_HRES_FWD = 132  # h (64 B of a 96 B row) + rms in, T out
BYTES_HRES_BWD = 264  # G, T, h, rms in; dh, drms out
BYTES_SKHRES_BWD = 200  # G, h, rms in; dh, drms out (M is recomputed from h)
FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 7700.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["newton", "sinkhorn", "hres", "sk_hres"], default="newton",
                    help="newton: the Newton forward + IFT backward (default, the headline metric); "
                         "sinkhorn: the fused exp + Sinkhorn-Knopp pair, 20 iterations; "
                         "hres: the projection fused with the mHC layer's H_res producer, forward + backward; "
                         "sk_hres: the Sinkhorn-Knopp pair (20 iterations) fused with that producer")
    ap.add_argument("--n", type=int, default=None, help="matrices per GPU (default 2^24, or 2^22 for sinkhorn)")
    ap.add_argument("--dist", default="normal", choices=["normal", "sigma_mix", "mixture", "wide"])
    ap.add_argument("--tol", type=float, default=1e-6)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--e2e-chunks", type=int, default=16, help="pieces of the e2e step's batch (pipelined copies)")
    ap.add_argument("--e2e-streams", type=int, default=3, help="streams the e2e pieces rotate over")
    ap.add_argument("--mixture-total", type=int, default=1 << 26,
                    help="matrices of the sharded mixture measurement (total over all ranks; 0 skips it)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return world, rank, local


def measured_peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_counts(kernel="forward"):
    """Per-matrix DRAM bytes, warp instructions and MUFU operations of a
    kernel ("forward", "sk_backward", ...) from the committed ncu summary
    (profiles/roofline_traffic.json), or Nones."""
    p = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)[kernel]
        return (float(d["dram_bytes_per_matrix"]), float(d.get("warp_instructions_per_matrix", "nan")),
                float(d.get("mufu_thread_ops_per_matrix", "nan")))
    except Exception:
        return None, None, None


def sm_count(dev):
    import torch

    return torch.cuda.get_device_properties(dev).multi_processor_count


def workload_config(args, world):
    if args.workload == "sinkhorn":
        what = "fused exp + Sinkhorn-Knopp n4 (20 iterations) forward + backward"
    elif args.workload == "sk_hres":
        what = ("H_res producer (exp(alpha*h/rms+b), h = columns 8..23 of an [N,24] projection) fused with "
                "Sinkhorn-Knopp n4 (20 iterations) forward + fused backward incl. dalpha, db batch sums")
    elif args.workload == "hres":
        what = (f"H_res producer (alpha*h/rms+b, h = columns 8..23 of an [N,24] projection) fused with the Newton "
                f"forward (tol {args.tol:g}) + fused backward incl. dalpha, db batch sums")
    else:
        what = f"Newton forward (tol {args.tol:g}) + IFT backward"
    return {
        "workload": f"{what}, N=2^{args.n.bit_length() - 1} fp32 4x4 per GPU, x~{args.dist}, G~N(0,1)",
        "n_per_gpu": args.n,
        "global_batch": args.n * world,
        "tol": args.tol,
        "distribution": args.dist,
        "seed": 0,
        "parallelism": f"dp{world} (batch-sharded, no collective)",
        "l2": "inputs larger than L2 (1 GiB per tensor vs 126 MB); no flush needed",
    }


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        if not getattr(self, "lines", None):
            return None
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        top = max(sm)
        loaded = [v for v in sm if v >= 0.5 * top] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# CPU baselines (the oracle's C port; vanilla PyTorch Sinkhorn)
# ---------------------------------------------------------------------------
def cpu_port_rate(seconds: float, chunk: int, dist: str, tol: float, threads: int = 0):
    """Newton fwd + IFT bwd with the C port of the reference algorithm on
    `threads` host threads (0 = all), on chunks of synthetic inputs until
    `seconds` have passed.  Returns (matrices/s, threads, matrices done)."""
    import numpy as np

    import oracle

    nt = threads or oracle.max_threads()
    rng = np.random.default_rng(0)
    R = rng.standard_normal((chunk, 4, 4), dtype=np.float32)
    if dist != "normal":
        R *= rng.uniform(0.5, 4.0, size=(chunk, 1, 1)).astype(np.float32)
    G = rng.standard_normal((chunk, 4, 4), dtype=np.float32)
    done, t0 = 0, time.perf_counter()
    while True:
        T = oracle.birkhoff_proj_n4(R, tol, threads=nt)
        oracle.birkhoff_proj_n4_backward(G, T, threads=nt)
        done += chunk
        el = time.perf_counter() - t0
        if el >= seconds:
            return done / el, nt, done


def vanilla_sk_cpu_rate(reps: int = 10):
    """The reference's vanilla PyTorch SK20 (README.md:37-46) forward +
    autograd backward on the host, N = 4096: all threads, and one thread."""
    import torch

    import oracle

    g = torch.Generator().manual_seed(123)
    x = torch.randn(4096, 4, 4, generator=g)
    G = torch.randn(4096, 4, 4, generator=g)
    prev = torch.get_num_threads()

    def rate(threads):
        torch.set_num_threads(threads)
        oracle.vanilla_sinkhorn(x, G)
        t0 = time.perf_counter()
        for _ in range(reps):
            oracle.vanilla_sinkhorn(x, G)
        return 4096 / ((time.perf_counter() - t0) / reps)

    all_threads = os.cpu_count() or 1
    v_all = rate(all_threads)
    v_one = rate(1)
    torch.set_num_threads(prev)
    return {"value": v_all, "unit": UNIT, "cores": all_threads, "one_thread": v_one,
            "sample": "vanilla PyTorch SK20 (eps 1e-6) fwd + autograd bwd, N=4096 x~N(0,1) seed 123, eager"}


# ---------------------------------------------------------------------------
# reference arm: the algorithm on the host CPU
# ---------------------------------------------------------------------------
def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    import numpy as np

    import oracle

    nt = oracle.max_threads()
    chunk = 1 << 18
    pool = 8  # chunks cycled through: 256 MiB of R and G, beyond the host's caches
    rng = np.random.default_rng(0)
    Rs = [rng.standard_normal((chunk, 4, 4), dtype=np.float32) for _ in range(pool)]
    Gs = [rng.standard_normal((chunk, 4, 4), dtype=np.float32) for _ in range(pool)]
    count = [0]

    def step():
        i = count[0] % pool
        count[0] += 1
        T = oracle.birkhoff_proj_n4(Rs[i], args.tol, threads=nt)
        oracle.birkhoff_proj_n4_backward(Gs[i], T, threads=nt)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = chunk * args.steps / el
    sample = (f"{chunk} matrices per step (x~N(0,1), G~N(0,1)) of the N=2^24 workload, cycling through {pool} "
              f"such chunks (256 MiB of inputs): Newton fwd + IFT bwd, C port of the reference algorithm, "
              f"{nt} pthreads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nt, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)

    import mhc_proj  # fails loudly without the native extension

    from mhc_proj.workloads import make_logits

    n = args.n
    R = make_logits(args.dist, n, seed=1000 + rank, device=dev)
    G = make_logits("normal", n, seed=2000 + rank, device=dev)
    tol = args.tol
    hres = None
    if args.workload == "sinkhorn":
        fwd = lambda: mhc_proj.torch.sinkhorn_knopp_n4_logits(R, 20)["T"]  # noqa: E731
        bwd = lambda T: mhc_proj.torch.sinkhorn_knopp_n4_logits_backward(G, R, 20)["D"]  # noqa: E731
    elif args.workload == "sk_hres":
        hres = hres_inputs(R, rank, dev)
        h, rms, a, b = hres
        fwd = lambda: mhc_proj.torch.sinkhorn_knopp_n4_hres(h, rms, a, b, 20)["T"]  # noqa: E731
        bwd = lambda T: mhc_proj.torch.sinkhorn_knopp_n4_hres_backward(G, h, rms, a, b, 20)  # noqa: E731
    elif args.workload == "hres":
        hres = hres_inputs(R, rank, dev)
        h, rms, a, b = hres
        fwd = lambda: mhc_proj.torch.birkhoff_proj_n4_hres(h, rms, a, b, tol)["T"]  # noqa: E731
        bwd = lambda T: mhc_proj.torch.birkhoff_proj_n4_hres_backward(G, T, h, rms, a, b_res=b)  # noqa: E731
    else:
        fwd = lambda: mhc_proj.torch.birkhoff_proj_n4(R, tol)["T"]  # noqa: E731
        bwd = lambda T: mhc_proj.torch.birkhoff_proj_n4_backward(G, T)["D"]  # noqa: E731

    def step(ev=None):
        if ev is not None:
            ev[0].record()
        T = fwd()
        if ev is not None:
            ev[1].record()
        D = bwd(T)
        if ev is not None:
            ev[2].record()
        return T, D

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(dev.index) as clk:
        barrier()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record()
        for i in range(args.steps):
            step(evs[i])
        t_end.record()
        barrier()
    total_ms = t_start.elapsed_time(t_end)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps

    # end to end through the public API with host buffers: pinned inputs go
    # up, T and D come back, chunks pipelined over two streams
    e2e = run_e2e(args, R, G, dev, world) if args.workload == "newton" else {"ms": float("nan"), "h2d": 0, "d2h": 0, "how": "not measured for this workload"}
    ceiling_ms = e2e.get("ceiling_ms", float("nan"))
    passes = forward_passes(R, tol) if args.workload == "newton" and rank == 0 else None
    bwd_cold_ms = backward_cold_l2_ms(bwd, fwd, dev) if args.workload == "newton" else float("nan")
    unfused_ms = sinkhorn_unfused_ms(R, G, args.steps) if args.workload == "sinkhorn" else None
    hw_rcp_fwd_ms = sinkhorn_hw_reciprocal_fwd_ms(R, args.steps) if args.workload == "sinkhorn" else None
    if args.workload == "hres":
        unfused_ms, plain_fwd_ms = hres_unfused_ms(hres, G, tol, args.steps)
    if args.workload == "sk_hres":
        unfused_ms = sk_hres_unfused_ms(hres, G, args.steps)

    stats = torch.tensor([total_ms, fwd_ms, bwd_ms, e2e["ms"], ceiling_ms, bwd_cold_ms], device=dev,
                         dtype=torch.float64)
    per_rank = [stats.clone()]
    if world > 1:
        per_rank = [torch.empty_like(stats) for _ in range(world)]
        dist.all_gather(per_rank, stats)
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    total_ms, fwd_ms, bwd_ms, e2e_ms, ceiling_ms, bwd_cold_ms = stats.tolist()
    ms_per_step = total_ms / args.steps
    del R, G
    mixture = None
    if args.workload == "newton" and args.mixture_total > 0:
        torch.cuda.empty_cache()
        mixture = sharded_mixture(args, dev, world, rank)

    if rank == 0:
        peak, peak_kind = measured_peak_hbm()
        fwd_gbs = BYTES_FWD * n / (fwd_ms * 1e-3) / 1e9
        bwd_gbs = BYTES_BWD * n / (bwd_ms * 1e-3) / 1e9
        step_gbs = (BYTES_FWD + BYTES_BWD) * n / (ms_per_step * 1e-3) / 1e9
        tpm, wipm, mufupm = ncu_counts()
        sms = sm_count(dev)
        clocks = clk.summary()
        mhz = clocks["sm_mhz"] if clocks else 1965.0
        rate_fwd = n / (fwd_ms * 1e-3)  # matrices/s through the forward kernel
        compute = None
        if wipm == wipm and mufupm == mufupm:  # not NaN
            issue_peak = sms * 4 * mhz * 1e6          # warp instructions/s: one per SM sub-partition per clock
            mufu_peak = sms * 16 * mhz * 1e6          # MUFU results/s: 16 per SM per clock
            compute = {"bound": "issue", "unit": "warp instructions/s",
                       "achieved": rate_fwd * wipm, "peak": issue_peak, "frac": rate_fwd * wipm / issue_peak,
                       "mufu_frac": rate_fwd * mufupm / mufu_peak,
                       "per_matrix": {"warp_instructions": wipm, "mufu_ops": mufupm},
                       "source": "per-matrix counts from ncu (profiles/roofline_traffic.json) x live forward rate; "
                                 "peaks from the SM count and the median SM clock seen"}
        line = {
            "metric": METRIC,
            "value": world * n / (ms_per_step * 1e-3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded torch generators; workload shape and distribution)",
            "config": workload_config(args, world),
            "roofline": {
                "bound": "hbm",
                "kernel": "sk_fwd_kernel (fused exp + Sinkhorn-Knopp)" if args.workload == "sinkhorn"
                          else "birkhoff_fwd_kernel (Newton forward)",
                "achieved": fwd_gbs, "peak": peak, "unit": "GB/s", "frac": fwd_gbs / peak,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "algorithmic_bytes_per_matrix": BYTES_FWD,
                "traffic": None if tpm is None else tpm * n,
                "step": {"achieved": step_gbs, "frac": step_gbs / peak,
                         "algorithmic_bytes_per_matrix": BYTES_FWD + BYTES_BWD},
                "kernels": {"forward_ms": fwd_ms, "backward_ms": bwd_ms,
                            "forward_gbs": fwd_gbs, "backward_gbs": bwd_gbs,
                            "backward_frac": bwd_gbs / peak,
                            "backward_ms_l2_flushed": bwd_cold_ms,
                            "backward_frac_l2_flushed": BYTES_BWD * n / (bwd_cold_ms * 1e-3) / 1e9 / peak,
                            "backward_note": "in the step the backward reads T right after the forward wrote it, "
                                             "so up to L2's 126 MB of T can be L2 hits; *_l2_flushed times it "
                                             "after a 512 MiB write evicts L2. Its reads:writes are 2:1, against "
                                             "the 1:1 of the copy that measured the peak"},
                "compute": compute,
            },
            "e2e": {"value": world * n / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                    "ms_per_step": e2e_ms, "how": e2e["how"],
                    "copy_ceiling": {"value": world * n / (ceiling_ms * 1e-3), "unit": UNIT,
                                     "ms_per_step": ceiling_ms,
                                     "host_link_gbs_per_gpu": (e2e["h2d"] + e2e["d2h"]) / (ceiling_ms * 1e-3) / 1e9,
                                     "how": "the same pinned host<->device copies (same chunks and streams) on every "
                                            "rank at once with no kernels: what the host links can move"},
                    "frac_of_copy_ceiling": ceiling_ms / e2e_ms},
            "gpu_launches": 2 * args.steps,
            "clocks": clocks,
            "per_rank": [{"rank": i, "ms_per_step": t[0] / args.steps, "forward_ms": t[1], "backward_ms": t[2]}
                         for i, t in enumerate(x.tolist() for x in per_rank)],
        }
        if args.workload == "sinkhorn":
            # the backward is the dominant kernel of this step
            line["metric"] = "Sinkhorn-Knopp n4 (20 iterations) fwd+bwd matrices/s"
            btpm, bwipm, _ = ncu_counts("sk_backward")
            rate_bwd = n / (bwd_ms * 1e-3)
            line["roofline"].update({
                "kernel": "sk_bwd_kernel (fused exp; exact VJP from the forward's potentials)",
                "achieved": bwd_gbs, "frac": bwd_gbs / peak, "algorithmic_bytes_per_matrix": BYTES_BWD,
                "traffic": None if btpm is None else btpm * n,
                "compute": None if bwipm is None or bwipm != bwipm else {
                    "bound": "issue", "unit": "warp instructions/s", "achieved": rate_bwd * bwipm,
                    "peak": sms * 4 * mhz * 1e6, "frac": rate_bwd * bwipm / (sms * 4 * mhz * 1e6),
                    "per_matrix": {"warp_instructions": bwipm},
                    "source": "per-matrix count from ncu (profiles/roofline_traffic.json sk_backward) x live "
                              "backward rate; peak from the SM count and the median SM clock seen"}})
            line["e2e"] = None
            line["forward_hw_reciprocal"] = {
                "forward_ms": hw_rcp_fwd_ms, "step_ms": hw_rcp_fwd_ms + bwd_ms,
                "value": n / ((hw_rcp_fwd_ms + bwd_ms) * 1e-3),
                "how": "the opt-in forward with the hardware reciprocal (MHC_SK_HW_RECIPROCAL; within 1e-6 of "
                       "the default forward's bits) with the same backward"}
            line["unfused_reference_composition"] = {
                "ms_per_step": unfused_ms, "value": n / (unfused_ms * 1e-3),
                "how": "torch.exp, sinkhorn_knopp_n4, sinkhorn_knopp_n4_backward, product with exp(R) "
                       "(the reference MHCSinkhornN4 composition) on this repository's kernels"}
        if args.workload == "hres":
            fwd_gbs = BYTES_HRES_FWD * n / (fwd_ms * 1e-3) / 1e9
            bwd_gbs = BYTES_HRES_BWD * n / (bwd_ms * 1e-3) / 1e9
            step_gbs = (BYTES_HRES_FWD + BYTES_HRES_BWD) * n / (ms_per_step * 1e-3) / 1e9
            line["metric"] = "H_res producer + Newton projection fwd+bwd matrices/s"
            line["roofline"].update({
                "kernel": "birkhoff_fwd_kernel<HResSource> (producer fused into the Newton forward)",
                "achieved": fwd_gbs, "frac": fwd_gbs / peak, "algorithmic_bytes_per_matrix": BYTES_HRES_FWD,
                "traffic": None,
                "step": {"achieved": step_gbs, "frac": step_gbs / peak,
                         "algorithmic_bytes_per_matrix": BYTES_HRES_FWD + BYTES_HRES_BWD},
                "kernels": {"forward_ms": fwd_ms, "backward_ms": bwd_ms, "forward_gbs": fwd_gbs,
                            "backward_gbs": bwd_gbs, "backward_frac": bwd_gbs / peak,
                            "backward_kernels": "birkhoff_hres_bwd_kernel + partial_sums_fold_kernel"}})
            line["roofline"]["compute"] = None
            line["e2e"] = None
            line["gpu_launches"] = 3 * args.steps
            line["unfused_composition"] = {
                "ms_per_step": unfused_ms, "value": n / (unfused_ms * 1e-3),
                "how": "R = alpha*h/rms + b with torch ops, birkhoff_proj_n4, birkhoff_proj_n4_backward, then "
                       "dh, drms, dalpha, db with torch ops (this repository's unfused kernels)",
                "plain_forward_ms": plain_fwd_ms,
                "plain_forward_how": "birkhoff_proj_n4 alone on the same logits materialised in HBM"}
        if args.workload == "sk_hres":
            fwd_gbs = BYTES_HRES_FWD * n / (fwd_ms * 1e-3) / 1e9
            bwd_gbs = BYTES_SKHRES_BWD * n / (bwd_ms * 1e-3) / 1e9
            step_gbs = (BYTES_HRES_FWD + BYTES_SKHRES_BWD) * n / (ms_per_step * 1e-3) / 1e9
            line["metric"] = "H_res producer + Sinkhorn-Knopp n4 (20 iterations) fwd+bwd matrices/s"
            btpm, bwipm, _ = ncu_counts("sk_hres_backward")
            rate_bwd = n / (bwd_ms * 1e-3)
            line["roofline"].update({
                "kernel": "sk_hres_bwd_kernel (the dominant kernel: the producer's chain rule fused into the "
                          "Sinkhorn-Knopp backward)",
                "achieved": bwd_gbs, "frac": bwd_gbs / peak, "algorithmic_bytes_per_matrix": BYTES_SKHRES_BWD,
                "traffic": None if btpm is None else btpm * n,
                "compute": None if bwipm is None or bwipm != bwipm else {
                    "bound": "issue", "unit": "warp instructions/s", "achieved": rate_bwd * bwipm,
                    "peak": sms * 4 * mhz * 1e6, "frac": rate_bwd * bwipm / (sms * 4 * mhz * 1e6),
                    "per_matrix": {"warp_instructions": bwipm},
                    "source": "per-matrix count from ncu (profiles/roofline_traffic.json sk_hres_backward) x "
                              "live backward rate; peak from the SM count and the median SM clock seen"},
                "step": {"achieved": step_gbs, "frac": step_gbs / peak,
                         "algorithmic_bytes_per_matrix": BYTES_HRES_FWD + BYTES_SKHRES_BWD},
                "kernels": {"forward_ms": fwd_ms, "backward_ms": bwd_ms, "forward_gbs": fwd_gbs,
                            "backward_gbs": bwd_gbs, "backward_frac": bwd_gbs / peak,
                            "backward_kernels": "sk_hres_bwd_kernel + partial_sums_fold_kernel"}})
            line["e2e"] = None
            line["gpu_launches"] = 3 * args.steps
            line["unfused_composition"] = {
                "ms_per_step": unfused_ms, "value": n / (unfused_ms * 1e-3),
                "how": "H_res = exp(alpha*h/rms + b) with torch ops, sinkhorn_knopp_n4, sinkhorn_knopp_n4_backward, "
                       "then dR = dM*M and dh, drms, dalpha, db with torch ops (this repository's unfused kernels)"}
        if mixture is not None:
            line["multi_gpu_mixture"] = mixture
        if passes is not None:
            line["forward_passes"] = passes
        rf = line["roofline"]
        rf["nominal"] = {"peak": NOMINAL_HBM_GBS, "unit": "GB/s", "frac": rf["achieved"] / NOMINAL_HBM_GBS,
                         "step_frac": rf["step"]["achieved"] / NOMINAL_HBM_GBS,
                         "note": "the same achieved figures against the nominal HGX B200 HBM3e bandwidth"}
        if world == 1 and not args.no_cpu_baseline and args.workload == "newton":
            rate, nt, done = cpu_port_rate(args.cpu_seconds, 1 << 18, args.dist, tol)
            line["cpu_baseline"] = {
                "value": rate, "unit": UNIT, "cores": nt, "kind": "port",
                "sample": f"{done} matrices in chunks of 2^18 (same distribution): Newton fwd + IFT bwd, "
                          f"C port of the reference algorithm in oracle/, {nt} pthreads",
                "vanilla_sk20_torch_cpu": vanilla_sk_cpu_rate(),
            }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
        dist.destroy_process_group()
    return 0


def hres_inputs(R, rank, dev):
    """The mHC layer's producer inputs of the hres workload: H_proj_concat
    [N, 24] with the logits' values in columns 8..23 (the H_res block), rms
    ~ U(0.5, 2), alpha_res = 1 and b_res ~ N(0,1) + 2 I, seeded per rank."""
    import torch

    n = R.shape[0]
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    H = torch.randn(n, 24, device=dev, generator=g)
    H[:, 8:24] = R.reshape(n, 16)
    rms = torch.rand(n, device=dev, generator=g) * 1.5 + 0.5
    b = torch.randn(16, device=dev, generator=g) + 2.0 * torch.eye(4, device=dev).reshape(16)
    a = torch.ones(1, device=dev)
    return H[:, 8:24], rms, a, b


def hres_unfused_ms(hres, G, tol, steps):
    """Device time of the same step as separate kernels: the producer's
    arithmetic and the chain rule as torch ops around the plain projection
    kernels."""
    import torch

    import mhc_proj

    h, rms, a, b = hres
    n = h.shape[0]

    def once():
        R = (a * h / rms[:, None] + b).reshape(n, 4, 4)
        T = mhc_proj.torch.birkhoff_proj_n4(R, tol)["T"]
        D = mhc_proj.torch.birkhoff_proj_n4_backward(G, T)["D"].reshape(n, 16)
        s = a / rms
        dh = D * s[:, None]
        q = (D * h).sum(1)
        drms = -(s / rms) * q
        return dh, drms, (q / rms).sum(), D.sum(0)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    R = (a * h / rms[:, None] + b).reshape(n, 4, 4)
    plain_fwd = timed(lambda: mhc_proj.torch.birkhoff_proj_n4(R, tol))
    return timed(once), plain_fwd


def sk_hres_unfused_ms(hres, G, steps):
    """Device time of the sk_hres step as separate kernels: the producer and
    the chain rule as torch ops around the plain Sinkhorn-Knopp kernels."""
    import torch

    import mhc_proj

    h, rms, a, b = hres
    n = h.shape[0]

    def once():
        M = torch.exp(a * h / rms[:, None] + b).reshape(n, 4, 4)
        mhc_proj.torch.sinkhorn_knopp_n4(M, 20)
        dR = (mhc_proj.torch.sinkhorn_knopp_n4_backward(G, M, 20)["D"] * M).reshape(n, 16)
        s = a / rms
        q = (dR * h).sum(1)
        return dR * s[:, None], -(s / rms) * q, (q / rms).sum(), dR.sum(0)

    for _ in range(3):
        once()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        once()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def sinkhorn_hw_reciprocal_fwd_ms(R, steps):
    """Device time of the fused Sinkhorn-Knopp forward with the hardware
    reciprocal (the opt-in MHC_SK_HW_RECIPROCAL)."""
    import torch

    import mhc_proj

    def once():
        return mhc_proj.torch.sinkhorn_knopp_n4_logits(R, 20, approx_reciprocal=True)["T"]

    for _ in range(3):
        once()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        once()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def sinkhorn_unfused_ms(R, G, steps):
    """Device time of the reference's MHCSinkhornN4 composition (module.py:46-72)
    on this repository's unfused kernels: exp, SK forward, SK backward, product."""
    import torch

    import mhc_proj

    def once():
        M = torch.exp(R)
        mhc_proj.torch.sinkhorn_knopp_n4(M, 20)
        return mhc_proj.torch.sinkhorn_knopp_n4_backward(G, M, 20)["D"] * M

    for _ in range(3):
        once()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        once()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def forward_passes(R, tol):
    """Where the forward's log-sum-exp passes go on this batch (an untimed run
    of the counting instantiation), per matrix."""
    from mhc_proj import capi

    _, _, _, c = capi.birkhoff_proj_n4_pass_counts_tensor(R, tol)
    m = c["matrices"]
    per = {k: v / m for k, v in c.items() if k not in ("matrices", "lane_slots", "busy_lane_slots")}
    state = c["busy_lane_slots"] / m
    return {"per_matrix": per, "state_machine_passes_per_matrix": state,
            "passes_per_matrix": state + per["fill"],
            "lane_utilisation": c["busy_lane_slots"] / c["lane_slots"],
            "how": "mhc_birkhoff_proj_n4_pass_counts on the timed batch, outside the timed region"}


def backward_cold_l2_ms(bwd, fwd, dev, reps: int = 5):
    """Device time of the backward alone after a 512 MiB write has evicted
    L2 (so T, written by the forward, comes from HBM)."""
    import torch

    T = fwd()
    flush = torch.empty(1 << 27, device=dev)  # 512 MiB, four times L2
    times = []
    for _ in range(reps):
        flush.fill_(1.0)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        bwd(T)
        e1.record()
        torch.cuda.synchronize(dev)
        times.append(e0.elapsed_time(e1))
    del flush, T
    return statistics.median(times)


def sharded_mixture(args, dev, world, rank):
    """The multi-GPU workload as configured: a fixed total of 2^26 matrices of
    the mixture (50% N(0,1), 25% N(0,9), 25% N(0,1) with +6 on one entry per
    row), G ~ N(0,1), split into contiguous shards over the ranks
    (mhc_proj.sharding.shard_range); each rank runs fwd+bwd on its shard.
    Every rank generates the whole batch from the same seeds and keeps its
    slice, so a matrix has the same logits at every world size.  Device time
    over the timed steps, barrier and synchronize around them, max over ranks;
    value = total / slowest rank's step."""
    import torch
    import torch.distributed as dist

    import mhc_proj
    from mhc_proj.sharding import shard_range
    from mhc_proj.workloads import make_logits

    total = args.mixture_total
    a, b = shard_range(total, rank, world)
    R = make_logits("mixture", total, seed=500, device=dev)[a:b].clone()
    torch.cuda.empty_cache()
    G = make_logits("normal", total, seed=501, device=dev)[a:b].clone()
    torch.cuda.empty_cache()
    steps = 3

    def step(ev):
        ev[0].record()
        T = mhc_proj.torch.birkhoff_proj_n4(R, args.tol)["T"]
        ev[1].record()
        mhc_proj.torch.birkhoff_proj_n4_backward(G, T)["D"]
        ev[2].record()

    warm = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    step(warm)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(steps):
        step(evs[i])
    t1.record()
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
    mine = torch.tensor([ms, fwd_ms, bwd_ms, float(b - a)], device=dev, dtype=torch.float64)
    ranks = [mine]
    if world > 1:
        ranks = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(ranks, mine)
    ranks = [r.tolist() for r in ranks]
    del R, G
    torch.cuda.empty_cache()
    slow = max(range(world), key=lambda i: ranks[i][0])
    per_gpu = [{"rank": i, "matrices": int(r[3]), "ms_per_step": r[0], "forward_ms": r[1], "backward_ms": r[2],
                "hbm_gbs": (BYTES_FWD + BYTES_BWD) * r[3] / (r[0] * 1e-3) / 1e9}
               for i, r in enumerate(ranks)]
    return {"workload": f"Newton forward (tol {args.tol:g}) + IFT backward on N=2^{total.bit_length() - 1} "
                        f"matrices in total of the mixture (50% N(0,1), 25% N(0,9), 25% N(0,1)+6 on one entry "
                        f"per row), G~N(0,1), batch-sharded over {world} GPU(s)",
            "total_matrices": total, "value": total / (ranks[slow][0] * 1e-3), "unit": UNIT,
            "scaling": "strong", "slowest_rank": slow, "ms_per_step": ranks[slow][0], "steps": steps,
            "per_gpu": per_gpu}


def run_e2e(args, R, G, dev, world):
    """End to end through mhc_proj.torch.* with host buffers: each step copies
    R and G from pinned host memory, runs the forward and backward, and copies
    T and D back to pinned host memory; the batch moves in chunks over three
    streams so copies in both directions overlap the kernels.  Then the copy
    ceiling: the same copies (same chunks, streams and pinned buffers) on every
    rank at once with no kernels."""
    import torch
    import torch.distributed as dist

    import mhc_proj

    n = R.shape[0]
    chunks = args.e2e_chunks if n >= (1 << 20) else 1
    Rh = R.cpu().pin_memory()
    Gh = G.cpu().pin_memory()
    Th = torch.empty_like(Rh).pin_memory()
    Dh = torch.empty_like(Rh).pin_memory()
    streams = [torch.cuda.Stream(device=dev) for _ in range(max(1, args.e2e_streams))]
    bounds = [(n * i // chunks, n * (i + 1) // chunks) for i in range(chunks)]
    tol = args.tol

    def step():
        for i, (a, b) in enumerate(bounds):
            s = streams[i % len(streams)]
            with torch.cuda.stream(s):
                r = Rh[a:b].to(dev, non_blocking=True)
                g = Gh[a:b].to(dev, non_blocking=True)
                T = mhc_proj.torch.birkhoff_proj_n4(r, tol)["T"]
                D = mhc_proj.torch.birkhoff_proj_n4_backward(g, T)["D"]
                Th[a:b].copy_(T, non_blocking=True)
                Dh[a:b].copy_(D, non_blocking=True)
                for t in (r, g, T, D):
                    t.record_stream(s)
        for s in streams:
            torch.cuda.current_stream(dev).wait_stream(s)

    for _ in range(2):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.e2e_steps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.e2e_steps

    Rd = torch.empty_like(R)
    Gd = torch.empty_like(R)

    def copies():
        for i, (a, b) in enumerate(bounds):
            s = streams[i % len(streams)]
            with torch.cuda.stream(s):
                Rd[a:b].copy_(Rh[a:b], non_blocking=True)
                Gd[a:b].copy_(Gh[a:b], non_blocking=True)
                Th[a:b].copy_(Rd[a:b], non_blocking=True)
                Dh[a:b].copy_(Gd[a:b], non_blocking=True)
        for s in streams:
            torch.cuda.current_stream(dev).wait_stream(s)

    copies()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
    e0.record()
    for _ in range(args.e2e_steps):
        copies()
    e1.record()
    torch.cuda.synchronize(dev)
    ceiling_ms = e0.elapsed_time(e1) / args.e2e_steps
    del Rd, Gd
    nbytes = n * 64
    return {"ms": ms, "ceiling_ms": ceiling_ms, "h2d": 2 * nbytes, "d2h": 2 * nbytes,
            "how": f"pinned host R,G -> device -> fwd+bwd (public API) -> T,D to pinned host; "
                   f"{chunks} chunks over {len(streams)} streams; {args.e2e_steps} steps timed with CUDA events"}


def main():
    args = parse_args()
    if args.n is None:
        args.n = (1 << 22) if args.workload in ("sinkhorn", "sk_hres") else (1 << 24)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
