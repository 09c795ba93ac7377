#!/usr/bin/env python
"""ACE features atoms/s at nu <= 4, l_max = 3 on 1..8 B200 (config C5 of the build spec).

One step = the whole hot path for one configuration of 2^20 atoms (periodic
cubic box at 0.05 atoms/A^3, 3 species, n_max 8, l_max 3, cutoff 5 A):
cell-list CSR neighbour list -> A-basis density (kernel 1) -> symmetric blocks
and all 25,328 nu <= 4 words / 41,168 L = 0 features per atom evaluated from
their compiled schedules on chip and contracted with a per-species linear
readout, together with dE/dA (kernel 2 and its adjoint) -> per-edge
gradients -> forces on every atom; total energy and forces are summed over
ranks with NCCL when N > 1.  --energy-only times the energy alone.
Atoms are block-partitioned across ranks (strong scaling of the fixed system).

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's CPU
path instead (the oracle restatement; see the cpu_baseline description).
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

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "ACE features atoms/sec at nu=4,l_max=3"
DENSITY = 0.05
CUTOFF = 5.0
LAMBDA = 5.0
PREFACTOR = [1.0, 0.75, 1.25]
SPECIES = 3
BUNDLE = "ace_n8_l3_nu4_L0"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--atoms", type=int, default=1 << 20)
    ap.add_argument("--bundle", default=BUNDLE)
    ap.add_argument("--cpu-sample", type=int, default=None,
                    help="atoms in the CPU baseline sample (default 512 with forces, 1024 energy only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", default="c5", choices=["c5", "c3", "c3f32", "c4"],
                    help="c5 (default): the headline 2^20-atom energy + forces step; c3/c3f32/c4: the "
                         "channel-diagonal descriptor configurations (mixed radial channels)")
    ap.add_argument("--recoupled", action="store_true",
                    help="B-basis through the recoupled passes (ye3t_b200.recoupling) instead of the "
                         "term-level schedule kernels")
    ap.add_argument("--recoupled-atoms", type=int, default=1,
                    help="atoms per CTA of the recoupled passes (1-4, within shared memory)")
    ap.add_argument("--recoupled-threads", type=int, default=256, choices=[256, 512],
                    help="threads per CTA of the recoupled passes")
    ap.add_argument("--recoupled-symmetric", action="store_true",
                    help="the recoupled passes over M >= 0 components (physical densities)")
    ap.add_argument("--no-recoupled-probe", action="store_true",
                    help="skip the one-off look at the recoupled passes after the measurement")
    ap.add_argument("--energy-only", action="store_true",
                    help="time the energy step alone (no adjoint, no forces)")
    return ap.parse_args()


def make_system(N):
    import torch
    box = (N / DENSITY) ** (1.0 / 3.0)
    pos = torch.rand(N, 3, dtype=torch.float64, generator=torch.Generator().manual_seed(0)) * box
    species = torch.randint(0, SPECIES, (N,), generator=torch.Generator().manual_seed(1)).to(torch.int32)
    return pos, species, box


def make_weights(F):
    import torch
    return torch.randn(SPECIES, F, dtype=torch.float64, generator=torch.Generator().manual_seed(2)) / F ** 0.5


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = str(gpu_index)
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax = float(parts[2])
                    power.append(float(parts[3]))
                except ValueError:
                    continue
                for name, flag in zip(names, parts[5:9]):
                    if flag.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def measure_fp64_peak(torch, nat, device):
    """FP64 FMA throughput of this GPU (TFLOP/s), best of 5 launches."""
    blocks, threads, iters = 148 * 8, 256, 40000
    sink = torch.empty(blocks * threads, dtype=torch.float64, device=device)
    flops = nat.DBL(0.0)
    s = nat.stream_of(device)
    best = 0.0
    for _ in range(6):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        nat.check(nat.lib().y3b_fma_peak_launch(nat.F64, blocks, threads, iters, sink.data_ptr(),
                                                 nat.ctypes.byref(flops), s), "fma_peak")
        b.record()
        b.synchronize()
        best = max(best, flops.value / (a.elapsed_time(b) * 1e-3) / 1e12)
    return best


def cpu_baseline(sample_atoms, bundle_stem, forces=True):
    """The reference CPU path restated (oracle) on a bounded sample, all host cores."""
    import numpy as np

    from oracle import oracle
    from ye3t_b200.schedules import ACEBundle
    cores = len(os.sched_getaffinity(0))
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", bundle_stem + ".npz"))
    M = int(sample_atoms)
    rng = np.random.default_rng(0)
    box = (M / DENSITY) ** (1 / 3)
    pos = rng.uniform(0, box, (M, 3))
    sp = rng.integers(0, SPECIES, M).astype(np.int32)
    w = np.random.default_rng(2).normal(size=(SPECIES, 41168 if bundle_stem == BUNDLE else b.feature_count))
    t0 = time.perf_counter()
    if forces:
        e, F = oracle.energy_forces(b, pos, box, sp, np.asarray(PREFACTOR), w, CUTOFF, LAMBDA, threads=cores)
        assert np.isfinite(e) and np.isfinite(F).all()
        what = ("then per word the reference block assembly (workflows.py:636-661), schedule evaluation "
                "(factorized_runtime.cpp:252-287 restated) and its adjoint (autograd of couplings.py:552-567), the "
                "symmetric-power adjoint, per-edge gradients and the force scatter")
    else:
        off, nbr, disp = oracle.neighbor_list(pos, box, CUTOFF)
        A = oracle.ace_density(disp, off, nbr, sp, np.asarray(PREFACTOR), b.nmax, b.lmax, CUTOFF, LAMBDA)
        e = oracle.bundle_energy(b, A, sp, w, threads=cores)
        assert np.isfinite(e).all()
        what = ("then per word the reference block assembly (workflows.py:636-661) and schedule evaluation "
                "(factorized_runtime.cpp:252-287 restated)")
    dt = time.perf_counter() - t0
    return {"value": M / dt, "unit": "atoms/s", "cores": cores, "kind": "port",
            "sample": f"{M} atoms of the same density/species/cutoff in a {box:.1f} A periodic box; brute-force "
                      f"neighbour list, A-basis, {what} ({cores} threads); {dt:.1f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    K, W = args.steps, args.warmup
    base = None
    times = []
    for i in range(W + K):
        cb = cpu_baseline(args.cpu_sample, args.bundle, forces=not args.energy_only)
        if i >= W:
            times.append(cb)
        base = cb
    vals = [t["value"] for t in times]
    value = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "atoms/s", "n_gpus": args.gpus,
            "steps": K, "warmup": W, "ms_per_step": 1e3 * args.cpu_sample / value,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": _config(args),
            "cpu_baseline": {"value": value, "unit": "atoms/s", "cores": base["cores"], "kind": "port",
                             "sample": base["sample"]},
            "e2e": {"value": value, "unit": "atoms/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def recoupled_probe(torch, ev, bundle, weights, device, pos_d, sp_d, box, forces, ref_ms, F_ref=None, E_ref=None):
    """One look at the recoupled B-basis passes on this run's own system, after every timed
    region and outside the reported value: the pass's CUDA-event time in two CTA shapes
    (best of three after one warm-up call) against the term-level kernels' stage time of the
    timed steps (``ref_ms``), and the largest relative difference of the energies (and of
    dE/dA with forces) from the term-level kernels on the same A."""
    try:
        from ye3t_b200.recoupling import RecoupledEvaluator, build_recoupled_plan
        N = pos_d.shape[0]
        row, nbr = ev.neighbor_list(pos_d, box, 0, N)
        A = ev.density(pos_d, sp_d, box, row, nbr, 0)
        sp = sp_d[:N].contiguous()

        def timed(fn):
            fn()
            best = None
            for _ in range(3):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                out = fn()
                b.record()
                torch.cuda.synchronize()
                best = a.elapsed_time(b) if best is None else min(best, a.elapsed_time(b))
            return best, out

        if forces:
            e0, G0 = ev.energy_grad(A, sp)
        else:
            e0 = ev.energy_from_density(A, sp)
        plan = build_recoupled_plan(bundle)
        try:  # the symmetric shapes are valid only for densities with the physical symmetry
            RecoupledEvaluator(bundle, device, None, plan=plan, symmetric=True).check_symmetry(A)
            density_symmetric = True
        except ValueError as exc:
            density_symmetric = str(exc)[:200]
        shapes, forward = {}, {}
        for na, th, symmetric in ((1, 256, False), (2, 256, False), (2, 512, False), (3, 512, False),
                                  (1, 256, True), (2, 256, True), (4, 256, True), (3, 512, True)):
            key = f"{'symmetric ' if symmetric else ''}{na}x{th}"
            try:  # one shape's failure is recorded beside it and does not hide the others
                rec = RecoupledEvaluator(bundle, device, weights, plan=plan, atoms_per_cta=na,
                                         threads_per_cta=th, symmetric=symmetric)
                if forces:
                    ms, (e1, G1) = timed(lambda: rec.energy_grad(A, sp))
                    gdiff = float((G1 - G0).abs().max() / G0.abs().max())
                    del G1
                else:
                    ms, e1 = timed(lambda: rec.energy(A, sp))
                    gdiff = None
                shapes[key] = {"ms": ms, "energy_max_rel_diff": float((e1 - e0).abs().max() / e0.abs().max()),
                               "dEdA_max_rel_diff": gdiff}
                if forces and (na, th) in ((1, 256), (2, 512), (4, 256)):
                    fms, e2 = timed(lambda: rec.energy(A, sp))
                    forward[key] = {"ms": fms,
                                    "energy_max_rel_diff": float((e2 - e0).abs().max() / e0.abs().max())}
            except Exception as exc:
                shapes[key] = {"error": f"{type(exc).__name__}: {exc}"[:200]}
        timed_ms = [v["ms"] for v in shapes.values() if "ms" in v]
        best = min(timed_ms) if timed_ms else None
        step = None
        if best is not None:
            try:  # one whole step with the fastest shape, its forces against the measured run's
                key = min((k for k in shapes if "ms" in shapes[k]), key=lambda k: shapes[k]["ms"])
                symmetric = key.startswith("symmetric")
                na, th = (int(v) for v in key.split()[-1].split("x"))
                rec = RecoupledEvaluator(bundle, device, weights, plan=plan, atoms_per_cta=na, threads_per_cta=th,
                                         symmetric=symmetric)

                def full_step():
                    r, nb = ev.neighbor_list(pos_d, box, 0, N)
                    Ad = ev.density(pos_d, sp_d, box, r, nb, 0)
                    if not forces:
                        return rec.energy(Ad, sp).sum(), None
                    e, G = rec.energy_grad(Ad, sp)
                    return e.sum(), ev.forces_from_edges(r, nb, ev.edge_grad(pos_d, sp_d, box, r, nb, G, begin=0))

                sms, (E, F) = timed(full_step)
                step = {"shape": key, "ms": sms, "atoms_per_s": N / (sms * 1e-3),
                        "energy_rel_diff": None if E_ref is None else float(abs(float(E) - E_ref) / abs(E_ref)),
                        "forces_max_rel_diff": None if F is None or F_ref is None else
                        float((F - F_ref).abs().max() / F_ref.abs().max())}
            except Exception as exc:
                step = {"error": f"{type(exc).__name__}: {exc}"[:200]}
        return {"pass": "energy_grad" if forces else "energy", "atoms": int(N),
                "term_level_ms": ref_ms, "shapes_atoms_x_threads": shapes,
                "speedup_vs_term_level": ref_ms / best if best else None,
                "forward_energy_shapes": forward or None, "whole_step_with_fastest_shape": step,
                "density_symmetric": density_symmetric,
                "note": "not part of value; timed after the timed regions, against the term-level stage time"}
    except Exception as exc:  # the probe must not take the measured line with it
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


def _config(args):
    what = "energy" if getattr(args, "energy_only", False) else "energy + forces"
    return {"workload": f"C5 scalar ACE {what}: 2^20 atoms (periodic cubic box, 0.05/A^3, 3 species), "
                        "n_max 8, l_max 3, nu<=4 (25,328 words / 41,168 L=0 features), fp64, per-species "
                        "linear readout",
            "atoms": args.atoms, "bundle": args.bundle, "cutoff_A": CUTOFF, "radial_lambda": LAMBDA,
            "parallelism": f"atom-block x{args.gpus}",
            "b_basis": (f"recoupled pair contractions ({'M >= 0 symmetric, ' if args.recoupled_symmetric else ''}"
                        f"{args.recoupled_atoms} atoms and {args.recoupled_threads} threads per CTA)"
                        if getattr(args, "recoupled", False) else "term-level factorized schedules"),
            "l2": "inputs larger than L2 (A-basis 2 GB, neighbour list 110 MB at 2^20 atoms)"}


def run_b200(args):
    import torch
    import torch.distributed as dist

    from ye3t_b200 import _native as nat
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    from ye3t_b200.schedules import ACEBundle

    from ye3t_b200.distributed import atom_block, init_from_env, max_over_ranks as _max_over_ranks
    from ye3t_b200.distributed import sum_over_ranks

    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    rank, world = init_from_env("nccl", 300.0, device)
    N = int(args.atoms)
    pos, species, box = make_system(N)
    bundle = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", args.bundle + ".npz"))
    weights = make_weights(bundle.feature_count)
    ev = ACEEvaluator(bundle, device, config=ACEConfig(CUTOFF, LAMBDA), species_prefactor=PREFACTOR,
                      weights=weights)
    begin, end = atom_block(rank, world, N)
    n_local = end - begin
    pos_h = pos.pin_memory()
    sp_h = species.pin_memory()
    pos_d = pos.to(device)
    sp_d = species.to(device)
    e_buf = torch.empty(n_local, dtype=torch.float64, device=device)
    F_buf = torch.empty((N, 3), dtype=torch.float64, device=device)
    forces = not args.energy_only
    stages = ("neighbors", "density", "energy_grad", "edge_grad", "forces") if forces else \
        ("neighbors", "density", "energy")
    timers = {k: [] for k in stages}
    # our kernels per step: 6 neighbour-count, 1 fill, density, then the
    # B-basis energy, or the B-basis adjoint (one launch per item class) + edge
    # gradients + force gather/scatter
    from ye3t_b200.packing import GRAD_CLASSES
    rec = None
    if args.recoupled:
        from ye3t_b200.recoupling import RecoupledEvaluator
        rec = RecoupledEvaluator(bundle, device, weights, atoms_per_cta=args.recoupled_atoms,
                                 threads_per_cta=args.recoupled_threads, symmetric=args.recoupled_symmetric)
    b_launches = 1 if rec is not None else GRAD_CLASSES
    launches_per_step = 8 + (b_launches + 2 if forces else 1)

    def step(record):
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(len(stages) + 1)] if record else None

        def mark(i):
            if record:
                marks[i].record()
        mark(0)
        row, nbr = ev.neighbor_list(pos_d, box, begin, end)
        mark(1)
        A = ev.density(pos_d, sp_d, box, row, nbr, begin)
        mark(2)
        if not forces:
            e_at = rec.energy(A, sp_d[begin:end]) if rec is not None else \
                ev.energy_from_density(A, sp_d[begin:end], out=e_buf)
            mark(3)
            return sum_over_ranks(e_at.sum()), None, marks
        e_at, G = rec.energy_grad(A, sp_d[begin:end]) if rec is not None else ev.energy_grad(A, sp_d[begin:end])
        mark(3)
        g = ev.edge_grad(pos_d, sp_d, box, row, nbr, G, begin=begin)
        mark(4)
        if world == 1:
            F = ev.forces_from_edges(row, nbr, g)
        else:
            F_buf.zero_()
            F = sum_over_ranks(ev.partial_forces_from_edges(row, nbr, g, begin, N, out=F_buf))
        mark(5)
        return sum_over_ranks(e_at.sum()), F, marks

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        return _max_over_ranks(x, device)

    for _ in range(args.warmup):
        step(False)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = []
    t0.record()
    for _ in range(args.steps):
        total, F_last, m = step(True)
        marks.append(m)
    t1.record()
    barrier()
    clock_info = clocks.stop()
    dev_ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
    for m in marks:
        for k, a, b in zip(stages, m[:-1], m[1:]):
            timers[k].append(a.elapsed_time(b))
    energy = float(total.item())

    # end to end through the public API with host buffers: H2D of positions
    # and species every step, D2H of the total energy (and the forces)
    for _ in range(max(1, args.warmup // 2)):
        pos_d.copy_(pos_h, non_blocking=True)
        sp_d.copy_(sp_h, non_blocking=True)
        step(False)[0].to("cpu", non_blocking=False)
    host_total = torch.empty(1, dtype=torch.float64).pin_memory()
    host_forces = torch.empty((N, 3), dtype=torch.float64).pin_memory() if forces else None
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        pos_d.copy_(pos_h, non_blocking=True)
        sp_d.copy_(sp_h, non_blocking=True)
        tot, Fd, _ = step(False)
        host_total.copy_(tot.reshape(1), non_blocking=True)
        if forces:
            host_forces.copy_(Fd, non_blocking=True)
    e1.record()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    peak = measure_fp64_peak(torch, nat, device)
    flops = ev.packed.flops_per_atom()
    kern_ms = statistics.mean(timers["energy_grad" if forces else "energy"])
    kern_flops = (flops["items_grad"] if forces else flops["items"]) + 2.0 * ev.feature_count
    if rec is not None:
        rflops = rec.tables.flops_per_atom()
        kern_flops = rflops["energy_grad" if forces else "energy"]
    sched_flops_launch = kern_flops * n_local
    term_flops_launch = (flops["terms"] + 2.0 * ev.feature_count) * n_local
    achieved = sched_flops_launch / (kern_ms * 1e-3) / 1e12
    W = (bundle.lmax + 1) ** 2
    dens_ms = statistics.mean(timers["density"])
    avg_deg = float(0.05 * 4.0 / 3.0 * 3.141592653589793 * CUTOFF ** 3)
    dens_bytes_atom = 3 * 8 + 4 + 8 + 4 * avg_deg + bundle.nmax * W * 16
    dens_gbs = dens_bytes_atom * n_local / (dens_ms * 1e-3) / 1e9
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as fh:
            hbm_peak = float(json.load(fh)["hbm_gbs"])
        hbm_src = "MEASURED_PEAKS.json hbm_gbs (measured copy)"
    except (OSError, KeyError, ValueError):
        hbm_peak, hbm_src = 6650.0, "fallback 6.65 TB/s"
    traffic = None
    tpath = os.path.join(REPO, "profiles", "ace_grad_traffic.json" if forces else "ace_energy_traffic.json")
    if rec is None and os.path.exists(tpath):
        with open(tpath) as fh:
            t = json.load(fh)
        traffic = t.get("dram_bytes_per_atom", 0) * n_local or None

    forces_abs_sum = float(F_last.abs().sum().item()) if forces else None
    probe = None
    if world == 1 and rec is None and not args.no_recoupled_probe:
        probe = recoupled_probe(torch, ev, bundle, weights, device, pos_d, sp_d, box, forces,
                                statistics.mean(timers["energy_grad" if forces else "energy"]),
                                F_ref=F_last if forces else None, E_ref=energy)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_sample, args.bundle, forces=not args.energy_only)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    value = N / (dev_ms * 1e-3)
    line = {
        "metric": METRIC, "value": value, "unit": "atoms/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded uniform positions, random readout)",
        "config": _config(args),
        "e2e": {"value": N / (e2e_ms * 1e-3), "unit": "atoms/s", "h2d_bytes_per_step": N * (24 + 4),
                "d2h_bytes_per_step": 8 + (N * 24 if forces else 0)},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": "fp64",
                     "kernel": (("recoupled_energy_grad_kernel (B-basis energy + dE/dA, recoupled)" if forces
                                 else "recoupled_forward_kernel<false> (B-basis energy, recoupled)")
                                if rec is not None else
                                ("ace_grad_kernel (B-basis energy + dE/dA)" if forces
                                 else "ace_eval_kernel<1> (B-basis energy, symmetric blocks on chip)")),
                     "achieved": achieved,
                     "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                     "flops_per_launch": sched_flops_launch,
                     "flops_note": ("FP64 flops of the recoupled pass counted from its tables "
                                    "(ye3t_b200.recoupling.RecoupledDeviceTables / RecoupledSymTables"
                                    ".flops_per_atom)"
                                    if rec is not None else
                                    "FP64 flops the item walk needs on valid tuples "
                                    "(ye3t_b200.packing.item_grad_flops_per_atom with forces, "
                                    "item_flops_per_atom without) plus the readout") +
                                   "; the reference's forward term-by-term count for the same features is "
                                   f"{term_flops_launch:.4g} per launch",
                     "peak_source": "FP64 FMA microbenchmark (y3b_fma_peak_launch) measured in this run; "
                                    "MEASURED_PEAKS.json has no FP64 figure"},
        "roofline_density": {"bound": "hbm", "kernel": "ace_density_kernel<3>", "achieved": dens_gbs,
                             "peak": hbm_peak, "unit": "GB/s", "frac": dens_gbs / hbm_peak,
                             "bytes_per_atom": dens_bytes_atom, "peak_source": hbm_src},
        "stage_ms": {k: statistics.mean(v) for k, v in timers.items()},
        "energy_total": energy,
        "forces_abs_sum": forces_abs_sum,
        "recoupled_probe": probe,
        "clocks": clock_info,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


# Channel-diagonal configurations: radial channels mixed per species pair,
# every word reading one mixed channel (packing bundles with nmax 1).
CHANNEL_CONFIGS = {
    "c3": dict(atoms=65536, species=4, nmax=12, channels=32, lmax=4, bundles=["ace_diag_l4_nu4_L0"], dtype="f64",
               workload="C3 multi-species scalar ACE: 65,536 atoms (periodic cubic box, 0.05/A^3), 4 species, "
                        "ChebExpCos n_max 12 mixed per species pair to 32 channels, l_max 4, nu<=4 "
                        "channel-diagonal words (53 words / 71 L=0 features per channel, 2,272 per atom)"),
    "c3f32": dict(atoms=65536, species=4, nmax=12, channels=32, lmax=4, bundles=["ace_diag_l4_nu4_L0"],
                  dtype="f32", workload="C3 as above, evaluated in fp32"),
    "c4": dict(atoms=32768, species=2, nmax=8, channels=64, lmax=3,
               bundles=["ace_diag_l3_nu3_L0", "ace_diag_l3_nu3_L1", "ace_diag_l3_nu3_L2"], dtype="f32",
               workload="C4 equivariant couplings: 32,768 atoms, 2 species, n_max 8 mixed per species pair to "
                        "64 channels, l_max 3, nu<=3 channel-diagonal words, outputs L = 0, 1, 2 (13 / 20 / 29 "
                        "labels per channel, 13,952 components per atom)"),
}


def _channel_system(cfg):
    import torch
    N = cfg["atoms"]
    box = (N / DENSITY) ** (1.0 / 3.0)
    pos = torch.rand(N, 3, dtype=torch.float64, generator=torch.Generator().manual_seed(0)) * box
    species = torch.randint(0, cfg["species"], (N,), generator=torch.Generator().manual_seed(1)).to(torch.int32)
    mix = torch.randn(cfg["species"], cfg["species"], cfg["channels"], cfg["nmax"], dtype=torch.float64,
                      generator=torch.Generator().manual_seed(2)) / cfg["nmax"] ** 0.5
    return pos, species, box, mix


def cpu_channels_baseline(cfg, sample_atoms):
    """The reference CPU path restated (oracle) for a channel configuration on a bounded sample."""
    import numpy as np

    from oracle import oracle
    from ye3t_b200.schedules import ACEBundle
    cores = len(os.sched_getaffinity(0))
    bundles = [ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", b + ".npz")) for b in cfg["bundles"]]
    M = int(sample_atoms)
    rng = np.random.default_rng(0)
    box = (M / DENSITY) ** (1 / 3)
    pos = rng.uniform(0, box, (M, 3))
    sp = rng.integers(0, cfg["species"], M).astype(np.int32)
    mix = rng.normal(size=(cfg["species"], cfg["species"], cfg["channels"], cfg["nmax"])) / cfg["nmax"] ** 0.5
    t0 = time.perf_counter()
    off, nbr, disp = oracle.neighbor_list(pos, box, CUTOFF)
    A = oracle.ace_density_mixed(disp, off, nbr, sp, mix, cfg["nmax"], cfg["lmax"], CUTOFF, LAMBDA)
    total = 0.0
    for b in bundles:
        for c in range(cfg["channels"]):
            total += float(np.abs(oracle.bundle_features(b, A[:, c:c + 1, :], threads=cores).real).sum())
    dt = time.perf_counter() - t0
    assert np.isfinite(total)
    return {"value": M / dt, "unit": "atoms/s", "cores": cores, "kind": "port",
            "sample": f"{M} atoms of the same density/species/cutoff in a {box:.1f} A periodic box; brute-force "
                      f"neighbour list, mixed A-basis (radial table, per-pair contraction as "
                      f"ye3t_runtime_core.cpp:651, harmonics, density_accumulate), then per channel and word the "
                      f"reference block assembly and schedule evaluation, fp64 ({cores} threads); {dt:.1f} s"}


def run_channels(args):
    import torch
    import torch.distributed as dist

    from ye3t_b200 import _native as nat
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    from ye3t_b200.distributed import atom_block, init_from_env, max_over_ranks as _max_over_ranks
    from ye3t_b200.schedules import ACEBundle

    cfg = CHANNEL_CONFIGS[args.config]
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    rank, world = init_from_env("nccl", 300.0, device)
    pos, species, box, mix = _channel_system(cfg)
    N = cfg["atoms"]
    rdt = torch.float64 if cfg["dtype"] == "f64" else torch.float32
    evs = [ACEEvaluator(ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", b + ".npz")), device,
                        config=ACEConfig(CUTOFF, LAMBDA)) for b in cfg["bundles"]]
    begin, end = atom_block(rank, world, N)
    n_local = end - begin
    pos_h, sp_h = pos.pin_memory(), species.pin_memory()
    pos_d, sp_d = pos.to(device), species.to(device)
    mix_d = mix.to(device, rdt)
    stages = ("neighbors", "density", "features")
    timers = {k: [] for k in stages}

    def step(record):
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        if record:
            marks[0].record()
        row, nbr = evs[0].neighbor_list(pos_d, box, begin, end)
        if record:
            marks[1].record()
        A = evs[0].density_mixed(pos_d, sp_d, box, row, nbr, mix_d, begin=begin, dtype=rdt)
        if record:
            marks[2].record()
        check = torch.zeros((), dtype=torch.float64, device=device)
        for ev in evs:
            check += ev.channel_features(A).real.abs().sum().to(torch.float64)
        if record:
            marks[3].record()
        return check, marks

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(False)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = []
    t0.record()
    for _ in range(args.steps):
        check, m = step(True)
        marks.append(m)
    t1.record()
    barrier()
    clock_info = clocks.stop()
    dev_ms = _max_over_ranks(t0.elapsed_time(t1) / args.steps, device)
    for m in marks:
        for k, a, b in zip(stages, m[:-1], m[1:]):
            timers[k].append(a.elapsed_time(b))
    host = torch.empty(1, dtype=torch.float64).pin_memory()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        pos_d.copy_(pos_h, non_blocking=True)
        sp_d.copy_(sp_h, non_blocking=True)
        c, _ = step(False)
        host.copy_(c.reshape(1), non_blocking=True)
    e1.record()
    barrier()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / args.steps, device)
    # roofline of the B-basis stage: algorithmic flops (needed item flops per
    # atom and channel) against the FMA peak of the compute type, and the
    # feature bytes written against HBM; the larger time is the bound
    best = 0.0
    sink = torch.empty(148 * 8 * 256, dtype=rdt, device=device)
    fl = nat.DBL(0.0)
    for _ in range(6):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        nat.check(nat.lib().y3b_fma_peak_launch(nat.dtype_code(rdt), 148 * 8, 256, 40000, sink.data_ptr(),
                                                 nat.ctypes.byref(fl), nat.stream_of(device)), "fma_peak")
        b.record()
        b.synchronize()
        best = max(best, fl.value / (a.elapsed_time(b) * 1e-3) / 1e12)
    C = cfg["channels"]
    feat_flops = sum(ev.packed.flops_per_atom()["items"] for ev in evs) * C * n_local
    cplx = 16 if rdt == torch.float64 else 8
    W = (cfg["lmax"] + 1) ** 2
    feat_bytes = (sum(ev.feature_count for ev in evs) * C + len(evs) * C * W) * cplx * n_local
    feat_ms = statistics.mean(timers["features"])
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as fh:
            hbm_peak = float(json.load(fh)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        hbm_peak = 6650.0
    t_fp = feat_flops / (best * 1e12)
    t_hbm = feat_bytes / (hbm_peak * 1e9)
    if t_fp >= t_hbm:
        roof = {"bound": cfg["dtype"], "achieved": feat_flops / (feat_ms * 1e-3) / 1e12, "peak": best,
                "unit": "TFLOP/s", "peak_source": f"{cfg['dtype']} FMA microbenchmark (y3b_fma_peak_launch) in "
                                                  "this run"}
    else:
        roof = {"bound": "hbm", "achieved": feat_bytes / (feat_ms * 1e-3) / 1e9, "peak": hbm_peak,
                "unit": "GB/s", "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured copy)"}
    roof.update({"kernel": f"ace_eval_kernel<{'double' if rdt == torch.float64 else 'float'}, 0> (features, "
                           "all channels of all bundles)",
                 "frac": roof["achieved"] / roof["peak"], "traffic": None,
                 "flops_per_step": feat_flops, "bytes_per_step": feat_bytes})
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_channels_baseline(cfg, 512)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": f"ACE channel-diagonal features atoms/sec ({args.config})", "value": N / (dev_ms * 1e-3),
        "unit": "atoms/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (seeded uniform positions, random mixing tables)",
        "config": {"workload": cfg["workload"], "atoms": N, "bundles": cfg["bundles"], "cutoff_A": CUTOFF,
                   "radial_lambda": LAMBDA, "parallelism": f"atom-block x{world}",
                   "l2": "feature output larger than L2 (written to HBM every step)"},
        "e2e": {"value": N / (e2e_ms * 1e-3), "unit": "atoms/s", "h2d_bytes_per_step": N * (24 + 4),
                "d2h_bytes_per_step": 8,
                "note": "features stay on the device (sharded descriptor); a checksum is read back"},
        "gpu_launches": (8 + len(evs)) * args.steps,  # 7 neighbour-list, mixed density, one per bundle
        "roofline": roof,
        "stage_ms": {k: statistics.mean(v) for k, v in timers.items()},
        "checksum": float(check.item()),
        "clocks": clock_info,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.config != "c5":
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                cfg = CHANNEL_CONFIGS[args.config]
                vals = [cpu_channels_baseline(cfg, 512) for _ in range(args.warmup + args.steps)][args.warmup:]
                v = statistics.median([x["value"] for x in vals])
                print(json.dumps({"impl": "reference", "metric": f"ACE channel-diagonal features atoms/sec "
                                                               f"({args.config})", "value": v, "unit": "atoms/s",
                                  "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                                  "higher_is_better": True, "cpu_baseline": dict(vals[-1], value=v),
                                  "e2e": {"value": v, "unit": "atoms/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}), flush=True)
            return
        run_channels(args)
        return
    if args.cpu_sample is None:
        args.cpu_sample = 1024 if args.energy_only else 512
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
