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
    ap.add_argument("--config", default="c5", choices=["c5", "c1", "c2", "c3", "c3f32", "c4"],
                    help="c5 (default): the headline 2^20-atom energy + forces step; c1: the quickstart "
                         "schedule over 4,096 atoms x 56 channel bindings; c2: 16,384-atom single-species "
                         "nu<=3 descriptor; c3/c3f32/c4: the channel-diagonal descriptor configurations "
                         "(mixed radial channels)")
    ap.add_argument("--b-basis", default="recoupled", choices=["recoupled", "term"],
                    help="B-basis of the C5 step: the recoupled passes (default) or the term-level kernels")
    ap.add_argument("--recoupled-atoms", type=int, default=0,
                    help="atoms per CTA of the recoupled passes (1-4; 0 = the evaluator's default)")
    ap.add_argument("--recoupled-threads", type=int, default=0, choices=[0, 256, 512],
                    help="threads per CTA of the recoupled passes (0 = the evaluator's default)")
    ap.add_argument("--tile-rows", type=int, default=-1, choices=[-1, 0, 8, 16],
                    help="segments per dense tile of the symmetric adjoint (0 = contraction lists; -1 = the "
                         "evaluator's default)")
    ap.add_argument("--recoupled-general", action="store_true",
                    help="the general recoupled passes instead of the M >= 0 (symmetric) ones")
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
                                          "--format=csv,noheader,nounits", "-lms", "25"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        # wait (at most 3 s) for the first sample, so that a short timed region that starts
        # right after this call is sampled from its beginning
        deadline = time.time() + 3.0
        while time.time() < deadline and self.proc.poll() is None:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.01)

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


def _cpu_sample(M, bundle_stem, forces, cores):
    """One oracle evaluation of an M-atom periodic sample; returns its wall time."""
    import numpy as np

    from oracle import oracle
    from ye3t_b200.schedules import ACEBundle
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", bundle_stem + ".npz"))
    rng = np.random.default_rng(0)
    box = (M / DENSITY) ** (1 / 3)
    pos = rng.uniform(0, box, (M, 3))
    sp = rng.integers(0, SPECIES, M).astype(np.int32)
    w = np.random.default_rng(2).normal(size=(SPECIES, b.feature_count))
    t0 = time.perf_counter()
    if forces:
        e, F = oracle.energy_forces(b, pos, box, sp, np.asarray(PREFACTOR), w, CUTOFF, LAMBDA, threads=cores)
        assert np.isfinite(e) and np.isfinite(F).all()
    else:
        off, nbr, disp = oracle.neighbor_list(pos, box, CUTOFF)
        A = oracle.ace_density(disp, off, nbr, sp, np.asarray(PREFACTOR), b.nmax, b.lmax, CUTOFF, LAMBDA)
        e = oracle.bundle_energy(b, A, sp, w, threads=cores)
        assert np.isfinite(e).all()
    return time.perf_counter() - t0


# Atoms of the small sample that measures the oracle's fixed per-step host
# cost (per-word block assembly and dispatch, which a full-size run amortises
# over 2^20 atoms); its box (13.7 A) is still larger than twice the cutoff.
CPU_FIXED_SAMPLE = 128


def _cpu_what(forces):
    if forces:
        return ("brute-force neighbour list, A-basis, then per word the reference block assembly "
                "(workflows.py:636-661), schedule evaluation (factorized_runtime.cpp:252-287 restated) and its "
                "adjoint (autograd of couplings.py:552-567), the symmetric-power adjoint, per-edge gradients and "
                "the force scatter")
    return ("brute-force neighbour list, A-basis, then per word the reference block assembly (workflows.py:636-661) "
            "and schedule evaluation (factorized_runtime.cpp:252-287 restated)")


def cpu_baseline(sample_atoms, bundle_stem, forces=True):
    """The reference CPU path restated (oracle) on all host cores, as a marginal per-atom rate:
    the time of a ``sample_atoms`` sample minus that of a 128-atom sample (the fixed per-step host
    cost), so that the rate is the one a full-size run would see."""
    cores = len(os.sched_getaffinity(0))
    M = int(sample_atoms)
    t_fixed = _cpu_sample(CPU_FIXED_SAMPLE, bundle_stem, forces, cores)
    t = _cpu_sample(M, bundle_stem, forces, cores)
    rate = (M - CPU_FIXED_SAMPLE) / max(t - t_fixed, 1e-9)
    return {"value": rate, "unit": "atoms/s", "cores": cores, "kind": "port",
            "sample": f"marginal rate: ({M} - {CPU_FIXED_SAMPLE}) atoms / ({t:.1f} s - {t_fixed:.1f} s), two "
                      f"periodic samples of the same density/species/cutoff; {_cpu_what(forces)} ({cores} "
                      f"threads); the plain {M}-atom rate is {M / t:.1f} atoms/s"}


def run_reference(args):
    """The reference's CPU path (oracle restatement) on rank 0: the warm-up's first sample
    measures the fixed per-step host cost on 128 atoms, every other step times a
    ``--cpu-sample``-atom sample; value = marginal atoms/s."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    K, W = args.steps, max(1, args.warmup)
    forces = not args.energy_only
    cores = len(os.sched_getaffinity(0))
    M = int(args.cpu_sample)
    t_fixed = _cpu_sample(CPU_FIXED_SAMPLE, args.bundle, forces, cores)
    for _ in range(W - 1):
        _cpu_sample(M, args.bundle, forces, cores)
    times = [_cpu_sample(M, args.bundle, forces, cores) for _ in range(K)]
    t = statistics.median(times)
    value = (M - CPU_FIXED_SAMPLE) / max(t - t_fixed, 1e-9)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "atoms/s", "n_gpus": args.gpus,
            "steps": K, "warmup": args.warmup, "ms_per_step": 1e3 * args.atoms / value,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": _config(args),
            "cpu_baseline": {"value": value, "unit": "atoms/s", "cores": cores, "kind": "port",
                             "sample": f"marginal rate: ({M} - {CPU_FIXED_SAMPLE}) atoms / (median {t:.1f} s of "
                                       f"{K} samples - {t_fixed:.1f} s); {_cpu_what(forces)} ({cores} threads); "
                                       f"ms_per_step is the {args.atoms}-atom step at that rate; the plain "
                                       f"{M}-atom rate is {M / t:.1f} atoms/s"},
            "e2e": {"value": value, "unit": "atoms/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _config(args):
    what = "energy" if getattr(args, "energy_only", False) else "energy + forces"
    rec = getattr(args, "b_basis", "recoupled") == "recoupled"
    sym = not getattr(args, "recoupled_general", False)
    return {"workload": f"C5 scalar ACE {what}: 2^20 atoms (periodic cubic box, 0.05/A^3, 3 species), "
                        "n_max 8, l_max 3, nu<=4 (25,328 words / 41,168 L=0 features), fp64, per-species "
                        "linear readout",
            "atoms": args.atoms, "bundle": args.bundle, "cutoff_A": CUTOFF, "radial_lambda": LAMBDA,
            "parallelism": f"atom-block x{args.gpus} (each rank bins its slab and a one-cell halo; forces "
                           "reduce-scattered)" if args.gpus > 1 else "atom-block x1",
            "atom_order": "cell order (z, y, x) of a cell list with cells >= the cutoff, so each rank's atom "
                          "block is a slab of the box",
            "b_basis": (f"recoupled pair contractions ({'M >= 0 symmetric passes' if sym else 'general passes'})"
                        if rec else "term-level factorized schedules"),
            "l2": "inputs larger than L2 (A-basis 2 GB, neighbour list 110 MB at 2^20 atoms)"}


def cell_order(pos, box, cutoff):
    """Permutation that sorts atoms by the (z, y, x) cell of a cell list whose cells are at
    least ``cutoff`` wide (stable within a cell)."""
    import numpy as np
    n = max(1, int(box / cutoff))
    c = np.clip(np.floor(np.mod(pos / box, 1.0) * n).astype(np.int64), 0, n - 1)
    return np.lexsort((c[:, 0], c[:, 1], c[:, 2]))


def run_b200(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from ye3t_b200 import _native as nat
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    from ye3t_b200.schedules import ACEBundle

    from ye3t_b200.distributed import atom_block, init_from_env, max_over_ranks as _max_over_ranks
    from ye3t_b200.distributed import block_forces, sum_over_ranks

    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    rank, world = init_from_env("nccl", 300.0, device)
    N = int(args.atoms)
    pos, species, box = make_system(N)
    order = torch.as_tensor(cell_order(pos.numpy(), box, CUTOFF))
    pos, species = pos[order].contiguous(), species[order].contiguous()
    bundle = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", args.bundle + ".npz"))
    weights = make_weights(bundle.feature_count)
    ev = ACEEvaluator(bundle, device, config=ACEConfig(CUTOFF, LAMBDA), species_prefactor=PREFACTOR,
                      weights=weights, b_basis=args.b_basis)
    forces = not args.energy_only
    physical = not args.recoupled_general
    if args.b_basis == "recoupled":
        if args.recoupled_atoms or args.recoupled_threads or args.tile_rows >= 0:
            base = (ev.RECOUPLED_TILED_SHAPE if physical else ev.RECOUPLED_GRAD_SHAPE) if forces else \
                ev.RECOUPLED_ENERGY_SHAPE
            rows = base[2] if args.tile_rows < 0 else args.tile_rows
            shape = (args.recoupled_atoms or (32 // rows if rows else base[0]), args.recoupled_threads or base[1],
                     rows)
            ev.RECOUPLED_TILED_SHAPE = ev.RECOUPLED_GRAD_SHAPE = ev.RECOUPLED_ENERGY_SHAPE = shape
        rec = ev.recoupled(physical, forces)
    else:
        rec = None
    begin, end = atom_block(rank, world, N)
    n_local = end - begin
    # this rank's slab of the box (cell-ordered atoms) with one cell layer of halo,
    # and a bound on its edge count (26.2 neighbours on average at this density),
    # so that the neighbour build neither bins the whole system nor syncs the host
    z_window = ev.slab_window(pos, box, begin, end)
    avg_deg = DENSITY * 4.0 / 3.0 * 3.141592653589793 * CUTOFF ** 3
    capacity = int(1.25 * avg_deg * n_local) + 4096
    nstatus = torch.zeros(1, dtype=torch.int32, device=device)
    pos_h = pos.pin_memory()
    sp_h = species.pin_memory()
    pos_d = pos.to(device)
    sp_d = species.to(device)
    sp_local = sp_d[begin:end]
    e_buf = torch.empty(n_local, dtype=torch.float64, device=device)
    # forces: each rank scatters its rows' edge gradients into a full array, and
    # a reduce-scatter leaves every rank the summed forces of its own block
    chunk = (N + world - 1) // world
    F_full = torch.empty((chunk * world, 3), dtype=torch.float64, device=device)
    F_block = torch.empty((chunk, 3), dtype=torch.float64, device=device)
    stages = ("neighbors", "density", "energy_grad", "edge_grad", "forces") if forces else \
        ("neighbors", "density", "energy")
    timers = {k: [] for k in stages}
    from ye3t_b200.packing import GRAD_CLASSES
    b_launches = 1 if rec is not None else GRAD_CLASSES
    # our kernels per step: 8 neighbour-count (cell binning and two two-launch prefix
    # sums included), 1 fill, density, the B-basis pass(es), then edge gradients and the
    # force gather/scatter
    launches_per_step = 10 + (b_launches + 2 if forces else 1) + (1 if world > 1 and forces else 0)

    def step(record):
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(len(stages) + 1)] if record else None

        def mark(i):
            if record:
                marks[i].record()
        mark(0)
        row, nbr = ev.neighbor_list(pos_d, box, begin, end, z_window=z_window, capacity=capacity, status=nstatus)
        mark(1)
        A = ev.density(pos_d, sp_d, box, row, nbr, begin)
        mark(2)
        if not forces:
            e_at = ev.energy_from_density(A, sp_local, out=e_buf, physical=physical)
            mark(3)
            return sum_over_ranks(e_at.sum()), None, marks
        e_at, G = ev.energy_grad(A, sp_local, physical=physical)
        mark(3)
        g = ev.edge_grad(pos_d, sp_d, box, row, nbr, G, begin=begin)
        mark(4)
        if world == 1:
            F = ev.forces_from_edges(row, nbr, g)
        else:
            F_full.zero_()
            ev.partial_forces_from_edges(row, nbr, g, begin, N, out=F_full[:N])
            F = block_forces(F_full, F_block)
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
    barrier()  # the ranks start the timed steps together (the samplers start at different times)
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
    if int(nstatus.item()) != 0:
        raise RuntimeError(f"neighbour build status {int(nstatus.item())}: slab window or edge capacity exceeded")
    forces_abs_sum = float(sum_over_ranks(F_last[:max(0, min(chunk, N - rank * chunk))].abs().sum()).item()) \
        if forces else None

    # end to end through the public API with host buffers: H2D of positions
    # and species every step, D2H of the total energy and this rank's forces
    my_rows = max(0, min(chunk, N - rank * chunk)) if world > 1 else N
    host_total = torch.empty(1, dtype=torch.float64).pin_memory()
    host_forces = torch.empty((max(my_rows, 1), 3), dtype=torch.float64).pin_memory() if forces else None

    def e2e_step():
        pos_d.copy_(pos_h, non_blocking=True)
        sp_d.copy_(sp_h, non_blocking=True)
        tot, Fd, _ = step(False)
        host_total.copy_(tot.reshape(1), non_blocking=True)
        if forces and my_rows:
            host_forces[:my_rows].copy_(Fd[:my_rows], non_blocking=True)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    peak = measure_fp64_peak(torch, nat, device)
    kern_ms = statistics.mean(timers["energy_grad" if forces else "energy"])
    flops = ev.packed.flops_per_atom()
    if rec is not None:
        kern_flops = rec.tables.flops_per_atom()["energy_grad" if forces else "energy"]
        kernel = ((f"recoupled_sym_tiled_grad_kernel<{32 // rec.tile_rows}, {rec._c.threads_per_cta}>"
                   if rec.tiles is not None else
                   f"recoupled_sym_energy_grad_kernel<{rec._c.atoms_per_cta}, {rec._c.threads_per_cta}>"
                   if forces else
                   f"recoupled_sym_energy_kernel<{rec._c.atoms_per_cta}, {rec._c.threads_per_cta}>")
                  if physical else
                  (f"recoupled_energy_grad_kernel<{rec._c.atoms_per_cta}, {rec._c.threads_per_cta}>" if forces
                   else f"recoupled_forward_kernel<false, {rec._c.atoms_per_cta}, {rec._c.threads_per_cta}>"))
        note = ("FP64 flops of the recoupled pass counted from its device tables "
                "(ye3t_b200.recoupling RecoupledSymTables / RecoupledDeviceTables .flops_per_atom)")
        tpath = os.path.join(REPO, "profiles", "recoupled_sym_grad_traffic.json" if forces and physical else "")
    else:
        kern_flops = (flops["items_grad"] if forces else flops["items"]) + 2.0 * ev.feature_count
        kernel = "ace_grad_kernel (B-basis energy + dE/dA)" if forces else "ace_eval_kernel<1> (B-basis energy)"
        note = ("FP64 flops the item walk needs on valid tuples (ye3t_b200.packing.item_grad_flops_per_atom with "
                "forces, item_flops_per_atom without) plus the readout")
        tpath = os.path.join(REPO, "profiles", "ace_grad_traffic.json" if forces else "ace_energy_traffic.json")
    sched_flops_launch = kern_flops * n_local
    term_flops_launch = (flops["terms"] + 2.0 * ev.feature_count) * n_local
    achieved = sched_flops_launch / (kern_ms * 1e-3) / 1e12
    traffic = None
    if os.path.isfile(tpath):
        with open(tpath) as fh:
            traffic = json.load(fh).get("dram_bytes_per_atom", 0) * n_local or None
    W = (bundle.lmax + 1) ** 2
    dens_ms = statistics.mean(timers["density"])
    avg_deg = float(0.05 * 4.0 / 3.0 * 3.141592653589793 * CUTOFF ** 3)
    dens_bytes_atom = 3 * 8 + 4 + 8 + 4 * avg_deg + bundle.nmax * W * 16
    dens_gbs = dens_bytes_atom * n_local / (dens_ms * 1e-3) / 1e9
    hbm_peak, hbm_src = _hbm_peak()

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
        "e2e": {"value": N / (e2e_ms * 1e-3), "unit": "atoms/s", "h2d_bytes_per_step": world * N * (24 + 4),
                "d2h_bytes_per_step": world * 8 + (N * 24 if forces else 0)},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": "fp64", "kernel": kernel, "achieved": achieved,
                     "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                     "flops_per_launch": sched_flops_launch,
                     "flops_note": note + "; the reference's forward term-by-term count for the same features is "
                                          f"{term_flops_launch:.4g} per launch",
                     "peak_source": "FP64 FMA microbenchmark (y3b_fma_peak_launch) measured in this run; "
                                    "MEASURED_PEAKS.json has no FP64 figure"},
        "roofline_density": {"bound": "hbm", "kernel": "ace_density_kernel<3>", "achieved": dens_gbs,
                             "peak": hbm_peak, "unit": "GB/s", "frac": dens_gbs / hbm_peak,
                             "bytes_per_atom": dens_bytes_atom, "peak_source": hbm_src},
        "stage_ms": {k: statistics.mean(v) for k, v in timers.items()},
        "energy_total": energy,
        "forces_abs_sum": forces_abs_sum,
        "clocks": clock_info,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def _hbm_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (measured copy)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


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
    tc_mix = evs[0].mixing_on_tensor_cores(mix.shape[0], mix.shape[2], mix.shape[3], rdt)
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
    barrier()  # the ranks start the timed steps together (the samplers start at different times)
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
        # 9 neighbour-list launches, the mixed density (species sums + tensor-core product in
        # fp32, one fused kernel in fp64), one feature launch per bundle
        "gpu_launches": (9 + (2 if tc_mix else 1) + len(evs)) * args.steps,
        "roofline": roof,
        "stage_ms": {k: statistics.mean(v) for k, v in timers.items()},
        "checksum": float(check.item()),
        "clocks": clock_info,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


# -- C1: the quickstart schedule over supplied factor arrays ---------------------------------
C1_WORKLOAD = ("C1 quickstart: compile_ace_factorized_schedules_by_L(content=(1,1,2), input_Ls=(1,1,0)), L = 0 "
               "(hash 00112c9d4a6cb444), Sym^2(V_1) -> 0 block and a leaf, on seeded N(0,1) factor arrays of 4,096 "
               "atoms x 8 radial channels (l = 1 and l = 0), all 56 ordered channel bindings (229,376 rows), fp64")


def _c1_inputs():
    """Seeded factor arrays (``torch.Generator().manual_seed(0)``: A1 then A0), the quickstart
    schedule record and the Sym^2(V_1) -> 0 table."""
    import numpy as np
    import torch

    from ye3t_b200.schedules import ACEBundle, ScheduleRecord
    g = np.load(os.path.join(REPO, "tests", "golden", "quickstart.npz"))
    specs = json.loads(bytes(g["q_specs"]).decode())
    rec = ScheduleRecord(rank=0, block_count=int(g["q_bm"].shape[1]), L_R=0, n_tuple=(), l_tuple=(),
                         block_specs=tuple(tuple(tuple(x) for x in label) for label in specs),
                         component_offsets=g["q_off"], component_label_index=g["q_cli"],
                         component_M_R=np.zeros_like(g["q_cli"]), block_m_tuples=g["q_bm"], coeffs=g["q_co"],
                         convention_hash=bytes(g["convention_hash"]).decode())
    gen = torch.Generator().manual_seed(0)
    A1 = torch.randn(4096, 8, 3, dtype=torch.float64, generator=gen)
    A0 = torch.randn(4096, 8, 1, dtype=torch.float64, generator=gen)
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", BUNDLE + ".npz"))
    pairs = [(n1, n2) for n1 in range(8) for n2 in range(8) if n1 != n2]
    return rec, A1, A0, b.sym_tables[(1, 2, 0, 0)], pairs


def _l2_flush(torch, device):
    """A buffer twice the size of L2 (126 MB), written between timed steps of small configurations."""
    buf = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    return lambda: buf.fill_(1)


def _capture(torch, fns):
    """CUDA graphs of the step functions ``fns`` (warmed up on a side stream first, as graph
    capture requires), as their replay methods; None if a capture fails (the caller then runs
    the functions directly)."""
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for fn in fns:
                fn()
        torch.cuda.current_stream().wait_stream(side)
        replays = []
        for fn in fns:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            replays.append(g.replay)
        torch.cuda.synchronize()
        return replays
    except RuntimeError as exc:
        print(f"bench: CUDA graph capture failed, running eagerly ({exc})", file=sys.stderr)
        torch.cuda.synchronize()
        return None


def _timed_steps(torch, step, steps, flush):
    """Sum of CUDA-event times of ``steps`` calls of ``step``, L2 flushed before each."""
    total = 0.0
    for _ in range(steps):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        b.synchronize()
        total += a.elapsed_time(b)
    return total / steps


def cpu_c1(steps=1):
    """The quickstart on the host, all 56 bindings.  Where the reference's own builds are present
    in oracle/_ref (its runtime core's grouped symmetric power, ye3t_runtime_core.h:1227, and its
    compiled schedule evaluator, factorized_runtime.cpp:426-548, parallel over atoms x components
    with torch's intra-op threads) they are timed (``kind: "reference"``) at the faster of one
    thread and all host cores;
    otherwise the oracle's restatement of both, one thread as the reference's serial loop
    (``kind: "port"``)."""
    import numpy as np

    from oracle import oracle
    rec, A1, A0, t, pairs = _c1_inputs()
    A1, A0 = A1.numpy(), A0.numpy()
    ref = oracle.refcore() is not None and oracle.refeval() is not None

    def once(cores):
        t0 = time.perf_counter()
        if ref:
            sym = oracle.ref_symmetric_power_monomial(A1.reshape(-1, 3), t.monomial_counts, t.output_offsets,
                                                      t.monomial_value.real, threads=cores).reshape(4096, 8)
        else:
            sym = oracle.symmetric_power_monomial(A1.reshape(-1, 3), t.monomial_counts, t.output_offsets,
                                                  t.monomial_value.real).reshape(4096, 8)
        bv = np.zeros((4096 * len(pairs), 1, 2, 1))
        for r, (n1, n2) in enumerate(pairs):
            bv[r * 4096:(r + 1) * 4096, 0, 0, 0] = sym[:, n1]
            bv[r * 4096:(r + 1) * 4096, 0, 1, 0] = A0[:, n2, 0]
        out = (oracle.ref_schedule_evaluate_record(bv, rec) if ref else oracle.schedule_evaluate_record(bv, rec))
        dt = time.perf_counter() - t0
        assert np.isfinite(out).all()
        return dt

    cores = 1
    if ref:
        # the workload is a few ms: thread start-up in the reference's parallel loops can cost more
        # than it saves, so one untimed pass at 1 thread and at all cores picks the faster
        import torch
        trial = {}
        for c in sorted({1, os.cpu_count() or 1}):
            torch.set_num_threads(c)
            once(c)
            trial[c] = min(once(c) for _ in range(3))
        cores = min(trial, key=trial.get)
        torch.set_num_threads(cores)
    best = min(once(cores) for _ in range(steps))
    if ref:
        what = ("the reference's own symmetric power (ye3t_runtime_core.h:1227) and compiled schedule "
                "evaluator (factorized_runtime.cpp:426-548), built from their sources, with numpy block "
                f"assembly (workflows.py:636-661), {cores} thread(s), the faster of 1 and all host cores")
    else:
        what = ("grouped symmetric power (ye3t_runtime_core.cpp:5279 restated), block assembly "
                "(workflows.py:636-661) and the schedule evaluation (factorized_runtime.cpp:252-287 restated), "
                "1 thread")
    return {"value": 4096 / best, "unit": "atoms/s", "cores": cores, "kind": "reference" if ref else "port",
            "sample": f"the whole C1 workload (4,096 atoms x 56 bindings): {what}; {best * 1e3:.1f} ms"}


def run_c1(args):
    import torch

    from ye3t_b200 import _native as nat
    from ye3t_b200.couplings import evaluate_factorized_schedule_torch
    from ye3t_b200.runtime import symmetric_power_monomial_contraction

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    rec, A1h, A0h, t, pairs = _c1_inputs()
    n1 = torch.tensor([p[0] for p in pairs], device=device)
    n2 = torch.tensor([p[1] for p in pairs], device=device)
    counts = torch.as_tensor(t.monomial_counts, device=device)
    offsets = torch.as_tensor(t.output_offsets, device=device)
    idx = torch.as_tensor(t.output_index, device=device)
    vals = torch.as_tensor(t.monomial_value.real.copy(), device=device)
    A1h, A0h = A1h.pin_memory(), A0h.pin_memory()
    A1 = A1h.to(device)
    A0 = A0h.to(device)
    host_out = torch.empty((4096 * len(pairs), 1), dtype=torch.float64).pin_memory()

    def step():
        sym = symmetric_power_monomial_contraction(A1.reshape(-1, 3), counts, offsets, idx, vals).reshape(4096, 8)
        bv = torch.stack((sym[:, n1].t().reshape(-1), A0[:, n2, 0].t().reshape(-1)), dim=1).reshape(-1, 1, 2, 1)
        return evaluate_factorized_schedule_torch(bv, rec)

    def e2e():
        A1.copy_(A1h, non_blocking=True)
        A0.copy_(A0h, non_blocking=True)
        host_out.copy_(step(), non_blocking=True)

    flush = _l2_flush(torch, device)
    for _ in range(args.warmup):
        step()
        e2e()
    torch.cuda.synchronize()
    # the step is a handful of short launches: capture it (and the end-to-end step with its
    # copies) in CUDA graphs and replay them; every kernel still runs on every replay
    graphs = _capture(torch, (step, e2e))
    run_step, run_e2e = graphs if graphs else (step, e2e)
    for _ in range(args.warmup):
        run_step()
        run_e2e()
    torch.cuda.synchronize()
    clocks = ClockSampler(device.index)
    clocks.start()
    ms = _timed_steps(torch, run_step, args.steps, flush)
    clock_info = clocks.stop()
    e2e_ms = _timed_steps(torch, run_e2e, args.steps, flush)
    rows = 4096 * len(pairs)
    # algorithmic bytes: the factor arrays read once, the 229,376 outputs written once
    nbytes = (4096 * 8 * 3 + 4096 * 8 + rows) * 8
    hbm_peak, hbm_src = _hbm_peak()
    gbs = nbytes / (ms * 1e-3) / 1e9
    cpu = None if args.no_cpu_baseline else cpu_c1(3)
    line = {"metric": "ACE quickstart schedule atoms/sec (c1)", "value": 4096 / (ms * 1e-3), "unit": "atoms/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded N(0,1) factors)",
            "config": {"workload": C1_WORKLOAD, "atoms": 4096, "bindings": len(pairs),
                       "l2": "L2 flushed (256 MB write) before every timed step",
                       "cuda_graph": bool(graphs)},
            "e2e": {"value": 4096 / (e2e_ms * 1e-3), "unit": "atoms/s",
                    "h2d_bytes_per_step": int(A1h.numel() + A0h.numel()) * 8, "d2h_bytes_per_step": rows * 8},
            "gpu_launches": 2 * args.steps,  # symmetric power + schedule evaluation (the binding gather is torch)
            "roofline": {"bound": "hbm", "kernel": "symmetric power + factorized schedule evaluation", "achieved": gbs,
                         "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak, "traffic": None,
                         "bytes_per_step": nbytes, "peak_source": hbm_src,
                         "note": "a few MB per step: launch-bound, not bandwidth-bound"},
            "clocks": clock_info, "cpu_baseline": cpu}
    print(json.dumps(line), flush=True)


# -- C2: single-species nu <= 3 descriptor ---------------------------------------------------
C2_BUNDLE = "ace_n8_l3_nu3_L0"
C2_WORKLOAD = ("C2 single-species scalar ACE descriptor: 16,384 atoms (periodic cubic box, 0.05/A^3), 1 species, "
               "ChebExpCos n_max 8, l_max 3, nu<=3 (3,280 words -> 2,344 L=0 features per atom), cutoff 5 A, fp64")


C2_CPU_FIXED_SAMPLE = 1024


def cpu_c2(sample_atoms):
    """The reference CPU path restated for the C2 descriptor, as a marginal per-atom rate."""
    import numpy as np

    from oracle import oracle
    from ye3t_b200.schedules import ACEBundle
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", C2_BUNDLE + ".npz"))
    cores = len(os.sched_getaffinity(0))

    def sample(M):
        rng = np.random.default_rng(0)
        box = (M / DENSITY) ** (1 / 3)
        pos = rng.uniform(0, box, (M, 3))
        sp = np.zeros(M, dtype=np.int32)
        t0 = time.perf_counter()
        off, nbr, disp = oracle.neighbor_list(pos, box, CUTOFF)
        A = oracle.ace_density(disp, off, nbr, sp, np.ones(1), b.nmax, b.lmax, CUTOFF, LAMBDA)
        F = oracle.bundle_features(b, A, threads=cores)
        assert np.isfinite(F).all()
        return time.perf_counter() - t0

    # the per-word host work is a fixed cost of about half a second, so the samples are large
    # enough that their difference is seconds of per-atom work
    fixed = C2_CPU_FIXED_SAMPLE
    sample_atoms = max(int(sample_atoms), 4 * fixed)
    t_fixed, t = sample(fixed), sample(sample_atoms)
    rate = (sample_atoms - fixed) / max(t - t_fixed, 1e-3)
    return {"value": rate, "unit": "atoms/s", "cores": cores, "kind": "port",
            "sample": f"marginal rate: ({sample_atoms} - {fixed}) atoms / ({t:.2f} s - {t_fixed:.2f} s); "
                      "brute-force neighbour list, A-basis, then per word the reference block assembly "
                      "(workflows.py:636-661) and schedule evaluation (factorized_runtime.cpp:252-287 restated) "
                      f"({cores} threads)"}


def run_c2(args):
    import torch

    from ye3t_b200 import _native as nat
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    from ye3t_b200.schedules import ACEBundle

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    N = 16384
    box = (N / DENSITY) ** (1.0 / 3.0)
    pos = torch.rand(N, 3, dtype=torch.float64, generator=torch.Generator().manual_seed(0)) * box
    pos = pos[torch.as_tensor(cell_order(pos.numpy(), box, CUTOFF))].contiguous()
    species = torch.zeros(N, dtype=torch.int32)
    bundle = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", C2_BUNDLE + ".npz"))
    ev = ACEEvaluator(bundle, device, config=ACEConfig(CUTOFF, LAMBDA), species_prefactor=[1.0])
    pos_h, sp_h = pos.pin_memory(), species.pin_memory()
    pos_d, sp_d = pos.to(device), species.to(device)
    F = torch.empty((N, ev.feature_count), dtype=torch.complex128, device=device)
    host_F = torch.empty((N, ev.feature_count), dtype=torch.complex128).pin_memory()
    stages = ("neighbors", "density", "features")
    timers = {k: [] for k in stages}
    # the neighbour array is sized from a bound (no host read of the edge count), so a step
    # has no host synchronisation and can be captured as a CUDA graph
    avg_deg = 0.05 * 4.0 / 3.0 * 3.141592653589793 * CUTOFF ** 3
    capacity = int(1.25 * avg_deg * N) + 4096
    nstatus = torch.zeros(1, dtype=torch.int32, device=device)

    def step(marks=None):
        if marks:
            marks[0].record()
        row, nbr = ev.neighbor_list(pos_d, box, capacity=capacity, status=nstatus)
        if marks:
            marks[1].record()
        A = ev.density(pos_d, sp_d, box, row, nbr)
        if marks:
            marks[2].record()
        ev.features(A, out=F)
        if marks:
            marks[3].record()
        return F

    def e2e():
        pos_d.copy_(pos_h, non_blocking=True)
        sp_d.copy_(sp_h, non_blocking=True)
        host_F.copy_(step(), non_blocking=True)

    for _ in range(args.warmup):
        step()
        e2e()
    torch.cuda.synchronize()
    # stage times from eager steps with events between the stages
    all_marks = []
    for _ in range(args.steps):
        m = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        all_marks.append(m)
        step(m)
    torch.cuda.synchronize()
    for m in all_marks:
        for k, a, b in zip(stages, m[:-1], m[1:]):
            timers[k].append(a.elapsed_time(b))
    # the step (11 launches, about 1 ms) and the end-to-end step replayed as CUDA graphs
    graphs = _capture(torch, (step, e2e))
    run_step, run_e2e = graphs if graphs else (step, e2e)
    for _ in range(args.warmup):
        run_step()
        run_e2e()
    torch.cuda.synchronize()
    clocks = ClockSampler(device.index)
    clocks.start()
    # the 614 MB feature output is larger than L2, so no flush is needed
    ms = _timed_steps(torch, run_step, args.steps, lambda: None)
    clock_info = clocks.stop()
    e2e_ms = _timed_steps(torch, run_e2e, args.steps, lambda: None)
    if int(nstatus.item()) != 0:
        raise RuntimeError(f"neighbour build status {int(nstatus.item())}: edge capacity exceeded")
    peak = measure_fp64_peak(torch, nat, device)
    feat_ms = statistics.mean(timers["features"])
    # the features come from the recoupled forward pass (fp64, scalar bundle): its
    # table-counted flops per atom
    rf = ev.recoupled_features()
    flops = rf.tables.flops_per_atom()["features"] * N
    nbytes = (ev.feature_count + bundle.nmax * (bundle.lmax + 1) ** 2) * 16 * N
    hbm_peak, hbm_src = _hbm_peak()
    if flops / (peak * 1e12) >= nbytes / (hbm_peak * 1e9):
        roof = {"bound": "fp64", "achieved": flops / (feat_ms * 1e-3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                "peak_source": "FP64 FMA microbenchmark (y3b_fma_peak_launch) in this run"}
    else:
        roof = {"bound": "hbm", "achieved": nbytes / (feat_ms * 1e-3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                "peak_source": hbm_src}
    roof.update({"kernel": "recoupled_forward_kernel<true, 1, 256> (features)", "frac": roof["achieved"] / roof["peak"],
                 "traffic": None, "flops_per_launch": flops, "bytes_per_launch": nbytes})
    cpu = None if args.no_cpu_baseline else cpu_c2(args.cpu_sample or 8192)
    line = {"metric": "ACE descriptor atoms/sec (c2)", "value": N / (ms * 1e-3), "unit": "atoms/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded uniform positions)",
            "config": {"workload": C2_WORKLOAD, "atoms": N, "bundle": C2_BUNDLE, "cutoff_A": CUTOFF,
                       "radial_lambda": LAMBDA, "l2": "feature output (614 MB) larger than L2",
                       "cuda_graph": bool(graphs), "stage_ms": "eager steps with events between the stages"},
            "e2e": {"value": N / (e2e_ms * 1e-3), "unit": "atoms/s", "h2d_bytes_per_step": N * 28,
                    "d2h_bytes_per_step": N * ev.feature_count * 16},
            "gpu_launches": 11 * args.steps,  # 9 neighbour-list, density, features
            "roofline": roof, "stage_ms": {k: statistics.mean(v) for k, v in timers.items()},
            "clocks": clock_info, "cpu_baseline": cpu}
    print(json.dumps(line), flush=True)


def _reference_line(args, metric, runs):
    """The reference arm's line from per-step ``cpu_baseline``-style records."""
    v = statistics.median([x["value"] for x in runs])
    print(json.dumps({"impl": "reference", "metric": metric, "value": v, "unit": "atoms/s", "n_gpus": args.gpus,
                      "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                      "cpu_baseline": dict(runs[-1], value=v),
                      "e2e": {"value": v, "unit": "atoms/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def main():
    args = parse()
    rank0 = int(os.environ.get("RANK", "0")) == 0
    if args.config == "c1":
        if args.impl == "reference":
            if rank0:
                _reference_line(args, "ACE quickstart schedule atoms/sec (c1)",
                                [cpu_c1() for _ in range(args.warmup + args.steps)][args.warmup:])
            return
        run_c1(args)
        return
    if args.config == "c2":
        if args.impl == "reference":
            if rank0:
                _reference_line(args, "ACE descriptor atoms/sec (c2)",
                                [cpu_c2(args.cpu_sample or 8192) for _ in range(args.steps)])
            return
        run_c2(args)
        return
    if args.config != "c5":
        if args.impl == "reference":
            if rank0:
                cfg = CHANNEL_CONFIGS[args.config]
                _reference_line(args, f"ACE channel-diagonal features atoms/sec ({args.config})",
                                [cpu_channels_baseline(cfg, 512) for _ in range(args.warmup + args.steps)]
                                [args.warmup:])
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
