"""Generate the golden fixtures in this directory from the reference ye3t.

Run only where the reference is importable and its torch-free runtime core has
been compiled into oracle/_ref (``make -C oracle ref``):

    PYTHONPATH=<ye3t checkout>:<this repo> python tests/golden/make_golden.py

Every expected value below is produced by the reference's own public
functions (cited per fixture); the inputs are seeded.  The GPU box never runs
this script: tests read the committed ``.npz`` files.
"""

from __future__ import annotations

import ctypes
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

os.environ.setdefault("YE3T_ENABLE_CPP_RUNTIME_JIT", "1")
os.environ.setdefault("TORCH_EXTENSIONS_DIR", os.path.join(REPO, "oracle", "_build", "torch_ext"))

from ye3t.couplings import compile_ace_factorized_schedules_by_L  # noqa: E402
from ye3t import couplings  # noqa: E402
from ye3t.runtime.execution_plan import (  # noqa: E402
    cheb_exp_cos_radial_table_with_derivative, density_accumulate,
    spherical_harmonics_table_with_derivative)
from ye3t.runtime.symmetric_power import symmetric_power_product_plan_contraction  # noqa: E402

from ye3t_b200.schedules import ACEBundle, ScheduleRecord  # noqa: E402

from oracle.reference import reference_dir  # noqa: E402

REF_DIR = reference_dir()
if REF_DIR is None:
    raise SystemExit("the reference checkout is needed: set YE3T_REFERENCE (oracle/reference.py)")
REF_FIXTURE = os.path.join(REF_DIR, "tests", "fixtures", "shared_monomial_plan_v1.txt")


def _record_arrays(prefix, rec: ScheduleRecord, out: dict):
    out[prefix + "off"] = rec.component_offsets
    out[prefix + "cli"] = rec.component_label_index
    out[prefix + "bm"] = rec.block_m_tuples
    out[prefix + "co"] = rec.coeffs
    out[prefix + "bl"] = rec.block_L_by_label()
    out[prefix + "specs"] = np.frombuffer(json.dumps(rec.block_specs).encode(), dtype=np.uint8)


SCHEDULE_CASES = [((1, 1, 2), (1, 1, 0), 0), ((1, 1, 2), (1, 1, 0), 2), ((1, 1, 2, 3), (1, 1, 2, 2), 1),
                  ((1, 2, 3, 4), (3, 3, 3, 3), 0), ((1, 2, 3, 4), (3, 3, 3, 3), 2),
                  ((1, 1, 2, 2), (2, 2, 3, 3), 4), ((1, 1, 1, 1), (3, 3, 3, 3), 6),
                  ((1, 2, 2, 3), (0, 1, 2, 3), 0)]


def schedules_fixture():
    """``ACEFactorizedScheduleReport.evaluate`` (``couplings/__init__.py:2574``) on seeded blocks."""
    cases = SCHEDULE_CASES
    out, meta = {}, []
    g = torch.Generator().manual_seed(2026)
    for i, (content, ls, L) in enumerate(cases):
        rep = compile_ace_factorized_schedules_by_L(content=content, input_Ls=ls)
        sched = rep.schedules_by_L[L]
        rec = ScheduleRecord.from_schedule(sched, rep.convention_hash)
        batch = 7
        mdim = rec.max_block_m_dim
        bl = rec.block_L_by_label()
        re = torch.randn(batch, rec.basis_count, rec.block_count, mdim, dtype=torch.float64, generator=g)
        im = torch.randn(batch, rec.basis_count, rec.block_count, mdim, dtype=torch.float64, generator=g)
        mask = torch.zeros(rec.basis_count, rec.block_count, mdim, dtype=torch.bool)
        for a in range(rec.basis_count):
            for b in range(rec.block_count):
                mask[a, b, : 2 * bl[a, b] + 1] = True
        bv_c = torch.complex(re, im) * mask
        bv_r = re * mask
        outc_cpp = rep.evaluate(bv_c, target_L=L, backend="cpp")
        outc_torch = rep.evaluate(bv_c, target_L=L, backend="torch")
        outr_cpp = rep.evaluate(bv_r, target_L=L, backend="cpp")
        bv_f = bv_r.to(torch.float32)
        outf_cpp = rep.evaluate(bv_f, target_L=L, backend="cpp")
        p = f"s{i}_"
        _record_arrays(p, rec, out)
        out[p + "bvc"] = bv_c.numpy()
        out[p + "bvr"] = bv_r.numpy()
        out[p + "outc_cpp"] = outc_cpp.numpy()
        out[p + "outc_torch"] = outc_torch.numpy()
        out[p + "outr_cpp"] = outr_cpp.numpy()
        out[p + "outf_cpp"] = outf_cpp.numpy()
        meta.append({"content": content, "input_Ls": ls, "L": L, "convention_hash": rep.convention_hash,
                     "basis_count": rec.basis_count, "component_count": rec.component_count,
                     "term_count": rec.term_count, "block_count": rec.block_count})
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "schedules.npz"), **out)
    print("schedules.npz", len(cases), "cases")


def quickstart_fixture():
    """Config C1: README quickstart schedule applied to seeded factor arrays.

    Block assembly follows ``ye3t/workflows.py:636-661``: channel ``(n, l)``
    is ``multiplets[l][..., n-1, :]``; symmetric blocks go through
    ``symmetric_power_product_plan_contraction`` with the plan built as in
    ``workflows.py:544-556``.
    """
    rep = compile_ace_factorized_schedules_by_L(content=(1, 1, 2), input_Ls=(1, 1, 0))
    g = torch.Generator().manual_seed(0)
    A1 = torch.randn(4096, 8, 3, dtype=torch.float64, generator=g)
    A0 = torch.randn(4096, 8, 1, dtype=torch.float64, generator=g)
    multiplets = {1: A1, 0: A0}
    sched = rep.schedules_by_L[0]
    width = 2 * int(sched.block_L_by_label().max()) + 1
    rows, prepared = [], {}
    for blocks in sched.block_specs:
        row = []
        for block in blocks:
            key = (block["n"], block["l"], block.get("k_b"), block.get("Lambda"), block.get("multiplicity_index"))
            if key not in prepared:
                src = multiplets[block["l"]][..., block["n"] - 1, :]
                if block["kind"] == "sym":
                    plan = couplings.symmetric_power_product_plan(
                        [{"descriptor_index": m, "power": block["k_b"], "input_L": block["l"],
                          "output_L": block["Lambda"], "multiplicity_index": block["multiplicity_index"],
                          "component_index": m, "channel_indices": tuple(range(2 * block["l"] + 1))}
                         for m in range(2 * block["Lambda"] + 1)],
                        descriptor_count=2 * block["Lambda"] + 1, channel_count=2 * block["l"] + 1,
                        basis_convention="complex_magnetic")
                    src = symmetric_power_product_plan_contraction(src, plan)
                prepared[key] = torch.nn.functional.pad(src, (0, width - src.shape[-1]))
            row.append(prepared[key])
        rows.append(torch.stack(row, dim=-2))
    bv = torch.stack(rows, dim=-3)
    out_cpp = rep.evaluate(bv, target_L=0, backend="cpp")
    out_torch = rep.evaluate(bv, target_L=0, backend="torch")
    rec = ScheduleRecord.from_schedule(sched, rep.convention_hash)
    # A1/A0 are regenerated by the tests from the same seed; the first rows
    # are kept to confirm the regeneration.
    arrays = {"A1_head": A1[:16].numpy(), "A0_head": A0[:16].numpy(), "bv": bv.numpy(), "out_cpp": out_cpp.numpy(),
              "out_torch": out_torch.numpy()}
    _record_arrays("q_", rec, arrays)
    arrays["convention_hash"] = np.frombuffer(rep.convention_hash.encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "quickstart.npz"), **arrays)
    print("quickstart.npz hash", rep.convention_hash, "out[:3]", out_cpp[:3].flatten())


def sympow_fixture():
    """Each symmetric block kind of the nu<=4 bundle through ``symmetric_power_product_plan_contraction``."""
    bundle = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu4_L0.npz"))
    g = torch.Generator().manual_seed(7)
    out = {}
    keys = sorted(bundle.sym_tables)
    for j, key in enumerate(keys):
        l, k, Lam, mu = key
        plan = couplings.symmetric_power_product_plan(
            [{"descriptor_index": m, "power": k, "input_L": l, "output_L": Lam, "multiplicity_index": mu,
              "component_index": m, "channel_indices": tuple(range(2 * l + 1))} for m in range(2 * Lam + 1)],
            descriptor_count=2 * Lam + 1, channel_count=2 * l + 1, basis_convention="complex_magnetic")
        x = torch.complex(torch.randn(33, 2 * l + 1, dtype=torch.float64, generator=g),
                          torch.randn(33, 2 * l + 1, dtype=torch.float64, generator=g))
        y = symmetric_power_product_plan_contraction(x, plan)
        out[f"k{j}_x"] = x.numpy()
        out[f"k{j}_y"] = y.numpy()
        out[f"k{j}_key"] = np.asarray(key, dtype=np.int64)
    # The reference's pinned shared-monomial fixture (real-tesseral, float64),
    # read as text from its test tree.
    fx = {}
    with open(REF_FIXTURE) as fh:
        for line in fh:
            parts = line.split()
            if not parts or parts[0] == "end":
                continue
            fx[parts[0]] = parts[1:]
    for name in ("monomial_counts", "output_offsets", "coefficient_terms", "coefficient_outputs"):
        out["fx_" + name] = np.asarray([int(v) for v in fx[name][1:]], dtype=np.int64)
    for name in ("coefficient_values", "input", "expected_output", "output_adjoint", "expected_input_adjoint"):
        out["fx_" + name] = np.asarray([float(v) for v in fx[name][1:]], dtype=np.float64)
    for name in ("batch_size", "input_dimension", "monomial_count", "output_dimension"):
        out["fx_" + name] = np.asarray(int(fx[name][0]))
    out["fx_convention_hash"] = np.frombuffer(fx["convention_hash"][0].encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "sympow.npz"), **out)
    print("sympow.npz", len(keys), "kinds + reference fixture", fx["convention_hash"][0])


def load_refcore():
    path = os.path.join(REPO, "oracle", "_ref", "libye3t_refcore.so")
    if not os.path.exists(path):
        raise SystemExit("build the reference core first: make -C oracle ref")
    return ctypes.CDLL(path)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def radial_sh_density_fixture():
    """Radial table (``execution_plan.py:7298``), harmonics (``:7479``) and density (``:7913``)."""
    ref = load_refcore()
    rng = np.random.default_rng(11)
    E = 257
    radii = np.concatenate([rng.uniform(0.0, 6.0, E - 5), [0.0, 5.0, 5.0 - 1e-12, 5.0 + 1e-12, 2.5]])
    rc = np.full(E, 5.0)
    lam = np.full(E, 5.0)
    kmax = 12
    val_t, der_t = cheb_exp_cos_radial_table_with_derivative(torch.tensor(radii), torch.tensor(rc),
                                                             torch.tensor(lam), kmax, backend="reference")
    val_n = np.zeros((E, kmax + 1))
    der_n = np.zeros((E, kmax + 1))
    ref.yr_cheb_exp_cos_radial_table_f64(_p(radii), _p(rc), _p(lam), ctypes.c_int64(E), ctypes.c_int64(kmax),
                                         _p(val_n), _p(der_n), ctypes.c_int(1))
    vec = rng.normal(size=(E, 3)) * rng.uniform(0.2, 5.0, size=(E, 1))
    vec[0] = [0.0, 0.0, 1.3]
    vec[1] = [0.0, 0.0, -0.7]
    vec[2] = [0.0, 0.0, 0.0]
    vec[3] = [1.2, -0.7, 0.5]
    vec[4] = [-0.4, 0.9, 0.0]
    vec[5] = [1e-13, 0.0, 0.0]
    lmax = 4
    W = (lmax + 1) ** 2
    shr_v = np.zeros((E, W)); shr_d = np.zeros((E, W, 3))
    ref.yr_real_spherical_harmonics_table_f64(_p(vec), ctypes.c_int64(E), ctypes.c_int64(lmax), ctypes.c_double(1e-12),
                                              _p(shr_v), _p(shr_d), ctypes.c_int(1))
    shc_v = np.zeros((E, W), dtype=np.complex128); shc_d = np.zeros((E, W, 3), dtype=np.complex128)
    ref.yr_complex_spherical_harmonics_table_f64(_p(vec), ctypes.c_int64(E), ctypes.c_int64(lmax),
                                                 ctypes.c_double(1e-12), _p(shc_v), _p(shc_d), ctypes.c_int(1))
    tv = torch.tensor(vec[6:])
    shc_t, shc_td = spherical_harmonics_table_with_derivative(tv, lmax, real_output=False, backend="reference")
    shr_t, shr_td = spherical_harmonics_table_with_derivative(tv, lmax, real_output=True, backend="reference")
    # density accumulation with the reference test's fixed centres
    # (tests/test_execution_plan_native.py:1521-1540).
    centers = np.asarray([0, 0, 2, 1, 2, 2, 3, 0, 3], dtype=np.int64)
    g = torch.Generator().manual_seed(3)
    ev_r = torch.randn(9, 7, dtype=torch.float64, generator=g)
    ev_c = torch.complex(torch.randn(9, 7, dtype=torch.float64, generator=g),
                         torch.randn(9, 7, dtype=torch.float64, generator=g))
    acc_r = density_accumulate(ev_r, torch.tensor(centers), 4, backend="reference")
    acc_c = density_accumulate(ev_c, torch.tensor(centers), 4, backend="reference")
    np.savez_compressed(os.path.join(HERE, "edge_ops.npz"), radii=radii, rc=rc, lam=lam, kmax=np.asarray(kmax),
                        rad_val_native=val_n, rad_der_native=der_n, rad_val_torch=val_t.detach().numpy(),
                        rad_der_torch=der_t.detach().numpy(), vec=vec, lmax=np.asarray(lmax),
                        shr_val_native=shr_v, shr_der_native=shr_d, shc_val_native=shc_v, shc_der_native=shc_d,
                        shc_val_torch=shc_t.detach().numpy(), shc_der_torch=shc_td.detach().numpy(),
                        shr_val_torch=shr_t.detach().numpy(), shr_der_torch=shr_td.detach().numpy(), centers=centers, ev_r=ev_r.numpy(), ev_c=ev_c.numpy(),
                        acc_r=acc_r.numpy(), acc_c=acc_c.numpy())
    print("edge_ops.npz")


def minimum_image_csr(pos, box, rc):
    N = pos.shape[0]
    d = pos[None, :, :] - pos[:, None, :]
    d -= box * np.round(d / box)
    r2 = (d ** 2).sum(-1)
    mask = (r2 <= rc * rc) & ~np.eye(N, dtype=bool)
    rows, cols = np.nonzero(mask)
    off = np.zeros(N + 1, dtype=np.int64)
    np.add.at(off, rows + 1, 1)
    off = np.cumsum(off)
    return off, cols.astype(np.int32), d[rows, cols]


def ace_fixture():
    """A small periodic system through the reference ops and per-word schedules.

    A-basis: reference radial table x complex harmonics x neighbour-species
    prefactor, accumulated by ``density_accumulate``.  B-basis: for each word,
    ``compile_ace_factorized_schedules_by_L`` on the word itself and the block
    assembly of ``workflows.py:636-661``, evaluated with ``backend="cpp"``.
    """
    N, density, rc, lam, nmax, lmax = 96, 0.05, 5.0, 5.0, 8, 3
    box = (N / density) ** (1.0 / 3.0)
    pos = torch.rand(N, 3, dtype=torch.float64, generator=torch.Generator().manual_seed(0)).numpy() * box
    species = torch.randint(0, 3, (N,), generator=torch.Generator().manual_seed(1)).numpy().astype(np.int32)
    prefactor = np.asarray([1.0, 0.75, 1.25])
    off, nbr, disp = minimum_image_csr(pos, box, rc)
    E = nbr.shape[0]
    r = np.sqrt((disp ** 2).sum(-1))
    Rv, _ = cheb_exp_cos_radial_table_with_derivative(torch.tensor(r), torch.full((E,), rc), torch.full((E,), lam),
                                                       nmax, backend="reference")
    ref = load_refcore()
    W = (lmax + 1) ** 2
    Yv = np.zeros((E, W), dtype=np.complex128); Yd = np.zeros((E, W, 3), dtype=np.complex128)
    ref.yr_complex_spherical_harmonics_table_f64(_p(np.ascontiguousarray(disp)), ctypes.c_int64(E),
                                                 ctypes.c_int64(lmax), ctypes.c_double(1e-12), _p(Yv), _p(Yd),
                                                 ctypes.c_int(1))
    Rv = Rv.detach()
    p = torch.tensor(prefactor[species[nbr]])
    edge = (p[:, None, None] * Rv[:, 1:, None]).to(torch.complex128) * torch.tensor(Yv)[:, None, :]
    centers = torch.tensor(np.repeat(np.arange(N), np.diff(off)))
    A = density_accumulate(edge.reshape(E, -1), centers, N, backend="reference").reshape(N, nmax, W)
    multiplets = {l: A[:, :, l * l:(l + 1) * (l + 1)] for l in range(lmax + 1)}

    def word_features(words):
        feats = []
        for word in words:
            rep = compile_ace_factorized_schedules_by_L(content=tuple(n for _, n in word),
                                                        input_Ls=tuple(l for l, _ in word))
            sched = rep.schedules_by_L[0]
            width = 2 * int(sched.block_L_by_label().max()) + 1
            rows, prepared = [], {}
            for blocks in sched.block_specs:
                row = []
                for block in blocks:
                    key = (block["n"], block["l"], block.get("k_b"), block.get("Lambda"),
                           block.get("multiplicity_index"))
                    if key not in prepared:
                        src = multiplets[block["l"]][..., block["n"] - 1, :]
                        if block["kind"] == "sym":
                            plan = couplings.symmetric_power_product_plan(
                                [{"descriptor_index": m, "power": block["k_b"], "input_L": block["l"],
                                  "output_L": block["Lambda"], "multiplicity_index": block["multiplicity_index"],
                                  "component_index": m, "channel_indices": tuple(range(2 * block["l"] + 1))}
                                 for m in range(2 * block["Lambda"] + 1)],
                                descriptor_count=2 * block["Lambda"] + 1, channel_count=2 * block["l"] + 1,
                                basis_convention="complex_magnetic")
                            src = symmetric_power_product_plan_contraction(src, plan)
                        prepared[key] = torch.nn.functional.pad(src, (0, width - src.shape[-1]))
                    row.append(prepared[key])
                rows.append(torch.stack(row, dim=-2))
            bv = torch.stack(rows, dim=-3)
            feats.append(rep.evaluate(bv, target_L=0, backend="cpp"))
        return torch.cat(feats, dim=1).numpy()

    b3 = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu3_L0.npz"))
    B3 = word_features(b3.words)
    b4 = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu4_L0.npz"))
    sample = np.arange(0, b4.word_count, 23, dtype=np.int64)
    B4 = word_features([b4.words[int(w)] for w in sample])
    rng = np.random.default_rng(2)
    w3 = rng.normal(size=(3, B3.shape[1])) / np.sqrt(B3.shape[1])
    energy3 = float(sum(np.dot(w3[species[i]], B3[i].real) for i in range(N)))
    np.savez_compressed(os.path.join(HERE, "ace_small.npz"), pos=pos, box=np.asarray(box), species=species,
                        prefactor=prefactor, rc=np.asarray(rc), lam=np.asarray(lam), nmax=np.asarray(nmax),
                        lmax=np.asarray(lmax), row_off=off, nbr=nbr, disp=disp, A=A.numpy(), B3=B3[:40],
                        B4=B4[:40], B4_words=sample, w3=w3, energy3=np.asarray(energy3))
    # Features of the first 40 atoms are stored; the energy covers all atoms.
    print("ace_small.npz N", N, "E", E, "B3", B3.shape, "B4", B4.shape, "energy3", energy3)


def _reference_energy_forces(words, weights_of):
    """Total energy and forces of the 96-atom system of ``ace_small.npz`` through the reference's
    differentiable torch ops, for a word list; ``weights_of(F)`` gives the per-species readout
    ``[3, F]`` over the words' L=0 features in order.

    Displacements are the minimum image of the CSR pairs with the image shift
    held fixed; the radial table (``execution_plan.py:6862`` reference
    formula), complex harmonics (``:6919``), ``density_accumulate`` and, per
    word, the symmetric-power contraction and ``evaluate(backend="torch")``
    are all differentiable torch code in the reference.  F = -dE/dr.
    """
    g = dict(np.load(os.path.join(HERE, "ace_small.npz")))
    N = g["pos"].shape[0]
    box = float(g["box"])
    rc, lam, nmax, lmax = float(g["rc"]), float(g["lam"]), int(g["nmax"]), int(g["lmax"])
    off, nbr = g["row_off"], g["nbr"]
    E = nbr.shape[0]
    centers = torch.tensor(np.repeat(np.arange(N), np.diff(off)))
    nbr_t = torch.tensor(nbr, dtype=torch.long)
    pos = torch.tensor(g["pos"], requires_grad=True)
    raw = (pos[nbr_t] - pos[centers]).detach()
    shift = box * torch.round(raw / box)
    disp = pos[nbr_t] - pos[centers] - shift
    r = torch.linalg.norm(disp, dim=-1)
    Rv, _ = cheb_exp_cos_radial_table_with_derivative(r, torch.full((E,), rc, dtype=torch.float64),
                                                       torch.full((E,), lam, dtype=torch.float64), nmax,
                                                       backend="reference")
    Yv, _ = spherical_harmonics_table_with_derivative(disp, lmax, real_output=False, backend="reference")
    p = torch.tensor(g["prefactor"][g["species"][nbr]])
    edge = (p[:, None, None] * Rv[:, 1:, None]).to(torch.complex128) * Yv[:, None, :]
    A = density_accumulate(edge.reshape(E, -1), centers, N, backend="reference").reshape(N, nmax, -1)
    multiplets = {l: A[:, :, l * l:(l + 1) * (l + 1)] for l in range(lmax + 1)}
    feats = []
    for word in words:
        rep = compile_ace_factorized_schedules_by_L(content=tuple(n for _, n in word),
                                                    input_Ls=tuple(l for l, _ in word))
        sched = rep.schedules_by_L[0]
        width = 2 * int(sched.block_L_by_label().max()) + 1
        rows, prepared = [], {}
        for blocks in sched.block_specs:
            row = []
            for block in blocks:
                key = (block["n"], block["l"], block.get("k_b"), block.get("Lambda"), block.get("multiplicity_index"))
                if key not in prepared:
                    src = multiplets[block["l"]][..., block["n"] - 1, :]
                    if block["kind"] == "sym":
                        plan = couplings.symmetric_power_product_plan(
                            [{"descriptor_index": m, "power": block["k_b"], "input_L": block["l"],
                              "output_L": block["Lambda"], "multiplicity_index": block["multiplicity_index"],
                              "component_index": m, "channel_indices": tuple(range(2 * block["l"] + 1))}
                             for m in range(2 * block["Lambda"] + 1)],
                            descriptor_count=2 * block["Lambda"] + 1, channel_count=2 * block["l"] + 1,
                            basis_convention="complex_magnetic")
                        src = symmetric_power_product_plan_contraction(src, plan, backend="reference")
                    prepared[key] = torch.nn.functional.pad(src, (0, width - src.shape[-1]))
                row.append(prepared[key])
            rows.append(torch.stack(row, dim=-2))
        bv = torch.stack(rows, dim=-3)
        feats.append(rep.evaluate(bv, target_L=0, backend="torch"))
    B = torch.cat(feats, dim=1)
    w_all = weights_of(B.shape[1])
    w = torch.tensor(w_all)[torch.tensor(g["species"], dtype=torch.long)]
    energy = (w * B.real).sum()
    (grad,) = torch.autograd.grad(energy, pos)
    return float(energy), (-grad).numpy(), w_all


def forces_fixture():
    """Energy and forces of the 96-atom system (nu <= 3, all 2,344 features) by reference autograd."""
    g = dict(np.load(os.path.join(HERE, "ace_small.npz")))
    b3 = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu3_L0.npz"))
    energy, forces, _ = _reference_energy_forces(b3.words, lambda F: g["w3"])
    np.savez_compressed(os.path.join(HERE, "forces_small.npz"), energy=np.asarray(energy), forces=forces)
    print("forces_small.npz energy", energy, "|F| max", float(np.abs(forces).max()))


def forces_nu4_fixture():
    """Energy and forces of the 96-atom system over every 23rd word of the nu <= 4 set (the C5
    bundle; 1,102 words with four-block words of every adjoint class) by reference autograd, with a
    seeded readout over those words' features (every other feature of the bundle has weight 0)."""
    b4 = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu4_L0.npz"))
    sample = np.arange(0, b4.word_count, 23, dtype=np.int64)
    rng = np.random.default_rng(44)
    energy, forces, w = _reference_energy_forces([b4.words[int(k)] for k in sample],
                                                 lambda F: rng.normal(size=(3, F)) / np.sqrt(F))
    np.savez_compressed(os.path.join(HERE, "forces_nu4.npz"), energy=np.asarray(energy), forces=forces,
                        words=sample, weights=w)
    print("forces_nu4.npz words", sample.shape[0], "energy", energy, "|F| max", float(np.abs(forces).max()))


def mixing_fixture():
    """Radial channel mixing through the reference core, and the mixed A-basis.

    Contraction: random inputs, derivatives and a [output][input] table through
    ``pace_radial_channel_contraction_with_derivative`` (the reference core,
    f64 and f32).  Mixed A-basis (4 species, n_max 12, 8 channels, l_max 4): the
    reference radial table, per edge the contraction with the table of the
    pair (z_i, z_j), the reference complex harmonics and ``density_accumulate``.
    """
    ref = load_refcore()
    rng = np.random.default_rng(5)
    out = {}
    for tag, dt, fn in (("f64", np.float64, ref.yr_pace_radial_channel_contraction_f64),
                        ("f32", np.float32, ref.yr_pace_radial_channel_contraction_f32)):
        P, I, O = 257, 12, 32
        x = rng.normal(size=(P, I)).astype(dt)
        dx = rng.normal(size=(P, I)).astype(dt)
        Wt = (rng.normal(size=(O, I)) / np.sqrt(I)).astype(dt)
        y = np.zeros((P, O), dtype=dt)
        dy = np.zeros((P, O), dtype=dt)
        fn(_p(x), _p(dx), _p(Wt), ctypes.c_int64(P), ctypes.c_int64(I), ctypes.c_int64(O), _p(y), _p(dy))
        out.update({f"c_{tag}_x": x, f"c_{tag}_dx": dx, f"c_{tag}_w": Wt, f"c_{tag}_y": y, f"c_{tag}_dy": dy})
    N, density, rc, lam, nmax, lmax, S, C = 64, 0.05, 5.0, 5.0, 12, 4, 4, 8
    box = (N / density) ** (1.0 / 3.0)
    pos = torch.rand(N, 3, dtype=torch.float64, generator=torch.Generator().manual_seed(0)).numpy() * box
    species = torch.randint(0, S, (N,), generator=torch.Generator().manual_seed(1)).numpy().astype(np.int32)
    mix = torch.randn(S, S, C, nmax, dtype=torch.float64, generator=torch.Generator().manual_seed(2)).numpy()
    mix /= np.sqrt(nmax)
    off, nbr, disp = minimum_image_csr(pos, box, rc)
    E = nbr.shape[0]
    r = np.sqrt((disp ** 2).sum(-1))
    Rv, Rd = cheb_exp_cos_radial_table_with_derivative(torch.tensor(r), torch.full((E,), rc), torch.full((E,), lam),
                                                        nmax, backend="reference")
    Rv = np.ascontiguousarray(Rv.detach().numpy()[:, 1:])
    Rd = np.ascontiguousarray(Rd.detach().numpy()[:, 1:])
    centers = np.repeat(np.arange(N), np.diff(off))
    Rm = np.zeros((E, C))
    scratch = np.zeros((1, C))
    for e in range(E):
        Wp = np.ascontiguousarray(mix[species[centers[e]], species[nbr[e]]])
        ref.yr_pace_radial_channel_contraction_f64(_p(Rv[e:e + 1]), _p(Rd[e:e + 1]), _p(Wp), ctypes.c_int64(1),
                                                   ctypes.c_int64(nmax), ctypes.c_int64(C), _p(Rm[e:e + 1]),
                                                   _p(scratch))
    W = (lmax + 1) ** 2
    Yv = np.zeros((E, W), dtype=np.complex128)
    Yd = np.zeros((E, W, 3), dtype=np.complex128)
    ref.yr_complex_spherical_harmonics_table_f64(_p(np.ascontiguousarray(disp)), ctypes.c_int64(E),
                                                 ctypes.c_int64(lmax), ctypes.c_double(1e-12), _p(Yv), _p(Yd),
                                                 ctypes.c_int(1))
    edge = torch.tensor(Rm)[:, :, None].to(torch.complex128) * torch.tensor(Yv)[:, None, :]
    A = density_accumulate(edge.reshape(E, -1), torch.tensor(centers), N, backend="reference").reshape(N, C, W)
    out.update({"pos": pos, "box": np.asarray(box), "species": species, "mixing": mix, "row_off": off, "nbr": nbr,
                "rc": np.asarray(rc), "lam": np.asarray(lam), "nmax": np.asarray(nmax), "lmax": np.asarray(lmax),
                "A": A.numpy()})
    np.savez_compressed(os.path.join(HERE, "mixing_small.npz"), **out)
    print("mixing_small.npz", N, "atoms", E, "edges", "A norm", float(np.abs(A.numpy()).sum()))


def real_schedules_fixture():
    """Real-tesseral schedules (``generate_real_factorized_coefficient_schedule_for_labels``) of a few
    words and targets, random real blocks and the reference's ``evaluate_real_factorized_schedule_torch``."""
    from ye3t.core.basis import ExactACELabeler
    from ye3t.core.couplings import (evaluate_real_factorized_schedule_torch,
                                     generate_real_factorized_coefficient_schedule_for_labels)
    cases = [((1, 2), (1, 1), 0), ((1, 2, 3), (1, 1, 2), 0), ((1, 1, 2, 3), (2, 2, 1, 3), 0), ((1, 2), (2, 3), 4),
             ((1, 2, 3), (1, 2, 3), 2)]
    out = {"count": np.asarray(len(cases))}
    g = torch.Generator().manual_seed(2040)
    for k, (n_tuple, l_tuple, L) in enumerate(cases):
        labels = ExactACELabeler(list(n_tuple), list(l_tuple), strict_target_validation=False) \
            .compact_labels_for_target(L)
        sch = generate_real_factorized_coefficient_schedule_for_labels(labels, component_indices=range(2 * L + 1))
        ts = sch.to_torch(dtype=torch.float64)
        bv = torch.randn(7, ts.basis_count, ts.block_count, ts.max_block_m_dim, dtype=torch.float64, generator=g)
        y = evaluate_real_factorized_schedule_torch(bv, ts)
        p = f"r{k}_"
        out.update({p + "off": np.asarray(sch.component_offsets, dtype=np.int64),
                    p + "cli": np.asarray(sch.component_label_index, dtype=np.int64),
                    p + "idx": np.asarray(sch.block_real_tuples, dtype=np.int64).reshape(-1, int(sch.block_count)),
                    p + "co": np.asarray(sch.coeffs, dtype=np.float64),
                    p + "bL": np.asarray(sch.block_L_by_label(dtype=np.int64)),
                    p + "basis": np.asarray(int(sch.basis_count)), p + "bv": bv.numpy(), p + "y": y.numpy()})
    np.savez_compressed(os.path.join(HERE, "real_schedules.npz"), **out)
    print("real_schedules.npz", len(cases), "schedules")


def hierarchical_fixture():
    """``block_symmetric_power`` execution plans and the reference module's outputs.

    Plans come from the reference's own test builders (``tests/test_execution_plan.py``,
    ``tests/test_hierarchical_runtime.py``: one to three blocks, schemas v1 and v2, target_L 0
    and 1, up to 1,430 tableaux) and from its scalar-ACE LAMMPS export example
    (``examples/compile_scalar_ace_lammps_plans.py``, ``ye3t/scalar_ace_export.py``: the
    manifest and every exported plan file, ranks 1-8 and 16).  Expected values are
    ``YE3THierarchicalRepeatedBlockModule(plan, backend="reference").forward`` on seeded
    complex block inputs (``ye3t/runtime/hierarchical.py:514``)."""
    import importlib.util
    import tempfile
    sys.path.insert(0, os.path.join(REF_DIR, "tests"))
    import test_execution_plan as te
    import test_hierarchical_runtime as th
    from ye3t.runtime import YE3THierarchicalRepeatedBlockModule

    builders = [("h4", lambda: te._ordinary_homogeneous_scalar_plan(4)), ("r3L1", lambda: th._rank3_plan(1)),
                ("r4", th._ordinary_rank4_plan), ("r6", lambda: th._ordinary_rank6_three_block_case()[0]),
                ("r6u", lambda: th._ordinary_rank6_uneven_three_block_case()[0]), ("r9", th._rank9_plan),
                ("r12", th._rank12_plan), ("r16", th._rank16_plan), ("r32", th._rank32_plan)]
    plans = [(name, build().to_json(), None) for name, build in builders]
    spec = importlib.util.spec_from_file_location(
        "compile_scalar_ace_lammps_plans", os.path.join(ref, "examples", "compile_scalar_ace_lammps_plans.py"))
    example = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(example)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        manifest = example.run_compile_scalar_ace_lammps_plans(
            config={"runtime": {"output_dir": os.path.join(tmp, "plans")}})
        text = open(manifest, encoding="utf-8").read()
        out["lammps_manifest"] = np.asarray(text)
        for case in json.loads(text)["cases"]:
            name = case["execution_plan"]["file"]
            body = open(os.path.join(tmp, "plans", name), encoding="utf-8").read()
            out["lammps_file_" + name] = np.asarray(body)
            plans.append(("lammps_" + case["name"], body, name))
    g = torch.Generator().manual_seed(7319)
    names = []
    for name, js, file in plans:
        module = YE3THierarchicalRepeatedBlockModule(json.loads(js), backend="reference", dtype=torch.complex128)
        inputs = [torch.complex(torch.randn(5, 2 * int(b["input_L"]) + 1, dtype=torch.float64, generator=g),
                                torch.randn(5, 2 * int(b["input_L"]) + 1, dtype=torch.float64, generator=g)) * 0.7
                  for b in module._blocks]
        y = module(*inputs)
        if file is None:
            out["plan_" + name] = np.asarray(js)
        else:  # an exported plan: stored once, under its file name
            out["planfile_" + name] = np.asarray(file)
        for b, x in enumerate(inputs):
            out[f"x{b}_{name}"] = x.numpy()
        out["y_" + name] = y.detach().numpy()
        names.append(name)
    out["names"] = np.asarray(names)
    np.savez_compressed(os.path.join(HERE, "hierarchical.npz"), **out)
    print("hierarchical.npz", len(names), "plans")


def edge_products_fixture():
    """``scheduled_radial_angular_channels_with_derivative`` (execution_plan.py:7675) and
    ``plain_site_basis_product_with_derivative`` (:7582) through the reference's own composition
    (``backend="reference"``) on seeded inputs."""
    from ye3t.runtime.execution_plan import (plain_site_basis_product_with_derivative,
                                             scheduled_radial_angular_channels_with_derivative)
    g = torch.Generator().manual_seed(5150)
    out = {}
    for tag, dt in (("f64", torch.float64), ("f32", torch.float32)):
        E, K, A, C = 37, 9, 16, 20
        d = torch.randn(E, 3, dtype=dt, generator=g)
        d = d / d.norm(dim=1, keepdim=True)
        args = dict(radial_values=torch.randn(E, K, dtype=dt, generator=g),
                    radial_derivatives=torch.randn(E, K, dtype=dt, generator=g),
                    angular_values=torch.randn(E, A, dtype=dt, generator=g),
                    angular_derivatives=torch.randn(E, A, 3, dtype=dt, generator=g), radial_directions=d,
                    edge_types=torch.randint(0, 3, (E,), generator=g),
                    channel_radial_indices=torch.randint(0, K, (C,), generator=g),
                    channel_angular_indices=torch.randint(0, A, (C,), generator=g),
                    channel_types=torch.randint(-1, 3, (C,), generator=g),
                    channel_scales=torch.randn(C, dtype=dt, generator=g))
        v, dv = scheduled_radial_angular_channels_with_derivative(**args, backend="reference")
        for k, x in args.items():
            out[f"s_{tag}_{k}"] = x.numpy()
        out[f"s_{tag}_values"], out[f"s_{tag}_derivatives"] = v.numpy(), dv.numpy()
    for tag, dt in (("f64", torch.float64), ("c128", torch.complex128), ("c64", torch.complex64)):
        G, T, E, C = 3, 10, 29, 14
        rdt = torch.float64 if dt != torch.float32 and dt != torch.complex64 else torch.float32

        def rnd(*shape):
            x = torch.randn(*shape, dtype=rdt, generator=g)
            return torch.complex(x, torch.randn(*shape, dtype=rdt, generator=g)) if dt.is_complex else x
        d = torch.randn(E, 3, dtype=rdt, generator=g)
        d = (d / d.norm(dim=1, keepdim=True)).to(dt)
        channels = torch.randperm(C, generator=g)[:T]
        args = dict(radial_values=rnd(G, E), radial_derivatives=rnd(G, E), angular_values=rnd(T, E),
                    angular_derivatives=rnd(T, E, 3), prefactors=rnd(G, E), prefactor_derivatives_center=rnd(G, E),
                    prefactor_derivatives_neighbor=rnd(G, E), radial_directions=d,
                    term_groups=torch.randint(0, G, (T,), generator=g), term_channels=channels, channel_count=C)
        res = plain_site_basis_product_with_derivative(**args, backend="reference")
        for k, x in args.items():
            out[f"p_{tag}_{k}"] = x.numpy() if torch.is_tensor(x) else np.asarray(x)
        for k, x in zip(("edge_values", "edge_derivatives", "charge_center", "charge_neighbor"), res):
            out[f"p_{tag}_{k}"] = x.numpy()
    np.savez_compressed(os.path.join(HERE, "edge_products.npz"), **out)
    print("edge_products.npz", len(out), "arrays")


def adjoints_fixture():
    """Standalone adjoints through the reference: ``plain_site_basis_product_adjoint``
    (execution_plan.py:7790, ``backend="reference"``) and the input gradient of
    ``symmetric_power_monomial_contraction`` (:11998) by torch autograd, for every symmetric
    block kind of the nu<=4 word set."""
    from ye3t.runtime.execution_plan import plain_site_basis_product_adjoint, symmetric_power_monomial_contraction
    g = torch.Generator().manual_seed(6021)
    out = {}
    for tag, dt in (("f64", torch.float64), ("c128", torch.complex128)):
        G, T, E, C = 3, 10, 29, 14

        def rnd(*shape):
            x = torch.randn(*shape, dtype=torch.float64, generator=g)
            return torch.complex(x, torch.randn(*shape, dtype=torch.float64, generator=g)) if dt.is_complex else x
        d = torch.randn(E, 3, dtype=torch.float64, generator=g)
        d = (d / d.norm(dim=1, keepdim=True)).to(dt)
        args = dict(radial_values=rnd(G, E), radial_derivatives=rnd(G, E), angular_values=rnd(T, E),
                    angular_derivatives=rnd(T, E, 3), prefactors=rnd(G, E), prefactor_derivatives_center=rnd(G, E),
                    prefactor_derivatives_neighbor=rnd(G, E), radial_directions=d, edge_weights=rnd(E),
                    edge_weight_derivatives=rnd(E, 3), term_groups=torch.randint(0, G, (T,), generator=g),
                    term_channels=torch.randperm(C, generator=g)[:T], edge_adjoint=rnd(E, C))
        res = plain_site_basis_product_adjoint(**args, backend="reference")
        for k, x in args.items():
            out[f"pa_{tag}_{k}"] = x.numpy()
        for k, x in zip(("position", "charge_center", "charge_neighbor"), res):
            out[f"pa_{tag}_{k}"] = x.numpy()
    bundle = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu4_L0.npz"))
    for j, key in enumerate(sorted(bundle.sym_tables)):
        t = bundle.sym_tables[key]
        width = t.monomial_counts.shape[1]
        x = torch.complex(torch.randn(33, width, dtype=torch.float64, generator=g),
                          torch.randn(33, width, dtype=torch.float64, generator=g)).requires_grad_(True)
        y = symmetric_power_monomial_contraction(x, torch.as_tensor(t.monomial_counts),
                                                 torch.as_tensor(t.output_offsets), torch.as_tensor(t.output_index),
                                                 torch.as_tensor(t.monomial_value), backend="reference")
        adj = torch.complex(torch.randn(*y.shape, dtype=torch.float64, generator=g),
                            torch.randn(*y.shape, dtype=torch.float64, generator=g))
        (grad,) = torch.autograd.grad(y, x, adj)
        out[f"sp{j}_key"] = np.asarray(key, dtype=np.int64)
        out[f"sp{j}_x"], out[f"sp{j}_adj"], out[f"sp{j}_grad"] = x.detach().numpy(), adj.numpy(), grad.numpy()
    np.savez_compressed(os.path.join(HERE, "adjoints.npz"), **out)
    print("adjoints.npz", len(out), "arrays")


def schedule_grads_fixture():
    """Gradients of the reference's torch schedule evaluator (``evaluate_factorized_schedule_torch``,
    ``core/couplings.py:481-567``, by torch autograd) for the schedules of ``schedules.npz``, complex and
    real block values, on seeded blocks and output adjoints."""
    g = torch.Generator().manual_seed(3141)
    out = {}
    for i, (content, ls, L) in enumerate(SCHEDULE_CASES):
        rep = compile_ace_factorized_schedules_by_L(content=content, input_Ls=ls)
        rec = ScheduleRecord.from_schedule(rep.schedules_by_L[L], rep.convention_hash)
        bl = rec.block_L_by_label()
        mdim = rec.max_block_m_dim
        mask = torch.zeros(rec.basis_count, rec.block_count, mdim, dtype=torch.bool)
        for a in range(rec.basis_count):
            for b in range(rec.block_count):
                mask[a, b, : 2 * bl[a, b] + 1] = True
        shape = (5, rec.basis_count, rec.block_count, mdim)
        re, im = torch.randn(*shape, dtype=torch.float64, generator=g), torch.randn(*shape, dtype=torch.float64,
                                                                                    generator=g)
        for tag, bv in (("c", torch.complex(re, im) * mask), ("r", re * mask)):
            x = bv.clone().requires_grad_(True)
            y = rep.evaluate(x, target_L=L, backend="torch")
            adj = torch.randn(*y.shape, dtype=torch.float64, generator=g)
            if y.is_complex():
                adj = torch.complex(adj, torch.randn(*y.shape, dtype=torch.float64, generator=g))
            (grad,) = torch.autograd.grad(y, x, adj)
            p = f"s{i}_{tag}_"
            out[p + "bv"], out[p + "adj"], out[p + "grad"] = bv.numpy(), adj.numpy(), grad.numpy()
    np.savez_compressed(os.path.join(HERE, "schedule_grads.npz"), **out)
    print("schedule_grads.npz", len(SCHEDULE_CASES), "schedules")


def hierarchical_grads_fixture():
    """Input gradients of ``YE3THierarchicalRepeatedBlockModule(backend="reference")`` by torch
    autograd (``ye3t/runtime/hierarchical.py:514``) for plans of ``hierarchical.npz``, on its
    inputs and seeded output adjoints."""
    from ye3t.runtime import YE3THierarchicalRepeatedBlockModule
    src = np.load(os.path.join(HERE, "hierarchical.npz"))
    g = torch.Generator().manual_seed(8080)
    out = {}
    names = ["h4", "r3L1", "r4", "r6", "r6u", "r9", "r12", "lammps_ta_r04_block_2_2_a1", "lammps_ta_r08_block_4_4_a2"]
    for name in names:
        js = str(src["plan_" + name]) if "plan_" + name in src.files else \
            str(src["lammps_file_" + str(src["planfile_" + name])])
        module = YE3THierarchicalRepeatedBlockModule(json.loads(js), backend="reference", dtype=torch.complex128)
        xs = []
        b = 0
        while f"x{b}_{name}" in src.files:
            xs.append(torch.as_tensor(src[f"x{b}_{name}"]).clone().requires_grad_(True))
            b += 1
        y = module(*xs)
        adj = torch.complex(torch.randn(*y.shape, dtype=torch.float64, generator=g),
                            torch.randn(*y.shape, dtype=torch.float64, generator=g))
        grads = torch.autograd.grad(y, xs, adj)
        out["adj_" + name] = adj.numpy()
        for k, gr in enumerate(grads):
            out[f"g{k}_{name}"] = gr.numpy()
    out["names"] = np.asarray(names)
    np.savez_compressed(os.path.join(HERE, "hierarchical_grads.npz"), **out)
    print("hierarchical_grads.npz", len(names), "plans")


if __name__ == "__main__":
    which = sys.argv[1:] or ["schedules", "quickstart", "sympow", "edge", "ace", "forces", "mixing", "real",
                             "hierarchical", "edge_products", "adjoints", "schedule_grads",
                             "hierarchical_grads", "forces_nu4"]
    if "schedules" in which:
        schedules_fixture()
    if "quickstart" in which:
        quickstart_fixture()
    if "sympow" in which:
        sympow_fixture()
    if "edge" in which:
        radial_sh_density_fixture()
    if "ace" in which:
        ace_fixture()
    if "forces" in which:
        forces_fixture()
    if "mixing" in which:
        mixing_fixture()
    if "real" in which:
        real_schedules_fixture()
    if "hierarchical" in which:
        hierarchical_fixture()
    if "edge_products" in which:
        edge_products_fixture()
    if "adjoints" in which:
        adjoints_fixture()
    if "schedule_grads" in which:
        schedule_grads_fixture()
    if "hierarchical_grads" in which:
        hierarchical_grads_fixture()
    if "forces_nu4" in which:
        forces_nu4_fixture()
