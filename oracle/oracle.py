"""numpy/ctypes face of the CPU oracle.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of bench.py, as the checker or the timed CPU baseline;
never by the ye3t_b200 product path.

``lib()`` loads the restatement (``ye3t_oracle.cpp``, built by ``make`` in this
directory on first use); ``refcore()`` loads the reference's own runtime core
compiled from its sources into ``_ref/`` (absent where the reference tree was
not available at build time); ``refeval()`` imports the reference's compiled
schedule evaluator (factorized_runtime.cpp, a torch extension) built there too.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None
_REFEVAL = None

I64 = ctypes.c_int64
VP = ctypes.c_void_p

_DT = {np.dtype(np.float32): 0, np.dtype(np.float64): 1, np.dtype(np.complex64): 2,
       np.dtype(np.complex128): 3}


def _p(a: np.ndarray):
    return a.ctypes.data_as(VP)


def build() -> str:
    path = os.path.join(HERE, "_build", "libye3t_oracle.so")
    src = os.path.join(HERE, "ye3t_oracle.cpp")
    if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    return path


def lib():
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(build())
        _LIB.yo_neighbor_list_bruteforce.restype = I64
    return _LIB


def refcore() -> Optional[ctypes.CDLL]:
    """The reference core library, or None if it was not built."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libye3t_refcore.so")
        if not os.path.exists(path):
            return None
        _REF = ctypes.CDLL(path)
    return _REF


def refeval():
    """The reference's compiled schedule evaluator (``ye3t_factorized_ref``, whose
    ``evaluate_factorized_schedule_cpu`` is factorized_runtime.cpp:426-548), or None if it
    was not built."""
    global _REFEVAL
    if _REFEVAL is None:
        path = os.path.join(HERE, "_ref", "ye3t_factorized_ref.so")
        if not os.path.exists(path):
            return None
        import importlib.util

        import torch  # noqa: F401  (the extension resolves its libtorch symbols through torch)
        spec = importlib.util.spec_from_file_location("ye3t_factorized_ref", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _REFEVAL = mod
    return _REFEVAL


def _c(a, dtype=None):
    return np.ascontiguousarray(a if dtype is None else np.asarray(a, dtype=dtype))


# -- schedule evaluation (factorized_runtime.cpp:252-287) -------------------
def schedule_evaluate(block_values, component_offsets, component_label_index, block_m_indices, coeffs,
                      component_count=None, threads=1):
    bv = _c(block_values)
    coeffs = _c(coeffs, bv.dtype)
    off = _c(component_offsets, np.int64)
    cli = _c(component_label_index, np.int64)
    midx = _c(block_m_indices, np.int64)
    comps = int(cli.shape[0]) if component_count is None else int(component_count)
    batch, basis, blocks, mdim = bv.shape
    out = np.zeros((batch, comps), dtype=bv.dtype)
    lib().yo_factorized_schedule_evaluate(ctypes.c_int(_DT[bv.dtype]), _p(bv), I64(batch), I64(basis),
                                          I64(blocks), I64(mdim), _p(off), _p(cli), _p(midx), _p(coeffs),
                                          I64(comps), _p(out), ctypes.c_int(threads))
    return out


def schedule_evaluate_record(block_values, record, threads=1):
    """Evaluate a ``ScheduleRecord`` with the reference's dtype rule (couplings.py:508-516)."""
    bv = _c(block_values)
    coeffs = record.coeffs
    if not np.iscomplexobj(bv):
        rc = record.real_coeffs()
        if rc is None:
            bv = bv.astype(np.complex128)
        else:
            coeffs = rc
    return schedule_evaluate(bv, record.component_offsets, record.component_label_index,
                             record.block_m_indices(), np.asarray(coeffs).astype(bv.dtype), threads=threads)


# -- symmetric powers (ye3t_runtime_core.cpp:5279, :5392) -------------------
def symmetric_power_monomial(x, monomial_counts, output_offsets, monomial_values):
    x = _c(x)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    counts = _c(monomial_counts, np.int64)
    off = _c(output_offsets, np.int64).reshape(-1)
    vals = _c(monomial_values, x.dtype).reshape(-1)
    out_dim = off.shape[0] - 1
    out = np.zeros((x2.shape[0], out_dim), dtype=x.dtype)
    lib().yo_symmetric_power_monomial(ctypes.c_int(_DT[x.dtype]), _p(x2), I64(x2.shape[0]), I64(x2.shape[1]),
                                      _p(counts), _p(off), _p(vals), I64(out_dim), _p(out))
    return out.reshape(*lead, out_dim)


def ref_symmetric_power_monomial(x, monomial_counts, output_offsets, monomial_values, threads=1):
    """The reference core's own ``symmetric_power_monomial_forward`` (ye3t_runtime_core.h:1227),
    real fp64, from the ``_ref`` build; the caller checks ``refcore()`` first."""
    x = _c(x, np.float64)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    counts = _c(monomial_counts, np.int64)
    off = _c(output_offsets, np.int64).reshape(-1)
    vals = _c(monomial_values, np.float64).reshape(-1)
    out_dim = off.shape[0] - 1
    out = np.zeros((x2.shape[0], out_dim))
    refcore().yr_symmetric_power_monomial_f64(_p(x2), I64(x2.shape[0]), I64(x2.shape[1]), _p(counts), _p(off),
                                              _p(vals), I64(vals.shape[0]), I64(out_dim), _p(out),
                                              ctypes.c_int(threads))
    return out.reshape(*lead, out_dim)


def ref_schedule_evaluate_record(block_values, record):
    """A ``ScheduleRecord`` through the reference's compiled evaluator
    (``evaluate_factorized_schedule_cpu``, factorized_runtime.cpp:426-548, on torch CPU
    tensors), with the dtype rule of ``schedule_evaluate_record``; the caller checks
    ``refeval()`` first.  The extension runs its batch loop under ``at::parallel_for``, so it
    uses torch's intra-op threads (``torch.set_num_threads``)."""
    import torch
    bv = _c(block_values)
    coeffs = record.coeffs
    if not np.iscomplexobj(bv):
        rc = record.real_coeffs()
        if rc is None:
            bv = bv.astype(np.complex128)
        else:
            coeffs = rc
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    out = refeval().evaluate_factorized_schedule_cpu(
        t(bv), t(np.asarray(record.component_offsets, np.int64)),
        t(np.asarray(record.component_label_index, np.int64)), t(record.block_m_indices()),
        t(np.asarray(coeffs).astype(bv.dtype)), int(record.component_count), False)
    return out.numpy()


def symmetric_power_shared_monomial(x, monomial_counts, output_offsets, coefficient_terms, coefficient_values):
    x = _c(x)
    x2 = x.reshape(-1, x.shape[-1])
    counts = _c(monomial_counts, np.int64).reshape(-1, x.shape[-1])
    off = _c(output_offsets, np.int64).reshape(-1)
    terms = _c(coefficient_terms, np.int64)
    vals = _c(coefficient_values, x.dtype)
    out_dim = off.shape[0] - 1
    out = np.zeros((x2.shape[0], out_dim), dtype=x.dtype)
    lib().yo_symmetric_power_shared_monomial(ctypes.c_int(_DT[x.dtype]), _p(x2), I64(x2.shape[0]),
                                             I64(x2.shape[1]), _p(counts), I64(counts.shape[0]), _p(off),
                                             _p(terms), _p(vals), I64(out_dim), _p(out))
    return out.reshape(*x.shape[:-1], out_dim)


# -- edge tables (ye3t_runtime_core.cpp:320-392, 226-290, 843-948) ---------
def radial_table(radii, cutoffs, lambdas, kmax):
    r = _c(radii)
    rc = _c(np.broadcast_to(cutoffs, r.shape), r.dtype)
    lam = _c(np.broadcast_to(lambdas, r.shape), r.dtype)
    E = r.shape[0]
    val = np.zeros((E, kmax + 1), dtype=r.dtype)
    der = np.zeros((E, kmax + 1), dtype=r.dtype)
    lib().yo_cheb_exp_cos_radial_table(ctypes.c_int(_DT[r.dtype]), _p(r), _p(rc), _p(lam), I64(E), I64(kmax),
                                       _p(val), _p(der))
    return val, der


def sh_table(vectors, lmax, real_output=False, epsilon=1e-12):
    v = _c(vectors)
    E = v.shape[0]
    W = (lmax + 1) ** 2
    dt = v.dtype if real_output else (np.complex128 if v.dtype == np.float64 else np.complex64)
    val = np.zeros((E, W), dtype=dt)
    der = np.zeros((E, W, 3), dtype=dt)
    lib().yo_spherical_harmonics_table(ctypes.c_int(_DT[v.dtype]), _p(v), I64(E), I64(lmax),
                                       ctypes.c_int(int(bool(real_output))), ctypes.c_double(epsilon),
                                       _p(val), _p(der))
    return val, der


def density_accumulate(edge_values, centers, atom_count):
    v = _c(edge_values)
    c = _c(centers, np.int64)
    E = v.shape[0]
    C = int(np.prod(v.shape[1:])) if v.ndim > 1 else 1
    out = np.zeros((atom_count,) + v.shape[1:], dtype=v.dtype)
    lib().yo_density_accumulate(ctypes.c_int(_DT[v.dtype]), _p(v), _p(c), I64(E), I64(C), I64(atom_count), _p(out))
    return out


def density_accumulate_adjoint(atomic_adjoint, centers):
    a = _c(atomic_adjoint)
    c = _c(centers, np.int64)
    C = int(np.prod(a.shape[1:]))
    out = np.zeros((c.shape[0],) + a.shape[1:], dtype=a.dtype)
    lib().yo_density_accumulate_adjoint(ctypes.c_int(_DT[a.dtype]), _p(a), _p(c), I64(c.shape[0]), I64(C), _p(out))
    return out


def neighbor_list(positions, box, cutoff):
    pos = _c(positions, np.float64)
    N = pos.shape[0]
    cap = max(1024, N * 64)
    while True:
        off = np.zeros(N + 1, dtype=np.int64)
        nbr = np.zeros(cap, dtype=np.int32)
        disp = np.zeros((cap, 3), dtype=np.float64)
        E = int(lib().yo_neighbor_list_bruteforce(_p(pos), I64(N), ctypes.c_double(box), ctypes.c_double(cutoff),
                                                  _p(off), _p(nbr), _p(disp), I64(cap)))
        if E >= 0:
            return off, nbr[:E].copy(), disp[:E].copy()
        cap *= 2


def ace_density(disp, row_off, nbr, species, prefactor, nmax, lmax, cutoff, lam):
    disp = _c(disp, np.float64)
    off = _c(row_off, np.int64)
    nbr = _c(nbr, np.int32)
    sp = _c(species, np.int32)
    pf = _c(prefactor, np.float64)
    N = off.shape[0] - 1
    A = np.zeros((N, nmax, (lmax + 1) ** 2), dtype=np.complex128)
    lib().yo_ace_density(_p(disp), _p(off), _p(nbr), _p(sp), _p(pf), I64(N), I64(nmax), I64(lmax),
                         ctypes.c_double(cutoff), ctypes.c_double(lam), _p(A))
    return A


# -- multi-word bundles ------------------------------------------------------
def sym_block_values(bundle, A):
    """``{(n, l, k, Lambda, mu): [N, 2 Lambda + 1]}`` for every symmetric block the bundle uses."""
    out = {}
    for key, table in bundle.sym_tables.items():
        l, k, Lam, mu = key
        for n in range(1, bundle.nmax + 1):
            x = A[:, n - 1, l * l:(l + 1) * (l + 1)]
            out[(n, l, k, Lam, mu)] = symmetric_power_monomial(x, table.monomial_counts, table.output_offsets,
                                                               table.monomial_value.astype(A.dtype))
    return out


def bundle_word_block_values(bundle, w, A, sym=None):
    """Block values ``[N, basis, B, mdim]`` of word ``w``, assembled as in workflows.py:636-661."""
    rec = bundle.word_schedule(w)
    mdim = rec.max_block_m_dim
    N = A.shape[0]
    bv = np.zeros((N, rec.basis_count, rec.block_count, mdim), dtype=A.dtype)
    for a, label in enumerate(rec.block_specs):
        for b, (kind, n, l, k, Lam, mu) in enumerate(label):
            if kind == "sym":
                if sym is not None and (n, l, k, Lam, mu) in sym:
                    src = sym[(n, l, k, Lam, mu)]
                else:
                    t = bundle.sym_tables[(l, k, Lam, mu)]
                    src = symmetric_power_monomial(A[:, n - 1, l * l:(l + 1) * (l + 1)], t.monomial_counts,
                                                   t.output_offsets, t.monomial_value.astype(A.dtype))
            else:
                src = A[:, n - 1, l * l:(l + 1) * (l + 1)]
            bv[:, a, b, :src.shape[1]] = src
    return rec, bv


def bundle_features(bundle, A, words=None, threads=1):
    """Features ``[N, F]`` (words in bundle order, components in schedule order)."""
    sym = sym_block_values(bundle, A)
    outs = []
    for w in (range(bundle.word_count) if words is None else words):
        rec, bv = bundle_word_block_values(bundle, int(w), A, sym)
        outs.append(schedule_evaluate_record(bv, rec, threads=threads))
    return np.concatenate(outs, axis=1)


def bundle_energy(bundle, A, species, weights, threads=1):
    """Per-atom energies ``e_i = sum_f w[z_i, f] Re(B_if)``."""
    B = bundle_features(bundle, A, threads=threads)
    W = np.asarray(weights)[np.asarray(species)]
    return (W * B.real).sum(axis=1)


# -- force path ----------------------------------------------------------------
def schedule_adjoint(block_values, record, gout, threads=1):
    """Holomorphic ``dL/dbv`` of the schedule evaluation given ``gout = dL/dout`` (complex128)."""
    bv = _c(block_values, np.complex128)
    go = _c(gout, np.complex128)
    batch, basis, blocks, mdim = bv.shape
    gbv = np.zeros_like(bv)
    off = _c(record.component_offsets, np.int64)
    lab = _c(record.component_label_index, np.int64)
    mi = _c(record.block_m_indices(), np.int64)
    co = _c(record.coeffs, np.complex128)
    lib().yo_factorized_schedule_adjoint(_p(bv), I64(batch), I64(basis), I64(blocks), I64(mdim), _p(off), _p(lab),
                                         _p(mi), _p(co), I64(go.shape[1]), _p(go), _p(gbv), ctypes.c_int(threads))
    return gbv


def symmetric_power_monomial_adjoint(x, monomial_counts, output_offsets, monomial_values, gout):
    """Holomorphic ``dL/dx`` of :func:`symmetric_power_monomial` given ``gout = dL/dout``."""
    xc = _c(x, np.complex128)
    cnt = _c(monomial_counts, np.int64)
    off = _c(output_offsets, np.int64)
    val = _c(monomial_values, np.complex128)
    go = _c(gout, np.complex128)
    gx = np.zeros_like(xc)
    lib().yo_symmetric_power_monomial_adjoint(_p(xc), I64(xc.shape[0]), I64(xc.shape[1]), _p(cnt), _p(off),
                                              _p(val), I64(go.shape[1]), _p(go), _p(gx))
    return gx


def bundle_energy_grad(bundle, A, species, weights, threads=1):
    """Per-atom energies and the holomorphic ``G = dE/dA`` (E = sum_i w[z_i] . Re(B_i))."""
    A = _c(A, np.complex128)
    N = A.shape[0]
    W = np.asarray(weights, dtype=np.float64)[np.asarray(species)]
    sym = sym_block_values(bundle, A)
    G = np.zeros_like(A)
    gsym = {}
    e = np.zeros(N)
    fo = 0
    for w in range(bundle.word_count):
        rec, bv = bundle_word_block_values(bundle, w, A, sym)
        out = schedule_evaluate_record(bv, rec, threads=threads)
        C = out.shape[1]
        wf = W[:, fo:fo + C]
        e += (wf * out.real).sum(axis=1)
        gbv = schedule_adjoint(bv, rec, wf.astype(np.complex128), threads=threads)
        for a, label in enumerate(rec.block_specs):
            for b, (kind, n, l, k, Lam, mu) in enumerate(label):
                if kind == "sym":
                    key = (n, l, k, Lam, mu)
                    g = gbv[:, a, b, :2 * Lam + 1]
                    gsym[key] = gsym[key] + g if key in gsym else g.copy()
                else:
                    G[:, n - 1, l * l:(l + 1) * (l + 1)] += gbv[:, a, b, :2 * l + 1]
        fo += C
    for (n, l, k, Lam, mu), g in gsym.items():
        t = bundle.sym_tables[(l, k, Lam, mu)]
        G[:, n - 1, l * l:(l + 1) * (l + 1)] += symmetric_power_monomial_adjoint(
            A[:, n - 1, l * l:(l + 1) * (l + 1)], t.monomial_counts, t.output_offsets,
            t.monomial_value.astype(np.complex128), g)
    return e, G


def ace_edge_grad(disp, row_off, nbr, species, prefactor, nmax, lmax, cutoff, lam, G):
    """``g_e = dE_i/dd_e`` [E, 3] for the CSR rows, from ``G = dE/dA``."""
    disp = _c(disp, np.float64)
    off = _c(row_off, np.int64)
    nb = _c(nbr, np.int32)
    sp = _c(species, np.int32)
    pf = _c(prefactor, np.float64)
    Gc = _c(G, np.complex128)
    g = np.zeros((nb.shape[0], 3))
    lib().yo_ace_edge_grad(_p(disp), _p(off), _p(nb), _p(sp), _p(pf), I64(off.shape[0] - 1), I64(nmax), I64(lmax),
                           ctypes.c_double(cutoff), ctypes.c_double(lam), _p(Gc), _p(g))
    return g


def forces_from_edges(row_off, nbr, g):
    """``F = -dE/dr`` from per-edge gradients of a full (all-centre) CSR list."""
    off = _c(row_off, np.int64)
    nb = _c(nbr, np.int32)
    gg = _c(g, np.float64)
    N = off.shape[0] - 1
    F = np.zeros((N, 3))
    lib().yo_forces_from_edges(_p(off), _p(nb), I64(N), _p(gg), _p(F))
    return F


def energy_forces(bundle, positions, box, species, prefactor, weights, cutoff, lam, threads=1):
    """Total energy and forces of a periodic system (brute-force neighbour list)."""
    off, nbr, disp = neighbor_list(positions, box, cutoff)
    A = ace_density(disp, off, nbr, species, prefactor, bundle.nmax, bundle.lmax, cutoff, lam)
    e, G = bundle_energy_grad(bundle, A, species, weights, threads=threads)
    g = ace_edge_grad(disp, off, nbr, species, prefactor, bundle.nmax, bundle.lmax, cutoff, lam, G)
    return float(e.sum()), forces_from_edges(off, nbr, g)


# -- radial channel mixing ------------------------------------------------------
def radial_channel_contraction(values, derivatives, coefficients):
    """``(values @ W.T, derivatives @ W.T)`` in input order (ye3t_runtime_core.cpp:651); f32 or f64."""
    x = _c(values)
    dt = x.dtype
    dx = _c(derivatives, dt)
    W = _c(coefficients, dt)
    P, I = x.shape
    O = W.shape[0]
    out = np.zeros((P, O), dtype=dt)
    dout = np.zeros((P, O), dtype=dt)
    lib().yo_radial_channel_contraction(ctypes.c_int(0 if dt == np.float32 else 1), _p(x), _p(dx), _p(W), I64(P),
                                        I64(I), I64(O), _p(out), _p(dout))
    return out, dout


def ace_density_mixed(disp, row_off, nbr, species, mixing, nmax, lmax, cutoff, lam):
    """A-basis ``[N, C, (lmax+1)^2]`` complex128 with channels mixed by ``mixing [S, S, C, nmax]``."""
    disp = _c(disp, np.float64)
    off = _c(row_off, np.int64)
    nb = _c(nbr, np.int32)
    sp = _c(species, np.int32)
    W = _c(mixing, np.float64)
    S, _, C, _ = W.shape
    N = off.shape[0] - 1
    A = np.zeros((N, C, (lmax + 1) ** 2), dtype=np.complex128)
    lib().yo_ace_density_mixed(_p(disp), _p(off), _p(nb), _p(sp), _p(W), I64(N), I64(S), I64(C), I64(nmax),
                               I64(lmax), ctypes.c_double(cutoff), ctypes.c_double(lam), _p(A))
    return A


# -- edge products (ye3t/runtime/execution_plan.py:7036-7220), numpy ------------------------
def scheduled_radial_angular_channels(rv, rd, av, ad, directions, edge_types, ch_rad, ch_ang, ch_type, ch_scale):
    """``_scheduled_radial_angular_channels_reference`` (execution_plan.py:7036-7080):
    values [E, C] and derivatives [E, C, 3], each elementwise operation rounded on its own."""
    R, dR = rv[:, ch_rad], rd[:, ch_rad]
    Y, dY = av[:, ch_ang], ad[:, ch_ang]
    active = ((ch_type < 0)[None, :] | (edge_types[:, None] == ch_type[None, :])).astype(rv.dtype)
    scale = active * ch_scale[None, :]
    values = R * Y * scale
    derivatives = scale[..., None] * (dR[..., None] * directions[:, None, :] * Y[..., None] + R[..., None] * dY)
    return values, derivatives


def _plain_terms(rv, rd, av, ad, pref, directions, groups):
    R, dR, P = rv[groups], rd[groups], pref[groups]
    values = P * R * av
    derivatives = P[..., None] * (dR[..., None] * directions[None, :, :] * av[..., None] + R[..., None] * ad)
    return R, values, derivatives


def plain_site_basis_product(rv, rd, av, ad, pref, pc, pn, directions, groups, channels, channel_count):
    """``_plain_site_basis_product_reference`` (execution_plan.py:7082-7155): edge values and
    derivatives per channel, and the two prefactor-derivative channels."""
    E = rv.shape[1]
    R, tv, td = _plain_terms(rv, rd, av, ad, pref, directions, groups)
    common = R * av
    out = [np.zeros((E, channel_count), dtype=rv.dtype), np.zeros((E, channel_count, 3), dtype=rv.dtype),
           np.zeros((E, channel_count), dtype=rv.dtype), np.zeros((E, channel_count), dtype=rv.dtype)]
    out[0][:, channels] = tv.T
    out[1][:, channels] = np.transpose(td, (1, 0, 2))
    out[2][:, channels] = (pc[groups] * common).T
    out[3][:, channels] = (pn[groups] * common).T
    return tuple(out)


def plain_site_basis_product_adjoint(rv, rd, av, ad, pref, pc, pn, directions, w, dw, groups, channels, adj):
    """``_plain_site_basis_product_adjoint_reference`` (execution_plan.py:7158-7220): the edge
    position adjoint [E, 3] and the two charge adjoints [E]."""
    R, tv, td = _plain_terms(rv, rd, av, ad, pref, directions, groups)
    a = adj[:, channels].T
    weighted = td * w[None, :, None] + tv[..., None] * dw[None, :, :]
    position = (a[..., None] * weighted).sum(axis=0)
    common = R * av * w[None, :]
    return position, (a * pc[groups] * common).sum(axis=0), (a * pn[groups] * common).sum(axis=0)
