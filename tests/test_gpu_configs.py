"""Parity at the benchmark configurations' own sizes.

Each test builds the full system of one configuration on the GPU (C5: 2^20 atoms;
C2: 16,384; C3: 65,536; C4: 32,768), runs the product path over every atom, and
checks a sample of atoms spread through the system against the CPU oracle run on
those atoms' own neighbourhoods (brute-force minimum image in the full box).  The
reference semantics are ``ye3t/workflows.py:636-661`` (block assembly) and
``ye3t/core/couplings.py:481-567`` (schedule evaluation); the oracle restates them
and is pinned to the reference's golden vectors elsewhere (test_oracle_golden.py).

Tolerances: fp64 1e-12 relative (A, energies, dE/dA, features), forces 1e-10;
fp32 1e-5 of the sample's largest feature.
"""

import os

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUTOFF, LAMBDA, DENSITY = 5.0, 5.0, 0.05
THREADS = max(1, min(16, len(os.sched_getaffinity(0))))


def _bundle(stem):
    from ye3t_b200.schedules import ACEBundle
    return ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", stem + ".npz"))


def _system(N, species_count):
    """The benchmark's seeded inputs: uniform positions (seed 0) in a periodic cube at
    0.05 atoms/A^3 and uniform species (seed 1)."""
    box = (N / DENSITY) ** (1.0 / 3.0)
    pos = torch.rand(N, 3, dtype=torch.float64, generator=torch.Generator().manual_seed(0)) * box
    species = torch.randint(0, species_count, (N,), generator=torch.Generator().manual_seed(1)).to(torch.int32)
    return pos.numpy(), species.numpy(), box


def _local_rows(pos, species, box, centres, extra=()):
    """CSR rows of ``centres`` (then of ``extra``) in a local index space: local atoms are the
    centres, the extra centres, then every other neighbour; neighbours within a row sorted by
    global index as the GPU builder sorts them.  Returns (disp, row_off, nbr_local,
    species_local, nbr_global, local_of_global)."""
    rows = list(centres) + [int(i) for i in extra if int(i) not in set(int(c) for c in centres)]
    local = {int(g): k for k, g in enumerate(rows)}
    disp, off, nbr_g = [], [0], []
    for i in rows:
        x = pos - pos[i]
        d = x - box * np.rint(x / box)
        r2 = (d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1]) + d[:, 2] * d[:, 2]
        r2[i] = np.inf
        j = np.nonzero(r2 <= CUTOFF * CUTOFF)[0]
        disp.append(d[j])
        nbr_g.append(j)
        off.append(off[-1] + j.shape[0])
    nbr_g = np.concatenate(nbr_g)
    for j in nbr_g:
        if int(j) not in local:
            local[int(j)] = len(local)
    glob = np.empty(len(local), dtype=np.int64)
    for g, k in local.items():
        glob[k] = g
    nbr_l = np.asarray([local[int(j)] for j in nbr_g], dtype=np.int32)
    return (np.concatenate(disp), np.asarray(off, dtype=np.int64), nbr_l, species[glob].astype(np.int32),
            nbr_g, local)


def _rel(a, b):
    """Largest norm-wise relative error over the rows (atoms)."""
    a = a.reshape(a.shape[0], -1)
    b = b.reshape(b.shape[0], -1)
    return float(np.max(np.linalg.norm(a - b, axis=1) / np.maximum(np.linalg.norm(b, axis=1), 1e-300)))


def test_c5_sampled_atoms_match_oracle():
    """C5 (2^20 atoms, 3 species, n_max 8, l_max 3, nu <= 4, fp64): A, per-atom energies and
    dE/dA of 64 atoms spread through the system, through the recoupled symmetric passes (the
    product default) and the term-level adjoint, and the forces of 3 atoms, against the oracle."""
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    N = 1 << 20
    pos, species, box = _system(N, 3)
    b = _bundle("ace_n8_l3_nu4_L0")
    prefactor = np.asarray([1.0, 0.75, 1.25])
    w = (torch.randn(3, b.feature_count, dtype=torch.float64, generator=torch.Generator().manual_seed(2))
         / b.feature_count ** 0.5).numpy()
    ev = ACEEvaluator(b, DEV, config=ACEConfig(CUTOFF, LAMBDA), species_prefactor=prefactor, weights=w)
    pos_d, sp_d = torch.as_tensor(pos, device=DEV), torch.as_tensor(species, device=DEV)
    row, nbr = ev.neighbor_list(pos_d, box)
    A = ev.density(pos_d, sp_d, box, row, nbr)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    e_rec, G_rec = ev.energy_grad(A, sp_d, status=status, physical=True)
    F_rec = ev.forces_from_edges(row, nbr, ev.edge_grad(pos_d, sp_d, box, row, nbr, G_rec))
    ev.b_basis = "term"
    e_term, G_term = ev.energy_grad(A, sp_d, status=status)
    F_term = ev.forces_from_edges(row, nbr, ev.edge_grad(pos_d, sp_d, box, row, nbr, G_term))
    assert int(status.item()) == 0

    sample = np.linspace(0, N - 1, 64).astype(np.int64)
    disp, off, nbr_l, sp_l, _, _ = _local_rows(pos, species, box, sample)
    A_ref = oracle.ace_density(disp, off, nbr_l, sp_l, prefactor, 8, 3, CUTOFF, LAMBDA)
    e_ref, G_ref = oracle.bundle_energy_grad(b, A_ref, species[sample], w, threads=THREADS)
    A_s = A[torch.as_tensor(sample, device=DEV)].cpu().numpy()
    assert np.abs(A_s - A_ref).max() <= 1e-12 * np.abs(A_ref).max()
    for e, G in ((e_rec, G_rec), (e_term, G_term)):
        e_s = e[torch.as_tensor(sample, device=DEV)].cpu().numpy()
        G_s = G[torch.as_tensor(sample, device=DEV)].cpu().numpy()
        assert np.abs(e_s - e_ref).max() <= 1e-12 * np.abs(e_ref).max()
        assert np.abs(G_s - G_ref).max() <= 1e-12 * np.abs(G_ref).max()

    # forces of 3 atoms: every row that touches them (their own and their neighbours')
    for k in (int(sample[5]), int(sample[31]), int(sample[60])):
        _, _, _, _, nb_k, _ = _local_rows(pos, species, box, [k])
        disp, off, nbr_l, sp_l, nbr_g, local = _local_rows(pos, species, box, [k], extra=nb_k)
        rows = off.shape[0] - 1
        A_k = oracle.ace_density(disp, off, nbr_l, sp_l, prefactor, 8, 3, CUTOFF, LAMBDA)
        _, G_k = oracle.bundle_energy_grad(b, A_k, sp_l[:rows], w, threads=THREADS)
        g = oracle.ace_edge_grad(disp, off, nbr_l, sp_l, prefactor, 8, 3, CUTOFF, LAMBDA, G_k)
        F_ref = g[off[0]:off[1]].sum(axis=0)  # row of k itself (local row 0)
        F_ref = F_ref - g[nbr_g == k].sum(axis=0)
        for F in (F_rec, F_term):
            got = F[k].cpu().numpy()
            assert np.abs(got - F_ref).max() <= 1e-10 * max(np.abs(F_ref).max(), 1e-300), (k, got, F_ref)


def test_c2_sampled_features_match_oracle():
    """C2 (16,384 atoms, 1 species, nu <= 3, fp64): the 2,344 features of 64 atoms."""
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    N = 16384
    pos, _, box = _system(N, 1)
    species = np.zeros(N, dtype=np.int32)
    b = _bundle("ace_n8_l3_nu3_L0")
    ev = ACEEvaluator(b, DEV, config=ACEConfig(CUTOFF, LAMBDA), species_prefactor=[1.0])
    pos_d, sp_d = torch.as_tensor(pos, device=DEV), torch.as_tensor(species, device=DEV)
    row, nbr = ev.neighbor_list(pos_d, box)
    F = ev.features(ev.density(pos_d, sp_d, box, row, nbr))
    sample = np.linspace(0, N - 1, 64).astype(np.int64)
    disp, off, nbr_l, sp_l, _, _ = _local_rows(pos, species, box, sample)
    A_ref = oracle.ace_density(disp, off, nbr_l, sp_l, np.ones(1), 8, 3, CUTOFF, LAMBDA)
    ref = oracle.bundle_features(b, A_ref, threads=THREADS)
    got = F[torch.as_tensor(sample, device=DEV)].cpu().numpy()
    assert got.shape == (64, 2344)
    assert _rel(got, ref) <= 1e-12


def _channel_case(N, S, nmax, C, lmax, stems, dtype, tol):
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    pos, species, box = _system(N, S)
    mix = (torch.randn(S, S, C, nmax, dtype=torch.float64, generator=torch.Generator().manual_seed(2))
           / nmax ** 0.5).numpy()
    evs = [ACEEvaluator(_bundle(s), DEV, config=ACEConfig(CUTOFF, LAMBDA)) for s in stems]
    pos_d, sp_d = torch.as_tensor(pos, device=DEV), torch.as_tensor(species, device=DEV)
    row, nbr = evs[0].neighbor_list(pos_d, box)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    A = evs[0].density_mixed(pos_d, sp_d, box, row, nbr, torch.as_tensor(mix, dtype=dtype, device=DEV),
                             dtype=dtype, status=status)
    assert int(status.item()) == 0
    sample = np.linspace(0, N - 1, 32).astype(np.int64)
    idx = torch.as_tensor(sample, device=DEV)
    disp, off, nbr_l, sp_l, _, _ = _local_rows(pos, species, box, sample)
    A_ref = oracle.ace_density_mixed(disp, off, nbr_l, sp_l, mix, nmax, lmax, CUTOFF, LAMBDA)
    err = np.abs(A[idx].cpu().numpy().astype(np.complex128) - A_ref).max() / np.abs(A_ref).max()
    assert err <= tol, err
    for ev in evs:
        got = ev.channel_features(A)[idx].cpu().numpy().astype(np.complex128)
        ref = np.concatenate([oracle.bundle_features(ev.bundle, A_ref[:, c:c + 1, :], threads=THREADS)
                              for c in range(C)], axis=1)
        assert got.shape == ref.shape
        err = np.abs(got - ref).max() / np.abs(ref).max()
        assert err <= tol, (ev.bundle.target_L, err)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-12), (torch.float32, 1e-5)])
def test_c3_sampled_channel_features_match_oracle(dtype, tol):
    """C3 (65,536 atoms, 4 species, n_max 12 mixed to 32 channels, l_max 4, nu <= 4
    channel-diagonal words): mixed A and the 2,272 features of 32 atoms, fp64 and fp32."""
    _channel_case(65536, 4, 12, 32, 4, ["ace_diag_l4_nu4_L0"], dtype, tol)


def test_c4_sampled_channel_features_match_oracle():
    """C4 (32,768 atoms, 2 species, n_max 8 mixed to 64 channels, l_max 3, nu <= 3, outputs
    L = 0, 1, 2, fp32): the 13,952 components of 32 atoms."""
    _channel_case(32768, 2, 8, 64, 3, ["ace_diag_l3_nu3_L0", "ace_diag_l3_nu3_L1", "ace_diag_l3_nu3_L2"],
                  torch.float32, 1e-5)
