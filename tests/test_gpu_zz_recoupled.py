"""Recoupled B-basis passes (y3b_ace_recoupled_*) on the GPU against the oracle and
against the term-level adjoint kernels."""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_CASES = {}


def _bundle(stem):
    from ye3t_b200.schedules import ACEBundle
    return ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", stem + ".npz"))


def _case(stem):
    """Bundle, plan, five atoms (one of a species outside the weights) and the oracle's results."""
    if stem not in _CASES:
        from oracle import oracle
        from ye3t_b200.recoupling import build_recoupled_plan
        b = _bundle(stem)
        rng = np.random.default_rng(21)
        A = rng.normal(size=(5, 8, 16)) + 1j * rng.normal(size=(5, 8, 16))
        species = np.array([0, 1, 2, 1, 0], dtype=np.int32)
        w = rng.normal(size=(3, b.feature_count)) / np.sqrt(b.feature_count)
        e0, G0 = oracle.bundle_energy_grad(b, A, species, w, threads=4)
        F0 = oracle.bundle_features(b, A, threads=4)
        _CASES[stem] = (b, build_recoupled_plan(b), A, species, w, e0, G0, F0)
    return _CASES[stem]


@pytest.mark.parametrize("stem, na", [("ace_n8_l3_nu3_L0", 1), ("ace_n8_l3_nu4_L0", 1), ("ace_n8_l3_nu4_L0", 2),
                                      ("ace_n8_l3_nu4_L0", 3), ("ace_n8_l3_nu3_L0", 4)])
def test_recoupled_passes_match_oracle(stem, na):
    from ye3t_b200.recoupling import RecoupledEvaluator
    b, plan, A, species, w, e0, G0, F0 = _case(stem)
    ev = RecoupledEvaluator(b, DEV, w, plan=plan, atoms_per_cta=na)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    Ad, sd = torch.as_tensor(A, device=DEV), torch.as_tensor(species, device=DEV)
    F = ev.features(Ad, status=st).cpu().numpy()
    e = ev.energy(Ad, sd, status=st).cpu().numpy()
    e2, G = (x.cpu().numpy() for x in ev.energy_grad(Ad, sd, status=st))
    assert int(st.item()) == 0
    assert np.abs(F - F0).max() <= 1e-12 * np.abs(F0).max()
    assert np.abs(e - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(e2 - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G - G0).max() <= 1e-12 * np.abs(G0).max()


def test_recoupled_adjoint_matches_term_level_adjoint_and_repeats():
    """3,000 atoms through the recoupled adjoint (several CTA shapes) and through the
    term-level adjoint (y3b_ace_energy_grad): same energies and dE/dA to 1e-12, and repeated
    calls are bitwise identical."""
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    from ye3t_b200.recoupling import RecoupledEvaluator
    b, plan, _, _, _, _, _, _ = _case("ace_n8_l3_nu4_L0")
    rng = np.random.default_rng(22)
    n = 3000
    A = torch.as_tensor(rng.normal(size=(n, 8, 16)) + 1j * rng.normal(size=(n, 8, 16)), device=DEV)
    sp = torch.as_tensor(rng.integers(0, 3, n).astype(np.int32), device=DEV)
    w = rng.normal(size=(3, b.feature_count)) / np.sqrt(b.feature_count)
    ref = ACEEvaluator(b, DEV, config=ACEConfig(5.0, 5.0), species_prefactor=[1.0, 0.75, 1.25], weights=w,
                       b_basis="term")
    e0, G0 = ref.energy_grad(A, sp)
    for na, th in ((1, 256), (3, 256), (2, 512)):
        rec = RecoupledEvaluator(b, DEV, w, plan=plan, atoms_per_cta=na, threads_per_cta=th)
        e1, G1 = rec.energy_grad(A, sp)
        e2, G2 = rec.energy_grad(A, sp)
        assert torch.equal(e1, e2) and torch.equal(G1, G2)
        assert float((e1 - e0).abs().max()) <= 1e-12 * float(e0.abs().max())
        assert float((G1 - G0).abs().max()) <= 1e-12 * float(G0.abs().max())
        e3 = rec.energy(A, sp)
        assert float((e3 - e0).abs().max()) <= 1e-12 * float(e0.abs().max())


def test_recoupled_species_out_of_range_sets_status():
    from ye3t_b200 import _native
    from ye3t_b200.recoupling import RecoupledEvaluator
    b, plan, A, _, _, _, _, _ = _case("ace_n8_l3_nu3_L0")
    w = np.random.default_rng(23).normal(size=(2, b.feature_count))
    ev = RecoupledEvaluator(b, DEV, w, plan=plan)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    e, G = ev.energy_grad(torch.as_tensor(A[:3], device=DEV), torch.tensor([0, 5, 1], dtype=torch.int32, device=DEV),
                          status=st)
    assert int(st.item()) & _native.STATUS_INDEX_RANGE
    assert torch.isfinite(e).all() and torch.isfinite(G).all()


def test_symmetric_passes_on_physical_densities(golden):
    """The symmetric passes (M >= 0 only) on densities from y3b_ace_density: against the oracle
    on six atoms of the golden system, and against the general recoupled pass and the
    term-level adjoint on 4,096 atoms of a random periodic system."""
    from oracle import oracle
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    from ye3t_b200.recoupling import RecoupledEvaluator
    b, plan, _, _, _, _, _, _ = _case("ace_n8_l3_nu4_L0")
    g = golden("ace_small")
    A6 = np.ascontiguousarray(np.asarray(g["A"])[:6])
    sp6 = np.asarray(g["species"])[:6].astype(np.int32)
    rng = np.random.default_rng(24)
    w = rng.normal(size=(3, b.feature_count)) / np.sqrt(b.feature_count)
    e0, G0 = oracle.bundle_energy_grad(b, A6, sp6, w, threads=4)
    for na, th in ((1, 256), (4, 256), (3, 512)):
        sym = RecoupledEvaluator(b, DEV, w, plan=plan, atoms_per_cta=na, threads_per_cta=th, symmetric=True)
        st = torch.zeros(1, dtype=torch.int32, device=DEV)
        e1, G1 = (x.cpu().numpy() for x in sym.energy_grad(torch.as_tensor(A6, device=DEV),
                                                            torch.as_tensor(sp6, device=DEV), status=st))
        assert int(st.item()) == 0
        assert np.abs(e1 - e0).max() <= 1e-12 * np.abs(e0).max()
        assert np.abs(G1 - G0).max() <= 1e-12 * np.abs(G0).max()
    n = 4096
    box = (n / 0.05) ** (1.0 / 3.0)
    pos = torch.as_tensor(rng.uniform(0, box, size=(n, 3)), device=DEV)
    sp = torch.as_tensor(rng.integers(0, 3, n).astype(np.int32), device=DEV)
    ev = ACEEvaluator(b, DEV, config=ACEConfig(5.0, 5.0), species_prefactor=[1.0, 0.75, 1.25], weights=w,
                      b_basis="term")
    row, nbr = ev.neighbor_list(pos, box)
    A = ev.density(pos, sp, box, row, nbr)
    et, Gt = ev.energy_grad(A, sp)
    gen = RecoupledEvaluator(b, DEV, w, plan=plan)
    sym = RecoupledEvaluator(b, DEV, w, plan=plan, atoms_per_cta=2, threads_per_cta=512, symmetric=True)
    eg, Gg = gen.energy_grad(A, sp)
    es, Gs = sym.energy_grad(A, sp)
    es2 = sym.energy(A, sp)
    for e, G in ((eg, Gg), (es, Gs)):
        assert float((e - et).abs().max()) <= 1e-12 * float(et.abs().max())
        assert float((G - Gt).abs().max()) <= 1e-12 * float(Gt.abs().max())
    assert float((es2 - et).abs().max()) <= 1e-12 * float(et.abs().max())
    # the dense-tile adjoint on the same densities: both block sizes, species-sorted and
    # index order; bitwise repeatable
    for rows, th, sort in ((8, 256, True), (8, 512, True), (8, 512, False)):
        tiled = RecoupledEvaluator(b, DEV, w, plan=plan, threads_per_cta=th, symmetric=True, tile_rows=rows,
                                   sort_species=sort)
        st = torch.zeros(1, dtype=torch.int32, device=DEV)
        e1, G1 = tiled.energy_grad(A, sp, status=st)
        e2, G2 = tiled.energy_grad(A, sp, status=st)
        assert int(st.item()) == 0
        assert torch.equal(e1, e2) and torch.equal(G1, G2)
        assert float((e1 - et).abs().max()) <= 1e-12 * float(et.abs().max())
        assert float((G1 - Gt).abs().max()) <= 1e-12 * float(Gt.abs().max())
        e6, G6 = (x.cpu().numpy() for x in tiled.energy_grad(torch.as_tensor(A6, device=DEV),
                                                              torch.as_tensor(sp6, device=DEV)))
        assert np.abs(e6 - e0).max() <= 1e-12 * np.abs(e0).max()
        assert np.abs(G6 - G0).max() <= 1e-12 * np.abs(G0).max()

