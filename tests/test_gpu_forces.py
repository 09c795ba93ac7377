"""Force path (B-basis adjoint, edge gradients, reverse-edge gather) against
reference forces from torch autograd through the reference ops."""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bundle(stem):
    from ye3t_b200.schedules import ACEBundle
    return ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", stem + ".npz"))


def _evaluator(small, stem, weights, b_basis="recoupled"):
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    return ACEEvaluator(_bundle(stem), DEV, config=ACEConfig(float(small["rc"]), float(small["lam"])),
                        species_prefactor=small["prefactor"], weights=weights, b_basis=b_basis)


# the B-basis adjoint of the product path (recoupled passes) and the term-level kernels
B_BASES = pytest.mark.parametrize("b_basis", ["recoupled", "term"])


@B_BASES
def test_forces_match_reference_autograd(golden, b_basis):
    small = golden("ace_small")
    ref = golden("forces_small")
    ev = _evaluator(small, "ace_n8_l3_nu3_L0", small["w3"], b_basis)
    pos = torch.as_tensor(small["pos"], device=DEV)
    sp = torch.as_tensor(small["species"], device=DEV)
    E, F = ev.energy_forces(pos, sp, float(small["box"]))
    assert abs(float(E) - float(ref["energy"])) <= 1e-12 * abs(float(ref["energy"]))
    Fr = ref["forces"]
    err = np.abs(F.cpu().numpy() - Fr).max() / np.abs(Fr).max()
    assert err <= 1e-10, err


@B_BASES
def test_forces_nu4_bundle_match_reference_autograd(golden, b_basis):
    """The C5 bundle (nu <= 4, all four adjoint classes) with a readout on every 23rd word
    (1,102 words; every other feature weighted 0): total energy and forces against torch
    autograd through the reference ops on the 96-atom system."""
    small = golden("ace_small")
    ref = golden("forces_nu4")
    bundle = _bundle("ace_n8_l3_nu4_L0")
    offsets = bundle.feature_offsets()
    W = np.zeros((3, bundle.feature_count))
    col = 0
    for w in ref["words"]:
        lo, hi = int(offsets[w]), int(offsets[w + 1])
        W[:, lo:hi] = ref["weights"][:, col:col + hi - lo]
        col += hi - lo
    assert col == ref["weights"].shape[1]
    ev = _evaluator(small, "ace_n8_l3_nu4_L0", W, b_basis)
    pos = torch.as_tensor(small["pos"], device=DEV)
    sp = torch.as_tensor(small["species"], device=DEV)
    E, F = ev.energy_forces(pos, sp, float(small["box"]))
    assert abs(float(E) - float(ref["energy"])) <= 1e-11 * abs(float(ref["energy"]))
    err = np.abs(F.cpu().numpy() - ref["forces"]).max() / np.abs(ref["forces"]).max()
    assert err <= 1e-10, err


@B_BASES
def test_energy_grad_energy_equals_forward_and_gradient_is_exact(golden, b_basis):
    small = golden("ace_small")
    rng = np.random.default_rng(4)
    ev = _evaluator(small, "ace_n8_l3_nu4_L0", rng.normal(size=(3, 41168)) / np.sqrt(41168), b_basis)
    N = 1024
    box = (N / 0.05) ** (1 / 3)
    pos = torch.as_tensor(rng.uniform(0, box, size=(N, 3)), device=DEV)
    sp = torch.as_tensor(rng.integers(0, 3, size=N), device=DEV)
    row, nbr = ev.neighbor_list(pos, box)
    A = ev.density(pos, sp, box, row, nbr)
    e_fwd = ev.energy_from_density(A, sp)
    e_adj, G = ev.energy_grad(A, sp)
    np.testing.assert_allclose(e_adj.cpu().numpy(), e_fwd.cpu().numpy(), rtol=1e-11, atol=1e-12)
    # dE/dA against a central difference along a random complex direction (B is a polynomial in A)
    dA = torch.complex(torch.randn_like(A.real), torch.randn_like(A.real)) * 1e-6
    ep = ev.energy_from_density(A + dA, sp).sum().item()
    em = ev.energy_from_density(A - dA, sp).sum().item()
    lin = (G * dA).real.sum().item()
    assert abs((ep - em) / 2 - lin) <= 1e-6 * abs(lin) + 1e-12


@B_BASES
def test_forces_sum_to_zero_and_match_finite_differences(golden, b_basis):
    small = golden("ace_small")
    rng = np.random.default_rng(5)
    ev = _evaluator(small, "ace_n8_l3_nu4_L0", rng.normal(size=(3, 41168)) / np.sqrt(41168), b_basis)
    N = 512
    box = (N / 0.05) ** (1 / 3)
    pos0 = rng.uniform(0, box, size=(N, 3))
    sp = torch.as_tensor(rng.integers(0, 3, size=N), device=DEV)
    E, F = ev.energy_forces(torch.as_tensor(pos0, device=DEV), sp, box)
    F = F.cpu().numpy()
    assert np.abs(F.sum(0)).max() <= 1e-9 * np.abs(F).max()  # momentum conservation
    h = 1e-5
    for k, ax in ((3, 0), (100, 1), (400, 2)):
        p = pos0.copy()
        p[k, ax] += h
        ep = float(ev.energy_forces(torch.as_tensor(p, device=DEV), sp, box)[0])
        p[k, ax] -= 2 * h
        em = float(ev.energy_forces(torch.as_tensor(p, device=DEV), sp, box)[0])
        fd = -(ep - em) / (2 * h)
        assert abs(fd - F[k, ax]) <= 1e-6 * max(1.0, abs(F[k, ax])), (k, ax, fd, F[k, ax])


def test_partial_forces_sum_to_gather_forces(golden):
    small = golden("ace_small")
    ev = _evaluator(small, "ace_n8_l3_nu3_L0", small["w3"])
    pos = torch.as_tensor(small["pos"], device=DEV)
    sp = torch.as_tensor(small["species"], device=DEV)
    box = float(small["box"])
    _, F = ev.energy_forces(pos, sp, box)
    N = pos.shape[0]
    acc = torch.zeros((N, 3), dtype=torch.float64, device=DEV)
    for b, e in ((0, 40), (40, 96)):  # two atom blocks, as two ranks would
        row, nbr = ev.neighbor_list(pos, box, b, e)
        A = ev.density(pos, sp, box, row, nbr, b)
        _, G = ev.energy_grad(A, sp[b:e])
        g = ev.edge_grad(pos, sp, box, row, nbr, G, begin=b)
        ev.partial_forces_from_edges(row, nbr, g, b, N, out=acc)
    np.testing.assert_allclose(acc.cpu().numpy(), F.cpu().numpy(), rtol=1e-10, atol=1e-12)


@B_BASES
def test_energy_grad_many_ctas_matches_forward_and_repeats(golden, b_basis):
    """Thousands of CTAs (races between loading A and the item walk, or between
    warps adding to G, would show here): the adjoint's energies equal the
    forward kernel's and a second run agrees with the first (bit for bit on the
    recoupled passes, whose sums have a fixed order; the term-level adjoint adds
    gradients with shared-memory atomics, so its repeats may differ in the last
    bits)."""
    small = golden("ace_small")
    rng = np.random.default_rng(11)
    ev = _evaluator(small, "ace_n8_l3_nu4_L0", rng.normal(size=(3, 41168)) / np.sqrt(41168), b_basis)
    N = 8192
    box = (N / 0.05) ** (1 / 3)
    pos = torch.as_tensor(rng.uniform(0, box, size=(N, 3)), device=DEV)
    sp = torch.as_tensor(rng.integers(0, 3, size=N), device=DEV)
    row, nbr = ev.neighbor_list(pos, box)
    A = ev.density(pos, sp, box, row, nbr)
    e_fwd = ev.energy_from_density(A, sp).cpu().numpy()
    e1, G1 = ev.energy_grad(A, sp)
    e2, G2 = ev.energy_grad(A, sp)
    np.testing.assert_allclose(e1.cpu().numpy(), e_fwd, rtol=1e-11, atol=1e-11)
    np.testing.assert_allclose(e2.cpu().numpy(), e_fwd, rtol=1e-11, atol=1e-11)
    scale = G1.abs().max().item()
    assert (G1 - G2).abs().max().item() <= 1e-12 * scale
    if b_basis == "recoupled":
        assert torch.equal(G1, G2) and torch.equal(e1, e2)
    # the symmetric passes on this physical density: the same energies and dE/dA
    e3, G3 = ev.energy_grad(A, sp, physical=True)
    np.testing.assert_allclose(e3.cpu().numpy(), e_fwd, rtol=1e-11, atol=1e-11)
    assert (G3 - G1).abs().max().item() <= 1e-12 * scale


@pytest.mark.parametrize("stem", ["ace_diag_l3_nu3_L0", "ace_diag_l4_nu4_L0"])
def test_energy_grad_single_slot_pool(golden, stem):
    """Channel-diagonal bundles (one radial channel, so one symmetric slot in the pool;
    l_max 4 adds four-block items whose last block of 9 indices exceeds the run path's
    staging windows and must take the general path): energies equal the forward
    kernel's, no status bit is set and G is the derivative of the energy."""
    small = golden("ace_small")
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    b = _bundle(stem)
    rng = np.random.default_rng(5)
    ev = ACEEvaluator(b, DEV, config=ACEConfig(float(small["rc"]), float(small["lam"])),
                      weights=rng.normal(size=(2, b.feature_count)), b_basis="term")
    N = 2048
    W = (b.lmax + 1) ** 2
    A = torch.complex(torch.randn(N, 1, W, dtype=torch.float64, device=DEV),
                      torch.randn(N, 1, W, dtype=torch.float64, device=DEV)) * 0.5
    sp = torch.as_tensor(rng.integers(0, 2, size=N), device=DEV, dtype=torch.int32)
    e_fwd = ev.energy_from_density(A, sp).cpu().numpy()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    e_adj, G = ev.energy_grad(A, sp, status=status)
    assert int(status.item()) == 0
    np.testing.assert_allclose(e_adj.cpu().numpy(), e_fwd, rtol=1e-11, atol=1e-12)
    dA = torch.complex(torch.randn_like(A.real), torch.randn_like(A.real)) * 1e-6
    ep = ev.energy_from_density(A + dA, sp).sum().item()
    em = ev.energy_from_density(A - dA, sp).sum().item()
    lin = (G * dA).real.sum().item()
    assert abs((ep - em) / 2 - lin) <= 1e-6 * abs(lin) + 1e-12


def test_energy_grad_flags_a_run_item_outside_its_bounds(golden):
    """A four-block item whose tables claim a last block longer than the run path's
    7-entry staging window is skipped before any staging access and reported with
    Y3B_STATUS_TABLE; with the table restored the flag stays clear."""
    from ye3t_b200 import _native as nat
    from ye3t_b200.packing import GRAD_CLASSES
    small = golden("ace_small")
    rng = np.random.default_rng(9)
    ev = _evaluator(small, "ace_n8_l3_nu4_L0", rng.normal(size=(3, 41168)) / np.sqrt(41168), "term")
    items, groups = ev.packed.arrays["items"], ev.packed.arrays["groups"]
    P = ev.packed.arrays["phases"].shape[0]
    off = ev.packed.arrays["group_offsets"].cpu().numpy().reshape(GRAD_CLASSES, P + 1)
    pairs = groups[int(off[3, 0]):int(off[3, 1])].cpu().numpy()
    i = int(pairs[pairs[:, 0] >= 0][0, 0])
    N = 64
    A = torch.complex(torch.randn(N, 8, 16, dtype=torch.float64, device=DEV),
                      torch.randn(N, 8, 16, dtype=torch.float64, device=DEV)) * 0.3
    sp = torch.as_tensor(rng.integers(0, 3, size=N), device=DEV, dtype=torch.int32)
    saved = int(items[i, 3])
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    try:
        items[i, 3] = 9
        ev.energy_grad(A, sp, status=status)
        assert int(status.item()) & nat.STATUS_TABLE
    finally:
        items[i, 3] = saved
    status.zero_()
    ev.energy_grad(A, sp, status=status)
    assert int(status.item()) == 0
