"""Fused ACE path (neighbour list, A-basis, on-chip symmetric blocks, bundle) against the
reference golden vectors and the oracle."""

import os

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bundle(stem):
    from ye3t_b200.schedules import ACEBundle
    return ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", stem + ".npz"))


@pytest.fixture(scope="module")
def small(golden):
    return golden("ace_small")


@pytest.fixture(scope="module")
def ev3(small):
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    return ACEEvaluator(_bundle("ace_n8_l3_nu3_L0"), DEV, config=ACEConfig(float(small["rc"]), float(small["lam"])),
                        species_prefactor=small["prefactor"], weights=small["w3"])


@pytest.fixture(scope="module")
def ev4(small):
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    rng = np.random.default_rng(4)
    b = _bundle("ace_n8_l3_nu4_L0")
    w = rng.normal(size=(3, 41168)) / np.sqrt(41168)
    return ACEEvaluator(b, DEV, config=ACEConfig(float(small["rc"]), float(small["lam"])),
                        species_prefactor=small["prefactor"], weights=w)


def _rel(a, b):
    return float(np.max(np.linalg.norm(a - b, axis=-1) / np.maximum(np.linalg.norm(b, axis=-1), 1e-300)))


def test_neighbor_list_bit_exact(small, ev3):
    pos = torch.as_tensor(small["pos"], device=DEV)
    row, nbr = ev3.neighbor_list(pos, float(small["box"]))
    np.testing.assert_array_equal(row.cpu().numpy(), small["row_off"])
    np.testing.assert_array_equal(nbr.cpu().numpy(), small["nbr"])


@pytest.mark.parametrize("N,begin,end", [(3000, 0, 3000), (3000, 1000, 2200), (40, 0, 40)])
def test_neighbor_list_matches_oracle(ev3, N, begin, end):
    rng = np.random.default_rng(N + begin)
    box = (N / 0.05) ** (1 / 3) if N > 100 else 9.0  # 9 A box: fewer than 3 cells per side
    pos = rng.uniform(0, box, size=(N, 3))
    off, nbr, _ = oracle.neighbor_list(pos, box, 5.0)
    row, got = ev3.neighbor_list(torch.as_tensor(pos, device=DEV), box, begin, end)
    ref_rows = off[begin:end + 1] - off[begin]
    np.testing.assert_array_equal(row.cpu().numpy(), ref_rows)
    np.testing.assert_array_equal(got.cpu().numpy(), nbr[off[begin]:off[end]])


def test_neighbor_list_slab_windows_match_full_build(ev3):
    """Atoms in cell order, four atom blocks: each block's rows built from its slab window
    (plus halo) with a capacity-sized neighbour array equal the full build bit for bit; a
    window one layer short flags the centres outside it, and a capacity one short flags the
    overflow."""
    import sys
    from ye3t_b200 import _native as nat
    sys.path.insert(0, REPO)
    import bench
    N = 20000
    box = (N / 0.05) ** (1 / 3)
    pos = np.random.default_rng(77).uniform(0, box, size=(N, 3))
    pos = pos[bench.cell_order(pos, box, 5.0)]
    pd = torch.as_tensor(pos, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for r in range(4):
        b, e = (N * r) // 4, (N * (r + 1)) // 4
        win = ev3.slab_window(pos, box, b, e)
        assert win is not None and win[1] < int(nat.lib().y3b_neighbor_cells_per_side(box, 5.0))
        row0, nbr0 = ev3.neighbor_list(pd, box, b, e)
        row1, nbr1 = ev3.neighbor_list(pd, box, b, e, z_window=win, capacity=nbr0.shape[0] + 100, status=status)
        assert int(status.item()) == 0
        assert torch.equal(row0, row1)
        assert torch.equal(nbr0, nbr1[:nbr0.shape[0]])
    short = (win[0] + 1, win[1] - 1)
    ev3.neighbor_list(pd, box, b, e, z_window=short, capacity=nbr0.shape[0], status=status)
    assert int(status.item()) & nat.STATUS_INDEX_RANGE
    status.zero_()
    ev3.neighbor_list(pd, box, b, e, z_window=win, capacity=nbr0.shape[0] - 1, status=status)
    assert int(status.item()) & nat.STATUS_CAPACITY


def test_density_matches_reference(small, ev3):
    pos = torch.as_tensor(small["pos"], device=DEV)
    sp = torch.as_tensor(small["species"], device=DEV)
    row, nbr = ev3.neighbor_list(pos, float(small["box"]))
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    A = ev3.density(pos, sp, float(small["box"]), row, nbr, status=status).cpu().numpy()
    assert int(status.item()) == 0
    ref = small["A"]
    assert np.max(np.abs(A - ref)) <= 1e-12 * np.max(np.abs(ref))
    # an atom block in the middle of the system
    row2, nbr2 = ev3.neighbor_list(pos, float(small["box"]), 30, 70)
    A2 = ev3.density(pos, sp, float(small["box"]), row2, nbr2, begin=30).cpu().numpy()
    assert np.max(np.abs(A2 - ref[30:70])) <= 1e-12 * np.max(np.abs(ref))


def test_features_match_reference(small, ev3, ev4):
    A = torch.as_tensor(small["A"], device=DEV)
    B3 = ev3.features(A).cpu().numpy()
    assert _rel(B3[:40], small["B3"]) <= 1e-12
    B4 = ev4.features(A[:40]).cpu().numpy()
    fo = ev4.bundle.feature_offsets()
    cols = np.concatenate([np.arange(fo[w], fo[w + 1]) for w in small["B4_words"]])
    assert _rel(B4[:, cols], small["B4"]) <= 1e-12


def test_energy_matches_reference(small, ev3):
    pos = torch.as_tensor(small["pos"], device=DEV)
    sp = torch.as_tensor(small["species"], device=DEV)
    e = ev3.energy(pos, sp, float(small["box"])).sum().item()
    assert abs(e - float(small["energy3"])) <= 1e-12 * abs(float(small["energy3"]))


def test_energy_equals_readout_of_features_nu4(ev4):
    # size-independent property at a larger size: energy mode == readout of features mode
    rng = np.random.default_rng(7)
    N = 1536
    box = (N / 0.05) ** (1 / 3)
    pos = torch.as_tensor(rng.uniform(0, box, size=(N, 3)), device=DEV)
    sp = torch.as_tensor(rng.integers(0, 3, size=N), device=DEV)
    row, nbr = ev4.neighbor_list(pos, box)
    A = ev4.density(pos, sp, box, row, nbr)
    e = ev4.energy_from_density(A, sp)
    sel = torch.arange(0, N, 61, device=DEV)
    Bs = ev4.features(A[sel])
    e_ref = (ev4.weights[sp[sel].long()] * Bs.real).sum(1)
    np.testing.assert_allclose(e[sel].cpu().numpy(), e_ref.cpu().numpy(), rtol=1e-11, atol=1e-12)
    # against the oracle on a few atoms
    A_np = A[sel[:4]].cpu().numpy()
    ref = oracle.bundle_energy(ev4.bundle, A_np, sp[sel[:4]].cpu().numpy(), ev4.weights.cpu().numpy(), threads=4)
    np.testing.assert_allclose(e[sel[:4]].cpu().numpy(), ref, rtol=1e-11, atol=1e-12)


def test_isolated_atom_and_rotation_invariance(ev3):
    # a small cluster in a large box: rotating it leaves L = 0 features unchanged
    rng = np.random.default_rng(3)
    pts = rng.normal(size=(12, 3)) * 1.8
    box = 60.0
    theta = 0.7
    R = np.array([[np.cos(theta), -np.sin(theta), 0], [np.sin(theta), np.cos(theta), 0], [0, 0, 1]])
    axis = np.array([1.0, 2.0, -0.5]) / np.linalg.norm([1.0, 2.0, -0.5])
    K = np.array([[0, -axis[2], axis[1]], [axis[2], 0, -axis[0]], [-axis[1], axis[0], 0]])
    R2 = np.eye(3) + np.sin(0.4) * K + (1 - np.cos(0.4)) * K @ K
    pos_a = pts + 30.0
    pos_b = pts @ (R2 @ R).T + 30.0
    pos_a = np.vstack([pos_a, [[5.0, 5.0, 5.0]]])  # isolated atom (no neighbours)
    pos_b = np.vstack([pos_b, [[5.0, 5.0, 5.0]]])
    sp = torch.as_tensor(rng.integers(0, 3, size=13), device=DEV)
    feats = []
    for pos in (pos_a, pos_b):
        p = torch.as_tensor(pos, device=DEV)
        row, nbr = ev3.neighbor_list(p, box)
        A = ev3.density(p, sp, box, row, nbr)
        feats.append(ev3.features(A).cpu().numpy())
    assert np.all(feats[0][12] == 0)
    assert _rel(feats[1][:12], feats[0][:12]) <= 1e-10
