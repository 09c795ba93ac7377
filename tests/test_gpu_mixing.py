"""Radial channel mixing (pace_radial_channel_contraction_with_derivative), the
mixed-channel A-basis and channel-diagonal features (configs 3 and 4) against
the reference core and the oracle."""

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


def _evaluator(stem, g):
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    return ACEEvaluator(_bundle(stem), DEV, config=ACEConfig(float(g["rc"]), float(g["lam"])))


def test_contraction_bit_exact_vs_reference_core(golden):
    from ye3t_b200.runtime import pace_radial_channel_contraction_with_derivative as op
    g = golden("mixing_small")
    for tag in ("f64", "f32"):
        x, dx, w = (torch.as_tensor(g[f"c_{tag}_{k}"], device=DEV) for k in ("x", "dx", "w"))
        y, dy = op(x, dx, w)
        assert np.array_equal(y.cpu().numpy(), g[f"c_{tag}_y"])
        assert np.array_equal(dy.cpu().numpy(), g[f"c_{tag}_dy"])


def test_contraction_edge_cases():
    from ye3t_b200 import _native as nat
    from ye3t_b200.runtime import pace_radial_channel_contraction_with_derivative as op
    x = torch.zeros((0, 5), dtype=torch.float64, device=DEV)
    y, dy = op(x, x, torch.ones((3, 5), dtype=torch.float64, device=DEV))
    assert y.shape == (0, 3) and dy.shape == (0, 3)
    with pytest.raises(ValueError):
        op(x, x, torch.ones((0, 5), dtype=torch.float64, device=DEV))
    # the C entry point refuses zero output counts like the reference (std::invalid_argument)
    rc = nat.lib().y3b_radial_channel_contraction(nat.F64, 0, 0, 0, 4, 5, 0, 0, 0, None)
    assert rc != 0


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-12), (torch.float32, 1e-5)])
def test_mixed_density_matches_reference_composition(golden, dtype, tol):
    g = golden("mixing_small")
    ev = _evaluator("ace_diag_l4_nu4_L0", g)
    pos = torch.as_tensor(g["pos"], device=DEV)
    sp = torch.as_tensor(g["species"], device=DEV)
    box = float(g["box"])
    row, nbr = ev.neighbor_list(pos, box)
    assert np.array_equal(row.cpu().numpy(), g["row_off"]) and np.array_equal(nbr.cpu().numpy(), g["nbr"])
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    A = ev.density_mixed(pos, sp, box, row, nbr, g["mixing"], dtype=dtype, status=status)
    assert int(status.item()) == 0
    ref = g["A"]
    err = np.abs(A.cpu().numpy().astype(np.complex128) - ref).max() / np.abs(ref).max()
    assert err <= tol, err


def test_mixed_density_flags_bad_species(golden):
    g = golden("mixing_small")
    ev = _evaluator("ace_diag_l4_nu4_L0", g)
    pos = torch.as_tensor(g["pos"], device=DEV)
    sp = torch.as_tensor(g["species"], device=DEV).clone()
    sp[3] = 7  # outside the 4 species of the mixing table
    box = float(g["box"])
    row, nbr = ev.neighbor_list(pos, box)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    A = ev.density_mixed(pos, sp, box, row, nbr, g["mixing"], status=status)
    assert int(status.item()) & 1
    assert torch.all(A[3] == 0)


def _oracle_channel_features(bundle, A):
    from oracle import oracle
    n, C, W = A.shape
    return np.concatenate([oracle.bundle_features(bundle, A[:, c:c + 1, :], threads=4) for c in range(C)], axis=1)


def test_channel_diagonal_features_config3(golden):
    """l_max 4, nu <= 4 channel-diagonal words on every mixed channel."""
    g = golden("mixing_small")
    ev = _evaluator("ace_diag_l4_nu4_L0", g)
    A = torch.as_tensor(g["A"], device=DEV)
    B = ev.channel_features(A).cpu().numpy()
    ref = _oracle_channel_features(ev.bundle, g["A"])
    assert B.shape == (A.shape[0], A.shape[1] * 71)
    err = np.abs(B - ref).max() / np.abs(ref).max()
    assert err <= 1e-12, err


@pytest.mark.parametrize("stem,count", [("ace_diag_l3_nu3_L0", 13), ("ace_diag_l3_nu3_L1", 60),
                                        ("ace_diag_l3_nu3_L2", 145)])
def test_channel_diagonal_features_config4(golden, stem, count):
    """l_max 3, nu <= 3, outputs L = 0, 1, 2 (all M components) on mixed channels."""
    g = golden("mixing_small")
    ev = _evaluator(stem, g)
    pos = torch.as_tensor(g["pos"], device=DEV)
    sp = torch.as_tensor(g["species"], device=DEV)
    box = float(g["box"])
    row, nbr = ev.neighbor_list(pos, box)
    A = ev.density_mixed(pos, sp, box, row, nbr, g["mixing"])
    B = ev.channel_features(A).cpu().numpy()
    ref = _oracle_channel_features(ev.bundle, A.cpu().numpy())
    assert B.shape == (A.shape[0], A.shape[1] * count)
    err = np.abs(B - ref).max() / np.abs(ref).max()
    assert err <= 1e-12, err


@pytest.mark.parametrize("stem", ["ace_diag_l4_nu4_L0", "ace_diag_l3_nu3_L2"])
def test_channel_diagonal_features_fp32(golden, stem):
    """Mixed density and B-basis evaluated in fp32 against the fp64 oracle (1e-5 of the largest feature)."""
    g = golden("mixing_small")
    ev = _evaluator(stem, g)
    pos = torch.as_tensor(g["pos"], device=DEV)
    sp = torch.as_tensor(g["species"], device=DEV)
    box = float(g["box"])
    row, nbr = ev.neighbor_list(pos, box)
    A64 = ev.density_mixed(pos, sp, box, row, nbr, g["mixing"], dtype=torch.float64)
    A32 = ev.density_mixed(pos, sp, box, row, nbr, g["mixing"], dtype=torch.float32)
    B = ev.channel_features(A32)
    assert B.dtype == torch.complex64
    ref = _oracle_channel_features(ev.bundle, A64.cpu().numpy())
    err = np.abs(B.cpu().numpy().astype(np.complex128) - ref).max() / np.abs(ref).max()
    assert err <= 1e-5, err
