"""Standalone edge-product operators against the reference's own composition
(``tests/golden/edge_products.npz``, ``backend="reference"``)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"

S_ARGS = ("radial_values", "radial_derivatives", "angular_values", "angular_derivatives", "radial_directions",
          "edge_types", "channel_radial_indices", "channel_angular_indices", "channel_types", "channel_scales")
P_ARGS = ("radial_values", "radial_derivatives", "angular_values", "angular_derivatives", "prefactors",
          "prefactor_derivatives_center", "prefactor_derivatives_neighbor", "radial_directions", "term_groups",
          "term_channels")


@pytest.mark.parametrize("tag", ["f64", "f32"])
def test_scheduled_channels_match_reference(golden, tag):
    from ye3t_b200.runtime import scheduled_radial_angular_channels_with_derivative as op
    g = golden("edge_products")
    v, d = op(*(torch.as_tensor(g[f"s_{tag}_{k}"], device=DEV) for k in S_ARGS))
    if tag == "f64":  # every product and sum rounded as the reference's tensor operations
        assert np.array_equal(v.cpu().numpy(), g["s_f64_values"])
        assert np.array_equal(d.cpu().numpy(), g["s_f64_derivatives"])
    else:
        np.testing.assert_allclose(v.cpu().numpy(), g["s_f32_values"], rtol=2e-6, atol=2e-6)
        np.testing.assert_allclose(d.cpu().numpy(), g["s_f32_derivatives"], rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("tag,tol", [("f64", 1e-13), ("c128", 1e-12), ("c64", 1e-5)])
def test_plain_site_basis_product_matches_reference(golden, tag, tol):
    from ye3t_b200.runtime import plain_site_basis_product_with_derivative as op
    g = golden("edge_products")
    outs = op(*(torch.as_tensor(g[f"p_{tag}_{k}"], device=DEV) for k in P_ARGS), int(g[f"p_{tag}_channel_count"]))
    for name, y in zip(("edge_values", "edge_derivatives", "charge_center", "charge_neighbor"), outs):
        ref = g[f"p_{tag}_{name}"]
        assert y.dtype == torch.as_tensor(ref).dtype
        err = np.abs(y.cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1.0)
        assert err <= tol, (name, err)
        unused = np.setdiff1d(np.arange(ref.shape[1]), g[f"p_{tag}_term_channels"])
        assert np.all(y.cpu().numpy()[:, unused] == 0)


def test_edge_products_reject_bad_indices(golden):
    from ye3t_b200.runtime import (plain_site_basis_product_with_derivative,
                                   scheduled_radial_angular_channels_with_derivative)
    g = golden("edge_products")
    args = [torch.as_tensor(g[f"s_f64_{k}"], device=DEV) for k in S_ARGS]
    args[6] = args[6] + 100  # radial index past the table
    with pytest.raises(IndexError):
        scheduled_radial_angular_channels_with_derivative(*args)
    args = [torch.as_tensor(g[f"p_f64_{k}"], device=DEV) for k in P_ARGS]
    with pytest.raises(IndexError):
        plain_site_basis_product_with_derivative(*args, 3)  # channels beyond a 3-channel output


PA_ARGS = ("radial_values", "radial_derivatives", "angular_values", "angular_derivatives", "prefactors",
           "prefactor_derivatives_center", "prefactor_derivatives_neighbor", "radial_directions", "edge_weights",
           "edge_weight_derivatives", "term_groups", "term_channels", "edge_adjoint")


@pytest.mark.parametrize("tag,tol", [("f64", 1e-13), ("c128", 1e-12)])
def test_plain_site_basis_product_adjoint_matches_reference(golden, tag, tol):
    from ye3t_b200.runtime import plain_site_basis_product_adjoint as op
    g = golden("adjoints")
    outs = op(*(torch.as_tensor(g[f"pa_{tag}_{k}"], device=DEV) for k in PA_ARGS))
    for name, y in zip(("position", "charge_center", "charge_neighbor"), outs):
        ref = g[f"pa_{tag}_{name}"]
        assert tuple(y.shape) == ref.shape
        err = np.abs(y.cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1.0)
        assert err <= tol, (name, err)


def test_symmetric_power_backward_matches_reference_autograd(golden):
    """Every symmetric block kind of the nu<=4 word set: the input gradient of the grouped
    contraction (GPU vector-Jacobian product) against torch autograd through the reference."""
    import os
    from ye3t_b200.runtime import symmetric_power_table_contraction
    from ye3t_b200.schedules import ACEBundle
    g = golden("adjoints")
    b = ACEBundle.load(os.path.join(os.path.dirname(os.path.dirname(__file__)), "ye3t_b200", "bundles",
                                    "ace_n8_l3_nu4_L0.npz"))
    j = 0
    while f"sp{j}_key" in g:
        t = b.sym_tables[tuple(int(v) for v in g[f"sp{j}_key"])]
        x = torch.as_tensor(g[f"sp{j}_x"], device=DEV).requires_grad_(True)
        y = symmetric_power_table_contraction(x, t)
        (grad,) = torch.autograd.grad(y, x, torch.as_tensor(g[f"sp{j}_adj"], device=DEV))
        ref = g[f"sp{j}_grad"]
        err = np.abs(grad.cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1.0)
        assert err <= 1e-12, (j, err)
        j += 1
    assert j == 23
