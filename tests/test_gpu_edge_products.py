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
