"""Hierarchical repeated-block plans on the GPU (symmetric-power kernel, then
the factorized-schedule kernel) against the reference module's outputs."""

import json
import os

import numpy as np
import pytest
import torch

from ye3t_b200.hierarchical import YE3THierarchicalRepeatedBlockModule, load_scalar_ace_plans

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _text(g, name):
    if "plan_" + name in g:
        return str(g["plan_" + name])
    return str(g["lammps_file_" + str(g["planfile_" + name])])


def _inputs(g, name, dtype=torch.complex128):
    xs, b = [], 0
    while f"x{b}_{name}" in g:
        xs.append(torch.as_tensor(g[f"x{b}_{name}"], device=DEV).to(dtype))
        b += 1
    return xs


@pytest.mark.parametrize("dtype,tol", [(torch.complex128, 1e-12), (torch.complex64, 2e-4)])
def test_forward_matches_reference_module(golden, dtype, tol):
    g = golden("hierarchical")
    for name in map(str, g["names"]):
        module = YE3THierarchicalRepeatedBlockModule(_text(g, name), dtype=dtype, device=DEV)
        y = module(*_inputs(g, name, dtype))
        ref = g["y_" + name]
        assert tuple(y.shape) == ref.shape, name
        assert y.dtype == dtype
        err = np.abs(y.cpu().numpy().astype(np.complex128) - ref).max() / max(np.abs(ref).max(), 1.0)
        assert err <= tol, (name, err)
        assert module.runtime_report()["last_backend"] == "cuda_symmetric_power_then_factorized_schedule"


def test_scalar_ace_manifest_modules(golden, tmp_path):
    """The reference's LAMMPS export, loaded from disk: every coordinate as exported."""
    g = golden("hierarchical")
    manifest = json.loads(str(g["lammps_manifest"]))
    for case in manifest["cases"]:
        name = case["execution_plan"]["file"]
        (tmp_path / name).write_text(str(g["lammps_file_" + name]), encoding="utf-8")
    (tmp_path / "manifest.json").write_text(str(g["lammps_manifest"]), encoding="utf-8")
    modules = load_scalar_ace_plans(os.fspath(tmp_path / "manifest.json"), device=DEV)
    assert list(modules) == [c["name"] for c in manifest["cases"]]
    for name, module in modules.items():
        key = "lammps_" + name
        y = module.forward_flat(*_inputs(g, key))
        ref = g["y_" + key].reshape(y.shape[0], -1)
        assert np.abs(y.cpu().numpy() - ref).max() <= 1e-12 * max(np.abs(ref).max(), 1.0), name


def test_linear_readout_and_input_checks(golden):
    g = golden("hierarchical")
    module = YE3THierarchicalRepeatedBlockModule(_text(g, "r12"), device=DEV)
    xs = _inputs(g, "r12")
    feats = module.forward_flat(*xs)
    w = torch.randn(module.output_dimension, dtype=torch.complex128, device=DEV)
    out = module.linear_readout(xs, w, 0.5)
    torch.testing.assert_close(out, feats @ w + 0.5)
    with pytest.raises(ValueError, match="width"):
        module.linear_readout(xs, w[:-1], 0.0)
    with pytest.raises(ValueError, match="block count"):
        module(xs[0])
    with pytest.raises(ValueError, match="multiplet width"):
        module(xs[0][:, :2], xs[1])
    with pytest.raises(ValueError, match="complex dtype"):
        YE3THierarchicalRepeatedBlockModule(_text(g, "r12"), dtype=torch.float64, device=DEV)
    # unbatched inputs keep the reference's shapes
    y = module(xs[0][0], xs[1][0])
    assert tuple(y.shape) == (module.channel_count, module.tableau_count, module.magnetic_count)


def test_input_gradients_match_reference_autograd(golden):
    """First-order autograd through the module (the symmetric-power and schedule
    vector-Jacobian products on the GPU) against the reference module's autograd."""
    g = golden("hierarchical")
    gg = golden("hierarchical_grads")
    for name in map(str, gg["names"]):
        module = YE3THierarchicalRepeatedBlockModule(_text(g, name), device=DEV)
        xs = [x.requires_grad_(True) for x in _inputs(g, name)]
        y = module(*xs)
        grads = torch.autograd.grad(y, xs, torch.as_tensor(gg["adj_" + name], device=DEV))
        for k, gr in enumerate(grads):
            ref = gg[f"g{k}_{name}"]
            err = np.abs(gr.cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1.0)
            assert err <= 1e-12, (name, k, err)
