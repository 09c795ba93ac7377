"""Standalone CUDA operators against the reference golden vectors and the oracle."""

import json

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


def _t(a):
    return torch.as_tensor(np.ascontiguousarray(a)).to(DEV)


def test_radial_table_matches_reference(golden):
    from ye3t_b200.runtime import cheb_exp_cos_radial_table_with_derivative as radial
    g = golden("edge_ops")
    v, d = radial(_t(g["radii"]), _t(g["rc"]), _t(g["lam"]), int(g["kmax"]))
    np.testing.assert_allclose(v.cpu().numpy(), g["rad_val_native"], rtol=2e-13, atol=2e-13)
    np.testing.assert_allclose(d.cpu().numpy(), g["rad_der_native"], rtol=2e-12, atol=2e-12)
    v32, _ = radial(_t(g["radii"].astype(np.float32)), 5.0, 5.0, int(g["kmax"]))
    # radii within fp32 rounding of the cutoff can land on the other side of it
    ok = np.abs(g["radii"] - 5.0) > 1e-5
    np.testing.assert_allclose(v32.cpu().numpy()[ok], g["rad_val_native"][ok], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("real_output", [True, False])
def test_spherical_table_matches_reference(golden, real_output):
    from ye3t_b200.runtime import spherical_harmonics_table_with_derivative as sh
    g = golden("edge_ops")
    lmax = int(g["lmax"])
    v, d = sh(_t(g["vec"]), lmax, real_output=real_output)
    tag = "shr" if real_output else "shc"
    np.testing.assert_allclose(v.cpu().numpy(), g[f"{tag}_val_native"], rtol=2e-12, atol=2e-12)
    np.testing.assert_allclose(d.cpu().numpy(), g[f"{tag}_der_native"], rtol=2e-11, atol=2e-11)
    v32, d32 = sh(_t(g["vec"].astype(np.float32)), lmax, real_output=real_output)
    ok = np.abs(g["vec"]).sum(1) > 1e-6  # fp32 epsilon regime differs for the ~0 vectors
    np.testing.assert_allclose(v32.cpu().numpy()[ok], g[f"{tag}_val_native"][ok], rtol=1e-5, atol=2e-5)


def test_density_accumulate_matches_reference(golden):
    from ye3t_b200.runtime import density_accumulate, density_accumulate_adjoint
    g = golden("edge_ops")
    for key in ("r", "c"):
        out = density_accumulate(_t(g[f"ev_{key}"]), _t(g["centers"]), 4, validate=True)
        np.testing.assert_allclose(out.cpu().numpy(), g[f"acc_{key}"], rtol=0, atol=1e-12)
    adj = density_accumulate_adjoint(_t(g["acc_c"]), _t(g["centers"]))
    np.testing.assert_array_equal(adj.cpu().numpy(), g["acc_c"][g["centers"]])


def test_density_accumulate_edge_cases_and_determinism():
    from ye3t_b200.runtime import density_accumulate
    rng = np.random.default_rng(1)
    # empty edges, isolated atoms, one huge row, unsorted centres
    out = density_accumulate(torch.zeros((0, 5), dtype=torch.float64, device=DEV),
                             torch.zeros(0, dtype=torch.int64, device=DEV), 3)
    assert out.shape == (3, 5) and float(out.abs().sum()) == 0.0
    E, N, C = 20000, 300, 37
    centers = rng.integers(0, N, size=E)
    centers[:5000] = 7  # one long row
    v = rng.normal(size=(E, C))
    ref = oracle.density_accumulate(v, centers, N)
    a = density_accumulate(_t(v), _t(centers), N, validate=True)
    b = density_accumulate(_t(v), _t(centers), N)
    np.testing.assert_allclose(a.cpu().numpy(), ref, rtol=1e-12, atol=1e-12)
    assert torch.equal(a, b)  # bit-stable run to run
    with pytest.raises(IndexError):
        density_accumulate(_t(v[:3]), _t(np.asarray([0, N, 1])), N, validate=True)


def test_density_accumulate_autograd():
    from ye3t_b200.runtime import density_accumulate
    centers = torch.tensor([0, 0, 2, 1, 2, 2, 3, 0, 3], device=DEV)
    ev = torch.randn(9, 7, dtype=torch.float64, device=DEV, requires_grad=True)
    out = density_accumulate(ev, centers, 4)
    (out * torch.arange(28, device=DEV, dtype=torch.float64).reshape(4, 7)).sum().backward()
    expect = torch.arange(28, device=DEV, dtype=torch.float64).reshape(4, 7)[centers]
    assert torch.equal(ev.grad, expect)


def test_symmetric_power_matches_reference(golden):
    from ye3t_b200.runtime import symmetric_power_table_contraction, symmetric_power_monomial_contraction
    from ye3t_b200.schedules import ACEBundle
    import os
    g = golden("sympow")
    b = ACEBundle.load(os.path.join(os.path.dirname(os.path.dirname(__file__)), "ye3t_b200", "bundles",
                                    "ace_n8_l3_nu4_L0.npz"))
    j = 0
    while f"k{j}_key" in g:
        t = b.sym_tables[tuple(int(v) for v in g[f"k{j}_key"])]
        y = symmetric_power_table_contraction(_t(g[f"k{j}_x"]), t)
        np.testing.assert_allclose(y.cpu().numpy(), g[f"k{j}_y"], rtol=1e-12, atol=1e-12)
        j += 1
    # the reference's pinned fixture (shared form lowered to grouped rows)
    dim = int(g["fx_input_dimension"])
    counts = g["fx_monomial_counts"].reshape(-1, dim)
    terms, outs, vals = g["fx_coefficient_terms"], g["fx_coefficient_outputs"], g["fx_coefficient_values"]
    order = np.argsort(outs, kind="stable")
    grouped_counts = counts[terms[order]]
    offsets = np.concatenate([[0], np.cumsum(np.bincount(outs, minlength=int(g["fx_output_dimension"])))])
    x = g["fx_input"].reshape(int(g["fx_batch_size"]), dim)
    y = symmetric_power_monomial_contraction(_t(x), _t(grouped_counts), _t(offsets), _t(outs[order]),
                                             _t(vals[order]))
    np.testing.assert_allclose(y.cpu().numpy().reshape(-1), g["fx_expected_output"], rtol=1e-13, atol=1e-13)


def test_symmetric_power_shared_monomial_matches_reference(golden):
    """The shared-monomial form (execution_plan.py:12502): the reference's pinned fixture as is,
    then every symmetric block kind of the nu<=4 word set lowered to unique monomials against the
    oracle (complex128 and complex64), and the table checks."""
    from oracle import oracle
    from ye3t_b200.runtime import symmetric_power_shared_monomial_contraction as op
    from ye3t_b200.schedules import ACEBundle
    import os
    g = golden("sympow")
    dim = int(g["fx_input_dimension"])
    x = g["fx_input"].reshape(int(g["fx_batch_size"]), dim)
    y = op(_t(x), _t(g["fx_monomial_counts"].reshape(-1, dim)), _t(g["fx_output_offsets"]),
           _t(g["fx_coefficient_terms"]), _t(g["fx_coefficient_outputs"]), _t(g["fx_coefficient_values"]))
    np.testing.assert_allclose(y.cpu().numpy().reshape(-1), g["fx_expected_output"], rtol=1e-13, atol=1e-13)
    b = ACEBundle.load(os.path.join(os.path.dirname(os.path.dirname(__file__)), "ye3t_b200", "bundles",
                                    "ace_n8_l3_nu4_L0.npz"))
    rng = np.random.default_rng(3)
    for key in sorted(b.sym_tables):
        t = b.sym_tables[key]
        unique, terms = np.unique(t.monomial_counts, axis=0, return_inverse=True)
        outs = np.repeat(np.arange(t.output_offsets.shape[0] - 1), np.diff(t.output_offsets))
        xs = rng.normal(size=(40, t.monomial_counts.shape[1])) + 1j * rng.normal(size=(40, t.monomial_counts.shape[1]))
        ref = oracle.symmetric_power_shared_monomial(xs, unique, t.output_offsets, terms.reshape(-1),
                                                     t.monomial_value)
        for dt, tol in ((torch.complex128, 1e-12), (torch.complex64, 1e-5)):
            y = op(torch.as_tensor(xs, device=DEV).to(dt), unique, t.output_offsets, terms.reshape(-1), outs,
                   torch.as_tensor(t.monomial_value).to(dt))
            err = np.abs(y.cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1.0)
            assert err <= tol, (key, dt, err)
    # the pinned fixture's input adjoint (its autograd), through the GPU backward
    xg = _t(x).requires_grad_(True)
    y = op(xg, _t(g["fx_monomial_counts"].reshape(-1, dim)), _t(g["fx_output_offsets"]),
           _t(g["fx_coefficient_terms"]), _t(g["fx_coefficient_outputs"]), _t(g["fx_coefficient_values"]))
    (grad,) = torch.autograd.grad(y, xg, _t(g["fx_output_adjoint"].reshape(y.shape)))
    np.testing.assert_allclose(grad.cpu().numpy().reshape(-1), g["fx_expected_input_adjoint"], rtol=1e-13,
                               atol=1e-13)
    counts = g["fx_monomial_counts"].reshape(-1, dim)
    with pytest.raises(ValueError, match="invalid monomial"):
        op(_t(x), _t(counts), _t(g["fx_output_offsets"]), _t(g["fx_coefficient_terms"] + 3),
           _t(g["fx_coefficient_outputs"]), _t(g["fx_coefficient_values"]))
    with pytest.raises(ValueError, match="length must match"):
        op(_t(x), _t(counts), _t(g["fx_output_offsets"]), _t(g["fx_coefficient_terms"]),
           _t(g["fx_coefficient_outputs"][:-1]), _t(g["fx_coefficient_values"]))


def _record(g, p):
    from ye3t_b200.schedules import ScheduleRecord
    specs = json.loads(bytes(g[p + "specs"]).decode())
    return ScheduleRecord(rank=0, block_count=int(g[p + "bm"].shape[1]), L_R=0, n_tuple=(), l_tuple=(),
                          block_specs=tuple(tuple(tuple(s) for s in label) for label in specs),
                          component_offsets=g[p + "off"], component_label_index=g[p + "cli"],
                          component_M_R=np.zeros_like(g[p + "cli"]), block_m_tuples=g[p + "bm"],
                          coeffs=g[p + "co"])


def test_factorized_schedule_matches_reference(golden):
    from ye3t_b200.couplings import evaluate_factorized_schedule_torch as ev
    g = golden("schedules")
    meta = json.loads(bytes(g["meta"]).decode())
    for i, _m in enumerate(meta):
        rec = _record(g, f"s{i}_")
        outc = ev(_t(g[f"s{i}_bvc"]), rec, validate=True).cpu().numpy()
        ref = g[f"s{i}_outc_cpp"]
        assert np.max(np.abs(outc - ref)) <= 1e-12 * max(1.0, np.abs(ref).max())
        outr = ev(_t(g[f"s{i}_bvr"]), rec).cpu().numpy()
        np.testing.assert_allclose(outr, g[f"s{i}_outr_cpp"], rtol=1e-12, atol=1e-12)
        outf = ev(_t(g[f"s{i}_bvr"].astype(np.float32)), rec).cpu().numpy()
        np.testing.assert_allclose(outf, g[f"s{i}_outf_cpp"], rtol=1e-5, atol=1e-5)
        outc64 = ev(_t(g[f"s{i}_bvc"].astype(np.complex64)), rec).cpu().numpy()
        np.testing.assert_allclose(outc64, ref, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("tag", ["c", "r"])
def test_factorized_schedule_backward_matches_reference_autograd(golden, tag):
    """Block-value gradients of evaluate_factorized_schedule_torch (GPU vector-Jacobian product)
    against torch autograd through the reference's torch evaluator."""
    from ye3t_b200.couplings import evaluate_factorized_schedule_torch
    g = golden("schedules")
    gg = golden("schedule_grads")
    i = 0
    while f"s{i}_off" in g:
        rec = _record(g, f"s{i}_")
        p = f"s{i}_{tag}_"
        x = _t(gg[p + "bv"]).requires_grad_(True)
        y = evaluate_factorized_schedule_torch(x, rec)
        (grad,) = torch.autograd.grad(y, x, _t(gg[p + "adj"]))
        ref = gg[p + "grad"]
        err = np.abs(grad.cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1.0)
        assert err <= 1e-12, (i, err)
        i += 1
    assert i == 8


def test_quickstart_config1(golden):
    from ye3t_b200.couplings import evaluate_factorized_schedule_torch as ev
    g = golden("quickstart")
    rec = _record(g, "q_")
    out = ev(_t(g["bv"]), rec).cpu().numpy()
    np.testing.assert_allclose(out, g["out_cpp"], rtol=1e-12, atol=1e-12)
    # Binding sweep over all 56 ordered channel pairs (batch 229,376): the
    # symmetric block Sym^2(V_1) -> 0 comes from the bundle's table; binding
    # (n1, n2) = (0, 1) must reproduce the golden block values.
    import os
    from ye3t_b200.schedules import ACEBundle
    b = ACEBundle.load(os.path.join(os.path.dirname(os.path.dirname(__file__)), "ye3t_b200", "bundles",
                                    "ace_n8_l3_nu4_L0.npz"))
    t = b.sym_tables[(1, 2, 0, 0)]
    gen = torch.Generator().manual_seed(0)
    A1 = torch.randn(4096, 8, 3, dtype=torch.float64, generator=gen).numpy()
    A0 = torch.randn(4096, 8, 1, dtype=torch.float64, generator=gen).numpy()
    sym = oracle.symmetric_power_monomial(A1.reshape(-1, 3), t.monomial_counts, t.output_offsets,
                                          t.monomial_value.real).reshape(4096, 8)
    np.testing.assert_allclose(sym[:, 0], g["bv"][:, 0, 0, 0], rtol=1e-14, atol=1e-14)
    pairs = [(n1, n2) for n1 in range(8) for n2 in range(8) if n1 != n2]
    bv = np.zeros((4096 * len(pairs), 1, 2, 1))
    for r, (n1, n2) in enumerate(pairs):
        bv[r * 4096:(r + 1) * 4096, 0, 0, 0] = sym[:, n1]
        bv[r * 4096:(r + 1) * 4096, 0, 1, 0] = A0[:, n2, 0]
    got = ev(_t(bv), rec).cpu().numpy()
    np.testing.assert_allclose(got, oracle.schedule_evaluate_record(bv, rec), rtol=1e-12, atol=1e-12)
    assert got.shape == (229376, 1)


def test_schedule_status_on_bad_index(golden):
    from ye3t_b200.couplings import evaluate_factorized_schedule_torch as ev
    from ye3t_b200.schedules import ScheduleRecord
    g = golden("schedules")
    rec = _record(g, "s0_")
    bad = ScheduleRecord(rank=0, block_count=rec.block_count, L_R=0, n_tuple=(), l_tuple=(),
                         block_specs=rec.block_specs, component_offsets=rec.component_offsets,
                         component_label_index=rec.component_label_index + 5,
                         component_M_R=rec.component_M_R, block_m_tuples=rec.block_m_tuples, coeffs=rec.coeffs)
    with pytest.raises(IndexError):
        ev(_t(g["s0_bvc"]), bad, validate=True)


def test_library_rejects_cpu_tensors():
    from ye3t_b200.runtime import density_accumulate
    with pytest.raises(ValueError):
        density_accumulate(torch.zeros(3, 2), torch.zeros(3, dtype=torch.int64), 2)
