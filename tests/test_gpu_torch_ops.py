"""torch.ops.ye3t_b200.* on the GPU: the same results as the runtime functions, and
autograd through the registered operators against the runtime's backward."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _t(a):
    return torch.as_tensor(a, device=DEV)


def test_torch_ops_match_runtime(golden):
    import ye3t_b200.torch_ops  # noqa: F401
    from ye3t_b200 import runtime as rt
    ops = torch.ops.ye3t_b200
    g = golden("edge_ops")
    r = _t(g["radii"])
    rc = _t(np.broadcast_to(g["rc"], g["radii"].shape).copy())
    lam = _t(np.broadcast_to(g["lam"], g["radii"].shape).copy())
    k = int(g["kmax"])
    for a, b in zip(ops.cheb_exp_cos_radial_table_with_derivative(r, rc, lam, k),
                    rt.cheb_exp_cos_radial_table_with_derivative(r, rc, lam, k)):
        assert torch.equal(a, b)
    vec = _t(np.random.default_rng(1).normal(size=(50, 3)))
    for a, b in zip(ops.spherical_harmonics_table_with_derivative(vec, 3, False, 1e-12),
                    rt.spherical_harmonics_table_with_derivative(vec, 3)):
        assert torch.equal(a, b)
    ev = _t(np.random.default_rng(2).normal(size=(40, 16)))
    centers = _t(np.random.default_rng(3).integers(0, 9, size=40))
    assert torch.equal(ops.density_accumulate(ev, centers, 9), rt.density_accumulate(ev, centers, 9))
    gs = golden("schedules")
    p = "s2_"
    bv = _t(gs[p + "bvc"])
    from ye3t_b200.schedules import ScheduleRecord
    import json
    rec = ScheduleRecord(rank=0, block_count=int(gs[p + "bm"].shape[1]), L_R=0, n_tuple=(), l_tuple=(),
                         block_specs=tuple(tuple(tuple(s) for s in label)
                                           for label in json.loads(bytes(gs[p + "specs"]).decode())),
                         component_offsets=gs[p + "off"], component_label_index=gs[p + "cli"],
                         component_M_R=np.zeros_like(gs[p + "cli"]), block_m_tuples=gs[p + "bm"], coeffs=gs[p + "co"])
    from ye3t_b200.couplings import evaluate_factorized_schedule_torch
    y = ops.factorized_schedule(bv, _t(rec.component_offsets), _t(rec.component_label_index),
                                _t(rec.block_m_indices()), _t(np.asarray(rec.coeffs)))
    assert torch.equal(y, evaluate_factorized_schedule_torch(bv, rec))


def test_torch_ops_autograd(golden):
    import ye3t_b200.torch_ops  # noqa: F401
    from ye3t_b200 import runtime as rt
    ops = torch.ops.ye3t_b200
    rng = np.random.default_rng(4)
    ev = _t(rng.normal(size=(40, 16)) + 1j * rng.normal(size=(40, 16))).requires_grad_(True)
    centers = _t(rng.integers(0, 9, size=40))
    adj = _t(rng.normal(size=(9, 16)) + 1j * rng.normal(size=(9, 16)))
    (g1,) = torch.autograd.grad(ops.density_accumulate(ev, centers, 9), ev, adj)
    assert torch.equal(g1, rt.density_accumulate_adjoint(adj, centers))
    gs = golden("adjoints")
    import os
    from ye3t_b200.schedules import ACEBundle
    b = ACEBundle.load(os.path.join(os.path.dirname(os.path.dirname(__file__)), "ye3t_b200", "bundles",
                                    "ace_n8_l3_nu4_L0.npz"))
    t = b.sym_tables[tuple(int(v) for v in gs["sp5_key"])]
    x = _t(gs["sp5_x"]).requires_grad_(True)
    y = ops.symmetric_power_monomial(x, _t(t.monomial_counts), _t(t.output_offsets), _t(t.output_index),
                                     _t(t.monomial_value))
    (g2,) = torch.autograd.grad(y, x, _t(gs["sp5_adj"]))
    ref = gs["sp5_grad"]
    assert np.abs(g2.cpu().numpy() - ref).max() <= 1e-12 * max(np.abs(ref).max(), 1.0)
