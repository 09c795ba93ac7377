"""Real-tesseral factorized schedules (ye3t/core/couplings.py:337-478, 570-610) on the GPU
against the reference's evaluate_real_factorized_schedule_torch."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


class _Record:
    """The fields of a RealFactorizedCoefficientSchedule, as stored in the fixture."""

    def __init__(self, g, p):
        self.component_offsets = g[p + "off"]
        self.component_label_index = g[p + "cli"]
        self.block_real_tuples = g[p + "idx"]
        self.coeffs = g[p + "co"]
        self.block_L = g[p + "bL"]
        self.block_count = int(g[p + "idx"].shape[1])
        self.basis_count = int(g[p + "basis"])


def test_real_schedules_match_reference(golden):
    from ye3t_b200.couplings import evaluate_real_factorized_schedule_torch as ev
    g = golden("real_schedules")
    for k in range(int(g["count"])):
        p = f"r{k}_"
        rec = _Record(g, p)
        bv = torch.as_tensor(g[p + "bv"], device=DEV)
        y = ev(bv, rec, validate=True).cpu().numpy()
        # same products in block order and sums in term order as the reference
        np.testing.assert_allclose(y, g[p + "y"], rtol=1e-14, atol=1e-14)
        y32 = ev(bv.float(), rec).cpu().numpy()
        assert y32.dtype == np.float32
        np.testing.assert_allclose(y32, g[p + "y"], rtol=1e-4, atol=1e-5)


def test_real_schedule_rejects_complex_and_bad_shapes(golden):
    from ye3t_b200.couplings import evaluate_real_factorized_schedule_torch as ev
    g = golden("real_schedules")
    rec = _Record(g, "r0_")
    bv = torch.as_tensor(g["r0_bv"], device=DEV)
    with pytest.raises(ValueError):
        ev(bv.to(torch.complex128), rec)
    with pytest.raises(ValueError):
        ev(bv[:, :, :1], rec)
    with pytest.raises(ValueError):
        ev(bv, rec, backend="torch")
