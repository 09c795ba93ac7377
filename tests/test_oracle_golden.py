"""The CPU oracle against the reference's golden vectors (no GPU)."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from ye3t_b200.schedules import ACEBundle, ScheduleRecord

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _record(g, p):
    specs = json.loads(bytes(g[p + "specs"]).decode())
    return ScheduleRecord(
        rank=len(specs[0][0]) if specs else 0, block_count=int(g[p + "bm"].shape[1]), L_R=0, n_tuple=(),
        l_tuple=(), block_specs=tuple(tuple(tuple(s) for s in label) for label in specs),
        component_offsets=g[p + "off"], component_label_index=g[p + "cli"],
        component_M_R=np.zeros_like(g[p + "cli"]), block_m_tuples=g[p + "bm"], coeffs=g[p + "co"])


def test_schedule_oracle_matches_reference_cpp(golden):
    g = golden("schedules")
    meta = json.loads(bytes(g["meta"]).decode())
    for i, m in enumerate(meta):
        rec = _record(g, f"s{i}_")
        assert rec.term_count == m["term_count"] and rec.basis_count == m["basis_count"]
        np.testing.assert_array_equal(rec.block_L_by_label(), g[f"s{i}_bl"])
        outc = oracle.schedule_evaluate_record(g[f"s{i}_bvc"], rec)
        ref = g[f"s{i}_outc_cpp"]
        assert np.max(np.abs(outc - ref)) <= 1e-12 * max(1.0, np.max(np.abs(ref)))
        np.testing.assert_allclose(outc, g[f"s{i}_outc_torch"], rtol=1e-12, atol=1e-12)
        outr = oracle.schedule_evaluate_record(g[f"s{i}_bvr"], rec)
        assert outr.dtype == np.float64
        np.testing.assert_allclose(outr, g[f"s{i}_outr_cpp"], rtol=1e-12, atol=1e-12)
        outf = oracle.schedule_evaluate_record(g[f"s{i}_bvr"].astype(np.float32), rec)
        np.testing.assert_allclose(outf, g[f"s{i}_outf_cpp"], rtol=1e-5, atol=1e-5)


def test_quickstart_config1(golden):
    g = golden("quickstart")
    assert bytes(g["convention_hash"]).decode() == "00112c9d4a6cb444"
    gen = torch.Generator().manual_seed(0)
    A1 = torch.randn(4096, 8, 3, dtype=torch.float64, generator=gen).numpy()
    A0 = torch.randn(4096, 8, 1, dtype=torch.float64, generator=gen).numpy()
    np.testing.assert_array_equal(A1[:16], g["A1_head"])
    np.testing.assert_array_equal(A0[:16], g["A0_head"])
    rec = _record(g, "q_")
    out = oracle.schedule_evaluate_record(g["bv"], rec)
    np.testing.assert_allclose(out, g["out_cpp"], rtol=1e-12, atol=1e-12)


def test_sympow_oracle_matches_reference(golden):
    g = golden("sympow")
    b = ACEBundle.load(_bundle_path("ace_n8_l3_nu4_L0"))
    j = 0
    while f"k{j}_key" in g:
        key = tuple(int(v) for v in g[f"k{j}_key"])
        t = b.sym_tables[key]
        y = oracle.symmetric_power_monomial(g[f"k{j}_x"], t.monomial_counts, t.output_offsets,
                                            t.monomial_value)
        np.testing.assert_allclose(y, g[f"k{j}_y"], rtol=1e-12, atol=1e-12)
        j += 1
    assert j == 23


def test_sympow_oracle_matches_reference_pinned_fixture(golden):
    # tests/fixtures/shared_monomial_plan_v1.txt of the reference, convention 60be803770d2499e
    g = golden("sympow")
    assert bytes(g["fx_convention_hash"]).decode() == "60be803770d2499e"
    dim = int(g["fx_input_dimension"])
    x = g["fx_input"].reshape(int(g["fx_batch_size"]), dim)
    y = oracle.symmetric_power_shared_monomial(x, g["fx_monomial_counts"], g["fx_output_offsets"],
                                               g["fx_coefficient_terms"], g["fx_coefficient_values"])
    np.testing.assert_allclose(y.reshape(-1), g["fx_expected_output"], rtol=1e-13, atol=1e-13)


def test_radial_oracle(golden):
    g = golden("edge_ops")
    v, d = oracle.radial_table(g["radii"], g["rc"], g["lam"], int(g["kmax"]))
    np.testing.assert_allclose(v, g["rad_val_native"], rtol=2e-13, atol=2e-13)
    np.testing.assert_allclose(d, g["rad_der_native"], rtol=2e-12, atol=2e-12)
    np.testing.assert_allclose(v, g["rad_val_torch"], rtol=2e-13, atol=2e-13)


def test_spherical_oracle(golden):
    g = golden("edge_ops")
    lmax = int(g["lmax"])
    vr, dr = oracle.sh_table(g["vec"], lmax, real_output=True)
    np.testing.assert_allclose(vr, g["shr_val_native"], rtol=2e-12, atol=2e-12)
    np.testing.assert_allclose(dr, g["shr_der_native"], rtol=2e-11, atol=2e-11)
    vc, dc = oracle.sh_table(g["vec"], lmax, real_output=False)
    np.testing.assert_allclose(vc, g["shc_val_native"], rtol=2e-12, atol=2e-12)
    np.testing.assert_allclose(dc, g["shc_der_native"], rtol=2e-11, atol=2e-11)
    np.testing.assert_allclose(vc[6:], g["shc_val_torch"], rtol=2e-12, atol=2e-12)
    np.testing.assert_allclose(vr[6:], g["shr_val_torch"], rtol=2e-12, atol=2e-12)


def test_density_oracle(golden):
    g = golden("edge_ops")
    np.testing.assert_allclose(oracle.density_accumulate(g["ev_r"], g["centers"], 4), g["acc_r"], atol=1e-12)
    np.testing.assert_allclose(oracle.density_accumulate(g["ev_c"], g["centers"], 4), g["acc_c"], atol=1e-12)


def test_ace_pipeline_oracle(golden):
    g = golden("ace_small")
    off, nbr, disp = oracle.neighbor_list(g["pos"], float(g["box"]), float(g["rc"]))
    np.testing.assert_array_equal(off, g["row_off"])
    np.testing.assert_array_equal(nbr, g["nbr"])
    np.testing.assert_allclose(disp, g["disp"], atol=1e-12)
    A = oracle.ace_density(disp, off, nbr, g["species"], g["prefactor"], int(g["nmax"]), int(g["lmax"]),
                           float(g["rc"]), float(g["lam"]))
    ref = g["A"]
    assert np.max(np.abs(A - ref)) <= 1e-12 * np.max(np.abs(ref))
    b3 = ACEBundle.load(_bundle_path("ace_n8_l3_nu3_L0"))
    B3 = oracle.bundle_features(b3, A[:40], threads=4)
    rel = np.linalg.norm(B3 - g["B3"], axis=1) / np.linalg.norm(g["B3"], axis=1)
    assert rel.max() <= 1e-12
    b4 = ACEBundle.load(_bundle_path("ace_n8_l3_nu4_L0"))
    B4 = oracle.bundle_features(b4, A[:40], words=g["B4_words"], threads=4)
    rel = np.linalg.norm(B4 - g["B4"], axis=1) / np.linalg.norm(g["B4"], axis=1)
    assert rel.max() <= 1e-12
    e = oracle.bundle_energy(b3, A, g["species"], g["w3"], threads=4).sum()
    assert abs(e - float(g["energy3"])) <= 1e-12 * abs(float(g["energy3"]))


def test_oracle_matches_reference_core_build():
    ref = oracle.refcore()
    if ref is None:
        pytest.skip("reference core not built (make -C oracle ref)")
    import ctypes
    rng = np.random.default_rng(5)
    E, lmax, kmax = 301, 3, 8
    vec = rng.normal(size=(E, 3)) * 3
    r = np.sqrt((vec ** 2).sum(1))
    v1, d1 = oracle.radial_table(r, 5.0, 5.0, kmax)
    v2 = np.zeros_like(v1); d2 = np.zeros_like(d1)
    rc = np.full(E, 5.0); lam = np.full(E, 5.0)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    ref.yr_cheb_exp_cos_radial_table_f64(P(r), P(rc), P(lam), ctypes.c_int64(E), ctypes.c_int64(kmax), P(v2), P(d2),
                                         ctypes.c_int(2))
    np.testing.assert_allclose(v1, v2, rtol=1e-13, atol=1e-14)
    np.testing.assert_allclose(d1, d2, rtol=1e-12, atol=1e-13)
    c1, cd1 = oracle.sh_table(vec, lmax)
    W = (lmax + 1) ** 2
    c2 = np.zeros((E, W), np.complex128); cd2 = np.zeros((E, W, 3), np.complex128)
    ref.yr_complex_spherical_harmonics_table_f64(P(vec), ctypes.c_int64(E), ctypes.c_int64(lmax),
                                                 ctypes.c_double(1e-12), P(c2), P(cd2), ctypes.c_int(2))
    np.testing.assert_allclose(c1, c2, rtol=1e-12, atol=1e-13)
    np.testing.assert_allclose(cd1, cd2, rtol=1e-11, atol=1e-12)


def test_reference_evaluator_build_matches_oracle_and_golden(golden):
    """The reference's compiled schedule evaluator and symmetric power, built from their
    sources into oracle/_ref, give the quickstart golden (out_cpp, written by the reference's
    own evaluate(backend="cpp")) and agree with the restatement, so the C1 CPU arm may time
    either."""
    if oracle.refeval() is None or oracle.refcore() is None:
        pytest.skip("reference builds absent (make -C oracle ref)")
    g = golden("quickstart")
    rec = _record(g, "q_")
    out = oracle.ref_schedule_evaluate_record(g["bv"], rec)
    np.testing.assert_allclose(out, g["out_cpp"], rtol=1e-13, atol=1e-13)
    np.testing.assert_allclose(out, oracle.schedule_evaluate_record(g["bv"], rec), rtol=1e-13, atol=1e-13)
    b = ACEBundle.load(_bundle_path("ace_n8_l3_nu4_L0"))
    t = b.sym_tables[(1, 2, 0, 0)]
    x = np.random.default_rng(3).normal(size=(257, 3))
    y = oracle.ref_symmetric_power_monomial(x, t.monomial_counts, t.output_offsets, t.monomial_value.real,
                                            threads=2)
    np.testing.assert_allclose(y, oracle.symmetric_power_monomial(x, t.monomial_counts, t.output_offsets,
                                                                  t.monomial_value.real), rtol=1e-14, atol=1e-14)


def _bundle_path(stem):
    import os
    return os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "ye3t_b200", "bundles",
                        stem + ".npz")


def test_oracle_forces_match_reference_autograd(golden):
    """The oracle's force path (schedule and symmetric-power adjoints, edge
    gradients, reverse-edge scatter) against torch autograd through the
    reference ops (tests/golden/make_golden.py forces_fixture)."""
    small = golden("ace_small")
    ref = golden("forces_small")
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu3_L0.npz"))
    E, F = oracle.energy_forces(b, small["pos"], float(small["box"]), small["species"], small["prefactor"],
                                small["w3"], float(small["rc"]), float(small["lam"]), threads=4)
    assert abs(E - float(ref["energy"])) <= 1e-12 * abs(float(ref["energy"]))
    err = np.abs(F - ref["forces"]).max() / np.abs(ref["forces"]).max()
    assert err <= 1e-11, err


def test_oracle_schedule_adjoint_is_the_holomorphic_derivative():
    """dL = Re(sum gbv dbv) for L = Re(sum gout out) along a random complex direction."""
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu3_L0.npz"))
    rng = np.random.default_rng(3)
    for w in (0, 17, b.word_count - 1):
        rec = b.word_schedule(w)
        shape = (3, rec.basis_count, rec.block_count, rec.max_block_m_dim)
        bv = rng.normal(size=shape) + 1j * rng.normal(size=shape)
        C = int(rec.component_offsets.shape[0]) - 1
        gout = rng.normal(size=(3, C)) + 1j * rng.normal(size=(3, C))
        gbv = oracle.schedule_adjoint(bv, rec, gout)
        d = (rng.normal(size=shape) + 1j * rng.normal(size=shape)) * 1e-6
        lp = (gout * oracle.schedule_evaluate_record(bv + d, rec)).real.sum()
        lm = (gout * oracle.schedule_evaluate_record(bv - d, rec)).real.sum()
        lin = (gbv * d).real.sum()
        assert abs((lp - lm) / 2 - lin) <= 1e-7 * abs(lin) + 1e-14


def test_oracle_radial_channel_contraction_matches_reference_core(golden):
    """Bit-exact against pace_radial_channel_contraction_with_derivative (reference core, f64 and f32)."""
    g = golden("mixing_small")
    for tag in ("f64", "f32"):
        y, dy = oracle.radial_channel_contraction(g[f"c_{tag}_x"], g[f"c_{tag}_dx"], g[f"c_{tag}_w"])
        assert np.array_equal(y, g[f"c_{tag}_y"]) and np.array_equal(dy, g[f"c_{tag}_dy"])


def test_oracle_mixed_density_matches_reference_composition(golden):
    """Mixed A-basis against the reference radial table, contraction, harmonics and density_accumulate."""
    g = golden("mixing_small")
    off, nbr, disp = oracle.neighbor_list(g["pos"], float(g["box"]), float(g["rc"]))
    assert np.array_equal(off, g["row_off"]) and np.array_equal(nbr, g["nbr"])
    A = oracle.ace_density_mixed(disp, off, nbr, g["species"], g["mixing"], int(g["nmax"]), int(g["lmax"]),
                                 float(g["rc"]), float(g["lam"]))
    err = np.abs(A - g["A"]).max() / np.abs(g["A"]).max()
    assert err <= 1e-13, err


def test_oracle_real_tesseral_schedules(golden):
    """Real-tesseral schedules (generate_real_factorized_coefficient_schedule_for_labels) through the
    oracle's schedule evaluator against the reference's evaluate_real_factorized_schedule_torch."""
    g = golden("real_schedules")
    for k in range(int(g["count"])):
        p = f"r{k}_"
        y = oracle.schedule_evaluate(g[p + "bv"], g[p + "off"], g[p + "cli"], g[p + "idx"], g[p + "co"])
        np.testing.assert_allclose(y, g[p + "y"], rtol=1e-13, atol=1e-13)


S_ARGS = ("radial_values", "radial_derivatives", "angular_values", "angular_derivatives", "radial_directions",
          "edge_types", "channel_radial_indices", "channel_angular_indices", "channel_types", "channel_scales")
P_ARGS = ("radial_values", "radial_derivatives", "angular_values", "angular_derivatives", "prefactors",
          "prefactor_derivatives_center", "prefactor_derivatives_neighbor", "radial_directions", "term_groups",
          "term_channels")


def _rel(a, ref):
    return np.abs(np.asarray(a) - ref).max() / max(np.abs(ref).max(), 1.0)


def test_oracle_edge_products_match_reference(golden):
    """Scheduled radial-angular channels and the plain site-basis product (and its adjoint)
    restated in numpy, against the reference's compositions (execution_plan.py:7036-7220)."""
    g = golden("edge_products")
    for tag in ("f64", "f32"):
        v, d = oracle.scheduled_radial_angular_channels(*(g[f"s_{tag}_{k}"] for k in S_ARGS))
        assert np.array_equal(v, g[f"s_{tag}_values"]) and np.array_equal(d, g[f"s_{tag}_derivatives"])
    for tag, tol in (("f64", 1e-14), ("c128", 1e-13), ("c64", 1e-5)):
        outs = oracle.plain_site_basis_product(*(g[f"p_{tag}_{k}"] for k in P_ARGS), int(g[f"p_{tag}_channel_count"]))
        for name, y in zip(("edge_values", "edge_derivatives", "charge_center", "charge_neighbor"), outs):
            assert _rel(y, g[f"p_{tag}_{name}"]) <= tol, (tag, name)
    ga = golden("adjoints")
    for tag in ("f64", "c128"):
        outs = oracle.plain_site_basis_product_adjoint(*(ga[f"pa_{tag}_{k}"] for k in P_ARGS[:8]),
                                                       ga[f"pa_{tag}_edge_weights"],
                                                       ga[f"pa_{tag}_edge_weight_derivatives"],
                                                       ga[f"pa_{tag}_term_groups"], ga[f"pa_{tag}_term_channels"],
                                                       ga[f"pa_{tag}_edge_adjoint"])
        for name, y in zip(("position", "charge_center", "charge_neighbor"), outs):
            assert _rel(y, ga[f"pa_{tag}_{name}"]) <= 1e-13, (tag, name)


def test_oracle_adjoints_match_reference_autograd(golden):
    """The oracle's holomorphic adjoints of the schedule evaluation and of the grouped symmetric
    power, against torch autograd through the reference (which returns conj(J)^T adj, i.e.
    conj(holomorphic adjoint of conj(adj)))."""
    g, gg = golden("schedules"), golden("schedule_grads")
    for i in range(8):
        rec = _record(g, f"s{i}_")
        for tag in ("c", "r"):
            p = f"s{i}_{tag}_"
            got = np.conj(oracle.schedule_adjoint(gg[p + "bv"], rec, np.conj(gg[p + "adj"])))
            if tag == "r":
                got = got.real
            assert _rel(got, gg[p + "grad"]) <= 1e-13, (i, tag)
    ga = golden("adjoints")
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu4_L0.npz"))
    j = 0
    while f"sp{j}_key" in ga:
        t = b.sym_tables[tuple(int(v) for v in ga[f"sp{j}_key"])]
        got = np.conj(oracle.symmetric_power_monomial_adjoint(ga[f"sp{j}_x"], t.monomial_counts, t.output_offsets,
                                                              t.monomial_value, np.conj(ga[f"sp{j}_adj"])))
        assert _rel(got, ga[f"sp{j}_grad"]) <= 1e-13, j
        j += 1
    assert j == 23
