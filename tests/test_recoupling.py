"""Recoupled plan of a scalar ACE bundle (host side, CPU).

The plan rewrites every feature as a sum of contractions of coupled channel
pairs with weights fitted per pattern; these tests pin it to the reference's
own features (the golden B-basis of the 96-atom system, computed by the
reference) and to the oracle's energy gradient, and check the plan's
structure and its per-atom costs."""

import math
import os

import numpy as np
import pytest

from ye3t_b200.recoupling import (SEG_CHANNEL, SEG_PAIR, SEG_UNIT, build_recoupled_plan, cg_table,
                                  clebsch_gordan)
from ye3t_b200.schedules import ACEBundle

import recoupled_numpy as rn

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bundle(stem):
    return ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", stem + ".npz"))


@pytest.fixture(scope="module")
def plan3():
    return build_recoupled_plan(_bundle("ace_n8_l3_nu3_L0"))


@pytest.fixture(scope="module")
def plan5():
    b = _bundle("ace_n8_l3_nu4_L0")
    return b, build_recoupled_plan(b)


def test_clebsch_gordan_values_and_orthonormality():
    # tabulated values (Condon-Shortley phase)
    assert clebsch_gordan(1, 0, 1, 0, 0, 0) == pytest.approx(-1 / math.sqrt(3), abs=1e-15)
    assert clebsch_gordan(1, 1, 1, -1, 0, 0) == pytest.approx(1 / math.sqrt(3), abs=1e-15)
    assert clebsch_gordan(1, 1, 1, 0, 2, 1) == pytest.approx(1 / math.sqrt(2), abs=1e-15)
    assert clebsch_gordan(1, 0, 1, 0, 2, 0) == pytest.approx(math.sqrt(2 / 3), abs=1e-15)
    assert clebsch_gordan(2, 1, 1, -1, 1, 0) == pytest.approx(math.sqrt(3 / 10), abs=1e-15)
    assert clebsch_gordan(1, 0, 1, 0, 1, 0) == 0.0
    # the coupling V_l1 x V_l2 -> sum_L V_L is orthogonal
    for l1 in range(4):
        for l2 in range(4):
            Ls = range(abs(l1 - l2), l1 + l2 + 1)
            U = np.zeros(((2 * l1 + 1) * (2 * l2 + 1), sum(2 * L + 1 for L in Ls)))
            col = 0
            for L in Ls:
                idx, val = cg_table(l1, l2, L)
                U[idx[:, 0] * (2 * l2 + 1) + idx[:, 1], col + idx[:, 2]] = val
                col += 2 * L + 1
            assert np.abs(U.T @ U - np.eye(U.shape[1])).max() < 1e-13


def test_plan_reproduces_reference_features_nu3(plan3, golden):
    g = golden("ace_small")
    A = np.asarray(g["A"])[:40]
    F = rn.features(plan3, A)
    ref = np.asarray(g["B3"])
    assert np.abs(F - ref).max() <= 1e-12 * np.abs(ref).max()


def test_plan_reproduces_reference_features_nu4(plan5, golden):
    b, plan = plan5
    g = golden("ace_small")
    A = np.asarray(g["A"])[:40]
    F = rn.features(plan, A)
    off = b.feature_offsets()
    cols = np.concatenate([np.arange(off[w], off[w + 1]) for w in np.asarray(g["B4_words"])])
    ref = np.asarray(g["B4"])
    assert ref.shape[1] == cols.shape[0]
    assert np.abs(F[:, cols] - ref).max() <= 1e-12 * np.abs(ref).max()


def test_plan_energy_gradient_matches_oracle(plan5):
    from oracle import oracle
    b, plan = plan5
    rng = np.random.default_rng(11)
    A = rng.normal(size=(3, 8, 16)) + 1j * rng.normal(size=(3, 8, 16))
    species = np.array([0, 2, 1], dtype=np.int32)
    w = rng.normal(size=(3, b.feature_count)) / np.sqrt(b.feature_count)
    e0, G0 = oracle.bundle_energy_grad(b, A, species, w, threads=4)
    e1, G1 = rn.energy_grad(plan, A, species, w)
    assert np.abs(e1 - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G1 - G0).max() <= 1e-12 * np.abs(G0).max()


def test_plan_structure_and_costs(plan3, plan5):
    b, plan = plan5
    for p in (plan3, plan):
        assert np.all(np.diff(p.seg_L) >= 0)
        assert np.array_equal(p.seg_offset, np.concatenate([[0], np.cumsum(2 * p.seg_L.astype(np.int64) + 1)]))
        assert np.array_equal(p.seg_L[p.dot_a], p.dot_L) and np.array_equal(p.seg_L[p.dot_b], p.dot_L)
        assert np.all(np.diff(p.dot_L) >= 0)
        assert np.unique(p.feat_index).shape[0] == p.feature_count
        assert p.feat_weight.dtype == np.float64
        pairs = p.seg_kind == SEG_PAIR
        assert np.all(p.seg_a[pairs] >= 0) and np.all(p.seg_b[pairs] >= 0)
        chans = p.seg_kind == SEG_CHANNEL
        ls = p.seg_a[chans] % (p.lmax + 1)
        assert np.array_equal(ls, p.seg_L[chans]) and np.all(p.seg_b[chans] == -1)
        assert int((p.seg_kind == SEG_UNIT).sum()) <= 1
    # the nu <= 4 set: one contraction per feature, and the per-atom work it needs
    assert plan.dot_count == plan.feature_count == 41168
    assert plan.costs() == {"pair_couplings": 20539, "contractions": 166072, "feature_weights": 57104,
                            "components": 6920}


def test_device_tables_walk_matches_oracle_and_validation_catches_damage(plan5):
    """The packed tables, walked loop for loop as the device pass walks them, give the
    oracle's energies and dE/dA; a damaged index is refused before any upload."""
    from oracle import oracle
    b, plan = plan5
    tabs = plan.device_tables()
    assert (tabs.pass_count, tabs.max_pass_components, tabs.row_width, tabs.dot_count) == (7, 2184, 128, 41168)
    assert tabs.smem_bytes() == 16 * (2 * 128 + 2 * 2184)
    assert tabs.dot_begin.tolist() == [0, 9260, 21018, 33932, 38500, 40888, 40958, 41168]
    # per-atom work of the passes, against 17.7 M (forward) / 33.7 M (adjoint) flops of the term-level walk
    fl = tabs.flops_per_atom()
    assert fl["energy"] < 1.7e6 and fl["energy_grad"] < 2.0e6 and fl["features"] < 1.8e6
    rng = np.random.default_rng(12)
    A = rng.normal(size=(3, 8, 16)) + 1j * rng.normal(size=(3, 8, 16))
    species = np.array([1, 0, 2], dtype=np.int32)
    w = rng.normal(size=(3, b.feature_count)) / np.sqrt(b.feature_count)
    e0, G0 = oracle.bundle_energy_grad(b, A, species, w, threads=4)
    e1, G1 = rn.walk_device_tables(tabs, A, species, plan.energy_weights(w))
    assert np.abs(e1 - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G1 - G0).max() <= 1e-12 * np.abs(G0).max()
    import copy
    F0 = oracle.bundle_features(b, A, threads=4)
    F1 = rn.walk_forward(tabs, A)
    assert np.abs(F1 - F0).max() <= 1e-12 * np.abs(F0).max()
    e2 = rn.walk_forward(tabs, A, species, plan.energy_weights(w))
    assert np.abs(e2 - e0).max() <= 1e-12 * np.abs(e0).max()
    for field, row, col, value in (("own", 5, 0, 10 ** 6), ("bp_gi", 3, None, -2), ("comp", 0, 0, 10 ** 4),
                                   ("dot", 7, 1, 10 ** 5), ("feat_index", 2, None, 10 ** 7)):
        bad = copy.deepcopy(tabs)
        arr = getattr(bad, field)
        if col is None:
            arr[row] = value
        else:
            arr[row, col] = value
        with pytest.raises(ValueError):
            bad.validate()


def test_recoupled_entry_point_checks_arguments_without_gpu(plan3):
    """The C entry points refuse null, misaligned and oversized tables before any CUDA call."""
    import ctypes

    import torch
    from ye3t_b200 import _native
    from ye3t_b200.recoupling import _TABLE_ARRAYS, ctypes_tables
    tabs = plan3.device_tables()
    arrays = {name: torch.as_tensor(np.ascontiguousarray(getattr(tabs, name))) for name in _TABLE_ARRAYS}
    ct = ctypes_tables(arrays, tabs)
    lib = _native.lib()
    f = lib.y3b_ace_recoupled_energy_grad
    assert f(ctypes.byref(ct), 0, 0, 0, 0, 1, 0, 0, 0, 0) == 0  # no atoms: nothing to do
    assert f(None, 0, 0, 0, 0, 1, 0, 0, 0, 0) == -1
    odd = ctypes_tables(arrays, tabs)
    odd.comp = ct.comp + 4
    assert f(ctypes.byref(odd), 0, 0, 0, 0, 1, 0, 0, 0, 0) == -1 and b"aligned" in lib.y3b_last_error()
    big = ctypes_tables(arrays, tabs)
    big.max_pass_components = 1 << 20
    assert f(ctypes.byref(big), 1, 4, 1, 1, 1, 1, 1, 0, 0) == -1 and b"shared memory" in lib.y3b_last_error()
    fe = lib.y3b_ace_recoupled_energy
    ff = lib.y3b_ace_recoupled_features
    assert fe(ctypes.byref(ct), 0, 0, 0, 0, 1, 0, 0, 0) == 0 and ff(ctypes.byref(ct), 0, 0, 0, 0, 0) == 0
    assert ff(ctypes.byref(ct), 1, 4, 0, 0, 0) == -1 and b"null features" in lib.y3b_last_error()
    assert fe(ctypes.byref(big), 1, 4, 1, 1, 1, 1, 0, 0) == -1 and b"shared memory" in lib.y3b_last_error()
    odd_dot = ctypes_tables(arrays, tabs)
    odd_dot.dot = ct.dot + 8
    assert ff(ctypes.byref(odd_dot), 1, 4, 1, 0, 0) == -1 and b"aligned" in lib.y3b_last_error()
    many = ctypes_tables(arrays, tabs)
    many.atoms_per_cta = 5
    assert f(ctypes.byref(many), 1, 4, 1, 1, 1, 1, 1, 0, 0) == -1 and b"atoms_per_cta" in lib.y3b_last_error()


def test_recoupled_atoms_per_cta_limited_by_shared_memory(plan5):
    """Four C5 atoms per CTA would need 296 KB of shared memory for the adjoint: refused
    before any CUDA call (three fit: 222 KB)."""
    import ctypes

    import torch
    from ye3t_b200 import _native
    from ye3t_b200.recoupling import _TABLE_ARRAYS, ctypes_tables
    tabs = plan5[1].device_tables()
    assert 3 * tabs.smem_bytes() <= 224 * 1024 < 4 * tabs.smem_bytes()
    arrays = {name: torch.as_tensor(np.ascontiguousarray(getattr(tabs, name))) for name in _TABLE_ARRAYS}
    ct = ctypes_tables(arrays, tabs)
    ct.atoms_per_cta = 4
    lib = _native.lib()
    assert lib.y3b_ace_recoupled_energy_grad(ctypes.byref(ct), 1, 4, 1, 1, 1, 1, 1, 0, 0) == -1
    assert b"4 atoms per CTA" in lib.y3b_last_error()


def test_plan_covers_channel_diagonal_l4_bundle():
    """The channel-diagonal nu <= 4, l <= 4 word set (intermediate L up to 8) recouples too."""
    from oracle import oracle
    b = _bundle("ace_diag_l4_nu4_L0")
    tabs = build_recoupled_plan(b).device_tables()
    assert tabs.pass_count == 7 and tabs.row_width == 25
    rng = np.random.default_rng(13)
    A = rng.normal(size=(6, 1, 25)) + 1j * rng.normal(size=(6, 1, 25))
    F0 = oracle.bundle_features(b, A, threads=2)
    assert np.abs(rn.walk_forward(tabs, A) - F0).max() <= 1e-12 * np.abs(F0).max()


@pytest.fixture(scope="module")
def emulated(tmp_path_factory):
    """The device source of the recoupled passes compiled as host C++ (tests/recoupled_emulation.cpp)."""
    import ctypes
    import shutil
    import subprocess
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no C++ compiler")
    out = tmp_path_factory.mktemp("emu") / "recoupled_emulation.so"
    subprocess.run([gxx, "-O2", "-std=c++20", "-pthread", "-fPIC", "-shared",
                    "-I", os.path.join(REPO, "include"), "-I", os.path.join(REPO, "ye3t_b200", "csrc"),
                    os.path.join(REPO, "tests", "recoupled_emulation.cpp"), "-o", str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    P, I64 = ctypes.c_void_p, ctypes.c_int64
    C = ctypes.c_int
    lib.emu_recoupled_energy_grad.argtypes = [C, C, P, P, I64, P, P, I64, P, P, P]
    lib.emu_recoupled_forward.argtypes = [C, C, C, P, P, I64, P, P, I64, P, P, P]
    return lib


def _emulate(lib, tabs, A, species, k, na, th=256):
    import ctypes

    import torch
    from ye3t_b200.recoupling import _TABLE_ARRAYS, ctypes_tables
    arrays = {name: torch.as_tensor(np.ascontiguousarray(getattr(tabs, name))) for name in _TABLE_ARRAYS}
    ct = ctypes_tables(arrays, tabs)
    n = A.shape[0]
    A = np.ascontiguousarray(A)
    sp = np.ascontiguousarray(species, dtype=np.int32)
    k = np.ascontiguousarray(k)
    e, G, e2 = np.zeros(n), np.zeros_like(A), np.zeros(n)
    F = np.zeros((n, tabs.feature_count), dtype=np.complex128)
    st = np.zeros(3, dtype=np.int32)
    ptr = lambda x: x.ctypes.data  # noqa: E731
    assert lib.emu_recoupled_energy_grad(na, th, ctypes.byref(ct), ptr(A), n, ptr(sp), ptr(k), k.shape[0],
                                         ptr(e), ptr(G), ptr(st)) == 0
    assert lib.emu_recoupled_forward(na, th, 0, ctypes.byref(ct), ptr(A), n, ptr(sp), ptr(k), k.shape[0], ptr(e2),
                                     None, st[1:].ctypes.data) == 0
    assert lib.emu_recoupled_forward(na, th, 1, ctypes.byref(ct), ptr(A), n, None, None, 0, None, ptr(F),
                                     st[2:].ctypes.data) == 0
    return e, G, e2, F, st


@pytest.fixture(scope="module")
def c5_case(plan5):
    """Five atoms (one of an out-of-range species) with the oracle's results."""
    from oracle import oracle
    b, plan = plan5
    rng = np.random.default_rng(30)
    A = rng.normal(size=(5, 8, 16)) + 1j * rng.normal(size=(5, 8, 16))
    species = np.array([0, 2, 1, 7, 1], dtype=np.int32)
    w = rng.normal(size=(3, b.feature_count)) / np.sqrt(b.feature_count)
    used = np.where(species >= 3, 0, species).astype(np.int32)
    e0, G0 = oracle.bundle_energy_grad(b, A, used, w, threads=4)
    F0 = oracle.bundle_features(b, A, threads=4)
    return A, species, plan.energy_weights(w), e0, G0, F0, w


@pytest.mark.parametrize("na, th", [(1, 256), (2, 256), (3, 256), (3, 512)])
def test_device_source_emulated_on_cpu_matches_oracle(emulated, plan5, c5_case, na, th):
    """The recoupled kernels' own source (recoupled_kernels.cuh), run on the CPU as one CTA of
    256 or 512 threads with real block barriers and warp exchanges, gives the oracle's energies,
    dE/dA and features for 1-3 atoms per CTA, including a partial last group and a species out
    of range (status INDEX_RANGE, species 0 used)."""
    A, species, k, e0, G0, F0, _ = c5_case
    e, G, e2, F, st = _emulate(emulated, plan5[1].device_tables(), A, species, k, na, th)
    assert st.tolist() == [1, 1, 0]
    assert np.abs(e - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(e2 - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G - G0).max() <= 1e-12 * np.abs(G0).max()
    assert np.abs(F - F0).max() <= 1e-12 * np.abs(F0).max()


def test_device_source_emulated_flags_damaged_tables(emulated, plan3):
    """Table entries outside their pass or array (a list partner, a back-propagation
    component, a contraction's segment, a coupling's A-row entry) set Y3B_STATUS_TABLE in
    the emulated device source and are skipped; the undamaged run sets nothing."""
    import copy

    from ye3t_b200 import _native
    tabs = plan3.device_tables()
    rng = np.random.default_rng(40)
    A = rng.normal(size=(2, 8, 16)) + 1j * rng.normal(size=(2, 8, 16))
    k = plan3.energy_weights(rng.normal(size=(3, tabs.feature_count)))
    species = np.array([0, 1], dtype=np.int32)
    assert _emulate(emulated, tabs, A, species, k, 1)[4].tolist() == [0, 0, 0]
    pair = int(np.nonzero(tabs.comp[:, 3] > 0)[0][0])
    for field, index, value in (("own", (3, 0), 10 ** 6), ("bp_gi", (5,), 10 ** 6), ("dot", (2, 1), 10 ** 6),
                                ("comp", (pair, 1), 10 ** 6)):
        bad = copy.deepcopy(tabs)
        getattr(bad, field)[index] = value
        st = _emulate(emulated, bad, A, species, k, 2)[4]
        assert st[0] & _native.STATUS_TABLE or st[1] & _native.STATUS_TABLE, field


def test_device_source_emulated_channel_diagonal_bundle(emulated):
    """A row of 25 entries (l <= 4, one channel) in the emulated device source: rows that do
    not divide the block, and back-propagation without the split (too few components to stage
    the parts)."""
    from oracle import oracle
    b = _bundle("ace_diag_l4_nu4_L0")
    plan = build_recoupled_plan(b)
    tabs = plan.device_tables()
    assert tabs.max_pass_components < (256 // tabs.row_width) * tabs.row_width
    rng = np.random.default_rng(50)
    A = rng.normal(size=(5, 1, 25)) + 1j * rng.normal(size=(5, 1, 25))
    species = np.array([0, 1, 0, 1, 1], dtype=np.int32)
    w = rng.normal(size=(2, b.feature_count))
    e0, G0 = oracle.bundle_energy_grad(b, A, species, w, threads=2)
    F0 = oracle.bundle_features(b, A, threads=2)
    for na, th in ((2, 256), (4, 512)):
        e, G, e2, F, st = _emulate(emulated, tabs, A, species, plan.energy_weights(w), na, th)
        assert st.tolist() == [0, 0, 0]
        assert np.abs(e - e0).max() <= 1e-12 * np.abs(e0).max()
        assert np.abs(e2 - e0).max() <= 1e-12 * np.abs(e0).max()
        assert np.abs(G - G0).max() <= 1e-12 * np.abs(G0).max()
        assert np.abs(F - F0).max() <= 1e-12 * np.abs(F0).max()


def test_evaluator_glue_through_emulated_entry_points(emulated, plan5, c5_case, monkeypatch):
    """RecoupledEvaluator's energy_grad / energy / features with their real ctypes bindings
    (_native._SIGS), the library swapped for the emulation harness, on CPU tensors: the same
    argument order, table struct and shapes as on the GPU, against the oracle."""
    import ctypes

    import torch
    from ye3t_b200 import _native
    from ye3t_b200.recoupling import RecoupledEvaluator
    for name in ("y3b_ace_recoupled_energy_grad", "y3b_ace_recoupled_energy", "y3b_ace_recoupled_features"):
        res, args = _native._SIGS[name]
        getattr(emulated, name).restype = res
        getattr(emulated, name).argtypes = args
    emulated.y3b_last_error.restype = ctypes.c_char_p
    monkeypatch.setattr(_native, "lib", lambda: emulated)
    monkeypatch.setattr(_native, "require_cuda", lambda *t, what="": torch.device("cpu"))
    monkeypatch.setattr(_native, "stream_of", lambda device: 0)
    b, plan = plan5
    A, species, _, e0, G0, F0, w = c5_case
    used = np.where(species >= 3, 0, species).astype(np.int32)
    ev = RecoupledEvaluator(b, "cpu", w, plan=plan, atoms_per_cta=2, threads_per_cta=512)
    st = torch.zeros(1, dtype=torch.int32)
    At, st_sp = torch.as_tensor(A), torch.as_tensor(used)
    e, G = ev.energy_grad(At, st_sp, status=st)
    e2 = ev.energy(At, st_sp, status=st)
    F = ev.features(At, status=st)
    assert int(st.item()) == 0
    assert np.abs(e.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(e2.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G.numpy() - G0).max() <= 1e-12 * np.abs(G0).max()
    assert np.abs(F.numpy() - F0).max() <= 1e-12 * np.abs(F0).max()
    with pytest.raises(ValueError):
        ev.energy_grad(At[:, :4], st_sp)


@pytest.fixture(scope="module")
def physical_case(plan5, golden):
    """Six atoms of the golden 96-atom system (physical densities from the reference) with
    the oracle's energies and dE/dA."""
    from oracle import oracle
    b, plan = plan5
    g = golden("ace_small")
    A = np.ascontiguousarray(np.asarray(g["A"])[:6])
    species = np.asarray(g["species"])[:6].astype(np.int32)
    w = np.random.default_rng(60).normal(size=(3, b.feature_count)) / np.sqrt(b.feature_count)
    e0, G0 = oracle.bundle_energy_grad(b, A, species, w, threads=4)
    return A, species, w, e0, G0


def test_symmetric_tables_walk_matches_oracle_on_physical_densities(plan5, physical_case):
    """The M >= 0 tables of the symmetric passes, walked loop for loop on the reference's own
    densities, give the oracle's energies and dE/dA; they hold 59 % of the components."""
    b, plan = plan5
    tabs = plan.sym_device_tables()
    assert (tabs.comp.shape[0], tabs.max_pass_components) == (4114, 1248)
    assert 4 * tabs.smem_bytes() <= 224 * 1024
    A, species, w, e0, G0 = physical_case
    k = plan.energy_weights(w)
    e1, G1 = rn.walk_sym_tables(tabs, A, species, k)
    e2 = rn.walk_sym_forward(tabs, A, species, k)
    assert np.abs(e1 - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(e2 - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G1 - G0).max() <= 1e-12 * np.abs(G0).max()


def test_symmetric_tables_refuse_an_odd_parity_word_set(plan5):
    """The symmetric passes need both segments of every contraction to share their parity,
    which holds for parity-even word sets only: a contraction of an odd pair with an even
    segment is refused."""
    import copy

    from ye3t_b200.recoupling import SEG_PAIR
    plan = copy.deepcopy(plan5[1])
    pairs = np.nonzero(plan.seg_kind == SEG_PAIR)[0]
    odd = [int(s) for s in pairs if (plan.seg_a[s] % 4 + plan.seg_b[s] % 4 - plan.seg_L[s]) % 2]
    assert odd
    L = int(plan.seg_L[odd[0]])
    even = [s for s in range(plan.segment_count) if s not in set(odd) and int(plan.seg_L[s]) == L]
    d = int(np.nonzero(plan.dot_L == L)[0][0])
    plan.dot_a[d], plan.dot_b[d] = odd[0], even[0]
    with pytest.raises(ValueError, match="parity-even"):
        plan.sym_device_tables()


@pytest.mark.parametrize("na, th", [(1, 256), (4, 256), (3, 512)])
def test_symmetric_device_source_emulated_matches_oracle(emulated, plan5, physical_case, na, th, monkeypatch):
    """The symmetric kernels' own source, emulated on the CPU through RecoupledEvaluator's real
    ctypes bindings (symmetric=True), on the reference's densities: the oracle's energies and
    dE/dA, with dE/dA's m < 0 half mirrored."""
    import ctypes

    import torch
    from ye3t_b200 import _native
    from ye3t_b200.recoupling import RecoupledEvaluator
    for name in ("y3b_ace_recoupled_energy_grad_symmetric", "y3b_ace_recoupled_energy_symmetric"):
        res, args = _native._SIGS[name]
        getattr(emulated, name).restype = res
        getattr(emulated, name).argtypes = args
    emulated.y3b_last_error.restype = ctypes.c_char_p
    monkeypatch.setattr(_native, "lib", lambda: emulated)
    monkeypatch.setattr(_native, "require_cuda", lambda *t, what="": torch.device("cpu"))
    monkeypatch.setattr(_native, "stream_of", lambda device: 0)
    b, plan = plan5
    A, species, w, e0, G0 = physical_case
    ev = RecoupledEvaluator(b, "cpu", w, plan=plan, atoms_per_cta=na, threads_per_cta=th, symmetric=True)
    st = torch.zeros(1, dtype=torch.int32)
    At, sp = torch.as_tensor(A), torch.as_tensor(species)
    e, G = ev.energy_grad(At, sp, status=st)
    e2 = ev.energy(At, sp, status=st)
    assert int(st.item()) == 0
    assert np.abs(e.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(e2.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G.numpy() - G0).max() <= 1e-12 * np.abs(G0).max()
    with pytest.raises(ValueError, match="general passes"):
        ev.features(At)


def _physical(rng, n, nmax, lmax):
    """Random densities with the physical symmetry A[l, -m] = (-1)^m conj(A[l, m])."""
    A = np.zeros((n, nmax, (lmax + 1) ** 2), dtype=np.complex128)
    for l in range(lmax + 1):
        for m in range(0, l + 1):
            v = rng.normal(size=(n, nmax)) + (1j * rng.normal(size=(n, nmax)) if m else 0)
            A[:, :, l * l + l + m] = v
            A[:, :, l * l + l - m] = (-1) ** m * np.conj(v)
    return A


def test_symmetric_device_source_emulated_channel_diagonal(emulated, monkeypatch):
    """The symmetric kernels' source on the 25-entry rows of the channel-diagonal l <= 4
    bundle (back-propagation unsplit, rows that do not divide the block), emulated through
    the real bindings, against the oracle."""
    import ctypes

    import torch
    from oracle import oracle
    from ye3t_b200 import _native
    from ye3t_b200.recoupling import RecoupledEvaluator
    for name in ("y3b_ace_recoupled_energy_grad_symmetric", "y3b_ace_recoupled_energy_symmetric"):
        res, args = _native._SIGS[name]
        getattr(emulated, name).restype = res
        getattr(emulated, name).argtypes = args
    emulated.y3b_last_error.restype = ctypes.c_char_p
    monkeypatch.setattr(_native, "lib", lambda: emulated)
    monkeypatch.setattr(_native, "require_cuda", lambda *t, what="": torch.device("cpu"))
    monkeypatch.setattr(_native, "stream_of", lambda device: 0)
    b = _bundle("ace_diag_l4_nu4_L0")
    rng = np.random.default_rng(70)
    A = _physical(rng, 7, 1, 4)
    species = np.array([0, 1, 1, 0, 1, 0, 0], dtype=np.int32)
    w = rng.normal(size=(2, b.feature_count))
    e0, G0 = oracle.bundle_energy_grad(b, A, species, w, threads=2)
    for na, th in ((3, 256), (4, 512)):
        ev = RecoupledEvaluator(b, "cpu", w, atoms_per_cta=na, threads_per_cta=th, symmetric=True)
        e, G = ev.energy_grad(torch.as_tensor(A), torch.as_tensor(species))
        e2 = ev.energy(torch.as_tensor(A), torch.as_tensor(species))
        assert np.abs(e.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
        assert np.abs(e2.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
        assert np.abs(G.numpy() - G0).max() <= 1e-12 * np.abs(G0).max()


def test_symmetry_check_refuses_non_physical_densities(plan5, physical_case):
    """RecoupledEvaluator.check_symmetry passes the reference's densities and refuses random
    complex ones (for which the symmetric passes would be wrong)."""
    import torch
    from ye3t_b200.recoupling import RecoupledEvaluator
    b, plan = plan5
    A, species, w, _, _ = physical_case
    ev = RecoupledEvaluator(b, "cpu", w, plan=plan, symmetric=True)
    ev.check_symmetry(torch.as_tensor(A))
    rng = np.random.default_rng(80)
    with pytest.raises(ValueError, match="physical symmetry"):
        ev.check_symmetry(torch.as_tensor(rng.normal(size=(2, 8, 16)) + 1j * rng.normal(size=(2, 8, 16))))


def _sub_bundle(b, keep):
    """The words of ``b`` that ``keep(word)`` accepts, with ``b``'s own compiled patterns."""
    import dataclasses
    sel = np.asarray([i for i, w in enumerate(b.words) if keep(w)], dtype=np.int64)
    return dataclasses.replace(b, words=[b.words[i] for i in sel], word_pattern_index=b.word_pattern_index[sel],
                               word_n_map=b.word_n_map[sel])


def test_emulated_adjoint_with_fewer_pass_components_than_row_entries(emulated, monkeypatch):
    """The nu <= 2 words of the n_max 8, l_max 3 set have passes of at most 64 components
    against rows of 128 entries; the adjoint's back-propagation still stages a part per row
    entry in the component region, which the kernels and the launch size as at least a row
    wide.  General and symmetric passes, emulated, against the oracle."""
    import ctypes

    import torch
    from oracle import oracle
    from ye3t_b200 import _native
    from ye3t_b200.recoupling import RecoupledEvaluator
    b = _sub_bundle(_bundle("ace_n8_l3_nu3_L0"), lambda w: len(w) <= 2)
    plan = build_recoupled_plan(b)
    gen, sym = plan.device_tables(), plan.sym_device_tables()
    assert gen.max_pass_components < gen.row_width and sym.max_pass_components < sym.row_width
    assert gen.smem_bytes() == 16 * 4 * gen.row_width
    rng = np.random.default_rng(60)
    A = _physical(rng, 5, 8, 3)
    species = np.array([0, 1, 2, 1, 0], dtype=np.int32)
    w = rng.normal(size=(3, b.feature_count))
    e0, G0 = oracle.bundle_energy_grad(b, A, species, w, threads=2)
    for na, th in ((1, 256), (3, 512)):
        e, G, _, _, st = _emulate(emulated, gen, A, species, plan.energy_weights(w), na, th)
        assert st.tolist() == [0, 0, 0]
        assert np.abs(e - e0).max() <= 1e-12 * np.abs(e0).max()
        assert np.abs(G - G0).max() <= 1e-12 * np.abs(G0).max()
    for name in ("y3b_ace_recoupled_energy_grad_symmetric", "y3b_ace_recoupled_energy_symmetric"):
        res, args = _native._SIGS[name]
        getattr(emulated, name).restype = res
        getattr(emulated, name).argtypes = args
    emulated.y3b_last_error.restype = ctypes.c_char_p
    monkeypatch.setattr(_native, "lib", lambda: emulated)
    monkeypatch.setattr(_native, "require_cuda", lambda *t, what="": torch.device("cpu"))
    monkeypatch.setattr(_native, "stream_of", lambda device: 0)
    ev = RecoupledEvaluator(b, "cpu", w, plan=plan, atoms_per_cta=2, threads_per_cta=256, symmetric=True)
    st = torch.zeros(1, dtype=torch.int32)
    e, G = ev.energy_grad(torch.as_tensor(A), torch.as_tensor(species), status=st)
    assert int(st.item()) == 0
    assert np.abs(e.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G.numpy() - G0).max() <= 1e-12 * np.abs(G0).max()


@pytest.mark.parametrize("rows", [8, 16])
def test_symmetric_tiles_walk_matches_oracle(plan5, physical_case, rows):
    """The contraction lists regrouped as dense tiles of 8 or 16 segments (every contraction
    lands in exactly two tile entries, or twice in one on the diagonal): the tiled walk gives
    the oracle's energies and dE/dA on the reference's densities, and the tiles keep most of
    their entries nonzero."""
    from ye3t_b200.recoupling import TILE_STEP
    b, plan = plan5
    tabs = plan.sym_device_tables()
    tiles = plan.sym_tiles(rows)
    assert tiles.efficiency() > (0.8 if rows == 8 else 0.65)
    assert np.all(np.diff(tiles.tile_col_begin) % TILE_STEP == 0)
    A, species, w, e0, G0 = physical_case
    k = plan.energy_weights(w)
    kv = tiles.tile_weights(k)
    assert np.isclose(kv.sum(), 2 * k.sum())
    e1, G1 = rn.walk_sym_tiled(tabs, tiles, A, species, k)
    assert np.abs(e1 - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G1 - G0).max() <= 1e-12 * np.abs(G0).max()


def _bind_emulated(emulated, monkeypatch, names):
    import ctypes

    import torch
    from ye3t_b200 import _native
    for name in names:
        res, args = _native._SIGS[name]
        getattr(emulated, name).restype = res
        getattr(emulated, name).argtypes = args
    emulated.y3b_last_error.restype = ctypes.c_char_p
    monkeypatch.setattr(_native, "lib", lambda: emulated)
    monkeypatch.setattr(_native, "require_cuda", lambda *t, what="": torch.device("cpu"))
    monkeypatch.setattr(_native, "stream_of", lambda device: 0)


@pytest.mark.parametrize("rows, th", [(8, 256), (8, 512)])
def test_tiled_device_source_emulated_matches_oracle(emulated, plan5, physical_case, rows, th, monkeypatch):
    """The tiled symmetric adjoint's own source (recoupled_sym_tiled_grad_kernel), emulated on
    the CPU through RecoupledEvaluator's real bindings: 4 atoms per CTA grouped in species
    order (a partial last group), step 2 from the warps' staging rings; the oracle's energies
    and dE/dA, with no status set."""
    import torch
    from ye3t_b200.recoupling import RecoupledEvaluator
    _bind_emulated(emulated, monkeypatch, ["y3b_ace_recoupled_energy_grad_tiled"])
    b, plan = plan5
    A, species, w, e0, G0 = physical_case
    ev = RecoupledEvaluator(b, "cpu", w, plan=plan, threads_per_cta=th, symmetric=True, tile_rows=rows)
    st = torch.zeros(1, dtype=torch.int32)
    e, G = ev.energy_grad(torch.as_tensor(A), torch.as_tensor(species), status=st)
    assert int(st.item()) == 0
    assert np.abs(e.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G.numpy() - G0).max() <= 1e-12 * np.abs(G0).max()
    # a damaged tile column is skipped and reported
    from ye3t_b200 import _native
    ev.tile_arrays["col_comp"][5] = 1 << 20
    st.zero_()
    ev.energy_grad(torch.as_tensor(A), torch.as_tensor(species), status=st)
    assert int(st.item()) & _native.STATUS_TABLE


@pytest.mark.parametrize("stem", ["ace_diag_l4_nu4_L0", "nu2"])
def test_tiled_device_source_emulated_small_rows(emulated, stem, monkeypatch):
    """The tiled adjoint on rows of 25 entries (l_max 4, intermediate L up to 8) and on the
    nu <= 2 words of the n_max 8 set (passes smaller than the row), emulated through the real
    bindings, against the oracle."""
    import torch
    from oracle import oracle
    from ye3t_b200.recoupling import RecoupledEvaluator
    _bind_emulated(emulated, monkeypatch, ["y3b_ace_recoupled_energy_grad_tiled"])
    if stem == "nu2":
        b = _sub_bundle(_bundle("ace_n8_l3_nu3_L0"), lambda w: len(w) <= 2)
        nmax, lmax, S = 8, 3, 3
    else:
        b = _bundle(stem)
        nmax, lmax, S = 1, 4, 2
    plan = build_recoupled_plan(b)
    rng = np.random.default_rng(61)
    A = _physical(rng, 6, nmax, lmax)
    species = rng.integers(0, S, 6).astype(np.int32)
    w = rng.normal(size=(S, b.feature_count))
    e0, G0 = oracle.bundle_energy_grad(b, A, species, w, threads=2)
    ev = RecoupledEvaluator(b, "cpu", w, plan=plan, threads_per_cta=256, symmetric=True, tile_rows=8)
    st = torch.zeros(1, dtype=torch.int32)
    e, G = ev.energy_grad(torch.as_tensor(A), torch.as_tensor(species), status=st)
    assert int(st.item()) == 0
    assert np.abs(e.numpy() - e0).max() <= 1e-12 * np.abs(e0).max()
    assert np.abs(G.numpy() - G0).max() <= 1e-12 * np.abs(G0).max()
