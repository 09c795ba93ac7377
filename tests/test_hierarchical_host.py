"""Hierarchical repeated-block plans (``block_symmetric_power``) on the host:
the oracle restatement and the product's lowering against the reference
module's outputs (``tests/golden/hierarchical.npz``), and the plan checks."""

import copy
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import hierarchical as oh
from ye3t_b200 import hierarchical as H


def _text(g, name):
    if "plan_" + name in g:
        return str(g["plan_" + name])
    return str(g["lammps_file_" + str(g["planfile_" + name])])


def _inputs(g, name):
    xs, b = [], 0
    while f"x{b}_{name}" in g:
        xs.append(g[f"x{b}_{name}"])
        b += 1
    return xs


def test_oracle_matches_reference_module(golden):
    g = golden("hierarchical")
    assert len(g["names"]) == 30
    for name in map(str, g["names"]):
        ref = g["y_" + name]
        y = oh.forward(_text(g, name), _inputs(g, name))
        assert y.shape == ref.shape, name
        assert np.abs(y - ref).max() <= 1e-13 * max(np.abs(ref).max(), 1.0), name


def test_lowered_schedule_matches_reference_module(golden):
    """The product's lowering (monomial tables + one factorized schedule with the
    routes and LR analysis folded in), evaluated here with numpy."""
    g = golden("hierarchical")
    for name in map(str, g["names"]):
        low = H.lower_hierarchical_instruction(_text(g, name))
        xs = _inputs(g, name)
        N = xs[0].shape[0]
        bv = np.zeros((N, low.block_count, low.block_width), dtype=np.complex128)
        for b, L, start, D, counts, offsets, index, values in low.power_tables:
            bv[:, b, start:start + D] = oh.power_eval(xs[b], counts, offsets, values)
        out = np.zeros((N, low.offsets.shape[0] - 1), dtype=np.complex128)
        for comp in range(out.shape[1]):
            for t in range(low.offsets[comp], low.offsets[comp + 1]):
                term = np.full(N, low.coeffs[t])
                for b in range(low.block_count):
                    term = term * bv[:, b, low.m_idx[t, b]]
                out[:, comp] += term
        ref = g["y_" + name].reshape(N, -1)
        assert out.shape[1] == low.output_dimension
        assert np.abs(out - ref).max() <= 1e-13 * max(np.abs(ref).max(), 1.0), name


def test_lowering_rejects_what_the_reference_rejects(golden):
    g = golden("hierarchical")
    plan = json.loads(_text(g, "r4"))
    for mutate, message in (
            (lambda p: p["instructions"][0].__setitem__("opcode", "coupled_product"), "block_symmetric_power"),
            (lambda p: p["instructions"][0]["metadata"].__setitem__("schema", "v9"), "schema"),
            (lambda p: p["instructions"][0]["metadata"].__setitem__("runtime_path_discovery", True),
             "path discovery"),
            (lambda p: p["instructions"][0]["metadata"]["routes"].reverse(), "canonical contiguous"),
            (lambda p: p["instructions"][0]["metadata"]["block_power_plans"].append(
                copy.deepcopy(p["instructions"][0]["metadata"]["block_power_plans"][0])), "duplicate")):
        bad = copy.deepcopy(plan)
        mutate(bad)
        with pytest.raises(ValueError, match=message):
            H.lower_hierarchical_instruction(bad)
    with pytest.raises(ValueError, match="instruction_id"):
        H.lower_hierarchical_instruction(plan, instruction_id="missing")


def test_scalar_ace_manifest_rejects_a_changed_plan(golden, tmp_path):
    g = golden("hierarchical")
    manifest = json.loads(str(g["lammps_manifest"]))
    for case in manifest["cases"]:
        name = case["execution_plan"]["file"]
        (tmp_path / name).write_text(str(g["lammps_file_" + name]), encoding="utf-8")
        assert hashlib.sha256((tmp_path / name).read_bytes()).hexdigest() == case["execution_plan"]["sha256"]
    first = manifest["cases"][0]["execution_plan"]["file"]
    (tmp_path / first).write_text(str(g["lammps_file_" + first]) + " ", encoding="utf-8")
    (tmp_path / "manifest.json").write_text(json.dumps(manifest), encoding="utf-8")
    with pytest.raises(ValueError, match="SHA-256"):
        H.load_scalar_ace_plans(os.fspath(tmp_path / "manifest.json"))
    manifest["schema"] = "something_else"
    (tmp_path / "manifest.json").write_text(json.dumps(manifest), encoding="utf-8")
    with pytest.raises(ValueError, match="manifest"):
        H.load_scalar_ace_plans(os.fspath(tmp_path / "manifest.json"))


def test_block_power_lowering_checks_and_merges(golden):
    """The grouped lowering merges terms with equal exponent rows, drops zero rows and rejects
    indices outside the plan (symmetric_power.py:740-868)."""
    g = golden("hierarchical")
    plan = json.loads(_text(g, "r4"))["instructions"][0]["metadata"]["block_power_plans"][1]["plan"]
    counts, offsets, index, values = H.lower_block_power_plan(plan)
    assert offsets[0] == 0 and offsets[-1] == counts.shape[0] == index.shape[0] == values.shape[0]
    assert np.all(np.diff(offsets) >= 0) and np.all(np.abs(values) > 1e-12)
    for d in range(offsets.shape[0] - 1):
        rows = [tuple(r) for r in counts[offsets[d]:offsets[d + 1]]]
        assert rows == sorted(set(rows))  # merged and ordered per descriptor
        assert np.all(index[offsets[d]:offsets[d + 1]] == d)
    doubled = copy.deepcopy(plan)
    for entry in doubled["entries"]:
        entry["component_terms"] = entry["component_terms"] * 2
    c2, o2, i2, v2 = H.lower_block_power_plan(doubled)
    assert np.array_equal(c2, counts) and np.allclose(v2, 2 * values)
    bad = copy.deepcopy(plan)
    bad["entries"][0]["descriptor_index"] = int(plan["descriptor_count"])
    with pytest.raises(ValueError, match="descriptor index"):
        H.lower_block_power_plan(bad)
    bad = copy.deepcopy(plan)
    bad["entries"][0]["channel_indices"] = [int(plan["channel_count"])] * len(bad["entries"][0]["channel_indices"])
    with pytest.raises(ValueError, match="channel index"):
        H.lower_block_power_plan(bad)


def test_scalar_ace_manifest_rejects_a_changed_plan_hash(golden, tmp_path):
    g = golden("hierarchical")
    manifest = json.loads(str(g["lammps_manifest"]))
    for case in manifest["cases"]:
        name = case["execution_plan"]["file"]
        (tmp_path / name).write_text(str(g["lammps_file_" + name]), encoding="utf-8")
    manifest["cases"][0]["execution_plan"]["plan_hash"] = "0" * 16
    (tmp_path / "manifest.json").write_text(json.dumps(manifest), encoding="utf-8")
    with pytest.raises(ValueError, match="plan hash"):
        H.load_scalar_ace_plans(os.fspath(tmp_path / "manifest.json"))
