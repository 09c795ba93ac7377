"""Hierarchical repeated-block instructions (``block_symmetric_power``) on B200.

``YE3THierarchicalRepeatedBlockModule`` keeps the constructor, ``forward``,
``forward_flat``, ``linear_readout``, ``block_power_requests`` and
``runtime_report`` of the reference module (ye3t/runtime/hierarchical.py:79-607)
and reads the same compiler-written execution plans (a plan dict, its JSON
text or a JSON file, or any object with ``to_json``).  The plan's arithmetic
is lowered once on the host into the two operations this package already runs
on the GPU:

1. every block power plan (block b, output L) becomes a grouped monomial
   table (the lowering of ``_symmetric_power_product_plan_count_table``,
   ye3t/runtime/symmetric_power.py:740-868) evaluated by
   ``y3b_symmetric_power_monomial``; block b's descriptors, all its L in
   increasing order, form one row of a ``[batch, 1, blocks, D]`` block array;
2. the routes and the Littlewood-Richardson analysis are multilinear in those
   descriptors, so each output component (channel = route x LR multiplicity,
   tableau, magnetic) is a list of terms ``coefficient x prod_b
   descriptor_b[index_b]`` evaluated by ``y3b_factorized_schedule_evaluate``.
   The coefficient folds ``conj(lr[mu, tau])`` into the route's own factor:
   one for a single-block selection (hierarchical.py:474-476),
   ``conj(CG[i (2L_r + 1) + j, M])`` for each nonzero entry of a two-block
   binary CG table (hierarchical.py:478-497), ``conj(value)`` for each entry
   of a schema-v2 sparse route (hierarchical.py:437-472).

Both GPU operations carry first-order autograd (their vector-Jacobian
products run on the GPU), so the module is differentiable once with respect
to its block inputs; second derivatives are not supported.  ``load_scalar_ace_plans`` reads the scalar
ACE LAMMPS export (ye3t/scalar_ace_export.py:52-114): its manifest, each plan
file checked against the recorded SHA-256 and plan hash, one module per
exported coordinate.
"""

from __future__ import annotations

import hashlib
import json
import math
import os

import numpy as np
import torch

from .couplings import evaluate_factorized_schedule_torch
from .runtime import symmetric_power_monomial_contraction

__all__ = ["YE3THierarchicalRepeatedBlockModule", "load_scalar_ace_plans", "lower_block_power_plan",
           "lower_hierarchical_instruction"]

_SCHEMAS = ("ye3t_hierarchical_repeated_angular_blocks_v1", "ye3t_hierarchical_repeated_angular_blocks_v2")
_MANIFEST_SCHEMA = "ye3t_scalar_ace_lammps_plan_example_v1"


def _cplx(v):
    if isinstance(v, (list, tuple)):
        return complex(float(v[0]), float(v[1]))
    return complex(v)


def _plan_dict(execution_plan):
    if isinstance(execution_plan, dict):
        return execution_plan
    if isinstance(execution_plan, (str, os.PathLike)):
        text = str(execution_plan)
        if not text.lstrip().startswith("{") and os.path.exists(text):
            with open(text, encoding="utf-8") as fh:
                text = fh.read()
        return json.loads(text)
    if hasattr(execution_plan, "to_json"):
        return json.loads(execution_plan.to_json())
    raise TypeError("execution_plan must be a plan dict, JSON text or path, or an object with to_json()")


def lower_block_power_plan(plan, imag_tol=1e-12):
    """Grouped monomial table of one symmetric-power product plan (dict form).

    Terms of a descriptor with the same exponent row over the plan's channels
    are merged, rows whose merged coefficient is at most ``imag_tol`` dropped,
    and each descriptor's rows sorted by exponent row, as the reference's
    lowering does.  Returns ``(counts [T, channel_count] int64, offsets
    [descriptor_count + 1] int64, output_index [T] int64, values [T] complex)``.
    """
    C, D = int(plan["channel_count"]), int(plan["descriptor_count"])
    merged = {}
    for entry in plan["entries"]:
        d = int(entry["descriptor_index"])
        if not 0 <= d < D:
            raise ValueError("symmetric-power plan descriptor index is outside descriptor_count")
        channels = [int(v) for v in entry["channel_indices"]]
        for term in entry["component_terms"]:
            exps = [int(v) for v in term["exponents"]]
            if len(exps) != len(channels):
                raise ValueError("symmetric-power plan exponent width does not match its channel indices")
            counts = [0] * C
            for local, e in enumerate(exps):
                if not 0 <= channels[local] < C:
                    raise ValueError("symmetric-power plan channel index is outside channel_count")
                counts[channels[local]] += e
            key = (d, tuple(counts))
            merged[key] = merged.get(key, 0j) + _cplx(term["coefficient"])
    by_desc = [[] for _ in range(D)]
    for (d, counts), v in merged.items():
        if abs(v) > imag_tol:
            by_desc[d].append((counts, v))
    rows, offsets = [], [0]
    for d in range(D):
        rows.extend((d, c, v) for c, v in sorted(by_desc[d], key=lambda cv: cv[0]))
        offsets.append(len(rows))
    counts = np.asarray([r[1] for r in rows], dtype=np.int64).reshape(-1, C)
    return (counts, np.asarray(offsets, dtype=np.int64), np.asarray([r[0] for r in rows], dtype=np.int64),
            np.asarray([r[2] for r in rows], dtype=np.complex128))


class _LoweredSchedule:
    """Factorized-schedule tables (the fields ``couplings.packed_schedule_tables`` reads)."""

    def __init__(self, offsets, m_idx, coeffs, block_count, max_m):
        comps = int(offsets.shape[0]) - 1
        self.component_offsets = torch.as_tensor(offsets, dtype=torch.int64)
        self.component_label_index = torch.zeros(comps, dtype=torch.int64)
        self.block_m_indices = torch.as_tensor(m_idx, dtype=torch.int64).reshape(-1, block_count)
        self.term_component_index = torch.repeat_interleave(torch.arange(comps),
                                                            torch.diff(self.component_offsets))
        self.coeffs = torch.as_tensor(coeffs, dtype=torch.complex128)
        self.component_count, self.block_count, self.basis_count, self.max_block_m_dim = comps, block_count, 1, max_m


def _dense(table):
    M = np.zeros((int(table["input_dimension"]), int(table["output_dimension"])), dtype=np.complex128)
    for r, c, v in zip(table["row_indices"], table["column_indices"], table["values"]):
        M[int(r), int(c)] += _cplx(v)
    return M


class HierarchicalLowering:
    """Host tables of one lowered ``block_symmetric_power`` instruction (numpy).

    ``power_tables``: per (block, L) ``(block, L, start, D, counts, offsets,
    output_index, values)``, the descriptors landing at ``[start, start + D)``
    of the block's row (``block_width`` = the widest row).  The schedule, per
    output component (channel, tableau, magnetic, in the output's flat order):
    ``offsets [components + 1]`` into its terms, ``m_idx [T, blocks]`` the
    descriptor each term reads from each block, ``coeffs [T]``.  The plan's
    identity and layout fields (``plan_hash``, ``channel_count``, ...) are
    copied as the reference module exposes them.
    """


def lower_hierarchical_instruction(execution_plan, instruction_id=None):
    """Validate one ``block_symmetric_power`` instruction as the reference
    constructor does (hierarchical.py:82-405) and lower it (module docstring)."""
    plan = _plan_dict(execution_plan)
    instructions = {str(i["instruction_id"]): i for i in plan["instructions"]}
    if instruction_id is None:
        if len(plan["forward_schedule"]) != 1:
            raise ValueError("instruction_id is required for a multi-instruction plan")
        instruction_id = plan["forward_schedule"][0]
    instruction_id = str(instruction_id)
    if instruction_id not in instructions:
        raise ValueError("instruction_id is not present in the execution plan")
    ins = instructions[instruction_id]
    md = dict(ins["metadata"])
    if ins["opcode"] != "block_symmetric_power":
        raise ValueError("hierarchical repeated-block runtime requires block_symmetric_power")
    schema = md.get("schema")
    if schema not in _SCHEMAS:
        raise ValueError("unsupported hierarchical repeated-block schema")
    if bool(md.get("runtime_path_discovery", True)):
        raise ValueError("hierarchical runtime forbids runtime path discovery")
    if bool(md.get("raw_angular_tree_forest_materialized", True)):
        raise ValueError("hierarchical runtime forbids raw angular tree forests")

    low = HierarchicalLowering()
    blocks = tuple(dict(b) for b in md["blocks"])
    powers = {}
    for rec in md["block_power_plans"]:
        key = (int(rec["block_index"]), int(rec["output_L"]))
        if key in powers:
            raise ValueError("duplicate hierarchical block power plan")
        if int(rec["plan"]["channel_count"]) != 2 * int(blocks[key[0]]["input_L"]) + 1:
            raise ValueError("hierarchical block power input width is inconsistent")
        powers[key] = rec["plan"]
    if not powers:
        raise ValueError("hierarchical instruction has no block power plans")
    tables = {t["table_id"]: t for t in plan["synthesis_tables"]}
    if str(md["lr_synthesis_table_id"]) not in tables:
        raise ValueError("hierarchical LR synthesis table is missing")
    lr = _dense(tables[str(md["lr_synthesis_table_id"])])
    routes = tuple(dict(r) for r in md["routes"])
    if tuple(int(r["route_index"]) for r in routes) != tuple(range(len(routes))):
        raise ValueError("hierarchical routes must use canonical contiguous indices")
    out_key = json.dumps(ins["output_carrier"], sort_keys=True)
    layouts = [lay for lay in plan["carrier_layouts"] if json.dumps(lay["key"], sort_keys=True) == out_key]
    if len(layouts) != 1:
        raise ValueError("hierarchical instruction must have one output layout")
    layout = layouts[0]

    low.instruction_id = instruction_id
    low.plan_hash = str(plan.get("plan_hash", ""))
    low.coefficient_hash = str(plan.get("coefficient_hash", ""))
    low.channel_count = int(layout["channel_count"])
    low.tableau_count = int(layout["tableau_count"])
    low.magnetic_count = int(layout["magnetic_count"])
    low.output_dimension = int(layout["width"])
    low.target_L = int(md["target_L"])
    low.target_parity = md.get("target_parity")
    low.lr_multiplicity = int(md["lr_multiplicity"])
    low.block_count = len(blocks)
    low.route_count = len(routes)
    low.hierarchical_schema = str(schema)
    low.blocks = blocks
    low.plans = powers
    if schema == _SCHEMAS[0] and low.block_count not in (1, 2):
        raise ValueError("hierarchical repeated-block runtime currently requires one or two "
                         "compiler-factored blocks")
    if low.channel_count != low.route_count * low.lr_multiplicity:
        raise ValueError("hierarchical route/LR count does not match output layout")
    if lr.shape != (low.lr_multiplicity, low.tableau_count):
        raise ValueError("hierarchical LR synthesis dimensions are inconsistent")
    if low.output_dimension != low.channel_count * low.tableau_count * low.magnetic_count:
        raise ValueError("hierarchical output layout width is inconsistent")

    # (1) block power tables and each (block, L)'s offset inside its block row
    low.power_tables = []
    base = {}
    widths = [0] * low.block_count
    for (b, L) in sorted(powers):
        counts, offsets, index, values = lower_block_power_plan(powers[(b, L)])
        D = int(offsets.shape[0]) - 1
        if D % (2 * L + 1):
            raise ValueError("block power descriptor layout is not multiplet-complete")
        base[(b, L)] = widths[b]
        low.power_tables.append((b, L, widths[b], D, counts, offsets, index, values))
        widths[b] += D
    low.block_width = max(widths)

    # (2) route terms per route and magnetic component: (coefficient, descriptor index per block)
    M = low.magnetic_count
    route_terms = [[[] for _ in range(M)] for _ in routes]

    def desc(b, L, mult, comp):
        if (b, L) not in base:
            raise ValueError("hierarchical route names a block power that the plan does not define")
        return base[(b, L)] + mult * (2 * L + 1) + comp

    for r, route in enumerate(routes):
        Ls = [int(v) for v in route["block_output_Ls"]]
        mults = [int(v) for v in route["block_multiplicity_indices"]]
        if len(Ls) != low.block_count:
            raise ValueError("hierarchical route must name every block")
        if schema == _SCHEMAS[1]:
            tab = tables[str(route["angular_synthesis_table_id"])]
            ws = [2 * L + 1 for L in Ls]
            for row, col, val in zip(tab["row_indices"], tab["column_indices"], tab["values"]):
                idx = [desc(b, Ls[b], mults[b], (int(row) // math.prod(ws[b + 1:])) % ws[b])
                       for b in range(low.block_count)]
                route_terms[r][int(col)].append((_cplx(val).conjugate(), idx))
        elif low.block_count == 1:
            for m in range(M):
                route_terms[r][m].append((1.0 + 0j, [desc(0, low.target_L, mults[0], m)]))
        else:
            cg = _dense(tables[str(route["angular_synthesis_table_id"])])
            wr = 2 * Ls[1] + 1
            for i, col in zip(*np.nonzero(cg)):
                route_terms[r][int(col)].append(
                    (cg[i, col].conjugate(), [desc(0, Ls[0], mults[0], int(i) // wr),
                                              desc(1, Ls[1], mults[1], int(i) % wr)]))
    # (3) LR analysis folded in: output (channel = r * lr_multiplicity + mu, tableau, m)
    lr_c = lr.conj()
    offsets, m_idx, coeffs = [0], [], []
    for r in range(low.route_count):
        for mu in range(low.lr_multiplicity):
            for tau in range(low.tableau_count):
                for m in range(M):
                    for c, idx in route_terms[r][m]:
                        coeffs.append(lr_c[mu, tau] * c)
                        m_idx.append(idx)
                    offsets.append(len(coeffs))
    low.offsets = np.asarray(offsets, dtype=np.int64)
    low.m_idx = np.asarray(m_idx, dtype=np.int64).reshape(-1, low.block_count)
    low.coeffs = np.asarray(coeffs, dtype=np.complex128)
    return low


class YE3THierarchicalRepeatedBlockModule(torch.nn.Module):
    """Evaluate one factored Schur/LR repeated-angular ``block_symmetric_power`` instruction on CUDA."""

    _FIELDS = ("instruction_id", "plan_hash", "coefficient_hash", "channel_count", "tableau_count",
               "magnetic_count", "output_dimension", "target_L", "target_parity", "lr_multiplicity",
               "block_count", "route_count", "hierarchical_schema")

    def __init__(self, execution_plan, instruction_id=None, backend="auto", dtype=None, device=None):
        super().__init__()
        backend = str(backend)
        if backend not in {"auto", "native", "reference"}:
            raise ValueError("backend must be auto, native, or reference")
        if backend == "reference":
            raise ValueError("backend 'reference' is the ye3t torch path; ye3t_b200 evaluates on CUDA only")
        if dtype is None:
            dtype = torch.complex128
        if dtype not in (torch.complex64, torch.complex128):
            raise ValueError("hierarchical complex-magnetic plans require a complex dtype")
        device = torch.device("cuda" if device is None else device)
        if device.type != "cuda":
            raise ValueError("ye3t_b200 hierarchical runtime evaluates on CUDA devices only")
        low = lower_hierarchical_instruction(execution_plan, instruction_id)
        for name in self._FIELDS:
            setattr(self, name, getattr(low, name))
        self.backend = backend
        self.last_backend = None
        self.last_linear_readout_backend = None
        self.dtype, self.device = dtype, device
        self._blocks = low.blocks
        self._plans = low.plans
        self._block_width = low.block_width
        self._power_tables = [
            (b, L, start, D, torch.as_tensor(counts).to(device), torch.as_tensor(offsets).to(device),
             torch.as_tensor(index).to(device), torch.as_tensor(values).to(device=device, dtype=dtype))
            for b, L, start, D, counts, offsets, index, values in low.power_tables]
        self._schedule = _LoweredSchedule(low.offsets, low.m_idx, low.coeffs, low.block_count, low.block_width)
        self.term_count = int(low.coeffs.shape[0])

    def block_power_requests(self):
        return tuple({"block_index": int(b), "output_L": int(L), "plan": self._plans[(b, L)]}
                     for (b, L) in sorted(self._plans))

    def _block_values(self, block_inputs):
        leading = None
        xs = []
        for block, value in zip(self._blocks, block_inputs):
            value = torch.as_tensor(value, dtype=self.dtype, device=self.device)
            if int(value.shape[-1]) != 2 * int(block["input_L"]) + 1:
                raise ValueError("hierarchical block input multiplet width is incorrect")
            if leading is None:
                leading = tuple(value.shape[:-1])
            elif tuple(value.shape[:-1]) != leading:
                raise ValueError("hierarchical block inputs require matching leading shapes")
            xs.append(value.reshape(-1, value.shape[-1]))
        n = xs[0].shape[0]
        bv = torch.zeros((n, 1, self.block_count, self._block_width), dtype=self.dtype, device=self.device)
        for b, L, start, D, counts, offsets, index, values in self._power_tables:
            bv[:, 0, b, start:start + D] = symmetric_power_monomial_contraction(xs[b], counts, offsets, index,
                                                                                values)
        return bv, leading

    def forward(self, *block_inputs):
        if len(block_inputs) == 1 and isinstance(block_inputs[0], (tuple, list)):
            block_inputs = tuple(block_inputs[0])
        if len(block_inputs) != self.block_count:
            raise ValueError("hierarchical input count does not match block count")
        bv, leading = self._block_values(block_inputs)
        out = evaluate_factorized_schedule_torch(bv, self._schedule, backend="native")
        self.last_backend = "cuda_symmetric_power_then_factorized_schedule"
        return out.reshape(leading + (self.channel_count, self.tableau_count, self.magnetic_count))

    def forward_flat(self, *block_inputs):
        output = self.forward(*block_inputs)
        return output.reshape(tuple(output.shape[:-3]) + (self.output_dimension,))

    def linear_readout(self, source, weight, bias):
        block_inputs = tuple(source) if isinstance(source, (tuple, list)) else (source,)
        features = self.forward_flat(*block_inputs)
        weight = torch.as_tensor(weight, dtype=features.dtype, device=features.device)
        bias = torch.as_tensor(bias, dtype=features.dtype, device=features.device).reshape(())
        if weight.ndim != 1 or int(weight.numel()) != self.output_dimension:
            raise ValueError("hierarchical readout weight has the wrong width")
        self.last_linear_readout_backend = "materialized_hierarchical_readout"
        return features @ weight + bias

    def runtime_report(self):
        return {
            "runtime": "YE3THierarchicalRepeatedBlockModule",
            "instruction_id": self.instruction_id,
            "plan_hash": self.plan_hash,
            "coefficient_hash": self.coefficient_hash,
            "block_count": self.block_count,
            "route_count": self.route_count,
            "channel_count": self.channel_count,
            "tableau_count": self.tableau_count,
            "magnetic_count": self.magnetic_count,
            "target_L": self.target_L,
            "target_parity": self.target_parity,
            "backend": self.backend,
            "last_backend": self.last_backend,
            "last_linear_readout_backend": self.last_linear_readout_backend,
            "runtime_path_discovery": False,
            "raw_angular_tree_forest_materialized": False,
            "composition": "cuda_block_power_then_factorized_schedule_with_folded_LR",
            "schedule_terms": self.term_count,
            "supports_autograd_vjp_hvp": False,
            "supports_autograd_vjp": True,
        }


def load_scalar_ace_plans(manifest_path, *, dtype=torch.complex128, device=None):
    """Modules for every coordinate of a scalar ACE LAMMPS export (``manifest.json``).

    Each plan file's SHA-256 and plan hash must equal the manifest's record.
    Returns ``{name: module}`` in manifest order; a module's block inputs are
    the coordinate's source bindings in block order (``module._blocks``).
    """
    manifest_path = os.fspath(manifest_path)
    with open(manifest_path, encoding="utf-8") as fh:
        manifest = json.load(fh)
    if manifest.get("schema") != _MANIFEST_SCHEMA:
        raise ValueError("not a scalar ACE LAMMPS plan manifest")
    root = os.path.dirname(manifest_path)
    out = {}
    for case in manifest["cases"]:
        record = case["execution_plan"]
        name = str(record["file"])
        if os.path.basename(name) != name:
            raise ValueError("execution-plan filenames must stay inside the export directory")
        with open(os.path.join(root, name), "rb") as fh:
            body = fh.read()
        if hashlib.sha256(body).hexdigest() != record["sha256"]:
            raise ValueError(f"{name}: SHA-256 does not match the manifest")
        plan = json.loads(body.decode("utf-8"))
        if str(plan.get("plan_hash")) != str(record["plan_hash"]):
            raise ValueError(f"{name}: plan hash does not match the manifest")
        out[str(case["name"])] = YE3THierarchicalRepeatedBlockModule(plan, dtype=dtype, device=device)
    return out
