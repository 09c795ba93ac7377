"""CPU restatement of the reference's hierarchical repeated-block runtime.

TEST INFRASTRUCTURE ONLY: the tests, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU baseline may call this module as the checker; no product
path imports it.

Follows ``YE3THierarchicalRepeatedBlockModule`` (ye3t/runtime/hierarchical.py:79)
term for term, reading the execution-plan dict (the JSON the reference's
``YE3TExecutionPlan.to_json`` writes) directly with numpy:

* block powers: ``_evaluate_block_plans`` (hierarchical.py:419-435) through the
  grouped lowering ``_symmetric_power_product_plan_count_table``
  (ye3t/runtime/symmetric_power.py:740-868);
* routes: schema v1 selects a multiplicity (one block, hierarchical.py:474-476)
  or couples two blocks with the dense binary CG table, ``(left x right) @
  conj(CG)`` (hierarchical.py:478-497); schema v2 sums the sparse route entries
  ``conj(value) * prod_b block_b[component]`` into their output columns
  (hierarchical.py:437-472, route buffers 296-357);
* LR analysis: the outer product with ``conj(lr_synthesis)`` and the
  ``[channel, tableau, magnetic]`` reshape (hierarchical.py:499-512);
* dense synthesis tables: ``_dense_synthesis_table`` (hierarchical.py:22-37).
"""

from __future__ import annotations

import json
import math

import numpy as np


def _cplx(v):
    if isinstance(v, (list, tuple)):
        return complex(float(v[0]), float(v[1]))
    return complex(v)


def plan_dict(plan):
    if isinstance(plan, dict):
        return plan
    if isinstance(plan, str):
        return json.loads(plan)
    return json.loads(plan.to_json())


def lower_power_plan(plan, imag_tol=1e-12):
    """Grouped monomial table of a symmetric-power product plan dict:
    (counts [T, channel_count], offsets [descriptor_count + 1], values [T])."""
    C, D = int(plan["channel_count"]), int(plan["descriptor_count"])
    acc = {}
    for entry in plan["entries"]:
        d = int(entry["descriptor_index"])
        ch = [int(v) for v in entry["channel_indices"]]
        for term in entry["component_terms"]:
            counts = [0] * C
            for local, e in enumerate(term["exponents"]):
                counts[ch[local]] += int(e)
            key = (d, tuple(counts))
            acc[key] = acc.get(key, 0j) + _cplx(term["coefficient"])
    rows, offsets = [], [0]
    for d in range(D):
        mine = sorted((c, v) for (dd, c), v in acc.items() if dd == d and abs(v) > imag_tol)
        rows.extend(mine)
        offsets.append(len(rows))
    counts = np.asarray([r[0] for r in rows], dtype=np.int64).reshape(-1, C)
    values = np.asarray([r[1] for r in rows], dtype=np.complex128)
    return counts, np.asarray(offsets, dtype=np.int64), values


def power_eval(x, counts, offsets, values):
    """out[n, d] = sum over the descriptor's terms of value * prod_i x[n, i]^counts[t, i]."""
    x = np.asarray(x, dtype=np.complex128)
    out = np.zeros((x.shape[0], offsets.shape[0] - 1), dtype=np.complex128)
    for d in range(offsets.shape[0] - 1):
        for t in range(offsets[d], offsets[d + 1]):
            m = np.full(x.shape[0], values[t], dtype=np.complex128)
            for i, e in enumerate(counts[t]):
                if e:
                    m = m * x[:, i] ** int(e)
            out[:, d] += m
    return out


def _dense(table):
    M = np.zeros((int(table["input_dimension"]), int(table["output_dimension"])), dtype=np.complex128)
    for r, c, v in zip(table["row_indices"], table["column_indices"], table["values"]):
        M[int(r), int(c)] += _cplx(v)
    return M


def forward(plan, block_inputs, instruction_id=None):
    """Reference forward of one ``block_symmetric_power`` instruction:
    block inputs ``[N, 2 l_b + 1]`` -> ``[N, channel, tableau, magnetic]``."""
    d = plan_dict(plan)
    instructions = {str(i["instruction_id"]): i for i in d["instructions"]}
    if instruction_id is None:
        instruction_id = d["forward_schedule"][0]
    ins = instructions[str(instruction_id)]
    md = ins["metadata"]
    tables = {t["table_id"]: t for t in d["synthesis_tables"]}
    xs = [np.asarray(x, dtype=np.complex128).reshape(-1, np.asarray(x).shape[-1]) for x in block_inputs]
    N = xs[0].shape[0]
    evaluated = {}
    for rec in md["block_power_plans"]:
        b, L = int(rec["block_index"]), int(rec["output_L"])
        counts, offsets, values = lower_power_plan(rec["plan"])
        v = power_eval(xs[b], counts, offsets, values)
        evaluated[(b, L)] = v.reshape(N, -1, 2 * L + 1)
    layout = [lay for lay in d["carrier_layouts"]
              if json.dumps(lay["key"], sort_keys=True) == json.dumps(ins["output_carrier"], sort_keys=True)][0]
    Mc, T = int(layout["magnetic_count"]), int(layout["tableau_count"])
    routes = sorted(md["routes"], key=lambda r: int(r["route_index"]))
    R = len(routes)
    route_values = np.zeros((N, R, Mc), dtype=np.complex128)
    v2 = md["schema"] == "ye3t_hierarchical_repeated_angular_blocks_v2"
    for r, route in enumerate(routes):
        Ls = [int(v) for v in route["block_output_Ls"]]
        mults = [int(v) for v in route["block_multiplicity_indices"]]
        if v2:
            tab = tables[route["angular_synthesis_table_id"]]
            widths = [2 * L + 1 for L in Ls]
            for row, col, val in zip(tab["row_indices"], tab["column_indices"], tab["values"]):
                term = np.full(N, _cplx(val).conjugate(), dtype=np.complex128)
                for b, w in enumerate(widths):
                    stride = math.prod(widths[b + 1:])
                    comp = (int(row) // stride) % w
                    term = term * evaluated[(b, Ls[b])][:, mults[b], comp]
                route_values[:, r, int(col)] += term
        elif len(Ls) == 1:
            route_values[:, r, :] = evaluated[(0, int(md["target_L"]))][:, mults[0], :]
        else:
            left = evaluated[(0, Ls[0])][:, mults[0], :]
            right = evaluated[(1, Ls[1])][:, mults[1], :]
            product = (left[:, :, None] * right[:, None, :]).reshape(N, -1)
            route_values[:, r, :] = product @ _dense(tables[route["angular_synthesis_table_id"]]).conj()
    lr = _dense(tables[md["lr_synthesis_table_id"]]).conj()  # [lr_multiplicity, tableau]
    out = route_values[:, :, None, None, :] * lr[None, None, :, :, None]
    return out.reshape(N, R * lr.shape[0], T, Mc)
