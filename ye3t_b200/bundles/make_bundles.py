"""Compile the ACE word-set bundles shipped with ye3t_b200.

Run where the reference ye3t package is importable (it is not needed at run
time: the bundles are plain arrays):

    PYTHONPATH=<ye3t checkout> python -m ye3t_b200.bundles.make_bundles [--check-every K]

Each pattern is compiled once with the reference's own public compiler,
``ye3t.couplings.compile_ace_factorized_schedules_by_L``
(``ye3t/couplings/__init__.py:2617``), and each symmetric block kind is
lowered with ``ye3t.couplings.symmetric_power_product_plan``
(``ye3t/couplings/__init__.py:4112``) and the grouped count-table lowering in
``ye3t/runtime/symmetric_power.py:740-868``, exactly as
``ye3t/workflows.py:544-556`` does for an ACE case.  Every K-th word is also
compiled directly and its tables compared bit-for-bit with the pattern
rebinding.
"""

from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from ye3t_b200.schedules import (ACEBundle, ScheduleRecord, SymPowerTable,  # noqa: E402
                                 enumerate_ace_words, schedule_table_hash)

# Word sets shipped with the package: (file stem, nmax, lmax, numax, target_L, parity).
# Symmetric-power tables are materialised exactly; Sym^4(V_4) (l_max 4) is
# over the reference's exact-symbolic resource limit and takes its "auto"
# policy (the reference's own advice), recorded in the bundle meta.
# The channel-diagonal sets (nmax 1) are evaluated once per mixed radial
# channel: every block of a word reads the same channel.
BUNDLES = [
    ("ace_n8_l3_nu4_L0", 8, 3, 4, 0, "even"),  # large-scale scalar ACE (nu <= 4, l_max 3)
    ("ace_n8_l3_nu3_L0", 8, 3, 3, 0, "even"),  # single-species scalar descriptor (nu <= 3)
    ("ace_diag_l4_nu4_L0", 1, 4, 4, 0, "even"),  # multi-species, mixed channels (l_max 4, nu <= 4)
    ("ace_diag_l3_nu3_L0", 1, 3, 3, 0, "all"),  # equivariant couplings, L = 0 outputs
    ("ace_diag_l3_nu3_L1", 1, 3, 3, 1, "all"),  # ... L = 1 outputs
    ("ace_diag_l3_nu3_L2", 1, 3, 3, 2, "all"),  # ... L = 2 outputs
]


def reference_compilers(target_L: int, materialization: str = "exact"):
    import torch
    from ye3t import couplings
    from ye3t.couplings import compile_ace_factorized_schedules_by_L
    from ye3t.runtime.symmetric_power import _symmetric_power_product_plan_count_table

    def compile_pattern(content, input_Ls):
        report = compile_ace_factorized_schedules_by_L(content=content, input_Ls=input_Ls)
        return report.schedules_by_L.get(target_L), report.convention_hash

    def sym_table_for(l, k, Lam, mu):
        plan = couplings.symmetric_power_product_plan(
            [{"descriptor_index": m, "power": k, "input_L": l, "output_L": Lam,
              "multiplicity_index": mu, "component_index": m,
              "channel_indices": tuple(range(2 * l + 1))} for m in range(2 * Lam + 1)],
            descriptor_count=2 * Lam + 1, channel_count=2 * l + 1,
            basis_convention="complex_magnetic", coefficient_materialization=materialization)
        grouped, _shared, _dt = _symmetric_power_product_plan_count_table(
            plan, device="cpu", dtype=torch.complex128, imag_tol=1e-12)
        counts, offsets, index, values = grouped
        return SymPowerTable(l, k, Lam, mu, monomial_counts=counts.numpy().astype(np.int64),
                             output_offsets=offsets.numpy().astype(np.int64),
                             output_index=index.numpy().astype(np.int64),
                             monomial_value=values.numpy().astype(np.complex128),
                             convention_hash=str(plan.convention_hash))

    return compile_pattern, sym_table_for


def check_rebinding(bundle: ACEBundle, every: int) -> int:
    from ye3t.couplings import compile_ace_factorized_schedules_by_L

    checked = 0
    for w in range(0, bundle.word_count, max(1, every)):
        word = bundle.words[w]
        rep = compile_ace_factorized_schedules_by_L(content=tuple(n for _, n in word),
                                                    input_Ls=tuple(l for l, _ in word))
        direct = ScheduleRecord.from_schedule(rep.schedules_by_L[bundle.target_L], rep.convention_hash)
        bound = bundle.word_schedule(w)
        if schedule_table_hash(direct) != schedule_table_hash(bound):
            raise AssertionError(f"word {word}: pattern rebinding differs from direct compile")
        checked += 1
    return checked


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--check-every", type=int, default=50)
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", default=None)
    args = ap.parse_args(argv)
    for stem, nmax, lmax, numax, L, parity in BUNDLES:
        if args.only and stem != args.only:
            continue
        t0 = time.time()
        words = enumerate_ace_words(nmax, lmax, numax, parity=parity)
        materialization = "auto" if lmax >= 4 else "exact"
        cp, st = reference_compilers(L, materialization)
        rule = "even sum(l)" if parity == "even" else "any sum(l) with a basis at target_L"
        b = ACEBundle.from_words(words, nmax, lmax, L, cp, st, meta={
            "word_rule": f"all multisets of (n,l), n in 1..nmax, l in 0..lmax, size 1..numax, {rule}",
            "nmax": nmax, "lmax": lmax, "numax": numax, "target_L": L, "parity": parity,
            "symmetric_power_materialization": materialization,
            "compiler": "ye3t.couplings.compile_ace_factorized_schedules_by_L (defaults)"})
        n_checked = check_rebinding(b, args.check_every)
        path = os.path.join(args.out, stem + ".npz")
        b.save(path)
        tot_terms = sum(b.patterns[p].term_count for p in b.word_pattern_index)
        print(f"{stem}: words={b.word_count} patterns={len(b.patterns)} features={b.feature_count} "
              f"terms/atom={tot_terms} sym_kinds={len(b.sym_tables)} checked={n_checked} "
              f"hash={b.table_hash()} ({time.time() - t0:.1f}s) -> {path}")


if __name__ == "__main__":
    main()
