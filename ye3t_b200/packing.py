"""Schedule-to-device table packing for the fused ACE kernels.

Turns an :class:`~ye3t_b200.schedules.ACEBundle` into the flat arrays of
``y3b_ace_tables`` (include/ye3t_b200.h).

Per-atom block pool (complex entries, atom-fastest on the device):

* A channels: ``(n-1) * (lmax+1)^2 + l^2 + (m + l)`` for ``n = 1..nmax``;
* then, for every symmetric block kind ``(l, k, Lambda, mu)`` in sorted
  order and every radial channel ``n``, the ``2 Lambda + 1`` outputs of
  ``Sym^k(A[n, l]) -> V_Lambda``.

A term of word ``w``, label ``a`` reads block ``b`` at
``pool[label_bases[word_label_base[w] + a][b] + m_idx]`` with
``m_idx = m + L_block`` exactly as ``TorchFactorizedCoefficientSchedule``'s
``block_m_indices`` (``ye3t/core/couplings.py:216-240``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict

import numpy as np
import torch

from . import _native as nat
from .schedules import ACEBundle

__all__ = ["PackedBundle", "pack_bundle"]


@dataclass
class PackedBundle:
    bundle: ACEBundle
    device: torch.device
    arrays: Dict[str, torch.Tensor]
    pool_size: int
    feature_count: int
    max_blocks: int
    sym_offsets: Dict
    term_count_per_atom: int
    term_block_count_per_atom: int
    sym_term_count_per_atom: int
    sym_flops_per_atom: float = 0.0

    def tables(self) -> nat.AceTables:
        a = self.arrays
        b = self.bundle
        t = nat.AceTables()
        t.nmax, t.lmax = b.nmax, b.lmax
        t.pool_size = self.pool_size
        t.word_count = b.word_count
        t.feature_count = self.feature_count
        t.sym_kind_count = int(a["sym_kind"].shape[0])
        t.max_blocks = self.max_blocks
        for name in ("word_pattern", "word_label_base", "word_feature_offset", "pattern_comp_begin",
                     "pattern_block_count", "comp_term_begin", "comp_label", "term_m", "term_coeff",
                     "label_bases", "sym_kind", "sym_term_factors", "sym_term_output", "sym_term_coeff"):
            setattr(t, name, ctypes.c_void_p(a[name].data_ptr()))
        return t

    def pool_index_A(self, n: int, l: int, m: int) -> int:
        W = (self.bundle.lmax + 1) ** 2
        return (n - 1) * W + l * l + l + m

    def flops_per_atom(self) -> Dict[str, float]:
        """Algorithmic complex-arithmetic counts of the bundle stage per atom (real flops).

        A term with B blocks costs one real x complex scaling (2 flops),
        B - 1 complex multiplies (6 flops each) and one complex add (2 flops);
        a symmetric-power term of degree k costs k complex multiplies
        (including the coefficient) plus one complex add.
        """
        terms = self.term_count_per_atom
        tb = self.term_block_count_per_atom
        sched = 2.0 * terms + 6.0 * (tb - terms) + 2.0 * terms
        return {"schedule": sched, "sym": float(self.sym_flops_per_atom)}


def _factors(row):
    out = []
    for comp, cnt in enumerate(row):
        out.extend([comp] * int(cnt))
    if len(out) > 4:
        raise ValueError("symmetric block degree above 4 is not supported by the fused kernel")
    packed = 0
    for k in range(4):
        v = out[k] if k < len(out) else 255
        packed |= int(v) << (8 * k)
    return packed


def pack_bundle(bundle: ACEBundle, device) -> PackedBundle:
    device = torch.device(device)
    nmax, lmax = bundle.nmax, bundle.lmax
    W = (lmax + 1) ** 2
    # symmetric pool layout
    sym_keys = sorted(bundle.sym_tables)
    sym_off = {}
    off = nmax * W
    sym_kind_rows, s_fac, s_out, s_co = [], [], [], []
    sym_flops = 0.0
    for key in sym_keys:
        t = bundle.sym_tables[key]
        l, k, Lam, mu = key
        sym_off[key] = off
        vals = np.asarray(t.monomial_value)
        if np.iscomplexobj(vals) and vals.size and np.max(np.abs(vals.imag)) > 1e-12:
            raise ValueError(f"symmetric table {key} has complex coefficients; not supported by the fused kernel")
        tb = len(s_fac)
        offsets = np.asarray(t.output_offsets, dtype=np.int64)
        for o in range(2 * Lam + 1):
            for q in range(int(offsets[o]), int(offsets[o + 1])):
                s_fac.append(_factors(t.monomial_counts[q]))
                s_out.append(o)
                s_co.append(float(np.real(vals[q])))
                sym_flops += 6.0 * int(np.sum(t.monomial_counts[q])) + 2.0
        sym_kind_rows.append([l, k, Lam, off, tb, len(s_fac)])
        off += nmax * (2 * Lam + 1)
    sym_flops *= nmax
    pool_size = off
    # pattern tables
    pcb, pbc, ctb, clab, tm, tco = [0], [], [0], [], [], []
    max_blocks = 1
    for p in bundle.patterns:
        if p.block_count > 4:
            raise ValueError("fused kernel supports at most 4 blocks per word")
        max_blocks = max(max_blocks, p.block_count)
        rc = p.real_coeffs()
        if rc is None:
            raise ValueError("fused kernel needs real schedule coefficients")
        bmi = p.block_m_indices()
        for c in range(p.component_count):
            t0, t1 = int(p.component_offsets[c]), int(p.component_offsets[c + 1])
            for q in range(t0, t1):
                packed = 0
                for b in range(p.block_count):
                    v = int(bmi[q, b])
                    if not 0 <= v < 255:
                        raise ValueError("magnetic index out of packable range")
                    packed |= v << (8 * b)
                tm.append(packed)
                tco.append(float(rc[q]))
            ctb.append(len(tm))
            clab.append(int(p.component_label_index[c]))
        pcb.append(len(clab))
        pbc.append(p.block_count)
    # per-word bindings
    wlb, lbases, wfo = [], [], []
    fo = 0
    terms_per_atom = 0
    term_blocks_per_atom = 0
    for w in range(bundle.word_count):
        rec = bundle.word_schedule(w)
        wlb.append(len(lbases))
        for label in rec.block_specs:
            row = [0, 0, 0, 0]
            for b, (kind, n, l, k, Lam, mu) in enumerate(label):
                if kind == "sym":
                    row[b] = sym_off[(l, k, Lam, mu)] + (n - 1) * (2 * Lam + 1)
                else:
                    row[b] = (n - 1) * W + l * l
            lbases.append(row)
        wfo.append(fo)
        fo += rec.component_count
        terms_per_atom += rec.term_count
        term_blocks_per_atom += rec.term_count * rec.block_count
    arrays_np = {
        "word_pattern": np.asarray(bundle.word_pattern_index, dtype=np.int32),
        "word_label_base": np.asarray(wlb, dtype=np.int32),
        "word_feature_offset": np.asarray(wfo, dtype=np.int64),
        "pattern_comp_begin": np.asarray(pcb, dtype=np.int32),
        "pattern_block_count": np.asarray(pbc, dtype=np.int32),
        "comp_term_begin": np.asarray(ctb, dtype=np.int32),
        "comp_label": np.asarray(clab, dtype=np.int32),
        "term_m": np.asarray(tm, dtype=np.uint32).view(np.int32),
        "term_coeff": np.asarray(tco, dtype=np.float64),
        "label_bases": np.asarray(lbases, dtype=np.int32).reshape(-1, 4),
        "sym_kind": np.asarray(sym_kind_rows, dtype=np.int32).reshape(-1, 6),
        "sym_term_factors": np.asarray(s_fac, dtype=np.uint32).view(np.int32),
        "sym_term_output": np.asarray(s_out, dtype=np.int32),
        "sym_term_coeff": np.asarray(s_co, dtype=np.float64),
    }
    arrays = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in arrays_np.items()}
    pb = PackedBundle(bundle=bundle, device=device, arrays=arrays, pool_size=pool_size, feature_count=fo,
                      max_blocks=max_blocks, sym_offsets=sym_off, term_count_per_atom=terms_per_atom,
                      term_block_count_per_atom=term_blocks_per_atom,
                      sym_term_count_per_atom=len(s_fac) * nmax, sym_flops_per_atom=sym_flops)
    return pb
