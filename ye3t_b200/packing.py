"""Schedule-to-device table packing for the fused ACE kernels.

Turns an :class:`~ye3t_b200.schedules.ACEBundle` into the flat arrays of
``y3b_ace_tables`` (include/ye3t_b200.h).

Per-CTA shared-memory block entries (complex, 32 atoms per entry):

* A channels: ``(n-1) * (lmax+1)^2 + l^2 + (m + l)`` for ``n = 1..nmax``;
* two slots, each holding, for one radial channel, every symmetric block
  kind ``(l, k, Lambda, mu)`` (sorted) as the ``2 Lambda + 1`` outputs of
  ``Sym^k(A[n, l]) -> V_Lambda``.

Words are scheduled in phases, one per pair of radial channels resident in
the two slots; a word's symmetric blocks read at most two radial channels.
A block's magnetic index is ``m + L_block`` exactly as
``TorchFactorizedCoefficientSchedule``'s ``block_m_indices``
(``ye3t/core/couplings.py:216-240``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, Optional

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
    item_flops: Optional[float] = None
    item_grad_flops: Optional[float] = None

    def tables(self) -> nat.AceTables:
        a = self.arrays
        b = self.bundle
        t = nat.AceTables()
        t.nmax, t.lmax = b.nmax, b.lmax
        t.smem_entries = self.pool_size
        t.feature_count = self.feature_count
        t.item_count = int(a["items"].shape[0])
        t.phase_count = int(a["phases"].shape[0])
        t.sym_output_count = int(a["sym_outputs"].shape[0])
        t.group_count = int(a["groups"].shape[0])
        t.sym_grad_count = int(a["sym_grad_coeff"].shape[0])
        t.sym_term_count = int(a["sym_term_coeff"].shape[0])
        for name in ("items", "item_coef", "phases", "sym_outputs", "sym_term_factors", "sym_term_coeff", "groups",
                     "group_offsets", "sym_grad_offsets", "sym_grad_index", "sym_grad_coeff"):
            setattr(t, name, ctypes.c_void_p(a[name].data_ptr()))
        return t

    def pool_index_A(self, n: int, l: int, m: int) -> int:
        W = (self.bundle.lmax + 1) ** 2
        return (n - 1) * W + l * l + l + m

    def flops_per_atom(self) -> Dict[str, float]:
        """FP64 flop counts of the bundle stage per atom.

        ``items``: what the item walk executes on valid tuples
        (:func:`item_flops_per_atom`).  ``terms``: the reference's
        term-by-term product count, sum over terms of (6 B - 2) flops (one
        real x complex scaling, B - 1 complex multiplies, one complex add).
        ``sym``: symmetric-block monomials.
        """
        terms = self.term_count_per_atom
        tb = self.term_block_count_per_atom
        sched = 2.0 * terms + 6.0 * (tb - terms) + 2.0 * terms
        if self.item_flops is None:
            items = self.arrays["items"].cpu().numpy()
            self.item_flops = item_flops_per_atom(items)
            self.item_grad_flops = item_grad_flops_per_atom(items)
        return {"items": self.item_flops, "items_grad": self.item_grad_flops, "terms": sched,
                "sym": float(self.sym_flops_per_atom)}


def item_grad_flops_per_atom(items: np.ndarray) -> float:
    """FP64 flops per atom of the energy-and-gradient walk (valid tuples only).

    Mirrors ace_grad.cu: per valid slot of a row the weighted coefficient
    (2 nc - 1), the product q (6), T += c q (4), x c (2), gvs += (x c) vl (8)
    and the last-block gradient (x c) vs (8); per row the energy (4) and the
    prefix gradients (8 or 14).  4-block items with a register block <= 7
    share q per anti-diagonal: per valid j there q (6), gvs (8) and the
    last-block gradient (8); per prefix x0 x1 (6), per j the weighted
    coefficient and the T and R multiply-adds (2 nc - 1 + 8), the energy (4)
    and two gradients (6 + 8).
    """
    flops = 0.0
    cache = {}
    for row in items:
        key = tuple(int(v) for v in row[:5])
        if key not in cache:
            sel, D0, D1, Dl, K = key
            nc = sel % 2 + 1
            B = (sel // 2) // 7 + 1
            ds = 2 * ((sel // 2) % 7) + 1
            wc = 2 * nc - 1
            smin, smax = K - (ds - 1) - (Dl - 1), K

            def valid(S):
                return sum(1 for j in range(ds) if 0 <= K - S - j < Dl)
            f = 0.0
            if B == 1:
                f = 4.0 * nc
            elif B == 2:
                f = valid(0) * (wc + 28.0) + 2.0
            elif B == 3:
                for i0 in range(D0):
                    if smin <= i0 <= smax:
                        f += valid(i0) * (wc + 28.0) + 4.0
            elif ds <= 7:
                for S in range(max(0, smin), min(D0 - 1 + D1 - 1, smax) + 1):
                    v = valid(S)
                    rows = sum(1 for i0 in range(D0) if 0 <= S - i0 < D1)
                    f += 22.0 * v + rows * (6.0 + ds * (wc + 8.0) + 18.0)
            else:
                for i0 in range(D0):
                    for i1 in range(D1):
                        S = i0 + i1
                        if smin <= S <= smax:
                            f += valid(S) * (wc + 28.0) + 6.0 + 4.0 + 14.0
            cache[key] = f
        flops += cache[key]
    return flops


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


# ---------------------------------------------------------------------------
# Evaluation items for the B-basis kernel.
#
# Within a pattern, components whose labels bind identical blocks and that
# share the same M form a group; the group's coefficients are laid out as a
# dense table over the magnetic index box of blocks 0..B-2 (the last block's
# index follows from M: i_last = K - sum_{b < B-1} i_b with
# K = M + sum_b L_b).  Blocks 0..B-3 are walked by runtime loops, block B-2
# by a loop unrolled at compile time (its values stay in registers), and the
# last block is read once per tuple.  A pass covers at most ITEM_MAX_NC
# components of a group; every word contributes one item per pass.
# ---------------------------------------------------------------------------
ITEM_MAX_NC = 2
ITEM_INTS = 16
MAX_STATIC_DIM = 13


def item_selector(B: int, ds: int, nc: int) -> int:
    """Kernel dispatch code of an item (mirrors ace.cu)."""
    return ((B - 1) * 7 + (ds - 1) // 2) * 2 + (nc - 1)


def _pattern_groups(p):
    """[(spec, M, [components])] in first-component order."""
    order, groups = [], {}
    for c in range(p.component_count):
        key = (p.block_specs[int(p.component_label_index[c])], int(p.component_M_R[c]))
        if key not in groups:
            groups[key] = []
            order.append(key)
        groups[key].append(c)
    return [(k[0], k[1], groups[k]) for k in order]


def _row_width(ds: int, nc: int) -> int:
    """Doubles per coefficient row (one prefix): nc per j, padded to even."""
    return 2 * ds if nc == 2 else (ds + 1) & ~1


def _block_order(spec):
    """Evaluation order of a group's blocks: ascending magnetic dimension
    (stable), so the two largest become the register-held and the implied
    last block and the short ones run as the outer loops."""
    dims = [2 * (s[4] if s[0] == "sym" else s[2]) + 1 for s in spec]
    return sorted(range(len(spec)), key=lambda b: dims[b])


def _group_pass_table(p, rc, spec, M, comps):
    """Coefficient table of one pass: rows (one per prefix of blocks 0..B-3) of
    ``_row_width`` doubles holding ``C[prefix, j, c]`` at ``j * nc + c``.

    ``spec`` is the group's block list already in evaluation order; term
    indices are permuted to it with ``order`` (original block of each slot)."""
    order = _block_order(spec)
    spec = [spec[b] for b in order]
    B = len(spec)
    lam = [s[4] if s[0] == "sym" else s[2] for s in spec]
    dims = [2 * L + 1 for L in lam]
    K = M + sum(lam)
    nc = len(comps)
    if B == 1:
        table = np.zeros((1, nc), dtype=np.float64)
    else:
        prefix_box = dims[:-2]
        ds = dims[-2]
        rows = int(np.prod(prefix_box)) if prefix_box else 1
        table = np.zeros((rows, _row_width(ds, nc)), dtype=np.float64)
    for k, c in enumerate(comps):
        for q in range(int(p.component_offsets[c]), int(p.component_offsets[c + 1])):
            idx = [int(p.block_m_tuples[q, order[b]]) + lam[b] for b in range(B)]
            if idx[-1] != K - sum(idx[:-1]):
                raise ValueError("term violates magnetic conservation")
            if B == 1:
                table[0, k] += float(rc[q])
            else:
                row = int(np.ravel_multi_index(tuple(idx[:-2]), dims[:-2])) if B > 2 else 0
                table[row, idx[-2] * nc + k] += float(rc[q])
    return dims, K, table, tuple(spec)


def _phase_pairs(nmax):
    """Channel pairs (slot 0, slot 1) visited by the kernel, in order."""
    if nmax == 1:
        return [(0, -1)]
    return [(a, b) for a in range(nmax) for b in range(a + 1, nmax)]


def _word_phase(sym_channels, nmax):
    """Phase pair holding every radial channel that a word's symmetric blocks read."""
    S = sorted(sym_channels)
    if nmax == 1:
        return (0, -1)
    if len(S) == 2:
        return (S[0], S[1])
    if len(S) == 1:
        a = S[0]
        return (a, a + 1) if a + 1 < nmax else (a - 1, a)
    return None


def _build_items(bundle, sym_local, sym_out_count, W):
    """Items grouped by phase, the coefficient array and the phase table.

    Shared-memory entries of a CTA: A channels ``(n-1) W + l^2 + (m + l)``,
    then two slots of ``sym_out_count`` symmetric outputs, each slot holding
    every symmetric block of one radial channel (``sym_local`` gives a
    block's first output inside a slot).
    """
    nmax = bundle.nmax
    coef_chunks, coef_len = [], 0
    pattern_passes = []
    for p in bundle.patterns:
        rc = p.real_coeffs()
        if rc is None:
            raise ValueError("fused kernel needs real schedule coefficients")
        passes = []
        for spec, M, comps in _pattern_groups(p):
            for s0 in range(0, len(comps), ITEM_MAX_NC):
                chunk = comps[s0:s0 + ITEM_MAX_NC]
                dims, K, table, spec_eval = _group_pass_table(p, rc, spec, M, chunk)
                if len(dims) > 4:
                    raise ValueError("fused kernel supports at most 4 blocks per word")
                if len(dims) >= 2 and dims[-2] > MAX_STATIC_DIM:
                    raise ValueError("block magnetic dimension above 13 is not supported")
                passes.append((dims, K, coef_len, chunk, spec_eval))
                flat = table.reshape(-1)
                if flat.size % 2:
                    flat = np.concatenate([flat, [0.0]])
                coef_chunks.append(flat)
                coef_len += flat.size
        pattern_passes.append(passes)
    pairs = _phase_pairs(nmax)
    phase_of = {pr: i for i, pr in enumerate(pairs)}
    phase_items = [[] for _ in pairs]
    phase_work = [0.0] * len(pairs)
    free_words = []
    fo = 0
    A_entries = nmax * W
    for w in range(bundle.word_count):
        pi = int(bundle.word_pattern_index[w])
        p = bundle.patterns[pi]
        n_map = {r: int(bundle.word_n_map[w, r]) for r in range(1, bundle.word_n_map.shape[1])
                 if bundle.word_n_map[w, r] > 0}
        sym_ch = {n_map[s[1]] - 1 for label in p.block_specs for s in label if s[0] == "sym"}
        pair = _word_phase(sym_ch, nmax)
        rows = []
        work = 0.0
        for dims, K, coff, chunk, spec in pattern_passes[pi]:
            B = len(dims)
            row = [0] * ITEM_INTS
            ds = dims[-2] if B >= 2 else 1
            row[0] = item_selector(B, ds, len(chunk))
            row[1] = dims[0] if B >= 3 else 1
            row[2] = dims[1] if B >= 4 else 1
            row[3] = dims[-1]
            row[4] = K
            row[5] = coff
            row[6] = fo + chunk[0]
            row[7] = fo + chunk[1] if len(chunk) > 1 else -1
            for b, (kind, n, l, k, Lam, mu) in enumerate(spec):
                n = n_map[n]
                if kind == "sym":
                    row[8 + b] = -1 - (n - 1)  # resolved once the phase is known
                    row[12 + b] = sym_local[(l, k, Lam, mu)]
                else:
                    row[8 + b] = (n - 1) * W + l * l
            rows.append(row)
            work += float(np.prod(dims[:-1])) if B > 1 else 1.0
        fo += p.component_count
        if pair is None:
            free_words.append((work, rows))
        else:
            phase_items[phase_of[pair]].append(rows)
            phase_work[phase_of[pair]] += work
    # words without symmetric blocks balance the phases (largest first)
    for work, rows in sorted(free_words, key=lambda x: -x[0]):
        i = int(np.argmin(phase_work))
        phase_items[i].append(rows)
        phase_work[i] += work
    items, phases = [], []
    for i, (a, b2) in enumerate(pairs):
        begin = len(items)
        # items sharing a coefficient table run next to each other, so the
        # CTA's warps (which take items round robin) read it from L1 together
        flat = sorted((row for rows in phase_items[i] for row in rows), key=lambda r: (r[5], r[6]))
        for rows in [flat]:
            for row in rows:
                row = list(row)
                for blk in range(4):
                    if row[8 + blk] < 0:
                        ch = -1 - row[8 + blk]
                        slot = 0 if ch == a else 1
                        if (slot == 1 and ch != b2) or (slot == 0 and ch != a):
                            raise AssertionError("word scheduled in a phase without its channels")
                        row[8 + blk] = A_entries + slot * sym_out_count + row[12 + blk]
                    row[12 + blk] = 0
                items.append(row)
        phases.append([a, b2, begin, len(items)])
    coef = np.concatenate(coef_chunks) if coef_chunks else np.zeros(0)
    return (np.asarray(items, dtype=np.int32).reshape(-1, ITEM_INTS), coef,
            np.asarray(phases, dtype=np.int32).reshape(-1, 4))


def item_flops_per_atom(items: np.ndarray) -> float:
    """FP64 flops per atom of the item walk (valid tuples only).

    Nested order: per tuple one complex multiply (6 flops) and a real x
    complex multiply-add per component (4); per runtime prefix row of a 3- or
    4-block item a complex multiply-add per component (8); per outer index of
    a 4-block item another (8 per component).
    """
    flops = 0.0
    cache = {}
    for row in items:
        key = tuple(int(v) for v in row[:5])
        if key in cache:
            flops += cache[key]
            continue
        before = flops
        sel = int(row[0])
        nc = sel % 2 + 1
        B = (sel // 2) // 7 + 1
        ds = 2 * ((sel // 2) % 7) + 1
        D0, D1, Dl, K = int(row[1]), int(row[2]), int(row[3]), int(row[4])
        if B == 1:
            flops += 4.0 * nc
            cache[key] = flops - before
            continue
        prefixes = [(0,)] if B == 2 else ([(i,) for i in range(D0)] if B == 3 else
                                          [(i, j) for i in range(D0) for j in range(D1)])
        smin, smax = K - (ds - 1) - (Dl - 1), K
        outer = set()
        for pre in prefixes:
            S = sum(pre) if B > 2 else 0
            if B > 2 and not smin <= S <= smax:
                continue
            valid = sum(1 for j in range(ds) if 0 <= K - S - j < Dl)
            flops += valid * (6.0 + 4.0 * nc) + (8.0 * nc if B > 2 else 0.0)
            if B == 4:
                outer.add(pre[0])
        flops += 8.0 * nc * len(outer)
        cache[key] = flops - before
    return flops


GRAD_GROUP = 2
GRAD_CLASSES = 4
GRAD_STAGE = 14  # staged gradient entries per lane in the adjoint kernel
GRAD_RUN_CLASSES = (2, 3)  # four-block classes: A entries only, one sorted run per warp
GRAD_RUN_WARPS = 8  # warps of a run-class CTA (csrc/ace_grad.cu Y3B_RUN_WARPS) and of a slot-class CTA
GRAD_SLOT_RUN_CLASS = 1  # three-block class: one sorted run per warp and phase
GRAD_RUN_BLOCK = 7  # longest prefix / last block of a run-class item (staging windows of 7 entries)


def grad_class(row, a_entries: int) -> int:
    """Adjoint item class (one kernel launch each, csrc/ace_grad.cu adj_class).

    2 / 3: four blocks with a register block of 3 or 5 / 7 indices whose
    blocks are all A entries (``< a_entries``; those kernels hold no
    symmetric slots) and fit the run path's staging windows (prefix and last
    blocks of at most GRAD_RUN_BLOCK indices); 1: three blocks with a
    register block of 5 or 7; 0: everything else (one and two blocks, small
    register blocks, four-block items reading symmetric outputs, and shapes
    the unrolled paths do not cover: wide register blocks, long last blocks).
    """
    sel, d0, d1, dl = int(row[0]), int(row[1]), int(row[2]), int(row[3])
    B = (sel // 2) // 7 + 1
    ds = 2 * ((sel // 2) % 7) + 1
    if (B == 4 and 3 <= ds <= 7 and max(d0, d1, dl) <= GRAD_RUN_BLOCK
            and all(int(row[8 + b]) + dim <= a_entries for b, dim in enumerate((d0, d1, ds, dl)))):
        return 2 if ds <= 5 else 3
    if B == 3 and 5 <= ds <= 7 and dl <= GRAD_STAGE:
        return 1
    return 0


GRAD_ITEM_OVERHEAD = 200.0  # flop-equivalents of an item's fixed work (loads, flushes), for balancing only


def _pair_cost(items: np.ndarray, i: int) -> float:
    """Balancing weight of one item pair (both halves run the same shape):
    its adjoint flops plus a fixed per-item charge."""
    return item_grad_flops_per_atom(items[i:i + 1]) + GRAD_ITEM_OVERHEAD


def _round_robin_balanced(pairs: list, costs: list) -> list:
    """Pairs ordered so that the kernel's round robin (pair g to warp g mod
    GRAD_RUN_WARPS) gives every warp a near-equal cost: longest first to the
    least loaded warp, then interleaved, null pairs filling the short warps."""
    sets = [[] for _ in range(GRAD_RUN_WARPS)]
    load = [0.0] * GRAD_RUN_WARPS
    for k in sorted(range(len(pairs)), key=lambda k: -costs[k]):
        w = min(range(GRAD_RUN_WARPS), key=lambda v: (load[v], len(sets[v]), v))
        sets[w].append(pairs[k])
        load[w] += costs[k]
    rounds = max((len(x) for x in sets), default=0)
    out = []
    for r in range(rounds):
        for w in range(GRAD_RUN_WARPS):
            out.append(sets[w][r] if r < len(sets[w]) else [-1, -1])
    return out


def _balanced_runs(shapes: Dict[tuple, list], items: np.ndarray, key) -> list:
    """Item pairs of one (class, phase) range laid out as GRAD_RUN_WARPS equal runs.

    Each shape's items are sorted by ``key`` (blocks first, so that
    consecutive items of a lane share blocks and the kernel adds a block's
    gradient to G only when the block changes) and split in two halves, one
    per half-warp.  The kernel cuts the range into GRAD_RUN_WARPS equal runs;
    item costs differ by shape, so each run holds an equal share of every
    shape, padded with null pairs (-1, -1) that the kernel skips.
    """
    runs = [[] for _ in range(GRAD_RUN_WARPS)]
    for shape in sorted(shapes):
        idx = sorted(shapes[shape], key=key)
        h = (len(idx) + 1) // 2
        pairs = [[idx[u], idx[u + h] if u + h < len(idx) else -1] for u in range(h)]
        # the longest runs so far take the smaller shares of this shape (an
        # assignment ordered by flop cost measured 2 % slower here)
        order = sorted(range(GRAD_RUN_WARPS), key=lambda w: (len(runs[w]), w))
        cut = np.linspace(0, h, GRAD_RUN_WARPS + 1).round().astype(int)
        shares = sorted((pairs[cut[k]:cut[k + 1]] for k in range(GRAD_RUN_WARPS)), key=len, reverse=True)
        for w, share in zip(order, shares):
            runs[w].extend(share)
    out = []
    if any(runs):
        per = max(len(r) for r in runs)
        for r in runs:
            out.extend(r + [[-1, -1]] * (per - len(r)))
    return out


def _grad_groups(items: np.ndarray, phases: np.ndarray, a_entries: int):
    """Item pairs of the adjoint kernel, per item class and phase.

    Each half-warp runs one item; pairing two items of one shape (dispatch
    code, loop extents, K) keeps the warp's control flow identical.  Class 0
    takes a phase's pairs round robin over the warps; class 1 gives each warp a sorted run of the
    phase (register block, last block, prefix); the A-entry-only run classes
    ignore phases (every pair in phase 0's range) and sort by (register
    block, last block, prefix blocks).  Returns ``groups [P, 2]`` (-1 for a
    shape's odd item out, (-1, -1) for run padding), ordered by class then
    phase, and ``group_offsets [GRAD_CLASSES, phase_count + 1]`` (flattened).
    Class 0's pairs are spread over the warps by cost (``_round_robin_balanced``),
    since a phase ends in a barrier that waits for its slowest warp.
    """
    groups = []
    offsets = np.zeros((GRAD_CLASSES, phases.shape[0] + 1), dtype=np.int32)
    for cls in range(GRAD_CLASSES):
        if cls in GRAD_RUN_CLASSES:
            offsets[cls, 0] = len(groups)
            shapes = {}
            for i in range(items.shape[0]):
                if grad_class(items[i], a_entries) == cls:
                    shapes.setdefault(tuple(int(v) for v in items[i, :5]), []).append(i)
            groups.extend(_balanced_runs(shapes, items, lambda i: (int(items[i, 10]), int(items[i, 11]),
                                                                   int(items[i, 8]), int(items[i, 9]),
                                                                   int(items[i, 5]))))
            offsets[cls, 1:] = len(groups)
            continue
        for ph, (_, _, begin, end) in enumerate(phases.tolist()):
            offsets[cls, ph] = len(groups)
            shapes = {}
            for i in range(begin, end):
                if grad_class(items[i], a_entries) == cls:
                    shapes.setdefault(tuple(int(v) for v in items[i, :5]), []).append(i)
            if cls == GRAD_SLOT_RUN_CLASS:
                groups.extend(_balanced_runs(shapes, items, lambda i: (int(items[i, 9]), int(items[i, 10]),
                                                                       int(items[i, 8]), int(items[i, 5]))))
                continue
            pairs, costs = [], []
            for key in sorted(shapes):
                idx = sorted(shapes[key], key=lambda i: (int(items[i, 5]), int(items[i, 6])))
                c = _pair_cost(items, idx[0])
                for u in range(0, len(idx), GRAD_GROUP):
                    g = idx[u:u + GRAD_GROUP]
                    pairs.append(g + [-1] * (GRAD_GROUP - len(g)))
                    costs.append(c)
            groups.extend(_round_robin_balanced(pairs, costs))
        offsets[cls, -1] = len(groups)
    return np.asarray(groups, dtype=np.int32).reshape(-1, GRAD_GROUP), offsets.reshape(-1)


def _sym_grad_terms(sym_out_rows, s_fac, s_co, W):
    """Component-major derivative table of the symmetric outputs.

    For a monomial ``c prod_k x_{f_k}`` of output ``o`` and each distinct
    component ``p`` among its factors (multiplicity ``m``), the derivative
    ``m c prod_{k != one p} x_{f_k}`` is listed under ``p`` (the component's
    index inside its radial channel, ``l^2 + m + l``).  Returns offsets
    ``[W + 1]``, ``index [T, 2]`` (output, 4 x u8 remaining factors with
    255 unused) and ``coeff [T]``.
    """
    per = [[] for _ in range(W)]
    for o, (base, tb, te, _) in enumerate(sym_out_rows):
        for q in range(tb, te):
            comps = [base + ci for ci in s_fac[q] if ci != 255]
            for p in sorted(set(comps)):
                rest = list(comps)
                rest.remove(p)
                packed = 0
                for k in range(4):
                    packed |= (rest[k] if k < len(rest) else 255) << (8 * k)
                per[p].append((o, packed, comps.count(p) * s_co[q]))
    offsets = np.zeros(W + 1, dtype=np.int32)
    index, coeff = [], []
    for p in range(W):
        for o, packed, c in per[p]:
            index.append((o, np.uint32(packed).view(np.int32)))
            coeff.append(c)
        offsets[p + 1] = len(index)
    return (offsets, np.asarray(index, dtype=np.int32).reshape(-1, 2),
            np.asarray(coeff, dtype=np.float64))


def pack_bundle(bundle: ACEBundle, device) -> PackedBundle:
    device = torch.device(device)
    nmax, lmax = bundle.nmax, bundle.lmax
    W = (lmax + 1) ** 2
    # symmetric outputs of one radial channel (one shared-memory slot)
    sym_keys = sorted(bundle.sym_tables)
    sym_local, sym_out_rows, s_fac, s_co = {}, [], [], []
    sym_flops = 0.0
    for key in sym_keys:
        t = bundle.sym_tables[key]
        l, k, Lam, mu = key
        sym_local[key] = len(sym_out_rows)
        vals = np.asarray(t.monomial_value)
        if np.iscomplexobj(vals) and vals.size and np.max(np.abs(vals.imag)) > 1e-12:
            raise ValueError(f"symmetric table {key} has complex coefficients; not supported by the fused kernel")
        offsets = np.asarray(t.output_offsets, dtype=np.int64)
        for o in range(2 * Lam + 1):
            tb = len(s_fac)
            for q in range(int(offsets[o]), int(offsets[o + 1])):
                s_fac.append(_factors(t.monomial_counts[q]))
                s_co.append(float(np.real(vals[q])))
                sym_flops += 6.0 * int(np.sum(t.monomial_counts[q])) + 2.0
            sym_out_rows.append([l * l, tb, len(s_fac), 0])
    sym_out_count = len(sym_out_rows)
    items, item_coef, phases = _build_items(bundle, sym_local, sym_out_count, W)
    max_blocks = max([p.block_count for p in bundle.patterns] + [1])
    fo = 0
    terms_per_atom = 0
    term_blocks_per_atom = 0
    for w in range(bundle.word_count):
        p = bundle.patterns[int(bundle.word_pattern_index[w])]
        fo += p.component_count
        terms_per_atom += p.term_count
        term_blocks_per_atom += p.term_count * p.block_count
    groups, group_offsets = _grad_groups(items, phases, nmax * W)
    unpacked = [[(f >> (8 * k)) & 255 for k in range(4)] for f in np.asarray(s_fac, dtype=np.uint32).tolist()]
    sg_off, sg_index, sg_coeff = _sym_grad_terms(sym_out_rows, unpacked, s_co, W)
    arrays_np = {
        "groups": groups,
        "group_offsets": group_offsets,
        "sym_grad_offsets": sg_off,
        "sym_grad_index": sg_index,
        "sym_grad_coeff": sg_coeff,
        "items": items,
        "item_coef": item_coef,
        "phases": phases,
        "sym_outputs": np.asarray(sym_out_rows, dtype=np.int32).reshape(-1, 4),
        "sym_term_factors": np.asarray(s_fac, dtype=np.uint32).view(np.int32),
        "sym_term_coeff": np.asarray(s_co, dtype=np.float64),
    }
    arrays = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in arrays_np.items()}
    # symmetric blocks of each visited slot channel are recomputed per phase change
    loads = 0
    prev = (None, None)
    for a, b2, _, _ in phases.tolist():
        loads += int(a != prev[0]) + int(b2 >= 0 and b2 != prev[1])
        prev = (a, b2)
    # a second symmetric slot only when some phase pairs two radial channels
    n_slots = 2 if any(int(ph[1]) >= 0 for ph in phases.tolist()) else 1
    pb = PackedBundle(bundle=bundle, device=device, arrays=arrays, pool_size=nmax * W + n_slots * sym_out_count,
                      feature_count=fo, max_blocks=max_blocks, sym_offsets=sym_local,
                      term_count_per_atom=terms_per_atom, term_block_count_per_atom=term_blocks_per_atom,
                      sym_term_count_per_atom=len(s_fac) * loads,
                      sym_flops_per_atom=sym_flops * loads)
    return pb
