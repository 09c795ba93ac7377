"""Recoupled plan of a scalar (L = 0) ACE bundle: every feature as a short sum of
contractions of coupled channel pairs.

A feature of the word ``((l_1, n_1), ..., (l_nu, n_nu))`` (nu <= 4, channels sorted) is a
rotation-invariant polynomial in the word's channel vectors
``a_i = A[n_i - 1, l_i^2 : (l_i + 1)^2]`` (complex Condon-Shortley components, ``m = -l .. l``).
The compiled schedule (``ye3t/core/couplings.py:481-567``) evaluates it term by term:
``F = sum_t c_t prod_j bv_j[m_tj]``, 1,332,116 terms per atom for the nu <= 4, l <= 3 word set.

The invariant multilinear forms on ``V_l1 x V_l2 x V_l3 x V_l4`` are spanned by the coupling
trees ``((l_1 l_2) L, (l_3 l_4) L) 0`` over the intermediate ``L`` in
``[|l_1 - l_2|, l_1 + l_2] & [|l_3 - l_4|, l_3 + l_4]``; a feature with repeated channels is
such a form evaluated on repeated arguments (the polarisation of an invariant polynomial is
invariant).  Hence, exactly,

    F_f = sum_L W[f, L] T_L,        T_L = sum_M (-1)^M I_A[M] I_B[-M],
    I_(a,b)^L[M] = sum_{m_a + m_b = M} <l_a m_a l_b m_b | L M> a[m_a] b[m_b],

with ``I_A`` the coupled first pair and ``I_B`` the coupled second pair.  Three-channel words
use the coupled first pair against the third channel (``L = l_3``), two-channel words the two
channels (``L = l_1 = l_2``), one-channel words the ``l = 0`` component.  The pair couplings
are shared by every word that contains the pair: for the nu <= 4, l <= 3, n <= 8 word set
(25,328 words, 41,168 features), 1,308 segments hold 6,920 coupled components per atom
(20,539 complex multiply-adds), and 41,168 contractions of 166,072 multiply-adds give every
feature, against the 1.33 M terms of the compiled schedules.

``W`` depends only on the word's pattern (its angular momenta and which channels repeat).
The builder fits it once per pattern on seeded random channel vectors: it evaluates the
pattern's schedule (block assembly as ``ye3t/workflows.py:636-661``, symmetric blocks as
``ye3t/runtime/symmetric_power.py:740-868``) and the candidate contractions, keeps the
cheapest contractions that span the features, and solves least squares.  It then checks the
fit on a second, independent sample.  ``W`` is therefore exact up to rounding (residuals
are about 1e-14 relative on the C5 set), and a pattern that does not fit raises.

The Clebsch-Gordan coefficients come from Racah's closed formula (G. Racah, Phys. Rev. 62,
438 (1942), eq. 16'); any fixed normalisation would do, since ``W`` absorbs it, but the
coupled components must be the irreducible ones so that only the needed ``L`` are stored.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from functools import lru_cache
from typing import Dict, List, Sequence, Tuple

import numpy as np

from .schedules import ACEBundle, ScheduleRecord, SymPowerTable

__all__ = ["clebsch_gordan", "cg_table", "RecoupledPlan", "RecoupledDeviceTables", "RecoupledSymTables",
           "RecoupledTiles", "TILE_STEP",
           "RecoupledEvaluator",
           "build_recoupled_plan", "ctypes_tables", "ctypes_sym_tables", "SEG_UNIT", "SEG_CHANNEL", "SEG_PAIR"]

SEG_UNIT, SEG_CHANNEL, SEG_PAIR = 0, 1, 2
_FIT_TOL = 1e-11


def clebsch_gordan(l1: int, m1: int, l2: int, m2: int, L: int, M: int) -> float:
    """``<l1 m1 l2 m2 | L M>`` for integer angular momenta (Racah's formula)."""
    if m1 + m2 != M or abs(m1) > l1 or abs(m2) > l2 or abs(M) > L or not abs(l1 - l2) <= L <= l1 + l2:
        return 0.0
    f = math.factorial
    pre = (2 * L + 1) * f(L + l1 - l2) * f(L - l1 + l2) * f(l1 + l2 - L) / f(l1 + l2 + L + 1)
    pre *= f(L + M) * f(L - M) * f(l1 - m1) * f(l1 + m1) * f(l2 - m2) * f(l2 + m2)
    s = 0.0
    for k in range(l1 + l2 - L + 1):
        d = (k, l1 + l2 - L - k, l1 - m1 - k, l2 + m2 - k, L - l2 + m1 + k, L - l1 - m2 + k)
        if min(d) < 0:
            continue
        s += (-1) ** k / float(np.prod([f(x) for x in d], dtype=np.float64))
    return math.sqrt(pre) * s


@lru_cache(maxsize=None)
def cg_table(l1: int, l2: int, L: int) -> Tuple[np.ndarray, np.ndarray]:
    """Nonzero couplings of ``V_l1 x V_l2 -> V_L``: ``(idx [K, 3], value [K])`` with rows
    ``(m1 + l1, m2 + l2, M + L)``, ordered by ``M`` then ``m1``."""
    rows, vals = [], []
    for M in range(-L, L + 1):
        for m1 in range(-l1, l1 + 1):
            m2 = M - m1
            if abs(m2) > l2:
                continue
            c = clebsch_gordan(l1, m1, l2, m2, L, M)
            if c != 0.0:
                rows.append((m1 + l1, m2 + l2, M + L))
                vals.append(c)
    return np.asarray(rows, dtype=np.int64).reshape(-1, 3), np.asarray(vals, dtype=np.float64)


def _couple(a: np.ndarray, la: int, b: np.ndarray, lb: int, L: int) -> np.ndarray:
    idx, val = cg_table(la, lb, L)
    out = np.zeros(a.shape[:-1] + (2 * L + 1,), dtype=np.result_type(a, b))
    np.add.at(out, (Ellipsis, idx[:, 2]), (val * a[..., idx[:, 0]] * b[..., idx[:, 1]]))
    return out


def _contract(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    L = (x.shape[-1] - 1) // 2
    sign = (-1.0) ** np.arange(-L, L + 1)
    return (sign * x * y[..., ::-1]).sum(axis=-1)


# -- the pattern's own features on sample channel vectors ------------------------------------
def _sym_values(table: SymPowerTable, x: np.ndarray) -> np.ndarray:
    """``out[s, o] = sum_t v_t prod_i x[s, i]^k[t, i]`` (grouped symmetric-power table)."""
    k = np.asarray(table.monomial_counts, dtype=np.int64)
    mono = np.prod(x[:, None, :] ** k[None, :, :], axis=2) * np.asarray(table.monomial_value)[None, :]
    off = np.asarray(table.output_offsets, dtype=np.int64)
    out = np.zeros((x.shape[0], off.shape[0] - 1), dtype=np.complex128)
    for o in range(off.shape[0] - 1):
        out[:, o] = mono[:, off[o]:off[o + 1]].sum(axis=1)
    return out


def _pattern_features(rec: ScheduleRecord, sym_tables: Dict, chan: Dict[Tuple[int, int], np.ndarray]) -> np.ndarray:
    """Schedule features ``[S, C]`` of a pattern record on channel vectors keyed ``(l, rank)``."""
    S = next(iter(chan.values())).shape[0]
    mdim = rec.max_block_m_dim
    bv = np.zeros((S, rec.basis_count, rec.block_count, mdim), dtype=np.complex128)
    for a, label in enumerate(rec.block_specs):
        for j, (kind, n, l, k, lam, mu) in enumerate(label):
            src = _sym_values(sym_tables[(l, k, lam, mu)], chan[(l, n)]) if kind == "sym" else chan[(l, n)]
            bv[:, a, j, :src.shape[1]] = src
    midx = rec.block_m_indices()
    counts = np.diff(rec.component_offsets)
    term_comp = np.repeat(np.arange(rec.component_count), counts)
    label = rec.component_label_index[term_comp]
    prod = np.broadcast_to(np.asarray(rec.coeffs)[None, :], (S, rec.term_count)).copy()
    for j in range(rec.block_count):
        prod = prod * bv[:, label, j, midx[:, j]]
    out = np.zeros((S, rec.component_count), dtype=np.complex128)
    np.add.at(out, (slice(None), term_comp), prod)
    return out


def _candidates(key: Sequence[Tuple[int, int]]) -> List[Tuple[Tuple, Tuple, int]]:
    """Candidate contractions of a word pattern: ``(segment A, segment B, L)`` with segments
    ``("unit",)``, ``("chan", i)`` or ``("pair", i, j)`` over word positions."""
    ls = [l for l, _ in key]
    if len(key) == 1:
        return [(("chan", 0), ("unit",), 0)] if ls[0] == 0 else []
    if len(key) == 2:
        return [(("chan", 0), ("chan", 1), ls[0])] if ls[0] == ls[1] else []
    if len(key) == 3:
        ok = abs(ls[0] - ls[1]) <= ls[2] <= ls[0] + ls[1]
        return [(("pair", 0, 1), ("chan", 2), ls[2])] if ok else []
    if len(key) == 4:
        lo = max(abs(ls[0] - ls[1]), abs(ls[2] - ls[3]))
        hi = min(ls[0] + ls[1], ls[2] + ls[3])
        return [(("pair", 0, 1), ("pair", 2, 3), L) for L in range(lo, hi + 1)]
    raise ValueError(f"words of {len(key)} channels are not supported (nu <= 4)")


def _segment_values(seg, L, key, chan):
    if seg[0] == "unit":
        return np.ones((next(iter(chan.values())).shape[0], 1), dtype=np.complex128)
    if seg[0] == "chan":
        return chan[key[seg[1]]]
    (la, ra), (lb, rb) = key[seg[1]], key[seg[2]]
    return _couple(chan[(la, ra)], la, chan[(lb, rb)], lb, L)


def _fit_pattern(rec: ScheduleRecord, key, sym_tables, seed: int):
    """Cheapest contractions spanning the pattern's features and their weights ``W [k, C]``."""
    cands = _candidates(key)
    C = rec.component_count
    ranks = sorted(set(key))

    def sample(rng, S):
        chan = {(l, r): rng.normal(size=(S, 2 * l + 1)) + 1j * rng.normal(size=(S, 2 * l + 1)) for l, r in ranks}
        F = _pattern_features(rec, sym_tables, chan)
        T = np.stack([_contract(_segment_values(a, L, key, chan), _segment_values(b, L, key, chan))
                      for a, b, L in cands], axis=1) if cands else np.zeros((S, 0), dtype=np.complex128)
        return F, T

    S = 12 + 3 * len(cands)
    F, T = sample(np.random.default_rng(seed), S)
    Fscale = max(float(np.abs(F).max()), 1e-300)
    order = sorted(range(len(cands)), key=lambda i: (cands[i][2], i))
    chosen: List[int] = []
    W = np.zeros((0, C), dtype=np.complex128)
    resid = float(np.abs(F).max()) / Fscale
    for i in order:
        if resid <= _FIT_TOL:
            break
        trial = chosen + [i]
        Tt = T[:, trial]
        if np.linalg.matrix_rank(Tt, tol=1e-10 * max(float(np.abs(Tt).max()), 1e-300)) < len(trial):
            continue
        Wt = np.linalg.lstsq(Tt, F, rcond=None)[0]
        chosen, W = trial, Wt
        resid = float(np.abs(Tt @ Wt - F).max()) / Fscale
    F2, T2 = sample(np.random.default_rng(seed + 1), S)
    check = float(np.abs(T2[:, chosen] @ W - F2).max()) / max(float(np.abs(F2).max()), 1e-300)
    if resid > _FIT_TOL or check > _FIT_TOL:
        raise ArithmeticError(f"pattern {key}: features are not spanned by the coupling trees "
                              f"(residual {max(resid, check):.3e})")
    return [cands[i] for i in chosen], W


@dataclass
class RecoupledPlan:
    """Segments, contractions and feature weights of a recoupled bundle.

    Per atom the evaluator forms every segment's components (``seg_offset`` into a
    ``[component_count]`` complex row, segments ordered by ``L``), then every contraction
    ``T_d = sum_M (-1)^M I[seg_a[d]][M] I[seg_b[d]][-M]`` (both segments of order ``dot_L[d]``;
    contractions ordered by ``L``, then first segment), then
    ``F[feat_index[z]] += feat_weight[z] T_d`` for ``z`` in ``dot_feat_offset[d] ..``.
    Channel ``c`` is ``(l, n) = (c % (lmax + 1), c // (lmax + 1) + 1)``; its components are
    ``A[n - 1, l^2 : (l + 1)^2]``.  A pair segment couples channels ``seg_a`` and ``seg_b``
    (``seg_a <= seg_b`` in the words' ``(l, n)`` order) through ``cg_table(l_a, l_b, L)``.
    """

    nmax: int
    lmax: int
    feature_count: int
    seg_kind: np.ndarray    # int8 [S]: SEG_UNIT, SEG_CHANNEL, SEG_PAIR
    seg_L: np.ndarray       # int32 [S]
    seg_a: np.ndarray       # int32 [S] channel (SEG_CHANNEL, SEG_PAIR), -1 for the unit segment
    seg_b: np.ndarray       # int32 [S] second channel of a pair, -1 otherwise
    seg_offset: np.ndarray  # int64 [S + 1] component offsets (ordered by L)
    dot_a: np.ndarray       # int32 [D]
    dot_b: np.ndarray       # int32 [D]
    dot_L: np.ndarray       # int32 [D]
    dot_word: np.ndarray    # int32 [D]
    dot_feat_offset: np.ndarray  # int64 [D + 1]
    feat_index: np.ndarray  # int64 [Z] global feature index
    feat_weight: np.ndarray  # float64 [Z] (real: the fitted weights of the C-S basis are real)

    @property
    def segment_count(self) -> int:
        return int(self.seg_kind.shape[0])

    @property
    def component_count(self) -> int:
        return int(self.seg_offset[-1])

    @property
    def dot_count(self) -> int:
        return int(self.dot_a.shape[0])

    def channel(self, c: int) -> Tuple[int, int]:
        return c % (self.lmax + 1), c // (self.lmax + 1) + 1

    def costs(self) -> Dict[str, int]:
        """Complex multiply-adds per atom: pair couplings, contractions, feature weights."""
        couple = 0
        for s in np.nonzero(self.seg_kind == SEG_PAIR)[0]:
            la, lb = self.channel(int(self.seg_a[s]))[0], self.channel(int(self.seg_b[s]))[0]
            couple += int(cg_table(la, lb, int(self.seg_L[s]))[1].shape[0])
        return {"pair_couplings": couple, "contractions": int((2 * self.dot_L + 1).sum()),
                "feature_weights": int(self.feat_weight.shape[0]), "components": self.component_count}

    def energy_weights(self, weights: np.ndarray) -> np.ndarray:
        """Per species, the real contraction weights ``k[s, d] = sum_f w[s, f] W[f, d]`` of the
        energy ``e = Re(sum_d k[z, d] T_d)`` (real readout ``w [species, feature_count]``)."""
        w = np.asarray(weights, dtype=np.float64)
        if w.ndim != 2 or w.shape[1] != self.feature_count:
            raise ValueError(f"weights must have shape [species, {self.feature_count}]")
        contrib = w[:, self.feat_index] * self.feat_weight[None, :]
        dot_of = np.repeat(np.arange(self.dot_count), np.diff(self.dot_feat_offset))
        k = np.zeros((w.shape[0], self.dot_count), dtype=np.float64)
        np.add.at(k, (slice(None), dot_of), contrib)
        return k

    def device_tables(self) -> "RecoupledDeviceTables":
        """The plan packed for the device pass (validated)."""
        return _device_tables(self)

    def sym_device_tables(self) -> "RecoupledSymTables":
        """The plan packed for the symmetric pass over physical densities (validated)."""
        return _sym_device_tables(self)

    def sym_tiles(self, rows: int = 8) -> "RecoupledTiles":
        """The symmetric pass's contraction lists as dense tiles of ``rows`` segments."""
        return _tiles(self, self.sym_device_tables(), rows)


@dataclass
class RecoupledDeviceTables:
    """The plan packed for the device pass over one atom (``y3b_recoupled_tables``).

    The kernel runs one pass per ``L``.  In pass ``L`` the components
    ``pass_begin[L] .. pass_begin[L + 1]`` are formed in shared memory (local index
    ``c - pass_begin[L]``), from the atom's A row of ``row_width`` complex entries:
    ``comp[c] = (a, b, cg_begin, cg_count, m, own_begin, own_count, 0)``.  ``a < 0`` is the
    unit; ``cg_count == 0`` copies ``A[a]``; otherwise
    ``I = sum_q cg_value[q] A[a + (cg_index[q] & 255)] A[b + (cg_index[q] >> 8)]``.
    Then each component's adjoint
    ``gI[c] = (-1)^(m - L) sum_q k[own[q, 1]] I[own[q, 0] + 2L - m]``
    (``q`` in ``own_begin .. + own_count``, ``own[q, 0]`` the partner segment's first local
    component, ``own[q, 1]`` the contraction), and the pass's energy share
    ``Re(I[c] gI[c]) / 2``.  Last, each A entry ``t`` adds
    ``sum_q bp_value[q] gI[bp_gi[q]] (A[bp_other[q]] or 1 when bp_other[q] < 0)`` over
    ``q`` in ``bp_begin[L * row_width + t] ..``."""

    pass_count: int
    max_pass_components: int
    row_width: int
    dot_count: int
    pass_begin: np.ndarray  # int32 [pass_count + 1]
    comp: np.ndarray        # int32 [C, 8]
    cg_index: np.ndarray    # int32 [K]
    cg_value: np.ndarray    # float64 [K]
    own: np.ndarray         # int32 [O, 2]
    bp_begin: np.ndarray    # int32 [pass_count * row_width + 1]
    bp_gi: np.ndarray       # int32 [Bp]
    bp_other: np.ndarray    # int32 [Bp]
    bp_value: np.ndarray    # float64 [Bp]
    feature_count: int = 0
    dot_begin: np.ndarray = None    # int32 [pass_count + 1] contractions of each pass
    dot: np.ndarray = None          # int32 [D, 4]: first local component of A, of B, feature range
    feat_index: np.ndarray = None   # int32 [Z]
    feat_weight: np.ndarray = None  # float64 [Z]

    def validate(self) -> None:
        """Every index the device pass follows stays inside its array or its pass."""
        P, W = self.pass_count, self.row_width
        pb = self.pass_begin.astype(np.int64)
        if pb.shape != (P + 1,) or pb[0] != 0 or np.any(np.diff(pb) < 0) or pb[-1] != self.comp.shape[0]:
            raise ValueError("pass_begin does not partition the components")
        if int(np.diff(pb).max(initial=0)) > self.max_pass_components:
            raise ValueError("a pass holds more components than max_pass_components")
        c = self.comp.astype(np.int64)
        Lc = np.repeat(np.arange(P), np.diff(pb))
        nc = np.diff(pb)[Lc]
        a, b, cg0, cgn, m, o0, on = (c[:, i] for i in range(7))
        unit, chan, pair = a < 0, (a >= 0) & (cgn == 0), cgn > 0
        if np.any(unit & ((a != -1) | (m != 0) | (Lc != 0))):
            raise ValueError("the unit component must be L = 0")
        if np.any(chan & (a >= W)):
            raise ValueError("channel component outside the A row")
        if np.any((m < 0) | (m > 2 * Lc)):
            raise ValueError("component m outside 0 .. 2L")
        if np.any(cg0 < 0) or np.any(cg0 + cgn > self.cg_value.shape[0]):
            raise ValueError("coupling range outside the coupling table")
        K = self.cg_index.astype(np.int64)
        for i in np.nonzero(pair)[0]:
            q = K[cg0[i]:cg0[i] + cgn[i]]
            if a[i] + (q & 255).max() >= W or b[i] < 0 or b[i] + (q >> 8).max() >= W:
                raise ValueError("coupling term outside the A row")
        if np.any(o0 < 0) or np.any(o0 + on > self.own.shape[0]):
            raise ValueError("adjoint list outside the list table")
        own = self.own.astype(np.int64)
        if own.size:
            idx = np.repeat(np.arange(c.shape[0]), on)
            q = np.concatenate([np.arange(o0[i], o0[i] + on[i]) for i in range(c.shape[0])]) if on.sum() else \
                np.zeros(0, dtype=np.int64)
            rd = own[q, 0] + 2 * Lc[idx] - m[idx]
            if np.any(own[q, 0] < 0) or np.any(rd >= nc[idx]) or np.any(rd < 0):
                raise ValueError("adjoint partner outside its pass")
            if np.any(own[q, 1] < 0) or np.any(own[q, 1] >= self.dot_count):
                raise ValueError("adjoint contraction outside the weights")
        bb = self.bp_begin.astype(np.int64)
        if bb.shape != (P * W + 1,) or bb[0] != 0 or np.any(np.diff(bb) < 0) or bb[-1] != self.bp_gi.shape[0]:
            raise ValueError("bp_begin does not partition the back-propagation entries")
        Lq = np.repeat(np.arange(P * W) // W, np.diff(bb))
        if np.any(self.bp_gi < 0) or np.any(self.bp_gi >= np.diff(pb)[Lq]):
            raise ValueError("back-propagation entry outside its pass")
        if np.any(self.bp_other >= W) or np.any(self.bp_other < -1):
            raise ValueError("back-propagation partner outside the A row")
        db = self.dot_begin.astype(np.int64)
        if db.shape != (P + 1,) or db[0] != 0 or np.any(np.diff(db) < 0) or db[-1] != self.dot_count \
                or self.dot.shape != (self.dot_count, 4):
            raise ValueError("dot_begin does not partition the contractions")
        dt = self.dot.astype(np.int64)
        Ld = np.repeat(np.arange(P), np.diff(db))
        ncd = np.diff(pb)[Ld]
        if np.any(dt[:, :2] < 0) or np.any(dt[:, 0] + 2 * Ld >= ncd) or np.any(dt[:, 1] + 2 * Ld >= ncd):
            raise ValueError("contraction segment outside its pass")
        if np.any(dt[:, 2] < 0) or np.any(dt[:, 3] < 0) or np.any(dt[:, 2] + dt[:, 3] > self.feat_index.shape[0]):
            raise ValueError("contraction feature range outside the feature table")
        if np.any(self.feat_index < 0) or np.any(self.feat_index >= self.feature_count):
            raise ValueError("feature index outside the features")

    def flops_per_atom(self) -> Dict[str, float]:
        """Real flops per atom of each pass, counted from the tables: a coupling term is a
        complex product scaled and added (10), a contraction term a complex multiply-add (8),
        an adjoint-list term a real weight times a complex value added (4), a coupled
        back-propagation term 10 and a copied one 2; the energy takes 2 per contraction
        (forward) or 4 per component (adjoint), a feature weight 4."""
        terms = float(self.comp[:, 3].astype(np.int64).sum())
        lists = float(self.comp[:, 6].astype(np.int64).sum())
        dot_L = np.repeat(np.arange(self.pass_count), np.diff(self.dot_begin.astype(np.int64)))
        macs = float((2 * dot_L + 1).sum())
        coupled = float((self.bp_other >= 0).sum())
        copied = float((self.bp_other < 0).sum())
        return {"energy": 10 * terms + 8 * macs + 2 * self.dot_count,
                "energy_grad": 10 * terms + 4 * lists + 4 * self.comp.shape[0] + 10 * coupled + 2 * copied,
                "features": 10 * terms + 8 * macs + 4 * float(self.feat_index.shape[0])}

    def smem_bytes(self) -> int:
        """Dynamic shared memory per atom of the adjoint pass: the A row and its adjoint, the
        pass's components and theirs (each region at least a row wide, since the
        back-propagation step stages its per-entry parts there)."""
        return 16 * (2 * self.row_width + 2 * max(self.row_width, self.max_pass_components))


def _device_tables(plan: "RecoupledPlan") -> RecoupledDeviceTables:
    L1 = plan.lmax + 1
    W = L1 * L1
    row_width = plan.nmax * W

    def base(c):  # first A-row entry of channel c
        l, n = c % L1, c // L1 + 1
        return (n - 1) * W + l * l

    P = int(plan.seg_L.max()) + 1 if plan.segment_count else 0
    seg_off = plan.seg_offset.astype(np.int64)
    pass_begin = np.zeros(P + 1, dtype=np.int64)
    for L in range(P):
        sel = np.nonzero(plan.seg_L == L)[0]
        pass_begin[L + 1] = seg_off[sel[-1] + 1] if sel.size else pass_begin[L]
    # coupling tables shared by (l_a, l_b, L, M)
    cg_index, cg_value, cg_at = [], [], {}

    def cg_range(la, lb, L, M):
        key = (la, lb, L, M)
        if key not in cg_at:
            idx, val = cg_table(la, lb, L)
            rows = np.nonzero(idx[:, 2] == M + L)[0]
            cg_at[key] = (len(cg_value), rows.shape[0])
            cg_index.extend(int(idx[r, 0]) | (int(idx[r, 1]) << 8) for r in rows)
            cg_value.extend(float(val[r]) for r in rows)
        return cg_at[key]

    # adjoint lists per segment: partner segment (local first component) and contraction
    lists: List[List[Tuple[int, int]]] = [[] for _ in range(plan.segment_count)]
    for d in range(plan.dot_count):
        a, b = int(plan.dot_a[d]), int(plan.dot_b[d])
        L = int(plan.dot_L[d])
        lists[a].append((int(seg_off[b] - pass_begin[L]), d))
        lists[b].append((int(seg_off[a] - pass_begin[L]), d))
    own, own_at = [], []
    for s in range(plan.segment_count):
        own_at.append(len(own))
        own.extend(lists[s])
    comp = np.zeros((int(seg_off[-1]), 8), dtype=np.int64)
    bp = [[[] for _ in range(row_width)] for _ in range(P)]
    for s in range(plan.segment_count):
        L, kind = int(plan.seg_L[s]), int(plan.seg_kind[s])
        for mi in range(2 * L + 1):
            c = int(seg_off[s]) + mi
            local = c - int(pass_begin[L])
            row = [-1, -1, 0, 0, mi, own_at[s], len(lists[s]), 0]
            if kind == SEG_CHANNEL:
                row[0] = base(int(plan.seg_a[s])) + mi
                bp[L][row[0]].append((local, -1, 1.0))
            elif kind == SEG_PAIR:
                ca, cb = int(plan.seg_a[s]), int(plan.seg_b[s])
                la, lb = ca % L1, cb % L1
                row[0], row[1] = base(ca), base(cb)
                q0, qn = cg_range(la, lb, L, mi - L)
                row[2], row[3] = q0, qn
                for q in range(q0, q0 + qn):
                    ia, ib, v = cg_index[q] & 255, cg_index[q] >> 8, cg_value[q]
                    bp[L][row[0] + ia].append((local, row[1] + ib, v))
                    bp[L][row[1] + ib].append((local, row[0] + ia, v))
            comp[c] = row
    bp_flat = [e for L in range(P) for t in range(row_width) for e in bp[L][t]]
    bp_begin = np.concatenate([[0], np.cumsum([len(bp[L][t]) for L in range(P) for t in range(row_width)])])
    dot_begin = np.searchsorted(plan.dot_L, np.arange(P + 1), side="left").astype(np.int64)
    dot_pass = plan.dot_L.astype(np.int64)
    dot = np.stack([seg_off[plan.dot_a] - pass_begin[dot_pass], seg_off[plan.dot_b] - pass_begin[dot_pass],
                    plan.dot_feat_offset[:-1], np.diff(plan.dot_feat_offset)], axis=1) if plan.dot_count else \
        np.zeros((0, 4), dtype=np.int64)
    tabs = RecoupledDeviceTables(
        feature_count=plan.feature_count, dot_begin=dot_begin.astype(np.int32), dot=dot.astype(np.int32),
        feat_index=plan.feat_index.astype(np.int32), feat_weight=np.ascontiguousarray(plan.feat_weight),
        pass_count=P, max_pass_components=int(np.diff(pass_begin).max(initial=0)), row_width=row_width,
        dot_count=plan.dot_count, pass_begin=pass_begin.astype(np.int32), comp=comp.astype(np.int32),
        cg_index=np.asarray(cg_index, dtype=np.int32), cg_value=np.asarray(cg_value, dtype=np.float64),
        own=np.asarray(own, dtype=np.int32).reshape(-1, 2), bp_begin=bp_begin.astype(np.int32),
        bp_gi=np.asarray([e[0] for e in bp_flat], dtype=np.int32),
        bp_other=np.asarray([e[1] for e in bp_flat], dtype=np.int32),
        bp_value=np.asarray([e[2] for e in bp_flat], dtype=np.float64))
    tabs.validate()
    return tabs


@dataclass
class RecoupledSymTables:
    """The plan packed for the symmetric device pass (``y3b_recoupled_sym_tables``), valid for
    physical densities, ``A[n, l, -m] = (-1)^m conj(A[n, l, m])`` (real radial functions and
    prefactors).  Then a segment of parity ``p`` (``l_a + l_b - L`` for a pair, 0 otherwise)
    has ``I[-M] = (-1)^(p + M) conj(I[M])``, and in a parity-even word set both segments of a
    contraction have the same parity, so only ``M >= 0`` is stored and

        gI[M] = (-1)^p conj(sum_q k[d_q] I_partner[M]),
        e = 1/2 Re(I[0] gI[0]) + sum_{M > 0} Re(I[M] gI[M]),

    and dE/dA has the density's symmetry: the pass forms the ``m >= 0`` half of each A row
    and mirrors the rest.  ``comp[c] = (a, b, cg_begin, cg_count, M, own_begin, own_count,
    (-1)^p)``; ``own`` as in the general tables with partners' first (``M = 0``) components;
    ``bp_gi`` is ``2 * component + (1 if the entry reads conj(gI) of a negative M)``;
    ``mirror[t]`` is ``2 * t_plus + (m & 1)`` for an A entry of negative ``m`` (``t_plus``
    the entry of ``-m``), else -1; ``dot[d] = (first local component of A, of B,
    (-1)^p_B, 0)`` for the forward energy ``T_d = (-1)^p_B (Re(I_A[0] conj(I_B[0])) +
    2 sum_{M > 0} Re(I_A[M] conj(I_B[M])))``."""

    pass_count: int
    max_pass_components: int
    row_width: int
    dot_count: int
    pass_begin: np.ndarray  # int32 [pass_count + 1]
    comp: np.ndarray        # int32 [C, 8]
    cg_index: np.ndarray    # int32 [K]
    cg_value: np.ndarray    # float64 [K]
    own: np.ndarray         # int32 [O, 2]
    bp_begin: np.ndarray    # int32 [pass_count * row_width + 1]
    bp_gi: np.ndarray       # int32 [Bp]
    bp_other: np.ndarray    # int32 [Bp]
    bp_value: np.ndarray    # float64 [Bp]
    mirror: np.ndarray      # int32 [row_width]
    dot_begin: np.ndarray   # int32 [pass_count + 1]
    dot: np.ndarray         # int32 [D, 4]

    def validate(self) -> None:
        P, W = self.pass_count, self.row_width
        pb = self.pass_begin.astype(np.int64)
        if pb.shape != (P + 1,) or pb[0] != 0 or np.any(np.diff(pb) < 0) or pb[-1] != self.comp.shape[0]:
            raise ValueError("pass_begin does not partition the components")
        if int(np.diff(pb).max(initial=0)) > self.max_pass_components:
            raise ValueError("a pass holds more components than max_pass_components")
        c = self.comp.astype(np.int64)
        Lc = np.repeat(np.arange(P), np.diff(pb))
        nc = np.diff(pb)[Lc]
        if np.any((c[:, 4] < 0) | (c[:, 4] > Lc)) or np.any(np.abs(c[:, 7]) != 1):
            raise ValueError("component M outside 0 .. L or parity sign not +-1")
        if np.any(c[:, 2] < 0) or np.any(c[:, 2] + c[:, 3] > self.cg_value.shape[0]):
            raise ValueError("coupling range outside the coupling table")
        if np.any(c[:, 0] >= W) or np.any((c[:, 3] > 0) & ((c[:, 1] < 0) | (c[:, 1] >= W))):
            raise ValueError("component channel outside the A row")
        if np.any(c[:, 5] < 0) or np.any(c[:, 5] + c[:, 6] > self.own.shape[0]):
            raise ValueError("adjoint list outside the list table")
        own = self.own.astype(np.int64)
        if own.size:
            idx = np.repeat(np.arange(c.shape[0]), c[:, 6])
            q = np.concatenate([np.arange(c[i, 5], c[i, 5] + c[i, 6]) for i in range(c.shape[0])])
            rd = own[q, 0] + c[idx, 4]
            if np.any(own[q, 0] < 0) or np.any(rd >= nc[idx]) or np.any(own[q, 1] < 0) or \
                    np.any(own[q, 1] >= self.dot_count):
                raise ValueError("adjoint partner outside its pass or weights")
        bb = self.bp_begin.astype(np.int64)
        if bb.shape != (P * W + 1,) or bb[0] != 0 or np.any(np.diff(bb) < 0) or bb[-1] != self.bp_gi.shape[0]:
            raise ValueError("bp_begin does not partition the back-propagation entries")
        Lq = np.repeat(np.arange(P * W) // W, np.diff(bb))
        if np.any(self.bp_gi < 0) or np.any((self.bp_gi >> 1) >= np.diff(pb)[Lq]):
            raise ValueError("back-propagation entry outside its pass")
        if np.any(self.bp_other >= W) or np.any(self.bp_other < -1):
            raise ValueError("back-propagation partner outside the A row")
        m = self.mirror.astype(np.int64)
        if m.shape != (W,) or np.any((m >= 0) & ((m >> 1) >= W)):
            raise ValueError("mirror entry outside the A row")
        db = self.dot_begin.astype(np.int64)
        if db.shape != (P + 1,) or db[0] != 0 or db[-1] != self.dot_count or self.dot.shape != (self.dot_count, 4):
            raise ValueError("dot_begin does not partition the contractions")
        Ld = np.repeat(np.arange(P), np.diff(db))
        dt = self.dot.astype(np.int64)
        if np.any(dt[:, :2] < 0) or np.any(dt[:, 0] + Ld >= np.diff(pb)[Ld]) or \
                np.any(dt[:, 1] + Ld >= np.diff(pb)[Ld]) or np.any(np.abs(dt[:, 2]) != 1):
            raise ValueError("contraction segment outside its pass")

    def smem_bytes(self) -> int:
        """Dynamic shared memory per atom of the adjoint pass: the A row and its adjoint, the
        pass's components and theirs (each region at least a row wide, since the
        back-propagation step stages its per-entry parts there)."""
        return 16 * (2 * self.row_width + 2 * max(self.row_width, self.max_pass_components))

    def flops_per_atom(self) -> Dict[str, float]:
        """Real flops per atom of the symmetric passes, counted as
        ``RecoupledDeviceTables.flops_per_atom`` counts the general ones (a contraction term of
        the forward energy, the real part of one complex product with its weight, counts 4)."""
        terms = float(self.comp[:, 3].astype(np.int64).sum())
        lists = float(self.comp[:, 6].astype(np.int64).sum())
        dot_L = np.repeat(np.arange(self.pass_count), np.diff(self.dot_begin.astype(np.int64)))
        halves = float((dot_L + 1).sum())
        coupled = float((self.bp_other >= 0).sum())
        copied = float((self.bp_other < 0).sum())
        return {"energy": 10 * terms + 4 * halves + 2 * self.dot_count,
                "energy_grad": 10 * terms + 4 * lists + 4 * self.comp.shape[0] + 10 * coupled + 2 * copied}


# Steps of a tile's column walk are padded to a multiple of this, so that the kernel
# reads four column offsets as one int4 and a row's four weights as two double2.
TILE_STEP = 4


@dataclass
class RecoupledTiles:
    """The contraction lists of the symmetric pass regrouped as dense tiles.

    Per pass ``L`` the adjoint of the components is ``J[s] = sum_s' K[z][s, s'] I[s']``
    over the pass's segments, with ``K[z]`` symmetric: a contraction ``d`` of segments
    ``(a, b)`` adds ``k[z, d]`` to ``K[a, b]`` and to ``K[b, a]`` (``2 k`` on the diagonal
    when ``a == b``).  A tile is ``rows`` segments (rows; ``-1`` pads a short tile) and
    the union of their nonzero columns, walked column by column: every lane of a warp
    holds one (row, atom), so one shared-memory read of a column component serves all the
    tile's rows.  Rows with the same column set share a tile where they can; the rest are
    merged greedily by the growth of the column union.  ``tile_row[t, r]`` and
    ``col_comp[q]`` are local component offsets of the segments' ``M = 0`` components (the
    symmetric layout, ``L + 1`` components per segment); a tile's columns
    ``[tile_col_begin[t], tile_col_begin[t + 1])`` are padded to a multiple of
    ``TILE_STEP`` with column 0 and weight 0.  The weights of species ``z`` are
    ``kval[z, rows * q + r]`` for column step ``q`` and tile row ``r`` (one step's
    weights of all rows contiguous; ``tile_weights``); ``dot_pos[d]`` are the two
    entries contraction ``d`` adds to.
    Tiles within a pass are ordered by decreasing column count."""

    rows: int
    pass_count: int
    tile_begin: np.ndarray      # int32 [pass_count + 1]
    tile_row: np.ndarray        # int32 [T, rows]
    tile_col_begin: np.ndarray  # int32 [T + 1]
    col_comp: np.ndarray        # int32 [Q]
    dot_pos: np.ndarray         # int64 [D, 2]
    nonzero: int                # (row, column) pairs with a contraction
    # back-propagation work items: each A-row entry's list of a pass cut into chunks of at
    # most ``bp_chunk`` entries, (entry t, first, end) into the symmetric tables' bp
    # arrays, longest first within a pass; t_item lists each entry's items in list order
    bp_chunk: int = 0
    bp_item_begin: np.ndarray = None  # int32 [pass_count + 1]
    bp_item: np.ndarray = None        # int32 [I, 4]: (t, q0, q1, 0)
    t_item_begin: np.ndarray = None   # int32 [pass_count * row_width + 1]
    t_item: np.ndarray = None         # int32 [I]: item index within its pass
    # the items' entries as 16-byte records (code, other, value) interleaved per group
    # of ``rows`` consecutive items of a pass: entry k of item j of group g at
    # bp_group_off[g] + k * rows + j, padded with null records (other -1, value 0) to
    # the group's longest item, so that a warp reads one contiguous row of records
    bp_group_begin: np.ndarray = None  # int32 [pass_count + 1]
    bp_group_off: np.ndarray = None    # int32 [groups + 1]
    bp_pack: np.ndarray = None         # int32 [packed, 4]: (code, other, value bits lo, hi)
    # step-2 work units: a tile's column steps cut into chunks of at most about
    # ``unit_quads`` quads of TILE_STEP steps, so that the warps of a CTA get even shares;
    # unit (tile, first step, end step, kind): kind -1 a whole tile, -2 the first chunk
    # of a cut tile (its sums go to the components' adjoint slots), s >= 0 a later chunk
    # (its sums go to scratch slot s); fix[f] = (tile, first slot, slot count, 0) adds a
    # cut tile's later chunks in slot order.  Units are ordered by decreasing length.
    unit_quads: int = 0
    scratch_slots: int = 0
    unit_begin: np.ndarray = None  # int32 [pass_count + 1]
    unit: np.ndarray = None        # int32 [U, 4]
    fix_begin: np.ndarray = None   # int32 [pass_count + 1]
    fix: np.ndarray = None         # int32 [F, 4]

    @property
    def tile_count(self) -> int:
        return int(self.tile_row.shape[0])

    @property
    def step_count(self) -> int:
        return int(self.col_comp.shape[0])

    def tile_weights(self, k: np.ndarray) -> np.ndarray:
        """``kval [species, rows * step_count]`` from the contraction weights ``k [species, D]``."""
        k = np.asarray(k, dtype=np.float64)
        out = np.zeros((k.shape[0], self.rows * self.step_count), dtype=np.float64)
        for z in range(k.shape[0]):
            np.add.at(out[z], self.dot_pos[:, 0], k[z])
            np.add.at(out[z], self.dot_pos[:, 1], k[z])
        return out

    def efficiency(self) -> float:
        """Nonzero (row, column) pairs over the padded tile entries the kernel walks."""
        return self.nonzero / max(1, self.rows * self.step_count)

    def validate(self, sym: "RecoupledSymTables") -> None:
        P, R = self.pass_count, self.rows
        tb = tb_ = self.tile_begin.astype(np.int64)
        if tb.shape != (P + 1,) or tb[0] != 0 or np.any(np.diff(tb) < 0) or tb[-1] != self.tile_count:
            raise ValueError("tile_begin does not partition the tiles")
        if self.tile_row.shape != (self.tile_count, R):
            raise ValueError("tile_row must be [tiles, rows]")
        cb = self.tile_col_begin.astype(np.int64)
        if cb.shape != (self.tile_count + 1,) or cb[0] != 0 or cb[-1] != self.step_count or \
                np.any(np.diff(cb) < 0) or np.any(np.diff(cb) % TILE_STEP):
            raise ValueError("tile_col_begin does not partition the steps in multiples of TILE_STEP")
        nc = np.diff(sym.pass_begin.astype(np.int64))
        Lt = np.repeat(np.arange(P), np.diff(tb))
        rows = self.tile_row.astype(np.int64)
        if np.any((rows >= 0) & (rows + Lt[:, None] >= nc[Lt][:, None])) or np.any(rows < -1):
            raise ValueError("tile row outside its pass")
        Lq = np.repeat(Lt, np.diff(cb))
        if np.any(self.col_comp < 0) or np.any(self.col_comp.astype(np.int64) + Lq >= nc[Lq]):
            raise ValueError("tile column outside its pass")
        if np.any(self.dot_pos < 0) or np.any(self.dot_pos >= R * self.step_count):
            raise ValueError("contraction position outside the weights")
        W = sym.row_width
        ib = self.bp_item_begin.astype(np.int64)
        if ib.shape != (P + 1,) or ib[0] != 0 or np.any(np.diff(ib) < 0) or ib[-1] != self.bp_item.shape[0]:
            raise ValueError("bp_item_begin does not partition the work items")
        cwidth = max(sym.max_pass_components, W)
        if np.any(np.diff(ib) > cwidth):
            raise ValueError("a pass has more back-propagation items than its part buffer holds")
        it = self.bp_item.astype(np.int64)
        Li = np.repeat(np.arange(P), np.diff(ib))
        bb = sym.bp_begin.astype(np.int64)
        if it.size and (np.any(it[:, 0] < 0) or np.any(it[:, 0] >= W) or np.any(it[:, 1] > it[:, 2]) or
                        np.any(it[:, 1] < bb[Li * W + it[:, 0]]) or np.any(it[:, 2] > bb[Li * W + it[:, 0] + 1])):
            raise ValueError("work item outside its entry's back-propagation list")
        tb = self.t_item_begin.astype(np.int64)
        if tb.shape != (P * W + 1,) or tb[0] != 0 or tb[-1] != self.t_item.shape[0] or np.any(np.diff(tb) < 0):
            raise ValueError("t_item_begin does not partition the items")
        Lt = np.repeat(np.arange(P * W) // W, np.diff(tb))
        if np.any(self.t_item < 0) or np.any(self.t_item >= np.diff(ib)[Lt]):
            raise ValueError("entry item outside its pass")
        gb = self.bp_group_begin.astype(np.int64)
        go = self.bp_group_off.astype(np.int64)
        if gb.shape != (P + 1,) or gb[0] != 0 or gb[-1] != go.shape[0] - 1 or np.any(np.diff(gb) < 0):
            raise ValueError("bp_group_begin does not partition the groups")
        if go[0] != 0 or go[-1] != self.bp_pack.shape[0] or np.any(np.diff(go) % R) or np.any(np.diff(go) < 0):
            raise ValueError("bp_group_off does not cut the records into rows of whole groups")
        if np.any(np.diff(gb) * R < np.diff(ib)) or np.any((np.diff(gb) - 1) * R >= np.maximum(np.diff(ib), 1)):
            raise ValueError("the groups of a pass do not hold its items")
        ub = self.unit_begin.astype(np.int64)
        if ub.shape != (P + 1,) or ub[0] != 0 or ub[-1] != self.unit.shape[0] or np.any(np.diff(ub) < 0):
            raise ValueError("unit_begin does not partition the work units")
        un = self.unit.astype(np.int64)
        Lu = np.repeat(np.arange(P), np.diff(ub))
        if un.size and (np.any(un[:, 0] < tb_[Lu]) or np.any(un[:, 0] >= tb_[Lu + 1]) or
                        np.any(un[:, 1] < 0) or np.any(un[:, 2] < un[:, 1]) or np.any(un[:, 1] % TILE_STEP) or
                        np.any(un[:, 2] % TILE_STEP) or np.any(un[:, 2] > np.diff(cb)[un[:, 0]]) or
                        np.any(un[:, 3] < -2) or np.any(un[:, 3] >= self.scratch_slots)):
            raise ValueError("work unit outside its pass, tile or scratch")
        fb = self.fix_begin.astype(np.int64)
        if fb.shape != (P + 1,) or fb[0] != 0 or fb[-1] != self.fix.shape[0] or np.any(np.diff(fb) < 0):
            raise ValueError("fix_begin does not partition the fix-ups")
        fx = self.fix.astype(np.int64)
        Lf = np.repeat(np.arange(P), np.diff(fb))
        mc = np.arange(P) + 1
        if fx.size and (np.any(fx[:, 1] < 0) or np.any(fx[:, 2] < 1) or
                        np.any((fx[:, 1] + fx[:, 2]) * mc[Lf] > self.scratch_slots)):
            raise ValueError("fix-up outside the scratch")
        if un.size and np.any((un[:, 3] >= 0) & ((un[:, 3] + 1) * mc[Lu] > self.scratch_slots)):
            raise ValueError("work unit's slot outside the scratch")
        pk = self.bp_pack.astype(np.int64)
        Lg = np.repeat(np.arange(P), np.diff(gb))
        Lr = np.repeat(Lg, np.diff(go))
        if pk.size and (np.any(pk[:, 0] < 0) or np.any((pk[:, 0] >> 1) >= nc[Lr]) or np.any(pk[:, 1] < -1) or
                        np.any(pk[:, 1] >= W)):
            raise ValueError("packed back-propagation record outside its pass or row")


def _parity_interleave(cols, off, base) -> list:
    """A tile's columns ordered so that consecutive columns alternate between even and odd
    component indices while both remain: the kernel reads the 4 columns of a step as 64-byte
    rows of shared memory, and rows of one parity share a half of the banks."""
    even = [c for c in cols if (int(off[c]) - base) % 2 == 0]
    odd = [c for c in cols if (int(off[c]) - base) % 2 == 1]
    out = []
    while even or odd:
        if even:
            out.append(even.pop(0))
        if odd:
            out.append(odd.pop(0))
    return out


def _tiles(plan: "RecoupledPlan", sym: RecoupledSymTables, rows: int) -> RecoupledTiles:
    if rows < 1 or rows > 32:
        raise ValueError("rows per tile must be in [1, 32]")
    half = plan.seg_L.astype(np.int64) + 1
    off = np.concatenate([[0], np.cumsum(half)])
    P = sym.pass_count
    tile_begin, tile_row, col_begin, col_comp = [0], [], [0], []
    pos_of = {}  # (global row segment, global column segment) -> flat weight index
    nonzero = 0
    for L in range(P):
        segs = np.nonzero(plan.seg_L == L)[0]
        support: Dict[int, set] = {int(s): set() for s in segs}
        for d in np.nonzero(plan.dot_L == L)[0]:
            a, b = int(plan.dot_a[d]), int(plan.dot_b[d])
            support[a].add(b)
            support[b].add(a)
        nonzero += sum(len(v) for v in support.values())
        groups: Dict[frozenset, List[int]] = {}
        for s in segs:
            groups.setdefault(frozenset(support[int(s)]), []).append(int(s))
        tiles, left = [], []
        for sig, members in sorted(groups.items(), key=lambda g: (-len(g[0]), min(g[1]))):
            while len(members) >= rows:
                tiles.append(members[:rows])
                members = members[rows:]
            left.extend(members)
        left.sort(key=lambda s: (min(support[s], default=-1), len(support[s]), s))
        while left:
            t = [left.pop(0)]
            union = set(support[t[0]])
            while len(t) < rows and left:
                best = min(range(len(left)), key=lambda i: (len(union | support[left[i]]) - len(union), i))
                t.append(left.pop(best))
                union |= support[t[-1]]
            tiles.append(t)
        cols_of = [sorted(set().union(*(support[s] for s in t))) for t in tiles]
        order = sorted(range(len(tiles)), key=lambda i: (-len(cols_of[i]), i))
        base = int(sym.pass_begin[L])
        for i in order:
            t, cols = tiles[i], _parity_interleave(cols_of[i], off, base)
            n = len(cols)
            npad = (n + TILE_STEP - 1) // TILE_STEP * TILE_STEP if n else 0
            q0 = col_begin[-1]
            for r, srow in enumerate(t):
                for qi, scol in enumerate(cols):
                    pos_of[(srow, scol)] = rows * (q0 + qi) + r
            tile_row.append([int(off[s]) - base for s in t] + [-1] * (rows - len(t)))
            col_comp.extend(int(off[c]) - base for c in cols)
            col_comp.extend([0] * (npad - n))
            col_begin.append(q0 + npad)
        tile_begin.append(len(tile_row))
    dot_pos = np.asarray([(pos_of[(int(a), int(b))], pos_of[(int(b), int(a))])
                          for a, b in zip(plan.dot_a, plan.dot_b)], dtype=np.int64).reshape(-1, 2)
    # back-propagation work items: chunks of BP_CHUNK entries, doubled while a pass's item
    # count would exceed its part buffer
    W = sym.row_width
    cwidth = max(sym.max_pass_components, W)
    bb = sym.bp_begin.astype(np.int64)
    chunk = BP_CHUNK
    while True:
        items_per_pass = [int(sum(max(1, -(-int(bb[L * W + t + 1] - bb[L * W + t]) // chunk)) if
                                  bb[L * W + t + 1] > bb[L * W + t] else 0 for t in range(W))) for L in range(P)]
        if max(items_per_pass, default=0) <= cwidth or chunk >= 1 << 20:
            break
        chunk *= 2
    item_begin, items, t_begin, t_items = [0], [], [0], []
    for L in range(P):
        pass_items = []
        for t in range(W):
            q0, q1 = int(bb[L * W + t]), int(bb[L * W + t + 1])
            for q in range(q0, q1, chunk):
                pass_items.append((t, q, min(q1, q + chunk)))
        order = sorted(range(len(pass_items)), key=lambda i: (-(pass_items[i][2] - pass_items[i][1]), i))
        where = np.empty(len(pass_items), dtype=np.int64)
        where[np.asarray(order, dtype=np.int64)] = np.arange(len(pass_items))
        items.extend((pass_items[i][0], pass_items[i][1], pass_items[i][2], 0) for i in order)
        item_begin.append(len(items))
        per_t: List[List[int]] = [[] for _ in range(W)]
        for i, (t, _, _) in enumerate(pass_items):
            per_t[t].append(int(where[i]))
        for t in range(W):
            t_items.extend(per_t[t])
            t_begin.append(len(t_items))
    # pack the items' entries per group of ``rows`` items
    group_begin, group_off, pack = [0], [0], []
    vbits = sym.bp_value.astype(np.float64).view(np.int32).reshape(-1, 2)
    for L in range(P):
        pass_items = items[item_begin[L]:item_begin[L + 1]]
        for g0 in range(0, len(pass_items), rows):
            grp = pass_items[g0:g0 + rows]
            longest = max(q1 - q0 for _, q0, q1, _ in grp)
            for k in range(longest):
                for j in range(rows):
                    if j < len(grp) and grp[j][1] + k < grp[j][2]:
                        q = grp[j][1] + k
                        pack.append((int(sym.bp_gi[q]), int(sym.bp_other[q]), int(vbits[q, 0]), int(vbits[q, 1])))
                    else:
                        pack.append((0, -1, 0, 0))
            group_off.append(len(pack))
        group_begin.append(len(group_off) - 1)
    tiles = RecoupledTiles(rows=rows, pass_count=P, tile_begin=np.asarray(tile_begin, dtype=np.int32),
                           tile_row=np.asarray(tile_row, dtype=np.int32).reshape(-1, rows),
                           tile_col_begin=np.asarray(col_begin, dtype=np.int32),
                           col_comp=np.asarray(col_comp, dtype=np.int32), dot_pos=dot_pos, nonzero=nonzero,
                           bp_chunk=chunk, bp_item_begin=np.asarray(item_begin, dtype=np.int32),
                           bp_item=np.asarray(items, dtype=np.int32).reshape(-1, 4),
                           t_item_begin=np.asarray(t_begin, dtype=np.int32),
                           t_item=np.asarray(t_items, dtype=np.int32),
                           bp_group_begin=np.asarray(group_begin, dtype=np.int32),
                           bp_group_off=np.asarray(group_off, dtype=np.int32),
                           bp_pack=np.asarray(pack, dtype=np.int32).reshape(-1, 4))
    _plan_units(tiles)
    tiles.validate(sym)
    return tiles


# Step-2 work units: the cuts aim at about two units for each of UNIT_WARPS warps (of
# the CTA's 16: coarser units than one pair per warp need fewer cut tiles and fix-ups,
# which measured 1 % faster at 8 than at 16 or 4), and the scratch bytes a CTA holds
# for the partial sums of cut tiles (a slot of a pass holds one chunk's sums: 8 rows x
# (L + 1) components x 4 atoms, complex, 512 (L + 1) bytes).
UNIT_WARPS = 8
SCRATCH_BYTES = 12 * 1024

# Entries per back-propagation work item (step 3), doubled for a pass whose items
# would not fit its part buffer; 16 measured faster than 8, 24 or 32.
BP_CHUNK = 16


def _plan_units(tiles: RecoupledTiles) -> None:
    """Cut each pass's tiles into work units of at most ``q`` quads, the smallest ``q``
    that gives about two units per warp and fits the cut tiles' later chunks into the
    scratch slots."""
    P = tiles.pass_count
    quads = np.diff(tiles.tile_col_begin.astype(np.int64)) // TILE_STEP
    unit_begin, units, fix_begin, fixes = [0], [], [0], []
    qmax_all = 0
    for L in range(P):
        t0, t1 = int(tiles.tile_begin[L]), int(tiles.tile_begin[L + 1])
        n = quads[t0:t1]
        total = int(n.sum())
        slots = SCRATCH_BYTES // (512 * (L + 1))
        q = max(1, -(-total // (2 * UNIT_WARPS)))
        while True:
            extra = int(sum(max(0, -(-int(x) // q) - 1) for x in n))
            if extra <= slots or q >= int(n.max(initial=1)):
                break
            q += 1
        pass_units, slot = [], 0
        for i, x in enumerate(n):
            tile = t0 + i
            k = max(1, -(-int(x) // q))
            if k == 1:
                pass_units.append((tile, 0, int(x) * TILE_STEP, -1))
                continue
            cuts = [int(x) * j // k for j in range(k + 1)]
            fixes.append((tile, slot, k - 1, 0))
            for j in range(k):
                kind = -2 if j == 0 else slot + j - 1
                pass_units.append((tile, cuts[j] * TILE_STEP, cuts[j + 1] * TILE_STEP, kind))
            slot += k - 1
        pass_units.sort(key=lambda u: (-(u[2] - u[1]), u[0], u[1]))
        units.extend(pass_units)
        unit_begin.append(len(units))
        fix_begin.append(len(fixes))
        qmax_all = max(qmax_all, q)
    tiles.unit_quads = qmax_all
    tiles.scratch_slots = SCRATCH_BYTES // 512
    tiles.unit_begin = np.asarray(unit_begin, dtype=np.int32)
    tiles.unit = np.asarray(units, dtype=np.int32).reshape(-1, 4)
    tiles.fix_begin = np.asarray(fix_begin, dtype=np.int32)
    tiles.fix = np.asarray(fixes, dtype=np.int32).reshape(-1, 4)


def _sym_device_tables(plan: "RecoupledPlan") -> RecoupledSymTables:
    L1 = plan.lmax + 1
    W = L1 * L1
    row_width = plan.nmax * W

    def base(c):
        l, n = c % L1, c // L1 + 1
        return (n - 1) * W + l * l

    def parity(s):
        L, kind = int(plan.seg_L[s]), int(plan.seg_kind[s])
        if kind != SEG_PAIR:
            return 0
        return (int(plan.seg_a[s]) % L1 + int(plan.seg_b[s]) % L1 - L) & 1

    S = plan.segment_count
    P = int(plan.seg_L.max()) + 1 if S else 0
    for d in range(plan.dot_count):
        if parity(int(plan.dot_a[d])) != parity(int(plan.dot_b[d])):
            raise ValueError("the symmetric pass needs a parity-even word set")
    # M >= 0 layout: segment s holds L + 1 components
    half = (plan.seg_L.astype(np.int64) + 1)
    off = np.concatenate([[0], np.cumsum(half)])
    pass_begin = np.zeros(P + 1, dtype=np.int64)
    for L in range(P):
        sel = np.nonzero(plan.seg_L == L)[0]
        pass_begin[L + 1] = off[sel[-1] + 1] if sel.size else pass_begin[L]
    cg_index, cg_value, cg_at = [], [], {}

    def cg_range(la, lb, L, M):
        key = (la, lb, L, M)
        if key not in cg_at:
            idx, val = cg_table(la, lb, L)
            rows = np.nonzero(idx[:, 2] == M + L)[0]
            cg_at[key] = (len(cg_value), rows.shape[0])
            cg_index.extend(int(idx[r, 0]) | (int(idx[r, 1]) << 8) for r in rows)
            cg_value.extend(float(val[r]) for r in rows)
        return cg_at[key]

    lists: List[List[Tuple[int, int]]] = [[] for _ in range(S)]
    for d in range(plan.dot_count):
        a, b = int(plan.dot_a[d]), int(plan.dot_b[d])
        L = int(plan.dot_L[d])
        lists[a].append((int(off[b] - pass_begin[L]), d))
        lists[b].append((int(off[a] - pass_begin[L]), d))
    own, own_at = [], []
    for s in range(S):
        own_at.append(len(own))
        own.extend(lists[s])
    comp = np.zeros((int(off[-1]), 8), dtype=np.int64)
    bp = [[[] for _ in range(row_width)] for _ in range(P)]
    for s in range(S):
        L, kind, p = int(plan.seg_L[s]), int(plan.seg_kind[s]), parity(s)
        for M in range(L + 1):
            c = int(off[s]) + M
            local = c - int(pass_begin[L])
            row = [-1, -1, 0, 0, M, own_at[s], len(lists[s]), -1 if p else 1]
            if kind == SEG_CHANNEL:
                row[0] = base(int(plan.seg_a[s])) + L + M
            elif kind == SEG_PAIR:
                ca, cb = int(plan.seg_a[s]), int(plan.seg_b[s])
                la, lb = ca % L1, cb % L1
                row[0], row[1] = base(ca), base(cb)
                row[2], row[3] = cg_range(la, lb, L, M)
            comp[c] = row
        # back-propagation into the m >= 0 half of the A row, over every M of the segment
        if kind == SEG_CHANNEL:
            for M in range(L + 1):
                t = base(int(plan.seg_a[s])) + L + M
                bp[L][t].append((2 * (int(off[s]) + M - int(pass_begin[L])), -1, 1.0))
        elif kind == SEG_PAIR:
            ca, cb = int(plan.seg_a[s]), int(plan.seg_b[s])
            la, lb = ca % L1, cb % L1
            idx, val = cg_table(la, lb, L)
            for (ia, ib, im), v in zip(idx, val):
                M = int(im) - L
                gi = int(off[s]) + abs(M) - int(pass_begin[L])
                conj = 1 if M < 0 else 0
                sign = (-1.0) ** ((p + M) & 1) if M < 0 else 1.0
                ma, mb = int(ia) - la, int(ib) - lb
                if ma >= 0:
                    bp[L][base(ca) + int(ia)].append((2 * gi + conj, base(cb) + int(ib), sign * float(v)))
                if mb >= 0:
                    bp[L][base(cb) + int(ib)].append((2 * gi + conj, base(ca) + int(ia), sign * float(v)))
    bp_flat = [e for L in range(P) for t in range(row_width) for e in bp[L][t]]
    bp_begin = np.concatenate([[0], np.cumsum([len(bp[L][t]) for L in range(P) for t in range(row_width)])])
    mirror = np.full(row_width, -1, dtype=np.int64)
    for n in range(plan.nmax):
        for l in range(L1):
            for m in range(-l, 0):
                t = n * W + l * l + l + m
                mirror[t] = 2 * (n * W + l * l + l - m) + (m & 1)
    dot_begin = np.searchsorted(plan.dot_L, np.arange(P + 1), side="left").astype(np.int64)
    dot = np.zeros((plan.dot_count, 4), dtype=np.int64)
    for d in range(plan.dot_count):
        L = int(plan.dot_L[d])
        a, b = int(plan.dot_a[d]), int(plan.dot_b[d])
        dot[d] = (off[a] - pass_begin[L], off[b] - pass_begin[L], -1 if parity(b) else 1, 0)
    tabs = RecoupledSymTables(
        pass_count=P, max_pass_components=int(np.diff(pass_begin).max(initial=0)), row_width=row_width,
        dot_count=plan.dot_count, pass_begin=pass_begin.astype(np.int32), comp=comp.astype(np.int32),
        cg_index=np.asarray(cg_index, dtype=np.int32), cg_value=np.asarray(cg_value, dtype=np.float64),
        own=np.asarray(own, dtype=np.int32).reshape(-1, 2), bp_begin=bp_begin.astype(np.int32),
        bp_gi=np.asarray([e[0] for e in bp_flat], dtype=np.int32),
        bp_other=np.asarray([e[1] for e in bp_flat], dtype=np.int32),
        bp_value=np.asarray([e[2] for e in bp_flat], dtype=np.float64), mirror=mirror.astype(np.int32),
        dot_begin=dot_begin.astype(np.int32), dot=dot.astype(np.int32))
    tabs.validate()
    return tabs


def build_recoupled_plan(bundle: ACEBundle, seed: int = 20260) -> RecoupledPlan:
    """Recoupled plan of an L = 0 bundle (weights fitted once per pattern)."""
    if bundle.target_L != 0:
        raise ValueError("the recoupled plan covers scalar (L = 0) bundles")
    fits = {}
    for p, (rec, key) in enumerate(zip(bundle.patterns, bundle.pattern_keys)):
        fits[p] = _fit_pattern(rec, key, bundle.sym_tables, seed + 7919 * p)

    L1 = bundle.lmax + 1
    chan_id = lambda l, n: (n - 1) * L1 + l  # noqa: E731
    seg_index: Dict[Tuple[int, int, int, int], int] = {}
    segs: List[Tuple[int, int, int, int]] = []

    def segment(kind: int, L: int, a: int, b: int) -> int:
        k = (kind, L, a, b)
        if k not in seg_index:
            seg_index[k] = len(segs)
            segs.append(k)
        return seg_index[k]

    dots = []  # (L, seg_a, seg_b, word, [(feature, weight)])
    offsets = bundle.feature_offsets()
    for w, word in enumerate(bundle.words):
        chosen, W = fits[int(bundle.word_pattern_index[w])]
        ch = [chan_id(l, n) for l, n in word]

        def seg_of(s, L):
            if s[0] == "unit":
                return segment(SEG_UNIT, 0, -1, -1)
            if s[0] == "chan":
                return segment(SEG_CHANNEL, L, ch[s[1]], -1)
            return segment(SEG_PAIR, L, ch[s[1]], ch[s[2]])

        for d, (sa, sb, L) in enumerate(chosen):
            feats = [(int(offsets[w]) + c, complex(W[d, c])) for c in range(W.shape[1])
                     if abs(W[d, c]) > 1e-14 * max(float(np.abs(W).max()), 1e-300)]
            dots.append((L, seg_of(sa, L), seg_of(sb, L), w, feats))

    # segments ordered by L, then by how many contractions use them (longest first, so that
    # a warp's components walk lists of similar length), then first appearance; contractions
    # by L, then first segment
    uses = np.zeros(len(segs), dtype=np.int64)
    for _, a, b, _, _ in dots:
        uses[a] += 1
        uses[b] += 1
    order = sorted(range(len(segs)), key=lambda s: (segs[s][1], -int(uses[s]), s))
    rank = np.empty(len(segs), dtype=np.int64)
    rank[np.asarray(order, dtype=np.int64)] = np.arange(len(segs))
    kinds = np.asarray([segs[s][0] for s in order], dtype=np.int8)
    Ls = np.asarray([segs[s][1] for s in order], dtype=np.int32)
    seg_offset = np.concatenate([[0], np.cumsum(2 * Ls.astype(np.int64) + 1)])
    dots = [(L, int(rank[a]), int(rank[b]), w, f) for L, a, b, w, f in dots]
    dots.sort(key=lambda t: (t[0], t[1], t[2], t[3]))
    nz = np.concatenate([[0], np.cumsum([len(t[4]) for t in dots])]).astype(np.int64)
    weights = np.asarray([v for t in dots for _, v in t[4]], dtype=np.complex128)
    scale = max(float(np.abs(weights).max()), 1e-300) if weights.size else 1.0
    if weights.size and float(np.abs(weights.imag).max()) > 1e-12 * scale:
        raise ArithmeticError("recoupled feature weights are not real")
    return RecoupledPlan(
        nmax=bundle.nmax, lmax=bundle.lmax, feature_count=bundle.feature_count,
        seg_kind=kinds, seg_L=Ls,
        seg_a=np.asarray([segs[s][2] for s in order], dtype=np.int32),
        seg_b=np.asarray([segs[s][3] for s in order], dtype=np.int32),
        seg_offset=seg_offset,
        dot_a=np.asarray([t[1] for t in dots], dtype=np.int32),
        dot_b=np.asarray([t[2] for t in dots], dtype=np.int32),
        dot_L=np.asarray([t[0] for t in dots], dtype=np.int32),
        dot_word=np.asarray([t[3] for t in dots], dtype=np.int32),
        dot_feat_offset=nz,
        feat_index=np.asarray([f for t in dots for f, _ in t[4]], dtype=np.int64),
        feat_weight=np.ascontiguousarray(weights.real))


def ctypes_tables(arrays: Dict[str, "object"], tabs: RecoupledDeviceTables):
    """``y3b_recoupled_tables`` over tensors holding ``tabs``' arrays (``arrays[name]``)."""
    from . import _native as nat
    return nat.RecoupledTables(
        pass_count=tabs.pass_count, max_pass_components=tabs.max_pass_components, row_width=tabs.row_width,
        dot_count=tabs.dot_count, component_count=int(tabs.comp.shape[0]), cg_count=int(tabs.cg_value.shape[0]),
        own_count=int(tabs.own.shape[0]), bp_count=int(tabs.bp_gi.shape[0]),
        feature_count=tabs.feature_count, feat_count=int(tabs.feat_index.shape[0]),
        **{name: arrays[name].data_ptr() for name in _TABLE_ARRAYS})


_TABLE_ARRAYS = ("pass_begin", "comp", "cg_index", "cg_value", "own", "bp_begin", "bp_gi", "bp_other", "bp_value",
                 "dot_begin", "dot", "feat_index", "feat_weight")
_TILE_ARRAYS = ("tile_begin", "tile_row", "tile_col_begin", "col_comp", "bp_item_begin", "t_item_begin", "t_item",
                "bp_group_begin", "bp_group_off", "bp_pack", "unit_begin", "unit", "fix_begin", "fix")
_SYM_ARRAYS = ("pass_begin", "comp", "cg_index", "cg_value", "own", "bp_begin", "bp_gi", "bp_other", "bp_value",
               "mirror", "dot_begin", "dot")


def ctypes_sym_tables(arrays: Dict[str, "object"], tabs: RecoupledSymTables):
    """``y3b_recoupled_sym_tables`` over tensors holding ``tabs``' arrays (``arrays[name]``)."""
    from . import _native as nat
    return nat.RecoupledSymTables(
        pass_count=tabs.pass_count, max_pass_components=tabs.max_pass_components, row_width=tabs.row_width,
        dot_count=tabs.dot_count, component_count=int(tabs.comp.shape[0]), cg_count=int(tabs.cg_value.shape[0]),
        own_count=int(tabs.own.shape[0]), bp_count=int(tabs.bp_gi.shape[0]),
        **{name: arrays[name].data_ptr() for name in _SYM_ARRAYS})


class RecoupledEvaluator:
    """The recoupled passes on one GPU: the tables and the per-species contraction weights
    are uploaded once; each call takes ``A [n, nmax, (lmax+1)^2]`` complex128 (and the
    atoms' species), like ``ACEEvaluator``'s ``energy_grad`` / ``energy_from_density`` /
    ``features``.  ``atoms_per_cta`` atoms share one CTA's walk of the tables (each table
    entry loaded once for all of them), within the 224 KB of shared memory; a CTA has
    ``threads_per_cta`` (256 or 512) threads.  ``symmetric`` selects the passes over the
    ``M >= 0`` components (``RecoupledSymTables``), valid only for physical densities
    ``A[n, l, -m] = (-1)^m conj(A[n, l, m])`` such as ``ACEEvaluator.density`` gives.

    ``tile_rows`` (8; symmetric passes only) makes ``energy_grad`` form the
    components' adjoints from dense tiles of the contraction weights
    (``RecoupledTiles``, ``y3b_ace_recoupled_energy_grad_tiled``): a CTA then holds
    4 atoms, grouped in species order so that a CTA's atoms share one species' tile
    weights (``sort_species``)."""

    def __init__(self, bundle: ACEBundle, device, weights: np.ndarray = None, plan: "RecoupledPlan" = None,
                 atoms_per_cta: int = 1, threads_per_cta: int = 256, symmetric: bool = False,
                 tile_rows: int = 0, sort_species: bool = True):
        import torch
        if not 1 <= int(atoms_per_cta) <= 4:
            raise ValueError("atoms_per_cta must be in [1, 4]")
        if int(threads_per_cta) not in (256, 512):
            raise ValueError("threads_per_cta must be 256 or 512")
        if int(tile_rows) not in (0, 8):
            raise ValueError("tile_rows must be 0 (lists) or 8")
        if tile_rows and not symmetric:
            raise ValueError("the tiled adjoint is a form of the symmetric passes (symmetric=True)")
        self.device = torch.device(device)
        self.symmetric = bool(symmetric)
        self.tile_rows = int(tile_rows)
        self.sort_species = bool(sort_species)
        self.plan = plan if plan is not None else build_recoupled_plan(bundle)
        self.tables = self.plan.sym_device_tables() if self.symmetric else self.plan.device_tables()
        names = _SYM_ARRAYS if self.symmetric else _TABLE_ARRAYS
        self.arrays = {name: torch.as_tensor(np.ascontiguousarray(getattr(self.tables, name))).to(self.device)
                       for name in names}
        self.weights = None if weights is None else \
            torch.as_tensor(self.plan.energy_weights(weights)).to(self.device).contiguous()
        self._c = (ctypes_sym_tables if self.symmetric else ctypes_tables)(self.arrays, self.tables)
        self._c.atoms_per_cta = int(atoms_per_cta)
        self._c.threads_per_cta = int(threads_per_cta)
        self.tiles = None
        if self.tile_rows:
            from . import _native as nat
            self.tiles = self.plan.sym_tiles(self.tile_rows)
            self.tile_arrays = {name: torch.as_tensor(np.ascontiguousarray(getattr(self.tiles, name))).to(self.device)
                                for name in _TILE_ARRAYS}
            self.kval = None if weights is None else torch.as_tensor(
                self.tiles.tile_weights(self.plan.energy_weights(weights))).to(self.device).contiguous()
            self._t = nat.RecoupledTileTables(
                rows=self.tiles.rows, pass_count=self.tiles.pass_count, tile_count=self.tiles.tile_count,
                step_count=self.tiles.step_count, item_count=int(self.tiles.bp_item.shape[0]),
                group_count=int(self.tiles.bp_group_off.shape[0] - 1), pack_count=int(self.tiles.bp_pack.shape[0]),
                unit_count=int(self.tiles.unit.shape[0]), fix_count=int(self.tiles.fix.shape[0]),
                scratch_slots=int(self.tiles.scratch_slots),
                **{name: self.tile_arrays[name].data_ptr() for name in self.tile_arrays},
                kval=0 if self.kval is None else self.kval.data_ptr())

    def _rows(self, A):
        import torch
        from . import _native as nat
        A = A.to(self.device, torch.complex128).contiguous()
        if A.ndim < 1 or A.shape[1:].numel() != self.tables.row_width:
            raise ValueError(f"A rows must hold {self.tables.row_width} complex entries")
        nat.require_cuda(A, what="recoupled pass")
        return A

    def check_symmetry(self, A, tol: float = 1e-12) -> None:
        """Raise ``ValueError`` unless ``A[n, l, -m] = (-1)^m conj(A[n, l, m])`` holds to ``tol``
        (relative to ``max |A|``): the condition of the symmetric passes."""
        import torch
        W = (self.plan.lmax + 1) ** 2
        neg, pos, sign = [], [], []
        for l in range(self.plan.lmax + 1):
            for m in range(1, l + 1):
                neg.append(l * l + l - m)
                pos.append(l * l + l + m)
                sign.append(-1.0 if m & 1 else 1.0)
        rows = A.reshape(A.shape[0], -1, W)
        scale = float(rows.abs().max()) if rows.numel() else 0.0
        dev = 0.0
        if neg:
            idx_n = torch.as_tensor(neg, device=rows.device)
            idx_p = torch.as_tensor(pos, device=rows.device)
            sg = torch.as_tensor(sign, dtype=torch.float64, device=rows.device)
            dev = float((rows[..., idx_n] - sg * rows[..., idx_p].conj()).abs().max())
        zero = torch.as_tensor([l * l + l for l in range(self.plan.lmax + 1)], device=rows.device)
        dev = max(dev, float(rows[..., zero].imag.abs().max()) if rows.numel() else 0.0)
        if dev > tol * max(scale, 1e-300):
            raise ValueError(f"A lacks the physical symmetry A[l,-m] = (-1)^m conj(A[l,m]) (deviation {dev:.3e}); "
                             "use the general passes (symmetric=False)")

    def _species(self, species, n):
        import torch
        if self.weights is None:
            raise ValueError("weights are required for the energy")
        sp = species.to(self.device, torch.int32).contiguous()
        if sp.shape != (n,):
            raise ValueError("one species per atom is required")
        return sp

    def energy_grad(self, A, species, status=None, check_symmetry: bool = True):
        """(per-atom energies, ``G = dE/dA``).  With ``symmetric`` passes the density's
        symmetry is checked first (``check_symmetry``, one pass over A and a host sync)
        unless ``check_symmetry=False``; a caller whose A comes from a physical density
        kernel (real radial functions and prefactors) may skip it."""
        import ctypes

        import torch
        from . import _native as nat
        A = self._rows(A)
        if self.symmetric and check_symmetry:
            self.check_symmetry(A)
        n = A.shape[0]
        sp = self._species(species, n)
        e = torch.empty(n, dtype=torch.float64, device=self.device)
        G = torch.empty_like(A)
        if self.tiles is not None:
            order = torch.sort(sp, stable=True).indices.to(torch.int32) if self.sort_species else None
            nat.check(nat.lib().y3b_ace_recoupled_energy_grad_tiled(
                ctypes.byref(self._c), ctypes.byref(self._t), A.data_ptr(), n, nat.ptr(order), sp.data_ptr(),
                self.kval.shape[0], e.data_ptr(), G.data_ptr(), nat.ptr(status), nat.stream_of(self.device)),
                "y3b_ace_recoupled_energy_grad_tiled")
            return e, G
        name = "y3b_ace_recoupled_energy_grad_symmetric" if self.symmetric else "y3b_ace_recoupled_energy_grad"
        nat.check(getattr(nat.lib(), name)(
            ctypes.byref(self._c), A.data_ptr(), n, sp.data_ptr(), self.weights.data_ptr(), self.weights.shape[0],
            e.data_ptr(), G.data_ptr(), nat.ptr(status), nat.stream_of(self.device)), name)
        return e, G

    def energy(self, A, species, status=None, check_symmetry: bool = True):
        """Per-atom energies (the symmetry check as in ``energy_grad``)."""
        import ctypes

        import torch
        from . import _native as nat
        A = self._rows(A)
        if self.symmetric and check_symmetry:
            self.check_symmetry(A)
        n = A.shape[0]
        sp = self._species(species, n)
        e = torch.empty(n, dtype=torch.float64, device=self.device)
        name = "y3b_ace_recoupled_energy_symmetric" if self.symmetric else "y3b_ace_recoupled_energy"
        nat.check(getattr(nat.lib(), name)(
            ctypes.byref(self._c), A.data_ptr(), n, sp.data_ptr(), self.weights.data_ptr(), self.weights.shape[0],
            e.data_ptr(), nat.ptr(status), nat.stream_of(self.device)), name)
        return e

    def features(self, A, status=None, out=None):
        """Features ``[n, feature_count]`` complex128 in the bundle's order (general passes only),
        into ``out`` when given (contiguous, complex128, that shape)."""
        import ctypes

        import torch
        from . import _native as nat
        if self.symmetric:
            raise ValueError("features need the general passes (symmetric=False)")
        A = self._rows(A)
        n = A.shape[0]
        shape = (n, self.tables.feature_count)
        if out is not None and (tuple(out.shape) != shape or out.dtype != torch.complex128 or
                                not out.is_contiguous() or out.device != self.device):
            raise ValueError(f"out must be a contiguous complex128 tensor of shape {shape} on {self.device}")
        F = out if out is not None else torch.empty(shape, dtype=torch.complex128, device=self.device)
        nat.check(nat.lib().y3b_ace_recoupled_features(
            ctypes.byref(self._c), A.data_ptr(), n, F.data_ptr(), nat.ptr(status), nat.stream_of(self.device)),
            "ace_recoupled_features")
        return F
