"""Host records for compiled ACE factorized schedules and multi-word bundles.

A :class:`ScheduleRecord` is a plain-array copy of the reference's
``FactorizedCoefficientSchedule`` (``ye3t/core/couplings.py:164-257``): the same
fields with the same meaning, so a schedule produced by
``ye3t.couplings.compile_ace_factorized_schedules_by_L``
(``ye3t/couplings/__init__.py:2617-2706``) converts without change.  Records are
also what the runtime packs into device tables.

An :class:`ACEBundle` is the unit the fused kernels consume: every word of a
descriptor word set, each bound to one compiled *pattern* schedule.  A word is
a multiset of radial/angular channels ``(n, l)``; its pattern replaces the
radial indices by their ranks (``n -> 1..k`` in increasing order), which keeps
the reference's own canonical block order (blocks sorted by ``(l, n)``), so
one compiled schedule serves every word with the same equality structure.
The bundle is saved as ``.npz`` (arrays plus one JSON header) and keyed by the
``convention_hash`` of each pattern compile plus a table hash of the packed
arrays.
"""

from __future__ import annotations

import hashlib
import itertools
import json
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

__all__ = [
    "ScheduleRecord",
    "SymPowerTable",
    "ACEBundle",
    "enumerate_ace_words",
    "word_pattern",
    "schedule_table_hash",
]

_BLOCK_SPEC_KEYS = ("kind", "n", "l", "k_b", "Lambda", "multiplicity_index")


def _spec_tuple(spec) -> Tuple:
    return (str(spec["kind"]), int(spec["n"]), int(spec["l"]), int(spec.get("k_b", 1)),
            int(spec.get("Lambda", spec["l"])), int(spec.get("multiplicity_index", 0)))


def _spec_dict(t) -> Dict:
    return dict(zip(_BLOCK_SPEC_KEYS, t))


@dataclass(frozen=True, eq=False)
class ScheduleRecord:
    """Plain-array form of one ``FactorizedCoefficientSchedule``.

    Field meanings follow ``ye3t/core/couplings.py:164-257``.  ``block_specs``
    is stored as a tuple (per basis label) of tuples (per block) of
    ``(kind, n, l, k_b, Lambda, multiplicity_index)``.
    """

    rank: int
    block_count: int
    L_R: int
    n_tuple: Tuple[int, ...]
    l_tuple: Tuple[int, ...]
    block_specs: Tuple[Tuple[Tuple, ...], ...]
    component_offsets: np.ndarray  # int64 [C+1]
    component_label_index: np.ndarray  # int64 [C]
    component_M_R: np.ndarray  # int64 [C]
    block_m_tuples: np.ndarray  # int16 [T, B]
    coeffs: np.ndarray  # complex128 [T]
    convention_hash: str = ""

    @property
    def basis_count(self) -> int:
        return len(self.block_specs)

    @property
    def component_count(self) -> int:
        return int(self.component_label_index.shape[0])

    @property
    def term_count(self) -> int:
        return int(self.coeffs.shape[0])

    def block_L_by_label(self) -> np.ndarray:
        """Block angular momentum per (label, block); ``couplings.py:203-214``."""
        if not self.block_specs:
            return np.zeros((0, self.block_count), dtype=np.int64)
        return np.asarray([[s[4] if s[0] == "sym" else s[2] for s in label]
                           for label in self.block_specs], dtype=np.int64)

    @property
    def max_block_m_dim(self) -> int:
        bl = self.block_L_by_label()
        return int(2 * bl.max() + 1) if bl.size else 0

    def block_m_indices(self) -> np.ndarray:
        """``m + L_block`` per term and block; ``couplings.py:216-240`` (to_torch)."""
        if self.term_count == 0 or self.block_count == 0:
            return np.zeros((0, self.block_count), dtype=np.int64)
        counts = np.diff(self.component_offsets)
        term_comp = np.repeat(np.arange(self.component_count), counts)
        term_label = self.component_label_index[term_comp]
        return self.block_m_tuples.astype(np.int64) + self.block_L_by_label()[term_label]

    def real_coeffs(self, tol: float = 1e-12) -> Optional[np.ndarray]:
        """Real part when every imaginary part is within ``tol`` (``couplings.py:508-516``)."""
        c = np.asarray(self.coeffs)
        if np.iscomplexobj(c):
            if c.size and float(np.max(np.abs(c.imag))) > tol:
                return None
            return np.ascontiguousarray(c.real, dtype=np.float64)
        return np.ascontiguousarray(c, dtype=np.float64)

    def block_specs_dicts(self):
        return tuple(tuple(_spec_dict(s) for s in label) for label in self.block_specs)

    @classmethod
    def from_schedule(cls, schedule, convention_hash: str = "") -> "ScheduleRecord":
        """Copy a reference ``FactorizedCoefficientSchedule`` (duck-typed)."""
        return cls(
            rank=int(schedule.rank),
            block_count=int(schedule.block_count),
            L_R=int(schedule.L_R),
            n_tuple=tuple(int(v) for v in schedule.n_tuple),
            l_tuple=tuple(int(v) for v in schedule.l_tuple),
            block_specs=tuple(tuple(_spec_tuple(s) for s in label) for label in schedule.block_specs),
            component_offsets=np.asarray(schedule.component_offsets, dtype=np.int64).copy(),
            component_label_index=np.asarray(schedule.component_label_index, dtype=np.int64).copy(),
            component_M_R=np.asarray(schedule.component_M_R, dtype=np.int64).copy(),
            block_m_tuples=np.asarray(schedule.block_m_tuples, dtype=np.int16).reshape(
                -1, int(schedule.block_count)).copy(),
            coeffs=np.asarray(schedule.coeffs).astype(np.complex128).copy(),
            convention_hash=str(convention_hash),
        )

    def rebind(self, n_map: Dict[int, int], convention_hash: Optional[str] = None) -> "ScheduleRecord":
        """Same tables with radial indices renamed through ``n_map``."""
        specs = tuple(tuple((s[0], int(n_map[s[1]]), s[2], s[3], s[4], s[5]) for s in label)
                      for label in self.block_specs)
        return ScheduleRecord(
            rank=self.rank, block_count=self.block_count, L_R=self.L_R,
            n_tuple=tuple(int(n_map[n]) for n in self.n_tuple), l_tuple=self.l_tuple,
            block_specs=specs, component_offsets=self.component_offsets,
            component_label_index=self.component_label_index, component_M_R=self.component_M_R,
            block_m_tuples=self.block_m_tuples, coeffs=self.coeffs,
            convention_hash=self.convention_hash if convention_hash is None else convention_hash)


def schedule_table_hash(record: ScheduleRecord) -> str:
    """sha256 over the integer tables and coefficient bytes of one record."""
    h = hashlib.sha256()
    for arr in (record.component_offsets, record.component_label_index, record.component_M_R,
                record.block_m_tuples, record.coeffs):
        a = np.ascontiguousarray(arr)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    h.update(json.dumps(record.block_specs).encode())
    return h.hexdigest()[:16]


@dataclass(frozen=True, eq=False)
class SymPowerTable:
    """Grouped symmetric-power table ``Sym^k(V_l) -> V_Lambda`` (complex-magnetic basis).

    Fields follow the grouped lowering of a compiler plan in
    ``ye3t/runtime/symmetric_power.py:740-868``: per term an exponent row over
    the ``2l+1`` input components, the output component it feeds
    (``output_offsets`` groups terms by output), and its coefficient.
    """

    l: int
    k: int
    Lambda: int
    multiplicity_index: int
    monomial_counts: np.ndarray  # int64 [T, 2l+1]
    output_offsets: np.ndarray  # int64 [2 Lambda + 2]
    output_index: np.ndarray  # int64 [T]
    monomial_value: np.ndarray  # complex128 [T]
    convention_hash: str = ""

    @property
    def key(self) -> Tuple[int, int, int, int]:
        return (self.l, self.k, self.Lambda, self.multiplicity_index)

    @property
    def term_count(self) -> int:
        return int(self.monomial_value.shape[0])


def enumerate_ace_words(nmax: int, lmax: int, numax: int, *, parity: str = "even"):
    """All multisets of channels ``(l, n)`` of size ``1..numax``.

    Channels are ``n in 1..nmax``, ``l in 0..lmax``; with ``parity="even"``
    only words with even ``sum(l)`` are kept (the parity-invariant scalar
    sector).  Words are tuples of ``(l, n)`` sorted lexicographically, which is
    the block order the reference compiler uses.  This word-set rule is this
    framework's (the reference leaves descriptor word sets to applications).
    """
    pairs = [(l, n) for l in range(lmax + 1) for n in range(1, nmax + 1)]
    out = []
    for k in range(1, numax + 1):
        for combo in itertools.combinations_with_replacement(pairs, k):
            if parity == "even" and sum(l for l, _ in combo) % 2:
                continue
            out.append(tuple(combo))
    return out


def word_pattern(word) -> Tuple[Tuple[Tuple[int, int], ...], Dict[int, int]]:
    """Rank-relabelled pattern of a word and the map ``pattern n -> word n``."""
    ns = sorted({n for _, n in word})
    rank = {n: i + 1 for i, n in enumerate(ns)}
    return tuple((l, rank[n]) for l, n in word), {r: n for n, r in rank.items()}


@dataclass(eq=False)
class ACEBundle:
    """Every word of an ACE word set bound to its compiled pattern schedule."""

    nmax: int
    lmax: int
    target_L: int
    words: List[Tuple[Tuple[int, int], ...]]
    word_pattern_index: np.ndarray  # int32 [W]
    word_n_map: np.ndarray  # int32 [W, 5]: pattern rank r (1..4) -> word n (0 unused)
    patterns: List[ScheduleRecord]  # with pattern ranks as n
    pattern_keys: List[Tuple[Tuple[int, int], ...]]
    sym_tables: Dict[Tuple[int, int, int, int], SymPowerTable] = field(default_factory=dict)
    meta: Dict = field(default_factory=dict)

    @property
    def word_count(self) -> int:
        return len(self.words)

    def word_schedule(self, w: int) -> ScheduleRecord:
        """The pattern schedule of word ``w`` with its own radial indices."""
        p = self.patterns[int(self.word_pattern_index[w])]
        n_map = {r: int(self.word_n_map[w, r]) for r in range(1, self.word_n_map.shape[1])
                 if self.word_n_map[w, r] > 0}
        return p.rebind(n_map)

    def feature_offsets(self) -> np.ndarray:
        """Start of each word's components in the flattened feature vector."""
        comps = np.asarray([self.patterns[int(p)].component_count for p in self.word_pattern_index],
                           dtype=np.int64)
        return np.concatenate([[0], np.cumsum(comps)])

    @property
    def feature_count(self) -> int:
        return int(self.feature_offsets()[-1])

    def table_hash(self) -> str:
        h = hashlib.sha256()
        for p in self.patterns:
            h.update(schedule_table_hash(p).encode())
        h.update(np.ascontiguousarray(self.word_pattern_index).tobytes())
        h.update(np.ascontiguousarray(self.word_n_map).tobytes())
        for key in sorted(self.sym_tables):
            t = self.sym_tables[key]
            for a in (t.monomial_counts, t.output_offsets, t.output_index, t.monomial_value):
                h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()[:16]

    # -- serialisation -----------------------------------------------------
    def save(self, path: str) -> None:
        arrays = {
            "word_pattern_index": self.word_pattern_index.astype(np.int32),
            "word_n_map": self.word_n_map.astype(np.int32),
            "words": np.asarray([[v for pair in w for v in pair] + [-1] * (2 * 4 - 2 * len(w))
                                 for w in self.words], dtype=np.int16),
        }
        pats = []
        for i, p in enumerate(self.patterns):
            arrays[f"p{i}_off"] = p.component_offsets
            arrays[f"p{i}_cli"] = p.component_label_index
            arrays[f"p{i}_cmr"] = p.component_M_R
            arrays[f"p{i}_bm"] = p.block_m_tuples
            arrays[f"p{i}_co"] = p.coeffs
            pats.append({"rank": p.rank, "block_count": p.block_count, "L_R": p.L_R,
                         "n_tuple": list(p.n_tuple), "l_tuple": list(p.l_tuple),
                         "block_specs": [[list(s) for s in label] for label in p.block_specs],
                         "convention_hash": p.convention_hash,
                         "pattern": [list(x) for x in self.pattern_keys[i]]})
        syms = []
        for j, key in enumerate(sorted(self.sym_tables)):
            t = self.sym_tables[key]
            arrays[f"s{j}_cnt"] = t.monomial_counts
            arrays[f"s{j}_off"] = t.output_offsets
            arrays[f"s{j}_idx"] = t.output_index
            arrays[f"s{j}_val"] = t.monomial_value
            syms.append({"key": list(key), "convention_hash": t.convention_hash})
        header = {"schema": "ye3t_b200_ace_bundle_v1", "nmax": self.nmax, "lmax": self.lmax,
                  "target_L": self.target_L, "patterns": pats, "sym_tables": syms,
                  "meta": self.meta, "table_hash": self.table_hash()}
        arrays["header"] = np.frombuffer(json.dumps(header).encode(), dtype=np.uint8)
        np.savez_compressed(path, **arrays)

    @classmethod
    def load(cls, path: str) -> "ACEBundle":
        z = np.load(path, allow_pickle=False)
        header = json.loads(bytes(z["header"]).decode())
        if header.get("schema") != "ye3t_b200_ace_bundle_v1":
            raise ValueError(f"{path}: not an ACE bundle (schema {header.get('schema')!r})")
        patterns, keys = [], []
        for i, ph in enumerate(header["patterns"]):
            patterns.append(ScheduleRecord(
                rank=ph["rank"], block_count=ph["block_count"], L_R=ph["L_R"],
                n_tuple=tuple(ph["n_tuple"]), l_tuple=tuple(ph["l_tuple"]),
                block_specs=tuple(tuple(tuple([s[0]] + [int(v) for v in s[1:]]) for s in label)
                                  for label in ph["block_specs"]),
                component_offsets=z[f"p{i}_off"], component_label_index=z[f"p{i}_cli"],
                component_M_R=z[f"p{i}_cmr"], block_m_tuples=z[f"p{i}_bm"], coeffs=z[f"p{i}_co"],
                convention_hash=ph["convention_hash"]))
            keys.append(tuple(tuple(x) for x in ph["pattern"]))
        syms = {}
        for j, sh in enumerate(header["sym_tables"]):
            key = tuple(int(v) for v in sh["key"])
            syms[key] = SymPowerTable(*key, monomial_counts=z[f"s{j}_cnt"],
                                      output_offsets=z[f"s{j}_off"], output_index=z[f"s{j}_idx"],
                                      monomial_value=z[f"s{j}_val"],
                                      convention_hash=sh["convention_hash"])
        raw = z["words"]
        words = []
        for row in raw:
            vals = [int(v) for v in row if v >= 0]
            words.append(tuple((vals[2 * i], vals[2 * i + 1]) for i in range(len(vals) // 2)))
        b = cls(nmax=header["nmax"], lmax=header["lmax"], target_L=header["target_L"],
                words=words, word_pattern_index=z["word_pattern_index"],
                word_n_map=z["word_n_map"], patterns=patterns, pattern_keys=keys,
                sym_tables=syms, meta=header.get("meta", {}))
        if header.get("table_hash") and b.table_hash() != header["table_hash"]:
            raise ValueError(f"{path}: table hash mismatch (file corrupted or edited)")
        return b

    # -- construction ------------------------------------------------------
    @classmethod
    def from_words(cls, words: Sequence, nmax: int, lmax: int, target_L: int, compile_pattern,
                   sym_table_for, meta: Optional[Dict] = None) -> "ACEBundle":
        """Build a bundle with caller-supplied compilers.

        ``compile_pattern(content, input_Ls) -> (schedule, convention_hash)``
        returns the schedule for ``target_L`` (or ``None`` when that ``L`` has
        no basis); ``sym_table_for(l, k, Lambda, mu) -> SymPowerTable``.  Words
        whose pattern has no basis at ``target_L`` are dropped.
        """
        patterns, keys, index = [], [], {}
        kept, wp, wn = [], [], []
        syms = {}
        for w in words:
            pat, rmap = word_pattern(w)
            if pat not in index:
                sched, chash = compile_pattern(tuple(n for _, n in pat), tuple(l for l, _ in pat))
                index[pat] = None if sched is None else len(patterns)
                if sched is not None:
                    rec = ScheduleRecord.from_schedule(sched, chash)
                    patterns.append(rec)
                    keys.append(pat)
                    for label in rec.block_specs:
                        for s in label:
                            if s[0] == "sym":
                                key = (s[2], s[3], s[4], s[5])
                                if key not in syms:
                                    syms[key] = sym_table_for(*key)
            pi = index[pat]
            if pi is None:
                continue
            kept.append(tuple(w))
            wp.append(pi)
            row = [0] * 5
            for r, n in rmap.items():
                row[r] = n
            wn.append(row)
        return cls(nmax=nmax, lmax=lmax, target_L=target_L, words=kept,
                   word_pattern_index=np.asarray(wp, dtype=np.int32),
                   word_n_map=np.asarray(wn, dtype=np.int32).reshape(-1, 5),
                   patterns=patterns, pattern_keys=keys, sym_tables=syms, meta=dict(meta or {}))
