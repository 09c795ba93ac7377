"""Host-side packing checked on CPU: a numpy emulation of the pool and bundle
kernels over the packed tables must reproduce the oracle's features."""

import os

import numpy as np
import pytest

from oracle import oracle
from ye3t_b200.packing import pack_bundle
from ye3t_b200.schedules import ACEBundle

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bundle(stem):
    return ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", stem + ".npz"))


def emulate_features(pb, A):
    """numpy walk of the packed phases and items, in the kernel's order."""
    from ye3t_b200.packing import ITEM_INTS
    a = {k: v.cpu().numpy() for k, v in pb.arrays.items()}
    N, nmax, W = A.shape
    na = nmax * W
    so = a["sym_outputs"].shape[0]
    sm = np.zeros((na + 2 * so, N), dtype=np.complex128)
    sm[:na] = A.reshape(N, na).T
    coef = a["item_coef"]
    out = np.zeros((N, pb.feature_count), dtype=np.complex128)

    def fill(slot, ch):
        for o, (l2, tb, te, _) in enumerate(a["sym_outputs"]):
            x = sm[ch * W + l2: ch * W + l2 + 16]
            acc = np.zeros(N, dtype=np.complex128)
            for q in range(tb, te):
                f = int(np.uint32(a["sym_term_factors"][q]))
                m = np.full(N, a["sym_term_coeff"][q], dtype=np.complex128)
                for kk in range(4):
                    ci = (f >> (8 * kk)) & 255
                    if ci == 255:
                        break
                    m = m * x[ci]
                acc += m
            sm[na + slot * so + o] = acc

    cur = (None, None)
    for c0, c1, ib, ie in a["phases"]:
        if c0 != cur[0]:
            fill(0, c0)
        if c1 >= 0 and c1 != cur[1]:
            fill(1, c1)
        cur = (c0, c1)
        for row in a["items"][ib:ie]:
            sel, d0, d1, dl, K, co, f0, f1 = (int(v) for v in row[:8])
            bases = [int(v) for v in row[8:12]]
            nc = sel % 2 + 1
            B = (sel // 2) // 7 + 1
            ds = 2 * ((sel // 2) % 7) + 1
            acc = [np.zeros(N, dtype=np.complex128) for _ in range(nc)]
            rw = 2 * ds if nc == 2 else (ds + 1) & ~1
            if B == 1:
                for k in range(nc):
                    acc[k] += coef[co + k] * sm[bases[0] + K]
            else:
                prefixes = [((), 0, np.ones(N, dtype=np.complex128))]
                if B == 3:
                    prefixes = [((i0,), i0 * rw, sm[bases[0] + i0]) for i0 in range(d0)]
                elif B == 4:
                    prefixes = [((i0, i1), (i0 * d1 + i1) * rw, sm[bases[0] + i0] * sm[bases[1] + i1])
                                for i0 in range(d0) for i1 in range(d1)]
                bs, bl = bases[B - 2], bases[B - 1]
                for pre, crow, x in prefixes:
                    S = sum(pre)
                    t = [np.zeros(N, dtype=np.complex128) for _ in range(nc)]
                    for j in range(ds):
                        li = K - S - j
                        if 0 <= li < dl:
                            q = sm[bs + j] * sm[bl + li]
                            for k in range(nc):
                                t[k] += coef[co + crow + j * nc + k] * q
                    for k in range(nc):
                        acc[k] += x * t[k]
            out[:, f0] = acc[0]
            if f1 >= 0:
                out[:, f1] = acc[1]
    assert a["items"].shape[1] == ITEM_INTS
    return out


def test_packing_layout_and_counts():
    b = _bundle("ace_n8_l3_nu4_L0")
    pb = pack_bundle(b, "cpu")
    assert pb.feature_count == 41168
    assert pb.term_count_per_atom == 1332116
    assert pb.term_block_count_per_atom == 5163248
    assert pb.pool_size == 8 * 16 + 2 * 89  # shared-memory entries per atom
    assert pb.arrays["phases"].shape[0] == 28
    assert pb.max_blocks == 4
    flops = pb.flops_per_atom()
    assert 0 < flops["items"] < flops["terms"]


@pytest.mark.parametrize("stem", ["ace_n8_l3_nu3_L0"])
def test_packed_tables_reproduce_oracle_features(golden, stem):
    g = golden("ace_small")
    A = g["A"][:6]
    b = _bundle(stem)
    pb = pack_bundle(b, "cpu")
    got = emulate_features(pb, A)
    ref = oracle.bundle_features(b, A)
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12 * np.abs(ref).max())
    np.testing.assert_allclose(got, g["B3"][:6], rtol=1e-11, atol=1e-12 * np.abs(ref).max())


@pytest.mark.parametrize("stem", ["ace_n8_l3_nu4_L0", "ace_diag_l3_nu3_L2"])
def test_adjoint_groups_cover_items_once(stem):
    """Every item sits in exactly one adjoint pair of its class; class 0 fills
    whole rounds of its round robin per phase, the three-block class splits
    each phase into equal per-warp runs; the four-block run
    classes hold no phases, split into equal per-warp runs whose costs differ
    by at most one item per shape."""
    from ye3t_b200.packing import GRAD_CLASSES, GRAD_RUN_CLASSES, GRAD_RUN_WARPS, grad_class, item_grad_flops_per_atom
    b = _bundle(stem)
    pb = pack_bundle(b, "cpu")
    items = pb.arrays["items"].numpy()
    groups = pb.arrays["groups"].numpy()
    P = pb.arrays["phases"].shape[0]
    off = pb.arrays["group_offsets"].numpy().reshape(GRAD_CLASSES, P + 1)
    na = b.nmax * (b.lmax + 1) ** 2
    seen = np.zeros(items.shape[0], dtype=np.int64)
    for cls in range(GRAD_CLASSES):
        assert off[cls, 0] == (off[cls - 1, -1] if cls else 0)
        assert np.all(np.diff(off[cls]) >= 0)
        rng = groups[off[cls, 0]:off[cls, -1]]
        real = rng[rng[:, 0] >= 0]
        if cls not in GRAD_RUN_CLASSES:
            # per phase: equal runs (class 1) or whole rounds of the round robin (class 0)
            assert np.all(np.diff(off[cls]) % GRAD_RUN_WARPS == 0)
        for x, y in real:
            for i in (x, y):
                if i >= 0:
                    seen[i] += 1
                    assert grad_class(items[i], na) == cls
            if y >= 0:
                assert np.array_equal(items[x, :5], items[y, :5])  # one shape per pair
        if cls in GRAD_RUN_CLASSES and len(rng):
            assert np.all(off[cls, 1:] == off[cls, -1])
            assert len(rng) % GRAD_RUN_WARPS == 0
            per = len(rng) // GRAD_RUN_WARPS
            costs = [item_grad_flops_per_atom(items[[x for x, _ in rng[w * per:(w + 1) * per] if x >= 0]])
                     for w in range(GRAD_RUN_WARPS)]
            worst = max(item_grad_flops_per_atom(items[x:x + 1]) for x, _ in real)
            shapes = len({tuple(items[x, :5]) for x, _ in real})
            assert max(costs) - min(costs) <= shapes * worst
    assert np.all(seen == 1)


def test_schedule_adjoint_slot_table(golden):
    """The transposed (slot -> term, component) table of the schedule adjoint, against a
    brute-force listing, for every schedule of the reference fixture."""
    import json as _json
    from ye3t_b200.couplings import packed_schedule_tables
    from ye3t_b200.schedules import ScheduleRecord
    g = golden("schedules")
    i = 0
    while f"s{i}_off" in g:
        p = f"s{i}_"
        specs = _json.loads(bytes(g[p + "specs"]).decode())
        rec = ScheduleRecord(rank=0, block_count=int(g[p + "bm"].shape[1]), L_R=0, n_tuple=(), l_tuple=(),
                             block_specs=tuple(tuple(tuple(s) for s in label) for label in specs),
                             component_offsets=g[p + "off"], component_label_index=g[p + "cli"],
                             component_M_R=np.zeros_like(g[p + "cli"]), block_m_tuples=g[p + "bm"],
                             coeffs=g[p + "co"])
        pk = packed_schedule_tables(rec, "cpu")
        mdim = rec.max_block_m_dim + 1  # wider than needed, as a caller's padded array may be
        off, terms, comps = (x.numpy() for x in pk.slot_table(mdim, "cpu"))
        midx = rec.block_m_indices()
        expect = {}
        for c in range(rec.component_count):
            for t in range(rec.component_offsets[c], rec.component_offsets[c + 1]):
                for j in range(rec.block_count):
                    s = (rec.component_label_index[c] * rec.block_count + j) * mdim + midx[t, j]
                    expect.setdefault(int(s), []).append((t, c))
        assert off.shape[0] == rec.basis_count * rec.block_count * mdim + 1
        for s in range(off.shape[0] - 1):
            got = list(zip(terms[off[s]:off[s + 1]].tolist(), comps[off[s]:off[s + 1]].tolist()))
            assert got == expect.get(s, []), (i, s)
        i += 1


@pytest.mark.parametrize("stem", sorted(f[:-4] for f in os.listdir(os.path.join(REPO, "ye3t_b200", "bundles"))
                                        if f.endswith(".npz")))
def test_adjoint_classes_respect_kernel_bounds(stem):
    """Every item of every shipped bundle sits in a class whose kernel path holds it: the run
    classes (per-lane staging windows of 7 entries, A entries only) and class 1 (last block
    staged in 14 entries, register block 5 or 7); everything else goes to class 0, whose general
    path has no staging bound."""
    from ye3t_b200.packing import GRAD_RUN_BLOCK, GRAD_STAGE, grad_class
    b = _bundle(stem)
    items = pack_bundle(b, "cpu").arrays["items"].numpy()
    na = b.nmax * (b.lmax + 1) ** 2
    for row in items:
        sel, d0, d1, dl = int(row[0]), int(row[1]), int(row[2]), int(row[3])
        B, ds = (sel // 2) // 7 + 1, 2 * ((sel // 2) % 7) + 1
        cls = grad_class(row, na)
        if cls in (2, 3):
            assert B == 4 and max(d0, d1, dl) <= GRAD_RUN_BLOCK
            assert ds in ((3, 5) if cls == 2 else (7,))
            assert all(int(row[8 + k]) + dim <= na for k, dim in enumerate((d0, d1, ds, dl)))
        elif cls == 1:
            assert B == 3 and ds in (5, 7) and dl <= GRAD_STAGE
