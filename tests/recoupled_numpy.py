"""Numpy restatement of the recoupled evaluation (test helper).

Per atom: segment components, contractions, features; and the holomorphic
``dE/dA`` of ``e = Re(sum_d k[z, d] T_d)`` by the chain rule through the
contractions and the pair couplings.  The order of operations is the one a
device kernel over ``RecoupledPlan`` follows (segments by L, contractions by
L then first segment), so a kernel can be checked against it term by term."""

import numpy as np

from ye3t_b200.recoupling import SEG_CHANNEL, SEG_PAIR, SEG_UNIT, cg_table


def _chan(plan, A, c):
    l, n = plan.channel(int(c))
    return A[:, n - 1, l * l:(l + 1) * (l + 1)]


def segments(plan, A):
    """``I [N, component_count]``."""
    N = A.shape[0]
    I = np.zeros((N, plan.component_count), dtype=np.complex128)
    for s in range(plan.segment_count):
        o0, o1 = int(plan.seg_offset[s]), int(plan.seg_offset[s + 1])
        kind, L = int(plan.seg_kind[s]), int(plan.seg_L[s])
        if kind == SEG_UNIT:
            I[:, o0] = 1.0
        elif kind == SEG_CHANNEL:
            I[:, o0:o1] = _chan(plan, A, plan.seg_a[s])
        else:
            a, b = int(plan.seg_a[s]), int(plan.seg_b[s])
            la, lb = plan.channel(a)[0], plan.channel(b)[0]
            idx, val = cg_table(la, lb, L)
            xa, xb = _chan(plan, A, a), _chan(plan, A, b)
            np.add.at(I, (slice(None), o0 + idx[:, 2]), val * xa[:, idx[:, 0]] * xb[:, idx[:, 1]])
    return I


def contractions(plan, I):
    """``T [N, dot_count]``."""
    T = np.zeros((I.shape[0], plan.dot_count), dtype=np.complex128)
    for L in np.unique(plan.dot_L):
        sel = np.nonzero(plan.dot_L == L)[0]
        M = np.arange(-L, L + 1)
        oa = plan.seg_offset[plan.dot_a[sel]][:, None] + (M + L)[None, :]
        ob = plan.seg_offset[plan.dot_b[sel]][:, None] + (L - M)[None, :]
        T[:, sel] = ((-1.0) ** M * I[:, oa] * I[:, ob]).sum(axis=2)
    return T


def features(plan, A):
    T = contractions(plan, segments(plan, A))
    dot_of = np.repeat(np.arange(plan.dot_count), np.diff(plan.dot_feat_offset))
    F = np.zeros((A.shape[0], plan.feature_count), dtype=np.complex128)
    np.add.at(F, (slice(None), plan.feat_index), T[:, dot_of] * plan.feat_weight[None, :])
    return F


def energy_grad(plan, A, species, weights):
    """Per-atom energies and the holomorphic ``G = dE/dA``."""
    k = plan.energy_weights(weights)[np.asarray(species)]  # [N, D]
    I = segments(plan, A)
    T = contractions(plan, I)
    e = (k * T).sum(axis=1).real
    gI = np.zeros_like(I)
    for L in np.unique(plan.dot_L):
        sel = np.nonzero(plan.dot_L == L)[0]
        M = np.arange(-L, L + 1)
        oa = plan.seg_offset[plan.dot_a[sel]][:, None] + (M + L)[None, :]
        ob = plan.seg_offset[plan.dot_b[sel]][:, None] + (L - M)[None, :]
        sgn = (-1.0) ** M
        kd = k[:, sel][:, :, None]
        np.add.at(gI, (slice(None), oa), kd * sgn * I[:, ob])
        np.add.at(gI, (slice(None), ob), kd * sgn * I[:, oa])
    G = np.zeros_like(A)
    for s in range(plan.segment_count):
        o0, o1 = int(plan.seg_offset[s]), int(plan.seg_offset[s + 1])
        kind, L = int(plan.seg_kind[s]), int(plan.seg_L[s])
        if kind == SEG_CHANNEL:
            l, n = plan.channel(int(plan.seg_a[s]))
            G[:, n - 1, l * l:(l + 1) * (l + 1)] += gI[:, o0:o1]
        elif kind == SEG_PAIR:
            a, b = int(plan.seg_a[s]), int(plan.seg_b[s])
            (la, na), (lb, nb) = plan.channel(a), plan.channel(b)
            idx, val = cg_table(la, lb, L)
            xa, xb = _chan(plan, A, a), _chan(plan, A, b)
            g = gI[:, o0 + idx[:, 2]] * val
            ga = np.zeros_like(xa)
            gb = np.zeros_like(xb)
            np.add.at(ga, (slice(None), idx[:, 0]), g * xb[:, idx[:, 1]])
            np.add.at(gb, (slice(None), idx[:, 1]), g * xa[:, idx[:, 0]])
            G[:, na - 1, la * la:(la + 1) * (la + 1)] += ga
            G[:, nb - 1, lb * lb:(lb + 1) * (lb + 1)] += gb
    return e, G


def walk_device_tables(tabs, A, species, k):
    """The device pass over ``RecoupledDeviceTables``, restated loop for loop
    (vectorised over atoms): per L, the components, their adjoints and the energy
    share, then the back-propagation into the A row.  Returns (energies, G)."""
    N = A.shape[0]
    W = tabs.row_width
    row = A.reshape(N, W)
    kz = np.asarray(k)[np.asarray(species)]  # [N, D]
    G = np.zeros((N, W), dtype=np.complex128)
    e = np.zeros(N)
    for L in range(tabs.pass_count):
        c0, c1 = int(tabs.pass_begin[L]), int(tabs.pass_begin[L + 1])
        I = np.zeros((N, c1 - c0), dtype=np.complex128)
        for c in range(c0, c1):
            a, b, q0, qn = (int(v) for v in tabs.comp[c, :4])
            if a < 0:
                I[:, c - c0] = 1.0
            elif qn == 0:
                I[:, c - c0] = row[:, a]
            else:
                q = tabs.cg_index[q0:q0 + qn]
                I[:, c - c0] = (tabs.cg_value[q0:q0 + qn] * row[:, a + (q & 255)] * row[:, b + (q >> 8)]).sum(axis=1)
        gI = np.zeros_like(I)
        for c in range(c0, c1):
            m, o0, on = (int(v) for v in tabs.comp[c, 4:7])
            ent = tabs.own[o0:o0 + on]
            acc = (kz[:, ent[:, 1]] * I[:, ent[:, 0] + 2 * L - m]).sum(axis=1)
            gI[:, c - c0] = -acc if (m - L) & 1 else acc
        e += 0.5 * (I * gI).sum(axis=1).real
        for t in range(W):
            b0, b1 = int(tabs.bp_begin[L * W + t]), int(tabs.bp_begin[L * W + t + 1])
            if b1 == b0:
                continue
            gi, other, val = tabs.bp_gi[b0:b1], tabs.bp_other[b0:b1], tabs.bp_value[b0:b1]
            partner = np.where(other[None, :] < 0, 1.0, row[:, np.maximum(other, 0)])
            G[:, t] += (val * gI[:, gi] * partner).sum(axis=1)
    return e, G.reshape(A.shape)


def walk_forward(tabs, A, species=None, k=None):
    """The forward device pass over ``RecoupledDeviceTables``: per L the components,
    then each contraction ``T_d`` once; returns the energies ``Re(sum_d k[z, d] T_d)``
    when ``k`` is given, else the features ``F [N, feature_count]``."""
    N = A.shape[0]
    W = tabs.row_width
    row = A.reshape(N, W)
    kz = None if k is None else np.asarray(k)[np.asarray(species)]
    e = np.zeros(N)
    F = np.zeros((N, tabs.feature_count), dtype=np.complex128)
    for L in range(tabs.pass_count):
        c0, c1 = int(tabs.pass_begin[L]), int(tabs.pass_begin[L + 1])
        I = np.zeros((N, c1 - c0), dtype=np.complex128)
        for c in range(c0, c1):
            a, b, q0, qn = (int(v) for v in tabs.comp[c, :4])
            if a < 0:
                I[:, c - c0] = 1.0
            elif qn == 0:
                I[:, c - c0] = row[:, a]
            else:
                q = tabs.cg_index[q0:q0 + qn]
                I[:, c - c0] = (tabs.cg_value[q0:q0 + qn] * row[:, a + (q & 255)] * row[:, b + (q >> 8)]).sum(axis=1)
        M = np.arange(-L, L + 1)
        for d in range(int(tabs.dot_begin[L]), int(tabs.dot_begin[L + 1])):
            oa, ob, f0, fn = (int(v) for v in tabs.dot[d])
            T = ((-1.0) ** M * I[:, oa + M + L] * I[:, ob + L - M]).sum(axis=1)
            if kz is not None:
                e += kz[:, d] * T.real
            else:
                F[:, tabs.feat_index[f0:f0 + fn]] += tabs.feat_weight[f0:f0 + fn][None, :] * T[:, None]
    return e if k is not None else F


def walk_sym_tables(tabs, A, species, k):
    """The symmetric device pass over ``RecoupledSymTables`` (physical densities), restated
    loop for loop: per L the ``M >= 0`` components, their adjoints
    ``(-1)^p conj(sum k I_partner[M])``, the energy share, the back-propagation into the
    ``m >= 0`` half of the A row; then the mirror.  Returns (energies, G)."""
    N = A.shape[0]
    W = tabs.row_width
    row = A.reshape(N, W)
    kz = np.asarray(k)[np.asarray(species)]
    G = np.zeros((N, W), dtype=np.complex128)
    e = np.zeros(N)
    for L in range(tabs.pass_count):
        c0, c1 = int(tabs.pass_begin[L]), int(tabs.pass_begin[L + 1])
        I = np.zeros((N, c1 - c0), dtype=np.complex128)
        for c in range(c0, c1):
            a, b, q0, qn = (int(v) for v in tabs.comp[c, :4])
            if a < 0:
                I[:, c - c0] = 1.0
            elif qn == 0:
                I[:, c - c0] = row[:, a]
            else:
                q = tabs.cg_index[q0:q0 + qn]
                I[:, c - c0] = (tabs.cg_value[q0:q0 + qn] * row[:, a + (q & 255)] * row[:, b + (q >> 8)]).sum(axis=1)
        gI = np.zeros_like(I)
        for c in range(c0, c1):
            M, o0, on, sgn = (int(v) for v in tabs.comp[c, 4:8])
            ent = tabs.own[o0:o0 + on]
            gI[:, c - c0] = sgn * np.conj((kz[:, ent[:, 1]] * I[:, ent[:, 0] + M]).sum(axis=1))
            wM = 0.5 if M == 0 else 1.0
            e += wM * (I[:, c - c0] * gI[:, c - c0]).real
        for t in range(W):
            b0, b1 = int(tabs.bp_begin[L * W + t]), int(tabs.bp_begin[L * W + t + 1])
            if b1 == b0:
                continue
            code, other, val = tabs.bp_gi[b0:b1], tabs.bp_other[b0:b1], tabs.bp_value[b0:b1]
            g = gI[:, code >> 1]
            g = np.where((code & 1)[None, :] == 1, np.conj(g), g)
            partner = np.where(other[None, :] < 0, 1.0, row[:, np.maximum(other, 0)])
            G[:, t] += (val * g * partner).sum(axis=1)
    for t in range(W):
        m = int(tabs.mirror[t])
        if m >= 0:
            G[:, t] = (-1.0 if m & 1 else 1.0) * np.conj(G[:, m >> 1])
    return e, G.reshape(A.shape)


def walk_sym_tiled(tabs, tiles, A, species, k):
    """The symmetric pass with the adjoints of the components formed by the dense tiles
    (``RecoupledTiles``) instead of the contraction lists, restated as the tiled kernel walks
    them: per tile and row, the sum over the tile's columns of the row's weight times the
    column's components; the rest as ``walk_sym_tables``.  Returns (energies, G)."""
    N = A.shape[0]
    W = tabs.row_width
    row = A.reshape(N, W)
    kval = tiles.tile_weights(k)[np.asarray(species)]  # [N, rows * steps]
    R = tiles.rows
    G = np.zeros((N, W), dtype=np.complex128)
    e = np.zeros(N)
    for L in range(tabs.pass_count):
        c0, c1 = int(tabs.pass_begin[L]), int(tabs.pass_begin[L + 1])
        I = np.zeros((N, c1 - c0), dtype=np.complex128)
        for c in range(c0, c1):
            a, b, q0, qn = (int(v) for v in tabs.comp[c, :4])
            if a < 0:
                I[:, c - c0] = 1.0
            elif qn == 0:
                I[:, c - c0] = row[:, a]
            else:
                q = tabs.cg_index[q0:q0 + qn]
                I[:, c - c0] = (tabs.cg_value[q0:q0 + qn] * row[:, a + (q & 255)] * row[:, b + (q >> 8)]).sum(axis=1)
        gI = np.zeros_like(I)
        for t in range(int(tiles.tile_begin[L]), int(tiles.tile_begin[L + 1])):
            q0, q1 = int(tiles.tile_col_begin[t]), int(tiles.tile_col_begin[t + 1])
            cols = tiles.col_comp[q0:q1]
            for r in range(R):
                rc = int(tiles.tile_row[t, r])
                if rc < 0:
                    continue
                kv = kval[:, R * q0 + r: R * q1: R]  # [N, steps]
                sgn = int(tabs.comp[c0 + rc, 7])
                for M in range(L + 1):
                    acc = (kv * I[:, cols + M]).sum(axis=1)
                    gI[:, rc + M] = sgn * np.conj(acc)
                    e += (0.5 if M == 0 else 1.0) * (I[:, rc + M] * gI[:, rc + M]).real
        for t in range(W):
            b0, b1 = int(tabs.bp_begin[L * W + t]), int(tabs.bp_begin[L * W + t + 1])
            if b1 == b0:
                continue
            code, other, val = tabs.bp_gi[b0:b1], tabs.bp_other[b0:b1], tabs.bp_value[b0:b1]
            g = gI[:, code >> 1]
            g = np.where((code & 1)[None, :] == 1, np.conj(g), g)
            partner = np.where(other[None, :] < 0, 1.0, row[:, np.maximum(other, 0)])
            G[:, t] += (val * g * partner).sum(axis=1)
    for t in range(W):
        m = int(tabs.mirror[t])
        if m >= 0:
            G[:, t] = (-1.0 if m & 1 else 1.0) * np.conj(G[:, m >> 1])
    return e, G.reshape(A.shape)


def walk_sym_forward(tabs, A, species, k):
    """The symmetric forward energy: ``T_d = (-1)^p_B (Re(I_A[0] conj(I_B[0])) +
    2 sum_{M > 0} Re(I_A[M] conj(I_B[M])))``, ``e = sum_d k[z, d] T_d``."""
    N = A.shape[0]
    row = A.reshape(N, tabs.row_width)
    kz = np.asarray(k)[np.asarray(species)]
    e = np.zeros(N)
    for L in range(tabs.pass_count):
        c0, c1 = int(tabs.pass_begin[L]), int(tabs.pass_begin[L + 1])
        I = np.zeros((N, c1 - c0), dtype=np.complex128)
        for c in range(c0, c1):
            a, b, q0, qn = (int(v) for v in tabs.comp[c, :4])
            if a < 0:
                I[:, c - c0] = 1.0
            elif qn == 0:
                I[:, c - c0] = row[:, a]
            else:
                q = tabs.cg_index[q0:q0 + qn]
                I[:, c - c0] = (tabs.cg_value[q0:q0 + qn] * row[:, a + (q & 255)] * row[:, b + (q >> 8)]).sum(axis=1)
        wts = np.array([1.0] + [2.0] * L)
        for d in range(int(tabs.dot_begin[L]), int(tabs.dot_begin[L + 1])):
            oa, ob, sgn, _ = (int(v) for v in tabs.dot[d])
            T = sgn * (wts * (I[:, oa:oa + L + 1] * np.conj(I[:, ob:ob + L + 1])).real).sum(axis=1)
            e += kz[:, d] * T
    return e
