"""Host-side packing checked on CPU: a numpy emulation of the pool and bundle
kernels over the packed tables must reproduce the oracle's features."""

import os

import numpy as np
import pytest
import torch

from oracle import oracle
from ye3t_b200.packing import pack_bundle
from ye3t_b200.schedules import ACEBundle

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bundle(stem):
    return ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", stem + ".npz"))


def emulate_pool(pb, A):
    a = {k: v.cpu().numpy() for k, v in pb.arrays.items()}
    N, nmax, W = A.shape
    pool = np.zeros((pb.pool_size, N), dtype=np.complex128)
    pool[: nmax * W] = A.reshape(N, nmax * W).T
    for l, k, Lam, off, tb, te in a["sym_kind"]:
        dimo = 2 * Lam + 1
        for n in range(nmax):
            x = A[:, n, l * l:(l + 1) * (l + 1)]
            for q in range(tb, te):
                f = int(np.uint32(a["sym_term_factors"][q]))
                m = np.full(N, a["sym_term_coeff"][q], dtype=np.complex128)
                for kk in range(4):
                    ci = (f >> (8 * kk)) & 255
                    if ci == 255:
                        break
                    m = m * x[:, ci]
                pool[off + n * dimo + a["sym_term_output"][q]] += m
    return pool


def emulate_features(pb, pool):
    a = {k: v.cpu().numpy() for k, v in pb.arrays.items()}
    N = pool.shape[1]
    out = np.zeros((N, pb.feature_count), dtype=np.complex128)
    for w in range(pb.bundle.word_count):
        p = a["word_pattern"][w]
        B = a["pattern_block_count"][p]
        lb = a["word_label_base"][w]
        fo = a["word_feature_offset"][w]
        c0, c1 = a["pattern_comp_begin"][p], a["pattern_comp_begin"][p + 1]
        for c in range(c0, c1):
            base = a["label_bases"][lb + a["comp_label"][c]]
            acc = np.zeros(N, dtype=np.complex128)
            for q in range(a["comp_term_begin"][c], a["comp_term_begin"][c + 1]):
                mm = int(np.uint32(a["term_m"][q]))
                v = a["term_coeff"][q] * pool[base[0] + (mm & 255)]
                for b in range(1, B):
                    v = v * pool[base[b] + ((mm >> (8 * b)) & 255)]
                acc += v
            out[:, fo + c - c0] = acc
    return out


def test_packing_layout_and_counts():
    b = _bundle("ace_n8_l3_nu4_L0")
    pb = pack_bundle(b, "cpu")
    assert pb.feature_count == 41168
    assert pb.term_count_per_atom == 1332116
    assert pb.term_block_count_per_atom == 5163248
    assert pb.pool_size == 8 * 16 + 8 * 89
    assert pb.max_blocks == 4


@pytest.mark.parametrize("stem", ["ace_n8_l3_nu3_L0"])
def test_packed_tables_reproduce_oracle_features(golden, stem):
    g = golden("ace_small")
    A = g["A"][:6]
    b = _bundle(stem)
    pb = pack_bundle(b, "cpu")
    pool = emulate_pool(pb, A)
    got = emulate_features(pb, pool)
    ref = oracle.bundle_features(b, A)
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12 * np.abs(ref).max())
    np.testing.assert_allclose(got, g["B3"][:6], rtol=1e-11, atol=1e-12 * np.abs(ref).max())
