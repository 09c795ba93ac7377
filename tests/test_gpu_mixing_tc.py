"""Mixed-channel A-basis with the mixing as a tensor-core product after per-species
edge sums (fp32: tcgen05 kind::tf32, 3xTF32; fp64: FP64 mma.sync) against the CPU
oracle (which restates ye3t_runtime_core.cpp:651 with the A-basis of
execution_plan.py:7298/:7479/:7913 and is pinned to the reference's golden mixed
density in test_oracle_golden.py) and against the fused per-edge CUDA-core kernel.
Tolerances: 1e-5 (fp32) and 1e-12 (fp64) of the largest |A|."""

import os

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _evaluator(stem, g):
    from ye3t_b200.ace import ACEConfig, ACEEvaluator
    from ye3t_b200.schedules import ACEBundle
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", stem + ".npz"))
    return ACEEvaluator(b, DEV, config=ACEConfig(float(g["rc"]), float(g["lam"])))


def _system(g, S):
    pos = torch.as_tensor(g["pos"], device=DEV)
    sp = torch.as_tensor(np.asarray(g["species"]) % S, dtype=torch.int32, device=DEV)
    return pos, sp, float(g["box"])


def _oracle(g, ev, pos, sp, box, row, nbr, mix, nmax):
    """The oracle's mixed density on the GPU's own neighbour rows (minimum-image
    displacements recomputed on the host)."""
    P = pos.cpu().numpy()
    r = row.cpu().numpy()
    n = nbr.cpu().numpy()[: int(r[-1])]
    centres = np.repeat(np.arange(r.shape[0] - 1), np.diff(r))
    d = P[n] - P[centres]
    d -= box * np.rint(d / box)
    return oracle.ace_density_mixed(d, r, n.astype(np.int32), sp.cpu().numpy().astype(np.int32), mix, nmax,
                                    ev.bundle.lmax, float(g["rc"]), float(g["lam"]))


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float64, 1e-12)])
@pytest.mark.parametrize("stem,S,C,nmax", [("ace_diag_l4_nu4_L0", 4, 32, 12),   # C3 shape
                                           ("ace_diag_l3_nu3_L0", 2, 64, 8),    # C4 shape
                                           ("ace_diag_l3_nu3_L0", 3, 16, 5)])   # padded K and N
def test_tensor_core_mixing_matches_oracle(golden, stem, S, C, nmax, dtype, tol):
    g = golden("mixing_small")
    ev = _evaluator(stem, g)
    pos, sp, box = _system(g, S)
    row, nbr = ev.neighbor_list(pos, box)
    mix = (torch.randn(S, S, C, nmax, dtype=torch.float64, generator=torch.Generator().manual_seed(7))
           / nmax ** 0.5).numpy()
    mix_t = torch.as_tensor(mix, dtype=dtype)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    A = ev.density_mixed(pos, sp, box, row, nbr, mix_t, dtype=dtype, status=status, tensor_cores=True)
    assert int(status.item()) == 0
    cdt = torch.complex64 if dtype == torch.float32 else torch.complex128
    assert A.dtype == cdt and A.shape == (pos.shape[0], C, (ev.bundle.lmax + 1) ** 2)
    ref = _oracle(g, ev, pos, sp, box, row, nbr, mix_t.to(torch.float64).numpy(), nmax)
    scale = np.abs(ref).max()
    err = np.abs(A.cpu().numpy().astype(np.complex128) - ref).max() / scale
    assert err <= tol, err
    # the fused per-edge CUDA-core kernel gives the same A within the rounding of the type
    A_cc = ev.density_mixed(pos, sp, box, row, nbr, mix_t, dtype=dtype, tensor_cores=False)
    assert (A - A_cc).abs().max().item() <= tol * scale


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_tensor_core_mixing_chunks_and_ranges(golden, dtype):
    """A workspace of a few centres (several chunks) and a centre sub-range give the rows
    of the one-chunk run bit for bit; a bad centre species gives a zero row and the flag."""
    from ye3t_b200 import _native as nat
    g = golden("mixing_small")
    ev = _evaluator("ace_diag_l4_nu4_L0", g)
    S, C, nmax = 4, 32, 12
    code = nat.dtype_code(dtype)
    pos, sp, box = _system(g, S)
    row, nbr = ev.neighbor_list(pos, box)
    mix = (torch.randn(S, S, C, nmax, dtype=dtype, generator=torch.Generator().manual_seed(3)) / nmax ** 0.5).to(DEV)
    full = ev.density_mixed(pos, sp, box, row, nbr, mix, dtype=dtype, tensor_cores=True)
    N = pos.shape[0]
    lib = nat.lib()
    per_atom = int(lib.y3b_ace_density_mixed_split_workspace_bytes(code, 1, S, C, nmax, 4))
    ws = torch.empty(per_atom * 5 + 7, dtype=torch.uint8, device=DEV)  # 5 centres per chunk
    out = torch.empty_like(full)
    nat.check(lib.y3b_ace_density_mixed_split(
        code, pos.data_ptr(), sp.data_ptr(), N, 0, N, box, row.data_ptr(), nbr.data_ptr(), mix.data_ptr(), S, C,
        nmax, 4, float(g["rc"]), float(g["lam"]), ws.data_ptr(), ws.numel(), out.data_ptr(), None,
        nat.stream_of(torch.device(DEV))), "ace_density_mixed_split")
    torch.cuda.synchronize()
    assert torch.equal(out, full)
    # centres [10, 40) with their own rows
    row_s, nbr_s = ev.neighbor_list(pos, box, 10, 40)
    part = ev.density_mixed(pos, sp, box, row_s, nbr_s, mix, begin=10, dtype=dtype, tensor_cores=True)
    assert torch.equal(part, full[10:40])
    # a bad centre species: zero row, INDEX_RANGE
    bad = sp.clone()
    bad[3] = 9
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    A = ev.density_mixed(pos, bad, box, row, nbr, mix, dtype=dtype, status=status, tensor_cores=True)
    assert int(status.item()) & nat.STATUS_INDEX_RANGE
    assert torch.all(A[3] == 0)
    # too small a workspace is refused before any launch
    rc = lib.y3b_ace_density_mixed_split(
        code, pos.data_ptr(), sp.data_ptr(), N, 0, N, box, row.data_ptr(), nbr.data_ptr(), mix.data_ptr(), S, C,
        nmax, 4, float(g["rc"]), float(g["lam"]), ws.data_ptr(), per_atom - 1, out.data_ptr(), None,
        nat.stream_of(torch.device(DEV)))
    assert rc == -3  # Y3B_ERR_WORKSPACE
    # shapes outside either product path are refused
    assert int(lib.y3b_ace_density_mixed_split_workspace_bytes(code, 1, S, 12, nmax, 4)) == -1
