"""Atom-block partition and the energy and force reductions, as 2 gloo ranks on CPU.

Each rank evaluates its centre block with the CPU oracle (the GPU kernels are
covered by the gpu tests); the summed energy must equal the single-process
energy, the summed partial forces must equal the reference's forces, and the
blocks must tile the system."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from ye3t_b200.distributed import atom_block

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_atom_blocks_tile_the_system():
    for N in (0, 1, 7, 96, 1 << 20):
        for P in (1, 2, 3, 4, 8):
            spans = [atom_block(r, P, N) for r in range(P)]
            assert spans[0][0] == 0 and spans[-1][1] == N
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(e - b for b, e in spans) - min(e - b for b, e in spans) <= 1
    with pytest.raises(ValueError):
        atom_block(2, 2, 10)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out_path):
    import sys
    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from oracle import oracle
    from ye3t_b200.distributed import atom_block, init_from_env, sum_over_ranks
    from ye3t_b200.schedules import ACEBundle
    import torch.distributed as dist
    r, w = init_from_env("gloo", 60.0)
    g = dict(np.load(os.path.join(REPO, "tests", "golden", "ace_small.npz")))
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu3_L0.npz"))
    N = g["pos"].shape[0]
    lo, hi = atom_block(r, w, N)
    A = oracle.ace_density(g["disp"], g["row_off"], g["nbr"], g["species"], g["prefactor"], 8, 3,
                           float(g["rc"]), float(g["lam"]))
    e = oracle.bundle_energy(b, A[lo:hi], g["species"][lo:hi], g["w3"], threads=2).sum()
    total = sum_over_ranks(torch.tensor([e], dtype=torch.float64))
    if r == 0:
        np.save(out_path, total.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_energy_equals_single_process(tmp_path, golden):
    out = str(tmp_path / "total.npy")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    total = float(np.load(out)[0])
    ref = float(golden("ace_small")["energy3"])
    assert abs(total - ref) <= 1e-12 * abs(ref)


def _rank_forces(rank, world, port, out_path):
    """One rank of the force decomposition: ``G = dE/dA`` of its centre block, the
    edge gradients of its CSR rows, and a full-length partial force array (each
    edge i->j adds ``g`` to atom i and subtracts it from atom j, both global
    indices); the ranks then sum the partial arrays."""
    import sys
    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from oracle import oracle
    from ye3t_b200.distributed import atom_block, init_from_env, sum_over_ranks
    from ye3t_b200.schedules import ACEBundle
    import torch.distributed as dist
    r, w = init_from_env("gloo", 60.0)
    g = dict(np.load(os.path.join(REPO, "tests", "golden", "ace_small.npz")))
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu3_L0.npz"))
    N = g["pos"].shape[0]
    rc, lam = float(g["rc"]), float(g["lam"])
    lo, hi = atom_block(r, w, N)
    A = oracle.ace_density(g["disp"], g["row_off"], g["nbr"], g["species"], g["prefactor"], 8, 3, rc, lam)
    e, G = oracle.bundle_energy_grad(b, A[lo:hi], g["species"][lo:hi], g["w3"], threads=2)
    off = g["row_off"].astype(np.int64)
    e0, e1 = int(off[lo]), int(off[hi])
    rows = off[lo:hi + 1] - e0
    nbr = g["nbr"][e0:e1]
    ge = oracle.ace_edge_grad(g["disp"][e0:e1], rows, nbr, g["species"], g["prefactor"], 8, 3, rc, lam, G)
    centre = np.repeat(np.arange(lo, hi), np.diff(rows))
    F = np.zeros((N, 3))
    np.add.at(F, centre, ge)
    np.add.at(F, nbr.astype(np.int64), -ge)
    total = sum_over_ranks(torch.tensor(np.concatenate([[e.sum()], F.reshape(-1)]), dtype=torch.float64))
    if r == 0:
        np.save(out_path, total.numpy())
    # the bench's collective: a reduce-scatter of the partial arrays (padded to
    # world * chunk rows) leaves each rank the forces of its own chunk
    from ye3t_b200.distributed import block_forces
    chunk = (N + w - 1) // w
    padded = torch.zeros((chunk * w, 3), dtype=torch.float64)
    padded[:N] = torch.as_tensor(F)
    mine = block_forces(padded, torch.empty((chunk, 3), dtype=torch.float64))
    np.save(f"{out_path}.block{r}.npy", mine.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_rank_partial_forces_sum_to_reference(tmp_path, golden, world):
    out = str(tmp_path / "forces.npy")
    mp.start_processes(_rank_forces, args=(world, _free_port(), out), nprocs=world, join=True,
                       start_method="spawn")
    total = np.load(out)
    ref = golden("forces_small")
    F_ref = np.asarray(ref["forces"])
    assert abs(total[0] - float(ref["energy"])) <= 1e-12 * abs(float(ref["energy"]))
    F = total[1:].reshape(-1, 3)
    assert np.abs(F - F_ref).max() <= 1e-10 * max(1.0, np.abs(F_ref).max())
    blocks = np.concatenate([np.load(f"{out}.block{r}.npy") for r in range(world)])[:F_ref.shape[0]]
    assert np.abs(blocks - F_ref).max() <= 1e-10 * max(1.0, np.abs(F_ref).max())
