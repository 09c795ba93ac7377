"""Fused ACE descriptor / energy evaluation on one GPU (or one atom block).

Pipeline for the centres ``[begin, end)`` of a periodic cubic box:

1. cell-list neighbour list in sorted CSR form (``y3b_neighbor_count`` /
   ``y3b_neighbor_fill``);
2. A-basis density (kernel 1, ``y3b_ace_density``): per centre
   ``A[n, lm] = sum_j p[z_j] R_n(r_ij) Yc_lm(r_ij)`` -- the composition of the
   reference's radial table (``ye3t/runtime/execution_plan.py:7298``), complex
   harmonics (``:7479``), per-neighbour prefactor (``:7582``) and
   ``density_accumulate`` (``:7913``), fused;
3. B-basis (kernel 2): every word's factorized schedule
   (``ACEFactorizedScheduleReport.evaluate``,
   ``ye3t/couplings/__init__.py:2574``) -- either written out as features or
   contracted with a per-species linear readout into per-atom energies.

   For energies (and dE/dA) of a scalar bundle the default B-basis is the
   recoupled plan (``ye3t_b200.recoupling``): each feature as contractions of
   coupled channel pairs, evaluated by the recoupled passes, with the
   ``M >= 0`` (symmetric) passes wherever A comes from this class's density
   kernel (real radial functions and prefactors give
   ``A[l, -m] = (-1)^m conj(A[l, m])``).  ``b_basis="term"`` selects the
   term-level kernels (``y3b_ace_energy`` / ``y3b_ace_energy_grad``: the
   symmetric blocks of ``ye3t/runtime/symmetric_power.py:879`` formed on chip,
   then the schedule items), which also serve features and L > 0 bundles.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _native as nat
from .packing import PackedBundle, pack_bundle
from .schedules import ACEBundle

__all__ = ["ACEConfig", "ACEEvaluator"]


@dataclass(frozen=True)
class ACEConfig:
    cutoff: float = 5.0
    radial_lambda: float = 5.0


class ACEEvaluator:
    """Evaluates one :class:`ACEBundle` on one CUDA device."""

    #: CTA shapes (atoms, threads, tile rows) of the recoupled passes used by default:
    #: the adjoint of a physical density through the dense tiles (4 atoms, 8-segment
    #: tiles), that of any other A through the general lists, and the energy alone
    RECOUPLED_TILED_SHAPE = (4, 512, 8)
    RECOUPLED_GRAD_SHAPE = (2, 256, 0)
    RECOUPLED_ENERGY_SHAPE = (1, 256, 0)

    def __init__(self, bundle: ACEBundle, device, *, config: ACEConfig = ACEConfig(),
                 species_prefactor=None, weights=None, b_basis: str = "recoupled"):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("ACEEvaluator runs on CUDA devices only")
        if b_basis not in ("recoupled", "term"):
            raise ValueError('b_basis must be "recoupled" or "term"')
        nat.lib()
        self.bundle = bundle
        self.config = config
        self.packed: PackedBundle = pack_bundle(bundle, self.device)
        self._tables = self.packed.tables()
        self.W = (bundle.lmax + 1) ** 2
        self.species_prefactor = None if species_prefactor is None else torch.as_tensor(
            species_prefactor, dtype=torch.float64, device=self.device).contiguous()
        self.weights = None if weights is None else torch.as_tensor(
            weights, dtype=torch.float64, device=self.device).contiguous()
        if self.weights is not None and self.weights.shape[-1] != self.packed.feature_count:
            raise ValueError(f"weights need {self.packed.feature_count} features per species")
        # energies and dE/dA of scalar bundles go through the recoupled passes
        # unless the term-level kernels are asked for
        self.b_basis = b_basis if bundle.target_L == 0 else "term"
        self._recoupled = {}

    def recoupled(self, symmetric: bool, grad: bool):
        """The :class:`~ye3t_b200.recoupling.RecoupledEvaluator` used for energies (``grad``
        False) or energies and dE/dA, built on first use (the plan is fitted once)."""
        key = (bool(symmetric), bool(grad))
        if key not in self._recoupled:
            from .recoupling import RecoupledEvaluator, build_recoupled_plan
            if self.weights is None:
                raise ValueError("weights are required for the energy")
            plan = next((r.plan for r in self._recoupled.values()), None) or build_recoupled_plan(self.bundle)
            if grad:
                na, th, rows = self.RECOUPLED_TILED_SHAPE if symmetric else self.RECOUPLED_GRAD_SHAPE
            else:
                na, th, rows = self.RECOUPLED_ENERGY_SHAPE
            self._recoupled[key] = RecoupledEvaluator(self.bundle, self.device, self.weights.cpu().numpy(),
                                                      plan=plan, atoms_per_cta=min(na, 4), threads_per_cta=th,
                                                      symmetric=symmetric, tile_rows=rows)
        return self._recoupled[key]

    def recoupled_features(self):
        """The general recoupled passes used for fp64 features (built on first use; no readout
        weights needed)."""
        if "features" not in self._recoupled:
            from .recoupling import RecoupledEvaluator, build_recoupled_plan
            plan = next((r.plan for r in self._recoupled.values()), None) or build_recoupled_plan(self.bundle)
            self._recoupled["features"] = RecoupledEvaluator(self.bundle, self.device, None, plan=plan,
                                                             atoms_per_cta=1, threads_per_cta=256)
        return self._recoupled["features"]

    @property
    def feature_count(self) -> int:
        return self.packed.feature_count

    def _stream(self):
        return nat.stream_of(self.device)

    def mixing_on_tensor_cores(self, species_count: int, channel_count: int, nmax: int, dtype) -> bool:
        """Whether ``density_mixed`` runs the mixing of this shape as a tensor-core product by
        default: fp32 (tcgen05, 3xTF32) needs C a multiple of 16, S * n_max <= 64 and
        S * C <= 256; fp64 (FP64 mma.sync) C a multiple of 8 up to 64 and S * n_max <= 64; both
        l_max <= 4 and n_max <= 16."""
        code = nat.F64 if dtype == torch.float64 else (nat.F32 if dtype == torch.float32 else None)
        if code is None:
            return False
        return int(nat.lib().y3b_ace_density_mixed_split_workspace_bytes(
            code, 1, int(species_count), int(channel_count), int(nmax), self.bundle.lmax)) > 0

    def _workspace(self, nbytes: int) -> torch.Tensor:
        """A device scratch buffer of at least ``nbytes`` (kept and grown between calls)."""
        ws = getattr(self, "_scratch", None)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=self.device)
            self._scratch = ws
        return ws

    # -- neighbour list --------------------------------------------------------
    def neighbor_list(self, positions: torch.Tensor, box: float, begin: int = 0,
                      end: Optional[int] = None, z_window: Optional[Tuple[int, int]] = None,
                      capacity: Optional[int] = None,
                      status: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """CSR rows ``(row_offsets [n+1] int64, neighbors [E] int32)`` for centres [begin, end).

        ``z_window = (first z cell layer, layer count)`` bins only that slab of the box
        (``y3b_neighbor_count_window``): the centres must be a slab inside it, one layer
        in from each side (``slab_window`` computes it).  With ``capacity`` the neighbour
        array is allocated at that size without reading the edge total back to the host
        (no device sync); ``neighbors`` is then the whole buffer, of which
        ``row_offsets[-1]`` entries are used, and an overflow sets
        ``Y3B_STATUS_CAPACITY`` in ``status``."""
        pos = positions.to(self.device, torch.float64).contiguous()
        N = pos.shape[0]
        end = N if end is None else int(end)
        lib = nat.lib()
        rc = float(self.config.cutoff)
        ws_bytes = int(lib.y3b_neighbor_workspace_bytes(N, float(box), rc))
        key = (N, ws_bytes)
        if getattr(self, "_nbr_ws_key", None) != key:
            self._nbr_ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=self.device)
            self._nbr_ws_key = key
        ws = self._nbr_ws
        row = torch.empty(end - begin + 1, dtype=torch.int64, device=self.device)
        s = self._stream()
        zb, zc = (0, 0) if z_window is None else (int(z_window[0]), int(z_window[1]))
        nat.check(lib.y3b_neighbor_count_window(pos.data_ptr(), N, begin, end, float(box), rc, zb, zc,
                                                ws.data_ptr(), ws_bytes, row.data_ptr(), nat.ptr(status), s),
                  "neighbor_count")
        if capacity is None:
            E = int(row[-1].item())
            cap = E
        else:
            E = cap = int(capacity)
        nbr = torch.empty(max(cap, 1), dtype=torch.int32, device=self.device)
        nat.check(lib.y3b_neighbor_fill_window(pos.data_ptr(), N, begin, end, float(box), rc, zb, zc,
                                               ws.data_ptr(), ws_bytes, row.data_ptr(), cap, nbr.data_ptr(),
                                               nat.ptr(status), s), "neighbor_fill")
        return row, nbr[:E]

    def slab_window(self, positions, box: float, begin: int, end: int) -> Optional[Tuple[int, int]]:
        """The z window ``(first layer, count)`` of the cell list that holds the centres
        ``[begin, end)`` with one layer of halo on each side, or None when that is the whole
        box.  Read from host positions; meant for atoms stored in cell order, where an atom
        block is a slab."""
        import numpy as np
        n = int(nat.lib().y3b_neighbor_cells_per_side(float(box), float(self.config.cutoff)))
        if n < 3 or end <= begin:
            return None
        z = np.asarray(positions[begin:end, 2].cpu() if hasattr(positions, "cpu") else positions[begin:end, 2],
                       dtype=np.float64)
        f = z / box
        cz = np.clip(((f - np.floor(f)) * n).astype(np.int64), 0, n - 1)
        layers = np.unique(cz)
        # the smallest periodic run of layers that holds every centre layer
        gaps = np.diff(np.concatenate([layers, [layers[0] + n]]))
        g = int(np.argmax(gaps))
        first = int(layers[(g + 1) % layers.shape[0]])
        span = int(n - gaps[g] + 1)
        if span + 2 >= n:
            return None
        return ((first - 1) % n, span + 2)

    # -- kernel 1 ----------------------------------------------------------------
    def density(self, positions, species, box, row_offsets, neighbors, begin: int = 0,
                status: Optional[torch.Tensor] = None) -> torch.Tensor:
        """A-basis ``[n_centres, nmax, (lmax+1)^2]`` complex128."""
        if self.species_prefactor is None:
            raise ValueError("species_prefactor is required for the density")
        pos = positions.to(self.device, torch.float64).contiguous()
        sp = species.to(self.device, torch.int32).contiguous()
        count = int(row_offsets.shape[0]) - 1
        A = torch.empty((count, self.bundle.nmax, self.W), dtype=torch.complex128, device=self.device)
        nat.check(nat.lib().y3b_ace_density(
            pos.data_ptr(), sp.data_ptr(), pos.shape[0], int(begin), count, float(box), row_offsets.data_ptr(),
            neighbors.data_ptr(), self.species_prefactor.data_ptr(), self.species_prefactor.numel(),
            self.bundle.nmax, self.bundle.lmax, float(self.config.cutoff), float(self.config.radial_lambda),
            A.data_ptr(), nat.ptr(status), self._stream()), "ace_density")
        return A

    def density_mixed(self, positions, species, box, row_offsets, neighbors, mixing, begin: int = 0,
                      dtype=torch.float64, status: Optional[torch.Tensor] = None,
                      tensor_cores: Optional[bool] = None) -> torch.Tensor:
        """A-basis ``[n_centres, C, (lmax+1)^2]`` with radial channels mixed per species pair.

        ``mixing [S, S, C, nmax]``: channel c of a pair (z_i, z_j) is
        ``sum_n mixing[z_i, z_j, c, n-1] R_n``.  ``dtype`` float64 gives
        complex128, float32 complex64 (computed in that precision).  The mixing runs
        as a tensor-core product after per-species edge sums
        (``y3b_ace_density_mixed_split``: tcgen05 in fp32, FP64 mma.sync in fp64)
        wherever its shape allows (``tensor_cores`` None); True requires that path,
        False uses the fused per-edge CUDA-core kernel.
        """
        pos = positions.to(self.device, torch.float64).contiguous()
        sp = species.to(self.device, torch.int32).contiguous()
        W = torch.as_tensor(mixing, dtype=dtype, device=self.device).contiguous()
        if W.dim() != 4 or W.shape[0] != W.shape[1]:
            raise ValueError("mixing must be [S, S, C, nmax]")
        count = int(row_offsets.shape[0]) - 1
        cdt = torch.complex128 if dtype == torch.float64 else torch.complex64
        A = torch.empty((count, W.shape[2], self.W), dtype=cdt, device=self.device)
        S, C, nmax = W.shape[0], W.shape[2], W.shape[3]
        tc_ok = self.mixing_on_tensor_cores(S, C, nmax, dtype)
        if tensor_cores and not tc_ok:
            raise ValueError("the tensor-core mixing needs l_max <= 4, n_max <= 16 and (fp32) C a multiple of 16, "
                             "S * n_max <= 64, S * C <= 256 or (fp64) C a multiple of 8 up to 64 and S * n_max <= 64")
        if tc_ok and tensor_cores is not False:
            code = nat.dtype_code(dtype)
            need = int(nat.lib().y3b_ace_density_mixed_split_workspace_bytes(code, count, S, C, nmax,
                                                                            self.bundle.lmax))
            ws = self._workspace(min(need, 1 << 30))
            nat.check(nat.lib().y3b_ace_density_mixed_split(
                code, pos.data_ptr(), sp.data_ptr(), pos.shape[0], int(begin), count, float(box),
                row_offsets.data_ptr(), neighbors.data_ptr(), W.data_ptr(), S, C, nmax, self.bundle.lmax,
                float(self.config.cutoff), float(self.config.radial_lambda), ws.data_ptr(), ws.numel(), A.data_ptr(),
                nat.ptr(status), self._stream()), "ace_density_mixed_split")
            return A
        nat.check(nat.lib().y3b_ace_density_mixed(
            nat.dtype_code(dtype), pos.data_ptr(), sp.data_ptr(), pos.shape[0], int(begin), count, float(box),
            row_offsets.data_ptr(), neighbors.data_ptr(), W.data_ptr(), W.shape[0], W.shape[2], W.shape[3],
            self.bundle.lmax, float(self.config.cutoff), float(self.config.radial_lambda), A.data_ptr(),
            nat.ptr(status), self._stream()), "ace_density_mixed")
        return A

    # -- kernel 2 ----------------------------------------------------------------
    def features(self, A: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """B-basis features ``[n, feature_count]`` from the A-basis.

        complex128 A gives complex128 features; complex64 A is evaluated in
        fp32 and gives complex64 features.  For a scalar bundle in fp64 with the
        recoupled B-basis (the default) the features come from the recoupled
        forward pass (``y3b_ace_recoupled_features``: each feature as its
        contractions of coupled channel pairs, about half the time of the
        term-level kernel at C2); otherwise from the term-level kernel.
        """
        dt = torch.complex64 if A.dtype == torch.complex64 else torch.complex128
        A = A.to(self.device, dt).contiguous()
        n = A.shape[0]
        if out is None:
            out = torch.empty((n, self.packed.feature_count), dtype=dt, device=self.device)
        if self.b_basis == "recoupled" and dt == torch.complex128:
            return self.recoupled_features().features(A, out=out)
        return self._term_features(A, out)

    def _term_features(self, A: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Features of contiguous device rows ``A`` into ``out`` by the term-level kernel."""
        n = A.shape[0]
        dt = A.dtype
        code = nat.C64 if dt == torch.complex64 else nat.C128
        nat.check(nat.lib().y3b_ace_features_typed(code, ctypes_ref(self._tables), A.data_ptr(), n, out.data_ptr(),
                                                   self._stream()), "ace_features")
        return out

    def channel_features(self, A: torch.Tensor) -> torch.Tensor:
        """Channel-diagonal features ``[n, C * feature_count]`` from mixed channels ``A [n, C, W]``.

        The bundle's words read a single radial channel (``nmax == 1``); every
        channel is evaluated with the same items, channel c's features at
        ``[c * F, (c + 1) * F)``.
        """
        if self.bundle.nmax != 1:
            raise ValueError("channel_features needs a channel-diagonal bundle (nmax == 1)")
        n, C, W = A.shape
        dt = torch.complex64 if A.dtype == torch.complex64 else torch.complex128
        rows = A.to(self.device, dt).reshape(n * C, 1, W).contiguous()
        # the term-level kernel: on rows of one channel it is faster than the recoupled pass
        out = torch.empty((n * C, self.packed.feature_count), dtype=dt, device=self.device)
        self._term_features(rows, out)
        return out.reshape(n, C * self.packed.feature_count)

    def energy_from_density(self, A: torch.Tensor, species_centres: torch.Tensor,
                            out: Optional[torch.Tensor] = None, physical: bool = False) -> torch.Tensor:
        """Per-atom energies ``sum_f w[z, f] Re(B_f)`` from the A-basis (B never stored).

        ``physical=True`` declares that A has the symmetry of a physical density
        (as ``density`` gives), which lets the recoupled B-basis use its
        ``M >= 0`` passes; any other A takes the general passes."""
        if self.weights is None:
            raise ValueError("weights are required for the energy")
        A = A.to(self.device, torch.complex128).contiguous()
        n = A.shape[0]
        sp = species_centres.to(self.device, torch.int32).contiguous()
        if self.b_basis == "recoupled":
            e = self.recoupled(physical, False).energy(A, sp, check_symmetry=False)
            if out is not None:
                out.copy_(e)
                return out
            return e
        if out is None:
            out = torch.empty(n, dtype=torch.float64, device=self.device)
        nat.check(nat.lib().y3b_ace_energy(ctypes_ref(self._tables), A.data_ptr(), n, sp.data_ptr(),
                                           self.weights.data_ptr(), self.weights.shape[0], out.data_ptr(),
                                           self._stream()), "ace_energy")
        return out

    # -- force path ------------------------------------------------------------------
    def energy_grad(self, A: torch.Tensor, species_centres: torch.Tensor, status: Optional[torch.Tensor] = None,
                    physical: bool = False):
        """(per-atom energies, G = dE/dA) from the A-basis (B is holomorphic in A: dE = Re(sum G dA)).

        ``physical`` as in ``energy_from_density``."""
        if self.weights is None:
            raise ValueError("weights are required for the energy")
        A = A.to(self.device, torch.complex128).contiguous()
        n = A.shape[0]
        sp = species_centres.to(self.device, torch.int32).contiguous()
        if self.b_basis == "recoupled":
            return self.recoupled(physical, True).energy_grad(A, sp, status=status, check_symmetry=False)
        e = torch.empty(n, dtype=torch.float64, device=self.device)
        G = torch.empty_like(A)
        nat.check(nat.lib().y3b_ace_energy_grad(ctypes_ref(self._tables), A.data_ptr(), n, sp.data_ptr(),
                                                self.weights.data_ptr(), self.weights.shape[0], e.data_ptr(),
                                                G.data_ptr(), nat.ptr(status), self._stream()), "ace_energy_grad")
        return e, G

    def edge_grad(self, positions, species, box, row_offsets, neighbors, dEdA, begin: int = 0,
                  status: Optional[torch.Tensor] = None) -> torch.Tensor:
        """g_e = dE_i/dd_e [E, 3] for the rows of centres [begin, begin + n)."""
        pos = positions.to(self.device, torch.float64).contiguous()
        sp = species.to(self.device, torch.int32).contiguous()
        count = int(row_offsets.shape[0]) - 1
        E = int(neighbors.shape[0])
        g = torch.empty((max(E, 1), 3), dtype=torch.float64, device=self.device)
        nat.check(nat.lib().y3b_ace_edge_grad(
            pos.data_ptr(), sp.data_ptr(), pos.shape[0], int(begin), count, float(box), row_offsets.data_ptr(),
            neighbors.data_ptr(), self.species_prefactor.data_ptr(), self.species_prefactor.numel(),
            self.bundle.nmax, self.bundle.lmax, float(self.config.cutoff), float(self.config.radial_lambda),
            dEdA.data_ptr(), g.data_ptr(), nat.ptr(status), self._stream()), "ace_edge_grad")
        return g[:E]

    def forces_from_edges(self, row_offsets, neighbors, edge_grad, status: Optional[torch.Tensor] = None):
        """F = -dE/dr for every atom from the rows of all atoms (deterministic gather)."""
        N = int(row_offsets.shape[0]) - 1
        F = torch.empty((N, 3), dtype=torch.float64, device=self.device)
        nat.check(nat.lib().y3b_forces_gather(row_offsets.data_ptr(), neighbors.data_ptr(), N,
                                              edge_grad.data_ptr(), F.data_ptr(), nat.ptr(status),
                                              self._stream()), "forces_gather")
        return F

    def partial_forces_from_edges(self, row_offsets, neighbors, edge_grad, begin: int, atom_count: int,
                                  out: Optional[torch.Tensor] = None):
        """This atom block's contribution to every atom's force (the sum over blocks is F)."""
        count = int(row_offsets.shape[0]) - 1
        if out is None:
            out = torch.zeros((atom_count, 3), dtype=torch.float64, device=self.device)
        nat.check(nat.lib().y3b_forces_scatter(row_offsets.data_ptr(), neighbors.data_ptr(), int(begin), count,
                                               int(atom_count), edge_grad.data_ptr(), out.data_ptr(),
                                               self._stream()), "forces_scatter")
        return out

    def energy_forces(self, positions, species, box):
        """(total energy, forces [N, 3]) of the whole system on this device."""
        row, nbr = self.neighbor_list(positions, box)
        A = self.density(positions, species, box, row, nbr)
        e, G = self.energy_grad(A, species.to(self.device, torch.int32), physical=True)
        g = self.edge_grad(positions, species, box, row, nbr, G)
        return e.sum(), self.forces_from_edges(row, nbr, g)

    # -- end to end ----------------------------------------------------------------
    def energy(self, positions, species, box, begin: int = 0, end: Optional[int] = None):
        """Per-atom energies of centres [begin, end) from positions."""
        N = positions.shape[0]
        end = N if end is None else int(end)
        row, nbr = self.neighbor_list(positions, box, begin, end)
        A = self.density(positions, species, box, row, nbr, begin)
        sp = species.to(self.device, torch.int32)[begin:end]
        return self.energy_from_density(A, sp, physical=True)


def ctypes_ref(tables):
    import ctypes
    return ctypes.byref(tables)
