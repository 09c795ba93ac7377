"""Drop-in evaluation of compiled ACE factorized schedules on B200.

``evaluate_factorized_schedule_torch`` keeps the signature and result of the
reference function ``ye3t/core/couplings.py:481-567``; ``evaluate_report``
is ``ACEFactorizedScheduleReport.evaluate`` (``ye3t/couplings/__init__.py:2574``).
Schedules are accepted as the reference's ``FactorizedCoefficientSchedule`` /
``TorchFactorizedCoefficientSchedule`` records (duck-typed) or as
:class:`~ye3t_b200.schedules.ScheduleRecord`; their device tables are packed
once per (schedule, device, dtype) and cached.
"""

from __future__ import annotations

import threading
import weakref

import numpy as np
import torch

from . import _native as nat
from .schedules import ScheduleRecord

__all__ = ["evaluate_factorized_schedule_torch", "evaluate_real_factorized_schedule_torch", "evaluate_report",
           "packed_schedule_tables"]

_CACHE = {}
_CACHE_LOCK = threading.Lock()


def _schedule_arrays(schedule):
    """(offsets, labels, block_m_indices, coeffs, component_count, block_count, basis_count, max_m)."""
    if hasattr(schedule, "block_m_indices") and hasattr(schedule, "term_component_index"):
        # TorchFactorizedCoefficientSchedule (couplings.py:259-335)
        off = schedule.component_offsets.detach().cpu().numpy().astype(np.int64)
        cli = schedule.component_label_index.detach().cpu().numpy().astype(np.int64)
        midx = schedule.block_m_indices.detach().cpu().numpy().astype(np.int64)
        coeffs = schedule.coeffs.detach().cpu().numpy()
        return (off, cli, midx, coeffs, int(schedule.component_count), int(schedule.block_count),
                int(schedule.basis_count), int(schedule.max_block_m_dim))
    rec = schedule if isinstance(schedule, ScheduleRecord) else ScheduleRecord.from_schedule(schedule)
    return (rec.component_offsets, rec.component_label_index, rec.block_m_indices(), np.asarray(rec.coeffs),
            rec.component_count, rec.block_count, rec.basis_count, rec.max_block_m_dim)


class _PackedSchedule:
    __slots__ = ("off", "cli", "midx", "coeffs_c", "coeffs_r", "comps", "blocks", "basis", "max_m", "terms",
                 "imag_max", "host", "slots")

    def slot_table(self, mdim, device):
        """Transposed table of the adjoint for block arrays of magnetic width
        ``mdim``: for every slot ``(label * blocks + j) * mdim + m`` the
        (term, component) pairs reading it, terms in order.  Built once per width."""
        hit = self.slots.get(mdim)
        if hit is None:
            off, cli, midx = self.host
            comp_of_term = np.repeat(np.arange(self.comps, dtype=np.int64), np.diff(off))
            T, B = midx.shape[0], self.blocks
            slot = ((cli[comp_of_term][:, None] * B + np.arange(B)[None, :]) * mdim + midx).reshape(-1)
            order = np.argsort(slot, kind="stable")  # by slot, then term
            S = self.basis * B * mdim
            counts = np.bincount(slot, minlength=S) if slot.size else np.zeros(S, dtype=np.int64)
            offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
            terms = np.repeat(np.arange(T, dtype=np.int64), B)[order]
            hit = (torch.as_tensor(offsets).to(device), torch.as_tensor(terms).to(device),
                   torch.as_tensor(comp_of_term[terms]).to(device))
            self.slots[mdim] = hit
        return hit


def packed_schedule_tables(schedule, device):
    """Device tables of one schedule, cached per (schedule object, device)."""
    key = (id(schedule), str(device))
    with _CACHE_LOCK:
        hit = _CACHE.get(key)
        if hit is not None and hit[0]() is schedule:
            return hit[1]
    off, cli, midx, coeffs, comps, blocks, basis, max_m = _schedule_arrays(schedule)
    p = _PackedSchedule()
    p.off = torch.as_tensor(off, dtype=torch.int64).to(device)
    p.cli = torch.as_tensor(cli, dtype=torch.int64).to(device)
    p.midx = torch.as_tensor(np.ascontiguousarray(midx).reshape(-1, blocks), dtype=torch.int64).to(device)
    c = np.asarray(coeffs)
    p.imag_max = float(np.max(np.abs(c.imag))) if (np.iscomplexobj(c) and c.size) else 0.0
    p.coeffs_c = torch.as_tensor(c.astype(np.complex128)).to(device)
    p.coeffs_r = torch.as_tensor(np.ascontiguousarray(c.real, dtype=np.float64)).to(device)
    p.comps, p.blocks, p.basis, p.max_m, p.terms = comps, blocks, basis, max_m, int(c.shape[0])
    p.host = (np.asarray(off, dtype=np.int64), np.asarray(cli, dtype=np.int64),
              np.ascontiguousarray(midx, dtype=np.int64).reshape(-1, blocks))
    p.slots = {}
    try:
        ref = weakref.ref(schedule)
    except TypeError:  # objects without weakref support: keep them alive in the cache
        ref = (lambda obj: (lambda: obj))(schedule)
    with _CACHE_LOCK:
        _CACHE[key] = (ref, p)
    return p


def evaluate_factorized_schedule_torch(block_values, schedule, *, backend="auto", validate=False):
    """Evaluate a factorized coefficient schedule on CUDA block values.

    ``block_values``: ``[batch, basis_count, block_count, max_block_m_dim]``
    with padded magnetic positions zero.  Returns ``[batch, component_count]``
    in the reference's value dtype: coefficients whose imaginary parts are all
    within 1e-12 are used as real numbers for real block values
    (``ye3t/core/couplings.py:508-516``).
    """
    backend = str(backend or "auto").strip().lower()
    if backend in ("cpp", "c++", "torch-cpp", "cpu-cpp", "torch", "pytorch", "reference"):
        raise ValueError(f"backend {backend!r} is a ye3t reference path; ye3t_b200 evaluates on CUDA only")
    if backend not in ("auto", "native", "cuda"):
        raise ValueError(f"Unknown factorized runtime backend: {backend!r}")
    bv = torch.as_tensor(block_values)
    dev = nat.require_cuda(bv, what="evaluate_factorized_schedule_torch")
    p = packed_schedule_tables(schedule, dev)
    if bv.ndim != 4:
        raise ValueError("block_values must have shape [batch, basis_count, block_count, max_block_m_dim].")
    if int(bv.shape[1]) < p.basis:
        raise ValueError("block_values basis dimension is smaller than schedule.basis_count.")
    if int(bv.shape[2]) != p.blocks:
        raise ValueError("block_values block dimension must equal schedule.block_count.")
    if int(bv.shape[3]) < p.max_m:
        raise ValueError("block_values magnetic dimension is smaller than schedule.max_block_m_dim.")
    if torch.is_complex(bv):
        value_dtype = bv.dtype
        coeffs = p.coeffs_c.to(value_dtype)
    elif p.imag_max > 1e-12:
        value_dtype = torch.complex128 if bv.dtype == torch.float64 else torch.complex64
        coeffs = p.coeffs_c.to(value_dtype)
    else:
        value_dtype = bv.dtype
        coeffs = p.coeffs_r.to(value_dtype)
    values = bv.to(value_dtype)
    if values.requires_grad and torch.is_grad_enabled():
        return _ScheduleEvaluate.apply(values, p, coeffs, bool(validate))
    return _schedule_forward(values.contiguous(), p, coeffs, validate)


def _schedule_forward(values, p, coeffs, validate):
    dev = values.device
    batch, basis, blocks, mdim = (int(s) for s in values.shape)
    out = torch.empty((batch, p.comps), dtype=values.dtype, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev) if validate else None
    nat.check(nat.lib().y3b_factorized_schedule_evaluate(
        nat.dtype_code(values.dtype), values.data_ptr(), batch, basis, blocks, mdim, p.off.data_ptr(),
        p.cli.data_ptr(), p.midx.data_ptr() if p.terms else 0, coeffs.data_ptr() if p.terms else 0, p.comps,
        p.terms, out.data_ptr(), nat.ptr(status), nat.stream_of(dev)), "evaluate_factorized_schedule_torch")
    if validate and int(status.item()):
        raise IndexError("evaluate_factorized_schedule_torch: schedule index out of range")
    return out


class _ScheduleEvaluate(torch.autograd.Function):
    """First-order autograd of the schedule evaluation: the backward is the
    vector-Jacobian product on the GPU (``y3b_factorized_schedule_adjoint``),
    gathered per block-value slot through the transposed table."""

    @staticmethod
    def forward(ctx, values, p, coeffs, validate):
        values = values.contiguous()
        ctx.save_for_backward(values, coeffs)
        ctx.p = p
        return _schedule_forward(values, p, coeffs, validate)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, adj):
        values, coeffs = ctx.saved_tensors
        p = ctx.p
        batch, basis, blocks, mdim = (int(s) for s in values.shape)
        slot_off, slot_term, slot_comp = p.slot_table(mdim, values.device)
        grad = torch.empty_like(values)
        adj = adj.to(values.dtype).contiguous()
        nat.check(nat.lib().y3b_factorized_schedule_adjoint(
            nat.dtype_code(values.dtype), adj.data_ptr(), values.data_ptr(), batch, basis, blocks, mdim,
            p.midx.data_ptr() if p.terms else 0, coeffs.data_ptr() if p.terms else 0, p.comps, p.terms,
            slot_off.data_ptr(), slot_term.data_ptr() if p.terms else 0, slot_comp.data_ptr() if p.terms else 0,
            grad.data_ptr(), None, nat.stream_of(values.device)), "evaluate_factorized_schedule_torch backward")
        return grad, None, None, None


def evaluate_report(report, block_values, *, target_L, backend="auto"):
    """``ACEFactorizedScheduleReport.evaluate`` on CUDA (``ye3t/couplings/__init__.py:2574-2591``)."""
    target_L = int(target_L)
    schedules = getattr(report, "schedules_by_target", None) or getattr(report, "schedules_by_L")
    if target_L not in schedules:
        raise ValueError("target_L is not present in this ACE schedule report.")
    return evaluate_factorized_schedule_torch(block_values, schedules[target_L], backend=backend)


# ---------------------------------------------------------------------------
# Real-tesseral schedules (ye3t/core/couplings.py:337-478, 570-610): the same
# contraction with real block values, real coefficients and real component
# indices (block_real_tuples), so the same native evaluator runs it in f32/f64.
# ---------------------------------------------------------------------------
def _real_schedule_arrays(schedule):
    """(offsets, labels, block_real_indices, coeffs, component_count, block_count, basis_count, max_dim)."""
    if hasattr(schedule, "block_real_indices") and hasattr(schedule, "term_component_index"):
        # TorchRealFactorizedCoefficientSchedule (couplings.py:398-478)
        off = schedule.component_offsets.detach().cpu().numpy().astype(np.int64)
        cli = schedule.component_label_index.detach().cpu().numpy().astype(np.int64)
        ridx = schedule.block_real_indices.detach().cpu().numpy().astype(np.int64)
        coeffs = schedule.coeffs.detach().cpu().numpy().astype(np.float64)
        return (off, cli, ridx, coeffs, int(schedule.component_count), int(schedule.block_count),
                int(schedule.basis_count), int(schedule.max_block_m_dim))
    # RealFactorizedCoefficientSchedule (couplings.py:337-397) or a record with its fields
    off = np.asarray(schedule.component_offsets, dtype=np.int64)
    cli = np.asarray(schedule.component_label_index, dtype=np.int64)
    blocks = int(schedule.block_count)
    ridx = np.asarray(schedule.block_real_tuples, dtype=np.int64).reshape(-1, blocks)
    coeffs = np.asarray(schedule.coeffs, dtype=np.float64)
    block_L = np.asarray(schedule.block_L_by_label(dtype=np.int64)) if hasattr(schedule, "block_L_by_label") \
        else np.asarray(schedule.block_L, dtype=np.int64)
    max_dim = int(2 * int(block_L.max()) + 1) if block_L.size else 0
    basis = int(schedule.basis_count)
    return off, cli, ridx, coeffs, int(cli.shape[0]), blocks, basis, max_dim


_REAL_CACHE = {}


def evaluate_real_factorized_schedule_torch(block_values, schedule, *, backend="auto", validate=False):
    """Evaluate a real-tesseral factorized schedule on CUDA block values.

    Mirrors ``ye3t/core/couplings.py:570-610``: ``block_values`` are real
    ``[batch, basis_count, block_count, max_block_m_dim]``; the result is
    ``[batch, component_count]`` in the block dtype (float32 or float64),
    ``out[b, c] = sum_t coeff_t prod_j bv[b, label_c, j, real_idx[t, j]]``
    with products in block order and sums in term order.
    """
    selected = str(backend or "auto").strip().lower()
    if selected in ("torch", "pytorch", "reference"):
        raise ValueError(f"backend {backend!r} is a ye3t reference path; ye3t_b200 evaluates on CUDA only")
    if selected not in ("auto", "native", "cuda", ""):
        raise ValueError(f"Unknown real factorized runtime backend: {backend!r}")
    bv = torch.as_tensor(block_values)
    if torch.is_complex(bv):
        raise ValueError("Real factorized schedule evaluation requires real block values.")
    dev = nat.require_cuda(bv, what="evaluate_real_factorized_schedule_torch")
    if bv.ndim != 4:
        raise ValueError("block_values must have shape [batch, basis_count, block_count, max_block_m_dim].")
    key = (id(schedule), str(dev))
    with _CACHE_LOCK:
        hit = _REAL_CACHE.get(key)
    if hit is None or hit[0]() is not schedule:
        off, cli, ridx, coeffs, comps, blocks, basis, max_dim = _real_schedule_arrays(schedule)
        tab = {"off": torch.as_tensor(off).to(dev), "cli": torch.as_tensor(cli).to(dev),
               "ridx": torch.as_tensor(np.ascontiguousarray(ridx)).to(dev),
               "coeffs": torch.as_tensor(np.ascontiguousarray(coeffs)).to(dev), "comps": comps, "blocks": blocks,
               "basis": basis, "max_dim": max_dim, "terms": int(coeffs.shape[0])}
        try:
            ref = weakref.ref(schedule)
        except TypeError:
            ref = (lambda obj: (lambda: obj))(schedule)
        with _CACHE_LOCK:
            _REAL_CACHE[key] = (ref, tab)
    else:
        tab = hit[1]
    if int(bv.shape[1]) < tab["basis"]:
        raise ValueError("block_values basis dimension is smaller than schedule.basis_count.")
    if int(bv.shape[2]) != tab["blocks"]:
        raise ValueError("block_values block dimension must equal schedule.block_count.")
    if int(bv.shape[3]) < tab["max_dim"]:
        raise ValueError("block_values real-component dimension is smaller than schedule.max_block_m_dim.")
    if bv.dtype not in (torch.float32, torch.float64):
        raise TypeError("block_values must be float32 or float64")
    values = bv.contiguous()
    coeffs = tab["coeffs"].to(values.dtype)
    batch, basis, blocks, mdim = (int(v) for v in values.shape)
    out = torch.empty((batch, tab["comps"]), dtype=values.dtype, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev) if validate else None
    nat.check(nat.lib().y3b_factorized_schedule_evaluate(
        nat.dtype_code(values.dtype), values.data_ptr(), batch, basis, blocks, mdim, tab["off"].data_ptr(),
        tab["cli"].data_ptr(), tab["ridx"].data_ptr() if tab["terms"] else 0,
        coeffs.data_ptr() if tab["terms"] else 0, tab["comps"], tab["terms"], out.data_ptr(), nat.ptr(status),
        nat.stream_of(dev)), "evaluate_real_factorized_schedule_torch")
    if validate and int(status.item()):
        raise IndexError("evaluate_real_factorized_schedule_torch: schedule index out of range")
    return out
