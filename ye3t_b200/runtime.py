"""``ye3t.runtime``-shaped operators backed by the sm_100a library.

Same names, argument meanings and result layouts as the reference wrappers in
``ye3t/runtime/execution_plan.py`` (cited per function).  ``backend`` accepts
``"auto"`` and ``"native"`` (both run the CUDA library) and rejects
``"reference"``: this package has no CPU or pure-torch fallback, and tensors
must live on a CUDA device.

Index checks run on the device: out-of-range centres or indices set a status
word and contribute zero.  With ``YE3T_B200_VALIDATE=1`` (or
``validate=True``) each call synchronises and raises ``IndexError`` when the
status word is set, matching the reference CPU path's eager checks
(``execution_plan_torch.cpp:1511-1515``).
"""

from __future__ import annotations

import os

import torch

from . import _native as nat

__all__ = [
    "cheb_exp_cos_radial_table_with_derivative",
    "spherical_harmonics_table_with_derivative",
    "density_accumulate",
    "density_accumulate_adjoint",
    "symmetric_power_monomial_contraction",
    "symmetric_power_shared_monomial_contraction",
    "scheduled_radial_angular_channels_with_derivative",
    "plain_site_basis_product_with_derivative",
    "plain_site_basis_product_adjoint",
    "symmetric_power_table_contraction",
    "pace_radial_channel_contraction_with_derivative",
    "native_execution_plan_capabilities",
]


def _check_backend(backend, allowed=("auto", "native")):
    backend = str(backend)
    if backend == "reference":
        raise ValueError("ye3t_b200 has no reference (CPU / pure torch) path; backend='reference' is the "
                         "ye3t package's own implementation")
    if backend not in allowed:
        raise ValueError(f"backend must be one of {allowed}, got {backend!r}")


def _validate_default(validate):
    if validate is None:
        return os.environ.get("YE3T_B200_VALIDATE", "0") not in ("", "0", "false", "False")
    return bool(validate)


def _status(device):
    return torch.zeros(1, dtype=torch.int32, device=device)


def _raise_on_status(status, what):
    v = int(status.item())
    if v & nat.STATUS_INDEX_RANGE:
        raise IndexError(f"{what}: index out of range")
    if v:
        raise RuntimeError(f"{what}: device status {v}")


# ---------------------------------------------------------------------------
def cheb_exp_cos_radial_table_with_derivative(radii, cutoffs, lambdas, maximum_radial_index, backend="auto"):
    """ChebExpCos radial table and d/dr; ``ye3t/runtime/execution_plan.py:7298``.

    Returns ``(values, derivatives)`` of shape ``[E, maximum_radial_index + 1]``.
    """
    _check_backend(backend)
    kmax = int(maximum_radial_index)
    if kmax < 0:
        raise ValueError("maximum_radial_index must be non-negative")
    radii = torch.as_tensor(radii)
    dev = nat.require_cuda(radii, what="cheb_exp_cos_radial_table_with_derivative")
    if radii.dtype not in (torch.float32, torch.float64):
        raise TypeError("radii must be float32 or float64")
    cutoffs = torch.as_tensor(cutoffs, dtype=radii.dtype, device=dev).expand_as(radii).contiguous()
    lambdas = torch.as_tensor(lambdas, dtype=radii.dtype, device=dev).expand_as(radii).contiguous()
    r = radii.contiguous().reshape(-1)
    E = r.numel()
    val = torch.empty((E, kmax + 1), dtype=radii.dtype, device=dev)
    der = torch.empty_like(val)
    nat.check(nat.lib().y3b_cheb_exp_cos_radial_table(nat.dtype_code(radii.dtype), r.data_ptr(),
                                                       cutoffs.data_ptr(), lambdas.data_ptr(), E, kmax,
                                                       val.data_ptr(), der.data_ptr(), nat.stream_of(dev)),
              "cheb_exp_cos_radial_table_with_derivative")
    return val, der


def spherical_harmonics_table_with_derivative(edge_vectors, maximum_angular_momentum, *, real_output=False,
                                              epsilon=1.0e-12, backend="auto"):
    """Packed harmonics for all ``l <= lmax`` and Cartesian derivatives.

    ``ye3t/runtime/execution_plan.py:7479``: values ``[E, (lmax+1)^2]``,
    derivatives ``[E, (lmax+1)^2, 3]``; complex Condon-Shortley unless
    ``real_output``.
    """
    _check_backend(backend)
    lmax = int(maximum_angular_momentum)
    if lmax < 0:
        raise ValueError("maximum_angular_momentum must be non-negative")
    v = torch.as_tensor(edge_vectors)
    dev = nat.require_cuda(v, what="spherical_harmonics_table_with_derivative")
    if v.dtype not in (torch.float32, torch.float64) or v.shape[-1] != 3:
        raise ValueError("edge_vectors must be real [E, 3]")
    v = v.contiguous().reshape(-1, 3)
    E = v.shape[0]
    W = (lmax + 1) ** 2
    out_dtype = v.dtype if real_output else (torch.complex128 if v.dtype == torch.float64 else torch.complex64)
    val = torch.empty((E, W), dtype=out_dtype, device=dev)
    der = torch.empty((E, W, 3), dtype=out_dtype, device=dev)
    nat.check(nat.lib().y3b_spherical_harmonics_table(nat.dtype_code(v.dtype), v.data_ptr(), E, lmax,
                                                       int(bool(real_output)), float(epsilon), val.data_ptr(),
                                                       der.data_ptr(), nat.stream_of(dev)),
              "spherical_harmonics_table_with_derivative")
    return val, der


def _index_range(t, n, what):
    if t.numel() and (int(t.min()) < 0 or int(t.max()) >= n):
        raise IndexError(f"{what}: index out of range")


def scheduled_radial_angular_channels_with_derivative(radial_values, radial_derivatives, angular_values,
                                                      angular_derivatives, radial_directions, edge_types,
                                                      channel_radial_indices, channel_angular_indices,
                                                      channel_types, channel_scales, backend="auto"):
    """Fixed radial x angular channel schedule and its analytic derivatives.

    ``ye3t/runtime/execution_plan.py:7675`` (composition :7036-7080): returns
    ``values [E, C]`` and ``derivatives [E, C, 3]`` with the reference's
    operation order and rounding (real dtypes).
    """
    _check_backend(backend)
    rv = torch.as_tensor(radial_values)
    dev = nat.require_cuda(rv, what="scheduled_radial_angular_channels_with_derivative")
    if rv.dtype not in (torch.float32, torch.float64):
        raise ValueError("scheduled radial-angular channels are real")
    rd, av, ad, dr, cs = (torch.as_tensor(v, dtype=rv.dtype, device=dev).contiguous()
                          for v in (radial_derivatives, angular_values, angular_derivatives, radial_directions,
                                    channel_scales))
    et, cr, ca, ct = (torch.as_tensor(v, dtype=torch.int64, device=dev).reshape(-1).contiguous()
                      for v in (edge_types, channel_radial_indices, channel_angular_indices, channel_types))
    rv = rv.contiguous()
    if rv.ndim != 2 or rd.shape != rv.shape or av.ndim != 2 or ad.shape != (*av.shape, 3):
        raise ValueError("radial tables must be [E, K] and angular tables [E, A] / [E, A, 3]")
    E, K, A, C = int(rv.shape[0]), int(rv.shape[1]), int(av.shape[1]), int(cr.numel())
    if av.shape[0] != E or dr.shape != (E, 3) or et.numel() != E:
        raise ValueError("edge tables disagree on the edge count")
    if ca.numel() != C or ct.numel() != C or cs.numel() != C:
        raise ValueError("channel tables must have one entry per channel")
    _index_range(cr, K, "channel_radial_indices")
    _index_range(ca, A, "channel_angular_indices")
    val = torch.empty((E, C), dtype=rv.dtype, device=dev)
    der = torch.empty((E, C, 3), dtype=rv.dtype, device=dev)
    nat.check(nat.lib().y3b_scheduled_radial_angular_channels(
        nat.dtype_code(rv.dtype), rv.data_ptr(), rd.data_ptr(), K, av.data_ptr(), ad.data_ptr(), A, dr.data_ptr(),
        et.data_ptr(), E, cr.data_ptr(), ca.data_ptr(), ct.data_ptr(), cs.data_ptr(), C, val.data_ptr(),
        der.data_ptr(), None, nat.stream_of(dev)), "scheduled_radial_angular_channels_with_derivative")
    return val, der


def plain_site_basis_product_with_derivative(radial_values, radial_derivatives, angular_values,
                                             angular_derivatives, prefactors, prefactor_derivatives_center,
                                             prefactor_derivatives_neighbor, radial_directions, term_groups,
                                             term_channels, channel_count, backend="auto"):
    """Grouped plain source channels and analytic edge derivatives.

    ``ye3t/runtime/execution_plan.py:7582`` (composition :7082-7155): returns
    ``(edge_values [E, C], edge_derivatives [E, C, 3], charge_center [E, C],
    charge_neighbor [E, C])`` in the dtype of ``radial_values`` (real or
    complex); term channels must be distinct.
    """
    _check_backend(backend)
    rv = torch.as_tensor(radial_values)
    dev = nat.require_cuda(rv, what="plain_site_basis_product_with_derivative")
    rd, av, ad, p, pc, pn, dr = (torch.as_tensor(v, dtype=rv.dtype, device=dev).contiguous()
                                 for v in (radial_derivatives, angular_values, angular_derivatives, prefactors,
                                           prefactor_derivatives_center, prefactor_derivatives_neighbor,
                                           radial_directions))
    tg, tc = (torch.as_tensor(v, dtype=torch.int64, device=dev).reshape(-1).contiguous()
              for v in (term_groups, term_channels))
    rv = rv.contiguous()
    C = int(channel_count)
    if rv.ndim != 2:
        raise ValueError("radial_values must be [group, E]")
    G, E = int(rv.shape[0]), int(rv.shape[1])
    T = int(tg.numel())
    if rd.shape != rv.shape or p.shape != rv.shape or pc.shape != rv.shape or pn.shape != rv.shape:
        raise ValueError("radial and prefactor tables must be [group, E]")
    if av.shape != (T, E) or ad.shape != (T, E, 3) or dr.shape != (E, 3) or tc.numel() != T:
        raise ValueError("angular tables must be [term, E] / [term, E, 3] and directions [E, 3]")
    _index_range(tg, G, "term_groups")
    _index_range(tc, C, "term_channels")
    outs = (torch.empty((E, C), dtype=rv.dtype, device=dev), torch.empty((E, C, 3), dtype=rv.dtype, device=dev),
            torch.empty((E, C), dtype=rv.dtype, device=dev), torch.empty((E, C), dtype=rv.dtype, device=dev))
    nat.check(nat.lib().y3b_plain_site_basis_product(
        nat.dtype_code(rv.dtype), rv.data_ptr(), rd.data_ptr(), G, av.data_ptr(), ad.data_ptr(), T, p.data_ptr(),
        pc.data_ptr(), pn.data_ptr(), dr.data_ptr(), E, tg.data_ptr(), tc.data_ptr(), C,
        *(o.data_ptr() for o in outs), None, nat.stream_of(dev)), "plain_site_basis_product_with_derivative")
    return outs


def plain_site_basis_product_adjoint(radial_values, radial_derivatives, angular_values, angular_derivatives,
                                     prefactors, prefactor_derivatives_center, prefactor_derivatives_neighbor,
                                     radial_directions, edge_weights, edge_weight_derivatives, term_groups,
                                     term_channels, edge_adjoint, backend="auto"):
    """Edge adjoints of the plain site-basis product; ``ye3t/runtime/execution_plan.py:7790``.

    Returns ``(edge_position_adjoint [E, 3], edge_charge_center [E],
    edge_charge_neighbor [E])`` (composition :7158-7220), one thread per edge.
    """
    _check_backend(backend)
    rv = torch.as_tensor(radial_values)
    dev = nat.require_cuda(rv, what="plain_site_basis_product_adjoint")
    rd, av, ad, p, pc, pn, dr, w, dw, adj = (
        torch.as_tensor(v, dtype=rv.dtype, device=dev).contiguous()
        for v in (radial_derivatives, angular_values, angular_derivatives, prefactors, prefactor_derivatives_center,
                  prefactor_derivatives_neighbor, radial_directions, edge_weights, edge_weight_derivatives,
                  edge_adjoint))
    tg, tc = (torch.as_tensor(v, dtype=torch.int64, device=dev).reshape(-1).contiguous()
              for v in (term_groups, term_channels))
    rv = rv.contiguous()
    if rv.ndim != 2:
        raise ValueError("radial_values must be [group, E]")
    G, E = int(rv.shape[0]), int(rv.shape[1])
    T = int(tg.numel())
    if rd.shape != rv.shape or p.shape != rv.shape or pc.shape != rv.shape or pn.shape != rv.shape:
        raise ValueError("radial and prefactor tables must be [group, E]")
    if av.shape != (T, E) or ad.shape != (T, E, 3) or dr.shape != (E, 3) or tc.numel() != T:
        raise ValueError("angular tables must be [term, E] / [term, E, 3] and directions [E, 3]")
    if w.reshape(-1).numel() != E or dw.shape != (E, 3) or adj.ndim != 2 or adj.shape[0] != E:
        raise ValueError("edge weights must be [E] / [E, 3] and the edge adjoint [E, channels]")
    C = int(adj.shape[1])
    _index_range(tg, G, "term_groups")
    _index_range(tc, C, "term_channels")
    pos = torch.empty((E, 3), dtype=rv.dtype, device=dev)
    cc = torch.empty((E,), dtype=rv.dtype, device=dev)
    cn = torch.empty((E,), dtype=rv.dtype, device=dev)
    nat.check(nat.lib().y3b_plain_site_basis_product_adjoint(
        nat.dtype_code(rv.dtype), rv.data_ptr(), rd.data_ptr(), G, av.data_ptr(), ad.data_ptr(), T, p.data_ptr(),
        pc.data_ptr(), pn.data_ptr(), dr.data_ptr(), w.data_ptr(), dw.data_ptr(), E, tg.data_ptr(), tc.data_ptr(),
        C, adj.data_ptr(), pos.data_ptr(), cc.data_ptr(), cn.data_ptr(), None, nat.stream_of(dev)),
        "plain_site_basis_product_adjoint")
    return pos, cc, cn


# ---------------------------------------------------------------------------
def _density_forward(edge_values, centers, atom_count, validate):
    dev = nat.require_cuda(edge_values, centers, what="density_accumulate")
    ev = edge_values.contiguous()
    E = ev.shape[0]
    C = 1
    for extent in ev.shape[1:]:
        C *= int(extent)
    centers = centers.to(device=dev, dtype=torch.int64).contiguous().reshape(-1)
    if centers.numel() != E:
        raise ValueError("centers must have one entry per edge row")
    out = torch.empty((int(atom_count),) + tuple(ev.shape[1:]), dtype=ev.dtype, device=dev)
    lib = nat.lib()
    ws_bytes = int(lib.y3b_density_accumulate_workspace_bytes(E, int(atom_count)))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    status = _status(dev)
    nat.check(lib.y3b_density_accumulate(nat.dtype_code(ev.dtype), ev.data_ptr(), centers.data_ptr(), E, C,
                                         int(atom_count), ws.data_ptr(), ws_bytes, out.data_ptr(),
                                         status.data_ptr(), nat.stream_of(dev)), "density_accumulate")
    if validate:
        _raise_on_status(status, "density_accumulate")
    return out


def _density_adjoint(atomic_adjoint, centers, validate):
    dev = nat.require_cuda(atomic_adjoint, centers, what="density_accumulate_adjoint")
    adj = atomic_adjoint.contiguous()
    centers = centers.to(device=dev, dtype=torch.int64).contiguous().reshape(-1)
    E = centers.numel()
    C = 1
    for extent in adj.shape[1:]:
        C *= int(extent)
    out = torch.empty((E,) + tuple(adj.shape[1:]), dtype=adj.dtype, device=dev)
    status = _status(dev)
    nat.check(nat.lib().y3b_density_accumulate_adjoint(nat.dtype_code(adj.dtype), adj.data_ptr(),
                                                        centers.data_ptr(), E, C, adj.shape[0], out.data_ptr(),
                                                        status.data_ptr(), nat.stream_of(dev)),
              "density_accumulate_adjoint")
    if validate:
        _raise_on_status(status, "density_accumulate_adjoint")
    return out


class _DensityAccumulate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, edge_values, centers, atom_count, validate):
        ctx.save_for_backward(centers)
        ctx.validate = validate
        return _density_forward(edge_values, centers, atom_count, validate)

    @staticmethod
    def backward(ctx, grad):
        (centers,) = ctx.saved_tensors
        return _density_adjoint(grad, centers, ctx.validate), None, None, None


def density_accumulate(edge_values, centers, atom_count, *, backend="auto", validate=None):
    """``A[centers[e]] += edge_values[e]``; ``ye3t/runtime/execution_plan.py:7913``.

    Deterministic (no floating-point atomics).  Differentiable in
    ``edge_values`` through :func:`density_accumulate_adjoint`.
    """
    _check_backend(backend, ("auto", "native", "deterministic"))
    edge_values = torch.as_tensor(edge_values)
    centers = torch.as_tensor(centers, device=edge_values.device)
    validate = _validate_default(validate)
    if edge_values.requires_grad and torch.is_grad_enabled():
        return _DensityAccumulate.apply(edge_values, centers, int(atom_count), validate)
    return _density_forward(edge_values, centers, int(atom_count), validate)


def density_accumulate_adjoint(atomic_adjoint, centers, *, backend="auto", validate=None):
    """Gather centre rows back to edge rows; ``ye3t/runtime/execution_plan.py:7987``."""
    _check_backend(backend, ("auto", "native", "deterministic"))
    atomic_adjoint = torch.as_tensor(atomic_adjoint)
    centers = torch.as_tensor(centers, device=atomic_adjoint.device)
    return _density_adjoint(atomic_adjoint, centers, _validate_default(validate))


# ---------------------------------------------------------------------------
def _sympow_forward(x2, counts, offsets, values, out_dim):
    out = torch.empty((x2.shape[0], out_dim), dtype=x2.dtype, device=x2.device)
    nat.check(nat.lib().y3b_symmetric_power_monomial(nat.dtype_code(x2.dtype), x2.data_ptr(), x2.shape[0],
                                                      x2.shape[1], counts.data_ptr(), offsets.data_ptr(),
                                                      values.data_ptr(), int(counts.shape[0]), out_dim,
                                                      out.data_ptr(), nat.stream_of(x2.device)),
              "symmetric_power_monomial_contraction")
    return out


def _sympow_adjoint(adj, x2, counts, indices, values, out_dim):
    grad = torch.empty_like(x2)
    status = _status(x2.device)
    nat.check(nat.lib().y3b_symmetric_power_monomial_adjoint(
        nat.dtype_code(x2.dtype), adj.data_ptr(), x2.data_ptr(), x2.shape[0], x2.shape[1], counts.data_ptr(),
        indices.data_ptr(), values.data_ptr(), int(counts.shape[0]), out_dim, grad.data_ptr(), status.data_ptr(),
        nat.stream_of(x2.device)), "symmetric_power_monomial_adjoint")
    _raise_on_status(status, "symmetric_power_monomial_adjoint")
    return grad


class _SymmetricPowerMonomial(torch.autograd.Function):
    """First-order autograd of the grouped table (execution_plan.py:4960-4990)."""

    @staticmethod
    def forward(ctx, x2, counts, offsets, indices, values, out_dim):
        ctx.save_for_backward(x2, counts, indices, values)
        ctx.out_dim = out_dim
        return _sympow_forward(x2, counts, offsets, values, out_dim)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, adj):
        x2, counts, indices, values = ctx.saved_tensors
        return _sympow_adjoint(adj.contiguous(), x2, counts, indices, values, ctx.out_dim), None, None, None, None, None


def symmetric_power_monomial_contraction(input, monomial_counts, output_offsets, output_indices,
                                         monomial_values, *, backend="auto"):
    """Grouped symmetric-power table contraction; ``ye3t/runtime/execution_plan.py:11998``.

    Differentiable with respect to ``input`` (first order): the backward is
    the table's vector-Jacobian product on the GPU
    (``y3b_symmetric_power_monomial_adjoint``).
    """
    _check_backend(backend)
    x = torch.as_tensor(input)
    dev = nat.require_cuda(x, what="symmetric_power_monomial_contraction")
    if x.ndim < 1:
        raise ValueError("symmetric-power input requires a feature axis")
    in_dim = int(x.shape[-1])
    counts = torch.as_tensor(monomial_counts, dtype=torch.int64, device=dev).contiguous()
    offsets = torch.as_tensor(output_offsets, dtype=torch.int64, device=dev).reshape(-1).contiguous()
    indices = torch.as_tensor(output_indices, dtype=torch.int64, device=dev).reshape(-1).contiguous()
    values = torch.as_tensor(monomial_values, dtype=x.dtype, device=dev).reshape(-1).contiguous()
    if counts.ndim != 2 or int(counts.shape[1]) != in_dim:
        raise ValueError("monomial_counts must have shape [term, input_dimension]")
    if int(indices.numel()) != int(counts.shape[0]) or int(values.numel()) != int(counts.shape[0]):
        raise ValueError("output_indices / monomial_values length must match the term count")
    out_dim = int(offsets.numel()) - 1
    x2 = x.contiguous().reshape(-1, in_dim)
    if x2.requires_grad and torch.is_grad_enabled():
        out = _SymmetricPowerMonomial.apply(x2, counts, offsets, indices, values, out_dim)
    else:
        out = _sympow_forward(x2, counts, offsets, values, out_dim)
    return out.reshape(*x.shape[:-1], out_dim)


def symmetric_power_shared_monomial_contraction(input, monomial_counts, output_offsets, coefficient_terms,
                                                coefficient_outputs, coefficient_values, *, backend="auto"):
    """Shared-monomial symmetric-power contraction; ``ye3t/runtime/execution_plan.py:12502``.

    Unique monomials ``prod_i x_i^counts[m, i]`` weighted by sparse
    coefficients: ``out[..., o] = sum_{t in [offsets[o], offsets[o+1])}
    values[t] * monomial[terms[t]]``.  The table checks (lengths, index
    ranges) and their messages follow the reference's
    ``symmetric_power_shared_monomial_reference`` (:12100-12160).
    """
    _check_backend(backend)
    x = torch.as_tensor(input)
    dev = nat.require_cuda(x, what="symmetric_power_shared_monomial_contraction")
    if x.ndim < 1:
        raise ValueError("symmetric-power input requires a feature axis")
    in_dim = int(x.shape[-1])
    counts = torch.as_tensor(monomial_counts, dtype=torch.int64, device=dev).contiguous()
    offsets = torch.as_tensor(output_offsets, dtype=torch.int64, device=dev).reshape(-1).contiguous()
    terms = torch.as_tensor(coefficient_terms, dtype=torch.int64, device=dev).reshape(-1).contiguous()
    outputs = torch.as_tensor(coefficient_outputs, dtype=torch.int64, device=dev).reshape(-1)
    values = torch.as_tensor(coefficient_values, dtype=x.dtype, device=dev).reshape(-1).contiguous()
    if counts.ndim != 2 or int(counts.shape[1]) != in_dim:
        raise ValueError("monomial_counts must have shape [monomial, input_dimension]")
    n_coef = int(terms.numel())
    if int(outputs.numel()) != n_coef:
        raise ValueError("coefficient_outputs length must match coefficient_terms")
    if int(values.numel()) != n_coef:
        raise ValueError("coefficient_values length must match coefficient_terms")
    if int(offsets.numel()) < 1:
        raise ValueError("output_offsets must contain at least one entry")
    out_dim = int(offsets.numel()) - 1
    if n_coef:
        if int(terms.min()) < 0:
            raise ValueError("coefficient_terms must be nonnegative")
        if int(terms.max()) >= int(counts.shape[0]):
            raise ValueError("coefficient_terms contains an invalid monomial")
        if int(outputs.min()) < 0:
            raise ValueError("coefficient_outputs must be nonnegative")
        if int(outputs.max()) >= out_dim:
            raise ValueError("coefficient_outputs contains an invalid output")
    x2 = x.contiguous().reshape(-1, in_dim)
    if x2.requires_grad and torch.is_grad_enabled():
        out = _SharedMonomial.apply(x2, counts, offsets, terms, outputs, values, out_dim)
    else:
        out = _shared_forward(x2, counts, offsets, terms, values, out_dim)
    return out.reshape(*x.shape[:-1], out_dim)


def _shared_forward(x2, counts, offsets, terms, values, out_dim):
    dev, n_coef = x2.device, int(terms.numel())
    out = torch.empty((x2.shape[0], out_dim), dtype=x2.dtype, device=dev)
    status = _status(dev)
    nat.check(nat.lib().y3b_symmetric_power_shared_monomial(
        nat.dtype_code(x2.dtype), x2.data_ptr(), x2.shape[0], x2.shape[1], counts.data_ptr() if counts.numel() else 0,
        int(counts.shape[0]), offsets.data_ptr(), out_dim, terms.data_ptr() if n_coef else 0,
        values.data_ptr() if n_coef else 0, n_coef, out.data_ptr(), status.data_ptr(), nat.stream_of(dev)),
        "symmetric_power_shared_monomial_contraction")
    _raise_on_status(status, "symmetric_power_shared_monomial_contraction")
    return out


class _SharedMonomial(torch.autograd.Function):
    """First-order autograd of the shared-monomial form: its backward is the
    grouped table's vector-Jacobian product with one row per coefficient (the
    coefficient's monomial exponents, its output index)."""

    @staticmethod
    def forward(ctx, x2, counts, offsets, terms, outputs, values, out_dim):
        ctx.save_for_backward(x2, counts, terms, outputs, values)
        ctx.out_dim = out_dim
        return _shared_forward(x2, counts, offsets, terms, values, out_dim)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, adj):
        x2, counts, terms, outputs, values = ctx.saved_tensors
        rows = counts.index_select(0, terms).contiguous()
        grad = _sympow_adjoint(adj.contiguous(), x2, rows, outputs.contiguous(), values, ctx.out_dim)
        return grad, None, None, None, None, None, None


def symmetric_power_table_contraction(input, table, *, backend="auto"):
    """Contract with a :class:`~ye3t_b200.schedules.SymPowerTable` (grouped plan table).

    Same role as ``symmetric_power_product_plan_contraction``
    (``ye3t/runtime/symmetric_power.py:879``) once the plan has been lowered.
    """
    x = torch.as_tensor(input)
    vals = torch.as_tensor(table.monomial_value)
    if not torch.is_complex(x) and torch.is_complex(vals):
        if vals.numel() and float(vals.imag.abs().max()) > 1e-12:
            x = x.to(torch.complex128 if x.dtype == torch.float64 else torch.complex64)
        else:
            vals = vals.real
    return symmetric_power_monomial_contraction(x, table.monomial_counts, table.output_offsets,
                                                table.output_index, vals, backend=backend)


def pace_radial_channel_contraction_with_derivative(values, derivatives, coefficients, backend="auto"):
    """Dense radial channel mixing; ``ye3t/runtime/csrc/ye3t_runtime_core.h:74-85``.

    ``values``/``derivatives`` ``[P, I]``, ``coefficients`` row-major ``[O, I]``;
    returns ``(values @ W^T, derivatives @ W^T)`` as ``[P, O]`` (products and
    sums in input order, as the reference loop).  float32 or float64.
    """
    _check_backend(backend)
    x = torch.as_tensor(values)
    dev = nat.require_cuda(x, what="pace_radial_channel_contraction_with_derivative")
    if x.dtype not in (torch.float32, torch.float64) or x.dim() != 2:
        raise ValueError("values must be real [P, I]")
    dx = torch.as_tensor(derivatives, device=dev)
    W = torch.as_tensor(coefficients, device=dev)
    if dx.shape != x.shape or dx.dtype != x.dtype or W.dtype != x.dtype or W.dim() != 2 or W.shape[1] != x.shape[1]:
        raise ValueError("derivatives must match values and coefficients must be [O, I] of the same dtype")
    if W.shape[0] <= 0 or x.shape[1] <= 0:
        raise ValueError("empty radial contraction")
    x, dx, W = x.contiguous(), dx.contiguous(), W.contiguous()
    P, I = x.shape
    O = W.shape[0]
    out = torch.empty((P, O), dtype=x.dtype, device=dev)
    dout = torch.empty_like(out)
    nat.check(nat.lib().y3b_radial_channel_contraction(nat.dtype_code(x.dtype), x.data_ptr(), dx.data_ptr(),
                                                       W.data_ptr(), P, I, O, out.data_ptr(), dout.data_ptr(),
                                                       nat.stream_of(dev)),
              "pace_radial_channel_contraction_with_derivative")
    return out, dout


def native_execution_plan_capabilities():
    """Capability report; the analogue of ``ye3t/runtime/execution_plan.py:6118``."""
    try:
        lib = nat.lib()
        loaded, abi, err = True, int(lib.y3b_abi_version()), None
    except Exception as exc:  # noqa: BLE001 - report, do not hide
        loaded, abi, err = False, None, str(exc)
    return {
        "library": nat.LIB_PATH,
        "loaded": loaded,
        "abi_version": abi,
        "error": err,
        "cuda": True,
        "cpu": False,
        "architecture": "sm_100a",
        "ops": {
            "cheb_exp_cos_radial_table_with_derivative": ["float32", "float64"],
            "spherical_harmonics_table_with_derivative": ["float32", "float64"],
            "density_accumulate": ["float32", "float64", "complex64", "complex128"],
            "density_accumulate_adjoint": ["float32", "float64", "complex64", "complex128"],
            "symmetric_power_monomial": ["float32", "float64", "complex64", "complex128"],
            "symmetric_power_shared_monomial": ["float32", "float64", "complex64", "complex128"],
            "scheduled_radial_angular_channels_with_derivative": ["float32", "float64"],
            "plain_site_basis_product_with_derivative": ["float32", "float64", "complex64", "complex128"],
            "plain_site_basis_product_adjoint": ["float32", "float64", "complex64", "complex128"],
            "symmetric_power_monomial_adjoint": ["float32", "float64", "complex64", "complex128"],
            "factorized_schedule": ["float32", "float64", "complex64", "complex128"],
            "ace_density": ["float64 -> complex128"],
            "ace_density_mixed": ["float32 -> complex64", "float64 -> complex128"],
            "pace_radial_channel_contraction_with_derivative": ["float32", "float64"],
            "ace_bundle": ["complex128"],
        },
        "density_accumulate_deterministic": True,
        "max_spherical_lmax": 8,
        "fused_ace_lmax": 4,
    }
