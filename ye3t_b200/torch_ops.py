"""The runtime operators as registered torch operators (``torch.ops.ye3t_b200``).

The reference registers its runtime under ``TORCH_LIBRARY(ye3t_runtime, ...)``
(ye3t/runtime/csrc/execution_plan_torch.cpp:7229-7731) with fake kernels so
that ``torch.compile`` can trace them (ye3t/runtime/execution_plan.py:392).
Importing this module registers the same operators, with the same argument
lists, in the ``ye3t_b200`` namespace: each implementation calls this
package's C ABI through :mod:`ye3t_b200.runtime` (CUDA tensors only), each has
a fake kernel giving output shapes and dtypes, and the density accumulation
and grouped symmetric power carry first-order autograd through their GPU
adjoints.  ``factorized_schedule`` is the schedule evaluator over raw table
tensors (the reference's ``evaluate_factorized_schedule_cpu`` arguments,
core/csrc/factorized_runtime.cpp:426); its autograd lives in
``ye3t_b200.couplings.evaluate_factorized_schedule_torch``.
"""

from __future__ import annotations

from typing import Tuple

import torch
from torch import Tensor
from torch.library import custom_op

from . import _native as nat
from . import runtime as rt

__all__ = ["NAMESPACE"]

NAMESPACE = "ye3t_b200"


def _complex_of(dtype):
    return torch.complex128 if dtype in (torch.float64, torch.complex128) else torch.complex64


# -- density accumulation (execution_plan.py:7913, :7987) ------------------------------------
@custom_op("ye3t_b200::density_accumulate", mutates_args=())
def density_accumulate(edge_values: Tensor, centers: Tensor, atom_count: int) -> Tensor:
    with torch.no_grad():
        return rt.density_accumulate(edge_values, centers, atom_count)


@density_accumulate.register_fake
def _(edge_values, centers, atom_count):
    return edge_values.new_empty((int(atom_count),) + tuple(edge_values.shape[1:]))


@custom_op("ye3t_b200::density_accumulate_adjoint", mutates_args=())
def density_accumulate_adjoint(atomic_adjoint: Tensor, centers: Tensor) -> Tensor:
    with torch.no_grad():
        return rt.density_accumulate_adjoint(atomic_adjoint, centers)


@density_accumulate_adjoint.register_fake
def _(atomic_adjoint, centers):
    return atomic_adjoint.new_empty((centers.shape[0],) + tuple(atomic_adjoint.shape[1:]))


def _density_setup(ctx, inputs, output):
    ctx.save_for_backward(inputs[1])


def _density_backward(ctx, grad):
    (centers,) = ctx.saved_tensors
    return torch.ops.ye3t_b200.density_accumulate_adjoint(grad.contiguous(), centers), None, None


density_accumulate.register_autograd(_density_backward, setup_context=_density_setup)


# -- edge tables (execution_plan.py:7298, :7479, :7675) -----------------------------------------
@custom_op("ye3t_b200::cheb_exp_cos_radial_table_with_derivative", mutates_args=())
def cheb_exp_cos_radial_table_with_derivative(radii: Tensor, cutoffs: Tensor, lambdas: Tensor,
                                              maximum_radial_index: int) -> Tuple[Tensor, Tensor]:
    with torch.no_grad():
        v, d = rt.cheb_exp_cos_radial_table_with_derivative(radii, cutoffs, lambdas, maximum_radial_index)
    return v, d


@cheb_exp_cos_radial_table_with_derivative.register_fake
def _(radii, cutoffs, lambdas, maximum_radial_index):
    shape = (radii.reshape(-1).shape[0], int(maximum_radial_index) + 1)
    return radii.new_empty(shape), radii.new_empty(shape)


@custom_op("ye3t_b200::spherical_harmonics_table_with_derivative", mutates_args=())
def spherical_harmonics_table_with_derivative(edge_vectors: Tensor, maximum_angular_momentum: int,
                                              real_output: bool, epsilon: float) -> Tuple[Tensor, Tensor]:
    with torch.no_grad():
        v, d = rt.spherical_harmonics_table_with_derivative(edge_vectors, maximum_angular_momentum,
                                                            real_output=real_output, epsilon=epsilon)
    return v, d


@spherical_harmonics_table_with_derivative.register_fake
def _(edge_vectors, maximum_angular_momentum, real_output, epsilon):
    E = edge_vectors.reshape(-1, 3).shape[0]
    W = (int(maximum_angular_momentum) + 1) ** 2
    dt = edge_vectors.dtype if real_output else _complex_of(edge_vectors.dtype)
    return edge_vectors.new_empty((E, W), dtype=dt), edge_vectors.new_empty((E, W, 3), dtype=dt)


@custom_op("ye3t_b200::scheduled_radial_angular_channels_with_derivative", mutates_args=())
def scheduled_radial_angular_channels_with_derivative(radial_values: Tensor, radial_derivatives: Tensor,
                                                      angular_values: Tensor, angular_derivatives: Tensor,
                                                      radial_directions: Tensor, edge_types: Tensor,
                                                      channel_radial_indices: Tensor, channel_angular_indices: Tensor,
                                                      channel_types: Tensor,
                                                      channel_scales: Tensor) -> Tuple[Tensor, Tensor]:
    with torch.no_grad():
        v, d = rt.scheduled_radial_angular_channels_with_derivative(
            radial_values, radial_derivatives, angular_values, angular_derivatives, radial_directions, edge_types,
            channel_radial_indices, channel_angular_indices, channel_types, channel_scales)
    return v, d


@scheduled_radial_angular_channels_with_derivative.register_fake
def _(radial_values, radial_derivatives, angular_values, angular_derivatives, radial_directions, edge_types,
      channel_radial_indices, channel_angular_indices, channel_types, channel_scales):
    E, C = radial_values.shape[0], channel_radial_indices.reshape(-1).shape[0]
    return radial_values.new_empty((E, C)), radial_values.new_empty((E, C, 3))


# -- symmetric powers (execution_plan_torch.cpp:7528, :7541) ------------------------------------
@custom_op("ye3t_b200::symmetric_power_monomial", mutates_args=())
def symmetric_power_monomial(input: Tensor, monomial_counts: Tensor, output_offsets: Tensor, output_indices: Tensor,
                             monomial_values: Tensor) -> Tensor:
    with torch.no_grad():
        return rt.symmetric_power_monomial_contraction(input, monomial_counts, output_offsets, output_indices,
                                                       monomial_values)


@symmetric_power_monomial.register_fake
def _(input, monomial_counts, output_offsets, output_indices, monomial_values):
    return input.new_empty(tuple(input.shape[:-1]) + (output_offsets.reshape(-1).shape[0] - 1,))


@custom_op("ye3t_b200::symmetric_power_monomial_adjoint", mutates_args=())
def symmetric_power_monomial_adjoint(output_adjoint: Tensor, input: Tensor, monomial_counts: Tensor,
                                     output_offsets: Tensor, output_indices: Tensor,
                                     monomial_values: Tensor) -> Tensor:
    x2 = input.contiguous().reshape(-1, input.shape[-1])
    adj = output_adjoint.to(input.dtype).contiguous().reshape(x2.shape[0], -1)
    counts = monomial_counts.to(torch.int64).contiguous()
    idx = output_indices.to(torch.int64).reshape(-1).contiguous()
    vals = monomial_values.to(input.dtype).reshape(-1).contiguous()
    out_dim = output_offsets.reshape(-1).shape[0] - 1
    with torch.no_grad():
        return rt._sympow_adjoint(adj, x2, counts, idx, vals, out_dim).reshape(input.shape)


@symmetric_power_monomial_adjoint.register_fake
def _(output_adjoint, input, monomial_counts, output_offsets, output_indices, monomial_values):
    return input.new_empty(input.shape)


def _sympow_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _sympow_backward(ctx, grad):
    x, counts, offsets, indices, values = ctx.saved_tensors
    return (torch.ops.ye3t_b200.symmetric_power_monomial_adjoint(grad, x, counts, offsets, indices, values),
            None, None, None, None)


symmetric_power_monomial.register_autograd(_sympow_backward, setup_context=_sympow_setup)


@custom_op("ye3t_b200::symmetric_power_shared_monomial", mutates_args=())
def symmetric_power_shared_monomial(input: Tensor, monomial_counts: Tensor, output_offsets: Tensor,
                                    coefficient_terms: Tensor, coefficient_outputs: Tensor,
                                    coefficient_values: Tensor) -> Tensor:
    with torch.no_grad():
        return rt.symmetric_power_shared_monomial_contraction(input, monomial_counts, output_offsets,
                                                              coefficient_terms, coefficient_outputs,
                                                              coefficient_values)


@symmetric_power_shared_monomial.register_fake
def _(input, monomial_counts, output_offsets, coefficient_terms, coefficient_outputs, coefficient_values):
    return input.new_empty(tuple(input.shape[:-1]) + (output_offsets.reshape(-1).shape[0] - 1,))


# -- factorized schedule over raw tables (factorized_runtime.cpp:426) ---------------------------
@custom_op("ye3t_b200::factorized_schedule", mutates_args=())
def factorized_schedule(block_values: Tensor, component_offsets: Tensor, component_label_index: Tensor,
                        block_m_indices: Tensor, coeffs: Tensor) -> Tensor:
    bv = block_values.contiguous()
    dev = nat.require_cuda(bv, what="factorized_schedule")
    if bv.ndim != 4:
        raise ValueError("block_values must have shape [batch, basis_count, block_count, max_block_m_dim].")
    off = component_offsets.to(device=dev, dtype=torch.int64).reshape(-1).contiguous()
    cli = component_label_index.to(device=dev, dtype=torch.int64).reshape(-1).contiguous()
    midx = block_m_indices.to(device=dev, dtype=torch.int64).contiguous()
    co = coeffs.to(device=dev, dtype=bv.dtype).reshape(-1).contiguous()
    batch, basis, blocks, mdim = (int(s) for s in bv.shape)
    comps, terms = int(off.shape[0]) - 1, int(co.shape[0])
    if int(cli.shape[0]) != comps or (terms and tuple(midx.shape) != (terms, blocks)):
        raise ValueError("schedule tables disagree on component or term counts")
    out = torch.empty((batch, comps), dtype=bv.dtype, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    nat.check(nat.lib().y3b_factorized_schedule_evaluate(
        nat.dtype_code(bv.dtype), bv.data_ptr(), batch, basis, blocks, mdim, off.data_ptr(), cli.data_ptr(),
        midx.data_ptr() if terms else 0, co.data_ptr() if terms else 0, comps, terms, out.data_ptr(),
        status.data_ptr(), nat.stream_of(dev)), "factorized_schedule")
    if int(status.item()):
        raise IndexError("factorized_schedule: schedule index out of range")
    return out


@factorized_schedule.register_fake
def _(block_values, component_offsets, component_label_index, block_m_indices, coeffs):
    return block_values.new_empty((block_values.shape[0], component_offsets.reshape(-1).shape[0] - 1))
