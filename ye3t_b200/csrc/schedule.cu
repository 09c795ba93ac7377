// Generic factorized-schedule evaluation and symmetric-power contraction.
//
// These are the drop-in kernels behind evaluate_factorized_schedule_torch and
// symmetric_power_monomial for arbitrary caller-supplied block arrays.  The
// fused bundle path (ace.cu) evaluates the same schedules from an on-device
// block pool.
#include "common.cuh"

namespace y3b {

// One thread per (batch row, component), component fastest, grid-stride.
// Consecutive threads read the same batch row (L1-resident) and write
// consecutive outputs.  Terms run in table order from the coefficient, as in
// factorized_runtime.cpp:268-283.
template <typename T>
__global__ void __launch_bounds__(256) schedule_eval_kernel(
    const T* __restrict__ bv, int64_t batch, int64_t basis, int64_t blocks, int64_t mdim,
    const int64_t* __restrict__ off, const int64_t* __restrict__ labels,
    const int64_t* __restrict__ midx, const T* __restrict__ coeffs, int64_t comps,
    T* __restrict__ out, int32_t* status) {
  const int64_t total = batch * comps;
  for (int64_t lin = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = lin / comps;
    const int64_t c = lin - b * comps;
    const int64_t label = __ldg(labels + c);
    T acc = zero<T>();
    if (label < 0 || label >= basis) {
      if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
    } else {
      const T* row = bv + (b * basis + label) * blocks * mdim;
      const int64_t t0 = __ldg(off + c), t1 = __ldg(off + c + 1);
      for (int64_t t = t0; t < t1; ++t) {
        T v = coeffs[t];
        const int64_t* mt = midx + t * blocks;
        for (int64_t j = 0; j < blocks; ++j) {
          const int64_t m = __ldg(mt + j);
          if (m < 0 || m >= mdim) {
            if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
            v = zero<T>();
            break;
          }
          v = mul(v, row[j * mdim + m]);
        }
        acc = add(acc, v);
      }
    }
    out[lin] = acc;
  }
}

// Integer power by square-and-multiply, the evaluation order of
// ye3t_runtime_core's integer_power (ye3t_runtime_core.cpp:98), so that
// powers round as the reference's do; an exponent of 0 yields exactly 1.
template <typename T>
__device__ __forceinline__ T ipow(T x, int64_t e) {
  T r = one<T>();
  while (e > 0) {
    if (e & 1) r = mul(r, x);
    e >>= 1;
    if (e > 0) x = mul(x, x);
  }
  return r;
}

// One thread per (batch row, output component).
template <typename T>
__global__ void __launch_bounds__(256) sympow_kernel(
    const T* __restrict__ x, int64_t batch, int64_t in_dim, const int64_t* __restrict__ counts,
    const int64_t* __restrict__ off, const T* __restrict__ vals, int64_t out_dim,
    T* __restrict__ out) {
  const int64_t total = batch * out_dim;
  for (int64_t lin = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = lin / out_dim;
    const int64_t o = lin - b * out_dim;
    const T* xr = x + b * in_dim;
    T acc = zero<T>();
    for (int64_t t = __ldg(off + o); t < __ldg(off + o + 1); ++t) {
      T m = vals[t];
      for (int64_t i = 0; i < in_dim; ++i) {
        const int64_t e = __ldg(counts + t * in_dim + i);
        if (e) m = mul(m, ipow(xr[i], e));
      }
      acc = add(acc, m);
    }
    out[lin] = acc;
  }
}

// Shared-monomial form: out[b, o] = sum over the output's coefficients t of
// values[t] * monomial[terms[t]], each monomial the product over all input
// components of x^count (ye3t_runtime_core.cpp:5392).  One thread per
// (batch row, output); a monomial is formed where a coefficient uses it.
// Monomial indices outside [0, monomial_count) set Y3B_STATUS_INDEX_RANGE and
// contribute 0.
template <typename T>
__global__ void __launch_bounds__(256) sympow_shared_kernel(
    const T* __restrict__ x, int64_t batch, int64_t in_dim, const int64_t* __restrict__ counts,
    int64_t monomials, const int64_t* __restrict__ off, const int64_t* __restrict__ terms,
    const T* __restrict__ vals, int64_t out_dim, T* __restrict__ out, int32_t* __restrict__ status) {
  const int64_t total = batch * out_dim;
  for (int64_t lin = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = lin / out_dim;
    const int64_t o = lin - b * out_dim;
    const T* xr = x + b * in_dim;
    T acc = zero<T>();
    for (int64_t t = __ldg(off + o); t < __ldg(off + o + 1); ++t) {
      const int64_t m = __ldg(terms + t);
      if (m < 0 || m >= monomials) {
        if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        continue;
      }
      T mono = one<T>();
      for (int64_t i = 0; i < in_dim; ++i) mono = mul(mono, ipow(xr[i], __ldg(counts + m * in_dim + i)));
      acc = add(acc, mul(vals[t], mono));
    }
    out[lin] = acc;
  }
}

// Conjugate-transposed derivative of the grouped table (the vector-Jacobian
// product autograd forms, execution_plan.py:4970-4990 / ye3t_runtime_core
// symmetric_power_monomial_adjoint): grad[b, i] = sum over terms t with
// counts[t, i] = e > 0 of adj[b, o_t] conj(e c_t x_i^(e-1) prod_{j != i}
// x_j^(e_j)).  One thread per (batch row, input component), so every entry has
// one owner; the derivative is formed without dividing by x_i.
template <typename T>
__device__ __forceinline__ T cconj(T a) { return a; }
template <>
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }
template <>
__device__ __forceinline__ double2 cconj(double2 a) { return make_double2(a.x, -a.y); }

template <typename T>
__global__ void __launch_bounds__(256) sympow_adjoint_kernel(
    const T* __restrict__ adj, const T* __restrict__ x, int64_t batch, int64_t in_dim,
    const int64_t* __restrict__ counts, const int64_t* __restrict__ oidx, const T* __restrict__ vals,
    int64_t terms, int64_t out_dim, T* __restrict__ grad, int32_t* __restrict__ status) {
  const int64_t total = batch * in_dim;
  for (int64_t lin = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = lin / in_dim, i = lin - b * in_dim;
    const T* xr = x + b * in_dim;
    T acc = zero<T>();
    for (int64_t t = 0; t < terms; ++t) {
      const int64_t e = __ldg(counts + t * in_dim + i);
      if (e <= 0) continue;
      const int64_t o = __ldg(oidx + t);
      if (o < 0 || o >= out_dim) {
        if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        continue;
      }
      T d = vals[t];
      for (int64_t j = 0; j < in_dim; ++j) {
        const int64_t ej = __ldg(counts + t * in_dim + j);
        d = mul(d, ipow(xr[j], j == i ? ej - 1 : ej));
      }
      using R = typename Real<T>::type;
      d = scale(R(e), d);
      acc = add(acc, mul(adj[b * out_dim + o], cconj(d)));
    }
    grad[lin] = acc;
  }
}

// Vector-Jacobian product of the schedule evaluation (what torch autograd
// forms through evaluate_factorized_schedule_torch, core/couplings.py:481-567):
//   grad[b, label, j, m] = sum over (t, c) reading slot (label, j, m) of
//                          adj[b, c] conj(coeff_t prod_{k != j} bv[b, label, k, midx[t, k]]).
// The (term, component) pairs of every slot s = (label * blocks + j) * mdim + m
// come from a transposed table built once per schedule on the host
// (slot_offsets [S + 1], slot_terms / slot_components [P]), so each gradient
// entry has one owning thread: no atomics, a fixed summation order.
template <typename T>
__global__ void __launch_bounds__(256) schedule_adjoint_kernel(
    const T* __restrict__ adj, const T* __restrict__ bv, int64_t batch, int64_t basis, int64_t blocks,
    int64_t mdim, const int64_t* __restrict__ midx, const T* __restrict__ coeffs, int64_t comps, int64_t terms,
    const int64_t* __restrict__ slot_off, const int64_t* __restrict__ slot_term,
    const int64_t* __restrict__ slot_comp, T* __restrict__ grad, int32_t* status) {
  const int64_t S = basis * blocks * mdim;
  const int64_t total = batch * S;
  for (int64_t lin = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = lin / S, s = lin - b * S;
    const int64_t label = s / (blocks * mdim), j = (s / mdim) % blocks;
    const T* row = bv + (b * basis + label) * blocks * mdim;
    T acc = zero<T>();
    for (int64_t p = __ldg(slot_off + s); p < __ldg(slot_off + s + 1); ++p) {
      const int64_t t = __ldg(slot_term + p), c = __ldg(slot_comp + p);
      if (t < 0 || t >= terms || c < 0 || c >= comps) {
        if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        continue;
      }
      T v = coeffs[t];
      const int64_t* mt = midx + t * blocks;
      bool ok = true;
      for (int64_t k = 0; k < blocks; ++k) {
        if (k == j) continue;
        const int64_t m = __ldg(mt + k);
        if (m < 0 || m >= mdim) {
          ok = false;
          break;
        }
        v = mul(v, row[k * mdim + m]);
      }
      if (!ok) {
        if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        continue;
      }
      acc = add(acc, mul(adj[b * comps + c], cconj(v)));
    }
    grad[lin] = acc;
  }
}

}  // namespace y3b

using namespace y3b;

extern "C" int y3b_factorized_schedule_evaluate(int dtype, const void* block_values, int64_t batch,
                                                int64_t basis_count, int64_t block_count,
                                                int64_t magnetic_dim,
                                                const int64_t* component_offsets,
                                                const int64_t* component_label_index,
                                                const int64_t* block_m_indices, const void* coeffs,
                                                int64_t component_count, int64_t term_count,
                                                void* out, int32_t* status, void* stream) {
  Y3B_CHECK_ARG(batch >= 0 && basis_count >= 0 && block_count >= 0 && magnetic_dim >= 0,
                "negative size");
  Y3B_CHECK_ARG(component_count >= 0 && term_count >= 0, "negative component/term count");
  const int64_t total = batch * component_count;
  if (total == 0) return Y3B_OK;
  Y3B_CHECK_ARG(block_values && component_offsets && component_label_index && out,
                "null pointer argument");
  Y3B_CHECK_ARG(term_count == 0 || (coeffs && (block_count == 0 || block_m_indices)),
                "null coefficient or index table");
  const int threads = 256;
  const int grid = grid_for(total, threads);
  Y3B_DISPATCH(dtype, T, {
    schedule_eval_kernel<T><<<grid, threads, 0, as_stream(stream)>>>(
        static_cast<const T*>(block_values), batch, basis_count, block_count, magnetic_dim,
        component_offsets, component_label_index, block_m_indices, static_cast<const T*>(coeffs),
        component_count, static_cast<T*>(out), status);
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_symmetric_power_monomial(int dtype, const void* input, int64_t batch,
                                            int64_t input_dim, const int64_t* monomial_counts,
                                            const int64_t* output_offsets,
                                            const void* monomial_values, int64_t term_count,
                                            int64_t output_dim, void* out, void* stream) {
  Y3B_CHECK_ARG(batch >= 0 && input_dim >= 0 && output_dim >= 0 && term_count >= 0,
                "negative size");
  const int64_t total = batch * output_dim;
  if (total == 0) return Y3B_OK;
  Y3B_CHECK_ARG(input && output_offsets && out && (term_count == 0 || (monomial_counts && monomial_values)),
                "null pointer argument");
  const int threads = 256;
  const int grid = grid_for(total, threads);
  Y3B_DISPATCH(dtype, T, {
    sympow_kernel<T><<<grid, threads, 0, as_stream(stream)>>>(
        static_cast<const T*>(input), batch, input_dim, monomial_counts, output_offsets,
        static_cast<const T*>(monomial_values), output_dim, static_cast<T*>(out));
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_symmetric_power_shared_monomial(int dtype, const void* input, int64_t batch,
                                                   int64_t input_dim, const int64_t* monomial_counts,
                                                   int64_t monomial_count, const int64_t* output_offsets,
                                                   int64_t output_dim, const int64_t* coefficient_terms,
                                                   const void* coefficient_values, int64_t coefficient_count,
                                                   void* out, int32_t* status, void* stream) {
  Y3B_CHECK_ARG(batch >= 0 && input_dim >= 0 && output_dim >= 0 && monomial_count >= 0 && coefficient_count >= 0,
                "negative size");
  const int64_t total = batch * output_dim;
  if (total == 0) return Y3B_OK;
  Y3B_CHECK_ARG(input && output_offsets && out &&
                    (coefficient_count == 0 || (coefficient_terms && coefficient_values)) &&
                    (monomial_count == 0 || monomial_counts),
                "null pointer argument");
  const int threads = 256;
  const int grid = grid_for(total, threads);
  Y3B_DISPATCH(dtype, T, {
    sympow_shared_kernel<T><<<grid, threads, 0, as_stream(stream)>>>(
        static_cast<const T*>(input), batch, input_dim, monomial_counts, monomial_count, output_offsets,
        coefficient_terms, static_cast<const T*>(coefficient_values), output_dim, static_cast<T*>(out), status);
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_symmetric_power_monomial_adjoint(int dtype, const void* output_adjoint, const void* input,
                                                    int64_t batch, int64_t input_dim, const int64_t* monomial_counts,
                                                    const int64_t* output_indices, const void* monomial_values,
                                                    int64_t term_count, int64_t output_dim, void* input_adjoint,
                                                    int32_t* status, void* stream) {
  Y3B_CHECK_ARG(batch >= 0 && input_dim >= 0 && output_dim >= 0 && term_count >= 0, "negative size");
  const int64_t total = batch * input_dim;
  if (total == 0) return Y3B_OK;
  Y3B_CHECK_ARG(output_adjoint && input && input_adjoint &&
                    (term_count == 0 || (monomial_counts && output_indices && monomial_values)),
                "null pointer argument");
  const int threads = 256;
  Y3B_DISPATCH(dtype, T, {
    sympow_adjoint_kernel<T><<<grid_for(total, threads), threads, 0, as_stream(stream)>>>(
        static_cast<const T*>(output_adjoint), static_cast<const T*>(input), batch, input_dim, monomial_counts,
        output_indices, static_cast<const T*>(monomial_values), term_count, output_dim,
        static_cast<T*>(input_adjoint), status);
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_factorized_schedule_adjoint(int dtype, const void* output_adjoint, const void* block_values,
                                               int64_t batch, int64_t basis_count, int64_t block_count,
                                               int64_t magnetic_dim, const int64_t* block_m_indices,
                                               const void* coeffs, int64_t component_count, int64_t term_count,
                                               const int64_t* slot_offsets, const int64_t* slot_terms,
                                               const int64_t* slot_components, void* block_values_adjoint,
                                               int32_t* status, void* stream) {
  Y3B_CHECK_ARG(batch >= 0 && basis_count >= 0 && block_count >= 0 && magnetic_dim >= 0 && component_count >= 0 &&
                    term_count >= 0,
                "negative size");
  const int64_t total = batch * basis_count * block_count * magnetic_dim;
  if (total == 0) return Y3B_OK;
  Y3B_CHECK_ARG(output_adjoint && block_values && slot_offsets && block_values_adjoint &&
                    (term_count == 0 || (coeffs && block_m_indices && slot_terms && slot_components)),
                "null pointer argument");
  const int threads = 256;
  Y3B_DISPATCH(dtype, T, {
    schedule_adjoint_kernel<T><<<grid_for(total, threads), threads, 0, as_stream(stream)>>>(
        static_cast<const T*>(output_adjoint), static_cast<const T*>(block_values), batch, basis_count, block_count,
        magnetic_dim, block_m_indices, static_cast<const T*>(coeffs), component_count, term_count, slot_offsets,
        slot_terms, slot_components, static_cast<T*>(block_values_adjoint), status);
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}
