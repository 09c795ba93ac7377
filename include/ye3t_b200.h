/*
 * ye3t_b200: C ABI of the B200 (sm_100a) evaluator for ye3t's compiled ACE
 * feature path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*), launches asynchronously on that stream and
 * returns Y3B_OK or a negative error code; y3b_last_error() gives the message
 * (thread-local).  Nothing here allocates device memory: callers pass outputs
 * and, where an operation needs scratch, a workspace sized by the matching
 * *_workspace_bytes() query.  Arrays are C-contiguous.  Complex arrays are
 * interleaved (re, im) pairs, the layout of std::complex / numpy / torch.
 *
 * Each entry point cites the reference interface (file:line inside the ye3t
 * project) that it replaces.
 */
#ifndef YE3T_B200_H
#define YE3T_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Y3B_ABI_VERSION 8

/* dtype codes */
#define Y3B_F32 0
#define Y3B_F64 1
#define Y3B_C64 2
#define Y3B_C128 3

/* status codes */
#define Y3B_OK 0
#define Y3B_ERR_ARGUMENT (-1)
#define Y3B_ERR_CUDA (-2)
#define Y3B_ERR_WORKSPACE (-3)
#define Y3B_ERR_UNSUPPORTED (-4)

/* device status word bits written by kernels that detect bad input */
#define Y3B_STATUS_INDEX_RANGE 1
#define Y3B_STATUS_CAPACITY 2
#define Y3B_STATUS_TABLE 4 /* a table entry outside the kernel's bounds was skipped */
#define Y3B_STATUS_TIMEOUT 8 /* a bounded wait on the tensor cores ran out; the output is incomplete */

/* ABI version; the reference's gate is core_abi_version()
 * (ye3t/runtime/csrc/execution_plan_torch.cpp:7925, checked at
 * ye3t/runtime/execution_plan.py:253-291). */
int32_t y3b_abi_version(void);
const char* y3b_last_error(void);

/* ------------------------------------------------------------------------
 * Factorized coefficient schedule evaluation.
 * Replaces evaluate_factorized_schedule_cpu
 * (ye3t/core/csrc/factorized_runtime.cpp:426-548) and the torch
 * gather/index_add path of evaluate_factorized_schedule_torch
 * (ye3t/core/couplings.py:481-567):
 *   out[b, c] = sum_{t in [off[c], off[c+1])} coeffs[t] *
 *               prod_j block_values[b, label[c], j, m_idx[t, j]]
 * block_values [batch, basis, blocks, mdim]; block_m_indices [terms, blocks]
 * (int64, m + L_block); coeffs and out share dtype.  Out-of-range labels or m
 * indices set Y3B_STATUS_INDEX_RANGE in *status (nullable) and contribute 0.
 * ---------------------------------------------------------------------- */
int y3b_factorized_schedule_evaluate(int dtype, const void* block_values, int64_t batch,
                                     int64_t basis_count, int64_t block_count, int64_t magnetic_dim,
                                     const int64_t* component_offsets,
                                     const int64_t* component_label_index,
                                     const int64_t* block_m_indices, const void* coeffs,
                                     int64_t component_count, int64_t term_count, void* out,
                                     int32_t* status, void* stream);

/* Vector-Jacobian product of the evaluation above (the backward torch autograd
 * forms through evaluate_factorized_schedule_torch, core/couplings.py:481-567):
 *   grad[b, label, j, m] = sum over (t, c) reading slot (label, j, m) of
 *                          adj[b, c] conj(coeffs[t] prod_{k != j} bv[b, label, k, m_idx[t, k]])
 * block_values and the gradient are [batch, basis, blocks, magnetic_dim];
 * slot s = (label * blocks + j) * magnetic_dim + m lists its (term,
 * component) pairs in slot_terms / slot_components[slot_offsets[s] ..
 * slot_offsets[s+1]) (host-built transposed table; ye3t_b200/couplings.py).
 * One thread per gradient entry: no atomics.  Indices out of range set
 * Y3B_STATUS_INDEX_RANGE in *status (nullable) and contribute 0. */
int y3b_factorized_schedule_adjoint(int dtype, const void* output_adjoint, const void* block_values, int64_t batch,
                                    int64_t basis_count, int64_t block_count, int64_t magnetic_dim,
                                    const int64_t* block_m_indices, const void* coeffs, int64_t component_count,
                                    int64_t term_count, const int64_t* slot_offsets, const int64_t* slot_terms,
                                    const int64_t* slot_components, void* block_values_adjoint, int32_t* status,
                                    void* stream);

/* Symmetric-power monomial contraction, grouped table.
 * Replaces ye3t_runtime::symmetric_power_monomial
 * (ye3t/runtime/csrc/execution_plan_torch.cpp:7528; CPU core
 * ye3t_runtime_core.cpp:5279):
 *   out[b, o] = sum_{t in [off[o], off[o+1])} values[t] prod_i x[b, i]^counts[t, i] */
int y3b_symmetric_power_monomial(int dtype, const void* input, int64_t batch, int64_t input_dim,
                                 const int64_t* monomial_counts, const int64_t* output_offsets,
                                 const void* monomial_values, int64_t term_count,
                                 int64_t output_dim, void* out, void* stream);

/* Symmetric-power contraction, shared-monomial table: each of monomial_count
 * unique monomials prod_i x[b, i]^counts[m, i] is weighted per coefficient.
 * Replaces ye3t_runtime::symmetric_power_shared_monomial
 * (ye3t/runtime/csrc/execution_plan_torch.cpp:7541; CPU core
 * ye3t_runtime_core.cpp:5392; Python entry execution_plan.py:12502):
 *   out[b, o] = sum_{t in [off[o], off[o+1])} values[t] monomial[b, terms[t]]
 * Monomial indices outside [0, monomial_count) set Y3B_STATUS_INDEX_RANGE in
 * *status (nullable) and contribute 0. */
/* Vector-Jacobian product of the grouped table (autograd of
 * symmetric_power_monomial, execution_plan.py:4970-4990; CPU core
 * symmetric_power_monomial_adjoint): input_adjoint[b, i] = sum over terms t of
 * output_adjoint[b, output_indices[t]] conj(d term_t / d x_i).  Output indices
 * outside [0, output_dim) set Y3B_STATUS_INDEX_RANGE and contribute 0. */
int y3b_symmetric_power_monomial_adjoint(int dtype, const void* output_adjoint, const void* input, int64_t batch,
                                         int64_t input_dim, const int64_t* monomial_counts,
                                         const int64_t* output_indices, const void* monomial_values,
                                         int64_t term_count, int64_t output_dim, void* input_adjoint,
                                         int32_t* status, void* stream);

int y3b_symmetric_power_shared_monomial(int dtype, const void* input, int64_t batch, int64_t input_dim,
                                        const int64_t* monomial_counts, int64_t monomial_count,
                                        const int64_t* output_offsets, int64_t output_dim,
                                        const int64_t* coefficient_terms, const void* coefficient_values,
                                        int64_t coefficient_count, void* out, int32_t* status, void* stream);

/* ChebExpCos radial table with d/dr, radial indices 0..maximum_radial_index.
 * Replaces ye3t_runtime::cheb_exp_cos_radial_table_with_derivative
 * (ye3t/runtime/csrc/execution_plan_torch.cpp:7238). Real dtypes only. */
int y3b_cheb_exp_cos_radial_table(int dtype, const void* radii, const void* cutoffs,
                                  const void* lambdas, int64_t edge_count,
                                  int64_t maximum_radial_index, void* values, void* derivatives,
                                  void* stream);

/* Packed spherical-harmonic table (all l <= lmax, columns [l^2, (l+1)^2))
 * with Cartesian derivatives [E, W, 3].  Real tesseral when real_output != 0,
 * else complex Condon-Shortley (values/derivatives then complex of the same
 * precision).  Replaces ye3t_runtime::spherical_harmonics_table_with_derivative
 * (ye3t/runtime/csrc/execution_plan_torch.cpp:7251). dtype is the real type
 * of edge_vectors. */
int y3b_spherical_harmonics_table(int dtype, const void* edge_vectors, int64_t edge_count,
                                  int64_t maximum_angular_momentum, int real_output,
                                  double epsilon, void* values, void* derivatives, void* stream);

/* Scheduled radial x angular channels with Cartesian derivatives (real dtypes):
 *   values[e, c] = R[e, rad_c] Y[e, ang_c] s_c
 *   derivatives[e, c, :] = s_c (R'[e, rad_c] d[e, :] Y[e, ang_c] + R[e, rad_c] dY[e, ang_c, :])
 * for channels whose type is negative or equals the edge's type, else 0.
 * R, R' [E, radial_count]; Y [E, angular_count]; dY [E, angular_count, 3];
 * d [E, 3] (unit edge directions).  Replaces
 * ye3t_runtime::scheduled_radial_angular_channels_with_derivative
 * (ye3t/runtime/csrc/execution_plan_torch.cpp:7268; Python entry
 * execution_plan.py:7675).  Radial / angular indices outside their tables set
 * Y3B_STATUS_INDEX_RANGE in *status (nullable) and give 0. */
int y3b_scheduled_radial_angular_channels(int dtype, const void* radial_values, const void* radial_derivatives,
                                          int64_t radial_count, const void* angular_values,
                                          const void* angular_derivatives, int64_t angular_count,
                                          const void* radial_directions, const int64_t* edge_types,
                                          int64_t edge_count, const int64_t* channel_radial_indices,
                                          const int64_t* channel_angular_indices, const int64_t* channel_types,
                                          const void* channel_scales, int64_t channel_count, void* values,
                                          void* derivatives, int32_t* status, void* stream);

/* Plain site-basis product with per-edge group prefactors (real or complex):
 * term t (group g_t, channel ch_t) of edge e gives
 *   edge_values[e, ch_t] = p[g_t, e] R[g_t, e] Y[t, e]
 *   edge_derivatives[e, ch_t, :] = p[g_t, e] (R'[g_t, e] d[e, :] Y[t, e] + R[g_t, e] dY[t, e, :])
 *   charge_center / charge_neighbor [e, ch_t] = pc / pn [g_t, e] R[g_t, e] Y[t, e]
 * and channels no term names are 0.  R, R', p, pc, pn [group_count, E];
 * Y [term_count, E]; dY [term_count, E, 3]; d [E, 3]; outputs [E, channel_count]
 * ([E, channel_count, 3] for the derivatives).  Term channels are distinct.
 * Replaces ye3t_runtime::plain_site_basis_product_with_derivative
 * (execution_plan_torch.cpp, schema beside :7268; Python entry
 * execution_plan.py:7582).  Groups or channels out of range set
 * Y3B_STATUS_INDEX_RANGE and write nothing. */
/* Adjoint of the plain site-basis product with edge weights w [E] and their
 * derivatives dw [E, 3] against edge-channel adjoints a [E, channel_count]:
 *   position_adjoint[e, :] = sum_t a[e, ch_t] (td[t, e, :] w[e] + tv[t, e] dw[e, :])
 *   charge_center / charge_neighbor _adjoint[e] = sum_t a[e, ch_t] pc / pn[g_t, e] R[g_t, e] Y[t, e] w[e]
 * (tv, td: the forward term values and derivatives above).  Replaces
 * ye3t_runtime::plain_site_basis_product_adjoint (Python entry
 * execution_plan.py:7790).  One thread per edge; no atomics. */
int y3b_plain_site_basis_product_adjoint(int dtype, const void* radial_values, const void* radial_derivatives,
                                         int64_t group_count, const void* angular_values,
                                         const void* angular_derivatives, int64_t term_count, const void* prefactors,
                                         const void* prefactor_derivatives_center,
                                         const void* prefactor_derivatives_neighbor, const void* radial_directions,
                                         const void* edge_weights, const void* edge_weight_derivatives,
                                         int64_t edge_count, const int64_t* term_groups,
                                         const int64_t* term_channels, int64_t channel_count,
                                         const void* edge_adjoint, void* position_adjoint,
                                         void* charge_center_adjoint, void* charge_neighbor_adjoint,
                                         int32_t* status, void* stream);

int y3b_plain_site_basis_product(int dtype, const void* radial_values, const void* radial_derivatives,
                                 int64_t group_count, const void* angular_values, const void* angular_derivatives,
                                 int64_t term_count, const void* prefactors, const void* prefactor_derivatives_center,
                                 const void* prefactor_derivatives_neighbor, const void* radial_directions,
                                 int64_t edge_count, const int64_t* term_groups, const int64_t* term_channels,
                                 int64_t channel_count, void* edge_values, void* edge_derivatives,
                                 void* charge_center, void* charge_neighbor, int32_t* status, void* stream);

/* Density accumulation A[centers[e], c] += edge_values[e, c] without global
 * floating-point atomics: centres are bucketed into CSR rows (integer
 * counting), each row is ordered by edge index, and every output row is
 * summed by one warp in edge order (deterministic).
 * Replaces ye3t_runtime::density_accumulate
 * (ye3t/runtime/csrc/execution_plan_torch.cpp:7285; CUDA atomics kernel
 * execution_plan_cuda.cu:281). */
int64_t y3b_density_accumulate_workspace_bytes(int64_t edge_count, int64_t atom_count);
int y3b_density_accumulate(int dtype, const void* edge_values, const int64_t* centers,
                           int64_t edge_count, int64_t channel_count, int64_t atom_count,
                           void* workspace, int64_t workspace_bytes, void* out, int32_t* status,
                           void* stream);

/* CSR form: row i sums edges [row_offsets[i], row_offsets[i+1]) in order;
 * edge_order (nullable) maps CSR slots to edge rows of edge_values. */
int y3b_density_accumulate_csr(int dtype, const void* edge_values, const int64_t* row_offsets,
                               const int64_t* edge_order, int64_t atom_count,
                               int64_t channel_count, void* out, void* stream);

/* Same result as y3b_density_accumulate, for callers that cannot allocate
 * device memory (no counterpart in the reference).  A host that owns all
 * device memory and forbids allocation while it runs -- an MD engine calling
 * the density from its per-timestep force loop, a server that reserves its
 * memory at start-up -- cannot hand this library a workspace per call, since
 * cudaMalloc would synchronise the device and may fail or be disallowed
 * mid-run.  This entry point allocates nothing: its scratch is a fixed
 * Y3B_NOALLOC_SCRATCH_BYTES array that every GPU loading the library keeps
 * until exit, enough when y3b_density_accumulate_workspace_bytes(E, N) is at
 * most that size; larger problems are rejected with Y3B_ERR_WORKSPACE.  The
 * first call on a device looks up the array's device address (make it before
 * any stream capture) and keeps it for the life of the process, so a device
 * reset (cudaDeviceReset) or a re-created primary context invalidates this
 * entry point for that device.  All calls on a device share the array: calls
 * that overlap on the GPU race and must be serialised by the caller. */
#define Y3B_NOALLOC_SCRATCH_BYTES (16ll * 1024 * 1024)
int y3b_density_accumulate_noalloc(int dtype, const void* edge_values, const int64_t* centers,
                                   int64_t edge_count, int64_t channel_count, int64_t atom_count,
                                   void* out, int32_t* status, void* stream);

/* edge_adjoint[e, c] = atomic_adjoint[centers[e], c].
 * Replaces ye3t_runtime::density_accumulate_adjoint
 * (execution_plan_torch.cpp, schema next to :7285; CUDA
 * execution_plan_cuda.cu:9241). */
int y3b_density_accumulate_adjoint(int dtype, const void* atomic_adjoint, const int64_t* centers,
                                   int64_t edge_count, int64_t channel_count, int64_t atom_count,
                                   void* edge_adjoint, int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Periodic cubic-box neighbour list (cell list) in CSR form for centres
 * [center_begin, center_end).  The reference has no neighbour-list code; this
 * builds the sorted CSR layout the A-basis kernel consumes.  Two passes:
 * y3b_neighbor_count writes per-centre counts into row_offsets[1..] and the
 * exclusive scan into row_offsets (row_offsets[0] = 0); the caller reads
 * row_offsets[count] for the edge total, then y3b_neighbor_fill writes
 * neighbour indices (int32), each row sorted by neighbour index.  Both
 * passes need the cell-list workspace built by the first.
 * ---------------------------------------------------------------------- */
int64_t y3b_neighbor_workspace_bytes(int64_t atom_count, double box, double cutoff);
int y3b_neighbor_count(const double* positions, int64_t atom_count, int64_t center_begin,
                       int64_t center_end, double box, double cutoff, void* workspace,
                       int64_t workspace_bytes, int64_t* row_offsets, void* stream);
int y3b_neighbor_fill(const double* positions, int64_t atom_count, int64_t center_begin,
                      int64_t center_end, double box, double cutoff, const void* workspace,
                      int64_t workspace_bytes, const int64_t* row_offsets, int32_t* neighbors,
                      void* stream);

/* The same two passes for an atom block that is a slab of the box (atoms
 * stored in cell order, one rank's block of a spatial decomposition): only
 * atoms in the z cell layers [z_cell_begin, z_cell_begin + z_cell_count)
 * (periodic, layers of y3b_neighbor_cells_per_side cells) are binned, so the
 * binning costs the slab and its halo instead of the whole system.  Every
 * centre's z layer and its two neighbours must lie in the window; a centre
 * outside sets Y3B_STATUS_INDEX_RANGE (its row is incomplete).  A window of
 * z_cell_count <= 0 or >= the layer count is the whole box.  The fill writes
 * at most neighbor_capacity indices: a list longer than that sets
 * Y3B_STATUS_CAPACITY, so a caller can size the neighbour array from a bound
 * instead of reading row_offsets[count] back to the host first. */
int64_t y3b_neighbor_cells_per_side(double box, double cutoff);
int y3b_neighbor_count_window(const double* positions, int64_t atom_count, int64_t center_begin,
                              int64_t center_end, double box, double cutoff, int64_t z_cell_begin,
                              int64_t z_cell_count, void* workspace, int64_t workspace_bytes,
                              int64_t* row_offsets, int32_t* status, void* stream);
int y3b_neighbor_fill_window(const double* positions, int64_t atom_count, int64_t center_begin,
                             int64_t center_end, double box, double cutoff, int64_t z_cell_begin,
                             int64_t z_cell_count, const void* workspace, int64_t workspace_bytes,
                             const int64_t* row_offsets, int64_t neighbor_capacity, int32_t* neighbors,
                             int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Radial channel mixing.
 * ---------------------------------------------------------------------- */

/* out[p, o] = sum_i W[o, i] in[p, i] and dout[p, o] = sum_i W[o, i] din[p, i]
 * (pace_radial_channel_contraction_with_derivative,
 * ye3t/runtime/csrc/ye3t_runtime_core.h:74-85, .cpp:651): W row-major
 * [output][input], points [point][input] -> [point][output]; products and
 * sums in input order without contraction, as the reference loop.  Real
 * dtypes.  Empty points are a no-op; zero input/output counts are an error. */
int y3b_radial_channel_contraction(int dtype, const void* input_values, const void* input_derivatives,
                                   const void* coefficients, int64_t point_count, int64_t input_count,
                                   int64_t output_count, void* output_values, void* output_derivatives,
                                   void* stream);

/* A-basis with radial channels mixed per species pair:
 *   A[i, c, l^2 + l + m] = sum_{j in row i} sum_n W[z_i, z_j, c, n-1] R_n(r_ij) Yc_lm(r_ij)
 * for n = 1..nmax (ChebExpCos), c < channel_count, complex Condon-Shortley
 * harmonics: the reference's radial table, the contraction above with the
 * pair's table and density_accumulate, fused.  mixing is [S, S, C, nmax]
 * in dtype (F32 or F64, which is also the compute and output type: A is
 * complex64 / complex128 [center_count, C, (lmax+1)^2]); positions are f64.
 * Bad species or neighbour indices set Y3B_STATUS_INDEX_RANGE and contribute 0. */
int y3b_ace_density_mixed(int dtype, const double* positions, const int32_t* species, int64_t atom_count,
                          int64_t center_begin, int64_t center_count, double box,
                          const int64_t* row_offsets, const int32_t* neighbors, const void* mixing,
                          int64_t species_count, int64_t channel_count, int64_t nmax, int64_t lmax,
                          double cutoff, double lambda, void* A, int32_t* status, void* stream);

/* The same A-basis with the mixing as a matrix product on the tensor cores:
 * per centre and neighbour species the edge sums S[i, lm, z, n] = sum_{z_j = z}
 * R_n Yc_lm (CUDA cores, in the real-harmonic basis), then A[i, c, lm] =
 * sum_{z, n} W[z_i, z, c, n] S[i, lm, z, n].  dtype F32: tcgen05 kind::tf32
 * with a 3xTF32 split, 128 rows (i, lm, part) by every centre species' table at
 * once (needs C a multiple of 16, S * nmax <= 64, S * C <= 256); F64: FP64
 * mma.sync m8n8k4 (tcgen05 has no FP64 kind; needs C a multiple of 8 up to
 * 64 and S * nmax <= 64).  Both need lmax <= 4 and nmax <= 16, else Y3B_ERR_UNSUPPORTED (use
 * y3b_ace_density_mixed).  mixing is [S, S, C, nmax] in dtype; A is complex64
 * / complex128 [center_count, C, (lmax+1)^2].  The workspace (16-byte aligned)
 * holds S for a chunk of centres; the full size is
 * y3b_ace_density_mixed_split_workspace_bytes (-1 for an unsupported shape), a
 * smaller one runs in chunks (at least one centre).  Bad indices set
 * Y3B_STATUS_INDEX_RANGE and give 0; a tensor-core wait that runs out sets
 * Y3B_STATUS_TIMEOUT. */
int64_t y3b_ace_density_mixed_split_workspace_bytes(int dtype, int64_t center_count, int64_t species_count,
                                                    int64_t channel_count, int64_t nmax, int64_t lmax);
int y3b_ace_density_mixed_split(int dtype, const double* positions, const int32_t* species, int64_t atom_count,
                                int64_t center_begin, int64_t center_count, double box,
                                const int64_t* row_offsets, const int32_t* neighbors, const void* mixing,
                                int64_t species_count, int64_t channel_count, int64_t nmax, int64_t lmax,
                                double cutoff, double lambda, void* workspace, int64_t workspace_bytes, void* A,
                                int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Fused ACE evaluation over a packed multi-word bundle.
 * ---------------------------------------------------------------------- */

/* Device tables of one packed bundle (all arrays device-resident).  Built on
 * the host from compiled schedules (compile_ace_factorized_schedules_by_L,
 * ye3t/couplings/__init__.py:2617) and symmetric-power plans
 * (ye3t/couplings/__init__.py:4112), see ye3t_b200/packing.py. */
typedef struct {
  int64_t nmax, lmax;             /* radial channels 1..nmax, l = 0..lmax */
  int64_t smem_entries;           /* complex entries per atom held in shared memory */
  int64_t feature_count;
  int64_t item_count;
  int64_t phase_count;
  int64_t sym_output_count;       /* symmetric outputs of one radial channel */
  const int32_t* items;           /* [item_count, 16] evaluation items grouped by phase: dispatch
                                     code, loop extents, K, coefficient offset, two feature
                                     indices, four shared-memory block bases */
  const double* item_coef;        /* dense coefficient tables of the items */
  const int32_t* phases;          /* [phase_count, 4]: slot-0 channel, slot-1 channel (-1 none),
                                     item begin, item end */
  const int32_t* sym_outputs;     /* [sym_output_count, 4]: l^2, term begin, term end, 0 */
  const uint32_t* sym_term_factors; /* [S] 4 x uint8 input components (255 = unused) */
  const double* sym_term_coeff;     /* [S] */
  /* adjoint only: items of one shape paired per phase (one per half-warp) */
  int64_t group_count;
  const int32_t* groups;          /* [group_count, 2] item indices (second -1: odd item out; both -1:
                                     null pair, skipped), by item class (one adjoint launch each)
                                     then phase; classes 2 and 3 are cut into equal runs, one per warp */
  const int32_t* group_offsets;   /* [4, phase_count + 1]: first group of each (class, phase) */
  /* adjoint only: derivatives of the symmetric outputs listed per input
     component (l^2 + m + l inside a radial channel) */
  int64_t sym_grad_count;
  const int32_t* sym_grad_offsets; /* [(lmax+1)^2 + 1] */
  const int32_t* sym_grad_index;   /* [sym_grad_count, 2]: output, 4 x u8 remaining factors (255 unused) */
  const double* sym_grad_coeff;    /* [sym_grad_count]: multiplicity x monomial coefficient */
  int64_t sym_term_count;          /* S: entries of sym_term_factors / sym_term_coeff */
} y3b_ace_tables;

/* A-basis density for centres [center_begin, center_begin + center_count):
 *   A[i, n-1, l^2 + l + m] = sum_{j in row i} p[z_j] R_n(r_ij) Yc_lm(r_ij)
 * n = 1..nmax (ChebExpCos, ye3t/runtime/execution_plan.py:7298), complex
 * Condon-Shortley harmonics (:7479), per-neighbour-species prefactor as in
 * plain_site_basis_product (:7582), accumulated per centre over its sorted
 * CSR row (density_accumulate, :7913) by one warp, without atomics.
 * r_ij = minimum image of r_j - r_i in a cubic box.  A is complex128
 * [center_count, nmax, (lmax+1)^2]; row_offsets are relative to the first
 * centre's row (row_offsets[0] may be nonzero). */
int y3b_ace_density(const double* positions, const int32_t* species, int64_t atom_count,
                    int64_t center_begin, int64_t center_count, double box,
                    const int64_t* row_offsets, const int32_t* neighbors,
                    const double* species_prefactor, int64_t species_count, int64_t nmax,
                    int64_t lmax, double cutoff, double lambda, void* A, int32_t* status,
                    void* stream);

/* Features [atom_count, feature_count] complex128 of every word's factorized
 * schedule (ACEFactorizedScheduleReport.evaluate,
 * ye3t/couplings/__init__.py:2574) from the A-basis, with every symmetric
 * block Sym^k(V_l) -> V_Lambda (symmetric_power_product_plan_contraction,
 * ye3t/runtime/symmetric_power.py:879) formed on chip.  A is the complex128
 * [atom_count, nmax, (lmax+1)^2] output of y3b_ace_density. */
int y3b_ace_features(const y3b_ace_tables* tables, const void* A, int64_t atom_count, void* features,
                     void* stream);

/* As y3b_ace_features with A and features in dtype Y3B_C128 (as above) or
 * Y3B_C64 (complex64, evaluated in fp32 with the fp64 coefficient tables
 * rounded on load). */
int y3b_ace_features_typed(int dtype, const y3b_ace_tables* tables, const void* A, int64_t atom_count,
                           void* features, void* stream);

/* Per-atom energy e[i] = sum_f weights[species[i], f] Re(B[i, f]) with B
 * evaluated on chip and never stored (species/energy indexed like A). */
int y3b_ace_energy(const y3b_ace_tables* tables, const void* A, int64_t atom_count,
                   const int32_t* species, const double* weights, int64_t species_count,
                   double* energy, void* stream);

/* ------------------------------------------------------------------------
 * Force path (the reverse of the two kernels above).  E = sum_i sum_f
 * w[z_i, f] Re(B_if); the reference obtains its gradient by torch autograd
 * through evaluate_factorized_schedule_torch (ye3t/core/couplings.py:552-567),
 * the symmetric-power adjoint (execution_plan_cuda.cu:5272) and
 * density_accumulate_adjoint (ye3t/runtime/execution_plan.py:7987).
 * ---------------------------------------------------------------------- */

/* Per-atom energies and G = dE/dA (complex128, A's layout; B is holomorphic
 * in A so dE = Re(sum G dA)).  Species outside [0, species_count) set
 * Y3B_STATUS_INDEX_RANGE in *status (nullable) and use species 0; an adjoint
 * item grouped into a class whose bounds it exceeds sets Y3B_STATUS_TABLE
 * and is skipped. */
int y3b_ace_energy_grad(const y3b_ace_tables* tables, const void* A, int64_t atom_count,
                        const int32_t* species, const double* weights, int64_t species_count,
                        double* energy, void* dEdA, int32_t* status, void* stream);

/* Per-edge g_e = dE_i/dd_e (f64 [E, 3], d_e = r_j - r_i minimum image) for the
 * rows of centres [center_begin, center_begin + center_count), from dEdA of
 * those centres (plain_site_basis_product_adjoint,
 * ye3t/runtime/execution_plan.py:7790, fused with the radial/harmonic
 * derivatives). */
int y3b_ace_edge_grad(const double* positions, const int32_t* species, int64_t atom_count,
                      int64_t center_begin, int64_t center_count, double box,
                      const int64_t* row_offsets, const int32_t* neighbors,
                      const double* species_prefactor, int64_t species_count, int64_t nmax,
                      int64_t lmax, double cutoff, double lambda, const void* dEdA,
                      double* edge_grad, int32_t* status, void* stream);

/* Recoupled form of the same adjoint (scalar bundles).  Each feature is a
 * short sum over intermediate L of contractions of Clebsch-Gordan coupled
 * channel pairs, F_f = sum_L W[f, L] sum_M (-1)^M I_A^L[M] I_B^L[-M], which
 * replaces the term-by-term schedules of evaluate_factorized_schedule_torch
 * (ye3t/core/couplings.py:552-567) for E = sum_i sum_f w[z_i, f] Re(B_if).
 * The tables are the device form of ye3t_b200.recoupling.RecoupledDeviceTables
 * (all arrays in device memory): per pass L the components
 * [pass_begin[L], pass_begin[L + 1]); comp holds two int4 per component,
 * (a, b, cg_begin, cg_count) and (m, own_begin, own_count, 0); own holds
 * (partner's first component in the pass, contraction) pairs; bp_* the
 * back-propagation entries of each A-row entry per pass. */
typedef struct {
  int32_t pass_count;          /* passes, one per intermediate L */
  int32_t max_pass_components; /* largest pass (shared-memory sizing) */
  int32_t row_width;           /* complex entries of one A row: nmax (lmax + 1)^2 */
  int32_t dot_count;           /* contractions: length of one species' weight row */
  int64_t component_count;     /* entries of comp / 8 */
  int64_t cg_count;            /* entries of cg_index and cg_value */
  int64_t own_count;           /* entries of own / 2 */
  int64_t bp_count;            /* entries of bp_gi, bp_other, bp_value */
  const int32_t* pass_begin;   /* [pass_count + 1] */
  const int32_t* comp;         /* [component_count, 8], 16-byte aligned */
  const int32_t* cg_index;     /* [cg_count]: m_a index | m_b index << 8 */
  const double* cg_value;      /* [cg_count] */
  const int32_t* own;          /* [own_count, 2], 8-byte aligned */
  const int32_t* bp_begin;     /* [pass_count * row_width + 1] */
  const int32_t* bp_gi;        /* [bp_count] component of the pass */
  const int32_t* bp_other;     /* [bp_count] A-row entry of the partner, -1 for a copied channel */
  const double* bp_value;      /* [bp_count] */
  int64_t feature_count;       /* features of the bundle */
  int64_t feat_count;          /* entries of feat_index and feat_weight */
  const int32_t* dot_begin;    /* [pass_count + 1] contractions of each pass */
  const int32_t* dot;          /* [dot_count, 4]: first local component of A, of B, feature range; 16-byte aligned */
  const int32_t* feat_index;   /* [feat_count] feature of each weight */
  const double* feat_weight;   /* [feat_count] W[f, d] */
  int32_t atoms_per_cta;       /* atoms sharing one CTA's table walk: 0 (one) or 1..4, within shared memory */
  int32_t threads_per_cta;     /* 0 (256), 256 or 512 */
} y3b_recoupled_tables;

/* Per-atom energies e_i = Re(sum_d k[z_i, d] T_d) and G = dE/dA (complex128,
 * A's layout [atom_count, row_width]), with contraction_weights k
 * [species_count, dot_count] (RecoupledPlan.energy_weights of the readout).
 * Species outside [0, species_count) set Y3B_STATUS_INDEX_RANGE and use
 * species 0; a table entry outside its pass or array sets Y3B_STATUS_TABLE and
 * is skipped.  Deterministic (fixed summation order, no atomics on data). */
int y3b_ace_recoupled_energy_grad(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                                  const int32_t* species, const double* contraction_weights,
                                  int64_t species_count, double* energy, void* dEdA, int32_t* status,
                                  void* stream);

/* Forward passes of the same plan: per-atom energies e_i = Re(sum_d k[z_i, d] T_d)
 * (each contraction once), or the features F [atom_count, feature_count]
 * complex128 in the bundle's feature order (ACEBundle.feature_offsets), with
 * the same status conventions. */
int y3b_ace_recoupled_energy(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                             const int32_t* species, const double* contraction_weights, int64_t species_count,
                             double* energy, int32_t* status, void* stream);
int y3b_ace_recoupled_features(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                               void* features, int32_t* status, void* stream);

/* Symmetric passes of the same plan for physical densities, A[n, l, -m] =
 * (-1)^m conj(A[n, l, m]) (real radial functions and prefactors, the densities
 * y3b_ace_density produces): only the M >= 0 components are formed, and dE/dA
 * is mirrored to m < 0.  Tables: ye3t_b200.recoupling.RecoupledSymTables
 * (comp (a, b, cg_begin, cg_count), (M, own_begin, own_count, (-1)^p); bp_gi
 * 2 * component + conj flag; mirror and dot as documented there).  A density
 * without the symmetry gives wrong results: use the general passes for it. */
typedef struct {
  int32_t pass_count;
  int32_t max_pass_components;
  int32_t row_width;
  int32_t dot_count;
  int64_t component_count;
  int64_t cg_count;
  int64_t own_count;
  int64_t bp_count;
  const int32_t* pass_begin; /* [pass_count + 1] */
  const int32_t* comp;       /* [component_count, 8], 16-byte aligned */
  const int32_t* cg_index;   /* [cg_count] */
  const double* cg_value;    /* [cg_count] */
  const int32_t* own;        /* [own_count, 2], 8-byte aligned */
  const int32_t* bp_begin;   /* [pass_count * row_width + 1] */
  const int32_t* bp_gi;      /* [bp_count] */
  const int32_t* bp_other;   /* [bp_count] */
  const double* bp_value;    /* [bp_count] */
  const int32_t* mirror;     /* [row_width] */
  const int32_t* dot_begin;  /* [pass_count + 1] */
  const int32_t* dot;        /* [dot_count, 4], 16-byte aligned */
  int32_t atoms_per_cta;     /* 0 (one) or 1..4, within shared memory */
  int32_t threads_per_cta;   /* 0 (256), 256 or 512 */
} y3b_recoupled_sym_tables;

int y3b_ace_recoupled_energy_grad_symmetric(const y3b_recoupled_sym_tables* tables, const void* A,
                                            int64_t atom_count, const int32_t* species,
                                            const double* contraction_weights, int64_t species_count,
                                            double* energy, void* dEdA, int32_t* status, void* stream);
int y3b_ace_recoupled_energy_symmetric(const y3b_recoupled_sym_tables* tables, const void* A, int64_t atom_count,
                                       const int32_t* species, const double* contraction_weights,
                                       int64_t species_count, double* energy, int32_t* status, void* stream);

/* The symmetric adjoint with the components' adjoints formed from dense tiles
 * of the contraction weights (ye3t_b200.recoupling.RecoupledTiles): per pass,
 * J[s] = sum_s' K[z][s, s'] I[s'] with K[z] symmetric, walked as tiles of
 * `rows` segments by the union of their columns, so that each shared-memory
 * read of a column component serves every row of the tile.  The same results
 * as y3b_ace_recoupled_energy_grad_symmetric (replaces the same reference
 * path: the autograd of ye3t/core/couplings.py:552-567 through the factorized
 * schedules), with the tile weights kval [species_count, rows * step_count]
 * (RecoupledTiles.tile_weights of the contraction weights) in place of the
 * contraction weights.  A CTA holds 32 / rows atoms (rows 8 or 16) and
 * threads_per_cta (256 or 512) threads; atoms_per_cta of `tables` is ignored.
 * atom_order (nullable) gives the order in which atoms are grouped into CTAs
 * (a species-sorted order lets a CTA's atoms share one species' weights);
 * energy and dEdA are indexed by atom either way. */
typedef struct {
  int32_t rows;              /* segments per tile: 8 or 16 */
  int32_t pass_count;        /* equal to the symmetric tables' */
  int64_t tile_count;
  int64_t step_count;
  int64_t item_count;
  int64_t group_count;
  int64_t pack_count;
  const int32_t* tile_begin;     /* [pass_count + 1] */
  const int32_t* tile_row;       /* [tile_count, rows]: local component of the row's M = 0, or -1 */
  const int32_t* tile_col_begin; /* [tile_count + 1], multiples of 4 */
  const int32_t* col_comp;       /* [step_count], 16-byte aligned */
  /* back-propagation work items: per pass, chunks of the A-row entries'
   * lists; item i of a pass (groups of `rows` items) writes a partial sum that
   * its entry adds in the order t_item lists them.  The items' records
   * (code, other, value as two int32) are packed per group, entry k of the
   * group's item j at bp_group_off[g] + k * rows + j, padded with null
   * records (other -1, value 0). */
  const int32_t* bp_item_begin;  /* [pass_count + 1] */
  const int32_t* t_item_begin;   /* [pass_count * row_width + 1] */
  const int32_t* t_item;         /* [item_count]: item index within its pass */
  const int32_t* bp_group_begin; /* [pass_count + 1] */
  const int32_t* bp_group_off;   /* [group_count + 1] */
  const int32_t* bp_pack;        /* [pack_count, 4], 16-byte aligned */
  /* step-2 work units per pass: (tile, first step, end step, kind), kind -1 a
   * whole tile, -2 the first column chunk of a cut tile, s >= 0 a later
   * chunk whose sums go to scratch slot s (slots of 512 * (L + 1) bytes,
   * scratch_slots * 512 bytes in all); fix (tile, first slot, slot count, 0)
   * adds a cut tile's later chunks in slot order */
  int64_t unit_count;
  int64_t fix_count;
  int32_t scratch_slots;
  const int32_t* unit_begin;     /* [pass_count + 1] */
  const int32_t* unit;           /* [unit_count, 4], 16-byte aligned */
  const int32_t* fix_begin;      /* [pass_count + 1] */
  const int32_t* fix;            /* [fix_count, 4], 16-byte aligned */
  const double* kval;            /* [species_count, rows * step_count], 16-byte aligned */
} y3b_recoupled_tile_tables;

int y3b_ace_recoupled_energy_grad_tiled(const y3b_recoupled_sym_tables* tables,
                                        const y3b_recoupled_tile_tables* tiles, const void* A,
                                        int64_t atom_count, const int32_t* atom_order, const int32_t* species,
                                        int64_t species_count, double* energy, void* dEdA, int32_t* status,
                                        void* stream);

/* Forces F_k = -dE/dr_k = sum_{e in row k} (g_e - g_rev(e)) from the rows of
 * all atoms (deterministic gather; rev(e) is the reverse edge). */
int y3b_forces_gather(const int64_t* row_offsets, const int32_t* neighbors, int64_t atom_count,
                      const double* edge_grad, double* forces, int32_t* status, void* stream);

/* Partial forces of local rows added into forces [atom_count, 3] (caller
 * zeroes it): F[k] += g_e, F[nbr] -= g_e (atomics).  Summing the partial
 * arrays of all atom blocks gives the forces. */
int y3b_forces_scatter(const int64_t* row_offsets, const int32_t* neighbors, int64_t center_begin,
                       int64_t center_count, int64_t atom_count, const double* edge_grad,
                       double* forces, void* stream);

/* ------------------------------------------------------------------------
 * Measurement support: an FP64 / FP32 FMA throughput kernel used to measure
 * the CUDA-core roofline.  Returns the flop count of one launch in *flops. */
int y3b_fma_peak_launch(int dtype, int32_t blocks, int32_t threads, int32_t iterations,
                        void* sink, double* flops, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* YE3T_B200_H */
