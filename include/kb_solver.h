/*
 * kb_solver.h -- C ABI of the kernel-bench B200 solver kernels (libkb_solver.so, sm_100a).
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream handle (cudaStream_t
 * passed as void*), enqueues its work on that stream and returns an int status:
 *   KB_OK (0), KB_ERR_ARG (1: invalid size/argument), KB_ERR_LAUNCH (2: CUDA launch failure),
 *   KB_ERR_SIZE (3: S above KB_MAX_S or an unsupported shape).
 * Nothing here allocates device memory; callers own every buffer.  Conventions:
 *   - float tensors are fp32, row-major, contiguous; a "[C,S]" array has row stride S;
 *   - node_* / leaf_state arrays are int32; row/split index arrays are int64;
 *   - boolean masks are uint8 (0/1);
 *   - jumps: [K,S] int32 pointer-doubling table, jumps[r*S+s] = 2^r-th ancestor of s or -1,
 *     K = ceil(log2(max_ancestor_depth)) (kb_build_jumps builds it);
 *   - compact levels: internal species nodes grouped by depth, deepest level first
 *     (lv_ptr int64 [n_levels+1], lv_par/lv_c1/lv_c2 int32).
 * References are to the reference project (SisyphusMountain/kernel-bench), file:line.
 */
#ifndef KB_SOLVER_H
#define KB_SOLVER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KB_MAX_S 8192

/* Version of this ABI (bumped on any signature change). */
int kb_abi_version(void);

/* Build the pointer-doubling ancestor table from node_parent on the device.
 * No reference counterpart (the reference caches an equivalent table on the host,
 * kbench/core/kernels/wave_step.py:35-55 _get_jumps). */
int kb_build_jumps(const int* node_parent, int S, int K, int* jumps, void* stream);

/* ---- E-step (kbench/core/kernels/e_step.py) ------------------------------------------- */

/* Replaces e_fixed_point_triton (e_step.py:438-501): iterate E <- F(E) on the device until
 * max|dE| < tol or max_iter iterations, then one more application for E_s1/E_s2/Ebar.
 * E_tmp is a [G,S] ping-pong buffer; *iters_out (device int) receives the iteration count. */
int kb_e_fixed_point(const float* E0, float* E_out, float* E_tmp, float* E_s1, float* E_s2, float* Ebar,
                     const float* log_pS, const float* log_pD, const float* log_pL, const float* max_coupling,
                     const float* col_log_probs, const int* node_parent, const int* node_child1,
                     const int* node_child2, const int* jumps, int K, int S, int G, int max_iter, double tol,
                     int use_col_weights, int* iters_out, void* stream);

/* Allocation-free variant of kb_e_fixed_point, for callers that cannot allocate device memory
 * (a host that owns all device memory through its own pool, or that must not trigger an
 * allocation at this point).  It has no counterpart in the reference.  Same inputs, outputs and
 * semantics as kb_e_fixed_point, without the E_tmp argument: the ping-pong buffer is a file-scope
 * device array of KB_NOALLOC_ESTEP_MAX floats (256 KiB, held by every GPU that loads the library
 * until exit).  G*S above KB_NOALLOC_ESTEP_MAX returns KB_ERR_SIZE.  The first call on a device
 * looks the array's address up (cudaGetSymbolAddress, no allocation) -- make it before any stream
 * capture.  The address is cached per device ordinal for the process's lifetime: it assumes the
 * CUDA runtime's primary context on that device (no cudaDeviceReset between calls, no other
 * driver context made current).  All calls share the array; calls that overlap on the GPU race. */
#define KB_NOALLOC_ESTEP_MAX 65536
int kb_e_fixed_point_noalloc(const float* E0, float* E_out, float* E_s1, float* E_s2, float* Ebar,
                             const float* log_pS, const float* log_pD, const float* log_pL,
                             const float* max_coupling, const float* col_log_probs, const int* node_parent,
                             const int* node_child1, const int* node_child2, const int* jumps, int K, int S, int G,
                             int max_iter, double tol, int use_col_weights, int* iters_out, void* stream);

/* Replaces _launch_e_step_forward_2d (e_step.py:244-287): one E application per item row;
 * max_diff_out [G] may be NULL. */
int kb_e_step_forward(const float* E, float* E_new, float* E_s1, float* E_s2, float* Ebar, float* max_diff_out,
                      const float* log_pS, const float* log_pD, const float* log_pL, const float* max_coupling,
                      const float* col_log_probs, const int* node_parent, const int* node_child1,
                      const int* node_child2, const int* jumps, int K, int S, int G, int use_col_weights,
                      void* stream);

/* Replaces _TritonEStep2D.backward (e_step.py:325-409; kernels :102-241): VJP of one E
 * application. g_* may be NULL (zero cotangent). grad_col [S] is overwritten (sum over rows). */
int kb_e_step_vjp(const float* E, const float* E_new, const float* E_s1, const float* E_s2, const float* Ebar,
                  const float* log_pS, const float* log_pD, const float* log_pL, const float* col_log_probs,
                  const int* node_parent, const int* node_child1, const int* node_child2, const int* jumps, int K,
                  const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1, const int* lv_c2,
                  const float* g_new, const float* g_s1, const float* g_s2, const float* g_ebar, float* grad_E,
                  float* grad_pS, float* grad_pD, float* grad_pL, float* grad_mc, float* grad_col, int S, int G,
                  int use_col_weights, void* stream);

/* Replaces the E-adjoint solve and the E-step parameter VJP of _implicit_grad.py:373-475 (the
 * BiCGSTAB of :28-94 with one e_step VJP per matvec) for ONE shared row, in one launch:
 *   q  = g_E + d/dE[n_fam * log2(1 - mean 2^E)] + VJP_E(E_s1, E_s2, Ebar cotangents),
 *   solve (I - J_E^T) w = q with the reference's stopping and breakdown rules,
 *   grad_params [5,S] = cotangents of (log_pS, log_pD, log_pL, max_coupling, col_log_probs) from
 *   the E step at w with Ebar cotangent g_Ebar (the caller adds the direct accumulators).
 * work: KB_EADJ_WORK_VECTORS * S floats of device scratch.  status [2] = (0 converged / 1 not,
 * iterations); rel_out [1] = last relative residual.  All arrays are [S] (row 0). */
#define KB_EADJ_WORK_VECTORS 17
int kb_e_adjoint_solve(const float* E, const float* log_pS, const float* log_pD, const float* log_pL,
                       const float* max_coupling, const float* col_log_probs, const int* node_parent,
                       const int* node_child1, const int* node_child2, const int* jumps, int K,
                       const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1, const int* lv_c2,
                       const float* g_E, const float* g_Ebar, const float* g_E_s1, const float* g_E_s2, double n_fam,
                       int max_iter, double tol, double breakdown_tol, float* work, float* w_out,
                       float* grad_params, int* status, float* rel_out, int S, int use_col_weights, void* stream);

/* ---- exact-Hessian HVP: second-order contractions (newton/hvp_exact.py) ---------------- */

/* Replaces wave_backward_so (kbench/core/kernels/wave_so.py:213-250, kernel :37-210): for wave
 * rows w < W (global row ws + w), at the FIXED adjoint v [W,S], the tangent along (dPi, dPibar and
 * the d-constants) of the self-loop J^T v (d_out [W,S], plus the rows ws.. of d_rhs [C,S] when
 * d_rhs != NULL) and of the parameter buckets (d_aw [6,W,S]: aw0, aw1, aw2, aw345, aw3, aw4).
 * Constants at item * const_row_stride + s (item = item_idx[ws + w]); leaf_state [C] (NULL = no
 * leaf term) with leaf_logp / dleaf_logp at item * S + s; dts_r / d_dts [W,S] both or neither.
 * jumps [K,S] (ancestor doubling) and the compact levels give the path and subtree sums. */
int kb_wave_backward_so(const float* Pi, const float* dPi, const float* Pibar, const float* dPibar, const float* v,
                        long long ws, int W, const float* pibar_row_max, const float* mc, const float* DL,
                        const float* dDL, const float* Ebar, const float* dEbar, const float* E, const float* dE,
                        const float* SL1, const float* dSL1, const float* SL2, const float* dSL2,
                        long long const_row_stride, const float* col_log_probs, int use_col_weights,
                        const int* node_parent, const int* node_child1, const int* node_child2, const int* jumps,
                        int K, const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1,
                        const int* lv_c2, const int* leaf_state, const float* leaf_logp, const float* dleaf_logp,
                        const long long* item_idx, const float* dts_r, const float* d_dts, const float* d_rhs,
                        float* d_out, float* d_aw, int S, void* stream);

/* Replaces dts_backward_so (kbench/core/kernels/dts_so.py:233-303, kernels :24-230): for the
 * wave's N splits (children sl / sr, parent ws + reduce_idx, split log-probabilities, NULL =
 * zeros) at the FIXED adjoint v [W,S]: the tangents of the split cotangents, added with atomics
 * into d_rhs [C,S] and d_grad_pD / d_grad_pS / d_grad_mt (rows item * S), and of both Pibar VJP
 * trees, added into d_rhs (child rows) and d_grad_col [S].  Rates at item * param_row_stride + s
 * (item = item_idx[item_offset + reduce_idx]), mt / dmt at item * mt_row_stride + s.  ud / dud
 * [2N,S] are scratch. */
int kb_dts_backward_so(const float* Pi, const float* dPi, const float* Pibar, const float* dPibar, const float* v,
                       long long ws, const long long* sl, const long long* sr, const long long* reduce_idx,
                       const float* log_split_probs, int N, long long item_offset, const long long* item_idx,
                       const float* log_pD, const float* log_pS, const float* dlog_pD, const float* dlog_pS,
                       long long param_row_stride, const float* mt, const float* dmt, long long mt_row_stride,
                       const float* pibar_row_max, const float* col_log_probs, int use_col_weights,
                       const int* node_child1, const int* node_child2, const long long* lv_ptr, int n_levels,
                       const int* lv_par, const int* lv_c1, const int* lv_c2, float* ud, float* dud, float* d_rhs,
                       float* d_grad_pD, float* d_grad_pS, float* d_grad_mt, float* d_grad_col, int S,
                       void* stream);

/* Replaces e_step_backward_so (kbench/core/kernels/e_step_so.py:188-220, kernels :23-185): the
 * tangent of the E-step VJP outputs at FIXED cotangents (g_new, g_ebar) [G,S] along (dE,
 * dE_new, dE_s1, dE_s2, dEbar, dlog_pS, dlog_pD, dlog_pL [G,S], dcol [S] or NULL).  Outputs
 * [G,S] (d_grad_col [S], overwritten: sum over rows). */
int kb_e_step_backward_so(const float* E, const float* E_new, const float* E_s1, const float* E_s2,
                          const float* Ebar, const float* log_pS, const float* log_pD, const float* log_pL,
                          const float* col_log_probs, const int* node_parent, const int* node_child1,
                          const int* node_child2, const int* jumps, int K, const long long* lv_ptr, int n_levels,
                          const int* lv_par, const int* lv_c1, const int* lv_c2, const float* g_new,
                          const float* g_ebar, const float* dE, const float* dE_new, const float* dE_s1,
                          const float* dE_s2, const float* dEbar, const float* dlog_pS, const float* dlog_pD,
                          const float* dlog_pL, const float* dcol, float* d_grad_E, float* d_grad_pS,
                          float* d_grad_pD, float* d_grad_pL, float* d_grad_mc, float* d_grad_col, int S, int G,
                          int use_col_weights, void* stream);

/* Column sums of one wave's six parameter buckets in the exact-Hessian HVP (the glue of
 * newton/hvp_exact.py:264-281 that sums the contraction's and the tangent adjoint's aw buckets):
 * c_aw [6,W,S] (aw0, aw1, aw2, aw345, aw3, aw4, from kb_wave_backward_so) plus l_aw* [W,S] (the
 * same buckets from kb_wave_adjoint), added into [S] accumulators: d_pD += aw0, d_pS += aw345,
 * d_E += aw0 + aw2, d_Ebar += aw1, d_Es1 += aw4, d_Es2 += aw3, d_mc += aw2 (fixed summation order). */
int kb_hvp_aw_accumulate(const float* c_aw, const float* l_aw0, const float* l_aw1, const float* l_aw2,
                         const float* l_aw345, const float* l_aw3, const float* l_aw4, int W, int S, float* d_pD,
                         float* d_pS, float* d_E, float* d_Ebar, float* d_Es1, float* d_Es2, float* d_mc,
                         void* stream);

/* ---- parameter extraction (kbench/core/parameters/extract_parameters.py) ---------------- */

/* Replaces col_valid_log_normalizer (extract_parameters.py:41-65): norm_out[s] =
 * -log2(max(1 - mass[s], FLT_MIN)) where 1 - mass[s] > 0, else -inf, mass[s] = sum of
 * 2^col_log_probs over the first max_ancestor_depth nodes of s's root path (self first, summed in
 * that order).  One launch; S <= KB_MAX_S. */
int kb_col_normalizer(const float* col_log_probs, const int* node_parent, int max_ancestor_depth, int S,
                      float* norm_out, void* stream);

/* VJP of kb_col_normalizer: grad_col_log_probs [S] (overwritten) from the cotangent g_norm [S].
 * The compact levels (internal nodes, deepest first) give the subtree sums; max_ancestor_depth
 * must cover every root path (as the static's does). */
int kb_col_normalizer_vjp(const float* col_log_probs, const int* node_parent, int max_ancestor_depth,
                          const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1,
                          const int* lv_c2, const float* g_norm, float* grad_col_log_probs, int S, void* stream);

/* ---- split reduction (kbench/core/kernels/dts_fused.py) ------------------------------- */

/* Replaces compute_dts_forward (dts_fused.py:171-231). out [W,S] must be pre-filled with -inf
 * (rows of inactive or split-less parents are not written). log_pD/log_pS are [rows,S] with row
 * stride param_row_stride (0: one shared row), row = item_idx[item_offset + parent].
 * out_row (may be NULL) remaps a parent's output row. */
int kb_dts_forward(const float* Pi, const float* Pibar, const long long* sl, const long long* sr,
                   const int* node_child1, const int* node_child2, const float* log_pD, const float* log_pS,
                   long long param_row_stride, const long long* item_idx, long long item_offset,
                   const float* log_split_probs, const long long* eq1_reduce_idx, int n_eq1,
                   const long long* ge2_ptr, const long long* ge2_parent_ids, int n_ge2,
                   const unsigned char* active_rows, float* out, const long long* out_row, int S, void* stream);

/* ---- forward wave (kbench/core/kernels/wave_step.py) ---------------------------------- */

/* Replaces compute_wave_step (wave_step.py:1128-1268): one Jacobi sweep of rows [ws, ws+W).
 * Reads pi_in rows [pi_ws, pi_ws+W), writes pi_out_rows[0..W); with store_final also writes the
 * final Pibar rows pibar[ws..ws+W) and pibar_row_max. residual [C] and dts [W,S] may be NULL.
 * Aliasing of pi_in/pi_out/pibar rows as done by kbench/core/inference/forward.py is allowed. */
int kb_wave_step(const float* pi_in, long long pi_ws, float* pi_out_rows, float* pibar, float* pibar_row_max,
                 float* residual, const float* dts, const float* mc, const float* dl, const float* ebar,
                 const float* e, const float* sl1, const float* sl2, long long const_row_stride,
                 const float* col_log_probs, int use_col_weights, const int* node_child1, const int* node_child2,
                 const int* jumps, int K, const int* leaf_state, const float* leaf_logp, const long long* item_idx,
                 int use_leaf, int store_final, int ws, int W, int S, void* stream);

/* Replaces compute_leaf_initial_wave_step (wave_step.py:1078-1126). */
int kb_leaf_initial(float* pi_out_rows, const float* mc, const float* dl, const float* ebar, const float* e,
                    const float* sl1, const float* sl2, long long const_row_stride, const float* col_log_probs,
                    int use_col_weights, const int* node_child1, const int* node_child2,
                    const int* node_subtree_start, const int* node_subtree_end, const int* leaf_state,
                    const float* leaf_logp, const long long* item_idx, int ws, int W, int S, void* stream);

/* Fused wave sweep: all pi_iters iterations of each listed row in one launch (leaf rows are
 * seeded as compute_leaf_initial_wave_step does; other rows start from their dts row).  Writes
 * the final Pi, Pibar rows and pibar_row_max -- the buffer state kbench/core/inference/
 * forward.py:60-115 leaves after the wave.  dts is [n_rows,S] aligned with rows. */
int kb_wave_sweep(const int* rows, int n_rows, const float* dts, float* pi, float* pibar, float* pibar_row_max,
                  float* residual, const float* mc, const float* dl, const float* ebar, const float* e,
                  const float* sl1, const float* sl2, long long const_row_stride, const float* col_log_probs,
                  int use_col_weights, const int* node_child1, const int* node_child2,
                  const int* node_subtree_start, const int* node_subtree_end, const int* jumps, int K,
                  const int* leaf_state, const float* leaf_logp, const long long* item_idx, int pi_iters, int S,
                  void* stream);

/* ---- backward (kbench/core/kernels/wave_backward.py) ---------------------------------- */

/* Replaces active_mask_from_rhs_absmax_fused (wave_backward.py:247-280). */
int kb_active_mask(const float* rhs, long long row_stride, int W, int S, float threshold, int strict_gt,
                   unsigned char* out, void* stream);

/* Replaces wave_backward_uniform_fused (wave_backward.py:1737-1867, Neumann solver):
 * per active row, v = sum_{n<=neumann_terms} (J^T)^n rhs and the parameter buckets aw0..aw4,
 * aw345 ([W,S] each; zero on inactive rows; v_k rows of inactive rows untouched).
 * const_mode: 0 shared [S] constants, 1 row-expanded [W,S], 2 item rows [G,S] via item_idx.
 * leaf_mode: 0 [S], 1 [G], 2 [G,S], 3 scalar. grad_col (may be NULL) is accumulated.
 * last_relres (may be NULL; [W]): |last Neumann term| / max(|v|, FLT_MIN) per row, 0 on inactive
 * rows -- the return_last_increment output (wave_backward.py:1596-1613).
 * initial_v (may be NULL; [W,S] rows at initial_v_row_stride): the warm-started solve of the
 * initial_v option (wave_backward.py:1493-1534): v = initial_v, then neumann_terms fixed-point
 * updates v <- rhs + J^T v per active row; inactive rows' v_k rows are set to initial_v; last_relres
 * must then be NULL (the reference returns no last increment for it, :1596-1600). */
int kb_wave_adjoint(const float* Pi, const float* Pibar, const float* pibar_row_max, const float* dts,
                    const float* rhs, long long rhs_row_stride, const unsigned char* active, const float* dl,
                    const float* ebar, const float* e, const float* sl1, const float* sl2, int const_mode,
                    const float* col_log_probs, int use_col_weights, const int* node_child1,
                    const int* node_child2, const int* node_parent, const int* jumps, int K,
                    const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1, const int* lv_c2,
                    int use_leaf_index, const int* leaf_state, const float* leaf_logp, int leaf_mode,
                    const float* leaf_term, const long long* item_idx, int neumann_terms,
                    const float* initial_v, long long initial_v_row_stride, float* grad_col, float* v_k,
                    float* aw0, float* aw1, float* aw2, float* aw345, float* aw3, float* aw4, float* last_relres,
                    int ws, int W, int S, void* stream);

/* The self_loop_grad_targets option of wave_backward_uniform_fused (wave_backward.py:1615-1640 and
 * the ACCUM_GRADS branch of its parameter store, :1208-1262): the column sums over the wave's rows
 * of the buckets kb_wave_adjoint wrote ([W,S] each, zero on inactive rows) are ADDED into the
 * caller's fp32 targets: grad_log_pD += aw0 and grad_log_pS += aw345 ([S] each with
 * param_grad_vector, else one scalar each: the sums over all columns), grad_E += aw0 + aw2,
 * grad_Ebar += aw1, grad_E_s1 += aw4, grad_E_s2 += aw3, grad_mt += aw2 ([S] each).  Sums in fp64
 * in a fixed order (the reference adds row by row with atomics).  col_tot: [2,S] fp64 scratch,
 * required without param_grad_vector (may be NULL with it). */
int kb_wave_adjoint_accum_targets(const float* aw0, const float* aw1, const float* aw2, const float* aw345,
                                  const float* aw3, const float* aw4, int W, int S, float* grad_log_pD,
                                  float* grad_log_pS, int param_grad_vector, float* grad_E, float* grad_Ebar,
                                  float* grad_E_s1, float* grad_E_s2, float* grad_mt, double* col_tot,
                                  void* stream);

/* The operator of the self-loop solve, A x = x - J_self^T x, per active row (one application of
 * the single-term kernel with OUTPUT_A, wave_backward.py:485-638, as the GMRES self-loop solver
 * calls it, :1439-1492); y rows of inactive rows are zero.  Same row coefficients as
 * kb_wave_adjoint (arguments as there); x rows at stride x_row_stride, y dense [W,S]. */
int kb_wave_adjoint_apply(const float* Pi, const float* Pibar, const float* pibar_row_max, const float* dts,
                          const unsigned char* active, const float* dl, const float* ebar, const float* e,
                          const float* sl1, const float* sl2, int const_mode, const float* col_log_probs,
                          int use_col_weights, const int* node_child1, const int* node_child2,
                          const int* node_parent, const int* jumps, int K, const long long* lv_ptr, int n_levels,
                          const int* lv_par, const int* lv_c1, const int* lv_c2, int use_leaf_index,
                          const int* leaf_state, const float* leaf_logp, int leaf_mode, const float* leaf_term,
                          const long long* item_idx, const float* x, long long x_row_stride, float* y, int ws,
                          int W, int S, void* stream);

/* Replaces dts_cross_backward_accum_fused (wave_backward.py:2319-2535): per split, the Pi
 * cotangents of both children (including the merged speciation terms) are added into
 * accumulated_rhs; the staged Pibar u_d rows / sums / side flags (output_ud) or grad_Pibar_l/r
 * rows are written; parameter cotangents are accumulated (accum_param/accum_mt) or written per
 * split.  Parameter/gradient addressing: value at base + item*row_stride + s*elem_stride. */
int kb_dts_adjoint(const float* Pi, const float* Pibar, const float* v_k, const unsigned char* active,
                   const long long* sl, const long long* sr, const long long* reduce_idx, const float* wlsp,
                   const float* log_pD, long long pD_row_stride, int pD_elem_stride, const float* log_pS,
                   long long pS_row_stride, int pS_elem_stride, const long long* item_idx, const int* node_child1,
                   const int* node_child2, float* accumulated_rhs, int output_ud, float* pibar_ud, float* pibar_A,
                   unsigned char* side_active, float side_threshold, int side_threshold_enabled,
                   int skip_inactive_zero, float* grad_Pibar_l, float* grad_Pibar_r, int accum_param,
                   float* grad_log_pD, float* grad_log_pS, long long gp_row_stride, int gp_elem_stride,
                   float* param_pD, float* param_pS, int accum_mt, float* grad_mt, long long gmt_row_stride,
                   int gmt_elem_stride, const float* mt, long long mt_row_stride, int mt_elem_stride,
                   const float* pibar_row_max, int ws, int N, int S, void* stream);

/* Replaces _pibar_ud_side_active_kernel (wave_backward.py:2536-2567). */
int kb_side_active(const float* pibar_ud, int rows, int S, float threshold, int threshold_enabled,
                   unsigned char* out, void* stream);

/* Replaces uniform_cross_pibar_vjp_tree_from_ud_fused (wave_backward.py:2748-2896): per active
 * split side, in-place subtree sums of pibar_ud, then p'(A - subtree) into the child's adjoint
 * row and grad_col (may be NULL). */
int kb_pibar_vjp_tree(const float* Pi, const float* col_log_probs, int use_col_weights, float* pibar_ud,
                      const float* pibar_A, const unsigned char* side_active, const long long* sl,
                      const long long* sr, const long long* reduce_idx, const unsigned char* active,
                      const float* pibar_row_max, const long long* lv_ptr, int n_levels, const int* lv_par,
                      const int* lv_c1, const int* lv_c2, float* accumulated_rhs, float* grad_col, int N, int S,
                      void* stream);

/* ---- fused level engine (no reference counterpart: B200 schedule of the same math) ------- */

/* Linear-space per-column constants of the wave update for [G,S] item rows (n = G*S):
 * linA = 2^dl + 2^ebar, linB = 2^(mc+e), linC1 = 2^sl1, linC2 = 2^sl2. */
int kb_lin_consts(const float* dl, const float* ebar, const float* mc, const float* e, const float* sl1,
                  const float* sl2, int n, float* linA, float* linB, float* linC1, float* linC2, void* stream);

/* Forward of one dependency level (replaces, for the rows listed, compute_dts_forward +
 * compute_leaf_initial_wave_step + pi_iters x compute_wave_step of kbench/core/inference/
 * forward.py:60-115): per row (one CTA) the split reduction over its splits
 * [split_ptr[b], split_ptr[b+1]) of (sl, sr, lsp) -- or the leaf seed for split-less leaf rows --
 * then all pi_iters iterations on chip; writes the final pi, pibar rows, pibar_row_max, the split
 * reduction (dts_save, may be NULL) and the last-iteration residual (may be NULL).
 * fallback_count (device int, may be NULL) counts rows recomputed in log space.  Uniform column
 * weights only (use_col_weights must be 0).  tour_tables: [3,NTV] uint32 tables of
 * kbench_b200/tree.py pack_forward() (children columns, byte offsets of the children's and the
 * column's own Euler-tour slots); when given and kb_tour_layout(S) accepts S, the tour kernel
 * runs (dts_save and tour_consts, from kb_lin_consts_tour, must then be non-NULL).  Otherwise
 * packed: the [5,NTV] tables of pack_columns(..., ntv) with NTV from the engine width, of which
 * this kernel reads rows 0-3 (children, Euler-tour enter/exit, preorder start/end, parent |
 * first-child flag; two 16-bit fields each).  The row iterations run in linear space relative to
 * a per-row scale; rows outside its exact range (see kb_engine.cu) are recomputed in log space
 * and counted in fallback_count; force_log_space != 0 sends every row there (set by the caller
 * when a constant 2^dl+2^ebar, 2^(mc+e), 2^sl1 or 2^sl2 is below 2^-26). */
int kb_level_forward(const int* rows, const long long* split_ptr, int n_rows, const long long* sl,
                     const long long* sr, const float* lsp, const float* Pi_src, const float* Pibar_src, float* pi,
                     float* pibar, float* pibar_row_max, float* dts_save, float* residual, int* fallback_count,
                     const float* mc, const float* dl, const float* ebar, const float* e, const float* sl1,
                     const float* sl2, const float* leaf_logp, const float* linA, const float* linB,
                     const float* linC1, const float* linC2, const float* log_pD, const float* log_pS,
                     long long param_row_stride, long long const_row_stride, const float* col_log_probs,
                     int use_col_weights, const int* node_parent, const int* node_child1, const int* node_child2,
                     const int* node_subtree_start, const int* node_subtree_end, const int* jumps, int K,
                     const long long* item_idx, const int* leaf_state, const unsigned* packed,
                     const unsigned* tour_tables, const float* tour_consts, int force_log_space, int pi_iters,
                     int S, void* stream);

/* The whole forward wave sweep in ONE persistent launch with a dataflow schedule (replaces the
 * per-level kb_level_forward launches, same per-row arithmetic as its tour kernel): a row starts
 * as soon as all of its child rows are final instead of after the whole previous level.
 * Rows' splits: row_split_ptr [C+1] into sl / sr / lsp (row-id order).  dep0 [C]: number of
 * distinct child rows; ready0 [n_ready0]: the rows with dep0 = 0; par_ptr [C+1] / par_idx: the
 * distinct parent rows of each row.  Scratch: queue [C], remaining [C] (int), counters [3]
 * (head, tail, error flag; error != 0 after the launch means a wait gave up after max_polls
 * polls: results are then invalid).  Pi / Pibar child rows are read from pi / pibar (in place).
 * force_log_flag (device int, may be NULL): a nonzero value forces the log-space iteration like
 * force_log_space, decided on the device (no host round trip).  start_order (int32 [C], may be
 * NULL): a fixed start order of all rows, every row after its child rows; CTAs take rows in that
 * order, each waiting (bounded) until its children are done, instead of taking rows as they
 * become ready.  Other arguments as kb_level_forward's tour path. */
int kb_flow_forward(int C, const long long* row_split_ptr, const long long* sl, const long long* sr,
                    const float* lsp, const int* dep0, const int* ready0, int n_ready0, const long long* par_ptr,
                    const int* par_idx, int* queue, int* remaining, unsigned* counters, long long max_polls,
                    float* pi, float* pibar, float* pibar_row_max, float* dts_save, float* residual,
                    int* fallback_count, const float* mc, const float* dl, const float* ebar, const float* e,
                    const float* sl1, const float* sl2, const float* leaf_logp, const float* log_pD,
                    const float* log_pS, long long param_row_stride, long long const_row_stride,
                    const int* node_parent, const int* node_child1, const int* node_child2,
                    const int* node_subtree_start, const int* node_subtree_end, const int* jumps, int K,
                    const long long* item_idx, const int* leaf_state, const unsigned* tour_tables,
                    const float* tour_consts, int force_log_space, const int* force_log_flag, const int* start_order,
                    int pi_iters, int S, void* stream);

/* The tour kernel's per-column constants, interleaved and zero-padded to NTV = kb_tour_layout(S):
 * out4 [G, NTV, 4] = (2^dl + 2^ebar, 2^(mc+e), 2^sl1, 2^sl2) from the [G,S] constant rows. */
int kb_lin_consts_tour(const float* dl, const float* ebar, const float* mc, const float* e, const float* sl1,
                       const float* sl2, int G, int S, float* out4, void* stream);

/* Layout of the forward tour kernel for S columns (host only): padded width NTV (smallest power
 * of two > S, at least 64), threads per row and columns per thread.  Returns 3 (KB_ERR_SIZE) with
 * *ntv = 0 when NTV would exceed 4096 (kb_level_forward then uses its packed-table kernel). */
int kb_tour_layout(int S, int* ntv, int* threads, int* cols_per_thread);

/* Layout of the backward kernels (kb_level_backward, kb_flow_backward) for S columns (host only;
 * no reference counterpart -- the reference sizes its Triton blocks per launch): the engine's
 * padded width NTV (that of the packed_padded tables), threads per CTA (always whole warps, at
 * most 1024) and columns per thread (1, 2, 4 or 8, threads x columns = NTV).  Returns 3
 * (KB_ERR_SIZE) where that needs more than 8 columns per thread (S = 8192) or S > KB_MAX_S. */
int kb_backward_layout(int S, int* ntv, int* threads, int* cols_per_thread);

/* Backward of one dependency level (replaces, for the rows listed, active_mask_from_rhs_absmax_
 * fused + compute_dts_forward + wave_backward_uniform_fused + dts_cross_backward_accum_fused +
 * uniform_cross_pibar_vjp_tree_from_ud_fused as driven by kbench/api/_implicit_grad.py:
 * 190-353).  Persistent: min(n_rows, n_slots) CTAs, CTA b takes rows b, b+grid, ...  Per active
 * row: the Neumann adjoint, its parameter and column cotangents (summed in shared memory per CTA
 * and added to that CTA's fp64 slot of grad_slots [n_slots, 8, NTV] at the end; slots persist
 * across levels and are reduced in a fixed order by kb_reduce_grad_slots), and every split's child
 * cotangents added into accumulated_rhs.  dts_saved may be NULL (recomputed); v_out [C,S] (may be
 * NULL) receives the solved adjoint row of every active row.  packed_padded: [5,NTV] tables of
 * pack_columns(..., ntv) with NTV = threads x columns-per-thread (kbench_b200/tree.py): rows 0-3
 * by column, row 4 by preorder position (subtree end | parent's position). */
int kb_level_backward(const int* rows, const long long* split_ptr, int n_rows, const long long* sl,
                      const long long* sr, const float* lsp, const float* Pi, const float* Pibar,
                      const float* pibar_row_max, const float* dts_saved, float* accumulated_rhs, float* v_out,
                      double* grad_slots, int n_slots, float threshold, int strict_gt, float side_threshold,
                      int side_threshold_enabled, int neumann_terms, const float* mc, const float* dl,
                      const float* ebar, const float* e, const float* sl1, const float* sl2,
                      const float* leaf_logp, const float* log_pD, const float* log_pS,
                      long long param_row_stride, long long const_row_stride, const float* col_log_probs,
                      int use_col_weights, const long long* item_idx, const int* leaf_state,
                      const unsigned* packed_padded, int S, void* stream);

/* The whole backward in ONE persistent launch with a dataflow schedule (replaces the per-level
 * kb_level_backward launches, same per-row arithmetic): a row starts as soon as every row that
 * lists it as a split child (its parents) has added its cotangents.  row_split_ptr [C+1] into sl /
 * sr / lsp (row-id order); dep0 [C]: number of distinct parent rows; ready0 [n_ready0]: rows
 * without parents (the roots); child_ptr [C+1] / child_idx: the distinct child rows of each row.
 * Scratch queue [C], remaining [C], counters [3] (head, tail, error: nonzero after the launch =
 * a wait gave up after max_polls polls, results invalid).  grad_slots [n_slots, 8, NTV]: one per
 * persistent CTA (n_slots CTAs run).  edge_rows (may be NULL: each split then adds its children's
 * cotangents into accumulated_rhs with fp32 atomics, whose order varies run to run): [2N,S]
 * scratch, row 2i / 2i+1 = split i's contribution to its left / right child (zeros when the row
 * is inactive); a row's adjoint is then accumulated_rhs[row] (its seed) plus its incoming rows
 * in_edge[in_ptr[row] .. in_ptr[row+1]) (edge ids 2i + side, ascending), added left to right, and
 * the column sums move to the fp64 slots after every row: the adjoint rows are bitwise the same
 * every run.  Other arguments as kb_level_backward. */
int kb_flow_backward(int C, const long long* row_split_ptr, const long long* sl, const long long* sr,
                     const float* lsp, const int* dep0, const int* ready0, int n_ready0, const long long* child_ptr,
                     const int* child_idx, int* queue, int* remaining, unsigned* counters, long long max_polls,
                     const float* Pi, const float* Pibar, const float* pibar_row_max, const float* dts_saved,
                     float* accumulated_rhs, float* v_out, double* grad_slots, int n_slots, float threshold,
                     int strict_gt, float side_threshold, int side_threshold_enabled, int neumann_terms,
                     const float* mc, const float* dl, const float* ebar, const float* e, const float* sl1,
                     const float* sl2, const float* leaf_logp, const float* log_pD, const float* log_pS,
                     long long param_row_stride, long long const_row_stride, const float* col_log_probs,
                     int use_col_weights, const long long* item_idx, const int* leaf_state,
                     const unsigned* packed_padded, const int* start_order, float* edge_rows,
                     const long long* in_ptr, const int* in_edge, int S, void* stream);

/* Number of backward CTAs that are resident at once on this device for S columns (SMs x CTAs
 * per SM): the slot count to give kb_level_backward / kb_flow_backward (host only). */
int kb_backward_ctas(int S, int* n_ctas);

/* Host query (no device work): CTAs of kb_flow_forward's persistent grid for rows of S columns
 * (SMs x resident CTAs per SM of its tour kernel). */
int kb_forward_ctas(int S, int* n_ctas);

/* Host-only (no device work; all pointers are HOST memory): the start order of a critical-path
 * list schedule of n rows on n_workers identical workers.  pred_ptr [n+1] / pred_idx: the rows
 * each row waits for; succ_ptr [n+1] / succ_idx: the rows waiting on each row (the same edges
 * reversed); cost [n] > 0: a row's modelled duration.  A ready row with the largest level (its cost
 * plus the largest level of its successors) starts first.  order_out [n]: rows in start order --
 * every row after its predecessors (the start_order of kb_flow_forward / kb_flow_backward);
 * makespan_out (may be NULL): the schedule's modelled length.  KB_ERR_ARG on a cycle or edges that
 * do not match the counts. */
int kb_list_schedule(int n, const long long* pred_ptr, const int* pred_idx, const long long* succ_ptr,
                     const int* succ_idx, const double* cost, int n_workers, int* order_out, double* makespan_out);

/* Fixed-order sum of kb_level_backward's fp64 slots -> out8 [8,S] fp32: the cotangents of
 * log_pD, log_pS, max_coupling, E, Ebar, E_s1, E_s2 and col_log_probs (in that order). */
int kb_reduce_grad_slots(const double* grad_slots, int n_slots, int S, float* out8, void* stream);

/* ---------------- forward-mode tangent (the tangent benchmark config) ---------------- */

/* E-step tangent fixed point (replaces e_tangent_fixed_point, kbench/core/kernels/
 * e_step_tangent.py:174-208, with its kernel _e_step_tangent_2d_kernel :23-150) for D directions
 * at once: one persistent CTA per direction iterates dE <- J_E dE + J_p dp at the frozen E_star
 * [G,S] from dE0 (NULL = zero) until max|dE_new - dE| <= tol * max(1, max|dE_new|) over the G rows
 * or max_iter, then applies once more for dE_s1 / dE_s2 / dEbar.  Direction-major buffers
 * [D,G,S]: dlog_pS, dlog_pD, dlog_pL, dmax_coupling, dE0, dE_out, scratch, dE_s1, dE_s2, dEbar;
 * iters_out [D] (may be NULL).  jumps / K: the ancestor jump table of kb_build_jumps. */
int kb_e_tangent_fixed_point(const float* E_star, const float* dlog_pS, const float* dlog_pD,
                             const float* dlog_pL, const float* dmax_coupling, const float* log_pS,
                             const float* log_pD, const float* log_pL, const float* max_coupling,
                             const float* col_log_probs, int use_col_weights, const int* node_child1,
                             const int* node_child2, const int* jumps, int K, int G, int S, int D, int max_iter,
                             float tol, const float* dE0, float* dE_out, float* scratch, float* dE_s1,
                             float* dE_s2, float* dEbar, int* iters_out, void* stream);

/* One linearised E application (replaces _launch_e_step_tangent_2d, e_step_tangent.py:153-171)
 * for D directions x G rows: dE_new, dE_s1, dE_s2, dEbar [D,G,S]; max_diff [D*G] (may be NULL). */
int kb_e_tangent_step(const float* E_star, const float* dE_in, const float* dlog_pS, const float* dlog_pD,
                      const float* dlog_pL, const float* dmax_coupling, const float* log_pS, const float* log_pD,
                      const float* log_pL, const float* max_coupling, const float* col_log_probs,
                      int use_col_weights, const int* node_child1, const int* node_child2, const int* jumps, int K,
                      int G, int S, int D, float* dE_new, float* dE_s1, float* dE_s2, float* dEbar,
                      float* max_diff, void* stream);

/* Tangent of the split reduction (replaces compute_dts_tangent, kbench/core/kernels/
 * dts_tangent.py:99-122): out[p,s] = sum over parent p's splits (order[ptr[p] .. ptr[p+1]),
 * indices into sl / sr / log_split_probs) of sum_k 2^(t_k - dts_r[p,s]) dt_k, in that fixed order
 * (no atomics); 0 where dts_r is -inf.  Parameters at item * param_row_stride + s, item =
 * item_idx[item_offset + p]. */
int kb_dts_tangent(const float* Pi, const float* Pibar, const float* dPi, const float* dPibar, const long long* sl,
                   const long long* sr, const float* log_split_probs, const long long* order, const long long* ptr,
                   int W, const int* node_child1, const int* node_child2, const float* log_pD,
                   const float* log_pS, const float* dlog_pD, const float* dlog_pS, long long param_row_stride,
                   const long long* item_idx, long long item_offset, const float* dts_r, float* out, int S,
                   void* stream);

/* Linearised wave step, n_iters in-place Jacobi steps on chip (replaces
 * compute_wave_step_tangent_selfloop, kbench/core/kernels/wave_tangent.py:339-389, and with
 * n_iters = 1 compute_wave_step_tangent :392-431): rows w < W read Pi_in / dPi_in at pi_ws + w,
 * write dPi_out[w] (dPi_out already offset to the wave; may alias dPi_in's rows) and, if
 * dPibar_out != NULL, dPibar_out[ws + w] from the last step.  Constants at item * const_row_stride
 * + s (item = item_idx[ws + w]); leaf_state_idx NULL = no leaf term; dts_reduced / d_dts [W,S]
 * both NULL or both given. */
int kb_wave_tangent(const float* Pi_in, const float* dPi_in, float* dPi_out, float* dPibar_out, long long ws,
                    long long pi_ws, int W, int S, int n_iters, const float* max_coupling, const float* dMC,
                    const float* DL, const float* dDL, const float* Ebar, const float* dEbar, const float* E,
                    const float* dE, const float* SL1, const float* dSL1, const float* SL2, const float* dSL2,
                    long long const_row_stride, const float* col_log_probs, int use_col_weights,
                    const int* node_child1, const int* node_child2, const int* jumps, int K,
                    const int* leaf_state_idx, const float* leaf_logp, const float* dleaf_logp,
                    const long long* item_idx, const float* dts_reduced, const float* d_dts, void* stream);

/* Tangent of one dependency level for D directions (replaces, for the rows listed,
 * compute_dts_tangent + compute_wave_step_tangent_selfloop as driven by newton/
 * forward_tangent.py:150-193 with self_iters = n_iters): one CTA per (row, direction) computes
 * the row's split tangent from the children's tangent rows, then n_iters Jacobi steps from a zero
 * tangent at the frozen primal row, and writes dPi / dPibar [D, C, S] (direction stride
 * dir_stride).  dts_saved: the forward's split reductions [C,S].  Tangent constants [D, G, S]
 * (direction stride tangent_dir_stride).  tour_tables: kbench_b200/tree.py pack_forward(); S must
 * be accepted by kb_tour_layout.  pair_tables (may be NULL): pack_tour_pair(), the enter / exit
 * offsets of the two-direction layout; when given, directions run in pairs per CTA (sharing the
 * primal weights and the addressing) and an odd last direction alone. */
int kb_level_tangent(const int* rows, const long long* split_ptr, int n_rows, const long long* sl,
                     const long long* sr, const float* lsp, const float* Pi, const float* Pibar,
                     const float* dts_saved, float* dPi, float* dPibar, long long dir_stride, int D, const float* mc,
                     const float* dl, const float* ebar, const float* e, const float* sl1, const float* sl2,
                     const float* leaf_logp, const float* log_pD, const float* log_pS, long long param_row_stride,
                     long long const_row_stride, const float* dMC, const float* dDL, const float* dEbar,
                     const float* dE, const float* dSL1, const float* dSL2, const float* dleaf, const float* dpD,
                     const float* dpS, long long tangent_dir_stride, const long long* item_idx,
                     const int* leaf_state, const unsigned* tour_tables, const unsigned* pair_tables,
                     int n_iters, int S, void* stream);

/* The whole tangent sweep for D (even) directions in ONE persistent launch with a dataflow
 * schedule (replaces the per-level kb_level_tangent launches, same per-row arithmetic as its
 * two-direction kernel): work items are (direction pair, row); an item starts when the same
 * pair's child rows are done.  Dependency arrays as kb_flow_forward (dep0 = distinct child rows,
 * ready0 = rows with none, par_ptr / par_idx = distinct parents).  Scratch queue / remaining
 * [C * D/2] int, counters [3] (head, tail, error; error != 0 = a wait gave up, results invalid).
 * pair_tables required.  Other arguments as kb_level_tangent. */
int kb_flow_tangent(int C, const long long* row_split_ptr, const long long* sl, const long long* sr,
                    const float* lsp, const int* dep0, const int* ready0, int n_ready0, const long long* par_ptr,
                    const int* par_idx, int* queue, int* remaining, unsigned* counters, long long max_polls,
                    const float* Pi, const float* Pibar, const float* dts_saved, float* dPi, float* dPibar,
                    long long dir_stride, int D, const float* mc, const float* dl, const float* ebar, const float* e,
                    const float* sl1, const float* sl2, const float* leaf_logp, const float* log_pD,
                    const float* log_pS, long long param_row_stride, long long const_row_stride, const float* dMC,
                    const float* dDL, const float* dEbar, const float* dE, const float* dSL1, const float* dSL2,
                    const float* dleaf, const float* dpD, const float* dpS, long long tangent_dir_stride,
                    const long long* item_idx, const int* leaf_state, const unsigned* tour_tables,
                    const unsigned* pair_tables, int n_iters, int S, void* stream);

/* ---- static builder: gene-tree topologies -> wave layout ------------------------------------
 * No reference counterpart: the reference reads this layout from an external capture
 * (kbench/runtime.py:47-60 make_static consumes it; capture/capture.py:17-18 notes that the
 * preprocessing is not part of the project).  The layout is the one kbench_b200/gen.py's host
 * generator writes (family_from_topologies + assemble_static); these entry points produce the
 * same arrays on the device for a batch of F families.
 *
 * Input: T topologies per family over G gene leaves, int32 left/right [F*T, 2G-1] (nodes
 * 0..G-1 are the gene leaves, G..2G-2 internal), int32 root [F*T], uint64 leaf_hash [F, G]
 * (random 64-bit gene-leaf hashes; ~0 is reserved), int64 leaf_species [F, G].
 * Per family, hash tables of 2^clade_cap_log2 clades and 2^split_cap_log2 splits.
 *
 * kb_build_workspace: bytes of the workspace (HOST *bytes_out).
 * kb_build_tables: clade hashes, clade / split tables, amalg_rounds amalgamation rounds,
 *   log2((count + alpha) / (n_obs + alpha * n_splits)) per split, rows sorted by
 *   (size, more than one split, family, hash | gene index), waves; synchronises the stream and
 *   writes HOST sizes_out[5] = {rows C, splits N, waves, status bits, splits added by the
 *   amalgamation}.  Status bits: 1 clade table full, 2 split table full (retry with a larger
 *   table), 4 reserved hash value, 8 malformed topology, 16 missing clade, 32 count overflow;
 *   the outputs are valid only when the status is 0.
 * kb_build_emit_scratch: bytes of the scratch kb_build_emit needs for N splits.
 * kb_build_emit: from the same workspace, the layout arrays: leaf_state int32 [C], item_idx /
 *   row_local (row - its wave's start) int64 [C], root_row_ids int64 [F]; per split in row order
 *   (each row's splits by the smaller child hash) sl / sr / reduce_idx / split_row (the parent
 *   row) int64 [N], row_split_ptr int64 [C+1] (each row's splits), log_split_probs f32 [N]; ge2_flat int64 [C + waves] (wave w's ge2_ptr is
 *   ge2_flat[t[7] .. t[7] + W - n_eq1]); wave_table int64 [waves, 8] rows t = {start, W, n_eq1,
 *   split begin, split end, ge2_max_fanout, clade size, ge2 slice start}; synchronises and
 *   writes HOST k_children_out[2] = {distinct child rows summed over waves, status bits}. */
int kb_build_workspace(int n_families, int n_topologies, int n_genes, int clade_cap_log2, int split_cap_log2,
                       long long* bytes_out);
int kb_build_tables(const int* left, const int* right, const int* root, const unsigned long long* leaf_hash,
                    int n_families, int n_topologies, int n_genes, int amalg_rounds, double alpha,
                    int clade_cap_log2, int split_cap_log2, void* ws, long long ws_bytes, long long* sizes_out,
                    void* stream);
int kb_build_emit_scratch(long long n_splits, long long* bytes_out);
int kb_build_emit(const void* ws, const unsigned long long* leaf_hash, const long long* leaf_species,
                  int n_families, int n_topologies, int n_genes, int clade_cap_log2, int split_cap_log2,
                  long long n_rows, long long n_splits, long long n_waves, int* leaf_state, long long* item_idx,
                  long long* root_row_ids, long long* row_local, long long* sl, long long* sr,
                  long long* reduce_idx, long long* split_row, long long* row_split_ptr, float* log_split_probs,
                  long long* ge2_flat, long long* wave_table, void* scratch, long long scratch_bytes,
                  long long* k_children_out, void* stream);

/* The fused engine's schedule (kbench_b200/engine.py build_plan) from a row-ordered layout:
 * split_row / sl / sr int64 [N] and lsp f32 [N] with the splits grouped by parent row in
 * increasing row order (the layout kb_build_emit writes), row_split_ptr int64 [C+1] (each row's
 * splits), wave_split_ptr HOST int64 [n_waves+1] (each wave's split range; a row's children lie in
 * earlier waves).  Outputs (device): rows int32 [C] (rows by dependency level, stable), split_ptr
 * int64 [C+1], sl_lv / sr_lv / lsp_lv [N] (splits in that order); dataflow arrays over the
 * distinct (parent, child) pairs P <= 2N: dep0 / dep_b int32 [C] (distinct children / parents),
 * ready0 / ready_b int32 [<= C] (rows with none), child_ptr / par_ptr int64 [C+1], child_idx /
 * par_idx int32 [<= 2N]; HOST level_ptr [n_waves+1] and children [n_waves] (distinct child rows
 * per level).  Synchronises; HOST sizes_out[5] = {levels, pairs P, ready0 count, ready_b count,
 * status}.  KB_ERR_ARG when a split's rows are out of range or parents are not in row order. */
int kb_plan_workspace(long long n_rows, long long n_splits, long long* bytes_out);
int kb_plan_build(long long n_rows, long long n_splits, int n_waves, const long long* wave_split_ptr,
                  const long long* split_row, const long long* sl, const long long* sr, const float* lsp,
                  const long long* row_split_ptr, void* ws, long long ws_bytes, int* rows, long long* split_ptr,
                  long long* sl_lv, long long* sr_lv, float* lsp_lv, int* dep0, int* ready0, long long* par_ptr,
                  int* par_idx, int* dep_b, int* ready_b, long long* child_ptr, int* child_idx,
                  long long* level_ptr, long long* children, long long* sizes_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KB_SOLVER_H */
