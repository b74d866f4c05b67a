// The fused B200 engine: one kernel per dependency level for the forward (split reduction + all
// pi_iters fixed-point iterations of each row) and one per level for the backward (active check,
// Neumann adjoint, parameter cotangents, split cotangents with the Pibar VJP trees).
//
// Numerics follow the reference kernels (kbench/core/kernels/{dts_fused,wave_step,
// wave_backward}.py, pristine copies in experiments/pristine_kernels/), reorganised for B200:
//
// Forward.  Rows are scheduled by dependency level (1 + max level of the row's split children)
// instead of by clade size; every row of a level is independent, so a level is one launch with
// one CTA per row.  The CTA computes the row's split reduction (dts) in registers, then runs the
// pi_iters Jacobi iterations of the row entirely on chip.  The iteration is carried in linear
// space relative to a per-row scale R: with P[s] = 2^(Pi[s]-R) the reference's update
//   Pi_new = lse2(dl+Pi, Pi+ebar, Pibar+e, sl1+Pi[c1], sl2+Pi[c2], leaf, dts)
// is, exactly in real arithmetic,
//   2^(Pi_new - R) = P*(2^dl+2^ebar) + D*2^(mc+e) + P[c1]*2^sl1 + P[c2]*2^sl2 + leaf + dts,
// D = rowsum(P) - ancestor-or-self pathsum(P) (the reference's Pibar denominator), so an
// iteration costs FMAs and shared-memory gathers instead of ~10 MUFU ex2/lg2 per element.  The
// row is renormalised by its max every iteration (P <= 1).  If any nonzero element falls below
// 2^-100 of the row max (where fp32 linear values would lose precision) the row is recomputed
// with the log-space iteration, so results never silently degrade.  Final Pi, Pibar and the row
// max are written once; the split reduction is also saved for the backward.
//
// Backward.  Reverse level order (a row's adjoint is complete once every level above it ran).
// One CTA per row: active check (max|rhs| vs threshold), coefficient precompute, all Neumann
// terms with shared-memory subtree sums (a block-wide scan over the preorder numbering: the
// subtree of x is the preorder range [pre(x), pre(x)+size(x))), the column gradient, the
// parameter cotangents, and then every split of the row: the split's Pi cotangents for both
// children (speciation terms gathered per child column instead of scattered), the two Pibar VJP
// trees (scan again), and ONE add per child element into the children's adjoint rows.  The
// solved adjoint row never leaves the chip.  Column sums go to fp64 accumulators.
#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

using namespace kb;

struct LevelConsts {
  const float* mc;
  const float* dl;
  const float* ebar;
  const float* e;
  const float* sl1;
  const float* sl2;
  const float* leaf_logp;  // [G,S] item*S + s
  const float* linA;       // [G,S] 2^dl + 2^ebar
  const float* linB;       // [G,S] 2^(mc+e)
  const float* linC1;      // [G,S] 2^sl1
  const float* linC2;      // [G,S] 2^sl2
  const float* log_pD;     // [G,S] split-term parameters (item*prs + s)
  const float* log_pS;
  long long prs;
  long long crs;
  const float* col;
  int use_col;
  const int* parent;
  const int* c1;
  const int* c2;
  const int* pre;
  const int* pre_end;
  const int* sub_start;
  const int* sub_end;
  const int* jumps;
  int K;
  const long long* item_idx;
  const int* leaf_state;
  int S;
};

struct SplitCSR {
  const int* rows;             // level rows (global ids)
  const long long* split_ptr;  // [n+1] into the split arrays
  const long long* sl;
  const long long* sr;
  const float* lsp;
};

// dts of one row from its splits (online LSE across splits), into x[] (log values).
template <int VPT>
__device__ __forceinline__ void dts_row(const LevelConsts& c, const float* __restrict__ Pi,
                                        const float* __restrict__ Pibar, const SplitCSR& sp, long long i0,
                                        long long i1, size_t pb, float* Pl, float* Pr, float* x) {
  const int S = c.S;
  float m[VPT], acc[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) { m[k] = neg_inf(); acc[k] = 0.f; }
  for (long long i = i0; i < i1; ++i) {
    const long long l = sp.sl[i], r = sp.sr[i];
    const float* pil = Pi + (size_t)l * S;
    const float* pir = Pi + (size_t)r * S;
    const float* pbl = Pibar + (size_t)l * S;
    const float* pbr = Pibar + (size_t)r * S;
    __syncthreads();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      Pl[s] = pil[s];
      Pr[s] = pir[s];
    }
    __syncthreads();
    const float lsp = sp.lsp[i];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s >= S) break;
      const float ld = c.log_pD[pb + s];
      const float ls = c.log_pS[pb + s];
      const int a = c.c1[s], b = c.c2[s];
      const bool av = (unsigned)a < (unsigned)S, bv = (unsigned)b < (unsigned)S;
      const float v0 = lsp + ld + Pl[s] + Pr[s];
      const float v1 = lsp + Pl[s] + pbr[s];
      const float v2 = lsp + Pr[s] + pbl[s];
      const float v3 = lsp + ls + (av ? Pl[a] : neg_inf()) + (bv ? Pr[b] : neg_inf());
      const float v4 = lsp + ls + (av ? Pr[a] : neg_inf()) + (bv ? Pl[b] : neg_inf());
      const float sm_ = fmaxf(fmaxf(fmaxf(v0, v1), fmaxf(v2, v3)), v4);
      const float sms = safe_max(sm_);
      const float ssum = ex2(v0 - sms) + ex2(v1 - sms) + ex2(v2 - sms) + ex2(v3 - sms) + ex2(v4 - sms);
      const float nm = fmaxf(m[k], sm_);
      const float nms = safe_max(nm);
      acc[k] = (is_neg_inf(m[k]) ? 0.f : acc[k] * ex2(m[k] - nms)) + ssum * ex2(sms - nms);
      m[k] = nm;
    }
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) x[k] = lg2(acc[k]) + m[k];
}

__device__ __forceinline__ float leaf_seed(const LevelConsts& c, size_t cb, long long item, int leaf, int s) {
  const int S = c.S;
  const float obs = c.leaf_logp[(size_t)item * S + leaf];
  const int ls = c.sub_start[leaf], le = c.sub_end[leaf];
  const int st = c.sub_start[s];
  const bool desc = (st >= ls) && (st < le);
  const bool hit = (s == leaf);
  const float colp = c.use_col ? c.col[leaf] : 0.f;
  const float pi_w = hit ? obs : neg_inf();
  const float pib = desc ? neg_inf() : c.mc[cb + s] + colp + obs;
  const float ps1 = (c.c1[s] == leaf) ? obs : neg_inf();
  const float ps2 = (c.c2[s] == leaf) ? obs : neg_inf();
  const float t0 = c.dl[cb + s] + pi_w;
  const float t1 = pi_w + c.ebar[cb + s];
  const float t2 = pib + c.e[cb + s];
  const float t3 = c.sl1[cb + s] + ps1;
  const float t4 = c.sl2[cb + s] + ps2;
  const float t5 = hit ? c.leaf_logp[(size_t)item * S + s] : neg_inf();
  const float m = fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(t4, t5));
  const float ms = safe_max(m);
  const float tot = ex2(t0 - ms) + ex2(t1 - ms) + ex2(t2 - ms) + ex2(t3 - ms) + ex2(t4 - ms) + ex2(t5 - ms);
  return lg2(tot) + m;
}

// Path sums (ancestor-or-self) of the values in X (Y scratch); returns the result buffer.
__device__ __forceinline__ const float* pathsums(float* X, float* Y, const LevelConsts& c) {
  return ancestor_sum_doubling(X, Y, c.jumps, c.K, c.S);
}

// Log-space Jacobi sweep (reference numerics) of the row in P (log values) -> out[].
template <int VPT>
__device__ __forceinline__ void log_iter(const float* P, float* X, float* Y, float* red, const LevelConsts& c,
                                         size_t cb, int leaf, float leafv, const float* dv, float* out) {
  const int S = c.S;
  float m = neg_inf();
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = P[s];
    if (c.use_col) w += c.col[s];
    m = fmaxf(m, w);
  }
  const float row_max = block_max(m, red);
  const float rms = safe_max(row_max);
  float sum = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = P[s];
    if (c.use_col) w += c.col[s];
    const float xv = ex2(w - rms);
    X[s] = xv;
    sum += xv;
  }
  const float row_sum = block_sum(sum, red);
  const float* anc = pathsums(X, Y, c);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s >= S) break;
    const float pi = P[s];
    const float denom = row_sum - anc[s];
    const float pib = denom > 0.f ? lg2(denom) + row_max + c.mc[cb + s] : neg_inf();
    const float t0 = c.dl[cb + s] + pi;
    const float t1 = pi + c.ebar[cb + s];
    const float t2 = pib + c.e[cb + s];
    const int a = c.c1[s], b = c.c2[s];
    const float t3 = ((unsigned)a < (unsigned)S) ? c.sl1[cb + s] + P[a] : neg_inf();
    const float t4 = ((unsigned)b < (unsigned)S) ? c.sl2[cb + s] + P[b] : neg_inf();
    const float t5 = (s == leaf) ? leafv : neg_inf();
    const float td = dv ? dv[k] : neg_inf();
    const float mm = fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(fmaxf(t4, t5), td));
    const float ms = safe_max(mm);
    float tot = (ex2(t0 - ms) + ex2(t1 - ms) + ex2(t2 - ms)) + (ex2(t3 - ms) + ex2(t4 - ms) + ex2(t5 - ms));
    if (dv) tot += ex2(td - ms);
    out[k] = lg2(tot) + mm;
  }
}

struct FwdArgs {
  LevelConsts c;
  SplitCSR sp;
  const float* Pi_src;    // children read from here (== pi)
  const float* Pibar_src;
  float* pi;
  float* pibar;
  float* row_max;
  float* dts_save;  // [C,S] or null
  float* residual;  // [C] or null
  int* fallback_count;  // device counter of rows recomputed in log space (may be null)
  int n_rows;
  int pi_iters;
};

template <int VPT>
__global__ void __launch_bounds__(512) level_forward_kernel(FwdArgs a) {
  extern __shared__ float sm[];
  const LevelConsts& c = a.c;
  const int S = c.S;
  float* P = sm;
  float* X = sm + S;
  float* Y = sm + 2 * S;
  float* red = sm + 3 * S;
  const int b = blockIdx.x;
  const long long row = a.sp.rows[b];
  const long long item = c.item_idx[row];
  const size_t cb = (size_t)(item * c.crs);
  const size_t pb = (size_t)(item * c.prs);
  const long long i0 = a.sp.split_ptr[b], i1 = a.sp.split_ptr[b + 1];
  const int leaf_raw = c.leaf_state[row];
  const bool is_leaf = (i0 == i1) && leaf_raw >= 0 && leaf_raw < S;
  const int leaf = is_leaf ? leaf_raw : -1;
  const float leafv = is_leaf ? c.leaf_logp[(size_t)item * S + leaf] : neg_inf();

  // ---- initial row (log values) ----
  float x[VPT];
  if (is_leaf) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      x[k] = s < S ? leaf_seed(c, cb, item, leaf, s) : neg_inf();
    }
  } else {
    dts_row<VPT>(c, a.Pi_src, a.Pibar_src, a.sp, i0, i1, pb, X, Y, x);
    if (a.dts_save) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * blockDim.x;
        if (s < S) a.dts_save[(size_t)row * S + s] = x[k];
      }
    }
  }
  float m0 = neg_inf();
#pragma unroll
  for (int k = 0; k < VPT; ++k) m0 = fmaxf(m0, x[k]);
  const float Rd = safe_max(block_max(m0, red));  // scale of the initial row (and of the dts term)

  // ---- linear-space iterations ----
  float pv[VPT], td[VPT];
  float psum = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    pv[k] = s < S ? ex2(x[k] - Rd) : 0.f;
    td[k] = is_leaf ? 0.f : pv[k];
    if (s < S) { P[s] = pv[k]; X[s] = pv[k]; }
    psum += pv[k];
  }
  float sumP = block_sum(psum, red);
  float R = Rd;
  bool fallback = false;
  float zl[VPT];  // last iteration's unnormalised values (relative to Rlast)
  float Rlast = R;
  for (int it = 1; it < a.pi_iters; ++it) {
    const float* anc = pathsums(X, Y, c);
    const float fd = ex2(Rd - R);
    const float lf = is_leaf ? ex2(leafv - R) : 0.f;
    float zmax = 0.f, zmin = 3.0e38f, zsum = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      float z = 0.f;
      if (s < S) {
        const float D = sumP - anc[s];
        z = pv[k] * __ldg(c.linA + cb + s);
        if (D > 0.f) z = fmaf(D, __ldg(c.linB + cb + s), z);
        const int ca = c.c1[s], cbb = c.c2[s];
        if ((unsigned)ca < (unsigned)S) z = fmaf(P[ca], __ldg(c.linC1 + cb + s), z);
        if ((unsigned)cbb < (unsigned)S) z = fmaf(P[cbb], __ldg(c.linC2 + cb + s), z);
        if (s == leaf) z += lf;
        z = fmaf(td[k], fd, z);
        zmax = fmaxf(zmax, z);
        if (z > 0.f) zmin = fminf(zmin, z);
        zsum += z;
      }
      zl[k] = z;
    }
    // one combined reduction: max, min-positive, sum
    {
      const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
      const int nw = (blockDim.x + 31) >> 5;
      zmax = warp_max(zmax);
      zmin = -warp_max(-zmin);
      zsum = warp_sum(zsum);
      __syncthreads();
      if (lane == 0) { red[wid] = zmax; red[32 + wid] = zmin; red[64 + wid] = zsum; }
      __syncthreads();
      float a1 = lane < nw ? red[lane] : 0.f;
      float a2 = lane < nw ? red[32 + lane] : 3.0e38f;
      float a3 = lane < nw ? red[64 + lane] : 0.f;
      zmax = warp_max(a1);
      zmin = -warp_max(-a2);
      zsum = warp_sum(a3);
    }
    if (zmax > 0.f && zmin < zmax * 7.8886091e-31f) {  // 2^-100
      fallback = true;
      break;
    }
    Rlast = R;
    if (it == a.pi_iters - 1) break;  // keep zl (relative to Rlast) for the final write
    const float inv = zmax > 0.f ? 1.0f / zmax : 0.f;
    R = zmax > 0.f ? R + lg2(zmax) : R;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      pv[k] = zl[k] * inv;
      if (s < S) { P[s] = pv[k]; X[s] = pv[k]; }
    }
    sumP = zsum * inv;
    __syncthreads();
  }

  float pf[VPT];  // final Pi (log values)
  if (!fallback) {
    if (a.residual) {
      float d = 0.f;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * blockDim.x;
        if (s < S && zl[k] > 0.f && pv[k] > 0.f) d = fmaxf(d, fabsf(lg2(zl[k]) - lg2(pv[k])));
      }
      d = block_max(d, red);
      if (threadIdx.x == 0) a.residual[row] = d;
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) pf[k] = lg2(zl[k]) + Rlast;
  } else {
    // log-space recomputation of the whole row from its initial values (rare)
    if (threadIdx.x == 0 && a.fallback_count) atomicAdd(a.fallback_count, 1);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) P[s] = x[k];
    }
    __syncthreads();
    float nv[VPT];
    for (int it = 1; it < a.pi_iters; ++it) {
      log_iter<VPT>(P, X, Y, red, c, cb, leaf, leafv, is_leaf ? nullptr : x, nv);
      if (a.residual && it == a.pi_iters - 1) {
        float d = 0.f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int s = threadIdx.x + k * blockDim.x;
          if (s < S && !is_neg_inf(nv[k]) && !is_neg_inf(P[s])) d = fmaxf(d, fabsf(nv[k] - P[s]));
        }
        d = block_max(d, red);
        if (threadIdx.x == 0) a.residual[row] = d;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * blockDim.x;
        if (s < S) P[s] = nv[k];
      }
      __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      pf[k] = s < S ? P[s] : neg_inf();
    }
  }

  // ---- final Pi, row max, Pibar (as the reference computes them from the final log row) ----
  float* prow = a.pi + (size_t)row * S;
  float mx = neg_inf();
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) {
      prow[s] = pf[k];
      float w = pf[k];
      if (c.use_col) w += c.col[s];
      mx = fmaxf(mx, w);
    }
  }
  const float row_max = block_max(mx, red);
  const float rms = safe_max(row_max);
  float sum = 0.f;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) {
      float w = pf[k];
      if (c.use_col) w += c.col[s];
      const float xv = ex2(w - rms);
      X[s] = xv;
      sum += xv;
    }
  }
  const float row_sum = block_sum(sum, red);
  const float* anc = pathsums(X, Y, c);
  float* brow = a.pibar + (size_t)row * S;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) {
      const float denom = row_sum - anc[s];
      brow[s] = denom > 0.f ? lg2(denom) + row_max + c.mc[cb + s] : neg_inf();
    }
  }
  if (threadIdx.x == 0) a.row_max[row] = row_max;
}

// ------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------

struct BwdArgs {
  LevelConsts c;
  SplitCSR sp;
  const float* Pi;
  const float* Pibar;
  const float* row_max;
  const float* dts_saved;  // [C,S] or null (recompute from the splits)
  float* acc;              // accumulated_rhs [C,S]
  float* v_out;            // [C,S] solved adjoint rows (active rows) or null
  double* gacc;            // [10,S]: aw0..aw5, dD, dS, dM, col
  float threshold;
  int strict_gt;
  float side_thr;
  int side_thr_enabled;
  int neumann_terms;
  int n_rows;
};

template <int VPT>
__global__ void __launch_bounds__(512) level_backward_kernel(BwdArgs a) {
  extern __shared__ float sm[];
  const LevelConsts& c = a.c;
  const int S = c.S;
  float* P = sm;             // Pi row (log)
  float* B0 = sm + S;
  float* B1 = sm + 2 * S;
  float* B2 = sm + 3 * S;
  float* B3 = sm + 4 * S;
  float* B4 = sm + 5 * S;
  float* red = sm + 6 * S;   // >= 96 floats
  const int b = blockIdx.x;
  const long long row = a.sp.rows[b];
  const long long item = c.item_idx[row];
  const size_t cb = (size_t)(item * c.crs);
  const size_t pb = (size_t)(item * c.prs);
  const long long i0 = a.sp.split_ptr[b], i1 = a.sp.split_ptr[b + 1];
  const bool has_splits = i1 > i0;
  const int leaf_raw = c.leaf_state[row];
  const int leaf = (!has_splits && leaf_raw >= 0 && leaf_raw < S) ? leaf_raw : -1;

  // ---- active check ----
  float v[VPT];
  float amax = 0.f;
  const float* rrow = a.acc + (size_t)row * S;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    v[k] = s < S ? rrow[s] : 0.f;
    amax = fmaxf(amax, fabsf(v[k]));
  }
  amax = block_max(amax, red);
  const bool active = a.strict_gt ? (amax > a.threshold) : (amax >= a.threshold);
  if (!active) return;

  // ---- dts row (log) ----
  float dv[VPT];
  if (has_splits) {
    if (a.dts_saved) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * blockDim.x;
        dv[k] = s < S ? a.dts_saved[(size_t)row * S + s] : neg_inf();
      }
    } else {
      dts_row<VPT>(c, a.Pi, a.Pibar, a.sp, i0, i1, pb, B0, B1, dv);
    }
  }

  // ---- precompute ----
  const float* pirow = a.Pi + (size_t)row * S;
  const float rmax = a.row_max[row];
  const float rms = safe_max(rmax);
  float pp[VPT];
  float psum = 0.f;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    pp[k] = 0.f;
    if (s < S) {
      const float pi = pirow[s];
      P[s] = pi;
      float w = pi;
      if (c.use_col) w += c.col[s];
      pp[k] = ex2(w - rms);
      B0[s] = pp[k];
      B2[s] = 0.f;
      psum += pp[k];
    }
  }
  const float row_sum = block_sum(psum, red);
  const float* anc = ancestor_sum_doubling(B0, B1, c.jumps, c.K, S);
  float diag[VPT], coef[VPT];
  const float* pbrow = a.Pibar + (size_t)row * S;
  const float leafv = leaf >= 0 ? c.leaf_logp[(size_t)item * S + leaf] : neg_inf();
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    diag[k] = coef[k] = 0.f;
    if (s < S) {
      const float pi = P[s];
      const float t0 = c.dl[cb + s] + pi;
      const float t1 = pi + c.ebar[cb + s];
      const float t2 = pbrow[s] + c.e[cb + s];
      const int ca = c.c1[s], cbb = c.c2[s];
      const bool av = (unsigned)ca < (unsigned)S, bv = (unsigned)cbb < (unsigned)S;
      const float t3 = c.sl1[cb + s] + (av ? P[ca] : neg_inf());
      const float t4 = c.sl2[cb + s] + (bv ? P[cbb] : neg_inf());
      const float t5 = (s == leaf) ? leafv : neg_inf();
      const float m = fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(t4, t5));
      const float ms = safe_max(m);
      const float e0 = ex2(t0 - ms), e1 = ex2(t1 - ms), e2 = ex2(t2 - ms), e3 = ex2(t3 - ms), e4 = ex2(t4 - ms),
                  e5 = ex2(t5 - ms);
      const float ssum = e0 + e1 + e2 + e3 + e4 + e5;
      const float inv_sum = ssum > 0.f ? 1.0f / ssum : 0.f;
      float wL = 1.0f;
      if (has_splits) {
        const float dlv = lg2(ssum) + m;
        const float pm = fmaxf(dlv, dv[k]);
        const float pms = safe_max(pm);
        const float pnew = lg2(ex2(dlv - pms) + ex2(dv[k] - pms)) + pm;
        wL = is_neg_inf(dlv) ? 0.f : ex2(dlv - pnew);
      }
      const float denom = row_sum - anc[s];
      const float inv_denom = denom > 0.f ? 1.0f / denom : 0.f;
      diag[k] = wL * (e0 + e1) * inv_sum;
      coef[k] = wL * e2 * inv_sum * inv_denom;
      if (av) B2[ca] = wL * e3 * inv_sum;   // edge weight of child ca (B2 = EDGE)
      if (bv) B2[cbb] = wL * e4 * inv_sum;
    }
  }
  __syncthreads();
  float edge[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    edge[k] = 0.f;
    if (s < S) {
      const int par = c.parent[s];
      edge[k] = ((unsigned)par < (unsigned)S) ? B2[s] : 0.f;
      B0[s] = v[k];  // T: current Neumann term
    }
  }

  // ---- Neumann series: T in B0, u scan in B1 ----
  float* T = B0;
  float* U = B1;
  for (int n = 0; n < a.neumann_terms; ++n) {
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) U[__ldg(c.pre + s)] = T[s] * coef[k];
    }
    const float A = block_exclusive_scan(U, S, red);
    float nv[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      nv[k] = 0.f;
      if (s < S) {
        const int pe = __ldg(c.pre_end + s);
        const float sub = (pe < S ? U[pe] : A) - U[__ldg(c.pre + s)];
        const int par = c.parent[s];
        const float pt = ((unsigned)par < (unsigned)S) ? T[par] : 0.f;
        nv[k] = T[s] * diag[k] + pp[k] * (A - sub) + pt * edge[k];
        v[k] += nv[k];
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) T[s] = nv[k];
    }
  }

  if (a.v_out) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) a.v_out[(size_t)row * S + s] = v[k];
    }
  }

  // ---- column gradient of the self-loop Pibar term ----
  float colacc[VPT];
  __syncthreads();
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) U[__ldg(c.pre + s)] = v[k] * coef[k];
  }
  {
    const float A = block_exclusive_scan(U, S, red);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      colacc[k] = 0.f;
      if (s < S) {
        const int pe = __ldg(c.pre_end + s);
        colacc[k] = pp[k] * (A - ((pe < S ? U[pe] : A) - U[__ldg(c.pre + s)]));
      }
    }
  }

  // ---- parameter cotangents of the self-loop (recomputes the terms) ----
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) {
      const float pi = P[s];
      const float t0 = c.dl[cb + s] + pi;
      const float t1 = pi + c.ebar[cb + s];
      const float t2 = pbrow[s] + c.e[cb + s];
      const int ca = c.c1[s], cbb = c.c2[s];
      const float t3 = c.sl1[cb + s] + (((unsigned)ca < (unsigned)S) ? P[ca] : neg_inf());
      const float t4 = c.sl2[cb + s] + (((unsigned)cbb < (unsigned)S) ? P[cbb] : neg_inf());
      const float t5 = (s == leaf) ? leafv : neg_inf();
      const float m = fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(t4, t5));
      const float ms = safe_max(m);
      const float e0 = ex2(t0 - ms), e1 = ex2(t1 - ms), e2 = ex2(t2 - ms), e3 = ex2(t3 - ms), e4 = ex2(t4 - ms),
                  e5 = ex2(t5 - ms);
      const float ssum = e0 + e1 + e2 + e3 + e4 + e5;
      const float inv_sum = ssum > 0.f ? 1.0f / ssum : 0.f;
      float wL = 1.0f;
      if (has_splits) {
        const float dlv = lg2(ssum) + m;
        const float pm = fmaxf(dlv, dv[k]);
        const float pms = safe_max(pm);
        const float pnew = lg2(ex2(dlv - pms) + ex2(dv[k] - pms)) + pm;
        wL = is_neg_inf(dlv) ? 0.f : ex2(dlv - pnew);
      }
      const float alpha = v[k] * wL;
      double* g = a.gacc;
      atomicAdd(g + 0 * (size_t)S + s, (double)(alpha * e0 * inv_sum));
      atomicAdd(g + 1 * (size_t)S + s, (double)(alpha * e1 * inv_sum));
      atomicAdd(g + 2 * (size_t)S + s, (double)(alpha * e2 * inv_sum));
      atomicAdd(g + 3 * (size_t)S + s, (double)(alpha * e3 * inv_sum));
      atomicAdd(g + 4 * (size_t)S + s, (double)(alpha * e4 * inv_sum));
      if (leaf >= 0) atomicAdd(g + 5 * (size_t)S + s, (double)(alpha * e5 * inv_sum));
    }
  }

  // ---- splits: cotangents of the split reduction + Pibar VJP trees ----
  float dD[VPT], dS[VPT], dM[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) dD[k] = dS[k] = dM[k] = 0.f;
  float pip[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    pip[k] = s < S ? pirow[s] : neg_inf();
  }
  // buffers in the split phase: B0/B1 child Pi rows, B2/B3 speciation cotangents (vd3, vd4),
  // B4/P the left/right Pibar u_d in preorder positions (scanned in place)
  for (long long i = i0; i < i1; ++i) {
    const long long l = a.sp.sl[i], r = a.sp.sr[i];
    const float lsp = a.sp.lsp[i];
    const float* pil = a.Pi + (size_t)l * S;
    const float* pir = a.Pi + (size_t)r * S;
    const float* pbl = a.Pibar + (size_t)l * S;
    const float* pbr = a.Pibar + (size_t)r * S;
    const float rml = a.row_max[l], rmr = a.row_max[r];
    const float rmls = safe_max(rml), rmrs = safe_max(rmr);
    const size_t mcl = (size_t)(c.item_idx[l] * c.crs), mcr = (size_t)(c.item_idx[r] * c.crs);
    __syncthreads();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      B0[s] = pil[s];
      B1[s] = pir[s];
    }
    __syncthreads();
    float cl[VPT], cr[VPT], ppl[VPT], ppr[VPT];
    float sabs_l = 0.f, sabs_r = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      cl[k] = cr[k] = ppl[k] = ppr[k] = 0.f;
      if (s < S) {
        const float pl = B0[s], pr = B1[s];
        const float ld = c.log_pD[pb + s];
        const float ls = c.log_pS[pb + s];
        const int ca = c.c1[s], cbb = c.c2[s];
        const bool av = (unsigned)ca < (unsigned)S, bv = (unsigned)cbb < (unsigned)S;
        const float d0 = ld + pl + pr;
        const float d1 = pl + pbr[s];
        const float d2 = pr + pbl[s];
        const float d3 = ls + (av ? B0[ca] : neg_inf()) + (bv ? B1[cbb] : neg_inf());
        const float d4 = ls + (av ? B1[ca] : neg_inf()) + (bv ? B0[cbb] : neg_inf());
        const float ppar = pip[k];
        const bool pv = !is_neg_inf(ppar);
        const float vd0 = v[k] * (pv ? ex2(lsp + d0 - ppar) : 0.f);
        const float vd1 = v[k] * (pv ? ex2(lsp + d1 - ppar) : 0.f);
        const float vd2 = v[k] * (pv ? ex2(lsp + d2 - ppar) : 0.f);
        const float vd3 = v[k] * (pv ? ex2(lsp + d3 - ppar) : 0.f);
        const float vd4 = v[k] * (pv ? ex2(lsp + d4 - ppar) : 0.f);
        dD[k] += vd0;
        dS[k] += vd3 + vd4;
        dM[k] += vd1 + vd2;
        cl[k] = vd0 + vd1;
        cr[k] = vd0 + vd2;
        B2[s] = vd3;
        B3[s] = vd4;
        const float bl = pbl[s], br = pbr[s];
        const float udl = is_neg_inf(bl) ? 0.f : vd2 * ex2(rml + c.mc[mcl + s] - bl);
        const float udr = is_neg_inf(br) ? 0.f : vd1 * ex2(rmr + c.mc[mcr + s] - br);
        const int ps = __ldg(c.pre + s);
        B4[ps] = udl;
        P[ps] = udr;
        sabs_l += fabsf(udl);
        sabs_r += fabsf(udr);
        float wl = pl, wr = pr;
        if (c.use_col) { wl += c.col[s]; wr += c.col[s]; }
        ppl[k] = ex2(wl - rmls);
        ppr[k] = ex2(wr - rmrs);
      }
    }
    bool side_l = true, side_r = true;
    if (a.side_thr_enabled) {
      sabs_l = block_sum(sabs_l, red);
      sabs_r = block_sum(sabs_r, red);
      side_l = sabs_l > a.side_thr;
      side_r = sabs_r > a.side_thr;
    }
    float Al, Ar;
    block_exclusive_scan2(B4, P, S, red, Al, Ar);
    float* rl = a.acc + (size_t)l * S;
    float* rr = a.acc + (size_t)r * S;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int x = threadIdx.x + k * blockDim.x;
      if (x < S) {
        const int par = c.parent[x];
        float sl_ = 0.f, sr_ = 0.f;
        if ((unsigned)par < (unsigned)S) {
          const bool first = c.c1[par] == x;
          sl_ = first ? B2[par] : B3[par];
          sr_ = first ? B3[par] : B2[par];
        }
        const int ps = __ldg(c.pre + x), pe = __ldg(c.pre_end + x);
        float tl_ = 0.f, tr_ = 0.f;
        if (side_l) tl_ = ppl[k] * (Al - ((pe < S ? B4[pe] : Al) - B4[ps]));
        if (side_r) tr_ = ppr[k] * (Ar - ((pe < S ? P[pe] : Ar) - P[ps]));
        colacc[k] += tl_ + tr_;
        atomicAdd(rl + x, cl[k] + sl_ + tl_);
        atomicAdd(rr + x, cr[k] + sr_ + tr_);
      }
    }
  }
  double* g = a.gacc;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) {
      if (has_splits) {
        atomicAdd(g + 6 * (size_t)S + s, (double)dD[k]);
        atomicAdd(g + 7 * (size_t)S + s, (double)dS[k]);
        atomicAdd(g + 8 * (size_t)S + s, (double)dM[k]);
      }
      atomicAdd(g + 9 * (size_t)S + s, (double)colacc[k]);
    }
  }
}

__global__ void finalize_grads_kernel(const double* __restrict__ g, int S, float* gpD, float* gpS, float* gmt,
                                      float* gE, float* gEbar, float* gEs1, float* gEs2, float* gcol) {
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < S; s += gridDim.x * blockDim.x) {
    const double a0 = g[s], a1 = g[S + s], a2 = g[2 * S + s], a3 = g[3 * S + s], a4 = g[4 * S + s],
                 a5 = g[5 * S + s], dD = g[6 * S + s], dS = g[7 * S + s], dM = g[8 * S + s], col = g[9 * S + s];
    gpD[s] = (float)(a0 + dD);
    gpS[s] = (float)(a3 + a4 + a5 + dS);
    gmt[s] = (float)(a2 + dM);
    gE[s] = (float)(a0 + a2);
    gEbar[s] = (float)a1;
    gEs1[s] = (float)a4;
    gEs2[s] = (float)a3;
    gcol[s] = (float)col;
  }
}

__global__ void lin_consts_kernel(const float* dl, const float* ebar, const float* mc, const float* e,
                                  const float* sl1, const float* sl2, int n, float* A, float* B, float* C1,
                                  float* C2) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    A[i] = ex2(dl[i]) + ex2(ebar[i]);
    B[i] = ex2(mc[i] + e[i]);
    C1[i] = ex2(sl1[i]);
    C2[i] = ex2(sl2[i]);
  }
}

int vpt_pick(int S, int& bd) {
  bd = 512;
  if (S <= 512) bd = ((S + 31) / 32) * 32;
  if (bd < 32) bd = 32;
  const int v = (S + bd - 1) / bd;
  if (v <= 1) return 1;
  if (v <= 2) return 2;
  if (v <= 4) return 4;
  if (v <= 8) return 8;
  return 16;
}

LevelConsts make_lc(const float* mc, const float* dl, const float* ebar, const float* e, const float* sl1,
                    const float* sl2, const float* leaf_logp, const float* linA, const float* linB,
                    const float* linC1, const float* linC2, const float* log_pD, const float* log_pS,
                    long long prs, long long crs, const float* col, int use_col, const int* parent, const int* c1,
                    const int* c2, const int* pre, const int* pre_end, const int* sub_start, const int* sub_end,
                    const int* jumps, int K, const long long* item_idx, const int* leaf_state, int S) {
  LevelConsts c;
  c.mc = mc; c.dl = dl; c.ebar = ebar; c.e = e; c.sl1 = sl1; c.sl2 = sl2; c.leaf_logp = leaf_logp;
  c.linA = linA; c.linB = linB; c.linC1 = linC1; c.linC2 = linC2; c.log_pD = log_pD; c.log_pS = log_pS;
  c.prs = prs; c.crs = crs; c.col = col; c.use_col = use_col; c.parent = parent; c.c1 = c1; c.c2 = c2;
  c.pre = pre; c.pre_end = pre_end; c.sub_start = sub_start; c.sub_end = sub_end; c.jumps = jumps; c.K = K;
  c.item_idx = item_idx; c.leaf_state = leaf_state; c.S = S;
  return c;
}

}  // namespace

extern "C" int kb_lin_consts(const float* dl, const float* ebar, const float* mc, const float* e, const float* sl1,
                             const float* sl2, int n, float* linA, float* linB, float* linC1, float* linC2,
                             void* stream) {
  if (n <= 0) return n == 0 ? KB_OK : KB_ERR_ARG;
  const int bd = 256;
  const int grid = (n + bd - 1) / bd;
  lin_consts_kernel<<<grid, bd, 0, (cudaStream_t)stream>>>(dl, ebar, mc, e, sl1, sl2, n, linA, linB, linC1, linC2);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_level_forward(const int* rows, const long long* split_ptr, int n_rows, const long long* sl,
                                const long long* sr, const float* lsp, const float* Pi_src, const float* Pibar_src,
                                float* pi, float* pibar, float* pibar_row_max, float* dts_save, float* residual,
                                int* fallback_count, const float* mc, const float* dl, const float* ebar,
                                const float* e, const float* sl1, const float* sl2, const float* leaf_logp,
                                const float* linA, const float* linB, const float* linC1, const float* linC2,
                                const float* log_pD, const float* log_pS, long long param_row_stride,
                                long long const_row_stride, const float* col_log_probs, int use_col_weights,
                                const int* node_parent, const int* node_child1, const int* node_child2,
                                const int* node_subtree_start, const int* node_subtree_end, const int* jumps, int K,
                                const long long* item_idx, const int* leaf_state, int pi_iters, int S,
                                void* stream) {
  if (S <= 0 || n_rows < 0 || K < 0 || pi_iters < 2) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (n_rows == 0) return KB_OK;
  FwdArgs a;
  a.c = make_lc(mc, dl, ebar, e, sl1, sl2, leaf_logp, linA, linB, linC1, linC2, log_pD, log_pS, param_row_stride,
                const_row_stride, col_log_probs, use_col_weights, node_parent, node_child1, node_child2,
                node_subtree_start, node_subtree_end, node_subtree_start, node_subtree_end, jumps, K, item_idx,
                leaf_state, S);
  a.sp = SplitCSR{rows, split_ptr, sl, sr, lsp};
  a.Pi_src = Pi_src; a.Pibar_src = Pibar_src; a.pi = pi; a.pibar = pibar; a.row_max = pibar_row_max;
  a.dts_save = dts_save; a.residual = residual; a.fallback_count = fallback_count; a.n_rows = n_rows;
  a.pi_iters = pi_iters;
  int bd;
  const int vpt = vpt_pick(S, bd);
  const size_t smem = (size_t)(3 * S + 128) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
#define KB_LF_CASE(V)                                                                                     \
  case V:                                                                                                 \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)level_forward_kernel<V>,                   \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) \
      return KB_ERR_LAUNCH;                                                                               \
    level_forward_kernel<V><<<n_rows, bd, smem, st>>>(a);                                                 \
    break;
  switch (vpt) {
    KB_LF_CASE(1) KB_LF_CASE(2) KB_LF_CASE(4) KB_LF_CASE(8) KB_LF_CASE(16)
    default: return KB_ERR_SIZE;
  }
#undef KB_LF_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_level_backward(const int* rows, const long long* split_ptr, int n_rows, const long long* sl,
                                 const long long* sr, const float* lsp, const float* Pi, const float* Pibar,
                                 const float* pibar_row_max, const float* dts_saved, float* accumulated_rhs,
                                 float* v_out, double* grad_acc, float threshold, int strict_gt, float side_threshold,
                                 int side_threshold_enabled, int neumann_terms, const float* mc, const float* dl,
                                 const float* ebar, const float* e, const float* sl1, const float* sl2,
                                 const float* leaf_logp, const float* log_pD, const float* log_pS,
                                 long long param_row_stride, long long const_row_stride, const float* col_log_probs,
                                 int use_col_weights, const int* node_parent, const int* node_child1,
                                 const int* node_child2, const int* node_pre, const int* node_pre_end,
                                 const int* jumps, int K, const long long* item_idx, const int* leaf_state, int S,
                                 void* stream) {
  if (S <= 0 || n_rows < 0 || K < 0 || neumann_terms < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (n_rows == 0) return KB_OK;
  BwdArgs a;
  a.c = make_lc(mc, dl, ebar, e, sl1, sl2, leaf_logp, nullptr, nullptr, nullptr, nullptr, log_pD, log_pS,
                param_row_stride, const_row_stride, col_log_probs, use_col_weights, node_parent, node_child1,
                node_child2, node_pre, node_pre_end, nullptr, nullptr, jumps, K, item_idx, leaf_state, S);
  a.sp = SplitCSR{rows, split_ptr, sl, sr, lsp};
  a.Pi = Pi; a.Pibar = Pibar; a.row_max = pibar_row_max; a.dts_saved = dts_saved; a.acc = accumulated_rhs;
  a.v_out = v_out; a.gacc = grad_acc; a.threshold = threshold; a.strict_gt = strict_gt; a.side_thr = side_threshold;
  a.side_thr_enabled = side_threshold_enabled; a.neumann_terms = neumann_terms; a.n_rows = n_rows;
  int bd;
  const int vpt = vpt_pick(S, bd);
  const size_t smem = (size_t)(6 * S + 128) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
#define KB_LB_CASE(V)                                                                                      \
  case V:                                                                                                  \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)level_backward_kernel<V>,                   \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))  \
      return KB_ERR_LAUNCH;                                                                                \
    level_backward_kernel<V><<<n_rows, bd, smem, st>>>(a);                                                 \
    break;
  switch (vpt) {
    KB_LB_CASE(1) KB_LB_CASE(2) KB_LB_CASE(4) KB_LB_CASE(8) KB_LB_CASE(16)
    default: return KB_ERR_SIZE;
  }
#undef KB_LB_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_finalize_grads(const double* grad_acc, int S, float* grad_log_pD, float* grad_log_pS,
                                 float* grad_mt, float* grad_E, float* grad_Ebar, float* grad_E_s1, float* grad_E_s2,
                                 float* grad_col, void* stream) {
  if (S <= 0) return KB_ERR_ARG;
  finalize_grads_kernel<<<(S + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      grad_acc, S, grad_log_pD, grad_log_pS, grad_mt, grad_E, grad_Ebar, grad_E_s1, grad_E_s2, grad_col);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
