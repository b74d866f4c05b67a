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
// with the log-space iteration, so results never silently degrade.  The same holds only while
// every product of a kept value (>= 2^-100) with a constant 2^dl+2^ebar, 2^(mc+e), 2^sl1, 2^sl2,
// or with the dts / leaf rescaling 2^(Rd-R), stays a normal fp32 number (>= 2^-126): a row whose
// initial values span more than 100 binades, or whose scale grows by more than 2^26, takes the
// log-space path too, and a problem whose constants fall below 2^-26 (extreme rates) sets
// force_log so that every row does.  Final Pi, Pibar and the row
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
  const unsigned* packed;  // [4,S]: children, Euler tour, preorder, parent (16-bit pairs)
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
  int force_log;        // every row takes the log-space iteration (constants below 2^-26)
  const int* force_log_dev;  // the same decision as a device word (ORed in; may be null)
  int n_rows;
  int pi_iters;
};

__device__ __forceinline__ unsigned lo16(unsigned v) { return v & 0xFFFFu; }
__device__ __forceinline__ unsigned hi16(unsigned v) { return v >> 16; }

// dts of one row from its splits (online LSE across splits) into x[] (log values); the two
// child Pi rows are staged in Pl / Pr (shared) for the speciation gathers.
template <int VPT>
__device__ __forceinline__ void dts_row2(const LevelConsts& c, const float* __restrict__ Pi,
                                         const float* __restrict__ Pibar, const SplitCSR& sp, long long i0,
                                         long long i1, size_t pb, const unsigned* cc, float* Pl, float* Pr,
                                         float* x) {
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
      if (s < S) {
        const float ld = c.log_pD[pb + s];
        const float ls = c.log_pS[pb + s];
        const unsigned a = lo16(cc[k]), b = hi16(cc[k]);
        const float pl = Pl[s], pr = Pr[s];
        const float v0 = lsp + ld + pl + pr;
        const float v1 = lsp + pl + pbr[s];
        const float v2 = lsp + pr + pbl[s];
        const float v3 = lsp + ls + (a < (unsigned)S ? Pl[a] : neg_inf()) + (b < (unsigned)S ? Pr[b] : neg_inf());
        const float v4 = lsp + ls + (a < (unsigned)S ? Pr[a] : neg_inf()) + (b < (unsigned)S ? Pl[b] : neg_inf());
        const float sm_ = fmaxf(fmaxf(fmaxf(v0, v1), fmaxf(v2, v3)), v4);
        const float sms = safe_max(sm_);
        const float ssum = ex2(v0 - sms) + ex2(v1 - sms) + ex2(v2 - sms) + ex2(v3 - sms) + ex2(v4 - sms);
        if (i == i0) {
          m[k] = sm_;
          acc[k] = ssum;
        } else {
          const float nm = fmaxf(m[k], sm_);
          const float nms = safe_max(nm);
          acc[k] = (is_neg_inf(m[k]) ? 0.f : acc[k] * ex2(m[k] - nms)) + ssum * ex2(sms - nms);
          m[k] = nm;
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) x[k] = lg2(acc[k]) + m[k];
}

// Ancestor-or-self path sums of the values pv[] through one scan of the Euler tour in T2
// (padded to blockDim.x * 2 * VPT floats, tail zero).  Returns path[] for the own columns.
template <int VPT>
__device__ __forceinline__ void tour_pathsums(float* T2, float* tmp, const unsigned* tr, const float* pv, int S,
                                              float* path);

// The same over all NTV = blockDim.x * VPT padded columns (the padded tour is a permutation of
// its 2 * NTV slots, so every slot is written and nothing needs clearing), fused with the block
// sum of `bsum` (one value per thread, returned).  Three barriers.
template <int VPT>
__device__ __forceinline__ float tour_pathsums_padded(float* T2, float* tmp, const unsigned* tr, const float* pv,
                                                      float bsum, float* path) {
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    T2[lo16(tr[k])] = pv[k];
    T2[hi16(tr[k])] = -pv[k];
  }
  __syncthreads();
  block_exclusive_scan_ch<2 * VPT, true>(T2, tmp, &bsum);
#pragma unroll
  for (int k = 0; k < VPT; ++k) path[k] = T2[lo16(tr[k])] + pv[k];
  return bsum;
}

template <int VPT>
__device__ __forceinline__ void tour_pathsums(float* T2, float* tmp, const unsigned* tr, const float* pv, int S,
                                              float* path) {
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) {
      T2[lo16(tr[k])] = pv[k];
      T2[hi16(tr[k])] = -pv[k];
    }
  }
  __syncthreads();
  block_exclusive_scan_ch<2 * VPT>(T2, tmp);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    path[k] = s < S ? T2[lo16(tr[k])] + pv[k] : 0.f;
  }
}

template <int VPT>
__global__ void __launch_bounds__(1024, 1) level_forward_kernel(FwdArgs a) {
  extern __shared__ float sm[];
  const LevelConsts& c = a.c;
  const int S = c.S;
  const int NT = blockDim.x;
  const int NTV = NT * VPT;                 // padded row width (columns >= S are zero columns)
  float* T2 = sm;                           // two Euler-tour buffers of 2*NTV floats
  float* PB = sm + 4 * NTV;                 // two row buffers of NTV floats
  float* red = sm + 6 * NTV;                // >= 96 floats
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
  const int leafk = (leaf >= 0 && leaf % NT == (int)threadIdx.x) ? leaf / NT : -1;

  // per-column topology (padded: invalid child -> zero column) and linear constants, once
  unsigned cc[VPT], tr[VPT];
  float kA[VPT], kB[VPT], kC1[VPT], kC2[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    cc[k] = c.packed[s];
    tr[k] = c.packed[NTV + s];
    const bool real = s < S;
    kA[k] = real ? c.linA[cb + s] : 0.f;
    kB[k] = real ? c.linB[cb + s] : 0.f;
    kC1[k] = real ? c.linC1[cb + s] : 0.f;
    kC2[k] = real ? c.linC2[cb + s] : 0.f;
  }

  // ---- initial row (log values) ----
  float x[VPT];
  if (is_leaf) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      x[k] = s < S ? leaf_seed(c, cb, item, leaf, s) : neg_inf();
    }
  } else {
    dts_row2<VPT>(c, a.Pi_src, a.Pibar_src, a.sp, i0, i1, pb, cc, T2, T2 + NTV, x);
    if (a.dts_save) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * NT;
        if (s < S) a.dts_save[(size_t)row * S + s] = x[k];
      }
    }
  }
  float m0 = neg_inf();
#pragma unroll
  for (int k = 0; k < VPT; ++k) m0 = fmaxf(m0, x[k]);
  const float Rd = safe_max(block_max(m0, red));  // scale of the initial row and of the dts term

  // ---- linear-space iterations on unnormalised values z (true value 2^(Pi - R) = z) ----
  // Every term of the update is linear in the row except the constant dts / leaf terms, so the
  // normalisation by the previous iteration's max (known only after its reduction) is folded into
  // the next update: z' = (z A + (zsum - path_z)+ B + z[c1] C1 + z[c2] C2) / zmax + dts + leaf,
  // with the dts / leaf terms taken relative to the new scale R + log2(zmax).
  float z[VPT], td[VPT];
  float zmax_l = 0.f, zsum_l = 0.f;
  bool init_bad = a.force_log != 0 || (a.force_log_dev != nullptr && *a.force_log_dev != 0);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    init_bad |= (s < S) && !is_neg_inf(x[k]) && (x[k] - Rd < -100.f);  // beyond the linear range
    z[k] = s < S ? ex2(x[k] - Rd) : 0.f;
    td[k] = is_leaf ? 0.f : z[k];
    PB[s] = z[k];
    T2[lo16(tr[k])] = z[k];
    T2[hi16(tr[k])] = -z[k];
    zmax_l = fmaxf(zmax_l, z[k]);
    zsum_l += z[k];
  }
  float R = Rd;
  bool fallback = __syncthreads_or(init_bad) != 0;
  int cur = 0;
  float dres = 0.f;  // last-iteration residual max|Pi_new - Pi_prev| (finite entries)
  for (int it = 1; it < a.pi_iters && !fallback; ++it) {
    float* Tc = T2 + cur * 2 * NTV;
    float* Pc = PB + cur * NTV;
    float* Tn = T2 + (cur ^ 1) * 2 * NTV;
    float* Pn = PB + (cur ^ 1) * NTV;
    __syncthreads();
    float zmax = zmax_l, zsum = zsum_l;
    block_scan_ch_maxsum<2 * VPT>(Tc, red, zmax, zsum);
    const float inv = zmax > 0.f ? 1.0f / zmax : 0.f;
    const float Rn = zmax > 0.f ? R + lg2(zmax) : R;
    const float fd = ex2(Rd - Rn);
    const float lf = is_leaf ? ex2(leafv - Rn) : 0.f;
    const float thresh = 7.8886091e-31f;  // 2^-100 of the (unit) row scale
    bool bad = Rn - Rd > 26.f;  // dts / leaf terms rescaled below the normal range
    zmax_l = 0.f;
    zsum_l = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      const float path = Tc[lo16(tr[k])] + z[k];
      const float D = fmaxf(zsum - path, 0.f);
      float lin = z[k] * kA[k];
      lin = fmaf(D, kB[k], lin);
      lin = fmaf(Pc[lo16(cc[k])], kC1[k], lin);
      lin = fmaf(Pc[hi16(cc[k])], kC2[k], lin);
      float zn = fmaf(lin, inv, td[k] * fd);
      if (k == leafk) zn += lf;
      bad |= (zn > 0.f) & (zn < thresh);
      if (a.residual && it == a.pi_iters - 1 && zn > 0.f && z[k] > 0.f)
        dres = fmaxf(dres, fabsf(lg2(zn) - lg2(z[k] * inv)));
      z[k] = zn;
      zmax_l = fmaxf(zmax_l, zn);
      zsum_l += zn;
      if (it < a.pi_iters - 1) {
        Pn[s] = zn;
        Tn[lo16(tr[k])] = zn;
        Tn[hi16(tr[k])] = -zn;
      }
    }
    R = Rn;
    if (__syncthreads_or(bad)) {
      fallback = true;
      break;
    }
    cur ^= 1;
  }

  float pf[VPT];  // final Pi (log values)
  if (!fallback) {
    if (a.residual) {
      const float d = block_max(dres, red);
      if (threadIdx.x == 0) a.residual[row] = d;
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) pf[k] = lg2(z[k]) + R;
  } else {
    // log-space recomputation of the whole row from its initial values (rare)
    if (threadIdx.x == 0 && a.fallback_count) atomicAdd(a.fallback_count, 1);
    float* P = PB;
    float* X = T2;
    float* Y = T2 + NTV;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) P[threadIdx.x + k * NT] = x[k];
    __syncthreads();
    float nv[VPT];
    for (int it = 1; it < a.pi_iters; ++it) {
      log_iter<VPT>(P, X, Y, red, c, cb, leaf, leafv, is_leaf ? nullptr : x, nv);
      if (a.residual && it == a.pi_iters - 1) {
        float d = 0.f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int s = threadIdx.x + k * NT;
          if (s < S && !is_neg_inf(nv[k]) && !is_neg_inf(P[s])) d = fmaxf(d, fabsf(nv[k] - P[s]));
        }
        d = block_max(d, red);
        if (threadIdx.x == 0) a.residual[row] = d;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * NT;
        if (s < S) P[s] = nv[k];
      }
      __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      pf[k] = s < S ? P[s] : neg_inf();
    }
  }

  // ---- final Pi, row max, Pibar (from the final log row, as the reference computes them) ----
  float* prow = a.pi + (size_t)row * S;
  float mx = neg_inf();
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    if (s < S) {
      prow[s] = pf[k];
      float w = pf[k];
      if (c.use_col) w += c.col[s];
      mx = fmaxf(mx, w);
    }
  }
  const float row_max = block_max(mx, red);
  const float rms = safe_max(row_max);
  float pe[VPT];
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    float w = pf[k];
    if (c.use_col && s < S) w += c.col[s];
    pe[k] = s < S ? ex2(w - rms) : 0.f;
    T2[lo16(tr[k])] = pe[k];
    T2[hi16(tr[k])] = -pe[k];
    sum += pe[k];
  }
  __syncthreads();
  float rmx_unused = 0.f;
  block_scan_ch_maxsum<2 * VPT>(T2, red, rmx_unused, sum);
  const float row_sum = sum;
  float* brow = a.pibar + (size_t)row * S;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    if (s < S) {
      const float denom = row_sum - (T2[lo16(tr[k])] + pe[k]);
      brow[s] = denom > 0.f ? lg2(denom) + row_max + c.mc[cb + s] : neg_inf();
    }
  }
  if (threadIdx.x == 0) a.row_max[row] = row_max;
}

// ------------------------------------------------------------------------------------------
// forward, tour-table variant (rows of up to 4096 padded columns)
// ------------------------------------------------------------------------------------------
//
// Same arithmetic as level_forward_kernel, with the work per column and iteration cut down:
//  * VF = 8 columns per thread (fewer threads per row amortise the block-wide scan);
//  * the Euler tour lives in a swizzled layout: thread t scans the 2*VF consecutive tour entries
//    [t*2VF, (t+1)*2VF) as float4 groups whose order inside the chunk is XOR-permuted by t, so the
//    vector loads of a quarter-warp hit distinct banks; the host tables hold the BYTE offsets of
//    every column's enter / exit slot and of its species children's enter slots, so a scatter or
//    gather is one mask/shift and one shared-memory access;
//  * the speciation gathers read the children's values from the tour buffer before it is scanned
//    (no separate row buffer);
//  * the leaf term is folded into the constant term (both are constants times 2^(R0 - R));
//  * the split reduction prefetches the next split's child rows with cp.async while it reduces
//    the current one (one barrier per split).

// Tour tables of one column (host: tree.pack_forward):
//   tb[s]         children columns c1 | c2 << 16 (missing child -> a padded column)
//   tb[NTV + s]   byte offsets of the children's enter slots (lo | hi << 16)
//   tb[2NTV + s]  byte offsets of the column's own enter | exit slots
__device__ __forceinline__ const float& lds_at(const char* base, unsigned off) {
  return *reinterpret_cast<const float*>(base + off);
}
__device__ __forceinline__ float& sts_at(char* base, unsigned off) { return *reinterpret_cast<float*>(base + off); }

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Exclusive scan, in place, of the swizzled tour buffer T (NT * 2VF floats), fused with the
// block max of mx and the block sum of sm (returned to every thread).  red >= 96 floats.
// The caller syncs before (the buffer is complete); two barriers inside, the second on exit.
template <int VF>
__device__ __forceinline__ void tour_scan_sw(float* T, float* red, float& mx, float& sm) {
  constexpr int Q = VF / 2;  // float4 groups per thread chunk
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5, nw = blockDim.x >> 5;
  const int sw = Q == 1 ? 0 : ((t / (8 / Q)) & (Q - 1));
  float4* base = reinterpret_cast<float4*>(T) + t * Q;
  float gs[Q];
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const float4 v = base[q ^ sw];
    gs[q] = (v.x + v.y) + (v.z + v.w);
  }
  float local = 0.f;
#pragma unroll
  for (int q = 0; q < Q; ++q) local += gs[q];
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  mx = warp_max(mx);
  sm = warp_sum(sm);
  if (lane == 31) red[wid] = incl;
  if (lane == 0) { red[32 + wid] = mx; red[64 + wid] = sm; }
  __syncthreads();
  float tt = lane < nw ? red[lane] : 0.f;
  const float bm = lane < nw ? red[32 + lane] : 0.f;
  const float bs = lane < nw ? red[64 + lane] : 0.f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, tt, o);
    if (lane >= o) tt += y;
  }
  mx = warp_max(bm);
  sm = warp_sum(bs);
  const float prev = __shfl_up_sync(0xffffffffu, tt, 1);
  float run = __shfl_sync(0xffffffffu, lane == 0 ? 0.f : prev, wid) + incl - local;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const float4 v = base[q ^ sw];
    float4 o;
    o.x = run;
    o.y = run + v.x;
    o.z = o.y + v.y;
    o.w = o.z + v.z;
    base[q ^ sw] = o;
    run += gs[q];
  }
  __syncthreads();
}

// The same scan with one barrier: T (the swizzled tour, NT * 2VF floats) is only read, and the
// WITHIN-WARP exclusive prefix of every slot goes to X (same layout) before the barrier that
// publishes the warp totals.  Lane w of every warp returns in wx the exclusive prefix of warp w's
// total, so the prefix of the slot at byte offset off is
//     lds_at(X, off) + __shfl_sync(full, wx, off / (4 * 64 * VF))
// (64 VF floats per warp), readable after the return without another barrier.  Block max of mx
// and block sum of sm as tour_scan_sw.  The caller syncs before (T complete); X's previous readers
// must be past a barrier that precedes this call.
template <int VF>
__device__ __forceinline__ void tour_scan_sw_wx(const float* T, float* X, float* red, float& mx, float& sm,
                                                float& wx) {
  constexpr int Q = VF / 2;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5, nw = blockDim.x >> 5;
  const int sw = Q == 1 ? 0 : ((t / (8 / Q)) & (Q - 1));
  const float4* base = reinterpret_cast<const float4*>(T) + t * Q;
  float4* xb = reinterpret_cast<float4*>(X) + t * Q;
  float4 v[Q];
  float gs[Q];
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    v[q] = base[q ^ sw];
    gs[q] = (v[q].x + v[q].y) + (v[q].z + v[q].w);
  }
  float local = 0.f;
#pragma unroll
  for (int q = 0; q < Q; ++q) local += gs[q];
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  float run = incl - local;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    float4 o;
    o.x = run;
    o.y = run + v[q].x;
    o.z = o.y + v[q].y;
    o.w = o.z + v[q].z;
    xb[q ^ sw] = o;
    run += gs[q];
  }
  mx = warp_max(mx);
  sm = warp_sum(sm);
  if (lane == 31) red[wid] = incl;
  if (lane == 0) { red[32 + wid] = mx; red[64 + wid] = sm; }
  __syncthreads();
  float tt = lane < nw ? red[lane] : 0.f;
  const float bm = lane < nw ? red[32 + lane] : 0.f;
  const float bs = lane < nw ? red[64 + lane] : 0.f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, tt, o);
    if (lane >= o) tt += y;
  }
  mx = warp_max(bm);
  sm = warp_sum(bs);
  const float prev = __shfl_up_sync(0xffffffffu, tt, 1);
  wx = lane == 0 ? 0.f : prev;
}

// The slot prefix of tour_scan_sw_wx at byte offset off.
template <int VF>
__device__ __forceinline__ float tour_prefix_wx(const char* X, unsigned off, float wx) {
  return lds_at(X, off) + __shfl_sync(0xffffffffu, wx, (int)(off / (4u * 64u * VF)));
}

struct Fwd4Args {
  FwdArgs f;
  const unsigned* tb;   // [3, NTV] tour tables
  const float4* k4;     // [G, NTV] (2^dl + 2^ebar, 2^(mc+e), 2^sl1, 2^sl2), zero on padded columns
  long long k4_rows;    // row stride of k4 in float4 (0: one shared item row)
};

__device__ __forceinline__ void cp_async16_cg(void* smem_dst, const void* gsrc) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}

// Starts copying one row of S floats at src (4-byte aligned) into the shared slot B (16-byte
// aligned, >= NTV + 4 floats) and returns the row's view P (P[s] = src[s]): the 16-byte aligned
// body goes by asynchronous L2 copies (cp.async.cg: no L1, so rows written earlier in the same
// launch are read correctly), the at most 3 + 3 unaligned end floats by loads; columns S..NTV-1
// of the view are set to -inf when pad_neg_inf.  The caller commits, waits and syncs before use.
__device__ __forceinline__ const float* stage_row_cg(float* B, const float* src, int S, int NTV, bool pad_neg_inf) {
  const int a = (int)(((16u - ((unsigned)(uintptr_t)src & 15u)) & 15u) >> 2);  // floats before a 16-B boundary
  float* P = B + ((4 - a) & 3);                                                 // P + a is 16-B aligned
  const int nb = S > a ? (S - a) >> 2 : 0;
  for (int j = threadIdx.x; j < nb; j += blockDim.x) cp_async16_cg(P + a + 4 * j, src + a + 4 * j);
  const int head = a < S ? a : S;
  for (int s = threadIdx.x; s < head; s += blockDim.x) P[s] = __ldcg(src + s);
  for (int s = head + 4 * nb + threadIdx.x; s < S; s += blockDim.x) P[s] = __ldcg(src + s);
  if (pad_neg_inf)
    for (int s = S + threadIdx.x; s < NTV; s += blockDim.x) P[s] = neg_inf();
  return P;
}

// ---- bulk (TMA) row copies into shared memory, completion counted on an mbarrier ----
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Split staging of the dataflow forward: the aligned middle of each child Pi row arrives by one
// bulk copy (issued by thread 0, counted on the buffer's mbarrier), the unaligned ends and the
// padding by plain loads.  Every thread tracks the parity of each buffer's next completion.
struct BulkStage {
  unsigned long long* bar;  // [2] mbarriers (one per staging buffer), shared memory
  unsigned phase;           // bit b: parity of bar[b]'s next completion
  int* error;               // set when a wait gives up
  long long max_polls;
};

// Stage rows s0 and s1 (S floats each) into slots B0 / B1 (NTV + 4 floats each), padded with
// `pad` up to NTV; returns the aligned views.  Called by all threads after the slots' previous
// readers are done (a barrier); one arrival on `bar` (with the copies' byte count) per call;
// completion: bulk_wait on the same mbarrier, then bulk_fix_pad on each view, then a barrier.
// Where the 16-byte aligned cover of a row, [row - lead, row + S rounded up), lies inside
// [lo, hi) (the buffer the rows belong to), ONE bulk copy brings the cover -- a few floats of
// the neighbouring rows included, never read -- and no thread loads the row's unaligned ends
// (they would hold their warp up for a load latency per split); otherwise the aligned middle
// goes by bulk copy and the ends by loads.
__device__ __forceinline__ void stage_rows_bulk(float* B0, const float* s0, float* B1, const float* s1, int S,
                                                int NTV, unsigned long long* bar, const float** v0,
                                                const float** v1, float pad = neg_inf(), const float* lo = nullptr,
                                                const float* hi = nullptr) {
  const int a0 = (int)(((16u - ((unsigned)(uintptr_t)s0 & 15u)) & 15u) >> 2);
  const int a1 = (int)(((16u - ((unsigned)(uintptr_t)s1 & 15u)) & 15u) >> 2);
  const int l0 = (4 - a0) & 3, l1 = (4 - a1) & 3;  // floats of the cover before the row
  float* P0 = B0 + l0;
  float* P1 = B1 + l1;
  const int c0 = (l0 + S + 3) >> 2, c1 = (l1 + S + 3) >> 2;  // 16-byte units of the covers
  const bool w0 = lo != nullptr && s0 - l0 >= lo && s0 - l0 + 4 * c0 <= hi;
  const bool w1 = lo != nullptr && s1 - l1 >= lo && s1 - l1 + 4 * c1 <= hi;
  const int nb0 = w0 ? c0 : (S > a0 ? (S - a0) >> 2 : 0), nb1 = w1 ? c1 : (S > a1 ? (S - a1) >> 2 : 0);
  if (threadIdx.x == 0) {
    // generic-proxy writes -> this thread's bulk copies: the child rows other CTAs wrote (made
    // visible to this thread by the queue's acquire).  The slots' previous readers finished before
    // the caller's barrier, which orders them before any write to the slots.
    asm volatile("fence.proxy.async.global;" ::: "memory");
    mbar_arrive_expect_tx(bar, (unsigned)(16 * (nb0 + nb1)));
    if (nb0) bulk_copy_g2s(w0 ? B0 : P0 + a0, w0 ? s0 - l0 : s0 + a0, (unsigned)(16 * nb0), bar);
    if (nb1) bulk_copy_g2s(w1 ? B1 : P1 + a1, w1 ? s1 - l1 : s1 + a1, (unsigned)(16 * nb1), bar);
  }
  if (!w0) {
    const int h0 = a0 < S ? a0 : S;
    for (int s = threadIdx.x; s < h0; s += blockDim.x) P0[s] = __ldcg(s0 + s);
    for (int s = h0 + 4 * nb0 + threadIdx.x; s < S; s += blockDim.x) P0[s] = __ldcg(s0 + s);
  }
  if (!w1) {
    const int h1 = a1 < S ? a1 : S;
    for (int s = threadIdx.x; s < h1; s += blockDim.x) P1[s] = __ldcg(s1 + s);
    for (int s = h1 + 4 * nb1 + threadIdx.x; s < S; s += blockDim.x) P1[s] = __ldcg(s1 + s);
  }
  // the padding the covers' copies may overwrite (at most 3 floats past S) is written by
  // bulk_fix_pad after the wait; the rest now
  for (int s = S + 3 + threadIdx.x; s < NTV; s += blockDim.x) {
    P0[s] = pad;
    P1[s] = pad;
  }
  *v0 = P0;
  *v1 = P1;
}

// The first padding entries of a staged view, after its copies completed (the same threads'
// bulk_wait) and before the barrier that publishes the slot.
__device__ __forceinline__ void bulk_fix_pad(const float* P, int S, int NTV, float pad = neg_inf()) {
  const int s = S + (int)threadIdx.x;
  if (threadIdx.x < 3 && s < NTV) const_cast<float*>(P)[s] = pad;
}

__device__ __forceinline__ void bulk_wait(BulkStage& bs, int b) {
  const unsigned parity = (bs.phase >> b) & 1u;
  long long polls = 0;
  while (!mbar_try_wait(bs.bar + b, parity)) {
    if (++polls > bs.max_polls) {  // cannot happen with valid copies; results flagged invalid
      if (bs.error) atomicExch(bs.error, 1);
      break;
    }
  }
  bs.phase ^= 1u << b;
}

// Loads of rows that other CTAs of the SAME launch produce (the dataflow schedule) bypass L1:
// L1 is not coherent across SMs, and a row's first and last cache lines are shared with its
// neighbours.  Level launches keep the cached / asynchronous paths.
template <bool DF>
__device__ __forceinline__ float ld_row(const float* p) {
  if constexpr (DF) return __ldcg(p);
  else return __ldg(p);
}

// One row of the forward tour kernel (the body of level_forward_tour_kernel and of the dataflow
// kernel): split reduction or leaf seed, pi_iters linear-space iterations, final Pi / Pibar.
// Splits [i0, i1) of the split arrays; sm: the CTA's dynamic shared memory.
template <int VF, bool DF>
__device__ __forceinline__ void forward_tour_row(const Fwd4Args& args, long long row, long long i0, long long i1,
                                                 float* sm, BulkStage* bs = nullptr) {
  const FwdArgs& a = args.f;
  const LevelConsts& c = a.c;
  const unsigned* __restrict__ tb = args.tb;
  const int S = c.S;
  const int NT = blockDim.x;
  const int NTV = NT * VF;
  const int TB = 2 * NTV;  // floats per tour buffer
  float* red = sm + 8 * (NTV + 4);  // after the split staging slots (the tour buffers alias them)
  char* T0 = reinterpret_cast<char*>(sm);
  char* T1 = reinterpret_cast<char*>(sm + TB);
  char* TX = reinterpret_cast<char*>(sm + 2 * TB);  // the iterations' scanned prefixes (6 NTV <= 8 (NTV + 4))
  const int tid = threadIdx.x;
  const long long item = c.item_idx[row];
  const size_t cb = (size_t)(item * c.crs);
  const size_t pb = (size_t)(item * c.prs);
  const int leaf_raw = c.leaf_state[row];
  const bool is_leaf = (i0 == i1) && leaf_raw >= 0 && leaf_raw < S;
  const int leaf = is_leaf ? leaf_raw : -1;
  const float leafv = is_leaf ? c.leaf_logp[(size_t)item * S + leaf] : neg_inf();

  // ---- initial row (log values): leaf seed or split reduction ----
  float x[VF];
  if (is_leaf) {
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const int s = tid + k * NT;
      x[k] = s < S ? leaf_seed(c, cb, item, leaf, s) : neg_inf();
    }
  } else {
    // Staging: per split the four child rows (Pi_l, Pi_r, Pibar_l, Pibar_r), double-buffered by
    // split parity, each row a view at a 16-byte aligned position of a slot of NTV + 4 floats.
    float* stg = sm;
    const int RS = NTV + 4;
    unsigned ccol[VF];
    float m[VF], acc[VF], kD[VF], kS[VF];
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const int s = tid + k * NT;
      ccol[k] = __ldg(tb + s);
      m[k] = neg_inf();
      acc[k] = 0.f;
      kD[k] = s < S ? __ldg(c.log_pD + pb + s) : 0.f;
      kS[k] = s < S ? __ldg(c.log_pS + pb + s) : 0.f;
    }
    // Pi rows are staged (the speciation terms gather them at the children's columns); Pibar rows
    // are only read at the own column and come straight from global memory
    const float *cPl, *cPr;
    const bool bulk = DF && bs != nullptr;
    {
      const long long l = a.sp.sl[i0], r = a.sp.sr[i0];
      if (bulk) {
        stage_rows_bulk(stg, a.Pi_src + (size_t)l * S, stg + RS, a.Pi_src + (size_t)r * S, S, NTV, bs->bar, &cPl,
                        &cPr, neg_inf(), a.Pi_src, a.Pi_src + (size_t)a.n_rows * S);
      } else {
        cPl = stage_row_cg(stg, a.Pi_src + (size_t)l * S, S, NTV, true);
        cPr = stage_row_cg(stg + RS, a.Pi_src + (size_t)r * S, S, NTV, true);
        cp_async_commit();
      }
    }
    for (long long i = i0; i < i1; ++i) {
      const int par = (int)((i - i0) & 1);
      const long long li = a.sp.sl[i], ri = a.sp.sr[i];
      float bl[VF], br[VF];  // issued before the wait: their latency overlaps it
#pragma unroll
      for (int k = 0; k < VF; ++k) {
        const int s = tid + k * NT;
        bl[k] = s < S ? ld_row<DF>(a.Pibar_src + (size_t)li * S + s) : 0.f;
        br[k] = s < S ? ld_row<DF>(a.Pibar_src + (size_t)ri * S + s) : 0.f;
      }
      if (bulk) {
        bulk_wait(*bs, par);
        bulk_fix_pad(cPl, S, NTV);
        bulk_fix_pad(cPr, S, NTV);
      } else {
        cp_async_wait_all();
      }
      __syncthreads();  // split i staged; everyone is done with split i-1's slots
      const float *nPl = nullptr, *nPr = nullptr;
      if (i + 1 < i1) {
        float* nb = stg + (par ^ 1) * 4 * RS;
        const long long l = a.sp.sl[i + 1], r = a.sp.sr[i + 1];
        if (bulk) {
          stage_rows_bulk(nb, a.Pi_src + (size_t)l * S, nb + RS, a.Pi_src + (size_t)r * S, S, NTV,
                          bs->bar + (par ^ 1), &nPl, &nPr, neg_inf(), a.Pi_src, a.Pi_src + (size_t)a.n_rows * S);
        } else {
          nPl = stage_row_cg(nb, a.Pi_src + (size_t)l * S, S, NTV, true);
          nPr = stage_row_cg(nb + RS, a.Pi_src + (size_t)r * S, S, NTV, true);
          cp_async_commit();
        }
      }
      const float lsp = a.sp.lsp[i];
#pragma unroll
      for (int k = 0; k < VF; ++k) {
        const int s = tid + k * NT;
        if (s < S) {
          const unsigned ca = ccol[k] & 0xFFFFu, cbb = ccol[k] >> 16;
          const float pl = cPl[s], pr = cPr[s];
          // left-to-right sums, as the reference forms the terms (dts_fused.py:54-60): at log
          // magnitudes ~1e2 a different association moves the terms by an ulp (~1e-5)
          const float lss = lsp + kS[k];
          const float v0 = lsp + kD[k] + pl + pr;
          const float v1 = lsp + pl + br[k];
          const float v2 = lsp + pr + bl[k];
          const float v3 = lss + cPl[ca] + cPr[cbb];
          const float v4 = lss + cPr[ca] + cPl[cbb];
          const float mx = fmaxf(fmaxf(fmaxf(m[k], v0), fmaxf(v1, v2)), fmaxf(v3, v4));
          const float ms = safe_max(mx);
          acc[k] = fmaf(acc[k], ex2(m[k] - ms),
                        ((ex2(v0 - ms) + ex2(v1 - ms)) + (ex2(v2 - ms) + ex2(v3 - ms))) + ex2(v4 - ms));
          m[k] = mx;
        }
      }
      cPl = nPl; cPr = nPr;
    }
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const int s = tid + k * NT;
      x[k] = s < S ? lg2(acc[k]) + m[k] : neg_inf();
      if (s < S) a.dts_save[(size_t)row * S + s] = x[k];
    }
  }
  float m0 = neg_inf();
#pragma unroll
  for (int k = 0; k < VF; ++k) m0 = fmaxf(m0, x[k]);
  const float Rd = safe_max(block_max(m0, red));  // scale of the initial row; syncs (staging done)

  // ---- linear-space iterations (see level_forward_kernel) ----
  const float4* __restrict__ k4 = args.k4 + (size_t)(item * args.k4_rows);
  unsigned ce[VF], tr[VF];
  float z[VF], td[VF], kA[VF], kB[VF], kC1[VF], kC2[VF];
  float zmax_l = 0.f, zsum_l = 0.f;
  bool bad = a.force_log != 0 || (a.force_log_dev != nullptr && *a.force_log_dev != 0);
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    const bool real = s < S;
    bad |= real && !is_neg_inf(x[k]) && (x[k] - Rd < -100.f);  // beyond the linear range
    ce[k] = __ldg(tb + NTV + s);
    tr[k] = __ldg(tb + 2 * NTV + s);
    const float4 kk = __ldg(k4 + s);  // zero on padded columns
    kA[k] = kk.x; kB[k] = kk.y; kC1[k] = kk.z; kC2[k] = kk.w;
    z[k] = real ? ex2(x[k] - Rd) : 0.f;
    td[k] = is_leaf ? (s == leaf ? ex2(leafv - Rd) : 0.f) : z[k];
    sts_at(T0, tr[k] & 0xFFFFu) = z[k];
    sts_at(T0, tr[k] >> 16) = -z[k];
    zmax_l = fmaxf(zmax_l, z[k]);
    zsum_l += z[k];
  }
  float R = Rd;
  bool fallback = false;
  float dres = 0.f;
  const int last = a.pi_iters - 1;
  for (int it = 1; it <= last; ++it) {
    char* Tc = (it & 1) ? T0 : T1;
    char* Tn = (it & 1) ? T1 : T0;
    if (__syncthreads_or(bad)) {
      fallback = true;
      break;
    }
    float part[VF];  // speciation terms z[c1] 2^sl1 + z[c2] 2^sl2, gathered before the scan
#pragma unroll
    for (int k = 0; k < VF; ++k)
      part[k] = fmaf(lds_at(Tc, ce[k] & 0xFFFFu), kC1[k], lds_at(Tc, ce[k] >> 16) * kC2[k]);
    // Tc stays as it is (the speciation gathers above read it); the prefixes go to TX, whose
    // readers of the previous iteration are past the barrier at the top of this one
    float zmax = zmax_l, zsum = zsum_l, wx;
    tour_scan_sw_wx<VF>(reinterpret_cast<const float*>(Tc), reinterpret_cast<float*>(TX), red, zmax, zsum, wx);
    const float inv = zmax > 0.f ? 1.0f / zmax : 0.f;
    const float Rn = zmax > 0.f ? R + lg2(zmax) : R;
    const float fd = ex2(Rd - Rn);
    unsigned mincode = 0xFFFFFFFFu;  // min over (bits(zn) - 1): < bits(2^-100) - 1 flags a tiny nonzero
    zmax_l = 0.f;
    zsum_l = 0.f;
    const bool resid = (it == last) && (a.residual != nullptr);
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const float path = tour_prefix_wx<VF>(TX, tr[k] & 0xFFFFu, wx) + z[k];
      const float D = fmaxf(zsum - path, 0.f);
      const float lin = fmaf(D, kB[k], fmaf(z[k], kA[k], part[k]));
      const float zn = fmaf(lin, inv, td[k] * fd);
      mincode = min(mincode, (unsigned)__float_as_int(zn) - 1u);
      if (resid && zn > 0.f && z[k] > 0.f) dres = fmaxf(dres, fabsf(lg2(zn) - lg2(z[k] * inv)));
      z[k] = zn;
      zmax_l = fmaxf(zmax_l, zn);
      zsum_l += zn;
      if (it < last) {
        sts_at(Tn, tr[k] & 0xFFFFu) = zn;
        sts_at(Tn, tr[k] >> 16) = -zn;
      }
    }
    bad = mincode < 0x0D7FFFFFu || Rn - Rd > 26.f;  // bits(2^-100) - 1; dts term below the normal range
    R = Rn;
  }
  if (!fallback && __syncthreads_or(bad)) fallback = true;

  float pf[VF];  // final Pi (log values)
  if (!fallback) {
    if (a.residual) {
      const float d = block_max(dres, red);
      if (tid == 0) a.residual[row] = d;
    }
#pragma unroll
    for (int k = 0; k < VF; ++k) pf[k] = lg2(z[k]) + R;
  } else {
    // log-space recomputation of the whole row from its initial values (rare)
    if (tid == 0 && a.fallback_count) atomicAdd(a.fallback_count, 1);
    float* P = sm;
    float* X = sm + NTV;
    float* Y = sm + 2 * NTV;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const int s = tid + k * NT;
      x[k] = s >= S ? neg_inf() : (is_leaf ? leaf_seed(c, cb, item, leaf, s) : a.dts_save[(size_t)row * S + s]);
      P[s] = x[k];
    }
    __syncthreads();
    float nv[VF];
    for (int it = 1; it < a.pi_iters; ++it) {
      log_iter<VF>(P, X, Y, red, c, cb, leaf, leafv, is_leaf ? nullptr : x, nv);
      if (a.residual && it == a.pi_iters - 1) {
        float d = 0.f;
#pragma unroll
        for (int k = 0; k < VF; ++k) {
          const int s = tid + k * NT;
          if (s < S && !is_neg_inf(nv[k]) && !is_neg_inf(P[s])) d = fmaxf(d, fabsf(nv[k] - P[s]));
        }
        d = block_max(d, red);
        if (tid == 0) a.residual[row] = d;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < VF; ++k) {
        const int s = tid + k * NT;
        if (s < S) P[s] = nv[k];
      }
      __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const int s = tid + k * NT;
      pf[k] = s < S ? P[s] : neg_inf();
    }
    __syncthreads();
  }

  // ---- final Pi, row max, Pibar (from the final log row, as the reference computes them) ----
  float* prow = a.pi + (size_t)row * S;
  float mx = neg_inf();
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    if (s < S) prow[s] = pf[k];
    mx = fmaxf(mx, pf[k]);
  }
  // the tour buffer not read by the last iteration (T0 when pi_iters-1 is odd) takes the weights
  char* Tf = fallback ? T1 : ((last & 1) ? T1 : T0);
  float* Tff = reinterpret_cast<float*>(Tf);
  const float row_max = block_max(mx, red);
  const float rms = safe_max(row_max);
  float pe[VF];
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    pe[k] = s < S ? ex2(pf[k] - rms) : 0.f;
    sts_at(Tf, tr[k] & 0xFFFFu) = pe[k];
    sts_at(Tf, tr[k] >> 16) = -pe[k];
    sum += pe[k];
  }
  __syncthreads();
  float unused = 0.f;
  tour_scan_sw<VF>(Tff, red, unused, sum);
  float* brow = a.pibar + (size_t)row * S;
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    if (s < S) {
      const float denom = sum - (lds_at(Tf, tr[k] & 0xFFFFu) + pe[k]);
      brow[s] = denom > 0.f ? lg2(denom) + row_max + c.mc[cb + s] : neg_inf();
    }
  }
  if (tid == 0) a.row_max[row] = row_max;
}

template <int VF>
__global__ void __launch_bounds__(512, 1) level_forward_tour_kernel(Fwd4Args args) {
  extern __shared__ __align__(16) float sm[];
  const int b = blockIdx.x;
  forward_tour_row<VF, false>(args, args.f.sp.rows[b], args.f.sp.split_ptr[b], args.f.sp.split_ptr[b + 1], sm);
}

// ------------------------------------------------------------------------------------------
// dataflow schedule: one persistent launch, rows start when their children are done
// ------------------------------------------------------------------------------------------
//
// Level launches make every row of a level wait for the slowest row of the previous level; near
// the root most levels hold fewer rows than there are SMs, so most of the GPU idles.  Here each
// row keeps a count of unfinished child rows; a CTA that finishes a row decrements the counts of
// the row's parents and appends those that reach zero to a device queue; persistent CTAs take
// queue slots in order.  Every wait on a queue slot is bounded: past the limit the CTA records an
// error and leaves (the host then reports the failure; it never hangs).  A CTA waiting on a slot
// relies on the CTAs that will fill it being resident, so the grid is sized from the occupancy
// query and launched cooperatively: the launch either makes every CTA co-resident or fails (on a
// GPU shared with other work, e.g. under MPS with fewer SMs), reported as a launch error.

// Work items are (group, row) pairs, item = group * C + row: one group for the forward and the
// backward, one per tangent direction pair; an item waits for the same group's dependencies.
struct Flow {
  int* queue;              // [n_items] items in start order; -1 = slot not yet filled
  int* remaining;          // [n_items] unfinished dependencies per item
  unsigned* head;          // next slot to take
  unsigned* tail;          // next slot to fill
  int* error;              // set to 1 when a wait gave up
  const long long* par_ptr;  // [C+1] CSR: the rows released by each row
  const int* par_idx;
  const long long* row_split_ptr;  // [C+1] splits of each row (row-id order)
  int C;
  long long max_polls;
  int n_items;             // C * groups
  // 1: the queue is pre-filled with every item in a fixed start order (dependencies first); a CTA
  // takes the next slot and waits until the item's remaining count reaches zero; finishing only
  // decrements the dependents' counts
  int static_order;
};

// Per-CTA state of the dataflow loop (shared memory; the poller sets next = -1 before the loop).
struct FlowSlot {
  int row;   // the claimed item, broadcast to the CTA
  int next;  // queue ticket taken ahead by flow_finish_row, -1 = none (read by the poller only)
};

// The one thread that takes queue tickets and waits on them: thread 32 (warp 1, so that warp 0
// releases dependent rows meanwhile), or thread 0 in a one-warp block (no ticket taken ahead).
__device__ __forceinline__ unsigned flow_poller() { return blockDim.x > 32 ? 32u : 0u; }

// Claims the next queue slot (the ticket taken ahead, if any) and waits (bounded) until it holds
// a row.  Returns the row, -1 when every row has been taken, -2 on a timeout (error recorded).
// Called by all threads.
__device__ __forceinline__ int flow_next_row(const Flow& f, FlowSlot* st) {
  if (threadIdx.x == flow_poller()) {
    const unsigned idx = st->next >= 0 ? (unsigned)st->next : atomicAdd(f.head, 1u);
    st->next = -1;
    int row = -1;
    if (idx < (unsigned)f.n_items) {
      const volatile int* q = f.queue + idx;
      long long polls = 0;
      row = *q;
      while (row < 0) {
        if (++polls > f.max_polls || *(volatile int*)f.error) {
          atomicExch(f.error, 1);
          row = -2;
          break;
        }
        __nanosleep(128);
        row = *q;
      }
      if (f.static_order && row >= 0) {  // the slot holds its item from the start: wait until it is ready
        const volatile int* rem = f.remaining + row;
        while (*rem > 0) {
          if (++polls > f.max_polls || *(volatile int*)f.error) {
            atomicExch(f.error, 1);
            row = -2;
            break;
          }
          __nanosleep(64);
        }
      }
      __threadfence();  // the row's children, written before it was queued (released), are visible
    }
    st->row = row;
  }
  __syncthreads();
  // st->row is written again only in the next call, after flow_finish_row's barrier, which every
  // thread reaches after this read
  return st->row;
}

// After a row's outputs are written by the whole CTA: release the rows that wait on it (one lane
// of warp 0 per dependent row) while the poller (thread 32) takes the CTA's next queue ticket; the
// ticket stays with the thread that waits on it, so no barrier follows.
__device__ __forceinline__ void flow_finish_row(const Flow& f, int row, FlowSlot* st) {
  __threadfence();  // every thread's outputs (stores and atomics) are device-visible ...
  __syncthreads();  // ... before warp 0 releases the dependent rows
  if (threadIdx.x < 32) {
    const int grp = row / f.C;
    const int r = row - grp * f.C;
    for (long long j = f.par_ptr[r] + threadIdx.x; j < f.par_ptr[r + 1]; j += 32) {
      const int p = grp * f.C + f.par_idx[j];
      if (f.static_order) {
        atomicSub(f.remaining + p, 1);  // value unused: a reduction, no round trip before the next row
      } else if (atomicSub(f.remaining + p, 1) == 1) {
        const unsigned slot = atomicAdd(f.tail, 1u);
        atomicExch(f.queue + slot, p);
      }
    }
  } else if (threadIdx.x == 32) {
    const unsigned idx = atomicAdd(f.head, 1u);
    st->next = idx < (unsigned)f.n_items ? (int)idx : f.n_items;  // >= n_items: nothing left
  }
}

template <int VF>
__global__ void __launch_bounds__(512, 1) flow_forward_kernel(Fwd4Args args, Flow f) {
  extern __shared__ __align__(16) float sm[];
  __shared__ FlowSlot fs;
  __shared__ __align__(8) unsigned long long bars[2];
  if (threadIdx.x == flow_poller()) fs.next = -1;
  if (threadIdx.x == 0) {
    mbar_init(bars, 1);
    mbar_init(bars + 1, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  BulkStage bs{bars, 0u, f.error, f.max_polls};
  for (;;) {
    const int row = flow_next_row(f, &fs);
    if (row < 0) break;
    forward_tour_row<VF, true>(args, row, f.row_split_ptr[row], f.row_split_ptr[row + 1], sm, &bs);
    flow_finish_row(f, row, &fs);
  }
}

// Queue / counter initialisation of one dataflow run: remaining = dep0 of each item's row, queue =
// the ready rows (n0 of them, given in ready0) of every group followed by -1, head = 0, tail =
// n0 * groups, error = 0.
__global__ void flow_init_kernel(Flow f, const int* dep0, const int* ready0, int n0) {
  const int groups = f.n_items / f.C;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < f.n_items; i += gridDim.x * blockDim.x) {
    f.remaining[i] = dep0[i % f.C];
    f.queue[i] = i < n0 * groups ? (i / n0) * f.C + ready0[i % n0] : -1;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *f.head = 0u;
    *f.tail = (unsigned)(n0 * groups);
    *f.error = 0;
  }
}

// ------------------------------------------------------------------------------------------
// tangent (forward-mode JVP) of one dependency level, every (row, direction) pair
// ------------------------------------------------------------------------------------------
//
// Restates, per row, newton/forward_tangent.py:150-193 for one wave row: the split tangent
// reduction (kbench/core/kernels/dts_tangent.py:23-96) followed by n_iters fixed-count Jacobi
// steps of the linearised wave step at the frozen primal row (wave_tangent.py:186-336), starting
// from a zero tangent.  The primal weights are folded into per-column coefficients once:
//   dPi' = cA dPi + c2 (dRS - dAS) + c3 dPi[c1] + c4 dPi[c2] + cst
// with dRS = sum_s r dPi, dAS = ancestor-or-self sum of r dPi (one Euler-tour scan per step),
// r = 2^(Pi - rowmax); dPibar = (dRS - dAS) / denom + dmc where the primal denominator is > 0.

struct TanArgs {
  SplitCSR sp;
  const float* Pi;      // primal [C,S]
  const float* Pibar;
  const float* dts;     // primal split reductions [C,S] (rows with splits)
  float* dPi;           // [D, C, S]
  float* dPibar;
  long long dstride;    // C * S
  const float* mc;      // primal constants (item * crs + s)
  const float* dl;
  const float* ebar;
  const float* e;
  const float* sl1;
  const float* sl2;
  const float* leaf_logp;  // item * S + s
  const float* log_pD;     // item * prs + s
  const float* log_pS;
  long long crs, prs;
  const float* dmc;     // tangent constants: direction * tstride + item * crs + s
  const float* ddl;
  const float* debar;
  const float* de;
  const float* dsl1;
  const float* dsl2;
  const float* dleaf;   // direction * tstride + item * S + s
  const float* dpD;     // direction * tstride + item * prs + s
  const float* dpS;
  long long tstride;
  const long long* item_idx;
  const int* leaf_state;
  const unsigned* tb;   // [3, NTV] tour tables
  const unsigned* tb2;  // [NTV] enter | exit byte offsets of the float2 (direction pair) tour layout
  int n_iters;
  int S;
};

template <int VF>
__global__ void __launch_bounds__(512, 1) level_tangent_kernel(TanArgs a) {
  extern __shared__ __align__(16) float sm[];
  const unsigned* __restrict__ tb = a.tb;
  const int S = a.S;
  const int NT = blockDim.x;
  const int NTV = NT * VF;
  const int TB = 2 * NTV;
  char* T0 = reinterpret_cast<char*>(sm);
  char* T1 = reinterpret_cast<char*>(sm + TB);
  float* DP0 = sm + 2 * TB;
  float* DP1 = DP0 + NTV;
  float* PR = DP1 + NTV;
  float* red = PR + NTV;
  const int tid = threadIdx.x;
  const int b = blockIdx.x;
  const int d = blockIdx.y;
  const long long row = a.sp.rows[b];
  const long long item = a.item_idx[row];
  const size_t cb = (size_t)(item * a.crs);
  const size_t pb = (size_t)(item * a.prs);
  const size_t tof = (size_t)d * a.tstride;
  const long long i0 = a.sp.split_ptr[b], i1 = a.sp.split_ptr[b + 1];
  const bool has_splits = i1 > i0;
  const int leaf_raw = a.leaf_state[row];
  const int leaf = (!has_splits && leaf_raw >= 0 && leaf_raw < S) ? leaf_raw : -1;

  unsigned ccol[VF], tr[VF];
  float pv[VF], r[VF];
  float m = neg_inf();
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    ccol[k] = __ldg(tb + s);
    tr[k] = __ldg(tb + 2 * NTV + s);
    pv[k] = s < S ? a.Pi[(size_t)row * S + s] : neg_inf();
    PR[s] = pv[k];
    m = fmaxf(m, pv[k]);
  }
  const float row_max = block_max(m, red);
  const float rms = safe_max(row_max);
  float rsum = 0.f;
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    r[k] = ex2(pv[k] - rms);  // 0 on padding (-inf)
    sts_at(T0, tr[k] & 0xFFFFu) = r[k];
    sts_at(T0, tr[k] >> 16) = -r[k];
    rsum += r[k];
  }
  __syncthreads();
  float unused = 0.f;
  tour_scan_sw<VF>(reinterpret_cast<float*>(T0), red, unused, rsum);
  const float row_sum = rsum;
  float cA[VF], c2[VF], c3[VF], c4[VF], cst[VF], cD[VF], invd[VF];
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    cA[k] = c2[k] = c3[k] = c4[k] = cst[k] = cD[k] = invd[k] = 0.f;
    if (s < S) {
      const float denom = row_sum - (lds_at(T0, tr[k] & 0xFFFFu) + r[k]);
      const bool pos = denom > 0.f;
      const float sd = pos ? denom : 1.f;
      invd[k] = pos ? 1.0f / sd : 0.f;
      const float pibar = pos ? lg2(sd) + row_max + a.mc[cb + s] : neg_inf();
      const float t0 = a.dl[cb + s] + pv[k];
      const float t1 = pv[k] + a.ebar[cb + s];
      const float t2 = pibar + a.e[cb + s];
      const float t3 = a.sl1[cb + s] + PR[ccol[k] & 0xFFFFu];
      const float t4 = a.sl2[cb + s] + PR[ccol[k] >> 16];
      const bool hit = s == leaf;
      const float t5 = hit ? a.leaf_logp[(size_t)item * S + s] : neg_inf();
      const float dv = has_splits ? a.dts[(size_t)row * S + s] : neg_inf();
      const float mm = fmaxf(fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(t4, t5)), dv);
      const float ms = safe_max(mm);
      const float e0 = ex2(t0 - ms), e1 = ex2(t1 - ms), e2 = ex2(t2 - ms), e3 = ex2(t3 - ms), e4 = ex2(t4 - ms),
                  e5 = ex2(t5 - ms), ed = ex2(dv - ms);
      const float tot = ((e0 + e1) + (e2 + e3)) + ((e4 + e5) + ed);
      if (!is_neg_inf(lg2(tot) + mm)) {
        const float inv = tot > 0.f ? 1.0f / tot : 0.f;
        const float dt5 = hit ? a.dleaf[tof + (size_t)item * S + s] : 0.f;
        const float dmcv = pos ? a.dmc[tof + cb + s] : 0.f;
        const float k0 = e0 * a.ddl[tof + cb + s] + e1 * a.debar[tof + cb + s] + e2 * (dmcv + a.de[tof + cb + s]) +
                         e3 * a.dsl1[tof + cb + s] + e4 * a.dsl2[tof + cb + s] + e5 * dt5;
        cA[k] = (e0 + e1) * inv;
        c2[k] = e2 * inv * invd[k];
        c3[k] = e3 * inv;
        c4[k] = e4 * inv;
        cst[k] = k0 * inv;
        cD[k] = ed * inv;
      }
    }
  }

  __syncthreads();  // the primal row in PR is no longer gathered: it keeps 1/denom from here on
#pragma unroll
  for (int k = 0; k < VF; ++k) PR[tid + k * NT] = invd[k];

  // ---- split tangent reduction: d_dts[s] = sum_splits sum_k 2^(t_k - dts[s]) dt_k ----
  if (has_splits) {
    float* Pl = sm;  // staging in the tour buffers: Pi_l, Pi_r, dPi_l, dPi_r
    float* Pr = sm + NTV;
    float* Ql = sm + 2 * NTV;
    float* Qr = sm + 3 * NTV;
    const float* dts_row = a.dts + (size_t)row * S;
    const float* dPi_d = a.dPi + (size_t)d * a.dstride;
    const float* dPb_d = a.dPibar + (size_t)d * a.dstride;
    for (long long i = i0; i < i1; ++i) {
      const long long l = a.sp.sl[i], rr = a.sp.sr[i];
      const float lsp = a.sp.lsp[i];
      __syncthreads();  // previous readers of the staging buffers (or of the scan) are done
#pragma unroll
      for (int k = 0; k < VF; ++k) {
        const int s = tid + k * NT;
        const bool real = s < S;
        Pl[s] = real ? a.Pi[(size_t)l * S + s] : neg_inf();
        Pr[s] = real ? a.Pi[(size_t)rr * S + s] : neg_inf();
        Ql[s] = real ? dPi_d[(size_t)l * S + s] : 0.f;
        Qr[s] = real ? dPi_d[(size_t)rr * S + s] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < VF; ++k) {
        const int s = tid + k * NT;
        const float dts = s < S ? __ldg(dts_row + s) : neg_inf();
        if (!is_neg_inf(dts)) {
          const unsigned ca = ccol[k] & 0xFFFFu, cbb = ccol[k] >> 16;
          const float ld = __ldg(a.log_pD + pb + s), ls = __ldg(a.log_pS + pb + s);
          const float dld = a.dpD[tof + pb + s], dls = a.dpS[tof + pb + s];
          const float pl = Pl[s], pr = Pr[s];
          const float t0 = lsp + ld + pl + pr;
          const float t1 = lsp + pl + a.Pibar[(size_t)rr * S + s];
          const float t2 = lsp + pr + a.Pibar[(size_t)l * S + s];
          const float t3 = lsp + ls + Pl[ca] + Pr[cbb];
          const float t4 = lsp + ls + Pr[ca] + Pl[cbb];
          const float dt0 = dld + Ql[s] + Qr[s];
          const float dt1 = Ql[s] + dPb_d[(size_t)rr * S + s];
          const float dt2 = Qr[s] + dPb_d[(size_t)l * S + s];
          const float dt3 = dls + Ql[ca] + Qr[cbb];
          const float dt4 = dls + Qr[ca] + Ql[cbb];
          cst[k] = fmaf(cD[k], ex2(t0 - dts) * dt0 + ex2(t1 - dts) * dt1 + ex2(t2 - dts) * dt2 +
                                   ex2(t3 - dts) * dt3 + ex2(t4 - dts) * dt4, cst[k]);
        }
      }
    }
  }

  // ---- fixed-count Jacobi steps from a zero tangent (the first one gives dPi = cst) ----
  float dp[VF], D[VF];
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    dp[k] = cst[k];
    D[k] = 0.f;
  }
  for (int it = 1; it < a.n_iters; ++it) {
    char* Tc = (it & 1) ? T0 : T1;
    float* Dc = (it & 1) ? DP0 : DP1;
    __syncthreads();  // previous step's (or the setup's) readers of Tc / Dc are done
    float ds = 0.f;
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const int s = tid + k * NT;
      const float v = r[k] * dp[k];
      sts_at(Tc, tr[k] & 0xFFFFu) = v;
      sts_at(Tc, tr[k] >> 16) = -v;
      Dc[s] = dp[k];
      ds += v;
    }
    __syncthreads();
    float g1[VF], g2[VF];
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      g1[k] = Dc[ccol[k] & 0xFFFFu];
      g2[k] = Dc[ccol[k] >> 16];
    }
    tour_scan_sw<VF>(reinterpret_cast<float*>(Tc), red, unused, ds);
    const float dRS = ds;
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      D[k] = dRS - (lds_at(Tc, tr[k] & 0xFFFFu) + r[k] * dp[k]);
      dp[k] = cA[k] * dp[k] + c2[k] * D[k] + c3[k] * g1[k] + c4[k] * g2[k] + cst[k];
    }
  }
  float* outp = a.dPi + (size_t)d * a.dstride + (size_t)row * S;
  float* outb = a.dPibar + (size_t)d * a.dstride + (size_t)row * S;
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    if (s < S) {
      outp[s] = dp[k];
      const float iv = PR[s];
      outb[s] = iv > 0.f ? D[k] * iv + a.dmc[tof + cb + s] : 0.f;
    }
  }
}

// Exclusive scan, in place, of a tour buffer of float2 entries (two tangent directions), in the
// swizzled pair layout (thread t scans the 2*VF consecutive entries of its chunk as VF float4
// groups XOR-permuted by t), fused with the block sums of sa and sb.  red >= 128 floats; the
// caller syncs before; two barriers inside, the second on exit.
template <int VF>
__device__ __forceinline__ void tour_scan_pair(float2* T, float* red, float& sa, float& sb) {
  constexpr int Q = VF;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5, nw = blockDim.x >> 5;
  const int sw = Q == 1 ? 0 : ((t / (8 / Q)) & (Q - 1));
  float4* base = reinterpret_cast<float4*>(T) + t * Q;
  float ga[Q], gb[Q];
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const float4 v = base[q ^ sw];
    ga[q] = v.x + v.z;
    gb[q] = v.y + v.w;
  }
  float la = 0.f, lb = 0.f;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    la += ga[q];
    lb += gb[q];
  }
  float ia = la, ib = lb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, ia, o);
    const float yb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ya;
      ib += yb;
    }
  }
  sa = warp_sum(sa);
  sb = warp_sum(sb);
  if (lane == 31) { red[wid] = ia; red[32 + wid] = ib; }
  if (lane == 0) { red[64 + wid] = sa; red[96 + wid] = sb; }
  __syncthreads();
  float ta = lane < nw ? red[lane] : 0.f;
  float tb2 = lane < nw ? red[32 + lane] : 0.f;
  const float bsa = lane < nw ? red[64 + lane] : 0.f;
  const float bsb = lane < nw ? red[96 + lane] : 0.f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, ta, o);
    const float yb = __shfl_up_sync(0xffffffffu, tb2, o);
    if (lane >= o) {
      ta += ya;
      tb2 += yb;
    }
  }
  sa = warp_sum(bsa);
  sb = warp_sum(bsb);
  const float pa = __shfl_up_sync(0xffffffffu, ta, 1);
  const float pb = __shfl_up_sync(0xffffffffu, tb2, 1);
  float ra = __shfl_sync(0xffffffffu, lane == 0 ? 0.f : pa, wid) + ia - la;
  float rb = __shfl_sync(0xffffffffu, lane == 0 ? 0.f : pb, wid) + ib - lb;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const float4 v = base[q ^ sw];
    base[q ^ sw] = make_float4(ra, rb, ra + v.x, rb + v.y);
    ra += ga[q];
    rb += gb[q];
  }
  __syncthreads();
}

__device__ __forceinline__ float2& pair_at(float2* base, unsigned off) {
  return *reinterpret_cast<float2*>(reinterpret_cast<char*>(base) + off);
}

// tour_scan_pair with one barrier, as tour_scan_sw_wx: T is only read, the within-warp exclusive
// prefixes of both sums go to X (same layout) before the barrier, and lane w returns in wa / wb the
// exclusive prefixes of warp w's totals; the slot at byte offset off then holds
//     pair_at(X, off) + (__shfl_sync(full, wa, off / (512 VF)), __shfl_sync(full, wb, ...))
// (2 VF float2 entries = 16 VF bytes per thread).  Block sums of sa and sb as tour_scan_pair.
template <int VF>
__device__ __forceinline__ void tour_scan_pair_wx(const float2* T, float2* X, float* red, float& sa, float& sb,
                                                  float& wa, float& wb) {
  constexpr int Q = VF;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5, nw = blockDim.x >> 5;
  const int sw = Q == 1 ? 0 : ((t / (8 / Q)) & (Q - 1));
  const float4* base = reinterpret_cast<const float4*>(T) + t * Q;
  float4* xb = reinterpret_cast<float4*>(X) + t * Q;
  float la = 0.f, lb = 0.f;  // the group sums are formed again below (no registers held across the scan)
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const float4 v = base[q ^ sw];
    la += v.x + v.z;
    lb += v.y + v.w;
  }
  float ia = la, ib = lb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, ia, o);
    const float yb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ya;
      ib += yb;
    }
  }
  float ra = ia - la, rb = ib - lb;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const float4 v = base[q ^ sw];
    xb[q ^ sw] = make_float4(ra, rb, ra + v.x, rb + v.y);
    ra += v.x + v.z;
    rb += v.y + v.w;
  }
  sa = warp_sum(sa);
  sb = warp_sum(sb);
  if (lane == 31) { red[wid] = ia; red[32 + wid] = ib; }
  if (lane == 0) { red[64 + wid] = sa; red[96 + wid] = sb; }
  __syncthreads();
  float ta = lane < nw ? red[lane] : 0.f;
  float tb2 = lane < nw ? red[32 + lane] : 0.f;
  const float bsa = lane < nw ? red[64 + lane] : 0.f;
  const float bsb = lane < nw ? red[96 + lane] : 0.f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, ta, o);
    const float yb = __shfl_up_sync(0xffffffffu, tb2, o);
    if (lane >= o) {
      ta += ya;
      tb2 += yb;
    }
  }
  sa = warp_sum(bsa);
  sb = warp_sum(bsb);
  const float pa = __shfl_up_sync(0xffffffffu, ta, 1);
  const float pb = __shfl_up_sync(0xffffffffu, tb2, 1);
  wa = lane == 0 ? 0.f : pa;
  wb = lane == 0 ? 0.f : pb;
}

// The slot prefix pair of tour_scan_pair_wx at byte offset off.
template <int VF>
__device__ __forceinline__ float2 tour_prefix_pair_wx(float2* X, unsigned off, float wa, float wb) {
  const int w = (int)(off / (512u * VF));
  const float2 p = pair_at(X, off);
  return make_float2(p.x + __shfl_sync(0xffffffffu, wa, w), p.y + __shfl_sync(0xffffffffu, wb, w));
}

// Tangent of one level for a PAIR of directions per CTA (blockIdx.y = pair index): the primal
// weights, the Euler-tour addressing and the split weights are shared by the two directions,
// which travel together as float2 through the tour scan and the gathers.  Same arithmetic as
// level_tangent_kernel.
template <int VF, bool DF>
__device__ __forceinline__ void tangent_pair_row(const TanArgs& a, long long row, long long i0, long long i1, int d0,
                                                 float* sm, BulkStage* bs = nullptr) {
  const unsigned* __restrict__ tb = a.tb;
  const unsigned* __restrict__ tp = a.tb2;
  const int S = a.S;
  const int NT = blockDim.x;
  const int NTV = NT * VF;
  float2* T0 = reinterpret_cast<float2*>(sm);
  float2* T1 = T0 + 2 * NTV;
  float2* DP0 = T1 + 2 * NTV;
  float2* DP1 = DP0 + NTV;
  float* PR = reinterpret_cast<float*>(DP1 + NTV);
  float* red = PR + NTV;
  const int tid = threadIdx.x;
  const long long item = a.item_idx[row];
  const size_t cb = (size_t)(item * a.crs);
  const size_t pb = (size_t)(item * a.prs);
  const size_t tofa = (size_t)d0 * a.tstride, tofb = tofa + (size_t)a.tstride;
  const bool has_splits = i1 > i0;
  const int leaf_raw = a.leaf_state[row];
  const int leaf = (!has_splits && leaf_raw >= 0 && leaf_raw < S) ? leaf_raw : -1;

  unsigned ccol[VF], tr[VF];
  float pv[VF], r[VF];
  float m = neg_inf();
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    ccol[k] = __ldg(tb + s);
    tr[k] = __ldg(tp + s);
    pv[k] = s < S ? a.Pi[(size_t)row * S + s] : neg_inf();
    PR[s] = pv[k];
    m = fmaxf(m, pv[k]);
  }
  const float row_max = block_max(m, red);
  const float rms = safe_max(row_max);
  float rsum = 0.f, zero = 0.f;
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    r[k] = ex2(pv[k] - rms);
    pair_at(T0, tr[k] & 0xFFFFu) = make_float2(r[k], 0.f);
    pair_at(T0, tr[k] >> 16) = make_float2(-r[k], 0.f);
    rsum += r[k];
  }
  __syncthreads();
  tour_scan_pair<VF>(T0, red, rsum, zero);
  const float row_sum = rsum;
  float cA[VF], c2[VF], c3[VF], c4[VF], ca_[VF], cb_[VF], cD[VF], invd[VF];
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    cA[k] = c2[k] = c3[k] = c4[k] = ca_[k] = cb_[k] = cD[k] = invd[k] = 0.f;
    if (s < S) {
      const float denom = row_sum - (pair_at(T0, tr[k] & 0xFFFFu).x + r[k]);
      const bool pos = denom > 0.f;
      const float sd = pos ? denom : 1.f;
      invd[k] = pos ? 1.0f / sd : 0.f;
      const float pibar = pos ? lg2(sd) + row_max + a.mc[cb + s] : neg_inf();
      const float t0 = a.dl[cb + s] + pv[k];
      const float t1 = pv[k] + a.ebar[cb + s];
      const float t2 = pibar + a.e[cb + s];
      const float t3 = a.sl1[cb + s] + PR[ccol[k] & 0xFFFFu];
      const float t4 = a.sl2[cb + s] + PR[ccol[k] >> 16];
      const bool hit = s == leaf;
      const float t5 = hit ? a.leaf_logp[(size_t)item * S + s] : neg_inf();
      const float dv = has_splits ? a.dts[(size_t)row * S + s] : neg_inf();
      const float mm = fmaxf(fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(t4, t5)), dv);
      const float ms = safe_max(mm);
      const float e0 = ex2(t0 - ms), e1 = ex2(t1 - ms), e2 = ex2(t2 - ms), e3 = ex2(t3 - ms), e4 = ex2(t4 - ms),
                  e5 = ex2(t5 - ms), ed = ex2(dv - ms);
      const float tot = ((e0 + e1) + (e2 + e3)) + ((e4 + e5) + ed);
      if (!is_neg_inf(lg2(tot) + mm)) {
        const float inv = tot > 0.f ? 1.0f / tot : 0.f;
        cA[k] = (e0 + e1) * inv;
        c2[k] = e2 * inv * invd[k];
        c3[k] = e3 * inv;
        c4[k] = e4 * inv;
        cD[k] = ed * inv;
        const size_t ia = tofa + cb + s, ib = tofb + cb + s;
        const float dta5 = hit ? a.dleaf[tofa + (size_t)item * S + s] : 0.f;
        const float dtb5 = hit ? a.dleaf[tofb + (size_t)item * S + s] : 0.f;
        const float dmca = pos ? a.dmc[ia] : 0.f, dmcb = pos ? a.dmc[ib] : 0.f;
        ca_[k] = inv * (e0 * a.ddl[ia] + e1 * a.debar[ia] + e2 * (dmca + a.de[ia]) + e3 * a.dsl1[ia] +
                        e4 * a.dsl2[ia] + e5 * dta5);
        cb_[k] = inv * (e0 * a.ddl[ib] + e1 * a.debar[ib] + e2 * (dmcb + a.de[ib]) + e3 * a.dsl1[ib] +
                        e4 * a.dsl2[ib] + e5 * dtb5);
      }
    }
  }
  __syncthreads();  // PR (primal row) no longer gathered: it keeps 1/denom from here on
  float* stash = reinterpret_cast<float*>(DP0);  // self-loop coefficients, parked during the splits
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    PR[s] = invd[k];
    stash[s] = cA[k];
    stash[NTV + s] = c2[k];
    stash[2 * NTV + s] = c3[k];
    stash[3 * NTV + s] = c4[k];
  }

  // ---- split tangent reduction, the weights shared by both directions ----
  if (has_splits) {
    float* Pl = sm;
    float* Pr = sm + NTV;
    float* Qla = sm + 2 * NTV;
    float* Qra = sm + 3 * NTV;
    float* Qlb = sm + 4 * NTV;
    float* Qrb = sm + 5 * NTV;
    const float* dPa = a.dPi + (size_t)d0 * a.dstride;
    const float* dPb = dPa + a.dstride;
    const float* dBa = a.dPibar + (size_t)d0 * a.dstride;
    const float* dBb = dBa + a.dstride;
    const float* dts_row = a.dts + (size_t)row * S;
    for (long long i = i0; i < i1; ++i) {
      const long long l = a.sp.sl[i], rr = a.sp.sr[i];
      const float lsp = a.sp.lsp[i];
      __syncthreads();
      const float *vPl = Pl, *vPr = Pr, *vQla = Qla, *vQra = Qra, *vQlb = Qlb, *vQrb = Qrb;
      if (bs) {
        // bulk copies of the six child rows (three arrivals on the split barrier); the tangent
        // rows are written by other CTAs of this launch, which a bulk copy reads through L2
        const size_t ol = (size_t)l * S, orr = (size_t)rr * S;
        const int RS = NTV + 4;
        float* b = sm;
        stage_rows_bulk(b, a.Pi + ol, b + RS, a.Pi + orr, S, NTV, bs->bar, &vPl, &vPr);
        stage_rows_bulk(b + 2 * RS, dPa + ol, b + 3 * RS, dPa + orr, S, NTV, bs->bar, &vQla, &vQra, 0.f);
        stage_rows_bulk(b + 4 * RS, dPb + ol, b + 5 * RS, dPb + orr, S, NTV, bs->bar, &vQlb, &vQrb, 0.f);
        bulk_wait(*bs, 0);
        bulk_fix_pad(vPl, S, NTV);
        bulk_fix_pad(vPr, S, NTV);
        bulk_fix_pad(vQla, S, NTV, 0.f);
        bulk_fix_pad(vQra, S, NTV, 0.f);
        bulk_fix_pad(vQlb, S, NTV, 0.f);
        bulk_fix_pad(vQrb, S, NTV, 0.f);
      } else {
#pragma unroll
        for (int k = 0; k < VF; ++k) {
          const int s = tid + k * NT;
          const bool real = s < S;
          const size_t ol = (size_t)l * S + s, orr = (size_t)rr * S + s;
          Pl[s] = real ? a.Pi[ol] : neg_inf();
          Pr[s] = real ? a.Pi[orr] : neg_inf();
          Qla[s] = real ? (DF ? __ldcg(dPa + ol) : dPa[ol]) : 0.f;  // DF: children written in this launch
          Qra[s] = real ? (DF ? __ldcg(dPa + orr) : dPa[orr]) : 0.f;
          Qlb[s] = real ? (DF ? __ldcg(dPb + ol) : dPb[ol]) : 0.f;
          Qrb[s] = real ? (DF ? __ldcg(dPb + orr) : dPb[orr]) : 0.f;
        }
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < VF; ++k) {
        const int s = tid + k * NT;
        const float dts = s < S ? __ldg(dts_row + s) : neg_inf();
        if (!is_neg_inf(dts)) {
          const unsigned ca = ccol[k] & 0xFFFFu, cbb = ccol[k] >> 16;
          const float ld = __ldg(a.log_pD + pb + s), ls = __ldg(a.log_pS + pb + s);
          const float pl = vPl[s], pr = vPr[s];
          const float w0 = ex2(lsp + ld + pl + pr - dts);
          const float w1 = ex2(lsp + pl + a.Pibar[(size_t)rr * S + s] - dts);
          const float w2 = ex2(lsp + pr + a.Pibar[(size_t)l * S + s] - dts);
          const float w3 = ex2(lsp + ls + vPl[ca] + vPr[cbb] - dts);
          const float w4 = ex2(lsp + ls + vPr[ca] + vPl[cbb] - dts);
          const size_t ol = (size_t)l * S + s, orr = (size_t)rr * S + s;
          const float bar_a = DF ? __ldcg(dBa + orr) : dBa[orr], bal_a = DF ? __ldcg(dBa + ol) : dBa[ol];
          const float bar_b = DF ? __ldcg(dBb + orr) : dBb[orr], bal_b = DF ? __ldcg(dBb + ol) : dBb[ol];
          const float xa = w0 * (a.dpD[tofa + pb + s] + vQla[s] + vQra[s]) + w1 * (vQla[s] + bar_a) +
                           w2 * (vQra[s] + bal_a) + w3 * (a.dpS[tofa + pb + s] + vQla[ca] + vQra[cbb]) +
                           w4 * (a.dpS[tofa + pb + s] + vQra[ca] + vQla[cbb]);
          const float xb = w0 * (a.dpD[tofb + pb + s] + vQlb[s] + vQrb[s]) + w1 * (vQlb[s] + bar_b) +
                           w2 * (vQrb[s] + bal_b) + w3 * (a.dpS[tofb + pb + s] + vQlb[ca] + vQrb[cbb]) +
                           w4 * (a.dpS[tofb + pb + s] + vQrb[ca] + vQlb[cbb]);
          ca_[k] = fmaf(cD[k], xa, ca_[k]);
          cb_[k] = fmaf(cD[k], xb, cb_[k]);
        }
      }
    }
  }

  // ---- fixed-count Jacobi steps from a zero tangent (the first one gives dPi = cst) ----
#pragma unroll
  for (int k = 0; k < VF; ++k) {  // own columns only: no barrier needed before the reload
    const int s = tid + k * NT;
    cA[k] = stash[s];
    c2[k] = stash[NTV + s];
    c3[k] = stash[2 * NTV + s];
    c4[k] = stash[3 * NTV + s];
  }
  float* outpa = a.dPi + (size_t)d0 * a.dstride + (size_t)row * S;
  float* outpb = outpa + a.dstride;
  float* outba = a.dPibar + (size_t)d0 * a.dstride + (size_t)row * S;
  float* outbb = outba + a.dstride;
  float dpa[VF], dpb[VF];
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    dpa[k] = ca_[k];
    dpb[k] = cb_[k];
  }
  const int last = a.n_iters - 1;
  if (last == 0) {  // one step: dPibar of the zero tangent
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const int s = tid + k * NT;
      if (s < S) {
        const float iv = PR[s];
        outba[s] = iv > 0.f ? a.dmc[tofa + cb + s] : 0.f;
        outbb[s] = iv > 0.f ? a.dmc[tofb + cb + s] : 0.f;
      }
    }
  }
  // Two barriers per step: the tour (T0) and the tangent row (DP0) are written, published, then
  // gathered and scanned, the scan leaving its prefixes in T1; the next step's stores come after
  // this step's scan barrier, which every reader of T0 and DP0 passed, and the prefixes' readers
  // pass the next step's publishing barrier before the next scan writes T1.  The barrier before
  // the first step ends the setup's and the splits' use of these buffers (DP0 held the parked
  // coefficients, read back by other threads' columns).
  __syncthreads();
  for (int it = 1; it <= last; ++it) {
    float2* Tc = T0;
    float2* Dc = DP0;
    float sa = 0.f, sbv = 0.f;
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const float va = r[k] * dpa[k], vb = r[k] * dpb[k];
      pair_at(Tc, tr[k] & 0xFFFFu) = make_float2(va, vb);
      pair_at(Tc, tr[k] >> 16) = make_float2(-va, -vb);
      Dc[tid + k * NT] = make_float2(dpa[k], dpb[k]);
      sa += va;
      sbv += vb;
    }
    __syncthreads();
    float pa[VF], pbv[VF];  // speciation terms, gathered before the scan
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const float2 g1 = Dc[ccol[k] & 0xFFFFu], g2 = Dc[ccol[k] >> 16];
      pa[k] = fmaf(c3[k], g1.x, c4[k] * g2.x);
      pbv[k] = fmaf(c3[k], g1.y, c4[k] * g2.y);
    }
    float wa, wb;
    tour_scan_pair_wx<VF>(Tc, T1, red, sa, sbv, wa, wb);
#pragma unroll
    for (int k = 0; k < VF; ++k) {
      const float2 p = tour_prefix_pair_wx<VF>(T1, tr[k] & 0xFFFFu, wa, wb);
      const float Da = sa - (p.x + r[k] * dpa[k]);
      const float Db = sbv - (p.y + r[k] * dpb[k]);
      dpa[k] = cA[k] * dpa[k] + c2[k] * Da + pa[k] + ca_[k];
      dpb[k] = cA[k] * dpb[k] + c2[k] * Db + pbv[k] + cb_[k];
      if (it == last) {
        const int s = tid + k * NT;
        if (s < S) {
          const float iv = PR[s];
          outba[s] = iv > 0.f ? Da * iv + a.dmc[tofa + cb + s] : 0.f;
          outbb[s] = iv > 0.f ? Db * iv + a.dmc[tofb + cb + s] : 0.f;
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < VF; ++k) {
    const int s = tid + k * NT;
    if (s < S) {
      outpa[s] = dpa[k];
      outpb[s] = dpb[k];
    }
  }
}

template <int VF>
__global__ void __launch_bounds__(512, 1) level_tangent2_kernel(TanArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int b = blockIdx.x;
  tangent_pair_row<VF, false>(a, a.sp.rows[b], a.sp.split_ptr[b], a.sp.split_ptr[b + 1], 2 * (int)blockIdx.y, sm);
}

// Dataflow tangent: items (direction pair, row); an item starts when the same pair's child rows
// are done.
template <int VF>
__global__ void __launch_bounds__(512, 1) flow_tangent2_kernel(TanArgs a, Flow f) {
  extern __shared__ __align__(16) float sm[];
  __shared__ FlowSlot fs;
  __shared__ __align__(8) unsigned long long bar;  // the split staging's bulk copies (3 arrivals)
  if (threadIdx.x == flow_poller()) fs.next = -1;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 3);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  BulkStage bs{&bar, 0u, f.error, f.max_polls};
  for (;;) {
    const int itm = flow_next_row(f, &fs);
    if (itm < 0) break;
    const int pair = itm / f.C, row = itm - pair * f.C;
    tangent_pair_row<VF, true>(a, row, f.row_split_ptr[row], f.row_split_ptr[row + 1], 2 * pair, sm, &bs);
    flow_finish_row(f, itm, &fs);
  }
}

// ------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------

// Exclusive scan, in place, of buf[0 .. blockDim.x*CH) float2 entries (two independent sums),
// thread t owning the consecutive entries [t*CH, (t+1)*CH); fused with the block sums of sa, sb
// (returned to every thread).  Returns the two totals in ta, tb.  red >= 128 floats.  The caller
// syncs before; two barriers inside, the second on exit.
template <int CH>
__device__ __forceinline__ void block_scan_pair_ch(float2* buf, float* red, float& sa, float& sb, float& ta,
                                                   float& tb) {
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5, nw = (blockDim.x + 31) >> 5;
  float2* base = buf + t * CH;
  float2 v[CH];
#pragma unroll
  for (int j = 0; j < CH; ++j) v[j] = base[j];
  float la = 0.f, lb = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    la += v[j].x;
    lb += v[j].y;
  }
  float ia = la, ib = lb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, ia, o);
    const float yb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ya;
      ib += yb;
    }
  }
  sa = warp_sum(sa);
  sb = warp_sum(sb);
  if (lane == 31) { red[wid] = ia; red[32 + wid] = ib; }
  if (lane == 0) { red[64 + wid] = sa; red[96 + wid] = sb; }
  __syncthreads();
  float xa = lane < nw ? red[lane] : 0.f;
  float xb = lane < nw ? red[32 + lane] : 0.f;
  const float bsa = lane < nw ? red[64 + lane] : 0.f;
  const float bsb = lane < nw ? red[96 + lane] : 0.f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, xa, o);
    const float yb = __shfl_up_sync(0xffffffffu, xb, o);
    if (lane >= o) {
      xa += ya;
      xb += yb;
    }
  }
  sa = warp_sum(bsa);
  sb = warp_sum(bsb);
  ta = __shfl_sync(0xffffffffu, xa, nw - 1);
  tb = __shfl_sync(0xffffffffu, xb, nw - 1);
  const float pa = __shfl_up_sync(0xffffffffu, xa, 1);
  const float pb = __shfl_up_sync(0xffffffffu, xb, 1);
  float ra = __shfl_sync(0xffffffffu, lane == 0 ? 0.f : pa, wid) + ia - la;
  float rb = __shfl_sync(0xffffffffu, lane == 0 ? 0.f : pb, wid) + ib - lb;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const float2 x = v[j];
    base[j] = make_float2(ra, rb);
    ra += x.x;
    rb += x.y;
  }
  __syncthreads();
}

struct BwdArgs {
  LevelConsts c;           // c.packed: padded [5, NTV] tables (invalid child/parent -> zero column NTV-1)
  SplitCSR sp;
  const float* Pi;
  const float* Pibar;
  const float* row_max;
  const float* dts_saved;  // [C,S] or null (recompute from the splits)
  float* acc;              // accumulated_rhs [C,S]
  float* v_out;            // [C,S] solved adjoint rows (active rows) or null
  double* slots;           // [gridDim.x, 8, NTV] fp64 per-CTA partial column sums (persist across levels)
  float threshold;
  int strict_gt;
  float side_thr;
  int side_thr_enabled;
  int neumann_terms;
  int n_rows;
  // Deterministic child adjoints (dataflow schedule; edge == null: atomic adds into acc).  Split i
  // (row-order index) writes its two children's contributions to edge rows 2i and 2i+1 (zeros when
  // its row is inactive); a row's adjoint is its seed acc[row] plus its incoming edge rows
  // in_edge[in_ptr[row] .. in_ptr[row+1]) (ascending edge ids), added left to right -- the same sum
  // in the same order whatever order the parents ran in.
  float* edge;                  // [2N, S]
  const long long* in_ptr;      // [C+1]
  const int* in_edge;           // [2N]
};

// accumulator rows of the per-CTA column sums
enum { G_PD = 0, G_PS, G_MT, G_E, G_EBAR, G_ES1, G_ES2, G_COL, G_N };
// the backward's shared fp32 rows 0..2 are G_PD, G_PS, G_MT (row 3 is G_COL)
static_assert(G_PD == 0 && G_PS == 1 && G_MT == 2, "shared column-sum rows");

#define KB_FLOW_FLUSH_ROWS 8
// Splits whose child rows are requested into L2 ahead of their turn (see bwd_prefetch_split).
#define KB_BWD_PREFETCH_SPLITS 4

// A hint (one thread): bring the row of n floats at p into L2 with one bulk prefetch.  The range
// is the row's 16-byte aligned cover rounded INWARD at the end (the start rounds down to at most
// 12 bytes before p, still inside the array, whose base is 16-byte aligned), so it never leaves
// the array; a prefetch changes no data, so the few floats it misses or adds do not matter.
__device__ __forceinline__ void l2_prefetch_row(const float* p, int n) {
  const unsigned long long a = (unsigned long long)(uintptr_t)p & ~15ull;
  const unsigned long long e = (unsigned long long)(uintptr_t)(p + n) & ~15ull;
  if (e > a)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"((unsigned)(e - a)) : "memory");
}

// The child rows split i of the backward reads: the children's Pi rows (staged), Pibar rows (read
// at the own columns) and adjoint rows (the targets of the split's atomic adds, when there are no
// edge rows).  A backward row's split phase otherwise meets each split's rows at the latency of HBM.
__device__ __forceinline__ void bwd_prefetch_split(const BwdArgs& a, long long i, int S) {
  const size_t l = (size_t)a.sp.sl[i] * S, r = (size_t)a.sp.sr[i] * S;
  l2_prefetch_row(a.Pi + l, S);
  l2_prefetch_row(a.Pi + r, S);
  l2_prefetch_row(a.Pibar + l, S);
  l2_prefetch_row(a.Pibar + r, S);
  if (a.edge == nullptr) {
    l2_prefetch_row(a.acc + l, S);
    l2_prefetch_row(a.acc + r, S);
  }
}

// A row's incoming edge rows travel to L2 ahead of its start (at most this many).
#define KB_BWD_PREFETCH_EDGES 16

// DF = the dataflow schedule (one persistent launch; f.par_ptr / par_idx then list each row's
// distinct CHILD rows, released when the row is done; a row is ready once all its parents ran).
template <int VPT, bool DF>
__global__ void __launch_bounds__(1024 / (VPT >= 8 ? 2 : 1), 1) level_backward_kernel(BwdArgs a, Flow f) {
  extern __shared__ float sm[];
  const LevelConsts& c = a.c;
  const int S = c.S;
  const int NT = blockDim.x;
  const int NTV = NT * VPT;
  // Column sums: G_PD, G_PS, G_MT and G_COL (updated per split) in fp32 shared rows ACC, moved
  // to the CTA's fp64 slot every few rows; G_E, G_EBAR, G_ES1, G_ES2 (once per row) straight to
  // the slot by fp64 reductions (each address is one thread's column: program order, so the
  // sums are deterministic).  KD / KS / KM hold log_pD, log_pS and mc when every row shares one
  // item row (the split phase reads them per column and split).
  // Shared memory, per phase of a row: the tour scan uses T and U[0, NTV) as one 2 NTV buffer;
  // the edge weights pass through SLb / SRb; the move to preorder positions uses T, U, U + NTV,
  // SLb and SRb; the Neumann sweep keeps the term in T and its prefix in U (U + NTV: the path
  // weights, read back by the column gradient); the splits stage child rows in SLb / SRb and
  // scan float2 pairs in U.
  float* P = sm;               // Pi row (log; -inf on padding), later speciation cotangents
  float* T = sm + NTV;         // tour (with U) / Neumann term / speciation cotangents
  float* U = sm + 2 * NTV;     // 2 NTV: tour, preorder prefix, float2 pairs in the split phase
  float2* U2 = reinterpret_cast<float2*>(U);
  float* ACC = sm + 4 * NTV;   // rows G_PD, G_PS, G_MT (0..2) and G_COL (3): fp32 column sums
  float* KD = ACC + 4 * NTV;   // log_pD, log_pS, mc of the shared item row
  float* KS = KD + NTV;
  float* KM = KS + NTV;
  float* SLb = KM + NTV;  // staged child Pi rows of the current split (NTV + 4 each)
  double* const slotd = a.slots + (size_t)blockIdx.x * G_N * NTV;
  const bool shared_consts = c.prs == 0 && c.crs == 0;
  float* SRb = SLb + NTV + 4;
  float* red = SRb + NTV + 4;
  unsigned cc[VPT], tr[VPT], pk[VPT], pa[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    cc[k] = c.packed[s];
    tr[k] = c.packed[NTV + s];
    pk[k] = c.packed[2 * NTV + s];
    pa[k] = c.packed[3 * NTV + s];
#pragma unroll
    for (int j = 0; j < 4; ++j) ACC[j * NTV + s] = 0.f;
    KD[s] = shared_consts && s < S ? c.log_pD[s] : 0.f;
    KS[s] = shared_consts && s < S ? c.log_pS[s] : 0.f;
    KM[s] = shared_consts && s < S ? c.mc[s] : 0.f;
  }
  __shared__ FlowSlot fs;
  if (threadIdx.x == flow_poller()) fs.next = -1;
  int b = blockIdx.x;
  int since_flush = 0;  // DF: rows accumulated in the fp32 shared sums since the last fp64 flush
  for (;;) {
    long long row, i0, i1;
    if (DF) {
      const int r = flow_next_row(f, &fs);
      if (r < 0) break;
      row = r;
      i0 = f.row_split_ptr[r];
      i1 = f.row_split_ptr[r + 1];
    } else {
      if (b >= a.n_rows) break;
      row = a.sp.rows[b];
      i0 = a.sp.split_ptr[b];
      i1 = a.sp.split_ptr[b + 1];
      b += gridDim.x;
    }
    const long long item = c.item_idx[row];
    const size_t cb = (size_t)(item * c.crs);
    const size_t pb = (size_t)(item * c.prs);
    const bool has_splits = i1 > i0;
    const int leaf_raw = c.leaf_state[row];
    const int leaf = (!has_splits && leaf_raw >= 0 && leaf_raw < S) ? leaf_raw : -1;

    // ---- active check ----
    float v[VPT];
    float amax = 0.f;
    const float* rrow = a.acc + (size_t)row * S;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      v[k] = s < S ? (DF ? __ldcg(rrow + s) : rrow[s]) : 0.f;  // DF: L2 (the atomic form's parents add there)
    }
    if (DF && a.edge) {  // the seed plus the incoming edge rows, left to right in edge order
      const int lane = threadIdx.x & 31;
      for (long long jb = a.in_ptr[row], je = a.in_ptr[row + 1]; jb < je; jb += 32) {
        const int nb = je - jb < 32 ? (int)(je - jb) : 32;
        const int mine = lane < nb ? __ldg(a.in_edge + jb + lane) : 0;  // a warp reads 32 ids at once
        int jj = 0;
        for (; jj + 4 <= nb; jj += 4) {  // four rows' loads in flight together
          float x[4][VPT];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float* er = a.edge + (size_t)__shfl_sync(0xffffffffu, mine, jj + u) * S;
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
              const int s = threadIdx.x + k * NT;
              x[u][k] = s < S ? __ldcg(er + s) : 0.f;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int k = 0; k < VPT; ++k) v[k] += x[u][k];
        }
        for (; jj < nb; ++jj) {
          const float* er = a.edge + (size_t)__shfl_sync(0xffffffffu, mine, jj) * S;
#pragma unroll
          for (int k = 0; k < VPT; ++k) {
            const int s = threadIdx.x + k * NT;
            if (s < S) v[k] += __ldcg(er + s);
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) amax = fmaxf(amax, fabsf(v[k]));
    // the block max compares above the threshold iff some thread's own max does: one barrier
    const bool active =
        __syncthreads_or(a.strict_gt ? (amax > a.threshold) : (amax >= a.threshold)) != 0;
    if (!active) {
      if (DF && a.edge) {  // the children add this row's edge rows whatever it did: zeros
        for (long long i = i0; i < i1; ++i) {
#pragma unroll
          for (int k = 0; k < VPT; ++k) {
            const int s = threadIdx.x + k * NT;
            if (s < S) {
              __stcg(a.edge + (size_t)(2 * i) * S + s, 0.f);
              __stcg(a.edge + (size_t)(2 * i + 1) * S + s, 0.f);
            }
          }
        }
      }
      if (DF) flow_finish_row(f, (int)row, &fs);
      continue;
    }
    // the first splits' child rows travel to L2 while the row's precompute and Neumann terms run
    if (has_splits && threadIdx.x == 0) {
      const long long pe = i1 < i0 + KB_BWD_PREFETCH_SPLITS ? i1 : i0 + KB_BWD_PREFETCH_SPLITS;
      for (long long i = i0; i < pe; ++i) bwd_prefetch_split(a, i, S);
    }

    // ---- dts row (log) ----
    float dv[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) dv[k] = neg_inf();
    if (has_splits) {
      if (a.dts_saved) {
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int s = threadIdx.x + k * NT;
          if (s < S) dv[k] = a.dts_saved[(size_t)row * S + s];
        }
      } else {
        dts_row2<VPT>(c, a.Pi, a.Pibar, a.sp, i0, i1, pb, cc, T, U, dv);
      }
    }

    // ---- precompute: p', path sums, self-loop coefficients ----
    const float* pirow = a.Pi + (size_t)row * S;
    const float* pbrow = a.Pibar + (size_t)row * S;
    const float rms = safe_max(a.row_max[row]);
    float pp[VPT];
    float psum = 0.f;
    if (has_splits && !a.dts_saved) __syncthreads();  // dts_row2's readers of T and U are done
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      const float pi = s < S ? pirow[s] : neg_inf();
      P[s] = pi;
      float w = pi;
      if (c.use_col && s < S) w += c.col[s];
      pp[k] = s < S ? ex2(w - rms) : 0.f;
      psum += pp[k];
    }
    // P and the tour buffer (T and U) are free: the previous row's readers finished before the
    // barriers of the queue and of the activity check
    float anc[VPT];
    const float row_sum = tour_pathsums_padded<VPT>(T, red, tr, pp, psum, anc);
    const float leafv = leaf >= 0 ? c.leaf_logp[(size_t)item * S + leaf] : neg_inf();
    float diag[VPT], coef[VPT];
    float a3v[VPT], a4v[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      diag[k] = coef[k] = a3v[k] = a4v[k] = 0.f;
      if (s < S) {
        const float pi = P[s];
        const float t0 = c.dl[cb + s] + pi;
        const float t1 = pi + c.ebar[cb + s];
        const float t2 = pbrow[s] + c.e[cb + s];
        const float t3 = c.sl1[cb + s] + P[lo16(cc[k])];
        const float t4 = c.sl2[cb + s] + P[hi16(cc[k])];
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
        const float denom = row_sum - anc[k];
        const float inv_denom = denom > 0.f ? 1.0f / denom : 0.f;
        diag[k] = wL * (e0 + e1) * inv_sum;
        coef[k] = wL * e2 * inv_sum * inv_denom;
        a3v[k] = wL * e3 * inv_sum;
        a4v[k] = wL * e4 * inv_sum;
      }
    }
    // the edge weights go through SLb / SRb (free until the split phase; no copy in flight),
    // so the tour scan's readers of T and U need no barrier here
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      SLb[s] = a3v[k];  // edge weight (speciation into child c1) of parent column s
      SRb[s] = a4v[k];  // ... into child c2
    }
    __syncthreads();
    float edge[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const unsigned par = lo16(pa[k]);
      edge[k] = hi16(pa[k]) ? SLb[par] : SRb[par];  // zero column for the root / padding
    }
    // ---- Neumann series over preorder positions ----
    // Thread t owns positions q = t*VPT + j, so the preorder prefix that gives every subtree sum
    // is a register scan with one barrier, and each term costs two barriers (scan, publish).
    // The five per-column vectors move to their positions q = pre(s) once, through T, U,
    // U + NTV, SLb and SRb (all free until the split phase); row 4 of the packed tables gives,
    // per position, the subtree end and the parent's position.
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const unsigned q = lo16(pk[k]);
      T[q] = v[k];
      U[q] = diag[k];
      U[NTV + q] = pp[k];
      SLb[q] = coef[k];
      SRb[q] = edge[k];
    }
    const int q0 = threadIdx.x * VPT;
    unsigned pq[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) pq[j] = __ldg(c.packed + 4 * NTV + q0 + j);
    __syncthreads();
    float tq[VPT], dq[VPT], cq[VPT], ppq[VPT], eq[VPT], vq[VPT];
    load_chunk<VPT>(tq, T + q0);
    load_chunk<VPT>(dq, U + q0);
    load_chunk<VPT>(ppq, U + NTV + q0);
    load_chunk<VPT>(cq, SLb + q0);
    load_chunk<VPT>(eq, SRb + q0);
#pragma unroll
    for (int j = 0; j < VPT; ++j) vq[j] = tq[j];
    // T: the current term by position, U: its exclusive prefix.  A term's gathers come before
    // the next term's scan barrier and its stores after it, so one buffer pair suffices.
    for (int n = 0; n < a.neumann_terms; ++n) {
      float x[VPT];
#pragma unroll
      for (int j = 0; j < VPT; ++j) x[j] = tq[j] * cq[j];
      const float A = reg_exclusive_scan<VPT>(x, red);
      store_chunk<VPT>(U + q0, x);
      store_chunk<VPT>(T + q0, tq);
      __syncthreads();
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const float sub = U[lo16(pq[j])] - x[j];
        const float nv = tq[j] * dq[j] + ppq[j] * (A - sub) + T[hi16(pq[j])] * eq[j];
        vq[j] += nv;
        tq[j] = nv;
      }
    }

    // ---- column gradient of the self-loop Pibar term; the solved row back to columns ----
    {
      float x[VPT];
#pragma unroll
      for (int j = 0; j < VPT; ++j) x[j] = vq[j] * cq[j];
      const float A = reg_exclusive_scan<VPT>(x, red);
      store_chunk<VPT>(U + q0, x);
      store_chunk<VPT>(T + q0, vq);
      __syncthreads();
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * NT;
        const unsigned q = lo16(pk[k]);
        v[k] = T[q];
        const float sub = U[hi16(pk[k])] - U[q];
        ACC[3 * NTV + s] += U[NTV + q] * (A - sub);
      }
    }
    if (a.v_out) {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * NT;
        if (s < S) a.v_out[(size_t)row * S + s] = v[k];
      }
    }

    // ---- parameter cotangents of the self-loop (terms recomputed) ----
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      if (s < S) {
        const float pi = P[s];
        const float t0 = c.dl[cb + s] + pi;
        const float t1 = pi + c.ebar[cb + s];
        const float t2 = pbrow[s] + c.e[cb + s];
        const float t3 = c.sl1[cb + s] + P[lo16(cc[k])];
        const float t4 = c.sl2[cb + s] + P[hi16(cc[k])];
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
        const float q0 = alpha * e0 * inv_sum, q1 = alpha * e1 * inv_sum, q2 = alpha * e2 * inv_sum;
        const float q3 = alpha * e3 * inv_sum, q4 = alpha * e4 * inv_sum, q5 = alpha * e5 * inv_sum;
        ACC[G_PD * NTV + s] += q0;
        ACC[G_PS * NTV + s] += q3 + q4 + q5;
        ACC[G_MT * NTV + s] += q2;
        atomicAdd(slotd + (size_t)G_E * NTV + s, (double)(q0 + q2));
        atomicAdd(slotd + (size_t)G_EBAR * NTV + s, (double)q1);
        atomicAdd(slotd + (size_t)G_ES1 * NTV + s, (double)q4);
        atomicAdd(slotd + (size_t)G_ES2 * NTV + s, (double)q3);
      }
    }

    // ---- splits: cotangents of the split reduction and the Pibar VJP trees ----
    // Per split: the split's Pi cotangents (5 terms) and Pibar cotangents of both children, then
    // both Pibar VJP trees at once (one scan of (left, right) pairs over the preorder numbering,
    // fused with the side-activity sums), and one atomic add per child element.  The next split's
    // child rows are fetched asynchronously while the current split's trees are scanned; the
    // children's Pibar values are loaded before the staging wait, and the children's column
    // weights for the trees come from the staged Pi rows (not re-read after the scan).
    if (has_splits) {
      float pip[VPT];
#pragma unroll
      for (int k = 0; k < VPT; ++k) pip[k] = P[threadIdx.x + k * NT];
      const float *cSL, *cSR;
      cSL = stage_row_cg(SLb, a.Pi + (size_t)a.sp.sl[i0] * S, S, NTV, true);
      cSR = stage_row_cg(SRb, a.Pi + (size_t)a.sp.sr[i0] * S, S, NTV, true);
      cp_async_commit();
      for (long long i = i0; i < i1; ++i) {
        const long long l = a.sp.sl[i], r = a.sp.sr[i];
        const float lsp = a.sp.lsp[i];
        const float* pbl = a.Pibar + (size_t)l * S;
        const float* pbr = a.Pibar + (size_t)r * S;
        const float rml = a.row_max[l], rmr = a.row_max[r];
        const float rmls = safe_max(rml), rmrs = safe_max(rmr);
        const size_t mcl = (size_t)(c.item_idx[l] * c.crs), mcr = (size_t)(c.item_idx[r] * c.crs);
        float bl[VPT], br[VPT];  // the children's Pibar at the own columns: issued before the wait
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int s = threadIdx.x + k * NT;
          bl[k] = s < S ? __ldcg(pbl + s) : neg_inf();
          br[k] = s < S ? __ldcg(pbr + s) : neg_inf();
        }
        cp_async_wait_all();
        __syncthreads();  // split i staged; the previous split's readers of P, T, U2 are done
        float cl[VPT], cr[VPT], wl[VPT], wr[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int s = threadIdx.x + k * NT;
          cl[k] = cr[k] = wl[k] = wr[k] = 0.f;
          float v3 = 0.f, v4 = 0.f, udl = 0.f, udr = 0.f;
          if (s < S) {
            const float pl = cSL[s], pr = cSR[s];
            {  // the children's column weights 2^(Pi + col - row max), used by the Pibar VJP trees
              const float cw = c.use_col ? c.col[s] : 0.f;
              wl[k] = ex2((c.use_col ? pl + cw : pl) - rmls);
              wr[k] = ex2((c.use_col ? pr + cw : pr) - rmrs);
            }
            const float ld = shared_consts ? KD[s] : c.log_pD[pb + s];
            const float ls = shared_consts ? KS[s] : c.log_pS[pb + s];
            const unsigned ca = lo16(cc[k]), cbb = hi16(cc[k]);
            const float d0 = ld + pl + pr;
            const float d1 = pl + br[k];
            const float d2 = pr + bl[k];
            const float d3 = ls + cSL[ca] + cSR[cbb];
            const float d4 = ls + cSR[ca] + cSL[cbb];
            const float ppar = pip[k];
            const bool pv = !is_neg_inf(ppar);
            const float vd0 = v[k] * (pv ? ex2(lsp + d0 - ppar) : 0.f);
            const float vd1 = v[k] * (pv ? ex2(lsp + d1 - ppar) : 0.f);
            const float vd2 = v[k] * (pv ? ex2(lsp + d2 - ppar) : 0.f);
            v3 = v[k] * (pv ? ex2(lsp + d3 - ppar) : 0.f);
            v4 = v[k] * (pv ? ex2(lsp + d4 - ppar) : 0.f);
            ACC[G_PD * NTV + s] += vd0;
            ACC[G_PS * NTV + s] += v3 + v4;
            ACC[G_MT * NTV + s] += vd1 + vd2;
            cl[k] = vd0 + vd1;
            cr[k] = vd0 + vd2;
            const float mcL = shared_consts ? KM[s] : c.mc[mcl + s];
            const float mcR = shared_consts ? KM[s] : c.mc[mcr + s];
            udl = is_neg_inf(bl[k]) ? 0.f : vd2 * ex2(rml + mcL - bl[k]);
            udr = is_neg_inf(br[k]) ? 0.f : vd1 * ex2(rmr + mcR - br[k]);
          }
          P[s] = v3;  // P no longer holds Pi (pip registers do)
          T[s] = v4;
          U2[lo16(pk[k])] = make_float2(udl, udr);
        }
        __syncthreads();  // P, T, U2 complete; the staged rows are no longer read
        if (i + 1 < i1) {
          cSL = stage_row_cg(SLb, a.Pi + (size_t)a.sp.sl[i + 1] * S, S, NTV, true);
          cSR = stage_row_cg(SRb, a.Pi + (size_t)a.sp.sr[i + 1] * S, S, NTV, true);
          cp_async_commit();
        }
        if (threadIdx.x == 0 && i + KB_BWD_PREFETCH_SPLITS < i1) bwd_prefetch_split(a, i + KB_BWD_PREFETCH_SPLITS, S);
        float sabs_l = 0.f, sabs_r = 0.f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {  // the scatter wrote each column's pair at pre(s)
          const float2 u = U2[lo16(pk[k])];
          sabs_l += fabsf(u.x);
          sabs_r += fabsf(u.y);
        }
        float Al, Ar;
        block_scan_pair_ch<VPT>(U2, red, sabs_l, sabs_r, Al, Ar);
        const bool side_l = !a.side_thr_enabled || sabs_l > a.side_thr;
        const bool side_r = !a.side_thr_enabled || sabs_r > a.side_thr;
        float* rl = a.acc + (size_t)l * S;
        float* rr = a.acc + (size_t)r * S;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int x = threadIdx.x + k * NT;
          if (x < S) {
            const unsigned par = lo16(pa[k]);
            const bool first = hi16(pa[k]) != 0;
            const float stl = first ? P[par] : T[par];
            const float str = first ? T[par] : P[par];
            const float2 ue = U2[hi16(pk[k])], ub = U2[lo16(pk[k])];
            const float tl = side_l ? wl[k] * (Al - (ue.x - ub.x)) : 0.f;
            const float trr = side_r ? wr[k] * (Ar - (ue.y - ub.y)) : 0.f;
            ACC[3 * NTV + x] += tl + trr;
            if (DF && a.edge) {
              __stcg(a.edge + (size_t)(2 * i) * S + x, cl[k] + stl + tl);
              __stcg(a.edge + (size_t)(2 * i + 1) * S + x, cr[k] + str + trr);
            } else {
              atomicAdd(rl + x, cl[k] + stl + tl);
              atomicAdd(rr + x, cr[k] + str + trr);
            }
          }
        }
      }
    }
    if (DF) {
      flow_finish_row(f, (int)row, &fs);
      // In a fixed start order the slot the poller just took names the CTA's next row: its own
      // rows travel to L2 while the CTA waits for it or flushes
      if (f.static_order && threadIdx.x == flow_poller() && fs.next >= 0 && fs.next < f.n_items) {
        const int nr = f.queue[fs.next];
        if (nr >= 0 && nr < f.C) {
          const size_t o = (size_t)nr * S;
          l2_prefetch_row(a.acc + o, S);
          l2_prefetch_row(a.Pi + o, S);
          l2_prefetch_row(a.Pibar + o, S);
          if (a.dts_saved) l2_prefetch_row(a.dts_saved + o, S);
          if (a.edge) {
            const long long j0 = a.in_ptr[nr], j1 = a.in_ptr[nr + 1];
            const long long je = j1 < j0 + KB_BWD_PREFETCH_EDGES ? j1 : j0 + KB_BWD_PREFETCH_EDGES;
            for (long long j = j0; j < je; ++j) l2_prefetch_row(a.edge + (size_t)a.in_edge[j] * S, S);
          }
        }
      }
      // A persistent CTA runs hundreds of rows: keep the fp32 partial sums short (as a level launch
      // does) by moving them into the fp64 slot every few rows.  Own columns only: no barrier.  With
      // the edge rows, after every row: which rows share a CTA varies run to run, so only a row's own
      // fp32 sums (formed in a fixed order) may be grouped before the fp64 slot.
      // The moves are fp64 reductions whose result nobody waits for (each address is this thread's
      // own column: program order, deterministic per CTA), not load-add-store round trips.
      if (++since_flush == (a.edge ? 1 : KB_FLOW_FLUSH_ROWS)) {
        since_flush = 0;
        double* slot = a.slots + (size_t)blockIdx.x * G_N * NTV;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          const int s = threadIdx.x + k * NT;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            atomicAdd(slot + (size_t)(j == 3 ? G_COL : j) * NTV + s, (double)ACC[j * NTV + s]);
            ACC[j * NTV + s] = 0.f;
          }
        }
      }
    }
  }
  // ---- flush this CTA's column sums into its fp64 slot ----
  double* slot = a.slots + (size_t)blockIdx.x * G_N * NTV;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
#pragma unroll
    for (int j = 0; j < 4; ++j) slot[(size_t)(j == 3 ? G_COL : j) * NTV + s] += (double)ACC[j * NTV + s];
  }
}

// Fixed-order sum of the per-CTA slots -> the eight fp32 cotangent vectors.  Block (x, j) covers
// 32 columns of accumulator row j: lane = column (coalesced reads), warp w sums its contiguous
// range of slots in order, then warp 0 adds the warps' partials in warp order -- the same
// association every run, however many slots there are.
#define KB_SLOT_WARPS 8
__global__ void __launch_bounds__(32 * KB_SLOT_WARPS) reduce_slots_kernel(const double* __restrict__ slots, int n_slots,
                                                                         int NTV, int S, float* out) {
  __shared__ double part[KB_SLOT_WARPS][32];
  const int j = blockIdx.y;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int s = blockIdx.x * 32 + lane;
  const int per = (n_slots + KB_SLOT_WARPS - 1) / KB_SLOT_WARPS;
  const int b0 = w * per, b1 = min(n_slots, b0 + per);
  double t = 0.0;
  if (s < S)
    for (int b = b0; b < b1; ++b) t += slots[((size_t)b * G_N + j) * NTV + s];
  part[w][lane] = t;
  __syncthreads();
  if (w == 0 && s < S) {
    double r = part[0][lane];
#pragma unroll
    for (int k = 1; k < KB_SLOT_WARPS; ++k) r += part[k][lane];
    out[(size_t)j * S + s] = (float)r;
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

// The forward tour kernel's per-column constants, interleaved and padded: out[g * ntv + s] =
// (2^dl + 2^ebar, 2^(mc+e), 2^sl1, 2^sl2) for s < S, zero for S <= s < ntv.
__global__ void lin_consts4_kernel(const float* dl, const float* ebar, const float* mc, const float* e,
                                   const float* sl1, const float* sl2, int G, int S, int ntv, float4* out) {
  const int n = G * ntv;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int g = i / ntv, s = i - g * ntv;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s < S) {
      const int j = g * S + s;
      v.x = ex2(dl[j]) + ex2(ebar[j]);
      v.y = ex2(mc[j] + e[j]);
      v.z = ex2(sl1[j]);
      v.w = ex2(sl2[j]);
    }
    out[i] = v;
  }
}

// Threads per CTA and columns per thread of the padded-row kernels; bd * vpt >= S + 1 leaves a
// zero padding column (mirrors kbench_b200/tree.py engine_width).
int engine_width(int S, int& bd) {
  bd = S > 1024 ? 1024 : ((S + 31) / 32) * 32;
  if (bd < 32) bd = 32;
  const int v0 = (S + bd - 1) / bd;
  int v = v0 <= 1 ? 1 : v0 <= 2 ? 2 : v0 <= 4 ? 4 : 8;
  if (bd * v < S + 1) v *= 2;
  return v;
}

// Threads and columns per thread of the backward kernel: the engine's padded width NTV with
// (where the row allows) KB_BWD_COLS columns per thread, so narrow rows leave room for several
// CTAs per SM.  The block stays a whole number of warps (its scans and reductions take one value
// from lane 31 of every warp) and at most 1024 threads: fewer columns per thread where NTV / 4
// is not a multiple of 32 (NTV = 608 for S = 599 runs 608 threads x 1 column), more where NTV
// exceeds 4096.
#ifndef KB_BWD_COLS
#define KB_BWD_COLS 4
#endif
int bwd_width(int S, int& bd) {
  int b0;
  const int ntv = engine_width(S, b0) * b0;
  int v = KB_BWD_COLS;
  while (v > 1 && (ntv % (32 * v) != 0 || ntv / v < 32)) v /= 2;
  while (ntv / v > 1024) v *= 2;
  bd = ntv / v;
  return v;
}

// Padded width, threads and columns per thread of the forward tour kernel (mirrors
// kbench_b200/tree.py tour_layout): NTV = smallest power of two > S (>= 64); 0 when NTV > 4096.
int tour_layout(int S, int& nt, int& vf) {
  int ntv = 64;
  while (ntv <= S) ntv <<= 1;
  if (ntv > 4096) return 0;
  vf = ntv / 32 < 8 ? ntv / 32 : 8;
  nt = ntv / vf;
  return ntv;
}

LevelConsts make_lc(const float* mc, const float* dl, const float* ebar, const float* e, const float* sl1,
                    const float* sl2, const float* leaf_logp, const float* linA, const float* linB,
                    const float* linC1, const float* linC2, const float* log_pD, const float* log_pS,
                    long long prs, long long crs, const float* col, int use_col, const int* parent, const int* c1,
                    const int* c2, const int* pre, const int* pre_end, const int* sub_start, const int* sub_end,
                    const int* jumps, int K, const long long* item_idx, const int* leaf_state,
                    const unsigned* packed, int S) {
  LevelConsts c;
  c.mc = mc; c.dl = dl; c.ebar = ebar; c.e = e; c.sl1 = sl1; c.sl2 = sl2; c.leaf_logp = leaf_logp;
  c.linA = linA; c.linB = linB; c.linC1 = linC1; c.linC2 = linC2; c.log_pD = log_pD; c.log_pS = log_pS;
  c.prs = prs; c.crs = crs; c.col = col; c.use_col = use_col; c.parent = parent; c.c1 = c1; c.c2 = c2;
  c.pre = pre; c.pre_end = pre_end; c.sub_start = sub_start; c.sub_end = sub_end; c.jumps = jumps; c.K = K;
  c.item_idx = item_idx; c.leaf_state = leaf_state; c.packed = packed; c.S = S;
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

extern "C" int kb_lin_consts_tour(const float* dl, const float* ebar, const float* mc, const float* e,
                                  const float* sl1, const float* sl2, int G, int S, float* out4, void* stream) {
  int nt, vf;
  const int ntv = tour_layout(S, nt, vf);
  if (G <= 0 || S <= 0 || out4 == nullptr) return KB_ERR_ARG;
  if (ntv == 0) return KB_ERR_SIZE;
  const int n = G * ntv;
  const int bd = 256;
  lin_consts4_kernel<<<(n + bd - 1) / bd, bd, 0, (cudaStream_t)stream>>>(dl, ebar, mc, e, sl1, sl2, G, S, ntv,
                                                                         reinterpret_cast<float4*>(out4));
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
                                const long long* item_idx, const int* leaf_state, const unsigned* packed,
                                const unsigned* tour_tables, const float* tour_consts, int force_log_space,
                                int pi_iters, int S, void* stream) {
  if (S <= 0 || n_rows < 0 || K < 0 || pi_iters < 2 || use_col_weights != 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (n_rows == 0) return KB_OK;
  FwdArgs a;
  a.c = make_lc(mc, dl, ebar, e, sl1, sl2, leaf_logp, linA, linB, linC1, linC2, log_pD, log_pS, param_row_stride,
                const_row_stride, col_log_probs, use_col_weights, node_parent, node_child1, node_child2,
                node_subtree_start, node_subtree_end, node_subtree_start, node_subtree_end, jumps, K, item_idx,
                leaf_state, packed, S);
  a.sp = SplitCSR{rows, split_ptr, sl, sr, lsp};
  a.Pi_src = Pi_src; a.Pibar_src = Pibar_src; a.pi = pi; a.pibar = pibar; a.row_max = pibar_row_max;
  a.dts_save = dts_save; a.residual = residual; a.fallback_count = fallback_count; a.n_rows = n_rows;
  a.force_log = force_log_space != 0;
  a.force_log_dev = nullptr;
  a.pi_iters = pi_iters;
  cudaStream_t st = (cudaStream_t)stream;
  int nt4, vf4;
  const int ntv4 = tour_layout(S, nt4, vf4);
  if (tour_tables != nullptr && ntv4 > 0) {
    // the log-space fallback re-reads the split reduction; the constants come interleaved
    if (dts_save == nullptr || tour_consts == nullptr) return KB_ERR_ARG;
    Fwd4Args a4;
    a4.f = a;
    a4.tb = tour_tables;
    a4.k4 = reinterpret_cast<const float4*>(tour_consts);
    a4.k4_rows = const_row_stride == 0 ? 0 : ntv4;
    const size_t smem4 = (size_t)(8 * (ntv4 + 4) + 96) * sizeof(float);
#define KB_LF4_CASE(V)                                                                                        \
  case V:                                                                                                     \
    if (smem4 > 48 * 1024 && cudaFuncSetAttribute((const void*)level_forward_tour_kernel<V>,                 \
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem4)) \
      return KB_ERR_LAUNCH;                                                                                   \
    level_forward_tour_kernel<V><<<n_rows, nt4, smem4, st>>>(a4);                                             \
    break;
    switch (vf4) {
      KB_LF4_CASE(2) KB_LF4_CASE(4) KB_LF4_CASE(8)
      default: return KB_ERR_SIZE;
    }
#undef KB_LF4_CASE
    return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
  }
  if (packed == nullptr) return KB_ERR_ARG;
  int bd;
  const int vpt = engine_width(S, bd);
  const size_t smem = (size_t)(6 * bd * vpt + 128) * sizeof(float);
#define KB_LF_CASE(V)                                                                                     \
  case V:                                                                                                 \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)level_forward_kernel<V>,                   \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) \
      return KB_ERR_LAUNCH;                                                                               \
    level_forward_kernel<V><<<n_rows, bd, smem, st>>>(a);                                                 \
    break;
  switch (vpt) {
    KB_LF_CASE(1) KB_LF_CASE(2) KB_LF_CASE(4) KB_LF_CASE(8)
    default: return KB_ERR_SIZE;
  }
#undef KB_LF_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_level_backward(const int* rows, const long long* split_ptr, int n_rows, const long long* sl,
                                 const long long* sr, const float* lsp, const float* Pi, const float* Pibar,
                                 const float* pibar_row_max, const float* dts_saved, float* accumulated_rhs,
                                 float* v_out, double* grad_slots, int n_slots, float threshold, int strict_gt,
                                 float side_threshold, int side_threshold_enabled, int neumann_terms,
                                 const float* mc, const float* dl, const float* ebar, const float* e,
                                 const float* sl1, const float* sl2, const float* leaf_logp, const float* log_pD,
                                 const float* log_pS, long long param_row_stride, long long const_row_stride,
                                 const float* col_log_probs, int use_col_weights, const long long* item_idx,
                                 const int* leaf_state, const unsigned* packed_padded, int S, void* stream) {
  if (S <= 0 || n_rows < 0 || neumann_terms < 0 || n_slots <= 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (n_rows == 0) return KB_OK;
  BwdArgs a{};  // value-initialised: the edge fields stay null unless set
  a.c = make_lc(mc, dl, ebar, e, sl1, sl2, leaf_logp, nullptr, nullptr, nullptr, nullptr, log_pD, log_pS,
                param_row_stride, const_row_stride, col_log_probs, use_col_weights, nullptr, nullptr, nullptr,
                nullptr, nullptr, nullptr, nullptr, nullptr, 0, item_idx, leaf_state, packed_padded, S);
  a.sp = SplitCSR{rows, split_ptr, sl, sr, lsp};
  a.Pi = Pi; a.Pibar = Pibar; a.row_max = pibar_row_max; a.dts_saved = dts_saved; a.acc = accumulated_rhs;
  a.v_out = v_out; a.slots = grad_slots; a.threshold = threshold; a.strict_gt = strict_gt;
  a.side_thr = side_threshold; a.side_thr_enabled = side_threshold_enabled; a.neumann_terms = neumann_terms;
  a.n_rows = n_rows;
  int bd;
  const int vpt = bwd_width(S, bd);
  const int ntv = bd * vpt;
  const size_t smem = (size_t)(11 * ntv + 2 * (ntv + 4) + 128) * sizeof(float);
  const int grid = n_rows < n_slots ? n_rows : n_slots;
  cudaStream_t st = (cudaStream_t)stream;
  const Flow nof{};
#define KB_LB_CASE(V)                                                                                      \
  case V:                                                                                                  \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)level_backward_kernel<V, false>,            \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))  \
      return KB_ERR_LAUNCH;                                                                                \
    level_backward_kernel<V, false><<<grid, bd, smem, st>>>(a, nof);                                       \
    break;
  switch (vpt) {
    KB_LB_CASE(1) KB_LB_CASE(2) KB_LB_CASE(4) KB_LB_CASE(8)
    default: return KB_ERR_SIZE;
  }
#undef KB_LB_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_reduce_grad_slots(const double* grad_slots, int n_slots, int S, float* out8, void* stream) {
  if (S <= 0 || n_slots <= 0) return KB_ERR_ARG;
  int bd;
  const int vpt = engine_width(S, bd);
  dim3 grid((S + 31) / 32, G_N);
  reduce_slots_kernel<<<grid, 32 * KB_SLOT_WARPS, 0, (cudaStream_t)stream>>>(grad_slots, n_slots, bd * vpt, S,
                                                                              out8);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_tour_layout(int S, int* ntv, int* threads, int* cols_per_thread) {
  if (S <= 0 || ntv == nullptr || threads == nullptr || cols_per_thread == nullptr) return KB_ERR_ARG;
  int nt = 0, vf = 0;
  const int n = tour_layout(S, nt, vf);
  *ntv = n;
  *threads = nt;
  *cols_per_thread = vf;
  return n > 0 ? KB_OK : KB_ERR_SIZE;
}

extern "C" int kb_backward_layout(int S, int* ntv, int* threads, int* cols_per_thread) {
  if (S <= 0 || ntv == nullptr || threads == nullptr || cols_per_thread == nullptr) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  int bd = 0;
  const int v = bwd_width(S, bd);
  *ntv = bd * v;
  *threads = bd;
  *cols_per_thread = v;
  return v <= 8 ? KB_OK : KB_ERR_SIZE;  // the kernels are built for 1, 2, 4 and 8 columns
}

extern "C" int kb_level_tangent(const int* rows, const long long* split_ptr, int n_rows, const long long* sl,
                                const long long* sr, const float* lsp, const float* Pi, const float* Pibar,
                                const float* dts_saved, float* dPi, float* dPibar, long long dir_stride, int D,
                                const float* mc, const float* dl, const float* ebar, const float* e, const float* sl1,
                                const float* sl2, const float* leaf_logp, const float* log_pD, const float* log_pS,
                                long long param_row_stride, long long const_row_stride, const float* dMC,
                                const float* dDL, const float* dEbar, const float* dE, const float* dSL1,
                                const float* dSL2, const float* dleaf, const float* dpD, const float* dpS,
                                long long tangent_dir_stride, const long long* item_idx, const int* leaf_state,
                                const unsigned* tour_tables, const unsigned* pair_tables, int n_iters, int S,
                                void* stream) {
  if (S <= 0 || n_rows < 0 || D <= 0 || n_iters < 1 || tour_tables == nullptr || dts_saved == nullptr)
    return KB_ERR_ARG;
  int nt, vf;
  const int ntv = tour_layout(S, nt, vf);
  if (ntv == 0) return KB_ERR_SIZE;
  if (n_rows == 0) return KB_OK;
  TanArgs a;
  a.sp = SplitCSR{rows, split_ptr, sl, sr, lsp};
  a.Pi = Pi; a.Pibar = Pibar; a.dts = dts_saved; a.dPi = dPi; a.dPibar = dPibar; a.dstride = dir_stride;
  a.mc = mc; a.dl = dl; a.ebar = ebar; a.e = e; a.sl1 = sl1; a.sl2 = sl2; a.leaf_logp = leaf_logp;
  a.log_pD = log_pD; a.log_pS = log_pS; a.crs = const_row_stride; a.prs = param_row_stride;
  a.dmc = dMC; a.ddl = dDL; a.debar = dEbar; a.de = dE; a.dsl1 = dSL1; a.dsl2 = dSL2; a.dleaf = dleaf;
  a.dpD = dpD; a.dpS = dpS; a.tstride = tangent_dir_stride; a.item_idx = item_idx; a.leaf_state = leaf_state;
  a.tb = tour_tables; a.tb2 = pair_tables; a.n_iters = n_iters; a.S = S;
  cudaStream_t st = (cudaStream_t)stream;
  int D1 = D;  // directions left for the one-direction kernel
  if (pair_tables != nullptr && D >= 2) {
    const size_t smem2 = (size_t)(13 * ntv + 128) * sizeof(float);
    dim3 grid2(n_rows, D / 2);
#define KB_LT2_CASE(V)                                                                                         \
  case V:                                                                                                      \
    if (smem2 > 48 * 1024 && cudaFuncSetAttribute((const void*)level_tangent2_kernel<V>,                      \
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2))   \
      return KB_ERR_LAUNCH;                                                                                    \
    level_tangent2_kernel<V><<<grid2, nt, smem2, st>>>(a);                                                     \
    break;
    switch (vf) {
      KB_LT2_CASE(2) KB_LT2_CASE(4) KB_LT2_CASE(8)
      default: return KB_ERR_SIZE;
    }
#undef KB_LT2_CASE
    if (cudaGetLastError() != cudaSuccess) return KB_ERR_LAUNCH;
    D1 = D % 2;
    if (D1 == 0) return KB_OK;
    // the odd last direction runs alone below
    const size_t od = (size_t)(D - 1) * dir_stride, ot = (size_t)(D - 1) * tangent_dir_stride;
    a.dPi += od; a.dPibar += od;
    a.dmc += ot; a.ddl += ot; a.debar += ot; a.de += ot; a.dsl1 += ot; a.dsl2 += ot; a.dleaf += ot;
    a.dpD += ot; a.dpS += ot;
  }
  const size_t smem = (size_t)(7 * ntv + 96) * sizeof(float);
  dim3 grid(n_rows, D1);
#define KB_LT_CASE(V)                                                                                          \
  case V:                                                                                                      \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)level_tangent_kernel<V>,                        \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))     \
      return KB_ERR_LAUNCH;                                                                                    \
    level_tangent_kernel<V><<<grid, nt, smem, st>>>(a);                                                        \
    break;
  switch (vf) {
    KB_LT_CASE(2) KB_LT_CASE(4) KB_LT_CASE(8)
    default: return KB_ERR_SIZE;
  }
#undef KB_LT_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_flow_forward(int C, const long long* row_split_ptr, const long long* sl, const long long* sr,
                               const float* lsp, const int* dep0, const int* ready0, int n_ready0,
                               const long long* par_ptr, const int* par_idx, int* queue, int* remaining,
                               unsigned* counters, long long max_polls, float* pi, float* pibar,
                               float* pibar_row_max, float* dts_save, float* residual, int* fallback_count,
                               const float* mc, const float* dl, const float* ebar, const float* e, const float* sl1,
                               const float* sl2, const float* leaf_logp, const float* log_pD, const float* log_pS,
                               long long param_row_stride, long long const_row_stride, const int* node_parent,
                               const int* node_child1, const int* node_child2, const int* node_subtree_start,
                               const int* node_subtree_end, const int* jumps, int K, const long long* item_idx,
                               const int* leaf_state, const unsigned* tour_tables, const float* tour_consts,
                               int force_log_space, const int* force_log_flag, const int* start_order, int pi_iters, int S,
                               void* stream) {
  if (S <= 0 || C < 0 || K < 0 || pi_iters < 2 || n_ready0 < 0 || n_ready0 > C || max_polls < 1) return KB_ERR_ARG;
  if (tour_tables == nullptr || tour_consts == nullptr || dts_save == nullptr || counters == nullptr) return KB_ERR_ARG;
  int nt, vf;
  const int ntv = tour_layout(S, nt, vf);
  if (ntv == 0) return KB_ERR_SIZE;
  if (C == 0) return KB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  FwdArgs a;
  a.c = make_lc(mc, dl, ebar, e, sl1, sl2, leaf_logp, nullptr, nullptr, nullptr, nullptr, log_pD, log_pS,
                param_row_stride, const_row_stride, nullptr, 0, node_parent, node_child1, node_child2,
                node_subtree_start, node_subtree_end, node_subtree_start, node_subtree_end, jumps, K, item_idx,
                leaf_state, nullptr, S);
  a.sp = SplitCSR{nullptr, nullptr, sl, sr, lsp};
  a.Pi_src = pi; a.Pibar_src = pibar; a.pi = pi; a.pibar = pibar; a.row_max = pibar_row_max;
  a.dts_save = dts_save; a.residual = residual; a.fallback_count = fallback_count; a.n_rows = C;
  a.force_log = force_log_space != 0;
  a.force_log_dev = force_log_flag;
  a.pi_iters = pi_iters;
  Fwd4Args a4;
  a4.f = a;
  a4.tb = tour_tables;
  a4.k4 = reinterpret_cast<const float4*>(tour_consts);
  a4.k4_rows = const_row_stride == 0 ? 0 : ntv;
  Flow f{queue, remaining, counters, counters + 1, reinterpret_cast<int*>(counters + 2), par_ptr, par_idx,
         row_split_ptr, C, max_polls, C};
  f.static_order = start_order != nullptr;
  if (start_order)  // every row queued in the given order from the start
    flow_init_kernel<<<(C + 255) / 256, 256, 0, st>>>(f, dep0, start_order, C);
  else
    flow_init_kernel<<<(C + 255) / 256, 256, 0, st>>>(f, dep0, ready0, n_ready0);
  if (cudaGetLastError() != cudaSuccess) return KB_ERR_LAUNCH;
  const size_t smem = (size_t)(8 * (ntv + 4) + 96) * sizeof(float);
  int dev = 0, n_sm = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return KB_ERR_LAUNCH;
#define KB_FF_CASE(V)                                                                                        \
  case V:                                                                                                    \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)flow_forward_kernel<V>,                       \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))   \
      return KB_ERR_LAUNCH;                                                                                  \
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, flow_forward_kernel<V>, nt, smem) !=          \
            cudaSuccess || per_sm < 1)                                                                       \
      return KB_ERR_LAUNCH;                                                                                  \
    {                                                                                                        \
      void* kargs[] = {(void*)&a4, (void*)&f};                                                               \
      if (cudaLaunchCooperativeKernel((const void*)flow_forward_kernel<V>,                                   \
                                      dim3(C < n_sm * per_sm ? C : n_sm * per_sm), dim3(nt), kargs, smem,   \
                                      st) != cudaSuccess)                                                    \
        return KB_ERR_LAUNCH;                                                                                \
    }                                                                                                        \
    break;
  switch (vf) {
    KB_FF_CASE(2) KB_FF_CASE(4) KB_FF_CASE(8)
    default: return KB_ERR_SIZE;
  }
#undef KB_FF_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_flow_backward(int C, const long long* row_split_ptr, const long long* sl, const long long* sr,
                                const float* lsp, const int* dep0, const int* ready0, int n_ready0,
                                const long long* child_ptr, const int* child_idx, int* queue, int* remaining,
                                unsigned* counters, long long max_polls, const float* Pi, const float* Pibar,
                                const float* pibar_row_max, const float* dts_saved, float* accumulated_rhs,
                                float* v_out, double* grad_slots, int n_slots, float threshold, int strict_gt,
                                float side_threshold, int side_threshold_enabled, int neumann_terms,
                                const float* mc, const float* dl, const float* ebar, const float* e,
                                const float* sl1, const float* sl2, const float* leaf_logp, const float* log_pD,
                                const float* log_pS, long long param_row_stride, long long const_row_stride,
                                const float* col_log_probs, int use_col_weights, const long long* item_idx,
                                const int* leaf_state, const unsigned* packed_padded, const int* start_order,
                                float* edge_rows, const long long* in_ptr, const int* in_edge, int S,
                                void* stream) {
  if (S <= 0 || C < 0 || neumann_terms < 0 || n_slots <= 0 || n_ready0 < 0 || n_ready0 > C || max_polls < 1 ||
      counters == nullptr)
    return KB_ERR_ARG;
  if (edge_rows && (!in_ptr || !in_edge)) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (C == 0) return KB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  BwdArgs a{};  // value-initialised: the edge fields stay null unless set
  a.c = make_lc(mc, dl, ebar, e, sl1, sl2, leaf_logp, nullptr, nullptr, nullptr, nullptr, log_pD, log_pS,
                param_row_stride, const_row_stride, col_log_probs, use_col_weights, nullptr, nullptr, nullptr,
                nullptr, nullptr, nullptr, nullptr, nullptr, 0, item_idx, leaf_state, packed_padded, S);
  a.sp = SplitCSR{nullptr, nullptr, sl, sr, lsp};
  a.Pi = Pi; a.Pibar = Pibar; a.row_max = pibar_row_max; a.dts_saved = dts_saved; a.acc = accumulated_rhs;
  a.v_out = v_out; a.slots = grad_slots; a.threshold = threshold; a.strict_gt = strict_gt;
  a.side_thr = side_threshold; a.side_thr_enabled = side_threshold_enabled; a.neumann_terms = neumann_terms;
  a.n_rows = C;
  a.edge = edge_rows; a.in_ptr = in_ptr; a.in_edge = in_edge;
  Flow f{queue, remaining, counters, counters + 1, reinterpret_cast<int*>(counters + 2), child_ptr, child_idx,
         row_split_ptr, C, max_polls, C};
  f.static_order = start_order != nullptr;
  if (start_order)  // every row queued in the given order from the start
    flow_init_kernel<<<(C + 255) / 256, 256, 0, st>>>(f, dep0, start_order, C);
  else
    flow_init_kernel<<<(C + 255) / 256, 256, 0, st>>>(f, dep0, ready0, n_ready0);
  if (cudaGetLastError() != cudaSuccess) return KB_ERR_LAUNCH;
  int bd;
  const int vpt = bwd_width(S, bd);
  const int ntv = bd * vpt;
  const size_t smem = (size_t)(11 * ntv + 2 * (ntv + 4) + 128) * sizeof(float);
  const int grid = C < n_slots ? C : n_slots;  // persistent CTAs, one fp64 slot each
#define KB_FB_CASE(V)                                                                                      \
  case V:                                                                                                  \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)level_backward_kernel<V, true>,             \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))  \
      return KB_ERR_LAUNCH;                                                                                \
    {                                                                                                      \
      void* kargs[] = {(void*)&a, (void*)&f};                                                              \
      if (cudaLaunchCooperativeKernel((const void*)level_backward_kernel<V, true>, dim3(grid), dim3(bd),  \
                                      kargs, smem, st) != cudaSuccess)                                     \
        return KB_ERR_LAUNCH;                                                                              \
    }                                                                                                      \
    break;
  switch (vpt) {
    KB_FB_CASE(1) KB_FB_CASE(2) KB_FB_CASE(4) KB_FB_CASE(8)
    default: return KB_ERR_SIZE;
  }
#undef KB_FB_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_flow_tangent(int C, const long long* row_split_ptr, const long long* sl, const long long* sr,
                               const float* lsp, const int* dep0, const int* ready0, int n_ready0,
                               const long long* par_ptr, const int* par_idx, int* queue, int* remaining,
                               unsigned* counters, long long max_polls, const float* Pi, const float* Pibar,
                               const float* dts_saved, float* dPi, float* dPibar, long long dir_stride, int D,
                               const float* mc, const float* dl, const float* ebar, const float* e, const float* sl1,
                               const float* sl2, const float* leaf_logp, const float* log_pD, const float* log_pS,
                               long long param_row_stride, long long const_row_stride, const float* dMC,
                               const float* dDL, const float* dEbar, const float* dE, const float* dSL1,
                               const float* dSL2, const float* dleaf, const float* dpD, const float* dpS,
                               long long tangent_dir_stride, const long long* item_idx, const int* leaf_state,
                               const unsigned* tour_tables, const unsigned* pair_tables, int n_iters, int S,
                               void* stream) {
  if (S <= 0 || C < 0 || D <= 0 || (D & 1) || n_iters < 1 || tour_tables == nullptr || pair_tables == nullptr ||
      dts_saved == nullptr || counters == nullptr || n_ready0 < 0 || n_ready0 > C || max_polls < 1)
    return KB_ERR_ARG;
  int nt, vf;
  const int ntv = tour_layout(S, nt, vf);
  if (ntv == 0) return KB_ERR_SIZE;
  if (C == 0) return KB_OK;
  if ((long long)C * (D / 2) > 0x7FFFFFFFLL) return KB_ERR_SIZE;
  TanArgs a;
  a.sp = SplitCSR{nullptr, nullptr, sl, sr, lsp};
  a.Pi = Pi; a.Pibar = Pibar; a.dts = dts_saved; a.dPi = dPi; a.dPibar = dPibar; a.dstride = dir_stride;
  a.mc = mc; a.dl = dl; a.ebar = ebar; a.e = e; a.sl1 = sl1; a.sl2 = sl2; a.leaf_logp = leaf_logp;
  a.log_pD = log_pD; a.log_pS = log_pS; a.crs = const_row_stride; a.prs = param_row_stride;
  a.dmc = dMC; a.ddl = dDL; a.debar = dEbar; a.de = dE; a.dsl1 = dSL1; a.dsl2 = dSL2; a.dleaf = dleaf;
  a.dpD = dpD; a.dpS = dpS; a.tstride = tangent_dir_stride; a.item_idx = item_idx; a.leaf_state = leaf_state;
  a.tb = tour_tables; a.tb2 = pair_tables; a.n_iters = n_iters; a.S = S;
  cudaStream_t st = (cudaStream_t)stream;
  const int n_items = C * (D / 2);
  Flow f{queue, remaining, counters, counters + 1, reinterpret_cast<int*>(counters + 2), par_ptr, par_idx,
         row_split_ptr, C, max_polls, n_items};
  flow_init_kernel<<<(n_items + 255) / 256 < 65535 ? (n_items + 255) / 256 : 65535, 256, 0, st>>>(f, dep0, ready0,
                                                                                                   n_ready0);
  if (cudaGetLastError() != cudaSuccess) return KB_ERR_LAUNCH;
  const size_t smem = (size_t)(13 * ntv + 128) * sizeof(float);
  int dev = 0, n_sm = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return KB_ERR_LAUNCH;
#define KB_FT_CASE(V)                                                                                        \
  case V:                                                                                                    \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)flow_tangent2_kernel<V>,                      \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))   \
      return KB_ERR_LAUNCH;                                                                                  \
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, flow_tangent2_kernel<V>, nt, smem) !=         \
            cudaSuccess || per_sm < 1)                                                                       \
      return KB_ERR_LAUNCH;                                                                                  \
    {                                                                                                        \
      void* kargs[] = {(void*)&a, (void*)&f};                                                                \
      if (cudaLaunchCooperativeKernel((const void*)flow_tangent2_kernel<V>,                                  \
                                      dim3(n_items < n_sm * per_sm ? n_items : n_sm * per_sm), dim3(nt),    \
                                      kargs, smem, st) != cudaSuccess)                                       \
        return KB_ERR_LAUNCH;                                                                                \
    }                                                                                                        \
    break;
  switch (vf) {
    KB_FT_CASE(2) KB_FT_CASE(4) KB_FT_CASE(8)
    default: return KB_ERR_SIZE;
  }
#undef KB_FT_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_forward_ctas(int S, int* n_ctas) {
  if (S <= 0 || n_ctas == nullptr) return KB_ERR_ARG;
  int nt, vf;
  const int ntv = tour_layout(S, nt, vf);
  if (ntv == 0) return KB_ERR_SIZE;
  const size_t smem = (size_t)(8 * (ntv + 4) + 96) * sizeof(float);
  int dev = 0, n_sm = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return KB_ERR_LAUNCH;
  const void* fn = vf == 2 ? (const void*)flow_forward_kernel<2>
                 : vf == 4 ? (const void*)flow_forward_kernel<4>
                           : (const void*)flow_forward_kernel<8>;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
    return KB_ERR_LAUNCH;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, nt, smem) != cudaSuccess || per_sm < 1)
    return KB_ERR_LAUNCH;
  *n_ctas = n_sm * per_sm;
  return KB_OK;
}

extern "C" int kb_backward_ctas(int S, int* n_ctas) {
  if (S <= 0 || S > KB_MAX_S || n_ctas == nullptr) return KB_ERR_ARG;
  int bd;
  const int vpt = bwd_width(S, bd);
  const int ntv = bd * vpt;
  const size_t smem = (size_t)(11 * ntv + 2 * (ntv + 4) + 128) * sizeof(float);
  int dev = 0, n_sm = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return KB_ERR_LAUNCH;
  const void* fn = vpt == 1 ? (const void*)level_backward_kernel<1, true>
                 : vpt == 2 ? (const void*)level_backward_kernel<2, true>
                 : vpt == 4 ? (const void*)level_backward_kernel<4, true>
                            : (const void*)level_backward_kernel<8, true>;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
    return KB_ERR_LAUNCH;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, bd, smem) != cudaSuccess || per_sm < 1)
    return KB_ERR_LAUNCH;
  *n_ctas = n_sm * per_sm;
  return KB_OK;
}
