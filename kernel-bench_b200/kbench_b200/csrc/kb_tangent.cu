// Forward-mode tangent (JVP) kernels of the solver: the tangent benchmark config.
//
// Restates the linearisations of the reference's tangent pass
//   kbench/core/kernels/e_step_tangent.py   _e_step_tangent_2d_kernel (:23-150),
//                                           e_tangent_fixed_point (:174-208)
//   kbench/core/kernels/dts_tangent.py      _dts_tangent_kernel (:23-96), compute_dts_tangent (:99-122)
//   kbench/core/kernels/wave_tangent.py     _wave_step_tangent_kernel (:34-183),
//                                           _wave_step_tangent_selfloop_kernel (:186-336)
// as driven by newton/forward_tangent.py:105-215 (jvp_root_scores, fixed-count fused self-loop).
//
// Every linearisation is taken at the frozen primal state, so per row (and per direction) the
// softmax weights, the ancestor sums of the primal row and the Pibar denominators are computed
// once and the iterations only carry the tangent row.  B200 design:
//  * E tangent: one persistent CTA per direction iterates on the device to the reference's
//    convergence rule (no per-iteration host sync);
//  * dts tangent: one CTA per parent row sums its splits in a fixed order (deterministic, no
//    atomics);
//  * wave self-loop tangent: one CTA per row, every iteration on chip;
//  * the fused level kernel runs, per dependency level, every (row, direction) pair of the level:
//    split tangent reduction + all self-loop iterations, on the Euler-tour tables of the forward.
#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

using namespace kb;

// ------------------------------------------------------------------------------------------
// E-step tangent
// ------------------------------------------------------------------------------------------

struct ETan {
  const float* E;    // [G,S] frozen fixed point
  const float* pS;   // [G,S]
  const float* pD;
  const float* pL;
  const float* mc;
  const float* col;  // [S]
  const float* dpS;  // [D,G,S] direction-major (stride dstride between directions)
  const float* dpD;
  const float* dpL;
  const float* dmc;
  long long dstride;
  const int* c1;
  const int* c2;
  const int* jumps;  // [K,S]
  int K;
  int S;
  int G;
  int use_col;
};

// One linearised E application on row g (direction d) from the tangent row dE (shared).
// Writes dE_new / dE_s1 / dE_s2 / dEbar rows (any may be null); returns max|dE_new - dE| and
// max|dE_new| through the references.
__device__ void e_tan_row(const ETan& q, int g, int d, const float* dE, float* X, float* Y, float* X2, float* Y2,
                          float* red, float* dE_new, float* o_s1, float* o_s2, float* o_bar, float& mdiff,
                          float& mabs) {
  const int S = q.S;
  const size_t base = (size_t)g * S;
  const size_t dbase = (size_t)d * q.dstride + base;
  float m = neg_inf();
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = q.E[base + s];
    if (q.use_col) w += q.col[s];
    m = fmaxf(m, w);
  }
  const float row_max = block_max(m, red);
  const float rms = safe_max(row_max);
  float sum = 0.f, dsum = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = q.E[base + s];
    if (q.use_col) w += q.col[s];
    const float r = ex2(w - rms);
    X[s] = r;
    X2[s] = r * dE[s];
    sum += r;
    dsum += r * dE[s];
  }
  const float row_sum = block_sum(sum, red);
  const float dRS = block_sum(dsum, red);
  const float* anc = ancestor_sum_doubling(X, Y, q.jumps, q.K, S);
  const float* dAS = ancestor_sum_doubling(X2, Y2, q.jumps, q.K, S);
  float md = 0.f, ma = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float e = q.E[base + s];
    const int a = q.c1[s], b = q.c2[s];
    const bool av = a >= 0 && a < S, bv = b >= 0 && b < S;
    const float es1 = av ? q.E[base + a] : neg_inf();
    const float es2 = bv ? q.E[base + b] : neg_inf();
    const float des1 = av ? dE[a] : 0.f;
    const float des2 = bv ? dE[b] : 0.f;
    const float denom = row_sum - anc[s];
    const bool pos = denom > 0.f;
    const float sd = pos ? denom : 1.f;
    const float ebar = pos ? lg2(sd) + row_max + q.mc[base + s] : neg_inf();
    const float debar = pos ? (dRS - dAS[s]) / sd + q.dmc[dbase + s] : 0.f;
    const float t0 = q.pS[base + s] + es1 + es2;
    const float t1 = q.pD[base + s] + 2.0f * e;
    const float t2 = e + ebar;
    const float t3 = q.pL[base + s];
    const float mm = fmaxf(fmaxf(t0, t1), fmaxf(t2, t3));
    const float ms = safe_max(mm);
    const float e0 = ex2(t0 - ms), e1 = ex2(t1 - ms), e2 = ex2(t2 - ms), e3 = ex2(t3 - ms);
    const float tot = e0 + e1 + e2 + e3;
    const float en = lg2(tot) + mm;
    const float inv = tot > 0.f ? 1.0f / tot : 0.f;
    const float dt0 = q.dpS[dbase + s] + des1 + des2;
    const float dt1 = q.dpD[dbase + s] + 2.0f * dE[s];
    const float dt2 = dE[s] + debar;
    const float dt3 = q.dpL[dbase + s];
    float dn = (e0 * inv) * dt0 + (e1 * inv) * dt1 + (e2 * inv) * dt2 + (e3 * inv) * dt3;
    if (is_neg_inf(en)) dn = 0.f;
    if (dE_new) dE_new[s] = dn;
    if (o_s1) o_s1[dbase + s] = des1;
    if (o_s2) o_s2[dbase + s] = des2;
    if (o_bar) o_bar[dbase + s] = debar;
    md = fmaxf(md, fabsf(dn - dE[s]));
    ma = fmaxf(ma, fabsf(dn));
  }
  mdiff = fmaxf(mdiff, block_max(md, red));
  mabs = fmaxf(mabs, block_max(ma, red));
}

// Richardson iteration of the E tangent for direction d = blockIdx.x; rows g = 0..G-1 share the
// convergence test (as the reference's max over item rows).  dE rows ping-pong between dE_out and
// scratch ([D,G,S] each); the converged dE is left in dE_out.
__global__ void e_tangent_fp_kernel(ETan q, const float* __restrict__ dE0, float* dE_out, float* scratch,
                                    float* dE_s1, float* dE_s2, float* dEbar, int max_iter, float tol,
                                    int* iters_out) {
  extern __shared__ float sm[];
  const int S = q.S, G = q.G;
  const int d = blockIdx.x;
  float* dEs = sm;
  float* nxt = sm + S;
  float* X = sm + 2 * S;
  float* Y = sm + 3 * S;
  float* X2 = sm + 4 * S;
  float* Y2 = sm + 5 * S;
  float* red = sm + 6 * S;
  const size_t dof = (size_t)d * q.dstride;
  float* bufs[2] = {dE_out + dof, scratch + dof};
  const float* cur = dE0 ? dE0 + dof : nullptr;  // null: the zero start
  int which = 0, it = 0;
  while (it < max_iter) {
    float* out = bufs[which];
    float mdiff = 0.f, mabs = 0.f;
    for (int g = 0; g < G; ++g) {
      __syncthreads();
      for (int s = threadIdx.x; s < S; s += blockDim.x) dEs[s] = cur ? cur[(size_t)g * S + s] : 0.f;
      __syncthreads();
      e_tan_row(q, g, d, dEs, X, Y, X2, Y2, red, nxt, nullptr, nullptr, nullptr, mdiff, mabs);
      __syncthreads();
      for (int s = threadIdx.x; s < S; s += blockDim.x) out[(size_t)g * S + s] = nxt[s];
    }
    __syncthreads();
    cur = out;
    which ^= 1;
    ++it;
    if (mdiff <= tol * fmaxf(1.0f, mabs)) break;
  }
  // final application at the last iterate for (dE_s1, dE_s2, dEbar); dE_out holds the iterate
  for (int g = 0; g < G; ++g) {
    __syncthreads();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      const float v = cur ? cur[(size_t)g * S + s] : 0.f;
      dEs[s] = v;
      dE_out[dof + (size_t)g * S + s] = v;
    }
    __syncthreads();
    float a = 0.f, b = 0.f;
    e_tan_row(q, g, d, dEs, X, Y, X2, Y2, red, nullptr, dE_s1, dE_s2, dEbar, a, b);
  }
  if (threadIdx.x == 0 && iters_out) iters_out[d] = it;
}

// One linearised application for every (row g, direction d): blockIdx.x = d * G + g.
__global__ void e_tangent_step_kernel(ETan q, const float* __restrict__ dE_in, float* dE_new, float* dE_s1,
                                      float* dE_s2, float* dEbar, float* max_diff) {
  extern __shared__ float sm[];
  const int S = q.S, G = q.G;
  const int d = blockIdx.x / G, g = blockIdx.x % G;
  float* dEs = sm;
  float* nxt = sm + S;
  float* X = sm + 2 * S;
  float* Y = sm + 3 * S;
  float* X2 = sm + 4 * S;
  float* Y2 = sm + 5 * S;
  float* red = sm + 6 * S;
  const size_t off = (size_t)d * q.dstride + (size_t)g * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x) dEs[s] = dE_in[off + s];
  __syncthreads();
  float mdiff = 0.f, mabs = 0.f;
  e_tan_row(q, g, d, dEs, X, Y, X2, Y2, red, nxt, dE_s1, dE_s2, dEbar, mdiff, mabs);
  __syncthreads();
  for (int s = threadIdx.x; s < S; s += blockDim.x) dE_new[off + s] = nxt[s];
  if (threadIdx.x == 0 && max_diff) max_diff[blockIdx.x] = mdiff;
}

// ------------------------------------------------------------------------------------------
// dts tangent (per parent row, splits in a fixed order)
// ------------------------------------------------------------------------------------------

struct DtsTan {
  const float* Pi;
  const float* Pibar;
  const float* dPi;
  const float* dPibar;
  const long long* sl;       // split children rows
  const long long* sr;
  const float* lsp;          // [N] or null
  const long long* order;    // splits sorted by parent (stable)
  const long long* ptr;      // [W+1] CSR into order
  const int* c1;
  const int* c2;
  const float* log_pD;       // item rows: item * prs + s
  const float* log_pS;
  const float* dlog_pD;
  const float* dlog_pS;
  long long prs;
  const long long* item_idx;
  long long item_offset;
  const float* dts_r;        // [W,S]
  float* out;                // [W,S]
  int S;
};

__global__ void dts_tangent_kernel(DtsTan a) {
  const int S = a.S;
  const int p = blockIdx.y;
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= S) return;
  const long long item = a.item_idx[a.item_offset + p];
  const size_t pb = (size_t)(item * a.prs);
  const float dts = a.dts_r[(size_t)p * S + s];
  float acc = 0.f;
  if (!is_neg_inf(dts)) {
    const float ld = a.log_pD[pb + s], ls = a.log_pS[pb + s];
    const float dld = a.dlog_pD[pb + s], dls = a.dlog_pS[pb + s];
    const int ca = a.c1[s], cb = a.c2[s];
    const bool av = ca >= 0 && ca < S, bv = cb >= 0 && cb < S;
    for (long long j = a.ptr[p]; j < a.ptr[p + 1]; ++j) {
      const long long n = a.order[j];
      const size_t bl = (size_t)a.sl[n] * S, br = (size_t)a.sr[n] * S;
      const float lsp = a.lsp ? a.lsp[n] : 0.f;
      const float pil = a.Pi[bl + s], pir = a.Pi[br + s];
      const float dpl = a.dPi[bl + s], dpr = a.dPi[br + s];
      const float plc1 = av ? a.Pi[bl + ca] : neg_inf(), prc2 = bv ? a.Pi[br + cb] : neg_inf();
      const float prc1 = av ? a.Pi[br + ca] : neg_inf(), plc2 = bv ? a.Pi[bl + cb] : neg_inf();
      const float dplc1 = av ? a.dPi[bl + ca] : 0.f, dprc2 = bv ? a.dPi[br + cb] : 0.f;
      const float dprc1 = av ? a.dPi[br + ca] : 0.f, dplc2 = bv ? a.dPi[bl + cb] : 0.f;
      const float t0 = lsp + ld + pil + pir;
      const float t1 = lsp + pil + a.Pibar[br + s];
      const float t2 = lsp + pir + a.Pibar[bl + s];
      const float t3 = lsp + ls + plc1 + prc2;
      const float t4 = lsp + ls + prc1 + plc2;
      const float dt0 = dld + dpl + dpr;
      const float dt1 = dpl + a.dPibar[br + s];
      const float dt2 = dpr + a.dPibar[bl + s];
      const float dt3 = dls + dplc1 + dprc2;
      const float dt4 = dls + dprc1 + dplc2;
      acc += ex2(t0 - dts) * dt0 + ex2(t1 - dts) * dt1 + ex2(t2 - dts) * dt2 + ex2(t3 - dts) * dt3 +
             ex2(t4 - dts) * dt4;
    }
  }
  a.out[(size_t)p * S + s] = acc;
}

// ------------------------------------------------------------------------------------------
// wave self-loop tangent (drop-in driver: one CTA per row of a wave)
// ------------------------------------------------------------------------------------------

struct WaveTan {
  const float* Pi;       // primal rows (read at pi_ws + w)
  const float* dPi_in;   // tangent rows (read at pi_ws + w)
  float* dPi_out;        // written at out row w (already offset to the wave)
  float* dPibar_out;     // [C,S] written at ws + w, or null
  long long ws, pi_ws;
  const float* mc;       // primal constants: item * crs + s
  const float* dl;
  const float* ebar;
  const float* e;
  const float* sl1;
  const float* sl2;
  const float* dmc;      // tangent constants, same layout
  const float* ddl;
  const float* debar;
  const float* de;
  const float* dsl1;
  const float* dsl2;
  long long crs;
  const float* col;
  int use_col;
  const int* c1;
  const int* c2;
  const int* jumps;
  int K;
  const int* leaf_state;     // [C] or null (no leaf term)
  const float* leaf_logp;    // item * S + s
  const float* dleaf_logp;
  const long long* item_idx;
  const float* dts;          // [W,S] or null
  const float* ddts;         // [W,S] or null
  int n_iters;
  int S;
};

template <int VPT>
__global__ void __launch_bounds__(1024) wave_tangent_kernel(WaveTan a) {
  extern __shared__ float sm[];
  const int S = a.S;
  const int NT = blockDim.x;
  float* P = sm;            // primal row (log)
  float* DP0 = sm + S;      // tangent row (two buffers)
  float* DP1 = sm + 2 * S;
  float* X = sm + 3 * S;
  float* Y = sm + 4 * S;
  float* red = sm + 5 * S;
  const int w = blockIdx.x;
  const long long prow = a.pi_ws + w;
  const long long item = a.item_idx[a.ws + w];
  const size_t cb = (size_t)(item * a.crs);
  const float* pi_g = a.Pi + (size_t)prow * S;
  const float* dpi_g = a.dPi_in + (size_t)prow * S;
  float r[VPT];
  float m = neg_inf();
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    if (s < S) {
      const float pv = pi_g[s];
      P[s] = pv;
      DP0[s] = dpi_g[s];
      float wv = pv;
      if (a.use_col) wv += a.col[s];
      m = fmaxf(m, wv);
    }
  }
  const float row_max = block_max(m, red);
  const float rms = safe_max(row_max);
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    r[k] = 0.f;
    if (s < S) {
      float wv = P[s];
      if (a.use_col) wv += a.col[s];
      r[k] = ex2(wv - rms);
      X[s] = r[k];
    }
    sum += r[k];
  }
  const float row_sum = block_sum(sum, red);
  const float* anc = ancestor_sum_doubling(X, Y, a.jumps, a.K, S);
  const int leaf = a.leaf_state ? a.leaf_state[a.ws + w] : -1;
  // frozen coefficients: dpi_new = cA dpi + c2 (dRS - dAS) + c3 dpi[c1] + c4 dpi[c2] + cst
  float cA[VPT], c2[VPT], c3[VPT], c4[VPT], cst[VPT], invd[VPT];
  bool posv[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    cA[k] = c2[k] = c3[k] = c4[k] = cst[k] = invd[k] = 0.f;
    posv[k] = false;
    if (s < S) {
      const float pv = P[s];
      const float denom = row_sum - anc[s];
      const bool pos = denom > 0.f;
      const float sd = pos ? denom : 1.f;
      posv[k] = pos;
      invd[k] = pos ? 1.0f / sd : 0.f;
      const float pibar = pos ? lg2(sd) + row_max + a.mc[cb + s] : neg_inf();
      const int ca = a.c1[s], cbb = a.c2[s];
      const bool av = ca >= 0 && ca < S, bv = cbb >= 0 && cbb < S;
      const float t0 = a.dl[cb + s] + pv;
      const float t1 = pv + a.ebar[cb + s];
      const float t2 = pibar + a.e[cb + s];
      const float t3 = av ? a.sl1[cb + s] + P[ca] : neg_inf();
      const float t4 = bv ? a.sl2[cb + s] + P[cbb] : neg_inf();
      const bool hit = (s == leaf);
      const float t5 = hit ? a.leaf_logp[(size_t)item * S + s] : neg_inf();
      float mm = fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(t4, t5));
      const float dv = a.dts ? a.dts[(size_t)w * S + s] : neg_inf();
      mm = fmaxf(mm, dv);
      const float ms = safe_max(mm);
      const float e0 = ex2(t0 - ms), e1 = ex2(t1 - ms), e2 = ex2(t2 - ms), e3 = ex2(t3 - ms), e4 = ex2(t4 - ms),
                  e5 = ex2(t5 - ms), ed = ex2(dv - ms);
      const float tot = ((e0 + e1) + (e2 + e3)) + ((e4 + e5) + ed);
      const float res = lg2(tot) + mm;
      if (!is_neg_inf(res)) {
        const float inv = tot > 0.f ? 1.0f / tot : 0.f;
        const float dt5 = hit ? a.dleaf_logp[(size_t)item * S + s] : 0.f;
        const float dmc = pos ? a.dmc[cb + s] : 0.f;
        float k0 = e0 * a.ddl[cb + s] + e1 * a.debar[cb + s] + e2 * (dmc + a.de[cb + s]) +
                   e3 * a.dsl1[cb + s] + e4 * a.dsl2[cb + s] + e5 * dt5;
        if (a.ddts) k0 += ed * a.ddts[(size_t)w * S + s];
        cA[k] = (e0 + e1) * inv;
        c2[k] = e2 * inv * invd[k];
        c3[k] = e3 * inv;
        c4[k] = e4 * inv;
        cst[k] = k0 * inv;
      }
    }
  }
  float dp[VPT], D[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    dp[k] = s < S ? DP0[s] : 0.f;
    D[k] = 0.f;
  }
  const int n_it = a.n_iters < 1 ? 1 : a.n_iters;
  for (int it = 0; it < n_it; ++it) {
    float* Dc = (it & 1) ? DP1 : DP0;  // holds dp (current)
    float* Dn = (it & 1) ? DP0 : DP1;
    float ds = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      const float v = r[k] * dp[k];
      if (s < S) X[s] = v;
      ds += v;
    }
    const float dRS = block_sum(ds, red);  // syncs: X and Dc complete
    const float* dAS = ancestor_sum_doubling(X, Y, a.jumps, a.K, S);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * NT;
      if (s < S) {
        const int ca = a.c1[s], cbb = a.c2[s];
        const float g1 = (ca >= 0 && ca < S) ? Dc[ca] : 0.f;
        const float g2 = (cbb >= 0 && cbb < S) ? Dc[cbb] : 0.f;
        D[k] = dRS - dAS[s];
        dp[k] = cA[k] * dp[k] + c2[k] * D[k] + c3[k] * g1 + c4[k] * g2 + cst[k];
        Dn[s] = dp[k];
      }
    }
  }
  float* out = a.dPi_out + (size_t)w * S;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * NT;
    if (s < S) {
      out[s] = dp[k];
      if (a.dPibar_out)
        a.dPibar_out[(size_t)(a.ws + w) * S + s] = posv[k] ? D[k] * invd[k] + a.dmc[cb + s] : 0.f;
    }
  }
}

int wave_threads(int S, int& vpt) {
  int bd = S > 1024 ? 1024 : ((S + 31) / 32) * 32;
  if (bd < 32) bd = 32;
  const int v = (S + bd - 1) / bd;
  vpt = v <= 1 ? 1 : v <= 2 ? 2 : v <= 4 ? 4 : 8;
  return bd;
}

}  // namespace

extern "C" int kb_e_tangent_fixed_point(const float* E_star, const float* dlog_pS, const float* dlog_pD,
                                        const float* dlog_pL, const float* dmax_coupling, const float* log_pS,
                                        const float* log_pD, const float* log_pL, const float* max_coupling,
                                        const float* col_log_probs, int use_col_weights, const int* node_child1,
                                        const int* node_child2, const int* jumps, int K, int G, int S, int D,
                                        int max_iter, float tol, const float* dE0, float* dE_out, float* scratch,
                                        float* dE_s1, float* dE_s2, float* dEbar, int* iters_out, void* stream) {
  if (S <= 0 || G <= 0 || D <= 0 || K < 0 || max_iter < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  ETan q{E_star, log_pS, log_pD, log_pL, max_coupling, col_log_probs, dlog_pS, dlog_pD, dlog_pL, dmax_coupling,
         (long long)G * S, node_child1, node_child2, jumps, K, S, G, use_col_weights};
  const size_t smem = (size_t)(6 * S + 96) * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute((const void*)e_tangent_fp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
    return KB_ERR_LAUNCH;
  e_tangent_fp_kernel<<<D, 1024, smem, (cudaStream_t)stream>>>(q, dE0, dE_out, scratch, dE_s1, dE_s2, dEbar,
                                                                max_iter, tol, iters_out);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_e_tangent_step(const float* E_star, const float* dE_in, const float* dlog_pS,
                                 const float* dlog_pD, const float* dlog_pL, const float* dmax_coupling,
                                 const float* log_pS, const float* log_pD, const float* log_pL,
                                 const float* max_coupling, const float* col_log_probs, int use_col_weights,
                                 const int* node_child1, const int* node_child2, const int* jumps, int K, int G,
                                 int S, int D, float* dE_new, float* dE_s1, float* dE_s2, float* dEbar,
                                 float* max_diff, void* stream) {
  if (S <= 0 || G <= 0 || D <= 0 || K < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  ETan q{E_star, log_pS, log_pD, log_pL, max_coupling, col_log_probs, dlog_pS, dlog_pD, dlog_pL, dmax_coupling,
         (long long)G * S, node_child1, node_child2, jumps, K, S, G, use_col_weights};
  const size_t smem = (size_t)(6 * S + 96) * sizeof(float);
  if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)e_tangent_step_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
    return KB_ERR_LAUNCH;
  e_tangent_step_kernel<<<D * G, 1024, smem, (cudaStream_t)stream>>>(q, dE_in, dE_new, dE_s1, dE_s2, dEbar,
                                                                      max_diff);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_dts_tangent(const float* Pi, const float* Pibar, const float* dPi, const float* dPibar,
                              const long long* sl, const long long* sr, const float* log_split_probs,
                              const long long* order, const long long* ptr, int W, const int* node_child1,
                              const int* node_child2, const float* log_pD, const float* log_pS,
                              const float* dlog_pD, const float* dlog_pS, long long param_row_stride,
                              const long long* item_idx, long long item_offset, const float* dts_r, float* out,
                              int S, void* stream) {
  if (S <= 0 || W < 0) return KB_ERR_ARG;
  if (W == 0) return KB_OK;
  DtsTan a{Pi, Pibar, dPi, dPibar, sl, sr, log_split_probs, order, ptr, node_child1, node_child2, log_pD, log_pS,
           dlog_pD, dlog_pS, param_row_stride, item_idx, item_offset, dts_r, out, S};
  const int bd = 256;
  dim3 grid((S + bd - 1) / bd, W);
  dts_tangent_kernel<<<grid, bd, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_wave_tangent(const float* Pi_in, const float* dPi_in, float* dPi_out, float* dPibar_out,
                               long long ws, long long pi_ws, int W, int S, int n_iters, const float* max_coupling,
                               const float* dMC, const float* DL, const float* dDL, const float* Ebar,
                               const float* dEbar, const float* E, const float* dE, const float* SL1,
                               const float* dSL1, const float* SL2, const float* dSL2, long long const_row_stride,
                               const float* col_log_probs, int use_col_weights, const int* node_child1,
                               const int* node_child2, const int* jumps, int K, const int* leaf_state_idx,
                               const float* leaf_logp, const float* dleaf_logp, const long long* item_idx,
                               const float* dts_reduced, const float* d_dts, void* stream) {
  if (S <= 0 || W < 0 || K < 0 || n_iters < 1) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (W == 0) return KB_OK;
  if ((dts_reduced == nullptr) != (d_dts == nullptr)) return KB_ERR_ARG;
  WaveTan a{Pi_in, dPi_in, dPi_out, dPibar_out, ws, pi_ws, max_coupling, DL, Ebar, E, SL1, SL2, dMC, dDL, dEbar, dE,
            dSL1, dSL2, const_row_stride, col_log_probs, use_col_weights, node_child1, node_child2, jumps, K,
            leaf_state_idx, leaf_logp, dleaf_logp, item_idx, dts_reduced, d_dts, n_iters, S};
  int vpt;
  const int bd = wave_threads(S, vpt);
  const size_t smem = (size_t)(5 * S + 96) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
#define KB_WT_CASE(V)                                                                                          \
  case V:                                                                                                      \
    if (smem > 48 * 1024 && cudaFuncSetAttribute((const void*)wave_tangent_kernel<V>,                         \
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))     \
      return KB_ERR_LAUNCH;                                                                                    \
    wave_tangent_kernel<V><<<W, bd, smem, st>>>(a);                                                            \
    break;
  switch (vpt) {
    KB_WT_CASE(1) KB_WT_CASE(2) KB_WT_CASE(4) KB_WT_CASE(8)
    default: return KB_ERR_SIZE;
  }
#undef KB_WT_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
