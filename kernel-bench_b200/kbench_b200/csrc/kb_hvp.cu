// Second-order contractions of the analytic exact-Hessian HVP (forward over reverse).
//
// Restates kbench/core/kernels/wave_so.py:37-250 (_wave_so_kernel),
// kbench/core/kernels/dts_so.py:24-230 (_dts_split_so_kernel, _dts_tree_so_kernel) and
// kbench/core/kernels/e_step_so.py:23-185 (_e_step_so_prepare/finalize_kernel): the tangent, along
// the primal tangent (dPi, dPibar, d-constants), of the backward's J^T applications and parameter
// cotangents at a FIXED adjoint.  Every output is invariant to the saved row maxima, which stay
// frozen (no tangent), as in the reference.
//
// B200 design: one CTA per row (wave rows, split sides, E rows) with the row and its path-sum
// buffers in shared memory; the reference's atomic ancestor walks become pointer-doubling path
// sums (ancestor-or-self) and bottom-up subtree sums over the compact levels, and the scatter of
// a column's contribution to its species children becomes a gather from the parent (no atomics
// inside a row).  Cross-row sums (child adjoint rows, parameter cotangents) use atomics as the
// reference does.
#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

using namespace kb;

constexpr float kLn2 = 0.6931471805599453f;

int so_block(int S) {
  int b = ((S + 31) / 32) * 32;
  return b > 1024 ? 1024 : (b < 32 ? 32 : b);
}

int so_smem(const void* fn, size_t bytes) {
  if (bytes > 48 * 1024 &&
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return KB_ERR_LAUNCH;
  return KB_OK;
}

// The value a column receives from its species parent's speciation term: vs1[par] when it is
// the parent's first child, vs2[par] when the second.
__device__ __forceinline__ float from_parent(const int* parent, const int* c1, const int* c2, const float* vs1,
                                             const float* vs2, int s, int S) {
  const int par = parent[s];
  float x = 0.f;
  if (par >= 0 && par < S) {
    if (c1[par] == s) x += vs1[par];
    if (c2[par] == s) x += vs2[par];
  }
  return x;
}

// ------------------------------------------------------------------------------------------------
// wave_so: per wave row w (global row ws + w)
// ------------------------------------------------------------------------------------------------

struct WaveSoArgs {
  const float *Pi, *dPi, *Pibar, *dPibar, *v;
  long long ws;
  int S;
  const float* row_max;
  const float *mc, *DL, *dDL, *Ebar, *dEbar, *E, *dE, *SL1, *dSL1, *SL2, *dSL2;
  long long crs;
  const float* col;
  int use_col;
  const int *parent, *c1, *c2, *jumps;
  int K;
  const long long* lv_ptr;
  int n_levels;
  const int *lv_par, *lv_c1, *lv_c2;
  const int* leaf_state;  // null: no leaf term
  const float *leaf_logp, *dleaf_logp;
  const long long* item_idx;
  const float *dts_r, *d_dts;  // [W,S] or null (rows without splits)
  const float* d_rhs;          // [C,S] folded into the output rows, or null
  float* d_out;                // [W,S]
  float* d_aw;                 // [6,W,S]: aw0, aw1, aw2, aw345, aw3, aw4
  long long aw_stride;         // W*S
};

__device__ __forceinline__ float p_of(const WaveSoArgs& a, float pi, int s, float rms) {
  float w = pi;
  if (a.use_col) w += a.col[s];
  return ex2(w - rms);
}

__global__ void __launch_bounds__(1024, 1) wave_so_kernel(WaveSoArgs a) {
  extern __shared__ float sm[];
  const int S = a.S;
  float* X = sm;
  float* Y = sm + S;
  float* X2 = sm + 2 * S;
  float* Y2 = sm + 3 * S;
  float* VS1 = sm + 4 * S;
  float* VS2 = sm + 5 * S;
  float* red = sm + 6 * S;
  const int w = blockIdx.x;
  const long long row = a.ws + w;
  const size_t pb = (size_t)row * S;
  const size_t ob = (size_t)w * S;
  const long long item = a.item_idx[row];
  const size_t cb = (size_t)(item * a.crs);
  const float rms = safe_max(a.row_max[row]);
  // p' = 2^(Pi - rowmax) (row max frozen) and its tangent; row sums; ancestor-or-self path sums
  float ps = 0.f, dps = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float p = p_of(a, a.Pi[pb + s], s, rms);
    const float dp = kLn2 * p * a.dPi[pb + s];
    X[s] = p;
    X2[s] = dp;
    ps += p;
    dps += dp;
  }
  const float row_sum = block_sum(ps, red);
  const float drow_sum = block_sum(dps, red);
  const float* anc = ancestor_sum_doubling(X, Y, a.jumps, a.K, S);
  const float* danc = ancestor_sum_doubling(X2, Y2, a.jumps, a.K, S);
  float* U = (anc == X) ? Y : X;      // the buffers the path sums do not occupy
  float* DU = (danc == X2) ? Y2 : X2;
  const int leaf = a.leaf_state ? a.leaf_state[row] : -1;
  float tu = 0.f, tdu = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float pi = a.Pi[pb + s], dpi = a.dPi[pb + s];
    const float pib = a.Pibar[pb + s], dpib = a.dPibar[pb + s];
    const float v = a.v[ob + s];
    const float denom = row_sum - anc[s];
    const float inv_denom = denom > 0.f ? 1.0f / denom : 0.f;
    const float ddenom = drow_sum - danc[s];
    const int k1 = a.c1[s], k2 = a.c2[s];
    const bool v1 = k1 >= 0 && k1 < S, v2 = k2 >= 0 && k2 < S;
    const float pi_s1 = v1 ? a.Pi[pb + k1] : neg_inf();
    const float pi_s2 = v2 ? a.Pi[pb + k2] : neg_inf();
    const float dpi_s1 = v1 ? a.dPi[pb + k1] : 0.f;
    const float dpi_s2 = v2 ? a.dPi[pb + k2] : 0.f;
    const float t0 = a.DL[cb + s] + pi, t1 = pi + a.Ebar[cb + s], t2 = pib + a.E[cb + s];
    const float t3 = a.SL1[cb + s] + pi_s1, t4 = a.SL2[cb + s] + pi_s2;
    const float dt0 = a.dDL[cb + s] + dpi, dt1 = dpi + a.dEbar[cb + s], dt2 = dpib + a.dE[cb + s];
    const float dt3 = a.dSL1[cb + s] + dpi_s1, dt4 = a.dSL2[cb + s] + dpi_s2;
    const bool hit = leaf == s;
    const float t5 = hit ? a.leaf_logp[(size_t)item * S + s] : neg_inf();
    const float dt5 = hit ? a.dleaf_logp[(size_t)item * S + s] : 0.f;
    const float m = fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(t4, t5));
    const float ms = safe_max(m);
    const float e0 = ex2(t0 - ms), e1 = ex2(t1 - ms), e2 = ex2(t2 - ms), e3 = ex2(t3 - ms), e4 = ex2(t4 - ms),
                e5 = ex2(t5 - ms);
    const float lsum = e0 + e1 + e2 + e3 + e4 + e5;
    const float inv_sum = lsum > 0.f ? 1.0f / lsum : 0.f;
    const float w0 = e0 * inv_sum, w1 = e1 * inv_sum, w2 = e2 * inv_sum, w3 = e3 * inv_sum, w4 = e4 * inv_sum,
                w5 = e5 * inv_sum;
    const float dlse = w0 * dt0 + w1 * dt1 + w2 * dt2 + w3 * dt3 + w4 * dt4 + w5 * dt5;
    const float dw0 = kLn2 * w0 * (dt0 - dlse), dw1 = kLn2 * w1 * (dt1 - dlse), dw2 = kLn2 * w2 * (dt2 - dlse);
    const float dw3 = kLn2 * w3 * (dt3 - dlse), dw4 = kLn2 * w4 * (dt4 - dlse), dw5 = kLn2 * w5 * (dt5 - dlse);
    float wL = 1.f, dwL = 0.f;
    if (a.dts_r) {
      const float dr = a.dts_r[ob + s];
      const float dts_l = lsum > 0.f ? lg2(lsum) + m : neg_inf();
      const float pm = fmaxf(dts_l, dr);
      const float pms = safe_max(pm);
      const float pnew = lg2(ex2(dts_l - pms) + ex2(dr - pms)) + pm;
      wL = is_neg_inf(dts_l) ? 0.f : ex2(dts_l - pnew);
      dwL = (!is_neg_inf(dr) && !is_neg_inf(dts_l)) ? kLn2 * wL * (1.0f - wL) * (dlse - a.d_dts[ob + s]) : 0.f;
    }
    const float da0 = v * (dwL * w0 + wL * dw0), da1 = v * (dwL * w1 + wL * dw1), da2 = v * (dwL * w2 + wL * dw2);
    const float da3 = v * (dwL * w3 + wL * dw3), da4 = v * (dwL * w4 + wL * dw4), da5 = v * (dwL * w5 + wL * dw5);
    a.d_aw[ob + s] = da0;
    a.d_aw[a.aw_stride + ob + s] = da1;
    a.d_aw[2 * a.aw_stride + ob + s] = da2;
    a.d_aw[3 * a.aw_stride + ob + s] = da3 + da4 + da5;
    a.d_aw[4 * a.aw_stride + ob + s] = da3;
    a.d_aw[5 * a.aw_stride + ob + s] = da4;
    const float coeff = wL * w2 * inv_denom;
    const float dcoeff = (dwL * w2 + wL * dw2) * inv_denom - coeff * inv_denom * ddenom;
    const float u = v * coeff, du = v * dcoeff;
    U[s] = u;
    DU[s] = du;
    tu += u;
    tdu += du;
    a.d_out[ob + s] = v * (dwL * (w0 + w1) + wL * (dw0 + dw1));
    VS1[s] = v * (dwL * w3 + wL * dw3);
    VS2[s] = v * (dwL * w4 + wL * dw4);
  }
  const float A = block_sum(tu, red);
  const float dA = block_sum(tdu, red);
  subtree_sums_levels(U, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
  subtree_sums_levels(DU, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float p = p_of(a, a.Pi[pb + s], s, rms);
    const float dp = kLn2 * p * a.dPi[pb + s];
    float val = a.d_out[ob + s] + dp * (A - U[s]) + p * (dA - DU[s]);
    if (a.d_rhs) val += a.d_rhs[pb + s];
    val += from_parent(a.parent, a.c1, a.c2, VS1, VS2, s, S);
    a.d_out[ob + s] = val;
  }
}

// ------------------------------------------------------------------------------------------------
// dts_so: split kernel (one CTA per split) and tree kernel (one CTA per split side)
// ------------------------------------------------------------------------------------------------

struct DtsSoArgs {
  const float *Pi, *dPi, *Pibar, *dPibar, *v;
  long long ws;
  const long long *sl, *sr, *red;
  const float* lsp;  // null: zeros
  int N;
  long long item_offset;
  const long long* item_idx;
  const float *pD, *pS, *dpD, *dpS;
  long long prs;
  const float *mt, *dmt;
  long long mrs;
  const float* row_max;
  const float* col;
  int use_col;
  const int *c1, *c2;
  const long long* lv_ptr;
  int n_levels;
  const int *lv_par, *lv_c1, *lv_c2;
  float *ud, *dud;  // [2N,S] staging: rows [0,N) left sides, [N,2N) right sides
  float *d_rhs, *g_pD, *g_pS, *g_mt, *g_col;
  int S;
};

__global__ void dts_so_split_kernel(DtsSoArgs a) {
  const int n = blockIdx.x;
  const int S = a.S;
  const long long w = a.red[n];
  const long long item = a.item_idx[a.item_offset + w];
  const long long l = a.sl[n], r = a.sr[n];
  const size_t bl = (size_t)l * S, br = (size_t)r * S, bp = (size_t)(a.ws + w) * S;
  const size_t prow = (size_t)(item * a.prs), mrow = (size_t)(item * a.mrs), grow = (size_t)item * S;
  const float lsp = a.lsp ? a.lsp[n] : 0.f;
  const float rm_l = a.row_max[l], rm_r = a.row_max[r];
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float pil = a.Pi[bl + s], pir = a.Pi[br + s], dpl = a.dPi[bl + s], dpr = a.dPi[br + s];
    const float pbl = a.Pibar[bl + s], pbr = a.Pibar[br + s], dbl = a.dPibar[bl + s], dbr = a.dPibar[br + s];
    const float pip = a.Pi[bp + s], dpip = a.dPi[bp + s];
    const float v = a.v[(size_t)w * S + s];
    const float ld = a.pD[prow + s], ls = a.pS[prow + s], dld = a.dpD[prow + s], dls = a.dpS[prow + s];
    const float mt = a.mt[mrow + s], dmt = a.dmt[mrow + s];
    const int k1 = a.c1[s], k2 = a.c2[s];
    const bool v1 = k1 >= 0 && k1 < S, v2 = k2 >= 0 && k2 < S;
    const float pl1 = v1 ? a.Pi[bl + k1] : neg_inf(), pr2 = v2 ? a.Pi[br + k2] : neg_inf();
    const float pr1 = v1 ? a.Pi[br + k1] : neg_inf(), pl2 = v2 ? a.Pi[bl + k2] : neg_inf();
    const float dpl1 = v1 ? a.dPi[bl + k1] : 0.f, dpr2 = v2 ? a.dPi[br + k2] : 0.f;
    const float dpr1 = v1 ? a.dPi[br + k1] : 0.f, dpl2 = v2 ? a.dPi[bl + k2] : 0.f;
    const float d0 = lsp + ld + pil + pir, d1 = lsp + pil + pbr, d2 = lsp + pir + pbl;
    const float d3 = lsp + ls + pl1 + pr2, d4 = lsp + ls + pr1 + pl2;
    const float dd0 = dld + dpl + dpr, dd1 = dpl + dbr, dd2 = dpr + dbl;
    const float dd3 = dls + dpl1 + dpr2, dd4 = dls + dpr1 + dpl2;
    const bool fin = !is_neg_inf(pip);
    const float w0 = fin ? ex2(d0 - pip) : 0.f, w1 = fin ? ex2(d1 - pip) : 0.f, w2 = fin ? ex2(d2 - pip) : 0.f;
    const float w3 = fin ? ex2(d3 - pip) : 0.f, w4 = fin ? ex2(d4 - pip) : 0.f;
    const float vd1 = v * w1, vd2 = v * w2;
    const float dvd0 = v * kLn2 * w0 * (dd0 - dpip), dvd1 = v * kLn2 * w1 * (dd1 - dpip);
    const float dvd2 = v * kLn2 * w2 * (dd2 - dpip), dvd3 = v * kLn2 * w3 * (dd3 - dpip);
    const float dvd4 = v * kLn2 * w4 * (dd4 - dpip);
    atomicAdd(a.d_rhs + bl + s, dvd0 + dvd1);
    atomicAdd(a.d_rhs + br + s, dvd0 + dvd2);
    if (v1) {
      atomicAdd(a.d_rhs + bl + k1, dvd3);
      atomicAdd(a.d_rhs + br + k1, dvd4);
    }
    if (v2) {
      atomicAdd(a.d_rhs + br + k2, dvd3);
      atomicAdd(a.d_rhs + bl + k2, dvd4);
    }
    const float f_l = is_neg_inf(pbl) ? 0.f : ex2(rm_l + mt - pbl);
    const float f_r = is_neg_inf(pbr) ? 0.f : ex2(rm_r + mt - pbr);
    a.ud[(size_t)n * S + s] = vd2 * f_l;
    a.ud[(size_t)(a.N + n) * S + s] = vd1 * f_r;
    a.dud[(size_t)n * S + s] = dvd2 * f_l + vd2 * kLn2 * f_l * (dmt - dbl);
    a.dud[(size_t)(a.N + n) * S + s] = dvd1 * f_r + vd1 * kLn2 * f_r * (dmt - dbr);
    atomicAdd(a.g_pD + grow + s, dvd0);
    atomicAdd(a.g_pS + grow + s, dvd3 + dvd4);
    atomicAdd(a.g_mt + grow + s, dvd1 + dvd2);
  }
}

__global__ void __launch_bounds__(1024, 1) dts_so_tree_kernel(DtsSoArgs a) {
  extern __shared__ float sm[];
  const int S = a.S;
  float* U = sm;
  float* DU = sm + S;
  float* red = sm + 2 * S;
  const int row = blockIdx.x;
  const int n = row < a.N ? row : row - a.N;
  const long long child = row < a.N ? a.sl[n] : a.sr[n];
  const size_t rb = (size_t)row * S, cbase = (size_t)child * S;
  float tu = 0.f, tdu = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float u = a.ud[rb + s], du = a.dud[rb + s];
    U[s] = u;
    DU[s] = du;
    tu += u;
    tdu += du;
  }
  const float A = block_sum(tu, red);
  const float dA = block_sum(tdu, red);
  subtree_sums_levels(U, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
  subtree_sums_levels(DU, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
  const float rms = safe_max(a.row_max[child]);
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float pi = a.Pi[cbase + s];
    float wv = pi;
    if (a.use_col) wv += a.col[s];
    const float p = is_neg_inf(pi) ? 0.f : ex2(wv - rms);
    const float dp = kLn2 * p * a.dPi[cbase + s];
    const float contrib = dp * (A - U[s]) + p * (dA - DU[s]);
    atomicAdd(a.d_rhs + cbase + s, contrib);
    atomicAdd(a.g_col + s, contrib);
  }
}

// ------------------------------------------------------------------------------------------------
// e_step_so: all G rows in one CTA (rows in order: deterministic column sums)
// ------------------------------------------------------------------------------------------------

struct ESoArgs {
  const float *E, *E_new, *E_s1, *E_s2, *Ebar, *pS, *pD, *pL, *col;
  const int *parent, *c1, *c2, *jumps;
  int K;
  const long long* lv_ptr;
  int n_levels;
  const int *lv_par, *lv_c1, *lv_c2;
  const float *g_new, *g_ebar;
  const float *dE, *dE_new, *dE_s1, *dE_s2, *dEbar, *dpS, *dpD, *dpL, *dcol;
  float *d_grad_E, *d_grad_pS, *d_grad_pD, *d_grad_pL, *d_grad_mc, *d_grad_col;
  int S, G, use_col;
};

__global__ void __launch_bounds__(1024, 1) e_step_so_kernel(ESoArgs a) {
  extern __shared__ float sm[];
  const int S = a.S;
  float* X = sm;
  float* Y = sm + S;
  float* X2 = sm + 2 * S;
  float* Y2 = sm + 3 * S;
  float* Q0 = sm + 4 * S;
  float* red = sm + 5 * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x) a.d_grad_col[s] = 0.f;
  for (int g = 0; g < a.G; ++g) {
    const size_t b = (size_t)g * S;
    __syncthreads();
    float m = neg_inf();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      float w = a.E[b + s];
      if (a.use_col) w += a.col[s];
      m = fmaxf(m, w);
    }
    const float rms = safe_max(block_max(m, red));
    float rs = 0.f, drs = 0.f;
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      float w = a.E[b + s], dw = a.dE[b + s];
      if (a.use_col) {
        w += a.col[s];
        if (a.dcol) dw += a.dcol[s];
      }
      const float r = ex2(w - rms);
      const float dr = kLn2 * r * dw;
      X[s] = r;
      X2[s] = dr;
      rs += r;
      drs += dr;
      const float gn = a.g_new[b + s];
      const float en = a.E_new[b + s], den = a.dE_new[b + s];
      const float e = a.E[b + s], de = a.dE[b + s];
      const float t0 = a.pS[b + s] + a.E_s1[b + s] + a.E_s2[b + s], t1 = a.pD[b + s] + 2.0f * e;
      const float t2 = e + a.Ebar[b + s], t3 = a.pL[b + s];
      const float dt0 = a.dpS[b + s] + a.dE_s1[b + s] + a.dE_s2[b + s], dt1 = a.dpD[b + s] + 2.0f * de;
      const float dt2 = de + a.dEbar[b + s], dt3 = a.dpL[b + s];
      const float q0 = gn * ex2(t0 - en), q1 = gn * ex2(t1 - en), q2 = gn * ex2(t2 - en);
      const float dq0 = kLn2 * q0 * (dt0 - den), dq1 = kLn2 * q1 * (dt1 - den), dq2 = kLn2 * q2 * (dt2 - den);
      const float dq3 = kLn2 * (gn * ex2(t3 - en)) * (dt3 - den);
      a.d_grad_pS[b + s] = dq0;
      a.d_grad_pD[b + s] = dq1;
      a.d_grad_pL[b + s] = dq3;
      a.d_grad_mc[b + s] = dq2;
      a.d_grad_E[b + s] = 2.0f * dq1 + dq2;
      Q0[s] = dq0;
    }
    const float row_sum = block_sum(rs, red);
    const float drow_sum = block_sum(drs, red);
    const float* anc = ancestor_sum_doubling(X, Y, a.jumps, a.K, S);
    const float* danc = ancestor_sum_doubling(X2, Y2, a.jumps, a.K, S);
    float* U = (anc == X) ? Y : X;
    float* DU = (danc == X2) ? Y2 : X2;
    float tu = 0.f, tdu = 0.f;
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      const float denom = row_sum - anc[s], ddenom = drow_sum - danc[s];
      const float gn = a.g_new[b + s];
      const float e = a.E[b + s];
      const float q2 = gn * ex2(e + a.Ebar[b + s] - a.E_new[b + s]);
      const float wbar = q2 + a.g_ebar[b + s];
      const float dwbar = a.d_grad_mc[b + s];
      const bool pos = denom > 0.f;
      const float u = pos ? wbar / denom : 0.f;
      const float du = pos ? (dwbar - u * ddenom) / denom : 0.f;
      U[s] = u;
      DU[s] = du;
      tu += u;
      tdu += du;
    }
    const float tot = block_sum(tu, red);
    const float dtot = block_sum(tdu, red);
    subtree_sums_levels(U, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
    subtree_sums_levels(DU, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      float w = a.E[b + s], dw = a.dE[b + s];
      if (a.use_col) {
        w += a.col[s];
        if (a.dcol) dw += a.dcol[s];
      }
      const float r = ex2(w - rms);
      const float dr = kLn2 * r * dw;
      const float d_pv = dr * (tot - U[s]) + r * (dtot - DU[s]);
      const float ge = a.d_grad_E[b + s] + from_parent(a.parent, a.c1, a.c2, Q0, Q0, s, S);
      a.d_grad_E[b + s] = ge + d_pv;
      a.d_grad_col[s] += d_pv;
    }
  }
}

}  // namespace

extern "C" int kb_wave_backward_so(const float* Pi, const float* dPi, const float* Pibar, const float* dPibar,
                                   const float* v, long long ws, int W, const float* pibar_row_max, const float* mc,
                                   const float* DL, const float* dDL, const float* Ebar, const float* dEbar,
                                   const float* E, const float* dE, const float* SL1, const float* dSL1,
                                   const float* SL2, const float* dSL2, long long const_row_stride,
                                   const float* col_log_probs, int use_col_weights, const int* node_parent,
                                   const int* node_child1, const int* node_child2, const int* jumps, int K,
                                   const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1,
                                   const int* lv_c2, const int* leaf_state, const float* leaf_logp,
                                   const float* dleaf_logp, const long long* item_idx, const float* dts_r,
                                   const float* d_dts, const float* d_rhs, float* d_out, float* d_aw, int S,
                                   void* stream) {
  if (S <= 0 || W < 0 || K < 0 || n_levels < 0 || ws < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if ((dts_r == nullptr) != (d_dts == nullptr)) return KB_ERR_ARG;
  if (leaf_state && (!leaf_logp || !dleaf_logp)) return KB_ERR_ARG;
  if (W == 0) return KB_OK;
  WaveSoArgs a;
  a.Pi = Pi; a.dPi = dPi; a.Pibar = Pibar; a.dPibar = dPibar; a.v = v; a.ws = ws; a.S = S;
  a.row_max = pibar_row_max; a.mc = mc; a.DL = DL; a.dDL = dDL; a.Ebar = Ebar; a.dEbar = dEbar; a.E = E; a.dE = dE;
  a.SL1 = SL1; a.dSL1 = dSL1; a.SL2 = SL2; a.dSL2 = dSL2; a.crs = const_row_stride;
  a.col = col_log_probs; a.use_col = use_col_weights;
  a.parent = node_parent; a.c1 = node_child1; a.c2 = node_child2; a.jumps = jumps; a.K = K;
  a.lv_ptr = lv_ptr; a.n_levels = n_levels; a.lv_par = lv_par; a.lv_c1 = lv_c1; a.lv_c2 = lv_c2;
  a.leaf_state = leaf_state; a.leaf_logp = leaf_logp; a.dleaf_logp = dleaf_logp; a.item_idx = item_idx;
  a.dts_r = dts_r; a.d_dts = d_dts; a.d_rhs = d_rhs; a.d_out = d_out; a.d_aw = d_aw;
  a.aw_stride = (long long)W * S;
  const size_t smem = (size_t)(6 * S + 64) * sizeof(float);
  if (so_smem((const void*)wave_so_kernel, smem)) return KB_ERR_LAUNCH;
  wave_so_kernel<<<W, so_block(S), smem, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_dts_backward_so(const float* Pi, const float* dPi, const float* Pibar, const float* dPibar,
                                  const float* v, long long ws, const long long* sl, const long long* sr,
                                  const long long* reduce_idx, const float* log_split_probs, int N,
                                  long long item_offset, const long long* item_idx, const float* log_pD,
                                  const float* log_pS, const float* dlog_pD, const float* dlog_pS,
                                  long long param_row_stride, const float* mt, const float* dmt,
                                  long long mt_row_stride, const float* pibar_row_max, const float* col_log_probs,
                                  int use_col_weights, const int* node_child1, const int* node_child2,
                                  const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1,
                                  const int* lv_c2, float* ud, float* dud, float* d_rhs, float* d_grad_pD,
                                  float* d_grad_pS, float* d_grad_mt, float* d_grad_col, int S, void* stream) {
  if (S <= 0 || N < 0 || n_levels < 0 || ws < 0 || item_offset < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (N == 0) return KB_OK;
  if (!ud || !dud || !d_rhs || !d_grad_pD || !d_grad_pS || !d_grad_mt || !d_grad_col) return KB_ERR_ARG;
  DtsSoArgs a;
  a.Pi = Pi; a.dPi = dPi; a.Pibar = Pibar; a.dPibar = dPibar; a.v = v; a.ws = ws;
  a.sl = sl; a.sr = sr; a.red = reduce_idx; a.lsp = log_split_probs; a.N = N;
  a.item_offset = item_offset; a.item_idx = item_idx;
  a.pD = log_pD; a.pS = log_pS; a.dpD = dlog_pD; a.dpS = dlog_pS; a.prs = param_row_stride;
  a.mt = mt; a.dmt = dmt; a.mrs = mt_row_stride; a.row_max = pibar_row_max;
  a.col = col_log_probs; a.use_col = use_col_weights; a.c1 = node_child1; a.c2 = node_child2;
  a.lv_ptr = lv_ptr; a.n_levels = n_levels; a.lv_par = lv_par; a.lv_c1 = lv_c1; a.lv_c2 = lv_c2;
  a.ud = ud; a.dud = dud; a.d_rhs = d_rhs; a.g_pD = d_grad_pD; a.g_pS = d_grad_pS; a.g_mt = d_grad_mt;
  a.g_col = d_grad_col; a.S = S;
  cudaStream_t st = (cudaStream_t)stream;
  dts_so_split_kernel<<<N, 256, 0, st>>>(a);
  if (cudaGetLastError() != cudaSuccess) return KB_ERR_LAUNCH;
  const size_t smem = (size_t)(2 * S + 64) * sizeof(float);
  if (so_smem((const void*)dts_so_tree_kernel, smem)) return KB_ERR_LAUNCH;
  dts_so_tree_kernel<<<2 * N, so_block(S), smem, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_e_step_backward_so(const float* E, const float* E_new, const float* E_s1, const float* E_s2,
                                     const float* Ebar, const float* log_pS, const float* log_pD,
                                     const float* log_pL, const float* col_log_probs, const int* node_parent,
                                     const int* node_child1, const int* node_child2, const int* jumps, int K,
                                     const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1,
                                     const int* lv_c2, const float* g_new, const float* g_ebar, const float* dE,
                                     const float* dE_new, const float* dE_s1, const float* dE_s2,
                                     const float* dEbar, const float* dlog_pS, const float* dlog_pD,
                                     const float* dlog_pL, const float* dcol, float* d_grad_E, float* d_grad_pS,
                                     float* d_grad_pD, float* d_grad_pL, float* d_grad_mc, float* d_grad_col,
                                     int S, int G, int use_col_weights, void* stream) {
  if (S <= 0 || G <= 0 || K < 0 || n_levels < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (!g_new || !g_ebar) return KB_ERR_ARG;
  ESoArgs a;
  a.E = E; a.E_new = E_new; a.E_s1 = E_s1; a.E_s2 = E_s2; a.Ebar = Ebar; a.pS = log_pS; a.pD = log_pD;
  a.pL = log_pL; a.col = col_log_probs; a.parent = node_parent; a.c1 = node_child1; a.c2 = node_child2;
  a.jumps = jumps; a.K = K; a.lv_ptr = lv_ptr; a.n_levels = n_levels; a.lv_par = lv_par; a.lv_c1 = lv_c1;
  a.lv_c2 = lv_c2; a.g_new = g_new; a.g_ebar = g_ebar; a.dE = dE; a.dE_new = dE_new; a.dE_s1 = dE_s1;
  a.dE_s2 = dE_s2; a.dEbar = dEbar; a.dpS = dlog_pS; a.dpD = dlog_pD; a.dpL = dlog_pL; a.dcol = dcol;
  a.d_grad_E = d_grad_E; a.d_grad_pS = d_grad_pS; a.d_grad_pD = d_grad_pD; a.d_grad_pL = d_grad_pL;
  a.d_grad_mc = d_grad_mc; a.d_grad_col = d_grad_col; a.S = S; a.G = G; a.use_col = use_col_weights;
  const size_t smem = (size_t)(5 * S + 64) * sizeof(float);
  if (so_smem((const void*)e_step_so_kernel, smem)) return KB_ERR_LAUNCH;
  e_step_so_kernel<<<1, so_block(S), smem, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

// Column sums of one wave's six parameter buckets (aw0, aw1, aw2, aw345, aw3, aw4 [W,S] each) from
// the second-order contraction (c_aw: one [6,W,S] buffer) plus the tangent adjoint's (l.p[0..5]),
// added into the tangent cotangent accumulators: d_pD += aw0, d_pS += aw345, d_E += aw0 + aw2,
// d_Ebar += aw1, d_Es1 += aw4, d_Es2 += aw3, d_mc += aw2.  Block (32, 32): 32 columns per block,
// the rows strided over 32 threads, then summed in a fixed order (deterministic).  The pointers
// travel by value in the launch (a CUDA graph replays them as they were).
struct AwBuckets {
  const float* p[6];
};

__global__ void __launch_bounds__(1024) aw_accumulate_kernel(const float* __restrict__ c_aw, AwBuckets l, int W,
                                                             int S, float* d_pD, float* d_pS, float* d_E,
                                                             float* d_Ebar, float* d_Es1, float* d_Es2,
                                                             float* d_mc) {
  __shared__ float part[6][32][33];
  const int lane = threadIdx.x, ty = threadIdx.y;
  const int s = blockIdx.x * 32 + lane;
  float acc[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (s < S) {
    const size_t WS = (size_t)W * S;
    for (int w = ty; w < W; w += 32) {
      const size_t o = (size_t)w * S + s;
#pragma unroll
      for (int k = 0; k < 6; ++k) acc[k] += c_aw[k * WS + o] + l.p[k][o];
    }
  }
#pragma unroll
  for (int k = 0; k < 6; ++k) part[k][ty][lane] = acc[k];
  __syncthreads();
  if (ty == 0 && s < S) {
    float tot[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      float t = 0.f;
      for (int y = 0; y < 32; ++y) t += part[k][y][lane];
      tot[k] = t;
    }
    d_pD[s] += tot[0];
    d_pS[s] += tot[3];
    d_E[s] += tot[0] + tot[2];
    d_Ebar[s] += tot[1];
    d_Es1[s] += tot[5];
    d_Es2[s] += tot[4];
    d_mc[s] += tot[2];
  }
}

extern "C" int kb_hvp_aw_accumulate(const float* c_aw, const float* l_aw0, const float* l_aw1, const float* l_aw2,
                                    const float* l_aw345, const float* l_aw3, const float* l_aw4, int W, int S,
                                    float* d_pD, float* d_pS, float* d_E, float* d_Ebar, float* d_Es1, float* d_Es2,
                                    float* d_mc, void* stream) {
  if (W < 0 || S <= 0 || !c_aw || !l_aw0 || !l_aw1 || !l_aw2 || !l_aw345 || !l_aw3 || !l_aw4) return KB_ERR_ARG;
  if (!d_pD || !d_pS || !d_E || !d_Ebar || !d_Es1 || !d_Es2 || !d_mc) return KB_ERR_ARG;
  if (W == 0) return KB_OK;
  AwBuckets l{{l_aw0, l_aw1, l_aw2, l_aw345, l_aw3, l_aw4}};
  aw_accumulate_kernel<<<(S + 31) / 32, dim3(32, 32), 0, (cudaStream_t)stream>>>(c_aw, l, W, S, d_pD, d_pS, d_E,
                                                                               d_Ebar, d_Es1, d_Es2, d_mc);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
