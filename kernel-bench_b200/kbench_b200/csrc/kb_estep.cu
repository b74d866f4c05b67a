// E-step kernels: the auxiliary S-column fixed point, one application, and its VJP.
//
// Restates kbench/core/kernels/e_step.py (reference): _e_step_forward_2d_kernel (:12-99),
// e_fixed_point_triton (:438-501), _e_step_backward_prepare/finalize_2d_kernel (:102-241).
// B200 design: the fixed point runs in ONE persistent CTA that iterates on the device until
// max|E_new - E| < tol or max_iter (no per-iteration host sync), with the row and the
// path-sum buffers resident in shared memory; the VJP replaces the reference's atomics by
// deterministic gathers (child -> parent edge and a bottom-up subtree sum).
#include "kb_common.cuh"
#include "kb_solver.h"

#include <mutex>

namespace {

using namespace kb;

struct EParams {
  const float* pS;   // [G,S]
  const float* pD;
  const float* pL;
  const float* mc;
  const float* col;  // [S]
  const int* parent;
  const int* c1;
  const int* c2;
  const int* jumps;  // [K,S]
  int K;
  int S;
  int use_col;
};

// One E application on row g. E (shared) holds the current row; X/Y are shared scratch (S each).
// Writes E_new/E_s1/E_s2/Ebar rows (any may be null) and returns max|E_new - E| on the row.
__device__ float e_apply_row(const float* E, float* X, float* Y, float* red, const EParams& p, int g,
                             float* E_new, float* E_s1o, float* E_s2o, float* Ebaro) {
  const int S = p.S;
  const size_t base = (size_t)g * S;
  float m = neg_inf();
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = E[s];
    if (p.use_col) w += p.col[s];
    m = fmaxf(m, w);
  }
  const float row_max = block_max(m, red);
  const float rms = safe_max(row_max);
  float sum = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = E[s];
    if (p.use_col) w += p.col[s];
    float x = ex2(w - rms);
    X[s] = x;
    sum += x;
  }
  const float row_sum = block_sum(sum, red);
  const float* anc = ancestor_sum_doubling(X, Y, p.jumps, p.K, S);
  float diff = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float e = E[s];
    const int a = p.c1[s], b = p.c2[s];
    const float es1 = (a >= 0 && a < S) ? E[a] : neg_inf();
    const float es2 = (b >= 0 && b < S) ? E[b] : neg_inf();
    const float denom = row_sum - anc[s];
    const float ebar = denom > 0.f ? lg2(denom) + row_max + p.mc[base + s] : neg_inf();
    const float t0 = p.pS[base + s] + es1 + es2;
    const float t1 = p.pD[base + s] + 2.0f * e;
    const float t2 = e + ebar;
    const float t3 = p.pL[base + s];
    const float mm = fmaxf(fmaxf(t0, t1), fmaxf(t2, t3));
    const float ms = safe_max(mm);
    const float tot = ex2(t0 - ms) + ex2(t1 - ms) + ex2(t2 - ms) + ex2(t3 - ms);
    const float en = lg2(tot) + mm;
    if (E_new) E_new[base + s] = en;
    if (E_s1o) E_s1o[base + s] = es1;
    if (E_s2o) E_s2o[base + s] = es2;
    if (Ebaro) Ebaro[base + s] = ebar;
    diff = fmaxf(diff, fabsf(en - e));
  }
  return block_max(diff, red);
}

__global__ void e_fixed_point_kernel(const float* __restrict__ E0, float* E_out, float* E_tmp,
                                     float* E_s1, float* E_s2, float* Ebar, EParams p, int G,
                                     int max_iter, double tol, int* iters_out) {
  extern __shared__ float sm[];
  const int S = p.S;
  float* E = sm;
  float* X = sm + S;
  float* Y = sm + 2 * S;
  float* red = sm + 3 * S;
  // ping-pong between E_out and E_tmp; start from E0
  const float* cur = E0;
  float* bufs[2] = {E_out, E_tmp};
  int which = 0;
  int it = 0;
  while (it < max_iter) {
    float* nxt = bufs[which];
    float mdiff = 0.f;
    for (int g = 0; g < G; ++g) {
      __syncthreads();
      for (int s = threadIdx.x; s < S; s += blockDim.x) E[s] = cur[(size_t)g * S + s];
      __syncthreads();
      float d = e_apply_row(E, X, Y, red, p, g, nxt, nullptr, nullptr, nullptr);
      mdiff = fmaxf(mdiff, d);
    }
    __syncthreads();
    cur = nxt;
    which ^= 1;
    ++it;
    if ((double)mdiff < tol) break;
  }
  // final application at the converged E for (E_s1, E_s2, Ebar); E_out must hold the final E
  for (int g = 0; g < G; ++g) {
    __syncthreads();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      float v = cur[(size_t)g * S + s];
      E[s] = v;
      E_out[(size_t)g * S + s] = v;
    }
    __syncthreads();
    e_apply_row(E, X, Y, red, p, g, nullptr, E_s1, E_s2, Ebar);
  }
  if (threadIdx.x == 0 && iters_out) *iters_out = it;
}

__global__ void e_step_forward_kernel(const float* __restrict__ Ein, float* E_new, float* E_s1, float* E_s2,
                                      float* Ebar, float* max_diff, EParams p) {
  extern __shared__ float sm[];
  const int S = p.S;
  float* E = sm;
  float* X = sm + S;
  float* Y = sm + 2 * S;
  float* red = sm + 3 * S;
  const int g = blockIdx.x;
  for (int s = threadIdx.x; s < S; s += blockDim.x) E[s] = Ein[(size_t)g * S + s];
  __syncthreads();
  float d = e_apply_row(E, X, Y, red, p, g, E_new, E_s1, E_s2, Ebar);
  if (threadIdx.x == 0 && max_diff) max_diff[g] = d;
}

// VJP of one E application for all G rows in one CTA (rows in order -> deterministic grad_col).
__global__ void e_step_vjp_kernel(const float* __restrict__ Ein, const float* __restrict__ Enew,
                                  const float* __restrict__ Es1, const float* __restrict__ Es2,
                                  const float* __restrict__ Ebar, EParams p, int G,
                                  const float* g_new, const float* g_s1, const float* g_s2, const float* g_ebar,
                                  float* grad_E, float* grad_pS, float* grad_pD, float* grad_pL, float* grad_mc,
                                  float* grad_col, const long long* lv_ptr, int n_levels, const int* lv_par,
                                  const int* lv_c1, const int* lv_c2) {
  extern __shared__ float sm[];
  const int S = p.S;
  float* R = sm;          // r = 2^(weighted - rowmax)
  float* Q0 = sm + S;     // q0 + per-child cotangent scratch
  float* U = sm + 2 * S;  // u, then subtree sums of u
  float* Y = sm + 3 * S;
  float* red = sm + 4 * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x) grad_col[s] = 0.f;
  for (int g = 0; g < G; ++g) {
    const size_t base = (size_t)g * S;
    __syncthreads();
    float m = neg_inf();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      float w = Ein[base + s];
      if (p.use_col) w += p.col[s];
      m = fmaxf(m, w);
    }
    const float row_max = block_max(m, red);
    const float rms = safe_max(row_max);
    float sum = 0.f;
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      float w = Ein[base + s];
      if (p.use_col) w += p.col[s];
      float r = ex2(w - rms);
      R[s] = r;
      U[s] = r;
      sum += r;
    }
    const float row_sum = block_sum(sum, red);
    // path sums of r (ancestor-or-self) into a copy (U is used as the doubling input)
    const float* anc = ancestor_sum_doubling(U, Y, p.jumps, p.K, S);
    // per element: q_k, wbar, u; own part of grad_E
    float* Ucopy = (anc == U) ? Y : U;  // the free buffer
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      const float e = Ein[base + s];
      const float en = Enew[base + s];
      const float gn = g_new ? g_new[base + s] : 0.f;
      const float t0 = p.pS[base + s] + Es1[base + s] + Es2[base + s];
      const float t1 = p.pD[base + s] + 2.0f * e;
      const float t2 = e + Ebar[base + s];
      const float t3 = p.pL[base + s];
      const float q0 = gn * ex2(t0 - en);
      const float q1 = gn * ex2(t1 - en);
      const float q2 = gn * ex2(t2 - en);
      const float q3 = gn * ex2(t3 - en);
      const float wbar = q2 + (g_ebar ? g_ebar[base + s] : 0.f);
      grad_pS[base + s] = q0;
      grad_pD[base + s] = q1;
      grad_pL[base + s] = q3;
      grad_mc[base + s] = wbar;
      Q0[s] = q0;
      grad_E[base + s] = 2.0f * q1 + q2;
      const float denom = row_sum - anc[s];
      const float u = denom > 0.f ? wbar / denom : 0.f;
      Ucopy[s] = u;
    }
    __syncthreads();
    float tu = 0.f;
    for (int s = threadIdx.x; s < S; s += blockDim.x) tu += Ucopy[s];
    const float total_u = block_sum(tu, red);
    subtree_sums_levels(Ucopy, lv_ptr, n_levels, lv_par, lv_c1, lv_c2, S);
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      float ge = grad_E[base + s];
      // child edge: s receives q0[parent] + g_s{1,2}[parent] when it is that parent's child
      const int par = p.parent[s];
      if (par >= 0 && par < S) {
        if (p.c1[par] == s) ge += Q0[par] + (g_s1 ? g_s1[base + par] : 0.f);
        if (p.c2[par] == s) ge += Q0[par] + (g_s2 ? g_s2[base + par] : 0.f);
      }
      const float pv = R[s] * (total_u - Ucopy[s]);
      grad_E[base + s] = ge + pv;
      grad_col[s] += pv;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// E adjoint: solve (I - J_E^T) w = q at the fixed point E* with BiCGSTAB inside ONE CTA.
//
// Restates _implicit_grad.py:373-475 (the aux VJP, the BiCGSTAB of :28-94 and the parameter
// VJP of the E step) for a single shared row.  The reference runs every BiCGSTAB scalar
// through the host (a synchronisation per test) and one VJP launch per matvec; here the whole
// solve is one launch.  J_E^T w is the E-step VJP with only the E_new cotangent set, and every
// factor of it that depends on E* alone is computed once:
//   q0 = w*C0, q1 = w*C1, q2 = w*C2 (C_k = 2^(t_k - E_new)),  u = q2 / denom,
//   J^T w [s] = 2 q1 + q2 + q0[parent] (when s is a child) + R[s] * (sum u - subtree_u[s]).
// Scalars are kept in fp64 and the dot products reduce in fp64; vectors stay fp32 like the
// reference's.  The stopping and breakdown rules are the reference's: converge when
// ||s||/max(||b||,1) or ||r||/max(||b||,1) <= tol; stop with failure when |rho|, |r_hat.v|,
// |t.t| or |omega| <= breakdown_tol, or after max_iter iterations.
// ---------------------------------------------------------------------------------------------

// Work layout (floats, S each): the E step at E*, the matvec factors, the BiCGSTAB vectors.
enum {
  EA_EN = 0, EA_S1, EA_S2, EA_EBAR, EA_C0, EA_C1, EA_C2, EA_C3, EA_R, EA_DN,
  EA_X, EA_RV, EA_RH, EA_P, EA_V, EA_SV, EA_T, EA_NVEC
};
static_assert(EA_NVEC == KB_EADJ_WORK_VECTORS, "work layout and header disagree");

struct EAdjArgs {
  EParams p;
  const long long* lv_ptr;
  int n_levels;
  const int* lv_par;
  const int* lv_c1;
  const int* lv_c2;
  const float* E;      // [S] fixed point
  const float* gE;     // [S] accumulated cotangents of E, E_bar, E_s1, E_s2
  const float* gEbar;
  const float* gEs1;
  const float* gEs2;
  double n_fam;        // weight of the direct log2(1 - mean 2^E) term
  int max_iter;
  double tol;
  double bdtol;
  float* work;         // [EA_NVEC, S]
  float* w_out;        // [S] the solution w
  float* grad_p;       // [5, S] cotangents of log_pS, log_pD, log_pL, max_coupling, col_log_probs
  int* status;         // [2] (0 converged / 1 failed, iterations)
  float* rel_out;      // [1] last relative residual
};

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Two fp64 block sums in one pass (scratch >= 64 doubles; two barriers).
__device__ __forceinline__ void block_sum2_d(double& a, double& b, double* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  a = warp_sum_d(a);
  b = warp_sum_d(b);
  __syncthreads();
  if (lane == 0) { scratch[wid] = a; scratch[32 + wid] = b; }
  __syncthreads();
  a = warp_sum_d(lane < nw ? scratch[lane] : 0.0);
  b = warp_sum_d(lane < nw ? scratch[32 + lane] : 0.0);
}

// u-part of the VJP: U[s] = num(s) / denom[s] (0 where denom <= 0), then its total and subtree sums.
// Returns the total; U holds subtree sums afterwards.
template <class Num>
__device__ __forceinline__ float eadj_u_sums(const EAdjArgs& a, float* U, float* red, Num num) {
  const int S = a.p.S;
  const float* Dn = a.work + (size_t)EA_DN * S;
  __syncthreads();
  float tu = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float dn = Dn[s];
    const float u = dn > 0.f ? num(s) / dn : 0.f;
    U[s] = u;
    tu += u;
  }
  const float total = block_sum(tu, red);
  subtree_sums_levels(U, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
  return total;
}

// out = in - J_E^T in.  Accumulates dot(out, y1) and dot(out, y2) (y may be null) per thread.
__device__ __forceinline__ void eadj_matvec(const EAdjArgs& a, const float* in, float* out, float* Q0, float* U,
                                            float* red, const float* y1, double& d1, const float* y2,
                                            double& d2) {
  const int S = a.p.S;
  const float* C0 = a.work + (size_t)EA_C0 * S;
  const float* C1 = a.work + (size_t)EA_C1 * S;
  const float* C2 = a.work + (size_t)EA_C2 * S;
  const float* R = a.work + (size_t)EA_R * S;
  __syncthreads();  // Q0 is free
  for (int s = threadIdx.x; s < S; s += blockDim.x) Q0[s] = in[s] * C0[s];
  const float total_u = eadj_u_sums(a, U, red, [&](int s) { return in[s] * C2[s]; });
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float g = in[s];
    const float q1 = g * C1[s];
    const float q2 = g * C2[s];
    float ge = 2.0f * q1 + q2;
    const int par = a.p.parent[s];
    if (par >= 0 && par < S) {
      if (a.p.c1[par] == s) ge += Q0[par];
      if (a.p.c2[par] == s) ge += Q0[par];
    }
    ge = ge + R[s] * (total_u - U[s]);
    const float o = g - ge;
    out[s] = o;
    if (y1) d1 += (double)o * (double)y1[s];
    if (y2) d2 += (double)o * (double)y2[s];
  }
}

__global__ void __launch_bounds__(1024, 1) e_adjoint_kernel(EAdjArgs a) {
  extern __shared__ float sm[];
  const int S = a.p.S;
  float* Es = sm;
  float* X = sm + S;
  float* Y = sm + 2 * S;
  float* red = sm + 3 * S;                                             // 64 floats
  double* redd = reinterpret_cast<double*>(sm + ((3 * S + 64 + 1) & ~1));  // 64 doubles, 8-byte aligned
  float* W = a.work;
  auto vec = [&](int k) { return W + (size_t)k * S; };

  // (1) the E step at E* (E_new, E_s1, E_s2, Ebar), as _TritonEStep2D.forward computes it
  for (int s = threadIdx.x; s < S; s += blockDim.x) Es[s] = a.E[s];
  __syncthreads();
  e_apply_row(Es, X, Y, red, a.p, 0, vec(EA_EN), vec(EA_S1), vec(EA_S2), vec(EA_EBAR));
  // (2) matvec factors: R = 2^(weighted E - row max), denom = row_sum - ancestor sum of R, C_k
  float m = neg_inf();
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = Es[s];
    if (a.p.use_col) w += a.p.col[s];
    m = fmaxf(m, w);
  }
  const float rms = safe_max(block_max(m, red));
  float sum = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = Es[s];
    if (a.p.use_col) w += a.p.col[s];
    const float r = ex2(w - rms);
    vec(EA_R)[s] = r;
    X[s] = r;
    sum += r;
  }
  const float row_sum = block_sum(sum, red);
  const float* anc = ancestor_sum_doubling(X, Y, a.p.jumps, a.p.K, S);
  double nrm = 0.0;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float e = Es[s];
    const float en = vec(EA_EN)[s];
    vec(EA_DN)[s] = row_sum - anc[s];
    vec(EA_C0)[s] = ex2(a.p.pS[s] + vec(EA_S1)[s] + vec(EA_S2)[s] - en);
    vec(EA_C1)[s] = ex2(a.p.pD[s] + 2.0f * e - en);
    vec(EA_C2)[s] = ex2(e + vec(EA_EBAR)[s] - en);
    vec(EA_C3)[s] = ex2(a.p.pL[s] - en);
    nrm += (double)ex2(e);
  }
  double dummy = 0.0;
  block_sum2_d(nrm, dummy, redd);
  // (3) right-hand side q = gE + d/dE [n_fam log2(1 - mean 2^E)] + VJP(E_s1, E_s2, Ebar cotangents)
  float* Q0 = X;
  float* U = Y;
  const float total_u0 = eadj_u_sums(a, U, red, [&](int s) { return a.gEbar[s]; });
  const float norm = (float)(1.0 - nrm / (double)S);
  const bool live = norm >= 1.17549435e-38f;  // torch clamp_min(tiny) passes the gradient where norm >= tiny
  const float dscale = live ? (float)(-a.n_fam / ((double)S * (double)norm)) : 0.f;
  double b2 = 0.0;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float ge = 0.f;
    const int par = a.p.parent[s];
    if (par >= 0 && par < S) {
      if (a.p.c1[par] == s) ge += a.gEs1[par];
      if (a.p.c2[par] == s) ge += a.gEs2[par];
    }
    ge = ge + vec(EA_R)[s] * (total_u0 - U[s]);
    const float aux = ge + dscale * ex2(Es[s]);
    const float b = a.gE[s] + aux;
    vec(EA_RV)[s] = b;   // r = b - A 0 = b
    vec(EA_RH)[s] = b;
    vec(EA_X)[s] = 0.f;
    vec(EA_P)[s] = 0.f;
    vec(EA_V)[s] = 0.f;
    b2 += (double)b * (double)b;
  }
  block_sum2_d(b2, dummy, redd);
  const double bnorm = fmax(sqrt(b2), 1.0);
  double rel = sqrt(b2) / bnorm;
  int code = 1, k = 0;
  double rho = b2;  // r_hat . r with r_hat = r = b
  if (rel <= a.tol) {
    code = 0;
  } else {
    double rho_old = 1.0, alpha = 1.0, omega = 1.0;
    for (k = 1; k <= a.max_iter; ++k) {
      if (fabs(rho) <= a.bdtol) break;
      const double beta = (rho / rho_old) * (alpha / omega);
      const float fb = (float)beta, fo = (float)omega;
      __syncthreads();
      for (int s = threadIdx.x; s < S; s += blockDim.x)
        vec(EA_P)[s] = vec(EA_RV)[s] + fb * (vec(EA_P)[s] - fo * vec(EA_V)[s]);
      double den = 0.0, d0 = 0.0;
      eadj_matvec(a, vec(EA_P), vec(EA_V), Q0, U, red, vec(EA_RH), den, nullptr, d0);
      block_sum2_d(den, d0, redd);
      if (fabs(den) <= a.bdtol) break;
      alpha = rho / den;
      const float fa = (float)alpha;
      double s2 = 0.0;
      for (int s = threadIdx.x; s < S; s += blockDim.x) {
        const float v = vec(EA_RV)[s] - fa * vec(EA_V)[s];
        vec(EA_SV)[s] = v;
        s2 += (double)v * (double)v;
      }
      block_sum2_d(s2, d0, redd);
      if (sqrt(s2) / bnorm <= a.tol) {
        for (int s = threadIdx.x; s < S; s += blockDim.x) vec(EA_X)[s] = vec(EA_X)[s] + fa * vec(EA_P)[s];
        rel = sqrt(s2) / bnorm;
        code = 0;
        break;
      }
      double tt = 0.0, ts = 0.0;
      eadj_matvec(a, vec(EA_SV), vec(EA_T), Q0, U, red, vec(EA_T), tt, vec(EA_SV), ts);
      block_sum2_d(tt, ts, redd);
      if (fabs(tt) <= a.bdtol) break;
      omega = ts / tt;
      const float fo2 = (float)omega;
      double r2 = 0.0, rr = 0.0;
      for (int s = threadIdx.x; s < S; s += blockDim.x) {
        const float sv = vec(EA_SV)[s];
        vec(EA_X)[s] = vec(EA_X)[s] + fa * vec(EA_P)[s] + fo2 * sv;
        const float r = sv - fo2 * vec(EA_T)[s];
        vec(EA_RV)[s] = r;
        r2 += (double)r * (double)r;
        rr += (double)vec(EA_RH)[s] * (double)r;
      }
      block_sum2_d(r2, rr, redd);
      rel = sqrt(r2) / bnorm;
      if (rel <= a.tol) { code = 0; break; }
      if (fabs(omega) <= a.bdtol) break;
      rho_old = rho;
      rho = rr;
    }
    if (k > a.max_iter) k = a.max_iter;
  }
  // (4) parameter cotangents of the E step at w (E_new cotangent w, Ebar cotangent gEbar)
  __syncthreads();
  const float* x = vec(EA_X);
  const float total_w = eadj_u_sums(a, U, red, [&](int s) { return x[s] * vec(EA_C2)[s] + a.gEbar[s]; });
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float g = x[s];
    a.w_out[s] = g;
    a.grad_p[s] = g * vec(EA_C0)[s];
    a.grad_p[(size_t)S + s] = g * vec(EA_C1)[s];
    a.grad_p[(size_t)2 * S + s] = g * vec(EA_C3)[s];
    a.grad_p[(size_t)3 * S + s] = g * vec(EA_C2)[s] + a.gEbar[s];
    // the reference's finalize kernel adds this to the column cotangent whether or not the
    // column weights enter the E step (e_step.py:238-241); kept for parity
    a.grad_p[(size_t)4 * S + s] = vec(EA_R)[s] * (total_w - U[s]);
  }
  if (threadIdx.x == 0) {
    a.status[0] = code;
    a.status[1] = k;
    a.rel_out[0] = (float)rel;
  }
}

int set_smem(const void* fn, size_t bytes) {
  if (bytes > 48 * 1024) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
      return KB_ERR_LAUNCH;
  }
  return KB_OK;
}

int block_for(int S) {
  int b = ((S + 31) / 32) * 32;
  if (b > 1024) b = 1024;
  if (b < 32) b = 32;
  return b;
}

EParams make_params(const float* pS, const float* pD, const float* pL, const float* mc, const float* col,
                    const int* parent, const int* c1, const int* c2, const int* jumps, int K, int S,
                    int use_col) {
  EParams p;
  p.pS = pS; p.pD = pD; p.pL = pL; p.mc = mc; p.col = col;
  p.parent = parent; p.c1 = c1; p.c2 = c2; p.jumps = jumps; p.K = K; p.S = S; p.use_col = use_col;
  return p;
}

}  // namespace

extern "C" int kb_e_fixed_point(const float* E0, float* E_out, float* E_tmp, float* E_s1, float* E_s2,
                                float* Ebar, const float* log_pS, const float* log_pD, const float* log_pL,
                                const float* max_coupling, const float* col_log_probs, const int* node_parent,
                                const int* node_child1, const int* node_child2, const int* jumps, int K, int S,
                                int G, int max_iter, double tol, int use_col_weights, int* iters_out,
                                void* stream) {
  if (S <= 0 || G <= 0 || max_iter < 1 || K < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  EParams p = make_params(log_pS, log_pD, log_pL, max_coupling, col_log_probs, node_parent, node_child1,
                          node_child2, jumps, K, S, use_col_weights);
  const size_t smem = (size_t)(3 * S + 64) * sizeof(float);
  if (set_smem((const void*)e_fixed_point_kernel, smem)) return KB_ERR_LAUNCH;
  e_fixed_point_kernel<<<1, block_for(S), smem, (cudaStream_t)stream>>>(E0, E_out, E_tmp, E_s1, E_s2, Ebar, p,
                                                                          G, max_iter, tol, iters_out);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_e_step_forward(const float* E, float* E_new, float* E_s1, float* E_s2, float* Ebar,
                                 float* max_diff_out, const float* log_pS, const float* log_pD,
                                 const float* log_pL, const float* max_coupling, const float* col_log_probs,
                                 const int* node_parent, const int* node_child1, const int* node_child2,
                                 const int* jumps, int K, int S, int G, int use_col_weights, void* stream) {
  if (S <= 0 || G <= 0 || K < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  EParams p = make_params(log_pS, log_pD, log_pL, max_coupling, col_log_probs, node_parent, node_child1,
                          node_child2, jumps, K, S, use_col_weights);
  const size_t smem = (size_t)(3 * S + 64) * sizeof(float);
  if (set_smem((const void*)e_step_forward_kernel, smem)) return KB_ERR_LAUNCH;
  e_step_forward_kernel<<<G, block_for(S), smem, (cudaStream_t)stream>>>(E, E_new, E_s1, E_s2, Ebar,
                                                                           max_diff_out, p);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_e_step_vjp(const float* E, const float* E_new, const float* E_s1, const float* E_s2,
                             const float* Ebar, const float* log_pS, const float* log_pD, const float* log_pL,
                             const float* col_log_probs, const int* node_parent, const int* node_child1,
                             const int* node_child2, const int* jumps, int K, const long long* lv_ptr,
                             int n_levels, const int* lv_par, const int* lv_c1, const int* lv_c2,
                             const float* g_new, const float* g_s1, const float* g_s2, const float* g_ebar,
                             float* grad_E, float* grad_pS, float* grad_pD, float* grad_pL, float* grad_mc,
                             float* grad_col, int S, int G, int use_col_weights, void* stream) {
  if (S <= 0 || G <= 0 || K < 0 || n_levels < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  EParams p = make_params(log_pS, log_pD, log_pL, nullptr, col_log_probs, node_parent, node_child1, node_child2,
                          jumps, K, S, use_col_weights);
  const size_t smem = (size_t)(4 * S + 64) * sizeof(float);
  if (set_smem((const void*)e_step_vjp_kernel, smem)) return KB_ERR_LAUNCH;
  e_step_vjp_kernel<<<1, block_for(S), smem, (cudaStream_t)stream>>>(
      E, E_new, E_s1, E_s2, Ebar, p, G, g_new, g_s1, g_s2, g_ebar, grad_E, grad_pS, grad_pD, grad_pL, grad_mc,
      grad_col, lv_ptr, n_levels, lv_par, lv_c1, lv_c2);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_e_adjoint_solve(const float* E, const float* log_pS, const float* log_pD, const float* log_pL,
                                  const float* max_coupling, const float* col_log_probs, const int* node_parent,
                                  const int* node_child1, const int* node_child2, const int* jumps, int K,
                                  const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1,
                                  const int* lv_c2, const float* g_E, const float* g_Ebar, const float* g_E_s1,
                                  const float* g_E_s2, double n_fam, int max_iter, double tol,
                                  double breakdown_tol, float* work, float* w_out, float* grad_params,
                                  int* status, float* rel_out, int S, int use_col_weights, void* stream) {
  if (S <= 0 || K < 0 || n_levels < 0 || max_iter < 1 || !(tol > 0.0) || !(breakdown_tol > 0.0)) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (!E || !g_E || !g_Ebar || !g_E_s1 || !g_E_s2 || !work || !w_out || !grad_params || !status || !rel_out)
    return KB_ERR_ARG;
  EAdjArgs a;
  a.p = make_params(log_pS, log_pD, log_pL, max_coupling, col_log_probs, node_parent, node_child1, node_child2,
                    jumps, K, S, use_col_weights);
  a.lv_ptr = lv_ptr; a.n_levels = n_levels; a.lv_par = lv_par; a.lv_c1 = lv_c1; a.lv_c2 = lv_c2;
  a.E = E; a.gE = g_E; a.gEbar = g_Ebar; a.gEs1 = g_E_s1; a.gEs2 = g_E_s2; a.n_fam = n_fam;
  a.max_iter = max_iter; a.tol = tol; a.bdtol = breakdown_tol;
  a.work = work; a.w_out = w_out; a.grad_p = grad_params; a.status = status; a.rel_out = rel_out;
  const size_t smem = (size_t)((3 * S + 64 + 1) & ~1) * sizeof(float) + 64 * sizeof(double);
  if (set_smem((const void*)e_adjoint_kernel, smem)) return KB_ERR_LAUNCH;
  e_adjoint_kernel<<<1, block_for(S), smem, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant of kb_e_fixed_point.
//
// Some hosts cannot allocate device memory at the point where they need the E fixed point: code
// that owns every device byte through its own pool and forbids driver allocations, or that runs
// where an allocation (and the synchronisation it may imply) is not allowed.  Such callers still
// pass their inputs and outputs, but the iteration's ping-pong buffer comes from this
// file-scope device array instead of a caller-provided scratch tensor.
//
// The array is part of the library image: every GPU that loads the library holds these
// KB_NOALLOC_ESTEP_MAX floats (256 KiB) until the process exits.  Host code cannot use the
// array's name as a device address, so the first call on each device (with that device
// current) looks the address up with cudaGetSymbolAddress and caches it; that first call should
// happen before any stream capture.  All calls share the array and it keeps the last call's
// contents (the iteration writes it before reading it, so nothing needs clearing); calls that
// overlap on the GPU -- concurrent streams, or several host threads -- race on it.
// ---------------------------------------------------------------------------------------------
namespace {

static __device__ __align__(256) float g_estep_noalloc_scratch[KB_NOALLOC_ESTEP_MAX];

constexpr int kMaxDevices = 64;
float* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mutex;

int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KB_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_estep_noalloc_scratch) != cudaSuccess || ptr == nullptr) return KB_ERR_LAUNCH;
    g_scratch_addr[dev] = static_cast<float*>(ptr);
  }
  *out = g_scratch_addr[dev];
  return KB_OK;
}

}  // namespace

extern "C" int kb_e_fixed_point_noalloc(const float* E0, float* E_out, float* E_s1, float* E_s2, float* Ebar,
                                        const float* log_pS, const float* log_pD, const float* log_pL,
                                        const float* max_coupling, const float* col_log_probs,
                                        const int* node_parent, const int* node_child1, const int* node_child2,
                                        const int* jumps, int K, int S, int G, int max_iter, double tol,
                                        int use_col_weights, int* iters_out, void* stream) {
  if (S <= 0 || G <= 0 || max_iter < 1 || K < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S || (long long)S * G > KB_NOALLOC_ESTEP_MAX) return KB_ERR_SIZE;
  float* scratch = nullptr;
  if (scratch_for_current_device(&scratch) != KB_OK) return KB_ERR_LAUNCH;
  EParams p = make_params(log_pS, log_pD, log_pL, max_coupling, col_log_probs, node_parent, node_child1,
                          node_child2, jumps, K, S, use_col_weights);
  const size_t smem = (size_t)(3 * S + 64) * sizeof(float);
  if (set_smem((const void*)e_fixed_point_kernel, smem)) return KB_ERR_LAUNCH;
  e_fixed_point_kernel<<<1, block_for(S), smem, (cudaStream_t)stream>>>(E0, E_out, scratch, E_s1, E_s2, Ebar, p, G,
                                                                          max_iter, tol, iters_out);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
