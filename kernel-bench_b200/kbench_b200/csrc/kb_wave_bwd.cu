// Backward (implicit adjoint) kernels for one wave.
//
// Restates kbench/core/kernels/wave_backward.py (reference; numerics of the pristine copy
// experiments/pristine_kernels/wave_backward.py):
//   * active_mask_from_rhs_absmax_fused                  (:166-201)
//   * wave_backward_uniform_fused: precompute (:203-417), Neumann J^T series (:419-570),
//     column gradient (:654-745), parameter store (:747-966), wrapper (:1270-1736)
//   * dts_cross_backward_accum_fused                     (:1529-1945, wrapper :1968-2180)
//   * uniform_cross_pibar_vjp_tree_from_ud_fused         (:2251-2446)
//
// B200 design: the whole per-row adjoint -- coefficient precompute, all Neumann terms, the
// column gradient and the parameter store -- runs in ONE launch with one CTA per row; the
// Neumann term, the bottom-up subtree sums and the coefficient rows stay in shared memory and
// registers, so a row is read from HBM once and its outputs written once (the reference makes
// neumann_terms + 3 launches, each a full read/write of several [W,S] scratch tensors).
#include <cfloat>

#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

using namespace kb;

__global__ void active_mask_kernel(const float* __restrict__ rhs, long long rs, int S, float thr, int strict,
                                   unsigned char* out) {
  __shared__ float red[64];
  const int w = blockIdx.x;
  const float* row = rhs + (size_t)w * rs;
  float m = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) m = fmaxf(m, fabsf(row[s]));
  m = block_max(m, red);
  if (threadIdx.x == 0) out[w] = strict ? (m > thr) : (m >= thr);
}

struct AdjArgs {
  const float* Pi;
  const float* Pibar;
  const float* row_max;  // [C]
  const float* dts;      // [W,S] or null
  const float* rhs;
  long long rhs_rs;
  const unsigned char* active;  // [W] or null
  const float* dl;
  const float* ebar;
  const float* e;
  const float* sl1;
  const float* sl2;
  int const_mode;  // 0 shared [S], 1 row-expanded [W,S], 2 item rows [G,S]
  const float* col;
  int use_col;
  const int* c1;
  const int* c2;
  const int* parent;
  const int* jumps;
  int K;
  const long long* lv_ptr;
  int n_levels;
  const int* lv_par;
  const int* lv_c1;
  const int* lv_c2;
  int use_leaf_index;
  const int* leaf_state;     // [C]
  const float* leaf_logp;    // addressed by leaf_mode
  int leaf_mode;             // 0 [S] shared, 1 [G] item scalar, 2 [G,S] item rows, 3 scalar
  const float* leaf_term;    // [W,S] materialised leaf term, or null
  const long long* item_idx; // [C] or null
  int neumann_terms;
  const float* init_v;       // [W,S] rows at stride init_rs, or null: with it the solve is the
  long long init_rs;         //   warm-started fixed point v <- rhs + J^T v (neumann_terms updates)
  float* grad_col;           // [S] or null (accumulated)
  float* v_k;
  float* aw0;
  float* aw1;
  float* aw2;
  float* aw345;
  float* aw3;
  float* aw4;
  float* last_relres;        // [W] or null: |last Neumann term| / |v| per row (0 on inactive rows)
  const float* apply_in;     // apply mode (apply_out != null): y = x - J^T x of one row per CTA,
  long long apply_rs;        //   x = apply_in rows (stride apply_rs); nothing else is written
  float* apply_out;          //   [W,S], zero on inactive rows
  int ws;
  int W;
  int S;
};

struct RowTerms {
  float e[6];
  float inv_sum;
  float w_L;
};

__device__ __forceinline__ RowTerms self_loop_terms(const AdjArgs& a, const float* P, size_t cb, long long rg, int w,
                                                     int s, long long item, int leaf) {
  const int S = a.S;
  const float pi = P[s];
  const float pib = a.Pibar[(size_t)rg * S + s];
  const float t0 = a.dl[cb + s] + pi;
  const float t1 = pi + a.ebar[cb + s];
  const float t2 = pib + a.e[cb + s];
  const int x = a.c1[s], y = a.c2[s];
  const float t3 = a.sl1[cb + s] + ((x >= 0 && x < S) ? P[x] : neg_inf());
  const float t4 = a.sl2[cb + s] + ((y >= 0 && y < S) ? P[y] : neg_inf());
  float t5 = neg_inf();
  if (a.use_leaf_index) {
    if (s == leaf) {
      switch (a.leaf_mode) {
        case 0: t5 = a.leaf_logp[s]; break;
        case 1: t5 = a.leaf_logp[item]; break;
        case 2: t5 = a.leaf_logp[(size_t)item * S + s]; break;
        default: t5 = a.leaf_logp[0]; break;
      }
    }
  } else if (a.leaf_term) {
    t5 = a.leaf_term[(size_t)w * S + s];
  }
  const float m = fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(t4, t5));
  const float ms = safe_max(m);
  RowTerms r;
  r.e[0] = ex2(t0 - ms);
  r.e[1] = ex2(t1 - ms);
  r.e[2] = ex2(t2 - ms);
  r.e[3] = ex2(t3 - ms);
  r.e[4] = ex2(t4 - ms);
  r.e[5] = ex2(t5 - ms);
  const float sum = r.e[0] + r.e[1] + r.e[2] + r.e[3] + r.e[4] + r.e[5];
  r.inv_sum = sum > 0.f ? 1.0f / sum : 0.f;
  if (a.dts) {
    const float dr = a.dts[(size_t)w * S + s];
    const float dlv = lg2(sum) + m;
    const float pm = fmaxf(dlv, dr);
    const float pms = safe_max(pm);
    const float pnew = lg2(ex2(dlv - pms) + ex2(dr - pms)) + pm;
    r.w_L = is_neg_inf(dlv) ? 0.f : ex2(dlv - pnew);
  } else {
    r.w_L = 1.0f;
  }
  return r;
}

template <int VPT>
__global__ void __launch_bounds__(512) wave_adjoint_kernel(AdjArgs a) {
  extern __shared__ float sm[];
  const int S = a.S;
  float* P = sm;
  float* X = sm + S;
  float* Y = sm + 2 * S;
  float* EDGE = sm + 3 * S;
  float* red = sm + 4 * S;
  const int w = blockIdx.x;
  const size_t ob = (size_t)w * S;
  if (a.active && a.active[w] == 0) {
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      if (a.apply_out) {
        a.apply_out[ob + s] = 0.f;
      } else {
        a.aw0[ob + s] = 0.f; a.aw1[ob + s] = 0.f; a.aw2[ob + s] = 0.f;
        a.aw345[ob + s] = 0.f; a.aw3[ob + s] = 0.f; a.aw4[ob + s] = 0.f;
        if (a.init_v) a.v_k[ob + s] = a.init_v[(size_t)w * a.init_rs + s];  // inactive rows keep it
      }
    }
    if (a.last_relres && threadIdx.x == 0) a.last_relres[w] = 0.f;
    return;
  }
  const long long rg = (long long)a.ws + w;
  const long long item = a.item_idx ? a.item_idx[rg] : 0;
  const size_t cb = a.const_mode == 0 ? 0 : (a.const_mode == 1 ? ob : (size_t)item * S);
  int leaf = -1;
  if (a.use_leaf_index) leaf = a.leaf_state[rg];
  const float* pirow = a.Pi + (size_t)rg * S;
  const float rmax = a.row_max[rg];
  const float rms = safe_max(rmax);
  float pp[VPT];
  float psum = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    pp[k] = 0.f;
    if (s < S) {
      const float pi = pirow[s];
      P[s] = pi;
      float wv = pi;
      if (a.use_col) wv += a.col[s];
      pp[k] = ex2(wv - rms);
      X[s] = pp[k];
      EDGE[s] = 0.f;
      psum += pp[k];
    }
  }
  const float row_sum = block_sum(psum, red);
  const float* anc = ancestor_sum_doubling(X, Y, a.jumps, a.K, S);
  float diag[VPT], coef[VPT], v[VPT], edge[VPT], nv[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    diag[k] = coef[k] = v[k] = 0.f;
    if (s < S) {
      const RowTerms t = self_loop_terms(a, P, cb, rg, w, s, item, leaf);
      const float denom = row_sum - anc[s];
      const float inv_denom = denom > 0.f ? 1.0f / denom : 0.f;
      diag[k] = t.w_L * (t.e[0] + t.e[1]) * t.inv_sum;
      coef[k] = t.w_L * t.e[2] * t.inv_sum * inv_denom;
      const float s1w = t.w_L * t.e[3] * t.inv_sum;
      const float s2w = t.w_L * t.e[4] * t.inv_sum;
      const int x = a.c1[s], y = a.c2[s];
      if (x >= 0 && x < S) EDGE[x] = s1w;
      if (y >= 0 && y < S) EDGE[y] = s2w;
      v[k] = a.apply_out ? a.apply_in[(size_t)w * a.apply_rs + s]
                         : (a.init_v ? a.init_v[(size_t)w * a.init_rs + s] : a.rhs[(size_t)w * a.rhs_rs + s]);
    }
  }
  __syncthreads();
  float* T = X;  // current Neumann term
  float* U = Y;  // u = term * coef, then its subtree sums
  if (anc == X) { T = Y; U = X; }
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    edge[k] = 0.f;
    if (s < S) {
      const int par = a.parent[s];
      edge[k] = (par >= 0 && par < S) ? EDGE[s] : 0.f;
      T[s] = v[k];
    }
  }
  const int n_terms = a.apply_out ? 1 : a.neumann_terms;
  for (int n = 0; n < n_terms; ++n) {
    float usum = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) {
        const float u = T[s] * coef[k];
        U[s] = u;
        usum += u;
      }
    }
    const float A = block_sum(usum, red);
    subtree_sums_levels(U, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      nv[k] = 0.f;
      if (s < S) {
        const int par = a.parent[s];
        const float base = T[s] * diag[k] + pp[k] * (A - U[s]);
        const float pt = (par >= 0 && par < S) ? T[par] : 0.f;
        nv[k] = base + pt * edge[k];
        if (a.init_v) {  // fixed-point update: the next iterate is rhs + J^T v, and is also the next T
          nv[k] = a.rhs[(size_t)w * a.rhs_rs + s] + nv[k];
          v[k] = nv[k];
        } else {
          v[k] += nv[k];
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) T[s] = nv[k];
    }
    __syncthreads();
  }
  if (a.apply_out) {  // T holds J^T x
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) a.apply_out[ob + s] = a.apply_in[(size_t)w * a.apply_rs + s] - T[s];
    }
    return;
  }
  if (a.last_relres) {  // T holds the last term added to v
    float tt = 0.f, vv = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) {
        tt += T[s] * T[s];
        vv += v[k] * v[k];
      }
    }
    tt = block_sum(tt, red);
    vv = block_sum(vv, red);
    if (threadIdx.x == 0) a.last_relres[w] = sqrtf(tt) / fmaxf(sqrtf(vv), FLT_MIN);
  }
  if (a.grad_col) {
    float usum = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) {
        const float u = v[k] * coef[k];
        U[s] = u;
        usum += u;
      }
    }
    const float A = block_sum(usum, red);
    subtree_sums_levels(U, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) atomicAdd(a.grad_col + s, pp[k] * (A - U[s]));
    }
  }
  // parameter store (recomputes the self-loop terms, as the reference does)
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) {
      const RowTerms t = self_loop_terms(a, P, cb, rg, w, s, item, leaf);
      const float alpha = v[k] * t.w_L;
      const float q0 = alpha * t.e[0] * t.inv_sum;
      const float q1 = alpha * t.e[1] * t.inv_sum;
      const float q2 = alpha * t.e[2] * t.inv_sum;
      const float q3 = alpha * t.e[3] * t.inv_sum;
      const float q4 = alpha * t.e[4] * t.inv_sum;
      const float q5 = alpha * t.e[5] * t.inv_sum;
      a.v_k[ob + s] = v[k];
      a.aw0[ob + s] = q0;
      a.aw1[ob + s] = q1;
      a.aw2[ob + s] = q2;
      a.aw345[ob + s] = q3 + q4 + q5;
      a.aw3[ob + s] = q3;
      a.aw4[ob + s] = q4;
    }
  }
}

struct ParamRef {   // value at base + item*row_stride + s*elem_stride
  const float* base;
  long long row_stride;
  int elem_stride;
};
struct GradRef {
  float* base;
  long long row_stride;
  int elem_stride;  // 0: one value per item row (block-reduced before the atomic)
};

struct DtsAdjArgs {
  const float* Pi;
  const float* Pibar;
  const float* v_k;  // [W,S]
  const unsigned char* active;
  const long long* sl;
  const long long* sr;
  const long long* reduce_idx;
  const float* wlsp;
  ParamRef pD;
  ParamRef pS;
  const long long* item_idx;  // [C] or null (item 0)
  const int* c1;
  const int* c2;
  float* rhs;  // accumulated_rhs [C,S]
  int output_ud;
  float* pibar_ud;       // [2N,S]
  float* pibar_A;        // [2N]
  unsigned char* side_active;  // [2N] or null
  float side_thr;
  int side_thr_enabled;
  int skip_inactive_zero;
  float* grad_Pibar_l;   // [N,S] (when !output_ud)
  float* grad_Pibar_r;
  int accum_param;
  GradRef g_pD;
  GradRef g_pS;
  float* param_pD;       // [N] when !accum_param
  float* param_pS;
  int accum_mt;
  GradRef g_mt;          // addressed by the child's item (left: vd2, right: vd1)
  ParamRef mt;           // addressed by the child's item
  const float* row_max;  // [C]
  int ws;
  int N;
  int S;
};

template <int VPT>
__global__ void __launch_bounds__(512) dts_adjoint_kernel(DtsAdjArgs a) {
  extern __shared__ float sm[];
  const int S = a.S;
  float* Pl = sm;
  float* Pr = sm + S;
  float* red = sm + 2 * S;
  const int i = blockIdx.x;
  const int N = a.N;
  const long long pw = a.reduce_idx[i];
  if (a.active && a.active[pw] == 0) {
    if (!a.accum_param && threadIdx.x == 0) { a.param_pD[i] = 0.f; a.param_pS[i] = 0.f; }
    if (a.output_ud) {
      if (a.side_active && threadIdx.x == 0) { a.side_active[i] = 0; a.side_active[N + i] = 0; }
      if (a.skip_inactive_zero) return;
      if (threadIdx.x == 0) { a.pibar_A[i] = 0.f; a.pibar_A[N + i] = 0.f; }
      for (int s = threadIdx.x; s < S; s += blockDim.x) {
        a.pibar_ud[(size_t)i * S + s] = 0.f;
        a.pibar_ud[(size_t)(N + i) * S + s] = 0.f;
      }
    } else {
      for (int s = threadIdx.x; s < S; s += blockDim.x) {
        a.grad_Pibar_l[(size_t)i * S + s] = 0.f;
        a.grad_Pibar_r[(size_t)i * S + s] = 0.f;
      }
    }
    return;
  }
  const long long l = a.sl[i], r = a.sr[i];
  const long long pg = (long long)a.ws + pw;
  const long long item = a.item_idx ? a.item_idx[pg] : 0;
  const long long item_l = a.item_idx ? a.item_idx[l] : 0;
  const long long item_r = a.item_idx ? a.item_idx[r] : 0;
  const float wl = a.wlsp[i];
  const float* pil = a.Pi + (size_t)l * S;
  const float* pir = a.Pi + (size_t)r * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    Pl[s] = pil[s];
    Pr[s] = pir[s];
  }
  __syncthreads();
  const float* pbl = a.Pibar + (size_t)l * S;
  const float* pbr = a.Pibar + (size_t)r * S;
  const float* ppar = a.Pi + (size_t)pg * S;
  const float* vk = a.v_k + (size_t)pw * S;
  float* rl = a.rhs + (size_t)l * S;
  float* rr = a.rhs + (size_t)r * S;
  const float rml = a.output_ud ? a.row_max[l] : 0.f;
  const float rmr = a.output_ud ? a.row_max[r] : 0.f;
  float sum_ud_l = 0.f, sum_ud_r = 0.f, abs_l = 0.f, abs_r = 0.f, max_l = 0.f, max_r = 0.f;
  float sum_pD = 0.f, sum_pS = 0.f, sum_mt = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s >= S) break;
    const float ld = a.pD.base[item * a.pD.row_stride + (long long)s * a.pD.elem_stride];
    const float ls = a.pS.base[item * a.pS.row_stride + (long long)s * a.pS.elem_stride];
    const int x = a.c1[s], y = a.c2[s];
    const bool xv = x >= 0 && x < S, yv = y >= 0 && y < S;
    const float d0 = ld + Pl[s] + Pr[s];
    const float d1 = Pl[s] + pbr[s];
    const float d2 = Pr[s] + pbl[s];
    const float d3 = ls + (xv ? Pl[x] : neg_inf()) + (yv ? Pr[y] : neg_inf());
    const float d4 = ls + (xv ? Pr[x] : neg_inf()) + (yv ? Pl[y] : neg_inf());
    const float pp = ppar[s];
    const bool pv = !is_neg_inf(pp);
    const float vv = vk[s];
    const float vd0 = vv * (pv ? ex2(wl + d0 - pp) : 0.f);
    const float vd1 = vv * (pv ? ex2(wl + d1 - pp) : 0.f);
    const float vd2 = vv * (pv ? ex2(wl + d2 - pp) : 0.f);
    const float vd3 = vv * (pv ? ex2(wl + d3 - pp) : 0.f);
    const float vd4 = vv * (pv ? ex2(wl + d4 - pp) : 0.f);
    atomicAdd(rl + s, vd0 + vd1);
    atomicAdd(rr + s, vd0 + vd2);
    if (xv) { atomicAdd(rl + x, vd3); atomicAdd(rr + x, vd4); }
    if (yv) { atomicAdd(rr + y, vd3); atomicAdd(rl + y, vd4); }
    if (a.output_ud) {
      const float mtl = a.mt.base[item_l * a.mt.row_stride + (long long)s * a.mt.elem_stride];
      const float mtr = a.mt.base[item_r * a.mt.row_stride + (long long)s * a.mt.elem_stride];
      const float bl = pbl[s], br = pbr[s];
      const float inv_l = is_neg_inf(bl) ? 0.f : ex2(rml + mtl - bl);
      const float inv_r = is_neg_inf(br) ? 0.f : ex2(rmr + mtr - br);
      const float udl = vd2 * inv_l;
      const float udr = vd1 * inv_r;
      a.pibar_ud[(size_t)i * S + s] = udl;
      a.pibar_ud[(size_t)(N + i) * S + s] = udr;
      sum_ud_l += udl;
      sum_ud_r += udr;
      abs_l += fabsf(udl);
      abs_r += fabsf(udr);
      max_l = fmaxf(max_l, fabsf(udl));
      max_r = fmaxf(max_r, fabsf(udr));
    } else {
      a.grad_Pibar_l[(size_t)i * S + s] = vd2;
      a.grad_Pibar_r[(size_t)i * S + s] = vd1;
    }
    if (a.accum_param) {
      if (a.g_pD.elem_stride) {
        atomicAdd(a.g_pD.base + item * a.g_pD.row_stride + s, vd0);
        atomicAdd(a.g_pS.base + item * a.g_pS.row_stride + s, vd3 + vd4);
      } else {
        sum_pD += vd0;
        sum_pS += vd3 + vd4;
      }
    } else {
      sum_pD += vd0;
      sum_pS += vd3 + vd4;
    }
    if (a.accum_mt) {
      if (a.g_mt.elem_stride) {
        atomicAdd(a.g_mt.base + item_l * a.g_mt.row_stride + s, vd2);
        atomicAdd(a.g_mt.base + item_r * a.g_mt.row_stride + s, vd1);
      } else {
        sum_mt += vd1 + vd2;
      }
    }
  }
  // block reductions for the per-split scalars (all threads participate)
  const bool need_param_sum = !a.accum_param || !a.g_pD.elem_stride;
  if (need_param_sum) {
    const float tpD = block_sum(sum_pD, red);
    const float tpS = block_sum(sum_pS, red);
    if (threadIdx.x == 0) {
      if (a.accum_param) {
        atomicAdd(a.g_pD.base + item * a.g_pD.row_stride, tpD);
        atomicAdd(a.g_pS.base + item * a.g_pS.row_stride, tpS);
      } else {
        a.param_pD[i] = tpD;
        a.param_pS[i] = tpS;
      }
    }
  }
  if (a.accum_mt && !a.g_mt.elem_stride) {
    const float t = block_sum(sum_mt, red);
    if (threadIdx.x == 0) atomicAdd(a.g_mt.base, t);
  }
  if (a.output_ud) {
    const float Al = block_sum(sum_ud_l, red);
    const float Ar = block_sum(sum_ud_r, red);
    const float bl = a.side_thr_enabled ? block_sum(abs_l, red) : block_max(max_l, red);
    const float br = a.side_thr_enabled ? block_sum(abs_r, red) : block_max(max_r, red);
    if (threadIdx.x == 0) {
      a.pibar_A[i] = Al;
      a.pibar_A[N + i] = Ar;
      if (a.side_active) {
        a.side_active[i] = a.side_thr_enabled ? (bl > a.side_thr) : (bl != 0.f);
        a.side_active[N + i] = a.side_thr_enabled ? (br > a.side_thr) : (br != 0.f);
      }
    }
  }
}

__global__ void side_active_kernel(const float* __restrict__ ud, int S, float thr, int thr_enabled,
                                   unsigned char* out) {
  __shared__ float red[64];
  const float* row = ud + (size_t)blockIdx.x * S;
  float mx = 0.f, sm = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float v = fabsf(row[s]);
    mx = fmaxf(mx, v);
    sm += v;
  }
  mx = block_max(mx, red);
  sm = block_sum(sm, red);
  if (threadIdx.x == 0) out[blockIdx.x] = thr_enabled ? (sm > thr) : (mx != 0.f);
}

struct TreeArgs {
  const float* Pi;
  const float* col;
  int use_col;
  float* pibar_ud;  // [2N,S] mutated in place (subtree sums)
  const float* pibar_A;
  const unsigned char* side_active;  // [2N] or null
  const long long* sl;
  const long long* sr;
  const long long* reduce_idx;       // needed with active
  const unsigned char* active;       // [W] or null
  const float* row_max;
  const long long* lv_ptr;
  int n_levels;
  const int* lv_par;
  const int* lv_c1;
  const int* lv_c2;
  float* rhs;
  float* grad_col;  // or null
  int N;
  int S;
};

__global__ void __launch_bounds__(512) pibar_tree_kernel(TreeArgs a) {
  extern __shared__ float sm[];
  const int S = a.S;
  const int row = blockIdx.x;
  const int N = a.N;
  const int i = row < N ? row : row - N;
  if (a.side_active && a.side_active[row] == 0) return;
  if (a.active && a.active[a.reduce_idx[i]] == 0) return;
  const long long child = row < N ? a.sl[i] : a.sr[i];
  float* U = sm;
  float* udrow = a.pibar_ud + (size_t)row * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x) U[s] = udrow[s];
  __syncthreads();
  subtree_sums_levels(U, a.lv_ptr, a.n_levels, a.lv_par, a.lv_c1, a.lv_c2, S);
  const float A = a.pibar_A[row];
  const float rm = a.row_max[child];
  const float rms = safe_max(rm);
  const float* pic = a.Pi + (size_t)child * S;
  float* rc = a.rhs + (size_t)child * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float sub = U[s];
    udrow[s] = sub;
    float wv = pic[s];
    if (a.use_col) wv += a.col[s];
    const float contrib = ex2(wv - rms) * (A - sub);
    atomicAdd(rc + s, contrib);
    if (a.grad_col) atomicAdd(a.grad_col + s, contrib);
  }
}

int vpt_for(int S, int& bd) {
  bd = 512;
  if (S <= 512) bd = ((S + 31) / 32) * 32;
  if (bd < 32) bd = 32;
  int v = (S + bd - 1) / bd;
  if (v <= 1) return 1;
  if (v <= 2) return 2;
  if (v <= 4) return 4;
  if (v <= 8) return 8;
  return 16;
}

int smem_attr(const void* fn, size_t bytes) {
  if (bytes > 48 * 1024 &&
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return KB_ERR_LAUNCH;
  return KB_OK;
}

}  // namespace

extern "C" int kb_active_mask(const float* rhs, long long row_stride, int W, int S, float threshold,
                              int strict_gt, unsigned char* out, void* stream) {
  if (W < 0 || S < 0) return KB_ERR_ARG;
  if (W == 0) return KB_OK;
  int bd = S >= 256 ? 256 : ((S + 31) / 32) * 32;
  if (bd < 32) bd = 32;
  active_mask_kernel<<<W, bd, 0, (cudaStream_t)stream>>>(rhs, row_stride, S, threshold, strict_gt, out);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

namespace {

// Column sums of one wave's six parameter buckets (aw0, aw1, aw2, aw345, aw3, aw4; [W,S], zero on
// inactive rows) added into the caller's gradient targets: the self_loop_grad_targets form of the
// parameter store (ACCUM_GRADS).  32 columns per CTA, ACC_ROWS row strides; every sum in fp64 and in a
// fixed order (the reference adds row by row with atomics).  pd_vector == 0: grad_pD / grad_pS are
// one scalar each; the per-column sums of aw0 / aw345 go to col_tot [2,S] and targets_scalar_kernel
// adds their totals.
struct AccumTargets {
  const float* aw[6];
  float* pD;
  float* pS;
  float* E;
  float* Ebar;
  float* Es1;
  float* Es2;
  float* mt;
  double* col_tot;  // [2,S] when !pd_vector
  int pd_vector;
};

constexpr int ACC_ROWS = 16;

__global__ void __launch_bounds__(32 * ACC_ROWS) accum_targets_kernel(AccumTargets t, int W, int S) {
  __shared__ double part[6][ACC_ROWS][33];
  const int lane = threadIdx.x, ty = threadIdx.y;
  const int s = blockIdx.x * 32 + lane;
  double acc[6] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
  if (s < S) {
    for (int w = ty; w < W; w += ACC_ROWS) {
      const size_t o = (size_t)w * S + s;
#pragma unroll
      for (int k = 0; k < 6; ++k) acc[k] += (double)t.aw[k][o];
    }
  }
#pragma unroll
  for (int k = 0; k < 6; ++k) part[k][ty][lane] = acc[k];
  __syncthreads();
  if (ty == 0 && s < S) {
    double tot[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      double v = 0.0;
      for (int y = 0; y < ACC_ROWS; ++y) v += part[k][y][lane];
      tot[k] = v;
    }
    if (t.pd_vector) {
      t.pD[s] = (float)((double)t.pD[s] + tot[0]);
      t.pS[s] = (float)((double)t.pS[s] + tot[3]);
    } else {
      t.col_tot[s] = tot[0];
      t.col_tot[S + s] = tot[3];
    }
    t.E[s] = (float)((double)t.E[s] + (tot[0] + tot[2]));
    t.Ebar[s] = (float)((double)t.Ebar[s] + tot[1]);
    t.Es1[s] = (float)((double)t.Es1[s] + tot[5]);
    t.Es2[s] = (float)((double)t.Es2[s] + tot[4]);
    t.mt[s] = (float)((double)t.mt[s] + tot[2]);
  }
}

// Scalar pD / pS targets: the totals of col_tot's two rows, in column order, by one warp each.
__global__ void targets_scalar_kernel(const double* __restrict__ col_tot, int S, float* pD, float* pS) {
  const int lane = threadIdx.x & 31, which = threadIdx.x >> 5;
  const double* row = col_tot + (size_t)which * S;
  double v = 0.0;
  for (int s = lane; s < S; s += 32) v += row[s];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  if (lane == 0) {
    float* dst = which == 0 ? pD : pS;
    dst[0] = (float)((double)dst[0] + v);
  }
}

AdjArgs adjoint_args(const float* Pi, const float* Pibar, const float* pibar_row_max, const float* dts,
                     const unsigned char* active, const float* dl, const float* ebar, const float* e,
                     const float* sl1, const float* sl2, int const_mode, const float* col_log_probs,
                     int use_col_weights, const int* node_child1, const int* node_child2, const int* node_parent,
                     const int* jumps, int K, const long long* lv_ptr, int n_levels, const int* lv_par,
                     const int* lv_c1, const int* lv_c2, int use_leaf_index, const int* leaf_state,
                     const float* leaf_logp, int leaf_mode, const float* leaf_term, const long long* item_idx,
                     int ws, int W, int S) {
  AdjArgs a = {};
  a.Pi = Pi; a.Pibar = Pibar; a.row_max = pibar_row_max; a.dts = dts;
  a.active = active; a.dl = dl; a.ebar = ebar; a.e = e; a.sl1 = sl1; a.sl2 = sl2; a.const_mode = const_mode;
  a.col = col_log_probs; a.use_col = use_col_weights; a.c1 = node_child1; a.c2 = node_child2;
  a.parent = node_parent; a.jumps = jumps; a.K = K; a.lv_ptr = lv_ptr; a.n_levels = n_levels;
  a.lv_par = lv_par; a.lv_c1 = lv_c1; a.lv_c2 = lv_c2; a.use_leaf_index = use_leaf_index;
  a.leaf_state = leaf_state; a.leaf_logp = leaf_logp; a.leaf_mode = leaf_mode; a.leaf_term = leaf_term;
  a.item_idx = item_idx; a.ws = ws; a.W = W; a.S = S;
  return a;
}

int launch_adjoint(const AdjArgs& a, void* stream) {
  const int S = a.S;
  int bd;
  const int vpt = vpt_for(S, bd);
  const size_t smem = (size_t)(4 * S + 64) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
#define KB_ADJ_CASE(V)                                                            \
  case V:                                                                         \
    if (smem_attr((const void*)wave_adjoint_kernel<V>, smem)) return KB_ERR_LAUNCH; \
    wave_adjoint_kernel<V><<<a.W, bd, smem, st>>>(a);                             \
    break;
  switch (vpt) {
    KB_ADJ_CASE(1) KB_ADJ_CASE(2) KB_ADJ_CASE(4) KB_ADJ_CASE(8) KB_ADJ_CASE(16)
    default: return KB_ERR_SIZE;
  }
#undef KB_ADJ_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

}  // namespace

extern "C" int kb_wave_adjoint(const float* Pi, const float* Pibar, const float* pibar_row_max, const float* dts,
                               const float* rhs, long long rhs_row_stride, const unsigned char* active,
                               const float* dl, const float* ebar, const float* e, const float* sl1,
                               const float* sl2, int const_mode, const float* col_log_probs, int use_col_weights,
                               const int* node_child1, const int* node_child2, const int* node_parent,
                               const int* jumps, int K, const long long* lv_ptr, int n_levels,
                               const int* lv_par, const int* lv_c1, const int* lv_c2, int use_leaf_index,
                               const int* leaf_state, const float* leaf_logp, int leaf_mode,
                               const float* leaf_term, const long long* item_idx, int neumann_terms,
                               const float* initial_v, long long initial_v_row_stride, float* grad_col,
                               float* v_k, float* aw0, float* aw1, float* aw2, float* aw345, float* aw3, float* aw4,
                               float* last_relres, int ws, int W, int S, void* stream) {
  if (S <= 0 || W < 0 || K < 0 || neumann_terms < 0 || n_levels < 0) return KB_ERR_ARG;
  if (initial_v && last_relres) return KB_ERR_ARG;  // no last increment for a warm-started solve
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (W == 0) return KB_OK;
  AdjArgs a = adjoint_args(Pi, Pibar, pibar_row_max, dts, active, dl, ebar, e, sl1, sl2, const_mode, col_log_probs,
                           use_col_weights, node_child1, node_child2, node_parent, jumps, K, lv_ptr, n_levels,
                           lv_par, lv_c1, lv_c2, use_leaf_index, leaf_state, leaf_logp, leaf_mode, leaf_term,
                           item_idx, ws, W, S);
  a.rhs = rhs; a.rhs_rs = rhs_row_stride;
  a.neumann_terms = neumann_terms; a.grad_col = grad_col; a.v_k = v_k;
  a.init_v = initial_v; a.init_rs = initial_v_row_stride;
  a.aw0 = aw0; a.aw1 = aw1; a.aw2 = aw2; a.aw345 = aw345; a.aw3 = aw3; a.aw4 = aw4;
  a.last_relres = last_relres;
  return launch_adjoint(a, stream);
}

extern "C" int kb_wave_adjoint_apply(const float* Pi, const float* Pibar, const float* pibar_row_max,
                                     const float* dts, const unsigned char* active, const float* dl,
                                     const float* ebar, const float* e, const float* sl1, const float* sl2,
                                     int const_mode, const float* col_log_probs, int use_col_weights,
                                     const int* node_child1, const int* node_child2, const int* node_parent,
                                     const int* jumps, int K, const long long* lv_ptr, int n_levels,
                                     const int* lv_par, const int* lv_c1, const int* lv_c2, int use_leaf_index,
                                     const int* leaf_state, const float* leaf_logp, int leaf_mode,
                                     const float* leaf_term, const long long* item_idx, const float* x,
                                     long long x_row_stride, float* y, int ws, int W, int S, void* stream) {
  if (S <= 0 || W < 0 || K < 0 || n_levels < 0 || !x || !y) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (W == 0) return KB_OK;
  AdjArgs a = adjoint_args(Pi, Pibar, pibar_row_max, dts, active, dl, ebar, e, sl1, sl2, const_mode, col_log_probs,
                           use_col_weights, node_child1, node_child2, node_parent, jumps, K, lv_ptr, n_levels,
                           lv_par, lv_c1, lv_c2, use_leaf_index, leaf_state, leaf_logp, leaf_mode, leaf_term,
                           item_idx, ws, W, S);
  a.apply_in = x; a.apply_rs = x_row_stride; a.apply_out = y;
  return launch_adjoint(a, stream);
}

extern "C" int kb_dts_adjoint(const float* Pi, const float* Pibar, const float* v_k, const unsigned char* active,
                              const long long* sl, const long long* sr, const long long* reduce_idx,
                              const float* wlsp, const float* log_pD, long long pD_row_stride, int pD_elem_stride,
                              const float* log_pS, long long pS_row_stride, int pS_elem_stride,
                              const long long* item_idx, const int* node_child1, const int* node_child2,
                              float* accumulated_rhs, int output_ud, float* pibar_ud, float* pibar_A,
                              unsigned char* side_active, float side_threshold, int side_threshold_enabled,
                              int skip_inactive_zero, float* grad_Pibar_l, float* grad_Pibar_r, int accum_param,
                              float* grad_log_pD, float* grad_log_pS, long long gp_row_stride, int gp_elem_stride,
                              float* param_pD, float* param_pS, int accum_mt, float* grad_mt,
                              long long gmt_row_stride, int gmt_elem_stride, const float* mt,
                              long long mt_row_stride, int mt_elem_stride, const float* pibar_row_max, int ws,
                              int N, int S, void* stream) {
  if (S <= 0 || N < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (N == 0) return KB_OK;
  DtsAdjArgs a;
  a.Pi = Pi; a.Pibar = Pibar; a.v_k = v_k; a.active = active; a.sl = sl; a.sr = sr; a.reduce_idx = reduce_idx;
  a.wlsp = wlsp;
  a.pD = ParamRef{log_pD, pD_row_stride, pD_elem_stride};
  a.pS = ParamRef{log_pS, pS_row_stride, pS_elem_stride};
  a.item_idx = item_idx; a.c1 = node_child1; a.c2 = node_child2; a.rhs = accumulated_rhs;
  a.output_ud = output_ud; a.pibar_ud = pibar_ud; a.pibar_A = pibar_A; a.side_active = side_active;
  a.side_thr = side_threshold; a.side_thr_enabled = side_threshold_enabled;
  a.skip_inactive_zero = skip_inactive_zero; a.grad_Pibar_l = grad_Pibar_l; a.grad_Pibar_r = grad_Pibar_r;
  a.accum_param = accum_param;
  a.g_pD = GradRef{grad_log_pD, gp_row_stride, gp_elem_stride};
  a.g_pS = GradRef{grad_log_pS, gp_row_stride, gp_elem_stride};
  a.param_pD = param_pD; a.param_pS = param_pS; a.accum_mt = accum_mt;
  a.g_mt = GradRef{grad_mt, gmt_row_stride, gmt_elem_stride};
  a.mt = ParamRef{mt, mt_row_stride, mt_elem_stride};
  a.row_max = pibar_row_max; a.ws = ws; a.N = N; a.S = S;
  int bd;
  const int vpt = vpt_for(S, bd);
  const size_t smem = (size_t)(2 * S + 64) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
#define KB_DADJ_CASE(V)                                                          \
  case V:                                                                        \
    if (smem_attr((const void*)dts_adjoint_kernel<V>, smem)) return KB_ERR_LAUNCH; \
    dts_adjoint_kernel<V><<<N, bd, smem, st>>>(a);                               \
    break;
  switch (vpt) {
    KB_DADJ_CASE(1) KB_DADJ_CASE(2) KB_DADJ_CASE(4) KB_DADJ_CASE(8) KB_DADJ_CASE(16)
    default: return KB_ERR_SIZE;
  }
#undef KB_DADJ_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_side_active(const float* pibar_ud, int rows, int S, float threshold, int threshold_enabled,
                              unsigned char* out, void* stream) {
  if (rows < 0 || S <= 0) return KB_ERR_ARG;
  if (rows == 0) return KB_OK;
  int bd = S >= 256 ? 256 : ((S + 31) / 32) * 32;
  side_active_kernel<<<rows, bd, 0, (cudaStream_t)stream>>>(pibar_ud, S, threshold, threshold_enabled, out);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_pibar_vjp_tree(const float* Pi, const float* col_log_probs, int use_col_weights, float* pibar_ud,
                                 const float* pibar_A, const unsigned char* side_active, const long long* sl,
                                 const long long* sr, const long long* reduce_idx, const unsigned char* active,
                                 const float* pibar_row_max, const long long* lv_ptr, int n_levels,
                                 const int* lv_par, const int* lv_c1, const int* lv_c2, float* accumulated_rhs,
                                 float* grad_col, int N, int S, void* stream) {
  if (S <= 0 || N < 0 || n_levels < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (N == 0) return KB_OK;
  TreeArgs a;
  a.Pi = Pi; a.col = col_log_probs; a.use_col = use_col_weights; a.pibar_ud = pibar_ud; a.pibar_A = pibar_A;
  a.side_active = side_active; a.sl = sl; a.sr = sr; a.reduce_idx = reduce_idx; a.active = active;
  a.row_max = pibar_row_max; a.lv_ptr = lv_ptr; a.n_levels = n_levels; a.lv_par = lv_par; a.lv_c1 = lv_c1;
  a.lv_c2 = lv_c2; a.rhs = accumulated_rhs; a.grad_col = grad_col; a.N = N; a.S = S;
  int bd = S >= 512 ? 512 : ((S + 31) / 32) * 32;
  if (bd < 32) bd = 32;
  const size_t smem = (size_t)S * sizeof(float);
  if (smem_attr((const void*)pibar_tree_kernel, smem)) return KB_ERR_LAUNCH;
  pibar_tree_kernel<<<2 * N, bd, smem, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_wave_adjoint_accum_targets(const float* aw0, const float* aw1, const float* aw2,
                                             const float* aw345, const float* aw3, const float* aw4, int W, int S,
                                             float* grad_log_pD, float* grad_log_pS, int param_grad_vector,
                                             float* grad_E, float* grad_Ebar, float* grad_E_s1, float* grad_E_s2,
                                             float* grad_mt, double* col_tot, void* stream) {
  if (W < 0 || S <= 0 || !aw0 || !aw1 || !aw2 || !aw345 || !aw3 || !aw4) return KB_ERR_ARG;
  if (!grad_log_pD || !grad_log_pS || !grad_E || !grad_Ebar || !grad_E_s1 || !grad_E_s2 || !grad_mt)
    return KB_ERR_ARG;
  if (!param_grad_vector && !col_tot) return KB_ERR_ARG;
  if (W == 0) return KB_OK;
  AccumTargets t;
  t.aw[0] = aw0; t.aw[1] = aw1; t.aw[2] = aw2; t.aw[3] = aw345; t.aw[4] = aw3; t.aw[5] = aw4;
  t.pD = grad_log_pD; t.pS = grad_log_pS; t.E = grad_E; t.Ebar = grad_Ebar; t.Es1 = grad_E_s1;
  t.Es2 = grad_E_s2; t.mt = grad_mt; t.col_tot = col_tot; t.pd_vector = param_grad_vector;
  cudaStream_t st = (cudaStream_t)stream;
  accum_targets_kernel<<<(S + 31) / 32, dim3(32, ACC_ROWS), 0, st>>>(t, W, S);
  if (cudaGetLastError() != cudaSuccess) return KB_ERR_LAUNCH;
  if (!param_grad_vector) targets_scalar_kernel<<<1, 64, 0, st>>>(col_tot, S, grad_log_pD, grad_log_pS);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
