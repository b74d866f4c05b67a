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
