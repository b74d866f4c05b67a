// Column-weight normaliser of the parameter extraction and its VJP.
//
// Restates kbench/core/parameters/extract_parameters.py:41-65 (reference):
//   mass[s] = sum over the ancestor-or-self path of s (at most max_depth nodes, self first) of
//             2^clp[a], added one node at a time from s upwards;
//   norm[s] = -log2(max(1 - mass[s], FLT_MIN)) where 1 - mass[s] > 0, else -inf.
// The reference runs this as a loop of max_depth rounds of gathers over all S columns (about ten
// tensor launches per round, forward and again backward); here each is ONE launch of one CTA
// with the parent table and 2^clp resident in shared memory.  Every thread walks its columns'
// root paths itself, so mass is summed in the reference's order (self, parent, grandparent, ...).
// The VJP is   grad_clp[a] = 2^clp[a] ln2 * sum over the subtree of a of g[s] / ((1 - mass[s]) ln2)
// (zero where the forward took the -inf or the clamped branch), with the subtree sums taken
// bottom-up over the compact levels -- deterministic, no atomics.
#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

using namespace kb;

constexpr float kLn2 = 0.6931471805599453f;
constexpr float kTiny = 1.17549435e-38f;  // FLT_MIN, torch.finfo(float32).tiny

__device__ __forceinline__ float path_mass(const int* par, const float* prob, int s, int S, int max_depth) {
  float mass = 0.f;
  int cur = s;
  for (int d = 0; d < max_depth; ++d) {
    if (cur < 0 || cur >= S) break;
    mass = mass + prob[cur];
    cur = par[cur];
  }
  return mass;
}

__device__ __forceinline__ void load_tables(const float* clp, const int* parent, int* par, float* prob, int S) {
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    par[s] = parent[s];
    prob[s] = exp2f(clp[s]);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(1024, 1) col_normalizer_kernel(const float* __restrict__ clp,
                                                                  const int* __restrict__ parent, int max_depth,
                                                                  int S, float* __restrict__ norm) {
  extern __shared__ float sm[];
  float* prob = sm;
  int* par = reinterpret_cast<int*>(sm + S);
  load_tables(clp, parent, par, prob, S);
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float vm = 1.0f - path_mass(par, prob, s, S, max_depth);
    norm[s] = vm > 0.f ? -log2f(fmaxf(vm, kTiny)) : neg_inf();
  }
}

__global__ void __launch_bounds__(1024, 1) col_normalizer_vjp_kernel(
    const float* __restrict__ clp, const int* __restrict__ parent, int max_depth, const long long* lv_ptr,
    int n_levels, const int* lv_par, const int* lv_c1, const int* lv_c2, const float* __restrict__ g_norm,
    float* __restrict__ grad_clp, int S) {
  extern __shared__ float sm[];
  float* prob = sm;
  int* par = reinterpret_cast<int*>(sm + S);
  float* acc = sm + 2 * S;
  load_tables(clp, parent, par, prob, S);
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float vm = 1.0f - path_mass(par, prob, s, S, max_depth);
    acc[s] = (vm > 0.f && vm >= kTiny) ? g_norm[s] / (vm * kLn2) : 0.f;
  }
  __syncthreads();
  subtree_sums_levels(acc, lv_ptr, n_levels, lv_par, lv_c1, lv_c2, S);
  for (int s = threadIdx.x; s < S; s += blockDim.x) grad_clp[s] = acc[s] * prob[s] * kLn2;
}

int block_for(int S) {
  int b = ((S + 31) / 32) * 32;
  return b > 1024 ? 1024 : (b < 32 ? 32 : b);
}

}  // namespace

extern "C" int kb_col_normalizer(const float* col_log_probs, const int* node_parent, int max_ancestor_depth, int S,
                                 float* norm_out, void* stream) {
  if (S <= 0 || max_ancestor_depth < 0 || !col_log_probs || !node_parent || !norm_out) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  const int depth = max_ancestor_depth < 1 ? 1 : max_ancestor_depth;
  const size_t smem = (size_t)2 * S * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute((const void*)col_normalizer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return KB_ERR_LAUNCH;
  col_normalizer_kernel<<<1, block_for(S), smem, (cudaStream_t)stream>>>(col_log_probs, node_parent, depth, S,
                                                                         norm_out);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_col_normalizer_vjp(const float* col_log_probs, const int* node_parent, int max_ancestor_depth,
                                     const long long* lv_ptr, int n_levels, const int* lv_par, const int* lv_c1,
                                     const int* lv_c2, const float* g_norm, float* grad_col_log_probs, int S,
                                     void* stream) {
  if (S <= 0 || max_ancestor_depth < 0 || n_levels < 0 || !col_log_probs || !node_parent || !g_norm ||
      !grad_col_log_probs)
    return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  const int depth = max_ancestor_depth < 1 ? 1 : max_ancestor_depth;
  const size_t smem = (size_t)3 * S * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute((const void*)col_normalizer_vjp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return KB_ERR_LAUNCH;
  col_normalizer_vjp_kernel<<<1, block_for(S), smem, (cudaStream_t)stream>>>(
      col_log_probs, node_parent, depth, lv_ptr, n_levels, lv_par, lv_c1, lv_c2, g_norm, grad_col_log_probs, S);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
