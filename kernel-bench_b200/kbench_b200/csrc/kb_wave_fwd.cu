// Forward wave kernels: one Jacobi sweep of a wave (drop-in), the leaf seed, and the fused
// sweep that runs all pi_iters iterations of a row in one launch.
//
// Restates kbench/core/kernels/wave_step.py (reference): _wave_step_kernel (pristine
// experiments/pristine_kernels/wave_step.py:92-220, optimized :848-985) and
// _leaf_initial_wave_step_kernel (:223-310), driven the way kbench/core/inference/forward.py:60-115
// drives them.
//
// B200 design: one CTA per row with the row resident in shared memory; the ancestor-or-self path
// sum of 2^(Pi - rowmax) is a shared-memory pointer-doubling scan over precomputed jump tables
// (ceil(log2 depth) barriers); the row max/sum are warp-shuffle reductions; ex2/lg2 run on MUFU.
// The fused sweep reads its input row once, iterates entirely on chip and writes only the final
// Pi row, the final Pibar row and the row max -- the per-iteration HBM round trips of the
// reference (one read + one write of the row per iteration) disappear.
#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

using namespace kb;

struct WaveConsts {
  const float* mc;
  const float* dl;
  const float* ebar;
  const float* e;
  const float* sl1;
  const float* sl2;
  long long crs;  // row stride of the constant tensors (0: one shared row)
  const float* col;
  int use_col;
  const int* c1;
  const int* c2;
  const int* jumps;
  int K;
  int S;
  const float* leaf_logp;  // [G,S] addressed item*S + s
  const long long* item_idx;
  const int* leaf_state;  // [C]
  const int* sub_start;   // leaf seed only
  const int* sub_end;
};

// Pibar path sums of the row held in P: returns the path-sum buffer; row_max/row_sum by ref.
__device__ __forceinline__ const float* row_pathsums(const float* P, float* X, float* Y, float* red,
                                                     const WaveConsts& c, float& row_max, float& row_sum) {
  const int S = c.S;
  float m = neg_inf();
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = P[s];
    if (c.use_col) w += c.col[s];
    m = fmaxf(m, w);
  }
  row_max = block_max(m, red);
  const float rms = safe_max(row_max);
  float sum = 0.f;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    float w = P[s];
    if (c.use_col) w += c.col[s];
    const float x = ex2(w - rms);
    X[s] = x;
    sum += x;
  }
  row_sum = block_sum(sum, red);
  return ancestor_sum_doubling(X, Y, c.jumps, c.K, S);
}

// One sweep of the row in P; new values land in out[] (thread-owned columns).
template <int VPT>
__device__ __forceinline__ void wave_iter(const float* P, float* X, float* Y, float* red, const WaveConsts& c,
                                          size_t cb, int leaf, float leafv, const float* dv, float* out) {
  const int S = c.S;
  float row_max, row_sum;
  const float* anc = row_pathsums(P, X, Y, red, c, row_max, row_sum);
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
    const float t3 = (a >= 0 && a < S) ? c.sl1[cb + s] + P[a] : neg_inf();
    const float t4 = (b >= 0 && b < S) ? c.sl2[cb + s] + P[b] : neg_inf();
    const float t5 = (s == leaf) ? leafv : neg_inf();
    const float td = dv ? dv[k] : neg_inf();
    float m = fmaxf(fmaxf(fmaxf(t0, t1), fmaxf(t2, t3)), fmaxf(fmaxf(t4, t5), td));
    const float ms = safe_max(m);
    float sum = (ex2(t0 - ms) + ex2(t1 - ms) + ex2(t2 - ms)) + (ex2(t3 - ms) + ex2(t4 - ms) + ex2(t5 - ms));
    if (dv) sum += ex2(td - ms);
    out[k] = lg2(sum) + m;
  }
}

// Final Pibar of the row in P: writes pibar_row[s] and returns the row max.
__device__ __forceinline__ float write_final_pibar(const float* P, float* X, float* Y, float* red,
                                                   const WaveConsts& c, size_t cb, float* pibar_row) {
  const int S = c.S;
  float row_max, row_sum;
  const float* anc = row_pathsums(P, X, Y, red, c, row_max, row_sum);
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const float denom = row_sum - anc[s];
    pibar_row[s] = denom > 0.f ? lg2(denom) + row_max + c.mc[cb + s] : neg_inf();
  }
  return row_max;
}

struct StepArgs {
  WaveConsts c;
  const float* pi_in;
  long long pi_ws;  // row of pi_in holding wave row 0
  float* pi_out_rows;
  float* pibar;     // full [C,S]
  float* pibar_row_max;
  float* residual;  // [C] or null
  const float* dts; // [W,S] or null
  int ws;
  int W;
  int use_leaf;
  int store_final;
};

template <int VPT>
__global__ void __launch_bounds__(512) wave_step_kernel(StepArgs a) {
  extern __shared__ float sm[];
  const WaveConsts& c = a.c;
  const int S = c.S;
  float* P = sm;
  float* X = sm + S;
  float* Y = sm + 2 * S;
  float* red = sm + 3 * S;
  const int w = blockIdx.x;
  const long long rg = (long long)a.ws + w;
  const long long item = c.item_idx[rg];
  const size_t cb = (size_t)(item * c.crs);
  const float* src = a.pi_in + (size_t)(a.pi_ws + w) * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x) P[s] = src[s];
  int leaf = -1;
  float leafv = neg_inf();
  if (a.use_leaf) {
    leaf = c.leaf_state[rg];
    if (leaf >= 0 && leaf < S) leafv = c.leaf_logp[(size_t)item * S + leaf];
    else leaf = -1;
  }
  float dv[VPT];
  const float* dvp = nullptr;
  if (a.dts) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      dv[k] = s < S ? a.dts[(size_t)w * S + s] : neg_inf();
    }
    dvp = dv;
  }
  __syncthreads();
  float nv[VPT];
  wave_iter<VPT>(P, X, Y, red, c, cb, leaf, leafv, dvp, nv);
  if (a.residual) {
    float d = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S && !is_neg_inf(nv[k]) && !is_neg_inf(P[s])) d = fmaxf(d, fabsf(nv[k] - P[s]));
    }
    d = block_max(d, red);
    if (threadIdx.x == 0) a.residual[rg] = d;
  }
  float* orow = a.pi_out_rows + (size_t)w * S;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) orow[s] = nv[k];
  }
  if (a.store_final) {
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) P[s] = nv[k];
    }
    __syncthreads();
    const float rm = write_final_pibar(P, X, Y, red, c, cb, a.pibar + (size_t)rg * S);
    if (threadIdx.x == 0) a.pibar_row_max[rg] = rm;
  }
}

// Leaf seed of one element (pristine wave_step.py:223-310).
__device__ __forceinline__ float leaf_seed_value(const WaveConsts& c, size_t cb, long long item, int leaf, int s) {
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

__global__ void leaf_initial_kernel(WaveConsts c, float* pi_out_rows, int ws) {
  const int w = blockIdx.x;
  const int S = c.S;
  const long long rg = (long long)ws + w;
  const long long item = c.item_idx[rg];
  const size_t cb = (size_t)(item * c.crs);
  const int leaf = c.leaf_state[rg];
  float* orow = pi_out_rows + (size_t)w * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x)
    orow[s] = (leaf >= 0 && leaf < S) ? leaf_seed_value(c, cb, item, leaf, s) : neg_inf();
}

struct SweepArgs {
  WaveConsts c;
  const int* rows;      // global row id per CTA
  const float* dts;     // [n_rows, S] aligned with rows (split rows), may be null if all leaves
  float* pi;            // [C,S] final Pi rows
  float* pibar;         // [C,S] final Pibar rows
  float* pibar_row_max; // [C]
  float* residual;      // [C] or null: max |Pi_last - Pi_prev| over finite entries
  int n_rows;
  int pi_iters;
};

template <int VPT>
__global__ void __launch_bounds__(512) wave_sweep_kernel(SweepArgs a) {
  extern __shared__ float sm[];
  const WaveConsts& c = a.c;
  const int S = c.S;
  float* P = sm;
  float* X = sm + S;
  float* Y = sm + 2 * S;
  float* red = sm + 3 * S;
  const int b = blockIdx.x;
  const long long rg = a.rows[b];
  const long long item = c.item_idx[rg];
  const size_t cb = (size_t)(item * c.crs);
  const int leaf_raw = c.leaf_state[rg];
  const bool is_leaf = leaf_raw >= 0 && leaf_raw < S;
  const int leaf = is_leaf ? leaf_raw : -1;
  const float leafv = is_leaf ? c.leaf_logp[(size_t)item * S + leaf] : neg_inf();
  float dv[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    float v = neg_inf();
    if (s < S) v = is_leaf ? leaf_seed_value(c, cb, item, leaf, s) : a.dts[(size_t)b * S + s];
    dv[k] = v;
    if (s < S) P[s] = v;
  }
  __syncthreads();
  float nv[VPT];
  for (int it = 1; it < a.pi_iters; ++it) {
    wave_iter<VPT>(P, X, Y, red, c, cb, leaf, leafv, is_leaf ? nullptr : dv, nv);
    if (a.residual && it == a.pi_iters - 1) {
      float d = 0.f;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int s = threadIdx.x + k * blockDim.x;
        if (s < S && !is_neg_inf(nv[k]) && !is_neg_inf(P[s])) d = fmaxf(d, fabsf(nv[k] - P[s]));
      }
      d = block_max(d, red);
      if (threadIdx.x == 0) a.residual[rg] = d;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s < S) P[s] = nv[k];
    }
    __syncthreads();
  }
  float* prow = a.pi + (size_t)rg * S;
  for (int s = threadIdx.x; s < S; s += blockDim.x) prow[s] = P[s];
  const float rm = write_final_pibar(P, X, Y, red, c, cb, a.pibar + (size_t)rg * S);
  if (threadIdx.x == 0) a.pibar_row_max[rg] = rm;
}

int pick_block(int S, int& vpt) {
  int bd = 512;
  if (S <= 512) bd = ((S + 31) / 32) * 32;
  if (bd < 32) bd = 32;
  vpt = (S + bd - 1) / bd;
  if (vpt <= 1) vpt = 1;
  else if (vpt <= 2) vpt = 2;
  else if (vpt <= 4) vpt = 4;
  else if (vpt <= 8) vpt = 8;
  else vpt = 16;
  return bd;
}

template <typename Kern>
int launch_rows(Kern kern, int grid, int bd, size_t smem, cudaStream_t st) {
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return KB_ERR_LAUNCH;
  }
  return KB_OK;
}

WaveConsts make_consts(const float* mc, const float* dl, const float* ebar, const float* e, const float* sl1,
                       const float* sl2, long long crs, const float* col, int use_col, const int* c1,
                       const int* c2, const int* jumps, int K, int S, const float* leaf_logp,
                       const long long* item_idx, const int* leaf_state, const int* sub_start,
                       const int* sub_end) {
  WaveConsts c;
  c.mc = mc; c.dl = dl; c.ebar = ebar; c.e = e; c.sl1 = sl1; c.sl2 = sl2; c.crs = crs;
  c.col = col; c.use_col = use_col; c.c1 = c1; c.c2 = c2; c.jumps = jumps; c.K = K; c.S = S;
  c.leaf_logp = leaf_logp; c.item_idx = item_idx; c.leaf_state = leaf_state;
  c.sub_start = sub_start; c.sub_end = sub_end;
  return c;
}

}  // namespace

extern "C" int kb_wave_step(const float* pi_in, long long pi_ws, float* pi_out_rows, float* pibar,
                            float* pibar_row_max, float* residual, const float* dts, const float* mc,
                            const float* dl, const float* ebar, const float* e, const float* sl1,
                            const float* sl2, long long const_row_stride, const float* col_log_probs,
                            int use_col_weights, const int* node_child1, const int* node_child2,
                            const int* jumps, int K, const int* leaf_state, const float* leaf_logp,
                            const long long* item_idx, int use_leaf, int store_final, int ws, int W, int S,
                            void* stream) {
  if (S <= 0 || W < 0 || K < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (W == 0) return KB_OK;
  StepArgs a;
  a.c = make_consts(mc, dl, ebar, e, sl1, sl2, const_row_stride, col_log_probs, use_col_weights, node_child1,
                    node_child2, jumps, K, S, leaf_logp, item_idx, leaf_state, nullptr, nullptr);
  a.pi_in = pi_in; a.pi_ws = pi_ws; a.pi_out_rows = pi_out_rows; a.pibar = pibar;
  a.pibar_row_max = pibar_row_max; a.residual = residual; a.dts = dts; a.ws = ws; a.W = W;
  a.use_leaf = use_leaf; a.store_final = store_final;
  int vpt;
  const int bd = pick_block(S, vpt);
  const size_t smem = (size_t)(3 * S + 64) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
#define KB_STEP_CASE(V)                                                         \
  case V:                                                                       \
    if (launch_rows(wave_step_kernel<V>, W, bd, smem, st)) return KB_ERR_LAUNCH; \
    wave_step_kernel<V><<<W, bd, smem, st>>>(a);                                \
    break;
  switch (vpt) {
    KB_STEP_CASE(1) KB_STEP_CASE(2) KB_STEP_CASE(4) KB_STEP_CASE(8) KB_STEP_CASE(16)
    default: return KB_ERR_SIZE;
  }
#undef KB_STEP_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_leaf_initial(float* pi_out_rows, const float* mc, const float* dl, const float* ebar,
                               const float* e, const float* sl1, const float* sl2, long long const_row_stride,
                               const float* col_log_probs, int use_col_weights, const int* node_child1,
                               const int* node_child2, const int* node_subtree_start,
                               const int* node_subtree_end, const int* leaf_state, const float* leaf_logp,
                               const long long* item_idx, int ws, int W, int S, void* stream) {
  if (S <= 0 || W < 0) return KB_ERR_ARG;
  if (W == 0) return KB_OK;
  WaveConsts c = make_consts(mc, dl, ebar, e, sl1, sl2, const_row_stride, col_log_probs, use_col_weights,
                             node_child1, node_child2, nullptr, 0, S, leaf_logp, item_idx, leaf_state,
                             node_subtree_start, node_subtree_end);
  int bd = S < 256 ? ((S + 31) / 32) * 32 : 256;
  leaf_initial_kernel<<<W, bd, 0, (cudaStream_t)stream>>>(c, pi_out_rows, ws);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}

extern "C" int kb_wave_sweep(const int* rows, int n_rows, const float* dts, float* pi, float* pibar,
                             float* pibar_row_max, float* residual, const float* mc, const float* dl,
                             const float* ebar, const float* e, const float* sl1, const float* sl2,
                             long long const_row_stride, const float* col_log_probs, int use_col_weights,
                             const int* node_child1, const int* node_child2, const int* node_subtree_start,
                             const int* node_subtree_end, const int* jumps, int K, const int* leaf_state,
                             const float* leaf_logp, const long long* item_idx, int pi_iters, int S,
                             void* stream) {
  if (S <= 0 || n_rows < 0 || K < 0 || pi_iters < 2) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  if (n_rows == 0) return KB_OK;
  SweepArgs a;
  a.c = make_consts(mc, dl, ebar, e, sl1, sl2, const_row_stride, col_log_probs, use_col_weights, node_child1,
                    node_child2, jumps, K, S, leaf_logp, item_idx, leaf_state, node_subtree_start,
                    node_subtree_end);
  a.rows = rows; a.dts = dts; a.pi = pi; a.pibar = pibar; a.pibar_row_max = pibar_row_max;
  a.residual = residual; a.n_rows = n_rows; a.pi_iters = pi_iters;
  int vpt;
  const int bd = pick_block(S, vpt);
  const size_t smem = (size_t)(3 * S + 64) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
#define KB_SWEEP_CASE(V)                                                           \
  case V:                                                                          \
    if (launch_rows(wave_sweep_kernel<V>, n_rows, bd, smem, st)) return KB_ERR_LAUNCH; \
    wave_sweep_kernel<V><<<n_rows, bd, smem, st>>>(a);                             \
    break;
  switch (vpt) {
    KB_SWEEP_CASE(1) KB_SWEEP_CASE(2) KB_SWEEP_CASE(4) KB_SWEEP_CASE(8) KB_SWEEP_CASE(16)
    default: return KB_ERR_SIZE;
  }
#undef KB_SWEEP_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
