// Split reduction (dts): per parent row, the log2-sum-exp2 of five terms over all of its splits.
//
// Restates kbench/core/kernels/dts_fused.py (reference): _dts_eq1_kernel (:18-62) for
// single-split parents and the two-stage tiled online LSE _dts_ge2_stage1/2 (:65-168) for
// multi-split parents, with the wrapper compute_dts_forward (:171-231).
//
// B200 design: one CTA per parent row (not per split and S-tile): it walks the parent's splits
// in order with a register-resident online LSE, so there are no partial-max/partial-sum buffers
// and no second pass; each child Pi row is staged once in shared memory for the two
// speciation gathers Pi[child][c1(s)], Pi[child][c2(s)].
#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

using namespace kb;

struct DtsArgs {
  const float* Pi;
  const float* Pibar;
  const long long* sl;
  const long long* sr;
  const int* c1;
  const int* c2;
  const float* log_pD;
  const float* log_pS;
  long long prs;  // parameter row stride (0: one shared row)
  const long long* item_idx;
  long long item_offset;
  const float* lsp;
  const long long* eq1_reduce_idx;
  int n_eq1;
  const long long* ge2_ptr;
  const long long* ge2_parent_ids;
  int n_ge2;
  const unsigned char* active;
  float* out;  // [W,S]
  const long long* out_row;  // optional: output row per parent (engine layout); null -> parent
  int S;
};

template <int VPT>
__global__ void __launch_bounds__(512) dts_forward_kernel(DtsArgs a) {
  extern __shared__ float sm[];
  const int S = a.S;
  float* Pl = sm;
  float* Pr = sm + S;
  const int g = blockIdx.x;
  long long parent, i0, i1;
  if (g < a.n_eq1) {
    parent = a.eq1_reduce_idx[g];
    i0 = g;
    i1 = g + 1;
  } else {
    const int h = g - a.n_eq1;
    parent = a.ge2_parent_ids[h];
    i0 = a.n_eq1 + a.ge2_ptr[h];
    i1 = a.n_eq1 + a.ge2_ptr[h + 1];
  }
  if (a.active && a.active[parent] == 0) return;  // row stays -inf (pre-filled)
  const long long item = a.item_idx[a.item_offset + parent];
  const size_t pb = (size_t)(item * a.prs);
  float m[VPT], acc[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) { m[k] = neg_inf(); acc[k] = 0.f; }
  for (long long i = i0; i < i1; ++i) {
    const long long l = a.sl[i], r = a.sr[i];
    const float* pil = a.Pi + (size_t)l * S;
    const float* pir = a.Pi + (size_t)r * S;
    const float* pbl = a.Pibar + (size_t)l * S;
    const float* pbr = a.Pibar + (size_t)r * S;
    __syncthreads();
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      Pl[s] = pil[s];
      Pr[s] = pir[s];
    }
    __syncthreads();
    const float lsp = a.lsp[i];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int s = threadIdx.x + k * blockDim.x;
      if (s >= S) break;
      const float ld = a.log_pD[pb + s];
      const float ls = a.log_pS[pb + s];
      const int x = a.c1[s], y = a.c2[s];
      const bool xv = x < S, yv = y < S;
      const float v0 = lsp + ld + Pl[s] + Pr[s];
      const float v1 = lsp + Pl[s] + pbr[s];
      const float v2 = lsp + Pr[s] + pbl[s];
      const float v3 = lsp + ls + (xv ? Pl[x] : neg_inf()) + (yv ? Pr[y] : neg_inf());
      const float v4 = lsp + ls + (xv ? Pr[x] : neg_inf()) + (yv ? Pl[y] : neg_inf());
      const float sm_ = fmaxf(fmaxf(fmaxf(v0, v1), fmaxf(v2, v3)), v4);
      const float sms = safe_max(sm_);
      const float ssum = ex2(v0 - sms) + ex2(v1 - sms) + ex2(v2 - sms) + ex2(v3 - sms) + ex2(v4 - sms);
      const float nm = fmaxf(m[k], sm_);
      const float nms = safe_max(nm);
      acc[k] = (is_neg_inf(m[k]) ? 0.f : acc[k] * ex2(m[k] - nms)) + ssum * ex2(sms - nms);
      m[k] = nm;
    }
  }
  const long long orow = a.out_row ? a.out_row[parent] : parent;
  float* o = a.out + (size_t)orow * S;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int s = threadIdx.x + k * blockDim.x;
    if (s < S) o[s] = lg2(acc[k]) + m[k];
  }
}

}  // namespace

extern "C" int kb_dts_forward(const float* Pi, const float* Pibar, const long long* sl, const long long* sr,
                              const int* node_child1, const int* node_child2, const float* log_pD,
                              const float* log_pS, long long param_row_stride, const long long* item_idx,
                              long long item_offset, const float* log_split_probs,
                              const long long* eq1_reduce_idx, int n_eq1, const long long* ge2_ptr,
                              const long long* ge2_parent_ids, int n_ge2, const unsigned char* active_rows,
                              float* out, const long long* out_row, int S, void* stream) {
  if (S <= 0 || n_eq1 < 0 || n_ge2 < 0) return KB_ERR_ARG;
  if (S > KB_MAX_S) return KB_ERR_SIZE;
  const int grid = n_eq1 + n_ge2;
  if (grid == 0) return KB_OK;
  DtsArgs a;
  a.Pi = Pi; a.Pibar = Pibar; a.sl = sl; a.sr = sr; a.c1 = node_child1; a.c2 = node_child2;
  a.log_pD = log_pD; a.log_pS = log_pS; a.prs = param_row_stride; a.item_idx = item_idx;
  a.item_offset = item_offset; a.lsp = log_split_probs; a.eq1_reduce_idx = eq1_reduce_idx; a.n_eq1 = n_eq1;
  a.ge2_ptr = ge2_ptr; a.ge2_parent_ids = ge2_parent_ids; a.n_ge2 = n_ge2; a.active = active_rows;
  a.out = out; a.out_row = out_row; a.S = S;
  int bd = 512;
  if (S <= 512) bd = ((S + 31) / 32) * 32;
  int vpt = (S + bd - 1) / bd;
  const size_t smem = (size_t)(2 * S) * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
#define KB_DTS_CASE(V)                                                                                   \
  case V:                                                                                                \
    if (smem > 48 * 1024 &&                                                                              \
        cudaFuncSetAttribute((const void*)dts_forward_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             (int)smem) != cudaSuccess)                                                  \
      return KB_ERR_LAUNCH;                                                                              \
    dts_forward_kernel<V><<<grid, bd, smem, st>>>(a);                                                    \
    break;
  if (vpt <= 1) vpt = 1; else if (vpt <= 2) vpt = 2; else if (vpt <= 4) vpt = 4; else if (vpt <= 8) vpt = 8;
  else vpt = 16;
  switch (vpt) {
    KB_DTS_CASE(1) KB_DTS_CASE(2) KB_DTS_CASE(4) KB_DTS_CASE(8) KB_DTS_CASE(16)
    default: return KB_ERR_SIZE;
  }
#undef KB_DTS_CASE
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
