// Shared device helpers for the kernel-bench B200 solver kernels (sm_100a).
//
// Conventions used by every kernel in this library:
//   * log2-space fp32 state; -inf marks an impossible state (never NaN);
//   * "safe max": a max that is -inf is replaced by 0 before it is subtracted, so that
//     exp2(-inf - 0) = 0 and an all -inf LSE yields -inf;
//   * one CTA owns one row of S columns; thread t owns columns t, t+blockDim, ...;
//   * every entry point returns an int status (KB_OK = 0) instead of trapping.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define KB_OK 0
#define KB_ERR_ARG 1
#define KB_ERR_LAUNCH 2
#define KB_ERR_SIZE 3

namespace kb {

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }
__device__ __forceinline__ bool is_neg_inf(float x) { return x == __int_as_float(0xff800000); }
__device__ __forceinline__ float safe_max(float m) { return is_neg_inf(m) ? 0.0f : m; }

// Base-2 exponential / logarithm on the special-function unit: one PTX `ex2.approx.f32` /
// `lg2.approx.f32` instruction each (ex2(-inf) = +0, lg2(+0) = -inf).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions. `scratch` must hold at least 32 floats; all threads of the block
// must call; the result is returned to every thread. Two barriers.
__device__ __forceinline__ float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? scratch[lane] : neg_inf();
  return warp_max(r);
}
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? scratch[lane] : 0.0f;
  return warp_sum(r);
}
// Max and sum in one pass (returns both); scratch >= 64 floats.
__device__ __forceinline__ void block_max_sum(float& m, float& s, float* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  m = warp_max(m);
  s = warp_sum(s);
  __syncthreads();
  if (lane == 0) { scratch[wid] = m; scratch[32 + wid] = s; }
  __syncthreads();
  float mm = (lane < nw) ? scratch[lane] : neg_inf();
  float ss = (lane < nw) ? scratch[32 + lane] : 0.0f;
  m = warp_max(mm);
  s = warp_sum(ss);
}

// Ancestor-or-self path sum by pointer doubling over precomputed jump tables:
// after round r, buf[s] holds the sum over the first 2^(r+1) nodes of s's root path.
// jumps: [K, S] int32, jumps[r*S + s] = 2^r-th ancestor of s or -1.  x and y are two
// shared-memory buffers of S floats; x holds the input; the result pointer is returned.
__device__ __forceinline__ float* ancestor_sum_doubling(float* x, float* y, const int* __restrict__ jumps,
                                                         int K, int S) {
  for (int r = 0; r < K; ++r) {
    __syncthreads();
    const int* jr = jumps + (size_t)r * S;
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      int j = __ldg(jr + s);
      float v = x[s];
      if (j >= 0) v += x[j];
      y[s] = v;
    }
    float* t = x; x = y; y = t;
  }
  __syncthreads();
  return x;
}

// Bottom-up subtree sums in place over compact levels (internal nodes, deepest level first):
// buf[p] = buf[p] + buf[c1] + buf[c2].  Caller syncs before; this syncs after every level.
__device__ __forceinline__ void subtree_sums_levels(float* buf, const long long* __restrict__ lv_ptr, int n_levels,
                                                    const int* __restrict__ lv_par,
                                                    const int* __restrict__ lv_c1,
                                                    const int* __restrict__ lv_c2, int S) {
  for (int lv = 0; lv < n_levels; ++lv) {
    const int a = (int)lv_ptr[lv], b = (int)lv_ptr[lv + 1];
    for (int i = a + threadIdx.x; i < b; i += blockDim.x) {
      const int p = __ldg(lv_par + i), c1 = __ldg(lv_c1 + i), c2 = __ldg(lv_c2 + i);
      float v = buf[p];
      if (c1 < S) v += buf[c1];
      if (c2 < S) v += buf[c2];
      buf[p] = v;
    }
    __syncthreads();
  }
}

}  // namespace kb
