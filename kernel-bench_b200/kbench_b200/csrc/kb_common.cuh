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

// Exclusive prefix sums of a block-wide sequence held in registers: thread t holds entries
// [t*CH, (t+1)*CH) in v, which become their exclusive prefixes; returns the total.  The same
// additions in the same order as block_exclusive_scan_ch.  ONE barrier: tmp (>= 32 floats) is
// read after it, so the caller must pass another barrier before tmp is written again.
template <int CH>
__device__ __forceinline__ float reg_exclusive_scan(float (&v)[CH], float* tmp) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  float local = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) local += v[j];
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) tmp[wid] = incl;
  __syncthreads();
  float t = lane < nw ? tmp[lane] : 0.f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, t, o);
    if (lane >= o) t += y;
  }
  const float prev = __shfl_up_sync(0xffffffffu, t, 1);
  const float wbase = __shfl_sync(0xffffffffu, lane == 0 ? 0.f : prev, wid);
  const float total = __shfl_sync(0xffffffffu, t, nw - 1);
  float run = wbase + incl - local;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const float x = v[j];
    v[j] = run;
    run += x;
  }
  return total;
}

// Stores CH consecutive floats at dst (16-byte aligned when CH % 4 == 0).
template <int CH>
__device__ __forceinline__ void store_chunk(float* dst, const float (&v)[CH]) {
  if constexpr (CH % 4 == 0) {
#pragma unroll
    for (int j = 0; j < CH; j += 4)
      *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < CH; ++j) dst[j] = v[j];
  }
}

// Loads CH consecutive floats from src (16-byte aligned when CH % 4 == 0).
template <int CH>
__device__ __forceinline__ void load_chunk(float (&v)[CH], const float* src) {
  if constexpr (CH % 4 == 0) {
#pragma unroll
    for (int j = 0; j < CH; j += 4) {
      const float4 q = *reinterpret_cast<const float4*>(src + j);
      v[j] = q.x; v[j + 1] = q.y; v[j + 2] = q.z; v[j + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < CH; ++j) v[j] = src[j];
  }
}

// Exclusive prefix sums in place over buf[0 .. blockDim.x*CH) (the caller zero-pads the tail);
// thread t owns the contiguous chunk [t*CH, (t+1)*CH).  Returns the total.  tmp >= 32 floats.
// Syncs on exit (the caller syncs before, after writing buf).  With SUM, *bsum (one value per
// thread) also becomes its block sum, on the scan's middle barrier (tmp >= 64 floats then; the
// same additions as block_sum).
template <int CH, bool SUM = false>
__device__ __forceinline__ float block_exclusive_scan_ch(float* buf, float* tmp, float* bsum = nullptr) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, wid = tid >> 5, nw = (blockDim.x + 31) >> 5;
  float v[CH];
  float* base = buf + tid * CH;
  if constexpr (CH % 4 == 0) {
#pragma unroll
    for (int j = 0; j < CH; j += 4) {
      const float4 q = *reinterpret_cast<const float4*>(base + j);
      v[j] = q.x; v[j + 1] = q.y; v[j + 2] = q.z; v[j + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < CH; ++j) v[j] = base[j];
  }
  float local = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) local += v[j];
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) tmp[wid] = incl;
  if constexpr (SUM) {
    const float ws = warp_sum(*bsum);
    if (lane == 0) tmp[32 + wid] = ws;
  }
  __syncthreads();
  if constexpr (SUM) {
    const float r = lane < nw ? tmp[32 + lane] : 0.0f;
    *bsum = warp_sum(r);
  }
  float wbase = 0.f, total;
  {
    float t = lane < nw ? tmp[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    // t = inclusive prefix of warp totals at warp index `lane`
    const float prev = __shfl_up_sync(0xffffffffu, t, 1);
    wbase = __shfl_sync(0xffffffffu, lane == 0 ? 0.f : prev, wid);
    total = __shfl_sync(0xffffffffu, t, nw - 1);
  }
  float run = wbase + incl - local;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const float x = v[j];
    v[j] = run;
    run += x;
  }
  if constexpr (CH % 4 == 0) {
#pragma unroll
    for (int j = 0; j < CH; j += 4)
      *reinterpret_cast<float4*>(base + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < CH; ++j) base[j] = v[j];
  }
  __syncthreads();
  return total;
}

// Exclusive scan of buf[0 .. blockDim.x*CH) fused with a block max and sum of one value per
// thread (mx, sm, returned block-wide).  tmp >= 96 floats.  Two barriers (after the per-warp
// partials, after the write-back).  The caller syncs before (after writing buf).
template <int CH>
__device__ __forceinline__ void block_scan_ch_maxsum(float* buf, float* tmp, float& mx, float& sm) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, wid = tid >> 5, nw = (blockDim.x + 31) >> 5;
  float v[CH];
  float* base = buf + tid * CH;
  if constexpr (CH % 4 == 0) {
#pragma unroll
    for (int j = 0; j < CH; j += 4) {
      const float4 q = *reinterpret_cast<const float4*>(base + j);
      v[j] = q.x; v[j + 1] = q.y; v[j + 2] = q.z; v[j + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < CH; ++j) v[j] = base[j];
  }
  float local = 0.f;
#pragma unroll
  for (int j = 0; j < CH; ++j) local += v[j];
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  mx = warp_max(mx);
  sm = warp_sum(sm);
  if (lane == 31) tmp[wid] = incl;
  if (lane == 0) { tmp[32 + wid] = mx; tmp[64 + wid] = sm; }
  __syncthreads();
  float t = lane < nw ? tmp[lane] : 0.f;
  float bm = lane < nw ? tmp[32 + lane] : 0.f;
  float bs = lane < nw ? tmp[64 + lane] : 0.f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, t, o);
    if (lane >= o) t += y;
  }
  mx = warp_max(bm);
  sm = warp_sum(bs);
  const float prev = __shfl_up_sync(0xffffffffu, t, 1);
  const float wbase = __shfl_sync(0xffffffffu, lane == 0 ? 0.f : prev, wid);
  float run = wbase + incl - local;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const float x = v[j];
    v[j] = run;
    run += x;
  }
  if constexpr (CH % 4 == 0) {
#pragma unroll
    for (int j = 0; j < CH; j += 4)
      *reinterpret_cast<float4*>(base + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < CH; ++j) base[j] = v[j];
  }
  __syncthreads();
}

}  // namespace kb
