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

namespace kb {

// In-place exclusive prefix sums of two shared buffers a[0..n), b[0..n) (each thread owns a
// contiguous chunk); returns the totals.  tmp must hold 64 floats.  Syncs on entry and exit.
__device__ __forceinline__ void block_exclusive_scan2(float* a, float* b, int n, float* tmp, float& tot_a,
                                                      float& tot_b) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5, nw = (nt + 31) >> 5;
  const int ch = (n + nt - 1) / nt;
  const int b0 = min(tid * ch, n), b1 = min(b0 + ch, n);
  __syncthreads();
  float la = 0.f, lb = 0.f;
  for (int i = b0; i < b1; ++i) { la += a[i]; lb += b[i]; }
  float ia = la, ib = lb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, ia, o);
    const float yb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) { ia += ya; ib += yb; }
  }
  if (lane == 31) { tmp[wid] = ia; tmp[32 + wid] = ib; }
  __syncthreads();
  if (wid == 0) {
    float ta = lane < nw ? tmp[lane] : 0.f;
    float tb = lane < nw ? tmp[32 + lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float ya = __shfl_up_sync(0xffffffffu, ta, o);
      const float yb = __shfl_up_sync(0xffffffffu, tb, o);
      if (lane >= o) { ta += ya; tb += yb; }
    }
    tmp[lane] = ta;
    tmp[32 + lane] = tb;
  }
  __syncthreads();
  float ra = (wid > 0 ? tmp[wid - 1] : 0.f) + ia - la;
  float rb = (wid > 0 ? tmp[32 + wid - 1] : 0.f) + ib - lb;
  tot_a = tmp[nw - 1];
  tot_b = tmp[32 + nw - 1];
  for (int i = b0; i < b1; ++i) {
    const float va = a[i], vb = b[i];
    a[i] = ra;
    b[i] = rb;
    ra += va;
    rb += vb;
  }
  __syncthreads();
}

// Single-buffer variant.
__device__ __forceinline__ float block_exclusive_scan(float* a, int n, float* tmp) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5, nw = (nt + 31) >> 5;
  const int ch = (n + nt - 1) / nt;
  const int b0 = min(tid * ch, n), b1 = min(b0 + ch, n);
  __syncthreads();
  float la = 0.f;
  for (int i = b0; i < b1; ++i) la += a[i];
  float ia = la;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, ia, o);
    if (lane >= o) ia += ya;
  }
  if (lane == 31) tmp[wid] = ia;
  __syncthreads();
  if (wid == 0) {
    float ta = lane < nw ? tmp[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float ya = __shfl_up_sync(0xffffffffu, ta, o);
      if (lane >= o) ta += ya;
    }
    tmp[lane] = ta;
  }
  __syncthreads();
  float ra = (wid > 0 ? tmp[wid - 1] : 0.f) + ia - la;
  const float tot = tmp[nw - 1];
  for (int i = b0; i < b1; ++i) {
    const float va = a[i];
    a[i] = ra;
    ra += va;
  }
  __syncthreads();
  return tot;
}

}  // namespace kb

namespace kb {

// Exclusive prefix sums in place over buf[0 .. blockDim.x*CH) (the caller zero-pads the tail);
// thread t owns the contiguous chunk [t*CH, (t+1)*CH).  Returns the total.  tmp >= 32 floats.
// Syncs on exit (the caller syncs before, after writing buf).
template <int CH>
__device__ __forceinline__ float block_exclusive_scan_ch(float* buf, float* tmp) {
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
  __syncthreads();
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

// Block max / min-of-positives / sum in one reduction; tmp >= 96 floats.  Two barriers.
__device__ __forceinline__ void block_max_minpos_sum(float& mx, float& mn, float& sm, float* tmp) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  mx = warp_max(mx);
  mn = -warp_max(-mn);
  sm = warp_sum(sm);
  __syncthreads();
  if (lane == 0) { tmp[wid] = mx; tmp[32 + wid] = mn; tmp[64 + wid] = sm; }
  __syncthreads();
  const float a1 = lane < nw ? tmp[lane] : 0.f;
  const float a2 = lane < nw ? tmp[32 + lane] : 3.0e38f;
  const float a3 = lane < nw ? tmp[64 + lane] : 0.f;
  mx = warp_max(a1);
  mn = -warp_max(-a2);
  sm = warp_sum(a3);
}

}  // namespace kb

namespace kb {

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
