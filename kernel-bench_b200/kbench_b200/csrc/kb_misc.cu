// ABI version and the species-tree pointer-doubling table.
#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

// jumps[0][s] = parent(s) (or -1); jumps[r][s] = jumps[r-1][jumps[r-1][s]] (or -1).
// One CTA, rounds in order with a barrier between them.
__global__ void build_jumps_kernel(const int* __restrict__ parent, int S, int K, int* jumps) {
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    const int p = parent[s];
    jumps[s] = (p >= 0 && p < S) ? p : -1;
  }
  for (int r = 1; r < K; ++r) {
    __syncthreads();
    const int* prev = jumps + (size_t)(r - 1) * S;
    int* cur = jumps + (size_t)r * S;
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
      const int j = prev[s];
      cur[s] = j >= 0 ? prev[j] : -1;
    }
  }
}

}  // namespace

extern "C" int kb_abi_version(void) { return 4; }

extern "C" int kb_build_jumps(const int* node_parent, int S, int K, int* jumps, void* stream) {
  if (S <= 0 || K < 0) return KB_ERR_ARG;
  if (K == 0) return KB_OK;
  build_jumps_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(node_parent, S, K, jumps);
  return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH;
}
