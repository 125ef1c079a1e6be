// Small engine-side kernels.
//
// gather_tokens: builds the input ids of a chained decode step on the device:
//   ids[i] = src[i] >= 0 ? prev_tokens[src[i]] : host_ids[i]
// so step N+1 can start from step N's sampled tokens before the host has read
// them (the chained-decode path of the engine).
#include "b200_common.cuh"

namespace b200 {

__global__ void gather_tokens_kernel(const int* __restrict__ prev, const int* __restrict__ src,
                                     const int* __restrict__ host_ids, int* __restrict__ ids, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int s = src[i];
  ids[i] = s >= 0 ? prev[s] : host_ids[i];
}

}  // namespace b200

extern "C" int b200_gather_tokens(const int* prev, const int* src, const int* host_ids, int* ids, int n,
                                  cudaStream_t st) {
  if (n <= 0) return 0;
  b200::gather_tokens_kernel<<<(n + 127) / 128, 128, 0, st>>>(prev, src, host_ids, ids, n);
  return (int)cudaGetLastError();
}

B200_STATUS_ACCESSORS(misc)
