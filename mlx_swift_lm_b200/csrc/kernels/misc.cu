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
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int s = src[i];
  ids[i] = s >= 0 ? prev[s] : host_ids[i];
}

}  // namespace b200

extern "C" int b200_gather_tokens(const int* prev, const int* src, const int* host_ids, int* ids, int n,
                                  cudaStream_t st) {
  if (n <= 0) return 0;
b200::launch_k(  b200::gather_tokens_kernel, dim3((n + 127) / 128), dim3(128), 0, st, 1, prev, src, host_ids, ids, n);
  return (int)cudaGetLastError();
}

B200_STATUS_ACCESSORS(misc)

// ---------------------------------------------------------------------------
// Programmatic-dependent-launch switch shared by every launcher of the library.
// On by default; B200LM_PDL=0 in the environment or b200_set_pdl(0) turns it off.
// ---------------------------------------------------------------------------
#include <cstdlib>
#include <cstring>

namespace b200 {
static int g_pdl = -1;
bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* e = std::getenv("B200LM_PDL");
    g_pdl = (e && std::strcmp(e, "0") == 0) ? 0 : 1;
  }
  return g_pdl != 0;
}
}  // namespace b200

extern "C" void b200_set_pdl(int on) { b200::g_pdl = on ? 1 : 0; }
extern "C" int b200_get_pdl() { return b200::pdl_enabled() ? 1 : 0; }
