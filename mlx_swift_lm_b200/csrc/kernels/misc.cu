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

// xIELU activation in place over bf16 x [n] (Apertus MLPs), from the layer's
// raw parameters p = {alpha_p, alpha_n, beta, eps}:
//   a_p = softplus(alpha_p), a_n = beta + softplus(alpha_n)
//   x > 0:  a_p x^2 + beta x
//   x <= 0: a_n (exp(min(x, eps)) - 1) - a_n x + beta x
__global__ void xielu_kernel(__nv_bfloat16* x, int64_t n, const float* p) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  const float sp_a = p[0] > 20.f ? p[0] : log1pf(expf(p[0]));
  const float sp_n = p[1] > 20.f ? p[1] : log1pf(expf(p[1]));
  const float beta = p[2], eps = p[3];
  const float an = beta + sp_n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = __bfloat162float(x[i]);
    const float y = v > 0.f ? sp_a * v * v + beta * v : an * expm1f(fminf(v, eps)) - an * v + beta * v;
    x[i] = __float2bfloat16_rn(y);
  }
}

extern "C" int b200_xielu(void* x, int64_t n, const float* params, cudaStream_t st) {
  if (n <= 0) return 0;
  const int blocks = (int)((n + 1023) / 1024 < 2048 ? (n + 1023) / 1024 : 2048);
  cudaError_t e = b200::launch_k(xielu_kernel, dim3(blocks), dim3(256), 0, st, 1,
                                 reinterpret_cast<__nv_bfloat16*>(x), n, params);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

extern "C" void b200_set_pdl(int on) { b200::g_pdl = on ? 1 : 0; }
extern "C" int b200_get_pdl() { return b200::pdl_enabled() ? 1 : 0; }
