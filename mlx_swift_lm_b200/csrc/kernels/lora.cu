// Batched multi-adapter LoRA (one adapter slot per token row) for serving
// several LoRA adapters in one decode batch without merging them into the
// base weights.
//
// For an adapted projection y = x W^T (W [N, K]) and adapter s with
// A_s [R, K], B_s [N, R] and scale c_s:
//     y += c_s * (x A_s^T) B_s^T
// Adapters are stacked per projection: A [S, R, K] and B^T [S, R, N] bf16
// (ranks zero-padded to R; the q / k / v or gate / up parts of a fused
// projection stack their A rows and place their B columns at the fused rows,
// so one shrink and one expand serve the whole fused weight).
//
//   lora_shrink   grid (T, ceil(R / 8)), one warp per (row, rank index):
//                 t[row, j] = A[slot, j, :] . x[row, :] in fp32
//   lora_expand   grid (ceil(N / 512), T), two outputs per thread, t[row]
//                 staged in shared memory, B^T read coalesced along N:
//                 y[row, n] = bf16(y[row, n] + c * sum_j B^T[slot, j, n] t[row, j])
//   lora_expand_glu  the same delta added to an interleaved gate|up
//                 pre-activation (64-row blocks) and the gated activation
//                 applied: out[row, f] = act(g + dg, u + du)
// Rows whose slot is negative carry no adapter and are left as they are.
// This replaces the reference's per-layer LoRALinear / DoRALinear
// (Adapters/LoRA/LoRA+Layers.swift:26, DoRA+Layers.swift:64), which applies
// one adapter to a whole model, with a per-row adapter choice.
#include "b200_common.cuh"

namespace b200 {

constexpr int kLoraMaxRank = 256;

__global__ void __launch_bounds__(256) lora_shrink_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                        const __nv_bfloat16* __restrict__ A, int R, int K,
                                                        const int* __restrict__ slots, int S,
                                                        float* __restrict__ t) {
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.y * 8 + warp;
  if (j >= R) return;
  const int s = slots[row];
  float acc = 0.f;
  if (s >= 0 && s < S) {
    const __nv_bfloat16* a = A + ((size_t)s * R + j) * K;
    const __nv_bfloat16* xr = x + (size_t)row * ldx;
    for (int k = lane * 8; k < K; k += 256) {
      const uint4 av = *reinterpret_cast<const uint4*>(a + k);
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + k);
      const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&av);
      const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 af = __bfloat1622float2(a2[e]), xf = __bfloat1622float2(x2[e]);
        acc = fmaf(af.x, xf.x, fmaf(af.y, xf.y, acc));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  } else if (s >= S && lane == 0 && j == 0) {
    set_status(kErrBounds);
  }
  if (lane == 0) t[(size_t)row * R + j] = acc;
}

// delta of outputs n and n + 1 (n even) of row `row` for slot s
__device__ __forceinline__ float2 lora_delta2(const __nv_bfloat16* __restrict__ Bt, int R, int N, int s, int n,
                                              const float* ts) {
  const __nv_bfloat16* b = Bt + (size_t)s * R * N + n;
  float d0 = 0.f, d1 = 0.f;
  for (int j = 0; j < R; ++j) {
    const float2 bv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(b + (size_t)j * N));
    d0 = fmaf(bv.x, ts[j], d0);
    d1 = fmaf(bv.y, ts[j], d1);
  }
  return make_float2(d0, d1);
}

__global__ void __launch_bounds__(256) lora_expand_kernel(__nv_bfloat16* __restrict__ y, int ldy,
                                                        const __nv_bfloat16* __restrict__ Bt, int R, int N,
                                                        const float* __restrict__ t,
                                                        const int* __restrict__ slots,
                                                        const float* __restrict__ scale, int S) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float ts[kLoraMaxRank];
  const int row = blockIdx.y;
  const int s = slots[row];
  if (s < 0 || s >= S) return;
  for (int j = threadIdx.x; j < R; j += blockDim.x) ts[j] = t[(size_t)row * R + j] * scale[s];
  __syncthreads();
  const int n = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (n >= N) return;
  const float2 d = lora_delta2(Bt, R, N, s, n, ts);
  __nv_bfloat162* yp = reinterpret_cast<__nv_bfloat162*>(y + (size_t)row * ldy + n);
  const float2 yv = __bfloat1622float2(*yp);
  *yp = __floats2bfloat162_rn(yv.x + d.x, yv.y + d.y);
}

// gu [T, 2F] interleaved gate|up pre-activation (64-row blocks) -> out [T, F]
__global__ void __launch_bounds__(256) lora_expand_glu_kernel(const __nv_bfloat16* __restrict__ gu, int ldg,
                                                            __nv_bfloat16* __restrict__ out, int ldo, int F,
                                                            const __nv_bfloat16* __restrict__ Bt, int R,
                                                            const float* __restrict__ t,
                                                            const int* __restrict__ slots,
                                                            const float* __restrict__ scale, int S, int act) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float ts[kLoraMaxRank];
  const int row = blockIdx.y;
  const int s = slots[row];
  const bool lora = s >= 0 && s < S;
  if (lora)
    for (int j = threadIdx.x; j < R; j += blockDim.x) ts[j] = t[(size_t)row * R + j] * scale[s];
  __syncthreads();
  const int f = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (f >= F) return;
  const int gi = (f >> 6) * 128 + (f & 63), ui = gi + 64;
  const __nv_bfloat16* g = gu + (size_t)row * ldg;
  float2 gv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(g + gi));
  float2 uv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(g + ui));
  if (lora) {
    const int N = 2 * F;
    const float2 dg = lora_delta2(Bt, R, N, s, gi, ts), du = lora_delta2(Bt, R, N, s, ui, ts);
    // the adapted projection rounds to bf16 like any linear output, then the activation runs in fp32
    gv = make_float2(bf2f(f2bf(gv.x + dg.x)), bf2f(f2bf(gv.y + dg.y)));
    uv = make_float2(bf2f(f2bf(uv.x + du.x)), bf2f(f2bf(uv.y + du.y)));
  }
  *reinterpret_cast<__nv_bfloat162*>(out + (size_t)row * ldo + f) =
      __floats2bfloat162_rn(glu_act(act, gv.x, uv.x), glu_act(act, gv.y, uv.y));
}

}  // namespace b200

using namespace b200;

extern "C" {

// t [T, R] fp32 scratch. x [T, K] bf16 (row stride ldx), A [S, R, K].
int b200_lora_shrink(const void* x, int ldx, const void* A, int R, int K, const int* slots, int S, float* t, int T,
                     cudaStream_t st) {
  if (T <= 0) return 0;
  if (R <= 0 || R > kLoraMaxRank || (K % 8) || (ldx % 8) || (((uintptr_t)x | (uintptr_t)A) & 15)) return -1;
  cudaError_t e = launch_k(lora_shrink_kernel, dim3(T, (R + 7) / 8), dim3(256), 0, st, 1,
                           reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<const __nv_bfloat16*>(A),
                           R, K, slots, S, t);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// y [T, N] bf16 updated in place; Bt [S, R, N]; scale [S] fp32.
int b200_lora_expand(void* y, int ldy, const void* Bt, int R, int N, const float* t, const int* slots,
                     const float* scale, int S, int T, cudaStream_t st) {
  if (T <= 0) return 0;
  if (R <= 0 || R > kLoraMaxRank || (N % 2) || (ldy % 2) || (((uintptr_t)y | (uintptr_t)Bt) & 3)) return -1;
  cudaError_t e = launch_k(lora_expand_kernel, dim3((N / 2 + 255) / 256, T), dim3(256), 0, st, 1,
                           reinterpret_cast<__nv_bfloat16*>(y), ldy, reinterpret_cast<const __nv_bfloat16*>(Bt), R, N,
                           t, slots, scale, S);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// gu [T, 2F] interleaved pre-activation -> out [T, F]; act: 1 SwiGLU, 4 GeGLU, 5 GPT-OSS.
int b200_lora_expand_glu(const void* gu, int ldg, void* out, int ldo, int F, const void* Bt, int R, const float* t,
                         const int* slots, const float* scale, int S, int act, int T, cudaStream_t st) {
  if (T <= 0) return 0;
  if (R <= 0 || R > kLoraMaxRank || (F % 64) || (ldg % 2) || (ldo % 2) ||
      (((uintptr_t)gu | (uintptr_t)out | (uintptr_t)Bt) & 3))
    return -1;
  if (act != kGluSwi && act != kGluGe && act != kGluOAI) return -1;
  cudaError_t e = launch_k(lora_expand_glu_kernel, dim3((F / 2 + 255) / 256, T), dim3(256), 0, st, 1,
                           reinterpret_cast<const __nv_bfloat16*>(gu), ldg, reinterpret_cast<__nv_bfloat16*>(out),
                           ldo, F, reinterpret_cast<const __nv_bfloat16*>(Bt), R, t, slots, scale, S, act);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"

B200_STATUS_ACCESSORS(lora)
