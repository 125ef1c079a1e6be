// Pairwise Givens rotation of activations (ParoQuant linears): per 128-channel
// group, the channels are scaled, then `krot` rounds of 64 disjoint channel
// pairs (i, j) are rotated by their angle: (a, b) <- (a c + b s, b c - a s).
// The rotated activations feed the ordinary quantised GEMM.
//
// Reference behaviour: MLXLMCommon/ParoQuant/PairwiseRotation.swift:60-120
// (pairs packed i | j << 16 as local channel indices of the group, cos / sin
// per pair slot and round, channel scales fused into the load, fp32 math,
// one rounding on the way out) and RotateQuantizedLinear.swift:70.
//
// B200 layout: one warp per (tile of kRows activation rows, channel group);
// a lane owns two pair slots of every round (their coefficients in
// registers) and four channels for the load / store; the tile lives in
// shared memory in fp32; rounds are separated by __syncwarp.
#include "b200_common.cuh"

namespace b200 {
namespace rot {

constexpr int kGroup = 128;
constexpr int kRows = 8;
constexpr int kMaxRot = 16;

__global__ void __launch_bounds__(32) pair_rotate_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int T, int K,
                                                        const float* __restrict__ cos_t,
                                                        const float* __restrict__ sin_t,
                                                        const int* __restrict__ pairs,
                                                        const float* __restrict__ scales, int krot,
                                                        __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float tile[kRows][kGroup];
  const int lane = threadIdx.x;
  const int row0 = blockIdx.x * kRows, g = blockIdx.y;
  const int gbase = g * kGroup;
  const int half_k = K / 2;
  float sc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) sc[i] = scales ? scales[gbase + lane * 4 + i] : 1.f;
  for (int r = 0; r < kRows; ++r) {
    const int row = row0 + r;
    if (row < T) {
      const uint2 raw = *reinterpret_cast<const uint2*>(x + (size_t)row * ldx + gbase + lane * 4);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) tile[r][lane * 4 + i] = bf2f(e[i]) * sc[i];
    }
  }
  __syncwarp();
  for (int k = 0; k < krot; ++k) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int idx = k * half_k + g * (kGroup / 2) + lane + u * 32;
      const float c = cos_t[idx], s = sin_t[idx];
      const int pr = pairs[idx];
      const int i = pr & 0xFFFF, j = pr >> 16;
      if (i >= kGroup || j >= kGroup) {
        set_status(kErrBounds);
        continue;
      }
      for (int m = 0; m < kRows; ++m) {
        const float a = tile[m][i], b = tile[m][j];
        tile[m][i] = a * c + b * s;
        tile[m][j] = b * c - a * s;
      }
    }
    __syncwarp();
  }
  for (int r = 0; r < kRows; ++r) {
    const int row = row0 + r;
    if (row < T) {
      uint2 raw;
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) e[i] = f2bf(tile[r][lane * 4 + i]);
      *reinterpret_cast<uint2*>(out + (size_t)row * ldo + gbase + lane * 4) = raw;
    }
  }
}

// Block Walsh-Hadamard transform of activations (Prism Hadamard checkpoints):
// per row and per `block` channels, y = H(s * x) / sqrt(block) (forward) or
// y = s * H(x) / sqrt(block) (inverse); H is the natural-order Walsh-Hadamard
// matrix, applied by log2(block) butterfly stages in shared memory. One CTA
// per (row, block).
__global__ void __launch_bounds__(512) block_hadamard_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int K,
                                                            int block, const float* __restrict__ signs, int inverse,
                                                            __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ float hb[];
  const int row = blockIdx.x, b0 = blockIdx.y * block;
  const __nv_bfloat16* xr = x + (size_t)row * ldx + b0;
  for (int i = threadIdx.x; i < block; i += blockDim.x) {
    float v = bf2f(xr[i]);
    if (!inverse && signs) v *= signs[b0 + i];
    hb[i] = v;
  }
  __syncthreads();
  for (int h = 1; h < block; h <<= 1) {
    for (int p = threadIdx.x; p < block / 2; p += blockDim.x) {
      const int i = (p / h) * 2 * h + (p % h), j = i + h;
      const float a = hb[i], b = hb[j];
      hb[i] = a + b;
      hb[j] = a - b;
    }
    __syncthreads();
  }
  const float sc = rsqrtf((float)block);
  __nv_bfloat16* orow = out + (size_t)row * ldo + b0;
  for (int i = threadIdx.x; i < block; i += blockDim.x) {
    float v = hb[i] * sc;
    if (inverse && signs) v *= signs[b0 + i];
    orow[i] = f2bf(v);
  }
}

}  // namespace rot
}  // namespace b200

using namespace b200;

extern "C" {

// x, out [T, K] bf16 (K % 128 == 0, rows 8-byte aligned); cos / sin / pairs
// [krot, K / 2]; scales [K] fp32 or null.
int b200_pair_rotate(const void* x, int ldx, int T, int K, const float* cos_t, const float* sin_t, const int* pairs,
                     const float* scales, int krot, void* out, int ldo, cudaStream_t st) {
  if (T <= 0) return 0;
  if ((K % rot::kGroup) || (ldx % 4) || (ldo % 4) || krot < 1 || krot > rot::kMaxRot) return -1;
  const dim3 grid((T + rot::kRows - 1) / rot::kRows, K / rot::kGroup);
  cudaError_t e = launch_k(rot::pair_rotate_kernel, grid, dim3(32), 0, st, 1,
                           reinterpret_cast<const __nv_bfloat16*>(x), ldx, T, K, cos_t, sin_t, pairs, scales, krot,
                           reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// x, out [T, K] bf16; block a power of two in [2, 8192] dividing K; signs [K] fp32 or null.
int b200_block_hadamard(const void* x, int ldx, int T, int K, int block, const float* signs, int inverse, void* out,
                        int ldo, cudaStream_t st) {
  if (T <= 0) return 0;
  if (block < 2 || block > 8192 || (block & (block - 1)) || (K % block)) return -1;
  const size_t smem = (size_t)block * sizeof(float);
  if (int e = b200::smem_attr_once<rot::block_hadamard_kernel>(8192 * 4)) return e;
  const int threads = block / 2 < 512 ? block / 2 : 512;
  cudaError_t e = launch_k(rot::block_hadamard_kernel, dim3(T, K / block), dim3(threads), smem, st, 1,
                           reinterpret_cast<const __nv_bfloat16*>(x), ldx, K, block, signs, inverse,
                           reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"

B200_STATUS_ACCESSORS(rotation)
