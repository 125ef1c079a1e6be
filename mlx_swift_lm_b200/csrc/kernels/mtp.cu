// MTP speculative-decoding round tail on the device: the greedy accept walk
// and the hidden-history update, so a whole round (draft steps, verify,
// accept) can run as one CUDA graph with one readback.
//
// Per request row r (one CTA), with the verify's greedy tokens pred
// [B, k+1], the drafts D [B, k] and the verify's final hiddens vh
// [B * (k+1), H]:
//   a      = forced[r] >= 0 ? min(forced[r], k)       (scheduled acceptance)
//                           : leading j with D[r, j] == pred[r, j]
//   res[r, 0..k] = D[r, 0..a-1], pred[r, a], -1 ...     (the a + 1 emitted tokens)
//   res[r, k+1]  = a                                     (res rows of k + 2 ints)
//   hist[hslot[r], K - a + j] = vh[r * (k+1) + j]      for j = 0..a
// (K >= k: the depth the history rows are sized for). The history row of a
// request holds, right-aligned, the target hiddens of
// the positions the next round's first draft step consumes (the accept walk
// of MTP/MTPFinalize.swift:101 and the round state of CBv2MTPRoundDriver.swift).
#include "b200_common.cuh"

namespace b200 {

__global__ void __launch_bounds__(256) mtp_accept_kernel(const int* __restrict__ pred, const int* __restrict__ D,
                                                       const int* __restrict__ forced, int k,
                                                       const int* __restrict__ hslot, int n_hist, int K,
                                                       const __nv_bfloat16* __restrict__ vh, int H,
                                                       __nv_bfloat16* __restrict__ hist, int* __restrict__ res) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int s_a;
  const int r = blockIdx.x;
  if (threadIdx.x == 0) {
    const int f = forced[r];
    int a = 0;
    if (f >= 0) {
      a = f < k ? f : k;
    } else {
      while (a < k && D[r * k + a] == pred[r * (k + 1) + a]) ++a;
    }
    int* row = res + (size_t)r * (k + 2);
    for (int j = 0; j <= k; ++j) row[j] = j < a ? D[r * k + j] : (j == a ? pred[r * (k + 1) + a] : -1);
    row[k + 1] = a;
    s_a = a;
  }
  __syncthreads();
  const int a = s_a;
  int hs = hslot[r];
  if (hs < 0 || hs >= n_hist) {
    if (threadIdx.x == 0) set_status(kErrBounds);
    return;
  }
  // a + 1 rows of H bf16, 8 elements per thread step
  const int per_row = H / 8;
  for (int idx = threadIdx.x; idx < (a + 1) * per_row; idx += blockDim.x) {
    const int j = idx / per_row, c = (idx % per_row) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(vh + ((size_t)r * (k + 1) + j) * H + c);
    *reinterpret_cast<uint4*>(hist + ((size_t)hs * (K + 1) + (K - a + j)) * H + c) = v;
  }
}

}  // namespace b200

using namespace b200;

extern "C" int b200_mtp_accept(const int* pred, const int* D, const int* forced, int k, const int* hslot, int n_hist,
                               int K, const void* vh, int H, void* hist, int* res, int B, cudaStream_t st) {
  if (B <= 0) return 0;
  if (k < 1 || K < k || (H % 8) || (((uintptr_t)vh | (uintptr_t)hist) & 15)) return -1;
  cudaError_t e = launch_k(mtp_accept_kernel, dim3(B), dim3(256), 0, st, 1, pred, D, forced, k, hslot, n_hist, K,
                           reinterpret_cast<const __nv_bfloat16*>(vh), H, reinterpret_cast<__nv_bfloat16*>(hist),
                           res);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

B200_STATUS_ACCESSORS(mtp)
