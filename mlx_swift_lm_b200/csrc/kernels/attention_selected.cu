// Decode attention over selected tokens of each row's paged KV (sparse /
// indexer-selected attention, e.g. DeepSeek-style sparse attention and the
// gathered / selected KV scopes of the reference's CBv2 engine).
//
// Reference behaviour: MLXLMCommon/ContinuousBatchingV2/Paged/
// PagedSelectedGather.swift (gather the selected rows of a sequence's pages)
// and the sparse-state readers of ContinuousBatchingV2/GLM5Next: each query
// attends only to the key / value rows whose positions its indexer chose.
//
// B200 layout: one CTA per (row, KV head), 4 warps. The G = H / KVH query
// heads of the group share every selected key. Warp w walks the row's
// selected entries w, w + 4, ...; a lane holds D / 32 channels of each head's
// query and of the loaded K / V row, scores reduce across the warp, and each
// warp keeps an online softmax per head; the four warps merge through shared
// memory. Entries that are negative or not below the row's length are
// skipped. Pages [P][KVH][16][D] bf16.
#include "b200_common.cuh"

namespace b200 {
namespace sel {

constexpr int kWarps = 4;
constexpr int kMaxG = 8;

template <int DPL>
__global__ void __launch_bounds__(128) selected_decode_kernel(const __nv_bfloat16* __restrict__ q,
                                                              const __nv_bfloat16* __restrict__ kc,
                                                              const __nv_bfloat16* __restrict__ vc,
                                                              const int* __restrict__ page_table, int maxp,
                                                              const int* __restrict__ seq_lens,
                                                              const int* __restrict__ sel, int S, int H, int KVH,
                                                              float scale, __nv_bfloat16* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int D = DPL * 32;
  __shared__ float sm_m[kWarps][kMaxG], sm_l[kWarps][kMaxG];
  __shared__ float sm_acc[kWarps][kMaxG][D];
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = H / KVH;
  const int L = seq_lens[b];
  float qv[kMaxG][DPL], acc[kMaxG][DPL], m[kMaxG], l[kMaxG];
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      acc[g][i] = 0.f;
      qv[g][i] = g < G ? bf2f(q[((size_t)b * H + kvh * G + g) * D + lane * DPL + i]) * scale : 0.f;
    }
  }
  const int* srow = sel + (size_t)b * S;
  const int* prow = page_table + (size_t)b * maxp;
  for (int j = warp; j < S; j += kWarps) {
    const int t = srow[j];
    if (t < 0 || t >= L) continue;
    const int page = prow[t >> 4];
    const size_t off = (((size_t)page * KVH + kvh) * 16 + (t & 15)) * D + lane * DPL;
    float kk[DPL], vv[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      kk[i] = bf2f(kc[off + i]);
      vv[i] = bf2f(vc[off + i]);
    }
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g >= G) break;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) s = fmaf(qv[g][i], kk[i], s);
      s = warp_sum(s);
      const float mn = fmaxf(m[g], s);
      const float c = __expf(m[g] - mn), p = __expf(s - mn);
      l[g] = l[g] * c + p;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[g][i] = fmaf(acc[g][i], c, p * vv[i]);
      m[g] = mn;
    }
  }
#pragma unroll
  for (int g = 0; g < kMaxG; ++g) {
    if (g >= G) break;
    if (lane == 0) {
      sm_m[warp][g] = m[g];
      sm_l[warp][g] = l[g];
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) sm_acc[warp][g][lane * DPL + i] = acc[g][i];
  }
  __syncthreads();
  // merge the warps: thread (g, d) for g < G, d < D
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int g = e / D, d = e % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, sm_m[w][g]);
    float num = 0.f, den = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float c = sm_m[w][g] == -INFINITY ? 0.f : __expf(sm_m[w][g] - mx);
        num = fmaf(sm_acc[w][g][d], c, num);
        den = fmaf(sm_l[w][g], c, den);
      }
    }
    out[((size_t)b * H + kvh * G + g) * D + d] = f2bf(den > 0.f ? num / den : 0.f);
  }
}

}  // namespace sel
}  // namespace b200

using namespace b200;

extern "C" {

// q [B][H][D] bf16; caches [P][KVH][16][D] bf16; page_table [B][maxp]; seq_lens [B];
// sel [B][S] int32 token positions (-1 = none); out [B][H][D] bf16. H / KVH <= 8.
int b200_paged_selected_decode(const void* q, const void* k_cache, const void* v_cache, const int* page_table,
                               int maxp, const int* seq_lens, const int* sel, int S, int B, int H, int KVH, int D,
                               float scale, void* out, cudaStream_t st) {
  if (B <= 0) return 0;
  if (KVH <= 0 || H % KVH || H / KVH > sel::kMaxG || S <= 0) return -1;
  const dim3 grid(B, KVH);
  const auto* qq = reinterpret_cast<const __nv_bfloat16*>(q);
  const auto* kk = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  const auto* vv = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  auto* oo = reinterpret_cast<__nv_bfloat16*>(out);
  cudaError_t e;
  switch (D) {
    case 64:
      e = launch_k(sel::selected_decode_kernel<2>, grid, dim3(128), 0, st, 1, qq, kk, vv, page_table, maxp, seq_lens,
                   sel, S, H, KVH, scale, oo);
      break;
    case 128:
      e = launch_k(sel::selected_decode_kernel<4>, grid, dim3(128), 0, st, 1, qq, kk, vv, page_table, maxp, seq_lens,
                   sel, S, H, KVH, scale, oo);
      break;
    default:
      return -1;
  }
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"
