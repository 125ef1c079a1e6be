// Paged prefill attention, CUDA-core variant (any head dim up to 256).
//
// Causal attention of a prefill chunk against the row's paged KV history
// (which already contains the chunk's own keys/values). This covers the
// reference's prefill path (gather pages then MLX SDPA,
// ContinuousBatchingV2/Paged/PagedLayerCache.swift:584-637) with sliding
// windows from absolute positions and learned sinks. It is the fallback for
// shapes the tensor-core kernel (attention_prefill_mma.cu) does not take
// (fp8 KV pages).
//
// Work unit: a tile of QT query tokens of one row x one KV head; each thread
// owns one (query, head-of-group) pair with an exact online softmax. KV pages
// are staged in shared memory and read as broadcasts.
#include "b200_common.cuh"

namespace b200 {

constexpr float kLog2eP = 1.4426950408889634f;

struct PrefillArgs {
  const __nv_bfloat16* q;  // [T, H, D]
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;  // [P, KVH, 16, D]
  const int* page_table;         // [R, ld_pt]
  const int* cu_q;               // [R+1] token offsets of each row's chunk
  const int* q_pos0;             // [R] absolute position of each row's first chunk token
  const int* tiles;              // [n_tiles, 2] (row, q offset within the row's chunk)
  const float* sinks;            // [H] or null
  __nv_bfloat16* out;            // [T, H, D]
  int H, KVH, ld_pt, window;
  int64_t num_pages;
  float scale, softcap;
};

template <int D, int G>
__global__ void __launch_bounds__(128) paged_prefill_simt_kernel(PrefillArgs a) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  constexpr int QT = 128 / G;  // queries per tile
  __shared__ __align__(16) __nv_bfloat16 ks[16][D];
  __shared__ __align__(16) __nv_bfloat16 vs[16][D];
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int row = a.tiles[2 * tile], qoff = a.tiles[2 * tile + 1];
  const int q0 = a.cu_q[row], qlen = a.cu_q[row + 1] - q0;
  const int pos0 = a.q_pos0[row];
  const int qi = threadIdx.x / G, hg = threadIdx.x % G;
  const int qidx = qoff + qi;
  const bool active = qidx < qlen;
  const int qpos = pos0 + (active ? qidx : 0);
  const int head = kvh * G + hg;
  const int kstart = a.window > 0 ? max(0, qpos - a.window + 1) : 0;
  // key range of the whole tile
  const int last_q = min(qlen, qoff + QT) - 1;
  const int tile_hi = pos0 + last_q;  // inclusive
  const int tile_lo = a.window > 0 ? max(0, pos0 + qoff - a.window + 1) : 0;

  float q[D];
  const float qmul = a.softcap > 0.f ? a.scale : a.scale * kLog2eP;
  if (active) {
    const __nv_bfloat16* qp = a.q + ((size_t)(q0 + qidx) * a.H + head) * D;
#pragma unroll
    for (int d = 0; d < D; ++d) q[d] = bf2f(qp[d]) * qmul;
  }
  float m = -INFINITY, l = 0.f;
  float acc[D];
#pragma unroll
  for (int d = 0; d < D; ++d) acc[d] = 0.f;

  const int* pt = a.page_table + (size_t)row * a.ld_pt;
  for (int pg = tile_lo / 16; pg <= tile_hi / 16; ++pg) {
    const int64_t page = checked_page(pt, pg, a.ld_pt, a.num_pages);
    __syncthreads();
    const size_t off = ((size_t)page * a.KVH + kvh) * 16 * D;
    for (int i = threadIdx.x * 8; i < 16 * D; i += blockDim.x * 8) {
      *reinterpret_cast<uint4*>(&ks[0][0] + i) = *reinterpret_cast<const uint4*>(a.k_cache + off + i);
      *reinterpret_cast<uint4*>(&vs[0][0] + i) = *reinterpret_cast<const uint4*>(a.v_cache + off + i);
    }
    __syncthreads();
    if (!active) continue;
    for (int t = 0; t < 16; ++t) {
      const int kp = pg * 16 + t;
      if (kp < kstart || kp > qpos) continue;
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < D; d += 8) {
        uint4 u = *reinterpret_cast<const uint4*>(&ks[t][d]);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __bfloat1622float2(h[j]);
          s += q[d + 2 * j] * f.x + q[d + 2 * j + 1] * f.y;
        }
      }
      if (a.softcap > 0.f) s = a.softcap * tanhf(s / a.softcap) * kLog2eP;
      const float mn = fmaxf(m, s);
      const float corr = exp2f(m - mn);
      const float p = exp2f(s - mn);
      l = l * corr + p;
#pragma unroll
      for (int d = 0; d < D; d += 8) {
        uint4 u = *reinterpret_cast<const uint4*>(&vs[t][d]);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __bfloat1622float2(h[j]);
          acc[d + 2 * j] = acc[d + 2 * j] * corr + p * f.x;
          acc[d + 2 * j + 1] = acc[d + 2 * j + 1] * corr + p * f.y;
        }
      }
      m = mn;
    }
  }
  if (!active) return;
  float den = l;
  float scale_out = 1.f;
  if (a.sinks) {
    const float sk = a.sinks[head] * kLog2eP;
    const float mn = fmaxf(m, sk);
    scale_out = exp2f(m - mn);
    den = l * scale_out + exp2f(sk - mn);
  }
  const float inv = den > 0.f ? scale_out / den : 0.f;
  __nv_bfloat16* o = a.out + ((size_t)(q0 + qidx) * a.H + head) * D;
#pragma unroll
  for (int d = 0; d < D; ++d) o[d] = f2bf(acc[d] * inv);
}

template <int D>
static int dispatch_prefill(const PrefillArgs& a, int n_tiles, int G, cudaStream_t st) {
  dim3 grid(n_tiles, a.KVH);
  switch (G) {
    case 1: launch_k(paged_prefill_simt_kernel<D, 1>, grid, dim3(128), 0, st, 1, a); break;
    case 2: launch_k(paged_prefill_simt_kernel<D, 2>, grid, dim3(128), 0, st, 1, a); break;
    case 4: launch_k(paged_prefill_simt_kernel<D, 4>, grid, dim3(128), 0, st, 1, a); break;
    case 8: launch_k(paged_prefill_simt_kernel<D, 8>, grid, dim3(128), 0, st, 1, a); break;
    case 16: launch_k(paged_prefill_simt_kernel<D, 16>, grid, dim3(128), 0, st, 1, a); break;
    default: return -1;
  }
  return (int)cudaGetLastError();
}

}  // namespace b200

using namespace b200;

extern "C" {

// Queries per tile for a GQA group size G (the host builds the tile list).
int b200_prefill_simt_q_tile(int G) { return 128 / G; }

int b200_paged_prefill_simt(const void* q, const void* k_cache, const void* v_cache, const int* page_table,
                            int ld_pt, const int* cu_q, const int* q_pos0, const int* tiles, int n_tiles,
                            const float* sinks, void* out, int H, int KVH, int D, int window, float scale,
                            float softcap, int64_t num_pages, cudaStream_t st) {
  if (n_tiles <= 0) return 0;
  PrefillArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  a.page_table = page_table;
  a.cu_q = cu_q;
  a.q_pos0 = q_pos0;
  a.tiles = tiles;
  a.sinks = sinks;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.H = H;
  a.KVH = KVH;
  a.ld_pt = ld_pt;
  a.window = window;
  a.num_pages = num_pages;
  a.scale = scale;
  a.softcap = softcap;
  const int G = H / KVH;
  switch (D) {
    case 64: return dispatch_prefill<64>(a, n_tiles, G, st);
    case 128: return dispatch_prefill<128>(a, n_tiles, G, st);
    default: return -1;
  }
}

}  // extern "C"

B200_STATUS_ACCESSORS(attn_prefill_simt)
