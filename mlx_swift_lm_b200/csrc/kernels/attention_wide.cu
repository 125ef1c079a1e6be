// Paged decode attention for wide heads (head dim 512: Gemma 4 global layers).
//
// Same contract and split-KV partial format as attention_decode.cu (fixed
// 256-token partitions in absolute positions, unnormalised partial outputs
// plus (max, sum) in the log2 domain, merged by paged_decode_merge_kernel),
// so the result is batch invariant in the same way.
//
// The narrow kernels give each lane D/8 dims of a query and split a page's
// tokens over lane groups; at D = 512 that is 64 registers per query head for
// q alone. Here the 32 lanes of a warp split the head dim instead (D/32 = 16
// dims per lane), a score is a warp reduction, and one warp serves
// ceil(G / 4) query heads of the CTA's KV head:
//   grid (partition, KV head, row), 128 threads;
//   K/V pages of the partition stream through a 2-stage shared ring filled by
//   the bulk-copy engine (one page of K and one of V per stage); every wait
//   is bounded.
#include "b200_common.cuh"

namespace b200 {
namespace wide {

constexpr int kPart = 256;  // tokens per partition (matches the merge pass)
constexpr int kPage = 16;
constexpr int kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;

struct Args {
  const __nv_bfloat16* q;  // [B, H, D]
  const void* k_cache;     // [P, KVH, 16, D]
  const void* v_cache;
  const int* page_table;  // [B, ld_pt]
  const int* seq_lens;    // [B]
  const float* k_scale;   // [KVH] (fp8 pages) or null
  const float* v_scale;
  float* part_acc;  // [B, H, max_parts, D]
  float* part_ml;   // [B, H, max_parts, 2]
  int H, KVH, ld_pt, max_parts, window;
  int64_t num_pages;
  float scale, softcap;
};

__device__ __forceinline__ void bulk_page(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// 16 consecutive page elements as fp32.
template <typename KVT>
__device__ __forceinline__ void load16(const KVT* p, float* out) {
  if constexpr (sizeof(KVT) == 2) {
    const uint4* u = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 w = u[c];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        out[c * 8 + 2 * j] = f.x;
        out[c * 8 + 2 * j + 1] = f.y;
      }
    }
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const __nv_fp8x2_e4m3* h = reinterpret_cast<const __nv_fp8x2_e4m3*>(&w);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 f = static_cast<float2>(h[j]);
      out[2 * j] = f.x;
      out[2 * j + 1] = f.y;
    }
  }
}

template <int D, int G, typename KVT>
__global__ void __launch_bounds__(128) wide_decode_part_kernel(Args a) {
  pdl_launch_dependents();
  pdl_wait();
  static_assert(D == 32 * 16, "16 dims per lane");
  constexpr int HPW = (G + 3) / 4;  // query heads per warp
  constexpr int kPageBytes = kPage * D * (int)sizeof(KVT);
  extern __shared__ __align__(128) uint8_t ring_raw[];  // [kStages][2][kPageBytes]
  __shared__ __align__(8) uint64_t bars[kStages];

  const int part = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = a.seq_lens[b];
  if (L <= 0) return;
  const int start = a.window > 0 ? max(0, L - a.window) : 0;
  if (part < start / kPart || part > (L - 1) / kPart) return;
  const int lo = max(start, part * kPart), hi = min(L, (part + 1) * kPart);
  const int pg_lo = lo / kPage, npages = (hi - 1) / kPage - pg_lo + 1;

  const float kscale = a.k_scale ? a.k_scale[kvh] : 1.f;
  const float qmul = (a.softcap > 0.f ? a.scale : a.scale * kLog2e) * kscale;
  float q[HPW][16], acc[HPW][16], m[HPW], l[HPW];
#pragma unroll
  for (int i = 0; i < HPW; ++i) {
    const int hg = warp + 4 * i;
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[i][j] = 0.f;
    if (hg < G) {
      const __nv_bfloat16* qp = a.q + ((size_t)b * a.H + kvh * G + hg) * D + lane * 16;
#pragma unroll
      for (int j = 0; j < 16; ++j) q[i][j] = bf2f(qp[j]) * qmul;
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) q[i][j] = 0.f;
    }
  }

  const uint32_t bar0 = smem_u32(&bars[0]);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const KVT* kc = reinterpret_cast<const KVT*>(a.k_cache);
  const KVT* vc = reinterpret_cast<const KVT*>(a.v_cache);
  const int* pt = a.page_table + (size_t)b * a.ld_pt;
  auto stage = [&](int s, int kv) { return ring_raw + (s * 2 + kv) * kPageBytes; };
  auto issue = [&](int i) {
    const int s = i % kStages;
    const int64_t page = checked_page(pt, pg_lo + i, a.ld_pt, a.num_pages);
    const size_t off = ((size_t)page * a.KVH + kvh) * kPage * D;
    mbar_arrive_expect_tx(bar0 + 8 * s, 2 * kPageBytes);
    bulk_page(smem_u32(stage(s, 0)), kc + off, kPageBytes, bar0 + 8 * s);
    bulk_page(smem_u32(stage(s, 1)), vc + off, kPageBytes, bar0 + 8 * s);
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kStages, npages); ++i) issue(i);

  bool ok = true;
  for (int i = 0; i < npages; ++i) {
    const int s = i % kStages;
    if (ok && !mbar_wait(bar0 + 8 * s, (i / kStages) & 1, kErrAttnWait)) ok = false;
    if (ok) {
      const KVT* ks = reinterpret_cast<const KVT*>(stage(s, 0));
      const KVT* vs = reinterpret_cast<const KVT*>(stage(s, 1));
      const int pos0 = (pg_lo + i) * kPage;
      float sc[HPW][kPage];
#pragma unroll
      for (int t = 0; t < kPage; ++t) {
        float kv[16];
        load16<KVT>(ks + t * D + lane * 16, kv);
        const bool valid = pos0 + t >= lo && pos0 + t < hi;
#pragma unroll
        for (int h = 0; h < HPW; ++h) {
          float d = 0.f;
#pragma unroll
          for (int j = 0; j < 16; ++j) d += q[h][j] * kv[j];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
          if (a.softcap > 0.f) d = a.softcap * tanhf(d / a.softcap) * kLog2e;
          sc[h][t] = valid ? d : -INFINITY;
        }
      }
#pragma unroll
      for (int h = 0; h < HPW; ++h) {
        float mx = m[h];
#pragma unroll
        for (int t = 0; t < kPage; ++t) mx = fmaxf(mx, sc[h][t]);
        const float corr = m[h] == -INFINITY ? 0.f : exp2f(m[h] - mx);
        l[h] *= corr;
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[h][j] *= corr;
#pragma unroll
        for (int t = 0; t < kPage; ++t) sc[h][t] = mx == -INFINITY ? 0.f : exp2f(sc[h][t] - mx);
        m[h] = mx;
      }
#pragma unroll
      for (int t = 0; t < kPage; ++t) {
        float vv[16];
        load16<KVT>(vs + t * D + lane * 16, vv);
#pragma unroll
        for (int h = 0; h < HPW; ++h) {
          l[h] += sc[h][t];
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[h][j] += sc[h][t] * vv[j];
        }
      }
    }
    __syncthreads();  // every warp is done with stage s
    if (threadIdx.x == 0 && ok && i + kStages < npages) issue(i + kStages);
  }
  const float vscale = a.v_scale ? a.v_scale[kvh] : 1.f;
#pragma unroll
  for (int h = 0; h < HPW; ++h) {
    const int hg = warp + 4 * h;
    if (hg >= G) continue;
    const size_t pidx = ((size_t)b * a.H + kvh * G + hg) * a.max_parts + part;
    float* dst = a.part_acc + pidx * D + lane * 16;
#pragma unroll
    for (int j = 0; j < 16; j += 4)
      *reinterpret_cast<float4*>(dst + j) =
          make_float4(acc[h][j] * vscale, acc[h][j + 1] * vscale, acc[h][j + 2] * vscale, acc[h][j + 3] * vscale);
    if (lane == 0) {
      a.part_ml[pidx * 2 + 0] = ok ? m[h] : -INFINITY;
      a.part_ml[pidx * 2 + 1] = ok ? l[h] : 0.f;
    }
  }
}

template <int G, typename KVT>
int launch(const Args& a, int B, cudaStream_t st) {
  constexpr int D = 512;
  constexpr int smem = kStages * 2 * kPage * D * (int)sizeof(KVT);
  if (int e = smem_attr_once<wide_decode_part_kernel<D, G, KVT>>(smem)) return e;
  cudaError_t e = launch_k(wide_decode_part_kernel<D, G, KVT>, dim3(a.max_parts, a.KVH, B), dim3(128), smem, st, 1, a);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

template <typename KVT>
int dispatch(const Args& a, int B, int G, cudaStream_t st) {
  switch (G) {
    case 1: return launch<1, KVT>(a, B, st);
    case 2: return launch<2, KVT>(a, B, st);
    case 4: return launch<4, KVT>(a, B, st);
    case 8: return launch<8, KVT>(a, B, st);
    case 16: return launch<16, KVT>(a, B, st);
    default: return -1;
  }
}

}  // namespace wide
}  // namespace b200

using namespace b200;

extern "C" {

// Partition pass for head dim 512; follow with b200_paged_decode_merge (D = 512).
// Scratch: part_acc B*H*max_parts*512 floats, part_ml B*H*max_parts*2 floats.
int b200_paged_decode_wide_part(const void* q, const void* k_cache, const void* v_cache, int kv_fp8,
                                const float* k_scale, const float* v_scale, const int* page_table, int ld_pt,
                                const int* seq_lens, float* part_acc, float* part_ml, int B, int H, int KVH, int D,
                                int max_parts, int window, float scale, float softcap, int64_t num_pages,
                                cudaStream_t st) {
  if (B <= 0) return 0;
  if (D != 512 || KVH <= 0 || H % KVH) return -1;
  wide::Args a{reinterpret_cast<const __nv_bfloat16*>(q), k_cache, v_cache, page_table, seq_lens, k_scale, v_scale,
               part_acc, part_ml, H, KVH, ld_pt, max_parts, window, num_pages, scale, softcap};
  const int G = H / KVH;
  return kv_fp8 ? wide::dispatch<uint8_t>(a, B, G, st) : wide::dispatch<__nv_bfloat16>(a, B, G, st);
}

}  // extern "C"

B200_STATUS_ACCESSORS(attn_wide)
