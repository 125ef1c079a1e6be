// Paged decode attention (flash-decoding, split over the KV sequence).
//
// Same contract as the reference's two-pass Metal kernel
// (ContinuousBatchingV2/Paged/pagedattention.metal:260-486 partition pass,
// :518-587 merge pass; dispatch PagedAttentionKernel.swift:636):
//   pass A, one CTA per (row, KV head, partition): online softmax over the
//           partition's tokens for every query head of the GQA group, writing
//           unnormalised partial outputs plus (max, sum);
//   pass B, one CTA per row: merge the partitions; learned sinks enter the
//           denominator only.
// Partition boundaries are fixed multiples of kPartTokens in absolute token
// positions, so a row's reduction order depends only on its own length: the
// result is bit-identical whatever its batch-mates are.
//
// B200 specifics: each KV page (16 tokens x D for one KV head, contiguous)
// is pulled into shared memory by the bulk-copy engine
// (cp.async.bulk ... mbarrier::complete_tx) through a 4-stage ring, and every
// warp of the CTA computes from shared memory; waits are bounded.
//
// Layouts
//   q          [B, H, D] bf16 (H = KVH * G), already normed and rotated
//   k/v cache  [num_pages, KVH, 16, D] bf16 or fp8-e4m3 (per-KV-head scale)
//   page_table [B, ld_pt] int32, seq_lens [B] int32 (tokens incl. current)
//   scratch    part_acc [B, H, max_parts, D] fp32, part_ml [B, H, max_parts, 2]
#include "b200_common.cuh"

namespace b200 {

constexpr int kPartTokens = 256;  // tokens per partition (16 pages)
constexpr int kPage = 16;
constexpr int kStages = 4;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

template <typename KVT, int N>
__device__ __forceinline__ void load_kv_vec(const KVT* p, float* out) {
  // N consecutive elements from shared memory, as fp32
  if constexpr (sizeof(KVT) == 2) {
    static_assert(N % 8 == 0, "vector width");
#pragma unroll
    for (int c = 0; c < N / 8; ++c) {
      uint4 u = reinterpret_cast<const uint4*>(p)[c];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        out[c * 8 + 2 * j] = f.x;
        out[c * 8 + 2 * j + 1] = f.y;
      }
    }
  } else {
    static_assert(N % 8 == 0, "vector width");
#pragma unroll
    for (int c = 0; c < N / 8; ++c) {
      uint2 u = reinterpret_cast<const uint2*>(p)[c];
      const __nv_fp8x2_e4m3* h = reinterpret_cast<const __nv_fp8x2_e4m3*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = static_cast<float2>(h[j]);
        out[c * 8 + 2 * j] = f.x;
        out[c * 8 + 2 * j + 1] = f.y;
      }
    }
  }
}

struct DecodeArgs {
  const __nv_bfloat16* q;
  const void* k_cache;
  const void* v_cache;
  const int* page_table;
  const int* seq_lens;
  const float* sinks;  // [H] natural-log units, or null
  const float* k_scale;
  const float* v_scale;
  float* part_acc;
  float* part_ml;
  __nv_bfloat16* out;
  int H, KVH, ld_pt, max_parts, window;
  int64_t num_pages;
  float scale, softcap;
};

// D: head dim; G: query heads per KV head.
template <int D, int G, typename KVT>
__global__ void __launch_bounds__(128) paged_decode_part_kernel(DecodeArgs a) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  constexpr int DL = D / 8;                      // dims per lane
  constexpr int HW = G >= 4 ? G / 4 : 1;         // heads per warp
  constexpr int TS = G >= 4 ? 1 : 4 / G;         // warps sharing one head (split tokens)
  constexpr int TPW = kPage / TS;                // tokens of a page handled by one warp
  constexpr int TPG = TPW / 4;                   // tokens per token-group per page
  constexpr int kPageBytes = kPage * D * (int)sizeof(KVT);
  static_assert(TPG >= 1, "layout");

  extern __shared__ __align__(128) uint8_t ring_raw[];  // [kStages][2][kPageBytes]
  auto ring = reinterpret_cast<uint8_t(*)[2][kPageBytes]>(ring_raw);
  __shared__ __align__(8) uint64_t bars[kStages];
  __shared__ float xw_m[4][HW], xw_l[4][HW];
  __shared__ float xw_acc[4][HW][TS > 1 ? D : 1];

  const int part = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tg = lane >> 3, sub = lane & 7;
  const int L = a.seq_lens[b];
  const int start = a.window > 0 ? max(0, L - a.window) : 0;
  if (L <= 0) return;
  const int p_first = start / kPartTokens, p_last = (L - 1) / kPartTokens;
  if (part < p_first || part > p_last) return;
  const int lo = max(start, part * kPartTokens);
  const int hi = min(L, (part + 1) * kPartTokens);
  const int pg_lo = lo / kPage, pg_hi = (hi - 1) / kPage;
  const int npages = pg_hi - pg_lo + 1;

  const int head0 = (G >= 4) ? warp * HW : warp / TS;  // first head (within group) of this warp
  const int tw = (G >= 4) ? 0 : warp % TS;             // token slice of this warp

  // q (pre-scaled into the log2 domain unless softcap is used)
  float q[HW][DL];
  const float kscale = a.k_scale ? a.k_scale[kvh] : 1.f;
  const float qmul = (a.softcap > 0.f ? a.scale : a.scale * kLog2e) * kscale;
#pragma unroll
  for (int h = 0; h < HW; ++h) {
    const __nv_bfloat16* qp = a.q + ((size_t)b * a.H + kvh * G + head0 + h) * D + sub * DL;
#pragma unroll
    for (int d = 0; d < DL; ++d) q[h][d] = bf2f(qp[d]) * qmul;
  }
  float m[HW], l[HW], acc[HW][DL];
#pragma unroll
  for (int h = 0; h < HW; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) acc[h][d] = 0.f;
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
  auto issue = [&](int i) {
    const int s = i % kStages;
    const int64_t page = checked_page(pt, pg_lo + i, a.ld_pt, a.num_pages);
    const size_t off = ((size_t)page * a.KVH + kvh) * kPage * D;
    mbar_arrive_expect_tx(bar0 + 8 * s, 2 * kPageBytes);
    bulk_copy_g2s(smem_u32(ring[s][0]), kc + off, kPageBytes, bar0 + 8 * s);
    bulk_copy_g2s(smem_u32(ring[s][1]), vc + off, kPageBytes, bar0 + 8 * s);
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kStages, npages); ++i) issue(i);

  bool ok = true;
  for (int i = 0; i < npages; ++i) {
    const int s = i % kStages;
    if (ok && !mbar_wait(bar0 + 8 * s, (i / kStages) & 1, kErrAttnWait)) ok = false;
    const KVT* ks = reinterpret_cast<const KVT*>(ring[s][0]);
    const KVT* vs = reinterpret_cast<const KVT*>(ring[s][1]);
    const int pos0 = (pg_lo + i) * kPage;
    if (ok) {
#pragma unroll
      for (int j = 0; j < TPG; ++j) {
        const int tok = tw * TPW + tg + 4 * j;  // token within page
        const int pos = pos0 + tok;
        // every lane runs the shuffles below; out-of-range tokens skip only the update
        const bool valid = pos >= lo && pos < hi;
        float kv[DL];
        load_kv_vec<KVT, DL>(ks + tok * D + sub * DL, kv);
        float sc[HW];
#pragma unroll
        for (int h = 0; h < HW; ++h) {
          float sdot = 0.f;
#pragma unroll
          for (int d = 0; d < DL; ++d) sdot += q[h][d] * kv[d];
          sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
          sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
          sdot += __shfl_xor_sync(0xffffffffu, sdot, 4);
          if (a.softcap > 0.f) sdot = a.softcap * tanhf(sdot / a.softcap) * kLog2e;
          sc[h] = sdot;
        }
        load_kv_vec<KVT, DL>(vs + tok * D + sub * DL, kv);
        if (!valid) continue;
#pragma unroll
        for (int h = 0; h < HW; ++h) {
          const float mn = fmaxf(m[h], sc[h]);
          const float corr = exp2f(m[h] - mn);  // m == -inf -> 0
          const float p = exp2f(sc[h] - mn);
          l[h] = l[h] * corr + p;
#pragma unroll
          for (int d = 0; d < DL; ++d) acc[h][d] = acc[h][d] * corr + p * kv[d];
          m[h] = mn;
        }
      }
    }
    __syncthreads();  // everyone is done with stage s
    if (threadIdx.x == 0 && ok && i + kStages < npages) issue(i + kStages);
  }

  // combine the 4 token groups of the warp (lanes with equal `sub`)
#pragma unroll
  for (int h = 0; h < HW; ++h) {
#pragma unroll
    for (int o = 8; o <= 16; o <<= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[h], o);
      const float lo_ = __shfl_xor_sync(0xffffffffu, l[h], o);
      const float mn = fmaxf(m[h], mo);
      const float c0 = (m[h] == -INFINITY) ? 0.f : exp2f(m[h] - mn);
      const float c1 = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
      l[h] = l[h] * c0 + lo_ * c1;
#pragma unroll
      for (int d = 0; d < DL; ++d) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[h][d], o);
        acc[h][d] = acc[h][d] * c0 + ao * c1;
      }
      m[h] = mn;
    }
  }
  // combine warps sharing a head (only when G < 4)
  if constexpr (TS > 1) {
    if (tg == 0) {
#pragma unroll
      for (int h = 0; h < HW; ++h) {
        if (sub == 0) {
          xw_m[warp][h] = m[h];
          xw_l[warp][h] = l[h];
        }
#pragma unroll
        for (int d = 0; d < DL; ++d) xw_acc[warp][h][sub * DL + d] = acc[h][d];
      }
    }
    __syncthreads();
    if (tw != 0) return;
    for (int w2 = warp + 1; w2 < warp + TS; ++w2) {
#pragma unroll
      for (int h = 0; h < HW; ++h) {
        const float mo = xw_m[w2][h], lo_ = xw_l[w2][h];
        const float mn = fmaxf(m[h], mo);
        const float c0 = (m[h] == -INFINITY) ? 0.f : exp2f(m[h] - mn);
        const float c1 = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
        l[h] = l[h] * c0 + lo_ * c1;
#pragma unroll
        for (int d = 0; d < DL; ++d) acc[h][d] = acc[h][d] * c0 + xw_acc[w2][h][sub * DL + d] * c1;
        m[h] = mn;
      }
    }
  }
  if (tg != 0) return;
  const float vscale = a.v_scale ? a.v_scale[kvh] : 1.f;
#pragma unroll
  for (int h = 0; h < HW; ++h) {
    const int head = kvh * G + head0 + h;
    const size_t pidx = ((size_t)b * a.H + head) * a.max_parts + part;
    float* dst = a.part_acc + pidx * D + sub * DL;
#pragma unroll
    for (int d = 0; d < DL; ++d) dst[d] = acc[h][d] * vscale;
    if (sub == 0) {
      a.part_ml[pidx * 2 + 0] = m[h];
      a.part_ml[pidx * 2 + 1] = l[h];
    }
  }
}

// ---------------------------------------------------------------------------
// Page-stream variant (the default). The 4 warps of a CTA form HG head groups
// x PS page streams (HG * PS = 4). Each stream owns a private 2-stage ring of
// K/V pages filled by the bulk-copy engine and consumes every PS-th page of
// the partition; a warp holds HW = G / HG query heads, so shared memory is
// read once per page per head group. Within a warp, 4 token groups of 8
// lanes take 4 tokens of a page each and apply one online-softmax update per
// 4 tokens.
// ---------------------------------------------------------------------------
template <int D, int G>
struct StreamCfg {
  static constexpr int DL = D / 8;
  static constexpr int HG = (G * DL <= 64) ? 1 : (G * DL <= 128 ? 2 : 4);
  static constexpr int HW = G / HG;
  static constexpr int PS = 4 / HG;
  static constexpr int NST = 2;
};

template <int D, int G, typename KVT>
__global__ void __launch_bounds__(128) paged_decode_stream_kernel(DecodeArgs a) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  using C = StreamCfg<D, G>;
  constexpr int DL = C::DL, HG = C::HG, HW = C::HW, PS = C::PS, NST = C::NST;
  constexpr int kPageBytes = kPage * D * (int)sizeof(KVT);
  static_assert(HW >= 1 && HG * HW == G, "head split");

  extern __shared__ __align__(128) uint8_t ring_raw[];  // [PS][NST][2][kPageBytes]
  __shared__ __align__(8) uint64_t full_bar[PS][NST];
  __shared__ __align__(8) uint64_t empty_bar[PS][NST];
  __shared__ float xw_m[4][HW], xw_l[4][HW];
  __shared__ float xw_acc[4][HW][PS > 1 ? D : 1];

  const int part = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tg = lane >> 3, sub = lane & 7;
  const int hg = warp / PS, ps = warp % PS;
  const int L = a.seq_lens[b];
  const int start = a.window > 0 ? max(0, L - a.window) : 0;
  if (L <= 0) return;
  const int p_first = start / kPartTokens, p_last = (L - 1) / kPartTokens;
  if (part < p_first || part > p_last) return;
  const int lo = max(start, part * kPartTokens);
  const int hi = min(L, (part + 1) * kPartTokens);
  const int pg_lo = lo / kPage, pg_hi = (hi - 1) / kPage;
  const int npages = pg_hi - pg_lo + 1;
  const int my_pages = npages > ps ? (npages - ps + PS - 1) / PS : 0;  // pages ps, ps+PS, ...

  float q[HW][DL];
  const float kscale = a.k_scale ? a.k_scale[kvh] : 1.f;
  const float qmul = (a.softcap > 0.f ? a.scale : a.scale * kLog2e) * kscale;
#pragma unroll
  for (int h = 0; h < HW; ++h) {
    const __nv_bfloat16* qp = a.q + ((size_t)b * a.H + kvh * G + hg * HW + h) * D + sub * DL;
#pragma unroll
    for (int d = 0; d < DL; d += 8) {
      uint4 u = *reinterpret_cast<const uint4*>(qp + d);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h2[j]);
        q[h][d + 2 * j] = f.x * qmul;
        q[h][d + 2 * j + 1] = f.y * qmul;
      }
    }
  }
  float m[HW], l[HW], acc[HW][DL];
#pragma unroll
  for (int h = 0; h < HW; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) acc[h][d] = 0.f;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < PS; ++s)
      for (int t = 0; t < NST; ++t) {
        mbar_init(smem_u32(&full_bar[s][t]), 1);
        mbar_init(smem_u32(&empty_bar[s][t]), HG);
      }
    fence_barrier_init();
  }
  __syncthreads();

  const KVT* kc = reinterpret_cast<const KVT*>(a.k_cache);
  const KVT* vc = reinterpret_cast<const KVT*>(a.v_cache);
  const int* pt = a.page_table + (size_t)b * a.ld_pt;
  uint8_t* my_ring = ring_raw + (size_t)ps * NST * 2 * kPageBytes;
  const bool producer = (hg == 0 && lane == 0);
  auto issue = [&](int i) {  // i-th page of this stream
    const int s = i % NST;
    const int64_t page = checked_page(pt, pg_lo + ps + i * PS, a.ld_pt, a.num_pages);
    const size_t off = ((size_t)page * a.KVH + kvh) * kPage * D;
    const uint32_t fb = smem_u32(&full_bar[ps][s]);
    mbar_arrive_expect_tx(fb, 2 * kPageBytes);
    bulk_copy_g2s(smem_u32(my_ring + (s * 2 + 0) * kPageBytes), kc + off, kPageBytes, fb);
    bulk_copy_g2s(smem_u32(my_ring + (s * 2 + 1) * kPageBytes), vc + off, kPageBytes, fb);
  };
  if (producer)
    for (int i = 0; i < min(NST, my_pages); ++i) issue(i);

  bool ok = true;
  for (int i = 0; i < my_pages; ++i) {
    const int s = i % NST;
    if (ok && !mbar_wait(smem_u32(&full_bar[ps][s]), (i / NST) & 1, kErrAttnWait)) ok = false;
    if (ok) {
      const KVT* ks = reinterpret_cast<const KVT*>(my_ring + (s * 2 + 0) * kPageBytes);
      const KVT* vs = reinterpret_cast<const KVT*>(my_ring + (s * 2 + 1) * kPageBytes);
      const int pos0 = (pg_lo + ps + i * PS) * kPage;
      float sc[4][HW];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int tok = tg + 4 * t;
        const int pos = pos0 + tok;
        const bool valid = pos >= lo && pos < hi;
        float kv[DL];
        load_kv_vec<KVT, DL>(ks + tok * D + sub * DL, kv);
#pragma unroll
        for (int h = 0; h < HW; ++h) {
          float sd = 0.f;
#pragma unroll
          for (int d = 0; d < DL; ++d) sd += q[h][d] * kv[d];
          sd += __shfl_xor_sync(0xffffffffu, sd, 1);
          sd += __shfl_xor_sync(0xffffffffu, sd, 2);
          sd += __shfl_xor_sync(0xffffffffu, sd, 4);
          if (a.softcap > 0.f) sd = a.softcap * tanhf(sd / a.softcap) * kLog2e;
          sc[t][h] = valid ? sd : -INFINITY;
        }
      }
      float p[4][HW];
#pragma unroll
      for (int h = 0; h < HW; ++h) {
        const float mx = fmaxf(fmaxf(sc[0][h], sc[1][h]), fmaxf(sc[2][h], sc[3][h]));
        const float mn = fmaxf(m[h], mx);
        if (mn == -INFINITY) {
#pragma unroll
          for (int t = 0; t < 4; ++t) p[t][h] = 0.f;
          continue;
        }
        const float corr = exp2f(m[h] - mn);
        float ps_ = 0.f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          p[t][h] = exp2f(sc[t][h] - mn);
          ps_ += p[t][h];
        }
        l[h] = l[h] * corr + ps_;
#pragma unroll
        for (int d = 0; d < DL; ++d) acc[h][d] *= corr;
        m[h] = mn;
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float vv[DL];
        load_kv_vec<KVT, DL>(vs + (tg + 4 * t) * D + sub * DL, vv);
        const int pos = pos0 + tg + 4 * t;
        if (pos < lo || pos >= hi) {  // stale slot of a partial page: never let it reach acc
#pragma unroll
          for (int d = 0; d < DL; ++d) vv[d] = 0.f;
        }
#pragma unroll
        for (int h = 0; h < HW; ++h)
#pragma unroll
          for (int d = 0; d < DL; ++d) acc[h][d] += p[t][h] * vv[d];
      }
    }
    // release the stage; the stream's producer refills it
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty_bar[ps][s]));
    if (producer && ok && i + NST < my_pages) {
      if (!mbar_wait(smem_u32(&empty_bar[ps][s]), (i / NST) & 1, kErrAttnWait)) ok = false;
      else issue(i + NST);
    }
  }

  // combine the 4 token groups of the warp (lanes with equal `sub`)
#pragma unroll
  for (int h = 0; h < HW; ++h) {
#pragma unroll
    for (int o = 8; o <= 16; o <<= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[h], o);
      const float lo_ = __shfl_xor_sync(0xffffffffu, l[h], o);
      const float mn = fmaxf(m[h], mo);
      const float c0 = (m[h] == -INFINITY) ? 0.f : exp2f(m[h] - mn);
      const float c1 = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
      l[h] = l[h] * c0 + lo_ * c1;
#pragma unroll
      for (int d = 0; d < DL; ++d) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[h][d], o);
        acc[h][d] = acc[h][d] * c0 + ao * c1;
      }
      m[h] = mn;
    }
  }
  // combine the PS page streams of each head group, in stream order
  if constexpr (PS > 1) {
    if (tg == 0) {
#pragma unroll
      for (int h = 0; h < HW; ++h) {
        if (sub == 0) {
          xw_m[warp][h] = m[h];
          xw_l[warp][h] = l[h];
        }
#pragma unroll
        for (int d = 0; d < DL; ++d) xw_acc[warp][h][sub * DL + d] = acc[h][d];
      }
    }
    __syncthreads();
    if (ps != 0) return;
    for (int w2 = warp + 1; w2 < warp + PS; ++w2) {
#pragma unroll
      for (int h = 0; h < HW; ++h) {
        const float mo = xw_m[w2][h], lo_ = xw_l[w2][h];
        const float mn = fmaxf(m[h], mo);
        const float c0 = (m[h] == -INFINITY) ? 0.f : exp2f(m[h] - mn);
        const float c1 = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
        l[h] = l[h] * c0 + lo_ * c1;
#pragma unroll
        for (int d = 0; d < DL; ++d) acc[h][d] = acc[h][d] * c0 + xw_acc[w2][h][sub * DL + d] * c1;
        m[h] = mn;
      }
    }
  }
  if (tg != 0) return;
  const float vscale = a.v_scale ? a.v_scale[kvh] : 1.f;
#pragma unroll
  for (int h = 0; h < HW; ++h) {
    const int head = kvh * G + hg * HW + h;
    const size_t pidx = ((size_t)b * a.H + head) * a.max_parts + part;
    float* dst = a.part_acc + pidx * D + sub * DL;
#pragma unroll
    for (int d = 0; d < DL; d += 4)
      *reinterpret_cast<float4*>(dst + d) =
          make_float4(acc[h][d] * vscale, acc[h][d + 1] * vscale, acc[h][d + 2] * vscale, acc[h][d + 3] * vscale);
    if (sub == 0) {
      a.part_ml[pidx * 2 + 0] = m[h];
      a.part_ml[pidx * 2 + 1] = l[h];
    }
  }
}

// One warp per (row, head); 4 warps per CTA. Writes bf16 output.
template <int D>
__global__ void __launch_bounds__(128) paged_decode_merge_kernel(DecodeArgs a, int B) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  constexpr int DL = D / 32 > 0 ? D / 32 : 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gi = blockIdx.x * 4 + warp;
  if (gi >= B * a.H) return;
  const int b = gi / a.H;
  const int L = a.seq_lens[b];
  const int start = a.window > 0 ? max(0, L - a.window) : 0;
  const int p_first = start / kPartTokens, p_last = L > 0 ? (L - 1) / kPartTokens : -1;
  {
    const int h = gi % a.H;
    __nv_bfloat16* o = a.out + ((size_t)b * a.H + h) * D;
    if (L <= 0) {
      for (int d = lane; d < D; d += 32) o[d] = f2bf(0.f);
      return;
    }
    const size_t base = ((size_t)b * a.H + h) * a.max_parts;
    float M = a.sinks ? a.sinks[h] * kLog2e : -INFINITY;
    for (int p = p_first; p <= p_last; ++p) M = fmaxf(M, a.part_ml[(base + p) * 2]);
    float den = a.sinks ? exp2f(a.sinks[h] * kLog2e - M) : 0.f;
    float accv[DL];
#pragma unroll
    for (int j = 0; j < DL; ++j) accv[j] = 0.f;
    for (int p = p_first; p <= p_last; ++p) {
      const float mp = a.part_ml[(base + p) * 2];
      const float w = (mp == -INFINITY) ? 0.f : exp2f(mp - M);
      den += a.part_ml[(base + p) * 2 + 1] * w;
      const float* src = a.part_acc + (base + p) * D;
#pragma unroll
      for (int j = 0; j < DL; ++j) {
        const int d = lane + 32 * j;
        if (d < D) accv[j] += src[d] * w;
      }
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
    for (int j = 0; j < DL; ++j) {
      const int d = lane + 32 * j;
      if (d < D) o[d] = f2bf(accv[j] * inv);
    }
  }
}

template <int D, int G, typename KVT>
static int launch_decode(const DecodeArgs& a, int B, cudaStream_t st) {
  using C = StreamCfg<D, G>;
  constexpr int smem = C::PS * C::NST * 2 * kPage * D * (int)sizeof(KVT);
  if (int e = b200::smem_attr_once<paged_decode_stream_kernel<D, G, KVT>>(smem)) return e;
  dim3 grid(a.max_parts, a.KVH, B);
b200::launch_k(  paged_decode_stream_kernel<D, G, KVT>, dim3(grid), dim3(128), smem, st, 1, a);
b200::launch_k(  paged_decode_merge_kernel<D>, dim3((B * a.H + 3) / 4), dim3(128), 0, st, 1, a, B);
  return (int)cudaGetLastError();
}

template <int D, typename KVT>
static int dispatch_g(const DecodeArgs& a, int B, int G, cudaStream_t st) {
  switch (G) {
    case 1: return launch_decode<D, 1, KVT>(a, B, st);
    case 2: return launch_decode<D, 2, KVT>(a, B, st);
    case 4: return launch_decode<D, 4, KVT>(a, B, st);
    case 8: return launch_decode<D, 8, KVT>(a, B, st);
    case 16: return launch_decode<D, 16, KVT>(a, B, st);
    default: return -1;
  }
}

}  // namespace b200

using namespace b200;

extern "C" {

int b200_paged_decode_part_tokens() { return kPartTokens; }

// Merge pass alone (used after the tensor-core partition pass).
int b200_paged_decode_merge(const float* part_acc, const float* part_ml, const int* seq_lens, const float* sinks,
                            void* out, int B, int H, int D, int max_parts, int window, cudaStream_t st) {
  if (B <= 0) return 0;
  DecodeArgs a = {};
  a.seq_lens = seq_lens;
  a.sinks = sinks;
  a.part_acc = const_cast<float*>(part_acc);
  a.part_ml = const_cast<float*>(part_ml);
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.H = H;
  a.max_parts = max_parts;
  a.window = window;
  cudaError_t e;
  const dim3 grid((B * H + 3) / 4);
  switch (D) {
    case 64: e = launch_k(paged_decode_merge_kernel<64>, grid, dim3(128), 0, st, 1, a, B); break;
    case 128: e = launch_k(paged_decode_merge_kernel<128>, grid, dim3(128), 0, st, 1, a, B); break;
    case 256: e = launch_k(paged_decode_merge_kernel<256>, grid, dim3(128), 0, st, 1, a, B); break;
    case 512: e = launch_k(paged_decode_merge_kernel<512>, grid, dim3(128), 0, st, 1, a, B); break;
    default: return -1;
  }
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// Scratch needed: part_acc B*H*max_parts*D floats, part_ml B*H*max_parts*2 floats.
int b200_paged_decode(const void* q, const void* k_cache, const void* v_cache, int kv_fp8, const float* k_scale,
                      const float* v_scale, const int* page_table, int ld_pt, const int* seq_lens,
                      const float* sinks, void* out, float* part_acc, float* part_ml, int B, int H, int KVH, int D,
                      int max_parts, int window, float scale, float softcap, int64_t num_pages, cudaStream_t st) {
  if (B <= 0) return 0;
  if (H % KVH) return -1;
  DecodeArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.page_table = page_table;
  a.seq_lens = seq_lens;
  a.sinks = sinks;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.part_acc = part_acc;
  a.part_ml = part_ml;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.H = H;
  a.KVH = KVH;
  a.ld_pt = ld_pt;
  a.max_parts = max_parts;
  a.window = window;
  a.num_pages = num_pages;
  a.scale = scale;
  a.softcap = softcap;
  const int G = H / KVH;
  if (kv_fp8) {
    switch (D) {
      case 64: return dispatch_g<64, uint8_t>(a, B, G, st);
      case 128: return dispatch_g<128, uint8_t>(a, B, G, st);
      case 256: return dispatch_g<256, uint8_t>(a, B, G, st);
      default: return -1;
    }
  }
  switch (D) {
    case 64: return dispatch_g<64, __nv_bfloat16>(a, B, G, st);
    case 128: return dispatch_g<128, __nv_bfloat16>(a, B, G, st);
    case 256: return dispatch_g<256, __nv_bfloat16>(a, B, G, st);
    default: return -1;
  }
}

}  // extern "C"

B200_STATUS_ACCESSORS(attn_decode)

// ---------------------------------------------------------------------------
// Variant of b200_paged_decode whose scratch is compiled into the library; it
// allocates no device memory. Contract, size limit and concurrency rules are
// in attention_decode_noalloc.h.
#include <mutex>

#include "attention_decode_noalloc.h"

namespace {

static __device__ __align__(256) float g_decode_noalloc_scratch[B200_DECODE_NOALLOC_SCRATCH_FLOATS];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of this device's scratch array; looked up once per device,
// with that device current, by the first call made on it.
int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return -1;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int b200_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, int kv_fp8,
                                         const float* k_scale, const float* v_scale, const int* page_table,
                                         int ld_pt, const int* seq_lens, const float* sinks, void* out, int B, int H,
                                         int KVH, int D, int max_parts, int window, float scale, float softcap,
                                         int64_t num_pages, cudaStream_t st) {
  if (B <= 0) return 0;
  if (H <= 0 || KVH <= 0 || H % KVH || max_parts <= 0) return -1;
  if (D != 64 && D != 128 && D != 256) return -1;
  const int64_t slots = (int64_t)B * H * max_parts;
  const int64_t acc_floats = (slots * D + 63) / 64 * 64;  // keeps part_ml on a 256-byte boundary
  if (acc_floats + slots * 2 > (int64_t)B200_DECODE_NOALLOC_SCRATCH_FLOATS) return B200_DECODE_NOALLOC_TOO_LARGE;
  float* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != 0) return rc;
  float* part_acc = scratch;
  float* part_ml = scratch + acc_floats;
  DecodeArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.page_table = page_table;
  a.seq_lens = seq_lens;
  a.sinks = sinks;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.part_acc = part_acc;
  a.part_ml = part_ml;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.H = H;
  a.KVH = KVH;
  a.ld_pt = ld_pt;
  a.max_parts = max_parts;
  a.window = window;
  a.num_pages = num_pages;
  a.scale = scale;
  a.softcap = softcap;
  const int G = H / KVH;
  if (kv_fp8) {
    switch (D) {
      case 64: return dispatch_g<64, uint8_t>(a, B, G, st);
      case 128: return dispatch_g<128, uint8_t>(a, B, G, st);
      default: return dispatch_g<256, uint8_t>(a, B, G, st);
    }
  }
  switch (D) {
    case 64: return dispatch_g<64, __nv_bfloat16>(a, B, G, st);
    case 128: return dispatch_g<128, __nv_bfloat16>(a, B, G, st);
    default: return dispatch_g<256, __nv_bfloat16>(a, B, G, st);
  }
}
