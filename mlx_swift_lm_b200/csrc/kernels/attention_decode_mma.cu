// Paged decode attention on the tensor cores (bf16 KV pages).
//
// Same contract and output as the CUDA-core kernel in attention_decode.cu
// (fixed 256-token partitions in absolute positions -> per-row results are
// independent of batch-mates; partials merged by paged_decode_merge_kernel).
//
// Decode attention is HBM-bound; the tensor core is used here to cut issue
// slots: per 16-token page, the scores S[16 x 16] = Q[16 heads (the GQA group,
// zero-padded) x D] . K^T and the update O += P . V each take D/8 warp MMAs
// (mma.sync m16n8k16 bf16, fp32 accumulate) instead of 16*G*D lane FMAs. The
// per-warp problem (16 x 16 x D per page) is far below the 64/128-row minimum
// tile of tcgen05, so the warp-level MMA is the right unit here.
//
// Each of the 4 warps is an independent page stream: it owns a 2-stage ring of
// K/V pages loaded by TMA with the 128-byte swizzle (so ldmatrix reads are
// bank-conflict free) and consumes every 4th page of the partition. P is kept
// in registers in the A-fragment layout (no shared-memory round trip). At the
// end the 4 streams are combined through shared memory.
#include <cudaTypedefs.h>

#include "b200_common.cuh"

namespace b200 {

bool make_tmap_2d(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows,
                  int box_cols, int dtype_bytes);

namespace mmadec {

constexpr int kPart = 256;
constexpr int kPage = 16;
constexpr int kNst = 2;
constexpr float kLog2e = 1.4426950408889634f;

struct Args {
  const __nv_bfloat16* q;
  const int* page_table;
  const int* seq_lens;
  float* part_acc;
  float* part_ml;
  int H, KVH, ld_pt, max_parts, window;
  int64_t num_pages;
  float scale, softcap;
  // fused merge (null counters: partials only, merged by paged_decode_merge_kernel)
  int* counters;        // [B * KVH] arrival counts, zero between launches (the merging CTA resets its own)
  const float* sinks;   // [H] or null
  __nv_bfloat16* out;   // [B, H, D]
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of (token r, dim d) (d a multiple of 8) in a page tile stored as
// D/64 boxes of [16 rows][128 bytes] with the 128-byte TMA swizzle.
__device__ __forceinline__ uint32_t sw_off(int r, int d) {
  const int half = d >> 6, chunk = (d & 63) >> 3;
  return (uint32_t)(half * (kPage * 128) + r * 128 + ((chunk ^ (r & 7)) << 4));
}

template <int D, int G>
__global__ void __launch_bounds__(128) decode_mma_kernel(const __grid_constant__ CUtensorMap tmK,
                                                         const __grid_constant__ CUtensorMap tmV, Args a) {
  constexpr int NB = D / 64;                       // 64-column boxes per page row
  constexpr int kTile = kPage * D * 2;             // bytes of one K or V page
  constexpr int kWarpRing = kNst * 2 * kTile;      // per-warp ring
  constexpr int NT = D / 8;                        // 8-wide n tiles of O
  static_assert(G <= 16 && D % 64 == 0, "shape");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[4][kNst];
  __shared__ float xm[4][16], xl[4][16];

  pdl_launch_dependents();
  const int part = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    for (int w = 0; w < 4; ++w)
      for (int s = 0; s < kNst; ++s) mbar_init(smem_u32(&full_bar[w][s]), 1);
    fence_barrier_init();
  }
  pdl_wait();
  const int L = a.seq_lens[b];
  const int start = a.window > 0 ? max(0, L - a.window) : 0;
  if (L <= 0) {
    // an empty row (graph padding): its output is zero, written once
    if (a.counters && part == 0)
      for (int e = threadIdx.x; e < G * D; e += 128)
        a.out[((size_t)b * a.H + kvh * G + e / D) * D + e % D] = f2bf(0.f);
    return;
  }
  const int p_first = start / kPart, p_last = (L - 1) / kPart;
  if (part < p_first || part > p_last) return;
  __syncthreads();
  const int lo = max(start, part * kPart);
  const int hi = min(L, (part + 1) * kPart);
  const int pg_lo = lo / kPage, pg_hi = (hi - 1) / kPage;
  const int npages = pg_hi - pg_lo + 1;
  const int my_pages = npages > warp ? (npages - warp + 3) / 4 : 0;

  // Q fragments (rows = heads of the group, zero beyond G), unscaled bf16
  uint32_t qa[D / 16][4];
  {
    const __nv_bfloat16* qb = a.q + ((size_t)b * a.H + kvh * G) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int c0 = ks * 16 + 2 * t4;
      qa[ks][0] = (g < G) ? *reinterpret_cast<const uint32_t*>(qb + g * D + c0) : 0u;
      qa[ks][1] = (g + 8 < G) ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + c0) : 0u;
      qa[ks][2] = (g < G) ? *reinterpret_cast<const uint32_t*>(qb + g * D + c0 + 8) : 0u;
      qa[ks][3] = (g + 8 < G) ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * D + c0 + 8) : 0u;
    }
  }
  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g and g+8
  const float smul = a.softcap > 0.f ? a.scale : a.scale * kLog2e;

  uint8_t* ring = smem + warp * kWarpRing;
  const uint32_t ring_s = smem_u32(ring);
  const int* pt = a.page_table + (size_t)b * a.ld_pt;
  auto issue = [&](int i) {
    const int s = i % kNst;
    const int64_t page = checked_page(pt, pg_lo + warp + 4 * i, a.ld_pt, a.num_pages);
    const int row = (int)((page * a.KVH + kvh) * kPage);
    const uint32_t fb = smem_u32(&full_bar[warp][s]);
    mbar_arrive_expect_tx(fb, 2 * kTile);
    const uint32_t kd = ring_s + s * 2 * kTile, vd = kd + kTile;
#pragma unroll
    for (int bx = 0; bx < NB; ++bx) {
      tma_load_2d(kd + bx * kPage * 128, &tmK, fb, bx * 64, row, 0ull);
      tma_load_2d(vd + bx * kPage * 128, &tmV, fb, bx * 64, row, 0ull);
    }
  };
  // TMA cache hints are not used for KV pages (they are read once per step)
  if (lane == 0)
    for (int i = 0; i < min(kNst, my_pages); ++i) issue(i);

  bool ok = true;
  for (int i = 0; i < my_pages; ++i) {
    const int s = i % kNst;
    if (ok && !mbar_wait(smem_u32(&full_bar[warp][s]), (i / kNst) & 1, kErrAttnWait)) ok = false;
    if (ok) {
      const uint32_t kbase = ring_s + s * 2 * kTile, vbase = kbase + kTile;
      const int pos0 = (pg_lo + warp + 4 * i) * kPage;
      // ---- S = Q K^T ----
      float sc[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
      const int mrow = lane & 7, mat = lane >> 3;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t b00, b01, b10, b11;
        const int tok = (mat >= 2 ? 8 : 0) + mrow;
        const int dim = ks * 16 + (mat & 1) * 8;
        ldsm_x4(kbase + sw_off(tok, dim), b00, b01, b10, b11);
        mma_bf16(sc[0], qa[ks], b00, b01);
        mma_bf16(sc[1], qa[ks], b10, b11);
      }
      // ---- online softmax (rows g, g+8; columns = tokens) ----
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int tok = n * 8 + 2 * t4 + c;
          const bool valid = (pos0 + tok) >= lo && (pos0 + tok) < hi;
          float v0 = sc[n][c] * smul, v1 = sc[n][2 + c] * smul;
          if (a.softcap > 0.f) {
            v0 = a.softcap * tanhf(v0 / a.softcap) * kLog2e;
            v1 = a.softcap * tanhf(v1 / a.softcap) * kLog2e;
          }
          sc[n][c] = valid ? v0 : -INFINITY;
          sc[n][2 + c] = valid ? v1 : -INFINITY;
          mx0 = fmaxf(mx0, sc[n][c]);
          mx1 = fmaxf(mx1, sc[n][2 + c]);
        }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float c0 = (mn0 == -INFINITY) ? 1.f : exp2f(m0 - mn0);
      const float c1 = (mn1 == -INFINITY) ? 1.f : exp2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      uint32_t pa[4];
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const float p00 = (mn0 == -INFINITY) ? 0.f : exp2f(sc[n][0] - mn0);
        const float p01 = (mn0 == -INFINITY) ? 0.f : exp2f(sc[n][1] - mn0);
        const float p10 = (mn1 == -INFINITY) ? 0.f : exp2f(sc[n][2] - mn1);
        const float p11 = (mn1 == -INFINITY) ? 0.f : exp2f(sc[n][3] - mn1);
        ps0 += p00 + p01;
        ps1 += p10 + p11;
        pa[2 * n + 0] = pack_bf16x2(p00, p01);
        pa[2 * n + 1] = pack_bf16x2(p10, p11);
      }
      l0 = l0 * c0 + ps0;
      l1 = l1 * c1 + ps1;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        o[j][0] *= c0;
        o[j][1] *= c0;
        o[j][2] *= c1;
        o[j][3] *= c1;
      }
      // ---- O += P V ----
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        uint32_t b0a, b1a, b0b, b1b;
        const int tok = (mat & 1) * 8 + mrow;
        const int dim = (j + (mat >> 1)) * 8;
        ldsm_x4_t(vbase + sw_off(tok, dim), b0a, b1a, b0b, b1b);
        mma_bf16(o[j], pa, b0a, b1a);
        mma_bf16(o[j + 1], pa, b0b, b1b);
      }
    }
    __syncwarp();
    if (lane == 0 && ok && i + kNst < my_pages) {
      fence_proxy_async_smem();
      issue(i + kNst);
    }
  }
  // row sums across the quad
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // ---- combine the 4 page streams through shared memory ----
  __syncthreads();  // all rings are drained; reuse them for the combine buffer
  float* xo = reinterpret_cast<float*>(smem);  // [4][G][D]
  if (t4 == 0) {
    if (g < G) {
      xm[warp][g] = m0;
      xl[warp][g] = l0;
    }
    if (g + 8 < G) {
      xm[warp][g + 8] = m1;
      xl[warp][g + 8] = l1;
    }
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + 2 * t4;
    if (g < G) {
      xo[(warp * G + g) * D + d] = o[j][0];
      xo[(warp * G + g) * D + d + 1] = o[j][1];
    }
    if (g + 8 < G) {
      xo[(warp * G + g + 8) * D + d] = o[j][2];
      xo[(warp * G + g + 8) * D + d + 1] = o[j][3];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += 128) {
    const int row = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, xm[w][row]);
    float acc = 0.f, Ls = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = xm[w][row];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      acc += xo[(w * G + row) * D + d] * f;
      Ls += xl[w][row] * f;
    }
    const size_t pidx = ((size_t)b * a.H + kvh * G + row) * a.max_parts + part;
    a.part_acc[pidx * D + d] = acc;
    if (d == 0) {
      a.part_ml[pidx * 2 + 0] = M;
      a.part_ml[pidx * 2 + 1] = Ls;
    }
  }
  if (!a.counters) return;
  // ---- fused merge: the last of the row's live partitions to finish merges
  // all of them, in partition order (the same sums as the separate merge pass)
  __shared__ int s_last;
  __threadfence();  // publish this CTA's partials before counting it
  __syncthreads();
  if (threadIdx.x == 0) {
    const int n_live = p_last - p_first + 1;
    int* cnt = a.counters + (size_t)b * a.KVH + kvh;
    const int prev = atomicAdd(cnt, 1);
    s_last = prev == n_live - 1;
    if (s_last) *cnt = 0;  // ready for the next launch (stream order separates them)
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // see the other CTAs' partials
  // (max, sum) pairs of the G heads' live partitions -> shared memory (the
  // page rings are free now), then per-head weights; partial rows are read
  // with cache-global loads (L1 does not hold other SMs' writes), all issued
  // independently so their L2 latencies overlap
  const int n_live = p_last - p_first + 1;
  if (3 * G * n_live + G > 128 * D) {  // more partitions than the staging area holds: direct loads
    for (int e = threadIdx.x; e < G * D; e += 128) {
      const int row = e / D, d = e % D, h = kvh * G + row;
      const size_t base = ((size_t)b * a.H + h) * a.max_parts;
      float M = a.sinks ? a.sinks[h] * kLog2e : -INFINITY;
      for (int p = p_first; p <= p_last; ++p) M = fmaxf(M, __ldcg(a.part_ml + (base + p) * 2));
      float den = a.sinks ? exp2f(a.sinks[h] * kLog2e - M) : 0.f, accv = 0.f;
      for (int p = p_first; p <= p_last; ++p) {
        const float mp = __ldcg(a.part_ml + (base + p) * 2);
        const float w = (mp == -INFINITY) ? 0.f : exp2f(mp - M);
        den += __ldcg(a.part_ml + (base + p) * 2 + 1) * w;
        accv += __ldcg(a.part_acc + (base + p) * D + d) * w;
      }
      a.out[((size_t)b * a.H + h) * D + d] = f2bf(accv * (den > 0.f ? 1.f / den : 0.f));
    }
    return;
  }
  float* sml = reinterpret_cast<float*>(smem);      // [G][n_live][2]
  float* swt = sml + 2 * G * n_live;                 // [G][n_live] weights
  float* sinv = swt + G * n_live;                    // [G] 1 / denominator
  for (int e = threadIdx.x; e < G * n_live; e += 128) {
    const int row = e / n_live, p = p_first + e % n_live;
    const float2 v = __ldcg(reinterpret_cast<const float2*>(a.part_ml) +
                            ((size_t)b * a.H + kvh * G + row) * a.max_parts + p);
    sml[2 * e] = v.x;
    sml[2 * e + 1] = v.y;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int row = threadIdx.x, h = kvh * G + row;
    float M = a.sinks ? a.sinks[h] * kLog2e : -INFINITY;
    for (int i = 0; i < n_live; ++i) M = fmaxf(M, sml[2 * (row * n_live + i)]);
    float den = a.sinks ? exp2f(a.sinks[h] * kLog2e - M) : 0.f;
    for (int i = 0; i < n_live; ++i) {
      const float mp = sml[2 * (row * n_live + i)];
      const float w = (mp == -INFINITY) ? 0.f : exp2f(mp - M);
      den += sml[2 * (row * n_live + i) + 1] * w;
      swt[row * n_live + i] = w;
    }
    sinv[row] = den > 0.f ? 1.f / den : 0.f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += 128) {
    const int row = e / D, d = e % D;
    const size_t base = ((size_t)b * a.H + kvh * G + row) * a.max_parts;
    float accv = 0.f;
    for (int i = 0; i < n_live; ++i) accv += __ldcg(a.part_acc + (base + p_first + i) * D + d) * swt[row * n_live + i];
    a.out[((size_t)b * a.H + kvh * G + row) * D + d] = f2bf(accv * sinv[row]);
  }
}

template <int D, int G>
int launch(const CUtensorMap& tk, const CUtensorMap& tv, const Args& a, int B, cudaStream_t st) {
  constexpr int smem = 4 * kNst * 2 * kPage * D * 2 + 1024;
  if (int e = smem_attr_once<decode_mma_kernel<D, G>>(smem)) return e;
  cudaError_t e = launch_k(decode_mma_kernel<D, G>, dim3(a.max_parts, a.KVH, B), dim3(128), smem, st, 1, tk, tv, a);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace mmadec
}  // namespace b200

using namespace b200;

// Partition pass only; the merge pass is b200_paged_decode_merge (attention_decode.cu).
extern "C" int b200_paged_decode_mma_part(const void* q, const void* k_cache, const void* v_cache,
                                          const int* page_table, int ld_pt, const int* seq_lens, float* part_acc,
                                          float* part_ml, int B, int H, int KVH, int D, int max_parts, int window,
                                          float scale, float softcap, int64_t num_pages, cudaStream_t st) {
  if (B <= 0) return 0;
  if (H % KVH) return -1;
  const int G = H / KVH;
  CUtensorMap tk, tv;
  const int64_t rows = num_pages * KVH * 16;
  if (!make_tmap_2d(&tk, k_cache, rows, D, D, 16, 64, 2)) return -1;
  if (!make_tmap_2d(&tv, v_cache, rows, D, D, 16, 64, 2)) return -1;
  mmadec::Args a{reinterpret_cast<const __nv_bfloat16*>(q), page_table, seq_lens, part_acc, part_ml, H, KVH, ld_pt,
                 max_parts, window, num_pages, scale, softcap, nullptr, nullptr, nullptr};
#define B200_DEC(DD, GG) \
  if (D == DD && G == GG) return mmadec::launch<DD, GG>(tk, tv, a, B, st);
  B200_DEC(64, 1) B200_DEC(64, 2) B200_DEC(64, 4) B200_DEC(64, 8) B200_DEC(64, 16)
  B200_DEC(128, 1) B200_DEC(128, 2) B200_DEC(128, 4) B200_DEC(128, 8) B200_DEC(128, 16)
  B200_DEC(256, 1) B200_DEC(256, 2) B200_DEC(256, 4) B200_DEC(256, 8)
#undef B200_DEC
  return -1;
}

// Partition pass with the merge fused in: the last CTA of each (row, KV head)
// to finish merges the row's partitions in partition order and writes `out`.
// `counters` [B * KVH] int32 must be zero at the first call; every call leaves
// it zero again.
extern "C" int b200_paged_decode_mma(const void* q, const void* k_cache, const void* v_cache,
                                          const int* page_table, int ld_pt, const int* seq_lens, float* part_acc,
                                          float* part_ml, int* counters, const float* sinks, void* out, int B, int H, int KVH,
                                     int D, int max_parts, int window,
                                          float scale, float softcap, int64_t num_pages, cudaStream_t st) {
  if (B <= 0) return 0;
  if (H % KVH || !counters || !out) return -1;
  const int G = H / KVH;
  CUtensorMap tk, tv;
  const int64_t rows = num_pages * KVH * 16;
  if (!make_tmap_2d(&tk, k_cache, rows, D, D, 16, 64, 2)) return -1;
  if (!make_tmap_2d(&tv, v_cache, rows, D, D, 16, 64, 2)) return -1;
  mmadec::Args a{reinterpret_cast<const __nv_bfloat16*>(q), page_table, seq_lens, part_acc, part_ml, H, KVH, ld_pt,
                 max_parts, window, num_pages, scale, softcap, counters, sinks,
                 reinterpret_cast<__nv_bfloat16*>(out)};
#define B200_DEC(DD, GG) \
  if (D == DD && G == GG) return mmadec::launch<DD, GG>(tk, tv, a, B, st);
  B200_DEC(64, 1) B200_DEC(64, 2) B200_DEC(64, 4) B200_DEC(64, 8) B200_DEC(64, 16)
  B200_DEC(128, 1) B200_DEC(128, 2) B200_DEC(128, 4) B200_DEC(128, 8) B200_DEC(128, 16)
  B200_DEC(256, 1) B200_DEC(256, 2) B200_DEC(256, 4) B200_DEC(256, 8)
#undef B200_DEC
  return -1;
}

B200_STATUS_ACCESSORS(attn_decode_mma)
