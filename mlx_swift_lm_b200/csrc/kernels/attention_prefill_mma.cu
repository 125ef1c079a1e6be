// Paged prefill attention on the tensor cores (bf16 KV pages, head dim 64 /
// 128 / 256).
//
// Same contract as the CUDA-core kernel in attention_prefill_simt.cu: causal
// attention of each row's prefill chunk against the row's paged KV history
// (which already holds the chunk's own K/V), sliding windows from absolute
// positions, learned sinks in the denominator only, optional logit softcap.
// Reference behaviour: gather pages, then SDPA
// (ContinuousBatchingV2/Paged/PagedLayerCache.swift:584-637).
//
// Work unit (CTA): 64 consecutive queries of one row x one query head; warp w
// owns query rows 16w..16w+15 and keeps its Q fragments, the online-softmax
// state and the O accumulator (D/8 n-tiles) in registers. The KV pages of the
// head's KV group stream through a 4-stage shared ring filled by TMA with the
// 128-byte swizzle (ldmatrix reads are bank-conflict free); per 16-key page a
// warp computes S = Q K^T (2 x D/16 mma.sync m16n8k16) and O += P V
// (D/8 mma.sync, V fragments via ldmatrix.trans, P kept in registers in the
// A-fragment layout). Pages past the tile's last query, or before its window,
// are never loaded.
#include <cudaTypedefs.h>

#include "b200_common.cuh"

namespace b200 {

bool make_tmap_2d(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows,
                  int box_cols, int dtype_bytes);

namespace mmapf {

constexpr int kPage = 16;
constexpr int kNst = 4;
constexpr int kQT = 64;  // queries per CTA
constexpr float kLog2e = 1.4426950408889634f;

struct Args {
  const __nv_bfloat16* q;   // [T, H, D]
  const int* page_table;    // [R, ld_pt]
  const int* cu_q;          // [R+1]
  const int* q_pos0;        // [R]
  const int* tiles;         // [n_tiles, 2] (row, q offset)
  const float* sinks;       // [H] or null
  __nv_bfloat16* out;       // [T, H, D]
  int H, KVH, ld_pt, window;
  int64_t num_pages;
  float scale, softcap;
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

template <int D>
__global__ void __launch_bounds__(128) prefill_mma_kernel(const __grid_constant__ CUtensorMap tmK,
                                                          const __grid_constant__ CUtensorMap tmV, Args a) {
  constexpr int NB = D / 64;
  constexpr int kTile = kPage * D * 2;  // bytes of one K or V page (one KV head)
  constexpr int NT = D / 8;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[kNst], empty_bar[kNst];

  pdl_launch_dependents();
  const int tile = blockIdx.x, head = blockIdx.y;
  const int kvh = head / (a.H / a.KVH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    for (int s = 0; s < kNst; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 4);  // one arrive per warp
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  const int row = a.tiles[2 * tile], qoff = a.tiles[2 * tile + 1];
  const int q0 = a.cu_q[row], qlen = a.cu_q[row + 1] - q0;
  const int pos0 = a.q_pos0[row];
  const int nq = min(kQT, qlen - qoff);  // queries of this tile
  if (nq <= 0) return;
  // window < 0: bidirectional (encoders) - every query sees the row's keys
  // [0, pos0 + qlen); else causal, with a sliding window when window > 0.
  const bool bidir = a.window < 0;
  // key range of the tile: [k_lo, k_hi] (absolute positions, inclusive)
  const int k_hi = bidir ? pos0 + qlen - 1 : pos0 + qoff + nq - 1;
  const int k_lo = a.window > 0 ? max(0, pos0 + qoff - a.window + 1) : 0;
  const int pg_lo = k_lo / kPage, pg_hi = k_hi / kPage;
  const int npages = pg_hi - pg_lo + 1;

  // this warp's query rows: r0 = 16*warp + g, r1 = r0 + 8
  const int r0 = warp * 16 + g, r1 = r0 + 8;
  const bool v0 = r0 < nq, v1 = r1 < nq;
  const int qp0 = pos0 + qoff + r0, qp1 = pos0 + qoff + r1;  // absolute positions
  uint32_t qa[D / 16][4];
  {
    const __nv_bfloat16* qb0 = a.q + ((size_t)(q0 + qoff + r0) * a.H + head) * D;
    const __nv_bfloat16* qb1 = a.q + ((size_t)(q0 + qoff + r1) * a.H + head) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int c0 = ks * 16 + 2 * t4;
      qa[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(qb0 + c0) : 0u;
      qa[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(qb1 + c0) : 0u;
      qa[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(qb0 + c0 + 8) : 0u;
      qa[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(qb1 + c0 + 8) : 0u;
    }
  }
  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float smul = a.softcap > 0.f ? a.scale : a.scale * kLog2e;
  // first / last key position this warp's rows can see (for page skipping)
  const int w_hi = bidir ? k_hi : pos0 + qoff + min(nq - 1, warp * 16 + 15);
  const int lim0 = bidir ? k_hi : qp0, lim1 = bidir ? k_hi : qp1;  // last visible key of each row
  const int w_lo = a.window > 0 ? max(0, pos0 + qoff + warp * 16 - a.window + 1) : 0;

  const uint32_t ring_s = smem_u32(smem);
  const int* pt = a.page_table + (size_t)row * a.ld_pt;
  auto issue = [&](int i) {
    const int s = i % kNst;
    const int64_t page = checked_page(pt, pg_lo + i, a.ld_pt, a.num_pages);
    const int krow = (int)((page * a.KVH + kvh) * kPage);
    const uint32_t fb = smem_u32(&full_bar[s]);
    mbar_arrive_expect_tx(fb, 2 * kTile);
    const uint32_t kd = ring_s + s * 2 * kTile, vd = kd + kTile;
#pragma unroll
    for (int bx = 0; bx < NB; ++bx) {
      tma_load_2d(kd + bx * kPage * 128, &tmK, fb, bx * 64, krow, 0ull);
      tma_load_2d(vd + bx * kPage * 128, &tmV, fb, bx * 64, krow, 0ull);
    }
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kNst, npages); ++i) issue(i);

  bool ok = true;
  const int mrow = lane & 7, mat = lane >> 3;
  for (int i = 0; i < npages; ++i) {
    const int s = i % kNst;
    if (ok && !mbar_wait(smem_u32(&full_bar[s]), (i / kNst) & 1, kErrAttnWait)) ok = false;
    const int kpos0 = (pg_lo + i) * kPage;
    // pages outside this warp's visible range need no math
    if (ok && kpos0 <= w_hi && kpos0 + kPage - 1 >= w_lo) {
      const uint32_t kbase = ring_s + s * 2 * kTile, vbase = kbase + kTile;
      float sc[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t b00, b01, b10, b11;
        const int tok = (mat >= 2 ? 8 : 0) + mrow;
        const int dim = ks * 16 + (mat & 1) * 8;
        ldsm_x4(kbase + sw_off(tok, dim), b00, b01, b10, b11);
        mma_bf16(sc[0], qa[ks], b00, b01);
        mma_bf16(sc[1], qa[ks], b10, b11);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int kp = kpos0 + n * 8 + 2 * t4 + c;
          const bool ok0 = v0 && kp <= lim0 && (a.window <= 0 || kp > qp0 - a.window);
          const bool ok1 = v1 && kp <= lim1 && (a.window <= 0 || kp > qp1 - a.window);
          float x0 = sc[n][c] * smul, x1 = sc[n][2 + c] * smul;
          if (a.softcap > 0.f) {
            x0 = a.softcap * tanhf(x0 / a.softcap) * kLog2e;
            x1 = a.softcap * tanhf(x1 / a.softcap) * kLog2e;
          }
          sc[n][c] = ok0 ? x0 : -INFINITY;
          sc[n][2 + c] = ok1 ? x1 : -INFINITY;
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
    // release the stage; thread 0 refills it once all four warps are done
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
    if (threadIdx.x == 0 && ok && i + kNst < npages) {
      if (!mbar_wait(smem_u32(&empty_bar[s]), (i / kNst) & 1, kErrAttnWait)) {
        ok = false;
      } else {
        issue(i + kNst);
      }
    }
    __syncwarp();  // warp 0 reconverges before the next aligned ldmatrix / mma
  }
  // make sure no copy is still landing when the CTA exits
  if (threadIdx.x == 0)
    for (int i = max(0, npages - kNst); i < npages; ++i)
      mbar_wait(smem_u32(&full_bar[i % kNst]), (i / kNst) & 1, kErrAttnWait);

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  float den0 = l0, den1 = l1;
  if (a.sinks) {
    const float sk = a.sinks[head] * kLog2e;
    den0 += (m0 == -INFINITY) ? 0.f : exp2f(sk - m0);
    den1 += (m1 == -INFINITY) ? 0.f : exp2f(sk - m1);
  }
  const float inv0 = den0 > 0.f ? 1.f / den0 : 0.f, inv1 = den1 > 0.f ? 1.f / den1 : 0.f;
  __nv_bfloat16* ob0 = a.out + ((size_t)(q0 + qoff + r0) * a.H + head) * D;
  __nv_bfloat16* ob1 = a.out + ((size_t)(q0 + qoff + r1) * a.H + head) * D;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + 2 * t4;
    if (v0) *reinterpret_cast<uint32_t*>(ob0 + d) = pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
    if (v1) *reinterpret_cast<uint32_t*>(ob1 + d) = pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
  }
}

template <int D>
int launch(const CUtensorMap& tk, const CUtensorMap& tv, const Args& a, int n_tiles, cudaStream_t st) {
  constexpr int smem = kNst * 2 * kPage * D * 2 + 1024;
  if (int e = smem_attr_once<prefill_mma_kernel<D>>(smem)) return e;
  cudaError_t e = launch_k(prefill_mma_kernel<D>, dim3(n_tiles, a.H), dim3(128), smem, st, 1, tk, tv, a);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace mmapf
}  // namespace b200

using namespace b200;

extern "C" {

int b200_prefill_mma_q_tile() { return mmapf::kQT; }

// tiles: [n_tiles, 2] (row, query offset within the row's chunk), offsets
// multiples of b200_prefill_mma_q_tile(). bf16 K/V pages, D in {64, 128, 256}.
int b200_paged_prefill_mma(const void* q, const void* k_cache, const void* v_cache, const int* page_table, int ld_pt,
                           const int* cu_q, const int* q_pos0, const int* tiles, int n_tiles, const float* sinks,
                           void* out, int H, int KVH, int D, int window, float scale, float softcap,
                           int64_t num_pages, cudaStream_t st) {
  if (n_tiles <= 0) return 0;
  if (H % KVH) return -1;
  CUtensorMap tk, tv;
  const int64_t rows = num_pages * KVH * 16;
  if (!make_tmap_2d(&tk, k_cache, rows, D, D, 16, 64, 2)) return -1;
  if (!make_tmap_2d(&tv, v_cache, rows, D, D, 16, 64, 2)) return -1;
  mmapf::Args a{reinterpret_cast<const __nv_bfloat16*>(q), page_table, cu_q, q_pos0, tiles, sinks,
                reinterpret_cast<__nv_bfloat16*>(out), H, KVH, ld_pt, window, num_pages, scale, softcap};
  switch (D) {
    case 64: return mmapf::launch<64>(tk, tv, a, n_tiles, st);
    case 128: return mmapf::launch<128>(tk, tv, a, n_tiles, st);
    case 256: return mmapf::launch<256>(tk, tv, a, n_tiles, st);
    default: return -1;
  }
}

}  // extern "C"

B200_STATUS_ACCESSORS(attn_prefill_mma)
