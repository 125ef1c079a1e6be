// Paged prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract as attention_prefill_mma.cu / attention_prefill_simt.cu:
// causal attention of each row's prefill chunk against the row's paged KV
// history (which already holds the chunk's own K/V), sliding windows from
// absolute positions (window < 0: bidirectional over the row's keys), learned
// sinks in the denominator only, optional logit softcap. bf16 K/V pages,
// head dim 64 or 128. Replaces the per-row gather + SDPA of the reference
// (ContinuousBatchingV2/Paged/PagedLayerCache.swift:584-637).
//
// Work unit (CTA): 128 consecutive queries of one row x one query head.
// Warps 0-3: softmax; thread t owns query row t (TMEM lane t). Warp 4: TMA
// producer. Warp 5: tcgen05 MMA issuer and tensor-memory owner.
// Tensor memory (512 columns): S0, S1 (128 fp32 columns each, double
// buffered), P (64 columns = 128 bf16 per row), O (D fp32 columns).
// Per 128-key block j (8 pages):
//   MMA:     S[j%2] = Q K_j^T            (kind::f16, A = Q smem, B = K smem, K-major)
//   softmax: row max / exp2 from S, O *= exp2(m_old - m_new) when the max
//            moves, P_j (bf16) -> tensor memory
//   MMA:     O += P_j V_j                (A = P from tensor memory, B = V smem, MN-major)
// QK of block j+1 is issued before PV of block j, so the softmax of one
// block overlaps the next block's scores. K/V blocks stream through a
// 2-stage ring: one full barrier per stage (TMA transaction bytes), freed by
// the MMA's commit after PV. Pages outside the tile's key range load a page
// of the range instead (finite data, masked to zero weight).
// Every wait is bounded (2 s): on expiry the kernel records kErrAttnWait and
// finishes without hanging.
#include <cudaTypedefs.h>

#include "b200_common.cuh"

namespace b200 {

bool make_tmap_2d(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows,
                  int box_cols, int dtype_bytes);

namespace tcpf {

constexpr int kPage = 16;
constexpr int kQT = 128;   // queries per CTA (TMEM lanes)
constexpr int kKB = 128;   // keys per block
constexpr int kNst = 2;    // K/V ring stages
constexpr int kThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColP = 256, kColO = 320;

struct Args {
  const int* page_table;  // [R, ld_pt]
  const int* cu_q;        // [R+1]
  const int* q_pos0;      // [R]
  const int* tiles;       // [n_tiles, 2] (row, q offset)
  const float* sinks;     // [H] or null
  __nv_bfloat16* out;     // [T, H, D]
  int H, KVH, ld_pt, window;
  int64_t num_pages;
  float scale, softcap;
};

template <int D>
struct Smem {
  static constexpr int kSub = kKB * 128;             // one 64-column sub-tile of a 128-row block (16 KB)
  static constexpr int kQBytes = (D / 64) * kQT * 128;
  static constexpr int kKVBytes = (D / 64) * kSub;   // K or V block
  static constexpr int kStage = 2 * kKVBytes;
  static constexpr int kQOff = 0;
  static constexpr int kRingOff = kQBytes;
  static constexpr int kTotal = kQBytes + kNst * kStage + 1024;  // + alignment slack
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                                 const __grid_constant__ CUtensorMap tmK,
                                                                 const __grid_constant__ CUtensorMap tmV, Args a) {
  using S = Smem<D>;
  constexpr int NB = D / 64;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  __shared__ __align__(8) uint64_t bar_q, bar_full[kNst], bar_empty[kNst], bar_s[2], bar_p, bar_o;
  __shared__ uint32_t tmem_slot;

  pdl_launch_dependents();
  const int tile = blockIdx.x, head = blockIdx.y;
  const int kvh = head / (a.H / a.KVH);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    mbar_init(smem_u32(&bar_q), 1);
    for (int s = 0; s < kNst; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 1);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    mbar_init(smem_u32(&bar_s[0]), 1);
    mbar_init(smem_u32(&bar_s[1]), 1);
    mbar_init(smem_u32(&bar_p), 4);  // one arrive per softmax warp
    mbar_init(smem_u32(&bar_o), 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(&tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  pdl_wait();

  const int row = a.tiles[2 * tile], qoff = a.tiles[2 * tile + 1];
  const int q0 = a.cu_q[row], qlen = a.cu_q[row + 1] - q0;
  const int pos0 = a.q_pos0[row];
  const int nq = min(kQT, qlen - qoff);
  const bool bidir = a.window < 0;
  // key range of the tile (absolute positions, inclusive)
  const int k_hi = bidir ? pos0 + qlen - 1 : pos0 + qoff + max(nq, 1) - 1;
  const int k_lo = a.window > 0 ? max(0, pos0 + qoff - a.window + 1) : 0;
  const int pg_lo = k_lo / kPage, pg_hi = k_hi / kPage;
  const int kb_lo = k_lo / kKB, kb_hi = k_hi / kKB;
  const int nblk = nq > 0 ? kb_hi - kb_lo + 1 : 0;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && nblk > 0) {
      mbar_arrive_expect_tx(smem_u32(&bar_q), S::kQBytes);
#pragma unroll
      for (int h = 0; h < NB; ++h)
        tma_load_2d(sbase + S::kQOff + h * kQT * 128, &tmQ, smem_u32(&bar_q), head * D + h * 64, q0 + qoff, 0ull);
      const int* pt = a.page_table + (size_t)row * a.ld_pt;
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kNst;
        if (j >= kNst && !mbar_wait(smem_u32(&bar_empty[s]), ((j / kNst) - 1) & 1, kErrAttnWait)) break;
        const uint32_t kd = sbase + S::kRingOff + s * S::kStage, vd = kd + S::kKVBytes;
        const uint32_t fb = smem_u32(&bar_full[s]);
        mbar_arrive_expect_tx(fb, S::kStage);
        for (int p = 0; p < kKB / kPage; ++p) {
          const int lp = min(max((kb_lo + j) * (kKB / kPage) + p, pg_lo), pg_hi);
          const int64_t page = checked_page(pt, lp, a.ld_pt, a.num_pages);
          const int r = (int)((page * a.KVH + kvh) * kPage);
#pragma unroll
          for (int h = 0; h < NB; ++h) {
            tma_load_2d(kd + h * S::kSub + p * kPage * 128, &tmK, fb, h * 64, r, 0ull);
            tma_load_2d(vd + h * S::kSub + p * kPage * 128, &tmV, fb, h * 64, r, 0ull);
          }
        }
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kQT, kKB);            // S = Q K^T: K-major A and B
      constexpr uint32_t idesc_o = umma_idesc_bf16(kQT, D, 0, 1);        // O += P V: V is MN-major
      bool ok = mbar_wait(smem_u32(&bar_q), 0, kErrAttnWait);
      auto issue_qk = [&](int j) {
        const int s = j % kNst;
        const uint32_t kd = sbase + S::kRingOff + s * S::kStage;
        const uint32_t dst = tmem + ((j & 1) ? kColS1 : kColS0);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t ad = umma_desc_k_sw128(sbase + S::kQOff + (k >> 2) * kQT * 128, 1024) + 2 * (k & 3);
          const uint64_t bd = umma_desc_k_sw128(kd + (k >> 2) * S::kSub, 1024) + 2 * (k & 3);
          tc_mma_f16(dst, ad, bd, idesc_s, k > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&bar_s[j & 1]));
      };
      if (ok) ok = mbar_wait(smem_u32(&bar_full[0]), 0, kErrAttnWait);
      if (ok) {
        tc_fence_after();
        issue_qk(0);
      }
      for (int j = 0; ok && j < nblk; ++j) {
        if (j + 1 < nblk) {
          const int s1 = (j + 1) % kNst;
          if (!mbar_wait(smem_u32(&bar_full[s1]), ((j + 1) / kNst) & 1, kErrAttnWait)) break;
          tc_fence_after();
          issue_qk(j + 1);
        }
        if (!mbar_wait(smem_u32(&bar_p), j & 1, kErrAttnWait)) break;
        tc_fence_after();
        const int s = j % kNst;
        const uint32_t vd = sbase + S::kRingOff + s * S::kStage + S::kKVBytes;
#pragma unroll
        for (int k = 0; k < kKB / 16; ++k) {
          // 16 keys = two 8-row swizzle atoms; the D halves are 16 KB apart
          const uint64_t bd = umma_desc_mn_sw128(vd + k * 2048, S::kSub, 1024);
          tc_mma_f16_ts(tmem + kColO, tmem + kColP + 8 * k, bd, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&bar_empty[s]));
        tc_commit(smem_u32(&bar_o));
      }
    }
  } else {
    // ---------------- softmax (thread t = query row t) ----------------
    const int t = threadIdx.x;
    const bool vrow = t < nq;
    const int qp = pos0 + qoff + t;                      // absolute query position
    const int kmax = bidir ? pos0 + qlen - 1 : qp;       // last visible key
    const int kmin = a.window > 0 ? qp - a.window + 1 : 0;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const float smul = a.softcap > 0.f ? a.scale : a.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk && ok; ++j) {
      if (!mbar_wait(smem_u32(&bar_s[j & 1]), (j >> 1) & 1, kErrAttnWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t scol = (j & 1) ? kColS1 : kColS0;
      const int kbase = (kb_lo + j) * kKB;
      // scaled, masked score of column c of this block (S is read twice from
      // tensor memory: once for the row max, once for the weights)
      auto score = [&](float x, int c) -> float {
        const int kp = kbase + c;
        float v = x * smul;
        if (a.softcap > 0.f) v = a.softcap * tanhf(v / a.softcap) * kLog2e;
        const bool valid = vrow && kp <= kmax && kp >= kmin && kp >= k_lo;
        return valid ? v : -INFINITY;
      };
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kKB; c += 32) {
        uint32_t r[32];
        tmem_ld32(lane_base + scol + c, r);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) mx = fmaxf(mx, score(__uint_as_float(r[e]), c + e));
      }
      const float m_new = fmaxf(m, mx);
      // PV of the previous block must be done before O is rescaled and P rewritten
      if (j > 0 && !mbar_wait(smem_u32(&bar_o), (j - 1) & 1, kErrAttnWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j > 0 && m_new > m && m != -INFINITY) {
        const float alpha = exp2f(m - m_new);
        l *= alpha;
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t r[32];
          tmem_ld32(lane_base + kColO + c, r);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
          tmem_st32(lane_base + kColO + c, r);
        }
      }
      m = m_new;
      float ps = 0.f;
#pragma unroll 1
      for (int c = 0; c < kKB; c += 32) {
        uint32_t r[32], pk[16];
        tmem_ld32(lane_base + scol + c, r);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float s0 = score(__uint_as_float(r[2 * e]), c + 2 * e);
          const float s1 = score(__uint_as_float(r[2 * e + 1]), c + 2 * e + 1);
          const float p0 = m == -INFINITY ? 0.f : exp2f(s0 - m);
          const float p1 = m == -INFINITY ? 0.f : exp2f(s1 - m);
          // the denominator sums the bf16-rounded weights that the PV product uses
          pk[e] = pack_bf16x2(p0, p1);
          const __nv_bfloat162 pb = *reinterpret_cast<const __nv_bfloat162*>(&pk[e]);
          ps += __bfloat162float(pb.x) + __bfloat162float(pb.y);
        }
        tmem_st16(lane_base + kColP + (c >> 1), pk);
      }
      l += ps;
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar_p));
    }
    // ---------------- epilogue: O / l -> out ----------------
    if (ok && nblk > 0 && !mbar_wait(smem_u32(&bar_o), (nblk - 1) & 1, kErrAttnWait)) ok = false;
    tc_fence_after();
    if (nblk > 0) {
      float den = l;
      if (a.sinks && m != -INFINITY) den += exp2f(a.sinks[head] * kLog2e - m);
      else if (a.sinks) den += 1.f;
      const float inv = (ok && den > 0.f) ? 1.f / den : 0.f;
      __nv_bfloat16* dst = a.out + ((size_t)(q0 + qoff + t) * a.H + head) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        tmem_ld32(lane_base + kColO + c, r);
        tc_wait_ld();
        if (vrow) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[e]) * inv, __uint_as_float(r[e + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(r[e + 2]) * inv, __uint_as_float(r[e + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(r[e + 4]) * inv, __uint_as_float(r[e + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(r[e + 6]) * inv, __uint_as_float(r[e + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c + e) = w;
          }
        }
      }
    }
  }
  // every TMA copy has landed before the CTA may exit (stage memory is released)
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const Args& a, int n_tiles,
           cudaStream_t st) {
  constexpr int smem = Smem<D>::kTotal;
  static_assert(smem <= 227 * 1024, "shared memory plan exceeds the per-CTA limit");
  if (int e = smem_attr_once<prefill_tc_kernel<D>>(smem)) return e;
  cudaError_t e = launch_k(prefill_tc_kernel<D>, dim3(n_tiles, a.H), dim3(kThreads), smem, st, 1, tq, tk, tv, a);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace tcpf
}  // namespace b200

using namespace b200;

extern "C" {

int b200_prefill_tc_q_tile() { return tcpf::kQT; }

// tiles: [n_tiles, 2] (row, query offset within the row's chunk), offsets
// multiples of b200_prefill_tc_q_tile(). bf16 q [T, H, D] and K/V pages, D 64 / 128.
int b200_paged_prefill_tc(const void* q, int T, const void* k_cache, const void* v_cache, const int* page_table,
                          int ld_pt, const int* cu_q, const int* q_pos0, const int* tiles, int n_tiles,
                          const float* sinks, void* out, int H, int KVH, int D, int window, float scale,
                          float softcap, int64_t num_pages, cudaStream_t st) {
  if (n_tiles <= 0) return 0;
  if (H % KVH || (D != 64 && D != 128)) return -1;
  CUtensorMap tq, tk, tv;
  const int64_t rows = num_pages * KVH * 16;
  if (!make_tmap_2d(&tq, q, T, (int64_t)H * D, (int64_t)H * D, tcpf::kQT, 64, 2)) return -1;
  if (!make_tmap_2d(&tk, k_cache, rows, D, D, 16, 64, 2)) return -1;
  if (!make_tmap_2d(&tv, v_cache, rows, D, D, 16, 64, 2)) return -1;
  tcpf::Args a{page_table, cu_q, q_pos0, tiles, sinks, reinterpret_cast<__nv_bfloat16*>(out), H, KVH, ld_pt,
               window, num_pages, scale, softcap};
  return D == 64 ? tcpf::launch<64>(tq, tk, tv, a, n_tiles, st) : tcpf::launch<128>(tq, tk, tv, a, n_tiles, st);
}

}  // extern "C"

B200_STATUS_ACCESSORS(attn_prefill_tc)
