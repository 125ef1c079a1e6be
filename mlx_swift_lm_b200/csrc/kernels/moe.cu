// Mixture-of-experts kernels: router top-k, expert sort, grouped tcgen05 GEMM,
// weighted combine.
//
// Reference behaviour: router top-k with normalisation in one threadgroup,
// bit-identical to sort+gather (MLXLMCommon/MoERouterTopK.swift:22-160);
// SwitchGLU gather -> expert matmuls -> weighted un-sort
// (SwitchLayers.swift:478, gatherSort :244, scatterUnsort :257,
// weightedExpertUnsort :149).
//
// B200 design:
//   moe_route_topk   one warp per token: softmax over experts then top-k (and
//                    optional renormalisation), or top-k logits then softmax;
//                    ties resolve to the lower expert id.
//   moe_sort         single-CTA counting sort of the T*k (token, expert) pairs
//                    by expert (stable in pair index -> deterministic), plus a
//                    work list of (expert, first row, rows) chunks of <= BN rows.
//   moe_gather       sorted activation rows.
//   grouped GEMM     tcgen05 swap-AB tiles: CTA (n tile, chunk) multiplies the
//                    chunk's rows by its expert's weight tile (TMA row offset
//                    expert * N); GLU epilogue for gate/up; grid sized for the
//                    worst case so it can live in a CUDA graph (idle CTAs exit).
//   moe_combine      out[t] = sum_j w[t, j] * y[pos(t, j)] in slot order j.
#include <cudaTypedefs.h>

#include <cuda_fp16.h>

#include "b200_common.cuh"
#include "b200_dequant.cuh"
#include "b200_moe.cuh"

namespace b200 {

bool make_tmap_2d(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows,
                  int box_cols, int dtype_bytes);
bool make_tmap_2d_sw(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows,
                     int box_cols, int dtype_bytes, bool swizzle128);

namespace moe {

// ---------------------------------------------------------------- router
__global__ void route_topk_kernel(const float* __restrict__ logits, int T, int E, int k, int mode, int norm_topk,
                                  int* __restrict__ ids, float* __restrict__ w, RouteExtra ex) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (warp >= T) return;
  route_topk_warp(logits + (size_t)warp * E, E, k, mode, norm_topk, ids + (size_t)warp * k, w + (size_t)warp * k, ex);
}

// ---------------------------------------------------------------- sort
// Outputs: perm [P] (pair index in expert order), pos [P] (sorted position of
// each pair), chunks [max_chunks][3] (expert, first sorted row, rows), and
// n_chunks. One CTA of 32 warps; warp w owns the contiguous pair range
// [w*seg, (w+1)*seg), so ranks come from per-warp per-expert counters
// (wcnt[32][E] in shared memory) plus __match_any_sync inside each 32-pair
// slab: the placement is stable in pair index, hence deterministic.
__global__ void __launch_bounds__(1024) sort_kernel(const int* __restrict__ ids, int P, int E, int BN,
                                                    int max_chunks, int* __restrict__ perm, int* __restrict__ pos,
                                                    int* __restrict__ chunks, int* __restrict__ n_chunks) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ int sm[];
  int* wcnt = sm;             // [32][E] counts, then exclusive bases
  int* off = sm + 32 * E;     // [E + 1] expert start offsets, then the valid total
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  const int seg = (P + 31) / 32;
  const int p0 = warp * seg, p1 = min(P, p0 + seg);
  for (int b = p0; b < p1; b += 32) {
    const int p = b + lane;
    const int e = p < p1 ? ids[p] : -1;
    const bool ok = e >= 0 && e < E;
    const unsigned grp = __match_any_sync(0xffffffffu, ok ? e : -1);
    if (ok && (grp & lt) == 0) wcnt[warp * E + e] += __popc(grp);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int acc = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = acc;
      acc += c;
    }
    off[e] = acc;  // total for now
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0, nc = 0;
    for (int e = 0; e < E; ++e) {
      const int c = off[e];
      off[e] = acc;
      for (int r = 0; r < c; r += BN) {
        if (nc < max_chunks) {
          chunks[3 * nc + 0] = e;
          chunks[3 * nc + 1] = acc + r;
          chunks[3 * nc + 2] = min(BN, c - r);
        }
        ++nc;
      }
      acc += c;
    }
    *n_chunks = min(nc, max_chunks);
    if (nc > max_chunks) set_status(kErrBounds);
    off[E] = acc;  // valid pairs
  }
  __syncthreads();
  // pairs with an id outside [0, E) (empty expert-parallel receive slots) get
  // pos -1 and leave the tail of perm at -1
  for (int s = off[E] + threadIdx.x; s < P; s += blockDim.x) perm[s] = -1;
  for (int b = p0; b < p1; b += 32) {
    const int p = b + lane;
    const int e = p < p1 ? ids[p] : -1;
    const bool ok = e >= 0 && e < E;
    const unsigned grp = __match_any_sync(0xffffffffu, ok ? e : -1);
    if (ok) {
      const int s = off[e] + wcnt[warp * E + e] + __popc(grp & lt);
      perm[s] = p;
      pos[p] = s;
    } else if (p < p1) {
      pos[p] = -1;
    }
    __syncwarp();
    if (ok && (grp & lt) == 0) wcnt[warp * E + e] += __popc(grp);
    __syncwarp();
  }
}

__global__ void gather_kernel(const __nv_bfloat16* __restrict__ x, int K, const int* __restrict__ perm, int P,
                              int k, __nv_bfloat16* __restrict__ xs, int to_f16) {
  pdl_launch_dependents();
  pdl_wait();
  const int s = blockIdx.x;
  if (s >= P || perm[s] < 0) return;
  const int t = perm[s] / k;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * K);
  uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)s * K);
  for (int i = threadIdx.x; i < K / 8; i += blockDim.x) {
    uint4 v = src[i];
    if (to_f16) {  // activations of the f16 MXFP4 path (saturating at the f16 range)
      uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
        const __half2 h = __floats2half2_rn(fminf(fmaxf(f.x, -65504.f), 65504.f), fminf(fmaxf(f.y, -65504.f), 65504.f));
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    dst[i] = v;
  }
}

__global__ void combine_kernel(const __nv_bfloat16* __restrict__ ys, int N, const int* __restrict__ pos,
                               const float* __restrict__ w, int k, __nv_bfloat16* __restrict__ out,
                               const __nv_bfloat16* __restrict__ bias_d, const int* __restrict__ ids) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      const int s = pos[t * k + j];
      float y = bf2f(ys[(size_t)s * N + i]);
      if (bias_d) y = bf2f(f2bf(y + bf2f(bias_d[(size_t)ids[t * k + j] * N + i])));
      acc += w[t * k + j] * y;
    }
    out[(size_t)t * N + i] = f2bf(acc);
  }
}

// ---------------------------------------------------------------- grouped GEMM
struct GArgs {
  __nv_bfloat16* Y;  // [P, ldy] sorted rows (f16 when y_f16)
  const __nv_bfloat16* bias;  // [E, N] or null
  const int* chunks;
  const int* n_chunks;
  int N, K, ldy, epi;
  int y_f16;  // f16 output rows (the f16 MXFP4 path's gate/up output feeds the f16 down GEMM)
};

__device__ __forceinline__ void store_y(const GArgs& a, size_t idx, float v) {
  if (a.y_f16) reinterpret_cast<__half*>(a.Y)[idx] = __float2half_rn(v);
  else a.Y[idx] = f2bf(v);
}

__device__ __forceinline__ float glu(int epi, float g, float u) { return glu_act(epi, g, u); }

// Quantised expert weights (WQ = 4 or 8): codes [E*N, K*WQ/8] bytes,
// scales / biases [K/gs, E*N] bf16 (layout of b200_dequant.cuh).
struct GQuant {
  const uint8_t* tiled;  // records [E][tiles_per_expert][K/64][rec_bytes] (tile-major, per expert)
  int gs, gpb, rec_bytes, kb_total, tiles_per_expert;
};

// Operand stages {A bf16 weight tile, B activation tile}; with quantised
// experts also a raw ring of small {codes, scales, biases} stages sized so two
// CTAs fit on an SM (one CTA's start-up latency overlaps the other's stream).
template <int BN, int STAGES, int WQ>
struct GSmem {
  static constexpr int kA = 128 * 128, kB = BN * 128;
  static constexpr int kCode = code_bits<WQ>() * 128 * 64 / 8, kGroup = 2 * 128 * 2;
  static constexpr int kRaw = WQ ? kCode + 2 * kGroup : 0;
  // bf16 experts: stages of {A weight tile, B activation tile}. Quantised
  // experts: A stages (dequantised weight tiles) and a deeper ring of B
  // activation tiles of their own, so an A stage's reuse waits for the
  // dequantisation and the MMA only, not for a fresh activation load.
  static constexpr int kStage = WQ ? kA : (kA + kB + 1023) / 1024 * 1024;
  static constexpr int kBStages = WQ ? (BN <= 16 ? 8 : BN <= 32 ? 4 : STAGES) : 0;
  static constexpr int kBOff = STAGES * kStage;
  static constexpr int kRawOff = kBOff + kBStages * kB;
  static constexpr int kRawStages = WQ ? (100 * 1024 - kRawOff) / kRaw : 0;
  static constexpr int kBars = (WQ ? 3 : 2) * STAGES + 2 * kRawStages + 2 * kBStages + 1;
  static constexpr int kTotal = kRawOff + kRawStages * kRaw + kBars * 8 + 16 + 1024;
  static constexpr int kThreads = WQ ? 384 : 128;
  static constexpr int kMinBlocks = WQ ? 2 : 1;
  static constexpr int kTmem = BN < 32 ? 32 : BN;
  static_assert(!WQ || kRawStages >= 4, "raw ring too shallow");
};

// F16: MXFP4 experts (natural-order records) dequantised to f16 and
// multiplied with f16 activations (kind::f16, both operands f16).
template <int BN, int STAGES, int WQ, bool F16 = false>
__global__ void __launch_bounds__(GSmem<BN, STAGES, WQ>::kThreads, GSmem<BN, STAGES, WQ>::kMinBlocks)
    grouped_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, GArgs a,
                   const __grid_constant__ GQuant q) {
  static_assert(!F16 || WQ == kWqE2M1, "the f16 path serves MXFP4 records");
  using S = GSmem<BN, STAGES, WQ>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  constexpr int RS = S::kRawStages;
  const uint32_t bar_full = sbase + S::kRawOff + RS * S::kRaw;
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  const uint32_t bar_acc = bar_empty + 8 * STAGES;
  const uint32_t bar_aready = bar_acc + 8;
  const uint32_t bar_rfull = bar_aready + 8 * STAGES;
  const uint32_t bar_rempty = bar_rfull + 8 * RS;
  constexpr int BS = S::kBStages;
  const uint32_t bar_bfull = bar_rempty + 8 * RS;  // quantised: B ring
  const uint32_t bar_bempty = bar_bfull + 8 * BS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kRawOff + RS * S::kRaw + S::kBars * 8);
  __shared__ float xbuf[64][17];
  pdl_launch_dependents();
  pdl_wait();
  const int chunk = blockIdx.y;
  if (chunk >= *a.n_chunks) return;
  const int e = a.chunks[3 * chunk], r0 = a.chunks[3 * chunk + 1], rc = a.chunks[3 * chunk + 2];
  const int n0 = blockIdx.x * 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (a.K + 63) / 64;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
      if constexpr (WQ != 0) mbar_init(bar_aready + 8 * s, 8);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(bar_rfull + 8 * s, 1);
      mbar_init(bar_rempty + 8 * s, 8);
    }
    for (int b = 0; b < BS; ++b) {
      mbar_init(bar_bfull + 8 * b, 1);
      mbar_init(bar_bempty + 8 * b, 1);
    }
    mbar_init(bar_acc, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), S::kTmem);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int wrow = e * a.N + n0;
  const uint64_t pw = l2_policy_evict_first(), px = l2_policy_evict_last();
  if (warp == 0 && lane == 0) {
    if constexpr (WQ == 0) {
      // operand producer: weight tile + activation tile per stage
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES, r = i / STAGES;
        if (r > 0 && !mbar_wait(bar_empty + 8 * s, (r - 1) & 1, kErrGemmWait)) break;
        const uint32_t st = sbase + s * S::kStage;
        mbar_arrive_expect_tx(bar_full + 8 * s, (uint32_t)(S::kA + S::kB));
        tma_load_2d(st, &tmW, bar_full + 8 * s, i * 64, wrow, pw);
        tma_load_2d(st + S::kA, &tmX, bar_full + 8 * s, i * 64, r0, px);
        issued = i + 1;
      }
      for (int i = max(0, issued - STAGES); i < issued; ++i)
        mbar_wait(bar_full + 8 * (i % STAGES), (i / STAGES) & 1, kErrGemmWait);
    } else {
      // activation tiles into the B ring, BS blocks ahead of the MMA
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int b = i % BS, rb = i / BS;
        if (rb > 0 && !mbar_wait(bar_bempty + 8 * b, (rb - 1) & 1, kErrGemmWait)) break;
        mbar_arrive_expect_tx(bar_bfull + 8 * b, (uint32_t)S::kB);
        tma_load_2d(sbase + S::kBOff + b * S::kB, &tmX, bar_bfull + 8 * b, i * 64, r0, px);
        issued = i + 1;
      }
      for (int i = max(0, issued - BS); i < issued; ++i)
        mbar_wait(bar_bfull + 8 * (i % BS), (i / BS) & 1, kErrGemmWait);
    }
  } else if (warp == 2 && lane == 0) {
    if constexpr (WQ != 0) {
      // raw producer: codes + scales + biases, RS stages ahead
      const uint8_t* tile = q.tiled + ((size_t)e * q.tiles_per_expert + blockIdx.x) * q.kb_total * q.rec_bytes;
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % RS, r = i / RS;
        if (r > 0 && !mbar_wait(bar_rempty + 8 * s, (r - 1) & 1, kErrGemmWait)) break;
        const uint32_t raw = sbase + S::kRawOff + s * S::kRaw;
        mbar_arrive_expect_tx(bar_rfull + 8 * s, (uint32_t)q.rec_bytes);
        bulk_g2s(raw, tile + (size_t)i * q.rec_bytes, (uint32_t)q.rec_bytes, bar_rfull + 8 * s, pw);
        issued = i + 1;
      }
      for (int i = max(0, issued - RS); i < issued; ++i)
        mbar_wait(bar_rfull + 8 * (i % RS), (i / RS) & 1, kErrGemmWait);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = F16 ? umma_idesc_f16(128, BN) : umma_idesc_bf16(128, BN);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES, r = i / STAGES;
      uint32_t baddr;
      if constexpr (WQ == 0) {
        if (!mbar_wait(bar_full + 8 * s, r & 1, kErrGemmWait)) break;
        baddr = sbase + s * S::kStage + S::kA;
      } else {
        const int b = i % BS;
        if (!mbar_wait(bar_bfull + 8 * b, (i / BS) & 1, kErrGemmWait)) break;
        if (!mbar_wait(bar_aready + 8 * s, r & 1, kErrGemmWait)) break;
        baddr = sbase + S::kBOff + b * S::kB;
      }
      tc_fence_after();
      const uint64_t ad = umma_desc_k_sw128(sbase + s * S::kStage, 1024);
      const uint64_t bd = umma_desc_k_sw128(baddr, 1024);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) tc_mma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      tc_commit(bar_empty + 8 * s);  // A stage (and, bf16, its activation tile) free
      if constexpr (WQ != 0) tc_commit(bar_bempty + 8 * (i % BS));
    }
    tc_commit(bar_acc);
  } else if (warp >= 4) {
    if constexpr (WQ != 0) {
      const int t = (threadIdx.x - 128) & 127, half = (threadIdx.x - 128) >> 7;
      const int g = q.gs == 16 ? 2 * half : q.gs == 32 ? half : 0;
      for (int i = 0; i < nkb; ++i) {
        const int rs = i % RS, rr = i / RS;
        const int s = i % STAGES, r = i / STAGES;
        if (!mbar_wait(bar_rfull + 8 * rs, rr & 1, kErrGemmWait)) break;
        if (r > 0 && !mbar_wait(bar_empty + 8 * s, (r - 1) & 1, kErrGemmWait)) break;
        if constexpr (F16) {
          dequant_half_row_e2m1_f16(smem + S::kRawOff + rs * S::kRaw, smem + s * S::kStage, t, half, g, q.gpb);
        } else {
          dequant_half_row<WQ>(smem + S::kRawOff + rs * S::kRaw, smem + s * S::kStage, t, half, g, q.gpb);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_rempty + 8 * rs);
          mbar_arrive(bar_aready + 8 * s);
        }
      }
    }
  }
  __syncwarp();
  const bool ok = __syncthreads_and(mbar_wait(bar_acc, 0, kErrTmemWait) ? 1 : 0) != 0;
  tc_fence_after();
  const bool ep = warp < 4;  // TMEM lanes 32*warp.. belong to warps 0..3
  const int rl = warp * 32 + lane;
  const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  const bool isglu = a.epi == 1 || a.epi == 4 || a.epi == 5;
  const float bb = (ep && a.bias && n0 + rl < a.N) ? bf2f(a.bias[(size_t)e * a.N + n0 + rl]) : 0.f;
  for (int jc = 0; jc < BN; jc += 16) {
    float f[16];
    if (ep) {
      uint32_t v[16];
      tmem_ld16(tl + jc, v);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) f[j] = ok ? __uint_as_float(v[j]) + bb : 0.f;
    }
    if (isglu) {
      __syncthreads();
      if (ep && warp >= 2) {
#pragma unroll
        for (int j = 0; j < 16; ++j) xbuf[rl - 64][j] = f[j];
      }
      __syncthreads();
      if (warp < 2) {
        const int fo = (n0 >> 1) + rl;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int row = jc + j;
          if (row < rc && fo < (a.N >> 1)) {
            const float gg = bf2f(f2bf(f[j])), u = bf2f(f2bf(xbuf[rl][j]));
            store_y(a, (size_t)(r0 + row) * a.ldy + fo, glu(a.epi, gg, u));
          }
        }
      }
    } else if (ep && n0 + rl < a.N) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int row = jc + j;
        if (row < rc) store_y(a, (size_t)(r0 + row) * a.ldy + n0 + rl, f[j]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmem);
  }
}

// ---------------------------------------------------------------- persistent grouped GEMM
// Decode-sized expert chunks (<= 32 rows) with quantised experts: one CTA per
// SM loops over the (chunk, 128-row weight tile) work items w = blockIdx.x,
// blockIdx.x + gridDim.x, ... (the same fixed item -> CTA map whatever the
// batch, each item's K order fixed). Set-up (barriers, tensor memory) is paid
// once per SM instead of once per item, and the pipelines run across item
// boundaries: the raw producer streams the next item's records while the
// current one finishes, and the accumulator is double-buffered in tensor
// memory so the epilogue of item j overlaps the MMAs of item j + 1.
// Warps: 0 activation TMA | 1 MMA | 2 raw records | 3 idle | 4-11 dequantise
// (thread = row t, half of the 64-input block) | 12-15 epilogue (tensor
// memory lanes 32 * (warp % 4)).
template <int BN, int WQ>
struct PSmem {
  static constexpr int kA = 128 * 128, kB = BN * 128;
  static constexpr int kStage = (kA + kB + 1023) / 1024 * 1024;
  static constexpr int kStages = 6;
  static constexpr int kCode = code_bits<WQ>() * 128 * 64 / 8, kGroup = 2 * 128 * 2;
  static constexpr int kRaw = kCode + 2 * kGroup;
  static constexpr int kRawOff = kStages * kStage;
  static constexpr int kRawStages = (196 * 1024 - kRawOff) / kRaw;
  static constexpr int kBars = 3 * kStages + 2 * kRawStages + 4;
  static constexpr int kXOff = kRawOff + kRawStages * kRaw;
  static constexpr int kXBytes = 64 * BN * 4;
  static constexpr int kTotal = kXOff + kXBytes + kBars * 8 + 16 + 1024;
  static constexpr int kThreads = 512;
  static constexpr int kAccCols = BN < 32 ? 32 : BN;
  static constexpr int kTmem = 2 * kAccCols;
  static_assert(kRawStages >= 8, "raw ring too shallow");
  static_assert(kTotal <= 227 * 1024, "shared memory plan exceeds the per-CTA limit");
};

__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int BN, int WQ, bool F16 = false>
__global__ void __launch_bounds__(512, 1)
    grouped_persistent_kernel(const __grid_constant__ CUtensorMap tmX, GArgs a, const __grid_constant__ GQuant q) {
  static_assert(!F16 || WQ == kWqE2M1, "the f16 path serves MXFP4 records");
  using S = PSmem<BN, WQ>;
  constexpr int ST = S::kStages, RS = S::kRawStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  float* xbuf = reinterpret_cast<float*>(smem + S::kXOff);  // [64][BN]: up rows handed to the gate warps
  const uint32_t bar_full = sbase + S::kXOff + S::kXBytes;
  const uint32_t bar_empty = bar_full + 8 * ST;
  const uint32_t bar_aready = bar_empty + 8 * ST;
  const uint32_t bar_rfull = bar_aready + 8 * ST;
  const uint32_t bar_rempty = bar_rfull + 8 * RS;
  const uint32_t bar_accf = bar_rempty + 8 * RS;  // [2]
  const uint32_t bar_acce = bar_accf + 16;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kXOff + S::kXBytes + S::kBars * 8);
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = a.K / 64;
  const int ntiles = (a.N + 127) / 128;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
      mbar_init(bar_aready + 8 * s, 8);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(bar_rfull + 8 * s, 1);
      mbar_init(bar_rempty + 8 * s, 8);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accf + 8 * b, 1);
      mbar_init(bar_acce + 8 * b, 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), S::kTmem);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  const int n_items = *a.n_chunks * ntiles;
  const uint64_t pw = l2_policy_evict_first(), px = l2_policy_evict_last();
  auto item = [&](int w, int& e, int& r0, int& rc, int& tile) {
    const int c = w / ntiles;
    tile = w - c * ntiles;
    e = a.chunks[3 * c];
    r0 = a.chunks[3 * c + 1];
    rc = a.chunks[3 * c + 2];
  };
  if (warp == 0) {
    if (lane == 0) {  // activation tiles: x rows r0.. of the item's chunk
      int g = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
        int e, r0, rc, tile;
        item(w, e, r0, rc, tile);
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % ST;
          if (g >= ST && !mbar_wait(bar_empty + 8 * s, ((g / ST) - 1) & 1, kErrGemmWait)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_full + 8 * s, (uint32_t)S::kB);
          tma_load_2d(sbase + s * S::kStage + S::kA, &tmX, bar_full + 8 * s, kb * 64, r0, px);
        }
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {  // raw weight records of the item's expert tile
      int g = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
        int e, r0, rc, tile;
        item(w, e, r0, rc, tile);
        const uint8_t* rec = q.tiled + ((size_t)e * q.tiles_per_expert + tile) * q.kb_total * q.rec_bytes;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % RS;
          if (g >= RS && !mbar_wait(bar_rempty + 8 * s, ((g / RS) - 1) & 1, kErrGemmWait)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_rfull + 8 * s, (uint32_t)q.rec_bytes);
          bulk_g2s(sbase + S::kRawOff + s * S::kRaw, rec + (size_t)kb * q.rec_bytes, (uint32_t)q.rec_bytes,
                   bar_rfull + 8 * s, pw);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer: item j accumulates into buffer j & 1
      constexpr uint32_t idesc = F16 ? umma_idesc_f16(128, BN) : umma_idesc_bf16(128, BN);
      int g = 0, j = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(bar_acce + 8 * b, ((j >> 1) - 1) & 1, kErrTmemWait)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * S::kAccCols);
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % ST;
          if (!mbar_wait(bar_full + 8 * s, (g / ST) & 1, kErrGemmWait) ||
              !mbar_wait(bar_aready + 8 * s, (g / ST) & 1, kErrGemmWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = umma_desc_k_sw128(sbase + s * S::kStage, 1024);
          const uint64_t bd = umma_desc_k_sw128(sbase + s * S::kStage + S::kA, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) tc_mma_f16(acc, ad + 2 * kk, bd + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit(bar_empty + 8 * s);
        }
        if (ok) tc_commit(bar_accf + 8 * b);
      }
    }
  } else if (warp >= 4 && warp < 12) {  // dequantise raw records into the A tiles
    const int t = (threadIdx.x - 128) & 127, half = (threadIdx.x - 128) >> 7;
    const int gsel = q.gs == 16 ? 2 * half : q.gs == 32 ? half : 0;
    int g = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb, ++g) {
        const int rs = g % RS, s = g % ST;
        if (!mbar_wait(bar_rfull + 8 * rs, (g / RS) & 1, kErrGemmWait) ||
            (g >= ST && !mbar_wait(bar_empty + 8 * s, ((g / ST) - 1) & 1, kErrGemmWait))) {
          ok = false;
          break;
        }
        if constexpr (F16) {
          dequant_half_row_e2m1_f16(smem + S::kRawOff + rs * S::kRaw, smem + s * S::kStage, t, half, gsel, q.gpb);
        } else {
          dequant_half_row<WQ>(smem + S::kRawOff + rs * S::kRaw, smem + s * S::kStage, t, half, gsel, q.gpb);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_rempty + 8 * rs);
          mbar_arrive(bar_aready + 8 * s);
        }
      }
    }
  } else if (warp >= 12) {  // epilogue: tensor memory -> rows of Y
    const int ew = warp & 3, rl = ew * 32 + lane;
    const bool isglu = a.epi == 1 || a.epi == 4 || a.epi == 5;
    int j = 0;
    for (int w = blockIdx.x; w < n_items; w += gridDim.x, ++j) {
      int e, r0, rc, tile;
      item(w, e, r0, rc, tile);
      const int n0 = tile * 128;
      const int b = j & 1;
      const bool ok = mbar_wait(bar_accf + 8 * b, (j >> 1) & 1, kErrTmemWait);
      tc_fence_after();
      const float bb = (a.bias && n0 + rl < a.N) ? bf2f(a.bias[(size_t)e * a.N + n0 + rl]) : 0.f;
      const uint32_t tl = tmem + (uint32_t)(b * S::kAccCols) + ((uint32_t)(ew * 32) << 16);
      for (int jc = 0; jc < BN; jc += 16) {
        float f[16];
        uint32_t v[16];
        tmem_ld16(tl + jc, v);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < 16; ++c) f[c] = ok ? __uint_as_float(v[c]) + bb : 0.f;
        if (isglu) {
          if (ew >= 2) {
#pragma unroll
            for (int c = 0; c < 16; ++c) xbuf[(rl - 64) * BN + jc + c] = f[c];
          }
          epi_bar_sync();
          if (ew < 2) {
            const int fo = (n0 >> 1) + rl;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              const int row = jc + c;
              if (row < rc && fo < (a.N >> 1)) {
                const float gg = bf2f(f2bf(f[c])), u = bf2f(f2bf(xbuf[rl * BN + jc + c]));
                store_y(a, (size_t)(r0 + row) * a.ldy + fo, glu(a.epi, gg, u));
              }
            }
          }
          epi_bar_sync();
        } else if (n0 + rl < a.N) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int row = jc + c;
            if (row < rc) store_y(a, (size_t)(r0 + row) * a.ldy + n0 + rl, f[c]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_acce + 8 * b);
      if (!ok) break;
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmem);
  }
}

template <int BN, int WQ, bool F16 = false>
int launch_persistent(const CUtensorMap& tx, const GArgs& a, const GQuant& q, int num_sms, cudaStream_t st) {
  using S = PSmem<BN, WQ>;
  if (int e = smem_attr_once<grouped_persistent_kernel<BN, WQ, F16>>(S::kTotal)) return e;
  cudaError_t e = launch_k(grouped_persistent_kernel<BN, WQ, F16>, dim3(num_sms), dim3(S::kThreads), S::kTotal, st,
                           1, tx, a, q);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

template <int WQ, bool F16 = false>
int dispatch_persistent(int BN, const CUtensorMap& tx, const GArgs& a, const GQuant& q, int num_sms,
                        cudaStream_t st) {
  switch (BN) {
    case 16: return launch_persistent<16, WQ, F16>(tx, a, q, num_sms, st);
    case 32: return launch_persistent<32, WQ, F16>(tx, a, q, num_sms, st);
    default: return -1;
  }
}

__global__ void e2m1_pairs_kernel(uint32_t* out) { out[threadIdx.x] = e2m1x2_to_f16x2(threadIdx.x); }

template <int BN, int STAGES, int WQ, bool F16>
int launch_grouped_f(const CUtensorMap& tw, const CUtensorMap& tx, const GArgs& a, const GQuant& q, int max_chunks,
                     cudaStream_t st) {
  using S = GSmem<BN, STAGES, WQ>;
  if (int e = smem_attr_once<grouped_kernel<BN, STAGES, WQ, F16>>(S::kTotal)) return e;
  cudaError_t e = launch_k(grouped_kernel<BN, STAGES, WQ, F16>, dim3((a.N + 127) / 128, max_chunks),
                           dim3(S::kThreads), S::kTotal, st, 1, tw, tx, a, q);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

inline int dispatch_grouped_f16(int BN, const CUtensorMap& tx, const GArgs& a, const GQuant& q, int max_chunks,
                                cudaStream_t st) {
  switch (BN) {
    case 16: return launch_grouped_f<16, 3, kWqE2M1, true>(tx, tx, a, q, max_chunks, st);
    case 32: return launch_grouped_f<32, 3, kWqE2M1, true>(tx, tx, a, q, max_chunks, st);
    case 64: return launch_grouped_f<64, 2, kWqE2M1, true>(tx, tx, a, q, max_chunks, st);
    case 128: return launch_grouped_f<128, 2, kWqE2M1, true>(tx, tx, a, q, max_chunks, st);
    default: return -1;
  }
}

template <int BN, int STAGES, int WQ>
int launch_grouped(const CUtensorMap& tw, const CUtensorMap& tx, const GArgs& a, const GQuant& q, int max_chunks,
                   cudaStream_t st) {
  using S = GSmem<BN, STAGES, WQ>;
  static_assert(S::kTotal <= 227 * 1024, "shared memory plan exceeds the per-CTA limit");
  if (int e = smem_attr_once<grouped_kernel<BN, STAGES, WQ>>(S::kTotal)) return e;
  cudaError_t e = launch_k(grouped_kernel<BN, STAGES, WQ>, dim3((a.N + 127) / 128, max_chunks), dim3(S::kThreads),
                           S::kTotal, st, 1, tw, tx, a, q);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

template <int WQ>
int dispatch_grouped(int BN, const CUtensorMap& tw, const CUtensorMap& tx, const GArgs& a, const GQuant& q,
                     int max_chunks, cudaStream_t st) {
  switch (BN) {
    case 16: return launch_grouped<16, WQ ? 3 : 6, WQ>(tw, tx, a, q, max_chunks, st);
    case 32: return launch_grouped<32, WQ ? 3 : 6, WQ>(tw, tx, a, q, max_chunks, st);
    case 64: return launch_grouped<64, WQ ? 2 : 4, WQ>(tw, tx, a, q, max_chunks, st);
    case 128: return launch_grouped<128, WQ ? 2 : 4, WQ>(tw, tx, a, q, max_chunks, st);
    default: return -1;
  }
}

}  // namespace moe
}  // namespace b200

using namespace b200;

extern "C" {

// mode 2 (sigmoid, group-limited, corrected selection): bias [E] or null,
// n_group dividing E (<= 32), topk_group <= n_group, scale on the weights
int b200_moe_route_topk(const float* logits, int T, int E, int k, int mode, int norm_topk, int* ids, float* w,
                        const float* bias, int n_group, int topk_group, float scale, cudaStream_t st) {
  if (T <= 0) return 0;
  if (E > 256 || k > 16 || mode < 0 || mode > 2) return -1;
  if (mode == 2 && (n_group < 1 || n_group > 32 || E % n_group || topk_group < 1 || topk_group > n_group ||
                    k > (E / n_group) * topk_group))
    return -1;
  RouteExtra ex;
  ex.bias = bias;
  ex.n_group = n_group;
  ex.topk_group = topk_group;
  ex.scale = scale;
  cudaError_t e = launch_k(moe::route_topk_kernel, dim3((T + 3) / 4), dim3(128), 0, st, 1, logits, T, E, k, mode,
                           norm_topk, ids, w, ex);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_moe_sort(const int* ids, int P, int E, int BN, int max_chunks, int* perm, int* pos, int* chunks,
                  int* n_chunks, cudaStream_t st) {
  if (E > 1024 || P <= 0) return P < 0 ? -1 : (E > 1024 ? -1 : 0);
  const int smem = (33 * E + 1) * (int)sizeof(int);
  if (int e = b200::smem_attr_once<moe::sort_kernel>((33 * 1024 + 1) * 4)) return e;
  cudaError_t e = launch_k(moe::sort_kernel, dim3(1), dim3(1024), smem, st, 1, ids, P, E, BN, max_chunks, perm, pos,
                           chunks, n_chunks);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_moe_gather(const void* x, int K, const int* perm, int P, int k, void* xs, int to_f16, cudaStream_t st) {
  if (P <= 0) return 0;
  if (K % 8) return -1;
  cudaError_t e = launch_k(moe::gather_kernel, dim3(P), dim3(128), 0, st, 1,
                           reinterpret_cast<const __nv_bfloat16*>(x), K, perm, P, k, reinterpret_cast<__nv_bfloat16*>(xs),
                           to_f16);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_moe_combine(const void* ys, int T, int N, const int* pos, const float* w, int k, void* out,
                     const void* bias_d, const int* ids, cudaStream_t st) {
  if (T <= 0) return 0;
  cudaError_t e = launch_k(moe::combine_kernel, dim3(T), dim3(256), 0, st, 1, reinterpret_cast<const __nv_bfloat16*>(ys),
                           N, pos, w, k, reinterpret_cast<__nv_bfloat16*>(out),
                           reinterpret_cast<const __nv_bfloat16*>(bias_d), ids);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// Grouped GEMM over expert chunks: Y[rows of chunk] = epi(Xs[rows] . W[e]^T (+ bias[e])).
// W: [E * N, K] (experts stacked), Xs: [P, K] sorted rows. BN is the chunk row cap.
int b200_moe_grouped_gemm(const void* xs, int P, int K, const void* W, int E, int N, void* Y, int ldy,
                          const void* bias, int epi, const int* chunks, const int* n_chunks, int max_chunks, int BN,
                          cudaStream_t st) {
  if (P <= 0) return 0;
  if (K % 8) return -1;
  CUtensorMap tw, tx;
  if (!make_tmap_2d(&tw, W, (int64_t)E * N, K, K, 128, 64, 2)) return -1;
  if (!make_tmap_2d(&tx, xs, P, K, K, BN, 64, 2)) return -1;
  moe::GArgs a{reinterpret_cast<__nv_bfloat16*>(Y), reinterpret_cast<const __nv_bfloat16*>(bias), chunks, n_chunks,
               N, K, ldy, epi, 0};
  moe::GQuant q = {};
  return moe::dispatch_grouped<0>(BN, tw, tx, a, q, max_chunks, st);
}

// Same with affine-quantised experts in the tile-major device layout: per
// expert ceil(N/128) tiles of K/64 records {codes [128][bits*8 B], scales,
// biases [gpb][128] bf16} (rows past N are zero).
// `persistent` > 0: chunks of <= 32 rows run on that many persistent CTAs
// (one per SM); 0 = one CTA per (tile, chunk).
// `f16` (MXFP4 only): natural-order records, f16 activation rows xs, f16
// dequantised weights (kind::f16 with both operands f16); `y_f16`: f16 Y.
int b200_moe_grouped_gemm_q(const void* xs, int P, int K, const void* tiled, int bits, int gs, int E, int N, void* Y,
                            int ldy, const void* bias, int epi, const int* chunks, const int* n_chunks, int max_chunks,
                            int BN, int persistent, int f16, int y_f16, cudaStream_t st) {
  if (P <= 0) return 0;
  if ((K % 64) || (gs == 128 && K % 128) || (N % 8) || (bits != 4 && bits != 8 && bits != kWqE2M1) ||
      (gs != 16 && gs != 32 && gs != 64 && gs != 128))
    return -1;
  if ((bits == kWqE2M1 ? (gs != 16 && gs != 32) : (gs == 16)) || ((uintptr_t)tiled & 15)) return -1;
  CUtensorMap tx;
  moe::GQuant q;
  q.tiled = reinterpret_cast<const uint8_t*>(tiled);
  q.gs = gs;
  q.gpb = gs == 16 ? 4 : gs == 32 ? 2 : 1;
  q.rec_bytes = bits == kWqE2M1 ? 4 * 128 * 8 + q.gpb * 256 : bits * 128 * 8 + q.gpb * 512;
  q.kb_total = K / 64;
  q.tiles_per_expert = (N + 127) / 128;
  if (!make_tmap_2d(&tx, xs, P, K, K, BN, 64, 2)) return -1;
  moe::GArgs a{reinterpret_cast<__nv_bfloat16*>(Y), reinterpret_cast<const __nv_bfloat16*>(bias), chunks, n_chunks,
               N, K, ldy, epi, y_f16};
  if (f16) {
    if (bits != kWqE2M1) return -1;
    if (BN <= 32 && persistent > 0) return moe::dispatch_persistent<kWqE2M1, true>(BN, tx, a, q, persistent, st);
    return moe::dispatch_grouped_f16(BN, tx, a, q, max_chunks, st);
  }
  if (BN <= 32 && persistent > 0) {  // decode-sized chunks: one CTA per SM over all work items
    if (bits == kWqE2M1) return moe::dispatch_persistent<kWqE2M1>(BN, tx, a, q, persistent, st);
    return bits == 4 ? moe::dispatch_persistent<4>(BN, tx, a, q, persistent, st)
                     : moe::dispatch_persistent<8>(BN, tx, a, q, persistent, st);
  }
  if (bits == kWqE2M1) return moe::dispatch_grouped<kWqE2M1>(BN, tx, tx, a, q, max_chunks, st);
  return bits == 4 ? moe::dispatch_grouped<4>(BN, tx, tx, a, q, max_chunks, st)
                   : moe::dispatch_grouped<8>(BN, tx, tx, a, q, max_chunks, st);
}

// Diagnostics / test hook: out[b] = cvt.rn.f16x2.e2m1x2 of byte b, b = 0..255.
int b200_e2m1_pairs(uint32_t* out, cudaStream_t st) {
  cudaError_t e = launch_k(moe::e2m1_pairs_kernel, dim3(1), dim3(256), 0, st, 0, out);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"

B200_STATUS_ACCESSORS(moe)
