// Dense bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// with split-K reduced inside a thread-block cluster over distributed shared
// memory.
//
//   Y[M, N] = epi(X[M, K] . W[N, K]^T + bias)     (X: activations, W: nn.Linear weight)
//
// Orientation ("swap AB"): the MMA's 128-row M side walks the weight rows
// (output features) and its N side walks the tokens, so a decode batch of
// 1..128 rows still fills the 128-lane accumulator.
//
// Grid (N/128, ceil(M/BN), S) with cluster (1, 1, S): the S CTAs of a cluster
// own the same 128 x BN output tile and disjoint, fixed ranges of 64-wide K
// blocks. Per CTA:
//   warp 0 / lane 0 : TMA producer (weights evict-first, activations evict-last)
//   warp 1 / lane 0 : MMA issuer (tcgen05.mma kind::f16, fp32 accumulator in TMEM)
//   warps 0..3      : drain TMEM -> this CTA's shared memory as an fp32 partial
// then, after a cluster barrier, CTA z reduces token columns [z*BN/S, ...) of
// the tile by reading the S partials through DSMEM (mapa + ld.shared::cluster)
// in split order 0..S-1, applies the epilogue and stores. S depends only on
// (N, K) - never on M - so a row's result is bit-identical whatever the batch
// (decode rows alone, or mixed with prefill chunks): the batch-composition
// invariance the reference engine guarantees (docs/engine-v2/TESTPLAN.md).
//
// Replaces the MLX matmul the reference uses for every Linear
// (Libraries/MLXLMCommon/SwitchLayers.swift:1361 and the model files).
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "b200_common.cuh"
#include "b200_comm.cuh"
#include "b200_dequant.cuh"

#include <memory>

namespace b200 {

enum GemmEpilogue : int {
  kEpiStoreBf16 = 0,  // Y = bf16(acc)
  kEpiSwiGLU = 1,     // W rows interleaved in 64-row gate/up halves: Y[:, f] = silu(gate) * up
  kEpiStoreF32 = 2,   // Y = acc (fp32)
  kEpiAddBf16 = 3,    // Y = bf16(bf16(acc) + R)   (R has Y's layout)
  kEpiGeGLU = 4,      // as kEpiSwiGLU with gelu(tanh approximation) on the gate
  kEpiSwiGLUOAI = 5,  // GPT-OSS gate: g=min(g,7), u=clamp(u,-7,7), (u+1)*g*sigmoid(1.702g)
  kEpiGelu = 6,       // Y = bf16(gelu(acc)), erf form (BERT-family FFNs)
  kEpiGeluTanh = 7,   // Y = bf16(gelu(acc)), tanh approximation
  kEpiQuickGelu = 8,  // Y = bf16(acc * sigmoid(1.702 acc)) (CLIP / Qwen-VL vision MLPs)
  kEpiRelu2 = 9,      // Y = bf16(relu(acc)^2) (NemotronH / Nemotron 3 MLPs)
  kEpiQKRope = 10,    // fused q|k|v projection, head dim 128: qk-norm + RoPE + paged K/V append (RopeKvEpi)
};

// kEpiQKRope: each 128-row weight tile is one head of the q|k|v projection
// (head dim 128, full non-interleaved rotary). The epilogue rounds the
// projection to bf16 (as the unfused GEMM output), applies the q/k RMSNorm
// weights (warp reduction over the head), rotates with the cos|sin table row
// of the token's position (partners 64 channels apart = lane ^ 16), stores q
// into q_out [M, H, 128] and k / v into the paged cache slot of the token
// (bf16, or fp8-e4m3 divided by the per-head scale); slot < 0 skips.
struct RopeKvEpi {
  const int* positions;
  const int64_t* slots;
  const float* cos_sin;  // [max_pos, 128] fp32: cos | sin
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  __nv_bfloat16* q_out;
  void* k_cache;  // [pages, KVH, 16, 128]
  void* v_cache;
  const float* k_scale;
  const float* v_scale;
  int64_t num_slots;
  float eps;
  int H, KVH, kv_fp8;
};

__device__ __forceinline__ float gelu_act(int epi, float x) {
  if (epi == kEpiGelu) return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
  if (epi == kEpiQuickGelu) return x / (1.f + __expf(-1.702f * x));
  if (epi == kEpiRelu2) return x > 0.f ? x * x : 0.f;
  const float c = 0.7978845608028654f;  // sqrt(2/pi)
  return 0.5f * x * (1.f + tanhf(c * (x + 0.044715f * x * x * x)));
}

static_assert(kEpiSwiGLU == kGluSwi && kEpiGeGLU == kGluGe && kEpiSwiGLUOAI == kGluOAI, "glu_act codes");

struct GemmArgs {
  void* Y;
  const __nv_bfloat16* R;
  const __nv_bfloat16* bias;  // [N] per row of W, or null
  int M, N, K, ldy, ldr;
  int kb_total, kb_per_split, ksplit;
  int epi;
  unsigned long long* trace;  // optional [ctas][6] %globaltimer stamps (diagnostics), null in production
  unsigned long long* ktrace;  // optional per-K-block stamps of CTA 0 (diagnostics), null in production
  RopeKvEpi rk;                // kEpiQKRope only
};

__device__ __forceinline__ void store4_kv(void* cache, bool fp8, size_t idx, const float* x, float sc) {
  if (fp8) {
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_fp8_e4m3 f(x[e] * sc);
      w |= (uint32_t)(*reinterpret_cast<uint8_t*>(&f)) << (8 * e);
    }
    *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(cache) + idx) = w;
  } else {
    __nv_bfloat16 o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = f2bf(x[e]);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(cache) + idx) = *reinterpret_cast<const uint2*>(o);
  }
}

// Shared-memory plan of one CTA.
// bf16 weights (WQ = 0): STAGES stages of {A weight tile (TMA), B activation
// tile}, barriers full/empty per stage.
// Quantised weights (WQ = 4 / 8): a deep raw ring of kRawStages records
// {codes [128][WQ*8 B], scales, biases [gpb][128] bf16}, one contiguous bulk
// copy each (a 4-bit record is only 4.5-5 KB, so many are in flight to cover
// DRAM latency). Eight dequantising warps (two groups of four taking
// alternate K blocks) expand a record into the bf16 A
// tile and write it straight into tensor memory (tcgen05.st; 32 columns per
// stage after the accumulator); the MMA reads A from there (tcgen05.mma with
// an A operand in tensor memory), so shared-memory stages hold only the
// activation tile. Barriers: full[s] (activation bytes + one arrive per
// dequantising warp + the producer's arrive), empty[s] (MMA consumed the
// stage), rfull/rempty per raw record.
// MT = 2 (bf16 weights, no split-K): two 128-row weight tiles share each
// activation tile, with two accumulators in tensor memory (2 x BN columns):
// a 256 x BN output tile per CTA moves half the operand bytes per FLOP of the
// 128 x BN tile, which keeps large (prefill) GEMMs off the L2-to-SM bandwidth
// limit.
template <int BN, int STAGES, int WQ = 0, int MT = 1>
struct GemmSmem {
  static constexpr int kABytes = 128 * 128;  // 128 rows x 64 bf16 (one weight tile of a stage)
  static constexpr int kBBytes = BN * 128;   // BN rows x 64 bf16
  static constexpr int kCodeBytes = code_bits<WQ>() * 128 * 64 / 8;
  static constexpr int kGroupBytes = 2 * 128 * 2;  // up to 2 groups x 128 rows x bf16
  static constexpr int kRawBytes = WQ ? kCodeBytes + 2 * kGroupBytes : 0;
  static constexpr int kStageBytes = ((WQ ? 0 : MT * kABytes) + kBBytes + 1023) / 1024 * 1024;
  static constexpr int kPipeBytes = STAGES * kStageBytes;
  static constexpr int kRawBudget = 200 * 1024 - kPipeBytes;
  static constexpr int kRawStages = WQ ? (kRawBudget / kRawBytes > 24 ? 24 : kRawBudget / kRawBytes) : 0;
  static constexpr int kRawOffset = kPipeBytes;
  static constexpr int kAllPipe = kPipeBytes + kRawStages * kRawBytes;
  static constexpr int kPartBytes = BN * 128 * 4;  // fp32 partial [BN][128]
  static constexpr int kMain = kAllPipe > kPartBytes ? kAllPipe : kPartBytes;
  static constexpr int kBarOffset = (kMain + 7) / 8 * 8;
  static constexpr int kNumBars = 2 * STAGES + 1 + (WQ ? 2 * kRawStages : 0);
  static constexpr int kTotal = kBarOffset + kNumBars * 8 + 16 + 1024;  // + alignment slack
  static constexpr int kAccCols = BN < 32 ? 32 : BN;
  static constexpr int kNeedCols = MT * kAccCols + (WQ ? STAGES * 32 : 0);
  static_assert(MT == 1 || WQ == 0, "two weight tiles per CTA serve bf16 weights only");
  static constexpr int kTmemCols = kNeedCols <= 32 ? 32 : kNeedCols <= 64 ? 64 : kNeedCols <= 128 ? 128
                                   : kNeedCols <= 256 ? 256 : 512;
  static_assert(kNeedCols <= 512, "tensor memory plan exceeds 512 columns");
  static constexpr int kThreads = WQ ? 384 : 128;  // + 8 dequantising warps (two per SM sub-partition)
  static_assert(!WQ || kRawStages >= 4, "raw ring too shallow");
};

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Generic address of the same shared-memory variable in cluster CTA `rank`
// (distributed shared memory); plain loads through it batch and overlap.
__device__ __forceinline__ const float* map_cluster_rank(const float* p, uint32_t rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
  return reinterpret_cast<const float*>(r);
}

// Collective modes of the GEMM (tensor parallelism over symmetric memory).
enum GemmMode : int {
  kModeLocal = 0,  // X from local memory, Y stored locally
  kModeAG = 1,     // all-gather prologue: X rows are fetched from every rank's published rows
  kModeRS = 2,     // reduce-scatter epilogue: fp32 partial rows stored into the owner rank's inbox
};

struct CollArgs {
  CUtensorMap peer_x[2 * kMaxRanks];  // AG: [parity] maps over this rank's gathered rows (entries 0, 1)
  CommCtx comm;
  int phase;   // collective phase index within the step (epoch = step * kPhasesPerStep + phase + 1)
  int parity;  // buffer slot of this call
  int rs_all;  // reduce-scatter epilogue: 1 = the partial rows go to every rank (each rank reduces all rows),
              // 2 = the same with bf16 partials, 3 = bf16 partials stored to this rank's own
              // multicast-bound buffer `nvls_local` (the combine sums them in the NVSwitch)
  __nv_bfloat16* nvls_local;  // [2][world*rows_per_rank][hidden] (rs_all == 3)
};

// Affine-quantised weights (WQ bits per code): w = scale[g] * q + bias[g] per
// group of `gs` inputs. codes: [N, K*WQ/8] bytes (4-bit words repacked so that
// nibble j of the low half-word and nibble j of the high half-word hold inputs
// 2j and 2j+1 of the word's 8); scales / biases: [K/gs, N] bf16.
struct QArgs {
  const uint8_t* tiled;  // tile-major records [N/128][K/64][rec_bytes]
  int gs, gpb, rec_bytes, kb_total;
};

template <int BN, int STAGES, int MODE, int WQ, int MT = 1>
__global__ void __launch_bounds__(GemmSmem<BN, STAGES, WQ, MT>::kThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                        GemmArgs args, const __grid_constant__ CollArgs coll, const __grid_constant__ QArgs qa) {
  using S = GemmSmem<BN, STAGES, WQ, MT>;
  constexpr int kThreads = S::kThreads;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  constexpr int RS = S::kRawStages;
  const uint32_t bar_full = sbase + S::kBarOffset;   // [STAGES] operands of the stage in place
  const uint32_t bar_empty = bar_full + STAGES * 8;  // [STAGES] stage consumed by the MMA
  const uint32_t bar_accum = bar_empty + STAGES * 8;
  const uint32_t bar_rfull = bar_accum + 8;          // [RS] quantised: raw record landed
  const uint32_t bar_rempty = bar_rfull + RS * 8;    // [RS] quantised: raw record consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kBarOffset + S::kNumBars * 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128 * MT;
  const int m0 = blockIdx.y * BN;
  const int z = blockIdx.z;
  const int kb_begin = z * args.kb_per_split;
  const int kb_end = min(args.kb_total, kb_begin + args.kb_per_split);
  const int nkb = kb_end - kb_begin;

  pdl_launch_dependents();
  unsigned long long* trace =
      args.trace ? args.trace + 6 * (blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)) : nullptr;
  if (trace && threadIdx.x == 0) trace[0] = globaltimer();
  if (threadIdx.x == 0) {
    if constexpr (WQ == 0) tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, WQ ? 5 : 1);  // quantised: activation producer + four dequantising warps
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(bar_rfull + 8 * s, 1);
      mbar_init(bar_rempty + 8 * s, 4);
    }
    mbar_init(bar_accum, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (trace && threadIdx.x == 0) trace[1] = globaltimer();

  if constexpr (WQ == 0) {
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    const uint64_t pol_w = l2_policy_evict_first();
    const uint64_t pol_x = l2_policy_evict_last();
    const uint32_t stage_tx = (uint32_t)(MT * S::kABytes + S::kBBytes);
    // Weights are written by no kernel: the first STAGES weight tiles are
    // requested before waiting on the previous kernel (PDL), so their HBM
    // latency overlaps the predecessor's tail.
    const int pre = min(STAGES, nkb);
    for (int i = 0; i < pre; ++i) {
      const uint32_t a = sbase + i * S::kStageBytes;
      mbar_arrive_expect_tx(bar_full + 8 * i, stage_tx);
#pragma unroll
      for (int h = 0; h < MT; ++h)
        tma_load_2d(a + h * S::kABytes, &tmW, bar_full + 8 * i, (kb_begin + i) * 64, n0 + 128 * h, pol_w);
    }
    pdl_wait();
    // Activation tile: local TMA; in all-gather mode from the gathered buffer
    // that every rank's combine kernel has pushed its rows into (local).
    auto load_x = [&](uint32_t b, uint32_t bar, int kc) {
      if constexpr (MODE == kModeAG) {
        tma_load_2d(b, &coll.peer_x[coll.parity], bar, kc, 0, pol_x);
      } else {
        tma_load_2d(b, &tmX, bar, kc, m0, pol_x);
      }
    };
    if constexpr (MODE == kModeAG) {
      // every rank must have published this phase's rows (bounded wait)
      const uint32_t ep = coll.comm.epoch(coll.phase);
      for (int j = 0; j < coll.comm.world; ++j) wait_counter(coll.comm.pad_ptr(coll.comm.rank, kPadAG, j), ep);
      if ((blockIdx.x | blockIdx.y | blockIdx.z) == 0) timeline_tag(0x200 + kPadAG);
    }
    for (int i = 0; i < pre; ++i)
      load_x(sbase + i * S::kStageBytes + MT * S::kABytes, bar_full + 8 * i, (kb_begin + i) * 64);
    int issued = pre;
    for (int i = pre; i < nkb; ++i) {
      const int s = i % STAGES, r = i / STAGES;
      if (r > 0 && !mbar_wait(bar_empty + 8 * s, (r - 1) & 1, kErrGemmWait)) break;
      const uint32_t a = sbase + s * S::kStageBytes;
      const uint32_t b = a + MT * S::kABytes;
      mbar_arrive_expect_tx(bar_full + 8 * s, stage_tx);
      const int kc = (kb_begin + i) * 64;
#pragma unroll
      for (int h = 0; h < MT; ++h) tma_load_2d(a + h * S::kABytes, &tmW, bar_full + 8 * s, kc, n0 + 128 * h, pol_w);
      load_x(b, bar_full + 8 * s, kc);
      issued = i + 1;
    }
    // make sure no copy issued here is still landing when the stage memory is reused
    for (int i = max(0, issued - STAGES); i < issued; ++i)
      mbar_wait(bar_full + 8 * (i % STAGES), (i / STAGES) & 1, kErrGemmWait);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES, r = i / STAGES;
      if (!mbar_wait(bar_full + 8 * s, r & 1, kErrGemmWait)) break;
      if (args.ktrace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) args.ktrace[2 * nkb + i] = globaltimer();
      if (trace && i == 0) trace[2] = globaltimer();
      tc_fence_after();
      const uint32_t a = sbase + s * S::kStageBytes;
      const uint32_t b = a + MT * S::kABytes;
      const uint64_t bd = umma_desc_k_sw128(b, 1024);
#pragma unroll
      for (int h = 0; h < MT; ++h) {
        const uint64_t ad = umma_desc_k_sw128(a + h * S::kABytes, 1024);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16(tmem + h * S::kAccCols, ad + 2 * k, bd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
      }
      tc_commit(bar_empty + 8 * s);
    }
    tc_commit(bar_accum);
  }
  } else {
  // ---------------- quantised weights ----------------
  if (warp == 0 && lane == 0) {
    // raw producer: one contiguous record {codes, scales, biases} per K block,
    // RS records ahead (weights are written by no kernel, so the ring is
    // requested before the PDL wait)
    const uint64_t pol_w = l2_policy_evict_first();
    const uint8_t* tile = qa.tiled + (size_t)blockIdx.x * qa.kb_total * qa.rec_bytes;
    int issued = 0;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % RS, r = i / RS;
      if (r > 0 && !mbar_wait(bar_rempty + 8 * s, (r - 1) & 1, kErrGemmWait)) break;
      const uint32_t raw = sbase + S::kRawOffset + s * S::kRawBytes;
      mbar_arrive_expect_tx(bar_rfull + 8 * s, (uint32_t)qa.rec_bytes);
      bulk_g2s(raw, tile + (size_t)(kb_begin + i) * qa.rec_bytes, (uint32_t)qa.rec_bytes, bar_rfull + 8 * s, pol_w);
      issued = i + 1;
    }
    for (int i = max(0, issued - RS); i < issued; ++i)
      mbar_wait(bar_rfull + 8 * (i % RS), (i / RS) & 1, kErrGemmWait);
  } else if (warp == 2 && lane == 0) {
    // activation producer
    const uint64_t pol_x = l2_policy_evict_last();
    pdl_wait();
    int issued = 0;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES, r = i / STAGES;
      if (r > 0 && !mbar_wait(bar_empty + 8 * s, (r - 1) & 1, kErrGemmWait)) break;
      mbar_arrive_expect_tx(bar_full + 8 * s, S::kBBytes);
      tma_load_2d(sbase + s * S::kStageBytes, &tmX, bar_full + 8 * s, (kb_begin + i) * 64, m0, pol_x);
      issued = i + 1;
    }
    for (int i = max(0, issued - STAGES); i < issued; ++i)
      mbar_wait(bar_full + 8 * (i % STAGES), (i / STAGES) & 1, kErrGemmWait);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % STAGES, r = i / STAGES;
      if (!mbar_wait(bar_full + 8 * s, r & 1, kErrGemmWait)) break;
      if (args.ktrace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) args.ktrace[2 * nkb + i] = globaltimer();
      if (trace && i == 0) trace[2] = globaltimer();
      tc_fence_after();
      const uint64_t bd = umma_desc_k_sw128(sbase + s * S::kStageBytes, 1024);
      const uint32_t at = tmem + S::kAccCols + s * 32;  // A stage: 32 columns = 64 bf16 per lane
#pragma unroll
      for (int k = 0; k < 4; ++k) tc_mma_f16_ts(tmem, at + 8 * k, bd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
      tc_commit(bar_empty + 8 * s);
    }
    tc_commit(bar_accum);
  } else if (warp >= 4) {
    // Eight dequantising warps in two groups of four; group g converts the
    // K blocks i with i % 2 == g, so two blocks are in flight at once. Thread
    // t of a group owns weight row t and stores its 64 inputs as 32
    // tensor-memory columns of lane t.
    const int t = (threadIdx.x - 128) & 127;
    const int grp = (threadIdx.x - 128) >> 7;
    const int g1 = qa.gs == 16 ? 2 : qa.gs == 32 ? 1 : 0;  // first group of the second half
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16) + S::kAccCols;
    for (int i = grp; i < nkb; i += 2) {
      const int rs = i % RS, rr = i / RS;
      const int s = i % STAGES, r = i / STAGES;
      if (!mbar_wait(bar_rfull + 8 * rs, rr & 1, kErrGemmWait)) break;
      const bool kt = args.ktrace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 128;
      if (kt) args.ktrace[i] = globaltimer();
      if (r > 0 && !mbar_wait(bar_empty + 8 * s, (r - 1) & 1, kErrGemmWait)) break;
      const uint8_t* raw = smem + S::kRawOffset + rs * S::kRawBytes;
      uint32_t v0[16], v1[16];
      dequant_half_row_regs<WQ>(raw, t, 0, 0, qa.gpb, v0);
      dequant_half_row_regs<WQ>(raw, t, 1, g1, qa.gpb, v1);
      tmem_st16(lane_base + s * 32, v0);
      tmem_st16(lane_base + s * 32 + 16, v1);
      tc_wait_st();
      tc_fence_before();
      if (kt) args.ktrace[nkb + i] = globaltimer();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar_rempty + 8 * rs);
        mbar_arrive(bar_full + 8 * s);
      }
    }
  }
  }
  __syncwarp();

  // every thread that touches global memory below orders itself after the
  // previous kernel (the producer thread already did)
  if (WQ != 0 || !(warp == 0 && lane == 0)) pdl_wait();
  // ---------------- drain TMEM into this CTA's fp32 partial [BN][128] ----------------
  const bool acc_ok = __syncthreads_and(mbar_wait(bar_accum, 0, kErrTmemWait) ? 1 : 0) != 0;
  tc_fence_after();
  if (trace && threadIdx.x == 0) trace[3] = globaltimer();
  // one pass per weight tile of the CTA (MT = 2: the second accumulator after the first)
  for (int hh = 0; hh < MT; ++hh) {
    const int n0e = n0 + 128 * hh;
    if (n0e >= args.N) break;     // a last CTA's second tile past the weight rows (uniform branch)
    if (hh > 0) __syncthreads();  // the previous pass's epilogue has finished reading the partial
    const int r = warp * 32 + lane;  // TMEM lane == weight row within the tile
    float* part = reinterpret_cast<float*>(smem);
    if (warp < 4) {
      const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16) + hh * S::kAccCols;
#pragma unroll 1
      for (int jc = 0; jc < BN; jc += 16) {
        uint32_t v[16];
        tmem_ld16(t_lane + jc, v);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) part[(jc + j) * 128 + r] = (acc_ok && nkb > 0) ? __uint_as_float(v[j]) : 0.f;
      }
    }
    tc_fence_before();
    if (args.ksplit > 1) cluster_sync();
    else __syncthreads();
    if (trace && threadIdx.x == 0) trace[4] = globaltimer();

    // ---------------- cluster reduction + epilogue ----------------
    const int ks = args.ksplit;
    const int js = (BN + ks - 1) / ks;
    const int j_lo = z * js;
    const int j_hi = min(BN, min(j_lo + js, args.M - m0));
    // Partials are [BN][128] fp32 rows = 32 float4 per token column. Each thread
    // sums whole float4s of the S partials in split order 0..S-1; all S loads of
    // a float4 are issued before the adds so their DSMEM latencies overlap.
    const float4* rp[8];
#pragma unroll
    for (int q = 0; q < 8; ++q)
      rp[q] = reinterpret_cast<const float4*>((q < ks) ? (ks > 1 ? map_cluster_rank(part, q) : part) : part);
    auto red4 = [&](int j, int r4) -> float4 {
      const int off = j * 32 + r4;
      float4 v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q < ks) v[q] = rp[q][off];
      float4 acc = v[0];
#pragma unroll
      for (int q = 1; q < 8; ++q)
        if (q < ks) {
          acc.x += v[q].x;
          acc.y += v[q].y;
          acc.z += v[q].z;
          acc.w += v[q].w;
        }
      return acc;
    };
    const bool glu = args.epi == kEpiSwiGLU || args.epi == kEpiGeGLU || args.epi == kEpiSwiGLUOAI;
    if (glu) {
      // 16 threads per token column (64 gate rows as 16 float4), 8 columns per pass
      const int jj = threadIdx.x >> 4, f4 = threadIdx.x & 15;
      constexpr int kColsPerPass = kThreads / 16;
      __nv_bfloat16* Y = reinterpret_cast<__nv_bfloat16*>(args.Y);
      float bg[4], bu[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        bg[e] = args.bias ? bf2f(args.bias[n0e + f4 * 4 + e]) : 0.f;
        bu[e] = args.bias ? bf2f(args.bias[n0e + 64 + f4 * 4 + e]) : 0.f;
      }
      for (int j = j_lo + jj; j < j_hi; j += kColsPerPass) {
        const float4 g4 = red4(j, f4), u4 = red4(j, f4 + 16);
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
        __nv_bfloat16 o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // round the gate and up projections to bf16 first, as an unfused bf16
          // model would, then apply the activation in fp32
          const float g = bf2f(f2bf(gv[e] + bg[e]));
          const float u = bf2f(f2bf(uv[e] + bu[e]));
          o[e] = f2bf(glu_act(args.epi, g, u));
        }
        const int f = (n0e >> 1) + f4 * 4;
        __nv_bfloat16* dst = Y + (size_t)(m0 + j) * args.ldy + f;
        if (f + 3 < (args.N >> 1) && (((uintptr_t)dst) & 7) == 0) {
          *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (f + e < (args.N >> 1)) dst[e] = o[e];
        }
      }
    } else {
      // 32 threads per token column (128 rows as 32 float4), 4 columns per pass
      const int jj = threadIdx.x >> 5, r4 = threadIdx.x & 31;
      constexpr int kColsPerPass = kThreads / 32;
      const int n = n0e + r4 * 4;
      float bb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) bb[e] = (args.bias && n + e < args.N) ? bf2f(args.bias[n + e]) : 0.f;
      for (int j = j_lo + jj; j < j_hi; j += kColsPerPass) {
        const float4 v4 = red4(j, r4);
        const float v[4] = {v4.x + bb[0], v4.y + bb[1], v4.z + bb[2], v4.w + bb[3]};
        const size_t m = (size_t)(m0 + j);
        if (MODE == kModeLocal && args.epi == kEpiQKRope) {
          // one warp per token column: the warp holds the token's whole head (4 channels per lane)
          const RopeKvEpi& rk = args.rk;
          const int head = n0e >> 7, d0 = r4 * 4;
          float x[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) x[e] = bf2f(f2bf(v[e]));
          const int64_t slot = rk.slots ? rk.slots[m] : -1;
          const bool slot_ok = slot >= 0 && slot < rk.num_slots;
          if (rk.slots && slot >= rk.num_slots && r4 == 0) set_status(kErrBounds);
          if (head < rk.H + rk.KVH) {
            const bool is_q = head < rk.H;
            const __nv_bfloat16* nw = is_q ? rk.qw : rk.kw;
            if (nw) {
              const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
              const float inv = rsqrtf(ss / 128.f + rk.eps);
#pragma unroll
              for (int e = 0; e < 4; ++e) x[e] = bf2f(f2bf(x[e] * inv * bf2f(nw[d0 + e])));
            }
            // cos|sin of the 4 channels' frequencies: two 16-byte loads
            const float* cs = rk.cos_sin + (size_t)rk.positions[m] * 128 + (d0 & 63);
            const float4 c4 = *reinterpret_cast<const float4*>(cs);
            const float4 s4 = *reinterpret_cast<const float4*>(cs + 64);
            const float cv[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float p = __shfl_xor_sync(0xffffffffu, x[e], 16);
              o[e] = d0 < 64 ? x[e] * cv[e] - p * sv[e] : x[e] * cv[e] + p * sv[e];
            }
            if (is_q) {
              __nv_bfloat16 q[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) q[e] = f2bf(o[e]);
              *reinterpret_cast<uint2*>(rk.q_out + (m * rk.H + head) * 128 + d0) = *reinterpret_cast<const uint2*>(q);
            } else if (slot_ok) {
              const int kvh = head - rk.H;
              float kb[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) kb[e] = bf2f(f2bf(o[e]));
              const size_t idx = ((size_t)((slot >> 4) * rk.KVH + kvh) * 16 + (slot & 15)) * 128 + d0;
              store4_kv(rk.k_cache, rk.kv_fp8, idx, kb, rk.k_scale ? 1.f / rk.k_scale[kvh] : 1.f);
            }
          } else if (slot_ok) {
            const int kvh = head - rk.H - rk.KVH;
            const size_t idx = ((size_t)((slot >> 4) * rk.KVH + kvh) * 16 + (slot & 15)) * 128 + d0;
            store4_kv(rk.v_cache, rk.kv_fp8, idx, x, rk.v_scale ? 1.f / rk.v_scale[kvh] : 1.f);
          }
          continue;
        }
        if constexpr (MODE == kModeRS) {
          const int rpr = coll.comm.rows_per_rank;
          const int W = coll.rs_all ? coll.comm.world : 1;
          for (int jj = 0; jj < W; ++jj) {
            // fp32 partial row m -> [parity][this rank][row] of its owner rank's inbox, or of
            // every rank's (rs_all, starting with this rank's own buffer)
            const int j = (coll.comm.rank + jj) % coll.comm.world;
            if (coll.rs_all == 3) {  // local store only; N % 4 == 0 here (checked at launch)
              __nv_bfloat16 o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) o[e] = f2bf(v[e]);
              const size_t M = (size_t)coll.comm.world * rpr;
              *reinterpret_cast<uint2*>(coll.nvls_local + ((size_t)coll.parity * M + m) * args.N + n) =
                  *reinterpret_cast<const uint2*>(o);
              break;
            }
            if (coll.rs_all == 2) {  // N % 4 == 0 here (checked at launch)
              __nv_bfloat16 o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) o[e] = f2bf(v[e]);
              *reinterpret_cast<uint2*>(coll.comm.recv_all_bf16(j, coll.parity, coll.comm.rank, (int)m) + n) =
                  *reinterpret_cast<const uint2*>(o);
              continue;
            }
            float* dst = coll.rs_all ? coll.comm.recv_all(j, coll.parity, coll.comm.rank, (int)m) + n
                                     : coll.comm.recv_row((int)m / rpr, coll.parity, coll.comm.rank, (int)m % rpr) + n;
            if (n + 3 < args.N) {
              *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (n + e < args.N) dst[e] = v[e];
            }
          }
        } else if (args.epi == kEpiStoreF32) {
          float* dst = reinterpret_cast<float*>(args.Y) + m * args.ldy + n;
          if (n + 3 < args.N && (((uintptr_t)dst) & 15) == 0) {
            *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (n + e < args.N) dst[e] = v[e];
          }
        } else {
          __nv_bfloat16 o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (args.epi == kEpiAddBf16) {
              const float rr = (n + e < args.N) ? bf2f(args.R[m * args.ldr + n + e]) : 0.f;
              o[e] = f2bf(bf2f(f2bf(v[e])) + rr);
            } else if (args.epi == kEpiGelu || args.epi == kEpiGeluTanh || args.epi == kEpiQuickGelu ||
                       args.epi == kEpiRelu2) {
              o[e] = f2bf(gelu_act(args.epi, v[e]));
            } else {
              o[e] = f2bf(v[e]);
            }
          }
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.Y) + m * args.ldy + n;
          if (n + 3 < args.N && (((uintptr_t)dst) & 7) == 0) {
            *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (n + e < args.N) dst[e] = o[e];
          }
        }
      }
    }
  }
  // stores made through the unicast address must be visible to peers that
  // read them through the multicast alias
  if constexpr (MODE == kModeRS) {
    if (coll.rs_all == 3) asm volatile("fence.proxy.alias;" ::: "memory");
  }
  // no CTA may leave while a peer still reads its partial
  if (args.ksplit > 1) cluster_sync();
  else __syncthreads();
  if constexpr (MODE == kModeRS) {
    if ((blockIdx.x | blockIdx.y | blockIdx.z) == 0 && threadIdx.x == 0) timeline_tag(0x300);  // epilogue done
    // all of this CTA's inbox stores are issued; the last CTA of the grid
    // publishes the phase to every rank
    if (threadIdx.x == 0) last_cta_signal(coll.comm, kPadRS, coll.comm.epoch(coll.phase));
  }
  if (trace && threadIdx.x == 0) trace[5] = globaltimer();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor-map cache + launch
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct TmKey {
  uintptr_t ptr;
  int64_t rows, cols, ld;
  int box_rows, box_cols, dtype_bytes;
  bool operator==(const TmKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows &&
           box_cols == o.box_cols && dtype_bytes == o.dtype_bytes;
  }
};
struct TmKeyHash {
  size_t operator()(const TmKey& k) const {
    size_t h = std::hash<uintptr_t>()(k.ptr);
    h ^= std::hash<int64_t>()(k.rows * 1315423911ll + k.cols * 2654435761ll + k.ld) + 0x9e3779b97f4a7c15ull + (h << 6);
    h ^= (size_t)(k.box_rows * 131 + k.box_cols * 7 + k.dtype_bytes);
    return h;
  }
};

// 2-D row-major tensor map, box = box_rows x box_cols, 128-byte swizzle or
// none. Returns false if the driver rejects the layout.
bool make_tmap_2d_sw(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows,
                     int box_cols, int dtype_bytes, bool swizzle128) {
  static std::mutex mu;
  static std::unordered_map<TmKey, CUtensorMap, TmKeyHash> cache;
  TmKey key{(uintptr_t)ptr, rows, cols, ld_elems, box_rows, box_cols, dtype_bytes * (swizzle128 ? 1 : 16)};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return true;
    }
  }
  auto enc = get_encode_fn();
  if (!enc) return false;
  CUtensorMapDataType dt = dtype_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : dtype_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)(ld_elems * dtype_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(out, dt, 2, const_cast<void*>(ptr), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, *out);
  return true;
}

// 2-D row-major tensor map with a 128-byte swizzle: box = box_rows x box_cols.
bool make_tmap_2d(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows,
                  int box_cols, int dtype_bytes) {
  return make_tmap_2d_sw(out, ptr, rows, cols, ld_elems, box_rows, box_cols, dtype_bytes, true);
}

static const QArgs& no_quant() {
  static QArgs q = {};
  return q;
}
static const CollArgs& local_coll_q() {
  static CollArgs c = {};
  return c;
}

template <int BN, int STAGES, int MODE, int WQ = 0, int MT = 1>
static int launch_gemm(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a, const CollArgs& coll,
                       int tiles_n, int tiles_m, cudaStream_t st, const QArgs& q = no_quant()) {
  using S = GemmSmem<BN, STAGES, WQ, MT>;
  static_assert(S::kTotal <= 227 * 1024, "shared memory plan exceeds the per-CTA limit");
  if (int e = smem_attr_once<gemm_bf16_tc_kernel<BN, STAGES, MODE, WQ, MT>>(S::kTotal)) return e;
  cudaError_t e = launch_k(gemm_bf16_tc_kernel<BN, STAGES, MODE, WQ, MT>, dim3(tiles_n, tiles_m, a.ksplit),
                           dim3(S::kThreads, 1, 1), S::kTotal, st, a.ksplit, tw, tx, a, coll, q);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}

template <int WQ>
static int launch_bn_q(int BN, const CUtensorMap& tx, const GemmArgs& a, const QArgs& q, int tiles_n, int tiles_m,
                       cudaStream_t st) {
  const CollArgs& c = local_coll_q();
  switch (BN) {
    // STAGES = tensor-memory A stages (32 columns each after the accumulator)
    // and activation stages in shared memory
    case 16: return launch_gemm<16, 14, kModeLocal, WQ>(tx, tx, a, c, tiles_n, tiles_m, st, q);
    case 32: return launch_gemm<32, 14, kModeLocal, WQ>(tx, tx, a, c, tiles_n, tiles_m, st, q);
    case 64: return launch_gemm<64, 12, kModeLocal, WQ>(tx, tx, a, c, tiles_n, tiles_m, st, q);
    case 128: return launch_gemm<128, 6, kModeLocal, WQ>(tx, tx, a, c, tiles_n, tiles_m, st, q);
    case 256: return launch_gemm<256, 3, kModeLocal, WQ>(tx, tx, a, c, tiles_n, tiles_m, st, q);
    default: return -1;
  }
}

template <int MODE>
static int launch_bn(int BN, const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a, const CollArgs& coll,
                     int tiles_n, int tiles_m, cudaStream_t st) {
  switch (BN) {
    case 16: return launch_gemm<16, 6, MODE>(tw, tx, a, coll, tiles_n, tiles_m, st);
    case 32: return launch_gemm<32, 5, MODE>(tw, tx, a, coll, tiles_n, tiles_m, st);
    case 64: return launch_gemm<64, 4, MODE>(tw, tx, a, coll, tiles_n, tiles_m, st);
    case 128: return launch_gemm<128, 3, MODE>(tw, tx, a, coll, tiles_n, tiles_m, st);
    case 256: return launch_gemm<256, 4, MODE>(tw, tx, a, coll, tiles_n, tiles_m, st);
    default: return -1;
  }
}

static const CollArgs& local_coll() {
  static CollArgs c = {};
  return c;
}

// Split count S (1..8, the cluster size) for a weight of N rows and K inputs.
// A function of (N, K) only: every M uses the same K partition and the same
// reduction order. Chosen so skinny (decode) GEMMs fill the machine with about
// two CTAs per SM while every split keeps at least 8 K blocks.
// Powers of two only (clusters of 2/4/8 pack into GPCs without stranding
// slots), the largest that keeps the grid within one wave of ~90% of the
// 2-per-SM CTA slots and at least 8 K blocks per split.
static int choose_splits(int N, int K, int num_sms, int ctas_per_sm = 2) {
  const int kb = (K + 63) / 64;
  const int tiles = (N + 127) / 128;
  const long budget = (long)(0.9 * ctas_per_sm * num_sms);
  int s = 1;
  while (s < 8 && (long)tiles * (s * 2) <= budget && (kb + 2 * s - 1) / (2 * s) >= 8) s *= 2;
  // the last split must own at least one K block
  while (s > 1 && (long)((kb + s - 1) / s) * (s - 1) >= kb) s /= 2;
  return s;
}

// Split count of the quantised GEMM (one CTA per SM): the largest S <= 8
// (any S: cluster sizes up to 8 are portable) that keeps the grid within one
// wave with at least 8 K blocks per split; a function of (N, K) only, so
// results do not depend on M.
static int choose_splits_q(int N, int K, int num_sms) {
  const int kb = K / 64;
  const int tiles = (N + 127) / 128;
  int best = 1;
  for (int s = 2; s <= 8; ++s) {
    if ((long)tiles * s > num_sms) break;
    if ((kb + s - 1) / s < 8) break;
    if ((long)((kb + s - 1) / s) * (s - 1) >= kb) continue;  // the last split must own a K block
    best = s;
  }
  return best;
}

}  // namespace b200

using namespace b200;

extern "C" {

// Diagnostics: when set, the next GEMM launches record 6 %globaltimer stamps per
// CTA (entry, prologue done, first stage landed, accumulator ready, partials
// published, exit) into this device buffer. Pass null to turn it off.
static unsigned long long* g_gemm_trace = nullptr;
void b200_gemm_set_trace(unsigned long long* buf) { g_gemm_trace = buf; }
// Diagnostics: per-K-block stamps of CTA (0,0,0) of the next launches:
// [4][nkb] = {raw/weights landed, operand ready (dequantised), MMA issued, activation landed}.
static unsigned long long* g_gemm_ktrace = nullptr;
void b200_gemm_set_ktrace(unsigned long long* buf) { g_gemm_ktrace = buf; }

// q|k|v projection with the qk-norm + RoPE + paged K/V append fused into the
// epilogue (kEpiQKRope): head dim 128, full non-interleaved rotary, N =
// (H + 2 KVH) * 128. Writes q_out [M, H, 128] and the K/V cache slots of the
// tokens; no projection output. Same K partition and reduction order as
// b200_gemm_bf16 for this (N, K). Returns 0, a CUDA error code, or -1.
int b200_gemm_qkv_rope(const void* X, int M, int K, int ldx, const void* W, int N, int ldw, const void* bias,
                       const int* positions, const int64_t* slots, const float* cos_sin, const void* qw,
                       const void* kw, float eps, void* q_out, void* k_cache, void* v_cache, int kv_fp8,
                       const float* k_scale, const float* v_scale, int H, int KVH, int64_t num_slots, int num_sms,
                       int force_splits, cudaStream_t stream) {
  if (M <= 0) return 0;
  if (N != (H + 2 * KVH) * 128 || !positions || !cos_sin || !q_out) return -1;
  if ((K % 8) || (ldx % 8) || (ldw % 8) || ((uintptr_t)X & 15) || ((uintptr_t)W & 15) || ((uintptr_t)q_out & 7))
    return -1;
  int BN = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  GemmArgs a = {};
  a.Y = nullptr;
  a.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  a.M = M;
  a.N = N;
  a.K = K;
  a.epi = kEpiQKRope;
  a.trace = g_gemm_trace;
  a.ktrace = g_gemm_ktrace;
  a.rk.positions = positions;
  a.rk.slots = slots;
  a.rk.cos_sin = cos_sin;
  a.rk.qw = reinterpret_cast<const __nv_bfloat16*>(qw);
  a.rk.kw = reinterpret_cast<const __nv_bfloat16*>(kw);
  a.rk.q_out = reinterpret_cast<__nv_bfloat16*>(q_out);
  a.rk.k_cache = k_cache;
  a.rk.v_cache = v_cache;
  a.rk.k_scale = k_scale;
  a.rk.v_scale = v_scale;
  a.rk.num_slots = k_cache ? num_slots : 0;
  a.rk.eps = eps;
  a.rk.H = H;
  a.rk.KVH = KVH;
  a.rk.kv_fp8 = kv_fp8;
  a.kb_total = (K + 63) / 64;
  const int s = force_splits > 0 ? force_splits : choose_splits(N, K, num_sms);
  if (s > 8) return -1;
  a.kb_per_split = (a.kb_total + s - 1) / s;
  a.ksplit = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  if (a.ksplit > 1 && BN == 256) BN = 128;  // as in b200_gemm_bf16
  CUtensorMap tw, tx;
  if (!make_tmap_2d(&tw, W, N, K, ldw, 128, 64, 2)) return -1;
  if (!make_tmap_2d(&tx, X, M, K, ldx, BN, 64, 2)) return -1;
  if (a.ksplit == 1 && BN == 256 && N > 128)  // prefill-sized, unsplit: 256 x 256 tiles
    return launch_gemm<256, 3, kModeLocal, 0, 2>(tw, tx, a, local_coll(), (N + 255) / 256, (M + 255) / 256, stream);
  const int tiles_n = N / 128, tiles_m = (M + BN - 1) / BN;
  return launch_bn<kModeLocal>(BN, tw, tx, a, local_coll(), tiles_n, tiles_m, stream);
}

int b200_gemm_num_splits(int M, int N, int K, int num_sms) {
  (void)M;
  return choose_splits(N, K, num_sms);
}

// Y[M, :] = epi(X[M, K] . W[N, K]^T + bias). X row stride ldx, W row stride ldw (elements).
// epi: 0 bf16 store, 1 SwiGLU (W rows interleaved gate/up per 64), 2 fp32 store, 3 bf16 add R,
// 4 GeGLU, 5 GPT-OSS SwiGLU. force_splits > 0 overrides the split count (tests / tuning).
// Returns 0 on success, a CUDA error code, or -1 for a bad layout.
int b200_gemm_bf16(const void* X, int M, int K, int ldx, const void* W, int N, int ldw, void* Y, int ldy,
                   const void* R, int ldr, const void* bias, int epi, int num_sms, int force_splits,
                   cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  if ((K % 8) || (ldx % 8) || (ldw % 8) || ((uintptr_t)X & 15) || ((uintptr_t)W & 15)) return -1;
  const bool glu = epi == kEpiSwiGLU || epi == kEpiGeGLU || epi == kEpiSwiGLUOAI;
  if (glu && (N % 128)) return -1;
  int BN = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  GemmArgs a;
  a.Y = Y;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldy = ldy;
  a.ldr = ldr;
  a.epi = epi;
  a.trace = g_gemm_trace;
  a.ktrace = g_gemm_ktrace;
  a.kb_total = (K + 63) / 64;
  const int s = force_splits > 0 ? force_splits : choose_splits(N, K, num_sms);
  if (s > 8) return -1;
  a.kb_per_split = (a.kb_total + s - 1) / s;
  a.ksplit = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  // split-K launches (decode rows) of more than 128 rows take 128-row tiles: twice
  // the CTAs and half the epilogue each; a row's K order is the same either way
  if (a.ksplit > 1 && BN == 256) BN = 128;
  CUtensorMap tw, tx;
  if (!make_tmap_2d(&tw, W, N, K, ldw, 128, 64, 2)) return -1;
  if (!make_tmap_2d(&tx, X, M, K, ldx, BN, 64, 2)) return -1;
  if (a.ksplit == 1 && BN == 256 && N > 128)  // prefill-sized, unsplit: 256 x 256 tiles
    return launch_gemm<256, 3, kModeLocal, 0, 2>(tw, tx, a, local_coll(), (N + 255) / 256, (M + 255) / 256, stream);
  const int tiles_n = (N + 127) / 128, tiles_m = (M + BN - 1) / BN;
  return launch_bn<kModeLocal>(BN, tw, tx, a, local_coll(), tiles_n, tiles_m, stream);
}

// Y[M, :] = epi(X[M, K] . dequant(W)^T + bias) with affine-quantised W
// (bits 4 or 8, group size 32 / 64 / 128) in the tile-major device layout:
// record (tile, K block) = {codes [128][bits*8 B] (4-bit words in the
// repacked nibble order), scales [gpb][128] bf16, biases [gpb][128] bf16},
// records contiguous per 128-row tile; gpb = 2 for group size 32, else 1 (a
// 128-input group repeats its scale and bias in both of its K blocks).
// Same epilogues and cluster split-K as b200_gemm_bf16; one CTA per SM.
int b200_gemm_q(const void* X, int M, int K, int ldx, const void* tiled, int N, int bits, int gs, void* Y, int ldy,
                const void* R, int ldr, const void* bias, int epi, int num_sms, int force_splits, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return 0;
  if ((bits != 4 && bits != 8 && bits != kWqE2M1) || (gs != 16 && gs != 32 && gs != 64 && gs != 128)) return -1;
  // e2m1 codes: MXFP4 (group 32) or NVFP4 (group 16); affine codes: groups 32 / 64 / 128
  if (bits == kWqE2M1 ? (gs != 16 && gs != 32) : (gs == 16)) return -1;
  if ((K % 64) || (gs == 128 && K % 128) || (ldx % 8) || ((uintptr_t)X & 15) || ((uintptr_t)tiled & 15) || (N % 8)) return -1;
  const bool glu = epi == kEpiSwiGLU || epi == kEpiGeGLU || epi == kEpiSwiGLUOAI;
  if (glu && (N % 128)) return -1;
  const int BN = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  QArgs q;
  q.tiled = reinterpret_cast<const uint8_t*>(tiled);
  q.gs = gs;
  q.gpb = gs == 16 ? 4 : gs == 32 ? 2 : 1;
  q.rec_bytes = bits == kWqE2M1 ? 4 * 128 * 8 + q.gpb * 256 : bits * 128 * 8 + q.gpb * 512;
  q.kb_total = K / 64;
  CUtensorMap tx;
  if (!make_tmap_2d(&tx, X, M, K, ldx, BN, 64, 2)) return -1;
  GemmArgs a = {};
  a.Y = Y;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  a.M = M;
  a.N = N;
  a.K = K;
  a.ldy = ldy;
  a.ldr = ldr;
  a.epi = epi;
  a.trace = g_gemm_trace;
  a.ktrace = g_gemm_ktrace;
  a.kb_total = K / 64;
  const int s = force_splits > 0 ? force_splits : choose_splits_q(N, K, num_sms);
  if (s > 8) return -1;
  a.kb_per_split = (a.kb_total + s - 1) / s;
  a.ksplit = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  const int tiles_n = (N + 127) / 128, tiles_m = (M + BN - 1) / BN;
  if (bits == kWqE2M1) return launch_bn_q<kWqE2M1>(BN, tx, a, q, tiles_n, tiles_m, stream);
  return bits == 4 ? launch_bn_q<4>(BN, tx, a, q, tiles_n, tiles_m, stream)
                   : launch_bn_q<8>(BN, tx, a, q, tiles_n, tiles_m, stream);
}

int b200_gemm_q_num_splits(int N, int K, int num_sms) { return choose_splits_q(N, K, num_sms); }

// ---------------------------------------------------------------------------
// Fused collective GEMMs (tensor parallelism). `comm_ctx` is a CommCtx blob
// (see b200_comm.cuh). Rows: M_pad = world * rows_per_rank, rank j owns rows
// [j*rpr, (j+1)*rpr); only the first M_real rows are meaningful.
// ---------------------------------------------------------------------------

// All-gather -> GEMM: X rows come from every rank's published rows of slot
// `parity`; waits (bounded) for phase `phase` on the AG pad. Y is local.
int b200_gemm_bf16_ag(const void* comm_ctx, int phase, int parity, int M_real, int K, const void* W, int N, int ldw,
                      void* Y, int ldy, const void* bias, int epi, int num_sms, int force_splits,
                      cudaStream_t stream) {
  CollArgs* coll = new CollArgs();  // heap: ~2 KB, copied into the launch
  std::unique_ptr<CollArgs> guard(coll);
  memcpy(&coll->comm, comm_ctx, sizeof(CommCtx));
  coll->phase = phase;
  coll->parity = parity;
  const CommCtx& c = coll->comm;
  const int M = c.world * c.rows_per_rank;
  if (M_real > M || (c.rows_per_rank % 8) || c.hidden != K) return -1;
  if (M != 16 && M != 32 && M != 64 && M != 128 && M != 256) return -1;
  if ((K % 8) || (ldw % 8)) return -1;
  const bool glu = epi == kEpiSwiGLU || epi == kEpiGeGLU || epi == kEpiSwiGLUOAI;
  if (glu && (N % 128)) return -1;
  CUtensorMap tw;
  if (!make_tmap_2d(&tw, W, N, K, ldw, 128, 64, 2)) return -1;
  for (int p = 0; p < 2; ++p) {
    const uint8_t* rows = c.base[c.rank] + c.h_off + (size_t)p * M * c.hidden * 2;
    if (!make_tmap_2d(&coll->peer_x[p], rows, M, K, K, M, 64, 2)) return -1;
  }
  GemmArgs a = {};
  a.Y = Y;
  a.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  a.M = M_real;
  a.N = N;
  a.K = K;
  a.ldy = ldy;
  a.epi = epi;
  a.trace = g_gemm_trace;
  a.ktrace = g_gemm_ktrace;
  a.kb_total = (K + 63) / 64;
  const int s = force_splits > 0 ? force_splits : choose_splits(N, K, num_sms);
  a.kb_per_split = (a.kb_total + s - 1) / s;
  a.ksplit = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  return launch_bn<kModeAG>(M, tw, tw, a, *coll, (N + 127) / 128, 1, stream);
}

// GEMM -> reduce-scatter: fp32 partial rows go to their owner rank's inbox
// slot `parity`; the last CTA publishes phase `phase` on the RS pad.
int b200_gemm_bf16_rs(const void* comm_ctx, int phase, int parity, const void* X, int M_real, int K, int ldx,
                      const void* W, int N, int ldw, const void* bias, int num_sms, int force_splits, int rs_all,
                      void* nvls_local, cudaStream_t stream) {
  CollArgs* coll = new CollArgs();
  std::unique_ptr<CollArgs> guard(coll);
  memcpy(&coll->comm, comm_ctx, sizeof(CommCtx));
  coll->phase = phase;
  coll->parity = parity;
  coll->rs_all = rs_all;
  if (rs_all >= 2 && (N % 4)) return -1;
  if (rs_all == 3 && (!nvls_local || (reinterpret_cast<uintptr_t>(nvls_local) % 16))) return -1;
  coll->nvls_local = reinterpret_cast<__nv_bfloat16*>(nvls_local);
  const CommCtx& c = coll->comm;
  const int M = c.world * c.rows_per_rank;
  if (M_real > M || c.hidden != N || (K % 8) || (ldx % 8) || (ldw % 8)) return -1;
  int BN = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  CUtensorMap tw, tx;
  if (!make_tmap_2d(&tw, W, N, K, ldw, 128, 64, 2)) return -1;
  if (!make_tmap_2d(&tx, X, M_real, K, ldx, BN, 64, 2)) return -1;
  GemmArgs a = {};
  a.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  a.M = M_real;
  a.N = N;
  a.K = K;
  a.epi = kEpiStoreF32;
  a.trace = g_gemm_trace;
  a.ktrace = g_gemm_ktrace;
  a.kb_total = (K + 63) / 64;
  const int s = force_splits > 0 ? force_splits : choose_splits(N, K, num_sms);
  a.kb_per_split = (a.kb_total + s - 1) / s;
  a.ksplit = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  return launch_bn<kModeRS>(BN, tw, tx, a, *coll, (N + 127) / 128, (M_real + BN - 1) / BN, stream);
}

}  // extern "C"

B200_STATUS_ACCESSORS(gemm)
