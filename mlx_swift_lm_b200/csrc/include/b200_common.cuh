// Shared device helpers for the sm_100a kernel library.
//
// Everything here is written for Blackwell (sm_100a): mbarrier-driven TMA
// pipelines, tcgen05 MMA with TMEM accumulators, 32-lane warp reductions.
// Every spin-wait is bounded by %globaltimer: on expiry the waiting thread
// records an error code in the library status word and returns false, so a
// broken pipeline ends the kernel with an error status that the host reads
// instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <atomic>
#include <utility>

namespace b200 {

// ---------------------------------------------------------------------------
// Status word (one per loaded library, per device). Bit meanings:
//   1 = mbarrier wait timed out in a GEMM pipeline
//   2 = TMEM accumulator wait timed out
//   4 = peer-flag wait timed out in a fused collective
//   8 = bounds check failed (page table / slot index out of range)
//  16 = attention pipeline wait timed out
// ---------------------------------------------------------------------------
// Each translation unit owns one status word (no relocatable device code is
// needed); B200_STATUS_ACCESSORS(tag) exports a host reader for it.
static __device__ unsigned int g_status;

constexpr unsigned kErrGemmWait = 1u;
constexpr unsigned kErrTmemWait = 2u;
constexpr unsigned kErrPeerWait = 4u;
constexpr unsigned kErrBounds = 8u;
constexpr unsigned kErrAttnWait = 16u;

// Default bound for device-side waits: 2 seconds of wall time.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ void set_status(unsigned code) { atomicOr(&g_status, code); }

// CHECKED builds (-DB200_CHECKED=1, the libb200kernels_checked.so variant)
// add bounds checks that the release build leaves out of the hot loops; a
// failed check records kErrBounds in the unit's status word and the access
// is redirected to a safe index instead of trapping.
#ifndef B200_CHECKED
#define B200_CHECKED 0
#endif

// Page id of entry `idx` of a row's page table: a page id outside the slab
// (always) or an entry past the row's `ld_pt` entries (CHECKED builds)
// records kErrBounds and reads page 0.
__device__ __forceinline__ int64_t checked_page(const int* row_table, int idx, int ld_pt, int64_t num_pages) {
  if (B200_CHECKED && (idx < 0 || idx >= ld_pt)) {
    set_status(kErrBounds);
    return 0;
  }
  int64_t page = row_table[idx];
  if (page < 0 || page >= num_pages) {
    set_status(kErrBounds);
    page = 0;
  }
  return page;
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024). `red` needs 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? red[lane] : 0.f;
  r = warp_sum(r);
  return r;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? red[lane] : -INFINITY;
  r = warp_max(r);
  return r;
}

// ---------------------------------------------------------------------------
// Shared-memory address helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier (shared::cta) with bounded waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete. Returns false (and
// records `err`) if it does not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      set_status(err);
      return false;
    }
  }
}

// Contiguous global -> shared copy by the bulk-copy engine, completing on an
// mbarrier (transaction bytes). Addresses and size must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// TMA tiled loads into this CTA's shared memory. Coordinates are element
// indices, innermost first.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1,
                                            uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(bar), "l"(cache_hint)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1, int c2,
                                            uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(bar), "l"(cache_hint)
      : "memory");
}
// L2 cache policies (createpolicy results are opaque 64-bit values).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core) helpers, cta_group::1
// ---------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to shared memory at `dst_smem`. Must be executed by a whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/f16 inputs, f32 accum).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T (A operand read from TMEM).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Load 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Load 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Store 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Store 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 64 bf16, 8-row / 1024-byte swizzle atoms; the tile
// base must be 1024-byte aligned). `sbo_bytes` is the distance between
// consecutive 8-row groups (1024 for a dense tile).
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t saddr, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);          // start address
  d |= (uint64_t)(1u) << 16;                         // LBO (unused for swizzled K-major)
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32; // SBO
  d |= (uint64_t)1 << 46;                            // descriptor version (Blackwell)
  d |= (uint64_t)2 << 61;                            // SWIZZLE_128B
  return d;
}
// MN-major operand with 128-byte swizzle: atoms of 64 MN-elements x 8 K-rows
// (1024 bytes). `lbo_bytes` = distance between consecutive 64-element MN
// chunks, `sbo_bytes` = distance between consecutive 8-row K groups.
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B, f32 accumulate.
// a_mn / b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, int a_mn = 0, int b_mn = 0) {
  return (1u << 4)                       // D format f32
         | (1u << 7)                     // A format bf16
         | (1u << 10)                    // B format bf16
         | ((uint32_t)a_mn << 15)        // A major
         | ((uint32_t)b_mn << 16)        // B major
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

// kind::f16 with both operands f16 (A and B must share the type).
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Byte offset of element (row, col) inside a 128B-swizzled K-major tile of
// 64-element (128-byte) rows: 16-byte chunk index XOR (row % 8).
__device__ __forceinline__ uint32_t sw128_offset(int row, int col_bytes) {
  const int chunk = (col_bytes >> 4) ^ (row & 7);
  return (uint32_t)(row * 128 + (chunk << 4) + (col_bytes & 15));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// Gated activations of an interleaved gate/up projection (codes shared with
// the GEMM epilogues): silu(g) * u, gelu-tanh(g) * u, and GPT-OSS's clamped
// (u + 1) * g * sigmoid(1.702 g).
enum GluKind : int { kGluSwi = 1, kGluGe = 4, kGluOAI = 5 };
__device__ __forceinline__ float glu_act(int kind, float g, float u) {
  if (kind == kGluGe) {
    const float c = 0.7978845608028654f;  // sqrt(2/pi)
    return 0.5f * g * (1.f + tanhf(c * (g + 0.044715f * g * g * g))) * u;
  }
  if (kind == kGluOAI) {
    g = fminf(g, 7.f);
    u = fminf(fmaxf(u, -7.f), 7.f);
    return (u + 1.f) * g / (1.f + __expf(-1.702f * g));
  }
  return silu(g) * u;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL). Kernels are launched with programmatic
// stream serialization, so the next kernel may start while this one runs.
// Contract for every kernel of this library:
//   * pdl_launch_dependents() at entry: lets the next kernel's CTAs be
//     scheduled once all CTAs of this grid have started;
//   * pdl_wait() before the first access to memory that an earlier kernel
//     writes, or that a later kernel may still read (WAR). Work on data no
//     kernel writes (weights, page tables set before the step) may precede it.
// pdl_wait() returns once all prerequisite grids have completed and their
// writes are visible; it is a no-op for launches without the attribute.
// ---------------------------------------------------------------------------
// Device timeline (diagnostics, off unless a buffer is installed through
// b200_timeline_<unit>): block (0,0,0) of every kernel records, right after
// its pdl_wait() returns, {globaltimer, launch signature} into a buffer shared
// by all units (one device counter hands out the entries). In a chain of
// dependent launches pdl_wait() returns when the previous grid has completed,
// so consecutive marks bracket each kernel's cost in the chain.
// Signature: grid x (20 bits) | y (12) | z (8) | block x (11) | 1 in bit 63.
static __device__ unsigned long long* g_tl_buf;  // [cap][2]
static __device__ unsigned int* g_tl_head;
static __device__ unsigned int g_tl_cap;

__device__ __forceinline__ void timeline_mark() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  const unsigned i = atomicAdd(g_tl_head, 1u);
  if (i < g_tl_cap) {
    const unsigned long long sig = (1ull << 63) | ((unsigned long long)(gridDim.x & 0xFFFFF) << 31) |
                                   ((unsigned long long)(gridDim.y & 0xFFF) << 19) |
                                   ((unsigned long long)(gridDim.z & 0xFF) << 11) | (blockDim.x & 0x7FF);
    g_tl_buf[2 * i] = t;
    g_tl_buf[2 * i + 1] = sig;
  }
}

// A tagged mark from the calling thread (bit 62 set, `tag` in the low bits):
// points inside a kernel (a wait returning, a signal going out).
__device__ __forceinline__ void timeline_tag(unsigned tag) {
  if (g_tl_buf == nullptr) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  const unsigned i = atomicAdd(g_tl_head, 1u);
  if (i < g_tl_cap) {
    g_tl_buf[2 * i] = t;
    g_tl_buf[2 * i + 1] = (1ull << 63) | (1ull << 62) | tag;
  }
}

__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0 && (blockIdx.x | blockIdx.y | blockIdx.z) == 0 && g_tl_buf != nullptr) timeline_mark();
}
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

}  // namespace b200

// Host: launch `kernel` with programmatic stream serialization (PDL) unless
// disabled by b200_set_pdl(0). Optional cluster dimension along z.
namespace b200 {
bool pdl_enabled();
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                   int cluster_z, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = cluster_z;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Host: raise `Kernel`'s dynamic shared-memory limit to `bytes` on the current
// device. cudaFuncSetAttribute acts on the calling device's context only, so
// the record of what was set is kept per device (up to 64 devices), in atomics:
// host threads may launch concurrently, and two of them setting the same
// attribute at once is harmless. Returns 0 or the CUDA error code.
constexpr int kMaxDevices = 64;
template <auto Kernel>
static inline int smem_attr_once(int bytes) {
  static std::atomic<int> set_bytes[kMaxDevices];  // zero-initialised (static storage)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
  if (set_bytes[dev].load(std::memory_order_acquire) >= bytes) return 0;
  e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return (int)e;
  int cur = set_bytes[dev].load(std::memory_order_relaxed);
  while (cur < bytes && !set_bytes[dev].compare_exchange_weak(cur, bytes, std::memory_order_acq_rel)) {
  }
  return 0;
}
}  // namespace b200

// Host accessor for this translation unit's status word: copies it out and
// clears it. Returns the CUDA error code of the copy.
#define B200_STATUS_ACCESSORS(tag)                                                              \
  extern "C" int b200_timeline_##tag(unsigned long long* buf, unsigned int* head, unsigned int cap) { \
    cudaError_t e = cudaMemcpyToSymbol(b200::g_tl_buf, &buf, sizeof(buf));                        \
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(b200::g_tl_head, &head, sizeof(head));             \
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(b200::g_tl_cap, &cap, sizeof(cap));                \
    return (int)e;                                                                              \
  }                                                                                             \
  extern "C" int b200_status_##tag(unsigned int* out, int clear) {                               \
    cudaError_t e = cudaMemcpyFromSymbol(out, b200::g_status, sizeof(unsigned int));              \
    if (e == cudaSuccess && clear) {                                                            \
      unsigned int z = 0;                                                                       \
      e = cudaMemcpyToSymbol(b200::g_status, &z, sizeof(unsigned int));                         \
    }                                                                                           \
    return (int)e;                                                                              \
  }
