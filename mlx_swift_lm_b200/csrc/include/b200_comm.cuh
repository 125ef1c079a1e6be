// Device-side view of the symmetric-memory communicator used by the fused
// collective kernels (tensor parallelism over NVLink / NVSwitch).
//
// Every rank's symmetric buffer has the same layout:
//   [pads]   kNumPads x kMaxRanks uint32 flags; flag(pad, src) on the owner's
//            buffer is written by rank `src` with release semantics
//   [recv]   2 x world x rows_per_rank x hidden fp32 - reduce-scatter inboxes
//   [h]      2 x (world * rows_per_rank) x hidden bf16 - the gathered
//            normalised rows feeding the next column-parallel GEMM; every
//            rank pushes its own rows into every rank's copy (NVLink stores),
//            so the GEMM's TMA reads local memory only
//   [xarg]   2 x world x rows x {float value, int index} - split-argmax inbox
// Parity (2 slots) alternates by phase so a writer can never overwrite data
// its reader has not consumed: a rank reaches phase p+2 only after every peer
// has signalled phase p+1, which it does only after reading phase p.
//
// Flags carry an epoch: epoch = step * kPhasesPerStep + phase, where `step`
// comes from device memory (so CUDA-graph replays advance it) and `phase` is
// the call site's index within the step. A reader waits until the flag
// reaches the epoch (wrap-safe compare), bounded by %globaltimer.
#pragma once

#include "b200_common.cuh"

namespace b200 {

constexpr int kMaxRanks = 8;
constexpr int kNumPads = 8;
constexpr uint32_t kPhasesPerStep = 1024;

enum CommPad : int { kPadRS = 0, kPadAG = 1, kPadArg = 2, kPadTest = 7 };

struct CommCtx {
  int rank, world;
  uint8_t* base[kMaxRanks];  // symmetric buffer of each rank (peer-mapped), [rank] = local
  uint64_t pads_off, recv_off, h_off, xarg_off;
  int rows_per_rank;     // rows each rank owns (multiple of 8)
  int hidden;            // row width of recv / h
  int max_rows;          // rows capacity of the xarg inbox
  const int* step_ptr;   // device int: current step number
  uint32_t* expect_local;  // local scratch [kNumPads][kMaxRanks] (used by the self-test)
  int* ticket;           // local device counter for last-CTA signalling (self-resetting)

  __device__ __forceinline__ uint32_t* pad_ptr(int owner, int pad, int src) const {
    return reinterpret_cast<uint32_t*>(base[owner] + pads_off) + pad * kMaxRanks + src;
  }
  __device__ __forceinline__ uint32_t expect(int pad, int src) const { return expect_local[pad * kMaxRanks + src]; }
  __device__ __forceinline__ void bump(int pad, int src, uint32_t n) const {
    expect_local[pad * kMaxRanks + src] += n;
  }
  __device__ __forceinline__ uint32_t epoch(int phase) const {
    return (uint32_t)(*step_ptr) * kPhasesPerStep + (uint32_t)phase + 1u;
  }
  // fp32 inbox row `lrow` written by `src`, in the buffer of `owner`
  __device__ __forceinline__ float* recv_row(int owner, int parity, int src, int lrow) const {
    float* r = reinterpret_cast<float*>(base[owner] + recv_off);
    return r + (((size_t)parity * world + src) * rows_per_rank + lrow) * hidden;
  }
  // fp32 partial of row `row` (0 .. world*rpr-1) from `src`, in the buffer of
  // `owner` (every rank receives every rank's partials of every row)
  __device__ __forceinline__ float* recv_all(int owner, int parity, int src, int row) const {
    float* r = reinterpret_cast<float*>(base[owner] + recv_off);
    const size_t M = (size_t)world * rows_per_rank;
    return r + (((size_t)parity * world + src) * M + row) * hidden;
  }
  // bf16 partials in the same region (half the bytes; used from 4 ranks up)
  __device__ __forceinline__ __nv_bfloat16* recv_all_bf16(int owner, int parity, int src, int row) const {
    __nv_bfloat16* r = reinterpret_cast<__nv_bfloat16*>(base[owner] + recv_off);
    const size_t M = (size_t)world * rows_per_rank;
    return r + (((size_t)parity * world + src) * M + row) * hidden;
  }
  // normalised row `grow` (global row index 0..world*rpr-1) in the gathered
  // buffer [2][world*rpr][hidden] of `owner`; every rank pushes its rows into
  // every rank's buffer, so the all-gather GEMM reads local memory only
  __device__ __forceinline__ __nv_bfloat16* h_row(int owner, int parity, int grow) const {
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(base[owner] + h_off);
    return h + ((size_t)parity * world * rows_per_rank + grow) * hidden;
  }
  __device__ __forceinline__ float2* xarg(int owner, int parity, int src) const {
    float2* x = reinterpret_cast<float2*>(base[owner] + xarg_off);
    return x + ((size_t)parity * world + src) * max_rows;
  }
};

__device__ __forceinline__ void signal_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void signal_store(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Wait until *p reaches `target` (wrap-safe). Bounded: false + kErrPeerWait on timeout.
__device__ __forceinline__ bool wait_counter(const uint32_t* p, uint32_t target) {
  if ((int32_t)(load_acquire(p) - target) >= 0) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if ((int32_t)(load_acquire(p) - target) >= 0) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      set_status(kErrPeerWait);
      return false;
    }
  }
}

__device__ __forceinline__ uint32_t ticket_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Called by thread 0 of every CTA of a kernel after the CTA's peer writes
// (behind a CTA barrier): the last CTA to arrive publishes `epoch` into
// flag(pad, rank) of every peer. Ordering without full fences: each CTA's
// ticket increment is a GPU-scope release (the CTA's writes, local and
// remote, precede it), the last CTA's increment also acquires every earlier
// release, and its flag stores are system-scope releases; a reader that
// acquires the flag (system scope) therefore sees every CTA's writes through
// the chain of release / acquire pairs. (Sequentially consistent system
// fences here cost ~10-20 us per signal on B200.)
__device__ __forceinline__ void last_cta_signal(const CommCtx& c, int pad, uint32_t epoch) {
  const int total = gridDim.x * gridDim.y * gridDim.z;
  const int t = (int)ticket_add_acq_rel(reinterpret_cast<uint32_t*>(c.ticket), 1u);
  if (t == total - 1) {
    *c.ticket = 0;  // self-reset for the next launch / graph replay (ordered before the flags)
    for (int j = 0; j < c.world; ++j) signal_store(c.pad_ptr(j, pad, c.rank), epoch);
    timeline_tag(0x100 + pad);  // diagnostics: the phase's signal went out
  }
}

// Wait for flag(pad, src) >= epoch for every src (thread 0), then block barrier.
__device__ __forceinline__ bool wait_all_ranks(const CommCtx& c, int pad, uint32_t epoch) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int j = 0; j < c.world; ++j) ok &= wait_counter(c.pad_ptr(c.rank, pad, j), epoch);
    s_ok = ok;
    if (blockIdx.x == 0) timeline_tag(0x200 + pad);  // diagnostics: every rank's signal arrived
  }
  __syncthreads();
  return s_ok != 0;
}

}  // namespace b200
