// Expert parallelism over symmetric memory: the MoE router top-k fused with
// the dispatch of each routed token row into the receive buffer of the rank
// that owns the expert (NVLink stores into peer memory), and the return of
// the expert outputs fused with the weighted combine. Ranks signal with epoch
// flags; no collective library on this path.
//
// Reference behaviour: the routed-expert MoE block (router top-k,
// MLXLMCommon/MoERouterTopK.swift:22; SwitchGLU gather -> expert matmuls ->
// weighted un-sort, MLXLMCommon/SwitchLayers.swift:478, :244, :149). The
// reference keeps every expert on every rank (its tensor-parallel models
// channel-split the experts); here experts are owned whole by ranks, E / world
// consecutive experts each.
//
// Symmetric buffer of every rank:
//   pads   [4][kMaxRanks] uint32   epoch flags; flag(pad, src) on the owner
//   rx     [world][cap][H] bf16    rows dispatched to this rank, by source
//   rmeta  [world][cap] int        local expert id of each received row
//   rcnt   [kMaxRanks] int         rows each source sent in this phase
//   ret    [world][cap][H] bf16    expert outputs returned to this rank, by owner
// One MoE layer (phase `ph` of the step):
//   source  ep_route_dispatch  router top-k per token; pair (t, j) -> owner
//                              e / E_local at a slot from a per-owner counter;
//                              row pushed to rx(owner, rank, slot)
//   owner   ep_prepare         wait for every source; local expert id of each
//                              of the world * cap slots, -1 when empty
//           moe sort / gather / grouped GEMMs over the slots (local memory)
//           ep_return          expert output of each filled slot pushed to
//                              ret(source, rank, slot)
//   source  ep_combine         wait for every owner; out[t] = sum_j w[t, j] *
//                              ret(owner_j, slot_j) in j order (fp32)
// Slots come from atomics, so the row order inside rx varies from run to run;
// every expert output row depends only on its own input row, and the combine
// sums in the fixed j order, so the result does not.
// Reuse of rx / ret needs no double buffering: a source dispatches layer l+1
// only after its combine of layer l saw every owner's return, which each
// owner issues after it has consumed its rows of layer l.
#include "b200_common.cuh"
#include "b200_comm.cuh"
#include "b200_moe.cuh"

namespace b200 {
namespace ep {

enum EpPad : int { kDispatch = 0, kReturn = 1 };

struct EpCtx {
  int rank, world;
  uint8_t* base[kMaxRanks];
  uint64_t pads_off, rx_off, rmeta_off, rcnt_off, ret_off;
  int cap, hidden, experts_local, num_experts;
  const int* step_ptr;
  int* ticket;  // [2] local grid tickets, self-resetting
  int* cnt;     // [kMaxRanks] local per-owner slot counters, self-resetting
  __device__ __forceinline__ uint32_t* pad(int owner, int p, int src) const {
    return reinterpret_cast<uint32_t*>(base[owner] + pads_off) + p * kMaxRanks + src;
  }
  __device__ __forceinline__ __nv_bfloat16* rx(int owner, int src, int slot) const {
    return reinterpret_cast<__nv_bfloat16*>(base[owner] + rx_off) + ((size_t)src * cap + slot) * hidden;
  }
  __device__ __forceinline__ int* rmeta(int owner, int src) const {
    return reinterpret_cast<int*>(base[owner] + rmeta_off) + (size_t)src * cap;
  }
  __device__ __forceinline__ int* rcnt(int owner) const { return reinterpret_cast<int*>(base[owner] + rcnt_off); }
  __device__ __forceinline__ __nv_bfloat16* ret(int owner, int from, int slot) const {
    return reinterpret_cast<__nv_bfloat16*>(base[owner] + ret_off) + ((size_t)from * cap + slot) * hidden;
  }
  __device__ __forceinline__ uint32_t epoch(int phase) const {
    return (uint32_t)(*step_ptr) * kPhasesPerStep + (uint32_t)phase + 1u;
  }
};

// H bf16 (H % 8 == 0) with 16-byte accesses by the threads [t0, t0 + nt)
__device__ __forceinline__ void copy_row(__nv_bfloat16* dst, const __nv_bfloat16* src, int H, int t, int nt) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int i = t; i < H / 8; i += nt) d[i] = s[i];
}

// The last CTA of a grid (thread 0, after its own writes, behind a CTA
// barrier) runs `last`, then publishes `epoch` to flag(pad, rank) of every
// rank. Ordering as in last_cta_signal (b200_comm.cuh): GPU-scope acq_rel
// ticket increments, system-scope release flag stores, no full fences.
template <typename F>
__device__ __forceinline__ void last_cta(const EpCtx& c, int* ticket, int pad, uint32_t epoch, F&& last) {
  const int t = (int)ticket_add_acq_rel(reinterpret_cast<uint32_t*>(ticket), 1u);
  if (t == (int)(gridDim.x * gridDim.y * gridDim.z) - 1) {
    *ticket = 0;
    last();
    for (int j = 0; j < c.world; ++j) signal_store(c.pad(j, pad, c.rank), epoch);
  }
}

// One CTA (128 threads) per token; grid max(T, 1). logits [T, E] fp32.
__global__ void __launch_bounds__(128) route_dispatch_kernel(EpCtx c, int phase, const float* __restrict__ logits,
                                                             int T, int k, int mode, int norm_topk,
                                                             const __nv_bfloat16* __restrict__ x,
                                                             int* __restrict__ ids_out, float* __restrict__ w_out,
                                                             int* __restrict__ slot_out) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int s_ids[16];
  __shared__ float s_w[16];
  __shared__ int s_slot[16];
  const int t = blockIdx.x;
  const int H = c.hidden, el = c.experts_local;
  if (t < T) {  // uniform over the block
    if (threadIdx.x < 32) route_topk_warp(logits + (size_t)t * c.num_experts, c.num_experts, k, mode, norm_topk,
                                          s_ids, s_w);
    __syncthreads();
    if (threadIdx.x < k) {
      const int j = threadIdx.x;
      const int e = s_ids[j];
      const int owner = e / el;
      int slot = -1;
      if (e >= 0 && owner < c.world) {
        slot = atomicAdd(&c.cnt[owner], 1);
        if (slot < c.cap) {
          c.rmeta(owner, c.rank)[slot] = e - owner * el;
        } else {
          set_status(kErrBounds);
          slot = -1;
        }
      } else {
        set_status(kErrBounds);
      }
      s_slot[j] = slot;
      ids_out[t * k + j] = e;
      w_out[t * k + j] = s_w[j];
      slot_out[t * k + j] = slot;
    }
    __syncthreads();
    const __nv_bfloat16* row = x + (size_t)t * H;
    // warp w pushes pairs w, w + 4, ...
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < k; j += 4) {
      const int sl = s_slot[j];
      if (sl >= 0) copy_row(c.rx(s_ids[j] / el, c.rank, sl), row, H, lane, 32);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    last_cta(c, &c.ticket[0], kDispatch, c.epoch(phase), [&] {
      for (int j = 0; j < c.world; ++j) c.rcnt(j)[c.rank] = min(atomicExch(&c.cnt[j], 0), c.cap);
    });
  }
}

// Owner: wait for every source, then the local expert id of each of the
// world * cap receive slots (-1 where a source sent fewer rows).
__global__ void __launch_bounds__(256) prepare_kernel(EpCtx c, int phase, int* __restrict__ ids_local) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    bool ok = true;
    const uint32_t ep = c.epoch(phase);
    for (int j = 0; j < c.world; ++j) ok &= wait_counter(c.pad(c.rank, kDispatch, j), ep);
    s_ok = ok;
  }
  __syncthreads();
  const int n_slots = c.world * c.cap;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_slots; i += gridDim.x * blockDim.x) {
    const int src = i / c.cap, slot = i - src * c.cap;
    const int cnt = c.rcnt(c.rank)[src];
    ids_local[i] = (s_ok && slot < cnt) ? c.rmeta(c.rank, src)[slot] : -1;
  }
}

// Owner: slot i (src = i / cap) has its expert output at sorted row pos[i] of
// ys; one warp per slot pushes it back to the source.
__global__ void __launch_bounds__(256) return_kernel(EpCtx c, int phase, const __nv_bfloat16* __restrict__ ys,
                                                     const int* __restrict__ pos,
                                                     const int* __restrict__ ids_local) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (blockDim.x >> 5);
  const int n_slots = c.world * c.cap;
  for (int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n_slots; i += nw) {
    if (ids_local[i] < 0) continue;
    const int p = pos[i];
    if (p < 0) continue;
    const int src = i / c.cap, slot = i - src * c.cap;
    copy_row(c.ret(src, c.rank, slot), ys + (size_t)p * c.hidden, c.hidden, lane, 32);
  }
  __syncthreads();
  if (threadIdx.x == 0) last_cta(c, &c.ticket[1], kReturn, c.epoch(phase), [] {});
}

// Source: wait for every owner, then out[t] = sum_j w[t, j] * y(t, j) in j
// order (fp32), bf16 out. One CTA per token; grid max(T, 1).
__global__ void __launch_bounds__(256) combine_kernel(EpCtx c, int phase, const int* __restrict__ ids,
                                                      const float* __restrict__ w, const int* __restrict__ slots,
                                                      int T, int k, __nv_bfloat16* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int s_ok;
  __shared__ const __nv_bfloat16* s_src[16];
  __shared__ float s_w[16];
  if (threadIdx.x == 0) {
    bool ok = true;
    const uint32_t ep = c.epoch(phase);
    for (int j = 0; j < c.world; ++j) ok &= wait_counter(c.pad(c.rank, kReturn, j), ep);
    s_ok = ok;
  }
  const int t = blockIdx.x;
  if (t < T && threadIdx.x < k) {
    const int j = threadIdx.x;
    const int sl = slots[t * k + j];
    s_src[j] = sl >= 0 ? c.ret(c.rank, ids[t * k + j] / c.experts_local, sl) : nullptr;
    s_w[j] = w[t * k + j];
  }
  __syncthreads();
  if (t >= T) return;
  const int H = c.hidden;
  for (int i = threadIdx.x; i < H / 2; i += blockDim.x) {
    float a0 = 0.f, a1 = 0.f;
    for (int j = 0; j < k; ++j) {
      const __nv_bfloat16* src = s_src[j];
      if (src == nullptr || !s_ok) continue;
      const __nv_bfloat162 y = reinterpret_cast<const __nv_bfloat162*>(src)[i];
      a0 += s_w[j] * __bfloat162float(y.x);
      a1 += s_w[j] * __bfloat162float(y.y);
    }
    reinterpret_cast<__nv_bfloat162*>(out + (size_t)t * H)[i] = __floats2bfloat162_rn(a0, a1);
  }
}

}  // namespace ep
}  // namespace b200

using namespace b200;

static bool load_ctx(ep::EpCtx* c, const void* ctx) {
  memcpy(c, ctx, sizeof(*c));
  return c->hidden % 8 == 0 && c->world >= 1 && c->world <= kMaxRanks && c->cap > 0 && c->experts_local > 0;
}

extern "C" {

int b200_ep_ctx_size() { return (int)sizeof(ep::EpCtx); }

// logits [T, E] fp32, x [T, H] bf16; ids/w/slots [T, k] outputs.
int b200_ep_route_dispatch(const void* ctx, int phase, const float* logits, int T, int k, int mode, int norm_topk,
                           const void* x, int* ids, float* w, int* slots, cudaStream_t st) {
  ep::EpCtx c;
  if (!load_ctx(&c, ctx) || k > 16 || c.num_experts > 256 || T < 0) return -1;
  cudaError_t e = launch_k(ep::route_dispatch_kernel, dim3(T > 0 ? T : 1), dim3(128), 0, st, 1, c, phase, logits, T,
                           k, mode, norm_topk, reinterpret_cast<const __nv_bfloat16*>(x), ids, w, slots);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_ep_prepare(const void* ctx, int phase, int* ids_local, cudaStream_t st) {
  ep::EpCtx c;
  if (!load_ctx(&c, ctx)) return -1;
  const int n = c.world * c.cap;
  const int grid = min((n + 255) / 256, 148);
  cudaError_t e = launch_k(ep::prepare_kernel, dim3(grid), dim3(256), 0, st, 1, c, phase, ids_local);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_ep_return(const void* ctx, int phase, const void* ys, const int* pos, const int* ids_local, int num_sms,
                   cudaStream_t st) {
  ep::EpCtx c;
  if (!load_ctx(&c, ctx)) return -1;
  const int n = c.world * c.cap;
  const int grid = max(1, min((n + 7) / 8, 2 * num_sms));
  cudaError_t e = launch_k(ep::return_kernel, dim3(grid), dim3(256), 0, st, 1, c, phase,
                           reinterpret_cast<const __nv_bfloat16*>(ys), pos, ids_local);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_ep_combine(const void* ctx, int phase, const int* ids, const float* w, const int* slots, int T, int k,
                    void* out, cudaStream_t st) {
  ep::EpCtx c;
  if (!load_ctx(&c, ctx) || k > 16 || T < 0) return -1;
  cudaError_t e = launch_k(ep::combine_kernel, dim3(T > 0 ? T : 1), dim3(256), 0, st, 1, c, phase, ids, w, slots, T,
                           k, reinterpret_cast<__nv_bfloat16*>(out));
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"

B200_STATUS_ACCESSORS(ep)
