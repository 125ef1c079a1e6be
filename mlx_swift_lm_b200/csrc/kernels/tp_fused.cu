// Companion kernels of the fused tensor-parallel decode path (symmetric memory).
//
// Rows are sequence-parallel between GEMMs: rank r owns rows [r*rpr, (r+1)*rpr)
// of the residual stream. Per layer:
//   gemm AG (qkv)  -> attention -> gemm RS (o_proj) -> tp_combine_norm
//   gemm AG (gate_up) -> gemm RS (down) -> tp_combine_norm
// tp_combine_norm sums the world fp32 partial rows of its inbox in rank order
// (deterministic), rounds the sum to bf16 (the unsharded model's o_proj/down
// output), adds it to the residual rows, applies RMSNorm, pushes the
// normalised rows into every rank's gathered buffer, then signals every rank.
// These replace the reference's injected allSum / reduceScatter / allGather
// closures (Gemma4TensorParallel.swift:196-236, GLM5NextTextModel.swift:455-498)
// with one-pass kernels over peer memory.
#include "b200_common.cuh"
#include "b200_comm.cuh"

namespace b200 {

// One CTA per local row. x_local [rpr, H] residual rows of this rank.
__global__ void __launch_bounds__(256) tp_combine_norm_kernel(CommCtx c, int phase_rs, int parity_rs, int phase_ag,
                                                             int parity_ag, __nv_bfloat16* x_local,
                                                             const __nv_bfloat16* w, float eps, int has_delta) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  const int lrow = blockIdx.x;
  const int H = c.hidden;
  if (has_delta) wait_all_ranks(c, kPadRS, c.epoch(phase_rs));
  __nv_bfloat16* xr = x_local + (size_t)lrow * H;
  extern __shared__ float rbuf[];
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    float r[4];
    uint2 xv = *reinterpret_cast<const uint2*>(xr + i);
    __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
    if (has_delta) {
      float4 acc = *reinterpret_cast<const float4*>(c.recv_row(c.rank, parity_rs, 0, lrow) + i);
      for (int j = 1; j < c.world; ++j) {
        const float4 p = *reinterpret_cast<const float4*>(c.recv_row(c.rank, parity_rs, j, lrow) + i);
        acc.x += p.x;
        acc.y += p.y;
        acc.z += p.z;
        acc.w += p.w;
      }
      const float d[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        xe[e] = f2bf(bf2f(xe[e]) + bf2f(f2bf(d[e])));
        r[e] = bf2f(xe[e]);
      }
      *reinterpret_cast<uint2*>(xr + i) = xv;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) r[e] = bf2f(xe[e]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      rbuf[i + e] = r[e];
      ss += r[e] * r[e];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
  // push the normalised row into every rank's gathered buffer (own rank first)
  const int grow = c.rank * c.rows_per_rank + lrow;
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    __nv_bfloat16 o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = f2bf(rbuf[i + e] * inv * bf2f(w[i + e]));
    const uint2 v = *reinterpret_cast<const uint2*>(o);
    for (int jj = 0; jj < c.world; ++jj) {
      const int j = (c.rank + jj) % c.world;
      *reinterpret_cast<uint2*>(c.h_row(j, parity_ag, grow) + i) = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) last_cta_signal(c, kPadAG, c.epoch(phase_ag));
}

// Every rank reduces every row (the RS GEMMs sent each rank all partials):
// one CTA per row m < M. With `has_delta`: wait for every rank's partials,
// sum them in rank order (the same order on every rank, so all ranks hold
// identical rows), round to bf16 and add to the replicated residual x[m];
// then h[m] = RMSNorm(x[m]) * w. No rows are pushed and nothing is signalled:
// the next GEMM reads h from local memory.
__global__ void __launch_bounds__(1024) tp_combine_all_kernel(CommCtx c, int phase_rs, int parity_rs,
                                                            __nv_bfloat16* x, const __nv_bfloat16* w, float eps,
                                                            __nv_bfloat16* h, int has_delta, int bf16_parts,
                                                            const __nv_bfloat16* nvls_mc) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  extern __shared__ float rbuf[];
  const int m = blockIdx.x;
  const int H = c.hidden;
  if (has_delta) {
    wait_all_ranks(c, kPadRS, c.epoch(phase_rs));
    // the partials were stored through unicast addresses; read them through the multicast alias
    if (nvls_mc) asm volatile("fence.proxy.alias;" ::: "memory");
  }
  __nv_bfloat16* xr = x + (size_t)m * H;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    uint2 xv = *reinterpret_cast<const uint2*>(xr + i);
    __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
    float r[4];
    if (has_delta && nvls_mc) {
      // the NVSwitch returns the sum over ranks of the bf16 partials (fp32 accumulation)
      const __nv_bfloat16* src = nvls_mc + ((size_t)parity_rs * c.world * c.rows_per_rank + m) * H + i;
      uint32_t u0, u1;
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v2.bf16x2 {%0, %1}, [%2];"
                   : "=r"(u0), "=r"(u1)
                   : "l"(src)
                   : "memory");
      const uint32_t uu[2] = {u0, u1};
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(uu);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        xe[e] = f2bf(bf2f(xe[e]) + bf2f(b[e]));
        r[e] = bf2f(xe[e]);
      }
      *reinterpret_cast<uint2*>(xr + i) = xv;
    } else if (has_delta) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < c.world; ++j) {  // rank order
        if (bf16_parts) {
          const uint2 u = *reinterpret_cast<const uint2*>(c.recv_all_bf16(c.rank, parity_rs, j, m) + i);
          const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
          for (int e = 0; e < 4; ++e) d[e] += bf2f(b[e]);
        } else {
          const float4 p = *reinterpret_cast<const float4*>(c.recv_all(c.rank, parity_rs, j, m) + i);
          d[0] += p.x;
          d[1] += p.y;
          d[2] += p.z;
          d[3] += p.w;
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        xe[e] = f2bf(bf2f(xe[e]) + bf2f(f2bf(d[e])));
        r[e] = bf2f(xe[e]);
      }
      *reinterpret_cast<uint2*>(xr + i) = xv;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) r[e] = bf2f(xe[e]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      rbuf[i + e] = r[e];
      ss += r[e] * r[e];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
  __nv_bfloat16* hr = h + (size_t)m * H;
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    __nv_bfloat16 o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = f2bf(rbuf[i + e] * inv * bf2f(w[i + e]));
    *reinterpret_cast<uint2*>(hr + i) = *reinterpret_cast<const uint2*>(o);
  }
}

// Embedding of this rank's rows into x_local (ids [T] of the whole step; rows
// past T are zero), without publishing.
__global__ void __launch_bounds__(256) tp_embed_kernel(CommCtx c, const int* ids, int T, const __nv_bfloat16* table,
                                                      int64_t vocab, __nv_bfloat16* x_local, float scale) {
  pdl_launch_dependents();
  pdl_wait();
  const int lrow = blockIdx.x;
  const int row = c.rank * c.rows_per_rank + lrow;
  const int H = c.hidden;
  __nv_bfloat16* dst = x_local + (size_t)lrow * H;
  if (row >= T) {
    for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = f2bf(0.f);
    return;
  }
  int64_t id = ids[row];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_status(kErrBounds);
    id = 0;
  }
  const __nv_bfloat16* src = table + id * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = scale == 1.f ? src[i] : f2bf(bf2f(src[i]) * scale);
}

// Split argmax: each rank reduces its vocabulary slice per row and writes
// (value, global index) into every rank's inbox; then every rank picks the
// winner (ties -> lowest index), so all ranks agree on the token.
__global__ void __launch_bounds__(1024) tp_argmax_exchange_kernel(CommCtx c, int phase, int parity,
                                                                  const float* logits, int64_t ld, int V_local,
                                                                  int vocab_offset) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int row = blockIdx.x;
  const float* lg = logits + (size_t)row * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V_local; i += blockDim.x)
    if (lg[i] > bv) {
      bv = lg[i];
      bi = i;
    }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sv[wid] = bv;
    si[wid] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w2 = 1; w2 < (int)(blockDim.x >> 5); ++w2)
      if (sv[w2] > bv || (sv[w2] == bv && si[w2] < bi)) {
        bv = sv[w2];
        bi = si[w2];
      }
    const float gidx = __int_as_float(bi == 0x7fffffff ? 0x7fffffff : bi + vocab_offset);
    for (int j = 0; j < c.world; ++j) c.xarg(j, parity, c.rank)[row] = make_float2(bv, gidx);
    last_cta_signal(c, kPadArg, c.epoch(phase));
  }
}

__global__ void tp_argmax_select_kernel(CommCtx c, int phase, int parity, int T, int* out, int* out2) {
  pdl_launch_dependents();
  pdl_wait();
  wait_all_ranks(c, kPadArg, c.epoch(phase));
  for (int row = threadIdx.x; row < T; row += blockDim.x) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = 0; j < c.world; ++j) {
      const float2 e = c.xarg(c.rank, parity, j)[row];
      const int ei = __float_as_int(e.y);
      if (e.x > bv || (e.x == bv && ei < bi)) {
        bv = e.x;
        bi = ei;
      }
    }
    const int tok = bi == 0x7fffffff ? 0 : bi;
    out[row] = tok;
    if (out2) out2[row] = tok;
  }
}

}  // namespace b200

using namespace b200;

extern "C" {

int b200_tp_combine_norm(const void* ctx, int phase_rs, int parity_rs, int phase_ag, int parity_ag, void* x_local,
                         const void* w, float eps, int has_delta, cudaStream_t st) {
  CommCtx c;
  memcpy(&c, ctx, sizeof(c));
  if (c.hidden % 4) return -1;
  cudaError_t e = launch_k(tp_combine_norm_kernel, dim3(c.rows_per_rank), dim3(256), c.hidden * sizeof(float), st, 1,
                           c, phase_rs, parity_rs, phase_ag, parity_ag, reinterpret_cast<__nv_bfloat16*>(x_local),
                           reinterpret_cast<const __nv_bfloat16*>(w), eps, has_delta);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_tp_combine_all(const void* ctx, int phase_rs, int parity_rs, void* x, const void* w, float eps, void* h,
                        int M, int has_delta, int bf16_parts, const void* nvls_mc, cudaStream_t st) {
  CommCtx c;
  memcpy(&c, ctx, sizeof(c));
  if ((c.hidden % 4) || M > c.world * c.rows_per_rank || M <= 0) return -1;
  // one pass per row: a thread per 4 elements (up to 1024 threads), so every load of the row is in flight at once
  const int threads = min(1024, ((c.hidden / 4 + 31) / 32) * 32);
  cudaError_t e = launch_k(tp_combine_all_kernel, dim3(M), dim3(threads), c.hidden * sizeof(float), st, 1, c, phase_rs,
                           parity_rs, reinterpret_cast<__nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(w),
                           eps, reinterpret_cast<__nv_bfloat16*>(h), has_delta, bf16_parts,
                           reinterpret_cast<const __nv_bfloat16*>(nvls_mc));
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_tp_embed(const void* ctx, const int* ids, int T, const void* table, int64_t vocab, void* x_local,
                  float scale, cudaStream_t st) {
  CommCtx c;
  memcpy(&c, ctx, sizeof(c));
  cudaError_t e = launch_k(tp_embed_kernel, dim3(c.rows_per_rank), dim3(256), 0, st, 1, c, ids, T,
                           reinterpret_cast<const __nv_bfloat16*>(table), vocab,
                           reinterpret_cast<__nv_bfloat16*>(x_local), scale);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_tp_argmax(const void* ctx, int phase, int parity, const float* logits, int64_t ld, int T, int V_local,
                   int vocab_offset, int* out, int* out2, cudaStream_t st) {
  CommCtx c;
  memcpy(&c, ctx, sizeof(c));
  if (T > c.max_rows) return -1;
  cudaError_t e = launch_k(tp_argmax_exchange_kernel, dim3(T), dim3(1024), 0, st, 1, c, phase, parity, logits, ld,
                           V_local, vocab_offset);
  if (e != cudaSuccess) return (int)e;
  e = launch_k(tp_argmax_select_kernel, dim3(1), dim3(256), 0, st, 1, c, phase, parity, T, out, out2);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"

B200_STATUS_ACCESSORS(tp_fused)
