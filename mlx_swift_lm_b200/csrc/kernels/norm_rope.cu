// Normalisation, RoPE and KV-append kernels.
//
//  * add_rmsnorm: residual add (rounded to the residual dtype) followed by
//    RMSNorm in one pass, the fusion of Libraries/MLXLMCommon/ResidualRMSNorm.swift:89.
//  * qk_norm_rope_kv_write: per-head RMSNorm of q and k (Qwen3 qk-norm,
//    MLXLLM/Models/Qwen3.swift:44-67), rotary embedding from a precomputed
//    cos/sin table (any RoPE variant of MLXLMCommon/RoPEUtils.swift reduces to
//    such a table), then the K/V append into the paged cache slot, the role of
//    paged_kv_write in ContinuousBatchingV2/Paged/pagedattention.metal:594-627.
//    KV pages may be bf16 or fp8 e4m3 with a per-KV-head scale.
//  * embedding gather.
#include "b200_common.cuh"

namespace b200 {

// One CTA per row. x is the residual stream (updated in place when delta is
// given), out receives RMSNorm(x) * w.
__global__ void add_rmsnorm_kernel(__nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ delta,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int H,
                                   int ldx, int ldd, int ldo, float eps, int w_offset_one) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  extern __shared__ float rbuf[];  // H floats
  __shared__ float red[32];
  const int row = blockIdx.x;
  __nv_bfloat16* xr = x + (size_t)row * ldx;
  const __nv_bfloat16* dr = delta ? delta + (size_t)row * ldd : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    uint4 xv = *reinterpret_cast<const uint4*>(xr + i);
    __nv_bfloat16* xe = reinterpret_cast<__nv_bfloat16*>(&xv);
    float r[8];
    if (dr) {
      uint4 dv = *reinterpret_cast<const uint4*>(dr + i);
      const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        __nv_bfloat16 s = f2bf(bf2f(xe[j]) + bf2f(de[j]));
        xe[j] = s;
        r[j] = bf2f(s);
      }
      *reinterpret_cast<uint4*>(xr + i) = xv;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = bf2f(xe[j]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      rbuf[i + j] = r[j];
      ss += r[j] * r[j];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
  __nv_bfloat16* orow = out + (size_t)row * ldo;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    uint4 wv = *reinterpret_cast<const uint4*>(w + i);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
    uint4 ov;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float ww = bf2f(we[j]) + (w_offset_one ? 1.f : 0.f);
      oe[j] = f2bf(rbuf[i + j] * inv * ww);
    }
    *reinterpret_cast<uint4*>(orow + i) = ov;
  }
}

// LayerNorm with bias over x + delta (BERT-family post-norm residual): one CTA
// per row; x <- bf16(x + delta) when delta is given, out = LN(x) * w + b
// (out may alias x).
__global__ void add_layernorm_kernel(__nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ delta,
                                     const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ b,
                                     __nv_bfloat16* out, int H, int ldx, int ldd, int ldo, float eps) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  extern __shared__ float rbuf[];  // H floats
  __shared__ float red[32];
  const int row = blockIdx.x;
  __nv_bfloat16* xr = x + (size_t)row * ldx;
  const __nv_bfloat16* dr = delta ? delta + (size_t)row * ldd : nullptr;
  float sum = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = bf2f(xr[i]);
    if (dr) {
      const __nv_bfloat16 s = f2bf(v + bf2f(dr[i]));
      xr[i] = s;
      v = bf2f(s);
    }
    rbuf[i] = v;
    sum += v;
  }
  const float mean = block_sum(sum, red) / (float)H;
  float var = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float d = rbuf[i] - mean;
    var += d * d;
  }
  __syncthreads();  // red[] is reused by the second reduction
  const float inv = rsqrtf(block_sum(var, red) / (float)H + eps);
  __nv_bfloat16* orow = out + (size_t)row * ldo;
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    orow[i] = f2bf((rbuf[i] - mean) * inv * bf2f(w[i]) + (b ? bf2f(b[i]) : 0.f));
}

// One CTA per token; one warp per head. Heads [0, H) are query heads,
// [H, H+KVH) key heads, [H+KVH, H+2KVH) value heads of the fused qkv row.
// cos_sin: [max_pos, rot_dim] fp32, first rot_dim/2 entries cos, then sin.
template <typename KVT>
__global__ void qk_norm_rope_kv_kernel(const __nv_bfloat16* __restrict__ qkv, int ld_qkv,
                                       const int* __restrict__ positions, const int64_t* __restrict__ slots,
                                       const float* __restrict__ cos_sin, int rot_dim, int interleaved,
                                       const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                       float eps, __nv_bfloat16* __restrict__ q_out, KVT* __restrict__ k_cache,
                                       KVT* __restrict__ v_cache, const float* __restrict__ k_scale,
                                       const float* __restrict__ v_scale, int H, int KVH, int D, int64_t num_slots,
                                       __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int pos = positions[t];
  const int64_t slot = slots ? slots[t] : -1;
  const bool slot_ok = slot >= 0 && slot < num_slots;
  if (slots && slot >= num_slots) {
    if (threadIdx.x == 0) set_status(kErrBounds);
  }
  const float* cs = cos_sin + (size_t)pos * rot_dim;
  const int half = rot_dim >> 1;
  const __nv_bfloat16* row = qkv + (size_t)t * ld_qkv;
  // one warp per head; blockIdx.y selects the group of nw heads
  for (int hh = blockIdx.y * nw + warp; hh < min(H + 2 * KVH, (int)(blockIdx.y + 1) * nw); hh += nw) {
    const __nv_bfloat16* src = row + (size_t)hh * D;
    const bool is_q = hh < H, is_k = !is_q && hh < H + KVH;
    if (!is_q && !is_k) {
      // value head: plain copy into the cache
      const int kvh = hh - H - KVH;
      if (slot_ok) {
        const int64_t page = slot >> 4, off = slot & 15;
        KVT* dst = v_cache + ((page * KVH + kvh) * 16 + off) * D;
        const float sc = v_scale ? 1.f / v_scale[kvh] : 1.f;
        for (int d = lane; d < D; d += 32) {
          if constexpr (sizeof(KVT) == 1) {
            __nv_fp8_e4m3 f(bf2f(src[d]) * sc);
            dst[d] = *reinterpret_cast<KVT*>(&f);
          } else {
            dst[d] = *reinterpret_cast<const KVT*>(&src[d]);
          }
        }
      }
      if (v_out)
        for (int d = lane; d < D; d += 32) v_out[((size_t)t * KVH + kvh) * D + d] = src[d];
      continue;
    }
    const __nv_bfloat16* nw_ = is_q ? qw : kw;
    // gather this lane's elements (D <= 512 -> at most 16 per lane)
    float v[16];
    float ss = 0.f;
    int cnt = 0;
    for (int d = lane; d < D; d += 32, ++cnt) {
      v[cnt] = bf2f(src[d]);
      ss += v[cnt] * v[cnt];
    }
    if (nw_) {
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)D + eps);
      cnt = 0;
      for (int d = lane; d < D; d += 32, ++cnt) v[cnt] = bf2f(f2bf(v[cnt] * inv * bf2f(nw_[d])));
    }
    // rotary: exchange partners through shared memory (one D-row per warp)
    extern __shared__ float hbuf[];
    float* hb = hbuf + warp * D;
    cnt = 0;
    for (int d = lane; d < D; d += 32, ++cnt) hb[d] = v[cnt];
    __syncwarp();
    cnt = 0;
    for (int d = lane; d < D; d += 32, ++cnt) {
      float o = hb[d];
      if (d < rot_dim) {
        int i, partner;
        float sign;
        if (interleaved) {
          i = d >> 1;
          partner = d ^ 1;
          sign = (d & 1) ? 1.f : -1.f;
        } else {
          i = d < half ? d : d - half;
          partner = d < half ? d + half : d - half;
          sign = d < half ? -1.f : 1.f;
        }
        const float c = cs[i], s = cs[half + i];
        o = hb[d] * c + sign * hb[partner] * s;
      }
      v[cnt] = o;
    }
    __syncwarp();
    if (is_q) {
      __nv_bfloat16* dst = q_out + ((size_t)t * H + hh) * D;
      cnt = 0;
      for (int d = lane; d < D; d += 32, ++cnt) dst[d] = f2bf(v[cnt]);
    } else {
      const int kvh = hh - H;
      if (slot_ok) {
        const int64_t page = slot >> 4, off = slot & 15;
        KVT* dst = k_cache + ((page * KVH + kvh) * 16 + off) * D;
        const float sc = k_scale ? 1.f / k_scale[kvh] : 1.f;
        cnt = 0;
        for (int d = lane; d < D; d += 32, ++cnt) {
          if constexpr (sizeof(KVT) == 1) {
            __nv_fp8_e4m3 f(bf2f(f2bf(v[cnt])) * sc);
            dst[d] = *reinterpret_cast<KVT*>(&f);
          } else {
            __nv_bfloat16 b = f2bf(v[cnt]);
            dst[d] = *reinterpret_cast<KVT*>(&b);
          }
        }
      }
      if (k_out) {
        cnt = 0;
        for (int d = lane; d < D; d += 32, ++cnt) k_out[((size_t)t * KVH + kvh) * D + d] = f2bf(v[cnt]);
      }
    }
  }
}

__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int H, int64_t vocab, float scale) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  const int t = blockIdx.x;
  int64_t id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_status(kErrBounds);
    id = 0;
  }
  const __nv_bfloat16* src = table + id * H;
  __nv_bfloat16* dst = out + (size_t)t * H;
  if (scale == 1.f) {
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8)
      *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + i);
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = f2bf(bf2f(src[i]) * scale);
  }
}

// out = silu(gate) * up for a [T, 2*F] tensor laid out [gate | up].
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int F,
                                int ld_in, int ld_out) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= F) return;
  const float g = bf2f(gu[(size_t)t * ld_in + i]);
  const float u = bf2f(gu[(size_t)t * ld_in + F + i]);
  out[(size_t)t * ld_out + i] = f2bf(silu(g) * u);
}

}  // namespace b200

using namespace b200;

extern "C" {

int b200_add_rmsnorm(void* x, const void* delta, const void* w, void* out, int T, int H, int ldx, int ldd, int ldo,
                     float eps, int w_offset_one, cudaStream_t st) {
  if (T <= 0) return 0;
  if (H % 8) return -1;
  int threads = ((H / 8 + 31) / 32) * 32;
  threads = threads > 1024 ? 1024 : threads;
b200::launch_k(  add_rmsnorm_kernel, dim3(T), dim3(threads), H * sizeof(float), st, 1, 
      reinterpret_cast<__nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(delta),
      reinterpret_cast<const __nv_bfloat16*>(w), reinterpret_cast<__nv_bfloat16*>(out), H, ldx, ldd, ldo, eps,
      w_offset_one);
  return (int)cudaGetLastError();
}

// kv_fp8: 0 -> bf16 pages, 1 -> fp8 e4m3 pages (k_scale / v_scale per KV head).
int b200_add_layernorm(void* x, const void* delta, const void* w, const void* b, void* out, int T, int H, int ldx,
                       int ldd, int ldo, float eps, cudaStream_t st) {
  if (T <= 0) return 0;
  const size_t smem = (size_t)H * sizeof(float);
  if (smem > 48 * 1024) return -1;
  cudaError_t e = launch_k(add_layernorm_kernel, dim3(T), dim3(256), smem, st, 1,
                           reinterpret_cast<__nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(delta),
                           reinterpret_cast<const __nv_bfloat16*>(w), reinterpret_cast<const __nv_bfloat16*>(b),
                           reinterpret_cast<__nv_bfloat16*>(out), H, ldx, ldd, ldo, eps);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_qk_norm_rope_kv(const void* qkv, int T, int ld_qkv, const int* positions, const int64_t* slots,
                         const float* cos_sin, int rot_dim, int interleaved, const void* qw, const void* kw,
                         float eps, void* q_out, void* k_cache, void* v_cache, int kv_fp8, const float* k_scale,
                         const float* v_scale, int H, int KVH, int D, int64_t num_slots, void* k_out, void* v_out,
                         cudaStream_t st) {
  if (T <= 0) return 0;
  if (D > 512 || (rot_dim & 1) || rot_dim > D) return -1;
  const int threads = 128;
  const size_t smem = (threads / 32) * D * sizeof(float);
  const dim3 grid(T, (H + 2 * KVH + threads / 32 - 1) / (threads / 32));
  if (kv_fp8) {
    launch_k(qk_norm_rope_kv_kernel<uint8_t>, grid, dim3(threads), smem, st, 1,
        reinterpret_cast<const __nv_bfloat16*>(qkv), ld_qkv, positions, slots, cos_sin, rot_dim, interleaved,
        reinterpret_cast<const __nv_bfloat16*>(qw), reinterpret_cast<const __nv_bfloat16*>(kw), eps,
        reinterpret_cast<__nv_bfloat16*>(q_out), reinterpret_cast<uint8_t*>(k_cache),
        reinterpret_cast<uint8_t*>(v_cache), k_scale, v_scale, H, KVH, D, num_slots,
        reinterpret_cast<__nv_bfloat16*>(k_out), reinterpret_cast<__nv_bfloat16*>(v_out));
  } else {
    launch_k(qk_norm_rope_kv_kernel<__nv_bfloat16>, grid, dim3(threads), smem, st, 1,
        reinterpret_cast<const __nv_bfloat16*>(qkv), ld_qkv, positions, slots, cos_sin, rot_dim, interleaved,
        reinterpret_cast<const __nv_bfloat16*>(qw), reinterpret_cast<const __nv_bfloat16*>(kw), eps,
        reinterpret_cast<__nv_bfloat16*>(q_out), reinterpret_cast<__nv_bfloat16*>(k_cache),
        reinterpret_cast<__nv_bfloat16*>(v_cache), k_scale, v_scale, H, KVH, D, num_slots,
        reinterpret_cast<__nv_bfloat16*>(k_out), reinterpret_cast<__nv_bfloat16*>(v_out));
  }
  return (int)cudaGetLastError();
}

int b200_embedding(const int* ids, const void* table, void* out, int T, int H, int64_t vocab, float scale,
                   cudaStream_t st) {
  if (T <= 0) return 0;
  if (H % 8) return -1;
b200::launch_k(  embedding_kernel, dim3(T), dim3(256), 0, st, 1, ids, reinterpret_cast<const __nv_bfloat16*>(table),
                                      reinterpret_cast<__nv_bfloat16*>(out), H, vocab, scale);
  return (int)cudaGetLastError();
}

int b200_silu_mul(const void* gu, void* out, int T, int F, int ld_in, int ld_out, cudaStream_t st) {
  if (T <= 0) return 0;
  dim3 grid((F + 255) / 256, T);
b200::launch_k(  silu_mul_kernel, dim3(grid), dim3(256), 0, st, 1, reinterpret_cast<const __nv_bfloat16*>(gu),
                                        reinterpret_cast<__nv_bfloat16*>(out), F, ld_in, ld_out);
  return (int)cudaGetLastError();
}

}  // extern "C"

B200_STATUS_ACCESSORS(norm)
