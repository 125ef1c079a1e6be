// Gated DeltaNet (linear attention) layers of hybrid models (Qwen3-Next,
// Qwen 3.5 / 3.6): causal depthwise conv + SiLU, q/k normalisation, decay and
// write gates, the gated delta-rule recurrence over a per-sequence fp32 state,
// and the gated RMSNorm of the output.
//
// Reference behaviour: MLXLMCommon/GatedDelta.swift:18-140 (decay gate
// g = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b), and the
// recurrence of `gated_delta_step`: S <- g S; u = (v - S k) beta; S <- S + u k^T;
// y = S q) and MLXLLM/Models/Qwen3Next.swift:165-415 (conv1d of kernel 4 over
// q|k|v with SiLU, q scaled by Dk^-1 and k by Dk^-1/2 after an unweighted
// RMSNorm, RMSNormGated(y, z) = rmsnorm(y) * w * silu(z)).
//
// B200 layout: one flattened batch of rows (decode rows of one token, then
// prefill chunks); `cu` [R+1] gives each row's tokens, `slot` [R] its state
// slot and `fresh` [R] whether the row starts at position 0 (zero state).
//   gdn_conv        one CTA per token: conv taps from the row's tokens or the
//                   slot's conv state, SiLU into shared memory, per-head q/k
//                   normalisation (a warp per head), gates; fp32 out.
//   gdn_recurrence  one warp per (row, value head, value row): the Dk state
//                   elements of that row live in registers (Dk / 32 per lane)
//                   across the row's tokens; two warp reductions per token.
//                   CTA (row, 0, 0) also rolls the conv state forward.
//   gdn_norm_gate   one CTA per token: per-head RMSNorm * w * silu(z), bf16.
// State: conv [S][3][C] bf16 (the last three pre-conv inputs), recurrent
// [S][Hv][Dv][Dk] fp32.
//
// Mamba-2 mixers (NemotronH, Mamba2, hybrid SSM models) run on the same
// kernels with mode 1. Reference behaviour: MLXLLM/Models/SSM.swift
// (computeDt: dt = clip(softplus(dt + dt_bias), limits); the ssm step
// state = exp(-exp(A_log) dt) state + dt x B^T, y = state C + D x) and
// MLXLLM/Models/NemotronH.swift:51-160 (conv1d with bias + SiLU over x|B|C,
// RMSNormGated: y * silu(z) normalised over groups of I / n_groups channels).
// The mapping: key heads = n_groups with key dim = state size (C plays q and
// B plays k), value heads = SSM heads with value dim = head dim (x plays v),
// beta = dt, and the delta rule's S k correction is skipped.
#include "b200_common.cuh"

namespace b200 {
namespace gdn {

constexpr int kTaps = 4;

__device__ __forceinline__ int find_row(const int* __restrict__ cu, int R, int t) {
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// P [T][ldp] bf16: q | k | v (C = 2 Hk Dk + Hv Dv channels) | z (Hv Dv) | b (Hv) | a (Hv)
// (mode 1, Mamba-2: C | B | x | z | dt, no b)
__global__ void __launch_bounds__(256) conv_kernel(int CB, int mode, const float* __restrict__ conv_b, float tmin,
                                                   float tmax, const __nv_bfloat16* __restrict__ P, int ldp, int T,
                                                   const int* __restrict__ cu, int R, const int* __restrict__ fresh,
                                                   const int* __restrict__ slot,
                                                   const __nv_bfloat16* __restrict__ conv_state,
                                                   const float* __restrict__ conv_w, int C, int Hk, int Dk, int Hv,
                                                   int Dv, const float* __restrict__ A_log,
                                                   const float* __restrict__ dt_bias, float eps,
                                                   float* __restrict__ qkv_out, float* __restrict__ gb_out) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ float y_sm[];  // [CB] channels of this block
  const int t = blockIdx.x;
  if (t >= T) return;
  // channel block [c0, c0 + CB): whole heads of Dk (q / k) or Dv (v) channels
  const int c0 = blockIdx.y * CB, c1 = min(C, c0 + CB);
  float* y = y_sm - c0;  // y[c] for c in [c0, c1)
  const int r = find_row(cu, R, t);
  const int s0 = cu[r], i = t - s0;
  const bool fr = fresh[r] != 0;
  const __nv_bfloat16* cs = conv_state + (size_t)slot[r] * (kTaps - 1) * C;
  for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
    float acc = conv_b ? conv_b[c] : 0.f;
#pragma unroll
    for (int j = 0; j < kTaps; ++j) {
      const int m = i - (kTaps - 1) + j;
      float x;
      if (m >= 0) x = bf2f(P[(size_t)(s0 + m) * ldp + c]);
      else x = fr ? 0.f : bf2f(cs[(size_t)(kTaps - 1 + m) * C + c]);
      acc = fmaf(conv_w[c * kTaps + j], x, acc);
    }
    y[c] = acc / (1.f + __expf(-acc));
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float* out = qkv_out + (size_t)t * C;
  const int h_lo = c0 / Dk, h_hi = mode == 1 ? 0 : min(2 * Hk, (c1 + Dk - 1) / Dk);
  for (int hh = h_lo + warp; hh < h_hi; hh += nw) {
    const float* src = y + hh * Dk;
    float ss = 0.f;
    for (int d = lane; d < Dk; d += 32) ss = fmaf(src[d], src[d], ss);
    ss = warp_sum(ss);
    const float sc = hh < Hk ? 1.f / (float)Dk : rsqrtf((float)Dk);
    const float inv = rsqrtf(ss / (float)Dk + eps) * sc;
    for (int d = lane; d < Dk; d += 32) out[hh * Dk + d] = src[d] * inv;
  }
  for (int c = (mode == 1 ? c0 : max(c0, 2 * Hk * Dk)) + threadIdx.x; c < c1; c += blockDim.x) out[c] = y[c];
  if (blockIdx.y != 0) return;
  const __nv_bfloat16* pb = P + (size_t)t * ldp + C + Hv * Dv;
  if (mode == 1) {
    for (int h = threadIdx.x; h < Hv; h += blockDim.x) {
      const float dt = fminf(fmaxf(softplus(bf2f(pb[h]) + dt_bias[h]), tmin), tmax);
      gb_out[(size_t)t * 2 * Hv + h] = __expf(-__expf(A_log[h]) * dt);
      gb_out[(size_t)t * 2 * Hv + Hv + h] = dt;
    }
    return;
  }
  for (int h = threadIdx.x; h < Hv; h += blockDim.x) {
    const float b = bf2f(pb[h]), a = bf2f(pb[Hv + h]);
    gb_out[(size_t)t * 2 * Hv + h] = __expf(-__expf(A_log[h]) * softplus(a + dt_bias[h]));
    gb_out[(size_t)t * 2 * Hv + Hv + h] = 1.f / (1.f + __expf(-b));
  }
}

// grid (R, Hv, Dv / (4 * RPW)), 128 threads: warp w owns the RPW value rows
// (blockIdx.z * 4 + w) * RPW .. + RPW - 1. Decode batches use RPW = 4 so
// each lane has 4 state loads of 16 bytes in flight (the step is a pure
// stream of the fp32 states); long prefill rows use RPW = 1 for parallelism.
template <int NK, int RPW, bool MAMBA>
__global__ void __launch_bounds__(128) recurrence_kernel(const float* __restrict__ qkv, const float* __restrict__ gb,
                                                         const int* __restrict__ cu, const int* __restrict__ fresh,
                                                         const int* __restrict__ slot, float* __restrict__ state,
                                                         int Hk, int Hv, int Dv, float* __restrict__ o,
                                                         const __nv_bfloat16* __restrict__ P, int ldp,
                                                         __nv_bfloat16* __restrict__ conv_state, int C,
                                                         const float* __restrict__ Dskip) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int Dk = NK * 32;
  static_assert(NK % 4 == 0 || NK == 2, "Dk of 64, 128 or 256");
  const int r = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dv0 = (blockIdx.z * 4 + warp) * RPW;
  const int hk = h / (Hv / Hk);
  const int s0 = cu[r], n = cu[r + 1] - s0;
  const bool fr = fresh[r] != 0;
  const int sl = slot[r];
  if (dv0 < Dv) {
    float* st = state + (((size_t)sl * Hv + h) * Dv + dv0) * Dk + lane * NK;
    float s[RPW][NK];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      if (fr) {
#pragma unroll
        for (int i = 0; i < NK; ++i) s[j][i] = 0.f;
      } else if constexpr (NK % 4 == 0) {
#pragma unroll
        for (int i = 0; i < NK; i += 4) {
          const float4 v = *reinterpret_cast<const float4*>(st + (size_t)j * Dk + i);
          s[j][i] = v.x, s[j][i + 1] = v.y, s[j][i + 2] = v.z, s[j][i + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < NK; ++i) s[j][i] = st[(size_t)j * Dk + i];
      }
    }
    const int C2 = 2 * Hk * Dk;
    for (int tt = 0; tt < n; ++tt) {
      const size_t t = (size_t)(s0 + tt);
      const float* q = qkv + t * C + hk * Dk + lane * NK;
      const float* k = qkv + t * C + Hk * Dk + hk * Dk + lane * NK;
      const float g = gb[t * 2 * Hv + h], beta = gb[t * 2 * Hv + Hv + h];
      float kk[NK], qq[NK], v[RPW];
#pragma unroll
      for (int i = 0; i < NK; ++i) {
        kk[i] = k[i];
        qq[i] = q[i];
      }
#pragma unroll
      for (int j = 0; j < RPW; ++j) v[j] = qkv[t * C + C2 + h * Dv + dv0 + j];
      float kv[RPW];
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        kv[j] = 0.f;
#pragma unroll
        for (int i = 0; i < NK; ++i) {
          s[j][i] *= g;
          if constexpr (!MAMBA) kv[j] = fmaf(s[j][i], kk[i], kv[j]);
        }
      }
      if constexpr (!MAMBA) {
#pragma unroll
        for (int j = 0; j < RPW; ++j) kv[j] = warp_sum(kv[j]);
      }
      float out[RPW];
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        const float delta = (v[j] - kv[j]) * beta;  // kv = 0 for Mamba-2: dt x
        out[j] = 0.f;
#pragma unroll
        for (int i = 0; i < NK; ++i) {
          s[j][i] = fmaf(kk[i], delta, s[j][i]);
          out[j] = fmaf(s[j][i], qq[i], out[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < RPW; ++j) out[j] = warp_sum(out[j]);
      if constexpr (MAMBA) {
        const float dd = Dskip[h];
#pragma unroll
        for (int j = 0; j < RPW; ++j) out[j] = fmaf(dd, v[j], out[j]);
      }
      if (lane < RPW) {  // lane j stores row j (registers indexed by unrolled compare)
        float oj = out[0];
#pragma unroll
        for (int j = 1; j < RPW; ++j)
          if (lane == j) oj = out[j];
        o[t * Hv * Dv + h * Dv + dv0 + lane] = oj;
      }
    }
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      if constexpr (NK % 4 == 0) {
#pragma unroll
        for (int i = 0; i < NK; i += 4)
          *reinterpret_cast<float4*>(st + (size_t)j * Dk + i) = make_float4(s[j][i], s[j][i + 1], s[j][i + 2],
                                                                            s[j][i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < NK; ++i) st[(size_t)j * Dk + i] = s[j][i];
      }
    }
  }
  // roll the conv state to the row's last three inputs (the conv kernel that
  // read the old state has completed: this grid waited for it)
  if (h == 0 && blockIdx.z == 0) {
    __nv_bfloat16* cs = conv_state + (size_t)sl * (kTaps - 1) * C;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
#pragma unroll
      for (int j = 0; j < kTaps - 1; ++j) {
        const int m = n - (kTaps - 1) + j;  // index of the input that becomes tap j
        __nv_bfloat16 x;
        if (m >= 0) x = P[(size_t)(s0 + m) * ldp + c];
        else x = fr ? f2bf(0.f) : cs[(size_t)(kTaps - 1 + m) * C + c];  // reads ahead of the writes
        cs[(size_t)j * C + c] = x;
      }
    }
  }
}

template <int NK, bool MAMBA>
static cudaError_t launch_rec(int rpw, int R, int Hv, int Dv, cudaStream_t st, const float* qkv, const float* gb,
                              const int* cu, const int* fresh, const int* slot, float* state, int Hk, float* o,
                              const __nv_bfloat16* p, int ldp, __nv_bfloat16* cs, int C, const float* Dskip) {
  if (rpw == 4) {
    const dim3 grid(R, Hv, (Dv + 15) / 16);
    return launch_k(recurrence_kernel<NK, 4, MAMBA>, grid, dim3(128), 0, st, 1, qkv, gb, cu, fresh, slot, state, Hk,
                    Hv, Dv, o, p, ldp, cs, C, Dskip);
  }
  const dim3 grid(R, Hv, (Dv + 3) / 4);
  return launch_k(recurrence_kernel<NK, 1, MAMBA>, grid, dim3(128), 0, st, 1, qkv, gb, cu, fresh, slot, state, Hk,
                  Hv, Dv, o, p, ldp, cs, C, Dskip);
}

template <int NK>
static cudaError_t launch_rec_mode(int mode, int rpw, int R, int Hv, int Dv, cudaStream_t st, const float* qkv,
                                   const float* gb, const int* cu, const int* fresh, const int* slot, float* state,
                                   int Hk, float* o, const __nv_bfloat16* p, int ldp, __nv_bfloat16* cs, int C,
                                   const float* Dskip) {
  if (mode == 1)
    return launch_rec<NK, true>(rpw, R, Hv, Dv, st, qkv, gb, cu, fresh, slot, state, Hk, o, p, ldp, cs, C, Dskip);
  return launch_rec<NK, false>(rpw, R, Hv, Dv, st, qkv, gb, cu, fresh, slot, state, Hk, o, p, ldp, cs, C, Dskip);
}

// Mamba-2 gated norm: one CTA per (token, norm group): v = y * silu(z),
// out = v * rsqrt(mean(v^2) + eps) * w over the group's channels -> bf16
__global__ void __launch_bounds__(256) group_norm_gate_kernel(const float* __restrict__ o, int T, int I, int gsize,
                                                              const __nv_bfloat16* __restrict__ z, int ldz,
                                                              const __nv_bfloat16* __restrict__ w, float eps,
                                                              __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  const int t = blockIdx.x, c0 = blockIdx.y * gsize;
  if (t >= T) return;
  const float* src = o + (size_t)t * I + c0;
  const __nv_bfloat16* zr = z + (size_t)t * ldz + c0;
  float ss = 0.f;
  for (int c = threadIdx.x; c < gsize; c += blockDim.x) {
    const float zz = bf2f(zr[c]);
    const float v = src[c] * (zz / (1.f + __expf(-zz)));
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    ss = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    ss = warp_sum(ss);
    if (lane == 0) red[0] = ss;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)gsize + eps);
  for (int c = threadIdx.x; c < gsize; c += blockDim.x) {
    const float zz = bf2f(zr[c]);
    const float v = src[c] * (zz / (1.f + __expf(-zz)));
    out[(size_t)t * ldo + c0 + c] = f2bf(v * inv * bf2f(w[c0 + c]));
  }
}

// one CTA per token; warp per value head: rmsnorm(o) * w * silu(z) -> bf16
__global__ void __launch_bounds__(256) norm_gate_kernel(const float* __restrict__ o, int T, int Hv, int Dv,
                                                        const __nv_bfloat16* __restrict__ z, int ldz,
                                                        const __nv_bfloat16* __restrict__ w, float eps,
                                                        __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= T) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int h = blockIdx.y * nw + warp; h < Hv; h += gridDim.y * nw) {
    const float* src = o + ((size_t)t * Hv + h) * Dv;
    float ss = 0.f;
    for (int d = lane; d < Dv; d += 32) ss = fmaf(src[d], src[d], ss);
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)Dv + eps);
    for (int d = lane; d < Dv; d += 32) {
      const float zz = bf2f(z[(size_t)t * ldz + h * Dv + d]);
      const float g = zz / (1.f + __expf(-zz));
      out[(size_t)t * ldo + h * Dv + d] = f2bf(src[d] * inv * bf2f(w[d]) * g);
    }
  }
}

// LFM2 short convolution (MLXLLM/Models/LFM2.swift:207-233): P [T][ldp] =
// B | C | x (C channels each); Bx = B * x; y = C * (sum_j w[c][j] Bx[t-L+1+j]
// (+ bias)), the taps before a row's chunk read the conv state (the row's
// last L - 1 Bx values, bf16). One thread per (token, channel); a second
// kernel rolls the state once every token has read it.
__global__ void __launch_bounds__(256) short_conv_kernel(const __nv_bfloat16* __restrict__ P, int ldp, int T,
                                                         const int* __restrict__ cu, int R,
                                                         const int* __restrict__ fresh, const int* __restrict__ slot,
                                                         const __nv_bfloat16* __restrict__ conv_state,
                                                         const float* __restrict__ w, const float* __restrict__ bias,
                                                         int C, int taps, __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x, c = blockIdx.y * blockDim.x + threadIdx.x;
  if (t >= T || c >= C) return;
  const int r = find_row(cu, R, t);
  const int s0 = cu[r], i = t - s0;
  const bool fr = fresh[r] != 0;
  const __nv_bfloat16* cs = conv_state + (size_t)slot[r] * (taps - 1) * C;
  float acc = bias ? bias[c] : 0.f;
  for (int j = 0; j < taps; ++j) {
    const int m = i - (taps - 1) + j;
    float bx;
    if (m >= 0) {
      const __nv_bfloat16* pr = P + (size_t)(s0 + m) * ldp;
      bx = bf2f(f2bf(bf2f(pr[c]) * bf2f(pr[2 * C + c])));  // Bx rounded as the stored state is
    } else {
      bx = fr ? 0.f : bf2f(cs[(size_t)(taps - 1 + m) * C + c]);
    }
    acc = fmaf(w[c * taps + j], bx, acc);
  }
  out[(size_t)t * ldo + c] = f2bf(bf2f(P[(size_t)t * ldp + C + c]) * acc);
}

__global__ void __launch_bounds__(256) short_conv_roll_kernel(const __nv_bfloat16* __restrict__ P, int ldp,
                                                              const int* __restrict__ cu,
                                                              const int* __restrict__ fresh,
                                                              const int* __restrict__ slot,
                                                              __nv_bfloat16* __restrict__ conv_state, int C,
                                                              int taps) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x, c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int s0 = cu[r], n = cu[r + 1] - s0;
  const bool fr = fresh[r] != 0;
  __nv_bfloat16* cs = conv_state + (size_t)slot[r] * (taps - 1) * C;
  for (int j = 0; j < taps - 1; ++j) {  // reads ahead of the writes (m - j >= ... keeps order)
    const int m = n - (taps - 1) + j;
    __nv_bfloat16 x;
    if (m >= 0) {
      const __nv_bfloat16* pr = P + (size_t)(s0 + m) * ldp;
      x = f2bf(bf2f(pr[c]) * bf2f(pr[2 * C + c]));
    } else {
      x = fr ? f2bf(0.f) : cs[(size_t)(taps - 1 + m) * C + c];
    }
    cs[(size_t)j * C + c] = x;
  }
}

// out = x * sigmoid(g) (gated attention output), bf16 [T][N]
__global__ void sigmoid_mul_kernel(const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ g,
                                   int ldg, int T, int N, __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t total = (size_t)T * N;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(e / N), c = (int)(e % N);
    const float gv = bf2f(g[(size_t)t * ldg + c]);
    out[(size_t)t * ldo + c] = f2bf(bf2f(x[(size_t)t * ldx + c]) / (1.f + __expf(-gv)));
  }
}

}  // namespace gdn
}  // namespace b200

using namespace b200;

extern "C" {

// mode 0: Gated DeltaNet; mode 1: Mamba-2 (conv bias, no q/k normalisation,
// dt gates clipped to [tmin, tmax], P without the b section)
int b200_gdn_conv(const void* P, int ldp, int T, const int* cu, int R, const int* fresh, const int* slot,
                  const void* conv_state, const float* conv_w, int C, int Hk, int Dk, int Hv, int Dv,
                  const float* A_log, const float* dt_bias, float eps, float* qkv_out, float* gb_out,
                  int mode, const float* conv_b, float tmin, float tmax, cudaStream_t st) {
  if (T <= 0) return 0;
  if (R <= 0 || C != 2 * Hk * Dk + Hv * Dv || ldp < C + Hv * Dv + (mode == 1 ? 1 : 2) * Hv ||
      (Dv % Dk && Dk % Dv))
    return -1;
  // channel blocks of whole heads: 8 key heads' worth (multiples of Dk and Dv)
  int CB = 8 * (Dk > Dv ? Dk : Dv);
  if ((2 * Hk * Dk) % CB) CB = Dk > Dv ? Dk : Dv;
  const size_t smem = (size_t)CB * sizeof(float);
  if (int e = b200::smem_attr_once<gdn::conv_kernel>(200 * 1024)) return e;
  cudaError_t e = launch_k(gdn::conv_kernel, dim3(T, (C + CB - 1) / CB), dim3(256), smem, st, 1, CB, mode, conv_b,
                           tmin, tmax, reinterpret_cast<const __nv_bfloat16*>(P), ldp, T, cu, R, fresh, slot,
                           reinterpret_cast<const __nv_bfloat16*>(conv_state), conv_w, C, Hk, Dk, Hv, Dv, A_log,
                           dt_bias, eps, qkv_out, gb_out);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// mode 1 (Mamba-2): no S k correction, y += D[h] x; Dskip [Hv] fp32
int b200_gdn_recurrence(const float* qkv, const float* gb, const int* cu, int R, const int* fresh, const int* slot,
                        float* state, int Hk, int Dk, int Hv, int Dv, float* o, const void* P, int ldp,
                        void* conv_state, int C, int T, int mode, const float* Dskip, cudaStream_t st) {
  if (R <= 0) return 0;
  if ((Hv % Hk) || (Dv % 16) || C != 2 * Hk * Dk + Hv * Dv || (mode == 1 && !Dskip)) return -1;
  const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(P);
  __nv_bfloat16* cs = reinterpret_cast<__nv_bfloat16*>(conv_state);
  // several value rows per warp when the batch alone fills the GPU (decode)
  const long warps4 = (long)R * Hv * Dv / 4;
  const int rpw = (T <= 2 * R && warps4 >= 148 * 16) ? 4 : 1;
  cudaError_t e;
  switch (Dk) {
    case 64:
      e = gdn::launch_rec_mode<2>(mode, rpw, R, Hv, Dv, st, qkv, gb, cu, fresh, slot, state, Hk, o, p, ldp, cs, C,
                                  Dskip);
      break;
    case 128:
      e = gdn::launch_rec_mode<4>(mode, rpw, R, Hv, Dv, st, qkv, gb, cu, fresh, slot, state, Hk, o, p, ldp, cs, C,
                                  Dskip);
      break;
    case 256:
      e = gdn::launch_rec_mode<8>(mode, rpw, R, Hv, Dv, st, qkv, gb, cu, fresh, slot, state, Hk, o, p, ldp, cs, C,
                                  Dskip);
      break;
    default: return -1;
  }
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_gdn_norm_gate(const float* o, int T, int Hv, int Dv, const void* z, int ldz, const void* w, float eps,
                       void* out, int ldo, cudaStream_t st) {
  if (T <= 0) return 0;
  cudaError_t e = launch_k(gdn::norm_gate_kernel, dim3(T, (Hv + 7) / 8), dim3(256), 0, st, 1, o, T, Hv, Dv,
                           reinterpret_cast<const __nv_bfloat16*>(z), ldz, reinterpret_cast<const __nv_bfloat16*>(w),
                           eps, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// o [T][I] fp32, z [T][ldz] bf16, w [I] bf16; groups of gsize channels (I % gsize == 0)
int b200_group_norm_gate(const float* o, int T, int I, int gsize, const void* z, int ldz, const void* w, float eps,
                         void* out, int ldo, cudaStream_t st) {
  if (T <= 0) return 0;
  if (gsize <= 0 || I % gsize) return -1;
  cudaError_t e = launch_k(gdn::group_norm_gate_kernel, dim3(T, I / gsize), dim3(256), 0, st, 1, o, T, I, gsize,
                           reinterpret_cast<const __nv_bfloat16*>(z), ldz, reinterpret_cast<const __nv_bfloat16*>(w),
                           eps, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// LFM2 short conv: P [T][ldp] (B | C | x), rows as the recurrent kernels
// take them, conv_state [S][taps-1][C] bf16, w [C][taps] fp32, bias [C] or
// null; out [T][ldo] bf16 = C * conv(B * x). Advances each row's state.
int b200_short_conv(const void* P, int ldp, int T, const int* cu, int R, const int* fresh, const int* slot,
                    void* conv_state, const float* w, const float* bias, int C, int taps, void* out, int ldo,
                    cudaStream_t st) {
  if (T <= 0 || R <= 0) return 0;
  if (taps < 2 || taps > 8 || ldp < 3 * C) return -1;
  const auto* p = reinterpret_cast<const __nv_bfloat16*>(P);
  auto* cs = reinterpret_cast<__nv_bfloat16*>(conv_state);
  cudaError_t e = launch_k(gdn::short_conv_kernel, dim3(T, (C + 255) / 256), dim3(256), 0, st, 1, p, ldp, T, cu, R,
                           fresh, slot, cs, w, bias, C, taps, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  if (e != cudaSuccess) return (int)e;
  e = launch_k(gdn::short_conv_roll_kernel, dim3(R, (C + 255) / 256), dim3(256), 0, st, 1, p, ldp, cu, fresh, slot,
               cs, C, taps);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_sigmoid_mul(const void* x, int ldx, const void* g, int ldg, int T, int N, void* out, int ldo,
                     cudaStream_t st) {
  if (T <= 0 || N <= 0) return 0;
  const size_t total = (size_t)T * N;
  const size_t blocks = (total + 255) / 256;
  const int grid = (int)(blocks < 148 * 8 ? blocks : 148 * 8);
  cudaError_t e = launch_k(gdn::sigmoid_mul_kernel, dim3(grid), dim3(256), 0, st, 1,
                           reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<const __nv_bfloat16*>(g),
                           ldg, T, N, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // extern "C"

B200_STATUS_ACCESSORS(gdn)
