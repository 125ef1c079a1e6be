// Fused sampling pipeline, one CTA per row, in the vLLM order that the
// reference's CBv2 sampler documents (DefaultSamplerV2.swift:84-183,
// LogitsPipelineV2.swift:292-357, docs/engine-v2/specs/E-sampling.md):
//   raw logprobs -> logit bias -> repetition penalty -> frequency/presence
//   penalties -> grammar/tool token mask -> temperature -> top-k -> top-p
//   -> min-p -> draw.
// The draw is Gumbel-max with a counter-based Philox-4x32-10 stream keyed by
// (seed, request id) and counted by (step, token), so a row's sample depends
// only on its own logits and key (batch-composition invariant, reproducible).
//
// top-k and top-p thresholds are found exactly by radix select over the
// order-preserving integer image of the scaled logits: 4 passes of 8-bit
// digits. For top-p the pass histograms accumulate probability mass as
// 2^30-scaled integers in 64-bit counters, so the result does not depend on
// the order of atomic additions.
#include <cfloat>

#include "b200_common.cuh"

namespace b200 {

// ---------------- Philox-4x32-10 (Salmon et al., SC'11) ----------------
__host__ __device__ __forceinline__ void philox_round(uint32_t c[4], uint32_t k[2]) {
  const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
  const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
  const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
  const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
  const uint32_t n0 = hi1 ^ c[1] ^ k[0];
  const uint32_t n2 = hi0 ^ c[3] ^ k[1];
  c[0] = n0;
  c[1] = lo1;
  c[2] = n2;
  c[3] = lo0;
}
__host__ __device__ __forceinline__ uint32_t philox_u32(uint64_t key, uint64_t step, uint32_t idx) {
  uint32_t c[4] = {idx, (uint32_t)step, (uint32_t)(step >> 32), 0x42323030u};
  uint32_t k[2] = {(uint32_t)key, (uint32_t)(key >> 32)};
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    philox_round(c, k);
    k[0] += 0x9E3779B9u;
    k[1] += 0xBB67AE85u;
  }
  return c[0];
}
// Uniform in (0, 1) from the top 24 bits.
__device__ __forceinline__ float philox_uniform(uint64_t key, uint64_t step, uint32_t idx) {
  const uint32_t x = philox_u32(key, step, idx);
  return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

// Order-preserving map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kThreads = 1024;

// ---------------- logits processing (in place) ----------------
struct ProcessArgs {
  float* logits;
  int64_t ld;
  int V;
  const int* bias_ids;
  const float* bias_vals;
  const int* n_bias;
  int ld_bias;
  const int* rep_ids;
  const int* n_rep;
  int ld_rep;
  const float* rep_penalty;
  const int* out_ids;
  const int* n_out;
  int ld_out;
  const float* freq_penalty;
  const float* pres_penalty;
  const uint32_t* allow_mask;  // [B, ld_mask] bit 1 = allowed, or null
  int ld_mask;
  const int* mask_rows;  // [B] 1 if the row's mask applies
};

__global__ void __launch_bounds__(kThreads) logits_process_kernel(ProcessArgs a) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  extern __shared__ uint32_t seen[];  // V bits
  const int b = blockIdx.x;
  float* lg = a.logits + (size_t)b * a.ld;
  const int words = (a.V + 31) / 32;
  // 1) logit bias (ids unique per row)
  if (a.n_bias) {
    const int nb = a.n_bias[b];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      const int id = a.bias_ids[(size_t)b * a.ld_bias + i];
      if (id >= 0 && id < a.V) lg[id] += a.bias_vals[(size_t)b * a.ld_bias + i];
    }
    __syncthreads();
  }
  // 2) repetition penalty over the recent-context window, once per distinct id
  if (a.n_rep && a.rep_penalty[b] != 1.f) {
    for (int i = threadIdx.x; i < words; i += blockDim.x) seen[i] = 0;
    __syncthreads();
    const int nr = a.n_rep[b];
    const float rp = a.rep_penalty[b];
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
      const int id = a.rep_ids[(size_t)b * a.ld_rep + i];
      if (id < 0 || id >= a.V) continue;
      const uint32_t bit = 1u << (id & 31);
      if (!(atomicOr(&seen[id >> 5], bit) & bit)) {
        const float x = lg[id];
        lg[id] = x > 0.f ? x / rp : x * rp;
      }
    }
    __syncthreads();
  }
  // 3) frequency / presence penalties over generated tokens: the first
  //    occurrence of an id counts all occurrences and applies one update.
  if (a.n_out && (a.freq_penalty[b] != 0.f || a.pres_penalty[b] != 0.f)) {
    const int no = a.n_out[b];
    const int* ids = a.out_ids + (size_t)b * a.ld_out;
    for (int i = threadIdx.x; i < no; i += blockDim.x) {
      const int id = ids[i];
      if (id < 0 || id >= a.V) continue;
      bool first = true;
      for (int j = 0; j < i; ++j)
        if (ids[j] == id) {
          first = false;
          break;
        }
      if (!first) continue;
      int cnt = 1;
      for (int j = i + 1; j < no; ++j) cnt += (ids[j] == id);
      lg[id] = lg[id] - ((float)cnt * a.freq_penalty[b] + a.pres_penalty[b]);
    }
    __syncthreads();
  }
  // 4) token mask
  if (a.allow_mask && a.mask_rows[b]) {
    const uint32_t* mk = a.allow_mask + (size_t)b * a.ld_mask;
    for (int i = threadIdx.x; i < a.V; i += blockDim.x)
      if (!((mk[i >> 5] >> (i & 31)) & 1u)) lg[i] = -INFINITY;
  }
}

// ---------------- sampling ----------------
struct SampleArgs {
  const float* logits;
  int64_t ld;
  int V;
  const float* temperature;  // [B]; <= 0 -> greedy
  const int* top_k;          // [B]; <= 0 -> off
  const float* top_p;        // [B]; >= 1 -> off
  const float* min_p;        // [B]; <= 0 -> off
  const uint64_t* keys;      // [B] RNG key (seed mixed with request id)
  const int64_t* steps;      // [B] RNG counter (generation step)
  int* out_tokens;           // [B]
  int* out_tokens2;          // optional second destination (next step's input ids)
  float* out_logit;          // optional [B] value of the chosen logit (raw)
  int* flags;                // optional [B]: 1 when the row holds a NaN or +-inf logit
};

__device__ __forceinline__ void block_argmax(float& v, int& idx, float* sv, int* si) {
  // ties -> smallest index
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  __syncthreads();
  if (lane == 0) {
    sv[wid] = v;
    si[wid] = idx;
  }
  __syncthreads();
  if (wid == 0) {
    v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    idx = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (lane == 0) {
      sv[0] = v;
      si[0] = idx;
    }
  }
  __syncthreads();
  v = sv[0];
  idx = si[0];
}

__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ unsigned long long hist[256];
  // per-warp private histograms [kThreads / 32][256] (dynamic shared memory):
  // with near-uniform logits almost every key of a radix pass falls into one
  // or two bins, and one block-wide histogram would serialise every thread's
  // atomic on those bins; integer sums keep the result order-independent
  extern __shared__ unsigned long long whist[];
  const int hw = threadIdx.x >> 5;
  auto hist_zero = [&]() {
    for (int i = threadIdx.x; i < (kThreads / 32) * 256; i += blockDim.x) whist[i] = 0;
    __syncthreads();
  };
  auto hist_collect = [&]() {  // after the adds: hist[bin] = sum over warps
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      unsigned long long t = 0;
      for (int w = 0; w < kThreads / 32; ++w) t += whist[w * 256 + i];
      hist[i] = t;
    }
    __syncthreads();
  };
  __shared__ uint32_t s_prefix;
  __shared__ unsigned long long s_rem;
  const int b = blockIdx.x;
  const float* lg = a.logits + (size_t)b * a.ld;
  const float T = a.temperature[b];

  // greedy / max pass (argmax of raw logits also gives the softmax max), and
  // the non-finite check (|x| <= FLT_MAX is false exactly for NaN and +-inf)
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  bool bad = false;
  for (int i = threadIdx.x; i < a.V; i += blockDim.x) {
    const float x = lg[i];
    bad |= !(fabsf(x) <= FLT_MAX);
    if (x > bv) {
      bv = x;
      bi = i;
    }
  }
  if (a.flags) {
    const int any_bad = __syncthreads_or(bad ? 1 : 0);
    if (threadIdx.x == 0) a.flags[b] = any_bad;
  }
  block_argmax(bv, bi, sv, si);
  if (T <= 0.f || bv == -INFINITY) {
    if (threadIdx.x == 0) {
      const int tok = bi == 0x7fffffff ? 0 : bi;
      a.out_tokens[b] = tok;
      if (a.out_tokens2) a.out_tokens2[b] = tok;
      if (a.out_logit) a.out_logit[b] = bv;
    }
    return;
  }
  const float invT = 1.f / T;
  const float mx = bv * invT;  // max scaled logit
  uint32_t thr = 0;            // keep keys >= thr

  // ---- top-k ----
  const int k = a.top_k[b];
  if (k > 0 && k < a.V) {
    uint32_t prefix = 0;
    unsigned long long rem = (unsigned long long)k;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      hist_zero();
      const uint32_t pmask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = threadIdx.x; i < a.V; i += blockDim.x) {
        const uint32_t key = fkey(lg[i] * invT);
        if ((key & pmask) == prefix) atomicAdd(&whist[hw * 256 + ((key >> shift) & 255u)], 1ull);
      }
      hist_collect();
      if (threadIdx.x == 0) {
        unsigned long long cum = 0;
        int d = 255;
        for (; d > 0; --d) {
          if (cum + hist[d] >= rem) break;
          cum += hist[d];
        }
        s_prefix = prefix | ((uint32_t)d << shift);
        s_rem = rem - cum;
      }
      __syncthreads();
      prefix = s_prefix;
      rem = s_rem;
    }
    thr = prefix;
  }

  // ---- top-p (exact, integer mass) ----
  const float p = a.top_p[b];
  if (p < 1.f) {
    // total mass of the top-k survivors
    unsigned long long tot = 0;
    for (int i = threadIdx.x; i < a.V; i += blockDim.x) {
      const float s = lg[i] * invT;
      if (fkey(s) >= thr) tot += (unsigned long long)__float2uint_rn(exp2f((s - mx) * 1.4426950408889634f) * 1073741824.f);
    }
    // block reduce (64-bit)
    __shared__ unsigned long long red64[32];
    {
      const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
      if (lane == 0) red64[wid] = tot;
      __syncthreads();
      if (threadIdx.x == 0) {
        unsigned long long t = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red64[w];
        red64[0] = t;
      }
      __syncthreads();
      tot = red64[0];
    }
    const unsigned long long target = (unsigned long long)ceil((double)p * (double)tot);
    uint32_t prefix = 0;
    unsigned long long rem = target > 0 ? target : 1;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      hist_zero();
      const uint32_t pmask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = threadIdx.x; i < a.V; i += blockDim.x) {
        const float s = lg[i] * invT;
        const uint32_t key = fkey(s);
        if (key >= thr && (key & pmask) == prefix)
          atomicAdd(&whist[hw * 256 + ((key >> shift) & 255u)],
                    (unsigned long long)__float2uint_rn(exp2f((s - mx) * 1.4426950408889634f) * 1073741824.f));
      }
      hist_collect();
      if (threadIdx.x == 0) {
        unsigned long long cum = 0;
        int d = 255;
        for (; d > 0; --d) {
          if (cum + hist[d] >= rem) break;
          cum += hist[d];
        }
        s_prefix = prefix | ((uint32_t)d << shift);
        s_rem = rem - cum;
      }
      __syncthreads();
      prefix = s_prefix;
      rem = s_rem;
    }
    thr = max(thr, prefix);
  }

  // ---- min-p: keep p_i >= min_p * p_max  <=>  s_i >= mx + ln(min_p) ----
  const float mp = a.min_p[b];
  if (mp > 0.f) thr = max(thr, fkey(mx + logf(mp)));

  // ---- Gumbel-max draw over the kept set ----
  const uint64_t key = a.keys[b];
  const uint64_t step = (uint64_t)a.steps[b];
  float best = -INFINITY;
  int besti = 0x7fffffff;
  for (int i = threadIdx.x; i < a.V; i += blockDim.x) {
    const float s = lg[i] * invT;
    if (fkey(s) < thr || s == -INFINITY) continue;
    const float u = philox_uniform(key, step, (uint32_t)i);
    const float g = -logf(-logf(u));
    const float v = s + g;
    if (v > best) {
      best = v;
      besti = i;
    }
  }
  block_argmax(best, besti, sv, si);
  if (threadIdx.x == 0) {
    const int tok = besti == 0x7fffffff ? 0 : besti;
    a.out_tokens[b] = tok;
    if (a.out_tokens2) a.out_tokens2[b] = tok;
    if (a.out_logit) a.out_logit[b] = lg[tok];
  }
}

// Greedy argmax only (the all-greedy fast path). With `flags`, flags[b] = 1
// when any logit of the row is NaN or +-infinity (NaN never wins the argmax,
// so the token alone cannot show it), else 0.
__global__ void __launch_bounds__(kThreads) argmax_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                          int* out, int* out2, int* flags) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int b = blockIdx.x;
  const float* lg = logits + (size_t)b * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const int V4 = (ld % 4 == 0) ? V / 4 : 0;
  const float4* lg4 = reinterpret_cast<const float4*>(lg);
  // |x| <= FLT_MAX is false exactly for NaN and +-infinity
  bool bad = false;
  for (int i = threadIdx.x; i < V4; i += blockDim.x) {
    const float4 x = lg4[i];
    bad |= !(fabsf(x.x) <= FLT_MAX) | !(fabsf(x.y) <= FLT_MAX) | !(fabsf(x.z) <= FLT_MAX) | !(fabsf(x.w) <= FLT_MAX);
    if (x.x > bv) { bv = x.x; bi = 4 * i; }
    if (x.y > bv) { bv = x.y; bi = 4 * i + 1; }
    if (x.z > bv) { bv = x.z; bi = 4 * i + 2; }
    if (x.w > bv) { bv = x.w; bi = 4 * i + 3; }
  }
  for (int i = 4 * V4 + threadIdx.x; i < V; i += blockDim.x) {
    bad |= !(fabsf(lg[i]) <= FLT_MAX);
    if (lg[i] > bv) {
      bv = lg[i];
      bi = i;
    }
  }
  const int any_bad = flags ? __syncthreads_or(bad ? 1 : 0) : 0;
  block_argmax(bv, bi, sv, si);
  if (threadIdx.x == 0) {
    const int tok = bi == 0x7fffffff ? 0 : bi;
    out[b] = tok;
    if (out2) out2[b] = tok;
    if (flags) flags[b] = any_bad;
  }
}

// Raw log-softmax statistics: logprob of `tokens[b]` and the top-n entries.
__global__ void __launch_bounds__(kThreads) logprobs_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                            const int* tokens, int n_top, float* out_lp,
                                                            int* top_ids, float* top_lp) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float red[32];
  const int b = blockIdx.x;
  const float* lg = logits + (size_t)b * ld;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, lg[i]);
  mx = block_max(mx, red);
  float se = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) se += expf(lg[i] - mx);
  se = block_sum(se, red);
  const float lse = mx + logf(se);
  if (threadIdx.x == 0 && tokens) out_lp[b] = lg[tokens[b]] - lse;
  // top-n by repeated argmax, excluding already chosen (n_top is small)
  float prev_v = INFINITY;
  int prev_i = -1;
  for (int r = 0; r < n_top; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float x = lg[i];
      // strictly after (prev_v, prev_i) in (value desc, index asc) order
      const bool after = (x < prev_v) || (x == prev_v && i > prev_i);
      if (after && (x > bv || (x == bv && i < bi))) {
        bv = x;
        bi = i;
      }
    }
    block_argmax(bv, bi, sv, si);
    if (threadIdx.x == 0) {
      top_ids[(size_t)b * n_top + r] = bi == 0x7fffffff ? -1 : bi;
      top_lp[(size_t)b * n_top + r] = bv - lse;
    }
    prev_v = bv;
    prev_i = bi;
  }
}

}  // namespace b200

using namespace b200;

extern "C" {

int b200_logits_process(float* logits, int64_t ld, int B, int V, const int* bias_ids, const float* bias_vals,
                        const int* n_bias, int ld_bias, const int* rep_ids, const int* n_rep, int ld_rep,
                        const float* rep_penalty, const int* out_ids, const int* n_out, int ld_out,
                        const float* freq_penalty, const float* pres_penalty, const uint32_t* allow_mask,
                        int ld_mask, const int* mask_rows, cudaStream_t st) {
  if (B <= 0) return 0;
  ProcessArgs a{logits, ld,      V,           bias_ids, bias_vals,    n_bias,       ld_bias,
                rep_ids, n_rep,  ld_rep,      rep_penalty, out_ids,   n_out,        ld_out,
                freq_penalty, pres_penalty, allow_mask, ld_mask, mask_rows};
  const size_t smem = ((V + 31) / 32) * sizeof(uint32_t);
  if (int e = b200::smem_attr_once<logits_process_kernel>(200 * 1024)) return e;
  if (smem > 200 * 1024) return -1;
b200::launch_k(  logits_process_kernel, dim3(B), dim3(kThreads), smem, st, 1, a);
  return (int)cudaGetLastError();
}

int b200_sample(const float* logits, int64_t ld, int B, int V, const float* temperature, const int* top_k,
                const float* top_p, const float* min_p, const uint64_t* keys, const int64_t* steps, int* out_tokens,
                int* out_tokens2, float* out_logit, int* flags, cudaStream_t st) {
  if (B <= 0) return 0;
  SampleArgs a{logits, ld, V, temperature, top_k, top_p, min_p, keys, steps, out_tokens, out_tokens2, out_logit,
               flags};
  constexpr int smem = (kThreads / 32) * 256 * (int)sizeof(unsigned long long);
  if (int r = b200::smem_attr_once<sample_kernel>(smem)) return r;
  cudaError_t e = b200::launch_k(sample_kernel, dim3(B), dim3(kThreads), smem, st, 1, a);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// Greedy token, its softmax probability (the confidence of mask-diffusion
// decoding) and the raw max logit per row, in one pass: each thread keeps a
// running (max, sum of exp(x - max), index), rescaling the sum when the max
// moves; warps and then the block merge the triples (ties -> smaller index).
// p(argmax) = exp(m - logsumexp) = 1 / sum exp(x - m).
__device__ __forceinline__ void msi_push(float& m, float& s, int& idx, float x, int i) {
  if (x > m) {
    s = (m == -INFINITY ? 0.f : s * __expf(m - x)) + 1.f;
    m = x;
    idx = i;
  } else if (x != -INFINITY) {
    s += __expf(x - m);
  }
}

// this thread's (max, sum, index) over lg[c0, c1): 16-byte loads (two in
// flight per iteration) when the range and the row are 4-aligned
__device__ __forceinline__ void msi_scan(const float* __restrict__ lg, int c0, int c1, bool vec, float& m, float& s,
                                         int& idx) {
  if (vec) {
    const float4* l4 = reinterpret_cast<const float4*>(lg);
    const int v0 = c0 >> 2, v1 = c1 >> 2;
#pragma unroll 2
    for (int i = v0 + (int)threadIdx.x; i < v1; i += blockDim.x) {
      const float4 x = l4[i];
      msi_push(m, s, idx, x.x, 4 * i);
      msi_push(m, s, idx, x.y, 4 * i + 1);
      msi_push(m, s, idx, x.z, 4 * i + 2);
      msi_push(m, s, idx, x.w, 4 * i + 3);
    }
    c0 = max(c0, v1 << 2);  // an empty range [c0, c1) stays empty
  }
  for (int i = c0 + threadIdx.x; i < c1; i += blockDim.x) msi_push(m, s, idx, lg[i], i);
}

__device__ __forceinline__ void merge_msi(float& m, float& s, int& i, float om, float os, int oi) {
  if (om > m || (om == m && oi < i)) {
    s = (m == -INFINITY ? 0.f : s * __expf(m - om)) + os;
    m = om;
    i = oi;
  } else if (om != -INFINITY) {
    s += os * __expf(om - m);
  }
}

__global__ void __launch_bounds__(kThreads) argmax_conf_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                               int* __restrict__ tok, float* __restrict__ conf,
                                                               float* __restrict__ mx) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  __shared__ float sm[32], ss[32];
  __shared__ int si[32];
  const float* lg = logits + (size_t)blockIdx.x * ld;
  float m = -INFINITY, s = 0.f;
  int idx = 0x7fffffff;
  msi_scan(lg, 0, V, (ld % 4) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0, m, s, idx);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    merge_msi(m, s, idx, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o),
              __shfl_xor_sync(0xffffffffu, idx, o));
  if (lane == 0) {
    sm[wid] = m;
    ss[wid] = s;
    si[wid] = idx;
  }
  __syncthreads();
  if (wid == 0) {
    const bool live = lane < (int)(blockDim.x >> 5);
    m = live ? sm[lane] : -INFINITY;
    s = live ? ss[lane] : 0.f;
    idx = live ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      merge_msi(m, s, idx, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o),
                __shfl_xor_sync(0xffffffffu, idx, o));
    if (lane == 0) {
      tok[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
      conf[blockIdx.x] = s > 0.f ? 1.f / s : 0.f;
      if (mx) mx[blockIdx.x] = m;
    }
  }
}

// Few rows (fewer CTAs than SMs): each row is split into `nsplit` chunks of
// `chunk` logits; a CTA per (row, chunk) writes its (max, sum, index) triple,
// and one warp per row merges the row's triples in chunk order.
__global__ void __launch_bounds__(kThreads) argmax_conf_part_kernel(const float* __restrict__ logits, int64_t ld,
                                                                    int V, int chunk, float* __restrict__ pm,
                                                                    float* __restrict__ ps, int* __restrict__ pi) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  __shared__ float sm[32], ss[32];
  __shared__ int si[32];
  const float* lg = logits + (size_t)blockIdx.x * ld;
  const int c0 = blockIdx.y * chunk, c1 = min(V, c0 + chunk);
  float m = -INFINITY, s = 0.f;
  int idx = 0x7fffffff;
  msi_scan(lg, c0, c1, (ld % 4) == 0 && (chunk % 4) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0, m, s,
           idx);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    merge_msi(m, s, idx, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o),
              __shfl_xor_sync(0xffffffffu, idx, o));
  if (lane == 0) {
    sm[wid] = m;
    ss[wid] = s;
    si[wid] = idx;
  }
  __syncthreads();
  if (wid == 0) {
    const bool live = lane < (int)(blockDim.x >> 5);
    m = live ? sm[lane] : -INFINITY;
    s = live ? ss[lane] : 0.f;
    idx = live ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      merge_msi(m, s, idx, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o),
                __shfl_xor_sync(0xffffffffu, idx, o));
    if (lane == 0) {
      const size_t o = (size_t)blockIdx.x * gridDim.y + blockIdx.y;
      pm[o] = m;
      ps[o] = s;
      pi[o] = idx;
    }
  }
}

__global__ void argmax_conf_merge_kernel(const float* __restrict__ pm, const float* __restrict__ ps,
                                         const int* __restrict__ pi, int nsplit, int B, int* __restrict__ tok,
                                         float* __restrict__ conf, float* __restrict__ mx) {
  b200::pdl_launch_dependents();
  b200::pdl_wait();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= B) return;
  float m = -INFINITY, s = 0.f;
  int idx = 0x7fffffff;
  for (int j = lane; j < nsplit; j += 32) {
    const size_t o = (size_t)row * nsplit + j;
    merge_msi(m, s, idx, pm[o], ps[o], pi[o]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    merge_msi(m, s, idx, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o),
              __shfl_xor_sync(0xffffffffu, idx, o));
  if (lane == 0) {
    tok[row] = idx == 0x7fffffff ? 0 : idx;
    conf[row] = s > 0.f ? 1.f / s : 0.f;
    if (mx) mx[row] = m;
  }
}

// scratch: 3 * B * nsplit words (fp32 max | fp32 sum | int32 index); nsplit <= 1 -> one CTA per row.
// The chunk size is ceil(V / nsplit) rounded up to a multiple of 4, and nsplit is
// reduced to the number of chunks that start inside the row.
int b200_argmax_conf(const float* logits, int64_t ld, int B, int V, int* tok, float* conf, float* mx, void* scratch,
                     int nsplit, cudaStream_t st) {
  if (B <= 0) return 0;
  cudaError_t e;
  if (nsplit <= 1 || !scratch) {
    e = b200::launch_k(argmax_conf_kernel, dim3(B), dim3(kThreads), 0, st, 1, logits, ld, V, tok, conf, mx);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
  }
  // chunks of whole float4s; no chunk starts at or past V
  const int chunk = ((V + nsplit - 1) / nsplit + 3) & ~3;
  nsplit = (V + chunk - 1) / chunk;
  float* pm = reinterpret_cast<float*>(scratch);
  float* ps = pm + (size_t)B * nsplit;
  int* pi = reinterpret_cast<int*>(ps + (size_t)B * nsplit);
  e = b200::launch_k(argmax_conf_part_kernel, dim3(B, nsplit), dim3(kThreads), 0, st, 1, logits, ld, V, chunk, pm,
                     ps, pi);
  if (e != cudaSuccess) return (int)e;
  e = b200::launch_k(argmax_conf_merge_kernel, dim3((B * 32 + 255) / 256), dim3(256), 0, st, 1, pm, ps, pi, nsplit,
                     B, tok, conf, mx);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_argmax(const float* logits, int64_t ld, int B, int V, int* out, int* out2, int* flags, cudaStream_t st) {
  if (B <= 0) return 0;
  cudaError_t e = b200::launch_k(argmax_kernel, dim3(B), dim3(kThreads), 0, st, 1, logits, ld, V, out, out2, flags);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int b200_logprobs(const float* logits, int64_t ld, int B, int V, const int* tokens, int n_top, float* out_lp,
                  int* top_ids, float* top_lp, cudaStream_t st) {
  if (B <= 0) return 0;
b200::launch_k(  logprobs_kernel, dim3(B), dim3(kThreads), 0, st, 1, logits, ld, V, tokens, n_top, out_lp, top_ids, top_lp);
  return (int)cudaGetLastError();
}

// Host-side Philox for tests and CPU oracles (same stream as the kernel).
uint32_t b200_philox_u32(uint64_t key, uint64_t step, uint32_t idx) { return philox_u32(key, step, idx); }

}  // extern "C"

B200_STATUS_ACCESSORS(sampling)
