// Router top-k of one token by one warp, shared by the MoE kernels and the
// expert-parallel dispatch.
//
// mode 0: softmax over all experts, take top-k, renormalise if norm_topk,
//         times `scale`; with n_group > 1 only the `topk_group` groups with
//         the highest best probability compete, the others' probabilities set
//         to 0 (DeepSeek V2 group_limited_greedy, MLXLLM/Models/DeepseekV2.swift:252-274).
// mode 1: top-k over the logits, softmax over the k (GPT-OSS).
// mode 2: sigmoid scores; selection by score + correction bias within the
//         `topk_group` groups (of n_group) whose two best biased scores sum
//         highest (the others' selection scores set to 0); weights are the
//         unbiased sigmoid scores of the chosen experts, renormalised when
//         norm_topk and k > 1, times `scale` (GLM-4.5 / DeepSeek-V3 routers,
//         MLXLLM/Models/GLM4MOE.swift:147-180).
// Ties resolve to the lower expert id (MLXLMCommon/MoERouterTopK.swift:22),
// tied groups to the lower group id.
// Lane 0 writes ids[0..k) and w[0..k). E <= 256, k <= 16, n_group <= 32.
#pragma once
#include "b200_common.cuh"

namespace b200 {

struct RouteExtra {
  const float* bias = nullptr;  // [E] selection-score correction (mode 2)
  int n_group = 1;
  int topk_group = 1;
  float scale = 1.f;
};

__device__ __forceinline__ void route_topk_warp(const float* __restrict__ lg, int E, int k, int mode, int norm_topk,
                                                int* ids, float* w, const RouteExtra& ex = RouteExtra()) {
  const int lane = threadIdx.x & 31;
  constexpr int kMaxPer = 8;
  float v[kMaxPer];
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
  for (int i = 0; i < per; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? lg[e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float denom = 1.f;
  float so[kMaxPer];  // mode 2: the unbiased sigmoid scores
  if (mode == 2) {
    for (int i = 0; i < per; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        so[i] = 1.f / (1.f + __expf(-v[i]));
        v[i] = so[i] + (ex.bias ? ex.bias[e] : 0.f);
      } else {
        so[i] = 0.f;
      }
    }
  }
  // group-limited selection: sigmoid_group ranks groups by the sum of their two
  // best biased scores, softmax_topk (DeepSeek V2 group_limited_greedy) by the
  // group's best logit, which orders groups as their best probability does
  unsigned keep = 0xffffffffu;  // bit g: group g survives
  if ((mode == 2 || mode == 0) && ex.n_group > 1) {
    {
      const int gsz = E / ex.n_group;
      keep = 0;
      float gscore[32];
      for (int g = 0; g < ex.n_group; ++g) {
        // best and second best biased score of the group (the best's lowest id excluded once)
        float b1 = -INFINITY;
        int i1 = 0x7fffffff;
        for (int i = 0; i < per; ++i) {
          const int e = lane + 32 * i;
          if (e < E && e / gsz == g && (v[i] > b1 || (v[i] == b1 && e < i1))) {
            b1 = v[i];
            i1 = e;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, b1, o);
          const int oi = __shfl_xor_sync(0xffffffffu, i1, o);
          if (ov > b1 || (ov == b1 && oi < i1)) {
            b1 = ov;
            i1 = oi;
          }
        }
        float b2 = -INFINITY;
        for (int i = 0; i < per; ++i) {
          const int e = lane + 32 * i;
          if (e < E && e / gsz == g && e != i1) b2 = fmaxf(b2, v[i]);
        }
        b2 = warp_max(b2);
        gscore[g] = mode == 0 ? b1 : b1 + (gsz > 1 ? b2 : 0.f);
      }
      for (int j = 0; j < ex.topk_group && j < ex.n_group; ++j) {
        int bg = -1;
        for (int g = 0; g < ex.n_group; ++g)
          if (!(keep >> g & 1u) && (bg < 0 || gscore[g] > gscore[bg])) bg = g;
        keep |= 1u << bg;
      }
      if (mode == 2)
        for (int i = 0; i < per; ++i) {
          const int e = lane + 32 * i;
          if (e < E && !(keep >> (e / gsz) & 1u)) v[i] = 0.f;
        }
    }
  }
  if (mode == 0) {
    float s = 0.f;
    for (int i = 0; i < per; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        v[i] = __expf(v[i] - mx);
        s += v[i];
      }
    }
    denom = warp_sum(s);
    if (ex.n_group > 1) {  // dropped groups' probabilities become 0 (still in the denominator)
      const int gsz = E / ex.n_group;
      for (int i = 0; i < per; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !(keep >> (e / gsz) & 1u)) v[i] = 0.f;
      }
    }
  }
  float sel_v[16], sel_s[16];
  int sel_i[16];
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY, bs = 0.f;
    int bi = 0x7fffffff;
    for (int i = 0; i < per; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
        bi = e;
        bs = mode == 2 ? so[i] : 0.f;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const float os = __shfl_xor_sync(0xffffffffu, bs, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
        bs = os;
      }
    }
    sel_v[j] = bv;
    sel_s[j] = bs;
    sel_i[j] = bi;
    for (int i = 0; i < per; ++i)
      if (lane + 32 * i == bi) v[i] = -INFINITY;
  }
  if (lane == 0) {
    if (mode == 2) {
      float s = 0.f;
      for (int j = 0; j < k; ++j) s += sel_s[j];
      const float inv = (norm_topk && k > 1 && s > 0.f) ? 1.f / s : 1.f;
      for (int j = 0; j < k; ++j) {
        ids[j] = sel_i[j];
        w[j] = sel_s[j] * inv * ex.scale;
      }
    } else if (mode == 0) {
      float s = 0.f;
      for (int j = 0; j < k; ++j) {
        sel_v[j] /= denom;
        s += sel_v[j];
      }
      for (int j = 0; j < k; ++j) {
        ids[j] = sel_i[j];
        w[j] = (norm_topk ? sel_v[j] / s : sel_v[j]) * ex.scale;
      }
    } else {
      const float m0 = sel_v[0];
      float s = 0.f;
      for (int j = 0; j < k; ++j) {
        sel_v[j] = __expf(sel_v[j] - m0);
        s += sel_v[j];
      }
      for (int j = 0; j < k; ++j) {
        ids[j] = sel_i[j];
        w[j] = sel_v[j] / s;
      }
    }
  }
}

}  // namespace b200
