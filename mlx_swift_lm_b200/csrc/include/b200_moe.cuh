// Router top-k of one token by one warp, shared by the MoE kernels and the
// expert-parallel dispatch.
//
// mode 0: softmax over all experts, take top-k, renormalise if norm_topk.
// mode 1: top-k over the logits, softmax over the k (GPT-OSS).
// Ties resolve to the lower expert id (MLXLMCommon/MoERouterTopK.swift:22).
// Lane 0 writes ids[0..k) and w[0..k). E <= 256, k <= 16.
#pragma once
#include "b200_common.cuh"

namespace b200 {

__device__ __forceinline__ void route_topk_warp(const float* __restrict__ lg, int E, int k, int mode, int norm_topk,
                                                int* ids, float* w) {
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
  }
  float sel_v[16];
  int sel_i[16];
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = 0; i < per; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    sel_v[j] = bv;
    sel_i[j] = bi;
    for (int i = 0; i < per; ++i)
      if (lane + 32 * i == bi) v[i] = -INFINITY;
  }
  if (lane == 0) {
    if (mode == 0) {
      float s = 0.f;
      for (int j = 0; j < k; ++j) {
        sel_v[j] /= denom;
        s += sel_v[j];
      }
      for (int j = 0; j < k; ++j) {
        ids[j] = sel_i[j];
        w[j] = norm_topk ? sel_v[j] / s : sel_v[j];
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
