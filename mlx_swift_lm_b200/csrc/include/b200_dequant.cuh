// Affine-quantised weight tiles -> bf16 MMA operand tiles in shared memory.
//
// Raw record of one 64-input K block for 128 weight rows (one contiguous
// bulk copy from the tile-major device layout):
//   codes   [128][WQ * 8] bytes. 8-bit: one code per byte in input order.
//           4-bit: 32-bit words of 8 inputs; input 2j in bits 4j..4j+3 and
//           input 2j+1 in bits 16+4j..19+4j (repacked from MLX at load).
//   scales  [gpb][128] bf16, then biases [gpb][128] bf16 (gpb = groups in the
//           block: 2 for group size 32, else 1).
// w = scale * q + bias with one rounding to bf16.
// WQ = kWqE2M1 (-4): 4-bit e2m1 codes (sign, 2 exponent bits, 1 mantissa bit)
// in the same repacked word order, scales [gpb][128] bf16, no biases;
// w = e2m1(q) * scale. MXFP4 (group 32, gpb 2): scales are powers of two
// 2^(e8m0 - 127) (exact). NVFP4 (group 16, gpb 4): scales are the e4m3 block
// scale times the tensor's global scale, rounded to bf16; `g` is then the
// first of the half's two groups (words 0-1 and 2-3).
// Output: row t of a K-major bf16 tile [128][64] with the 128-byte swizzle
// the UMMA descriptor expects (16-byte chunk c of row t at c ^ (t & 7)).
#pragma once

#include <cuda_fp16.h>

#include "b200_common.cuh"

namespace b200 {

constexpr int kWqE2M1 = -4;
template <int WQ>
__host__ __device__ constexpr int code_bits() {
  return WQ < 0 ? -WQ : WQ;
}

// bf16 pair of two e2m1 codes at bits 0..3 and 16..19 of v, times s2. The
// magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6} have bf16 patterns 0x0000 0x3F00
// 0x3F80 0x3FC0 0x4000 0x4040 0x4080 0x40C0: two byte permutes look the low
// and high bytes up in 8-entry tables held in registers; the sign bit moves
// to bit 15 of each half.
__device__ __forceinline__ uint32_t de2m1_pair(uint32_t v, __nv_bfloat162 s2) {
  const uint32_t mag = v & 0x00070007u;
  const uint32_t sel = mag | (mag >> 8);  // selector nibbles: 0 = m0, 2 = m1
  const uint32_t lo = __byte_perm(0xC0800000u, 0xC0804000u, sel);
  const uint32_t hi = __byte_perm(0x3F3F3F00u, 0x40404040u, sel << 4);
  const uint32_t x = (lo & 0x00FF00FFu) | (hi & 0xFF00FF00u) | ((v & 0x00080008u) << 12);
  const __nv_bfloat162 w = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&x), s2);
  return *reinterpret_cast<const uint32_t*>(&w);
}

// Hardware conversion of the two e2m1 codes of one byte to an f16 pair
// (cvt.rn.f16x2.e2m1x2, sm_100a): which code lands in which half is pinned by
// tests/test_moe_gpu.py through b200_e2m1_pairs.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{\n .reg .b8 b;\n cvt.u8.u32 b, %1;\n cvt.rn.f16x2.e2m1x2 %0, b;\n}" : "=r"(r) : "r"(byte));
  return r;
}

// MXFP4 records in natural order (input 2j in the low nibble of byte j, 2j+1
// in the high nibble), dequantised to f16 for f16 x f16 MMAs: one hardware
// conversion per pair of inputs and one f16 multiply by the block scale
// (a power of two, exact while the product stays in f16 range). Thread
// (t, half) converts inputs [32*half, 32*half + 32) of row t into the
// 128B-swizzled f16 tile.
__device__ __forceinline__ void dequant_half_row_e2m1_f16(const uint8_t* raw, uint8_t* atile, int t, int half,
                                                          int g, int gpb) {
  constexpr int kCodeBytes = 4 * 128 * 64 / 8;
  const __nv_bfloat16* sc = reinterpret_cast<const __nv_bfloat16*>(raw + kCodeBytes);
  const __half s0 = __float2half(bf2f(sc[g * 128 + t]));
  const __half s1 = gpb == 4 ? __float2half(bf2f(sc[(g + 1) * 128 + t])) : s0;
  const uint4 c = *reinterpret_cast<const uint4*>(raw + t * 32 + half * 16);
  const uint32_t words[4] = {c.x, c.y, c.z, c.w};
  uint8_t* arow = atile + t * 128;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t v = words[w];
    const __half sw = w < 2 ? s0 : s1;
    const __half2 s2 = __halves2half2(sw, sw);
    uint32_t o[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t p = e2m1x2_to_f16x2((v >> (8 * b)) & 0xFFu);
      const __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&p), s2);
      o[b] = *reinterpret_cast<const uint32_t*>(&h);
    }
    const int chunk = half * 4 + w;
    *reinterpret_cast<uint4*>(arow + ((chunk ^ (t & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// bf16 pair (q_lo + 128, q_hi + 128) from two 4-bit codes placed at bits 0..3
// and 16..19 of v (exact: 128..143 are bf16 integers), minus 128, then
// scale * q + bias with one rounding.
__device__ __forceinline__ uint32_t dq4_pair(uint32_t v, __nv_bfloat162 s2, __nv_bfloat162 b2) {
  const uint32_t x = (v & 0x000F000Fu) | 0x43004300u;
  const __nv_bfloat162 c128 = __floats2bfloat162_rn(128.f, 128.f);
  const __nv_bfloat162 q = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&x), c128);
  const __nv_bfloat162 w = __hfma2(q, s2, b2);
  return *reinterpret_cast<const uint32_t*>(&w);
}

// Thread (t, half) converts inputs [32*half, 32*half + 32) of row t. `g` is
// the group of that half (0, or `half` when the group size is 32).
template <int WQ>
__device__ __forceinline__ void dequant_half_row(const uint8_t* raw, uint8_t* atile, int t, int half, int g,
                                                 int gpb) {
  constexpr int kCodeBytes = code_bits<WQ>() * 128 * 64 / 8;
  const __nv_bfloat16* sc = reinterpret_cast<const __nv_bfloat16*>(raw + kCodeBytes);
  const __nv_bfloat16* bi = reinterpret_cast<const __nv_bfloat16*>(raw + kCodeBytes + gpb * 256);
  const __nv_bfloat16 sv = sc[g * 128 + t];
  uint8_t* arow = atile + t * 128;
  if constexpr (WQ == kWqE2M1) {
    const uint4 c = *reinterpret_cast<const uint4*>(raw + t * 32 + half * 16);
    const uint32_t words[4] = {c.x, c.y, c.z, c.w};
    const __nv_bfloat16 sv2 = gpb == 4 ? sc[(g + 1) * 128 + t] : sv;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t v = words[w];
      const __nv_bfloat16 sw = w < 2 ? sv : sv2;
      const __nv_bfloat162 s2 = __halves2bfloat162(sw, sw);
      uint4 o;
      o.x = de2m1_pair(v, s2);
      o.y = de2m1_pair(v >> 4, s2);
      o.z = de2m1_pair(v >> 8, s2);
      o.w = de2m1_pair(v >> 12, s2);
      const int chunk = half * 4 + w;
      *reinterpret_cast<uint4*>(arow + ((chunk ^ (t & 7)) << 4)) = o;
    }
  } else if constexpr (WQ == 4) {
    const __nv_bfloat16 bv = bi[g * 128 + t];
    const uint4 c = *reinterpret_cast<const uint4*>(raw + t * 32 + half * 16);
    const uint32_t words[4] = {c.x, c.y, c.z, c.w};
    const __nv_bfloat162 s2 = __halves2bfloat162(sv, sv), b2 = __halves2bfloat162(bv, bv);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t v = words[w];
      uint4 o;
      o.x = dq4_pair(v, s2, b2);
      o.y = dq4_pair(v >> 4, s2, b2);
      o.z = dq4_pair(v >> 8, s2, b2);
      o.w = dq4_pair(v >> 12, s2, b2);
      const int chunk = half * 4 + w;
      *reinterpret_cast<uint4*>(arow + ((chunk ^ (t & 7)) << 4)) = o;
    }
  } else {
    const __nv_bfloat16 bv = bi[g * 128 + t];
    static_assert(WQ == 8, "4- or 8-bit codes");
    const uint4* cw = reinterpret_cast<const uint4*>(raw + t * 64 + half * 32);
    const uint4 q0 = cw[0], q1 = cw[1];
    const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const float sf = bf2f(sv), bf = bf2f(bv);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t v = words[2 * h + e];
        o[2 * e] = pack_bf16x2(fmaf((float)(v & 0xFF), sf, bf), fmaf((float)((v >> 8) & 0xFF), sf, bf));
        o[2 * e + 1] = pack_bf16x2(fmaf((float)((v >> 16) & 0xFF), sf, bf), fmaf((float)(v >> 24), sf, bf));
      }
      const int chunk = half * 4 + h;
      *reinterpret_cast<uint4*>(arow + ((chunk ^ (t & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Same conversion into 16 registers of packed bf16 pairs (inputs 32*half +
// 2c and 2c+1 in register c): 16 consecutive 32-bit tensor-memory columns of
// lane t, the layout of an MMA A operand read from tensor memory.
template <int WQ>
__device__ __forceinline__ void dequant_half_row_regs(const uint8_t* raw, int t, int half, int g, int gpb,
                                                      uint32_t* v) {
  constexpr int kCodeBytes = code_bits<WQ>() * 128 * 64 / 8;
  const __nv_bfloat16* sc = reinterpret_cast<const __nv_bfloat16*>(raw + kCodeBytes);
  const __nv_bfloat16* bi = reinterpret_cast<const __nv_bfloat16*>(raw + kCodeBytes + gpb * 256);
  const __nv_bfloat16 sv = sc[g * 128 + t];
  if constexpr (WQ == kWqE2M1) {
    const uint4 c = *reinterpret_cast<const uint4*>(raw + t * 32 + half * 16);
    const uint32_t words[4] = {c.x, c.y, c.z, c.w};
    const __nv_bfloat16 sv2 = gpb == 4 ? sc[(g + 1) * 128 + t] : sv;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t x = words[w];
      const __nv_bfloat16 sw = w < 2 ? sv : sv2;
      const __nv_bfloat162 s2 = __halves2bfloat162(sw, sw);
      v[4 * w + 0] = de2m1_pair(x, s2);
      v[4 * w + 1] = de2m1_pair(x >> 4, s2);
      v[4 * w + 2] = de2m1_pair(x >> 8, s2);
      v[4 * w + 3] = de2m1_pair(x >> 12, s2);
    }
  } else if constexpr (WQ == 4) {
    const __nv_bfloat16 bv = bi[g * 128 + t];
    const uint4 c = *reinterpret_cast<const uint4*>(raw + t * 32 + half * 16);
    const uint32_t words[4] = {c.x, c.y, c.z, c.w};
    const __nv_bfloat162 s2 = __halves2bfloat162(sv, sv), b2 = __halves2bfloat162(bv, bv);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t x = words[w];
      v[4 * w + 0] = dq4_pair(x, s2, b2);
      v[4 * w + 1] = dq4_pair(x >> 4, s2, b2);
      v[4 * w + 2] = dq4_pair(x >> 8, s2, b2);
      v[4 * w + 3] = dq4_pair(x >> 12, s2, b2);
    }
  } else {
    static_assert(WQ == 8, "4- or 8-bit codes");
    const __nv_bfloat16 bv = bi[g * 128 + t];
    const uint4* cw = reinterpret_cast<const uint4*>(raw + t * 64 + half * 32);
    const uint4 q0 = cw[0], q1 = cw[1];
    const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const float sf = bf2f(sv), bf = bf2f(bv);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t x = words[w];
      v[2 * w] = pack_bf16x2(fmaf((float)(x & 0xFF), sf, bf), fmaf((float)((x >> 8) & 0xFF), sf, bf));
      v[2 * w + 1] = pack_bf16x2(fmaf((float)((x >> 16) & 0xFF), sf, bf), fmaf((float)(x >> 24), sf, bf));
    }
  }
}

}  // namespace b200
